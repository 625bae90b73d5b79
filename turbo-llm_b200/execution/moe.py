"""MoEExecutor drop-in (reference: execution/moe.py:1-208).

``execute_layer(layer_id, hidden_states [T,H], top_k_indices [T,k],
top_k_weights [T,k])`` returns a new ``[T,H]`` tensor (same dtype/device);
inputs are not modified.  It streams the layer's packed FP8 experts through
two kernels:

* K2 ``tm_moe_decode_gateup``: gate+up dequant-GEMV with SwiGLU for every
  (expert, token) pair of the routing plan (and the shared expert);
* K3 ``tm_moe_decode_down_combine``: down dequant-GEMV, routing-weighted
  combine in top-k order, sigmoid-gated shared expert.

The routing plan comes from the RouterExecutor call that produced
``top_k_indices`` (same workspace); indices from anywhere else get a plan
built on the device by ``tm_route_plan``.  No host synchronisation happens
on this path (the reference's ``.tolist()`` at moe.py:39/132 is gone).

``last_gemm_ms`` is the device time of the last call's expert kernels,
measured with CUDA events and read lazily (reading it waits for the call).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from turbomoe import ops


def moe_seq(hidden_states, gate_weights, up_weights, down_weights, top_k_weights):
    """Interface-compatible ``moe_seq`` (reference moe.py:7-20) over already
    dequantised dense expert weights, as ``ExpertLoader.load_expert`` returns
    them.  A compatibility helper for callers that hold dense weights; the
    executor below never calls it (it streams the packed FP8 experts)."""
    final_output = torch.zeros_like(hidden_states)
    for i in range(top_k_weights.shape[1]):
        g = F.linear(hidden_states, gate_weights[i])
        u = F.linear(hidden_states, up_weights[i])
        final_output += F.linear(F.silu(g) * u, down_weights[i]) * top_k_weights[0, i]
    return final_output


class MoEExecutor:

    def __init__(self, loader, record_timing=True):
        self.loader = loader
        self.record_timing = record_timing
        self._events = None
        self._last_ms = 0.0

    @property
    def last_gemm_ms(self) -> float:
        if self._events is not None:
            start, end = self._events
            end.synchronize()
            self._last_ms = start.elapsed_time(end)
            self._events = None
        return self._last_ms

    def execute_decode(self, layer_id, hidden_states, top_k_indices, top_k_weights):
        return self.execute_layer(layer_id, hidden_states, top_k_indices, top_k_weights)

    def execute_layer(self, layer_id, hidden_states, top_k_indices, top_k_weights, residual=None,
                      out=None):
        pl = self.loader.packed_layer(layer_id)
        ws = self.loader.workspace(hidden_states.device, top_k_indices.shape[1])
        timing = self.record_timing and not torch.cuda.is_current_stream_capturing()
        if timing:
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
        y = ops.moe_experts(hidden_states, top_k_indices, top_k_weights, pl.experts, ws,
                            shared=pl.shared, shared_gate_w=pl.shared_gate, residual=residual, out=out)
        spec = getattr(self.loader, "next_layer_prefetch", None)
        if spec is not None:  # the speculative prefetch branch forked by RouterExecutor rejoins here
            spec.layer_done(layer_id)
        if timing:
            end.record()
            self._events = (start, end)
        return y
