"""Qwen3.5 linear attention decode step on tm_gdn_decode.

The reference's Qwen3.5 layers of type "linear_attention" call Hugging Face's
``Qwen3_5MoeGatedDeltaNet`` (execution/layer_executor.py:134-139) with the
reference's ``Qwen35Cache`` holding each layer's conv and recurrent state
(cache/qwen35_cache.py:43-64).  ``GatedDeltaNetDecode`` runs that module's
decode step (one token per sequence, a cached state present) with the conv
update, gates, gated delta rule and gated RMSNorm in one kernel; the
in_proj_* and out_proj GEMMs stay the module's own ``nn.Linear`` calls.

State handling follows the cache's interface: the recurrent state (fp32
[B, Hv, 128, 128]) is updated in place; the conv state is written to a second
buffer that replaces the cache's through ``update_conv_state`` (the kernel
cannot shift it in place), and the replaced buffer becomes the module's
output buffer for its next decode step, whichever cache that step uses, so a
step allocates nothing after the first.  Caches must therefore not share
conv-state tensors (clone the states to copy a cache).

``install(module)`` routes the module's decode calls here.  Calls without a
cached state or with more than one token (the prompt, which the module runs
in its chunked form) go to the module's own forward: this file implements the
decode step only.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import TurboMoEError


class GatedDeltaNetDecode:
    """Decode step of one ``Qwen3_5MoeGatedDeltaNet`` (CUDA tensors)."""

    def __init__(self, module):
        if module.head_k_dim != 128 or module.head_v_dim != 128:
            raise TurboMoEError("tm_gdn_decode implements head dims of 128")
        self.m = module
        self.layer_idx = module.layer_idx
        self.n_k_heads = module.num_k_heads
        self.conv_w = module.conv1d.weight.detach()[:, 0].contiguous()
        self.A_log = module.A_log.detach().float().contiguous()
        self.dt_bias = module.dt_bias.detach().float().contiguous()
        self.norm_w = module.norm.weight.detach().contiguous()
        self.eps = float(module.layer_norm_epsilon)
        self._spare = None

    def __call__(self, hidden_states: torch.Tensor, cache_params) -> torch.Tensor:
        B, T, _ = hidden_states.shape
        li = self.layer_idx
        if T != 1 or cache_params is None or not cache_params.has_previous_state(li):
            raise TurboMoEError("GatedDeltaNetDecode runs one token per sequence on a cached state")
        st = cache_params.layers[li]
        S = st.recurrent_states
        if S.dtype != torch.float32 or not S.is_contiguous():
            S = S.to(torch.float32).contiguous()
            cache_params.update_recurrent_state(S, li)
        conv = st.conv_states
        spare = self._spare
        if spare is None or spare.shape != conv.shape or spare.dtype != conv.dtype or \
                spare.device != conv.device or spare.data_ptr() == conv.data_ptr():
            spare = torch.empty_like(conv, memory_format=torch.contiguous_format)
        m = self.m
        # the module's own projection calls on [B, 1, H] (the same GEMMs, so the same roundings)
        qkv, z, a, b = (p(hidden_states)[:, 0] for p in (m.in_proj_qkv, m.in_proj_z, m.in_proj_a, m.in_proj_b))
        core = ops.gdn_decode(qkv, z, a, b, self.conv_w, self.A_log, self.dt_bias, self.norm_w, conv, spare, S,
                              self.n_k_heads, self.eps)
        cache_params.update_conv_state(spare, li)
        self._spare = conv if conv.is_contiguous() else None
        return m.out_proj(core[:, None])


def install(module) -> GatedDeltaNetDecode:
    """Route ``module``'s decode calls (one token, cached state) to
    ``GatedDeltaNetDecode``; other calls keep the module's own forward."""
    step = GatedDeltaNetDecode(module)
    own_forward = module.forward

    def forward(hidden_states, cache_params=None, attention_mask=None):
        if (hidden_states.shape[1] == 1 and cache_params is not None
                and cache_params.has_previous_state(step.layer_idx)):
            return step(hidden_states, cache_params)
        return own_forward(hidden_states, cache_params=cache_params, attention_mask=attention_mask)

    module.forward = forward
    return step
