"""RouterExecutor drop-in (reference: execution/router.py:1-42).

``compute_routing`` runs the fused router kernel K1 (``tm_router_topk``):
logits GEMV in the activation dtype with fp32 accumulation, fp32 softmax,
top-k (ties: lower expert id first), renormalisation, cast back to the
activation dtype -- and, in the same launch, the routing plan (per-expert
histogram, offsets and stable token permutation) that MoEExecutor consumes,
so the reference's ``torch.unique(...).tolist()`` host sync disappears.
"""
from __future__ import annotations

from turbomoe import ops


class RouterExecutor:

    def __init__(self, loader, num_layers, top_k=8):
        self.loader = loader
        self.num_layers = num_layers
        self.top_k = top_k
        self.routers = {}
        for i in range(self.num_layers):
            self.routers[i] = self.loader.load_weight(self.loader.layout.router_tensor(i)).contiguous()

    def compute_routing(self, layer_id, hidden_states, top_k=None):
        """hidden_states: [batch, seq, H] or [seq, H] -> (idx int64 [T,k], w [T,k])."""
        router_weight = self.routers[layer_id]
        flat = hidden_states.reshape(-1, hidden_states.shape[-1])
        k = top_k if top_k is not None else self.top_k
        ws = self.loader.workspace(flat.device, k)
        return ops.router_topk(flat, router_weight, k, ws)

    def compute_routing_with_logits(self, layer_id, hidden_states, top_k=None):
        """Same as ``compute_routing`` plus the act-dtype logits ``[T, E]``."""
        flat = hidden_states.reshape(-1, hidden_states.shape[-1])
        k = top_k if top_k is not None else self.top_k
        return ops.router_topk(flat, self.routers[layer_id], k, self.loader.workspace(flat.device, k),
                               want_logits=True)
