"""RouterExecutor drop-in (reference: execution/router.py:1-42).

``compute_routing`` runs the fused router kernel K1 (``tm_router_topk``):
logits GEMV in the activation dtype with fp32 accumulation, fp32 softmax,
top-k (ties: lower expert id first), renormalisation, cast back to the
activation dtype -- and, in the same launch, the routing plan (per-expert
histogram, offsets and stable token permutation) that MoEExecutor consumes,
so the reference's ``torch.unique(...).tolist()`` host sync disappears.
"""
from __future__ import annotations

import torch

from turbomoe import ops


class NextLayerPrefetch:
    """Speculative L2 prefetch of the next layer's experts (opt-in).

    After the router of layer l is launched, a side stream applies layer
    l+1's router to the same hidden state (the residual stream moves little
    from one layer to the next), and bulk-prefetches the gate/up weights of
    the experts it picks into L2 (``tm_prefetch_experts_l2``).  That work
    runs while the current layer's expert kernels read from L2, and layer
    l+1's gate/up kernel then finds the experts predicted correctly in L2.
    The prediction is a hint only: routing and outputs are unchanged.
    ``MoEExecutor.execute_layer`` rejoins the side stream after its kernels
    (``layer_done``) every ``join_every`` layers and after the last one, so a
    graph captured over whole layers has no loose branch.
    """

    def __init__(self, loader, routers, top_k, join_every=1):
        self.loader = loader
        self.routers = routers
        self.top_k = top_k
        self.join_every = max(1, int(join_every))
        self.stream = None
        self.ws = None
        self.pending = None

    def fork(self, layer_id, flat):
        nxt = layer_id + 1
        if nxt not in self.routers or flat.shape[0] > 8:
            return
        dev = flat.device
        if self.stream is None:
            self.stream = torch.cuda.Stream(device=dev)
            self.ws = ops.Workspace(dev, self.routers[nxt].shape[0], self.top_k, flat.shape[1], 128, 0)
        self.ws.ensure(flat.shape[0])
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            idx, _ = ops.router_topk(flat, self.routers[nxt], self.top_k, self.ws)
            ops.prefetch_experts_l2(self.loader.packed_layer(nxt).experts, idx)
            done = torch.cuda.Event()
            done.record(self.stream)
        if not torch.cuda.is_current_stream_capturing():
            flat.record_stream(self.stream)
            idx.record_stream(self.stream)
        self.pending = done

    def join(self):
        if self.pending is not None:
            torch.cuda.current_stream().wait_event(self.pending)
            self.pending = None

    def layer_done(self, layer_id):
        """After a layer's expert kernels: rejoin the side stream every
        ``join_every`` layers and after the last layer with a router."""
        if (layer_id + 1) % self.join_every == 0 or layer_id + 1 >= len(self.routers):
            self.join()


class RouterExecutor:

    def __init__(self, loader, num_layers, top_k=8, prefetch_next_layer=False, prefetch_join_every=1):
        self.loader = loader
        self.num_layers = num_layers
        self.top_k = top_k
        self.routers = {}
        for i in range(self.num_layers):
            self.routers[i] = self.loader.load_weight(self.loader.layout.router_tensor(i)).contiguous()
        # decode calls (<= 8 tokens): speculative L2 prefetch of layer l+1's experts
        self.next_layer_prefetch = (NextLayerPrefetch(loader, self.routers, top_k, prefetch_join_every)
                                    if prefetch_next_layer else None)
        if self.next_layer_prefetch is not None:
            loader.next_layer_prefetch = self.next_layer_prefetch

    def compute_routing(self, layer_id, hidden_states, top_k=None):
        """hidden_states: [batch, seq, H] or [seq, H] -> (idx int64 [T,k], w [T,k])."""
        router_weight = self.routers[layer_id]
        flat = hidden_states.reshape(-1, hidden_states.shape[-1])
        k = top_k if top_k is not None else self.top_k
        ws = self.loader.workspace(flat.device, k)
        out = ops.router_topk(flat, router_weight, k, ws)
        if self.next_layer_prefetch is not None and k == self.top_k:
            self.next_layer_prefetch.fork(layer_id, flat)
        return out

    def compute_routing_with_logits(self, layer_id, hidden_states, top_k=None):
        """Same as ``compute_routing`` plus the act-dtype logits ``[T, E]``."""
        flat = hidden_states.reshape(-1, hidden_states.shape[-1])
        k = top_k if top_k is not None else self.top_k
        return ops.router_topk(flat, self.routers[layer_id], k, self.loader.workspace(flat.device, k),
                               want_logits=True)
