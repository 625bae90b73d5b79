"""Expert parallelism for batched decode: experts sharded over the ranks of a
process group, tokens dispatched to the expert owners and the results combined
back (all-to-all over NCCL / NVLink).

Rank g of a group of G holds the experts [g * E/G, (g + 1) * E/G) of every MoE
layer and its own tokens (data-parallel attention).  One layer call:

  1. route the local tokens (fused router: top-k + routing plan).  The plan's
     slot order is experts ascending, so the rows bound for each owner rank
     are contiguous in it;
  2. gather the routed token rows in slot order; exchange per-rank row counts
     (an all-to-all of G ints, read on the host to size the exchange);
  3. dispatch: all-to-all of the rows and of their expert ids local to the
     owner;
  4. the owner runs its experts on the received rows (one expert per row,
     weight 1: the decode kernels, or the tcgen05 grouped GEMMs from 256 rows);
  5. combine: all-to-all of the expert outputs back to the token owners, then
     the routing-weighted sum in top-k order (tm_combine_slots).

Per token the arithmetic is that of MoEExecutor.execute_layer
(execution/moe.py:99-208): the same experts, weights and SwiGLU; only the
summation order of the k expert outputs differs (top-k order, fp32).  The
reference engine itself runs batch 1 on one device and has no expert
parallelism.

The exchange logic is independent of where the compute runs: `route_fn`,
`expert_fn` and `combine_fn` are supplied by the caller.  `cuda_functions`
builds the product ones from this library's kernels.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass
class Routing:
    """Top-k routing of the local tokens and its plan (slots = routed pairs in
    expert-ascending, then token-ascending order)."""
    idx: torch.Tensor          # [T, k] int64 expert ids
    w: torch.Tensor            # [T, k] routing weights (act dtype)
    slot_token: torch.Tensor   # [P] int64 token of each slot
    slot_expert: torch.Tensor  # [P] int64 expert of each slot
    pair_slot: torch.Tensor    # [T * k] slot of (token t, rank r) at t * k + r
    counts: torch.Tensor       # [E] int64 slots per expert


class ExpertParallelMoE:
    """One expert-parallel MoE layer call per `forward` (all ranks of `group`
    must call it, in the same order, with their own tokens)."""

    def __init__(self, n_experts: int, top_k: int, route_fn: Callable[[torch.Tensor], Routing],
                 expert_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
                 combine_fn: Callable[[torch.Tensor, Routing, torch.Tensor | None], torch.Tensor],
                 group=None):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.G:
            raise ValueError(f"{n_experts} experts do not shard over {self.G} ranks")
        self.E, self.k = n_experts, top_k
        self.E_loc = n_experts // self.G
        self.route_fn, self.expert_fn, self.combine_fn = route_fn, expert_fn, combine_fn
        self.last_counts = None  # (send, recv) rows per rank of the last call, for reporting

    def local_experts(self) -> range:
        return range(self.rank * self.E_loc, (self.rank + 1) * self.E_loc)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x.shape
        r = self.route_fn(x)
        # 2. rows in slot order (grouped by owner rank) and the row counts
        send_rows = x.index_select(0, r.slot_token)
        send_eid = (r.slot_expert % self.E_loc).to(torch.int32)
        send_counts = r.counts.view(self.G, self.E_loc).sum(1).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        self.last_counts = (sc, rc)
        # 3. dispatch
        R = sum(rc)
        recv_rows = x.new_empty(R, H)
        recv_eid = send_eid.new_empty(R)
        dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=self.group)
        dist.all_to_all_single(recv_eid, send_eid, rc, sc, group=self.group)
        # 4. local experts
        y_recv = self.expert_fn(recv_rows, recv_eid) if R else x.new_empty(0, H)
        # 5. combine
        y_slots = x.new_empty(send_rows.shape[0], H)
        dist.all_to_all_single(y_slots, y_recv.contiguous(), sc, rc, group=self.group)
        return self.combine_fn(y_slots, r, residual)


def cuda_functions(router_w: torch.Tensor, local_experts, top_k: int, n_experts: int, hidden: int, inter: int):
    """(route_fn, expert_fn, combine_fn) on this library's kernels for one
    layer: `router_w` [E, H] (act dtype), `local_experts` the PackedExperts of
    this rank's shard."""
    from . import ops
    dev = router_w.device
    ws_route = ops.Workspace(dev, n_experts, top_k, hidden, inter, 0)
    ws_expert = ops.Workspace(dev, local_experts.n_experts, 1, hidden, inter, 0)

    def route_fn(x):
        T = x.shape[0]
        idx, w = ops.router_topk(x, router_w, top_k, ws_route)
        pv = ops.plan_views(ws_route, T, top_k)
        slot_pair = pv["slot_pair"].long()
        return Routing(idx=idx, w=w, slot_token=pv["slot_token"].long(), slot_expert=idx.view(-1)[slot_pair],
                       pair_slot=pv["pair_slot"].clone(), counts=pv["counts"].long())

    def expert_fn(rows, eid):
        R = rows.shape[0]
        ones = torch.ones(R, 1, dtype=rows.dtype, device=rows.device)
        return ops.moe_experts(rows, eid.long().view(R, 1), ones, local_experts, ws_expert)

    def combine_fn(y_slots, r, residual):
        out = torch.empty(r.w.shape[0], y_slots.shape[1], dtype=y_slots.dtype, device=y_slots.device)
        return ops.combine_slots(y_slots, r.w, r.pair_slot, out, residual)

    return route_fn, expert_fn, combine_fn


class PeerExpertParallelMoE:
    """Expert-parallel MoE layer over NVLink peer memory (the tm_ep_* entry
    points of libturbomoe): dispatch, the owner's grouped GEMMs and the return
    of the outputs are device kernels with bounded waits, so a call has no
    collective, no host synchronisation and can be captured in a CUDA graph.

    Every rank of `group` (one process per GPU of one node) constructs it with
    its own shard `local_experts` (PackedExperts of experts
    [rank * E/G, (rank + 1) * E/G)) - construction is collective (it exchanges
    the buffers' IPC handles) - and calls `forward` in the same order.  Without
    an initialised process group, or with ``single=True``, it runs as a single
    rank owning every expert.

    ``channel``: another PeerExpertParallelMoE of the same shape whose context
    (peer buffers, workspaces) this layer reuses.  The layers of a model run
    one after the other on one stream, and a source dispatches call n + 1 only
    after every owner has returned call n, so one context can carry every
    layer: construction is then local (no handle exchange) and only the
    instance that created the context may ``close`` it."""

    def __init__(self, router_w: torch.Tensor, local_experts, top_k: int, max_tokens: int, group=None,
                 timeout_s: float = 2.0, channel: "PeerExpertParallelMoE | None" = None, single: bool = False):
        import ctypes as C
        from . import ops
        from ._lib import TM_EP_HANDLE_BYTES, check, lib
        self._C, self._ops, self._check, self._L = C, ops, check, lib()
        E, H = router_w.shape
        self.router_w = router_w.contiguous()
        self.local = local_experts
        if channel is not None:
            if (channel.E, channel.k, channel.H, channel.I) != (E, top_k, H, local_experts.inter) or \
                    channel.router_w.dtype != router_w.dtype or max_tokens > channel.max_tokens or \
                    local_experts.n_experts != channel.local.n_experts:
                raise ValueError("channel has another expert-parallel shape")
            self.group, self.G, self.rank = channel.group, channel.G, channel.rank
            self.E, self.k, self.H, self.I = E, top_k, H, local_experts.inter
            self.max_tokens = channel.max_tokens
            self.ctx, self.ws, self.owner_ws = channel.ctx, channel.ws, channel.owner_ws
            self._owner = False
            return
        self._owner = True
        single = single or not (dist.is_available() and dist.is_initialized())
        self.group = group
        self.G = 1 if single else dist.get_world_size(group)
        self.rank = 0 if single else dist.get_rank(group)
        self.E, self.k, self.H, self.I = E, top_k, H, local_experts.inter
        if E % self.G or local_experts.n_experts != E // self.G:
            raise ValueError(f"{local_experts.n_experts} local experts do not match {E} over {self.G} ranks")
        self.max_tokens = max_tokens
        dev = router_w.device
        code = ops._code(router_w.dtype)
        self.ctx = C.c_void_p()
        handle = (C.c_char * TM_EP_HANDLE_BYTES)()
        check(self._L.tm_ep_create(self.rank, self.G, E, top_k, H, self.I, code, max_tokens, handle,
                                   C.byref(self.ctx)), "tm_ep_create")
        mine = (bytes(handle), (E, top_k, H, self.I, code, max_tokens))
        if single:
            everyone = [mine]
        else:
            everyone = [None] * self.G
            dist.all_gather_object(everyone, mine, group=group)
        if any(s != mine[1] for _, s in everyone):
            raise ValueError(f"ranks disagree on the expert-parallel shape: {[s for _, s in everyone]}")
        check(self._L.tm_ep_connect(self.ctx, b"".join(h for h, _ in everyone)), "tm_ep_connect")
        check(self._L.tm_ep_set_timeout(self.ctx, int(timeout_s * 1e9)), "tm_ep_set_timeout")
        self.ws = ops.Workspace(dev, E, top_k, H, self.I, 0)
        self.ws.ensure(max_tokens)
        n = self._L.tm_ep_owner_workspace_bytes(self.ctx)
        self.owner_ws = torch.empty(n, dtype=torch.uint8, device=dev)
        check(self._L.tm_workspace_init(self.owner_ws.data_ptr(), n, ops._stream(self.owner_ws)), "tm_workspace_init")

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                out: torch.Tensor | None = None, marks=None) -> torch.Tensor:
        """One layer call.  ``marks``: optional list of 5 CUDA events recorded
        on the stream before the router, the dispatch, the experts, the combine
        and after it (per-phase timing)."""
        ops, check, L = self._ops, self._check, self._L
        x = x.contiguous()
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens {self.max_tokens}")
        mark = (lambda i: marks[i].record()) if marks is not None else (lambda i: None)
        mark(0)
        idx, w = ops.router_topk(x, self.router_w, self.k, self.ws)
        s = ops._stream(x)
        buf = self.ws.buf
        mark(1)
        check(L.tm_ep_dispatch(self.ctx, x.data_ptr(), T, idx.data_ptr(), buf.data_ptr(), buf.numel(), s),
              "tm_ep_dispatch")
        le = self.local
        mark(2)
        check(L.tm_ep_experts(self.ctx, le.w13.data_ptr(), le.s13.data_ptr(), le.w2.data_ptr(), le.s2.data_ptr(),
                              self.owner_ws.data_ptr(), self.owner_ws.numel(), s), "tm_ep_experts")
        if out is None:
            out = torch.empty_like(x)
        res = residual.contiguous() if residual is not None else None
        mark(3)
        check(L.tm_ep_combine(self.ctx, w.data_ptr(), T, buf.data_ptr(), buf.numel(),
                              res.data_ptr() if res is not None else None, out.data_ptr(), s), "tm_ep_combine")
        mark(4)
        return out

    def status(self) -> int:
        """TM_STATUS_* bits of the calls since the last status() (synchronises)."""
        C, ops = self._C, self._ops
        v = C.c_uint32(0)
        self._check(self._L.tm_ep_status(self.ctx, C.byref(v), ops._stream(self.owner_ws)), "tm_ep_status")
        o = C.c_uint32(0)
        self._check(self._L.tm_workspace_status(self.owner_ws.data_ptr(), self.owner_ws.numel(), C.byref(o),
                                                ops._stream(self.owner_ws)), "tm_workspace_status")
        return int(v.value) | int(o.value) | self.ws.status()

    def close(self):
        """Collective: every rank, after its last forward (a no-op on a layer
        that borrowed another one's context)."""
        if not self._owner:
            self.ctx = self._C.c_void_p()
            return
        if self.ctx:
            torch.cuda.synchronize()
            if self.G > 1:
                dist.barrier(group=self.group)
            self._check(self._L.tm_ep_disconnect(self.ctx), "tm_ep_disconnect")
            if self.G > 1:
                dist.barrier(group=self.group)  # nobody maps a buffer that is freed
            self._check(self._L.tm_ep_destroy(self.ctx), "tm_ep_destroy")
            self.ctx = self._C.c_void_p()
