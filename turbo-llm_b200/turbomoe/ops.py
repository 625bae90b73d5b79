"""Tensor-level wrappers over the C ABI (device memory owned by PyTorch).

Every function launches on ``torch.cuda.current_stream()`` and requires CUDA
tensors; there is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import (TM_DTYPE_BF16, TM_DTYPE_F16, TM_DTYPE_F32, TurboMoEError, check, lib)

DTYPE_CODE = {torch.float32: TM_DTYPE_F32, torch.float16: TM_DTYPE_F16, torch.bfloat16: TM_DTYPE_BF16}


def _code(dtype):
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise TurboMoEError(f"unsupported activation dtype {dtype}") from None


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise TurboMoEError("turbomoe kernels need CUDA tensors (there is no CPU fallback)")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _u8(t):
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


# ------------------------------------------------------------------ K0 ----
def dequant_fp8_block(w: torch.Tensor, scale: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """``ExpertLoader.dequantize_weight`` on the device (bit-exact, see K0)."""
    _need_cuda(w, scale)
    w = _u8(w).contiguous()
    scale = scale.float().contiguous()
    M, N = w.shape
    out = torch.empty(M, N, dtype=dtype, device=w.device)
    check(lib().tm_dequant_fp8_block(w.data_ptr(), scale.data_ptr(), M, N, out.data_ptr(), _code(dtype),
                                     _stream(w)), "tm_dequant_fp8_block")
    return out


# ------------------------------------------------------------------ K5 ----
@dataclass
class PackedExperts:
    """Device-resident packed experts of one layer (or the shared expert)."""
    w13: torch.Tensor   # uint8 [E * 2*I*H]
    s13: torch.Tensor   # fp32  [E * 2*(I/128)*(H/128)]
    w2: torch.Tensor    # uint8 [E * H*I]
    s2: torch.Tensor    # fp32  [E * (H/128)*(I/128)]
    n_experts: int
    hidden: int
    inter: int

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.w13, self.s13, self.w2, self.s2))

    def expert_views(self, e: int):
        L = lib()
        H, I = self.hidden, self.inter
        n13, ns13 = L.tm_packed_w13_bytes(H, I), L.tm_packed_s13_floats(H, I)
        n2, ns2 = L.tm_packed_w2_bytes(H, I), L.tm_packed_s2_floats(H, I)
        return (self.w13[e * n13:(e + 1) * n13], self.s13[e * ns13:(e + 1) * ns13],
                self.w2[e * n2:(e + 1) * n2], self.s2[e * ns2:(e + 1) * ns2])


def alloc_packed(n_experts: int, hidden: int, inter: int, device) -> PackedExperts:
    L = lib()
    e = n_experts
    return PackedExperts(
        torch.empty(e * L.tm_packed_w13_bytes(hidden, inter), dtype=torch.uint8, device=device),
        torch.empty(e * L.tm_packed_s13_floats(hidden, inter), dtype=torch.float32, device=device),
        torch.empty(e * L.tm_packed_w2_bytes(hidden, inter), dtype=torch.uint8, device=device),
        torch.empty(e * L.tm_packed_s2_floats(hidden, inter), dtype=torch.float32, device=device),
        n_experts, hidden, inter)


def pack_experts(gate, gate_s, up, up_s, down, down_s, out: PackedExperts | None = None,
                 first: int = 0) -> PackedExperts:
    """Pack stacked checkpoint tensors (``gate/up [n, I, H]``, ``down [n, H, I]``
    e4m3 plus their ``[n, ., .]`` fp32 scales, all on the device) into
    ``out`` starting at expert ``first`` (a new PackedExperts when ``out`` is None)."""
    if gate.dim() == 2:
        gate, gate_s, up, up_s, down, down_s = (t.unsqueeze(0) for t in (gate, gate_s, up, up_s, down, down_s))
    _need_cuda(gate, gate_s, up, up_s, down, down_s)
    n, I, H = gate.shape
    if out is None:
        out = alloc_packed(n, H, I, gate.device)
    if first + n > out.n_experts or out.hidden != H or out.inter != I:
        raise TurboMoEError("pack_experts: destination shape mismatch")
    L = lib()
    ts = [_u8(t).contiguous() for t in (gate, up, down)]
    ss = [s.float().contiguous() for s in (gate_s, up_s, down_s)]
    o13 = first * L.tm_packed_w13_bytes(H, I)
    os13 = first * L.tm_packed_s13_floats(H, I)
    o2 = first * L.tm_packed_w2_bytes(H, I)
    os2 = first * L.tm_packed_s2_floats(H, I)
    check(L.tm_pack_experts(ts[0].data_ptr(), ss[0].data_ptr(), ts[1].data_ptr(), ss[1].data_ptr(),
                            ts[2].data_ptr(), ss[2].data_ptr(), n, H, I,
                            out.w13[o13:].data_ptr(), out.s13[os13:].data_ptr(),
                            out.w2[o2:].data_ptr(), out.s2[os2:].data_ptr(), _stream(gate)),
          "tm_pack_experts")
    return out


def unpack_expert(p: PackedExperts, e: int, dtype, which=("gate", "up", "down")):
    """Dense dequantised (gate [I,H], up [I,H], down [H,I]) of expert ``e``."""
    H, I = p.hidden, p.inter
    w13, s13, w2, s2 = p.expert_views(e)
    dev = w13.device
    g = torch.empty(I, H, dtype=dtype, device=dev) if "gate" in which else None
    u = torch.empty(I, H, dtype=dtype, device=dev) if "up" in which else None
    d = torch.empty(H, I, dtype=dtype, device=dev) if "down" in which else None
    check(lib().tm_unpack_expert(w13.data_ptr(), s13.data_ptr(), w2.data_ptr(), s2.data_ptr(), H, I,
                                 _ptr(g), _ptr(u), _ptr(d), _code(dtype), _stream(w13)),
          "tm_unpack_expert")
    return g, u, d


# ----------------------------------------------------------- workspace ----
class Workspace:
    """One caller-owned workspace per device for a model shape; grows with T.

    The routing plan written by ``router_topk`` / ``route_plan`` lives here and
    is consumed by ``moe_gateup`` / ``moe_down_combine`` of the same layer call,
    so all of them must use the same Workspace on the same stream.
    """

    def __init__(self, device, n_experts, top_k, hidden, inter, shared_inter=0):
        self.device = torch.device(device)
        self.E, self.k, self.H, self.I, self.Is = n_experts, top_k, hidden, inter, shared_inter
        self.buf = None
        self.capacity_tokens = 0
        # the top-k tensor the current plan was built from (a strong reference, so
        # its memory cannot be recycled into a look-alike) and its version counter
        self.plan_idx = None
        self.plan_version = -1

    def nbytes_for(self, tokens, top_k=None):
        return lib().tm_workspace_bytes(tokens, self.E, top_k or self.k, self.H, self.I, self.Is)

    def ensure(self, tokens, top_k=None) -> torch.Tensor:
        need = self.nbytes_for(tokens, top_k)
        if need < 0:
            raise TurboMoEError("invalid workspace shape")
        if self.buf is None or self.buf.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise TurboMoEError("workspace must be sized (ensure) before CUDA graph capture")
            cap = max(need, 2 * (self.buf.numel() if self.buf is not None else 0))
            self.buf = torch.empty(cap, dtype=torch.uint8, device=self.device)
            check(lib().tm_workspace_init(self.buf.data_ptr(), cap, _stream(self.buf)), "tm_workspace_init")
            self.plan_idx = None
        return self.buf

    def status(self) -> int:
        import ctypes
        v = ctypes.c_uint32(0)
        check(lib().tm_workspace_status(self.buf.data_ptr(), self.buf.numel(), ctypes.byref(v),
                                        _stream(self.buf)), "tm_workspace_status")
        return int(v.value)


def _set_plan(ws: Workspace, idx: torch.Tensor):
    ws.plan_idx = idx
    ws.plan_version = idx._version


def plan_matches(ws: Workspace, idx: torch.Tensor) -> bool:
    return ws.plan_idx is idx and ws.plan_version == idx._version


# ------------------------------------------------------------------ K1 ----
def router_topk(x: torch.Tensor, router_w: torch.Tensor, top_k: int, ws: Workspace,
                want_logits: bool = False):
    """Fused router: returns ``(idx int64 [T,k], w [T,k] act dtype[, logits [T,E]])``
    and leaves the routing plan for these indices in ``ws``."""
    _need_cuda(x, router_w)
    if x.dtype != router_w.dtype:
        raise TurboMoEError(f"router weight dtype {router_w.dtype} != hidden dtype {x.dtype}")
    x = x.contiguous()
    router_w = router_w.contiguous()
    T, H = x.shape
    E = router_w.shape[0]
    buf = ws.ensure(T, top_k)
    idx = torch.empty(T, top_k, dtype=torch.int64, device=x.device)
    w = torch.empty(T, top_k, dtype=x.dtype, device=x.device)
    logits = torch.empty(T, E, dtype=x.dtype, device=x.device) if want_logits else None
    check(lib().tm_router_topk(x.data_ptr(), T, H, _code(x.dtype), router_w.data_ptr(), E, top_k,
                               idx.data_ptr(), w.data_ptr(), _ptr(logits), buf.data_ptr(), buf.numel(),
                               _stream(x)), "tm_router_topk")
    _set_plan(ws, idx)
    return (idx, w, logits) if want_logits else (idx, w)


def rmsnorm_router_topk(x: torch.Tensor, norm_w: torch.Tensor, eps: float, router_w: torch.Tensor, top_k: int,
                        ws: Workspace, x_norm_out: torch.Tensor):
    """One token: RMSNorm of ``x`` (written to ``x_norm_out``) and the router on
    the normalised token in one launch (tm_rmsnorm_router_topk).  Returns
    ``(idx, w)`` and leaves the plan in ``ws``, like ``router_topk``."""
    _need_cuda(x, norm_w, router_w, x_norm_out)
    T, H = x.shape
    if T != 1:
        raise TurboMoEError("rmsnorm_router_topk takes one token")
    E = router_w.shape[0]
    buf = ws.ensure(1, top_k)
    idx = torch.empty(1, top_k, dtype=torch.int64, device=x.device)
    w = torch.empty(1, top_k, dtype=x.dtype, device=x.device)
    check(lib().tm_rmsnorm_router_topk(x.contiguous().data_ptr(), H, _code(x.dtype), norm_w.data_ptr(), eps,
                                       x_norm_out.data_ptr(), router_w.contiguous().data_ptr(), E, top_k,
                                       idx.data_ptr(), w.data_ptr(), None, buf.data_ptr(), buf.numel(),
                                       _stream(x)), "tm_rmsnorm_router_topk")
    _set_plan(ws, idx)
    return idx, w


def read_plan(ws: Workspace, tokens: int, top_k: int):
    """Copy the routing plan of the last router/plan call out of ``ws`` (host
    tensors; synchronises).  Returns dict(n_active, counts [E], offsets [E+1],
    experts (ascending active ids), slot_token, slot_pair, pair_slot)."""
    import ctypes
    off = (ctypes.c_int64 * 8)()
    check(lib().tm_plan_offsets(tokens, ws.E, top_k, off), "tm_plan_offsets")
    b = ws.buf
    P = tokens * top_k

    def i32(o, n):
        return b[o:o + 4 * n].view(torch.int32).cpu()

    meta = i32(off[0], 3)
    na = int(meta[0])
    return {"n_active": na, "pairs": int(meta[1]), "tokens": int(meta[2]),
            "counts": i32(off[1], ws.E), "offsets": i32(off[2], ws.E + 1),
            "experts": i32(off[3], na), "slot_token": i32(off[4], P), "slot_pair": i32(off[5], P),
            "pair_slot": i32(off[6], P)}


def plan_views(ws: Workspace, tokens: int, top_k: int):
    """Device int32 views (no copy) of the routing plan in ``ws``: dict of
    counts [E], offsets [E+1], slot_token [P], slot_pair [P], pair_slot [P]."""
    import ctypes
    off = (ctypes.c_int64 * 8)()
    check(lib().tm_plan_offsets(tokens, ws.E, top_k, off), "tm_plan_offsets")
    b = ws.buf
    P = tokens * top_k

    def i32(o, n):
        return b[o:o + 4 * n].view(torch.int32)

    return {"counts": i32(off[1], ws.E), "offsets": i32(off[2], ws.E + 1), "slot_token": i32(off[4], P),
            "slot_pair": i32(off[5], P), "pair_slot": i32(off[6], P)}


def combine_slots(y: torch.Tensor, w: torch.Tensor, pair_slot: torch.Tensor, out: torch.Tensor,
                  residual: torch.Tensor | None = None):
    """out[t] = residual[t] + sum_r w[t,r] * y[pair_slot[t*k+r]] (tm_combine_slots)."""
    _need_cuda(y, w, pair_slot, out)
    T, k = w.shape
    ps = pair_slot.to(torch.int32).contiguous()
    w = w.to(out.dtype).contiguous()
    y = y.contiguous()
    check(lib().tm_combine_slots(y.data_ptr(), w.data_ptr(), ps.data_ptr(), T, out.shape[1], k, _code(out.dtype),
                                 _ptr(residual.contiguous() if residual is not None else None), out.data_ptr(),
                                 _stream(out)), "tm_combine_slots")
    return out


def route_plan(idx: torch.Tensor, n_experts: int, ws: Workspace):
    _need_cuda(idx)
    src = idx
    idx = idx.to(torch.int64).contiguous()
    T, k = idx.shape
    buf = ws.ensure(T, k)
    check(lib().tm_route_plan(idx.data_ptr(), T, k, n_experts, buf.data_ptr(), buf.numel(), _stream(idx)),
          "tm_route_plan")
    _set_plan(ws, src)


# --------------------------------------------------------------- K2/K3 ----
def moe_gateup(x: torch.Tensor, top_k: int, packed: PackedExperts, ws: Workspace,
               shared: PackedExperts | None = None, shared_gate_w: torch.Tensor | None = None,
               prefetch_down: bool = False):
    """K2 alone: gate+up + SwiGLU for the plan already in ``ws`` (h stays in ``ws``).
    ``prefetch_down``: also pull the down projections of the same experts into
    L2 for the K3 call that follows (tm_moe_decode_gateup_prefetch)."""
    T, H = x.shape
    Is = shared.inter if shared is not None else 0
    if shared is not None and shared_gate_w is None:
        raise TurboMoEError("shared expert needs its gate weight")
    sgw = shared_gate_w.reshape(-1).to(x.dtype).contiguous() if shared is not None else None
    buf = ws.buf
    head = (x.data_ptr(), T, H, packed.inter, packed.n_experts, top_k, _code(x.dtype),
            packed.w13.data_ptr(), packed.s13.data_ptr(),
            _ptr(shared.w13) if shared else None, _ptr(shared.s13) if shared else None, Is, _ptr(sgw))
    if prefetch_down:
        check(lib().tm_moe_decode_gateup_prefetch(*head, packed.w2.data_ptr(), _ptr(shared.w2) if shared else None,
                                                  buf.data_ptr(), buf.numel(), _stream(x)),
              "tm_moe_decode_gateup_prefetch")
    else:
        check(lib().tm_moe_decode_gateup(*head, buf.data_ptr(), buf.numel(), _stream(x)), "tm_moe_decode_gateup")


def prefetch_experts_l2(packed: PackedExperts, expert_ids: torch.Tensor):
    """Bulk-prefetch the gate/up weights of ``expert_ids`` (device int64, any
    shape; ids outside [0, E) skipped) of one packed layer into L2 on the
    current stream.  A hint: no result depends on it."""
    ids = expert_ids.reshape(-1)
    if ids.dtype != torch.int64 or not ids.is_contiguous():
        raise TurboMoEError("expert ids must be a contiguous int64 tensor")
    n13 = lib().tm_packed_w13_bytes(packed.hidden, packed.inter)
    check(lib().tm_prefetch_experts_l2(packed.w13.data_ptr(), n13, packed.n_experts, ids.data_ptr(), ids.numel(),
                                       _stream(ids)), "tm_prefetch_experts_l2")


def moe_down_combine(w: torch.Tensor, packed: PackedExperts, ws: Workspace, out: torch.Tensor,
                     shared: PackedExperts | None = None, residual: torch.Tensor | None = None):
    """K3 alone: down projection + weighted combine into ``out`` (after K2)."""
    T, H = out.shape
    k = w.shape[1]
    Is = shared.inter if shared is not None else 0
    buf = ws.buf
    check(lib().tm_moe_decode_down_combine(T, H, packed.inter, packed.n_experts, k, _code(out.dtype), w.data_ptr(),
                                           packed.w2.data_ptr(), packed.s2.data_ptr(),
                                           _ptr(shared.w2) if shared else None, _ptr(shared.s2) if shared else None,
                                           Is, _ptr(residual), out.data_ptr(), buf.data_ptr(), buf.numel(),
                                           _stream(out)), "tm_moe_decode_down_combine")


# Calls with at least this many tokens (16-bit activations, a shared expert
# only of the routed experts' inter size) run on tensor-core grouped GEMMs.
# Measured on B200, Qwen3-30B-A3B layer (128 experts, top-8): the decode
# kernels win at 4 tokens (55 vs 92 us), tie at 8, and the grouped GEMMs win
# from 16 tokens (167 vs 181 us) to 2048 (298 us vs 9.7 ms).
PREFILL_MIN_TOKENS = 16
# bf16 calls with up to this many (token, expert) pairs per expert on average
# (T * top_k / n_experts) use the FP8 grouped GEMMs (K7, tm_moe_grouped_f8);
# busier experts and fp16 use the dequantising ones (K4,
# tm_moe_prefill_grouped).  K7 multiplies groups of <= 32 tokens per weight
# tile, so its cost grows with the rows per expert while K4's barely does.
# Measured on B200 (K7 / K4, us): Qwen3-30B-A3B layer (128 experts, top-8)
# 111 / 170 at 16 tokens, 149 / 233 at 64, 166 / 235 at 256, 228 / 237 at 512
# (32 per expert), 373 / 247 at 1024 (64 per expert); 64 experts x 256 tokens
# (32 per expert) 132 / 143; 16 experts x 256 tokens (128 per expert) 104 /
# 70; Qwen3.5 64-token layer 177 / 281.
F8_MAX_ROWS_PER_EXPERT = 32
F8_MAX_TOKENS = 512   # the Qwen3-30B-A3B bound of the rule above (512 * 8 / 128)


def f8_eligible(T: int, dtype, packed: PackedExperts, top_k: int) -> bool:
    """Whether a grouped call (prefill_eligible) runs on K7 rather than K4."""
    return dtype == torch.bfloat16 and T * top_k <= F8_MAX_ROWS_PER_EXPERT * packed.n_experts


def prefill_eligible(T: int, dtype, packed: PackedExperts, shared, top_k: int = 8) -> bool:
    """Whether a call of T tokens runs on the tcgen05 grouped GEMMs (K4): 16-bit
    activations, hidden % 256 == 0, and a shared expert (if any) of the routed
    experts' inter size."""
    if shared is not None and (shared.inter != packed.inter or packed.n_experts <= top_k):
        return False
    return T >= PREFILL_MIN_TOKENS and dtype in (torch.bfloat16, torch.float16) and packed.hidden % 256 == 0


def moe_prefill(x: torch.Tensor, w: torch.Tensor, packed: PackedExperts, ws: Workspace, out: torch.Tensor,
                residual: torch.Tensor | None = None, shared: PackedExperts | None = None,
                shared_gate_w: torch.Tensor | None = None):
    """K4: grouped-GEMM expert FFN (+ gated shared expert) + combine for the
    plan already in ``ws``."""
    T, H = x.shape
    k = w.shape[1]
    if shared is not None and shared_gate_w is None:
        raise TurboMoEError("shared expert needs its gate weight")
    if shared is not None and ws.Is < shared.inter:
        raise TurboMoEError("workspace was sized without the shared expert")
    buf = ws.buf
    gate = shared_gate_w.reshape(-1).to(x.dtype).contiguous() if shared is not None else None
    sh = (shared.w13.data_ptr(), shared.s13.data_ptr(), shared.w2.data_ptr(), shared.s2.data_ptr(), shared.inter,
          gate.data_ptr()) if shared is not None else (None, None, None, None, 0, None)
    check(lib().tm_moe_prefill_grouped(x.data_ptr(), T, H, packed.inter, packed.n_experts, k, _code(x.dtype),
                                       w.data_ptr(), packed.w13.data_ptr(), packed.s13.data_ptr(),
                                       packed.w2.data_ptr(), packed.s2.data_ptr(), *sh, _ptr(residual),
                                       out.data_ptr(), buf.data_ptr(), buf.numel(), _stream(x)),
          "tm_moe_prefill_grouped")


def moe_grouped_f8(x: torch.Tensor, w: torch.Tensor, packed: PackedExperts, ws: Workspace, out: torch.Tensor,
                   residual: torch.Tensor | None = None, shared: PackedExperts | None = None,
                   shared_gate_w: torch.Tensor | None = None):
    """K7: the same call as ``moe_prefill`` on the FP8 tensor-core GEMMs
    (tm_moe_grouped_f8; bf16 activations) for the plan already in ``ws``."""
    T, H = x.shape
    k = w.shape[1]
    if shared is not None and shared_gate_w is None:
        raise TurboMoEError("shared expert needs its gate weight")
    if shared is not None and ws.Is < shared.inter:
        raise TurboMoEError("workspace was sized without the shared expert")
    buf = ws.buf
    gate = shared_gate_w.reshape(-1).to(x.dtype).contiguous() if shared is not None else None
    sh = (shared.w13.data_ptr(), shared.s13.data_ptr(), shared.w2.data_ptr(), shared.s2.data_ptr(), shared.inter,
          gate.data_ptr()) if shared is not None else (None, None, None, None, 0, None)
    check(lib().tm_moe_grouped_f8(x.data_ptr(), T, H, packed.inter, packed.n_experts, k, _code(x.dtype),
                                  w.data_ptr(), packed.w13.data_ptr(), packed.s13.data_ptr(),
                                  packed.w2.data_ptr(), packed.s2.data_ptr(), *sh, _ptr(residual),
                                  out.data_ptr(), buf.data_ptr(), buf.numel(), _stream(x)),
          "tm_moe_grouped_f8")


def moe_experts(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, packed: PackedExperts, ws: Workspace,
                shared: PackedExperts | None = None, shared_gate_w: torch.Tensor | None = None,
                residual: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts (+ sigmoid-gated shared expert, + residual) for tokens
    ``x [T,H]`` routed by ``idx/w [T,k]``.  Reuses the plan in ``ws`` when it
    was built from this very ``idx`` tensor; otherwise builds it."""
    _need_cuda(x, idx, w)
    x = x.contiguous()
    T, H = x.shape
    k = idx.shape[1]
    if not plan_matches(ws, idx):
        route_plan(idx, packed.n_experts, ws)
    ws.ensure(T, k)
    if w.dtype != x.dtype:
        w = w.to(x.dtype)
    w = w.contiguous()
    if out is None:
        out = torch.empty_like(x)
    if prefill_eligible(T, x.dtype, packed, shared, k):
        fn = moe_grouped_f8 if f8_eligible(T, x.dtype, packed, k) else moe_prefill
        fn(x, w, packed, ws, out, residual.contiguous() if residual is not None else None, shared, shared_gate_w)
        return out
    moe_gateup(x, k, packed, ws, shared, shared_gate_w, prefetch_down=True)
    moe_down_combine(w, packed, ws, out, shared, residual.contiguous() if residual is not None else None)
    return out


# ------------------------------------------------ dense FP8 linear (K6) ----
@dataclass
class PackedLinear:
    """One FP8 block-scaled dense weight [out_features, in_features], packed for
    tm_fp8_linear (scales kept in the checkpoint layout)."""
    w: torch.Tensor       # uint8 [N * K], packed
    s: torch.Tensor       # fp32 [N/128, K/128]
    out_features: int
    in_features: int


def pack_linear(w_fp8: torch.Tensor, scale_inv: torch.Tensor) -> PackedLinear:
    """Pack a checkpoint's e4m3 ``weight`` [N, K] + ``weight_scale_inv`` [N/128, K/128]."""
    _need_cuda(w_fp8, scale_inv)
    N, K = w_fp8.shape
    w = _u8(w_fp8).contiguous()
    out = torch.empty(N * K, dtype=torch.uint8, device=w.device)
    check(lib().tm_pack_linear(w.data_ptr(), N, K, out.data_ptr(), _stream(w)), "tm_pack_linear")
    return PackedLinear(out, scale_inv.float().contiguous(), N, K)


def rmsnorm_fp8_linear(x: torch.Tensor, norm_w: torch.Tensor, eps: float, pl: PackedLinear,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """One token: ``F.linear(RMSNorm(x), dequantize(W))`` in one kernel
    (tm_rmsnorm_fp8_linear; hidden 2048 or 4096, bf16/fp16)."""
    _need_cuda(x, norm_w)
    T, K = x.shape
    if T != 1 or K != pl.in_features:
        raise TurboMoEError(f"rmsnorm_fp8_linear takes one token of {pl.in_features} features")
    if out is None:
        out = torch.empty(1, pl.out_features, dtype=x.dtype, device=x.device)
    check(lib().tm_rmsnorm_fp8_linear(x.contiguous().data_ptr(), K, _code(x.dtype), norm_w.data_ptr(), eps,
                                      pl.out_features, pl.w.data_ptr(), pl.s.data_ptr(), None, out.data_ptr(), None,
                                      _stream(x)), "tm_rmsnorm_fp8_linear")
    return out


def fp8_linear(x: torch.Tensor, pl: PackedLinear, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(x, dequantize(W))`` (+ residual) on the packed FP8 weight;
    x [T, K] bf16/fp16 -> [T, N] in x's dtype."""
    _need_cuda(x)
    x = x.contiguous()
    T, K = x.shape
    if K != pl.in_features:
        raise TurboMoEError(f"x has {K} features, the weight expects {pl.in_features}")
    if out is None:
        out = torch.empty(T, pl.out_features, dtype=x.dtype, device=x.device)
    res = residual.contiguous() if residual is not None else None
    check(lib().tm_fp8_linear(x.data_ptr(), T, K, pl.out_features, _code(x.dtype), pl.w.data_ptr(),
                              pl.s.data_ptr(), _ptr(res), out.data_ptr(), None, _stream(x)), "tm_fp8_linear")
    return out


# ------------------------------------------------------------------ K9 ----
def gdn_decode(qkv: torch.Tensor, z: torch.Tensor, a: torch.Tensor, b: torch.Tensor, conv_w: torch.Tensor,
               A_log: torch.Tensor, dt_bias: torch.Tensor, norm_w: torch.Tensor, conv_state: torch.Tensor,
               conv_state_out: torch.Tensor, recurrent_state: torch.Tensor, n_k_heads: int, eps: float = 1e-6,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode token of Qwen3.5 linear attention per batch row
    (tm_gdn_decode): conv-state update + depthwise conv + SiLU, q/k l2norm,
    gates, gated delta rule on the fp32 ``recurrent_state`` [B, Hv, 128, 128]
    (updated in place) and the gated RMSNorm.  ``conv_state`` [B, conv_dim,
    K] is read; the shifted state goes to ``conv_state_out`` (a different
    buffer).  qkv [B, conv_dim], z [B, Hv*128], a/b [B, Hv], conv_w
    [conv_dim, K], norm_w [128] in the act dtype; A_log, dt_bias [Hv] (any
    float dtype, passed as fp32).  Returns [B, Hv*128] in the act dtype."""
    _need_cuda(qkv, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, conv_state_out, recurrent_state)
    B, conv_dim = qkv.shape
    Hv = a.shape[-1]
    K = conv_w.shape[-1]
    dt = qkv.dtype
    if recurrent_state.dtype != torch.float32 or tuple(recurrent_state.shape) != (B, Hv, 128, 128):
        raise TurboMoEError(f"recurrent_state must be fp32 [{B}, {Hv}, 128, 128]")
    if not recurrent_state.is_contiguous():
        raise TurboMoEError("recurrent_state must be contiguous (it is updated in place)")
    if conv_dim != 2 * n_k_heads * 128 + Hv * 128 or tuple(conv_w.shape) != (conv_dim, K):
        raise TurboMoEError(f"qkv [{B}, {conv_dim}] / conv_w {tuple(conv_w.shape)} do not match "
                            f"{n_k_heads} key heads and {Hv} value heads of 128")
    for name, t, shape in (("z", z, (B, Hv * 128)), ("a", a, (B, Hv)), ("b", b, (B, Hv)),
                           ("conv_state", conv_state, (B, conv_dim, K)),
                           ("conv_state_out", conv_state_out, (B, conv_dim, K)), ("norm_w", norm_w, (128,))):
        if tuple(t.shape) != shape or t.dtype != dt:
            raise TurboMoEError(f"{name} must be {dt} {list(shape)}, got {t.dtype} {list(t.shape)}")
    if not conv_state_out.is_contiguous():
        raise TurboMoEError("conv_state_out must be contiguous")
    if A_log.numel() != Hv or dt_bias.numel() != Hv:
        raise TurboMoEError(f"A_log and dt_bias must hold {Hv} values (one per value head)")
    if out is None:
        out = torch.empty(B, Hv * 128, dtype=dt, device=qkv.device)
    elif tuple(out.shape) != (B, Hv * 128) or out.dtype != dt or not out.is_contiguous():
        raise TurboMoEError(f"out must be a contiguous {dt} [{B}, {Hv * 128}] tensor")
    qkv, z, a, b, conv_w, conv_state = (t.contiguous() for t in (qkv, z, a, b, conv_w, conv_state))
    A32 = A_log.float().contiguous()
    dt32 = dt_bias.float().contiguous()
    check(lib().tm_gdn_decode(qkv.data_ptr(), z.data_ptr(), a.data_ptr(), b.data_ptr(), B, n_k_heads, Hv, 128, 128,
                              K, _code(dt), conv_w.data_ptr(), A32.data_ptr(), dt32.data_ptr(),
                              norm_w.contiguous().data_ptr(), eps, conv_state.data_ptr(), conv_state_out.data_ptr(),
                              recurrent_state.data_ptr(), out.data_ptr(), _stream(qkv)), "tm_gdn_decode")
    return out
