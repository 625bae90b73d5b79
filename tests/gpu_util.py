"""Helpers shared by the GPU parity tests."""
import torch

from oracle import moe_oracle as O


def packed_from_layer(lw, device="cuda"):
    """(routed PackedExperts, shared PackedExperts|None, shared gate [H]|None)
    for LayerWeights ``lw`` (any device), packed by tm_pack_experts."""
    from turbomoe import ops
    d = lambda t: t.to(device)
    experts = ops.pack_experts(d(lw.gate), d(lw.gate_s), d(lw.up), d(lw.up_s), d(lw.down), d(lw.down_s))
    shared = gate = None
    if lw.sh_gate is not None:
        shared = ops.pack_experts(d(lw.sh_gate), d(lw.sh_gate_s), d(lw.sh_up), d(lw.sh_up_s),
                                  d(lw.sh_down), d(lw.sh_down_s))
        gate = d(lw.sh_router).reshape(-1)
    return experts, shared, gate


def workspace_for(shape, device="cuda"):
    from turbomoe import ops
    return ops.Workspace(device, shape.experts, shape.top_k, shape.hidden, shape.inter, shape.shared_inter)


def run_moe(lw, shape, x, idx, w, ws=None, residual=None):
    from turbomoe import ops
    experts, shared, gate = packed_from_layer(lw)
    ws = ws or workspace_for(shape)
    g = gate.to(x.dtype) if gate is not None else None
    return ops.moe_experts(x.cuda(), idx.cuda(), w.cuda(), experts, ws, shared=shared, shared_gate_w=g,
                           residual=residual)


def oracle_fp32(lw, x, idx, w):
    """The reference algorithm evaluated in fp32 (loader dtype fp32, fp32 act):
    the precision the kernels compute in."""
    layer = O.OracleLayer(lw, torch.float32)
    return O.execute_layer(layer, x.float().cpu(), idx.cpu(), w.float().cpu())


def assert_close(out, ref, maxabs, cos, what=""):
    m, c = O.compare(out.cpu(), ref.cpu())
    assert m <= maxabs and c >= cos, f"{what}: max-abs {m:.3e} (<= {maxabs}), cos {c:.7f} (>= {cos})"
    return m, c


def fp32_cos(T, dtype, n_experts=128, top_k=8):
    """Cosine bar against the fp32 evaluation of the reference's algorithm.
    0.99999 where the kernels round only the outputs; 0.99995 for bf16 calls
    that run on the FP8 grouped GEMMs (turbomoe.ops.f8_eligible), which also
    round g, u, silu(g) and h to bf16 where the reference's bf16 F.linear /
    F.silu / * round them (four roundings of up to 2^-9 relative each)."""
    from turbomoe import ops
    if (dtype == torch.bfloat16 and T >= ops.PREFILL_MIN_TOKENS
            and T * top_k <= ops.F8_MAX_ROWS_PER_EXPERT * n_experts):
        return 0.99995
    return 0.99999


def k7_layer(x, idx, w, packed, ws, residual=None):
    """The routed layer on the FP8 grouped GEMMs (K7) whatever the rows per
    expert: the kernels an expert-parallel owner runs (tm_ep_experts), so an
    EP output can be compared with it bit for bit."""
    from turbomoe import ops
    ws.ensure(x.shape[0], idx.shape[1])
    if not ops.plan_matches(ws, idx):
        ops.route_plan(idx, packed.n_experts, ws)
    out = torch.empty_like(x)
    ops.moe_grouped_f8(x, w.to(x.dtype).contiguous(), packed, ws, out,
                       residual.contiguous() if residual is not None else None)
    return out
