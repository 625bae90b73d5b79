"""GPU parity of the tensor-core prefill path (tm_moe_prefill_grouped).

The kernels multiply dequantised weights with the activations on the tensor
cores and accumulate in fp32, rounding h and y to the act dtype as the
reference's F.linear outputs are.  The weights are the reference's own
dequantisation in the act dtype, except for the gate/up GEMM of bf16 calls,
which runs on f16 operands (`gateup_weight`; finer rounding than the
reference's bf16).  `emulate` restates exactly that on the CPU, so the
kernels must agree with it up to fp32 accumulation order: max-abs <= 1e-2,
cosine >= 0.99999 and most elements bitwise equal.  Against the reference's
own golden output (2048-token prefill of a Qwen3-30B-A3B layer) the
layer-output tolerance applies (max-abs 2e-2, cosine 0.9995).
"""
import pytest
import torch
import torch.nn.functional as F

from golden_util import case_layer, case_x, fixture
from gpu_util import assert_close, packed_from_layer, workspace_for
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

MAXABS, COS = 1e-2, 0.99999


def gateup_weight(q, s, dt):
    """The gate/up GEMM's weights: for fp16 activations the reference's fp16
    dequantisation; for bf16 activations the GEMM runs on f16 operands with
    weights round_f16(w * round_f16(scale * 2^8)) / 2^8 (activations enter
    exactly, shifted by a power of 2)."""
    if dt != torch.bfloat16:
        return O.dequantize_weight(q, s, dt).float()
    sf = (s.float() * 256).to(torch.float16)
    sf = sf.repeat_interleave(128, 0).repeat_interleave(128, 1)
    return (q.float().to(torch.float16) * sf).float() / 256


def emulate(lw, x, idx, w, residual=None):
    """CPU restatement of the kernels' arithmetic (see module docstring)."""
    dt = x.dtype
    T, H = x.shape
    k = idx.shape[1]
    xf = x.float()
    ypair = torch.zeros(T, k, H)
    for e in torch.unique(idx[(idx >= 0) & (idx < lw.gate.shape[0])]).tolist():
        t, r = torch.where(idx == e)
        wg = gateup_weight(lw.gate[e], lw.gate_s[e], dt)
        wu = gateup_weight(lw.up[e], lw.up_s[e], dt)
        wd = O.dequantize_weight(lw.down[e], lw.down_s[e], dt).float()
        xe = xf[t]
        h = (F.silu(xe @ wg.T) * (xe @ wu.T)).to(dt).float()
        ypair[t, r] = (h @ wd.T).to(dt).float()
    acc = torch.zeros(T, H)
    for r in range(k):
        acc = acc + w[:, r].float().unsqueeze(1) * ypair[:, r]
    if residual is not None:
        acc = acc + residual.float()
    return acc.to(dt)


def run_prefill(lw, shape, x, idx, w, residual=None):
    from turbomoe import ops
    experts, _, _ = packed_from_layer(lw)
    ws = workspace_for(shape)
    xd, idd, wd = x.cuda(), idx.cuda(), w.to(x.dtype).cuda()
    ops.route_plan(idd, shape.experts, ws)
    ws.ensure(x.shape[0], idx.shape[1])
    out = torch.empty_like(xd)
    ops.moe_prefill(xd, wd, experts, ws, out, residual.cuda() if residual is not None else None)
    st = ws.status()
    return out.cpu(), st


def _check(out, ref, what, min_equal=0.9):
    m, c = assert_close(out.float(), ref.float(), MAXABS, COS, what)
    eq = (out == ref).float().mean().item()
    assert eq >= min_equal, f"{what}: only {eq:.3f} of elements bitwise equal"


def _routing(shape, lw, x):
    layer = O.OracleLayer(lw, x.dtype)
    return O.compute_routing(x, layer.router, shape.top_k)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_prefill_vs_emulation(dt):
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 16, 4, 0)
    lw = synth.make_layer(shape, 21, 0)
    T = 600                       # ~150 tokens per expert: ragged, several token tiles
    x = synth.make_hidden(T, 512, 3, dtype=dt)
    idx, w = _routing(shape, lw, x)
    out, st = run_prefill(lw, shape, x, idx, w)
    assert st == 0
    _check(out, emulate(lw, x, idx, w), f"prefill {dt}")


def test_prefill_hot_experts_residual_and_min_hidden():
    """Few experts with hundreds of tokens each (several token tiles per
    expert, last one ragged), inactive experts, a residual, H = 256."""
    from turbomoe import synth
    shape = synth.MoEShape(256, 384, 12, 2, 0)
    lw = synth.make_layer(shape, 5, 0)
    T = 517
    x = synth.make_hidden(T, 256, 4, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    idx = torch.stack([torch.tensor([0, 3]) if t % 3 else torch.tensor([7, 3]) for t in range(T)])
    w = torch.rand(T, 2, generator=g).to(torch.bfloat16)
    res = torch.randn(T, 256, generator=g).to(torch.bfloat16)
    out, st = run_prefill(lw, shape, x, idx, w, residual=res)
    assert st == 0
    _check(out, emulate(lw, x, idx, w, residual=res), "hot experts + residual")


def test_prefill_invalid_ids_skipped_and_flagged():
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 8, 2, 0)
    lw = synth.make_layer(shape, 6, 0)
    T = 300
    x = synth.make_hidden(T, 512, 5, dtype=torch.bfloat16)
    idx, w = _routing(shape, lw, x)
    idx[::7, 1] = 99
    out, st = run_prefill(lw, shape, x, idx, w)
    assert st == 1                # TM_STATUS_BAD_EXPERT_ID (from the plan)
    _check(out, emulate(lw, x, idx, w), "invalid ids")


def test_prefill_matches_decode_kernels():
    """The two expert paths agree on the same routed tokens."""
    from turbomoe import ops, synth
    shape = synth.MoEShape(512, 256, 16, 4, 0)
    lw = synth.make_layer(shape, 8, 0)
    T = 400
    x = synth.make_hidden(T, 512, 6, dtype=torch.bfloat16)
    idx, w = _routing(shape, lw, x)
    out_pf, _ = run_prefill(lw, shape, x, idx, w)
    experts, _, _ = packed_from_layer(lw)
    ws = workspace_for(shape)
    xd, idd, wd = x.cuda(), idx.cuda(), w.cuda()
    ops.route_plan(idd, shape.experts, ws)
    ws.ensure(T, shape.top_k)
    out_dec = torch.empty_like(xd)
    ops.moe_gateup(xd, shape.top_k, experts, ws)
    ops.moe_down_combine(wd, experts, ws, out_dec)
    assert_close(out_pf.float(), out_dec.cpu().float(), 2e-2, 0.9999, "prefill vs decode kernels")


def test_prefill_qwen3_layer_vs_reference_golden():
    """2048-token prefill of a Qwen3-30B-A3B MoE layer (128 experts, top-8):
    the reference's own output, and the emulation on the golden rows."""
    from turbomoe import ops
    name, T = "q3_c1", 2048
    shape, lw, info = case_layer(name)
    fx = fixture(name)
    x = case_x(name, T, fx)
    idx, w = fx[f"T{T}.idx"].long(), fx[f"T{T}.w"]
    assert T >= ops.PREFILL_MIN_TOKENS     # the layer drop-in routes this call here too
    out, st = run_prefill(lw, shape, x, idx, w)
    assert st == 0
    rows = fx[f"T{T}.rows"]
    assert_close(out[rows].float(), fx[f"T{T}.y_rows"].float(), 2e-2, 0.9995, "q3_c1 vs reference")
    sub = rows[:64]
    ref = emulate(lw, x[sub], idx[sub], w[sub])
    _check(out[sub], ref, "q3_c1 vs emulation")


def emulate_shared(lw, x):
    """The shared expert's term as the kernels compute it: one more group of
    the same GEMMs over every token, times sigmoid(x . gate) with F.linear's
    output and the sigmoid each rounded to the act dtype (moe.py:191-200)."""
    dt = x.dtype
    xf = x.float()
    wg = gateup_weight(lw.sh_gate, lw.sh_gate_s, dt)
    wu = gateup_weight(lw.sh_up, lw.sh_up_s, dt)
    wd = O.dequantize_weight(lw.sh_down, lw.sh_down_s, dt).float()
    h = (F.silu(xf @ wg.T) * (xf @ wu.T)).to(dt).float()
    y = (h @ wd.T).to(dt).float()
    logit = (xf @ lw.sh_router.to(dt).float().reshape(-1)).to(dt).float()
    score = torch.sigmoid(logit).to(dt).float()
    return score.unsqueeze(1) * y


@pytest.mark.parametrize("dt,T", [(torch.bfloat16, 64), (torch.bfloat16, 17), (torch.float16, 40)])
def test_prefill_shared_expert(dt, T):
    """Qwen3.5-style layer (FP8 shared expert of the routed experts' size):
    the shared expert runs as one more group of the grouped GEMMs; the output
    matches the CPU restatement of that arithmetic and, within the
    layer-output tolerance, the fp32 oracle of the reference's layer."""
    from turbomoe import ops, synth
    from gpu_util import oracle_fp32
    shape = synth.MoEShape(512, 256, 16, 4, 256)
    lw = synth.make_layer(shape, 31 + T, 0)
    x = synth.make_hidden(T, 512, 7 + T, dtype=dt)
    layer = O.OracleLayer(lw, dt)
    idx, w = O.compute_routing(x, layer.router, shape.top_k)
    res = torch.randn(T, 512, generator=torch.Generator().manual_seed(T)).to(dt)
    experts, shared, gate = packed_from_layer(lw)
    ws = workspace_for(shape)
    xd, idd, wd = x.cuda(), idx.cuda(), w.to(dt).cuda()
    ops.route_plan(idd, shape.experts, ws)
    ws.ensure(T, shape.top_k)
    assert ops.prefill_eligible(T, dt, experts, shared, shape.top_k)
    out = torch.empty_like(xd)
    ops.moe_prefill(xd, wd, experts, ws, out, res.cuda(), shared, gate.to(dt).cuda())
    assert ws.status() == 0
    out = out.cpu()
    # routed part as emulate() (unrounded), plus the shared term, in the kernels' order
    dtp = x.dtype
    xf = x.float()
    k = idx.shape[1]
    ypair = torch.zeros(T, k, 512)
    for e in torch.unique(idx).tolist():
        t, r = torch.where(idx == e)
        wg = gateup_weight(lw.gate[e], lw.gate_s[e], dtp)
        wu = gateup_weight(lw.up[e], lw.up_s[e], dtp)
        wdn = O.dequantize_weight(lw.down[e], lw.down_s[e], dtp).float()
        h = (F.silu(xf[t] @ wg.T) * (xf[t] @ wu.T)).to(dtp).float()
        ypair[t, r] = (h @ wdn.T).to(dtp).float()
    acc = torch.zeros(T, 512)
    for r in range(k):
        acc = acc + w.to(dtp)[:, r].float().unsqueeze(1) * ypair[:, r]
    want = (acc + emulate_shared(lw, x) + res.float()).to(dtp)
    _check(out, want, f"shared {dt} T={T}", min_equal=0.8)
    ref32 = oracle_fp32(lw, x, idx, w) + res.float()
    assert_close(out.float(), ref32, 2e-2, 0.9995, f"shared {dt} T={T} vs fp32 oracle")
