"""GPU parity of the FP8 tensor-core grouped GEMMs (tm_moe_grouped_f8, K7).

The kernels multiply the exact e4m3 weights with the tokens (two e4m3 terms,
exact for bf16 values), apply each 128 x 128 block scale to its fp32 partial
sum, and round g, u, silu(g), h and y to bf16 where the reference's bf16
F.linear / F.silu / * round them (execution/moe.py:157-202).  `emulate`
restates that on the CPU with the exactly dequantised weights (fp32), so the
kernels must agree with it up to the order of the fp32 sums: max-abs <= 1e-2,
cosine >= 0.99999 and most elements bitwise equal.  Against the reference's
own golden outputs the layer-output tolerance applies (max-abs 2e-2, cosine 0.9995).
"""
import pytest
import torch
import torch.nn.functional as F

from golden_util import case_layer, case_x, fixture
from gpu_util import assert_close, packed_from_layer, workspace_for
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

MAXABS, COS = 1e-2, 0.99999
BF = torch.bfloat16


def _r(t):
    return t.to(BF).float()


def _expert(x32, g, gs, u, us, d, ds):
    wg, wu, wd = O.dequant_fp32_exact(g, gs), O.dequant_fp32_exact(u, us), O.dequant_fp32_exact(d, ds)
    gg, uu = _r(x32 @ wg.T), _r(x32 @ wu.T)
    h = _r(_r(F.silu(gg)) * uu)
    return _r(h @ wd.T)


def emulate(lw, x, idx, w, residual=None, shared=False):
    T, H = x.shape
    k = idx.shape[1]
    x32 = x.float()
    ypair = torch.zeros(T, k, H)
    E = lw.gate.shape[0]
    for e in torch.unique(idx[(idx >= 0) & (idx < E)]).tolist():
        t, r = torch.where(idx == e)
        ypair[t, r] = _expert(x32[t], lw.gate[e], lw.gate_s[e], lw.up[e], lw.up_s[e], lw.down[e], lw.down_s[e])
    acc = torch.zeros(T, H)
    for r in range(k):
        acc = acc + w[:, r].float().unsqueeze(1) * ypair[:, r]
    if shared:
        y = _expert(x32, lw.sh_gate, lw.sh_gate_s, lw.sh_up, lw.sh_up_s, lw.sh_down, lw.sh_down_s)
        score = _r(torch.sigmoid(_r(x32 @ lw.sh_router.to(BF).float().reshape(-1))))
        acc = acc + score.unsqueeze(1) * y
    if residual is not None:
        acc = acc + residual.float()
    return acc.to(BF)


def run_f8(lw, shape, x, idx, w, residual=None, shared=False):
    from turbomoe import ops
    experts, sh, gate = packed_from_layer(lw)
    ws = workspace_for(shape)
    xd, idd, wd = x.cuda(), idx.cuda(), w.to(BF).cuda()
    ops.route_plan(idd, shape.experts, ws)
    ws.ensure(x.shape[0], idx.shape[1])
    out = torch.empty_like(xd)
    ops.moe_grouped_f8(xd, wd, experts, ws, out, residual.cuda() if residual is not None else None,
                       sh if shared else None, gate.to(BF).cuda() if shared else None)
    st = ws.status()
    return out.cpu(), st


def _check(out, ref, what, min_equal=0.8):
    m, c = assert_close(out.float(), ref.float(), MAXABS, COS, what)
    eq = (out == ref).float().mean().item()
    assert eq >= min_equal, f"{what}: only {eq:.3f} of elements bitwise equal"


def _routing(shape, lw, x):
    layer = O.OracleLayer(lw, x.dtype)
    return O.compute_routing(x, layer.router, shape.top_k)


@pytest.mark.parametrize("T", [16, 200, 600])
def test_f8_vs_emulation(T):
    """Ragged experts: ~4, ~50 and ~150 tokens per expert (1 and 3 token
    groups of <= 64 per expert)."""
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 16, 4, 0)
    lw = synth.make_layer(shape, 41, 0)
    x = synth.make_hidden(T, 512, 3 + T, dtype=BF)
    idx, w = _routing(shape, lw, x)
    out, st = run_f8(lw, shape, x, idx, w)
    assert st == 0
    _check(out, emulate(lw, x, idx, w), f"f8 T={T}")


def test_f8_hot_experts_residual_and_invalid_ids():
    """Few experts with hundreds of tokens (several groups), idle experts, a
    residual, and out-of-range ids (skipped, flagged)."""
    from turbomoe import synth
    shape = synth.MoEShape(256, 384, 12, 2, 0)
    lw = synth.make_layer(shape, 5, 0)
    T = 517
    x = synth.make_hidden(T, 256, 4, dtype=BF)
    g = torch.Generator().manual_seed(1)
    idx = torch.stack([torch.tensor([0, 3]) if t % 3 else torch.tensor([7, 3]) for t in range(T)])
    w = torch.rand(T, 2, generator=g).to(BF)
    res = torch.randn(T, 256, generator=g).to(BF)
    out, st = run_f8(lw, shape, x, idx, w, residual=res)
    assert st == 0
    _check(out, emulate(lw, x, idx, w, residual=res), "hot experts + residual")
    idx[::7, 1] = 99
    out, st = run_f8(lw, shape, x, idx, w, residual=res)
    assert st == 1                # TM_STATUS_BAD_EXPERT_ID, from the plan
    _check(out, emulate(lw, x, idx, w, residual=res), "invalid ids")


@pytest.mark.parametrize("T", [64, 17])
def test_f8_shared_expert(T):
    from turbomoe import synth
    from gpu_util import oracle_fp32
    shape = synth.MoEShape(512, 256, 16, 4, 256)
    lw = synth.make_layer(shape, 51 + T, 0)
    x = synth.make_hidden(T, 512, 9 + T, dtype=BF)
    idx, w = _routing(shape, lw, x)
    res = torch.randn(T, 512, generator=torch.Generator().manual_seed(T)).to(BF)
    out, st = run_f8(lw, shape, x, idx, w, residual=res, shared=True)
    assert st == 0
    _check(out, emulate(lw, x, idx, w, residual=res, shared=True), f"shared T={T}")
    ref32 = oracle_fp32(lw, x, idx, w) + res.float()
    assert_close(out.float(), ref32, 2e-2, 0.9995, f"shared T={T} vs fp32 oracle")


def test_f8_qwen3_layer_vs_reference_golden():
    """2048 tokens of a Qwen3-30B-A3B layer: the reference's own output."""
    name, T = "q3_c1", 2048
    shape, lw, info = case_layer(name)
    fx = fixture(name)
    x = case_x(name, T, fx)
    idx, w = fx[f"T{T}.idx"].long(), fx[f"T{T}.w"]
    out, st = run_f8(lw, shape, x, idx, w)
    assert st == 0
    rows = fx[f"T{T}.rows"]
    assert_close(out[rows].float(), fx[f"T{T}.y_rows"].float(), 2e-2, 0.9995, "q3_c1 vs reference")
    sub = rows[:48]
    _check(out[sub], emulate(lw, x[sub], idx[sub], w[sub]), "q3_c1 vs emulation")


def test_f8_qwen35_layer_vs_reference_golden():
    """64 tokens of a Qwen3.5-shaped layer (256 experts, FP8 shared expert):
    the reference's own (fp32) output."""
    name, T = "q35_c3", 64
    shape, lw, info = case_layer(name)
    fx = fixture(name)
    x = case_x(name, T, fx).to(BF)
    idx, w = fx[f"T{T}.idx"].long(), fx[f"T{T}.w"]
    out, st = run_f8(lw, shape, x, idx, w, shared=True)
    assert st == 0
    assert_close(out.float(), fx[f"T{T}.y"].float(), 2e-2, 0.9995, "q35_c3 vs reference")


def test_f8_graph_replay_is_bitwise_stable():
    from turbomoe import ops, synth
    shape = synth.MoEShape(512, 256, 16, 4, 0)
    lw = synth.make_layer(shape, 61, 0)
    T = 96
    x = synth.make_hidden(T, 512, 2, dtype=BF).cuda()
    experts, _, _ = packed_from_layer(lw)
    ws = workspace_for(shape)
    router = lw.router.to(BF).cuda()
    idx, w = ops.router_topk(x, router, shape.top_k, ws)
    out = torch.empty_like(x)
    ops.moe_grouped_f8(x, w, experts, ws, out)
    eager = out.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        idx, w = ops.router_topk(x, router, shape.top_k, ws)
        ops.moe_grouped_f8(x, w, experts, ws, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        idx, w = ops.router_topk(x, router, shape.top_k, ws)
        ops.moe_grouped_f8(x, w, experts, ws, out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert ws.status() == 0
