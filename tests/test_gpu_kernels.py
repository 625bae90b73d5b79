"""GPU parity of the CUDA kernels against the oracle and the reference's
golden outputs (tests/golden, recorded from the reference itself).

Tolerances: bit-exact for dequantised FP8 -> fp32 weights,
top-k indices and the permutation; max-abs <= 2e-2 and cosine >= 0.9995 for
bf16 layer outputs against the reference.  Against the fp32 evaluation of
the same algorithm (what the kernels compute), the bar is tighter.
"""
import pytest
import torch

from golden_util import DTYPES, case_layer, case_x, fixture, meta
from gpu_util import assert_close, fp32_cos, oracle_fp32, packed_from_layer, run_moe, workspace_for
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

REF_MAXABS, REF_COS = 2e-2, 0.9995        # layer-output tolerance vs the reference outputs
FP32_COS = 0.99999                       # vs the fp32 oracle (output rounding only; see fp32_cos)


def _bits(t):
    t = t.contiguous().cpu()
    return t.view(torch.int32) if t.dtype == torch.float32 else t.view(torch.int16)


# ------------------------------------------------------------------ K0 ----
@pytest.mark.parametrize("mat", ["gate_proj", "down_proj", "allbits"])
@pytest.mark.parametrize("dn", ["fp32", "bf16", "fp16"])
def test_dequant_bit_exact_vs_reference(mat, dn):
    from turbomoe import ops
    fx = fixture("dequant")
    out = ops.dequant_fp8_block(fx[f"{mat}.w"].cuda(), fx[f"{mat}.s"].cuda(), DTYPES[dn])
    ref = fx[f"{mat}.out_{dn}"]
    nan = torch.isnan(out.float().cpu()) & torch.isnan(ref.float())
    assert bool(((_bits(out) == _bits(ref)) | nan).all())


def test_dequant_full_expert_bit_exact():
    from turbomoe import ops, synth
    lw = synth.make_layer(synth.MoEShape(2048, 768, 2, 2, 0), 7, 0)
    out = ops.dequant_fp8_block(lw.gate[1].cuda(), lw.gate_s[1].cuda(), torch.float32)
    ref = O.dequant_fp32_exact(lw.gate[1], lw.gate_s[1])
    assert torch.equal(_bits(out), _bits(ref))


# ------------------------------------------------------------------ K5 ----
@pytest.mark.parametrize("dn", ["fp32", "bf16"])
def test_pack_unpack_round_trip(dn):
    from turbomoe import ops, synth
    shape = synth.MoEShape(512, 256, 4, 2, 0)
    lw = synth.make_layer(shape, 3, 0)
    experts, _, _ = packed_from_layer(lw)
    dt = DTYPES[dn]
    for e in range(shape.experts):
        g, u, d = ops.unpack_expert(experts, e, dt)
        assert torch.equal(_bits(g), _bits(O.dequantize_weight(lw.gate[e], lw.gate_s[e], dt)))
        assert torch.equal(_bits(u), _bits(O.dequantize_weight(lw.up[e], lw.up_s[e], dt)))
        assert torch.equal(_bits(d), _bits(O.dequantize_weight(lw.down[e], lw.down_s[e], dt)))


# ------------------------------------------------------------------ K1 ----
ROUTER_CASES = [("q3_small", 1), ("q3_small", 5), ("q3_small", 64), ("q3_small_fp16", 33),
                ("q35_small", 64), ("q3_c0", 1), ("q3_c1", 2048), ("q35_c3", 64)]


def _router(name, T):
    from turbomoe import ops
    shape, lw, info = case_layer(name)
    fx = fixture(name)
    x = case_x(name, T, fx)
    dt = DTYPES[info["dtype"]]
    ws = workspace_for(shape)
    idx, w, logits = ops.router_topk(x.cuda(), lw.router.to(dt).cuda(), shape.top_k, ws, want_logits=True)
    return shape, lw, fx, x, ws, idx.cpu(), w.cpu(), logits.cpu()


@pytest.mark.parametrize("name,T", ROUTER_CASES)
def test_router_topk(name, T):
    """Top-k is bit-exact given the logits; logits agree with the reference's
    F.linear to within one act-dtype ulp (accumulation order differs)."""
    from turbomoe import ops
    shape, lw, fx, x, ws, idx, w, logits = _router(name, T)
    # (1) selection: identical to the stated policy applied to the kernel's own logits
    ref_idx, ref_p = O.topk_from_logits_stable(logits, shape.top_k)
    assert torch.equal(idx, ref_idx)
    ref_w = O.renormalise(ref_p, logits.dtype)
    assert (w.float() - ref_w.float()).abs().max().item() <= 2 * torch.finfo(logits.dtype).eps
    # (2) logits vs the reference's F.linear output
    if f"T{T}.rows" in fx:
        rows = fx[f"T{T}.rows"]
        gl, kl = fx[f"T{T}.logits_rows"].float(), logits[rows].float()
        gidx, kidx = fx[f"T{T}.idx"].long()[rows], idx[rows]
    else:
        gl, kl, gidx, kidx = fx[f"T{T}.logits"].float(), logits.float(), fx[f"T{T}.idx"].long(), idx
    # one act-dtype ulp, plus fp32 accumulation-order noise for fp32 logits
    ulp = torch.finfo(logits.dtype).eps * gl.abs().clamp_min(1e-3) * 1.01 + 2e-5
    assert bool(((gl - kl).abs() <= ulp).all())
    # (3) where the reference's own logits have no tie/near-tie at the top-k
    # boundary, the selected sets agree with the reference
    srt = torch.sort(gl, dim=-1, descending=True).values
    gap = srt[:, shape.top_k - 1] - srt[:, shape.top_k]
    clear = gap > 2 * ulp.max(dim=-1).values
    if gl.shape[0] >= 32:        # most rows of a large batch have a clear boundary
        assert clear.float().mean().item() > 0.5
    same = (torch.sort(kidx, -1).values == torch.sort(gidx, -1).values).all(-1)
    assert bool(same[clear].all())
    # (4) the plan in the workspace is the reference's grouping of these indices
    plan = ops.read_plan(ws, T, shape.top_k)
    grp = O.routing_groups(idx, shape.experts)
    assert torch.equal(plan["counts"].long(), grp["counts"])
    assert torch.equal(plan["offsets"].long(), grp["offsets"])
    assert plan["experts"].tolist() == grp["experts"]
    assert torch.equal(plan["slot_token"].long(), grp["tokens"])
    assert torch.equal((plan["slot_pair"] % shape.top_k).long(), grp["kpos"])
    inv = torch.empty_like(plan["pair_slot"])
    inv[plan["slot_pair"].long()] = torch.arange(T * shape.top_k, dtype=torch.int32)
    assert torch.equal(inv, plan["pair_slot"])


def test_route_plan_matches_grouping_and_flags_bad_ids():
    from turbomoe import ops, synth
    shape = synth.MoEShape(512, 256, 32, 4, 0)
    ws = workspace_for(shape)
    g = torch.Generator().manual_seed(0)
    for T in (1, 3, 100, 1000):
        idx = torch.stack([torch.randperm(32, generator=g)[:4] for _ in range(T)])
        ops.route_plan(idx.cuda(), 32, ws)
        plan = ops.read_plan(ws, T, 4)
        grp = O.routing_groups(idx, 32)
        assert torch.equal(plan["slot_token"].long(), grp["tokens"])
        assert torch.equal(plan["counts"].long(), grp["counts"])
        assert ws.status() == 0
    bad = torch.tensor([[0, 40], [-1, 3]])
    ops.route_plan(bad.cuda(), 32, ws)
    assert ws.status() == 1          # TM_STATUS_BAD_EXPERT_ID
    assert ws.status() == 0          # reading clears it


# --------------------------------------------------------------- K2/K3 ----
LAYER_CASES = [("q3_small", 1), ("q3_small", 5), ("q3_small", 64), ("q3_small_fp16", 1),
               ("q3_small_fp16", 33), ("q35_small", 1), ("q35_small", 64), ("q3_c0", 1),
               ("q35_c3", 64), ("q3_c1", 2048)]


@pytest.mark.parametrize("name,T", LAYER_CASES)
def test_layer_vs_reference_golden(name, T):
    """Same idx/w as the reference run -> layer output within the layer-output
    tolerance of the reference's own output, and tight vs the fp32 oracle."""
    shape, lw, info = case_layer(name)
    fx = fixture(name)
    x = case_x(name, T, fx)
    idx, w = fx[f"T{T}.idx"].long(), fx[f"T{T}.w"]
    y = run_moe(lw, shape, x, idx, w).cpu()
    if f"T{T}.rows" in fx:
        rows = fx[f"T{T}.rows"]
        assert_close(y[rows], fx[f"T{T}.y_rows"], REF_MAXABS, REF_COS, f"{name} T={T} vs reference")
    else:
        assert_close(y, fx[f"T{T}.y"], REF_MAXABS, REF_COS, f"{name} T={T} vs reference")
    if T <= 64:
        ref32 = oracle_fp32(lw, x, idx, w)
        tol = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1e-2}[x.dtype]
        assert_close(y, ref32, tol, fp32_cos(T, x.dtype, shape.experts, shape.top_k), f"{name} T={T} vs fp32 oracle")


@pytest.mark.parametrize("T", [1, 2, 3, 4, 7, 8, 9, 16, 63, 64, 65, 200])
def test_token_counts_and_ragged_groups(T):
    """Every tokens-per-pass variant, ragged expert groups, T around the
    in-kernel combine limit."""
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 16, 4, 0)
    lw = synth.make_layer(shape, 100 + T, 0)
    x = synth.make_hidden(T, 512, T, dtype=torch.bfloat16)
    layer = O.OracleLayer(lw, torch.bfloat16)
    idx, w = O.compute_routing(x, layer.router, shape.top_k)
    y = run_moe(lw, shape, x, idx, w)
    assert_close(y, oracle_fp32(lw, x, idx, w), 1e-2, fp32_cos(T, torch.bfloat16, shape.experts, shape.top_k),
                 f"T={T}")


def test_shared_expert_and_residual():
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 16, 4, 256)
    lw = synth.make_layer(shape, 9, 0)
    T = 12
    x = synth.make_hidden(T, 512, 1, dtype=torch.float32)
    layer = O.OracleLayer(lw, torch.float32)
    idx, w = O.compute_routing(x, layer.router, shape.top_k)
    res = torch.randn(T, 512)
    y = run_moe(lw, shape, x, idx, w, residual=res.cuda())
    ref = O.execute_layer(layer, x, idx, w) + res
    assert_close(y, ref, 1e-4, 0.999999, "shared+residual fp32")


def test_invalid_expert_ids_are_skipped():
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 8, 2, 0)
    lw = synth.make_layer(shape, 4, 0)
    x = synth.make_hidden(3, 512, 2, dtype=torch.float32)
    idx = torch.tensor([[1, 99], [2, 3], [-5, 0]])
    w = torch.full((3, 2), 0.5)
    ws = workspace_for(shape)
    y = run_moe(lw, shape, x, idx, w, ws=ws)
    keep = idx.clamp(0, 7)
    wk = w * ((idx >= 0) & (idx < 8)).float()
    ref = O.execute_layer(O.OracleLayer(lw, torch.float32), x, keep, wk)
    assert_close(y, ref, 1e-4, 0.99999, "invalid ids")
    assert ws.status() == 1


def test_permutation_equivariance_full_size():
    """Size-independent property at the full Qwen3 layer: permuting the tokens
    permutes the outputs bit-exactly (each token's math is independent)."""
    from turbomoe import ops, synth
    shape = synth.QWEN3_30B_A3B
    lw = synth.make_layer(shape, 5, 0, device="cuda")
    T = 48
    x = synth.make_hidden(T, shape.hidden, 8, dtype=torch.bfloat16, device="cuda")
    ws = workspace_for(shape)
    router = lw.router.cuda()
    idx, w = ops.router_topk(x, router, 8, ws)
    y = run_moe(lw, shape, x, idx, w, ws=ws)
    perm = torch.randperm(T, generator=torch.Generator().manual_seed(1)).cuda()
    idx2, w2 = ops.router_topk(x[perm], router, 8, ws)
    assert torch.equal(idx2, idx[perm]) and torch.equal(w2, w[perm])
    y2 = run_moe(lw, shape, x[perm], idx2, w2, ws=ws)
    assert torch.equal(y2, y[perm])


def test_weight_linearity_full_size():
    """Scaling the routing weights by 2 scales the output by 2 (exact in fp32)."""
    from turbomoe import synth
    shape = synth.QWEN3_30B_A3B
    lw = synth.make_layer(shape, 6, 0, device="cuda")
    x = synth.make_hidden(4, shape.hidden, 3, dtype=torch.float32, device="cuda")
    layer_idx = torch.stack([torch.randperm(128)[:8] for _ in range(4)]).cuda()
    w = torch.rand(4, 8, device="cuda")
    y1 = run_moe(lw, shape, x, layer_idx, w)
    y2 = run_moe(lw, shape, x, layer_idx, 2 * w)
    assert torch.equal(y2, 2 * y1)


def test_cuda_graph_replay_matches_eager():
    from turbomoe import ops, synth
    shape = synth.MoEShape(512, 256, 16, 4, 256)
    lw = synth.make_layer(shape, 12, 0, device="cuda")
    experts, shared, gate = packed_from_layer(lw)
    ws = workspace_for(shape)
    x = synth.make_hidden(2, 512, 3, dtype=torch.bfloat16, device="cuda")
    router = lw.router.cuda()
    ws.ensure(2)

    def step():
        idx, w = ops.router_topk(x, router, 4, ws)
        return ops.moe_experts(x, idx, w, experts, ws, shared=shared, shared_gate_w=gate.to(x.dtype))

    eager = step().clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


# Router tile shapes: one 16-token tile (3, 9, 16 tokens), a ragged second
# tile (17, 40), 64-token tiles with a ragged last one (600), experts that do not fill the last warp (60) and 1..16 n-tiles per
# warp (60, 128, 512, 1024 experts).  Logits against an fp64 dot product of the
# same act-dtype inputs, rounded once: within one act-dtype ulp.
# hidden 4096: two staged passes of the token tile per CTA; hidden 2176: CTAs of
# 8 and 9 chunks (a second pass of one chunk)
TILE_CASES = [(60, 4, 1024, torch.float16), (128, 8, 2048, torch.bfloat16), (512, 10, 1024, torch.bfloat16),
              (1024, 8, 512, torch.float16), (128, 8, 4096, torch.bfloat16), (256, 8, 2176, torch.float16)]


@pytest.mark.parametrize("E,k,H,dt", TILE_CASES)
@pytest.mark.parametrize("T", [3, 9, 16, 17, 40, 600])
def test_router_tile_shapes(E, k, H, dt, T):
    from turbomoe import ops, synth
    g = torch.Generator().manual_seed(E * 100 + T)
    x = torch.randn(T, H, generator=g).to(dt)
    rw = (torch.randn(E, H, generator=g) * 0.05).to(dt)
    ws = ops.Workspace("cuda", E, k, H, 128, 0)
    idx, w, logits = ops.router_topk(x.cuda(), rw.cuda(), k, ws, want_logits=True)
    idx, w, logits = idx.cpu(), w.cpu(), logits.cpu()
    exact = x.double() @ rw.double().T
    ulp = torch.finfo(dt).eps * exact.abs().clamp_min(1e-3) * 1.01
    assert bool(((logits.double() - exact).abs() <= ulp).all())
    ref_idx, ref_p = O.topk_from_logits_stable(logits, k)
    assert torch.equal(idx, ref_idx)
    assert (w.float() - O.renormalise(ref_p, dt).float()).abs().max().item() <= 2 * torch.finfo(dt).eps
    plan = ops.read_plan(ws, T, k)
    grp = O.routing_groups(idx, E)
    assert torch.equal(plan["counts"].long(), grp["counts"])
    assert torch.equal(plan["offsets"].long(), grp["offsets"])
    assert plan["experts"].tolist() == grp["experts"]
    assert torch.equal(plan["slot_token"].long(), grp["tokens"])
    assert torch.equal((plan["slot_pair"] % k).long(), grp["kpos"])
    assert ws.status() == 0


def test_route_plan_many_pairs_flags_bad_ids():
    """The multi-CTA plan (more than 2048 pairs): a bad id gets pair_slot -1,
    is left out of the counts, and sets the status bit; the others keep the
    reference's grouping."""
    from turbomoe import ops, synth
    shape = synth.MoEShape(512, 256, 64, 4, 0)
    ws = workspace_for(shape)
    g = torch.Generator().manual_seed(3)
    T = 700
    idx = torch.stack([torch.randperm(64, generator=g)[:4] for _ in range(T)])
    bad = idx.clone()
    bad[308, 2] = 64                       # pair 1234
    ops.route_plan(bad.cuda(), 64, ws)
    plan = ops.read_plan(ws, T, 4)
    assert ws.status() == 1
    assert int(plan["pair_slot"][1234]) == -1
    counts = torch.bincount(idx.flatten(), minlength=64)
    counts[idx[308, 2]] -= 1
    assert torch.equal(plan["counts"].long(), counts)
    ops.route_plan(idx.cuda(), 64, ws)
    plan = ops.read_plan(ws, T, 4)
    grp = O.routing_groups(idx, 64)
    assert torch.equal(plan["slot_token"].long(), grp["tokens"])
    assert torch.equal((plan["slot_pair"] % 4).long(), grp["kpos"])
    assert ws.status() == 0


@pytest.mark.parametrize("T,shared_inter", [(1, 0), (5, 0), (1, 512), (3, 512)])
def test_gateup_prefetch_matches_plain_gateup(T, shared_inter):
    """tm_moe_decode_gateup_prefetch (K2 that also pulls the down projections
    into L2) gives bit for bit the output of tm_moe_decode_gateup + K3."""
    from turbomoe import ops, synth
    shape = synth.MoEShape(2048, 768, 128, 8, shared_inter)
    lw = synth.make_layer(shape, 31 + T, 0, device="cuda")
    experts, shared, gate = packed_from_layer(lw)
    ws = workspace_for(shape)
    x = synth.make_hidden(T, shape.hidden, 4, dtype=torch.bfloat16, device="cuda")
    idx, w = ops.router_topk(x, lw.router.cuda(), 8, ws)
    g = gate.to(x.dtype) if gate is not None else None
    outs = []
    for pf in (False, True, False, True):
        ops.route_plan(idx, 128, ws)
        ops.moe_gateup(x, 8, experts, ws, shared, g, prefetch_down=pf)
        out = torch.empty_like(x)
        ops.moe_down_combine(w, experts, ws, out, shared, residual=x)
        outs.append(out)
    torch.cuda.synchronize()
    assert ws.status() == 0
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("I", [384, 640, 1536])
def test_one_token_down_inner_sizes(I):
    """One token through k3_down_t1_f8 with inner sizes of 3, 5 and 12
    128-column blocks: K halves of unequal length, and above 1024 the h row
    staged by TMA instead of loaded straight into registers; against the fp32
    evaluation of the reference's algorithm."""
    from turbomoe import synth
    shape = synth.MoEShape(512, I, 8, 2, 0)
    lw = synth.make_layer(shape, 900 + I, 0)
    x = synth.make_hidden(1, 512, I, dtype=torch.bfloat16)
    layer = O.OracleLayer(lw, torch.bfloat16)
    idx, w = O.compute_routing(x, layer.router, shape.top_k)
    y = run_moe(lw, shape, x, idx, w)
    assert_close(y, oracle_fp32(lw, x, idx, w), 1e-2, 0.99999, f"I={I}")
