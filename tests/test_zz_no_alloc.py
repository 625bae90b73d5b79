"""tm_moe_decode_layer_noalloc: the whole decode layer on the library's static
scratch (no caller workspace) against the workspace entry points.

Collected last on purpose (file name): it must pass both alone in a fresh
process (its first call does the per-device set-up) and after every other test
has run the workspace path on the same device.  Two calls in a row with
different inputs and shapes check that nothing from the previous call leaks
through the shared scratch.

Tolerance: none.  Both paths run the same kernels (the router, K2 with the L2
prefetch of the down projections, K3) on the same inputs, so indices, weights
and outputs must be identical bit for bit.
"""
import pytest
import torch

from gpu_util import packed_from_layer, workspace_for

pytestmark = pytest.mark.gpu


def _layer(shape, seed):
    from turbomoe import synth
    lw = synth.make_layer(shape, seed, 0)
    experts, shared, gate = packed_from_layer(lw)
    return lw, experts, shared, gate


def _workspace_path(shape, lw, experts, shared, gate, x, residual):
    """The same three kernels through the workspace entry points (K1, K2 with
    the down-projection prefetch, K3: the no-alloc call never uses the grouped
    GEMMs)."""
    from turbomoe import ops
    ws = workspace_for(shape)
    idx, w = ops.router_topk(x, lw.router.cuda().to(x.dtype), shape.top_k, ws)
    ws.ensure(x.shape[0], shape.top_k)
    out = torch.empty_like(x)
    ops.moe_gateup(x, shape.top_k, experts, ws, shared, gate.to(x.dtype) if gate is not None else None,
                   prefetch_down=True)
    ops.moe_down_combine(w, experts, ws, out, shared, residual)
    return idx, w, out


def _noalloc(shape, lw, experts, shared, gate, x, residual, tokens=None):
    from turbomoe import ops
    from turbomoe._lib import lib
    T = tokens or x.shape[0]
    router_w = lw.router.cuda().to(x.dtype).contiguous()
    idx = torch.full((T, shape.top_k), -7, dtype=torch.int64, device="cuda")
    w = torch.zeros(T, shape.top_k, dtype=x.dtype, device="cuda")
    out = torch.zeros(T, shape.hidden, dtype=x.dtype, device="cuda")
    status = torch.full((1,), 0xFFFF, dtype=torch.int32, device="cuda")
    g = gate.to(x.dtype).contiguous() if gate is not None else None
    p = lambda t: t.data_ptr() if t is not None else None
    rc = lib().tm_moe_decode_layer_noalloc(
        x.data_ptr(), T, shape.hidden, shape.inter, shape.experts, shape.top_k, ops._code(x.dtype),
        router_w.data_ptr(), experts.w13.data_ptr(), experts.s13.data_ptr(), experts.w2.data_ptr(),
        experts.s2.data_ptr(), p(shared.w13 if shared else None), p(shared.s13 if shared else None),
        p(shared.w2 if shared else None), p(shared.s2 if shared else None), shape.shared_inter,
        p(g), p(residual), idx.data_ptr(), w.data_ptr(), out.data_ptr(), status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    return rc, idx, w, out, status


def _check(shape, layer, x, residual):
    ref_idx, ref_w, ref_out = _workspace_path(shape, *layer, x, residual)
    rc, idx, w, out, status = _noalloc(shape, *layer, x, residual)
    torch.cuda.synchronize()
    assert rc == 0
    assert int(status.item()) == 0
    assert torch.equal(idx, ref_idx)
    assert torch.equal(w, ref_w)
    assert torch.equal(out, ref_out), "noalloc output differs from the workspace path"


def test_noalloc_matches_workspace_path_two_calls():
    from turbomoe import synth
    # 1) Qwen3-30B-A3B-sized experts (H 2048, I 768, top-8), one decode token
    s1 = synth.MoEShape(2048, 768, 32, 8, 0)
    l1 = _layer(s1, 11)
    x1 = synth.make_hidden(1, s1.hidden, 5, device="cuda")
    _check(s1, l1, x1, None)
    # 2) straight after: a Qwen3.5-style layer with a shared expert and 64
    #    tokens, with a residual (more of the scratch, different plan)
    s2 = synth.MoEShape(1024, 512, 64, 8, 512)
    l2 = _layer(s2, 12)
    x2 = synth.make_hidden(64, s2.hidden, 6, device="cuda")
    r2 = synth.make_hidden(64, s2.hidden, 7, device="cuda")
    _check(s2, l2, x2, r2)
    # 3) and the first shape again with other tokens: nothing leaks from (2)
    x3 = synth.make_hidden(4, s1.hidden, 8, device="cuda")
    _check(s1, l1, x3, None)


def test_noalloc_rejects_calls_beyond_the_static_scratch():
    from turbomoe import synth
    from turbomoe._lib import TM_ERR_WORKSPACE, TM_NOALLOC_SCRATCH_BYTES, lib
    s = synth.MoEShape(2048, 768, 32, 8, 0)
    layer = _layer(s, 13)
    T = 256   # needs ~24 MB of scratch
    assert lib().tm_workspace_bytes(T, s.experts, s.top_k, s.hidden, s.inter, 0) > TM_NOALLOC_SCRATCH_BYTES
    x = synth.make_hidden(T, s.hidden, 9, device="cuda")
    rc, idx, w, out, status = _noalloc(s, *layer, x, None)
    torch.cuda.synchronize()
    assert rc == TM_ERR_WORKSPACE
    assert b"static scratch" in lib().tm_last_error()
    assert bool((idx == -7).all()) and int(status.item()) == 0xFFFF   # nothing ran
    # and the scratch is still good for a call that fits
    _check(s, layer, x[:2].contiguous(), None)
