"""Expert parallelism over peer memory (tm_ep_*) on one GPU.

* One rank owning every expert: dispatch to itself, the owner's grouped GEMMs
  over the received rows, the return and the combine give the same output
  as the single-GPU layer call (bit-exact where both run the tcgen05 GEMMs,
  >= 16 tokens; the oracle's tolerance below that), across calls of different
  token counts and across CUDA-graph replays (device-side epoch).
* A rank whose peer never sends: every bounded wait runs out, the context's
  status reports TM_STATUS_TIMEOUT, and the CUDA context stays usable.
"""
import ctypes as C

import pytest
import torch

from gpu_util import oracle_fp32
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 256, 16, 4


def _layer(seed=77):
    from turbomoe import ops, synth
    shape = synth.MoEShape(H, I, E, K, 0)
    lw = synth.make_layer(shape, seed, 0)
    d = lambda t: t.cuda()
    full = ops.pack_experts(d(lw.gate), d(lw.gate_s), d(lw.up), d(lw.up_s), d(lw.down), d(lw.down_s))
    return shape, lw, full


def test_ep_p2p_single_rank_matches_layer():
    from turbomoe import ops, synth
    from turbomoe.ep import PeerExpertParallelMoE
    shape, lw, full = _layer()
    router = lw.router.cuda()
    ep = PeerExpertParallelMoE(router, full, K, max_tokens=320)
    ws = ops.Workspace("cuda", E, K, H, I, 0)
    try:
        for T in (40, 5, 300, 16):
            x = synth.make_hidden(T, H, 900 + T, device="cuda")
            res = torch.randn(x.shape, generator=torch.Generator(device="cuda").manual_seed(T),
                              device="cuda").to(x.dtype)
            out = ep.forward(x, residual=res)
            idx, w = ops.router_topk(x, router, K, ws)
            ref = ops.moe_experts(x, idx, w, full, ws, residual=res)
            assert ep.status() == 0
            if T >= ops.PREFILL_MIN_TOKENS:
                assert torch.equal(out, ref), (T, (out.float() - ref.float()).abs().max().item())
            # against the fp32 oracle of the reference's layer, same routing
            want = oracle_fp32(lw, x, idx, w) + res.float().cpu()
            maxabs, cos = O.compare(out.cpu(), want)
            assert maxabs <= 2e-2 and cos >= 0.9999, (T, maxabs, cos)
        # CUDA graph: the epoch lives on the device, so replays keep exchanging
        T = 64
        x = synth.make_hidden(T, H, 5, device="cuda")
        eager = ep.forward(x).clone()
        out = torch.empty_like(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep.forward(x, out=out)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ep.forward(x, out=out)
        for _ in range(3):
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, eager)
        assert ep.status() == 0
        del g
    finally:
        ep.close()


def test_ep_p2p_timeout_sets_status():
    """Rank 0 of a 2-rank context whose peer (a second context on the same
    GPU) never runs: the owner's wait for the peer's rows and the source's
    wait for the peer's outputs both expire after the 20 ms limit."""
    from turbomoe import ops, synth
    from turbomoe._lib import TM_EP_HANDLE_BYTES, TM_STATUS_TIMEOUT, check, lib
    L = lib()
    shape, lw, full = _layer(78)
    router = lw.router.cuda()
    code = ops._code(router.dtype)
    ctx = [C.c_void_p(), C.c_void_p()]
    for r in range(2):
        h = (C.c_char * TM_EP_HANDLE_BYTES)()
        check(L.tm_ep_create(r, 2, E, K, H, I, code, 64, h, C.byref(ctx[r])), "tm_ep_create")
    try:
        peers = (C.c_void_p * 2)(None, L.tm_ep_local_buffer(ctx[1]))
        check(L.tm_ep_connect_ptrs(ctx[0], peers), "tm_ep_connect_ptrs")
        check(L.tm_ep_set_timeout(ctx[0], 20_000_000), "tm_ep_set_timeout")
        d = lambda t: t.cuda()
        half = slice(0, E // 2)
        local = ops.pack_experts(d(lw.gate[half]), d(lw.gate_s[half]), d(lw.up[half]), d(lw.up_s[half]),
                                 d(lw.down[half]), d(lw.down_s[half]))
        ws = ops.Workspace("cuda", E, K, H, I, 0)
        ws.ensure(64)
        n = L.tm_ep_owner_workspace_bytes(ctx[0])
        ows = torch.empty(n, dtype=torch.uint8, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        check(L.tm_workspace_init(ows.data_ptr(), n, s), "tm_workspace_init")
        x = synth.make_hidden(24, H, 3, device="cuda")
        idx, w = ops.router_topk(x, router, K, ws)
        out = torch.empty_like(x)
        b = ws.buf
        check(L.tm_ep_dispatch(ctx[0], x.data_ptr(), 24, idx.data_ptr(), b.data_ptr(), b.numel(), s), "dispatch")
        check(L.tm_ep_experts(ctx[0], local.w13.data_ptr(), local.s13.data_ptr(), local.w2.data_ptr(),
                              local.s2.data_ptr(), ows.data_ptr(), n, s), "experts")
        check(L.tm_ep_combine(ctx[0], w.data_ptr(), 24, b.data_ptr(), b.numel(), None, out.data_ptr(), s),
              "combine")
        torch.cuda.synchronize()
        st = C.c_uint32(0)
        check(L.tm_ep_status(ctx[0], C.byref(st), s), "tm_ep_status")
        assert st.value & TM_STATUS_TIMEOUT
        # the context is still usable
        y = torch.ones(8, device="cuda") * 2
        assert float(y.sum()) == 16.0
        check(L.tm_ep_status(ctx[0], C.byref(st), s), "tm_ep_status")
        assert st.value == 0
    finally:
        torch.cuda.synchronize()
        for c in ctx:
            L.tm_ep_destroy(c)
