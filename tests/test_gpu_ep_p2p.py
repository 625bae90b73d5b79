"""Expert parallelism over peer memory (tm_ep_*) on one GPU.

* One rank owning every expert: dispatch to itself, the owner's grouped GEMMs
  over the received rows, the return and the combine give the same output
  as the single-GPU layer call (bit-exact where both run the tcgen05 GEMMs,
  >= 16 tokens; the oracle's tolerance below that), across calls of different
  token counts and across CUDA-graph replays (device-side epoch).
* A rank whose peer never sends: every bounded wait runs out, the context's
  status reports TM_STATUS_TIMEOUT, and the CUDA context stays usable.
* An owner that gives up on a call tells every source (TM_STATUS_PEER_FAILED).
"""
import ctypes as C

import pytest
import torch

from gpu_util import k7_layer, oracle_fp32
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
            assert ep.status() == 0
            if T >= ops.PREFILL_MIN_TOKENS:   # the owner's kernels (K7) on one GPU: the same bits
                ref = k7_layer(x, idx, w, full, ws, residual=res)
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


def test_ep_p2p_owner_failure_reaches_every_source():
    """Three contexts on one GPU (ranks 0-2 of one expert-parallel group, E 24:
    8 experts each), all kernels on one stream.  Owner 1 runs its expert step
    before source 2 has dispatched, so its bounded wait (20 ms) runs out and it
    processes nothing.  Owners 0 and 2 run after every dispatch and succeed.
    Sources 0 and 2 then see owner 1's return flag for this call: it must tell
    them that owner 1 failed (TM_STATUS_PEER_FAILED), otherwise they would sum
    the stale rows of owner 1's return region with a clean status."""
    from turbomoe import ops, synth
    from turbomoe._lib import (TM_EP_HANDLE_BYTES, TM_STATUS_PEER_FAILED, TM_STATUS_TIMEOUT, check, lib)
    L = lib()
    E3, G = 24, 3
    shape = synth.MoEShape(H, I, E3, K, 0)
    lw = synth.make_layer(shape, 79, 0)
    router = lw.router.cuda()
    code = ops._code(router.dtype)
    T = 24
    ctx = [C.c_void_p() for _ in range(G)]
    for r in range(G):
        h = (C.c_char * TM_EP_HANDLE_BYTES)()
        check(L.tm_ep_create(r, G, E3, K, H, I, code, T, h, C.byref(ctx[r])), "tm_ep_create")
    try:
        bases = [L.tm_ep_local_buffer(c) for c in ctx]
        for r in range(G):
            check(L.tm_ep_connect_ptrs(ctx[r], (C.c_void_p * G)(*bases)), "tm_ep_connect_ptrs")
            check(L.tm_ep_set_timeout(ctx[r], 20_000_000 if r == 1 else 500_000_000), "tm_ep_set_timeout")
        d = lambda t: t.cuda()
        s = torch.cuda.current_stream().cuda_stream
        per = E3 // G
        local, ows, wss, xs, ws_, outs = [], [], [], [], [], []
        for r in range(G):
            sl = slice(r * per, (r + 1) * per)
            local.append(ops.pack_experts(d(lw.gate[sl]), d(lw.gate_s[sl]), d(lw.up[sl]), d(lw.up_s[sl]),
                                          d(lw.down[sl]), d(lw.down_s[sl])))
            n = L.tm_ep_owner_workspace_bytes(ctx[r])
            ows.append(torch.empty(n, dtype=torch.uint8, device="cuda"))
            check(L.tm_workspace_init(ows[r].data_ptr(), n, s), "tm_workspace_init")
            wss.append(ops.Workspace("cuda", E3, K, H, I, 0))
            xs.append(synth.make_hidden(T, H, 30 + r, device="cuda"))
            ws_.append(ops.router_topk(xs[r], router, K, wss[r]))
            outs.append(torch.empty_like(xs[r]))

        def dispatch(r):
            b = wss[r].buf
            check(L.tm_ep_dispatch(ctx[r], xs[r].data_ptr(), T, ws_[r][0].data_ptr(), b.data_ptr(), b.numel(), s),
                  "dispatch")

        def experts(r):
            le = local[r]
            check(L.tm_ep_experts(ctx[r], le.w13.data_ptr(), le.s13.data_ptr(), le.w2.data_ptr(),
                                  le.s2.data_ptr(), ows[r].data_ptr(), ows[r].numel(), s), "experts")

        def combine(r):
            b = wss[r].buf
            check(L.tm_ep_combine(ctx[r], ws_[r][1].data_ptr(), T, b.data_ptr(), b.numel(), None,
                                  outs[r].data_ptr(), s), "combine")

        dispatch(0)
        dispatch(1)
        experts(1)          # source 2 has not dispatched yet: owner 1 gives up
        dispatch(2)
        experts(0)
        experts(2)
        for r in range(G):
            combine(r)
        torch.cuda.synchronize()
        st = []
        for r in range(G):
            v = C.c_uint32(0)
            check(L.tm_ep_status(ctx[r], C.byref(v), s), "tm_ep_status")
            st.append(int(v.value))
        assert st[1] & TM_STATUS_TIMEOUT, st            # the owner that gave up
        for r in (0, 2):                                 # healthy ranks learn of it
            assert st[r] & TM_STATUS_PEER_FAILED, st
            assert not st[r] & TM_STATUS_TIMEOUT, st     # their own waits were satisfied
        y = torch.ones(8, device="cuda") * 2              # the CUDA context stays usable
        assert float(y.sum()) == 16.0
    finally:
        torch.cuda.synchronize()
        for c in ctx:
            L.tm_ep_disconnect(c)
        for c in ctx:
            L.tm_ep_destroy(c)
