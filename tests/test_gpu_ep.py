"""Expert-parallel MoE layer on 2 GPUs (NCCL, one process per GPU) with this
library's kernels: every rank's output matches the whole layer computed on
one GPU for its tokens (bf16: max-abs 2e-2, cosine 0.9999 - the two sides may
run different expert kernels: an owner that receives >= 256 rows uses the
tcgen05 grouped GEMMs).  Skipped with fewer than 2 GPUs."""
import datetime
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, q):
    try:
        import sys, os
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "turbo-llm_b200"))
        from turbomoe import ops, synth
        from turbomoe.ep import ExpertParallelMoE, cuda_functions
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        H, I, E, k = 512, 256, 16, 4
        shape = synth.MoEShape(H, I, E, k, 0)
        lw = synth.make_layer(shape, 55, 0)
        dev = torch.device("cuda", rank)
        d = lambda t: t.to(dev)
        E_loc = E // world
        sl = slice(rank * E_loc, (rank + 1) * E_loc)
        local = ops.pack_experts(d(lw.gate[sl]), d(lw.gate_s[sl]), d(lw.up[sl]), d(lw.up_s[sl]),
                                 d(lw.down[sl]), d(lw.down_s[sl]))
        full = ops.pack_experts(d(lw.gate), d(lw.gate_s), d(lw.up), d(lw.up_s), d(lw.down), d(lw.down_s))
        router = d(lw.router)
        x = synth.make_hidden(T + 7 * rank, H, 300 + rank, device=dev)
        res = torch.randn(x.shape, generator=torch.Generator(device=dev).manual_seed(rank), device=dev).to(x.dtype)
        ep = ExpertParallelMoE(E, k, *cuda_functions(router, local, k, E, H, I))
        out = ep.forward(x, residual=res)
        ws = ops.Workspace(dev, E, k, H, I, 0)
        idx, w = ops.router_topk(x, router, k, ws)
        ref = ops.moe_experts(x, idx, w, full, ws, residual=res)
        a, b = out.float().cpu().double().flatten(), ref.float().cpu().double().flatten()
        q.put((rank, (a - b).abs().max().item(), torch.nn.functional.cosine_similarity(a, b, dim=0).item(),
               ep.last_counts))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("T", [40, 300])
def test_ep_two_gpus_matches_single_gpu(T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, maxabs, cos, counts in results:
        assert not isinstance(maxabs, str), maxabs
        assert maxabs <= 2e-2 and cos >= 0.9999, (rank, maxabs, cos, counts)


def _worker_p2p(rank, world, port, T, q):
    """Peer-memory path (tm_ep_*): eager call, then three replays of a CUDA
    graph of the call; every output equals the single-GPU layer for this
    rank's tokens (bit-exact: both sides run the tcgen05 GEMMs row by row)."""
    try:
        import sys, os
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "turbo-llm_b200"))
        from turbomoe import ops, synth
        from turbomoe.ep import PeerExpertParallelMoE
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        H, I, E, k = 512, 256, 16, 4
        shape = synth.MoEShape(H, I, E, k, 0)
        lw = synth.make_layer(shape, 56, 0)
        dev = torch.device("cuda", rank)
        d = lambda t: t.to(dev)
        E_loc = E // world
        sl = slice(rank * E_loc, (rank + 1) * E_loc)
        local = ops.pack_experts(d(lw.gate[sl]), d(lw.gate_s[sl]), d(lw.up[sl]), d(lw.up_s[sl]),
                                 d(lw.down[sl]), d(lw.down_s[sl]))
        full = ops.pack_experts(d(lw.gate), d(lw.gate_s), d(lw.up), d(lw.up_s), d(lw.down), d(lw.down_s))
        router = d(lw.router)
        Tr = T + 7 * rank
        x = synth.make_hidden(Tr, H, 400 + rank, device=dev)
        res = torch.randn(x.shape, generator=torch.Generator(device=dev).manual_seed(rank), device=dev).to(x.dtype)
        ep = PeerExpertParallelMoE(router, local, k, max_tokens=T + 7 * world)
        out = ep.forward(x, residual=res)
        ws = ops.Workspace(dev, E, k, H, I, 0)
        idx, w = ops.router_topk(x, router, k, ws)
        if Tr >= ops.PREFILL_MIN_TOKENS:   # the owners' kernels (K7) on one GPU: the same bits
            from gpu_util import k7_layer
            ref = k7_layer(x, idx, w, full, ws, residual=res)
        else:
            ref = ops.moe_experts(x, idx, w, full, ws, residual=res)
        a, b = out.float().cpu().double().flatten(), ref.float().cpu().double().flatten()
        worst = [(a - b).abs().max().item(), torch.nn.functional.cosine_similarity(a, b, dim=0).item(),
                 bool(torch.equal(out, ref))]
        # graph replays: the epoch advances on the device
        g_out = torch.empty_like(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep.forward(x, residual=res, out=g_out)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ep.forward(x, residual=res, out=g_out)
        same = True
        for _ in range(3):
            g_out.zero_()
            g.replay()
            torch.cuda.synchronize()
            same &= bool(torch.equal(g_out, out))
        st = ep.status()
        del g
        ep.close()
        q.put((rank, worst, same, st))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("T", [1, 40, 300])
def test_ep_p2p_two_gpus_matches_single_gpu(T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_p2p, args=(r, 2, port, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, worst, same, st in results:
        assert not isinstance(worst, str), worst
        maxabs, cos, exact = worst
        assert st == 0, (rank, st)
        assert same, rank
        if T >= 16:
            assert exact, (rank, maxabs, cos)
        assert maxabs <= 2e-2 and cos >= 0.9999, (rank, maxabs, cos)
