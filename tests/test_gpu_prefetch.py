"""Speculative next-layer L2 prefetch (RouterExecutor(prefetch_next_layer=
True)): a hint only, so the decode chain through the executors must give the
same bits with and without it, eagerly and from a CUDA graph; the prefetch
kernel must accept out-of-range ids (skipped) without touching the output."""
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYERS = 4


def _chain(router, moe, x):
    for l in range(LAYERS):
        idx, w = router.compute_routing(l, x)
        x = moe.execute_layer(l, x, idx, w, residual=x)
    return x


def test_next_layer_prefetch_same_bits():
    from execution.moe import MoEExecutor
    from execution.router import RouterExecutor
    from loader.expert_loader import ExpertLoader
    from turbomoe import synth
    dev = torch.device("cuda", 0)
    shape = synth.QWEN3_30B_A3B
    loader = ExpertLoader.synthetic(shape, seed=99, num_layers=LAYERS, dtype=torch.bfloat16, device=dev)
    loader.upload()
    moe = MoEExecutor(loader, record_timing=False)
    x0 = synth.make_hidden(1, shape.hidden, 5, rms_normalise=True, device=dev)
    plain = RouterExecutor(loader, LAYERS)
    ref = _chain(plain, moe, x0.clone())
    spec = RouterExecutor(loader, LAYERS, prefetch_next_layer=True)
    eager = _chain(spec, moe, x0.clone())
    torch.cuda.synchronize()
    assert torch.equal(eager, ref)
    # captured: the side branch is forked and rejoined inside every layer
    x_in = x0.clone()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _chain(spec, moe, x_in)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = _chain(spec, moe, x_in)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    assert spec.next_layer_prefetch.pending is None
    assert loader.workspace(dev).status() == 0


def test_prefetch_kernel_skips_bad_ids():
    from turbomoe import ops
    dev = torch.device("cuda", 0)
    packed = ops.alloc_packed(4, 256, 128, dev)
    packed.w13.fill_(7)
    ids = torch.tensor([0, 3, -1, 4, 99], dtype=torch.int64, device=dev)
    ops.prefetch_experts_l2(packed, ids)
    torch.cuda.synchronize()
    assert bool((packed.w13 == 7).all())
