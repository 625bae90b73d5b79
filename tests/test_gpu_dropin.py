"""The drop-in classes (RouterExecutor, MoEExecutor, ExpertLoader) used the way
the reference engine uses them (runtime/engine.py:14-21,
execution/layer_executor.py:157-213), on an on-disk synthetic FP8 checkpoint."""
import pytest
import torch

from gpu_util import assert_close, fp32_cos
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from turbomoe import synth
    shape = synth.MoEShape(512, 256, 32, 8, 256)
    path = str(tmp_path_factory.mktemp("ckpt"))
    synth.write_checkpoint(path, shape, seed=77, layers=2)
    return path, shape


def _stack(ckpt_path, dtype):
    from execution.moe import MoEExecutor
    from execution.router import RouterExecutor
    from loader.expert_loader import ExpertLoader
    L = ExpertLoader(ckpt_path, config={"execution": {"dtype": dtype}})
    R = RouterExecutor(L, 2)
    M = MoEExecutor(L)
    return L, R, M


@pytest.mark.parametrize("dtype,T", [("bf16", 1), ("bf16", 17), ("fp32", 5), ("fp16", 1)])
def test_layer_executor_flow(ckpt, dtype, T):
    from turbomoe import synth
    path, shape = ckpt
    L, R, M = _stack(path, dtype)
    dt = L.dtype
    for layer in (0, 1):
        lw = synth.make_layer(shape, 77, layer)
        x = synth.make_hidden(T, shape.hidden, layer, dtype=torch.bfloat16).to(dt)
        idx, w = R.compute_routing(layer, x.cuda().view(1, T, -1))      # 3-D like post_norm output
        assert idx.dtype == torch.int64 and w.dtype == dt and idx.shape == (T, 8)
        y = M.execute_layer(layer, x.cuda(), idx, w)
        assert y.shape == x.shape and y.dtype == dt
        assert M.last_gemm_ms > 0.0
        ref = O.execute_layer(O.OracleLayer(lw, torch.float32), x.float(), idx.cpu(), w.float().cpu())
        tol = {"fp32": 1e-4, "fp16": 2e-3, "bf16": 1e-2}[dtype]
        assert_close(y, ref, tol, fp32_cos(T, dt), f"{dtype} T={T} layer {layer}")


def test_loader_interface(ckpt):
    from turbomoe import synth
    path, shape = ckpt
    L, R, M = _stack(path, "bf16")
    lw = synth.make_layer(shape, 77, 1)
    g, u, d = L.load_expert(1, 5)
    assert torch.equal(g.cpu(), O.dequantize_weight(lw.gate[5], lw.gate_s[5], torch.bfloat16))
    assert torch.equal(d.cpu(), O.dequantize_weight(lw.down[5], lw.down_s[5], torch.bfloat16))
    assert L.gpu_hits >= 1 and L.expert_metadata[L.expert_cache[(1, 5)]]["hits"] >= 1
    w, s = L.load_weight_raw("model.layers.1.mlp.experts.5.up_proj.weight")
    assert torch.equal(L.dequantize_weight(w, s, torch.float32).cpu(), O.dequant_fp32_exact(lw.up[5], lw.up_s[5]))
    full = L.load_weight("model.layers.1.mlp.experts.5.up_proj.weight")
    assert torch.equal(full.cpu(), O.dequantize_weight(lw.up[5], lw.up_s[5], torch.bfloat16))
    out, c_ms, d_ms = L.load_weight_split("model.layers.1.mlp.experts.5.up_proj.weight")
    assert torch.equal(out, full) and c_ms >= 0 and d_ms >= 0
    # prefill-time fetch (load_expert_dynamic): fresh tensors, the reference's dequantisation
    hits = L.gpu_hits
    dg, du, dd = L.load_expert_dynamic(0, 7)
    lw0 = synth.make_layer(shape, 77, 0)
    for got, q, s_ in ((dg, lw0.gate[7], lw0.gate_s[7]), (du, lw0.up[7], lw0.up_s[7]),
                       (dd, lw0.down[7], lw0.down_s[7])):
        assert got.is_cuda and got.dtype == torch.bfloat16
        assert torch.equal(got.cpu(), O.dequantize_weight(q, s_, torch.bfloat16))
    assert L.gpu_hits == hits + 1
    dg.zero_()                        # not a view of anything the next call returns
    dg2, _, _ = L.load_expert_dynamic(0, 7)
    assert torch.equal(dg2.cpu(), O.dequantize_weight(lw0.gate[7], lw0.gate_s[7], torch.bfloat16))
    # raw FP8 + scales of one expert (load_expert_raw)
    raw = L.load_expert_raw(0, 7)
    assert len(raw) == 6
    assert torch.equal(raw[0].cpu().view(torch.uint8), lw0.gate[7].view(torch.uint8))
    assert torch.equal(raw[5].cpu(), lw0.down_s[7].float())
    for a in ("DEVICE", "dtype", "layout", "weight_map", "expert_cache", "expert_metadata", "cache_limit",
              "num_slots", "ram_cache", "gpu_hits", "ram_hits", "ssd_hits", "load_ms_accum",
              "dequant_ms_accum", "evict_ms_accum", "lock"):
        assert hasattr(L, a), a
    L.clear_pinned_slots()
    L.upload()                        # one-time upload of every layer
    L.adjust_cache_limit()
    assert L.cache_limit == 2 * 32 and len(L.expert_cache) == 2 * 32
    L.close()


def test_foreign_indices_get_a_plan(ckpt):
    """execute_layer with indices that did not come from compute_routing."""
    from turbomoe import synth
    path, shape = ckpt
    L, R, M = _stack(path, "fp32")
    lw = synth.make_layer(shape, 77, 0)
    T = 6
    x = synth.make_hidden(T, shape.hidden, 9, dtype=torch.float32)
    idx_a, w_a = R.compute_routing(0, x.cuda())
    idx = torch.stack([torch.randperm(32)[:8] for _ in range(T)]).cuda()
    w = torch.softmax(torch.randn(T, 8), -1).cuda()
    y = M.execute_layer(0, x.cuda(), idx, w)
    ref = O.execute_layer(O.OracleLayer(lw, torch.float32), x, idx.cpu(), w.cpu())
    assert_close(y, ref, 1e-4, 0.999999, "foreign idx")
    # and the router's own indices still work afterwards (plan rebuilt)
    y_a = M.execute_layer(0, x.cuda(), idx_a, w_a)
    ref_a = O.execute_layer(O.OracleLayer(lw, torch.float32), x, idx_a.cpu(), w_a.cpu())
    assert_close(y_a, ref_a, 1e-4, 0.999999, "router idx after foreign idx")


def test_cpu_tensors_raise(ckpt):
    from turbomoe._lib import TurboMoEError
    path, shape = ckpt
    L, R, M = _stack(path, "bf16")
    with pytest.raises(TurboMoEError):
        R.compute_routing(0, torch.zeros(1, shape.hidden, dtype=torch.bfloat16))
