"""Dense FP8 block-scaled linear (tm_fp8_linear) against the oracle.

The kernel multiplies the exact dequantised weights (e4m3 x fp32 block
scale) with the activations (exact in f16 after a power-of-2 shift), fp32
accumulation, one rounding to the act dtype: against an fp32 evaluation of
the same product it must agree to one act-dtype rounding (max-abs within one
ulp of the largest output, at least 1e-2; cosine >= 0.99999).  The reference's own path
(load_weight dequantises W to the act dtype, then F.linear in that dtype,
loader/expert_loader.py:109-112) rounds W first; against it the layer-output
tolerance applies (cosine >= 0.9995).
"""
import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_close
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def _one_rounding(want, dt):
    """Max-abs bar for one rounding to dt: one ulp at the largest output (>= 1e-2)."""
    return max(1e-2, float(want.abs().max()) * torch.finfo(dt).eps)


def _weight(N, K, seed):
    from turbomoe import synth
    g = torch.Generator().manual_seed(seed)
    return synth.quantize_fp8_block(torch.randn(N, K, generator=g) * 0.02)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [1, 3, 8, 9, 40])
def test_fp8_linear_matches_oracle(dt, T):
    from turbomoe import ops, synth
    N, K = 640, 1024
    w, s = _weight(N, K, 10 + T)
    pl = ops.pack_linear(w.cuda(), s.cuda())
    x = synth.make_hidden(T, K, 3 + T, dtype=dt)
    out = ops.fp8_linear(x.cuda(), pl).cpu()
    want32 = F.linear(x.float(), O.dequantize_weight(w, s, torch.float32))
    assert_close(out.float(), want32, _one_rounding(want32, dt), 0.99999, f"fp8_linear {dt} T={T} vs fp32")
    ref = F.linear(x, O.dequantize_weight(w, s, dt)).float()     # the reference's arithmetic
    assert_close(out.float(), ref, 2e-2, 0.9995, f"fp8_linear {dt} T={T} vs reference path")


def test_fp8_linear_residual():
    from turbomoe import ops, synth
    N, K, T = 256, 512, 9
    w, s = _weight(N, K, 77)
    pl = ops.pack_linear(w.cuda(), s.cuda())
    x = synth.make_hidden(T, K, 8, dtype=torch.float16)
    res = torch.randn(T, N, generator=torch.Generator().manual_seed(1)).to(torch.float16)
    out = ops.fp8_linear(x.cuda(), pl, residual=res.cuda()).cpu()
    want32 = F.linear(x.float(), O.dequantize_weight(w, s, torch.float32)) + res.float()
    assert_close(out.float(), want32, 5e-3, 0.99999, "fp8_linear + residual")


@pytest.mark.parametrize("N,K", [(4096, 2048), (512, 2048), (2048, 4096)])
def test_fp8_linear_attention_shapes(N, K):
    """The q/k/v/o projection shapes of a Qwen3-30B-A3B layer, one decode token."""
    from turbomoe import ops, synth
    w, s = _weight(N, K, N + K)
    pl = ops.pack_linear(w.cuda(), s.cuda())
    x = synth.make_hidden(1, K, 5, rms_normalise=True)
    out = ops.fp8_linear(x.cuda(), pl).cpu()
    want32 = F.linear(x.float(), O.dequantize_weight(w, s, torch.float32))
    assert_close(out.float(), want32, _one_rounding(want32, torch.bfloat16), 0.99999, f"fp8_linear {N}x{K}")


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N,K", [(5120, 2048), (128, 4096), (256, 6144)])
def test_fp8_linear_one_token_fp8_path(dt, N, K):
    """One-token calls with K % 2048 == 0 run on FP8 MMAs with the token split
    into three e4m3 terms (k6_linear_t1_f8): within one act-dtype rounding of
    the fp32 product, with and without the residual; the fused q/k/v shape
    and K = 6144 (24 MMA steps per warp)."""
    from turbomoe import ops, synth
    w, s = _weight(N, K, 3 * N + K)
    pl = ops.pack_linear(w.cuda(), s.cuda())
    x = synth.make_hidden(1, K, N, dtype=dt)
    res = torch.randn(1, N, generator=torch.Generator().manual_seed(N)).to(dt)
    want32 = F.linear(x.float(), O.dequantize_weight(w, s, torch.float32))
    out = ops.fp8_linear(x.cuda(), pl).cpu()
    assert_close(out.float(), want32, _one_rounding(want32, dt), 0.99999, f"fp8_linear t1 {dt} {N}x{K}")
    out_r = ops.fp8_linear(x.cuda(), pl, residual=res.cuda()).cpu()
    want_r = want32 + res.float()
    assert_close(out_r.float(), want_r, _one_rounding(want_r, dt), 0.99999, f"fp8_linear t1 + residual {dt}")
