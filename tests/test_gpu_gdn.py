"""Qwen3.5 linear attention decode step (tm_gdn_decode) against the oracle,
the reference-run golden fixtures and Hugging Face's module on the GPU.

Tolerances.  The conv state is a shift of act-dtype values: bit-exact.  The
kernel follows the CUDA rounding of torch.rsqrt (fp32, one rounding), so it
is compared with the oracle run with ``cuda_rsqrt=True`` (the oracle's
default reproduces the CPU ops, which round a short bf16 tensor's rsqrt
twice, and is bit-exact against the CPU-recorded fixtures).  The kernel sums
in another order than PyTorch (warp partials of 8 state rows, then 16
warps), so against that oracle:
* fp32: out max-abs <= 1e-4 x max(1, |out|max), recurrent state max-abs <= 1e-5;
* bf16/fp16: out max-abs <= two act-dtype ulps at the largest output
  (>= 2e-2), cosine >= 0.9999 and >= 99 % of elements bitwise equal (only
  roundings that fall on a tie of the summation order differ); recurrent
  state (fp32) max-abs <= 2e-3 (one act-dtype ulp of a conv output that
  rounds the other way moves state elements by up to ~5e-4) and
  ||dS|| / ||S|| <= 1e-4.
Against the recorded fixtures themselves (bf16: CPU rsqrt roundings) the
layer-output tolerance applies: max-abs 2e-2, cosine 0.9995.  The comparison
with the Hugging Face module run on the GPU is tests/test_zy_linear_attn_dropin.py.
"""
import os

import pytest
import torch

from oracle import gdn_oracle as G

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _check_out(got, want, dt):
    got, want = got.float().cpu(), want.float().cpu()
    d = float((got - want).abs().max())
    if dt == torch.float32:
        assert d <= 1e-4 * max(1.0, float(want.abs().max())), d
        return
    bar = max(2e-2, 2 * float(want.abs().max()) * torch.finfo(dt).eps)
    cos = float(torch.nn.functional.cosine_similarity(got.flatten(), want.flatten(), dim=0))
    eq = float((got == want).float().mean())
    assert d <= bar and cos >= 0.9999 and eq >= 0.99, (d, bar, cos, eq)


def _check_layer(got, want):
    a, b = got.float().cpu().flatten(), want.float().cpu().flatten()
    cos = float(torch.nn.functional.cosine_similarity(a, b, dim=0))
    assert float((a - b).abs().max()) <= 2e-2 and cos >= 0.9995, cos


def _check_state(got, want, dt, bar16=2e-3, rel16=1e-4):
    diff = got.cpu() - want
    d = float(diff.abs().max())
    if dt == torch.float32:
        assert d <= 1e-5, d
        return
    rel = float(diff.norm() / want.norm())
    assert d <= bar16 and rel <= rel16, (d, rel)


def _steps(inputs, conv_w, A_log, dt_bias, norm_w, conv0, S0, n_k_heads, eps=1e-6):
    """Run the kernel and the oracle over the same steps; yields both results
    per step (the kernel ping-pongs two conv-state buffers)."""
    from turbomoe import ops
    dev = torch.device("cuda")
    cw, al, db, nw = (t.to(dev) for t in (conv_w, A_log, dt_bias, norm_w))
    conv_a, conv_b = conv0.to(dev).contiguous(), torch.empty_like(conv0, device=dev)
    S = S0.to(dev).contiguous().clone()
    conv_o, S_o = conv0, S0
    for qkv, z, a, b in inputs:
        out = ops.gdn_decode(qkv.to(dev), z.to(dev), a.to(dev), b.to(dev), cw, al, db, nw, conv_a, conv_b, S,
                             n_k_heads, eps)
        conv_a, conv_b = conv_b, conv_a
        ref, conv_o, S_o = G.gdn_decode(qkv, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_o, S_o, n_k_heads, eps,
                                        cuda_rsqrt=True)
        torch.cuda.synchronize()
        yield out, conv_a, S, ref, conv_o, S_o


@pytest.mark.parametrize("name", ["fp32", "bf16"])
def test_gdn_decode_vs_reference_golden(name):
    """Replay the decode steps recorded from the Hugging Face module with the
    reference's Qwen35Cache: outputs and recurrent state against the oracle
    (CUDA rsqrt rounding) and the recorded outputs, conv states bit-exact."""
    from safetensors import safe_open
    f = safe_open(os.path.join(GOLDEN, f"gdn_{name}.safetensors"), "pt")
    meta = f.metadata()
    t = {k: f.get_tensor(k) for k in f.keys()}
    dt = t["qkv_0"].dtype
    inputs = [tuple(t[f"{k}_{s}"] for k in ("qkv", "z", "a", "b")) for s in range(int(meta["steps"]))]
    run = _steps(inputs, t["conv_w"], t["A_log"], t["dt_bias"], t["norm_w"], t["conv_state_0"],
                 t["recurrent_state_0"], int(meta["n_k_heads"]), float(meta["eps"]))
    for s, (out, conv, S, ref, conv_o, S_o) in enumerate(run):
        _check_out(out, ref, dt)
        _check_layer(out, t[f"core_{s}"])
        if dt == torch.float32:
            _check_out(out, t[f"core_{s}"], dt)
        assert torch.equal(conv.cpu(), t[f"conv_state_{s + 1}"])
        _check_state(S, S_o, dt)
    _check_state(S, t["recurrent_state_final"], dt, bar16=5e-3, rel16=1e-3)


def _random_case(dt, B, Hk, Hv, K, steps, seed):
    g = torch.Generator().manual_seed(seed)
    C = 2 * Hk * 128 + Hv * 128
    conv_w = (torch.randn(C, K, generator=g) * 0.5).to(dt)
    A_log = torch.log(torch.rand(Hv, generator=g) * 16 + 1e-3)
    dt_bias = torch.randn(Hv, generator=g) * 0.5
    norm_w = (1 + 0.1 * torch.randn(128, generator=g)).to(dt)
    conv0 = torch.randn(B, C, K, generator=g).to(dt)
    S0 = torch.randn(B, Hv, 128, 128, generator=g) * 0.05
    inputs = [(torch.randn(B, C, generator=g).to(dt), torch.randn(B, Hv * 128, generator=g).to(dt),
               torch.randn(B, Hv, generator=g).to(dt), torch.randn(B, Hv, generator=g).to(dt))
              for _ in range(steps)]
    return inputs, conv_w, A_log, dt_bias, norm_w, conv0, S0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_gdn_decode_qwen35_shape_vs_oracle(dt):
    """Qwen3.5's linear-attention shape (16 key heads, 32 value heads, conv
    kernel 4), three sequences, four steps on an evolving state."""
    inputs, *rest = _random_case(dt, B=3, Hk=16, Hv=32, K=4, steps=4, seed=11)
    for out, conv, S, ref, conv_o, S_o in _steps(inputs, *rest, n_k_heads=16):
        _check_out(out, ref, dt)
        assert torch.equal(conv.cpu(), conv_o)
        _check_state(S, S_o, dt)


@pytest.mark.parametrize("B,Hk,Hv,K", [(1, 2, 2, 4), (2, 1, 4, 2), (5, 4, 8, 3), (1, 1, 1, 1)])
def test_gdn_decode_shapes_vs_oracle(B, Hk, Hv, K):
    """Value heads per key head 1/2/4/1, conv kernels 1-4, batch 1-5 (bf16)."""
    dt = torch.bfloat16
    inputs, *rest = _random_case(dt, B=B, Hk=Hk, Hv=Hv, K=K, steps=2, seed=100 + B * Hv + K)
    for out, conv, S, ref, conv_o, S_o in _steps(inputs, *rest, n_k_heads=Hk):
        _check_out(out, ref, dt)
        assert torch.equal(conv.cpu(), conv_o)
        _check_state(S, S_o, dt)
