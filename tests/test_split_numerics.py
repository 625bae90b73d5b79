"""Precision of the three-term e4m3 activation used by the one-token FP8
decode kernels (k2_gateup_f8, k3_down_t1_f8; `e4m3_split3` and `e4m3_shift` in
turbo-llm_b200/csrc/tm_common.cuh).

The kernels scale a token's values by a power of 2 so that the largest
magnitude lies in [128, 256), then write each value v as three e4m3 terms,
each rounded to nearest: hi = e4m3(v), mid = e4m3(16 (v - hi)),
lo = e4m3(16 (16 (v - hi) - mid)), and multiply the weights by
hi + mid/16 + lo/256 (one MMA column per term).  This restates that
arithmetic with torch's round-to-nearest float8_e4m3fn conversion and checks,
over every bf16 / fp16 value in range:

* bf16 values with |v| >= 2^-10 and fp16 values with |v| >= 2^-7 are
  represented exactly (so every value within 2^-18 / 2^-15 of the token's
  largest enters the MMA unchanged);
* smaller values are off by at most 2^-18 in absolute terms, under 2^-25 of
  the token's largest magnitude.
CPU only: the GPU parity tests check the kernels end to end.
"""
import pytest
import torch


def _e4m3(t):
    return t.to(torch.float8_e4m3fn).float()


def _three_terms(v):
    hi = _e4m3(v)
    r1 = (v - hi) * 16
    mid = _e4m3(r1)
    r2 = (r1 - mid) * 16
    lo = _e4m3(r2)
    return hi + mid / 16 + lo / 256


def _all_values(dtype, top_bits):
    bits = torch.arange(0, top_bits, dtype=torch.int32).to(torch.int16)
    x = bits.view(dtype).float()
    x = x[(x > 0) & (x < 256)]
    return torch.cat([x, -x])


@pytest.mark.parametrize("dtype,top_bits,exact_from", [(torch.bfloat16, 0x7F80, 2.0 ** -10),
                                                       (torch.float16, 0x7C00, 2.0 ** -7)])
def test_three_term_e4m3_split(dtype, top_bits, exact_from):
    v = _all_values(dtype, top_bits)
    err = (_three_terms(v) - v).abs()
    big = v.abs() >= exact_from
    assert bool((err[big] == 0).all())
    assert err.max().item() <= 2.0 ** -18
    # relative to the largest scaled magnitude (at least 128)
    assert err.max().item() / 128 <= 2.0 ** -25


def test_scale_maps_largest_into_128_256():
    """e4m3_shift: s = clamp(8 - e, -100, 100) with max = f * 2^e, f in
    [0.5, 1); the clamp only binds for magnitudes below 2^-92 or above 2^108."""
    for m in [2.0 ** -90, 3.1e-5, 0.7, 1.0, 127.9, 128.0, 300.0, 6.5e4, 3.0e38]:
        _, e = torch.frexp(torch.tensor(m, dtype=torch.float32))
        s = max(-100, min(100, 8 - int(e)))
        scaled = m * 2.0 ** s
        assert 128 <= scaled < 256 or abs(s) == 100
