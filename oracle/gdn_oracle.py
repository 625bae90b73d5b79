"""ORACLE -- test infrastructure only, never part of the product path.

CPU restatement of one decode step of Qwen3.5 linear attention (the gated
delta rule) as the reference runs it.  The reference's Qwen3.5 layers of type
"linear_attention" call Hugging Face's ``Qwen3_5MoeGatedDeltaNet`` with the
reference's ``Qwen35Cache`` (execution/layer_executor.py:134-139,
cache/qwen35_cache.py:43-64).  The arithmetic lives in that third-party
module: transformers 5.5.0, ``models/qwen3_5_moe/modeling_qwen3_5_moe.py``,
whose torch fallbacks run on this image (the fused flash-linear-attention and
causal-conv1d kernels are not installed):

* ``conv_update``     <- ``torch_causal_conv1d_update`` :211-226
* ``l2norm``          <- ``l2norm`` :229-232
* ``gates``           <- ``Qwen3_5MoeGatedDeltaNet.forward`` :504-507
* ``delta_rule_step`` <- ``torch_recurrent_gated_delta_rule`` :315-354 (one token)
* ``gated_rmsnorm``   <- ``Qwen3_5MoeRMSNormGated.forward`` :182-191
* ``gdn_decode``      <- ``Qwen3_5MoeGatedDeltaNet.forward`` :423-533 from the
  in-projection outputs to the out_proj input, ``use_precomputed_states``

Each function uses the same PyTorch CPU ops in the same dtypes as the lines
it cites.  Only ``tests/`` and the smoke entry point import this module.

One op rounds differently on the CPU than on CUDA, where the reference runs
its layers: ``torch.rsqrt`` of a bf16/fp16 tensor.  ATen's CUDA kernel
evaluates rsqrt in fp32 and rounds once; the CPU's scalar loop (tensors
shorter than a vector, such as the per-head sums of squares of a small batch)
rounds the square root and then its reciprocal, so 6.375 gives 0.39453125
instead of 0.396484375.  ``cuda_rsqrt=True`` evaluates ``l2norm``'s rsqrt the
CUDA way (fp32, one rounding); the default reproduces the CPU ops literally,
which is what the recorded fixtures hold.

Parity is pinned: ``tests/golden/make_gdn_golden.py`` runs the Hugging Face
module with the reference's ``Qwen35Cache`` (a prefill, then decode steps)
and records its inputs, states and outputs; ``tests/test_oracle_golden.py``
checks this module against them.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

HEAD_DIM = 128


def conv_update(x: torch.Tensor, conv_state: torch.Tensor, conv_w: torch.Tensor):
    """x [B, C] (this token's in_proj_qkv row), conv_state [B, C, K],
    conv_w [C, K] -> (SiLU(conv) [B, C] in x's dtype, new state [B, C, K])."""
    window = torch.cat([conv_state, x[:, :, None]], dim=-1).to(conv_w.dtype)
    new_state = window[:, :, -conv_state.shape[-1]:].clone()
    y = F.conv1d(window, conv_w.unsqueeze(1), None, padding=0, groups=window.shape[1])
    return F.silu(y[:, :, -1:]).to(x.dtype)[:, :, 0], new_state


def l2norm(x: torch.Tensor, eps: float = 1e-6, cuda_rsqrt: bool = False) -> torch.Tensor:
    s = (x * x).sum(dim=-1, keepdim=True) + eps
    inv = torch.rsqrt(s.float()).to(s.dtype) if cuda_rsqrt else torch.rsqrt(s)
    return x * inv


def gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """a, b [B, Hv] act -> beta [B, Hv] act, g [B, Hv] fp32."""
    beta = b.sigmoid()
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias)
    return beta, g


def delta_rule_step(q, k, v, g, beta, state, cuda_rsqrt: bool = False):
    """One token of the recurrence.  q, k [B, Hv, Dk] and v [B, Hv, Dv] in the
    act dtype (q/k not yet normalised), g fp32 [B, Hv], beta act [B, Hv],
    state fp32 [B, Hv, Dk, Dv] -> (o act [B, Hv, Dv], new fp32 state)."""
    act = q.dtype
    q = l2norm(q, cuda_rsqrt=cuda_rsqrt)
    k = l2norm(k, cuda_rsqrt=cuda_rsqrt)
    q, k, v, beta, g = (t.to(torch.float32) for t in (q, k, v, beta, g))
    q = q * (1 / (q.shape[-1] ** 0.5))
    S = state.to(torch.float32) * g.exp()[..., None, None]
    kv_mem = (S * k[..., :, None]).sum(dim=-2)
    delta = (v - kv_mem) * beta[..., None]
    S = S + k[..., :, None] * delta[..., None, :]
    o = (S * q[..., :, None]).sum(dim=-2)
    return o.to(act), S


def gated_rmsnorm(o: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """o, z [..., Dv] act; RMSNorm before the SiLU gate."""
    dt = o.dtype
    h = o.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    h = weight * h.to(dt)
    h = h * F.silu(z.to(torch.float32))
    return h.to(dt)


def gdn_decode(qkv, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, recurrent_state, n_k_heads: int,
               eps: float = 1e-6, cuda_rsqrt: bool = False):
    """One decode token per batch row, from the in-projection outputs
    (qkv [B, C], z [B, Hv*128], a/b [B, Hv]) to the out_proj input.
    Returns (out [B, Hv*128] act, new conv state [B, C, K], new fp32
    recurrent state [B, Hv, 128, 128]); the inputs are not modified.
    ``cuda_rsqrt``: the l2norm's rsqrt rounded as on CUDA (module docstring)."""
    B = qkv.shape[0]
    Hv = a.shape[-1]
    key_dim = n_k_heads * HEAD_DIM
    y, new_conv = conv_update(qkv, conv_state, conv_w)
    q, k, v = torch.split(y, [key_dim, key_dim, Hv * HEAD_DIM], dim=-1)
    q = q.reshape(B, n_k_heads, HEAD_DIM)
    k = k.reshape(B, n_k_heads, HEAD_DIM)
    v = v.reshape(B, Hv, HEAD_DIM)
    beta, g = gates(a, b, A_log, dt_bias)
    if Hv // n_k_heads > 1:
        q = q.repeat_interleave(Hv // n_k_heads, dim=1)
        k = k.repeat_interleave(Hv // n_k_heads, dim=1)
    o, S = delta_rule_step(q, k, v, g, beta, recurrent_state, cuda_rsqrt)
    out = gated_rmsnorm(o.reshape(-1, HEAD_DIM), z.reshape(-1, HEAD_DIM), norm_w, eps)
    return out.reshape(B, Hv * HEAD_DIM), new_conv, S
