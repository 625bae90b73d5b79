"""Record decode steps of Qwen3.5 linear attention as the reference runs them.

    python tests/golden/make_gdn_golden.py <path to the reference checkout> [--dtype fp32|bf16|fp16]

The reference's Qwen3.5 "linear_attention" layers call Hugging Face's
``Qwen3_5MoeGatedDeltaNet`` with the reference's ``Qwen35Cache``
(execution/layer_executor.py:134-139, cache/qwen35_cache.py).  This script
builds that module (transformers, torch fallbacks: the fused libraries are
not installed) on the CPU with seeded weights, runs a prompt of ``PREFILL``
tokens through it with a ``Qwen35Cache`` imported from the reference
checkout (the chunked path fills the conv and recurrent states), then
``STEPS`` single-token decode steps (the ``use_precomputed_states`` path).
Writes ``tests/golden/gdn_<dtype>.safetensors`` with, per decode step, the
module's in-projection outputs (qkv, z, a, b: the inputs of the kernel), the
out_proj input (the kernel's output, captured by a forward pre-hook) and the
conv state after the step; the recurrent state before the first and after
the last step; the module's conv weight, A_log, dt_bias and norm weight.

Shape: batch 2, hidden 256, 1 key head and 2 value heads of 128 (two value
heads share a key head), conv kernel 4.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
BATCH, HIDDEN, HK, HV, KCONV, PREFILL, STEPS, SEED = 2, 256, 1, 2, 4, 5, 3, 7


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("reference", help="path to the reference checkout")
    ap.add_argument("--dtype", choices=["fp32", "bf16", "fp16"], default="fp32")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from cache.qwen35_cache import Qwen35Cache
    from safetensors.torch import save_file
    from transformers import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M

    assert not M.is_fast_path_available, "the fused linear-attention libraries changed the path"
    dt = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[args.dtype]
    cfg = Qwen3_5MoeTextConfig(hidden_size=HIDDEN, linear_num_key_heads=HK, linear_num_value_heads=HV,
                               linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=KCONV,
                               rms_norm_eps=1e-6)
    torch.manual_seed(SEED)
    mod = M.Qwen3_5MoeGatedDeltaNet(cfg, layer_idx=0)
    with torch.no_grad():
        mod.norm.weight.copy_(1.0 + 0.1 * torch.randn(128))
        mod.dt_bias.copy_(0.5 * torch.randn(HV))
    mod = mod.to(dt).eval()

    cache = Qwen35Cache(num_layers=1)
    g = torch.Generator().manual_seed(SEED + 1)
    rec = {}
    captured = []
    mod.out_proj.register_forward_pre_hook(lambda m, inp: captured.append(inp[0].detach().clone()))
    with torch.no_grad():
        x0 = torch.randn(BATCH, PREFILL, HIDDEN, generator=g).to(dt)
        mod(x0, cache_params=cache)
        assert cache.has_previous_state(0)
        rec["conv_state_0"] = cache.layers[0].conv_states.clone()
        rec["recurrent_state_0"] = cache.layers[0].recurrent_states.clone()
        for s in range(STEPS):
            x = torch.randn(BATCH, 1, HIDDEN, generator=g).to(dt)
            rec[f"qkv_{s}"] = mod.in_proj_qkv(x)[:, 0].clone()
            rec[f"z_{s}"] = mod.in_proj_z(x)[:, 0].clone()
            rec[f"a_{s}"] = mod.in_proj_a(x)[:, 0].clone()
            rec[f"b_{s}"] = mod.in_proj_b(x)[:, 0].clone()
            captured.clear()
            y = mod(x, cache_params=cache)
            rec[f"core_{s}"] = captured[0].reshape(BATCH, HV * 128).clone()
            rec[f"out_{s}"] = y[:, 0].clone()
            rec[f"conv_state_{s + 1}"] = cache.layers[0].conv_states.clone()
        rec["recurrent_state_final"] = cache.layers[0].recurrent_states.clone()
    rec["conv_w"] = mod.conv1d.weight.detach()[:, 0].clone()
    rec["A_log"] = mod.A_log.detach().clone()
    rec["dt_bias"] = mod.dt_bias.detach().clone()
    rec["norm_w"] = mod.norm.weight.detach().clone()
    rec = {k: v.contiguous() for k, v in rec.items()}
    meta = {"batch": str(BATCH), "n_k_heads": str(HK), "n_v_heads": str(HV), "conv_kernel": str(KCONV),
            "steps": str(STEPS), "prefill": str(PREFILL), "eps": str(cfg.rms_norm_eps), "dtype": args.dtype,
            "torch": torch.__version__, "transformers": __import__("transformers").__version__}
    path = os.path.join(HERE, f"gdn_{args.dtype}.safetensors")
    save_file(rec, path, metadata=meta)
    print("wrote", path, {k: tuple(v.shape) for k, v in rec.items() if k.endswith("_0")})


if __name__ == "__main__":
    main()
