"""Seeded synthetic FP8 MoE checkpoints (Qwen3-MoE / Qwen3.5-MoE layout).

No real checkpoint exists on either machine, so every weight this package
runs on is drawn here.  The recipe follows the workload definitions of the
reference's MoE path:

* expert and router weights ~ N(0, 0.02) from a seeded torch generator;
* each expert matrix is quantised per 128x128 block: ``scale = amax / 448``,
  ``q = e4m3(w / scale)``, stored as ``<name>.weight`` (float8_e4m3fn) plus
  ``<name>.weight_scale_inv`` (fp32, ``[M/128, N/128]``) -- the on-disk
  format that ``loader/expert_loader.py:89-114`` and ``:127-160`` read;
* router (``mlp.gate.weight``) is bf16 ``[E, H]``;
* an optional shared expert (Qwen3.5) is FP8 like the routed ones, with a
  bf16 ``mlp.shared_expert_gate.weight`` ``[1, H]``.

Qwen3 checkpoints carry no shared expert, but the reference's
``MoEExecutor`` loads one unconditionally (``execution/moe.py:53-67``), so
``write_checkpoint(..., zero_shared=True)`` adds an all-zero bf16 shared
expert, which is an exact no-op (silu(0)*0 = 0, sigmoid(0)*0 = 0).

Generation is per layer: one generator seeded with ``layer_seed(seed, l)``
draws router, gate, up, down (and the shared expert) in that order, so any
layer can be regenerated alone, on the CPU or on a CUDA device.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import torch

FP8_MAX = 448.0
BLOCK = 128


@dataclass(frozen=True)
class MoEShape:
    hidden: int = 2048          # H
    inter: int = 768            # I (moe_intermediate_size)
    experts: int = 128          # E
    top_k: int = 8
    shared_inter: int = 0       # 0 = no shared expert (Qwen3); 512 for Qwen3.5-style

    def check(self):
        for name, v in (("hidden", self.hidden), ("inter", self.inter)):
            if v % BLOCK:
                raise ValueError(f"{name}={v} must be a multiple of {BLOCK}")
        if self.shared_inter % BLOCK:
            raise ValueError("shared_inter must be a multiple of 128")


QWEN3_30B_A3B = MoEShape(2048, 768, 128, 8, 0)
QWEN35_LAYER = MoEShape(2048, 512, 256, 8, 512)


def layer_seed(seed: int, layer: int) -> int:
    return (int(seed) * 1_000_003 + int(layer) * 7919 + 17) % (2**62)


def quantize_fp8_block(w: torch.Tensor):
    """Per-128x128-block e4m3 quantisation of ``w`` (``[..., M, N]`` fp32).

    Returns ``(q float8_e4m3fn [..., M, N], scale_inv fp32 [..., M/128, N/128])``
    with ``w ~= q.float() * scale_inv`` blockwise.
    """
    *lead, M, N = w.shape
    b = w.reshape(*lead, M // BLOCK, BLOCK, N // BLOCK, BLOCK)
    amax = b.abs().amax(dim=(-3, -1)).float()
    s = amax.clamp_min(1e-12) / FP8_MAX
    q = (b / s.unsqueeze(-1).unsqueeze(-3)).to(torch.float8_e4m3fn)
    return q.reshape(*lead, M, N), s


@dataclass
class LayerWeights:
    """Raw checkpoint tensors of one MoE layer (any device)."""
    router: torch.Tensor                 # [E, H] bf16
    gate: torch.Tensor                   # [E, I, H] float8_e4m3fn
    gate_s: torch.Tensor                 # [E, I/128, H/128] fp32
    up: torch.Tensor
    up_s: torch.Tensor
    down: torch.Tensor                   # [E, H, I] float8_e4m3fn
    down_s: torch.Tensor                 # [E, H/128, I/128] fp32
    sh_gate: torch.Tensor | None = None  # [Is, H] fp8
    sh_gate_s: torch.Tensor | None = None
    sh_up: torch.Tensor | None = None
    sh_up_s: torch.Tensor | None = None
    sh_down: torch.Tensor | None = None  # [H, Is] fp8
    sh_down_s: torch.Tensor | None = None
    sh_router: torch.Tensor | None = None  # [1, H] bf16 (shared_expert_gate)


def make_layer(shape: MoEShape, seed: int, layer: int, device="cpu", std=0.02) -> LayerWeights:
    shape.check()
    H, I, E = shape.hidden, shape.inter, shape.experts
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(layer_seed(seed, layer))

    def rnd(*s):
        return torch.randn(*s, generator=g, device=dev, dtype=torch.float32) * std

    router = rnd(E, H).to(torch.bfloat16)
    gate, gate_s = quantize_fp8_block(rnd(E, I, H))
    up, up_s = quantize_fp8_block(rnd(E, I, H))
    down, down_s = quantize_fp8_block(rnd(E, H, I))
    lw = LayerWeights(router, gate, gate_s, up, up_s, down, down_s)
    if shape.shared_inter:
        Is = shape.shared_inter
        lw.sh_gate, lw.sh_gate_s = quantize_fp8_block(rnd(Is, H))
        lw.sh_up, lw.sh_up_s = quantize_fp8_block(rnd(Is, H))
        lw.sh_down, lw.sh_down_s = quantize_fp8_block(rnd(H, Is))
        lw.sh_router = rnd(1, H).to(torch.bfloat16)
    return lw


def make_hidden(tokens: int, hidden: int, seed: int, rms_normalise=False,
                dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    """bf16 N(0,1) hidden states ``[tokens, hidden]``; optionally RMS-normalised."""
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(int(seed) * 31 + 5)
    x = torch.randn(tokens, hidden, generator=g, device=device, dtype=torch.float32)
    if rms_normalise:
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
    return x.to(dtype)


def zipf_expert_bias(experts: int, seed: int, s: float = 1.2) -> torch.Tensor:
    """Per-expert logit bias log p_e with p_e proportional to rank_e^-s over a
    seeded permutation of the experts (rank 1 = the hottest), shifted so the
    hottest expert's bias is 0: the skewed-routing workload of batched decode
    (a few experts receive most tokens)."""
    g = torch.Generator()
    g.manual_seed(int(seed) * 131 + 17)
    perm = torch.randperm(experts, generator=g)
    rank = torch.empty(experts)
    rank[perm] = torch.arange(1, experts + 1, dtype=torch.float32)
    return -float(s) * torch.log(rank)


def router_with_bias(router_w: torch.Tensor, bias: torch.Tensor, dim: int | None = None) -> torch.Tensor:
    """Carry a per-expert logit bias through an unchanged router: router
    column ``dim`` (default the last) is replaced by the bias, so for tokens
    whose coordinate ``dim`` is 1 (``tokens_for_bias``) the logits are
    sum_{j != dim} W[e, j] x[j] + bias[e].  Returns a new tensor."""
    d = router_w.shape[1] - 1 if dim is None else dim
    w = router_w.clone()
    w[:, d] = bias.to(device=w.device, dtype=w.dtype)
    return w


def tokens_for_bias(x: torch.Tensor, dim: int | None = None) -> torch.Tensor:
    """Copy of the tokens ``x`` [T, H] with coordinate ``dim`` (default the
    last) set to 1, the carrier of ``router_with_bias``'s bias."""
    d = x.shape[1] - 1 if dim is None else dim
    xb = x.clone()
    xb[:, d] = 1
    return xb


def tensor_names(layer: int, expert: int, prefix="model.layers"):
    p = f"{prefix}.{layer}.mlp.experts.{expert}"
    return {m: f"{p}.{m}.weight" for m in ("gate_proj", "up_proj", "down_proj")}


def layer_state_dict(lw: LayerWeights, layer: int, prefix="model.layers", zero_shared=False):
    """Checkpoint tensor dict of one layer, named as the reference's ModelLayout expects."""
    sd = {}
    p = f"{prefix}.{layer}.mlp"
    sd[f"{p}.gate.weight"] = lw.router.contiguous().cpu()
    E = lw.gate.shape[0]
    for e in range(E):
        for m, (w, s) in (("gate_proj", (lw.gate, lw.gate_s)), ("up_proj", (lw.up, lw.up_s)),
                          ("down_proj", (lw.down, lw.down_s))):
            sd[f"{p}.experts.{e}.{m}.weight"] = w[e].contiguous().cpu()
            sd[f"{p}.experts.{e}.{m}.weight_scale_inv"] = s[e].contiguous().cpu()
    if lw.sh_gate is not None:
        for m, (w, s) in (("gate_proj", (lw.sh_gate, lw.sh_gate_s)), ("up_proj", (lw.sh_up, lw.sh_up_s)),
                          ("down_proj", (lw.sh_down, lw.sh_down_s))):
            sd[f"{p}.shared_expert.{m}.weight"] = w.contiguous().cpu()
            sd[f"{p}.shared_expert.{m}.weight_scale_inv"] = s.contiguous().cpu()
        sd[f"{p}.shared_expert_gate.weight"] = lw.sh_router.contiguous().cpu()
    elif zero_shared:
        H = lw.router.shape[1]
        I = lw.gate.shape[1]
        z = torch.zeros
        sd[f"{p}.shared_expert.gate_proj.weight"] = z(I, H, dtype=torch.bfloat16)
        sd[f"{p}.shared_expert.up_proj.weight"] = z(I, H, dtype=torch.bfloat16)
        sd[f"{p}.shared_expert.down_proj.weight"] = z(H, I, dtype=torch.bfloat16)
        sd[f"{p}.shared_expert_gate.weight"] = z(1, H, dtype=torch.bfloat16)
    return sd


def write_checkpoint(path: str, shape: MoEShape, seed: int, layers: int = 1,
                     zero_shared: bool | None = None, model_type=None, device="cpu"):
    """Write a seeded FP8 safetensors checkpoint directory (config.json,
    model.safetensors.index.json, one shard per layer).  ``device``: where the
    weights are generated (the seeded values differ between CPU and CUDA
    generators; the files are the same format)."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    if zero_shared is None:
        zero_shared = shape.shared_inter == 0
    weight_map = {}
    for l in range(layers):
        lw = make_layer(shape, seed, l, device=device)
        sd = layer_state_dict(lw, l, zero_shared=zero_shared)
        del lw
        fname = f"layer-{l:05d}.safetensors"
        save_file(sd, os.path.join(path, fname))
        weight_map.update({k: fname for k in sd})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": dict(sorted(weight_map.items()))}, f)
    mt = model_type or ("qwen3_5_moe" if shape.shared_inter else "qwen3_moe")
    cfg = {
        "model_type": mt,
        "hidden_size": shape.hidden,
        "moe_intermediate_size": shape.inter,
        "num_experts": shape.experts,
        "num_experts_per_tok": shape.top_k,
        "num_hidden_layers": layers,
        "shared_expert_intermediate_size": shape.shared_inter,
        "synthetic_seed": seed,
    }
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return path
