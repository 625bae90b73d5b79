"""Seeded random-init Qwen3-30B-A3B-FP8 checkpoint, generated tensor by tensor.

The full model (48 layers, 29 GB of FP8 experts, two 622 MB bf16 vocabulary
matrices) is too large to write to disk or to draw with ``torch.randn`` on the
host of every machine that needs it.  Here every tensor of the checkpoint is a
pure function of (seed, tensor name, element index) computed with integer
arithmetic only, so the same call gives the same bits on the CPU and on a CUDA
device, in any order and in any chunking:

* a 32-bit integer hash of the element index, keyed by the tensor name, picks
  an entry of a 65536-entry inverse-CDF table of N(0, 1): e4m3 codes of
  N(0, 112) for FP8 weights (a 128x128 block of N(0, sigma) weights quantised
  with scale = amax / 448 has codes of standard deviation ~112), bf16 values of
  N(0, 0.02) for bf16 weights;
* the FP8 block scale (``weight_scale_inv``) of block b is
  (176 + hash(b) mod 16) * 2^-20 (exact in fp32), so dequantised weights have
  standard deviation ~0.02;
* RMSNorm weights are ones (the Hugging Face initialisation).

The tables are computed once from ``torch.special.ndtri`` in float64 on the
host; ``table_digest()`` pins them.  Names and shapes follow the Hugging Face
Qwen3-MoE-FP8 checkpoint layout that the reference's ModelLayout reads
(loader/model_layout.py:90-136).
"""
from __future__ import annotations

import hashlib
import zlib

import torch

M32 = 0xFFFFFFFF

# Hugging Face Qwen3MoeConfig of Qwen3-30B-A3B (the architecture only)
QWEN3_30B_A3B_CONFIG = {
    "architectures": ["Qwen3MoeForCausalLM"],
    "model_type": "qwen3_moe",
    "vocab_size": 151936,
    "hidden_size": 2048,
    "intermediate_size": 6144,
    "num_hidden_layers": 48,
    "num_attention_heads": 32,
    "num_key_value_heads": 4,
    "head_dim": 128,
    "hidden_act": "silu",
    "max_position_embeddings": 40960,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "tie_word_embeddings": False,
    "attention_bias": False,
    "attention_dropout": 0.0,
    "num_experts": 128,
    "num_experts_per_tok": 8,
    "moe_intermediate_size": 768,
    "norm_topk_prob": True,
    "decoder_sparse_step": 1,
    "mlp_only_layers": [],
    "output_router_logits": False,
    "router_aux_loss_coef": 0.001,
    "initializer_range": 0.02,
    "use_cache": True,
    "torch_dtype": "bfloat16",
    "bos_token_id": 151643,
    "eos_token_id": 151645,
}


def config(**overrides) -> dict:
    c = dict(QWEN3_30B_A3B_CONFIG)
    c.update(overrides)
    return c


# ------------------------------------------------------------- hashing ----
def _mix32(x: torch.Tensor) -> torch.Tensor:
    """32-bit avalanche mix on int64 tensors holding values < 2^32.  Every
    multiplier is < 2^31, so no intermediate product reaches 2^63."""
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & M32
    x = x ^ (x >> 15)
    x = (x * 0x2C1B3C6D) & M32
    x = x ^ (x >> 13)
    x = (x * 0x297A2D39) & M32
    return x ^ (x >> 16)


def _key(seed: int, name: str) -> int:
    return (zlib.crc32(name.encode()) ^ ((int(seed) * 0x9E3779B1) & M32)) & M32


def _hash_range(key: int, start: int, n: int, device) -> torch.Tensor:
    i = torch.arange(start, start + n, dtype=torch.int64, device=device)
    return _mix32(_mix32(i ^ key) ^ ((key * 0x2545F491) & M32))


# -------------------------------------------------------------- tables ----
_TABLES = {}


def _tables(device):
    dev = torch.device(device)
    k = (dev.type, dev.index)
    if k not in _TABLES:
        if ("cpu", None) not in _TABLES:
            u = (torch.arange(65536, dtype=torch.float64) + 0.5) / 65536.0
            z = torch.special.ndtri(u)
            fp8 = (z * 112.0).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
            bf16 = (z * 0.02).to(torch.bfloat16)
            _TABLES[("cpu", None)] = (fp8.contiguous(), bf16.contiguous())
        fp8, bf16 = _TABLES[("cpu", None)]
        _TABLES[k] = (fp8.to(dev), bf16.to(dev))
    return _TABLES[k]


def table_digest() -> str:
    """sha256 of the two tables (host copies): pins the generator."""
    fp8, bf16 = _tables("cpu")
    h = hashlib.sha256()
    h.update(fp8.numpy().tobytes())
    h.update(bf16.view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def fp8_codes(seed: int, name: str, shape, device="cpu", chunk: int = 1 << 24) -> torch.Tensor:
    """float8_e4m3fn tensor of ``shape``: codes of N(0, 112) (see module doc)."""
    n = 1
    for s in shape:
        n *= s
    fp8, _ = _tables(device)
    out = torch.empty(n, dtype=torch.uint8, device=device)
    key = _key(seed, name)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        out[a:b] = fp8[_hash_range(key, a, b - a, device) & 0xFFFF]
    return out.view(torch.float8_e4m3fn).reshape(*shape)


def block_scales(seed: int, name: str, shape, device="cpu") -> torch.Tensor:
    """fp32 ``weight_scale_inv`` [M/128, N/128]: (176 + h mod 16) * 2^-20."""
    M, N = shape
    nb = (M // 128) * (N // 128)
    h = _hash_range(_key(seed, name + "_scale_inv"), 0, nb, device)
    return ((176 + (h & 15)).to(torch.float32) * (2.0 ** -20)).reshape(M // 128, N // 128)


def bf16_normal(seed: int, name: str, shape, device="cpu", chunk: int = 1 << 24) -> torch.Tensor:
    """bf16 tensor of ``shape`` ~ N(0, 0.02) (table values, see module doc)."""
    n = 1
    for s in shape:
        n *= s
    _, tab = _tables(device)
    out = torch.empty(n, dtype=torch.bfloat16, device=device)
    key = _key(seed, name)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        out[a:b] = tab[_hash_range(key, a, b - a, device) & 0xFFFF]
    return out.reshape(*shape)


# -------------------------------------------------------- checkpoint ----
def tensor_specs(cfg: dict) -> dict:
    """name -> (shape, kind) of every tensor of the checkpoint.  kind is
    'fp8' (with a ``_scale_inv`` companion listed as 'scale'), 'bf16' or 'ones'."""
    H, V = cfg["hidden_size"], cfg["vocab_size"]
    nh, nkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    E, I = cfg["num_experts"], cfg["moe_intermediate_size"]
    specs = {"model.embed_tokens.weight": ((V, H), "bf16"), "model.norm.weight": ((H,), "ones"),
             "lm_head.weight": ((V, H), "bf16")}

    def fp8(name, shape):
        specs[name] = (shape, "fp8")
        specs[name + "_scale_inv"] = ((shape[0] // 128, shape[1] // 128), "scale")

    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}"
        specs[f"{p}.input_layernorm.weight"] = ((H,), "ones")
        specs[f"{p}.post_attention_layernorm.weight"] = ((H,), "ones")
        fp8(f"{p}.self_attn.q_proj.weight", (nh * hd, H))
        fp8(f"{p}.self_attn.k_proj.weight", (nkv * hd, H))
        fp8(f"{p}.self_attn.v_proj.weight", (nkv * hd, H))
        fp8(f"{p}.self_attn.o_proj.weight", (H, nh * hd))
        specs[f"{p}.self_attn.q_norm.weight"] = ((hd,), "ones")
        specs[f"{p}.self_attn.k_norm.weight"] = ((hd,), "ones")
        specs[f"{p}.mlp.gate.weight"] = ((E, H), "bf16")
        for e in range(E):
            fp8(f"{p}.mlp.experts.{e}.gate_proj.weight", (I, H))
            fp8(f"{p}.mlp.experts.{e}.up_proj.weight", (I, H))
            fp8(f"{p}.mlp.experts.{e}.down_proj.weight", (H, I))
    return specs


def make_tensor(seed: int, name: str, spec, device="cpu") -> torch.Tensor:
    shape, kind = spec
    if kind == "fp8":
        return fp8_codes(seed, name, shape, device)
    if kind == "scale":
        return block_scales(seed, name[: -len("_scale_inv")], (shape[0] * 128, shape[1] * 128), device)
    if kind == "bf16":
        return bf16_normal(seed, name, shape, device)
    if kind == "ones":
        return torch.ones(shape, dtype=torch.bfloat16, device=device)
    raise KeyError(kind)


class ModelSource:
    """Tensor source of ``loader.expert_loader.ExpertLoader`` for the seeded
    random-init model: ``get(name)`` generates the tensor on ``device``."""

    def __init__(self, cfg: dict, seed: int, device="cuda"):
        self.cfg = cfg
        self.seed = seed
        self.device = device
        self.specs = tensor_specs(cfg)
        self.weight_map = {n: "synthetic" for n in self.specs}
        self.config = dict(cfg)

    def has(self, name):
        return name in self.specs

    def get(self, name):
        return make_tensor(self.seed, name, self.specs[name], self.device)

    def layer_experts(self, layout, layer, n_experts, device):
        out = []
        for mk in (layout.gate_tensor, layout.up_tensor, layout.down_tensor):
            names = [mk(layer, e) for e in range(n_experts)]
            w = torch.stack([make_tensor(self.seed, n, self.specs[n], device) for n in names])
            s = torch.stack([make_tensor(self.seed, n + "_scale_inv", self.specs[n + "_scale_inv"], device)
                             for n in names])
            out += [w, s]
        return out

    def close(self):
        pass
