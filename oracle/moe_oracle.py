"""ORACLE -- test infrastructure only, never part of the product path.

CPU restatement of the reference's FP8 MoE expert path (router + expert FFN)
from kaushikharsh99/Turbo-LLM.  It exists to check the CUDA kernels: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it.  Nothing under ``turbo-llm_b200/`` imports it.

The reference is pure Python over PyTorch ops, so this restatement uses the
same PyTorch CPU ops, in the same order and dtypes, as the reference
functions it cites (paths relative to the reference checkout):

* ``dequantize_weight``  <- ``loader/expert_loader.py:127-160``
* ``load_weight``        <- ``loader/expert_loader.py:89-114`` (CUDA branch)
* ``compute_routing``    <- ``execution/router.py:15-42``
* ``routing_groups``     <- ``execution/moe.py:132,164-165`` (implicit grouping)
* ``moe_seq``            <- ``execution/moe.py:7-20``
* ``shared_expert``      <- ``execution/moe.py:73-85`` / ``:191-202``
* ``execute_decode``     <- ``execution/moe.py:26-97``
* ``execute_layer``      <- ``execution/moe.py:99-208``

plus a bit-exact e4m3 decode table (``fp8_e4m3_table``) written from the
format definition (1 sign, 4 exponent bits with bias 7, 3 mantissa bits,
subnormals at exponent 0, NaN at 0x7F/0xFF, no infinities).

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference
itself (in the container where it is mounted) and records its outputs on
seeded inputs; ``tests/test_oracle_golden.py`` checks this module against
those fixtures.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

# ---------------------------------------------------------------------------
# e4m3 decode (format definition, no library involvement)
# ---------------------------------------------------------------------------


def fp8_e4m3_table() -> np.ndarray:
    """float32 value of each of the 256 e4m3fn bit patterns."""
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** (-6)
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


def as_u8(w: torch.Tensor) -> torch.Tensor:
    return w.view(torch.uint8) if w.dtype == torch.float8_e4m3fn else w


def dequant_fp32_exact(w_fp8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Blockwise ``float(w) * scale`` in fp32 via the decode table (one RN multiply)."""
    tab = torch.from_numpy(fp8_e4m3_table())
    w = tab[as_u8(w_fp8).long()]
    M, N = w.shape
    return (w.view(M // 128, 128, N // 128, 128) * scale.float().view(M // 128, 1, N // 128, 1)).view(M, N)


# ---------------------------------------------------------------------------
# loader/expert_loader.py
# ---------------------------------------------------------------------------


def dequantize_weight(w_fp8, scale, dtype):
    """``ExpertLoader.dequantize_weight`` CUDA/CPU branch (expert_loader.py:149-160):
    cast both operands to ``dtype`` and multiply blockwise in ``dtype``."""
    if scale is None:
        return w_fp8.to(dtype=dtype)
    w = w_fp8.to(dtype=dtype)
    scale_d = scale.to(dtype=dtype)
    M, N = w.shape
    return (w.view(M // 128, 128, N // 128, 128) * scale_d.view(M // 128, 1, N // 128, 1)).view(M, N)


def load_weight(tensor, scale, dtype):
    """``ExpertLoader.load_weight`` on a CUDA device (expert_loader.py:107-112):
    FP8 tensors with a ``_scale_inv`` are dequantised in ``dtype``; others cast."""
    if scale is not None:
        return dequantize_weight(tensor, scale, dtype)
    return tensor.to(dtype=dtype)


class OracleLayer:
    """One MoE layer's raw checkpoint tensors plus the loader dtype.

    ``expert(e)`` plays ``ExpertLoader.load_expert`` / ``load_expert_dynamic``
    (expert_loader.py:269-360, :362-576): it returns the dequantised
    ``(gate [I,H], up [I,H], down [H,I])`` in ``dtype``.
    """

    def __init__(self, lw, dtype=torch.bfloat16):
        self.lw = lw
        self.dtype = dtype
        self._cache = {}

    @property
    def router(self):
        return self.lw.router.to(self.dtype)

    def expert(self, e):
        if e not in self._cache:
            lw = self.lw
            self._cache[e] = (dequantize_weight(lw.gate[e], lw.gate_s[e], self.dtype),
                              dequantize_weight(lw.up[e], lw.up_s[e], self.dtype),
                              dequantize_weight(lw.down[e], lw.down_s[e], self.dtype))
        return self._cache[e]

    def drop_cache(self):
        self._cache.clear()

    def shared(self):
        """The four shared-expert tensors (moe.py:53-67), or None for Qwen3."""
        lw = self.lw
        if lw.sh_gate is None:
            return None
        return (load_weight(lw.sh_gate, lw.sh_gate_s, self.dtype),
                load_weight(lw.sh_up, lw.sh_up_s, self.dtype),
                load_weight(lw.sh_down, lw.sh_down_s, self.dtype),
                load_weight(lw.sh_router, None, self.dtype))


# ---------------------------------------------------------------------------
# execution/router.py
# ---------------------------------------------------------------------------


def router_logits(hidden_states, router_weight):
    """router.py:24-27: flatten to ``[T, H]`` and ``F.linear`` in the act dtype."""
    flat = hidden_states.view(-1, hidden_states.shape[-1])
    return F.linear(flat, router_weight)


def compute_routing(hidden_states, router_weight, top_k):
    """``RouterExecutor.compute_routing`` (router.py:15-42)."""
    logits = router_logits(hidden_states, router_weight)
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    top_k_weights, top_k_indices = torch.topk(probs, top_k, dim=-1)
    top_k_weights = top_k_weights / top_k_weights.sum(dim=-1, keepdim=True)
    top_k_weights = top_k_weights.to(logits.dtype)
    return top_k_indices, top_k_weights


def topk_from_logits_stable(logits, top_k):
    """Same selection as ``compute_routing`` but with a stated tie policy:
    value descending, then expert id ascending.  Returns (idx, probs fp32)."""
    probs = F.softmax(logits, dtype=torch.float, dim=-1)
    T, E = logits.shape
    key_vals = logits.float()
    # stable descending sort keeps the lower index first among equal values
    order = torch.sort(key_vals, dim=-1, descending=True, stable=True).indices[:, :top_k]
    return order, torch.gather(probs, 1, order)


def renormalise(top_probs, out_dtype):
    """router.py:37-40: divide by the row sum in fp32, cast to the act dtype."""
    w = top_probs / top_probs.sum(dim=-1, keepdim=True)
    return w.to(out_dtype)


# ---------------------------------------------------------------------------
# execution/moe.py
# ---------------------------------------------------------------------------


def routing_groups(top_k_indices, num_experts=None):
    """The grouping ``execute_layer`` performs implicitly (moe.py:132,164-165):
    unique experts ascending; per expert, ``torch.where(idx == e)`` order
    (token ascending, then k position).  Returns a dict with
    ``counts [E]``, ``offsets [E+1]``, ``tokens [T*k]``, ``kpos [T*k]``
    (slot order) and ``experts`` (the ascending unique list)."""
    idx = top_k_indices
    T, k = idx.shape
    E = num_experts if num_experts is not None else int(idx.max()) + 1
    unique = torch.unique(idx).tolist()
    tokens, kpos = [], []
    counts = torch.zeros(E, dtype=torch.int64)
    for e in unique:
        ti, kp = torch.where(idx == e)
        tokens.append(ti)
        kpos.append(kp)
        counts[e] = ti.numel()
    offsets = torch.zeros(E + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, 0)
    cat = (lambda xs: torch.cat(xs) if xs else torch.zeros(0, dtype=torch.int64))
    return {"counts": counts, "offsets": offsets, "tokens": cat(tokens),
            "kpos": cat(kpos), "experts": unique}


def moe_seq(hidden_states, gate_weights, up_weights, down_weights, top_k_weights):
    """moe.py:7-20."""
    final_output = torch.zeros_like(hidden_states)
    top_k = top_k_weights.shape[1]
    for i in range(top_k):
        g = F.linear(hidden_states, gate_weights[i])
        u = F.linear(hidden_states, up_weights[i])
        inter = F.silu(g) * u
        o = F.linear(inter, down_weights[i])
        final_output += o * top_k_weights[0, i]
    return final_output


def shared_expert(hidden_states, shared):
    """moe.py:74-85 (decode) and :191-202 (multi-token): sigmoid-gated SwiGLU."""
    sg, su, sd, sgate = shared
    shared_hidden = F.silu(F.linear(hidden_states, sg)) * F.linear(hidden_states, su)
    shared_output = F.linear(shared_hidden, sd)
    shared_gate_score = torch.sigmoid(F.linear(hidden_states, sgate))
    return shared_gate_score * shared_output


def execute_decode(layer: OracleLayer, hidden_states, top_k_indices, top_k_weights):
    """moe.py:26-97 (single token)."""
    expert_ids = top_k_indices[0].tolist()
    gates, ups, downs = [], [], []
    for e in expert_ids:
        g, u, d = layer.expert(e)
        gates.append(g)
        ups.append(u)
        downs.append(d)
    final_output = moe_seq(hidden_states, gates, ups, downs, top_k_weights)
    sh = layer.shared()
    if sh is not None:
        final_output += shared_expert(hidden_states, sh)
    return final_output


def execute_layer(layer: OracleLayer, hidden_states, top_k_indices, top_k_weights):
    """moe.py:99-208: T == 1 goes to ``execute_decode``; otherwise per unique
    expert (ascending) gather -> SwiGLU -> weighted scatter-add, then the
    shared expert."""
    if hidden_states.shape[0] == 1:
        return execute_decode(layer, hidden_states, top_k_indices, top_k_weights)
    final_output = torch.zeros_like(hidden_states)
    unique_experts = torch.unique(top_k_indices).tolist()
    if not unique_experts:
        return final_output
    for e in unique_experts:
        gate_proj, up_proj, down_proj = layer.expert(e)
        token_indices, top_k_pos = torch.where(top_k_indices == e)
        if len(token_indices) > 0:
            expert_input = hidden_states[token_indices]
            inter = F.silu(F.linear(expert_input, gate_proj)) * F.linear(expert_input, up_proj)
            expert_output = F.linear(inter, down_proj)
            weights = top_k_weights[token_indices, top_k_pos].unsqueeze(-1)
            final_output[token_indices] += weights * expert_output
    sh = layer.shared()
    if sh is not None:
        final_output += shared_expert(hidden_states, sh)
    return final_output


# ---------------------------------------------------------------------------
# comparison helpers
# ---------------------------------------------------------------------------


def compare(out, ref):
    """(max-abs, cosine) of two tensors, reduced in float64 (an fp32 dot
    product over ~1e5+ elements carries ~1e-5 of rounding, the size of the
    cosine gaps the tests resolve)."""
    a = out.double().flatten()
    b = ref.double().flatten()
    maxabs = (a - b).abs().max().item() if a.numel() else 0.0
    cos = F.cosine_similarity(a, b, dim=0).item() if a.numel() else 1.0
    return maxabs, cos
