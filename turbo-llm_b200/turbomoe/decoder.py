"""Batch-1 greedy decode of a Qwen3-MoE FP8 model on one GPU, every step one
CUDA graph of this library's kernels.

The reference's step loop (runtime/engine.py:98-162) drives Hugging Face
modules layer by layer (execution/layer_executor.py:108-213): embedding,
per layer input RMSNorm -> q/k/v projections (FP8 weights dequantised by
``load_weight``, loader/expert_loader.py:89-114) -> q/k RMSNorm -> rotary
embedding -> KV cache -> attention -> o projection + residual ->
post-attention RMSNorm -> router -> experts + residual, then the final norm,
the LM head and ``torch.argmax``; it reads the chosen token back to the host
with ``.item()`` every step (runtime/engine.py:213,224,254,262).

Here the same step runs as one device-resident sequence: ``tm_embed``,
``tm_rmsnorm``, ``tm_fp8_linear`` (q/k/v fused into one packed [5120, 2048]
weight, o with the residual add), ``tm_qk_rope_kv``, ``tm_attn_decode``, the
drop-in ``RouterExecutor`` / ``MoEExecutor`` (the MoE hot path), and
``tm_lm_head_argmax``, which writes the next token id into the device buffer
the next step's embedding reads.  The position lives on the device too, so
the captured step is replayed with no host round trip; generated ids are
copied out once at the end.

Precision follows the activation dtype of the loader (``loader.dtype``):
bf16/fp16 steps use the tensor-core FP8 kernels; fp32 steps use the fp32
variants (CUDA-core FP8 linear, fp32 router/experts).  KV cache and rotary
table are in the activation dtype, as the reference's.
"""
from __future__ import annotations

import math

import torch

from . import ops
from ._lib import TurboMoEError, check, lib


def rope_table(head_dim: int, theta: float, max_len: int, dtype) -> torch.Tensor:
    """[max_len, 2, head_dim] (cos, sin) exactly as Qwen3MoeRotaryEmbedding
    computes them (host fp32: inv_freq, position * inv_freq, cos/sin, rounded
    to ``dtype``)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))
    pos = torch.arange(max_len, dtype=torch.int64).float()
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return torch.stack((emb.cos() * 1.0, emb.sin() * 1.0), dim=1).to(dtype).contiguous()


class Qwen3MoeDecoder:
    """Greedy batch-1 decoder over an ``ExpertLoader`` (any tensor source:
    safetensors snapshot or a synthetic model) for a Qwen3-MoE config dict."""

    def __init__(self, loader, cfg: dict, max_len: int, attn_splits: int = 37, device=None):
        from execution.moe import MoEExecutor
        from execution.router import RouterExecutor
        self.loader, self.cfg = loader, cfg
        self.dev = torch.device(device or "cuda", torch.cuda.current_device()) if device is None else \
            torch.device(device)
        dt = loader.dtype
        self.dtype = dt
        self.L = cfg["num_hidden_layers"]
        self.H, self.V = cfg["hidden_size"], cfg["vocab_size"]
        self.nh, self.nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        self.hd = cfg.get("head_dim") or self.H // self.nh
        if self.hd != 128:
            raise TurboMoEError(f"head_dim {self.hd} unsupported (128)")
        self.eps = float(cfg.get("rms_norm_eps", 1e-6))
        self.max_len = max_len
        self.splits = attn_splits
        dev = self.dev
        src = loader.source
        get_raw = lambda n: src.get(n).to(dev)
        self.embed = get_raw("model.embed_tokens.weight").to(torch.bfloat16).contiguous()
        self.lm_head = get_raw("lm_head.weight").to(torch.bfloat16).contiguous()
        self.final_norm = loader.load_weight("model.norm.weight", device=dev).contiguous()
        self.layers = []
        for l in range(self.L):
            p = f"model.layers.{l}"
            raw = [loader.load_weight_raw(f"{p}.self_attn.{m}_proj.weight", device=dev) for m in ("q", "k", "v")]
            w_qkv = torch.cat([r[0].view(torch.uint8) for r in raw], 0)
            s_qkv = torch.cat([r[1].float() for r in raw], 0)
            wo, so = loader.load_weight_raw(f"{p}.self_attn.o_proj.weight", device=dev)
            self.layers.append({
                "in_norm": loader.load_weight(f"{p}.input_layernorm.weight", device=dev).contiguous(),
                "post_norm": loader.load_weight(f"{p}.post_attention_layernorm.weight", device=dev).contiguous(),
                "q_norm": loader.load_weight(f"{p}.self_attn.q_norm.weight", device=dev).contiguous(),
                "k_norm": loader.load_weight(f"{p}.self_attn.k_norm.weight", device=dev).contiguous(),
                "qkv": ops.pack_linear(w_qkv, s_qkv),
                "o": ops.pack_linear(wo, so),
            })
            del raw, w_qkv, s_qkv, wo, so
        self.router = RouterExecutor(loader, self.L, top_k=cfg.get("num_experts_per_tok", 8))
        self.moe = MoEExecutor(loader, record_timing=False)
        loader.upload()
        H, nh, nkv, hd = self.H, self.nh, self.nkv, self.hd
        self.kv = torch.zeros(self.L, 2, nkv, max_len, hd, dtype=dt, device=dev)
        self.rope = rope_table(hd, float(cfg.get("rope_theta", 1e6)), max_len, dt).to(dev)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.x = torch.zeros(1, H, dtype=dt, device=dev)
        self.normed = torch.zeros(1, H, dtype=dt, device=dev)
        self.qkv = torch.zeros(1, (nh + 2 * nkv) * hd, dtype=dt, device=dev)
        self.q = torch.zeros(1, nh * hd, dtype=dt, device=dev)
        self.attn = torch.zeros(1, nh * hd, dtype=dt, device=dev)
        self.x_attn = torch.zeros(1, H, dtype=dt, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        Lb = lib()
        self.attn_ws = torch.zeros(Lb.tm_attn_decode_workspace_bytes(nh, nkv, self.splits), dtype=torch.uint8,
                                   device=dev)
        self.lm_ws = torch.zeros(Lb.tm_lm_head_workspace_bytes(), dtype=torch.uint8, device=dev)
        self.code = ops._code(dt)
        self.scale = 1.0 / math.sqrt(hd)
        # 16-bit activations of the Qwen3-30B-A3B shape: the input norm runs
        # inside the q/k/v projection and the post-attention norm inside the
        # router (two launches fewer per layer, the same bits)
        self.fused_norms = (dt in (torch.bfloat16, torch.float16) and H == 2048
                            and loader.num_experts <= 128 and self.router.top_k <= 8)
        # 16-bit: q/k norm, rotary and the KV append run inside the attention
        # launch (tm_qk_rope_attn_decode; positions are checked on the host)
        self.fused_rope = dt in (torch.bfloat16, torch.float16) and nh // nkv <= 16
        self.graph = None
        loader.workspace(dev).ensure(1)

    # ------------------------------------------------------------ one step ----
    def _step(self):
        """Token ``self.token`` at position ``self.pos`` through the model;
        leaves the greedy next token in ``self.token`` and advances ``self.pos``."""
        Lb, s = lib(), torch.cuda.current_stream(self.dev).cuda_stream
        H, nh, nkv, hd, code = self.H, self.nh, self.nkv, self.hd, self.code
        st = self.status.data_ptr()
        check(Lb.tm_embed(self.token.data_ptr(), 1, self.embed.data_ptr(), H, self.V, code, self.x.data_ptr(), st,
                          s), "tm_embed")
        x = self.x
        for l, ly in enumerate(self.layers):
            if self.fused_norms:
                ops.rmsnorm_fp8_linear(x, ly["in_norm"], self.eps, ly["qkv"], out=self.qkv)
            else:
                check(Lb.tm_rmsnorm(x.data_ptr(), 1, H, code, ly["in_norm"].data_ptr(), self.eps,
                                    self.normed.data_ptr(), s), "tm_rmsnorm")
                ops.fp8_linear(self.normed, ly["qkv"], out=self.qkv)
            kc, vc = self.kv[l, 0], self.kv[l, 1]
            if self.fused_rope:
                check(Lb.tm_qk_rope_attn_decode(self.qkv.data_ptr(), ly["q_norm"].data_ptr(), ly["k_norm"].data_ptr(),
                                                self.eps, self.rope.data_ptr(), self.pos.data_ptr(), self.max_len,
                                                nh, nkv, hd, code, self.scale, self.splits, kc.data_ptr(),
                                                vc.data_ptr(), self.attn.data_ptr(), s), "tm_qk_rope_attn_decode")
            else:
                check(Lb.tm_qk_rope_kv(self.qkv.data_ptr(), 1, nh, nkv, hd, code, ly["q_norm"].data_ptr(),
                                       ly["k_norm"].data_ptr(), self.eps, self.rope.data_ptr(), self.pos.data_ptr(),
                                       self.max_len, self.q.data_ptr(), kc.data_ptr(), vc.data_ptr(), st, s),
                      "tm_qk_rope_kv")
                check(Lb.tm_attn_decode(self.q.data_ptr(), kc.data_ptr(), vc.data_ptr(), self.pos.data_ptr(),
                                        self.max_len, nh, nkv, hd, code, self.scale, self.splits,
                                        self.attn.data_ptr(), self.attn_ws.data_ptr(), self.attn_ws.numel(), s),
                      "tm_attn_decode")
            ops.fp8_linear(self.attn, ly["o"], residual=x, out=self.x_attn)
            if self.fused_norms:
                idx, w = ops.rmsnorm_router_topk(self.x_attn, ly["post_norm"], self.eps, self.router.routers[l],
                                                 self.router.top_k, self.loader.workspace(self.dev), self.normed)
            else:
                check(Lb.tm_rmsnorm(self.x_attn.data_ptr(), 1, H, code, ly["post_norm"].data_ptr(), self.eps,
                                    self.normed.data_ptr(), s), "tm_rmsnorm")
                idx, w = self.router.compute_routing(l, self.normed)
            self.moe.execute_layer(l, self.normed, idx, w, residual=self.x_attn, out=self.x)
        check(Lb.tm_rmsnorm(x.data_ptr(), 1, H, code, self.final_norm.data_ptr(), self.eps,
                            self.normed.data_ptr(), s), "tm_rmsnorm")
        check(Lb.tm_lm_head_argmax(self.normed.data_ptr(), H, code, self.lm_head.data_ptr(), self.V, None,
                                   self.token.data_ptr(), self.lm_ws.data_ptr(), self.lm_ws.numel(), s),
              "tm_lm_head_argmax")
        self.pos.add_(1)

    def capture(self):
        """Record one step in a CUDA graph (replayed by ``step``)."""
        tok, pos = self.token.clone(), self.pos.clone()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step()
        self.graph = g
        # the warm-up and the capture itself advanced nothing that matters:
        # restore the token, the position and the cache row they touched
        self.token.copy_(tok)
        self.pos.copy_(pos)
        return g

    def step(self):
        if self.graph is None:
            self._step()
        else:
            self.graph.replay()

    def reset(self):
        self.kv.zero_()
        self.pos.zero_()
        self.status.zero_()

    def teacher_forced(self, ids) -> list:
        """Feed ``ids`` one per step (positions 0, 1, ...); returns the greedy
        choice after each position (what the model would emit next)."""
        ids = list(int(t) for t in ids)
        if len(ids) > self.max_len:
            raise TurboMoEError(f"{len(ids)} positions exceed max_len {self.max_len}")
        self.reset()
        out = torch.empty(len(ids), dtype=torch.int64, device=self.dev)
        host = torch.tensor(ids, dtype=torch.int64).pin_memory()
        for i in range(len(ids)):
            self.token.copy_(host[i:i + 1], non_blocking=True)
            self.step()
            out[i:i + 1].copy_(self.token)
        if int(self.status.item()):
            raise TurboMoEError(f"decode status {int(self.status.item()):#x}")
        return out.tolist()

    def generate(self, prompt_ids, steps: int) -> list:
        """Greedy continuation of ``prompt_ids`` (host ints): the prompt enters
        one token per step (the causal prefill, one position at a time), then
        ``steps`` tokens are generated.  Returns the generated ids."""
        prompt = list(int(t) for t in prompt_ids)
        if len(prompt) + steps > self.max_len:
            raise TurboMoEError(f"{len(prompt)} + {steps} positions exceed max_len {self.max_len}")
        self.reset()
        out = torch.empty(steps, dtype=torch.int64, device=self.dev)
        host = torch.tensor(prompt, dtype=torch.int64).pin_memory()
        for i, _t in enumerate(prompt):
            self.token.copy_(host[i:i + 1], non_blocking=True)
            self.step()
        out[0:1].copy_(self.token)
        for i in range(1, steps):
            self.step()
            out[i:i + 1].copy_(self.token)
        if int(self.status.item()):
            raise TurboMoEError(f"decode status {int(self.status.item()):#x}")
        return out.tolist()
