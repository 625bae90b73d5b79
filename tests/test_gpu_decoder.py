"""The decode-step kernels around the MoE path (tm_embed, tm_rmsnorm,
tm_qk_rope_kv, tm_attn_decode, tm_lm_head_argmax, the fp32 tm_fp8_linear) and
the whole greedy decoder (turbomoe/decoder.py), against the Hugging Face
Qwen3-MoE modules that the reference engine drives (transformers is installed
on every machine): Qwen3MoeRMSNorm, Qwen3MoeRotaryEmbedding +
apply_rotary_pos_emb, scaled-dot-product attention, F.linear, torch.argmax,
and a whole Qwen3MoeForCausalLM for a small configuration.

Tolerances: fp32 results within 1e-5 relative of the fp32 reference (only the
order of sums differs); bf16/fp16 results within one act-dtype rounding of
the reference computed the same way (products and sums of the reference's
rounding points reproduced; accumulation order and rsqrt/exp implementations
may move a value across one rounding boundary).
"""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _lib():
    from turbomoe._lib import lib
    return lib()


def _s():
    return torch.cuda.current_stream().cuda_stream


def _ulp_close(got, want, dt, frac=0.01):
    """All elements within 2 act-dtype ulps, and at most `frac` of them off by
    more than one rounding of their magnitude."""
    got, want = got.float().cpu(), want.float().cpu()
    eps = torch.finfo(dt).eps
    tol = want.abs().clamp_min(1e-3) * eps
    d = (got - want).abs()
    assert bool((d <= 2 * tol + 1e-6).all()), f"max diff {float(d.max()):.3e}"
    assert float((d > tol + 1e-7).float().mean()) <= frac


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_rmsnorm_matches_hf(dt):
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeRMSNorm
    from turbomoe import ops
    g = torch.Generator(device="cuda").manual_seed(1)
    x = (torch.randn(3, 2048, generator=g, device="cuda") * 3).to(dt)
    w = (1 + 0.1 * torch.randn(2048, generator=g, device="cuda")).to(dt)
    ref = Qwen3MoeRMSNorm(2048, eps=1e-6).cuda().to(dt)
    ref.weight.data.copy_(w)
    want = ref(x)
    out = torch.empty_like(x)
    assert _lib().tm_rmsnorm(x.data_ptr(), 3, 2048, ops._code(dt), w.data_ptr(), 1e-6, out.data_ptr(), _s()) == 0
    if dt == torch.float32:
        torch.testing.assert_close(out, want, rtol=1e-5, atol=1e-6)
    else:
        _ulp_close(out, want, dt)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("pos", [0, 37, 4000])
def test_qk_rope_kv_matches_hf(dt, pos):
    from transformers.models.qwen3_moe.modeling_qwen3_moe import (Qwen3MoeRMSNorm, Qwen3MoeRotaryEmbedding,
                                                                   apply_rotary_pos_emb, Qwen3MoeConfig)
    from turbomoe import ops, synth_model
    from turbomoe.decoder import rope_table
    nh, nkv, hd, max_len = 32, 4, 128, 4096 + 8
    g = torch.Generator(device="cuda").manual_seed(2 + pos)
    qkv = (torch.randn(1, (nh + 2 * nkv) * hd, generator=g, device="cuda")).to(dt)
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")).to(dt)
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")).to(dt)
    cfg = Qwen3MoeConfig(**{k: v for k, v in synth_model.config().items() if k not in ("architectures", "torch_dtype")})
    rot = Qwen3MoeRotaryEmbedding(cfg)     # on the host, where the reference engine ran it
    cos, sin = rot(qkv.view(1, 1, -1).cpu(), torch.tensor([[pos]]))
    cos, sin = cos.cuda(), sin.cuda()
    qnm, knm = Qwen3MoeRMSNorm(hd, 1e-6).cuda().to(dt), Qwen3MoeRMSNorm(hd, 1e-6).cuda().to(dt)
    qnm.weight.data.copy_(qn)
    knm.weight.data.copy_(kn)
    q = qnm(qkv[:, :nh * hd].view(1, 1, nh, hd)).transpose(1, 2)
    k = knm(qkv[:, nh * hd:(nh + nkv) * hd].view(1, 1, nkv, hd)).transpose(1, 2)
    qe, ke = apply_rotary_pos_emb(q, k, cos, sin)
    table = rope_table(hd, 1e6, max_len, dt).cuda()
    assert torch.equal(table[pos, 0], cos[0, 0]) and torch.equal(table[pos, 1], sin[0, 0])
    q_out = torch.empty(1, nh * hd, dtype=dt, device="cuda")
    kc = torch.zeros(nkv, max_len, hd, dtype=dt, device="cuda")
    vc = torch.zeros_like(kc)
    p = torch.tensor([pos], device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib().tm_qk_rope_kv(qkv.data_ptr(), 1, nh, nkv, hd, ops._code(dt), qn.data_ptr(), kn.data_ptr(), 1e-6,
                              table.data_ptr(), p.data_ptr(), max_len, q_out.data_ptr(), kc.data_ptr(),
                              vc.data_ptr(), st.data_ptr(), _s())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(vc[:, pos], qkv[0, (nh + nkv) * hd:].view(nkv, hd))
    assert int(kc[:, :pos].abs().sum() + kc[:, pos + 1:].abs().sum()) == 0
    if dt == torch.float32:
        torch.testing.assert_close(q_out.view(nh, hd), qe[0, :, 0], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(kc[:, pos], ke[0, :, 0], rtol=1e-5, atol=1e-6)
    else:
        _ulp_close(q_out.view(nh, hd), qe[0, :, 0], dt)
        _ulp_close(kc[:, pos], ke[0, :, 0], dt)
    # a position outside the cache is refused on the device
    p.fill_(max_len)
    _lib().tm_qk_rope_kv(qkv.data_ptr(), 1, nh, nkv, hd, ops._code(dt), qn.data_ptr(), kn.data_ptr(), 1e-6,
                         table.data_ptr(), p.data_ptr(), max_len, q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                         st.data_ptr(), _s())
    torch.cuda.synchronize()
    from turbomoe._lib import TM_STATUS_BAD_TOKEN_ID
    assert int(st.item()) & TM_STATUS_BAD_TOKEN_ID


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n,splits", [(1, 37), (33, 37), (1000, 37), (2100, 8), (2100, 1), (65, 3)])
def test_attn_decode_matches_sdpa(dt, n, splits):
    from turbomoe import ops
    nh, nkv, hd, max_len = 32, 4, 128, 2200
    g = torch.Generator(device="cuda").manual_seed(n * 7 + splits)
    q = torch.randn(nh, hd, generator=g, device="cuda").to(dt)
    kc = torch.randn(nkv, max_len, hd, generator=g, device="cuda").to(dt)
    vc = torch.randn(nkv, max_len, hd, generator=g, device="cuda").to(dt)
    # poison the rows past the context: they must not be read
    kc[:, n:] = float("nan")
    vc[:, n:] = float("nan")
    scale = 1.0 / math.sqrt(hd)
    qf = q.float().view(1, nh, 1, hd)
    kf = kc[:, :n].float().repeat_interleave(nh // nkv, 0).unsqueeze(0)
    vf = vc[:, :n].float().repeat_interleave(nh // nkv, 0).unsqueeze(0)
    want = F.scaled_dot_product_attention(qf, kf, vf, scale=scale)[0, :, 0]
    ws = torch.zeros(_lib().tm_attn_decode_workspace_bytes(nh, nkv, splits), dtype=torch.uint8, device="cuda")
    out = torch.empty(nh * hd, dtype=dt, device="cuda")
    pos = torch.tensor([n - 1], device="cuda")
    for _ in range(2):   # twice: the merge counters reset themselves
        out.zero_()
        rc = _lib().tm_attn_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), max_len, nh, nkv, hd,
                                   ops._code(dt), scale, splits, out.data_ptr(), ws.data_ptr(), ws.numel(), _s())
        assert rc == 0
        torch.cuda.synchronize()
        got = out.view(nh, hd).float()
        if dt == torch.float32:
            torch.testing.assert_close(got, want, rtol=1e-5, atol=2e-6)
        else:
            _ulp_close(got, want.to(dt), dt)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("nh,nkv,n,splits", [(16, 4, 300, 16), (24, 2, 777, 5), (32, 2, 129, 16), (8, 8, 2048, 12),
                                             (32, 4, 4096, 64)])
def test_attn_decode_group_sizes(dt, nh, nkv, n, splits):
    """Query-head groups of 4, 12, 16 and 1 heads (one and two 8-column MMA
    blocks, unused columns), requests above the 16-CTA cluster, 16-bit
    activations: within one act-dtype rounding of fp32 attention."""
    from turbomoe import ops
    hd, max_len = 128, 4100
    g = torch.Generator(device="cuda").manual_seed(nh * 31 + n)
    q = torch.randn(nh, hd, generator=g, device="cuda").to(dt)
    kc = torch.randn(nkv, max_len, hd, generator=g, device="cuda").to(dt)
    vc = torch.randn(nkv, max_len, hd, generator=g, device="cuda").to(dt)
    kc[:, n:] = float("nan")
    vc[:, n:] = float("nan")
    scale = 1.0 / math.sqrt(hd)
    qf = q.float().view(1, nh, 1, hd)
    kf = kc[:, :n].float().repeat_interleave(nh // nkv, 0).unsqueeze(0)
    vf = vc[:, :n].float().repeat_interleave(nh // nkv, 0).unsqueeze(0)
    want = F.scaled_dot_product_attention(qf, kf, vf, scale=scale)[0, :, 0]
    ws = torch.zeros(_lib().tm_attn_decode_workspace_bytes(nh, nkv, splits), dtype=torch.uint8, device="cuda")
    out = torch.full((nh * hd,), float("nan"), dtype=dt, device="cuda")
    pos = torch.tensor([n - 1], device="cuda")
    rc = _lib().tm_attn_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), max_len, nh, nkv, hd,
                               ops._code(dt), scale, splits, out.data_ptr(), ws.data_ptr(), ws.numel(), _s())
    assert rc == 0
    torch.cuda.synchronize()
    _ulp_close(out.view(nh, hd).float(), want.to(dt), dt)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("nh,nkv,splits", [(32, 4, 1), (32, 4, 3), (16, 1, 16)])
def test_attn_decode_batched_ragged(dt, nh, nkv, splits):
    """tm_attn_decode_batched: five sequences with their own context lengths
    (1 to the whole cache), caches one padded stride apart, positions past each
    context poisoned; each sequence within one act-dtype rounding of fp32
    attention, and bit-identical to the one-sequence entry point."""
    from turbomoe import ops
    B, hd, max_len = 5, 128, 700
    lengths = [1, 33, 700, 257, 64]
    stride = nkv * max_len * hd + 8 * hd          # elements between sequences (padded)
    g = torch.Generator(device="cuda").manual_seed(nh + splits)
    q = torch.randn(B, nh, hd, generator=g, device="cuda").to(dt)
    kbuf = torch.randn(B * stride, generator=g, device="cuda").to(dt)
    vbuf = torch.randn(B * stride, generator=g, device="cuda").to(dt)
    kc = kbuf.view(B, stride)[:, : nkv * max_len * hd].view(B, nkv, max_len, hd)
    vc = vbuf.view(B, stride)[:, : nkv * max_len * hd].view(B, nkv, max_len, hd)
    for b, n in enumerate(lengths):
        kc[b, :, n:] = float("nan")
        vc[b, :, n:] = float("nan")
    pos = torch.tensor([n - 1 for n in lengths], device="cuda")
    out = torch.full((B, nh * hd), float("nan"), dtype=dt, device="cuda")
    scale = 1.0 / math.sqrt(hd)
    rc = _lib().tm_attn_decode_batched(q.data_ptr(), kbuf.data_ptr(), vbuf.data_ptr(), pos.data_ptr(), B, stride,
                                       max_len, nh, nkv, hd, ops._code(dt), scale, splits, out.data_ptr(), _s())
    assert rc == 0
    torch.cuda.synchronize()
    for b, n in enumerate(lengths):
        qf = q[b].float().view(1, nh, 1, hd)
        kf = kc[b, :, :n].float().repeat_interleave(nh // nkv, 0).unsqueeze(0)
        vf = vc[b, :, :n].float().repeat_interleave(nh // nkv, 0).unsqueeze(0)
        want = F.scaled_dot_product_attention(qf, kf, vf, scale=scale)[0, :, 0]
        _ulp_close(out[b].view(nh, hd).float(), want.to(dt), dt)
    # sequence 3 through the one-sequence entry point: the same kernel, the same bits
    ws = torch.zeros(_lib().tm_attn_decode_workspace_bytes(nh, nkv, splits), dtype=torch.uint8, device="cuda")
    one = torch.empty(nh * hd, dtype=dt, device="cuda")
    kc3, vc3 = kc[3].contiguous(), vc[3].contiguous()
    assert _lib().tm_attn_decode(q[3].contiguous().data_ptr(), kc3.data_ptr(), vc3.data_ptr(), pos[3:4].data_ptr(),
                                 max_len, nh, nkv, hd, ops._code(dt), scale, splits, one.data_ptr(), ws.data_ptr(),
                                 ws.numel(), _s()) == 0
    torch.cuda.synchronize()
    assert torch.equal(one, out[3])


def test_attn_decode_batched_rejects():
    """Host checks of the batched entry point (no launch): fp32, a stride
    shorter than one sequence's caches, batch 0."""
    from turbomoe import ops
    t = torch.zeros(4096, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(2, dtype=torch.int64, device="cuda")
    L = _lib()
    args = lambda dt, B, stride: (t.data_ptr(), t.data_ptr(), t.data_ptr(), pos.data_ptr(), B, stride, 8, 8, 1, 128,
                                  ops._code(dt), 0.1, 1, t.data_ptr(), _s())
    assert L.tm_attn_decode_batched(*args(torch.float32, 2, 1024)) != 0
    assert L.tm_attn_decode_batched(*args(torch.bfloat16, 2, 512)) != 0
    assert L.tm_attn_decode_batched(*args(torch.bfloat16, 0, 1024)) != 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_lm_head_argmax(dt):
    from turbomoe import ops
    V, H = 50021, 2048
    g = torch.Generator(device="cuda").manual_seed(3)
    w = (torch.randn(V, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(H, generator=g, device="cuda").to(dt)
    ws = torch.zeros(_lib().tm_lm_head_workspace_bytes(), dtype=torch.uint8, device="cuda")
    tok = torch.full((1,), -5, dtype=torch.int64, device="cuda")
    logits = torch.empty(V, dtype=dt, device="cuda")

    def run():
        rc = _lib().tm_lm_head_argmax(x.data_ptr(), H, ops._code(dt), w.data_ptr(), V, logits.data_ptr(),
                                      tok.data_ptr(), ws.data_ptr(), ws.numel(), _s())
        assert rc == 0
        torch.cuda.synchronize()
        return int(tok.item())

    want = (x.float() @ w.float().T).to(dt)
    t = run()
    if dt == torch.float32:
        torch.testing.assert_close(logits, want, rtol=1e-5, atol=1e-5)
        assert t == int(torch.argmax(want))
    else:
        _ulp_close(logits, want, dt)
    assert t == int(torch.argmax(logits))   # the first index of the largest of its own logits
    # ties: copy the winning row to a lower and a higher index: the lowest wins
    r = int(torch.argmax(logits))
    lo, hi = 17, V - 3
    w[lo] = w[r]
    w[hi] = w[r]
    assert run() == min(lo, r)
    # the counter reset itself: the same call again gives the same answer
    assert run() == min(lo, r)


def test_embed_and_bad_ids():
    from turbomoe import ops
    from turbomoe._lib import TM_STATUS_BAD_TOKEN_ID
    V, H = 1000, 512
    table = torch.randn(V, H, device="cuda").to(torch.bfloat16)
    ids = torch.tensor([5, 999, 0], device="cuda")
    out = torch.empty(3, H, dtype=torch.float32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _lib().tm_embed(ids.data_ptr(), 3, table.data_ptr(), H, V, ops._code(torch.float32), out.data_ptr(),
                           st.data_ptr(), _s()) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids].float()) and int(st.item()) == 0
    ids[1] = V
    _lib().tm_embed(ids.data_ptr(), 3, table.data_ptr(), H, V, ops._code(torch.float32), out.data_ptr(),
                    st.data_ptr(), _s())
    torch.cuda.synchronize()
    assert int(st.item()) & TM_STATUS_BAD_TOKEN_ID and float(out[1].abs().sum()) == 0.0


@pytest.mark.parametrize("T", [1, 5])
def test_fp8_linear_fp32_matches_dequant_linear(T):
    from turbomoe import ops, synth
    from oracle import moe_oracle as O
    N, K = 640, 2048
    g = torch.Generator().manual_seed(9 + T)
    w, s = synth.quantize_fp8_block(torch.randn(N, K, generator=g) * 0.02)
    pl = ops.pack_linear(w.cuda(), s.cuda())
    x = torch.randn(T, K, generator=g)
    res = torch.randn(T, N, generator=g)
    want = F.linear(x.double(), O.dequant_fp32_exact(w, s).double()) + res.double()
    got = ops.fp8_linear(x.cuda(), pl, residual=res.cuda())
    torch.testing.assert_close(got.cpu().double(), want, rtol=2e-5, atol=2e-5)


# ------------------------------------------------------- whole decoder ----
SMALL = dict(vocab_size=3000, hidden_size=512, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
             head_dim=128, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256,
             max_position_embeddings=4096)


def _hf_model(cfg, seed, dtype):
    """Qwen3MoeForCausalLM with the synthetic model's weights, FP8 tensors
    dequantised exactly (fp32), on the GPU."""
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM
    from turbomoe import synth_model as S
    hc = Qwen3MoeConfig(**{k: v for k, v in cfg.items() if k not in ("architectures", "torch_dtype")})
    hc._attn_implementation = "sdpa"
    m = Qwen3MoeForCausalLM(hc).to(torch.float32).cuda().eval()
    specs = S.tensor_specs(cfg)

    def get(name):
        t = S.make_tensor(seed, name, specs[name], "cuda")
        if specs[name][1] == "fp8":
            sc = S.make_tensor(seed, name + "_scale_inv", specs[name + "_scale_inv"], "cuda")
            M, N = t.shape
            t = (t.float().view(M // 128, 128, N // 128, 128) * sc.view(M // 128, 1, N // 128, 1)).view(M, N)
        return t.float()

    sd = {}
    E = cfg["num_experts"]
    for name in specs:
        if name.endswith("_scale_inv") or ".experts." in name:
            continue
        sd[name] = get(name)
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}.mlp.experts"
        gate = torch.stack([get(f"{p}.{e}.gate_proj.weight") for e in range(E)])
        up = torch.stack([get(f"{p}.{e}.up_proj.weight") for e in range(E)])
        sd[f"{p}.gate_up_proj"] = torch.cat([gate, up], 1)
        sd[f"{p}.down_proj"] = torch.stack([get(f"{p}.{e}.down_proj.weight") for e in range(E)])
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in k for k in missing), missing
    return m.to(dtype)


def _decoder(cfg, seed, dtype, max_len):
    from loader.expert_loader import ExpertLoader
    from turbomoe import synth_model as S
    from turbomoe.decoder import Qwen3MoeDecoder
    dn = {torch.float32: "fp32", torch.bfloat16: "bf16"}[dtype]
    L = ExpertLoader(None, config={"execution": {"dtype": dn}}, source=S.ModelSource(cfg, seed, "cuda"))
    return Qwen3MoeDecoder(L, cfg, max_len=max_len, attn_splits=5)


def _hf_greedy(m, prompt, steps):
    """Greedy continuation by the Hugging Face model (whole sequence per step)."""
    seq = list(prompt)
    with torch.no_grad():
        for _ in range(steps):
            logits = m(torch.tensor([seq], device="cuda")).logits
            seq.append(int(torch.argmax(logits[0, -1])))
    return seq[len(prompt):]


def test_small_model_greedy_fp32_matches_hf():
    """fp32: identical greedy tokens to Qwen3MoeForCausalLM over 24 steps,
    eager and from the captured CUDA graph."""
    from turbomoe import synth_model as S
    cfg = S.config(**SMALL)
    m = _hf_model(cfg, 11, torch.float32)
    prompt = [7, 2999, 123, 0, 42, 1777]
    want = _hf_greedy(m, prompt, 24)
    dec = _decoder(cfg, 11, torch.float32, 64)
    assert dec.generate(prompt, 24) == want
    dec.capture()
    assert dec.generate(prompt, 24) == want


def test_small_model_bf16_teacher_forced():
    """bf16 (the product dtype): fed the fp32 reference's own sequence, the
    decoder's greedy choice agrees with the reference at every position whose
    reference top-2 logit margin exceeds the bf16 resolution of the logits."""
    from turbomoe import synth_model as S
    cfg = S.config(**SMALL)
    m = _hf_model(cfg, 12, torch.float32)
    prompt = [11, 2, 2500, 77]
    ref = _hf_greedy(m, prompt, 24)
    seq = prompt + ref
    with torch.no_grad():
        logits = m(torch.tensor([seq], device="cuda")).logits[0].float()
    dec = _decoder(cfg, 12, torch.bfloat16, 64)
    dec.capture()
    got = dec.teacher_forced(seq[:-1])
    checked = 0
    for i in range(len(prompt) - 1, len(seq) - 1):
        top2 = torch.topk(logits[i], 2).values
        margin = float(top2[0] - top2[1])
        if margin > 4 * float(top2[0].abs()) * torch.finfo(torch.bfloat16).eps:
            checked += 1
            assert got[i] == seq[i + 1], (i, got[i], seq[i + 1], margin)
    assert checked >= 8


# ------------------------------------------------------------ fused norms ----
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_rmsnorm_fused_entry_points_same_bits(dt):
    """tm_rmsnorm_fp8_linear == tm_rmsnorm then tm_fp8_linear, and
    tm_rmsnorm_router_topk == tm_rmsnorm then tm_router_topk (indices, weights,
    the normalised token), bit for bit: the fused kernels use tm_rmsnorm's
    thread decomposition and order of sums."""
    from turbomoe import ops, synth
    H, N, E, k = 2048, 5120, 128, 8
    g = torch.Generator(device="cuda").manual_seed(5)
    x = (torch.randn(1, H, generator=g, device="cuda") * 3).to(dt)
    nw = (1 + 0.1 * torch.randn(H, generator=g, device="cuda")).to(dt)
    w8, s8 = synth.quantize_fp8_block(torch.randn(N, H, generator=torch.Generator().manual_seed(9)) * 0.02)
    pl = ops.pack_linear(w8.cuda(), s8.cuda())
    router = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(dt)
    L = _lib()
    normed = torch.empty_like(x)
    assert L.tm_rmsnorm(x.data_ptr(), 1, H, ops._code(dt), nw.data_ptr(), 1e-6, normed.data_ptr(), _s()) == 0
    want_lin = ops.fp8_linear(normed, pl)
    got_lin = ops.rmsnorm_fp8_linear(x, nw, 1e-6, pl)
    ws = ops.Workspace("cuda", E, k, H, 768)
    want_idx, want_w = ops.router_topk(normed, router, k, ws)
    xn = torch.full_like(x, float("nan"))
    got_idx, got_w = ops.rmsnorm_router_topk(x, nw, 1e-6, router, k, ws, xn)
    torch.cuda.synchronize()
    assert torch.equal(got_lin, want_lin)
    assert torch.equal(xn, normed)
    assert torch.equal(got_idx, want_idx) and torch.equal(got_w, want_w)


def test_decoder_fused_norms_same_bits():
    """The bf16 decoder with its norms fused into the q/k/v projection and the
    router, and its q/k norm + rotary + KV append fused into the attention,
    gives the same hidden states, KV caches and greedy choices as with the
    separate kernels (hidden 2048, two layers, 40 positions: several tiles
    and splits)."""
    from turbomoe import synth_model as S
    cfg = S.config(**dict(SMALL, hidden_size=2048, num_attention_heads=8, num_key_value_heads=2))
    dec = _decoder(cfg, 21, torch.bfloat16, 64)
    assert dec.fused_norms and dec.fused_rope
    seq = [(5 + 37 * i) % 3000 for i in range(40)]
    got_f = dec.teacher_forced(seq)
    x_f, kv_f = dec.x.clone(), dec.kv.clone()
    dec.fused_norms = False
    dec.fused_rope = False
    dec.reset()
    got_u = dec.teacher_forced(seq)
    torch.cuda.synchronize()
    assert got_f == got_u
    assert torch.equal(dec.x, x_f)
    assert torch.equal(dec.kv, kv_f)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("pos,splits", [(0, 16), (31, 1), (32, 5), (63, 16), (200, 3), (1000, 16)])
def test_qk_rope_attn_decode_same_bits(dt, pos, splits):
    """tm_qk_rope_attn_decode == tm_qk_rope_kv then tm_attn_decode: the same
    output bits and the same appended k/v rows, the position at the start,
    inside and at the end of a 32-row tile and of a split."""
    from turbomoe import ops
    nh, nkv, hd, max_len = 32, 4, 128, 1100
    g = torch.Generator(device="cuda").manual_seed(pos * 3 + splits)
    qkv = torch.randn(1, (nh + 2 * nkv) * hd, generator=g, device="cuda").to(dt)
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")).to(dt)
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")).to(dt)
    from turbomoe.decoder import rope_table
    rope = rope_table(hd, 1e6, max_len, dt).cuda()
    kc0 = torch.randn(nkv, max_len, hd, generator=g, device="cuda").to(dt)
    vc0 = torch.randn(nkv, max_len, hd, generator=g, device="cuda").to(dt)
    p = torch.tensor([pos], device="cuda")
    L = _lib()
    code = ops._code(dt)
    scale = 1.0 / math.sqrt(hd)
    # separate calls
    kc1, vc1 = kc0.clone(), vc0.clone()
    q = torch.empty(1, nh * hd, dtype=dt, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.tm_qk_rope_kv(qkv.data_ptr(), 1, nh, nkv, hd, code, qn.data_ptr(), kn.data_ptr(), 1e-6, rope.data_ptr(),
                           p.data_ptr(), max_len, q.data_ptr(), kc1.data_ptr(), vc1.data_ptr(), st.data_ptr(),
                           _s()) == 0
    ws = torch.zeros(L.tm_attn_decode_workspace_bytes(nh, nkv, splits), dtype=torch.uint8, device="cuda")
    want = torch.empty(nh * hd, dtype=dt, device="cuda")
    assert L.tm_attn_decode(q.data_ptr(), kc1.data_ptr(), vc1.data_ptr(), p.data_ptr(), max_len, nh, nkv, hd, code,
                            scale, splits, want.data_ptr(), ws.data_ptr(), ws.numel(), _s()) == 0
    # fused
    kc2, vc2 = kc0.clone(), vc0.clone()
    got = torch.full((nh * hd,), float("nan"), dtype=dt, device="cuda")
    assert L.tm_qk_rope_attn_decode(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), 1e-6, rope.data_ptr(), p.data_ptr(),
                                    max_len, nh, nkv, hd, code, scale, splits, kc2.data_ptr(), vc2.data_ptr(),
                                    got.data_ptr(), _s()) == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
    assert torch.equal(got, want)
