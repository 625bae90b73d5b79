"""Greedy tokens of the full random-init Qwen3-30B-A3B-FP8 model (48 layers,
128 experts, vocab 151936) against the reference engine's own tokens.

The fixtures ``tests/golden/q3_model_greedy_<dtype>.json`` were recorded by
``tests/golden/make_greedy_golden.py``, which runs the reference's
TurboEngine / LayerExecutor / RouterExecutor / MoEExecutor / ExpertLoader on
the CPU over the same seeded weights (``turbomoe/synth_model.py``, pinned by
its table digest).  Here the drop-in runs the same loop on the GPU through
``turbomoe.decoder.Qwen3MoeDecoder`` (one CUDA graph per step):

* fp32 activations: every one of the recorded greedy tokens must be identical
  (the reference's fp32 path and ours differ only in the order of sums);
* bf16 activations (the product dtype), fed the fp32 reference's sequence
  (teacher forcing): the greedy choice must agree wherever the reference's
  top-2 logit margin exceeds the resolution of bf16 logits (4 ulps of the top
  logit), and agree on at least 90 % of all positions.
"""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "q3_model_greedy_fp32.json")


def _golden():
    if not os.path.exists(FIXTURE):
        pytest.skip("greedy-token fixture not recorded")
    with open(FIXTURE) as f:
        return json.load(f)


def _decoder(g, dtype):
    from loader.expert_loader import ExpertLoader
    from turbomoe import synth_model as S
    from turbomoe.decoder import Qwen3MoeDecoder
    assert S.table_digest() == g["table_digest"]
    cfg = S.config(num_hidden_layers=g["layers"])
    dn = {torch.float32: "fp32", torch.bfloat16: "bf16"}[dtype]
    L = ExpertLoader(None, config={"execution": {"dtype": dn}}, source=S.ModelSource(cfg, g["seed"], "cuda"))
    dec = Qwen3MoeDecoder(L, cfg, max_len=g["prompt_len"] + g["steps"] + 8)
    dec.capture()
    return dec


def test_greedy_tokens_fp32_identical_to_reference():
    g = _golden()
    dec = _decoder(g, torch.float32)
    got = dec.generate(g["prompt"], g["steps"])
    first = next((i for i, (a, b) in enumerate(zip(got, g["tokens"])) if a != b), None)
    assert got == g["tokens"], f"first difference at step {first}: {got[first]} vs {g['tokens'][first]}"


def test_greedy_tokens_bf16_teacher_forced():
    g = _golden()
    dec = _decoder(g, torch.bfloat16)
    seq = g["prompt"] + g["tokens"]
    got = dec.teacher_forced(seq[:-1])
    P = g["prompt_len"]
    eps = torch.finfo(torch.bfloat16).eps
    agree, resolvable = 0, 0
    for j, ((i0, v0), (_i1, v1)) in enumerate(g["top2"]):
        pred = got[P - 1 + j]
        agree += pred == i0
        if v0 - v1 > 4 * abs(v0) * eps:
            resolvable += 1
            assert pred == i0, (j, pred, i0, v0 - v1)
    assert agree >= 0.9 * len(g["tokens"]), (agree, len(g["tokens"]))
    assert resolvable >= len(g["tokens"]) // 2
