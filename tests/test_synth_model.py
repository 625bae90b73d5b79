"""The seeded random-init Qwen3-30B-A3B-FP8 generator (turbomoe/synth_model.py):
pinned tables, values independent of how a tensor is chunked, the weight
statistics the workload asks for (N(0, 0.02) after dequantisation), the
checkpoint names the reference's ModelLayout expects, and agreement with the
generator the greedy-token fixtures were recorded with."""
import json
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))

TABLE_DIGEST = "ff3d9967285f2a0c6caafd8492ba81bd1feab82b888427dcb57b71b2ebba8a20"


def test_tables_are_pinned():
    from turbomoe import synth_model as S
    assert S.table_digest() == TABLE_DIGEST
    for name in ("q3_model_greedy_fp32.json", "q3_model_greedy_bf16.json"):
        p = os.path.join(HERE, "golden", name)
        if os.path.exists(p):
            with open(p) as f:
                assert json.load(f)["table_digest"] == TABLE_DIGEST, name


def test_values_do_not_depend_on_chunking():
    from turbomoe import synth_model as S
    name = "model.layers.3.mlp.experts.7.down_proj.weight"
    a = S.fp8_codes(5, name, (2048, 768))
    b = S.fp8_codes(5, name, (2048, 768), chunk=1 << 17)
    assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    c = S.bf16_normal(5, "lm_head.weight", (1000, 256))
    d = S.bf16_normal(5, "lm_head.weight", (1000, 256), chunk=4093)
    assert torch.equal(c.view(torch.int16), d.view(torch.int16))
    # another name or seed gives other values
    e = S.fp8_codes(6, name, (2048, 768))
    assert not torch.equal(a.view(torch.uint8), e.view(torch.uint8))


def test_weight_statistics():
    from turbomoe import synth_model as S
    name = "model.layers.0.self_attn.q_proj.weight"
    q = S.fp8_codes(1, name, (4096, 2048))
    s = S.block_scales(1, name, (4096, 2048))
    assert s.shape == (32, 16) and bool((s >= 176 * 2.0 ** -20).all()) and bool((s <= 191 * 2.0 ** -20).all())
    w = (q.float().view(32, 128, 16, 128) * s.view(32, 1, 16, 1)).reshape(4096, 2048)
    assert abs(float(w.std()) - 0.02) < 1e-3 and abs(float(w.mean())) < 1e-4
    assert float(q.float().abs().max()) <= 448.0
    r = S.bf16_normal(1, "model.layers.0.mlp.gate.weight", (128, 2048))
    assert abs(float(r.float().std()) - 0.02) < 1e-3


def test_checkpoint_names_match_the_layout():
    from loader.expert_loader import ExpertLoader
    from turbomoe import synth_model as S
    cfg = S.config(num_hidden_layers=2)
    src = S.ModelSource(cfg, 1, "cpu")
    L = ExpertLoader(None, config={"execution": {"dtype": "bf16"}}, source=src)
    assert L.num_layers == 2 and L.num_experts == 128
    assert L.layout.router_tensor(1) == "model.layers.1.mlp.gate.weight"
    assert L.layout.gate_tensor(1, 5) == "model.layers.1.mlp.experts.5.gate_proj.weight"
    specs = S.tensor_specs(cfg)
    assert specs["model.layers.1.self_attn.o_proj.weight"] == ((2048, 4096), "fp8")
    assert specs["model.layers.1.self_attn.o_proj.weight_scale_inv"] == ((16, 32), "scale")
    assert specs["lm_head.weight"] == ((151936, 2048), "bf16")
    t = src.get("model.layers.1.self_attn.k_norm.weight")
    assert t.dtype == torch.bfloat16 and bool((t == 1).all())
