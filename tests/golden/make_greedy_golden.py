"""Record the reference engine's greedy tokens for the seeded random-init
Qwen3-30B-A3B-FP8 model (the full architecture: 48 layers, 128 experts).

    python tests/golden/make_greedy_golden.py <path to the reference checkout> \
        [--dtype fp32|bf16] [--prompt 16] [--steps 64] [--layers 48] [--seed 2024]

Runs the reference itself on the CPU: its ``ExpertLoader``
(loader/expert_loader.py), ``TurboEngine`` with ``RouterExecutor``,
``MoEExecutor`` and ``LayerExecutor`` (runtime/engine.py:14-21,
execution/layer_executor.py), the ``Qwen3MoeAdapter`` (models/qwen3_moe.py)
over a Hugging Face Qwen3MoeForCausalLM built on the meta device, and the
reference's ``KVCache``.  The generation loop is runtime/engine.py:98-162
without the tokenizer: the prompt is ``--prompt`` token ids drawn uniformly
from the vocabulary with a seeded generator, then ``--steps`` greedy steps
(argmax of the last position's logits).  Writes
``tests/golden/q3_model_greedy_<dtype>.json`` with the prompt, the generated
ids and, per step, the two largest logits (the margin a re-implementation
must resolve to pick the same token).

The weights are ``turbomoe/synth_model.py``'s integer-hash tensors, served by
replacing ``ExpertLoader._get_tensor`` (no 30 GB checkpoint is written); the
generator is pinned by ``table_digest()``, recorded here.  Harness details:
* ``accelerate`` is not installed: a small stand-in provides
  ``init_empty_weights`` (parameters created on the meta device, buffers
  not) and ``utils.set_module_tensor_to_device`` (value cast to the
  parameter's dtype), the two names the reference imports;
* Qwen3 has no shared expert but ``execution/moe.py:53-67`` loads one on every
  call: all-zero bf16 tensors are served for it (an exact no-op);
* ``ExpertLoader`` ignores ``execution.dtype`` (``loader/expert_loader.py:28``
  tests a top-level key), so ``loader.dtype`` is set directly.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import json
import os
import sys
import tempfile
import time
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def load_synth_model():
    spec = importlib.util.spec_from_file_location(
        "tm_synth_model_for_golden", os.path.join(REPO, "turbo-llm_b200", "turbomoe", "synth_model.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def install_accelerate_stand_in():
    acc = types.ModuleType("accelerate")
    utils = types.ModuleType("accelerate.utils")

    @contextlib.contextmanager
    def init_empty_weights(include_buffers=False):
        orig = torch.nn.Module.register_parameter

        def register_parameter(module, name, param):
            orig(module, name, param)
            if param is not None:
                p = module._parameters[name]
                module._parameters[name] = torch.nn.Parameter(p.to("meta"), requires_grad=p.requires_grad)

        torch.nn.Module.register_parameter = register_parameter
        try:
            yield
        finally:
            torch.nn.Module.register_parameter = orig

    def set_module_tensor_to_device(module, tensor_name, device, value=None, dtype=None):
        *path, leaf = tensor_name.split(".")
        for p in path:
            module = getattr(module, p)
        old = getattr(module, leaf)
        if value is None:
            value = old
        value = value.to(dtype if dtype is not None else old.dtype)
        if leaf in module._parameters:
            module._parameters[leaf] = torch.nn.Parameter(value.to(device), requires_grad=False)
        else:
            module._buffers[leaf] = value.to(device)

    acc.init_empty_weights = init_empty_weights
    utils.set_module_tensor_to_device = set_module_tensor_to_device
    acc.utils = utils
    sys.modules["accelerate"] = acc
    sys.modules["accelerate.utils"] = utils


def write_snapshot(path, cfg, specs):
    """config.json + an index naming every tensor (the data never hits disk)."""
    os.makedirs(path, exist_ok=True)
    names = dict(specs)
    H, I = cfg["hidden_size"], cfg["moe_intermediate_size"]
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}.mlp"
        names[f"{p}.shared_expert.gate_proj.weight"] = ((I, H), "zeros")
        names[f"{p}.shared_expert.up_proj.weight"] = ((I, H), "zeros")
        names[f"{p}.shared_expert.down_proj.weight"] = ((H, I), "zeros")
        names[f"{p}.shared_expert_gate.weight"] = ((1, H), "zeros")
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": {n: "synthetic.safetensors" for n in sorted(names)}}, f)
    return names


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("reference")
    ap.add_argument("--dtype", choices=["fp32", "bf16"], default="fp32")
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--out", default=None)
    a = ap.parse_args()

    # transformers first: it probes for accelerate and must find none
    from transformers import AutoConfig, AutoModelForCausalLM                # noqa: E402
    install_accelerate_stand_in()
    sys.path.insert(0, a.reference)
    sys.dont_write_bytecode = True
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    S = load_synth_model()
    from loader.expert_loader import ExpertLoader                           # noqa: E402  (reference)
    from models.qwen3_moe import Qwen3MoeAdapter                            # noqa: E402  (reference)
    from runtime.engine import TurboEngine                                  # noqa: E402  (reference)
    from accelerate import init_empty_weights                              # noqa: E402  (stand-in)

    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}[a.dtype]
    cfg = S.config(num_hidden_layers=a.layers)
    specs = S.tensor_specs(cfg)
    snap = tempfile.mkdtemp(prefix="tm_greedy_")
    names = write_snapshot(snap, cfg, specs)

    def get_tensor(self, name):
        shape, kind = names[name]
        if kind == "zeros":
            return torch.zeros(shape, dtype=torch.bfloat16)
        return S.make_tensor(a.seed, name, (shape, kind), "cpu")

    ExpertLoader._get_tensor = get_tensor
    loader = ExpertLoader(snap)
    loader.dtype = dtype
    hf_config = AutoConfig.from_pretrained(snap)
    with init_empty_weights():
        model = AutoModelForCausalLM.from_config(hf_config, dtype=dtype)
    adapter = Qwen3MoeAdapter(model, loader)
    t0 = time.time()
    engine = TurboEngine(adapter)
    t_build = time.time() - t0

    g = torch.Generator().manual_seed(a.seed + 1)
    prompt = torch.randint(0, cfg["vocab_size"], (1, a.prompt), generator=g)
    P = prompt.shape[1]
    kv_cache = adapter.create_cache(P + a.steps)
    out_ids, top2 = [], []
    next_token_id = None
    t0 = time.time()
    with torch.no_grad():
        # runtime/engine.py:98-162 (greedy, no tokenizer, no collector)
        for step in range(a.steps):
            if step == 0:
                input_to_model = prompt
                position_ids = torch.arange(P).unsqueeze(0)
            else:
                input_to_model = next_token_id.view(1, 1)
                position_ids = torch.tensor([[P + step - 1]])
            hidden_states = adapter.embed(input_to_model)
            position_embeddings = adapter.rotary_embeddings(hidden_states, position_ids)
            causal_mask = adapter.create_attention_mask(hidden=hidden_states, kv_cache=kv_cache,
                                                        position_ids=position_ids)
            for layer_id in range(adapter.num_layers):
                hidden_states, _ = engine.layer.execute_layer(
                    layer_id=layer_id, hidden_states=hidden_states, attention_mask=causal_mask,
                    position_ids=position_ids, position_embeddings=position_embeddings, kv_cache=kv_cache)
            hidden_states = adapter.final_norm(hidden_states)
            logits = adapter.lm_head(hidden_states)
            next_token_logits = logits[0, -1, :]
            next_token_id = torch.argmax(next_token_logits, dim=-1)
            v, i = torch.topk(next_token_logits.float(), 2)
            out_ids.append(int(next_token_id))
            top2.append([[int(i[0]), float(v[0])], [int(i[1]), float(v[1])]])
            print(f"step {step}: token {out_ids[-1]} margin {float(v[0] - v[1]):.5f} "
                  f"({time.time() - t0:.0f} s)", flush=True)
    import transformers
    rec = {"what": "greedy tokens of the reference engine (runtime/engine.py:98-162) on the seeded random-init "
                   "Qwen3-30B-A3B-FP8 model, CPU",
           "dtype": a.dtype, "seed": a.seed, "layers": a.layers, "prompt_len": P, "steps": a.steps,
           "prompt": prompt[0].tolist(), "tokens": out_ids, "top2": top2,
           "table_digest": S.table_digest(), "torch": torch.__version__, "transformers": transformers.__version__,
           "attn_implementation": getattr(hf_config, "_attn_implementation", None),
           "build_s": round(t_build, 1), "generate_s": round(time.time() - t0, 1)}
    out = a.out or os.path.join(HERE, f"q3_model_greedy_{a.dtype}.json")
    with open(out, "w") as f:
        json.dump(rec, f, indent=1)
    print("wrote", out)


if __name__ == "__main__":
    main()
