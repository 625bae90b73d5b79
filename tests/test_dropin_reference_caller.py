"""The drop-in under the reference's own caller (CPU, in a container that has
a checkout of the reference; skipped elsewhere).

With ``turbo-llm_b200`` ahead of the reference checkout on the path:
* ``execution.router``, ``execution.moe``, ``loader.expert_loader``,
  ``loader.model_layout`` and ``cache.ram_cache`` resolve to the drop-in, while
  the reference's other modules of those packages (``execution.layer_executor``,
  ``cache.kv_cache``) and its ``runtime.engine`` still import from the checkout;
* every call the reference's engine and layer executor make into the swapped
  classes (runtime/engine.py:14-21, execution/layer_executor.py:108-213,
  phase2_generate.py:24) binds to the drop-in's signatures, and every loader
  attribute they read exists.

The calls are found by parsing the reference's source, so a change of the
reference's call sites shows up here.  Device numerics of the same loop are
checked on the GPU (tests/test_gpu_decoder.py, tests/test_gpu_greedy.py).
"""
import ast
import inspect
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "turbo-llm_b200")
# the reference checkout: TURBO_LLM_REFERENCE, else a directory `reference` beside this repository
REF = os.environ.get("TURBO_LLM_REFERENCE", os.path.join(os.path.dirname(REPO), "reference"))

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "execution")),
                                reason="no reference checkout")

RESOLVE = r"""
import importlib.util as u, json, sys
sys.path[:0] = [sys.argv[1], sys.argv[2]]
out = {m: u.find_spec(m).origin for m in sys.argv[3:]}
print(json.dumps(out))
"""


def test_module_resolution():
    mods = ["execution.router", "execution.moe", "execution.layer_executor", "loader.expert_loader",
            "loader.model_layout", "cache.ram_cache", "cache.kv_cache", "runtime.engine", "models.qwen3_moe"]
    r = subprocess.run([sys.executable, "-c", RESOLVE, PKG, REF, *mods], capture_output=True, text=True, check=True)
    import json
    got = json.loads(r.stdout)
    ours = {"execution.router", "execution.moe", "loader.expert_loader", "loader.model_layout", "cache.ram_cache"}
    for m, path in got.items():
        want_root = PKG if m in ours else REF
        assert path.startswith(want_root + os.sep), (m, path)


def _calls(path, attr):
    """(positional count, keyword names) of every call ``<x>.<attr>(...)`` in ``path``."""
    tree = ast.parse(open(path).read())
    out = []
    for n in ast.walk(tree):
        if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute) and n.func.attr == attr:
            out.append((len(n.args), [k.arg for k in n.keywords]))
        elif isinstance(n, ast.Call) and isinstance(n.func, ast.Name) and n.func.id == attr:
            out.append((len(n.args), [k.arg for k in n.keywords]))
    return out


def _bind(fn, npos, kws, bound_method=True):
    sig = inspect.signature(fn)
    args = [object()] * (npos + (1 if bound_method else 0))
    sig.bind(*args, **{k: object() for k in kws})


def test_reference_call_sites_bind_to_the_drop_in():
    sys.path.insert(0, PKG)
    try:
        from execution.moe import MoEExecutor
        from execution.router import RouterExecutor
        from loader.expert_loader import ExpertLoader
    finally:
        sys.path.remove(PKG)
    le = os.path.join(REF, "execution", "layer_executor.py")
    eng = os.path.join(REF, "runtime", "engine.py")
    gen = os.path.join(REF, "phase2_generate.py")
    checks = [
        (le, "compute_routing", RouterExecutor.compute_routing),
        (le, "execute_layer", MoEExecutor.execute_layer),
        (le, "load_weight", ExpertLoader.load_weight),
        (eng, "RouterExecutor", RouterExecutor.__init__),
        (eng, "MoEExecutor", MoEExecutor.__init__),
        (gen, "ExpertLoader", ExpertLoader.__init__),
    ]
    for path, name, fn in checks:
        sites = _calls(path, name)
        assert sites, (path, name)
        for npos, kws in sites:
            _bind(fn, npos, kws)
    # every loader / layout attribute the engine and the layer executor read
    import re
    src = open(le).read() + open(eng).read()
    loader = ExpertLoader(None, source=_TinySource())
    names = set(re.findall(r"self\.loader\.([A-Za-z_]\w*)", src))
    assert {"DEVICE", "load_weight", "load_ms_accum", "gpu_hits", "snapshot_path"} <= names
    for a in names:
        assert hasattr(loader, a), a
    for a in set(re.findall(r"self\.loader\.layout\.([A-Za-z_]\w*)", src)):
        assert hasattr(loader.layout, a), a
    assert "last_gemm_ms" in dir(MoEExecutor)
    # what the layer executor reads of the MoE executor (last_gemm_ms)
    assert set(re.findall(r"self\.moe_exec\.([A-Za-z_]\w*)", src)) <= set(dir(MoEExecutor))


class _TinySource:
    """Smallest tensor source an ExpertLoader accepts (names only)."""
    weight_map = {"model.layers.0.mlp.experts.0.gate_proj.weight": "x", "model.layers.0.mlp.gate.weight": "x"}
    config = {"model_type": "qwen3_moe", "num_experts": 1, "num_hidden_layers": 1, "num_experts_per_tok": 1}

    def has(self, name):
        return name in self.weight_map

    def close(self):
        pass


LINEAR_ATTN = r"""
import copy, json, sys
import torch
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import cache.qwen35_cache as qc
from turbomoe import linear_attn
from turbomoe._lib import TurboMoEError
from transformers import Qwen3_5MoeTextConfig
from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
cfg = Qwen3_5MoeTextConfig(hidden_size=256, linear_num_key_heads=1, linear_num_value_heads=2,
                           linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4)
torch.manual_seed(0)
ref = M.Qwen3_5MoeGatedDeltaNet(cfg, layer_idx=0).eval()
mod = copy.deepcopy(ref)
linear_attn.install(mod)
ca, cb = qc.Qwen35Cache(num_layers=1), qc.Qwen35Cache(num_layers=1)
x = torch.randn(1, 4, 256)
out = {"cache_module": qc.__file__}
with torch.no_grad():
    ya = ref(hidden_states=x, cache_params=ca, attention_mask=None)
    yb = mod(hidden_states=x, cache_params=cb, attention_mask=None)
    out["prompt_equal"] = bool(torch.equal(ya, yb))
    out["state_equal"] = bool(torch.equal(ca.layers[0].recurrent_states, cb.layers[0].recurrent_states))
    try:
        mod(hidden_states=x[:, :1], cache_params=cb, attention_mask=None)
        out["decode"] = "ran"
    except TurboMoEError as e:
        out["decode"] = str(e)
print(json.dumps(out))
"""


def test_linear_attention_call_site_with_the_reference_cache():
    """execution/layer_executor.py:134-139 calls ``layer_module.linear_attn(
    hidden_states=..., cache_params=kv_cache, attention_mask=...)`` with the
    reference's Qwen35Cache.  After ``turbomoe.linear_attn.install`` the call
    site binds, the prompt runs the module's own forward with that cache (same
    outputs and states as the unmodified module), and a decode step goes to
    tm_gdn_decode, which on the CPU refuses (no CPU fallback)."""
    sites = _calls(os.path.join(REF, "execution", "layer_executor.py"), "linear_attn")
    assert sites and all(npos == 0 and set(kws) == {"hidden_states", "cache_params", "attention_mask"}
                         for npos, kws in sites), sites
    r = subprocess.run([sys.executable, "-c", LINEAR_ATTN, PKG, REF], capture_output=True, text=True, check=True,
                       timeout=600)
    import json
    got = json.loads(r.stdout.strip().splitlines()[-1])
    assert got["cache_module"].startswith(REF + os.sep), got
    assert got["prompt_equal"] and got["state_equal"], got
    assert "CUDA" in got["decode"], got
