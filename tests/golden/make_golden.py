"""Generate the golden fixtures by running the REFERENCE itself.

Run where a checkout of the reference is available, giving its path:

    python tests/golden/make_golden.py <path to the reference checkout>

It writes seeded synthetic FP8 checkpoints to a temporary directory, imports
the reference's ``ExpertLoader`` (loader/expert_loader.py), ``RouterExecutor``
(execution/router.py) and ``MoEExecutor`` (execution/moe.py), runs them on
the CPU, and stores inputs and outputs under ``tests/golden/*.safetensors``.
Weights are not stored: they are regenerated from the recorded seed by
``turbomoe/synth.py``; a sha256 of every raw weight tensor is stored so a
test can prove the regenerated weights are the ones the reference saw.

Notes on how the reference is driven (all CPU, act dtype as recorded):
* Qwen3-shaped layers get an all-zero bf16 shared expert because
  ``execution/moe.py:53-67`` loads one unconditionally (exact no-op).
* ``ExpertLoader`` ignores ``execution.dtype`` (it tests a top-level key,
  ``loader/expert_loader.py:28``), so ``loader.dtype`` is set directly.
* Layers with an FP8 shared expert run in fp32: on the CPU
  ``load_weight`` casts FP8 to fp16 (``loader/expert_loader.py:102-106``)
  and the bf16 path then fails in ``F.linear``.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import tempfile

import torch
from safetensors.torch import save_file

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def load_synth():
    spec = importlib.util.spec_from_file_location(
        "tm_synth_for_golden", os.path.join(REPO, "turbo-llm_b200", "turbomoe", "synth.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def weight_hashes(lw):
    out = {}
    for name in ("router", "gate", "gate_s", "up", "up_s", "down", "down_s",
                 "sh_gate", "sh_gate_s", "sh_up", "sh_up_s", "sh_down", "sh_down_s", "sh_router"):
        v = getattr(lw, name)
        if v is not None:
            out[name] = sha(v)
    return out


DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    sys.dont_write_bytecode = True
    from loader.expert_loader import ExpertLoader          # noqa: E402  (reference)
    from execution.router import RouterExecutor            # noqa: E402  (reference)
    from execution.moe import MoEExecutor                  # noqa: E402  (reference)
    synth = load_synth()
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    meta = {"torch": torch.__version__, "cases": {}}
    tmp = tempfile.mkdtemp(prefix="tm_golden_")

    # ---------------- dequant (loader/expert_loader.py:127-160) ----------------
    ck = synth.write_checkpoint(os.path.join(tmp, "dq"), synth.MoEShape(512, 256, 2, 2, 0), seed=11)
    L = ExpertLoader(ck)
    t = {}
    for mname in ("gate_proj", "down_proj"):
        w, s = L.load_weight_raw(f"model.layers.0.mlp.experts.1.{mname}.weight")
        w, s = w[:128].contiguous(), s[:1].contiguous()   # first 128-row block keeps the fixture small
        t[f"{mname}.w"] = w.view(torch.uint8).clone()
        t[f"{mname}.s"] = s.clone()
        for dn, dt in DTYPES.items():
            t[f"{mname}.out_{dn}"] = L.dequantize_weight(w, s, dtype=dt).contiguous()
    # every e4m3 bit pattern, 128 x 256 (one pattern per column of a row, shifted per row)
    rows = torch.arange(128).view(128, 1)
    cols = torch.arange(256).view(1, 256)
    allbits = ((rows * 7 + cols) % 256).to(torch.uint8)
    g = torch.Generator().manual_seed(5)
    sc = torch.rand(1, 2, generator=g) * 1e-3 + 1e-5
    t["allbits.w"] = allbits
    t["allbits.s"] = sc
    for dn, dt in DTYPES.items():
        t[f"allbits.out_{dn}"] = L.dequantize_weight(allbits.view(torch.float8_e4m3fn), sc, dtype=dt).contiguous()
    save_file(t, os.path.join(HERE, "dequant.safetensors"))
    meta["cases"]["dequant"] = {"seed": 11, "shape": [512, 256, 2, 2, 0]}

    # ---------------- router + layer cases ----------------
    cases = [
        # name, shape(H, I, E, k, Is), seed, act dtype, token counts, rms-normalise x
        ("q3_small", (512, 256, 32, 8, 0), 21, "bf16", (1, 5, 64), False),
        ("q3_small_fp16", (512, 256, 32, 8, 0), 22, "fp16", (1, 33), False),
        ("q35_small", (512, 256, 64, 8, 256), 23, "fp32", (1, 64), False),
        ("q3_c0", (2048, 768, 128, 8, 0), 1, "bf16", (1,), True),
        ("q3_c1", (2048, 768, 128, 8, 0), 1, "bf16", (2048,), False),
        ("q35_c3", (2048, 512, 256, 8, 512), 3, "fp32", (64,), False),
    ]
    for name, shp, seed, dn, tcounts, rms in cases:
        shape = synth.MoEShape(*shp)
        dt = DTYPES[dn]
        ck = synth.write_checkpoint(os.path.join(tmp, name), shape, seed=seed)
        lw = synth.make_layer(shape, seed, 0)
        L = ExpertLoader(ck)
        L.dtype = dt
        R = RouterExecutor(L, 1, top_k=shape.top_k)
        M = MoEExecutor(L)
        tens = {}
        info = {"shape": list(shp), "seed": seed, "dtype": dn, "tokens": list(tcounts),
                "rms": rms, "weights_sha256": weight_hashes(lw)}
        for T in tcounts:
            xseed = seed * 100 + T
            x = synth.make_hidden(T, shape.hidden, xseed, rms_normalise=rms, dtype=torch.bfloat16).to(dt)
            logits = torch.nn.functional.linear(x, R.routers[0])
            idx, w = R.compute_routing(0, x)
            y = M.execute_layer(0, x, idx, w)
            big = T * shape.hidden > 64 * 2048
            small_x = T * shape.hidden <= 64 * 512
            tens[f"T{T}.idx"] = idx.to(torch.int16 if shape.experts < 32768 else torch.int32).contiguous()
            tens[f"T{T}.w"] = w.contiguous()
            if big:
                # keep fixtures small: every 32nd row of logits / outputs + hashes of the rest
                rows = torch.arange(0, T, 32)
                tens[f"T{T}.rows"] = rows
                tens[f"T{T}.logits_rows"] = logits[rows].contiguous()
                tens[f"T{T}.y_rows"] = y[rows].contiguous()
                info[f"T{T}.x_sha256"] = sha(x)
            else:
                if small_x:
                    tens[f"T{T}.x"] = x.contiguous()
                else:
                    info[f"T{T}.x_sha256"] = sha(x)
                tens[f"T{T}.logits"] = logits.contiguous()
                tens[f"T{T}.y"] = y.contiguous()
            info[f"T{T}.xseed"] = xseed
            print(f"{name} T={T}: |y|max {y.float().abs().max().item():.4f}", flush=True)
        save_file(tens, os.path.join(HERE, f"{name}.safetensors"))
        meta["cases"][name] = info
        del L, R, M
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
