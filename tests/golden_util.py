"""Loading helpers for the golden fixtures written by tests/golden/make_golden.py."""
import hashlib
import json
import os

import torch
from safetensors.torch import load_file

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def meta():
    with open(os.path.join(GOLDEN, "golden_meta.json")) as f:
        return json.load(f)


def fixture(name):
    return load_file(os.path.join(GOLDEN, f"{name}.safetensors"))


def sha(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def case_layer(name, device="cpu"):
    """(shape, LayerWeights, info) regenerated from the recorded seed; the
    sha256 of every raw tensor is checked against what the reference saw."""
    from turbomoe import synth
    info = meta()["cases"][name]
    shape = synth.MoEShape(*info["shape"])
    lw = synth.make_layer(shape, info["seed"], 0)
    for k, h in info["weights_sha256"].items():
        assert sha(getattr(lw, k)) == h, f"{name}: regenerated {k} differs from the golden run"
    if device != "cpu":
        for k in list(vars(lw)):
            v = getattr(lw, k)
            if v is not None:
                setattr(lw, k, v.to(device))
    return shape, lw, info


def case_x(name, T, fx=None):
    from turbomoe import synth
    info = meta()["cases"][name]
    fx = fx if fx is not None else fixture(name)
    dt = DTYPES[info["dtype"]]
    if f"T{T}.x" in fx:
        return fx[f"T{T}.x"]
    x = synth.make_hidden(T, info["shape"][0], info[f"T{T}.xseed"], rms_normalise=info["rms"],
                          dtype=torch.bfloat16).to(dt)
    assert sha(x) == info[f"T{T}.x_sha256"], f"{name}: regenerated x differs"
    return x
