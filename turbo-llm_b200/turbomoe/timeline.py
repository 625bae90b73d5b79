"""Per-CTA timeline of the batch-1 decode step (router, K2, K3 of every
layer) from the trace build of the library.

    python turbo-llm_b200/turbomoe/build.py --trace
    python turbo-llm_b200/turbomoe/timeline.py [--layers 48]

Runs the same step as bench.py (one token through the MoE layers of the
Qwen3-30B-A3B shape, seeded synthetic FP8 weights, one CUDA graph) on
libturbomoe_trace.so, whose kernels record per CTA (event, globaltimer,
clock64) marks into the workspace.  Prints, per kernel and event, the (min,
median, max over CTAs) time after the layer's router passed its dependency
wait (x ready), median over the middle layers; and the SM clock (cycles per
ns) between consecutive marks of one CTA, which separates slow clocks from
long dependency chains.  Events: 0 enter, 1 dependency wait passed, 2 data
(weights or x) landed, 3 exit / logits gathered (router CTA 0), 4 MMAs or dot
product done, 6 plan written, 7 dot product reduced.  The trace build's
marks cost a few tens of nanoseconds each; its step time is printed beside.
"""
import argparse
import ctypes as C
import os
import sys

import numpy as np

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))  # turbo-llm_b200/
if PKG_ROOT not in sys.path:
    sys.path.insert(0, PKG_ROOT)
import torch  # noqa: E402

ap = argparse.ArgumentParser()
ap.add_argument("--lib", default=None, help="trace build of the library (default: turbomoe/libturbomoe_trace.so)")
ap.add_argument("--layers", type=int, default=48)
args = ap.parse_args()

import turbomoe._lib as TL  # noqa: E402
from turbomoe import build as B  # noqa: E402
TL.LIB_PATH = args.lib or B.TRACE_LIB
if not os.path.exists(TL.LIB_PATH):
    raise SystemExit(f"{TL.LIB_PATH} is missing: build it with `python turbo-llm_b200/turbomoe/build.py --trace`")
lib = TL.lib()
if not hasattr(lib, "tm_trace_offset"):
    raise SystemExit(f"{TL.LIB_PATH} is not a trace build")
lib.tm_trace_offset.restype = C.c_int64
OFF = lib.tm_trace_offset()
CAP = 1 << 20

from execution.moe import MoEExecutor  # noqa: E402
from execution.router import RouterExecutor  # noqa: E402
from loader.expert_loader import ExpertLoader  # noqa: E402
from turbomoe import synth  # noqa: E402

LAYERS = args.layers
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
shape = synth.QWEN3_30B_A3B
loader = ExpertLoader.synthetic(shape, seed=1234, num_layers=LAYERS, dtype=torch.bfloat16, device=dev)
loader.upload()
router = RouterExecutor(loader, LAYERS)
moe = MoEExecutor(loader, record_timing=False)
ws = loader.workspace(dev)
ws.ensure(1)
x0 = synth.make_hidden(1, shape.hidden, 1241, rms_normalise=True, device=dev)


def step(x):
    for l in range(LAYERS):
        idx, w = router.compute_routing(l, x)
        x = moe.execute_layer(l, x, idx, w, residual=x)
    return x


s = torch.cuda.Stream(device=dev)
s.wait_stream(torch.cuda.current_stream())
with torch.cuda.stream(s):
    for _ in range(2):
        step(x0)
torch.cuda.current_stream().wait_stream(s)
g = torch.cuda.CUDAGraph()
with torch.cuda.graph(g):
    y = step(x0)
for _ in range(5):
    g.replay()
torch.cuda.synchronize()
e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
e0.record()
for _ in range(10):
    g.replay()
e1.record()
torch.cuda.synchronize()
print(f"trace build: {e0.elapsed_time(e1) / 10 * 1000 / LAYERS:.2f} us per layer (graph)")
buf = ws.buf
buf[OFF:OFF + 16 + 16 * CAP].zero_()
g.replay()
torch.cuda.synchronize()
n = min(int(buf[OFF:OFF + 4].view(torch.int32).item()), CAP)
ev = buf[OFF + 16:OFF + 16 + 16 * n].view(torch.int64).reshape(n, 2).cpu().numpy().astype(np.uint64)
nres = n // 16
blk = ev[:nres * 16].reshape(nres, 8, 2, 2)      # [reservation][event][time|clock][header, value]
hdr = blk[:, :, 0, 0]
present = hdr != 0
kidm = (hdr >> np.uint64(56)).astype(int)
ctam = (hdr & np.uint64(0xffffffffffff)).astype(int)
tim = blk[:, :, 0, 1].astype(np.int64)
clk = blk[:, :, 1, 1].astype(np.int64)
t0g = tim[present].min()
rows_ = []
for r in range(nres):
    evs = np.flatnonzero(present[r])
    if len(evs) == 0:
        continue
    rows_.append((kidm[r, evs[0]], ctam[r, evs[0]], {int(e): (int(tim[r, e] - t0g), int(clk[r, e])) for e in evs}))
print(f"{len(rows_)} CTA records")
NAMES = {1: "router", 2: "k2", 3: "k3", 4: "k3t1", 5: "plan"}
EVN = {0: "enter", 1: "waited", 2: "data", 3: "exit", 4: "mark4", 5: "mark5", 6: "done", 7: "mark7"}
by = {}
for k, c, d in rows_:
    by.setdefault((k, c), []).append(d)
launch = {}
for (k, c), lst in by.items():
    lst.sort(key=lambda d: min(v[0] for v in d.values()))
    for j, d in enumerate(lst):
        launch.setdefault((k, j), []).append(d)
L = max(j for (k, j) in launch if k == 1) + 1
base = [min(d[1][0] for d in launch[(1, j)] if 1 in d) for j in range(L)]
mid = range(4, L - 4) if L > 12 else range(L)
print(f"layers: {L}")
print(f"{'kernel':8s} {'event':6s} {'min':>8s} {'med':>8s} {'max':>8s}   (us after router waited, median over layers)")
for k in sorted({k for (k, j) in launch}):
    for e in range(8):
        vals = []
        for j in mid:
            ts = [d[e][0] for d in launch.get((k, j), []) if e in d]
            if ts:
                vals.append((min(ts) - base[j], np.median(ts) - base[j], max(ts) - base[j]))
        if len(vals) < len(mid) // 2:
            continue
        v = np.median(np.array(vals), axis=0) / 1e3
        print(f"{NAMES.get(k, k):8s} {EVN.get(e, e):6s} {v[0]:8.2f} {v[1]:8.2f} {v[2]:8.2f}")
print("SM clock between consecutive marks of one CTA (MHz = cycles / ns * 1000), median:")
for k in sorted({k for (k, j) in launch}):
    ph = {}
    for j in mid:
        for d in launch.get((k, j), []):
            es = sorted(d)
            for a_, b_ in zip(es, es[1:]):
                dt = d[b_][0] - d[a_][0]
                dc = d[b_][1] - d[a_][1]
                if dt > 50:
                    ph.setdefault((a_, b_), []).append((dc / dt * 1000, dt, dc))
    for (a_, b_), v in sorted(ph.items()):
        v = np.array(v)
        print(f"  {NAMES.get(k, k):8s} {EVN.get(a_, a_)}->{EVN.get(b_, b_)}: {np.median(v[:, 0]):7.0f} MHz  "
              f"{np.median(v[:, 1]) / 1e3:6.2f} us  {np.median(v[:, 2]):8.0f} cycles  (n={len(v)})")
period = np.median(np.diff(base)[list(mid)[:-1]]) / 1e3
print(f"layer period (router waited -> next router waited): {period:.2f} us")
