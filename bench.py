"""Benchmark: batch-1 decode through the 48 MoE layers of Qwen3-30B-A3B-FP8.

One step = one token through all 48 MoE layers of the model (router + FP8
expert FFN per layer, chained by the residual: x_{l+1} = x_l + moe_l(x_l)),
with every expert of every layer resident in HBM (29 GB of packed FP8).
Attention, norms and the LM head are outside the MoE hot path and not run.
Weights are seeded synthetic N(0, 0.02) (no checkpoint exists here); the
token's hidden state is bf16 N(0,1), RMS-normalised.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Our arm: ``value`` = tokens/s from CUDA events around K replays of a CUDA
graph of the step (max over ranks; N>1 runs independent replicas: the decode
config does not shard).  ``e2e`` = the same step through the public API
(RouterExecutor.compute_routing + MoEExecutor.execute_layer) including the
H2D copy of the token's hidden state from pinned memory and the D2H read of
the result every step.  ``roofline`` covers the dominant kernel (K2, gate+up),
timed on its own stream with CUDA events.  The weights read per step (1.8 GB)
are ~15x the 126 MB L2, so no L2 flush is needed between steps.

Reference arm (``--impl reference``): the oracle port of the reference's CPU
path (oracle/moe_oracle.py, torch CPU ops in the reference's order and dtypes)
on the host cores, warm (experts already dequantised, the reference's best
case), on a bounded sample (a subset of distinct layers cycled through the 48).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "turbo-llm_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "decode tok/s (bs=1) Qwen3-30B-A3B-FP8 MoE layers"
LAYERS = 48
SEED = 1234
# algorithmic bytes, one layer-token (T=1, E=128, k=8, H=2048, I=768)
EXPERT_BYTES = 3 * 768 * 2048                      # 4,718,592 B FP8 per expert
# K2 (tm_moe_decode_gateup_prefetch) reads its own operands (gate/up weights +
# scales + x, writes h) and pulls the 8 experts' down projections into L2 for K3
K2_OWN_BYTES = 8 * 2 * 768 * 2048 + 8 * 2 * 6 * 16 * 4 + 2048 * 2 + 8 * 768 * 4   # 25,200,640
K2_BYTES = K2_OWN_BYTES + 8 * 2048 * 768                                         # + 12,582,912 down
LAYER_BYTES = 8 * EXPERT_BYTES + 8 * 288 * 4 + 128 * 2048 * 2 + 2 * 2048 * 2  # 38.29 MB
# dram__bytes_read.sum + dram__bytes_write.sum of one K2 launch of this
# workload, read from an ncu capture (not measured by this script: ncu replays
# kernels, so it cannot run inside a timed bench)
K2_TRAFFIC = 37789440
K2_TRAFFIC_SOURCE = ("ncu --set full capture of k2_gateup_f8<bf16, 8, 8> in this workload (4-layer decode step, "
                     "dram__bytes_read.sum + dram__bytes_write.sum of one launch: 37,789,440 + 0 B)")


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons polled through NVML every 5 ms while the
    timed region runs (a background thread; read-only queries)."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = None
        self._thread = None

    def _handle(self):
        import pynvml
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.gpu_index)
        bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
        try:  # CUDA ordinals need not match NVML's: find the device by PCI bus id
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.gpu_index)

    def _run(self, h):
        import pynvml
        while not self._stop.is_set():
            try:
                self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.005)

    def __enter__(self):
        import threading
        try:
            import pynvml
            h = self._handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._run, args=(h,), daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(n):
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------- our arm ----
def run_ours(args, rank, world, local):
    LAYERS = args.layers
    from execution.moe import MoEExecutor
    from execution.router import RouterExecutor
    from loader.expert_loader import ExpertLoader
    from turbomoe import ops, synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shape = synth.QWEN3_30B_A3B
    loader = ExpertLoader.synthetic(shape, seed=SEED, num_layers=LAYERS, dtype=torch.bfloat16, device=dev)
    t0 = time.time()
    loader.upload()
    upload_s = time.time() - t0
    # opt-in: speculative L2 prefetch of each next layer's experts (slower as it stands)
    use_pf = args.tokens <= 8 and args.next_layer_prefetch
    router = RouterExecutor(loader, LAYERS, prefetch_next_layer=use_pf, prefetch_join_every=args.prefetch_join_every)
    moe = MoEExecutor(loader, record_timing=False)
    ws = loader.workspace(dev)
    ws.ensure(args.tokens)
    x0 = synth.make_hidden(args.tokens, shape.hidden, SEED + 7, rms_normalise=True, device=dev)

    def step(x):
        for l in range(LAYERS):
            idx, w = router.compute_routing(l, x)
            x = moe.execute_layer(l, x, idx, w, residual=x)
        return x

    x_in = x0.clone()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step(x_in)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        x_out = step(x_in)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    ms_per_step = ms / args.steps
    value = world * args.tokens * args.steps / (ms / 1000.0)
    assert torch.isfinite(x_out.float()).all(), "non-finite output"

    # the same step without the next-layer prefetch (same outputs, bit for bit)
    next_layer_prefetch = None
    if use_pf:
        router_plain = RouterExecutor(loader, LAYERS)

        def step_plain(x):
            for l in range(LAYERS):
                idx, w = router_plain.compute_routing(l, x)
                x = moe.execute_layer(l, x, idx, w, residual=x)
            return x

        graph_p = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_p):
            x_out_p = step_plain(x_in)
        for _ in range(args.warmup):
            graph_p.replay()
        torch.cuda.synchronize()
        barrier(world)
        ev0.record()
        for _ in range(args.steps):
            graph_p.replay()
        ev1.record()
        torch.cuda.synchronize()
        ms_p = max_over_ranks(ev0.elapsed_time(ev1), world)
        graph.replay()
        torch.cuda.synchronize()
        next_layer_prefetch = {
            "what": "layer l+1's router applied to layer l's input on a side stream names the experts whose "
                    "gate/up weights are bulk-prefetched into L2 (tm_prefetch_experts_l2) while HBM is idle; "
                    "a hint only",
            "value_without": round(world * args.tokens * args.steps / (ms_p / 1000.0), 2),
            "ms_per_step_without": round(ms_p / args.steps, 4),
            "same_output_bits": bool(torch.equal(x_out, x_out_p)),
            "join_every": args.prefetch_join_every,
        }
        del graph_p

    # ---- e2e: public API, host buffers, H2D + D2H inside the timed region ----
    x_host = x0.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x0)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        y_dev = step(x_dev)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        g2.replay()
        y_host.copy_(y_dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def e2e_eager():
        x = x_host.to(dev, non_blocking=True)
        y = step(x)
        y_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for f in (e2e_step, e2e_eager):
        for _ in range(args.warmup):
            f()
    barrier(world)
    t = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t, world)
    barrier(world)
    t = time.perf_counter()
    for _ in range(args.steps):
        e2e_eager()
    eager_s = max_over_ranks(time.perf_counter() - t, world)

    # ---- dominant kernel (K2): its marginal device time inside CUDA graphs ----
    # Graph A runs, per layer, the plan kernel for that layer's stored top-k then
    # K2; graph B runs the plan kernels alone; graph C adds K3.  Each graph is
    # timed with CUDA events over R replays on the capturing stream:
    # K2 = (A - B) / launches, K3 = (C - A) / launches.
    pls = [loader.packed_layer(l) for l in range(LAYERS)]
    xs = [x0.clone()]
    for l in range(LAYERS):
        idx, w = router.compute_routing(l, xs[-1])
        xs.append(moe.execute_layer(l, xs[-1], idx, w, residual=xs[-1]))
    routes = [router.compute_routing(l, xs[l]) for l in range(LAYERS)]
    out = torch.empty_like(x0)
    torch.cuda.synchronize()
    if next_layer_prefetch is not None and LAYERS > 1:
        # share of the experts each layer routes to that the prediction from the previous layer's input named
        pws = ops.Workspace(dev, 128, 8, shape.hidden, shape.inter, 0)
        pws.ensure(args.tokens)
        hits = total = 0
        for l in range(LAYERS - 1):
            pred, _ = ops.router_topk(xs[l], router.routers[l + 1], 8, pws)
            act = routes[l + 1][0]
            for t in range(args.tokens):
                hits += len(set(pred[t].tolist()) & set(act[t].tolist()))
                total += act.shape[1]
        next_layer_prefetch["hit_rate"] = round(hits / max(total, 1), 4)

    def run_parts(with_k2, with_k3):
        for l in range(LAYERS):
            idx, w = routes[l]
            ops.route_plan(idx, 128, ws)
            if with_k2:
                ops.moe_gateup(xs[l], 8, pls[l].experts, ws, prefetch_down=True)
            if with_k3:
                ops.moe_down_combine(w, pls[l].experts, ws, out, residual=xs[l])

    def graph_time(with_k2, with_k3, reps):
        s2 = torch.cuda.Stream(device=dev)
        s2.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s2):
            run_parts(with_k2, with_k3)
        torch.cuda.current_stream().wait_stream(s2)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            run_parts(with_k2, with_k3)
        for _ in range(3):
            gr.replay()
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        for _ in range(reps):
            gr.replay()
        b_.record()
        torch.cuda.synchronize()
        return a_.elapsed_time(b_) / reps

    # ---- prefill (tcgen05 grouped GEMMs): one 2048-token call of layer 0 ----
    prefill = None
    if args.prefill_tokens > 0:
        Tp = args.prefill_tokens
        pl0 = pls[0]
        wsp = ops.Workspace(dev, 128, 8, shape.hidden, shape.inter, 0)
        xp = synth.make_hidden(Tp, shape.hidden, SEED + 11, device=dev)
        idx_p, w_p = ops.router_topk(xp, router.routers[0], 8, wsp)
        outp = torch.empty_like(xp)
        for _ in range(3):
            ops.moe_prefill(xp, w_p, pl0.experts, wsp, outp)
        torch.cuda.synchronize()
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        for _ in range(10):
            ops.moe_prefill(xp, w_p, pl0.experts, wsp, outp)
        b_.record()
        torch.cuda.synchronize()
        us = a_.elapsed_time(b_) / 10 * 1000
        a_.record()
        for _ in range(10):
            ops.router_topk(xp, router.routers[0], 8, wsp)
        b_.record()
        torch.cuda.synchronize()
        router_us_eager = a_.elapsed_time(b_) / 10 * 1000  # bound by the Python call
        # device time: the same 10 calls replayed from one CUDA graph
        sr = torch.cuda.Stream(device=dev)
        sr.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(sr):
            ops.router_topk(xp, router.routers[0], 8, wsp)
        torch.cuda.current_stream().wait_stream(sr)
        gr_router = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr_router):
            for _ in range(10):
                ops.router_topk(xp, router.routers[0], 8, wsp)
        gr_router.replay()
        torch.cuda.synchronize()
        a_.record()
        gr_router.replay()
        b_.record()
        torch.cuda.synchronize()
        router_us = a_.elapsed_time(b_) / 10 * 1000
        del gr_router
        flops = 2.0 * Tp * 8 * 3 * shape.hidden * shape.inter
        wbytes = 128 * EXPERT_BYTES
        prefill = {"workload": f"one MoE layer call with {Tp} tokens (router excluded): tcgen05 grouped GEMMs",
                   "us_per_layer": round(us, 1), "tokens_per_s_per_layer": round(Tp / (us * 1e-6), 1),
                   "tflops": round(flops / (us * 1e-6) / 1e12, 1), "algorithmic_flops": flops,
                   "weight_bytes": wbytes, "hbm_gbs": round(wbytes / (us * 1e-6) / 1e9, 1),
                   "router_us": round(router_us, 1),
                   "router_timing": "router + plan for the same tokens, 10 calls replayed from one CUDA graph "
                                    "(device time); router_us_eager: the same calls from Python",
                   "router_us_eager": round(router_us_eager, 1),
                   "status": ws.status() | wsp.status()}
        assert torch.isfinite(outp.float()).all(), "non-finite prefill output"

    # ---- FP8 attention projections (q/k/v/o of Qwen3-30B-A3B), one decode token ----
    attn = None
    if args.attn_layers > 0:
        La = args.attn_layers
        # q, k, v share their input: their rows are packed as one [5120, 2048]
        # weight (one launch); o [2048, 4096] follows attention (one launch)
        shapes = [(4096 + 512 + 512, 2048), (2048, 4096)]  # [out, in]
        ga = torch.Generator(device=dev)
        ga.manual_seed(SEED + 21)
        lins = []
        for _l in range(La):
            for N, K in shapes:
                qa, sa = synth.quantize_fp8_block(torch.randn(N, K, generator=ga, device=dev) * 0.02)
                lins.append(ops.pack_linear(qa, sa))
                del qa
        xa = synth.make_hidden(1, 2048, SEED + 22, rms_normalise=True, device=dev)
        xo = synth.make_hidden(1, 4096, SEED + 23, device=dev)
        outs = {N: torch.empty(1, N, dtype=torch.bfloat16, device=dev) for N in (5120, 2048)}

        def attn_step():
            for pl in lins:
                ops.fp8_linear(xo if pl.in_features == 4096 else xa, pl, out=outs[pl.out_features])

        sa_ = torch.cuda.Stream(device=dev)
        sa_.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(sa_):
            attn_step()
        torch.cuda.current_stream().wait_stream(sa_)
        ga_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ga_):
            attn_step()
        for _ in range(3):
            ga_.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            ga_.replay()
        e1.record()
        torch.cuda.synchronize()
        usa = e0.elapsed_time(e1) / 10 * 1000 / La
        ba = sum(N * K + (N // 128) * (K // 128) * 4 + (K + N) * 2 for N, K in shapes)
        hbm, _src = _peaks()
        attn = {"workload": f"FP8 block-scaled attention projections (tm_fp8_linear) of {La} Qwen3-30B-A3B "
                            f"layers, one decode token: fused q/k/v [5120, 2048] + o [2048, 4096], CUDA graph",
                "us_per_layer": round(usa, 2), "algorithmic_bytes_per_layer": ba,
                "hbm_gbs": round(ba / (usa * 1e-6) / 1e9, 1), "frac": round(ba / (usa * 1e-6) / 1e9 / hbm, 4),
                "launches_per_layer": len(shapes)}
        del ga_, lins
        assert all(torch.isfinite(o.float()).all() for o in outs.values()), "non-finite linear output"

    # ---- Qwen3.5-shaped layer (256 experts, I 512, FP8 shared expert), 64 tokens ----
    c3 = None
    if args.c3_tokens > 0:
        T3 = args.c3_tokens
        sh3 = synth.QWEN35_LAYER
        lw3 = synth.make_layer(sh3, SEED + 3, 0, device=dev)
        ex3 = ops.pack_experts(lw3.gate, lw3.gate_s, lw3.up, lw3.up_s, lw3.down, lw3.down_s)
        shx3 = ops.pack_experts(lw3.sh_gate, lw3.sh_gate_s, lw3.sh_up, lw3.sh_up_s, lw3.sh_down, lw3.sh_down_s)
        r3 = lw3.router.to(torch.bfloat16).contiguous()
        g3 = lw3.sh_router.to(torch.bfloat16).reshape(-1).contiguous()
        del lw3
        ws3 = ops.Workspace(dev, sh3.experts, sh3.top_k, sh3.hidden, sh3.inter, sh3.shared_inter)
        ws3.ensure(T3)
        x3 = synth.make_hidden(T3, sh3.hidden, SEED + 13, device=dev)
        out3 = torch.empty_like(x3)

        def call3():
            idx3, w3 = ops.router_topk(x3, r3, sh3.top_k, ws3)
            ops.moe_experts(x3, idx3, w3, ex3, ws3, shared=shx3, shared_gate_w=g3, residual=x3, out=out3)
            return idx3

        s3 = torch.cuda.Stream(device=dev)
        s3.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s3):
            for _ in range(2):
                call3()
        torch.cuda.current_stream().wait_stream(s3)
        g3r = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g3r):
            idx3 = call3()
        for _ in range(3):
            g3r.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            g3r.replay()
        e1.record()
        torch.cuda.synchronize()
        us3 = e0.elapsed_time(e1) / 20 * 1000
        U = int(torch.unique(idx3).numel())
        e_bytes = 3 * sh3.inter * sh3.hidden
        e_scales = 3 * (sh3.inter // 128) * (sh3.hidden // 128) * 4
        b3 = (U + 1) * (e_bytes + e_scales) + sh3.experts * sh3.hidden * 2 + sh3.hidden * 2 + 2 * T3 * sh3.hidden * 2
        hbm, _src = _peaks()
        c3 = {"workload": f"one Qwen3.5-shaped MoE layer call (E 256, top-8, I 512, FP8 shared expert I 512) "
                          f"with {T3} tokens: router + experts + shared expert + residual (CUDA graph)",
              "us_per_layer": round(us3, 1), "unique_experts": U, "algorithmic_bytes": b3,
              "hbm_gbs": round(b3 / (us3 * 1e-6) / 1e9, 1), "frac": round(b3 / (us3 * 1e-6) / 1e9 / hbm, 4),
              "status": ws3.status()}
        del g3r
        assert torch.isfinite(out3.float()).all(), "non-finite C3 output"

    reps = max(5, args.steps)
    t_b = graph_time(False, False, reps)
    t_a = graph_time(True, False, reps)
    t_c = graph_time(True, True, reps)
    k2 = max(t_a - t_b, 1e-6) / LAYERS
    k3 = max(t_c - t_a, 1e-6) / LAYERS
    peak, peak_kind = _peaks()
    k2_gbs = K2_BYTES / (k2 / 1000.0) / 1e9
    layer_gbs = LAYER_BYTES * LAYERS / (ms_per_step / 1000.0) / 1e9
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 weights, bf16 act, fp32 math",
        "data": "synthetic (seeded N(0,0.02) FP8 block-scaled weights, bf16 N(0,1) RMS-normalised token)",
        "config": {"workload": f"Qwen3-30B-A3B-FP8 MoE hot path: {LAYERS} layers x (router + top-8 of 128 FP8 experts), "
                               "bs=1 decode, attention excluded",
                   "hidden": 2048, "experts": 128, "top_k": 8, "moe_intermediate": 768, "layers": LAYERS,
                   "tokens_per_step": args.tokens, "parallelism": f"replicas x{world}",
                   "l2": "weights read per step 1.8 GB >> 126 MB L2 (no flush needed)",
                   "timing": "CUDA graph of the step, CUDA events, max over ranks"},
        "e2e": {"value": round(world * args.tokens * args.steps / e2e_s, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                "d2h_bytes_per_step": y_host.numel() * y_host.element_size(),
                "path": "RouterExecutor.compute_routing + MoEExecutor.execute_layer x48 captured in a CUDA graph",
                "eager_value": round(world * args.tokens * args.steps / eager_s, 2)},
        "roofline": {"bound": "hbm", "kernel": "k2_gateup (gate+up dequant-GEMV + SwiGLU; pulls the experts' down "
                                                     "projections into L2 for K3)",
                     "achieved": round(k2_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(k2_gbs / peak, 4), "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": K2_BYTES, "launch_us": round(k2 * 1000, 3),
                     "launch_timing": "marginal device time of K2 in a CUDA graph of 48 layers (events)",
                     "traffic": K2_TRAFFIC, "traffic_source": K2_TRAFFIC_SOURCE},
        "moe_layer": {"gbs": round(layer_gbs, 1), "frac": round(layer_gbs / peak, 4),
                      "bytes_per_layer": LAYER_BYTES, "us_per_layer": round(ms_per_step * 1000 / LAYERS, 3),
                      "k3_us": round(k3 * 1000, 3)},
        "gpu_launches": args.steps * (LAYERS * 3 + ((LAYERS - 1) * 2 if use_pf else 0)),
        "clocks": clk.summary(),
        "upload_s": round(upload_s, 1),
    }
    if next_layer_prefetch is not None:
        res["next_layer_prefetch"] = next_layer_prefetch
    if args.ep_tokens > 0:
        res["ep"] = ep_measure(args, rank, world, local, loader, router)
    if args.loader_layers > 0 and world == 1:
        res["loader"] = loader_measure(args, local)
    if args.model_tokens > 0 and world == 1:
        res["full_model"] = model_measure(args, local)
    if prefill is not None:
        res["prefill"] = prefill
    if c3 is not None:
        res["qwen35_layer"] = c3
    if attn is not None:
        res["attention_linears"] = attn
    if args.gdn_batches and world == 1:
        try:
            res["qwen35_linear_attention"] = gdn_measure(args, local)
        except Exception as e:  # recorded on the line; the measurements above stand
            res["qwen35_linear_attention"] = {"error": f"{type(e).__name__}: {e}"}
    return res


def gdn_measure(args, local):
    """Qwen3.5 linear-attention decode step (tm_gdn_decode) at 16 key heads,
    32 value heads of 128, conv kernel 4, bf16: one launch per layer, batch B
    sequences per launch, timed with CUDA events around a CUDA graph of
    L layers' launches (L layers' distinct states: >= 256 MB, more than L2).
    Algorithmic bytes per launch: the fp32 recurrent state read and written
    (B x 32 x 64 KB x 2), the conv state read and written, this token's
    qkv/z/a/b rows and the output, and the conv and norm weights."""
    from turbomoe import ops
    dev = torch.device("cuda", local)
    Hk, Hv, K, dt = 16, 32, 4, torch.bfloat16
    C = 2 * Hk * 128 + Hv * 128
    hbm, src = _peaks()
    g = torch.Generator(device=dev).manual_seed(SEED + 9)
    conv_w = (torch.randn(C, K, generator=g, device=dev) * 0.5).to(dt)
    A_log = torch.log(torch.rand(Hv, generator=g, device=dev) * 16 + 1e-3)
    dt_bias = torch.randn(Hv, generator=g, device=dev) * 0.5
    norm_w = torch.ones(128, dtype=dt, device=dev)
    out = {}
    for B in [int(b) for b in args.gdn_batches.split(",") if b]:
        state_bytes = B * Hv * 128 * 128 * 4
        L = max(2, -(-(256 << 20) // state_bytes))
        layers = []
        for _ in range(L):
            layers.append(dict(
                qkv=torch.randn(B, C, generator=g, device=dev).to(dt),
                z=torch.randn(B, Hv * 128, generator=g, device=dev).to(dt),
                a=torch.randn(B, Hv, generator=g, device=dev).to(dt),
                b=torch.randn(B, Hv, generator=g, device=dev).to(dt),
                cin=torch.randn(B, C, K, generator=g, device=dev).to(dt),
                cout=torch.empty(B, C, K, dtype=dt, device=dev),
                S=torch.randn(B, Hv, 128, 128, generator=g, device=dev) * 0.05,
                o=torch.empty(B, Hv * 128, dtype=dt, device=dev)))

        def run():
            for t in layers:
                ops.gdn_decode(t["qkv"], t["z"], t["a"], t["b"], conv_w, A_log, dt_bias, norm_w, t["cin"],
                               t["cout"], t["S"], Hk, 1e-6, out=t["o"])

        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(3):
                run()
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                run()
            for _ in range(3):
                graph.replay()
            reps = max(3, (20 << 30) // (L * state_bytes * 2 + 1))
            reps = min(reps, 200)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(dev)
            e0.record(s)
            for _ in range(reps):
                graph.replay()
            e1.record(s)
            torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1000.0 / (reps * L)
        per_seq = 2 * Hv * 128 * 128 * 4 + 2 * C * K * 2 + (C + 2 * Hv * 128 + 2 * Hv) * 2
        nbytes = B * per_seq + C * K * 2 + 128 * 2 + 2 * Hv * 4
        gbs = nbytes / (us * 1e-6) / 1e9
        out[f"batch_{B}"] = {"us_per_layer": round(us, 3), "algorithmic_bytes": nbytes, "gbs": round(gbs, 1),
                             "frac": round(gbs / hbm, 4), "layers_rotated": L, "replays": reps}
        del graph, layers
        torch.cuda.empty_cache()
    out["workload"] = ("Qwen3.5 linear-attention decode step (gated delta rule: conv update, q/k l2norm, "
                       "gates, fp32 state update, gated RMSNorm; 16 key / 32 value heads of 128, conv 4, bf16), "
                       "one launch per layer, states rotated over more than L2")
    out["peak"] = {"hbm_gbs": hbm, "source": src}
    return out


# ------------------------------------------ full-model greedy decode ----
def model_measure(args, local):
    """Batch-1 greedy decode of the whole random-init Qwen3-30B-A3B-FP8 model
    (48 layers with attention, LM head and argmax; turbomoe.decoder, one CUDA
    graph per step): the prompt of ``args.model_prompt`` tokens enters one
    position per step, then ``args.model_tokens`` tokens are generated.
    ``tokens_per_s`` = generated tokens / device time of their steps (CUDA
    events); ``e2e`` = the public ``generate`` call with the prompt ids from
    host memory and the generated ids read back, prefill included."""
    from loader.expert_loader import ExpertLoader
    from turbomoe import synth_model as S
    from turbomoe.decoder import Qwen3MoeDecoder
    dev = torch.device("cuda", local)
    cfg = S.config()
    P, N = args.model_prompt, args.model_tokens
    t0 = time.time()
    L = ExpertLoader(None, config={"execution": {"dtype": "bf16"}}, source=S.ModelSource(cfg, SEED, dev))
    dec = Qwen3MoeDecoder(L, cfg, max_len=P + N + 8, device=dev)
    dec.capture()
    build_s = time.time() - t0
    g = torch.Generator().manual_seed(SEED + 5)
    prompt = torch.randint(0, cfg["vocab_size"], (P,), generator=g).tolist()
    dec.teacher_forced(prompt)             # fills the cache of the prompt positions
    for _ in range(3):                      # warm-up steps beyond the prompt (replaced below)
        dec.step()
    dec.pos.fill_(P)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(N):
        dec.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    st = int(dec.status.item())
    fused = bool(dec.fused_norms)
    fused_rope = bool(dec.fused_rope)
    t = time.perf_counter()
    toks = dec.generate(prompt, N)
    e2e_s = time.perf_counter() - t
    # per generated token: 8 experts, the router, the q/k/v/o weights and the
    # KV rows of every layer (mean context P + N/2), plus the LM head
    layer_bytes = (8 * 3 * 768 * 2048 + 128 * 2048 * 2 + 5120 * 2048 + 2048 * 4096
                   + 2 * 4 * (P + N // 2) * 128 * 2)
    step_bytes = 48 * layer_bytes + 151936 * 2048 * 2
    hbm, _src = _peaks()
    out = {"workload": f"Qwen3-30B-A3B-FP8 random-init, batch-1 greedy decode of {N} tokens after a {P}-token "
                       "prompt (48 layers: FP8 q/k/v/o, GQA attention over the bf16 KV cache, MoE, bf16 LM head, "
                       "device argmax); one CUDA graph per step",
           "tokens_per_s": round(N / (ms / 1000.0), 1), "ms_per_token": round(ms / N, 4),
           "algorithmic_bytes_per_token": step_bytes,
           "hbm_gbs": round(step_bytes / (ms / N / 1000.0) / 1e9, 1),
           "frac": round(step_bytes / (ms / N / 1000.0) / 1e9 / hbm, 4),
           "e2e": {"tokens_per_s_incl_prefill": round(N / e2e_s, 1), "seconds": round(e2e_s, 3),
                   "path": "Qwen3MoeDecoder.generate (prompt ids from host, one position per step, ids read back)"},
           "kernel_launches_per_token": 3 + 48 * (9 - (2 if fused else 0) - (1 if fused_rope else 0)),
           "norms_fused": fused, "rope_fused_into_attention": fused_rope,
           "build_s": round(build_s, 1), "status": st, "distinct_generated": len(set(toks))}
    del dec, L
    torch.cuda.empty_cache()
    return out


def loader_measure(args, local):
    """The safetensors -> packed upload path (ExpertLoader on an HF snapshot:
    SafetensorsSource.layer_experts reads, stacks and pins each layer's 384
    e4m3 tensors and their scales, copies them to the GPU, tm_pack_experts
    packs them): a Qwen3-30B-A3B-shaped seeded checkpoint of
    ``args.loader_layers`` layers written to a temporary directory, then
    ExpertLoader(snapshot).upload() timed by the host clock with the device
    synchronised.  The files were just written, so they are read from the page
    cache: this times the host and PCIe side of the path, not a disk."""
    import shutil
    import tempfile
    from loader.expert_loader import ExpertLoader
    from turbomoe import synth
    shape = synth.QWEN3_30B_A3B
    n = args.loader_layers
    dev = torch.device("cuda", local)
    d = tempfile.mkdtemp(prefix="tm_snapshot_")
    try:
        t0 = time.time()
        synth.write_checkpoint(d, shape, SEED, layers=n, device=dev)
        write_s = time.time() - t0
        file_bytes = sum(os.path.getsize(os.path.join(d, f)) for f in os.listdir(d))
        torch.cuda.synchronize()
        t0 = time.time()
        L = ExpertLoader(d, config={"execution": {"dtype": "bf16"}})
        L.upload()
        torch.cuda.synchronize()
        up_s = time.time() - t0
        expert_bytes = n * shape.experts * (EXPERT_BYTES + 288 * 4)
        del L
        torch.cuda.empty_cache()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return {"workload": f"safetensors snapshot of {n} Qwen3-30B-A3B layer(s) ({shape.experts} FP8 experts each) -> "
                        "packed device layout (ExpertLoader.upload: safetensors reads, stack + pin, H2D, "
                        "tm_pack_experts); files in the page cache",
            "layers": n, "file_bytes": file_bytes, "expert_bytes": expert_bytes, "upload_s": round(up_s, 3),
            "gb_per_s": round(expert_bytes / up_s / 1e9, 2),
            "model_48_layers_s_estimate": round(48 * up_s / n, 1), "checkpoint_write_s": round(write_s, 1)}


# ------------------------------------- expert parallelism on every line ----
def _fp32_layer(x, idx, w, packed, tokens):
    """fp32 evaluation of the routed experts for the first ``tokens`` tokens:
    weights dequantised exactly (K0 in fp32, bit-exact to the reference's
    dequantisation), then plain PyTorch fp32 matmuls in the order of
    MoEExecutor.execute_layer (execution/moe.py:164-176).  A numerics
    reference of the same op, used to check the expert-parallel output."""
    from turbomoe import ops
    xs = x[:tokens].float()
    y = torch.zeros_like(xs)
    cache = {}
    for t in range(tokens):
        for r in range(idx.shape[1]):
            e = int(idx[t, r])
            if e not in cache:
                cache[e] = ops.unpack_expert(packed, e, torch.float32)
            g, u, d = cache[e]
            h = torch.nn.functional.silu(xs[t] @ g.T) * (xs[t] @ u.T)
            y[t] += float(w[t, r]) * (h @ d.T)
    return y


def _cmp(a, b):
    a, b = a.float(), b.float()
    cos = torch.nn.functional.cosine_similarity(a.reshape(1, -1), b.reshape(1, -1)).item()
    return float((a - b).abs().max()), cos


def ep_measure(args, rank, world, local, loader, router):
    """Expert-parallel batched decode of the Qwen3-30B-A3B MoE layers: the
    ``args.ep_tokens`` sequences (one token each) split over the ranks, the
    128 experts of every layer sharded E/N per GPU (views into the packed
    layers the loader already holds), dispatch / experts / return over NVLink
    peer memory (tm_ep_*), the whole step of ``args.layers`` layers in one CUDA
    graph.  Uniform routing and, with ``args.ep_zipf`` > 0, Zipf-skewed routing.
    Reports tokens/s (CUDA events, max over ranks), a per-phase split of an
    eager pass, the single-GPU number of the same workload (rank 0 alone) for
    the strong-scaling efficiency, and a parity block per rank."""
    from turbomoe import ops, synth
    from turbomoe._lib import lib
    from turbomoe.ep import PeerExpertParallelMoE
    shape = synth.QWEN3_30B_A3B
    E, k, H, I = shape.experts, shape.top_k, shape.hidden, shape.inter
    Lr = args.layers
    E_loc = E // world
    T = args.ep_tokens // world
    dev = torch.device("cuda", local)
    Lb = lib()
    n13, ns13 = Lb.tm_packed_w13_bytes(H, I), Lb.tm_packed_s13_floats(H, I)
    n2, ns2 = Lb.tm_packed_w2_bytes(H, I), Lb.tm_packed_s2_floats(H, I)

    def shard(pe, a, b):
        return ops.PackedExperts(pe.w13[a * n13:b * n13], pe.s13[a * ns13:b * ns13], pe.w2[a * n2:b * n2],
                                 pe.s2[a * ns2:b * ns2], b - a, H, I)

    full = [loader.packed_layer(l).experts for l in range(Lr)]
    mine = [shard(pe, rank * E_loc, (rank + 1) * E_loc) for pe in full]
    routers = {"uniform": [router.routers[l] for l in range(Lr)]}
    if args.ep_zipf > 0:
        routers["zipf"] = [synth.router_with_bias(router.routers[l], synth.zipf_expert_bias(E, SEED + l, args.ep_zipf))
                           .contiguous() for l in range(Lr)]
    x_u = synth.make_hidden(T, H, SEED + 100 + rank, rms_normalise=True, device=dev)
    inputs = {"uniform": x_u, "zipf": synth.tokens_for_bias(x_u)}
    bufs = [torch.empty_like(x_u) for _ in range(2)]

    def build(shards, single=False, tokens=T):
        chan = PeerExpertParallelMoE(routers["uniform"][0], shards[0], k, max_tokens=tokens, single=single)
        out = {}
        for name, rw in routers.items():
            out[name] = [chan if (name == "uniform" and l == 0) else
                         PeerExpertParallelMoE(rw[l], shards[l], k, tokens, channel=chan) for l in range(Lr)]
        return chan, out

    def step(eps, x, bb, marks=None):
        for i, ep in enumerate(eps):
            x = ep.forward(x, residual=x, out=bb[i % 2], marks=None if marks is None else marks[i])
        return x

    def capture(eps, x, bb):
        for _ in range(args.warmup):
            step(eps, x, bb)
        torch.cuda.synchronize()
        s_ = torch.cuda.Stream(device=dev)
        s_.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_):
            step(eps, x, bb)
        torch.cuda.current_stream().wait_stream(s_)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(eps, x, bb)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        return g

    def timed(g, n_steps, group_world):
        barrier(group_world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n_steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        barrier(group_world)
        return max_over_ranks(e0.elapsed_time(e1), group_world)

    chan, layers = build(mine)
    res = {"workload": f"{args.ep_tokens} sequences x 1 token through {Lr} Qwen3-30B-A3B MoE layers, experts "
                       f"sharded {E_loc} per GPU over {world} GPU(s); dispatch / owner grouped GEMMs / return "
                       "by NVLink peer stores (tm_ep_*), step in one CUDA graph",
           "tokens_per_rank": T, "experts_per_rank": E_loc, "parallelism": f"ep{world}", "scaling": "strong",
           "timing": "CUDA events around graph replays, max over ranks"}
    with ClockSampler(local) as clk:
        for name in routers:
            g = capture(layers[name], inputs[name], bufs)
            ms = timed(g, args.steps, world)
            del g
            res[name] = {"tokens_per_s": round(T * world * args.steps / (ms / 1000.0), 1),
                         "us_per_layer": round(ms / args.steps / Lr * 1000, 1)}
    res["clocks"] = clk.summary()
    # per-phase split (eager pass; the experts phase includes the wait for the
    # sources' rows, the combine phase the wait for the owners' outputs)
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(Lr)]
    for name in routers:
        torch.cuda.synchronize()
        barrier(world)
        step(layers[name], inputs[name], bufs, marks)
        torch.cuda.synchronize()
        ph = [sum(m[i].elapsed_time(m[i + 1]) for m in marks) / Lr * 1000 for i in range(4)]
        ph = [max_over_ranks(v, world) for v in ph]
        res[name]["phase_us_per_layer"] = {"router": round(ph[0], 1), "dispatch": round(ph[1], 1),
                                           "experts_incl_wait": round(ph[2], 1),
                                           "combine_incl_wait": round(ph[3], 1)}
        lim = max(range(4), key=lambda i: ph[i])
        res[name]["limiting_phase"] = ["router", "dispatch", "experts_incl_wait", "combine_incl_wait"][lim]
    # load balance of the first layer: routed pairs per owner rank, all ranks' tokens
    ws0 = ops.Workspace(dev, E, k, H, I)
    for name in routers:
        idx0, _ = ops.router_topk(inputs[name], routers[name][0], k, ws0)
        pairs = torch.bincount(idx0.reshape(-1) // E_loc, minlength=world).to(torch.float64)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(pairs)
        res[name]["owner_load_max_over_mean"] = round(float(pairs.max() / pairs.mean()), 3)
        res[name]["distinct_experts_layer0_rank"] = int(torch.unique(idx0).numel())
    # parity: layer 0 on this rank's tokens, EP vs the whole layer on this GPU
    # (all 128 experts, same kernels: bit-exact expected) and vs fp32
    par = {}
    for name in routers:
        xin = inputs[name]
        y_ep = layers[name][0].forward(xin).clone()
        idx, w = ops.router_topk(xin, routers[name][0], k, ws0)
        y_1 = ops.moe_experts(xin, idx, w, full[0], ws0)
        ns = min(T, 8)
        y32 = _fp32_layer(xin, idx, w, full[0], ns)
        torch.cuda.synchronize()
        m1, c1 = _cmp(y_ep, y_1)
        m32, c32 = _cmp(y_ep[:ns], y32)
        ok = float(m32 <= 2e-2 and c32 >= 0.9995)
        stats = torch.tensor([m1, -c1, m32, -c32, float(torch.equal(y_ep, y_1)), ok], dtype=torch.float64,
                             device=dev)
        if world > 1:
            import torch.distributed as dist
            lo = stats.clone()
            lo[4:] *= -1
            dist.all_reduce(lo, op=dist.ReduceOp.MAX)   # worst over ranks (min of the flags)
            lo[4:] *= -1
            stats = lo
        st = stats.tolist()
        par[name] = {"vs_single_gpu_layer": {"max_abs": st[0], "cos": -st[1], "bit_exact_all_ranks": bool(st[4])},
                     "vs_fp32": {"max_abs": st[2], "cos": -st[3], "tokens_per_rank": ns,
                                 "within_2e-2_0.9995_all_ranks": bool(st[5])}}
    res["parity_layer0"] = par
    status = max_over_ranks(float(layers["uniform"][0].status()), world)
    res["status"] = int(status)
    for name in routers:
        for ep in layers[name]:
            if ep is not chan:
                ep.close()
    chan.close()
    # the same workload on one GPU (rank 0 alone, all experts local): the
    # denominator of the strong-scaling efficiency
    if world > 1:
        if rank == 0:
            chan1, layers1 = build(full, single=True, tokens=args.ep_tokens)
            x1 = synth.make_hidden(args.ep_tokens, H, SEED + 100, rms_normalise=True, device=dev)
            b1 = [torch.empty_like(x1) for _ in range(2)]
            g = capture(layers1["uniform"], x1, b1)
            ms1 = timed(g, args.steps, 1)
            del g
            for ep in layers1["uniform"] + layers1.get("zipf", []):
                if ep is not chan1:
                    ep.close()
            chan1.close()
            one = args.ep_tokens * args.steps / (ms1 / 1000.0)
            res["single_gpu_tokens_per_s"] = round(one, 1)
            res["strong_scaling_efficiency"] = round(res["uniform"]["tokens_per_s"] / (world * one), 3)
        barrier(world)
    else:
        res["single_gpu_tokens_per_s"] = res["uniform"]["tokens_per_s"]
        res["strong_scaling_efficiency"] = 1.0
    if args.ep_ctx > 0:
        res["attention"] = ep_attention(args, rank, world, local)
    if "zipf" in routers:
        res["zipf"]["routing"] = (f"Zipf s={args.ep_zipf}: router column {H - 1} replaced by log p_e (p_e ~ rank^-s "
                                  f"over a seeded expert permutation) and token coordinate {H - 1} set to 1, so the "
                                  "experts also see that modified coordinate")
    return res


def ep_attention(args, rank, world, local):
    """Decode attention of the batched-decode step: this rank's
    T = ep_tokens / N sequences (data-parallel: each GPU holds its own
    sequences' caches) at ``args.ep_ctx`` tokens of bf16 KV context, one layer
    of the Qwen3-30B-A3B attention (32 query / 4 KV heads, head_dim 128)
    through tm_attn_decode_batched.  CUDA events over ``args.steps`` calls
    (layers' caches alternating so that every call reads HBM), max over
    ranks; HBM bytes = the K and V rows of every sequence's context."""
    import math
    from turbomoe import ops
    from turbomoe._lib import lib
    Lb = lib()
    T, ctx = args.ep_tokens // world, args.ep_ctx
    nh, nkv, hd = 32, 4, 128
    dev = torch.device("cuda", local)
    per = nkv * ctx * hd                                     # elements of one sequence's K (or V) cache
    layer_bytes = 2 * T * per * 2
    n_layers = max(1, min(4, -(-(1 << 30) // layer_bytes)))  # >= 1 GiB of caches in rotation
    g = torch.Generator(device=dev).manual_seed(SEED + 7 + rank)
    caches = [(torch.randn(T * per, generator=g, device=dev).to(torch.bfloat16),
               torch.randn(T * per, generator=g, device=dev).to(torch.bfloat16)) for _ in range(n_layers)]
    q = torch.randn(T, nh, hd, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(T, nh * hd, dtype=torch.bfloat16, device=dev)
    pos = torch.full((T,), ctx - 1, dtype=torch.int64, device=dev)
    splits = max(1, min(16, -(-2 * 148 // (nkv * T))))
    s = torch.cuda.current_stream(dev).cuda_stream
    code = ops._code(torch.bfloat16)

    def call(i):
        kc, vc = caches[i % n_layers]
        rc = Lb.tm_attn_decode_batched(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), T, per, ctx, nh,
                                       nkv, hd, code, 1.0 / math.sqrt(hd), splits, out.data_ptr(), s)
        if rc != 0:
            raise RuntimeError(f"tm_attn_decode_batched: {Lb.tm_last_error().decode()}")

    for i in range(args.warmup):
        call(i)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        call(i)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    us = max_over_ranks(e0.elapsed_time(e1), world) / args.steps * 1000
    gbs = T * per * 2 * 2 / (us * 1e-6) / 1e9
    peak = _peaks()[0]
    del caches
    return {"kernel": "k8_attn_mma via tm_attn_decode_batched (mma.sync, splits of a KV head merged in a cluster)",
            "sequences_per_rank": T, "context": ctx, "heads": f"{nh} q / {nkv} kv x {hd}", "splits": splits,
            "us_per_layer": round(us, 1), "hbm_gbs": round(gbs, 1),
            "frac": round(gbs / peak, 3) if peak else None,
            "bytes_per_layer_per_rank": T * per * 2 * 2,
            "timing": f"CUDA events over {args.steps} calls, {n_layers} layers' caches in rotation, max over ranks"}


# ------------------------------------------------- expert-parallel decode ----
def run_ep(args, rank, world, local):
    """Expert-parallel batched decode: `--ep-tokens` sequences (one token each)
    split over the ranks, the 128 experts of every layer sharded over them;
    one step = the tokens through `--layers` MoE layers (dispatch / experts /
    combine per layer).  `--ep-impl peer` (default): the tm_ep_* kernels over
    NVLink peer memory, the step captured in one CUDA graph; `nccl`: NCCL
    all-to-all exchange with host-read row counts (eager).  Timed with CUDA
    events, max over ranks."""
    from turbomoe import ops, synth
    from turbomoe.ep import ExpertParallelMoE, PeerExpertParallelMoE, cuda_functions
    import torch.distributed as dist
    if world == 1 and not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % (29500 + os.getpid() % 1000),
                                rank=0, world_size=1)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shape = synth.QWEN3_30B_A3B
    E, k, H, I = shape.experts, shape.top_k, shape.hidden, shape.inter
    E_loc = E // world
    T = args.ep_tokens // world
    peer = args.ep_impl == "peer"
    layers = []
    for l in range(args.layers):
        lw = synth.make_layer(shape, SEED, l, device=dev)
        sl = slice(rank * E_loc, (rank + 1) * E_loc)
        local_experts = ops.pack_experts(lw.gate[sl], lw.gate_s[sl], lw.up[sl], lw.up_s[sl], lw.down[sl],
                                         lw.down_s[sl])
        router_w = lw.router.to(torch.bfloat16).contiguous()
        if args.ep_zipf > 0:  # skewed routing: logit bias log p_e carried by the last coordinate
            router_w = synth.router_with_bias(router_w, synth.zipf_expert_bias(E, SEED + l, args.ep_zipf)).contiguous()
        if l == 0:
            router_w0 = router_w
        del lw
        if peer:
            layers.append(PeerExpertParallelMoE(router_w, local_experts, k, max_tokens=T))
        else:
            layers.append(ExpertParallelMoE(E, k, *cuda_functions(router_w, local_experts, k, E, H, I)))
    torch.cuda.empty_cache()
    x0 = synth.make_hidden(T, H, SEED + 100 + rank, rms_normalise=True, device=dev)
    if args.ep_zipf > 0:
        x0 = synth.tokens_for_bias(x0)
    bufs = [torch.empty_like(x0) for _ in range(2)]
    # load balance of the first layer: routed pairs per owner rank, all ranks' tokens
    ws0 = ops.Workspace(dev, E, k, H, I)
    idx0, _ = ops.router_topk(x0, router_w0, k, ws0)
    owner_pairs = torch.bincount(idx0.reshape(-1) // E_loc, minlength=world).to(torch.float64)
    if world > 1:
        dist.all_reduce(owner_pairs)
    owner_imbalance = float(owner_pairs.max() / owner_pairs.mean())
    del ws0, idx0

    def step(x):
        for i, ep in enumerate(layers):
            x = ep.forward(x, residual=x, out=bufs[i % 2]) if peer else ep.forward(x, residual=x)
        return x

    for _ in range(args.warmup):
        step(x0)
    torch.cuda.synchronize()
    eager_ms = None
    run = lambda: step(x0)
    graph = None
    if peer:
        barrier(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(args.steps):
            step(x0)
        ev1.record()
        torch.cuda.synchronize()
        eager_ms = max_over_ranks(ev0.elapsed_time(ev1), world)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step(x0)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y_graph = step(x0)
        for _ in range(max(3, args.warmup)):
            graph.replay()
        run = graph.replay
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            y = run()
        ev1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    if peer:
        y = y_graph
        st = max_over_ranks(float(sum(ep.status() for ep in layers)), world)
        assert st == 0, f"expert-parallel status {st}"
    assert torch.isfinite(y.float()).all(), "non-finite output"
    res = {"metric": "expert-parallel batched decode tok/s, Qwen3-30B-A3B-FP8 MoE layers",
           "value": round(T * world * args.steps / (ms / 1000.0), 1), "unit": "tokens/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "e4m3 weights, bf16 act, fp32 math",
           "data": "synthetic (seeded weights, " + (f"Zipf routing s={args.ep_zipf}: logit bias log p_e, p_e ~ "
                                                    "rank^-s over a seeded expert permutation)"
                                                    if args.ep_zipf > 0 else "uniform routing)"),
           "owner_load_max_over_mean": round(owner_imbalance, 3),
           "config": {"workload": f"{args.ep_tokens} sequences x 1 token through {args.layers} MoE layers, "
                                  f"experts sharded {E_loc} per GPU, " +
                                  ("dispatch/return by NVLink peer stores (tm_ep_*), step in one CUDA graph"
                                   if peer else "all-to-all dispatch/combine (NCCL), eager"),
                      "tokens_per_rank": T, "experts_per_rank": E_loc, "parallelism": f"ep{world}",
                      "ep_impl": args.ep_impl},
           "us_per_layer": round(ms / args.steps / args.layers * 1000, 1),
           "clocks": clk.summary()}
    if peer:
        res["eager_value"] = round(T * world * args.steps / (eager_ms / 1000.0), 1)
        del graph
        torch.cuda.synchronize()
        for ep in layers:
            ep.close()
    else:
        sc, rc = layers[-1].last_counts
        res["rows_sent_last_layer_rank0"], res["rows_recv_last_layer_rank0"] = sc, rc
    return res


# ------------------------------------------------------- CPU reference ----
def cpu_reference(steps, warmup, distinct_layers=2, threads=None, LAYERS=LAYERS, cold_steps=1):
    """Time the oracle (the reference's CPU path) on the host cores: warm
    (every expert already dequantised, the reference's best case) and cold
    (each layer call dequantises its routed experts, as the reference's slot
    cache does when 48 layers x 8 experts per token exceed its slots).
    Returns (warm tokens/s, warm seconds per step, description, threads,
    cold {tokens/s, seconds per step, steps})."""
    from oracle import moe_oracle as O
    from turbomoe import synth

    threads = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    shape = synth.QWEN3_30B_A3B
    layers = []
    for l in range(distinct_layers):
        lw = synth.make_layer(shape, SEED, l)
        ol = O.OracleLayer(lw, torch.bfloat16)
        for e in range(shape.experts):
            ol.expert(e)                       # warm: every expert already dequantised
        layers.append(ol)
    x0 = synth.make_hidden(1, shape.hidden, SEED + 7, rms_normalise=True)

    def step():
        x = x0
        for l in range(LAYERS):
            ol = layers[l % distinct_layers]
            idx, w = O.compute_routing(x, ol.router, 8)
            x = x + O.execute_layer(ol, x, idx, w)
        return x

    for _ in range(warmup):
        step()
    t = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t) / steps
    desc = (f"oracle port of RouterExecutor.compute_routing + MoEExecutor.execute_decode (torch CPU, bf16, "
            f"warm: dequantised experts cached), {steps} steps of {LAYERS} layer calls cycling {distinct_layers} "
            f"distinct synthetic layers, {threads} threads, {os.cpu_count()} cores visible")

    def cold_step():
        x = x0
        for l in range(LAYERS):
            ol = layers[l % distinct_layers]
            ol.drop_cache()                    # cold: the routed experts are dequantised in the call
            idx, w = O.compute_routing(x, ol.router, 8)
            x = x + O.execute_layer(ol, x, idx, w)
        return x

    cold = None
    if cold_steps > 0:
        t = time.perf_counter()
        for _ in range(cold_steps):
            cold_step()
        cdt = (time.perf_counter() - t) / cold_steps
        cold = {"value": round(1.0 / cdt, 4), "unit": "tokens/s", "ms_per_step": round(cdt * 1000, 3),
                "steps": cold_steps,
                "sample": "the same calls with each layer's routed experts dequantised in the call (no cache)"}
    return 1.0 / dt, dt, desc, threads, cold


def run_reference(args, rank, world):
    if rank != 0:
        return None
    tps, dt, desc, threads, cold = cpu_reference(args.steps, args.warmup, LAYERS=args.layers)
    return {"metric": METRIC, "value": round(tps, 4), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1000, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (reference CPU path)",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "Qwen3-30B-A3B-FP8 MoE hot path: 48 layers x (router + top-8 of 128 FP8 "
                                   "experts), bs=1 decode, attention excluded", "parallelism": "cpu"},
            "cpu_baseline": {"value": round(tps, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": desc, "cold": cold},
            "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--layers", type=int, default=LAYERS, help="MoE layers per step (48 = the model)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--next-layer-prefetch", action="store_true",
                    help="decode with the speculative L2 prefetch of each next layer's experts (also times the "
                         "step without it)")
    ap.add_argument("--prefetch-join-every", type=int, default=1,
                    help="with --next-layer-prefetch: rejoin the prefetch branch every this many layers")
    ap.add_argument("--prefill-tokens", type=int, default=2048,
                    help="also time one prefill layer call of this many tokens (0 = skip)")
    ap.add_argument("--attn-layers", type=int, default=48,
                    help="also time the FP8 q/k/v/o projections of this many layers, one token (0 = skip)")
    ap.add_argument("--c3-tokens", type=int, default=64,
                    help="also time one Qwen3.5-shaped layer call (shared expert) of this many tokens (0 = skip)")
    ap.add_argument("--model-tokens", type=int, default=256,
                    help="also time greedy decode of the whole model: tokens generated (0 = skip; 1 GPU only)")
    ap.add_argument("--model-prompt", type=int, default=2048, help="prompt length of the whole-model decode")
    ap.add_argument("--loader-layers", type=int, default=1,
                    help="also time the safetensors -> packed upload of a snapshot of this many layers "
                         "(0 = skip; 1 GPU only)")
    ap.add_argument("--workload", choices=["decode", "ep"], default="decode",
                    help="decode: batch-1 decode (replicas for N>1); ep: expert-parallel batched decode")
    ap.add_argument("--ep-tokens", type=int, default=256,
                    help="expert-parallel batched decode: sequences over all ranks (0 = skip the ep object)")
    ap.add_argument("--ep-ctx", type=int, default=4096,
                    help="expert-parallel decode: also time the batched decode attention of each rank's sequences "
                         "at this KV context (0 = skip)")
    ap.add_argument("--ep-zipf", type=float, default=1.2,
                    help="expert-parallel decode: also time Zipf-skewed routing with this exponent (0 = skip)")
    ap.add_argument("--gdn-batches", default="1,256",
                    help="also time the Qwen3.5 linear-attention decode step at these batch sizes, comma-separated "
                         "(empty = skip; 1 GPU only)")
    ap.add_argument("--ep-impl", choices=["peer", "nccl"], default="peer",
                    help="ep workload: NVLink peer-memory kernels (tm_ep_*) or NCCL all-to-all")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", 0))
        world = int(os.environ.get("WORLD_SIZE", 1))
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    rank, world, local = dist_setup(args.gpus)
    if args.workload == "ep":
        res = run_ep(args, rank, world, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
        return
    res = run_ours(args, rank, world, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, dt, desc, threads, cold = cpu_reference(steps=3, warmup=1, LAYERS=args.layers)
        res["cpu_baseline"] = {"value": round(tps, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                               "sample": desc, "cold": cold}
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
