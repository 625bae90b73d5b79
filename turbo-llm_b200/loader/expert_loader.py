"""ExpertLoader drop-in: one-time upload of every FP8 expert into a packed,
device-resident layout.

Replaces the reference's loader/expert_loader.py (the SSD -> RAM -> VRAM
slot cache with on-the-fly dequantisation, :17-602).  A whole Qwen3-30B-A3B
FP8 model is ~29 GB of expert weights, so on a B200 (180 GB HBM) every expert
is uploaded once, packed by ``tm_pack_experts`` into the layout the decode and
prefill kernels stream, and never evicted.  The public surface is kept:

* attributes ``DEVICE, dtype, layout, weight_map, expert_cache,
  expert_metadata, cache_limit, num_slots, ram_cache, gpu_hits, ram_hits,
  ssd_hits, load_ms_accum, dequant_ms_accum, evict_ms_accum, lock`` (read by
  runtime/engine.py and the backend);
* methods ``load_weight, load_weight_raw, dequantize_weight,
  load_weight_split, load_expert, load_expert_dynamic, load_expert_raw,
  clear_pinned_slots, adjust_cache_limit, close``.

``load_expert`` returns dense dequantised tensors (``tm_unpack_expert``), as
the reference's slot views were; the MoE executor does not call it -- it
streams the packed FP8 weights directly.  Everything runs on CUDA; there is
no CPU path (a CPU call raises).
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass

import torch

from cache.ram_cache import RAMCache
from loader.model_layout import ModelLayout
from turbomoe import ops
from turbomoe._lib import TurboMoEError

_DTYPES = {"bf16": torch.bfloat16, "bfloat16": torch.bfloat16, "fp16": torch.float16,
           "float16": torch.float16, "fp32": torch.float32, "float32": torch.float32}


@dataclass
class PackedLayer:
    """Everything the MoE kernels read for one layer."""
    experts: ops.PackedExperts
    shared: ops.PackedExperts | None = None
    shared_gate: torch.Tensor | None = None   # [H] act dtype (mlp.shared_expert_gate.weight)


class SafetensorsSource:
    """Tensors of an on-disk HF snapshot (``model.safetensors.index.json``)."""

    def __init__(self, snapshot_path, weight_map):
        self.snapshot_path = snapshot_path
        self.weight_map = weight_map
        self.files = {}

    def has(self, name):
        return name in self.weight_map

    def get(self, name):
        from safetensors import safe_open
        fn = self.weight_map[name]
        if fn not in self.files:
            self.files[fn] = safe_open(os.path.join(self.snapshot_path, fn), framework="pt", device="cpu")
        return self.files[fn].get_tensor(name)

    def layer_experts(self, layout, layer, n_experts, device):
        """Stacked raw tensors of one layer's experts, copied to ``device``."""
        out = []
        for mk in (layout.gate_tensor, layout.up_tensor, layout.down_tensor):
            ws = [self.get(mk(layer, e)) for e in range(n_experts)]
            ss = [self.get(mk(layer, e) + "_scale_inv") for e in range(n_experts)]
            w = torch.stack([t.view(torch.uint8) for t in ws]).pin_memory()
            s = torch.stack([t.float() for t in ss]).pin_memory()
            out += [w.to(device, non_blocking=True), s.to(device, non_blocking=True)]
        return out

    def close(self):
        self.files.clear()


class SyntheticSource:
    """Seeded synthetic FP8 weights generated directly on the device
    (``turbomoe.synth``): no files, no host round trip.  Used by the benchmark,
    where a 48-layer checkpoint is too large to write to disk."""

    def __init__(self, shape, seed, num_layers, device="cuda"):
        from turbomoe import synth
        self.synth = synth
        self.shape = shape
        self.seed = seed
        self.num_layers = num_layers
        self.device = device
        self._cache = (None, None)
        wm = {}
        for l in range(num_layers):
            p = f"model.layers.{l}.mlp"
            wm[f"{p}.gate.weight"] = "synthetic"
            for e in range(shape.experts):
                for m in ("gate_proj", "up_proj", "down_proj"):
                    wm[f"{p}.experts.{e}.{m}.weight"] = "synthetic"
                    wm[f"{p}.experts.{e}.{m}.weight_scale_inv"] = "synthetic"
            if shape.shared_inter:
                for m in ("gate_proj", "up_proj", "down_proj"):
                    wm[f"{p}.shared_expert.{m}.weight"] = "synthetic"
                    wm[f"{p}.shared_expert.{m}.weight_scale_inv"] = "synthetic"
                wm[f"{p}.shared_expert_gate.weight"] = "synthetic"
        self.weight_map = wm
        self.config = {"model_type": "qwen3_5_moe" if shape.shared_inter else "qwen3_moe",
                       "hidden_size": shape.hidden, "moe_intermediate_size": shape.inter,
                       "num_experts": shape.experts, "num_experts_per_tok": shape.top_k,
                       "num_hidden_layers": num_layers, "shared_expert_intermediate_size": shape.shared_inter}

    def layer(self, l):
        if self._cache[0] != l:
            self._cache = (l, self.synth.make_layer(self.shape, self.seed, l, device=self.device))
        return self._cache[1]

    def has(self, name):
        return name in self.weight_map

    def get(self, name):
        parts = name.split(".")
        l = int(parts[2])
        lw = self.layer(l)
        rest = ".".join(parts[4:])
        if rest == "gate.weight":
            return lw.router
        if rest == "shared_expert_gate.weight":
            return lw.sh_router
        scale = rest.endswith("_scale_inv")
        if rest.startswith("experts."):
            e = int(parts[5])
            m = parts[6]
            w, s = {"gate_proj": (lw.gate, lw.gate_s), "up_proj": (lw.up, lw.up_s),
                    "down_proj": (lw.down, lw.down_s)}[m]
            return s[e] if scale else w[e]
        if rest.startswith("shared_expert."):
            m = parts[5]
            w, s = {"gate_proj": (lw.sh_gate, lw.sh_gate_s), "up_proj": (lw.sh_up, lw.sh_up_s),
                    "down_proj": (lw.sh_down, lw.sh_down_s)}[m]
            return s if scale else w
        raise KeyError(name)

    def layer_experts(self, layout, layer, n_experts, device):
        lw = self.layer(layer)
        return [lw.gate, lw.gate_s, lw.up, lw.up_s, lw.down, lw.down_s]

    def close(self):
        self._cache = (None, None)


class ExpertLoader:
    DEVICE = "cuda" if torch.cuda.is_available() else "cpu"

    def __init__(self, snapshot_path, config=None, source=None):
        self.snapshot_path = snapshot_path
        self.config = config
        self.max_vram_gb = 180.0
        if config and "memory" in config and "max_vram_mb" in config["memory"]:
            self.max_vram_gb = config["memory"]["max_vram_mb"] / 1024.0
        # activation / dequantisation dtype: execution.dtype when given (the
        # reference tests a top-level key here, expert_loader.py:28, so its
        # default fp16 always wins; the intended setting is honoured instead)
        self.dtype = torch.float16
        if config and "execution" in config and "dtype" in config["execution"]:
            self.dtype = _DTYPES.get(str(config["execution"]["dtype"]), self.dtype)
        if source is None:
            self.layout = ModelLayout(snapshot_path)
            source = SafetensorsSource(snapshot_path, self.layout.weight_map)
        else:
            self.layout = ModelLayout(snapshot_path, config=source.config, weight_map=source.weight_map)
        self.source = source
        self.weight_map = self.layout.weight_map
        self.files = getattr(source, "files", {})
        self.expert_cache = {}
        self.expert_metadata = {}
        self.num_experts = self.layout.num_experts()
        self.num_layers = self.layout.num_layers()
        self.cache_limit = self.num_experts * self.num_layers
        self.num_slots = 0
        self.free_slots = []
        self.pinned_slots = set()
        self.lock = threading.RLock()
        self.load_ms_accum = 0.0
        self.dequant_ms_accum = 0.0
        self.evict_ms_accum = 0.0
        self.ram_cache = RAMCache(config=config)
        self.gpu_hits = 0
        self.ram_hits = 0
        self.ssd_hits = 0
        self.load_counter = 0
        self.ssd_load_counter = 0
        self.packed = {}
        self._workspaces = {}
        self.top_k = int(self.layout.config.get("num_experts_per_tok", 8))

    @classmethod
    def synthetic(cls, shape, seed=0, num_layers=1, dtype=torch.bfloat16, device=None, config=None):
        """A loader over seeded synthetic weights generated on the device."""
        dev = device or cls.DEVICE
        ld = cls(None, config=config, source=SyntheticSource(shape, seed, num_layers, dev))
        ld.dtype = dtype
        return ld

    # ------------------------------------------------------------ helpers ----
    def _require_cuda(self, device=None):
        dev = torch.device(device or self.DEVICE)
        if dev.type != "cuda":
            raise TurboMoEError("ExpertLoader needs a CUDA device: the FP8 MoE path has no CPU fallback")
        return dev

    def _get_tensor(self, weight_name):
        return self.source.get(weight_name)

    # ------------------------------------------------------ packed upload ----
    def packed_layer(self, layer_id) -> PackedLayer:
        pl = self.packed.get(layer_id)
        if pl is None:
            with self.lock:
                pl = self.packed.get(layer_id)
                if pl is None:
                    pl = self._upload_layer(layer_id)
                    self.packed[layer_id] = pl
        return pl

    def upload(self, layers=None):
        """Upload (and pack) every expert of the given layers (default: all)."""
        for l in (range(self.num_layers) if layers is None else layers):
            self.packed_layer(l)
        if isinstance(self.source, SyntheticSource):
            self.source.close()
        return self

    def _upload_layer(self, layer_id) -> PackedLayer:
        dev = self._require_cuda()
        t0 = time.time()
        E = self.num_experts
        g, gs, u, us, d, ds = self.source.layer_experts(self.layout, layer_id, E, dev)
        experts = ops.pack_experts(g, gs, u, us, d, ds)
        del g, gs, u, us, d, ds
        shared = shared_gate = None
        names = [self.layout.shared_tensor(layer_id, p) for p in ("gate_proj", "up_proj", "down_proj")]
        if all(self.source.has(n) for n in names):
            raw = [self.source.get(n) for n in names]
            if all(self.source.has(n + "_scale_inv") for n in names):
                sc = [self.source.get(n + "_scale_inv") for n in names]
                shared = ops.pack_experts(*[t.to(dev) for t in (raw[0], sc[0], raw[1], sc[1], raw[2], sc[2])])
                shared_gate = self.source.get(self.layout.shared_gate_tensor(layer_id)).to(dev, self.dtype)
                shared_gate = shared_gate.reshape(-1).contiguous()
            elif not any(bool(t.any()) for t in raw):
                shared = None   # an all-zero shared expert contributes exactly nothing
            else:
                raise TurboMoEError(f"layer {layer_id}: shared expert is not FP8 block-scaled")
        torch.cuda.current_stream(dev).synchronize()
        ms = (time.time() - t0) * 1000.0
        per = experts.nbytes() // E
        for e in range(E):
            slot = layer_id * E + e
            self.expert_cache[(layer_id, e)] = slot
            self.expert_metadata[slot] = {"hits": 0, "load_ms": ms / E, "vram_cost": per,
                                          "key": (layer_id, e)}
        self.num_slots = len(self.expert_cache)
        self.ssd_hits += E
        self.load_ms_accum += ms
        return PackedLayer(experts, shared, shared_gate)

    def workspace(self, device=None, top_k=None) -> ops.Workspace:
        dev = torch.device(device or self.DEVICE)
        key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
        ws = self._workspaces.get(key)
        if ws is None:
            pl = self.packed_layer(0)
            Is = pl.shared.inter if pl.shared is not None else 0
            ws = ops.Workspace(dev, self.num_experts, top_k or self.top_k, pl.experts.hidden,
                               pl.experts.inter, Is)
            self._workspaces[key] = ws
        return ws

    # ---------------------------------------------- reference interface ----
    def load_weight(self, weight_name, device=None, dtype=None):
        """Tensor by name on the device; FP8 tensors with a ``_scale_inv`` are
        dequantised by K0 with the reference's arithmetic (:89-114)."""
        dev = self._require_cuda(device)
        dtype = dtype or self.dtype
        t = self._get_tensor(weight_name)
        scale_name = f"{weight_name}_scale_inv"
        if self.source.has(scale_name):
            return ops.dequant_fp8_block(t.to(dev), self._get_tensor(scale_name).to(dev), dtype)
        return t.to(device=dev, dtype=dtype)

    def load_weight_raw(self, weight_name, device=None):
        dev = self._require_cuda(device)
        t = self._get_tensor(weight_name).to(dev)
        scale_name = f"{weight_name}_scale_inv"
        if self.source.has(scale_name):
            return t, self._get_tensor(scale_name).to(dev)
        return t, None

    def dequantize_weight(self, w_fp8, scale, dtype=None):
        dtype = dtype or self.dtype
        if scale is None:
            return w_fp8.to(dtype=dtype)
        self._require_cuda(w_fp8.device)
        return ops.dequant_fp8_block(w_fp8, scale.to(w_fp8.device), dtype)

    def load_weight_split(self, weight_name, device=None, dtype=None):
        t0 = time.time()
        w, s = self.load_weight_raw(weight_name, device)
        copy_ms = (time.time() - t0) * 1000.0
        t1 = time.time()
        out = self.dequantize_weight(w, s, dtype)
        return out, copy_ms, (time.time() - t1) * 1000.0

    def clear_pinned_slots(self):
        with self.lock:
            self.pinned_slots.clear()

    def adjust_cache_limit(self, max_vram_gb=None, is_decode=True):
        # every expert is resident; the limit is the number of experts
        self.cache_limit = self.num_experts * self.num_layers

    def _expert_hit(self, layer_id, expert_id):
        with self.lock:
            self.gpu_hits += 1
            slot = self.expert_cache.get((layer_id, expert_id))
            if slot is not None:
                self.expert_metadata[slot]["hits"] += 1

    def load_expert(self, layer_id, expert_id, is_decode=True):
        """Dense dequantised (gate [I,H], up [I,H], down [H,I]) in ``dtype``."""
        pl = self.packed_layer(layer_id)
        self._expert_hit(layer_id, expert_id)
        return ops.unpack_expert(pl.experts, expert_id, self.dtype)

    def load_expert_dynamic(self, layer_id, expert_id):
        """Prefill-time expert fetch (loader/expert_loader.py:269-360): fresh
        dense dequantised (gate [I,H], up [I,H], down [H,I]) in ``dtype``,
        outside any slot.  The reference counts a RAM or SSD hit; here every
        expert is resident, so the lookup counts as a GPU hit."""
        pl = self.packed_layer(layer_id)
        with self.lock:
            self.gpu_hits += 1
        return ops.unpack_expert(pl.experts, expert_id, self.dtype)

    def load_expert_raw(self, layer_id, expert_id, is_decode=True):
        p = self.layout.expert_prefix_name(layer_id, expert_id)
        g, gs = self.load_weight_raw(f"{p}.gate_proj.weight")
        u, us = self.load_weight_raw(f"{p}.up_proj.weight")
        d, ds = self.load_weight_raw(f"{p}.down_proj.weight")
        return g, gs, u, us, d, ds

    def close(self):
        with self.lock:
            self.source.close()
            self.expert_cache.clear()
            self.expert_metadata.clear()
            self.packed.clear()
            self._workspaces.clear()
            self.free_slots.clear()
