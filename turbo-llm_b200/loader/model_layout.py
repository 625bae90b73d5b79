"""Checkpoint tensor naming (drop-in for the reference's loader/model_layout.py).

Reads ``config.json`` and ``model.safetensors.index.json`` of a snapshot and
derives the names the MoE path needs.  Same rules as the reference
(loader/model_layout.py:34-88): the layer prefix is the part before
``.<layer>.mlp.experts.<e>.gate_proj.weight``; the router is the first
``<prefix>.0.mlp.<name>.weight`` whose ``<name>`` has no dot and is not a
gate/up/down projection.
"""
from __future__ import annotations

import json
import os
import re

_EXPERT_RE = re.compile(r"(.*)\.(\d+)\.mlp\.experts\.(\d+)\.gate_proj\.weight")


class ModelLayout:

    def __init__(self, snapshot_path, config=None, weight_map=None):
        self.snapshot_path = snapshot_path
        if config is None:
            with open(os.path.join(snapshot_path, "config.json")) as f:
                config = json.load(f)
        if weight_map is None:
            with open(os.path.join(snapshot_path, "model.safetensors.index.json")) as f:
                weight_map = json.load(f)["weight_map"]
        self.config = config
        self.weight_map = weight_map
        self.model_type = config.get("model_type", "unknown")
        self.layer_prefix = None
        self.expert_prefix = None
        self.gate_name = self.up_name = self.down_name = None
        self.router_name = None
        self._detect_layout()

    def _detect_layout(self):
        for name in self.weight_map:
            m = _EXPERT_RE.match(name)
            if m:
                self.layer_prefix = m.group(1)
                self.expert_prefix = "mlp.experts"
                self.gate_name, self.up_name, self.down_name = "gate_proj", "up_proj", "down_proj"
                break
        if self.layer_prefix is None:
            raise RuntimeError(f"Unsupported model layout ({self.model_type})")
        head = f"{self.layer_prefix}.0.mlp."
        projections = {self.gate_name, self.up_name, self.down_name}
        for name in self.weight_map:
            if not name.startswith(head) or not name.endswith(".weight"):
                continue
            stem = name[len(head):-len(".weight")]
            if "." in stem or stem in projections:
                continue
            self.router_name = stem
            break
        if self.router_name is None:
            raise RuntimeError("Could not detect router tensor.")

    # --- names (reference loader/model_layout.py:90-149) ---
    def expert_prefix_name(self, layer, expert):
        return f"{self.layer_prefix}.{layer}.{self.expert_prefix}.{expert}"

    def gate_tensor(self, layer, expert):
        return f"{self.expert_prefix_name(layer, expert)}.{self.gate_name}.weight"

    def up_tensor(self, layer, expert):
        return f"{self.expert_prefix_name(layer, expert)}.{self.up_name}.weight"

    def down_tensor(self, layer, expert):
        return f"{self.expert_prefix_name(layer, expert)}.{self.down_name}.weight"

    def router_tensor(self, layer):
        return f"{self.layer_prefix}.{layer}.mlp.{self.router_name}.weight"

    def shared_tensor(self, layer, proj):
        return f"{self.layer_prefix}.{layer}.mlp.shared_expert.{proj}.weight"

    def shared_gate_tensor(self, layer):
        return f"{self.layer_prefix}.{layer}.mlp.shared_expert_gate.weight"

    def embed_tensor(self):
        if self.layer_prefix.startswith("model.language_model"):
            return "model.language_model.embed_tokens.weight"
        return "model.embed_tokens.weight"

    def norm_tensor(self):
        if self.layer_prefix.startswith("model.language_model"):
            return "model.language_model.norm.weight"
        return "model.norm.weight"

    def lm_head_tensor(self):
        return "lm_head.weight"

    def layer_prefix_name(self, layer):
        return f"{self.layer_prefix}.{layer}"

    def module_name(self, tensor_name):
        if tensor_name.startswith("model.language_model."):
            return tensor_name.replace("model.language_model.", "model.", 1)
        return tensor_name

    # --- layer / expert counts (used to size the one-time upload) ---
    def num_experts(self):
        n = self.config.get("num_experts") or self.config.get("n_routed_experts")
        if n:
            return int(n)
        head = f"{self.layer_prefix}.0.mlp.experts."
        ids = {int(k[len(head):].split(".")[0]) for k in self.weight_map if k.startswith(head)}
        return max(ids) + 1

    def num_layers(self):
        n = self.config.get("num_hidden_layers")
        if n:
            return int(n)
        pat = re.compile(re.escape(self.layer_prefix) + r"\.(\d+)\.mlp\.")
        return 1 + max(int(m.group(1)) for k in self.weight_map for m in [pat.match(k)] if m)
