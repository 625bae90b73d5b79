"""Host RAM tier of the expert cache: the interface of the reference's
cache/ram_cache.py:6-101, kept for the engine and the backend, which read
``stats()`` (runtime/engine.py:327-337, backend/api/routes/metrics.py:52,101).

With every expert of every layer packed once into device memory
(``ExpertLoader.upload``), no expert is ever staged in host RAM: the MoE path
has no RAM or SSD miss to serve.  So this tier holds nothing.  ``put`` is
accepted and dropped, ``get`` always misses, and ``stats()`` reports an empty
cache against the reference's byte budget (a percentage of available RAM,
``memory.max_ram_percent``, default 35).
"""
from __future__ import annotations

import psutil


class RAMCache:

    def __init__(self, config=None):
        self.config = config
        self.current = 0
        self.max_bytes = self.compute_limit()

    def compute_limit(self):
        pct = 35
        if self.config and "memory" in self.config and "max_ram_percent" in self.config["memory"]:
            pct = self.config["memory"]["max_ram_percent"]
        return int(psutil.virtual_memory().available * (pct / 100.0))

    def get(self, key):
        return None

    def put(self, key, value):
        return None

    def clear(self):
        self.current = 0

    def stats(self):
        return {"entries": 0, "current_bytes": 0, "max_bytes": self.max_bytes, "usage_percent": 0.0}

    def __contains__(self, key):
        return False

    def __len__(self):
        return 0
