"""Host LRU cache of raw FP8 expert tuples (interface of the reference's
cache/ram_cache.py:6-101, kept for callers that read its stats).

With the packed, fully device-resident expert layout the MoE path never
streams experts from host memory, so the loader only uses this cache as a
staging record; the eviction policy (least recently used, byte budget of a
percentage of available RAM) is the reference's.
"""
from __future__ import annotations

from collections import OrderedDict

import psutil


class RAMCache:

    def __init__(self, config=None):
        self.cache = OrderedDict()
        self.current = 0
        self.config = config
        self.max_bytes = self.compute_limit()

    def compute_limit(self):
        pct = 35
        if self.config and "memory" in self.config and "max_ram_percent" in self.config["memory"]:
            pct = self.config["memory"]["max_ram_percent"]
        return int(psutil.virtual_memory().available * (pct / 100.0))

    @staticmethod
    def _size(value):
        if isinstance(value, (list, tuple)):
            return sum(t.numel() * t.element_size() for t in value if t is not None)
        return value.numel() * value.element_size()

    def get(self, key):
        if key not in self.cache:
            return None
        self.cache.move_to_end(key)
        return self.cache[key][0]

    def put(self, key, value):
        size = self._size(value)
        if size > self.max_bytes:
            return
        if key in self.cache:
            self.current -= self.cache.pop(key)[1]
        while self.current + size > self.max_bytes and self.cache:
            _, (_, old) = self.cache.popitem(last=False)
            self.current -= old
        self.cache[key] = (value, size)
        self.current += size

    def clear(self):
        self.cache.clear()
        self.current = 0

    def stats(self):
        return {"entries": len(self.cache), "current_bytes": self.current, "max_bytes": self.max_bytes,
                "usage_percent": 100 * self.current / self.max_bytes if self.max_bytes else 0}

    def __contains__(self, key):
        return key in self.cache

    def __len__(self):
        return len(self.cache)
