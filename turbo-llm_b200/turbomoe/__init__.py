"""turbomoe: Python host side of libturbomoe.so (B200 FP8 MoE kernels).

``turbomoe.synth`` (seeded synthetic checkpoints) imports without the shared
library; ``turbomoe.ops`` loads it on first use and raises if it is missing.
"""
__all__ = ["ops", "synth", "build"]
