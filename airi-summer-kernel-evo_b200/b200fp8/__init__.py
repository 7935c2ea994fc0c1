"""b200fp8 — B200-native FP8 kernel library (tcgen05 / TMA / TMEM, sm_100a).

Host side of the hot path of bulatsharif/airi-summer-kernel-evo's FP8 task suite: e4m3
GEMMs with fused epilogues, fused attention, residual+norm+quantise, and the GPT-2 /
Qwen decoder blocks built from them.  Every op calls libb200fp8.so; there is no CPU
or library fallback.
"""
from . import _lib  # noqa: F401
from ._lib import B2FError, device_status  # noqa: F401

__all__ = ["B2FError", "device_status"]
