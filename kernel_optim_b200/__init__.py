"""kernel_optim_b200: B200-native (sm_100a) decode attention for the Qwen3-4B engine.

The hot path is the reference's per-layer attention step (GodRishUniverse/kernel_optim,
engine/kernels/fused.py:99-234 as called from engine/engine.py:328-330): QK-norm + RoPE + KV append
and split-K GQA flash-decoding, here one sm_100a launch behind the C ABI in include/kopt.h.
"""

from ._lib import KoptError  # noqa: F401

__all__ = ["KoptError"]
