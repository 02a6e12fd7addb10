"""cev_b200: B200-native kernels and host code for cev's one-pass decision
forward (packed block-masked Qwen3 prefill, Qwen3.5 Gated DeltaNet hybrid,
LFM2 short-conv hybrid), mirroring the reference's model/engine interfaces.
"""
from ._lib import CevkError, lib  # noqa: F401

__all__ = ["CevkError", "lib"]
