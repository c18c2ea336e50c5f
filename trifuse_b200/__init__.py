"""trifuse_b200: B200-native (sm_100a) OLMoE sparse-MoE forward path.

A drop-in for TriFuse's MLX OLMoE adapter path behind a C ABI
(``include/trifuse_b200.h``, library ``trifuse_b200/lib/libtrifuse_b200.so``).
``trifuse_b200.ops`` mirrors the reference's operator surface;
``trifuse_b200.model`` drives the device-resident model and its sessions.
"""
from ._lib import LIB_PATH, TriFuseError, lib  # noqa: F401

__all__ = ["LIB_PATH", "TriFuseError", "lib"]
