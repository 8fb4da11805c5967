"""voxcpm-rs_b200: B200-native (sm_100a) implementation of the voxcpm-rs hot path.

The compute lives in ``libvoxcpm_b200.so`` (hand-written CUDA behind the C ABI in
``include/voxcpm_b200.h``).  The Python modules here mirror the reference crate's
operator surface on top of that ABI through ctypes.  There is no CPU fallback: every
op raises if the CUDA library or a GPU is missing.
"""
from . import config, synth  # noqa: F401

__all__ = ["config", "synth"]
