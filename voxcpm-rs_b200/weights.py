"""Checkpoint ingestion (reference ``src/weights.rs``): ``Checkpoint`` opens a
``.safetensors`` file or a PyTorch zip checkpoint (``.pth`` / ``.pt``) through the library
(host-side parsing, memory-mapped), and ``load_pretrained`` fills the model objects from an
upstream snapshot directory the way ``load_pretrained`` (``weights.rs:56-133``) does:
``model.safetensors`` (else ``model.pth`` / ``model.pt``) and ``audiovae.safetensors`` (else
``audiovae.pth``)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import lib, ptr

DT_F32, DT_F16, DT_BF16, DT_F64, DT_I64, DT_I32, DT_I16, DT_I8, DT_U8, DT_BOOL = range(10)
DT_NAMES = {DT_F32: "F32", DT_F16: "F16", DT_BF16: "BF16", DT_F64: "F64", DT_I64: "I64", DT_I32: "I32",
            DT_I16: "I16", DT_I8: "I8", DT_U8: "U8", DT_BOOL: "BOOL"}


def _check(rc):
    if rc != 0:
        raise _lib.VxError(rc, lib().vx_weights_last_error().decode())


class Checkpoint:
    """A checkpoint file opened on the host (``vx_weights``)."""

    def __init__(self, path):
        h = C.c_void_p()
        _check(lib().vx_weights_open(os.fsencode(path), C.byref(h)))
        self.h = h

    def names(self):
        L = lib()
        return [L.vx_weights_name(self.h, i).decode() for i in range(L.vx_weights_count(self.h))]

    def info(self, name):
        """``(dtype name, shape)`` of a stored tensor."""
        i = lib().vx_weights_find(self.h, name.encode())
        if i < 0:
            raise KeyError(name)
        dt = C.c_int()
        shape = (C.c_int64 * 8)()
        nd = lib().vx_weights_info(self.h, i, C.byref(dt), shape, 8)
        return DT_NAMES[dt.value], tuple(shape[:nd])

    def read(self, name, shape, dtype="f32"):
        """Tensor ``name`` (or its materialised weight_norm pair) as f32, or as bf16 bits
        (uint16) with ``dtype="bf16"``."""
        out = np.empty(shape, np.float32 if dtype == "f32" else np.uint16)
        _check(lib().vx_weights_read(self.h, name.encode(), DT_F32 if dtype == "f32" else DT_BF16, ptr(out),
                                     out.size))
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().vx_weights_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _first(d, names):
    for n in names:
        p = os.path.join(d, n)
        if os.path.exists(p):
            return p
    return None


def load_pretrained(model, snapshot_dir, vae=None):
    """Load a VoxCPM2 snapshot directory into ``model`` (``voxcpm.VoxCpm2Model``) and, if
    given, ``vae`` (``audiovae.AudioVae``)."""
    from ._lib import check
    mp = _first(snapshot_dir, ["model.safetensors", "model.pth", "model.pt"])
    if mp is None:
        raise FileNotFoundError(f"no model weights in {snapshot_dir} (expected model.safetensors or model.pth)")
    with Checkpoint(mp) as ck:
        check(lib().vx_voxcpm2_load_weights(model.h, ck.h), model.ctx.h)
    if vae is not None:
        vp = _first(snapshot_dir, ["audiovae.safetensors", "audiovae.pth"])
        if vp is None:
            raise FileNotFoundError(f"no audiovae weights in {snapshot_dir}")
        with Checkpoint(vp) as ck:
            check(lib().vx_vae_load_weights(vae.h, ck.h, None), vae.ctx.h)
