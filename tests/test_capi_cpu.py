"""CPU-side checks of the C ABI: the library builds, loads and exports every symbol the
header declares; the host-only entry points (LongRoPE table) match the oracle; device
entry points fail cleanly (no crash) when no GPU is present."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from oracle import minicpm4 as om

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "voxcpm_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vx_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("vx_ctx_create", "vx_rmsnorm_residual", "vx_attention_decode", "vx_lm_greedy", "vx_cfg_euler"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from voxcpm_rs_b200 import _lib
    L = _lib.lib()
    missing = [n for n in _declared() if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"
    # and every declared symbol has a ctypes signature in the binding
    assert set(_declared()) <= set(_lib.SIGNATURES), set(_declared()) - set(_lib.SIGNATURES)


def test_version():
    from voxcpm_rs_b200._lib import lib
    assert lib().vx_version() >= 100


@pytest.mark.parametrize("max_pos", [32768, 65536, 16384])
def test_longrope_table_host(max_pos):
    """vx_longrope_table (host code) vs the oracle's f64 table (rope.rs:16-54)."""
    from voxcpm_rs_b200 import config
    from voxcpm_rs_b200.minicpm4 import longrope_table
    cfg = config.lm_decode_config(layers=1, vocab=0, max_position_embeddings=max_pos)
    cos, sin = longrope_table(cfg, 4096)
    cr, sr = om.longrope_table(cfg, 4096)
    assert np.abs(cos - cr).max() <= 1e-7 and np.abs(sin - sr).max() <= 1e-7


def test_longrope_factor_length_checked():
    """rope.rs:32 asserts len(factors) == head_dim/2; the ABI returns InvalidConfig."""
    from voxcpm_rs_b200 import _lib, config
    cfg = config.lm_decode_config(layers=1, vocab=0)
    cfg.rope_scaling.short_factor = cfg.rope_scaling.short_factor[:10]
    s = _lib.config_struct(cfg)
    out = np.empty((4, 128), np.float32)
    assert _lib.lib().vx_longrope_table(C.byref(s), 4, out.ctypes.data, out.ctypes.data) == _lib.VX_ERR_CONFIG


def test_ctx_create_without_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from voxcpm_rs_b200._lib import VX_ERR_NO_DEVICE, lib
    h = C.c_void_p()
    assert lib().vx_ctx_create(0, C.byref(h)) == VX_ERR_NO_DEVICE
    assert h.value is None


def test_null_arguments_rejected():
    from voxcpm_rs_b200._lib import VX_ERR_ARG, lib
    assert lib().vx_rmsnorm_residual(None, None, None, None, 1.0, 1e-6, 1, 4, None, None, None) == VX_ERR_ARG
    assert lib().vx_lm_greedy(None, None, 0, 0, None) == VX_ERR_ARG


def test_context_close_destroys_its_objects_first(monkeypatch):
    """Closing a Context destroys the library objects created on it before the context
    itself, so an object that outlives its context (a failed test's local, a dropped
    reference) never reaches a freed vx_ctx.  Runs on a recording stand-in for the library."""
    from voxcpm_rs_b200 import _lib, audiovae, locdit, minicpm4

    calls = []

    class Fake:
        def __getattr__(self, name):
            def fn(*args):
                calls.append(name)
                return 0
            return fn

    fake = Fake()
    for mod in (_lib, minicpm4, locdit, audiovae):
        monkeypatch.setattr(mod, "lib", lambda: fake)
    monkeypatch.setattr(_lib, "config_struct", lambda cfg: C.c_int(0))
    ctx = minicpm4.Context(0)
    ctx.h = C.c_void_p(1)
    m = minicpm4.MiniCpmModel(ctx, cfg=None)
    m.h = C.c_void_p(2)
    ctx.close()
    assert calls.index("vx_lm_destroy") < calls.index("vx_ctx_destroy")
    assert m.h is None and ctx.h is None
    m.close()  # a second close after the context is gone touches nothing
    assert calls.count("vx_lm_destroy") == 1
