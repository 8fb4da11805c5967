"""Host-side mirror of LocDiT V2 and the unified CFM sampler (reference
``src/locdit/local_dit.rs``, ``src/locdit/unified_cfm.rs``), backed by the CUDA library."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import check, lib, ptr


class VoxCpmLocDiTV2:
    """``VoxCpmLocDiTV2`` + ``UnifiedCfm`` as one library object (``vx_dit``)."""

    def __init__(self, ctx, dcfg, weights=None, in_channels=64, max_rows=16):
        self.ctx, self.cfg, self.in_channels = ctx, dcfg, in_channels
        s = _lib.config_struct(dcfg)
        h = C.c_void_p()
        check(lib().vx_dit_create(ctx.h, C.byref(s), in_channels, max_rows, C.byref(h)), ctx.h)
        self.h = h
        ctx._adopt(self)
        if weights is not None:
            self.load(weights)

    def load(self, w):
        """Weights from ``synth.locdit_weights`` (bf16 bits + f32 biases)."""
        L = lib()
        a = lambda x, dt=None: np.ascontiguousarray(x, dtype=dt) if dt else np.ascontiguousarray(x)  # noqa: E731
        arrs = [a(w["in_proj_w"]), a(w["in_proj_b"], np.float32), a(w["cond_proj_w"]), a(w["cond_proj_b"], np.float32),
                a(w["out_proj_w"]), a(w["out_proj_b"], np.float32)]
        for name in ("time_mlp", "delta_time_mlp"):
            t = w[name]
            arrs += [a(t["w1"]), a(t["b1"], np.float32), a(t["w2"]), a(t["b2"], np.float32)]
        check(L.vx_dit_load(self.h, *[ptr(x) for x in arrs]), self.ctx.h)
        dec = w["decoder"]
        for i, lw in enumerate(dec["layers"]):
            ls = [a(lw[k]) for k in ("q", "k", "v", "o", "gate", "up", "down")]
            ns = [a(lw[k], np.float32) for k in ("ln_in", "ln_post")]
            check(L.vx_dit_load_layer(self.h, i, *[ptr(x) for x in ls], *[ptr(x) for x in ns]), self.ctx.h)
        check(L.vx_dit_load_norm(self.h, ptr(a(dec["norm"], np.float32))), self.ctx.h)

    def forward(self, x, mu, t, cond, dt):
        """``VoxCpmLocDiTV2::forward``: x [N,C,T], mu [N,C_mu], t/dt [N], cond [N,C,Tc]."""
        import torch
        n, c, tl = x.shape
        out = torch.empty_like(x)
        t = np.ascontiguousarray(t, np.float32)
        dt = np.ascontiguousarray(dt, np.float32)
        torch.cuda.synchronize()
        check(lib().vx_dit_forward(self.h, ptr(x), ptr(mu), ptr(t), ptr(cond), ptr(dt), n, mu.shape[1], tl,
                                   cond.shape[2], ptr(out)), self.ctx.h)
        return out

    def cfm_forward(self, mu, n_timesteps, cond, z, cfg_value, sway_sampling_coef=1.0, use_cfg_zero_star=True):
        """``UnifiedCfm::forward`` with the noise ``z`` [B, C, patch] given (already scaled by
        temperature)."""
        import torch
        b, c, tl = z.shape
        out = torch.empty_like(z)
        torch.cuda.synchronize()
        check(lib().vx_cfm_solve(self.h, ptr(mu), ptr(cond), ptr(z), b, mu.shape[1], tl, cond.shape[2], n_timesteps,
                                 cfg_value, sway_sampling_coef, int(use_cfg_zero_star), ptr(out)), self.ctx.h)
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().vx_dit_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
