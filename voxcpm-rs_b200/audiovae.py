"""Host-side mirror of the AudioVAE v2 decoder (reference ``src/audiovae/``), backed by the
CUDA library: ``AudioVae.decode`` (``vae.rs:55-59``)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import check, lib, ptr


class AudioVae:
    """Decoder half of ``AudioVae`` as one library object (``vx_vae``); weights from
    ``synth.vae_weights`` (bf16 conv weights, f32 alphas / biases / SR tables)."""

    def __init__(self, ctx, vcfg, weights=None):
        self.ctx, self.cfg = ctx, vcfg
        self._rates = np.ascontiguousarray(vcfg.decoder_rates, np.int32)
        bnd = vcfg.sr_bin_boundaries or []
        self._bnd = np.ascontiguousarray(bnd if bnd else [0], np.int32)
        s = _lib.VaeConfigC(vcfg.latent_dim, vcfg.decoder_dim, self._rates.ctypes.data_as(C.POINTER(C.c_int)),
                            len(self._rates), int(vcfg.depthwise), int(vcfg.use_noise_block), vcfg.out_sample_rate,
                            self._bnd.ctypes.data_as(C.POINTER(C.c_int)), len(bnd))
        h = C.c_void_p()
        check(lib().vx_vae_create(ctx.h, C.byref(s), C.byref(h)), ctx.h)
        self.h = h
        ctx._adopt(self)
        if weights is not None:
            self.load(weights)

    def load(self, w):
        L = lib()
        keep = []

        def a(x, dt=None):
            arr = np.ascontiguousarray(x, dtype=dt) if dt else np.ascontiguousarray(x)
            keep.append(arr)
            return ptr(arr)
        check(L.vx_vae_load_first(self.h, a(w["first_dw_w"]), a(w["first_dw_b"], np.float32), a(w["first_pw_w"]),
                                  a(w["first_pw_b"], np.float32)), self.ctx.h)
        for i, blk in enumerate(w["blocks"]):
            bw = _lib.VaeBlockWeightsC()
            bw.alpha, bw.up_w, bw.up_b = a(blk["alpha"], np.float32), a(blk["up_w"]), a(blk["up_b"], np.float32)
            for u, r in enumerate(blk["res"]):
                bw.res_alpha1[u] = a(r["alpha1"], np.float32)
                bw.res_w1[u] = a(r["w1"])
                bw.res_b1[u] = a(r["b1"], np.float32)
                bw.res_alpha2[u] = a(r["alpha2"], np.float32)
                bw.res_w2[u] = a(r["w2"])
                bw.res_b2[u] = a(r["b2"], np.float32)
            if w.get("sr_cond"):
                bw.sr_scale = a(w["sr_cond"][i]["scale"], np.float32)
                bw.sr_bias = a(w["sr_cond"][i]["bias"], np.float32)
            check(L.vx_vae_load_block(self.h, i, C.byref(bw)), self.ctx.h)
        check(L.vx_vae_load_out(self.h, a(w["alpha_out"], np.float32), a(w["last_w"]), a(w["last_b"], np.float32)),
              self.ctx.h)

    def decode(self, z):
        """z [B, latent, T] (torch CUDA f32) -> wav [B, 1, T * prod(rates)]."""
        import torch
        b, _, t = z.shape
        hop = int(np.prod(self._rates))
        out = torch.empty(b, 1, t * hop, device=z.device, dtype=torch.float32)
        torch.cuda.synchronize()
        check(lib().vx_vae_decode(self.h, ptr(z.contiguous()), b, t, ptr(out)), self.ctx.h)
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().vx_vae_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class AudioVaeStream:
    """Stateful chunked decoding of B utterances (``vx_vae_stream``): each ``decode`` of T new
    latent frames returns exactly the samples that decoding the whole latent would give for
    them; ``reset`` starts new utterances."""

    def __init__(self, vae, B=1):
        self.vae, self.ctx, self.B = vae, vae.ctx, B
        h = C.c_void_p()
        check(lib().vx_vae_stream_create(vae.h, B, C.byref(h)), self.ctx.h)
        self.h = h
        self.ctx._adopt(self)

    def reset(self):
        check(lib().vx_vae_stream_reset(self.h), self.ctx.h)

    def decode(self, z):
        """z [B, latent, T] (torch CUDA f32) -> wav [B, 1, T * prod(rates)]."""
        import torch
        b, _, t = z.shape
        hop = int(np.prod(self.vae._rates))
        out = torch.empty(b, 1, t * hop, device=z.device, dtype=torch.float32)
        torch.cuda.synchronize()
        check(lib().vx_vae_stream_decode(self.h, ptr(z.contiguous()), t, ptr(out)), self.ctx.h)
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().vx_vae_stream_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
