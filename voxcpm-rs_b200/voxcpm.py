"""Host-side mirror of ``VoxCPM::generate`` / ``GenerateOptions`` / ``CancelToken``
(reference ``src/voxcpm2/wrapper.rs``) over the library's synthesis loop: greedy MiniCPM-4
decode, a LocDiT CFM solve per step, AudioVAE decode."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import check, lib, ptr


@dataclass
class GenerateOptions:
    """``GenerateOptions`` (``wrapper.rs:146-187``) fields the synthesis loop uses, with the
    reference defaults; ``sway_sampling_coef`` / ``use_cfg_zero_star`` are what ``dit_step``
    passes (``voxcpm2/model.rs:229-238``)."""
    cfg_value: float = 2.0
    inference_timesteps: int = 10
    max_len: int = 2000
    patch_size: int = 4
    sway_sampling_coef: float = 1.0
    use_cfg_zero_star: bool = True

    def to_c(self):
        return _lib.GenerateOptionsC(self.cfg_value, self.inference_timesteps, self.max_len, self.patch_size,
                                     self.sway_sampling_coef, int(self.use_cfg_zero_star))


class CancelToken:
    """``CancelToken`` (``wrapper.rs:47-65``): ``cancel()`` is safe from any thread."""

    def __init__(self, ctx):
        self.ctx = ctx

    def cancel(self):
        self.ctx.cancel()

    def reset(self):
        self.ctx.cancel_reset()


class ScalarQuantizationLayer:
    """``ScalarQuantizationLayer`` (reference ``src/fsq.rs``): ``forward(h)`` =
    ``out_proj(round(tanh(in_proj(h)) * scale) / scale)`` on the device.  Weights are torch
    CUDA tensors: ``w_in`` [latent, in] and ``w_out`` [out, latent] as bf16 bits (int16),
    biases f32 or None."""

    def __init__(self, ctx, w_in, b_in, w_out, b_out, scale=9):
        self.ctx, self.w_in, self.b_in, self.w_out, self.b_out = ctx, w_in, b_in, w_out, b_out
        self.scale = float(scale)
        self.latent_dim, self.in_dim = w_in.shape
        self.out_dim = w_out.shape[0]

    def forward(self, hidden, stream=None):
        import torch
        h = hidden.reshape(-1, self.in_dim).contiguous()
        out = torch.empty(h.shape[0], self.out_dim, device=h.device, dtype=torch.float32)
        check(lib().vx_fsq(self.ctx.h, ptr(self.w_in), ptr(self.b_in), ptr(self.w_out), ptr(self.b_out), self.in_dim,
                           self.latent_dim, self.out_dim, self.scale, ptr(h), h.shape[0], ptr(out), stream), self.ctx.h)
        return out.reshape(*hidden.shape[:-1], self.out_dim)


class VoxCPM:
    """Owns the LM (``MiniCpmModel``), the DiT (``VoxCpmLocDiTV2``) and the VAE
    (``AudioVae``) objects on one context."""

    def __init__(self, ctx, lm, dit, vae):
        self.ctx, self.lm, self.dit, self.vae = ctx, lm, dit, vae

    def generate(self, prompt_ids, opts: GenerateOptions, noise, return_latent=False):
        """``VoxCPM::generate`` with token ids instead of text and the diffusion noise given:
        noise [max_len, C, patch_size] (float32, ~N(0,1) * temperature).  Returns the mono
        waveform (and the stacked latent [C, max_len*patch_size])."""
        ids = np.ascontiguousarray(prompt_ids, np.int32)
        noise = np.ascontiguousarray(noise, np.float32)
        c = self.dit.in_channels
        frames = opts.max_len * opts.patch_size
        hop = int(np.prod(self.vae.cfg.decoder_rates))
        wav = np.empty(frames * hop, np.float32)
        latent = np.empty((c, frames), np.float32) if return_latent else None
        o = opts.to_c()
        check(lib().vx_generate(self.lm.h, self.dit.h, self.vae.h, ptr(ids), len(ids), C.byref(o), ptr(noise),
                                ptr(wav), ptr(latent)), self.ctx.h)
        return (wav, latent) if return_latent else wav

    def generate_batch(self, prompt_ids, opts: GenerateOptions, noise, return_latent=False):
        """B utterances at once (``vx_generate_batch``): prompt_ids [B, n] (equal lengths),
        noise [B, max_len, C, patch_size].  Returns wav [B, samples] (and latents
        [B, C, max_len*patch_size]).  The LM needs max_batch >= B, the DiT max_rows >= 2B."""
        ids = np.ascontiguousarray(prompt_ids, np.int32)
        b, n = ids.shape
        noise = np.ascontiguousarray(noise, np.float32)
        c = self.dit.in_channels
        frames = opts.max_len * opts.patch_size
        hop = int(np.prod(self.vae.cfg.decoder_rates))
        wav = np.empty((b, frames * hop), np.float32)
        latent = np.empty((b, c, frames), np.float32) if return_latent else None
        o = opts.to_c()
        check(lib().vx_generate_batch(self.lm.h, self.dit.h, self.vae.h, ptr(ids), b, n, C.byref(o), ptr(noise),
                                      ptr(wav), ptr(latent)), self.ctx.h)
        return (wav, latent) if return_latent else wav


class VoxCpm2Model:
    """``VoxCpm2Model`` (reference ``src/voxcpm2/model.rs``): base LM, residual LM, local
    encoder, LocDiT, FSQ and projection layers on one context (``vx_voxcpm2``).  ``inference``
    is ``VoxCpm2Model::inference`` with the per-step CFM noise given; ``generate`` adds the
    AudioVAE decode (``VoxCPM::generate`` without the tokenizer)."""

    def __init__(self, ctx, vcfg, weights=None, max_len=64, max_length=None):
        from .locdit import VoxCpmLocDiTV2
        from .minicpm4 import MiniCpmModel
        self.ctx, self.cfg = ctx, vcfg
        max_length = max_length or vcfg.max_length
        self.base = MiniCpmModel(ctx, vcfg.lm_config, None, max_length=max_length)
        self.residual = MiniCpmModel(ctx, vcfg.residual_lm_config(), None, max_length=max_length)
        self.encoder = MiniCpmModel(ctx, vcfg.encoder_lm_config(), None, max_length=vcfg.patch_size + 1)
        self.dit = VoxCpmLocDiTV2(ctx, vcfg.dit_lm_config(), None, in_channels=vcfg.feat_dim, max_rows=2)
        h = C.c_void_p()
        check(lib().vx_voxcpm2_create(self.base.h, self.residual.h, self.encoder.h, self.dit.h, vcfg.feat_dim,
                                      vcfg.patch_size, vcfg.scalar_quantization_latent_dim,
                                      vcfg.scalar_quantization_scale, max_len, C.byref(h)), ctx.h)
        self.h = h
        ctx._adopt(self)
        self.max_len = max_len
        if weights is not None:
            self.load(weights)

    def load(self, w):
        """Weights from ``synth.voxcpm2_weights``."""
        self.base.load(w["base"])
        self.residual.load(w["residual"])
        self.encoder.load(w["encoder"])
        self.dit.load(w["dit"])
        names = [f for f, _ in _lib.VoxCpm2WeightsC._fields_]
        src = {"special_token": w["special"]}
        src.update({n: w[n] for n in names if n != "special_token"})
        keep = {n: np.ascontiguousarray(v, dtype=np.float32 if v.dtype != np.uint16 else np.uint16)
                for n, v in src.items()}
        s = _lib.VoxCpm2WeightsC(*[ptr(keep[n]) for n in names])
        check(lib().vx_voxcpm2_load(self.h, C.byref(s)), self.ctx.h)

    def locenc(self, feat):
        """``VoxCpmLocEnc::forward`` of N patches: feat [N, P, D] -> [N, enc_hidden]."""
        import torch
        x = torch.as_tensor(np.ascontiguousarray(feat, np.float32)).cuda(self.ctx.device)
        out = torch.empty(x.shape[0], self.encoder.cfg.hidden_size, device=x.device)
        torch.cuda.synchronize()
        check(lib().vx_locenc_forward(self.h, ptr(x), x.shape[0], ptr(out)), self.ctx.h)
        return out.cpu().numpy()

    def inference(self, text_token, text_mask, feat, feat_mask, min_len, max_len, inference_timesteps, cfg_value,
                  noise):
        """Returns ``(latent [D, n*P], stop logits [n, 2])``."""
        ids = np.ascontiguousarray(text_token, np.int32)
        tm = np.ascontiguousarray(text_mask, np.float32)
        fm = np.ascontiguousarray(feat_mask, np.float32)
        feat = np.ascontiguousarray(feat, np.float32)
        noise = np.ascontiguousarray(noise, np.float32)
        D, P = self.cfg.feat_dim, self.cfg.patch_size
        lat = np.empty((D, max_len * P), np.float32)
        logits = np.empty((max_len, 2), np.float32)
        n = C.c_int()
        check(lib().vx_voxcpm2_inference(self.h, ptr(ids), ptr(tm), ptr(feat), ptr(fm), len(ids), min_len, max_len,
                                         inference_timesteps, cfg_value, ptr(noise), ptr(lat), C.byref(n),
                                         ptr(logits)), self.ctx.h)
        k = n.value
        return np.ascontiguousarray(lat.reshape(-1)[:D * k * P].reshape(D, k * P)), logits[:k]

    def generate(self, vae, text_token, text_mask, feat, feat_mask, min_len, max_len, inference_timesteps,
                 cfg_value, noise):
        ids = np.ascontiguousarray(text_token, np.int32)
        noise = np.ascontiguousarray(noise, np.float32)
        hop = int(np.prod(vae.cfg.decoder_rates))
        wav = np.empty(max_len * self.cfg.patch_size * hop, np.float32)
        n = C.c_int()
        check(lib().vx_voxcpm2_generate(self.h, vae.h, ptr(ids), ptr(np.ascontiguousarray(text_mask, np.float32)),
                                        ptr(np.ascontiguousarray(feat, np.float32)),
                                        ptr(np.ascontiguousarray(feat_mask, np.float32)), len(ids), min_len, max_len,
                                        inference_timesteps, cfg_value, ptr(noise), ptr(wav), C.byref(n)),
              self.ctx.h)
        return wav[:n.value]

    def generate_stream(self, vae, text_token, text_mask, feat, feat_mask, min_len, max_len, inference_timesteps,
                        cfg_value, noise, chunk_patches=5):
        """``VoxCPM::generate_stream`` (``wrapper.rs:456-492, 680-724``): yields mono audio
        chunks as AR steps complete, ``chunk_patches`` patches at a time; each chunk is decoded
        by a stateful AudioVAE stream (only the new frames), so the concatenated chunks equal
        ``generate``'s waveform."""
        import torch
        from .audiovae import AudioVaeStream
        ids = np.ascontiguousarray(text_token, np.int32)
        noise = np.ascontiguousarray(noise, np.float32)
        check(lib().vx_voxcpm2_begin(self.h, ptr(ids), ptr(np.ascontiguousarray(text_mask, np.float32)),
                                     ptr(np.ascontiguousarray(feat, np.float32)),
                                     ptr(np.ascontiguousarray(feat_mask, np.float32)), len(ids), min_len, max_len,
                                     inference_timesteps, cfg_value, ptr(noise)), self.ctx.h)
        D, P = self.cfg.feat_dim, self.cfg.patch_size
        stream = AudioVaeStream(vae, 1)
        try:
            lat = torch.empty(D * chunk_patches * P, device=f"cuda:{self.ctx.device}")
            n, fin = C.c_int(), C.c_int(0)
            while not fin.value:
                torch.cuda.synchronize()
                check(lib().vx_voxcpm2_advance(self.h, chunk_patches, ptr(lat), C.byref(n), C.byref(fin)),
                      self.ctx.h)
                if n.value:
                    z = lat[:D * n.value * P].reshape(1, D, n.value * P)
                    yield stream.decode(z).reshape(-1).cpu().numpy()
        finally:
            stream.close()

    def close(self):
        if getattr(self, "h", None):
            lib().vx_voxcpm2_destroy(self.h)
            self.h = None
        for m in ("dit", "encoder", "residual", "base"):
            if getattr(self, m, None) is not None:
                getattr(self, m).close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
