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
