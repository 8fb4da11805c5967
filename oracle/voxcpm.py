"""numpy-f32 restatement of the end-to-end synthesis loop this library runs, shaped like
``VoxCpm2Model::inference`` (reference ``src/voxcpm2/model.rs:301-375``) and
``VoxCPM::generate`` (``src/voxcpm2/wrapper.rs:401-423``).

Test infrastructure only (see ``oracle/__init__.py``); parity unpinned.

Step i: greedy MiniCPM-4 decode step i (``minicpm4.greedy_generate``), then
``UnifiedCfm::forward`` with mu = the step's final-norm hidden, cond = the previous patch
(zeros first, ``model.rs:233,241``) and the given noise; patches are stacked
(``stack_pred_feats``, ``model.rs:283-287``) and decoded by the AudioVAE.
"""
from __future__ import annotations

import numpy as np

from . import audiovae as oav
from . import locdit as old
from . import minicpm4 as om

F32 = np.float32


def generate(lm_cfg, lm_w, dit_cfg, dit_w, vae_cfg, vae_w, prompt_ids, max_len, noise, inference_timesteps=10,
             cfg_value=2.0, sway_sampling_coef=1.0, use_cfg_zero_star=True, patch_size=4):
    """Returns ``(wav [max_len*P*hop], latent [C, max_len*P], token ids)``."""
    toks, hiddens = om.greedy_generate(lm_cfg, lm_w, prompt_ids, max_len, len(prompt_ids) + max_len + 1,
                                       return_hidden=True)
    c = noise.shape[1]
    cond = np.zeros((1, c, patch_size), F32)
    patches = []
    for i in range(max_len):
        mu = hiddens[i + 1][None].astype(F32)  # final-norm hidden after decode step i+1
        x = old.cfm_forward(dit_cfg, dit_w, mu, inference_timesteps, cond, noise[i][None], cfg_value,
                            sway_sampling_coef, use_cfg_zero_star)
        patches.append(x[0])
        cond = x
    latent = np.concatenate(patches, axis=1)  # [C, T*P]: latent[:, i*P + p] = patch_i[:, p]
    wav = oav.decoder_forward(vae_cfg, vae_w, latent[None])[0, 0]
    return wav, latent, toks


def round_half_away(x):
    """Rust ``f32::round`` (ties away from zero), elementwise in f32."""
    x = np.asarray(x, F32)
    return (np.sign(x) * np.floor(np.abs(x) + F32(0.5))).astype(F32)


def scalar_quantization(h, w_in, b_in, w_out, b_out, scale):
    """``ScalarQuantizationLayer::forward`` (reference ``src/fsq.rs:24-29``):
    ``out_proj(round(tanh(in_proj(h)) * scale) / scale)``; ``w_*`` in the ``[out, in]``
    layout (f32 copies of the bf16 weights), biases may be None.  Also returns the
    pre-rounding values ``tanh(in_proj(h)) * scale`` so callers can check tie margins."""
    h = np.asarray(h, F32)
    lat = h @ np.asarray(w_in, F32).T
    if b_in is not None:
        lat = lat + np.asarray(b_in, F32)
    pre = (np.tanh(lat.astype(F32)) * F32(scale)).astype(F32)
    q = (round_half_away(pre) / F32(scale)).astype(F32)
    out = q @ np.asarray(w_out, F32).T
    if b_out is not None:
        out = out + np.asarray(b_out, F32)
    return out.astype(F32), pre
