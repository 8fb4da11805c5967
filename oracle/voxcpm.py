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
