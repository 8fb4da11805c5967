"""numpy-f32 restatement of the VoxCPM2 autoregressive model (reference
``src/voxcpm2/model.rs``, ``src/locenc.rs``, ``src/fsq.rs``).

Test infrastructure only (see ``oracle/__init__.py``); parity unpinned.

Weights dict ``w``::

    {"base": MiniCPM dict (with embed), "residual": MiniCPM dict (embed None),
     "encoder": MiniCPM dict (embed None), "dit": LocDiT dict,
     "special": [enc_h], "enc_in_w" [enc_h, D], "enc_in_b",
     "enc_to_lm_w" [H, enc_h], "enc_to_lm_b", "lm_to_dit_w" [dit_h, H], "lm_to_dit_b",
     "res_to_dit_w" [dit_h, H], "res_to_dit_b", "fusion_w" [H, 2H], "fusion_b",
     "stop_proj_w" [H, H], "stop_proj_b", "stop_head_w" [2, H],
     "fsq_in_w" [latent, H], "fsq_in_b", "fsq_out_w" [H, latent], "fsq_out_b"}

``cfgs``: ``{"base", "residual", "encoder", "dit"}`` MiniCPM-4 configs plus
``"patch_size"``, ``"feat_dim"``, ``"sq_scale"``.

The diffusion noise is injected (``noise[i]`` is step i's ``z`` ``[D, P]``) because the
reference draws it from the backend RNG (``src/locdit/unified_cfm.rs:47-52``).
"""
from __future__ import annotations

import numpy as np

from . import locdit as old
from . import minicpm4 as om
from .voxcpm import scalar_quantization

F32 = np.float32


def locenc_forward(ecfg, w, x):
    """``VoxCpmLocEnc::forward`` (``src/locenc.rs:32-44``): x ``[B, T, P, D]`` ->
    ``in_proj`` -> prepend the special token -> non-causal MiniCPM-4 over ``P + 1``
    positions -> the cls row, ``[B, T, enc_h]``."""
    b, t, p, _ = x.shape
    h = om.linear(x.reshape(b * t * p, -1), w["enc_in_w"], w["enc_in_b"]).reshape(b * t, p, -1)
    special = np.broadcast_to(np.asarray(w["special"], F32), (b * t, 1, h.shape[-1]))
    seq = np.concatenate([special, h], axis=1).astype(F32)
    out, _ = om.model_forward(ecfg, w["encoder"], seq, False)
    return out[:, 0].reshape(b, t, -1).astype(F32)


def fsq(w, h, scale):
    """``ScalarQuantizationLayer::forward`` (``src/fsq.rs:24-29``)."""
    return scalar_quantization(h, w["fsq_in_w"], w["fsq_in_b"], w["fsq_out_w"], w["fsq_out_b"], scale)[0]


class State:
    """``InferenceState`` (``src/voxcpm2/model.rs:378-395``)."""

    def __init__(self, lm_hidden, residual_hidden, prefix, base_cache, res_cache, base_rope, res_rope):
        self.lm_hidden = lm_hidden          # [1, H]
        self.residual_hidden = residual_hidden  # [1, H]
        self.prefix = prefix                # [P, D] (prefix_feat_cond)
        self.base_cache, self.res_cache = base_cache, res_cache
        self.base_rope, self.res_rope = base_rope, res_rope


def prefill(cfgs, w, text_token, text_mask, feat, feat_mask, max_len):
    """``VoxCpm2Model::prefill`` (``src/voxcpm2/model.rs:128-207``) for B = 1:
    text_token ``[S]`` ids, masks ``[S]``, feat ``[S, P, D]``."""
    bc, rc = cfgs["base"], cfgs["residual"]
    s = len(text_token)
    feat = np.asarray(feat, F32)
    tm = np.asarray(text_mask, F32)[None, :, None]
    fm = np.asarray(feat_mask, F32)[None, :, None]
    feat_embed = locenc_forward(cfgs["encoder"], w, feat[None])                  # [1, S, enc_h]
    feat_embed = om.linear(feat_embed, w["enc_to_lm_w"], w["enc_to_lm_b"])       # [1, S, H]
    text_embed = om.embed(bc, w["base"], np.asarray(text_token)[None])           # * scale_emb
    combined = (text_embed * tm + feat_embed * fm).astype(F32)
    prefix = feat[s - 1].copy()                                                  # [P, D]
    max_ctx = s + max_len + 1
    base_rope = None if bc.no_rope else om.RopeRows(bc, max_ctx)
    res_rope = None if rc.no_rope else om.RopeRows(rc, max_ctx)
    enc_out, base_kv = om.model_forward(bc, w["base"], combined, True, base_rope)
    enc_out = (fsq(w, enc_out, cfgs["sq_scale"]) * fm + enc_out * tm).astype(F32)
    res_in = om.linear(np.concatenate([enc_out, feat_embed * fm], axis=2).astype(F32), w["fusion_w"], w["fusion_b"])
    res_out, res_kv = om.model_forward(rc, w["residual"], res_in, True, res_rope)
    d = om.head_dim(bc)
    base_cache = om.StaticKvCache(bc.num_hidden_layers, bc.num_key_value_heads, d, 1, max_ctx)
    base_cache.fill(base_kv)
    res_cache = om.StaticKvCache(rc.num_hidden_layers, rc.num_key_value_heads, om.head_dim(rc), 1, max_ctx)
    res_cache.fill(res_kv)
    return State(enc_out[:, s - 1], res_out[:, s - 1], prefix, base_cache, res_cache, base_rope, res_rope)


def stop_logits(w, lm_hidden):
    """``stop_head(silu(stop_proj(lm_hidden)))`` (``src/voxcpm2/model.rs:244-246``)."""
    h = om.silu_stable(om.linear(lm_hidden, w["stop_proj_w"], w["stop_proj_b"]))
    return om.linear(h, w["stop_head_w"])


def dit_step(cfgs, w, st, z, inference_timesteps, cfg_value):
    """``VoxCpm2Model::dit_step`` (``src/voxcpm2/model.rs:215-256``): returns the predicted
    patch ``[D, P]`` (channel-major, as the CFM returns it), the stop flag and the stop
    logits.  z ``[D, P]``."""
    dit1 = om.linear(st.lm_hidden, w["lm_to_dit_w"], w["lm_to_dit_b"])
    dit2 = om.linear(st.residual_hidden, w["res_to_dit_w"], w["res_to_dit_b"])
    mu = np.concatenate([dit1, dit2], axis=1).astype(F32)                       # [1, 2 dit_h]
    cond = st.prefix.T[None]                                                     # [1, D, P]
    pred = old.cfm_forward(cfgs["dit"], w["dit"], mu, inference_timesteps, cond, np.asarray(z, F32)[None],
                           cfg_value, 1.0, True)[0]                              # [D, P]
    st.prefix = pred.T.copy()
    lg = stop_logits(w, st.lm_hidden)[0]
    return pred, om.argmax_first(lg) == 1, lg


def lm_step(cfgs, w, st, pred):
    """``VoxCpm2Model::lm_step`` (``src/voxcpm2/model.rs:261-279``); pred ``[D, P]``."""
    bc, rc = cfgs["base"], cfgs["residual"]
    curr = locenc_forward(cfgs["encoder"], w, pred.T[None, None])                # [1, 1, enc_h]
    curr = om.linear(curr, w["enc_to_lm_w"], w["enc_to_lm_b"])[:, 0]             # [1, H]
    pos = st.base_cache.step()
    lm_hidden = om.model_forward_step(bc, w["base"], curr, pos, st.base_cache, st.base_rope)
    lm_hidden = fsq(w, lm_hidden, cfgs["sq_scale"])
    res_in = om.linear(np.concatenate([lm_hidden, curr], axis=1).astype(F32), w["fusion_w"], w["fusion_b"])
    pos = st.res_cache.step()
    st.residual_hidden = om.model_forward_step(rc, w["residual"], res_in, pos, st.res_cache, st.res_rope)
    st.lm_hidden = lm_hidden


def inference(cfgs, w, text_token, text_mask, feat, feat_mask, min_len, max_len, inference_timesteps, cfg_value,
              noise):
    """``VoxCpm2Model::inference`` (``src/voxcpm2/model.rs:301-375``).  Returns
    ``(latent [D, T*P], stop logits [T, 2])`` where T is the number of patches produced
    (the loop breaks after pushing patch i when ``i > min_len`` and the stop head fires)."""
    st = prefill(cfgs, w, text_token, text_mask, feat, feat_mask, max_len)
    preds, logits = [], []
    for i in range(max_len):
        pred, stop, lg = dit_step(cfgs, w, st, noise[i], inference_timesteps, cfg_value)
        preds.append(pred)
        logits.append(lg)
        if i > min_len and stop:
            break
        lm_step(cfgs, w, st, pred)
    latent = np.concatenate(preds, axis=1).astype(F32)  # stack_pred_feats: [D, T*P]
    return latent, np.stack(logits).astype(F32)
