"""numpy-f32 restatement of LocDiT V2 and the unified CFM sampler
(reference ``src/locdit/local_dit.rs`` and ``src/locdit/unified_cfm.rs``).

Test infrastructure only (see ``oracle/__init__.py``); parity unpinned.

A DiT is a dict ``{"in_proj_w", "in_proj_b", "cond_proj_w", "cond_proj_b",
"out_proj_w", "out_proj_b", "time_mlp": {"w1","b1","w2","b2"},
"delta_time_mlp": {...}, "decoder": <MiniCPM model dict, embed None>}``.
"""
from __future__ import annotations

import math

import numpy as np

from . import minicpm4 as m4

F32 = np.float32


def sinusoidal_pos_emb(x, dim, scale):
    """``SinusoidalPosEmb::forward`` (``src/locdit/local_dit.rs:24-32``).

    ``freqs_i = exp(-ln(1e4) * i / (half - 1))`` in f64 rounded to f32;
    ``angles = (x * scale) * freqs``; returns ``[sin(angles), cos(angles)]`` ``[N, dim]``.
    """
    half = dim // 2
    emb_scale = math.log(10000.0) / (half - 1.0)
    freqs = np.exp(-emb_scale * np.arange(half, dtype=np.float64)).astype(F32)
    ang = (np.asarray(x, F32)[:, None] * F32(scale)) * freqs[None, :]
    return np.concatenate([np.sin(ang), np.cos(ang)], axis=1).astype(F32)


def timestep_embedding(tw, sample):
    """``TimestepEmbedding::forward`` (``src/locdit/local_dit.rs:50-54``)."""
    h = m4.linear(sample, tw["w1"], tw["b1"])
    return m4.linear(m4.silu_stable(h), tw["w2"], tw["b2"])


def dit_prepare(dcfg, dw, mu, cond, dt):
    """``VoxCpmLocDiTV2::prepare`` (``src/locdit/local_dit.rs:116-134``).

    mu ``[N, C_mu]``, cond ``[N, C, T']``, dt ``[N]``.  Returns the cached
    ``(mu [N, mu_tokens, H], cond [N, T', H], dt_emb [N, H])``.
    """
    hidden = dcfg.hidden_size
    condp = m4.linear(np.swapaxes(cond, 1, 2), dw["cond_proj_w"], dw["cond_proj_b"])
    dt_emb = timestep_embedding(dw["delta_time_mlp"], sinusoidal_pos_emb(dt, hidden, 1000.0))
    n = mu.shape[0]
    mu_tokens = mu.shape[1] // hidden
    return mu.reshape(n, mu_tokens, hidden).astype(F32), condp, dt_emb


def dit_forward_cached(dcfg, dw, x, t, cache, rope=None):
    """``VoxCpmLocDiTV2::forward_cached`` (``src/locdit/local_dit.rs:138-159``).

    Sequence order ``[mu tokens, t token, cond tokens, x tokens]``; the non-causal
    decoder output is narrowed at ``skip = prefix + mu_tokens + 1``.
    x ``[N, C, T]`` -> ``[N, C, T]``.
    """
    mu, condp, dt_emb = cache
    time_len = x.shape[2]
    xp = m4.linear(np.swapaxes(x, 1, 2), dw["in_proj_w"], dw["in_proj_b"])
    t_emb = timestep_embedding(dw["time_mlp"], sinusoidal_pos_emb(t, dcfg.hidden_size, 1000.0))
    t_tok = (t_emb + dt_emb)[:, None, :]
    seq = np.concatenate([mu, t_tok, condp, xp], axis=1).astype(F32)
    hid, _ = m4.model_forward(dcfg, dw["decoder"], seq, False, rope)
    skip = condp.shape[1] + mu.shape[1] + 1
    out = m4.linear(hid[:, skip:skip + time_len], dw["out_proj_w"], dw["out_proj_b"])
    return np.swapaxes(out, 1, 2).astype(F32)


def dit_forward(dcfg, dw, x, mu, t, cond, dt, rope=None):
    """``VoxCpmLocDiTV2::forward`` (``src/locdit/local_dit.rs:102-112``)."""
    return dit_forward_cached(dcfg, dw, x, t, dit_prepare(dcfg, dw, mu, cond, dt), rope)


def t_span(n_timesteps, sway_sampling_coef):
    """``UnifiedCfm::forward`` time grid (``src/locdit/unified_cfm.rs:59-67``):
    ``t_i = 1 - i/n`` in f64 rounded to f32, then the sway transform in f64."""
    n = n_timesteps + 1
    step = 1.0 / n_timesteps
    out = []
    for i in range(n):
        t = float(F32(1.0 - i * step))
        tr = t + sway_sampling_coef * (math.cos(math.pi / 2 * t) - 1.0 + t)
        out.append(F32(tr))
    return np.array(out, dtype=F32)


def zero_init_steps(n_span):
    """``unified_cfm.rs:85``: ``max(len * 0.04, 1) as usize``."""
    return int(max(n_span * 0.04, 1.0))


def cfg_combine(pos, neg, cfg_value, use_cfg_zero_star):
    """CFG / CFG-zero-star velocity (``src/locdit/unified_cfm.rs:132-152``).

    pos, neg ``[B, C, T]``.  Zero-star: ``st = <pos,neg> / (|neg|^2 + 1e-8)`` per batch,
    ``v = neg * (st * (1-cfg)) + pos * cfg``; plain CFG: ``v = neg + (pos-neg) * cfg``.
    """
    b = pos.shape[0]
    if use_cfg_zero_star:
        pf = pos.reshape(b, -1)
        nf = neg.reshape(b, -1)
        dot = np.sum(pf * nf, axis=1, keepdims=True, dtype=F32)
        sq = np.sum(nf * nf, axis=1, keepdims=True, dtype=F32) + F32(1e-8)
        st = (dot / sq)[:, :, None].astype(F32)
        return (neg * (st * F32(1.0 - cfg_value)) + pos * F32(cfg_value)).astype(F32)
    return (neg + (pos - neg) * F32(cfg_value)).astype(F32)


def euler_update(x, dphi, dt):
    """``x = x - dphi * dt`` with ``dt`` an f64 scalar applied as f32 (``unified_cfm.rs:155``)."""
    return (x - dphi * F32(dt)).astype(F32)


def solve_euler(dcfg, dw, x, tspan, mu, cond, cfg_value, use_cfg_zero_star, rope=None,
                trace=None):
    """``UnifiedCfm::solve_euler`` (``src/locdit/unified_cfm.rs:72-163``), non-mean mode.

    x ``[B, C, T]`` is the initial noise z; mu ``[B, C_mu]``; cond ``[B, C, T']``.
    The uncond branch zeroes mu only; cond is duplicated (``:96-98``); the DiT cache
    is prepared once with ``dt = 0`` (``:105-110``).
    """
    b = x.shape[0]
    t = float(tspan[0])
    dt = float(F32(tspan[0] - tspan[1]))
    zis = zero_init_steps(len(tspan))
    mu_in = np.concatenate([mu, np.zeros_like(mu)], axis=0).astype(F32)
    cond_in = np.concatenate([cond, cond], axis=0).astype(F32)
    cache = dit_prepare(dcfg, dw, mu_in, cond_in, np.zeros(2 * b, F32))
    for step in range(1, len(tspan)):
        if use_cfg_zero_star and step <= zis:
            dphi = np.zeros_like(x)
        else:
            x_in = np.concatenate([x, x], axis=0)
            out = dit_forward_cached(dcfg, dw, x_in, np.full(2 * b, F32(t), F32), cache, rope)
            dphi = cfg_combine(out[:b], out[b:], cfg_value, use_cfg_zero_star)
        if trace is not None:
            trace.append((t, dt, dphi.copy()))
        x = euler_update(x, dphi, dt)
        t -= dt
        if step < len(tspan) - 1:
            dt = t - float(tspan[step + 1])
    return x


def cfm_forward(dcfg, dw, mu, n_timesteps, cond, z, cfg_value, sway_sampling_coef,
                use_cfg_zero_star, rope=None):
    """``UnifiedCfm::forward`` (``src/locdit/unified_cfm.rs:34-70``) with the noise ``z``
    injected (``[B, C, patch]``, already multiplied by temperature) instead of drawn
    from the backend RNG."""
    ts = t_span(n_timesteps, sway_sampling_coef)
    return solve_euler(dcfg, dw, z.astype(F32), ts, mu, cond, cfg_value, use_cfg_zero_star, rope)
