"""numpy-f32 restatement of the MiniCPM-4 backbone (reference ``src/minicpm4/``).

Test infrastructure only (see ``oracle/__init__.py``); parity unpinned.

Weights use the model layout the reference holds after loading: linear weights are
``[out, in]`` (PyTorch order; ``src/weights.rs:637-772`` concatenates q|k|v and
gate|up along ``out``), so ``Linear`` is ``y = x @ W.T (+ b)``.

A model is a dict ``{"embed": [V,H] or None, "layers": [...], "norm": [H]}``; each
layer is ``{"wqkv", "wo", "wgu", "wd", "ln_in", "ln_post"}``.  A config is any object
with the attribute names of ``MiniCpm4Config`` (``src/config.rs:51-84``).
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def head_dim(cfg) -> int:
    """``MiniCpm4Config::head_dim`` (``src/config.rs:78-83``)."""
    return cfg.kv_channels if cfg.kv_channels else cfg.hidden_size // cfg.num_attention_heads


def residual_scale(cfg):
    """``MiniCpmDecoderLayer::new`` muP residual scale (``src/minicpm4/layer.rs:20-22``).

    ``scale_depth`` is an f32 config field widened to f64, divided by sqrt(L) in f64;
    ``mul_scalar`` then applies it as an f32 scalar.
    """
    if not cfg.use_mup:
        return None
    return F32(float(F32(cfg.scale_depth)) / math.sqrt(cfg.num_hidden_layers))


def scale_emb(cfg) -> np.float32:
    """``MiniCpmModel::scale_emb`` (``src/minicpm4/model.rs:94-100``)."""
    return F32(cfg.scale_emb) if cfg.use_mup else F32(1.0)


def linear(x, w, b=None):
    """``burn::nn::Linear::forward``: ``x @ W.T + b`` in f32 (``[out, in]`` weights)."""
    y = np.matmul(x.astype(F32, copy=False), w.T.astype(F32, copy=False))
    if b is not None:
        y = y + b.astype(F32, copy=False)
    return y.astype(F32, copy=False)


def silu_stable(x):
    """``silu_stable`` (``src/minicpm4/mod.rs:29-33``): ``x * sigmoid(x)`` in f32."""
    x = x.astype(F32, copy=False)
    with np.errstate(over="ignore"):
        sig = F32(1.0) / (F32(1.0) + np.exp(-x))
    return (x * sig).astype(F32, copy=False)


def rms_norm(x, w, eps):
    """``MiniCpmRmsNorm::forward`` (``src/minicpm4/mod.rs:54-68``).

    ``variance = mean(x*x)``; ``inv = sqrt(variance + eps)^-1``; ``x * inv * w``.
    ``eps`` is an f64 field applied through ``add_scalar`` as an f32 scalar.
    """
    x = x.astype(F32, copy=False)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    inv = F32(1.0) / np.sqrt(var + F32(eps))
    return ((x * inv) * w.astype(F32, copy=False)).astype(F32, copy=False)


def add_residual(residual, branch, scale):
    """``MiniCpmDecoderLayer::add_residual`` (``src/minicpm4/layer.rs:33-38``)."""
    if scale is None:
        return (residual + branch).astype(F32, copy=False)
    return (residual + branch * F32(scale)).astype(F32, copy=False)


def rmsnorm_residual(x, r, w, eps, scale=None):
    """The fused op measured by the RMSNorm microbenchmark workload:
    ``h = add_residual(r, x)`` then ``y = rms_norm(h)``.  ``r=None`` means no residual.
    Returns ``(h, y)``.  Follows ``layer.rs:33-38`` then ``mod.rs:54-68``.
    """
    h = x.astype(F32) if r is None else add_residual(r, x, scale)
    return h, rms_norm(h, w, eps)


# --------------------------------------------------------------------------- RoPE

def longrope_params(cfg):
    """The f64 quantities ``MiniCpmLongRope::new`` derives (``src/minicpm4/rope.rs:16-32``).

    Returns ``(inv_freq[half] f64, ext[half] f64, scaling_factor f64)``.
    """
    d = head_dim(cfg)
    half = d // 2
    base = float(F32(cfg.rope_theta))
    max_pos = cfg.max_position_embeddings
    orig = cfg.rope_scaling.original_max_position_embeddings
    scale = max_pos / orig
    v = 1.0 + math.log(scale) / math.log(orig)
    sf = math.sqrt(v) if v >= 0 else float("nan")
    # Rust f64::max ignores NaN: NaN.max(1.0) == 1.0
    sf = 1.0 if (sf != sf or sf < 1.0) else sf
    factors = cfg.rope_scaling.long_factor if max_pos > orig else cfg.rope_scaling.short_factor
    ext = np.asarray(factors, dtype=F32).astype(np.float64)
    if ext.shape[0] != half:
        raise ValueError("rope_scaling factor length must equal head_dim/2")
    i = np.arange(half, dtype=np.float64)
    inv_freq = 1.0 / np.power(base, 2.0 * i / d)
    return inv_freq, ext, sf


def longrope_table(cfg, n_pos=None):
    """``MiniCpmLongRope::new`` cos/sin tables (``src/minicpm4/rope.rs:34-48``).

    Computed in f64 and rounded to f32; rows ``0..n_pos`` (default: all
    ``max_position_embeddings`` rows).  Each row is ``[c_0..c_{h-1}, c_0..c_{h-1}]``.
    """
    inv_freq, ext, sf = longrope_params(cfg)
    n = cfg.max_position_embeddings if n_pos is None else n_pos
    t = np.arange(n, dtype=np.float64)[:, None]
    freq = t * inv_freq[None, :] / ext[None, :]
    c = (np.cos(freq) * sf).astype(F32)
    s = (np.sin(freq) * sf).astype(F32)
    return np.concatenate([c, c], axis=1), np.concatenate([s, s], axis=1)


def rotate_half(x):
    """``rotate_half`` (``src/minicpm4/rope.rs:66-73``): ``[-x2, x1]`` on the last dim."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_rotary_pos_emb(q, k, cos, sin):
    """``apply_rotary_pos_emb`` (``src/minicpm4/rope.rs:76-95``).

    q ``[B,Hq,S,D]``, k ``[B,Hk,S,D]``, cos/sin ``[S,D]``.
    """
    c = cos[None, None].astype(F32)
    s = sin[None, None].astype(F32)
    qe = q * c + rotate_half(q) * s
    ke = k * c + rotate_half(k) * s
    return qe.astype(F32), ke.astype(F32)


# ---------------------------------------------------------------------- attention

def repeat_kv(x, n_rep):
    """``repeat_kv`` (``src/minicpm4/attention.rs:196-204``): kv head g serves q heads
    ``g*n_rep .. g*n_rep+n_rep``."""
    if n_rep == 1:
        return x
    b, h, s, d = x.shape
    return np.broadcast_to(x[:, :, None], (b, h, n_rep, s, d)).reshape(b, h * n_rep, s, d)


def softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(x - m)
    return (e / np.sum(e, axis=axis, keepdims=True, dtype=F32)).astype(F32)


def sdpa(q, k, v, scale, is_causal):
    """``MiniCpmAttention::sdpa`` (``src/minicpm4/attention.rs:156-192``)."""
    scores = np.matmul(q, np.swapaxes(k, 2, 3)).astype(F32) * F32(scale)
    if is_causal:
        s_q, s_k = scores.shape[-2:]
        mask = np.arange(s_k)[None, :] > np.arange(s_q)[:, None]
        scores = np.where(mask[None, None], F32(-np.inf), scores)
    return np.matmul(softmax(scores, -1), v).astype(F32)


def attention_forward(cfg, lw, x, cos, sin, is_causal):
    """``MiniCpmAttention::forward`` (prefill / non-causal, ``attention.rs:55-88``).

    x ``[B,S,H]``; cos/sin ``[S,D]`` or None (no_rope).  Returns
    ``(out [B,S,H], (k, v))`` where k is post-RoPE ``[B,Hkv,S,D]``.
    """
    b, s, _ = x.shape
    nh, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, head_dim(cfg)
    qs, ks = nh * d, nkv * d
    qkv = linear(x, lw["wqkv"])
    q = qkv[..., :qs].reshape(b, s, nh, d).transpose(0, 2, 1, 3)
    k = qkv[..., qs:qs + ks].reshape(b, s, nkv, d).transpose(0, 2, 1, 3)
    v = qkv[..., qs + ks:qs + 2 * ks].reshape(b, s, nkv, d).transpose(0, 2, 1, 3)
    if cos is not None:
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
    n_rep = nh // nkv
    attn = sdpa(q, repeat_kv(k, n_rep), repeat_kv(v, n_rep), 1.0 / math.sqrt(d), is_causal)
    attn = attn.transpose(0, 2, 1, 3).reshape(b, s, nh * d)
    return linear(attn, lw["wo"]), (np.ascontiguousarray(k), np.ascontiguousarray(v))


def attention_forward_step(cfg, lw, x, cos_row, sin_row, pos, kcache, vcache):
    """``MiniCpmAttention::forward_step`` (``src/minicpm4/attention.rs:91-154``).

    x ``[B,H]`` (already normed); cos/sin rows ``[1,D]`` or None; kcache/vcache
    ``[B,Hkv,S_max,D]`` are updated in place at ``pos`` with post-RoPE k and v
    (``attention.rs:119-127``) and attention runs over ``0..pos+1`` (``:134-150``).
    """
    b = x.shape[0]
    nh, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, head_dim(cfg)
    qs, ks = nh * d, nkv * d
    qkv = linear(x, lw["wqkv"])
    q = qkv[:, :qs].reshape(b, 1, nh, d).transpose(0, 2, 1, 3)
    k = qkv[:, qs:qs + ks].reshape(b, 1, nkv, d).transpose(0, 2, 1, 3)
    v = qkv[:, qs + ks:qs + 2 * ks].reshape(b, 1, nkv, d).transpose(0, 2, 1, 3)
    if cos_row is not None:
        q, k = apply_rotary_pos_emb(q, k, cos_row, sin_row)
    kcache[:, :, pos] = k[:, :, 0]
    vcache[:, :, pos] = v[:, :, 0]
    n_rep = nh // nkv
    kv = repeat_kv(kcache[:, :, :pos + 1], n_rep)
    vv = repeat_kv(vcache[:, :, :pos + 1], n_rep)
    attn = sdpa(q, kv, vv, 1.0 / math.sqrt(d), False)
    attn = attn.transpose(0, 2, 1, 3).reshape(b, nh * d)
    return linear(attn, lw["wo"])


def mlp(cfg, lw, x):
    """``MiniCpmMlp::forward`` (``src/minicpm4/mlp.rs:28-34``): gate is the first
    ``intermediate_size`` outputs of the fused gate|up projection."""
    inter = cfg.intermediate_size
    gu = linear(x, lw["wgu"])
    gate, up = gu[..., :inter], gu[..., inter:]
    return linear(silu_stable(gate) * up, lw["wd"])


def layer_forward(cfg, lw, x, cos, sin, is_causal):
    """``MiniCpmDecoderLayer::forward`` (``src/minicpm4/layer.rs:40-55``)."""
    s = residual_scale(cfg)
    eps = cfg.rms_norm_eps
    h, kv = attention_forward(cfg, lw, rms_norm(x, lw["ln_in"], eps), cos, sin, is_causal)
    h = add_residual(x, h, s)
    out = add_residual(h, mlp(cfg, lw, rms_norm(h, lw["ln_post"], eps)), s)
    return out, kv


def layer_forward_step(cfg, lw, x, cos_row, sin_row, pos, kcache, vcache):
    """``MiniCpmDecoderLayer::forward_step`` (``src/minicpm4/layer.rs:57-73``)."""
    s = residual_scale(cfg)
    eps = cfg.rms_norm_eps
    h = attention_forward_step(cfg, lw, rms_norm(x, lw["ln_in"], eps), cos_row, sin_row,
                               pos, kcache, vcache)
    h = add_residual(x, h, s)
    return add_residual(h, mlp(cfg, lw, rms_norm(h, lw["ln_post"], eps)), s)


class StaticKvCache:
    """``StaticKvCache`` (``src/minicpm4/cache.rs:9-74``): zero-filled per-layer
    ``[B,Hkv,S_max,D]`` K and V, a fill from prefill, and a position counter."""

    def __init__(self, num_layers, nkv, d, batch, max_length):
        self.k = [np.zeros((batch, nkv, max_length, d), F32) for _ in range(num_layers)]
        self.v = [np.zeros((batch, nkv, max_length, d), F32) for _ in range(num_layers)]
        self.current_length = 0
        self.max_length = max_length

    def fill(self, kvs):
        s = kvs[0][0].shape[2]
        self.current_length = s
        for i, (k, v) in enumerate(kvs):
            self.k[i][:, :, :s] = k
            self.v[i][:, :, :s] = v

    def step(self):
        if not self.current_length < self.max_length:
            raise RuntimeError("KV cache is full")
        pos = self.current_length
        self.current_length += 1
        return pos


class RopeRows:
    """Caches ``longrope_table`` rows for one config (only the rows a run touches)."""

    def __init__(self, cfg, n_pos):
        self.cos, self.sin = longrope_table(cfg, n_pos)

    def rows(self, start, stop):
        return self.cos[start:stop], self.sin[start:stop]


def model_forward(cfg, mw, x, is_causal, rope=None):
    """``MiniCpmModel::forward`` (``src/minicpm4/model.rs:43-62``): rope rows
    ``0..S``; returns ``(norm(hidden) [B,S,H], [(k, v)] per layer)``."""
    s = x.shape[1]
    cos = sin = None
    if not cfg.no_rope:
        rope = rope or RopeRows(cfg, s)
        cos, sin = rope.rows(0, s)
    h = x.astype(F32)
    caches = []
    for lw in mw["layers"]:
        h, kv = layer_forward(cfg, lw, h, cos, sin, is_causal)
        caches.append(kv)
    return rms_norm(h, mw["norm"], cfg.rms_norm_eps), caches


def model_forward_step(cfg, mw, x, pos, cache: StaticKvCache, rope=None):
    """``MiniCpmModel::forward_step`` (``src/minicpm4/model.rs:64-84``)."""
    cos = sin = None
    if not cfg.no_rope:
        rope = rope or RopeRows(cfg, pos + 1)
        cos, sin = rope.rows(pos, pos + 1)
    h = x.astype(F32)
    for i, lw in enumerate(mw["layers"]):
        h = layer_forward_step(cfg, lw, h, cos, sin, pos, cache.k[i], cache.v[i])
    return rms_norm(h, mw["norm"], cfg.rms_norm_eps)


def embed(cfg, mw, ids):
    """``MiniCpmModel::embed`` then the caller's ``* scale_emb``
    (``src/minicpm4/model.rs:87-100``, ``src/voxcpm2/model.rs:144-145``)."""
    return (mw["embed"][np.asarray(ids)] * scale_emb(cfg)).astype(F32)


def argmax_first(x):
    """Greedy pick; ties go to the lowest index (assumed burn ``argmax`` semantics)."""
    return int(np.argmax(x))


def greedy_generate(cfg, mw, prompt_ids, n_steps, max_length, return_margins=False,
                    return_hidden=False):
    """Greedy LM decode harness over the tied embedding (the reference has no LM head;
    ``logits = y_final @ E.T``, next id = argmax, next input = ``E[id] * scale_emb``).

    Prefill runs ``model_forward(causal)`` and ``StaticKvCache::fill``
    (``src/voxcpm2/model.rs:157,173-191``); each decode step is ``cache.step()`` +
    ``model_forward_step``.  Returns ``n_steps + 1`` token ids (the first comes from the
    prefill's last row) and optionally the top-2 logit margins per pick and the last
    hidden row per pick.
    """
    d = head_dim(cfg)
    n_prompt = len(prompt_ids)
    rope = None if cfg.no_rope else RopeRows(cfg, n_prompt + n_steps + 1)
    cache = StaticKvCache(cfg.num_hidden_layers, cfg.num_key_value_heads, d, 1, max_length)
    x = embed(cfg, mw, np.asarray(prompt_ids)[None])
    y, kvs = model_forward(cfg, mw, x, True, rope)
    cache.fill(kvs)
    E = mw["embed"]
    toks, margins, hiddens = [], [], []
    last = y[:, -1]
    for step in range(n_steps + 1):
        logits = linear(last, E)[0]
        t = argmax_first(logits)
        toks.append(t)
        if return_margins:
            top2 = np.partition(logits, -2)[-2:]
            margins.append(float(top2[1] - top2[0]))
        if return_hidden:
            hiddens.append(last[0].copy())
        if step == n_steps:
            break
        pos = cache.step()
        last = model_forward_step(cfg, mw, embed(cfg, mw, [t]), pos, cache, rope)
    out = [toks]
    if return_margins:
        out.append(margins)
    if return_hidden:
        out.append(np.stack(hiddens))
    return out[0] if len(out) == 1 else tuple(out)
