"""Host-side mirror of the reference's MiniCPM-4 operator surface (``src/minicpm4/``),
backed by ``libvoxcpm_b200.so``.

Device buffers are torch CUDA tensors (torch is used for device memory and streams only);
every computation is a call into the CUDA library.  Names follow the reference:
``MiniCpmRmsNorm.forward``, ``apply_rotary_pos_emb``, ``MiniCpmLongRope``, ``MiniCpmMlp``,
``MiniCpmAttention`` (decode sdpa), ``StaticKvCache`` and ``MiniCpmModel``.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _lib
from ._lib import check, lib, ptr


def _torch():
    import torch
    return torch


class Context:
    """A ``vx_ctx``: one CUDA device, its stream and scratch pool (one host thread)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        rc = lib().vx_ctx_create(device, C.byref(h))
        if rc != 0:
            raise _lib.VxError(rc, f"vx_ctx_create(device={device}) failed")
        self.h = h
        self.device = device
        self._owned = weakref.WeakSet()

    def _adopt(self, obj):
        """Register a library object created on this context: closing the context closes it
        first, so no native object outlives the context it points to."""
        self._owned.add(obj)

    @property
    def stream(self):
        return lib().vx_ctx_stream(self.h)

    def synchronize(self):
        check(lib().vx_ctx_synchronize(self.h), self.h)

    def cancel(self):
        """``CancelToken::cancel`` (``src/voxcpm2/wrapper.rs:57-59``); thread-safe."""
        lib().vx_cancel(self.h)

    def cancel_reset(self):
        lib().vx_cancel_reset(self.h)

    def memcpy(self, dst, src, nbytes):
        check(lib().vx_memcpy(self.h, ptr(dst), ptr(src), nbytes), self.h)

    def close(self):
        if getattr(self, "h", None):
            for obj in list(getattr(self, "_owned", ())):
                obj.close()
            lib().vx_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _stream_of(t):
    torch = _torch()
    return torch.cuda.current_stream(t.device).cuda_stream


# ---------------------------------------------------------------------------- ops

class MiniCpmRmsNorm:
    """``MiniCpmRmsNorm`` (``src/minicpm4/mod.rs:39-69``) with the residual add of
    ``MiniCpmDecoderLayer::add_residual`` (``layer.rs:33-38``) fused in."""

    def __init__(self, ctx: Context, weight, eps: float):
        self.ctx, self.weight, self.eps = ctx, weight, float(eps)

    def forward(self, x, residual=None, resid_scale: float = 1.0, return_residual=False):
        torch = _torch()
        hidden = x.shape[-1]
        rows = x.numel() // hidden
        y = torch.empty_like(x)
        h = torch.empty_like(x) if return_residual else None
        check(lib().vx_rmsnorm_residual(self.ctx.h, ptr(x), ptr(residual), ptr(self.weight),
                                        resid_scale, self.eps, rows, hidden, ptr(h), ptr(y),
                                        _stream_of(x)), self.ctx.h)
        return (h, y) if return_residual else y


def longrope_table(cfg, n_pos):
    """``MiniCpmLongRope::new`` cos/sin rows ``0..n_pos`` (``src/minicpm4/rope.rs:16-54``),
    computed on the host by the library in f64."""
    d = cfg.head_dim()
    cos = np.empty((n_pos, d), np.float32)
    sin = np.empty((n_pos, d), np.float32)
    s = _lib.config_struct(cfg)
    check(lib().vx_longrope_table(C.byref(s), n_pos, cos.ctypes.data, sin.ctypes.data))
    return cos, sin


class MiniCpmLongRope:
    """``MiniCpmLongRope`` (``src/minicpm4/rope.rs:9-63``): device cos/sin tables and
    ``gather`` of rows by position id."""

    def __init__(self, cfg, n_pos=None, device="cuda"):
        torch = _torch()
        n = cfg.max_position_embeddings if n_pos is None else n_pos
        cos, sin = longrope_table(cfg, n)
        self.cos = torch.from_numpy(cos).to(device)
        self.sin = torch.from_numpy(sin).to(device)
        self.head_dim = cfg.head_dim()

    def gather(self, position_ids):
        return self.cos[position_ids].contiguous(), self.sin[position_ids].contiguous()


def apply_rotary_pos_emb(ctx: Context, q, k, cos, sin):
    """``apply_rotary_pos_emb`` (``src/minicpm4/rope.rs:76-95``) on q ``[B,Hq,S,D]`` and
    k ``[B,Hk,S,D]`` with cos/sin ``[S,D]``; returns new tensors."""
    q, k = q.contiguous().clone(), k.contiguous().clone()
    b, hq, s, d = q.shape
    check(lib().vx_rope_apply(ctx.h, ptr(q), ptr(k), ptr(cos), ptr(sin), b, hq, k.shape[1], s, d,
                              _stream_of(q)), ctx.h)
    return q, k


def linear_bf16(ctx: Context, w_bits, x, bias=None):
    """``burn::nn::Linear::forward`` with bf16 weights ``[out, in]`` (int16/uint16 bits)."""
    torch = _torch()
    n, k = w_bits.shape
    m = x.numel() // k
    y = torch.empty(*x.shape[:-1], n, device=x.device, dtype=torch.float32)
    check(lib().vx_linear_bf16(ctx.h, ptr(w_bits), ptr(bias), ptr(x), m, n, k, ptr(y),
                               _stream_of(x)), ctx.h)
    return y


def attention_decode(ctx: Context, q, kcache, vcache, cur_len):
    """``MiniCpmAttention::sdpa`` + ``repeat_kv`` over a static cache for one query token
    (``src/minicpm4/attention.rs:129-204``): q ``[B, nh*d]``, caches ``[B, nkv, S_max, d]``."""
    torch = _torch()
    b, nkv, s_max, d = kcache.shape
    nh = q.shape[-1] // d
    out = torch.empty_like(q)
    check(lib().vx_attention_decode(ctx.h, ptr(q), ptr(kcache), ptr(vcache), b, nh, nkv, d, s_max,
                                    cur_len, ptr(out), _stream_of(q)), ctx.h)
    return out


class MiniCpmMlp:
    """``MiniCpmMlp`` (``src/minicpm4/mlp.rs:8-35``): fused gate|up and down, bf16 bits."""

    def __init__(self, ctx: Context, w_gate_up, w_down):
        self.ctx, self.w_gate_up, self.w_down = ctx, w_gate_up, w_down
        self.inter = w_down.shape[1]

    def forward(self, x):
        torch = _torch()
        hidden = x.shape[-1]
        rows = x.numel() // hidden
        out = torch.empty_like(x)
        check(lib().vx_mlp_swiglu(self.ctx.h, ptr(self.w_gate_up), ptr(self.w_down), ptr(x), rows,
                                  hidden, self.inter, ptr(out), _stream_of(x)), self.ctx.h)
        return out


# ---------------------------------------------------------------------------- model

class MiniCpmModel:
    """``MiniCpmModel`` + its ``StaticKvCache`` (``src/minicpm4/model.rs``, ``cache.rs``) as
    one library object.  Weights come from ``synth.minicpm_weights`` (checkpoint layout)."""

    def __init__(self, ctx: Context, cfg, weights=None, max_batch=1, max_length=4096):
        self.ctx, self.cfg = ctx, cfg
        self.max_length = max_length
        s = _lib.config_struct(cfg)
        h = C.c_void_p()
        check(lib().vx_lm_create(ctx.h, C.byref(s), max_batch, max_length, C.byref(h)), ctx.h)
        self.h = h
        ctx._adopt(self)
        if weights is not None:
            self.load(weights)

    def load(self, w):
        L = lib()
        for i, lw in enumerate(w["layers"]):
            arrs = [np.ascontiguousarray(lw[k]) for k in ("q", "k", "v", "o", "gate", "up", "down")]
            norms = [np.ascontiguousarray(lw[k], dtype=np.float32) for k in ("ln_in", "ln_post")]
            check(L.vx_lm_load_layer(self.h, i, *[ptr(a) for a in arrs], *[ptr(a) for a in norms]),
                  self.ctx.h)
        check(L.vx_lm_load_norm(self.h, ptr(np.ascontiguousarray(w["norm"], dtype=np.float32))),
              self.ctx.h)
        if w.get("embed") is not None:
            check(L.vx_lm_load_embed(self.h, ptr(np.ascontiguousarray(w["embed"]))), self.ctx.h)

    # StaticKvCache surface
    @property
    def current_length(self):
        return lib().vx_lm_position(self.h)

    def reset(self):
        check(lib().vx_lm_reset(self.h), self.ctx.h)

    def set_position(self, pos):
        check(lib().vx_lm_set_position(self.h, pos), self.ctx.h)

    def kv_write(self, layer, k, v, b=0):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        check(lib().vx_lm_kv_write(self.h, layer, b, ptr(k), ptr(v), k.shape[-2]), self.ctx.h)

    def kv_read(self, layer, n_pos, b=0):
        d, nkv = self.cfg.head_dim(), self.cfg.num_key_value_heads
        k = np.empty((nkv, n_pos, d), np.float32)
        v = np.empty((nkv, n_pos, d), np.float32)
        check(lib().vx_lm_kv_read(self.h, layer, b, ptr(k), ptr(v), n_pos), self.ctx.h)
        return k, v

    # MiniCpmModel surface
    def embed(self, ids):
        torch = _torch()
        ids = torch.as_tensor(ids, dtype=torch.int32, device=f"cuda:{self.ctx.device}").reshape(-1)
        out = torch.empty(ids.numel(), self.cfg.hidden_size, device=ids.device)
        torch.cuda.synchronize()
        check(lib().vx_lm_embed(self.h, ptr(ids), ids.numel(), ptr(out)), self.ctx.h)
        self.ctx.synchronize()
        return out

    def forward(self, inputs_embeds, is_causal, fill_cache=False):
        torch = _torch()
        b, s, hdim = inputs_embeds.shape
        x = inputs_embeds.contiguous()
        out = torch.empty_like(x)
        torch.cuda.synchronize()
        check(lib().vx_lm_forward(self.h, ptr(x), b, s, int(is_causal), int(fill_cache), ptr(out)),
              self.ctx.h)
        self.ctx.synchronize()
        return out

    def forward_step(self, inputs_embeds):
        torch = _torch()
        x = inputs_embeds.contiguous().reshape(-1)
        out = torch.empty_like(x)
        torch.cuda.synchronize()
        check(lib().vx_lm_forward_step(self.h, ptr(x), ptr(out)), self.ctx.h)
        self.ctx.synchronize()
        return out

    def layer_forward_step(self, layer, hidden, pos):
        torch = _torch()
        h = hidden.contiguous().reshape(-1).clone()
        torch.cuda.synchronize()
        check(lib().vx_lm_layer_forward_step(self.h, layer, ptr(h), pos), self.ctx.h)
        self.ctx.synchronize()
        return h

    def greedy(self, prompt_ids, n_steps):
        ids = np.ascontiguousarray(prompt_ids, dtype=np.int32)
        out = np.empty(n_steps + 1, np.int32)
        check(lib().vx_lm_greedy(self.h, ptr(ids), len(ids), n_steps, ptr(out)), self.ctx.h)
        return out

    def last_logits(self):
        out = np.empty(self.cfg.vocab_size, np.float32)
        check(lib().vx_lm_last_logits(self.h, ptr(out)), self.ctx.h)
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().vx_lm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
