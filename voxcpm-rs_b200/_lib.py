"""ctypes binding of ``libvoxcpm_b200.so`` (declarations in ``include/voxcpm_b200.h``).

The library is the product; this module only declares signatures and turns non-zero
status codes into ``VxError``.  There is no fallback: if the library is missing, or a
call needs a GPU and none is present, the call raises.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libvoxcpm_b200.so")

VX_OK, VX_ERR_SHAPE, VX_ERR_CONFIG, VX_ERR_CANCELLED, VX_ERR_KV_FULL = 0, 1, 2, 3, 4
VX_ERR_CUDA, VX_ERR_TIMEOUT, VX_ERR_ARG, VX_ERR_OOM, VX_ERR_NO_DEVICE = 5, 6, 7, 8, 9
STATUS_NAMES = {0: "OK", 1: "ShapeMismatch", 2: "InvalidConfig", 3: "Cancelled", 4: "KvCacheFull",
                5: "Cuda", 6: "Timeout", 7: "InvalidArgument", 8: "OutOfMemory", 9: "NoDevice"}


class VxError(RuntimeError):
    """A non-zero ``vx_status``; ``code`` mirrors the reference ``Error`` variant."""

    def __init__(self, code, msg):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class Cancelled(VxError):
    """``Error::Cancelled`` (reference ``src/error.rs:49-51``)."""


class MiniCpm4ConfigC(C.Structure):
    _fields_ = [("hidden_size", C.c_int), ("intermediate_size", C.c_int),
                ("num_attention_heads", C.c_int), ("num_key_value_heads", C.c_int),
                ("num_hidden_layers", C.c_int), ("vocab_size", C.c_int), ("kv_channels", C.c_int),
                ("max_position_embeddings", C.c_int), ("original_max_position_embeddings", C.c_int),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("use_mup", C.c_int),
                ("scale_emb", C.c_float), ("scale_depth", C.c_float), ("no_rope", C.c_int),
                ("rope_short_factor", C.POINTER(C.c_float)), ("rope_long_factor", C.POINTER(C.c_float)),
                ("rope_factor_len", C.c_int)]


P = C.c_void_p
I32 = C.c_int
F32 = C.c_float
F64 = C.c_double


class VaeConfigC(C.Structure):
    _fields_ = [("latent_dim", C.c_int), ("decoder_dim", C.c_int), ("rates", C.POINTER(C.c_int)),
                ("n_rates", C.c_int), ("depthwise", C.c_int), ("use_noise_block", C.c_int),
                ("out_sample_rate", C.c_int), ("sr_boundaries", C.POINTER(C.c_int)), ("n_sr_boundaries", C.c_int)]


class GenerateOptionsC(C.Structure):
    _fields_ = [("cfg_value", C.c_float), ("inference_timesteps", C.c_int), ("max_len", C.c_int),
                ("patch_size", C.c_int), ("sway_sampling_coef", C.c_float), ("use_cfg_zero_star", C.c_int)]


class VaeBlockWeightsC(C.Structure):
    _fields_ = [("alpha", P), ("up_w", P), ("up_b", P), ("res_alpha1", P * 3), ("res_w1", P * 3),
                ("res_b1", P * 3), ("res_alpha2", P * 3), ("res_w2", P * 3), ("res_b2", P * 3),
                ("sr_scale", P), ("sr_bias", P)]

class VoxCpm2WeightsC(C.Structure):
    _fields_ = [(n, P) for n in ("special_token", "enc_in_w", "enc_in_b", "enc_to_lm_w", "enc_to_lm_b",
                                 "lm_to_dit_w", "lm_to_dit_b", "res_to_dit_w", "res_to_dit_b", "fusion_w",
                                 "fusion_b", "stop_proj_w", "stop_proj_b", "stop_head_w", "fsq_in_w", "fsq_in_b",
                                 "fsq_out_w", "fsq_out_b")]


# name -> (restype, argtypes)
SIGNATURES = {
    "vx_version": (I32, []),
    "vx_launch_count": (C.c_ulonglong, []),
    "vx_lm_last_timing": (I32, [P, C.POINTER(F32), C.POINTER(F32)]),
    "vx_lm_profile_decode_step": (I32, [P, I32, P, I32]),
    "vx_lm_trace_decode_step": (I32, [P, I32, P, I32, P]),
    "vx_ctx_create": (I32, [I32, C.POINTER(P)]),
    "vx_ctx_destroy": (None, [P]),
    "vx_last_error": (C.c_char_p, [P]),
    "vx_ctx_stream": (P, [P]),
    "vx_ctx_synchronize": (I32, [P]),
    "vx_cancel": (None, [P]),
    "vx_cancel_reset": (None, [P]),
    "vx_memcpy": (I32, [P, P, P, C.c_size_t]),
    "vx_rmsnorm_residual": (I32, [P, P, P, P, F32, F32, I32, I32, P, P, P]),
    "vx_longrope_table": (I32, [C.POINTER(MiniCpm4ConfigC), I32, P, P]),
    "vx_rope_apply": (I32, [P, P, P, P, P, I32, I32, I32, I32, I32, P]),
    "vx_linear_bf16": (I32, [P, P, P, P, I32, I32, I32, P, P]),
    "vx_attention_decode": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I32, P, P]),
    "vx_attention_decode_static": (I32, [P, P, P, I32, I32, I32, I32, I32, I32, P, P]),
    "vx_mlp_swiglu": (I32, [P, P, P, P, I32, I32, I32, P, P]),
    "vx_cfg_euler": (I32, [P, P, P, I32, I32, I32, F32, F64, I32, P]),
    "vx_fsq": (I32, [P, P, P, P, P, I32, I32, I32, F32, P, I32, P, P]),
    "vx_lm_create": (I32, [P, C.POINTER(MiniCpm4ConfigC), I32, I32, C.POINTER(P)]),
    "vx_lm_destroy": (None, [P]),
    "vx_lm_load_layer": (I32, [P, I32, P, P, P, P, P, P, P, P, P]),
    "vx_lm_load_norm": (I32, [P, P]),
    "vx_lm_load_embed": (I32, [P, P]),
    "vx_lm_reset": (I32, [P]),
    "vx_lm_position": (I32, [P]),
    "vx_lm_set_position": (I32, [P, I32]),
    "vx_lm_kv_write": (I32, [P, I32, I32, P, P, I32]),
    "vx_lm_kv_read": (I32, [P, I32, I32, P, P, I32]),
    "vx_lm_embed": (I32, [P, P, I32, P]),
    "vx_lm_forward": (I32, [P, P, I32, I32, I32, I32, P]),
    "vx_lm_forward_step": (I32, [P, P, P]),
    "vx_lm_layer_forward_step": (I32, [P, I32, P, I32]),
    "vx_lm_greedy": (I32, [P, P, I32, I32, P]),
    "vx_dit_create": (I32, [P, C.POINTER(MiniCpm4ConfigC), I32, I32, C.POINTER(P)]),
    "vx_dit_destroy": (None, [P]),
    "vx_dit_load": (I32, [P] + [P] * 14),
    "vx_dit_load_layer": (I32, [P, I32, P, P, P, P, P, P, P, P, P]),
    "vx_dit_load_norm": (I32, [P, P]),
    "vx_dit_trace": (I32, [P, P, I32, C.POINTER(I32), C.POINTER(I32)]),
    "vx_lm_batch_trace": (I32, [P, P, I32, C.POINTER(I32), C.POINTER(I32)]),
    "vx_dit_forward": (I32, [P, P, P, P, P, P, I32, I32, I32, I32, P]),
    "vx_cfm_solve": (I32, [P, P, P, P, I32, I32, I32, I32, I32, F32, F32, I32, P]),
    "vx_vae_create": (I32, [P, C.POINTER(VaeConfigC), C.POINTER(P)]),
    "vx_vae_destroy": (None, [P]),
    "vx_vae_load_first": (I32, [P, P, P, P, P]),
    "vx_vae_load_block": (I32, [P, I32, C.POINTER(VaeBlockWeightsC)]),
    "vx_vae_load_out": (I32, [P, P, P, P]),
    "vx_vae_decode": (I32, [P, P, I32, I32, P]),
    "vx_generate": (I32, [P, P, P, P, I32, C.POINTER(GenerateOptionsC), P, P, P]),
    "vx_generate_batch": (I32, [P, P, P, P, I32, I32, C.POINTER(GenerateOptionsC), P, P, P]),
    "vx_lm_last_logits": (I32, [P, P]),
    "vx_voxcpm2_create": (I32, [P, P, P, P, I32, I32, I32, I32, I32, C.POINTER(P)]),
    "vx_voxcpm2_destroy": (None, [P]),
    "vx_voxcpm2_load": (I32, [P, C.POINTER(VoxCpm2WeightsC)]),
    "vx_locenc_forward": (I32, [P, P, I32, P]),
    "vx_voxcpm2_inference": (I32, [P, P, P, P, P, I32, I32, I32, I32, F32, P, P, C.POINTER(I32), P]),
    "vx_voxcpm2_generate": (I32, [P, P, P, P, P, P, I32, I32, I32, I32, F32, P, P, C.POINTER(I32)]),
    "vx_voxcpm2_begin": (I32, [P, P, P, P, P, I32, I32, I32, I32, F32, P]),
    "vx_voxcpm2_advance": (I32, [P, I32, P, C.POINTER(I32), C.POINTER(I32)]),
    "vx_vae_stream_create": (I32, [P, I32, C.POINTER(P)]),
    "vx_vae_stream_destroy": (None, [P]),
    "vx_vae_stream_reset": (I32, [P]),
    "vx_vae_stream_decode": (I32, [P, P, I32, P]),
    "vx_weights_open": (I32, [C.c_char_p, C.POINTER(P)]),
    "vx_weights_close": (None, [P]),
    "vx_weights_last_error": (C.c_char_p, []),
    "vx_weights_count": (I32, [P]),
    "vx_weights_name": (C.c_char_p, [P, I32]),
    "vx_weights_find": (I32, [P, C.c_char_p]),
    "vx_weights_info": (I32, [P, I32, C.POINTER(I32), P, I32]),
    "vx_weights_read": (I32, [P, C.c_char_p, I32, P, C.c_size_t]),
    "vx_lm_load_weights": (I32, [P, P, C.c_char_p]),
    "vx_dit_load_weights": (I32, [P, P, C.c_char_p]),
    "vx_vae_load_weights": (I32, [P, P, C.c_char_p]),
    "vx_voxcpm2_load_weights": (I32, [P, P]),
}

_lib = None


def lib():
    """Load the library once (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with voxcpm-rs_b200/build.py "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, ctx=None):
    if rc != VX_OK:
        msg = lib().vx_last_error(ctx).decode() if ctx else STATUS_NAMES.get(rc, str(rc))
        if rc == VX_ERR_CANCELLED:
            raise Cancelled(rc, msg)
        raise VxError(rc, msg)


def ptr(x):
    """Raw pointer of a torch tensor / numpy array / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(type(x))


def config_struct(cfg):
    """Build a ``vx_minicpm4_config`` from a ``MiniCpm4Config``; keeps the factor arrays
    alive on the returned struct."""
    import numpy as np
    d = cfg.head_dim()
    short = np.ascontiguousarray(cfg.rope_scaling.short_factor, dtype=np.float32)
    long_ = np.ascontiguousarray(cfg.rope_scaling.long_factor, dtype=np.float32)
    s = MiniCpm4ConfigC(
        cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.num_key_value_heads,
        cfg.num_hidden_layers, cfg.vocab_size, cfg.kv_channels or 0, cfg.max_position_embeddings,
        cfg.rope_scaling.original_max_position_embeddings, cfg.rms_norm_eps, cfg.rope_theta,
        int(cfg.use_mup), cfg.scale_emb, cfg.scale_depth, int(cfg.no_rope),
        short.ctypes.data_as(C.POINTER(C.c_float)), long_.ctypes.data_as(C.POINTER(C.c_float)),
        len(short) if len(short) == len(long_) else -1)
    s._keep = (short, long_)
    return s
