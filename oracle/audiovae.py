"""numpy-f32 restatement of the AudioVAE v2 causal decoder
(reference ``src/audiovae/layers.rs``, ``decoder.rs``, ``vae.rs``).

Test infrastructure only (see ``oracle/__init__.py``); parity unpinned.

Tensors are ``[B, C, T]``.  Conv weights use the PyTorch/Burn layouts:
``Conv1d`` ``[C_out, C_in/groups, K]``, ``ConvTranspose1d`` ``[C_in, C_out/groups, K]``.
A decoder is a dict (see ``voxcpm-rs_b200``'s ``synth.vae_weights`` for the keys).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def snake(x, alpha):
    """``Snake1d::forward`` (``src/audiovae/layers.rs:118-123``):
    ``x + (alpha + 1e-9)^-1 * sin(alpha * x)^2``; alpha ``[C]``."""
    a = alpha.astype(F32)[None, :, None]
    denom = F32(1.0) / (a + F32(1e-9))
    s = np.sin(a * x)
    return (x + denom * (s * s)).astype(F32)


def conv1d(x, w, b, dilation=1, groups=1):
    """Valid ``Conv1d`` (stride 1) in f32.  x ``[B,Cin,T]``, w ``[Cout,Cin/g,K]``."""
    bsz, cin, t = x.shape
    cout, cpg, k = w.shape
    t_out = t - dilation * (k - 1)
    if groups == cin and cpg == 1 and cout == cin:
        out = np.zeros((bsz, cout, t_out), F32)
        for j in range(k):
            out += w[None, :, 0, j, None] * x[:, :, j * dilation:j * dilation + t_out]
    elif groups == 1:
        if k == 1:
            out = np.einsum("oc,bct->bot", w[:, :, 0], x, optimize=True).astype(F32)
        else:
            cols = np.stack([x[:, :, j * dilation:j * dilation + t_out] for j in range(k)], axis=2)
            out = np.einsum("ock,bckt->bot", w, cols, optimize=True).astype(F32)
    else:
        raise NotImplementedError("grouped conv other than depthwise")
    if b is not None:
        out = out + b.astype(F32)[None, :, None]
    return out.astype(F32)


def causal_conv1d(x, w, b, dilation, groups, padding, output_padding):
    """``CausalConv1d`` (``src/audiovae/layers.rs:13-53``): left-pad by
    ``2*padding - output_padding`` zeros, then a valid conv."""
    left = padding * 2 - output_padding
    if left > 0:
        x = np.pad(x, ((0, 0), (0, 0), (left, 0)))
    return conv1d(x, w, b, dilation, groups)


def conv_transpose1d(x, w, b, stride):
    """``ConvTranspose1d`` with padding 0, groups 1 (scatter form):
    ``out[co, t*stride + k] += x[ci, t] * w[ci, co, k]``."""
    bsz, cin, t = x.shape
    _, cout, k = w.shape
    t_full = (t - 1) * stride + k
    out = np.zeros((bsz, cout, t_full), F32)
    for j in range(k):
        y = np.einsum("ic,bit->bct", w[:, :, j], x, optimize=True).astype(F32)
        out[:, :, j:j + stride * (t - 1) + 1:stride] += y
    if b is not None:
        out = out + b.astype(F32)[None, :, None]
    return out.astype(F32)


def causal_transpose_conv1d(x, w, b, stride):
    """``CausalTransposeConv1d`` as a decoder block builds it
    (``src/audiovae/layers.rs:60-100``, ``decoder.rs:31-36``): kernel ``2*stride``,
    then trim ``2*ceil(stride/2) - stride%2`` samples on the right."""
    pad = -(-stride // 2)
    trim = 2 * pad - stride % 2
    out = conv_transpose1d(x, w, b, stride)
    return out[:, :, :out.shape[2] - trim] if trim > 0 else out


def residual_unit(ru, x, dilation, groups):
    """``CausalResidualUnit::forward`` (``src/audiovae/layers.rs:139-156``):
    ``x + conv1x1(snake(dwconv7_dil(snake(x))))``."""
    pad = (6 * dilation) // 2
    y = snake(x, ru["alpha1"])
    y = causal_conv1d(y, ru["w1"], ru["b1"], dilation, groups, pad, 0)
    y = snake(y, ru["alpha2"])
    y = causal_conv1d(y, ru["w2"], ru["b2"], 1, 1, 0, 0)
    return (x + y).astype(F32)


def decoder_block(blk, x, stride, groups):
    """``CausalDecoderBlock::forward`` (``src/audiovae/decoder.rs:45-55``), noise block off."""
    x = snake(x, blk["alpha"])
    x = causal_transpose_conv1d(x, blk["up_w"], blk["up_b"], stride)
    for ru, dil in zip(blk["res"], (1, 3, 9)):
        x = residual_unit(ru, x, dil, groups)
    return x


def sr_bucket(sr, boundaries):
    """``sr_bucket`` (``src/audiovae/layers.rs:225-228``)."""
    for i, bnd in enumerate(boundaries):
        if sr < bnd:
            return i
    return len(boundaries)


def sr_cond(layer, x, idx):
    """``SampleRateConditionLayer::forward`` (``src/audiovae/layers.rs:213-220``)."""
    return (x * layer["scale"][idx][None, :, None] + layer["bias"][idx][None, :, None]).astype(F32)


def decoder_forward(vcfg, vw, z, target_sr=None):
    """``CausalDecoder::forward`` (``src/audiovae/decoder.rs:149-167``) via
    ``AudioVae::decode`` (``vae.rs:56-59``).  z ``[B, latent, T]`` -> ``[B, 1, T*prod(rates)]``."""
    sr = vcfg.out_sample_rate if target_sr is None else target_sr
    idx = None if vcfg.sr_bin_boundaries is None else sr_bucket(sr, vcfg.sr_bin_boundaries)
    if vcfg.depthwise:
        h = causal_conv1d(z, vw["first_dw_w"], vw["first_dw_b"], 1, z.shape[1], 3, 0)
        h = causal_conv1d(h, vw["first_pw_w"], vw["first_pw_b"], 1, 1, 0, 0)
    else:
        h = causal_conv1d(z, vw["first_pw_w"], vw["first_pw_b"], 1, 1, 3, 0)
    ch = vcfg.decoder_dim
    for i, stride in enumerate(vcfg.decoder_rates):
        out_dim = ch // 2 ** (i + 1)
        if idx is not None:
            h = sr_cond(vw["sr_cond"][i], h, idx)
        h = decoder_block(vw["blocks"][i], h, stride, out_dim if vcfg.depthwise else 1)
    h = snake(h, vw["alpha_out"])
    h = causal_conv1d(h, vw["last_w"], vw["last_b"], 1, 1, 3, 0)
    return np.tanh(h).astype(F32)
