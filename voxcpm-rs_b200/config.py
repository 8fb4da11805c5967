"""Configuration structs mirroring the reference's serde configs (``src/config.rs``),
plus the named synthetic workloads this library is measured on.

Field names follow ``MiniCpm4Config`` (``src/config.rs:51-84``), ``RopeScalingConfig``
(``:42-49``), ``VoxCpmDitConfig`` (``:198-213``) and ``AudioVaeConfig`` (``:219-309``) so a
HuggingFace ``config.json`` maps field for field.
"""
from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class RopeScalingConfig:
    long_factor: List[float]
    short_factor: List[float]
    original_max_position_embeddings: int
    kind: str = "longrope"


@dataclass
class MiniCpm4Config:
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    num_hidden_layers: int
    vocab_size: int
    rope_scaling: RopeScalingConfig
    max_position_embeddings: int = 32768
    rms_norm_eps: float = 1e-6
    use_mup: bool = True
    scale_emb: float = 12.0
    dim_model_base: float = 256.0
    scale_depth: float = 1.4
    rope_theta: float = 10000.0
    kv_channels: Optional[int] = None
    no_rope: bool = False
    bos_token_id: int = 1
    eos_token_id: int = 2

    def head_dim(self) -> int:
        """``MiniCpm4Config::head_dim`` (``src/config.rs:78-83``)."""
        return self.kv_channels or self.hidden_size // self.num_attention_heads

    def derive(self, **kw) -> "MiniCpm4Config":
        c = copy.deepcopy(self)
        for k, v in kw.items():
            setattr(c, k, v)
        return c


@dataclass
class VoxCpmDitConfig:
    hidden_dim: int = 1024
    ffn_dim: int = 4096
    num_heads: int = 16
    num_layers: int = 4
    kv_channels: Optional[int] = None
    dit_mean_mode: bool = False


@dataclass
class VoxCpmEncoderConfig:
    """``VoxCpmEncoderConfig`` (``src/config.rs:158-184``)."""
    hidden_dim: int = 1024
    ffn_dim: int = 4096
    num_heads: int = 16
    num_layers: int = 4
    kv_channels: Optional[int] = None


@dataclass
class VoxCpm2Config:
    """``VoxCpm2Config`` (``src/config.rs:316-341``) fields the model uses, with the
    reference defaults, and its derivation helpers (``config.rs:421-453``).  ``dit_rope``
    / ``enc_rope`` override the inherited LongRoPE factors when a head_dim needs vectors of
    another length (``rope.rs:32``)."""
    lm_config: MiniCpm4Config
    encoder_config: VoxCpmEncoderConfig
    dit_config: VoxCpmDitConfig
    patch_size: int = 4
    feat_dim: int = 64
    residual_lm_num_layers: int = 8
    residual_lm_no_rope: bool = False
    scalar_quantization_latent_dim: int = 512
    scalar_quantization_scale: int = 9
    max_length: int = 8192
    enc_rope: Optional[RopeScalingConfig] = None
    dit_rope: Optional[RopeScalingConfig] = None

    def residual_lm_config(self) -> MiniCpm4Config:
        return self.lm_config.derive(num_hidden_layers=self.residual_lm_num_layers, vocab_size=0,
                                     no_rope=self.residual_lm_no_rope)

    def encoder_lm_config(self) -> MiniCpm4Config:
        e = self.encoder_config
        return self.lm_config.derive(hidden_size=e.hidden_dim, intermediate_size=e.ffn_dim,
                                     num_attention_heads=e.num_heads, num_hidden_layers=e.num_layers,
                                     kv_channels=e.kv_channels, vocab_size=0,
                                     rope_scaling=self.enc_rope or copy.deepcopy(self.lm_config.rope_scaling))

    def dit_lm_config(self) -> MiniCpm4Config:
        return dit_lm_config(self.lm_config, self.dit_config, self.dit_rope)


def dit_lm_config(lm: MiniCpm4Config, d: VoxCpmDitConfig,
                  rope_scaling: Optional[RopeScalingConfig] = None) -> MiniCpm4Config:
    """``VoxCpm2Config::dit_lm_config`` (``src/config.rs:443-453``): the LM config with the
    DiT's width/depth, ``vocab_size = 0`` and everything else (kv heads, rope, muP)
    inherited.  ``rope_scaling`` overrides the inherited factors when the DiT head_dim
    needs factor vectors of a different length (``rope.rs:32`` asserts ``len == d/2``)."""
    return lm.derive(hidden_size=d.hidden_dim, intermediate_size=d.ffn_dim,
                     num_attention_heads=d.num_heads, num_hidden_layers=d.num_layers,
                     kv_channels=d.kv_channels, vocab_size=0,
                     rope_scaling=rope_scaling or copy.deepcopy(lm.rope_scaling))


@dataclass
class AudioVaeConfig:
    latent_dim: int = 64
    decoder_dim: int = 2048
    decoder_rates: List[int] = field(default_factory=lambda: [8, 6, 5, 2, 2, 2])
    depthwise: bool = True
    sample_rate: int = 16000
    out_sample_rate: int = 48000
    use_noise_block: bool = False
    sr_bin_boundaries: Optional[List[int]] = field(default_factory=lambda: [20000, 30000, 40000])
    cond_type: str = "scale_bias"

    def decode_chunk_size(self) -> int:
        """``AudioVaeConfig::decode_chunk_size`` (``src/config.rs:286-288``)."""
        p = 1
        for r in self.decoder_rates:
            p *= r
        return p


def sr_bucket(sr: int, boundaries) -> int:
    """``sr_bucket`` (``src/audiovae/layers.rs:225-228``)."""
    for i, b in enumerate(boundaries):
        if sr < b:
            return i
    return len(boundaries)


# ------------------------------------------------------------------ workloads

def _factors(rng, n):
    return [float(v) for v in rng.uniform(1.0, 4.0, size=n).astype("float32")]


def lm_decode_config(layers=28, vocab=73448, seed=0, max_position_embeddings=32768):
    """MiniCPM4 decoder: hidden 2048, 16 q / 2 kv heads, head_dim 128, SwiGLU 6144,
    LongRoPE factors [64] ~U(1,4), original max position 32768, rope base 1e4.
    ``max_position_embeddings`` 32768 selects the short factors with scale 1.0;
    anything larger selects the long factors (``rope.rs:22-29``)."""
    import numpy as np
    rng = np.random.default_rng(seed + 1000)
    rs = RopeScalingConfig(long_factor=_factors(rng, 64), short_factor=_factors(rng, 64),
                           original_max_position_embeddings=32768)
    return MiniCpm4Config(hidden_size=2048, intermediate_size=6144, num_attention_heads=16,
                          num_key_value_heads=2, num_hidden_layers=layers, vocab_size=vocab,
                          rope_scaling=rs, max_position_embeddings=max_position_embeddings)


def locdit_config(lm: MiniCpm4Config, layers=8, seed=0):
    """LocDiT decoder: 8 layers, hidden 1024, 16 heads, MLP 4096, kv heads inherited (2),
    head_dim 64.  Its LongRoPE factor vectors are 32 long (head_dim/2) ~U(1,4)."""
    import numpy as np
    rng = np.random.default_rng(seed + 2000)
    rs = RopeScalingConfig(long_factor=_factors(rng, 32), short_factor=_factors(rng, 32),
                           original_max_position_embeddings=lm.rope_scaling.original_max_position_embeddings)
    return dit_lm_config(lm, VoxCpmDitConfig(hidden_dim=1024, ffn_dim=4096, num_heads=16,
                                             num_layers=layers), rs)


def vae_config(**kw) -> AudioVaeConfig:
    """AudioVAE decoder of the end-to-end workload: latent 64, decoder_dim 2048,
    rates [2,5,8,8] (channels 1024/512/256/128), depthwise, 16 kHz output (hop 640)."""
    base = dict(latent_dim=64, decoder_dim=2048, decoder_rates=[2, 5, 8, 8], depthwise=True,
                sample_rate=16000, out_sample_rate=16000)
    base.update(kw)
    return AudioVaeConfig(**base)


def voxcpm2_config(base: MiniCpm4Config, residual_layers=8, enc=None, dit=None, enc_rope=None, dit_rope=None,
                   latent=512, scale=9, feat_dim=64, patch_size=4) -> VoxCpm2Config:
    """A ``VoxCpm2Config`` over a base LM config (encoder / DiT default to the reference's
    1024-wide, 16-head stacks: 4 encoder layers, DiT layers as given)."""
    return VoxCpm2Config(lm_config=base, encoder_config=enc or VoxCpmEncoderConfig(),
                         dit_config=dit or VoxCpmDitConfig(), patch_size=patch_size, feat_dim=feat_dim,
                         residual_lm_num_layers=residual_layers, scalar_quantization_latent_dim=latent,
                         scalar_quantization_scale=scale, enc_rope=enc_rope, dit_rope=dit_rope)
