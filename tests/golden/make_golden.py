"""Generate the golden fixtures under tests/golden/ from the oracle.

The reference crate cannot run here (no Rust toolchain) and ships no golden vectors, so
these fixtures pin the oracle's own outputs on small seeded cases (regression anchors) and
give the GPU tests committed expected values.  Weights are not stored: they are
regenerated from their seeds by ``synth`` (PCG64 streams), only inputs' seeds and outputs
are.  Run: ``python tests/golden/make_golden.py``.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

load_package()
from voxcpm_rs_b200 import config, synth  # noqa: E402

from oracle import audiovae as oav  # noqa: E402
from oracle import locdit as old  # noqa: E402
from oracle import minicpm4 as om  # noqa: E402


def small_lm_config():
    """hidden 512, 8 q heads / 1 kv head (head_dim 64), SwiGLU 512, 2 layers, vocab 512."""
    rng = np.random.default_rng(77)
    rs = config.RopeScalingConfig(long_factor=[float(v) for v in rng.uniform(1, 4, 32).astype(np.float32)],
                                  short_factor=[float(v) for v in rng.uniform(1, 4, 32).astype(np.float32)],
                                  original_max_position_embeddings=32768)
    return config.MiniCpm4Config(hidden_size=512, intermediate_size=512, num_attention_heads=8,
                                 num_key_value_heads=1, num_hidden_layers=2, vocab_size=512, rope_scaling=rs)


def lm_case():
    cfg = small_lm_config()
    # std 0.2 (rather than the 0.02 of the full-size workloads) so that greedy decoding does
    # not lock onto one repeated id: the fixture then pins a varied id sequence.
    fw = synth.minicpm_f32_view(synth.minicpm_weights(cfg, seed=5, std=0.2))
    rng = np.random.default_rng(50)
    x = rng.standard_normal((1, 16, 512), dtype=np.float32)
    hid_causal, kvs = om.model_forward(cfg, fw, x, True)
    hid_full, _ = om.model_forward(cfg, fw, x, False)
    cache = om.StaticKvCache(2, 1, 64, 1, 64)
    cache.fill(kvs)
    e = rng.standard_normal((1, 512), dtype=np.float32)
    pos = cache.step()
    step = om.model_forward_step(cfg, fw, e, pos, cache)
    prompt = synth.prompt_ids(12, cfg.vocab_size, seed=3)
    toks, margins = om.greedy_generate(cfg, fw, prompt, 20, 64, return_margins=True)
    return {"prefill_causal": hid_causal, "forward_noncausal": hid_full, "k_layer1": kvs[1][0],
            "step_out": step, "greedy_ids": np.asarray(toks, np.int32),
            "greedy_margins": np.asarray(margins, np.float32), "prompt": prompt}


def small_dit_config():
    lm = small_lm_config()
    return config.dit_lm_config(lm, config.VoxCpmDitConfig(hidden_dim=512, ffn_dim=512, num_heads=8,
                                                            num_layers=2))


def cfm_case():
    dcfg = small_dit_config()
    dw = synth.locdit_f32_view(synth.locdit_weights(dcfg, in_channels=64, seed=6))
    rng = np.random.default_rng(60)
    mu = rng.standard_normal((1, 1024), dtype=np.float32)
    cond = rng.standard_normal((1, 64, 4), dtype=np.float32)
    z = rng.standard_normal((1, 64, 4), dtype=np.float32)
    out = {}
    out["x_uniform"] = old.cfm_forward(dcfg, dw, mu, 4, cond, z, 2.0, 0.0, False)
    out["x_sway_zero_star"] = old.cfm_forward(dcfg, dw, mu, 4, cond, z, 2.0, 1.0, True)
    x2 = rng.standard_normal((2, 64, 4), dtype=np.float32)
    mu2 = np.concatenate([mu, np.zeros_like(mu)])
    out["dit_forward"] = old.dit_forward(dcfg, dw, x2, mu2, np.array([0.7, 0.7], np.float32),
                                         np.concatenate([cond, cond]), np.zeros(2, np.float32))
    return out


def small_vae_config():
    """decoder_dim 512, rates [2, 5, 8]: channels 512 -> 256 -> 128 -> 64, hop 80."""
    return config.vae_config(decoder_dim=512, decoder_rates=[2, 5, 8])


def vae_case():
    vcfg = small_vae_config()
    vw = synth.vae_f32_view(synth.vae_weights(vcfg, seed=7))
    z = np.random.default_rng(70).standard_normal((1, 64, 8), dtype=np.float32)
    return {"wav": oav.decoder_forward(vcfg, vw, z)}


def main():
    np.savez_compressed(os.path.join(HERE, "lm_small.npz"), **lm_case())
    np.savez_compressed(os.path.join(HERE, "cfm_small.npz"), **cfm_case())
    np.savez_compressed(os.path.join(HERE, "vae_small.npz"), **vae_case())
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
