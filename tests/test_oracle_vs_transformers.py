"""The oracle's MiniCPM-4 path against an independent implementation of the same architecture
family: transformers' Llama (RMSNorm, grouped-query attention with half-split rotary
embeddings and LongRoPE scaling, SwiGLU MLP), run on the CPU in f32 on small random-init
models.

The reference crate itself cannot run here, so these tests cross-check the oracle's
restatement of ``src/minicpm4/`` against a third-party implementation rather than against
the reference.  MiniCPM-4's muP terms map onto Llama weights exactly: the residual scale
``scale_depth / sqrt(L)`` (``layer.rs:20-22,33-38``) multiplies o_proj and down_proj, and
``scale_emb`` (``model.rs:94-100``) multiplies the input embedding table while the greedy head
reads the unscaled tied table.  The reference selects the LongRoPE factor vector once, from
``max_position_embeddings > original_max_position_embeddings`` (``rope.rs:24-32``), where
transformers switches per sequence length; the Llama config is therefore given the
reference's chosen vector as both its short and its long factors.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import minicpm4 as om
from tests.golden.make_golden import small_lm_config

transformers = pytest.importorskip("transformers")


def _weights(cfg, seed, std):
    from voxcpm_rs_b200 import synth
    return synth.minicpm_f32_view(synth.minicpm_weights(cfg, seed=seed, std=std))


def _llama(cfg, fw):
    """A LlamaForCausalLM holding the oracle model ``fw`` (f32, eager attention)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    d = om.head_dim(cfg)
    _, ext, _ = om.longrope_params(cfg)
    factors = [float(v) for v in ext]
    hc = LlamaConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                     intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                     num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                     head_dim=d, hidden_act="silu", max_position_embeddings=cfg.max_position_embeddings,
                     rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=False, attention_bias=False,
                     mlp_bias=False, pad_token_id=0, bos_token_id=None, eos_token_id=None,
                     rope_parameters={"rope_type": "longrope", "rope_theta": float(cfg.rope_theta),
                                      "short_factor": factors, "long_factor": factors,
                                      "original_max_position_embeddings":
                                          cfg.rope_scaling.original_max_position_embeddings})
    hc._attn_implementation = "eager"
    m = LlamaForCausalLM(hc).float().eval()
    rs = om.residual_scale(cfg)
    s = np.float32(1.0) if rs is None else rs
    qs, ks = cfg.num_attention_heads * d, cfg.num_key_value_heads * d
    I = cfg.intermediate_size
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))  # noqa: E731
    with torch.no_grad():
        m.model.embed_tokens.weight.copy_(t(fw["embed"] * om.scale_emb(cfg)))
        m.lm_head.weight.copy_(t(fw["embed"]))
        m.model.norm.weight.copy_(t(fw["norm"]))
        for layer, lw in zip(m.model.layers, fw["layers"]):
            wqkv = lw["wqkv"]
            layer.self_attn.q_proj.weight.copy_(t(wqkv[:qs]))
            layer.self_attn.k_proj.weight.copy_(t(wqkv[qs:qs + ks]))
            layer.self_attn.v_proj.weight.copy_(t(wqkv[qs + ks:]))
            layer.self_attn.o_proj.weight.copy_(t(lw["wo"] * s))
            layer.mlp.gate_proj.weight.copy_(t(lw["wgu"][:I]))
            layer.mlp.up_proj.weight.copy_(t(lw["wgu"][I:]))
            layer.mlp.down_proj.weight.copy_(t(lw["wd"] * s))
            layer.input_layernorm.weight.copy_(t(lw["ln_in"]))
            layer.post_attention_layernorm.weight.copy_(t(lw["ln_post"]))
    return m


def _configs():
    base = small_lm_config()
    # max_position_embeddings above the original: the long factors and the LongRoPE attention
    # factor sqrt(1 + ln 2 / ln 32768) (rope.rs:24-32)
    return {"short": base, "long": base.derive(max_position_embeddings=65536)}


@pytest.mark.parametrize("which", ["short", "long"])
def test_longrope_tables_vs_transformers(which):
    """cos / sin rows of ``MiniCpmLongRope::new`` (rope.rs:16-54) against transformers'
    longrope rotary embedding (f32 angles there, f64 in the reference: positions < 256)."""
    cfg = _configs()[which]
    cos, sin = om.longrope_table(cfg, 256)
    m = _llama(cfg, _weights(cfg, 5, 0.2))
    pos = torch.arange(256)[None]
    x = torch.zeros(1, 256, cfg.hidden_size)
    with torch.no_grad():
        hc, hs = m.model.rotary_emb(x, pos)
    np.testing.assert_allclose(hc[0].numpy(), cos, rtol=0, atol=2e-5)
    np.testing.assert_allclose(hs[0].numpy(), sin, rtol=0, atol=2e-5)


@pytest.mark.parametrize("which", ["short", "long"])
def test_prefill_forward_vs_transformers(which):
    """``MiniCpmModel::forward`` (model.rs:64-84; causal, final norm) on 16 embedded rows
    against LlamaModel's last hidden state."""
    cfg = _configs()[which]
    fw = _weights(cfg, 5, 0.2)
    ids = np.random.default_rng(11).integers(0, cfg.vocab_size, 16)
    x = om.embed(cfg, fw, ids[None])
    want, _ = om.model_forward(cfg, fw, x, True, om.RopeRows(cfg, 16))
    m = _llama(cfg, fw)
    with torch.no_grad():
        got = m.model(input_ids=torch.from_numpy(ids)[None]).last_hidden_state[0].numpy()
    assert np.abs(got - want[0]).max() < 2e-4 * max(1.0, float(np.abs(want).max()))


@pytest.mark.parametrize("which", ["short", "long"])
def test_greedy_ids_vs_transformers(which):
    """The oracle's greedy decode over the static KV cache (prefill, then forward_step per
    token; model.rs:64-84, attention.rs:156-204, cache.rs) against transformers' greedy
    generate with its dynamic cache: the same 21 ids."""
    cfg = _configs()[which]
    fw = _weights(cfg, 5, 0.2)
    from voxcpm_rs_b200 import synth
    prompt = synth.prompt_ids(12, cfg.vocab_size, seed=3)
    want, margins = om.greedy_generate(cfg, fw, prompt, 20, 64, return_margins=True)
    m = _llama(cfg, fw)
    with torch.no_grad():
        out = m.generate(torch.from_numpy(np.asarray(prompt, dtype=np.int64))[None], do_sample=False,
                         max_new_tokens=21, min_new_tokens=21, num_beams=1)
    got = out[0, len(prompt):].tolist()
    print(f"{which}: ids {want}, top-2 margin min {min(margins):.4f} max {max(margins):.4f}")
    assert got == list(want)


def test_noncausal_forward_vs_transformers():
    """The non-causal ``MiniCpmModel::forward`` that LocDiT and LocEnc run (model.rs:64-84
    with ``is_causal`` false) against LlamaModel given an all-zero additive attention mask
    (every row attends to every position)."""
    cfg = _configs()["short"]
    fw = _weights(cfg, 5, 0.2)
    ids = np.random.default_rng(11).integers(0, cfg.vocab_size, 16)
    x = om.embed(cfg, fw, ids[None])
    want, _ = om.model_forward(cfg, fw, x, False, om.RopeRows(cfg, 16))
    causal, _ = om.model_forward(cfg, fw, x, True, om.RopeRows(cfg, 16))
    m = _llama(cfg, fw)
    with torch.no_grad():
        got = m.model(input_ids=torch.from_numpy(ids)[None],
                      attention_mask=torch.zeros(1, 1, 16, 16)).last_hidden_state[0].numpy()
    assert np.abs(got - want[0]).max() < 2e-4 * max(1.0, float(np.abs(want).max()))
    assert np.abs(got - causal[0]).max() > 0.1  # the mask really lifted causality
