"""Checkpoint loading on the GPU: a VoxCPM2 model and an AudioVAE written in the upstream key
layout (safetensors and PyTorch zip, weight_norm pairs for the VAE convs, a fused qkv /
gate_up variant) and loaded through vx_voxcpm2_load_weights / vx_vae_load_weights give the
same outputs as the same weights uploaded from arrays."""
import numpy as np
import pytest
import torch

from tests.conftest import assert_close

pytestmark = pytest.mark.gpu


def _bf(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _f(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))


def lm_state(w, prefix, fused=False):
    sd = {}
    for i, l in enumerate(w["layers"]):
        p = f"{prefix}layers.{i}."
        if fused:
            sd[p + "self_attn.qkv_proj.weight"] = _bf(np.concatenate([l["q"], l["k"], l["v"]], 0))
            sd[p + "mlp.gate_up_proj.weight"] = _bf(np.concatenate([l["gate"], l["up"]], 0))
        else:
            for n in ("q", "k", "v"):
                sd[p + f"self_attn.{n}_proj.weight"] = _bf(l[n])
            sd[p + "mlp.gate_proj.weight"] = _bf(l["gate"])
            sd[p + "mlp.up_proj.weight"] = _bf(l["up"])
        sd[p + "self_attn.o_proj.weight"] = _bf(l["o"])
        sd[p + "mlp.down_proj.weight"] = _bf(l["down"])
        sd[p + "input_layernorm.weight"] = _f(l["ln_in"])
        sd[p + "post_attention_layernorm.weight"] = _f(l["ln_post"])
    sd[prefix + "norm.weight"] = _f(w["norm"])
    if w.get("embed") is not None:
        sd[prefix + "embed_tokens.weight"] = _bf(w["embed"])
    return sd


def voxcpm2_state(w, He):
    """The upstream model.safetensors layout of a VoxCpm2Model (module paths of
    src/voxcpm2/model.rs:22-37); the residual LM stores fused qkv / gate_up tensors."""
    sd = {}
    sd.update(lm_state(w["base"], "base_lm."))
    sd.update(lm_state(w["residual"], "residual_lm.", fused=True))
    sd.update(lm_state(w["encoder"], "feat_encoder.encoder."))
    d = w["dit"]
    P = "feat_decoder.estimator."
    sd.update(lm_state(d["decoder"], P + "decoder."))
    for n in ("in_proj", "cond_proj", "out_proj"):
        sd[P + n + ".weight"], sd[P + n + ".bias"] = _bf(d[n + "_w"]), _f(d[n + "_b"])
    for n in ("time_mlp", "delta_time_mlp"):
        t = d[n]
        sd[P + n + ".linear_1.weight"], sd[P + n + ".linear_1.bias"] = _bf(t["w1"]), _f(t["b1"])
        sd[P + n + ".linear_2.weight"], sd[P + n + ".linear_2.bias"] = _bf(t["w2"]), _f(t["b2"])
    sd["feat_encoder.special_token"] = _f(w["special"]).reshape(1, 1, 1, He)
    sd["feat_encoder.in_proj.weight"], sd["feat_encoder.in_proj.bias"] = _bf(w["enc_in_w"]), _f(w["enc_in_b"])
    for key, n in (("fsq_layer.in_proj", "fsq_in"), ("fsq_layer.out_proj", "fsq_out"), ("enc_to_lm_proj", "enc_to_lm"),
                   ("lm_to_dit_proj", "lm_to_dit"), ("res_to_dit_proj", "res_to_dit"),
                   ("fusion_concat_proj", "fusion"), ("stop_proj", "stop_proj")):
        sd[key + ".weight"], sd[key + ".bias"] = _bf(w[n + "_w"]), _f(w[n + "_b"])
    sd["stop_head.weight"] = _bf(w["stop_head_w"])
    return sd


def _wn(sd, key, bits):
    """Store a conv weight as a weight_norm pair (g = per-output-channel norm, v = w) in f32."""
    v = torch.from_numpy((np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32).copy())
    g = v.reshape(v.shape[0], -1).norm(dim=1).reshape([v.shape[0]] + [1] * (v.dim() - 1))
    sd[key + ".weight_g"], sd[key + ".weight_v"] = g.contiguous(), v.contiguous()


def vae_state(w):
    """The upstream audiovae checkpoint layout (nn.Sequential numbering, weight_norm convs)."""
    sd = {}
    P = "decoder."
    _wn(sd, P + "model.0", w["first_dw_w"])
    sd[P + "model.0.bias"] = _f(w["first_dw_b"])
    _wn(sd, P + "model.1", w["first_pw_w"])
    sd[P + "model.1.bias"] = _f(w["first_pw_b"])
    for i, blk in enumerate(w["blocks"]):
        b = f"{P}model.{2 + i}.block."
        sd[b + "0.alpha"] = _f(blk["alpha"]).reshape(1, -1, 1)
        _wn(sd, b + "1", blk["up_w"])
        sd[b + "1.bias"] = _f(blk["up_b"])
        for u, r in enumerate(blk["res"]):
            q = f"{b}{2 + u}.block."
            sd[q + "0.alpha"] = _f(r["alpha1"]).reshape(1, -1, 1)
            _wn(sd, q + "1", r["w1"])
            sd[q + "1.bias"] = _f(r["b1"])
            sd[q + "2.alpha"] = _f(r["alpha2"]).reshape(1, -1, 1)
            _wn(sd, q + "3", r["w2"])
            sd[q + "3.bias"] = _f(r["b2"])
        sd[f"{P}sr_cond_model.{2 + i}.scale_embed.weight"] = _f(w["sr_cond"][i]["scale"])
        sd[f"{P}sr_cond_model.{2 + i}.bias_embed.weight"] = _f(w["sr_cond"][i]["bias"])
    n = len(w["blocks"])
    sd[f"{P}model.{2 + n}.alpha"] = _f(w["alpha_out"]).reshape(1, -1, 1)
    _wn(sd, f"{P}model.{3 + n}", w["last_w"])
    sd[f"{P}model.{3 + n}.bias"] = _f(w["last_b"])
    sd[P + "sr_bin_boundaries"] = torch.tensor([20000, 30000, 40000], dtype=torch.int64)
    return sd


@pytest.mark.parametrize("fmt", ["safetensors", "pth"])
def test_voxcpm2_from_checkpoint(ctx, tmp_path, fmt):
    from tests.test_gpu_voxcpm2 import inputs, small_voxcpm2
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.voxcpm import VoxCpm2Model
    from voxcpm_rs_b200.weights import load_pretrained
    v = small_voxcpm2()
    w = synth.voxcpm2_weights(v, seed=2, std=0.05)
    sd = voxcpm2_state(w, v.encoder_lm_config().hidden_size)
    if fmt == "safetensors":
        from safetensors.torch import save_file
        save_file(sd, str(tmp_path / "model.safetensors"))
    else:
        torch.save({"state_dict": sd}, str(tmp_path / "model.pth"))
    ids, tm, feat, fm, noise = inputs(2)
    ref = VoxCpm2Model(ctx, v, w, max_len=12, max_length=64)
    want = ref.inference(ids, tm, feat, fm, 2, 12, 10, 2.0, noise)
    ref.close()
    m = VoxCpm2Model(ctx, v, None, max_len=12, max_length=64)
    load_pretrained(m, str(tmp_path))
    got = m.inference(ids, tm, feat, fm, 2, 12, 10, 2.0, noise)
    m.close()
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])


def test_vae_from_weight_norm_checkpoint(ctx, tmp_path):
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.weights import Checkpoint
    from voxcpm_rs_b200._lib import check, lib
    vcfg = config.vae_config(decoder_dim=256, decoder_rates=[2, 5])
    w = synth.vae_weights(vcfg, seed=4)
    p = str(tmp_path / "audiovae.pth")
    torch.save(vae_state(w), p)
    z = torch.from_numpy(np.random.default_rng(6).standard_normal((1, 64, 12), dtype=np.float32)).cuda()
    ref = AudioVae(ctx, vcfg, w)
    want = ref.decode(z).cpu().numpy()
    ref.close()
    vae = AudioVae(ctx, vcfg, None)
    with Checkpoint(p) as ck:
        check(lib().vx_vae_load_weights(vae.h, ck.h, None), ctx.h)
    got = vae.decode(z).cpu().numpy()
    vae.close()
    # g * v / ||v|| reproduces v up to f32 rounding, so the bf16 weights match except at rare
    # rounding ties
    assert_close(got, want, atol=2e-3, rtol=2e-3, what="VAE from weight_norm checkpoint")
