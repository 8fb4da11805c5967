"""End-to-end synthesis on the GPU (vx_generate) against the oracle's loop: greedy LM decode,
a CFM solve per step on the step's final-norm hidden, stacked latent, AudioVAE decode.
Small models (2-layer LM at full width with vocab 4096, 2-layer DiT of hidden 512, a
512-wide 3-block VAE) and 6 patches.  Tolerance 2e-2 max-abs/rel."""
import numpy as np
import pytest

from oracle import voxcpm as ovx
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-2, rtol=2e-2)


def test_generate_small(ctx):
    from tests.golden.make_golden import small_dit_config, small_vae_config
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    from voxcpm_rs_b200.voxcpm import GenerateOptions, VoxCPM
    lm_cfg = config.lm_decode_config(layers=2, vocab=4096)
    lm_w = synth.minicpm_weights(lm_cfg, seed=3)
    dcfg, vcfg = small_dit_config(), small_vae_config()
    dit_w = synth.locdit_weights(dcfg, in_channels=64, seed=4)
    vae_w = synth.vae_weights(vcfg, seed=5)
    prompt = synth.prompt_ids(16, lm_cfg.vocab_size, seed=1)
    opts = GenerateOptions(max_len=6, inference_timesteps=4)
    noise = np.random.default_rng(8).standard_normal((6, 64, 4), dtype=np.float32)
    want_wav, want_lat, _ = ovx.generate(lm_cfg, synth.minicpm_f32_view(lm_w), dcfg, synth.locdit_f32_view(dit_w),
                                         vcfg, synth.vae_f32_view(vae_w), prompt, 6, noise, inference_timesteps=4)
    vox = VoxCPM(ctx, MiniCpmModel(ctx, lm_cfg, lm_w, max_length=64), VoxCpmLocDiTV2(ctx, dcfg, dit_w),
                 AudioVae(ctx, vcfg, vae_w))
    wav, lat = vox.generate(prompt, opts, noise, return_latent=True)
    assert wav.shape == (6 * 4 * 80,)
    assert_close(lat, want_lat, **TOL, what="latent")
    assert_close(wav, want_wav, **TOL, what="wav")
    # cancellation between steps surfaces as Error::Cancelled
    from voxcpm_rs_b200._lib import Cancelled
    ctx.cancel()
    try:
        with pytest.raises(Cancelled):
            vox.generate(prompt, opts, noise)
    finally:
        ctx.cancel_reset()


def test_generate_batch_small(ctx):
    """vx_generate_batch: 3 utterances (different prompts of one length, different noise) in
    one batched run, each against the oracle's single-utterance loop; also the batched LM
    decode's ids against the oracle's greedy ids."""
    from tests.golden.make_golden import small_dit_config, small_vae_config
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    from voxcpm_rs_b200.voxcpm import GenerateOptions, VoxCPM
    B, n, steps = 3, 16, 5
    lm_cfg = config.lm_decode_config(layers=2, vocab=4096)
    lm_w = synth.minicpm_weights(lm_cfg, seed=3)
    dcfg, vcfg = small_dit_config(), small_vae_config()
    dit_w = synth.locdit_weights(dcfg, in_channels=64, seed=4)
    vae_w = synth.vae_weights(vcfg, seed=5)
    prompts = np.stack([synth.prompt_ids(n, lm_cfg.vocab_size, seed=10 + b) for b in range(B)])
    noise = np.random.default_rng(9).standard_normal((B, steps, 64, 4), dtype=np.float32)
    opts = GenerateOptions(max_len=steps, inference_timesteps=4)
    vox = VoxCPM(ctx, MiniCpmModel(ctx, lm_cfg, lm_w, max_batch=B, max_length=64),
                 VoxCpmLocDiTV2(ctx, dcfg, dit_w, max_rows=2 * B), AudioVae(ctx, vcfg, vae_w))
    wav, lat = vox.generate_batch(prompts, opts, noise, return_latent=True)
    assert wav.shape == (B, steps * 4 * 80) and lat.shape == (B, 64, steps * 4)
    fl, fd, fv = synth.minicpm_f32_view(lm_w), synth.locdit_f32_view(dit_w), synth.vae_f32_view(vae_w)
    for b in range(B):
        want_wav, want_lat, _ = ovx.generate(lm_cfg, fl, dcfg, fd, vcfg, fv, prompts[b], steps, noise[b],
                                             inference_timesteps=4)
        assert_close(lat[b], want_lat, **TOL, what=f"latent[{b}]")
        assert_close(wav[b], want_wav, **TOL, what=f"wav[{b}]")


@pytest.mark.slow
def test_generate_full_width(ctx):
    """vx_generate at the end-to-end workload's widths: a 4-layer LM of the decode workload
    (hidden 2048, 16/2 heads, SwiGLU 6144, vocab 73448), the 8-layer hidden-1024 LocDiT, the
    2048-wide AudioVAE with rates [2,5,8,8]; 64-id prompt, 8 patches, 10 Euler steps with
    the reference-default sampler (sway 1, CFG-zero-star, CFG 2)."""
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    from voxcpm_rs_b200.voxcpm import GenerateOptions, VoxCPM
    lm_cfg = config.lm_decode_config(layers=4)
    lm_w = synth.minicpm_weights(lm_cfg, seed=11)
    dcfg, vcfg = config.locdit_config(lm_cfg), config.vae_config()
    dit_w = synth.locdit_weights(dcfg, in_channels=64, seed=12)
    vae_w = synth.vae_weights(vcfg, seed=13)
    prompt = synth.prompt_ids(64, lm_cfg.vocab_size, seed=14)
    steps = 8
    noise = np.random.default_rng(15).standard_normal((steps, 64, 4), dtype=np.float32)
    opts = GenerateOptions(max_len=steps, inference_timesteps=10)
    vox = VoxCPM(ctx, MiniCpmModel(ctx, lm_cfg, lm_w, max_length=128), VoxCpmLocDiTV2(ctx, dcfg, dit_w),
                 AudioVae(ctx, vcfg, vae_w))
    wav, lat = vox.generate(prompt, opts, noise, return_latent=True)
    vox.dit.close()
    vox.vae.close()
    vox.lm.close()
    want_wav, want_lat, _ = ovx.generate(lm_cfg, synth.minicpm_f32_view(lm_w), dcfg, synth.locdit_f32_view(dit_w),
                                         vcfg, synth.vae_f32_view(vae_w), prompt, steps, noise,
                                         inference_timesteps=10)
    assert wav.shape == (steps * 4 * 640,)
    assert_close(lat, want_lat, **TOL, what="latent")
    assert_close(wav, want_wav, **TOL, what="wav")


@pytest.mark.slow
def test_generate_batch_full_width(ctx):
    """vx_generate_batch at the end-to-end workload's widths (a 4-layer LM of the decode
    workload, the 8-layer LocDiT, the 2048-wide AudioVAE): 4 utterances, 3 patches.  The
    batched LM step runs as one persistent launch (decode attention over the static cache);
    two utterances are checked against the oracle's single-utterance loop, and the whole run
    against the per-kernel LM step (VX_LM_BATCH_PERSIST=0)."""
    import os
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    from voxcpm_rs_b200.voxcpm import GenerateOptions, VoxCPM
    B, n, steps = 4, 64, 3
    lm_cfg = config.lm_decode_config(layers=4)
    lm_w = synth.minicpm_weights(lm_cfg, seed=21)
    dcfg, vcfg = config.locdit_config(lm_cfg), config.vae_config()
    dit_w = synth.locdit_weights(dcfg, in_channels=64, seed=22)
    vae_w = synth.vae_weights(vcfg, seed=23)
    prompts = np.stack([synth.prompt_ids(n, lm_cfg.vocab_size, seed=30 + b) for b in range(B)])
    noise = np.random.default_rng(24).standard_normal((B, steps, 64, 4), dtype=np.float32)
    opts = GenerateOptions(max_len=steps, inference_timesteps=10)
    outs = []
    for flag in (None, "0"):
        old_env = os.environ.get("VX_LM_BATCH_PERSIST")
        if flag is not None:
            os.environ["VX_LM_BATCH_PERSIST"] = flag
        try:
            lm = MiniCpmModel(ctx, lm_cfg, lm_w, max_batch=B, max_length=128)
        finally:
            if old_env is None:
                os.environ.pop("VX_LM_BATCH_PERSIST", None)
            else:
                os.environ["VX_LM_BATCH_PERSIST"] = old_env
        vox = VoxCPM(ctx, lm, VoxCpmLocDiTV2(ctx, dcfg, dit_w, max_rows=2 * B), AudioVae(ctx, vcfg, vae_w))
        outs.append(vox.generate_batch(prompts, opts, noise, return_latent=True))
        vox.dit.close()
        vox.vae.close()
        vox.lm.close()
    (wav, lat), (wav0, lat0) = outs
    assert_close(lat, lat0, atol=2e-3, rtol=2e-3, what="latent: persistent vs per-kernel batched LM step")
    fl, fd, fv = synth.minicpm_f32_view(lm_w), synth.locdit_f32_view(dit_w), synth.vae_f32_view(vae_w)
    for b in (0, 3):
        want_wav, want_lat, _ = ovx.generate(lm_cfg, fl, dcfg, fd, vcfg, fv, prompts[b], steps, noise[b],
                                             inference_timesteps=10)
        assert_close(lat[b], want_lat, **TOL, what=f"latent[{b}]")
        assert_close(wav[b], want_wav, **TOL, what=f"wav[{b}]")
