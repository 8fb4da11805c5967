"""AudioVAE decoder on the GPU through the C ABI: golden fixture (small decoder), the
end-to-end workload's decoder (latent 64, decoder_dim 2048, rates [2,5,8,8], 16 kHz) against
the oracle, and the causal-prefix property the reference's streaming relies on
(voxcpm2/wrapper.rs:439-442: decoding a longer latent reproduces the shorter decode's
samples).  Tolerance 2e-2 max-abs/rel (bf16-weight path)."""
import os

import numpy as np
import pytest

from oracle import audiovae as oav
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-2, rtol=2e-2)
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_golden_vae_small(ctx):
    from tests.golden.make_golden import small_vae_config
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.audiovae import AudioVae
    g = dict(np.load(os.path.join(GOLDEN, "vae_small.npz")))
    vcfg = small_vae_config()
    vae = AudioVae(ctx, vcfg, synth.vae_weights(vcfg, seed=7))
    z = np.random.default_rng(70).standard_normal((1, 64, 8), dtype=np.float32)
    got = vae.decode(_t(z)).cpu().numpy()
    assert_close(got, g["wav"], **TOL, what="small VAE")
    vae.close()


@pytest.fixture(scope="module")
def c5_vae():
    from voxcpm_rs_b200 import config, synth
    vcfg = config.vae_config()
    w = synth.vae_weights(vcfg, seed=0)
    return vcfg, w, synth.vae_f32_view(w)


@pytest.mark.parametrize("T,B", [(16, 1), (24, 2)])
def test_vae_decode_c5(ctx, c5_vae, T, B):
    from voxcpm_rs_b200.audiovae import AudioVae
    vcfg, w, fw = c5_vae
    z = np.random.default_rng(T).standard_normal((B, 64, T), dtype=np.float32)
    want = oav.decoder_forward(vcfg, fw, z)
    vae = AudioVae(ctx, vcfg, w)
    got = vae.decode(_t(z)).cpu().numpy()
    assert got.shape == (B, 1, T * 640)
    assert_close(got, want, **TOL, what="VAE decode")
    assert np.abs(got - want).max() < 2e-3
    vae.close()


def test_vae_causal_prefix(ctx, c5_vae):
    """Decoding the first 12 latent frames gives exactly the first 12*640 samples of
    decoding all 20 (the decoder is causal)."""
    from voxcpm_rs_b200.audiovae import AudioVae
    vcfg, w, _ = c5_vae
    z = np.random.default_rng(5).standard_normal((1, 64, 20), dtype=np.float32)
    vae = AudioVae(ctx, vcfg, w)
    full = vae.decode(_t(z)).cpu().numpy()
    part = vae.decode(_t(z[:, :, :12])).cpu().numpy()
    assert np.array_equal(part, full[:, :, :12 * 640])
    vae.close()


@pytest.mark.slow
def test_vae_decode_c5_t256(ctx, c5_vae):
    """The end-to-end workload's decoder at T = 256 latent frames (163,840 samples): the
    full channel ladder 2048 -> 1024 -> 512 -> 256 -> 128 at a length where every block's
    tiles run many times over."""
    from voxcpm_rs_b200.audiovae import AudioVae
    vcfg, w, fw = c5_vae
    z = np.random.default_rng(256).standard_normal((1, 64, 256), dtype=np.float32)
    want = oav.decoder_forward(vcfg, fw, z)
    vae = AudioVae(ctx, vcfg, w)
    got = vae.decode(_t(z)).cpu().numpy()
    vae.close()
    assert got.shape == (1, 1, 256 * 640)
    assert_close(got, want, **TOL, what="VAE decode T=256")
    assert np.abs(got - want).max() < 2e-3


@pytest.mark.parametrize("chunks", [[5, 3, 7, 1, 4], [1] * 10, [16]])
def test_vae_stream_bit_exact(ctx, c5_vae, chunks):
    """Stateful chunked decode (vx_vae_stream_decode) reproduces the one-shot decode bit for
    bit, whatever the chunking (generate_stream's chunks, voxcpm2/wrapper.rs:669-724), for two
    utterances at once; reset starts over."""
    from voxcpm_rs_b200.audiovae import AudioVae, AudioVaeStream
    vcfg, w, _ = c5_vae
    T = sum(chunks)
    z = np.random.default_rng(77).standard_normal((2, 64, T), dtype=np.float32)
    vae = AudioVae(ctx, vcfg, w)
    full = vae.decode(_t(z)).cpu().numpy()
    st = AudioVaeStream(vae, B=2)
    for rep in range(2):
        parts, t0 = [], 0
        for c in chunks:
            parts.append(st.decode(_t(z[:, :, t0:t0 + c])).cpu().numpy())
            t0 += c
        got = np.concatenate(parts, axis=2)
        assert got.shape == full.shape
        assert np.array_equal(got, full), f"max diff {np.abs(got - full).max()}"
        st.reset()
    st.close()
    vae.close()
