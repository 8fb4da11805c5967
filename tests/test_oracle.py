"""CPU checks of the oracle: against independent torch-CPU implementations of the same
operators, against the committed golden fixtures, and the host-side arithmetic the
reference does in f64 (t-span / sway, zero-init steps, LongRoPE scaling, SR buckets)."""
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import audiovae as oav
from oracle import locdit as old
from oracle import minicpm4 as om

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_rms_norm_vs_torch():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((16, 2048), dtype=np.float32)
    w = (1 + 0.02 * rng.standard_normal(2048)).astype(np.float32)
    want = F.rms_norm(torch.from_numpy(x), (2048,), torch.from_numpy(w), 1e-6).numpy()
    assert np.abs(om.rms_norm(x, w, 1e-6) - want).max() < 1e-5


@pytest.mark.parametrize("causal", [True, False])
def test_sdpa_vs_torch(causal):
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((2, 8, 13, 64), dtype=np.float32) for _ in range(3))
    want = F.scaled_dot_product_attention(*map(torch.from_numpy, (q, k, v)), is_causal=causal).numpy()
    assert np.abs(om.sdpa(q, k, v, 1 / math.sqrt(64), causal) - want).max() < 1e-5


def test_rope_rotate_half_vs_torch():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((1, 2, 3, 8), dtype=np.float32)
    want = torch.cat([-torch.from_numpy(x)[..., 4:], torch.from_numpy(x)[..., :4]], -1).numpy()
    assert np.array_equal(om.rotate_half(x), want)


def test_silu_vs_torch():
    x = np.linspace(-30, 30, 1001, dtype=np.float32)
    assert np.abs(om.silu_stable(x) - F.silu(torch.from_numpy(x)).numpy()).max() < 1e-5


@pytest.mark.parametrize("stride", [2, 5, 8])
def test_conv_transpose_vs_torch(stride):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1, 12, 9), dtype=np.float32)
    w = rng.standard_normal((12, 6, 2 * stride), dtype=np.float32)
    b = rng.standard_normal(6, dtype=np.float32)
    want = F.conv_transpose1d(*map(torch.from_numpy, (x, w, b)), stride=stride).numpy()
    assert np.abs(oav.conv_transpose1d(x, w, b, stride) - want).max() < 1e-4
    trimmed = oav.causal_transpose_conv1d(x, w, b, stride)
    assert trimmed.shape[2] == 9 * stride


@pytest.mark.parametrize("dil", [1, 3, 9])
def test_causal_depthwise_conv_vs_torch(dil):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 16, 40), dtype=np.float32)
    w = rng.standard_normal((16, 1, 7), dtype=np.float32)
    b = rng.standard_normal(16, dtype=np.float32)
    pad = 3 * dil
    want = F.conv1d(F.pad(torch.from_numpy(x), (2 * pad, 0)), torch.from_numpy(w), torch.from_numpy(b),
                    dilation=dil, groups=16).numpy()
    got = oav.causal_conv1d(x, w, b, dil, 16, pad, 0)
    assert got.shape == (1, 16, 40)
    assert np.abs(got - want).max() < 1e-4


def test_pointwise_and_dense_conv_vs_torch():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 8, 20), dtype=np.float32)
    w1 = rng.standard_normal((4, 8, 1), dtype=np.float32)
    w7 = rng.standard_normal((4, 8, 7), dtype=np.float32)
    b = rng.standard_normal(4, dtype=np.float32)
    for w, pad in ((w1, 0), (w7, 3)):
        want = F.conv1d(F.pad(torch.from_numpy(x), (2 * pad, 0)), torch.from_numpy(w), torch.from_numpy(b)).numpy()
        assert np.abs(oav.causal_conv1d(x, w, b, 1, 1, pad, 0) - want).max() < 1e-4


def test_t_span_and_zero_init():
    """unified_cfm.rs:59-67,85: uniform grid without sway, sway transform with coef 1."""
    t = old.t_span(10, 0.0)
    assert t[0] == 1.0 and t[-1] == 0.0 and len(t) == 11
    assert np.allclose(np.diff(t), -0.1, atol=1e-6)
    ts = old.t_span(10, 1.0)
    tt = 0.5
    assert abs(float(ts[5]) - (tt + (math.cos(math.pi / 4) - 1 + tt))) < 1e-6
    assert old.zero_init_steps(11) == 1 and old.zero_init_steps(51) == 2 and old.zero_init_steps(25) == 1


def test_longrope_scaling():
    """rope.rs:22-29: short factors and scale 1 at max_pos == original; long factors and
    sqrt(1 + ln(2)/ln(32768)) at 65536."""
    from voxcpm_rs_b200 import config
    c1 = config.lm_decode_config(layers=1, vocab=0)
    c2 = config.lm_decode_config(layers=1, vocab=0, max_position_embeddings=65536)
    inv1, ext1, sf1 = om.longrope_params(c1)
    inv2, ext2, sf2 = om.longrope_params(c2)
    assert sf1 == 1.0 and abs(sf2 - math.sqrt(1 + math.log(2) / math.log(32768))) < 1e-15
    assert np.array_equal(ext1, np.asarray(c1.rope_scaling.short_factor, np.float32).astype(np.float64))
    assert np.array_equal(ext2, np.asarray(c2.rope_scaling.long_factor, np.float32).astype(np.float64))
    cos, sin = om.longrope_table(c1, 8)
    assert np.array_equal(cos[:, :64], cos[:, 64:]) and np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)


def test_sr_bucket():
    """layers.rs:225-228 bucketize."""
    b = [20000, 30000, 40000]
    assert [oav.sr_bucket(s, b) for s in (16000, 20000, 29999, 44100, 48000)] == [0, 1, 1, 3, 3]


def test_cfg_zero_star_algebra():
    """unified_cfm.rs:143-149: neg*st*(1-cfg) + pos*cfg == neg*st + (pos - neg*st)*cfg."""
    rng = np.random.default_rng(6)
    pos, neg = rng.standard_normal((2, 3, 64, 4)).astype(np.float32)
    v = old.cfg_combine(pos, neg, 2.0, True)
    st = (np.sum(pos * neg, axis=(1, 2)) / (np.sum(neg * neg, axis=(1, 2)) + 1e-8))[:, None, None]
    assert np.abs(v - (neg * st + (pos - neg * st) * 2.0)).max() < 1e-4


def _golden(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.fail(f"missing golden fixture {path}; run tests/golden/make_golden.py")
    return dict(np.load(path, allow_pickle=False))


def test_golden_lm():
    """The oracle reproduces its committed small-LM fixture (prefill, steps, greedy ids)."""
    from tests.golden.make_golden import lm_case
    g = _golden("lm_small.npz")
    got = lm_case()
    for k, v in g.items():
        if v.dtype.kind in "iu":
            assert np.array_equal(got[k], v), k
        else:
            assert np.abs(got[k] - v).max() <= 1e-5 * max(1.0, np.abs(v).max()), k


def test_golden_cfm():
    from tests.golden.make_golden import cfm_case
    g = _golden("cfm_small.npz")
    got = cfm_case()
    for k, v in g.items():
        assert np.abs(got[k] - v).max() <= 1e-5 * max(1.0, np.abs(v).max()), k


def test_golden_vae():
    from tests.golden.make_golden import vae_case
    g = _golden("vae_small.npz")
    got = vae_case()
    for k, v in g.items():
        assert np.abs(got[k] - v).max() <= 1e-5 * max(1.0, np.abs(v).max()), k


def test_round_half_away():
    """Rust f32::round semantics used by the FSQ restatement: ties away from zero."""
    from oracle.voxcpm import round_half_away
    got = round_half_away(np.array([0.5, 1.5, 2.5, -0.5, -1.5, 0.49, -2.51], np.float32))
    assert got.tolist() == [1.0, 2.0, 3.0, -1.0, -2.0, 0.0, -3.0]


def test_scalar_quantization_vs_torch():
    """ScalarQuantizationLayer::forward (fsq.rs:24-29) restated in numpy vs torch-CPU."""
    import torch
    from oracle.voxcpm import scalar_quantization
    rng = np.random.default_rng(3)
    h = rng.standard_normal((3, 256), dtype=np.float32)
    w_in = (0.05 * rng.standard_normal((64, 256))).astype(np.float32)
    b_in = (0.02 * rng.standard_normal(64)).astype(np.float32)
    w_out = (0.05 * rng.standard_normal((128, 64))).astype(np.float32)
    b_out = (0.02 * rng.standard_normal(128)).astype(np.float32)
    got, _ = scalar_quantization(h, w_in, b_in, w_out, b_out, 9)
    t = lambda a: torch.from_numpy(a)  # noqa: E731
    lat = torch.tanh(torch.nn.functional.linear(t(h), t(w_in), t(b_in))) * 9
    q = torch.sign(lat) * torch.floor(lat.abs() + 0.5) / 9
    want = torch.nn.functional.linear(q, t(w_out), t(b_out)).numpy()
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=1e-5)


def test_voxcpm2_loop_semantics():
    """oracle.voxcpm2.inference follows model.rs:318-347: the stop head only ends the loop at
    a step i > min_len, the patch of the stopping step is kept, and with min_len >= max_len
    every step runs; the stacked latent's prefix does not depend on min_len."""
    import numpy as np
    from oracle import voxcpm2 as ov2
    from tests.test_gpu_voxcpm2 import inputs, oracle_cfgs, small_voxcpm2
    from voxcpm_rs_b200 import synth
    v = small_voxcpm2()
    fw = synth.voxcpm2_f32_view(synth.voxcpm2_weights(v, seed=2, std=0.05))
    ids, tm, feat, fm, noise = inputs(2)
    lat, lg = ov2.inference(oracle_cfgs(v), fw, ids, tm, feat, fm, 2, 12, 10, 2.0, noise)
    n = lat.shape[1] // 4
    stops = lg[:, 1] > lg[:, 0]
    assert stops[n - 1] and n - 1 > 2 and not any(stops[3:n - 1])
    lat_all, lg_all = ov2.inference(oracle_cfgs(v), fw, ids, tm, feat, fm, 12, 12, 10, 2.0, noise)
    assert lat_all.shape[1] == 48
    assert np.array_equal(lat_all[:, :4 * n], lat)
