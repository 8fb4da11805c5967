"""LocDiT forward and the CFM solve on the GPU through the C ABI, against the golden
fixture (small DiT) and the oracle (the full LocDiT workload: 8 layers, hidden 1024,
16/2 heads, head_dim 64, MLP 4096, 4-frame x 64-dim patches, CFG 2.0, 10 Euler steps).
Tolerance 2e-2 max-abs/rel (bf16-weight path)."""
import os

import numpy as np
import pytest

from oracle import locdit as old
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-2, rtol=2e-2)
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_golden_cfm_small(ctx):
    from tests.golden.make_golden import small_dit_config
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    g = dict(np.load(os.path.join(GOLDEN, "cfm_small.npz")))
    dcfg = small_dit_config()
    dit = VoxCpmLocDiTV2(ctx, dcfg, synth.locdit_weights(dcfg, in_channels=64, seed=6))
    rng = np.random.default_rng(60)
    mu = rng.standard_normal((1, 1024), dtype=np.float32)
    cond = rng.standard_normal((1, 64, 4), dtype=np.float32)
    z = rng.standard_normal((1, 64, 4), dtype=np.float32)
    got = dit.cfm_forward(_t(mu), 4, _t(cond), _t(z), 2.0, 0.0, False).cpu().numpy()
    assert_close(got, g["x_uniform"], **TOL, what="cfm uniform")
    got = dit.cfm_forward(_t(mu), 4, _t(cond), _t(z), 2.0, 1.0, True).cpu().numpy()
    assert_close(got, g["x_sway_zero_star"], **TOL, what="cfm sway + zero-star")
    x2 = rng.standard_normal((2, 64, 4), dtype=np.float32)
    mu2 = np.concatenate([mu, np.zeros_like(mu)])
    got = dit.forward(_t(x2), _t(mu2), [0.7, 0.7], _t(np.concatenate([cond, cond])), [0.0, 0.0]).cpu().numpy()
    assert_close(got, g["dit_forward"], **TOL, what="dit forward")
    dit.close()


@pytest.fixture(scope="module")
def full_dit():
    from voxcpm_rs_b200 import config, synth
    lm = config.lm_decode_config(layers=1, vocab=0)
    dcfg = config.locdit_config(lm)
    w = synth.locdit_weights(dcfg, in_channels=64, seed=0)
    return dcfg, w, synth.locdit_f32_view(w)


def test_dit_forward_full(ctx, full_dit):
    """One LocDiT forward at the full width with per-row t and dt (mean-mode inputs)."""
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    dcfg, w, fw = full_dit
    rng = np.random.default_rng(20)
    x = rng.standard_normal((2, 64, 4), dtype=np.float32)
    mu = rng.standard_normal((2, 2048), dtype=np.float32)
    cond = rng.standard_normal((2, 64, 4), dtype=np.float32)
    t = np.array([0.3, 0.9], np.float32)
    dt = np.array([0.1, 0.0], np.float32)
    want = old.dit_forward(dcfg, fw, x, mu, t, cond, dt)
    dit = VoxCpmLocDiTV2(ctx, dcfg, w)
    got = dit.forward(_t(x), _t(mu), t, _t(cond), dt).cpu().numpy()
    assert_close(got, want, **TOL, what="dit forward")
    dit.close()


@pytest.mark.parametrize("sway,zero_star", [(0.0, False), (1.0, True)])
def test_cfm_solve_full(ctx, full_dit, sway, zero_star):
    """UnifiedCfm::forward at the LocDiT workload: CFG 2.0, 10 Euler steps, t uniform
    (sway 0, zero-star off) and the reference default (sway 1, zero-star on); B = 2."""
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    dcfg, w, fw = full_dit
    rng = np.random.default_rng(21)
    B = 2
    mu = rng.standard_normal((B, 2048), dtype=np.float32)
    cond = np.zeros((B, 64, 4), np.float32)
    cond[1] = rng.standard_normal((64, 4), dtype=np.float32)
    z = rng.standard_normal((B, 64, 4), dtype=np.float32)
    want = old.cfm_forward(dcfg, fw, mu, 10, cond, z, 2.0, sway, zero_star)
    dit = VoxCpmLocDiTV2(ctx, dcfg, w)
    got = dit.cfm_forward(_t(mu), 10, _t(cond), _t(z), 2.0, sway, zero_star).cpu().numpy()
    assert_close(got, want, **TOL, what="cfm solve")
    assert np.abs(got - want).max() < 2e-3
    dit.close()


@pytest.mark.parametrize("knob", ["VX_PRESPLIT", "VX_ATT_ROPE_FUSED"])
def test_dit_forward_fusions_are_exact(full_dit, knob):
    """Fusions that must not change a bit of the per-kernel LocDiT forward:
    VX_PRESPLIT — the RMSNorm, attention and SiLU*up kernels write the few-row GEMMs' split
    operand themselves (default) instead of a separate split kernel;
    VX_ATT_ROPE_FUSED — the attention rotates q / k as it loads them from the fused
    projection (default) instead of after a separate RoPE + scatter pass."""
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import Context
    dcfg, w, _ = full_dit
    rng = np.random.default_rng(22)
    x = rng.standard_normal((2, 64, 4), dtype=np.float32)
    mu = rng.standard_normal((2, 2048), dtype=np.float32)
    cond = rng.standard_normal((2, 64, 4), dtype=np.float32)
    outs = []
    for flag in ("0", "1"):
        old_env = os.environ.get(knob)
        os.environ[knob] = flag
        try:
            c = Context(0)
        finally:
            if old_env is None:
                del os.environ[knob]
            else:
                os.environ[knob] = old_env
        dit = VoxCpmLocDiTV2(c, dcfg, w)
        outs.append(dit.forward(_t(x), _t(mu), [0.4, 0.4], _t(cond), [0.0, 0.0]).cpu().numpy())
        dit.close()
        c.close()
    assert np.array_equal(outs[0], outs[1]), np.abs(outs[0] - outs[1]).max()


def _dit_with_env(ctx, dcfg, w, persist):
    """A DiT whose decoder forward policy is fixed by VX_DIT_PERSIST (read at creation)."""
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    old_env = os.environ.get("VX_DIT_PERSIST")
    os.environ["VX_DIT_PERSIST"] = persist
    try:
        return VoxCpmLocDiTV2(ctx, dcfg, w)
    finally:
        if old_env is None:
            del os.environ["VX_DIT_PERSIST"]
        else:
            os.environ["VX_DIT_PERSIST"] = old_env


@pytest.mark.parametrize("persist", ["1", "0"])
def test_dit_forward_full_both_paths(ctx, full_dit, persist):
    """The full-width LocDiT forward through the persistent one-launch decoder (forced at two
    sequences) and through the per-kernel decoder, each against the oracle."""
    dcfg, w, fw = full_dit
    rng = np.random.default_rng(23)
    x = rng.standard_normal((2, 64, 4), dtype=np.float32)
    mu = rng.standard_normal((2, 2048), dtype=np.float32)
    cond = rng.standard_normal((2, 64, 4), dtype=np.float32)
    t = np.array([0.6, 0.2], np.float32)
    dt = np.array([0.0, 0.3], np.float32)
    want = old.dit_forward(dcfg, fw, x, mu, t, cond, dt)
    dit = _dit_with_env(ctx, dcfg, w, persist)
    got = dit.forward(_t(x), _t(mu), t, _t(cond), dt).cpu().numpy()
    assert_close(got, want, **TOL, what=f"dit forward (VX_DIT_PERSIST={persist})")
    dit.close()


def test_cfm_solve_batch8(ctx, full_dit):
    """The CFM solve for 8 patches at once (16 CFG sequences, 176 decoder rows: the persistent
    decoder by default) against the oracle, and bit-identical when run twice (the split-K
    partials are summed in a fixed order)."""
    dcfg, w, fw = full_dit
    rng = np.random.default_rng(24)
    B = 8
    mu = rng.standard_normal((B, 2048), dtype=np.float32)
    cond = (0.5 * rng.standard_normal((B, 64, 4))).astype(np.float32)
    z = rng.standard_normal((B, 64, 4), dtype=np.float32)
    want = old.cfm_forward(dcfg, fw, mu, 10, cond, z, 2.0, 1.0, True)
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    dit = VoxCpmLocDiTV2(ctx, dcfg, w)
    got = dit.cfm_forward(_t(mu), 10, _t(cond), _t(z), 2.0, 1.0, True).cpu().numpy()
    again = dit.cfm_forward(_t(mu), 10, _t(cond), _t(z), 2.0, 1.0, True).cpu().numpy()
    assert_close(got, want, **TOL, what="cfm solve B=8")
    assert np.abs(got - want).max() < 2e-3
    assert np.array_equal(got, again)
    dit.close()


@pytest.mark.parametrize("B", [3, 11])
def test_cfm_solve_ragged_batches(ctx, full_dit, B):
    """Patch counts whose decoder rows are not a multiple of 32 (3 patches: 66 rows, padded to
    96; 11 patches: 242 rows, padded to 256, the largest stack) through the persistent decoder,
    against the oracle."""
    dcfg, w, fw = full_dit
    rng = np.random.default_rng(25 + B)
    mu = rng.standard_normal((B, 2048), dtype=np.float32)
    cond = (0.5 * rng.standard_normal((B, 64, 4))).astype(np.float32)
    z = rng.standard_normal((B, 64, 4), dtype=np.float32)
    want = old.cfm_forward(dcfg, fw, mu, 10, cond, z, 2.0, 1.0, True)
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    dit = VoxCpmLocDiTV2(ctx, dcfg, w, max_rows=2 * B)
    got = dit.cfm_forward(_t(mu), 10, _t(cond), _t(z), 2.0, 1.0, True).cpu().numpy()
    assert_close(got, want, **TOL, what=f"cfm solve B={B}")
    assert np.abs(got - want).max() < 2e-3
    dit.close()
