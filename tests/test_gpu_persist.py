"""The persistent decode step (one launch per token) against the per-kernel step and the
oracle: greedy ids bit-exact, last logits within the bf16-weight tolerance, one kernel per
replayed step, long-context attention (32 splits), the once-per-KV-head split merge at short
caches, and a second run after reset."""
import os

import numpy as np
import pytest

from oracle import minicpm4 as om
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu

BF16_TOL = dict(atol=2e-2, rtol=2e-2)


def _context(persist, **env):
    """A context created with VX_PERSIST (and any other VX_* settings in ``env``) set; the
    library reads them at context creation."""
    from voxcpm_rs_b200.minicpm4 import Context
    env = {"VX_PERSIST": "1" if persist else "0", **env}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        return Context(0)
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


@pytest.fixture(scope="module")
def two_layer():
    from voxcpm_rs_b200 import config, synth
    cfg = config.lm_decode_config(layers=2, vocab=4096)
    w = synth.minicpm_weights(cfg, seed=0, std=0.2)
    return cfg, w, synth.minicpm_f32_view(w)


def _steps_launches(m, prompt, n):
    from voxcpm_rs_b200._lib import lib
    L = lib()
    c0 = L.vx_launch_count()
    m.greedy(prompt, n)
    return L.vx_launch_count() - c0


def test_persist_matches_per_kernel_and_oracle(two_layer):
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    cfg, w, fw = two_layer
    prompt = synth.prompt_ids(64, cfg.vocab_size, seed=0)
    n_steps = 24
    want, margins = om.greedy_generate(cfg, fw, prompt, n_steps, 4096, return_margins=True)
    assert len(set(want)) > 10 and min(margins) > 1e-3
    got, logits = {}, {}
    for persist in (True, False):
        ctx = _context(persist)
        m = MiniCpmModel(ctx, cfg, w, max_length=4096)
        got[persist] = m.greedy(prompt, n_steps).tolist()
        logits[persist] = m.last_logits().copy()
        # one launch per replayed step on the persistent path, 141-style sequences otherwise
        d8 = _steps_launches(m, prompt, 8)
        d16 = _steps_launches(m, prompt, 16)
        per_step = (d16 - d8) / 8
        assert per_step == (1 if persist else 5 * cfg.num_hidden_layers + 1), per_step
        m.close()
        ctx.close()
    assert got[True] == want, f"persistent: {got[True]} vs {want}"
    assert got[False] == want
    assert_close(logits[True], logits[False], atol=1e-4, rtol=1e-4, what="persistent vs per-kernel logits")


def test_persist_merge_once_short_cache(two_layer):
    """VX_PERSIST_MERGE_TILES=0: at positions 64-88 (3 tiles) the attention splits are merged
    once per KV head by the last split (the long-cache path) instead of by every o_proj CTA;
    ids bit-exact with the oracle, logits within 1e-4 of the default merge."""
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    cfg, w, fw = two_layer
    prompt = synth.prompt_ids(64, cfg.vocab_size, seed=0)
    n_steps = 24
    want = om.greedy_generate(cfg, fw, prompt, n_steps, 4096)
    got, logits = {}, {}
    for tiles in ("16", "0"):
        ctx = _context(True, VX_PERSIST_MERGE_TILES=tiles)
        m = MiniCpmModel(ctx, cfg, w, max_length=4096)
        got[tiles] = m.greedy(prompt, n_steps).tolist()
        logits[tiles] = m.last_logits().copy()
        m.close()
        ctx.close()
    assert got["0"] == want and got["16"] == want
    assert_close(logits["0"], logits["16"], atol=1e-4, rtol=1e-4, what="merge once vs every-CTA merge logits")


def test_persist_long_context(two_layer):
    """1000-id prompt: the attention phase runs 32 splits of 32 positions with the
    last-arriving split merging; ids bit-exact with the oracle, margins checked."""
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    cfg, w, fw = two_layer
    prompt = synth.prompt_ids(1000, cfg.vocab_size, seed=3)
    n_steps = 8
    want, margins = om.greedy_generate(cfg, fw, prompt, n_steps, 4096, return_margins=True)
    ctx = _context(True)
    m = MiniCpmModel(ctx, cfg, w, max_length=4096)
    got = m.greedy(prompt, n_steps).tolist()
    assert got == want, f"{got} vs {want} (margins {margins})"
    m.reset()
    assert m.greedy(prompt, n_steps).tolist() == want
    m.close()
    ctx.close()


def test_persist_small_heads():
    """head_dim 64, hidden 512 (K chunk 512, 24-stage ring) against the oracle."""
    from tests.golden.make_golden import small_lm_config
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    cfg = small_lm_config()
    w = synth.minicpm_weights(cfg, seed=5, std=0.2)
    fw = synth.minicpm_f32_view(w)
    prompt = synth.prompt_ids(40, cfg.vocab_size, seed=5)
    want, margins = om.greedy_generate(cfg, fw, prompt, 30, 512, return_margins=True)
    c = _context(True)
    m = MiniCpmModel(c, cfg, w, max_length=512)
    got = m.greedy(prompt, 30).tolist()
    logits = m.last_logits()
    m.close()
    c.close()
    assert got == want, f"{got} vs {want} (margins {margins})"
    assert np.isfinite(logits).all()
