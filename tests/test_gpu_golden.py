"""GPU path against the committed golden fixtures (small MiniCPM-4: hidden 512, 8/1 heads,
head_dim 64, 2 layers, vocab 512): prefill (causal and not), forward_step, greedy ids."""
import os

import numpy as np
import pytest

from tests.conftest import assert_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = dict(atol=2e-2, rtol=2e-2)


@pytest.fixture(scope="module")
def lm_golden():
    from tests.golden.make_golden import small_lm_config
    from voxcpm_rs_b200 import synth
    cfg = small_lm_config()
    return cfg, synth.minicpm_weights(cfg, seed=5, std=0.2), dict(np.load(os.path.join(GOLDEN, "lm_small.npz")))


def test_golden_prefill_and_step(ctx, lm_golden):
    import torch
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    cfg, w, g = lm_golden
    rng = np.random.default_rng(50)
    x = rng.standard_normal((1, 16, 512), dtype=np.float32)
    e = rng.standard_normal((1, 512), dtype=np.float32)
    m = MiniCpmModel(ctx, cfg, w, max_length=64)
    assert_close(m.forward(torch.from_numpy(x).cuda(), False).cpu().numpy(), g["forward_noncausal"], **TOL,
                 what="non-causal")
    assert_close(m.forward(torch.from_numpy(x).cuda(), True, fill_cache=True).cpu().numpy(), g["prefill_causal"],
                 **TOL, what="causal prefill")
    k1, _ = m.kv_read(1, 16)
    assert_close(k1, g["k_layer1"][0], **TOL, what="k cache layer 1")
    assert_close(m.forward_step(torch.from_numpy(e).cuda()).cpu().numpy()[None], g["step_out"], **TOL,
                 what="forward_step")
    m.close()


def test_golden_greedy_ids(ctx, lm_golden):
    from voxcpm_rs_b200.minicpm4 import MiniCpmModel
    cfg, w, g = lm_golden
    m = MiniCpmModel(ctx, cfg, w, max_length=64)
    assert m.greedy(g["prompt"], 20).tolist() == g["greedy_ids"].tolist()
    m.close()
