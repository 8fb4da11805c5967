"""tcgen05 few-row GEMM (bf16 weights x hi/lo-split activations, f32 accumulation in TMEM)
through vx_linear_bf16 against the oracle's f32 Linear, over the row counts the prefill and
the DiT use, with and without bias, single K split and split-K with the last-CTA reduction,
and output widths that are not a multiple of 128 (the batched greedy head's 73,448-row
tied embedding).
Tolerance 2e-2 (bf16-weight path); the split keeps the error near f32 (< 1e-4 checked)."""
import numpy as np
import pytest

from oracle import minicpm4 as om
from tests.conftest import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k,bias", [(2, 1024, 64, True), (3, 128, 128, False), (16, 1024, 1024, True),
                                        (22, 1280, 1024, False), (22, 8192, 1024, False), (22, 1024, 4096, True),
                                        (64, 2560, 2048, False), (100, 2048, 6144, False), (128, 12288, 2048, True),
                                        (129, 1024, 1024, False), (176, 1280, 1024, True), (176, 1024, 4096, False),
                                        (256, 2048, 2048, True), (300, 1024, 1024, False),
                                        (8, 1000, 2048, True), (8, 73448, 2048, False), (3, 200, 128, False)])
def test_tc_linear(ctx, m, n, k, bias):
    import torch
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import linear_bf16
    rng = np.random.default_rng(m * 7 + n + k)
    wb = synth.bf16_bits(0.02 * rng.standard_normal((n, k), dtype=np.float32))
    x = rng.standard_normal((m, k), dtype=np.float32)
    b = (0.02 * rng.standard_normal(n)).astype(np.float32) if bias else None
    want = om.linear(x, synth.bf16_to_f32(wb), b)
    got = linear_bf16(ctx, torch.from_numpy(wb.view(np.int16)).cuda(), torch.from_numpy(x).cuda(),
                      None if b is None else torch.from_numpy(b).cuda())
    ctx.synchronize()
    got = got.cpu().numpy()
    assert_close(got, want, atol=2e-2, rtol=2e-2, what="tc linear")
    assert np.abs(got - want).max() < 1e-4, np.abs(got - want).max()
