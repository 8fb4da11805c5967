"""The allocation-free decode attention entry point (vx_attention_decode_static).

It exists for callers that cannot allocate device memory: hosts that give this library a
fixed memory budget, or real-time threads where a cudaMalloc could stall the device.  Its
scratch lives in a file-scope device array shared by every call.  This test calls it twice
in a row through the C ABI (different lengths, so the second call runs on scratch the
first one left behind) and checks each result against the allocating entry point
vx_attention_decode within the f32 tolerance the other tests use (1e-3 max-abs/rel).

The file name sorts last so that, if it fails, a run that stops at the first failure has
already run every other test.  It needs no state from other tests: it passes alone in a
fresh process and after the full suite.
"""
import numpy as np
import pytest

from tests.conftest import assert_close

pytestmark = pytest.mark.gpu
F32_TOL = dict(atol=1e-3, rtol=1e-3)


def _case(rng, nh, nkv, d, s_max, cur_len, b=1):
    import torch
    q = torch.from_numpy(rng.standard_normal((b, nh * d), dtype=np.float32)).cuda()
    kc = np.zeros((b, nkv, s_max, d), np.float32)
    vc = np.zeros((b, nkv, s_max, d), np.float32)
    kc[:, :, :cur_len] = rng.standard_normal((b, nkv, cur_len, d), dtype=np.float32)
    vc[:, :, :cur_len] = rng.standard_normal((b, nkv, cur_len, d), dtype=np.float32)
    return q, torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()


def test_attention_decode_static_matches_allocating_entry_point(ctx):
    import torch
    from voxcpm_rs_b200._lib import check, lib, ptr
    L = lib()
    rng = np.random.default_rng(99)
    cases = [(16, 2, 128, 4096, 1001, 1), (16, 2, 64, 512, 77, 2)]
    for nh, nkv, d, s_max, cur_len, b in cases:  # two calls in a row on the shared scratch
        q, kc, vc = _case(rng, nh, nkv, d, s_max, cur_len, b)
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        torch.cuda.synchronize()
        check(L.vx_attention_decode(ctx.h, ptr(q), ptr(kc), ptr(vc), b, nh, nkv, d, s_max, cur_len, ptr(want),
                                    None), ctx.h)
        rc = L.vx_attention_decode_static(ptr(q), ptr(kc), ptr(vc), b, nh, nkv, d, s_max, cur_len, ptr(got), None)
        assert rc == 0, f"vx_attention_decode_static returned {rc}"
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), want.cpu().numpy(), **F32_TOL, what=f"static attention len {cur_len}")


def test_attention_decode_static_rejects_oversized_scratch():
    """Shapes whose partials exceed the 1 MiB array are refused with VX_ERR_SHAPE, before
    any device work."""
    from voxcpm_rs_b200._lib import VX_ERR_SHAPE, lib
    L = lib()
    # B * nkv = 8 -> 8 * 16 * 8 * 130 * 4 B = 532,480 B fits; B * nkv = 16 -> 1,064,960 B does not
    dummy = 1 << 20  # never dereferenced: the size check comes first
    assert L.vx_attention_decode_static(dummy, dummy, dummy, 8, 16, 2, 128, 64, 10, dummy, None) == VX_ERR_SHAPE
