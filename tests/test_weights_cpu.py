"""Checkpoint parsing on the host (no GPU): safetensors and PyTorch zip checkpoints read
through the C ABI (``vx_weights_*``) against what the files were written from, the
state-dict flattening / prefix stripping of ``load_single_pth`` (weights.rs:400-411), the
weight_norm materialisation (weights.rs:447-471) against torch, and malformed files
rejected with an error instead of a crash."""
import os

import numpy as np
import pytest
import torch


def _ck(path):
    from voxcpm_rs_b200.weights import Checkpoint
    return Checkpoint(path)


def _tensors():
    g = torch.Generator().manual_seed(0)
    return {"a.weight": torch.randn(3, 4, generator=g),
            "a.bias": torch.randn(4, generator=g).to(torch.float16),
            "b.w": torch.randn(5, 2, 3, generator=g).to(torch.bfloat16),
            "c.ids": torch.arange(7, dtype=torch.int64),
            "d.scalar": torch.tensor(2.5, dtype=torch.float64)}


def _check_all(ck, ts, prefix=""):
    names = set(ck.names())
    assert names == {prefix + k for k in ts}
    for k, t in ts.items():
        dt, shape = ck.info(prefix + k)
        assert shape == tuple(t.shape), k
        got = ck.read(prefix + k, tuple(t.shape))
        assert np.array_equal(got, t.to(torch.float32).numpy()), k
        if t.dtype == torch.bfloat16:
            bits = ck.read(prefix + k, tuple(t.shape), dtype="bf16")
            assert np.array_equal(bits, t.view(torch.int16).numpy().view(np.uint16))
        if t.dtype == torch.float32:  # f32 -> bf16 rounds to nearest even, as torch does
            bits = ck.read(prefix + k, tuple(t.shape), dtype="bf16")
            assert np.array_equal(bits, t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def test_safetensors_roundtrip(tmp_path):
    from safetensors.torch import save_file
    ts = _tensors()
    p = str(tmp_path / "m.safetensors")
    save_file(ts, p, metadata={"format": "pt"})
    with _ck(p) as ck:
        _check_all(ck, ts)


@pytest.mark.parametrize("wrap", [None, "state_dict", "model_state_dict", "module"])
def test_torch_zip_roundtrip(tmp_path, wrap):
    ts = _tensors()
    obj = dict(ts)
    if wrap == "module":
        obj = {"module." + k: v for k, v in ts.items()}
    elif wrap:
        obj = {wrap: dict(ts), "epoch": 3}
    p = str(tmp_path / "m.pth")
    torch.save(obj, p)
    with _ck(p) as ck:
        _check_all(ck, ts)


def test_torch_zip_nested_and_parameters(tmp_path):
    """Nested dicts flatten with '.', nn.Parameter values load like tensors; a
    non-contiguous view is refused."""
    lin = torch.nn.Linear(4, 3)
    sd = {"enc": {"proj": lin.state_dict()}, "p": torch.nn.Parameter(torch.ones(2))}
    p = str(tmp_path / "n.pth")
    torch.save(sd, p)
    with _ck(p) as ck:
        assert set(ck.names()) == {"enc.proj.weight", "enc.proj.bias", "p"}
        assert np.array_equal(ck.read("enc.proj.weight", (3, 4)), lin.weight.detach().numpy())
        assert np.array_equal(ck.read("p", (2,)), np.ones(2, np.float32))
    q = str(tmp_path / "t.pth")
    torch.save({"x": torch.randn(4, 6).t()}, q)
    from voxcpm_rs_b200._lib import VxError
    with pytest.raises(VxError):
        _ck(q)


def test_weight_norm_materialised(tmp_path):
    """X.weight_g + X.weight_v -> X.weight = g * v / ||v|| per output channel (dim 0), as
    torch's weight_norm computes it; for a ConvTranspose1d weight [C_in, C_out, k] dim 0 is
    C_in, as in the checkpoint."""
    from safetensors.torch import save_file
    torch.manual_seed(1)
    conv = torch.nn.utils.weight_norm(torch.nn.Conv1d(6, 5, 7))
    up = torch.nn.utils.weight_norm(torch.nn.ConvTranspose1d(8, 4, 4, stride=2))
    sd = {"c." + k: v.detach().contiguous() for k, v in conv.state_dict().items()}
    sd.update({"u." + k: v.detach().contiguous() for k, v in up.state_dict().items()})
    p = str(tmp_path / "wn.safetensors")
    save_file(sd, p)
    conv_w = torch._weight_norm(conv.weight_v, conv.weight_g, 0).detach().numpy()
    up_w = torch._weight_norm(up.weight_v, up.weight_g, 0).detach().numpy()
    with _ck(p) as ck:
        np.testing.assert_allclose(ck.read("c.weight", conv_w.shape), conv_w, rtol=2e-6, atol=1e-7)
        np.testing.assert_allclose(ck.read("u.weight", up_w.shape), up_w, rtol=2e-6, atol=1e-7)
        assert np.array_equal(ck.read("c.bias", (5,)), conv.bias.detach().numpy())
        from voxcpm_rs_b200._lib import VxError
        with pytest.raises(VxError):
            ck.read("c.weight", (5, 6, 6))  # wrong element count
        with pytest.raises(VxError):
            ck.read("missing.weight", (1,))


def test_malformed_files_rejected(tmp_path):
    from safetensors.torch import save_file
    from voxcpm_rs_b200._lib import VxError
    good = str(tmp_path / "g.safetensors")
    save_file({"a": torch.ones(1000)}, good)
    raw = open(good, "rb").read()
    cases = {"trunc.safetensors": raw[:len(raw) // 2], "hdr.safetensors": raw[:8] + b"{nope" + raw[13:],
             "junk.bin": os.urandom(4096), "tiny.bin": b"abc", "zip.pth": b"PK" + os.urandom(300)}
    for name, data in cases.items():
        p = tmp_path / name
        p.write_bytes(data)
        with pytest.raises(VxError):
            _ck(str(p))
    with pytest.raises(VxError):
        _ck(str(tmp_path / "does_not_exist.safetensors"))
