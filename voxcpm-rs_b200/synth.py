"""Seeded random-init weights and inputs (the counterpart of ``VoxCPM::from_config``,
reference ``src/voxcpm2/wrapper.rs:266-281``, which builds a randomly initialised model).

Weights are produced in the checkpoint layout the reference loads
(``src/weights.rs:637-772``): linear weights ``[out, in]`` with separate q/k/v and
gate/up tensors, stored as bf16 bit patterns (``uint16``), so that the same host
arrays feed the CUDA library (which keeps bf16) and any f32 restatement (which
upcasts them exactly, as ``weights.rs:35-44`` does).

Every tensor draws from its own ``numpy.random.default_rng([seed, tag...])`` (PCG64)
stream so that generating one layer never depends on generating another.
"""
from __future__ import annotations

import zlib

import numpy as np

F32 = np.float32


def bf16_bits(a) -> np.ndarray:
    """Round f32 to bf16 (round-to-nearest-even) and return the bit patterns."""
    import torch  # host-side conversion only (multi-threaded RNE cast)
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=F32))
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def bf16_to_f32(bits) -> np.ndarray:
    """Exact upcast of bf16 bit patterns to f32 (torch's multi-threaded cast: the bits are
    moved into the high half of each f32, nothing is rounded)."""
    import torch
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).float().numpy()


def _rng(seed, *tags):
    key = [int(seed)] + [zlib.crc32(str(t).encode()) for t in tags]
    return np.random.default_rng(key)


def normal(seed, shape, std=1.0, mean=0.0, *tags):
    g = _rng(seed, *tags)
    x = g.standard_normal(size=shape, dtype=F32)
    if std != 1.0:
        x *= F32(std)
    if mean != 0.0:
        x += F32(mean)
    return x


def normal_bf16(seed, shape, std, mean, *tags):
    return bf16_bits(normal(seed, shape, std, mean, *tags))


# -------------------------------------------------------------------- MiniCPM-4

def _parallel(jobs):
    """Run independent ``(key, fn)`` draws on a thread pool (numpy releases the GIL while
    filling large arrays; each tensor has its own stream, so the order is irrelevant)."""
    from concurrent.futures import ThreadPoolExecutor
    import os
    with ThreadPoolExecutor(max(1, min(16, os.cpu_count() or 1))) as ex:
        futs = {k: ex.submit(fn) for k, fn in jobs}
        return {k: f.result() for k, f in futs.items()}


def minicpm_weights(cfg, seed=0, std=0.02, prefix="lm"):
    """Random-init MiniCPM-4 weights: bf16 linears ~N(0, std), bf16 norm weights
    ~N(1, 0.02), tied bf16 embedding ~N(0, std) when ``vocab_size > 0``."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    d = cfg.head_dim()
    qs, ks = cfg.num_attention_heads * d, cfg.num_key_value_heads * d
    shapes = {"q": (qs, H), "k": (ks, H), "v": (ks, H), "o": (H, qs),
              "gate": (I, H), "up": (I, H), "down": (H, I)}
    jobs = []
    for li in range(cfg.num_hidden_layers):
        for name, shp in shapes.items():
            jobs.append(((li, name), lambda li=li, name=name, shp=shp:
                         normal_bf16(seed, shp, std, 0.0, prefix, li, name)))
        for name in ("ln_in", "ln_post"):
            jobs.append(((li, name), lambda li=li, name=name:
                         bf16_to_f32(normal_bf16(seed, (H,), 0.02, 1.0, prefix, li, name))))
    if cfg.vocab_size > 0:
        jobs.append((("embed",), lambda: normal_bf16(seed, (cfg.vocab_size, H), std, 0.0, prefix, "embed")))
    got = _parallel(jobs)
    layers = [{name: got[(li, name)] for name in list(shapes) + ["ln_in", "ln_post"]}
              for li in range(cfg.num_hidden_layers)]
    return {"layers": layers,
            "norm": bf16_to_f32(normal_bf16(seed, (H,), 0.02, 1.0, prefix, "norm")),
            "embed": got.get(("embed",))}


def minicpm_f32_view(w):
    """f32 model-layout view (q|k|v and gate|up fused along ``out``, as
    ``src/weights.rs:648-772`` fuses them) for an f32 restatement."""
    def layer(l):
        return {
            "wqkv": bf16_to_f32(np.concatenate([l["q"], l["k"], l["v"]], 0)),
            "wo": bf16_to_f32(l["o"]),
            "wgu": bf16_to_f32(np.concatenate([l["gate"], l["up"]], 0)),
            "wd": bf16_to_f32(l["down"]),
            "ln_in": l["ln_in"], "ln_post": l["ln_post"],
        }
    got = _parallel([(i, lambda l=l: layer(l)) for i, l in enumerate(w["layers"])])
    return {
        "embed": None if w["embed"] is None else bf16_to_f32(w["embed"]),
        "norm": w["norm"],
        "layers": [got[i] for i in range(len(w["layers"]))],
    }


# ------------------------------------------------------------------------ LocDiT

def _lin(seed, out_f, in_f, std, *tags):
    return (normal_bf16(seed, (out_f, in_f), std, 0.0, *tags, "w"),
            bf16_to_f32(normal_bf16(seed, (out_f,), std, 0.0, *tags, "b")))


def locdit_weights(dcfg, in_channels=64, seed=0, std=0.02):
    """Random-init ``VoxCpmLocDiTV2`` (``src/locdit/local_dit.rs:83-96``): biased
    in/cond/out projections and time MLPs, plus a MiniCPM-4 decoder without vocab."""
    H = dcfg.hidden_size
    w = {}
    w["in_proj_w"], w["in_proj_b"] = _lin(seed, H, in_channels, std, "dit", "in_proj")
    w["cond_proj_w"], w["cond_proj_b"] = _lin(seed, H, in_channels, std, "dit", "cond_proj")
    w["out_proj_w"], w["out_proj_b"] = _lin(seed, in_channels, H, std, "dit", "out_proj")
    for name in ("time_mlp", "delta_time_mlp"):
        w1, b1 = _lin(seed, H, H, std, "dit", name, 1)
        w2, b2 = _lin(seed, H, H, std, "dit", name, 2)
        w[name] = {"w1": w1, "b1": b1, "w2": w2, "b2": b2}
    w["decoder"] = minicpm_weights(dcfg, seed, std, prefix="dit")
    return w


def locdit_f32_view(w):
    f = {k: (bf16_to_f32(v) if k.endswith("_w") else v) for k, v in w.items()
         if k.endswith("_w") or k.endswith("_b")}
    for name in ("time_mlp", "delta_time_mlp"):
        t = w[name]
        f[name] = {"w1": bf16_to_f32(t["w1"]), "b1": t["b1"], "w2": bf16_to_f32(t["w2"]), "b2": t["b2"]}
    f["decoder"] = minicpm_f32_view(w["decoder"])
    return f


# ----------------------------------------------------------------------- VoxCPM2

def voxcpm2_weights(vcfg, seed=0, std=0.02):
    """Random-init ``VoxCpm2Model`` (``src/voxcpm2/model.rs:41-100``): base LM (with the tied
    vocabulary), residual LM, local encoder (MiniCPM-4 + in_proj + special token ~N(0,1),
    ``src/locenc.rs:17-28``), LocDiT, FSQ and the projection layers (biased except
    ``stop_head``)."""
    base = vcfg.lm_config
    H, D = base.hidden_size, vcfg.feat_dim
    ecfg, dcfg = vcfg.encoder_lm_config(), vcfg.dit_lm_config()
    He, Hd, Lq = ecfg.hidden_size, dcfg.hidden_size, vcfg.scalar_quantization_latent_dim
    w = {"base": minicpm_weights(base, seed, std, prefix="base"),
         "residual": minicpm_weights(vcfg.residual_lm_config(), seed, std, prefix="residual"),
         "encoder": minicpm_weights(ecfg, seed, std, prefix="encoder"),
         "dit": locdit_weights(dcfg, in_channels=D, seed=seed, std=std)}
    w["special"] = bf16_to_f32(normal_bf16(seed, (He,), 1.0, 0.0, "vox", "special"))
    for name, out_f, in_f in (("enc_in", He, D), ("enc_to_lm", H, He), ("lm_to_dit", Hd, H), ("res_to_dit", Hd, H),
                              ("fusion", H, 2 * H), ("stop_proj", H, H), ("fsq_in", Lq, H), ("fsq_out", H, Lq)):
        w[name + "_w"], w[name + "_b"] = _lin(seed, out_f, in_f, std, "vox", name)
    w["stop_head_w"] = normal_bf16(seed, (2, H), std, 0.0, "vox", "stop_head")
    return w


def voxcpm2_f32_view(w):
    """f32 view of ``voxcpm2_weights`` for the restatement (``oracle/voxcpm2.py``)."""
    f = {k: (bf16_to_f32(v) if k.endswith("_w") else v) for k, v in w.items()
         if k.endswith("_w") or k.endswith("_b") or k == "special"}
    f["base"] = minicpm_f32_view(w["base"])
    f["residual"] = minicpm_f32_view(w["residual"])
    f["encoder"] = minicpm_f32_view(w["encoder"])
    f["dit"] = locdit_f32_view(w["dit"])
    return f


# ---------------------------------------------------------------------- AudioVAE

def vae_weights(vcfg, seed=0):
    """Random-init AudioVAE decoder (``src/audiovae/decoder.rs:102-147``), bf16 conv
    weights scaled by fan-in so activations stay O(1) through the stack
    (depthwise ``1/sqrt(7)``, pointwise ``0.5/sqrt(C)``, transposed ``1/sqrt(2*C_in)``),
    snake alpha ~N(1, 0.02), biases ~N(0, 0.02), SR scale ~N(1, 0.02) / bias ~N(0, 0.02).
    Returned as bf16 bits for weights and f32 for alpha / bias / SR tables."""
    def wb(shape, std, *t):
        return normal_bf16(seed, shape, std, 0.0, "vae", *t)

    def b(n, *t):
        return bf16_to_f32(normal_bf16(seed, (n,), 0.02, 0.0, "vae", *t, "b"))

    def alpha(n, *t):
        return bf16_to_f32(normal_bf16(seed, (n,), 0.02, 1.0, "vae", *t, "alpha"))

    L, C0 = vcfg.latent_dim, vcfg.decoder_dim
    w = {}
    if vcfg.depthwise:
        w["first_dw_w"], w["first_dw_b"] = wb((L, 1, 7), 7 ** -0.5, "first_dw"), b(L, "first_dw")
        w["first_pw_w"], w["first_pw_b"] = wb((C0, L, 1), L ** -0.5, "first_pw"), b(C0, "first_pw")
    else:
        w["first_pw_w"], w["first_pw_b"] = wb((C0, L, 7), (7 * L) ** -0.5, "first_pw"), b(C0, "first_pw")
    blocks, srs = [], []
    for i, s in enumerate(vcfg.decoder_rates):
        cin, cout = C0 // 2 ** i, C0 // 2 ** (i + 1)
        blk = {"alpha": alpha(cin, i, "snake"),
               "up_w": wb((cin, cout, 2 * s), (2 * cin) ** -0.5, i, "up"),
               "up_b": b(cout, i, "up"), "res": []}
        g = cout if vcfg.depthwise else 1
        for j in range(3):
            blk["res"].append({
                "alpha1": alpha(cout, i, j, 1), "alpha2": alpha(cout, i, j, 2),
                "w1": wb((cout, cout // g, 7), (7 * cout // g) ** -0.5, i, j, "dw"),
                "b1": b(cout, i, j, "dw"),
                "w2": wb((cout, cout, 1), 0.5 * cout ** -0.5, i, j, "pw"),
                "b2": b(cout, i, j, "pw"),
            })
        blocks.append(blk)
        if vcfg.sr_bin_boundaries is not None:
            nb = len(vcfg.sr_bin_boundaries) + 1
            srs.append({"scale": bf16_to_f32(normal_bf16(seed, (nb, cin), 0.02, 1.0, "vae", i, "sr_s")),
                        "bias": bf16_to_f32(normal_bf16(seed, (nb, cin), 0.02, 0.0, "vae", i, "sr_b"))})
    cl = C0 // 2 ** len(vcfg.decoder_rates)
    w["blocks"], w["sr_cond"] = blocks, srs
    w["alpha_out"] = alpha(cl, "out")
    w["last_w"], w["last_b"] = wb((1, cl, 7), 0.5 * (7 * cl) ** -0.5, "last"), b(1, "last")
    return w


def vae_f32_view(w):
    def conv(x):
        return bf16_to_f32(x) if isinstance(x, np.ndarray) and x.dtype == np.uint16 else x
    out = {k: conv(v) for k, v in w.items() if k not in ("blocks", "sr_cond")}
    out["blocks"] = [{k: (conv(v) if k != "res" else [{kk: conv(vv) for kk, vv in r.items()} for r in v])
                      for k, v in blk.items()} for blk in w["blocks"]]
    out["sr_cond"] = w["sr_cond"]
    return out


# ------------------------------------------------------------------------ inputs

def prompt_ids(n, vocab, seed=0):
    """Prompt token ids ~U[0, vocab)."""
    return _rng(seed, "prompt").integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)
