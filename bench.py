#!/usr/bin/env python
"""Benchmark of the MiniCPM-4 LM decode workload on B200.

Workload (one "step" = one utterance): 28-layer MiniCPM-4 (hidden 2048, 16 q / 2 kv heads,
head_dim 128, SwiGLU 6144), tied bf16 embedding of 73448 ids, bf16 weights ~N(0, 0.02)
(random init, synthetic), a 64-id prompt ~U[0, 73448), then 256 greedy decode steps over a
static KV cache of capacity 4096, batch 1.

  value   decode tok/s over the 256 greedy steps, device-timed with CUDA events on the
          library stream (weights and prompt resident; the prefill is excluded and reported
          separately), summed over ranks (one independent utterance per GPU).
  e2e     the same tok/s through the public C ABI call vx_lm_greedy with host buffers:
          prompt H2D, prefill, 256 steps, token ids D2H, wall clock around every call.

Multi-GPU: one process per GPU (torchrun), each decodes its own utterance; no collective on
the data path (timing only: barrier + max over ranks).  ``--impl reference`` times the CPU
restatement of the same path on the host cores instead.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, HIDDEN, INTER, NH, NKV, HD, VOCAB = 28, 2048, 6144, 16, 2, 128, 73448
PROMPT, STEPS_PER_UTT, MAX_LEN = 64, 256, 4096
SYN_B = 8  # utterances resident per GPU in the batched-synthesis side figure
WORKLOAD = ("MiniCPM-4 LM greedy decode: 28 layers, hidden 2048, 16/2 heads, head_dim 128, SwiGLU 6144, tied vocab "
            "73448, bf16 weights ~N(0,0.02) (seed 0), 64-id prompt + 256 greedy steps, KV capacity 4096, batch 1 per GPU")
HEADLINE_METRICS = "LM decode tok/s/GPU, audio-s/s at 1/2/4/8 B200; fused-op HBM GB/s vs peak"

# Algorithmic bytes (the roofline basis): bf16 weights of one decoder layer, the tied
# embedding read by the greedy head, and the KV rows read by attention at position p.
LAYER_WEIGHT_BYTES = ((NH + 2 * NKV) * HD * HIDDEN + HIDDEN * NH * HD + 2 * INTER * HIDDEN + HIDDEN * INTER) * 2
EMBED_BYTES = VOCAB * HIDDEN * 2
GATE_UP_BYTES = 2 * INTER * HIDDEN * 2 + HIDDEN * 4 + INTER * 4  # one gate_up GEMV launch


def kv_bytes(pos):
    return LAYERS * 2 * NKV * (pos + 1) * HD * 4


def decode_bytes_per_utt():
    return sum(LAYERS * LAYER_WEIGHT_BYTES + EMBED_BYTES + kv_bytes(p) for p in range(PROMPT, PROMPT + STEPS_PER_UTT))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks sampling
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ model setup
def lm_config():
    from voxcpm_rs_b200 import config
    return config.lm_decode_config(layers=LAYERS, vocab=VOCAB)


def device_weights(seed, device):
    """Random-init bf16 weights ~N(0, 0.02) generated on the device (torch RNG), in the
    checkpoint layout.  Norm weights ~N(1, 0.02)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.bfloat16).view(torch.int16)

    def n(k):
        return (1 + 0.02 * torch.randn(k, generator=g, device=device)).to(torch.bfloat16).float()

    layers = [{"q": w(NH * HD, HIDDEN), "k": w(NKV * HD, HIDDEN), "v": w(NKV * HD, HIDDEN), "o": w(HIDDEN, NH * HD),
               "gate": w(INTER, HIDDEN), "up": w(INTER, HIDDEN), "down": w(HIDDEN, INTER),
               "ln_in": n(HIDDEN), "ln_post": n(HIDDEN)} for _ in range(LAYERS)]
    return {"layers": layers, "norm": n(HIDDEN), "embed": w(VOCAB, HIDDEN)}


def load_device_weights(model, w):
    from voxcpm_rs_b200._lib import check, lib, ptr
    L = lib()
    for i, lw in enumerate(w["layers"]):
        check(L.vx_lm_load_layer(model.h, i, *[ptr(lw[k]) for k in ("q", "k", "v", "o", "gate", "up", "down")],
                                 ptr(lw["ln_in"]), ptr(lw["ln_post"])), model.ctx.h)
    check(L.vx_lm_load_norm(model.h, ptr(w["norm"])), model.ctx.h)
    check(L.vx_lm_load_embed(model.h, ptr(w["embed"])), model.ctx.h)


# ------------------------------------------------------------------ CPU restatement timing
def cpu_threads():
    """All host cores for the CPU arms: torch and the BLAS pool numpy uses (torchrun sets
    OMP_NUM_THREADS=1 in every process, so the pool is set explicitly)."""
    import torch
    from threadpoolctl import threadpool_limits
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    threadpool_limits(limits=n)
    return n


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_rate_1thread(fw, prompt, n_steps):
    """The same greedy decode on one host thread (BLAS pool limited to 1)."""
    from threadpoolctl import threadpool_limits
    with threadpool_limits(limits=1):
        r, _, _ = cpu_decode_rate(fw, prompt, n_steps, warm=1)
    return r


def cpu_decode_rate(fw, prompt, n_steps, warm=1):
    """Time the oracle's greedy decode steps (after its causal prefill) on the host cores.
    Returns (tok/s, steps timed, seconds)."""
    import numpy as np
    from oracle import minicpm4 as om
    cfg = lm_config()
    rope = om.RopeRows(cfg, PROMPT + n_steps + warm + 2)
    cache = om.StaticKvCache(LAYERS, NKV, HD, 1, MAX_LEN)
    y, kvs = om.model_forward(cfg, fw, om.embed(cfg, fw, np.asarray(prompt)[None]), True, rope)
    cache.fill(kvs)
    tok = om.argmax_first(om.linear(y[:, -1], fw["embed"])[0])
    t0 = None
    for s in range(warm + n_steps):
        if s == warm:
            t0 = time.perf_counter()
        pos = cache.step()
        h = om.model_forward_step(cfg, fw, om.embed(cfg, fw, [tok]), pos, cache, rope)
        tok = om.argmax_first(om.linear(h, fw["embed"])[0])
    dt = time.perf_counter() - t0
    return n_steps / dt, n_steps, dt


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    """--impl reference: the CPU restatement of the path (the reference crate itself cannot
    be built: no Rust toolchain) on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import synth
    threads = cpu_threads()
    cfg = lm_config()
    fw = synth.minicpm_f32_view(synth.minicpm_weights(cfg, seed=0))
    prompt = synth.prompt_ids(PROMPT, VOCAB, seed=0)
    per_step = 2  # decode tokens per timed step (bounded sample)
    rates = []
    for i in range(args.warmup + args.steps):
        r, _, _ = cpu_decode_rate(fw, prompt, per_step, warm=1)
        if i >= args.warmup:
            rates.append(r)
    value = statistics.mean(rates)
    line = {"impl": "reference", "metric": "LM decode tok/s", "value": value, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * per_step / value, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (random-init weights, seeded prompt)",
            "config": {"workload": WORKLOAD,
                       "sample": f"{per_step} timed greedy decode steps per step, after a 64-id prefill "
                                 f"and one untimed decode step"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "cpu_model": cpu_model(), "value_1_thread": cpu_rate_1thread(fw, prompt, 1),
                             "sample": f"{per_step} decode steps per step, numpy f32 restatement "
                                       f"(oracle/) with {threads} BLAS threads"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def measure_rmsnorm(ctx, device):
    """RMSNorm + residual op at [512, 2048] f32, eps 1e-6 (x, r ~N(0,1), w ~N(1,0.02), seed 0):
    16 rotating buffer sets (268 MB > L2).  The 16 calls (one per set) are captured once into a
    CUDA graph through the public op, so the timing is the device's and not the interpreter's
    launch rate: 2 warm-up + 64 timed replays = 1024 calls (CUDA events)."""
    import torch
    from voxcpm_rs_b200.minicpm4 import MiniCpmRmsNorm
    g = torch.Generator(device=device)
    g.manual_seed(0)
    sets = [(torch.randn(512, 2048, generator=g, device=device), torch.randn(512, 2048, generator=g, device=device),
             torch.empty(512, 2048, device=device), torch.empty(512, 2048, device=device)) for _ in range(16)]
    norm = MiniCpmRmsNorm(ctx, 1 + 0.02 * torch.randn(2048, generator=g, device=device), 1e-6)
    from voxcpm_rs_b200._lib import check, lib, ptr
    L = lib()

    def call(i, stream):
        x, r, h, y = sets[i % 16]
        check(L.vx_rmsnorm_residual(ctx.h, ptr(x), ptr(r), ptr(norm.weight), 1.0, 1e-6, 512, 2048, ptr(h), ptr(y),
                                    stream), ctx.h)
    side = torch.cuda.Stream(device=device)
    with torch.cuda.stream(side):
        for i in range(16):  # eager warm-up on the capture stream
            call(i, side.cuda_stream)
    side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(16):
            call(i, side.cuda_stream)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(64):
        graph.replay()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000 / (64 * 16)
    nbytes = 16_785_408
    return {"workload": "RMSNorm + residual [512, 2048] f32", "us_per_call": us, "gb_s": nbytes / (us * 1e-6) / 1e9,
            "algorithmic_bytes": nbytes, "timing": "CUDA graph of 16 op calls, 64 replays"}


def measure_layer_step(model, device, peak):
    """One MiniCPM-4 decoder layer, single-token decode at position 1000 (cache filled with
    N(0,1) up to 1000) through the per-kernel layer step (5 kernels + the hidden copy in and
    out): 20 steps captured once in a CUDA graph on the library stream and replayed 5 times
    (device time, CUDA events), and 100 eager calls after 10 warm-up (host launch rate
    included)."""
    import numpy as np
    import torch
    rng = np.random.default_rng(0)
    k = rng.standard_normal((NKV, 1000, HD), dtype=np.float32)
    v = rng.standard_normal((NKV, 1000, HD), dtype=np.float32)
    model.kv_write(0, k, v)
    from voxcpm_rs_b200._lib import check, lib, ptr
    L = lib()
    h = torch.randn(HIDDEN, device=device)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(model.ctx.stream, device=device)
    for _ in range(10):
        check(L.vx_lm_layer_forward_step(model.h, 0, ptr(h), 1000), model.ctx.h)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(100):
        check(L.vx_lm_layer_forward_step(model.h, 0, ptr(h), 1000), model.ctx.h)
    e1.record(stream)
    e1.synchronize()
    eager_us = e0.elapsed_time(e1) * 1000 / 100
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(20):
            check(L.vx_lm_layer_forward_step(model.h, 0, ptr(h), 1000), model.ctx.h)
    with torch.cuda.stream(stream):  # replays go to the current stream: the library's
        graph.replay()
        stream.synchronize()
        e0.record(stream)
        for _ in range(5):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000 / 100
    del graph
    nbytes = LAYER_WEIGHT_BYTES + 2 * NKV * 1001 * HD * 4
    return {"workload": "one decoder layer, decode step at p=1000 (per-kernel step: 5 kernels)", "us_per_step": us,
            "gb_s": nbytes / (us * 1e-6) / 1e9, "frac_of_hbm_peak": nbytes / (us * 1e-6) / 1e9 / peak,
            "algorithmic_bytes": nbytes, "timing": "CUDA graph of 20 steps replayed 5 times (device time)",
            "eager_us_per_step": eager_us}


def measure_cfm(ctx, device, dcfg, dit_w):
    """LocDiT CFM solve (8 layers, hidden 1024, CFG 2.0, 10 Euler steps, B=1) in both modes:
    uniform t (sway 0, zero-star off) and the reference default (sway 1, zero-star on)."""
    import numpy as np
    import torch
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    dit = VoxCpmLocDiTV2(ctx, dcfg, dit_w)
    rng = np.random.default_rng(0)
    mu = torch.from_numpy(rng.standard_normal((1, 2048), dtype=np.float32)).to(device)
    cond = torch.zeros(1, 64, 4, device=device)
    z = torch.from_numpy(rng.standard_normal((1, 64, 4), dtype=np.float32)).to(device)
    out = {"workload": "LocDiT CFM solve, 8 layers, CFG 2.0, 10 Euler steps, 1 patch [64, 4]"}
    for name, sway, zs in (("uniform", 0.0, False), ("sway_zero_star", 1.0, True)):
        for _ in range(3):
            dit.cfm_forward(mu, 10, cond, z, 2.0, sway, zs)
        t0 = time.perf_counter()
        for _ in range(20):
            dit.cfm_forward(mu, 10, cond, z, 2.0, sway, zs)
        dt = (time.perf_counter() - t0) / 20
        out[f"patches_per_s_{name}"] = 1.0 / dt
    # the batched synthesis solves 8 patches at once (16 CFG sequences, 176 decoder rows), which
    # runs the persistent decoder forward
    mu8 = torch.from_numpy(rng.standard_normal((8, 2048), dtype=np.float32)).to(device)
    cond8 = torch.zeros(8, 64, 4, device=device)
    z8 = torch.from_numpy(rng.standard_normal((8, 64, 4), dtype=np.float32)).to(device)
    for _ in range(3):
        dit.cfm_forward(mu8, 10, cond8, z8, 2.0, 1.0, True)
    t0 = time.perf_counter()
    for _ in range(20):
        dit.cfm_forward(mu8, 10, cond8, z8, 2.0, 1.0, True)
    dt = (time.perf_counter() - t0) / 20
    out["batch8_ms_per_solve"] = dt * 1e3
    out["patches_per_s_batch8"] = 8.0 / dt
    dit.close()
    return out




def vae_flops(vcfg, T):
    """Algorithmic FLOPs of one AudioVAE decode of T latent frames: the causal transposed
    convs (2 * C_out * 2 C_in per output sample), the pointwise convs (2 * C^2 per sample, 3
    per block), the first pointwise conv, the depthwise k7 convs and the last k7 conv."""
    f = 2.0 * vcfg.decoder_dim * vcfg.latent_dim * T + 2.0 * 7 * vcfg.latent_dim * T
    t, c = T, vcfg.decoder_dim
    for s in vcfg.decoder_rates:
        co = c // 2
        t *= s
        f += 2.0 * co * 2 * c * t + 3 * (2.0 * co * co * t + 2.0 * 7 * co * t)
        c = co
    return f + 2.0 * 7 * c * t


def measure_vae(ctx, device, rank):
    """AudioVAE decoder of the end-to-end workload (latent 64, decoder_dim 2048, rates
    [2,5,8,8], 16 kHz) on T = 1024 latent frames (one 40.96 s utterance): device time per
    decode (CUDA events on the context stream, 5 calls after 2 warm-up), algorithmic TFLOP/s
    against the measured sustained bf16 peak."""
    import numpy as np
    import torch
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200._lib import check, lib, ptr
    from voxcpm_rs_b200.audiovae import AudioVae
    vcfg = config.vae_config()
    vae = AudioVae(ctx, vcfg, synth.vae_weights(vcfg, seed=rank))
    z = torch.from_numpy(np.random.default_rng(1).standard_normal((1, 64, 1024), dtype=np.float32)).to(device)
    wav = torch.empty(1, 1, 1024 * 640, device=device)
    L = lib()
    for _ in range(2):
        check(L.vx_vae_decode(vae.h, ptr(z), 1, 1024, ptr(wav)), ctx.h)
    stream = torch.cuda.ExternalStream(ctx.stream, device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(5):
        check(L.vx_vae_decode(vae.h, ptr(z), 1, 1024, ptr(wav)), ctx.h)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / 5
    vae.close()
    flops = vae_flops(vcfg, 1024)
    try:
        peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops_sustained"])
        kind = "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    except Exception:
        peak, kind = 1400.0, "fallback"
    tf = flops / (ms * 1e-3) / 1e12
    return {"workload": "AudioVAE decode, latent 64 x 1024 frames -> 655,360 samples (rates 2,5,8,8; channels "
                        "2048 -> 128)", "ms": ms, "algorithmic_gflop": flops / 1e9, "tflops": tf,
            "peak_tflops": peak, "peak_kind": kind, "frac_of_tensor_peak": tf / peak,
            "math": "pointwise and transposed convs on tcgen05 (bf16 weights x bf16 hi/lo activations, f32 TMEM "
                    "accumulators); depthwise k7 convs on CUDA cores"}


def gemv_graph_us(ctx, weights, x, reps):
    """Average device time of one streamed-GEMV launch over ``weights`` (each [N, K] bf16
    bits), measured by replaying a CUDA graph of one launch per weight ``reps`` times between
    CUDA events on the launching stream (no per-call host overhead inside the timed region;
    the first, module-loading launch happens before capture)."""
    import torch
    from voxcpm_rs_b200._lib import check, lib, ptr
    L = lib()
    n, k = weights[0].shape
    ys = [torch.empty(1, n, device=x.device) for _ in weights]

    def launch_all():
        s = torch.cuda.current_stream().cuda_stream
        for w, y in zip(weights, ys):
            check(L.vx_linear_bf16(ctx.h, ptr(w), None, ptr(x), 1, n, k, ptr(y), s), ctx.h)
    launch_all()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch_all()
    graph.replay()
    cur = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(reps):
        graph.replay()
    e1.record(cur)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * len(weights))
    del graph
    return us


def run_kernel_only():
    """Small profiling case for the dominant kernel: the streamed GEMV on gate|up-shaped
    weights (N=12288, K=2048, 50 MB each, 4 distinct matrices = 201 MB > L2).  Launches: 4
    (direct, module load) + 4 (graph capture warm replay) + 4 x 3 (timed replays)."""
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200.minicpm4 import Context
    ctx = Context(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    ws = [(torch.randn(2 * INTER, HIDDEN, generator=g, device="cuda") * 0.02).to(torch.bfloat16).view(torch.int16)
          for _ in range(4)]
    x = torch.randn(1, HIDDEN, device="cuda")
    us = gemv_graph_us(ctx, ws, x, 3)
    print(json.dumps({"kernel": "gemv_bf16_kernel gate|up", "launch_us": us,
                      "achieved_gbs": GATE_UP_BYTES / (us * 1e-6) / 1e9}))
    ctx.close()
    return 0


def run_lm_only(layers=LAYERS):
    """Small profiling case for the decode step: the LM-decode model (28 layers unless
    `layers` says fewer; vocab 73448), two greedy runs of a 64-id prompt + 32 steps.  Per run:
    the prefill launches + first pick, then 32 decode steps (1 persistent launch each, or
    5 * layers + 1 with VX_PERSIST=0)."""
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import Context, MiniCpmModel
    global LAYERS
    LAYERS = layers
    ctx = Context(0)
    model = MiniCpmModel(ctx, lm_config(), None, max_length=MAX_LEN)
    load_device_weights(model, device_weights(1234, "cuda:0"))
    prompt = synth.prompt_ids(PROMPT, VOCAB, seed=0)
    from voxcpm_rs_b200._lib import check, lib
    pf, dc = ctypes.c_float(), ctypes.c_float()
    for _ in range(2):
        t0 = time.perf_counter()
        toks = model.greedy(prompt, 32)
        torch.cuda.synchronize()
        check(lib().vx_lm_last_timing(model.h, ctypes.byref(pf), ctypes.byref(dc)), ctx.h)
        print(json.dumps({"greedy_32_ms": (time.perf_counter() - t0) * 1e3, "prefill_ms": pf.value,
                          "decode_ms_per_token": dc.value / 32, "ids": toks.tolist()[:12]}))
    model.close()
    ctx.close()
    return 0


def phase_trace(model, ctx, pos, layers):
    """Phase trace of one persistent decode step of `model` at position `pos`
    (vx_lm_trace_decode_step): per phase kind, medians over layers 2..L-2 of the time after
    the previous phase was published at which the median CTA saw the dependency met, had its
    input's bytes (before the RMSNorm / attention merge), had its inputs ready, finished its
    last unit and published, and the phase duration (microseconds).  Advances the model's
    position like a decode step."""
    import numpy as np
    from voxcpm_rs_b200._lib import check, lib
    nph = 4 * layers + 1
    n = nph * 4096 * 8
    buf = (ctypes.c_ulonglong * n)()
    grid = ctypes.c_int()
    for _ in range(3):
        check(lib().vx_lm_trace_decode_step(model.h, pos, buf, n, ctypes.byref(grid)), ctx.h)
    G = grid.value
    t = np.frombuffer(buf, dtype=np.uint64)[:nph * G * 8].reshape(nph, G, 8).astype(np.int64)
    tt = np.where(t > 0, (t - t[t > 0].min()) / 1000.0, np.nan)
    pub = [np.nanmax(tt[p, :, 2]) if p < nph - 1 else np.nanmax(tt[p, :, 5]) for p in range(nph)]
    out = {}
    for k, name in enumerate(["qkv_rope", "attention", "o_proj", "mlp", "head"]):
        ps = [nph - 1] if name == "head" else [p for p in range(nph - 1) if p % 4 == k and 2 <= p // 4 < layers - 1]
        rows = []
        for p in ps:
            a = tt[p]
            has = ~np.isnan(a[:, 0])
            prev = pub[p - 1]
            rows.append([pub[p] - prev, np.median(a[has, 1] - prev), np.median(a[has, 5] - prev),
                         np.max(a[has, 5] - prev), np.median(a[has, 2] - prev) if name != "head" else np.nan,
                         int(has.sum()), np.median(a[has, 6] - prev),
                         np.nanmedian(a[has, 7] - prev) if name != "attention" else np.nan])
        r = np.median(np.array(rows, dtype=np.float64), axis=0)
        out[name] = {"duration_us": round(r[0], 2), "dependency_met_us": round(r[6], 2),
                     "input_bytes_in_us": None if name == "attention" else round(r[7], 2),
                     "inputs_ready_us": round(r[1], 2),
                     "last_unit_median_us": round(r[2], 2), "last_unit_max_us": round(r[3], 2),
                     "published_us": None if name == "head" else round(r[4], 2), "ctas": int(r[5])}
    layer_us = [pub[p + 3] - pub[p - 1] for p in range(4, nph - 1, 4) if 2 <= p // 4 < layers - 1]
    return {"phase_trace": out, "position": pos, "grid": G, "layers": layers,
            "layer_us_median": round(float(np.median(layer_us)), 2), "step_us": round(float(np.nanmax(tt)), 1)}


def run_phase_trace(pos=200, layers=LAYERS):
    """--phase-trace: the LM-decode model after a 64-id prompt + 8 greedy steps, traced at `pos`."""
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200.minicpm4 import Context, MiniCpmModel
    global LAYERS
    LAYERS = layers
    ctx = Context(0)
    model = MiniCpmModel(ctx, lm_config(), None, max_length=MAX_LEN)
    load_device_weights(model, device_weights(1234, "cuda:0"))
    model.greedy(synth.prompt_ids(PROMPT, VOCAB, seed=0), 8)
    torch.cuda.synchronize()
    print(json.dumps(phase_trace(model, ctx, pos, layers)))
    model.close()
    ctx.close()
    return 0


def run_vae_only():
    """Small profiling case: the end-to-end workload's AudioVAE decoder on 1024 latent frames,
    two decodes (the first allocates its buffers)."""
    import numpy as np
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.minicpm4 import Context
    ctx = Context(0)
    vcfg = config.vae_config()
    vae = AudioVae(ctx, vcfg, synth.vae_weights(vcfg, seed=0))
    z = torch.from_numpy(np.random.default_rng(1).standard_normal((1, 64, 1024), dtype=np.float32)).cuda()
    for _ in range(2):
        t0 = time.perf_counter()
        vae.decode(z)
        torch.cuda.synchronize()
        print(json.dumps({"vae_decode_ms": (time.perf_counter() - t0) * 1e3}))
    vae.close()
    ctx.close()
    return 0


def run_dit_trace(batch=8):
    """--dit-trace B: timeline of the persistent LocDiT decoder forward inside a CFM solve of B
    patches (2B sequences of 11 rows; forced onto the persistent path): per phase kind, the
    median over layers of the phase time (last CTA through the grid barrier to the next), the
    slowest CTA's work and the barrier wait; GEMM phases also report when the slowest CTA's first
    segment finished its MMAs."""
    import ctypes
    import numpy as np
    import torch
    os.environ["VX_DIT_TRACE"] = "1"
    os.environ["VX_DIT_PERSIST"] = "1"
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200._lib import lib
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import Context
    ctx = Context(0)
    dcfg = config.locdit_config(lm_config())
    dit = VoxCpmLocDiTV2(ctx, dcfg, synth.locdit_weights(dcfg, in_channels=64, seed=0))
    rng = np.random.default_rng(0)
    mu = torch.from_numpy(rng.standard_normal((batch, 2048), dtype=np.float32)).cuda()
    cond = torch.zeros(batch, 64, 4, device="cuda")
    z = torch.from_numpy(rng.standard_normal((batch, 64, 4), dtype=np.float32)).cuda()
    for _ in range(3):
        dit.cfm_forward(mu, 10, cond, z, 2.0, 0.0, False)
    torch.cuda.synchronize()
    n = (8 * dcfg.num_hidden_layers + 1) * 1024 * 4
    buf = (ctypes.c_ulonglong * n)()
    grid, phases = ctypes.c_int(), ctypes.c_int()
    rc = lib().vx_dit_trace(dit.h, buf, n, ctypes.byref(grid), ctypes.byref(phases))
    if rc:
        raise SystemExit(f"vx_dit_trace: {rc}")
    P, G = phases.value, grid.value
    t = np.frombuffer(buf, dtype=np.uint64)[:P * G * 4].reshape(P, G, 4).astype(np.int64)
    t0 = t[:, :, 0][t[:, :, 0] > 0].min()
    t = np.where(t > 0, t - t0, -1) / 1000.0
    start = t[:, :, 0].max(axis=1)
    names = ["RES_A", "QKV", "ATT", "O", "RES_B", "GU", "ACT", "DOWN"]
    res = {}
    for p in range(P - 1):
        d = res.setdefault(names[p % 8], {"phase_us": [], "work_us": [], "first_mma_us": [], "barrier_us": []})
        work = t[p, :, 2]
        wmax = work[work >= 0].max() if (work >= 0).any() else start[p]
        m = t[p, :, 1]
        d["phase_us"].append(start[p + 1] - start[p])
        d["work_us"].append(wmax - start[p])
        d["first_mma_us"].append(m[m >= 0].max() - start[p] if (m >= 0).any() and names[p % 8] in ("QKV", "O", "GU", "DOWN") else 0.0)
        d["barrier_us"].append(start[p + 1] - wmax)
    out = {k: {kk: round(float(np.median(vv)), 2) for kk, vv in v.items()} for k, v in res.items()}
    print(json.dumps({"dit_trace": {"patches": batch, "rows": 2 * batch * 11, "grid": G,
                                    "forward_us": round(float(start[-1]), 1), "phases": out}}))
    dit.close()
    ctx.close()
    return 0


def run_gen_batch(steps=12, trace=False):
    """--gen-batch N: small profiling case of the batched synthesis (8 utterances, 64-id
    prompts, N patches): the LM of the decode workload with 8 rows per greedy step (its decoder
    layers one persistent launch per step), an 8-patch CFM solve per step, the AudioVAE.
    --lm-batch-trace: the same, then the persistent LM step's phase timeline (last step)."""
    import ctypes
    import numpy as np
    import torch
    if trace:
        os.environ["VX_LM_BATCH_TRACE"] = "1"
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200._lib import lib
    from voxcpm_rs_b200.audiovae import AudioVae
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import Context, MiniCpmModel
    from voxcpm_rs_b200.voxcpm import GenerateOptions, VoxCPM
    ctx = Context(0)
    cfg = lm_config()
    lm = MiniCpmModel(ctx, cfg, synth.minicpm_weights(cfg, seed=0), max_batch=SYN_B, max_length=512)
    dcfg = config.locdit_config(cfg)
    dit = VoxCpmLocDiTV2(ctx, dcfg, synth.locdit_weights(dcfg, in_channels=64, seed=0), max_rows=2 * SYN_B)
    vcfg = config.vae_config()
    vae = AudioVae(ctx, vcfg, synth.vae_weights(vcfg, seed=0))
    vox = VoxCPM(ctx, lm, dit, vae)
    prompts = np.stack([synth.prompt_ids(PROMPT, VOCAB, seed=b) for b in range(SYN_B)])
    noise = np.random.default_rng(0).standard_normal((SYN_B, steps, 64, 4), dtype=np.float32)
    t0 = time.perf_counter()
    vox.generate_batch(prompts, GenerateOptions(max_len=steps), noise)
    torch.cuda.synchronize()
    out = {"gen_batch_ms": (time.perf_counter() - t0) * 1e3, "utterances": SYN_B, "patches": steps}
    if trace:
        n = (8 * cfg.num_hidden_layers + 1) * 1024 * 4
        buf = (ctypes.c_ulonglong * n)()
        grid, phases = ctypes.c_int(), ctypes.c_int()
        if lib().vx_lm_batch_trace(lm.h, buf, n, ctypes.byref(grid), ctypes.byref(phases)) == 0:
            P, G = phases.value, grid.value
            t = np.frombuffer(buf, dtype=np.uint64)[:P * G * 4].reshape(P, G, 4).astype(np.int64)
            tz = t[:, :, 0][t[:, :, 0] > 0].min()
            t = np.where(t > 0, t - tz, -1) / 1000.0
            start = t[:, :, 0].max(axis=1)
            names = ["RES_A", "QKV", "ATT", "O", "RES_B", "GU", "ACT", "DOWN"]
            res = {}
            for p in range(P - 1):
                d = res.setdefault(names[p % 8], {"phase_us": [], "work_us": []})
                work = t[p, :, 2]
                wmax = work[work >= 0].max() if (work >= 0).any() else start[p]
                d["phase_us"].append(start[p + 1] - start[p])
                d["work_us"].append(wmax - start[p])
            out["lm_batch_trace"] = {"position": PROMPT + steps - 1, "grid": G, "step_us": round(float(start[-1]), 1),
                                     "phases": {k: {kk: round(float(np.median(vv)), 2) for kk, vv in v.items()}
                                                for k, v in res.items()}}
    print(json.dumps(out))
    ctx.close()
    return 0


def run_cfm_only(batch=1):
    """Small profiling case: the LocDiT CFM solve (8 layers, hidden 1024, CFG 2.0, 10 uniform
    Euler steps, `batch` patches) run twice (the first call captures the solve graph)."""
    import numpy as np
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import config, synth
    from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
    from voxcpm_rs_b200.minicpm4 import Context
    ctx = Context(0)
    dcfg = config.locdit_config(lm_config())
    dit = VoxCpmLocDiTV2(ctx, dcfg, synth.locdit_weights(dcfg, in_channels=64, seed=0))
    rng = np.random.default_rng(0)
    mu = torch.from_numpy(rng.standard_normal((batch, 2048), dtype=np.float32)).cuda()
    cond = torch.zeros(batch, 64, 4, device="cuda")
    z = torch.from_numpy(rng.standard_normal((batch, 64, 4), dtype=np.float32)).cuda()
    for _ in range(2):
        t0 = time.perf_counter()
        dit.cfm_forward(mu, 10, cond, z, 2.0, 0.0, False)
        print(json.dumps({"cfm_solve_ms": (time.perf_counter() - t0) * 1e3, "batch": batch}))
    dit.close()
    ctx.close()
    return 0


def run_rmsnorm_only():
    """Small profiling case: the RMSNorm + residual op at [512, 2048] (16 rotating buffer sets,
    1,024 timed calls in a replayed CUDA graph, as in extras.rmsnorm)."""
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200.minicpm4 import Context
    ctx = Context(0)
    print(json.dumps(measure_rmsnorm(ctx, torch.device("cuda", 0))))
    ctx.close()
    return 0


# ------------------------------------------------------------------ our arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the side workloads (RMSNorm, layer, CFM, synthesis)")
    ap.add_argument("--cpu-steps", type=int, default=6)
    ap.add_argument("--kernel-only", action="store_true",
                    help="profiling case: only the gate|up GEMV over 4 distinct 50 MB weights")
    ap.add_argument("--cfm-only", action="store_true",
                    help="profiling case: two CFM solves of the LocDiT workload (10 Euler steps)")
    ap.add_argument("--cfm-batch", type=int, default=1, help="patches per solve of --cfm-only")
    ap.add_argument("--gen-batch", type=int, default=None, metavar="N",
                    help="profiling case: batched synthesis of 8 utterances, N patches")
    ap.add_argument("--lm-batch-trace", type=int, default=None, metavar="N",
                    help="phase timeline of the persistent 8-row LM step after N batched patches")
    ap.add_argument("--dit-trace", type=int, default=None, metavar="B",
                    help="phase timeline of the persistent LocDiT forward in a CFM solve of B patches")
    ap.add_argument("--vae-only", action="store_true",
                    help="profiling case: two AudioVAE decodes of 1024 latent frames")
    ap.add_argument("--rmsnorm-only", action="store_true",
                    help="profiling case: the RMSNorm + residual op at [512, 2048] (extras.rmsnorm)")
    ap.add_argument("--lm-only", action="store_true",
                    help="profiling case: the LM-decode model, two greedy runs of 32 decode steps each")
    ap.add_argument("--lm-layers", type=int, default=LAYERS,
                    help="decoder layers of the --lm-only case (fewer for an ncu capture)")
    ap.add_argument("--phase-trace", type=int, default=None, metavar="POS",
                    help="print the phase trace of one persistent decode step at position POS")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel_only:
        return run_kernel_only()
    if args.phase_trace is not None:
        return run_phase_trace(args.phase_trace, args.lm_layers)
    if args.lm_only:
        return run_lm_only(args.lm_layers)
    if args.cfm_only:
        return run_cfm_only(args.cfm_batch)
    if args.dit_trace is not None:
        return run_dit_trace(args.dit_trace)
    if args.gen_batch is not None:
        return run_gen_batch(args.gen_batch)
    if args.lm_batch_trace is not None:
        return run_gen_batch(args.lm_batch_trace, trace=True)
    if args.vae_only:
        return run_vae_only()
    if args.rmsnorm_only:
        return run_rmsnorm_only()
    args.warmup = max(3, args.warmup)

    import numpy as np
    import torch
    from __graft_entry__ import load_package
    load_package()
    from voxcpm_rs_b200 import synth
    from voxcpm_rs_b200._lib import check, lib
    from voxcpm_rs_b200.minicpm4 import Context, MiniCpmModel, linear_bf16

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))

    def barrier():
        if dist is not None:
            dist.barrier()

    from voxcpm_rs_b200 import dist as vxd

    def allmax(x):
        return vxd.allmax(x, device=f"cuda:{local}")

    device = f"cuda:{local}"
    ctx = Context(local)
    cfg = lm_config()
    # the same seeded checkpoint-layout weights on every rank and in the CPU arms (host bf16
    # bits, uploaded once); each rank decodes its own prompt
    w = synth.minicpm_weights(cfg, seed=0)
    # batch capacity for the batched-synthesis side figure; the headline decode uses row 0
    model = MiniCpmModel(ctx, cfg, w, max_batch=1 if args.no_extras else SYN_B, max_length=MAX_LEN)
    prompt = synth.prompt_ids(PROMPT, VOCAB, seed=rank)
    prompt_pinned = torch.from_numpy(prompt).pin_memory()
    tokens_pinned = torch.empty(STEPS_PER_UTT + 1, dtype=torch.int32).pin_memory()
    L = lib()
    pf, dc = ctypes.c_float(), ctypes.c_float()

    def one_utterance():
        check(L.vx_lm_greedy(model.h, prompt_pinned.data_ptr(), PROMPT, STEPS_PER_UTT, tokens_pinned.data_ptr()),
              ctx.h)
        check(L.vx_lm_last_timing(model.h, ctypes.byref(pf), ctypes.byref(dc)), ctx.h)
        return pf.value, dc.value

    for _ in range(args.warmup):
        one_utterance()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = L.vx_launch_count()
    stream = torch.cuda.ExternalStream(ctx.stream, device=device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    t0 = time.perf_counter()
    prefill_ms = decode_ms = 0.0
    for _ in range(args.steps):
        a, b = one_utterance()
        prefill_ms += a
        decode_ms += b
    wall = time.perf_counter() - t0
    ev1.record(stream)
    ev1.synchronize()
    total_ms = ev0.elapsed_time(ev1)
    launches = L.vx_launch_count() - launches0
    clk = clocks.stop()
    torch.cuda.synchronize()
    barrier()
    decode_ms_max = allmax(decode_ms)
    total_ms_max = allmax(total_ms)
    wall_max = allmax(wall)
    prefill_ms_max = allmax(prefill_ms)
    tokens_total = STEPS_PER_UTT * args.steps * world
    value = tokens_total / (decode_ms_max / 1000.0)
    e2e = tokens_total / wall_max

    # ---- dominant kernel: the persistent decode step, one launch per token (the per-kernel
    # step when VX_PERSIST=0).  Its launch duration is the device time of the replayed steps
    # (CUDA events on the context stream the graphs run on) divided by the steps.
    persistent = os.environ.get("VX_PERSIST", "1") != "0"
    peak, peak_kind = measured_peaks()
    step_bytes = decode_bytes_per_utt()
    launch_us = decode_ms_max * 1000.0 / (args.steps * STEPS_PER_UTT)
    bytes_per_launch = step_bytes / STEPS_PER_UTT
    achieved = bytes_per_launch / (launch_us * 1e-6) / 1e9
    traffic = None
    prof = os.path.join(ROOT, "profiles", "persist_decode_traffic.json")
    if persistent and os.path.exists(prof):
        try:
            traffic = json.load(open(prof)).get("bytes_per_launch")
        except Exception:
            traffic = None
    # the per-kernel step's dominant kernel, live: the streamed GEMV on the 28 gate|up weights
    # (50 MB each, 1.4 GB rotation > L2), graph-replayed between CUDA events
    gu = [torch.from_numpy(np.concatenate([l["gate"], l["up"]], 0).view(np.int16)).to(device) for l in w["layers"]]
    xs = torch.randn(1, HIDDEN, device=device)
    gemv_us = gemv_graph_us(ctx, gu, xs, 5)
    gemv_gbs = GATE_UP_BYTES / (gemv_us * 1e-6) / 1e9
    del gu

    # ---- the other workloads, measured once per run (side figures, not the headline)
    extras = {}
    if not args.no_extras:
        import numpy as np
        from voxcpm_rs_b200 import config
        from voxcpm_rs_b200.audiovae import AudioVae
        from voxcpm_rs_b200.locdit import VoxCpmLocDiTV2
        from voxcpm_rs_b200.voxcpm import GenerateOptions, VoxCPM
        extras["rmsnorm"] = measure_rmsnorm(ctx, device)
        extras["decoder_layer_step"] = measure_layer_step(model, device, peak)
        if persistent:
            # the same layer step inside the one-launch decode step (config 2's layer, p = 1000):
            # median time from a layer's qkv phase start to its MLP publish, phase trace
            tr = phase_trace(model, ctx, 1000, LAYERS)
            lb = LAYER_WEIGHT_BYTES + 2 * NKV * 1001 * HD * 4
            extras["decoder_layer_step_persistent"] = {
                "workload": "one decoder layer of the persistent decode step at p=1000 (phase trace, median layer)",
                "us_per_layer": tr["layer_us_median"], "gb_s": lb / (tr["layer_us_median"] * 1e-6) / 1e9,
                "frac_of_hbm_peak": lb / (tr["layer_us_median"] * 1e-6) / 1e9 / peak, "algorithmic_bytes": lb,
                "phases_us": {k: v["duration_us"] for k, v in tr["phase_trace"].items()}}
        dcfg = config.locdit_config(cfg)
        dit_w = synth.locdit_weights(dcfg, in_channels=64, seed=rank)
        extras["locdit_cfm"] = measure_cfm(ctx, device, dcfg, dit_w)
        extras["vae"] = measure_vae(ctx, device, rank)
        # end-to-end synthesis: one utterance per GPU (LM 64-id prompt + 256 steps, a CFM solve
        # per step with the reference-default sampler, AudioVAE 16 kHz); weak scaling
        vcfg = config.vae_config()
        vox = VoxCPM(ctx, model, VoxCpmLocDiTV2(ctx, dcfg, dit_w), AudioVae(ctx, vcfg, synth.vae_weights(vcfg, seed=rank)))
        noise = np.random.default_rng(100 + rank).standard_normal((STEPS_PER_UTT, 64, 4), dtype=np.float32)
        vox.generate(prompt, GenerateOptions(max_len=4), noise[:4])
        runs = []
        for _ in range(5):  # one utterance is about a second of wall clock: median of five
            barrier()
            t0 = time.perf_counter()
            wav = vox.generate(prompt, GenerateOptions(max_len=STEPS_PER_UTT), noise)
            runs.append(allmax(time.perf_counter() - t0))
        e2e_s = sorted(runs)[2]
        audio_s = len(wav) / 16000.0
        extras["synthesis"] = {"workload": "end-to-end synthesis, 1 utterance per GPU: LM (64-id prompt, 256 steps) "
                                           "+ CFM solve per step (sway 1, zero-star, CFG 2, 10 steps) + AudioVAE "
                                           "(rates 2,5,8,8; 16 kHz)",
                               "audio_seconds_per_utterance": audio_s, "wall_s": e2e_s, "wall_s_runs": runs,
                               "audio_s_per_s": world * audio_s / e2e_s, "n_gpus": world}
        # the end-to-end synthesis workload: 64 independent utterances partitioned over the ranks
        # (contiguous blocks of 64/N), each rank decoding its block in waves of SYN_B
        # utterances (vx_generate_batch: the LM runs SYN_B rows per step, each patch's CFM solve
        # 2*SYN_B DiT rows); whole-job audio-s/s = 64 x 40.96 s over the slowest rank's wall time
        n_utt = 64

        def work_batch(ids):
            prompts = np.stack([synth.prompt_ids(PROMPT, VOCAB, seed=1000 + u) for u in ids])
            noise = np.stack([np.random.default_rng(2000 + u).standard_normal((STEPS_PER_UTT, 64, 4),
                                                                                 dtype=np.float32) for u in ids])
            wav = vox.generate_batch(prompts, GenerateOptions(max_len=STEPS_PER_UTT), noise)
            return [w.shape[0] for w in wav]
        warm_ids = list(range(SYN_B))
        vox.generate_batch(np.stack([synth.prompt_ids(PROMPT, VOCAB, seed=1000 + u) for u in warm_ids]),
                           GenerateOptions(max_len=4), np.zeros((SYN_B, 4, 64, 4), np.float32))
        # the AudioVAE's work buffers grow to a full wave's latent once, outside the timed runs
        vox.vae.decode(torch.zeros(SYN_B, 64, STEPS_PER_UTT * 4, device=device))
        torch.cuda.synchronize()
        part_runs = []
        for _ in range(3):  # the whole job three times: median wall clock (single waves see rare host stalls)
            barrier()
            t0 = time.perf_counter()
            got = vxd.run_partitioned(list(range(n_utt)), work_batch, batch=SYN_B)
            torch.cuda.synchronize()
            part_runs.append(allmax(time.perf_counter() - t0))
        part_max = sorted(part_runs)[1]
        samples = sum(got.values())
        total_samples = samples
        if dist is not None:
            t = torch.tensor([float(samples)], dtype=torch.float64, device=device)
            dist.all_reduce(t)
            total_samples = float(t.item())
        extras["synthesis_partitioned"] = {
            "workload": f"end-to-end synthesis of {n_utt} utterances partitioned over {world} GPU(s) ({n_utt // world} "
                        f"per GPU, waves of {SYN_B} decoded together): LM 64-id prompt + 256 greedy steps, a CFM solve "
                        "per step (sway 1, zero-star, CFG 2, 10 steps), AudioVAE (rates 2,5,8,8; 16 kHz)",
            "metric": "audio-s/s", "value": total_samples / 16000.0 / part_max, "unit": "audio-s/s",
            "utterances": n_utt, "utterances_per_gpu": n_utt // world, "wave": SYN_B, "wall_s": part_max,
            "wall_s_runs": part_runs,
            "audio_seconds": total_samples / 16000.0, "n_gpus": world, "scaling": "strong (64 utterances in total)",
            "timing": "wall clock around every rank's waves (barrier before, max over ranks); median of 3 runs"}
        vox.dit.close()
        vox.vae.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        fw = synth.minicpm_f32_view(w)
        rate, n, secs = cpu_decode_rate(fw, prompt, args.cpu_steps)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
               "value_1_thread": cpu_rate_1thread(fw, prompt, 2),
               "sample": f"{n} greedy decode steps of the same 28-layer model after a 64-id prefill "
                         f"({secs:.1f} s), numpy f32 restatement (oracle/), {threads} BLAS threads"}
        del fw

    if rank == 0:
        line = {
            "metric": "LM decode tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (bf16 weights)", "data": "synthetic (random-init weights, seeded prompt)",
            "headline_metrics": HEADLINE_METRICS,
            "config": {"workload": WORKLOAD,
                       "global_batch": world, "seq_len": PROMPT + STEPS_PER_UTT, "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (2.94 GB of weights read per decode step)",
                       "value_scope": "256 decode steps per step, device time; prefill excluded (see prefill_ms)"},
            "prefill_ms_per_step": prefill_ms_max / args.steps,
            "decode_ms_per_token": decode_ms_max / (args.steps * STEPS_PER_UTT),
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 4,
                    "d2h_bytes_per_step": (STEPS_PER_UTT + 1) * 4,
                    "scope": "vx_lm_greedy with host buffers: prompt H2D + prefill + 256 steps + ids D2H, wall clock"},
            "roofline": {"bound": "hbm",
                         "kernel": "persist_decode_kernel (whole decode step, one launch per token)" if persistent
                         else "decode step (141 launches per token)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": bytes_per_launch,
                         "launch_us": launch_us,
                         "basis": "28 layers x 94,371,840 B bf16 weights + 300,843,008 B tied embedding + KV rows "
                                  "read at each position, averaged over the 256 steps"},
            "gemv_roofline": {"kernel": "gemv_bf16_kernel (gate|up, N=12288, K=2048), per-kernel step",
                              "achieved": gemv_gbs, "peak": peak, "unit": "GB/s", "frac": gemv_gbs / peak,
                              "launch_us": gemv_us, "algorithmic_bytes_per_launch": GATE_UP_BYTES},
            "gpu_launches": int(launches),
            "clocks": clk,
            "cpu_baseline": cpu,
            "extras": extras,
        }
        print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
