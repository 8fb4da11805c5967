"""CPU oracle for the voxcpm-rs hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy float32, the arithmetic the reference crate
(mii-nipah/voxcpm-rs, Burn 0.20.1 on the burn-ndarray f32 CPU backend) performs on
the MiniCPM4 decode step, the LocDiT flow-matching step and the AudioVAE decoder.
Every function cites the reference file:line it follows.

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, and only as the checker
or the timed CPU baseline.  The shipped product path (``voxcpm-rs_b200`` and its
CUDA library) never imports, links or calls anything here.

Parity status: **parity unpinned**.  The reference has no unit tests and no
committed golden vectors for this path, its arithmetic lives in third-party crates
that are absent (burn-ndarray 0.20.1, ndarray 0.17.2, matrixmultiply 0.3.10 /
openblas-src 0.10.15, macerator 0.2.10), and it cannot be compiled here (no Rust
toolchain, no crate mirror).  The restatement is therefore checked (a) against
independent torch-CPU implementations of the same operators and (b) against the
golden fixtures under ``tests/golden/`` that this restatement generated
(regression pins), not against outputs of the reference itself.

Semantics assumed where the third-party source is absent:
  * softmax is the max-subtracted form ``exp(x - max) / sum``;
  * argmax breaks ties toward the lowest index;
  * ``round`` (used by the FSQ layer) rounds half away from zero (Rust ``f32::round``);
  * matmul accumulates in f32 (sgemm), summation order unspecified;
  * bf16 checkpoints are upcast to f32 at load, so a bf16-weight path is the f32
    computation on bf16-rounded weights (reference ``src/weights.rs:35-44``).
"""
