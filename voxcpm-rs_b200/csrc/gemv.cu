// Streamed bf16-weight GEMV for the batch-1 decode step (sm_100a).
//
// Work decomposition: the N output rows are cut into groups of 8 rows.  A CTA owns
// `groups_per_cta` groups (mapped so that RoPE pairs / gate-up pairs land in one CTA) and
// streams them, K chunk by K chunk, through a ring of shared-memory stages with 1-D bulk
// copies (the TMA engine) issued by one producer warp.  Eight consumer warps each take one
// row of a stage and dot it against the input vector, which every CTA RMS-normalises for
// itself in its prologue (8 KB read from L2, no separate norm kernel).  Accumulation is
// f32; each row's total is a warp tree reduction (deterministic).
//
// Weights never change inside a decode step, so the producer starts streaming them before
// the programmatic-dependent-launch wait; only the consumers wait for the previous kernel.
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "gemv.cuh"

namespace vx {

constexpr int GEMV_CWARPS = 8;
constexpr int GEMV_THREADS = (GEMV_CWARPS + 1) * 32;
constexpr int GEMV_ROWS = 8;
constexpr int GEMV_MAX_ROWS = 512;

__device__ __forceinline__ int gemv_group_row(const GemvArgs& a, int vg) {
  if (a.map_mode == MAP_ROPE_PAIRS) {
    const int hg = a.map_param;  // 8-row groups per half head
    const int head = vg / (2 * hg), w = vg % (2 * hg);
    return (head * 2 * hg + (w & 1) * hg + (w >> 1)) * GEMV_ROWS;
  }
  if (a.map_mode == MAP_GATE_UP) {
    const int ig = a.map_param;  // 8-row groups in the gate half
    return ((vg & 1) * ig + (vg >> 1)) * GEMV_ROWS;
  }
  return vg * GEMV_ROWS;
}

__host__ __device__ constexpr int gemv_smem_bytes(int kc, int nst, int K) {
  return nst * GEMV_ROWS * kc * 2 + K * 4 + GEMV_MAX_ROWS * 4 + 64 * 4 + 2 * 8 * 8;
}

template <int EPI>
__device__ void gemv_epilogue(const GemvArgs& a, const float* ys, int g0, int ng, float* red, int* flag);

template <int KC, int NST, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS, 2) gemv_bf16_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint16_t* stages = reinterpret_cast<uint16_t*>(smem_raw);
  float* xs = reinterpret_cast<float*>(smem_raw + NST * GEMV_ROWS * KC * 2);
  float* ys = xs + a.K;
  float* red = ys + GEMV_MAX_ROWS;  // 64 floats of scratch
  int* flag = reinterpret_cast<int*>(red + 60);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 64);
  uint64_t* empty = full + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g0 = blockIdx.x * a.groups_per_cta;
  const int ng = min(a.groups_per_cta, a.groups_total - g0);
  const int nchunks = a.K / KC;
  const int nstage_total = ng * nchunks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], GEMV_CWARPS);
    }
    *flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == GEMV_CWARPS) {
    // ---------------- producer warp: stream weight groups
    if (lane == 0) {
      bool ok = true;
      for (int s = 0; s < nstage_total; ++s) {
        const int slot = s % NST;
        if (s >= NST && !mbar_wait(&empty[slot], ((s / NST) - 1) & 1, a.err)) {
          ok = false;
          break;
        }
        const int g = s / nchunks, c = s % nchunks;
        const int row0 = gemv_group_row(a, g0 + g);
        uint16_t* dst = stages + slot * GEMV_ROWS * KC;
        mbar_arrive_expect_tx(&full[slot], GEMV_ROWS * KC * 2);
        if (nchunks == 1) {
          bulk_g2s(dst, a.W + (size_t)row0 * a.K, GEMV_ROWS * KC * 2, &full[slot]);
        } else {
          for (int r = 0; r < GEMV_ROWS; ++r)
            bulk_g2s(dst + r * KC, a.W + (size_t)(row0 + r) * a.K + (size_t)c * KC, KC * 2, &full[slot]);
        }
        if (s == NST - 1 || (s == nstage_total - 1 && nstage_total < NST)) prefetch_share_l2(a.pf_ptr, a.pf_bytes);
      }
      if (!ok) {  // give copies already in flight time to land before the CTA can exit
        const long long t0 = clock64();
        while (clock64() - t0 < 400000) {
        }
      }
    }
    return;
  }

  // ---------------- consumer warps
  const int tid = threadIdx.x;  // 0..255
  pdl_wait();
  float ss = 0.f;
  for (int k = tid * 4; k < a.K; k += 256 * 4) {
    const float4 v = *reinterpret_cast<const float4*>(a.x + k);
    *reinterpret_cast<float4*>(xs + k) = v;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  if (a.norm_w != nullptr) {
    // MiniCpmRmsNorm::forward (src/minicpm4/mod.rs:62-67): x * (mean(x^2)+eps).sqrt().recip() * w
    ss = group_sum(ss, red, GEMV_CWARPS, 1);
    const float inv = 1.0f / sqrtf(ss / (float)a.K + a.eps);
    for (int k = tid * 4; k < a.K; k += 256 * 4) {
      float4 v = *reinterpret_cast<float4*>(xs + k);
      const float4 w = *reinterpret_cast<const float4*>(a.norm_w + k);
      v.x = (v.x * inv) * w.x;
      v.y = (v.y * inv) * w.y;
      v.z = (v.z * inv) * w.z;
      v.w = (v.w * inv) * w.w;
      *reinterpret_cast<float4*>(xs + k) = v;
    }
  }
  named_sync(1, GEMV_CWARPS * 32);
  if (a.norm_out != nullptr && blockIdx.x == 0)
    for (int k = tid * 4; k < a.K; k += 256 * 4)
      *reinterpret_cast<float4*>(a.norm_out + k) = *reinterpret_cast<const float4*>(xs + k);

  constexpr int NJ = KC / 256;
  float xr[NJ * 8];
  float acc0 = 0.f, acc1 = 0.f;
  bool ok = true;
  for (int s = 0; s < nstage_total; ++s) {
    const int slot = s % NST;
    const int g = s / nchunks, c = s % nchunks;
    if (nchunks > 1 || s == 0) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const float4 v0 = *reinterpret_cast<const float4*>(xs + c * KC + j * 256 + lane * 8);
        const float4 v1 = *reinterpret_cast<const float4*>(xs + c * KC + j * 256 + lane * 8 + 4);
        xr[j * 8 + 0] = v0.x; xr[j * 8 + 1] = v0.y; xr[j * 8 + 2] = v0.z; xr[j * 8 + 3] = v0.w;
        xr[j * 8 + 4] = v1.x; xr[j * 8 + 5] = v1.y; xr[j * 8 + 6] = v1.z; xr[j * 8 + 7] = v1.w;
      }
    }
    if (!mbar_wait(&full[slot], (s / NST) & 1, a.err)) {
      ok = false;
      break;
    }
    const uint4* wr = reinterpret_cast<const uint4*>(stages + slot * GEMV_ROWS * KC + warp * KC);
#pragma unroll
    for (int j = 0; j < NJ; j += 2) {
      acc0 = dot8(wr[j * 32 + lane], &xr[j * 8], acc0);
      if (j + 1 < NJ) acc1 = dot8(wr[(j + 1) * 32 + lane], &xr[(j + 1) * 8], acc1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (c == nchunks - 1) {
      const float t = warp_sum(acc0 + acc1);
      if (lane == 0) ys[g * GEMV_ROWS + warp] = t;
      acc0 = acc1 = 0.f;
    }
  }
  if (!ok && lane == 0) atomicExch(flag, 1);
  named_sync(1, GEMV_CWARPS * 32);
  if (*flag) return;
  gemv_epilogue<EPI>(a, ys, g0, ng, red, flag);
}

// --------------------------------------------------------------------------- epilogues

template <>
__device__ void gemv_epilogue<EPI_STORE>(const GemvArgs& a, const float* ys, int g0, int ng, float*, int*) {
  for (int i = threadIdx.x; i < ng * GEMV_ROWS; i += GEMV_CWARPS * 32) {
    const int row = gemv_group_row(a, g0 + i / GEMV_ROWS) + (i % GEMV_ROWS);
    float v = ys[i];
    if (a.bias) v += a.bias[row];
    // MiniCpmDecoderLayer::add_residual (src/minicpm4/layer.rs:33-38): residual + branch*s
    if (a.residual) v = a.residual[row] + v * a.res_scale;
    a.y[row] = v;
  }
}

template <>
__device__ void gemv_epilogue<EPI_QKV_ROPE>(const GemvArgs& a, const float* ys, int g0, int ng, float*,
                                            int*) {
  // apply_rotary_pos_emb (src/minicpm4/rope.rs:76-95) on q and k; post-RoPE k and raw v go
  // to the cache at position_id (src/minicpm4/attention.rs:119-127).  Angles are formed in
  // f64 exactly as MiniCpmLongRope::new does (rope.rs:38-46) and rounded to f32.
  const int pos = a.pos_ptr ? *a.pos_ptr : a.pos_val;
  const int half = a.hd / 2;
  for (int i = threadIdx.x; i < (ng / 2) * GEMV_ROWS; i += GEMV_CWARPS * 32) {
    const int p = i / GEMV_ROWS, r = i % GEMV_ROWS;
    const int row_a = gemv_group_row(a, g0 + 2 * p) + r;
    const float ya = ys[(2 * p) * GEMV_ROWS + r], yb = ys[(2 * p + 1) * GEMV_ROWS + r];
    const int head = row_a / a.hd, ii = row_a % a.hd;
    float oa = ya, ob = yb;
    if (head < a.nh + a.nkv && a.rope != nullptr) {
      const double f = ((double)pos * a.rope->inv_freq[ii]) / a.rope->ext[ii];
      double sd, cd;
      sincos(f, &sd, &cd);
      const float c = (float)(cd * a.rope->scaling_factor);
      const float sn = (float)(sd * a.rope->scaling_factor);
      oa = __fadd_rn(__fmul_rn(ya, c), __fmul_rn(-yb, sn));
      ob = __fadd_rn(__fmul_rn(yb, c), __fmul_rn(ya, sn));
    }
    if (head < a.nh) {
      a.q_out[head * a.hd + ii] = oa;
      a.q_out[head * a.hd + ii + half] = ob;
    } else if (head < a.nh + a.nkv) {
      float* dst = a.kcache + ((size_t)(head - a.nh) * a.s_max + pos) * a.hd;
      dst[ii] = oa;
      dst[ii + half] = ob;
    } else {
      float* dst = a.vcache + ((size_t)(head - a.nh - a.nkv) * a.s_max + pos) * a.hd;
      dst[ii] = ya;
      dst[ii + half] = yb;
    }
  }
}

template <>
__device__ void gemv_epilogue<EPI_SILU_MUL>(const GemvArgs& a, const float* ys, int g0, int ng, float*, int*) {
  // MiniCpmMlp::forward (src/minicpm4/mlp.rs:31-33): silu_stable(gate) * up
  for (int i = threadIdx.x; i < (ng / 2) * GEMV_ROWS; i += GEMV_CWARPS * 32) {
    const int p = i / GEMV_ROWS, r = i % GEMV_ROWS;
    const int row = gemv_group_row(a, g0 + 2 * p) + r;
    const float g = ys[(2 * p) * GEMV_ROWS + r], u = ys[(2 * p + 1) * GEMV_ROWS + r];
    a.act[row] = silu(g) * u;
  }
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <>
__device__ void gemv_epilogue<EPI_ARGMAX>(const GemvArgs& a, const float* ys, int g0, int ng, float* red,
                                          int* flag) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float bv = -FLT_MAX;
  int bi = INT_MAX;
  for (int i = tid; i < ng * GEMV_ROWS; i += GEMV_CWARPS * 32) {
    const int row = (g0 + i / GEMV_ROWS) * GEMV_ROWS + (i % GEMV_ROWS);
    const float v = ys[i];
    if (a.logits) a.logits[row] = v;
    if (better(v, row, bv, bi)) {
      bv = v;
      bi = row;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  int* redi = reinterpret_cast<int*>(red + 16);
  if (lane == 0) {
    red[warp] = bv;
    redi[warp] = bi;
  }
  named_sync(1, GEMV_CWARPS * 32);
  if (tid == 0) {
    for (int w = 1; w < GEMV_CWARPS; ++w)
      if (better(red[w], redi[w], bv, bi)) {
        bv = red[w];
        bi = redi[w];
      }
    a.partials[blockIdx.x] = make_float2(bv, __int_as_float(bi));
    __threadfence();
    const unsigned prev = atomicAdd(a.counter, 1u);
    *flag = (prev == gridDim.x - 1) ? 2 : 0;
  }
  named_sync(1, GEMV_CWARPS * 32);
  if (*flag != 2) return;
  // last CTA: reduce the per-CTA partials (ties -> lowest index)
  __threadfence();
  bv = -FLT_MAX;
  bi = INT_MAX;
  for (int i = tid; i < (int)gridDim.x; i += GEMV_CWARPS * 32) {
    const float2 p = __ldcg(&a.partials[i]);
    const int pi = __float_as_int(p.y);
    if (better(p.x, pi, bv, bi)) {
      bv = p.x;
      bi = pi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    red[32 + warp] = bv;
    redi[24 + warp] = bi;
  }
  named_sync(1, GEMV_CWARPS * 32);
  if (tid == 0) {
    for (int w = 0; w < GEMV_CWARPS; ++w)
      if (better(red[32 + w], redi[24 + w], bv, bi)) {
        bv = red[32 + w];
        bi = redi[24 + w];
      }
    if (bi < 0 || bi >= a.N) bi = 0;
    const int slot = a.step_ptr ? *a.step_ptr : 0;
    if (a.token_out) a.token_out[slot] = bi;
    if (a.step_ptr) *a.step_ptr = slot + 1;
    if (a.pos_inc) *a.pos_inc += 1;
    *a.counter = 0u;
    redi[0] = bi;
  }
  named_sync(1, GEMV_CWARPS * 32);
  const int tok = redi[0];
  if (a.next_x) {
    // next input = embed(tok) * scale_emb (src/minicpm4/model.rs:87-92, voxcpm2/model.rs:145)
    const uint16_t* e = a.embed + (size_t)tok * a.embed_dim;
    for (int k = tid; k < a.embed_dim; k += GEMV_CWARPS * 32)
      a.next_x[k] = __uint_as_float(((uint32_t)e[k]) << 16) * a.embed_scale;
  }
}

// --------------------------------------------------------------------------- launch

template <int KC, int NST, int EPI>
static cudaError_t launch_one(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
  const int smem = gemv_smem_bytes(KC, NST, a.K);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, gemv_bf16_kernel<KC, NST, EPI>, a);
}

template <int EPI>
static cudaError_t launch_epi(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
  if (a.kc == 2048) {
    if (a.K <= 2048) return launch_one<2048, 3, EPI>(a, grid, st, pdl);
    return launch_one<2048, 2, EPI>(a, grid, st, pdl);
  }
  if (a.kc == 1024) return launch_one<1024, 4, EPI>(a, grid, st, pdl);
  if (a.kc == 512) return launch_one<512, 4, EPI>(a, grid, st, pdl);
  if (a.kc == 256) return launch_one<256, 4, EPI>(a, grid, st, pdl);
  return cudaErrorInvalidValue;
}

template <int KC, int NST>
static cudaError_t configure_kc() {
  const void* fns[] = {(const void*)gemv_bf16_kernel<KC, NST, EPI_STORE>,
                       (const void*)gemv_bf16_kernel<KC, NST, EPI_QKV_ROPE>,
                       (const void*)gemv_bf16_kernel<KC, NST, EPI_SILU_MUL>,
                       (const void*)gemv_bf16_kernel<KC, NST, EPI_ARGMAX>};
  for (const void* f : fns) {
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Raise the dynamic shared-memory limit of every GEMV instantiation on the current device.
// Called once per context, before any launch or graph capture.
cudaError_t gemv_configure() {
  cudaError_t e;
  if ((e = configure_kc<2048, 3>()) != cudaSuccess) return e;
  if ((e = configure_kc<2048, 2>()) != cudaSuccess) return e;
  if ((e = configure_kc<1024, 4>()) != cudaSuccess) return e;
  if ((e = configure_kc<512, 4>()) != cudaSuccess) return e;
  return configure_kc<256, 4>();
}

int gemv_pick_kc(int K) {
  for (int kc : {2048, 1024, 512, 256})
    if (K % kc == 0) return kc;
  return 0;
}

cudaError_t launch_gemv(GemvArgs a, int epi, cudaStream_t st, bool pdl, int* err) {
  a.err = err;
  if (a.kc == 0) a.kc = gemv_pick_kc(a.K);
  if (a.kc == 0 || a.N % GEMV_ROWS != 0) return cudaErrorInvalidValue;
  a.groups_total = a.N / GEMV_ROWS;
  if (a.groups_per_cta <= 0) a.groups_per_cta = 1;
  if (a.groups_per_cta * GEMV_ROWS > GEMV_MAX_ROWS) return cudaErrorInvalidValue;
  const int grid = (a.groups_total + a.groups_per_cta - 1) / a.groups_per_cta;
  switch (epi) {
    case EPI_STORE: return launch_epi<EPI_STORE>(a, grid, st, pdl);
    case EPI_QKV_ROPE: return launch_epi<EPI_QKV_ROPE>(a, grid, st, pdl);
    case EPI_SILU_MUL: return launch_epi<EPI_SILU_MUL>(a, grid, st, pdl);
    case EPI_ARGMAX: return launch_epi<EPI_ARGMAX>(a, grid, st, pdl);
  }
  return cudaErrorInvalidValue;
}

int gemv_grid(const GemvArgs& a) {
  const int gt = a.N / GEMV_ROWS;
  return (gt + a.groups_per_cta - 1) / a.groups_per_cta;
}

}  // namespace vx
