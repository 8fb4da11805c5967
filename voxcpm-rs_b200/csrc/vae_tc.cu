// AudioVAE convolutions on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a:
// the k = 1 pointwise convs (DecoderFirstConv's pw, CausalResidualUnit's conv2; reference
// src/audiovae/decoder.rs:83-89, layers.rs:130-157) and the causal transposed convs of the
// decoder blocks (layers.rs:60-100) as implicit GEMMs over channel-major activations.
//
// Operands.  The weights are the MMA's A operand, bf16 and exact.  The activations are f32;
// a split pass (vae_split_kernel) applies the consumer's per-channel input transform
// (SampleRateConditionLayer scale / bias, Snake1d) and writes them time-major as two bf16
// planes, x = hi + lo (hi = bf16(x), lo = bf16(x - hi)), so that every product is exact in the
// f32 accumulator and the result carries about 2^-16 relative error per term.  Each K step
// issues one MMA with the hi plane and one with the lo plane into the same TMEM accumulator.
//
// Transposed conv with stride s and kernel 2s (the right trim drops the j = T_in tail):
// output sample t = j*s + r of channel m is W[:, m, r]^T x[:, j] + W[:, m, r+s]^T x[:, j-1].
// The s phases are folded into the MMA's M dimension: a 128-row A tile holds cpt = 128 / s
// channels x s phases (row = channel * s + phase, the remaining rows zero), so one CTA
// produces every phase of its channels and, in the epilogue, the s lanes of one channel
// write s consecutive samples.  The j - 1 tap is the same activation tile loaded one row
// earlier (a TMA load may start at row -1: that row reads as zero, the causal left edge).
//
// Pipeline per CTA (one 128-row A tile x 128 time columns): warp 0 lane 0 issues the TMA
// tile loads (SWIZZLE_128B, each into this CTA only) into a ring of shared-memory stages; warp 1 lane 0
// issues tcgen05.mma (kind::f16) and releases each stage with tcgen05.commit; all four warps
// then read the accumulator (tcgen05.ld; warp w owns TMEM lanes 32w..32w+31) and store
// bias (+ residual) + acc.  Every mbarrier wait is bounded; on a timeout the CTA records an
// error, waits for its own copies in flight, frees its TMEM and returns.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"

namespace vx {

namespace {

constexpr int VT_N = 128;        // time columns per tile (MMA N)
constexpr int VT_THREADS = 128;
constexpr int VT_A_BYTES = TC_BM * TC_BK * 2;
constexpr int VT_B_BYTES = VT_N * TC_BK * 2;
constexpr int VT_STAGE = VT_A_BYTES + 2 * VT_B_BYTES;

struct VaeTcArgs {
  int B, T_in, Cin, Cout, s, taps, cpt, kchunks, nstages;
  int row_off;        // rows of history ahead of the chunk in the activation operand (0 or 1)
  const float* bias;  // [Cout]
  const float* R;     // residual [B, Cout, T_out] or null (may alias Y)
  float* Y;           // [B, Cout, T_out]
  int* err;
};

__device__ __forceinline__ float snake_f(float x, float alpha) {
  // x + (alpha + 1e-9)^-1 * sin(alpha * x)^2   (layers.rs:119-122)
  const float inv = 1.0f / (alpha + 1e-9f);
  const float s = sinf(alpha * x);
  return x + inv * (s * s);
}

// X [B, C, T] f32 -> xs [2][B][lead + T][C] bf16 (plane 0: hi, plane 1: lo), after the
// optional SR conditioning (x * scale[c] + bias[c], layers.rs:213-220) and Snake1d (alpha[c]).
// lead = 1 puts the previous chunk's last input frame hist[B, C] in row 0 (streaming decode:
// the transposed conv's j - 1 tap of the chunk's first frame).  Tile of 64 channels x 32
// rows per block, transposed through shared memory.
__global__ void __launch_bounds__(256) vae_split_kernel(const float* __restrict__ X, int B, int C, int T,
                                                        const float* __restrict__ alpha,
                                                        const float* __restrict__ sc, const float* __restrict__ sb,
                                                        uint16_t* __restrict__ xs, const float* __restrict__ hist,
                                                        int lead) {
  __shared__ float tile[64][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 64, b = blockIdx.z;
  const int tid = threadIdx.x;
  const int rows = T + lead;
  {
    const int tt = tid & 31, cr = tid >> 5;  // 8 channel rows per pass
    for (int c = cr; c < 64; c += 8) {
      const int ch = c0 + c, t = t0 + tt;
      float v = 0.f;
      if (ch < C && t < rows) {
        v = t < lead ? hist[(size_t)b * C + ch] : X[((size_t)b * C + ch) * T + t - lead];
        if (sc) v = v * sc[ch] + sb[ch];
        if (alpha) v = snake_f(v, alpha[ch]);
      }
      tile[c][tt] = v;
    }
  }
  __syncthreads();
  // each thread writes 2 channels (one 32-bit word per plane) of one time row
  const int cp = tid & 31, tr = tid >> 5;
  for (int t = tr; t < 32; t += 8) {
    const int tg = t0 + t, ch = c0 + 2 * cp;
    if (tg >= rows || ch >= C) continue;
    const float v0 = tile[2 * cp][t], v1 = tile[2 * cp + 1][t];
    const __nv_bfloat16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
    const __nv_bfloat16 l0 = __float2bfloat16_rn(v0 - __bfloat162float(h0));
    const __nv_bfloat16 l1 = __float2bfloat16_rn(v1 - __bfloat162float(h1));
    const size_t row = ((size_t)b * rows + tg) * C + ch;
    const uint32_t hw = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
    const uint32_t lw = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
    *reinterpret_cast<uint32_t*>(xs + row) = hw;
    *reinterpret_cast<uint32_t*>(xs + (size_t)B * rows * C + row) = lw;
  }
}

__global__ void __launch_bounds__(VT_THREADS, 1)
    vae_tc_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmX,
                       const VaeTcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + a.nstages * VT_STAGE);
  uint64_t* empty = full + a.nstages;
  uint64_t* done = empty + a.nstages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j0 = blockIdx.x * VT_N, mt = blockIdx.y, b = blockIdx.z;
  const int nit = a.taps * a.kchunks, nst = a.nstages;
  constexpr uint32_t kCols = VT_N;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    flags[0] = 0;
    fence_barrier_init();
  }
  if (warp == 0) {  // TMEM allocation (warp-wide, converged)
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: per K step the A tile and the hi / lo activation tiles
    int issued = 0;
    bool aborted = false;
    for (int it = 0; it < nit; ++it) {
      const int s = it % nst;
      if (it >= nst && !mbar_wait(&empty[s], ((it / nst) - 1) & 1, a.err)) {
        atomicExch(&flags[0], 1);
        aborted = true;
        break;
      }
      const int tap = it / a.kchunks, kc = it % a.kchunks;
      unsigned char* st = base + s * VT_STAGE;
      mbar_arrive_expect_tx(&full[s], VT_STAGE);
      tma_load_2d(st, &tmA, tap * a.Cin + kc * TC_BK, mt * TC_BM, &full[s]);
      tma_load_3d(st + VT_A_BYTES, &tmX, kc * TC_BK, j0 + a.row_off - tap, b, &full[s]);
      tma_load_3d(st + VT_A_BYTES + VT_B_BYTES, &tmX, kc * TC_BK, j0 + a.row_off - tap, a.B + b, &full[s]);
      issued = it + 1;
    }
    if (aborted || *reinterpret_cast<volatile int*>(&flags[0])) {
      // no copy may land in this CTA's shared memory after it leaves
      for (int j = issued > nst ? issued - nst : 0; j < issued; ++j) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&full[j % nst], (j / nst) & 1))
          if (clock64() - t0 > kWaitLimitCycles) break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: D += A . X_hi^T, then D += A . X_lo^T, 16 K elements at a time
    const uint32_t idesc = tc_idesc(VT_N);
    for (int it = 0; it < nit; ++it) {
      const int s = it % nst;
      if (!mbar_wait(&full[s], (it / nst) & 1, a.err)) {
        atomicExch(&flags[0], 1);
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(base + s * VT_STAGE);
      const uint32_t sh = sa + VT_A_BYTES, sl = sh + VT_B_BYTES;
#pragma unroll
      for (int kk = 0; kk < TC_BK / 16; ++kk) {
        tc_mma(tmem, sw128_desc(sa + kk * 32), sw128_desc(sh + kk * 32), idesc, (it > 0 || kk > 0) ? 1 : 0);
        tc_mma(tmem, sw128_desc(sa + kk * 32), sw128_desc(sl + kk * 32), idesc, 1);
      }
      tc_commit(&empty[s]);
    }
    tc_commit(done);  // completes once every MMA issued above has finished
  }
  __syncwarp();
  // ---- epilogue: TMEM lane i = A row i of the tile = (channel, phase)
  const bool ok = mbar_wait(done, 0, a.err);
  tc_fence_after();
  if (!ok) atomicExch(&flags[0], 1);
  __syncthreads();
  if (!flags[0]) {
    const int i = warp * 32 + lane;
    const int m = mt * a.cpt + i / a.s, r = i % a.s;
    const bool row_ok = i < a.cpt * a.s && m < a.Cout;
    const size_t T_out = (size_t)a.T_in * a.s;
    const float bm = row_ok ? a.bias[m] : 0.f;
    float* yr = a.Y + ((size_t)b * a.Cout + (row_ok ? m : 0)) * T_out;
    const float* rr = a.R ? a.R + ((size_t)b * a.Cout + (row_ok ? m : 0)) * T_out : nullptr;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    for (int c0 = 0; c0 < VT_N; c0 += 16) {
      float v[16];
      tmem_ld16(trow + c0, v);  // warp-collective: every lane takes part
      if (!row_ok || j0 + c0 >= a.T_in) continue;
      if (a.s == 1 && (a.T_in & 3) == 0 && j0 + c0 + 16 <= a.T_in) {  // rows 16-byte aligned
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const size_t t = (size_t)j0 + c0 + 4 * q;
          float4 o = make_float4(v[4 * q] + bm, v[4 * q + 1] + bm, v[4 * q + 2] + bm, v[4 * q + 3] + bm);
          if (rr) {
            const float4 rv = *reinterpret_cast<const float4*>(rr + t);
            o.x += rv.x;
            o.y += rv.y;
            o.z += rv.z;
            o.w += rv.w;
          }
          *reinterpret_cast<float4*>(yr + t) = o;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int j = j0 + c0 + e;
          if (j >= a.T_in) break;
          const size_t t = (size_t)j * a.s + r;
          float o = v[e] + bm;
          if (rr) o += rr[t];  // CausalResidualUnit: x + conv2(...) (layers.rs:150-156)
          yr[t] = o;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

}  // namespace

cudaError_t vae_tc_configure() {
  return cudaFuncSetAttribute(vae_tc_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

int vae_tc_rows(int cout, int s) {
  const int cpt = TC_BM / s;
  return ((cout + cpt - 1) / cpt) * TC_BM;
}

cudaError_t launch_vae_split(const float* X, int B, int C, int T, const float* alpha, const float* sr_scale,
                             const float* sr_bias, uint16_t* xs, cudaStream_t st, const float* hist) {
  if (C % 2) return cudaErrorInvalidValue;
  const int lead = hist ? 1 : 0;
  dim3 grid((T + lead + 31) / 32, (C + 63) / 64, B);
  count_launch();
  vae_split_kernel<<<grid, 256, 0, st>>>(X, B, C, T, alpha, sr_scale, sr_bias, xs, hist, lead);
  return cudaGetLastError();
}

cudaError_t launch_vae_tc_conv(const uint16_t* xs, int B, int T_in, int Cin, int Cout, int s, const uint16_t* A,
                               const float* bias, const float* R, float* Y, int* err, cudaStream_t st,
                               int row_off) {
  if (Cin % TC_BK || s < 1 || s > TC_BM || T_in <= 0 || B <= 0 || row_off < 0 || row_off > 1)
    return cudaErrorInvalidValue;
  const int taps = s > 1 ? 2 : 1, cpt = TC_BM / s;
  const int a_rows = s > 1 ? vae_tc_rows(Cout, s) : Cout;
  CUtensorMap tmA, tmX;
  cudaError_t e;
  if ((e = tc_map_2d(&tmA, A, a_rows, taps * Cin, TC_BM)) != cudaSuccess) return e;
  if ((e = tc_map_3d(&tmX, xs, 2 * B, T_in + row_off, Cin, VT_N)) != cudaSuccess) return e;
  VaeTcArgs a = {};
  a.B = B;
  a.T_in = T_in;
  a.Cin = Cin;
  a.Cout = Cout;
  a.s = s;
  a.taps = taps;
  a.cpt = cpt;
  a.kchunks = Cin / TC_BK;
  a.nstages = std::max(1, std::min(4, taps * a.kchunks));
  a.row_off = row_off;
  a.bias = bias;
  a.R = R;
  a.Y = Y;
  a.err = err;
  const int smem = 1024 + a.nstages * VT_STAGE + 256;
  dim3 grid((T_in + VT_N - 1) / VT_N, (Cout + cpt - 1) / cpt, B);
  count_launch();
  vae_tc_conv_kernel<<<grid, VT_THREADS, smem, st>>>(tmA, tmX, a);
  return cudaGetLastError();
}

}  // namespace vx
