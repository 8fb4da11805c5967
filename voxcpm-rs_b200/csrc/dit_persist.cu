// Persistent forward of a MiniCPM-4 stack over a few token rows on the tensor cores (sm_100a),
// one cooperative launch for all layers, in two attention modes:
//   DP_ATT_SEQ     the LocDiT decoder of every CFM Euler step: non-causal attention within
//                  each sequence of S <= 16 rows (reference MiniCpmModel::forward with
//                  is_causal = false, src/minicpm4/model.rs:43-62, as VoxCpmLocDiTV2::
//                  forward_cached runs it, src/locdit/local_dit.rs:138-159);
//   DP_ATT_DECODE  a batched greedy step: one new row per sequence at the device position,
//                  attending to the static KV cache after writing its k, v there (forward_step,
//                  model.rs:64-84, attention.rs:91-154, cache.rs:47-58).
// Per layer
//
//   RES_A   x = x1 + s * down (layer 0: the input rows); x_n = RMSNorm(x)   -> split operand
//   QKV     qkv = W_qkv x_n                                                  (tcgen05 GEMM)
//   ATT     LongRoPE on q, k; softmax(q k^T / sqrt(d)) v (GQA)               -> split operand
//   O       o = W_o attn                                                     (tcgen05 GEMM)
//   RES_B   x1 = x + s * o; x1_n = RMSNorm(x1)                               -> split operand
//   GU      [g | u] = W_gu x1_n                                              (tcgen05 GEMM)
//   ACT     a = silu(g) * u                                                  -> split operand
//   DOWN    down = W_d a                                                     (tcgen05 GEMM)
//
// and a final phase writes RMSNorm(x1 + s * down) (layer.rs:57-73, mlp.rs:28-34,
// attention.rs:55-88, mod.rs:54-68).  Phases are separated by a grid barrier (release /
// acquire counters; all CTAs are resident).
//
// GEMM phases: the weights are the A operand (units of UM = 128 or 256 rows, one UM x 64 TMA
// box per K chunk, SWIZZLE_128B, into this CTA only); the activations are the B operand: the row
// phase before wrote them as two bf16 planes x = hi + lo ([2][Rpad][K], token-major), both
// fetched by one 3-D box, so each K chunk is 2 UM / 128 MMAs (per 128-row tile: hi, lo) into
// UM / 128 f32 TMEM accumulators of Rpad columns.  256-row units (stacks of <= 64 rows) halve
// the copies per byte of weights: the TMA engine's per-SM copy rate, not the bytes, bounds
// these phases at few activation rows.  A phase's (unit, K chunk) pairs are dealt to its CTAs
// in contiguous runs, so a unit's K range may be split over CTAs: each run inside one unit (a
// segment) stores its f32 partial tile into its own slot of the partial buffer with plain
// stores, and the phase that consumes the GEMM sums a unit's slots in slot order.  No atomics:
// the sum, and so the forward, does not depend on the order in which CTAs finish
// (deterministic; the decode attention's split merge is in split order too).
//
// Warps: 4 issues the TMA loads, 5 the MMAs, 0-3 read TMEM; the row phases run on the other
// eleven warps (RES on eight of them): their partial sums are L2 reads, whose rate grows with
// the loads in flight per SM, and the producer warp meanwhile streams the next GEMM phase's
// first weight tiles into the ring.  Every wait is bounded; a timeout records an error and the
// CTA stops cleanly (in-flight copies landed, TMEM freed).
#include <cuda_bf16.h>

#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "runtime.cuh"
#include "dit_persist.cuh"
#include "tc_common.cuh"

namespace vx {

namespace {

constexpr int DP_WARPS = 12;
constexpr int DP_THREADS = DP_WARPS * 32;
constexpr int DP_EPI_THREADS = 128;  // warps 0-3: GEMM epilogue (TMEM lanes 0-127)
constexpr int DP_ROW_THREADS = DP_THREADS - 32;  // row phases: every warp but the producer's (warp 4)
constexpr int DP_RES_THREADS = 256;  // RES rows: the first 8 row warps
constexpr int DP_UM_MAX = 2 * TC_BM;  // weight rows per unit: one or two 128-row MMA tiles (a.um)
constexpr int DP_SMAX = 16;          // tokens per sequence
constexpr int DP_QS = 68;            // shared-memory row stride of q, k, v (floats; float4 aligned)
constexpr int DP_SEGTAB_MAX = 2048;  // ints of segment tables held in shared memory
constexpr int DP_HPU = 2;            // most query heads per attention unit
constexpr int DP_ATT_FLOATS =
    (DP_HPU + 2) * DP_SMAX * DP_QS + DP_HPU * (DP_SMAX * DP_SMAX + DP_SMAX) + 2 * DP_SMAX * 32;  // + cos / sin
// decode attention scratch: q [nq][d], k, v [d], cos / sin [d/2] (nq <= 12 warps, d = 128);
// then two buffers of a 32-position K tile and V tile
constexpr int DP_DEC_NQ = 12, DP_DEC_D = 128, DP_DEC_TILE = 32;
constexpr int DP_DEC_SPLITS = 16;      // most CTAs sharing one (sequence, KV head)'s cache walk
constexpr int DP_DEC_TILE_OFF = 2048;  // floats; >= the scratch above, a multiple of 4
constexpr int DP_DEC_FLOATS = DP_DEC_TILE_OFF + 2 * 2 * DP_DEC_TILE * DP_DEC_D;
static_assert(DP_DEC_NQ * DP_DEC_D + 3 * DP_DEC_D <= DP_DEC_TILE_OFF, "decode scratch");
__host__ __device__ constexpr int dp_att_floats(int mode) { return mode == DP_ATT_DECODE ? DP_DEC_FLOATS : DP_ATT_FLOATS; }
enum { PH_RES_A, PH_QKV, PH_ATT, PH_O, PH_RES_B, PH_GU, PH_ACT, PH_DOWN, PH_N };

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Sm {
  unsigned char* stages;  // [nst][A 16 KB | B hi Rpad*128 | B lo Rpad*128]
  float* att;             // attention scratch: q, k, v [16][DP_QS], scores [16][16], 1/sum [16]
  float* red;             // [32] block reductions
  uint64_t* full;
  uint64_t* empty;
  uint64_t* seg_done;
  uint64_t* acc_free;
  uint64_t* fin;          // the MMA thread's last commit before TMEM is freed
  uint64_t* att_bar;      // [2] decode attention: K / V tile copies
  uint32_t* tmem_slot;
  volatile int* flags;    // [0] abort
  int* segtab;            // copy of the segment tables
};

// Named barriers: 1 = warps 0-3 (epilogue), 2 = the whole CTA, 3 = warps 0-7 (RES rows); every
// lane of a warp reaches them together (__syncwarp first: a lane may come from a longer run of
// a per-thread loop).

// A thread's rank among the row-phase threads: warps 0-3 and 5-11.  Warp 4 (the TMA producer)
// sits the row phases out, so its prefetch of the next GEMM phase's weight tiles (about half a
// microsecond per copy) never holds up their barriers; -1 there.
__device__ __forceinline__ int row_rank() {
  const int w = threadIdx.x >> 5;
  return w == 4 ? -1 : (w < 4 ? (int)threadIdx.x : (int)threadIdx.x - 32);
}
__device__ __forceinline__ void row_sync() {
  __syncwarp();
  named_sync(4, DP_ROW_THREADS);
}
// Barrier 4 that ORs a per-thread flag (a uniform decision over the row threads).
__device__ __forceinline__ bool row_or(bool v) {
  int r;
  __syncwarp();
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 4, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v), "r"(DP_ROW_THREADS)
      : "memory");
  return r != 0;
}

// Barrier 1 that ORs a per-thread flag, so every epilogue thread takes the same decision.
__device__ __forceinline__ bool epi_or(bool v) {
  int r;
  __syncwarp();
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v), "r"(DP_EPI_THREADS)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void res_sync() {
  __syncwarp();
  named_sync(3, DP_RES_THREADS);
}
__device__ __forceinline__ void cta_sync() {
  __syncwarp();
  named_sync(2, DP_THREADS);
}
// Barrier 2 that ORs a per-thread flag (a uniform decision over the whole CTA).
__device__ __forceinline__ bool cta_or(bool v) {
  int r;
  __syncwarp();
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 2, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v), "r"(DP_THREADS)
      : "memory");
  return r != 0;
}

// Grid barrier: thread 0 waits (bounded) for `target` arrivals on cnt, then the CTA syncs.
__device__ bool grid_wait(const DitPersistArgs& a, const unsigned* cnt, unsigned target, const Sm& sm) {
  if (threadIdx.x == 0) {
    bool bad = sm.flags[0] != 0;
    if (!bad && ld_acquire(cnt) < target) {
      const long long t0 = clock64();
      int n = 0;
      while (ld_acquire(cnt) < target) {
        if ((++n & 63) == 0) {
          if (*reinterpret_cast<volatile int*>(a.err) != 0 || clock64() - t0 > kWaitLimitCycles) {
            record_error(a.err, VX_DEVICE_ERR_TIMEOUT);
            bad = true;
            break;
          }
        }
      }
    }
    if (bad) sm.flags[0] = 1;
    // data written through the generic proxy by other CTAs is read by this CTA's TMA loads
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  cta_sync();
  return sm.flags[0] == 0;
}

__device__ void grid_arrive(unsigned* cnt) {
  cta_sync();
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
  }
}

// ------------------------------------------------------------------ partial sums

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// The partial slots of one GEMM output: slot k of (row r, channels c..c+3) is b[k * stride].
struct PRange {
  const float* b;
  int n;
};

struct Parts {
  const float* p;        // [segments][Rpad][128]
  const int* seg_off;    // [tiles + 1], in shared memory (plain loads: not the global-only __ldg)
  size_t stride;         // Rpad * um
  int ush;               // log2 of the weight rows per unit (7 or 8)
  __device__ PRange at(int r, int c) const {
    const int t = c >> ush, s0 = seg_off[t];
    return {p + (size_t)s0 * stride + ((size_t)r << ush) + (c & ((1 << ush) - 1)), seg_off[t + 1] - s0};
  }
};

// o[k] = sum over the slots of x[k] in slot order; NR ranges x BT slots of loads in flight.
template <int NR, int BT>
__device__ __forceinline__ void psum(const PRange* x, size_t stride, float4* o) {
  int nmax = 0;
#pragma unroll
  for (int k = 0; k < NR; ++k) {
    o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    nmax = max(nmax, x[k].n);
  }
  for (int s = 0; s < nmax; s += BT) {
    float4 v[NR][BT];
#pragma unroll
    for (int k = 0; k < NR; ++k)
#pragma unroll
      for (int i = 0; i < BT; ++i)
        v[k][i] = s + i < x[k].n ? ldcg4(x[k].b + (size_t)(s + i) * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < NR; ++k)
#pragma unroll
      for (int i = 0; i < BT; ++i)
        if (s + i < x[k].n) o[k] = add4(o[k], v[k][i]);
  }
}

__device__ __forceinline__ Parts parts_of(const DitPersistArgs& a, const Sm& sm, int kind) {
  return Parts{a.part, sm.segtab + a.tab_off[kind], (size_t)a.Rpad * a.um, a.um == DP_UM_MAX ? 8 : 7};
}

// Optional timeline: %globaltimer into trace [phase][CTA][4] (0: phase start, 1: first segment's
// MMAs done, 2: this CTA's work done).
__device__ __forceinline__ void trace_at(const DitPersistArgs& a, int ph, int slot) {
  if (a.trace) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.trace[((size_t)ph * gridDim.x + blockIdx.x) * 4 + slot] = t;
  }
}

// ------------------------------------------------------------------ row phases

// Per-row sums over the DP_RES_THREADS RES threads (fixed order).
__device__ void res_sum2(float& v0, float& v1, float* red) {
  v0 = warp_sum(v0);
  v1 = warp_sum(v1);
  const int w = row_rank() >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[w] = v0;
    red[8 + w] = v1;
  }
  res_sync();
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < DP_RES_THREADS / 32; ++i) {
    s0 += red[i];
    s1 += red[8 + i];
  }
  res_sync();
  v0 = s0;
  v1 = s1;
}

__device__ __forceinline__ void split1(float v, uint16_t& h, uint16_t& l) {
  const __nv_bfloat16 bh = __float2bfloat16_rn(v);
  h = __bfloat16_as_ushort(bh);
  l = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(bh)));
}

__device__ __forceinline__ void store_split(uint16_t* xs, size_t plane, size_t idx, float v) {
  uint16_t h, l;
  split1(v, h, l);
  xs[idx] = h;
  xs[plane + idx] = l;
}

// Four consecutive elements (idx % 4 == 0) into the split operand.
__device__ __forceinline__ void store_split4(uint16_t* xs, size_t plane, size_t idx, float4 v) {
  uint16_t h[4], l[4];
  split1(v.x, h[0], l[0]);
  split1(v.y, h[1], l[1]);
  split1(v.z, h[2], l[2]);
  split1(v.w, h[3], l[3]);
  *reinterpret_cast<uint2*>(xs + idx) = make_uint2(h[0] | ((unsigned)h[1] << 16), h[2] | ((unsigned)h[3] << 16));
  *reinterpret_cast<uint2*>(xs + plane + idx) =
      make_uint2(l[0] | ((unsigned)l[1] << 16), l[2] | ((unsigned)l[3] << 16));
}

// RES rows: v = base[r] + s * (the GEMM output, summed from its partials; none for the input
// rows), optionally stored to `store`; then RMSNorm(v) * w into the split operand (K = H), or
// into final_out.  Run by the DP_RES_THREADS threads.  NG = 1 (H <= 1024): thread t holds
// channels 4t.. of two rows at a time (rows r and r + grid); NG = 2 (H <= 2048): channels
// 4t.. and 1024 + 4t.. of one row.  Either way two partial ranges are summed together.
template <int NG>
__device__ void res_norm_rows(const DitPersistArgs& a, const float* base, const Parts* q, float* store,
                              const float* w, uint16_t* xs, float* final_out, const Sm& sm) {
  constexpr int NR = NG == 1 ? 2 : 1;  // rows per pass
  const int H = a.H, G = gridDim.x;
  const size_t plane = (size_t)a.Rpad * H;
  int cc[2];
  float4 g[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    cc[k] = row_rank() * 4 + (NG == 2 ? k * 4 * DP_RES_THREADS : 0);
    g[k] = cc[k] < H ? __ldg(reinterpret_cast<const float4*>(w + cc[k])) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int r0 = blockIdx.x; r0 < a.R; r0 += NR * G) {
    int rr[2];
    bool live[2];
    float4 v[2];  // range i: row rr[i], channels cc[i]
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rr[i] = NG == 1 ? r0 + i * G : r0;
      live[i] = rr[i] < a.R && cc[i] < H;
      v[i] = live[i] ? ldcg4(base + (size_t)rr[i] * H + cc[i]) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (q) {
      PRange x[2] = {live[0] ? q->at(rr[0], cc[0]) : PRange{nullptr, 0}, live[1] ? q->at(rr[1], cc[1]) : PRange{nullptr, 0}};
      float4 o[2];
      psum<2, 4>(x, q->stride, o);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        v[i].x += o[i].x * a.res_scale;
        v[i].y += o[i].y * a.res_scale;
        v[i].z += o[i].z * a.res_scale;
        v[i].w += o[i].w * a.res_scale;
      }
    }
    float ss[2] = {0.f, 0.f};  // per row (NG = 1) or both halves of one row (NG = 2, summed below)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (!live[i]) continue;
      if (store) *reinterpret_cast<float4*>(store + (size_t)rr[i] * H + cc[i]) = v[i];
      float t = ss[i];
      t = fmaf(v[i].x, v[i].x, t);
      t = fmaf(v[i].y, v[i].y, t);
      t = fmaf(v[i].z, v[i].z, t);
      t = fmaf(v[i].w, v[i].w, t);
      ss[i] = t;
    }
    if (NG == 2) {
      ss[0] += ss[1];
      ss[1] = 0.f;
    }
    res_sum2(ss[0], ss[1], sm.red);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (!live[i]) continue;
      const float inv = 1.0f / sqrtf((NG == 1 ? ss[i] : ss[0]) / (float)H + a.eps);
      const float4 gw = g[i];
      const float4 y = make_float4((v[i].x * inv) * gw.x, (v[i].y * inv) * gw.y, (v[i].z * inv) * gw.z,
                                   (v[i].w * inv) * gw.w);
      const size_t at = (size_t)rr[i] * H + cc[i];
      if (final_out)
        *reinterpret_cast<float4*>(final_out + at) = y;
      else
        store_split4(xs, plane, at, y);
    }
  }
}

__device__ void res_rows(const DitPersistArgs& a, const float* base, const Parts* q, float* store, const float* w,
                         uint16_t* xs, float* final_out, const Sm& sm) {
  if (a.H <= 4 * DP_RES_THREADS)
    res_norm_rows<1>(a, base, q, store, w, xs, final_out, sm);
  else
    res_norm_rows<2>(a, base, q, store, w, xs, final_out, sm);
}

// LongRoPE cos / sin (x scaling factor) at positions 0..S-1 (rope.rs:76-95), f64 as the
// reference computes them, into rope_tab [2][16][64] (grid-stride over the RES threads).
__device__ void rope_table(const DitPersistArgs& a) {
  const int half = a.d / 2;
  for (int i = blockIdx.x * DP_RES_THREADS + row_rank(); i < a.S * half; i += gridDim.x * DP_RES_THREADS) {
    const int p = i / half, j = i % half;
    const double f = ((double)p * a.rope->inv_freq[j]) / a.rope->ext[j];
    double sd, cd;
    sincos(f, &sd, &cd);
    a.rope_tab[p * 64 + j] = (float)(cd * a.rope->scaling_factor);
    a.rope_tab[DP_SMAX * 64 + p * 64 + j] = (float)(sd * a.rope->scaling_factor);
  }
}

// Attention for one sequence n and hpu query heads h0.. of one KV head g (GQA, no mask) over the
// S keys of sequence n: q, k, v summed from the QKV partials, LongRoPE on q and k, softmax with
// the max subtracted (attention.rs:186-191); output into the split operand (K = nh * d).  Run
// by all DP_THREADS threads of the CTA.
__device__ void att_unit(const DitPersistArgs& a, const Parts& q, int n, int h0, int hpu, int ph, const Sm& sm) {
  const int S = a.S, d = a.d, half = d / 2, d4 = d / 4, g = h0 / (a.nh / a.nkv);
  float* qs = sm.att;                               // [hpu][16][DP_QS]
  float* ks = qs + hpu * DP_SMAX * DP_QS;           // [16][DP_QS]
  float* vs = ks + DP_SMAX * DP_QS;                 // [16][DP_QS]
  float* sc = sm.att + (DP_HPU + 2) * DP_SMAX * DP_QS;  // [hpu][16][16]
  float* inv = sc + DP_HPU * DP_SMAX * DP_SMAX;     // [hpu][16]
  float* rt = inv + DP_HPU * DP_SMAX;               // [2][16][32] cos, sin of positions 0..S-1
  const int tid = row_rank(), rows = (hpu + 2) * S, cells = rows * d4;
  // the rope values are loaded while the partial sums below are in flight
  static_assert(2 * DP_ROW_THREADS >= DP_SMAX * 32, "rope values per thread");
  float rc[2] = {0.f, 0.f}, rs[2] = {0.f, 0.f};
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = tid + k * DP_ROW_THREADS;
    if (a.rope && i < S * half) {
      rc[k] = __ldcg(a.rope_tab + (i / half) * 64 + i % half);
      rs[k] = __ldcg(a.rope_tab + DP_SMAX * 64 + (i / half) * 64 + i % half);
    }
  }
  // q, k, v rows: two float4 cells per thread, eight slots each in flight
  for (int i0 = tid; i0 < cells; i0 += 2 * DP_ROW_THREADS) {
    PRange x[2];
    int dst[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = i0 + k * DP_ROW_THREADS;
      x[k] = PRange{nullptr, 0};
      dst[k] = -1;
      if (i < cells) {
        const int which = i / (S * d4), rem = i % (S * d4), s = rem / d4, e = (rem % d4) * 4;
        const int cb = which < hpu ? (h0 + which) * d : which == hpu ? (a.nh + g) * d : (a.nh + a.nkv + g) * d;
        x[k] = q.at(n * S + s, cb + e);
        dst[k] = (which * DP_SMAX + s) * DP_QS + e;
      }
    }
    float4 o[2];
    psum<2, 8>(x, q.stride, o);
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (dst[k] >= 0) *reinterpret_cast<float4*>(qs + dst[k]) = o[k];
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = tid + k * DP_ROW_THREADS;
    if (a.rope && i < S * half) {
      rt[(i / half) * 32 + i % half] = rc[k];
      rt[DP_SMAX * 32 + (i / half) * 32 + i % half] = rs[k];
    }
  }
  row_sync();
  if (threadIdx.x == 0 && n * (a.nh / hpu) + h0 / hpu == (int)blockIdx.x) trace_at(a, ph, 1);
  if (a.rope) {  // rows 0..hpu S-1 are q, rows hpu S.. are k (one rotation pair per thread)
    for (int i = tid; i < (hpu + 1) * S * half; i += DP_ROW_THREADS) {
      const int row = i / half, j = i % half, s = row % S;
      float* v = qs + ((row / S) * DP_SMAX + s) * DP_QS;
      const float c = rt[s * 32 + j], si = rt[DP_SMAX * 32 + s * 32 + j];
      const float x1 = v[j], x2 = v[j + half];
      v[j] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, si));
      v[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, si));
    }
    row_sync();
  }
  if (threadIdx.x == 0 && n * (a.nh / hpu) + h0 / hpu == (int)blockIdx.x) trace_at(a, ph, 3);
  for (int i = tid; i < hpu * S * S; i += DP_ROW_THREADS) {
    const int hh = i / (S * S), s = (i / S) % S, t = i % S;
    const float4* qr = reinterpret_cast<const float4*>(qs + (hh * DP_SMAX + s) * DP_QS);
    const float4* kr = reinterpret_cast<const float4*>(ks + t * DP_QS);
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int e = 0; e < d4; ++e) {
      const float4 x = qr[e], y = kr[e];
      a0 = fmaf(x.x, y.x, a0);
      a1 = fmaf(x.y, y.y, a1);
      a2 = fmaf(x.z, y.z, a2);
      a3 = fmaf(x.w, y.w, a3);
    }
    sc[(hh * DP_SMAX + s) * DP_SMAX + t] = ((a0 + a1) + (a2 + a3)) * a.attn_scale;
  }
  row_sync();
  if (tid < hpu * S) {
    float* row = sc + ((tid / S) * DP_SMAX + tid % S) * DP_SMAX;
    float mx = -FLT_MAX;
    for (int t = 0; t < S; ++t) mx = fmaxf(mx, row[t]);
    float den = 0.f;
    for (int t = 0; t < S; ++t) {
      const float e = expf(row[t] - mx);
      row[t] = e;
      den += e;
    }
    inv[(tid / S) * DP_SMAX + tid % S] = 1.0f / den;
  }
  row_sync();
  const size_t plane = (size_t)a.Rpad * a.nh * d;
  for (int i = tid; i < hpu * S * d4; i += DP_ROW_THREADS) {
    const int hh = i / (S * d4), s = (i / d4) % S, e = (i % d4) * 4;
    const float* p = sc + (hh * DP_SMAX + s) * DP_SMAX;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < S; ++t) {
      const float pt = p[t];
      const float4 v = *reinterpret_cast<const float4*>(vs + t * DP_QS + e);
      o.x = fmaf(pt, v.x, o.x);
      o.y = fmaf(pt, v.y, o.y);
      o.z = fmaf(pt, v.z, o.z);
      o.w = fmaf(pt, v.w, o.w);
    }
    const float iv = inv[hh * DP_SMAX + s];
    store_split4(a.xs, plane, (size_t)(n * S + s) * a.nh * d + (h0 + hh) * d + e,
                 make_float4(o.x * iv, o.y * iv, o.z * iv, o.w * iv));
  }
  row_sync();  // the scratch is free for the next unit
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Decode attention for sequence n's new row at position pos and KV head g with its
// nq = nh / nkv query heads (attention.rs:91-154): q, k, v summed from the QKV partials;
// LongRoPE at pos (f64 angles, rope.rs:76-95); k, v written into the static cache at pos
// (cache.rs:47-58); then cache positions 0..pos in 32-position K / V tiles that bulk copies
// bring into shared memory (two buffers: the next tile lands while this one is used).  Warp h
// owns query head h, each lane 4 of its 128 dims: a tile's 32 scores are the lanes' partial
// dot products summed by a butterfly reduce-scatter (31 shuffles; lane j ends with position
// j), then an online softmax in registers (running max and sum: the max-subtracted softmax of
// attention.rs:186-191, accumulated tile by tile) and P V with the probabilities broadcast by
// shuffles.  Output into the split operand (K = nh * d).  Run by the DP_ROW_THREADS row threads
// (row warps >= nq only help with the loads); `uses` counts each tile buffer's completed copies
// (uniform over the CTA).  Returns false if a copy wait gave up (error recorded).
__device__ bool att_decode_unit(const DitPersistArgs& a, const Parts& q, int n, int g, int split, int nsplit, int l,
                                int pos, const Sm& sm, unsigned* uses, int ph) {
  constexpr int d = DP_DEC_D, half = d / 2, d4 = d / 4;
  const int nq = a.nh / a.nkv, tid = row_rank(), warp = tid >> 5, lane = tid & 31;
  float* qs = sm.att;  // [nq][d], then k [d], v [d]
  float* kn = qs + nq * d;
  float* vn = kn + d;
  float* cs = vn + d;  // [half] cos, [half] sin
  float* sn = cs + half;
  float* tiles = sm.att + DP_DEC_TILE_OFF;
  const size_t seq = ((size_t)n * a.nkv + g) * a.max_len * d;
  float* kc = a.kcache + (size_t)l * a.kv_layer_stride + seq;
  float* vc = a.vcache + (size_t)l * a.kv_layer_stride + seq;
  const int ntt = pos / DP_DEC_TILE + 1;  // tiles of positions 0..pos; this split walks [t0, nt)
  const int t0 = (int)((long long)split * ntt / nsplit), nt = (int)((long long)(split + 1) * ntt / nsplit);
  const bool last_split = nt == ntt;      // its range holds position pos (this step's k, v)
  unsigned issued[2] = {uses[0], uses[1]};
  int next = t0;  // thread 0: the next tile to copy
  auto issue = [&](int t) {  // thread 0
    const int rows = min(DP_DEC_TILE, pos + 1 - t * DP_DEC_TILE), b = t & 1;
    const uint32_t bytes = (uint32_t)rows * d * 4;
    float* kt = tiles + b * 2 * DP_DEC_TILE * d;
    mbar_arrive_expect_tx(&sm.att_bar[b], 2 * bytes);
    bulk_g2s(kt, kc + (size_t)t * DP_DEC_TILE * d, bytes, &sm.att_bar[b]);
    bulk_g2s(kt + DP_DEC_TILE * d, vc + (size_t)t * DP_DEC_TILE * d, bytes, &sm.att_bar[b]);
    ++issued[b];
    next = t + 1;
  };
  // tiles of earlier positions only do not depend on this step: they land during the setup
  if (tid == 0)
    while (next < t0 + 2 && next < ntt - 1 && next < nt) issue(next);
  const int cells = (nq + 2) * d4;
  for (int i0 = tid; i0 < cells; i0 += 2 * DP_ROW_THREADS) {
    PRange x[2];
    int dst[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = i0 + k * DP_ROW_THREADS;
      x[k] = PRange{nullptr, 0};
      dst[k] = -1;
      if (i < cells) {
        const int which = i / d4, e = (i % d4) * 4;
        const int c = which < nq ? (g * nq + which) * d : which == nq ? (a.nh + g) * d : (a.nh + a.nkv + g) * d;
        x[k] = q.at(n, c + e);
        dst[k] = which * d + e;
      }
    }
    float4 o[2];
    psum<2, 8>(x, q.stride, o);
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (dst[k] >= 0) *reinterpret_cast<float4*>(qs + dst[k]) = o[k];
  }
  if (a.rope && tid < half) {  // the table built at load time from the same f64 angles (rope.rs:76-95)
    cs[tid] = __ldg(a.rope_pos + ((size_t)pos * 2) * half + tid);
    sn[tid] = __ldg(a.rope_pos + ((size_t)pos * 2 + 1) * half + tid);
  }
  row_sync();
  if (tid == 0) trace_at(a, ph, 3);
  if (a.rope) {  // rows 0..nq-1 are the queries, row nq the key (one rotation pair per thread)
    for (int i = tid; i < (nq + 1) * half; i += DP_ROW_THREADS) {
      float* v = qs + (i / half) * d;
      const int j = i % half;
      const float c = cs[j], si = sn[j];
      const float x1 = v[j], x2 = v[j + half];
      v[j] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, si));
      v[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, si));
    }
    row_sync();
  }
  if (last_split) {
    for (int e = tid; e < d; e += DP_ROW_THREADS) {
      kc[(size_t)pos * d + e] = kn[e];
      vc[(size_t)pos * d + e] = vn[e];
    }
    // the bulk copies below read the row just written through the generic proxy
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  row_sync();
  if (tid == 0) {
    trace_at(a, ph, 1);
    if (next == t0) issue(t0);
  }
  // warp h < nq: query head h, lane: dims 4 lane .. 4 lane + 3
  const bool head = warp < nq;
  const float4 qv = head ? *reinterpret_cast<const float4*>(qs + warp * d + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  float m_run = -FLT_MAX, l_run = 0.f;
  bool good = true;
  for (int t = t0; t < nt; ++t) {
    if (tid == 0 && next == t + 1 && next < nt) issue(next);  // its buffer was released by the sync ending t - 1
    const int b = t & 1, rows = min(DP_DEC_TILE, pos + 1 - t * DP_DEC_TILE);
    const bool w = mbar_wait(&sm.att_bar[b], uses[b] & 1, a.err);
    ++uses[b];
    if (row_or(!w)) {
      good = false;
      break;
    }
    if (head) {
      const float* kt = tiles + b * 2 * DP_DEC_TILE * d;
      const float* vt = kt + DP_DEC_TILE * d;
      float v[DP_DEC_TILE];  // this lane's partial dot product with every position of the tile
#pragma unroll
      for (int j = 0; j < DP_DEC_TILE; ++j) {
        const float4 k4 = j < rows ? *reinterpret_cast<const float4*>(kt + j * d + lane * 4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        v[j] = fmaf(qv.x, k4.x, fmaf(qv.y, k4.y, fmaf(qv.z, k4.z, qv.w * k4.w)));
      }
      // reduce-scatter: after the step with offset `off`, lane keeps the half of the remaining
      // positions selected by its bit `off`; lane j ends with position j's full sum in v[0]
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < off; ++i) {
          const float send = upper ? v[i] : v[i + off];
          const float keep = upper ? v[i + off] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const float sv = lane < rows ? v[0] * a.attn_scale : -FLT_MAX;
      const float m_new = fmaxf(m_run, warp_max(sv));
      const float p = lane < rows ? expf(sv - m_new) : 0.f;
      const float al = expf(m_run - m_new);
      l_run = l_run * al + warp_sum(p);
      m_run = m_new;
      o.x *= al;
      o.y *= al;
      o.z *= al;
      o.w *= al;
#pragma unroll
      for (int j = 0; j < DP_DEC_TILE; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);  // 0 past the tile's rows
        if (j < rows) {
          const float4 v4 = *reinterpret_cast<const float4*>(vt + j * d + lane * 4);
          o.x = fmaf(pj, v4.x, o.x);
          o.y = fmaf(pj, v4.y, o.y);
          o.z = fmaf(pj, v4.z, o.z);
          o.w = fmaf(pj, v4.w, o.w);
        }
      }
    }
    row_sync();  // every reader of this buffer is done before the copy issued at t + 1 reuses it
  }
  if (!good) {  // copies still in flight land before the CTA leaves
    if (tid == 0)
      for (int b = 0; b < 2; ++b)
        for (; uses[b] < issued[b]; ++uses[b]) mbar_wait(&sm.att_bar[b], uses[b] & 1, a.err);
    row_sync();
    return false;
  }
  const size_t out_at = (size_t)n * a.nh * d + (g * nq + warp) * d + lane * 4;
  const size_t plane = (size_t)a.Rpad * a.nh * d;
  if (nsplit == 1) {
    if (head) {
      const float iv = 1.0f / l_run;
      store_split4(a.xs, plane, out_at, make_float4(o.x * iv, o.y * iv, o.z * iv, o.w * iv));
    }
    row_sync();  // the scratch is free for the next unit
    return true;
  }
  // split partials: [unit][split][head][d + 4] = o (unnormalised), running max, running sum, 2
  // pad floats (16-byte aligned rows);
  // the last split to arrive merges them in split order (the same sum whichever CTA it is)
  const int unit = n * a.nkv + g;
  float* part = a.att_part + ((size_t)unit * DP_DEC_SPLITS + split) * nq * (d + 4);
  if (head) {
    *reinterpret_cast<float4*>(part + warp * (d + 4) + lane * 4) = o;
    if (lane == 0) {
      part[warp * (d + 4) + d] = m_run;
      part[warp * (d + 4) + d + 1] = l_run;
    }
  }
  row_sync();
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.att_cnt + unit, 1u);
    sm.flags[1] = prev == (unsigned)nsplit - 1;
    if (sm.flags[1]) {
      __threadfence();
      a.att_cnt[unit] = 0u;  // ready for the next layer
    }
  }
  row_sync();
  if (sm.flags[1] && head) {
    const float* pu = a.att_part + (size_t)unit * DP_DEC_SPLITS * nq * (d + 4) + warp * (d + 4);
    float mx = -FLT_MAX;
    for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, __ldcg(pu + (size_t)sp * nq * (d + 4) + d));
    float den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* ps = pu + (size_t)sp * nq * (d + 4);
      const float w = expf(__ldcg(ps + d) - mx);
      den = fmaf(__ldcg(ps + d + 1), w, den);
      const float4 os = ldcg4(ps + lane * 4);
      acc.x = fmaf(os.x, w, acc.x);
      acc.y = fmaf(os.y, w, acc.y);
      acc.z = fmaf(os.z, w, acc.z);
      acc.w = fmaf(os.w, w, acc.w);
    }
    const float iv = 1.0f / den;
    store_split4(a.xs, plane, out_at, make_float4(acc.x * iv, acc.y * iv, acc.z * iv, acc.w * iv));
  }
  row_sync();  // the scratch and the flag are free for the next unit
  return true;
}

// ACT: silu(gate) * up, both summed from the GU partials, into the split operand (K = I);
// two groups of four elements per thread in flight; run by the DP_ROW_THREADS row threads.
__device__ void act_rows(const DitPersistArgs& a, const Parts& q) {
  const int I = a.I, i4 = I / 4;
  const size_t plane = (size_t)a.Rpad * I, n = (size_t)a.R * i4;
  const size_t step = (size_t)gridDim.x * DP_ROW_THREADS;
  for (size_t i0 = (size_t)blockIdx.x * DP_ROW_THREADS + row_rank(); i0 < n; i0 += 2 * step) {
    PRange x[4];
    int rr[2], jj[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const size_t i = i0 + k * step;
      rr[k] = -1;
      x[2 * k] = x[2 * k + 1] = PRange{nullptr, 0};
      if (i < n) {
        rr[k] = (int)(i / i4);
        jj[k] = (int)(i % i4) * 4;
        x[2 * k] = q.at(rr[k], jj[k]);
        x[2 * k + 1] = q.at(rr[k], I + jj[k]);
      }
    }
    float4 o[4];
    psum<4, 4>(x, q.stride, o);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (rr[k] < 0) continue;
      const float4 gt = o[2 * k], up = o[2 * k + 1];
      store_split4(a.xs_i, plane, (size_t)rr[k] * I + jj[k],
                   make_float4(silu(gt.x) * up.x, silu(gt.y) * up.y, silu(gt.z) * up.z, silu(gt.w) * up.w));
    }
  }
}

// ------------------------------------------------------------------ the kernel

// Static description of one GEMM phase (kind PH_QKV / PH_O / PH_GU / PH_DOWN of layer l) and
// the contiguous run [c0, c1) of its (tile, K chunk) pairs this CTA takes.
struct GemmPh {
  int n_out, kch, gk, c0, c1;
  int b;  // this CTA's rank among the phase's CTAs (the grid rotated by the kind's offset)
  const CUtensorMap* wmap;
  const CUtensorMap* xmap;
};

__device__ GemmPh gemm_phase(const DitPersistArgs& a, int kind, int l) {
  GemmPh g;
  int K, wi;
  if (kind == PH_QKV) { g.n_out = (a.nh + 2 * a.nkv) * a.d; K = a.H; wi = 0; g.gk = DP_KIND_QKV; g.xmap = &a.xmaps[0]; }
  else if (kind == PH_O) { g.n_out = a.H; K = a.nh * a.d; wi = 1; g.gk = DP_KIND_O; g.xmap = &a.xmaps[0]; }
  else if (kind == PH_GU) { g.n_out = 2 * a.I; K = a.H; wi = 2; g.gk = DP_KIND_GU; g.xmap = &a.xmaps[0]; }
  else { g.n_out = a.H; K = a.I; wi = 3; g.gk = DP_KIND_DOWN; g.xmap = &a.xmaps[1]; }
  g.wmap = &a.wmaps[l * 4 + wi];
  g.kch = K / TC_BK;
  const int G = gridDim.x;
  const int total = (g.n_out / a.um) * g.kch, nc = a.ncta[g.gk], b = ((int)blockIdx.x + G - a.cta_off[g.gk]) % G;
  g.b = b;
  g.c0 = b < nc ? (int)((long long)b * total / nc) : 0;
  g.c1 = b < nc ? (int)((long long)(b + 1) * total / nc) : 0;
  return g;
}

__device__ __forceinline__ void tmap_prefetch(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

// MODE: the ATT phase's attention (DP_ATT_SEQ or DP_ATT_DECODE); one instantiation each, so
// neither pays the other's registers.
template <int MODE, int UM>
__global__ void __launch_bounds__(DP_THREADS, 1) dit_persist_kernel(const DitPersistArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int plane_bytes = a.Rpad * TC_BK * 2;
  const int a_bytes = UM * TC_BK * 2;                  // one um x 64 weight box
  const int stage_bytes = a_bytes + 2 * plane_bytes;     // weights, then the hi and lo planes
  Sm sm;
  sm.stages = base;
  sm.att = reinterpret_cast<float*>(base + (size_t)a.nst * stage_bytes);
  sm.red = sm.att + dp_att_floats(MODE);
  sm.full = reinterpret_cast<uint64_t*>(sm.red + 32);
  sm.empty = sm.full + a.nst;
  sm.seg_done = sm.empty + a.nst;
  sm.acc_free = sm.seg_done + 1;
  sm.fin = sm.acc_free + 1;
  sm.att_bar = sm.fin + 1;
  sm.tmem_slot = reinterpret_cast<uint32_t*>(sm.att_bar + 2);
  sm.flags = reinterpret_cast<volatile int*>(sm.tmem_slot + 2);
  sm.segtab = const_cast<int*>(reinterpret_cast<volatile int*>(sm.flags + 2));
  for (int i = threadIdx.x; i < a.tab_len; i += DP_THREADS) sm.segtab[i] = __ldg(a.segtab + i);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t ncols = 32;  // um / 128 accumulators of Rpad columns (at most 512 columns)
  while ((int)ncols < (UM / TC_BM) * a.Rpad) ncols <<= 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nst; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(sm.seg_done, 1);
    mbar_init(sm.acc_free, DP_EPI_THREADS);
    mbar_init(sm.fin, 1);
    mbar_init(&sm.att_bar[0], 1);
    mbar_init(&sm.att_bar[1], 1);
    sm.flags[0] = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(sm.tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  // per-role persistent state: ring position (producer, MMA), segments done
  int prod_i = 0, mma_i = 0, seg_g = 0;
  int pre_n = 0, pre_kind = 0, pre_l = 0;  // producer: weight tiles of the next GEMM phase already armed
  unsigned att_uses[2] = {0u, 0u};         // decode attention: completed copies per tile buffer
  const int dec_pos = MODE == DP_ATT_DECODE ? *a.pos : 0;
  if (warp == 4 && lane == 0) {  // descriptors of layer 0's weight maps and the activation maps
    for (int i = 0; i < 4; ++i) tmap_prefetch(&a.wmaps[i]);
    tmap_prefetch(&a.xmaps[0]);
    tmap_prefetch(&a.xmaps[1]);
  }
  bool ok = true;
  if (MODE == DP_ATT_DECODE && (dec_pos < 0 || dec_pos >= a.max_len)) {  // no cache row for it: stop
    if (threadIdx.x == 0) record_error(a.err, VX_DEVICE_ERR_BOUNDS);
    ok = false;
  }
  const int G = gridDim.x;
  const int nph = a.L * PH_N + 1;

  for (int ph = 0; ph < nph && ok; ++ph) {
    if (ph > 0 && !grid_wait(a, a.bar + ph - 1, (unsigned)G, sm)) {
      ok = false;
      break;
    }
    if (threadIdx.x == 0) trace_at(a, ph, 0);
    const int l = ph / PH_N, kind = ph == nph - 1 ? -1 : ph % PH_N;
    if (warp == 4 && lane == 0 && kind == PH_RES_A && l + 1 < a.L)  // the next layer's weight maps
      for (int i = 0; i < 4; ++i) tmap_prefetch(&a.wmaps[(l + 1) * 4 + i]);
    const DitPersistLayer* w = a.layers + (l < a.L ? l : 0);
    const bool gemm = kind == PH_QKV || kind == PH_O || kind == PH_GU || kind == PH_DOWN;
    if (!gemm) {
      if (warp == 4 && lane == 0 && kind >= 0) {
        // the next phase is a GEMM: its first weight tiles do not depend on this phase, so they
        // stream into the (free) ring during it; the activation planes follow after the barrier
        if (kind != PH_ATT) trace_at(a, ph, 3);
        const GemmPh g = gemm_phase(a, kind + 1, l);
        pre_kind = kind + 1;
        pre_l = l;
        pre_n = 0;
        for (int j = 0; j < std::min(a.pf_stages, g.c1 - g.c0); ++j) {
          const int pi = prod_i + j, s = pi % a.nst, c = g.c0 + j;
          if (pi >= a.nst && !mbar_wait(&sm.empty[s], ((pi / a.nst) - 1) & 1, a.err)) {
            sm.flags[0] = 1;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[s], stage_bytes);
          tma_load_2d(sm.stages + (size_t)s * stage_bytes, g.wmap, (c % g.kch) * TC_BK, (c / g.kch) * UM,
                      &sm.full[s]);
          pre_n = j + 1;
        }
        if (kind != PH_ATT) trace_at(a, ph, 1);
      }
      if (warp == 4) {
        // the producer sits the row phases out (its weight prefetch is in flight)
      } else if (kind == PH_ATT) {  // the row warps
        const Parts q = parts_of(a, sm, DP_KIND_QKV);
        if constexpr (MODE == DP_ATT_DECODE) {  // unit = (sequence, KV head, run of cache tiles)
          const int nbg = a.N * a.nkv;
          const int nsplit = max(1, min(min(DP_DEC_SPLITS, G / nbg), dec_pos / DP_DEC_TILE + 1));
          for (int u = blockIdx.x; u < nbg * nsplit; u += G)
            if (!att_decode_unit(a, q, (u % nbg) / a.nkv, (u % nbg) % a.nkv, u / nbg, nsplit, l, dec_pos, sm,
                                 att_uses, ph)) {
              if (threadIdx.x == 0) sm.flags[0] = 1;
              break;
            }
        } else {  // two heads per unit when one per unit would not fit the grid
          const int hpu = a.N * a.nh > G && (a.nh / a.nkv) % DP_HPU == 0 ? DP_HPU : 1, per = a.nh / hpu;
          for (int u = blockIdx.x; u < a.N * per; u += G) att_unit(a, q, u / per, (u % per) * hpu, hpu, ph, sm);
        }
      } else if (kind == PH_ACT) {  // the row warps
        act_rows(a, parts_of(a, sm, DP_KIND_GU));
      } else if (row_rank() < DP_RES_THREADS) {
        if (kind == -1) {  // final: RMSNorm(x1 + s * down) with the final norm weight
          const Parts q = parts_of(a, sm, DP_KIND_DOWN);
          res_rows(a, a.x1, &q, nullptr, a.final_norm, nullptr, a.out, sm);
        } else if (kind == PH_RES_A) {
          if (l == 0) {
            if (MODE == DP_ATT_SEQ && a.rope) rope_table(a);
            res_rows(a, a.x_in, nullptr, a.x, w->ln_in, a.xs, nullptr, sm);
          } else {
            const Parts q = parts_of(a, sm, DP_KIND_DOWN);
            res_rows(a, a.x1, &q, a.x, w->ln_in, a.xs, nullptr, sm);
          }
        } else {  // PH_RES_B
          const Parts q = parts_of(a, sm, DP_KIND_O);
          res_rows(a, a.x, &q, a.x1, w->ln_post, a.xs, nullptr, sm);
        }
      }
      if (threadIdx.x == 0) trace_at(a, ph, 2);
      if (ph < nph - 1) grid_arrive(a.bar + ph);
      else cta_sync();
      if (sm.flags[0]) ok = false;
      continue;
    }
    // ---- GEMM phase
    const GemmPh g = gemm_phase(a, kind, l);
    const int n_out = g.n_out, kch = g.kch, gk = g.gk, c0 = g.c0, c1 = g.c1, b = g.b, nc = a.ncta[gk];
    const CUtensorMap* wmap = g.wmap;
    const CUtensorMap* xmap = g.xmap;
    if (warp == 4) {
      if (lane == 0) {  // TMA producer
        // the activation operand was written by other CTAs' generic stores before the barrier
        asm volatile("fence.proxy.async.global;" ::: "memory");
        for (int c = c0; c < c1; ++c, ++prod_i) {
          const int s = prod_i % a.nst;
          unsigned char* st = sm.stages + (size_t)s * stage_bytes;
          const int kx = (c % kch) * TC_BK, tile = c / kch;
          if (c - c0 >= pre_n) {  // not armed in the phase before
            if (prod_i >= a.nst && !mbar_wait(&sm.empty[s], ((prod_i / a.nst) - 1) & 1, a.err)) {
              sm.flags[0] = 1;
              break;
            }
            mbar_arrive_expect_tx(&sm.full[s], stage_bytes);
            tma_load_2d(st, wmap, kx, tile * UM, &sm.full[s]);
          }
          tma_load_3d(st + a_bytes, xmap, kx, 0, 0, &sm.full[s]);  // both planes in one box, or the hi plane
          if (a.split_b) tma_load_3d(st + a_bytes + plane_bytes, xmap, kx, 0, 1, &sm.full[s]);
        }
        pre_n = 0;
      }
    } else if (warp == 5) {
      if (lane == 0) {  // MMA issuer
        const uint32_t idesc = tc_idesc(a.Rpad);
        int seg_local = seg_g;
        for (int c = c0; c < c1; ++c, ++mma_i) {
          const bool first = c == c0 || c % kch == 0;
          if (first && seg_local > 0 && !mbar_wait(sm.acc_free, (seg_local - 1) & 1, a.err)) {
            sm.flags[0] = 1;
            break;
          }
          const int s = mma_i % a.nst;
          if (!mbar_wait(&sm.full[s], (mma_i / a.nst) & 1, a.err)) {
            sm.flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(sm.stages + (size_t)s * stage_bytes);
          const uint32_t sh = sa + a_bytes, sl = sh + plane_bytes;
          for (int m = 0; m < UM / TC_BM; ++m) {  // accumulator m: weight rows 128 m .. 128 m + 127 of the unit
            const uint32_t am = sa + m * (TC_BM * TC_BK * 2), dm = tmem + m * a.Rpad;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk) {
              tc_mma(dm, sw128_desc(am + kk * 32), sw128_desc(sh + kk * 32), idesc, (!first || kk > 0) ? 1 : 0);
              tc_mma(dm, sw128_desc(am + kk * 32), sw128_desc(sl + kk * 32), idesc, 1);
            }
          }
          tc_commit(&sm.empty[s]);
          if (c == c1 - 1 || (c + 1) % kch == 0) {
            tc_commit(sm.seg_done);  // the segment's accumulator is complete once its MMAs finish
            ++seg_local;
          }
        }
      }
    } else if (warp < 4) {
      // ---- epilogue (warps 0-3): each segment's partial tile into its slot, rows < R
      const Parts q = parts_of(a, sm, gk);
      int seg = b < nc ? sm.segtab[a.tab_off[gk] + n_out / UM + 1 + b] : 0;
      for (int c = c0; c < c1; ++seg) {
        const int tile = c / kch, cend = std::min(c1, (tile + 1) * kch);
        const bool good = mbar_wait(sm.seg_done, seg_g & 1, a.err);
        tc_fence_after();
        if (!good) sm.flags[0] = 1;
        if (epi_or(!good || sm.flags[0] != 0)) break;  // uniform over the four warps
        if (threadIdx.x == 0 && c == c0) trace_at(a, ph, 1);
        const int nm = UM / TC_BM;
        for (int m = 0; m < nm; ++m) {
          const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16) + m * a.Rpad;
          float* dst = a.part + (size_t)seg * q.stride + m * TC_BM + warp * 32 + lane;
          for (int sl = 0; sl < a.Rpad / 32; ++sl) {
            float v[32];
            tmem_ld16(trow + sl * 32, v);
            tmem_ld16(trow + sl * 32 + 16, v + 16);
            if (m == nm - 1 && sl == a.Rpad / 32 - 1) {  // last TMEM read of the segment: the MMA warp may reuse it
              tc_fence_before();
              mbar_arrive(sm.acc_free);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (sl * 32 + j < a.R) __stcg(dst + (size_t)(sl * 32 + j) * UM, v[j]);
          }
        }
        ++seg_g;
        c = cend;
      }
      if (threadIdx.x == 0) trace_at(a, ph, 2);
    }
    // the MMA thread counts this phase's segments too (its seg_g drives the acc_free parity)
    if (warp == 5) {
      for (int c = c0; c < c1;) {
        c = std::min(c1, (c / kch + 1) * kch);
        ++seg_g;
      }
    }
    if (ph < nph - 1) grid_arrive(a.bar + ph);
    else cta_sync();
    // read after the CTA barrier, where no thread of the CTA still writes the flag
    if (sm.flags[0]) ok = false;
  }

  // ---- leave: no MMA may still be writing TMEM and no copy still landing in shared memory;
  // free TMEM; the last CTA out resets the barrier counters.  Stages armed for a GEMM phase that
  // never ran (abort) get their activation planes too, so the drain below sees them complete.
  if (warp == 4 && lane == 0 && pre_n > 0) {
    const GemmPh g = gemm_phase(a, pre_kind, pre_l);
    for (int j = 0; j < pre_n; ++j, ++prod_i) {
      unsigned char* st = sm.stages + (size_t)(prod_i % a.nst) * stage_bytes;
      const int kx = ((g.c0 + j) % g.kch) * TC_BK;
      tma_load_3d(st + UM * TC_BK * 2, g.xmap, kx, 0, 0, &sm.full[prod_i % a.nst]);
      if (a.split_b) tma_load_3d(st + UM * TC_BK * 2 + plane_bytes, g.xmap, kx, 0, 1, &sm.full[prod_i % a.nst]);
    }
    pre_n = 0;
  }
  if (warp == 5 && lane == 0) {
    tc_commit(sm.fin);
    const long long t0 = clock64();
    while (!mbar_try_wait(sm.fin, 0))
      if (clock64() - t0 > kWaitLimitCycles) break;
  }
  if (warp == 4 && lane == 0) {
    for (int j = prod_i > a.nst ? prod_i - a.nst : 0; j < prod_i; ++j) {
      const long long t0 = clock64();
      while (!mbar_try_wait(&sm.full[j % a.nst], (j / a.nst) & 1))
        if (clock64() - t0 > kWaitLimitCycles) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.bar + nph, 1u);
    if (prev == (unsigned)G - 1) {
      for (int i = 0; i <= nph; ++i) a.bar[i] = 0u;
      if (MODE == DP_ATT_DECODE)  // zero already unless a split gave up (error path)
        for (int i = 0; i < a.N * a.nkv; ++i) a.att_cnt[i] = 0u;
      __threadfence();
    }
  }
}

}  // namespace

int dit_persist_segments(int tiles, int kch, int ncta, int* tab) {
  const int total = tiles * kch;
  int* seg_off = tab;
  int* first = tab + tiles + 1;
  for (int t = 0; t <= tiles; ++t) seg_off[t] = 0;
  int seg = 0;
  for (int b = 0; b < ncta; ++b) {
    const int c0 = (int)((long long)b * total / ncta), c1 = (int)((long long)(b + 1) * total / ncta);
    first[b] = seg;
    for (int c = c0; c < c1;) {
      const int t = c / kch;
      ++seg_off[t + 1];
      ++seg;
      c = std::min(c1, (t + 1) * kch);
    }
  }
  for (int t = 0; t < tiles; ++t) seg_off[t + 1] += seg_off[t];
  return seg;
}

size_t dit_persist_smem(int rpad, int um, int att_mode, int* nst) {
  const int stage = um * TC_BK * 2 + 2 * rpad * TC_BK * 2;
  const size_t fixed = 1024 + (size_t)(dp_att_floats(att_mode) + 32) * 4 + 8 * 32 + 128 + DP_SEGTAB_MAX * 4;
  const int n = (int)std::min<size_t>(6, (227 * 1024 - fixed) / stage);
  *nst = n;
  return fixed + (size_t)n * stage;
}

cudaError_t dit_persist_configure() {
  const void* fns[4] = {(const void*)dit_persist_kernel<DP_ATT_SEQ, TC_BM>,
                        (const void*)dit_persist_kernel<DP_ATT_SEQ, DP_UM_MAX>,
                        (const void*)dit_persist_kernel<DP_ATT_DECODE, TC_BM>,
                        (const void*)dit_persist_kernel<DP_ATT_DECODE, DP_UM_MAX>};
  for (const void* f : fns) {
    const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int dit_persist_grid() {
  int dev = 0, sms = 0, per = 0;
  int nst = 0;
  const size_t smem = std::max(dit_persist_smem(256, TC_BM, DP_ATT_SEQ, &nst),
                               dit_persist_smem(64, DP_UM_MAX, DP_ATT_DECODE, &nst));
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, dit_persist_kernel<DP_ATT_SEQ, TC_BM>, DP_THREADS, smem) !=
          cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return per >= 1 ? sms : 0;
}

cudaError_t launch_dit_persist(const DitPersistArgs& a, int grid, cudaStream_t st) {
  int nst = 0;
  const size_t smem = dit_persist_smem(a.Rpad, a.um, a.att_mode, &nst);
  DitPersistArgs b = a;
  b.nst = nst;
  b.pf_stages = std::max(0, std::min(a.pf_stages, nst));
  if (nst < 2 || grid <= 0 || !a.xmaps || (a.um != TC_BM && a.um != DP_UM_MAX) || a.um * a.Rpad > 512 * TC_BM)
    return cudaErrorInvalidValue;
  if (a.att_mode == DP_ATT_DECODE &&
      (a.S != 1 || !a.kcache || !a.vcache || !a.pos || (a.rope && !a.rope_pos) || !a.att_part || !a.att_cnt))
    return cudaErrorInvalidValue;
  for (int k = 0; k < DP_KINDS; ++k)
    if (a.ncta[k] < 1 || a.ncta[k] > grid || a.cta_off[k] < 0 || a.cta_off[k] >= grid) return cudaErrorInvalidValue;
  if (a.tab_len < 1 || a.tab_len > DP_SEGTAB_MAX) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(DP_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  if (a.att_mode == DP_ATT_DECODE)
    return a.um == DP_UM_MAX ? cudaLaunchKernelEx(&cfg, dit_persist_kernel<DP_ATT_DECODE, DP_UM_MAX>, b)
                             : cudaLaunchKernelEx(&cfg, dit_persist_kernel<DP_ATT_DECODE, TC_BM>, b);
  return a.um == DP_UM_MAX ? cudaLaunchKernelEx(&cfg, dit_persist_kernel<DP_ATT_SEQ, DP_UM_MAX>, b)
                           : cudaLaunchKernelEx(&cfg, dit_persist_kernel<DP_ATT_SEQ, TC_BM>, b);
}



bool persist_stack_prepare(PersistStack& ps, const LmStackView& v, int max_rows, bool trace, bool* oom,
                           int rope_positions) {
  *oom = false;
  if (ps.grid >= 0) return ps.grid > 0;
  ps.grid = 0;
  ps.view = v;
  const int nq = v.nkv > 0 ? v.nh / v.nkv : 0;
  // few rows (<= 64): 256-row units (one 32 KB weight copy per K chunk: the copy count bounds
  // those phases); more rows: 128-row units (twice the units to spread over the CTAs)
  const int rmax = std::min(256, (std::max(max_rows, 1) + 31) / 32 * 32);
  int um = rmax <= 64 ? DP_UM_MAX : TC_BM;
  if (const char* e = getenv("VX_DIT_UM")) um = atoi(e) == DP_UM_MAX ? DP_UM_MAX : TC_BM;
  ps.split_b = false;
  if (const char* e = getenv("VX_DIT_SPLIT_B")) ps.split_b = atoi(e) != 0;
  if (const char* e = getenv("VX_DIT_PF")) ps.pf_stages = std::max(0, atoi(e));
  const bool shape_ok = v.L > 0 && v.L <= 64 && v.H <= 2048 && v.H % um == 0 && v.nh * v.d == v.H &&
                        v.d % 4 == 0 && v.nkv > 0 && v.nh % v.nkv == 0 && ((v.nh + 2 * v.nkv) * v.d) % um == 0 &&
                        (2 * v.I) % um == 0 && v.I % 64 == 0 && max_rows > 0;
  if (!shape_ok) return false;
  ps.seq_ok = v.d <= 64;
  ps.decode_ok = v.d == DP_DEC_D && nq <= DP_DEC_NQ && nq <= DP_ROW_THREADS / 32;
  if (dit_persist_configure() != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const int grid = dit_persist_grid();
  cudaGetLastError();
  if (grid <= 0) return false;
  const size_t H = v.H, I = v.I, qkv = (size_t)(v.nh + 2 * v.nkv) * v.d;
  // segment tables: each GEMM kind deals its (tile, K chunk) pairs to ncta CTAs, at least
  // `min_pairs` pairs each (env VX_DIT_PAIRS="qkv,o,gu,down" overrides the minimums)
  const int tiles[DP_KINDS] = {(int)(qkv / um), v.H / um, (int)(2 * I / um), v.H / um};
  const int kchs[DP_KINDS] = {v.H / 64, v.nh * v.d / 64, v.H / 64, (int)(I / 64)};
  // (fewer CTAs per unit: fewer partial slots for the next row phase to sum; measured best for
  // the 8-row LM step at 256-row units, and for the 176-row DiT forward at 128-row units)
  // 176-row DiT forward (8-patch CFM solve): {4, 4, 8, 8} 5.16 ms per solve against 5.36 for {2, 2, 8, 4},
  // 5.30-5.32 for 8 or 6 instead of any one 4 or 8, 5.51 for gate|up at 16 (same box)
  int min_pairs[DP_KINDS] = {4, 4, 8, 8};
  if (um == DP_UM_MAX) {                    // 8-row LM step: 2.14 -> 2.05 ms against {2, 2, 1, 4}
    min_pairs[DP_KIND_QKV] = 4;
    min_pairs[DP_KIND_O] = 4;
    min_pairs[DP_KIND_GU] = 1;
    min_pairs[DP_KIND_DOWN] = 8;
  }
  if (const char* e = getenv("VX_DIT_PAIRS"))
    sscanf(e, "%d,%d,%d,%d", &min_pairs[0], &min_pairs[1], &min_pairs[2], &min_pairs[3]);
  std::vector<int> tab;
  int max_segs = 0;
  for (int k = 0; k < DP_KINDS; ++k) {
    const int total = tiles[k] * kchs[k];
    ps.ncta[k] = std::max(1, std::min(grid, total / std::max(1, min_pairs[k])));
    ps.tab_off[k] = (int)tab.size();
    tab.resize(tab.size() + tiles[k] + 1 + ps.ncta[k]);
    max_segs = std::max(max_segs, dit_persist_segments(tiles[k], kchs[k], ps.ncta[k], tab.data() + ps.tab_off[k]));
  }
  ps.tab_len = (int)tab.size();
  if (ps.tab_len > DP_SEGTAB_MAX) return false;
  std::vector<CUtensorMap> maps(4 * v.L);
  const size_t nph = 8 * (size_t)v.L + 1;
  bool ok = cudaMalloc(&ps.layers, sizeof(DitPersistLayer) * v.L) == cudaSuccess &&
            cudaMemcpy(ps.layers, v.layers.data(), sizeof(DitPersistLayer) * v.L, cudaMemcpyHostToDevice) ==
                cudaSuccess &&
            cudaMalloc(&ps.bar, (nph + 1) * sizeof(unsigned)) == cudaSuccess &&
            cudaMemset(ps.bar, 0, (nph + 1) * sizeof(unsigned)) == cudaSuccess &&
            cudaMalloc(&ps.x, (size_t)rmax * H * 4) == cudaSuccess &&
            cudaMalloc(&ps.x1, (size_t)rmax * H * 4) == cudaSuccess &&
            cudaMalloc(&ps.xs, 2 * (size_t)rmax * H * 2) == cudaSuccess &&
            cudaMalloc(&ps.xsi, 2 * (size_t)rmax * I * 2) == cudaSuccess &&
            cudaMemset(ps.xs, 0, 2 * (size_t)rmax * H * 2) == cudaSuccess &&
            cudaMemset(ps.xsi, 0, 2 * (size_t)rmax * I * 2) == cudaSuccess &&
            cudaMalloc(&ps.part, (size_t)max_segs * rmax * um * 4) == cudaSuccess &&
            cudaMalloc(&ps.rope_tab, 2 * 16 * 64 * 4) == cudaSuccess &&
            cudaMalloc(&ps.segtab, tab.size() * 4) == cudaSuccess &&
            cudaMemcpy(ps.segtab, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaMalloc(&ps.maps, sizeof(CUtensorMap) * 4 * v.L) == cudaSuccess;
  for (int l = 0; ok && l < v.L; ++l) {
    const DitPersistLayer& w = v.layers[l];
    ok = tc_map_2d(&maps[4 * l + 0], w.wqkv, (int)qkv, (int)H, um) == cudaSuccess &&
         tc_map_2d(&maps[4 * l + 1], w.wo, (int)H, v.nh * v.d, um) == cudaSuccess &&
         tc_map_2d(&maps[4 * l + 2], w.wgu, (int)(2 * I), (int)H, um) == cudaSuccess &&
         tc_map_2d(&maps[4 * l + 3], w.wd, (int)H, (int)I, um) == cudaSuccess;
  }
  ok = ok && cudaMemcpy(ps.maps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok && trace)
    ok = cudaMalloc(&ps.trace, nph * grid * 4 * 8) == cudaSuccess &&
         cudaMemset(ps.trace, 0, nph * grid * 4 * 8) == cudaSuccess;
  if (ok && ps.decode_ok) {  // split partials of the decode attention and their arrival counters
    const size_t units = (size_t)rmax * v.nkv;
    ok = cudaMalloc(&ps.att_part, units * DP_DEC_SPLITS * nq * (v.d + 4) * 4) == cudaSuccess &&
         cudaMalloc(&ps.att_cnt, units * 4) == cudaSuccess && cudaMemset(ps.att_cnt, 0, units * 4) == cudaSuccess;
  }
  if (ok && v.rope && rope_positions > 0) {
    const int half = v.d / 2;
    ok = cudaMalloc(&ps.rope_pos, (size_t)rope_positions * 2 * half * 4) == cudaSuccess;
    if (ok)
      ok = launch_rope_table(v.rope, rope_positions, half, ps.rope_pos, 0) == cudaSuccess &&
           cudaDeviceSynchronize() == cudaSuccess;
  }
  if (!ok) {
    cudaGetLastError();
    persist_stack_free(ps);
    ps.grid = 0;
    *oom = true;
    return false;
  }
  ps.rmax = rmax;
  ps.um = um;
  ps.grid = grid;
  return true;
}

bool persist_stack_rows(PersistStack& ps, int rpad) {
  if (ps.grid <= 0 || rpad > ps.rmax || rpad % 32 != 0) return false;
  if (ps.xmaps.count(rpad)) return true;
  CUtensorMap xm[2];
  CUtensorMap* dev = nullptr;
  const int bp = ps.split_b ? 1 : 2;
  const bool ok = tc_map_3d(&xm[0], ps.xs, 2, rpad, ps.view.H, rpad, bp) == cudaSuccess &&
                  tc_map_3d(&xm[1], ps.xsi, 2, rpad, ps.view.I, rpad, bp) == cudaSuccess &&
                  cudaMalloc(&dev, sizeof(xm)) == cudaSuccess &&
                  cudaMemcpy(dev, xm, sizeof(xm), cudaMemcpyHostToDevice) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    if (dev) cudaFree(dev);
    return false;
  }
  ps.xmaps[rpad] = dev;
  return true;
}

void persist_stack_free(PersistStack& ps) {
  for (void* p : {(void*)ps.layers, (void*)ps.maps, (void*)ps.x, (void*)ps.x1, (void*)ps.part, (void*)ps.rope_tab,
                  (void*)ps.rope_pos, (void*)ps.att_part, (void*)ps.att_cnt,
                  (void*)ps.xs, (void*)ps.xsi, (void*)ps.segtab, (void*)ps.bar, (void*)ps.trace})
    if (p) cudaFree(p);
  for (auto& kv : ps.xmaps) cudaFree(kv.second);
  ps.xmaps.clear();
  ps.layers = nullptr;
  ps.maps = nullptr;
  ps.x = ps.x1 = ps.part = ps.rope_tab = ps.rope_pos = ps.att_part = nullptr;
  ps.att_cnt = nullptr;
  ps.xs = ps.xsi = nullptr;
  ps.segtab = nullptr;
  ps.bar = nullptr;
  ps.trace = nullptr;
}

DitPersistArgs persist_stack_args(const PersistStack& ps, int N, int S, const float* x_in, float* out, int* err) {
  const LmStackView& v = ps.view;
  DitPersistArgs a = {};
  a.L = v.L;
  a.H = v.H;
  a.I = v.I;
  a.nh = v.nh;
  a.nkv = v.nkv;
  a.d = v.d;
  a.S = S;
  a.N = N;
  a.R = N * S;
  a.Rpad = (a.R + 31) / 32 * 32;
  a.att_mode = DP_ATT_SEQ;
  a.um = ps.um;
  a.split_b = ps.split_b ? 1 : 0;
  a.eps = v.eps;
  a.res_scale = v.res_scale;
  a.attn_scale = v.attn_scale;
  a.layers = ps.layers;
  a.wmaps = ps.maps;
  const auto it = ps.xmaps.find(a.Rpad);
  a.xmaps = it == ps.xmaps.end() ? nullptr : it->second;
  a.rope = v.rope;
  a.final_norm = v.norm_w;
  a.x_in = x_in;
  a.x = ps.x;
  a.x1 = ps.x1;
  a.out = out;
  a.xs = ps.xs;
  a.xs_i = ps.xsi;
  a.part = ps.part;
  a.rope_tab = ps.rope_tab;
  a.rope_pos = ps.rope_pos;
  a.att_part = ps.att_part;
  a.att_cnt = ps.att_cnt;
  a.pf_stages = ps.pf_stages;
  a.segtab = ps.segtab;
  a.tab_len = ps.tab_len;
  for (int k = 0; k < DP_KINDS; ++k) {
    a.tab_off[k] = ps.tab_off[k];
    a.ncta[k] = ps.ncta[k];
  }
  a.bar = ps.bar;
  a.err = err;
  a.trace = ps.trace;
  return a;
}

}  // namespace vx
