// Attention kernels (sm_100a), replacing MiniCpmAttention::sdpa + repeat_kv
// (reference src/minicpm4/attention.rs:156-204).
//
// * attn_decode_kernel: one query token per batch row against the static KV cache
//   (forward_step, attention.rs:129-150).  Split-K flash-decode over GQA groups:
//   grid = (max_splits, n_kv_heads, B); only ceil(len/32) splits (at most max_splits) are
//   active, each covering a contiguous span of the filled prefix 0..len.  A CTA stages
//   32-position K/V tiles of its KV head in shared memory ONCE and all n_rep (= 8) query
//   heads of the group read them there: warp r is query head r, lane j scores position j of
//   the tile (K tile XOR-swizzled in 16-byte chunks so the row-per-lane reads are
//   conflict-free), an online softmax runs per warp, and P.V accumulates d/32 output dims
//   per lane.  With one active split the CTA writes the result directly; otherwise each
//   writes an (m, l, o[d]) partial to scratch and the last CTA to arrive (atomic counter,
//   no waiting) merges them lane-parallel and resets the counter, so the kernel replays
//   inside a CUDA graph with no host work.
// * attn_prefill_kernel: S query rows against S keys of a KV layout [B, nkv, s_max, d]
//   (forward / prefill and the non-causal DiT / LocEnc paths, attention.rs:55-88), causal
//   or not, one warp per query row with an online softmax.
#include <cfloat>
#include <cmath>
#include <mutex>

#include "../../include/voxcpm_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace vx {

constexpr int ATT_TILE = 32;

template <int D>
__device__ __forceinline__ int kswz(int row, int chunk) {  // float4-chunk index inside a K row
  return row * (D / 4) + (chunk ^ (row & 7));
}

template <int D, int NREP>
__global__ void __launch_bounds__(32 * NREP) attn_decode_kernel(const AttnDecodeArgs a) {
  constexpr int DPL = D / 32;  // output dims per lane
  constexpr int NC = D / 4;    // float4 chunks per row
  __shared__ __align__(16) float qs[NREP][D];
  __shared__ __align__(16) float4 ks[ATT_TILE * NC];
  __shared__ __align__(16) float vs[ATT_TILE][D];
  __shared__ int last_flag;

  pdl_wait();
  pdl_launch_dependents();
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int len = a.pos_ptr ? (*a.pos_ptr + 1) : a.len;
  const int active = min(a.nsplit, (len + ATT_TILE - 1) / ATT_TILE);
  if (split >= active) return;
  const int span = (len + active - 1) / active;
  const int j0 = split * span, j1 = min(len, j0 + span);

  for (int i = tid; i < NREP * D; i += 32 * NREP) qs[i / D][i % D] = a.q[(size_t)b * a.nh * D + g * NREP * D + i];

  const float* kb = a.kcache + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const float* vb = a.vcache + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const int r = warp;  // query head within the group
  float m = -INFINITY, l = 0.f, o[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) o[e] = 0.f;

  for (int t0 = j0; t0 < j1; t0 += ATT_TILE) {
    const int nt = min(ATT_TILE, j1 - t0);
    __syncthreads();  // previous tile fully consumed (and qs written on the first pass)
    for (int c = tid; c < ATT_TILE * NC; c += 32 * NREP) {
      const int row = c / NC, ch = c % NC;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (row < nt) {
        kv = __ldg(reinterpret_cast<const float4*>(kb + (size_t)(t0 + row) * D) + ch);
        vv = __ldg(reinterpret_cast<const float4*>(vb + (size_t)(t0 + row) * D) + ch);
      }
      ks[kswz<D>(row, ch)] = kv;
      *reinterpret_cast<float4*>(&vs[row][ch * 4]) = vv;
    }
    __syncthreads();
    // scores: lane j <-> position t0 + j;  scores = q.k^T * scale (attention.rs:166)
    float s = 0.f;
#pragma unroll 8
    for (int ch = 0; ch < NC; ++ch) {
      const float4 kk = ks[kswz<D>(lane, ch)];
      const float4 qq = *reinterpret_cast<const float4*>(&qs[r][ch * 4]);
      s = fmaf(qq.x, kk.x, s);
      s = fmaf(qq.y, kk.y, s);
      s = fmaf(qq.z, kk.z, s);
      s = fmaf(qq.w, kk.w, s);
    }
    s = lane < nt ? s * a.scale : -INFINITY;
    const float mn = fmaxf(m, warp_max(s));
    const float alpha = expf(m - mn);  // m == -inf on the first tile -> 0
    const float p = lane < nt ? expf(s - mn) : 0.f;
    l = l * alpha + warp_sum(p);
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[e] *= alpha;
    for (int jj = 0; jj < nt; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      if constexpr (DPL == 4) {
        const float4 vv = *reinterpret_cast<const float4*>(&vs[jj][lane * 4]);
        o[0] = fmaf(pj, vv.x, o[0]);
        o[1] = fmaf(pj, vv.y, o[1]);
        o[2] = fmaf(pj, vv.z, o[2]);
        o[3] = fmaf(pj, vv.w, o[3]);
      } else {
        const float2 vv = *reinterpret_cast<const float2*>(&vs[jj][lane * 2]);
        o[0] = fmaf(pj, vv.x, o[0]);
        o[1] = fmaf(pj, vv.y, o[1]);
      }
    }
    m = mn;
  }

  float* outp = a.out + (size_t)b * a.nh * D + (g * NREP + r) * D + lane * DPL;
  if (active == 1) {
#pragma unroll
    for (int e = 0; e < DPL; ++e) outp[e] = o[e] / l;
    return;
  }
  // partial (o[d], m, l) of this split for head r
  float* p = a.partials + (((size_t)(b * a.nkv + g) * a.nsplit + split) * NREP + r) * (D + 2);
#pragma unroll
  for (int e = 0; e < DPL; ++e) p[lane * DPL + e] = o[e];
  if (lane == 0) {
    p[D] = m;
    p[D + 1] = l;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&a.counters[b * a.nkv + g], 1u);
    last_flag = (prev == (unsigned)active - 1);
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // last CTA: merge the `active` partials of head r, lane-parallel over splits
  const float* pb = a.partials + ((size_t)(b * a.nkv + g) * a.nsplit * NREP + r) * (D + 2);
  const size_t sstride = (size_t)NREP * (D + 2);
  const float ms = lane < active ? __ldcg(pb + lane * sstride + D) : -INFINITY;
  const float M = warp_max(ms);
  const float f = lane < active ? expf(ms - M) : 0.f;
  const float L = warp_sum(lane < active ? f * __ldcg(pb + lane * sstride + D + 1) : 0.f);
  float acc[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
  for (int sp = 0; sp < active; ++sp) {
    const float fs = __shfl_sync(0xffffffffu, f, sp);
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] = fmaf(fs, __ldcg(pb + sp * sstride + lane * DPL + e), acc[e]);
  }
#pragma unroll
  for (int e = 0; e < DPL; ++e) outp[e] = acc[e] / L;
  if (tid == 0) a.counters[b * a.nkv + g] = 0u;
}

cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  const int nrep = a.nh / a.nkv;
  if (nrep != 8 || (a.d != 128 && a.d != 64) || a.nsplit < 1 || a.nsplit > 32) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nsplit, a.nkv, a.B);
  cfg.blockDim = dim3(32 * 8);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  if (a.d == 128) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<128, 8>, a);
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<64, 8>, a);
}

// --------------------------------------------------------------------------- prefill



template <int D>
__global__ void __launch_bounds__(256) attn_prefill_kernel(const AttnPrefillArgs a) {
  // The 8 query rows of a CTA share one (batch, head) and so one KV head: 32-position K/V
  // tiles are staged in shared memory once per CTA (coalesced) and every warp reads them there.
  // With a.qkv the rows come straight from the fused projection and q / k are rotated here
  // (apply_rotary_pos_emb, rope.rs:76-95): k in shared memory once per staged tile, q per lane.
  constexpr int DPL = D / 32, HALF = D / 2;
  __shared__ __align__(16) float ks[ATT_TILE][D];
  __shared__ __align__(16) float vs[ATT_TILE][D];
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 8 + warp;  // query row
  const int h = blockIdx.y, b = blockIdx.z;
  const bool active = i < a.S;
  const int g = h / (a.nh / a.nkv);  // repeat_kv head map (attention.rs:196-204)
  const bool fused = a.qkv != nullptr;
  const size_t W = (size_t)(a.nh + 2 * a.nkv) * D;  // fused projection row width
  float qr[DPL], o[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    const int c = lane * DPL + e;
    float x = 0.f;
    if (active && !fused) {
      x = a.q[((size_t)b * a.S + i) * a.nh * D + h * D + c];
    } else if (active) {
      const float* qrow = a.qkv + ((size_t)b * a.S + i) * W + (size_t)h * D;
      x = qrow[c];
      if (a.rope_tab) {  // q'[c] = q[c] cos - q[c+half] sin (c < half); q[c] cos + q[c-half] sin
        const float xp = qrow[c < HALF ? c + HALF : c - HALF];
        const float cs = a.rope_tab[(size_t)i * D + c % HALF], sn = a.rope_tab[(size_t)i * D + HALF + c % HALF];
        x = c < HALF ? __fadd_rn(__fmul_rn(x, cs), __fmul_rn(-xp, sn)) : __fadd_rn(__fmul_rn(x, cs), __fmul_rn(xp, sn));
      }
    }
    qr[e] = x;
    o[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const float* kb = fused ? a.qkv + (size_t)b * a.S * W + (size_t)(a.nh + g) * D
                          : a.k + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const float* vb = fused ? a.qkv + (size_t)b * a.S * W + (size_t)(a.nh + a.nkv + g) * D
                          : a.v + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const size_t kv_stride = fused ? W : (size_t)D;  // floats between consecutive positions
  // keys this CTA needs: all S (non-causal) or up to its last query row (causal mask j > i)
  const int last_row = min(a.S, (int)blockIdx.x * 8 + 8);
  const int jmax = a.causal ? last_row : a.S;
  const int jn = a.causal ? (i + 1) : a.S;  // this warp's keys (attention.rs:168-182)
  for (int t0 = 0; t0 < jmax; t0 += ATT_TILE) {
    const int nt = min(ATT_TILE, jmax - t0);
    __syncthreads();
    for (int c = threadIdx.x; c < nt * (D / 4); c += 256) {
      const int row = c / (D / 4), ch = c % (D / 4);
      *reinterpret_cast<float4*>(&ks[row][ch * 4]) =
          __ldg(reinterpret_cast<const float4*>(kb + (size_t)(t0 + row) * kv_stride) + ch);
      *reinterpret_cast<float4*>(&vs[row][ch * 4]) =
          __ldg(reinterpret_cast<const float4*>(vb + (size_t)(t0 + row) * kv_stride) + ch);
    }
    __syncthreads();
    if (fused && a.rope_tab) {  // rotate the staged k rows in place, one (position, pair) per thread
      for (int c = threadIdx.x; c < nt * HALF; c += 256) {
        const int row = c / HALF, j = c % HALF;
        const float cs = a.rope_tab[(size_t)(t0 + row) * D + j], sn = a.rope_tab[(size_t)(t0 + row) * D + HALF + j];
        const float xa = ks[row][j], xb = ks[row][j + HALF];
        ks[row][j] = __fadd_rn(__fmul_rn(xa, cs), __fmul_rn(-xb, sn));
        ks[row][j + HALF] = __fadd_rn(__fmul_rn(xb, cs), __fmul_rn(xa, sn));
      }
      __syncthreads();
    }
    if (!active) continue;
    const int jend = min(nt, jn - t0);
    for (int jj = 0; jj < jend; ++jj) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) s = fmaf(qr[e], ks[jj][lane * DPL + e], s);
      s = warp_sum(s) * a.scale;
      const float mn = fmaxf(m, s);
      const float alpha = expf(m - mn), p = expf(s - mn);
      l = l * alpha + p;
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[e] = fmaf(p, vs[jj][lane * DPL + e], o[e] * alpha);
      m = mn;
    }
  }
  if (!active) return;
  const size_t orow_i = (size_t)b * a.S + i;
  if (a.xs) {  // straight into the o_proj GEMM's split operand
    const int M = a.B * a.S, K = a.nh * D;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      const float v = o[e] / l;
      const __nv_bfloat16 hb = __float2bfloat16_rn(v);
      a.xs[orow_i * K + h * D + lane * DPL + e] = __bfloat16_as_ushort(hb);
      a.xs[((size_t)M + orow_i) * K + h * D + lane * DPL + e] =
          __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(hb)));
    }
    return;
  }
  float* orow = a.out + orow_i * a.nh * D + h * D;
#pragma unroll
  for (int e = 0; e < DPL; ++e) orow[lane * DPL + e] = o[e] / l;
}

cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t st, bool pdl) {
  if (a.nh % a.nkv != 0 || (a.d != 128 && a.d != 64)) return cudaErrorInvalidValue;
  if (a.qkv && a.S > ATT_FUSED_ROPE_MAX_S) return cudaErrorInvalidValue;  // every CTA rotates all S keys
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.S + 7) / 8, a.nh, a.B);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  count_launch();
  if (a.d == 128) return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<128>, a);
  return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<64>, a);
}

}  // namespace vx

// --------------------------------------------------------------------------- no allocation
//
// Decode attention for callers that must not allocate device memory.  Some hosts of this
// library hand it a fixed memory budget (an audio server that reserves everything at
// start-up, a plugin whose host owns the allocator) or call it from threads where a
// cudaMalloc would stall the device (cudaMalloc can synchronise, which breaks real-time
// audio deadlines).  vx_attention_decode needs a context, whose creation and scratch pool
// allocate; this variant takes no context and keeps its split partials and arrival
// counters in file-scope __device__ arrays instead:
//   * partials: 1 MiB (kStaticPartialBytes), enough for B * n_kv_heads * 16 splits *
//     8 heads * (head_dim + 2) floats; larger shapes are rejected with VX_ERR_SHAPE;
//   * counters: 64 words, so B * n_kv_heads <= 64.
// Every GPU that loads the library holds these arrays until the process exits.  All calls
// share them: two calls whose kernels overlap on the GPU (different streams, or different
// host threads) race on the same scratch and must be serialised by the caller.
namespace vx {
namespace {

constexpr size_t kStaticPartialBytes = 1u << 20;
constexpr int kStaticCounters = 64;
constexpr int kStaticMaxSplits = 16;

static __device__ __align__(256) float g_static_partials[kStaticPartialBytes / sizeof(float)];
static __device__ __align__(256) unsigned int g_static_counters[kStaticCounters];

// Device addresses of the two arrays, looked up once per device.  In host code the array
// names are host-side stand-ins, not device addresses, so they are never passed to a kernel.
// The cached addresses belong to the device's primary context: after a cudaDeviceReset the
// module is loaded again and they are stale (documented for callers in the header).
struct StaticScratchAddr {
  float* partials = nullptr;
  unsigned int* counters = nullptr;
};
StaticScratchAddr g_static_addr[128];
std::mutex g_static_mu;

int static_scratch_for_current_device(StaticScratchAddr* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return VX_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_static_mu);
  StaticScratchAddr& a = g_static_addr[dev];
  if (!a.partials) {
    void* p = nullptr;
    void* c = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_partials) != cudaSuccess) return VX_ERR_CUDA;
    if (cudaGetSymbolAddress(&c, g_static_counters) != cudaSuccess) return VX_ERR_CUDA;
    a.partials = static_cast<float*>(p);
    a.counters = static_cast<unsigned int*>(c);
  }
  *out = a;
  return VX_OK;
}

}  // namespace
}  // namespace vx

extern "C" int vx_attention_decode_static(const float* q, const float* kcache, const float* vcache, int B,
                                          int nh, int nkv, int head_dim, int s_max, int cur_len, float* out,
                                          void* stream) {
  using namespace vx;
  if (!q || !kcache || !vcache || !out) return VX_ERR_ARG;
  if (B <= 0 || nkv <= 0 || nh % nkv != 0 || nh / nkv != 8 || (head_dim != 128 && head_dim != 64))
    return VX_ERR_SHAPE;
  if (cur_len <= 0 || cur_len > s_max) return VX_ERR_SHAPE;
  const size_t need = (size_t)B * nkv * kStaticMaxSplits * 8 * (head_dim + 2) * sizeof(float);
  if (B * nkv > kStaticCounters || need > kStaticPartialBytes) return VX_ERR_SHAPE;
  StaticScratchAddr sa;
  const int rc = static_scratch_for_current_device(&sa);
  if (rc != VX_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the arrays keep the previous call's contents: start this call's counters from zero
  if (cudaMemsetAsync(sa.counters, 0, (size_t)B * nkv * sizeof(unsigned int), st) != cudaSuccess)
    return VX_ERR_CUDA;
  AttnDecodeArgs a = {q, kcache, vcache, B, nh, nkv, head_dim, s_max, nullptr, cur_len,
                      (float)(1.0 / std::sqrt((double)head_dim)), kStaticMaxSplits, sa.partials, sa.counters, out};
  return launch_attn_decode(a, st, false) == cudaSuccess ? VX_OK : VX_ERR_CUDA;
}
