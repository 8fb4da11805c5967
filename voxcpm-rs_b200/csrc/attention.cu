// Attention kernels (sm_100a), replacing MiniCpmAttention::sdpa + repeat_kv
// (reference src/minicpm4/attention.rs:156-204).
//
// * attn_decode_kernel: one query token per batch row against the static KV cache
//   (forward_step, attention.rs:129-150).  Split-K flash-decode: the filled prefix 0..len is
//   cut into `nsplit` chunks; grid = (nsplit, n_kv_heads, B).  Each CTA serves all n_rep
//   query heads of its KV head (GQA without materialising repeat_kv), keeps an online
//   softmax per head, and writes (m, l, o[d]) partials to scratch.  The last CTA to finish
//   for a (batch, kv head) merges the partials and writes the output; it also resets the
//   arrival counter, so the kernel replays inside a CUDA graph with no host work.
// * attn_prefill_kernel: S query rows against S keys of a KV layout [B, nkv, s_max, d]
//   (forward / prefill and the non-causal DiT / LocEnc paths, attention.rs:55-88), causal
//   or not, one warp per query row with an online softmax.
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"

namespace vx {



template <int D, int NREP>
__global__ void __launch_bounds__(256) attn_decode_kernel(const AttnDecodeArgs a) {
  constexpr int DPL = D / 32;  // dims per lane
  __shared__ float qs[NREP][D];
  __shared__ float wm[8][NREP], wl[8][NREP];
  __shared__ float wo[8][NREP][D];
  __shared__ int last_flag;

  pdl_wait();
  pdl_launch_dependents();
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int len = a.pos_ptr ? (*a.pos_ptr + 1) : a.len;
  const int chunk = (len + a.nsplit - 1) / a.nsplit;
  const int j0 = split * chunk, j1 = min(len, j0 + chunk);

  for (int i = tid; i < NREP * D; i += 256) {
    const int r = i / D, e = i % D;
    qs[r][e] = a.q[(size_t)b * a.nh * D + (g * NREP + r) * D + e];
  }
  __syncthreads();

  float qr[NREP][DPL], o[NREP][DPL], m[NREP], l[NREP];
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      qr[r][e] = qs[r][lane * DPL + e];
      o[r][e] = 0.f;
    }
  }
  const float* kb = a.kcache + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const float* vb = a.vcache + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  for (int j = j0 + warp; j < j1; j += 8) {
    float kr[DPL], vr[DPL];
    if constexpr (DPL == 4) {
      const float4 k4 = __ldg(reinterpret_cast<const float4*>(kb + (size_t)j * D) + lane);
      const float4 v4 = __ldg(reinterpret_cast<const float4*>(vb + (size_t)j * D) + lane);
      kr[0] = k4.x; kr[1] = k4.y; kr[2] = k4.z; kr[3] = k4.w;
      vr[0] = v4.x; vr[1] = v4.y; vr[2] = v4.z; vr[3] = v4.w;
    } else {
      const float2 k2 = __ldg(reinterpret_cast<const float2*>(kb + (size_t)j * D) + lane);
      const float2 v2 = __ldg(reinterpret_cast<const float2*>(vb + (size_t)j * D) + lane);
      kr[0] = k2.x; kr[1] = k2.y;
      vr[0] = v2.x; vr[1] = v2.y;
    }
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) s = fmaf(qr[r][e], kr[e], s);
      s = warp_sum(s) * a.scale;  // scores = q.k^T * scale (attention.rs:166)
      const float mn = fmaxf(m[r], s);
      const float alpha = expf(m[r] - mn);
      const float p = expf(s - mn);
      l[r] = l[r] * alpha + p;
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[r][e] = fmaf(p, vr[e], o[r][e] * alpha);
      m[r] = mn;
    }
  }
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    if (lane == 0) {
      wm[warp][r] = m[r];
      wl[warp][r] = l[r];
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) wo[warp][r][lane * DPL + e] = o[r][e];
  }
  __syncthreads();
  // merge the 8 warps of this CTA into one (m, l, o) partial per head
  const size_t pbase = ((size_t)((b * a.nkv + g) * a.nsplit + split)) * NREP * (D + 2);
  for (int i = tid; i < NREP * D; i += 256) {
    const int r = i / D, e = i % D;
    float M = -INFINITY;
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w][r]);
    float L = 0.f, O = 0.f;
    if (M > -INFINITY) {
      for (int w = 0; w < 8; ++w) {
        const float f = (wm[w][r] > -INFINITY) ? expf(wm[w][r] - M) : 0.f;
        L = fmaf(wl[w][r], f, L);
        O = fmaf(wo[w][r][e], f, O);
      }
    }
    float* p = a.partials + pbase + (size_t)r * (D + 2);
    p[e] = O;
    if (e == 0) {
      p[D] = M;
      p[D + 1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&a.counters[b * a.nkv + g], 1u);
    last_flag = (prev == (unsigned)a.nsplit - 1);
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  const size_t cbase = ((size_t)((b * a.nkv + g) * a.nsplit)) * NREP * (D + 2);
  for (int i = tid; i < NREP * D; i += 256) {
    const int r = i / D, e = i % D;
    float M = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s)
      M = fmaxf(M, __ldcg(a.partials + cbase + ((size_t)s * NREP + r) * (D + 2) + D));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float* p = a.partials + cbase + ((size_t)s * NREP + r) * (D + 2);
      const float ms = __ldcg(p + D);
      if (ms == -INFINITY) continue;
      const float f = expf(ms - M);
      L = fmaf(__ldcg(p + D + 1), f, L);
      O = fmaf(__ldcg(p + e), f, O);
    }
    a.out[(size_t)b * a.nh * D + (g * NREP + r) * D + e] = O / L;
  }
  if (tid == 0) a.counters[b * a.nkv + g] = 0u;
}

cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  const int nrep = a.nh / a.nkv;
  if (nrep != 8 || (a.d != 128 && a.d != 64)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nsplit, a.nkv, a.B);
  cfg.blockDim = dim3(256);
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
  constexpr int DPL = D / 32;
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 8 + warp;  // query row
  const int h = blockIdx.y, b = blockIdx.z;
  if (i >= a.S) return;
  const int g = h / (a.nh / a.nkv);  // repeat_kv head map (attention.rs:196-204)
  const float* qrow = a.q + ((size_t)b * a.S + i) * a.nh * D + h * D;
  float qr[DPL], o[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    qr[e] = qrow[lane * DPL + e];
    o[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const float* kb = a.k + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const float* vb = a.v + ((size_t)(b * a.nkv + g) * a.s_max) * D;
  const int jn = a.causal ? (i + 1) : a.S;  // causal mask: j > i -> -inf (attention.rs:168-182)
  for (int j = 0; j < jn; ++j) {
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) s = fmaf(qr[e], kb[(size_t)j * D + lane * DPL + e], s);
    s = warp_sum(s) * a.scale;
    const float mn = fmaxf(m, s);
    const float alpha = expf(m - mn), p = expf(s - mn);
    l = l * alpha + p;
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[e] = fmaf(p, vb[(size_t)j * D + lane * DPL + e], o[e] * alpha);
    m = mn;
  }
  float* orow = a.out + ((size_t)b * a.S + i) * a.nh * D + h * D;
#pragma unroll
  for (int e = 0; e < DPL; ++e) orow[lane * DPL + e] = o[e] / l;
}

cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t st, bool pdl) {
  if (a.nh % a.nkv != 0 || (a.d != 128 && a.d != 64)) return cudaErrorInvalidValue;
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
