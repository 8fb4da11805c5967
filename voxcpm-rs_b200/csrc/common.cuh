// Shared device helpers for the voxcpm B200 kernels (sm_100a).
//
// - bf16 unpacking (weights are stored as raw bf16 bit patterns, upcast exactly to f32)
// - warp / block reductions
// - mbarrier + 1-D bulk-copy (TMA engine) wrappers with BOUNDED waits: every wait gives up
//   after ~2 s of clock64 cycles, records an error code in the library's device error word
//   and lets the kernel return, so a lost arrival never hangs the GPU.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#define VX_DEVICE_ERR_TIMEOUT 1
#define VX_DEVICE_ERR_BOUNDS 2

namespace vx {

// Host side: number of kernels this thread has launched through the library (graph replays
// add the number of kernels the graph holds).  Reported by vx_launch_count.
extern thread_local unsigned long long g_launches;
inline void count_launch(unsigned long long n = 1) { g_launches += n; }

constexpr long long kWaitLimitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// Kernels that can give up on a wait get a pointer to their context's device error word
// (read and cleared by vx_ctx_synchronize).
__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// dot of 8 bf16 (packed in a uint4) with 8 f32
__device__ __forceinline__ float dot8(const uint4 w, const float* x, float acc) {
  acc = fmaf(bf16lo(w.x), x[0], acc);
  acc = fmaf(bf16hi(w.x), x[1], acc);
  acc = fmaf(bf16lo(w.y), x[2], acc);
  acc = fmaf(bf16hi(w.y), x[3], acc);
  acc = fmaf(bf16lo(w.z), x[4], acc);
  acc = fmaf(bf16hi(w.z), x[5], acc);
  acc = fmaf(bf16lo(w.w), x[6], acc);
  acc = fmaf(bf16hi(w.w), x[7], acc);
  return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum over `nwarps` warps using `red` (>= nwarps floats of shared memory).
// Every thread of the block gets the total.  `bar_id`/`nthreads` select a named barrier
// so a subset of warps (e.g. consumer warps only) can reduce among themselves.
__device__ __forceinline__ void named_sync(int bar_id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float group_sum(float v, float* red, int nwarps, int bar_id) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  named_sync(bar_id, nwarps * 32);
  float t = 0.f;
  for (int i = 0; i < nwarps; ++i) t += red[i];
  named_sync(bar_id, nwarps * 32);
  return t;
}

// ------------------------------------------------------------------ mbarrier / bulk copy

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records VX_DEVICE_ERR_TIMEOUT) if the phase did not
// complete within the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(err, VX_DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared through the TMA engine, completing `bytes` of
// transaction count on `bar`.  dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy that makes the lines a load touches the first to be evicted (data read once).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 cache-policy hint (e.g. l2_policy_evict_first()).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Bulk prefetch of a global range into L2 (TMA engine, no shared-memory destination).
// addr 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Issue L2 prefetches for this CTA's 1/gridDim share of [ptr, ptr + bytes), 32 KB per request.
__device__ __forceinline__ void prefetch_share_l2(const void* ptr, size_t bytes) {
  if (!ptr || bytes == 0) return;
  const size_t share = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
  size_t b0 = share * blockIdx.x;
  const size_t b1 = b0 + share < bytes ? b0 + share : bytes;
  const char* p = static_cast<const char*>(ptr);
  for (; b0 < b1; b0 += 32768) {
    const size_t n = (b1 - b0) < 32768 ? (b1 - b0) : 32768;
    bulk_prefetch_l2(p + b0, (uint32_t)(n & ~size_t(15)));
  }
}

// Programmatic dependent launch: wait for the preceding grid's memory to be visible /
// allow the next grid to start launching.  Both are no-ops without the launch attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch configuration with programmatic dependent launch: the kernel may be scheduled while
// its predecessor in the stream drains; it must call pdl_wait() before touching anything the
// predecessor writes or reads.
struct PdlLaunch {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  PdlLaunch(dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
};

// Four consecutive f32 activations (row r, columns k..k+3) stored as the tcgen05 GEMM's split
// operand: bf16(v) in row r and bf16(v - bf16(v)) in row M + r of a [2M, K] bf16 buffer
// (k a multiple of 4).
__device__ __forceinline__ void store_split4(uint16_t* xs, int M, int K, size_t r, int k, float4 v) {
  const float f[4] = {v.x, v.y, v.z, v.w};
  uint16_t hi[4], lo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat16 h = __float2bfloat16_rn(f[i]);
    hi[i] = __bfloat16_as_ushort(h);
    lo[i] = __bfloat16_as_ushort(__float2bfloat16_rn(f[i] - __bfloat162float(h)));
  }
  *reinterpret_cast<uint2*>(xs + r * K + k) =
      make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
  *reinterpret_cast<uint2*>(xs + ((size_t)M + r) * K + k) =
      make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
}

// silu_stable: x * sigmoid(x) in f32 (reference src/minicpm4/mod.rs:29-33)
__device__ __forceinline__ float silu(float x) { return x * (1.0f / (1.0f + expf(-x))); }

}  // namespace vx
