// Few-row GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   Y[m, n] = sum_k W[n, k] * X[m, k]  (+ bias[n]) (or Y = R + s * (...))   m < M <= 128
//
// W is a bf16 weight matrix [N, K] (checkpoint [out, in] layout), X f32 activations.  The
// weights are the MMA's A operand (M_mma = 128 weight rows per tile) and the activations
// the B operand ("swap AB": tokens become the MMA N dimension, so 1..128 tokens map onto
// N = 16..256 without padding the weight side).  For f32-grade accuracy the activations are
// split exactly into two bf16 halves, X = X_hi + X_lo (X_hi = bf16(X), X_lo = bf16(X - X_hi)),
// stacked as 2M B-rows; products of bf16 values are exact in the f32 accumulator, so the
// result carries ~2^-16 relative error per term instead of bf16's 2^-8.  The epilogue adds
// the hi and lo columns.
//
// Pipeline per CTA (one 128-row weight tile x one K split): warp 0 lane 0 issues TMA tile
// loads (SWIZZLE_128B, 64-element K blocks, each into this CTA only) into a ring of shared-memory
// stages; warp 1 lane 0 issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32 in TMEM) and
// releases each stage with tcgen05.commit; after the last block all four warps read the
// accumulator with tcgen05.ld (warp w owns TMEM lanes 32w..32w+31 = weight rows).  With
// K split across CTAs, each writes an f32 partial tile to scratch and the last CTA to
// arrive (atomic counter, no waiting) sums the splits in order (deterministic) and runs
// the epilogue.  Every mbarrier wait is bounded; on a timeout the CTA records an error,
// frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"

namespace vx {

constexpr int TC_THREADS = 128;
constexpr int TC_MAX_SPLITS = 8;  // K splits per tile (partials summed by the last CTA)

struct TcGemmArgs {
  int M, N, K, NB;       // NB = padded B rows (2M rounded up to 16)
  int splits, kblocks_per_split;
  const float* bias;     // [N] or null
  const float* R;        // residual [M, ldy] or null (may alias Y)
  float res_scale;
  float* Y;              // [M, ldy]
  int ldy;
  float* partials;       // [tiles][splits][M][128]
  unsigned int* counters;  // [tiles], zero-initialised, reset by the last CTA
  int* err;
  int nstages;
  int cluster;  // 1: the K splits of a tile form one thread-block cluster and sum through DSMEM
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory address of `p` in the CTA of cluster rank `rank` (DSMEM window).
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ int ld_dsmem_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcGemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned stage buffers: [A tile 16 KB | B tile NB*128 B] per stage
  unsigned char* base = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int a_bytes = TC_BM * TC_BK * 2;
  const int b_bytes = a.NB * TC_BK * 2;
  const int stage_bytes = a_bytes + ((b_bytes + 1023) & ~1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + a.nstages * stage_bytes);
  uint64_t* empty = full + a.nstages;
  uint64_t* done = empty + a.nstages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] abort, [1] last-CTA
  // cluster mode: this split's partial tile [M][128] f32, read by the cluster's other CTAs
  float* spart = reinterpret_cast<float*>(base + a.nstages * stage_bytes + 1024);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int kb0 = split * a.kblocks_per_split;
  const int nkb = a.kblocks_per_split;
  uint32_t ncols = 32;
  while ((int)ncols < a.NB) ncols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  if (warp == 0) {  // TMEM allocation (warp-wide, converged)
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The weights never depend on the previous kernel: under programmatic dependent launch the
  // producer issues the first stages' weight tiles before waiting for it, so they stream
  // while the previous kernel drains; the activation tiles follow the wait.
  const int pre = nkb < a.nstages ? nkb : a.nstages;
  if (warp == 0 && lane == 0)
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], a_bytes + b_bytes);
      tma_load_2d(base + i * stage_bytes, &tmW, (kb0 + i) * TC_BK, tile * TC_BM, &full[i]);
    }
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0 && lane == 0) {
    // ---- TMA producer
    int issued = pre;  // stages whose copies have been issued
    bool aborted = false;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % a.nstages;
      if (i >= a.nstages && !mbar_wait(&empty[s], ((i / a.nstages) - 1) & 1, a.err)) {
        atomicExch(&flags[0], 1);
        aborted = true;
        break;
      }
      unsigned char* st = base + s * stage_bytes;
      const int kx = (kb0 + i) * TC_BK;
      if (i >= pre) {
        mbar_arrive_expect_tx(&full[s], a_bytes + b_bytes);
        tma_load_2d(st, &tmW, kx, tile * TC_BM, &full[s]);
      }
      tma_load_2d(st + a_bytes, &tmX, kx, 0, &full[s]);
      issued = i + 1 > issued ? i + 1 : issued;
    }
    if (aborted || *reinterpret_cast<volatile int*>(&flags[0])) {
      // do not let the CTA leave while a copy into its shared memory may still land: wait
      // (bounded) for the stages issued and not yet known to be consumed
      for (int j = issued > a.nstages ? issued - a.nstages : 0; j < issued; ++j) {
        const long long t0 = clock64();
        while (!mbar_try_wait(&full[j % a.nstages], (j / a.nstages) & 1))
          if (clock64() - t0 > kWaitLimitCycles) break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    const uint32_t idesc = tc_idesc(a.NB);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % a.nstages;
      if (!mbar_wait(&full[s], (i / a.nstages) & 1, a.err)) {
        atomicExch(&flags[0], 1);
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(base + s * stage_bytes);
      const uint32_t sb = sa + a_bytes;
#pragma unroll
      for (int kk = 0; kk < TC_BK / 16; ++kk)  // 16-element K steps: +32 bytes inside the swizzle row
        tc_mma(tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (i > 0 || kk > 0) ? 1 : 0);
      tc_commit(&empty[s]);
    }
    // always: `done` completes once every MMA issued above has finished, so TMEM is never
    // freed under an in-flight MMA, also on the abort path
    tc_commit(done);
  }
  __syncwarp();
  // ---- epilogue: all four warps
  const bool ok = mbar_wait(done, 0, a.err);
  tc_fence_after();
  if (!ok) atomicExch(&flags[0], 1);
  __syncthreads();
  const int n = tile * TC_BM + warp * 32 + lane;  // this thread's weight row
  if (!flags[0]) {
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    float* part = a.splits == 1 ? nullptr
                  : a.cluster   ? spart
                                : a.partials + (((size_t)tile * a.splits + split) * a.M) * TC_BM;
    for (int c0 = 0; c0 < a.M; c0 += 16) {
      float hi[16], lo[16];
      tmem_ld16(trow + c0, hi);
      tmem_ld16(trow + a.M + c0, lo);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = c0 + j;
        if (m >= a.M) break;
        const float acc = hi[j] + lo[j];
        if (part) {
          part[(size_t)m * TC_BM + warp * 32 + lane] = acc;
        } else if (n < a.N) {
          float v = acc;
          if (a.bias) v += a.bias[n];
          if (a.R) v = a.R[(size_t)m * a.ldy + n] + v * a.res_scale;
          a.Y[(size_t)m * a.ldy + n] = v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  if (a.splits > 1 && a.cluster) {
    // ---- split-K inside the cluster: every CTA of the tile reaches both cluster barriers (also
    // after an abort); CTA r then sums output rows [r*ceil(M/S), ...) over the S partials in
    // split order (deterministic), reading the other CTAs' partial tiles through DSMEM
    cluster_sync_all();
    const int S = a.splits;
    bool any_abort = false;
    for (int r = 0; r < S; ++r) any_abort |= ld_dsmem_s32(dsmem_addr(&flags[0], r)) != 0;
    const int per = (a.M + S - 1) / S;
    const int m0 = split * per, m1 = min(a.M, m0 + per);
    if (!any_abort && n < a.N) {
      const float bn = a.bias ? a.bias[n] : 0.f;
      for (int m = m0; m < m1; ++m) {
        const float* src = spart + (size_t)m * TC_BM + threadIdx.x;
        float acc = 0.f;
        for (int r = 0; r < S; ++r) acc += ld_dsmem_f32(dsmem_addr(src, r));
        float y = acc + bn;
        if (a.R) y = a.R[(size_t)m * a.ldy + n] + y * a.res_scale;
        a.Y[(size_t)m * a.ldy + n] = y;
      }
    }
    cluster_sync_all();  // the partial tiles stay alive until every CTA has read them
    return;
  }
  if (flags[0] || a.splits == 1) return;
  // ---- split-K: the last CTA of this tile sums the partials in split order
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[tile], 1u);
    flags[1] = (prev == (unsigned)a.splits - 1);
  }
  __syncthreads();
  if (!flags[1]) return;
  __threadfence();
  const float* __restrict__ pt = a.partials + ((size_t)tile * a.splits * a.M) * TC_BM + threadIdx.x;
  const float bn = (a.bias && n < a.N) ? a.bias[n] : 0.f;
  constexpr int RB = 4;  // rows per batch: RB * splits independent loads in flight
  for (int m0 = 0; m0 < a.M; m0 += RB) {
    float v[RB][TC_MAX_SPLITS];
    float r[RB];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const int m = m0 + i;
#pragma unroll
      for (int s = 0; s < TC_MAX_SPLITS; ++s)
        v[i][s] = (m < a.M && s < a.splits) ? __ldcg(pt + ((size_t)s * a.M + m) * TC_BM) : 0.f;
      r[i] = (a.R && m < a.M && n < a.N) ? a.R[(size_t)m * a.ldy + n] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const int m = m0 + i;
      if (m >= a.M || n >= a.N) continue;
      float acc = 0.f;  // split order: deterministic
#pragma unroll
      for (int s = 0; s < TC_MAX_SPLITS; ++s)
        if (s < a.splits) acc += v[i][s];
      float y = acc + bn;
      if (a.R) y = r[i] + y * a.res_scale;
      a.Y[(size_t)m * a.ldy + n] = y;
    }
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;
}

// X [M, K] f32 (row stride ldx) -> Xs [NB, K] bf16: rows 0..M hi, M..2M lo, the rest zero.
__global__ void split_bf16_kernel(const float* __restrict__ X, int ldx, int M, int K, int NB, uint16_t* __restrict__ Xs) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t total = (size_t)NB * K;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / K), k = (int)(i % K);
    float v = 0.f;
    if (r < M) {
      v = X[(size_t)r * ldx + k];
    } else if (r < 2 * M) {
      const float x = X[(size_t)(r - M) * ldx + k];
      v = x - __bfloat162float(__float2bfloat16_rn(x));
    }
    Xs[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
}

// ------------------------------------------------------------------ host side

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;

cudaError_t get_encoder() {
  std::lock_guard<std::mutex> lk(g_encode_mu);
  if (g_encode) return cudaSuccess;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return cudaSuccess;
}

cudaError_t make_map(CUtensorMap* m, const void* ptr, int rows, int K, int box_rows) {
  if (((uintptr_t)ptr & 15) || (K * 2) % 16) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_map_3d(CUtensorMap* m, const void* ptr, int planes, int rows, int K, int box_rows, int box_planes) {
  if (((uintptr_t)ptr & 15) || (K * 2) % 16 || box_planes < 1 || box_planes > planes) return cudaErrorInvalidValue;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)K * 2 * rows};
  cuuint32_t box[3] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows, (cuuint32_t)box_planes};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Whether clusters of `splits` CTAs with `smem` bytes each can be resident (cached per shape).
bool cluster_fits(int splits, int smem) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, bool> memo;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(splits, smem);
  auto it = memo.find(key);
  if (it != memo.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, splits);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const bool ok = cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel, &cfg) == cudaSuccess && n >= 1;
  cudaGetLastError();
  memo[key] = ok;
  return ok;
}

}  // namespace

// Raise the dynamic shared-memory limit on the current device; called once per context,
// before any launch or capture.
cudaError_t tc_gemm_configure() {
  cudaError_t e = get_encoder();
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t tc_map_2d(CUtensorMap* m, const void* ptr, int rows, int K, int box_rows) {
  cudaError_t e = get_encoder();
  return e != cudaSuccess ? e : make_map(m, ptr, rows, K, box_rows);
}

cudaError_t tc_map_3d(CUtensorMap* m, const void* ptr, int planes, int rows, int K, int box_rows, int box_planes) {
  cudaError_t e = get_encoder();
  return e != cudaSuccess ? e : make_map_3d(m, ptr, planes, rows, K, box_rows, box_planes);
}

// N need not be a multiple of 128: the last weight tile's rows past N read as zeros (TMA) and
// its outputs past N are not stored; at most 1024 tiles (the split-K counters).
bool tc_gemm_supported(int M, int N, int K) {
  return M >= 1 && M <= 128 && N >= 1 && N <= 1024 * TC_BM && K % TC_BK == 0 && K > 0;
}

// Scratch needed by launch_tc_gemm for these shapes (bf16 split X, split-K partials): the
// grid is at most max(target_ctas, N/128) CTAs, each with one [M, 128] partial.
size_t tc_gemm_scratch_bytes(int M, int N, int K, int target_ctas) {
  const int NB = ((2 * M + 15) / 16) * 16;
  const int tiles = (N + TC_BM - 1) / TC_BM;
  const size_t xs = ((size_t)NB * K * 2 + 255) & ~(size_t)255;
  const size_t part = (size_t)std::max(tiles, target_ctas) * M * TC_BM * 4;
  return xs + part + 4096;
}

// scratch: >= tc_gemm_scratch_bytes; counters: >= N/128 zeroed words (reset by the kernel).
namespace {

// The GEMM proper over the split activations at the start of `scratch`: rows [0, M) bf16(x),
// rows [M, 2M) bf16(x - bf16(x)); the tensor map covers `x_rows` rows (2M: the TMA box's
// rows past them read as zeros; NB: the split kernel wrote the zero rows).
cudaError_t tc_gemm_core(int M, int N, int K, int x_rows, const uint16_t* W, const float* bias, const float* R,
                         float res_scale, float* Y, int ldy, void* scratch, unsigned* counters, int* err,
                         cudaStream_t st, int target_ctas) {
  cudaError_t e;
  const int NB = ((2 * M + 15) / 16) * 16;
  const int tiles = (N + TC_BM - 1) / TC_BM, kblocks = K / TC_BK;
  // K splits: the largest divisor of the K blocks (at most TC_MAX_SPLITS) keeping the grid
  // within about one CTA per SM; a tile's CTAs each stream >= 1 K block of 16 KB
  int splits = 1;
  const int cap = std::max(tiles, target_ctas / 2);
  for (int s = 1; s <= std::min(TC_MAX_SPLITS, kblocks); ++s)
    if (kblocks % s == 0 && tiles * s <= cap) splits = s;
  const uint16_t* Xs = static_cast<const uint16_t*>(scratch);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(scratch) + (((size_t)NB * K * 2 + 255) & ~(size_t)255));
  CUtensorMap tmW, tmX;
  if ((e = make_map(&tmW, W, N, K, TC_BM)) != cudaSuccess) return e;
  if ((e = make_map(&tmX, Xs, x_rows, K, NB)) != cudaSuccess) return e;
  TcGemmArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.NB = NB;
  a.splits = splits;
  a.kblocks_per_split = kblocks / splits;
  a.bias = bias;
  a.R = R;
  a.res_scale = res_scale;
  a.Y = Y;
  a.ldy = ldy;
  a.partials = partials;
  a.counters = counters;
  a.err = err;
  const int stage_bytes = TC_BM * TC_BK * 2 + ((NB * TC_BK * 2 + 1023) & ~1023);
  const int part_bytes = splits > 1 ? M * TC_BM * 4 : 0;  // the cluster reduction's partial tile
  a.nstages = std::max(1, std::min({6, a.kblocks_per_split, (200 * 1024 - part_bytes) / stage_bytes}));
  const int smem = 1024 + a.nstages * stage_bytes + 1024 + part_bytes + 256;
  count_launch();
  PdlLaunch l(dim3(tiles, splits), dim3(TC_THREADS), smem, st);
  // the K splits of a tile as one cluster (DSMEM reduction) when the device can hold it
  cudaLaunchAttribute attrs[2] = {l.attr[0], {}};
  a.cluster = 0;
  if (splits > 1 && cluster_fits(splits, smem)) {
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = 1;
    attrs[1].val.clusterDim.y = splits;
    attrs[1].val.clusterDim.z = 1;
    l.cfg.attrs = attrs;
    l.cfg.numAttrs = 2;
    a.cluster = 1;
  }
  return cudaLaunchKernelEx(&l.cfg, tc_gemm_kernel, tmW, tmX, a);
}

}  // namespace

cudaError_t launch_tc_gemm(const float* X, int ldx, int M, int N, int K, const uint16_t* W, const float* bias,
                           const float* R, float res_scale, float* Y, int ldy, void* scratch, unsigned* counters,
                           int* err, cudaStream_t st, int target_ctas) {
  if (!tc_gemm_supported(M, N, K)) return cudaErrorInvalidValue;
  cudaError_t e = get_encoder();
  if (e != cudaSuccess) return e;
  const int NB = ((2 * M + 15) / 16) * 16;
  count_launch();
  {
    PdlLaunch l(dim3(std::min(4096, (NB * K + 255) / 256)), dim3(256), 0, st);
    if ((e = cudaLaunchKernelEx(&l.cfg, split_bf16_kernel, X, ldx, M, K, NB, static_cast<uint16_t*>(scratch))) !=
        cudaSuccess)
      return e;
  }
  return tc_gemm_core(M, N, K, NB, W, bias, R, res_scale, Y, ldy, scratch, counters, err, st, target_ctas);
}

uint16_t* tc_gemm_presplit_buffer(void* scratch) { return static_cast<uint16_t*>(scratch); }

cudaError_t launch_tc_gemm_presplit(int M, int N, int K, const uint16_t* W, const float* bias, const float* R,
                                    float res_scale, float* Y, int ldy, void* scratch, unsigned* counters, int* err,
                                    cudaStream_t st, int target_ctas) {
  if (!tc_gemm_supported(M, N, K)) return cudaErrorInvalidValue;
  cudaError_t e = get_encoder();
  if (e != cudaSuccess) return e;
  return tc_gemm_core(M, N, K, 2 * M, W, bias, R, res_scale, Y, ldy, scratch, counters, err, st, target_ctas);
}

}  // namespace vx
