// Persistent batch-1 decode step (sm_100a): ONE launch per token runs every decoder layer
// and the greedy head (reference MiniCpmModel::forward_step, src/minicpm4/model.rs:64-84).
//
// Why: the per-kernel decode step is 5 launches per layer; each streams a few MB of weights
// and loses microseconds to its pipeline ramp and tail.  Here one CTA per SM stays resident
// for the whole token and its producer warp streams ALL of that CTA's operand tiles, phase
// after phase, through one shared-memory ring with 1-D bulk copies (the TMA engine).
// Weights never depend on activations, and neither do the KV-cache rows of earlier
// positions, so while the consumer warps wait for the previous phase's result the producer
// already fills the ring with the next phase's tiles: HBM stays busy across the phase
// boundaries that cost a ramp and a tail per launch before.
//
// Phases per layer (the unit a CTA owns; units spread round-robin with a rotating offset so
// every CTA streams about the same bytes per token):
//   Q    input RMSNorm -> qkv_proj rows -> LongRoPE -> q buffer, k/v into the static cache
//        (layer.rs:64-66, attention.rs:102-127); unit = a rotate_half pair of 8-row groups
//   ATT  flash-decode over the cached prefix (attention.rs:129-150, 156-204); unit = one KV
//        head's 8 query heads against a span of positions whose K/V rows arrive through the
//        ring (the row of the current position, written by Q, is read after the wait); the
//        last split to finish merges the online-softmax partials
//   O    o_proj + residual into x1 (attention.rs:153, layer.rs:67); unit = 8 rows
//   GU   post-attention RMSNorm -> gate|up rows -> silu(gate)*up (layer.rs:69-71,
//        mlp.rs:29-33); unit = matching gate and up 8-row groups
//   D    down_proj + residual into x0 (mlp.rs:33, layer.rs:72); unit = 8 rows
// then the greedy head: final norm -> tied-embedding logits -> argmax -> next input
// embedding, position and step advanced on the device.
//
// Phase ordering: a CTA that finishes its units of phase p adds 1 to counter[p] (release
// after a CTA barrier); a CTA with units in phase p+1 waits (acquire) until counter[p] has
// heard from every CTA that owns units of p.  Data produced inside the launch is read with
// L2-coherent loads (ld.global.cg).  Every wait is bounded; on a timeout or an error raised
// elsewhere the CTA records it, stops cleanly (all in-flight copies landed) and the host
// reports VX_ERR_TIMEOUT.  The last CTA to leave zeroes the counters for the next launch.
//
// GEMV arithmetic per output row is the same as the per-kernel step's streamed GEMV (same
// per-lane partial sums and warp tree), so the two paths agree to rounding in attention.
#include <algorithm>
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "persist.cuh"

namespace vx {

namespace {

constexpr int PK_CWARPS = 8;
constexpr int PK_CTHREADS = PK_CWARPS * 32;
constexpr int PK_THREADS = PK_CTHREADS + 32;
constexpr int PK_ROWS = 8;
constexpr int PK_MAX_SMEM = 232448;  // 227 KB opt-in dynamic shared memory per CTA
constexpr int PK_MISC_FLOATS = 64 + 64 + 64;  // rope tables, reduction scratch
constexpr int PK_RES_UNITS = 4;      // residual rows preloaded per warp and phase
constexpr int PK_XREG = 4;           // float4 per thread held by a normalising load_x (K <= 4096)

enum { PH_Q = 0, PH_ATT = 1, PH_O = 2, PH_GU = 3, PH_D = 4, PH_PER_LAYER = 5, PH_HEAD = 5 };

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Named barrier over the consumer warps that also ORs a per-thread flag: every thread gets
// the same answer, so abort decisions stay uniform across the CTA.
__device__ __forceinline__ bool sync_or(bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v), "r"(PK_CTHREADS)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void csync() { named_sync(1, PK_CTHREADS); }

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void trace_mark(const PersistArgs& a, int p, int k) {
  if (a.trace) a.trace[((size_t)p * gridDim.x + blockIdx.x) * PERSIST_TRACE_FIELDS + k] = gtimer();
}

// flags[0]: consumers stopped (producer must stop too); flags[1]: last-arrival broadcast;
// flags[2]: picked token broadcast; flags[3]: producer gave up.
struct Smem {
  uint16_t* ring;
  float* xs;
  float* ctab;  // [64]
  float* stab;  // [64]
  float* red;   // [64]: [0,8) group sums / merge, [16,32) per-warp argmax, [48,50) CTA argmax
  volatile int* flags;
  uint64_t* full;
  uint64_t* empty;
};

// Attention split layout of this launch, the same in every CTA.
struct AttGeo {
  int pos, len, span, nsplit, ns_max, items;
};

// Bounded wait for a ring stage, by every consumer thread.  Returns false on failure.
__device__ __forceinline__ bool wait_full(uint64_t* bar, uint32_t parity, int* err, volatile int* flags) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!flags[0] && !flags[3]) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(err, VX_DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
  return false;
}

// Bounded wait (consumer thread 0) until `cnt` reaches `target`, then a CTA barrier that
// makes the outcome uniform.  Returns false when the step must stop.
__device__ bool dep_wait(const unsigned* cnt, unsigned target, int* err, bool bad) {
  if (threadIdx.x == 0 && !bad) {
    if (ld_acquire(cnt) < target) {
      const long long t0 = clock64();
      int n = 0;
      while (ld_acquire(cnt) < target) {
        if ((++n & 63) == 0) {
          if (*reinterpret_cast<volatile int*>(err) != 0) {
            bad = true;
            break;
          }
          if (clock64() - t0 > kWaitLimitCycles) {
            record_error(err, VX_DEVICE_ERR_TIMEOUT);
            bad = true;
            break;
          }
        }
      }
    }
  }
  return !sync_or(bad);
}

// Publish this CTA's completion of a phase (after all its stores).
__device__ __forceinline__ void arrive(unsigned* cnt) {
  csync();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
}

struct Geo {
  const uint16_t* W;
  int K;
  int U;    // units in the phase
  int gpu;  // 8-row groups per unit
  int kind;
};

__device__ __forceinline__ int unit_row(const PersistArgs& a, int kind, int u, int gi) {
  if (kind == PH_Q) {  // rotate_half pair: rows j*8.. of the first and second half of a head
    const int hp = a.d / 16;
    return (u / hp) * a.d + (u % hp) * PK_ROWS + gi * (a.d / 2);
  }
  if (kind == PH_GU) return gi * a.I + u * PK_ROWS;  // gate rows, then the matching up rows
  return u * PK_ROWS;
}

__device__ __forceinline__ Geo geo_of(const PersistArgs& a, int l, int kind, const AttGeo& at) {
  const PersistLayer& w = a.layers[l < a.L ? l : 0];
  switch (kind) {
    case PH_Q: return {w.wqkv, a.H, (a.nh + 2 * a.nkv) * a.d / 16, 2, PH_Q};
    case PH_ATT: return {nullptr, 0, at.items, 1, PH_ATT};
    case PH_O: return {w.wo, a.nh * a.d, a.H / PK_ROWS, 1, PH_O};
    case PH_GU: return {w.wgu, a.H, a.I / PK_ROWS, 2, PH_GU};
    case PH_D: return {w.wd, a.I, a.H / PK_ROWS, 1, PH_D};
    default: return {a.embed, a.H, a.V / PK_ROWS, 1, PH_HEAD};
  }
}

__device__ __forceinline__ int first_unit(int off, int G) {
  return ((int)blockIdx.x - off % G + G) % G;
}

// ---------------------------------------------------------------- producer warp (lane 0)

// Position in this CTA's stage sequence: phases in order (5 per layer, then the head), this
// CTA's units of each phase, the 8-row groups of a unit, the K chunks of a group (an
// attention unit is one stage).
struct Cursor {
  int l, kind, off;
  int u, gi, c, nch;
  Geo g;
  bool valid;
};

template <int KC>
__device__ void cursor_seek(const PersistArgs& a, Cursor& k, const AttGeo& at) {
  const int G = gridDim.x;
  while (true) {
    k.g = geo_of(a, k.l, k.kind, at);
    const int first = first_unit(k.off, G);
    if (first < k.g.U) {
      k.u = first;
      k.gi = 0;
      k.c = 0;
      k.nch = k.kind == PH_ATT ? 1 : k.g.K / KC;
      k.valid = true;
      return;
    }
    k.off = (k.off + k.g.U) % G;
    if (k.kind == PH_HEAD) break;
    if (++k.kind == PH_PER_LAYER) {
      k.kind = 0;
      if (++k.l == a.L) k.kind = PH_HEAD;
    }
  }
  k.valid = false;
}

template <int KC>
__device__ void cursor_init(const PersistArgs& a, Cursor& k, const AttGeo& at) {
  k.l = 0;
  k.kind = a.L > 0 ? 0 : PH_HEAD;
  k.off = 0;
  cursor_seek<KC>(a, k, at);
}

template <int KC>
__device__ void cursor_next(const PersistArgs& a, Cursor& k, const AttGeo& at) {
  if (++k.c < k.nch) return;
  k.c = 0;
  if (++k.gi < k.g.gpu) return;
  k.gi = 0;
  k.u += gridDim.x;
  if (k.u < k.g.U) return;
  k.off = (k.off + k.g.U) % gridDim.x;
  if (k.kind == PH_HEAD) {
    k.valid = false;
    return;
  }
  if (++k.kind == PH_PER_LAYER) {
    k.kind = 0;
    if (++k.l == a.L) k.kind = PH_HEAD;
  }
  cursor_seek<KC>(a, k, at);
}

__device__ __forceinline__ int cursor_phase(const PersistArgs& a, const Cursor& k) {
  return k.kind == PH_HEAD ? a.L * PH_PER_LAYER : k.l * PH_PER_LAYER + k.kind;
}

// Streams this CTA's stages into the shared-memory ring (about 100 KB in flight per SM
// already saturates HBM; deeper L2 prefetching measured slower).
template <int KC>
__device__ void produce(const PersistArgs& a, const Smem& sm, int nst, const AttGeo& at) {
  Cursor cp;
  cursor_init<KC>(a, cp, at);
  int s = 0, last_phase = -1;
  bool ok = true;
  while (cp.valid && ok) {
    const int slot = s % nst;
    if (s >= nst) {
      const uint32_t par = ((s / nst) - 1) & 1;
      if (!mbar_try_wait(&sm.empty[slot], par)) {
        const long long t0 = clock64();
        while (true) {
          if (sm.flags[0]) {
            ok = false;
            break;
          }
          if (mbar_try_wait(&sm.empty[slot], par)) break;
          if (clock64() - t0 > kWaitLimitCycles) {
            record_error(a.err, VX_DEVICE_ERR_TIMEOUT);
            sm.flags[3] = 1;
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
    }
    const int ph = cursor_phase(a, cp);
    if (ph != last_phase) {
      if (last_phase >= 0) trace_mark(a, last_phase, 4);
      trace_mark(a, ph, 3);
      last_phase = ph;
    }
    uint16_t* dst = sm.ring + (size_t)slot * PK_ROWS * KC;
    if (cp.kind == PH_ATT) {
      // K/V rows of positions [j0, min(j1, pos)) of one KV head (the current position's row is
      // written during this launch and read by the consumers after the dependency wait)
      const int g = cp.u / at.nsplit, sp = cp.u % at.nsplit;
      const int j0 = sp * at.span, j1 = min(at.len, j0 + at.span);
      const int nold = max(0, min(j1, at.pos) - j0);
      const uint32_t bytes = (uint32_t)nold * a.d * 4;
      if (bytes == 0) {
        mbar_arrive(&sm.full[slot]);
      } else {
        const size_t base = (size_t)cp.l * a.kv_layer_stride + ((size_t)g * a.s_max + j0) * a.d;
        mbar_arrive_expect_tx(&sm.full[slot], 2 * bytes);
        bulk_g2s(dst, a.kcache + base, bytes, &sm.full[slot]);
        bulk_g2s(reinterpret_cast<float*>(dst) + (size_t)at.span * a.d, a.vcache + base, bytes, &sm.full[slot]);
      }
    } else {
      const int row0 = unit_row(a, cp.kind, cp.u, cp.gi);
      mbar_arrive_expect_tx(&sm.full[slot], PK_ROWS * KC * 2);
      if (cp.nch == 1) {
        bulk_g2s(dst, cp.g.W + (size_t)row0 * cp.g.K, PK_ROWS * KC * 2, &sm.full[slot]);
      } else {
        for (int r = 0; r < PK_ROWS; ++r)
          bulk_g2s(dst + r * KC, cp.g.W + (size_t)(row0 + r) * cp.g.K + (size_t)cp.c * KC, KC * 2, &sm.full[slot]);
      }
    }
    ++s;
    cursor_next<KC>(a, cp, at);
  }
  if (last_phase >= 0) trace_mark(a, last_phase, 4);
  // Do not leave while a copy into this CTA's shared memory may still be in flight.
  for (int i = (s > nst ? s - nst : 0); i < s; ++i) {
    const long long t0 = clock64();
    while (!mbar_try_wait(&sm.full[i % nst], (i / nst) & 1))
      if (clock64() - t0 > kWaitLimitCycles) break;
  }
}

// ---------------------------------------------------------------- consumer warps

// x (f32 [K], produced in this launch or the previous one) -> xs, optionally RMS-normalised
// exactly as MiniCpmRmsNorm::forward (src/minicpm4/mod.rs:62-67).  With a norm, x and the
// norm weight are fetched in one round trip and held in registers (K <= 4096).
__device__ void load_x(const float* x, const float* norm_w, int K, float eps, const Smem& sm) {
  const int tid = threadIdx.x;
  if (norm_w == nullptr) {
#pragma unroll 4
    for (int k = tid * 4; k < K; k += PK_CTHREADS * 4) *reinterpret_cast<float4*>(sm.xs + k) = ldcg4(x + k);
    csync();
    return;
  }
  float4 v[PK_XREG], w[PK_XREG];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PK_XREG; ++i) {
    const int k = (tid + i * PK_CTHREADS) * 4;
    if (k < K) {
      v[i] = ldcg4(x + k);
      w[i] = __ldg(reinterpret_cast<const float4*>(norm_w + k));
    }
  }
#pragma unroll
  for (int i = 0; i < PK_XREG; ++i) {
    if ((tid + i * PK_CTHREADS) * 4 < K) {
      ss = fmaf(v[i].x, v[i].x, ss);
      ss = fmaf(v[i].y, v[i].y, ss);
      ss = fmaf(v[i].z, v[i].z, ss);
      ss = fmaf(v[i].w, v[i].w, ss);
    }
  }
  ss = group_sum(ss, sm.red, PK_CWARPS, 1);
  const float inv = 1.0f / sqrtf(ss / (float)K + eps);
#pragma unroll
  for (int i = 0; i < PK_XREG; ++i) {
    const int k = (tid + i * PK_CTHREADS) * 4;
    if (k < K) {
      float4 o;
      o.x = (v[i].x * inv) * w[i].x;
      o.y = (v[i].y * inv) * w[i].y;
      o.z = (v[i].z * inv) * w[i].z;
      o.w = (v[i].w * inv) * w[i].w;
      *reinterpret_cast<float4*>(sm.xs + k) = o;
    }
  }
  csync();
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// One attention unit, K/V rows in ring slot `kv` (K [span][D] then V [span][D]): query heads
// g*8..g*8+7 against positions [j0, j1) (attention.rs:129-150 for one split).  Warp r is query
// head r, lane j scores position j0 + j (dims visited in a lane-rotated order so the row-per-
// lane reads hit distinct banks).  Writes the normalised output directly when there is one
// split, else the (o, m, l) partial; the last split to finish merges them.  Returns false if
// the CTA must stop.
template <int D>
__device__ bool att_unit(const PersistArgs& a, const AttGeo& at, int l, int u, float* kv, bool lbad, const Smem& sm) {
  constexpr int NC = D / 4, DPL = D / 32, NREP = 8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = u / at.nsplit, sp = u % at.nsplit;
  const int j0 = sp * at.span, j1 = min(at.len, j0 + at.span), nt = j1 - j0;
  float* Ks = kv;
  float* Vs = kv + (size_t)at.span * D;
  float* qs = sm.xs;  // [8][D]
  // post-RoPE queries of this KV head's 8 query heads, and the current position's K/V row
  for (int i = tid; i < NREP * NC; i += PK_CTHREADS)
    *reinterpret_cast<float4*>(qs + i * 4) = ldcg4(a.q + (size_t)g * NREP * D + i * 4);
  if (at.pos >= j0 && at.pos < j1 && tid < 2 * NC) {
    const size_t src = (size_t)l * a.kv_layer_stride + ((size_t)g * a.s_max + at.pos) * D;
    const int c = tid % NC;
    float* dst = (tid < NC ? Ks : Vs) + (size_t)(at.pos - j0) * D + c * 4;
    *reinterpret_cast<float4*>(dst) = ldcg4((tid < NC ? a.kcache : a.vcache) + src + c * 4);
    // the slot is refilled by bulk copies (async proxy) once released
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (sync_or(lbad)) return false;
  // scores q.k^T * scale (attention.rs:166)
  float sc = 0.f;
  if (lane < nt) {
    const float* kr = Ks + (size_t)lane * D;
    const float* qr = qs + warp * D;
#pragma unroll 8
    for (int ch = 0; ch < NC; ++ch) {
      const int c = (ch + lane) & (NC - 1);
      const float4 kk = *reinterpret_cast<const float4*>(kr + c * 4);
      const float4 qq = *reinterpret_cast<const float4*>(qr + c * 4);
      sc = fmaf(qq.x, kk.x, sc);
      sc = fmaf(qq.y, kk.y, sc);
      sc = fmaf(qq.z, kk.z, sc);
      sc = fmaf(qq.w, kk.w, sc);
    }
  }
  const bool valid = lane < nt;
  const float sv = valid ? sc * a.attn_scale : -INFINITY;
  const float m = warp_max(sv);
  const float p = valid ? expf(sv - m) : 0.f;
  const float lsum = warp_sum(p);
  float o[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) o[e] = 0.f;
  for (int j = 0; j < nt; ++j) {
    const float pj = __shfl_sync(0xffffffffu, p, j);
    const float* vr = Vs + (size_t)j * D + lane * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[e] = fmaf(pj, vr[e], o[e]);
  }
  __syncwarp();
  float* outp = a.attn + (size_t)(g * NREP + warp) * D + lane * DPL;
  if (at.nsplit == 1) {
#pragma unroll
    for (int e = 0; e < DPL; ++e) outp[e] = o[e] / lsum;
    return true;
  }
  float* pp = a.att_part + (((size_t)g * at.ns_max + sp) * NREP + warp) * (D + 2);
#pragma unroll
  for (int e = 0; e < DPL; ++e) pp[lane * DPL + e] = o[e];
  if (lane == 0) {
    pp[D] = m;
    pp[D + 1] = lsum;
  }
  csync();
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&a.att_cnt[g], 1u);
    sm.flags[1] = (prev == (unsigned)at.nsplit - 1) ? 1 : 0;
  }
  csync();
  if (!sm.flags[1]) return true;
  __threadfence();
  // last split: merge the nsplit partials of head `warp` (m, l staged in shared memory)
  const float* pb = a.att_part + ((size_t)g * at.ns_max * NREP + warp) * (D + 2);
  const size_t sstride = (size_t)NREP * (D + 2);
  float* fm = sm.xs + NREP * D + (size_t)warp * 2 * at.ns_max;
  float M = -INFINITY;
  for (int q = lane; q < at.nsplit; q += 32) {
    const float mq = __ldcg(pb + q * sstride + D);
    fm[q] = mq;
    fm[at.ns_max + q] = __ldcg(pb + q * sstride + D + 1);
    M = fmaxf(M, mq);
  }
  M = warp_max(M);
  float Ls = 0.f;
  for (int q = lane; q < at.nsplit; q += 32) {
    const float f = expf(fm[q] - M);
    fm[q] = f;
    Ls = fmaf(f, fm[at.ns_max + q], Ls);
  }
  Ls = warp_sum(Ls);
  __syncwarp();
  float acc[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
#pragma unroll 4
  for (int q = 0; q < at.nsplit; ++q) {
    const float f = fm[q];
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] = fmaf(f, __ldcg(pb + q * sstride + lane * DPL + e), acc[e]);
  }
#pragma unroll
  for (int e = 0; e < DPL; ++e) outp[e] = acc[e] / Ls;
  if (tid == 0) a.att_cnt[g] = 0u;
  return true;
}

// Consumer state carried across phases (returned by value from the out-of-line phase bodies).
struct CState {
  int s;    // ring stages consumed
  int bad;  // the step must stop
};

// This CTA's units of one GEMV phase (after its dependency is met): x -> xs (optional RMSNorm),
// then the streamed dot products.  Warp w owns row w of every 8-row group, so each warp
// applies its rows' epilogue itself (its rotate_half partner and its matching up row come from
// the same warp) and the warps run through the ring independently: no CTA barrier per unit.
// Shared by every phase kind from one call site, so one copy of the streaming loop stays hot
// in the instruction cache.
template <int KC>
__device__ __forceinline__ CState gemv_units(const PersistArgs& a, const Smem& sm, CState st, int nst, int kind, int l,
                                          int pos, int U, int K, int gpu, int first, const float* xsrc,
                                          const float* norm_w, const float* resid) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  // residual of this warp's row in each of its first PK_RES_UNITS units, fetched together
  // with x (one round trip) so the epilogues never wait on memory
  float resv[PK_RES_UNITS];
#pragma unroll
  for (int k = 0; k < PK_RES_UNITS; ++k) {
    const int u = first + k * G;
    resv[k] = (resid != nullptr && lane == 0 && u < U) ? __ldcg(resid + (size_t)u * PK_ROWS + warp) : 0.f;
  }
  load_x(xsrc, norm_w, K, a.eps, sm);
  if (tid == 0) trace_mark(a, kind == PH_HEAD ? a.L * PH_PER_LAYER : l * PH_PER_LAYER + kind, 1);
  constexpr int NJ = KC / 256;
  float xr[NJ * 8];
  const int nch = K / KC;
  bool lbad = false, first_stage = true;
  float bv = -FLT_MAX;  // head: this warp's running argmax
  int bi = INT_MAX;
  int k = 0;
  for (int u = first; u < U; u += G, ++k) {
    float t[2] = {0.f, 0.f};
    for (int gi = 0; gi < gpu; ++gi) {
      float acc0 = 0.f, acc1 = 0.f;
      for (int c = 0; c < nch; ++c) {
        if (nch > 1 || first_stage) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const float4 v0 = *reinterpret_cast<const float4*>(sm.xs + c * KC + j * 256 + lane * 8);
            const float4 v1 = *reinterpret_cast<const float4*>(sm.xs + c * KC + j * 256 + lane * 8 + 4);
            xr[j * 8 + 0] = v0.x; xr[j * 8 + 1] = v0.y; xr[j * 8 + 2] = v0.z; xr[j * 8 + 3] = v0.w;
            xr[j * 8 + 4] = v1.x; xr[j * 8 + 5] = v1.y; xr[j * 8 + 6] = v1.z; xr[j * 8 + 7] = v1.w;
          }
          first_stage = false;
        }
        const int slot = st.s % nst;
        if (!lbad && !wait_full(&sm.full[slot], (st.s / nst) & 1, a.err, sm.flags)) lbad = true;
        if (tid == 0 && k == 0 && gi == 0 && c == 0)
          trace_mark(a, kind == PH_HEAD ? a.L * PH_PER_LAYER : l * PH_PER_LAYER + kind, 6);
        if (!lbad) {
          const uint4* wr = reinterpret_cast<const uint4*>(sm.ring + (size_t)slot * PK_ROWS * KC + warp * KC);
#pragma unroll
          for (int j = 0; j < NJ; j += 2) {
            acc0 = dot8(wr[j * 32 + lane], &xr[j * 8], acc0);
            if (j + 1 < NJ) acc1 = dot8(wr[(j + 1) * 32 + lane], &xr[(j + 1) * 8], acc1);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        ++st.s;
      }
      t[gi] = warp_sum(acc0 + acc1);
    }
    if (tid == 0 && k == 0) trace_mark(a, kind == PH_HEAD ? a.L * PH_PER_LAYER : l * PH_PER_LAYER + kind, 7);
    // ---- this warp's row epilogue (lane 0)
    if (lbad || lane != 0) continue;
    const int row = unit_row(a, kind, u, 0) + warp;
    if (kind == PH_HEAD) {
      if (a.logits) a.logits[row] = t[0];
      if (better(t[0], row, bv, bi)) {
        bv = t[0];
        bi = row;
      }
    } else if (kind == PH_Q) {
      // LongRoPE on q/k rows (rope.rs:76-95), post-RoPE k and v into the cache at `pos`
      const int head = row / a.d, ii = row % a.d, half = a.d / 2;
      const float ya = t[0], yb = t[1];
      float oa = ya, ob = yb;
      if (head < a.nh + a.nkv && a.rope != nullptr) {
        const float c = sm.ctab[ii], sn = sm.stab[ii];
        oa = __fadd_rn(__fmul_rn(ya, c), __fmul_rn(-yb, sn));
        ob = __fadd_rn(__fmul_rn(yb, c), __fmul_rn(ya, sn));
      }
      if (head < a.nh) {
        a.q[head * a.d + ii] = oa;
        a.q[head * a.d + ii + half] = ob;
      } else {
        const bool isk = head < a.nh + a.nkv;
        float* dst = (isk ? a.kcache : a.vcache) + (size_t)l * a.kv_layer_stride +
                     ((size_t)(head - a.nh - (isk ? 0 : a.nkv)) * a.s_max + pos) * a.d;
        dst[ii] = isk ? oa : ya;
        dst[ii + half] = isk ? ob : yb;
      }
    } else if (kind == PH_GU) {
      a.act[row] = silu(t[0]) * t[1];  // mlp.rs:31-33
    } else {
      // o_proj / down_proj + residual (layer.rs:33-38): x1 = x0 + s*o, x0 = x1 + s*down
      float r = 0.f;
#pragma unroll
      for (int q = 0; q < PK_RES_UNITS; ++q)
        if (q == k) r = resv[q];
      if (k >= PK_RES_UNITS) r = __ldcg(resid + row);
      (kind == PH_O ? a.x1 : a.x0)[row] = r + t[0] * a.res_scale;
    }
  }
  if (kind == PH_HEAD && lane == 0) {
    sm.red[16 + warp] = bv;
    reinterpret_cast<int*>(sm.red)[24 + warp] = bi;
  }
  if (sync_or(lbad)) st.bad = 1;
  if (kind == PH_HEAD && tid == 0) {  // CTA best over the warps (ties -> lowest id)
    for (int w = 0; w < PK_CWARPS; ++w) {
      const float v = sm.red[16 + w];
      const int i = reinterpret_cast<int*>(sm.red)[24 + w];
      if (better(v, i, sm.red[48], reinterpret_cast<int*>(sm.red)[49])) {
        sm.red[48] = v;
        reinterpret_cast<int*>(sm.red)[49] = i;
      }
    }
  }
  return st;
}

// This CTA's attention units of layer l (after the Q phase is published).
template <int KC, int D>
__device__ __forceinline__ CState att_units(const PersistArgs& a, const Smem& sm, CState st, int nst, const AttGeo& at,
                                         int l, int first) {
  const int lane = threadIdx.x & 31;
  for (int u = first; u < at.items; u += gridDim.x) {
    const int slot = st.s % nst;
    const bool lbad = !wait_full(&sm.full[slot], (st.s / nst) & 1, a.err, sm.flags);
    float* kv = reinterpret_cast<float*>(sm.ring + (size_t)slot * PK_ROWS * KC);
    const bool ok = att_unit<D>(a, at, l, u, kv, lbad, sm);
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
    ++st.s;
    csync();  // xs (queries, merge scratch) reused by the next unit
    if (!ok) {
      st.bad = 1;
      break;
    }
  }
  return st;
}

template <int KC, int D>
__global__ void __launch_bounds__(PK_THREADS, 1) persist_decode_kernel(const PersistArgs a, int nst, int xs_floats,
                                                                        int att_span) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem sm;
  sm.ring = reinterpret_cast<uint16_t*>(smem_raw);
  sm.xs = reinterpret_cast<float*>(smem_raw + (size_t)nst * PK_ROWS * KC * 2);
  sm.ctab = sm.xs + xs_floats;
  sm.stab = sm.ctab + 64;
  sm.red = sm.stab + 64;
  sm.flags = reinterpret_cast<volatile int*>(sm.red + 64);
  sm.full = reinterpret_cast<uint64_t*>(sm.red + 64 + 8);
  sm.empty = sm.full + nst;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x;
  AttGeo at;
  at.pos = *a.pos;  // position of the token being decoded (advanced by this launch)
  at.len = at.pos + 1;
  at.span = att_span;
  at.nsplit = (at.len + att_span - 1) / att_span;
  at.ns_max = (a.s_max + att_span - 1) / att_span;
  at.items = a.nkv * at.nsplit;
  const int pos = at.pos;

  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], PK_CWARPS);
    }
    for (int i = 0; i < 8; ++i) sm.flags[i] = 0;
    sm.red[48] = -FLT_MAX;  // running argmax of the head (value, index)
    reinterpret_cast<int*>(sm.red)[49] = INT_MAX;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == PK_CWARPS) {
    if (lane == 0) produce<KC>(a, sm, nst, at);
    return;
  }

  // LongRoPE angles of this position, formed in f64 as MiniCpmLongRope::new does
  // (src/minicpm4/rope.rs:38-46) and rounded to f32.
  if (a.rope != nullptr && tid < a.d / 2) {
    const double f = ((double)pos * a.rope->inv_freq[tid]) / a.rope->ext[tid];
    double sd, cd;
    sincos(f, &sd, &cd);
    sm.ctab[tid] = (float)(cd * a.rope->scaling_factor);
    sm.stab[tid] = (float)(sd * a.rope->scaling_factor);
  }

  CState st = {0, 0};
  int off = 0;
  const unsigned* prev_cnt = nullptr;
  unsigned prev_target = 0;
  const int nphase = a.L * PH_PER_LAYER + 1;
  for (int ph = 0; ph < nphase && !st.bad; ++ph) {
    const bool head = ph == nphase - 1;
    const int l = head ? a.L : ph / PH_PER_LAYER;
    const int kind = head ? PH_HEAD : ph % PH_PER_LAYER;
    const Geo g = geo_of(a, l, kind, at);
    unsigned* cnt = a.phase_cnt + ph;
    const int first = first_unit(off, G);
    if (first < g.U) {
      if (tid == 0) trace_mark(a, ph, 0);
      if (prev_cnt != nullptr && !dep_wait(prev_cnt, prev_target, a.err, false)) {
        st.bad = 1;
        break;
      }
      if (kind == PH_ATT) {
        if (tid == 0) trace_mark(a, ph, 1);
        st = att_units<KC, D>(a, sm, st, nst, at, l, first);
      } else {
        const PersistLayer* w = a.layers + (l < a.L ? l : 0);
        const float* xsrc = kind == PH_O ? a.attn : kind == PH_GU ? a.x1 : kind == PH_D ? a.act : a.x0;
        const float* norm_w = kind == PH_Q ? w->ln_in : kind == PH_GU ? w->ln_post : head ? a.final_norm : nullptr;
        const float* resid = kind == PH_O ? a.x0 : kind == PH_D ? a.x1 : nullptr;
        st = gemv_units<KC>(a, sm, st, nst, kind, l, pos, g.U, g.K, g.gpu, first, xsrc, norm_w, resid);
      }
      if (tid == 0) trace_mark(a, ph, 5);
      if (st.bad) break;
      if (!head) {
        arrive(cnt);
        if (tid == 0) trace_mark(a, ph, 2);
      }
    }
    prev_cnt = cnt;
    prev_target = (unsigned)min(g.U, G);
    off = (off + g.U) % G;
  }

  // ---- greedy head reduction: per-CTA best -> am_part, last CTA picks the token, writes the
  // next input embedding and advances position and step
  if (!st.bad) {
    const int U = a.V / PK_ROWS;
    const int off_h = (off - U % G + G) % G;  // the head phase's offset
    const int fh = first_unit(off_h, G);
    if (fh < U) {
      csync();
      if (fh == 0)  // owner of unit 0 publishes the final-norm hidden (still in xs)
        for (int k = tid * 4; k < a.H; k += PK_CTHREADS * 4)
          *reinterpret_cast<float4*>(a.hid_norm + k) = *reinterpret_cast<const float4*>(sm.xs + k);
      unsigned* hcnt = a.phase_cnt + (size_t)a.L * PH_PER_LAYER;
      if (tid == 0) {
        a.am_part[blockIdx.x] = make_float2(sm.red[48], __int_as_float(reinterpret_cast<int*>(sm.red)[49]));
        __threadfence();
        const unsigned prev = atomicAdd(hcnt, 1u);
        sm.flags[1] = (prev == (unsigned)min(U, G) - 1) ? 1 : 0;
        trace_mark(a, a.L * PH_PER_LAYER, 2);
      }
      csync();
      if (sm.flags[1]) {
        __threadfence();
        const int nparts = min(U, G);
        float rv = -FLT_MAX;
        int ri = INT_MAX;
        for (int i = tid; i < nparts; i += PK_CTHREADS) {
          const float2 p = __ldcg(&a.am_part[(off_h + i) % G]);
          const int pi = __float_as_int(p.y);
          if (better(p.x, pi, rv, ri)) {
            rv = p.x;
            ri = pi;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, rv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, ri, o);
          if (better(ov, oi, rv, ri)) {
            rv = ov;
            ri = oi;
          }
        }
        int* redi = reinterpret_cast<int*>(sm.red + 32);
        if (lane == 0) {
          sm.red[warp] = rv;
          redi[warp] = ri;
        }
        csync();
        if (tid == 0) {
          for (int w2 = 0; w2 < PK_CWARPS; ++w2)
            if (better(sm.red[w2], redi[w2], rv, ri)) {
              rv = sm.red[w2];
              ri = redi[w2];
            }
          if (ri < 0 || ri >= a.V) ri = 0;
          const int slot = *a.step;
          a.tokens[slot] = ri;
          *a.step = slot + 1;
          *a.pos = pos + 1;
          sm.flags[2] = ri;
        }
        csync();
        // next input = embed(tok) * scale_emb (src/minicpm4/model.rs:87-92, voxcpm2/model.rs:145)
        const uint16_t* e = a.embed + (size_t)sm.flags[2] * a.H;
        for (int k = tid; k < a.H; k += PK_CTHREADS) a.x0[k] = __uint_as_float(((uint32_t)e[k]) << 16) * a.emb_scale;
      }
    }
  }

  // Leave: stop the producer if this CTA gave up; the last CTA out zeroes the counters.
  if (st.bad) {
    if (tid == 0) sm.flags[0] = 1;
    return;
  }
  if (tid == 0) {
    const int nc = a.L * PH_PER_LAYER + 2;
    __threadfence();
    const unsigned prev = atomicAdd(a.phase_cnt + nc - 1, 1u);
    if (prev == (unsigned)G - 1) {
      for (int i = 0; i < nc; ++i) a.phase_cnt[i] = 0u;
      __threadfence();
    }
  }
}

int pick_kc(int H, int I, int qd) {
  for (int kc : {2048, 1024, 512, 256})
    if (H % kc == 0 && I % kc == 0 && qd % kc == 0) return kc;
  return 0;
}

struct PkShape {
  int kc = 0, d = 0, xs_floats = 0, nst = 0, span = 0;
  size_t smem = 0;
};

PkShape shape_of(int H, int I, int nh, int d, int s_max, int nst_cap) {
  PkShape p;
  p.kc = pick_kc(H, I, nh * d);
  p.d = d;
  if (!p.kc || d <= 0) return p;
  p.span = std::min(32, 2 * p.kc / d);  // K and V rows of `span` positions fill one ring stage
  const int ns_max = (s_max + p.span - 1) / p.span;
  const int m = std::max(std::max(H, I), std::max(nh * d, 8 * d + 16 * ns_max));
  p.xs_floats = (m + 3) & ~3;
  const int fixed = p.xs_floats * 4 + PK_MISC_FLOATS * 4 + 32;
  p.nst = std::min(nst_cap > 1 ? nst_cap : 64, (PK_MAX_SMEM - fixed) / (16 * p.kc + 16));
  p.smem = (size_t)p.nst * 16 * p.kc + fixed + 16 * (size_t)p.nst;
  return p;
}

using KernelFn = void (*)(const PersistArgs, int, int, int);

KernelFn kernel_of(int kc, int d) {
  if (d == 128) {
    switch (kc) {
      case 2048: return persist_decode_kernel<2048, 128>;
      case 1024: return persist_decode_kernel<1024, 128>;
      case 512: return persist_decode_kernel<512, 128>;
      case 256: return persist_decode_kernel<256, 128>;
    }
  } else if (d == 64) {
    switch (kc) {
      case 2048: return persist_decode_kernel<2048, 64>;
      case 1024: return persist_decode_kernel<1024, 64>;
      case 512: return persist_decode_kernel<512, 64>;
      case 256: return persist_decode_kernel<256, 64>;
    }
  }
  return nullptr;
}

}  // namespace

bool persist_supported(int H, int I, int nh, int nkv, int d, int V, int s_max) {
  if (nkv <= 0 || nh != 8 * nkv || (d != 64 && d != 128) || V <= 0 || V % PK_ROWS != 0 || s_max <= 0) return false;
  if (H > PK_XREG * PK_CTHREADS * 4) return false;  // normalised inputs are [H]
  const PkShape p = shape_of(H, I, nh, d, s_max, 0);
  return p.kc != 0 && p.nst >= 2 && p.span >= 1;
}

size_t persist_att_part_floats(int nkv, int nh, int d, int H, int I, int s_max) {
  const PkShape p = shape_of(H, I, nh, d, s_max, 0);
  if (!p.span) return 0;
  return (size_t)nkv * ((s_max + p.span - 1) / p.span) * (nh / nkv) * (d + 2);
}

int persist_configure(int H, int I, int nh, int nkv, int d, int s_max, int nst_cap) {
  (void)nkv;
  const PkShape p = shape_of(H, I, nh, d, s_max, nst_cap);
  KernelFn fn = kernel_of(p.kc, d);
  if (!fn || p.nst < 2) return 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, PK_THREADS, p.smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (per_sm < 1) return 0;
  return std::min(sms, 4096);  // one CTA per SM (am_part holds 4096 partials)
}

cudaError_t launch_persist(const PersistArgs& a, int grid, int nst_cap, cudaStream_t st, bool cooperative) {
  const PkShape p = shape_of(a.H, a.I, a.nh, a.d, a.s_max, nst_cap);
  KernelFn fn = kernel_of(p.kc, a.d);
  if (!fn || grid <= 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(PK_THREADS);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cooperative ? 1 : 0;
  count_launch();
  return cudaLaunchKernelEx(&cfg, fn, a, p.nst, p.xs_floats, p.span);
}

}  // namespace vx
