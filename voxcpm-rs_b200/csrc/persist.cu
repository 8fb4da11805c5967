// Persistent batch-1 decode step (sm_100a): ONE launch per token runs every decoder layer
// and the greedy head (reference MiniCpmModel::forward_step, src/minicpm4/model.rs:64-84).
//
// Why: a per-kernel decode step is several launches per layer; each streams a few MB of
// weights and loses microseconds to its pipeline ramp and tail.  Here one CTA per SM stays
// resident for the whole token and its producer warp streams ALL of that CTA's operand tiles,
// phase after phase, through one shared-memory ring with 1-D bulk copies (the TMA engine).
// Weights never depend on activations, and neither do the KV-cache rows of earlier
// positions, so while the consumer warps wait for the previous phase's result the producer
// already fills the ring with the next phase's tiles.  Every stage is ONE 32 KB bulk copy
// (the TMA engine issues a bounded number of copies per SM per second, so smaller pieces
// would cap the stream below the HBM rate).
//
// Phases per layer (the unit a CTA owns; units spread round-robin with a rotating offset so
// every CTA streams about the same bytes per token):
//   Q    input RMSNorm -> qkv_proj rows -> LongRoPE -> q buffer, k/v into the static cache
//        (layer.rs:64-66, attention.rs:102-127); unit = a rotate_half pair of 8-row groups
//        of the q / k heads, then 8 v rows
//   ATT  flash-decode over the cached prefix (attention.rs:129-150, 156-204); unit = one KV
//        head's 8 query heads against a run of 32-position tiles whose K/V rows arrive
//        through the ring (the current position's row, written by Q, is read after the
//        wait); warp = query head, its lanes split the head's dims and a butterfly
//        reduce-scatter gives lane j position j's score; each unit leaves its online-softmax
//        partial (o, max, sum) in global memory.  Caches of more than merge_tiles tiles (16
//        by default) get a unit per tile (up to 64 per KV head) and the last unit of a KV
//        head to finish merges its partials into the attention output.
//   O    the attention output (short caches: every CTA merges the <= 8 partials per KV head
//        itself from one bulk copy) -> o_proj + residual into x1 (attention.rs:153,
//        layer.rs:67); unit = 8 rows.  Also seeds the next layer's residual accumulator
//        with x1 (fixed point, below).
//   M    post-attention RMSNorm -> gate|up rows -> silu(gate)*up -> down_proj (mlp.rs:28-34,
//        layer.rs:69-72); unit = 8 MLP channels j: their gate row, up row and down column
//        (a row of the transposed down weight).  Each warp accumulates its slice of the
//        2048 outputs across the CTA's units; at the end of the phase the CTA adds
//        res_scale * its partial into the next layer's residual accumulator with one bulk
//        integer reduce-add.  Fusing the down projection removes a dependency round trip
//        per layer.
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
// Every GEMV output row is summed in a fixed order: each lane's run of KC/256 products, the
// lane butterfly within a warp, then the 8 warps' K slices in warp order.  The per-kernel
// step's GEMV sums in another order, so the two agree to rounding, not bit for bit.  The down
// projection's CTA partials arrive in any order, so the residual stream of layers 1..L is
// kept in fixed point (x * 2^32 in int64; |x| < 2^31 / grid): each partial is rounded once
// to that grid and the integer sum is exact, hence independent of the arrival order, and
// readers convert it back to f32 with one rounding.  The whole step is deterministic: the
// same inputs give the same bits, run after run.
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
constexpr int PK_MAX_LAYERS = 64;                  // layer-table entries held in shared memory
constexpr int PK_MAX_SMEM = 232448 - PK_MAX_LAYERS * (int)sizeof(PersistLayer);  // 227 KB per CTA, less the table
constexpr int PK_KP_FLOATS = 2 * 2 * PK_ROWS * PK_CWARPS;  // per-warp row partials: 2 units x 2 row groups
constexpr int PK_MISC_FLOATS = 64 + 64 + 64 + PK_KP_FLOATS;  // rope tables, reduction scratch, row partials
constexpr int PK_RES_UNITS = 4;                    // residual rows preloaded per warp and phase
constexpr int NREP = 8;                            // query heads per KV head

enum { PH_Q = 0, PH_ATT = 1, PH_O = 2, PH_M = 3, PH_PER_LAYER = PERSIST_PHASES_PER_LAYER, PH_HEAD = 4 };
static_assert(PH_PER_LAYER == 4, "phase kinds per layer");

// The layer table, copied from a.layers at kernel start: the producer looks up weight
// pointers at every phase change, and a global load there (about 1 us under a saturated HBM)
// would stall the copy stream.
__shared__ PersistLayer s_lay[PK_MAX_LAYERS];

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

// Fixed point of the residual accumulators: value x 2^32 in int64.
__device__ __forceinline__ long long to_fix(float v) { return __float2ll_rn(v * 4294967296.0f); }
__device__ __forceinline__ float from_fix(long long v) { return __ll2float_rn(v) * 2.3283064365386963e-10f; }

// The input of layer l (layer L: the head's input): layer 0 reads the f32 embedding buffer,
// later layers the fixed-point accumulator the previous layer's O and M phases wrote.
struct XIn {
  const float* f;
  const long long* i;
};
__device__ __forceinline__ XIn xin_of(const PersistArgs& a, int l) {
  return l == 0 ? XIn{a.x0, nullptr} : XIn{nullptr, a.xacc + (size_t)(l & 1) * a.H};
}
__device__ __forceinline__ float4 ldx4(const XIn& x, int k) {
  if (x.i == nullptr) return __ldcg(reinterpret_cast<const float4*>(x.f + k));
  const longlong2 p = __ldcg(reinterpret_cast<const longlong2*>(x.i + k));
  const longlong2 q = __ldcg(reinterpret_cast<const longlong2*>(x.i + k + 2));
  return make_float4(from_fix(p.x), from_fix(p.y), from_fix(q.x), from_fix(q.y));
}
__device__ __forceinline__ float ldx1(const XIn& x, int k) {
  return x.i == nullptr ? __ldcg(x.f + k) : from_fix(__ldcg(x.i + k));
}

// flags[0]: consumers stopped (producer must stop too); flags[1]: last-arrival broadcast;
// flags[2]: picked token broadcast; flags[3]: producer gave up.
struct Smem {
  uint16_t* ring;
  float* xs;
  float* parts;  // attention split partials of one layer, as in att_part
  float* ctab;  // [64]
  float* stab;  // [64]
  float* red;   // [64]: [0,8) group sums / merge, [16,32) per-warp argmax, [48,50) CTA argmax
  float* kp;    // [2][2][PK_ROWS][PK_CWARPS]: each warp's K-slice sums of a unit's rows (row
                // group, row, warp), double-buffered by unit parity
  volatile int* flags;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* pbar;  // completion of the partials' bulk copies
};

// Attention geometry of this launch, the same in every CTA: `ntiles` tiles of `span`
// positions cover [0, len); split sp of a KV head covers tiles [sp*tps, (sp+1)*tps).
struct AttGeo {
  int pos, len, span, ntiles, nsplit, tps, items;
  bool merge_once;  // the last split of a KV head merges its splits (else every o_proj CTA does)
};

__device__ __forceinline__ int att_tiles(const AttGeo& at, int u) {
  const int t0 = (u % at.nsplit) * at.tps;
  return min(at.ntiles, t0 + at.tps) - t0;
}

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

// Publish this CTA's completion of a phase (after all its stores and reductions).
__device__ __forceinline__ void arrive(unsigned* cnt) {
  csync();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
}

struct Geo {
  const uint16_t* W;
  int K;
  int U;    // units in the phase
  int gpu;  // 8-row groups per unit (attention: tiles per split)
  int kind;
};

// Q phase: units [0, q_pair_units) are rotate_half pairs of 8-row groups of the q and k
// heads (two stages each); the v rows follow as plain 8-row units (one stage each), so the
// phase's 2.16 stages per CTA spread as at most 3 instead of two whole pair units (4).
__device__ __forceinline__ int q_pair_units(const PersistArgs& a) { return (a.nh + a.nkv) * a.d / 16; }

__device__ __forceinline__ int unit_row(const PersistArgs& a, int kind, int u, int gi) {
  if (kind == PH_Q) {  // rotate_half pair: rows j*8.. of the first and second half of a head
    const int hp = a.d / 16, up = q_pair_units(a);
    if (u >= up) return (a.nh + a.nkv) * a.d + (u - up) * PK_ROWS;
    return (u / hp) * a.d + (u % hp) * PK_ROWS + gi * (a.d / 2);
  }
  if (kind == PH_M) return (gi == 1 ? a.I : 0) + u * PK_ROWS;  // gate rows, up rows, wdt rows
  return u * PK_ROWS;
}

__device__ __forceinline__ Geo geo_of(const PersistArgs& a, int l, int kind, const AttGeo& at) {
  const PersistLayer& w = s_lay[l < a.L ? l : 0];
  switch (kind) {
    case PH_Q: return {w.wqkv, a.H, q_pair_units(a) + a.nkv * a.d / PK_ROWS, 2, PH_Q};
    case PH_ATT: return {nullptr, 0, at.items, at.tps, PH_ATT};
    case PH_O: return {w.wo, a.nh * a.d, a.H / PK_ROWS, 1, PH_O};
    case PH_M: return {w.wgu, a.H, a.I / PK_ROWS, 3, PH_M};
    default: return {a.embed, a.H, a.V / PK_ROWS, 1, PH_HEAD};
  }
}

__device__ __forceinline__ int first_unit(int off, int G) {
  return ((int)blockIdx.x - off % G + G) % G;
}

// ---------------------------------------------------------------- producer warp (lane 0)

// Position in this CTA's stage sequence: phases in order (4 per layer, then the head), this
// CTA's units of each phase, the 8-row groups (or attention tiles) of a unit, the K chunks of
// a group.
struct Cursor {
  int l, kind, off;
  int u, gi, ngi, c, nch;
  Geo g;
  bool valid;
};

__device__ __forceinline__ int unit_groups(const PersistArgs& a, const Cursor& k, const AttGeo& at) {
  if (k.kind == PH_Q && k.u >= q_pair_units(a)) return 1;
  return k.kind == PH_ATT ? att_tiles(at, k.u) : k.g.gpu;
}

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
      k.ngi = unit_groups(a, k, at);
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
  if (++k.gi < k.ngi) return;
  k.gi = 0;
  k.u += gridDim.x;
  if (k.u < k.g.U) {
    k.ngi = unit_groups(a, k, at);
    return;
  }
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

// K/V rows of positions [j0, min(j1, pos)) of tile gi of attention unit u: element offset
// and bytes (the current position's row is written during this launch and patched in by the
// consumers after the dependency wait).
__device__ __forceinline__ uint32_t att_old_rows(const PersistArgs& a, const AttGeo& at, int l, int u, int gi,
                                                 size_t* base) {
  const int g = u / at.nsplit, t = (u % at.nsplit) * at.tps + gi;
  const int j0 = t * at.span, j1 = min(at.len, j0 + at.span);
  const int nold = max(0, min(j1, at.pos) - j0);
  *base = (size_t)l * a.kv_layer_stride + ((size_t)g * a.s_max + j0) * a.d;
  return (uint32_t)nold * a.d * 4;
}


// First row of the 8-row group at cursor k (rows are k.g.K elements apart) plus the chunk.
template <int KC>
__device__ __forceinline__ const uint16_t* group_src(const PersistArgs& a, const Cursor& k) {
  const uint16_t* W = (k.kind == PH_M && k.gi == 2) ? s_lay[k.l].wdt : k.g.W;
  return W + (size_t)unit_row(a, k.kind, k.u, k.gi) * k.g.K + (size_t)k.c * KC;
}

// L2 prefetch of the bytes of the stage at cursor k (nothing lands in shared memory).
template <int KC>
__device__ __forceinline__ void prefetch_stage(const PersistArgs& a, const Cursor& k, const AttGeo& at) {
  if (k.kind == PH_ATT) {
    size_t base;
    const uint32_t bytes = att_old_rows(a, at, k.l, k.u, k.gi, &base);
    if (bytes) {
      bulk_prefetch_l2(a.kcache + base, bytes);
      bulk_prefetch_l2(a.vcache + base, bytes);
    }
  } else {
    const uint16_t* src = group_src<KC>(a, k);
    if (k.nch == 1) {
      bulk_prefetch_l2(src, PK_ROWS * KC * 2);
    } else {
      for (int r = 0; r < PK_ROWS; ++r) bulk_prefetch_l2(src + (size_t)r * k.g.K, KC * 2);
    }
  }
}

// Streams this CTA's stages into the shared-memory ring.  With a.pf_stages > 0 a second
// cursor runs that many stages ahead of the newest ring copy and prefetches them into L2.
template <int KC>
__device__ void produce(const PersistArgs& a, const Smem& sm, int nst, const AttGeo& at) {
  Cursor cp;
  cursor_init<KC>(a, cp, at);
  Cursor cq = cp;  // L2 prefetch cursor, stage index sq
  int sq = 0;
  if (a.pf_stages > 0)
    for (; sq < nst && cq.valid; ++sq) cursor_next<KC>(a, cq, at);  // the first nst stages are copied at once
  const uint64_t pol = a.evict_first ? l2_policy_evict_first() : 0ull;
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
    // Pacing: at most a.inflight copies issued and not yet landed, so the memory system stays
    // near its unloaded latency and the other ring slots hold landed stages that carry the
    // stream through the consumers' pauses (input loads, publish fences, merges).
    if (a.inflight > 0 && s >= a.inflight) {
      const int o = s - a.inflight;
      if (!mbar_try_wait(&sm.full[o % nst], (o / nst) & 1)) {
        const long long t0 = clock64();
        while (true) {
          if (sm.flags[0]) {
            ok = false;
            break;
          }
          if (mbar_try_wait(&sm.full[o % nst], (o / nst) & 1)) break;
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
      size_t base;
      const uint32_t bytes = att_old_rows(a, at, cp.l, cp.u, cp.gi, &base);
      if (bytes == 0) {
        mbar_arrive(&sm.full[slot]);
      } else {
        mbar_arrive_expect_tx(&sm.full[slot], 2 * bytes);
        bulk_g2s(dst, a.kcache + base, bytes, &sm.full[slot]);
        bulk_g2s(reinterpret_cast<float*>(dst) + (size_t)at.span * a.d, a.vcache + base, bytes, &sm.full[slot]);
      }
    } else {
      const uint16_t* src = group_src<KC>(a, cp);
      mbar_arrive_expect_tx(&sm.full[slot], PK_ROWS * KC * 2);
      if (cp.nch == 1) {
        if (a.evict_first)
          bulk_g2s_hint(dst, src, PK_ROWS * KC * 2, &sm.full[slot], pol);
        else
          bulk_g2s(dst, src, PK_ROWS * KC * 2, &sm.full[slot]);
      } else {
        for (int r = 0; r < PK_ROWS; ++r) {
          if (a.evict_first)
            bulk_g2s_hint(dst + r * KC, src + (size_t)r * cp.g.K, KC * 2, &sm.full[slot], pol);
          else
            bulk_g2s(dst + r * KC, src + (size_t)r * cp.g.K, KC * 2, &sm.full[slot]);
        }
      }
    }
    ++s;
    cursor_next<KC>(a, cp, at);
    for (; a.pf_stages > 0 && cq.valid && sq < s + a.pf_stages; ++sq) {
      prefetch_stage<KC>(a, cq, at);
      cursor_next<KC>(a, cq, at);
    }
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
// norm weight are fetched in one round trip and held in registers (K <= KC).
template <int KC>
__device__ void load_x(const PersistArgs& a, int tph, const XIn& x, const float* norm_w, int K, float eps,
                       const Smem& sm) {
  constexpr int PK_XREG = (KC + PK_CTHREADS * 4 - 1) / (PK_CTHREADS * 4);  // float4 per thread
  const int tid = threadIdx.x;
  if (norm_w == nullptr) {
#pragma unroll 4
    for (int k = tid * 4; k < K; k += PK_CTHREADS * 4) *reinterpret_cast<float4*>(sm.xs + k) = ldx4(x, k);
    csync();
    return;
  }
  // the input's two encodings are told apart outside the load loops, and a fixed-point input
  // is converted only after all its loads are in flight, so no conversion waits on one load
  // while the next is still to be issued
  float4 v[PK_XREG], w[PK_XREG];
  float ss = 0.f;
  if (x.i == nullptr) {
#pragma unroll
    for (int i = 0; i < PK_XREG; ++i) {
      const int k = (tid + i * PK_CTHREADS) * 4;
      if (k < K) {
        v[i] = __ldcg(reinterpret_cast<const float4*>(x.f + k));
        w[i] = __ldg(reinterpret_cast<const float4*>(norm_w + k));
      }
    }
  } else {
    longlong2 p[PK_XREG], q[PK_XREG];
#pragma unroll
    for (int i = 0; i < PK_XREG; ++i) {
      const int k = (tid + i * PK_CTHREADS) * 4;
      if (k < K) {
        p[i] = __ldcg(reinterpret_cast<const longlong2*>(x.i + k));
        q[i] = __ldcg(reinterpret_cast<const longlong2*>(x.i + k + 2));
        w[i] = __ldg(reinterpret_cast<const float4*>(norm_w + k));
      }
    }
#pragma unroll
    for (int i = 0; i < PK_XREG; ++i)
      if ((tid + i * PK_CTHREADS) * 4 < K)
        v[i] = make_float4(from_fix(p[i].x), from_fix(p[i].y), from_fix(q[i].x), from_fix(q[i].y));
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
  if (threadIdx.x == 0) trace_mark(a, tph, 7);
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

// The merged attention output and the arrival counters behind the split partials in att_part.
__device__ __forceinline__ float* att_out(const PersistArgs& a, int D) {
  return a.att_part + persist_att_partials_floats(a.nkv, a.nh, D);
}
__device__ __forceinline__ unsigned* att_counters(const PersistArgs& a, int D) {
  return reinterpret_cast<unsigned*>(att_out(a, D) + (size_t)a.nh * D);
}

// Short caches (at most PERSIST_ATT_SPLITS splits per KV head): the attention output [nh*D]
// -> xs in every CTA of the o_proj phase: per query head, the merge of its KV head's split
// partials (o unnormalised, max m, sum l): out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s
// with M the largest m_s (attention.rs:186-191 over the whole prefix).  One bulk copy per KV
// head brings the partials into shared memory (one L2 round trip; they were written by other
// CTAs' generic stores, hence the proxy fence), then the merge reads shared memory only.
// `use` counts this CTA's earlier merges (the parity of sm.pbar).  Returns false on a failed
// wait.
template <int D>
__device__ bool att_merge(const PersistArgs& a, const AttGeo& at, const Smem& sm, int use, int tph) {
  const int nhd = a.nh * D, ns = at.nsplit;
  const size_t gstride = (size_t)PERSIST_ATT_SPLITS * NREP * (D + 4);      // shared floats per KV head
  const size_t gsrc = (size_t)PERSIST_ATT_SPLITS_MAX * NREP * (D + 4);    // global floats per KV head
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    const uint32_t bytes = (uint32_t)(ns * NREP * (D + 4) * 4);
    mbar_arrive_expect_tx(sm.pbar, bytes * a.nkv);
    for (int g = 0; g < a.nkv; ++g) bulk_g2s(sm.parts + g * gstride, a.att_part + g * gsrc, bytes, sm.pbar);
  }
  const bool ok = wait_full(sm.pbar, use & 1, a.err, sm.flags);
  if (threadIdx.x == 0) trace_mark(a, tph, 7);
  if (ok) {
    for (int e = threadIdx.x * 4; e < nhd; e += PK_CTHREADS * 4) {
      const int h = e / D, dd = e % D;
      const float* p0 = sm.parts + (size_t)(h / NREP) * gstride + (size_t)(h % NREP) * (D + 4);
      const size_t ss = (size_t)NREP * (D + 4);
      float M = p0[D];
      for (int sp = 1; sp < ns; ++sp) M = fmaxf(M, p0[sp * ss + D]);
      float Ls = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < ns; ++sp) {
        const float* pp = p0 + sp * ss;
        const float f = expf(pp[D] - M);
        const float4 o = *reinterpret_cast<const float4*>(pp + dd);
        Ls = fmaf(f, pp[D + 1], Ls);
        acc.x = fmaf(f, o.x, acc.x);
        acc.y = fmaf(f, o.y, acc.y);
        acc.z = fmaf(f, o.z, acc.z);
        acc.w = fmaf(f, o.w, acc.w);
      }
      float4 r;
      r.x = acc.x / Ls;
      r.y = acc.y / Ls;
      r.z = acc.z / Ls;
      r.w = acc.w / Ls;
      *reinterpret_cast<float4*>(sm.xs + e) = r;
    }
  }
  return !sync_or(!ok);
}

// After attention unit u (its partial stored by every warp, then a consumer barrier): count
// it in for its KV head; the last split to arrive merges the head group's split partials
// (o unnormalised, max m, sum l): out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s with M
// the largest m_s (attention.rs:186-191 over the whole prefix), in split order, into the
// attention output (warp = query head, lane = DPL dims).  The counter is left at zero.
template <int D>
__device__ void att_finish(const PersistArgs& a, const AttGeo& at, int u, const Smem& sm) {
  constexpr int DPL = D / 32;
  const int g = u / at.nsplit, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    unsigned* cnt = att_counters(a, D) + g;
    // release: this CTA's partial (stored before the consumer barrier) is visible to the split
    // that arrives last; acquire: the last split then sees every other split's partial
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(cnt) : "memory");
    sm.flags[1] = prev == (unsigned)at.nsplit - 1 ? 1 : 0;
    if (sm.flags[1]) *cnt = 0u;
  }
  csync();
  if (sm.flags[1]) {
    // warp = query head: lane s holds split s's (m, l) (and s + 32), the max and the weighted
    // sum are warp reductions, then every split's o slice is loaded with the weights broadcast
    const float* p0 = a.att_part + ((size_t)g * PERSIST_ATT_SPLITS_MAX * NREP + warp) * (D + 4);
    const size_t ss = (size_t)NREP * (D + 4);
    static_assert(PERSIST_ATT_SPLITS_MAX <= 64, "two splits per lane");
    const int ns = at.nsplit;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    // the first 16 splits' o slices are requested together with the (m, l) pairs
    constexpr int MB = 16;
    float ov[MB][DPL];
    auto load_o = [&](int s0) {
#pragma unroll
      for (int i = 0; i < MB; ++i) {
        if (DPL == 4) {
          const float4 v = s0 + i < ns ? ldcg4(p0 + (s0 + i) * ss + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
          ov[i][0] = v.x;
          ov[i][1 % DPL] = v.y;
          ov[i][2 % DPL] = v.z;
          ov[i][3 % DPL] = v.w;
        } else {
#pragma unroll
          for (int e = 0; e < DPL; ++e) ov[i][e] = s0 + i < ns ? __ldcg(p0 + (s0 + i) * ss + lane * DPL + e) : 0.f;
        }
      }
    };
    if (lane < ns) {
      m0 = __ldcg(p0 + lane * ss + D);
      l0 = __ldcg(p0 + lane * ss + D + 1);
    }
    if (lane + 32 < ns) {
      m1 = __ldcg(p0 + (lane + 32) * ss + D);
      l1 = __ldcg(p0 + (lane + 32) * ss + D + 1);
    }
    load_o(0);
    const float M = warp_max(fmaxf(m0, m1));
    const float f0 = lane < ns ? expf(m0 - M) : 0.f, f1 = lane + 32 < ns ? expf(m1 - M) : 0.f;
    const float Ls = warp_sum(f0 * l0 + f1 * l1);
    float acc[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
    for (int s0 = 0; s0 < ns; s0 += MB) {
      if (s0 > 0) load_o(s0);
#pragma unroll
      for (int i = 0; i < MB; ++i) {
        const int sp = s0 + i;
        const float f = __shfl_sync(0xffffffffu, sp < 32 ? f0 : f1, sp & 31);
        if (sp < ns)
#pragma unroll
          for (int e = 0; e < DPL; ++e) acc[e] = fmaf(f, ov[i][e], acc[e]);
      }
    }
    float* out = att_out(a, D) + (size_t)(g * NREP + warp) * D + lane * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e) out[e] = acc[e] / Ls;
  }
  csync();  // flags[1] is free again
}

// The attention output [nh*D] -> xs for the o_proj phase: one bulk copy (one L2 round trip;
// written by other CTAs' generic stores, hence the proxy fence).  `use` counts this CTA's
// earlier copies (the parity of sm.pbar).  Returns false on a failed wait.
template <int D>
__device__ bool att_load(const PersistArgs& a, const Smem& sm, int use) {
  const uint32_t bytes = (uint32_t)a.nh * D * 4;
  csync();  // nobody still reads xs
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(sm.pbar, bytes);
    bulk_g2s(sm.xs, att_out(a, D), bytes, sm.pbar);
  }
  const bool ok = wait_full(sm.pbar, use & 1, a.err, sm.flags);
  return !sync_or(!ok);
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Consumer state carried across phases (returned by value from the out-of-line phase bodies).
struct CState {
  int s;      // ring stages consumed
  int bad;    // the step must stop
  int merges; // attention output copies done (parity of sm.pbar)
};

// One attention unit: query heads g*8..g*8+7 against the positions of its tiles
// (attention.rs:129-150 for one split).  Warp r is query head r; its lanes split the head's
// dims for the dot products and the reduce-scatter hands lane j the score of position j0 + j
// of a tile; the softmax runs online across the unit's tiles.  Leaves the partial (o, m, l)
// in att_part.  Returns false if the CTA must stop.
template <int KC, int D>
__device__ bool att_unit(const PersistArgs& a, const AttGeo& at, int l, int u, const Smem& sm, CState& st, int nst) {
  constexpr int NC = D / 4, DPL = D / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = u / at.nsplit, sp = u % at.nsplit;
  const int t0 = sp * at.tps, t1 = min(at.ntiles, t0 + at.tps);
  float* qs = sm.xs;  // [8][D]
  // the 8 query rows and the current position's K/V row (both written by this launch's Q
  // phase) are fetched in one round trip; the row is patched into its tile's ring slot below
  static_assert(NREP * NC <= 4 * PK_CTHREADS, "query rows per thread");
  float4 qv[(NREP * NC + PK_CTHREADS - 1) / PK_CTHREADS];
#pragma unroll
  for (int i = 0; i < (NREP * NC + PK_CTHREADS - 1) / PK_CTHREADS; ++i)
    if (tid + i * PK_CTHREADS < NREP * NC) qv[i] = ldcg4(a.q + (size_t)g * NREP * D + (tid + i * PK_CTHREADS) * 4);
  const int tpos = at.pos / at.span;  // tile holding the current position
  float4 cur = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tpos >= t0 && tpos < t1 && tid < 2 * NC) {
    const size_t src = (size_t)l * a.kv_layer_stride + ((size_t)g * a.s_max + at.pos) * D + (tid % NC) * 4;
    cur = ldcg4((tid < NC ? a.kcache : a.vcache) + src);
  }
#pragma unroll
  for (int i = 0; i < (NREP * NC + PK_CTHREADS - 1) / PK_CTHREADS; ++i)
    if (tid + i * PK_CTHREADS < NREP * NC) *reinterpret_cast<float4*>(qs + (tid + i * PK_CTHREADS) * 4) = qv[i];
  float m = -INFINITY, lsum = 0.f;
  float o[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) o[e] = 0.f;
  for (int t = t0; t < t1; ++t) {
    const int slot = st.s % nst;
    bool lbad = !wait_full(&sm.full[slot], (st.s / nst) & 1, a.err, sm.flags);
    float* Ks = reinterpret_cast<float*>(sm.ring + (size_t)slot * PK_ROWS * KC);
    float* Vs = Ks + (size_t)at.span * D;
    const int j0 = t * at.span, j1 = min(at.len, j0 + at.span), nt = j1 - j0;
    if (!lbad && t == tpos && tid < 2 * NC) {
      float* dst = (tid < NC ? Ks : Vs) + (size_t)(at.pos - j0) * D + (tid % NC) * 4;
      *reinterpret_cast<float4*>(dst) = cur;
      // the slot is refilled by bulk copies (async proxy) once released
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (sync_or(lbad)) return false;
    // scores q.k^T * scale (attention.rs:166): lane l holds dims [l DPL, (l + 1) DPL) of its
    // warp's query head and forms its partial dot product with every position of the tile
    // (a K row is one contiguous 32-lane read); a butterfly reduce-scatter over the lanes then
    // leaves position l's full score in lane l (fixed order: deterministic)
    float qv[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) qv[e] = qs[warp * D + lane * DPL + e];
    float sc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float t = 0.f;
      if (j < nt) {
        const float* kr = Ks + (size_t)j * D + lane * DPL;
        if constexpr (DPL == 4) {
          const float4 kk = *reinterpret_cast<const float4*>(kr);
          t = fmaf(qv[0], kk.x, t);
          t = fmaf(qv[1], kk.y, t);
          t = fmaf(qv[2], kk.z, t);
          t = fmaf(qv[3], kk.w, t);
        } else {
#pragma unroll
          for (int e = 0; e < DPL; ++e) t = fmaf(qv[e], kr[e], t);
        }
      }
      sc[j] = t;
    }
#pragma unroll
    for (int bit = 16; bit >= 1; bit >>= 1) {  // keep the half of the positions whose bit matches
      const bool up = (lane & bit) != 0;
#pragma unroll
      for (int i = 0; i < bit; ++i) {
        const float send = up ? sc[i] : sc[i + bit];
        sc[i] = (up ? sc[i + bit] : sc[i]) + __shfl_xor_sync(0xffffffffu, send, bit);
      }
    }
    const bool valid = lane < nt;
    const float sv = valid ? sc[0] * a.attn_scale : -INFINITY;
    const float mn = fmaxf(m, warp_max(sv));
    const float corr = expf(m - mn);  // 0 on the first tile (m = -inf)
    const float p = valid ? expf(sv - mn) : 0.f;
    // the weights go through shared memory so the P.V loop below can run ahead of them
    float* ps = sm.xs + NREP * D + warp * 32;
    ps[lane] = p;
    lsum = lsum * corr + warp_sum(p);
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[e] *= corr;
    __syncwarp();
#pragma unroll 8
    for (int j = 0; j < nt; ++j) {
      const float pj = ps[j];
      const float* vr = Vs + (size_t)j * D + lane * DPL;
      if constexpr (DPL == 4) {
        const float4 vv = *reinterpret_cast<const float4*>(vr);
        o[0] = fmaf(pj, vv.x, o[0]);
        o[1] = fmaf(pj, vv.y, o[1]);
        o[2] = fmaf(pj, vv.z, o[2]);
        o[3] = fmaf(pj, vv.w, o[3]);
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[e] = fmaf(pj, vr[e], o[e]);
      }
    }
    __syncwarp();  // ps is rewritten by the next tile
    m = mn;
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
    ++st.s;
  }
  float* pp = a.att_part + (((size_t)g * PERSIST_ATT_SPLITS_MAX + sp) * NREP + warp) * (D + 4);
#pragma unroll
  for (int e = 0; e < DPL; ++e) pp[lane * DPL + e] = o[e];
  if (lane == 0) {
    pp[D] = m;
    pp[D + 1] = lsum;
  }
  return true;
}

// This CTA's attention units of layer l (after the Q phase is published).
template <int KC, int D>
__device__ __forceinline__ CState att_units(const PersistArgs& a, const Smem& sm, CState st, int nst, const AttGeo& at,
                                            int l, int first) {
  for (int u = first; u < at.items; u += gridDim.x) {
    const bool ok = att_unit<KC, D>(a, at, l, u, sm, st, nst);
    csync();  // xs (queries) reused by the next unit; every warp's partial is stored
    if (!ok) {
      st.bad = 1;
      break;
    }
    if (at.merge_once) att_finish<D>(a, at, u, sm);
  }
  return st;
}

// Sum over the warp's 32 lanes of eight per-lane values, one per row: three exchange steps that
// each halve the rows a lane carries (lanes differing in bit 4, 3, 2 swap the halves they do
// not keep), then two plain butterfly steps.  Lane l returns the sum of v[(l >> 2) & 7].
__device__ __forceinline__ float warp_rows_sum(const float (&v)[PK_ROWS], int lane) {
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
  float b[4], c[2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    b[i] = (h16 ? v[i + 4] : v[i]) + __shfl_xor_sync(0xffffffffu, h16 ? v[i] : v[i + 4], 16);
#pragma unroll
  for (int i = 0; i < 2; ++i)
    c[i] = (h8 ? b[i + 2] : b[i]) + __shfl_xor_sync(0xffffffffu, h8 ? b[i] : b[i + 2], 8);
  float d = (h4 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, h4 ? c[0] : c[1], 4);
  d += __shfl_xor_sync(0xffffffffu, d, 2);
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  return d;
}

// Sum of 8 consecutive floats of shared memory, in index order.
__device__ __forceinline__ float sum8(const float* p) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  return ((((((a.x + a.y) + a.z) + a.w) + b.x) + b.y) + b.z) + b.w;
}

// CPL consecutive bf16 of shared memory -> f32.
template <int CPL>
__device__ __forceinline__ void load_bf16(const uint16_t* p, float* out) {
  if constexpr (CPL == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    out[0] = bf16lo(v.x); out[1] = bf16hi(v.x); out[2] = bf16lo(v.y); out[3] = bf16hi(v.y);
    out[4] = bf16lo(v.z); out[5] = bf16hi(v.z); out[6] = bf16lo(v.w); out[7] = bf16hi(v.w);
  } else if constexpr (CPL == 4) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    out[0] = bf16lo(v.x); out[1] = bf16hi(v.x); out[2] = bf16lo(v.y); out[3] = bf16hi(v.y);
  } else if constexpr (CPL == 2) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
    out[0] = bf16lo(v); out[1] = bf16hi(v);
  } else {
    out[0] = __uint_as_float(((uint32_t)*p) << 16);
  }
}

// L2 line prefetches (load/store path, no data returned) of MLP stages [s0, s1) of this
// CTA in layer l: stage q is unit first_m + (q / 3) * grid, group q % 3 (gate rows, up rows,
// rows of the transposed down weight), 32 KB contiguous; each consumer thread takes one 128 B
// line of each stage.  Issued while the warps wait on an earlier phase, so the MLP phase
// finds most of its weights in L2 instead of waiting on HBM behind the ring.
template <int KC>
__device__ __forceinline__ void prefetch_mlp(const PersistArgs& a, int l, int first_m, int s0, int s1) {
  const int U = a.I / PK_ROWS, G = gridDim.x;
  for (int q = s0; q < s1; ++q) {
    const int u = first_m + (q / 3) * G, gi = q % 3;
    if (u >= U) break;
    const uint16_t* W = gi == 2 ? s_lay[l].wdt : s_lay[l].wgu;
    const char* src = reinterpret_cast<const char*>(W + (size_t)unit_row(a, PH_M, u, gi) * a.H);
    const int lines = PK_ROWS * KC * 2 / 128;
    for (int i = threadIdx.x; i < lines; i += PK_CTHREADS)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(src + (size_t)i * 128));
  }
}

// This CTA's units of a GEMV phase (Q, O, MLP, head) after its dependency is met: x -> xs
// (optional RMSNorm; O: the attention merge), then the streamed dot products.  Warp w owns the
// K slice [w*KC/8, (w+1)*KC/8) of every row, so a lane holds only KC/256 input values and each
// stage is 8 independent FMA chains per lane; the warps' row partials meet in sm.kp behind one
// CTA barrier per unit, after which warp w applies row w's epilogue (Q: its rotate_half
// partner is row w of the unit's second group).
template <int KC, int D>
__device__ __forceinline__ CState gemv_units(const PersistArgs& a, const Smem& sm, CState st, int nst, int kind, int l,
                                             int pos, int U, int K, int gpu, int first, const XIn xsrc,
                                             const float* norm_w, const XIn resid, const AttGeo& at) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  // residual of this warp's row in each of its first PK_RES_UNITS units, fetched together
  // with x (one round trip) so the epilogues never wait on memory
  float resv[PK_RES_UNITS];
#pragma unroll
  for (int k = 0; k < PK_RES_UNITS; ++k) {
    const int u = first + k * G;
    resv[k] = (kind == PH_O && lane == 0 && u < U) ? ldx1(resid, u * PK_ROWS + warp) : 0.f;
  }
  if (kind == PH_O) {
    if (!(at.merge_once ? att_load<D>(a, sm, st.merges++)
                                         : att_merge<D>(a, at, sm, st.merges++, l * PH_PER_LAYER + kind))) {
      st.bad = 1;
      return st;
    }
  } else {
    load_x<KC>(a, kind == PH_HEAD ? a.L * PH_PER_LAYER : l * PH_PER_LAYER + kind, xsrc, norm_w, K, a.eps, sm);
  }
  if (tid == 0) trace_mark(a, kind == PH_HEAD ? a.L * PH_PER_LAYER : l * PH_PER_LAYER + kind, 1);
  // Each warp owns a K slice of every row (columns warp*SL + lane*CPL ..), so a lane needs
  // only CPL elements of the phase input; the warps' row partials meet in sm.kp.
  constexpr int CPL = KC / 256, SL = KC / PK_CWARPS;
  // MLP: this lane's CPL down_proj accumulators (output columns warp*SL + lane*CPL..) live
  // in shared memory, xs[H, 2H) being free in this phase
  float* dacc = sm.xs + a.H + warp * SL + lane * CPL;
  if (kind == PH_M) {
#pragma unroll
    for (int e = 0; e < CPL; ++e) dacc[e] = 0.f;
  }
  // this lane's slice of the input (K == KC), loaded once for the phase
  float xr[CPL];
#pragma unroll
  for (int e = 0; e < CPL; ++e) xr[e] = sm.xs[warp * SL + lane * CPL + e];
  (void)K;
  int slot = st.s % nst;  // ring position, advanced incrementally
  uint32_t par = (st.s / nst) & 1;
  bool lbad = false;
  float bv = -FLT_MAX;  // head: this warp's running argmax
  int bi = INT_MAX;
  long long* xnext = a.xacc + (size_t)((l + 1) & 1) * a.H;  // the next layer's accumulator
  float mvr[PK_ROWS];  // MLP: silu(gate) * up of the unit's 8 channels
  const int rrow = (lane >> 2) & 7;  // the row whose warp sum this lane holds after a reduction
  const int qpu = q_pair_units(a);
  // head: the warps' row partials of all this CTA's units are kept in sm.parts (free in this
  // phase) and summed once after the last unit, instead of a CTA barrier per unit
  const bool defer = kind == PH_HEAD && (size_t)((U - first + G - 1) / G) * (PK_ROWS * PK_CWARPS) <=
                                            persist_att_part_floats(a.nkv, a.nh, D);
  int k = 0;
  for (int u = first; u < U; u += G, ++k) {
    float* kpb = sm.kp + (k & 1) * (2 * PK_ROWS * PK_CWARPS);
    float t0 = 0.f, t1 = 0.f;
    const int ng = (kind == PH_Q && u >= qpu) ? 1 : gpu;  // Q: v rows are one group
    const int last_group = kind == PH_M ? 1 : ng - 1;
    for (int gi = 0; gi < ng; ++gi) {
      if (kind == PH_M && gi == 2) {
        // down_proj column block (mlp.rs:33): accumulate this warp's SL output columns over
        // rows j0..j0+7 of wdt, weighted by the unit's 8 silu(gate)*up values
        if (!lbad && !wait_full(&sm.full[slot], par, a.err, sm.flags)) lbad = true;
        if (!lbad) {
          const uint16_t* wr = sm.ring + (size_t)slot * PK_ROWS * KC + warp * SL + lane * CPL;
          float d[CPL];
#pragma unroll
          for (int e = 0; e < CPL; ++e) d[e] = dacc[e];
#pragma unroll
          for (int r = 0; r < PK_ROWS; ++r) {
            float wv[CPL];
            load_bf16<CPL>(wr + r * KC, wv);
#pragma unroll
            for (int e = 0; e < CPL; ++e) d[e] = fmaf(mvr[r], wv[e], d[e]);
          }
#pragma unroll
          for (int e = 0; e < CPL; ++e) dacc[e] = d[e];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        if (++slot == nst) {
          slot = 0;
          par ^= 1u;
        }
        ++st.s;
        continue;
      }
      // the stage's 8 rows over this warp's K slice: 8 independent FMA chains
      float acc[PK_ROWS];
#pragma unroll
      for (int r = 0; r < PK_ROWS; ++r) acc[r] = 0.f;
      if (!lbad && !wait_full(&sm.full[slot], par, a.err, sm.flags)) lbad = true;
      if (!lbad) {
        const uint16_t* wr = sm.ring + (size_t)slot * PK_ROWS * KC + warp * SL + lane * CPL;
#pragma unroll
        for (int r = 0; r < PK_ROWS; ++r) {
          float wv[CPL];
          load_bf16<CPL>(wr + r * KC, wv);
#pragma unroll
          for (int e = 0; e < CPL; ++e) acc[r] = fmaf(wv[e], xr[e], acc[r]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
      if (++slot == nst) {
        slot = 0;
        par ^= 1u;
      }
      ++st.s;
      const float ws = warp_rows_sum(acc, lane);
      if (defer) {
        if ((lane & 3) == 0) sm.parts[(k * PK_ROWS + rrow) * PK_CWARPS + warp] = ws;
        continue;
      }
      if ((lane & 3) == 0) kpb[(gi * PK_ROWS + rrow) * PK_CWARPS + warp] = ws;
      if (gi == last_group) {
        // every warp's partials of the unit are in: row totals over the warps, in warp order
        csync();
        if (kind == PH_M) {
          // lanes 0..7: silu(gate) * up of channel `lane` (mlp.rs:31-33), then to every lane
          float m = 0.f;
          if (lane < PK_ROWS) m = silu(sum8(kpb + lane * PK_CWARPS)) * sum8(kpb + (PK_ROWS + lane) * PK_CWARPS);
#pragma unroll
          for (int r = 0; r < PK_ROWS; ++r) mvr[r] = __shfl_sync(0xffffffffu, m, r);
        } else if (lane == 0) {
          t0 = sum8(kpb + warp * PK_CWARPS);
          if (ng == 2) t1 = sum8(kpb + (PK_ROWS + warp) * PK_CWARPS);
        }
      }
    }
    // ---- this warp's row epilogue (lane 0)
    if (kind == PH_M || defer || lbad || lane != 0) continue;
    const int row = unit_row(a, kind, u, 0) + warp;
    if (kind == PH_HEAD) {
      if (a.logits) a.logits[row] = t0;
      if (better(t0, row, bv, bi)) {
        bv = t0;
        bi = row;
      }
    } else if (kind == PH_Q && ng == 1) {
      // a v row: straight into the cache at `pos`
      const int head = row / a.d, ii = row % a.d;
      a.vcache[(size_t)l * a.kv_layer_stride + ((size_t)(head - a.nh - a.nkv) * a.s_max + pos) * a.d + ii] = t0;
    } else if (kind == PH_Q) {
      // LongRoPE on q/k rows (rope.rs:76-95), post-RoPE q and k into the cache at `pos`
      const int head = row / a.d, ii = row % a.d, half = a.d / 2;
      const float ya = t0, yb = t1;
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
        float* dst = a.kcache + (size_t)l * a.kv_layer_stride + ((size_t)(head - a.nh) * a.s_max + pos) * a.d;
        dst[ii] = oa;
        dst[ii + half] = ob;
      }
    } else {
      // o_proj + residual (layer.rs:33-38): x1 = x0 + s*o; x1 also seeds the next layer's
      // accumulator, into which the MLP phase adds s*down
      float r = 0.f;
#pragma unroll
      for (int q = 0; q < PK_RES_UNITS; ++q)
        if (q == k) r = resv[q];
      if (k >= PK_RES_UNITS) r = ldx1(resid, row);
      const float x1 = r + t0 * a.res_scale;
      a.x1[row] = x1;
      xnext[row] = to_fix(x1);
    }
  }
  if (defer) {
    // the logits of this CTA's k units: thread t sums row t % 8 of its unit t / 8 over the warps
    csync();
    for (int t = tid; t < k * PK_ROWS; t += PK_CTHREADS) {
      const int row = (first + (t / PK_ROWS) * G) * PK_ROWS + t % PK_ROWS;
      const float v = sum8(sm.parts + t * PK_CWARPS);
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
  }
  if (kind == PH_HEAD && lane == 0) {
    sm.red[16 + warp] = bv;
    reinterpret_cast<int*>(sm.red)[24 + warp] = bi;
  }
  if (kind == PH_M) {
    // this CTA's res_scale * down partial (xs[H, 2H), the warps' column slices side by side)
    // into the next layer's accumulator, seeded with x1 by the O phase: x0' = x1 + s * down
    // (layer.rs:33-38, 72).  The partial is rounded to the accumulator's fixed point in
    // xs[0, 2H) viewed as int64 [H] (the phase input there is no longer read: each lane holds
    // its slice in registers), then one bulk integer reduce-add through the TMA engine per
    // CTA: 128-byte reductions at L2, exact in any arrival order.
    const bool mine = !lbad && k > 0;
    float dv[CPL];
#pragma unroll
    for (int e = 0; e < CPL; ++e) dv[e] = dacc[e] * a.res_scale;
    csync();  // every lane's accumulators are in registers before the int64 image overwrites xs
    if (mine) {
      long long* fx = reinterpret_cast<long long*>(sm.xs) + warp * SL + lane * CPL;
#pragma unroll
      for (int e = 0; e < CPL; ++e) fx[e] = to_fix(dv[e]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // read by the async proxy
    }
    if (sync_or(lbad)) st.bad = 1;
    if (mine && !st.bad && tid == 0) {
      // the destination was seeded by other CTAs' generic stores (acquired at the phase start)
      asm volatile("fence.proxy.async.global;" ::: "memory");
      asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.u64 [%0], [%1], %2;" ::"l"(xnext),
                   "r"(smem_u32(sm.xs)), "r"((uint32_t)a.H * 8u)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      asm volatile("fence.proxy.async.global;" ::: "memory");  // before the generic release
    }
    return st;
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

template <int KC, int D>
__global__ void __launch_bounds__(PK_THREADS, 1) persist_decode_kernel(const PersistArgs a, int nst, int xs_floats,
                                                                        int att_span) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem sm;
  sm.ring = reinterpret_cast<uint16_t*>(smem_raw);
  sm.xs = reinterpret_cast<float*>(smem_raw + (size_t)nst * PK_ROWS * KC * 2);
  sm.parts = sm.xs + xs_floats;
  sm.ctab = sm.parts + persist_att_part_floats(a.nkv, a.nh, D);
  sm.stab = sm.ctab + 64;
  sm.red = sm.stab + 64;
  sm.kp = sm.red + 64;
  sm.flags = reinterpret_cast<volatile int*>(sm.kp + PK_KP_FLOATS);
  sm.full = reinterpret_cast<uint64_t*>(sm.kp + PK_KP_FLOATS + 8);
  sm.empty = sm.full + nst;
  sm.pbar = sm.empty + nst;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int G = gridDim.x;
  AttGeo at;
  at.pos = *a.pos;  // position of the token being decoded (advanced by this launch)
  at.len = at.pos + 1;
  at.span = att_span;
  at.ntiles = (at.len + att_span - 1) / att_span;
  // up to merge_tiles tiles: at most PERSIST_ATT_SPLITS splits, merged from shared memory in
  // every o_proj CTA; longer caches: a split per tile (up to the grid), merged once per KV head
  at.merge_once = at.ntiles > a.merge_tiles;
  at.nsplit = !at.merge_once ? min(at.ntiles, PERSIST_ATT_SPLITS)
                             : min(at.ntiles, min(PERSIST_ATT_SPLITS_MAX, max(1, G / a.nkv)));
  at.tps = (at.ntiles + at.nsplit - 1) / at.nsplit;
  at.nsplit = (at.ntiles + at.tps - 1) / at.tps;
  at.items = a.nkv * at.nsplit;
  const int pos = at.pos;

  for (int i = tid; i < a.L * (int)(sizeof(PersistLayer) / 8); i += PK_THREADS)
    reinterpret_cast<unsigned long long*>(s_lay)[i] = reinterpret_cast<const unsigned long long*>(a.layers)[i];
  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], PK_CWARPS);
    }
    mbar_init(sm.pbar, 1);
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

  CState st = {0, 0, 0};
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
    // while this phase waits on the previous one, stage a share of the coming MLP phase's
    // weights in L2 (Q, ATT, O phases each take the next a.mlp_pf stages after the ring's)
    if (a.mlp_pf > 0 && !head && kind != PH_M) {
      int off_m = off;
      for (int k2 = kind; k2 < PH_M; ++k2) off_m += geo_of(a, l, k2, at).U;
      const int s0 = nst + kind * a.mlp_pf;
      prefetch_mlp<KC>(a, l, first_unit(off_m % G, G), s0, s0 + a.mlp_pf);
    }
    if (first < g.U) {
      if (tid == 0) trace_mark(a, ph, 0);
      if (prev_cnt != nullptr && !dep_wait(prev_cnt, prev_target, a.err, false)) {
        st.bad = 1;
        break;
      }
      if (tid == 0) trace_mark(a, ph, 6);
      if (kind == PH_ATT) {
        if (tid == 0) trace_mark(a, ph, 1);
        st = att_units<KC, D>(a, sm, st, nst, at, l, first);
      } else {
        const PersistLayer* w = s_lay + (l < a.L ? l : 0);
        // Q: the layer input; M: x1; head: the last layer's output (O merges attention)
        const XIn xsrc = kind == PH_M ? XIn{a.x1, nullptr} : xin_of(a, l);
        const float* norm_w = kind == PH_Q ? w->ln_in : kind == PH_M ? w->ln_post : head ? a.final_norm : nullptr;
        const XIn resid = xin_of(a, l);
        st = gemv_units<KC, D>(a, sm, st, nst, kind, l, pos, g.U, g.K, g.gpu, first, xsrc, norm_w, resid, at);
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
      for (int g = 0; g < a.nkv; ++g) att_counters(a, D)[g] = 0u;  // zero already unless a unit gave up
      __threadfence();
    }
  }
}

__global__ void transpose_u16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int R, int C) {
  __shared__ uint16_t tile[32][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = blockIdx.y * 32 + i;
    if (r < R && c < C) tile[i][threadIdx.x] = src[(size_t)r * C + c];
  }
  __syncthreads();
  const int r2 = blockIdx.y * 32 + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c2 = blockIdx.x * 32 + i;
    if (c2 < C && r2 < R) dst[(size_t)c2 * R + r2] = tile[threadIdx.x][i];
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

// Ring depth: about 128 KB of copies in flight per SM streams HBM fastest (4 x 32 KB measured
// 7.4 TB/s over 148 SMs; 6 x 32 KB 6.9 TB/s).  nst_cap > 1 overrides it.
constexpr int PK_RING_BYTES = 131072;

PkShape shape_of(int H, int I, int nh, int nkv, int d, int nst_cap) {
  PkShape p;
  p.kc = pick_kc(H, I, nh * d);
  p.d = d;
  if (!p.kc || d <= 0 || nkv <= 0) return p;
  p.span = std::min(32, 2 * p.kc / d);  // K and V rows of `span` positions fill one ring stage
  // xs holds an input vector (x, normalised x1, or the attention output); the MLP phase also
  // keeps its down_proj accumulators in xs[H, 2H)
  const int m = std::max(2 * H, std::max(nh * d, NREP * d + NREP * 32));  // attention: q rows + weights
  p.xs_floats = (m + 3) & ~3;
  const size_t fixed = (size_t)p.xs_floats * 4 + persist_att_part_floats(nkv, nh, d) * 4 + PK_MISC_FLOATS * 4 + 32 + 8;
  const int stage = PK_ROWS * p.kc * 2;
  const int want = nst_cap > 1 ? nst_cap : std::max(2, PK_RING_BYTES / stage);
  const int fit = (int)(((size_t)PK_MAX_SMEM - fixed) / (stage + 16));
  p.nst = std::min(want, fit);
  p.smem = (size_t)p.nst * stage + fixed + 16 * (size_t)p.nst;
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

bool persist_supported(int L, int H, int I, int nh, int nkv, int d, int V, int s_max) {
  if (L <= 0 || L > PK_MAX_LAYERS) return false;
  if (nkv <= 0 || nh != NREP * nkv || (d != 64 && d != 128) || V <= 0 || V % PK_ROWS != 0 || s_max <= 0) return false;
  if (I % PK_ROWS != 0) return false;
  static_assert(sizeof(PersistLayer) % 8 == 0, "layer table copied in 8-byte words");
  const PkShape p = shape_of(H, I, nh, nkv, d, 0);
  // every row is one K chunk (the streaming loop keeps that chunk of x in registers): the
  // chunk must equal H and the attention width nh*d
  return p.kc != 0 && p.kc == H && nh * d == H && p.nst >= 2 && p.span >= 1;
}

int persist_configure(int H, int I, int nh, int nkv, int d, int s_max, int nst_cap, int grid_cap) {
  (void)s_max;
  const PkShape p = shape_of(H, I, nh, nkv, d, nst_cap);
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
  // one CTA per SM (am_part holds 4096 partials), at most grid_cap
  return std::min(std::min(sms, 4096), grid_cap > 0 ? grid_cap : sms);
}

cudaError_t launch_persist(const PersistArgs& a, int grid, int nst_cap, cudaStream_t st, bool cooperative) {
  const PkShape p = shape_of(a.H, a.I, a.nh, a.nkv, a.d, nst_cap);
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

cudaError_t transpose_bf16(const uint16_t* src, uint16_t* dst, int R, int C, cudaStream_t st) {
  if (R <= 0 || C <= 0) return cudaErrorInvalidValue;
  const dim3 grid((C + 31) / 32, (R + 31) / 32);
  count_launch();
  transpose_u16_kernel<<<grid, dim3(32, 8), 0, st>>>(src, dst, R, C);
  return cudaGetLastError();
}

}  // namespace vx
