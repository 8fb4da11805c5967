// Persistent batch-1 decode step: one launch per token runs every decoder layer and the
// greedy head (reference MiniCpmModel::forward_step, src/minicpm4/model.rs:64-84, with the
// layer / attention / MLP steps of layer.rs:57-73, attention.rs:91-154, mlp.rs:28-34).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "gemv.cuh"

namespace vx {

struct PersistLayer {
  const uint16_t* wqkv;  // [(nh+2nkv)*d, H]
  const uint16_t* wo;    // [H, nh*d]
  const uint16_t* wgu;   // [2I, H]
  const uint16_t* wdt;   // [I, H]: down_proj transposed (row j = the weights input j feeds)
  const float* ln_in;    // [H]
  const float* ln_post;  // [H]
};

// Phases per decoder layer: qkv+rope, attention, o_proj, MLP (gate|up + down); then the head.
constexpr int PERSIST_PHASES_PER_LAYER = 4;
// Attention splits per KV head: the cache walk of a KV head is split over up to
// PERSIST_ATT_SPLITS_MAX units (whole 32-position tiles each); each leaves its online-softmax
// partial (o, m, l) in att_part and the last to finish merges them (split order) into the
// attention output that the o_proj phase copies in.  PERSIST_ATT_SPLITS sizes the kernel's
// shared scratch (the head phase keeps its row partials there).
constexpr int PERSIST_ATT_SPLITS = 8;
constexpr int PERSIST_ATT_SPLITS_MAX = 64;

struct PersistArgs {
  int L, H, I, nh, nkv, d, V, s_max;
  float eps, res_scale, attn_scale, emb_scale;
  const PersistLayer* layers;  // device array [L]
  const float* final_norm;     // [H]
  const uint16_t* embed;       // [V, H] (tied input embedding and LM head)
  const RopeParams* rope;      // nullptr = no_rope
  float* kcache;               // layer l at kcache + l * kv_layer_stride, layout [nkv][s_max][d]
  float* vcache;
  size_t kv_layer_stride;      // elements
  int* pos;                    // device position of the token being decoded (incremented)
  int* step;                   // device greedy step index (incremented)
  int* tokens;                 // picked ids, tokens[*step]
  float* x0;                   // layer 0's input [H]: receives the next token's embedding
  long long* xacc;             // [2][H] residual stream of layers 1..L in fixed point (value x
                               // 2^32, int64): layer l >= 1 reads xacc[l & 1].  Integer sums
                               // are exact, so the order in which the CTAs' down-projection
                               // partials arrive cannot change a bit of the result.
  float* x1;                   // residual stream after attention [H]
  float* q;                    // post-RoPE queries [nh*d]
  float* logits;               // optional [V]
  float* hid_norm;             // final-norm hidden [H]
  float* att_part;             // [nkv][PERSIST_ATT_SPLITS_MAX][nh/nkv][d+4] split partials (o, m, l),
                               // then the merged output [nh][d], then [nkv] arrival counters (zeroed)
  float2* am_part;             // [grid] per-CTA argmax partials
  unsigned* phase_cnt;         // [4L + 2] phase arrival counters, zero between launches
  int* err;                    // device error word
  // L2 staging ahead of the shared-memory ring: the producer issues L2 prefetches for the
  // stages pf_stages beyond its newest ring copy (0: off).  evict_first: weight copies into
  // the ring mark their L2 lines evict-first.
  int pf_stages;
  int evict_first;
  // Ring copies in flight (issued, not landed) at most; 0: as many as there are free slots.
  int inflight;
  // MLP stages each of the Q, ATT and O phases prefetches into L2 for the layer's MLP phase.
  int mlp_pf;
  // Caches of more than merge_tiles 32-position tiles: one attention split per tile, the last
  // split of a KV head to finish merges them once; shorter caches: at most
  // PERSIST_ATT_SPLITS splits, merged by every o_proj CTA.
  int merge_tiles;
  // Optional phase trace (nullptr: off): per phase p (4 per layer, then the head) and CTA c,
  // trace[(p * grid + c) * PERSIST_TRACE_FIELDS + k] = %globaltimer ns at k = 0 consumer
  // phase start, 1 inputs ready (dependency met, x loaded), 2 phase published, 3 producer's
  // first copy of the phase issued, 4 its last copy issued, 5 last unit computed, 6 dependency
  // met (the previous phase's counter seen), 7 the phase input's bytes arrived (before the
  // RMSNorm or attention-merge arithmetic; GEMV phases).  Zero where the CTA had no units.
  unsigned long long* trace;
};

constexpr int PERSIST_TRACE_FIELDS = 8;
inline size_t persist_phase_count(int L) { return (size_t)PERSIST_PHASES_PER_LAYER * L + 1; }
inline size_t persist_trace_entries(int L, int grid) { return persist_phase_count(L) * grid * PERSIST_TRACE_FIELDS; }

// Sizes of the device buffers the caller provides.
inline size_t persist_counter_count(int L) { return (size_t)PERSIST_PHASES_PER_LAYER * L + 2; }
__host__ __device__ inline size_t persist_att_part_floats(int nkv, int nh, int d) {
  return (size_t)nkv * PERSIST_ATT_SPLITS * (nh / (nkv > 0 ? nkv : 1)) * (d + 4);
}
// att_part as allocated: the partials of PERSIST_ATT_SPLITS_MAX splits, the merged output and
// the counters (one 4-byte word per KV head).
__host__ __device__ inline size_t persist_att_partials_floats(int nkv, int nh, int d) {
  return (size_t)nkv * PERSIST_ATT_SPLITS_MAX * (nh / (nkv > 0 ? nkv : 1)) * (d + 4);
}
__host__ __device__ inline size_t persist_att_global_floats(int nkv, int nh, int d) {
  return persist_att_partials_floats(nkv, nh, d) + (size_t)nh * d + (size_t)((nkv + 3) / 4) * 4;
}

// Whether the persistent step supports this model shape (else the per-kernel step is used).
bool persist_supported(int L, int H, int I, int nh, int nkv, int d, int V, int s_max);
// Once per context, before capture: raise the kernel's shared-memory limit and return the
// grid (one CTA per SM, at most grid_cap when > 0) or 0 when the device cannot hold it.
// nst_cap (> 1) sets the ring depth in stages (0: about 128 KB of stages).
int persist_configure(int H, int I, int nh, int nkv, int d, int s_max, int nst_cap, int grid_cap);
cudaError_t launch_persist(const PersistArgs& a, int grid, int nst_cap, cudaStream_t st, bool cooperative);
// dst [C, R] = transpose of src [R, C] (bf16 bit patterns); used to lay down_proj out as wdt.
cudaError_t transpose_bf16(const uint16_t* src, uint16_t* dst, int R, int C, cudaStream_t st);

}  // namespace vx
