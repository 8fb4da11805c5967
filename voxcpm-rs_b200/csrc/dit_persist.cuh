// Persistent non-causal MiniCPM-4 stack forward on tcgen05 (dit_persist.cu): arguments and
// host entry points.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <map>
#include <vector>

#include "gemv.cuh"

namespace vx {

struct DitPersistLayer {
  const uint16_t* wqkv;  // [(nh + 2 nkv) d, H]
  const uint16_t* wo;    // [H, nh d]
  const uint16_t* wgu;   // [2 I, H]
  const uint16_t* wd;    // [H, I]
  const float* ln_in;    // [H]
  const float* ln_post;  // [H]
};

// A MiniCPM-4 stack's shape and weights as the persistent forward reads them.
struct LmStackView {
  int L, H, I, nh, nkv, d;
  float eps, res_scale, attn_scale;
  const RopeParams* rope;
  const float* norm_w;
  std::vector<DitPersistLayer> layers;
};

// GEMM phases deal their (um-row weight unit, 64-element K chunk) pairs to ncta CTAs in
// contiguous runs: the CTA of rank b < ncta (rank = (blockIdx - cta_off) mod grid) takes pairs
// [b T / ncta, (b + 1) T / ncta) of T.  Every
// maximal run inside one tile is a segment; segments are numbered CTA-major (which is also
// tile-major), each writes its f32 partial tile to its own slot and the consumer sums a tile's
// slots in ascending order (deterministic).
enum { DP_KIND_QKV, DP_KIND_O, DP_KIND_GU, DP_KIND_DOWN, DP_KINDS };

// Attention of the ATT phase: DP_ATT_SEQ = non-causal attention among each sequence's S rows
// (LocDiT decoder, rope positions 0..S-1); DP_ATT_DECODE = one new row per sequence at the
// device position *pos, attending to the static KV cache 0..pos after writing its k, v there
// (a batched decode step, MiniCpmModel::forward_step).
enum { DP_ATT_SEQ = 0, DP_ATT_DECODE = 1 };

struct DitPersistArgs {
  int L, H, I, nh, nkv, d;
  int S, N, R, Rpad;            // tokens per sequence, sequences, rows = N S, rows rounded up to 32
  int att_mode;                 // DP_ATT_SEQ or DP_ATT_DECODE (S = 1)
  int um;                       // weight rows per GEMM unit: 128, or 256 (two MMA tiles, two accumulators)
  int split_b;                  // 1: the hi and lo activation planes as two copies (else one 3-D box)
  float* kcache;                // DP_ATT_DECODE: layer l, sequence n, KV head g at kcache +
  float* vcache;                //   l kv_layer_stride + (n nkv + g) max_len d, [max_len][d]
  size_t kv_layer_stride;
  int max_len;
  const int* pos;               // device position of the new rows
  const float* rope_pos;        // DP_ATT_DECODE: [max_len][2][d/2] LongRoPE cos, sin per position
  float* att_part;              // DP_ATT_DECODE: per (sequence, KV head) split partials of the cache walk
  unsigned* att_cnt;            //   and their arrival counters (zero between layers)
  float eps, res_scale, attn_scale;
  const DitPersistLayer* layers;  // device [L]
  const CUtensorMap* wmaps;       // device [L][4]: qkv, o, gate|up, down (um-row x 64 boxes)
  const CUtensorMap* xmaps;       // device [2]: the split operand as K = H and K = I (64 x Rpad x 2 boxes)
  const RopeParams* rope;         // null: no rope
  const float* final_norm;        // [H]
  const float* x_in;              // [R, H]: the input rows
  float* x;                       // [R, H]: each layer's input
  float* x1;                      // [R, H]: the residual stream after attention
  float* out;                     // [R, H]: RMSNorm of the last layer's output
  uint16_t* xs;                   // split operand [2][Rpad][H] (rows >= R stay zero)
  uint16_t* xs_i;                 // split operand [2][Rpad][I] of the down projection
  float* part;                    // segment partial tiles [segments][Rpad][um]
  float* rope_tab;                // [2][16][64]: cos, sin (x scaling factor) at positions 0..15
  const int* segtab;              // per kind: seg_off [tiles + 1] then first_seg [ncta]
  int tab_off[DP_KINDS];          // offset of each kind's table in segtab
  int tab_len;                    // ints in segtab (at most 2048)
  int ncta[DP_KINDS];             // CTAs each GEMM kind deals its pairs to
  int cta_off[DP_KINDS];          // ... starting at this CTA (ranks rotate through the grid)
  unsigned* bar;                  // [8 L + 2] zeroed; the last CTA out resets them
  int* err;
  int nst;                        // ring stages (set by the launcher)
  int pf_stages;                  // weight stages of the next GEMM phase copied during a row phase (clamped to nst)
  unsigned long long* trace;      // optional [phases][grid][4] timeline (%globaltimer)
};

// Segment table of one GEMM kind with `tiles` weight tiles of `kch` K chunks dealt to `ncta`
// CTAs: appends seg_off [tiles + 1] and first_seg [ncta] to tab; returns the segment count.
int dit_persist_segments(int tiles, int kch, int ncta, int* tab);

// Shared memory of the kernel for Rpad activation rows and an attention mode; *nst receives
// the ring depth.
size_t dit_persist_smem(int rpad, int um, int att_mode, int* nst);
cudaError_t dit_persist_configure();
// One CTA per SM when the device can hold it, else 0.
int dit_persist_grid();
cudaError_t launch_dit_persist(const DitPersistArgs& a, int grid, cudaStream_t st);

// Host state of one model's persistent forward: buffers allocated once for the most rows the
// model takes (so captured graphs never see them move), the weight tensor maps, the segment
// tables and the activation maps per padded row count.
struct PersistStack {
  int grid = -1;             // -1: not prepared; 0: unsupported shape or device
  int rmax = 0;              // activation rows the buffers hold (a multiple of 32, <= 256)
  int um = 128;              // weight rows per GEMM unit (256 when rmax <= 64; env VX_DIT_UM)
  bool split_b = false;      // the activation planes as two copies (env VX_DIT_SPLIT_B=1)
  bool seq_ok = false;       // DP_ATT_SEQ supported (head_dim <= 64, even)
  bool decode_ok = false;    // DP_ATT_DECODE supported (head_dim <= 128, nh / nkv <= 16)
  LmStackView view;
  DitPersistLayer* layers = nullptr;
  CUtensorMap* maps = nullptr;                 // device [4 L]
  std::map<int, CUtensorMap*> xmaps;           // device [2] per padded row count
  float *x = nullptr, *x1 = nullptr, *part = nullptr, *rope_tab = nullptr;
  float* rope_pos = nullptr;                   // [positions][2][d/2] (decode attention)
  float* att_part = nullptr;                   // decode attention split partials
  unsigned* att_cnt = nullptr;                 // and their counters
  uint16_t *xs = nullptr, *xsi = nullptr;
  int* segtab = nullptr;
  unsigned* bar = nullptr;
  unsigned long long* trace = nullptr;         // optional phase timeline
  int tab_off[DP_KINDS] = {}, ncta[DP_KINDS] = {}, tab_len = 0;
  // weight stages of the next GEMM phase each CTA copies during a row phase (env VX_DIT_PF):
  // one keeps the row phase's L2 reads clear of the weight stream (8-row step 2.06 -> 2.03 ms,
  // 8-patch CFM 5.15 -> 5.12 ms against a full ring; none: 2.14 ms / 5.22 ms)
  int pf_stages = 1;
};
// Once, outside any capture: check the shape (hidden <= 2048, a multiple of 128), allocate
// for up to max_rows rows, build the weight maps and segment tables.  False (ps.grid = 0)
// when the persistent forward cannot run; *oom is set when an allocation failed.
// rope_positions > 0: also tabulate LongRoPE cos / sin for positions 0..rope_positions-1 (the
// decode attention reads the table instead of evaluating f64 sincos).
bool persist_stack_prepare(PersistStack& ps, const LmStackView& v, int max_rows, bool trace, bool* oom,
                           int rope_positions = 0);
// Activation maps for rpad rows (kept per count); false on failure.
bool persist_stack_rows(PersistStack& ps, int rpad);
void persist_stack_free(PersistStack& ps);
// The launch arguments shared by both attention modes for R rows of N sequences of S tokens
// (persist_stack_rows must have succeeded for R rounded up to 32).
DitPersistArgs persist_stack_args(const PersistStack& ps, int N, int S, const float* x_in, float* out, int* err);

}  // namespace vx
