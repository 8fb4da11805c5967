// Persistent non-causal MiniCPM-4 stack forward on tcgen05 (dit_persist.cu): arguments and
// host entry points.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

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

// GEMM phases deal their (128-row weight tile, 64-element K chunk) pairs to the first ncta
// CTAs in contiguous runs: CTA b < ncta takes pairs [b T / ncta, (b + 1) T / ncta) of T.  Every
// maximal run inside one tile is a segment; segments are numbered CTA-major (which is also
// tile-major), each writes its f32 partial tile to its own slot and the consumer sums a tile's
// slots in ascending order (deterministic).
enum { DP_KIND_QKV, DP_KIND_O, DP_KIND_GU, DP_KIND_DOWN, DP_KINDS };

struct DitPersistArgs {
  int L, H, I, nh, nkv, d;
  int S, N, R, Rpad;            // tokens per sequence, sequences, rows = N S, rows rounded up to 32
  float eps, res_scale, attn_scale;
  const DitPersistLayer* layers;  // device [L]
  const CUtensorMap* wmaps;       // device [L][4]: qkv, o, gate|up, down (128-row x 64 boxes)
  const CUtensorMap* xmaps;       // device [2]: the split operand as K = H and K = I
  const RopeParams* rope;         // null: no rope
  const float* final_norm;        // [H]
  const float* x_in;              // [R, H]: the input rows
  float* x;                       // [R, H]: each layer's input
  float* x1;                      // [R, H]: the residual stream after attention
  float* out;                     // [R, H]: RMSNorm of the last layer's output
  uint16_t* xs;                   // split operand [2][Rpad][H] (rows >= R stay zero)
  uint16_t* xs_i;                 // split operand [2][Rpad][I] of the down projection
  float* part;                    // segment partial tiles [segments][Rpad][128]
  float* rope_tab;                // [2][16][64]: cos, sin (x scaling factor) at positions 0..15
  const int* segtab;              // per kind: seg_off [tiles + 1] then first_seg [ncta]
  int tab_off[DP_KINDS];          // offset of each kind's table in segtab
  int tab_len;                    // ints in segtab (at most 2048)
  int ncta[DP_KINDS];             // CTAs each GEMM kind deals its pairs to
  unsigned* bar;                  // [8 L + 2] zeroed; the last CTA out resets them
  int* err;
  int nst;                        // ring stages (set by the launcher)
  unsigned long long* trace;      // optional [phases][grid][4] timeline (%globaltimer)
};

// Segment table of one GEMM kind with `tiles` weight tiles of `kch` K chunks dealt to `ncta`
// CTAs: appends seg_off [tiles + 1] and first_seg [ncta] to tab; returns the segment count.
int dit_persist_segments(int tiles, int kch, int ncta, int* tab);

// Shared memory of the kernel for Rpad activation rows; *nst receives the ring depth.
size_t dit_persist_smem(int rpad, int* nst);
cudaError_t dit_persist_configure();
// One CTA per SM when the device can hold it, else 0.
int dit_persist_grid();
cudaError_t launch_dit_persist(const DitPersistArgs& a, int grid, cudaStream_t st);

}  // namespace vx
