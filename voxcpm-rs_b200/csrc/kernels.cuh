// Argument blocks of the attention and few-row GEMM kernels (shared by the kernels and
// the host runtime).
#pragma once
#include <cstdint>

namespace vx {

struct AttnDecodeArgs {
  const float* q;       // [B, nh*d]
  const float* kcache;  // [B, nkv, s_max, d]
  const float* vcache;
  int B, nh, nkv, d, s_max;
  const int* pos_ptr;  // if non-null: len = *pos_ptr + 1 (device position of the new token)
  int len;             // otherwise the filled length
  float scale;
  int nsplit;
  float* partials;         // [B, nkv, nsplit, n_rep, d + 2]
  unsigned int* counters;  // [B * nkv], zero-initialised; reset by the kernel
  float* out;              // [B, nh*d]
};

struct AttnPrefillArgs {
  const float* q;  // [B, S, nh*d]
  const float* k;  // [B, nkv, s_max, d]
  const float* v;
  int B, S, nh, nkv, d, s_max;
  float scale;
  int causal;
  float* out;    // [B, S, nh*d]
  uint16_t* xs;  // optional: out written instead as the tcgen05 GEMM's split operand [2 B S, nh*d]
  // optional (no KV cache, S <= ATT_FUSED_ROPE_MAX_S): q, k, v read from the fused projection
  // rows [B*S, (nh+2nkv)*d] instead of q/k/v, with LongRoPE applied to q and k as they are
  // loaded (rope_tab: cos / sin rows [S][2][d/2] of positions 0..S-1; null: no rotation);
  // k, v and s_max are then unused
  const float* qkv;
  const float* rope_tab;
};
constexpr int ATT_FUSED_ROPE_MAX_S = 64;

struct GemmArgs {
  const float* X;  // [M, K] (row stride ldx)
  int ldx;
  const uint16_t* W;  // [N, K]
  const float* bias;  // [N] or null
  const float* R;     // [M, N] residual or null (row stride ldy); may alias Y
  float res_scale;
  float* Y;  // [M, N] (row stride ldy)
  int ldy;
  int M, N, K;
};

}  // namespace vx
