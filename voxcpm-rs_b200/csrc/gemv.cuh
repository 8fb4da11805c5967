// Streamed bf16-weight GEMV (one activation row) with fused prologues / epilogues.
//
// y[n] = sum_k W[n,k] * x[k],  W bf16 [N,K] row-major (the checkpoint's [out,in] layout),
// x f32, f32 accumulation.  This is every `Linear` of the batch-1 decode step
// (reference src/minicpm4/attention.rs:102,153, mlp.rs:29,33 via burn::nn::Linear).
#pragma once
#include <cstdint>

namespace vx {

enum GemvEpi : int {
  EPI_STORE = 0,     // y[row] = acc (+ bias[row]) ; or residual[row] + res_scale*acc
  EPI_QKV_ROPE = 1,  // LongRoPE on q/k rows, k/v written into the static KV cache
  EPI_SILU_MUL = 2,  // act[i] = silu(gate_i) * up_i
  EPI_ARGMAX = 3,    // greedy LM head: argmax over rows, next-token embedding, pos++
};

enum GemvMap : int {
  MAP_LINEAR = 0,     // virtual group g -> rows [8g, 8g+8)
  MAP_ROPE_PAIRS = 1, // group pairs (j, j + d/16) of one head share a CTA (rotate_half pairs)
  MAP_GATE_UP = 2,    // group pairs (j, j + I/8): gate rows and matching up rows
};

struct RopeParams {
  // f64 quantities of MiniCpmLongRope::new (src/minicpm4/rope.rs:16-32)
  double inv_freq[128];
  double ext[128];
  double scaling_factor;
  int half;
};

struct GemvArgs {
  const uint16_t* W;  // [N, K] bf16 bits
  int N, K;
  int kc;              // K chunk per stage (K % kc == 0); kc in {256,...,2048}
  int groups_total;    // N / 8
  int groups_per_cta;
  int map_mode, map_param;

  // prologue: x (f32 [K]); optional RMSNorm (norm_w != nullptr)
  const float* x;
  const float* norm_w;
  float eps;

  // EPI_STORE
  float* y;
  const float* bias;
  const float* residual;  // if non-null: y = residual + res_scale * acc
  float res_scale;

  // EPI_QKV_ROPE
  int nh, nkv, hd;
  const RopeParams* rope;  // nullptr = no_rope
  const int* pos_ptr;      // device position (nullptr -> pos_val)
  int pos_val;
  float* q_out;            // [nh*hd]
  float* kcache;           // [nkv, s_max, hd] (this layer, this batch row)
  float* vcache;
  int s_max;

  // EPI_SILU_MUL
  int inter;
  float* act;  // [inter]

  // EPI_ARGMAX
  float* logits;            // optional [N]
  float2* partials;         // [gridDim.x] (value, index as float bits)
  unsigned int* counter;    // zero-initialised; reset by the last CTA
  int* token_out;           // token written here (index *step_ptr if step_ptr)
  int* step_ptr;            // optional device step counter (incremented)
  const uint16_t* embed;    // [N, K_embed] bf16 for the next-token embedding
  int embed_dim;
  float embed_scale;
  float* next_x;            // next input embedding [embed_dim]
  int* pos_inc;             // optional device position to increment

  int* err;  // device error word (bounded waits record VX_DEVICE_ERR_TIMEOUT here)

  // Optional copy of the normalised input vector (CTA 0 writes it), e.g. the final-norm
  // hidden state the greedy head sees, which the synthesis loop feeds to the DiT.
  float* norm_out;

  // Optional L2 prefetch of the next kernel's weights (split evenly over the CTAs), issued
  // once this CTA's first stages are in flight, so HBM stays busy across kernel boundaries.
  const void* pf_ptr;
  size_t pf_bytes;
};

}  // namespace vx
