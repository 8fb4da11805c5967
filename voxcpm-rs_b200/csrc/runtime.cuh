// Host-side runtime shared by the C ABI translation units: the context, status handling
// and the kernel launcher declarations.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/voxcpm_b200.h"
#include "dit_persist.cuh"
#include "gemv.cuh"
#include "kernels.cuh"

namespace vx {

// Groups (or group pairs) per CTA so that a GEMV grid is about two CTAs per SM.
inline int pick_groups(int units, int target_ctas = 296) {
  int g = (units + target_ctas - 1) / target_ctas;
  return g < 1 ? 1 : g;
}

cudaError_t launch_gemv(GemvArgs a, int epi, cudaStream_t st, bool pdl, int* err);
cudaError_t gemv_configure();
int gemv_grid(const GemvArgs& a);
int gemv_pick_kc(int K);
cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_gemm_smallm(const GemmArgs& a, cudaStream_t st);
bool tc_gemm_supported(int M, int N, int K);
size_t tc_gemm_scratch_bytes(int M, int N, int K, int target_ctas);
cudaError_t launch_tc_gemm(const float* X, int ldx, int M, int N, int K, const uint16_t* W, const float* bias,
                           const float* R, float res_scale, float* Y, int ldy, void* scratch, unsigned* counters,
                           int* err, cudaStream_t st, int target_ctas);
// The same GEMM with its activations already split by their producer into the buffer
// tc_gemm_presplit_buffer(scratch): rows [0, M) bf16(x), rows [M, 2M) bf16(x - bf16(x)),
// row stride K (no split kernel launch).
uint16_t* tc_gemm_presplit_buffer(void* scratch);
cudaError_t launch_tc_gemm_presplit(int M, int N, int K, const uint16_t* W, const float* bias, const float* R,
                                    float res_scale, float* Y, int ldy, void* scratch, unsigned* counters, int* err,
                                    cudaStream_t st, int target_ctas);
// xs: also (y_out may be null: instead) store y as the tcgen05 GEMM's split operand [2 rows, hidden]
cudaError_t launch_rmsnorm_residual(const float* x, const float* r, const float* w, float resid_scale, float eps,
                                    int rows, int hidden, float* h_out, float* y_out, cudaStream_t st,
                                    uint16_t* xs = nullptr);
cudaError_t launch_rope_table(const RopeParams* rp, int n_pos, int half, float* out, cudaStream_t st);
cudaError_t launch_rope_scatter(const float* qkv, int B, int S, int nh, int nkv, int d, const RopeParams* rope,
                                int pos0, float* q_out, float* kcache, float* vcache, int s_max, cudaStream_t st,
                                const int* pos_ptr = nullptr);
cudaError_t launch_argmax_rows(const float* logits, int B, int V, const int* step, int* tokens, int ld_tokens,
                               const uint16_t* E, int H, float scale, float* next_x, cudaStream_t st);
cudaError_t launch_advance(int* pos, int* step, bool inc_pos, cudaStream_t st);
cudaError_t launch_rope_apply(float* x, int B, int H, int S, int d, const float* cos, const float* sin,
                              cudaStream_t st);
// xs: write silu(gate)*up as the tcgen05 GEMM's split operand [2M, inter] instead of act
cudaError_t launch_silu_mul(const float* gu, int M, int inter, float* act, cudaStream_t st, uint16_t* xs = nullptr);
cudaError_t launch_embed(const uint16_t* E, const int* ids, int n, int H, int V, float scale, float* out,
                         cudaStream_t st);
cudaError_t launch_fsq_quant(float* h, size_t n, float scale, cudaStream_t st);
cudaError_t launch_cfg_euler(const float* out2b, float* x, int B, int n, double cfg, double dt, int zero_star,
                             cudaStream_t st);

// A growable device scratch region owned by a context (op-level calls that need
// workspace).  Counters that kernels use for last-CTA detection live in a separate
// zero-initialised region that kernels reset after use.
struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};

}  // namespace vx

struct vx_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string last_error;
  std::atomic<int> cancel{0};
  vx::Scratch scratch;
  unsigned int* counters = nullptr;  // 4096 zeroed counters
  int* dev_err = nullptr;            // device error word written by bounded waits
  bool pdl = true;                   // programmatic dependent launch between decode kernels
  int gemv_ctas = 296;               // target GEMV grid (CTAs); env VX_GEMV_CTAS overrides
  bool tc_gemm = true;               // tcgen05 path for few-row GEMMs (env VX_TC_GEMM=0: CUDA cores)
  bool presplit = true;              // producers write the tcgen05 GEMM's split operand (env VX_PRESPLIT=0: a split kernel)
  bool l2_prefetch = false;          // decode kernels prefetch the next kernel's weights into L2
                                     // (env VX_L2_PREFETCH=1; measured: no gain with separate kernels)
  bool persist = true;               // batch-1 decode step as one persistent launch (env VX_PERSIST=0: 141 launches)
  int persist_nst = 0;               // its ring depth cap in stages, 0 = shared-memory limit (env VX_PERSIST_NST)
  int persist_grid = 0;              // its CTA count cap (env VX_PERSIST_GRID), 0 = one CTA per SM
  int persist_inflight = 0;          // its ring copies in flight cap (env VX_PERSIST_INFLIGHT), 0 = none
  int persist_mlp_pf = 0;            // its MLP stages staged in L2 per earlier phase (env VX_PERSIST_MLP_PF)
  int persist_merge_tiles = 16;      // caches of more tiles merge the attention splits once per KV head
                                     // (env VX_PERSIST_MERGE_TILES; fewer: every o_proj CTA merges)
  int persist_pf = 0;                // its L2 prefetch distance beyond the ring, in stages (env VX_PERSIST_PF)
  int persist_ef = 0;                // its weight copies mark L2 lines evict-first (env VX_PERSIST_EF)
  bool att_rope_fused = true;        // few-row uncached attention applies RoPE at load (env VX_ATT_ROPE_FUSED=0: separate pass)
};

namespace vx {

inline int fail(vx_ctx* ctx, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (ctx) ctx->last_error = buf;
  return code;
}

inline int cuda_fail(vx_ctx* ctx, cudaError_t e, const char* where) {
  return fail(ctx, VX_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

#define VX_CUDA(ctx, call)                                   \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return vx::cuda_fail(ctx, e_, #call); \
  } while (0)

// Op-level calls run on the caller's stream; NULL is the legacy default stream (as in
// cuBLAS), so work queued by a framework on its default stream is ordered before them.
inline cudaStream_t pick_stream(vx_ctx*, vx_stream s) { return reinterpret_cast<cudaStream_t>(s); }

// Ensure the context scratch has at least `bytes`; returns nullptr on failure.
void* ctx_scratch(vx_ctx* ctx, size_t bytes);

inline double residual_scale_of(const vx_minicpm4_config& c) {
  // MiniCpmDecoderLayer::new (minicpm4/layer.rs:20-22): scale_depth (f32) / sqrt(L) in f64
  return c.use_mup ? (double)c.scale_depth / std::sqrt((double)c.num_hidden_layers) : 1.0;
}

int fill_rope_params(const vx_minicpm4_config& c, RopeParams* rp, std::string* err);

// Workspace for linear(): bf16-split activations and split-K partials of the tcgen05 path,
// plus its zeroed tile counters.  Sized for up to 128 rows, N <= max_n, K <= max_k.
struct LinearWorkspace {
  void* scratch = nullptr;
  size_t bytes = 0;
  unsigned* counters = nullptr;  // 1024 zeroed words
};
int workspace_init(vx_ctx* ctx, LinearWorkspace* ws, int max_n, int max_k);
void workspace_free(LinearWorkspace* ws);

// burn::nn::Linear for M rows: Y[m, :] = X[m, :] . W^T (+ bias) (or Y = R + s * (...)).
// M == 1: streamed GEMV; 2..128-row chunks: tcgen05 GEMM; otherwise the CUDA-core GEMM.
int linear(vx_ctx* ctx, const LinearWorkspace* ws, const float* X, int ldx, int M, int N, int K, const uint16_t* W,
           const float* bias, const float* R, float res_scale, float* Y, int ldy, cudaStream_t st);
// Whether linear() over M rows takes the tcgen05 path as one chunk, so that the producer of X
// may write it split (tc_gemm_presplit_buffer(ws->scratch)) and linear_presplit() run the GEMM.
bool presplit_ok(vx_ctx* ctx, const LinearWorkspace* ws, int M, int N, int K);
int linear_presplit(vx_ctx* ctx, const LinearWorkspace* ws, int M, int N, int K, const uint16_t* W, const float* bias,
                    const float* R, float res_scale, float* Y, int ldy, cudaStream_t st);

// Greedy LM decoding, split for the synthesis loop (lm.cu).
vx_ctx* lm_ctx(vx_lm* lm);
const LinearWorkspace* lm_workspace(const vx_lm* lm);
// Grow the forward() work buffers to `rows` token rows (so a later capture allocates nothing).
int lm_prepare_rows(vx_lm* lm, size_t rows);
cudaError_t tc_gemm_configure();
// AudioVAE convolutions on tcgen05 (vae_tc.cu).  launch_vae_split writes X [B, C, T] (after
// the optional SR conditioning and snake) as the bf16 hi / lo operand xs [2][B][T][C];
// launch_vae_tc_conv runs a pointwise conv (s = 1, A = W [Cout, Cin]) or a causal transposed
// conv (stride s, A = the phase-folded weight [vae_tc_rows(Cout, s), 2 Cin]) over it.
cudaError_t vae_tc_configure();
int vae_tc_rows(int cout, int s);
// hist (streaming, transposed-conv inputs only): the previous chunk's last frame [B, C],
// written as row 0 ahead of the chunk; the conv then reads with row_off = 1.
cudaError_t launch_vae_split(const float* X, int B, int C, int T, const float* alpha, const float* sr_scale,
                             const float* sr_bias, uint16_t* xs, cudaStream_t st, const float* hist = nullptr);
cudaError_t launch_vae_tc_conv(const uint16_t* xs, int B, int T_in, int Cin, int Cout, int s, const uint16_t* A,
                               const float* bias, const float* R, float* Y, int* err, cudaStream_t st,
                               int row_off = 0);
int lm_hidden_size(const vx_lm* lm);
const float* lm_hid_norm(const vx_lm* lm);
int lm_greedy_begin(vx_lm* lm, const int32_t* prompt_ids, int n_prompt, int n_steps);
int lm_greedy_step(vx_lm* lm);
// Batched greedy decode (B rows in lockstep, equal prompt lengths): prefill + first pick, then
// one graph-replayed step per call; the final-norm hiddens [B, H] and the ids
// [step][max_batch] stay on the device.
int lm_batch_begin(vx_lm* lm, const int32_t* prompt_ids, int B, int n_prompt, int n_steps);
int lm_batch_step(vx_lm* lm);
const float* lm_batch_hidden(const vx_lm* lm);
const int* lm_batch_tokens(const vx_lm* lm);
int lm_max_batch(const vx_lm* lm);
int lm_vocab_size(const vx_lm* lm);
// A model's stack as the persistent DiT-forward kernel sees it (dit_persist.cuh).
void lm_stack_view(const vx_lm* lm, LmStackView* v);
void lm_dims(const vx_lm* lm, int* L, int* H, int* I, int* qs, int* ks, int* V);
int lm_max_length(const vx_lm* lm);
// DiT / VAE accessors (dit.cu, vae.cu).
int cfm_solve_enqueue(vx_dit* d, const float* mu, const float* cond, const float* z, int B, int C_mu, int T, int Tc,
                      int n_timesteps, float cfg_value, float sway_sampling_coef, int use_cfg_zero_star,
                      float* x_out);
int dit_hidden_size(const vx_dit* d);
int dit_trace_copy(vx_dit* d, unsigned long long* out, int n, int* grid, int* phases);
vx_lm* dit_decoder(vx_dit* d, int* H, int* C);
struct VaeDims {
  int latent, dim, nblocks, rates[8], n_buckets;  // n_buckets 0: no sample-rate conditioning
};
void vae_dims(const vx_vae* v, VaeDims* out);
void voxcpm2_parts(vx_voxcpm2* m, vx_lm** base, vx_lm** res, vx_lm** enc, vx_dit** dit, int dims[6]);
vx_ctx* dit_ctx(vx_dit* d);
int dit_in_channels(const vx_dit* d);
vx_ctx* vae_ctx(vx_vae* v);
int vae_latent(const vx_vae* v);
int vae_hop(const vx_vae* v);

}  // namespace vx
