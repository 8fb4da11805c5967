// VoxCPM2 autoregressive model: prefill, dit_step, lm_step and the inference loop
// (reference src/voxcpm2/model.rs:128-375), with the local feature encoder
// (src/locenc.rs:32-44) and the scalar-quantization layer (src/fsq.rs:24-29).
//
// The model object composes four MiniCPM-4 stacks the library already runs (the base LM
// with its tied vocabulary, the residual LM, the LocEnc encoder, the LocDiT decoder inside
// vx_dit) with the projection layers of VoxCpm2Model.  Every step is queued on the context
// stream; the loop never waits for the GPU to finish a step before queueing the next one:
// the stop head's argmax is written to device memory and copied to pinned host memory, and
// the host reads the flag of step i only after it has queued step i + 1 (which is
// discarded if step i stopped), so the device always has the next step's work.
#include <cstring>
#include <vector>

#include "common.cuh"
#include "runtime.cuh"

using namespace vx;

namespace {

// LocEnc input rows (locenc.rs:35-39): seq[n, 0, :] = the special token, seq[n, 1 + p, :] =
// in_proj(x(n, p, :)) for the patch's P frames.  x(n, p, c) is read from [N, P, D]
// (row-major frames, the reference's [B, T, P, D]) or from [N, D, P] (channel-major, the
// layout the CFM solve returns).  grid (N * (P + 1), ceil(He / 256)), D % 8 == 0.
__global__ void __launch_bounds__(256) locenc_seq_kernel(const float* __restrict__ x, int P, int D, int chan_major,
                                                         const uint16_t* __restrict__ W, const float* __restrict__ b,
                                                         const float* __restrict__ special, int He,
                                                         float* __restrict__ seq) {
  extern __shared__ float xs[];  // [D]
  const int n = blockIdx.x / (P + 1), r = blockIdx.x % (P + 1);
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  float* dst = seq + ((size_t)n * (P + 1) + r) * He;
  if (r == 0) {  // uniform per block
    if (h < He) dst[h] = special[h];
    return;
  }
  const int p = r - 1;
  for (int c = threadIdx.x; c < D; c += blockDim.x)
    xs[c] = chan_major ? x[((size_t)n * D + c) * P + p] : x[((size_t)n * P + p) * D + c];
  __syncthreads();
  if (h >= He) return;
  const uint4* w = reinterpret_cast<const uint4*>(W + (size_t)h * D);
  float acc = 0.f;
  for (int c8 = 0; c8 < D / 8; ++c8) acc = dot8(__ldg(w + c8), xs + c8 * 8, acc);
  dst[h] = acc + b[h];
}

// out[r, :] = a[r, :] * ma[r] + b[r, :] * mb[r]   (prefill's text / feature mixing,
// model.rs:147-150)
__global__ void mask_mix_kernel(const float* __restrict__ a, const float* __restrict__ ma,
                                const float* __restrict__ b, const float* __restrict__ mb, int rows, int H,
                                float* __restrict__ out) {
  const size_t n = (size_t)rows * H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / H);
    out[i] = a[i] * ma[r] + b[i] * mb[r];
  }
}

// The residual LM's prefill input before fusion_concat_proj (model.rs:157-166):
// out[r, 0:H] = fsq(enc)[r] * fm[r] + enc[r] * tm[r];  out[r, H:2H] = femb[r] * fm[r].
__global__ void fusion_rows_kernel(const float* __restrict__ enc, const float* __restrict__ fsq,
                                   const float* __restrict__ femb, const float* __restrict__ tm,
                                   const float* __restrict__ fm, int rows, int H, float* __restrict__ out) {
  const size_t n = (size_t)rows * H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / H), h = (int)(i % H);
    out[(size_t)r * 2 * H + h] = fsq[i] * fm[r] + enc[i] * tm[r];
    out[(size_t)r * 2 * H + H + h] = femb[i] * fm[r];
  }
}

// Stop head of one step (model.rs:244-253): logits = stop_head(silu(h)) with h =
// stop_proj(lm_hidden) already formed; flag = argmax == 1 (ties -> index 0).  One block.
__global__ void __launch_bounds__(256) stop_head_kernel(const float* __restrict__ h, const uint16_t* __restrict__ Wh,
                                                        int H, float* __restrict__ logits, int* __restrict__ flag) {
  __shared__ float red[2][8];
  float a0 = 0.f, a1 = 0.f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float s = silu(h[k]);
    a0 = fmaf(__uint_as_float(((uint32_t)Wh[k]) << 16), s, a0);
    a1 = fmaf(__uint_as_float(((uint32_t)Wh[H + k]) << 16), s, a1);
  }
  a0 = warp_sum(a0);
  a1 = warp_sum(a1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][warp] = a0;
    red[1][warp] = a1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float l0 = 0.f, l1 = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      l0 += red[0][w];
      l1 += red[1][w];
    }
    logits[0] = l0;
    logits[1] = l1;
    *flag = l1 > l0 ? 1 : 0;
  }
}

int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, 148 * 8); }

}  // namespace

struct vx_voxcpm2 {
  vx_ctx* ctx = nullptr;
  vx_lm *base = nullptr, *res = nullptr, *enc = nullptr;
  vx_dit* dit = nullptr;
  int H = 0, He = 0, Hd = 0, D = 0, P = 0, Lq = 0, max_len = 0;
  float sq_scale = 9.f;
  LinearWorkspace ws;
  // weights (bf16 bit patterns [out, in]; f32 biases and special token)
  void* slab = nullptr;
  float* special = nullptr;
  uint16_t *enc_in_w = nullptr, *enc_to_lm_w = nullptr, *lm_to_dit_w = nullptr, *res_to_dit_w = nullptr,
           *fusion_w = nullptr, *stop_proj_w = nullptr, *stop_head_w = nullptr, *fsq_in_w = nullptr,
           *fsq_out_w = nullptr;
  float *enc_in_b = nullptr, *enc_to_lm_b = nullptr, *lm_to_dit_b = nullptr, *res_to_dit_b = nullptr,
        *fusion_b = nullptr, *stop_proj_b = nullptr, *fsq_in_b = nullptr, *fsq_out_b = nullptr;
  // AR-step state and buffers
  float* fuse_in = nullptr;   // [2H]: lm_hidden (after FSQ) | curr_embed
  float* lm_tmp = nullptr;    // [H] base LM output before FSQ
  float* lat = nullptr;       // [rows, Lq] FSQ latent
  float* res_in = nullptr;    // [H]
  float* res_hidden = nullptr;  // [H]
  float* mu = nullptr;        // [2 Hd]
  float* stop_h = nullptr;    // [H]
  float* stop_logits = nullptr;  // [max_len, 2]
  int* stop_flags = nullptr;  // [max_len]
  int* h_flags = nullptr;     // pinned [max_len]
  float* patch[2] = {nullptr, nullptr};  // [D, P] channel-major
  float* latent = nullptr;    // [D, max_len * P]
  float* noise = nullptr;     // [max_len, D, P]
  float *enc_seq = nullptr, *enc_out = nullptr;  // [rows, He] LocEnc rows
  size_t enc_rows = 0;
  cudaEvent_t ev[2] = {nullptr, nullptr};
  // the generation in progress (vx_voxcpm2_begin / advance): next patch index, the CFM's
  // current condition buffer, the options, and whether the loop has ended
  int s_i = 0, s_cur = 0, s_min_len = 0, s_max_len = 0, s_steps = 0;
  float s_cfg = 0.f;
  bool s_finished = true, s_active = false;
  // prefill buffers (grown to S rows)
  int pf_cap = 0;
  int* pf_ids = nullptr;
  float *pf_tm = nullptr, *pf_fm = nullptr, *pf_feat = nullptr, *pf_femb = nullptr, *pf_temb = nullptr,
        *pf_comb = nullptr, *pf_enc = nullptr, *pf_fsq = nullptr, *pf_fuse = nullptr, *pf_rin = nullptr,
        *pf_rout = nullptr;
};

namespace {

void free_prefill(vx_voxcpm2* m) {
  for (float** p : {&m->pf_tm, &m->pf_fm, &m->pf_feat, &m->pf_femb, &m->pf_temb, &m->pf_comb, &m->pf_enc, &m->pf_fsq,
                    &m->pf_fuse, &m->pf_rin, &m->pf_rout}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  if (m->pf_ids) cudaFree(m->pf_ids);
  m->pf_ids = nullptr;
  m->pf_cap = 0;
}

int ensure_prefill(vx_voxcpm2* m, int S) {
  if (S <= m->pf_cap) return VX_OK;
  free_prefill(m);
  const size_t s = S, H = m->H;
  bool ok = cudaMalloc(&m->pf_ids, s * 4) == cudaSuccess && cudaMalloc(&m->pf_tm, s * 4) == cudaSuccess &&
            cudaMalloc(&m->pf_fm, s * 4) == cudaSuccess &&
            cudaMalloc(&m->pf_feat, s * m->P * m->D * 4) == cudaSuccess &&
            cudaMalloc(&m->pf_femb, s * H * 4) == cudaSuccess && cudaMalloc(&m->pf_temb, s * H * 4) == cudaSuccess &&
            cudaMalloc(&m->pf_comb, s * H * 4) == cudaSuccess && cudaMalloc(&m->pf_enc, s * H * 4) == cudaSuccess &&
            cudaMalloc(&m->pf_fsq, s * H * 4) == cudaSuccess && cudaMalloc(&m->pf_fuse, s * 2 * H * 4) == cudaSuccess &&
            cudaMalloc(&m->pf_rin, s * H * 4) == cudaSuccess && cudaMalloc(&m->pf_rout, s * H * 4) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    free_prefill(m);
    return fail(m->ctx, VX_ERR_OOM, "voxcpm2: prefill buffers (%d rows) allocation failed", S);
  }
  m->pf_cap = S;
  return VX_OK;
}

int ensure_enc_rows(vx_voxcpm2* m, size_t patches) {
  const size_t rows = patches * (m->P + 1);
  if (rows <= m->enc_rows) return VX_OK;
  if (m->enc_seq) cudaFree(m->enc_seq);
  if (m->enc_out) cudaFree(m->enc_out);
  m->enc_seq = m->enc_out = nullptr;
  m->enc_rows = 0;
  if (cudaMalloc(&m->enc_seq, rows * m->He * 4) != cudaSuccess ||
      cudaMalloc(&m->enc_out, rows * m->He * 4) != cudaSuccess) {
    cudaGetLastError();
    return fail(m->ctx, VX_ERR_OOM, "voxcpm2: LocEnc buffers allocation failed");
  }
  m->enc_rows = rows;
  return lm_prepare_rows(m->enc, rows);
}

int lin(vx_voxcpm2* m, const float* X, int ldx, int M, int N, int K, const uint16_t* W, const float* b, float* Y,
        int ldy) {
  return linear(m->ctx, &m->ws, X, ldx, M, N, K, W, b, nullptr, 1.f, Y, ldy, m->ctx->stream);
}

// VoxCpmLocEnc::forward + enc_to_lm_proj for N patches x (layout as locenc_seq_kernel):
// out [N, H] (row stride ldo).
int locenc_to_lm(vx_voxcpm2* m, const float* x, int N, int chan_major, float* out, int ldo) {
  vx_ctx* ctx = m->ctx;
  cudaStream_t st = ctx->stream;
  int rc = ensure_enc_rows(m, N);
  if (rc) return rc;
  count_launch();
  locenc_seq_kernel<<<dim3(N * (m->P + 1), (m->He + 255) / 256), 256, m->D * sizeof(float), st>>>(
      x, m->P, m->D, chan_major, m->enc_in_w, m->enc_in_b, m->special, m->He, m->enc_seq);
  VX_CUDA(ctx, cudaGetLastError());
  rc = vx_lm_forward(m->enc, m->enc_seq, N, m->P + 1, 0, 0, m->enc_out);
  if (rc) return rc;
  // the cls row of every patch (outputs.narrow(1, 0, 1), locenc.rs:42) -> enc_to_lm_proj
  return lin(m, m->enc_out, (m->P + 1) * m->He, N, m->H, m->He, m->enc_to_lm_w, m->enc_to_lm_b, out, ldo);
}

// ScalarQuantizationLayer::forward over `rows` rows of x [rows, H] -> out (row stride ldo).
int fsq_rows(vx_voxcpm2* m, const float* x, int rows, float* out, int ldo) {
  int rc = lin(m, x, m->H, rows, m->Lq, m->H, m->fsq_in_w, m->fsq_in_b, m->lat, m->Lq);
  if (rc) return rc;
  VX_CUDA(m->ctx, launch_fsq_quant(m->lat, (size_t)rows * m->Lq, m->sq_scale, m->ctx->stream));
  return lin(m, m->lat, m->Lq, rows, m->H, m->Lq, m->fsq_out_w, m->fsq_out_b, out, ldo);
}

// dit_step (model.rs:215-256) for step i: mu = [lm_to_dit(lm_hidden) | res_to_dit(res_hidden)],
// CFM solve (sway 1, CFG-zero-star) with cond = patch[cur], z = noise[i] -> patch[cur ^ 1],
// stacked into the latent, and the stop head -> stop_flags[i] (copied to pinned memory).
int dit_step(vx_voxcpm2* m, int i, int cur, int timesteps, float cfg_value) {
  vx_ctx* ctx = m->ctx;
  cudaStream_t st = ctx->stream;
  const int Hd = m->Hd, DP = m->D * m->P;
  int rc = lin(m, m->fuse_in, m->H, 1, Hd, m->H, m->lm_to_dit_w, m->lm_to_dit_b, m->mu, 2 * Hd);
  if (!rc) rc = lin(m, m->res_hidden, m->H, 1, Hd, m->H, m->res_to_dit_w, m->res_to_dit_b, m->mu + Hd, 2 * Hd);
  if (!rc)
    rc = cfm_solve_enqueue(m->dit, m->mu, m->patch[cur], m->noise + (size_t)i * DP, 1, 2 * Hd, m->P, m->P, timesteps,
                           cfg_value, 1.0f, 1, m->patch[cur ^ 1]);
  if (rc) return rc;
  // stack_pred_feats (model.rs:283-287): latent[:, i*P + p] = pred[:, p]
  VX_CUDA(ctx, cudaMemcpy2DAsync(m->latent + (size_t)i * m->P, (size_t)m->max_len * m->P * 4, m->patch[cur ^ 1],
                                 (size_t)m->P * 4, (size_t)m->P * 4, m->D, cudaMemcpyDeviceToDevice, st));
  rc = lin(m, m->fuse_in, m->H, 1, m->H, m->H, m->stop_proj_w, m->stop_proj_b, m->stop_h, m->H);
  if (rc) return rc;
  count_launch();
  stop_head_kernel<<<1, 256, 0, st>>>(m->stop_h, m->stop_head_w, m->H, m->stop_logits + 2 * (size_t)i,
                                      m->stop_flags + i);
  VX_CUDA(ctx, cudaGetLastError());
  VX_CUDA(ctx, cudaMemcpyAsync(m->h_flags + i, m->stop_flags + i, 4, cudaMemcpyDeviceToHost, st));
  VX_CUDA(ctx, cudaEventRecord(m->ev[i & 1], st));
  return VX_OK;
}

// lm_step (model.rs:261-279) on the patch the last dit_step predicted (patch[p], [D, P]).
int lm_step(vx_voxcpm2* m, int p) {
  const int H = m->H;
  float* lm_hidden = m->fuse_in;
  float* curr = m->fuse_in + H;
  int rc = locenc_to_lm(m, m->patch[p], 1, 1, curr, H);
  if (!rc) rc = vx_lm_forward_step(m->base, curr, m->lm_tmp);
  if (!rc) rc = fsq_rows(m, m->lm_tmp, 1, lm_hidden, H);
  if (!rc) rc = lin(m, m->fuse_in, 2 * H, 1, H, 2 * H, m->fusion_w, m->fusion_b, m->res_in, H);
  if (!rc) rc = vx_lm_forward_step(m->res, m->res_in, m->res_hidden);
  return rc;
}

// VoxCpm2Model::prefill (model.rs:128-207) for one sequence of S positions.
int prefill(vx_voxcpm2* m, const int32_t* ids, const float* tmask, const float* fmask, const float* feat, int S) {
  vx_ctx* ctx = m->ctx;
  cudaStream_t st = ctx->stream;
  const int H = m->H, V = lm_vocab_size(m->base);
  for (int i = 0; i < S; ++i)
    if (ids[i] < 0 || ids[i] >= V) return fail(ctx, VX_ERR_ARG, "text token %d at %d outside the vocabulary", ids[i], i);
  int rc = ensure_prefill(m, S);
  if (!rc) rc = ensure_enc_rows(m, S);
  if (rc) return rc;
  VX_CUDA(ctx, cudaMemcpyAsync(m->pf_ids, ids, (size_t)S * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(m->pf_tm, tmask, (size_t)S * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(m->pf_fm, fmask, (size_t)S * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(m->pf_feat, feat, (size_t)S * m->P * m->D * 4, cudaMemcpyDefault, st));
  // 1) feat_encoder + enc_to_lm_proj; 2) embed * scale_emb; 3) masked mix
  rc = locenc_to_lm(m, m->pf_feat, S, 0, m->pf_femb, H);
  if (!rc) rc = vx_lm_embed(m->base, m->pf_ids, S, m->pf_temb);
  if (rc) return rc;
  count_launch();
  mask_mix_kernel<<<grid_for((size_t)S * H), 256, 0, st>>>(m->pf_temb, m->pf_tm, m->pf_femb, m->pf_fm, S, H,
                                                            m->pf_comb);
  VX_CUDA(ctx, cudaGetLastError());
  // 5) base LM prefill (causal, cache filled), FSQ on the audio rows
  rc = vx_lm_forward(m->base, m->pf_comb, 1, S, 1, 1, m->pf_enc);
  for (int r0 = 0; !rc && r0 < S; r0 += 128) {
    const int rows = std::min(128, S - r0);
    rc = fsq_rows(m, m->pf_enc + (size_t)r0 * H, rows, m->pf_fsq + (size_t)r0 * H, H);
  }
  if (rc) return rc;
  count_launch();
  fusion_rows_kernel<<<grid_for((size_t)S * H), 256, 0, st>>>(m->pf_enc, m->pf_fsq, m->pf_femb, m->pf_tm, m->pf_fm, S,
                                                               H, m->pf_fuse);
  VX_CUDA(ctx, cudaGetLastError());
  // 6) residual LM prefill
  rc = lin(m, m->pf_fuse, 2 * H, S, H, 2 * H, m->fusion_w, m->fusion_b, m->pf_rin, H);
  if (!rc) rc = vx_lm_forward(m->res, m->pf_rin, 1, S, 1, 1, m->pf_rout);
  if (rc) return rc;
  // the last position starts the loop: lm_hidden = enc_outputs[S-1], residual_hidden
  VX_CUDA(ctx, cudaMemcpyAsync(m->fuse_in, m->pf_fuse + (size_t)(S - 1) * 2 * H, (size_t)H * 4,
                               cudaMemcpyDeviceToDevice, st));
  VX_CUDA(ctx, cudaMemcpyAsync(m->res_hidden, m->pf_rout + (size_t)(S - 1) * H, (size_t)H * 4,
                               cudaMemcpyDeviceToDevice, st));
  return VX_OK;
}

}  // namespace

extern "C" {

int vx_voxcpm2_create(vx_lm* base_lm, vx_lm* residual_lm, vx_lm* encoder, vx_dit* dit, int feat_dim, int patch_size,
                      int sq_latent_dim, int sq_scale, int max_len, vx_voxcpm2** out) {
  if (!base_lm || !residual_lm || !encoder || !dit || !out) return VX_ERR_ARG;
  *out = nullptr;
  vx_ctx* ctx = lm_ctx(base_lm);
  if (lm_ctx(residual_lm) != ctx || lm_ctx(encoder) != ctx || dit_ctx(dit) != ctx)
    return fail(ctx, VX_ERR_ARG, "voxcpm2: the models must share one context");
  const int H = lm_hidden_size(base_lm), He = lm_hidden_size(encoder), Hd = dit_hidden_size(dit);
  if (lm_hidden_size(residual_lm) != H) return fail(ctx, VX_ERR_CONFIG, "voxcpm2: residual LM width != base LM width");
  if (lm_vocab_size(base_lm) <= 0) return fail(ctx, VX_ERR_CONFIG, "voxcpm2: the base LM needs its vocabulary");
  if (dit_in_channels(dit) != feat_dim) return fail(ctx, VX_ERR_CONFIG, "voxcpm2: DiT channels != feat_dim");
  if (feat_dim <= 0 || feat_dim % 8 || patch_size <= 0 || sq_latent_dim <= 0 || sq_latent_dim % 64 || sq_scale <= 0 ||
      max_len <= 0 || H % 64 || He % 64 || Hd % 8)
    return fail(ctx, VX_ERR_CONFIG, "voxcpm2: unsupported dimensions");
  cudaSetDevice(ctx->device);
  vx_voxcpm2* m = new vx_voxcpm2();
  m->ctx = ctx;
  m->base = base_lm;
  m->res = residual_lm;
  m->enc = encoder;
  m->dit = dit;
  m->H = H;
  m->He = He;
  m->Hd = Hd;
  m->D = feat_dim;
  m->P = patch_size;
  m->Lq = sq_latent_dim;
  m->sq_scale = (float)sq_scale;
  m->max_len = max_len;
  // one slab for the weights: bf16 matrices, then f32 vectors
  const size_t nw = (size_t)He * feat_dim + (size_t)H * He + 2 * (size_t)Hd * H + 2 * (size_t)H * H + (size_t)H * H +
                    2 * (size_t)H + 2 * (size_t)sq_latent_dim * H;
  const size_t nf = (size_t)He * 2 + H + 2 * (size_t)Hd + H + H + sq_latent_dim + H;
  const size_t wbytes = ((nw * 2 + 255) & ~size_t(255)) + nf * 4;
  auto fail_free = [&](int code, const char* what) {
    vx_voxcpm2_destroy(m);
    return fail(ctx, code, "%s", what);
  };
  if (cudaMalloc(&m->slab, wbytes) != cudaSuccess) {
    cudaGetLastError();
    return fail_free(VX_ERR_OOM, "voxcpm2: weight allocation failed");
  }
  uint16_t* wp = static_cast<uint16_t*>(m->slab);
  auto takew = [&](size_t n) {
    uint16_t* p = wp;
    wp += n;
    return p;
  };
  m->enc_in_w = takew((size_t)He * feat_dim);
  m->enc_to_lm_w = takew((size_t)H * He);
  m->lm_to_dit_w = takew((size_t)Hd * H);
  m->res_to_dit_w = takew((size_t)Hd * H);
  m->fusion_w = takew(2 * (size_t)H * H);
  m->stop_proj_w = takew((size_t)H * H);
  m->stop_head_w = takew(2 * (size_t)H);
  m->fsq_in_w = takew((size_t)sq_latent_dim * H);
  m->fsq_out_w = takew((size_t)H * sq_latent_dim);
  float* fp = reinterpret_cast<float*>(static_cast<char*>(m->slab) + ((nw * 2 + 255) & ~size_t(255)));
  auto takef = [&](size_t n) {
    float* p = fp;
    fp += n;
    return p;
  };
  m->special = takef(He);
  m->enc_in_b = takef(He);
  m->enc_to_lm_b = takef(H);
  m->lm_to_dit_b = takef(Hd);
  m->res_to_dit_b = takef(Hd);
  m->fusion_b = takef(H);
  m->stop_proj_b = takef(H);
  m->fsq_in_b = takef(sq_latent_dim);
  m->fsq_out_b = takef(H);
  const size_t DP = (size_t)feat_dim * patch_size;
  const int rows_max = std::max(128, lm_max_length(base_lm));
  bool ok = cudaMalloc(&m->fuse_in, 2 * (size_t)H * 4) == cudaSuccess &&
            cudaMalloc(&m->lm_tmp, (size_t)H * 4) == cudaSuccess &&
            cudaMalloc(&m->lat, (size_t)std::min(rows_max, 128) * sq_latent_dim * 4) == cudaSuccess &&
            cudaMalloc(&m->res_in, (size_t)H * 4) == cudaSuccess &&
            cudaMalloc(&m->res_hidden, (size_t)H * 4) == cudaSuccess &&
            cudaMalloc(&m->mu, 2 * (size_t)Hd * 4) == cudaSuccess && cudaMalloc(&m->stop_h, (size_t)H * 4) == cudaSuccess &&
            cudaMalloc(&m->stop_logits, (size_t)max_len * 2 * 4) == cudaSuccess &&
            cudaMalloc(&m->stop_flags, (size_t)max_len * 4) == cudaSuccess &&
            cudaMallocHost(&m->h_flags, (size_t)max_len * 4) == cudaSuccess &&
            cudaMalloc(&m->patch[0], DP * 4) == cudaSuccess && cudaMalloc(&m->patch[1], DP * 4) == cudaSuccess &&
            cudaMalloc(&m->latent, DP * max_len * 4) == cudaSuccess &&
            cudaMalloc(&m->noise, DP * max_len * 4) == cudaSuccess &&
            cudaEventCreateWithFlags(&m->ev[0], cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&m->ev[1], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return fail_free(VX_ERR_OOM, "voxcpm2: buffer allocation failed");
  }
  const int max_n = std::max({H, Hd, He, sq_latent_dim}), max_k = std::max({2 * H, He, sq_latent_dim});
  if (workspace_init(ctx, &m->ws, max_n, max_k) != VX_OK) return fail_free(VX_ERR_OOM, "voxcpm2: workspace failed");
  *out = m;
  return VX_OK;
}

void vx_voxcpm2_destroy(vx_voxcpm2* m) {
  if (!m) return;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  free_prefill(m);
  workspace_free(&m->ws);
  for (void* p : {(void*)m->slab, (void*)m->fuse_in, (void*)m->lm_tmp, (void*)m->lat, (void*)m->res_in,
                  (void*)m->res_hidden, (void*)m->mu, (void*)m->stop_h, (void*)m->stop_logits, (void*)m->stop_flags,
                  (void*)m->patch[0], (void*)m->patch[1], (void*)m->latent, (void*)m->noise, (void*)m->enc_seq,
                  (void*)m->enc_out})
    if (p) cudaFree(p);
  if (m->h_flags) cudaFreeHost(m->h_flags);
  for (cudaEvent_t e : m->ev)
    if (e) cudaEventDestroy(e);
  delete m;
}

int vx_voxcpm2_load(vx_voxcpm2* m, const vx_voxcpm2_weights* w) {
  if (!m || !w) return VX_ERR_ARG;
  const void* need[] = {w->special_token, w->enc_in_w,  w->enc_in_b,    w->enc_to_lm_w, w->enc_to_lm_b,
                        w->lm_to_dit_w,   w->lm_to_dit_b, w->res_to_dit_w, w->res_to_dit_b, w->fusion_w,
                        w->fusion_b,      w->stop_proj_w, w->stop_proj_b, w->stop_head_w, w->fsq_in_w,
                        w->fsq_in_b,      w->fsq_out_w,   w->fsq_out_b};
  for (const void* p : need)
    if (!p) return fail(m->ctx, VX_ERR_ARG, "voxcpm2_load: missing weight");
  vx_ctx* ctx = m->ctx;
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t H = m->H, He = m->He, Hd = m->Hd, D = m->D, Lq = m->Lq;
  struct Cp {
    void* dst;
    const void* src;
    size_t bytes;
  } cps[] = {{m->special, w->special_token, He * 4},      {m->enc_in_w, w->enc_in_w, He * D * 2},
             {m->enc_in_b, w->enc_in_b, He * 4},          {m->enc_to_lm_w, w->enc_to_lm_w, H * He * 2},
             {m->enc_to_lm_b, w->enc_to_lm_b, H * 4},     {m->lm_to_dit_w, w->lm_to_dit_w, Hd * H * 2},
             {m->lm_to_dit_b, w->lm_to_dit_b, Hd * 4},    {m->res_to_dit_w, w->res_to_dit_w, Hd * H * 2},
             {m->res_to_dit_b, w->res_to_dit_b, Hd * 4},  {m->fusion_w, w->fusion_w, 2 * H * H * 2},
             {m->fusion_b, w->fusion_b, H * 4},           {m->stop_proj_w, w->stop_proj_w, H * H * 2},
             {m->stop_proj_b, w->stop_proj_b, H * 4},     {m->stop_head_w, w->stop_head_w, 2 * H * 2},
             {m->fsq_in_w, w->fsq_in_w, Lq * H * 2},      {m->fsq_in_b, w->fsq_in_b, Lq * 4},
             {m->fsq_out_w, w->fsq_out_w, H * Lq * 2},    {m->fsq_out_b, w->fsq_out_b, H * 4}};
  for (const Cp& c : cps) VX_CUDA(ctx, cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaStreamSynchronize(st));
  return VX_OK;
}

int vx_locenc_forward(vx_voxcpm2* m, const float* feat, int N, float* out) {
  if (!m || !feat || !out || N <= 0) return VX_ERR_ARG;
  vx_ctx* ctx = m->ctx;
  cudaSetDevice(ctx->device);
  int rc = ensure_enc_rows(m, N);
  if (rc) return rc;
  count_launch();
  locenc_seq_kernel<<<dim3(N * (m->P + 1), (m->He + 255) / 256), 256, m->D * sizeof(float), ctx->stream>>>(
      feat, m->P, m->D, 0, m->enc_in_w, m->enc_in_b, m->special, m->He, m->enc_seq);
  VX_CUDA(ctx, cudaGetLastError());
  rc = vx_lm_forward(m->enc, m->enc_seq, N, m->P + 1, 0, 0, m->enc_out);
  if (rc) return rc;
  VX_CUDA(ctx, cudaMemcpy2DAsync(out, (size_t)m->He * 4, m->enc_out, (size_t)(m->P + 1) * m->He * 4,
                                 (size_t)m->He * 4, N, cudaMemcpyDefault, ctx->stream));
  return vx_ctx_synchronize(ctx);
}

int vx_voxcpm2_begin(vx_voxcpm2* m, const int32_t* text_token, const float* text_mask, const float* feat,
                     const float* feat_mask, int S, int min_len, int max_len, int inference_timesteps,
                     float cfg_value, const float* noise) {
  if (!m || !text_token || !text_mask || !feat || !feat_mask || !noise) return VX_ERR_ARG;
  vx_ctx* ctx = m->ctx;
  m->s_active = false;
  if (S <= 0 || max_len <= 0 || max_len > m->max_len || min_len < 0 || inference_timesteps < 1)
    return fail(ctx, VX_ERR_SHAPE, "voxcpm2: S=%d, max_len=%d (<= %d), steps=%d", S, max_len, m->max_len,
                inference_timesteps);
  if (S + max_len > lm_max_length(m->base) || S + max_len > lm_max_length(m->res))
    return fail(ctx, VX_ERR_KV_FULL, "voxcpm2: %d positions + %d steps exceed the KV cache", S, max_len);
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t DP = (size_t)m->D * m->P;
  // the last prompt patch conditions the first step (prefix_feat_cond, model.rs:153-154),
  // transposed to the CFM's channel-major [D, P]
  std::vector<float> last(DP);
  {
    std::vector<float> row(DP);
    VX_CUDA(ctx, cudaMemcpy(row.data(), feat + (size_t)(S - 1) * DP, DP * 4, cudaMemcpyDefault));
    for (int p = 0; p < m->P; ++p)
      for (int c = 0; c < m->D; ++c) last[(size_t)c * m->P + p] = row[(size_t)p * m->D + c];
  }
  VX_CUDA(ctx, cudaMemcpyAsync(m->noise, noise, DP * max_len * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(m->patch[0], last.data(), DP * 4, cudaMemcpyHostToDevice, st));
  const int rc = prefill(m, text_token, text_mask, feat_mask, feat, S);
  if (rc) {
    cudaStreamSynchronize(st);
    return rc;
  }
  m->s_i = 0;
  m->s_cur = 0;
  m->s_min_len = min_len;
  m->s_max_len = max_len;
  m->s_steps = inference_timesteps;
  m->s_cfg = cfg_value;
  m->s_finished = false;
  m->s_active = true;
  return VX_OK;
}

// Up to `budget` more AR steps of the loop of model.rs:318-347: dit_step(i); stop if
// i > min_len and the head fires; else lm_step.  Inside a call, the flag of step i is read
// after step i + 1 is queued (step i + 1's work is discarded if step i stopped); the last step
// of a call reads its own flag before deciding on its lm_step.  Returns the patches produced
// through *n_new; they start at patch index *first.
static int advance(vx_voxcpm2* m, int budget, int* first, int* n_new) {
  vx_ctx* ctx = m->ctx;
  cudaStream_t st = ctx->stream;
  *first = m->s_i;
  *n_new = 0;
  int rc = VX_OK;
  for (int j = 0; j < budget && !m->s_finished; ++j) {
    const int i = m->s_i;
    if (i >= m->s_max_len) {
      m->s_finished = true;
      break;
    }
    if (ctx->cancel.load(std::memory_order_relaxed)) {  // model.rs:323-328
      cudaStreamSynchronize(st);
      m->s_active = false;
      return fail(ctx, VX_ERR_CANCELLED, "generation cancelled");
    }
    rc = dit_step(m, i, m->s_cur, m->s_steps, m->s_cfg);
    if (rc) break;
    if (j > 0) {
      VX_CUDA(ctx, cudaEventSynchronize(m->ev[(i - 1) & 1]));
      if (i - 1 > m->s_min_len && m->h_flags[i - 1]) {
        m->s_finished = true;  // step i - 1 was the last; step i is discarded
        break;
      }
    }
    m->s_i = i + 1;
    *n_new += 1;
    if (i == m->s_max_len - 1) {
      m->s_finished = true;
      break;
    }
    if (j == budget - 1) {  // the call's last step: decide its lm_step on its own flag
      VX_CUDA(ctx, cudaEventSynchronize(m->ev[i & 1]));
      if (i > m->s_min_len && m->h_flags[i]) {
        m->s_finished = true;
        break;
      }
    }
    rc = lm_step(m, m->s_cur ^ 1);
    if (rc) break;
    m->s_cur ^= 1;
  }
  if (rc) {
    cudaStreamSynchronize(st);
    m->s_active = false;
    return rc;
  }
  // a step past the stopping one was queued and discarded: it is not part of the output
  if (m->s_finished && *first + *n_new > 0) {
    const int lastp = *first + *n_new - 1;
    VX_CUDA(ctx, cudaEventSynchronize(m->ev[lastp & 1]));
  }
  return VX_OK;
}

int vx_voxcpm2_advance(vx_voxcpm2* m, int max_patches, float* latent_out, int* n_new, int* finished) {
  if (!m || !latent_out || !n_new || !finished || max_patches <= 0) return VX_ERR_ARG;
  *n_new = 0;
  *finished = 1;
  if (!m->s_active) return fail(m->ctx, VX_ERR_ARG, "voxcpm2_advance: no generation begun");
  int first = 0, n = 0;
  const int rc = advance(m, max_patches, &first, &n);
  if (rc) return rc;
  const size_t frames = (size_t)n * m->P;
  if (n > 0)
    VX_CUDA(m->ctx, cudaMemcpy2DAsync(latent_out, frames * 4, m->latent + (size_t)first * m->P,
                                      (size_t)m->max_len * m->P * 4, frames * 4, m->D, cudaMemcpyDefault,
                                      m->ctx->stream));
  *n_new = n;
  *finished = m->s_finished ? 1 : 0;
  return vx_ctx_synchronize(m->ctx);
}

int vx_voxcpm2_inference(vx_voxcpm2* m, const int32_t* text_token, const float* text_mask, const float* feat,
                         const float* feat_mask, int S, int min_len, int max_len, int inference_timesteps,
                         float cfg_value, const float* noise, float* latent_out, int* n_patches,
                         float* stop_logits_out) {
  if (!m || !latent_out || !n_patches) return VX_ERR_ARG;
  *n_patches = 0;
  int rc = vx_voxcpm2_begin(m, text_token, text_mask, feat, feat_mask, S, min_len, max_len, inference_timesteps,
                            cfg_value, noise);
  if (rc) return rc;
  int first = 0, n = 0;
  rc = advance(m, max_len, &first, &n);
  if (rc) return rc;
  vx_ctx* ctx = m->ctx;
  *n_patches = n;
  const size_t frames = (size_t)n * m->P;
  VX_CUDA(ctx, cudaMemcpy2DAsync(latent_out, frames * 4, m->latent, (size_t)m->max_len * m->P * 4, frames * 4, m->D,
                                 cudaMemcpyDefault, ctx->stream));
  if (stop_logits_out)
    VX_CUDA(ctx, cudaMemcpyAsync(stop_logits_out, m->stop_logits, (size_t)n * 2 * 4, cudaMemcpyDefault, ctx->stream));
  return vx_ctx_synchronize(ctx);
}

int vx_voxcpm2_generate(vx_voxcpm2* m, vx_vae* vae, const int32_t* text_token, const float* text_mask,
                        const float* feat, const float* feat_mask, int S, int min_len, int max_len,
                        int inference_timesteps, float cfg_value, const float* noise, float* wav_out,
                        int* n_samples) {
  if (!m || !vae || !wav_out || !n_samples) return VX_ERR_ARG;
  vx_ctx* ctx = m->ctx;
  *n_samples = 0;
  if (vae_ctx(vae) != ctx) return fail(ctx, VX_ERR_ARG, "voxcpm2_generate: the VAE must share the context");
  if (vae_latent(vae) != m->D) return fail(ctx, VX_ERR_CONFIG, "voxcpm2_generate: VAE latent != feat_dim");
  int n = 0;
  std::vector<float> lat((size_t)m->D * m->P * std::max(1, max_len));
  int rc = vx_voxcpm2_inference(m, text_token, text_mask, feat, feat_mask, S, min_len, max_len, inference_timesteps,
                                cfg_value, noise, lat.data(), &n, nullptr);
  if (rc) return rc;
  // decode_latent_to_samples (wrapper.rs:616-629): AudioVae::decode of [1, D, n*P]
  const size_t frames = (size_t)n * m->P, samples = frames * vae_hop(vae);
  float *d_lat = nullptr, *d_wav = nullptr;
  if (cudaMalloc(&d_lat, (size_t)m->D * frames * 4) != cudaSuccess || cudaMalloc(&d_wav, samples * 4) != cudaSuccess) {
    cudaGetLastError();
    if (d_lat) cudaFree(d_lat);
    return fail(ctx, VX_ERR_OOM, "voxcpm2_generate: buffer allocation failed");
  }
  rc = VX_OK;
  if (cudaMemcpyAsync(d_lat, lat.data(), (size_t)m->D * frames * 4, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
    rc = fail(ctx, VX_ERR_CUDA, "voxcpm2_generate: latent upload failed");
  if (!rc) rc = vx_vae_decode(vae, d_lat, 1, (int)frames, d_wav);
  if (!rc && cudaMemcpy(wav_out, d_wav, samples * 4, cudaMemcpyDefault) != cudaSuccess)
    rc = fail(ctx, VX_ERR_CUDA, "voxcpm2_generate: download failed");
  cudaFree(d_lat);
  cudaFree(d_wav);
  if (!rc) *n_samples = (int)samples;
  return rc;
}

}  // extern "C"

namespace vx {
void voxcpm2_parts(vx_voxcpm2* m, vx_lm** base, vx_lm** res, vx_lm** enc, vx_dit** dit, int dims[6]) {
  *base = m->base;
  *res = m->res;
  *enc = m->enc;
  *dit = m->dit;
  dims[0] = m->H;
  dims[1] = m->He;
  dims[2] = m->Hd;
  dims[3] = m->D;
  dims[4] = m->P;
  dims[5] = m->Lq;
}
}  // namespace vx
