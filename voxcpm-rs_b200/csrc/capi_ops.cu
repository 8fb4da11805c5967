// C ABI: context management and op-level entry points.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "runtime.cuh"

namespace vx {

thread_local unsigned long long g_launches = 0;

void* ctx_scratch(vx_ctx* ctx, size_t bytes) {
  if (ctx->scratch.bytes >= bytes) return ctx->scratch.ptr;
  // scratch may be in use by earlier launches on any stream; wait before replacing it
  cudaDeviceSynchronize();
  if (ctx->scratch.ptr) cudaFree(ctx->scratch.ptr);
  ctx->scratch.ptr = nullptr;
  ctx->scratch.bytes = 0;
  size_t want = bytes < (16u << 20) ? (16u << 20) : bytes;
  if (cudaMalloc(&ctx->scratch.ptr, want) != cudaSuccess) return nullptr;
  ctx->scratch.bytes = want;
  return ctx->scratch.ptr;
}

int workspace_init(vx_ctx* ctx, LinearWorkspace* ws, int max_n, int max_k) {
  ws->bytes = tc_gemm_scratch_bytes(128, max_n, max_k, ctx->gemv_ctas);
  if (cudaMalloc(&ws->scratch, ws->bytes) != cudaSuccess || cudaMalloc(&ws->counters, 1024 * 4) != cudaSuccess ||
      cudaMemset(ws->counters, 0, 1024 * 4) != cudaSuccess) {
    cudaGetLastError();
    workspace_free(ws);
    return fail(ctx, VX_ERR_OOM, "linear workspace allocation failed");
  }
  return VX_OK;
}

void workspace_free(LinearWorkspace* ws) {
  if (ws->scratch) cudaFree(ws->scratch);
  if (ws->counters) cudaFree(ws->counters);
  ws->scratch = nullptr;
  ws->counters = nullptr;
  ws->bytes = 0;
}

int linear(vx_ctx* ctx, const LinearWorkspace* ws, const float* X, int ldx, int M, int N, int K, const uint16_t* W,
           const float* bias, const float* R, float res_scale, float* Y, int ldy, cudaStream_t st) {
  if (M == 1 && N % 8 == 0 && gemv_pick_kc(K) != 0 && ((uintptr_t)X & 15) == 0) {
    GemvArgs a = {};
    a.W = W;
    a.N = N;
    a.K = K;
    a.x = X;
    a.y = Y;
    a.bias = bias;
    a.residual = R;
    a.res_scale = R ? res_scale : 1.f;
    a.groups_per_cta = pick_groups(N / 8, ctx->gemv_ctas);
    VX_CUDA(ctx, launch_gemv(a, EPI_STORE, st, false, ctx->dev_err));
    return VX_OK;
  }
  if (ctx->tc_gemm && ws && ws->scratch && tc_gemm_supported(std::min(M, 128), N, K) &&
      tc_gemm_scratch_bytes(std::min(M, 128), N, K, ctx->gemv_ctas) <= ws->bytes) {
    for (int m0 = 0; m0 < M; m0 += 128) {
      const int mm = std::min(128, M - m0);
      VX_CUDA(ctx, launch_tc_gemm(X + (size_t)m0 * ldx, ldx, mm, N, K, W, bias, R ? R + (size_t)m0 * ldy : nullptr,
                                  res_scale, Y + (size_t)m0 * ldy, ldy, ws->scratch, ws->counters, ctx->dev_err, st,
                                  ctx->gemv_ctas));
    }
    return VX_OK;
  }
  if (K % 64 != 0) return fail(ctx, VX_ERR_SHAPE, "linear: K must be a multiple of 64 (got %d)", K);
  GemmArgs g = {X, ldx, W, bias, R, res_scale, Y, ldy, M, N, K};
  VX_CUDA(ctx, launch_gemm_smallm(g, st));
  return VX_OK;
}

bool presplit_ok(vx_ctx* ctx, const LinearWorkspace* ws, int M, int N, int K) {
  return ctx->tc_gemm && ctx->presplit && ws && ws->scratch && M > 1 && M <= 128 && tc_gemm_supported(M, N, K) &&
         tc_gemm_scratch_bytes(M, N, K, ctx->gemv_ctas) <= ws->bytes;
}

int linear_presplit(vx_ctx* ctx, const LinearWorkspace* ws, int M, int N, int K, const uint16_t* W, const float* bias,
                    const float* R, float res_scale, float* Y, int ldy, cudaStream_t st) {
  VX_CUDA(ctx, launch_tc_gemm_presplit(M, N, K, W, bias, R, res_scale, Y, ldy, ws->scratch, ws->counters,
                                       ctx->dev_err, st, ctx->gemv_ctas));
  return VX_OK;
}

int fill_rope_params(const vx_minicpm4_config& c, RopeParams* rp, std::string* err) {
  // MiniCpmLongRope::new (src/minicpm4/rope.rs:16-32), all in f64
  const int d = c.kv_channels > 0 ? c.kv_channels : c.hidden_size / c.num_attention_heads;
  const int half = d / 2;
  if (half > 128) {
    *err = "head_dim > 256 unsupported";
    return VX_ERR_CONFIG;
  }
  if (c.rope_factor_len != half || !c.rope_short_factor || !c.rope_long_factor) {
    *err = "rope_scaling factor length must equal head_dim/2";
    return VX_ERR_CONFIG;
  }
  const double base = (double)c.rope_theta;
  const int max_pos = c.max_position_embeddings, orig = c.original_max_position_embeddings;
  const double scale = (double)max_pos / (double)orig;
  double sf = std::sqrt(1.0 + std::log(scale) / std::log((double)orig));
  if (!(sf >= 1.0)) sf = 1.0;  // f64::max(1.0) ignores NaN
  const float* ext = max_pos > orig ? c.rope_long_factor : c.rope_short_factor;
  memset(rp, 0, sizeof(*rp));
  for (int i = 0; i < half; ++i) {
    rp->inv_freq[i] = 1.0 / std::pow(base, 2.0 * (double)i / (double)d);
    rp->ext[i] = (double)ext[i];
  }
  rp->scaling_factor = sf;
  rp->half = half;
  return VX_OK;
}

}  // namespace vx

using namespace vx;

extern "C" {

int vx_version(void) { return 100; }

unsigned long long vx_launch_count(void) { return g_launches; }

int vx_ctx_create(int device, vx_ctx** out) {
  if (!out) return VX_ERR_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) return VX_ERR_NO_DEVICE;
  if (device < 0 || device >= n) return VX_ERR_ARG;
  vx_ctx* ctx = new vx_ctx();
  ctx->device = device;
  // tuning knobs read from the environment: GEMV grid target, programmatic dependent launch,
  // the tcgen05 few-row GEMM and the persistent decode step's ring / grid / prefetch settings
  if (const char* s = getenv("VX_GEMV_CTAS")) ctx->gemv_ctas = std::max(1, atoi(s));
  if (const char* s = getenv("VX_PDL")) ctx->pdl = atoi(s) != 0;
  if (const char* s = getenv("VX_L2_PREFETCH")) ctx->l2_prefetch = atoi(s) != 0;
  if (const char* s = getenv("VX_TC_GEMM")) ctx->tc_gemm = atoi(s) != 0;
  if (const char* s = getenv("VX_PERSIST")) ctx->persist = atoi(s) != 0;
  if (const char* s = getenv("VX_PERSIST_NST")) ctx->persist_nst = std::max(0, atoi(s));
  if (const char* s = getenv("VX_PERSIST_GRID")) ctx->persist_grid = std::max(0, atoi(s));
  if (const char* s = getenv("VX_PERSIST_INFLIGHT")) ctx->persist_inflight = std::max(0, atoi(s));
  if (const char* s = getenv("VX_PERSIST_MLP_PF")) ctx->persist_mlp_pf = std::max(0, std::min(64, atoi(s)));
  if (const char* s = getenv("VX_PERSIST_MERGE_TILES")) ctx->persist_merge_tiles = std::max(0, atoi(s));
  if (const char* s = getenv("VX_PERSIST_PF")) ctx->persist_pf = std::max(0, std::min(256, atoi(s)));
  if (const char* s = getenv("VX_PERSIST_EF")) ctx->persist_ef = atoi(s) != 0;
  if (const char* s = getenv("VX_PRESPLIT")) ctx->presplit = atoi(s) != 0;
  if (const char* s = getenv("VX_ATT_ROPE_FUSED")) ctx->att_rope_fused = atoi(s) != 0;
  if (cudaSetDevice(device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->counters, 4096 * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(ctx->counters, 0, 4096 * sizeof(unsigned)) != cudaSuccess ||
      cudaMalloc(&ctx->dev_err, 64) != cudaSuccess || cudaMemset(ctx->dev_err, 0, 64) != cudaSuccess ||
      gemv_configure() != cudaSuccess || tc_gemm_configure() != cudaSuccess ||
      vae_tc_configure() != cudaSuccess) {
    cudaGetLastError();
    delete ctx;
    return VX_ERR_CUDA;
  }
  if (!ctx_scratch(ctx, 16u << 20)) {
    delete ctx;
    return VX_ERR_OOM;
  }
  *out = ctx;
  return VX_OK;
}

void vx_ctx_destroy(vx_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch.ptr) cudaFree(ctx->scratch.ptr);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
}

const char* vx_last_error(const vx_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

void* vx_ctx_stream(vx_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int vx_ctx_synchronize(vx_ctx* ctx) {
  if (!ctx) return VX_ERR_ARG;
  cudaSetDevice(ctx->device);
  VX_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  int derr = 0;
  VX_CUDA(ctx, cudaMemcpy(&derr, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (derr) {
    cudaMemset(ctx->dev_err, 0, sizeof(int));
    if (derr == VX_DEVICE_ERR_BOUNDS)  // a kernel's own bounds check refused an index (nothing written)
      return fail(ctx, VX_ERR_ARG, "device-side bounds check failed (code %d)", derr);
    return fail(ctx, VX_ERR_TIMEOUT, "device-side wait gave up (code %d)", derr);
  }
  return VX_OK;
}

void vx_cancel(vx_ctx* ctx) {
  if (ctx) ctx->cancel.store(1, std::memory_order_relaxed);
}

void vx_cancel_reset(vx_ctx* ctx) {
  if (ctx) ctx->cancel.store(0, std::memory_order_relaxed);
}

int vx_memcpy(vx_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes)) return VX_ERR_ARG;
  cudaSetDevice(ctx->device);
  VX_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, ctx->stream));
  VX_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return VX_OK;
}

int vx_rmsnorm_residual(vx_ctx* ctx, const float* x, const float* r, const float* w, float resid_scale,
                        float eps, int rows, int hidden, float* h_out, float* y_out, vx_stream stream) {
  if (!ctx || !x || !w || !y_out) return VX_ERR_ARG;
  if (rows <= 0 || hidden <= 0 || hidden % 4 != 0 || hidden > 8192)
    return fail(ctx, VX_ERR_SHAPE, "rmsnorm: hidden must be a positive multiple of 4 <= 8192 (got %d)", hidden);
  cudaSetDevice(ctx->device);
  VX_CUDA(ctx, launch_rmsnorm_residual(x, r, w, resid_scale, eps, rows, hidden, h_out, y_out,
                                       pick_stream(ctx, stream)));
  return VX_OK;
}

int vx_longrope_table(const vx_minicpm4_config* cfg, int n_pos, float* cos_out, float* sin_out) {
  if (!cfg || !cos_out || !sin_out || n_pos < 0) return VX_ERR_ARG;
  RopeParams rp;
  std::string err;
  int st = fill_rope_params(*cfg, &rp, &err);
  if (st != VX_OK) return st;
  const int half = rp.half, d = 2 * half;
  for (int t = 0; t < n_pos; ++t) {
    for (int i = 0; i < half; ++i) {
      // rope.rs:38-46: freq = t * inv_freq / ext in f64; cos/sin scaled, then cast to f32
      const double f = (double)t * rp.inv_freq[i] / rp.ext[i];
      const float c = (float)(std::cos(f) * rp.scaling_factor);
      const float s = (float)(std::sin(f) * rp.scaling_factor);
      cos_out[(size_t)t * d + i] = c;
      cos_out[(size_t)t * d + i + half] = c;
      sin_out[(size_t)t * d + i] = s;
      sin_out[(size_t)t * d + i + half] = s;
    }
  }
  return VX_OK;
}

int vx_rope_apply(vx_ctx* ctx, float* q, float* k, const float* cos, const float* sin, int B, int nh, int nkv,
                  int S, int head_dim, vx_stream stream) {
  if (!ctx || !q || !k || !cos || !sin) return VX_ERR_ARG;
  if (head_dim % 2 != 0 || B <= 0 || S <= 0) return fail(ctx, VX_ERR_SHAPE, "rope_apply: bad shape");
  cudaSetDevice(ctx->device);
  cudaStream_t st = pick_stream(ctx, stream);
  VX_CUDA(ctx, launch_rope_apply(q, B, nh, S, head_dim, cos, sin, st));
  VX_CUDA(ctx, launch_rope_apply(k, B, nkv, S, head_dim, cos, sin, st));
  return VX_OK;
}

int vx_linear_bf16(vx_ctx* ctx, const uint16_t* w, const float* bias, const float* x, int M, int N, int K,
                   float* y, vx_stream stream) {
  if (!ctx || !w || !x || !y) return VX_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0) return fail(ctx, VX_ERR_SHAPE, "linear: empty shape");
  cudaSetDevice(ctx->device);
  cudaStream_t st = pick_stream(ctx, stream);
  LinearWorkspace ws;
  if (M > 1 && ctx->tc_gemm && tc_gemm_supported(std::min(M, 128), N, K)) {
    ws.bytes = tc_gemm_scratch_bytes(std::min(M, 128), N, K, ctx->gemv_ctas);
    ws.scratch = ctx_scratch(ctx, ws.bytes);
    if (!ws.scratch) return fail(ctx, VX_ERR_OOM, "linear: scratch allocation failed");
    ws.counters = ctx->counters;
  }
  return linear(ctx, &ws, x, K, M, N, K, w, bias, nullptr, 1.f, y, N, st);
}

int vx_attention_decode(vx_ctx* ctx, const float* q, const float* kcache, const float* vcache, int B, int nh,
                        int nkv, int head_dim, int s_max, int cur_len, float* out, vx_stream stream) {
  if (!ctx || !q || !kcache || !vcache || !out) return VX_ERR_ARG;
  if (B <= 0 || nkv <= 0 || nh % nkv != 0 || nh / nkv != 8 || (head_dim != 128 && head_dim != 64))
    return fail(ctx, VX_ERR_SHAPE, "attention_decode: needs nh/nkv == 8 and head_dim in {64,128}");
  if (cur_len <= 0 || cur_len > s_max) return fail(ctx, VX_ERR_SHAPE, "attention_decode: cur_len out of range");
  if (B * nkv > 4096) return fail(ctx, VX_ERR_SHAPE, "attention_decode: B*nkv > 4096");
  cudaSetDevice(ctx->device);
  const int nsplit = 32;  // upper bound; the kernel activates ceil(cur_len/32) of them
  const size_t pbytes = (size_t)B * nkv * nsplit * 8 * (head_dim + 2) * sizeof(float);
  float* partials = static_cast<float*>(ctx_scratch(ctx, pbytes));
  if (!partials) return fail(ctx, VX_ERR_OOM, "attention_decode: scratch allocation failed");
  AttnDecodeArgs a = {q, kcache, vcache, B, nh, nkv, head_dim, s_max, nullptr, cur_len,
                      (float)(1.0 / std::sqrt((double)head_dim)), nsplit, partials, ctx->counters, out};
  VX_CUDA(ctx, launch_attn_decode(a, pick_stream(ctx, stream), false));
  return VX_OK;
}

int vx_fsq(vx_ctx* ctx, const uint16_t* w_in, const float* b_in, const uint16_t* w_out, const float* b_out,
           int in_dim, int latent_dim, int out_dim, float scale, const float* hidden, int rows, float* out,
           vx_stream stream) {
  if (!ctx || !w_in || !w_out || !hidden || !out) return VX_ERR_ARG;
  if (rows <= 0 || in_dim <= 0 || latent_dim <= 0 || out_dim <= 0 || !(scale > 0.f))
    return fail(ctx, VX_ERR_SHAPE, "fsq: empty shape or non-positive scale");
  if (in_dim % 64 != 0 || latent_dim % 64 != 0 || out_dim % 8 != 0)
    return fail(ctx, VX_ERR_SHAPE, "fsq: in_dim and latent_dim must be multiples of 64, out_dim of 8");
  cudaSetDevice(ctx->device);
  cudaStream_t st = pick_stream(ctx, stream);
  // scratch: the latent activations, then the few-row GEMM workspace
  const size_t lat_bytes = (((size_t)rows * latent_dim * 4) + 255) & ~size_t(255);
  size_t gb = 0;
  const int mm = std::min(rows, 128);
  if (rows > 1 && ctx->tc_gemm) {
    if (tc_gemm_supported(mm, latent_dim, in_dim)) gb = std::max(gb, tc_gemm_scratch_bytes(mm, latent_dim, in_dim, ctx->gemv_ctas));
    if (tc_gemm_supported(mm, out_dim, latent_dim)) gb = std::max(gb, tc_gemm_scratch_bytes(mm, out_dim, latent_dim, ctx->gemv_ctas));
  }
  char* base = static_cast<char*>(ctx_scratch(ctx, lat_bytes + gb));
  if (!base) return fail(ctx, VX_ERR_OOM, "fsq: scratch allocation failed");
  LinearWorkspace ws;
  if (gb) {
    ws.scratch = base + lat_bytes;
    ws.bytes = gb;
    ws.counters = ctx->counters;
  }
  float* lat = reinterpret_cast<float*>(base);
  int rc = linear(ctx, &ws, hidden, in_dim, rows, latent_dim, in_dim, w_in, b_in, nullptr, 1.f, lat, latent_dim, st);
  if (rc) return rc;
  VX_CUDA(ctx, launch_fsq_quant(lat, (size_t)rows * latent_dim, scale, st));
  return linear(ctx, &ws, lat, latent_dim, rows, out_dim, latent_dim, w_out, b_out, nullptr, 1.f, out, out_dim, st);
}

int vx_mlp_swiglu(vx_ctx* ctx, const uint16_t* w_gate_up, const uint16_t* w_down, const float* x, int rows,
                  int hidden, int inter, float* out, vx_stream stream) {
  if (!ctx || !w_gate_up || !w_down || !x || !out) return VX_ERR_ARG;
  if (rows <= 0 || hidden % 64 != 0 || inter % 64 != 0)
    return fail(ctx, VX_ERR_SHAPE, "mlp: hidden and inter must be multiples of 64");
  cudaSetDevice(ctx->device);
  cudaStream_t st = pick_stream(ctx, stream);
  float* act = static_cast<float*>(ctx_scratch(ctx, (size_t)rows * inter * 3 * sizeof(float)));
  if (!act) return fail(ctx, VX_ERR_OOM, "mlp: scratch allocation failed");
  if (rows == 1 && gemv_pick_kc(hidden) && gemv_pick_kc(inter)) {
    GemvArgs a = {};
    a.W = w_gate_up;
    a.N = 2 * inter;
    a.K = hidden;
    a.x = x;
    a.map_mode = MAP_GATE_UP;
    a.map_param = inter / 8;
    a.groups_per_cta = 2 * pick_groups(inter / 8);
    a.inter = inter;
    a.act = act;
    VX_CUDA(ctx, launch_gemv(a, EPI_SILU_MUL, st, false, ctx->dev_err));
    GemvArgs b = {};
    b.W = w_down;
    b.N = hidden;
    b.K = inter;
    b.x = act;
    b.y = out;
    b.res_scale = 1.f;
    b.groups_per_cta = 1;
    VX_CUDA(ctx, launch_gemv(b, EPI_STORE, st, false, ctx->dev_err));
    return VX_OK;
  }
  float* gu = act + (size_t)rows * inter;
  GemmArgs g1 = {x, hidden, w_gate_up, nullptr, nullptr, 1.f, gu, 2 * inter, rows, 2 * inter, hidden};
  VX_CUDA(ctx, launch_gemm_smallm(g1, st));
  VX_CUDA(ctx, launch_silu_mul(gu, rows, inter, act, st));
  GemmArgs g2 = {act, inter, w_down, nullptr, nullptr, 1.f, out, hidden, rows, hidden, inter};
  VX_CUDA(ctx, launch_gemm_smallm(g2, st));
  return VX_OK;
}

int vx_cfg_euler(vx_ctx* ctx, const float* out2b, float* x, int B, int C, int T, float cfg, double dt,
                 int zero_star, vx_stream stream) {
  if (!ctx || !out2b || !x) return VX_ERR_ARG;
  if (B <= 0 || C <= 0 || T <= 0) return fail(ctx, VX_ERR_SHAPE, "cfg_euler: empty shape");
  cudaSetDevice(ctx->device);
  VX_CUDA(ctx, launch_cfg_euler(out2b, x, B, C * T, (double)cfg, dt, zero_star, pick_stream(ctx, stream)));
  return VX_OK;
}

}  // extern "C"
