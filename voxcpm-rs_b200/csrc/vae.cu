// AudioVAE v2 causal decoder (reference src/audiovae/layers.rs, decoder.rs, vae.rs).
//
// Activations stay channel-major [B, C, T] like the reference's tensors.  Kernels:
//   * dw_conv_kernel: CausalConv1d depthwise k=7 (layers.rs:13-53) with optional Snake1d
//     (layers.rs:118-123) on its input and on its output, so a residual unit's
//     snake -> dwconv(dilation) -> snake is one pass; the causal left halo (2*pad zeros) is
//     staged in shared memory with the tile.
//   * conv_gemm_kernel: the k=1 pointwise convs (bias + residual add fused) and the causal
//     transposed convs as a polyphase GEMM: for stride s and kernel 2s, output sample j*s+r
//     is W[:, :, r]^T x[:, j] + W[:, :, r+s]^T x[:, j-1] (the right trim of
//     CausalTransposeConv1d drops exactly the j = T tail), so phase r is a GEMM with
//     K = 2*C_in over [x[:, j]; x[:, j-1]].  Weights are re-laid per phase at upload.  The
//     operand loader applies SampleRateConditionLayer (layers.rs:213-220) and the block's
//     Snake1d to the input on the fly, so neither is a separate pass.
//   * last_conv_kernel: snake_out -> CausalConv1d(C -> 1, k=7) -> tanh (decoder.rs:164-166).
// conv_gemm_kernel is the CUDA-core (f32 FMA) form of the same GEMMs; the decoder runs the
// pointwise and transposed convs on tcgen05 (vae_tc.cu) and keeps conv_gemm_kernel for a
// latent width that is not a multiple of 64 and for A/B timing (env VX_VAE_TC=0).
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "runtime.cuh"

using namespace vx;

namespace {

__device__ __forceinline__ float snake(float x, float alpha) {
  // x + (alpha + 1e-9)^-1 * sin(alpha * x)^2   (layers.rs:119-122)
  const float inv = 1.0f / (alpha + 1e-9f);
  const float s = sinf(alpha * x);
  return x + inv * (s * s);
}

constexpr int DW_TT = 1024;  // outputs per CTA

// y[b,c,t] = post(bias[c] + sum_j w[c,j] * pre(x[b,c,t + j*dil - 6*dil]))   (pre/post: optional snake)
__global__ void __launch_bounds__(256) dw_conv_kernel(const float* __restrict__ x, int C, int T,
                                                      const uint16_t* __restrict__ w, const float* __restrict__ bias,
                                                      int dil, const float* __restrict__ a_pre,
                                                      const float* __restrict__ a_post, float* __restrict__ y,
                                                      const float* __restrict__ hist) {
  __shared__ float xs[DW_TT + 6 * 9];
  const int c = blockIdx.y, b = blockIdx.z;
  const int t0 = blockIdx.x * DW_TT;
  const int halo = 6 * dil;
  const float* xr = x + ((size_t)b * C + c) * T;
  const float* hr = hist ? hist + ((size_t)b * C + c) * halo : nullptr;  // the last `halo` inputs before x
  const float ap = a_pre ? a_pre[c] : 0.f;
  for (int i = threadIdx.x; i < DW_TT + halo; i += 256) {
    const int t = t0 - halo + i;
    float v = 0.f;  // causal left padding: zeros after the pre-snake (layers.rs:46-48)
    if (t >= 0 && t < T) {
      v = xr[t];
      if (a_pre) v = snake(v, ap);
    } else if (t < 0 && hr) {  // streaming: the previous chunk's inputs
      v = hr[halo + t];
      if (a_pre) v = snake(v, ap);
    }
    xs[i] = v;
  }
  __syncthreads();
  float wk[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) wk[j] = __uint_as_float(((uint32_t)w[c * 7 + j]) << 16);
  const float bc = bias[c];
  const float aq = a_post ? a_post[c] : 0.f;
  float* yr = y + ((size_t)b * C + c) * T;
  for (int i = threadIdx.x; i < DW_TT; i += 256) {
    const int t = t0 + i;
    if (t >= T) break;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 7; ++j) acc = fmaf(wk[j], xs[i + j * dil], acc);
    float v = acc + bc;
    if (a_post) v = snake(v, aq);
    yr[t] = v;
  }
}

struct ConvGemmArgs {
  const uint16_t* A;     // [phases][M][K] bf16
  const float* bias;     // [M]
  const float* X;        // [B, C_in, T_in]
  const float* R;        // residual [B, M, T_out] or null (may alias Y)
  float* Y;              // [B, M, T_out]
  int B, M, K, C_in, T_in, stride;  // stride 1: pointwise (K = C_in); s > 1: transposed (K = 2*C_in)
  const float* in_alpha;  // optional snake on the input (per input channel)
  const float* in_scale;  // optional SR-cond scale / bias (per input channel)
  const float* in_bias;
};

constexpr int CG_BM = 64, CG_BN = 128, CG_BK = 16;

__device__ __forceinline__ float conv_input(const ConvGemmArgs& a, int b, int kk, int j) {
  int ci = kk, jj = j;
  if (a.stride > 1 && kk >= a.C_in) {  // second tap: x[:, j-1]
    ci = kk - a.C_in;
    jj = j - 1;
  }
  if (jj < 0 || jj >= a.T_in) return 0.f;
  float v = a.X[((size_t)b * a.C_in + ci) * a.T_in + jj];
  if (a.in_scale) v = v * a.in_scale[ci] + a.in_bias[ci];
  if (a.in_alpha) v = snake(v, a.in_alpha[ci]);
  return v;
}

__global__ void __launch_bounds__(256) conv_gemm_kernel(const ConvGemmArgs a) {
  __shared__ __align__(16) float As[CG_BK][CG_BM + 4];
  __shared__ __align__(16) float Bs[CG_BK][CG_BN + 4];
  const int tid = threadIdx.x;
  const int j0 = blockIdx.x * CG_BN, m0 = blockIdx.y * CG_BM;
  const int phases = a.stride;
  const int b = blockIdx.z / phases, r = blockIdx.z % phases;
  const uint16_t* A = a.A + (size_t)r * a.M * a.K;
  const int ty = tid >> 4, tx = tid & 15;  // rows ty*4..+4, cols tx*8..+8
  float acc[4][8] = {};
  const bool plain = (a.stride == 1 && !a.in_alpha && !a.in_scale && (a.T_in % 4 == 0));
  for (int k0 = 0; k0 < a.K; k0 += CG_BK) {
    {  // A tile 64 x 16: thread loads 4 consecutive k of one row
      const int row = tid >> 2, kc = (tid & 3) * 4;
      const uint2 wv = *reinterpret_cast<const uint2*>(A + (size_t)(m0 + row) * a.K + k0 + kc);
      As[kc + 0][row] = bf16lo(wv.x);
      As[kc + 1][row] = bf16hi(wv.x);
      As[kc + 2][row] = bf16lo(wv.y);
      As[kc + 3][row] = bf16hi(wv.y);
    }
    {  // B tile 16 x 128: thread loads 8 consecutive j of one k row
      const int kr = tid >> 4, col = (tid & 15) * 8;
      const int kk = k0 + kr, j = j0 + col;
      if (plain && j + 8 <= a.T_in) {
        const float4* src = reinterpret_cast<const float4*>(a.X + ((size_t)b * a.C_in + kk) * a.T_in + j);
        const float4 v0 = src[0], v1 = src[1];
        *reinterpret_cast<float4*>(&Bs[kr][col]) = v0;
        *reinterpret_cast<float4*>(&Bs[kr][col + 4]) = v1;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) Bs[kr][col + e] = (j + e < a.T_in) ? conv_input(a, b, kk, j + e) : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < CG_BK; ++k) {
      const float4 av = *reinterpret_cast<const float4*>(&As[k][ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[k][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[k][tx * 8 + 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float br[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[i][e] = fmaf(ar[i], br[e], acc[i][e]);
    }
    __syncthreads();
  }
  const int T_out = a.T_in * a.stride;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    const float bm = a.bias[m];
    float* yr = a.Y + ((size_t)b * a.M + m) * T_out;
    const float* rr = a.R ? a.R + ((size_t)b * a.M + m) * T_out : nullptr;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = j0 + tx * 8 + e;
      if (j >= a.T_in) continue;
      const int t = j * a.stride + r;
      float v = acc[i][e] + bm;
      if (rr) v = rr[t] + v;  // CausalResidualUnit: x + conv2(...) (layers.rs:150-156)
      yr[t] = v;
    }
  }
}

constexpr int LC_TT = 1024;

// wav[b, t] = tanh(bias + sum_c sum_j w[c, j] * snake(h[b, c, t + j - 6], alpha[c]))
__global__ void __launch_bounds__(256) last_conv_kernel(const float* __restrict__ h, int C, int T,
                                                        const float* __restrict__ alpha, const uint16_t* __restrict__ w,
                                                        const float* __restrict__ bias, float* __restrict__ wav,
                                                        const float* __restrict__ hist) {
  __shared__ float xs[LC_TT + 6];
  const int b = blockIdx.y, t0 = blockIdx.x * LC_TT;
  float acc[LC_TT / 256] = {};
  for (int c = 0; c < C; ++c) {
    const float* hr = h + ((size_t)b * C + c) * T;
    const float al = alpha[c];
    __syncthreads();
    const float* hh = hist ? hist + ((size_t)b * C + c) * 6 : nullptr;
    for (int i = threadIdx.x; i < LC_TT + 6; i += 256) {
      const int t = t0 - 6 + i;
      xs[i] = (t >= 0 && t < T) ? snake(hr[t], al) : (t < 0 && hh) ? snake(hh[6 + t], al) : 0.f;
    }
    __syncthreads();
    float wk[7];
#pragma unroll
    for (int j = 0; j < 7; ++j) wk[j] = __uint_as_float(((uint32_t)w[c * 7 + j]) << 16);
#pragma unroll
    for (int q = 0; q < LC_TT / 256; ++q) {
      const int i = threadIdx.x + q * 256;
#pragma unroll
      for (int j = 0; j < 7; ++j) acc[q] = fmaf(wk[j], xs[i + j], acc[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < LC_TT / 256; ++q) {
    const int t = t0 + threadIdx.x + q * 256;
    if (t < T) wav[(size_t)b * T + t] = tanhf(acc[q] + bias[0]);
  }
}

// Streaming state: hist[b, c, 0..H) <- the last H samples of [hist | x[b, c, 0..T)] (one
// block per row; the old row is read before any of it is overwritten).
__global__ void __launch_bounds__(64) hist_update_kernel(float* __restrict__ hist, const float* __restrict__ x,
                                                         int T, int H) {
  __shared__ float old[64];
  const size_t row = blockIdx.x;
  const int k = threadIdx.x;
  if (k < H) old[k] = hist[row * H + k];
  __syncthreads();
  if (k < H) {
    const int src = T - H + k;
    hist[row * H + k] = src >= 0 ? x[row * T + src] : old[k + T];
  }
}

struct VaeUnit {
  float *alpha1 = nullptr, *alpha2 = nullptr, *b1 = nullptr, *b2 = nullptr;
  uint16_t *w1 = nullptr, *w2 = nullptr;  // dw [C, 7], pw [C, C]
};

struct VaeBlock {
  int cin = 0, cout = 0, stride = 0;
  float* alpha = nullptr;
  uint16_t* up_w = nullptr;   // [stride][cout][2*cin] per-phase GEMM layout (CUDA-core path)
  uint16_t* up_wt = nullptr;  // [vae_tc_rows(cout, stride)][2*cin] phase-folded layout (tcgen05 path)
  float* up_b = nullptr;
  VaeUnit res[3];
  float* sr_scale = nullptr;  // [cin] for the configured output sample rate (or null)
  float* sr_bias = nullptr;
};

}  // namespace

struct vx_vae {
  vx_ctx* ctx = nullptr;
  int latent = 0, dim = 0, depthwise = 1, nblocks = 0, sr_idx = -1, out_sr = 0, n_buckets = 0;
  std::vector<int> rates;
  float *first_dw_b = nullptr, *first_pw_b = nullptr, *alpha_out = nullptr, *last_b = nullptr;
  uint16_t *first_dw_w = nullptr, *first_pw_w = nullptr, *last_w = nullptr;
  std::vector<VaeBlock> blocks;
  std::vector<void*> allocs;
  size_t buf_elems = 0;
  float *buf0 = nullptr, *buf1 = nullptr, *buf2 = nullptr;
  bool tc = true;             // convolutions on tcgen05 (env VX_VAE_TC=0: CUDA-core FMA)
  uint16_t* xs = nullptr;     // split operand of the tcgen05 convs [2][B][T][C]
  size_t xs_elems = 0;

  template <typename T>
  T* alloc(size_t n) {
    void* p = nullptr;
    if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) return nullptr;
    allocs.push_back(p);
    return static_cast<T*>(p);
  }
};

namespace {

int vae_split_buffer(vx_vae* v, size_t elems) {
  if (elems <= v->xs_elems) return VX_OK;
  if (v->xs) cudaFree(v->xs);
  v->xs = nullptr;
  v->xs_elems = 0;
  if (cudaMalloc(&v->xs, elems * 2) != cudaSuccess) {
    cudaGetLastError();
    return fail(v->ctx, VX_ERR_OOM, "VAE split operand (%zu bf16) allocation failed", elems);
  }
  v->xs_elems = elems;
  return VX_OK;
}

int vae_buffers(vx_vae* v, size_t elems) {
  if (elems <= v->buf_elems) return VX_OK;
  for (float** p : {&v->buf0, &v->buf1, &v->buf2}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  v->buf_elems = 0;
  if (cudaMalloc(&v->buf0, elems * 4) != cudaSuccess || cudaMalloc(&v->buf1, elems * 4) != cudaSuccess ||
      cudaMalloc(&v->buf2, elems * 4) != cudaSuccess) {
    cudaGetLastError();
    return fail(v->ctx, VX_ERR_OOM, "VAE activation buffers (%zu floats x3) allocation failed", elems);
  }
  v->buf_elems = elems;
  return VX_OK;
}

cudaError_t launch_conv_gemm(const ConvGemmArgs& a, cudaStream_t st) {
  if (a.M % CG_BM != 0 || a.K % CG_BK != 0) return cudaErrorInvalidValue;
  dim3 grid((a.T_in + CG_BN - 1) / CG_BN, a.M / CG_BM, a.B * a.stride);
  count_launch();
  conv_gemm_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_dw(const float* x, int B, int C, int T, const uint16_t* w, const float* bias, int dil,
                      const float* a_pre, const float* a_post, float* y, cudaStream_t st,
                      const float* hist = nullptr) {
  if (dil < 1 || dil > 9) return cudaErrorInvalidValue;
  dim3 grid((T + DW_TT - 1) / DW_TT, C, B);
  count_launch();
  dw_conv_kernel<<<grid, 256, 0, st>>>(x, C, T, w, bias, dil, a_pre, a_post, y, hist);
  return cudaGetLastError();
}

cudaError_t launch_hist_update(float* hist, const float* x, int rows, int T, int H, cudaStream_t st) {
  if (H > 64) return cudaErrorInvalidValue;
  count_launch();
  hist_update_kernel<<<rows, 64, 0, st>>>(hist, x, T, H);
  return cudaGetLastError();
}

}  // namespace

// Streaming decode state: the last inputs of every causal layer (vx_vae_stream_*).
struct vx_vae_stream {
  vx_vae* v = nullptr;
  int B = 0;
  bool started = false;  // false: the next chunk is an utterance's first (zero padding)
  float* first = nullptr;                 // [B, latent, 6]: first depthwise conv input
  float* up[8] = {};                      // [B, C_in]: each transposed conv's last input frame
  float* unit[8][3] = {};                 // [B, C_out, 6 * dilation]: residual-unit depthwise inputs
  float* last = nullptr;                  // [B, C_last, 6]: last conv input
  std::vector<float*> allocs;
  std::vector<size_t> alloc_bytes;
};

namespace {

// AudioVae::decode (vae.rs:55-59) of z [B, latent, T].  With a stream state whose utterance
// has started, every causal layer reads the previous chunk's inputs as its left context instead
// of zero padding, and the state then takes this chunk's tail: chunk by chunk, the samples are
// identical to decoding the whole latent at once (the decoder is causal).
int vae_run(vx_vae* v, const float* z, int B, int T, float* wav, vx_vae_stream* sst) {
  vx_ctx* ctx = v->ctx;
  if (B <= 0 || T <= 0) return fail(ctx, VX_ERR_SHAPE, "vae_decode: empty input");
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  const bool hist = sst && sst->started;
  // largest activation: max over stages of C * T_stage
  size_t elems = (size_t)std::max(v->latent, v->dim) * T;
  size_t t = T;
  for (int i = 0; i < v->nblocks; ++i) {
    t *= v->rates[i];
    elems = std::max(elems, (size_t)v->blocks[i].cout * t);
  }
  elems *= B;
  int rc = vae_buffers(v, elems);
  if (rc) return rc;
  // the split operand of the tcgen05 convs: two bf16 planes of the largest conv input (one row
  // of history ahead of a streamed chunk)
  size_t xs_elems = (size_t)v->latent * T;
  t = T;
  for (int i = 0; i < v->nblocks; ++i) {
    xs_elems = std::max(xs_elems, (size_t)v->blocks[i].cin * (t + 1));
    t *= v->rates[i];
    xs_elems = std::max(xs_elems, (size_t)v->blocks[i].cout * t);
  }
  const bool tc_first = v->tc && v->latent % 64 == 0;
  if (v->tc && (rc = vae_split_buffer(v, 2 * xs_elems * B))) return rc;
  float *h = v->buf0, *y = v->buf1, *tmp = v->buf2;
  // first conv: depthwise k7 over the latent channels, then pointwise latent -> dim (decoder.rs:83-89)
  VX_CUDA(ctx, launch_dw(z, B, v->latent, T, v->first_dw_w, v->first_dw_b, 1, nullptr, nullptr, y, st,
                         hist ? sst->first : nullptr));
  if (sst) VX_CUDA(ctx, launch_hist_update(sst->first, z, B * v->latent, T, 6, st));
  if (tc_first) {
    VX_CUDA(ctx, launch_vae_split(y, B, v->latent, T, nullptr, nullptr, nullptr, v->xs, st));
    VX_CUDA(ctx, launch_vae_tc_conv(v->xs, B, T, v->latent, v->dim, 1, v->first_pw_w, v->first_pw_b, nullptr, h,
                                    ctx->dev_err, st));
  } else {
    ConvGemmArgs f = {v->first_pw_w, v->first_pw_b, y, nullptr, h, B, v->dim, v->latent, v->latent, T, 1,
                      nullptr, nullptr, nullptr};
    VX_CUDA(ctx, launch_conv_gemm(f, st));
  }
  int tl = T;
  for (int i = 0; i < v->nblocks; ++i) {
    VaeBlock& bl = v->blocks[i];
    // SR cond -> snake -> causal transposed conv (decoder.rs:158-162, 45-47)
    if (v->tc) {
      VX_CUDA(ctx, launch_vae_split(h, B, bl.cin, tl, bl.alpha, bl.sr_scale, bl.sr_bias, v->xs, st,
                                    hist ? sst->up[i] : nullptr));
      if (sst) VX_CUDA(ctx, launch_hist_update(sst->up[i], h, B * bl.cin, tl, 1, st));
      VX_CUDA(ctx, launch_vae_tc_conv(v->xs, B, tl, bl.cin, bl.cout, bl.stride, bl.up_wt, bl.up_b, nullptr, tmp,
                                      ctx->dev_err, st, hist ? 1 : 0));
    } else {
      ConvGemmArgs up = {bl.up_w, bl.up_b, h, nullptr, tmp, B, bl.cout, 2 * bl.cin, bl.cin, tl, bl.stride,
                         bl.alpha, bl.sr_scale, bl.sr_bias};
      VX_CUDA(ctx, launch_conv_gemm(up, st));
    }
    tl *= bl.stride;
    std::swap(h, tmp);
    const int dils[3] = {1, 3, 9};
    for (int u = 0; u < 3; ++u) {
      const VaeUnit& r = bl.res[u];
      // CausalResidualUnit: x + conv1x1(snake(dwconv7_dil(snake(x))))  (layers.rs:150-156)
      VX_CUDA(ctx, launch_dw(h, B, bl.cout, tl, r.w1, r.b1, dils[u], r.alpha1, r.alpha2, y, st,
                             hist ? sst->unit[i][u] : nullptr));
      if (sst) VX_CUDA(ctx, launch_hist_update(sst->unit[i][u], h, B * bl.cout, tl, 6 * dils[u], st));
      if (v->tc) {
        VX_CUDA(ctx, launch_vae_split(y, B, bl.cout, tl, nullptr, nullptr, nullptr, v->xs, st));
        VX_CUDA(ctx, launch_vae_tc_conv(v->xs, B, tl, bl.cout, bl.cout, 1, r.w2, r.b2, h, h, ctx->dev_err, st));
      } else {
        ConvGemmArgs pw = {r.w2, r.b2, y, h, h, B, bl.cout, bl.cout, bl.cout, tl, 1, nullptr, nullptr, nullptr};
        VX_CUDA(ctx, launch_conv_gemm(pw, st));
      }
    }
  }
  const int cl = v->dim >> v->nblocks;
  dim3 grid((tl + LC_TT - 1) / LC_TT, B);
  count_launch();
  last_conv_kernel<<<grid, 256, 0, st>>>(h, cl, tl, v->alpha_out, v->last_w, v->last_b, wav,
                                         hist ? sst->last : nullptr);
  VX_CUDA(ctx, cudaGetLastError());
  if (sst) VX_CUDA(ctx, launch_hist_update(sst->last, h, B * cl, tl, 6, st));
  return VX_OK;
}

}  // namespace

extern "C" {

int vx_vae_create(vx_ctx* ctx, const vx_vae_config* cfg, vx_vae** out) {
  if (!ctx || !cfg || !out) return VX_ERR_ARG;
  *out = nullptr;
  if (cfg->n_rates <= 0 || cfg->n_rates > 8 || cfg->latent_dim <= 0 || cfg->decoder_dim <= 0)
    return fail(ctx, VX_ERR_CONFIG, "vae_create: bad rates / dims");
  if (cfg->use_noise_block) return fail(ctx, VX_ERR_CONFIG, "NoiseBlock is not supported (off in VoxCPM2 weights)");
  if (!cfg->depthwise) return fail(ctx, VX_ERR_CONFIG, "only the depthwise decoder is supported");
  cudaSetDevice(ctx->device);
  vx_vae* v = new vx_vae();
  v->ctx = ctx;
  v->latent = cfg->latent_dim;
  v->dim = cfg->decoder_dim;
  v->depthwise = cfg->depthwise;
  v->nblocks = cfg->n_rates;
  v->out_sr = cfg->out_sample_rate;
  if (const char* e = getenv("VX_VAE_TC")) v->tc = atoi(e) != 0;
  for (int i = 0; i < cfg->n_rates; ++i) v->rates.push_back(cfg->rates[i]);
  // sr_bucket (layers.rs:225-228)
  if (cfg->n_sr_boundaries > 0) {
    int idx = cfg->n_sr_boundaries;
    for (int i = 0; i < cfg->n_sr_boundaries; ++i)
      if (cfg->out_sample_rate < cfg->sr_boundaries[i]) {
        idx = i;
        break;
      }
    v->sr_idx = idx;
    v->n_buckets = cfg->n_sr_boundaries + 1;
  }
  const int L = v->latent, D = v->dim;
  bool ok = (v->first_dw_w = v->alloc<uint16_t>((size_t)L * 7)) && (v->first_dw_b = v->alloc<float>(L)) &&
            (v->first_pw_w = v->alloc<uint16_t>((size_t)D * L)) && (v->first_pw_b = v->alloc<float>(D));
  for (int i = 0; ok && i < v->nblocks; ++i) {
    VaeBlock bl;
    bl.cin = D >> i;
    bl.cout = D >> (i + 1);
    bl.stride = v->rates[i];
    if (bl.cout % CG_BM != 0 || (2 * bl.cin) % CG_BK != 0 || bl.cout % CG_BK != 0) {
      vx_vae_destroy(v);
      return fail(ctx, VX_ERR_CONFIG, "block %d channels %d->%d must be multiples of 64", i, bl.cin, bl.cout);
    }
    ok = (bl.alpha = v->alloc<float>(bl.cin)) &&
         (bl.up_w = v->alloc<uint16_t>((size_t)bl.stride * bl.cout * 2 * bl.cin)) &&
         (bl.up_wt = v->alloc<uint16_t>((size_t)vae_tc_rows(bl.cout, bl.stride) * 2 * bl.cin)) &&
         (bl.up_b = v->alloc<float>(bl.cout));
    for (int u = 0; ok && u < 3; ++u) {
      VaeUnit& r = bl.res[u];
      ok = (r.alpha1 = v->alloc<float>(bl.cout)) && (r.alpha2 = v->alloc<float>(bl.cout)) &&
           (r.w1 = v->alloc<uint16_t>((size_t)bl.cout * 7)) && (r.b1 = v->alloc<float>(bl.cout)) &&
           (r.w2 = v->alloc<uint16_t>((size_t)bl.cout * bl.cout)) && (r.b2 = v->alloc<float>(bl.cout));
    }
    if (ok && v->sr_idx >= 0) ok = (bl.sr_scale = v->alloc<float>(bl.cin)) && (bl.sr_bias = v->alloc<float>(bl.cin));
    v->blocks.push_back(bl);
  }
  const int cl = D >> v->nblocks;
  ok = ok && (v->alpha_out = v->alloc<float>(cl)) && (v->last_w = v->alloc<uint16_t>((size_t)cl * 7)) &&
       (v->last_b = v->alloc<float>(1));
  if (!ok) {
    cudaGetLastError();
    vx_vae_destroy(v);
    return fail(ctx, VX_ERR_OOM, "VAE weight allocation failed");
  }
  *out = v;
  return VX_OK;
}

void vx_vae_destroy(vx_vae* v) {
  if (!v) return;
  cudaSetDevice(v->ctx->device);
  cudaStreamSynchronize(v->ctx->stream);
  for (void* p : v->allocs) cudaFree(p);
  for (float* p : {v->buf0, v->buf1, v->buf2})
    if (p) cudaFree(p);
  if (v->xs) cudaFree(v->xs);
  delete v;
}

int vx_vae_load_first(vx_vae* v, const uint16_t* dw_w, const float* dw_b, const uint16_t* pw_w, const float* pw_b) {
  if (!v || !dw_w || !dw_b || !pw_w || !pw_b) return VX_ERR_ARG;
  vx_ctx* ctx = v->ctx;
  cudaSetDevice(ctx->device);
  const size_t L = v->latent, D = v->dim;
  VX_CUDA(ctx, cudaMemcpy(v->first_dw_w, dw_w, L * 7 * 2, cudaMemcpyDefault));
  VX_CUDA(ctx, cudaMemcpy(v->first_dw_b, dw_b, L * 4, cudaMemcpyDefault));
  VX_CUDA(ctx, cudaMemcpy(v->first_pw_w, pw_w, D * L * 2, cudaMemcpyDefault));
  VX_CUDA(ctx, cudaMemcpy(v->first_pw_b, pw_b, D * 4, cudaMemcpyDefault));
  return VX_OK;
}

int vx_vae_load_block(vx_vae* v, int i, const vx_vae_block_weights* w) {
  if (!v || !w || !w->alpha || !w->up_w || !w->up_b) return VX_ERR_ARG;
  vx_ctx* ctx = v->ctx;
  if (i < 0 || i >= v->nblocks) return fail(ctx, VX_ERR_ARG, "block %d out of range", i);
  cudaSetDevice(ctx->device);
  VaeBlock& bl = v->blocks[i];
  const int ci = bl.cin, co = bl.cout, s = bl.stride;
  VX_CUDA(ctx, cudaMemcpy(bl.alpha, w->alpha, ci * 4, cudaMemcpyDefault));
  VX_CUDA(ctx, cudaMemcpy(bl.up_b, w->up_b, co * 4, cudaMemcpyDefault));
  // ConvTranspose1d weight [C_in, C_out, 2s] -> per-phase GEMM layout [s][C_out][2*C_in]:
  // A_r[o, k*C_in + c] = W[c, o, r + k*s]
  std::vector<uint16_t> src((size_t)ci * co * 2 * s), dst((size_t)s * co * 2 * ci);
  VX_CUDA(ctx, cudaMemcpy(src.data(), w->up_w, src.size() * 2, cudaMemcpyDefault));
  for (int r = 0; r < s; ++r)
    for (int o = 0; o < co; ++o)
      for (int k = 0; k < 2; ++k)
        for (int c = 0; c < ci; ++c)
          dst[((size_t)r * co + o) * 2 * ci + (size_t)k * ci + c] = src[((size_t)c * co + o) * 2 * s + r + k * s];
  VX_CUDA(ctx, cudaMemcpy(bl.up_w, dst.data(), dst.size() * 2, cudaMemcpyHostToDevice));
  // the tcgen05 path folds the phases into 128-row tiles of cpt = 128 / s channels: row
  // tile * 128 + q * s + r holds phase r of channel tile * cpt + q; rows past cpt * s are zero
  {
    const int cpt = 128 / s, rows = vae_tc_rows(co, s);
    std::vector<uint16_t> ft((size_t)rows * 2 * ci, 0);
    for (int row = 0; row < rows; ++row) {
      const int tile = row / 128, i = row % 128;
      const int o = tile * cpt + i / s, r = i % s;
      if (i >= cpt * s || o >= co) continue;
      for (int k = 0; k < 2; ++k)
        for (int c = 0; c < ci; ++c)
          ft[(size_t)row * 2 * ci + (size_t)k * ci + c] = src[((size_t)c * co + o) * 2 * s + r + k * s];
    }
    VX_CUDA(ctx, cudaMemcpy(bl.up_wt, ft.data(), ft.size() * 2, cudaMemcpyHostToDevice));
  }
  for (int u = 0; u < 3; ++u) {
    if (!w->res_alpha1[u] || !w->res_w1[u] || !w->res_b1[u] || !w->res_alpha2[u] || !w->res_w2[u] || !w->res_b2[u])
      return VX_ERR_ARG;
    VaeUnit& r = bl.res[u];
    VX_CUDA(ctx, cudaMemcpy(r.alpha1, w->res_alpha1[u], co * 4, cudaMemcpyDefault));
    VX_CUDA(ctx, cudaMemcpy(r.alpha2, w->res_alpha2[u], co * 4, cudaMemcpyDefault));
    VX_CUDA(ctx, cudaMemcpy(r.w1, w->res_w1[u], (size_t)co * 7 * 2, cudaMemcpyDefault));
    VX_CUDA(ctx, cudaMemcpy(r.b1, w->res_b1[u], co * 4, cudaMemcpyDefault));
    VX_CUDA(ctx, cudaMemcpy(r.w2, w->res_w2[u], (size_t)co * co * 2, cudaMemcpyDefault));
    VX_CUDA(ctx, cudaMemcpy(r.b2, w->res_b2[u], co * 4, cudaMemcpyDefault));
  }
  if (v->sr_idx >= 0) {
    // SampleRateConditionLayer embedding rows [buckets, C_in]: keep the configured bucket's row
    if (!w->sr_scale || !w->sr_bias) return VX_ERR_ARG;
    VX_CUDA(ctx, cudaMemcpy(bl.sr_scale, w->sr_scale + (size_t)v->sr_idx * ci, ci * 4, cudaMemcpyDefault));
    VX_CUDA(ctx, cudaMemcpy(bl.sr_bias, w->sr_bias + (size_t)v->sr_idx * ci, ci * 4, cudaMemcpyDefault));
  }
  return VX_OK;
}

int vx_vae_load_out(vx_vae* v, const float* alpha_out, const uint16_t* last_w, const float* last_b) {
  if (!v || !alpha_out || !last_w || !last_b) return VX_ERR_ARG;
  vx_ctx* ctx = v->ctx;
  cudaSetDevice(ctx->device);
  const int cl = v->dim >> v->nblocks;
  VX_CUDA(ctx, cudaMemcpy(v->alpha_out, alpha_out, cl * 4, cudaMemcpyDefault));
  VX_CUDA(ctx, cudaMemcpy(v->last_w, last_w, (size_t)cl * 7 * 2, cudaMemcpyDefault));
  VX_CUDA(ctx, cudaMemcpy(v->last_b, last_b, 4, cudaMemcpyDefault));
  return VX_OK;
}

int vx_vae_decode(vx_vae* v, const float* z, int B, int T, float* wav) {
  if (!v || !z || !wav) return VX_ERR_ARG;
  const int rc = vae_run(v, z, B, T, wav, nullptr);
  return rc ? rc : vx_ctx_synchronize(v->ctx);
}

int vx_vae_stream_create(vx_vae* v, int B, vx_vae_stream** out) {
  if (!v || !out || B <= 0) return VX_ERR_ARG;
  *out = nullptr;
  vx_ctx* ctx = v->ctx;
  if (!v->tc || v->latent % 64)
    return fail(ctx, VX_ERR_CONFIG, "streaming decode needs the tcgen05 convolutions (latent multiple of 64)");
  cudaSetDevice(ctx->device);
  vx_vae_stream* s = new vx_vae_stream();
  s->v = v;
  s->B = B;
  auto alloc = [&](size_t n) {
    float* p = nullptr;
    if (cudaMalloc(&p, n * 4) != cudaSuccess) {
      cudaGetLastError();
      return (float*)nullptr;
    }
    s->allocs.push_back(p);
    s->alloc_bytes.push_back(n * 4);
    return p;
  };
  const int dils[3] = {1, 3, 9};
  bool ok = (s->first = alloc((size_t)B * v->latent * 6)) != nullptr;
  for (int i = 0; ok && i < v->nblocks; ++i) {
    const VaeBlock& bl = v->blocks[i];
    ok = (s->up[i] = alloc((size_t)B * bl.cin)) != nullptr;
    for (int u = 0; ok && u < 3; ++u) ok = (s->unit[i][u] = alloc((size_t)B * bl.cout * 6 * dils[u])) != nullptr;
  }
  ok = ok && (s->last = alloc((size_t)B * (v->dim >> v->nblocks) * 6)) != nullptr;
  if (!ok) {
    vx_vae_stream_destroy(s);
    return fail(ctx, VX_ERR_OOM, "VAE stream state allocation failed");
  }
  *out = s;
  return vx_vae_stream_reset(s);
}

void vx_vae_stream_destroy(vx_vae_stream* s) {
  if (!s) return;
  cudaSetDevice(s->v->ctx->device);
  cudaStreamSynchronize(s->v->ctx->stream);
  for (float* p : s->allocs) cudaFree(p);
  delete s;
}

int vx_vae_stream_reset(vx_vae_stream* s) {
  if (!s) return VX_ERR_ARG;
  // the next chunk starts an utterance: histories of zeros are the causal zero padding (the
  // depthwise and last convs apply Snake1d to them, and snake(0) = 0); the transposed convs,
  // whose input transform does not map 0 to 0, read no history until a chunk has run
  s->started = false;
  vx_ctx* ctx = s->v->ctx;
  cudaSetDevice(ctx->device);
  for (size_t i = 0; i < s->allocs.size(); ++i)
    VX_CUDA(ctx, cudaMemsetAsync(s->allocs[i], 0, s->alloc_bytes[i], ctx->stream));
  return vx_ctx_synchronize(ctx);
}

int vx_vae_stream_decode(vx_vae_stream* s, const float* z, int T, float* wav) {
  if (!s || !z || !wav) return VX_ERR_ARG;
  const int rc = vae_run(s->v, z, s->B, T, wav, s);
  if (rc) return rc;
  s->started = true;
  return vx_ctx_synchronize(s->v->ctx);
}

}  // extern "C"

namespace vx {
vx_ctx* vae_ctx(vx_vae* v) { return v->ctx; }
int vae_latent(const vx_vae* v) { return v->latent; }
void vae_dims(const vx_vae* v, VaeDims* out) {
  out->latent = v->latent;
  out->dim = v->dim;
  out->nblocks = v->nblocks;
  for (int i = 0; i < 8; ++i) out->rates[i] = i < v->nblocks ? v->rates[i] : 0;
  out->n_buckets = v->n_buckets;
}
int vae_hop(const vx_vae* v) {
  int h = 1;
  for (int r : v->rates) h *= r;
  return h;
}
}  // namespace vx
