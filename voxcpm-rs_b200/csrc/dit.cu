// LocDiT V2 + unified CFM sampler (reference src/locdit/local_dit.rs, unified_cfm.rs).
//
// The DiT decoder is a MiniCPM-4 model object (vx_lm without vocabulary) run non-causally
// over the token sequence [mu tokens | time token | cond tokens | x tokens]
// (local_dit.rs:152).  Around it, small kernels do the channel-major projections
// (in_proj / cond_proj read [N, C, T] directly, out_proj writes [N, C, T] directly, so no
// swap_dims copies exist), the sinusoidal time embedding and the sequence assembly.
// vx_cfm_solve runs UnifiedCfm::forward + solve_euler with the noise z supplied by the
// caller; each Euler step is: time MLP (one row: t is the same for every row) -> assemble ->
// decoder -> out_proj -> fused CFG(-zero-star) + Euler update.
#include <cmath>
#include <map>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "runtime.cuh"
#include "tc_common.cuh"

using namespace vx;

namespace {

// dst[(n + k*Ns), row_off + t, h] = b[h] + sum_c W[h, c] * src[n, c, t]   for k < copies
// src [Ns, C, T] (channel-major, as the reference's [N, C, T] tensors), W bf16 [H, C].
__global__ void chan_proj_kernel(const float* __restrict__ src, int Ns, int C, int T, const uint16_t* __restrict__ W,
                                 const float* __restrict__ b, int H, float* __restrict__ dst, int S, int row_off,
                                 int copies) {
  // grid (Ns*T, ceil(H/256)): one output channel h per thread; the W row is read in 16-byte
  // chunks (C % 8 == 0), the input column (n, :, t) is staged in shared memory
  extern __shared__ float xs[];  // [C] column of one (n, t)
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x / T, t = blockIdx.x % T;
  for (int c = threadIdx.x; c < C; c += blockDim.x) xs[c] = src[((size_t)n * C + c) * T + t];
  __syncthreads();
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  if (h >= H) return;
  const uint4* w = reinterpret_cast<const uint4*>(W + (size_t)h * C);
  float acc = 0.f;
  for (int c8 = 0; c8 < C / 8; ++c8) acc = dot8(__ldg(w + c8), xs + c8 * 8, acc);
  const float v = acc + b[h];
  for (int k = 0; k < copies; ++k) dst[((size_t)(n + k * Ns) * S + row_off + t) * H + h] = v;
}

void launch_chan_proj(const float* src, int Ns, int C, int T, const uint16_t* W, const float* b, int H, float* dst,
                      int S, int row_off, int copies, cudaStream_t st) {
  count_launch();
  PdlLaunch l(dim3(Ns * T, (H + 255) / 256), dim3(256), C * sizeof(float), st);
  cudaLaunchKernelEx(&l.cfg, chan_proj_kernel, src, Ns, C, T, W, b, H, dst, S, row_off, copies);
}

// out[n, c, t] = b[c] + sum_h W[c, h] * hid[n, skip + t, h]   (out_proj + swap_dims, local_dit.rs:155-158)
__global__ void out_proj_kernel(const float* __restrict__ hid, int N, int S, int skip, int T, int H,
                                const uint16_t* __restrict__ W, const float* __restrict__ b, int C,
                                float* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N * C * T) return;
  const int t = warp % T, c = (warp / T) % C, n = warp / (T * C);
  const float* x = hid + ((size_t)n * S + skip + t) * H;
  const uint16_t* w = W + (size_t)c * H;
  float acc = 0.f;
  for (int h = lane; h < H; h += 32) acc = fmaf(__uint_as_float(((uint32_t)w[h]) << 16), x[h], acc);
  acc = warp_sum(acc);
  if (lane == 0) out[((size_t)n * C + c) * T + t] = acc + b[c];
}

// SinusoidalPosEmb::forward (local_dit.rs:24-32): out[n] = [sin(t_n*scale*f), cos(t_n*scale*f)]
// with f32 frequencies formed in f64 on the host.
__global__ void sinusoidal_kernel(const float* __restrict__ t, int n, float scale, const float* __restrict__ freqs,
                                  int half, float* __restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * half; i += gridDim.x * blockDim.x) {
    const int r = i / half, k = i % half;
    const float a = (t[r] * scale) * freqs[k];
    out[(size_t)r * 2 * half + k] = sinf(a);
    out[(size_t)r * 2 * half + half + k] = cosf(a);
  }
}

__global__ void silu_inplace_kernel(float* x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = silu(x[i]);
}

// seq rows 0..mu_tokens: mu (reshape [N, C_mu] -> [N, mu_tokens, H]); row mu_tokens: the time
// token temb[n % nt] + dtemb[n % nd] (local_dit.rs:147-152).
__global__ void seq_head_kernel(const float* __restrict__ mu, int mu_tokens, const float* __restrict__ temb, int nt,
                                const float* __restrict__ dtemb, int nd, int N, int S, int H, float* __restrict__ seq) {
  pdl_wait();
  pdl_launch_dependents();
  const int n = blockIdx.x;
  for (int i = threadIdx.x; i < (mu_tokens + 1) * H; i += blockDim.x) {
    const int r = i / H, h = i % H;
    float v;
    if (r < mu_tokens)
      v = mu[(size_t)n * mu_tokens * H + i];
    else
      v = temb[(size_t)(n % nt) * H + h] + dtemb[(size_t)(n % nd) * H + h];
    seq[((size_t)n * S + r) * H + h] = v;
  }
}

// Everything a captured CFM solve graph depends on besides the (fixed) buffers.
struct CfmKey {
  int B, C_mu, T, Tc, steps;
  float cfg, sway;
  int zero_star;
  bool operator==(const CfmKey& o) const {
    return B == o.B && C_mu == o.C_mu && T == o.T && Tc == o.Tc && steps == o.steps && cfg == o.cfg &&
           sway == o.sway && zero_star == o.zero_star;
  }
};

}  // namespace

struct vx_dit {
  vx_ctx* ctx = nullptr;
  vx_lm* dec = nullptr;
  int H = 0, C = 0, max_rows = 0;
  float emb_scale_unused = 0.f;
  // weights
  uint16_t *in_w = nullptr, *cond_w = nullptr, *out_w = nullptr, *t1_w = nullptr, *t2_w = nullptr,
           *dt1_w = nullptr, *dt2_w = nullptr;
  float *in_b = nullptr, *cond_b = nullptr, *out_b = nullptr, *t1_b = nullptr, *t2_b = nullptr, *dt1_b = nullptr,
        *dt2_b = nullptr;
  float* freqs = nullptr;  // [H/2]
  // work buffers (grown on demand)
  int cap_rows = 0, cap_S = 0;
  float *seq = nullptr, *hid = nullptr, *temb = nullptr, *dtemb = nullptr, *tmp = nullptr, *tvals = nullptr,
        *out2b = nullptr, *mu_in = nullptr, *cond_in = nullptr;
  // CFM solve: staged x, the per-step time schedule, and the captured solve graph
  float* xw = nullptr;
  size_t xw_cap = 0;
  float* tsched = nullptr;
  int tsched_cap = 0;
  float* temb_all = nullptr;  // [steps][H]: every Euler step's time embedding, computed once per solve
  float* temb_tmp = nullptr;  // [steps][H]: its scratch
  cudaGraphExec_t solve_exec = nullptr;
  CfmKey solve_key{};
  unsigned long long solve_kernels = 0;
  // persistent decoder forward (dit_persist.cu): one cooperative launch per DiT forward
  int dp_mode = -1;              // env VX_DIT_PERSIST: 0 never, 1 always, unset: above kDpMinRows rows
  PersistStack dp;               // persistent decoder forward state (dit_persist.cu)
};

namespace {

// The persistent forward (one cooperative launch per DiT forward) beats the per-kernel forward
// once the activation rows outgrow one 128-row GEMM pass's economy: measured CFM solve (10
// steps, CFG) per-kernel / persistent, ms: B=1 3.34 / 4.26, B=2 4.05 / 4.41, B=3 4.68 / 4.64,
// B=4 5.36 / 4.72, B=8 11.25 / 5.50 (B sequences pairs of 11 rows).
constexpr int kDpMinRows = 64;

int dit_buffers(vx_dit* d, int rows, int S, int C, int T, int Tc, int Cmu) {
  if (rows <= d->cap_rows && S <= d->cap_S) return VX_OK;
  float** bufs[] = {&d->seq, &d->hid, &d->temb, &d->dtemb, &d->tmp, &d->tvals, &d->out2b, &d->mu_in, &d->cond_in};
  for (float** p : bufs) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  const size_t H = d->H;
  const int r = std::max(rows, 2), s = std::max(S, 16);
  // T, Tc <= S and C_mu <= S*H, so sizing by s covers every later call with S <= cap_S
  (void)T;
  (void)Tc;
  (void)Cmu;
  const int tt = s, tc = s, cmu = s * (int)H;
  bool ok = cudaMalloc(&d->seq, (size_t)r * s * H * 4) == cudaSuccess &&
            cudaMalloc(&d->hid, (size_t)r * s * H * 4) == cudaSuccess &&
            cudaMalloc(&d->temb, (size_t)r * H * 4) == cudaSuccess && cudaMalloc(&d->dtemb, (size_t)r * H * 4) == cudaSuccess &&
            cudaMalloc(&d->tmp, (size_t)r * H * 4) == cudaSuccess && cudaMalloc(&d->tvals, (size_t)r * 4 + 64) == cudaSuccess &&
            cudaMalloc(&d->out2b, (size_t)r * C * tt * 4) == cudaSuccess &&
            cudaMalloc(&d->mu_in, (size_t)r * cmu * 4) == cudaSuccess &&
            cudaMalloc(&d->cond_in, (size_t)r * C * tc * 4) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    d->cap_rows = 0;
    return fail(d->ctx, VX_ERR_OOM, "DiT work buffers allocation failed");
  }
  d->cap_rows = r;
  d->cap_S = s;
  return VX_OK;
}

// tmp: scratch of rows x H floats (default d->tmp, which holds the forward's rows).
int launch_time_mlp(vx_dit* d, const uint16_t* w1, const float* b1, const uint16_t* w2, const float* b2,
                    const float* tvals, int rows, float* out, cudaStream_t st, float* tmp = nullptr) {
  // TimestepEmbedding::forward(SinusoidalPosEmb(t, 1000)) (local_dit.rs:50-54, 147-148)
  vx_ctx* ctx = d->ctx;
  const int H = d->H, half = H / 2;
  if (!tmp) tmp = d->tmp;
  count_launch();
  sinusoidal_kernel<<<std::max(1, (rows * half + 255) / 256), 256, 0, st>>>(tvals, rows, 1000.0f, d->freqs, half,
                                                                              tmp);
  VX_CUDA(ctx, cudaGetLastError());
  const LinearWorkspace* ws = lm_workspace(d->dec);
  int rc = linear(ctx, ws, tmp, H, rows, H, H, w1, b1, nullptr, 1.f, out, H, st);
  if (rc) return rc;
  count_launch();
  silu_inplace_kernel<<<std::max(1, (rows * H + 255) / 256), 256, 0, st>>>(out, (size_t)rows * H);
  VX_CUDA(ctx, cudaGetLastError());
  rc = linear(ctx, ws, out, H, rows, H, H, w2, b2, nullptr, 1.f, tmp, H, st);
  if (rc) return rc;
  VX_CUDA(ctx, cudaMemcpyAsync(out, tmp, (size_t)rows * H * 4, cudaMemcpyDeviceToDevice, st));
  return VX_OK;
}

// Prepare the persistent forward for N sequences of S tokens (outside any capture): check the
// shape once, allocate its buffers once for the most rows this DiT can take (so a captured graph
// never sees them move), and build the activation tensor maps for this row count (kept per
// count).  Returns false when the per-kernel forward must be used.
bool dp_wanted(const vx_dit* d, int N, int S) {
  return S <= 16 && (d->dp_mode == 1 || (d->dp_mode < 0 && N * S > kDpMinRows));
}

bool dp_prepare(vx_dit* d, int N, int S) {
  if (!dp_wanted(d, N, S)) return false;
  if (d->dp.grid < 0) {
    LmStackView v;
    lm_stack_view(d->dec, &v);
    bool oom = false;
    persist_stack_prepare(d->dp, v, d->max_rows * 16, getenv("VX_DIT_TRACE") != nullptr, &oom);
    if (oom) fail(d->ctx, VX_ERR_OOM, "persistent DiT buffers: allocation or tensor maps failed");
  }
  if (d->dp.grid <= 0 || !d->dp.seq_ok || N * S > d->dp.rmax) return false;
  return persist_stack_rows(d->dp, (N * S + 31) / 32 * 32);
}

// The decoder stack (MiniCpmModel::forward, non-causal) over N sequences of S rows of `in`,
// writing the final-norm rows into `out`: one persistent launch when prepared, else lm.cu's
// per-kernel forward.
int dit_decoder_forward(vx_dit* d, const float* in, int N, int S, float* out, cudaStream_t st) {
  vx_ctx* ctx = d->ctx;
  const int R = N * S;
  if (d->dp.grid > 0 && d->dp.seq_ok && dp_wanted(d, N, S) && d->dp.xmaps.count((R + 31) / 32 * 32)) {
    const DitPersistArgs a = persist_stack_args(d->dp, N, S, in, out, ctx->dev_err);
    VX_CUDA(ctx, launch_dit_persist(a, d->dp.grid, st));
    return VX_OK;
  }
  return vx_lm_forward(d->dec, in, N, S, 0, 0, out);
}

// One DiT forward on prepared inputs: seq rows [0, mu_tokens] already hold mu and the time
// token, rows [mu_tokens+1, mu_tokens+1+Tc) the projected cond.  Writes x tokens, runs the
// decoder and out_proj into `out` [N, C, T].
int dit_forward_prepared(vx_dit* d, const float* x, int Nx, int copies, int N, int S, int skip, int T, float* out,
                         cudaStream_t st) {
  vx_ctx* ctx = d->ctx;
  const int H = d->H, C = d->C;
  launch_chan_proj(x, Nx, C, T, d->in_w, d->in_b, H, d->seq, S, skip, copies, st);
  VX_CUDA(ctx, cudaGetLastError());
  int rc = dit_decoder_forward(d, d->seq, N, S, d->hid, st);
  if (rc) return rc;
  const int warps = N * C * T;
  count_launch();
  PdlLaunch lo(dim3((warps * 32 + 255) / 256), dim3(256), 0, st);
  VX_CUDA(ctx, cudaLaunchKernelEx(&lo.cfg, out_proj_kernel, (const float*)d->hid, N, S, skip, T, H,
                                  (const uint16_t*)d->out_w, (const float*)d->out_b, C, out));
  return VX_OK;
}

// Capture UnifiedCfm::solve_euler (unified_cfm.rs:72-163) for one shape / schedule as a CUDA
// graph over the staged buffers (mu_in, cond_in, xw).  The time grid (unified_cfm.rs:59-67,
// f64 arithmetic, f32 storage) is computed here and uploaded before the capture; skipped
// zero-star steps (dphi = 0, so x - 0*dt == x) are simply not recorded.
int build_solve_graph(vx_dit* d, const CfmKey& k) {
  vx_ctx* ctx = d->ctx;
  cudaStream_t st = ctx->stream;
  const int H = d->H, C = d->C, B = k.B, N = 2 * B;
  const int mu_tokens = k.C_mu / H, skip = k.Tc + mu_tokens + 1, S = skip + k.T;
  const int n = k.steps + 1;
  std::vector<float> ts(n);
  const double stepw = 1.0 / (double)k.steps;
  for (int i = 0; i < n; ++i) {
    const double tt = (double)(float)(1.0 - (double)i * stepw);
    ts[i] = (float)(tt + (double)k.sway * (std::cos(M_PI / 2.0 * tt) - 1.0 + tt));
  }
  double t = ts[0];
  double dt = (double)(ts[0] - ts[1]);
  const int zero_init_steps = (int)std::max((double)n * 0.04, 1.0);
  std::vector<float> tt(n, 0.f);  // tt[0] = 0: the delta-time embedding (non-mean mode, dt = 0)
  std::vector<double> dts(n, 0.0);
  std::vector<char> run(n, 0);
  for (int step = 1; step < n; ++step) {
    run[step] = !(k.zero_star && step <= zero_init_steps);
    tt[step] = (float)t;
    dts[step] = dt;
    t -= dt;
    if (step < n - 1) dt = t - (double)ts[step + 1];
  }
  VX_CUDA(ctx, cudaMemcpy(d->tsched, tt.data(), (size_t)n * 4, cudaMemcpyHostToDevice));

  const unsigned long long before = g_launches;
  cudaGraph_t g = nullptr;
  VX_CUDA(ctx, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  int rc = VX_OK;
  do {
    launch_chan_proj(d->cond_in, B, C, k.Tc, d->cond_w, d->cond_b, H, d->seq, S, mu_tokens + 1, 2, st);
    if (cudaGetLastError() != cudaSuccess) {
      rc = fail(ctx, VX_ERR_CUDA, "cfm graph: cond projection launch failed");
      break;
    }
    rc = launch_time_mlp(d, d->dt1_w, d->dt1_b, d->dt2_w, d->dt2_b, d->tsched, 1, d->dtemb, st);
    // the time embeddings of all steps at once (the t schedule is known up front): one
    // multi-row GEMM per layer of the time MLP instead of a GEMV pair per step
    if (!rc)
      rc = launch_time_mlp(d, d->t1_w, d->t1_b, d->t2_w, d->t2_b, d->tsched + 1, n - 1, d->temb_all, st, d->temb_tmp);
    for (int step = 1; step < n && !rc; ++step) {
      if (!run[step]) continue;
      count_launch();
      PdlLaunch lh(dim3(N), dim3(256), 0, st);
      if (cudaLaunchKernelEx(&lh.cfg, seq_head_kernel, (const float*)d->mu_in, mu_tokens,
                             (const float*)(d->temb_all + (size_t)(step - 1) * H), 1, (const float*)d->dtemb, 1, N, S,
                             H, d->seq) != cudaSuccess) {
        rc = fail(ctx, VX_ERR_CUDA, "cfm graph: sequence assembly launch failed");
        break;
      }
      rc = dit_forward_prepared(d, d->xw, B, 2, N, S, skip, k.T, d->out2b, st);
      if (rc) break;
      if (launch_cfg_euler(d->out2b, d->xw, B, C * k.T, (double)k.cfg, dts[step], k.zero_star, st) != cudaSuccess)
        rc = fail(ctx, VX_ERR_CUDA, "cfm graph: CFG/Euler launch failed");
    }
  } while (0);
  const cudaError_t e = cudaStreamEndCapture(st, &g);
  d->solve_kernels = g_launches - before;  // captured, not launched
  g_launches = before;
  if (rc || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return rc ? rc : cuda_fail(ctx, e, "cudaStreamEndCapture (cfm solve)");
  }
  const cudaError_t ei = cudaGraphInstantiate(&d->solve_exec, g, 0);
  cudaGraphDestroy(g);
  if (ei != cudaSuccess) return cuda_fail(ctx, ei, "cudaGraphInstantiate (cfm solve)");
  d->solve_key = k;
  return VX_OK;
}

}  // namespace

extern "C" {

int vx_dit_create(vx_ctx* ctx, const vx_minicpm4_config* cfg, int in_channels, int max_rows, vx_dit** out) {
  if (!ctx || !cfg || !out || in_channels <= 0 || max_rows <= 0) return VX_ERR_ARG;
  *out = nullptr;
  if (cfg->vocab_size != 0) return fail(ctx, VX_ERR_CONFIG, "vocab_size must be 0 for local DiT");
  if (cfg->hidden_size % 2) return fail(ctx, VX_ERR_CONFIG, "SinusoidalPosEmb requires even dim");
  if (in_channels % 8) return fail(ctx, VX_ERR_CONFIG, "in_channels must be a multiple of 8");
  vx_dit* d = new vx_dit();
  d->ctx = ctx;
  d->H = cfg->hidden_size;
  d->C = in_channels;
  d->max_rows = max_rows;
  if (const char* e = getenv("VX_DIT_PERSIST")) d->dp_mode = atoi(e) != 0 ? 1 : 0;
  int rc = vx_lm_create(ctx, cfg, max_rows, 64, &d->dec);
  if (rc) {
    delete d;
    return rc;
  }
  cudaSetDevice(ctx->device);
  const size_t H = d->H, C = in_channels;
  bool ok = cudaMalloc(&d->in_w, H * C * 2) == cudaSuccess && cudaMalloc(&d->cond_w, H * C * 2) == cudaSuccess &&
            cudaMalloc(&d->out_w, C * H * 2) == cudaSuccess && cudaMalloc(&d->t1_w, H * H * 2) == cudaSuccess &&
            cudaMalloc(&d->t2_w, H * H * 2) == cudaSuccess && cudaMalloc(&d->dt1_w, H * H * 2) == cudaSuccess &&
            cudaMalloc(&d->dt2_w, H * H * 2) == cudaSuccess && cudaMalloc(&d->in_b, H * 4) == cudaSuccess &&
            cudaMalloc(&d->cond_b, H * 4) == cudaSuccess && cudaMalloc(&d->out_b, C * 4) == cudaSuccess &&
            cudaMalloc(&d->t1_b, H * 4) == cudaSuccess && cudaMalloc(&d->t2_b, H * 4) == cudaSuccess &&
            cudaMalloc(&d->dt1_b, H * 4) == cudaSuccess && cudaMalloc(&d->dt2_b, H * 4) == cudaSuccess &&
            cudaMalloc(&d->freqs, H / 2 * 4) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    vx_dit_destroy(d);
    return fail(ctx, VX_ERR_OOM, "DiT allocation failed");
  }
  // SinusoidalPosEmb frequencies: exp(-ln(1e4) * i / (half - 1)) in f64, stored as f32
  const int half = d->H / 2;
  std::vector<float> f(half);
  const double emb_scale = std::log(10000.0) / ((double)half - 1.0);
  for (int i = 0; i < half; ++i) f[i] = (float)std::exp(-emb_scale * (double)i);
  if (cudaMemcpy(d->freqs, f.data(), half * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    vx_dit_destroy(d);
    return fail(ctx, VX_ERR_CUDA, "DiT frequency upload failed");
  }
  *out = d;
  return VX_OK;
}

void vx_dit_destroy(vx_dit* d) {
  if (!d) return;
  cudaSetDevice(d->ctx->device);
  cudaStreamSynchronize(d->ctx->stream);
  if (d->solve_exec) cudaGraphExecDestroy(d->solve_exec);
  persist_stack_free(d->dp);
  if (d->dec) vx_lm_destroy(d->dec);
  void* ptrs[] = {d->in_w, d->cond_w, d->out_w, d->t1_w, d->t2_w, d->dt1_w, d->dt2_w, d->in_b, d->cond_b,
                  d->out_b, d->t1_b, d->t2_b, d->dt1_b, d->dt2_b, d->freqs, d->seq, d->hid, d->temb,
                  d->dtemb, d->tmp, d->tvals, d->out2b, d->mu_in, d->cond_in, d->xw, d->tsched, d->temb_all, d->temb_tmp};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  delete d;
}

int vx_dit_load(vx_dit* d, const uint16_t* in_w, const float* in_b, const uint16_t* cond_w, const float* cond_b,
                const uint16_t* out_w, const float* out_b, const uint16_t* t1_w, const float* t1_b,
                const uint16_t* t2_w, const float* t2_b, const uint16_t* dt1_w, const float* dt1_b,
                const uint16_t* dt2_w, const float* dt2_b) {
  if (!d || !in_w || !in_b || !cond_w || !cond_b || !out_w || !out_b || !t1_w || !t1_b || !t2_w || !t2_b ||
      !dt1_w || !dt1_b || !dt2_w || !dt2_b)
    return VX_ERR_ARG;
  vx_ctx* ctx = d->ctx;
  cudaSetDevice(ctx->device);
  const size_t H = d->H, C = d->C;
  struct Cp {
    void* dst;
    const void* src;
    size_t n;
  } cps[] = {{d->in_w, in_w, H * C * 2},   {d->in_b, in_b, H * 4},     {d->cond_w, cond_w, H * C * 2},
             {d->cond_b, cond_b, H * 4},   {d->out_w, out_w, C * H * 2}, {d->out_b, out_b, C * 4},
             {d->t1_w, t1_w, H * H * 2},   {d->t1_b, t1_b, H * 4},     {d->t2_w, t2_w, H * H * 2},
             {d->t2_b, t2_b, H * 4},       {d->dt1_w, dt1_w, H * H * 2}, {d->dt1_b, dt1_b, H * 4},
             {d->dt2_w, dt2_w, H * H * 2}, {d->dt2_b, dt2_b, H * 4}};
  for (const Cp& c : cps) VX_CUDA(ctx, cudaMemcpy(c.dst, c.src, c.n, cudaMemcpyDefault));
  return VX_OK;
}

int vx_dit_load_layer(vx_dit* d, int layer, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const uint16_t* o, const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                      const float* ln_in, const float* ln_post) {
  if (!d) return VX_ERR_ARG;
  return vx_lm_load_layer(d->dec, layer, q, k, v, o, gate, up, down, ln_in, ln_post);
}

int vx_dit_load_norm(vx_dit* d, const float* w) {
  if (!d) return VX_ERR_ARG;
  return vx_lm_load_norm(d->dec, w);
}

int vx_dit_forward(vx_dit* d, const float* x, const float* mu, const float* t, const float* cond, const float* dt,
                   int N, int C_mu, int T, int Tc, float* out) {
  if (!d || !x || !mu || !t || !cond || !dt || !out) return VX_ERR_ARG;
  vx_ctx* ctx = d->ctx;
  const int H = d->H, C = d->C;
  if (N <= 0 || N > d->max_rows || T <= 0 || Tc <= 0 || C_mu % H != 0)
    return fail(ctx, VX_ERR_SHAPE, "dit_forward: N=%d (max %d), T=%d, Tc=%d, C_mu=%d (multiple of %d)", N, d->max_rows,
                T, Tc, C_mu, H);
  const int mu_tokens = C_mu / H, skip = Tc + mu_tokens + 1, S = skip + T;
  if (S > 64) return fail(ctx, VX_ERR_SHAPE, "dit_forward: sequence %d > 64", S);
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  int rc = dit_buffers(d, N, S, C, T, Tc, C_mu);
  if (rc) return rc;
  dp_prepare(d, N, S);
  // prepare (local_dit.rs:116-134): cond_proj, delta-time MLP(dt)
  launch_chan_proj(cond, N, C, Tc, d->cond_w, d->cond_b, H, d->seq, S, mu_tokens + 1, 1, st);
  VX_CUDA(ctx, cudaGetLastError());
  VX_CUDA(ctx, cudaMemcpyAsync(d->tvals, dt, (size_t)N * 4, cudaMemcpyDefault, st));
  rc = launch_time_mlp(d, d->dt1_w, d->dt1_b, d->dt2_w, d->dt2_b, d->tvals, N, d->dtemb, st);
  if (rc) return rc;
  VX_CUDA(ctx, cudaMemcpyAsync(d->tvals, t, (size_t)N * 4, cudaMemcpyDefault, st));
  rc = launch_time_mlp(d, d->t1_w, d->t1_b, d->t2_w, d->t2_b, d->tvals, N, d->temb, st);
  if (rc) return rc;
  count_launch();
  seq_head_kernel<<<N, 256, 0, st>>>(mu, mu_tokens, d->temb, N, d->dtemb, N, N, S, H, d->seq);
  VX_CUDA(ctx, cudaGetLastError());
  rc = dit_forward_prepared(d, x, N, 1, N, S, skip, T, out, st);
  if (rc) return rc;
  return vx_ctx_synchronize(ctx);
}

int vx_cfm_solve(vx_dit* d, const float* mu, const float* cond, const float* z, int B, int C_mu, int T, int Tc,
                 int n_timesteps, float cfg_value, float sway_sampling_coef, int use_cfg_zero_star, float* x_out) {
  const int rc = vx::cfm_solve_enqueue(d, mu, cond, z, B, C_mu, T, Tc, n_timesteps, cfg_value, sway_sampling_coef,
                                       use_cfg_zero_star, x_out);
  if (rc) return rc;
  return vx_ctx_synchronize(d->ctx);
}

int vx_dit_trace(vx_dit* d, unsigned long long* out, int n, int* grid, int* phases) {
  return vx::dit_trace_copy(d, out, n, grid, phases);
}

}  // extern "C"

namespace vx {

// vx_cfm_solve without the final synchronisation: the solve is queued on the context stream
// (inputs staged, the captured graph launched, the result copied to x_out).
int cfm_solve_enqueue(vx_dit* d, const float* mu, const float* cond, const float* z, int B, int C_mu, int T, int Tc,
                      int n_timesteps, float cfg_value, float sway_sampling_coef, int use_cfg_zero_star,
                      float* x_out) {
  if (!d || !mu || !cond || !z || !x_out) return VX_ERR_ARG;
  vx_ctx* ctx = d->ctx;
  const int H = d->H, C = d->C, N = 2 * B;
  if (B <= 0 || N > d->max_rows || T <= 0 || Tc <= 0 || C_mu % H != 0 || n_timesteps < 1)
    return fail(ctx, VX_ERR_SHAPE, "cfm_solve: B=%d (2B <= %d), T=%d, Tc=%d, C_mu=%d, steps=%d", B, d->max_rows, T, Tc,
                C_mu, n_timesteps);
  const int mu_tokens = C_mu / H, skip = Tc + mu_tokens + 1, S = skip + T;
  if (S > 64) return fail(ctx, VX_ERR_SHAPE, "cfm_solve: sequence %d > 64", S);
  if (ctx->cancel.load(std::memory_order_relaxed)) return fail(ctx, VX_ERR_CANCELLED, "generation cancelled");
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  // every allocation happens here, outside any capture
  int rc = dit_buffers(d, N, S, C, T, Tc, C_mu);
  if (rc) return rc;
  rc = lm_prepare_rows(d->dec, (size_t)N * S);
  if (rc) return rc;
  dp_prepare(d, N, S);
  if (!d->xw || d->xw_cap < (size_t)B * C * T) {
    if (d->xw) cudaFree(d->xw);
    d->xw = nullptr;
    d->xw_cap = 0;
    VX_CUDA(ctx, cudaMalloc(&d->xw, (size_t)B * C * T * 4));
    d->xw_cap = (size_t)B * C * T;
  }
  if (!d->tsched || d->tsched_cap < n_timesteps + 2) {
    if (d->tsched) cudaFree(d->tsched);
    d->tsched = nullptr;
    VX_CUDA(ctx, cudaMalloc(&d->tsched, (size_t)(n_timesteps + 2) * 4));
    d->tsched_cap = n_timesteps + 2;
    for (float** p : {&d->temb_all, &d->temb_tmp}) {
      if (*p) cudaFree(*p);
      *p = nullptr;
      VX_CUDA(ctx, cudaMalloc(p, (size_t)(n_timesteps + 2) * d->H * 4));
    }
  }
  // inputs staged into fixed buffers so one captured graph serves every call with this shape:
  // mu_in = [mu; 0], cond_in = [cond; cond] (unified_cfm.rs:96-98), x = z
  VX_CUDA(ctx, cudaMemcpyAsync(d->mu_in, mu, (size_t)B * C_mu * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemsetAsync(d->mu_in + (size_t)B * C_mu, 0, (size_t)B * C_mu * 4, st));
  VX_CUDA(ctx, cudaMemcpyAsync(d->cond_in, cond, (size_t)B * C * Tc * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(d->xw, z, (size_t)B * C * T * 4, cudaMemcpyDefault, st));
  const CfmKey key = {B, C_mu, T, Tc, n_timesteps, cfg_value, sway_sampling_coef, use_cfg_zero_star};
  if (!d->solve_exec || !(key == d->solve_key)) {
    if (d->solve_exec) cudaGraphExecDestroy(d->solve_exec);
    d->solve_exec = nullptr;
    rc = build_solve_graph(d, key);
    if (rc) return rc;
  }
  VX_CUDA(ctx, cudaGraphLaunch(d->solve_exec, st));
  count_launch(d->solve_kernels);
  VX_CUDA(ctx, cudaMemcpyAsync(x_out, d->xw, (size_t)B * C * T * 4, cudaMemcpyDefault, st));
  return VX_OK;
}

vx_ctx* dit_ctx(vx_dit* d) { return d->ctx; }
int dit_in_channels(const vx_dit* d) { return d->C; }
int dit_trace_copy(vx_dit* d, unsigned long long* out, int n, int* grid, int* phases) {
  if (!d || !out || !grid || !phases || !d->dp.trace) return VX_ERR_ARG;
  *grid = d->dp.grid;
  *phases = 8 * d->dp.view.L + 1;
  const size_t need = (size_t)*grid * *phases * 4;
  if ((size_t)n < need) return VX_ERR_ARG;
  VX_CUDA(d->ctx, cudaMemcpy(out, d->dp.trace, need * 8, cudaMemcpyDeviceToHost));
  return VX_OK;
}
int dit_hidden_size(const vx_dit* d) { return d->H; }
vx_lm* dit_decoder(vx_dit* d, int* H, int* C) {
  *H = d->H;
  *C = d->C;
  return d->dec;
}
}  // namespace vx
