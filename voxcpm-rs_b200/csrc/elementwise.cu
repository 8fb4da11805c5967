// Row-wise and elementwise kernels of the hot path (sm_100a):
//   * fused residual-add + RMSNorm          (layer.rs:33-38 + mod.rs:54-68)
//   * RoPE + KV-cache scatter for S>1 rows  (rope.rs:76-95, attention.rs:55-88, cache.rs:47-58)
//   * SiLU-gate multiply for S>1 rows       (mlp.rs:31-33)
//   * token embedding * scale_emb           (minicpm4/model.rs:87-92, voxcpm2/model.rs:145)
//   * fused CFG(-zero-star) + Euler update   (unified_cfm.rs:132-158)
#include <algorithm>
#include <cfloat>
#include <climits>

#include "common.cuh"
#include "gemv.cuh"

namespace vx {

// ------------------------------------------------------------ residual add + RMSNorm
// h = r + x * resid_scale (h = x when r is absent); y = h * (mean(h^2)+eps)^-1/2 * w.
// One CTA per row; each thread keeps its slice of the row in registers (hidden <= 8192).
// Every load of the row (x, r and the norm weight) is issued before the first arithmetic on
// them, so a CTA waits for one DRAM round trip (loads interleaved with their uses behind the
// residual and bounds branches had cost a second one), and h, which does not depend on the
// norm, is stored before the reduction: 4.66 -> 4.09 us per call at [512, 2048].
template <int VPT, bool EXACT, bool HAS_R>  // VPT float4 per thread; EXACT: hidden == VPT * 1024
__global__ void __launch_bounds__(256) rmsnorm_residual_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ r,
                                                               const float* __restrict__ w, float resid_scale,
                                                               float eps, int hidden, float* h_out, float* y_out,
                                                               uint16_t* xs) {
  __shared__ float red[8];
  pdl_wait();
  pdl_launch_dependents();
  const size_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * hidden);
  const float4* rr = HAS_R ? reinterpret_cast<const float4*>(r + row * hidden) : nullptr;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const int n4 = hidden / 4;
  float4 v[VPT], b[VPT], ww[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * 256;
    if (EXACT || c < n4) {
      v[i] = __ldcs(xr + c);
      if (HAS_R) b[i] = __ldcs(rr + c);
      ww[i] = __ldg(w4 + c);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * 256;
    if (EXACT || c < n4) {
      float4 a = v[i];
      if (HAS_R) {
        a.x = b[i].x + a.x * resid_scale;
        a.y = b[i].y + a.y * resid_scale;
        a.z = b[i].z + a.z * resid_scale;
        a.w = b[i].w + a.w * resid_scale;
      }
      v[i] = a;
      ss = fmaf(a.x, a.x, ss);
      ss = fmaf(a.y, a.y, ss);
      ss = fmaf(a.z, a.z, ss);
      ss = fmaf(a.w, a.w, ss);
      if (h_out) __stcs(reinterpret_cast<float4*>(h_out + row * hidden) + c, a);
    }
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)hidden + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * 256;
    if (EXACT || c < n4) {
      float4 y;
      y.x = (v[i].x * inv) * ww[i].x;
      y.y = (v[i].y * inv) * ww[i].y;
      y.z = (v[i].z * inv) * ww[i].z;
      y.w = (v[i].w * inv) * ww[i].w;
      if (y_out) __stcs(reinterpret_cast<float4*>(y_out + row * hidden) + c, y);
      if (xs) store_split4(xs, gridDim.x, hidden, row, c * 4, y);
    }
  }
}

template <int VPT>
static cudaError_t launch_rmsnorm_vpt(const cudaLaunchConfig_t& cfg, const float* x, const float* r, const float* w,
                                      float resid_scale, float eps, int hidden, float* h_out, float* y_out,
                                      uint16_t* xs) {
  const bool exact = hidden == VPT * 1024;
  if (exact && r)
    return cudaLaunchKernelEx(&cfg, rmsnorm_residual_kernel<VPT, true, true>, x, r, w, resid_scale, eps, hidden, h_out,
                              y_out, xs);
  if (exact)
    return cudaLaunchKernelEx(&cfg, rmsnorm_residual_kernel<VPT, true, false>, x, r, w, resid_scale, eps, hidden,
                              h_out, y_out, xs);
  if (r)
    return cudaLaunchKernelEx(&cfg, rmsnorm_residual_kernel<VPT, false, true>, x, r, w, resid_scale, eps, hidden,
                              h_out, y_out, xs);
  return cudaLaunchKernelEx(&cfg, rmsnorm_residual_kernel<VPT, false, false>, x, r, w, resid_scale, eps, hidden, h_out,
                            y_out, xs);
}

cudaError_t launch_rmsnorm_residual(const float* x, const float* r, const float* w, float resid_scale,
                                    float eps, int rows, int hidden, float* h_out, float* y_out,
                                    cudaStream_t st, uint16_t* xs) {
  if (hidden % 4 != 0 || hidden > 8192 || rows <= 0) return cudaErrorInvalidValue;
  const int n4 = hidden / 4;
  const int vpt = (n4 + 255) / 256;
  count_launch();
  // programmatic dependent launch: the kernel waits for its predecessor at entry, so its CTAs
  // may be scheduled while the previous kernel drains
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vpt <= 1) return launch_rmsnorm_vpt<1>(cfg, x, r, w, resid_scale, eps, hidden, h_out, y_out, xs);
  if (vpt <= 2) return launch_rmsnorm_vpt<2>(cfg, x, r, w, resid_scale, eps, hidden, h_out, y_out, xs);
  if (vpt <= 4) return launch_rmsnorm_vpt<4>(cfg, x, r, w, resid_scale, eps, hidden, h_out, y_out, xs);
  return launch_rmsnorm_vpt<8>(cfg, x, r, w, resid_scale, eps, hidden, h_out, y_out, xs);
}

// ------------------------------------------------------------ RoPE + KV scatter (S rows)
// qkv [B*S, (nh+2nkv)*d] raw projections.  q_out [B*S, nh*d] (rotated);
// k (rotated) and v written to cache [B, nkv, s_max, d] at position pos0 + s, where pos0 is
// *pos_ptr when pos_ptr is given (a graph-replayed batched decode step).
// Rope angles use position pos0 + s, formed in f64 (rope.rs:38-46).
__global__ void rope_scatter_kernel(const float* __restrict__ qkv, int B, int S, int nh, int nkv, int d,
                                    const RopeParams* rope, int pos0, const int* pos_ptr, float* q_out, float* kcache,
                                    float* vcache, int s_max) {
  pdl_wait();
  pdl_launch_dependents();
  const int half = d / 2;
  const int heads = nh + 2 * nkv;
  if (pos_ptr) pos0 = *pos_ptr;
  const size_t total = (size_t)B * S * heads * half;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int i = idx % half;
    const int h = (idx / half) % heads;
    const size_t tok = idx / ((size_t)half * heads);
    const int b = tok / S, s = tok % S;
    const int pos = pos0 + s;
    const float* src = qkv + tok * (size_t)heads * d + (size_t)h * d;
    const float xa = src[i], xb = src[i + half];
    float oa = xa, ob = xb;
    if (h < nh + nkv && rope != nullptr) {
      const double f = ((double)pos * rope->inv_freq[i]) / rope->ext[i];
      double sd, cd;
      sincos(f, &sd, &cd);
      const float c = (float)(cd * rope->scaling_factor), sn = (float)(sd * rope->scaling_factor);
      oa = __fadd_rn(__fmul_rn(xa, c), __fmul_rn(-xb, sn));
      ob = __fadd_rn(__fmul_rn(xb, c), __fmul_rn(xa, sn));
    }
    if (h < nh) {
      float* dst = q_out + tok * (size_t)nh * d + (size_t)h * d;
      dst[i] = oa;
      dst[i + half] = ob;
    } else {
      const bool is_k = h < nh + nkv;
      const int g = is_k ? h - nh : h - nh - nkv;
      float* dst = (is_k ? kcache : vcache) + (((size_t)b * nkv + g) * s_max + pos) * d;
      dst[i] = oa;
      dst[i + half] = ob;
    }
  }
}

cudaError_t launch_rope_scatter(const float* qkv, int B, int S, int nh, int nkv, int d, const RopeParams* rope,
                                int pos0, float* q_out, float* kcache, float* vcache, int s_max,
                                cudaStream_t st, const int* pos_ptr) {
  const size_t total = (size_t)B * S * (nh + 2 * nkv) * (d / 2);
  const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  count_launch();
  PdlLaunch l(dim3(grid), dim3(256), 0, st);
  return cudaLaunchKernelEx(&l.cfg, rope_scatter_kernel, qkv, B, S, nh, nkv, d, rope, pos0, pos_ptr, q_out, kcache,
                            vcache, s_max);
}

// ------------------------------------------------------------ LongRoPE table
// cos / sin (x scaling factor) at positions 0..n_pos-1 from the f64 angles (rope.rs:38-46,
// the same expression as rope_scatter_kernel, so a table entry has the bits that kernel
// computes in place): out [n_pos][2][half] (cos row, then sin row).
__global__ void rope_table_kernel(const RopeParams* rp, int n_pos, int half, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_pos * half) return;
  const int p = i / half, j = i % half;
  const double f = ((double)p * rp->inv_freq[j]) / rp->ext[j];
  double sd, cd;
  sincos(f, &sd, &cd);
  out[(size_t)p * 2 * half + j] = (float)(cd * rp->scaling_factor);
  out[(size_t)p * 2 * half + half + j] = (float)(sd * rp->scaling_factor);
}

cudaError_t launch_rope_table(const RopeParams* rp, int n_pos, int half, float* out, cudaStream_t st) {
  const int n = n_pos * half;
  if (n <= 0) return cudaErrorInvalidValue;
  count_launch();
  rope_table_kernel<<<(n + 255) / 256, 256, 0, st>>>(rp, n_pos, half, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------ RoPE apply on [B,H,S,D]
// apply_rotary_pos_emb with explicit cos/sin rows [S, D] (rope.rs:76-95), in place.
__global__ void rope_apply_kernel(float* x, int B, int H, int S, int d, const float* cos, const float* sin) {
  const int half = d / 2;
  const size_t total = (size_t)B * H * S * half;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int i = idx % half;
    const size_t rowi = idx / half;  // (b, h, s)
    const int s = rowi % S;
    float* p = x + rowi * d;
    const float xa = p[i], xb = p[i + half];
    const float ca = cos[(size_t)s * d + i], cb = cos[(size_t)s * d + i + half];
    const float sa = sin[(size_t)s * d + i], sb = sin[(size_t)s * d + i + half];
    p[i] = __fadd_rn(__fmul_rn(xa, ca), __fmul_rn(-xb, sa));
    p[i + half] = __fadd_rn(__fmul_rn(xb, cb), __fmul_rn(xa, sb));
  }
}

cudaError_t launch_rope_apply(float* x, int B, int H, int S, int d, const float* cos, const float* sin,
                              cudaStream_t st) {
  const size_t total = (size_t)B * H * S * (d / 2);
  if (total == 0) return cudaSuccess;
  const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  count_launch();
  rope_apply_kernel<<<grid, 256, 0, st>>>(x, B, H, S, d, cos, sin);
  return cudaGetLastError();
}

// ------------------------------------------------------------ SiLU gate * up (S rows)
__global__ void silu_mul_kernel(const float* __restrict__ gu, int M, int inter, float* __restrict__ act,
                                uint16_t* __restrict__ xs) {
  pdl_wait();
  pdl_launch_dependents();
  if (xs) {  // straight into the down projection's split operand, four channels per thread
    const size_t total4 = (size_t)M * inter / 4;
    for (size_t q = blockIdx.x * (size_t)blockDim.x + threadIdx.x; q < total4; q += (size_t)gridDim.x * blockDim.x) {
      const size_t m = q / (inter / 4);
      const int i = (int)(q % (inter / 4)) * 4;
      const float4 g = *reinterpret_cast<const float4*>(gu + m * 2 * inter + i);
      const float4 u = *reinterpret_cast<const float4*>(gu + m * 2 * inter + inter + i);
      store_split4(xs, M, inter, m, i, make_float4(silu(g.x) * u.x, silu(g.y) * u.y, silu(g.z) * u.z, silu(g.w) * u.w));
    }
    return;
  }
  const size_t total = (size_t)M * inter;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t m = idx / inter, i = idx % inter;
    const float g = gu[m * 2 * inter + i], u = gu[m * 2 * inter + inter + i];
    act[idx] = silu(g) * u;
  }
}

cudaError_t launch_silu_mul(const float* gu, int M, int inter, float* act, cudaStream_t st, uint16_t* xs) {
  if (xs && (inter % 4 != 0 || ((uintptr_t)gu & 15))) return cudaErrorInvalidValue;
  const size_t total = xs ? (size_t)M * inter / 4 : (size_t)M * inter;
  const int grid = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  count_launch();
  PdlLaunch l(dim3(grid), dim3(256), 0, st);
  return cudaLaunchKernelEx(&l.cfg, silu_mul_kernel, gu, M, inter, act, xs);
}

// ------------------------------------------------------------ embedding gather
__global__ void embed_kernel(const uint16_t* __restrict__ E, const int* __restrict__ ids, int n, int H, int V,
                             float scale, float* __restrict__ out) {
  for (int m = blockIdx.x; m < n; m += gridDim.x) {
    int id = ids[m];
    if (id < 0 || id >= V) id = 0;  // out-of-range ids never index past the table
    const uint16_t* e = E + (size_t)id * H;
    for (int k = threadIdx.x; k < H; k += blockDim.x)
      out[(size_t)m * H + k] = __uint_as_float(((uint32_t)e[k]) << 16) * scale;
  }
}

cudaError_t launch_embed(const uint16_t* E, const int* ids, int n, int H, int V, float scale, float* out,
                         cudaStream_t st) {
  count_launch();
  embed_kernel<<<n < 1024 ? n : 1024, 256, 0, st>>>(E, ids, n, H, V, scale, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------ batched greedy pick
// One CTA per row b of logits [B, V]: argmax (ties -> lowest id), the id goes to
// tokens[*step * ld_tokens + b] and the row's next input embed(id) * scale to next_x [B, H].
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ logits, int V, const int* step,
                                                           int* tokens, int ld_tokens, const uint16_t* __restrict__ E,
                                                           int H, float scale, float* next_x) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = logits + (size_t)b * V;
  float bv = -FLT_MAX;
  int bi = INT_MAX;
  for (int i = tid; i < V; i += blockDim.x) {
    const float v = __ldg(row + i);
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
        bv = sv[w];
        bi = si[w];
      }
    if (bi < 0 || bi >= V) bi = 0;
    tokens[(size_t)(*step) * ld_tokens + b] = bi;
    si[0] = bi;
  }
  __syncthreads();
  const uint16_t* e = E + (size_t)si[0] * H;
  for (int k = tid; k < H; k += blockDim.x) next_x[(size_t)b * H + k] = __uint_as_float(((uint32_t)e[k]) << 16) * scale;
}

__global__ void advance_kernel(int* pos, int* step, int inc_pos) {
  if (inc_pos) *pos += 1;
  *step += 1;
}

cudaError_t launch_argmax_rows(const float* logits, int B, int V, const int* step, int* tokens, int ld_tokens,
                               const uint16_t* E, int H, float scale, float* next_x, cudaStream_t st) {
  count_launch();
  argmax_rows_kernel<<<B, 1024, 0, st>>>(logits, V, step, tokens, ld_tokens, E, H, scale, next_x);
  return cudaGetLastError();
}

cudaError_t launch_advance(int* pos, int* step, bool inc_pos, cudaStream_t st) {
  count_launch();
  advance_kernel<<<1, 1, 0, st>>>(pos, step, inc_pos ? 1 : 0);
  return cudaGetLastError();
}

// ------------------------------------------------------------ CFG + Euler (fused)
// out2b [2B, C, T]: rows 0..B are the conditional (pos) branch, B..2B the unconditional
// (neg) one.  One CTA per batch element: the zero-star projection st = <pos,neg>/(|neg|^2+1e-8)
// is a block reduction, then v and x <- x - dt * v are applied in the same pass.
__global__ void __launch_bounds__(256) cfg_euler_kernel(const float* __restrict__ out2b, float* __restrict__ x,
                                                        int B, int n, float cfg, float one_minus_cfg, float dt,
                                                        int zero_star) {
  __shared__ float red[2][8];
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const float* pos = out2b + (size_t)b * n;
  const float* neg = out2b + (size_t)(B + b) * n;
  float* xb = x + (size_t)b * n;
  float st_scaled = 0.f;
  if (zero_star) {
    float dot = 0.f, sq = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) {
      const float p = pos[i], q = neg[i];
      dot = fmaf(p, q, dot);
      sq = fmaf(q, q, sq);
    }
    dot = warp_sum(dot);
    sq = warp_sum(sq);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
      red[0][warp] = dot;
      red[1][warp] = sq;
    }
    __syncthreads();
    float D = 0.f, Q = 0.f;
    for (int w = 0; w < 8; ++w) {
      D += red[0][w];
      Q += red[1][w];
    }
    const float st = D / (Q + 1e-8f);
    st_scaled = st * one_minus_cfg;  // st.mul_scalar(1 - cfg), 1-cfg formed in f64 (unified_cfm.rs:148)
  }
  for (int i = threadIdx.x; i < n; i += 256) {
    const float p = pos[i], q = neg[i];
    float v;
    if (zero_star)
      v = q * st_scaled + p * cfg;  // neg*st*(1-cfg) + pos*cfg (unified_cfm.rs:149)
    else
      v = q + (p - q) * cfg;  // neg + (pos-neg)*cfg (unified_cfm.rs:151)
    xb[i] = xb[i] - v * dt;   // x - dphi*dt (unified_cfm.rs:155)
  }
}

// ScalarQuantizationLayer::forward's quantiser (fsq.rs:26-27): round(tanh(h) * scale) / scale,
// each step in f32 (the reference's f64 scalar is applied to an f32 tensor), round half away
// from zero as Rust's f32::round.
__global__ void __launch_bounds__(256) fsq_quant_kernel(float* __restrict__ h, size_t n, float scale) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    h[i] = roundf(tanhf(h[i]) * scale) / scale;
}

cudaError_t launch_fsq_quant(float* h, size_t n, float scale, cudaStream_t st) {
  count_launch();
  const int grid = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  fsq_quant_kernel<<<grid, 256, 0, st>>>(h, n, scale);
  return cudaGetLastError();
}

cudaError_t launch_cfg_euler(const float* out2b, float* x, int B, int n, double cfg, double dt, int zero_star,
                             cudaStream_t st) {
  count_launch();
  PdlLaunch l(dim3(B), dim3(256), 0, st);
  return cudaLaunchKernelEx(&l.cfg, cfg_euler_kernel, out2b, x, B, n, (float)cfg, (float)(1.0 - cfg), (float)dt,
                            zero_star);
}

}  // namespace vx
