// Few-row GEMM on CUDA cores: Y[M,N] = X[M,K] . W[N,K]^T (+ bias) (optionally
// Y = R + s * (...)), bf16 weights, f32 activations and accumulation.
//
// Used for the prefill / DiT / LocEnc linears where M (tokens) is small but > 1.
// CTA tile: 64 weight rows x 32 tokens, K streamed in steps of 64 through shared memory
// (weights upcast to f32 on the way in).  Each thread owns 4 rows x 2 tokens.
#include "common.cuh"
#include "kernels.cuh"

namespace vx {



__global__ void __launch_bounds__(256) gemm_smallm_kernel(const GemmArgs a) {
  __shared__ __align__(16) float Ws[64][64 + 4];
  __shared__ __align__(16) float Xs[64][32 + 4];
  pdl_wait();
  pdl_launch_dependents();
  const int t = threadIdx.x;
  const int n0 = blockIdx.x * 64, m0 = blockIdx.y * 32;
  const int rr = t & 15, tt = t >> 4;  // rows rr*4..+4, tokens tt*2..+2
  float acc[4][2] = {};
  for (int k0 = 0; k0 < a.K; k0 += 64) {
    // W tile: 64 rows x 64 k  (512 chunks of 8 bf16)
    for (int c = t; c < 512; c += 256) {
      const int row = c >> 3, kk = (c & 7) * 8;
      uint4 w = make_uint4(0, 0, 0, 0);
      if (n0 + row < a.N) w = __ldg(reinterpret_cast<const uint4*>(a.W + (size_t)(n0 + row) * a.K + k0 + kk));
      Ws[kk + 0][row] = bf16lo(w.x); Ws[kk + 1][row] = bf16hi(w.x);
      Ws[kk + 2][row] = bf16lo(w.y); Ws[kk + 3][row] = bf16hi(w.y);
      Ws[kk + 4][row] = bf16lo(w.z); Ws[kk + 5][row] = bf16hi(w.z);
      Ws[kk + 6][row] = bf16lo(w.w); Ws[kk + 7][row] = bf16hi(w.w);
    }
    // X tile: 32 tokens x 64 k (512 float4)
    for (int c = t; c < 512; c += 256) {
      const int tok = c >> 4, kk = (c & 15) * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + tok < a.M) x = *reinterpret_cast<const float4*>(a.X + (size_t)(m0 + tok) * a.ldx + k0 + kk);
      Xs[kk + 0][tok] = x.x; Xs[kk + 1][tok] = x.y; Xs[kk + 2][tok] = x.z; Xs[kk + 3][tok] = x.w;
    }
    __syncthreads();
#pragma unroll 16
    for (int k = 0; k < 64; ++k) {
      const float4 w4 = *reinterpret_cast<const float4*>(&Ws[k][rr * 4]);
      const float2 x2 = *reinterpret_cast<const float2*>(&Xs[k][tt * 2]);
      acc[0][0] = fmaf(w4.x, x2.x, acc[0][0]); acc[0][1] = fmaf(w4.x, x2.y, acc[0][1]);
      acc[1][0] = fmaf(w4.y, x2.x, acc[1][0]); acc[1][1] = fmaf(w4.y, x2.y, acc[1][1]);
      acc[2][0] = fmaf(w4.z, x2.x, acc[2][0]); acc[2][1] = fmaf(w4.z, x2.y, acc[2][1]);
      acc[3][0] = fmaf(w4.w, x2.x, acc[3][0]); acc[3][1] = fmaf(w4.w, x2.y, acc[3][1]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = n0 + rr * 4 + i;
    if (n >= a.N) continue;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int m = m0 + tt * 2 + j;
      if (m >= a.M) continue;
      float v = acc[i][j];
      if (a.bias) v += a.bias[n];
      if (a.R) v = a.R[(size_t)m * a.ldy + n] + v * a.res_scale;
      a.Y[(size_t)m * a.ldy + n] = v;
    }
  }
}

cudaError_t launch_gemm_smallm(const GemmArgs& a, cudaStream_t st) {
  if (a.K % 64 != 0 || a.M <= 0 || a.N <= 0) return cudaErrorInvalidValue;
  dim3 grid((a.N + 63) / 64, (a.M + 31) / 32);
  count_launch();
  gemm_smallm_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace vx
