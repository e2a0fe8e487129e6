// latent.cu -- the two projections and the norm of Kimi K3's latent MoE wrapper
// (kimi_k3::moe::latent_moe, src/kimi_k3/moe.rs:64-116): x_latent = x . down^T before the routed
// experts, RMSNorm of each token's summed routed row (kimi_linear::ops::rmsnorm,
// src/kimi_linear/ops.rs:46-53), out = y . up^T after them.
//
// The projections are memory-bound matrix-vector products for decode-sized T: one warp per
// output row streams that row of W once (16-byte loads) and multiplies it against up to eight
// tokens at a time (x stays in L1/L2; larger T take several passes over W).
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

namespace {

template <int WD>
__device__ __forceinline__ void load_w8(const void* w, size_t i, float (&v)[8]) {
  if (WD == kBF16) {
    const uint4 r = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(w) + i);
    const uint32_t q[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[2 * j] = __uint_as_float(q[j] << 16);
      v[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(w) + i);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(w) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

constexpr int kProjTok = 8;  // tokens per pass over W

// y[t][n] = sum_k x[t][k] w[n][k] for tokens t0 .. t0 + nt - 1 (nt <= kProjTok); K % 8 == 0.
template <int WD, int XD>
__global__ void __launch_bounds__(256) latent_proj_kernel(const void* __restrict__ w, const void* __restrict__ x,
                                                          int T, int K, int N, float* __restrict__ y) {
  const int lane = threadIdx.x % 32;
  const int warps = gridDim.x * (blockDim.x / 32);
  for (int n = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; n < N; n += warps) {
    for (int t0 = 0; t0 < T; t0 += kProjTok) {
      const int nt = min(kProjTok, T - t0);
      float acc[kProjTok];
#pragma unroll
      for (int t = 0; t < kProjTok; t++) acc[t] = 0.0f;
      for (int k0 = lane * 8; k0 < K; k0 += 4 * 256) {
        float wv[4][8];  // four 16-byte weight loads in flight per lane
#pragma unroll
        for (int u = 0; u < 4; u++)
          if (k0 + u * 256 < K) load_w8<WD>(w, static_cast<size_t>(n) * K + k0 + u * 256, wv[u]);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int k = k0 + u * 256;
          if (k >= K) break;
#pragma unroll
          for (int t = 0; t < kProjTok; t++) {
            if (t >= nt) break;
            float xv[8];
            load_w8<XD>(x, static_cast<size_t>(t0 + t) * K + k, xv);
#pragma unroll
            for (int j = 0; j < 8; j++) acc[t] = fmaf(xv[j], wv[u][j], acc[t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kProjTok; t++) {
        if (t >= nt) break;
        const float s = warp_sum(acc[t]);
        if (lane == 0) y[static_cast<size_t>(t0 + t) * N + n] = s;
      }
    }
  }
}

// In place, one 1024-thread block per row: v *= r * w with r = 1 / sqrt(mean(v^2) + eps), the
// mean of squares accumulated in f64 as the reference does. The row is read once into registers
// (up to kNormPer values per thread, loads issued together).
constexpr int kNormPer = 8;
__global__ void __launch_bounds__(1024) rmsnorm_rows_kernel(float* __restrict__ v, int n, const float* __restrict__ w,
                                                            float eps) {
  __shared__ double part[32];
  float* row = v + static_cast<size_t>(blockIdx.x) * n;
  float a[kNormPer];
#pragma unroll
  for (int j = 0; j < kNormPer; j++) {
    const int i = threadIdx.x + j * blockDim.x;
    a[j] = i < n ? row[i] : 0.0f;
  }
  double s = 0.0;
#pragma unroll
  for (int j = 0; j < kNormPer; j++) s += static_cast<double>(a[j]) * static_cast<double>(a[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = s;
  __syncthreads();
  double tot = 0.0;
  for (int i = 0; i < static_cast<int>(blockDim.x / 32); i++) tot += part[i];
  const float ms = static_cast<float>(tot / static_cast<double>(n));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
#pragma unroll
  for (int j = 0; j < kNormPer; j++) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < n) row[i] = a[j] * __fmul_rn(r, w[i]);
  }
}

}  // namespace

cudaError_t launch_latent_proj(const void* w, int w_dtype, const void* x, int x_dtype, int T, int K, int N, float* y,
                               cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (K % 8) return cudaErrorInvalidValue;
  const int blocks = (N + 7) / 8;
  if (w_dtype == kBF16 && x_dtype == kBF16) latent_proj_kernel<kBF16, kBF16><<<blocks, 256, 0, st>>>(w, x, T, K, N, y);
  else if (w_dtype == kBF16) latent_proj_kernel<kBF16, kF32><<<blocks, 256, 0, st>>>(w, x, T, K, N, y);
  else if (x_dtype == kBF16) latent_proj_kernel<kF32, kBF16><<<blocks, 256, 0, st>>>(w, x, T, K, N, y);
  else latent_proj_kernel<kF32, kF32><<<blocks, 256, 0, st>>>(w, x, T, K, N, y);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(float* v, int rows, int n, const float* w, float eps, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (n > 1024 * kNormPer) return cudaErrorInvalidValue;
  rmsnorm_rows_kernel<<<rows, 1024, 0, st>>>(v, n, w, eps);
  return cudaGetLastError();
}

}  // namespace rmoe
