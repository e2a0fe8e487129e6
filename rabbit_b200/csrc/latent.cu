// latent.cu -- the two projections and the norm of Kimi K3's latent MoE wrapper
// (kimi_k3::moe::latent_moe, src/kimi_k3/moe.rs:64-116): x_latent = x . down^T before the routed
// experts, RMSNorm of each token's summed routed row (kimi_linear::ops::rmsnorm,
// src/kimi_linear/ops.rs:46-53), out = y . up^T after them.
//
// The projections are memory-bound matrix-vector products for decode-sized T: one warp per
// output row streams that row of W once (16-byte loads, eight in flight per lane) against the
// tokens of x staged in shared memory, eight tokens per pass (larger T: several passes over W).
// The norm runs inside the up projection, on each block's staged copy of the rows.
#include <algorithm>

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

constexpr int kProjTok = 8;        // tokens per pass over W
constexpr int kProjWarps = 16;     // output rows per block
constexpr int kProjSmem = 96 * 1024;
constexpr int kProjLoads = 8;      // 16-byte weight loads in flight per lane

// y[t][n] = sum_k x'[t][k] w[n][k]; K % 8 == 0. Each block stages up to `tg` tokens of x in
// shared memory (f32) and its 16 warps each stream one row of W against them. With `norm`
// set, x' is each token's row RMS-normalized on the way in (x * (r * norm[k]),
// r = 1 / sqrt(mean(x^2) + eps), the mean of squares accumulated in f64): every block normalizes
// its staged copy itself, so the norm needs no launch of its own.
template <int WD, int XD>
__global__ void __launch_bounds__(32 * kProjWarps) latent_proj_kernel(const void* __restrict__ w,
                                                                      const void* __restrict__ x, int T, int K, int N,
                                                                      int tg, const float* __restrict__ norm, float eps,
                                                                      float* __restrict__ y) {
  extern __shared__ __align__(16) float px[];  // [tg][K]
  __shared__ double red[kProjWarps];
  const int lane = threadIdx.x % 32, wi = threadIdx.x / 32;
  for (int n0 = blockIdx.x * kProjWarps; n0 < N; n0 += gridDim.x * kProjWarps) {
    const int n = n0 + wi;
    for (int t0 = 0; t0 < T; t0 += tg) {
      const int nt = min(tg, T - t0);
      __syncthreads();  // (the previous group's reads are done)
      for (int i = threadIdx.x * 8; i < nt * K; i += blockDim.x * 8) {
        float v[8];
        load_w8<XD>(x, static_cast<size_t>(t0) * K + i, v);
#pragma unroll
        for (int j = 0; j < 8; j++) px[i + j] = v[j];
      }
      __syncthreads();
      if (norm) {
        for (int t = 0; t < nt; t++) {
          float* row = px + static_cast<size_t>(t) * K;
          double ss = 0.0;
          for (int i = threadIdx.x; i < K; i += blockDim.x) ss += static_cast<double>(row[i]) * row[i];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
          if (lane == 0) red[wi] = ss;
          __syncthreads();
          double tot = 0.0;
          for (int q = 0; q < kProjWarps; q++) tot += red[q];
          const float ms = static_cast<float>(tot / static_cast<double>(K));
          const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
          __syncthreads();  // (red is read by every thread before the next token's sums)
          for (int i = threadIdx.x; i < K; i += blockDim.x) row[i] = row[i] * __fmul_rn(r, norm[i]);
        }
        __syncthreads();
      }
      if (n >= N) continue;
      for (int ts = 0; ts < nt; ts += kProjTok) {
        const int ns = min(kProjTok, nt - ts);
        float acc[kProjTok];
#pragma unroll
        for (int t = 0; t < kProjTok; t++) acc[t] = 0.0f;
        for (int k0 = lane * 8; k0 < K; k0 += kProjLoads * 256) {
          float wv[kProjLoads][8];  // kProjLoads 16-byte weight loads in flight per lane
#pragma unroll
          for (int u = 0; u < kProjLoads; u++)
            if (k0 + u * 256 < K) load_w8<WD>(w, static_cast<size_t>(n) * K + k0 + u * 256, wv[u]);
#pragma unroll
          for (int u = 0; u < kProjLoads; u++) {
            const int k = k0 + u * 256;
            if (k >= K) break;
#pragma unroll
            for (int t = 0; t < kProjTok; t++) {
              if (t >= ns) break;
              const float* xr = px + static_cast<size_t>(ts + t) * K + k;
              const float4 a = *reinterpret_cast<const float4*>(xr);
              const float4 b = *reinterpret_cast<const float4*>(xr + 4);
              const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
              for (int j = 0; j < 8; j++) acc[t] = fmaf(xv[j], wv[u][j], acc[t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < kProjTok; t++) {
          if (t >= ns) break;
          const float sum = warp_sum(acc[t]);
          if (lane == 0) y[static_cast<size_t>(t0 + ts + t) * N + n] = sum;
        }
      }
    }
  }
}

}  // namespace

cudaError_t launch_latent_proj(const void* w, int w_dtype, const void* x, int x_dtype, int T, int K, int N, float* y,
                               cudaStream_t st, const float* norm, float eps) {
  if (T <= 0) return cudaSuccess;
  if (K % 8 || static_cast<size_t>(K) * 4 > kProjSmem) return cudaErrorInvalidValue;
  const int tg = std::min(T, static_cast<int>(kProjSmem / (static_cast<size_t>(K) * 4)));
  const size_t smem = static_cast<size_t>(tg) * K * 4;
  void (*kern)(const void*, const void*, int, int, int, int, const float*, float, float*) =
      w_dtype == kBF16 ? (x_dtype == kBF16 ? latent_proj_kernel<kBF16, kBF16> : latent_proj_kernel<kBF16, kF32>)
                       : (x_dtype == kBF16 ? latent_proj_kernel<kF32, kBF16> : latent_proj_kernel<kF32, kF32>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int blocks = std::min((N + kProjWarps - 1) / kProjWarps, 148 * 4);
  kern<<<blocks, 32 * kProjWarps, smem, st>>>(w, x, T, K, N, tg, norm, eps, y);
  return cudaGetLastError();
}

}  // namespace rmoe
