// latent.cu -- the two projections and the norm of Kimi K3's latent MoE wrapper
// (kimi_k3::moe::latent_moe, src/kimi_k3/moe.rs:64-116): x_latent = x . down^T before the routed
// experts, RMSNorm of each token's summed routed row (kimi_linear::ops::rmsnorm,
// src/kimi_linear/ops.rs:46-53), out = y . up^T after them.
//
// The projections are memory-bound matrix-vector products for decode-sized T: one warp per
// output row streams that row of W once (16-byte streaming loads, all of a 4096-element pass in
// flight per lane) against the tokens of x staged in shared memory, eight tokens per pass
// (larger T: several passes over W).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "pipe.cuh"

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
constexpr int kProjWarps = 8;      // output rows per block
constexpr int kProjLoads = 16;     // 16-byte weight loads in flight per lane
constexpr int kProjSmem = 96 * 1024;

// y[t][n] = sum_k x[t][k] w[n][k]; K % 8 == 0. Each block stages up to `tg` tokens of x in
// shared memory (f32) and its 16 warps each stream one row of W against them.
template <int WD, int XD, int TOK>
__global__ void __launch_bounds__(32 * kProjWarps) latent_proj_kernel(const void* __restrict__ w,
                                                                      const void* __restrict__ x, int T, int K, int N,
                                                                      int tg, float* __restrict__ y,
                                                                      const float* __restrict__ norm_w, float eps) {
  extern __shared__ __align__(16) float px[];  // [tg][K]
  const int lane = threadIdx.x % 32, wi = threadIdx.x / 32;
  // (launched as a programmatic dependent of the kernel that writes x: wait for it here)
  griddep_wait();
  // all tokens fit in one group: x is staged once and the block walks its rows
  const bool once = T <= tg;
  if (once && norm_w) {
    // RMSNorm of each row while it is staged (kimi_linear::ops::rmsnorm,
    // src/kimi_linear/ops.rs:46-53): the row's values and the norm weights are loaded together,
    // the mean of squares accumulated in f64, and px = v * (r * w) -- rmsnorm_rows_kernel's
    // arithmetic, done by every block on its own copy of the rows
    constexpr int kMaxC = 4;  // 8-element pieces per thread (K <= 8192)
    __shared__ double part[kProjWarps];
    for (int t = 0; t < T; t++) {
      float v[kMaxC][8], nw[kMaxC][8];
      double sq = 0.0;
#pragma unroll
      for (int c = 0; c < kMaxC; c++) {
        const int i = (threadIdx.x + c * blockDim.x) * 8;
        if (i < K) {
          load_w8<XD>(x, static_cast<size_t>(t) * K + i, v[c]);
          load_w8<kF32>(norm_w, i, nw[c]);
#pragma unroll
          for (int j = 0; j < 8; j++) sq += static_cast<double>(v[c][j]) * static_cast<double>(v[c][j]);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(kFull, sq, o);
      if (lane == 0) part[wi] = sq;
      __syncthreads();
      double tot = 0.0;
      for (int q = 0; q < kProjWarps; q++) tot += part[q];
      const float ms = static_cast<float>(tot / static_cast<double>(K));
      const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
#pragma unroll
      for (int c = 0; c < kMaxC; c++) {
        const int i = (threadIdx.x + c * blockDim.x) * 8;
        if (i < K)
#pragma unroll
          for (int j = 0; j < 8; j++) px[static_cast<size_t>(t) * K + i + j] = v[c][j] * __fmul_rn(r, nw[c][j]);
      }
      __syncthreads();  // (the partials are read before the next row reuses them; px complete)
    }
  } else if (once) {
    for (int i = threadIdx.x * 8; i < T * K; i += blockDim.x * 8) {
      float v[8];
      load_w8<XD>(x, i, v);
#pragma unroll
      for (int j = 0; j < 8; j++) px[i + j] = v[j];
    }
    __syncthreads();
  }
  for (int n0 = blockIdx.x * kProjWarps; n0 < N; n0 += gridDim.x * kProjWarps) {
    const int n = n0 + wi;
    for (int t0 = 0; t0 < T; t0 += tg) {
      const int nt = min(tg, T - t0);
      if (!once) {
        __syncthreads();  // (the previous group's reads are done)
        for (int i = threadIdx.x * 8; i < nt * K; i += blockDim.x * 8) {
          float v[8];
          load_w8<XD>(x, static_cast<size_t>(t0) * K + i, v);
#pragma unroll
          for (int j = 0; j < 8; j++) px[i + j] = v[j];
        }
        __syncthreads();
      }
      if (n >= N) continue;
      for (int ts = 0; ts < nt; ts += TOK) {
        const int ns = min(TOK, nt - ts);
        float acc[TOK];
#pragma unroll
        for (int t = 0; t < TOK; t++) acc[t] = 0.0f;
        for (int k0 = lane * 8; k0 < K; k0 += kProjLoads * 256) {
          // every 16-byte weight load of this pass in flight at once (a 7 KB bf16 row: one pass),
          // converted when used
          uint4 raw[kProjLoads][WD == kBF16 ? 1 : 2];
#pragma unroll
          for (int u = 0; u < kProjLoads; u++)
            if (k0 + u * 256 < K) {
              const size_t i = static_cast<size_t>(n) * K + k0 + u * 256;
              if (WD == kBF16) {
                raw[u][0] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(w) + i));
              } else {
                raw[u][0] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const float*>(w) + i));
                raw[u][WD == kBF16 ? 0 : 1] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const float*>(w) + i + 4));
              }
            }
#pragma unroll
          for (int u = 0; u < kProjLoads; u++) {
            const int k = k0 + u * 256;
            if (k >= K) break;
            float wv[8];
            if (WD == kBF16) {
              const uint32_t q[4] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w};
#pragma unroll
              for (int j = 0; j < 4; j++) {
                wv[2 * j] = __uint_as_float(q[j] << 16);
                wv[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
              }
            } else {
              const uint4 a = raw[u][0], b = raw[u][WD == kBF16 ? 0 : 1];
              wv[0] = __uint_as_float(a.x); wv[1] = __uint_as_float(a.y); wv[2] = __uint_as_float(a.z); wv[3] = __uint_as_float(a.w);
              wv[4] = __uint_as_float(b.x); wv[5] = __uint_as_float(b.y); wv[6] = __uint_as_float(b.z); wv[7] = __uint_as_float(b.w);
            }
#pragma unroll
            for (int t = 0; t < TOK; t++) {
              if (t >= ns) break;
              const float* xr = px + static_cast<size_t>(ts + t) * K + k;
              const float4 a = *reinterpret_cast<const float4*>(xr);
              const float4 b = *reinterpret_cast<const float4*>(xr + 4);
              const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
              for (int j = 0; j < 8; j++) acc[t] = fmaf(xv[j], wv[j], acc[t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < TOK; t++) {
          if (t >= ns) break;
          const float sum = warp_sum(acc[t]);
          if (lane == 0) y[static_cast<size_t>(t0 + ts + t) * N + n] = sum;
        }
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
                               cudaStream_t st, const float* norm_w, float eps) {
  if (T <= 0) return cudaSuccess;
  if (K % 8 || static_cast<size_t>(K) * 4 > kProjSmem) return cudaErrorInvalidValue;
  const int tg = std::min(T, static_cast<int>(kProjSmem / (static_cast<size_t>(K) * 4)));
  if (norm_w && (tg < T || K > 8192)) return cudaErrorInvalidValue;  // (the norm stages every row at once)
  const size_t smem = static_cast<size_t>(tg) * K * 4;
  // (one token: a one-token instance, whose fewer registers let two blocks share an SM)
  void (*kern)(const void*, const void*, int, int, int, int, float*, const float*, float) =
      T == 1 ? (w_dtype == kBF16 ? (x_dtype == kBF16 ? latent_proj_kernel<kBF16, kBF16, 1> : latent_proj_kernel<kBF16, kF32, 1>)
                                 : (x_dtype == kBF16 ? latent_proj_kernel<kF32, kBF16, 1> : latent_proj_kernel<kF32, kF32, 1>))
             : (w_dtype == kBF16 ? (x_dtype == kBF16 ? latent_proj_kernel<kBF16, kBF16, kProjTok> : latent_proj_kernel<kBF16, kF32, kProjTok>)
                                 : (x_dtype == kBF16 ? latent_proj_kernel<kF32, kBF16, kProjTok> : latent_proj_kernel<kF32, kF32, kProjTok>));
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  // one group of tokens: two resident blocks per SM walk the rows (x staged once per block);
  // more tokens: a block per row group, x staged per group
  const int blocks = std::min((N + kProjWarps - 1) / kProjWarps, device_sm_count() * (T <= tg ? 2 : 8));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(32 * kProjWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, w, x, T, K, N, tg, y, norm_w, eps);
}

bool latent_proj_one_group(int T, int K) {
  return T >= 1 && static_cast<size_t>(T) * K * 4 <= kProjSmem && K <= 8192 && K % 8 == 0;
}

cudaError_t launch_rmsnorm_rows(float* v, int rows, int n, const float* w, float eps, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (n > 1024 * kNormPer) return cudaErrorInvalidValue;
  rmsnorm_rows_kernel<<<rows, 1024, 0, st>>>(v, n, w, eps);
  return cudaGetLastError();
}

}  // namespace rmoe
