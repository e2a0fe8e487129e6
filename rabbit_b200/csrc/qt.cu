// qt.cu -- matmul_qt for the per-row quantized QT kinds (kernels::matmul_qt, src/kernels.rs:1104-1132):
// int8 and int4 weights through integer dot products with int8-quantized activations (the
// reference's IDOT path, bit-exact: the dot is an exact integer and the two scale multiplies
// round like the reference's), and the float-weight int4 / int2 paths. One warp per output row
// and up to 8 tokens: the weight row streams once, in 16-byte loads, for all of them.
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

// kernels::qrow_i8 (src/kernels.rs:301-309) per activation row: s = max(amax / 127, 1e-12),
// q = round_ties_even(x * (1 / s)). One block per row.
__global__ void __launch_bounds__(256) qrow_i8_kernel(const void* __restrict__ x, int x_dtype, int i,
                                                      int8_t* __restrict__ xq, float* __restrict__ sx) {
  const int r = blockIdx.x;
  const size_t base = static_cast<size_t>(r) * i;
  float amax = 0.0f;
  for (int k = threadIdx.x; k < i; k += blockDim.x) amax = fmaxf(amax, fabsf(load_elem(x, x_dtype, base + k)));
  __shared__ float red[8];
  amax = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(amax)));  // (non-negative floats)
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0f;
    v = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(v)));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float sc = fmaxf(__fdiv_rn(red[0], 127.0f), 1e-12f);
  const float inv = __fdiv_rn(1.0f, sc);
  for (int k = threadIdx.x; k < i; k += blockDim.x)
    xq[base + k] = static_cast<int8_t>(__float2int_rn(__fmul_rn(load_elem(x, x_dtype, base + k), inv)));
  if (threadIdx.x == 0) sx[r] = sc;
}

// The nibble pair of byte b as two int8 lanes-worth: (lo - 8, hi - 8).
__device__ __forceinline__ int nib(uint32_t word, int j) { return static_cast<int>((word >> (4 * j)) & 15u) - 8; }

// y[t][o] = float(dot(w_o, xq_t)) * scale[o] * sx[t] (kernels.rs:1063-1098). W4: int4 offset-binary
// nibbles, else int8. MT tokens per warp.
template <bool W4, int MT>
__global__ void __launch_bounds__(256) idot_kernel(const void* __restrict__ w, const float* __restrict__ scale,
                                                   const int8_t* __restrict__ xq, const float* __restrict__ sx, int S,
                                                   int I, int O, float* __restrict__ y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  const int tiles_t = (S + MT - 1) / MT;
  if (warp >= O * tiles_t) return;
  const int o = warp / tiles_t, t0 = (warp % tiles_t) * MT;
  const int nt = min(MT, S - t0);
  const size_t rb = W4 ? (static_cast<size_t>(I) + 1) / 2 : static_cast<size_t>(I);
  const uint8_t* wr = static_cast<const uint8_t*>(w) + static_cast<size_t>(o) * rb;
  int acc[MT];
#pragma unroll
  for (int t = 0; t < MT; t++) acc[t] = 0;
  // vector part: 32 elements per lane step when the rows are 16-byte aligned
  const bool vec = (I % 32 == 0) && (reinterpret_cast<uintptr_t>(wr) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(xq) % 16 == 0) && (I % 16 == 0);
  int k0 = 0;
  if (vec) {
    constexpr int kStep = W4 ? 32 : 16;  // elements per lane per step (16 bytes of weights)
    for (int k = lane * kStep; k + kStep <= I; k += 32 * kStep) {
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + (W4 ? k / 2 : k));
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int t = 0; t < MT; t++) {
        if (t >= nt) break;
        const int8_t* xr = xq + static_cast<size_t>(t0 + t) * I + k;
        if (W4) {
          const uint4 xa = *reinterpret_cast<const uint4*>(xr);
          const uint4 xb = *reinterpret_cast<const uint4*>(xr + 16);
          const uint32_t xx[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
          for (int q = 0; q < 4; q++) {
            // 8 nibbles of word q = elements 8q .. 8q+7 -> two packed int8x4 words
            const uint32_t wq = ww[q];
            const int a0 = (nib(wq, 0) & 255) | ((nib(wq, 1) & 255) << 8) | ((nib(wq, 2) & 255) << 16) |
                           ((nib(wq, 3) & 255) << 24);
            const int a1 = (nib(wq, 4) & 255) | ((nib(wq, 5) & 255) << 8) | ((nib(wq, 6) & 255) << 16) |
                           ((nib(wq, 7) & 255) << 24);
            acc[t] = __dp4a(a0, static_cast<int>(xx[2 * q]), acc[t]);
            acc[t] = __dp4a(a1, static_cast<int>(xx[2 * q + 1]), acc[t]);
          }
        } else {
          const uint4 xa = *reinterpret_cast<const uint4*>(xr);
          acc[t] = __dp4a(static_cast<int>(ww[0]), static_cast<int>(xa.x), acc[t]);
          acc[t] = __dp4a(static_cast<int>(ww[1]), static_cast<int>(xa.y), acc[t]);
          acc[t] = __dp4a(static_cast<int>(ww[2]), static_cast<int>(xa.z), acc[t]);
          acc[t] = __dp4a(static_cast<int>(ww[3]), static_cast<int>(xa.w), acc[t]);
        }
      }
    }
    k0 = I;  // (I % 32 == 0: the vector loop covered every element)
  }
  for (int k = k0 + lane; k < I; k += 32) {  // element-wise (unaligned or ragged rows)
    int wv;
    if (W4) {
      const uint8_t b = wr[k >> 1];
      wv = static_cast<int>((k & 1) ? (b >> 4) : (b & 15)) - 8;
    } else {
      wv = static_cast<int8_t>(wr[k]);
    }
#pragma unroll
    for (int t = 0; t < MT; t++)
      if (t < nt) acc[t] += wv * static_cast<int>(xq[static_cast<size_t>(t0 + t) * I + k]);
  }
  const float sc = scale[o];
#pragma unroll
  for (int t = 0; t < MT; t++) {
    int v = acc[t];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
    if (lane == 0 && t < nt)
      y[static_cast<size_t>(t0 + t) * O + o] = __fmul_rn(__fmul_rn(__int2float_rn(v), sc), sx[t0 + t]);
  }
}

// Float-weight paths with a per-row scale: BITS 4 (matmul_i4, kernels.rs:167-193) or 2
// (matmul_i2, :206-224): y = (sum_k x_k * v_k) * scale[o], f32 accumulation (the reference's own
// AVX tiers reassociate too, so these agree with its scalar tier within rounding).
template <int BITS, int MT>
__global__ void __launch_bounds__(256) qt_float_kernel(const void* __restrict__ x, int x_dtype,
                                                       const uint8_t* __restrict__ w, const float* __restrict__ scale,
                                                       int S, int I, int O, float* __restrict__ y) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  const int tiles_t = (S + MT - 1) / MT;
  if (warp >= O * tiles_t) return;
  const int o = warp / tiles_t, t0 = (warp % tiles_t) * MT;
  const int nt = min(MT, S - t0);
  constexpr int per_byte = 8 / BITS;
  const size_t rb = (static_cast<size_t>(I) + per_byte - 1) / per_byte;
  const uint8_t* wr = w + static_cast<size_t>(o) * rb;
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; t++) acc[t] = 0.0f;
  for (int k = lane; k < I; k += 32) {
    const uint8_t b = wr[k / per_byte];
    const int sh = (k % per_byte) * BITS;
    const float wv = static_cast<float>(static_cast<int>((b >> sh) & ((1 << BITS) - 1)) - (1 << (BITS - 1)));
#pragma unroll
    for (int t = 0; t < MT; t++)
      if (t < nt) acc[t] = fmaf(load_elem(x, x_dtype, static_cast<size_t>(t0 + t) * I + k), wv, acc[t]);
  }
  const float sc = scale[o];
#pragma unroll
  for (int t = 0; t < MT; t++) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
    if (lane == 0 && t < nt) y[static_cast<size_t>(t0 + t) * O + o] = v * sc;
  }
}

size_t matmul_idot_workspace_bytes(int s, int i) {
  return static_cast<size_t>(s) * i + static_cast<size_t>(s) * sizeof(float) + 256;
}

static int warps_grid(long long warps) {
  const long long blocks = (warps + 7) / 8;
  return static_cast<int>(blocks > 0 ? blocks : 1);
}

cudaError_t launch_matmul_idot(float* y, const void* x, int x_dtype, const void* w, bool w4, const float* scale, int s,
                               int i, int o, void* workspace, cudaStream_t st) {
  if (s <= 0 || o <= 0) return cudaSuccess;
  int8_t* xq = static_cast<int8_t*>(workspace);
  float* sx = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(xq + static_cast<size_t>(s) * i) + 15) & ~uintptr_t(15));
  qrow_i8_kernel<<<s, 256, 0, st>>>(x, x_dtype, i, xq, sx);
  const long long warps = static_cast<long long>(o) * ((s + 7) / 8);
  if (w4) idot_kernel<true, 8><<<warps_grid(warps), 256, 0, st>>>(w, scale, xq, sx, s, i, o, y);
  else idot_kernel<false, 8><<<warps_grid(warps), 256, 0, st>>>(w, scale, xq, sx, s, i, o, y);
  return cudaGetLastError();
}

cudaError_t launch_matmul_qt_float(float* y, const void* x, int x_dtype, const uint8_t* w, int bits, const float* scale,
                                   int s, int i, int o, cudaStream_t st) {
  if (s <= 0 || o <= 0) return cudaSuccess;
  const long long warps = static_cast<long long>(o) * ((s + 7) / 8);
  if (bits == 4) qt_float_kernel<4, 8><<<warps_grid(warps), 256, 0, st>>>(x, x_dtype, w, scale, s, i, o, y);
  else qt_float_kernel<2, 8><<<warps_grid(warps), 256, 0, st>>>(x, x_dtype, w, scale, s, i, o, y);
  return cudaGetLastError();
}

}  // namespace rmoe
