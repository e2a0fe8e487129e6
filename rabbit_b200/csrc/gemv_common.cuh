// gemv_common.cuh -- the per-block dequantize-and-dot machinery shared by the GEMV kernels.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace rmoe {

// Scale of block b (32 elements) of one weight row.
template <int FMT>
__device__ __forceinline__ float block_scale(const void* srow, int b, const ExpertFormat& f) {
  if (FMT == kMxfp4) return e8m0_to_f32(__ldg(static_cast<const uint8_t*>(srow) + b));
  const int g = (b * 32) / f.group_size;
  if (f.scale_dtype == kBF16) return bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(srow) + g));
  return __ldg(static_cast<const float*>(srow) + g);
}

// Same, for a scale row staged in shared memory.
template <int FMT>
__device__ __forceinline__ float block_scale_smem(const void* srow, int b, const ExpertFormat& f) {
  if (FMT == kMxfp4) return e8m0_to_f32(static_cast<const uint8_t*>(srow)[b]);
  const int g = (b * 32) / f.group_size;
  if (f.scale_dtype == kBF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(srow)[g]);
  return static_cast<const float*>(srow)[g];
}

template <int FMT>
__device__ __forceinline__ void decode_block(const uint4& w, uint32_t (&h)[16]) {
  uint32_t t[4];
  if (FMT == kMxfp4) {
    e2m1x8_to_h2(w.x, t); h[0] = t[0]; h[1] = t[1]; h[2] = t[2]; h[3] = t[3];
    e2m1x8_to_h2(w.y, t); h[4] = t[0]; h[5] = t[1]; h[6] = t[2]; h[7] = t[3];
    e2m1x8_to_h2(w.z, t); h[8] = t[0]; h[9] = t[1]; h[10] = t[2]; h[11] = t[3];
    e2m1x8_to_h2(w.w, t); h[12] = t[0]; h[13] = t[1]; h[14] = t[2]; h[15] = t[3];
  } else {
    i4x8_to_h2(w.x, t); h[0] = t[0]; h[1] = t[1]; h[2] = t[2]; h[3] = t[3];
    i4x8_to_h2(w.y, t); h[4] = t[0]; h[5] = t[1]; h[6] = t[2]; h[7] = t[3];
    i4x8_to_h2(w.z, t); h[8] = t[0]; h[9] = t[1]; h[10] = t[2]; h[11] = t[3];
    i4x8_to_h2(w.w, t); h[12] = t[0]; h[13] = t[1]; h[14] = t[2]; h[15] = t[3];
  }
}

// acc[r][m] += sum over this lane's blocks of row r . x_m. NR weight rows (pointers `rows`,
// scale rows `srows`, K elements each) against up to MT activation rows `xr[m]` (f16, K).
template <int FMT, int NR, int MT>
__device__ __forceinline__ void gemv_accumulate(const uint8_t* const (&rows)[NR],
                                                const void* const (&srows)[NR],
                                                const uint16_t* const (&xr)[MT], int n, int K,
                                                const ExpertFormat& f, float (&acc)[NR][MT]) {
  const int lane = threadIdx.x % 32;
  const int nblk = K / 32;
  for (int b = lane; b < nblk; b += 32) {
    uint4 w[NR];
    float sc[NR];
#pragma unroll
    for (int r = 0; r < NR; r++) w[r] = ldg_stream(rows[r] + static_cast<size_t>(b) * 16);
#pragma unroll
    for (int r = 0; r < NR; r++) sc[r] = block_scale<FMT>(srows[r], b, f);
    uint32_t hw[NR][16];
#pragma unroll
    for (int r = 0; r < NR; r++) decode_block<FMT>(w[r], hw[r]);
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m >= n) break;
      const uint4* xp = reinterpret_cast<const uint4*>(xr[m] + static_cast<size_t>(b) * 32);
      uint32_t xv[16];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        uint4 v = __ldg(xp + q);
        xv[4 * q] = v.x; xv[4 * q + 1] = v.y; xv[4 * q + 2] = v.z; xv[4 * q + 3] = v.w;
      }
#pragma unroll
      for (int r = 0; r < NR; r++) {
        uint32_t a0 = 0, a1 = 0;
#pragma unroll
        for (int q = 0; q < 16; q += 2) {
          a0 = hfma2u(hw[r][q], xv[q], a0);
          a1 = hfma2u(hw[r][q + 1], xv[q + 1], a1);
        }
        acc[r][m] = fmaf(h2sum_f32(a0) + h2sum_f32(a1), sc[r], acc[r][m]);
      }
    }
  }
}

template <int NR, int MT>
__device__ __forceinline__ void warp_reduce_all(float (&acc)[NR][MT]) {
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) acc[r][m] = warp_sum(acc[r][m]);
}

__device__ __forceinline__ int find_chunk(const int32_t* __restrict__ task0, int n_chunks, int task) {
  int lo = 0, hi = n_chunks - 1;  // largest c with task0[c] <= task
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(task0 + mid) <= task) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ ExpertPtrs expert_ptrs(const ExpertTable& tab, int slot) {
  if (slot >= tab.n_local) return tab.shared;
  const uint8_t* b = tab.base + static_cast<size_t>(slot) * tab.stride;
  ExpertPtrs p;
  p.gate = b;
  p.up = b + tab.off_up;
  p.down = b + tab.off_down;
  p.gate_scale = b + tab.off_gs;
  p.up_scale = b + tab.off_us;
  p.down_scale = b + tab.off_ds;
  return p;
}

__host__ __device__ __forceinline__ size_t scale_row_bytes(const ExpertFormat& f, int K) {
  if (f.fmt == kMxfp4) return static_cast<size_t>(K) / 32;
  return static_cast<size_t>(K / f.group_size) * (f.scale_dtype == kBF16 ? 2 : 4);
}


}  // namespace rmoe

namespace rmoe {
inline size_t scale_row_bytes_host(const ExpertFormat& f, int K) { return scale_row_bytes(f, K); }
}  // namespace rmoe
