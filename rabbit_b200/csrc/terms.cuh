// terms.cuh -- the four-term E2M1 expansion of activations, one warp per 32-element block.
//
// For a block of 32 values (one per lane): term 0 is the value rounded to the nearest E2M1 grid
// point (0, .5, 1, 1.5, 2, 3, 4, 6) under the smallest power-of-two scale 2^e with
// max |v| / 2^e <= 6; term j + 1 is the same rounding of what term j left over. The scale is the
// E8M0 byte e + 127. Every term removes at least log2(6) bits of the block's range, so four terms
// keep about 11 significant bits; the products with E2M1 weights are exact in the tensor core.
#pragma once

#include "common.cuh"

namespace rmoe {

__device__ __forceinline__ int e2m1_nearest(float v) {  // 0 <= v <= 6
  return v < 0.25f ? 0 : v < 0.75f ? 1 : v < 1.25f ? 2 : v < 1.75f ? 3 : v < 2.5f ? 4 : v < 3.5f ? 5 : v < 5.0f ? 6 : 7;
}
__device__ __forceinline__ float e2m1_magnitude(int c) {
  return c < 4 ? 0.5f * c : static_cast<float>(2 << ((c - 4) >> 1)) * (1.0f + 0.5f * (c & 1));
}

// Smallest e with amax <= 6 * 2^e (amax > 0), clamped to the normal range.
__device__ __forceinline__ int e2m1_block_exponent(float amax) {
  const int e0 = ilogbf(amax);  // amax in [2^e0, 2^(e0+1))
  const int e = amax <= 6.0f * exp2i(max(e0 - 2, -149)) ? e0 - 2 : e0 - 1;
  return max(-126, min(127, e));
}

// Lane l holds element l of a 32-block. Writes term j's 16 E2M1 bytes to rows + j * pitch and its
// scale byte to sf + j * sf_pitch (lane 0 stores). All 32 lanes must call.
__device__ __forceinline__ void warp_terms4(float r, uint8_t* rows, size_t pitch, uint8_t* sf, size_t sf_pitch) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int j = 0; j < 4; j++) {
    const float amax = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(fabsf(r))));
    int e = 0;
    uint32_t nib = 0;
    if (amax > 0.0f) {
      e = e2m1_block_exponent(amax);
      const bool neg = r < 0.0f;
      const int c = e2m1_nearest(fminf(fabsf(r) * exp2i(-e), 6.0f));
      const float q = e2m1_magnitude(c) * exp2i(e);
      r = neg ? r + q : r - q;
      nib = static_cast<uint32_t>(c) | (neg && c ? 8u : 0u);
    }
    const uint32_t sh = nib << (4 * (lane & 7));
    uint32_t w[4];
#pragma unroll
    for (int g = 0; g < 4; g++) w[g] = __reduce_or_sync(kFull, (lane >> 3) == g ? sh : 0u);
    if (lane == 0) {
      *reinterpret_cast<uint4*>(rows + j * pitch) = make_uint4(w[0], w[1], w[2], w[3]);
      sf[j * sf_pitch] = static_cast<uint8_t>(amax > 0.0f ? e + 127 : 127);
    }
  }
}

// One thread, one 32-block held in registers: the same four-term expansion as warp_terms4,
// serially over the 32 values; writes term j's 16 bytes to rows + j * pitch and its scale byte
// to sf + j * sf_pitch.
__device__ __forceinline__ void thread_terms4(float (&r)[32], uint8_t* rows, size_t pitch, uint8_t* sf,
                                              size_t sf_pitch) {
#pragma unroll 1
  for (int j = 0; j < 4; j++) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(r[i]));
    uint32_t w[4] = {0, 0, 0, 0};
    int e = 0;
    if (amax > 0.0f) {
      e = e2m1_block_exponent(amax);
      const float inv = exp2i(-e), sc = exp2i(e);
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const bool neg = r[i] < 0.0f;
        const int c = e2m1_nearest(fminf(fabsf(r[i]) * inv, 6.0f));
        const float q = e2m1_magnitude(c) * sc;
        r[i] = neg ? r[i] + q : r[i] - q;
        w[i / 8] |= (static_cast<uint32_t>(c) | (neg && c ? 8u : 0u)) << (4 * (i % 8));
      }
    }
    *reinterpret_cast<uint4*>(rows + j * pitch) = make_uint4(w[0], w[1], w[2], w[3]);
    sf[j * sf_pitch] = static_cast<uint8_t>(amax > 0.0f ? e + 127 : 127);
  }
}

}  // namespace rmoe
