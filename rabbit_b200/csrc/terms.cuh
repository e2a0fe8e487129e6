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

// Branch-free (lanes of a warp take different codes): code = number of rounding boundaries at or
// below v, i.e. ties round up.
__device__ __forceinline__ int e2m1_nearest(float v) {  // 0 <= v <= 6
  return (v >= 0.25f) + (v >= 0.75f) + (v >= 1.25f) + (v >= 1.75f) + (v >= 2.5f) + (v >= 3.5f) + (v >= 5.0f);
}
// |value| of code c: 0, .5, 1, 1.5, 2, 3, 4, 6 (c >= 2: 2^((c >> 1) - 1) * (1 + (c & 1) / 2)).
__device__ __forceinline__ float e2m1_magnitude(int c) {
  const uint32_t hi = (static_cast<uint32_t>((c >> 1) + 126) << 23) | (static_cast<uint32_t>(c & 1) << 22);
  return __uint_as_float(c >= 2 ? hi : (c ? 0x3F000000u : 0u));
}

// Smallest e with amax <= 6 * 2^e (amax > 0), clamped to the normal range. For a normal amax =
// 2^e0 * (1 + f): amax <= 6 * 2^(e0 - 2) = 1.5 * 2^e0 iff f <= 1/2.
__device__ __forceinline__ int e2m1_block_exponent(float amax) {
  const uint32_t b = __float_as_uint(amax);
  int e;
  if (b >= 0x00800000u) {
    const int e0 = static_cast<int>(b >> 23) - 127;
    e = (b & 0x7FFFFFu) <= 0x400000u ? e0 - 2 : e0 - 1;
  } else {  // subnormal
    const int e0 = ilogbf(amax);
    e = amax <= 6.0f * exp2i(max(e0 - 2, -149)) ? e0 - 2 : e0 - 1;
  }
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

// Four lanes, one 32-block: lane s (= lane % 4 within its aligned quad) holds elements
// 8s .. 8s + 7. The same expansion as warp_terms4 (amax over the quad by two shuffles); each lane
// writes its own 32-bit word of term j's 16 bytes to rows + j * pitch (rows already offset by 4s)
// and the quad's lane 0 the scale byte. All 32 lanes of the warp must call (quads independent);
// `store` gates the memory writes only.
__device__ __forceinline__ void quad_terms4(float (&r)[8], uint8_t* rows, size_t pitch, uint8_t* sf,
                                            size_t sf_pitch, bool lead, bool store) {
#pragma unroll 1
  for (int j = 0; j < 4; j++) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(r[i]));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
    uint32_t w = 0;
    int e = 0;
    if (amax > 0.0f) {
      e = e2m1_block_exponent(amax);
      const float inv = exp2i(-e), sc = exp2i(e);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const bool neg = r[i] < 0.0f;
        const int c = e2m1_nearest(fminf(fabsf(r[i]) * inv, 6.0f));
        const float q = e2m1_magnitude(c) * sc;
        r[i] = neg ? r[i] + q : r[i] - q;
        w |= (static_cast<uint32_t>(c) | (neg && c ? 8u : 0u)) << (4 * i);
      }
    }
    if (store) {
      *reinterpret_cast<uint32_t*>(rows + j * pitch) = w;
      if (lead) sf[j * sf_pitch] = static_cast<uint8_t>(amax > 0.0f ? e + 127 : 127);
    }
  }
}

}  // namespace rmoe
