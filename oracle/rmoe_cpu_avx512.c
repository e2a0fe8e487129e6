/*
 * rmoe_cpu_avx512.c -- the timed CPU baseline: a restatement of rabbit's AVX-512F/BW MXFP4
 * tier (src/kernels.rs:703-749 dot_mxfp4_f32_avx512, :783-797 matmul_mxfp4_avx512).
 * TEST/BENCH INFRASTRUCTURE ONLY -- never linked into the product library.
 *
 * Per 32-element MXFP4 block: unpack 16 bytes into 32 nibbles (low nibble = even column), look
 * the magnitudes up with a lane permute, XOR the sign bit in, multiply by the block's E8M0
 * factor, and FMA against x in two 16-lane accumulators; one horizontal reduce at the end and
 * a scalar tail, exactly the arithmetic of the reference tier. Output rows run in parallel
 * (OpenMP here, rayon in the reference).
 */
#include <immintrin.h>
#include <stddef.h>
#include <stdint.h>

#include "rmoe_oracle.h"

int orc_has_avx512(void) {
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw");
}

__attribute__((target("avx512f,avx512bw"))) static float dot_row_avx512(const uint8_t* w,
                                                                        const uint8_t* bs,
                                                                        const float* xs,
                                                                        size_t n) {
  const __m128i m4 = _mm_set1_epi8(0x0F);
  const __m512i idx_mask = _mm512_set1_epi32(0x7);
  const __m512i sign_mask = _mm512_set1_epi32(0x8);
  const __m512 table = _mm512_setr_ps(0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f, 0.0f,
                                      0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f);
  __m512 acc0 = _mm512_setzero_ps(), acc1 = _mm512_setzero_ps();
  size_t i = 0;
  for (; i + 32 <= n; i += 32) {
    __m512 sv = _mm512_set1_ps(orc_e8m0_decode(bs[i / 32]));
    __m128i by = _mm_loadu_si128((const __m128i*)(w + (i >> 1)));
    __m128i lo = _mm_and_si128(by, m4);
    __m128i hi = _mm_and_si128(_mm_srli_epi16(by, 4), m4);
    __m512i n0 = _mm512_cvtepu8_epi32(_mm_unpacklo_epi8(lo, hi));
    __m512i n1 = _mm512_cvtepu8_epi32(_mm_unpackhi_epi8(lo, hi));
    __m512 mag0 = _mm512_permutexvar_ps(_mm512_and_si512(n0, idx_mask), table);
    __m512i s0 = _mm512_slli_epi32(_mm512_and_si512(n0, sign_mask), 28);
    __m512 w0 = _mm512_mul_ps(_mm512_castsi512_ps(_mm512_xor_si512(_mm512_castps_si512(mag0), s0)), sv);
    __m512 mag1 = _mm512_permutexvar_ps(_mm512_and_si512(n1, idx_mask), table);
    __m512i s1 = _mm512_slli_epi32(_mm512_and_si512(n1, sign_mask), 28);
    __m512 w1 = _mm512_mul_ps(_mm512_castsi512_ps(_mm512_xor_si512(_mm512_castps_si512(mag1), s1)), sv);
    acc0 = _mm512_fmadd_ps(_mm512_loadu_ps(xs + i), w0, acc0);
    acc1 = _mm512_fmadd_ps(_mm512_loadu_ps(xs + i + 16), w1, acc1);
  }
  float a = _mm512_reduce_add_ps(_mm512_add_ps(acc0, acc1));
  for (; i < n; i++) {
    uint8_t byte = w[i >> 1];
    uint8_t nib = (i & 1) == 0 ? (byte & 0xF) : (byte >> 4);
    float t = xs[i] * orc_e2m1_decode(nib);
    a = a + t * orc_e8m0_decode(bs[i / 32]);
  }
  return a;
}

void orc_matmul_mxfp4_avx512(float* y, const float* x, const uint8_t* data, const uint8_t* bs,
                             size_t s, size_t i, size_t o) {
  size_t rb = (i + 1) / 2, bpr = (i + 31) / 32;
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++)
    for (size_t si = 0; si < s; si++)
      y[si * o + (size_t)oi] =
          dot_row_avx512(data + (size_t)oi * rb, bs + (size_t)oi * bpr, x + si * i, i);
}
