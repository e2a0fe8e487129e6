// common.cuh -- shared device helpers for the routed-MoE kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rmoe {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// Activation / weight element types accepted at the boundary.
enum : int { kF32 = 0, kBF16 = 1 };
// Expert weight formats.
enum : int { kMxfp4 = 0, kInt4g = 1 };

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Element idx of an f32 or bf16 array, widened exactly to f32.
__device__ __forceinline__ float load_elem(const void* p, int dtype, size_t idx) {
  if (dtype == kBF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[idx]);
  return static_cast<const float*>(p)[idx];
}

// E8M0 byte -> 2^(b-127); byte 0 is the f32 subnormal 2^-127 (rabbit quant.rs:391-396).
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
  return b == 0 ? __uint_as_float(1u << 22) : __uint_as_float(b << 23);
}

// Exact power of two 2^e for e in [-149, 127].
__device__ __forceinline__ float exp2i(int e) {
  if (e >= -126) return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
  return __uint_as_float(1u << (e + 149));
}

// Eight E2M1 nibbles (one 32-bit word, low nibble = even column) -> four f16x2 registers, each
// holding the (even, odd) column pair of one byte: .x = low nibble, .y = high nibble.
__device__ __forceinline__ void e2m1x8_to_h2(uint32_t w, uint32_t (&h)[4]) {
  asm("{ .reg .b8 b0,b1,b2,b3;\n\t"
      "mov.b32 {b0,b1,b2,b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3; }"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// Eight offset-binary int4 nibbles (value + 8, low nibble first) -> four f16x2 holding
// (v - 8) exactly. Pairs are (n0,n4), (n1,n5), (n2,n6), (n3,n7): the f16 bit pattern
// 0x6400 | n is 1024 + n, so one LOP3 and one HSUB2 per pair.
__device__ __forceinline__ void i4x8_to_h2(uint32_t w, uint32_t (&h)[4]) {
  const uint32_t kMagic = 0x64086408u;  // (1032, 1032)
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t) : "r"(w >> (4 * q)), "r"(0x000f000fu),
        "r"(0x64006400u));  // (a & b) | c
    __half2 v = __hsub2(*reinterpret_cast<__half2*>(&t),
                        *reinterpret_cast<const __half2*>(&kMagic));
    h[q] = *reinterpret_cast<uint32_t*>(&v);
  }
}

__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                      *reinterpret_cast<__half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ float h2sum_f32(uint32_t a) {
  __half2 v = *reinterpret_cast<__half2*>(&a);
  return __low2float(v) + __high2float(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Streaming 16-byte global load that skips L1 (weights are read exactly once per call).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// The exponent e such that |amax| * 2^e lies in [2^7, 2^8): the power-of-two scale that puts
// a row into f16 range for the HFMA2 dot products (block partial sums stay below 6*32*256).
__device__ __forceinline__ int f16_row_exponent(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 0;
  int ex = static_cast<int>((__float_as_uint(amax) >> 23) & 0xff) - 127;  // floor(log2) for normals
  if (ex == -127) ex = -127 + (31 - __clz(__float_as_uint(amax) & 0x7fffff)) - 22;  // subnormal
  int e = 7 - ex;
  return e > 120 ? 120 : (e < -120 ? -120 : e);
}

// sigmoid / silu exactly as the reference spells them in f32: 1/(1+exp(-x)), x/(1+exp(-x)).
// exp is evaluated in double and rounded once to f32 (glibc's expf is within 0.502 ulp of the
// true value, so the two agree except within a hair of a rounding midpoint).
__device__ __forceinline__ float exp_f32(float x) { return static_cast<float>(exp(static_cast<double>(x))); }
__device__ __forceinline__ float sigmoid_ref(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-x)));
}
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, exp_f32(-x))); }
// The expert gate (glm52::moe::Activation::combine, src/glm52/moe.rs:58-70): SiLU, or Kimi
// K3's SituAndMul beta tanh(g / beta) sigmoid(g) * u' (u' = lb tanh(u / lb) with a linear beta lb,
// kimi_linear::ops::situ_and_mul). kind: 0 SiLU, 1 Situ. `exact_silu` selects the correctly
// rounded exp of the reference for SiLU (the CUDA-core paths keep it; the tensor-core paths
// expand h into E2M1 terms next and use expf).
__device__ __forceinline__ float silu_f32(float x);
__device__ __forceinline__ float act_gate(int kind, float beta, float linear_beta, float g, float u,
                                          bool exact_silu) {
  if (kind == 0) return __fmul_rn(exact_silu ? silu_ref(g) : silu_f32(g), u);
  const float uu = linear_beta > 0.0f ? linear_beta * tanhf(u / linear_beta) : u;
  const float situ = beta * tanhf(g / beta) * (1.0f / (1.0f + expf(-g)));
  return situ * uu;
}

// silu with the single-precision expf (<= 2 ulp): for h that is expanded into E2M1 terms next
// (~11 bits kept), where the reference's correctly rounded exp buys nothing and costs a
// double-precision exp per element.
__device__ __forceinline__ float silu_f32(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

}  // namespace rmoe
