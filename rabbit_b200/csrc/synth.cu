// synth.cu -- seeded synthetic weight bytes, written straight into device memory.
// The stream is SplitMix64 from state `key`: word i = fmix64(key + (i + 1) * golden). Byte j
// of a uniform tensor is byte (j % 8) of word j / 8; an E8M0 byte j is
// 127 + lo + (word_j >> 32) % (hi - lo + 1). rabbit_b200/synth.py generates the same bytes.
#include "common.cuh"
#include "kernels.h"

namespace rmoe {

__device__ __forceinline__ uint64_t fmix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_uniform_kernel(uint8_t* __restrict__ dst, size_t n, uint64_t key) {
  const size_t nw = (n + 7) / 8;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nw;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint64_t v = fmix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
    const size_t b0 = i * 8;
    if (b0 + 8 <= n && (reinterpret_cast<uintptr_t>(dst + b0) & 7) == 0) {
      *reinterpret_cast<uint64_t*>(dst + b0) = v;
    } else {
      for (int q = 0; q < 8 && b0 + q < n; q++) dst[b0 + q] = static_cast<uint8_t>(v >> (8 * q));
    }
  }
}

__global__ void synth_e8m0_kernel(uint8_t* __restrict__ dst, size_t n, uint64_t key, int lo, int hi) {
  const uint64_t span = static_cast<uint64_t>(hi - lo + 1);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint64_t v = fmix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
    dst[i] = static_cast<uint8_t>(127 + lo + static_cast<int>((v >> 32) % span));
  }
}

cudaError_t launch_synth_bytes(void* dst, size_t n, uint64_t key, int mode, int lo, int hi,
                               cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const int blocks = 148 * 8;
  if (mode == 0) {
    synth_uniform_kernel<<<blocks, 256, 0, st>>>(static_cast<uint8_t*>(dst), n, key);
  } else {
    if (hi < lo || 127 + lo < 0 || 127 + hi > 254) return cudaErrorInvalidValue;
    synth_e8m0_kernel<<<blocks, 256, 0, st>>>(static_cast<uint8_t*>(dst), n, key, lo, hi);
  }
  return cudaGetLastError();
}

}  // namespace rmoe
