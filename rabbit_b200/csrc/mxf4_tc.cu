// mxf4_tc.cu -- y[S,O] = x[S,I] . W^T for MXFP4 weights on the 5th-generation tensor cores.
//
// The weights stay in the checkpoint's bytes: E2M1 nibbles (low nibble = even column) and one
// E8M0 scale per 32 columns, which is exactly the operand format of tcgen05 kind::mxf4 with
// block32 scaling, so the tensor core decodes them and no CUDA-core dequantization runs.
//
// The activations become a four-term E2M1 expansion: for each 32-block, term 0 is x rounded to
// E2M1 under the smallest power-of-two scale with |x| / scale <= 6, term j+1 the same rounding of
// what term j left over. Each term gains at least log2(6) bits, so four terms carry ~11 bits
// (f16-like); every product is exact in the tensor core and the sum is accumulated in f32.
// The terms of token t are operand-B rows 4t..4t+3; the epilogue adds their four columns.
//
// Kernel: one CTA per 128 weight rows x up to 32 tokens. Warp 0 issues TMA tile loads (weights
// and activation terms, 128-byte swizzle) into a 4-stage ring; warps 2-5 write each stage's scale
// factors into TMEM; warp 1 issues 4 MMAs (K = 64 each) per 256-column stage and commits the
// stage back to the producers; warps 2-5 then read the f32 accumulators from TMEM. Every wait
// is bounded: on timeout the kernel flags `err`, stops issuing, drains and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace rmoe {

constexpr int kTcStages = 4;
constexpr int kTcThreads = 192;
constexpr int kTcKStage = 256;      // K elements per stage (128 bytes of E2M1 per row)
constexpr int kTcTokTile = 32;      // tokens per CTA (N = 4 terms x 32 = 128)

// ---------------------------------------------------------------------- activation terms
__device__ __forceinline__ int e2m1_code(float v) {  // v >= 0, v <= 6: nearest grid point
  return v < 0.25f ? 0 : v < 0.75f ? 1 : v < 1.25f ? 2 : v < 1.75f ? 3 : v < 2.5f ? 4 : v < 3.5f ? 5 : v < 5.0f ? 6 : 7;
}
__device__ __forceinline__ float e2m1_value(int c) {  // 0, .5, 1, 1.5, 2, 3, 4, 6
  return c < 4 ? 0.5f * c : static_cast<float>(2 << ((c - 4) >> 1)) * (1.0f + 0.5f * (c & 1));
}

// One thread per (token, 32-block). xt: [4S][I/2] E2M1 bytes, xsf: [4S][I/32] E8M0.
__global__ void __launch_bounds__(256) mxf4_terms_kernel(const void* __restrict__ x, int x_dtype,
                                                         int S, int I, uint8_t* __restrict__ xt,
                                                         uint8_t* __restrict__ xsf) {
  const int nb = I / 32;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= S * nb) return;
  const int s = idx / nb, b = idx % nb;
  float r[32];
#pragma unroll
  for (int i = 0; i < 32; i++) r[i] = load_elem(x, x_dtype, static_cast<size_t>(s) * I + b * 32 + i);
#pragma unroll 1
  for (int j = 0; j < 4; j++) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(r[i]));
    int e = 0;
    if (amax > 0.0f) {
      const int e0 = ilogbf(amax);  // amax in [2^e0, 2^(e0+1))
      e = amax <= 6.0f * exp2i(max(e0 - 2, -149)) ? e0 - 2 : e0 - 1;
      e = max(-127, min(127, e));
    }
    const float inv = exp2i(max(-e, -149)), sc = e >= -126 ? exp2i(e) : 0.0f;
    uint32_t packed[4] = {0, 0, 0, 0};
    if (amax > 0.0f && sc > 0.0f) {
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const bool neg = r[i] < 0.0f;
        const int c = e2m1_code(fminf(fabsf(r[i]) * inv, 6.0f));
        const float q = e2m1_value(c) * sc;
        r[i] = neg ? r[i] + q : r[i] - q;
        const uint32_t nib = static_cast<uint32_t>(c) | (neg && c ? 8u : 0u);
        packed[i / 8] |= nib << (4 * (i % 8));
      }
    }
    const size_t row = static_cast<size_t>(4 * s + j);
    uint4* dst = reinterpret_cast<uint4*>(xt + row * (I / 2) + b * 16);
    *dst = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    xsf[row * nb + b] = static_cast<uint8_t>(amax > 0.0f ? e + 127 : 127);
  }
}

// ---------------------------------------------------------------------- the GEMM
struct TcGemmArgs {
  const uint8_t* w_sf;   // [O][I/32] E8M0
  const uint8_t* x_sf;   // [4S][I/32] E8M0
  float* y;              // [S][O]
  int S, O, I;
  int b_rows;            // rows of the activation-term box (multiple of 8, <= 128)
  unsigned* err;
};

// Scale-factor word of rows `row` (4 k-blocks starting at kb0), 127 (= 1.0) past the edges.
__device__ __forceinline__ uint32_t sf_word(const uint8_t* sf, int row, int rows, int kb0, int nkb) {
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int kb = kb0 + i;
    const uint32_t v = (row < rows && kb < nkb) ? __ldg(sf + static_cast<size_t>(row) * nkb + kb) : 127u;
    w |= v << (8 * i);
  }
  return w;
}

__global__ void __launch_bounds__(kTcThreads, 1) mxf4_tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                                   const __grid_constant__ CUtensorMap tmap_x,
                                                                   TcGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_bytes = 128 * 128;
  const int b_bytes = a.b_rows * 128;
  const int stage_bytes = a_bytes + ((b_bytes + 1023) & ~1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * stage_bytes);
  uint64_t* sf_full = full + kTcStages;
  uint64_t* empty = sf_full + kTcStages;
  uint64_t* acc_full = empty + kTcStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * 128;
  const int t0 = blockIdx.y * kTcTokTile;
  const int ntok = min(kTcTokTile, a.S - t0);
  const int N = ((4 * ntok + 7) / 8) * 8;
  const int nk = (a.I + kTcKStage - 1) / kTcKStage;
  const int nkb = a.I / 32;
  const uint32_t acc_cols = 128;                 // accumulator columns reserved (N <= 128)
  const uint32_t tmem_cols = 256;                // + 4 stages x 16 scale-factor columns

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcStages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&sf_full[i], 128);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_x);
      int issued = 0;
      for (int ks = 0; ks < nk; ks++, issued++) {
        const int slot = ks % kTcStages;
        if (ks >= kTcStages &&
            !mbar_wait_bounded(&empty[slot], ((ks / kTcStages) - 1) & 1, a.err, 16u)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* sa = smem + slot * stage_bytes;
        mbar_arrive_expect_tx(&full[slot], a_bytes + b_bytes);
        tma_load_2d(sa, &tmap_w, ks * 128, m0, &full[slot]);
        tma_load_2d(sa + a_bytes, &tmap_x, ks * 128, 4 * t0, &full[slot]);
      }
      // copies still landing (only after an abort) must finish before the CTA exits
      for (int ks = max(0, issued - kTcStages); ks < issued; ks++)
        mbar_wait_bounded(&full[ks % kTcStages], (ks / kTcStages) & 1, a.err, 512u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = mxf4_idesc(N);
      bool ok = true;
      for (int ks = 0; ks < nk && ok; ks++) {
        const int slot = ks % kTcStages;
        const uint32_t ph = (ks / kTcStages) & 1;
        if (!mbar_wait_bounded(&full[slot], ph, a.err, 32u) || !mbar_wait_bounded(&sf_full[slot], ph, a.err, 64u)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* sa = smem + slot * stage_bytes;
        const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + a_bytes);
        const uint32_t sfa = tbase + acc_cols + slot * 16, sfb = sfa + 8;
#pragma unroll
        for (int s = 0; s < 4; s++) {
          const uint32_t byte = static_cast<uint32_t>(2 * (s & 1)) << 30;
          mma_mxf4(tbase, da + 2 * s, db + 2 * s, idesc, (sfa + 4 * (s >> 1)) | byte,
                   (sfb + 4 * (s >> 1)) | byte, (ks > 0 || s > 0) ? 1u : 0u);
        }
        tc_commit(&empty[slot]);
      }
      tc_commit(acc_full);  // also when aborted: the epilogue then skips its stores
    }
  } else {
    // ------------------------------------------------------------- scale factors + epilogue
    const int q = warp & 3;                       // TMEM sub-partition of this warp
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    for (int ks = 0; ks < nk; ks++) {
      const int slot = ks % kTcStages;
      if (ks >= kTcStages && !mbar_wait_bounded(&empty[slot], ((ks / kTcStages) - 1) & 1, a.err, 128u)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      const uint32_t sfa = tbase + acc_cols + slot * 16, sfb = sfa + 8;
#pragma unroll
      for (int g = 0; g < 2; g++) {
        const int kb0 = ks * 8 + 4 * g;
        uint32_t wa[4], wb[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          wa[j] = sf_word(a.w_sf, m0 + lane + 32 * j, a.O, kb0, nkb);
          const int n = lane + 32 * j;  // operand-B row = 4 * token + term
          wb[j] = n < 4 * ntok ? sf_word(a.x_sf, 4 * t0 + n, 4 * a.S, kb0, nkb) : 0x7f7f7f7fu;
        }
        tmem_st4(lane_addr | (sfa + 4 * g), wa[0], wa[1], wa[2], wa[3]);
        tmem_st4(lane_addr | (sfb + 4 * g), wb[0], wb[1], wb[2], wb[3]);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sf_full[slot]);
    }
    // epilogue: row = m0 + 32 q + lane; columns 4t..4t+3 are token t's terms
    const bool got = mbar_wait_bounded(acc_full, 0, a.err, 256u);
    tc_fence_after();
    const int row = m0 + 32 * q + lane;
    if (got && !*abort_flag) {
      for (int c0 = 0; c0 < N; c0 += 8) {
        float v[8];
        tmem_ld8(tbase + lane_addr + c0, v);
        if (row < a.O) {
          const int ta = c0 / 4;
          if (ta < ntok) a.y[static_cast<size_t>(t0 + ta) * a.O + row] = ((v[0] + v[1]) + v[2]) + v[3];
          if (ta + 1 < ntok) a.y[static_cast<size_t>(t0 + ta + 1) * a.O + row] = ((v[4] + v[5]) + v[6]) + v[7];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, tmem_cols);
  }
}

// ---------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Byte matrix [rows][row_bytes] as a 2-D tensor, box = 128 bytes x box_rows, 128-byte swizzle.
bool make_tmap_sw128(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Byte matrix [rows][row_bytes] as a 2-D tensor, box = box_bytes x box_rows, no swizzle.
bool make_tmap_rows(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                    uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_bytes, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool mxf4_tc_supported(int S, int I, int O) {
  return S > 0 && O > 0 && I % 32 == 0 && (I / 2) % 16 == 0 && encode_fn() != nullptr;
}

size_t mxf4_tc_workspace_bytes(int S, int I) {
  return static_cast<size_t>(4) * S * (I / 2) + static_cast<size_t>(4) * S * (I / 32) + 256;
}

cudaError_t launch_mxf4_tc_matmul(float* y, const void* x, int x_dtype, const uint8_t* w,
                                  const uint8_t* w_sf, int S, int I, int O, void* ws, size_t ws_bytes,
                                  unsigned* err, cudaStream_t st) {
  if (S <= 0 || O <= 0) return cudaSuccess;
  if (!mxf4_tc_supported(S, I, O) || ws_bytes < mxf4_tc_workspace_bytes(S, I)) return cudaErrorInvalidValue;
  uint8_t* xt = static_cast<uint8_t*>(ws);
  uint8_t* xsf = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(xt + static_cast<size_t>(4) * S * (I / 2)) + 15) & ~uintptr_t(15));
  const int nthr = S * (I / 32);
  mxf4_terms_kernel<<<(nthr + 255) / 256, 256, 0, st>>>(x, x_dtype, S, I, xt, xsf);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int b_rows = std::min(128, ((4 * S + 7) / 8) * 8);
  CUtensorMap tw, tx;
  if (!make_tmap_sw128(&tw, w, I / 2, O, 128) || !make_tmap_sw128(&tx, xt, I / 2, 4 * S, b_rows))
    return cudaErrorInvalidValue;
  TcGemmArgs a{};
  a.w_sf = w_sf; a.x_sf = xsf; a.y = y; a.S = S; a.O = O; a.I = I; a.b_rows = b_rows; a.err = err;
  const int stage_bytes = 128 * 128 + ((b_rows * 128 + 1023) & ~1023);
  // at least 80 KB so that at most two CTAs share an SM (2 x 256 TMEM columns = all 512)
  const size_t smem = std::max<size_t>(80 * 1024, 1024 + static_cast<size_t>(kTcStages) * stage_bytes + 256);
  e = cudaFuncSetAttribute(mxf4_tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid((O + 127) / 128, (S + kTcTokTile - 1) / kTcTokTile);
  mxf4_tc_gemm_kernel<<<grid, kTcThreads, smem, st>>>(tw, tx, a);
  return cudaGetLastError();
}

}  // namespace rmoe
