// i4_tc.cu -- the routed-expert GEMMs of a grouped-int4 layer (QTKind::I4Grouped, src/quant.rs:100;
// matmul_i4_grouped, src/kernels.rs:276-296) on the tcgen05 tensor cores, for batches of tokens.
//
// The int4 weights stay 4-bit in HBM and in shared memory: each stage of a weight tile lands by
// one bulk copy, and sixteen dequantizing warps turn it into f16 straight into TMEM, where
// tcgen05.mma kind::f16 reads its A operand (the "A from tensor memory" form). So shared memory
// carries only the packed nibbles and the activations, never the 4x wider f16 weights. Per
// element: (nibble - 8) is exact in f16, and (nibble - 8) x scale is exact in f16 whenever the
// product is in f16's normal range (a bf16-representable scale has 8 significant bits, a nibble
// 3); products below 2^-14 round to f16 subnormals (an absolute error under 2^-25, far inside
// the 1e-2 tolerance). Activations are f16 rows per dispatch position (x gathered per position
// for gate/up, h written by the gate/up epilogue for down), f32 accumulation in TMEM. Like the
// CUDA-core int4 path, this assumes activations and h within f16's range (|v| < 65504).
//
// Tiles: GATE_UP tile m = 64 gate rows 64m.. then the same 64 up rows (the epilogue pairs them
// for the SwiGLU), K = hidden; DOWN tile m = 128 hidden rows, K = inter. A unit of work is one
// (chunk of <= 32 positions of one expert, tile) pair over its whole K; units are dealt round
// robin to the persistent CTAs (all units have the same length, so the split is even to one).
//
// Weight layout (written once at upload by i4_relayout_kernel): for every tile m and 256-column
// stage ks one block of kI4Block bytes = [128 rows x 128 B of nibbles] + [128 rows x 8 f32 group
// scales of the stage's eight 32-column groups]. Inside each 32-bit word the eight nibbles of
// columns 8w..8w+7 sit in the order 0,2,4,6,1,3,5,7, so that (word >> 4j) & 0x000F000F puts
// columns 2j and 2j+1 into the two halves of an f16x2 (magic 0x6400: 1024 + nibble).
//
// Stages are 256 columns deep (20 KB of weights, 16 KB of activations) and five of them sit in
// shared memory per SM, ~180 KB in flight: what HBM's latency under load needs for the SM's share
// of bandwidth. Dequantized A has its own three-stage ring in TMEM.
//
// What bounds it (measured at C4, ~16 positions per expert): the MMAs themselves. One kind::f16
// MMA (M 128, N 32, K 16) with A from TMEM takes ~100 cycles of the tensor pipe however small N
// is, and the dequantizing warps' TMEM stores contend with the MMAs' A reads (a stage of 16 MMAs:
// 0.87 us without the stores, 1.4 us with them). HBM would allow ~0.35 us per stage.
//
// Warp roles (704 threads): warp 0 stage copies (weights by bulk copy, activations by TMA), warp
// 1 MMA issuer, warps 2-17 dequantize (warp w: TMEM lanes 32 (w % 4).., quarter (w - 2) / 4 of the
// stage's K), warps 18-21 epilogue. Every wait is bounded;
// on a timeout the roles stop, drain their copies and the MMAs, and free TMEM.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace rmoe {

constexpr int kI4KStage = 256;    // K elements per stage
constexpr int kI4N = kI4Chunk;    // positions per chunk = MMA N (32)
constexpr int kI4Ring = 5;        // stages of nibbles + activations in shared memory
constexpr int kI4ARing = 3;       // stages of dequantized A in TMEM
constexpr int kI4RowBytes = kI4KStage / 2;                          // nibbles of one row per stage
constexpr int kI4Groups = kI4KStage / 32;                           // scale groups of 32 per stage
constexpr int kI4Block = 128 * kI4RowBytes + 128 * kI4Groups * 4;   // one weight stage (20 KB)
constexpr int kI4BBox = kI4N * 128;                                 // 32 rows x 64 f16 (one SW128 box)
constexpr int kI4BSlot = kI4BBox * (kI4KStage / 64);                // one activation stage (16 KB)
constexpr int kI4DqWarps = 16;    // dequantizing warps: 4 sub-partitions x 4 quarters of the stage
constexpr int kI4Threads = (6 + kI4DqWarps) * 32;
constexpr uint32_t kI4TmemCols = 512;
constexpr uint32_t kI4AccCols = 32;               // one accumulator: 32 f32 columns
constexpr int kI4Acc = 4;
constexpr uint32_t kI4ACols = kI4KStage / 2;      // TMEM columns of one A stage (two f16 per column)

struct I4Args {
  const int32_t* ch_expert;
  const int32_t* ch_pos;
  const int32_t* ch_n;
  const int32_t* n_chunks;
  const int32_t* offsets;   // positions per slot (a single-chunk expert's weights are read once)
  const float* perm_w;      // weight of each position (routing weight or shared gate)
  const uint8_t* tiles;     // tile-major weights of slot 0 (this projection)
  size_t stride;            // bytes between slots
  int K, out_rows;          // GATE_UP: hidden, inter; DOWN: inter, hidden
  int inter, hidden;
  __half* h;                // GATE_UP out: [P][inter] f16
  float* y;                 // DOWN out: [P][hidden] f32
  ActParams act;
  unsigned* err;
  unsigned long long spin_ns;
  unsigned long long* trace;  // optional: CTA 0's first 512 stages, [8] timestamps each
};

struct I4Smem {
  uint8_t raw[kI4Ring][kI4Block];
  alignas(1024) uint8_t b[kI4Ring][kI4BSlot];
  float ubuf[64][kI4N + 1];
  uint64_t raw_full[kI4Ring], b_full[kI4Ring], b_empty[kI4Ring];
  uint64_t a_full[kI4ARing], a_empty[kI4ARing];
  uint64_t acc_full[kI4Acc], acc_empty[kI4Acc];
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};
static_assert(sizeof(I4Smem) + 1024 <= 227 * 1024, "i4 shared memory");
static_assert(kI4Acc * kI4AccCols + kI4ARing * kI4ACols <= kI4TmemCols, "i4 TMEM columns");

__host__ __device__ constexpr uint32_t f16_idesc(int n) {
  return (1u << 4)                                 // D format F32
         | (0u << 7) | (0u << 10)                  // A, B format F16
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(128 >> 4) << 24);  // M / 16
}

// D[tmem_d] (+)= A[tmem_a] . B[desc_b]^T, A (M = 128 rows in TMEM lanes, 16 f16 of K packed two per
// column) from tensor memory, B K-major from shared memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// All four epilogue warps agree (named barrier 1, AND of the predicate).
__device__ __forceinline__ bool i4_epi_all(bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\t"
      "setp.ne.s32 a, %1, 0;\n\t"
      "bar.red.and.pred b, 1, 128, a;\n\t"
      "selp.s32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"(static_cast<int>(p))
      : "memory");
  return r != 0;
}

template <int MODE>  // 0 gate/up, 1 down
__global__ void __launch_bounds__(kI4Threads, 1) i4_moe_kernel(const __grid_constant__ CUtensorMap bmap, I4Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  I4Smem& sm = *reinterpret_cast<I4Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int S = kI4Ring, SA = kI4ARing;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&sm.raw_full[i], 1);
      mbar_init(&sm.b_full[i], 1);
      mbar_init(&sm.b_empty[i], 1);
    }
    for (int i = 0; i < SA; i++) {
      mbar_init(&sm.a_full[i], kI4DqWarps);
      mbar_init(&sm.a_empty[i], 1);
    }
    for (int i = 0; i < kI4Acc; i++) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], 4);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_slot, kI4TmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_slot;
  volatile int* abort_flag = &sm.abort_flag;
  griddep_wait();  // dispatch, the activation rows (and for DOWN the gate/up kernel's h)
  if (threadIdx.x == 0) griddep_launch_dependents();
  const int nch = *a.n_chunks;
  const int kst = a.K / kI4KStage;
  const int ntm = MODE == 0 ? a.out_rows / 64 : a.out_rows / 128;
  const int total = nch * ntm;
  const int G = gridDim.x;
  const uint32_t a_base = tbase + kI4Acc * kI4AccCols;  // TMEM columns of the A stage ring
  constexpr int kEpi0 = 2 + kI4DqWarps;  // first epilogue warp

  if (warp == 0) {
    // ------------------------------------------------------------------ stage copies
    // one thread issues each stage's weight copy and activation loads together, both gated by the
    // completion of the MMAs of the stage that used the slot before (the dequantizing warps have
    // consumed its nibbles by then), so neither stream queues up behind the other
    if (lane == 0) {
      tma_prefetch_desc(&bmap);
      int i = 0;
      for (int u = blockIdx.x; u < total && !*abort_flag; u += G) {
        const int c = u / ntm, m = u % ntm;
        const int e = __ldg(a.ch_expert + c);
        const int p0 = __ldg(a.ch_pos + c);
        const bool once = __ldg(a.offsets + e + 1) - __ldg(a.offsets + e) <= kI4N;  // one chunk: read once
        const uint8_t* src = a.tiles + static_cast<size_t>(e) * a.stride + static_cast<size_t>(m) * kst * kI4Block;
        bool ok = true;
        for (int ks = 0; ks < kst; ks++, i++) {
          const int slot = i % S;
          if (i >= S && !mbar_wait_bounded(&sm.b_empty[slot], ((i / S) - 1) & 1, a.err, 0x1u)) {
            ok = false;
            break;
          }
          if (a.trace && blockIdx.x == 0 && i < 512) a.trace[8 * i + 0] = global_ns();
          mbar_arrive_expect_tx(&sm.raw_full[slot], kI4Block);
          if (once) bulk_g2s_once(sm.raw[slot], src + static_cast<size_t>(ks) * kI4Block, kI4Block, &sm.raw_full[slot]);
          else bulk_g2s(sm.raw[slot], src + static_cast<size_t>(ks) * kI4Block, kI4Block, &sm.raw_full[slot]);
          mbar_arrive_expect_tx(&sm.b_full[slot], kI4BSlot);
#pragma unroll
          for (int j = 0; j < kI4KStage / 64; j++)
            tma_load_2d(sm.b[slot] + j * kI4BBox, &bmap, ks * (kI4KStage * 2) + j * 128, p0, &sm.b_full[slot]);
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      for (int j = (i > S ? i - S : 0); j < i; j++) {  // copies still landing (after an abort)
        mbar_wait_bounded(&sm.raw_full[j % S], (j / S) & 1, a.err, 0x2u);
        mbar_wait_bounded(&sm.b_full[j % S], (j / S) & 1, a.err, 0x8u);
      }
    }
  } else if (warp >= 2 && warp < kEpi0) {
    // ------------------------------------------------------------------ dequantize into TMEM
    // warp w: rows 32 (w % 4).. (its TMEM sub-partition), quarter ((w - 2) / 4) of the stage's K
    const int q = warp % 4, quarter = (warp - 2) / 4;
    const int row = 32 * q + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    int i = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += G) {
      for (int ks = 0; ks < kst; ks++, i++) {
        const int slot = i % S, as = i % SA;
        bool got = mbar_wait_bounded(&sm.raw_full[slot], (i / S) & 1, a.err, 0x10u);
        if (a.trace && blockIdx.x == 0 && i < 512 && warp == 2 && lane == 0) a.trace[8 * i + 1] = global_ns();
        if (got && i >= SA) got = mbar_wait_bounded(&sm.a_empty[as], ((i / SA) - 1) & 1, a.err, 0x20u);
        if (!__all_sync(kFull, got && !*abort_flag)) {
          ok = false;
          break;
        }
        if (a.trace && blockIdx.x == 0 && i < 512 && warp == 2 && lane == 0) a.trace[8 * i + 2] = global_ns();
        // this quarter: 64 K elements = 32 nibble bytes, two groups of 32
        const uint8_t* rb = sm.raw[slot] + row * kI4RowBytes + quarter * 32;
        const uint4 wa = *reinterpret_cast<const uint4*>(rb);
        const uint4 wb = *reinterpret_cast<const uint4*>(rb + 16);
        const float2 sc = *reinterpret_cast<const float2*>(sm.raw[slot] + 128 * kI4RowBytes +
                                                           (row * kI4Groups + quarter * 2) * 4);
        const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const __half2 s0 = __float2half2_rn(sc.x), s1 = __float2half2_rn(sc.y);
        uint32_t v[32];
#pragma unroll
        for (int wi = 0; wi < 8; wi++) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const uint32_t bits = ((ww[wi] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
            const __half2 x = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&bits), off), wi < 4 ? s0 : s1);
            v[4 * wi + j] = *reinterpret_cast<const uint32_t*>(&x);
          }
        }
        tmem_st32(lane_addr | (a_base + as * kI4ACols + quarter * 32), v);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.a_full[as]);
        if (a.trace && blockIdx.x == 0 && i < 512 && warp == 2 && lane == 0) a.trace[8 * i + 3] = global_ns();
      }
    }
    if (!ok) *abort_flag = 1;
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = f16_idesc(kI4N);
      const uint64_t db0 = sw128_desc(sm.b[0]);
      int i = 0, n = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok && !*abort_flag; u += G, n++) {
        const int buf = n % kI4Acc;
        if (n >= kI4Acc && !mbar_wait_bounded(&sm.acc_empty[buf], ((n / kI4Acc) - 1) & 1, a.err, 0x40u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tbase + buf * kI4AccCols;
        for (int ks = 0; ks < kst; ks++, i++) {
          const int slot = i % S, as = i % SA;
          const bool ga = mbar_wait_bounded(&sm.a_full[as], (i / SA) & 1, a.err, 0x80u);
          if (a.trace && blockIdx.x == 0 && i < 512) a.trace[8 * i + 5] = global_ns();
          if (!ga || !mbar_wait_bounded(&sm.b_full[slot], (i / S) & 1, a.err, 0x80u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (a.trace && blockIdx.x == 0 && i < 512) a.trace[8 * i + 4] = global_ns();
          const uint64_t db = db0 + static_cast<uint64_t>((slot * kI4BSlot) >> 4);
#pragma unroll
          for (int kk = 0; kk < kI4KStage / 16; kk++)
            mma_f16_ts(dacc, a_base + as * kI4ACols + kk * 8,
                       db + static_cast<uint64_t>(((kk / 4) * kI4BBox + 32 * (kk % 4)) >> 4), idesc,
                       (ks > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sm.a_empty[as]);   // A's TMEM slot free again
          tc_commit(&sm.b_empty[slot]);  // B's shared slot free again
        }
        if (!ok) break;
        tc_commit(&sm.acc_full[buf]);
      }
      if (!ok) *abort_flag = 1;
      tc_drain(&sm.drain, a.err);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (the last four warps)
    const int q = warp % 4;
    const int row = 32 * q + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    int n = 0;
    for (int u = blockIdx.x; u < total; u += G, n++) {
      const int buf = n % kI4Acc;
      const bool got = mbar_wait_bounded_sleep(&sm.acc_full[buf], (n / kI4Acc) & 1, a.err, 0x100u);
      if (!i4_epi_all(got && !*abort_flag)) break;
      tc_fence_after();
      float acc[32];
      tmem_ld32(tbase + buf * kI4AccCols + lane_addr, acc);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
      const int c = u / ntm, m = u % ntm;
      const int p0 = __ldg(a.ch_pos + c), nn = __ldg(a.ch_n + c);
      if (MODE == 0) {
        // rows 0..63 gate, 64..127 up of inter rows 64 m + (row % 64)
        if (row >= 64) {
#pragma unroll
          for (int t = 0; t < kI4N; t++) sm.ubuf[row - 64][t] = acc[t];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (row < 64) {
          const int ir = 64 * m + row;
#pragma unroll
          for (int t = 0; t < kI4N; t++) {
            if (t < nn) {
              const float hv = act_gate(a.act.kind, a.act.beta, a.act.linear_beta, acc[t], sm.ubuf[row][t], false) *
                               __ldg(a.perm_w + p0 + t);
              a.h[static_cast<size_t>(p0 + t) * a.inter + ir] = __float2half_rn(hv);
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      } else {
        const int orow = 128 * m + row;
#pragma unroll
        for (int t = 0; t < kI4N; t++)
          if (t < nn) a.y[static_cast<size_t>(p0 + t) * a.hidden + orow] = acc[t];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kI4TmemCols);
  }
}

// x gathered per dispatch position as f16: xh[p] = x[perm_tok[p]] for the P = total[0] positions.
__global__ void i4_gather_x_kernel(const void* __restrict__ x, int x_dtype, int H, const int32_t* __restrict__ perm_tok,
                                   const int32_t* __restrict__ total, __half* __restrict__ xh) {
  const int p = blockIdx.x;
  if (p >= *total) return;
  const size_t src = static_cast<size_t>(__ldg(perm_tok + p)) * H;
  for (int k = threadIdx.x * 2; k < H; k += blockDim.x * 2) {
    const float a = load_elem(x, x_dtype, src + k), b = load_elem(x, x_dtype, src + k + 1);
    *reinterpret_cast<__half2*>(xh + static_cast<size_t>(p) * H + k) = __floats2half2_rn(a, b);
  }
}

// Reference layout (rows of K/2 nibble bytes, scales per group_size of K) -> tile blocks.
// Tile row r: m0 row (m * half + r) for r < half, else m1 row (m * half + r - half).
__global__ void i4_relayout_kernel(const uint8_t* __restrict__ m0, const uint8_t* __restrict__ m1,
                                   const void* __restrict__ s0, const void* __restrict__ s1, int scale_bf16, int K,
                                   int gs, int half, int ntiles, uint8_t* __restrict__ dst) {
  const int KS = K / kI4KStage;
  constexpr int kWords = kI4RowBytes / 4;  // nibble words of one row per stage
  const size_t nwords = static_cast<size_t>(ntiles) * KS * 128 * kWords;
  const size_t nscales = static_cast<size_t>(ntiles) * KS * 128 * kI4Groups;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const int ng = (K + gs - 1) / gs;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nwords; i += stride) {
    const int wi = static_cast<int>(i % kWords), r = static_cast<int>((i / kWords) % 128);
    const size_t blk = i / (kWords * 128);
    const int m = static_cast<int>(blk / KS), ks = static_cast<int>(blk % KS);
    const uint8_t* row = r < half ? m0 + static_cast<size_t>(m * half + r) * (K / 2)
                                  : m1 + static_cast<size_t>(m * half + r - half) * (K / 2);
    const uint32_t src = *reinterpret_cast<const uint32_t*>(row + ks * kI4RowBytes + wi * 4);  // columns 8wi..8wi+7
    uint32_t out = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      out |= ((src >> (8 * j)) & 15u) << (4 * j);             // column 2j -> nibble slot j
      out |= ((src >> (8 * j + 4)) & 15u) << (4 * (j + 4));   // column 2j+1 -> nibble slot j + 4
    }
    *reinterpret_cast<uint32_t*>(dst + blk * kI4Block + r * kI4RowBytes + wi * 4) = out;
  }
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nscales; i += stride) {
    const int g = static_cast<int>(i % kI4Groups), r = static_cast<int>((i / kI4Groups) % 128);
    const size_t blk = i / (kI4Groups * 128);
    const int m = static_cast<int>(blk / KS), ks = static_cast<int>(blk % KS);
    const bool lo = r < half;
    const size_t srow = lo ? static_cast<size_t>(m * half + r) : static_cast<size_t>(m * half + r - half);
    const void* sp = lo ? s0 : s1;
    const size_t gi = srow * ng + (ks * kI4KStage + 32 * g) / gs;
    const float v = scale_bf16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(sp)[gi]) : static_cast<const float*>(sp)[gi];
    *reinterpret_cast<float*>(dst + blk * kI4Block + 128 * kI4RowBytes + (r * kI4Groups + g) * 4) = v;
  }
}

bool i4_tc_supported(int H, int I, int Is, int gs) {
  return H % 128 == 0 && I % 64 == 0 && H % kI4KStage == 0 && I % kI4KStage == 0 && gs % 32 == 0 &&
         (Is == 0 || Is == I);
}

size_t i4_tc_region_bytes(int H, int I, int down) {
  return down ? static_cast<size_t>(H / 128) * (I / kI4KStage) * kI4Block
              : static_cast<size_t>(I / 64) * (H / kI4KStage) * kI4Block;
}

cudaError_t launch_i4_relayout(int down, const uint8_t* m0, const uint8_t* m1, const void* s0, const void* s1,
                               int scale_bf16, int H, int I, int gs, uint8_t* dst, cudaStream_t st) {
  const int K = down ? I : H, half = down ? 128 : 64, ntiles = down ? H / 128 : I / 64;
  i4_relayout_kernel<<<4 * device_sm_count(), 256, 0, st>>>(m0, down ? m0 : m1, s0, down ? s0 : s1, scale_bf16, K,
                                                            gs, half, ntiles, dst);
  return cudaGetLastError();
}

cudaError_t launch_i4_gather_x(const void* x, int x_dtype, int H, const int32_t* perm_tok, const int32_t* total,
                               int P_max, __half* xh, cudaStream_t st) {
  if (P_max <= 0) return cudaSuccess;
  i4_gather_x_kernel<<<P_max, 256, 0, st>>>(x, x_dtype, H, perm_tok, total, xh);
  return cudaGetLastError();
}

bool make_tmap_sw128(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);

// Tensor map of f16 activation rows [rows][K] in 32-row, 64-element (128-byte) boxes, SW128.
bool i4_make_act_map(void* map, const void* base, int K, int rows) {
  return make_tmap_sw128(static_cast<CUtensorMap*>(map), base, static_cast<uint64_t>(K) * 2, rows, kI4N);
}

size_t i4_act_map_bytes() { return sizeof(CUtensorMap); }

cudaError_t launch_i4_moe(int mode, const void* act_map, const DispatchBuffers& d, const int32_t* slot_offsets,
                          int H, int I, const uint8_t* tiles, size_t stride, __half* h, float* y, ActParams act,
                          unsigned* err, unsigned long long spin_ns, cudaStream_t st, unsigned long long* trace) {
  I4Args a{};
  a.trace = trace;
  a.ch_expert = d.ch_expert;
  a.ch_pos = d.ch_pos;
  a.ch_n = d.ch_n;
  a.n_chunks = d.n_chunks;
  a.offsets = slot_offsets;
  a.perm_w = d.perm_w;
  a.tiles = tiles;
  a.stride = stride;
  a.K = mode == 0 ? H : I;
  a.out_rows = mode == 0 ? I : H;
  a.inter = I;
  a.hidden = H;
  a.h = h;
  a.y = y;
  a.act = act;
  a.err = err;
  a.spin_ns = spin_ns;
  const size_t smem = sizeof(I4Smem) + 1024;
  void (*kern)(const CUtensorMap, I4Args) = mode == 0 ? i4_moe_kernel<0> : i4_moe_kernel<1>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // one CTA per SM (each holds all 512 TMEM columns); the CTAs never wait on one another
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(device_sm_count());
  cfg.blockDim = dim3(kI4Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, *static_cast<const CUtensorMap*>(act_map), a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace rmoe
