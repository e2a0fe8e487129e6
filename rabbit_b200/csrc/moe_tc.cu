// moe_tc.cu -- the routed-expert GEMMs of an MXFP4 layer on the tcgen05 tensor cores.
//
// Operands. Expert weights are consumed as stored (E2M1 nibbles + E8M0 per 32) by
// tcgen05.mma kind::mxf4 block32. Activations enter as four-term E2M1 expansions (see
// mxf4_tc.cu): operand-B rows 4p..4p+3 are the terms of dispatch position p.
//
// One persistent kernel per projection, one CTA per SM, each CTA an equal contiguous share of
// the flattened (tile, K-stage) list, so every SM streams the same number of weight bytes:
//   GATE_UP  tile = (chunk, 64 inter rows): A rows 0..63 = gate rows, 64..127 = the same up rows;
//            K = hidden. Epilogue: h = silu(g) * u * (routing weight or shared gate) of each
//            position, written straight back as the four-term operand of the down GEMM.
//   DOWN     tile = (chunk, 128 hidden rows), K = inter; epilogue y[position][row].
//   DOWN_ONE (a single token) tile = 128 hidden rows, K = the token's k routed experts and the
//            shared expert back to back: the routing weights already sit in the operand, so the
//            accumulator is the combined output row and no combine pass follows.
// A tile whose stages straddle two CTAs is accumulated in parts; each part is stored, and the
// CTA that completes the tile's last part adds the parts in K order (deterministic).
//
// Warp roles (320 threads): warp 0 issues the TMA loads of a stage (weights and their scale
// rows, activation terms and their scale rows); warps 2-5 copy the stage's scale factors from
// shared memory into TMEM; warp 1 issues 8 MMAs (K = 64 each) per 512-column stage into one of
// two TMEM accumulators; warps 6-9 drain finished accumulators. All waits are bounded: a
// timeout sets a bit in `err`, the roles stop issuing, wait for their copies and free TMEM.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"
#include "terms.cuh"

namespace rmoe {

constexpr int kMtThreads = 320;
constexpr int kMtKStage = 512;            // K elements per stage (two 128-byte swizzle columns)
constexpr int kMtMaxStages = 6;
constexpr int kMtAccCols = 128;           // one accumulator: N <= 128 (32 positions x 4 terms)
constexpr int kMtSfCols = 32;             // per stage: 16 columns of A scales + 16 of B scales
constexpr uint32_t kMtTmemCols = 512;

enum { kModeGateUp = 0, kModeDown = 1, kModeDownOne = 2 };

struct MoeTcMaps {
  CUtensorMap a0;   // GATE_UP: gate data rows; DOWN: down data rows   (box 128 B x 64 rows, SW128)
  CUtensorMap a1;   // GATE_UP: up data rows;   DOWN: unused
  CUtensorMap s0;   // scale rows of a0 (box 16 B x 64 rows)
  CUtensorMap s1;   // scale rows of a1
  CUtensorMap b;    // activation terms (box 128 B x 8 rows, SW128)
  CUtensorMap bs;   // their scale rows (box 16 B x 8 rows)
};

struct MoeTcArgs {
  const int32_t* ch_expert;
  const int32_t* ch_pos;
  const int32_t* ch_n;
  const int32_t* n_chunks;
  const float* perm_w;
  int K;               // reduction length of one expert (GATE_UP: hidden, DOWN: inter)
  int out_rows;        // GATE_UP: inter; DOWN: hidden
  int rows_per_expert_data;  // row offset between experts in the a0/a1 views
  int rows_per_expert_sf;    // row offset between experts in the s0/s1 views
  int b_boxes;         // activation boxes (8 rows) reserved per stage
  int stages;          // ring depth
  uint8_t* ht;         // GATE_UP out: h terms [4P][inter/2]
  uint8_t* hsf;        // GATE_UP out: their scales [4P][inter/32]
  int inter;           // GATE_UP: row pitch source of ht / hsf
  float* y;            // DOWN: [P][hidden]; DOWN_ONE: [hidden]
  int hidden;
  float* partial;      // [grid][2][32][128]
  int32_t* tile_cnt;   // parts finished per tile (reset by the finishing CTA)
  unsigned* err;
  const int32_t* b_tok;  // non-null (one position per chunk): B rows are the token's, 4 * b_tok[p0]
};

struct StageMeta {
  int tile, u, c, m, ks, e, p0, n, nb, first, last, pad;
};

// Shared-memory carve-up (offsets from the 1024-aligned base).
struct MtLayout {
  int stage_pitch, off_bar, off_meta, off_misc, off_ubuf, total;
};
__host__ __device__ inline MtLayout mt_layout(int stages, int b_boxes) {
  MtLayout l;
  const int sb = 32768 + 2 * b_boxes * 1024 + 2048 + b_boxes * 128;
  l.stage_pitch = (sb + 1023) & ~1023;
  l.off_bar = stages * l.stage_pitch;                          // 3 * stages + 4 mbarriers
  l.off_meta = l.off_bar + (3 * stages + 4) * 8;
  l.off_misc = l.off_meta + stages * static_cast<int>(sizeof(StageMeta));
  l.off_ubuf = (l.off_misc + 16 + 15) & ~15;                   // tmem slot, abort, last flag
  l.total = l.off_ubuf + 32 * 64 * 4;
  return l;
}

// True on every epilogue thread iff p holds on all 128 of them (named barrier 1 with an AND
// reduction): keeps their control flow identical, so barrier 1 can never be left half-entered.
__device__ __forceinline__ bool epi_all(bool p) {
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

__device__ __forceinline__ int cta_of(long long s, long long total, int grid) {
  return static_cast<int>(((s + 1) * grid + total - 1) / total) - 1;
}

// Tile / chunk / K-stage of flat stage s of the work list.
template <int MODE>
__device__ __forceinline__ void decode_stage(long long s, int L, int ntm, int kst, StageMeta& m) {
  m.tile = static_cast<int>(s / L);
  m.u = static_cast<int>(s % L);
  if (MODE == kModeDownOne) {
    m.m = m.tile;
    m.c = m.u / kst;
    m.ks = m.u % kst;
  } else {
    m.c = m.tile / ntm;
    m.m = m.tile % ntm;
    m.ks = m.u;
  }
}

template <int MODE>
__global__ void __launch_bounds__(kMtThreads, 1) moe_tc_kernel(const __grid_constant__ MoeTcMaps maps,
                                                             MoeTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const int bsub = a.b_boxes * 1024;                     // one 128-byte column of B
  const MtLayout lay = mt_layout(S, a.b_boxes);
  const int stage_pitch = lay.stage_pitch;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.off_bar);
  uint64_t* sf_full = full + S;
  uint64_t* empty = sf_full + S;
  uint64_t* acc_full = empty + S;       // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + lay.off_meta);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + lay.off_misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;
  float* ubuf = reinterpret_cast<float*>(smem + lay.off_ubuf);  // [32][64] up values (GATE_UP)

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nch = *a.n_chunks;
  const int kst = a.K / kMtKStage;
  const int ntm = MODE == kModeGateUp ? a.out_rows / 64 : a.out_rows / 128;
  const int L = MODE == kModeDownOne ? max(1, nch * kst) : kst;
  const long long ntiles = MODE == kModeDownOne ? ntm : static_cast<long long>(nch) * ntm;
  const long long total = ntiles * L;
  const int grid = gridDim.x;
  const long long s_begin = total * blockIdx.x / grid, s_end = total * (blockIdx.x + 1) / grid;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&sf_full[i], 128);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kMtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t sf_base = tbase + 2 * kMtAccCols;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && s_begin < s_end) {
      tma_prefetch_desc(&maps.a0);
      tma_prefetch_desc(&maps.b);
      long long issued = 0;
      int cc = -1, ce = 0, cp0 = 0, cn = 0, cb = 0;  // chunk fields of the previous stage
      for (long long s = s_begin; s < s_end; s++, issued++) {
        const int slot = static_cast<int>(issued % S);
        if (issued >= S && !mbar_wait_bounded(&empty[slot], ((issued / S) - 1) & 1, a.err, 0x100u)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        StageMeta m;
        decode_stage<MODE>(s, L, ntm, kst, m);
        if (m.c != cc) {
          cc = m.c;
          ce = __ldg(a.ch_expert + cc);
          cp0 = __ldg(a.ch_pos + cc);
          cn = __ldg(a.ch_n + cc);
          if (a.b_tok) cb = __ldg(a.b_tok + cp0);
        }
        m.e = ce;
        m.p0 = cp0;
        m.n = cn;
        m.nb = (4 * cn + 7) / 8;
        m.first = (m.u == 0 || s == s_begin) ? 1 : 0;
        m.last = (m.u == L - 1 || s == s_end - 1) ? 1 : 0;
        meta[slot] = m;
        uint8_t* st = smem + slot * stage_pitch;
        uint8_t* sb = st + 32768;
        uint8_t* ssa = sb + 2 * bsub;
        uint8_t* ssb = ssa + 2048;
        const uint32_t bytes = 32768 + 2048 + m.nb * (2 * 1024 + 128);
        mbar_arrive_expect_tx(&full[slot], bytes);
        const int kx = m.ks * (kMtKStage / 2);       // byte column of this stage in a row
        const int ksf = m.ks * (kMtKStage / 32);     // scale byte column
        const int erow = m.e * a.rows_per_expert_data;
        const int esf = m.e * a.rows_per_expert_sf;
        if (MODE == kModeGateUp) {
          const int r0 = m.m * 64;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            tma_load_2d(st + h * 16384, &maps.a0, kx + 128 * h, erow + r0, &full[slot]);
            tma_load_2d(st + h * 16384 + 8192, &maps.a1, kx + 128 * h, erow + r0, &full[slot]);
          }
          tma_load_2d(ssa, &maps.s0, ksf, esf + r0, &full[slot]);
          tma_load_2d(ssa + 1024, &maps.s1, ksf, esf + r0, &full[slot]);
        } else {
          const int r0 = m.m * 128;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            tma_load_2d(st + h * 16384, &maps.a0, kx + 128 * h, erow + r0, &full[slot]);
            tma_load_2d(st + h * 16384 + 8192, &maps.a0, kx + 128 * h, erow + r0 + 64, &full[slot]);
          }
          tma_load_2d(ssa, &maps.s0, ksf, esf + r0, &full[slot]);
          tma_load_2d(ssa + 1024, &maps.s0, ksf, esf + r0 + 64, &full[slot]);
        }
        for (int bx = 0; bx < m.nb; bx++) {
          const int brow = 4 * (a.b_tok ? cb : m.p0) + 8 * bx;
          tma_load_2d(sb + bx * 1024, &maps.b, kx, brow, &full[slot]);
          tma_load_2d(sb + bsub + bx * 1024, &maps.b, kx + 128, brow, &full[slot]);
          tma_load_2d(ssb + bx * 128, &maps.bs, ksf, brow, &full[slot]);
        }
      }
      // copies still landing (only after an abort) finish before the CTA exits
      for (long long i = (issued > S ? issued - S : 0); i < issued; i++)
        mbar_wait_bounded(&full[i % S], (i / S) & 1, a.err, 0x200u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && s_begin < s_end) {
      long long i = 0;
      int buf = 0, tiles_done = 0;
      bool ok = true;
      for (long long s = s_begin; s < s_end && ok; s++, i++) {
        const int slot = static_cast<int>(i % S);
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait_bounded(&full[slot], ph, a.err, 0x400u) ||
            !mbar_wait_bounded(&sf_full[slot], ph, a.err, 0x800u)) {
          ok = false;
          break;
        }
        const StageMeta m = meta[slot];
        if (m.first && tiles_done >= 2 &&
            !mbar_wait_bounded(&acc_empty[buf], ((tiles_done / 2) - 1) & 1, a.err, 0x1000u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* st = smem + slot * stage_pitch;
        const uint64_t da = sw128_desc(st), db = sw128_desc(st + 32768);
        const uint32_t idesc = mxf4_idesc(8 * m.nb);
        const uint32_t sfa = sf_base + slot * kMtSfCols, sfb = sfa + 16;
        const uint32_t dacc = tbase + buf * kMtAccCols;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const int h = k >> 2, w = k & 3;  // swizzle column, 32-byte step inside it
          const uint64_t adv = static_cast<uint64_t>((32 * w) >> 4);
          const uint64_t da_k = da + static_cast<uint64_t>((h * 16384) >> 4) + adv;
          const uint64_t db_k = db + static_cast<uint64_t>((h * bsub) >> 4) + adv;
          const uint32_t byte = static_cast<uint32_t>(2 * (k & 1)) << 30;
          mma_mxf4(dacc, da_k, db_k, idesc, (sfa + 4 * (k >> 1)) | byte, (sfb + 4 * (k >> 1)) | byte,
                   (m.first && k == 0) ? 0u : 1u);
        }
        tc_commit(&empty[slot]);
        if (m.last) {
          tc_commit(&acc_full[buf]);
          buf ^= 1;
          tiles_done++;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ scale factors -> TMEM
    const int q = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    long long i = 0;
    for (long long s = s_begin; s < s_end; s++, i++) {
      const int slot = static_cast<int>(i % S);
      if (!mbar_wait_bounded(&full[slot], (i / S) & 1, a.err, 0x4000u)) break;
      if (*abort_flag) break;
      const uint8_t* st = smem + slot * stage_pitch;
      const uint8_t* ssa = st + 32768 + 2 * bsub;
      const uint8_t* ssb = ssa + 2048;
      const int nrows_b = 8 * meta[slot].nb;
      const uint32_t sfa = sf_base + slot * kMtSfCols, sfb = sfa + 16;
      // row (lane + 32 j) of A / B: 16 scale bytes = 4 words (k-groups g = 0..3)
      uint4 ra[4], rb[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        ra[j] = *reinterpret_cast<const uint4*>(ssa + (lane + 32 * j) * 16);
        const int n = lane + 32 * j;
        rb[j] = n < nrows_b ? *reinterpret_cast<const uint4*>(ssb + n * 16) : make_uint4(0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
      }
      tmem_st4(lane_addr | (sfa + 0), ra[0].x, ra[1].x, ra[2].x, ra[3].x);
      tmem_st4(lane_addr | (sfa + 4), ra[0].y, ra[1].y, ra[2].y, ra[3].y);
      tmem_st4(lane_addr | (sfa + 8), ra[0].z, ra[1].z, ra[2].z, ra[3].z);
      tmem_st4(lane_addr | (sfa + 12), ra[0].w, ra[1].w, ra[2].w, ra[3].w);
      tmem_st4(lane_addr | (sfb + 0), rb[0].x, rb[1].x, rb[2].x, rb[3].x);
      tmem_st4(lane_addr | (sfb + 4), rb[0].y, rb[1].y, rb[2].y, rb[3].y);
      tmem_st4(lane_addr | (sfb + 8), rb[0].z, rb[1].z, rb[2].z, rb[3].z);
      tmem_st4(lane_addr | (sfb + 12), rb[0].w, rb[1].w, rb[2].w, rb[3].w);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sf_full[slot]);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int et = threadIdx.x - 192;   // 0..127 within the epilogue warps
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    const int row = 32 * q + lane;      // accumulator row (A-tile row)
    const long long first_tile = s_begin / L;
    const long long last_tile = s_begin < s_end ? (s_end - 1) / L : first_tile - 1;
    int buf = 0, seen = 0;
    for (long long tile = first_tile; tile <= last_tile; tile++) {
      const bool got = mbar_wait_bounded(&acc_full[buf], (seen / 2) & 1, a.err, 0x8000u);
      if (!epi_all(got && !*abort_flag)) break;
      tc_fence_after();
      StageMeta m;
      decode_stage<MODE>(tile * L, L, ntm, kst, m);
      m.e = __ldg(a.ch_expert + m.c);
      m.p0 = __ldg(a.ch_pos + m.c);
      m.n = __ldg(a.ch_n + m.c);
      m.nb = (4 * m.n + 7) / 8;
      if (MODE == kModeDownOne) {  // K runs over every chunk; the output is the one token
        m.n = 1;
        m.nb = 1;
      }
      float v[32];
      const uint32_t dacc = tbase + buf * kMtAccCols;
      for (int c0 = 0; c0 < 8 * m.nb; c0 += 8) {
        float r[8];
        tmem_ld8(dacc + lane_addr + c0, r);
        v[c0 / 4] = ((r[0] + r[1]) + r[2]) + r[3];
        v[c0 / 4 + 1] = ((r[4] + r[5]) + r[6]) + r[7];
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      buf ^= 1;
      seen++;
      // ---- whole tile here, or the last of its parts?
      const long long ts = static_cast<long long>(m.tile) * L, te = ts + L;
      const bool whole = ts >= s_begin && te <= s_end;
      (void)et;
      if (!whole) {
        const int slot2 = (m.tile == first_tile) ? 0 : 1;
        float* pp = a.partial + (static_cast<size_t>(blockIdx.x) * 2 + slot2) * 32 * 128;
        for (int t = 0; t < m.n; t++) pp[t * 128 + row] = v[t];
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (et == 0) {
          const int c0 = cta_of(ts, total, grid), c1 = cta_of(te - 1, total, grid);
          const int old = atomicAdd(a.tile_cnt + m.tile, 1);
          *last_flag = old == c1 - c0;
          if (old == c1 - c0) a.tile_cnt[m.tile] = 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!*last_flag) continue;
        __threadfence();
        const int c0 = cta_of(ts, total, grid), c1 = cta_of(te - 1, total, grid);
        for (int t = 0; t < m.n; t++) v[t] = 0.0f;
        for (int cc = c0; cc <= c1; cc++) {
          const long long fb = total * cc / grid;
          const int sl = (m.tile == fb / L) ? 0 : 1;
          const float* qp = a.partial + (static_cast<size_t>(cc) * 2 + sl) * 32 * 128;
          for (int t = 0; t < m.n; t++) v[t] += __ldcg(qp + t * 128 + row);
        }
      }
      // ---- finalize
      if (MODE == kModeGateUp) {
        // rows 0..63 gate, 64..127 up (of inter rows m*64 ..): h = silu(g) u w
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (q >= 2)
          for (int t = 0; t < m.n; t++) ubuf[t * 64 + (row - 64)] = v[t];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (q < 2) {
          const int i0 = m.m * 64 + 32 * q;  // first inter index of this warp's 32-block
          for (int t = 0; t < m.n; t++) {
            const int p = m.p0 + t;
            float hv = __fmul_rn(silu_ref(v[t]), ubuf[t * 64 + row]);
            hv *= __ldg(a.perm_w + p);
            const size_t trow = static_cast<size_t>(4 * p);
            warp_terms4(hv, a.ht + trow * (a.inter / 2) + i0 / 2, a.inter / 2,
                        a.hsf + trow * (a.inter / 32) + i0 / 32, a.inter / 32);
          }
        }
      } else if (MODE == kModeDown) {
        const int orow = m.m * 128 + row;
        for (int t = 0; t < m.n; t++) a.y[static_cast<size_t>(m.p0 + t) * a.hidden + orow] = v[t];
      } else {
        a.y[m.m * 128 + row] = v[0];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kMtTmemCols);
  }
}

// ---------------------------------------------------------------------- activation terms per position
// xt rows 4p..4p+3 = terms of x[perm_tok[p]]; one warp per (position, 32-block).
__global__ void __launch_bounds__(256) terms_by_position_kernel(const void* __restrict__ x, int x_dtype, int H,
                                                                const int32_t* __restrict__ perm_tok,
                                                                const int32_t* __restrict__ n_pos, int P_bound,
                                                                uint8_t* __restrict__ xt, uint8_t* __restrict__ xsf) {
  const int nb = H / 32;
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (wid >= P_bound * nb) return;
  const int p = wid / nb, b = wid % nb;
  if (p >= *n_pos) return;
  const int tok = perm_tok[p];
  const float r = load_elem(x, x_dtype, static_cast<size_t>(tok) * H + b * 32 + lane);
  warp_terms4(r, xt + static_cast<size_t>(4 * p) * (H / 2) + b * 16, H / 2, xsf + static_cast<size_t>(4 * p) * nb + b, nb);
}

// ---------------------------------------------------------------------- host side
bool make_tmap_sw128(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);
bool make_tmap_rows(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                    uint32_t box_rows);

struct MoeTcPlanImpl {
  MoeTcMaps gu, dn;
};

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

bool moe_tc_supported(int H, int I, int Is, int fmt) {
  return fmt == kMxfp4 && H % kMtKStage == 0 && H % 128 == 0 && I % kMtKStage == 0 && I % 64 == 0 &&
         (Is == 0 || Is == I);
}

size_t moe_tc_plan_bytes() { return sizeof(MoeTcPlanImpl); }

// Tensor maps of one layer (built once: every pointer is fixed at layer creation).
bool moe_tc_plan(void* plan, const uint8_t* arena, size_t stride, int n_slots, size_t off_gate, size_t off_up,
                 size_t off_down, size_t off_gs, size_t off_us, size_t off_ds, int H, int I, const uint8_t* xt,
                 const uint8_t* xsf, const uint8_t* ht, const uint8_t* hsf, int term_rows) {
  MoeTcPlanImpl* p = static_cast<MoeTcPlanImpl*>(plan);
  const uint64_t bytes = stride * static_cast<uint64_t>(n_slots);
  bool ok = true;
  ok = ok && make_tmap_sw128(&p->gu.a0, arena + off_gate, H / 2, (bytes - off_gate) / (H / 2), 64);
  ok = ok && make_tmap_sw128(&p->gu.a1, arena + off_up, H / 2, (bytes - off_up) / (H / 2), 64);
  ok = ok && make_tmap_rows(&p->gu.s0, arena + off_gs, H / 32, (bytes - off_gs) / (H / 32), 16, 64);
  ok = ok && make_tmap_rows(&p->gu.s1, arena + off_us, H / 32, (bytes - off_us) / (H / 32), 16, 64);
  ok = ok && make_tmap_sw128(&p->gu.b, xt, H / 2, term_rows, 8);
  ok = ok && make_tmap_rows(&p->gu.bs, xsf, H / 32, term_rows, 16, 8);
  ok = ok && make_tmap_sw128(&p->dn.a0, arena + off_down, I / 2, (bytes - off_down) / (I / 2), 64);
  p->dn.a1 = p->dn.a0;
  ok = ok && make_tmap_rows(&p->dn.s0, arena + off_ds, I / 32, (bytes - off_ds) / (I / 32), 16, 64);
  p->dn.s1 = p->dn.s0;
  ok = ok && make_tmap_sw128(&p->dn.b, ht, I / 2, term_rows, 8);
  ok = ok && make_tmap_rows(&p->dn.bs, hsf, I / 32, term_rows, 16, 8);
  return ok;
}

cudaError_t launch_terms_by_position(const void* x, int x_dtype, int H, const int32_t* perm_tok,
                                     const int32_t* n_pos, int P_bound, uint8_t* xt, uint8_t* xsf,
                                     cudaStream_t st) {
  if (P_bound <= 0) return cudaSuccess;
  const int n = P_bound * (H / 32) * 32;
  terms_by_position_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, x_dtype, H, perm_tok, n_pos, P_bound, xt, xsf);
  return cudaGetLastError();
}

static size_t moe_tc_smem(int stages, int b_boxes) {
  return 1024 + static_cast<size_t>(mt_layout(stages, b_boxes).total);
}

// mode: 0 gate/up, 1 down, 2 down for one token. mt = positions per chunk (<= 32).
cudaError_t launch_moe_tc(int mode, const void* plan, const DispatchBuffers& d, int mt, int H, int I,
                          size_t stride, uint8_t* ht, uint8_t* hsf, float* y, float* partial,
                          int32_t* tile_cnt, unsigned* err, cudaStream_t st, const int32_t* b_token_rows) {
  const MoeTcPlanImpl* p = static_cast<const MoeTcPlanImpl*>(plan);
  MoeTcArgs a{};
  a.ch_expert = d.ch_expert; a.ch_pos = d.ch_pos; a.ch_n = d.ch_n; a.n_chunks = d.n_chunks;
  a.perm_w = d.perm_w;
  a.K = mode == 0 ? H : I;
  a.out_rows = mode == 0 ? I : H;
  a.rows_per_expert_data = static_cast<int>(stride / (a.K / 2));
  a.rows_per_expert_sf = static_cast<int>(stride / (a.K / 32));
  a.b_boxes = (4 * mt + 7) / 8;
  a.ht = ht; a.hsf = hsf; a.inter = I;
  a.y = y; a.hidden = H;
  a.partial = partial; a.tile_cnt = tile_cnt; a.err = err;
  a.b_tok = b_token_rows;
  int stages = kMtMaxStages;
  while (stages > 2 && moe_tc_smem(stages, a.b_boxes) > 227 * 1024) stages--;
  a.stages = stages;
  const size_t smem = moe_tc_smem(stages, a.b_boxes);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  const MoeTcMaps& maps = mode == 0 ? p->gu : p->dn;
  const int grid = sm_count();
  cudaError_t e;
  switch (mode) {
    case 0:
      e = cudaFuncSetAttribute(moe_tc_kernel<kModeGateUp>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      moe_tc_kernel<kModeGateUp><<<grid, kMtThreads, smem, st>>>(maps, a);
      break;
    case 1:
      e = cudaFuncSetAttribute(moe_tc_kernel<kModeDown>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      moe_tc_kernel<kModeDown><<<grid, kMtThreads, smem, st>>>(maps, a);
      break;
    default:
      e = cudaFuncSetAttribute(moe_tc_kernel<kModeDownOne>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      moe_tc_kernel<kModeDownOne><<<grid, kMtThreads, smem, st>>>(maps, a);
      break;
  }
  return cudaGetLastError();
}

}  // namespace rmoe
