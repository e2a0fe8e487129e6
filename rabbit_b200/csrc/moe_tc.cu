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

constexpr int kMtThreads = 352;
constexpr int kMtKStage = 512;            // K elements per stage (two 128-byte swizzle columns)
constexpr int kMtMaxStages = 6;
constexpr int kMtAccCols = 128;           // one accumulator: N <= 128 (32 positions x 4 terms)
constexpr int kMtSfCols = 32;             // per stage: 16 columns of A scales + 16 of B scales
constexpr uint32_t kMtTmemCols = 512;

enum { kModeGateUp = 0, kModeDown = 1, kModeDownOne = 2 };

struct MoeTcMaps {
  CUtensorMap b;     // activation terms (box 128 B x 8 rows, SW128)
  CUtensorMap bs;    // their scale rows (box 16 B x 8 rows)
  CUtensorMap b128;  // the same with 128-row boxes (chunks of up to 32 positions)
  CUtensorMap bs128;
};

// Expert weights of a tensor-core layer are stored tile-major: for each 128-row tile m and
// 512-column stage ks one block of kTileBlock bytes =
//   [2 x 16 KB: 128 rows x 128 B of E2M1 for columns 256 h .. 256 h + 255 of the stage, each row's
//    16-byte chunk c at chunk position c ^ (row & 7) (the 128-byte swizzle image)]
//   [2 KB of E8M0 words: word (g * 128 + L * 4 + j) = scales of k-blocks 4g..4g+3 of row L + 32 j,
//    i.e. per k-group g a 32 x 16-byte block that one tcgen05.cp places in TMEM as the MMA reads it]
// GATE_UP tiles hold gate rows 64m..64m+63 then the same up rows; DOWN tiles down rows 128m...
// A stage is then one contiguous bulk copy, already in the shape the MMA and TMEM want.
constexpr int kTileBlock = 32768 + 2048;

struct MoeTcArgs {
  const int32_t* ch_expert;
  const int32_t* ch_pos;
  const int32_t* ch_n;
  const int32_t* n_chunks;
  const float* perm_w;
  int K;               // reduction length of one expert (GATE_UP: hidden, DOWN: inter)
  int out_rows;        // GATE_UP: inter; DOWN: hidden
  const uint8_t* wbase; // tile blocks of expert slot 0 for this projection
  size_t wstride;       // bytes between expert slots
  int b_boxes;         // activation boxes (8 rows) reserved per stage
  int stages;          // ring depth
  uint8_t* ht;         // GATE_UP out: h terms [4P][inter/2]
  uint8_t* hsf;        // GATE_UP out: their scales [4P][inter/32]
  int inter;           // GATE_UP: row pitch source of ht / hsf
  float* y;            // DOWN: [P][hidden]; DOWN_ONE: [hidden]
  int hidden;
  float* partial;      // [units][8][128] unit parts of split tiles
  int32_t* tile_cnt;   // parts finished per tile (reset by the finishing CTA)
  unsigned* err;
  const int32_t* b_tok;  // non-null (one position per chunk): B rows are the token's, 4 * b_tok[p0]
  unsigned long long* trace;  // optional: CTA 0's per-stage timestamps [stage][4] (ns)
  int* work;           // [4] units claimed, CTAs finished, h slices ready, parts stored (zero between launches)
  int unit_stages;     // stages per claimed unit (split tiles when smaller than a tile)
  ActParams act;       // gating activation (gate/up epilogue, h from the parts)
  // gate/up with split tiles: parts stored per tile (each part released on this counter; the
  // last CTA out zeroes them); the CTAs' idle warps form h of a tile once all its parts are in
  int* gu_tile_cnt;
  int* h_done;         // gate/up: h items finished (released per item; the down kernel's counter)
  int h_split;         // down: gate/up split its tiles, its helper warps write h (wait on h_done)
  int weights_once;    // every weight tile is read by one unit only (one chunk per expert): evict-first
  unsigned long long spin_ns;  // limit of each wait on another CTA's counter (then err, abort)
};

struct StageMeta {
  int nb, pad0, pad1, pad2;
};

// One unit of work as handed from the weight producer to the other roles.
struct PartRec {
  int tile;   // -1: no more work
  int uit;    // unit index inside the tile
  int unit;   // global unit id
  int e;      // expert slot of the unit's first stage
  int p0;     // first position of the tile's chunk
  int n;      // positions in the chunk
  int brow;   // first activation row of the chunk (4 * token or 4 * position)
  int pad;
};
constexpr int kRecRing = 4;

constexpr int kBOff = (kTileBlock + 1023) & ~1023;

// Shared-memory carve-up (offsets from the 1024-aligned base).
struct MtLayout {
  int stage_pitch, off_bar, off_meta, off_rec, off_misc, off_ubuf, total;
};
__host__ __device__ inline MtLayout mt_layout(int stages, int b_boxes) {
  MtLayout l;
  // [A tile + its scales: kTileBlock][pad to 1 KB][B: 2 x b_boxes KB][B scales: b_boxes x 128 B]
  const int sb = kBOff + 2 * b_boxes * 1024 + b_boxes * 128;
  l.stage_pitch = (sb + 1023) & ~1023;
  l.off_bar = stages * l.stage_pitch;  // 5 * stages + 8 + 2 * kRecRing mbarriers
  l.off_meta = l.off_bar + (5 * stages + 8 + 2 * kRecRing) * 8;
  l.off_rec = l.off_meta + stages * static_cast<int>(sizeof(StageMeta));
  l.off_misc = (l.off_rec + kRecRing * static_cast<int>(sizeof(PartRec)) + 15) & ~15;
  // tmem slot, abort, last flag, pad, then two drain mbarriers (tc_drain)
  l.off_ubuf = (l.off_misc + 32 + 15) & ~15;
  l.total = l.off_ubuf + 128 * 33 * 4;  // [128 tile rows][32 positions] (+1 pad)
  return l;
}

// Release increment without a returned value: the issuing thread does not wait for its earlier
// stores (nor, through the preceding barrier, its CTA's) to be performed, unlike a full fence.
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
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

// Gate/up with split tiles: h of one (tile, 32 inter rows) item from the tile's unit parts, once
// all of them are in (the tile's counter, released per part, reaches the units per tile):
// parts added in K order (loads issued four at a time), h = act(g, u) w, written as the four-term
// operand of the down GEMM. One warp.
__device__ __forceinline__ void h_item(const MoeTcArgs& a, int it, int ntm, int upt, unsigned* err, int lane) {
  const int tile = it / 2, hf = it % 2;
  const int c = tile / ntm, m = tile % ntm;
  const int p0 = __ldg(a.ch_pos + c), n = __ldg(a.ch_n + c);
  const int i0 = m * 64 + hf * 32;
  bool ready = true;
  if (lane == 0) {
    const uint64_t t0 = global_ns();
    while (ld_acquire_gpu(a.gu_tile_cnt + tile) < upt) {
      if (global_ns() - t0 > a.spin_ns) {
        atomicOr(err, 0x80000u);
        ready = false;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!__shfl_sync(kFull, ready, 0)) return;
  __syncwarp();
  for (int t = 0; t < n; t++) {
    const float* base = a.partial + static_cast<size_t>(tile) * upt * 8 * 128 + t * 128 + hf * 32 + lane;
    float g = 0.0f, u = 0.0f;
    int j = 0;
    for (; j + 4 <= upt; j += 4) {
      float gg[4], uu[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        gg[q] = __ldcg(base + static_cast<size_t>(j + q) * 8 * 128);
        uu[q] = __ldcg(base + static_cast<size_t>(j + q) * 8 * 128 + 64);
      }
#pragma unroll
      for (int q = 0; q < 4; q++) {
        g += gg[q];
        u += uu[q];
      }
    }
    for (; j < upt; j++) {
      g += __ldcg(base + static_cast<size_t>(j) * 8 * 128);
      u += __ldcg(base + static_cast<size_t>(j) * 8 * 128 + 64);
    }
    const int p = p0 + t;
    const float hv = act_gate(a.act.kind, a.act.beta, a.act.linear_beta, g, u, false) * __ldg(a.perm_w + p);
    const size_t trow = static_cast<size_t>(4 * p);
    warp_terms4(hv, a.ht + trow * (a.inter / 2) + i0 / 2, a.inter / 2, a.hsf + trow * (a.inter / 32) + i0 / 32,
                a.inter / 32);
  }
}

// Walks consecutive stages of the flat list (tile-major, L stages per tile) from stage s.
template <int MODE>
struct StageWalker {
  int u, c, m, ks, L, ntm, kst;
  __device__ __forceinline__ void init(int s, int L_, int ntm_, int kst_) {
    L = L_; ntm = ntm_; kst = kst_;
    const int tile = s / L;
    u = s % L;
    if (MODE == kModeDownOne) {
      m = tile;
      c = u / kst;
      ks = u % kst;
    } else {
      c = tile / ntm;
      m = tile % ntm;
      ks = u;
    }
  }
  __device__ __forceinline__ void next() {
    u++;
    if (MODE == kModeDownOne) {
      if (++ks == kst) { ks = 0; c++; }
      if (u == L) { u = 0; ks = 0; c = 0; m++; }
    } else {
      ks = u;
      if (u == L) { u = 0; ks = 0; if (++m == ntm) { m = 0; c++; } }
    }
  }
};

// Work is claimed dynamically: unit = U consecutive stages of one tile (U divides L), claimed in
// increasing order from a device counter, so SMs that stream faster take more units. A tile cut
// into several units is accumulated per unit; the CTA finishing the tile's last unit adds the
// unit parts in K order (deterministic). The last CTA to exit resets the counters.
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
  uint64_t* bfull = empty + S;          // activation operand of the stage landed
  uint64_t* acc_full = bfull + S;       // [4]
  uint64_t* acc_empty = acc_full + 4;   // [4]
  uint64_t* rec_full = acc_empty + 4;   // [kRecRing]
  uint64_t* rec_empty = rec_full + kRecRing;
  uint64_t* sfa_done = rec_empty + kRecRing;  // [S] A's scale factors copied into TMEM
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + lay.off_meta);
  PartRec* recs = reinterpret_cast<PartRec*>(smem + lay.off_rec);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + lay.off_misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* drain = reinterpret_cast<uint64_t*>(smem + lay.off_misc + 16);  // [2] one-use (tc_drain)
  volatile int* last_flag = abort_flag + 1;
  float* ubuf = reinterpret_cast<float*>(smem + lay.off_ubuf);  // [32][64] up values (GATE_UP)

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (a.trace && threadIdx.x == 0) a.trace[1024 + 4 * blockIdx.x] = global_ns();

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&sf_full[i], 128);
      mbar_init(&empty[i], 1);
      mbar_init(&bfull[i], 1);
      mbar_init(&sfa_done[i], 1);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    for (int i = 0; i < kRecRing; i++) {
      mbar_init(&rec_full[i], 1);
      mbar_init(&rec_empty[i], 2 + 128 + 128);  // activation producer, MMA issuer, epilogue, scale warps
    }
    *abort_flag = 0;
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kMtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  // Launched with programmatic stream serialization this kernel may start while the previous
  // one (gate/up: the front end or the activation terms; down: gate/up) still runs. Gate/up
  // reads that kernel's routing and terms from the start and waits here; the down kernels read
  // only data of the kernel before gate/up (routing, dispatch: complete once gate/up passed its
  // own wait) until the h operand, which the roles needing it wait for below; their weight
  // stream starts at once.
  if (MODE == kModeGateUp) griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  const int nch = *a.n_chunks;
  const int kst = a.K / kMtKStage;
  const int ntm = MODE == kModeGateUp ? a.out_rows / 64 : a.out_rows / 128;
  const int L = MODE == kModeDownOne ? max(1, nch * kst) : kst;
  const int U = a.unit_stages < L && L % a.unit_stages == 0 ? a.unit_stages : L;
  const int upt = L / U;  // units per tile
  const int ntiles = MODE == kModeDownOne ? ntm : nch * ntm;
  const int total_units = ntiles * upt;
  // accumulators: N <= 8 * b_boxes columns each; four when they fit in 256 columns
  const int acc_cols = ((8 * a.b_boxes + 31) / 32) * 32;
  const int nacc = acc_cols <= 64 ? 4 : 2;
  const uint32_t sf_base = tbase + 256;
  if (a.trace && threadIdx.x == 0) a.trace[1024 + 4 * blockIdx.x + 1] = global_ns();

  if (warp == 0) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      int slot = 0, ph = 0, rslot = 0, rph = 0, issued = 0;
      int cc = -1, ce = 0, cn = 0;  // chunk fields of the current stage
      // the first unit is this CTA's own (unit blockIdx.x); later ones are claimed from the
      // counter, which therefore hands out units gridDim.x, gridDim.x + 1, ...
      int unit = blockIdx.x;
      int ue = 0, up0 = 0, un = 0, ubr = 0;
      auto chunk_of = [&](int u, int& c) {  // chunk of the unit's first stage
        const int t = u / upt;
        c = MODE == kModeDownOne ? ((u % upt) * U) / kst : t / ntm;
      };
      auto load_unit = [&](int u) {
        if (u >= total_units) return;
        int c;
        chunk_of(u, c);
        ue = __ldg(a.ch_expert + c);
        up0 = __ldg(a.ch_pos + c);  // (one token: the position the unit's K run starts on)
        un = MODE == kModeDownOne ? 1 : __ldg(a.ch_n + c);
        ubr = 4 * (a.b_tok ? __ldg(a.b_tok + up0) : up0);
      };
      if (a.trace && blockIdx.x == 0) a.trace[1700] = global_ns();
      load_unit(unit);
      if (a.trace && blockIdx.x == 0) a.trace[1701] = global_ns();
      for (int part = 0;; part++) {
        const bool stop = unit >= total_units || *abort_flag;
        int nxt = unit;  // next claim: made after this unit's first stage is issued
        if (part >= kRecRing && !mbar_wait_bounded(&rec_empty[rslot], rph ^ 1, a.err, 0x10u)) {
          *abort_flag = 1;
          break;
        }
        PartRec& r = recs[rslot];
        r.tile = stop ? -1 : unit / upt;
        r.uit = stop ? 0 : unit % upt;
        r.unit = unit;
        r.e = ue;
        r.p0 = up0;
        r.n = un;
        r.brow = ubr;
        mbar_arrive(&rec_full[rslot]);
        if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
        if (stop) break;
        StageWalker<MODE> w;
        w.init((unit / upt) * L + (unit % upt) * U, L, ntm, kst);
        cc = w.c;
        ce = ue;
        cn = un;
        for (int j = 0; j < U; j++, w.next(), issued++) {
          if (issued >= S && !mbar_wait_bounded(&empty[slot], ph ^ 1, a.err, 0x100u)) {
            *abort_flag = 1;
            break;
          }
          if (w.c != cc) {  // (one token: the K run crosses experts inside a tile)
            cc = w.c;
            ce = __ldg(a.ch_expert + cc);
          }
          meta[slot].nb = MODE == kModeDownOne ? 1 : (4 * cn + 7) / 8;
          uint8_t* st = smem + slot * stage_pitch;
          if (a.trace && blockIdx.x == 0 && issued < 256) a.trace[issued * 4 + 0] = global_ns();
          mbar_arrive_expect_tx(&full[slot], kTileBlock);
          const uint8_t* blk = a.wbase + static_cast<size_t>(ce) * a.wstride +
                               (static_cast<size_t>(w.m) * kst + w.ks) * kTileBlock;
          if (a.weights_once)
            bulk_g2s_once(st, blk, kTileBlock, &full[slot]);
          else
            bulk_g2s(st, blk, kTileBlock, &full[slot]);
          if (++slot == S) { slot = 0; ph ^= 1; }
          if (j == 0) {  // claim the next unit and load its fields while this one streams
            nxt = static_cast<int>(gridDim.x) + atomicAdd(a.work, 1);
            load_unit(nxt);
          }
        }
        // (after an abort the loop's next pass publishes an end record in ring order: a record
        // is never rewritten while a consumer may still be reading it)
        unit = nxt;
      }
      // copies still landing (only after an abort) finish before the CTA exits
      for (int i = (issued > S ? issued - S : 0); i < issued; i++)
        mbar_wait_bounded(&full[i % S], (i / S) & 1, a.err, 0x200u);
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------------ activation producer
    if (lane == 0) {
      if (MODE != kModeGateUp) {
        // the activation operand is h, written by gate/up with plain stores: for split tiles by
        // its helper warps, each finished item released on this kernel's work[2] (acquired here,
        // without waiting for gate/up's whole grid to complete); else by its epilogue (grid wait)
        if (a.h_split) {
          const int items = 2 * nch * (a.inter / 64);
          const uint64_t t0 = global_ns();
          while (ld_acquire_gpu(a.work + 2) < items) {
            if (global_ns() - t0 > a.spin_ns) {
              atomicOr(a.err, 0x40000u);
              *abort_flag = 1;
              break;
            }
            __nanosleep(32);
          }
        } else {
          griddep_wait();
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      if (a.trace && blockIdx.x == 0) a.trace[1720] = global_ns();
      tma_prefetch_desc(&maps.b);
      tma_prefetch_desc(&maps.bs);
      int slot = 0, ph = 0, rslot = 0, rph = 0, issued = 0;
      for (;;) {
        if (!mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x20u)) break;
        const PartRec r = recs[rslot];
        mbar_arrive(&rec_empty[rslot]);
        if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
        if (r.tile < 0 || *abort_flag) break;
        StageWalker<MODE> w;
        w.init(r.tile * L + r.uit * U, L, ntm, kst);
        const int nb = MODE == kModeDownOne ? 1 : (4 * r.n + 7) / 8;
        int brow0 = r.brow, cc = w.c;
        bool ok = true;
        for (int j = 0; j < U; j++, w.next(), issued++) {
          if (issued >= S && !mbar_wait_bounded(&empty[slot], ph ^ 1, a.err, 0x100u)) {
            ok = false;
            break;
          }
          if (MODE == kModeDownOne && w.c != cc) {  // the K run moved to the next position
            cc = w.c;
            const int p = __ldg(a.ch_pos + cc);
            brow0 = 4 * (a.b_tok ? __ldg(a.b_tok + p) : p);
          }
          uint8_t* sb = smem + slot * stage_pitch + kBOff;
          uint8_t* ssb = sb + 2 * bsub;
          const int kx = w.ks * (kMtKStage / 2);       // byte column of this stage in a B row
          const int ksf = w.ks * (kMtKStage / 32);     // scale byte column
          if (a.b_boxes == 16) {
            // up to 32 positions: one 128-row box per column (rows past the chunk are not used)
            mbar_arrive_expect_tx(&bfull[slot], 2 * 16384 + 2048);
            tma_load_2d(sb, &maps.b128, kx, brow0, &bfull[slot]);
            tma_load_2d(sb + bsub, &maps.b128, kx + 128, brow0, &bfull[slot]);
            tma_load_2d(ssb, &maps.bs128, ksf, brow0, &bfull[slot]);
          } else {
            mbar_arrive_expect_tx(&bfull[slot], nb * (2 * 1024 + 128));
            for (int bx = 0; bx < nb; bx++) {
              const int brow = brow0 + 8 * bx;
              tma_load_2d(sb + bx * 1024, &maps.b, kx, brow, &bfull[slot]);
              tma_load_2d(sb + bsub + bx * 1024, &maps.b, kx + 128, brow, &bfull[slot]);
              tma_load_2d(ssb + bx * 128, &maps.bs, ksf, brow, &bfull[slot]);
            }
          }
          if (++slot == S) { slot = 0; ph ^= 1; }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      for (int i = (issued > S ? issued - S : 0); i < issued; i++)
        mbar_wait_bounded(&bfull[i % S], (i / S) & 1, a.err, 0x200u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int i = 0, buf = 0, parts = 0, rslot = 0, rph = 0;
      bool ok = true;
      const uint64_t da0 = sw128_desc(smem), db0 = sw128_desc(smem + kBOff);  // slot 0
      for (;;) {
        if (!mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x20u)) break;
        const int tile = recs[rslot].tile;
        mbar_arrive(&rec_empty[rslot]);
        if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
        if (tile < 0 || *abort_flag) break;
        if (parts >= nacc && !mbar_wait_bounded(&acc_empty[buf], ((parts / nacc) - 1) & 1, a.err, 0x1000u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tbase + buf * acc_cols;
        for (int j = 0; j < U && ok; j++, i++) {
          const int slot = i % S;
          const uint32_t ph = (i / S) & 1;
          if (a.trace && blockIdx.x == 0 && i < 256) a.trace[i * 4 + 2] = global_ns();
          // both operands' scale factors in TMEM: A's copies committed to sfa_done (issued
          // once the stage's data landed), B's stores behind sf_full (after the B operand landed)
          if (!mbar_wait_bounded(&sfa_done[slot], ph, a.err, 0x800u) ||
              !mbar_wait_bounded(&sf_full[slot], ph, a.err, 0x800u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // operands of the stage's 8 MMAs computed first, then issued back to back
          const uint64_t da = da0 + static_cast<uint64_t>((slot * stage_pitch) >> 4);
          const uint64_t db = db0 + static_cast<uint64_t>((slot * stage_pitch) >> 4);
          const uint32_t idesc = mxf4_idesc(8 * meta[slot].nb);
          const uint32_t sfa = sf_base + slot * kMtSfCols, sfb = sfa + 16;
          uint64_t dak[8], dbk[8];
          uint32_t idk[8], sak[8], sbk[8];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const uint32_t adv = (32 * (k & 3)) >> 4;
            dak[k] = da + ((k >> 2) * (16384 >> 4) + adv);
            dbk[k] = db + ((k >> 2) * (bsub >> 4) + adv);
            const uint32_t sid = static_cast<uint32_t>(2 * (k & 1));
            sak[k] = (sfa + 4 * (k >> 1)) | (sid << 30);
            sbk[k] = (sfb + 4 * (k >> 1)) | (sid << 30);
            idk[k] = idesc | (sid << 29) | (sid << 4);
          }
          const uint32_t acc0 = j == 0 ? 0u : 1u;
#pragma unroll
          for (int k = 0; k < 8; k++) mma_mxf4_run(dacc, dak[k], dbk[k], idk[k], sak[k], sbk[k], k == 0 ? acc0 : 1u);
          tc_commit(&empty[slot]);
          if (a.trace && blockIdx.x == 0 && i < 256) a.trace[i * 4 + 3] = global_ns();
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
        if (++buf == nacc) buf = 0;
        parts++;
      }
      if (!ok) *abort_flag = 1;
      tc_drain(&drain[0], a.err);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ B scale factors -> TMEM
    const int q = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    int i = 0, rslot = 0, rph = 0;
    bool ok = true;
    while (ok) {
      if (!__all_sync(kFull, mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x40u))) break;
      const int tile = __shfl_sync(kFull, recs[rslot].tile, 0);  // (one value for the warp)
      mbar_arrive(&rec_empty[rslot]);
      if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
      if (tile < 0) break;
      for (int j = 0; j < U; j++, i++) {
        const int slot = i % S;
        // (every exit below is decided warp-wide: the TMEM stores are .sync.aligned)
        if (q == 2) {
          // A's scale factors: each k-group's 32 x 16-byte block straight into TMEM
          bool got = lane != 0 || mbar_wait_bounded(&full[slot], (i / S) & 1, a.err, 0x4000u);
          got = __shfl_sync(kFull, got, 0);
          if (!got) {
            ok = false;
            break;
          }
          if (lane == 0) {
            tc_fence_after();
            const uint8_t* ssa = smem + slot * stage_pitch + 32768;
            const uint32_t sfa = sf_base + slot * kMtSfCols;
#pragma unroll
            for (int g = 0; g < 4; g++) tmem_cp_rows16_x4(sfa + 4 * g, rows16_desc(ssa + g * 512));
            tc_commit(&sfa_done[slot]);  // the MMA issuer waits for it; this warp runs ahead
          }
          __syncwarp();
        }
        const bool gotb = mbar_wait_bounded(&bfull[slot], (i / S) & 1, a.err, 0x4000u) && !*abort_flag;
        if (!__all_sync(kFull, gotb)) {
          ok = false;
          break;
        }
        if (a.trace && blockIdx.x == 0 && i < 256 && q == 0 && lane == 0) a.trace[i * 4 + 1] = global_ns();
        const uint8_t* ssb = smem + slot * stage_pitch + kBOff + 2 * bsub;
        // every row the stage buffer holds (rows past the chunk's are never read by the MMA);
        // meta[] is not read here: only the weight producer's barrier orders its writes
        const int nrows_b = 8 * a.b_boxes;
        const uint32_t sfb = sf_base + slot * kMtSfCols + 16;
        uint4 rb[4];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
          const int n = lane + 32 * jj;
          rb[jj] = n < nrows_b ? *reinterpret_cast<const uint4*>(ssb + n * 16) : make_uint4(0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
        }
        tmem_st4(lane_addr | (sfb + 0), rb[0].x, rb[1].x, rb[2].x, rb[3].x);
        tmem_st4(lane_addr | (sfb + 4), rb[0].y, rb[1].y, rb[2].y, rb[3].y);
        tmem_st4(lane_addr | (sfb + 8), rb[0].z, rb[1].z, rb[2].z, rb[3].z);
        tmem_st4(lane_addr | (sfb + 12), rb[0].w, rb[1].w, rb[2].w, rb[3].w);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sf_full[slot]);
      }
    }
    if (q == 2 && lane == 0) tc_drain(&drain[1], a.err);  // (its scale-factor copies)
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int et = threadIdx.x - 192;   // 0..127 within the epilogue warps
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    const int row = 32 * q + lane;      // accumulator row (A-tile row)
    int buf = 0, seen = 0, rslot = 0, rph = 0;
    for (;;) {
      const bool gotr = mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x40u);
      if (!epi_all(gotr)) break;
      const PartRec r = recs[rslot];
      mbar_arrive(&rec_empty[rslot]);
      if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
      const unsigned long long e0 = a.trace && blockIdx.x == 0 ? global_ns() : 0;
      // (the end record and every exit are decided by all 128 threads together)
      const bool got = r.tile >= 0 && mbar_wait_bounded(&acc_full[buf], (seen / nacc) & 1, a.err, 0x8000u);
      if (!epi_all(got && !*abort_flag)) break;
      if (a.trace && blockIdx.x == 0 && et == 0 && seen < 128) {
        a.trace[3072 + seen * 4 + 0] = e0;
        a.trace[3072 + seen * 4 + 1] = global_ns();
        a.trace[3072 + seen * 4 + 3] = r.tile * 16 + r.uit;
      }
      tc_fence_after();
      const int mm = MODE == kModeDownOne ? r.tile : r.tile % ntm;
      const int p0 = r.p0;
      const int n = r.n;
      const int nb = (4 * n + 7) / 8;
      float v[32];
      const bool tr2 = MODE == kModeGateUp && a.trace && blockIdx.x == 0 && et == 64 && seen < 128;
      if (tr2) a.trace[3584 + seen * 4 + 0] = global_ns();
      const uint32_t dacc = tbase + buf * acc_cols;
      for (int c0 = 0; c0 < 8 * nb; c0 += 32) {  // (columns past 8 * nb are read, never used)
        float rr[32];
        tmem_ld32(dacc + lane_addr + c0, rr);
#pragma unroll
        for (int i = 0; i < 8; i++) v[c0 / 4 + i] = ((rr[4 * i] + rr[4 * i + 1]) + rr[4 * i + 2]) + rr[4 * i + 3];
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      if (++buf == nacc) buf = 0;
      seen++;
      if (upt > 1) {
        // one unit of a split tile: store its part; the parts are added in K order by the pass
        // that needs the tile (the down kernel's prologue for gate/up, the end of this kernel
        // for the one-token down projection)
        float* pp = a.partial + static_cast<size_t>(r.unit) * 8 * 128;
        if (a.trace && blockIdx.x == 0 && et == 0 && seen <= 4) a.trace[1710 + seen] = global_ns();
        for (int t = 0; t < n; t++) pp[t * 128 + row] = v[t];
        if (MODE == kModeGateUp && a.gu_tile_cnt) {
          // the part is in: count it for its tile (a release that nothing here waits for)
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (et == 0) red_release_gpu_add(a.gu_tile_cnt + r.tile, 1);
        }
        if (a.trace && blockIdx.x == 0 && et == 0 && seen <= 128) a.trace[3072 + (seen - 1) * 4 + 2] = global_ns();
        continue;
      }
      // ---- finalize
      if (MODE == kModeGateUp) {
        // rows 0..63 gate, 64..127 up (inter rows mm*64 ..): the tile goes through shared memory
        // as [row][position]; then four threads per (position t, 32-row block hb), 8 inter rows
        // each, form h = silu(g) u w and expand it into the four-term operand together
        if (tr2) a.trace[3584 + (seen - 1) * 4 + 1] = global_ns();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        for (int t = 0; t < n; t++) ubuf[row * 33 + t] = v[t];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (tr2) a.trace[3584 + (seen - 1) * 4 + 2] = global_ns();
        for (int item0 = 32 * q; item0 < 8 * n; item0 += 128) {  // warp-uniform trip count
          const int item = item0 + lane;
          const bool valid = item < 8 * n;  // whole quads: 8 n is a multiple of 4
          const int jb = item >> 2, s4 = item & 3;
          const int hb = valid ? jb / n : 0, t = valid ? jb - hb * n : 0;
          const int p = p0 + t;
          const float wp = valid ? __ldg(a.perm_w + p) : 0.0f;
          float h[8];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const int rr = hb * 32 + 8 * s4 + i;
            const float g = ubuf[rr * 33 + t], u = ubuf[(64 + rr) * 33 + t];
            h[i] = valid ? act_gate(a.act.kind, a.act.beta, a.act.linear_beta, g, u, false) * wp : 0.0f;
          }
          const int i0 = mm * 64 + hb * 32;
          const size_t trow = static_cast<size_t>(4 * p);
          quad_terms4(h, a.ht + trow * (a.inter / 2) + i0 / 2 + 4 * s4, a.inter / 2,
                      a.hsf + trow * (a.inter / 32) + i0 / 32, a.inter / 32, s4 == 0, valid);
        }
        if (tr2) a.trace[3584 + (seen - 1) * 4 + 3] = global_ns();
      } else if (MODE == kModeDown) {
        const int orow = mm * 128 + row;
        for (int t = 0; t < n; t++) a.y[static_cast<size_t>(p0 + t) * a.hidden + orow] = v[t];
      } else {
        a.y[mm * 128 + row] = v[0];
      }
      if (a.trace && blockIdx.x == 0 && et == 0 && seen <= 128) a.trace[3072 + (seen - 1) * 4 + 2] = global_ns();
    }
  }
  if (MODE == kModeDownOne && upt > 1 && warp >= 6 && warp < 10) {
    // every CTA's parts stored -> each CTA adds the parts of its share of output rows in K order
    const int et = threadIdx.x - 192;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (et == 0) {
      red_release_gpu_add(a.work + 3, 1);
      const uint64_t t0 = global_ns();
      while (ld_acquire_gpu(a.work + 3) < static_cast<int>(gridDim.x)) {
        if (global_ns() - t0 > a.spin_ns) {
          atomicOr(a.err, 0x20000u);
          *abort_flag = 1;
          break;
        }
        __nanosleep(64);
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (!*abort_flag) {
      for (int orow = blockIdx.x * 128 + et; orow < a.hidden; orow += gridDim.x * 128) {
        const int tile = orow / 128, rr = orow % 128;
        float v = 0.0f;
        for (int j = 0; j < upt; j++) v += __ldcg(a.partial + static_cast<size_t>(tile * upt + j) * 8 * 128 + rr);
        a.y[orow] = v;
      }
    }
  }
  if (MODE == kModeGateUp && upt > 1 && a.gu_tile_cnt && warp >= 2 && warp < 10) {
    // this CTA's units are done: its scale-factor and epilogue warps finish h of split tiles,
    // items claimed in tile order from the counter (a tile's item waits for its last part)
    const int items = 2 * nch * ntm;
    for (;;) {
      int it = 0;
      if (lane == 0) it = atomicAdd(a.work + 2, 1);
      it = __shfl_sync(kFull, it, 0);
      if (it >= items || *abort_flag) break;
      h_item(a, it, ntm, upt, a.err, lane);
      __syncwarp();
      if (lane == 0) red_release_gpu_add(a.h_done, 1);  // (the item's stores precede, warp-ordered)
    }
  }
  if (a.trace && warp == 6 && lane == 0) a.trace[1024 + 4 * blockIdx.x + 2] = global_ns();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kMtTmemCols);
  }
  if (threadIdx.x == 0) {
    // the last CTA out resets the work counters for the next launch
    __threadfence();
    const int old = atomicAdd(a.work + 1, 1);
    if (old == static_cast<int>(gridDim.x) - 1) {
      a.work[0] = 0;
      a.work[1] = 0;
      a.work[2] = 0;
      a.work[3] = 0;
      // every h item of this launch is done: zero the tile counters for the next forward
      if (MODE == kModeGateUp && upt > 1 && a.gu_tile_cnt)
        for (int i = 0; i < nch * ntm; i++) a.gu_tile_cnt[i] = 0;
    }
  }
  if (a.trace && threadIdx.x == 32) a.trace[1024 + 4 * blockIdx.x + 3] = global_ns();
}

// ---------------------------------------------------------------------- one token, fused experts
// The whole expert part of a one-token forward in one persistent kernel: every CTA claims work
// units from one counter, first the gate/up units (U_gu stages of a 64-row gate + 64-row up tile
// of a chunk's expert), then the down units (all stages of one 128-row down tile of one expert,
// expert-major), so SMs flow from gate/up into down work without a kernel boundary. Gate/up parts
// are released per tile; each CTA's warp 11 forms h of its share of the tiles (tile-major, about
// the order they finish) once a tile's parts are all in (parts added in K order, h = act(g, u) w,
// four-term operand) and counts it per chunk; a down unit's activation loads wait only for its
// own chunk's h. The down parts are added per output row in chunk order after one
// bounded grid barrier. The roles and rings are those of moe_tc_kernel.
struct FusedArgs {
  const int32_t* ch_expert;
  const int32_t* ch_pos;
  const float* perm_w;
  const int32_t* n_chunks;
  int max_chunks;   // entries of ch_expert / ch_pos
  int H, I;
  const uint8_t* arena;
  size_t stride, off_down;
  uint8_t* ht;
  uint8_t* hsf;
  float* part_gu;   // [gate/up units][128]
  float* part_dn;   // [down units][128]
  int* tile_cnt;    // [chunks * I / 64] gate/up parts stored per tile
  int* h_ready;     // [chunks] gate/up tiles whose h is written
  int* work;        // [4] units claimed, -, down parts stored, h tiles claimed (zeroed by the front end)
  unsigned* err;
  float* out;       // [H]
  ActParams act;
  int stages;
  int u_gu;         // stages per gate/up unit
  int sh_slot;      // expert slot of the shared expert (the last chunk), -1: none
  unsigned long long* trace;  // optional: per CTA [8] entry, set-up, first copy, first down unit,
                              // epilogue done, barrier passed, exit (global timer)
  unsigned long long spin_ns;  // limit of each wait on another CTA's counter (then err, abort)
};

constexpr int kFusedThreads = kMtThreads + 32;  // + warp 11: forms h of finished gate/up tiles

__global__ void __launch_bounds__(kFusedThreads, 1) moe_decode_fused_kernel(const __grid_constant__ MoeTcMaps mgu,
                                                                       const __grid_constant__ MoeTcMaps mdn,
                                                                       FusedArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  constexpr int kBoxes = 1;                 // one token: 4 term rows in one 8-row box
  const int bsub = kBoxes * 1024;
  const MtLayout lay = mt_layout(S, kBoxes);
  const int stage_pitch = lay.stage_pitch;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.off_bar);
  uint64_t* sf_full = full + S;
  uint64_t* empty = sf_full + S;
  uint64_t* bfull = empty + S;
  uint64_t* acc_full = bfull + S;
  uint64_t* acc_empty = acc_full + 4;
  uint64_t* rec_full = acc_empty + 4;
  uint64_t* rec_empty = rec_full + kRecRing;
  uint64_t* sfa_done = rec_empty + kRecRing;
  PartRec* recs = reinterpret_cast<PartRec*>(smem + lay.off_rec);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + lay.off_misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* drain = reinterpret_cast<uint64_t*>(smem + lay.off_misc + 16);  // [2] one-use (tc_drain)
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  unsigned long long* trc = a.trace ? a.trace + 8 * blockIdx.x : nullptr;
  if (trc && threadIdx.x == 0) {
    trc[0] = global_ns();
    trc[3] = 0;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&sf_full[i], 128);
      mbar_init(&empty[i], 1);
      mbar_init(&bfull[i], 1);
      mbar_init(&sfa_done[i], 1);
    }
    for (int i = 0; i < 4; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    for (int i = 0; i < kRecRing; i++) {
      mbar_init(&rec_full[i], 1);
      mbar_init(&rec_empty[i], 2 + 128 + 128);
    }
    *abort_flag = 0;
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kMtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int kst_gu = a.H / kMtKStage, kst_dn = a.I / kMtKStage;
  const int ntm_gu = a.I / 64, ntm_dn = a.H / 128;
  const int U_gu = a.u_gu, upt_gu = kst_gu / U_gu;
  // The shared expert (always the last chunk) does not depend on the routing: CTA b < n_pre
  // starts the weight copies of the shared expert's gate/up unit b before the front end is done
  const int n_pre = a.sh_slot >= 0 ? ntm_gu * upt_gu : 0;
  const int pre = static_cast<int>(blockIdx.x) < n_pre ? min(U_gu, S) : 0;
  if (warp == 0 && lane == 0 && pre) {
    const int b = blockIdx.x;
    const uint8_t* base = a.arena + static_cast<size_t>(a.sh_slot) * a.stride;
    const size_t blk0 = static_cast<size_t>(b / upt_gu) * kst_gu + (b % upt_gu) * U_gu;
    for (int j = 0; j < pre; j++) {
      mbar_arrive_expect_tx(&full[j], kTileBlock);
      bulk_g2s_once(smem + j * stage_pitch, base + (blk0 + j) * kTileBlock, kTileBlock, &full[j]);
    }
    if (trc) trc[2] = global_ns();
  }
  griddep_wait();  // routing, dispatch and the token's terms (the front end)
  if (trc && threadIdx.x == 0) trc[1] = global_ns();
  if (threadIdx.x == 0) griddep_launch_dependents();
  // the first 32 chunks' experts and positions, loaded together with the chunk count (the
  // weight producer's first units need them at once)
  __shared__ int s_ce[32], s_cp[32];
  // a CTA whose first unit was preloaded claims its second one now, beside these loads
  int claim2 = 0;
  if (warp == 0 && lane == 0 && pre) claim2 = static_cast<int>(gridDim.x) + atomicAdd(a.work, 1);
  if (warp == 0 && lane < a.max_chunks) {
    s_ce[lane] = __ldg(a.ch_expert + lane);
    s_cp[lane] = __ldg(a.ch_pos + lane);
  }
  if (warp == 0) __syncwarp();
  const int nch = *a.n_chunks;
  // down units: a tile's K in dsplit parts (smaller last units: the CTAs finish closer together)
  const int dsplit = kst_dn % 2 == 0 ? 2 : 1;
  const int n_gu = nch * ntm_gu * upt_gu, n_dn = nch * ntm_dn * dsplit;
  const int total_units = n_gu + n_dn;
  // claim index -> unit: the shared expert's gate/up units first (claims 0..n_pre-1, the CTAs
  // that preloaded them), then every other unit in order
  const int sh_gu0 = (nch - 1) * ntm_gu * upt_gu;
  auto unit_of_claim = [&](int q) {
    if (q < n_pre) return sh_gu0 + q;
    const int r = q - n_pre;
    return r < sh_gu0 ? r : r + n_pre;
  };
  constexpr int acc_cols = 32, nacc = 4;
  const uint32_t sf_base = tbase + 256;

  // unit u -> (kind, tile, uit, chunk, stages, first stage)
  struct Unit {
    int kind, tile, uit, c, m, ns, ks0;
  };
  auto decode = [&](int u) {
    Unit x;
    if (u < n_gu) {
      x.kind = 0;
      x.tile = u / upt_gu;
      x.uit = u % upt_gu;
      x.c = x.tile / ntm_gu;
      x.m = x.tile % ntm_gu;
      x.ns = U_gu;
      x.ks0 = x.uit * U_gu;
    } else {
      const int d = u - n_gu, dt = d / dsplit;
      x.kind = 1;
      x.c = dt / ntm_dn;
      x.m = dt % ntm_dn;
      x.tile = x.m;
      x.uit = d % dsplit;
      x.ns = kst_dn / dsplit;
      x.ks0 = x.uit * x.ns;
    }
    return x;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      int slot = 0, ph = 0, rslot = 0, rph = 0, issued = 0;
      int unit = static_cast<int>(blockIdx.x) < total_units ? unit_of_claim(blockIdx.x) : total_units;
      if (n_pre && (nch - 1 < 32 ? s_ce[nch - 1] : __ldg(a.ch_expert + nch - 1)) != a.sh_slot) {  // (the dispatch put it last)
        atomicOr(a.err, 0x200000u);
        *abort_flag = 1;
      }
      for (int part = 0;; part++) {
        const bool stop = unit >= total_units || *abort_flag;
        int nxt = unit;
        if (part >= kRecRing && !mbar_wait_bounded(&rec_empty[rslot], rph ^ 1, a.err, 0x10u)) {
          *abort_flag = 1;
          break;
        }
        Unit x{};
        int e = 0, p = 0;
        if (!stop) {
          x = decode(unit);
          e = x.c < 32 ? s_ce[x.c] : __ldg(a.ch_expert + x.c);
          p = x.c < 32 ? s_cp[x.c] : __ldg(a.ch_pos + x.c);
        }
        PartRec& r = recs[rslot];
        r.tile = stop ? -1 : x.tile;
        r.uit = x.ns;    // (stages of this unit)
        r.unit = unit;
        r.e = e;
        r.p0 = p;
        r.n = x.c;
        r.brow = x.kind ? 4 * p : 0;  // one token: its terms are rows 0..3; h of position p
        r.pad = x.kind;
        mbar_arrive(&rec_full[rslot]);
        if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
        if (stop) break;
        const uint8_t* base = a.arena + static_cast<size_t>(e) * a.stride + (x.kind ? a.off_down : 0);
        const int kst = x.kind ? kst_dn : kst_gu;
        if (trc && part == 0 && !pre) trc[2] = global_ns();
        if (trc && x.kind == 1 && !trc[3]) trc[3] = global_ns();
        for (int j = 0; j < x.ns; j++, issued++) {
          if (part > 0 || j >= pre) {  // (the preloaded stages were issued before the front end)
            if (issued >= S && !mbar_wait_bounded(&empty[slot], ph ^ 1, a.err, 0x100u)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&full[slot], kTileBlock);
            bulk_g2s_once(smem + slot * stage_pitch,
                          base + (static_cast<size_t>(x.m) * kst + x.ks0 + j) * kTileBlock, kTileBlock, &full[slot]);
          }
          if (++slot == S) { slot = 0; ph ^= 1; }
          // the next claim at the unit's last stage (the ring still holds the stages before it):
          // near the end a CTA then holds one unit ahead, not two
          if (j == x.ns - 1) {
            const int q = part == 0 && pre ? claim2 : static_cast<int>(gridDim.x) + atomicAdd(a.work, 1);
            nxt = q < total_units ? unit_of_claim(q) : total_units;
          }
        }
        // (after an abort the loop's next pass publishes an end record in ring order: a record
        // is never rewritten while a consumer may still be reading it)
        unit = nxt;
      }
      if (issued < pre) issued = pre;  // (stopped before the preloaded unit: its copies are in flight)
      for (int i = (issued > S ? issued - S : 0); i < issued; i++)
        mbar_wait_bounded(&full[i % S], (i / S) & 1, a.err, 0x200u);
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------------ activation producer
    if (lane == 0) {
      tma_prefetch_desc(&mgu.b);
      tma_prefetch_desc(&mdn.b);
      int slot = 0, ph = 0, rslot = 0, rph = 0, issued = 0;
      for (;;) {
        if (!mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x20u)) break;
        const PartRec r = recs[rslot];
        mbar_arrive(&rec_empty[rslot]);
        if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
        if (r.tile < 0 || *abort_flag) break;
        const int kind = r.pad, ns = r.uit, c = r.n;
        if (kind == 1) {
          // this expert's h: all of its gate/up tiles finished
          const uint64_t t0 = global_ns();
          while (ld_acquire_gpu(a.h_ready + c) < ntm_gu) {
            if (global_ns() - t0 > a.spin_ns) {
              atomicOr(a.err, 0x40000u);
              *abort_flag = 1;
              break;
            }
            __nanosleep(32);
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");  // h: plain stores
        }
        const Unit x = decode(r.unit);
        const MoeTcMaps& mp = kind ? mdn : mgu;
        bool ok = true;
        for (int j = 0; j < ns; j++, issued++) {
          if (issued >= S && !mbar_wait_bounded(&empty[slot], ph ^ 1, a.err, 0x100u)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + slot * stage_pitch + kBOff;
          const int ks = x.ks0 + j;
          mbar_arrive_expect_tx(&bfull[slot], 2 * 1024 + 128);
          tma_load_2d(sb, &mp.b, ks * (kMtKStage / 2), r.brow, &bfull[slot]);
          tma_load_2d(sb + bsub, &mp.b, ks * (kMtKStage / 2) + 128, r.brow, &bfull[slot]);
          tma_load_2d(sb + 2 * bsub, &mp.bs, ks * (kMtKStage / 32), r.brow, &bfull[slot]);
          if (++slot == S) { slot = 0; ph ^= 1; }
        }
        if (!ok || *abort_flag) {
          *abort_flag = 1;
          break;
        }
      }
      for (int i = (issued > S ? issued - S : 0); i < issued; i++)
        mbar_wait_bounded(&bfull[i % S], (i / S) & 1, a.err, 0x200u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int i = 0, buf = 0, parts = 0, rslot = 0, rph = 0;
      bool ok = true;
      const uint64_t da0 = sw128_desc(smem), db0 = sw128_desc(smem + kBOff);
      const uint32_t idesc = mxf4_idesc(8);
      for (;;) {
        if (!mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x20u)) break;
        const int tile = recs[rslot].tile, ns = recs[rslot].uit;
        mbar_arrive(&rec_empty[rslot]);
        if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
        if (tile < 0 || *abort_flag) break;
        if (parts >= nacc && !mbar_wait_bounded(&acc_empty[buf], ((parts / nacc) - 1) & 1, a.err, 0x1000u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dacc = tbase + buf * acc_cols;
        for (int j = 0; j < ns && ok; j++, i++) {
          const int slot = i % S;
          const uint32_t ph = (i / S) & 1;
          if (!mbar_wait_bounded(&sfa_done[slot], ph, a.err, 0x800u) ||
              !mbar_wait_bounded(&sf_full[slot], ph, a.err, 0x800u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = da0 + static_cast<uint64_t>((slot * stage_pitch) >> 4);
          const uint64_t db = db0 + static_cast<uint64_t>((slot * stage_pitch) >> 4);
          const uint32_t sfa = sf_base + slot * kMtSfCols, sfb = sfa + 16;
          uint64_t dak[8], dbk[8];
          uint32_t idk[8], sak[8], sbk[8];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const uint32_t adv = (32 * (k & 3)) >> 4;
            dak[k] = da + ((k >> 2) * (16384 >> 4) + adv);
            dbk[k] = db + ((k >> 2) * (bsub >> 4) + adv);
            const uint32_t sid = static_cast<uint32_t>(2 * (k & 1));
            sak[k] = (sfa + 4 * (k >> 1)) | (sid << 30);
            sbk[k] = (sfb + 4 * (k >> 1)) | (sid << 30);
            idk[k] = idesc | (sid << 29) | (sid << 4);
          }
          const uint32_t acc0 = j == 0 ? 0u : 1u;
#pragma unroll
          for (int k = 0; k < 8; k++) mma_mxf4_run(dacc, dak[k], dbk[k], idk[k], sak[k], sbk[k], k == 0 ? acc0 : 1u);
          tc_commit(&empty[slot]);
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
        if (++buf == nacc) buf = 0;
        parts++;
      }
      if (!ok) *abort_flag = 1;
      tc_drain(&drain[0], a.err);
      if (trc) trc[7] = global_ns();
    }
  } else if (warp == 11) {
    // ------------------------------------------------------------------ h of finished gate/up tiles
    // tiles claimed in order from work[3] (a CTA that starts late, e.g. on an SM still busy with
    // another kernel, then holds up no tile)
    for (;;) {
      int tile = 0;
      if (lane == 0) tile = atomicAdd(a.work + 3, 1);
      tile = __shfl_sync(kFull, tile, 0);
      if (tile >= nch * ntm_gu || *abort_flag) break;
      bool ready = true;
      if (lane == 0) {
        const uint64_t t0 = global_ns();
        while (ld_acquire_gpu(a.tile_cnt + tile) < upt_gu) {
          if (global_ns() - t0 > a.spin_ns || *abort_flag) {
            atomicOr(a.err, 0x80000u);
            ready = false;
            break;
          }
          __nanosleep(64);
        }
      }
      if (!__shfl_sync(kFull, ready, 0)) break;
      __syncwarp();
      const int c = tile / ntm_gu, m = tile % ntm_gu;
      const int p = __ldg(a.ch_pos + c);
      const float wp = __ldg(a.perm_w + p);
      for (int hf = 0; hf < 2; hf++) {
        const float* base = a.part_gu + static_cast<size_t>(tile) * upt_gu * 128 + hf * 32 + lane;
        float g = 0.0f, u = 0.0f;
        for (int j = 0; j < upt_gu; j++) {
          g += __ldcg(base + static_cast<size_t>(j) * 128);
          u += __ldcg(base + static_cast<size_t>(j) * 128 + 64);
        }
        const int i0 = m * 64 + hf * 32;
        const float hv = act_gate(a.act.kind, a.act.beta, a.act.linear_beta, g, u, false) * wp;
        const size_t trow = static_cast<size_t>(4 * p);
        warp_terms4(hv, a.ht + trow * (a.I / 2) + i0 / 2, a.I / 2, a.hsf + trow * (a.I / 32) + i0 / 32, a.I / 32);
      }
      __syncwarp();
      if (lane == 0) red_release_gpu_add(a.h_ready + c, 1);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ scale factors -> TMEM
    const int q = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    int i = 0, rslot = 0, rph = 0;
    bool ok = true;
    while (ok) {
      if (!__all_sync(kFull, mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x40u))) break;
      const int tile = __shfl_sync(kFull, recs[rslot].tile, 0);  // (one value for the warp)
      const int ns = __shfl_sync(kFull, recs[rslot].uit, 0);
      mbar_arrive(&rec_empty[rslot]);
      if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
      if (tile < 0) break;
      for (int j = 0; j < ns; j++, i++) {
        const int slot = i % S;
        if (q == 2) {
          bool got = lane != 0 || mbar_wait_bounded(&full[slot], (i / S) & 1, a.err, 0x4000u);
          got = __shfl_sync(kFull, got, 0);
          if (!got) {
            ok = false;
            break;
          }
          if (lane == 0) {
            tc_fence_after();
            const uint8_t* ssa = smem + slot * stage_pitch + 32768;
            const uint32_t sfa = sf_base + slot * kMtSfCols;
#pragma unroll
            for (int g = 0; g < 4; g++) tmem_cp_rows16_x4(sfa + 4 * g, rows16_desc(ssa + g * 512));
            tc_commit(&sfa_done[slot]);
          }
          __syncwarp();
        }
        const bool gotb = mbar_wait_bounded(&bfull[slot], (i / S) & 1, a.err, 0x4000u) && !*abort_flag;
        if (!__all_sync(kFull, gotb)) {
          ok = false;
          break;
        }
        const uint8_t* ssb = smem + slot * stage_pitch + kBOff + 2 * bsub;
        const uint32_t sfb = sf_base + slot * kMtSfCols + 16;
        uint4 rb[4];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
          const int n = lane + 32 * jj;
          rb[jj] = n < 8 ? *reinterpret_cast<const uint4*>(ssb + n * 16)
                         : make_uint4(0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu, 0x7f7f7f7fu);
        }
        tmem_st4(lane_addr | (sfb + 0), rb[0].x, rb[1].x, rb[2].x, rb[3].x);
        tmem_st4(lane_addr | (sfb + 4), rb[0].y, rb[1].y, rb[2].y, rb[3].y);
        tmem_st4(lane_addr | (sfb + 8), rb[0].z, rb[1].z, rb[2].z, rb[3].z);
        tmem_st4(lane_addr | (sfb + 12), rb[0].w, rb[1].w, rb[2].w, rb[3].w);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sf_full[slot]);
      }
    }
    if (q == 2 && lane == 0) tc_drain(&drain[1], a.err);  // (its scale-factor copies)
  } else if (warp < 10) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int et = threadIdx.x - 192;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    const int row = 32 * q + lane;
    int buf = 0, seen = 0, rslot = 0, rph = 0;
    for (;;) {
      const bool gotr = mbar_wait_bounded(&rec_full[rslot], rph, a.err, 0x40u);
      if (!epi_all(gotr)) break;
      const PartRec r = recs[rslot];
      mbar_arrive(&rec_empty[rslot]);
      if (++rslot == kRecRing) { rslot = 0; rph ^= 1; }
      // (the end record and every exit are decided by all 128 threads together)
      const bool got = r.tile >= 0 && mbar_wait_bounded(&acc_full[buf], (seen / nacc) & 1, a.err, 0x8000u);
      if (!epi_all(got && !*abort_flag)) break;
      tc_fence_after();
      float rr[8];
      tmem_ld8(tbase + buf * acc_cols + lane_addr, rr);
      const float v = ((rr[0] + rr[1]) + rr[2]) + rr[3];
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      if (++buf == nacc) buf = 0;
      seen++;
      if (r.pad == 1) {
        a.part_dn[static_cast<size_t>(r.unit - n_gu) * 128 + row] = v;
        continue;
      }
      // gate/up part, released on its tile's counter (warp 11 of some CTA forms the tile's h)
      a.part_gu[static_cast<size_t>(r.unit) * 128 + row] = v;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (et == 0) red_release_gpu_add(a.tile_cnt + r.tile, 1);
    }
    // every CTA's down parts stored (grid barrier), then the whole grid adds them up below
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (trc && et == 0) trc[4] = global_ns();
    if (et == 0) {
      red_release_gpu_add(a.work + 2, 1);
      const uint64_t t0 = global_ns();
      while (ld_acquire_gpu(a.work + 2) < static_cast<int>(gridDim.x)) {
        if (global_ns() - t0 > a.spin_ns) {
          atomicOr(a.err, 0x20000u);
          *abort_flag = 1;
          break;
        }
        __nanosleep(64);
      }
      if (trc) trc[5] = global_ns();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kMtTmemCols);
  }
  // out[row] = the sum of the row's nch * dsplit down parts: four threads per row (every thread
  // of the grid, one round of loads), each adding every fourth part in order, then the four sums
  // combined in a fixed tree -- a deterministic order
  if (!*abort_flag) {
    const int np = nch * dsplit, rows_per_cta = blockDim.x / 4, q4 = threadIdx.x % 4;
    for (int r0 = blockIdx.x * rows_per_cta; r0 < a.H; r0 += gridDim.x * rows_per_cta) {
      const int orow = r0 + threadIdx.x / 4;
      const bool on = orow < a.H;
      const int m = on ? orow / 128 : 0, rr = orow % 128;
      float pv[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int qi = q4 + 4 * j, c = qi / dsplit, h = qi % dsplit;
        pv[j] = on && qi < np ? __ldcg(a.part_dn + static_cast<size_t>((c * ntm_dn + m) * dsplit + h) * 128 + rr)
                              : 0.0f;
      }
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; j++) acc += pv[j];
      for (int qi = q4 + 32; qi < np; qi += 4) {  // (more than 32 parts: rare)
        const int c = qi / dsplit, h = qi % dsplit;
        if (on) acc += __ldcg(a.part_dn + static_cast<size_t>((c * ntm_dn + m) * dsplit + h) * 128 + rr);
      }
      acc += __shfl_xor_sync(kFull, acc, 1);
      acc += __shfl_xor_sync(kFull, acc, 2);
      if (on && q4 == 0) a.out[orow] = acc;
    }
  }
  // (the counters are zeroed by the next launch's front end)
  if (trc && threadIdx.x == 0) trc[6] = global_ns();
}

// ---------------------------------------------------------------------- activation terms per position
// xt rows 4p..4p+3 = terms of the token of position p, stored at each of the token's routed
// positions (inv) and its shared one. One block per (token, 1024 columns): each warp computes the
// four E2M1 terms of four 32-column k-blocks (amax by a warp reduction, each term rounding what
// the previous ones left) into shared memory; then the block writes each of the token's
// positions' term rows as 512-byte spans (32 k-blocks x 16 bytes, one 16-byte store per lane)
// and 32-byte scale runs, so every store fills its sectors.
constexpr int kTermSpan = 32;  // k-blocks per block
__global__ void __launch_bounds__(256) terms_by_position_kernel(const void* __restrict__ x, int x_dtype, int H, int T,
                                                                int k, const int32_t* __restrict__ inv,
                                                                const int32_t* __restrict__ shared_pos0,
                                                                uint8_t* __restrict__ xt, uint8_t* __restrict__ xsf) {
  __shared__ uint4 sterm[4][kTermSpan];  // [term][k-block of the span]
  __shared__ __align__(16) uint8_t ssf[4][kTermSpan];
  __shared__ int spos[32];
  const int nb = H / 32;
  const int spans = (nb + kTermSpan - 1) / kTermSpan;
  const int t = blockIdx.x / spans, b0 = (blockIdx.x % spans) * kTermSpan;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nvb = min(kTermSpan, nb - b0);  // k-blocks in this span
  if (threadIdx.x < 32) {
    int pos = -1;
    if (lane < k) pos = __ldg(inv + t * k + lane);
    else if (lane == k && shared_pos0) pos = __ldg(shared_pos0) + t;
    spos[lane] = pos;
  }
  // the warp's k-blocks' activations loaded together, then their terms
  float rv[kTermSpan / 8];
#pragma unroll
  for (int i = 0; i < kTermSpan / 8; i++) {
    const int kb = warp + 8 * i;
    rv[i] = kb < nvb ? load_elem(x, x_dtype, static_cast<size_t>(t) * H + (b0 + kb) * 32 + lane) : 0.0f;
  }
#pragma unroll
  for (int i = 0; i < kTermSpan / 8; i++) {
    const int kb = warp + 8 * i;
    if (kb >= nvb) break;
    float r = rv[i];
#pragma unroll
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
        sterm[j][kb] = make_uint4(w[0], w[1], w[2], w[3]);
        ssf[j][kb] = static_cast<uint8_t>(amax > 0.0f ? e + 127 : 127);
      }
    }
  }
  __syncthreads();
  // (position slot s, term j): one warp-wide 512-byte row span per item, 32-byte scale runs
  const int np = k + 1;
  for (int it = warp; it < np * 4; it += 8) {
    const int s = it / 4, j = it % 4;
    const int pos = spos[s];
    if (pos < 0) continue;
    const size_t row = static_cast<size_t>(4 * pos + j);
    if (lane < nvb) *reinterpret_cast<uint4*>(xt + row * (H / 2) + (b0 + lane) * 16) = sterm[j][lane];
    if (lane < nvb) xsf[row * nb + b0 + lane] = ssf[j][lane];
  }
}

// One token on given routing, one launch before the one-token expert kernel: block 0's first
// warp builds the chunk table (positions by ascending expert id among the local slots, a
// repeated expert once at its first slot, the shared expert last -- as the one-token dispatch),
// block 0's other threads zero the expert kernel's counters, and every block writes the four
// term rows of its 32 k-blocks of x once (rows 0..3: the one-token kernel reads the token's own
// rows for every position).
__global__ void __launch_bounds__(256) one_token_prep_kernel(const void* __restrict__ x, int x_dtype, int H,
                                                             const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                             int k, int e_begin, int e_end, int n_loc, int has_shared,
                                                             const float* __restrict__ shared_gate_w, DispatchBuffers d,
                                                             int* __restrict__ zero_buf, int zero_n,
                                                             uint8_t* __restrict__ xt, uint8_t* __restrict__ xsf) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // the expert kernel launched next may start now: it waits for this grid before reading any of
  // what it writes (as after the one-token front end)
  if (threadIdx.x == 0) griddep_launch_dependents();
  if (blockIdx.x == 0 && warp == 0) {
    const int sid = lane < k ? ids[lane] : -1;
    const float wv = lane < k ? w[lane] : 0.0f;
    bool first = true;
    for (int j = 0; j < k; j++) {
      const int o = __shfl_sync(kFull, sid, j);
      first &= !(j < lane && o == sid);
    }
    const bool local = lane < k && first && sid >= e_begin && sid < e_end;
    const uint32_t local_mask = __ballot_sync(kFull, local);
    int pos = 0;
    for (int j = 0; j < k; j++) {
      const int o = __shfl_sync(kFull, sid, j);
      pos += ((local_mask >> j) & 1u) && o < sid ? 1 : 0;
    }
    const int n_routed = __popc(local_mask);
    if (lane < k) d.inv[lane] = local ? pos : -1;
    if (local) {
      d.ch_expert[pos] = sid - e_begin;
      d.ch_pos[pos] = pos;
      d.ch_n[pos] = 1;
      d.perm_tok[pos] = 0;
      d.perm_w[pos] = wv;
    }
    if (lane == 0) {
      if (has_shared) {
        d.ch_expert[n_routed] = n_loc;
        d.ch_pos[n_routed] = n_routed;
        d.ch_n[n_routed] = 1;
        d.perm_tok[n_routed] = 0;
        d.perm_w[n_routed] = shared_gate_w ? shared_gate_w[0] : 1.0f;
      }
      d.n_chunks[0] = n_routed + has_shared;
      d.offsets[n_loc] = n_routed;
      d.offsets[n_loc + has_shared] = n_routed + has_shared;
    }
  } else if (blockIdx.x == 0) {
    for (int i = threadIdx.x - 32; i < zero_n; i += blockDim.x - 32) zero_buf[i] = 0;
  }
  const int nb = H / 32;
  const int b0 = blockIdx.x * kTermSpan;
#pragma unroll
  for (int i = 0; i < kTermSpan / 8; i++) {
    const int kb = warp + 8 * i;
    if (b0 + kb >= nb) break;
    const float r = load_elem(x, x_dtype, static_cast<size_t>(b0 + kb) * 32 + lane);
    warp_terms4(r, xt + (b0 + kb) * 16, H / 2, xsf + b0 + kb, H / 32);
  }
}

cudaError_t launch_one_token_prep(const void* x, int x_dtype, int H, const int32_t* ids, const float* w, int k,
                                  int e_begin, int e_end, int n_loc, int has_shared, const float* shared_gate_w,
                                  const DispatchBuffers& d, int* zero_buf, int zero_n, uint8_t* xt, uint8_t* xsf,
                                  cudaStream_t st) {
  if (k > 32 || H % 32) return cudaErrorInvalidValue;
  const int blocks = (H / 32 + kTermSpan - 1) / kTermSpan;
  one_token_prep_kernel<<<blocks, 256, 0, st>>>(x, x_dtype, H, ids, w, k, e_begin, e_end, n_loc, has_shared, shared_gate_w,
                                                d, zero_buf, zero_n, xt, xsf);
  return cudaGetLastError();
}

// Token-major activation terms (the payload expert parallelism exchanges): rows 4t..4t+3 of
// xt / xsf are the four-term E2M1 expansion of token t. One warp per (token, 32-column k-block).
__global__ void __launch_bounds__(256) terms_rows_kernel(const void* __restrict__ x, int x_dtype, int H, int T,
                                                         uint8_t* __restrict__ xt, uint8_t* __restrict__ xsf) {
  const int nb = H / 32;
  const long long wid = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32;
  if (wid >= static_cast<long long>(T) * nb) return;
  const int t = static_cast<int>(wid / nb), b = static_cast<int>(wid % nb);
  const float r = load_elem(x, x_dtype, static_cast<size_t>(t) * H + b * 32 + (threadIdx.x & 31));
  warp_terms4(r, xt + static_cast<size_t>(4 * t) * (H / 2) + b * 16, H / 2, xsf + static_cast<size_t>(4 * t) * nb + b, nb);
}

cudaError_t launch_terms_rows(const void* x, int x_dtype, int H, int T, uint8_t* xt, uint8_t* xsf, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (H % 32) return cudaErrorInvalidValue;
  const long long warps = static_cast<long long>(T) * (H / 32);
  terms_rows_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, st>>>(x, x_dtype, H, T, xt, xsf);
  return cudaGetLastError();
}

// The position rows of the expert kernels from token-major terms: position inv[t][j] (>= 0)
// gets token t's four rows and their scales. One block per (token, slot).
__global__ void __launch_bounds__(256) terms_gather_kernel(const uint8_t* __restrict__ tt, const uint8_t* __restrict__ tsf,
                                                           int H, int k, const int32_t* __restrict__ inv,
                                                           uint8_t* __restrict__ xt, uint8_t* __restrict__ xsf) {
  const int q = blockIdx.x, t = q / k;
  const int pos = inv[q];
  if (pos < 0) return;
  const size_t rb = static_cast<size_t>(H) / 2, nb = static_cast<size_t>(H) / 32;
  const uint4* src = reinterpret_cast<const uint4*>(tt + static_cast<size_t>(4 * t) * rb);
  uint4* dst = reinterpret_cast<uint4*>(xt + static_cast<size_t>(4 * pos) * rb);
  for (size_t i = threadIdx.x; i < 4 * rb / 16; i += blockDim.x) dst[i] = src[i];
  for (size_t i = threadIdx.x; i < 4 * nb; i += blockDim.x) xsf[static_cast<size_t>(4 * pos) * nb + i] = tsf[static_cast<size_t>(4 * t) * nb + i];
}

cudaError_t launch_terms_gather(const uint8_t* tt, const uint8_t* tsf, int H, int T, int k, const int32_t* inv,
                                uint8_t* xt, uint8_t* xsf, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (H % 32 || reinterpret_cast<uintptr_t>(tt) % 16 || reinterpret_cast<uintptr_t>(xt) % 16) return cudaErrorInvalidValue;
  terms_gather_kernel<<<T * k, 256, 0, st>>>(tt, tsf, H, k, inv, xt, xsf);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------- host side
bool make_tmap_sw128(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);
bool make_tmap_rows(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                    uint32_t box_rows);

struct MoeTcPlanImpl {
  MoeTcMaps gu, dn;
};

static int sm_count() { return device_sm_count(); }

// Grid of a persistent kernel whose CTAs wait on one another: as many CTAs as can be resident
// at once (SMs x the occupancy the kernel's shared memory allows, which is one per SM for these
// kernels), so every CTA of the grid runs together. If other work holds SMs when the kernel
// starts (another context, an MPS client limit), a CTA can still wait for a peer that never
// arrives; those waits are bounded (~2 s) and end the call with RMOE_TIMEOUT rather than hang.
static int resident_grid(const void* kern, int threads, size_t smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return sm_count() * per_sm;
}

// Stages per work unit for batches of <= 8 tokens: 4 when that divides the per-expert stage
// count kst (then it also divides the one-token down projection's run over experts), else whole
// tiles. (Smaller units balance better on paper but their per-unit epilogue and part traffic
// cost more than they save: measured at the K3 shapes, kst 7 and 6.)
static int small_unit_stages(int kst) { return kst % 4 == 0 ? 4 : kst; }

size_t moe_tc_partial_floats(int H, int I, int k, int n_slots) {
  const size_t chunks = static_cast<size_t>(8) * k + 8 + n_slots;  // at most, with <= 8 tokens
  const int kst_gu = H / kMtKStage, kst_dn = I / kMtKStage;
  const size_t gu = chunks * (I / 64) * (kst_gu / small_unit_stages(kst_gu));      // units of split tiles
  const size_t dn = chunks * (H / 128) * (kst_dn / small_unit_stages(kst_dn));
  return (std::max(gu, dn) + 64) * 8 * 128;
}

bool moe_tc_supported(int H, int I, int Is, int fmt) {
  return fmt == kMxfp4 && H % kMtKStage == 0 && H % 128 == 0 && I % kMtKStage == 0 && I % 64 == 0 &&
         (Is == 0 || Is == I);
}

size_t moe_tc_plan_bytes() { return sizeof(MoeTcPlanImpl); }

// Tensor maps of one layer (built once: every pointer is fixed at layer creation).
bool moe_tc_plan(void* plan, int H, int I, const uint8_t* xt, const uint8_t* xsf, const uint8_t* ht,
                 const uint8_t* hsf, int term_rows) {
  MoeTcPlanImpl* p = static_cast<MoeTcPlanImpl*>(plan);
  bool ok = true;
  ok = ok && make_tmap_sw128(&p->gu.b, xt, H / 2, term_rows, 8);
  ok = ok && make_tmap_rows(&p->gu.bs, xsf, H / 32, term_rows, 16, 8);
  ok = ok && make_tmap_sw128(&p->dn.b, ht, I / 2, term_rows, 8);
  ok = ok && make_tmap_rows(&p->dn.bs, hsf, I / 32, term_rows, 16, 8);
  ok = ok && make_tmap_sw128(&p->gu.b128, xt, H / 2, term_rows, 128);
  ok = ok && make_tmap_rows(&p->gu.bs128, xsf, H / 32, term_rows, 16, 128);
  ok = ok && make_tmap_sw128(&p->dn.b128, ht, I / 2, term_rows, 128);
  ok = ok && make_tmap_rows(&p->dn.bs128, hsf, I / 32, term_rows, 16, 128);
  return ok;
}

// Bytes of one expert's tile-major gate/up and down regions.
size_t moe_tc_region_bytes(int H, int I, int down) {
  return down ? static_cast<size_t>(H / 128) * (I / kMtKStage) * kTileBlock
              : static_cast<size_t>(I / 64) * (H / kMtKStage) * kTileBlock;
}

// Reference row-major matrices (E2M1 rows of K/2 bytes, E8M0 rows of K/32 bytes) -> tile blocks.
// Tile row r is row m * half + r of m0 (r < half) or row m * half + r - half of m1.
__global__ void tc_relayout_kernel(const uint8_t* __restrict__ m0, const uint8_t* __restrict__ m1,
                                   const uint8_t* __restrict__ s0, const uint8_t* __restrict__ s1, int K,
                                   int half, int ntiles, uint8_t* __restrict__ dst) {
  const int KS = K / kMtKStage;
  const size_t nchunk = static_cast<size_t>(ntiles) * KS * 2 * 128 * 8;
  const size_t nword = static_cast<size_t>(ntiles) * KS * 512;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nchunk; i += stride) {
    const int c = i & 7, r = (i >> 3) & 127, h = (i >> 10) & 1;
    const size_t blk = i >> 11;
    const int m = static_cast<int>(blk / KS), ks = static_cast<int>(blk % KS);
    const uint8_t* row = r < half ? m0 + static_cast<size_t>(m * half + r) * (K / 2)
                                  : m1 + static_cast<size_t>(m * half + r - half) * (K / 2);
    const uint4 v = *reinterpret_cast<const uint4*>(row + 256 * ks + 128 * h + 16 * c);
    *reinterpret_cast<uint4*>(dst + blk * kTileBlock + h * 16384 + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nword; i += stride) {
    const int j = i & 3, g = (i >> 2) & 3, L = (i >> 4) & 31;
    const size_t blk = i >> 9;
    const int m = static_cast<int>(blk / KS), ks = static_cast<int>(blk % KS);
    const int r = L + 32 * j;
    const uint8_t* row = r < half ? s0 + static_cast<size_t>(m * half + r) * (K / 32)
                                  : s1 + static_cast<size_t>(m * half + r - half) * (K / 32);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 16 * ks + 4 * g);
    *reinterpret_cast<uint32_t*>(dst + blk * kTileBlock + 32768 + ((g * 128 + L * 4 + j) << 2)) = w;
  }
}

// gate/up: m0 = gate, m1 = up (K = hidden); down: m0 = down (K = inter), m1 unused.
cudaError_t launch_tc_relayout(int down, const uint8_t* m0, const uint8_t* m1, const uint8_t* s0,
                               const uint8_t* s1, int H, int I, uint8_t* dst, cudaStream_t st) {
  const int K = down ? I : H, half = down ? 128 : 64, ntiles = down ? H / 128 : I / 64;
  tc_relayout_kernel<<<1184, 256, 0, st>>>(m0, down ? m0 : m1, s0, down ? s0 : s1, K, half, ntiles, dst);
  return cudaGetLastError();
}

cudaError_t launch_terms_by_position(const void* x, int x_dtype, int H, int T, int k, const int32_t* inv,
                                     const int32_t* shared_pos0, uint8_t* xt, uint8_t* xsf, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (k > 31) return cudaErrorInvalidValue;
  const long long n = static_cast<long long>(T) * ((H / 32 + kTermSpan - 1) / kTermSpan);
  terms_by_position_kernel<<<static_cast<unsigned>(n), 256, 0, st>>>(x, x_dtype, H, T, k, inv, shared_pos0,
                                                                                  xt, xsf);
  return cudaGetLastError();
}

static size_t moe_tc_smem(int stages, int b_boxes) {
  return 1024 + static_cast<size_t>(mt_layout(stages, b_boxes).total);
}

// mode: 0 gate/up, 1 down, 2 down for one token. mt = positions per chunk (<= 32).
cudaError_t launch_moe_tc(int mode, const void* plan, const DispatchBuffers& d, int mt, int H, int I,
                          const uint8_t* arena, size_t stride, size_t off_down, uint8_t* ht, uint8_t* hsf, float* y, float* partial,
                          int32_t* tile_cnt, int* work, unsigned* err, cudaStream_t st, const int32_t* b_token_rows,
                          unsigned long long* trace, ActParams act, int32_t* gu_tile_cnt, int* h_done,
                          bool weights_once, unsigned long long spin_ns) {
  const MoeTcPlanImpl* p = static_cast<const MoeTcPlanImpl*>(plan);
  MoeTcArgs a{};
  a.ch_expert = d.ch_expert; a.ch_pos = d.ch_pos; a.ch_n = d.ch_n; a.n_chunks = d.n_chunks;
  a.perm_w = d.perm_w;
  a.K = mode == 0 ? H : I;
  a.out_rows = mode == 0 ? I : H;
  a.wbase = arena + (mode == 0 ? 0 : off_down);
  a.wstride = stride;
  a.b_boxes = (4 * mt + 7) / 8;
  a.ht = ht; a.hsf = hsf; a.inter = I;
  a.y = y; a.hidden = H;
  a.partial = partial; a.tile_cnt = tile_cnt; a.err = err;
  a.b_tok = b_token_rows;
  a.trace = trace;
  a.work = work;
  // Small batches split tiles into 4-stage units (small_unit_stages), so ~10 units per SM
  // balance the streams.
  const int kst_own = (mode == 0 ? H : I) / kMtKStage;
  // (the several-token down projection never splits: its epilogue writes whole tiles)
  a.unit_stages = mt <= 8 && mode != 1 ? small_unit_stages(kst_own) : 1 << 30;
  a.act = act;
  a.gu_tile_cnt = gu_tile_cnt;
  a.h_done = h_done;
  a.weights_once = weights_once ? 1 : 0;
  a.spin_ns = spin_ns;
  a.h_split = (mode != 0 && mt <= 8 && small_unit_stages(H / kMtKStage) < H / kMtKStage) ? 1 : 0;
  int stages = kMtMaxStages;
  while (stages > 2 && moe_tc_smem(stages, a.b_boxes) > 227 * 1024) stages--;
  a.stages = stages;
  const size_t smem = moe_tc_smem(stages, a.b_boxes);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  const MoeTcMaps& maps = mode == 0 ? p->gu : p->dn;
  // Down kernels whose CTAs wait on each other (h slices, the one-token output sum) rely on all
  // CTAs being resident together: the grid is one CTA per SM and a CTA needs most of an SM's
  // shared memory, so no two of them share an SM; the waits are bounded either way. (A
  // cooperative launch would also guarantee residency, but inside a CUDA graph it waits for the
  // order-resolving kernel running beside it.)
  const bool coop = false;
  void (*kern)(const MoeTcMaps, MoeTcArgs) = mode == 0 ? moe_tc_kernel<kModeGateUp>
                                             : mode == 1 ? moe_tc_kernel<kModeDown> : moe_tc_kernel<kModeDownOne>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int grid = resident_grid(reinterpret_cast<const void*>(kern), kMtThreads, smem);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMtThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = coop ? 1 : 0;
  // programmatic dependent launch: set-up (TMEM, barriers, tensor maps) and, for the down
  // kernels, the first weight stages overlap the previous kernel's tail
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, maps, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// One token after the fused front end: the gate/up and down units of every routed expert and
// the shared one in one persistent launch (moe_decode_fused_kernel), out = the combined row.
cudaError_t launch_moe_decode_fused(const void* plan, const DispatchBuffers& d, int H, int I, const uint8_t* arena,
                                    size_t stride, size_t off_down, uint8_t* ht, uint8_t* hsf, float* part_gu,
                                    float* part_dn, int32_t* tile_cnt, int32_t* h_ready, int* work, unsigned* err,
                                    float* out, ActParams act, int sh_slot, cudaStream_t st,
                                    unsigned long long* trace, unsigned long long spin_ns) {
  const MoeTcPlanImpl* p = static_cast<const MoeTcPlanImpl*>(plan);
  FusedArgs a{};
  a.trace = trace;
  a.ch_expert = d.ch_expert; a.ch_pos = d.ch_pos; a.perm_w = d.perm_w; a.n_chunks = d.n_chunks;
  a.max_chunks = d.max_chunks;
  a.H = H; a.I = I;
  a.arena = arena; a.stride = stride; a.off_down = off_down;
  a.ht = ht; a.hsf = hsf;
  a.part_gu = part_gu; a.part_dn = part_dn;
  a.tile_cnt = tile_cnt; a.h_ready = h_ready; a.work = work; a.err = err; a.out = out;
  a.act = act;
  a.u_gu = small_unit_stages(H / kMtKStage);
  a.sh_slot = sh_slot;
  a.spin_ns = spin_ns;
  int stages = kMtMaxStages;
  while (stages > 2 && moe_tc_smem(stages, 1) > 227 * 1024) stages--;
  a.stages = stages;
  const size_t smem = moe_tc_smem(stages, 1);
  cudaError_t e = cudaFuncSetAttribute(moe_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(resident_grid(reinterpret_cast<const void*>(moe_decode_fused_kernel), kFusedThreads, smem));
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel, p->gu, p->dn, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace rmoe
