// gemv_pipe.cu -- the expert GEMVs as persistent, TMA-staged kernels (one CTA per SM).
//
// Weight rows stream HBM -> shared memory through a 16-slot ring of bulk copies
// (cp.async.bulk + mbarrier complete_tx), issued by one producer warp; eight consumer warps
// dequantize from shared memory in registers and dot with the activations. Every CTA owns one
// contiguous, equal share of the flattened task list, so all SMs stream the same number of
// bytes and finish together; ~140 KB per SM is in flight, enough to cover HBM latency at full
// bandwidth. No spin is unbounded: a wait that exceeds its limit sets a flag and returns.
//
//   MODE 0 (gate/up):  stage = gate row r + up row r of a chunk's expert (K = H); epilogue
//                      h = silu(g) * u per token (glm52/moe.rs:58-70) and |h| max per position.
//   MODE 1 (down):     stage = 8 down rows of a chunk's expert (K = inter); h enters as f32 and
//                      is scaled into f16 on the fly; epilogue y[position][row].
//   MODE 2 (down + combine, one token per stage): task = (token, 8 output rows); its stages
//                      are the 8 down rows of each of the token's k experts and of the shared
//                      expert, accumulated in rank order with their routing weight / shared gate
//                      into out[token][rows] (glm52/moe.rs:508-512, qwen38/generate.rs:346-349).
#include <algorithm>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "pipe.cuh"

namespace rmoe {

constexpr int kStages = 16;
constexpr int kConsumers = 8;
constexpr int kPipeThreads = (kConsumers + 1) * 32;
constexpr int kDownRows = 8;

struct PipeArgs {
  ExpertTable tab;
  ExpertFormat f;
  DispatchBuffers d;
  const void* xin;       // MODE 0: xq f16 [T][x_ld] by token; MODE 1/2: h f32 [P][x_ld]
  const int32_t* xexp;   // MODE 0: per-token exponent
  const uint32_t* hmax;  // MODE 0: written (|h| max per position); MODE 1/2: read
  int x_ld;
  float* out;            // MODE 0: h [P][out_ld]; MODE 1: y [P][out_ld]; MODE 2: out [T][out_ld]
  int out_ld;
  int H;
  int slot_bytes;
  int T, k;              // MODE 2
  const int32_t* ids;    // MODE 2: routing [T][k] (positions from d.inv)
  int e_begin;           // MODE 2
  int hbuf_ok;           // MODE 2: the h rows of one token fit in the shared-memory cache
  unsigned* err_flag;
};

// What the consumers of one slot need besides the weights, written by the producer so that no
// consumer waits on a dependent global load.
struct SlotMeta {
  int r, eslot, p0, n;
  int row[8];   // activation row of each chunk position (token for MODE 0, position otherwise)
  int xe[8];    // its power-of-two exponent
  float w;      // MODE 2: routing weight / shared gate of this stage's position
  int last;     // MODE 2: 1 on the task's final stage
};

__device__ __forceinline__ void load_x_f16(const void* xin, int row, int x_ld, int b,
                                           uint32_t (&xv)[16]) {
  const uint4* xp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xin) +
                                                   static_cast<size_t>(row) * x_ld + b * 32);
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const uint4 v = __ldg(xp + q);
    xv[4 * q] = v.x; xv[4 * q + 1] = v.y; xv[4 * q + 2] = v.z; xv[4 * q + 3] = v.w;
  }
}

// 32 f32 activations scaled by 2^e into f16 pairs in the format's pair order.
template <int FMT>
__device__ __forceinline__ void load_x_f32(const void* xin, int row, int x_ld, int b, float sc,
                                           uint32_t (&xv)[16]) {
  const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(xin) +
                                                     static_cast<size_t>(row) * x_ld + b * 32);
#pragma unroll
  for (int g = 0; g < 4; g++) {  // 8-element groups
    const float4 lo = __ldg(xp + 2 * g), hi = __ldg(xp + 2 * g + 1);
    const float v[8] = {lo.x * sc, lo.y * sc, lo.z * sc, lo.w * sc,
                        hi.x * sc, hi.y * sc, hi.z * sc, hi.w * sc};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      __half2 h2 = FMT == kMxfp4 ? __floats2half2_rn(v[2 * q], v[2 * q + 1])
                                 : __floats2half2_rn(v[q], v[q + 4]);
      xv[4 * g + q] = *reinterpret_cast<uint32_t*>(&h2);
    }
  }
}

template <int FMT, int MT, int MODE>
__global__ void __launch_bounds__(kPipeThreads, 1) gemv_pipe_kernel(PipeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NR = MODE == 0 ? 2 : kDownRows;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * a.slot_bytes);
  uint64_t* empty = full + kStages;
  SlotMeta* meta = reinterpret_cast<SlotMeta*>(empty + kStages);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int32_t* task0 = MODE == 0 ? a.d.ch_task_gu : a.d.ch_task_dn;
  const int n_chunks = *a.d.n_chunks;
  const int has_shared = a.tab.shared_inter > 0;
  const int S = MODE == 2 ? a.k + has_shared : 1;  // stages per task
  const int n_tasks = MODE == 2 ? a.T * (a.H / kDownRows) : task0[n_chunks];
  const int t_begin = static_cast<int>((static_cast<long long>(n_tasks) * blockIdx.x) / gridDim.x);
  const int t_end = static_cast<int>((static_cast<long long>(n_tasks) * (blockIdx.x + 1)) / gridDim.x);
  const int my_tasks = t_end - t_begin;
  // Consumer warp w owns local tasks w, w + 8, ... and ring slots 2w and 2w + 1; its q-th stage
  // (task w + 8 * (q / S), sub-stage q % S) lives in slot 2w + (q & 1), phase q / 2. Every slot
  // therefore has exactly one consumer, which never waits more than one phase ahead.
  auto warp_stages = [&](int w) { return w < my_tasks ? ((my_tasks - 1 - w) / kConsumers + 1) * S : 0; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ------------------------------------------------------------ producer (round-robin)
    if (lane == 0 && my_tasks > 0) {
      int c = 0, c_end = 0;
      SlotMeta cm{};
      ExpertPtrs ep{};
      auto enter_chunk = [&](int cc) {
        c_end = task0[cc + 1];
        cm.eslot = a.d.ch_expert[cc];
        cm.p0 = a.d.ch_pos[cc];
        cm.n = a.d.ch_n[cc];
#pragma unroll
        for (int m = 0; m < 8; m++) {
          const int mm = m < cm.n ? m : 0;
          const int row = MODE == 0 ? a.d.perm_tok[cm.p0 + mm] : cm.p0 + mm;
          cm.row[m] = row;
          cm.xe[m] = MODE == 0 ? a.xexp[row] : f16_row_exponent(__uint_as_float(a.hmax[row]));
        }
        ep = expert_ptrs(a.tab, cm.eslot);
      };
      if (MODE != 2) {
        c = find_chunk(task0, n_chunks, t_begin);
        enter_chunk(c);
      }
      const int rounds = warp_stages(0);
      for (int q = 0; q < rounds; q++) {
        for (int w = 0; w < kConsumers; w++) {
          if (q >= warp_stages(w)) continue;
          const int task = t_begin + w + kConsumers * (q / S);
          const int j = q % S;
          const int slot = 2 * w + (q & 1);
          int r = 0;
          if (MODE == 2) {
            const int t = task / (a.H / kDownRows);
            r = task % (a.H / kDownRows);
            int p = -1, eslot = 0;
            if (j < a.k) {
              p = a.d.inv[t * a.k + j];
              if (p >= 0) eslot = a.ids[t * a.k + j] - a.e_begin;
            } else {
              p = a.d.offsets[a.tab.n_local] + t;
              eslot = a.tab.n_local;
            }
            cm.eslot = eslot;
            cm.p0 = p;
            cm.n = p >= 0 ? 1 : 0;
            cm.row[0] = p;
            cm.xe[0] = p >= 0 ? f16_row_exponent(__uint_as_float(a.hmax[p])) : 0;
            cm.w = p >= 0 ? a.d.perm_w[p] : 0.0f;
            cm.last = j == S - 1;
            ep = expert_ptrs(a.tab, eslot);
          } else {
            while (task >= c_end) enter_chunk(++c);
            r = task - task0[c];
          }
          if (q >= 2 && !mbar_wait_bounded(&empty[slot], ((q / 2) - 1) & 1, a.err_flag, 1u)) return;
          uint8_t* dst = smem + static_cast<size_t>(slot) * a.slot_bytes;
          cm.r = r;
          meta[slot] = cm;
          if (MODE == 0) {
            const uint32_t rb = a.H / 2, sb = static_cast<uint32_t>(scale_row_bytes(a.f, a.H));
            mbar_arrive_expect_tx(&full[slot], 2 * (rb + sb));
            bulk_g2s(dst, ep.gate + static_cast<size_t>(r) * rb, rb, &full[slot]);
            bulk_g2s(dst + rb, ep.up + static_cast<size_t>(r) * rb, rb, &full[slot]);
            bulk_g2s(dst + 2 * rb, static_cast<const uint8_t*>(ep.gate_scale) + static_cast<size_t>(r) * sb, sb,
                     &full[slot]);
            bulk_g2s(dst + 2 * rb + sb, static_cast<const uint8_t*>(ep.up_scale) + static_cast<size_t>(r) * sb,
                     sb, &full[slot]);
          } else if (cm.n == 0) {
            mbar_arrive(&full[slot]);  // nothing to load for a position on another EP rank
          } else {
            const int K = cm.eslot >= a.tab.n_local ? a.tab.shared_inter : a.tab.inter;
            const uint32_t rb = K / 2, sb = static_cast<uint32_t>(scale_row_bytes(a.f, K));
            const size_t row0 = static_cast<size_t>(r) * NR;
            mbar_arrive_expect_tx(&full[slot], NR * (rb + sb));
            bulk_g2s(dst, ep.down + row0 * rb, NR * rb, &full[slot]);
            bulk_g2s(dst + NR * rb, static_cast<const uint8_t*>(ep.down_scale) + row0 * sb, NR * sb, &full[slot]);
          }
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // MODE 2: the h rows (f16, scaled) of the first token this CTA serves live in shared memory,
  // loaded once; stages of that token read them from there.
  uint16_t* hbuf = reinterpret_cast<uint16_t*>(meta + kStages);
  int h_tok = -1;
  const int kmax = max(a.tab.inter, a.tab.shared_inter);
  if (MODE == 2 && a.hbuf_ok && my_tasks > 0) {
    h_tok = t_begin / (a.H / kDownRows);
    for (int jj = 0; jj < S; jj++) {
      int p;
      int Kj;
      if (jj < a.k) {
        p = a.d.inv[h_tok * a.k + jj];
        Kj = a.tab.inter;
      } else {
        p = a.d.offsets[a.tab.n_local] + h_tok;
        Kj = a.tab.shared_inter;
      }
      if (p < 0) continue;
      const float sc = exp2i(f16_row_exponent(__uint_as_float(a.hmax[p])));
      const float* src = static_cast<const float*>(a.xin) + static_cast<size_t>(p) * a.x_ld;
      uint16_t* dst = hbuf + static_cast<size_t>(jj) * kmax;
      for (int i = threadIdx.x * 8; i < Kj; i += kConsumers * 32 * 8) {
        const float4 lo = __ldg(reinterpret_cast<const float4*>(src + i));
        const float4 hi = __ldg(reinterpret_cast<const float4*>(src + i + 4));
        const float v[8] = {lo.x * sc, lo.y * sc, lo.z * sc, lo.w * sc,
                            hi.x * sc, hi.y * sc, hi.z * sc, hi.w * sc};
        uint32_t pk[4];
#pragma unroll
        for (int qq = 0; qq < 4; qq++) {
          __half2 h2 = FMT == kMxfp4 ? __floats2half2_rn(v[2 * qq], v[2 * qq + 1])
                                     : __floats2half2_rn(v[qq], v[qq + 4]);
          pk[qq] = *reinterpret_cast<uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(dst + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32));  // consumer warps only
  }

  // MODE 0 with one token per chunk: the lane's activation blocks stay in registers across
  // stages (reloaded only when the chunk's token changes).
  constexpr int XB = 8;  // blocks per lane cached (H <= 8192)
  uint32_t xc[XB][16];
  int xc_row = -1;
  const bool xcache = MODE == 0 && MT == 1 && (a.H / 32) <= 32 * XB;

  int q = 0;  // this warp's stage counter
  for (int tk = warp; tk < my_tasks; tk += kConsumers) {
    float comb[NR];  // MODE 2: weighted sum over the task's stages (per-lane partials)
#pragma unroll
    for (int qq = 0; qq < NR; qq++) comb[qq] = 0.0f;
    const int t_task = MODE == 2 ? (t_begin + tk) / (a.H / kDownRows) : 0;
    for (int j = 0; j < S; j++, q++) {
      const int slot = 2 * warp + (q & 1);
      if (!mbar_wait_bounded(&full[slot], (q / 2) & 1, a.err_flag, 2u)) return;
      const SlotMeta& sm = meta[slot];
      const int r = sm.r, eslot = sm.eslot, p0 = sm.p0, n = sm.n;
      const int K = MODE == 0 ? a.H : (eslot >= a.tab.n_local ? a.tab.shared_inter : a.tab.inter);
      const uint32_t rb = K / 2, sb = static_cast<uint32_t>(scale_row_bytes(a.f, K));
      const uint8_t* base = smem + static_cast<size_t>(slot) * a.slot_bytes;
      int rows[MT], xe[MT];
#pragma unroll
      for (int m = 0; m < MT; m++) {
        rows[m] = sm.row[m];
        xe[m] = sm.xe[m];
      }
      const float wstage = sm.w;
      const int last = sm.last;
      float acc[NR][MT];
#pragma unroll
      for (int qq = 0; qq < NR; qq++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[qq][m] = 0.0f;
      const int nblk = K / 32;
      if (MODE == 0 && xcache) {
        // ---- gate/up, one token: x blocks from registers
        if (rows[0] != xc_row) {
#pragma unroll
          for (int jb = 0; jb < XB; jb++) {
            const int b = lane + 32 * jb;
            if (b < nblk) load_x_f16(a.xin, rows[0], a.x_ld, b, xc[jb]);
          }
          xc_row = rows[0];
        }
#pragma unroll
        for (int jb = 0; jb < XB; jb++) {
          const int b = lane + 32 * jb;
          if (b >= nblk) break;
          uint32_t hg[16], hu[16];
          decode_block<FMT>(*reinterpret_cast<const uint4*>(base + b * 16), hg);
          decode_block<FMT>(*reinterpret_cast<const uint4*>(base + rb + b * 16), hu);
          const float sg = block_scale_smem<FMT>(base + 2 * rb, b, a.f);
          const float su = block_scale_smem<FMT>(base + 2 * rb + sb, b, a.f);
          uint32_t g0 = 0, g1 = 0, u0 = 0, u1 = 0;
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            g0 = hfma2u(hg[e], xc[jb][e], g0);
            g1 = hfma2u(hg[e + 1], xc[jb][e + 1], g1);
            u0 = hfma2u(hu[e], xc[jb][e], u0);
            u1 = hfma2u(hu[e + 1], xc[jb][e + 1], u1);
          }
          acc[0][0] = fmaf(h2sum_f32(g0) + h2sum_f32(g1), sg, acc[0][0]);
          acc[NR > 1 ? 1 : 0][0] = fmaf(h2sum_f32(u0) + h2sum_f32(u1), su, acc[NR > 1 ? 1 : 0][0]);
        }
      } else if (MODE == 2) {
        // ---- down + combine, one position: h blocks from shared memory (or converted from
        //      global for a token other than the cached one); each block serves all 8 rows
        if (n > 0) {
          const bool from_smem = t_task == h_tok;
          for (int b = lane; b < nblk; b += 32) {
            uint32_t xv[16];
            if (from_smem) {
              const uint4* hp = reinterpret_cast<const uint4*>(hbuf + static_cast<size_t>(j) * kmax + b * 32);
#pragma unroll
              for (int qq = 0; qq < 4; qq++) {
                const uint4 v = hp[qq];
                xv[4 * qq] = v.x; xv[4 * qq + 1] = v.y; xv[4 * qq + 2] = v.z; xv[4 * qq + 3] = v.w;
              }
            } else {
              load_x_f32<FMT>(a.xin, rows[0], a.x_ld, b, exp2i(xe[0]), xv);
            }
#pragma unroll
            for (int g0 = 0; g0 < NR; g0 += 4) {
              uint32_t hw[4][16];
              float sc[4];
#pragma unroll
              for (int qq = 0; qq < 4; qq++) {
                decode_block<FMT>(*reinterpret_cast<const uint4*>(base + (g0 + qq) * rb + b * 16), hw[qq]);
                sc[qq] = block_scale_smem<FMT>(base + NR * rb + (g0 + qq) * sb, b, a.f);
              }
#pragma unroll
              for (int qq = 0; qq < 4; qq++) {
                uint32_t a0 = 0, a1 = 0;
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                  a0 = hfma2u(hw[qq][e], xv[e], a0);
                  a1 = hfma2u(hw[qq][e + 1], xv[e + 1], a1);
                }
                acc[g0 + qq][0] = fmaf(h2sum_f32(a0) + h2sum_f32(a1), sc[qq], acc[g0 + qq][0]);
              }
            }
          }
        }
      } else {
        // ---- general: rows in groups of (at most) 4 keep the decoded nibbles in registers
#pragma unroll
        for (int g0 = 0; g0 < NR; g0 += 4) {
          constexpr int G = NR < 4 ? NR : 4;
          for (int b = lane; b < nblk; b += 32) {
            uint32_t hw[G][16];
            float sc[G];
#pragma unroll
            for (int qq = 0; qq < G; qq++) {
              const uint4 w = *reinterpret_cast<const uint4*>(base + (g0 + qq) * rb + b * 16);
              decode_block<FMT>(w, hw[qq]);
              sc[qq] = block_scale_smem<FMT>(base + NR * rb + (g0 + qq) * sb, b, a.f);
            }
#pragma unroll
            for (int m = 0; m < MT; m++) {
              if (m >= n) break;
              uint32_t xv[16];
              if (MODE == 0) load_x_f16(a.xin, rows[m], a.x_ld, b, xv);
              else load_x_f32<FMT>(a.xin, rows[m], a.x_ld, b, exp2i(xe[m]), xv);
#pragma unroll
              for (int qq = 0; qq < G; qq++) {
                uint32_t a0 = 0, a1 = 0;
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                  a0 = hfma2u(hw[qq][e], xv[e], a0);
                  a1 = hfma2u(hw[qq][e + 1], xv[e + 1], a1);
                }
                acc[g0 + qq][m] = fmaf(h2sum_f32(a0) + h2sum_f32(a1), sc[qq], acc[g0 + qq][m]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // this slot's shared memory is no longer read
      if (MODE == 2) {
        if (n > 0) {
          const float wu = wstage * exp2i(-xe[0]);
#pragma unroll
          for (int qq = 0; qq < NR; qq++) comb[qq] = fmaf(wu, acc[qq][0], comb[qq]);
        }
        if (last) {
#pragma unroll
          for (int qq = 0; qq < NR; qq++) comb[qq] = warp_sum(comb[qq]);
          if (lane < NR) {
            float v = comb[0];
#pragma unroll
            for (int qq = 1; qq < NR; qq++)
              if (lane == qq) v = comb[qq];
            a.out[static_cast<size_t>(t_task) * a.out_ld + r * NR + lane] = v;
          }
        }
        continue;
      }
#pragma unroll
      for (int qq = 0; qq < NR; qq++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[qq][m] = warp_sum(acc[qq][m]);
      if (MODE == 0) {
#pragma unroll
        for (int m = 0; m < MT; m++) {
          if (m >= n) break;
          if (lane == m) {
            const float unscale = exp2i(-xe[m]);
            const float g = acc[0][m] * unscale, u = acc[NR > 1 ? 1 : 0][m] * unscale;
            const float hv = act_gate(a.f.act.kind, a.f.act.beta, a.f.act.linear_beta, g, u, true);
            a.out[static_cast<size_t>(p0 + m) * a.out_ld + r] = hv;
            atomicMax(const_cast<uint32_t*>(a.hmax) + p0 + m, __float_as_uint(fabsf(hv)));
          }
        }
      } else {
#pragma unroll
        for (int m = 0; m < MT; m++) {
          if (m >= n) break;
          if (lane < NR) {
            float v = acc[0][m];
#pragma unroll
            for (int qq = 1; qq < NR; qq++)
              if (lane == qq) v = acc[qq][m];
            a.out[static_cast<size_t>(p0 + m) * a.out_ld + r * NR + lane] = v * exp2i(-xe[m]);
          }
        }
      }
    }
  }
}

template <int FMT, int MODE>
static cudaError_t launch_pipe_fmt(int mt, const PipeArgs& a, int grid, size_t smem, cudaStream_t st) {
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<grid, kPipeThreads, smem, st>>>(a);
    return cudaGetLastError();
  };
  if (MODE == 2) return go(gemv_pipe_kernel<FMT, 1, MODE>);
  switch (mt) {
    case 1: return go(gemv_pipe_kernel<FMT, 1, MODE>);
    case 2: return go(gemv_pipe_kernel<FMT, 2, MODE>);
    case 4: return go(gemv_pipe_kernel<FMT, 4, MODE>);
    default: return go(gemv_pipe_kernel<FMT, 8, MODE>);
  }
}

bool pipe_supported(const ExpertFormat& f, int H, int inter, int shared_inter) {
  // every bulk copy must be a multiple of 16 bytes at 16-byte aligned addresses
  auto ok_k = [&](int K, int rows) {
    return K % 32 == 0 && (K / 2) % 16 == 0 && (scale_row_bytes_host(f, K) * rows) % 16 == 0;
  };
  if (H % kDownRows || !ok_k(H, 1)) return false;
  if (!ok_k(inter, kDownRows)) return false;
  if (shared_inter && !ok_k(shared_inter, kDownRows)) return false;
  return true;
}

static int num_sms() { return device_sm_count(); }

static size_t pipe_smem(int slot_bytes) {
  return static_cast<size_t>(kStages) * slot_bytes + kStages * 16 + kStages * sizeof(SlotMeta);
}

cudaError_t launch_pipe_gate_up(const ExpertTable& tab, const ExpertFormat& f,
                                const DispatchBuffers& d, const uint16_t* xq,
                                const int32_t* xexp, int H, int mt, float* h, uint32_t* hmax,
                                int h_ld, unsigned* err_flag, cudaStream_t st) {
  PipeArgs a{};
  a.tab = tab; a.f = f; a.d = d; a.xin = xq; a.xexp = xexp; a.hmax = hmax; a.x_ld = H;
  a.out = h; a.out_ld = h_ld; a.H = H; a.err_flag = err_flag;
  a.slot_bytes = static_cast<int>((2 * (H / 2 + scale_row_bytes_host(f, H)) + 127) / 128 * 128);
  const size_t smem = pipe_smem(a.slot_bytes);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (f.fmt == kMxfp4) return launch_pipe_fmt<kMxfp4, 0>(mt, a, num_sms(), smem, st);
  return launch_pipe_fmt<kInt4g, 0>(mt, a, num_sms(), smem, st);
}

static int down_slot_bytes(const ExpertTable& tab, const ExpertFormat& f) {
  const int K = std::max(tab.inter, tab.shared_inter);
  return static_cast<int>((kDownRows * (K / 2 + scale_row_bytes_host(f, K)) + 127) / 128 * 128);
}

cudaError_t launch_pipe_down(const ExpertTable& tab, const ExpertFormat& f,
                             const DispatchBuffers& d, const float* h, const uint32_t* hmax,
                             int H, int mt, int h_ld, float* y, unsigned* err_flag,
                             cudaStream_t st) {
  PipeArgs a{};
  a.tab = tab; a.f = f; a.d = d; a.xin = h; a.hmax = hmax; a.x_ld = h_ld;
  a.out = y; a.out_ld = H; a.H = H; a.err_flag = err_flag;
  a.slot_bytes = down_slot_bytes(tab, f);
  const size_t smem = pipe_smem(a.slot_bytes);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (f.fmt == kMxfp4) return launch_pipe_fmt<kMxfp4, 1>(mt, a, num_sms(), smem, st);
  return launch_pipe_fmt<kInt4g, 1>(mt, a, num_sms(), smem, st);
}

cudaError_t launch_pipe_down_combine(const ExpertTable& tab, const ExpertFormat& f,
                                     const DispatchBuffers& d, const float* h,
                                     const uint32_t* hmax, const int32_t* ids, int T, int k,
                                     int e_begin, int H, int h_ld, float* out, unsigned* err_flag,
                                     cudaStream_t st) {
  PipeArgs a{};
  a.tab = tab; a.f = f; a.d = d; a.xin = h; a.hmax = hmax; a.x_ld = h_ld;
  a.out = out; a.out_ld = H; a.H = H; a.err_flag = err_flag;
  a.T = T; a.k = k; a.ids = ids; a.e_begin = e_begin;
  a.slot_bytes = down_slot_bytes(tab, f);
  const int kmax = std::max(tab.inter, tab.shared_inter);
  const size_t hbuf = static_cast<size_t>(k + (tab.shared_inter > 0 ? 1 : 0)) * kmax * 2;
  size_t smem = pipe_smem(a.slot_bytes);
  if (smem + hbuf <= 227 * 1024) {
    a.hbuf_ok = 1;
    smem += hbuf;
  }
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (f.fmt == kMxfp4) return launch_pipe_fmt<kMxfp4, 2>(1, a, num_sms(), smem, st);
  return launch_pipe_fmt<kInt4g, 2>(1, a, num_sms(), smem, st);
}

}  // namespace rmoe
