// gemv_pipe.cu -- the expert GEMVs as persistent, TMA-staged kernels (one CTA per SM).
//
// Weight rows stream HBM -> shared memory through a 16-slot ring of bulk copies
// (cp.async.bulk + mbarrier complete_tx), issued by one producer warp; eight consumer warps
// dequantize from shared memory in registers and dot with the activations. Every CTA owns one
// contiguous, equal share of the flattened task list, so all SMs stream the same number of
// bytes and finish together; ~140 KB per SM is in flight, enough to cover HBM latency at full
// bandwidth. No spin is unbounded: a wait that exceeds its limit sets a flag and returns.
//
//   MODE 0 (gate/up): task = one row index r of one chunk: gate row r and up row r (K = H);
//                     epilogue h = silu(g) * u per token (glm52/moe.rs:58-70), |h| max per row.
//   MODE 1 (down):    task = 8 consecutive rows of the chunk expert's down matrix (K = inter);
//                     epilogue y[position][row] for the chunk's positions.
#include <algorithm>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "pipe.cuh"

namespace rmoe {

constexpr int kStages = 16;
constexpr int kConsumers = 8;
constexpr int kPipeThreads = (kConsumers + 1) * 32;

struct PipeArgs {
  ExpertTable tab;
  ExpertFormat f;
  DispatchBuffers d;
  const uint16_t* xin;   // MODE 0: xq [T][x_ld] by token; MODE 1: hq [P][x_ld] by position
  const int32_t* xexp;   // MODE 0: per token; MODE 1: per position
  int x_ld;
  float* out;            // MODE 0: h [P][out_ld]; MODE 1: y [P][out_ld]
  int out_ld;
  uint32_t* hmax;        // MODE 0 only
  int H;
  int slot_bytes;
  unsigned* err_flag;
};

template <int MODE>
struct PipeGeom;
template <>
struct PipeGeom<0> {
  static constexpr int kRows = 2;  // gate row + up row
};
template <>
struct PipeGeom<1> {
  static constexpr int kRows = 8;  // 8 down rows
};

// What the consumers of one slot need besides the weights, written by the producer so that no
// consumer waits on a dependent global load: chunk, row index, expert slot, first position,
// positions in the chunk, and each position's activation row and power-of-two exponent.
struct SlotMeta {
  int c, r, eslot, p0, n;
  int row[8];
  int xe[8];
};

template <int FMT, int MT, int MODE>
__global__ void __launch_bounds__(kPipeThreads, 1) gemv_pipe_kernel(PipeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NR = PipeGeom<MODE>::kRows;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * a.slot_bytes);
  uint64_t* empty = full + kStages;
  SlotMeta* meta = reinterpret_cast<SlotMeta*>(empty + kStages);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int32_t* task0 = MODE == 0 ? a.d.ch_task_gu : a.d.ch_task_dn;
  const int n_chunks = *a.d.n_chunks;
  const int n_tasks = task0[n_chunks];
  const int t_begin = static_cast<int>((static_cast<long long>(n_tasks) * blockIdx.x) / gridDim.x);
  const int t_end = static_cast<int>((static_cast<long long>(n_tasks) * (blockIdx.x + 1)) / gridDim.x);
  const int my_tasks = t_end - t_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && my_tasks > 0) {
      // tasks of this CTA are contiguous: one search, then the chunk index only moves forward
      int c = find_chunk(task0, n_chunks, t_begin);
      SlotMeta cm;
      int c_end = 0;
      ExpertPtrs ep{};
      auto enter_chunk = [&](int cc) {
        c_end = task0[cc + 1];
        cm.c = cc;
        cm.eslot = a.d.ch_expert[cc];
        cm.p0 = a.d.ch_pos[cc];
        cm.n = a.d.ch_n[cc];
#pragma unroll
        for (int m = 0; m < 8; m++) {
          const int mm = m < cm.n ? m : 0;
          const int row = MODE == 0 ? a.d.perm_tok[cm.p0 + mm] : cm.p0 + mm;
          cm.row[m] = row;
          cm.xe[m] = a.xexp[row];
        }
        ep = expert_ptrs(a.tab, cm.eslot);
      };
      enter_chunk(c);
      for (int i = 0; i < my_tasks; i++) {
        const int slot = i % kStages;
        const int task = t_begin + i;
        while (task >= c_end) enter_chunk(++c);
        const int r = task - task0[c];
        const int eslot = cm.eslot;
        if (i >= kStages && !mbar_wait_bounded(&empty[slot], ((i / kStages) - 1) & 1, a.err_flag, 1u))
          return;
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
          bulk_g2s(dst + 2 * rb + sb, static_cast<const uint8_t*>(ep.up_scale) + static_cast<size_t>(r) * sb, sb,
                   &full[slot]);
        } else {
          const int K = eslot >= a.tab.n_local ? a.tab.shared_inter : a.tab.inter;
          const uint32_t rb = K / 2, sb = static_cast<uint32_t>(scale_row_bytes(a.f, K));
          const size_t row0 = static_cast<size_t>(r) * NR;
          mbar_arrive_expect_tx(&full[slot], NR * (rb + sb));
          bulk_g2s(dst, ep.down + row0 * rb, NR * rb, &full[slot]);
          bulk_g2s(dst + NR * rb, static_cast<const uint8_t*>(ep.down_scale) + row0 * sb, NR * sb, &full[slot]);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  for (int i = warp; i < my_tasks; i += kConsumers) {
    const int slot = i % kStages;
    if (!mbar_wait_bounded(&full[slot], (i / kStages) & 1, a.err_flag, 2u)) return;
    const SlotMeta& sm = meta[slot];
    const int r = sm.r;
    const int eslot = sm.eslot;
    const int p0 = sm.p0, n = sm.n;
    const int K = MODE == 0 ? a.H : (eslot >= a.tab.n_local ? a.tab.shared_inter : a.tab.inter);
    const uint32_t rb = K / 2, sb = static_cast<uint32_t>(scale_row_bytes(a.f, K));
    const uint8_t* base = smem + static_cast<size_t>(slot) * a.slot_bytes;
    const uint16_t* xr[MT];
    int xe[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) {
      xr[m] = a.xin + static_cast<size_t>(sm.row[m]) * a.x_ld;
      xe[m] = sm.xe[m];
    }
    float acc[NR][MT];
#pragma unroll
    for (int q = 0; q < NR; q++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[q][m] = 0.0f;
    const int nblk = K / 32;
    // rows in groups of (at most) 4 keep the decoded nibbles in registers
#pragma unroll
    for (int g0 = 0; g0 < NR; g0 += 4) {
      constexpr int G = NR < 4 ? NR : 4;
      for (int b = lane; b < nblk; b += 32) {
        uint32_t hw[G][16];
        float sc[G];
#pragma unroll
        for (int q = 0; q < G; q++) {
          const uint4 w = *reinterpret_cast<const uint4*>(base + (g0 + q) * rb + b * 16);
          decode_block<FMT>(w, hw[q]);
          sc[q] = block_scale_smem<FMT>(base + NR * rb + (g0 + q) * sb, b, a.f);
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
          if (m >= n) break;
          const uint4* xp = reinterpret_cast<const uint4*>(xr[m] + static_cast<size_t>(b) * 32);
          uint32_t xv[16];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const uint4 v = __ldg(xp + q);
            xv[4 * q] = v.x; xv[4 * q + 1] = v.y; xv[4 * q + 2] = v.z; xv[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int q = 0; q < G; q++) {
            uint32_t a0 = 0, a1 = 0;
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              a0 = hfma2u(hw[q][e], xv[e], a0);
              a1 = hfma2u(hw[q][e + 1], xv[e + 1], a1);
            }
            acc[g0 + q][m] = fmaf(h2sum_f32(a0) + h2sum_f32(a1), sc[q], acc[g0 + q][m]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // shared memory of this slot is no longer read
#pragma unroll
    for (int q = 0; q < NR; q++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[q][m] = warp_sum(acc[q][m]);
    if (MODE == 0) {
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m >= n) break;
        if (lane == m) {
          const float unscale = exp2i(-xe[m]);
          const float g = acc[0][m] * unscale, u = acc[1][m] * unscale;
          const float hv = __fmul_rn(silu_ref(g), u);
          a.out[static_cast<size_t>(p0 + m) * a.out_ld + r] = hv;
          atomicMax(a.hmax + p0 + m, __float_as_uint(fabsf(hv)));
        }
      }
    } else {
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m >= n) break;
        if (lane < NR) {
          float v = acc[0][m];
#pragma unroll
          for (int q = 1; q < NR; q++)
            if (lane == q) v = acc[q][m];
          a.out[static_cast<size_t>(p0 + m) * a.out_ld + r * NR + lane] = v * exp2i(-xe[m]);
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
  if (!ok_k(H, 1)) return false;
  if (!ok_k(inter, PipeGeom<1>::kRows)) return false;
  if (shared_inter && !ok_k(shared_inter, PipeGeom<1>::kRows)) return false;
  return true;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

cudaError_t launch_pipe_gate_up(const ExpertTable& tab, const ExpertFormat& f,
                                const DispatchBuffers& d, const uint16_t* xq,
                                const int32_t* xexp, int H, int mt, float* h, uint32_t* hmax,
                                int h_ld, unsigned* err_flag, cudaStream_t st) {
  PipeArgs a{tab, f, d, xq, xexp, H, h, h_ld, hmax, H, 0, err_flag};
  a.slot_bytes = static_cast<int>(2 * (H / 2 + scale_row_bytes_host(f, H)));
  a.slot_bytes = (a.slot_bytes + 127) / 128 * 128;
  const size_t smem = static_cast<size_t>(kStages) * a.slot_bytes + kStages * 16 + kStages * sizeof(SlotMeta);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (f.fmt == kMxfp4) return launch_pipe_fmt<kMxfp4, 0>(mt, a, num_sms(), smem, st);
  return launch_pipe_fmt<kInt4g, 0>(mt, a, num_sms(), smem, st);
}

cudaError_t launch_pipe_down(const ExpertTable& tab, const ExpertFormat& f,
                             const DispatchBuffers& d, const uint16_t* hq, const int32_t* hexp,
                             int H, int mt, int h_ld, float* y, unsigned* err_flag,
                             cudaStream_t st) {
  PipeArgs a{tab, f, d, hq, hexp, h_ld, y, H, nullptr, H, 0, err_flag};
  const int K = std::max(tab.inter, tab.shared_inter);
  a.slot_bytes = static_cast<int>(PipeGeom<1>::kRows * (K / 2 + scale_row_bytes_host(f, K)));
  a.slot_bytes = (a.slot_bytes + 127) / 128 * 128;
  const size_t smem = static_cast<size_t>(kStages) * a.slot_bytes + kStages * 16 + kStages * sizeof(SlotMeta);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (f.fmt == kMxfp4) return launch_pipe_fmt<kMxfp4, 1>(mt, a, num_sms(), smem, st);
  return launch_pipe_fmt<kInt4g, 1>(mt, a, num_sms(), smem, st);
}

}  // namespace rmoe
