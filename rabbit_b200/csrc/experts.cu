// experts.cu -- the grouped expert products on CUDA cores: activation prep, the fused
// gate/up + SwiGLU GEMV, the down GEMV, the weighted combine, and the generic matmul_qt-style
// entry points.
//
// Weights stream from HBM exactly once per call in the reference byte layout (no re-packing):
// a lane owns one 32-element block per step = one 16-byte load of nibbles + its scale. Nibbles
// become f16 pairs in registers (cvt.rn.f16x2.e2m1x2 for MXFP4, a LOP3/HSUB2 trick for int4),
// are multiplied with f16 activations by HFMA2 into a per-block f16x2 partial, and every block
// partial is widened to f32 and scaled by its E8M0 / group scale. Activations enter f16 with a
// per-row power-of-two scale (exact, undone on output), so the f16 range never limits inputs.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.h"

namespace rmoe {

// ------------------------------------------------------------------------------ prep
// One block per token: amax -> power-of-two exponent, the f16 copy in the format's pair order
// (MXFP4: natural; int4: within each 8-group the pairs are (0,4),(1,5),(2,6),(3,7)), and the
// Qwen shared-expert gate sigmoid(x . g).
__global__ void __launch_bounds__(256) prep_tokens_kernel(const void* __restrict__ x, int x_dtype,
                                                          int H, int fmt,
                                                          const float* __restrict__ gvec,
                                                          uint16_t* __restrict__ xq,
                                                          int32_t* __restrict__ xexp,
                                                          float* __restrict__ gate_out) {
  const int t = blockIdx.x;
  __shared__ float red[2][8];
  float amax = 0.0f, dot = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = load_elem(x, x_dtype, static_cast<size_t>(t) * H + i);
    amax = fmaxf(amax, fabsf(v));
    if (gvec) dot = fmaf(v, gvec[i], dot);
  }
  amax = warp_max(amax);
  dot = warp_sum(dot);
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    red[0][wi] = amax;
    red[1][wi] = dot;
  }
  __syncthreads();
  if (wi == 0) {
    float a = lane < 8 ? red[0][lane] : 0.0f;
    float d = lane < 8 ? red[1][lane] : 0.0f;
    a = warp_max(a);
    d = warp_sum(d);
    if (lane == 0) {
      red[0][0] = a;
      red[1][0] = d;
    }
  }
  __syncthreads();
  const int e = f16_row_exponent(red[0][0]);
  if (threadIdx.x == 0) {
    xexp[t] = e;
    if (gate_out) gate_out[t] = gvec ? sigmoid_ref(red[1][0]) : 1.0f;
  }
  const float sc = exp2i(e);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = load_elem(x, x_dtype, static_cast<size_t>(t) * H + i) * sc;
    int dst = i;
    if (fmt == kInt4g) {
      const int g = i & ~7, q = i & 7;
      dst = g + (q < 4 ? 2 * q : 2 * (q - 4) + 1);
    }
    xq[static_cast<size_t>(t) * H + dst] = __half_as_ushort(__float2half_rn(v));
  }
}

cudaError_t launch_prep_tokens(const void* x, int x_dtype, int T, int H, int fmt,
                               const float* shared_gate_vec, uint16_t* xq, int32_t* xexp,
                               float* gate_out, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  prep_tokens_kernel<<<T, 256, 0, st>>>(x, x_dtype, H, fmt, shared_gate_vec, xq, xexp, gate_out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ gate/up
// Warp task = (chunk, two row pairs): gate rows 2r, 2r+1 and up rows 2r, 2r+1 of the chunk's
// expert against the chunk's (<= MT) tokens; epilogue h = silu(g) * u (glm52/moe.rs:58-70).
template <int FMT, int MT>
__global__ void __launch_bounds__(256) gemv_gate_up_kernel(ExpertTable tab, ExpertFormat f,
                                                           DispatchBuffers d,
                                                           const uint16_t* __restrict__ xq,
                                                           const int32_t* __restrict__ xexp, int H,
                                                           float* __restrict__ h,
                                                           uint32_t* __restrict__ hmax, int h_ld) {
  const int n_chunks = *d.n_chunks;
  const int n_tasks = d.ch_task_gu[n_chunks];
  const int lane = threadIdx.x % 32;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nw = gridDim.x * (blockDim.x / 32);
  const size_t row_bytes = static_cast<size_t>(H) / 2;
  const size_t srow = scale_row_bytes(f, H);
  for (int task = gw; task < n_tasks; task += nw) {
    const int c = find_chunk(d.ch_task_gu, n_chunks, task);
    const int slot = d.ch_expert[c];
    const int r0 = (task - d.ch_task_gu[c]) * 2;
    const int p0 = d.ch_pos[c], n = d.ch_n[c];
    const ExpertPtrs ep = expert_ptrs(tab, slot);
    const uint8_t* rows[4] = {ep.gate + r0 * row_bytes, ep.gate + (r0 + 1) * row_bytes,
                              ep.up + r0 * row_bytes, ep.up + (r0 + 1) * row_bytes};
    const void* srows[4] = {static_cast<const uint8_t*>(ep.gate_scale) + r0 * srow,
                            static_cast<const uint8_t*>(ep.gate_scale) + (r0 + 1) * srow,
                            static_cast<const uint8_t*>(ep.up_scale) + r0 * srow,
                            static_cast<const uint8_t*>(ep.up_scale) + (r0 + 1) * srow};
    const uint16_t* xr[MT];
    int tok[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) {
      tok[m] = m < n ? d.perm_tok[p0 + m] : 0;
      xr[m] = xq + static_cast<size_t>(tok[m]) * H;
    }
    float acc[4][MT];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;
    gemv_accumulate<FMT, 4, MT>(rows, srows, xr, n, H, f, acc);
    warp_reduce_all<4, MT>(acc);
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m >= n) break;
      if (lane < 2) {
        const float unscale = exp2i(-xexp[tok[m]]);
        const float g = (lane == 0 ? acc[0][m] : acc[1][m]) * unscale;
        const float u = (lane == 0 ? acc[2][m] : acc[3][m]) * unscale;
        const float hv = act_gate(f.act.kind, f.act.beta, f.act.linear_beta, g, u, true);
        h[static_cast<size_t>(p0 + m) * h_ld + r0 + lane] = hv;
        atomicMax(hmax + p0 + m, __float_as_uint(fabsf(hv)));
      }
    }
  }
}

template <int FMT>
static void launch_gu_fmt(int mt, dim3 grid, const ExpertTable& tab, const ExpertFormat& f,
                          const DispatchBuffers& d, const uint16_t* xq, const int32_t* xexp,
                          int H, float* h, uint32_t* hmax, int h_ld, cudaStream_t st) {
  switch (mt) {
    case 1: gemv_gate_up_kernel<FMT, 1><<<grid, 256, 0, st>>>(tab, f, d, xq, xexp, H, h, hmax, h_ld); break;
    case 2: gemv_gate_up_kernel<FMT, 2><<<grid, 256, 0, st>>>(tab, f, d, xq, xexp, H, h, hmax, h_ld); break;
    case 4: gemv_gate_up_kernel<FMT, 4><<<grid, 256, 0, st>>>(tab, f, d, xq, xexp, H, h, hmax, h_ld); break;
    default: gemv_gate_up_kernel<FMT, 8><<<grid, 256, 0, st>>>(tab, f, d, xq, xexp, H, h, hmax, h_ld); break;
  }
}

static int gemv_grid(int max_tasks) {
  const int warps_per_block = 8;
  int blocks = (max_tasks + warps_per_block - 1) / warps_per_block;
  return std::max(1, std::min(blocks, device_sm_count() * 4));
}

cudaError_t launch_gemv_gate_up(const ExpertTable& tab, const ExpertFormat& f,
                                const DispatchBuffers& d, const uint16_t* xq,
                                const int32_t* xexp, int H, int mt, int max_tasks, float* h,
                                uint32_t* hmax, int h_ld, cudaStream_t st) {
  dim3 grid(gemv_grid(max_tasks));
  if (f.fmt == kMxfp4) launch_gu_fmt<kMxfp4>(mt, grid, tab, f, d, xq, xexp, H, h, hmax, h_ld, st);
  else launch_gu_fmt<kInt4g>(mt, grid, tab, f, d, xq, xexp, H, h, hmax, h_ld, st);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ h -> f16
__global__ void __launch_bounds__(256) quant_h_kernel(const float* __restrict__ h,
                                                      const uint32_t* __restrict__ hmax,
                                                      const int32_t* __restrict__ total_pos,
                                                      int inter_ld, int fmt,
                                                      uint16_t* __restrict__ hq,
                                                      int32_t* __restrict__ hexp) {
  const int p = blockIdx.x;
  if (p >= *total_pos) return;
  const int e = f16_row_exponent(__uint_as_float(hmax[p]));
  if (threadIdx.x == 0) hexp[p] = e;
  const float sc = exp2i(e);
  for (int i = threadIdx.x; i < inter_ld; i += blockDim.x) {
    float v = h[static_cast<size_t>(p) * inter_ld + i] * sc;
    int dst = i;
    if (fmt == kInt4g) {
      const int g = i & ~7, q = i & 7;
      dst = g + (q < 4 ? 2 * q : 2 * (q - 4) + 1);
    }
    hq[static_cast<size_t>(p) * inter_ld + dst] = __half_as_ushort(__float2half_rn(v));
  }
}

cudaError_t launch_quant_h(const float* h, const uint32_t* hmax, const int32_t* total_pos,
                           int P_max, int inter_ld, int fmt, uint16_t* hq, int32_t* hexp,
                           cudaStream_t st) {
  if (P_max <= 0) return cudaSuccess;
  quant_h_kernel<<<P_max, 256, 0, st>>>(h, hmax, total_pos, inter_ld, fmt, hq, hexp);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ down
// Warp task = (chunk, four output rows of the expert's down matrix) over the chunk's positions.
template <int FMT, int MT>
__global__ void __launch_bounds__(256) gemv_down_kernel(ExpertTable tab, ExpertFormat f,
                                                        DispatchBuffers d,
                                                        const uint16_t* __restrict__ hq,
                                                        const int32_t* __restrict__ hexp, int H,
                                                        int h_ld, float* __restrict__ y) {
  const int n_chunks = *d.n_chunks;
  const int n_tasks = d.ch_task_dn[n_chunks];
  const int lane = threadIdx.x % 32;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nw = gridDim.x * (blockDim.x / 32);
  for (int task = gw; task < n_tasks; task += nw) {
    const int c = find_chunk(d.ch_task_dn, n_chunks, task);
    const int slot = d.ch_expert[c];
    const int K = slot >= tab.n_local ? tab.shared_inter : tab.inter;
    const size_t row_bytes = static_cast<size_t>(K) / 2;
    const size_t srow = scale_row_bytes(f, K);
    const int o0 = (task - d.ch_task_dn[c]) * 4;
    const int p0 = d.ch_pos[c], n = d.ch_n[c];
    const ExpertPtrs ep = expert_ptrs(tab, slot);
    const uint8_t* rows[4];
    const void* srows[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      rows[r] = ep.down + (o0 + r) * row_bytes;
      srows[r] = static_cast<const uint8_t*>(ep.down_scale) + (o0 + r) * srow;
    }
    const uint16_t* xr[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) xr[m] = hq + static_cast<size_t>(p0 + (m < n ? m : 0)) * h_ld;
    float acc[4][MT];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;
    gemv_accumulate<FMT, 4, MT>(rows, srows, xr, n, K, f, acc);
    warp_reduce_all<4, MT>(acc);
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m >= n) break;
      if (lane < 4) {
        const float unscale = exp2i(-hexp[p0 + m]);
        const float v = (lane == 0 ? acc[0][m] : lane == 1 ? acc[1][m] : lane == 2 ? acc[2][m] : acc[3][m]);
        y[static_cast<size_t>(p0 + m) * H + o0 + lane] = v * unscale;
      }
    }
  }
}

template <int FMT>
static void launch_dn_fmt(int mt, dim3 grid, const ExpertTable& tab, const ExpertFormat& f,
                          const DispatchBuffers& d, const uint16_t* hq, const int32_t* hexp,
                          int H, int h_ld, float* y, cudaStream_t st) {
  switch (mt) {
    case 1: gemv_down_kernel<FMT, 1><<<grid, 256, 0, st>>>(tab, f, d, hq, hexp, H, h_ld, y); break;
    case 2: gemv_down_kernel<FMT, 2><<<grid, 256, 0, st>>>(tab, f, d, hq, hexp, H, h_ld, y); break;
    case 4: gemv_down_kernel<FMT, 4><<<grid, 256, 0, st>>>(tab, f, d, hq, hexp, H, h_ld, y); break;
    default: gemv_down_kernel<FMT, 8><<<grid, 256, 0, st>>>(tab, f, d, hq, hexp, H, h_ld, y); break;
  }
}

cudaError_t launch_gemv_down(const ExpertTable& tab, const ExpertFormat& f,
                             const DispatchBuffers& d, const uint16_t* hq, const int32_t* hexp,
                             int H, int mt, int max_tasks, int h_ld, float* y, cudaStream_t st) {
  dim3 grid(gemv_grid(max_tasks));
  if (f.fmt == kMxfp4) launch_dn_fmt<kMxfp4>(mt, grid, tab, f, d, hq, hexp, H, h_ld, y, st);
  else launch_dn_fmt<kInt4g>(mt, grid, tab, f, d, hq, hexp, H, h_ld, y, st);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ combine
// out[t] = sum_j w[t][j] * y[inv[t][j]] (rank order) + gate_t * y[shared position of t]
// (glm52/moe.rs:508-512 weighted scatter-add, qwen38/generate.rs:346-349 shared added last),
// as a deterministic gather: no atomics, fixed order per token.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ y,
                                                      const int32_t* __restrict__ inv,
                                                      const float* __restrict__ rw,
                                                      const int32_t* __restrict__ shared_pos0,
                                                      const float* __restrict__ perm_w, int k,
                                                      int H, int has_shared,
                                                      float* __restrict__ out) {
  const int t = blockIdx.y;
  const int o = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (o >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < k; j++) {
    const int p = inv[t * k + j];
    if (p < 0) continue;
    const float wv = rw ? rw[t * k + j] : 1.0f;  // null: weights already inside y
    const float4 v = *reinterpret_cast<const float4*>(y + static_cast<size_t>(p) * H + o);
    acc.x = fmaf(wv, v.x, acc.x);
    acc.y = fmaf(wv, v.y, acc.y);
    acc.z = fmaf(wv, v.z, acc.z);
    acc.w = fmaf(wv, v.w, acc.w);
  }
  if (has_shared) {
    const int p = *shared_pos0 + t;
    const float g = rw ? perm_w[p] : 1.0f;
    const float4 v = *reinterpret_cast<const float4*>(y + static_cast<size_t>(p) * H + o);
    acc.x = fmaf(g, v.x, acc.x);
    acc.y = fmaf(g, v.y, acc.y);
    acc.z = fmaf(g, v.z, acc.z);
    acc.w = fmaf(g, v.w, acc.w);
  }
  *reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H + o) = acc;
}

cudaError_t launch_combine(const float* y, const DispatchBuffers& d, const float* rw, int T,
                           int k, int H, int shared_slot, int has_shared, float* out,
                           cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  dim3 grid((H / 4 + 255) / 256, T);
  combine_kernel<<<grid, 256, 0, st>>>(y, d.inv, rw, d.offsets + shared_slot, d.perm_w, k, H,
                                       has_shared, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ rank-order sum
// out[r] = ((parts[0][r] + parts[1][r]) + ... + parts[n-1][r]) + last[r]: the owner-side combine
// of expert parallelism, every rank's partial sum of a token's routed slots added in rank order
// and the (gated) shared expert last, as moe_forward adds it after the routed experts
// (src/qwen38/generate.rs:324-349). One thread per 4 consecutive floats of the rows.
__global__ void __launch_bounds__(256) sum_rank_parts_kernel(const float* __restrict__ parts, int n,
                                                             size_t count4, const float* __restrict__ last,
                                                             float* __restrict__ out) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count4; i += stride) {
    float4 acc = __ldcs(reinterpret_cast<const float4*>(parts) + i);
    for (int r = 1; r < n; r++) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(parts) + static_cast<size_t>(r) * count4 + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if (last) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(last) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
}

cudaError_t launch_sum_rank_parts(const float* parts, int n, size_t count, const float* last, float* out,
                                  cudaStream_t st) {
  if (count == 0 || n <= 0) return cudaSuccess;
  const size_t count4 = count / 4;
  const int blocks = static_cast<int>(std::min<size_t>((count4 + 255) / 256, static_cast<size_t>(device_sm_count()) * 8));
  sum_rank_parts_kernel<<<blocks, 256, 0, st>>>(parts, n, count4, last, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------ matmul_qt
// y[S,O] = x[S,I] . W^T for one MXFP4 / grouped-int4 matrix (kernels.rs:233-244, :276-296).
template <int FMT, int MT>
__global__ void __launch_bounds__(256) gemv_plain_kernel(const uint8_t* __restrict__ data,
                                                         const void* __restrict__ scale,
                                                         ExpertFormat f,
                                                         const uint16_t* __restrict__ xq,
                                                         const int32_t* __restrict__ xexp, int S,
                                                         int K, int O, float* __restrict__ y) {
  const int lane = threadIdx.x % 32;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int nw = gridDim.x * (blockDim.x / 32);
  const int row_groups = (O + 3) / 4;
  const int n_chunks = (S + MT - 1) / MT;
  const int n_tasks = row_groups * n_chunks;
  const size_t row_bytes = static_cast<size_t>(K) / 2;
  const size_t srow = scale_row_bytes(f, K);
  for (int task = gw; task < n_tasks; task += nw) {
    const int c = task / row_groups;
    const int o0 = (task % row_groups) * 4;
    const int s0 = c * MT, n = min(MT, S - s0);
    const uint8_t* rows[4];
    const void* srows[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int o = min(o0 + r, O - 1);  // duplicate the last row for a ragged group
      rows[r] = data + o * row_bytes;
      srows[r] = static_cast<const uint8_t*>(scale) + o * srow;
    }
    const uint16_t* xr[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) xr[m] = xq + static_cast<size_t>(s0 + (m < n ? m : 0)) * K;
    float acc[4][MT];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;
    gemv_accumulate<FMT, 4, MT>(rows, srows, xr, n, K, f, acc);
    warp_reduce_all<4, MT>(acc);
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m >= n) break;
      if (lane < 4 && o0 + lane < O) {
        const float unscale = exp2i(-xexp[s0 + m]);
        const float v = (lane == 0 ? acc[0][m] : lane == 1 ? acc[1][m] : lane == 2 ? acc[2][m] : acc[3][m]);
        y[static_cast<size_t>(s0 + m) * O + o0 + lane] = v * unscale;
      }
    }
  }
}

// Any shape: one thread per output, the reference's scalar element order in f32
// ((x * w) * scale, summed left to right) -- used when I is not a multiple of 32 or the group
// size is not, i.e. for the small ragged shapes the reference's own tests use.
__global__ void matmul_q_scalar_kernel(float* __restrict__ y, const void* __restrict__ x,
                                       int x_dtype, const uint8_t* __restrict__ data,
                                       const void* __restrict__ scale, ExpertFormat f, int S,
                                       int I, int O) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= S * O) return;
  const int s = idx / O, o = idx % O;
  const size_t rb = (static_cast<size_t>(I) + 1) / 2;
  const uint8_t* wr = data + o * rb;
  float a = 0.0f;
  if (f.fmt == kMxfp4) {
    const size_t bpr = (static_cast<size_t>(I) + 31) / 32;
    const uint8_t* bs = static_cast<const uint8_t*>(scale) + o * bpr;
    for (int k = 0; k < I; k++) {
      const uint8_t byte = wr[k >> 1];
      const uint8_t nib = (k & 1) ? (byte >> 4) : (byte & 0xF);
      const float mags[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
      float wv = mags[nib & 7];
      if (nib & 8) wv = -wv;
      float tv = __fmul_rn(load_elem(x, x_dtype, static_cast<size_t>(s) * I + k), wv);
      tv = __fmul_rn(tv, e8m0_to_f32(bs[k / 32]));
      a = __fadd_rn(a, tv);
    }
  } else {
    const size_t ng = (static_cast<size_t>(I) + f.group_size - 1) / f.group_size;
    for (int k = 0; k < I; k++) {
      const uint8_t byte = wr[k >> 1];
      const int nib = (k & 1) ? (byte >> 4) : (byte & 0xF);
      const size_t si = o * ng + k / f.group_size;
      const float sc = f.scale_dtype == kBF16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(scale)[si])
                                              : static_cast<const float*>(scale)[si];
      float tv = __fmul_rn(load_elem(x, x_dtype, static_cast<size_t>(s) * I + k), static_cast<float>(nib - 8));
      tv = __fmul_rn(tv, sc);
      a = __fadd_rn(a, tv);
    }
  }
  y[static_cast<size_t>(s) * O + o] = a;
}

size_t matmul_q_workspace_bytes(int s, int i) {
  return static_cast<size_t>(s) * i * sizeof(uint16_t) + static_cast<size_t>(s) * sizeof(int32_t) + 256;
}

template <int FMT>
static void launch_plain_fmt(int mt, dim3 grid, const uint8_t* data, const void* scale,
                             const ExpertFormat& f, const uint16_t* xq, const int32_t* xexp, int S,
                             int K, int O, float* y, cudaStream_t st) {
  switch (mt) {
    case 1: gemv_plain_kernel<FMT, 1><<<grid, 256, 0, st>>>(data, scale, f, xq, xexp, S, K, O, y); break;
    case 2: gemv_plain_kernel<FMT, 2><<<grid, 256, 0, st>>>(data, scale, f, xq, xexp, S, K, O, y); break;
    case 4: gemv_plain_kernel<FMT, 4><<<grid, 256, 0, st>>>(data, scale, f, xq, xexp, S, K, O, y); break;
    default: gemv_plain_kernel<FMT, 8><<<grid, 256, 0, st>>>(data, scale, f, xq, xexp, S, K, O, y); break;
  }
}

cudaError_t launch_matmul_q(float* y, const void* x, int x_dtype, const uint8_t* data,
                            const void* scale, const ExpertFormat& f, int s, int i, int o,
                            void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (s <= 0 || o <= 0) return cudaSuccess;
  const bool fast = (i % 32 == 0) && (f.fmt == kMxfp4 || f.group_size % 32 == 0);
  if (!fast || workspace == nullptr || ws_bytes < matmul_q_workspace_bytes(s, i)) {
    const int n = s * o;
    matmul_q_scalar_kernel<<<(n + 255) / 256, 256, 0, st>>>(y, x, x_dtype, data, scale, f, s, i, o);
    return cudaGetLastError();
  }
  uint16_t* xq = static_cast<uint16_t*>(workspace);
  int32_t* xexp = reinterpret_cast<int32_t*>(
      (reinterpret_cast<uintptr_t>(xq + static_cast<size_t>(s) * i) + 15) & ~uintptr_t(15));
  cudaError_t err = launch_prep_tokens(x, x_dtype, s, i, f.fmt, nullptr, xq, xexp, nullptr, st);
  if (err != cudaSuccess) return err;
  const int mt = s >= 8 ? 8 : (s >= 4 ? 4 : (s >= 2 ? 2 : 1));
  const int tasks = ((o + 3) / 4) * ((s + mt - 1) / mt);
  dim3 grid(gemv_grid(tasks));
  if (f.fmt == kMxfp4) launch_plain_fmt<kMxfp4>(mt, grid, data, scale, f, xq, xexp, s, i, o, y, st);
  else launch_plain_fmt<kInt4g>(mt, grid, data, scale, f, xq, xexp, s, i, o, y, st);
  return cudaGetLastError();
}

}  // namespace rmoe
