// route_small.cu -- the decode-sized (T <= 32) front end of the layer in two launches:
//
//  1. router_certified_kernel: every router logit as a value plus a rigorous bound on how far
//     the reference's own sequential f32 chain (kernels::matmul, src/kernels.rs:113-124) can be
//     from it. A warp per expert, each lane owning one contiguous H/32 slice of the dot product.
//  2. prologue_small_kernel (one block): top-k with a certificate that the reference picks the
//     same experts in the same order; tokens whose certificate fails recompute the contending
//     logits with the exact chain, so routing indices stay bit-exact. Then the dispatch
//     (positions grouped by expert, ascending token), the chunk lists, and the f16 activations.
//
// The bound. The reference computes S^_j = fl(S^_{j-1} + p^_j) with p^_j = fl(x_j w_j), so
// |S^_n - sum p_j| <= u/(1-u) * sum_j |S^_j| + u * sum_j |p_j| (u = 2^-24). With lane l's slice
// starting at the exact prefix O_l and local prefixes b_j, sum over the slice of |S_j| is at
// most c*|O_l| + sum_j |b_j| (c = slice length). The kernel's own f32 evaluation adds at most
// u * sum_l sum_j |b^_j| (local chains) + 6u * sum_l |B_l| (the 32-lane scan), so
//   err = (1.01 + 2nu) * u * ( sum_l (c|O_l| + 2 A_l + 6 |B_l|) + P (1 + nu) )
// with A_l = sum |b_j|, B_l the slice sum, P = sum |p_j|, n = H. Second-order terms are covered
// by the 1.01 and 2nu factors for any H with n*u < 0.01.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "pipe.cuh"
#include "select.cuh"
#include "terms.cuh"

namespace rmoe {

constexpr int kSmallT = 32;

// 8 consecutive elements of an f32 / bf16 row as f32.
__device__ __forceinline__ void load8(const void* p, int dtype, size_t idx, float (&v)[8]) {
  if (dtype == kBF16) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + idx));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      v[2 * q] = __uint_as_float(w[q] << 16);
      v[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    }
  } else {
    const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(p) + idx);
    const float4 a = __ldg(f), b = __ldg(f + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// grid: ceil(E/4) blocks of 4 warps; warp = one expert, all T tokens (groups of TB). Each
// lane's weight slice streams in batches of NB x 8 elements whose loads are all issued before
// the (serial) local chain consumes them.
template <int TB>
__global__ void __launch_bounds__(128) router_certified_kernel(
    const void* __restrict__ x, int x_dtype, const void* __restrict__ w, int w_dtype,
    float* __restrict__ mid, float* __restrict__ err, int T, int H, int E) {
  constexpr int NB = TB == 1 ? 8 : 4;
  const int e = blockIdx.x * 4 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (e >= E) return;
  const int c = H / 32;  // slice length (multiple of 8)
  const size_t wrow = static_cast<size_t>(e) * H + static_cast<size_t>(lane) * c;
  const float u = 5.9604645e-08f;  // 2^-24
  const float n = static_cast<float>(H);
  const float safety = 1.01f + 2.0f * n * u;
  for (int t0 = 0; t0 < T; t0 += TB) {
    float b[TB], A[TB], P[TB];
#pragma unroll
    for (int q = 0; q < TB; q++) b[q] = A[q] = P[q] = 0.0f;
    for (int j0 = 0; j0 < c; j0 += 8 * NB) {
      float wv[NB][8], xv[NB][TB][8];
#pragma unroll
      for (int bb = 0; bb < NB; bb++) {
        const int j = j0 + 8 * bb;
        if (j < c) {
          load8(w, w_dtype, wrow + j, wv[bb]);
#pragma unroll
          for (int q = 0; q < TB; q++)
            if (t0 + q < T)
              load8(x, x_dtype, static_cast<size_t>(t0 + q) * H + static_cast<size_t>(lane) * c + j, xv[bb][q]);
        }
      }
#pragma unroll
      for (int bb = 0; bb < NB; bb++) {
        if (j0 + 8 * bb >= c) break;
#pragma unroll
        for (int q = 0; q < TB; q++) {
          if (t0 + q >= T) break;
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float p = __fmul_rn(xv[bb][q][i], wv[bb][i]);
            b[q] = __fadd_rn(b[q], p);
            A[q] += fabsf(b[q]);
            P[q] += fabsf(p);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < TB; q++) {
      if (t0 + q >= T) break;
      // inclusive scan of slice sums across lanes -> exclusive prefix O_l and the total S
      float incl = b[q];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
      }
      const float O = incl - b[q];
      const float S = __shfl_sync(kFull, incl, 31);
      float term = static_cast<float>(c) * fabsf(O) + 2.0f * A[q] + 6.0f * fabsf(b[q]);
      float Pt = P[q];
      term = warp_sum(term);
      Pt = warp_sum(Pt);
      if (lane == 0) {
        const size_t o = static_cast<size_t>(t0 + q) * E + e;
        mid[o] = S;
        err[o] = safety * u * (term + Pt * (1.0f + n * u)) + 1e-37f;
      }
    }
  }
}

// One token (decode): a block of 4 warps per expert, 128 slices of c = H/128 elements. Every
// load of a lane's slice (up to 64 weights and 64 activations) is issued before the chain
// consumes any, so each warp has a single memory round trip. Same bound as above with the
// 128-slice scan: each slice sum passes through at most 5 (warp scan) + 4 (cross-warp) roundings,
// counted as 10 |B_l|.
// 8 elements of a DT row as raw 16-byte words (bf16: one word, f32: two) and their f32 values.
template <int DT>
__device__ __forceinline__ void load_raw8(const void* p, size_t idx, uint4 (&r)[2]) {
  if (DT == kBF16) {
    r[0] = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + idx));
  } else {
    const uint4* f = reinterpret_cast<const uint4*>(static_cast<const float*>(p) + idx);
    r[0] = __ldg(f);
    r[1] = __ldg(f + 1);
  }
}

template <int DT>
__device__ __forceinline__ void expand8(const uint4 (&r)[2], float (&v)[8]) {
  if (DT == kBF16) {
    const uint32_t w[4] = {r[0].x, r[0].y, r[0].z, r[0].w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      v[2 * q] = __uint_as_float(w[q] << 16);
      v[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    }
  } else {
    v[0] = __uint_as_float(r[0].x); v[1] = __uint_as_float(r[0].y);
    v[2] = __uint_as_float(r[0].z); v[3] = __uint_as_float(r[0].w);
    v[4] = __uint_as_float(r[1].x); v[5] = __uint_as_float(r[1].y);
    v[6] = __uint_as_float(r[1].z); v[7] = __uint_as_float(r[1].w);
  }
}

template <int XD, int WD>
__global__ void __launch_bounds__(128, 4) router_certified_t1_kernel(
    const void* __restrict__ x, const void* __restrict__ w, float* __restrict__ mid,
    float* __restrict__ err, int H) {
  __shared__ float s_tot[4], s_term[4], s_p[4];
  const int e = blockIdx.x;
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int c = H / 128;  // multiple of 8
  const size_t off = static_cast<size_t>(threadIdx.x) * c;
  const size_t wrow = static_cast<size_t>(e) * H + off;
  float b = 0.0f, A = 0.0f, P = 0.0f;
  for (int j0 = 0; j0 < c; j0 += 64) {
    uint4 wr[8][2], xr[8][2];
#pragma unroll
    for (int g = 0; g < 8; g++) {
      if (j0 + 8 * g < c) {
        load_raw8<WD>(w, wrow + j0 + 8 * g, wr[g]);
        load_raw8<XD>(x, off + j0 + 8 * g, xr[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < 8; g++) {
      if (j0 + 8 * g >= c) break;
      float wv[8], xv[8];
      expand8<WD>(wr[g], wv);
      expand8<XD>(xr[g], xv);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float p = __fmul_rn(xv[i], wv[i]);
        b = __fadd_rn(b, p);
        A += fabsf(b);
        P += fabsf(p);
      }
    }
  }
  float incl = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  float excl = __shfl_up_sync(kFull, incl, 1);
  if (lane == 0) excl = 0.0f;
  if (lane == 31) s_tot[wi] = incl;
  __syncthreads();
  float pref = 0.0f;
  for (int q = 0; q < wi; q++) pref += s_tot[q];
  const float O = pref + excl;
  float term = static_cast<float>(c) * fabsf(O) + 2.0f * A + 10.0f * fabsf(b);
  term = warp_sum(term);
  P = warp_sum(P);
  if (lane == 0) {
    s_term[wi] = term;
    s_p[wi] = P;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const float u = 5.9604645e-08f;  // 2^-24
    const float n = static_cast<float>(H);
    const float S = ((s_tot[0] + s_tot[1]) + s_tot[2]) + s_tot[3];
    const float tt = ((s_term[0] + s_term[1]) + s_term[2]) + s_term[3];
    const float Pt = ((s_p[0] + s_p[1]) + s_p[2]) + s_p[3];
    mid[e] = S;
    err[e] = (1.01f + 2.0f * n * u) * u * (tt + Pt * (1.0f + n * u)) + 1e-37f;
  }
}

cudaError_t launch_router_certified(const void* x, int x_dtype, const void* w, int w_dtype,
                                    float* mid, float* err, int T, int H, int E,
                                    cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (H % 256 != 0 || T > kSmallT) return cudaErrorInvalidValue;
  if (T == 1 && H % 1024 == 0) {
    if (x_dtype == kBF16 && w_dtype == kBF16) router_certified_t1_kernel<kBF16, kBF16><<<E, 128, 0, st>>>(x, w, mid, err, H);
    else if (x_dtype == kBF16) router_certified_t1_kernel<kBF16, kF32><<<E, 128, 0, st>>>(x, w, mid, err, H);
    else if (w_dtype == kBF16) router_certified_t1_kernel<kF32, kBF16><<<E, 128, 0, st>>>(x, w, mid, err, H);
    else router_certified_t1_kernel<kF32, kF32><<<E, 128, 0, st>>>(x, w, mid, err, H);
    return cudaGetLastError();
  }
  const int blocks = (E + 3) / 4;
  if (T == 1) router_certified_kernel<1><<<blocks, 128, 0, st>>>(x, x_dtype, w, w_dtype, mid, err, T, H, E);
  else router_certified_kernel<4><<<blocks, 128, 0, st>>>(x, x_dtype, w, w_dtype, mid, err, T, H, E);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
__device__ __forceinline__ bool ahead(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

__device__ __forceinline__ void warp_best(float& v, int& id) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(kFull, v, o);
    const int oid = __shfl_xor_sync(kFull, id, o);
    if (ahead(ov, oid, v, id)) {
      v = ov;
      id = oid;
    }
  }
}

// The reference chain for one (token, expert): a = -0.0; a = fl(a + fl(x_k * w_k)), k ascending.
// The 8192 adds are inherently serial; the loads run 32 elements ahead of the chain so only the
// add latency remains (~4 cycles per element).
__device__ __noinline__ float exact_logit(const void* x, int x_dtype, const void* w, int w_dtype, int t, int e,
                             int H) {
  float a = -0.0f;
  const size_t xo = static_cast<size_t>(t) * H, wo = static_cast<size_t>(e) * H;
  float xc[32], wc[32];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    load8(x, x_dtype, xo + 8 * q, *reinterpret_cast<float(*)[8]>(&xc[8 * q]));
    load8(w, w_dtype, wo + 8 * q, *reinterpret_cast<float(*)[8]>(&wc[8 * q]));
  }
  for (int k = 0; k < H; k += 32) {
    float xn[32], wn[32];
    const bool more = k + 32 < H;
    if (more) {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        load8(x, x_dtype, xo + k + 32 + 8 * q, *reinterpret_cast<float(*)[8]>(&xn[8 * q]));
        load8(w, w_dtype, wo + k + 32 + 8 * q, *reinterpret_cast<float(*)[8]>(&wn[8 * q]));
      }
    }
    float p[32];
#pragma unroll
    for (int i = 0; i < 32; i++) p[i] = __fmul_rn(xc[i], wc[i]);
#pragma unroll
    for (int i = 0; i < 32; i++) a = __fadd_rn(a, p[i]);
    if (more) {
#pragma unroll
      for (int i = 0; i < 32; i++) {
        xc[i] = xn[i];
        wc[i] = wn[i];
      }
    }
  }
  return a;
}


// Block-wide selection of the kk best (value, id) pairs (kk <= 32), one pair per thread (threads
// without an expert hold (-inf, unique id above every expert)). Two levels: each warp ranks its
// 32 pairs by shuffles and keeps its kk best; every kept candidate then counts the candidates
// ahead of it. Writes rank-ordered ids/values to out_id/out_v[0..kk). Two independent lists are
// ranked at once (`v2`/`out2_*`), sharing the barriers. Contains __syncthreads: call from all
// threads.

constexpr int kMaxPL = 32;  // experts per lane (E <= 1024)

// One block of 512 threads. Warp w routes tokens w, w + 16, ...; then the block builds the dispatch and
// converts the activations. Produces exactly what the generic route/dispatch/prep kernels do.
template <int PL>
__global__ void __launch_bounds__(512) prologue_small_kernel(SmallPrologue a, DispatchBuffers d) {
  __shared__ int s_ids[kSmallT * RMOE_MAX_TOPK_DEV];
  __shared__ float s_w[kSmallT * RMOE_MAX_TOPK_DEV];
  __shared__ int s_pos[kSmallT * RMOE_MAX_TOPK_DEV];
  __shared__ int s_nch[kSmallT * RMOE_MAX_TOPK_DEV];
  __shared__ int s_misc[4];
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int T = a.T, E = a.E, k = a.k;
  const int kk = min(k, E);

  // ---------------- 1a. route, one or two tokens: the whole block, one expert per thread
  const bool block_route = T <= 2 && E <= static_cast<int>(blockDim.x);
  if (block_route) {
    __shared__ float c1[kSmallT * RMOE_MAX_TOPK_DEV / 2], c2[kSmallT * RMOE_MAX_TOPK_DEV / 2];
    __shared__ int c1i[kSmallT * RMOE_MAX_TOPK_DEV / 2], c2i[kSmallT * RMOE_MAX_TOPK_DEV / 2];
    __shared__ int sel_id[RMOE_MAX_TOPK_DEV], lo_id[RMOE_MAX_TOPK_DEV];
    __shared__ float sel_v[RMOE_MAX_TOPK_DEV], lo_v[RMOE_MAX_TOPK_DEV];
    __shared__ float s_lo[1024], s_hi[1024];
    __shared__ float s_lk;
    __shared__ int s_nc;
    const int e = threadIdx.x;
    const bool valid = e < E;
    const int id = valid ? e : 0x40000000 + e;
    for (int t = 0; t < T; t++) {
      float lo = -INFINITY, hi = -INFINITY, v = -INFINITY;
      if (valid) {
        const float m = a.mid[static_cast<size_t>(t) * E + e];
        const float r = a.err[static_cast<size_t>(t) * E + e];
        lo = __fsub_rd(m, r);
        hi = __fadd_ru(m, r);
        v = m;
        if (a.bias) {
          const float bb = a.bias[e];
          lo = __fadd_rn(lo, bb);
          hi = __fadd_rn(hi, bb);
          v = __fadd_rn(v, bb);
        }
        s_lo[e] = lo;
        s_hi[e] = hi;
      }
      // winners by value, and the kk-th largest lower bound
      // certified set: the kk-th largest lower bound Lk; exactly kk experts reaching it with
      // their upper bounds are the top kk, ranked by their values
      const float Lk = block_kth_largest(lo, id, kk, c1, c1i, &s_lk);
      const bool cont = valid && hi >= Lk;
      const int n_cont = __syncthreads_count(cont);
      const bool set_ok = n_cont == kk;
      if (set_ok) block_rank_few(cont, v, id, kk, c2, c2i, &s_nc, sel_id, sel_v);
      const int r = threadIdx.x;
      const bool pair_ok = !set_ok || r >= kk - 1 || s_lo[sel_id[r]] > s_hi[sel_id[r + 1]];
      const bool order_ok = __syncthreads_and(pair_ok);
      if (!set_ok) {
        // exact chains for every contender, then the selection on exact values
        float ex = -INFINITY;
        if (valid && hi >= Lk) {
          ex = exact_logit(a.x, a.x_dtype, a.w, a.w_dtype, t, e, a.H);
          if (a.bias) ex = __fadd_rn(ex, a.bias[e]);
        }
        block_select2(ex, ex, id, kk, c1, c1i, c2, c2i, sel_id, sel_v, lo_id, lo_v);
        if (threadIdx.x == 0) atomicAdd(a.fallback_count, 1u);
      }
      if (wi == 0) {
        if (lane == 0) {
          const int pend = set_ok && !order_ok ? 1 : 0;
          a.pending[t] = pend;
          if (pend) atomicAdd(a.order_pending_count, 1u);
        }
        const float sv = lane < kk ? sel_v[lane] : -INFINITY;
        const float mx = __shfl_sync(kFull, sv, 0);
        const float exv = lane < kk ? exp_f32(__fsub_rn(sv, mx)) : 0.0f;
        float sum = 0.0f;
        for (int j = 0; j < kk; j++) sum = __fadd_rn(sum, __shfl_sync(kFull, exv, j));
        if (lane < k) {
          const float wv = lane < kk ? __fdiv_rn(exv, sum) : 0.0f;
          const int sid = lane < kk ? sel_id[lane] : -1;
          s_ids[t * k + lane] = sid;
          s_w[t * k + lane] = wv;
          a.ids[t * k + lane] = sid;
          a.rw[t * k + lane] = wv;
        }
      }
      __syncthreads();
    }
  }

  // ---------------- 1b. route (warp per token)
  for (int t = wi; t < (block_route ? 0 : T); t += blockDim.x / 32) {
    float lo[PL], hi[PL], v[PL];
#pragma unroll
    for (int q = 0; q < PL; q++) {
      const int e = q * 32 + lane;
      if (e < E) {
        const float m = a.mid[static_cast<size_t>(t) * E + e];
        const float r = a.err[static_cast<size_t>(t) * E + e];
        float l = __fsub_rd(m, r), h = __fadd_ru(m, r), vv = m;
        if (a.bias) {
          const float bb = a.bias[e];
          l = __fadd_rn(l, bb);
          h = __fadd_rn(h, bb);
          vv = __fadd_rn(vv, bb);
        }
        lo[q] = l;
        hi[q] = h;
        v[q] = vv;
      } else {
        lo[q] = hi[q] = v[q] = -INFINITY;
      }
    }
    // k-th largest lower bound
    unsigned taken = 0;
    float Lk = INFINITY;
    for (int r = 0; r < kk; r++) {
      float bv = -INFINITY;
      int bid = 0x7fffffff;
#pragma unroll
      for (int q = 0; q < PL; q++) {
        const int e = q * 32 + lane;
        if (e < E && !((taken >> q) & 1) && ahead(lo[q], e, bv, bid)) {
          bv = lo[q];
          bid = e;
        }
      }
      warp_best(bv, bid);
      if ((bid & 31) == lane) taken |= 1u << (bid >> 5);
      Lk = bv;
    }
    // contenders: hi >= Lk
    int n_cont = 0;
#pragma unroll
    for (int q = 0; q < PL; q++) {
      const int e = q * 32 + lane;
      n_cont += __popc(__ballot_sync(kFull, e < E && hi[q] >= Lk));
    }
    // selection by value, then the order certificate
    auto select = [&](int* sel_id, float* sel_v) {
      unsigned tk = 0;
      for (int r = 0; r < kk; r++) {
        float bv = -INFINITY;
        int bid = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < PL; q++) {
          const int e = q * 32 + lane;
          if (e < E && !((tk >> q) & 1) && ahead(v[q], e, bv, bid)) {
            bv = v[q];
            bid = e;
          }
        }
        warp_best(bv, bid);
        if ((bid & 31) == lane) tk |= 1u << (bid >> 5);
        if (lane == r) {
          *sel_id = bid;
          *sel_v = bv;
        }
      }
    };
    int sel_id = -1;
    float sel_v = -INFINITY;
    select(&sel_id, &sel_v);
    // interval of the winner of each rank
    float my_lo = -INFINITY, my_hi = INFINITY;
#pragma unroll
    for (int q = 0; q < PL; q++) {
      // fetch lo/hi of expert sel_id: it lives in lane sel_id%32, slot sel_id/32
      const int src = sel_id >= 0 ? (sel_id & 31) : 0;
      const float l = __shfl_sync(kFull, lo[q], src);
      const float h = __shfl_sync(kFull, hi[q], src);
      if (sel_id >= 0 && q == (sel_id >> 5)) {
        my_lo = l;
        my_hi = h;
      }
    }
    const float next_hi = __shfl_down_sync(kFull, my_hi, 1);
    const bool pair_ok = (lane >= kk - 1) || (my_lo > next_hi);
    const bool set_ok = n_cont == kk;
    const bool order_ok = __all_sync(kFull, pair_ok);
    if (set_ok && !order_ok) {
      // the expert set is certain, only the rank order of near-tied winners is not: the expert
      // products do not depend on it, so the exact order is resolved off the critical path
      if (lane == 0) {
        a.pending[t] = 1;
        atomicAdd(a.order_pending_count, 1u);
      }
    } else if (lane == 0) {
      a.pending[t] = 0;
    }
    if (!set_ok) {
      // exact chains for every contender, then select on exact values among them
#pragma unroll
      for (int q = 0; q < PL; q++) {
        const int e = q * 32 + lane;
        const bool cont = e < E && hi[q] >= Lk;
        if (cont) {
          float ex = exact_logit(a.x, a.x_dtype, a.w, a.w_dtype, t, e, a.H);
          if (a.bias) ex = __fadd_rn(ex, a.bias[e]);
          v[q] = ex;
        } else {
          v[q] = -INFINITY;
        }
      }
      select(&sel_id, &sel_v);
      if (lane == 0) atomicAdd(a.fallback_count, 1u);
    }
    // softmax over the winners (qwen38/moe.rs:64-75): exp(l - max), sum from +0.0, divide
    const float mx = __shfl_sync(kFull, sel_v, 0);
    const float exv = lane < kk ? exp_f32(__fsub_rn(sel_v, mx)) : 0.0f;
    float sum = 0.0f;
    for (int j = 0; j < kk; j++) sum = __fadd_rn(sum, __shfl_sync(kFull, exv, j));
    if (lane < k) {
      const float wv = lane < kk ? __fdiv_rn(exv, sum) : 0.0f;
      const int id = lane < kk ? sel_id : -1;
      s_ids[t * k + lane] = id;
      s_w[t * k + lane] = wv;
      a.ids[t * k + lane] = id;
      a.rw[t * k + lane] = wv;
    }
  }
  __syncthreads();

  // ---------------- 2. dispatch: positions grouped by expert id, ascending token inside
  const int n = T * k;
  for (int q = threadIdx.x; q < n; q += blockDim.x) {
    const int e = s_ids[q];
    const bool local = e >= a.e_begin && e < a.e_end;
    // (rank-order-independent: positions depend only on the expert set of each token)
    int pos = -1, nch = 0;
    if (local) {
      int less = 0, same = 0, first = 1;
      const int t = q / k;
      for (int r = 0; r < n; r++) {
        const int e2 = s_ids[r];
        if (e2 < a.e_begin || e2 >= a.e_end) continue;
        if (e2 < e || (e2 == e && r / k < t)) less++;
        if (e2 == e) {
          same++;
          if (r / k < t) first = 0;
        }
      }
      pos = less;
      if (first) nch = (same + a.mt - 1) / a.mt;
    }
    s_pos[q] = pos;
    s_nch[q] = nch;  // chunks, counted once per expert on its first (lowest-token) entry
    d.inv[q] = pos;
    if (local) {
      d.perm_tok[pos] = q / k;
      d.perm_w[pos] = s_w[q];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int routed = 0, chunks = 0;
    for (int q = 0; q < n; q++) {
      routed += s_pos[q] >= 0;
      chunks += s_nch[q];
    }
    s_misc[0] = routed;
    s_misc[1] = chunks;
  }
  __syncthreads();
  const int routed = s_misc[0], routed_chunks = s_misc[1];
  // chunk lists: each expert's first entry writes its chunks; chunk base = chunks of experts
  // with a lower position
  for (int q = threadIdx.x; q < n; q += blockDim.x) {
    if (s_nch[q] == 0) continue;
    int base = 0;
    for (int r = 0; r < n; r++)
      if (s_nch[r] > 0 && s_pos[r] < s_pos[q]) base += s_nch[r];
    int cnt = 0;
    const int e = s_ids[q];
    for (int r = 0; r < n; r++) cnt += s_ids[r] == e;
    for (int i = 0; i < s_nch[q]; i++) {
      const int c = base + i;
      d.ch_expert[c] = e - a.e_begin;
      d.ch_pos[c] = s_pos[q] + i * a.mt;
      d.ch_n[c] = min(a.mt, cnt - i * a.mt);
      d.ch_task_gu[c] = c * a.tpc_gu;
      d.ch_task_dn[c] = c * a.tpc_dn;
    }
  }
  const int sh_chunks = a.has_shared ? (T + a.mt - 1) / a.mt : 0;
  for (int i = threadIdx.x; i < sh_chunks; i += blockDim.x) {
    const int c = routed_chunks + i;
    d.ch_expert[c] = a.n_loc;
    d.ch_pos[c] = routed + i * a.mt;
    d.ch_n[c] = min(a.mt, T - i * a.mt);
    d.ch_task_gu[c] = routed_chunks * a.tpc_gu + i * a.tpc_gu_shared;
    d.ch_task_dn[c] = c * a.tpc_dn;
  }
  if (threadIdx.x == 0) {
    const int nc = routed_chunks + sh_chunks;
    d.n_chunks[0] = nc;
    d.ch_task_gu[nc] = routed_chunks * a.tpc_gu + sh_chunks * a.tpc_gu_shared;
    d.ch_task_dn[nc] = nc * a.tpc_dn;
    d.offsets[a.n_loc] = routed;                             // first shared position
    d.offsets[a.n_loc + (a.has_shared ? 1 : 0)] = routed + (a.has_shared ? T : 0);  // total
  }

  // ---------------- 3. activations: f16 copy with a power-of-two scale, shared gate.
  // The whole block works on one token at a time, 8 consecutive elements per thread.
  __shared__ float red[2][16];
  for (int t = 0; t < T; t++) {
    float amax = 0.0f, dot = 0.0f;
    for (int i = threadIdx.x * 8; i < a.H; i += blockDim.x * 8) {
      float xv[8];
      load8(a.x, a.x_dtype, static_cast<size_t>(t) * a.H + i, xv);
#pragma unroll
      for (int q = 0; q < 8; q++) {
        amax = fmaxf(amax, fabsf(xv[q]));
        if (a.gvec) dot = fmaf(xv[q], a.gvec[i + q], dot);
      }
    }
    amax = warp_max(amax);
    dot = warp_sum(dot);
    if (lane == 0) {
      red[0][wi] = amax;
      red[1][wi] = dot;
    }
    __syncthreads();
    if (wi == 0) {
      float am = lane < (int)(blockDim.x / 32) ? red[0][lane] : 0.0f;
      float dt = lane < (int)(blockDim.x / 32) ? red[1][lane] : 0.0f;
      am = warp_max(am);
      dt = warp_sum(dt);
      if (lane == 0) {
        red[0][0] = am;
        red[1][0] = dt;
      }
    }
    __syncthreads();
    const int ex = f16_row_exponent(red[0][0]);
    const float g = a.gvec ? sigmoid_ref(red[1][0]) : 1.0f;
    if (threadIdx.x == 0) {
      a.xexp[t] = ex;
      a.gate[t] = g;
      if (a.has_shared) {
        d.perm_w[routed + t] = g;
        d.perm_tok[routed + t] = t;
      }
    }
    const float sc = exp2i(ex);
    for (int i = threadIdx.x * 8; i < a.H; i += blockDim.x * 8) {
      float xv[8];
      load8(a.x, a.x_dtype, static_cast<size_t>(t) * a.H + i, xv);
      uint16_t hv[8];
#pragma unroll
      for (int q = 0; q < 8; q++) {
        // int4 layout pairs (0,4),(1,5),(2,6),(3,7) inside each 8-group
        const int dst = a.fmt == kInt4g ? (q < 4 ? 2 * q : 2 * (q - 4) + 1) : q;
        hv[dst] = __half_as_ushort(__float2half_rn(xv[q] * sc));
      }
      uint4 pk;
      pk.x = hv[0] | (static_cast<uint32_t>(hv[1]) << 16);
      pk.y = hv[2] | (static_cast<uint32_t>(hv[3]) << 16);
      pk.z = hv[4] | (static_cast<uint32_t>(hv[5]) << 16);
      pk.w = hv[6] | (static_cast<uint32_t>(hv[7]) << 16);
      *reinterpret_cast<uint4*>(a.xq + static_cast<size_t>(t) * a.H + i) = pk;
    }
    __syncthreads();
  }
}


// ---------------------------------------------------------------------------------------
// One token, one launch: blocks [0, E/2) compute the certified router logits of two experts each
// (16 warps, 512 slices of H/512 elements, the loads of both experts issued before either chain;
// each slice sum passes through at most 5 + 15 + 1 roundings in the scan, counted as 22 |B_l|);
// the next block the shared-expert gate
// sigmoid(x . g); blocks after it the four-term E2M1 expansion of x (one warp per 32-block).
// The block that finishes last (a device counter, reset by it) runs the top-k with its
// certificate and the dispatch of the single token.
template <int XD, int WD>
__global__ void __launch_bounds__(512, 2) decode_front_kernel(DecodeFront a) {
  __shared__ float s_tot[2][16], s_term[2][16], s_p[2][16];
  __shared__ int s_last;
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int E = a.E, H = a.H;
  const int nrb = (E + 1) / 2;  // router blocks: experts 2b, 2b + 1
  const int b = blockIdx.x;
  if (a.trace && b == 0 && threadIdx.x == 0) a.trace[0] = global_ns();
  // the expert kernel that follows may launch now: it waits for this grid before reading
  if (threadIdx.x == 0) griddep_launch_dependents();
  if (b < nrb) {
    const int c = H / 512;  // multiple of 8
    const size_t off = static_cast<size_t>(threadIdx.x) * c;
    float bs[2] = {0.0f, 0.0f}, A[2] = {0.0f, 0.0f}, P[2] = {0.0f, 0.0f};
    for (int j0 = 0; j0 < c; j0 += 16) {
      uint4 wr[2][2][2], xr[2][2];
#pragma unroll
      for (int g = 0; g < 2; g++) {
        if (j0 + 8 * g < c) {
          load_raw8<XD>(a.x, off + j0 + 8 * g, xr[g]);
#pragma unroll
          for (int q = 0; q < 2; q++) {
            const int e = min(2 * b + q, E - 1);
            load_raw8<WD>(a.w, static_cast<size_t>(e) * H + off + j0 + 8 * g, wr[q][g]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < 2; g++) {
        if (j0 + 8 * g >= c) break;
        float xv[8];
        expand8<XD>(xr[g], xv);
#pragma unroll
        for (int q = 0; q < 2; q++) {
          float wv[8];
          expand8<WD>(wr[q][g], wv);
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float pp = __fmul_rn(xv[i], wv[i]);
            bs[q] = __fadd_rn(bs[q], pp);
            A[q] += fabsf(bs[q]);
            P[q] += fabsf(pp);
          }
        }
      }
    }
    float excl[2];
#pragma unroll
    for (int q = 0; q < 2; q++) {
      float incl = bs[q];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
      }
      excl[q] = __shfl_up_sync(kFull, incl, 1);
      if (lane == 0) excl[q] = 0.0f;
      if (lane == 31) s_tot[q][wi] = incl;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 2; q++) {
      float pref = 0.0f;
      for (int w = 0; w < wi; w++) pref += s_tot[q][w];
      const float O = pref + excl[q];
      float term = static_cast<float>(c) * fabsf(O) + 2.0f * A[q] + 22.0f * fabsf(bs[q]);
      term = warp_sum(term);
      const float Pw = warp_sum(P[q]);
      if (lane == 0) {
        s_term[q][wi] = term;
        s_p[q][wi] = Pw;
      }
    }
    __syncthreads();
    if (threadIdx.x < 2 && 2 * b + static_cast<int>(threadIdx.x) < E) {
      const int q = threadIdx.x;
      const float u = 5.9604645e-08f;  // 2^-24
      const float n = static_cast<float>(H);
      float S = 0.0f, tt = 0.0f, Pt = 0.0f;
      for (int w = 0; w < 16; w++) {
        S += s_tot[q][w];
        tt += s_term[q][w];
        Pt += s_p[q][w];
      }
      a.mid[2 * b + q] = S;
      a.err[2 * b + q] = (1.01f + 2.0f * n * u) * u * (tt + Pt * (1.0f + n * u)) + 1e-37f;
    }
  } else if (b == nrb) {
    // the one-token expert kernel's counters (it reads them only after this grid completes)
    for (int i = threadIdx.x; i < a.zero_n; i += blockDim.x) a.zero_buf[i] = 0;
    if (a.gvec) {
      float dot = 0.0f;
      for (int i = threadIdx.x * 8; i < H; i += 512 * 8) {
        float xv[8];
        load8(a.x, XD, i, xv);
#pragma unroll
        for (int q = 0; q < 8; q++) dot = fmaf(xv[q], a.gvec[i + q], dot);
      }
      dot = warp_sum(dot);
      if (lane == 0) s_tot[0][wi] = dot;
      __syncthreads();
      if (threadIdx.x == 0) {
        float d = 0.0f;
        for (int q = 0; q < 16; q++) d += s_tot[0][q];
        a.gate[0] = sigmoid_ref(d);
      }
    } else if (threadIdx.x == 0) {
      a.gate[0] = 1.0f;
    }
  } else {
    const int blk = (b - nrb - 1) * 16 + wi;  // 32-block of x
    if (blk < H / 32) {
      const float r = load_elem(a.x, XD, static_cast<size_t>(blk) * 32 + lane);
      warp_terms4(r, a.xt + blk * 16, H / 2, a.xsf + blk, H / 32);
    }
  }
  // ---- the last block to finish runs the front end
  if (a.trace && threadIdx.x == 0) atomicMax(a.trace + (b < nrb ? 1 : 2), global_ns());
  // the block's writes (ordered before thread 0 by the barrier) are released by thread 0's
  // counter increment; the last block's thread 0 acquires everyone's through the same atomic
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.counter) : "memory");
    s_last = old == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __shared__ float c1[16 * RMOE_MAX_TOPK_DEV], c2[16 * RMOE_MAX_TOPK_DEV];
  __shared__ int c1i[16 * RMOE_MAX_TOPK_DEV], c2i[16 * RMOE_MAX_TOPK_DEV];
  __shared__ int sel_id[RMOE_MAX_TOPK_DEV], lo_id[RMOE_MAX_TOPK_DEV];
  __shared__ float sel_v[RMOE_MAX_TOPK_DEV], lo_v[RMOE_MAX_TOPK_DEV];
  __shared__ float s_lo[512], s_hi[512], s_v[512];
  __shared__ __align__(16) uint32_t s_key[512];
  __shared__ __align__(16) unsigned long long s_cand[16 * RMOE_MAX_TOPK_DEV];
  __shared__ int s_top[RMOE_MAX_TOPK_DEV];
  __shared__ float s_lk;
  // (the shared expert's gate, read at the end: its load is issued now)
  const float gate_pf = threadIdx.x == 0 && a.has_shared ? __ldcg(a.gate) : 0.0f;
  const int k = a.k, kk = min(k, E);
  const int e = threadIdx.x;
  const bool valid = e < E;
  const int id = valid ? e : 0x40000000 + e;
  float lo = -INFINITY, hi = -INFINITY, v = -INFINITY;
  if (valid) {
    const float m = __ldcg(a.mid + e);
    const float r = __ldcg(a.err + e);
    lo = __fsub_rd(m, r);
    hi = __fadd_ru(m, r);
    v = m;
    if (a.bias) {
      const float bb = a.bias[e];
      lo = __fadd_rn(lo, bb);
      hi = __fadd_rn(hi, bb);
      v = __fadd_rn(v, bb);
    }
  }
  s_lo[e] = lo;
  s_hi[e] = hi;
  s_v[e] = v;
  if (a.trace && threadIdx.x == 0) a.trace[3] = global_ns();
  // certified set: the kk-th largest lower bound Lk; exactly kk experts reaching it with their
  // upper bounds are the top kk (every other value is below all of theirs), ranked by value.
  // Lk by counting, in two levels: each entry's rank by (lo desc, id asc) inside its warp (the
  // warp's keys through shared memory), then the warps' first kk entries ranked against each
  // other; the one of rank kk - 1 holds Lk. Ids ascend with the thread index (invalid entries
  // after every expert), so ties go to the lower index.
  const uint32_t klo = order_key(lo);
  s_key[e] = klo;
  __syncwarp();
  {
    int wr = 0;
    const uint32_t* wk = s_key + wi * 32;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const uint4 q = *reinterpret_cast<const uint4*>(wk + j);
      wr += (q.x > klo || (q.x == klo && j + 0 < lane)) ? 1 : 0;
      wr += (q.y > klo || (q.y == klo && j + 1 < lane)) ? 1 : 0;
      wr += (q.z > klo || (q.z == klo && j + 2 < lane)) ? 1 : 0;
      wr += (q.w > klo || (q.w == klo && j + 3 < lane)) ? 1 : 0;
    }
    if (wr < kk) s_cand[wi * kk + wr] = (static_cast<unsigned long long>(klo) << 32) | (0xffffffffu - e);
  }
  __syncthreads();
  if (wi == 0) {
    // warp 0 merges the 16 warps' sorted lists (lane w holds the head of warp w's list): each
    // round takes the largest head -- (key, then the lower id) as one 64-bit value -- and
    // advances that list
    const int nw = blockDim.x / 32;
    int h = 0;
    for (int r = 0; r < kk; r++) {
      const unsigned long long hv = lane < nw && h < kk ? s_cand[lane * kk + h] : 0ull;
      const uint32_t hi = static_cast<uint32_t>(hv >> 32), lo32 = static_cast<uint32_t>(hv);
      const uint32_t mhi = __reduce_max_sync(kFull, hi);
      const uint32_t mlo = __reduce_max_sync(kFull, hi == mhi ? lo32 : 0u);
      if (hv != 0ull && hi == mhi && lo32 == mlo) h++;
      if (lane == 0) {
        const int idx = static_cast<int>(0xffffffffu - mlo);
        s_top[r] = idx;
        if (r == kk - 1) s_lk = s_lo[idx];
      }
    }
  }
  __syncthreads();
  const float Lk = s_lk;
  if (a.trace && threadIdx.x == 0) a.trace[4] = global_ns();
  const bool cont = valid && hi >= Lk;
  const int n_cont = __syncthreads_count(cont);
  const bool set_ok = n_cont == kk;
  bool order_ok = true;
  if (set_ok) {
    // the kk contenders are the top kk by lo (hi >= lo >= Lk for each): warp 0 ranks them by
    // (value desc, id asc) and checks that neighbours' intervals are apart
    if (wi != 0) return;
    const bool has = lane < kk;
    const int ei = has ? s_top[lane] : 0x7fffffff;
    const float vi = has ? s_v[ei] : -INFINITY;
    const uint32_t kv = has ? order_key(vi) : 0u;
    int vr = 0;
    for (int j = 0; j < kk; j++) {
      const uint32_t kj = __shfl_sync(kFull, kv, j);
      const int ej = __shfl_sync(kFull, ei, j);
      vr += (kj > kv || (kj == kv && ej < ei)) ? 1 : 0;
    }
    if (has) {
      sel_id[vr] = ei;
      sel_v[vr] = vi;
    }
    __syncwarp();
    const bool pok = lane >= kk - 1 || s_lo[sel_id[lane]] > s_hi[sel_id[lane + 1]];
    order_ok = __all_sync(kFull, pok);
  }
  if (!set_ok) {
    float ex = -INFINITY;
    if (valid && hi >= Lk) {
      ex = exact_logit(a.x, XD, a.w, WD, 0, e, H);
      if (a.bias) ex = __fadd_rn(ex, a.bias[e]);
    }
    block_select2(ex, ex, id, kk, c1, c1i, c2, c2i, sel_id, sel_v, lo_id, lo_v);
    if (threadIdx.x == 0) atomicAdd(a.fallback_count, 1u);
  }
  if (a.trace && threadIdx.x == 0) a.trace[5] = global_ns();
  if (wi == 0) {
    if (lane == 0) {
      const int pend = set_ok && !order_ok ? 1 : 0;
      a.pending[0] = pend;
      if (pend) atomicAdd(a.order_pending_count, 1u);
    }
    const float sv = lane < kk ? sel_v[lane] : -INFINITY;
    const float mx = __shfl_sync(kFull, sv, 0);
    // (single-precision exp here: the weights come from certified values, a few ulps from the
    // reference's anyway, and the double-precision exp would cost ~0.45 us on the critical path)
    const float exv = lane < kk ? expf(__fsub_rn(sv, mx)) : 0.0f;
    float sum = 0.0f;
    for (int j = 0; j < kk; j++) sum = __fadd_rn(sum, __shfl_sync(kFull, exv, j));
    const float wv = lane < kk ? __fdiv_rn(exv, sum) : 0.0f;
    const int sid = lane < kk ? sel_id[lane] : -1;
    if (lane < k) {
      a.ids[lane] = sid;
      a.rw[lane] = wv;
    }
    // dispatch of the one token: positions by ascending expert id, one chunk per position
    const bool local = lane < kk && sid >= a.e_begin && sid < a.e_end;
    int pos = 0;
    for (int j = 0; j < kk; j++) {
      const int o = __shfl_sync(kFull, sid, j);
      pos += (o >= a.e_begin && o < a.e_end && o < sid) ? 1 : 0;
    }
    const int n_routed = __popc(__ballot_sync(kFull, local));
    if (lane < k) a.d.inv[lane] = local ? pos : -1;
    if (local) {
      a.d.ch_expert[pos] = sid - a.e_begin;
      a.d.ch_pos[pos] = pos;
      a.d.ch_n[pos] = 1;
      a.d.perm_tok[pos] = 0;
      a.d.perm_w[pos] = wv;
    }
    if (lane == 0) {
      if (a.has_shared) {
        a.d.ch_expert[n_routed] = a.n_loc;
        a.d.ch_pos[n_routed] = n_routed;
        a.d.ch_n[n_routed] = 1;
        a.d.perm_tok[n_routed] = 0;
        a.d.perm_w[n_routed] = gate_pf;
      }
      a.d.n_chunks[0] = n_routed + a.has_shared;
      a.d.offsets[a.n_loc] = n_routed;
      a.d.offsets[a.n_loc + a.has_shared] = n_routed + a.has_shared;
      *a.counter = 0;
      if (a.trace) a.trace[6] = global_ns();
    }
  }
}

cudaError_t launch_decode_front(const DecodeFront& a, cudaStream_t st) {
  if (a.H % 4096 != 0 || a.E > 512 || a.k > RMOE_MAX_TOPK_DEV) return cudaErrorInvalidValue;
  const int blocks = (a.E + 1) / 2 + 1 + (a.H / 32 + 15) / 16;
  if (a.x_dtype == kBF16 && a.w_dtype == kBF16) decode_front_kernel<kBF16, kBF16><<<blocks, 512, 0, st>>>(a);
  else if (a.x_dtype == kBF16) decode_front_kernel<kBF16, kF32><<<blocks, 512, 0, st>>>(a);
  else if (a.w_dtype == kBF16) decode_front_kernel<kF32, kBF16><<<blocks, 512, 0, st>>>(a);
  else decode_front_kernel<kF32, kF32><<<blocks, 512, 0, st>>>(a);
  return cudaGetLastError();
}

constexpr int kResolveThreads = 128;  // threads per (token, winner) chain
constexpr int kResolvePer = 64;       // elements each thread holds per segment
constexpr int kResolveSeg = kResolveThreads * kResolvePer;

// Final routing in the reference's rank order. Tokens whose order certificate failed get the
// exact reference chain for each of their k winners (the set is already certain) --
// a = -0.0; a = fl(a + fl(x_i * w_i)), i ascending -- and are re-ranked on those values; other
// tokens are copied. One 128-thread block per (token, winner): the token's activations and the
// winner's router row are loaded into registers at once (64 elements a thread), then the chain
// runs through the threads in element order, each adding its own products and handing the sum to
// the next (shuffles inside a warp, shared memory between warps). The block is small (no dynamic
// shared memory) so it runs beside the expert kernels on the side stream. The last block of a
// token (per-token counter) ranks the k exact values and writes the token's routing.
template <int XD, int WD>
__global__ void __launch_bounds__(kResolveThreads) resolve_order_kernel(SmallPrologue a, int32_t* ids_final,
                                                                        float* w_final, float* exact_v,
                                                                        int32_t* done_cnt) {
  constexpr int XV = XD == kBF16 ? 1 : 2, WV = WD == kBF16 ? 1 : 2;  // uint4 per 8 elements
  __shared__ float hand[kResolveThreads / 32];
  __shared__ int last;
  const int k = a.k, kk = min(a.k, a.E);
  const int t = blockIdx.x / kk, j = blockIdx.x % kk;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  if (!a.pending[t]) {
    if (j == 0 && tid < k) {
      ids_final[t * k + tid] = a.ids[t * k + tid];
      w_final[t * k + tid] = a.rw[t * k + tid];
    }
    return;
  }
  const int e = a.ids[t * k + j];
  const uint4* xg = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) +
                                                   static_cast<size_t>(t) * a.H * (XD == kBF16 ? 2 : 4));
  const uint4* wg = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.w) +
                                                   static_cast<size_t>(e) * a.H * (WD == kBF16 ? 2 : 4));
  float acc = -0.0f;
  for (int seg = 0; seg < a.H; seg += kResolveSeg) {
    const int i0 = seg + tid * kResolvePer;
    const int n = max(0, min(kResolvePer, a.H - i0));  // a multiple of 16 (H % 16 == 0)
    uint4 xr[kResolvePer / 8][XV], wr[kResolvePer / 8][WV];
#pragma unroll
    for (int c = 0; c < kResolvePer / 8; c++) {
      if (8 * c < n) {
#pragma unroll
        for (int q = 0; q < XV; q++) xr[c][q] = __ldg(xg + (i0 / 8 + c) * XV + q);
#pragma unroll
        for (int q = 0; q < WV; q++) wr[c][q] = __ldg(wg + (i0 / 8 + c) * WV + q);
      }
    }
    for (int w = 0; w < kResolveThreads / 32; w++) {
      if (warp == w) {
        for (int l = 0; l < 32; l++) {
          if (lane == l) {
#pragma unroll
            for (int c = 0; c < kResolvePer / 8; c++) {
              if (8 * c < n) {
                float xv[8], wv[8];
                uint4 x2[2] = {xr[c][0], xr[c][XV - 1]}, w2[2] = {wr[c][0], wr[c][WV - 1]};
                expand8<XD>(x2, xv);
                expand8<WD>(w2, wv);
#pragma unroll
                for (int i = 0; i < 8; i++) acc = __fadd_rn(acc, __fmul_rn(xv[i], wv[i]));
              }
            }
          }
          acc = __shfl_sync(kFull, acc, l);
        }
        if (lane == 0) hand[w] = acc;
      }
      __syncthreads();
      acc = hand[w];
    }
  }
  if (tid == 0) {
    if (a.bias) acc = __fadd_rn(acc, a.bias[e]);
    exact_v[t * k + j] = acc;
    __threadfence();
    last = atomicAdd(done_cnt + t, 1) == kk - 1;
  }
  __syncthreads();
  if (!last || warp != 0) return;
  __threadfence();
  // the token's last block: rank the kk exact values (ties: lower expert id first)
  const int el = lane < kk ? a.ids[t * k + lane] : -1;
  const float v = lane < kk ? __ldcg(exact_v + t * k + lane) : -INFINITY;
  if (lane == 0) done_cnt[t] = 0;  // (zero for the next call)
  unsigned tk = 0;
  int sel_id = -1;
  float sel_v = -INFINITY;
  for (int r = 0; r < kk; r++) {
    float bv = (el >= 0 && !tk) ? v : -INFINITY;
    int bid = (el >= 0 && !tk) ? el : 0x7fffffff;
    warp_best(bv, bid);
    if (bid == el) tk = 1;
    if (lane == r) {
      sel_id = bid;
      sel_v = bv;
    }
  }
  const float mx = __shfl_sync(kFull, sel_v, 0);
  const float exv = lane < kk ? exp_f32(__fsub_rn(sel_v, mx)) : 0.0f;
  float sum = 0.0f;
  for (int i = 0; i < kk; i++) sum = __fadd_rn(sum, __shfl_sync(kFull, exv, i));
  if (lane < k) {
    ids_final[t * k + lane] = lane < kk ? sel_id : -1;
    w_final[t * k + lane] = lane < kk ? __fdiv_rn(exv, sum) : 0.0f;
  }
}

cudaError_t launch_resolve_order(const SmallPrologue& a, int32_t* ids_final, float* w_final, float* exact_v,
                                 int32_t* done_cnt, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  const int kk = min(a.k, a.E);
  if (a.H % 16 != 0 || kk <= 0) return cudaErrorInvalidValue;
  auto go = [&](auto kern) -> cudaError_t {
    kern<<<a.T * kk, kResolveThreads, 0, st>>>(a, ids_final, w_final, exact_v, done_cnt);
    return cudaGetLastError();
  };
  if (a.x_dtype == kBF16 && a.w_dtype == kBF16) return go(resolve_order_kernel<kBF16, kBF16>);
  if (a.x_dtype == kBF16) return go(resolve_order_kernel<kBF16, kF32>);
  if (a.w_dtype == kBF16) return go(resolve_order_kernel<kF32, kBF16>);
  return go(resolve_order_kernel<kF32, kF32>);
}

cudaError_t launch_prologue_small(const SmallPrologue& a, const DispatchBuffers& d,
                                  cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  if (a.T > kSmallT || a.k > RMOE_MAX_TOPK_DEV || a.E > 1024) return cudaErrorInvalidValue;
  if (a.E <= 64) prologue_small_kernel<2><<<1, 512, 0, st>>>(a, d);
  else if (a.E <= 256) prologue_small_kernel<8><<<1, 512, 0, st>>>(a, d);
  else if (a.E <= 512) prologue_small_kernel<16><<<1, 512, 0, st>>>(a, d);
  else prologue_small_kernel<32><<<1, 512, 0, st>>>(a, d);
  return cudaGetLastError();
}

}  // namespace rmoe
