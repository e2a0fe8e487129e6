// select.cuh -- block-wide top-k selection by (value desc, id asc) with warp reductions.
#pragma once

#include "common.cuh"

namespace rmoe {

// Order-preserving 32-bit key of a float (larger value -> larger key; -0 and +0 equal, as the
// float comparison in ahead() treats them).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One selection round over a warp: the lane entry ahead of all others (largest key, then
// smallest id) among those not yet taken. Returns its id; *val gets its value.
__device__ __forceinline__ int warp_pick(uint32_t key, int id, float v, bool taken, float* val) {
  const uint32_t m = __reduce_max_sync(kFull, taken ? 0u : key);
  const int w = __reduce_min_sync(kFull, (!taken && key == m) ? id : 0x7fffffff);
  const unsigned who = __ballot_sync(kFull, !taken && key == m && id == w);
  *val = __shfl_sync(kFull, v, __ffs(who) - 1);
  return w;
}

// Top-kk of (v, id) and of (v2, id) over the block (one entry per thread, ids distinct), each
// by (value desc, id asc) -- the order ahead() defines -- into out_id/out_v and out2_id/out2_v.
// Every warp first selects its own top-kk of both lists (kk rounds of warp reductions); then
// warp 0 merges the warps' sorted lists of the first and warp 1 those of the second (one list
// head per lane, kk rounds). cand/cand_i/cand2/cand2_i: nw * kk scratch entries each.
__device__ __forceinline__ void block_select2(float v, float v2, int id, int kk, float* cand, int* cand_i,
                              float* cand2, int* cand2_i, int* out_id, float* out_v,
                              int* out2_id, float* out2_v) {
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nw = blockDim.x / 32;
  {
    const uint32_t k1 = order_key(v), k2 = order_key(v2);
    bool t1 = false, t2 = false;
    for (int r = 0; r < kk; r++) {
      float a1, a2;
      const int w1 = warp_pick(k1, id, v, t1, &a1);
      const int w2 = warp_pick(k2, id, v2, t2, &a2);
      t1 = t1 || id == w1;
      t2 = t2 || id == w2;
      if (lane == 0) {
        cand[wi * kk + r] = a1;
        cand_i[wi * kk + r] = w1;
        cand2[wi * kk + r] = a2;
        cand2_i[wi * kk + r] = w2;
      }
    }
  }
  __syncthreads();
  if (wi < 2) {
    const float* cv = wi == 0 ? cand : cand2;
    const int* ci = wi == 0 ? cand_i : cand2_i;
    int h = 0;  // head of list `lane` (lanes >= nw hold none)
    for (int r = 0; r < kk; r++) {
      const bool has = lane < nw && h < kk;
      const float hv = has ? cv[lane * kk + h] : -INFINITY;
      const int hid = has ? ci[lane * kk + h] : 0x7fffffff;
      float val;
      const int w = warp_pick(has ? order_key(hv) : 0u, hid, hv, !has, &val);
      if (has && hid == w) h++;
      if (lane == 0) {
        if (wi == 0) {
          out_id[r] = w;
          out_v[r] = val;
        } else {
          out2_id[r] = w;
          out2_v[r] = val;
        }
      }
    }
  }
  __syncthreads();
}

// The value ranked kk - 1 by (value desc, id asc) over the block (one entry per thread, ids
// distinct), to every thread: each warp selects its own top kk, warp 0 merges the warps' lists.
// cand/cand_i: nw * kk scratch entries; s_out: one shared float.
__device__ __forceinline__ float block_kth_largest(float v, int id, int kk, float* cand, int* cand_i, float* s_out) {
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nw = blockDim.x / 32;
  {
    const uint32_t key = order_key(v);
    bool taken = false;
    for (int r = 0; r < kk; r++) {
      float a;
      const int w = warp_pick(key, id, v, taken, &a);
      taken = taken || id == w;
      if (lane == 0) {
        cand[wi * kk + r] = a;
        cand_i[wi * kk + r] = w;
      }
    }
  }
  __syncthreads();
  if (wi == 0) {
    int h = 0;
    float last = 0.0f;
    for (int r = 0; r < kk; r++) {
      const bool has = lane < nw && h < kk;
      const float hv = has ? cand[lane * kk + h] : -INFINITY;
      const int hid = has ? cand_i[lane * kk + h] : 0x7fffffff;
      const int w = warp_pick(has ? order_key(hv) : 0u, hid, hv, !has, &last);
      if (has && hid == w) h++;
    }
    if (lane == 0) *s_out = last;
  }
  __syncthreads();
  return *s_out;
}

// Exactly kk (<= 32) threads of the block have cont set: their (v, id) ranked by (value desc,
// id asc) into out_id/out_v[0 .. kk) (one warp ranks them). cv/ci: 32 scratch entries; s_cnt: a
// shared int.
__device__ __forceinline__ void block_rank_few(bool cont, float v, int id, int kk, float* cv, int* ci, int* s_cnt,
                                               int* out_id, float* out_v) {
  if (threadIdx.x == 0) *s_cnt = 0;
  __syncthreads();
  if (cont) {
    const int slot = atomicAdd(s_cnt, 1);
    cv[slot] = v;
    ci[slot] = id;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const bool has = lane < kk;
    const float hv = has ? cv[lane] : -INFINITY;
    const int hid = has ? ci[lane] : 0x7fffffff;
    const uint32_t key = has ? order_key(hv) : 0u;
    bool taken = !has;
    for (int r = 0; r < kk; r++) {
      float a;
      const int w = warp_pick(key, hid, hv, taken, &a);
      taken = taken || hid == w;
      if (lane == 0) {
        out_id[r] = w;
        out_v[r] = a;
      }
    }
  }
  __syncthreads();
}

}  // namespace rmoe
