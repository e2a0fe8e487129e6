// dispatch.cu -- token -> expert dispatch: histogram, exclusive prefix sum, stable permute.
//
// rabbit applies each routed expert to "the tokens that picked it, in ascending token order"
// (glm52::moe::apply_single_expert, src/glm52/moe.rs:465-470) and walks experts in batch
// first-occurrence order (unique_experts, :333-344). Both are reproduced exactly, with no
// order-dependent atomics: every (token, slot) sets one bit in a per-expert token bitmap, a
// warp per expert prefix-sums the bitmap's popcounts, and a token's rank inside its expert is
// that prefix plus the popcount of the lower bits of its own word. Ranks therefore equal the
// ascending-token order by construction, independent of scheduling.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace rmoe {

__global__ void dispatch_mark_kernel(const int32_t* __restrict__ ids, int T, int k, int e_begin,
                                     int e_end, int words, uint32_t* __restrict__ bits,
                                     int32_t* __restrict__ first_occ) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= T * k) return;
  const int e = ids[q];
  if (e < e_begin || e >= e_end) return;
  const int t = q / k, el = e - e_begin;
  atomicOr(&bits[static_cast<size_t>(el) * words + (t >> 5)], 1u << (t & 31));
  atomicMin(&first_occ[el], q);
}

// One warp per local expert: exclusive popcount prefix over the bitmap words in use.
__global__ void dispatch_scan_kernel(const uint32_t* __restrict__ bits, int n_loc, int words,
                                     int nw, int32_t* __restrict__ wpre, int32_t* __restrict__ counts) {
  const int el = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (el >= n_loc) return;
  const uint32_t* b = bits + static_cast<size_t>(el) * words;
  int32_t* p = wpre + static_cast<size_t>(el) * words;
  int base = 0;
  for (int w0 = 0; w0 < nw; w0 += 32) {
    const int wi = w0 + lane;
    const int c = wi < nw ? __popc(b[wi]) : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    if (wi < nw) p[wi] = base + incl - c;
    base += __shfl_sync(kFull, incl, 31);
  }
  if (lane == 0) counts[el] = base;
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024); returns the total.
__device__ int block_exclusive_scan(int v, int& excl) {
  __shared__ int warp_tot[32];
  __shared__ int grand_total;
  const int lane = threadIdx.x % 32, wi = threadIdx.x / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int u = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) warp_tot[wi] = incl;
  __syncthreads();
  if (wi == 0) {
    const int nwarps = (blockDim.x + 31) / 32;
    int t = lane < nwarps ? warp_tot[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(kFull, ti, o);
      if (lane >= o) ti += u;
    }
    if (lane < nwarps) warp_tot[lane] = ti - t;  // exclusive prefix of warp totals
    if (lane == 31) grand_total = ti;
  }
  __syncthreads();
  excl = warp_tot[wi] + incl - v;
  const int total = grand_total;
  __syncthreads();
  return total;
}

// Single block (1024 threads): expert offsets, the chunk/task lists and the first-occurrence
// order (the placement itself follows in dispatch_perm_kernel, spread over the grid).
__global__ void __launch_bounds__(1024) dispatch_place_kernel(
    const int32_t* __restrict__ ids, const float* __restrict__ w, int T, int k, int e_begin,
    int n_loc, int words, int mt, int has_shared, const float* __restrict__ shared_gate_w,
    int tpc_gu, int tpc_gu_shared, int tpc_dn, DispatchBuffers d) {
  __shared__ int s_off[1025 + 1];
  __shared__ int s_chunk0[1025 + 1];
  const int tid = threadIdx.x;
  const int n_slots = n_loc + (has_shared ? 1 : 0);  // the shared expert is slot n_loc
  // counts -> offsets, chunks per slot -> chunk bases (n_slots <= 1025: loop twice if needed)
  int carry_off = 0, carry_ch = 0;
  for (int base = 0; base < n_slots; base += blockDim.x) {
    const int s = base + tid;
    int cnt = 0;
    if (s < n_slots) cnt = (s < n_loc) ? d.counts[s] : T;
    const int nch = (cnt + mt - 1) / mt;
    int ex_off, ex_ch;
    const int tot_off = block_exclusive_scan(cnt, ex_off);
    const int tot_ch = block_exclusive_scan(nch, ex_ch);
    if (s < n_slots) {
      s_off[s] = carry_off + ex_off;
      s_chunk0[s] = carry_ch + ex_ch;
      if (s == n_loc) d.counts[n_loc] = T;
    }
    carry_off += tot_off;
    carry_ch += tot_ch;
    __syncthreads();
  }
  if (tid == 0) {
    s_off[n_slots] = carry_off;
    s_chunk0[n_slots] = carry_ch;
    d.n_chunks[0] = carry_ch;
  }
  __syncthreads();
  for (int s = tid; s <= n_slots; s += blockDim.x) d.offsets[s] = s_off[s];
  const int n_routed_chunks = s_chunk0[n_loc];
  // chunk lists
  for (int s = tid; s < n_slots; s += blockDim.x) {
    const int cnt = s_off[s + 1] - s_off[s];
    const int c0 = s_chunk0[s];
    const int nch = (cnt + mt - 1) / mt;
    for (int i = 0; i < nch; i++) {
      const int c = c0 + i;
      d.ch_expert[c] = s;
      d.ch_pos[c] = s_off[s] + i * mt;
      d.ch_n[c] = min(mt, cnt - i * mt);
      d.ch_task_gu[c] = c < n_routed_chunks
                            ? c * tpc_gu
                            : n_routed_chunks * tpc_gu + (c - n_routed_chunks) * tpc_gu_shared;
      d.ch_task_dn[c] = c * tpc_dn;
    }
  }
  if (tid == 0) {
    const int nc = s_chunk0[n_slots];
    d.ch_task_gu[nc] = nc <= n_routed_chunks
                           ? nc * tpc_gu
                           : n_routed_chunks * tpc_gu + (nc - n_routed_chunks) * tpc_gu_shared;
    d.ch_task_dn[nc] = nc * tpc_dn;
  }
  // first-occurrence order of the local experts that were picked: slot q is the first
  // occurrence of its expert iff first_occ[expert] == q, so the order is a prefix count over
  // the slots (O(T k), not a scan of every expert per picked expert)
  {
    int carry = 0;
    for (int base = 0; base < T * k; base += blockDim.x) {
      const int q = base + tid;
      int flag = 0, e = -1;
      if (q < T * k) {
        e = ids[q];
        const int el = e - e_begin;
        flag = e >= 0 && el >= 0 && el < n_loc && d.first_occ[el] == q;
      }
      int ex;
      const int tot = block_exclusive_scan(flag, ex);
      if (flag) d.uniq[carry + ex] = e;
      carry += tot;
      __syncthreads();
    }
    if (tid == 0) d.n_uniq[0] = carry;
  }
}

// The stable placement of every (token, slot) and the shared expert's positions, one thread per
// slot over the whole grid (after dispatch_place_kernel wrote the expert offsets): a slot's
// position is its expert's offset plus the token's rank in the expert's bitmap.
__global__ void dispatch_perm_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w, int T, int k,
                                     int e_begin, int n_loc, int words, int has_shared,
                                     const float* __restrict__ shared_gate_w, DispatchBuffers d) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q < T * k) {
    const int e = ids[q];
    const int el = e - e_begin;
    if (e < 0 || el < 0 || el >= n_loc) {
      d.inv[q] = -1;
    } else {
      const int t = q / k;
      // a token that names an expert in two slots gets it once, with the first slot's weight
      // (apply_single_expert takes the first matching pick, src/glm52/moe.rs:465-470)
      bool dup = false;
      for (int j = t * k; j < q; j++) dup |= ids[j] == e;
      if (dup) {
        d.inv[q] = -1;
      } else {
        const uint32_t word = d.bits[static_cast<size_t>(el) * words + (t >> 5)];
        const int rank = d.wpre[static_cast<size_t>(el) * words + (t >> 5)] + __popc(word & ((1u << (t & 31)) - 1u));
        const int pos = d.offsets[el] + rank;
        d.perm_tok[pos] = t;
        d.perm_w[pos] = w[q];
        d.inv[q] = pos;
      }
    }
  }
  if (has_shared && q < T) {
    const int pos = d.offsets[n_loc] + q;
    d.perm_tok[pos] = q;
    d.perm_w[pos] = shared_gate_w ? shared_gate_w[q] : 1.0f;
  }
}

cudaError_t launch_dispatch(const int32_t* ids, const float* w, int T, int k, int e_begin,
                            int e_end, int mt, int has_shared, const float* shared_gate_w,
                            int inter, int shared_inter, int hidden, int rows_per_task_gu,
                            int rows_per_task_dn, const DispatchBuffers& d, cudaStream_t st) {
  const int n_loc = e_end - e_begin;
  if (n_loc + 1 > 1025 || T > d.words * 32) return cudaErrorInvalidValue;
  const int nw = (T + 31) / 32;
  cudaError_t err;
  if ((err = cudaMemsetAsync(d.bits, 0, sizeof(uint32_t) * static_cast<size_t>(n_loc) * d.words, st)))
    return err;
  if ((err = cudaMemsetAsync(d.first_occ, 0x7f, sizeof(int32_t) * n_loc, st))) return err;
  if (T * k > 0) {
    dispatch_mark_kernel<<<(T * k + 255) / 256, 256, 0, st>>>(ids, T, k, e_begin, e_end, d.words,
                                                              d.bits, d.first_occ);
  }
  dispatch_scan_kernel<<<(n_loc + 7) / 8, 256, 0, st>>>(d.bits, n_loc, d.words, nw, d.wpre,
                                                        d.counts);
  const int tpc_gu = inter / rows_per_task_gu;
  const int tpc_gu_sh = shared_inter > 0 ? shared_inter / rows_per_task_gu : 0;
  const int tpc_dn = hidden / rows_per_task_dn;
  dispatch_place_kernel<<<1, 1024, 0, st>>>(ids, w, T, k, e_begin, n_loc, d.words, mt, has_shared,
                                            shared_gate_w, tpc_gu, tpc_gu_sh, tpc_dn, d);
  const int n = std::max(T * k, T);
  if (n > 0)
    dispatch_perm_kernel<<<(n + 255) / 256, 256, 0, st>>>(ids, w, T, k, e_begin, n_loc, d.words, has_shared,
                                                          shared_gate_w, d);
  return cudaGetLastError();
}

// One token for the one-token expert kernel: positions by ascending expert id among the local
// slots, one chunk per position, the shared expert last. Fills what that kernel and the
// activation terms read (inv, the chunk table, perm_tok / perm_w, n_chunks, the shared offsets).
__global__ void dispatch_one_token_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w, int k,
                                          int e_begin, int e_end, int n_loc, int has_shared,
                                          const float* __restrict__ shared_gate_w, DispatchBuffers d) {
  const int lane = threadIdx.x;
  const int sid = lane < k ? ids[lane] : -1;
  const float wv = lane < k ? w[lane] : 0.0f;
  // a repeated expert counts once, at its first slot (the reference applies the first
  // matching pick, src/glm52/moe.rs:465-470); later repeats contribute nothing
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
}

cudaError_t launch_dispatch_one_token(const int32_t* ids, const float* w, int k, int e_begin, int e_end, int n_loc,
                                      int has_shared, const float* shared_gate_w, const DispatchBuffers& d,
                                      cudaStream_t st) {
  if (k > 32) return cudaErrorInvalidValue;
  dispatch_one_token_kernel<<<1, 32, 0, st>>>(ids, w, k, e_begin, e_end, n_loc, has_shared, shared_gate_w, d);
  return cudaGetLastError();
}

}  // namespace rmoe
