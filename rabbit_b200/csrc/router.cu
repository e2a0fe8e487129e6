// router.cu -- router logits (bit-exact with the reference's sequential f32 dot) and the
// warp-per-token top-k selectors (softmax/renormalise for Qwen, sigmoid+bias grouped for GLM).
#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "pipe.cuh"
#include "select.cuh"

namespace rmoe {

// ---------------------------------------------------------------------------------------
// Exact router logits. rabbit's kernels::matmul (src/kernels.rs:113-124) computes every logit
// as `xs.iter().zip(wr).map(|(a, b)| a * b).sum()`: a left-to-right chain of separately rounded
// f32 multiplies and adds starting from -0.0. Routing indices are only bit-exact if every logit
// is, so each output element here is exactly that chain (__fmul_rn / __fadd_rn cannot be
// contracted into FMAs). Parallelism comes from the (token, expert) grid, never from the sum.
// ---------------------------------------------------------------------------------------

// Small T: a block is 32 experts (lanes) x BT tokens (warps). The [32 x KC] weight tile and
// [BT x KC] token tile are staged in shared memory.
template <int BT>
__global__ void __launch_bounds__(32 * BT) router_exact_small_kernel(
    const void* __restrict__ x, int x_dtype, const void* __restrict__ w, int w_dtype,
    float* __restrict__ logits, int T, int H, int E) {
  constexpr int KC = 64;
  __shared__ float ws[32][KC + 1];
  __shared__ float xs[BT][KC];
  const int lane = threadIdx.x, ty = threadIdx.y;
  const int tid = ty * 32 + lane;
  const int e0 = blockIdx.x * 32, t0 = blockIdx.y * BT;
  const int e = e0 + lane, t = t0 + ty;
  float acc = -0.0f;
  constexpr int NT = 32 * BT;
  for (int k0 = 0; k0 < H; k0 += KC) {
    const int kc = min(KC, H - k0);
    __syncthreads();
    for (int q = tid; q < 32 * KC; q += NT) {
      int r = q / KC, c = q % KC;
      float v = 0.0f;
      if (e0 + r < E && c < kc) v = load_elem(w, w_dtype, static_cast<size_t>(e0 + r) * H + k0 + c);
      ws[r][c] = v;
    }
    for (int q = tid; q < BT * KC; q += NT) {
      int r = q / KC, c = q % KC;
      float v = 0.0f;
      if (t0 + r < T && c < kc) v = load_elem(x, x_dtype, static_cast<size_t>(t0 + r) * H + k0 + c);
      xs[r][c] = v;
    }
    __syncthreads();
    for (int c = 0; c < kc; c++) acc = __fadd_rn(acc, __fmul_rn(xs[ty][c], ws[lane][c]));
  }
  if (e < E && t < T) logits[static_cast<size_t>(t) * E + e] = acc;
}

// Large T: 64 tokens x 64 experts per 256-thread block, each thread 4x4 independent chains
// (register tiling only re-uses operands; every chain still walks k in order).
__global__ void __launch_bounds__(256) router_exact_tiled_kernel(
    const void* __restrict__ x, int x_dtype, const void* __restrict__ w, int w_dtype,
    float* __restrict__ logits, int T, int H, int E) {
  constexpr int BM = 64, BN = 64, KC = 16;
  __shared__ __align__(16) float xs[KC][BM + 4];
  __shared__ __align__(16) float ws[KC][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int t0 = blockIdx.y * BM, e0 = blockIdx.x * BN;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) acc[a][b] = -0.0f;
  // each thread stages 4 elements of each tile: row = tid / 4, cols 4*(tid%4) .. +3
  const int lr = threadIdx.x / 4, lc = (threadIdx.x % 4) * 4;
  for (int k0 = 0; k0 < H; k0 += KC) {
    float xv[4], wv[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      int kk = k0 + lc + q;
      xv[q] = (t0 + lr < T && kk < H) ? load_elem(x, x_dtype, static_cast<size_t>(t0 + lr) * H + kk) : 0.0f;
      wv[q] = (e0 + lr < E && kk < H) ? load_elem(w, w_dtype, static_cast<size_t>(e0 + lr) * H + kk) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; q++) {
      xs[lc + q][lr] = xv[q];
      ws[lc + q][lr] = wv[q];
    }
    __syncthreads();
    const int kc = min(KC, H - k0);
    if (kc == KC) {
#pragma unroll
      for (int c = 0; c < KC; c++) {
        float4 xa = *reinterpret_cast<const float4*>(&xs[c][ty * 4]);
        float4 wb = *reinterpret_cast<const float4*>(&ws[c][tx * 4]);
        const float xr[4] = {xa.x, xa.y, xa.z, xa.w};
        const float wr[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int b = 0; b < 4; b++) acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(xr[a], wr[b]));
      }
    } else {
      for (int c = 0; c < kc; c++) {
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int b = 0; b < 4; b++)
            acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(xs[c][ty * 4 + a], ws[c][tx * 4 + b]));
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    int t = t0 + ty * 4 + a;
    if (t >= T) continue;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      int e = e0 + tx * 4 + b;
      if (e < E) logits[static_cast<size_t>(t) * E + e] = acc[a][b];
    }
  }
}

// Few tokens: one warp per (token, expert) chain, 8 experts of one token per 256-thread block
// with the token's row in shared memory. Per 1024-element chunk the lanes form the products
// (fmul, coalesced weight loads) into the warp's buffer and lane 0 adds them in k order; the
// next chunk's weights are loaded before that serial run, so their latency hides behind it.
// The chain (x[k] * w[e][k] added from -0.0 in k order) is exactly the reference matmul's.
constexpr int kRwChunk = 1024;
template <int D>
__device__ __forceinline__ void load8_t(const void* p, size_t i, float (&v)[8]) {
  if (D == kBF16) {
    const uint4 r = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i);
    const uint32_t q[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[2 * j] = __uint_as_float(q[j] << 16);
      v[2 * j + 1] = __uint_as_float(q[j] & 0xffff0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// H % 1024 == 0. Lane l holds elements u * 256 + 8 l .. + 7 of a chunk (u < 4), 16-byte loads.
template <int XD, int WD>
__global__ void __launch_bounds__(256) router_exact_warp_kernel(const void* __restrict__ x, const void* __restrict__ w,
                                                                float* __restrict__ logits, int T, int H, int E) {
  extern __shared__ __align__(16) float rw_smem[];
  float* xs = rw_smem;                                           // [H]
  const int wi = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* buf = rw_smem + H + wi * kRwChunk;                     // [kRwChunk] per warp
  const int blocks_per_t = (E + 7) / 8;
  const int t = blockIdx.x / blocks_per_t;
  const int e = (blockIdx.x % blocks_per_t) * 8 + wi;
  for (int k = threadIdx.x * 8; k < H; k += blockDim.x * 8) {
    float v[8];
    load8_t<XD>(x, static_cast<size_t>(t) * H + k, v);
#pragma unroll
    for (int j = 0; j < 8; j++) xs[k + j] = v[j];
  }
  __syncthreads();
  if (e >= E) return;
  const size_t wrow = static_cast<size_t>(e) * H;
  float wv[4][8];
  auto load_chunk = [&](int c0) {
#pragma unroll
    for (int u = 0; u < 4; u++) load8_t<WD>(w, wrow + c0 + u * 256 + lane * 8, wv[u]);
  };
  float acc = -0.0f;
  load_chunk(0);
  for (int c0 = 0; c0 < H; c0 += kRwChunk) {
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int kk = u * 256 + lane * 8 + j;
        buf[kk] = __fmul_rn(xs[c0 + kk], wv[u][j]);
      }
    if (c0 + kRwChunk < H) load_chunk(c0 + kRwChunk);
    __syncwarp();
    if (lane == 0) {
      // 16 products per step; the next step's shared-memory loads are issued before this step's
      // dependent adds, so only the add latency remains
      float4 q[4], nq[4];
#pragma unroll
      for (int u = 0; u < 4; u++) q[u] = *reinterpret_cast<const float4*>(buf + 4 * u);
      for (int i = 0; i < kRwChunk; i += 16) {
        if (i + 16 < kRwChunk) {
#pragma unroll
          for (int u = 0; u < 4; u++) nq[u] = *reinterpret_cast<const float4*>(buf + i + 16 + 4 * u);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
          acc = __fadd_rn(acc, q[u].x);
          acc = __fadd_rn(acc, q[u].y);
          acc = __fadd_rn(acc, q[u].z);
          acc = __fadd_rn(acc, q[u].w);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) q[u] = nq[u];
      }
    }
    __syncwarp();
  }
  if (lane == 0) logits[static_cast<size_t>(t) * E + e] = acc;
}

// One token: a block owns 32 experts. Three producer warps stream the 32 router rows through a ring
// of slabs (one bulk copy per slab: the rows' 256-element pieces stored contiguously, rows 16
// bytes apart beyond their length so 16-byte reads by the 32 lanes hit distinct banks -- the
// slab layout written once at router upload) and form the products x[k] * w[e][k] of each slab
// into a double-buffered [32][256] product tile; the chain warp's lane e then adds its expert's
// products in k order. The chain is the reference's (fmul then fadd per element, from -0.0) and
// its serial add latency -- H dependent adds, ~4.5 cycles each when fed from shared memory -- is
// the kernel's bound: the chain lanes do nothing else and the 32 chains of a block advance
// together. (Per-row 512-byte copies, 32 per slab, measured 3.5x slower: the copy engine's
// per-request cost, not bandwidth, paced them.) Needs T == 1 and H % 256 == 0.
constexpr int kRcSlabEl = 256;           // elements per slab
constexpr int kRcProd = 3;               // producer warps (8-element pieces of every row slab, round robin)
constexpr int kRcThreads = 32 * (kRcProd + 1);  // warps 0-2 producers, warp 3 the chains (its own scheduler)

// (d0, d1) = (a0 * b0, a1 * b1) on f32 bit patterns, each rounded to nearest even
__device__ __forceinline__ void mul2_rn(uint32_t& d0, uint32_t& d1, uint32_t a0, uint32_t a1, uint32_t b0, uint32_t b1) {
  uint64_t d;
  const uint64_t a = static_cast<uint64_t>(a0) | (static_cast<uint64_t>(a1) << 32);
  const uint64_t b = static_cast<uint64_t>(b0) | (static_cast<uint64_t>(b1) << 32);
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  d0 = static_cast<uint32_t>(d);
  d1 = static_cast<uint32_t>(d >> 32);
}

template <int WD>
struct RcLayout {
  static constexpr int esz = WD == kBF16 ? 2 : 4;
  static constexpr int nring = WD == kBF16 ? 6 : 3;              // router-row slabs in flight
  static constexpr int row_bytes = kRcSlabEl * esz;
  static constexpr int pitch = row_bytes + 16;
  static constexpr int ring = 0;                                  // [nring][32][pitch]
  static constexpr int prod = ring + nring * 32 * pitch;        // [2][32][kRcSlabEl + 4] f32
  static constexpr int prod_pitch = kRcSlabEl + 4;
  static constexpr int xs = prod + 2 * 32 * prod_pitch * 4;       // [H] f32, then [H] bf16 staging
  __host__ __device__ static size_t bars(int H) { return xs + static_cast<size_t>(H) * 6; }
  static size_t bytes(int H) { return bars(H) + (nring + 5) * 8; }
};

// The slab layout: block b, slab j = rows 32 b .. 32 b + 31, elements 256 j .. 256 j + 255, row r at
// byte r * pitch of the slab's 32 * pitch bytes (rows past E zero).
__global__ void router_slab_relayout_kernel(const uint8_t* __restrict__ w, int esz, int E, int H,
                                            uint8_t* __restrict__ dst) {
  const int row_bytes = kRcSlabEl * esz, pitch = row_bytes + 16, nslab = H / kRcSlabEl;
  const int chunks = row_bytes / 16;
  const long long n = static_cast<long long>((E + 31) / 32) * nslab * 32 * chunks;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % chunks);
    const long long rr = i / chunks;
    const int r = static_cast<int>(rr % 32);
    const long long bj = rr / 32;
    const int j = static_cast<int>(bj % nslab), b = static_cast<int>(bj / nslab);
    const int e = b * 32 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (e < E) v = *reinterpret_cast<const uint4*>(w + (static_cast<size_t>(e) * H + static_cast<size_t>(j) * kRcSlabEl) * esz + c * 16);
    *reinterpret_cast<uint4*>(dst + (static_cast<size_t>(bj) * 32 + r) * pitch + c * 16) = v;
  }
}

size_t router_slab_bytes(int E, int H, int w_dtype) {
  if (H % kRcSlabEl) return 0;
  const int esz = w_dtype == kBF16 ? 2 : 4;
  return static_cast<size_t>((E + 31) / 32) * (H / kRcSlabEl) * 32 * (kRcSlabEl * esz + 16);
}

cudaError_t launch_router_slabs(const void* w, int w_dtype, int E, int H, uint8_t* dst, cudaStream_t st) {
  if (H % kRcSlabEl || reinterpret_cast<uintptr_t>(w) % 16) return cudaErrorInvalidValue;
  router_slab_relayout_kernel<<<1184, 256, 0, st>>>(static_cast<const uint8_t*>(w), w_dtype == kBF16 ? 2 : 4, E, H, dst);
  return cudaGetLastError();
}

template <int XD, int WD>
__global__ void __launch_bounds__(kRcThreads) router_exact_chain_kernel(const void* __restrict__ x,
                                                                        const uint8_t* __restrict__ wslab,
                                                                        float* __restrict__ logits, int H, int E,
                                                                        unsigned* err) {
  using Lo = RcLayout<WD>;
  extern __shared__ __align__(16) uint8_t rc_smem[];
  uint8_t* ring = rc_smem + Lo::ring;
  float* prod = reinterpret_cast<float*>(rc_smem + Lo::prod);
  float* xs = reinterpret_cast<float*>(rc_smem + Lo::xs);
  uint64_t* bars = reinterpret_cast<uint64_t*>(rc_smem + Lo::bars(H));
  uint64_t* wfull = bars;                        // [Lo::nring] slab landed
  uint64_t* pfull = bars + Lo::nring;            // [2] products formed (one arrival per producer thread)
  uint64_t* pempty = bars + Lo::nring + 2;       // [2] products consumed (32 chain arrivals)
  uint64_t* xbar = bars + Lo::nring + 4;         // the token's row landed
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nslab = H / kRcSlabEl;
  if (threadIdx.x == 0) {
    for (int q = 0; q < Lo::nring; q++) mbar_init(&wfull[q], 1);
    mbar_init(&pfull[0], 32 * kRcProd);
    mbar_init(&pfull[1], 32 * kRcProd);
    mbar_init(&pempty[0], 32);
    mbar_init(&pempty[1], 32);
    mbar_init(xbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) griddep_launch_dependents();  // (the top-k waits for this grid's logits)
  if (warp < kRcProd) {
    // ---- producers: thread (warp h, lane r) forms row r's products of the slab's 8-element
    // pieces h, h + kRcProd, ...
    const int r = lane, h = warp;
    const uint8_t* wblk = wslab + static_cast<size_t>(blockIdx.x) * nslab * 32 * Lo::pitch;
    auto issue = [&](int j) {  // (warp 0, lane 0: the whole slab in one copy)
      const int q = j % Lo::nring;
      if (lane == 0) {
        mbar_arrive_expect_tx(&wfull[q], 32 * Lo::pitch);
        bulk_g2s_once(ring + q * 32 * Lo::pitch, wblk + static_cast<size_t>(j) * 32 * Lo::pitch, 32 * Lo::pitch, &wfull[q]);
      }
    };
    // the token's row by one bulk copy (f32 straight into xs; bf16 into the staging area, then
    // widened), so its latency overlaps the first slabs' instead of a chain of small loads
    const int xbytes = H * (XD == kBF16 ? 2 : 4);
    uint8_t* xdst = XD == kBF16 ? reinterpret_cast<uint8_t*>(xs + H) : reinterpret_cast<uint8_t*>(xs);
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(xbar, xbytes);
      bulk_g2s(xdst, x, xbytes, xbar);
    }
    if (warp == 0)
      for (int j = 0; j < min(Lo::nring, nslab); j++) issue(j);
    bool ok = __all_sync(kFull, mbar_wait_bounded(xbar, 0, err, 0x1000000u));
    if (XD == kBF16 && ok) {
      const uint16_t* xb = reinterpret_cast<const uint16_t*>(xdst);
      for (int i = threadIdx.x * 8; i < H; i += 32 * kRcProd * 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xb + i);
        *reinterpret_cast<float4*>(xs + i) = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                                                         __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u));
        *reinterpret_cast<float4*>(xs + i + 4) = make_float4(__uint_as_float(raw.z << 16), __uint_as_float(raw.z & 0xFFFF0000u),
                                                             __uint_as_float(raw.w << 16), __uint_as_float(raw.w & 0xFFFF0000u));
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kRcProd) : "memory");
    int issued = min(Lo::nring, nslab);
    for (int j = 0; j < nslab && ok; j++) {
      const int q = j % Lo::nring, pb = j & 1;
      ok = __all_sync(kFull, mbar_wait_bounded(&wfull[q], (j / Lo::nring) & 1, err, 0x1000000u));
      if (ok && j >= 2) ok = __all_sync(kFull, mbar_wait_bounded(&pempty[pb], ((j - 2) >> 1) & 1, err, 0x2000000u));
      if (!ok) break;
      const uint8_t* src = ring + (q * 32 + r) * Lo::pitch;
      const float* xk = xs + j * kRcSlabEl;
      float* dst = prod + (pb * 32 + r) * Lo::prod_pitch;
#pragma unroll
      for (int c = 8 * h; c < kRcSlabEl; c += 8 * kRcProd) {
        uint32_t wv[8];  // f32 bit patterns
        if (WD == kBF16) {
          const uint4 raw = *reinterpret_cast<const uint4*>(src + c * 2);
          wv[0] = raw.x << 16; wv[1] = raw.x & 0xFFFF0000u; wv[2] = raw.y << 16; wv[3] = raw.y & 0xFFFF0000u;
          wv[4] = raw.z << 16; wv[5] = raw.z & 0xFFFF0000u; wv[6] = raw.w << 16; wv[7] = raw.w & 0xFFFF0000u;
        } else {
          const uint4 r0 = *reinterpret_cast<const uint4*>(src + c * 4);
          const uint4 r1 = *reinterpret_cast<const uint4*>(src + c * 4 + 16);
          wv[0] = r0.x; wv[1] = r0.y; wv[2] = r0.z; wv[3] = r0.w; wv[4] = r1.x; wv[5] = r1.y; wv[6] = r1.z; wv[7] = r1.w;
        }
        const uint4 x0 = *reinterpret_cast<const uint4*>(xk + c);
        const uint4 x1 = *reinterpret_cast<const uint4*>(xk + c + 4);
        // products two at a time (mul.rn.f32x2: each half rounded like __fmul_rn; stored, never fused)
        uint4 p0, p1;
        mul2_rn(p0.x, p0.y, x0.x, x0.y, wv[0], wv[1]);
        mul2_rn(p0.z, p0.w, x0.z, x0.w, wv[2], wv[3]);
        mul2_rn(p1.x, p1.y, x1.x, x1.y, wv[4], wv[5]);
        mul2_rn(p1.z, p1.w, x1.z, x1.w, wv[6], wv[7]);
        *reinterpret_cast<uint4*>(dst + c) = p0;
        *reinterpret_cast<uint4*>(dst + c + 4) = p1;
      }
      mbar_arrive(&pfull[pb]);
      // every producer warp is done with slot q: warp 0 refills it
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kRcProd) : "memory");
      if (warp == 0 && j + Lo::nring < nslab) {
        issue(j + Lo::nring);
        issued = j + Lo::nring + 1;
      }
    }
    if (!ok) {
      if (warp == 0)  // copies still in flight land (bounded) before the block leaves
        for (int j = max(0, issued - Lo::nring); j < issued; j++)
          mbar_wait_bounded(&wfull[j % Lo::nring], (j / Lo::nring) & 1, err, 0x1000000u, 1000000ull);
    }
  } else {
    // ---- chains: lane e adds its expert's products in k order
    float acc = -0.0f;
    bool ok = true;
    for (int j = 0; j < nslab; j++) {
      const int pb = j & 1;
      ok = __all_sync(kFull, mbar_wait_bounded(&pfull[pb], (j >> 1) & 1, err, 0x4000000u));
      if (!ok) break;
      const float* pr = prod + (pb * 32 + lane) * Lo::prod_pitch;
      // 16 products in registers while the next 16 load (the loads' latency stays off the chain)
      float4 q[4], nq[4];
#pragma unroll
      for (int u = 0; u < 4; u++) q[u] = *reinterpret_cast<const float4*>(pr + 4 * u);
#pragma unroll 2
      for (int c = 0; c < kRcSlabEl; c += 16) {
#pragma unroll
        for (int u = 0; u < 4; u++)
          nq[u] = c + 16 < kRcSlabEl ? *reinterpret_cast<const float4*>(pr + c + 16 + 4 * u) : q[u];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          acc = __fadd_rn(acc, q[u].x);
          acc = __fadd_rn(acc, q[u].y);
          acc = __fadd_rn(acc, q[u].z);
          acc = __fadd_rn(acc, q[u].w);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) q[u] = nq[u];
      }
      mbar_arrive(&pempty[pb]);
    }
    const int e = blockIdx.x * 32 + lane;
    if (ok && e < E) logits[e] = acc;
  }
}

cudaError_t launch_router_logits_exact(const void* x, int x_dtype, const void* w, int w_dtype,
                                       float* logits, int T, int H, int E, cudaStream_t st, unsigned* err,
                                       const void* w_slabs) {
  if (T <= 0) return cudaSuccess;
  // one token through a layer (its router in the slab layout, its error flags for the waits)
  const size_t chain_smem = w_dtype == kBF16 ? RcLayout<kBF16>::bytes(H) : RcLayout<kF32>::bytes(H);
  if (T == 1 && w_slabs && err && H % kRcSlabEl == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
      chain_smem <= 227 * 1024) {
    void (*kern)(const void*, const uint8_t*, float*, int, int, unsigned*) =
        x_dtype == kBF16 ? (w_dtype == kBF16 ? router_exact_chain_kernel<kBF16, kBF16> : router_exact_chain_kernel<kBF16, kF32>)
                         : (w_dtype == kBF16 ? router_exact_chain_kernel<kF32, kBF16> : router_exact_chain_kernel<kF32, kF32>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(chain_smem));
    if (e != cudaSuccess) return e;
    kern<<<(E + 31) / 32, kRcThreads, chain_smem, st>>>(x, static_cast<const uint8_t*>(w_slabs), logits, H, E, err);
    return cudaGetLastError();
  }
  const size_t warp_smem = (static_cast<size_t>(H) + 8 * kRwChunk) * 4;
  if (T <= 16 && H % kRwChunk == 0 && warp_smem <= 160 * 1024) {
    void (*kern)(const void*, const void*, float*, int, int, int) =
        x_dtype == kBF16 ? (w_dtype == kBF16 ? router_exact_warp_kernel<kBF16, kBF16> : router_exact_warp_kernel<kBF16, kF32>)
                         : (w_dtype == kBF16 ? router_exact_warp_kernel<kF32, kBF16> : router_exact_warp_kernel<kF32, kF32>);
    if (warp_smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(warp_smem));
      if (e != cudaSuccess) return e;
    }
    kern<<<T * ((E + 7) / 8), 256, warp_smem, st>>>(x, w, logits, T, H, E);
    return cudaGetLastError();
  }
  // 64 x 64 tiles, or one chain per thread when that is faster: a tile block alone on an SM takes
  // ~0.72 ms per 8192 columns (measured: the 512 x 256 GLM router, 32 blocks, 0.54 ms at 6144),
  // a wave of them no longer; the one-chain kernel sustains ~2.5e9 chain steps per ms over the
  // GPU (the same router, 0.32 ms). So the 512 x 256 GLM router takes one chain per thread,
  // while 2048 x 512 (0.99 against 2.4 ms measured) and an expert-parallel rank's 512-1024 x 512
  // keep the tiles.
  const int sms = device_sm_count();
  const long long tiles = static_cast<long long>((E + 63) / 64) * ((T + 63) / 64);
  const double t_tiled = static_cast<double>(H) / 8192.0 * 0.72 * static_cast<double>((tiles + sms - 1) / sms);
  const double t_chain = static_cast<double>(T) * E * H / 2.5e9;
  if (T >= 64 && t_tiled <= t_chain) {
    dim3 grid((E + 63) / 64, (T + 63) / 64);
    router_exact_tiled_kernel<<<grid, 256, 0, st>>>(x, x_dtype, w, w_dtype, logits, T, H, E);
  } else if (T == 1) {
    dim3 grid((E + 31) / 32, 1);
    router_exact_small_kernel<1><<<grid, dim3(32, 1), 0, st>>>(x, x_dtype, w, w_dtype, logits, T, H, E);
  } else {
    dim3 grid((E + 31) / 32, (T + 7) / 8);
    router_exact_small_kernel<8><<<grid, dim3(32, 8), 0, st>>>(x, x_dtype, w, w_dtype, logits, T, H, E);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Top-k selection, one warp per token.
// ---------------------------------------------------------------------------------------

// (value desc, id asc) total order: true when (va, ia) ranks ahead of (vb, ib).
__device__ __forceinline__ bool ranks_ahead(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Warp argmax over per-lane candidates under ranks_ahead; returns the winner to all lanes.
__device__ __forceinline__ void warp_argmax(float& v, int& id) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(kFull, v, o);
    int oid = __shfl_xor_sync(kFull, id, o);
    if (ranks_ahead(ov, oid, v, id)) {
      v = ov;
      id = oid;
    }
  }
}

constexpr int kMaxE = 1024;  // experts per token held in registers: 32 lanes x PL

// qwen38::moe::route (src/qwen38/moe.rs:41-76). Its strict-'>' running insertion keeps the k
// largest logits ordered by (logit desc, id asc) -- a total order, so k rounds of a warp argmax
// pick the same ids in the same rank order. Weights: exp(l - l_max) over the k winners, summed
// left to right from +0.0, each divided by the sum.
template <int PL>
__global__ void topk_softmax_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                    int T, int E, int k, int32_t* __restrict__ ids,
                                    float* __restrict__ wout) {
  const int warps = blockDim.x / 32;
  const int t = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float v[PL];
  const float* row = logits + static_cast<size_t>(t) * E;
#pragma unroll
  for (int q = 0; q < PL; q++) {
    int e = q * 32 + lane;
    float l = -INFINITY;
    if (e < E) {
      l = row[e];
      if (bias) l = __fadd_rn(l, bias[e]);
    }
    v[q] = l;
  }
  unsigned taken = 0;
  float sel_v = 0.0f;  // lane j keeps the j-th winner
  int sel_id = -1;
  const int kk = min(k, E);
  for (int r = 0; r < kk; r++) {
    float bv = -INFINITY;
    int bid = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < PL; q++) {
      int e = q * 32 + lane;
      if (e < E && !((taken >> q) & 1) && ranks_ahead(v[q], e, bv, bid)) {
        bv = v[q];
        bid = e;
      }
    }
    warp_argmax(bv, bid);
    if (lane == r) {
      sel_v = bv;
      sel_id = bid;
    }
    if ((bid & 31) == lane) taken |= 1u << (bid >> 5);
  }
  const float mx = __shfl_sync(kFull, sel_v, 0);
  float ex = (lane < kk) ? exp_f32(__fsub_rn(sel_v, mx)) : 0.0f;
  float sum = 0.0f;
  for (int j = 0; j < kk; j++) sum = __fadd_rn(sum, __shfl_sync(kFull, ex, j));
  if (lane < kk) {
    ids[static_cast<size_t>(t) * k + lane] = sel_id;
    wout[static_cast<size_t>(t) * k + lane] = __fdiv_rn(ex, sum);
  } else if (lane < k) {
    ids[static_cast<size_t>(t) * k + lane] = -1;
    wout[static_cast<size_t>(t) * k + lane] = 0.0f;
  }
}

template <int PL>
static void launch_softmax_pl(const float* logits, const float* bias, int T, int E, int k,
                              int32_t* ids, float* w, cudaStream_t st) {
  const int warps = 8;
  topk_softmax_kernel<PL><<<(T + warps - 1) / warps, warps * 32, 0, st>>>(logits, bias, T, E, k, ids, w);
}

cudaError_t launch_topk_softmax(const float* logits, const float* bias, int T, int E, int k,
                                int32_t* ids, float* w, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (E > kMaxE || k > 32 || k < 1) return cudaErrorInvalidValue;
  if (E <= 32) launch_softmax_pl<1>(logits, bias, T, E, k, ids, w, st);
  else if (E <= 64) launch_softmax_pl<2>(logits, bias, T, E, k, ids, w, st);
  else if (E <= 128) launch_softmax_pl<4>(logits, bias, T, E, k, ids, w, st);
  else if (E <= 256) launch_softmax_pl<8>(logits, bias, T, E, k, ids, w, st);
  else if (E <= 512) launch_softmax_pl<16>(logits, bias, T, E, k, ids, w, st);
  else launch_softmax_pl<32>(logits, bias, T, E, k, ids, w, st);
  return cudaGetLastError();
}

// glm52::moe::route (src/glm52/moe.rs:131-260) for one token per warp:
//   logit_e = sigmoid(l_e) (1/(1+exp(-l)) in f32), choice_e = logit_e + bias_e;
//   group score = top2_sum of choice over each of n_group contiguous groups (:193-205);
//   keep the topk_group best groups, ties to the lower group index (:214-229);
//   k rounds of a strict '>' scan from -1e30 over allowed, untaken experts (ties -> lower id);
//   weight = plain logit; norm_topk: divide by (sum from -0.0) + 1e-20; times routed_scale.
template <int PL>
__global__ void topk_grouped_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                    int T, int E, int k, int n_group, int topk_group,
                                    int norm_topk, float routed_scale, int32_t* __restrict__ ids,
                                    float* __restrict__ wout) {
  extern __shared__ float choice_smem[];  // [warps][E]
  const int warps = blockDim.x / 32;
  const int wi = threadIdx.x / 32;
  const int t = blockIdx.x * warps + wi;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float* cs = choice_smem + static_cast<size_t>(wi) * E;
  float sg[PL], ch[PL];
  const float* row = logits + static_cast<size_t>(t) * E;
#pragma unroll
  for (int q = 0; q < PL; q++) {
    int e = q * 32 + lane;
    float s = 0.0f, c = -INFINITY;
    if (e < E) {
      s = sigmoid_ref(row[e]);
      c = __fadd_rn(s, bias ? bias[e] : 0.0f);
      cs[e] = c;
    }
    sg[q] = s;
    ch[q] = c;
  }
  __syncwarp();
  unsigned allowed_groups = 0xffffffffu;
  const int gsz = n_group > 1 ? E / n_group : E;
  if (n_group > 1) {
    // lane g scans group g in index order exactly as top2_sum does
    float score = -INFINITY;
    if (lane < n_group) {
      float t1 = -INFINITY, t2 = -INFINITY;
      for (int i = 0; i < gsz; i++) {
        float val = cs[lane * gsz + i];
        if (val > t1) {
          t2 = t1;
          t1 = val;
        } else if (val > t2) {
          t2 = val;
        }
      }
      score = isfinite(t2) ? __fadd_rn(t1, t2) : t1;
    }
    allowed_groups = 0;
    for (int r = 0; r < topk_group && r < n_group; r++) {
      bool cand = lane < n_group && !((allowed_groups >> lane) & 1);
      float bv = cand ? score : -INFINITY;
      int bid = cand ? lane : 0x7fffffff;
      warp_argmax(bv, bid);
      if (bid < n_group) allowed_groups |= 1u << bid;
    }
  }
  const int n_allowed = n_group > 1 ? __popc(allowed_groups) * gsz : E;
  const int kk = min(k, n_allowed);
  float sel_w = 0.0f;
  int sel_id = -1;
  unsigned taken = 0;
  for (int r = 0; r < kk; r++) {
    float bv = -1e30f;
    int bid = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < PL; q++) {
      int e = q * 32 + lane;
      if (e >= E || ((taken >> q) & 1)) continue;
      if (n_group > 1 && !((allowed_groups >> (e / gsz)) & 1)) continue;
      if (ch[q] > bv) {  // strict '>' from -1e30, ids ascending within the lane
        bv = ch[q];
        bid = e;
      }
    }
    warp_argmax(bv, bid);
    float wv = 0.0f;
    const bool found = bid != 0x7fffffff;
    if (found && (bid & 31) == lane) {
      taken |= 1u << (bid >> 5);
#pragma unroll
      for (int q = 0; q < PL; q++)
        if (q == (bid >> 5)) wv = sg[q];
    }
    wv = __shfl_sync(kFull, wv, found ? (bid & 31) : 0);
    if (lane == r) {
      sel_id = found ? bid : -1;
      sel_w = found ? wv : 0.0f;
    }
  }
  if (norm_topk) {
    float sum = -0.0f;
    for (int j = 0; j < kk; j++) sum = __fadd_rn(sum, __shfl_sync(kFull, sel_w, j));
    sum = __fadd_rn(sum, 1e-20f);
    sel_w = __fdiv_rn(sel_w, sum);
  }
  sel_w = __fmul_rn(sel_w, routed_scale);
  if (lane < k) {
    ids[static_cast<size_t>(t) * k + lane] = lane < kk ? sel_id : -1;
    wout[static_cast<size_t>(t) * k + lane] = lane < kk ? sel_w : 0.0f;
  }
}

// Ungrouped sigmoid router (n_group <= 1): one 1024-thread block per token, one thread per
// expert, with a certificate. The choice values c = sigmoid(logit) + bias are first bounded from
// the single-precision expf (<= 2 ulp; the bound used is 2^-20 relative, widened outward with
// directed rounding), which decides who can be in the top k at all: every expert whose upper
// bound reaches the k-th largest lower bound. Only those contenders evaluate the reference's
// correctly rounded sigmoid (an f64 exp, slow on this part, here one per contender thread in
// parallel) and are ranked exactly by (c desc, id asc); the weights are those exact sigmoids,
// normalized and scaled as in glm52::moe::route. Both selections are block-wide warp-reduction
// rounds (select.cuh).
__global__ void __launch_bounds__(1024) topk_sigmoid_block_kernel(const float* __restrict__ logits,
                                                                  const float* __restrict__ bias, int T, int E, int k,
                                                                  int norm_topk, float routed_scale,
                                                                  int32_t* __restrict__ ids, float* __restrict__ wout) {
  __shared__ float c1[32 * 32], c2[32 * 32];
  __shared__ int c1i[32 * 32], c2i[32 * 32];
  __shared__ int sel_id[32], lo_id[32];
  __shared__ float sel_v[32], lo_v[32];
  __shared__ float s_sig[1024];
  // (launched as a programmatic dependent of the router logits: wait for them here)
  griddep_wait();
  const int t = blockIdx.x, e = threadIdx.x;
  const bool valid = e < E;
  const int id = valid ? e : 0x40000000 + e;
  const float* row = logits + static_cast<size_t>(t) * E;
  const int kk = min(k, E);
  float x = 0.0f, b = 0.0f, lo = -INFINITY, hi = -INFINITY;
  if (valid) {
    x = row[e];
    b = bias ? bias[e] : 0.0f;
    const float sf = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    // |sf - sigmoid| <= 3 * 2^-23 sf (expf 2 ulp, then two roundings) and the reference's value
    // is within 1.5 * 2^-23 sf of the same sigmoid: 2^-20 sf covers both, with room
    const float d = fmaf(sf, 9.54e-7f, 1e-37f);
    lo = __fadd_rd(__fsub_rd(sf, d), b);
    hi = __fadd_ru(__fadd_ru(sf, d), b);
  }
  // Lk, the kk-th largest lower bound, by a bitwise search over the order-preserving keys (one
  // block count per bit); the contenders are the experts whose upper bound reaches it -- every
  // member of the true top kk is one of them
  const uint32_t klo = valid ? order_key(lo) : 0u;
  uint32_t X = 0;
  for (int bit = 31; bit >= 0; bit--) {
    const uint32_t cand = X | (1u << bit);
    if (__syncthreads_count(klo >= cand) >= kk) X = cand;
  }
  const bool cont = valid && order_key(hi) >= X;
  float sx = 0.0f, cx = -INFINITY;
  if (cont) {
    sx = sigmoid_ref(x);
    cx = __fadd_rn(sx, b);
  }
  s_sig[e] = sx;
  __shared__ int s_n;
  if (threadIdx.x == 0) s_n = 0;
  const int n_cont = __syncthreads_count(cont);
  if (n_cont <= 32) {
    // one warp ranks the contenders by (value desc, id asc): each lane counts those ahead of it
    if (cont) {
      const int slot = atomicAdd(&s_n, 1);
      c1[slot] = cx;
      c1i[slot] = e;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      const bool has = lane < n_cont;
      const float v = has ? c1[lane] : -INFINITY;
      const int vid = has ? c1i[lane] : 0x7fffffff;
      const uint32_t kv = order_key(v);
      int rank = 0;
      for (int j = 0; j < n_cont; j++) {
        const uint32_t kj = __shfl_sync(kFull, kv, j);
        const int ij = __shfl_sync(kFull, vid, j);
        rank += (kj > kv || (kj == kv && ij < vid)) ? 1 : 0;
      }
      if (has && rank < kk) sel_id[rank] = vid;
    }
    __syncthreads();
  } else {
    block_select2(cx, cx, id, kk, c1, c1i, c2, c2i, sel_id, sel_v, lo_id, lo_v);
  }
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float w = lane < kk ? s_sig[sel_id[lane]] : 0.0f;
    if (norm_topk) {
      float sum = -0.0f;
      for (int j = 0; j < kk; j++) sum = __fadd_rn(sum, __shfl_sync(kFull, w, j));
      sum = __fadd_rn(sum, 1e-20f);
      w = __fdiv_rn(w, sum);
    }
    w = __fmul_rn(w, routed_scale);
    if (lane < k) {
      ids[static_cast<size_t>(t) * k + lane] = lane < kk ? sel_id[lane] : -1;
      wout[static_cast<size_t>(t) * k + lane] = lane < kk ? w : 0.0f;
    }
  }
}

template <int PL>
static void launch_grouped_pl(const float* logits, const float* bias, int T, int E, int k,
                              int n_group, int topk_group, int norm_topk, float routed_scale,
                              int32_t* ids, float* w, cudaStream_t st) {
  const int warps = 8;
  size_t smem = static_cast<size_t>(warps) * E * sizeof(float);
  topk_grouped_kernel<PL><<<(T + warps - 1) / warps, warps * 32, smem, st>>>(
      logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w);
}

cudaError_t launch_topk_grouped(const float* logits, const float* bias, int T, int E, int k,
                                int n_group, int topk_group, int norm_topk, float routed_scale,
                                int32_t* ids, float* w, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (E > kMaxE || k > 32 || k < 1 || n_group > 32) return cudaErrorInvalidValue;
  if (n_group > 1 && E % n_group != 0) return cudaErrorInvalidValue;
  if (n_group <= 1) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(T);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, topk_sigmoid_block_kernel, logits, bias, T, E, k, norm_topk, routed_scale, ids, w);
  }
  if (E <= 32) launch_grouped_pl<1>(logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w, st);
  else if (E <= 64) launch_grouped_pl<2>(logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w, st);
  else if (E <= 128) launch_grouped_pl<4>(logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w, st);
  else if (E <= 256) launch_grouped_pl<8>(logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w, st);
  else if (E <= 512) launch_grouped_pl<16>(logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w, st);
  else launch_grouped_pl<32>(logits, bias, T, E, k, n_group, topk_group, norm_topk, routed_scale, ids, w, st);
  return cudaGetLastError();
}

// CACHE_ROUTE (glm52::moe::route_cache_aware + cache_route_select, src/glm52/moe.rs:272-323):
// rank the top m = max(route_m, k) experts by choice = sigmoid(logit) + bias (rank_top,
// :148-166: strict '>' from -1e30, ties to the lower id), keep the top j = min(route_j, k)
// always, fill the remaining slots with the resident experts among ranked[j..] in rank order,
// then with the rest of ranked[j..] in rank order; weights are the plain sigmoids, normalized
// and scaled (normalize_and_scale, :231-241). Like the reference it ranks over every expert (no
// grouping). One warp per token; resident: [E] bytes, nonzero = resident (NULL = all).
template <int PL>
__global__ void topk_cache_route_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int T, int E,
                                        int k, int route_j, int route_m, const uint8_t* __restrict__ resident,
                                        int norm_topk, float routed_scale, int32_t* __restrict__ ids,
                                        float* __restrict__ wout) {
  const int warps = blockDim.x / 32;
  const int t = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= T) return;
  float sg[PL], ch[PL];
  const float* row = logits + static_cast<size_t>(t) * E;
#pragma unroll
  for (int q = 0; q < PL; q++) {
    const int e = q * 32 + lane;
    float sv = 0.0f, c = -INFINITY;
    if (e < E) {
      sv = sigmoid_ref(row[e]);
      c = __fadd_rn(sv, bias ? bias[e] : 0.0f);
    }
    sg[q] = sv;
    ch[q] = c;
  }
  const int m = min(max(route_m, k), E);
  // ranked[r] (r < m) held by lane r: id, sigmoid, resident flag
  int r_id = -1;
  float r_w = 0.0f;
  unsigned taken = 0;
  for (int r = 0; r < m; r++) {
    float bv = -1e30f;
    int bid = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < PL; q++) {
      const int e = q * 32 + lane;
      if (e >= E || ((taken >> q) & 1)) continue;
      if (ch[q] > bv) {
        bv = ch[q];
        bid = e;
      }
    }
    warp_argmax(bv, bid);
    float wv = 0.0f;
    if ((bid & 31) == lane) {
      taken |= 1u << (bid >> 5);
#pragma unroll
      for (int q = 0; q < PL; q++)
        if (q == (bid >> 5)) wv = sg[q];
    }
    wv = __shfl_sync(kFull, wv, bid & 31);
    if (lane == r) {
      r_id = bid;
      r_w = wv;
    }
  }
  const int j = min(min(route_j, k), m);
  const bool res = lane < m && (!resident || resident[r_id] != 0);
  // pass 1: ranked[0..j) always, then resident ranked[j..) in order, up to k slots
  const unsigned res_mask = __ballot_sync(kFull, lane >= j && res);
  const unsigned jmask = j >= 32 ? kFull : ((1u << j) - 1u);
  unsigned pick = jmask;
  int need = k - j;
  unsigned rm = res_mask;
  while (need > 0 && rm) {
    const int b = __ffs(rm) - 1;
    pick |= 1u << b;
    rm &= rm - 1;
    need--;
  }
  // pass 2: the rest of ranked[j..) in order
  const unsigned mmask = m >= 32 ? kFull : ((1u << m) - 1u);
  unsigned rest = mmask & ~pick;
  while (need > 0 && rest) {
    const int b = __ffs(rest) - 1;
    pick |= 1u << b;
    rest &= rest - 1;
    need--;
  }
  // slot order: ranked[0..j), then pass-1 picks in rank order, then pass-2 picks in rank order
  const unsigned p1 = pick & res_mask & ~jmask, p2 = pick & ~res_mask & ~jmask;
  int slot = -1;
  if ((pick >> lane) & 1u) {
    const unsigned below = (1u << lane) - 1u;
    if (lane < j) slot = lane;
    else if ((p1 >> lane) & 1u) slot = j + __popc(p1 & below);
    else slot = j + __popc(p1) + __popc(p2 & below);
  }
  const int kk = __popc(pick);
  // gather per slot: lane s takes the entry whose slot is s
  float w = 0.0f;
  int id = -1;
  for (int src = 0; src < 32; src++) {
    const int sl = __shfl_sync(kFull, slot, src);
    const int sid = __shfl_sync(kFull, r_id, src);
    const float sw = __shfl_sync(kFull, r_w, src);
    if (sl == lane) {
      id = sid;
      w = sw;
    }
  }
  if (norm_topk) {
    float sum = -0.0f;
    for (int q = 0; q < kk; q++) sum = __fadd_rn(sum, __shfl_sync(kFull, w, q));
    sum = __fadd_rn(sum, 1e-20f);
    w = __fdiv_rn(w, sum);
  }
  w = __fmul_rn(w, routed_scale);
  if (lane < k) {
    ids[static_cast<size_t>(t) * k + lane] = lane < kk ? id : -1;
    wout[static_cast<size_t>(t) * k + lane] = lane < kk ? w : 0.0f;
  }
}

template <int PL>
static void launch_cache_route_pl(const float* logits, const float* bias, int T, int E, int k, int route_j,
                                  int route_m, const uint8_t* resident, int norm_topk, float routed_scale,
                                  int32_t* ids, float* w, cudaStream_t st) {
  const int warps = 8;
  topk_cache_route_kernel<PL><<<(T + warps - 1) / warps, warps * 32, 0, st>>>(
      logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w);
}

cudaError_t launch_topk_cache_route(const float* logits, const float* bias, int T, int E, int k, int route_j,
                                    int route_m, const uint8_t* resident, int norm_topk, float routed_scale,
                                    int32_t* ids, float* w, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (E > kMaxE || k > 32 || k < 1 || route_m > 32 || route_j < 0) return cudaErrorInvalidValue;
  if (E <= 32) launch_cache_route_pl<1>(logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w, st);
  else if (E <= 64) launch_cache_route_pl<2>(logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w, st);
  else if (E <= 128) launch_cache_route_pl<4>(logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w, st);
  else if (E <= 256) launch_cache_route_pl<8>(logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w, st);
  else if (E <= 512) launch_cache_route_pl<16>(logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w, st);
  else launch_cache_route_pl<32>(logits, bias, T, E, k, route_j, route_m, resident, norm_topk, routed_scale, ids, w, st);
  return cudaGetLastError();
}

}  // namespace rmoe
