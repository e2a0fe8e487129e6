// kernels.h -- host-side launchers of the routed-MoE kernels (internal to librmoe.so).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rmoe {

// Limit of a persistent kernel's wait on another CTA's counter (grid barriers, h readiness):
// 2 s, after which the kernel records a device error flag and stops (rmoe_layer_set_wait_limit).
constexpr unsigned long long kDefaultSpinNs = 2000000000ull;

// SMs of the current device (grids of the persistent and grid-stride kernels scale with it).
inline int device_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Where one expert's six tensors live on the device. gate/up: [inter, hidden]; down:
// [hidden, inter]. scales are E8M0 bytes (MXFP4) or f32/bf16 per group (int4).
struct ExpertPtrs {
  const uint8_t* gate;
  const uint8_t* up;
  const uint8_t* down;
  const void* gate_scale;
  const void* up_scale;
  const void* down_scale;
};

// Format of every expert of a layer.
// The expert gating activation: kind 0 silu(g) u; kind 1 Kimi K3's SituAndMul,
// beta tanh(g / beta) sigmoid(g) u' with u' = lb tanh(u / lb) when lb = linear_beta > 0.
struct ActParams {
  int kind;
  float beta, linear_beta;
};

struct ExpertFormat {
  int fmt;          // kMxfp4 | kInt4g
  int group_size;   // int4 elements per scale (multiple of 32); 32 for MXFP4
  int scale_dtype;  // int4 scale storage kF32 | kBF16
  ActParams act;    // gating activation of the experts
};

// Device-side expert table: local routed experts are contiguous, `stride` bytes apart, each
// laid out [gate data][up data][down data][gate scales][up scales][down scales]; the shared
// expert (if any) has its own pointers and width.
struct ExpertTable {
  const uint8_t* base;
  size_t stride;
  size_t off_up, off_down, off_gs, off_us, off_ds;  // byte offsets inside one expert
  int n_local;                                      // local routed experts
  int inter;                                        // routed expert width
  ExpertPtrs shared;
  int shared_inter;                                 // 0 = no shared expert
};

// One group of up to MT positions of one expert ("chunk"), the unit the GEMV kernels stream
// an expert's weights for. Built on the device by the dispatch kernel.
struct DispatchBuffers {
  // sizes: E_loc = local routed experts (+1 slot for the shared expert)
  uint32_t* bits;       // [E_loc][words] token bitmap per expert
  int32_t* first_occ;   // [E_loc] first (t*k+j) that picked the expert
  int32_t* wpre;        // [E_loc][words] exclusive popcount prefix per word
  int32_t* counts;      // [E_loc + 1]
  int32_t* offsets;     // [E_loc + 2]
  int32_t* uniq;        // [E_loc]
  int32_t* n_uniq;      // [1]
  int32_t* perm_tok;    // [P] token of each position
  float* perm_w;        // [P] combine weight of each position (routing weight or shared gate)
  int32_t* inv;         // [T][k] position of (t, j); -1 when the slot is not local
  int32_t* ch_expert;   // [max_chunks] local expert index (n_local = the shared expert)
  int32_t* ch_pos;      // [max_chunks] first position
  int32_t* ch_n;        // [max_chunks] positions in the chunk (<= MT)
  int32_t* ch_task_gu;  // [max_chunks + 1] prefix of gate/up warp tasks
  int32_t* ch_task_dn;  // [max_chunks + 1] prefix of down warp tasks
  int32_t* n_chunks;    // [1]
  int words;            // ceil(max_tokens / 32)
  int max_chunks;
};

constexpr int RMOE_MAX_TOPK_DEV = 32;

// Inputs/outputs of the fused small-T front end (route_small.cu).
struct SmallPrologue {
  int T, E, k, H, mt;
  int e_begin, e_end, n_loc, has_shared, fmt;
  int tpc_gu, tpc_gu_shared, tpc_dn;  // warp tasks per chunk (gate/up routed, shared; down)
  const float* mid;                   // [T][E] certified logit values
  const float* err;                   // [T][E] their error bounds
  const float* bias;                  // [E] logit bias or null
  const void* x;
  int x_dtype;
  const void* w;                      // router [E][H] (exact fallback chains)
  int w_dtype;
  const float* gvec;                  // shared-expert gate vector [H] or null
  int32_t* ids;                       // [T][k]
  float* rw;                          // [T][k]
  uint16_t* xq;                       // [T][H] f16
  int32_t* xexp;                      // [T]
  float* gate;                        // [T]
  unsigned* fallback_count;           // tokens whose expert set was uncertain (exact recompute)
  unsigned* order_pending_count;      // tokens whose rank order was resolved off the critical path
  int32_t* pending;                   // [T] 1 = order to be resolved by launch_resolve_order
  unsigned* errflag;                  // bounded-wait failures
};

// One-token front end of a tensor-core layer (route_small.cu): router logits + certificate,
// shared gate, activation terms and dispatch in one launch.
struct DecodeFront {
  const void* x;
  int x_dtype;
  const void* w;                  // router [E][H]
  int w_dtype;
  const float* bias;              // logit bias or null
  const float* gvec;              // shared gate vector or null
  int H, E, k;
  int e_begin, e_end, n_loc, has_shared;
  float* mid;                     // [E]
  float* err;                     // [E]
  float* gate;                    // [1]
  uint8_t* xt;                    // token terms: rows 0..3 of [.][H/2]
  uint8_t* xsf;                   // [.][H/32]
  int32_t* ids;                   // [k]
  float* rw;                      // [k]
  int32_t* pending;               // [1]
  unsigned* fallback_count;
  unsigned* order_pending_count;
  unsigned* counter;              // finished blocks (zero between launches)
  int32_t* zero_buf;              // zeroed by the front end (the expert kernel's counters), or null
  int zero_n;
  DispatchBuffers d;
  unsigned long long* trace;      // optional diagnostics: [0] block 0 start, [1] last router
                                  // block end, [2] last terms block end, [3..6] last block phases
};
cudaError_t launch_decode_front(const DecodeFront& a, cudaStream_t st);

// ---- router (router.cu, route_small.cu) ----
// Certified logits for T <= 32 tokens (H % 256 == 0): value + rigorous error bound.
cudaError_t launch_router_certified(const void* x, int x_dtype, const void* w, int w_dtype,
                                    float* mid, float* err, int T, int H, int E, cudaStream_t st);
// Top-k + certificate (+ exact fallback), dispatch, activation prep in one block.
cudaError_t launch_prologue_small(const SmallPrologue& a, const DispatchBuffers& d,
                                  cudaStream_t st);
// Final reference-order routing (exact chains for order-pending tokens); one block per
// (token, winner). exact_v: [T][k] scratch; done_cnt: [T] zeroed counters (left zeroed).
cudaError_t launch_resolve_order(const SmallPrologue& a, int32_t* ids_final, float* w_final, float* exact_v,
                                 int32_t* done_cnt, cudaStream_t st);
// logits[T][E] = exact reference chain of x[t] . w[e] (fmul then fadd per element, from -0.0)
// err: the layer's device error flags (a bounded copy wait that runs out sets a bit). w_slabs: the
// router in the slab layout (launch_router_slabs); with err, one token uses the slab kernel.
cudaError_t launch_router_logits_exact(const void* x, int x_dtype, const void* w, int w_dtype,
                                       float* logits, int T, int H, int E, cudaStream_t st,
                                       unsigned* err = nullptr, const void* w_slabs = nullptr);
// The router rows re-laid out for the one-token exact kernel (0 bytes when H % 256 != 0).
size_t router_slab_bytes(int E, int H, int w_dtype);
cudaError_t launch_router_slabs(const void* w, int w_dtype, int E, int H, uint8_t* dst, cudaStream_t st);
// Qwen: top-k by (logit+bias desc, id asc), softmax over the winners.
cudaError_t launch_topk_softmax(const float* logits, const float* bias, int T, int E, int k,
                                int32_t* ids, float* w, cudaStream_t st);
// GLM noaux_tc: sigmoid, +bias for selection, group top-2 sums, grouped top-k, normalize.
// ---- grouped-int4 experts on the tensor cores (i4_tc.cu) ----
constexpr int kI4MinTokens = 8;   // batches above this take the tensor-core path
constexpr int kI4Chunk = 32;      // positions per chunk (the MMA's N)
bool i4_tc_supported(int H, int I, int Is, int gs);
size_t i4_tc_region_bytes(int H, int I, int down);
cudaError_t launch_i4_relayout(int down, const uint8_t* m0, const uint8_t* m1, const void* s0, const void* s1,
                               int scale_bf16, int H, int I, int gs, uint8_t* dst, cudaStream_t st);
cudaError_t launch_i4_gather_x(const void* x, int x_dtype, int H, const int32_t* perm_tok, const int32_t* total,
                               int P_max, __half* xh, cudaStream_t st);
bool i4_make_act_map(void* map, const void* base, int K, int rows);
size_t i4_act_map_bytes();
cudaError_t launch_i4_moe(int mode, const void* act_map, const DispatchBuffers& d, const int32_t* slot_offsets,
                          int H, int I, const uint8_t* tiles, size_t stride, __half* h, float* y, ActParams act,
                          unsigned* err, unsigned long long spin_ns, cudaStream_t st,
                          unsigned long long* trace = nullptr);

// matmul_qt's per-row quantized kinds (qt.cu): the integer-dot path (int8 or int4 weights, int8
// activations quantized per row into `workspace` of matmul_idot_workspace_bytes) and the
// float-weight int4 / int2 paths.
size_t matmul_idot_workspace_bytes(int s, int i);
cudaError_t launch_matmul_idot(float* y, const void* x, int x_dtype, const void* w, bool w4, const float* scale, int s,
                               int i, int o, void* workspace, cudaStream_t st);
cudaError_t launch_matmul_qt_float(float* y, const void* x, int x_dtype, const uint8_t* w, int bits, const float* scale,
                                   int s, int i, int o, cudaStream_t st);
// CACHE_ROUTE selection for the sigmoid router (glm52::moe::route_cache_aware); resident: [E]
// bytes (nonzero = resident) or NULL (every expert resident).
cudaError_t launch_topk_cache_route(const float* logits, const float* bias, int T, int E, int k, int route_j,
                                    int route_m, const uint8_t* resident, int norm_topk, float routed_scale,
                                    int32_t* ids, float* w, cudaStream_t st);
cudaError_t launch_topk_grouped(const float* logits, const float* bias, int T, int E, int k,
                                int n_group, int topk_group, int norm_topk, float routed_scale,
                                int32_t* ids, float* w, cudaStream_t st);

// ---- dispatch (dispatch.cu) ----
// e_begin/e_end: the local routed expert range. mt: positions per chunk. has_shared: append
// the shared expert's T positions (weights from shared_gate[t], or 1).
cudaError_t launch_dispatch(const int32_t* ids, const float* w, int T, int k, int e_begin,
                            int e_end, int mt, int has_shared, const float* shared_gate_w,
                            int inter, int shared_inter, int hidden, int rows_per_task_gu,
                            int rows_per_task_dn, const DispatchBuffers& d, cudaStream_t st);
// One token (k <= 32) for the one-token expert kernel: inv, chunk table, perm, n_chunks only.
cudaError_t launch_dispatch_one_token(const int32_t* ids, const float* w, int k, int e_begin, int e_end, int n_loc,
                                      int has_shared, const float* shared_gate_w, const DispatchBuffers& d,
                                      cudaStream_t st);

// ---- expert compute (experts.cu) ----
// x[T][H] -> xq[T][H] f16 (power-of-two scaled, format pairing), xexp[T] (the exponent), and
// the Qwen shared gate sigmoid(x . g) (g may be null -> 1).
cudaError_t launch_prep_tokens(const void* x, int x_dtype, int T, int H, int fmt,
                               const float* shared_gate_vec, uint16_t* xq, int32_t* xexp,
                               float* gate_out, cudaStream_t st);
cudaError_t launch_gemv_gate_up(const ExpertTable& tab, const ExpertFormat& f,
                                const DispatchBuffers& d, const uint16_t* xq,
                                const int32_t* xexp, int H, int mt, int max_tasks, float* h,
                                uint32_t* hmax, int h_ld, cudaStream_t st);
// total_pos: device int holding the number of positions (offsets[n_slots]).
cudaError_t launch_quant_h(const float* h, const uint32_t* hmax, const int32_t* total_pos,
                           int P_max, int inter_ld, int fmt, uint16_t* hq, int32_t* hexp,
                           cudaStream_t st);
cudaError_t launch_gemv_down(const ExpertTable& tab, const ExpertFormat& f,
                             const DispatchBuffers& d, const uint16_t* hq, const int32_t* hexp,
                             int H, int mt, int max_tasks, int h_ld, float* y, cudaStream_t st);
// shared_slot: index of the shared expert in d.offsets (= local routed experts).
cudaError_t launch_combine(const float* y, const DispatchBuffers& d, const float* rw, int T,
                           int k, int H, int shared_slot, int has_shared, float* out,
                           cudaStream_t st);

// ---- TMA-staged expert GEMVs (gemv_pipe.cu): one task = one gate/up row index, or 8 down
//      rows; tasks per chunk are therefore inter (gate/up) and hidden / 8 (down) ----
bool pipe_supported(const ExpertFormat& f, int H, int inter, int shared_inter);
cudaError_t launch_pipe_gate_up(const ExpertTable& tab, const ExpertFormat& f,
                                const DispatchBuffers& d, const uint16_t* xq,
                                const int32_t* xexp, int H, int mt, float* h, uint32_t* hmax,
                                int h_ld, unsigned* err_flag, cudaStream_t st);
// h enters as f32 [P][h_ld] with its per-position |h| max; scaled to f16 inside the kernel.
cudaError_t launch_pipe_down(const ExpertTable& tab, const ExpertFormat& f,
                             const DispatchBuffers& d, const float* h, const uint32_t* hmax,
                             int H, int mt, int h_ld, float* y, unsigned* err_flag,
                             cudaStream_t st);
// out = parts[0] + ... + parts[n-1] (+ last), in that order; count floats per part (multiple of 4,
// 16-byte aligned pointers).
cudaError_t launch_sum_rank_parts(const float* parts, int n, size_t count, const float* last, float* out,
                                  cudaStream_t st);
// Down projection fused with the weighted combine and the gated shared expert (small T).
cudaError_t launch_pipe_down_combine(const ExpertTable& tab, const ExpertFormat& f,
                                     const DispatchBuffers& d, const float* h,
                                     const uint32_t* hmax, const int32_t* ids, int T, int k,
                                     int e_begin, int H, int h_ld, float* out, unsigned* err_flag,
                                     cudaStream_t st);

// ---- generic GEMM entry points (experts.cu) ----
cudaError_t launch_matmul_q(float* y, const void* x, int x_dtype, const uint8_t* data,
                            const void* scale, const ExpertFormat& f, int s, int i, int o,
                            void* workspace, size_t ws_bytes, cudaStream_t st);
size_t matmul_q_workspace_bytes(int s, int i);

// ---- tensor-core MXFP4 GEMM (mxf4_tc.cu) ----
bool mxf4_tc_supported(int S, int I, int O);
size_t mxf4_tc_workspace_bytes(int S, int I);
cudaError_t launch_mxf4_tc_matmul(float* y, const void* x, int x_dtype, const uint8_t* w,
                                  const uint8_t* w_sf, int S, int I, int O, void* ws, size_t ws_bytes,
                                  unsigned* err, cudaStream_t st);

// ---- tensor-core expert GEMMs of an MXFP4 layer (moe_tc.cu) ----
bool moe_tc_supported(int H, int I, int Is, int fmt);
size_t moe_tc_plan_bytes();
bool moe_tc_plan(void* plan, int H, int I, const uint8_t* xt, const uint8_t* xsf, const uint8_t* ht,
                 const uint8_t* hsf, int term_rows);
size_t moe_tc_region_bytes(int H, int I, int down);
cudaError_t launch_tc_relayout(int down, const uint8_t* m0, const uint8_t* m1, const uint8_t* s0,
                               const uint8_t* s1, int H, int I, uint8_t* dst, cudaStream_t st);
// One token on given routing (one launch): the one-token dispatch, the one-token expert kernel's
// counters zeroed (zero_n ints), and x's four term rows (rows 0..3 of xt / xsf).
cudaError_t launch_one_token_prep(const void* x, int x_dtype, int H, const int32_t* ids, const float* w, int k,
                                  int e_begin, int e_end, int n_loc, int has_shared, const float* shared_gate_w,
                                  const DispatchBuffers& d, int* zero_buf, int zero_n, uint8_t* xt, uint8_t* xsf,
                                  cudaStream_t st);
// Token-major activation terms: rows 4t..4t+3 of xt ([4T][H/2]) / xsf ([4T][H/32]) are token t's.
cudaError_t launch_terms_rows(const void* x, int x_dtype, int H, int T, uint8_t* xt, uint8_t* xsf, cudaStream_t st);
// Position rows from token-major terms (inv [T][k]: each slot's position or -1).
cudaError_t launch_terms_gather(const uint8_t* tt, const uint8_t* tsf, int H, int T, int k, const int32_t* inv,
                                uint8_t* xt, uint8_t* xsf, cudaStream_t st);
cudaError_t launch_terms_by_position(const void* x, int x_dtype, int H, int T, int k, const int32_t* inv,
                                     const int32_t* shared_pos0, uint8_t* xt, uint8_t* xsf, cudaStream_t st);
// mode 0: gate/up (-> h terms), 1: down (-> y per position), 2: down of one token (-> out row)
cudaError_t launch_moe_tc(int mode, const void* plan, const DispatchBuffers& d, int mt, int H, int I,
                          const uint8_t* arena, size_t stride, size_t off_down, uint8_t* ht, uint8_t* hsf, float* y, float* partial,
                          int32_t* tile_cnt, int* work, unsigned* err, cudaStream_t st,
                          const int32_t* b_token_rows = nullptr, unsigned long long* trace = nullptr,
                          ActParams act = ActParams{0, 0.0f, 0.0f}, int32_t* gu_tile_cnt = nullptr,
                          int* h_done = nullptr, bool weights_once = false,
                          unsigned long long spin_ns = kDefaultSpinNs);
// Unit parts of split tiles (floats) a layer must provide for batches of up to 8 tokens.
size_t moe_tc_partial_floats(int H, int I, int k, int n_slots);

// ---- synthetic bytes (synth.cu) ----
cudaError_t launch_synth_bytes(void* dst, size_t n, uint64_t key, int mode, int lo, int hi,
                               cudaStream_t st);

// One token after the fused front end: gate/up and down of all its experts in one launch.
cudaError_t launch_moe_decode_fused(const void* plan, const DispatchBuffers& d, int H, int I, const uint8_t* arena,
                                    size_t stride, size_t off_down, uint8_t* ht, uint8_t* hsf, float* part_gu,
                                    float* part_dn, int32_t* tile_cnt, int32_t* h_ready, int* work, unsigned* err,
                                    float* out, ActParams act, int sh_slot, cudaStream_t st,
                                    unsigned long long* trace = nullptr,
                                    unsigned long long spin_ns = kDefaultSpinNs);

// ---- latent MoE wrapper (latent.cu) ----
// y[T][N] = x[T][K] . w[N][K]^T (w bf16 or f32, x bf16 or f32; K % 8 == 0)
// True when T rows of K fit the projection's one staging group (the norm can be folded in).
bool latent_proj_one_group(int T, int K);
// norm_w: RMSNorm each row of x first (weights [K], eps; the rows must fit in one staging group).
cudaError_t launch_latent_proj(const void* w, int w_dtype, const void* x, int x_dtype, int T, int K, int N, float* y,
                               cudaStream_t st, const float* norm_w = nullptr, float eps = 0.0f);
// v[r] *= w / sqrt(mean(v[r]^2) + eps) for each of `rows` rows of n
cudaError_t launch_rmsnorm_rows(float* v, int rows, int n, const float* w, float eps, cudaStream_t st);

}  // namespace rmoe
