// api.cu -- the C ABI (include/rmoe.h): contexts, layers with HBM-resident experts, uploads
// in the reference byte layout, and the stream-ordered forward pipeline.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "rmoe.h"

using namespace rmoe;

namespace {

thread_local std::string g_last_error;

rmoe_status fail(rmoe_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

rmoe_status cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // a handled (non-sticky) error must not resurface in a later check
  return fail(e == cudaErrorMemoryAllocation ? RMOE_OUT_OF_MEMORY : RMOE_CUDA_ERROR, "%s: %s",
              what, cudaGetErrorString(e));
}

#define RMOE_CUDA(call, what)                         \
  do {                                                \
    cudaError_t _e = (call);                          \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device allocations of one layer, freed together.
struct DevArena {
  std::vector<void*> ptrs;
  ~DevArena() {
    for (void* p : ptrs) cudaFree(p);
  }
  template <typename T>
  cudaError_t alloc(T** out, size_t count) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 16));
    if (e != cudaSuccess) return e;
    ptrs.push_back(p);
    *out = static_cast<T*>(p);
    return cudaSuccess;
  }
};

}  // namespace

// The thread's error text, for the other translation units of the library (the checkpoint loader).
void rmoe_set_error(const char* msg) { g_last_error = msg; }

struct rmoe_ctx {
  int device;
};

// One captured forward (CUDA graph) for a (T, dtype, routing-out, profiling) combination. The
// caller's buffers are reached through memcpy nodes whose pointers are set per launch.
// A kernel node of a captured forward whose arguments hold the staging input or output pointer:
// the caller's x / out are written into a copy of its argument bytes at each launch.
struct NodePatch {
  cudaGraphNode_t node = nullptr;
  cudaKernelNodeParams params{};
  std::vector<std::vector<uint8_t>> args;  // argument bytes
  std::vector<void*> arg_ptrs;             // -> args[i].data()
  struct Site {
    size_t arg, off;
    bool out;
  };
  std::vector<Site> sites;
};

struct GraphEntry {
  cudaGraph_t graph = nullptr;  // kept alive: its node handles address the exec's nodes
  cudaGraphExec_t exec = nullptr;
  // direct_io: the kernels read x / write out through patched arguments (no copy nodes)
  bool direct_io = false;
  std::vector<NodePatch> patches;
  cudaGraphNode_t in_node = nullptr, out_node = nullptr, ids_node = nullptr, w_node = nullptr;
  size_t x_bytes = 0, out_bytes = 0, rt_bytes = 0;
  const void* ids_src = nullptr;
  const void* w_src = nullptr;
  bool profiled = false, pending = false;
  cudaEvent_t ev[RMOE_NUM_STAGES + 1] = {};
  int launches = 0;
};

struct rmoe_layer {
  rmoe_ctx* ctx = nullptr;
  rmoe_layer_desc desc{};
  int e_begin = 0, e_end = 0, n_loc = 0;
  bool has_shared = false;
  ExpertFormat fmt{};
  DevArena arena;
  // weights
  void* router = nullptr;
  int router_dtype = kF32;
  uint8_t* router_slabs = nullptr;  // the router in the one-token exact kernel's slab layout
  int hr = 0;  // router width = width of the caller's x (the latent layers' full hidden size)
  // latent wrapper (router_hidden != hidden): projections, norm, activations between them
  void* lat_down = nullptr;   // [hidden][hr]
  void* lat_up = nullptr;     // [hr][hidden]
  int lat_dtype = kF32;
  float* lat_norm = nullptr;  // [hidden]
  float lat_eps = 0.0f;
  bool has_latent = false, lat_has_norm = false;
  float* lat_x = nullptr;     // [max_tokens][hidden]
  float* lat_y = nullptr;     // [max_tokens][hidden]
  float* router_bias = nullptr;
  bool has_router = false, has_bias = false, has_shared_w = false;
  uint8_t* experts = nullptr;
  ExpertTable tab{};
  uint8_t* shared = nullptr;
  float* shared_gate_vec = nullptr;
  std::vector<uint8_t> uploaded;
  // workspace
  int max_tokens = 0, P_max = 0, h_ld = 0;
  float* logits = nullptr;
  float* logit_err = nullptr;
  unsigned* fallbacks = nullptr;
  unsigned* dev_err = nullptr;   // bounded-wait failures of the pipelined kernels
  unsigned* order_pending = nullptr;  // tokens whose rank order was resolved beside the GEMVs
  int32_t* pending = nullptr;    // [min(T, 32)] per-token order-pending flags
  int32_t* ids_final = nullptr;  // [T][k] routing in the reference's rank order
  float* w_final = nullptr;
  float* exact_v = nullptr;      // [min(T, 32)][k] exact router values of order-pending tokens
  int32_t* resolve_cnt = nullptr;  // [min(T, 32)] chains finished per token (zero between calls)
  cudaStream_t side = nullptr;   // resolves rank order concurrently with the expert GEMVs
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  bool use_pipe = false;         // TMA-staged GEMVs (shape permitting)
  int rpt_gu = 2, rpt_dn = 4;    // rows per warp task of the gate/up and down GEMVs
  int32_t* ids = nullptr;
  float* rw = nullptr;
  DispatchBuffers d{};
  uint16_t* xq = nullptr;
  int32_t* xexp = nullptr;
  float* gate = nullptr;
  float* h = nullptr;
  uint32_t* hmax = nullptr;
  uint16_t* hq = nullptr;
  int32_t* hexp = nullptr;
  float* y = nullptr;
  // host-buffer entry point
  cudaStream_t stream = nullptr;
  void* x_dev = nullptr;
  float* out_dev = nullptr;
  rmoe_layer_stats stats{};
  // profiling: one event per stage boundary per profiled call
  bool profiling = false;
  std::vector<cudaEvent_t> ev_free, ev_pending;  // pending: groups of RMOE_NUM_STAGES + 1
  uint64_t prof_calls = 0;
  double prof_ms[RMOE_NUM_STAGES] = {};
  // CUDA graphs of the small-T forward
  bool use_graphs = true;
  std::map<uint64_t, GraphEntry> graphs;
  cudaStream_t cap = nullptr;    // capture stream
  void* x_stage = nullptr;       // host entry point: H2D target, copied into x_dev by the graph
  float* out_stage = nullptr;    // host entry point: graph output, copied to the host
  int32_t* ids_host_stage = nullptr;
  float* w_host_stage = nullptr;
  int last_launches = 0;         // kernels launched by the last forward_into
  // tensor-core expert path (MXFP4)
  bool use_tc = false;
  void* tc_plan = nullptr;       // tensor maps (64-byte aligned host copy, passed by value)
  uint8_t* xt = nullptr;         // [4 P_max + 16][H/2] activation terms per position
  uint8_t* xsf = nullptr;        // [4 P_max + 16][H/32]
  uint8_t* ht = nullptr;         // [4 P_max + 16][inter/2] h terms per position
  uint8_t* hsf = nullptr;        // [4 P_max + 16][inter/32]
  float* partial = nullptr;      // gate/up unit parts of split tiles
  float* partial2 = nullptr;     // down unit parts of split tiles
  int32_t* tile_cnt = nullptr;   // [max tiles]
  unsigned* front_counter = nullptr;  // one-token front end: finished blocks
  size_t tile_cnt_half = 0;      // tile_cnt: [0, half) gate/up tiles, [half, 2 half) down tiles
  int32_t* fused_cnt = nullptr;  // one-token fused kernel: [8] work, [fused_tiles] tiles, [33] h ready
  int fused_tiles = 0;           // (zeroed by the one-token front end before each launch)
  int* tc_work = nullptr;        // [8] work counters: [0..3] gate/up, [4..7] down (they may overlap)
  size_t tc_off_down = 0;        // tile-major down region inside an expert slot
  uint8_t* tc_stage = nullptr;   // one expert in the reference layout, before retiling
  unsigned long long* tc_trace = nullptr;  // RMOE_TC_TRACE=1: gate/up stage timestamps of CTA 0
  bool tc_trace_print = true;              // RMOE_TC_TRACE=2: record only (summary on get_stats)
  bool use_fused = true;                   // one token: the fused gate/up + down kernel (RMOE_DISABLE_FUSED=1: two kernels)
  unsigned long long spin_ns = kDefaultSpinNs;  // limit of the kernels' waits on other CTAs
  // grouped-int4 layers on the tensor cores (i4_tc.cu), for batches of more than kI4MinTokens
  bool use_i4tc = false;
  uint8_t* i4_tiles = nullptr;   // tile-major copy of every slot's weights
  size_t i4_stride = 0, i4_off_down = 0;
  __half* i4_xh = nullptr;       // [P_max + 32][hidden] f16 activations per position
  __half* i4_hh = nullptr;       // [P_max + 32][inter] f16 h per position
  void* i4_map_x = nullptr;      // tensor maps of the two (host copies, 64-byte aligned)
  void* i4_map_h = nullptr;
  unsigned err_seen = 0;                   // device error flags already reported (and cleared)
  // CACHE_ROUTE (sigmoid routers): keep the top route_j, prefer resident experts among the next
  // ranked up to route_m (src/glm52/moe.rs:99-127)
  bool cache_route = false;
  int route_j = 2, route_m = 12;
  uint8_t* resident = nullptr;   // [E] residency mask (device)
  bool resident_all = true;      // no mask given: every expert resident
  bool diag_host = false;                  // RMOE_DIAG_HOST=1: kernel trace in mapped host memory
  unsigned* err_host = nullptr;            // pinned: the error flags, copied behind a host forward's outputs
  void* diag_buf = nullptr;
  ~rmoe_layer() {
    for (cudaEvent_t e : ev_free) cudaEventDestroy(e);
    for (cudaEvent_t e : ev_pending) cudaEventDestroy(e);
    for (auto& kv : graphs) {
      if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
      if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
      for (cudaEvent_t e : kv.second.ev)
        if (e) cudaEventDestroy(e);
    }
    if (cap) cudaStreamDestroy(cap);
    if (diag_buf) cudaFreeHost(diag_buf);
    if (err_host) cudaFreeHost(err_host);
    free(tc_plan);
    free(i4_map_x);
    free(i4_map_h);
  }
};

namespace {
// Records a stage boundary when profiling is on.
struct StageMarks {
  rmoe_layer* L;
  cudaStream_t st;
  std::vector<cudaEvent_t> evs;
  const cudaEvent_t* fixed = nullptr;  // graph capture: the entry's own events
  int n_fixed = 0;
  StageMarks(rmoe_layer* l, cudaStream_t s) : L(l), st(s) {}
  void mark() {
    if (!L->profiling) return;
    if (fixed) {
      // inside stream capture only an "external" record becomes an event node of the graph
      if (n_fixed < RMOE_NUM_STAGES + 1) cudaEventRecordWithFlags(fixed[n_fixed++], st, cudaEventRecordExternal);
      return;
    }
    cudaEvent_t e;
    if (!L->ev_free.empty()) {
      e = L->ev_free.back();
      L->ev_free.pop_back();
    } else if (cudaEventCreate(&e) != cudaSuccess) {
      return;
    }
    cudaEventRecord(e, st);
    evs.push_back(e);
  }
  void commit() {
    if (!L->profiling || fixed) return;
    if (evs.size() == RMOE_NUM_STAGES + 1) {
      L->ev_pending.insert(L->ev_pending.end(), evs.begin(), evs.end());
    } else {
      L->ev_free.insert(L->ev_free.end(), evs.begin(), evs.end());
    }
    evs.clear();
  }
};
}  // namespace

// ------------------------------------------------------------------------------ misc
extern "C" const char* rmoe_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* rmoe_status_string(rmoe_status s) {
  switch (s) {
    case RMOE_OK: return "ok";
    case RMOE_INVALID_ARG: return "invalid argument";
    case RMOE_SHAPE_MISMATCH: return "shape mismatch";
    case RMOE_CUDA_ERROR: return "cuda error";
    case RMOE_NCCL_ERROR: return "nccl error";
    case RMOE_TIMEOUT: return "timeout";
    case RMOE_IO_ERROR: return "i/o error";
    case RMOE_MISSING_TENSOR: return "missing tensor";
    case RMOE_NOT_SUPPORTED: return "not supported";
    case RMOE_OUT_OF_MEMORY: return "out of memory";
  }
  return "unknown status";
}

extern "C" int rmoe_abi_version(void) { return RMOE_ABI_VERSION; }

extern "C" rmoe_status rmoe_init(int device, rmoe_ctx** out) {
  if (!out) return fail(RMOE_INVALID_ARG, "rmoe_init: out is null");
  int n = 0;
  RMOE_CUDA(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(RMOE_INVALID_ARG, "rmoe_init: device %d of %d", device, n);
  RMOE_CUDA(cudaSetDevice(device), "cudaSetDevice");
  rmoe_ctx* c = new (std::nothrow) rmoe_ctx{device};
  if (!c) return fail(RMOE_OUT_OF_MEMORY, "rmoe_init: host allocation");
  *out = c;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_shutdown(rmoe_ctx* ctx) {
  delete ctx;
  return RMOE_OK;
}

// ------------------------------------------------------------------------------ layer
static size_t scale_bytes_for(const ExpertFormat& f, size_t rows, size_t cols) {
  if (f.fmt == kMxfp4) return rows * ((cols + 31) / 32);
  return rows * ((cols + f.group_size - 1) / f.group_size) * (f.scale_dtype == kBF16 ? 2 : 4);
}

extern "C" rmoe_status rmoe_layer_create(rmoe_ctx* ctx, const rmoe_layer_desc* desc,
                                         rmoe_layer** out) {
  if (!ctx || !desc || !out) return fail(RMOE_INVALID_ARG, "rmoe_layer_create: null argument");
  const rmoe_layer_desc& D = *desc;
  if (D.hidden <= 0 || D.moe_inter <= 0 || D.n_experts <= 0 || D.topk <= 0 || D.max_tokens <= 0)
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: hidden, moe_inter, n_experts, topk, max_tokens must be > 0");
  if (D.topk > RMOE_MAX_TOPK || D.topk > D.n_experts)
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: topk %d (max %d, n_experts %d)", D.topk, RMOE_MAX_TOPK, D.n_experts);
  if (D.n_experts > 1024) return fail(RMOE_NOT_SUPPORTED, "rmoe_layer_create: n_experts %d > 1024", D.n_experts);
  if (D.hidden % 32 || D.moe_inter % 32 || D.shared_inter % 32 || D.shared_inter < 0)
    return fail(RMOE_NOT_SUPPORTED, "rmoe_layer_create: hidden/moe_inter/shared_inter must be multiples of 32");
  if (D.router_kind != RMOE_ROUTER_SOFTMAX_TOPK && D.router_kind != RMOE_ROUTER_SIGMOID_GROUPED)
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: router_kind %d", D.router_kind);
  if (D.router_kind == RMOE_ROUTER_SIGMOID_GROUPED && D.n_group > 1) {
    if (D.n_group > 32 || D.n_experts % D.n_group)
      return fail(RMOE_INVALID_ARG, "rmoe_layer_create: n_group %d must divide n_experts and be <= 32", D.n_group);
    if (D.topk_group < 1 || D.topk_group > D.n_group)
      return fail(RMOE_INVALID_ARG, "rmoe_layer_create: topk_group %d", D.topk_group);
  }
  ExpertFormat f{};
  if (D.weight_format == RMOE_FMT_MXFP4) {
    f = ExpertFormat{kMxfp4, 32, kF32};
  } else if (D.weight_format == RMOE_FMT_I4_GROUPED) {
    if (D.group_size <= 0 || D.group_size % 32)
      return fail(RMOE_NOT_SUPPORTED, "rmoe_layer_create: int4 group_size %d must be a multiple of 32", D.group_size);
    if (D.hidden % D.group_size || D.moe_inter % D.group_size || (D.shared_inter && D.shared_inter % D.group_size))
      return fail(RMOE_NOT_SUPPORTED, "rmoe_layer_create: group_size must divide hidden and inter");
    if (D.scale_dtype != RMOE_F32 && D.scale_dtype != RMOE_BF16)
      return fail(RMOE_INVALID_ARG, "rmoe_layer_create: scale_dtype %d", D.scale_dtype);
    f = ExpertFormat{kInt4g, D.group_size, D.scale_dtype == RMOE_BF16 ? kBF16 : kF32};
  } else {
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: weight_format %d", D.weight_format);
  }
  if (D.activation != RMOE_ACT_SILU && D.activation != RMOE_ACT_SITU)
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: activation %d", D.activation);
  if (D.activation == RMOE_ACT_SITU && !(D.situ_beta > 0.0f))
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: Situ needs situ_beta > 0");
  f.act = ActParams{D.activation, D.situ_beta, D.situ_linear_beta > 0.0f ? D.situ_linear_beta : 0.0f};
  if (D.router_hidden < 0 || (D.router_hidden && D.router_hidden % 32))
    return fail(RMOE_NOT_SUPPORTED, "rmoe_layer_create: router_hidden %d (a multiple of 32)", D.router_hidden);
  if (D.router_hidden && D.router_hidden != D.hidden && D.hidden > 8192)
    return fail(RMOE_NOT_SUPPORTED, "rmoe_layer_create: a latent layer's expert width %d exceeds 8192", D.hidden);
  const int ep_size = D.ep_size <= 0 ? 1 : D.ep_size;
  if (D.n_experts % ep_size || D.ep_rank < 0 || D.ep_rank >= ep_size)
    return fail(RMOE_INVALID_ARG, "rmoe_layer_create: ep_rank %d / ep_size %d / n_experts %d", D.ep_rank, ep_size, D.n_experts);

  RMOE_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
  rmoe_layer* L = new (std::nothrow) rmoe_layer();
  if (!L) return fail(RMOE_OUT_OF_MEMORY, "rmoe_layer_create: host allocation");
  L->ctx = ctx;
  L->desc = D;
  L->desc.ep_size = ep_size;
  L->fmt = f;
  L->n_loc = D.n_experts / ep_size;
  L->e_begin = D.ep_rank * L->n_loc;
  L->e_end = L->e_begin + L->n_loc;
  L->has_shared = D.shared_inter > 0;
  L->uploaded.assign(L->n_loc, 0);
  auto cleanup = [&](rmoe_status s) {
    if (L->stream) cudaStreamDestroy(L->stream);
    if (L->side) cudaStreamDestroy(L->side);
    if (L->ev_fork) cudaEventDestroy(L->ev_fork);
    if (L->ev_join) cudaEventDestroy(L->ev_join);
    delete L;
    return s;
  };
#define ALLOC(ptr, n)                                                          \
  do {                                                                         \
    cudaError_t _e = L->arena.alloc(&(ptr), (n));                              \
    if (_e != cudaSuccess) return cleanup(cuda_fail(_e, "cudaMalloc " #ptr)); \
  } while (0)

  const size_t H = D.hidden, I = D.moe_inter, Is = D.shared_inter, E = D.n_experts;
  // expert table: [gate][up][down][gate sc][up sc][down sc], each region 4096-byte aligned so
  // that every matrix of every expert is one 2-D tensor view of the whole table (row pitch =
  // row bytes). A shared expert of the routed width takes the slot after the routed ones.
  const size_t gd = I * (H / 2), dd = H * (I / 2);
  size_t off = 0;
  const size_t o_gate = off; off = align_up(off + gd, 4096);
  const size_t o_up = off; off = align_up(off + gd, 4096);
  const size_t o_down = off; off = align_up(off + dd, 4096);
  const size_t o_gs = off; off = align_up(off + scale_bytes_for(f, I, H), 4096);
  const size_t o_us = off; off = align_up(off + scale_bytes_for(f, I, H), 4096);
  const size_t o_ds = off; off = align_up(off + scale_bytes_for(f, H, I), 4096);
  const bool shared_in_table = L->has_shared && Is == I;
  {
    const char* notc = getenv("RMOE_DISABLE_TC");
    L->use_tc = moe_tc_supported(static_cast<int>(H), static_cast<int>(I), static_cast<int>(Is), f.fmt) &&
                !(notc && notc[0] == '1') && (!L->has_shared || shared_in_table);
  }
  if (L->use_tc) {
    // tensor-core layers keep their weights tile-major (moe_tc.cu): [gate/up tiles][down tiles]
    L->tc_off_down = align_up(moe_tc_region_bytes(static_cast<int>(H), static_cast<int>(I), 0), 4096);
    off = align_up(L->tc_off_down + moe_tc_region_bytes(static_cast<int>(H), static_cast<int>(I), 1), 4096);
  }
  const size_t stride = off;
  const int table_slots = L->n_loc + (shared_in_table ? 1 : 0);
  ALLOC(L->experts, stride * table_slots);
  L->tab.base = L->experts;
  L->tab.stride = stride;
  L->tab.off_up = o_up - o_gate;
  L->tab.off_down = o_down;
  L->tab.off_gs = o_gs;
  L->tab.off_us = o_us;
  L->tab.off_ds = o_ds;
  L->tab.n_local = L->n_loc;
  L->tab.inter = static_cast<int>(I);
  L->tab.shared_inter = static_cast<int>(Is);
  if (shared_in_table) {
    uint8_t* b = L->experts + stride * L->n_loc;
    L->tab.shared = ExpertPtrs{b, b + o_up, b + o_down, b + o_gs, b + o_us, b + o_ds};
    ALLOC(L->shared_gate_vec, H);
  } else if (L->has_shared) {
    const size_t sgd = Is * (H / 2), sdd = H * (Is / 2);
    size_t so = 0;
    const size_t s_up = so = align_up(sgd, 256);
    const size_t s_down = so = align_up(so + sgd, 256);
    const size_t s_gs = so = align_up(so + sdd, 256);
    const size_t s_us = so = align_up(so + scale_bytes_for(f, Is, H), 256);
    const size_t s_ds = so = align_up(so + scale_bytes_for(f, Is, H), 256);
    so = align_up(so + scale_bytes_for(f, H, Is), 256);
    ALLOC(L->shared, so);
    L->tab.shared = ExpertPtrs{L->shared, L->shared + s_up, L->shared + s_down, L->shared + s_gs,
                               L->shared + s_us, L->shared + s_ds};
    ALLOC(L->shared_gate_vec, H);
  }
  ALLOC(L->router_bias, E);
  L->hr = D.router_hidden > 0 ? D.router_hidden : static_cast<int>(H);
  {
    uint8_t* r = nullptr;
    ALLOC(r, E * L->hr * 4);
    L->router = r;
    const size_t sb = router_slab_bytes(static_cast<int>(E), L->hr, kF32);  // (f32 size: either dtype fits)
    if (sb) ALLOC(L->router_slabs, sb);
  }
  if (L->hr != static_cast<int>(H)) {
    uint8_t* dp = nullptr;
    uint8_t* up = nullptr;
    ALLOC(dp, H * L->hr * 4);
    ALLOC(up, H * L->hr * 4);
    L->lat_down = dp;
    L->lat_up = up;
    ALLOC(L->lat_norm, H);
    ALLOC(L->lat_x, static_cast<size_t>(D.max_tokens) * H);
    ALLOC(L->lat_y, static_cast<size_t>(D.max_tokens) * H);
  }
  // workspace
  const int T = D.max_tokens, k = D.topk;
  const int n_slots = L->n_loc + (L->has_shared ? 1 : 0);
  L->max_tokens = T;
  L->P_max = T * k + (L->has_shared ? T : 0);
  L->h_ld = static_cast<int>(std::max(I, Is));
  const int words = (T + 31) / 32;
  const int max_chunks = L->P_max + n_slots + 1;
  ALLOC(L->logits, static_cast<size_t>(T) * E);
  ALLOC(L->logit_err, static_cast<size_t>(std::min(T, 32)) * E);
  ALLOC(L->fallbacks, 1);
  if (const char* dg = getenv("RMOE_DIAG_HOST")) L->diag_host = dg[0] == '1';
  if (L->diag_host) {
    // diagnostics: the kernel trace in mapped host memory (plain stores only), readable on the
    // host even after a fault has ended the context
    void* hp = nullptr;
    if (cudaHostAlloc(&hp, 8192 * 8 + 64, cudaHostAllocMapped) != cudaSuccess)
      return cleanup(fail(RMOE_CUDA_ERROR, "diagnostic host buffer"));
    memset(hp, 0, 8192 * 8 + 64);
    L->diag_buf = hp;
    void* dp = nullptr;
    if (cudaHostGetDevicePointer(&dp, hp, 0) != cudaSuccess) return cleanup(fail(RMOE_CUDA_ERROR, "diagnostic map"));
    L->tc_trace = static_cast<unsigned long long*>(dp);
    L->tc_trace_print = false;
  }
  ALLOC(L->dev_err, 1);
  {
    void* hp = nullptr;
    if (cudaHostAlloc(&hp, 64, cudaHostAllocDefault) != cudaSuccess) return cleanup(fail(RMOE_CUDA_ERROR, "error flag host copy"));
    L->err_host = static_cast<unsigned*>(hp);
    *L->err_host = 0;
  }
  ALLOC(L->order_pending, 1);
  ALLOC(L->pending, std::min(T, 32));
  ALLOC(L->ids_final, static_cast<size_t>(T) * k);
  ALLOC(L->w_final, static_cast<size_t>(T) * k);
  ALLOC(L->exact_v, static_cast<size_t>(std::min(T, 32)) * k);
  ALLOC(L->resolve_cnt, std::min(T, 32));
  {
    cudaError_t e = cudaMemset(L->fallbacks, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(L->dev_err, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(L->order_pending, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(L->resolve_cnt, 0, 4 * std::min(T, 32));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemset"));
  }
  {
    const char* off = getenv("RMOE_DISABLE_PIPE");
    L->use_pipe = pipe_supported(f, static_cast<int>(H), static_cast<int>(I), static_cast<int>(Is)) &&
                  !(off && off[0] == '1');
    const char* nog = getenv("RMOE_DISABLE_GRAPH");
    L->use_graphs = !(nog && nog[0] == '1');
    L->rpt_gu = L->use_pipe ? 1 : 2;
    L->rpt_dn = L->use_pipe ? 8 : 4;
  }
  ALLOC(L->ids, static_cast<size_t>(T) * k);
  ALLOC(L->rw, static_cast<size_t>(T) * k);
  DispatchBuffers& d = L->d;
  d.words = words;
  d.max_chunks = max_chunks;
  ALLOC(d.bits, static_cast<size_t>(L->n_loc) * words);
  ALLOC(d.first_occ, L->n_loc);
  ALLOC(d.wpre, static_cast<size_t>(L->n_loc) * words);
  ALLOC(d.counts, n_slots + 1);
  ALLOC(d.offsets, n_slots + 2);
  ALLOC(d.uniq, L->n_loc);
  ALLOC(d.n_uniq, 1);
  ALLOC(d.perm_tok, L->P_max);
  ALLOC(d.perm_w, L->P_max);
  ALLOC(d.inv, static_cast<size_t>(T) * k);
  ALLOC(d.ch_expert, max_chunks);
  ALLOC(d.ch_pos, max_chunks);
  ALLOC(d.ch_n, max_chunks);
  ALLOC(d.ch_task_gu, max_chunks + 1);
  ALLOC(d.ch_task_dn, max_chunks + 1);
  ALLOC(d.n_chunks, 1);
  ALLOC(L->xq, static_cast<size_t>(T) * H);
  ALLOC(L->xexp, T);
  ALLOC(L->gate, T);
  ALLOC(L->h, static_cast<size_t>(L->P_max) * L->h_ld);
  ALLOC(L->hmax, L->P_max);
  ALLOC(L->hq, static_cast<size_t>(L->P_max) * L->h_ld);
  ALLOC(L->hexp, L->P_max);
  ALLOC(L->y, static_cast<size_t>(L->P_max) * H);
  if (L->use_tc) {
    const size_t rows = static_cast<size_t>(4) * L->P_max + 16;
    ALLOC(L->tc_stage, 2 * gd + dd + 2 * (I * H / 32) + H * I / 32);  // one expert as uploaded
    ALLOC(L->xt, rows * (H / 2));
    ALLOC(L->xsf, rows * (H / 32));
    ALLOC(L->ht, rows * (I / 2));
    ALLOC(L->hsf, rows * (I / 32));
    ALLOC(L->partial, moe_tc_partial_floats(static_cast<int>(H), static_cast<int>(I), k, n_slots));
    ALLOC(L->partial2, moe_tc_partial_floats(static_cast<int>(H), static_cast<int>(I), k, n_slots));
    ALLOC(L->tc_work, 8);
    const size_t max_tiles = static_cast<size_t>(max_chunks) * std::max(I / 64, H / 128);
    L->tile_cnt_half = max_tiles;
    ALLOC(L->tile_cnt, 2 * max_tiles);
    ALLOC(L->front_counter, 1);
    L->fused_tiles = (RMOE_MAX_TOPK_DEV + 1) * static_cast<int>(I / 64);
    ALLOC(L->fused_cnt, 8 + L->fused_tiles + RMOE_MAX_TOPK_DEV + 1);
    if (const char* nf = getenv("RMOE_DISABLE_FUSED")) L->use_fused = nf[0] != '1';
    if (const char* tr = getenv("RMOE_TC_TRACE"); tr && !L->diag_host) {
      if (tr[0] == '1' || tr[0] == '2') {
        L->tc_trace_print = tr[0] == '1';
        ALLOC(L->tc_trace, 8192);
        if (cudaMemset(L->tc_trace, 0, 8192 * 8) != cudaSuccess) return cleanup(fail(RMOE_CUDA_ERROR, "trace"));
      }
    }
    cudaError_t e = cudaMemset(L->tile_cnt, 0, 2 * max_tiles * 4);
    if (e == cudaSuccess) e = cudaMemset(L->fused_cnt, 0, (8 + L->fused_tiles + RMOE_MAX_TOPK_DEV + 1) * 4);
    if (e == cudaSuccess) e = cudaMemset(L->front_counter, 0, 4);
    if (e == cudaSuccess) e = cudaMemset(L->tc_work, 0, 32);
    if (e == cudaSuccess) e = cudaMemset(L->xt, 0, rows * (H / 2));
    if (e == cudaSuccess) e = cudaMemset(L->xsf, 127, rows * (H / 32));
    if (e == cudaSuccess) e = cudaMemset(L->ht, 0, rows * (I / 2));
    if (e == cudaSuccess) e = cudaMemset(L->hsf, 127, rows * (I / 32));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemset"));
    const size_t pb = (moe_tc_plan_bytes() + 63) / 64 * 64;
    L->tc_plan = aligned_alloc(64, pb);
    if (!L->tc_plan) return cleanup(fail(RMOE_OUT_OF_MEMORY, "rmoe_layer_create: host allocation"));
    if (!moe_tc_plan(L->tc_plan, static_cast<int>(H), static_cast<int>(I), L->xt, L->xsf, L->ht, L->hsf,
                     static_cast<int>(rows)))
      return cleanup(fail(RMOE_CUDA_ERROR, "rmoe_layer_create: tensor map encoding failed"));
  }
  {
    const char* no4 = getenv("RMOE_DISABLE_I4TC");
    L->use_i4tc = f.fmt == kInt4g && !(no4 && no4[0] == '1') &&
                  i4_tc_supported(static_cast<int>(H), static_cast<int>(I), static_cast<int>(Is), f.group_size) &&
                  (!L->has_shared || shared_in_table) && T > kI4MinTokens;
  }
  if (L->use_i4tc) {
    L->i4_off_down = align_up(i4_tc_region_bytes(static_cast<int>(H), static_cast<int>(I), 0), 4096);
    L->i4_stride = align_up(L->i4_off_down + i4_tc_region_bytes(static_cast<int>(H), static_cast<int>(I), 1), 4096);
    ALLOC(L->i4_tiles, L->i4_stride * table_slots);
    const size_t prow = static_cast<size_t>(L->P_max) + 32;
    ALLOC(L->i4_xh, prow * H);
    ALLOC(L->i4_hh, prow * I);
    const size_t mb = (i4_act_map_bytes() + 63) / 64 * 64;
    L->i4_map_x = aligned_alloc(64, mb);
    L->i4_map_h = aligned_alloc(64, mb);
    if (!L->i4_map_x || !L->i4_map_h) return cleanup(fail(RMOE_OUT_OF_MEMORY, "rmoe_layer_create: host allocation"));
    if (cudaMemset(L->i4_xh, 0, prow * H * 2) != cudaSuccess || cudaMemset(L->i4_hh, 0, prow * I * 2) != cudaSuccess)
      return cleanup(fail(RMOE_CUDA_ERROR, "rmoe_layer_create: cudaMemset"));
    if (!i4_make_act_map(L->i4_map_x, L->i4_xh, static_cast<int>(H), static_cast<int>(prow)) ||
        !i4_make_act_map(L->i4_map_h, L->i4_hh, static_cast<int>(I), static_cast<int>(prow)))
      return cleanup(fail(RMOE_CUDA_ERROR, "rmoe_layer_create: tensor map encoding failed"));
    if (const char* tr = getenv("RMOE_TC_TRACE"); tr && tr[0] == '2' && !L->tc_trace) {
      ALLOC(L->tc_trace, 8192);  // the int4 gate/up kernel's stage timeline (printed by get_stats)
      if (cudaMemset(L->tc_trace, 0, 8192 * 8) != cudaSuccess) return cleanup(fail(RMOE_CUDA_ERROR, "trace"));
    }
  }
  {
    uint8_t* xd = nullptr;
    ALLOC(xd, static_cast<size_t>(T) * H * 4);
    L->x_dev = xd;
  }
  ALLOC(L->out_dev, static_cast<size_t>(T) * H);
  ALLOC(L->out_stage, static_cast<size_t>(T) * H);
  {
    uint8_t* xs = nullptr;
    ALLOC(xs, static_cast<size_t>(T) * H * 4);
    L->x_stage = xs;
  }
  ALLOC(L->ids_host_stage, static_cast<size_t>(T) * k);
  ALLOC(L->w_host_stage, static_cast<size_t>(T) * k);
  {
    cudaError_t e = cudaStreamCreateWithFlags(&L->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&L->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&L->cap, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->ev_join, cudaEventDisableTiming);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "cudaStreamCreate"));
  }
#undef ALLOC
  L->stats.local_expert_begin = L->e_begin;
  L->stats.local_expert_end = L->e_end;
  L->stats.device_bytes = stride * table_slots + E * H * 4;
  *out = L;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_layer_destroy(rmoe_layer* L) {
  if (!L) return RMOE_OK;
  cudaSetDevice(L->ctx->device);
  if (L->stream) {
    cudaStreamSynchronize(L->stream);
    cudaStreamDestroy(L->stream);
  }
  if (L->side) {
    cudaStreamSynchronize(L->side);
    cudaStreamDestroy(L->side);
  }
  if (L->ev_fork) cudaEventDestroy(L->ev_fork);
  if (L->ev_join) cudaEventDestroy(L->ev_join);
  delete L;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_layer_get_desc(const rmoe_layer* L, rmoe_layer_desc* out) {
  if (!L || !out) return fail(RMOE_INVALID_ARG, "rmoe_layer_get_desc: null argument");
  *out = L->desc;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_layer_get_stats(const rmoe_layer* L, rmoe_layer_stats* out) {
  if (!L || !out) return fail(RMOE_INVALID_ARG, "rmoe_layer_get_stats: null argument");
  *out = L->stats;
  unsigned fb = 0;
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  RMOE_CUDA(cudaMemcpy(&fb, L->fallbacks, 4, cudaMemcpyDeviceToHost), "read fallback counter");
  out->router_fallbacks = fb;
  unsigned ef = 0;
  RMOE_CUDA(cudaMemcpy(&ef, L->dev_err, 4, cudaMemcpyDeviceToHost), "read device error flags");
  out->device_error_flags = ef | L->err_seen;
  unsigned op = 0;
  RMOE_CUDA(cudaMemcpy(&op, L->order_pending, 4, cudaMemcpyDeviceToHost), "read order counter");
  out->router_order_resolved = op;
  if (L->tc_trace && L->use_i4tc) {
    // diagnostics: the int4 gate/up kernel's first stages on CTA 0 (µs from the first copy)
    static unsigned long long tr[4096];
    RMOE_CUDA(cudaDeviceSynchronize(), "trace sync");
    RMOE_CUDA(cudaMemcpy(tr, L->tc_trace, sizeof(tr), cudaMemcpyDeviceToHost), "trace read");
    const unsigned long long t0 = tr[0];
    auto rel = [&](unsigned long long t) { return t ? (double)(long long)(t - t0) * 1e-3 : -1.0; };
    fprintf(stderr, "int4 gate/up stages (copies issued, weights landed, dequant start, dequant done, A ready at MMA, "
                    "activations landed at MMA):\n");
    for (int i = 0; i < 512; i += (i < 24 ? 1 : 32))
      fprintf(stderr, "  %3d: %.2f %.2f %.2f %.2f %.2f %.2f\n", i, rel(tr[8 * i]), rel(tr[8 * i + 1]), rel(tr[8 * i + 2]),
              rel(tr[8 * i + 3]), rel(tr[8 * i + 5]), rel(tr[8 * i + 4]));
    return RMOE_OK;
  }
  if (L->tc_trace && !L->tc_trace_print) {
    // diagnostics: the last one-token forward's kernel timeline (global timer, µs from the
    // front end's start)
    static unsigned long long tr[8192];
    RMOE_CUDA(cudaDeviceSynchronize(), "trace sync");
    RMOE_CUDA(cudaMemcpy(tr, L->tc_trace, sizeof(tr), cudaMemcpyDeviceToHost), "trace read");
    const unsigned long long f0 = tr[4000];
    auto rel = [&](unsigned long long t) { return t ? (double)(long long)(t - f0) * 1e-3 : -1.0; };
    fprintf(stderr, "timeline: front end %.2f (router blocks %.2f, other blocks %.2f, last block %.2f, select %.2f, certificate %.2f)",
            rel(tr[4006]), rel(tr[4001]), rel(tr[4002]), rel(tr[4003]), rel(tr[4004]), rel(tr[4005]));
    if (L->use_fused) {
      const unsigned long long* b = tr + 4096 + 2048;
      const char* nm[7] = {"entry", "set-up", "first copy", "first down unit", "epilogue done", "barrier passed", "exit"};
      for (int f = 0; f < 7; f++) {
        unsigned long long lo = ~0ull, hi = 0;
        for (int c = 0; c < 148; c++) {
          const unsigned long long v = b[8 * c + f];
          if (!v) continue;
          lo = std::min(lo, v);
          hi = std::max(hi, v);
        }
        if (hi) fprintf(stderr, " | fused %s %.2f..%.2f", nm[f], rel(lo), rel(hi));
      }
      fprintf(stderr, "\n");
      // per CTA: epilogue done, barrier passed, exit
      fprintf(stderr, "fused per CTA (epilogue done / barrier / exit):");
      for (int c = 0; c < 148; c++)
        fprintf(stderr, "%s%d:%.1f/%.1f/%.1f", c % 8 ? " " : "\n  ", c, rel(b[8 * c + 4]), rel(b[8 * c + 5]),
                rel(b[8 * c + 6]));
      fprintf(stderr, "\n");
      RMOE_CUDA(cudaMemset(L->tc_trace + 4096 + 2048, 0, 148 * 8 * 8), "fused trace reset");
    }
    for (int k = 0; k < 2; k++) {
      const unsigned long long* b = tr + 4096 * k;
      unsigned long long e0 = ~0ull, e1 = 0, x0 = ~0ull, x1 = 0, s1 = 0;
      for (int c = 0; c < 148 && b[1024 + 4 * c]; c++) {
        e0 = std::min(e0, b[1024 + 4 * c]); e1 = std::max(e1, b[1024 + 4 * c]);
        s1 = std::max(s1, b[1024 + 4 * c + 1]);
        x0 = std::min(x0, b[1024 + 4 * c + 3]); x1 = std::max(x1, b[1024 + 4 * c + 3]);
      }
      fprintf(stderr, " | %s: CTA entry %.2f..%.2f set-up done %.2f first issue %.2f exit %.2f..%.2f",
              k ? "down" : "gate/up", rel(e0), rel(e1), rel(s1), rel(b[0]), rel(x0), rel(x1));
    }
    fprintf(stderr, "\n");
    for (int k = 0; k < 2; k++) {
      const unsigned long long* b = tr + 4096 * k;
      fprintf(stderr, "  %s CTA 0 parts (accumulator ready -> epilogue done):", k ? "down" : "gate/up");
      for (int i = 0; i < 16 && b[3072 + i * 4]; i++) fprintf(stderr, " %.1f->%.1f", rel(b[3072 + i * 4 + 1]), rel(b[3072 + i * 4 + 2]));
      fprintf(stderr, "\n");
      fprintf(stderr, "    producer role start %.2f unit fields %.2f; part stores begin %.2f %.2f %.2f %.2f\n", rel(b[1700]),
              rel(b[1701]), rel(b[1711]), rel(b[1712]), rel(b[1713]), rel(b[1714]));
      if (k) fprintf(stderr, "    h: act producer wait done %.2f, barrier poll from %.2f seen %.2f; epilogue wait done %.2f, finalize done %.2f;"
                     " first B landed %.2f\n", rel(b[1720]), rel(b[1721]), rel(b[1722]), rel(b[1723]), rel(b[1724]), rel(b[1]));
    }
  }
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_layer_set_profiling(rmoe_layer* L, int on) {
  if (!L) return fail(RMOE_INVALID_ARG, "rmoe_layer_set_profiling: null layer");
  L->profiling = on != 0;
  return RMOE_OK;
}

static rmoe_status drain_graph_profile(rmoe_layer* L, GraphEntry& g);

// Reads the layer's device error flags (bounded waits of its kernels that ran out) once the
// work on the layer's streams is done. Nonzero: the outputs of the calls since the last check
// are invalid, and the persistent kernels' work counters may be left mid-count, so they are
// zeroed (with the device idle) and the flags cleared: the next call runs normally.
// Destroys the captured forward graphs (after the device is idle): a change of the layer's
// kernel parameters or routing configuration is captured again on the next call.
static rmoe_status drop_graphs(rmoe_layer* L) {
  if (L->graphs.empty()) return RMOE_OK;
  RMOE_CUDA(cudaDeviceSynchronize(), "drop graphs: synchronize");
  for (auto& kv : L->graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
    for (cudaEvent_t e : kv.second.ev)
      if (e) cudaEventDestroy(e);
  }
  L->graphs.clear();
  return RMOE_OK;
}

// ef_read: the flags already copied to the host behind the call's work (else read them here).
static rmoe_status take_device_errors(rmoe_layer* L, const char* what, const unsigned* ef_read = nullptr) {
  unsigned ef = 0;
  if (ef_read)
    ef = *ef_read;
  else
    RMOE_CUDA(cudaMemcpy(&ef, L->dev_err, 4, cudaMemcpyDeviceToHost), "read device error flags");
  if (!ef) return RMOE_OK;
  RMOE_CUDA(cudaDeviceSynchronize(), "timeout recovery: synchronize");
  const int T = L->max_tokens;
  RMOE_CUDA(cudaMemset(L->dev_err, 0, 4), "timeout recovery");
  RMOE_CUDA(cudaMemset(L->resolve_cnt, 0, 4 * std::min(T, 32)), "timeout recovery");
  if (L->use_tc) {
    RMOE_CUDA(cudaMemset(L->tile_cnt, 0, 2 * L->tile_cnt_half * 4), "timeout recovery");
    RMOE_CUDA(cudaMemset(L->fused_cnt, 0, (8 + L->fused_tiles + RMOE_MAX_TOPK_DEV + 1) * 4), "timeout recovery");
    RMOE_CUDA(cudaMemset(L->front_counter, 0, 4), "timeout recovery");
    RMOE_CUDA(cudaMemset(L->tc_work, 0, 32), "timeout recovery");
  }
  L->err_seen |= ef;
  return fail(RMOE_TIMEOUT,
              "%s: a bounded device-side wait ran out (flags 0x%x); the outputs of the calls since the "
              "last check are invalid; the layer's counters were reset for the next call",
              what, ef);
}

extern "C" rmoe_status rmoe_layer_check(rmoe_layer* L, void* stream) {
  if (!L) return fail(RMOE_INVALID_ARG, "rmoe_layer_check: null layer");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  RMOE_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "rmoe_layer_check synchronize");
  RMOE_CUDA(cudaStreamSynchronize(L->side), "rmoe_layer_check synchronize");
  return take_device_errors(L, "rmoe_layer_check");
}

extern "C" rmoe_status rmoe_layer_set_wait_limit(rmoe_layer* L, uint64_t ns) {
  if (!L) return fail(RMOE_INVALID_ARG, "rmoe_layer_set_wait_limit: null layer");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  const unsigned long long v = ns ? ns : kDefaultSpinNs;
  if (v == L->spin_ns) return RMOE_OK;
  // the captured one-token graphs hold the old limit in their kernel arguments
  rmoe_status s = drop_graphs(L);
  if (s != RMOE_OK) return s;
  L->spin_ns = v;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_set_route_config(rmoe_layer* L, int32_t cache_route, int32_t route_j, int32_t route_m,
                                             const uint8_t* resident) {
  const char* what = "rmoe_set_route_config";
  if (!L) return fail(RMOE_INVALID_ARG, "%s: null layer", what);
  if (cache_route && L->desc.router_kind != RMOE_ROUTER_SIGMOID_GROUPED)
    return fail(RMOE_NOT_SUPPORTED, "%s: CACHE_ROUTE applies to the sigmoid router only (the softmax router has none)", what);
  if (cache_route && (route_j < 0 || route_m < 0 || std::max<int>(route_m, L->desc.topk) > 32))
    return fail(RMOE_INVALID_ARG, "%s: route_j %d, route_m %d (0 <= route_j, max(route_m, k) <= 32)", what, route_j, route_m);
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  rmoe_status s = drop_graphs(L);
  if (s != RMOE_OK) return s;
  if (resident) {
    if (!L->resident) {
      void* p = nullptr;
      RMOE_CUDA(cudaMalloc(&p, L->desc.n_experts), "rmoe_set_route_config resident mask");
      L->arena.ptrs.push_back(p);
      L->resident = static_cast<uint8_t*>(p);
    }
    RMOE_CUDA(cudaMemcpy(L->resident, resident, L->desc.n_experts, cudaMemcpyDefault), "resident mask");
  }
  L->cache_route = cache_route != 0;
  L->route_j = route_j;
  L->route_m = route_m;
  L->resident_all = resident == nullptr;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_layer_get_profile(rmoe_layer* L, rmoe_profile* out) {
  if (!L || !out) return fail(RMOE_INVALID_ARG, "rmoe_layer_get_profile: null argument");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  for (auto& kv : L->graphs) {
    rmoe_status s = drain_graph_profile(L, kv.second);
    if (s != RMOE_OK) return s;
  }
  const size_t G = RMOE_NUM_STAGES + 1;
  for (size_t g = 0; g + G <= L->ev_pending.size(); g += G) {
    RMOE_CUDA(cudaEventSynchronize(L->ev_pending[g + G - 1]), "profile event");
    for (int s = 0; s < RMOE_NUM_STAGES; s++) {
      float ms = 0.0f;
      RMOE_CUDA(cudaEventElapsedTime(&ms, L->ev_pending[g + s], L->ev_pending[g + s + 1]), "profile elapsed");
      L->prof_ms[s] += ms;
    }
    L->prof_calls++;
  }
  L->ev_free.insert(L->ev_free.end(), L->ev_pending.begin(), L->ev_pending.end());
  L->ev_pending.clear();
  out->calls = L->prof_calls;
  for (int s = 0; s < RMOE_NUM_STAGES; s++) out->stage_ms[s] = L->prof_ms[s];
  L->prof_calls = 0;
  for (double& v : L->prof_ms) v = 0.0;
  return RMOE_OK;
}

// ------------------------------------------------------------------------------ uploads
extern "C" rmoe_status rmoe_upload_router(rmoe_layer* L, const void* w, int32_t dtype, size_t bytes) {
  if (!L || !w) return fail(RMOE_INVALID_ARG, "rmoe_upload_router: null argument");
  if (dtype != RMOE_F32 && dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "rmoe_upload_router: dtype %d", dtype);
  const size_t want = static_cast<size_t>(L->desc.n_experts) * L->hr * (dtype == RMOE_BF16 ? 2 : 4);
  if (bytes != want)
    return fail(RMOE_SHAPE_MISMATCH, "rmoe_upload_router: %zu bytes, [%d, %d] needs %zu", bytes,
                L->desc.n_experts, L->hr, want);
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  RMOE_CUDA(cudaMemcpy(L->router, w, bytes, cudaMemcpyDefault), "rmoe_upload_router copy");
  L->router_dtype = dtype == RMOE_BF16 ? kBF16 : kF32;
  if (L->router_slabs) {
    RMOE_CUDA(launch_router_slabs(L->router, L->router_dtype, L->desc.n_experts, L->hr, L->router_slabs, nullptr),
              "router slab layout");
    RMOE_CUDA(cudaDeviceSynchronize(), "router slab layout");
  }
  L->has_router = true;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_upload_router_bias(rmoe_layer* L, const float* bias, size_t n) {
  if (!L || !bias) return fail(RMOE_INVALID_ARG, "rmoe_upload_router_bias: null argument");
  if (n != static_cast<size_t>(L->desc.n_experts))
    return fail(RMOE_SHAPE_MISMATCH, "rmoe_upload_router_bias: %zu values for %d experts", n, L->desc.n_experts);
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  RMOE_CUDA(cudaMemcpy(L->router_bias, bias, n * 4, cudaMemcpyDefault), "rmoe_upload_router_bias copy");
  L->has_bias = true;
  return RMOE_OK;
}

// Checks (data, scale) byte counts of one [rows, cols] matrix like mxfp4_from_raw
// (src/expert_cache.rs:1245-1256) and copies them.
static rmoe_status put_matrix(const rmoe_layer* L, const char* what, size_t rows, size_t cols,
                              const void* data, size_t data_bytes, const void* scale,
                              size_t scale_bytes, uint8_t* ddst, uint8_t* sdst) {
  if (!data || !scale) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  const size_t want_d = rows * ((cols + 1) / 2);
  const size_t want_s = scale_bytes_for(L->fmt, rows, cols);
  if (data_bytes != want_d)
    return fail(RMOE_SHAPE_MISMATCH, "%s: %zu data bytes, [%zu, %zu] needs %zu", what, data_bytes, rows, cols, want_d);
  if (scale_bytes != want_s)
    return fail(RMOE_SHAPE_MISMATCH, "%s: %zu scale bytes, [%zu, %zu] needs %zu", what, scale_bytes, rows, cols, want_s);
  RMOE_CUDA(cudaMemcpy(ddst, data, data_bytes, cudaMemcpyDefault), what);
  RMOE_CUDA(cudaMemcpy(sdst, scale, scale_bytes, cudaMemcpyDefault), what);
  return RMOE_OK;
}

// Tensor-core layers: the three matrices go through a staging copy in the reference layout and
// are retiled into the expert's slot (gate/up tiles, then down tiles).
static rmoe_status put_tiled(rmoe_layer* L, const char* what, const void* gate, size_t gate_bytes,
                             const void* gate_scale, size_t gate_scale_bytes, const void* up, size_t up_bytes,
                             const void* up_scale, size_t up_scale_bytes, const void* down, size_t down_bytes,
                             const void* down_scale, size_t down_scale_bytes, uint8_t* slot) {
  const size_t H = L->desc.hidden, I = L->desc.moe_inter;
  const size_t gd = I * (H / 2), dd = H * (I / 2), gs = I * (H / 32), ds = H * (I / 32);
  uint8_t* g = L->tc_stage;
  uint8_t* u = g + gd;
  uint8_t* dn = u + gd;
  uint8_t* gsc = dn + dd;
  uint8_t* usc = gsc + gs;
  uint8_t* dsc = usc + gs;
  rmoe_status s;
  if ((s = put_matrix(L, what, I, H, gate, gate_bytes, gate_scale, gate_scale_bytes, g, gsc)) != RMOE_OK) return s;
  if ((s = put_matrix(L, what, I, H, up, up_bytes, up_scale, up_scale_bytes, u, usc)) != RMOE_OK) return s;
  if ((s = put_matrix(L, what, H, I, down, down_bytes, down_scale, down_scale_bytes, dn, dsc)) != RMOE_OK) return s;
  cudaError_t e = launch_tc_relayout(0, g, u, gsc, usc, static_cast<int>(H), static_cast<int>(I), slot, 0);
  if (e == cudaSuccess)
    e = launch_tc_relayout(1, dn, nullptr, dsc, nullptr, static_cast<int>(H), static_cast<int>(I),
                           slot + L->tc_off_down, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return RMOE_OK;
}

// Grouped-int4 layers on the tensor cores: the slot's matrices (already uploaded in the
// reference layout at gate/up/down) retiled into the slot's tile-major copy.
static rmoe_status put_i4_tiles(rmoe_layer* L, const char* what, const uint8_t* gate, const uint8_t* up,
                                const uint8_t* down, const void* gsc, const void* usc, const void* dsc, int slot) {
  if (!L->use_i4tc) return RMOE_OK;
  const int H = L->desc.hidden, I = L->desc.moe_inter, gs = L->fmt.group_size;
  const int bf = L->fmt.scale_dtype == kBF16 ? 1 : 0;
  uint8_t* dst = L->i4_tiles + L->i4_stride * slot;
  cudaError_t e = launch_i4_relayout(0, gate, up, gsc, usc, bf, H, I, gs, dst, 0);
  if (e == cudaSuccess) e = launch_i4_relayout(1, down, nullptr, dsc, nullptr, bf, H, I, gs, dst + L->i4_off_down, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return RMOE_OK;
}

static rmoe_status local_slot(const rmoe_layer* L, int32_t eid, const char* what, int* slot) {
  if (!L) return fail(RMOE_INVALID_ARG, "%s: null layer", what);
  if (eid < 0 || eid >= L->desc.n_experts)
    return fail(RMOE_INVALID_ARG, "%s: expert %d out of range [0, %d)", what, eid, L->desc.n_experts);
  if (eid < L->e_begin || eid >= L->e_end)
    return fail(RMOE_INVALID_ARG, "%s: expert %d is not resident on EP rank %d (experts %d..%d)", what, eid,
                L->desc.ep_rank, L->e_begin, L->e_end - 1);
  *slot = eid - L->e_begin;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_upload_expert(rmoe_layer* L, int32_t eid, const void* gate,
                                          size_t gate_bytes, const void* gate_scale,
                                          size_t gate_scale_bytes, const void* up, size_t up_bytes,
                                          const void* up_scale, size_t up_scale_bytes,
                                          const void* down, size_t down_bytes,
                                          const void* down_scale, size_t down_scale_bytes) {
  int slot = 0;
  rmoe_status s = local_slot(L, eid, "rmoe_upload_expert", &slot);
  if (s != RMOE_OK) return s;
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  const size_t H = L->desc.hidden, I = L->desc.moe_inter;
  uint8_t* b = L->experts + L->tab.stride * slot;
  if (L->use_tc) {
    if ((s = put_tiled(L, "rmoe_upload_expert", gate, gate_bytes, gate_scale, gate_scale_bytes, up, up_bytes,
                       up_scale, up_scale_bytes, down, down_bytes, down_scale, down_scale_bytes, b)) != RMOE_OK)
      return s;
    L->uploaded[slot] = 1;
    return RMOE_OK;
  }
  if ((s = put_matrix(L, "rmoe_upload_expert gate", I, H, gate, gate_bytes, gate_scale,
                      gate_scale_bytes, b, b + L->tab.off_gs)) != RMOE_OK)
    return s;
  if ((s = put_matrix(L, "rmoe_upload_expert up", I, H, up, up_bytes, up_scale, up_scale_bytes,
                      b + L->tab.off_up, b + L->tab.off_us)) != RMOE_OK)
    return s;
  if ((s = put_matrix(L, "rmoe_upload_expert down", H, I, down, down_bytes, down_scale,
                      down_scale_bytes, b + L->tab.off_down, b + L->tab.off_ds)) != RMOE_OK)
    return s;
  if ((s = put_i4_tiles(L, "rmoe_upload_expert (int4 tiles)", b, b + L->tab.off_up, b + L->tab.off_down,
                        b + L->tab.off_gs, b + L->tab.off_us, b + L->tab.off_ds, slot)) != RMOE_OK)
    return s;
  L->uploaded[slot] = 1;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_upload_expert_fused(rmoe_layer* L, int32_t eid, const void* gate_up,
                                                size_t gate_up_bytes, const void* gate_up_scale,
                                                size_t gate_up_scale_bytes, const void* down,
                                                size_t down_bytes, const void* down_scale,
                                                size_t down_scale_bytes) {
  if (!L || !gate_up || !gate_up_scale) return fail(RMOE_INVALID_ARG, "rmoe_upload_expert_fused: null argument");
  const size_t H = L->desc.hidden, I = L->desc.moe_inter;
  const size_t half_d = I * ((H + 1) / 2), half_s = scale_bytes_for(L->fmt, I, H);
  if (gate_up_bytes != 2 * half_d || gate_up_scale_bytes != 2 * half_s)
    return fail(RMOE_SHAPE_MISMATCH, "rmoe_upload_expert_fused: %zu/%zu bytes, [2*%zu, %zu] needs %zu/%zu",
                gate_up_bytes, gate_up_scale_bytes, I, H, 2 * half_d, 2 * half_s);
  // gate rows 0..I then up rows I..2I: the same bytes as Separate{gate, up} back to back
  const uint8_t* gu = static_cast<const uint8_t*>(gate_up);
  const uint8_t* gus = static_cast<const uint8_t*>(gate_up_scale);
  return rmoe_upload_expert(L, eid, gu, half_d, gus, half_s, gu + half_d, half_d, gus + half_s,
                            half_s, down, down_bytes, down_scale, down_scale_bytes);
}

extern "C" rmoe_status rmoe_upload_shared(rmoe_layer* L, const void* gate, size_t gate_bytes,
                                          const void* gate_scale, size_t gate_scale_bytes,
                                          const void* up, size_t up_bytes, const void* up_scale,
                                          size_t up_scale_bytes, const void* down,
                                          size_t down_bytes, const void* down_scale,
                                          size_t down_scale_bytes, const float* shared_gate) {
  if (!L) return fail(RMOE_INVALID_ARG, "rmoe_upload_shared: null layer");
  if (!L->has_shared) return fail(RMOE_INVALID_ARG, "rmoe_upload_shared: layer was created with shared_inter = 0");
  if (L->desc.shared_gated && !shared_gate)
    return fail(RMOE_INVALID_ARG, "rmoe_upload_shared: shared_gated layer needs shared_gate");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  const size_t H = L->desc.hidden, Is = L->desc.shared_inter;
  const ExpertPtrs& p = L->tab.shared;
  rmoe_status s;
  if (L->use_tc) {
    if ((s = put_tiled(L, "rmoe_upload_shared", gate, gate_bytes, gate_scale, gate_scale_bytes, up, up_bytes,
                       up_scale, up_scale_bytes, down, down_bytes, down_scale, down_scale_bytes,
                       L->experts + L->tab.stride * L->n_loc)) != RMOE_OK)
      return s;
    if (shared_gate && L->desc.shared_gated)
      RMOE_CUDA(cudaMemcpy(L->shared_gate_vec, shared_gate, H * 4, cudaMemcpyDefault), "rmoe_upload_shared gate vector");
    L->has_shared_w = true;
    return RMOE_OK;
  }
  if ((s = put_matrix(L, "rmoe_upload_shared gate", Is, H, gate, gate_bytes, gate_scale, gate_scale_bytes,
                      const_cast<uint8_t*>(p.gate), (uint8_t*)p.gate_scale)) != RMOE_OK)
    return s;
  if ((s = put_matrix(L, "rmoe_upload_shared up", Is, H, up, up_bytes, up_scale, up_scale_bytes,
                      const_cast<uint8_t*>(p.up), (uint8_t*)p.up_scale)) != RMOE_OK)
    return s;
  if ((s = put_matrix(L, "rmoe_upload_shared down", H, Is, down, down_bytes, down_scale, down_scale_bytes,
                      const_cast<uint8_t*>(p.down), (uint8_t*)p.down_scale)) != RMOE_OK)
    return s;
  if ((s = put_i4_tiles(L, "rmoe_upload_shared (int4 tiles)", p.gate, p.up, p.down, p.gate_scale, p.up_scale,
                        p.down_scale, L->n_loc)) != RMOE_OK)
    return s;
  if (shared_gate && L->desc.shared_gated)
    RMOE_CUDA(cudaMemcpy(L->shared_gate_vec, shared_gate, H * 4, cudaMemcpyDefault), "rmoe_upload_shared gate vector");
  L->has_shared_w = true;
  return RMOE_OK;
}

// ------------------------------------------------------------------------------ forward
static rmoe_status check_ready(const rmoe_layer* L, const char* what, int T, int x_dtype) {
  if (!L) return fail(RMOE_INVALID_ARG, "%s: null layer", what);
  if (T < 0 || T > L->max_tokens)
    return fail(RMOE_INVALID_ARG, "%s: T = %d outside [0, max_tokens = %d]", what, T, L->max_tokens);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  if (!L->has_router) return fail(RMOE_INVALID_ARG, "%s: router weights were never uploaded", what);
  if (L->desc.router_kind == RMOE_ROUTER_SIGMOID_GROUPED && !L->has_bias)
    return fail(RMOE_INVALID_ARG, "%s: sigmoid router needs rmoe_upload_router_bias", what);
  return RMOE_OK;
}

static rmoe_status route_into(rmoe_layer* L, const void* x, int x_dtype, int T, cudaStream_t st,
                              StageMarks* marks = nullptr) {
  const rmoe_layer_desc& D = L->desc;
  cudaError_t e = launch_router_logits_exact(x, x_dtype == RMOE_BF16 ? kBF16 : kF32, L->router,
                                             L->router_dtype, L->logits, T, L->hr, D.n_experts, st, L->dev_err,
                                             L->router_slabs);
  if (e != cudaSuccess) return cuda_fail(e, "router logits");
  if (marks) marks->mark();
  if (D.router_kind == RMOE_ROUTER_SOFTMAX_TOPK)
    e = launch_topk_softmax(L->logits, L->has_bias ? L->router_bias : nullptr, T, D.n_experts, D.topk,
                            L->ids, L->rw, st);
  else if (L->cache_route)
    e = launch_topk_cache_route(L->logits, L->router_bias, T, D.n_experts, D.topk, L->route_j, L->route_m,
                                L->resident_all ? nullptr : L->resident, D.norm_topk, D.routed_scale, L->ids, L->rw,
                                st);
  else
    e = launch_topk_grouped(L->logits, L->router_bias, T, D.n_experts, D.topk, D.n_group,
                            D.topk_group, D.norm_topk, D.routed_scale, L->ids, L->rw, st);
  if (e != cudaSuccess) return cuda_fail(e, "router top-k");
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_route(rmoe_layer* L, const void* x, int32_t x_dtype, int32_t T,
                                  int32_t* ids, float* weights, void* stream) {
  rmoe_status s = check_ready(L, "rmoe_route", T, x_dtype);
  if (s != RMOE_OK) return s;
  if (T == 0) return RMOE_OK;
  if (!x || !ids || !weights) return fail(RMOE_INVALID_ARG, "rmoe_route: null pointer");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((s = route_into(L, x, x_dtype, T, st)) != RMOE_OK) return s;
  const size_t n = static_cast<size_t>(T) * L->desc.topk;
  RMOE_CUDA(cudaMemcpyAsync(ids, L->ids, n * 4, cudaMemcpyDeviceToDevice, st), "rmoe_route ids");
  RMOE_CUDA(cudaMemcpyAsync(weights, L->rw, n * 4, cudaMemcpyDeviceToDevice, st), "rmoe_route weights");
  return RMOE_OK;
}

// The decode-sized front end: softmax router, T <= 32, H a multiple of 256.
static bool small_path(const rmoe_layer* L, int T) {
  return T <= 32 && L->desc.router_kind == RMOE_ROUTER_SOFTMAX_TOPK && L->desc.hidden % 256 == 0 &&
         L->desc.topk <= 32 && L->hr == L->desc.hidden;
}

static int chunk_tokens(int T) { return T >= 8 ? 8 : (T >= 4 ? 4 : (T >= 2 ? 2 : 1)); }

static rmoe_status dispatch_into(rmoe_layer* L, int T, int mt, const float* gate, cudaStream_t st,
                                 bool hs) {
  const rmoe_layer_desc& D = L->desc;
  cudaError_t e = launch_dispatch(L->ids, L->rw, T, D.topk, L->e_begin, L->e_end, mt,
                                  hs ? 1 : 0, gate, D.moe_inter, D.shared_inter,
                                  D.hidden, L->rpt_gu, L->rpt_dn, L->d, st);
  if (e != cudaSuccess) return cuda_fail(e, "dispatch");
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_dispatch(rmoe_layer* L, const int32_t* ids, int32_t T, int32_t* counts,
                                     int32_t* offsets, int32_t* perm_token, int32_t* uniq,
                                     int32_t* n_uniq, void* stream) {
  if (!L || (!ids && T > 0)) return fail(RMOE_INVALID_ARG, "rmoe_dispatch: null argument");
  if (T < 0 || T > L->max_tokens) return fail(RMOE_INVALID_ARG, "rmoe_dispatch: T = %d", T);
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t n = static_cast<size_t>(T) * L->desc.topk;
  RMOE_CUDA(cudaMemcpyAsync(L->ids, ids, n * 4, cudaMemcpyDeviceToDevice, st), "rmoe_dispatch ids");
  RMOE_CUDA(cudaMemsetAsync(L->rw, 0, n * 4, st), "rmoe_dispatch weights");
  rmoe_status s = dispatch_into(L, T, chunk_tokens(T), nullptr, st, L->has_shared);
  if (s != RMOE_OK) return s;
  const int E = L->n_loc;
  if (counts) RMOE_CUDA(cudaMemcpyAsync(counts, L->d.counts, E * 4, cudaMemcpyDeviceToDevice, st), "counts");
  if (offsets) RMOE_CUDA(cudaMemcpyAsync(offsets, L->d.offsets, (E + 1) * 4, cudaMemcpyDeviceToDevice, st), "offsets");
  if (perm_token) RMOE_CUDA(cudaMemcpyAsync(perm_token, L->d.perm_tok, n * 4, cudaMemcpyDeviceToDevice, st), "perm");
  if (uniq) RMOE_CUDA(cudaMemcpyAsync(uniq, L->d.uniq, E * 4, cudaMemcpyDeviceToDevice, st), "uniq");
  if (n_uniq) RMOE_CUDA(cudaMemcpyAsync(n_uniq, L->d.n_uniq, 4, cudaMemcpyDeviceToDevice, st), "n_uniq");
  return RMOE_OK;
}

// Diagnostics (RMOE_TC_TRACE=1, direct launches only): CTA 0's stage timeline and every CTA's
// entry / exit of the last tensor-core kernel, to stderr.
static rmoe_status print_tc_trace(rmoe_layer* L, cudaStream_t st, const char* what, size_t off) {
  fprintf(stderr, "== %s\n", what);
  {
    unsigned long long t0h = 0;
    RMOE_CUDA(cudaMemcpy(&t0h, L->tc_trace + off, 8, cudaMemcpyDeviceToHost), "trace t0");
    fprintf(stderr, "   t0 (first issue, globaltimer) = %llu ns\n", t0h);
  }
      static unsigned long long tr[4096];
      RMOE_CUDA(cudaStreamSynchronize(st), "trace sync");
      RMOE_CUDA(cudaMemcpy(tr, L->tc_trace + off, sizeof(tr), cudaMemcpyDeviceToHost), "trace read");
      const unsigned long long t0 = tr[0];
      unsigned long long s0 = ~0ull, s1 = 0, e0 = ~0ull, e1 = 0;
      for (int c = 0; c < 256 && tr[1024 + 4 * c]; c++) {
        s0 = std::min(s0, tr[1024 + 4 * c]); s1 = std::max(s1, tr[1024 + 4 * c]);
        e0 = std::min(e0, tr[1024 + 4 * c + 3]); e1 = std::max(e1, tr[1024 + 4 * c + 3]);
      }
      fprintf(stderr, "cta entry %.2f..%.2f  exit %.2f..%.2f us (rel. cta0 first issue); cta0 setup done %.2f epi done %.2f exit %.2f\n",
              (double)(long long)(s0 - t0) * 1e-3, (double)(long long)(s1 - t0) * 1e-3, (double)(long long)(e0 - t0) * 1e-3,
              (double)(long long)(e1 - t0) * 1e-3, (double)(long long)(tr[1025] - t0) * 1e-3,
              (double)(long long)(tr[1026] - t0) * 1e-3, (double)(long long)(tr[1027] - t0) * 1e-3);
      for (int c = 0; c < 148 && tr[1024 + 4 * c]; c += 16)
        fprintf(stderr, "  cta %3d entry %.2f exit %.2f\n", c, (double)(long long)(tr[1024 + 4 * c] - t0) * 1e-3,
                (double)(long long)(tr[1024 + 4 * c + 3] - t0) * 1e-3);
      for (int i = 0; i < 32 && tr[3072 + i * 4]; i++)
        fprintf(stderr, "  epi part %2d (tile*16+unit %4llu): wait from %7.2f got %7.2f done %7.2f us\n", i, tr[3072 + i * 4 + 3],
                (double)(long long)(tr[3072 + i * 4] - t0) * 1e-3, (double)(long long)(tr[3072 + i * 4 + 1] - t0) * 1e-3,
                (double)(long long)(tr[3072 + i * 4 + 2] - t0) * 1e-3);
      if (off == 0 && tr[4000])
        fprintf(stderr, "  front: block0 start 0, router blocks done %.2f, terms blocks done %.2f, last block: "
                "enter %.2f select %.2f certificate %.2f end %.2f us (GU t0 %.2f)\n",
                (double)(long long)(tr[4001] - tr[4000]) * 1e-3, (double)(long long)(tr[4002] - tr[4000]) * 1e-3,
                (double)(long long)(tr[4003] - tr[4000]) * 1e-3, (double)(long long)(tr[4004] - tr[4000]) * 1e-3,
                (double)(long long)(tr[4005] - tr[4000]) * 1e-3, (double)(long long)(tr[4006] - tr[4000]) * 1e-3,
                (double)(long long)(t0 - tr[4000]) * 1e-3);
      for (int i = 0; i < 32 && tr[3584 + i * 4]; i++)
        fprintf(stderr, "  epi(q0) %2d: got %7.2f ld %7.2f ubuf %7.2f done %7.2f us\n", i,
                (double)(long long)(tr[3584 + i * 4] - t0) * 1e-3, (double)(long long)(tr[3584 + i * 4 + 1] - t0) * 1e-3,
                (double)(long long)(tr[3584 + i * 4 + 2] - t0) * 1e-3, (double)(long long)(tr[3584 + i * 4 + 3] - t0) * 1e-3);
      for (int i = 0; i < 64 && tr[i * 4]; i++)
        fprintf(stderr, "  mma %2d: A-sf cp issued %7.2f  sfa ok %7.2f  sfb ok %7.2f  mmas issued %7.2f us\n", i,
                (double)(long long)(tr[2048 + i * 4 + 3] - t0) * 1e-3, (double)(long long)(tr[2048 + i * 4] - t0) * 1e-3,
                (double)(long long)(tr[2048 + i * 4 + 1] - t0) * 1e-3, (double)(long long)(tr[2048 + i * 4 + 2] - t0) * 1e-3);
      for (int i = 0; i < 64 && tr[i * 4]; i++)
        fprintf(stderr, "stage %2d issue %7.2f full %7.2f sf %7.2f mma %7.2f us\n", i, (tr[i * 4] - t0) * 1e-3,
                (tr[i * 4 + 1] - t0) * 1e-3, (tr[i * 4 + 2] - t0) * 1e-3, (tr[i * 4 + 3] - t0) * 1e-3);
      RMOE_CUDA(cudaMemset(L->tc_trace + off, 0, sizeof(tr)), "trace reset");
      return RMOE_OK;
}

// The expert part of a forward once routing and dispatch are on the device: activation operands,
// gate/up, down and the combine into `out`. hs: the shared expert takes part (its positions are
// in the dispatch); terms_done: the front end already wrote the token's activation terms;
// fused_ok: the small-batch front end ran (one-token / fused down+combine paths allowed).
// Batches of more than kI4MinTokens tokens of a grouped-int4 layer run on the tensor cores.
static bool i4_path(const rmoe_layer* L, int T) { return L->use_i4tc && T > kI4MinTokens; }

static rmoe_status enqueue_experts(rmoe_layer* L, const void* x, int xdt, int T, int mt, bool hs, bool terms_done,
                                   bool fused_ok, float* out, cudaStream_t st, StageMarks& marks, int* launches_io) {
  const rmoe_layer_desc& D = L->desc;
  const int H = D.hidden, k = D.topk;
  cudaError_t e = cudaSuccess;
  rmoe_status s = RMOE_OK;
  int& launches = *launches_io;
  const int P = T * k + (hs ? T : 0);
  const int n_slots = L->n_loc + (hs ? 1 : 0);
  if (i4_path(L, T)) {
    // grouped int4 on the tensor cores: x gathered per position (f16), gate/up (-> h per position,
    // routing weight folded in), down (-> y per position), deterministic combine
    e = launch_i4_gather_x(x, xdt, H, L->d.perm_tok, L->d.offsets + n_slots, L->P_max, L->i4_xh, st);
    if (e != cudaSuccess) return cuda_fail(e, "int4 activations");
    marks.mark();
    e = launch_i4_moe(0, L->i4_map_x, L->d, L->d.offsets, H, D.moe_inter, L->i4_tiles, L->i4_stride, L->i4_hh,
                      nullptr, L->fmt.act, L->dev_err, L->spin_ns, st, L->tc_trace);
    if (e != cudaSuccess) return cuda_fail(e, "gate/up (int4 tensor cores)");
    marks.mark();
    marks.mark();  // (h is formed in the gate/up epilogue)
    e = launch_i4_moe(1, L->i4_map_h, L->d, L->d.offsets, H, D.moe_inter, L->i4_tiles + L->i4_off_down, L->i4_stride,
                      nullptr, L->y, L->fmt.act, L->dev_err, L->spin_ns, st);
    if (e != cudaSuccess) return cuda_fail(e, "down (int4 tensor cores)");
    marks.mark();
    e = launch_combine(L->y, L->d, nullptr, T, k, H, L->n_loc, hs ? 1 : 0, out, st);
    if (e != cudaSuccess) return cuda_fail(e, "combine");
    marks.mark();
    launches = 8;  // logits, top-k, prep, dispatch, gather, gate/up, down, combine
    return RMOE_OK;
  }
  if (L->use_tc) {
    // tensor-core experts: activation terms per position, gate/up (-> h terms with the routing
    // weight folded in), down: one token = combined row directly, else y per position + sum
    if (!terms_done && x) {  // (x null: the caller already placed the position rows)
      e = launch_terms_by_position(x, xdt, H, T, k, L->d.inv, hs ? L->d.offsets + L->n_loc : nullptr,
                                   L->xt, L->xsf, st);
      if (e != cudaSuccess) return cuda_fail(e, "activation terms");
    }
    marks.mark();
    if (T == 1 && L->use_fused && (!L->tc_trace || !L->tc_trace_print)) {
      // one token: gate/up and down of all its experts in one launch. The one-token front end
      // zeroes the kernel's counters and puts the shared expert last (its copies may start
      // before the front end is done); other callers zero them here and preload nothing.
      if (!terms_done)
        RMOE_CUDA(cudaMemsetAsync(L->fused_cnt, 0, (8 + L->fused_tiles + RMOE_MAX_TOPK_DEV + 1) * 4, st),
                  "fused counters");
      e = launch_moe_decode_fused(L->tc_plan, L->d, H, D.moe_inter, L->experts, L->tab.stride, L->tc_off_down, L->ht,
                                  L->hsf, L->partial, L->partial2, L->fused_cnt + 8, L->fused_cnt + 8 + L->fused_tiles,
                                  L->fused_cnt, L->dev_err, out, L->fmt.act, terms_done && hs ? L->n_loc : -1, st,
                                  L->tc_trace ? L->tc_trace + 4096 + 2048 : nullptr, L->spin_ns);
      if (e != cudaSuccess) return cuda_fail(e, "fused experts (tensor cores)");
      marks.mark();
      marks.mark();
      marks.mark();
      marks.mark();
      // front, order resolve (side stream), fused experts; or the generic front plus terms
      launches = terms_done ? 3 : (fused_ok ? 5 : 8);
      return RMOE_OK;
    }
    // one token: every position reads the token's own term rows (0..3)
    e = launch_moe_tc(0, L->tc_plan, L->d, mt, H, D.moe_inter, L->experts, L->tab.stride, L->tc_off_down, L->ht, L->hsf, nullptr,
                      L->partial, L->tile_cnt, L->tc_work, L->dev_err, st, terms_done ? L->d.perm_tok : nullptr,
                      L->tc_trace, L->fmt.act, L->tile_cnt, L->tc_work + 6, T <= mt, L->spin_ns);
    if (e != cudaSuccess) return cuda_fail(e, "gate/up (tensor cores)");

    marks.mark();
    marks.mark();  // (h is quantized inside the gate/up epilogue)
    if (T == 1) {
      e = launch_moe_tc(2, L->tc_plan, L->d, mt, H, D.moe_inter, L->experts, L->tab.stride, L->tc_off_down, L->ht, L->hsf, out,
                        L->partial2, L->tile_cnt + L->tile_cnt_half, L->tc_work + 4, L->dev_err, st, nullptr,
                        L->tc_trace ? L->tc_trace + 4096 : nullptr, L->fmt.act, nullptr, nullptr, T <= mt, L->spin_ns);
      if (e != cudaSuccess) return cuda_fail(e, "down (tensor cores)");
      if (L->tc_trace && L->tc_trace_print) {
        if ((s = print_tc_trace(L, st, "gate/up", 0)) != RMOE_OK) return s;
        if ((s = print_tc_trace(L, st, "down (one token)", 4096)) != RMOE_OK) return s;
      }
      marks.mark();
      launches = terms_done ? 4 : (fused_ok ? 6 : 9);  // front (+ order resolve), gate/up, down
    } else {
      e = launch_moe_tc(1, L->tc_plan, L->d, mt, H, D.moe_inter, L->experts, L->tab.stride, L->tc_off_down, L->ht, L->hsf, L->y,
                        L->partial2, L->tile_cnt + L->tile_cnt_half, L->tc_work + 4, L->dev_err, st, nullptr,
                        L->tc_trace ? L->tc_trace + 4096 : nullptr, L->fmt.act, nullptr, nullptr, T <= mt, L->spin_ns);
      if (e != cudaSuccess) return cuda_fail(e, "down (tensor cores)");
      if (L->tc_trace && L->tc_trace_print) {
        if ((s = print_tc_trace(L, st, "gate/up", 0)) != RMOE_OK) return s;
        if ((s = print_tc_trace(L, st, "down", 4096)) != RMOE_OK) return s;
      }
      marks.mark();
      e = launch_combine(L->y, L->d, nullptr, T, k, H, L->n_loc, hs ? 1 : 0, out, st);
      if (e != cudaSuccess) return cuda_fail(e, "combine");
      launches = fused_ok ? 7 : 10;
    }
    marks.mark();
    return RMOE_OK;
  }
  RMOE_CUDA(cudaMemsetAsync(L->hmax, 0, static_cast<size_t>(P) * 4, st), "hmax reset");
  const int max_chunks = std::min(T * k, L->n_loc) + (T * k + mt - 1) / mt + (hs ? (T + mt - 1) / mt : 0);
  const int tasks_gu = max_chunks * (std::max(D.moe_inter, D.shared_inter) / 2);
  const int tasks_dn = max_chunks * (H / 4);
  marks.mark();
  if (L->use_pipe)
    e = launch_pipe_gate_up(L->tab, L->fmt, L->d, L->xq, L->xexp, H, mt, L->h, L->hmax, L->h_ld,
                            L->dev_err, st);
  else
    e = launch_gemv_gate_up(L->tab, L->fmt, L->d, L->xq, L->xexp, H, mt, tasks_gu, L->h, L->hmax,
                            L->h_ld, st);
  if (e != cudaSuccess) return cuda_fail(e, "gate/up");
  marks.mark();
  if (L->use_pipe && fused_ok && hs == L->has_shared) {
    // down projection + weighted combine + gated shared expert in one kernel
    marks.mark();  // (h quantization happens inside the down kernel)
    e = launch_pipe_down_combine(L->tab, L->fmt, L->d, L->h, L->hmax, L->ids, T, k, L->e_begin,
                                 H, L->h_ld, out, L->dev_err, st);
    if (e != cudaSuccess) return cuda_fail(e, "down + combine");
    marks.mark();
    launches -= 2;
  } else if (L->use_pipe) {
    marks.mark();  // (h quantization happens inside the down kernel)
    e = launch_pipe_down(L->tab, L->fmt, L->d, L->h, L->hmax, H, mt, L->h_ld, L->y, L->dev_err, st);
    if (e != cudaSuccess) return cuda_fail(e, "down");
    marks.mark();
    e = launch_combine(L->y, L->d, L->rw, T, k, H, L->n_loc, hs ? 1 : 0, out, st);
    if (e != cudaSuccess) return cuda_fail(e, "combine");
    launches -= 1;
  } else {
    e = launch_quant_h(L->h, L->hmax, L->d.offsets + n_slots, P, L->h_ld, L->fmt.fmt, L->hq, L->hexp, st);
    if (e != cudaSuccess) return cuda_fail(e, "h quantize");
    marks.mark();
    e = launch_gemv_down(L->tab, L->fmt, L->d, L->hq, L->hexp, H, mt, tasks_dn, L->h_ld, L->y, st);
    if (e != cudaSuccess) return cuda_fail(e, "down");
    marks.mark();
    e = launch_combine(L->y, L->d, L->rw, T, k, H, L->n_loc, hs ? 1 : 0, out, st);
    if (e != cudaSuccess) return cuda_fail(e, "combine");
  }
  marks.mark();
  return RMOE_OK;
}


// Enqueues one forward on `st` (stream-ordered, capturable): x -> out, routing left in
// *ids_src / *w_src (reference rank order). L->last_launches = kernels it launched.
static rmoe_status enqueue_forward(rmoe_layer* L, const void* x, int x_dtype, int T, float* out,
                                   cudaStream_t st, StageMarks& marks, const int32_t** ids_src,
                                   const float** w_src) {
  const rmoe_layer_desc& D = L->desc;
  const int H = D.hidden, k = D.topk;
  const int xdt = x_dtype == RMOE_BF16 ? kBF16 : kF32;
  const bool gated = L->has_shared && D.shared_gated;
  const int mt = L->use_tc ? std::min(T, 32) : (i4_path(L, T) ? kI4Chunk : chunk_tokens(T));
  rmoe_status s = RMOE_OK;
  cudaError_t e = cudaSuccess;
  int launches = 10;
  bool resolved = false;
  const bool one_front = L->use_tc && T == 1 && small_path(L, T) && H % 4096 == 0 && D.n_experts <= 512;
  bool terms_done = false;
  if (small_path(L, T)) {
    // certified router + one-block front end (top-k, dispatch, activation prep); for one token
    // on the tensor-core path all of it (and the activation terms) is a single launch
    marks.mark();
    if (!one_front) {
      e = launch_router_certified(x, xdt, L->router, L->router_dtype, L->logits, L->logit_err, T, H,
                                  D.n_experts, st);
      if (e != cudaSuccess) return cuda_fail(e, "certified router");
    }
    marks.mark();
    SmallPrologue a{};
    a.T = T; a.E = D.n_experts; a.k = k; a.H = H; a.mt = mt;
    a.e_begin = L->e_begin; a.e_end = L->e_end; a.n_loc = L->n_loc;
    a.has_shared = L->has_shared ? 1 : 0; a.fmt = L->fmt.fmt;
    a.tpc_gu = D.moe_inter / L->rpt_gu; a.tpc_gu_shared = D.shared_inter / L->rpt_gu;
    a.tpc_dn = H / L->rpt_dn;
    a.mid = L->logits; a.err = L->logit_err; a.bias = L->has_bias ? L->router_bias : nullptr;
    a.x = x; a.x_dtype = xdt; a.w = L->router; a.w_dtype = L->router_dtype;
    a.gvec = gated ? L->shared_gate_vec : nullptr;
    a.ids = L->ids; a.rw = L->rw; a.xq = L->xq; a.xexp = L->xexp; a.gate = L->gate;
    a.fallback_count = L->fallbacks;
    a.order_pending_count = L->order_pending;
    a.pending = L->pending;
    a.errflag = L->dev_err;
    if (one_front) {
      DecodeFront f{};
      f.x = x; f.x_dtype = xdt; f.w = L->router; f.w_dtype = L->router_dtype;
      f.bias = a.bias; f.gvec = a.gvec;
      f.H = H; f.E = D.n_experts; f.k = k;
      f.e_begin = L->e_begin; f.e_end = L->e_end; f.n_loc = L->n_loc; f.has_shared = a.has_shared;
      f.mid = L->logits; f.err = L->logit_err; f.gate = L->gate;
      f.xt = L->xt; f.xsf = L->xsf;
      f.ids = L->ids; f.rw = L->rw; f.pending = L->pending;
      f.fallback_count = L->fallbacks; f.order_pending_count = L->order_pending;
      f.counter = L->front_counter;
      f.zero_buf = L->fused_cnt;  // (null unless the tensor-core path allocated it)
      f.zero_n = L->fused_cnt ? 8 + L->fused_tiles + RMOE_MAX_TOPK_DEV + 1 : 0;
      f.d = L->d;
      f.trace = L->tc_trace ? L->tc_trace + 4000 : nullptr;
      if (f.trace) RMOE_CUDA(cudaMemsetAsync(f.trace, 0, 8 * 8, st), "front trace reset");
      e = launch_decode_front(f, st);
      if (e != cudaSuccess) return cuda_fail(e, "one-token front end");
      terms_done = true;
    } else {
      e = launch_prologue_small(a, L->d, st);
      if (e != cudaSuccess) return cuda_fail(e, "small-T prologue");
    }
    marks.mark();  // top-k, certificate, dispatch and activation prep
    marks.mark();  // (prep and dispatch are folded into the prologue)
    // rank order of near-tied winners: resolved on a side stream, joined before returning
    RMOE_CUDA(cudaEventRecord(L->ev_fork, st), "fork");
    RMOE_CUDA(cudaStreamWaitEvent(L->side, L->ev_fork, 0), "fork wait");
    e = launch_resolve_order(a, L->ids_final, L->w_final, L->exact_v, L->resolve_cnt, L->side);
    if (e != cudaSuccess) return cuda_fail(e, "order resolve");
    RMOE_CUDA(cudaEventRecord(L->ev_join, L->side), "join");
    resolved = true;
    launches = 7;
  } else {
    marks.mark();
    s = route_into(L, x, x_dtype, T, st, &marks);
    if (s != RMOE_OK) return s;
    marks.mark();  // end of top-k
    e = launch_prep_tokens(x, xdt, T, H, L->fmt.fmt, gated ? L->shared_gate_vec : nullptr,
                           L->xq, L->xexp, L->gate, st);
    if (e != cudaSuccess) return cuda_fail(e, "prep tokens");
    marks.mark();
    if ((s = dispatch_into(L, T, mt, gated ? L->gate : nullptr, st, L->has_shared)) != RMOE_OK) return s;
  }
  if ((s = enqueue_experts(L, x, xdt, T, mt, L->has_shared, terms_done, small_path(L, T), out, st, marks,
                            &launches)) != RMOE_OK)
    return s;
  // the rank-order resolver joins back before the forward counts as done
  if (resolved) RMOE_CUDA(cudaStreamWaitEvent(st, L->ev_join, 0), "join wait");
  *ids_src = resolved ? L->ids_final : L->ids;
  *w_src = resolved ? L->w_final : L->rw;
  L->last_launches = launches;
  return RMOE_OK;
}

static rmoe_status check_uploaded(const rmoe_layer* L) {
  for (int s = 0; s < L->n_loc; s++)
    if (!L->uploaded[s])
      return fail(RMOE_INVALID_ARG, "rmoe_moe_forward: expert %d was never uploaded", L->e_begin + s);
  if (L->has_shared && !L->has_shared_w) return fail(RMOE_INVALID_ARG, "rmoe_moe_forward: shared expert never uploaded");
  return RMOE_OK;
}

// Direct launches (large T, or graphs disabled).
static rmoe_status forward_direct(rmoe_layer* L, const void* x, int x_dtype, int T, float* out,
                                  int32_t* ids_out, float* w_out, cudaStream_t st) {
  StageMarks marks(L, st);
  const int32_t* ids_src = nullptr;
  const float* w_src = nullptr;
  rmoe_status s = enqueue_forward(L, x, x_dtype, T, out, st, marks, &ids_src, &w_src);
  if (s != RMOE_OK) return s;
  marks.commit();
  const size_t n = static_cast<size_t>(T) * L->desc.topk;
  if (ids_out) RMOE_CUDA(cudaMemcpyAsync(ids_out, ids_src, n * 4, cudaMemcpyDefault, st), "ids out");
  if (w_out) RMOE_CUDA(cudaMemcpyAsync(w_out, w_src, n * 4, cudaMemcpyDefault, st), "weights out");
  L->stats.kernel_launches += L->last_launches;
  L->stats.forward_calls++;
  L->stats.tokens_routed += T;
  return RMOE_OK;
}

// Folds the stage events of a profiled graph launch into the profile (waits for them).
static rmoe_status drain_graph_profile(rmoe_layer* L, GraphEntry& g) {
  if (!g.pending) return RMOE_OK;
  RMOE_CUDA(cudaEventSynchronize(g.ev[RMOE_NUM_STAGES]), "profile event");
  for (int s = 0; s < RMOE_NUM_STAGES; s++) {
    float ms = 0.0f;
    RMOE_CUDA(cudaEventElapsedTime(&ms, g.ev[s], g.ev[s + 1]), "profile elapsed");
    L->prof_ms[s] += ms;
  }
  L->prof_calls++;
  g.pending = false;
  return RMOE_OK;
}

// Captures the forward for (T, dtype, routing out, profiling) once; the caller's x / out /
// routing buffers are bound per launch through memcpy nodes at the graph's ends.
// Kernel argument layout (offset, size) of argument i, from the driver (cuFuncGetParamInfo).
typedef CUresult (*PFN_funcGetParamInfo)(CUfunction, size_t, size_t*, size_t*);
static PFN_funcGetParamInfo param_info_fn() {
  static PFN_funcGetParamInfo fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuFuncGetParamInfo", &p, 12040, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_funcGetParamInfo>(p);
  });
  return fn;
}

// Finds every kernel-argument word of the captured forward equal to the staging input (x_dev)
// or output (out_dev) pointer. True when the forward can run on the caller's buffers directly:
// at least one reader of x and one writer of out were found, and no copy or memset node (whose
// pointers cannot be patched this way) touches either buffer.
static bool find_io_patches(rmoe_layer* L, const std::vector<cudaGraphNode_t>& nodes, std::vector<NodePatch>& out) {
  auto fn = param_info_fn();
  if (!fn) return false;
  const uint64_t xv = reinterpret_cast<uintptr_t>(L->x_dev), ov = reinterpret_cast<uintptr_t>(L->out_dev);
  int nx = 0, no = 0;
  for (cudaGraphNode_t nd : nodes) {
    cudaGraphNodeType type;
    if (cudaGraphNodeGetType(nd, &type) != cudaSuccess) return false;
    if (type == cudaGraphNodeTypeMemcpy) {
      cudaMemcpy3DParms m{};
      if (cudaGraphMemcpyNodeGetParams(nd, &m) != cudaSuccess) return false;
      const uint64_t a = reinterpret_cast<uintptr_t>(m.srcPtr.ptr), b = reinterpret_cast<uintptr_t>(m.dstPtr.ptr);
      if (a == xv || a == ov || b == xv || b == ov) return false;
      continue;
    }
    if (type == cudaGraphNodeTypeMemset) {
      cudaMemsetParams m{};
      if (cudaGraphMemsetNodeGetParams(nd, &m) != cudaSuccess) return false;
      const uint64_t b = reinterpret_cast<uintptr_t>(m.dst);
      if (b == xv || b == ov) return false;
      continue;
    }
    if (type != cudaGraphNodeTypeKernel) continue;
    NodePatch np;
    np.node = nd;
    if (cudaGraphKernelNodeGetParams(nd, &np.params) != cudaSuccess || np.params.extra) return false;
    cudaFunction_t f = nullptr;
    if (cudaGetFuncBySymbol(&f, np.params.func) != cudaSuccess) return false;
    for (size_t i = 0;; i++) {
      size_t off = 0, sz = 0;
      if (fn(reinterpret_cast<CUfunction>(f), i, &off, &sz) != CUDA_SUCCESS) break;
      const uint8_t* src = static_cast<const uint8_t*>(np.params.kernelParams[i]);
      np.args.emplace_back(src, src + sz);
      for (size_t o = 0; o + 8 <= sz; o += 8) {
        uint64_t v;
        memcpy(&v, src + o, 8);
        if (v == xv || v == ov) {
          np.sites.push_back({i, o, v == ov});
          (v == ov ? no : nx)++;
        }
      }
    }
    if (!np.sites.empty()) out.push_back(std::move(np));
  }
  return nx > 0 && no > 0;  // (argument pointer arrays are set at each launch)
}

static rmoe_status capture_graph(rmoe_layer* L, int x_dtype, int T, bool want_rt, GraphEntry& g) {
  const size_t H = L->desc.hidden;
  g.x_bytes = static_cast<size_t>(T) * H * (x_dtype == RMOE_BF16 ? 2 : 4);
  g.out_bytes = static_cast<size_t>(T) * H * 4;
  g.rt_bytes = static_cast<size_t>(T) * L->desc.topk * 4;
  g.profiled = L->profiling;
  StageMarks marks(L, L->cap);
  if (g.profiled) {
    for (cudaEvent_t& e : g.ev) RMOE_CUDA(cudaEventCreate(&e), "graph profile event");
    marks.fixed = g.ev;
  }
  const int32_t* ids_src = nullptr;
  const float* w_src = nullptr;
  RMOE_CUDA(cudaStreamBeginCapture(L->cap, cudaStreamCaptureModeThreadLocal), "begin capture");
  rmoe_status s = enqueue_forward(L, L->x_dev, x_dtype, T, L->out_dev, L->cap, marks, &ids_src, &w_src);
  cudaGraph_t graph = nullptr;
  cudaError_t ce = cudaStreamEndCapture(L->cap, &graph);
  if (s != RMOE_OK) {
    if (graph) cudaGraphDestroy(graph);
    return s;
  }
  if (ce != cudaSuccess) return cuda_fail(ce, "end capture");
  g.ids_src = ids_src;
  g.w_src = w_src;
  g.launches = L->last_launches;
  auto done = [&](cudaError_t e, const char* what) {
    cudaGraphDestroy(graph);
    return cuda_fail(e, what);
  };
  size_t n_roots = 0, n_nodes = 0;
  cudaError_t e = cudaGraphGetRootNodes(graph, nullptr, &n_roots);
  if (e != cudaSuccess) return done(e, "graph roots");
  std::vector<cudaGraphNode_t> roots(n_roots);
  if ((e = cudaGraphGetRootNodes(graph, roots.data(), &n_roots)) != cudaSuccess) return done(e, "graph roots");
  if ((e = cudaGraphGetNodes(graph, nullptr, &n_nodes)) != cudaSuccess) return done(e, "graph nodes");
  std::vector<cudaGraphNode_t> nodes(n_nodes), leaves;
  if ((e = cudaGraphGetNodes(graph, nodes.data(), &n_nodes)) != cudaSuccess) return done(e, "graph nodes");
  for (cudaGraphNode_t nd : nodes) {
    size_t nd_out = 0;
    if ((e = cudaGraphNodeGetDependentNodes(nd, nullptr, &nd_out)) != cudaSuccess) return done(e, "graph deps");
    if (nd_out == 0) leaves.push_back(nd);
  }
  g.direct_io = find_io_patches(L, nodes, g.patches);
  if (!g.direct_io) {
    g.patches.clear();
    if ((e = cudaGraphAddMemcpyNode1D(&g.in_node, graph, nullptr, 0, L->x_dev, L->x_stage, g.x_bytes,
                                      cudaMemcpyDeviceToDevice)) != cudaSuccess)
      return done(e, "graph input node");
    for (cudaGraphNode_t r : roots)
      if ((e = cudaGraphAddDependencies(graph, &g.in_node, &r, 1)) != cudaSuccess) return done(e, "graph input deps");
    if ((e = cudaGraphAddMemcpyNode1D(&g.out_node, graph, leaves.data(), leaves.size(), L->out_stage,
                                      L->out_dev, g.out_bytes, cudaMemcpyDeviceToDevice)) != cudaSuccess)
      return done(e, "graph output node");
  }
  if (want_rt) {
    if ((e = cudaGraphAddMemcpyNode1D(&g.ids_node, graph, leaves.data(), leaves.size(), L->ids_host_stage,
                                      g.ids_src, g.rt_bytes, cudaMemcpyDeviceToDevice)) != cudaSuccess)
      return done(e, "graph ids node");
    if ((e = cudaGraphAddMemcpyNode1D(&g.w_node, graph, leaves.data(), leaves.size(), L->w_host_stage,
                                      g.w_src, g.rt_bytes, cudaMemcpyDeviceToDevice)) != cudaSuccess)
      return done(e, "graph weights node");
  }
  if ((e = cudaGraphInstantiate(&g.exec, graph, 0)) != cudaSuccess) return done(e, "graph instantiate");
  g.graph = graph;
  return RMOE_OK;
}

// One graph launch per call; x/out/ids/w are device pointers of the caller.
static rmoe_status forward_graph(rmoe_layer* L, const void* x, int x_dtype, int T, float* out,
                                 int32_t* ids_out, float* w_out, cudaStream_t st) {
  const bool want_rt = ids_out || w_out;
  const uint64_t key = static_cast<uint64_t>(T) | (static_cast<uint64_t>(x_dtype) << 24) |
                       (static_cast<uint64_t>(want_rt) << 28) |
                       (static_cast<uint64_t>(L->profiling) << 29);
  auto it = L->graphs.find(key);
  if (it == L->graphs.end()) {
    GraphEntry g;
    rmoe_status s = capture_graph(L, x_dtype, T, want_rt, g);
    if (s != RMOE_OK) {
      if (g.exec) cudaGraphExecDestroy(g.exec);
      if (g.graph) cudaGraphDestroy(g.graph);
      for (cudaEvent_t e : g.ev)
        if (e) cudaEventDestroy(e);
      return s;
    }
    it = L->graphs.emplace(key, g).first;
  }
  GraphEntry& g = it->second;
  rmoe_status s = drain_graph_profile(L, g);
  if (s != RMOE_OK) return s;
  // the kernels' vector loads and stores want 16-byte aligned x and out; other buffers go
  // through the staging ones
  const bool staged = g.direct_io && (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16);
  if (staged) {
    RMOE_CUDA(cudaMemcpyAsync(L->x_dev, x, g.x_bytes, cudaMemcpyDeviceToDevice, st), "stage x");
  }
  if (g.direct_io) {
    const uint64_t xv = reinterpret_cast<uintptr_t>(staged ? L->x_dev : x);
    const uint64_t ov = reinterpret_cast<uintptr_t>(staged ? L->out_dev : out);
    for (NodePatch& np : g.patches) {
      // (pointers into this entry's own argument copies: the entry may have been copied)
      np.arg_ptrs.resize(np.args.size());
      for (size_t i = 0; i < np.args.size(); i++) np.arg_ptrs[i] = np.args[i].data();
      np.params.kernelParams = np.arg_ptrs.data();
      for (const NodePatch::Site& st : np.sites) memcpy(np.args[st.arg].data() + st.off, st.out ? &ov : &xv, 8);
      RMOE_CUDA(cudaGraphExecKernelNodeSetParams(g.exec, np.node, &np.params), "bind x / out");
    }
  } else {
    RMOE_CUDA(cudaGraphExecMemcpyNodeSetParams1D(g.exec, g.in_node, L->x_dev, x, g.x_bytes, cudaMemcpyDeviceToDevice),
              "bind x");
    RMOE_CUDA(cudaGraphExecMemcpyNodeSetParams1D(g.exec, g.out_node, out, L->out_dev, g.out_bytes,
                                                 cudaMemcpyDeviceToDevice),
              "bind out");
  }
  if (want_rt) {
    RMOE_CUDA(cudaGraphExecMemcpyNodeSetParams1D(g.exec, g.ids_node, ids_out ? static_cast<void*>(ids_out) : L->ids_host_stage,
                                                 g.ids_src, g.rt_bytes, cudaMemcpyDeviceToDevice),
              "bind ids");
    RMOE_CUDA(cudaGraphExecMemcpyNodeSetParams1D(g.exec, g.w_node, w_out ? static_cast<void*>(w_out) : L->w_host_stage,
                                                 g.w_src, g.rt_bytes, cudaMemcpyDeviceToDevice),
              "bind weights");
  }
  RMOE_CUDA(cudaGraphLaunch(g.exec, st), "graph launch");
  if (staged) RMOE_CUDA(cudaMemcpyAsync(out, L->out_dev, g.out_bytes, cudaMemcpyDeviceToDevice, st), "unstage out");
  g.pending = g.profiled;
  L->stats.kernel_launches += g.launches;
  L->stats.forward_calls++;
  L->stats.tokens_routed += T;
  return RMOE_OK;
}

static bool graph_path(const rmoe_layer* L, int T) { return L->use_graphs && small_path(L, T); }

static rmoe_status forward_into(rmoe_layer* L, const void* x, int x_dtype, int T, float* out,
                                int32_t* ids_out, float* w_out, cudaStream_t st) {
  rmoe_status s = check_uploaded(L);
  if (s != RMOE_OK) return s;
  if (graph_path(L, T)) return forward_graph(L, x, x_dtype, T, out, ids_out, w_out, st);
  // the kernels' vector loads and stores want 16-byte aligned x and out: others are staged
  const bool staged = reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16;
  if (!staged) return forward_direct(L, x, x_dtype, T, out, ids_out, w_out, st);
  const size_t H = L->desc.hidden;
  RMOE_CUDA(cudaMemcpyAsync(L->x_dev, x, static_cast<size_t>(T) * H * (x_dtype == RMOE_BF16 ? 2 : 4),
                            cudaMemcpyDeviceToDevice, st),
            "stage x");
  if ((s = forward_direct(L, L->x_dev, x_dtype, T, L->out_dev, ids_out, w_out, st)) != RMOE_OK) return s;
  RMOE_CUDA(cudaMemcpyAsync(out, L->out_dev, static_cast<size_t>(T) * H * 4, cudaMemcpyDeviceToDevice, st),
            "unstage out");
  return RMOE_OK;
}


extern "C" rmoe_status rmoe_moe_forward(rmoe_layer* L, const void* x, int32_t x_dtype, int32_t T,
                                        float* out, int32_t* ids_out, float* w_out, void* stream) {
  rmoe_status s = check_ready(L, "rmoe_moe_forward", T, x_dtype);
  if (s != RMOE_OK) return s;
  if (L->hr != L->desc.hidden)
    return fail(RMOE_INVALID_ARG, "rmoe_moe_forward: a latent layer (router_hidden != hidden) runs through rmoe_latent_moe");
  if (T == 0) return RMOE_OK;
  if (!x || !out) return fail(RMOE_INVALID_ARG, "rmoe_moe_forward: null x/out");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  return forward_into(L, x, x_dtype, T, out, ids_out, w_out, static_cast<cudaStream_t>(stream));
}

// out[t] = sum_j w[t][j] * expert_{ids[t][j]}(x[t]) (+ the gated shared expert), given routing:
// the expert loop of glm52::moe::moe with its Routing (apply_single_expert, src/glm52/moe.rs:463-513).
// Slots naming an expert that is not resident here (or -1) contribute nothing, so expert-parallel
// ranks run it on the token rows they receive.
// The expert products for the routing already in L->ids / L->rw (T tokens of x, `hs`: with
// the shared expert): activation prep, dispatch, gate/up, down, combine into out.
static rmoe_status experts_for_routing(rmoe_layer* L, const void* x, int xdt, int T, bool hs, float* out,
                                       cudaStream_t st) {
  const rmoe_layer_desc& D = L->desc;
  const bool gated = hs && D.shared_gated;
  const int mt = L->use_tc ? std::min(T, 32) : (i4_path(L, T) ? kI4Chunk : chunk_tokens(T));
  if (!L->use_tc || gated) {  // (the tensor-core path forms its own activation terms)
    cudaError_t e = launch_prep_tokens(x, xdt, T, D.hidden, L->fmt.fmt, gated ? L->shared_gate_vec : nullptr, L->xq,
                                       L->xexp, L->gate, st);
    if (e != cudaSuccess) return cuda_fail(e, "prep tokens");
  }
  rmoe_status s = RMOE_OK;
  bool prepared = false;
  if (T == 1 && L->use_tc && L->use_fused && (!L->tc_trace || !L->tc_trace_print) && D.topk <= 32) {
    // (the one-token expert kernel reads only the chunk table, its zeroed counters and the token's
    // four term rows: one launch prepares all three)
    cudaError_t e = launch_one_token_prep(x, xdt, static_cast<int>(D.hidden), L->ids, L->rw, D.topk, L->e_begin, L->e_end,
                                          L->n_loc, hs ? 1 : 0, gated ? L->gate : nullptr, L->d, L->fused_cnt,
                                          8 + L->fused_tiles + RMOE_MAX_TOPK_DEV + 1, L->xt, L->xsf, st);
    if (e != cudaSuccess) return cuda_fail(e, "one-token prep");
    prepared = true;
  } else if ((s = dispatch_into(L, T, mt, gated ? L->gate : nullptr, st, hs)) != RMOE_OK) {
    return s;
  }
  StageMarks marks(L, st);
  const bool prof = L->profiling;
  L->profiling = false;  // (stage events cover rmoe_moe_forward only)
  int launches = 0;
  s = enqueue_experts(L, x, xdt, T, mt, hs, prepared, false, out, st, marks, &launches);
  L->profiling = prof;
  L->stats.kernel_launches += launches;
  return s;
}

extern "C" rmoe_status rmoe_moe_forward_routed(rmoe_layer* L, const void* x, int32_t x_dtype, int32_t T,
                                               const int32_t* ids, const float* weights, int32_t with_shared,
                                               float* out, void* stream) {
  const char* what = "rmoe_moe_forward_routed";
  if (!L) return fail(RMOE_INVALID_ARG, "%s: null layer", what);
  if (T < 0 || T > L->max_tokens)
    return fail(RMOE_INVALID_ARG, "%s: T = %d outside [0, max_tokens = %d]", what, T, L->max_tokens);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  if (T == 0) return RMOE_OK;
  if (!x || !ids || !weights || !out) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  rmoe_status s = check_uploaded(L);
  if (s != RMOE_OK) return s;
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const rmoe_layer_desc& D = L->desc;
  const int H = D.hidden, k = D.topk;
  const int xdt = x_dtype == RMOE_BF16 ? kBF16 : kF32;
  const bool hs = with_shared && L->has_shared;
  const bool gated = hs && D.shared_gated;
  // 16-byte aligned x and out are used in place; others go through the staging buffers
  float* const out_user = out;
  const bool staged = reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16;
  if (staged) {
    RMOE_CUDA(cudaMemcpyAsync(L->x_dev, x, static_cast<size_t>(T) * H * (x_dtype == RMOE_BF16 ? 2 : 4),
                              cudaMemcpyDeviceToDevice, st),
              "stage x");
    x = L->x_dev;
    out = L->out_dev;
  }
  const size_t n = static_cast<size_t>(T) * k;
  RMOE_CUDA(cudaMemcpyAsync(L->ids, ids, n * 4, cudaMemcpyDefault, st), "routed ids");
  RMOE_CUDA(cudaMemcpyAsync(L->rw, weights, n * 4, cudaMemcpyDefault, st), "routed weights");
  if ((s = experts_for_routing(L, x, xdt, T, hs, out, st)) != RMOE_OK) return s;
  if (staged)
    RMOE_CUDA(cudaMemcpyAsync(out_user, out, static_cast<size_t>(T) * H * 4, cudaMemcpyDeviceToDevice, st),
              "unstage out");
  L->stats.forward_calls++;
  L->stats.tokens_routed += T;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_activation_terms(rmoe_layer* L, const void* x, int32_t x_dtype, int32_t T, uint8_t* terms,
                                             uint8_t* term_scales, void* stream) {
  const char* what = "rmoe_activation_terms";
  if (!L) return fail(RMOE_INVALID_ARG, "%s: null layer", what);
  if (!L->use_tc) return fail(RMOE_NOT_SUPPORTED, "%s: the layer's experts are not on the MXFP4 tensor-core path", what);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  if (T < 0) return fail(RMOE_INVALID_ARG, "%s: T = %d", what, T);
  if (T == 0) return RMOE_OK;
  if (!x || !terms || !term_scales) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  RMOE_CUDA(launch_terms_rows(x, x_dtype == RMOE_BF16 ? kBF16 : kF32, L->desc.hidden, T, terms, term_scales,
                              static_cast<cudaStream_t>(stream)),
            what);
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_moe_forward_routed_terms(rmoe_layer* L, const uint8_t* terms, const uint8_t* term_scales,
                                                     int32_t T, const int32_t* ids, const float* weights, float* out,
                                                     void* stream) {
  const char* what = "rmoe_moe_forward_routed_terms";
  if (!L) return fail(RMOE_INVALID_ARG, "%s: null layer", what);
  if (!L->use_tc) return fail(RMOE_NOT_SUPPORTED, "%s: the layer's experts are not on the MXFP4 tensor-core path", what);
  if (T < 0 || T > L->max_tokens)
    return fail(RMOE_INVALID_ARG, "%s: T = %d outside [0, max_tokens = %d]", what, T, L->max_tokens);
  if (T == 0) return RMOE_OK;
  if (!terms || !term_scales || !ids || !weights || !out) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  if (reinterpret_cast<uintptr_t>(terms) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(RMOE_INVALID_ARG, "%s: terms and out must be 16-byte aligned", what);
  rmoe_status s = check_uploaded(L);
  if (s != RMOE_OK) return s;
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const rmoe_layer_desc& D = L->desc;
  const int k = D.topk, mt = std::min(T, 32);
  const size_t n = static_cast<size_t>(T) * k;
  RMOE_CUDA(cudaMemcpyAsync(L->ids, ids, n * 4, cudaMemcpyDefault, st), "routed ids");
  RMOE_CUDA(cudaMemcpyAsync(L->rw, weights, n * 4, cudaMemcpyDefault, st), "routed weights");
  if ((s = dispatch_into(L, T, mt, nullptr, st, false)) != RMOE_OK) return s;
  cudaError_t e = launch_terms_gather(terms, term_scales, D.hidden, T, k, L->d.inv, L->xt, L->xsf, st);
  if (e != cudaSuccess) return cuda_fail(e, "position rows from terms");
  StageMarks marks(L, st);
  const bool prof = L->profiling;
  L->profiling = false;
  int launches = 0;
  s = enqueue_experts(L, nullptr, kF32, T, mt, false, false, false, out, st, marks, &launches);
  L->profiling = prof;
  L->stats.kernel_launches += launches + 2;
  L->stats.forward_calls++;
  L->stats.tokens_routed += T;
  return s;
}

extern "C" rmoe_status rmoe_upload_latent(rmoe_layer* L, const void* down_proj, const void* up_proj, int32_t proj_dtype,
                                          const float* norm, float eps) {
  const char* what = "rmoe_upload_latent";
  if (!L || !down_proj || !up_proj) return fail(RMOE_INVALID_ARG, "%s: null argument", what);
  if (L->hr == L->desc.hidden) return fail(RMOE_INVALID_ARG, "%s: not a latent layer (router_hidden == hidden)", what);
  if (proj_dtype != RMOE_F32 && proj_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: dtype %d", what, proj_dtype);
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  const size_t bytes = static_cast<size_t>(L->desc.hidden) * L->hr * (proj_dtype == RMOE_BF16 ? 2 : 4);
  RMOE_CUDA(cudaMemcpy(L->lat_down, down_proj, bytes, cudaMemcpyDefault), "latent down_proj");
  RMOE_CUDA(cudaMemcpy(L->lat_up, up_proj, bytes, cudaMemcpyDefault), "latent up_proj");
  L->lat_dtype = proj_dtype == RMOE_BF16 ? kBF16 : kF32;
  L->lat_has_norm = norm != nullptr;
  if (norm) RMOE_CUDA(cudaMemcpy(L->lat_norm, norm, static_cast<size_t>(L->desc.hidden) * 4, cudaMemcpyDefault), "latent norm");
  L->lat_eps = eps;
  L->has_latent = true;
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_latent_moe(rmoe_layer* L, const void* x, int32_t x_dtype, int32_t T, float* out,
                                       int32_t* ids_out, float* w_out, void* stream) {
  const char* what = "rmoe_latent_moe";
  rmoe_status s = check_ready(L, what, T, x_dtype);
  if (s != RMOE_OK) return s;
  if (!L->has_latent) return fail(RMOE_INVALID_ARG, "%s: latent projections were never uploaded", what);
  if (T == 0) return RMOE_OK;
  if (!x || !out) return fail(RMOE_INVALID_ARG, "%s: null x/out", what);
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(RMOE_INVALID_ARG, "%s: x and out must be 16-byte aligned", what);
  if ((s = check_uploaded(L)) != RMOE_OK) return s;
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = L->desc.hidden, Hr = L->hr, k = L->desc.topk;
  const int xdt = x_dtype == RMOE_BF16 ? kBF16 : kF32;
  // x_latent = x . down^T (:91-92) on the side stream, beside the routing: the projection streams
  // its weights from HBM while the router's exact chains are latency-bound
  RMOE_CUDA(cudaEventRecord(L->ev_fork, st), "fork");
  RMOE_CUDA(cudaStreamWaitEvent(L->side, L->ev_fork, 0), "fork wait");
  cudaError_t e = launch_latent_proj(L->lat_down, L->lat_dtype, x, xdt, T, Hr, H, L->lat_x, L->side);
  if (e != cudaSuccess) return cuda_fail(e, "latent down projection");
  RMOE_CUDA(cudaEventRecord(L->ev_join, L->side), "join");
  // routing at the full width, on x itself (src/kimi_k3/moe.rs:84-86)
  if ((s = route_into(L, x, x_dtype, T, st)) != RMOE_OK) return s;
  RMOE_CUDA(cudaStreamWaitEvent(st, L->ev_join, 0), "join wait");
  // the routed experts at the latent width (:94-104); no shared expert here (the caller's)
  if ((s = experts_for_routing(L, L->lat_x, kF32, T, false, L->lat_y, st)) != RMOE_OK) return s;
  // RMSNorm of each token's summed routed row (:106-110), then out = y . up^T (:112)
  // (the norm folds into the up projection's staging of the rows when they fit in one group)
  const bool fold = L->lat_has_norm && latent_proj_one_group(T, H);
  if (L->lat_has_norm && !fold && (e = launch_rmsnorm_rows(L->lat_y, T, H, L->lat_norm, L->lat_eps, st)) != cudaSuccess)
    return cuda_fail(e, "latent norm");
  if ((e = launch_latent_proj(L->lat_up, L->lat_dtype, L->lat_y, kF32, T, H, Hr, out, st, fold ? L->lat_norm : nullptr,
                              L->lat_eps)) != cudaSuccess)
    return cuda_fail(e, "latent up projection");
  const size_t n = static_cast<size_t>(T) * k;
  if (ids_out) RMOE_CUDA(cudaMemcpyAsync(ids_out, L->ids, n * 4, cudaMemcpyDeviceToDevice, st), "latent ids");
  if (w_out) RMOE_CUDA(cudaMemcpyAsync(w_out, L->rw, n * 4, cudaMemcpyDeviceToDevice, st), "latent weights");
  L->stats.forward_calls++;
  L->stats.tokens_routed += T;
  return RMOE_OK;
}

// RMOE_DIAG_HOST=1: after a failed call, the fused one-token kernel's per-CTA
// timeline (read from mapped host memory, so also after a fault) to stderr.
static void diag_dump(const rmoe_layer* L) {
  if (!L->diag_buf) return;
  const volatile unsigned long long* tr = static_cast<const volatile unsigned long long*>(L->diag_buf);
  const unsigned long long f0 = tr[4000];
  fprintf(stderr, "diag: front end start %llu\n", f0);
  const char* nm[8] = {"entry", "set-up", "first copy", "first down", "epilogue done", "barrier", "exit", "mma drained"};
  for (int c = 0; c < 148; c++) {
    fprintf(stderr, "diag cta %3d:", c);
    for (int f = 0; f < 8; f++) {
      const unsigned long long v = tr[4096 + 2048 + 8 * c + f];
      fprintf(stderr, " %s=%.2f", nm[f], v && f0 ? (double)(long long)(v - f0) * 1e-3 : -1.0);
    }
    fprintf(stderr, "\n");
  }
}

extern "C" rmoe_status rmoe_moe_forward_host(rmoe_layer* L, const void* x_host, int32_t x_dtype,
                                             int32_t T, float* out_host, int32_t* ids_host,
                                             float* w_host) {
  rmoe_status s = check_ready(L, "rmoe_moe_forward_host", T, x_dtype);
  if (s != RMOE_OK) return s;
  if (L->hr != L->desc.hidden)
    return fail(RMOE_INVALID_ARG, "rmoe_moe_forward_host: a latent layer runs through rmoe_latent_moe");
  if (T == 0) return RMOE_OK;
  if (!x_host || !out_host) return fail(RMOE_INVALID_ARG, "rmoe_moe_forward_host: null x/out");
  RMOE_CUDA(cudaSetDevice(L->ctx->device), "cudaSetDevice");
  const size_t H = L->desc.hidden;
  const size_t xb = static_cast<size_t>(T) * H * (x_dtype == RMOE_BF16 ? 2 : 4);
  RMOE_CUDA(cudaMemcpyAsync(L->x_stage, x_host, xb, cudaMemcpyHostToDevice, L->stream), "x to device");
  const size_t n = static_cast<size_t>(T) * L->desc.topk;
  const bool rt = ids_host || w_host;
  if ((s = forward_into(L, L->x_stage, x_dtype, T, L->out_stage, rt ? L->ids_host_stage : nullptr,
                        rt ? L->w_host_stage : nullptr, L->stream)) != RMOE_OK)
    return s;
  RMOE_CUDA(cudaMemcpyAsync(out_host, L->out_stage, static_cast<size_t>(T) * H * 4, cudaMemcpyDeviceToHost, L->stream),
            "out to host");
  if (ids_host) RMOE_CUDA(cudaMemcpyAsync(ids_host, L->ids_host_stage, n * 4, cudaMemcpyDeviceToHost, L->stream), "ids to host");
  if (w_host) RMOE_CUDA(cudaMemcpyAsync(w_host, L->w_host_stage, n * 4, cudaMemcpyDeviceToHost, L->stream), "weights to host");
  // the error flags ride behind the outputs (no second round trip after the synchronize)
  if (L->err_host) RMOE_CUDA(cudaMemcpyAsync(L->err_host, L->dev_err, 4, cudaMemcpyDeviceToHost, L->stream), "error flags to host");
  {
    cudaError_t e = cudaStreamSynchronize(L->stream);
    if (e != cudaSuccess) {
      diag_dump(L);
      return cuda_fail(e, "rmoe_moe_forward_host synchronize");
    }
  }
  return take_device_errors(L, "rmoe_moe_forward_host", L->err_host);
}

// ------------------------------------------------------------------------------ matmuls
static rmoe_status matmul_q(const char* what, float* y, const void* x, int32_t x_dtype,
                            const uint8_t* data, const void* scale, const ExpertFormat& f, int32_t s,
                            int32_t i, int32_t o, void* stream) {
  if (!y || !x || !data || !scale) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  if (s < 0 || i <= 0 || o < 0) return fail(RMOE_INVALID_ARG, "%s: s=%d i=%d o=%d", what, s, i, o);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t ws = matmul_q_workspace_bytes(s, i);
  void* buf = nullptr;
  RMOE_CUDA(cudaMallocAsync(&buf, ws, st), "matmul workspace");
  cudaError_t e = launch_matmul_q(y, x, x_dtype == RMOE_BF16 ? kBF16 : kF32, data, scale, f, s, i, o, buf, ws, st);
  cudaError_t e2 = cudaFreeAsync(buf, st);
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (e2 != cudaSuccess) return cuda_fail(e2, what);
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_matmul_mxfp4(float* y, const void* x, int32_t x_dtype,
                                         const uint8_t* data, const uint8_t* block_scale, int32_t s,
                                         int32_t i, int32_t o, void* stream) {
  return matmul_q("rmoe_matmul_mxfp4", y, x, x_dtype, data, block_scale, ExpertFormat{kMxfp4, 32, kF32},
                  s, i, o, stream);
}

extern "C" rmoe_status rmoe_matmul_mxfp4_tc(float* y, const void* x, int32_t x_dtype,
                                            const uint8_t* data, const uint8_t* block_scale, int32_t s,
                                            int32_t i, int32_t o, void* stream) {
  const char* what = "rmoe_matmul_mxfp4_tc";
  if (!y || !x || !data || !block_scale) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  if (s < 0 || i <= 0 || o < 0) return fail(RMOE_INVALID_ARG, "%s: s=%d i=%d o=%d", what, s, i, o);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  if (s == 0 || o == 0) return RMOE_OK;
  if (!mxf4_tc_supported(s, i, o)) return fail(RMOE_NOT_SUPPORTED, "%s: i=%d (needs a multiple of 32)", what, i);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t ws = mxf4_tc_workspace_bytes(s, i) + 16;
  void* buf = nullptr;
  RMOE_CUDA(cudaMallocAsync(&buf, ws, st), "tc matmul workspace");
  unsigned* err = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(buf) + ws - 16);
  cudaError_t e = cudaMemsetAsync(err, 0, 4, st);
  if (e == cudaSuccess)
    e = launch_mxf4_tc_matmul(y, x, x_dtype == RMOE_BF16 ? kBF16 : kF32, data, block_scale, s, i, o, buf,
                              ws - 16, err, st);
  cudaError_t e2 = cudaFreeAsync(buf, st);
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (e2 != cudaSuccess) return cuda_fail(e2, what);
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_matmul_i4_grouped(float* y, const void* x, int32_t x_dtype,
                                              const uint8_t* q4, const void* scale,
                                              int32_t scale_dtype, int32_t group_size, int32_t s,
                                              int32_t i, int32_t o, void* stream) {
  if (group_size <= 0) return fail(RMOE_INVALID_ARG, "rmoe_matmul_i4_grouped: group_size %d", group_size);
  if (scale_dtype != RMOE_F32 && scale_dtype != RMOE_BF16)
    return fail(RMOE_INVALID_ARG, "rmoe_matmul_i4_grouped: scale_dtype %d", scale_dtype);
  return matmul_q("rmoe_matmul_i4_grouped", y, x, x_dtype, q4, scale,
                  ExpertFormat{kInt4g, group_size, scale_dtype == RMOE_BF16 ? kBF16 : kF32}, s, i, o, stream);
}

extern "C" rmoe_status rmoe_matmul_f32(float* y, const void* x, int32_t x_dtype, const void* w,
                                       int32_t w_dtype, int32_t s, int32_t i, int32_t o, void* stream) {
  if (!y || !x || !w) return fail(RMOE_INVALID_ARG, "rmoe_matmul_f32: null pointer");
  if (s < 0 || i <= 0 || o < 0) return fail(RMOE_INVALID_ARG, "rmoe_matmul_f32: s=%d i=%d o=%d", s, i, o);
  cudaError_t e = launch_router_logits_exact(x, x_dtype == RMOE_BF16 ? kBF16 : kF32, w,
                                             w_dtype == RMOE_BF16 ? kBF16 : kF32, y, s, i, o,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmoe_matmul_f32");
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_matmul_qt(float* y, const void* x, int32_t x_dtype, int32_t kind, const void* data,
                                      const void* scale, int32_t group_size, int32_t s, int32_t i, int32_t o,
                                      void* stream) {
  const char* what = "rmoe_matmul_qt";
  if (!y || !x || !data || (kind != RMOE_QT_F32 && !scale)) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  if (s < 0 || i <= 0 || o < 0) return fail(RMOE_INVALID_ARG, "%s: s=%d i=%d o=%d", what, s, i, o);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int xdt = x_dtype == RMOE_BF16 ? kBF16 : kF32;
  switch (kind) {
    case RMOE_QT_F32:
      return rmoe_matmul_f32(y, x, x_dtype, data, RMOE_F32, s, i, o, stream);
    case RMOE_QT_MXFP4:
      return matmul_q(what, y, x, x_dtype, static_cast<const uint8_t*>(data), scale, ExpertFormat{kMxfp4, 32, kF32}, s, i,
                      o, stream);
    case RMOE_QT_I4_GROUPED:
      if (group_size <= 0) return fail(RMOE_INVALID_ARG, "%s: group_size %d", what, group_size);
      return matmul_q(what, y, x, x_dtype, static_cast<const uint8_t*>(data), scale,
                      ExpertFormat{kInt4g, group_size, kF32}, s, i, o, stream);
    case RMOE_QT_I2:
    case RMOE_QT_I4:
      // int4 at s >= 2 and int8 always take the integer-dot path, like the reference dispatcher
      if (kind == RMOE_QT_I2 || s < 2) {
        cudaError_t e = launch_matmul_qt_float(y, x, xdt, static_cast<const uint8_t*>(data), kind == RMOE_QT_I2 ? 2 : 4,
                                               static_cast<const float*>(scale), s, i, o, st);
        if (e != cudaSuccess) return cuda_fail(e, what);
        return RMOE_OK;
      }
      [[fallthrough]];
    case RMOE_QT_I8: {
      if (s == 0 || o == 0) return RMOE_OK;
      const size_t ws = matmul_idot_workspace_bytes(s, i);
      void* buf = nullptr;
      RMOE_CUDA(cudaMallocAsync(&buf, ws, st), "matmul_qt workspace");
      cudaError_t e = launch_matmul_idot(y, x, xdt, data, kind == RMOE_QT_I4, static_cast<const float*>(scale), s, i, o,
                                         buf, st);
      cudaError_t e2 = cudaFreeAsync(buf, st);
      if (e != cudaSuccess) return cuda_fail(e, what);
      if (e2 != cudaSuccess) return cuda_fail(e2, what);
      return RMOE_OK;
    }
    default:
      return fail(RMOE_INVALID_ARG, "%s: kind %d", what, kind);
  }
}

extern "C" rmoe_status rmoe_synth_bytes(void* dst, size_t n, uint64_t key, int32_t mode, int32_t lo,
                                        int32_t hi, void* stream) {
  if (!dst && n) return fail(RMOE_INVALID_ARG, "rmoe_synth_bytes: null dst");
  if (mode != 0 && mode != 1) return fail(RMOE_INVALID_ARG, "rmoe_synth_bytes: mode %d", mode);
  cudaError_t e = launch_synth_bytes(dst, n, key, mode, lo, hi, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmoe_synth_bytes");
  return RMOE_OK;
}

extern "C" rmoe_status rmoe_sum_rank_parts(float* out, const float* parts, int32_t n_parts, int64_t rows,
                                           int32_t hidden, const float* last, void* stream) {
  const char* what = "rmoe_sum_rank_parts";
  if (n_parts <= 0 || rows < 0 || hidden <= 0) return fail(RMOE_INVALID_ARG, "%s: n_parts=%d rows=%lld hidden=%d", what, n_parts, static_cast<long long>(rows), hidden);
  if (rows == 0) return RMOE_OK;
  if (!out || !parts) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  if (hidden % 4 || reinterpret_cast<uintptr_t>(out) % 16 || reinterpret_cast<uintptr_t>(parts) % 16 ||
      reinterpret_cast<uintptr_t>(last) % 16)
    return fail(RMOE_INVALID_ARG, "%s: hidden %% 4 and 16-byte aligned buffers required", what);
  cudaError_t e = launch_sum_rank_parts(parts, n_parts, static_cast<size_t>(rows) * hidden, last, out,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, what);
  return RMOE_OK;
}

// ------------------------------------------------------------------- no-allocation matmul
// rmoe_matmul_mxfp4 takes its activation scratch (f16 rows + per-row exponents) from
// cudaMallocAsync on every call. Some callers cannot allocate at that point: a serving loop
// that has reserved the device's free memory for its own page arena (so a pool allocation can
// fail with out-of-memory, or make the driver trim/grow the pool mid-decode), or a caller whose
// allocator policy forbids device allocations on the hot path. This variant takes the same
// scratch from a fixed file-scope device array instead, so it never allocates or frees.
//
// The scratch holds s*i f16 values + s int32 exponents (+256 bytes of alignment slack):
// matmul_q_workspace_bytes(s, i) <= RMOE_NOALLOC_SCRATCH_BYTES (8 MiB + 4 KiB): s*i <= 4M
// elements for s <= 512, e.g. 512 rows at i = 8192. The prep kernel writes every scratch byte the GEMV reads before
// the GEMV runs, so nothing has to start at zero. Calls that overlap in time on one device
// (two streams, or two host threads, with no ordering between them) share the array and race;
// order them on one stream.
static __device__ __align__(256) unsigned char g_noalloc_scratch[RMOE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};
}  // namespace

extern "C" rmoe_status rmoe_matmul_mxfp4_noalloc(float* y, const void* x, int32_t x_dtype,
                                                 const uint8_t* data, const uint8_t* block_scale,
                                                 int32_t s, int32_t i, int32_t o, void* stream) {
  const char* what = "rmoe_matmul_mxfp4_noalloc";
  if (!y || !x || !data || !block_scale) return fail(RMOE_INVALID_ARG, "%s: null pointer", what);
  if (s < 0 || i <= 0 || o < 0) return fail(RMOE_INVALID_ARG, "%s: s=%d i=%d o=%d", what, s, i, o);
  if (x_dtype != RMOE_F32 && x_dtype != RMOE_BF16) return fail(RMOE_INVALID_ARG, "%s: x_dtype %d", what, x_dtype);
  // only the vectorised path (i a multiple of 32) uses the scratch; others need none
  const size_t ws = i % 32 == 0 ? matmul_q_workspace_bytes(s, i) : 0;
  if (ws > RMOE_NOALLOC_SCRATCH_BYTES)
    return fail(RMOE_INVALID_ARG, "%s: s=%d i=%d needs %zu scratch bytes, above the fixed %zu (split the rows)",
                what, s, i, ws, static_cast<size_t>(RMOE_NOALLOC_SCRATCH_BYTES));
  int dev = -1;
  RMOE_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(RMOE_INVALID_ARG, "%s: device %d", what, dev);
  void* scratch = nullptr;
  {
    // First call on a device (that device current): resolve the array's address once. The
    // cached address belongs to the device's primary context: after cudaDeviceReset (or any
    // teardown of that context) it is stale, so this entry point must not be used afterwards.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      RMOE_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)");
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  cudaError_t e = launch_matmul_q(y, x, x_dtype == RMOE_BF16 ? kBF16 : kF32, data, block_scale,
                                  ExpertFormat{kMxfp4, 32, kF32}, s, i, o, ws ? scratch : nullptr, ws,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, what);
  return RMOE_OK;
}
