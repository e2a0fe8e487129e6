/*
 * rmoe.h -- C ABI of the B200-native routed-MoE layer (the drop-in boundary).
 *
 * Plain pointers and sizes only; no CUDA or torch types. `stream` arguments are a
 * cudaStream_t passed as void* (NULL = the legacy default stream). Device-pointer entry points
 * are asynchronous and stream-ordered; the *_host entry points synchronize before returning.
 * Every function returns rmoe_status; on failure rmoe_last_error() (thread-local) says why.
 * Nothing aborts or throws across this boundary.
 *
 * Each entry point names the reference interface it replaces (ferrumox/rabbit v0.29.1, paths
 * relative to that crate).
 */
#ifndef RMOE_H
#define RMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define RMOE_API __attribute__((visibility("default")))
#else
#define RMOE_API
#endif

#define RMOE_ABI_VERSION 4
#define RMOE_MAX_TOPK 32

typedef enum rmoe_status {
  RMOE_OK = 0,
  RMOE_INVALID_ARG = 1,     /* null pointer, out-of-range id, bad enum */
  RMOE_SHAPE_MISMATCH = 2,  /* byte counts that do not match the declared shape */
  RMOE_CUDA_ERROR = 3,
  RMOE_NCCL_ERROR = 4,
  RMOE_TIMEOUT = 5,         /* a bounded device-side wait gave up */
  RMOE_NOT_SUPPORTED = 6,   /* a shape the kernels do not handle (see rmoe_layer_create) */
  RMOE_OUT_OF_MEMORY = 7,
  RMOE_IO_ERROR = 8,        /* a checkpoint file could not be read, or its header is malformed */
  RMOE_MISSING_TENSOR = 9   /* a checkpoint has no tensor of the requested name */
} rmoe_status;

typedef enum rmoe_router_kind {
  /* qwen38::moe::route: top-k of the logits, softmax over the k winners (weights sum to 1) */
  RMOE_ROUTER_SOFTMAX_TOPK = 0,
  /* glm52::moe::route: sigmoid scores + correction bias, grouped top-k, norm_topk, scale */
  RMOE_ROUTER_SIGMOID_GROUPED = 1
} rmoe_router_kind;

typedef enum rmoe_weight_format {
  RMOE_FMT_MXFP4 = 0,      /* QTKind::MxFp4: E2M1 nibbles low-first + E8M0 byte per 32 */
  RMOE_FMT_I4_GROUPED = 1  /* QTKind::I4Grouped: offset-binary nibbles + scale per group */
} rmoe_weight_format;

typedef enum rmoe_dtype { RMOE_F32 = 0, RMOE_BF16 = 1 } rmoe_dtype;

/* The expert gating activation (glm52::moe::Activation, src/glm52/moe.rs:49-70). */
typedef enum rmoe_activation {
  RMOE_ACT_SILU = 0,  /* silu(g) * u */
  /* Kimi K3 SituAndMul: beta tanh(g / beta) sigmoid(g) * u', u' = lb tanh(u / lb) when a linear
   * beta lb is set (situ_linear_beta > 0), else u */
  RMOE_ACT_SITU = 1
} rmoe_activation;

typedef struct rmoe_ctx rmoe_ctx;
typedef struct rmoe_layer rmoe_layer;
typedef struct rmoe_shards rmoe_shards;

/* The on-disk tensor names of a routed expert (ExpertNaming, src/expert_cache.rs:66-131). */
typedef enum rmoe_expert_naming {
  /* model.layers.{L}.mlp.experts.{E}.{gate,up,down}_proj.weight (+ .qs int4 scales) */
  RMOE_NAMING_GLM52 = 0,
  /* model.layers.{L}.mlp.experts.{E}.{gate_up,down}_proj.weight, gate_up = [2I, H] */
  RMOE_NAMING_GLM52_FUSED_GATE_UP = 1,
  /* model.layers.{L}.block_sparse_moe.experts.{E}.{w1,w3,w2}.weight (w1 gate, w3 up, w2 down) */
  RMOE_NAMING_KIMI_LINEAR = 2,
  /* the same under language_model. */
  RMOE_NAMING_KIMI_K3 = 3,
  /* K3's MXFP4 checkpoint: {base}.weight_packed + {base}.weight_scale per matrix */
  RMOE_NAMING_KIMI_K3_MXFP4 = 4,
  /* Qwen3.8's MXFP4 checkpoint: model.layers.{L}.mlp.experts.{E}.{gate,up,down}_proj.weight +
   * .weight_scale */
  RMOE_NAMING_QWEN38_MXFP4 = 5
} rmoe_expert_naming;

/* Whose MoeWeights tensor names rmoe_load_moe_weights reads (router, bias, shared expert). */
typedef enum rmoe_model_family {
  RMOE_FAMILY_QWEN38 = 0,  /* qwen38::model (src/qwen38/model.rs:319-326) */
  RMOE_FAMILY_GLM52 = 1    /* glm52::model (src/glm52/model.rs:249-253) */
} rmoe_model_family;

#define RMOE_DTYPE_NAME_BYTES 16
#define RMOE_MAX_TENSOR_DIMS 8

/* Mirrors the routing/expert fields of qwen38::config::Cfg (src/qwen38/config.rs:71-102) and
 * glm52::config::Cfg (src/glm52/config.rs:26-46). */
typedef struct rmoe_layer_desc {
  int32_t hidden;         /* H: cfg.hidden (multiple of 32) */
  int32_t moe_inter;      /* I: cfg.moe_inter (multiple of 32) */
  int32_t shared_inter;   /* shared expert width (Qwen shared_inter, GLM moe_inter*n_shared); 0 = none */
  int32_t n_experts;      /* E: routed experts in the whole model (all EP ranks) */
  int32_t topk;           /* k: cfg.topk (<= RMOE_MAX_TOPK, <= n_experts) */
  int32_t router_kind;    /* rmoe_router_kind */
  int32_t n_group;        /* GLM n_group (<= 1 = ungrouped); must divide n_experts */
  int32_t topk_group;     /* GLM topk_group */
  int32_t norm_topk;      /* GLM norm_topk_prob (Qwen always renormalizes) */
  float routed_scale;     /* GLM routed_scaling_factor (Qwen: 1) */
  int32_t weight_format;  /* rmoe_weight_format, for routed and shared experts alike */
  int32_t group_size;     /* I4_GROUPED: elements per scale (multiple of 32); MXFP4: 32 */
  int32_t scale_dtype;    /* I4_GROUPED scale storage: RMOE_F32 (reference .qs) or RMOE_BF16 */
  int32_t shared_gated;   /* Qwen: shared expert scaled by sigmoid(x . shared_gate) */
  int32_t max_tokens;     /* largest T any call will pass (sizes the workspace) */
  int32_t ep_rank;        /* expert parallel rank (0 when unsharded) */
  int32_t ep_size;        /* expert parallel world size (1 when unsharded) */
  int32_t activation;     /* rmoe_activation (0 = SiLU) */
  float situ_beta;        /* RMOE_ACT_SITU: beta (> 0) */
  float situ_linear_beta; /* RMOE_ACT_SITU: linear beta; <= 0 = none */
  /* Kimi K3 latent MoE (kimi_k3::moe::latent_moe, src/kimi_k3/moe.rs:64-116): the router and
   * the caller's x are router_hidden wide while the experts work at `hidden` (the latent width);
   * 0 = the same as hidden. A layer with router_hidden != hidden runs through rmoe_latent_moe. */
  int32_t router_hidden;
} rmoe_layer_desc;

typedef struct rmoe_layer_stats {
  uint64_t forward_calls;
  uint64_t tokens_routed;
  uint64_t kernel_launches;      /* this library's kernels launched by forward calls */
  uint64_t router_fallbacks;     /* tokens whose fast-router expert set was uncertain and
                                    were re-ranked on exact reference-order logits */
  uint64_t router_order_resolved; /* tokens whose set was certain but whose rank order was
                                    settled on exact logits beside the expert products */
  uint64_t device_error_flags;   /* nonzero: a bounded device-side wait gave up (bit 0 producer,
                                    bit 1 consumer); the results of that call are invalid */
  uint64_t device_bytes;         /* resident expert + router bytes */
  int32_t local_expert_begin;    /* experts [begin, end) are resident on this device */
  int32_t local_expert_end;
} rmoe_layer_stats;

/* Stages of one forward call, in launch order (rmoe_layer_get_profile). */
typedef enum rmoe_stage {
  RMOE_STAGE_ROUTER_LOGITS = 0,
  RMOE_STAGE_TOPK = 1,
  RMOE_STAGE_PREP = 2,
  RMOE_STAGE_DISPATCH = 3,
  RMOE_STAGE_GATE_UP = 4,
  RMOE_STAGE_QUANT_H = 5,
  RMOE_STAGE_DOWN = 6,
  RMOE_STAGE_COMBINE = 7,
  RMOE_NUM_STAGES = 8
} rmoe_stage;

typedef struct rmoe_profile {
  uint64_t calls;                       /* forward calls profiled since the last read */
  double stage_ms[RMOE_NUM_STAGES];     /* summed device time per stage (CUDA events) */
} rmoe_profile;

RMOE_API const char* rmoe_last_error(void);
RMOE_API const char* rmoe_status_string(rmoe_status s);
RMOE_API int rmoe_abi_version(void);

/* ---- context / layer lifetime (replaces ExpertCache construction, src/expert_cache.rs:698-760:
 *      all experts become HBM-resident instead of an LRU of streamed ones) ---- */
RMOE_API rmoe_status rmoe_init(int device, rmoe_ctx** out);
RMOE_API rmoe_status rmoe_shutdown(rmoe_ctx* ctx);
RMOE_API rmoe_status rmoe_layer_create(rmoe_ctx* ctx, const rmoe_layer_desc* desc, rmoe_layer** out);
RMOE_API rmoe_status rmoe_layer_destroy(rmoe_layer* layer);
RMOE_API rmoe_status rmoe_layer_get_stats(const rmoe_layer* layer, rmoe_layer_stats* out);
/* The descriptor the layer was created with (no counterpart in the reference, whose Cfg the caller
 * already holds). */
RMOE_API rmoe_status rmoe_layer_get_desc(const rmoe_layer* layer, rmoe_layer_desc* out);
/* Per-stage CUDA-event timing of forward calls (no counterpart in the reference, whose
 * Phases/StepProfile timers in src/generate.rs:192-203 play this role on the CPU). While on,
 * every forward records one event per stage boundary on its stream. get_profile waits for
 * those events, returns the sums since the last read and resets them. */
RMOE_API rmoe_status rmoe_layer_set_profiling(rmoe_layer* layer, int on);
RMOE_API rmoe_status rmoe_layer_get_profile(rmoe_layer* layer, rmoe_profile* out);

/* Error status of the work already queued on a layer (the counterpart of the reference's
 * Result<_, ModelError> on every MoE call, src/glm52/moe.rs:350-362, for the asynchronous
 * device-pointer entry points). Synchronizes `stream` and the layer's own streams; returns
 * RMOE_TIMEOUT when a bounded device-side wait of the layer's kernels ran out since the last
 * check (the outputs of those calls are invalid; the layer resets its work counters and is usable
 * again), else RMOE_OK. rmoe_moe_forward_host performs this check itself before returning. */
RMOE_API rmoe_status rmoe_layer_check(rmoe_layer* layer, void* stream);
/* No counterpart in the reference. Limit, in nanoseconds, of each wait of the layer's persistent
 * kernels on another CTA's progress (grid barriers, readiness of h); 0 = the default, 2 s. The
 * kernels assume all their CTAs are resident together (one per SM); if other work holds SMs
 * those waits can run out, and the call then reports RMOE_TIMEOUT instead of hanging. */
RMOE_API rmoe_status rmoe_layer_set_wait_limit(rmoe_layer* layer, uint64_t ns);

/* Opt-in CACHE_ROUTE routing for the sigmoid router (RouteConfig + route_cache_aware,
 * src/glm52/moe.rs:99-127, :272-323), off by default: the top route_j experts by choice are always
 * taken; the remaining k - route_j slots prefer experts marked resident among the next ranked up to
 * max(route_m, k), in rank order, then fall back to rank order. Like the reference it ranks over
 * all experts (no grouping). resident: [n_experts] bytes, nonzero = resident (host or device),
 * or NULL = every expert resident (then the selection equals plain top-k). cache_route = 0 restores
 * the plain router. RMOE_NOT_SUPPORTED on a softmax-router layer (the reference has no
 * CACHE_ROUTE there). */
RMOE_API rmoe_status rmoe_set_route_config(rmoe_layer* layer, int32_t cache_route, int32_t route_j, int32_t route_m,
                                           const uint8_t* resident);

/* ---- weights, taken in the reference's byte layout verbatim. Pointers may be host or device
 *      memory (unified addressing). Byte counts are checked like mxfp4_from_raw
 *      (src/expert_cache.rs:1245-1256): MXFP4 data = rows*ceil(cols/2), scales =
 *      rows*ceil(cols/32); I4_GROUPED scales = rows*ceil(cols/gs)*sizeof(scale). ---- */

/* MoeWeights::router (src/qwen38/model.rs:89-92, src/glm52/model.rs:50): [E, H] row-major. */
RMOE_API rmoe_status rmoe_upload_router(rmoe_layer* layer, const void* w, int32_t dtype, size_t bytes);
/* SIGMOID_GROUPED: MoeWeights::router_bias [E] (selection-only correction bias).
 * SOFTMAX_TOPK: optional f32 bias added to every logit before selection and softmax (the
 * Qwen router itself has none; this carries a harness popularity skew). */
RMOE_API rmoe_status rmoe_upload_router_bias(rmoe_layer* layer, const float* bias, size_t n);
/* ExpertSlot{gate_up: GateUp::Separate{gate, up}, down} (src/expert_cache.rs:640-650).
 * gate/up are [I, H], down is [H, I]. eid is global; only this rank's experts are accepted. */
RMOE_API rmoe_status rmoe_upload_expert(rmoe_layer* layer, int32_t eid,
                               const void* gate, size_t gate_bytes,
                               const void* gate_scale, size_t gate_scale_bytes,
                               const void* up, size_t up_bytes,
                               const void* up_scale, size_t up_scale_bytes,
                               const void* down, size_t down_bytes,
                               const void* down_scale, size_t down_scale_bytes);
/* GateUp::Fused{gate_up} [2I, H]: gate rows 0..I, then up rows I..2I (expert_cache.rs:69-74). */
RMOE_API rmoe_status rmoe_upload_expert_fused(rmoe_layer* layer, int32_t eid,
                                     const void* gate_up, size_t gate_up_bytes,
                                     const void* gate_up_scale, size_t gate_up_scale_bytes,
                                     const void* down, size_t down_bytes,
                                     const void* down_scale, size_t down_scale_bytes);
/* MoeWeights::{sh_gate, sh_up, sh_down, shared_gate} (src/qwen38/model.rs:93-99). shared_gate
 * ([H] f32) may be NULL when desc.shared_gated == 0. Same format as the routed experts. */
RMOE_API rmoe_status rmoe_upload_shared(rmoe_layer* layer,
                               const void* gate, size_t gate_bytes,
                               const void* gate_scale, size_t gate_scale_bytes,
                               const void* up, size_t up_bytes,
                               const void* up_scale, size_t up_scale_bytes,
                               const void* down, size_t down_bytes,
                               const void* down_scale, size_t down_scale_bytes,
                               const float* shared_gate);

/* ---- checkpoints: .safetensors shards straight into the HBM expert tables (the replacement of
 *      the reference's expert streaming tier, src/expert_cache.rs; host file I/O, no GPU work
 *      besides the uploads) ---- */

/* Shards::open_multi (src/safetensors.rs:248-349): every *.safetensors file of the n_dirs
 * directories, sorted by file name, headers parsed and checked (header length within the file,
 * data_offsets ordered and inside it). Errors: RMOE_IO_ERROR (unreadable file, malformed header). */
RMOE_API rmoe_status rmoe_shards_open(const char* const* dirs, int32_t n_dirs, rmoe_shards** out);
RMOE_API rmoe_status rmoe_shards_close(rmoe_shards* shards);
RMOE_API rmoe_status rmoe_shards_count(const rmoe_shards* shards, int64_t* n_tensors);
/* Shards::find (:355): dtype (e.g. "U8", "F32", "BF16"; RMOE_DTYPE_NAME_BYTES bytes, NUL-padded),
 * shape (up to RMOE_MAX_TENSOR_DIMS dims), ndim and byte count of one tensor; any output may be
 * NULL. RMOE_MISSING_TENSOR when absent. */
RMOE_API rmoe_status rmoe_shards_tensor(const rmoe_shards* shards, const char* name, char* dtype, uint64_t* shape,
                                        int32_t* ndim, uint64_t* nbytes);
/* Shards::read_raw (:438-447): the tensor's bytes verbatim into host memory; dst_bytes must equal
 * the tensor's size (else RMOE_SHAPE_MISMATCH). */
RMOE_API rmoe_status rmoe_shards_read_raw(const rmoe_shards* shards, const char* name, void* dst, size_t dst_bytes);
/* One routed expert of checkpoint layer `layer_index` into `layer` (ExpertCache::load_expert with
 * qt_load_mxfp4 / mxfp4_from_raw, src/expert_cache.rs:1232-1256, or qt_load with a .qs sidecar,
 * src/glm52/model.rs:137-156): MXFP4 namings read the packed + scale pair verbatim (lengths
 * rows*ceil(cols/2) and rows*ceil(cols/32), else RMOE_SHAPE_MISMATCH naming the tensor); the other
 * namings read int4 bytes + f32 .qs group scales (layer format RMOE_FMT_I4_GROUPED, scale_dtype
 * RMOE_F32). Plain float expert tensors, which the reference quantizes while loading, are
 * RMOE_NOT_SUPPORTED. */
RMOE_API rmoe_status rmoe_load_expert(rmoe_layer* layer, const rmoe_shards* shards, int32_t naming,
                                      int32_t layer_index, int32_t eid);
/* The rest of a layer's MoeWeights: the router [E, H] (F32 kept f32, BF16 kept bf16, F16 widened),
 * GLM's e_score_correction_bias [E], and the shared expert (Qwen: shared_expert.* plus
 * shared_expert_gate.weight when the layer is gated; GLM: shared_experts.*) in the layer's
 * weight format (MXFP4 pair or int4 + .qs). */
RMOE_API rmoe_status rmoe_load_moe_weights(rmoe_layer* layer, const rmoe_shards* shards, int32_t family,
                                           int32_t layer_index);

/* ---- the hot path (device pointers) ---- */

/* Router matmul + top-k for T tokens: replaces kernels::matmul (src/kernels.rs:113-124) +
 * qwen38::moe::route (src/qwen38/moe.rs:41-76) or glm52::moe::route (src/glm52/moe.rs:247-260).
 * x: [T, H] of x_dtype. ids/weights: [T, k], in the reference's rank order. */
RMOE_API rmoe_status rmoe_route(rmoe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                       int32_t* ids, float* weights, void* stream);

/* Token -> expert dispatch from a routing: unique_experts (src/glm52/moe.rs:333-344) and the
 * per-expert ascending-token row lists of apply_single_expert (:465-470). ids: [T, k].
 * counts: [E] tokens per expert; offsets: [E+1] exclusive prefix; perm_token: [T*k] tokens of
 * expert e at perm_token[offsets[e] .. offsets[e+1]) ascending; uniq: [E] experts in
 * first-occurrence order, n_uniq: [1]. All device pointers; any output may be NULL. */
RMOE_API rmoe_status rmoe_dispatch(rmoe_layer* layer, const int32_t* ids, int32_t T, int32_t* counts,
                          int32_t* offsets, int32_t* perm_token, int32_t* uniq, int32_t* n_uniq,
                          void* stream);

/* The whole MoE block for T tokens: qwen38::generate::moe_forward (src/qwen38/generate.rs:
 * 262-351) or glm52::moe::moe (src/glm52/moe.rs:350-451). out [T, H] f32 is overwritten.
 * ids_out/w_out ([T, k]) receive the routing when non-NULL. x and out are read and written in
 * place when 16-byte aligned (any other alignment is staged through internal buffers). */
RMOE_API rmoe_status rmoe_moe_forward(rmoe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                             float* out, int32_t* ids_out, float* w_out, void* stream);

/* Weights of the latent wrapper of a layer created with router_hidden != hidden: down_proj
 * [hidden][router_hidden] and up_proj [router_hidden][hidden], row-major, proj_dtype RMOE_F32 or
 * RMOE_BF16 (host or device pointers); norm [hidden] f32 (the routed-expert RMSNorm weight) or
 * NULL for none; eps its epsilon. (LatentMoeWeights, src/kimi_k3/moe.rs:42-56.) */
RMOE_API rmoe_status rmoe_upload_latent(rmoe_layer* layer, const void* down_proj, const void* up_proj,
                               int32_t proj_dtype, const float* norm, float eps);

/* Kimi K3 latent MoE for T tokens (kimi_k3::moe::latent_moe, src/kimi_k3/moe.rs:64-116): routes
 * x [T, router_hidden] with the layer's router, projects x down to the experts' width, runs the
 * routed experts there (the shared expert is not included: the caller adds it, as in the
 * reference), RMSNorms each token's summed routed row when a norm weight was uploaded, and
 * projects it back up into out [T, router_hidden] f32 (overwritten). ids_out/w_out ([T, k]) get
 * the routing when non-NULL. Device pointers. */
RMOE_API rmoe_status rmoe_latent_moe(rmoe_layer* layer, const void* x, int32_t x_dtype, int32_t T, float* out,
                            int32_t* ids_out, float* w_out, void* stream);

/* The expert loop with routing given (glm52::moe::moe's loop over Routing via apply_single_expert,
 * src/glm52/moe.rs:463-513): out[t] = sum_j weights[t][j] * expert_{ids[t][j]}(x[t]), plus the
 * (gated) shared expert when with_shared != 0. ids/weights [T][k] (device or host pointers); slots
 * with id -1 or an expert not resident on this layer's EP rank contribute nothing (the building
 * block of expert parallelism: each rank runs it on the token rows it receives). A token that
 * names one expert in several slots gets it once, with the first such slot's weight (the
 * reference's first-match row gather, src/glm52/moe.rs:465-470). */
RMOE_API rmoe_status rmoe_moe_forward_routed(rmoe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                                    const int32_t* ids, const float* weights, int32_t with_shared,
                                    float* out, void* stream);

/* The activation operand of a tensor-core MXFP4 layer for T token rows, token-major: terms
 * [T][4][hidden/2] (four E2M1 terms per row, each rounding what the previous ones left, low
 * nibble first) and term_scales [T][4][hidden/32] (an E8M0 byte per term and 32 columns). No
 * reference counterpart: it is what expert parallelism exchanges instead of x (17 bytes per 32
 * columns against 128 for f32). RMOE_NOT_SUPPORTED on layers off the MXFP4 tensor-core path. */
RMOE_API rmoe_status rmoe_activation_terms(rmoe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                                           uint8_t* terms, uint8_t* term_scales, void* stream);

/* rmoe_moe_forward_routed (without the shared expert) on rows given as their activation terms
 * (rmoe_activation_terms' layout): the same expert loop (apply_single_expert,
 * src/glm52/moe.rs:463-513), the same outputs bit for bit as rmoe_moe_forward_routed on the x the
 * terms were formed from. terms and out 16-byte aligned device pointers. */
RMOE_API rmoe_status rmoe_moe_forward_routed_terms(rmoe_layer* layer, const uint8_t* terms, const uint8_t* term_scales,
                                                   int32_t T, const int32_t* ids, const float* weights, float* out,
                                                   void* stream);

/* Owner-side combine of expert parallelism: out[r] = ((parts[0][r] + parts[1][r]) + ... +
 * parts[n_parts-1][r]) + last[r] for rows x hidden floats, parts [n_parts][rows][hidden] (each
 * rank's partial sum of the token's routed slots, in rank order), last [rows][hidden] the gated
 * shared expert or NULL -- routed contributions first and the shared expert last, the order of
 * qwen38::generate::moe_forward (src/qwen38/generate.rs:324-349). hidden % 4 == 0, 16-byte
 * aligned device pointers; deterministic (no atomics). */
RMOE_API rmoe_status rmoe_sum_rank_parts(float* out, const float* parts, int32_t n_parts, int64_t rows,
                                         int32_t hidden, const float* last, void* stream);

/* Same, with HOST buffers as the Rust call sites hold them (x: &[f32] / bf16 bits, out:
 * &mut [f32]): copies in, runs, copies out and synchronizes. The drop-in for moe_forward's
 * signature. */
RMOE_API rmoe_status rmoe_moe_forward_host(rmoe_layer* layer, const void* x_host, int32_t x_dtype,
                                  int32_t T, float* out_host, int32_t* ids_host,
                                  float* w_host);

/* ---- generic expert-format GEMMs, y[S,O] = x[S,I] . W^T (device pointers) ---- */

/* kernels::matmul_mxfp4 (src/kernels.rs:233-244) */
RMOE_API rmoe_status rmoe_matmul_mxfp4(float* y, const void* x, int32_t x_dtype, const uint8_t* data,
                              const uint8_t* block_scale, int32_t s, int32_t i, int32_t o,
                              void* stream);
/* No counterpart in the reference: kernels::matmul_mxfp4 on the tcgen05 tensor cores. The
 * weights are consumed as stored (E2M1 + E8M0 per 32, kind::mxf4 block32); x becomes a four-term
 * E2M1 expansion (~11 significant bits), products are exact and accumulated in f32. Needs
 * i % 32 == 0 (else RMOE_NOT_SUPPORTED). */
RMOE_API rmoe_status rmoe_matmul_mxfp4_tc(float* y, const void* x, int32_t x_dtype, const uint8_t* data,
                                 const uint8_t* block_scale, int32_t s, int32_t i, int32_t o,
                                 void* stream);
/* No counterpart in the reference: rmoe_matmul_mxfp4 without any device allocation, for callers
 * that cannot allocate on the hot path (device memory reserved by their own arena). Scratch is a
 * fixed device array of RMOE_NOALLOC_SCRATCH_BYTES; shapes needing more (16-bit s*i + 4*s + 256
 * bytes) are rejected with RMOE_INVALID_ARG. The first call on each device (with that device
 * current) resolves the array's address and caches it for the process: make it before any stream
 * capture, and do not call this entry point after cudaDeviceReset on that device (the cached
 * address would be stale). Only i % 32 == 0 uses the scratch (other i take a scalar kernel that
 * needs none, so the size limit does not apply to them). Calls that overlap
 * in time on one device share the scratch and race: order them on one stream. */
#define RMOE_NOALLOC_SCRATCH_BYTES ((8u << 20) + 4096u) /* s*i <= 4M at s <= 512, e.g. 512 x 8192 */
RMOE_API rmoe_status rmoe_matmul_mxfp4_noalloc(float* y, const void* x, int32_t x_dtype,
                                      const uint8_t* data, const uint8_t* block_scale, int32_t s,
                                      int32_t i, int32_t o, void* stream);
/* kernels::matmul_i4_grouped (src/kernels.rs:276-296) */
RMOE_API rmoe_status rmoe_matmul_i4_grouped(float* y, const void* x, int32_t x_dtype, const uint8_t* q4,
                                   const void* scale, int32_t scale_dtype, int32_t group_size,
                                   int32_t s, int32_t i, int32_t o, void* stream);
/* The QT kinds of quant::QTKind (src/quant.rs:80-109). */
typedef enum rmoe_qt_kind {
  RMOE_QT_F32 = 0,        /* f32 [O, I] */
  RMOE_QT_I8 = 1,         /* int8 [O, I] + f32 scale per row */
  RMOE_QT_I4 = 2,         /* offset-binary nibbles [O, ceil(I/2)] (low first) + f32 scale per row */
  RMOE_QT_I2 = 3,         /* 2-bit values + 2, 4 per byte low bits first [O, ceil(I/4)] + f32 scale per row */
  RMOE_QT_I4_GROUPED = 4, /* nibbles + f32 scale per group_size elements of a row */
  RMOE_QT_MXFP4 = 5       /* E2M1 nibbles + E8M0 byte per 32 */
} rmoe_qt_kind;

/* kernels::matmul_qt (src/kernels.rs:1104-1132), the dispatcher every layer calls: y[S,O] =
 * x[S,I] . W^T for a weight of any QT kind, with the reference's per-kind paths -- I8 always and
 * I4 at s >= 2 through integer dot products against int8-quantized activations (qrow_i8 per row,
 * y = float(dot) * scale[o] * sx[s]: bit-exact with the reference), I4 at s == 1 and I2 as
 * float-weight products, F32 as rmoe_matmul_f32 (exact chains), I4_GROUPED and MXFP4 as
 * rmoe_matmul_i4_grouped / rmoe_matmul_mxfp4. Device pointers; group_size only for I4_GROUPED. */
RMOE_API rmoe_status rmoe_matmul_qt(float* y, const void* x, int32_t x_dtype, int32_t kind, const void* data,
                                    const void* scale, int32_t group_size, int32_t s, int32_t i, int32_t o,
                                    void* stream);
/* kernels::matmul (src/kernels.rs:113-124) for f32/bf16 weights: each y element is the
 * reference's exact left-to-right f32 chain (separate multiply and add, from -0.0). */
RMOE_API rmoe_status rmoe_matmul_f32(float* y, const void* x, int32_t x_dtype, const void* w,
                            int32_t w_dtype, int32_t s, int32_t i, int32_t o, void* stream);

/* ---- seeded synthetic bytes for benches/tests (SplitMix64 counter stream; identical to the
 *      host generator rabbit_b200/synth.py). mode 0: uniform bytes; mode 1: E8M0 bytes
 *      127+lo .. 127+hi. ---- */
RMOE_API rmoe_status rmoe_synth_bytes(void* dst, size_t n, uint64_t key, int32_t mode, int32_t lo,
                             int32_t hi, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RMOE_H */
