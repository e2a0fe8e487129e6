/*
 * rmoe_oracle.h -- CPU restatement of rabbit's routed-MoE path (TEST INFRASTRUCTURE ONLY).
 *
 * This is the parity checker for the CUDA path in rabbit_b200/, never part of it. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may load it.
 *
 * Every function restates one reference function (ferrumox/rabbit v0.29.1, paths relative to
 * that crate) in plain C, compiled with -ffp-contract=off so each Rust `a * b + c` stays a
 * separately rounded multiply and add, exactly like rustc emits it. `expf` is glibc's, which is
 * what Rust's f32::exp lowers to on Linux. Rust's float `Sum` folds from -0.0; the reference's
 * hand-written loops that start from `0f32` start from +0.0 here too.
 *
 * Parity pin: the reference's own known-answer unit tests are restated as self-tests in
 * tests/test_oracle.py (E2M1/E8M0 tables, the -320 and 9.0 matmul answers, route picks, group
 * ties, ...). The reference crate itself cannot be built in this image (no Rust toolchain).
 */
#ifndef RMOE_ORACLE_H
#define RMOE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- formats: src/quant.rs ---- */
float orc_e2m1_decode(uint8_t nibble);                 /* quant.rs:348-356 */
float orc_e8m0_decode(uint8_t byte);                   /* quant.rs:391-396 */
uint8_t orc_e2m1_encode(float value);                  /* quant.rs:361-374 */
void orc_choose_block_scale(float amax, uint8_t* byte, float* scale); /* quant.rs:404-410 */
void orc_pack_mxfp4(const float* w, uint8_t* q, uint8_t* block_scale, size_t rows,
                    size_t cols);                      /* quant.rs:413-435 */
void orc_quant_int4_grouped(const float* w, size_t rows, size_t cols, int bits, size_t gs,
                            uint8_t* out, float* scale); /* quant.rs:486-517 */
void orc_row_f32_mxfp4(const uint8_t* data, const uint8_t* bs, size_t cols, size_t row,
                       float* out);                    /* quant.rs:330-341 */

/* ---- kernels: src/kernels.rs (y[S,O] = x[S,I] . W^T) ---- */
void orc_matmul_f32(float* y, const float* x, const float* w, size_t s, size_t i,
                    size_t o);                         /* kernels.rs:113-124 */
void orc_matmul_mxfp4(float* y, const float* x, const uint8_t* data, const uint8_t* bs,
                      size_t s, size_t i, size_t o);   /* kernels.rs:247-267 (scalar tier) */
void orc_matmul_i4_grouped(float* y, const float* x, const uint8_t* q4, const float* scale,
                           size_t gs, size_t s, size_t i, size_t o); /* kernels.rs:276-296 */

/* ---- activations: src/glm52/moe.rs:33-35, src/kimi_linear/ops.rs:22-28 ---- */
float orc_siluf(float x);
float orc_sigmoid(float x);

/* ---- Qwen router: src/qwen38/moe.rs:41-76. Returns k; ids/w must hold min(topk, n). ---- */
size_t orc_qwen_route(const float* logits, size_t n, size_t topk, int32_t* ids, float* w);

/* ---- GLM noaux_tc router: src/glm52/moe.rs:131-260 ---- */
float orc_top2_sum(const float* vals, size_t n);       /* moe.rs:193-205 */
/* rank_top_grouped on precomputed choice/logit (moe.rs:214-229); returns k */
size_t orc_rank_top_grouped(const float* choice, const float* logit, size_t e, size_t k,
                            size_t n_group, size_t topk_group, int32_t* ids, float* w);
/* route() for s tokens: router matmul + sigmoid + bias + grouped top-k + normalize_and_scale */
size_t orc_cache_route_select(const float* choice, const float* logit, size_t e, size_t k, size_t route_j,
                              size_t route_m, const uint8_t* resident, int32_t* ids, float* w);
void orc_glm_route_cache(const float* x, const float* router, const float* bias, size_t s, size_t d,
                         size_t e, size_t k, size_t route_j, size_t route_m, const uint8_t* resident,
                         int norm_topk, float routed_scale, int32_t* ids, float* w);
void orc_glm_route(const float* x, const float* router, const float* bias, size_t s,
                   size_t d, size_t e, size_t k, size_t n_group, size_t topk_group,
                   int norm_topk, float routed_scale, int32_t* ids, float* w);

/* ---- dispatch: unique_experts (moe.rs:333-344) + apply_single_expert row lists (:465-470) */
size_t orc_unique_experts(const int32_t* ids, size_t s, size_t k, int32_t* uniq);
/* For expert eid: tokens (ascending) that picked it and the weight of that slot. Returns nr. */
size_t orc_expert_rows(const int32_t* ids, const float* w, size_t s, size_t k, int32_t eid,
                       int32_t* rows, float* row_w);

/* ---- one expert's weights in the reference's byte layout ----
 * fmt 0 = MXFP4 (E2M1 nibbles low-first + one E8M0 byte per 32 along the row),
 * fmt 1 = grouped int4 (offset-binary nibbles low-first + one f32 scale per `gs` along the row).
 * gate/up are [inter, hidden]; down is [hidden, inter]. */
typedef struct orc_expert {
  const uint8_t* gate; const void* gate_scale;
  const uint8_t* up;   const void* up_scale;
  const uint8_t* down; const void* down_scale;
} orc_expert;

/* matmul_qt restricted to the two routed-expert formats. */
float orc_qrow_i8(const float* x, size_t n, int8_t* q);
int32_t orc_dot_i8i8(const int8_t* w, const int8_t* x, size_t n);
int32_t orc_dot_i4i8(const uint8_t* w4, const int8_t* x, size_t n);
void orc_matmul_q(float* y, const float* x, const int8_t* q, const float* scale, size_t s, size_t i, size_t o);
void orc_matmul_i4(float* y, const float* x, const uint8_t* q4, const float* scale, size_t s, size_t i, size_t o);
void orc_matmul_i2(float* y, const float* x, const uint8_t* q2, const float* scale, size_t s, size_t i, size_t o);
void orc_matmul_qt_kind(float* y, const float* x, int kind, const void* data, const void* scale, size_t gs,
                        size_t s, size_t i, size_t o);
void orc_matmul_qt(float* y, const float* x, const uint8_t* data, const void* scale, int fmt,
                   size_t gs, size_t s, size_t i, size_t o);

/* apply_single_expert (moe.rs:463-513), Separate gate/up, Silu: out[token] += w * down(...) */
void orc_apply_single_expert(const orc_expert* ex, int fmt, size_t gs, int32_t eid,
                             const int32_t* ids, const float* w, size_t s, size_t k,
                             const float* x, size_t d, size_t inter, float* out);

/* Qwen moe_forward (qwen38/generate.rs:262-351) minus the expert cache. `logit_bias` (nullable,
 * [E]) is this harness's Zipf popularity skew, added to every router logit before route();
 * the reference router has no bias. `shared` may be NULL (no shared expert). `shared_gate`
 * ([d] f32) may be NULL (ungated). Experts are applied in unique_experts() order, shared last.
 * Writes the routing it used to ids/w ([s,k]) when non-NULL. */
void orc_moe_forward_qwen(const float* x, size_t s, size_t d, size_t e, size_t k,
                          size_t inter, size_t shared_inter, const float* router,
                          const float* logit_bias, const orc_expert* experts,
                          const orc_expert* shared, const float* shared_gate, int fmt,
                          size_t gs, float* out, int32_t* ids_out, float* w_out);

/* GLM moe() (glm52/moe.rs:350-451) minus the expert cache: grouped sigmoid routing, routed
 * experts in unique order, shared expert (ungated) added last. */
void orc_moe_glm(const float* x, size_t s, size_t d, size_t e, size_t k, size_t inter,
                 size_t shared_inter, const float* router, const float* bias, size_t n_group,
                 size_t topk_group, int norm_topk, float routed_scale,
                 const orc_expert* experts, const orc_expert* shared, int fmt, size_t gs,
                 float* out, int32_t* ids_out, float* w_out);

/* ---- the timed CPU baseline: AVX-512F/BW tier (kernels.rs:703-749, :783-797) ---- */
int orc_has_avx512(void);
void orc_matmul_mxfp4_avx512(float* y, const float* x, const uint8_t* data, const uint8_t* bs,
                             size_t s, size_t i, size_t o);
/* Whole Qwen layer with the AVX-512 tier for MXFP4 products (same structure as
 * orc_moe_forward_qwen). nthreads <= 0 means all OpenMP threads. */
void orc_moe_forward_qwen_fast(const float* x, size_t s, size_t d, size_t e, size_t k,
                               size_t inter, size_t shared_inter, const float* router,
                               const float* logit_bias, const orc_expert* experts,
                               const orc_expert* shared, const float* shared_gate, float* out,
                               int32_t* ids_out, float* w_out);
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
