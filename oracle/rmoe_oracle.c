/*
 * rmoe_oracle.c -- CPU restatement of rabbit's routed-MoE path. TEST INFRASTRUCTURE ONLY:
 * the parity checker for the CUDA path, never linked into the product library.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp). Each function
 * cites the reference function it restates (ferrumox/rabbit v0.29.1, crate-relative paths).
 * Parity pin: the reference's own known-answer tests, restated in tests/test_oracle.py.
 */
#include "rmoe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Rust's `impl Sum for f32` folds from -0.0 (the identity that keeps sum([-0.0]) == -0.0). */
#define RUST_SUM_INIT (-0.0f)

/* ------------------------------------------------------------------ formats (quant.rs) */

static const float kE2m1Mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* quant.rs:353-356: bit 3 = sign, bits 2..0 index the 8 magnitudes; code 8 is -0.0. */
float orc_e2m1_decode(uint8_t nibble) {
  float mag = kE2m1Mag[nibble & 0x7];
  return (nibble & 0x8) ? -mag : mag;
}

/* quant.rs:391-396: the byte is f32's own biased exponent; byte 0 is the subnormal 2^-127. */
float orc_e8m0_decode(uint8_t byte) {
  uint32_t bits = byte == 0 ? (1u << 22) : ((uint32_t)byte << 23);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* quant.rs:361-374: nearest of the 8 magnitudes, strict '<' so ties keep the lower index;
 * sign only for negative non-zero values. */
uint8_t orc_e2m1_encode(float value) {
  uint8_t sign = (signbit(value) && value != 0.0f) ? 0x8 : 0;
  float av = fabsf(value);
  size_t best = 0;
  float best_diff = 3.40282347e+38f;
  for (size_t i = 0; i < 8; i++) {
    float diff = fabsf(av - kE2m1Mag[i]);
    if (diff < best_diff) {
      best_diff = diff;
      best = i;
    }
  }
  return sign | (uint8_t)best;
}

/* quant.rs:404-410: shared_exp = floor(log2(amax)) - 2 clamped to [-127,127]. */
void orc_choose_block_scale(float amax, uint8_t* byte, float* scale) {
  if (amax <= 0.0f) {
    *byte = 127;
    *scale = 1.0f;
    return;
  }
  int e = (int)floorf(log2f(amax)) - 2;
  if (e < -127) e = -127;
  if (e > 127) e = 127;
  *byte = (uint8_t)(e + 127);
  /* 2f32.powi(e): exact power of two (subnormal at -127) */
  *scale = ldexpf(1.0f, e);
}

/* quant.rs:413-435 */
void orc_pack_mxfp4(const float* w, uint8_t* q, uint8_t* block_scale, size_t rows,
                    size_t cols) {
  size_t rb = (cols + 1) / 2, bpr = (cols + 31) / 32;
  for (size_t o = 0; o < rows; o++) {
    const float* wr = w + o * cols;
    uint8_t* qr = q + o * rb;
    for (size_t b = 0; b < bpr; b++) {
      size_t start = b * 32, end = start + 32 < cols ? start + 32 : cols;
      float amax = 0.0f;
      for (size_t k = start; k < end; k++) amax = fmaxf(amax, fabsf(wr[k]));
      uint8_t byte;
      float scale;
      orc_choose_block_scale(amax, &byte, &scale);
      block_scale[o * bpr + b] = byte;
      for (size_t k = start; k < end; k++) {
        uint8_t code = orc_e2m1_encode(wr[k] / scale);
        if ((k & 1) == 0)
          qr[k >> 1] = (uint8_t)((qr[k >> 1] & 0xF0) | code);
        else
          qr[k >> 1] = (uint8_t)((qr[k >> 1] & 0x0F) | (code << 4));
      }
    }
  }
}

/* lrintf under the default rounding mode == Rust's round_ties_even (quant.rs:40-43) */
static int32_t rne(float x) { return (int32_t)nearbyintf(x); }

/* quant.rs:486-517 */
void orc_quant_int4_grouped(const float* w, size_t rows, size_t cols, int bits, size_t gs,
                            uint8_t* out, float* scale) {
  int32_t qmax = (1 << (bits - 1)) - 1;
  size_t ng = (cols + gs - 1) / gs, rb = (cols + 1) / 2;
  memset(out, 0, rows * rb);
  for (size_t o = 0; o < rows; o++) {
    const float* wr = w + o * cols;
    for (size_t g = 0; g < ng; g++) {
      size_t start = g * gs, end = start + gs < cols ? start + gs : cols;
      float amax = 0.0f;
      for (size_t k = start; k < end; k++) amax = fmaxf(amax, fabsf(wr[k]));
      float sc = amax / (float)qmax;
      scale[o * ng + g] = sc > 1e-8f ? sc : 1e-8f;
    }
    uint8_t* qr = out + o * rb;
    for (size_t i = 0; i < cols; i += 2) {
      float s0 = scale[o * ng + i / gs];
      int32_t v0 = rne(wr[i] / s0);
      v0 = v0 < -8 ? -8 : (v0 > qmax ? qmax : v0);
      int32_t v1 = 0;
      if (i + 1 < cols) {
        float s1 = scale[o * ng + (i + 1) / gs];
        v1 = rne(wr[i + 1] / s1);
        v1 = v1 < -8 ? -8 : (v1 > qmax ? qmax : v1);
      }
      qr[i / 2] = (uint8_t)((uint8_t)(v0 + 8) | (uint8_t)((v1 + 8) << 4));
    }
  }
}

/* quant.rs:330-341 */
void orc_row_f32_mxfp4(const uint8_t* data, const uint8_t* bs, size_t cols, size_t row,
                       float* out) {
  size_t rb = (cols + 1) / 2, bpr = (cols + 31) / 32;
  const uint8_t* wr = data + row * rb;
  const uint8_t* bsr = bs + row * bpr;
  for (size_t k = 0; k < cols; k++) {
    uint8_t byte = wr[k >> 1];
    uint8_t nib = (k & 1) == 0 ? (byte & 0xF) : (byte >> 4);
    out[k] = orc_e2m1_decode(nib) * orc_e8m0_decode(bsr[k / 32]);
  }
}

/* ------------------------------------------------------------------ kernels.rs */

/* kernels.rs:113-124: per (token, output row) a sequential f32 fold of x*w from -0.0.
 * Rows in parallel, as rayon does; the per-element arithmetic is unchanged by that. */
void orc_matmul_f32(float* y, const float* x, const float* w, size_t s, size_t i, size_t o) {
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++) {
    const float* wr = w + (size_t)oi * i;
    for (size_t si = 0; si < s; si++) {
      const float* xs = x + si * i;
      float a = RUST_SUM_INIT;
      for (size_t k = 0; k < i; k++) a = a + xs[k] * wr[k];
      y[si * o + (size_t)oi] = a;
    }
  }
}

/* kernels.rs:247-267 (the scalar tier): a += (x * e2m1) * e8m0, from +0.0. */
void orc_matmul_mxfp4(float* y, const float* x, const uint8_t* data, const uint8_t* bs,
                      size_t s, size_t i, size_t o) {
  size_t rb = (i + 1) / 2, bpr = (i + 31) / 32;
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++) {
    const uint8_t* wr = data + (size_t)oi * rb;
    const uint8_t* bsr = bs + (size_t)oi * bpr;
    for (size_t si = 0; si < s; si++) {
      const float* xs = x + si * i;
      float a = 0.0f;
      for (size_t k = 0; k < i; k++) {
        uint8_t byte = wr[k >> 1];
        uint8_t nib = (k & 1) == 0 ? (byte & 0xF) : (byte >> 4);
        float t = xs[k] * orc_e2m1_decode(nib);
        t = t * orc_e8m0_decode(bsr[k / 32]);
        a = a + t;
      }
      y[si * o + (size_t)oi] = a;
    }
  }
}

/* kernels.rs:276-296: a += (x * (nibble - 8)) * scale[k / gs], from +0.0. */
void orc_matmul_i4_grouped(float* y, const float* x, const uint8_t* q4, const float* scale,
                           size_t gs, size_t s, size_t i, size_t o) {
  size_t rb = (i + 1) / 2, ng = (i + gs - 1) / gs;
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++) {
    const uint8_t* wr = q4 + (size_t)oi * rb;
    const float* sc = scale + (size_t)oi * ng;
    for (size_t si = 0; si < s; si++) {
      const float* xs = x + si * i;
      float a = 0.0f;
      for (size_t k = 0; k < i; k++) {
        uint8_t byte = wr[k >> 1];
        uint8_t nib = (k & 1) == 0 ? (byte & 0xF) : (byte >> 4);
        float t = xs[k] * (float)((int32_t)nib - 8);
        t = t * sc[k / gs];
        a = a + t;
      }
      y[si * o + (size_t)oi] = a;
    }
  }
}

void orc_matmul_qt(float* y, const float* x, const uint8_t* data, const void* scale, int fmt,
                   size_t gs, size_t s, size_t i, size_t o) {
  if (fmt == 0)
    orc_matmul_mxfp4(y, x, data, (const uint8_t*)scale, s, i, o);
  else
    orc_matmul_i4_grouped(y, x, data, (const float*)scale, gs, s, i, o);
}

/* ---- the other QT kinds of matmul_qt (kernels.rs:1104-1132) */

/* kernels.rs:301-309 qrow_i8: s = max(amax / 127, 1e-12), q = round_ties_even(x * (1 / s)) */
float orc_qrow_i8(const float* x, size_t n, int8_t* q) {
  float amax = 0.0f;
  for (size_t k = 0; k < n; k++) amax = fmaxf(amax, fabsf(x[k]));
  float sc = fmaxf(amax / 127.0f, 1e-12f);
  float inv = 1.0f / sc;
  for (size_t k = 0; k < n; k++) q[k] = (int8_t)(int32_t)nearbyintf(x[k] * inv);
  return sc;
}

/* kernels.rs:331-337 */
int32_t orc_dot_i8i8(const int8_t* w, const int8_t* x, size_t n) {
  int32_t sum = 0;
  for (size_t k = 0; k < n; k++) sum += (int32_t)w[k] * (int32_t)x[k];
  return sum;
}

/* kernels.rs:355-368: nibble - 8 (low nibble first) times int8 */
int32_t orc_dot_i4i8(const uint8_t* w4, const int8_t* x, size_t n) {
  int32_t sum = 0;
  for (size_t k = 0; k < n; k++) {
    uint8_t b = w4[k >> 1];
    int32_t v = (int32_t)((k & 1) ? (b >> 4) : (b & 0xF)) - 8;
    sum += v * (int32_t)x[k];
  }
  return sum;
}

/* kernels.rs:135-148 matmul_q (int8 weights, per-row scale, float path): a = sum x * w from
 * +0.0 (iterator sum), then a * scale */
void orc_matmul_q(float* y, const float* x, const int8_t* q, const float* scale, size_t s, size_t i, size_t o) {
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++)
    for (size_t si = 0; si < s; si++) {
      float a = RUST_SUM_INIT;
      for (size_t k = 0; k < i; k++) a = a + x[si * i + k] * (float)q[(size_t)oi * i + k];
      y[si * o + oi] = a * scale[oi];
    }
}

/* kernels.rs:167-193 matmul_i4_scalar: pairs a += x0 * lo + x1 * hi (left to right), tail
 * nibble alone, then a * scale */
void orc_matmul_i4(float* y, const float* x, const uint8_t* q4, const float* scale, size_t s, size_t i, size_t o) {
  size_t rb = (i + 1) / 2;
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++)
    for (size_t si = 0; si < s; si++) {
      const uint8_t* w = q4 + (size_t)oi * rb;
      const float* xs = x + si * i;
      float a = 0.0f;
      size_t k = 0;
      for (; k + 1 < i; k += 2) {
        uint8_t b = w[k >> 1];
        float lo = (float)((int32_t)(b & 0xF) - 8), hi = (float)((int32_t)(b >> 4) - 8);
        a = a + (xs[k] * lo + xs[k + 1] * hi);
      }
      if (k < i) a = a + xs[k] * (float)((int32_t)(w[k >> 1] & 0xF) - 8);
      y[si * o + oi] = a * scale[oi];
    }
}

/* kernels.rs:206-224 matmul_i2_scalar: 4 values per byte, low bits first, value + 2 stored */
void orc_matmul_i2(float* y, const float* x, const uint8_t* q2, const float* scale, size_t s, size_t i, size_t o) {
  size_t rb = (i + 3) / 4;
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++)
    for (size_t si = 0; si < s; si++) {
      const uint8_t* w = q2 + (size_t)oi * rb;
      const float* xs = x + si * i;
      float a = 0.0f;
      for (size_t k = 0; k < i; k++) {
        int32_t v = (int32_t)((w[k >> 2] >> ((k & 3) * 2)) & 3) - 2;
        a = a + xs[k] * (float)v;
      }
      y[si * o + oi] = a * scale[oi];
    }
}

/* kernels.rs:1063-1098 matmul_q_idot / matmul_i4_idot: activations quantized per row (qrow_i8),
 * y = (float)dot * scale[o] * sx[s] */
static void matmul_idot(float* y, const float* x, const void* w, int w4, const float* scale, size_t s, size_t i,
                        size_t o) {
  int8_t* xq = (int8_t*)malloc(s * i + 1);
  float* sx = (float*)malloc((s + 1) * sizeof(float));
  for (size_t si = 0; si < s; si++) sx[si] = orc_qrow_i8(x + si * i, i, xq + si * i);
  size_t rb = w4 ? (i + 1) / 2 : i;
#pragma omp parallel for schedule(static)
  for (long oi = 0; oi < (long)o; oi++)
    for (size_t si = 0; si < s; si++) {
      int32_t d = w4 ? orc_dot_i4i8((const uint8_t*)w + (size_t)oi * rb, xq + si * i, i)
                     : orc_dot_i8i8((const int8_t*)w + (size_t)oi * rb, xq + si * i, i);
      y[si * o + oi] = (float)d * scale[oi] * sx[si];
    }
  free(xq);
  free(sx);
}

/* kernels.rs:1104-1132 matmul_qt for every QT kind: 0 F32, 1 I8 (IDOT), 2 I4 (IDOT at s >= 2,
 * else the float path), 3 I2, 4 I4Grouped, 5 MxFp4 */
void orc_matmul_qt_kind(float* y, const float* x, int kind, const void* data, const void* scale, size_t gs,
                        size_t s, size_t i, size_t o) {
  switch (kind) {
    case 0: orc_matmul_f32(y, x, (const float*)data, s, i, o); break;
    case 1: matmul_idot(y, x, data, 0, (const float*)scale, s, i, o); break;
    case 2:
      if (s >= 2) matmul_idot(y, x, data, 1, (const float*)scale, s, i, o);
      else orc_matmul_i4(y, x, (const uint8_t*)data, (const float*)scale, s, i, o);
      break;
    case 3: orc_matmul_i2(y, x, (const uint8_t*)data, (const float*)scale, s, i, o); break;
    case 4: orc_matmul_i4_grouped(y, x, (const uint8_t*)data, (const float*)scale, gs, s, i, o); break;
    default: orc_matmul_mxfp4(y, x, (const uint8_t*)data, (const uint8_t*)scale, s, i, o); break;
  }
}

/* ------------------------------------------------------------------ activations */

/* glm52/moe.rs:33-35 siluf == kimi_linear/ops.rs:22-24 swish */
float orc_siluf(float x) { return x / (1.0f + expf(-x)); }
/* kimi_linear/ops.rs:26-28 */
float orc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

/* ------------------------------------------------------------------ Qwen router */

/* qwen38/moe.rs:41-76: running top-k by (logit desc, id asc) via strict '>' insertion, then a
 * max-subtracted softmax over the k winners with a sequential sum from +0.0. */
size_t orc_qwen_route(const float* logits, size_t n, size_t topk, int32_t* ids, float* w) {
  size_t k = topk < n ? topk : n;
  if (k == 0) return 0;
  size_t len = 0;
  for (size_t id = 0; id < n; id++) {
    float l = logits[id];
    size_t pos = len;
    for (size_t p = 0; p < len; p++)
      if (l > w[p]) {
        pos = p;
        break;
      }
    if (pos < len) {
      size_t last = len < k ? len : k - 1; /* insert, dropping the tail when full */
      for (size_t q = last; q > pos; q--) {
        ids[q] = ids[q - 1];
        w[q] = w[q - 1];
      }
      ids[pos] = (int32_t)id;
      w[pos] = l;
      if (len < k) len++;
    } else if (len < k) {
      ids[len] = (int32_t)id;
      w[len] = l;
      len++;
    }
  }
  float mx = w[0], sum = 0.0f;
  for (size_t j = 0; j < k; j++) {
    w[j] = expf(w[j] - mx);
    sum = sum + w[j];
  }
  for (size_t j = 0; j < k; j++) w[j] = w[j] / sum;
  return k;
}

/* ------------------------------------------------------------------ GLM router */

/* glm52/moe.rs:193-205 */
float orc_top2_sum(const float* vals, size_t n) {
  float t1 = -INFINITY, t2 = -INFINITY;
  for (size_t j = 0; j < n; j++) {
    float v = vals[j];
    if (v > t1) {
      t2 = t1;
      t1 = v;
    } else if (v > t2) {
      t2 = v;
    }
  }
  return isfinite(t2) ? t1 + t2 : t1;
}

/* glm52/moe.rs:148-188: k rounds of a strict '>' scan from -1e30 over untaken (and allowed)
 * experts; the stored weight is the plain logit (sigmoid), never the biased choice. */
static size_t rank_top_within(const float* choice, const float* logit, size_t e, size_t k,
                              const uint8_t* allowed, int32_t* ids, float* w) {
  size_t n_allowed = 0;
  for (size_t j = 0; j < e; j++) n_allowed += allowed ? allowed[j] != 0 : 1;
  if (k > n_allowed) k = n_allowed;
  uint8_t* taken = (uint8_t*)calloc(e, 1);
  for (size_t r = 0; r < k; r++) {
    long best = -1;
    float bv = -1e30f;
    for (size_t j = 0; j < e; j++)
      if (!taken[j] && (!allowed || allowed[j]) && choice[j] > bv) {
        bv = choice[j];
        best = (long)j;
      }
    if (best < 0) { /* the reference panics here (all scores <= -1e30 or NaN) */
      ids[r] = -1;
      w[r] = 0.0f;
      continue;
    }
    taken[best] = 1;
    ids[r] = (int32_t)best;
    w[r] = logit[best];
  }
  free(taken);
  return k;
}

typedef struct { size_t g; float score; } gscore;
static int cmp_gscore(const void* a, const void* b) {
  const gscore* x = (const gscore*)a;
  const gscore* y = (const gscore*)b;
  if (x->score > y->score) return -1; /* descending score */
  if (x->score < y->score) return 1;
  return x->g < y->g ? -1 : (x->g > y->g); /* ties: lower group first */
}

/* glm52/moe.rs:214-229 */
size_t orc_rank_top_grouped(const float* choice, const float* logit, size_t e, size_t k,
                            size_t n_group, size_t topk_group, int32_t* ids, float* w) {
  if (n_group <= 1) return rank_top_within(choice, logit, e, k, NULL, ids, w);
  size_t gsz = e / n_group;
  gscore* gs = (gscore*)malloc(n_group * sizeof(gscore));
  for (size_t g = 0; g < n_group; g++) {
    gs[g].g = g;
    gs[g].score = orc_top2_sum(choice + g * gsz, gsz);
  }
  qsort(gs, n_group, sizeof(gscore), cmp_gscore);
  uint8_t* allowed = (uint8_t*)calloc(e, 1);
  for (size_t t = 0; t < topk_group && t < n_group; t++)
    for (size_t j = 0; j < gsz; j++) allowed[gs[t].g * gsz + j] = 1;
  size_t r = rank_top_within(choice, logit, e, k, allowed, ids, w);
  free(allowed);
  free(gs);
  return r;
}

/* glm52/moe.rs:131-141 router_scores + :247-260 route + :231-241 normalize_and_scale */
void orc_glm_route(const float* x, const float* router, const float* bias, size_t s,
                   size_t d, size_t e, size_t k, size_t n_group, size_t topk_group,
                   int norm_topk, float routed_scale, int32_t* ids, float* w) {
  float* logit = (float*)malloc(e * sizeof(float));
  float* choice = (float*)malloc(e * sizeof(float));
  for (size_t si = 0; si < s; si++) {
    const float* xs = x + si * d;
    for (size_t j = 0; j < e; j++) {
      const float* wr = router + j * d;
      float a = RUST_SUM_INIT;
      for (size_t q = 0; q < d; q++) a = a + xs[q] * wr[q];
      logit[j] = 1.0f / (1.0f + expf(-a));
      choice[j] = logit[j] + bias[j];
    }
    int32_t* pi = ids + si * k;
    float* pw = w + si * k;
    size_t kk = orc_rank_top_grouped(choice, logit, e, k, n_group, topk_group, pi, pw);
    if (norm_topk) {
      float sum = RUST_SUM_INIT;
      for (size_t j = 0; j < kk; j++) sum = sum + pw[j];
      sum = sum + 1e-20f;
      for (size_t j = 0; j < kk; j++) pw[j] = pw[j] / sum;
    }
    for (size_t j = 0; j < kk; j++) pw[j] = pw[j] * routed_scale;
    for (size_t j = kk; j < k; j++) {
      pi[j] = -1;
      pw[j] = 0.0f;
    }
  }
  free(logit);
  free(choice);
}

/* glm52/moe.rs:293-323 cache_route_select: rank the top m = max(route_m, k) by choice
 * (rank_top, :148-166), keep ranked[0..j), j = min(route_j, k, m), fill with resident ranked[j..]
 * in order, then with any not-yet-picked ranked[j..] in order. resident NULL = every expert
 * resident. Returns the number picked (ids/w: k entries, the rest -1 / 0). */
size_t orc_cache_route_select(const float* choice, const float* logit, size_t e, size_t k, size_t route_j,
                              size_t route_m, const uint8_t* resident, int32_t* ids, float* w) {
  size_t m = route_m > k ? route_m : k;
  if (m > e) m = e;
  int32_t* rid = (int32_t*)malloc((m + 1) * sizeof(int32_t));
  float* rw = (float*)malloc((m + 1) * sizeof(float));
  rank_top_within(choice, logit, e, m, NULL, rid, rw);
  size_t jj = route_j < k ? route_j : k;
  if (jj > m) jj = m;
  size_t n = 0;
  for (size_t r = 0; r < jj; r++, n++) {
    ids[n] = rid[r];
    w[n] = rw[r];
  }
  for (size_t r = jj; r < m && n < k; r++)
    if (!resident || resident[rid[r]]) {
      ids[n] = rid[r];
      w[n] = rw[r];
      n++;
    }
  for (size_t r = jj; r < m && n < k; r++) {
    int dup = 0;
    for (size_t q = 0; q < n; q++) dup |= ids[q] == rid[r];
    if (dup) continue;
    ids[n] = rid[r];
    w[n] = rw[r];
    n++;
  }
  for (size_t j = n; j < k; j++) {
    ids[j] = -1;
    w[j] = 0.0f;
  }
  free(rid);
  free(rw);
  return n;
}

/* glm52/moe.rs:272-290 route_cache_aware: router_scores, cache_route_select, normalize_and_scale */
void orc_glm_route_cache(const float* x, const float* router, const float* bias, size_t s, size_t d,
                         size_t e, size_t k, size_t route_j, size_t route_m, const uint8_t* resident,
                         int norm_topk, float routed_scale, int32_t* ids, float* w) {
  float* logit = (float*)malloc(e * sizeof(float));
  float* choice = (float*)malloc(e * sizeof(float));
  for (size_t si = 0; si < s; si++) {
    const float* xs = x + si * d;
    for (size_t j = 0; j < e; j++) {
      const float* wr = router + j * d;
      float a = RUST_SUM_INIT;
      for (size_t q = 0; q < d; q++) a = a + xs[q] * wr[q];
      logit[j] = 1.0f / (1.0f + expf(-a));
      choice[j] = logit[j] + bias[j];
    }
    int32_t* pi = ids + si * k;
    float* pw = w + si * k;
    size_t n = orc_cache_route_select(choice, logit, e, k, route_j, route_m, resident, pi, pw);
    if (norm_topk) {
      float sum = RUST_SUM_INIT;
      for (size_t j = 0; j < n; j++) sum = sum + pw[j];
      sum = sum + 1e-20f;
      for (size_t j = 0; j < n; j++) pw[j] = pw[j] / sum;
    }
    for (size_t j = 0; j < n; j++) pw[j] = pw[j] * routed_scale;
  }
  free(logit);
  free(choice);
}

/* ------------------------------------------------------------------ dispatch */

/* glm52/moe.rs:333-344: batch union in first-occurrence order */
size_t orc_unique_experts(const int32_t* ids, size_t s, size_t k, int32_t* uniq) {
  size_t n = 0;
  for (size_t q = 0; q < s * k; q++) {
    int32_t eid = ids[q];
    if (eid < 0) continue;
    int seen = 0;
    for (size_t u = 0; u < n; u++)
      if (uniq[u] == eid) {
        seen = 1;
        break;
      }
    if (!seen) uniq[n++] = eid;
  }
  return n;
}

/* glm52/moe.rs:465-470: ascending tokens that picked eid, with that slot's weight (first match) */
size_t orc_expert_rows(const int32_t* ids, const float* w, size_t s, size_t k, int32_t eid,
                       int32_t* rows, float* row_w) {
  size_t nr = 0;
  for (size_t si = 0; si < s; si++)
    for (size_t j = 0; j < k; j++)
      if (ids[si * k + j] == eid) {
        rows[nr] = (int32_t)si;
        row_w[nr] = w[si * k + j];
        nr++;
        break;
      }
  return nr;
}

/* ------------------------------------------------------------------ expert compute */

typedef void (*mxfp4_mm_fn)(float*, const float*, const uint8_t*, const uint8_t*, size_t,
                            size_t, size_t);

static void matmul_qt_with(mxfp4_mm_fn mx, float* y, const float* x, const uint8_t* data,
                           const void* scale, int fmt, size_t gs, size_t s, size_t i,
                           size_t o) {
  if (fmt == 0)
    mx(y, x, data, (const uint8_t*)scale, s, i, o);
  else
    orc_matmul_i4_grouped(y, x, data, (const float*)scale, gs, s, i, o);
}

/* glm52/moe.rs:463-513, GateUp::Separate + Activation::Silu */
static void apply_single_expert_with(mxfp4_mm_fn mx, const orc_expert* ex, int fmt, size_t gs,
                                     int32_t eid, const int32_t* ids, const float* w, size_t s,
                                     size_t k, const float* x, size_t d, size_t inter,
                                     float* out) {
  int32_t* rows = (int32_t*)malloc(s * sizeof(int32_t));
  float* rw = (float*)malloc(s * sizeof(float));
  size_t nr = orc_expert_rows(ids, w, s, k, eid, rows, rw);
  if (nr == 0) {
    free(rows);
    free(rw);
    return;
  }
  float* xg = (float*)malloc(nr * d * sizeof(float));
  for (size_t r = 0; r < nr; r++) memcpy(xg + r * d, x + (size_t)rows[r] * d, d * sizeof(float));
  float* gg = (float*)malloc(nr * inter * sizeof(float));
  float* uu = (float*)malloc(nr * inter * sizeof(float));
  matmul_qt_with(mx, gg, xg, ex->gate, ex->gate_scale, fmt, gs, nr, d, inter);
  matmul_qt_with(mx, uu, xg, ex->up, ex->up_scale, fmt, gs, nr, d, inter);
  for (size_t z = 0; z < nr * inter; z++) gg[z] = orc_siluf(gg[z]) * uu[z];
  float* hh = (float*)malloc(nr * d * sizeof(float));
  matmul_qt_with(mx, hh, gg, ex->down, ex->down_scale, fmt, gs, nr, inter, d);
  for (size_t r = 0; r < nr; r++) {
    float wg = rw[r];
    float* o = out + (size_t)rows[r] * d;
    for (size_t dd = 0; dd < d; dd++) o[dd] = o[dd] + wg * hh[r * d + dd];
  }
  free(hh);
  free(uu);
  free(gg);
  free(xg);
  free(rw);
  free(rows);
}

void orc_apply_single_expert(const orc_expert* ex, int fmt, size_t gs, int32_t eid,
                             const int32_t* ids, const float* w, size_t s, size_t k,
                             const float* x, size_t d, size_t inter, float* out) {
  apply_single_expert_with(orc_matmul_mxfp4, ex, fmt, gs, eid, ids, w, s, k, x, d, inter, out);
}

/* Shared SwiGLU expert -> hh[s,d] (qwen38/generate.rs:305-315, glm52/moe.rs:411-417). */
static void shared_expert(mxfp4_mm_fn mx, const orc_expert* sh, int fmt, size_t gs,
                          const float* x, size_t s, size_t d, size_t si_, float* hh) {
  float* sg = (float*)malloc(s * si_ * sizeof(float));
  float* su = (float*)malloc(s * si_ * sizeof(float));
  matmul_qt_with(mx, sg, x, sh->gate, sh->gate_scale, fmt, gs, s, d, si_);
  matmul_qt_with(mx, su, x, sh->up, sh->up_scale, fmt, gs, s, d, si_);
  for (size_t z = 0; z < s * si_; z++) sg[z] = orc_siluf(sg[z]) * su[z];
  matmul_qt_with(mx, hh, sg, sh->down, sh->down_scale, fmt, gs, s, si_, d);
  free(su);
  free(sg);
}

static void moe_forward_qwen_with(mxfp4_mm_fn mx, const float* x, size_t s, size_t d,
                                  size_t e, size_t k, size_t inter, size_t shared_inter,
                                  const float* router, const float* logit_bias,
                                  const orc_expert* experts, const orc_expert* shared,
                                  const float* shared_gate, int fmt, size_t gs, float* out,
                                  int32_t* ids_out, float* w_out) {
  size_t kk = k < e ? k : e;
  float* logits = (float*)malloc(s * e * sizeof(float));
  orc_matmul_f32(logits, x, router, s, d, e);
  if (logit_bias)
    for (size_t si = 0; si < s; si++)
      for (size_t j = 0; j < e; j++) logits[si * e + j] = logits[si * e + j] + logit_bias[j];
  int32_t* ids = (int32_t*)malloc(s * kk * sizeof(int32_t));
  float* w = (float*)malloc(s * kk * sizeof(float));
  for (size_t si = 0; si < s; si++) orc_qwen_route(logits + si * e, e, k, ids + si * kk, w + si * kk);
  memset(out, 0, s * d * sizeof(float));
  int32_t* uniq = (int32_t*)malloc((s * kk + 1) * sizeof(int32_t));
  size_t nu = orc_unique_experts(ids, s, kk, uniq);
  float* sh = NULL;
  if (shared) {
    sh = (float*)malloc(s * d * sizeof(float));
    shared_expert(mx, shared, fmt, gs, x, s, d, shared_inter, sh);
    if (shared_gate)
      for (size_t si = 0; si < s; si++) {
        float lg = RUST_SUM_INIT;
        for (size_t q = 0; q < d; q++) lg = lg + x[si * d + q] * shared_gate[q];
        float sc = orc_sigmoid(lg);
        for (size_t q = 0; q < d; q++) sh[si * d + q] = sh[si * d + q] * sc;
      }
  }
  for (size_t u = 0; u < nu; u++)
    apply_single_expert_with(mx, &experts[uniq[u]], fmt, gs, uniq[u], ids, w, s, kk, x, d,
                             inter, out);
  if (sh)
    for (size_t z = 0; z < s * d; z++) out[z] = out[z] + sh[z];
  if (ids_out) memcpy(ids_out, ids, s * kk * sizeof(int32_t));
  if (w_out) memcpy(w_out, w, s * kk * sizeof(float));
  free(sh);
  free(uniq);
  free(w);
  free(ids);
  free(logits);
}

void orc_moe_forward_qwen(const float* x, size_t s, size_t d, size_t e, size_t k,
                          size_t inter, size_t shared_inter, const float* router,
                          const float* logit_bias, const orc_expert* experts,
                          const orc_expert* shared, const float* shared_gate, int fmt,
                          size_t gs, float* out, int32_t* ids_out, float* w_out) {
  moe_forward_qwen_with(orc_matmul_mxfp4, x, s, d, e, k, inter, shared_inter, router,
                        logit_bias, experts, shared, shared_gate, fmt, gs, out, ids_out, w_out);
}

void orc_moe_forward_qwen_fast(const float* x, size_t s, size_t d, size_t e, size_t k,
                               size_t inter, size_t shared_inter, const float* router,
                               const float* logit_bias, const orc_expert* experts,
                               const orc_expert* shared, const float* shared_gate, float* out,
                               int32_t* ids_out, float* w_out) {
  moe_forward_qwen_with(orc_has_avx512() ? orc_matmul_mxfp4_avx512 : orc_matmul_mxfp4, x, s, d,
                        e, k, inter, shared_inter, router, logit_bias, experts, shared,
                        shared_gate, 0, 32, out, ids_out, w_out);
}

void orc_moe_glm(const float* x, size_t s, size_t d, size_t e, size_t k, size_t inter,
                 size_t shared_inter, const float* router, const float* bias, size_t n_group,
                 size_t topk_group, int norm_topk, float routed_scale,
                 const orc_expert* experts, const orc_expert* shared, int fmt, size_t gs,
                 float* out, int32_t* ids_out, float* w_out) {
  int32_t* ids = (int32_t*)malloc(s * k * sizeof(int32_t));
  float* w = (float*)malloc(s * k * sizeof(float));
  orc_glm_route(x, router, bias, s, d, e, k, n_group, topk_group, norm_topk, routed_scale, ids,
                w);
  memset(out, 0, s * d * sizeof(float));
  int32_t* uniq = (int32_t*)malloc((s * k + 1) * sizeof(int32_t));
  size_t nu = orc_unique_experts(ids, s, k, uniq);
  float* sh = NULL;
  if (shared) {
    sh = (float*)malloc(s * d * sizeof(float));
    shared_expert(orc_matmul_mxfp4, shared, fmt, gs, x, s, d, shared_inter, sh);
  }
  for (size_t u = 0; u < nu; u++)
    apply_single_expert_with(orc_matmul_mxfp4, &experts[uniq[u]], fmt, gs, uniq[u], ids, w, s,
                             k, x, d, inter, out);
  if (sh)
    for (size_t z = 0; z < s * d; z++) out[z] = out[z] + sh[z];
  if (ids_out) memcpy(ids_out, ids, s * k * sizeof(int32_t));
  if (w_out) memcpy(w_out, w, s * k * sizeof(float));
  free(sh);
  free(uniq);
  free(w);
  free(ids);
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
