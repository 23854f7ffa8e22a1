/*
 * TEST INFRASTRUCTURE ONLY — the parity oracle and the timed CPU baseline.
 *
 * A plain-C restatement of the reference CPU path for llambda's quantized FFN
 * (jrm-code-project/llambda, "L" = llambda.lisp).  The reference is Common
 * Lisp for SBCL with sb-simd AVX2 and lparallel; SBCL is not installed, and
 * the Lisp loads kernel32 at L3-6, so it cannot run here.  This file follows
 * its arithmetic step by step instead:
 *
 *   - single-precision products and differences are rounded one at a time
 *     (built with -ffp-contract=off), and only the reference's explicit
 *     f32.8 FMA (sb-simd fmadd) is an fmaf;
 *   - the Q4_K / Q6_K row dots keep eight lane accumulators exactly as the
 *     reference's f32.8 register does, and reduce them in lane order at the
 *     end (L4345-4350, L4453-4458);
 *   - rows of a Q4_K / Q6_K GEMV with at least 96 rows are split into
 *     min(rows, workers) contiguous parts on OpenMP threads, like lparallel
 *     pdotimes (L4600-4653, L806-817); every row is computed independently,
 *     so results do not depend on the worker count;
 *   - exp of a single-float is evaluated in double and rounded to single,
 *     as SBCL does, and silu/sigmoid then divide in double (L926-930).
 *
 * Parity is pinned by the reference's own known-answer tests (tests.lisp
 * T2257-2450, T298-344), reproduced in tests/test_oracle.py.
 */
#include "llambda_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../llambda_b200/csrc/synth.h"

#define OR_QK_K 256
#define OR_Q4K_BLOCK 144 /* 4 + 12 + 128, L2142 */
#define OR_Q6K_BLOCK 210 /* 2 + 16 + 192, L2144 */
#define OR_Q5K_BLOCK 176 /* 4 + 12 + 32 + 128, L2143 */
#define OR_Q5_0_BLOCK 22 /* 2 + 4 + 16, L2139 */
#define OR_Q8_0_BLOCK 34 /* 2 + 32, L2140 */

static __thread char or_error[512];
static int or_workers = 24; /* *gemv-worker-count*, L36 */
#define OR_MIN_PARALLEL_ROWS 96 /* *gemv-min-parallel-rows*, L37 */

static void or_fail(const char *fmt, const char *detail) {
  snprintf(or_error, sizeof(or_error), fmt, detail ? detail : "");
}

const char *or_last_error(void) { return or_error; }
void or_set_workers(int workers) { or_workers = workers > 0 ? workers : 1; }
int or_get_workers(void) { return or_workers; }

/* fp16-to-single-float, L716-733: subnormals are decoded exactly, exponent 31
 * (Inf/NaN) is an error. */
float or_fp16_to_f32(uint16_t bits, int *error) {
  int sign = (bits >> 15) & 1;
  int exponent = (bits >> 10) & 31;
  int fraction = bits & 1023;
  double v;
  if (exponent == 0) {
    if (fraction == 0) return sign ? -0.0f : 0.0f;
    v = ldexp(fraction / 1024.0, -14);
  } else if (exponent == 31) {
    if (error) *error = 1;
    snprintf(or_error, sizeof(or_error),
             "Unsupported fp16 special value: %x.", bits);
    return 0.0f;
  } else {
    v = ldexp(1.0 + fraction / 1024.0, exponent - 15);
  }
  return (float)(sign ? -v : v);
}

static float or_read_fp16(const uint8_t *p, int *error) {
  return or_fp16_to_f32((uint16_t)(p[0] | (p[1] << 8)), error);
}

/* get-scale-min-k4-at, L4316-4336 (same as get-scale-min-k4, L6794-6813). */
void or_get_scale_min_k4(const uint8_t *s, int j, int *scale, int *min) {
  if (j < 4) {
    *scale = s[j] & 63;
    *min = s[j + 4] & 63;
  } else {
    *scale = (s[j + 4] & 0x0F) | (((s[j - 4] & 0xC0) >> 6) << 4);
    *min = (s[j + 4] >> 4) | (((s[j] & 0xC0) >> 6) << 4);
  }
}

/* dequantize-q4-k-m, L6815-6859: w = d*sc*q - dmin*m, each step rounded. */
int or_dequantize_q4_k(const uint8_t *p, size_t count, float *out) {
  if (count % OR_QK_K) {
    or_fail("Q4_K_M dequantization requires ELEMENT-COUNT to be a multiple of 256.%s", 0);
    return -1;
  }
  for (size_t b = 0; b < count / OR_QK_K; ++b) {
    const uint8_t *blk = p + b * OR_Q4K_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err), dmin = or_read_fp16(blk + 2, &err);
    if (err) return -1;
    const uint8_t *scales = blk + 4, *qs = blk + 16;
    float *r = out + b * OR_QK_K;
    for (int chunk = 0; chunk < 4; ++chunk) {
      int sc0, m0, sc1, m1;
      or_get_scale_min_k4(scales, 2 * chunk, &sc0, &m0);
      or_get_scale_min_k4(scales, 2 * chunk + 1, &sc1, &m1);
      float delta0 = d * (float)sc0, offset0 = dmin * (float)m0;
      float delta1 = d * (float)sc1, offset1 = dmin * (float)m1;
      for (int lane = 0; lane < 32; ++lane) {
        int packed = qs[chunk * 32 + lane];
        float lo = delta0 * (float)(packed & 0x0F);
        float hi = delta1 * (float)(packed >> 4);
        r[chunk * 64 + lane] = lo - offset0;
        r[chunk * 64 + 32 + lane] = hi - offset1;
      }
    }
  }
  return 0;
}

/* dequantize-q6-k, L6919-6978: w = (d*sc)*q, q = 6-bit value - 32. */
int or_dequantize_q6_k(const uint8_t *p, size_t count, float *out) {
  if (count % OR_QK_K) {
    or_fail("Q6_K dequantization requires ELEMENT-COUNT to be a multiple of 256.%s", 0);
    return -1;
  }
  for (size_t b = 0; b < count / OR_QK_K; ++b) {
    const uint8_t *blk = p + b * OR_Q6K_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk + 208, &err);
    if (err) return -1;
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    float *r = out + b * OR_QK_K;
    for (int chunk = 0; chunk < 2; ++chunk) {
      for (int lane = 0; lane < 32; ++lane) {
        int is = lane / 16;
        int lo = ql[chunk * 64 + lane], hi = ql[chunk * 64 + 32 + lane];
        int top = qh[chunk * 32 + lane];
        int q1 = ((lo & 0x0F) | ((top & 3) << 4)) - 32;
        int q2 = ((hi & 0x0F) | (((top >> 2) & 3) << 4)) - 32;
        int q3 = ((lo >> 4) | (((top >> 4) & 3) << 4)) - 32;
        int q4 = ((hi >> 4) | (((top >> 6) & 3) << 4)) - 32;
        const int8_t *s = sc + chunk * 8 + is;
        r[chunk * 128 + lane] = (d * (float)s[0]) * (float)q1;
        r[chunk * 128 + 32 + lane] = (d * (float)s[2]) * (float)q2;
        r[chunk * 128 + 64 + lane] = (d * (float)s[4]) * (float)q3;
        r[chunk * 128 + 96 + lane] = (d * (float)s[6]) * (float)q4;
      }
    }
  }
  return 0;
}

/* f32.8-horizontal+ of the eight lane accumulators, in lane order. */
static float or_hsum8(const float *s) {
  float t = s[0];
  for (int i = 1; i < 8; ++i) t += s[i];
  return t;
}

/* dot-product-with-q4-k-m-tensor-data, L4338-4382, with the inner body of
 * expand-q4-k-body, L4145-4201: four 8-lane groups per sub-block pair, low
 * nibbles against x[0..31], high nibbles against x[32..63]. */
int or_dot_q4_k(const uint8_t *row, const float *x, size_t count, float *out) {
  if (count % OR_QK_K) {
    or_fail("Q4_K_M dot product requires ELEMENT-COUNT to be a multiple of 256.%s", 0);
    return -1;
  }
  float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t b = 0; b < count / OR_QK_K; ++b) {
    const uint8_t *blk = row + b * OR_Q4K_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err), dmin = or_read_fp16(blk + 2, &err);
    if (err) return -1;
    const uint8_t *scales = blk + 4, *qs = blk + 16;
    const float *xb = x + b * OR_QK_K;
    for (int pair = 0; pair < 4; ++pair) { /* accumulate-body (2p, 2p+1) */
      int sc0, m0, sc1, m1;
      or_get_scale_min_k4(scales, 2 * pair, &sc0, &m0);
      or_get_scale_min_k4(scales, 2 * pair + 1, &sc1, &m1);
      float delta0 = d * (float)sc0, offset0 = dmin * (float)m0;
      float delta1 = d * (float)sc1, offset1 = dmin * (float)m1;
      const uint8_t *q = qs + 32 * pair;
      const float *xv = xb + 64 * pair;
      for (int group = 0; group < 4; ++group) {
        int base = group * 8;
        for (int i = 0; i < 8; ++i) {
          int packed = q[base + i];
          float lw = (float)(packed & 0x0F) * delta0;
          float hw = (float)(packed >> 4) * delta1;
          lw = lw - offset0;
          hw = hw - offset1;
          sum[i] = fmaf(hw, xv[32 + base + i], fmaf(lw, xv[base + i], sum[i]));
        }
      }
    }
  }
  *out = or_hsum8(sum);
  return 0;
}

/* One Q5_K value (dot-product-with-q5-k-tensor-data, L4418-4423;
 * dequantize-q5-k, L6900-6911): in sub-block pair `group` (values
 * 64*group .. +63), lane l's low nibble of qs[32*group + l] with qh bit
 * 2*group is value l, its high nibble with qh bit 2*group + 1 is value 32 + l. */
static int or_q5_k_value(const uint8_t *qh, const uint8_t *qs, int group, int lane, int high) {
  const int packed = qs[32 * group + lane], bits = qh[lane];
  const int u = 1 << (2 * group + high);
  return (high ? (packed >> 4) : (packed & 0x0F)) + ((bits & u) ? 16 : 0);
}

/* dequantize-q5-k, L6861-6917: w = d*sc*q - dmin*m, each step rounded. */
int or_dequantize_q5_k(const uint8_t *p, size_t count, float *out) {
  if (count % OR_QK_K) {
    or_fail("Q5_K dequantization requires ELEMENT-COUNT to be a multiple of 256.%s", 0);
    return -1;
  }
  for (size_t b = 0; b < count / OR_QK_K; ++b) {
    const uint8_t *blk = p + b * OR_Q5K_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err), dmin = or_read_fp16(blk + 2, &err);
    if (err) return -1;
    const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
    float *r = out + b * OR_QK_K;
    for (int group = 0; group < 4; ++group) {
      int sc0, m0, sc1, m1;
      or_get_scale_min_k4(scales, 2 * group, &sc0, &m0);
      or_get_scale_min_k4(scales, 2 * group + 1, &sc1, &m1);
      float delta0 = d * (float)sc0, offset0 = dmin * (float)m0;
      float delta1 = d * (float)sc1, offset1 = dmin * (float)m1;
      for (int lane = 0; lane < 32; ++lane) {
        float lo = delta0 * (float)or_q5_k_value(qh, qs, group, lane, 0);
        float hi = delta1 * (float)or_q5_k_value(qh, qs, group, lane, 1);
        r[group * 64 + lane] = lo - offset0;
        r[group * 64 + 32 + lane] = hi - offset1;
      }
    }
  }
  return 0;
}

/* dot-product-with-q5-k-tensor-data, L4387-4441: one single-float sum over
 * the row, in order: for each sub-block pair, for each lane, the low value's
 * product then the high value's, every multiply, subtract and add rounded on
 * its own (no FMA: the reference's scalar loop, not an f32.8 one). */
int or_dot_q5_k(const uint8_t *row, const float *x, size_t count, float *out) {
  if (count % OR_QK_K) {
    or_fail("Q5_K dot product requires ELEMENT-COUNT to be a multiple of 256.%s", 0);
    return -1;
  }
  float sum = 0.0f;
  for (size_t b = 0; b < count / OR_QK_K; ++b) {
    const uint8_t *blk = row + b * OR_Q5K_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err), dmin = or_read_fp16(blk + 2, &err);
    if (err) return -1;
    const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
    const float *xb = x + b * OR_QK_K;
    for (int group = 0; group < 4; ++group) {
      int sc0, m0, sc1, m1;
      or_get_scale_min_k4(scales, 2 * group, &sc0, &m0);
      or_get_scale_min_k4(scales, 2 * group + 1, &sc1, &m1);
      float delta0 = d * (float)sc0, offset0 = dmin * (float)m0;
      float delta1 = d * (float)sc1, offset1 = dmin * (float)m1;
      for (int lane = 0; lane < 32; ++lane) {
        float w0 = delta0 * (float)or_q5_k_value(qh, qs, group, lane, 0);
        float w1 = delta1 * (float)or_q5_k_value(qh, qs, group, lane, 1);
        w0 = w0 - offset0;
        w1 = w1 - offset1;
        float p0 = xb[64 * group + lane] * w0;
        sum = sum + p0;
        float p1 = xb[64 * group + 32 + lane] * w1;
        sum = sum + p1;
      }
    }
  }
  *out = sum;
  return 0;
}

/* dot-product-with-q6-k-tensor-data, L4446-4506, with expand-q6-k-group,
 * L4203-4310, and the q6-quant-1..4 bit extraction, L4115-4137. */
int or_dot_q6_k(const uint8_t *row, const float *x, size_t count, float *out) {
  if (count % OR_QK_K) {
    or_fail("Q6_K dot product requires ELEMENT-COUNT to be a multiple of 256.%s", 0);
    return -1;
  }
  float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (size_t b = 0; b < count / OR_QK_K; ++b) {
    const uint8_t *blk = row + b * OR_Q6K_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk + 208, &err);
    if (err) return -1;
    for (int chunk = 0; chunk < 2; ++chunk) {
      const uint8_t *ql = blk + chunk * 64, *qh = blk + 128 + chunk * 32;
      const int8_t *sc = (const int8_t *)(blk + 192 + chunk * 8);
      const float *xv = x + b * OR_QK_K + chunk * 128;
      for (int half = 0; half < 2; ++half) { /* start-lane 0 then 16 */
        float d1 = d * (float)sc[half + 0], d2 = d * (float)sc[half + 2];
        float d3 = d * (float)sc[half + 4], d4 = d * (float)sc[half + 6];
        for (int group = 0; group < 2; ++group) {
          int base = half * 16 + group * 8;
          for (int i = 0; i < 8; ++i) {
            int lo = ql[base + i], hi = ql[32 + base + i], top = qh[base + i];
            float w1 = (float)(((lo & 0x0F) | ((top & 3) << 4)) - 32) * d1;
            float w2 = (float)(((hi & 0x0F) | (((top >> 2) & 3) << 4)) - 32) * d2;
            float w3 = (float)(((lo >> 4) | (((top >> 4) & 3) << 4)) - 32) * d3;
            float w4 = (float)(((hi >> 4) | (((top >> 6) & 3) << 4)) - 32) * d4;
            float s = fmaf(w1, xv[base + i], sum[i]);
            s = fmaf(w2, xv[32 + base + i], s);
            s = fmaf(w3, xv[64 + base + i], s);
            sum[i] = fmaf(w4, xv[96 + base + i], s);
          }
        }
      }
    }
  }
  *out = or_hsum8(sum);
  return 0;
}

/* dot-product-with-f32-tensor-data, L4096-4107: sequential, unfused. */
/* The 5-bit value of position j (0..31) of a Q5_0 block: nibble j (low) or
 * j-16 (high) of qs, bit j of qh as bit 4, minus 16 (L3978-3983). */
static int or_q5_0_value(const uint8_t *blk, uint32_t qh, int j) {
  int packed = blk[6 + (j & 15)];
  int nib = j < 16 ? (packed & 0x0F) : (packed >> 4);
  return (nib | (((qh >> j) & 1) << 4)) - 16;
}

static uint32_t or_read_u32(const uint8_t *p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* dequantize-q5-0, L3965-3990: w = d * q, rounded once. */
int or_dequantize_q5_0(const uint8_t *p, size_t count, float *out) {
  if (count % 32) {
    or_fail("Q5_0 dequantization requires ELEMENT-COUNT to be a multiple of 32.%s", 0);
    return -1;
  }
  for (size_t b = 0; b < count / 32; ++b) {
    const uint8_t *blk = p + b * OR_Q5_0_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err);
    if (err) return -1;
    uint32_t qh = or_read_u32(blk + 2);
    for (int j = 0; j < 32; ++j) out[b * 32 + j] = d * (float)or_q5_0_value(blk, qh, j);
  }
  return 0;
}

/* dequantize-q8-0, L3992-4009: w = d * q (signed bytes). */
int or_dequantize_q8_0(const uint8_t *p, size_t count, float *out) {
  if (count % 32) {
    or_fail("Q8_0 dequantization requires ELEMENT-COUNT to be a multiple of 32.%s", 0);
    return -1;
  }
  for (size_t b = 0; b < count / 32; ++b) {
    const uint8_t *blk = p + b * OR_Q8_0_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err);
    if (err) return -1;
    for (int j = 0; j < 32; ++j) out[b * 32 + j] = d * (float)(int8_t)blk[2 + j];
  }
  return 0;
}

/* dot-product-with-q5-0-tensor-data, L4037-4068: per pair j of a block,
 * sum += d * (q0 * x[j] + q1 * x[16 + j]), single-float steps in order. */
int or_dot_q5_0(const uint8_t *row, const float *x, size_t count, float *out) {
  if (count % 32) {
    or_fail("Q5_0 dot product requires ELEMENT-COUNT to be a multiple of 32.%s", 0);
    return -1;
  }
  float sum = 0.0f;
  for (size_t b = 0; b < count / 32; ++b) {
    const uint8_t *blk = row + b * OR_Q5_0_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err);
    if (err) return -1;
    uint32_t qh = or_read_u32(blk + 2);
    const float *xb = x + b * 32;
    for (int j = 0; j < 16; ++j) {
      float p0 = (float)or_q5_0_value(blk, qh, j) * xb[j];
      float p1 = (float)or_q5_0_value(blk, qh, j + 16) * xb[16 + j];
      float pair = p0 + p1;
      float term = d * pair;
      sum = sum + term;
    }
  }
  *out = sum;
  return 0;
}

/* dot-product-with-q8-0-tensor-data, L4070-4094: sum += (d * q) * x[j]. */
int or_dot_q8_0(const uint8_t *row, const float *x, size_t count, float *out) {
  if (count % 32) {
    or_fail("Q8_0 dot product requires ELEMENT-COUNT to be a multiple of 32.%s", 0);
    return -1;
  }
  float sum = 0.0f;
  for (size_t b = 0; b < count / 32; ++b) {
    const uint8_t *blk = row + b * OR_Q8_0_BLOCK;
    int err = 0;
    float d = or_read_fp16(blk, &err);
    if (err) return -1;
    const float *xb = x + b * 32;
    for (int j = 0; j < 32; ++j) {
      float dq = d * (float)(int8_t)blk[2 + j];
      float term = dq * xb[j];
      sum = sum + term;
    }
  }
  *out = sum;
  return 0;
}

float or_dot_f32(const float *row, const float *x, size_t count) {
  float sum = 0.0f;
  for (size_t i = 0; i < count; ++i) {
    float p = x[i] * row[i];
    sum = sum + p;
  }
  return sum;
}

/* dot-product, L3491-3500. */
float or_dot_product(const float *a, const float *b, size_t count) {
  float sum = 0.0f;
  for (size_t i = 0; i < count; ++i) {
    float p = a[i] * b[i];
    sum = sum + p;
  }
  return sum;
}

/* tensor-row-byte-size via ggml-tensor-byte-size, L2147-2155, L3397-3400. */
size_t or_row_bytes(int type, size_t columns) {
  switch (type) {
    case OR_TYPE_F32: return columns * 4;
    case OR_TYPE_Q4_K: return columns % OR_QK_K ? 0 : columns / OR_QK_K * OR_Q4K_BLOCK;
    case OR_TYPE_Q6_K: return columns % OR_QK_K ? 0 : columns / OR_QK_K * OR_Q6K_BLOCK;
    case OR_TYPE_Q5_K: return columns % OR_QK_K ? 0 : columns / OR_QK_K * OR_Q5K_BLOCK;
    case OR_TYPE_Q5_0: return columns % 32 ? 0 : columns / 32 * OR_Q5_0_BLOCK;
    case OR_TYPE_Q8_0: return columns % 32 ? 0 : columns / 32 * OR_Q8_0_BLOCK;
    default: return 0;
  }
}

/* %gguf-model-matrix-vector-multiply-into, L4542-4658: rows
 * [start_row, start_row + row_count) of the flattened tensor. */
int or_gemv(const or_tensor *t, size_t start_row, size_t row_count,
            const float *x, float *y) {
  size_t cols = t->ne0;
  size_t flat_rows = t->ne1 * (t->ne2 ? t->ne2 : 1);
  size_t rb = or_row_bytes(t->type, cols);
  if (!rb) {
    or_fail("Unsupported tensor type or column count for GEMV.%s", 0);
    return -1;
  }
  if (start_row + row_count > flat_rows) {
    or_fail("Requested row range exceeds flattened row count.%s", 0);
    return -1;
  }
  const uint8_t *base = (const uint8_t *)t->data + start_row * rb;
  if (t->type == OR_TYPE_F32) {
    for (size_t r = 0; r < row_count; ++r)
      y[r] = or_dot_f32((const float *)(base + r * rb), x, cols);
    return 0;
  }
  if (t->type == OR_TYPE_Q5_0 || t->type == OR_TYPE_Q8_0) { /* sequential rows, L4582-4593 */
    for (size_t r = 0; r < row_count; ++r) {
      int rc = t->type == OR_TYPE_Q5_0 ? or_dot_q5_0(base + r * rb, x, cols, &y[r])
                                       : or_dot_q8_0(base + r * rb, x, cols, &y[r]);
      if (rc) return -1;
    }
    return 0;
  }
  int failed = 0;
  int parts = row_count >= OR_MIN_PARALLEL_ROWS
                  ? (int)(row_count < (size_t)or_workers ? row_count : (size_t)or_workers)
                  : 1;
  long n = (long)row_count;
#pragma omp parallel for num_threads(parts) schedule(static) reduction(| : failed)
  for (long r = 0; r < n; ++r) {
    /* Q4_K, Q5_K and Q6_K rows split over the workers (L4600-4650) */
    int rc = t->type == OR_TYPE_Q4_K   ? or_dot_q4_k(base + r * rb, x, cols, &y[r])
             : t->type == OR_TYPE_Q5_K ? or_dot_q5_k(base + r * rb, x, cols, &y[r])
                                       : or_dot_q6_k(base + r * rb, x, cols, &y[r]);
    failed |= rc != 0;
  }
  if (failed) { /* worker threads keep their own error text */
    or_fail("Unsupported fp16 special value in tensor data.%s", 0);
    return -1;
  }
  return 0;
}

/* select-top-k-logits-into, L5265-5292: insertion, strict >, so ties keep
 * the lower index first; output in rank order. */
void or_select_top_k(const float *logits, size_t count, int k,
                     int32_t *top_indices, float *top_logits) {
  for (int i = 0; i < k; ++i) {
    top_indices[i] = -1;
    top_logits[i] = -3.40282347e38f; /* most-negative-single-float */
  }
  for (size_t li = 0; li < count; ++li) {
    float v = logits[li];
    if (v > top_logits[k - 1]) {
      int at = k - 1;
      while (at > 0 && v > top_logits[at - 1]) {
        top_logits[at] = top_logits[at - 1];
        top_indices[at] = top_indices[at - 1];
        --at;
      }
      top_logits[at] = v;
      top_indices[at] = (int32_t)li;
    }
  }
}

/* exp of a single-float: evaluated in double, rounded to single (SBCL). */
static float or_exp_single(float v) { return (float)exp((double)v); }

/* sigmoid, L929-930. */
float or_sigmoid(float v) {
  return (float)(1.0 / (1.0 + (double)or_exp_single(-v)));
}

/* silu, L926-927. */
float or_silu(float v) {
  return (float)((double)v / (1.0 + (double)or_exp_single(-v)));
}

/* relu-squared, L938-940. */
float or_relu_squared(float v) {
  float x = v > 0.0f ? v : 0.0f;
  return x * x;
}

/* rms-norm-into, L859-879 (sum-square-elements, L819-829): sequential sum of
 * squares, scale = 1/sqrt(mean + eps), dest = (x * w) * scale. */
void or_rms_norm(const float *x, const float *w, size_t n, float eps, float *out) {
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float sq = x[i] * x[i];
    sum = sum + sq;
  }
  float ms = sum / (float)n;
  float scale = 1.0f / sqrtf(ms + eps);
  for (size_t i = 0; i < n; ++i) {
    float p = x[i] * w[i];
    out[i] = p * scale;
  }
}

/* GEMV of expert `e` (gguf-model-expert-matrix-vector-multiply-into,
 * L4951-4971) or of a plain 2-D tensor (e < 0).  An input shorter than the
 * tensor's row width is zero-padded: K-quant rows need a multiple of 256
 * columns, and the benchmark's Nemotron shapes are padded that way. */
static int or_project(const or_tensor *t, int e, const float *x, size_t n,
                      float *pad, float *y) {
  const float *in = x;
  if (n != t->ne0) {
    if (n > t->ne0) {
      or_fail("Vector length does not match tensor row width.%s", 0);
      return -1;
    }
    memcpy(pad, x, n * sizeof(float));
    memset(pad + n, 0, (t->ne0 - n) * sizeof(float));
    in = pad;
  }
  if (e >= 0) {
    if ((size_t)e >= (t->ne2 ? t->ne2 : 1)) {
      or_fail("Expert index is out of range.%s", 0);
      return -1;
    }
    return or_gemv(t, (size_t)e * t->ne1, t->ne1, in, y);
  }
  return or_gemv(t, 0, t->ne1, in, y);
}

/* vector-add-scaled-in-place, L3465-3477: dest += scale * src, unfused. */
static void or_add_scaled(float *dest, const float *src, size_t n, float s) {
  for (size_t i = 0; i < n; ++i) {
    float p = s * src[i];
    dest[i] = dest[i] + p;
  }
}

static size_t or_max(size_t a, size_t b) { return a > b ? a : b; }

/* qwen3next-moe-into, L5321-5426 (routed part L5354-5409, shared expert
 * L5410-5426), and nemotron-h-moe-ffn-into, L5827-5949, with its optional
 * latent projections: the experts run on latent_down . x (L5845-5855,
 * L5883-5887), their weighted sum has the latent width, and latent_up maps
 * it back to the hidden size before the shared expert is added (L5933-5938);
 * the router and the shared expert see x itself.  Tokens are independent
 * calls, as in the reference.  selected/weights (optional) receive the top-k
 * indices and final weights. */
int or_moe_forward(const or_moe_layer *L, const float *x, size_t tokens,
                   float *out, int32_t *selected, float *weights) {
  size_t H = L->hidden;
  size_t E = L->router.ne1;
  int k = L->top_k < (int)E ? L->top_k : (int)E;
  size_t inter = L->up_exps.ne1, inter_sh = L->up_shexp.data ? L->up_shexp.ne1 : 0;
  const int latent = L->arch == 1 && L->latent_down.data && L->latent_up.data;
  size_t LD = latent ? L->latent_down.ne1 : H; /* the experts' input and output width */
  size_t width = or_max(or_max(H, inter), inter_sh);
  width = or_max(width, or_max(L->up_exps.ne0, L->down_exps.ne0));
  if (L->up_shexp.data) width = or_max(width, or_max(L->up_shexp.ne0, L->down_shexp.ne0));
  if (latent) width = or_max(width, or_max(L->latent_down.ne0, L->latent_up.ne0));
  float *logits = malloc(E * sizeof(float));
  float *pad = malloc(width * sizeof(float));
  float *gate = malloc(width * sizeof(float));
  float *up = malloc(width * sizeof(float));
  float *down = malloc(width * sizeof(float));
  int32_t *ti = malloc((size_t)k * sizeof(int32_t));
  float *tl = malloc((size_t)k * sizeof(float));
  float *tw = malloc((size_t)k * sizeof(float));
  float *xn = malloc(H * sizeof(float));
  float *xe = malloc(width * sizeof(float)); /* expert input (latent) */
  float *mo = malloc(width * sizeof(float)); /* routed sum (latent) */
  int rc = -1;
  if (!logits || !pad || !gate || !up || !down || !ti || !tl || !tw || !xn || !xe || !mo) {
    or_fail("Out of memory.%s", 0);
    goto done;
  }
  for (size_t t = 0; t < tokens; ++t) {
    const float *xt = x + t * H;
    float *dest = out + t * H;
    if (L->input_norm) { /* rms-norm-into ffn-input, L5739-5744 */
      or_rms_norm(xt, L->input_norm, H, L->norm_epsilon, xn);
      xt = xn;
    }
    memset(dest, 0, H * sizeof(float));
    /* the experts' input: latent_down . x (L5883-5887), else x */
    const float *xin = xt;
    float *acc = dest;
    if (latent) {
      if (or_project(&L->latent_down, -1, xt, H, pad, xe)) goto done;
      xin = xe;
      memset(mo, 0, LD * sizeof(float));
      acc = mo;
    }
    if (or_gemv(&L->router, 0, E, xt, logits)) goto done;
    if (L->arch == 1 && L->router_bias) /* vector-add-bias-in-place, L5892 */
      for (size_t i = 0; i < E; ++i) logits[i] = logits[i] + L->router_bias[i];
    or_select_top_k(logits, E, k, ti, tl);
    float weight_sum = 0.0f;
    for (int i = 0; i < k; ++i) {
      tw[i] = or_sigmoid(tl[i]);
      weight_sum = weight_sum + tw[i];
    }
    if (L->arch == 0 || L->weights_norm) {
      if (!(weight_sum > 0.0f)) {
        or_fail("MoE router produced non-positive top-k weight sum.%s", 0);
        goto done;
      }
      for (int i = 0; i < k; ++i) tw[i] = tw[i] / weight_sum;
    }
    if (L->arch == 1)
      for (int i = 0; i < k; ++i) tw[i] = L->weight_scale * tw[i];
    for (int i = 0; i < k; ++i) {
      int e = ti[i];
      if (L->arch == 0) {
        if (or_project(&L->gate_exps, e, xt, H, pad, gate)) goto done;
        if (or_project(&L->up_exps, e, xt, H, pad, up)) goto done;
        for (size_t j = 0; j < inter; ++j) gate[j] = or_silu(gate[j]);
        for (size_t j = 0; j < inter; ++j) gate[j] = gate[j] * up[j];
      } else {
        if (or_project(&L->up_exps, e, xin, LD, pad, gate)) goto done;
        for (size_t j = 0; j < inter; ++j) gate[j] = or_relu_squared(gate[j]);
      }
      if (or_project(&L->down_exps, e, gate, inter, pad, down)) goto done;
      or_add_scaled(acc, down, LD, tw[i]);
    }
    if (latent) /* dest = latent_up . moe-output (L5933-5938) */
      if (or_project(&L->latent_up, -1, mo, LD, pad, dest)) goto done;
    if (L->arch == 0 && L->up_shexp.data) {
      float sw = or_sigmoid(or_dot_product(L->shared_gate_inp, xt, H));
      if (or_project(&L->gate_shexp, -1, xt, H, pad, gate)) goto done;
      if (or_project(&L->up_shexp, -1, xt, H, pad, up)) goto done;
      for (size_t j = 0; j < inter_sh; ++j) gate[j] = or_silu(gate[j]);
      for (size_t j = 0; j < inter_sh; ++j) gate[j] = gate[j] * up[j];
      if (or_project(&L->down_shexp, -1, gate, inter_sh, pad, down)) goto done;
      or_add_scaled(dest, down, H, sw);
    } else if (L->arch == 1 && L->up_shexp.data && L->down_shexp.data) {
      if (or_project(&L->up_shexp, -1, xt, H, pad, up)) goto done;
      for (size_t j = 0; j < inter_sh; ++j) up[j] = or_relu_squared(up[j]);
      if (or_project(&L->down_shexp, -1, up, inter_sh, pad, down)) goto done;
      for (size_t j = 0; j < H; ++j) dest[j] = dest[j] + down[j];
    }
    if (L->add_residual) /* vector-add-into x x ffn-output, L5746 */
      for (size_t j = 0; j < H; ++j) dest[j] = x[t * H + j] + dest[j];
    if (selected) memcpy(selected + t * (size_t)k, ti, (size_t)k * sizeof(int32_t));
    if (weights) memcpy(weights + t * (size_t)k, tw, (size_t)k * sizeof(float));
  }
  rc = 0;
done:
  free(logits); free(pad); free(gate); free(up); free(down);
  free(ti); free(tl); free(tw); free(xn); free(xe); free(mo);
  return rc;
}

void or_synth_q4k(uint64_t seed, uint64_t stream, uint64_t first_block,
                  size_t blocks, float dscale, uint8_t *out) {
  float s = lb_sigma_scale(dscale);
  long n = (long)blocks;
#pragma omp parallel for schedule(static)
  for (long b = 0; b < n; ++b)
    lb_q4k_block(seed, stream, first_block + b, s, out + b * OR_Q4K_BLOCK);
}

void or_synth_q6k(uint64_t seed, uint64_t stream, uint64_t first_block,
                  size_t blocks, float dscale, uint8_t *out) {
  float s = lb_sigma_scale(dscale);
  long n = (long)blocks;
#pragma omp parallel for schedule(static)
  for (long b = 0; b < n; ++b)
    lb_q6k_block(seed, stream, first_block + b, s, out + b * OR_Q6K_BLOCK);
}

void or_synth_f32(uint64_t seed, uint64_t stream, uint64_t first, size_t count,
                  float sigma, float *out) {
  float s = lb_sigma_scale(sigma);
  long n = (long)count;
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; ++i) out[i] = lb_f32_value(seed, stream, first + (size_t)i, s);
}

uint16_t or_f32_to_f16(float f) { return lb_f32_to_f16_rne(f); }
