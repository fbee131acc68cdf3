/*
 * apx_oracle.c — CPU restatement of apeiron's integer Q8-activation projection.
 *
 * TEST INFRASTRUCTURE ONLY (see apx_oracle.h).  The product library never links it.
 *
 * Two independent restatements live here, as in the reference:
 *   - the contract: row dequantization to Q32.32 and an exact checked i128 dot
 *     (`matvec_fixed`, src/engine/ops/matvec.rs:86-222);
 *   - the fused row kernel: per 32-lane group `acc += S_b*(w_scale*D - w_min*sum(xq))`
 *     (`matvec_q8act`, src/engine/chart/mod.rs:497-1013, 1645-1925).
 * tests/test_oracle_golden.py checks them against each other and against the reference's
 * known-answer values.  Paths in comments are relative to the apeiron source tree.
 */
#include "apx_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

typedef __int128 i128;
typedef unsigned __int128 u128;

#define I128_MAX ((i128)(((u128)1 << 127) - 1))
#define ACT_QK 32
#define QK_K 256
#define Q8_0_BYTES 34
#define Q4_K_BYTES 144
#define Q6_K_BYTES 210

static int fail(apx_err *e, int code) {
  if (e) {
    memset(e, 0, sizeof *e);
    e->code = code;
  }
  return code;
}

static void clear(apx_err *e) {
  if (e) memset(e, 0, sizeof *e);
}

/* round_shift_32 (src/engine/num/value.rs:10-12): floor((v + 2^31) / 2^32), evaluated as
 * q + [r >= 2^31] with v = q*2^32 + r so the add cannot leave i128. */
static i128 rs32(i128 v) {
  i128 q = v >> 32;
  uint64_t r = (uint64_t)v & 0xFFFFFFFFull;
  return q + (r >= 0x80000000ull ? 1 : 0);
}

void apxo_round_shift_32(int64_t hi, uint64_t lo, int64_t *out_hi, uint64_t *out_lo) {
  i128 v = ((i128)hi << 64) | (i128)lo;
  i128 r = rs32(v);
  *out_hi = (int64_t)(r >> 64);
  *out_lo = (uint64_t)r;
}

/* `round_to_i64` (chart/mod.rs:1746-1753): the rounded value when it fits i64. */
static int round_to_i64(i128 acc, int64_t *out) {
  i128 r = rs32(acc);
  if (r > (i128)INT64_MAX || r < (i128)INT64_MIN) return 1;
  *out = (int64_t)r;
  return 0;
}

/* f16_to_fixed (src/engine/num/dequant.rs:25-42). */
int apxo_f16_to_fixed(uint16_t h, int64_t *out) {
  uint16_t sign = h >> 15, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  int64_t mag;
  if (e == 0) {
    mag = (int64_t)m << 8;
  } else if (e == 0x1f) {
    return APX_ERR_NONFINITE_SCALE;
  } else {
    mag = ((int64_t)m + 1024) << (e + 7);
  }
  *out = sign ? -mag : mag;
  return 0;
}

/* f16_split (src/engine/kern/pow2.rs:52-64). */
int apxo_f16_split(uint16_t h, int32_t *m, uint32_t *k) {
  uint32_t e = (h >> 10) & 0x1f;
  int32_t f = (int32_t)(h & 0x3ff);
  if (e == 31) return 1;
  int32_t mm = e == 0 ? f : f + 1024;
  uint32_t kk = e == 0 ? 8 : e + 7;
  *m = (h >> 15) ? -mm : mm;
  *k = kk;
  return 0;
}

/* act_scale (src/engine/kern/pow2.rs:22-39). */
int apxo_act_scale(uint64_t absmax, uint64_t *s_out) {
  if (absmax == 0) {
    *s_out = 0;
    return 0;
  }
  uint64_t need = absmax / 127 + (absmax % 127 != 0);
  uint64_t s = 1;
  uint32_t steps = 0;
  while (s < need && steps < 62) {
    s *= 2;
    steps++;
  }
  if (s < need) return 1;
  *s_out = s;
  return 0;
}

/* finish (src/engine/kern/pow2.rs:76-96). */
int apxo_finish(int64_t acc, uint32_t s, int64_t *out) {
  i128 wide = acc, v;
  if (s >= 32) {
    uint32_t up = s - 32;
    if (acc == 0) {
      v = 0;
    } else if (up > 63) {
      return 1;
    } else {
      /* wide * 2^up with up <= 63 fits i128 for any i64 wide. */
      v = wide * ((i128)1 << up);
    }
  } else {
    uint32_t down = 32 - s;
    v = (wide + ((i128)1 << (down - 1))) >> down;
  }
  if (v < (i128)INT64_MIN || v > (i128)INT64_MAX) return 1;
  *out = (int64_t)v;
  return 0;
}

/* F32::to_q32 (src/engine/num/fp.rs:186-230) behind f32_to_fixed (f32_convert.rs:44-49):
 * round(v * 2^32) with ties away from zero; None for NaN/Inf or outside [-2^63, 2^63). */
int apxo_f32_to_q32(uint32_t bits, int64_t *out) {
  uint32_t e = (bits >> 23) & 0xff;
  if (e == 0xff) return 1;
  uint32_t frac = bits & 0x007fffff;
  uint64_t m = e == 0 ? frac : (frac | 0x00800000u);
  int neg = (bits & 0x80000000u) != 0;
  uint32_t ee = e == 0 ? 1 : e;
  u128 mag;
  if (ee >= 118) {
    uint32_t k = ee - 118;
    if (k > 40) return 1;
    mag = (u128)m << k;
  } else {
    uint32_t sh = 118 - ee;
    if (sh > 24)
      mag = 0;
    else
      mag = (u128)((m + (1ull << (sh - 1))) >> sh);
  }
  u128 lim = (u128)1 << 63;
  if (neg) {
    if (mag > lim) return 1;
    if (mag == lim) {
      *out = INT64_MIN;
      return 0;
    }
    *out = -(int64_t)mag;
    return 0;
  }
  if (mag >= lim) return 1;
  *out = (int64_t)mag;
  return 0;
}

/* QuantAct::dequantizes (chart/mod.rs:124-146). */
static int dequantizes(const int8_t *codes, size_t n, const int64_t *scales) {
  size_t nb = (n + ACT_QK - 1) / ACT_QK;
  for (size_t b = 0; b < nb; b++) {
    int64_t p;
    if (__builtin_mul_overflow(scales[b], (int64_t)127, &p)) {
      size_t end = (b + 1) * ACT_QK < n ? (b + 1) * ACT_QK : n;
      for (size_t l = b * ACT_QK; l < end; l++)
        if (__builtin_mul_overflow(scales[b], (int64_t)codes[l], &p)) return 0;
    }
  }
  return 1;
}

/* quant_act (src/engine/chart/mod.rs:258-334). */
int apxo_quant_act(const int64_t *x, size_t n, int8_t *codes, int64_t *scales) {
  size_t blocks = (n + ACT_QK - 1) / ACT_QK;
  for (size_t b = 0; b < blocks; b++) {
    size_t base = b * ACT_QK;
    size_t take = n - base < ACT_QK ? n - base : ACT_QK;
    uint64_t absmax = 0;
    for (size_t l = 0; l < take; l++) {
      int64_t v = x[base + l];
      uint64_t mag = v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v;
      if (mag > absmax) absmax = mag;
    }
    uint64_t s;
    if (apxo_act_scale(absmax, &s)) s = UINT64_MAX;
    if (s > (uint64_t)INT64_MAX) return 1;
    scales[b] = (int64_t)s;
    for (size_t l = 0; l < take; l++) {
      int64_t v = x[base + l];
      int8_t code = 0;
      if (s != 0) {
        uint64_t m = v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v;
        uint32_t shift = (uint32_t)__builtin_ctzll(s);
        uint64_t q = m >> shift, r = m & (s - 1);
        uint64_t mag = q + (2 * r >= s ? 1 : 0);
        if (mag > 127) return 1;
        code = (int8_t)(v < 0 ? -(int64_t)mag : (int64_t)mag);
      }
      codes[base + l] = code;
    }
  }
  if (!dequantizes(codes, n, scales)) return 1;
  return 0;
}

/* QuantAct::dequant (chart/mod.rs:188-212). */
int apxo_dequant_act(const int8_t *codes, size_t n, const int64_t *scales,
                     size_t n_scales, int64_t *out) {
  for (size_t i = 0; i < n; i++) {
    if (i / ACT_QK >= n_scales) return 1;
    if (__builtin_mul_overflow(scales[i / ACT_QK], (int64_t)codes[i], &out[i])) return 1;
  }
  return 0;
}

/* block_geom (src/format/quant.rs:129-148), restricted to the served families. */
static int geom(uint32_t t, size_t *qk, size_t *bb) {
  switch (t) {
    case APX_GGML_TYPE_Q8_0: *qk = 32; *bb = Q8_0_BYTES; return 1;
    case APX_GGML_TYPE_Q5_0: *qk = 32; *bb = 22; return 1;
    case APX_GGML_TYPE_Q4_K: *qk = QK_K; *bb = Q4_K_BYTES; return 1;
    case APX_GGML_TYPE_Q6_K: *qk = QK_K; *bb = Q6_K_BYTES; return 1;
    default: return 0;
  }
}

/* fused_type (src/engine/ops/fused.rs): the families with a fused row kernel. */
static int fused_type(uint32_t t) {
  return t == 8 || t == 6 || t == 10 || t == 11 || t == 12 || t == 14;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static int nonfinite(apx_err *err, uint16_t bits) {
  fail(err, APX_ERR_NONFINITE_SCALE);
  if (err) err->bits = bits;
  return APX_ERR_NONFINITE_SCALE;
}

/* get_scale_min_k4 (src/format/quant.rs:482-491). */
static void q4k_scale_min(const uint8_t *sc, int j, int *s, int *m) {
  if (j < 4) {
    *s = sc[j] & 63;
    *m = sc[j + 4] & 63;
  } else {
    *s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
    *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
}

/* q6_k_codes (src/format/quant.rs:574-599): 256 signed codes in output order. */
static void q6k_codes(const uint8_t *blk, int8_t *out) {
  const uint8_t *ql = blk, *qh = blk + 128;
  for (int n = 0; n < 2; n++) {
    for (int l = 0; l < 32; l++) {
      uint8_t hi = qh[32 * n + l];
      out[128 * n + l] = (int8_t)(((ql[64 * n + l] & 0xF) | (((hi >> 0) & 3) << 4)) - 32);
      out[128 * n + l + 32] = (int8_t)(((ql[64 * n + l + 32] & 0xF) | (((hi >> 2) & 3) << 4)) - 32);
      out[128 * n + l + 64] = (int8_t)(((ql[64 * n + l] >> 4) | (((hi >> 4) & 3) << 4)) - 32);
      out[128 * n + l + 96] = (int8_t)(((ql[64 * n + l + 32] >> 4) | (((hi >> 6) & 3) << 4)) - 32);
    }
  }
}

static int mul_chk(int64_t a, int64_t b, int64_t *o, apx_err *err) {
  if (__builtin_mul_overflow(a, b, o)) return fail(err, APX_ERR_FIXED_OVERFLOW);
  return 0;
}

/* dequant_row_fixed (src/engine/num/dequant.rs:99-129) with the Q8_0 (:311-346),
 * Q4_K (:487-593) and Q6_K (:595-640) row bodies. */
int apxo_dequant_row(uint32_t t, const uint8_t *row, size_t row_len, size_t n,
                     int64_t *out, apx_err *err) {
  size_t qk, bb;
  clear(err);
  if (!geom(t, &qk, &bb)) return fail(err, APX_ERR_UNSUPPORTED_QUANT);
  size_t blocks = (n + qk - 1) / qk;
  if (blocks * bb > row_len) return fail(err, APX_ERR_SHORT_PAYLOAD);
  size_t pushed = 0;
  for (size_t b = 0; b < blocks; b++) {
    const uint8_t *blk = row + b * bb;
    size_t take = n - b * qk < qk ? n - b * qk : qk;
    int64_t v;
    if (t == APX_GGML_TYPE_Q8_0) {
      int64_t d;
      if (apxo_f16_to_fixed(rd16(blk), &d)) return nonfinite(err, rd16(blk));
      for (size_t l = 0; l < take; l++) {
        if (mul_chk(d, (int8_t)blk[2 + l], &v, err)) return APX_ERR_FIXED_OVERFLOW;
        out[pushed++] = v;
      }
    } else if (t == APX_GGML_TYPE_Q5_0) {
      /* dequant_q5_0_row (num/dequant.rs:137-145, 357-390) on q5_0_codes (quant.rs:280-299):
       * output j < 16 is the low nibble of qs[j] with qh bit j as its fifth bit, output
       * 16 + j the high nibble with qh bit 16 + j; code - 16 times d */
      int64_t d;
      if (apxo_f16_to_fixed(rd16(blk), &d)) return nonfinite(err, rd16(blk));
      const uint8_t *qh = blk + 2, *qs = blk + 6;
      for (size_t l = 0; l < take; l++) {
        const size_t j = l % 16;
        const int hi = l >= 16;
        const int bit = (qh[(hi ? 2 : 0) + j / 8] >> (j % 8)) & 1;
        const int nib = hi ? (qs[j] >> 4) : (qs[j] & 0xF);
        if (mul_chk(d, (int64_t)((nib | (bit << 4)) - 16), &v, err)) return APX_ERR_FIXED_OVERFLOW;
        out[pushed++] = v;
      }
    } else if (t == APX_GGML_TYPE_Q4_K) {
      int64_t d, dmin, vals[QK_K];
      if (apxo_f16_to_fixed(rd16(blk), &d)) return nonfinite(err, rd16(blk));
      if (apxo_f16_to_fixed(rd16(blk + 2), &dmin)) return nonfinite(err, rd16(blk + 2));
      const uint8_t *sc = blk + 4, *qs = blk + 16;
      for (int g = 0; g < 4; g++) {
        int sl, ml, sh, mh;
        q4k_scale_min(sc, 2 * g, &sl, &ml);
        q4k_scale_min(sc, 2 * g + 1, &sh, &mh);
        int64_t slope_lo, icpt_lo, slope_hi, icpt_hi;
        if (mul_chk(d, sl, &slope_lo, err) || mul_chk(dmin, ml, &icpt_lo, err) ||
            mul_chk(d, sh, &slope_hi, err) || mul_chk(dmin, mh, &icpt_hi, err))
          return APX_ERR_FIXED_OVERFLOW;
        for (int l = 0; l < 32; l++) {
          int64_t p;
          if (mul_chk(slope_lo, qs[32 * g + l] & 0xF, &p, err) ||
              __builtin_sub_overflow(p, icpt_lo, &vals[64 * g + l]))
            return fail(err, APX_ERR_FIXED_OVERFLOW);
          if (mul_chk(slope_hi, qs[32 * g + l] >> 4, &p, err) ||
              __builtin_sub_overflow(p, icpt_hi, &vals[64 * g + 32 + l]))
            return fail(err, APX_ERR_FIXED_OVERFLOW);
        }
      }
      for (size_t l = 0; l < take; l++) out[pushed++] = vals[l];
    } else { /* Q6_K */
      int64_t d, vals[QK_K];
      int8_t codes[QK_K];
      uint16_t dbits = rd16(blk + 208);
      if (apxo_f16_to_fixed(dbits, &d)) return nonfinite(err, dbits);
      q6k_codes(blk, codes);
      for (int g = 0; g < 16; g++) {
        int64_t slope;
        if (mul_chk(d, (int8_t)blk[192 + g], &slope, err)) return APX_ERR_FIXED_OVERFLOW;
        for (int l = 0; l < 16; l++)
          if (mul_chk(slope, codes[16 * g + l], &vals[16 * g + l], err))
            return APX_ERR_FIXED_OVERFLOW;
      }
      for (size_t l = 0; l < take; l++) out[pushed++] = vals[l];
    }
  }
  return 0;
}

/* The shared geometry checks of matvec_fixed (ops/matvec.rs:156-172). */
static int row_geometry(uint32_t t, size_t n_out, size_t n_in, size_t raw_len,
                        size_t *row_bytes, apx_err *err) {
  size_t qk = 1, bb = 0, need;
  geom(t, &qk, &bb);
  size_t blocks = (n_in + qk - 1) / qk;
  if (__builtin_mul_overflow(blocks, bb, row_bytes)) return fail(err, APX_ERR_LENGTH_OVERFLOW);
  if (__builtin_mul_overflow(n_out, *row_bytes, &need)) return fail(err, APX_ERR_LENGTH_OVERFLOW);
  if (raw_len < need) {
    fail(err, APX_ERR_SHORT_PAYLOAD);
    if (err) {
      err->a = need;
      err->b = raw_len;
    }
    return APX_ERR_SHORT_PAYLOAD;
  }
  return 0;
}

static int shape_mismatch(apx_err *err, size_t x, size_t n_in) {
  fail(err, APX_ERR_SHAPE_MISMATCH);
  if (err) {
    err->a = x;
    err->b = n_in;
  }
  return APX_ERR_SHAPE_MISMATCH;
}

/* matvec_fixed (src/engine/ops/matvec.rs:149-222) with row_dot_fixed (:86-119). */
int apxo_matvec_fixed(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                      size_t n_in, const int64_t *x, size_t x_len, int64_t *out,
                      apx_err *err) {
  size_t qk, bb, row_bytes;
  clear(err);
  if (!geom(t, &qk, &bb)) {
    fail(err, APX_ERR_UNSUPPORTED_QUANT);
    if (err) err->ggml_type = t;
    return APX_ERR_UNSUPPORTED_QUANT;
  }
  if (x_len != n_in) return shape_mismatch(err, x_len, n_in);
  int rc = row_geometry(t, n_out, n_in, raw_len, &row_bytes, err);
  if (rc) return rc;
  int64_t *w = (int64_t *)malloc((n_in ? n_in : 1) * sizeof(int64_t));
  for (size_t o = 0; o < n_out; o++) {
    rc = apxo_dequant_row(t, raw + o * row_bytes, row_bytes, n_in, w, err);
    if (rc) {
      if (err) err->row = o;
      free(w);
      return rc;
    }
    i128 acc = 0;
    for (size_t i = 0; i < n_in; i++) {
      i128 prod = (i128)w[i] * (i128)x[i]; /* |i64 * i64| < 2^126: no overflow */
      if (__builtin_add_overflow(acc, prod, &acc)) {
        fail(err, APX_ERR_ACCUMULATOR_OVERFLOW);
        if (err) err->row = o;
        free(w);
        return APX_ERR_ACCUMULATOR_OVERFLOW;
      }
    }
    if (round_to_i64(acc, &out[o])) {
      fail(err, APX_ERR_OUTPUT_OVERFLOW);
      if (err) err->row = o;
      free(w);
      return APX_ERR_OUTPUT_OVERFLOW;
    }
  }
  free(w);
  return 0;
}

/* ---- the fused rows (chart/mod.rs:497-1013) ------------------------------------ */

/* QuantAct::magnitude (chart/mod.rs:159-181): 0 exact, 1 NoQ32, 2 TotalOverflow. */
static int magnitude(const int8_t *codes, size_t n, const int64_t *scales, size_t n_scales) {
  i128 acc = 0;
  for (size_t i = 0; i < n; i++) {
    if (i / ACT_QK >= n_scales) return 1;
    int64_t v;
    if (__builtin_mul_overflow(scales[i / ACT_QK], (int64_t)codes[i], &v)) return 1;
    i128 mag = v < 0 ? -(i128)v : (i128)v;
    if (__builtin_add_overflow(acc, mag, &acc)) return 2;
  }
  return 0;
}

static i128 sat_mul(i128 a, i128 b) {
  i128 r;
  if (__builtin_mul_overflow(a, b, &r)) return I128_MAX;
  return r;
}

/* q8act_fast_bound_ok (chart/mod.rs:362-383). */
static int fast_bound_ok(size_t n_in, i128 top, const int64_t *scales, size_t n_scales,
                         int narrow) {
  i128 s_max = 0;
  for (size_t b = 0; b < n_scales; b++) {
    i128 a = scales[b] < 0 ? -(i128)scales[b] : (i128)scales[b];
    if (a > s_max) s_max = a;
  }
  if (narrow && sat_mul(s_max, 32 * top * 127) > (i128)INT64_MAX) return 0;
  i128 f16max = (i128)65504 << 32;
  i128 bound = sat_mul(sat_mul(sat_mul(sat_mul((i128)n_in, f16max), top), 127), s_max);
  return bound < I128_MAX;
}

/* One fast row's exact pre-rounding accumulator (RowAcc over the family decoder's
 * groups, chart/mod.rs:497-514, 554-938, 947-1013); 1 on a non-finite scale. */
static int fast_row(uint32_t t, const uint8_t *row, size_t n_in, const int8_t *codes,
                    const int64_t *S, i128 *acc_out) {
  i128 acc = 0;
  size_t groups = n_in / ACT_QK;
  if (t == APX_GGML_TYPE_Q8_0) {
    for (size_t g = 0; g < groups; g++) {
      const uint8_t *blk = row + g * Q8_0_BYTES;
      int64_t d;
      if (apxo_f16_to_fixed(rd16(blk), &d)) return 1;
      const int8_t *q = (const int8_t *)(blk + 2);
      const int8_t *x = codes + g * ACT_QK;
      int32_t dot = 0;
      for (int l = 0; l < 32; l++) dot += (int32_t)q[l] * (int32_t)x[l];
      acc += (i128)S[g] * ((i128)d * (i128)dot);
    }
  } else if (t == APX_GGML_TYPE_Q5_0) {
    /* Q5_0Decoder (chart/mod.rs:630-712): one pure 32-lane group per block, w = d·(c − 16)
     * with c the five-bit code (qs nibble, qh bit as the fifth bit; quant.rs:280-299). */
    for (size_t g = 0; g < groups; g++) {
      const uint8_t *blk = row + g * 22;
      int64_t d;
      if (apxo_f16_to_fixed(rd16(blk), &d)) return 1;
      const uint8_t *qh = blk + 2, *qs = blk + 6;
      const int8_t *x = codes + g * ACT_QK;
      int32_t dot = 0;
      for (int l = 0; l < 32; l++) {
        const int j = l % 16, hi = l >= 16;
        const int bit = (qh[(hi ? 2 : 0) + j / 8] >> (j % 8)) & 1;
        const int nib = hi ? (qs[j] >> 4) : (qs[j] & 0xF);
        dot += ((nib | (bit << 4)) - 16) * (int32_t)x[l];
      }
      acc += (i128)S[g] * ((i128)d * (i128)dot);
    }
  } else if (t == APX_GGML_TYPE_Q4_K) {
    for (size_t g = 0; g < groups; g += 2) {
      size_t pp = g / 2, b = pp / 4, p = pp % 4;
      const uint8_t *blk = row + b * Q4_K_BYTES;
      int64_t d, dmin;
      if (apxo_f16_to_fixed(rd16(blk), &d)) return 1;
      if (apxo_f16_to_fixed(rd16(blk + 2), &dmin)) return 1;
      int sl, ml, sh, mh;
      q4k_scale_min(blk + 4, (int)(2 * p), &sl, &ml);
      q4k_scale_min(blk + 4, (int)(2 * p + 1), &sh, &mh);
      const uint8_t *qs = blk + 16 + 32 * p;
      const int8_t *xl = codes + g * ACT_QK, *xh = codes + (g + 1) * ACT_QK;
      int32_t dl = 0, dh = 0, sxl = 0, sxh = 0;
      for (int l = 0; l < 32; l++) {
        dl += (int32_t)(qs[l] & 0xF) * xl[l];
        dh += (int32_t)(qs[l] >> 4) * xh[l];
        sxl += xl[l];
        sxh += xh[l];
      }
      i128 in_lo = (i128)(d * sl) * dl - (i128)(dmin * ml) * sxl;
      i128 in_hi = (i128)(d * sh) * dh - (i128)(dmin * mh) * sxh;
      acc += (i128)S[g] * in_lo;
      acc += (i128)S[g + 1] * in_hi;
    }
  } else { /* Q6_K, n_in % 256 == 0 */
    for (size_t b = 0; b < n_in / QK_K; b++) {
      const uint8_t *blk = row + b * Q6_K_BYTES;
      int64_t d;
      if (apxo_f16_to_fixed(rd16(blk + 208), &d)) return 1;
      int8_t q[QK_K];
      q6k_codes(blk, q);
      for (int c = 0; c < 8; c++) {
        int64_t gd = 0;
        for (int h = 0; h < 2; h++) {
          int g16 = 2 * c + h;
          int32_t dot = 0;
          for (int l = 0; l < 16; l++)
            dot += (int32_t)q[16 * g16 + l] * codes[(b * 16 + g16) * 16 + l];
          gd += (int64_t)(int8_t)blk[192 + g16] * dot;
        }
        acc += (i128)S[b * 8 + c] * ((i128)d * gd);
      }
    }
  }
  *acc_out = acc;
  return 0;
}

/* The plan of matvec_q8act (q8act_plan, chart/mod.rs:1676-1727) reduced to what the
 * result depends on: 0 = fused fast rows, 1 = the contract (matvec_fixed on x-hat),
 * 2 = NoQ32 (FixedOverflow refusal). */
static int plan(uint32_t t, size_t n_in, const int8_t *codes, size_t q_len,
                const int64_t *scales, size_t n_scales, int *fast) {
  int mag = magnitude(codes, q_len, scales, n_scales);
  if (mag == 1) return 2;
  if (mag == 2 || !fused_type(t)) return 1;
  *fast = 0;
  if (t == APX_GGML_TYPE_Q8_0 && n_in % 32 == 0)
    *fast = fast_bound_ok(n_in, 128, scales, n_scales, 1);
  else if (t == APX_GGML_TYPE_Q5_0 && n_in % 32 == 0)
    *fast = fast_bound_ok(n_in, 16, scales, n_scales, 1);
  else if (t == APX_GGML_TYPE_Q4_K && n_in % 64 == 0)
    *fast = fast_bound_ok(n_in, 1008, scales, n_scales, 0);
  else if (t == APX_GGML_TYPE_Q6_K && n_in % 256 == 0)
    *fast = fast_bound_ok(n_in, 4096, scales, n_scales, 0);
  return 0;
}

static int contract(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                    size_t n_in, const int8_t *codes, size_t q_len,
                    const int64_t *scales, size_t n_scales, int64_t *out, apx_err *err) {
  int64_t *xhat = (int64_t *)malloc((q_len ? q_len : 1) * sizeof(int64_t));
  if (apxo_dequant_act(codes, q_len, scales, n_scales, xhat)) {
    free(xhat);
    return fail(err, APX_ERR_FIXED_OVERFLOW);
  }
  int rc = apxo_matvec_fixed(t, raw, raw_len, n_out, n_in, xhat, q_len, out, err);
  free(xhat);
  return rc;
}

/* Fast rows [lo, hi): 0 ok, APX_ERR_OUTPUT_OVERFLOW (row in *bad), or -1 for a
 * non-finite scale at row *bad (the caller falls back to the contract). */
static int fast_rows(uint32_t t, const uint8_t *raw, size_t row_bytes, size_t lo,
                     size_t hi, size_t n_in, const int8_t *codes, const int64_t *S,
                     int64_t *out, size_t *bad) {
  for (size_t o = lo; o < hi; o++) {
    i128 acc;
    if (fast_row(t, raw + o * row_bytes, n_in, codes, S, &acc)) {
      *bad = o;
      return -1;
    }
    if (round_to_i64(acc, &out[o])) {
      *bad = o;
      return APX_ERR_OUTPUT_OVERFLOW;
    }
  }
  return 0;
}

/* matvec_q8act (src/engine/chart/mod.rs:1887-1925) with q8act_rows (:1777-1859). */
int apxo_matvec_q8act(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                      size_t n_in, const int8_t *codes, size_t q_len,
                      const int64_t *scales, size_t n_scales, int64_t *out,
                      apx_err *err) {
  clear(err);
  int fast = 0;
  int p = plan(t, n_in, codes, q_len, scales, n_scales, &fast);
  if (p == 2) return fail(err, APX_ERR_FIXED_OVERFLOW);
  if (p == 1)
    return contract(t, raw, raw_len, n_out, n_in, codes, q_len, scales, n_scales, out, err);
  size_t qk, bb, row_bytes;
  if (!geom(t, &qk, &bb)) {
    fail(err, APX_ERR_UNSUPPORTED_QUANT);
    if (err) err->ggml_type = t;
    return APX_ERR_UNSUPPORTED_QUANT;
  }
  if (q_len != n_in) return shape_mismatch(err, q_len, n_in);
  int rc = row_geometry(t, n_out, n_in, raw_len, &row_bytes, err);
  if (rc) return rc;
  if (!fast)
    return contract(t, raw, raw_len, n_out, n_in, codes, q_len, scales, n_scales, out, err);
  size_t bad = 0;
  rc = fast_rows(t, raw, row_bytes, 0, n_out, n_in, codes, scales, out, &bad);
  if (rc == -1)
    return contract(t, raw, raw_len, n_out, n_in, codes, q_len, scales, n_scales, out, err);
  if (rc) {
    fail(err, rc);
    if (err) err->row = bad;
  }
  return rc;
}

/* matvec_q8act_quant_chunked (src/engine/chart/ffn.rs:667-745): with more than one
 * chunk the payload and shape checks run before the plan. */
int apxo_matvec_q8act_chunked(uint32_t t, const uint8_t *raw, size_t raw_len,
                              size_t n_out, size_t n_in, const int8_t *codes,
                              size_t q_len, const int64_t *scales, size_t n_scales,
                              size_t chunks, int64_t *out, apx_err *err) {
  size_t upper = n_out == 0 ? 1 : n_out, actual = chunks < 8 ? chunks : 8;
  if (actual < 1) actual = 1;
  if (actual > upper) actual = upper;
  size_t qk, bb, row_bytes;
  if (actual == 1 || !geom(t, &qk, &bb))
    return apxo_matvec_q8act(t, raw, raw_len, n_out, n_in, codes, q_len, scales, n_scales,
                             out, err);
  clear(err);
  int rc = row_geometry(t, n_out, n_in, raw_len, &row_bytes, err);
  if (rc) return rc;
  if (q_len != n_in) return shape_mismatch(err, q_len, n_in);
  return apxo_matvec_q8act(t, raw, raw_len, n_out, n_in, codes, q_len, scales, n_scales,
                           out, err);
}

/* matmat_q8act (src/engine/kern/matmat.rs:92-134): column c equals the per-column
 * call; the call refuses with the lowest refusing column's refusal. */
int apxo_matmat_q8act(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                      size_t n_in, size_t k_cols, const int8_t *codes, size_t q_len,
                      const int64_t *scales, int64_t *out, apx_err *err) {
  size_t nb = (q_len + ACT_QK - 1) / ACT_QK;
  clear(err);
  for (size_t c = 0; c < k_cols; c++) {
    int rc = apxo_matvec_q8act(t, raw, raw_len, n_out, n_in, codes + c * q_len, q_len,
                               scales + c * nb, nb, out + c * n_out, err);
    if (rc) {
      if (err) err->col = c;
      return rc;
    }
  }
  return 0;
}

/* exact_dot (src/engine/kern/gemm.rs:470-486). */
int apxo_exact_dot_q8_0(const uint8_t *row, size_t blocks, const int8_t *codes,
                        const int64_t *scales, int64_t *out) {
  i128 acc = 0;
  for (size_t b = 0; b < blocks; b++) {
    const uint8_t *blk = row + b * Q8_0_BYTES;
    int32_t m;
    uint32_t k;
    if (apxo_f16_split(rd16(blk), &m, &k)) return 1;
    int32_t dot = 0;
    for (int l = 0; l < 32; l++) dot += (int32_t)(int8_t)blk[2 + l] * codes[b * 32 + l];
    i128 d = (i128)m << k, term;
    if (__builtin_mul_overflow(d, (i128)scales[b], &term)) return 1;
    if (__builtin_mul_overflow(term, (i128)dot, &term)) return 1;
    if (__builtin_add_overflow(acc, term, &acc)) return 1;
  }
  return round_to_i64(acc, out);
}

/* Exact int32 group dots (the decoders' `dot` values, chart/mod.rs:554-938). */
int apxo_block_dots(uint32_t t, const uint8_t *raw, size_t n_out, size_t n_in,
                    const int8_t *codes, int32_t *dots) {
  size_t qk, bb;
  if (!geom(t, &qk, &bb)) return APX_ERR_UNSUPPORTED_QUANT;
  size_t blocks = (n_in + qk - 1) / qk, row_bytes = blocks * bb;
  size_t per_row = t == APX_GGML_TYPE_Q6_K ? blocks * 16 : blocks * (qk / 32);
  for (size_t o = 0; o < n_out; o++) {
    const uint8_t *row = raw + o * row_bytes;
    int32_t *dst = dots + o * per_row;
    for (size_t b = 0; b < blocks; b++) {
      const uint8_t *blk = row + b * bb;
      if (t == APX_GGML_TYPE_Q8_0) {
        int32_t dot = 0;
        for (int l = 0; l < 32; l++) dot += (int32_t)(int8_t)blk[2 + l] * codes[b * 32 + l];
        dst[b] = dot;
      } else if (t == APX_GGML_TYPE_Q4_K) {
        for (int p = 0; p < 4; p++) {
          int32_t dl = 0, dh = 0;
          for (int l = 0; l < 32; l++) {
            dl += (int32_t)(blk[16 + 32 * p + l] & 0xF) * codes[b * 256 + 64 * p + l];
            dh += (int32_t)(blk[16 + 32 * p + l] >> 4) * codes[b * 256 + 64 * p + 32 + l];
          }
          dst[b * 8 + 2 * p] = dl;
          dst[b * 8 + 2 * p + 1] = dh;
        }
      } else {
        int8_t q[QK_K];
        q6k_codes(blk, q);
        for (int g = 0; g < 16; g++) {
          int32_t dot = 0;
          for (int l = 0; l < 16; l++) dot += (int32_t)q[16 * g + l] * codes[b * 256 + 16 * g + l];
          dst[b * 16 + g] = dot;
        }
      }
    }
  }
  return 0;
}

/* ---- CPU baseline: the fused rows over contiguous row chunks on threads ------------
 * (the pool split of matvec_q8act_quant_chunked, src/engine/chart/ffn.rs:667-745). */

/* The vector rows of apx_oracle_x86.c (the reference's AVX2 / AVX-VNNI row cores), one build
 * per instruction set, and the f16 -> Q32.32 table they read (chart/portable.rs:15-79: the
 * exact decode of every finite pattern, 1 for Inf/NaN; every finite decode is even). */
typedef int (*x86_rows_fn)(uint32_t, const uint8_t *, size_t, size_t, size_t, size_t,
                           const int8_t *, const int64_t *, const int32_t *, const int64_t *,
                           int64_t *, size_t *);
int apxo_x86_rows_avx2(uint32_t, const uint8_t *, size_t, size_t, size_t, size_t,
                       const int8_t *, const int64_t *, const int32_t *, const int64_t *,
                       int64_t *, size_t *);
int apxo_x86_rows_vnni(uint32_t, const uint8_t *, size_t, size_t, size_t, size_t,
                       const int8_t *, const int64_t *, const int32_t *, const int64_t *,
                       int64_t *, size_t *);

static int64_t f16_table[65536];
static pthread_once_t f16_table_once = PTHREAD_ONCE_INIT;

static void f16_table_build(void) {
  for (uint32_t h = 0; h < 65536; h++) {
    int64_t v;
    f16_table[h] = apxo_f16_to_fixed((uint16_t)h, &v) ? 1 : v;
  }
}

/* APXO_NO_VNNI=1 in the environment selects the AVX2 build on an AVX-VNNI host, so the tests
 * check both builds against the scalar rows. */
int apxo_simd_features(void) {
  __builtin_cpu_init();
  int f = 0;
  if (__builtin_cpu_supports("avx2")) f |= 1;
  const char *no_vnni = getenv("APXO_NO_VNNI");
  if ((f & 1) && __builtin_cpu_supports("avxvnni") && !(no_vnni && no_vnni[0] == '1')) f |= 2;
  return f;
}

static x86_rows_fn x86_rows(void) {
  int f = apxo_simd_features();
  if (!(f & 1)) return NULL;
  pthread_once(&f16_table_once, f16_table_build);
  return (f & 2) ? apxo_x86_rows_vnni : apxo_x86_rows_avx2;
}

/* The vector rows take Q8_0 and Q5_0 on whole 32-lane blocks, Q4_K on whole 64-lane windows and Q6_K
 * on whole super-blocks, the widths the reference's AVX2 rows take (`tiled2` for whole
 * super-blocks, x86.rs:782-800, the single-row cores otherwise, chart/mod.rs:719-938); their
 * byte dots also
 * need every activation code in [-127, 127] (the |w|·sign(x, w) form), which quant_act
 * guarantees. */
static int x86_shape(uint32_t t, size_t n_in) {
  return ((t == APX_GGML_TYPE_Q8_0 || t == APX_GGML_TYPE_Q5_0) && n_in % ACT_QK == 0) ||
         (t == APX_GGML_TYPE_Q4_K && n_in % 64 == 0) ||
         (t == APX_GGML_TYPE_Q6_K && n_in % QK_K == 0);
}

typedef struct {
  uint32_t t;
  const uint8_t *raw;
  size_t row_bytes, lo, hi, n_in, k_cols, n_out;
  const int8_t *codes;
  const int64_t *scales;
  const int32_t *xsums; /* [k_cols][n_in / 32], vector rows only */
  x86_rows_fn vec;      /* NULL: the scalar fast rows */
  const int64_t *xhat;  /* [k_cols][n_in] dequantized activations: the contract's rows */
  int64_t *out;
  int rc;
  size_t bad;
} mt_task;

static void *mt_run(void *arg) {
  mt_task *a = (mt_task *)arg;
  size_t nb = (a->n_in + ACT_QK - 1) / ACT_QK;
  a->rc = 0;
  for (size_t c = 0; c < a->k_cols && a->rc == 0; c++) {
    if (a->xhat)
      a->rc = apxo_matvec_fixed(a->t, a->raw + a->lo * a->row_bytes,
                                (a->hi - a->lo) * a->row_bytes, a->hi - a->lo, a->n_in,
                                a->xhat + c * a->n_in, a->n_in, a->out + c * a->n_out + a->lo,
                                NULL);
    else if (a->vec)
      a->rc = a->vec(a->t, a->raw, a->row_bytes, a->lo, a->hi, a->n_in,
                     a->codes + c * a->n_in, a->scales + c * nb,
                     a->xsums ? a->xsums + c * nb : NULL, f16_table, a->out + c * a->n_out,
                     &a->bad);
    else
      a->rc = fast_rows(a->t, a->raw, a->row_bytes, a->lo, a->hi, a->n_in,
                        a->codes + c * a->n_in, a->scales + c * nb, a->out + c * a->n_out,
                        &a->bad);
  }
  return NULL;
}

/* A persistent pool of host threads, as the reference's decode runs its row chunks on a
 * global pool started once (src/engine/chart/pool.rs): workers are created on first use (and
 * added when a call asks for more), sleep on a condition variable between jobs and take task
 * i of a job; the calling thread runs task 0.  One job at a time.  A forked child starts with
 * no workers (pthread_atfork), since only the forking thread exists there. */
#define POOL_MAX 256
static pthread_mutex_t pool_job = PTHREAD_MUTEX_INITIALIZER;
static pthread_mutex_t pool_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t pool_go = PTHREAD_COND_INITIALIZER;
static pthread_cond_t pool_done = PTHREAD_COND_INITIALIZER;
static int pool_size, pool_pending, pool_ntasks;
static unsigned long pool_gen;
static void (*pool_fn)(void *, int);
static void *pool_ctx;
static pthread_once_t pool_fork_once = PTHREAD_ONCE_INIT;

static void pool_after_fork(void) {
  pthread_mutex_init(&pool_job, NULL);
  pthread_mutex_init(&pool_mu, NULL);
  pthread_cond_init(&pool_go, NULL);
  pthread_cond_init(&pool_done, NULL);
  pool_size = pool_pending = pool_ntasks = 0;
  pool_fn = NULL;
}

static void pool_register_fork(void) { pthread_atfork(NULL, NULL, pool_after_fork); }

static unsigned long pool_born[POOL_MAX + 1]; /* the job count when worker i was created */

static void *pool_worker(void *arg) {
  int me = (int)(intptr_t)arg;
  pthread_mutex_lock(&pool_mu);
  unsigned long seen = pool_born[me];
  for (;;) {
    while (pool_gen == seen) pthread_cond_wait(&pool_go, &pool_mu);
    seen = pool_gen;
    int run = me < pool_ntasks;
    void (*fn)(void *, int) = pool_fn;
    void *ctx = pool_ctx;
    pthread_mutex_unlock(&pool_mu);
    if (run) fn(ctx, me);
    pthread_mutex_lock(&pool_mu);
    if (--pool_pending == 0) pthread_cond_signal(&pool_done);
  }
  return NULL;
}

/* Runs fn(ctx, i) for i in [0, n) on the pool and the calling thread; returns when all are
 * done. */
static void pool_run(void (*fn)(void *, int), void *ctx, int n) {
  pthread_once(&pool_fork_once, pool_register_fork);
  pthread_mutex_lock(&pool_job);
  pthread_mutex_lock(&pool_mu);
  while (pool_size < n - 1) { /* workers 1 .. n-1 */
    pthread_t tid;
    pthread_attr_t at;
    pthread_attr_init(&at);
    pthread_attr_setdetachstate(&at, PTHREAD_CREATE_DETACHED);
    pool_born[pool_size + 1] = pool_gen;
    if (pthread_create(&tid, &at, pool_worker, (void *)(intptr_t)(pool_size + 1)) != 0) {
      pthread_attr_destroy(&at);
      break;
    }
    pthread_attr_destroy(&at);
    pool_size++;
  }
  int workers = pool_size;
  pool_fn = fn;
  pool_ctx = ctx;
  pool_ntasks = n < workers + 1 ? n : workers + 1;
  pool_pending = workers;
  pool_gen++;
  pthread_cond_broadcast(&pool_go);
  pthread_mutex_unlock(&pool_mu);
  fn(ctx, 0);
  for (int i = workers + 1; i < n; i++) fn(ctx, i); /* tasks no worker could take */
  pthread_mutex_lock(&pool_mu);
  while (pool_pending > 0) pthread_cond_wait(&pool_done, &pool_mu);
  pool_fn = NULL;
  pthread_mutex_unlock(&pool_mu);
  pthread_mutex_unlock(&pool_job);
}

static void mt_item(void *ctx, int i) { mt_run(&((mt_task *)ctx)[i]); }

static int run_mt(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                  size_t n_in, size_t k_cols, const int8_t *codes, const int64_t *scales,
                  int threads, int simd, int64_t *out, apx_err *err) {
  size_t nb = (n_in + ACT_QK - 1) / ACT_QK;
  clear(err);
  /* Columns whose plan is the contract (an unfused family or width, or the call bound failing)
   * run matvec_fixed on the dequantized activation, split over the same row chunks: the
   * chunked caller runs every row range on the pool whatever its plan (ffn.rs:705-726). */
  int contract_rows = 0;
  for (size_t c = 0; c < k_cols; c++) {
    int fast = 0;
    int p = plan(t, n_in, codes + c * n_in, n_in, scales + c * nb, nb, &fast);
    if (p == 2)
      return apxo_matmat_q8act(t, raw, raw_len, n_out, n_in, k_cols, codes, n_in, scales,
                               out, err);
    if (p != 0 || !fast) contract_rows = 1;
  }
  size_t qk, bb, row_bytes;
  if (!geom(t, &qk, &bb))
    return apxo_matmat_q8act(t, raw, raw_len, n_out, n_in, k_cols, codes, n_in, scales, out,
                             err);
  int rc = row_geometry(t, n_out, n_in, raw_len, &row_bytes, err);
  if (rc) return rc;
  int64_t *xhat = NULL;
  if (contract_rows) {
    xhat = (int64_t *)malloc((k_cols * n_in > 0 ? k_cols * n_in : 1) * sizeof(int64_t));
    for (size_t c = 0; c < k_cols; c++)
      if (apxo_dequant_act(codes + c * n_in, n_in, scales + c * nb, nb, xhat + c * n_in)) {
        free(xhat);
        return apxo_matmat_q8act(t, raw, raw_len, n_out, n_in, k_cols, codes, n_in, scales,
                                 out, err);
      }
  }
  x86_rows_fn vec = simd && !contract_rows && x86_shape(t, n_in) ? x86_rows() : NULL;
  for (size_t i = 0; vec && i < k_cols * n_in; i++)
    if (codes[i] == -128) vec = NULL;
  int32_t *xsums = NULL;
  if (vec && t == APX_GGML_TYPE_Q4_K) { /* block_xsums (chart/portable.rs:163-177) */
    xsums = (int32_t *)malloc(k_cols * nb * sizeof(int32_t));
    for (size_t g = 0; g < k_cols * nb; g++) {
      int32_t s = 0;
      for (int l = 0; l < ACT_QK; l++) s += codes[g * ACT_QK + l];
      xsums[g] = s;
    }
  }
  if (threads < 1) threads = 1;
  if (threads > POOL_MAX) threads = POOL_MAX;
  if ((size_t)threads > n_out) threads = n_out ? (int)n_out : 1;
  mt_task *tasks = (mt_task *)calloc((size_t)threads, sizeof(mt_task));
  size_t per = (n_out + (size_t)threads - 1) / (size_t)threads;
  if (vec) per += per & 1; /* whole row pairs per chunk */
  for (int i = 0; i < threads; i++) {
    size_t lo = (size_t)i * per, hi = lo + per < n_out ? lo + per : n_out;
    if (lo > n_out) lo = n_out;
    tasks[i] = (mt_task){t, raw, row_bytes, lo, hi, n_in, k_cols, n_out,
                         codes, scales, xsums, vec, xhat, out, 0, 0};
  }
  pool_run(mt_item, tasks, threads);
  rc = 0;
  for (int i = 0; i < threads && rc == 0; i++) rc = tasks[i].rc;
  free(tasks);
  free(xsums);
  free(xhat);
  if (rc != 0) /* any refusal: the single-threaded contract decides it */
    return apxo_matmat_q8act(t, raw, raw_len, n_out, n_in, k_cols, codes, n_in, scales,
                             out, err);
  return 0;
}

int apxo_matvec_q8act_mt(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                         size_t n_in, const int8_t *codes, const int64_t *scales,
                         int threads, int64_t *out, apx_err *err) {
  return run_mt(t, raw, raw_len, n_out, n_in, 1, codes, scales, threads, 0, out, err);
}

int apxo_matmat_q8act_mt(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                         size_t n_in, size_t k_cols, const int8_t *codes,
                         const int64_t *scales, int threads, int64_t *out, apx_err *err) {
  return run_mt(t, raw, raw_len, n_out, n_in, k_cols, codes, scales, threads, 0, out, err);
}

int apxo_matvec_q8act_simd_mt(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                              size_t n_in, const int8_t *codes, const int64_t *scales,
                              int threads, int64_t *out, apx_err *err) {
  return run_mt(t, raw, raw_len, n_out, n_in, 1, codes, scales, threads, 1, out, err);
}

/* ---- the prefill baseline: the k-column Q8_0 GEMM (src/engine/kern/gemm.rs:498-580) ------
 * Its row kernel is apxo_x86_gemm_rows (apx_oracle_x86.c, AVX-VNNI build); here are the
 * column pack (gemm.rs:131-264) and the row split over the pool. */
int apxo_x86_gemm_rows(const uint8_t *raw, size_t row_bytes, size_t blocks, size_t lo,
                       size_t hi, size_t k_cols, size_t n_in, const uint32_t *words,
                       const int64_t *shift, const uint32_t *emin, const uint32_t *gspread,
                       uint32_t limit, const int8_t *codes, const int64_t *scales,
                       int64_t *out, size_t n_out);

typedef struct {
  const uint8_t *raw;
  size_t row_bytes, blocks, n_out, n_in, k_cols, per;
  const uint32_t *words, *emin, *gspread;
  const int64_t *shift, *scales;
  const int8_t *codes;
  uint32_t limit;
  int64_t *out;
  int bail[POOL_MAX];
} gemm_job;

static void gemm_item(void *ctx, int i) {
  gemm_job *j = (gemm_job *)ctx;
  size_t lo = (size_t)i * j->per, hi = lo + j->per < j->n_out ? lo + j->per : j->n_out;
  j->bail[i] = lo < hi ? apxo_x86_gemm_rows(j->raw, j->row_bytes, j->blocks, lo, hi,
                                            j->k_cols, j->n_in, j->words, j->shift, j->emin,
                                            j->gspread, j->limit, j->codes, j->scales, j->out,
                                            j->n_out)
                       : 0;
}

/* spread_limit (gemm.rs:99-102): 33 − ⌈log2 blocks⌉. */
static uint32_t spread_limit(size_t blocks) {
  uint32_t log = 0;
  while (((size_t)1 << log) < blocks) log++;
  return log >= 33 ? 0 : 33 - log;
}

/* 1 when the GEMM ran and wrote every output; 0 when the call takes the per-column rows. */
static int gemm_q8_0_mt(const uint8_t *raw, size_t raw_len, size_t n_out, size_t n_in,
                        size_t k_cols, const int8_t *codes, const int64_t *scales, int threads,
                        int64_t *out) {
  size_t blocks = n_in / ACT_QK;
  if (n_in % ACT_QK || blocks == 0 || blocks > 512 || k_cols == 0 || n_out == 0) return 0;
  if ((apxo_simd_features() & 3) != 3) return 0;
  if (raw_len / Q8_0_BYTES / blocks < n_out) return 0;
  for (size_t c = 0; c < k_cols; c++) { /* fast_columns_ok (gemm.rs:283-300) */
    int fast = 0;
    if (plan(APX_GGML_TYPE_Q8_0, n_in, codes + c * n_in, n_in, scales + c * blocks, blocks,
             &fast) != 0 || !fast)
      return 0;
  }
  size_t groups = (k_cols + 7) / 8;
  uint32_t *words = (uint32_t *)malloc(groups * blocks * 64 * sizeof(uint32_t));
  int64_t *shift = (int64_t *)calloc(groups * blocks * 8, sizeof(int64_t));
  uint32_t *emin = (uint32_t *)calloc(groups * 8, sizeof(uint32_t));
  uint32_t *gspread = (uint32_t *)calloc(groups, sizeof(uint32_t));
  gemm_job *job = (gemm_job *)calloc(1, sizeof(gemm_job));
  int ok = words && shift && emin && gspread && job;
  for (size_t g = 0; ok && g < groups; g++) {
    for (size_t lane = 0; lane < 8; lane++) {
      size_t c = g * 8 + lane;
      uint32_t e_lo = UINT32_MAX;
      for (size_t b = 0; c < k_cols && b < blocks; b++) {
        int64_t S = scales[c * blocks + b];
        if (S < 0 || (S & (S - 1))) ok = 0; /* not 0 or a power of two */
        if (S > 0 && (uint32_t)__builtin_ctzll((uint64_t)S) < e_lo)
          e_lo = (uint32_t)__builtin_ctzll((uint64_t)S);
      }
      if (e_lo == UINT32_MAX) e_lo = 0;
      emin[c] = e_lo;
      for (size_t b = 0; b < blocks; b++) {
        int64_t S = c < k_cols ? scales[c * blocks + b] : 0;
        uint32_t sh = S > 0 ? (uint32_t)__builtin_ctzll((uint64_t)S) - e_lo : 0;
        shift[(g * blocks + b) * 8 + lane] = sh;
        if (sh > gspread[g]) gspread[g] = sh;
        for (int q = 0; q < 8; q++) {
          uint32_t w = 0;
          for (int i = 0; i < 4; i++) {
            int8_t x = S > 0 ? codes[c * n_in + b * 32 + 4 * q + i] : 0;
            w |= (uint32_t)(uint8_t)(x + 128) << (8 * i);
          }
          words[((g * blocks + b) * 8 + q) * 8 + lane] = w;
        }
      }
    }
  }
  int done = 0;
  if (ok) {
    if (threads < 1) threads = 1;
    if (threads > POOL_MAX) threads = POOL_MAX;
    if ((size_t)threads > n_out) threads = (int)n_out;
    size_t per = (n_out + (size_t)threads - 1) / (size_t)threads;
    per += per & 1;
    *job = (gemm_job){raw, blocks * Q8_0_BYTES, blocks, n_out, n_in, k_cols, per, words, emin,
                      gspread, shift, scales, codes, spread_limit(blocks), out, {0}};
    pool_run(gemm_item, job, threads);
    done = 1;
    for (int i = 0; i < threads; i++) done &= !job->bail[i];
  }
  free(words);
  free(shift);
  free(emin);
  free(gspread);
  free(job);
  return done;
}

extern unsigned long apxo_x86_gemm_exact_groups;
static unsigned long gemm_calls, q4k_calls, q6k_calls;
unsigned long apxo_q4k_exact_groups, apxo_q6k_exact_groups;

void apxo_gemm_counts(uint64_t *calls, uint64_t *exact_groups) {
  *calls = __atomic_load_n(&gemm_calls, __ATOMIC_RELAXED);
  *exact_groups = __atomic_load_n(&apxo_x86_gemm_exact_groups, __ATOMIC_RELAXED);
}

void apxo_q4k_counts(uint64_t *calls, uint64_t *exact_groups) {
  *calls = __atomic_load_n(&q4k_calls, __ATOMIC_RELAXED);
  *exact_groups = __atomic_load_n(&apxo_q4k_exact_groups, __ATOMIC_RELAXED);
}

void apxo_q6k_counts(uint64_t *calls, uint64_t *exact_groups) {
  *calls = __atomic_load_n(&q6k_calls, __ATOMIC_RELAXED);
  *exact_groups = __atomic_load_n(&apxo_q6k_exact_groups, __ATOMIC_RELAXED);
}

/* A Q6_K super-block's 256 unsigned 6-bit codes (q, before the −32 offset). */
void apxo_q6k_codes_u6(const uint8_t *blk, uint8_t *out) {
  int8_t q[QK_K];
  q6k_codes(blk, q);
  for (int i = 0; i < QK_K; i++) out[i] = (uint8_t)(q[i] + 32);
}

/* One fused row's rounded value for the vector kernels' exact fallback: 0 ok, 1 a non-finite
 * scale, 2 an output outside i64. */
int apxo_fast_row_value(uint32_t t, const uint8_t *row, size_t n_in, const int8_t *codes,
                        const int64_t *S, int64_t *out) {
  i128 acc;
  if (fast_row(t, row, n_in, codes, S, &acc)) return 1;
  return round_to_i64(acc, out) ? 2 : 0;
}

/* ---- the k-column Q4_K and Q6_K projections (chart/kcols.rs:1406-1518): the column pack
 * (pack_cols, kcols.rs:505-614) and the row split; the rows are apx_oracle_x86.c's. */
typedef int (*q4k_rows_fn)(const uint8_t *, size_t, size_t, size_t, size_t, size_t, size_t,
                           const uint32_t *, const int32_t *, const int64_t *, const int64_t *,
                           const uint32_t *, const uint32_t *, uint32_t, const int8_t *,
                           const int64_t *, int64_t *, size_t);
int apxo_x86_q4k_rows_avx2(const uint8_t *, size_t, size_t, size_t, size_t, size_t, size_t,
                           const uint32_t *, const int32_t *, const int64_t *, const int64_t *,
                           const uint32_t *, const uint32_t *, uint32_t, const int8_t *,
                           const int64_t *, int64_t *, size_t);
int apxo_x86_q4k_rows_vnni(const uint8_t *, size_t, size_t, size_t, size_t, size_t, size_t,
                           const uint32_t *, const int32_t *, const int64_t *, const int64_t *,
                           const uint32_t *, const uint32_t *, uint32_t, const int8_t *,
                           const int64_t *, int64_t *, size_t);
int apxo_x86_q6k_rows_avx2(const uint8_t *, size_t, size_t, size_t, size_t, size_t, size_t,
                           const uint32_t *, const int32_t *, const int64_t *, const int64_t *,
                           const uint32_t *, const uint32_t *, uint32_t, const int8_t *,
                           const int64_t *, int64_t *, size_t);
int apxo_x86_q6k_rows_vnni(const uint8_t *, size_t, size_t, size_t, size_t, size_t, size_t,
                           const uint32_t *, const int32_t *, const int64_t *, const int64_t *,
                           const uint32_t *, const uint32_t *, uint32_t, const int8_t *,
                           const int64_t *, int64_t *, size_t);

typedef struct {
  q4k_rows_fn fn;
  const uint8_t *raw;
  size_t row_bytes, sblocks, n_out, n_in, k_cols, per;
  const uint32_t *words, *emin, *cspread;
  const int32_t *xs;
  const int64_t *she, *sho, *scales;
  const int8_t *codes;
  uint32_t limit;
  int64_t *out;
  int bail[POOL_MAX];
} q4k_job;

static void q4k_item(void *ctx, int i) {
  q4k_job *j = (q4k_job *)ctx;
  size_t lo = (size_t)i * j->per, hi = lo + j->per < j->n_out ? lo + j->per : j->n_out;
  j->bail[i] = lo < hi ? j->fn(j->raw, j->row_bytes, j->sblocks, lo, hi, j->k_cols, j->n_in,
                               j->words, j->xs, j->she, j->sho, j->emin, j->cspread, j->limit,
                               j->codes, j->scales, j->out, j->n_out)
                       : 0;
}

/* lane_spread_limit (kcols.rs:455-462): 62 − 34 − ⌈log2 groups⌉. */
static uint32_t lane_spread_limit(size_t groups) {
  uint32_t log = 0;
  while (((size_t)1 << log) < groups) log++;
  return log >= 28 ? 0 : 28 - log;
}

/* 1 when the k-column Q4_K / Q6_K kernel ran and wrote every output; 0 when the call takes
 * the per-column rows (which also decide every refusal).  Q6_K keeps its block sums per
 * 16-lane group (xs), Q4_K per 32-lane group. */
static int gemm_kq_mt(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out, size_t n_in,
                      size_t k_cols, const int8_t *codes, const int64_t *scales, int threads,
                      int64_t *out) {
  int q6 = t == APX_GGML_TYPE_Q6_K;
  size_t sblocks = n_in / QK_K, G = n_in / ACT_QK, block_bytes = q6 ? Q6_K_BYTES : Q4_K_BYTES;
  size_t xlanes = q6 ? 16 : 32, XG = n_in / xlanes;
  if (n_in % QK_K || sblocks == 0 || sblocks > 256 || k_cols == 0 || n_out == 0) return 0;
  int f = apxo_simd_features();
  if (!(f & 1)) return 0;
  q4k_rows_fn fn = q6 ? ((f & 2) ? apxo_x86_q6k_rows_vnni : apxo_x86_q6k_rows_avx2)
                      : ((f & 2) ? apxo_x86_q4k_rows_vnni : apxo_x86_q4k_rows_avx2);
  if (raw_len / block_bytes / sblocks < n_out) return 0;
  for (size_t c = 0; c < k_cols; c++) { /* every column on its fast row, narrow bound */
    int fast = 0;
    if (plan(t, n_in, codes + c * n_in, n_in, scales + c * G, G, &fast) != 0 || !fast ||
        !fast_bound_ok(n_in, q6 ? 4096 : 1008, scales + c * G, G, 1))
      return 0;
  }
  pthread_once(&f16_table_once, f16_table_build);
  size_t groups = (k_cols + 7) / 8;
  uint32_t *words = (uint32_t *)calloc(groups * G * 64, sizeof(uint32_t));
  int32_t *xs = (int32_t *)calloc(groups * XG * 8, sizeof(int32_t));
  int64_t *she = (int64_t *)calloc(groups * G * 4, sizeof(int64_t));
  int64_t *sho = (int64_t *)calloc(groups * G * 4, sizeof(int64_t));
  uint32_t *emin = (uint32_t *)calloc(groups * 8, sizeof(uint32_t));
  uint32_t *cspread = (uint32_t *)calloc(groups, sizeof(uint32_t));
  q4k_job *job = (q4k_job *)calloc(1, sizeof(q4k_job));
  int ok = words && xs && she && sho && emin && cspread && job;
  for (size_t c = 0; ok && c < k_cols; c++) {
    size_t cg = c / 8, lane = c % 8;
    uint32_t e_lo = UINT32_MAX;
    for (size_t g = 0; g < G; g++) {
      int64_t S = scales[c * G + g];
      if (S < 0 || (S & (S - 1))) ok = 0;
      if (S > 0 && (uint32_t)__builtin_ctzll((uint64_t)S) < e_lo)
        e_lo = (uint32_t)__builtin_ctzll((uint64_t)S);
    }
    if (e_lo == UINT32_MAX) e_lo = 0;
    emin[c] = e_lo;
    for (size_t g = 0; ok && g < G; g++) {
      int64_t S = scales[c * G + g];
      size_t gi = cg * G + g;
      uint32_t sh = S > 0 ? (uint32_t)__builtin_ctzll((uint64_t)S) - e_lo : 0;
      if (sh > cspread[cg]) cspread[cg] = sh;
      (lane & 1 ? sho : she)[gi * 4 + lane / 2] = sh;
      int32_t sum[2] = {0, 0};
      for (int q = 0; q < 8; q++) {
        uint32_t w = 0;
        for (int i = 0; i < 4; i++) {
          int8_t x = S > 0 ? codes[c * n_in + g * 32 + 4 * q + i] : 0;
          sum[q / 4] += x;
          w |= (uint32_t)(uint8_t)x << (8 * i);
        }
        words[(gi * 8 + q) * 8 + lane] = w;
      }
      if (q6) {
        xs[(cg * XG + 2 * g) * 8 + lane] = sum[0];
        xs[(cg * XG + 2 * g + 1) * 8 + lane] = sum[1];
      } else {
        xs[gi * 8 + lane] = sum[0] + sum[1];
      }
    }
  }
  int done = 0;
  if (ok) {
    if (threads < 1) threads = 1;
    if (threads > POOL_MAX) threads = POOL_MAX;
    if ((size_t)threads > n_out) threads = (int)n_out;
    size_t per = (n_out + (size_t)threads - 1) / (size_t)threads;
    per += per & 1;
    *job = (q4k_job){fn, raw, sblocks * block_bytes, sblocks, n_out, n_in, k_cols, per, words,
                     emin, cspread, xs, she, sho, scales, codes, lane_spread_limit(XG), out,
                     {0}};
    pool_run(q4k_item, job, threads);
    done = 1;
    for (int i = 0; i < threads; i++) done &= !job->bail[i];
  }
  free(words);
  free(xs);
  free(she);
  free(sho);
  free(emin);
  free(cspread);
  free(job);
  return done;
}

int apxo_x86_q8_0_kcols_avx2(const uint8_t *, size_t, size_t, size_t, size_t, size_t,
                             const int8_t *, const int64_t *, const int64_t *, int64_t *,
                             size_t);
int apxo_x86_q8_0_kcols_vnni(const uint8_t *, size_t, size_t, size_t, size_t, size_t,
                             const int8_t *, const int64_t *, const int64_t *, int64_t *,
                             size_t);
static unsigned long kcols_calls;

void apxo_kcols_counts(uint64_t *calls) {
  *calls = __atomic_load_n(&kcols_calls, __ATOMIC_RELAXED);
}

typedef struct {
  int (*fn)(const uint8_t *, size_t, size_t, size_t, size_t, size_t, const int8_t *,
            const int64_t *, const int64_t *, int64_t *, size_t);
  const uint8_t *raw;
  size_t row_bytes, n_out, n_in, k_cols, per;
  const int8_t *codes;
  const int64_t *scales;
  int64_t *out;
  int bail[POOL_MAX];
} kcols_job;

static void kcols_item(void *ctx, int i) {
  kcols_job *j = (kcols_job *)ctx;
  size_t lo = (size_t)i * j->per, hi = lo + j->per < j->n_out ? lo + j->per : j->n_out;
  j->bail[i] = lo < hi ? j->fn(j->raw, j->row_bytes, lo, hi, j->n_in, j->k_cols, j->codes,
                               j->scales, f16_table, j->out, j->n_out)
                       : 0;
}

/* The Q8_0 columns in runs of 16 over one pass of each row (pooled_q8_0, kern/matmat.rs:
 * 198-206), what the reference runs when its GEMM does not; 1 when it wrote every output. */
static int q8_0_kcols_mt(const uint8_t *raw, size_t raw_len, size_t n_out, size_t n_in,
                         size_t k_cols, const int8_t *codes, const int64_t *scales, int threads,
                         int64_t *out) {
  size_t blocks = n_in / ACT_QK;
  if (n_in % ACT_QK || blocks == 0 || k_cols == 0 || n_out == 0) return 0;
  x86_rows_fn vec = x86_rows(); /* AVX2 present; builds the f16 table */
  if (!vec) return 0;
  if (raw_len / Q8_0_BYTES / blocks < n_out) return 0;
  for (size_t c = 0; c < k_cols; c++) {
    int fast = 0;
    if (plan(APX_GGML_TYPE_Q8_0, n_in, codes + c * n_in, n_in, scales + c * blocks, blocks,
             &fast) != 0 || !fast)
      return 0;
  }
  for (size_t i = 0; i < k_cols * n_in; i++)
    if (codes[i] == -128) return 0;
  kcols_job *job = (kcols_job *)calloc(1, sizeof(kcols_job));
  if (!job) return 0;
  if (threads < 1) threads = 1;
  if (threads > POOL_MAX) threads = POOL_MAX;
  if ((size_t)threads > n_out) threads = (int)n_out;
  size_t per = (n_out + (size_t)threads - 1) / (size_t)threads;
  job->fn = (apxo_simd_features() & 2) ? apxo_x86_q8_0_kcols_vnni : apxo_x86_q8_0_kcols_avx2;
  job->raw = raw;
  job->row_bytes = blocks * Q8_0_BYTES;
  job->n_out = n_out;
  job->n_in = n_in;
  job->k_cols = k_cols;
  job->per = per;
  job->codes = codes;
  job->scales = scales;
  job->out = out;
  pool_run(kcols_item, job, threads);
  int done = 1;
  for (int i = 0; i < threads; i++) done &= !job->bail[i];
  free(job);
  return done;
}

/* With AVX-VNNI, Q8_0 calls whose every column takes the fast rows run the k-column GEMM, as
 * the reference's matmat_q8act tries gemm_q8_0 first (kern/matmat.rs:134-146); Q8_0 calls the GEMM
 * does not take (no AVX-VNNI) run their columns in runs of 16 per row pass (pooled_q8_0); Q4_K
 * and Q6_K calls on whole super-blocks run the k-column kernels (gemm_q4_k / gemm_q6_k,
 * matmat.rs:163-177); everything
 * else (and every call those kernels bail on) runs the vector rows per column. */
int apxo_matmat_q8act_simd_mt(uint32_t t, const uint8_t *raw, size_t raw_len, size_t n_out,
                              size_t n_in, size_t k_cols, const int8_t *codes,
                              const int64_t *scales, int threads, int64_t *out,
                              apx_err *err) {
  if (t == APX_GGML_TYPE_Q8_0 &&
      gemm_q8_0_mt(raw, raw_len, n_out, n_in, k_cols, codes, scales, threads, out)) {
    __atomic_fetch_add(&gemm_calls, 1, __ATOMIC_RELAXED);
    clear(err);
    return 0;
  }
  if (t == APX_GGML_TYPE_Q8_0 && k_cols > 1 &&
      q8_0_kcols_mt(raw, raw_len, n_out, n_in, k_cols, codes, scales, threads, out)) {
    __atomic_fetch_add(&kcols_calls, 1, __ATOMIC_RELAXED);
    clear(err);
    return 0;
  }
  if ((t == APX_GGML_TYPE_Q4_K || t == APX_GGML_TYPE_Q6_K) &&
      gemm_kq_mt(t, raw, raw_len, n_out, n_in, k_cols, codes, scales, threads, out)) {
    __atomic_fetch_add(t == APX_GGML_TYPE_Q4_K ? &q4k_calls : &q6k_calls, 1, __ATOMIC_RELAXED);
    clear(err);
    return 0;
  }
  return run_mt(t, raw, raw_len, n_out, n_in, k_cols, codes, scales, threads, 1, out, err);
}

/* ---- the FFN hidden activation: SwiGLU under either carrier ----------------------------- */

/* fixed_exp (src/numeric/fixed_exp.rs:1-184): e^x in Q32.32 for x in [-16, 21]: x = k·ln2 + r
 * with k = round(x·log2(e)) (Q32.32 constants LN2 = 2977044472, 1/LN2 = 6196328019, product
 * rounded at 2^64), the degree-7 Taylor polynomial in r by Horner with each step rounded
 * (half away from zero) at 2^32, then a shift by k (rounded right shifts for k < 0).
 * 0 ok, 1 OutOfRange. */
static i128 rdiv_2p32(i128 v) {
  const i128 half = (i128)1 << 31;
  return v >= 0 ? (v + half) >> 32 : -((-v + half) >> 32);
}

int apxo_fixed_exp(int64_t x, int64_t *out) {
  const int64_t one = (int64_t)1 << 32;
  if (x < -16 * one || x > 21 * one) return 1;
  const i128 prod = (i128)x * (i128)6196328019LL;
  const i128 sh = (prod + ((i128)1 << 63)) >> 64;
  if (sh > (i128)INT64_MAX || sh < (i128)INT64_MIN) return 1;
  const int64_t k = (int64_t)sh;
  const i128 kl = (i128)k * (i128)2977044472LL;
  if (kl > (i128)INT64_MAX || kl < (i128)INT64_MIN) return 1;
  const i128 r = (i128)(x - (int64_t)kl);
  static const int64_t c[8] = {852176, 5965232, 35791394, 178956971, 715827883,
                               2147483648LL, 4294967296LL, 4294967296LL};
  i128 acc = c[0];
  for (int i = 1; i < 8; i++) acc = rdiv_2p32(acc * r) + c[i];
  i128 v;
  if (k >= 0) {
    if (k >= 64) return 1;
    v = acc << k;
  } else {
    const uint64_t n = (uint64_t)(-k);
    if (n >= 64) {
      *out = 0;
      return 0;
    }
    v = (acc + ((i128)1 << (n - 1))) >> n;
  }
  if (v > (i128)INT64_MAX || v < (i128)INT64_MIN) return 1;
  *out = (int64_t)v;
  return 0;
}

/* silu_fixed (src/engine/ops/silu.rs:53-100): v >= 16 -> v, v <= -21 -> 0, else
 * sign(v)·div_round_nearest(|v|·2^32, 2^32 + fixed_exp(-v)) (value.rs:5-7, ties upward).
 * 0 ok, else the FfnError kind (1 ExpOutOfRange, 2 ZeroDenominator, 3 Overflow). */
int apxo_silu_fixed(int64_t v, int64_t *out) {
  const int64_t one = (int64_t)1 << 32;
  if (v >= 16 * one) {
    *out = v;
    return 0;
  }
  if (v <= -21 * one) {
    *out = 0;
    return 0;
  }
  int64_t e;
  if (apxo_fixed_exp(-v, &e)) return 1;
  int64_t den;
  if (__builtin_add_overflow(one, e, &den)) return 3;
  if (den <= 0) return 2;
  const i128 mag = v < 0 ? -(i128)v : (i128)v;
  const i128 num = mag * (i128)one;
  const i128 q = (num + (i128)den / 2) / (i128)den;
  const i128 sgn = v < 0 ? -q : q;
  if (sgn > (i128)INT64_MAX || sgn < (i128)INT64_MIN) return 3;
  *out = (int64_t)sgn;
  return 0;
}

/* exp_f32_scalar (src/engine/mixer/f32_carrier.rs:262-324): Cephes-style binary32 exp, every
 * operation one IEEE binary32 rounding (no contraction: this file builds with
 * -ffp-contract=off).  Bits in, bits out. */
static float f32_of(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static uint32_t bits_of(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

static float exp_ref(float x) {
  if (x != x) return f32_of(0x7fc00000u);
  if (x < f32_of(0xc2b00000u)) return 0.0f;
  if (x > f32_of(0x42b17218u)) return f32_of(0x7f800000u);
  const float z = x * f32_of(0x3fb8aa3bu);
  const float n_flt = rintf(z);
  const int32_t n_int = (int32_t)n_flt;
  const float r = (x - n_flt * f32_of(0x3f318000u)) - n_flt * f32_of(0xb95e8083u);
  const float r2 = r * r;
  float p = f32_of(0x39506967u);
  p = p * r + f32_of(0x3ab743ceu);
  p = p * r + f32_of(0x3c088908u);
  p = p * r + f32_of(0x3d2aa9c1u);
  p = p * r + f32_of(0x3e2aaaaau);
  p = p * r + f32_of(0x3f000000u);
  const float y = (1.0f + r) + (r2 * p);
  const int32_t n1 = n_int >> 1, n2 = n_int - n1;
  const float s1 = f32_of((uint32_t)(n1 + 127) << 23), s2 = f32_of((uint32_t)(n2 + 127) << 23);
  return (y * s1) * s2;
}

uint32_t apxo_exp_f32(uint32_t x) { return bits_of(exp_ref(f32_of(x))); }

/* silu_f32_scalar (f32_carrier.rs:372-375): x / (1 + exp(-x)). */
uint32_t apxo_silu_f32(uint32_t x) {
  const float f = f32_of(x);
  return bits_of(f / (1.0f + exp_ref(-f)));
}

/* swiglu_one under a carrier (src/engine/chart/ffn.rs:246-284):
 *   carrier 0 (F32): to_q32(silu(from_q32(gate)) · from_q32(up)), from_q32(x) = RN(x)/2^32
 *     (fp.rs:176-178); Overflow where the product is not finite or leaves Q32.32;
 *   carrier 1 (Q32): round_shift_32(silu_fixed(gate) · up) narrowed to i64, else Overflow.
 * 0 ok, else the FfnError kind (3 Overflow). */
int apxo_swiglu(int64_t gate, int64_t up, int carrier, int64_t *out) {
  if (carrier == 0) {
    const float g = (float)gate * 0x1p-32f, u = (float)up * 0x1p-32f;
    const float s = g / (1.0f + exp_ref(-g));
    const float prod = s * u;
    if (!(prod - prod == 0.0f)) return 3;
    return apxo_f32_to_q32(bits_of(prod), out) ? 3 : 0;
  }
  int64_t s;
  const int rc = apxo_silu_fixed(gate, &s);
  if (rc) return rc;
  const i128 v = rs32((i128)s * (i128)up);
  if (v > (i128)INT64_MAX || v < (i128)INT64_MIN) return 3;
  *out = (int64_t)v;
  return 0;
}

