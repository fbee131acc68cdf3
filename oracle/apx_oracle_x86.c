/*
 * apx_oracle_x86.c — vector kernels of the timed CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY (see apx_oracle.h): bench.py's cpu_baseline and `--impl reference`
 * legs time these rows; tests/test_oracle_x86.py checks them against the scalar fused rows of
 * apx_oracle.c.  The product library never links this file.
 *
 * The reference's decode rows on x86 are AVX2 cores that take two weight rows per pass and
 * share each activation load between them (`tiled2`, `q8_0_rows2_avx2`, `q4_k_rows2_avx2`,
 * src/engine/chart/x86.rs:782-1200).  This file restates those cores so the CPU baseline runs
 * at the reference's own speed class instead of a scalar loop's:
 *   - a 32-lane byte dot is |w| (unsigned) times sign(x, w) (signed), which is exact in
 *     either instruction form: `vpmaddubsw` + `vpmaddwd` (pair sums ≤ 2·128·127 < 2^15, so no
 *     saturation) or, with AVX-VNNI, one `vpdpbusd` (x86.rs:177-210);
 *   - f16 block scales decode through one 65,536-entry table whose odd entries mark the
 *     non-finite patterns (every finite decode is a multiple of 2^8), ORed into one word per
 *     row pair and tested after the loop (chart/portable.rs:15-79);
 *   - the folds are the scalar fast row's, in its group order, with the same exact integers:
 *     Q8_0 `acc += d·(S·D)` (S·D fits i64 under the narrow call bound), Q4_K
 *     `acc += S·((d·sc)·D − (dmin·m)·Σxq)` per 32-lane group.
 * Integer sums are exact, so each row's accumulator equals the scalar fast row's bit for bit.
 *
 * The multi-column (prefill) kernels follow, each in its own section: the k-column Q8_0 GEMM
 * (AVX-VNNI build only, kern/gemm.rs:498-580), the k-column Q4_K and Q6_K kernels
 * (chart/kcols.rs:1406-1518) and the Q8_0 column runs of 16 the reference uses without AVX-VNNI
 * (kern/matmat.rs:198-206).  Every one of them reports a case it cannot finish exactly (a
 * non-finite scale, an output outside i64) to its caller, which redecides the call on the
 * per-column rows, so refusals are always the contract's.
 *
 * This file is compiled twice (oracle/Makefile): with APX_X86_VNNI=0 for AVX2 and with
 * APX_X86_VNNI=1 under -mavxvnni; apx_oracle.c picks one at run time from CPUID.
 * Paths in comments are relative to the apeiron source tree.
 */
#include <immintrin.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>

#include "../include/apeiron_cuda.h"

typedef __int128 i128;

#if APX_X86_VNNI
#define ROWS_NAME apxo_x86_rows_vnni
#else
#define ROWS_NAME apxo_x86_rows_avx2
#endif

#define Q8_0_BYTES 34
#define Q4_K_BYTES 144

/* Eight i32 lane sums of w·x over 32 byte lanes (x86.rs:177-210). */
static inline __m256i dot_lanes(__m256i w, __m256i x) {
  __m256i u = _mm256_abs_epi8(w), s = _mm256_sign_epi8(x, w);
#if APX_X86_VNNI
  return _mm256_dpbusd_avx_epi32(_mm256_setzero_si256(), u, s);
#else
  return _mm256_madd_epi16(_mm256_maddubs_epi16(u, s), _mm256_set1_epi16(1));
#endif
}

/* The four totals [Σp0, Σp1, Σp2, Σp3] of four lane vectors (x86.rs:148-160). */
static inline __m128i sum4(__m256i p0, __m256i p1, __m256i p2, __m256i p3) {
  __m256i h = _mm256_hadd_epi32(_mm256_hadd_epi32(p0, p1), _mm256_hadd_epi32(p2, p3));
  return _mm_add_epi32(_mm256_castsi256_si128(h), _mm256_extracti128_si256(h, 1));
}

static inline int32_t sum1(__m256i p) {
  __m128i v = _mm_add_epi32(_mm256_castsi256_si128(p), _mm256_extracti128_si256(p, 1));
  v = _mm_hadd_epi32(v, v);
  v = _mm_hadd_epi32(v, v);
  return _mm_cvtsi128_si32(v);
}

static inline uint16_t word(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static inline __m256i ld(const void *p) { return _mm256_loadu_si256((const __m256i *)p); }

/* get_scale_min_k4 (src/format/quant.rs:482-491). */
static inline void scale_min(const uint8_t *q, int j, int *s, int *m) {
  if (j < 4) {
    *s = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *s = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* Two Q8_0 rows (r0, r1) of `blocks` blocks: the accumulators before rounding; returns the
 * OR of the four scale-table entries' low bits (1 = a non-finite scale in either row). */
static int q8_0_pair(const uint8_t *r0, const uint8_t *r1, size_t blocks, const int8_t *codes,
                     const int64_t *S, const int64_t *tab, i128 acc[2]) {
  i128 a0 = 0, a1 = 0;
  int64_t bad = 0;
  size_t b = 0;
  for (; b + 4 <= blocks; b += 4) {
    const uint8_t *p0 = r0 + b * Q8_0_BYTES, *p1 = r1 + b * Q8_0_BYTES;
    const int8_t *x = codes + b * 32;
    __m256i x0 = ld(x), x1 = ld(x + 32), x2 = ld(x + 64), x3 = ld(x + 96);
    __m128i t0 = sum4(dot_lanes(ld(p0 + 2), x0), dot_lanes(ld(p0 + 2 + Q8_0_BYTES), x1),
                      dot_lanes(ld(p0 + 2 + 2 * Q8_0_BYTES), x2),
                      dot_lanes(ld(p0 + 2 + 3 * Q8_0_BYTES), x3));
    __m128i t1 = sum4(dot_lanes(ld(p1 + 2), x0), dot_lanes(ld(p1 + 2 + Q8_0_BYTES), x1),
                      dot_lanes(ld(p1 + 2 + 2 * Q8_0_BYTES), x2),
                      dot_lanes(ld(p1 + 2 + 3 * Q8_0_BYTES), x3));
    int32_t d0[4], d1[4];
    _mm_storeu_si128((__m128i *)d0, t0);
    _mm_storeu_si128((__m128i *)d1, t1);
    for (int j = 0; j < 4; j++) {
      int64_t w0 = tab[word(p0 + j * Q8_0_BYTES)], w1 = tab[word(p1 + j * Q8_0_BYTES)];
      bad |= w0 | w1;
      int64_t s = S[b + j];
      a0 += (i128)w0 * (i128)(s * (int64_t)d0[j]);
      a1 += (i128)w1 * (i128)(s * (int64_t)d1[j]);
    }
  }
  for (; b < blocks; b++) {
    const uint8_t *p0 = r0 + b * Q8_0_BYTES, *p1 = r1 + b * Q8_0_BYTES;
    __m256i x = ld(codes + b * 32);
    int64_t w0 = tab[word(p0)], w1 = tab[word(p1)];
    bad |= w0 | w1;
    int64_t s = S[b];
    a0 += (i128)w0 * (i128)(s * (int64_t)sum1(dot_lanes(ld(p0 + 2), x)));
    a1 += (i128)w1 * (i128)(s * (int64_t)sum1(dot_lanes(ld(p1 + 2), x)));
  }
  acc[0] = a0;
  acc[1] = a1;
  return (int)(bad & 1);
}

/* Two Q4_K rows of `sblocks` whole super-blocks and then `tail` 64-lane windows of the next
 * one (a width that is a multiple of 64 but not of 256, as the reference's single-row core
 * takes it window by window, chart/mod.rs:719-838); xsums[g] = Σ codes over 32-lane group g. */
static int q4_k_pair(const uint8_t *r0, const uint8_t *r1, size_t sblocks, int tail,
                     const int8_t *codes, const int64_t *S, const int32_t *xsums,
                     const int64_t *tab, i128 acc[2]) {
  const __m256i nib = _mm256_set1_epi8(0x0F);
  i128 a[2] = {0, 0};
  int64_t bad = 0;
  for (size_t b = 0; b < sblocks; b++) {
    const int8_t *x = codes + b * 256;
    __m256i x0 = ld(x), x1 = ld(x + 32), x2 = ld(x + 64), x3 = ld(x + 96);
    __m256i x4 = ld(x + 128), x5 = ld(x + 160), x6 = ld(x + 192), x7 = ld(x + 224);
    for (int r = 0; r < 2; r++) {
      const uint8_t *blk = (r ? r1 : r0) + b * Q4_K_BYTES;
      int64_t d = tab[word(blk)], dmin = tab[word(blk + 2)];
      bad |= d | dmin;
      const uint8_t *qs = blk + 16;
      __m256i q0 = ld(qs), q1 = ld(qs + 32), q2 = ld(qs + 64), q3 = ld(qs + 96);
      __m128i lo = sum4(dot_lanes(_mm256_and_si256(q0, nib), x0),
                        dot_lanes(_mm256_and_si256(q1, nib), x2),
                        dot_lanes(_mm256_and_si256(q2, nib), x4),
                        dot_lanes(_mm256_and_si256(q3, nib), x6));
      __m256i h0 = _mm256_and_si256(_mm256_srli_epi16(q0, 4), nib);
      __m256i h1 = _mm256_and_si256(_mm256_srli_epi16(q1, 4), nib);
      __m256i h2 = _mm256_and_si256(_mm256_srli_epi16(q2, 4), nib);
      __m256i h3 = _mm256_and_si256(_mm256_srli_epi16(q3, 4), nib);
      __m128i hi = sum4(dot_lanes(h0, x1), dot_lanes(h1, x3), dot_lanes(h2, x5),
                        dot_lanes(h3, x7));
      int32_t dl[4], dh[4];
      _mm_storeu_si128((__m128i *)dl, lo);
      _mm_storeu_si128((__m128i *)dh, hi);
      for (int p = 0; p < 4; p++) {
        int sl, ml, sh, mh;
        scale_min(blk + 4, 2 * p, &sl, &ml);
        scale_min(blk + 4, 2 * p + 1, &sh, &mh);
        size_t g = b * 8 + 2 * (size_t)p;
        i128 in_lo = (i128)(d * sl) * dl[p] - (i128)(dmin * ml) * xsums[g];
        i128 in_hi = (i128)(d * sh) * dh[p] - (i128)(dmin * mh) * xsums[g + 1];
        a[r] += (i128)S[g] * in_lo + (i128)S[g + 1] * in_hi;
      }
    }
  }
  if (tail > 0) {
    const size_t b = sblocks;
    const int8_t *x = codes + b * 256;
    for (int r = 0; r < 2; r++) {
      const uint8_t *blk = (r ? r1 : r0) + b * Q4_K_BYTES;
      int64_t d = tab[word(blk)], dmin = tab[word(blk + 2)];
      bad |= d | dmin;
      for (int p = 0; p < tail; p++) {
        __m256i q = ld(blk + 16 + 32 * p);
        int32_t dl = sum1(dot_lanes(_mm256_and_si256(q, nib), ld(x + 64 * p)));
        int32_t dh = sum1(dot_lanes(_mm256_and_si256(_mm256_srli_epi16(q, 4), nib),
                                    ld(x + 64 * p + 32)));
        int sl, ml, sh, mh;
        scale_min(blk + 4, 2 * p, &sl, &ml);
        scale_min(blk + 4, 2 * p + 1, &sh, &mh);
        size_t g = b * 8 + 2 * (size_t)p;
        i128 in_lo = (i128)(d * sl) * dl - (i128)(dmin * ml) * xsums[g];
        i128 in_hi = (i128)(d * sh) * dh - (i128)(dmin * mh) * xsums[g + 1];
        a[r] += (i128)S[g] * in_lo + (i128)S[g + 1] * in_hi;
      }
    }
  }
  acc[0] = a[0];
  acc[1] = a[1];
  return (int)(bad & 1);
}

/* The 256 codes q − 32 of a Q6_K super-block in lane order, 8 vectors of 32 (quant.rs:574-599:
 * low nibbles of ql with two bits of qh above them). */
static inline void q6_k_codes8(const uint8_t *blk, __m256i w[8]) {
  const __m256i m4 = _mm256_set1_epi8(0x0F), m2 = _mm256_set1_epi8(0x03);
  const __m256i off = _mm256_set1_epi8(32);
  for (int n = 0; n < 2; n++) {
    __m256i l0 = ld(blk + 64 * n), l1 = ld(blk + 64 * n + 32), h = ld(blk + 128 + 32 * n);
    __m256i h0 = _mm256_slli_epi16(_mm256_and_si256(h, m2), 4);
    __m256i h1 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 2), m2), 4);
    __m256i h2 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 4), m2), 4);
    __m256i h3 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 6), m2), 4);
    w[4 * n + 0] = _mm256_sub_epi8(_mm256_or_si256(_mm256_and_si256(l0, m4), h0), off);
    w[4 * n + 1] = _mm256_sub_epi8(_mm256_or_si256(_mm256_and_si256(l1, m4), h1), off);
    w[4 * n + 2] = _mm256_sub_epi8(
        _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l0, 4), m4), h2), off);
    w[4 * n + 3] = _mm256_sub_epi8(
        _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l1, 4), m4), h3), off);
  }
}

/* Two Q6_K rows of `sblocks` super-blocks (the reference's Q6_K core, x86.rs:713-780): per
 * 32-lane activation group c, `acc += S_c·(d·(sc_2c·D_2c + sc_2c+1·D_2c+1))` over the two
 * 16-lane halves, the halves' dots being the low and high 128 bits of one lane vector. */
static int q6_k_pair(const uint8_t *r0, const uint8_t *r1, size_t sblocks, const int8_t *codes,
                     const int64_t *S, const int64_t *tab, i128 acc[2]) {
  i128 a[2] = {0, 0};
  int64_t bad = 0;
  for (size_t b = 0; b < sblocks; b++) {
    const int8_t *x = codes + b * 256;
    __m256i xv[8];
    for (int c = 0; c < 8; c++) xv[c] = ld(x + 32 * c);
    for (int r = 0; r < 2; r++) {
      const uint8_t *blk = (r ? r1 : r0) + b * 210;
      int64_t d = tab[word(blk + 208)];
      bad |= d;
      __m256i w[8];
      q6_k_codes8(blk, w);
      for (int c = 0; c < 8; c++) {
        __m256i p = dot_lanes(w[c], xv[c]);
        __m128i lo = _mm256_castsi256_si128(p), hi = _mm256_extracti128_si256(p, 1);
        __m128i t = _mm_hadd_epi32(lo, hi);
        t = _mm_hadd_epi32(t, t); /* [D_lo, D_hi, D_lo, D_hi] */
        int32_t dlo = _mm_cvtsi128_si32(t), dhi = _mm_extract_epi32(t, 1);
        int64_t gd = (int64_t)(int8_t)blk[192 + 2 * c] * dlo +
                     (int64_t)(int8_t)blk[192 + 2 * c + 1] * dhi;
        a[r] += (i128)S[b * 8 + (size_t)c] * ((i128)d * gd);
      }
    }
  }
  acc[0] = a[0];
  acc[1] = a[1];
  return (int)(bad & 1);
}

/* The 32 weights c − 16 of a Q5_0 block (quant.rs:280-299): lane j < 16 the low nibble of qs[j],
 * lane 16 + j the high one, each with qh bit j (resp. 16 + j) as its fifth bit. */
static inline __m256i q5_0_codes(const uint8_t *blk) {
  const __m128i qs = _mm_loadu_si128((const __m128i *)(blk + 6));
  const __m128i m4 = _mm_set1_epi8(0x0F);
  __m256i nib = _mm256_set_m128i(_mm_and_si128(_mm_srli_epi16(qs, 4), m4), _mm_and_si128(qs, m4));
  uint32_t qh;
  __builtin_memcpy(&qh, blk + 2, 4);
  /* byte j of the lane vector takes qh byte j / 8, then its bit j % 8 */
  const __m256i spread = _mm256_setr_epi8(0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1, 2, 2, 2,
                                          2, 2, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3, 3);
  const __m256i bits = _mm256_set1_epi64x((long long)0x8040201008040201ull);
  __m256i hb = _mm256_shuffle_epi8(_mm256_set1_epi32((int)qh), spread);
  hb = _mm256_cmpeq_epi8(_mm256_and_si256(hb, bits), bits);
  __m256i c = _mm256_or_si256(nib, _mm256_and_si256(hb, _mm256_set1_epi8(0x10)));
  return _mm256_sub_epi8(c, _mm256_set1_epi8(16));
}

/* Two Q5_0 rows of `blocks` blocks (q5_0_rows2_avx2, x86.rs:957-1058): per block
 * `acc += d·(S·D)` with D the exact dot of c − 16 against the codes. */
static int q5_0_pair(const uint8_t *r0, const uint8_t *r1, size_t blocks, const int8_t *codes,
                     const int64_t *S, const int64_t *tab, i128 acc[2]) {
  i128 a0 = 0, a1 = 0;
  int64_t bad = 0;
  for (size_t b = 0; b < blocks; b++) {
    const uint8_t *p0 = r0 + b * 22, *p1 = r1 + b * 22;
    __m256i x = ld(codes + b * 32);
    int64_t w0 = tab[word(p0)], w1 = tab[word(p1)];
    bad |= w0 | w1;
    int64_t s = S[b];
    a0 += (i128)w0 * (i128)(s * (int64_t)sum1(dot_lanes(q5_0_codes(p0), x)));
    a1 += (i128)w1 * (i128)(s * (int64_t)sum1(dot_lanes(q5_0_codes(p1), x)));
  }
  acc[0] = a0;
  acc[1] = a1;
  return (int)(bad & 1);
}

/* round_shift_32 then the i64 range check (src/engine/num/value.rs:10-12,
 * chart/mod.rs:1746-1753). */
static int finish_row(i128 acc, int64_t *out) {
  i128 q = acc >> 32;
  q += ((uint64_t)acc & 0xFFFFFFFFull) >= 0x80000000ull;
  if (q > (i128)INT64_MAX || q < (i128)INT64_MIN) return 1;
  *out = (int64_t)q;
  return 0;
}

/* Rows [lo, hi) of a Q8_0 or Q5_0 (n_in % 32 == 0), Q4_K (n_in % 64 == 0) or Q6_K
 * (n_in % 256 == 0) projection whose call
 * plan chose the fast rows.  Returns 0, APX_ERR_OUTPUT_OVERFLOW with the first such row in
 * *bad, or -1 when a block scale is non-finite (the caller then runs the contract). */
int ROWS_NAME(uint32_t t, const uint8_t *raw, size_t row_bytes, size_t lo, size_t hi,
              size_t n_in, const int8_t *codes, const int64_t *S, const int32_t *xsums,
              const int64_t *tab, int64_t *out, size_t *bad) {
  for (size_t o = lo; o < hi; o += 2) {
    const uint8_t *r0 = raw + o * row_bytes;
    const uint8_t *r1 = o + 1 < hi ? r0 + row_bytes : r0;
    i128 acc[2];
    int nf = t == APX_GGML_TYPE_Q8_0   ? q8_0_pair(r0, r1, n_in / 32, codes, S, tab, acc)
             : t == APX_GGML_TYPE_Q5_0 ? q5_0_pair(r0, r1, n_in / 32, codes, S, tab, acc)
             : t == APX_GGML_TYPE_Q6_K ? q6_k_pair(r0, r1, n_in / 256, codes, S, tab, acc)
                                       : q4_k_pair(r0, r1, n_in / 256, (int)(n_in % 256) / 64,
                                                   codes, S, xsums, tab, acc);
    if (nf) {
      *bad = o;
      return -1;
    }
    for (size_t r = 0; r < 2 && o + r < hi; r++) {
      if (finish_row(acc[r], &out[o + r])) {
        *bad = o + r;
        return APX_ERR_OUTPUT_OVERFLOW;
      }
    }
  }
  return 0;
}

#if APX_X86_VNNI
/* ---- the k-column Q8_0 GEMM of the prefill baseline (src/engine/kern/gemm.rs:498-580) ----
 *
 * The reference's prefill runs Q8_0 projections of many tokens through `gemm_q8_0` when the
 * host has AVX-VNNI: every weight row is read once per call and its 32-byte blocks are dotted
 * against groups of 8 token columns with `vpdpbusd`, the activation stored as x + 128 (u8) and
 * the weight as i8, so each lane's sum is D + 128·Σw and one subtraction of the row's
 * 128·Σw recovers the exact block dot D.  The row's f16 scales are split as m·2^k (|m| ≤ 2047,
 * pow2.rs:52-64) and each (row, token) accumulates `(m·D) << (k − kmin + e − emin)` in i64
 * (|m·D| < 2^30), exact while the row's k spread plus the group's e spread stays within
 * `33 − ⌈log2 blocks⌉` (spread_limit, gemm.rs:99-102); a (row, group) past it takes the
 * i128 `exact_dot`.  The output is `finish(acc, kmin + emin)` (pow2.rs:76-96).  Two rows per
 * pass share every activation load. */

int apxo_f16_split(uint16_t h, int32_t *m, uint32_t *k);
int apxo_finish(int64_t acc, uint32_t s, int64_t *out);
int apxo_exact_dot_q8_0(const uint8_t *row, size_t blocks, const int8_t *codes,
                        const int64_t *scales, int64_t *out);

#define GEMM_MAX_BLOCKS 512

/* (row, group) pairs that took the exact i128 dot, for the tests (apxo_gemm_counts). */
unsigned long apxo_x86_gemm_exact_groups;

/* A row's per-block m, k − kmin and 128·Σw (row_scales, gemm.rs:438-456); 1 on a non-finite
 * scale. */
static int row_scales(const uint8_t *row, size_t blocks, int32_t *m, int64_t *kd, int32_t *bsum,
                      uint32_t *kmin_out, uint32_t *spread_out) {
  uint32_t kmin = UINT32_MAX, kmax = 0;
  for (size_t b = 0; b < blocks; b++) {
    const uint8_t *blk = row + b * Q8_0_BYTES;
    uint32_t k;
    if (apxo_f16_split(word(blk), &m[b], &k)) return 1;
    kd[b] = k;
    kmin = k < kmin ? k : kmin;
    kmax = k > kmax ? k : kmax;
    int32_t sum = 0;
    for (int l = 0; l < 32; l++) sum += (int8_t)blk[2 + l];
    bsum[b] = 128 * sum;
  }
  for (size_t b = 0; b < blocks; b++) kd[b] -= kmin;
  *kmin_out = kmin;
  *spread_out = kmax - kmin;
  return 0;
}

/* One row's 8 lanes of one block: (m·(acc − 128Σw)) << (kd + shift) added to lo/hi. */
static inline void fold8(__m256i dots, int32_t m, int64_t kd, int32_t bsum, __m256i sh0,
                         __m256i sh1, __m256i *lo, __m256i *hi) {
  __m256i t = _mm256_mullo_epi32(_mm256_sub_epi32(dots, _mm256_set1_epi32(bsum)),
                                 _mm256_set1_epi32(m));
  __m256i kv = _mm256_set1_epi64x(kd);
  *lo = _mm256_add_epi64(*lo, _mm256_sllv_epi64(_mm256_cvtepi32_epi64(_mm256_castsi256_si128(t)),
                                                _mm256_add_epi64(sh0, kv)));
  *hi = _mm256_add_epi64(*hi,
                         _mm256_sllv_epi64(_mm256_cvtepi32_epi64(_mm256_extracti128_si256(t, 1)),
                                           _mm256_add_epi64(sh1, kv)));
}

/* Rows [lo, hi) of the GEMM.  words: [group][block][quad][lane] u32 (4 bytes x + 128 of
 * column 8·group + lane); shift: [group][block][lane] i64 (e − emin, 0 for zero blocks and
 * padding lanes); emin per column; gspread per group.  out[c·n_out + o].  Returns 0, or 1 when
 * the caller must redecide the call on the per-column path (a non-finite scale, an output
 * outside i64, an exact dot past i128). */
int apxo_x86_gemm_rows(const uint8_t *raw, size_t row_bytes, size_t blocks, size_t lo,
                       size_t hi, size_t k_cols, size_t n_in, const uint32_t *words,
                       const int64_t *shift, const uint32_t *emin, const uint32_t *gspread,
                       uint32_t limit, const int8_t *codes, const int64_t *scales,
                       int64_t *out, size_t n_out) {
  int32_t ma[GEMM_MAX_BLOCKS], mb[GEMM_MAX_BLOCKS], sa[GEMM_MAX_BLOCKS], sb[GEMM_MAX_BLOCKS];
  int64_t ka[GEMM_MAX_BLOCKS], kb[GEMM_MAX_BLOCKS];
  size_t groups = (k_cols + 7) / 8;
  for (size_t o = lo; o < hi; o += 2) {
    int two = o + 1 < hi;
    const uint8_t *ra = raw + o * row_bytes, *rb = two ? ra + row_bytes : ra;
    uint32_t kmina, spra, kminb, sprb;
    if (row_scales(ra, blocks, ma, ka, sa, &kmina, &spra) ||
        row_scales(rb, blocks, mb, kb, sb, &kminb, &sprb))
      return 1;
    for (size_t g = 0; g < groups; g++) {
      size_t c0 = g * 8, nc = k_cols - c0 < 8 ? k_cols - c0 : 8;
      if (spra + gspread[g] > limit || sprb + gspread[g] > limit) {
        __atomic_fetch_add(&apxo_x86_gemm_exact_groups, 1, __ATOMIC_RELAXED);
        for (size_t c = c0; c < c0 + nc; c++)
          for (int r = 0; r <= two; r++)
            if (apxo_exact_dot_q8_0(r ? rb : ra, blocks, codes + c * n_in,
                                    scales + c * blocks, &out[c * n_out + o + r]))
              return 1;
        continue;
      }
      const uint32_t *wg = words + g * blocks * 64;
      const int64_t *sg = shift + g * blocks * 8;
      __m256i a0 = _mm256_setzero_si256(), a1 = a0, b0 = a0, b1 = a0;
      for (size_t b = 0; b < blocks; b++) {
        const uint8_t *ca = ra + b * Q8_0_BYTES + 2, *cb = rb + b * Q8_0_BYTES + 2;
        const uint32_t *wb = wg + b * 64;
        __m256i da = _mm256_setzero_si256(), db = da;
        for (int q = 0; q < 8; q++) {
          __m256i act = ld(wb + 8 * q);
          int32_t wa, wbq;
          __builtin_memcpy(&wa, ca + 4 * q, 4);
          __builtin_memcpy(&wbq, cb + 4 * q, 4);
          da = _mm256_dpbusd_avx_epi32(da, act, _mm256_set1_epi32(wa));
          db = _mm256_dpbusd_avx_epi32(db, act, _mm256_set1_epi32(wbq));
        }
        __m256i sh0 = ld(sg + b * 8), sh1 = ld(sg + b * 8 + 4);
        fold8(da, ma[b], ka[b], sa[b], sh0, sh1, &a0, &a1);
        fold8(db, mb[b], kb[b], sb[b], sh0, sh1, &b0, &b1);
      }
      int64_t la[8], lb[8];
      _mm256_storeu_si256((__m256i *)la, a0);
      _mm256_storeu_si256((__m256i *)(la + 4), a1);
      _mm256_storeu_si256((__m256i *)lb, b0);
      _mm256_storeu_si256((__m256i *)(lb + 4), b1);
      for (size_t c = 0; c < nc; c++) {
        if (apxo_finish(la[c], kmina + emin[c0 + c], &out[(c0 + c) * n_out + o])) return 1;
        if (two && apxo_finish(lb[c], kminb + emin[c0 + c], &out[(c0 + c) * n_out + o + 1]))
          return 1;
      }
    }
  }
  return 0;
}
#endif

/* ---- the k-column Q4_K projection of the prefill baseline (chart/kcols.rs:1406-1464) -------
 *
 * The reference runs multi-column Q4_K calls (n_in % 256 == 0, every column on its fast row
 * under the narrow bound) through one pass over each weight row: the row's nibbles are dotted
 * against groups of 8 token columns (unsigned nibble × signed code, `vpdpbusd` or
 * `vpmaddubsw` + `vpmaddwd`, both exact: pair sums ≤ 2·15·127), and each 32-lane group g adds
 *     ((m_d·sc_g)·D_g) << (k_d − kmin + e_g − emin) − ((m_m·m_g)·X_g) << (k_m − kmin + e_g − emin)
 * to the column's i64 lane (d = m_d·2^k_d, dmin = m_m·2^k_m by f16_split, X_g = Σ codes of the
 * group).  A term is below 2^33 + 2^29 < 2^34, so G groups with every shift at most `spread`
 * stay below 2^(34 + ⌈log2 G⌉ + spread): past lane_spread_limit (kcols.rs:455-462) a (row,
 * column group) takes the exact i128 fast row instead.  The output is finish(acc, kmin + emin).
 * 64-bit products come from `vpmuldq`, which reads the even 32-bit lanes, so the column shifts
 * are kept per group in two orders: even columns (0, 2, 4, 6) and odd ones. */

#if APX_X86_VNNI
#define Q4K_NAME apxo_x86_q4k_rows_vnni
#else
#define Q4K_NAME apxo_x86_q4k_rows_avx2
#endif

int apxo_fast_row_value(uint32_t t, const uint8_t *row, size_t n_in, const int8_t *codes,
                        const int64_t *S, int64_t *out);
int apxo_f16_split(uint16_t h, int32_t *m, uint32_t *k);
int apxo_finish(int64_t acc, uint32_t s, int64_t *out);

/* (row, column group) pairs sent to the exact rows, for the tests (defined in apx_oracle.c). */
extern unsigned long apxo_q4k_exact_groups;

#define Q4K_MAX_SBLOCKS 256 /* n_in <= 65536 */

static inline __m256i quad_dot(__m256i acc, __m256i w_u8, __m256i x_i8) {
#if APX_X86_VNNI
  return _mm256_dpbusd_avx_epi32(acc, w_u8, x_i8);
#else
  return _mm256_add_epi32(acc, _mm256_madd_epi16(_mm256_maddubs_epi16(w_u8, x_i8),
                                                 _mm256_set1_epi16(1)));
#endif
}

/* One row's per-group coefficients and weight bytes; 1 on a non-finite scale. */
typedef struct {
  uint8_t *w;      /* n_in unpacked nibbles, lane order */
  int64_t *c1, *c2; /* m_d·sc_g, m_m·m_g per group */
  int64_t *a, *b;   /* k_d − kmin, k_m − kmin per group */
  uint32_t kmin, spread;
} q4k_row;

static int q4k_row_prep(const uint8_t *row, size_t sblocks, q4k_row *r) {
  uint32_t kmin = UINT32_MAX, kmax = 0;
  int32_t md[Q4K_MAX_SBLOCKS], mm[Q4K_MAX_SBLOCKS];
  uint32_t kd[Q4K_MAX_SBLOCKS], km[Q4K_MAX_SBLOCKS];
  for (size_t b = 0; b < sblocks; b++) {
    const uint8_t *blk = row + b * Q4_K_BYTES;
    if (apxo_f16_split(word(blk), &md[b], &kd[b]) || apxo_f16_split(word(blk + 2), &mm[b], &km[b]))
      return 1;
    uint32_t lo = kd[b] < km[b] ? kd[b] : km[b], hi = kd[b] < km[b] ? km[b] : kd[b];
    kmin = lo < kmin ? lo : kmin;
    kmax = hi > kmax ? hi : kmax;
  }
  const __m256i nib = _mm256_set1_epi8(0x0F);
  for (size_t b = 0; b < sblocks; b++) {
    const uint8_t *blk = row + b * Q4_K_BYTES;
    for (int p = 0; p < 4; p++) {
      __m256i q = ld(blk + 16 + 32 * p);
      _mm256_storeu_si256((__m256i *)(r->w + b * 256 + 64 * p), _mm256_and_si256(q, nib));
      _mm256_storeu_si256((__m256i *)(r->w + b * 256 + 64 * p + 32),
                          _mm256_and_si256(_mm256_srli_epi16(q, 4), nib));
    }
    for (int j = 0; j < 8; j++) {
      int sc, m;
      scale_min(blk + 4, j, &sc, &m);
      size_t g = b * 8 + (size_t)j;
      r->c1[g] = (int64_t)md[b] * sc;
      r->c2[g] = (int64_t)mm[b] * m;
      r->a[g] = (int64_t)kd[b] - kmin;
      r->b[g] = (int64_t)km[b] - kmin;
    }
  }
  r->kmin = kmin;
  r->spread = kmax - kmin;
  return 0;
}

static inline void q4k_fold(__m256i d, __m256i x, const q4k_row *r, size_t g, __m256i she,
                            __m256i sho, __m256i *ae, __m256i *ao) {
  __m256i c1 = _mm256_set1_epi64x(r->c1[g]), c2 = _mm256_set1_epi64x(r->c2[g]);
  __m256i a = _mm256_set1_epi64x(r->a[g]), b = _mm256_set1_epi64x(r->b[g]);
  __m256i de = d, dodd = _mm256_srli_epi64(d, 32), xe = x, xodd = _mm256_srli_epi64(x, 32);
  *ae = _mm256_add_epi64(*ae, _mm256_sllv_epi64(_mm256_mul_epi32(de, c1), _mm256_add_epi64(she, a)));
  *ae = _mm256_sub_epi64(*ae, _mm256_sllv_epi64(_mm256_mul_epi32(xe, c2), _mm256_add_epi64(she, b)));
  *ao = _mm256_add_epi64(*ao, _mm256_sllv_epi64(_mm256_mul_epi32(dodd, c1), _mm256_add_epi64(sho, a)));
  *ao = _mm256_sub_epi64(*ao, _mm256_sllv_epi64(_mm256_mul_epi32(xodd, c2), _mm256_add_epi64(sho, b)));
}

/* Rows [lo, hi) of the k-column Q4_K projection.  words: [cgroup][g][quad][lane] u32 (four
 * codes of column 8·cgroup + lane, zero for zero-scale groups and padding lanes); xs:
 * [cgroup][g][lane] i32; she/sho: [cgroup][g][4] i64 (e − emin of the even / odd columns);
 * emin per column; cspread per column group.  out[c·n_out + o].  Returns 0, or 1 when the
 * caller must redecide the call on the per-column path. */
int Q4K_NAME(const uint8_t *raw, size_t row_bytes, size_t sblocks, size_t lo, size_t hi,
             size_t k_cols, size_t n_in, const uint32_t *words, const int32_t *xs,
             const int64_t *she, const int64_t *sho, const uint32_t *emin,
             const uint32_t *cspread, uint32_t limit, const int8_t *codes,
             const int64_t *scales, int64_t *out, size_t n_out) {
  size_t G = sblocks * 8, groups = (k_cols + 7) / 8;
  uint8_t *wbuf = (uint8_t *)malloc(2 * n_in);
  int64_t *coef = (int64_t *)malloc(8 * G * sizeof(int64_t));
  if (!wbuf || !coef) {
    free(wbuf);
    free(coef);
    return 1;
  }
  q4k_row rr[2];
  for (int r = 0; r < 2; r++)
    rr[r] = (q4k_row){wbuf + r * n_in, coef + (4 * r) * G, coef + (4 * r + 1) * G,
                      coef + (4 * r + 2) * G, coef + (4 * r + 3) * G, 0, 0};
  int bail = 0;
  for (size_t o = lo; o < hi && !bail; o += 2) {
    int two = o + 1 < hi;
    const uint8_t *ra = raw + o * row_bytes, *rb = two ? ra + row_bytes : ra;
    if (q4k_row_prep(ra, sblocks, &rr[0]) || q4k_row_prep(rb, sblocks, &rr[1])) {
      bail = 1;
      break;
    }
    for (size_t cg = 0; cg < groups && !bail; cg++) {
      size_t c0 = cg * 8, nc = k_cols - c0 < 8 ? k_cols - c0 : 8;
      if (rr[0].spread + cspread[cg] > limit || rr[1].spread + cspread[cg] > limit) {
        __atomic_fetch_add(&apxo_q4k_exact_groups, 1, __ATOMIC_RELAXED);
        for (size_t c = c0; c < c0 + nc && !bail; c++)
          for (int r = 0; r <= two && !bail; r++)
            if (apxo_fast_row_value(APX_GGML_TYPE_Q4_K, r ? rb : ra, n_in, codes + c * n_in,
                                    scales + c * (n_in / 32), &out[c * n_out + o + r]))
              bail = 1;
        continue;
      }
      __m256i ae0 = _mm256_setzero_si256(), ao0 = ae0, ae1 = ae0, ao1 = ae0;
      const uint32_t *wg = words + cg * G * 64;
      for (size_t g = 0; g < G; g++) {
        const uint32_t *wq = wg + g * 64;
        const uint8_t *w0 = rr[0].w + g * 32, *w1 = rr[1].w + g * 32;
        __m256i d0 = _mm256_setzero_si256(), d1 = d0;
        for (int q = 0; q < 8; q++) {
          __m256i x = ld(wq + 8 * q);
          int32_t u0, u1;
          __builtin_memcpy(&u0, w0 + 4 * q, 4);
          __builtin_memcpy(&u1, w1 + 4 * q, 4);
          d0 = quad_dot(d0, _mm256_set1_epi32(u0), x);
          d1 = quad_dot(d1, _mm256_set1_epi32(u1), x);
        }
        size_t gi = cg * G + g;
        __m256i xv = ld(xs + gi * 8), she_v = ld(she + gi * 4), sho_v = ld(sho + gi * 4);
        q4k_fold(d0, xv, &rr[0], g, she_v, sho_v, &ae0, &ao0);
        q4k_fold(d1, xv, &rr[1], g, she_v, sho_v, &ae1, &ao1);
      }
      int64_t e0[4], od0[4], e1[4], od1[4];
      _mm256_storeu_si256((__m256i *)e0, ae0);
      _mm256_storeu_si256((__m256i *)od0, ao0);
      _mm256_storeu_si256((__m256i *)e1, ae1);
      _mm256_storeu_si256((__m256i *)od1, ao1);
      for (size_t c = 0; c < nc && !bail; c++) {
        int64_t v0 = c & 1 ? od0[c / 2] : e0[c / 2], v1 = c & 1 ? od1[c / 2] : e1[c / 2];
        if (apxo_finish(v0, rr[0].kmin + emin[c0 + c], &out[(c0 + c) * n_out + o]) ||
            (two && apxo_finish(v1, rr[1].kmin + emin[c0 + c], &out[(c0 + c) * n_out + o + 1])))
          bail = 1;
      }
    }
  }
  free(wbuf);
  free(coef);
  return bail;
}

/* ---- the k-column Q6_K projection (chart/kcols.rs:1466-1518) --------------------------------
 *
 * Q6_K weights are d·sc_h·(q − 32) over 16-lane groups h (q a 6-bit code, sc an int8).  Per
 * 16-lane group the unsigned codes are dotted against the token codes (u8 × i8, exact in
 * either instruction form: pair sums ≤ 2·63·127) and D_h = Σ q·x − 32·X_h (X_h = Σ x over the
 * group, |D_h| < 2^16) is folded as ((m_d·sc_h)·D_h) << (k_d − kmin + e − emin), a term below
 * 2^34, under lane_spread_limit(n_in / 16). */

#if APX_X86_VNNI
#define Q6K_NAME apxo_x86_q6k_rows_vnni
#else
#define Q6K_NAME apxo_x86_q6k_rows_avx2
#endif

void apxo_q6k_codes_u6(const uint8_t *blk, uint8_t *out);
extern unsigned long apxo_q6k_exact_groups;

typedef struct {
  uint8_t *w;  /* n_in unsigned codes */
  int64_t *c;  /* m_d·sc_h per 16-lane group */
  int64_t *a;  /* k_d − kmin per super-block */
  uint32_t kmin, spread;
} q6k_row;

static int q6k_row_prep(const uint8_t *row, size_t sblocks, q6k_row *r) {
  uint32_t kmin = UINT32_MAX, kmax = 0;
  int32_t md[Q4K_MAX_SBLOCKS];
  uint32_t kd[Q4K_MAX_SBLOCKS];
  for (size_t b = 0; b < sblocks; b++) {
    if (apxo_f16_split(word(row + b * 210 + 208), &md[b], &kd[b])) return 1;
    kmin = kd[b] < kmin ? kd[b] : kmin;
    kmax = kd[b] > kmax ? kd[b] : kmax;
  }
  for (size_t b = 0; b < sblocks; b++) {
    const uint8_t *blk = row + b * 210;
    apxo_q6k_codes_u6(blk, r->w + b * 256);
    for (int h = 0; h < 16; h++) r->c[b * 16 + h] = (int64_t)md[b] * (int8_t)blk[192 + h];
    r->a[b] = (int64_t)kd[b] - kmin;
  }
  r->kmin = kmin;
  r->spread = kmax - kmin;
  return 0;
}

static inline void q6k_fold(__m256i d, __m256i x16, int64_t c, int64_t a, __m256i she,
                            __m256i sho, __m256i *ae, __m256i *ao) {
  d = _mm256_sub_epi32(d, _mm256_slli_epi32(x16, 5));
  __m256i cv = _mm256_set1_epi64x(c), av = _mm256_set1_epi64x(a);
  *ae = _mm256_add_epi64(*ae, _mm256_sllv_epi64(_mm256_mul_epi32(d, cv), _mm256_add_epi64(she, av)));
  *ao = _mm256_add_epi64(*ao, _mm256_sllv_epi64(_mm256_mul_epi32(_mm256_srli_epi64(d, 32), cv),
                                                _mm256_add_epi64(sho, av)));
}

/* Rows [lo, hi) of the k-column Q6_K projection; the arguments are the Q4_K kernel's, with xs
 * per 16-lane group ([cgroup][n_in / 16][lane]). */
int Q6K_NAME(const uint8_t *raw, size_t row_bytes, size_t sblocks, size_t lo, size_t hi,
             size_t k_cols, size_t n_in, const uint32_t *words, const int32_t *xs,
             const int64_t *she, const int64_t *sho, const uint32_t *emin,
             const uint32_t *cspread, uint32_t limit, const int8_t *codes,
             const int64_t *scales, int64_t *out, size_t n_out) {
  size_t G = sblocks * 8, groups = (k_cols + 7) / 8;
  uint8_t *wbuf = (uint8_t *)malloc(2 * n_in);
  int64_t *coef = (int64_t *)malloc(2 * (16 + 1) * sblocks * sizeof(int64_t));
  if (!wbuf || !coef) {
    free(wbuf);
    free(coef);
    return 1;
  }
  q6k_row rr[2];
  for (int r = 0; r < 2; r++)
    rr[r] = (q6k_row){wbuf + r * n_in, coef + r * 17 * sblocks, coef + r * 17 * sblocks + 16 * sblocks,
                      0, 0};
  int bail = 0;
  for (size_t o = lo; o < hi && !bail; o += 2) {
    int two = o + 1 < hi;
    const uint8_t *ra = raw + o * row_bytes, *rb = two ? ra + row_bytes : ra;
    if (q6k_row_prep(ra, sblocks, &rr[0]) || q6k_row_prep(rb, sblocks, &rr[1])) {
      bail = 1;
      break;
    }
    for (size_t cg = 0; cg < groups && !bail; cg++) {
      size_t c0 = cg * 8, nc = k_cols - c0 < 8 ? k_cols - c0 : 8;
      if (rr[0].spread + cspread[cg] > limit || rr[1].spread + cspread[cg] > limit) {
        __atomic_fetch_add(&apxo_q6k_exact_groups, 1, __ATOMIC_RELAXED);
        for (size_t c = c0; c < c0 + nc && !bail; c++)
          for (int r = 0; r <= two && !bail; r++)
            if (apxo_fast_row_value(APX_GGML_TYPE_Q6_K, r ? rb : ra, n_in, codes + c * n_in,
                                    scales + c * (n_in / 32), &out[c * n_out + o + r]))
              bail = 1;
        continue;
      }
      __m256i ae0 = _mm256_setzero_si256(), ao0 = ae0, ae1 = ae0, ao1 = ae0;
      const uint32_t *wg = words + cg * G * 64;
      for (size_t g = 0; g < G; g++) { /* 32-lane activation groups: two 16-lane halves */
        size_t gi = cg * G + g;
        __m256i she_v = ld(she + gi * 4), sho_v = ld(sho + gi * 4);
        int64_t a0 = rr[0].a[g / 8], a1 = rr[1].a[g / 8];
        for (int h = 0; h < 2; h++) {
          const uint32_t *wq = wg + g * 64 + h * 32;
          const uint8_t *w0 = rr[0].w + g * 32 + h * 16, *w1 = rr[1].w + g * 32 + h * 16;
          __m256i d0 = _mm256_setzero_si256(), d1 = d0;
          for (int q = 0; q < 4; q++) {
            __m256i x = ld(wq + 8 * q);
            int32_t u0, u1;
            __builtin_memcpy(&u0, w0 + 4 * q, 4);
            __builtin_memcpy(&u1, w1 + 4 * q, 4);
            d0 = quad_dot(d0, _mm256_set1_epi32(u0), x);
            d1 = quad_dot(d1, _mm256_set1_epi32(u1), x);
          }
          size_t H = 2 * g + (size_t)h;
          __m256i x16 = ld(xs + (cg * 2 * G + H) * 8);
          q6k_fold(d0, x16, rr[0].c[H], a0, she_v, sho_v, &ae0, &ao0);
          q6k_fold(d1, x16, rr[1].c[H], a1, she_v, sho_v, &ae1, &ao1);
        }
      }
      int64_t e0[4], od0[4], e1[4], od1[4];
      _mm256_storeu_si256((__m256i *)e0, ae0);
      _mm256_storeu_si256((__m256i *)od0, ao0);
      _mm256_storeu_si256((__m256i *)e1, ae1);
      _mm256_storeu_si256((__m256i *)od1, ao1);
      for (size_t c = 0; c < nc && !bail; c++) {
        int64_t v0 = c & 1 ? od0[c / 2] : e0[c / 2], v1 = c & 1 ? od1[c / 2] : e1[c / 2];
        if (apxo_finish(v0, rr[0].kmin + emin[c0 + c], &out[(c0 + c) * n_out + o]) ||
            (two && apxo_finish(v1, rr[1].kmin + emin[c0 + c], &out[(c0 + c) * n_out + o + 1])))
          bail = 1;
      }
    }
  }
  free(wbuf);
  free(coef);
  return bail;
}

/* ---- the k-column Q8_0 rows without AVX-VNNI (kern/matmat.rs:198-206, pooled_q8_0) ----------
 *
 * Without AVX-VNNI the reference's matmat_q8act runs Q8_0 columns in runs of at most 16 over
 * one pass of each weight row (`q8_0_row_kcols_avx2`): a block's codes and scale are read once
 * and dotted against every column of the run (|w| · sign(x, w), `vpmaddubsw` + `vpmaddwd`),
 * each column folding `acc += d·(S·D)` in i128, the fast row's arithmetic. */

#if APX_X86_VNNI
#define KCOLS_NAME apxo_x86_q8_0_kcols_vnni
#else
#define KCOLS_NAME apxo_x86_q8_0_kcols_avx2
#endif

#define KCOLS_RUN 16

/* Rows [lo, hi) against k_cols columns (codes [c][n_in], S [c][n_in / 32]) in runs of 16;
 * out[c·n_out + o].  Returns 0, or 1 when the caller must redecide the call (a non-finite
 * scale or an output outside i64). */
int KCOLS_NAME(const uint8_t *raw, size_t row_bytes, size_t lo, size_t hi, size_t n_in,
               size_t k_cols, const int8_t *codes, const int64_t *S, const int64_t *tab,
               int64_t *out, size_t n_out) {
  size_t blocks = n_in / 32;
  for (size_t o = lo; o < hi; o++) {
    const uint8_t *row = raw + o * row_bytes;
    for (size_t c0 = 0; c0 < k_cols; c0 += KCOLS_RUN) {
      size_t nc = k_cols - c0 < KCOLS_RUN ? k_cols - c0 : KCOLS_RUN;
      i128 acc[KCOLS_RUN] = {0};
      int64_t bad = 0;
      for (size_t b = 0; b < blocks; b++) {
        const uint8_t *blk = row + b * Q8_0_BYTES;
        int64_t d = tab[word(blk)];
        bad |= d;
        __m256i w = ld(blk + 2);
        size_t c = 0;
        for (; c + 4 <= nc; c += 4) {
          const int8_t *x = codes + (c0 + c) * n_in + b * 32;
          int32_t dots[4];
          _mm_storeu_si128((__m128i *)dots,
                           sum4(dot_lanes(w, ld(x)), dot_lanes(w, ld(x + n_in)),
                                dot_lanes(w, ld(x + 2 * n_in)), dot_lanes(w, ld(x + 3 * n_in))));
          for (int j = 0; j < 4; j++)
            acc[c + j] += (i128)d * (i128)(S[(c0 + c + j) * blocks + b] * (int64_t)dots[j]);
        }
        for (; c < nc; c++) {
          int32_t dot = sum1(dot_lanes(w, ld(codes + (c0 + c) * n_in + b * 32)));
          acc[c] += (i128)d * (i128)(S[(c0 + c) * blocks + b] * (int64_t)dot);
        }
      }
      if (bad & 1) return 1;
      for (size_t c = 0; c < nc; c++)
        if (finish_row(acc[c], &out[(c0 + c) * n_out + o])) return 1;
    }
  }
  return 0;
}
