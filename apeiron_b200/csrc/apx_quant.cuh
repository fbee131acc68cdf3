// apx_quant.cuh — the activation quantizer's per-block arithmetic, shared by the quantization
// kernels (apx_quant.cu) and the prefill GEMM's fused quantize-and-prep kernel (apx_gemm.cu).
//
// quant_act (src/engine/chart/mod.rs:258-334) after f32_to_fixed (F32::to_q32,
// src/engine/num/fp.rs:186-230): per 32-lane block the smallest S = 2^e with 127·S >= absmax
// (act_scale, src/engine/kern/pow2.rs:22-39), codes round(|x|/S) ties away from zero, refusal
// exactly where the reference returns None.
#pragma once

#include "apx_common.cuh"

namespace apx {

__device__ __forceinline__ unsigned long long uabs64(long long v) {
  return v < 0 ? 0ull - (unsigned long long)v : (unsigned long long)v;
}

// act_scale exponent, or -1 for a zero block, or 99 when the reference returns None: the
// smallest e >= 0 with 127·2^e >= absmax (pow2.rs:22-39).  With bl the bit length of absmax
// and e0 = max(0, bl − 7), 127·2^(e0−1) < 2^(bl−1) <= absmax, so e is e0 or e0 + 1; 127·2^e0
// stays below 2^64 for every absmax <= 2^63.  No division.
__device__ __forceinline__ int act_scale_exp(unsigned long long absmax) {
  if (absmax == 0) return -1;
  const int bl = 64 - __clzll((long long)absmax);
  const int e0 = bl > 7 ? bl - 7 : 0;
  const int e = (127ull << e0) >= absmax ? e0 : e0 + 1;
  return e > 62 ? 99 : e;
}

// S·code fits i64 for S = 2^e (QuantAct::dequant's checked product).
__device__ __forceinline__ bool product_fits(int code, int e) {
  if (e <= 56) return true;  // 128·2^56 = 2^63: every int8 code fits except -128·2^56 = i64::MIN
  long long lim = 1ll << (63 - e);
  return code >= -lim && code <= lim - 1;
}

// F32::to_q32 (src/engine/num/fp.rs:186-230): round(v·2^32), ties away from zero.
__device__ __forceinline__ bool f32_to_q32(float f, long long &out) {
  unsigned bits = __float_as_uint(f);
  unsigned e = (bits >> 23) & 0xFFu;
  if (e == 0xFFu) return false;
  unsigned frac = bits & 0x007FFFFFu;
  unsigned long long m = e == 0 ? frac : (frac | 0x00800000u);
  bool neg = (bits & 0x80000000u) != 0;
  unsigned ee = e == 0 ? 1 : e;
  unsigned long long mag;
  if (ee >= 118) {
    unsigned k = ee - 118;
    if (k > 40) return false;
    if (k >= 40 && m >= (1ull << 23)) {
      // m·2^k >= 2^63: the positive side refuses, the negative side only at exactly 2^63
      if (neg && m == (1ull << 23)) {
        out = (long long)(1ull << 63);
        return true;
      }
      return false;
    }
    mag = m << k;
  } else {
    unsigned sh = 118 - ee;
    mag = sh > 24 ? 0ull : (m + (1ull << (sh - 1))) >> sh;
  }
  const unsigned long long lim = 1ull << 63;
  if (neg) {
    if (mag > lim) return false;
    out = mag == lim ? (long long)lim : -(long long)mag;
    return true;
  }
  if (mag >= lim) return false;
  out = (long long)mag;
  return true;
}

// Round-half-up right shift of a value below 2^25 (0 for shifts past its bit length).
__device__ __forceinline__ unsigned rshift_round(unsigned x, unsigned s) {
  return s == 0 ? x : s > 25 ? 0u : (x + (1u << (s - 1))) >> s;
}

// Largest |f| bit pattern the 32-bit route takes: 127·2^24.  Below it every lane converts,
// act_scale gives e <= 56 and every code times 2^e fits i64, so nothing refuses.
constexpr unsigned kFastAbsMax = 0x4EFE0000u;

// act_scale exponent of a block whose largest |f| has bit pattern A <= kFastAbsMax, from the
// f32 fields: with M the 24-bit significand and E the biased exponent, round(A·2^32) is
// M·2^(E−118) for E >= 118 (bit length E − 94, so e = E − 101 or one more when M > 127·2^17),
// and below that a value under 2^25 formed by one rounding shift.
__device__ __forceinline__ int fast_scale_exp(unsigned A) {
  const unsigned E = A >> 23, M = (A & 0x7FFFFFu) | (E ? 0x800000u : 0u);
  if (E >= 118) return (int)E - 101 + (M > 0xFE0000u ? 1 : 0);
  const unsigned vm = rshift_round(M, 118 - (E ? E : 1));
  if (vm == 0) return -1;
  const int bl = 32 - __clz((int)vm);
  const int e0 = bl > 7 ? bl - 7 : 0;
  return (127u << e0) >= vm ? e0 : e0 + 1;
}

// Code of one lane (f32 bits) under block exponent e >= 0: round(|f|·2^32) then round by 2^e,
// ties away from zero both times.  Where round(|f|·2^32) is exact (E >= 118) the two
// roundings are one shift of the significand.
__device__ __forceinline__ int fast_code(unsigned bits, int e) {
  const unsigned b = bits & 0x7FFFFFFFu, E = b >> 23, M = (b & 0x7FFFFFu) | (E ? 0x800000u : 0u);
  const unsigned mag = E >= 118 ? rshift_round(M, (unsigned)e + 118 - E)
                                : rshift_round(rshift_round(M, 118 - (E ? E : 1)), (unsigned)e);
  return (bits >> 31) ? -(int)mag : (int)mag;
}

// One thread's four consecutive lanes (one 16-byte load) of a 32-lane block, the block's 8
// threads together (every lane of the warp calls this for the same round: the block decisions
// are shuffles within 8-lane groups).  Blocks whose absmax is at most kFastAbsMax take 32-bit
// arithmetic on the f32 fields; a warp holding any other block takes the Q32.32 route
// (f32_to_q32, act_scale, checked product) for all its lanes.  packed: the four int8 codes;
// e: the block's exponent (-1 for a zero block); blk_ok: false when the reference refuses it.
__device__ __forceinline__ void quant_quad(const float4 f4, uint32_t &packed, int &e,
                                           bool &blk_ok) {
  const unsigned bits[4] = {__float_as_uint(f4.x), __float_as_uint(f4.y),
                            __float_as_uint(f4.z), __float_as_uint(f4.w)};
  unsigned amax = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) amax = max(amax, bits[k] & 0x7FFFFFFFu);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  e = -1;
  packed = 0;
  blk_ok = true;
  if (__all_sync(0xFFFFFFFFu, amax <= kFastAbsMax)) {
    e = fast_scale_exp(amax);
    if (e >= 0) {
#pragma unroll
      for (int k = 0; k < 4; k++)
        packed |= ((uint32_t)(uint8_t)(int8_t)fast_code(bits[k], e)) << (8 * k);
    }
  } else {
    // Q32.32 route (f32_to_q32, act_scale, checked product) for every lane of the warp
    long long v[4];
    bool ok = true;
#pragma unroll
    for (int k = 0; k < 4; k++) ok &= f32_to_q32(__uint_as_float(bits[k]), v[k]);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ok &= __shfl_xor_sync(0xFFFFFFFFu, (int)ok, o) != 0;
    blk_ok = ok;
    if (blk_ok) {
      long long vm;
      const unsigned long long mx =
          f32_to_q32(__uint_as_float(amax), vm) ? (unsigned long long)vm : 1ull << 63;
      e = act_scale_exp(mx);
      if (e == 99) blk_ok = false;
    }
    bool bad = false;
    if (blk_ok && e >= 0) {
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const unsigned long long m = uabs64(v[k]);
        const unsigned long long S = 1ull << e, q = m >> e, r = m & (S - 1);
        const unsigned long long mag = q + (2 * r >= S ? 1ull : 0ull);
        const int code = v[k] < 0 ? -(int)mag : (int)mag;
        bad |= mag > 127 || !product_fits(code, e);
        packed |= ((uint32_t)(uint8_t)(int8_t)code) << (8 * k);
      }
    }
    // every lane takes part in the group reduction (the branch above is group-dependent)
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) bad |= __shfl_xor_sync(0xFFFFFFFFu, (int)bad, o) != 0;
    if (bad) blk_ok = false;
  }
}

}  // namespace apx
