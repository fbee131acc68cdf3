// apx_swiglu.cuh — swiglu_one under the engine's carriers on the device (ops/ffn.rs:246-284).
//
//   F32 (the engine's default): g = from_q32(gate), u = from_q32(up) (RN(x)/2^32, fp.rs:176-178),
//       h = to_q32(silu(g)·u) with silu(x) = x / (1 + exp(-x)) in binary32 and exp the reference's
//       Cephes-style polynomial (mixer/f32_carrier.rs:262-375); every operation one IEEE binary32
//       rounding (the __f*_rn intrinsics: never contracted), Overflow where h leaves Q32.32;
//   Q32: h = round_shift_32(silu_fixed(gate)·up) (ops/silu.rs:53-100 on fixed_exp,
//       numeric/fixed_exp.rs:1-184), Overflow where h leaves i64.
//
// Shared by the FFN hidden-activation kernel (apx_ffn.cu) and the plan kernel's fused gate/up
// finish (apx_plan.cu).
#pragma once

#include <climits>

#include "apx_common.cuh"
#include "apx_quant.cuh"

namespace apx {

typedef __int128 i128;

constexpr int kFfnOverflow = 3;  // FfnError::Overflow (ops/ffn.rs:23-24)
constexpr long long kOne = 1ll << 32;

// ---- Q32 carrier ---------------------------------------------------------------------------

// round(v / 2^32), half away from zero (fixed_exp.rs round_div_2p32).
__device__ __forceinline__ i128 rdiv_2p32(i128 v) {
  const i128 half = (i128)1 << 31;
  return v >= 0 ? (v + half) >> 32 : -((-v + half) >> 32);
}

// fixed_exp: x = k·ln2 + r (k = round(x·log2 e), the product rounded at 2^64), the degree-7
// Taylor polynomial in r by Horner with each step rounded at 2^32, then a shift by k.  The
// constants are the reference's Q32.32 values of ln 2, 1/ln 2 and 1/i!.  false: out of range.
static __device__ bool fixed_exp_dev(long long x, long long &out) {
  if (x < -16 * kOne || x > 21 * kOne) return false;
  const i128 prod = (i128)x * (i128)6196328019ll;
  const i128 sh = (prod + ((i128)1 << 63)) >> 64;
  const long long k = (long long)sh;  // |x| <= 21·2^32: |k| <= 31
  const long long r = x - (long long)((i128)k * (i128)2977044472ll);
  const long long c[8] = {852176, 5965232, 35791394, 178956971, 715827883,
                          2147483648ll, 4294967296ll, 4294967296ll};
  i128 acc = c[0];
#pragma unroll
  for (int i = 1; i < 8; i++) acc = rdiv_2p32(acc * (i128)r) + c[i];
  i128 v;
  if (k >= 0) {
    v = acc << k;
  } else {
    const int n = (int)-k;
    v = (acc + ((i128)1 << (n - 1))) >> n;
  }
  if (v > (i128)LLONG_MAX || v < (i128)LLONG_MIN) return false;
  out = (long long)v;
  return true;
}

// silu_fixed: v >= 16 -> v, v <= -21 -> 0, else sign(v)·round(|v|·2^32 / (2^32 + e^-v)) with ties
// upward (value.rs:5-7).  In that window the denominator is positive and the quotient at most
// |v|, so only fixed_exp could refuse (it cannot for |v| < 21).  0 or the FfnError kind.
static __device__ int silu_fixed_dev(long long v, long long &out) {
  if (v >= 16 * kOne) {
    out = v;
    return 0;
  }
  if (v <= -21 * kOne) {
    out = 0;
    return 0;
  }
  long long e;
  if (!fixed_exp_dev(-v, e)) return 1;  // ExpOutOfRange
  const long long den = kOne + e;
  const i128 mag = v < 0 ? -(i128)v : (i128)v;
  const i128 q = (mag * (i128)kOne + (i128)(den / 2)) / (i128)den;
  out = (long long)(v < 0 ? -q : q);
  return 0;
}

// ---- F32 carrier ---------------------------------------------------------------------------

// exp_f32_scalar: the reference's binary32 exp (range reduction by n = rint(x·log2 e) with ln 2
// split in two, a degree-5 polynomial, and the scale 2^n applied in two halves), one rounding
// per operation.  The constants are its bit patterns.
__device__ __forceinline__ float exp_ref(float x) {
  if (x != x) return __int_as_float(0x7fc00000);
  if (x < __int_as_float((int)0xc2b00000u)) return 0.0f;
  if (x > __int_as_float(0x42b17218)) return __int_as_float(0x7f800000);
  const float z = __fmul_rn(x, __int_as_float(0x3fb8aa3b));
  const float n_flt = rintf(z);
  const int n_int = (int)n_flt;
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(n_flt, __int_as_float(0x3f318000))),
                            __fmul_rn(n_flt, __int_as_float((int)0xb95e8083u)));
  const float r2 = __fmul_rn(r, r);
  float p = __int_as_float(0x39506967);
  p = __fadd_rn(__fmul_rn(p, r), __int_as_float(0x3ab743ce));
  p = __fadd_rn(__fmul_rn(p, r), __int_as_float(0x3c088908));
  p = __fadd_rn(__fmul_rn(p, r), __int_as_float(0x3d2aa9c1));
  p = __fadd_rn(__fmul_rn(p, r), __int_as_float(0x3e2aaaaa));
  p = __fadd_rn(__fmul_rn(p, r), __int_as_float(0x3f000000));
  const float y = __fadd_rn(__fadd_rn(1.0f, r), __fmul_rn(r2, p));
  const int n1 = n_int >> 1, n2 = n_int - n1;
  return __fmul_rn(__fmul_rn(y, __int_as_float((n1 + 127) << 23)),
                   __int_as_float((n2 + 127) << 23));
}

// swiglu_one under the carrier: 0 (h set) or the FfnError kind.
static __device__ int swiglu_dev(long long gate, long long up, int carrier, long long &h) {
  if (carrier == APX_CARRIER_F32) {
    const float g = __fmul_rn(__ll2float_rn(gate), 0x1p-32f);
    const float u = __fmul_rn(__ll2float_rn(up), 0x1p-32f);
    const float s = __fdiv_rn(g, __fadd_rn(1.0f, exp_ref(-g)));
    const float prod = __fmul_rn(s, u);
    return f32_to_q32(prod, h) ? 0 : kFfnOverflow;  // false for non-finite or out of range
  }
  long long s;
  const int rc = silu_fixed_dev(gate, s);
  if (rc) return rc;
  const i128 v = ((i128)s * (i128)up + ((i128)1 << 31)) >> 32;  // round_shift_32
  if (v > (i128)LLONG_MAX || v < (i128)LLONG_MIN) return kFfnOverflow;
  h = (long long)v;
  return 0;
}

}  // namespace apx
