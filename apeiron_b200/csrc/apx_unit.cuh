// apx_unit.cuh — one 32-lane unit of the repacked layout seen by a warp: its weight registers,
// the exact fold of a unit against a staged activation slot, and the staging of that slot.
//
// Shared by the GEMV kernels (apx_gemv.cu) and the persistent plan kernel (apx_plan.cu).  A
// unit's weights are loaded first (they depend on nothing an earlier kernel writes); the fold
// reads the activation slot from shared memory, staged by the warp from 16-byte chunks of the
// codes with the per-block exponent data and Σxq each family needs.
#pragma once

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"

namespace apx {

// ---- per-unit exact accumulation ---------------------------------------------------------
// Each family splits a unit into its weight registers (loaded first, before anything the
// previous kernel produces is read) and the exact fold of those registers.

template <uint32_t T>
struct UnitRegs;
template <>
struct UnitRegs<kQ8_0> {
  uint4 q[8];
  uint2 s;
};
template <>
struct UnitRegs<kQ4_K> {
  uint4 q[8];
  uint4 h;
};
template <>
struct UnitRegs<kQ6_K> {
  uint4 q[12];
  uint4 sc;
  unsigned short d;
};

__device__ __forceinline__ void load_unit(UnitRegs<kQ8_0> &w, const uint8_t *ub, int lane) {
#pragma unroll
  for (int c = 0; c < 8; c++) w.q[c] = ld_stream(ub + (c * 32 + lane) * 16);
  w.s = ld_stream8(ub + 4096 + lane * 8);
}
__device__ __forceinline__ void load_unit(UnitRegs<kQ4_K> &w, const uint8_t *ub, int lane) {
#pragma unroll
  for (int c = 0; c < 8; c++) w.q[c] = ld_stream(ub + (c * 32 + lane) * 16);
  w.h = ld_stream(ub + 4096 + lane * 16);
}
__device__ __forceinline__ void load_unit(UnitRegs<kQ6_K> &w, const uint8_t *ub, int lane) {
#pragma unroll
  for (int c = 0; c < 12; c++) w.q[c] = ld_stream(ub + (c * 32 + lane) * 16);
  w.sc = ld_stream(ub + 6144 + lane * 16);
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(w.d) : "l"(ub + 6656 + lane * 2));
}

// The same registers from a unit already staged in shared memory.
__device__ __forceinline__ void load_unit_smem(UnitRegs<kQ8_0> &w, const uint8_t *ub, int lane) {
#pragma unroll
  for (int c = 0; c < 8; c++) w.q[c] = *reinterpret_cast<const uint4 *>(ub + (c * 32 + lane) * 16);
  w.s = *reinterpret_cast<const uint2 *>(ub + 4096 + lane * 8);
}
__device__ __forceinline__ void load_unit_smem(UnitRegs<kQ4_K> &w, const uint8_t *ub, int lane) {
#pragma unroll
  for (int c = 0; c < 8; c++) w.q[c] = *reinterpret_cast<const uint4 *>(ub + (c * 32 + lane) * 16);
  w.h = *reinterpret_cast<const uint4 *>(ub + 4096 + lane * 16);
}
__device__ __forceinline__ void load_unit_smem(UnitRegs<kQ6_K> &w, const uint8_t *ub, int lane) {
#pragma unroll
  for (int c = 0; c < 12; c++)
    w.q[c] = *reinterpret_cast<const uint4 *>(ub + (c * 32 + lane) * 16);
  w.sc = *reinterpret_cast<const uint4 *>(ub + 6144 + lane * 16);
  w.d = *reinterpret_cast<const unsigned short *>(ub + 6656 + lane * 2);
}

// Two views of a unit for the folds: its registers, loaded beforehand (RegView), or its copy in
// shared memory, each chunk read where the fold uses it (SmemView: fewer live registers).
template <uint32_t T>
struct RegView {
  const UnitRegs<T> &w;
  __device__ __forceinline__ uint4 chunk(int c) const { return w.q[c]; }
};
template <uint32_t T>
struct SmemView {
  const uint8_t *ub;
  int lane;
  __device__ __forceinline__ uint4 chunk(int c) const {
    return *reinterpret_cast<const uint4 *>(ub + (c * 32 + lane) * 16);
  }
};
__device__ __forceinline__ uint2 q8_scales(const RegView<kQ8_0> &v) { return v.w.s; }
__device__ __forceinline__ uint2 q8_scales(const SmemView<kQ8_0> &v) {
  return *reinterpret_cast<const uint2 *>(v.ub + 4096 + v.lane * 8);
}
__device__ __forceinline__ uint4 q4_head(const RegView<kQ4_K> &v) { return v.w.h; }
__device__ __forceinline__ uint4 q4_head(const SmemView<kQ4_K> &v) {
  return *reinterpret_cast<const uint4 *>(v.ub + 4096 + v.lane * 16);
}
__device__ __forceinline__ unsigned q6_word(const RegView<kQ6_K> &v, int k) {
  return reinterpret_cast<const unsigned *>(v.w.q)[k];
}
__device__ __forceinline__ unsigned q6_word(const SmemView<kQ6_K> &v, int k) {
  return *reinterpret_cast<const unsigned *>(v.ub + ((k / 4) * 32 + v.lane) * 16 + (k % 4) * 4);
}
__device__ __forceinline__ uint4 q6_scales(const RegView<kQ6_K> &v) { return v.w.sc; }
__device__ __forceinline__ uint4 q6_scales(const SmemView<kQ6_K> &v) {
  return *reinterpret_cast<const uint4 *>(v.ub + 6144 + v.lane * 16);
}
__device__ __forceinline__ unsigned q6_d(const RegView<kQ6_K> &v) { return v.w.d; }
__device__ __forceinline__ unsigned q6_d(const SmemView<kQ6_K> &v) {
  return *reinterpret_cast<const unsigned short *>(v.ub + 6656 + v.lane * 2);
}

template <class V>
__device__ __forceinline__ void fold_q8_0(Acc128 &acc, const V &w, const int *a,
                                          const int *eabs) {
#pragma unroll
  for (int bi = 0; bi < 4; bi++) {
    const int *x = a + bi * 8;
    const uint4 q0 = w.chunk(2 * bi), q1 = w.chunk(2 * bi + 1);
    int d = 0;
    d = dp4a_ss((int)q0.x, x[0], d);
    d = dp4a_ss((int)q0.y, x[1], d);
    d = dp4a_ss((int)q0.z, x[2], d);
    d = dp4a_ss((int)q0.w, x[3], d);
    d = dp4a_ss((int)q1.x, x[4], d);
    d = dp4a_ss((int)q1.y, x[5], d);
    d = dp4a_ss((int)q1.z, x[6], d);
    d = dp4a_ss((int)q1.w, x[7], d);
    const uint2 sv = q8_scales(w);
    unsigned bits = ((bi < 2 ? sv.x : sv.y) >> (16 * (bi & 1))) & 0xFFFFu;
    int m;
    unsigned k;
    f16_split(bits, m, k);
    int e = eabs[bi];
    if (e >= 0) acc_add_shl(acc, (long long)(m * d), k + (unsigned)e);
  }
}
__device__ __forceinline__ void fold_unit(Acc128 &acc, const UnitRegs<kQ8_0> &w, const int *a,
                                          const int *eabs, const long long *, int) {
  fold_q8_0(acc, RegView<kQ8_0>{w}, a, eabs);
}

__device__ __forceinline__ unsigned byte_of(unsigned w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Group p's two dots (low nibbles: group 2p, high nibbles in place as 16·D: group 2p+1).
template <class V>
__device__ __forceinline__ void q4k_dots(const V &w, const int *a, int p, int &dl,
                                         int &dh) {
  const uint4 w0 = w.chunk(2 * p), w1 = w.chunk(2 * p + 1);
  const int *xl = a + 16 * p, *xh = a + 16 * p + 8;
  dl = dp4a_us(w0.x & 0x0F0F0F0Fu, xl[0], 0);
  dl = dp4a_us(w0.y & 0x0F0F0F0Fu, xl[1], dl);
  dl = dp4a_us(w0.z & 0x0F0F0F0Fu, xl[2], dl);
  dl = dp4a_us(w0.w & 0x0F0F0F0Fu, xl[3], dl);
  dl = dp4a_us(w1.x & 0x0F0F0F0Fu, xl[4], dl);
  dl = dp4a_us(w1.y & 0x0F0F0F0Fu, xl[5], dl);
  dl = dp4a_us(w1.z & 0x0F0F0F0Fu, xl[6], dl);
  dl = dp4a_us(w1.w & 0x0F0F0F0Fu, xl[7], dl);
  dh = dp4a_us(w0.x & 0xF0F0F0F0u, xh[0], 0);
  dh = dp4a_us(w0.y & 0xF0F0F0F0u, xh[1], dh);
  dh = dp4a_us(w0.z & 0xF0F0F0F0u, xh[2], dh);
  dh = dp4a_us(w0.w & 0xF0F0F0F0u, xh[3], dh);
  dh = dp4a_us(w1.x & 0xF0F0F0F0u, xh[4], dh);
  dh = dp4a_us(w1.y & 0xF0F0F0F0u, xh[5], dh);
  dh = dp4a_us(w1.z & 0xF0F0F0F0u, xh[6], dh);
  dh = dp4a_us(w1.w & 0xF0F0F0F0u, xh[7], dh);
}

// er: the blocks' exponents relative to the call's smallest; xs: the blocks' Σxq.  When all
// eight exponents are at most kQ4Narrow, each group's terms are below 975360·63·2^2 in
// magnitude (|16·D| <= 16·32·15·127, scale <= 63) and eight of them stay below 2^31, so the
// super-block folds in int32; otherwise in int64 (the call's spread limit keeps that exact).
constexpr int kQ4Narrow = 2;
// ev: the eight group exponents relative to `ebase`, each in [0, emax8], emax8 <= es_limit.
template <class V>
__device__ __forceinline__ void fold_q4_k_ev(Acc128 &acc, const V &w, const int *a,
                                             const int (&ev)[8], int emax8, const long long *xs,
                                             int ebase) {
  // get_scale_min_k4 (format/quant.rs:482-491) for all 8 pairs at once.
  const uint4 h = q4_head(w);
  const unsigned sc_lo = h.y & 0x3F3F3F3Fu, mn_lo = h.z & 0x3F3F3F3Fu;
  const unsigned sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const unsigned mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  long long A16, B;
  if (emax8 <= kQ4Narrow) {
    int A32 = 0, B32 = 0;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      int dl, dh;
      q4k_dots(w, a, p, dl, dh);
      const int gl = 2 * p, gh = 2 * p + 1;
      const unsigned scl = byte_of(gl < 4 ? sc_lo : sc_hi, gl & 3);
      const unsigned sch = byte_of(gh < 4 ? sc_lo : sc_hi, gh & 3);
      const unsigned mnl = byte_of(gl < 4 ? mn_lo : mn_hi, gl & 3);
      const unsigned mnh = byte_of(gh < 4 ? mn_lo : mn_hi, gh & 3);
      A32 += (dl << 4) * (int)(scl << ev[gl]) + dh * (int)(sch << ev[gh]);
      B32 += (int)xs[gl] * (int)(mnl << ev[gl]) + (int)xs[gh] * (int)(mnh << ev[gh]);
    }
    A16 = A32;
    B = B32;
  } else {
    A16 = 0;
    B = 0;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      int dl, dh;
      q4k_dots(w, a, p, dl, dh);
      const int gl = 2 * p, gh = 2 * p + 1;
      const unsigned scl = byte_of(gl < 4 ? sc_lo : sc_hi, gl & 3);
      const unsigned sch = byte_of(gh < 4 ? sc_lo : sc_hi, gh & 3);
      const unsigned mnl = byte_of(gl < 4 ? mn_lo : mn_hi, gl & 3);
      const unsigned mnh = byte_of(gh < 4 ? mn_lo : mn_hi, gh & 3);
      A16 += (long long)(dl << 4) * (long long)(int)(scl << ev[gl]);
      A16 += (long long)dh * (long long)(int)(sch << ev[gh]);
      B += (xs[gl] << ev[gl]) * (long long)mnl + (xs[gh] << ev[gh]) * (long long)mnh;
    }
  }
  int md, mm;
  unsigned kd, km;
  f16_split(h.x & 0xFFFFu, md, kd);
  f16_split(h.x >> 16, mm, km);
  acc_add_shl(acc, (long long)md * A16, kd + (unsigned)ebase - 4u);
  acc_sub_shl(acc, (long long)mm * B, km + (unsigned)ebase);
}
__device__ __forceinline__ void load_ev8(const int *er, int (&ev)[8]) {
  const int4 e0 = reinterpret_cast<const int4 *>(er)[0], e1 = reinterpret_cast<const int4 *>(er)[1];
  ev[0] = e0.x; ev[1] = e0.y; ev[2] = e0.z; ev[3] = e0.w;
  ev[4] = e1.x; ev[5] = e1.y; ev[6] = e1.z; ev[7] = e1.w;
}
template <class V>
__device__ __forceinline__ void fold_q4_k(Acc128 &acc, const V &w, const int *a, const int *er,
                                          const long long *xs, int emin) {
  int ev[8];
  load_ev8(er, ev);
  const int emax8 = max(max(max(ev[0], ev[1]), max(ev[2], ev[3])),
                        max(max(ev[4], ev[5]), max(ev[6], ev[7])));
  fold_q4_k_ev(acc, w, a, ev, emax8, xs, emin);
}
__device__ __forceinline__ void fold_unit(Acc128 &acc, const UnitRegs<kQ4_K> &w, const int *a,
                                          const int *er, const long long *xs, int emin) {
  fold_q4_k(acc, RegView<kQ4_K>{w}, a, er, xs, emin);
}

// ev: the eight 32-element blocks' exponents relative to `ebase`, each at most es_limit; xs16
// the 16-element groups' Σxq, already shifted by their block's ev unless kShiftXs.
template <bool kShiftXs, class V>
__device__ __forceinline__ void fold_q6_k_ev(Acc128 &acc, const V &wr, const int *a,
                                             const int (&ev)[8], const long long *xs16,
                                             int ebase) {
  // ql words 0..31, qh words 32..47
  int du[16];
#pragma unroll
  for (int g = 0; g < 16; g++) du[g] = 0;
#pragma unroll
  for (int n = 0; n < 2; n++) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      unsigned ql0 = q6_word(wr, 16 * n + j), ql1 = q6_word(wr, 16 * n + 8 + j),
               qh = q6_word(wr, 32 + 8 * n + j);
      unsigned u1 = (ql0 & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
      unsigned u2 = (ql1 & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
      unsigned u3 = ((ql0 >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
      unsigned u4 = ((ql1 >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
      const int g = 8 * n + j / 4;
      du[g] = dp4a_us(u1, a[32 * n + j], du[g]);
      du[g + 2] = dp4a_us(u2, a[32 * n + 8 + j], du[g + 2]);
      du[g + 4] = dp4a_us(u3, a[32 * n + 16 + j], du[g + 4]);
      du[g + 6] = dp4a_us(u4, a[32 * n + 24 + j], du[g + 6]);
    }
  }
  const uint4 scv = q6_scales(wr);
  const unsigned scw[4] = {scv.x, scv.y, scv.z, scv.w};
  long long A = 0, B = 0;
#pragma unroll
  for (int g = 0; g < 16; g++) {
    int sc = (int)(signed char)byte_of(scw[g / 4], g % 4);
    A += (long long)du[g] * (long long)(sc * (1 << ev[g / 2]));
    B += (kShiftXs ? xs16[g] << ev[g / 2] : xs16[g]) * (long long)sc;
  }
  long long Tv = A - 32 * B;  // codes are u - 32 (format/quant.rs:574-599)
  int md;
  unsigned kd;
  f16_split(q6_d(wr), md, kd);
  acc_add_shl(acc, (long long)md * Tv, kd + (unsigned)ebase);
}
template <class V>
__device__ __forceinline__ void fold_q6_k(Acc128 &acc, const V &wr, const int *a, const int *er,
                                          const long long *xs16, int emin) {
  int ev[8];
  load_ev8(er, ev);
  fold_q6_k_ev<false>(acc, wr, a, ev, xs16, emin);
}
__device__ __forceinline__ void fold_unit(Acc128 &acc, const UnitRegs<kQ6_K> &wr, const int *a,
                                          const int *er, const long long *xs16, int emin) {
  fold_q6_k(acc, RegView<kQ6_K>{wr}, a, er, xs16, emin);
}

// The wide folds: each group's term goes into the 128-bit accumulator with its own shift, so any
// activation exponent spread folds exactly whenever the call-level bound holds (every partial
// sum is then inside i128, chart/mod.rs:362-383).  The fast folds above sum a super-block's
// groups in i64 first, which needs the spread within the family's es_limit.  er and xs as the
// staging writes them with `wide` set (Q6_K's Σxq unshifted).
template <class V>
__device__ __forceinline__ void fold_q4_k_wide(Acc128 &acc, const V &w, const int *a,
                                               const int *er, const long long *xs, int emin) {
  // Within one super-block the spread is usually small even when the call's is not: the
  // fast fold then runs on exponents relative to the super-block's own smallest.
  int ev[8];
  load_ev8(er, ev);
  const int lo = min(min(min(ev[0], ev[1]), min(ev[2], ev[3])), min(min(ev[4], ev[5]), min(ev[6], ev[7])));
  const int hi = max(max(max(ev[0], ev[1]), max(ev[2], ev[3])), max(max(ev[4], ev[5]), max(ev[6], ev[7])));
  if (hi - lo <= Fam<kQ4_K>::es_limit) {
#pragma unroll
    for (int i = 0; i < 8; i++) ev[i] -= lo;
    fold_q4_k_ev(acc, w, a, ev, hi - lo, xs, emin + lo);
    return;
  }
  const uint4 h = q4_head(w);
  const unsigned sc_lo = h.y & 0x3F3F3F3Fu, mn_lo = h.z & 0x3F3F3F3Fu;
  const unsigned sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const unsigned mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  int md, mm;
  unsigned kd, km;
  f16_split(h.x & 0xFFFFu, md, kd);
  f16_split(h.x >> 16, mm, km);
#pragma unroll
  for (int p = 0; p < 4; p++) {
    int dl, dh;
    q4k_dots(w, a, p, dl, dh);
    const int gl = 2 * p, gh = 2 * p + 1;
    const long long scl = byte_of(gl < 4 ? sc_lo : sc_hi, gl & 3);
    const long long sch = byte_of(gh < 4 ? sc_lo : sc_hi, gh & 3);
    const long long mnl = byte_of(gl < 4 ? mn_lo : mn_hi, gl & 3);
    const long long mnh = byte_of(gh < 4 ? mn_lo : mn_hi, gh & 3);
    // the low nibbles' dot is scaled by 16 to share the high nibbles' shift (kd + e - 4)
    acc_add_shl(acc, (long long)md * ((long long)(dl << 4) * scl),
                kd + (unsigned)(emin + er[gl]) - 4u);
    acc_add_shl(acc, (long long)md * ((long long)dh * sch), kd + (unsigned)(emin + er[gh]) - 4u);
    acc_sub_shl(acc, (long long)mm * (xs[gl] * mnl), km + (unsigned)(emin + er[gl]));
    acc_sub_shl(acc, (long long)mm * (xs[gh] * mnh), km + (unsigned)(emin + er[gh]));
  }
}

template <class V>
__device__ __forceinline__ void fold_q6_k_wide(Acc128 &acc, const V &wr, const int *a,
                                               const int *er, const long long *xs16, int emin) {
  int ev[8];  // as in fold_q4_k_wide: the fast fold relative to the super-block's smallest
  load_ev8(er, ev);
  const int lo = min(min(min(ev[0], ev[1]), min(ev[2], ev[3])), min(min(ev[4], ev[5]), min(ev[6], ev[7])));
  const int hi = max(max(max(ev[0], ev[1]), max(ev[2], ev[3])), max(max(ev[4], ev[5]), max(ev[6], ev[7])));
  if (hi - lo <= Fam<kQ6_K>::es_limit) {
#pragma unroll
    for (int i = 0; i < 8; i++) ev[i] -= lo;
    fold_q6_k_ev<true>(acc, wr, a, ev, xs16, emin + lo);
    return;
  }
  int du[16];
#pragma unroll
  for (int g = 0; g < 16; g++) du[g] = 0;
#pragma unroll
  for (int n = 0; n < 2; n++) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      unsigned ql0 = q6_word(wr, 16 * n + j), ql1 = q6_word(wr, 16 * n + 8 + j),
               qh = q6_word(wr, 32 + 8 * n + j);
      unsigned u1 = (ql0 & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
      unsigned u2 = (ql1 & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
      unsigned u3 = ((ql0 >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
      unsigned u4 = ((ql1 >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
      const int g = 8 * n + j / 4;
      du[g] = dp4a_us(u1, a[32 * n + j], du[g]);
      du[g + 2] = dp4a_us(u2, a[32 * n + 8 + j], du[g + 2]);
      du[g + 4] = dp4a_us(u3, a[32 * n + 16 + j], du[g + 4]);
      du[g + 6] = dp4a_us(u4, a[32 * n + 24 + j], du[g + 6]);
    }
  }
  const uint4 scv = q6_scales(wr);
  const unsigned scw[4] = {scv.x, scv.y, scv.z, scv.w};
  int md;
  unsigned kd;
  f16_split(q6_d(wr), md, kd);
#pragma unroll
  for (int g = 0; g < 16; g++) {
    const long long sc = (signed char)byte_of(scw[g / 4], g % 4);
    const long long t = (long long)du[g] * sc - 32 * xs16[g] * sc;  // codes are u - 32
    acc_add_shl(acc, (long long)md * t, kd + (unsigned)(emin + er[g / 2]));
  }
}

// The fold of a unit read from its copy in shared memory.
template <uint32_t T>
__device__ __forceinline__ void fold_unit_smem(Acc128 &acc, const uint8_t *ub, int lane,
                                               const int *a, const int *er, const long long *xs,
                                               int emin, bool wide = false) {
  if (T == kQ8_0) fold_q8_0(acc, SmemView<kQ8_0>{ub, lane}, a, er);  // per block already
  else if (T == kQ4_K && wide) fold_q4_k_wide(acc, SmemView<kQ4_K>{ub, lane}, a, er, xs, emin);
  else if (T == kQ4_K) fold_q4_k(acc, SmemView<kQ4_K>{ub, lane}, a, er, xs, emin);
  else if (wide) fold_q6_k_wide(acc, SmemView<kQ6_K>{ub, lane}, a, er, xs, emin);
  else fold_q6_k(acc, SmemView<kQ6_K>{ub, lane}, a, er, xs, emin);
}

// The same from the unit's registers.
__device__ __forceinline__ void fold_unit_wide(Acc128 &acc, const UnitRegs<kQ8_0> &w,
                                               const int *a, const int *eabs, const long long *,
                                               int) {
  fold_q8_0(acc, RegView<kQ8_0>{w}, a, eabs);
}
__device__ __forceinline__ void fold_unit_wide(Acc128 &acc, const UnitRegs<kQ4_K> &w,
                                               const int *a, const int *er, const long long *xs,
                                               int emin) {
  fold_q4_k_wide(acc, RegView<kQ4_K>{w}, a, er, xs, emin);
}
__device__ __forceinline__ void fold_unit_wide(Acc128 &acc, const UnitRegs<kQ6_K> &w,
                                               const int *a, const int *er, const long long *xs,
                                               int emin) {
  fold_q6_k_wide(acc, RegView<kQ6_K>{w}, a, er, xs, emin);
}


// The wide folds' condition: the call-level bound, and no code of -128 (those activations take
// the checked rows, as the fast path's do).
template <uint32_t T>
__device__ __forceinline__ bool wide_path(const ActDesc &desc, size_t n_in) {
  return desc.status == APX_OK && bound_ok((long long)n_in, Fam<T>::top, desc.emax) &&
         !(desc.pad[0] & 1u);
}

template <uint32_t T>
__device__ __forceinline__ bool fast_path(const ActDesc &desc, size_t n_in) {
  const int es = desc.emax >= 0 ? desc.emax - desc.emin : 0;
  return bound_ok((long long)n_in, Fam<T>::top, desc.emax) && es <= Fam<T>::es_limit &&
         !(desc.pad[0] & 1u);  // pad[0] bit 0: a code of -128 is present
}

// ---- activation staging --------------------------------------------------------------------
// A warp stages the activation of the L K-slots its unit covers: int8 codes (zero for a
// zero-scale block or past n_in), and per 32-lane block the exponent data and Σxq the
// family's fold reads.  Lanes load 16-byte chunks; slot s of the unit is chunks
// [s·span/16, (s+1)·span/16).

// A slot's codes are followed by 16 spare bytes, so that the L lanes of a row, which read
// the same offset of L different slots, fall into different shared-memory banks.
template <uint32_t T>
__host__ __device__ constexpr int slot_ints() { return Fam<T>::span / 4 + 4; }

template <uint32_t T>
struct WarpAct {
  int codes[4 * slot_ints<T>()];
  int e[4 * Fam<T>::span / 32];  // Q8_0: absolute exponent or -1; k-quants: er
  long long xs[4 * Fam<T>::nxs];  // Q6_K: Σxq·2^er per 16 lanes; Q4_K: Σxq per 32 lanes
};

struct Chunk {
  uint4 v;
  unsigned e;
};

// Chunk c of the activation whose first element is k_first (16 elements).
__device__ __forceinline__ Chunk load_chunk(const int8_t *codes, const uint8_t *exps,
                                            size_t n_in, size_t j) {
  Chunk s{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
  if (j < n_in) {
    s.e = exps[j / 32];
    if (j + 16 <= n_in && ((reinterpret_cast<uintptr_t>(codes + j) & 15) == 0)) {
      s.v = __ldg(reinterpret_cast<const uint4 *>(codes + j));
    } else {
      unsigned t[4] = {0, 0, 0, 0};
      for (int i = 0; i < 16; i++)
        if (j + i < n_in) t[i / 4] |= ((unsigned)(uint8_t)codes[j + i]) << (8 * (i % 4));
      s.v = make_uint4(t[0], t[1], t[2], t[3]);
    }
  }
  return s;
}

// The same for an activation written by this launch or the one before it: L2-coherent loads
// (the read-only path could hold a line from before the writer's store).
__device__ __forceinline__ Chunk load_chunk_cg(const int8_t *codes, const uint8_t *exps,
                                               size_t n_in, size_t j) {
  Chunk s{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
  if (j < n_in) {
    s.e = __ldcg(exps + j / 32);
    if (j + 16 <= n_in && ((reinterpret_cast<uintptr_t>(codes + j) & 15) == 0)) {
      s.v = __ldcg(reinterpret_cast<const uint4 *>(codes + j));
    } else {
      unsigned t[4] = {0, 0, 0, 0};
      for (int i = 0; i < 16; i++)
        if (j + i < n_in) t[i / 4] |= ((unsigned)(uint8_t)__ldcg(codes + j + i)) << (8 * (i % 4));
      s.v = make_uint4(t[0], t[1], t[2], t[3]);
    }
  }
  return s;
}

// Stage chunk c (of the staged region) with its sums; every lane of the warp calls this
// for the same c-round (the pair sum is a shuffle).
template <uint32_t T>
__device__ __forceinline__ void store_chunk(WarpAct<T> &w, Chunk s, int c, bool in, int emin,
                                            bool wide = false) {
  const bool zero = s.e == APX_EXP_ZERO;
  const uint4 v = zero ? make_uint4(0, 0, 0, 0) : s.v;
  const int er = zero ? 0 : (int)s.e - emin;
  int s16 = dp4a_ss((int)v.x, 0x01010101, 0);
  s16 = dp4a_ss((int)v.y, 0x01010101, s16);
  s16 = dp4a_ss((int)v.z, 0x01010101, s16);
  s16 = dp4a_ss((int)v.w, 0x01010101, s16);
  const int s32 = s16 + __shfl_xor_sync(0xFFFFFFFFu, s16, 1);
  if (!in) return;
  reinterpret_cast<uint4 *>(w.codes)[c + c / (Fam<T>::span / 16)] = v;  // past the slot pads
  if (T == kQ6_K) w.xs[c] = wide ? (long long)s16 : (long long)s16 << er;
  if ((c & 1) == 0) {
    w.e[c / 2] = T == kQ8_0 ? (zero ? -1 : (int)s.e) : er;
    if (T == kQ4_K) w.xs[c / 2] = s32;
  }
}

// Elements of chunk c of unit j (K-slots j·L .. j·L+L-1).
template <uint32_t T>
__device__ __forceinline__ size_t chunk_first(int j, int L, int c) {
  constexpr int per = Fam<T>::span / 16;
  return ((size_t)j * L + c / per) * Fam<T>::span + 16 * (size_t)(c % per);
}

}  // namespace apx
