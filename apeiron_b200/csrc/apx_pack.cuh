// apx_pack.cuh — the repacked weight layout seen from device code, and the checked row path.
//
// Shared by the GEMV (apx_gemv.cu) and the prefill GEMM (apx_gemm.cu): the family traits,
// where a row's K-slot lives in the packed units, the exact Q32.32 weight of one element,
// and matvec_fixed over one row with i128 overflow detection.
#pragma once

#include "apx_common.cuh"
#include "apx_kernels.h"

namespace apx {

// ---- family traits ---------------------------------------------------------------------

template <uint32_t T>
struct Fam;

template <>
struct Fam<kQ8_0> {
  static constexpr int span = 128;  // activation elements per K-slot
  static constexpr int unit_bytes = kUnitQ8_0;
  static constexpr int es_limit = 1 << 30;  // no spread limit: per-block i128 terms
  static constexpr long long top = 128;    // chart/mod.rs:1697
  static constexpr int nxs = 4;            // Σxq entries per K-slot (unused)
};
template <>
struct Fam<kQ4_K> {
  static constexpr int span = 256;
  static constexpr int unit_bytes = kUnitQ4_K;
  static constexpr int es_limit = 23;
  static constexpr long long top = 1008;  // chart/mod.rs:1703
  static constexpr int nxs = 8;           // per 32 lanes
};
template <>
struct Fam<kQ6_K> {
  static constexpr int span = 256;
  static constexpr int unit_bytes = kUnitQ6_K;
  static constexpr int es_limit = 22;
  static constexpr long long top = 4096;  // chart/mod.rs:1706
  static constexpr int nxs = 16;          // per 16 lanes
};

static __host__ __device__ int unit_bytes_of(uint32_t t) {
  return t == kQ8_0 ? kUnitQ8_0 : (t == kQ4_K ? kUnitQ4_K : kUnitQ6_K);
}

// The call-level bound of q8act_fast_bound_ok (chart/mod.rs:362-383):
// n_in·(65504·2^32)·top·127·S_max < 2^127 with S_max = 2^emax, decided exactly.
__device__ __forceinline__ bool bound_ok(long long n_in, long long top, int emax) {
  if (emax < 0) return true;  // every scale is zero
  // P = n_in·65504·top·127 < 2^64 for n_in < 2^29; need P < 2^(95 - emax).
  unsigned long long P = (unsigned long long)n_in * 65504ull * (unsigned long long)top * 127ull;
  int room = 95 - emax;
  if (room <= 0) return false;
  if (room >= 64) return true;
  return P < (1ull << room);
}

// Where row `row`'s K-slot `slot` lives: the unit's first byte and the lane inside it.
struct PackGeo {
  const uint8_t *pack;
  int units;  // units per row tile (K-slots / L, rounded up)
  int L;      // lanes per row
};

__host__ __device__ __forceinline__ const uint8_t *slot_unit(const PackGeo &g, uint32_t type,
                                                             size_t row, size_t slot,
                                                             int &lane) {
  const int H = 32 / g.L;
  const size_t rt = row / H;
  lane = (int)(row % H) * g.L + (int)(slot % g.L);
  return g.pack + (rt * g.units + slot / g.L) * (size_t)unit_bytes_of(type);
}
// ---- checked path: matvec_fixed in element order ------------------------------------------

// Exact Q32.32 weight of element i of `row` (dequant_row_fixed, src/engine/num/dequant.rs:
// 311-640, read from the repacked bytes).
template <uint32_t T>
__device__ long long weight_at(const PackGeo &g, size_t row, size_t i) {
  int lane;
  if (T == kQ8_0) {
    const uint8_t *ub = slot_unit(g, T, row, i / 128, lane);
    const int bi = (int)(i % 128) / 32, qi = (int)(i % 32);
    const int c = 2 * bi + qi / 16;
    const signed char code = (signed char)ub[(c * 32 + lane) * 16 + qi % 16];
    const unsigned bits = ub[4096 + lane * 8 + 2 * bi] | (ub[4096 + lane * 8 + 2 * bi + 1] << 8);
    int m;
    unsigned k;
    f16_split(bits, m, k);
    return ((long long)m << k) * code;
  } else if (T == kQ4_K) {
    const uint8_t *ub = slot_unit(g, T, row, i / 256, lane);
    const int p = (int)(i % 256);
    const int wb = 32 * (p / 64) + p % 32;
    const unsigned byte = ub[((wb / 16) * 32 + lane) * 16 + wb % 16];
    const unsigned code = (p % 64) < 32 ? (byte & 0xF) : (byte >> 4);
    const uint8_t *hd = ub + 4096 + lane * 16;
    const int j = p / 32;
    int sc, mn;
    if (j < 4) {
      sc = hd[4 + j] & 63;
      mn = hd[4 + j + 4] & 63;
    } else {
      sc = (hd[4 + j + 4] & 0xF) | ((hd[4 + j - 4] >> 6) << 4);
      mn = (hd[4 + j + 4] >> 4) | ((hd[4 + j] >> 6) << 4);
    }
    int md, mm;
    unsigned kd, km;
    f16_split(hd[0] | (hd[1] << 8), md, kd);
    f16_split(hd[2] | (hd[3] << 8), mm, km);
    const long long d = (long long)md << kd, dmin = (long long)mm << km;
    return (d * sc) * (long long)code - dmin * mn;
  } else {
    const uint8_t *ub = slot_unit(g, T, row, i / 256, lane);
    const int p = (int)(i % 256);
    const int n = p / 128, r = p % 128, quarter = r / 32, l = r % 32;
    const int qlb = 64 * n + l + ((quarter & 1) ? 32 : 0);
    const int qhb = 128 + 32 * n + l;
    const unsigned qlv = ub[((qlb / 16) * 32 + lane) * 16 + qlb % 16];
    const unsigned qhv = ub[((qhb / 16) * 32 + lane) * 16 + qhb % 16];
    const unsigned lo = quarter < 2 ? (qlv & 0xF) : (qlv >> 4);
    const int code = (int)(lo | (((qhv >> (2 * quarter)) & 3) << 4)) - 32;
    const int sc = (int)(signed char)ub[6144 + lane * 16 + p / 16];
    int md;
    unsigned kd;
    f16_split(ub[6656 + lane * 2] | (ub[6656 + lane * 2 + 1] << 8), md, kd);
    return (((long long)md << kd) * sc) * code;
  }
}

// 128-bit signed add with overflow detection.
__device__ __forceinline__ bool add_checked(Acc128 &a, long long plo, long long phi) {
  unsigned long long lo = a.lo + (unsigned long long)plo;
  unsigned long long carry = lo < a.lo ? 1ull : 0ull;
  long long hi = (long long)(a.hi + (unsigned long long)phi + carry);
  bool ovf = ((long long)a.hi >= 0) == (phi >= 0) && ((hi >= 0) != (phi >= 0));
  a.lo = lo;
  a.hi = (unsigned long long)hi;
  return !ovf;
}

// This output also into the other ranks' gather buffers (constant indices: no local copy of
// the parameter block).
__device__ __forceinline__ void store_peers(const PeerRows &pr, size_t row, long long v) {
#pragma unroll
  for (int i = 0; i < 7; i++)
    if (i < pr.n) pr.dst[i][row] = v;
}

// matvec_fixed of one row: whether it produced an output, and the output.
struct RowOut {
  long long v;
  bool ok;
};

template <uint32_t T>
__device__ __noinline__ RowOut checked_row(const PackGeo g, size_t row, size_t n_out,
                                           size_t n_in, const int8_t *codes, const uint8_t *exps,
                                           long long *out_q32, float *out_f32,
                                           unsigned long long *status) {
  if (row >= n_out) return RowOut{0, false};
  Acc128 acc;
  acc_zero(acc);
  for (size_t i = 0; i < n_in; i++) {
    const unsigned e = exps[i / 32];
    // S·xq fits i64: the descriptor refused every activation where it does not
    const long long x = e == APX_EXP_ZERO ? 0 : (long long)codes[i] * (1ll << e);
    const long long w = weight_at<T>(g, row, i);
    if (!add_checked(acc, w * x, __mul64hi(w, x))) {
      atomicMin(status, pack_status(row, kKindAccOverflow, 0));
      return RowOut{0, false};
    }
  }
  long long v;
  if (!acc_round_to_i64(acc, v)) {
    atomicMin(status, pack_status(row, kKindOutputOverflow, 0));
    return RowOut{0, false};
  }
  if (out_q32) out_q32[row] = v;
  if (out_f32) out_f32[row] = __ll2float_rn(v) * 2.3283064365386963e-10f;
  return RowOut{v, true};
}

__device__ __forceinline__ void finish_row(const Acc128 &s, size_t row, size_t n_out,
                                           long long *out_q32, float *out_f32,
                                           unsigned long long *status, const PeerRows &peers) {
  if (row >= n_out) return;
  long long v;
  if (!acc_round_to_i64(s, v)) {
    atomicMin(status, pack_status(row, kKindOutputOverflow, 0));
  } else {
    if (out_q32) out_q32[row] = v;
    if (out_f32) out_f32[row] = __ll2float_rn(v) * 2.3283064365386963e-10f;
    store_peers(peers, row, v);
  }
}

// Programmatic dependent launch: the next projection may start streaming its (constant)
// weights as soon as every CTA of this one is running; it waits for this grid's completion
// before it reads anything this grid or an earlier kernel writes.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace apx
