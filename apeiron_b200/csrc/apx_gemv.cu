// apx_gemv.cu — exact Q8-activation GEMV for GGUF Q8_0 / Q4_K / Q6_K on sm_100a.
//
// Contract (src/engine/chart/mod.rs:1887-1925): out[r] = round_shift_32(Σ_i w_ri·x̂_i) with
// w the Q32.32 dequantized weight and x̂_i = S_b·xq_i, i.e. `matvec_fixed(W, dequant(q))`
// (src/engine/ops/matvec.rs:149-222), bit for bit, with the same refusals.
//
// Layout in HBM.  At upload each tensor is regrouped once into units of 32 rows (one row per
// lane) × one K-slice: 4 Q8_0 blocks, or one Q4_K / Q6_K super-block.  Inside a unit the
// 16-byte chunk c of lane l sits at (c*32 + l)*16, so every warp-wide 16-byte load reads 512
// contiguous bytes; the per-row block headers follow the chunks.  The bytes are the GGUF
// bytes, only their positions change (format/quant.rs:52-68 block layouts).
//
// Work.  One warp streams one unit: lane l owns row 32*rt + l and accumulates its exact
// contribution in a 128-bit integer (apx_common.cuh).  The activation codes of the CTA's
// K-range live in shared memory and are read as warp-wide broadcasts.  Units of one row tile
// are spread over the warps of a CTA and, for long rows, over the CTAs of a thread-block
// cluster; partial sums meet in shared memory and then through distributed shared memory.
//
// Exactness.  The kernels run when every partial sum is provably inside i128 (the reference's
// call-level bound q8act_fast_bound_ok, chart/mod.rs:362-383, evaluated from the largest
// activation exponent) and the activation exponent spread fits the family's i64 super-block
// fold; otherwise the same kernel takes the checked path, one lane per row summing
// Σ w_i·x̂_i in element order with i128 overflow detection, which is matvec_fixed itself.
#include <algorithm>
#include <cstdlib>

#include "apx_common.cuh"
#include "apx_kernels.h"

namespace apx {

// ---- upload-time repack ----------------------------------------------------------------

__global__ void repack_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ pack,
                              uint32_t type, size_t n_out, size_t row_bytes, int units,
                              int nblk, size_t total) {
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    int unit_bytes = type == kQ8_0 ? kUnitQ8_0 : (type == kQ4_K ? kUnitQ4_K : kUnitQ6_K);
    size_t unit = idx / unit_bytes;
    int off = (int)(idx % unit_bytes);
    size_t rt = unit / units;
    int u = (int)(unit % units);
    int lane, blk;
    size_t src;  // byte offset inside the row
    if (type == kQ8_0) {
      if (off < 4096) {
        int c = off / 512, i = off % 16;
        lane = (off / 16) % 32;
        blk = 4 * u + c / 2;
        src = (size_t)blk * 34 + 2 + 16 * (c % 2) + i;
      } else {
        int o2 = off - 4096;
        lane = o2 / 8;
        blk = 4 * u + (o2 % 8) / 2;
        src = (size_t)blk * 34 + (o2 % 2);
      }
    } else if (type == kQ4_K) {
      blk = u;
      if (off < 4096) {
        lane = (off / 16) % 32;
        src = (size_t)u * 144 + 16 + 16 * (off / 512) + off % 16;
      } else {
        lane = (off - 4096) / 16;
        src = (size_t)u * 144 + (off - 4096) % 16;
      }
    } else {
      blk = u;
      if (off < 6144) {
        lane = (off / 16) % 32;
        src = (size_t)u * 210 + 16 * (off / 512) + off % 16;
      } else if (off < 6656) {
        lane = (off - 6144) / 16;
        src = (size_t)u * 210 + 192 + (off - 6144) % 16;
      } else {
        lane = (off - 6656) / 2;
        src = (size_t)u * 210 + 208 + (off - 6656) % 2;
      }
    }
    size_t row = rt * 32 + lane;
    pack[idx] = (row < n_out && blk < nblk) ? raw[row * row_bytes + src] : (uint8_t)0;
  }
}

// ---- family traits ---------------------------------------------------------------------

template <uint32_t T>
struct Fam;

template <>
struct Fam<kQ8_0> {
  static constexpr int span = 128;  // activation elements per unit
  static constexpr int unit_bytes = kUnitQ8_0;
  static constexpr int es_limit = 1 << 30;  // no spread limit: per-block i128 terms
  static constexpr long long top = 128;    // chart/mod.rs:1697
};
template <>
struct Fam<kQ4_K> {
  static constexpr int span = 256;
  static constexpr int unit_bytes = kUnitQ4_K;
  static constexpr int es_limit = 23;
  static constexpr long long top = 1008;  // chart/mod.rs:1703
};
template <>
struct Fam<kQ6_K> {
  static constexpr int span = 256;
  static constexpr int unit_bytes = kUnitQ6_K;
  static constexpr int es_limit = 22;
  static constexpr long long top = 4096;  // chart/mod.rs:1706
};

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

__device__ __forceinline__ void fold_unit(Acc128 &acc, const UnitRegs<kQ8_0> &w, const int *a,
                                          const int *eabs, const long long *, int) {
#pragma unroll
  for (int bi = 0; bi < 4; bi++) {
    const int *x = a + bi * 8;
    const uint4 q0 = w.q[2 * bi], q1 = w.q[2 * bi + 1];
    int d = 0;
    d = dp4a_ss((int)q0.x, x[0], d);
    d = dp4a_ss((int)q0.y, x[1], d);
    d = dp4a_ss((int)q0.z, x[2], d);
    d = dp4a_ss((int)q0.w, x[3], d);
    d = dp4a_ss((int)q1.x, x[4], d);
    d = dp4a_ss((int)q1.y, x[5], d);
    d = dp4a_ss((int)q1.z, x[6], d);
    d = dp4a_ss((int)q1.w, x[7], d);
    unsigned bits = ((bi < 2 ? w.s.x : w.s.y) >> (16 * (bi & 1))) & 0xFFFFu;
    int m;
    unsigned k;
    f16_split(bits, m, k);
    int e = eabs[bi];
    if (e >= 0) acc_add_shl(acc, (long long)(m * d), k + (unsigned)e);
  }
}

__device__ __forceinline__ unsigned byte_of(unsigned w, int i) { return (w >> (8 * i)) & 0xFFu; }

__device__ __forceinline__ void fold_unit(Acc128 &acc, const UnitRegs<kQ4_K> &w, const int *a,
                                          const int *er, const long long *xs, int emin) {
  // get_scale_min_k4 (format/quant.rs:482-491) for all 8 pairs at once.
  const uint4 h = w.h;
  unsigned sc_lo = h.y & 0x3F3F3F3Fu, mn_lo = h.z & 0x3F3F3F3Fu;
  unsigned sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  unsigned mn_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  long long A16 = 0, B = 0;
#pragma unroll
  for (int p = 0; p < 4; p++) {
    const uint4 w0 = w.q[2 * p], w1 = w.q[2 * p + 1];
    const int *xl = a + 16 * p, *xh = a + 16 * p + 8;
    int dl = 0, dh = 0;
    dl = dp4a_us(w0.x & 0x0F0F0F0Fu, xl[0], dl);
    dl = dp4a_us(w0.y & 0x0F0F0F0Fu, xl[1], dl);
    dl = dp4a_us(w0.z & 0x0F0F0F0Fu, xl[2], dl);
    dl = dp4a_us(w0.w & 0x0F0F0F0Fu, xl[3], dl);
    dl = dp4a_us(w1.x & 0x0F0F0F0Fu, xl[4], dl);
    dl = dp4a_us(w1.y & 0x0F0F0F0Fu, xl[5], dl);
    dl = dp4a_us(w1.z & 0x0F0F0F0Fu, xl[6], dl);
    dl = dp4a_us(w1.w & 0x0F0F0F0Fu, xl[7], dl);
    // high nibbles in place: the dot comes out as 16·D
    dh = dp4a_us(w0.x & 0xF0F0F0F0u, xh[0], dh);
    dh = dp4a_us(w0.y & 0xF0F0F0F0u, xh[1], dh);
    dh = dp4a_us(w0.z & 0xF0F0F0F0u, xh[2], dh);
    dh = dp4a_us(w0.w & 0xF0F0F0F0u, xh[3], dh);
    dh = dp4a_us(w1.x & 0xF0F0F0F0u, xh[4], dh);
    dh = dp4a_us(w1.y & 0xF0F0F0F0u, xh[5], dh);
    dh = dp4a_us(w1.z & 0xF0F0F0F0u, xh[6], dh);
    dh = dp4a_us(w1.w & 0xF0F0F0F0u, xh[7], dh);
    const int gl = 2 * p, gh = 2 * p + 1;
    unsigned scl = byte_of(gl < 4 ? sc_lo : sc_hi, gl & 3);
    unsigned sch = byte_of(gh < 4 ? sc_lo : sc_hi, gh & 3);
    unsigned mnl = byte_of(gl < 4 ? mn_lo : mn_hi, gl & 3);
    unsigned mnh = byte_of(gh < 4 ? mn_lo : mn_hi, gh & 3);
    A16 += (long long)(dl << 4) * (long long)(int)(scl << er[gl]);
    A16 += (long long)dh * (long long)(int)(sch << er[gh]);
    B += xs[gl] * (long long)mnl + xs[gh] * (long long)mnh;
  }
  int md, mm;
  unsigned kd, km;
  f16_split(h.x & 0xFFFFu, md, kd);
  f16_split(h.x >> 16, mm, km);
  acc_add_shl(acc, (long long)md * A16, kd + (unsigned)emin - 4u);
  acc_sub_shl(acc, (long long)mm * B, km + (unsigned)emin);
}

__device__ __forceinline__ void fold_unit(Acc128 &acc, const UnitRegs<kQ6_K> &wr, const int *a,
                                          const int *er, const long long *xs16, int emin) {
  const unsigned *w = reinterpret_cast<const unsigned *>(wr.q);  // ql words 0..31, qh 32..47
  int du[16];
#pragma unroll
  for (int g = 0; g < 16; g++) du[g] = 0;
#pragma unroll
  for (int n = 0; n < 2; n++) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      unsigned ql0 = w[16 * n + j], ql1 = w[16 * n + 8 + j], qh = w[32 + 8 * n + j];
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
  const unsigned scw[4] = {wr.sc.x, wr.sc.y, wr.sc.z, wr.sc.w};
  long long A = 0, B = 0;
#pragma unroll
  for (int g = 0; g < 16; g++) {
    int sc = (int)(signed char)byte_of(scw[g / 4], g % 4);
    A += (long long)du[g] * (long long)(sc * (1 << er[g / 2]));
    B += xs16[g] * (long long)sc;
  }
  long long Tv = A - 32 * B;  // codes are u - 32 (format/quant.rs:574-599)
  int md;
  unsigned kd;
  f16_split(wr.d, md, kd);
  acc_add_shl(acc, (long long)md * Tv, kd + (unsigned)emin);
}

// ---- checked path: matvec_fixed in element order ------------------------------------------

// Exact Q32.32 weight of element i of the row held by `lane` in row tile `rt`
// (dequant_row_fixed, src/engine/num/dequant.rs:311-640, from the repacked bytes).
template <uint32_t T>
__device__ long long weight_at(const uint8_t *pack, int units, size_t rt, int lane, size_t i) {
  if (T == kQ8_0) {
    size_t b = i / 32;
    const uint8_t *ub = pack + (rt * units + b / 4) * (size_t)kUnitQ8_0;
    int bi = (int)(b % 4), qi = (int)(i % 32);
    int c = 2 * bi + qi / 16;
    signed char code = (signed char)ub[(c * 32 + lane) * 16 + qi % 16];
    unsigned bits = ub[4096 + lane * 8 + 2 * bi] | (ub[4096 + lane * 8 + 2 * bi + 1] << 8);
    int m;
    unsigned k;
    f16_split(bits, m, k);
    return ((long long)m << k) * code;
  } else if (T == kQ4_K) {
    size_t s = i / 256;
    int p = (int)(i % 256);
    const uint8_t *ub = pack + (rt * units + s) * (size_t)kUnitQ4_K;
    int wb = 32 * (p / 64) + p % 32;
    unsigned byte = ub[((wb / 16) * 32 + lane) * 16 + wb % 16];
    unsigned code = (p % 64) < 32 ? (byte & 0xF) : (byte >> 4);
    const uint8_t *hd = ub + 4096 + lane * 16;
    int j = p / 32, sc, mn;
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
    long long d = (long long)md << kd, dmin = (long long)mm << km;
    return (d * sc) * (long long)code - dmin * mn;
  } else {
    size_t s = i / 256;
    int p = (int)(i % 256);
    const uint8_t *ub = pack + (rt * units + s) * (size_t)kUnitQ6_K;
    int n = p / 128, r = p % 128, quarter = r / 32, l = r % 32;
    int qlb = 64 * n + l + ((quarter & 1) ? 32 : 0);
    int qhb = 128 + 32 * n + l;
    unsigned qlv = ub[((qlb / 16) * 32 + lane) * 16 + qlb % 16];
    unsigned qhv = ub[((qhb / 16) * 32 + lane) * 16 + qhb % 16];
    unsigned lo = quarter < 2 ? (qlv & 0xF) : (qlv >> 4);
    int code = (int)(lo | (((qhv >> (2 * quarter)) & 3) << 4)) - 32;
    int sc = (int)(signed char)ub[6144 + lane * 16 + p / 16];
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

template <uint32_t T>
__device__ __noinline__ void checked_rows(const uint8_t *pack, int units, size_t rt, int lane,
                                          size_t n_out, size_t n_in, const int8_t *codes,
                                          const uint8_t *exps, long long *out_q32,
                                          float *out_f32, unsigned long long *status) {
  size_t row = rt * 32 + lane;
  if (row >= n_out) return;
  Acc128 acc;
  acc_zero(acc);
  for (size_t i = 0; i < n_in; i++) {
    unsigned e = exps[i / 32];
    long long x = e == APX_EXP_ZERO ? 0 : (long long)codes[i] << e;  // fits: desc checked
    long long w = weight_at<T>(pack, units, rt, lane, i);
    long long plo = w * x;                          // low 64 bits of the exact product
    long long phi = __mul64hi(w, x);                // high 64 bits
    if (!add_checked(acc, plo, phi)) {
      atomicMin(status, pack_status(row, kKindAccOverflow, 0));
      return;
    }
  }
  long long v;
  if (!acc_round_to_i64(acc, v)) {
    atomicMin(status, pack_status(row, kKindOutputOverflow, 0));
    return;
  }
  if (out_q32) out_q32[row] = v;
  if (out_f32) out_f32[row] = __ll2float_rn(v) * 2.3283064365386963e-10f;
}

// ---- the projection kernel --------------------------------------------------------------

struct GemvArgs {
  const uint8_t *pack;
  int units;        // units per row tile
  size_t n_rt;      // row tiles
  size_t n_out, n_in;
  const int8_t *codes;
  const uint8_t *exps;
  const ActDesc *desc;
  long long *out_q32;
  float *out_f32;
  unsigned long long *status;
  Acc128 *partials;     // [n_rt][ksplit][32] partial sums of a K-split row tile
  unsigned *counters;   // [n_rt] arrivals of a K-split row tile (self-resetting)
  int R, P, ksplit;     // row tiles per CTA, warps per row tile, CTAs per row tile along K
};

// Programmatic dependent launch: the next projection may start streaming its (constant)
// weights as soon as every CTA of this one is running; it waits for this grid's completion
// before it reads anything this grid or an earlier kernel writes.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Per-warp activation staging of one unit: its int8 codes (zero for a zero-scale block or
// past n_in), and per 32-lane block the exponent data and Σxq the family's fold reads.
template <uint32_t T>
struct WarpAct {
  int codes[Fam<T>::span / 4];
  int e[Fam<T>::span / 32];                     // Q8_0: absolute exponent or -1; else er
  long long xs[T == kQ6_K ? 16 : Fam<T>::span / 32];  // Σxq·2^er (per 16 lanes for Q6_K)
};

// The raw activation bytes a lane stages for unit u: 16 codes and their block's exponent,
// loaded together (one round trip) right after the dependency wait.
struct StageRegs {
  uint4 v;
  unsigned e;
};

template <uint32_t T>
__device__ __forceinline__ StageRegs stage_load(const int8_t *codes, const uint8_t *exps,
                                                size_t n_in, int u, int lane) {
  constexpr int span = Fam<T>::span;
  StageRegs s{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
  if (lane < span / 16) {
    const size_t j = (size_t)u * span + 16 * lane;
    const size_t b = j / 32;
    if (j < n_in) {
      s.e = exps[b];
      if (j + 16 <= n_in && ((reinterpret_cast<uintptr_t>(codes + j) & 15) == 0)) {
        s.v = __ldg(reinterpret_cast<const uint4 *>(codes + j));
      } else {
        unsigned t[4] = {0, 0, 0, 0};
        for (int i = 0; i < 16; i++)
          if (j + i < n_in) t[i / 4] |= ((unsigned)(uint8_t)codes[j + i]) << (8 * (i % 4));
        s.v = make_uint4(t[0], t[1], t[2], t[3]);
      }
    }
  }
  return s;
}

template <uint32_t T>
__device__ __forceinline__ void stage_store(WarpAct<T> &w, StageRegs s, int emin, int lane) {
  constexpr int span = Fam<T>::span;
  const bool zero = s.e == APX_EXP_ZERO;
  const uint4 v = zero ? make_uint4(0, 0, 0, 0) : s.v;
  const int er = zero ? 0 : (int)s.e - emin;
  const int eabs = zero ? -1 : (int)s.e;
  if (lane < span / 16) reinterpret_cast<uint4 *>(w.codes)[lane] = v;
  // Σ of this lane's 16 codes, then the 32-lane block's sum across the lane pair
  int s16 = dp4a_ss((int)v.x, 0x01010101, 0);
  s16 = dp4a_ss((int)v.y, 0x01010101, s16);
  s16 = dp4a_ss((int)v.z, 0x01010101, s16);
  s16 = dp4a_ss((int)v.w, 0x01010101, s16);
  const int s32 = s16 + __shfl_xor_sync(0xFFFFFFFFu, s16, 1);
  if (lane < span / 16) {
    if (T == kQ6_K) w.xs[lane] = (long long)s16 << er;
    if ((lane & 1) == 0) {
      w.e[lane / 2] = T == kQ8_0 ? eabs : er;
      if (T == kQ4_K) w.xs[lane / 2] = (long long)s32 << er;
    }
  }
  __syncwarp();
}

template <uint32_t T>
__device__ __forceinline__ void fold(Acc128 &acc, const UnitRegs<T> &r, const WarpAct<T> &w,
                                     int emin) {
  fold_unit(acc, r, w.codes, w.e, w.xs, emin);
}

template <uint32_t T, bool PIPE>
__global__ void __launch_bounds__(PIPE ? 256 : 512) gemv_kernel(GemvArgs g) {
  extern __shared__ __align__(16) unsigned char smem[];
  using F = Fam<T>;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ks = (int)(blockIdx.x % g.ksplit);
  const size_t rt0 = (size_t)(blockIdx.x / g.ksplit) * g.R;
  const int k0 = (int)((long long)g.units * ks / g.ksplit);
  const int k1 = (int)((long long)g.units * (ks + 1) / g.ksplit);
  const int r = warp / g.P, p = warp % g.P;
  const size_t rt = rt0 + r;
  const bool active = r < g.R && rt < g.n_rt;
  const uint8_t *base = g.pack + rt * (size_t)g.units * F::unit_bytes;

  pdl_launch_dependents();
  // weights first: they depend on nothing the previous kernel writes
  UnitRegs<T> cur;
  const bool first = active && k0 + p < k1;
  if (first) load_unit(cur, base + (size_t)(k0 + p) * F::unit_bytes, lane);
  pdl_wait();

  // the descriptor and the first unit's activation bytes in one round trip
  const ActDesc desc = *g.desc;
  StageRegs sr = first ? stage_load<T>(g.codes, g.exps, g.n_in, k0 + p, lane)
                       : StageRegs{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
  if (desc.status != APX_OK) {  // the activation itself is refused (chart/mod.rs:1904-1907)
    if (blockIdx.x == 0 && threadIdx.x == 0)
      atomicMin(g.status, pack_status(0, (unsigned)desc.status, 0));
    return;
  }
  const int es = desc.emax >= 0 ? desc.emax - desc.emin : 0;
  const bool fast = bound_ok((long long)g.n_in, F::top, desc.emax) && es <= F::es_limit &&
                    !(desc.pad[0] & 1u);  // pad[0] bit 0: a code of -128 is present
  if (!fast) {
    if (ks == 0 && p == 0 && active)
      checked_rows<T>(g.pack, g.units, rt, lane, g.n_out, g.n_in, g.codes, g.exps, g.out_q32,
                      g.out_f32, g.status);
    return;
  }

  // -- stream the units: each warp stages its unit's activation and folds its registers ---
  WarpAct<T> *wact = reinterpret_cast<WarpAct<T> *>(smem) + warp;
  Acc128 acc;
  acc_zero(acc);
  if (active) {
    for (int u = k0 + p; u < k1; u += g.P) {
      UnitRegs<T> nxt;
      const bool more = u + g.P < k1;
      if (PIPE && more) load_unit(nxt, base + (size_t)(u + g.P) * F::unit_bytes, lane);
      if (!PIPE && u != k0 + p) load_unit(cur, base + (size_t)u * F::unit_bytes, lane);
      if (u != k0 + p) {
        __syncwarp();  // the previous unit's reads of the staging are done
        sr = stage_load<T>(g.codes, g.exps, g.n_in, u, lane);
      }
      stage_store<T>(*wact, sr, desc.emin, lane);
      fold<T>(acc, cur, *wact, desc.emin);
      if (PIPE && more) cur = nxt;
    }
  }

  // -- reduce: warps of a row tile in shared memory, CTAs of a row tile through scratch ----
  __syncthreads();  // the staging region is reused for the partial sums
  Acc128 *part = reinterpret_cast<Acc128 *>(smem);  // [R*P][32]
  part[warp * 32 + lane] = acc;
  __syncthreads();
  Acc128 s;
  acc_zero(s);
  if (p == 0 && r < g.R) {
    s = part[(r * g.P) * 32 + lane];
    for (int q = 1; q < g.P; q++) acc_add(s, part[(r * g.P + q) * 32 + lane]);
  }
  bool finalize = ks == 0;
  if (g.ksplit > 1) {
    // last-arriving CTA of the row tile sums the others' partials (threadfence reduction)
    unsigned *ticket = reinterpret_cast<unsigned *>(part + g.R * g.P * 32);
    if (p == 0 && active) {
      Acc128 *slot = g.partials + (rt * g.ksplit + ks) * 32 + lane;
      slot->lo = s.lo;
      slot->hi = s.hi;
      __threadfence();
    }
    __syncthreads();
    if (threadIdx.x < (unsigned)g.R)
      ticket[threadIdx.x] = rt0 + threadIdx.x < g.n_rt
                                ? atomicAdd(g.counters + rt0 + threadIdx.x, 1u)
                                : 0u;
    __syncthreads();
    finalize = active && ticket[r] == (unsigned)(g.ksplit - 1);
    if (finalize && p == 0) {
      __threadfence();
      acc_zero(s);
      for (int q = 0; q < g.ksplit; q++) {
        const Acc128 *src = g.partials + (rt * g.ksplit + q) * 32 + lane;
        acc_add(s, __ldcg(&src->lo), __ldcg(&src->hi));
      }
      if (lane == 0) g.counters[rt] = 0u;  // ready for the next call
    }
  }
  if (finalize && p == 0 && active) {
    const size_t row = rt * 32 + lane;
    if (row < g.n_out) {
      long long v;
      if (!acc_round_to_i64(s, v)) {
        atomicMin(g.status, pack_status(row, kKindOutputOverflow, 0));
      } else {
        if (g.out_q32) g.out_q32[row] = v;
        if (g.out_f32) g.out_f32[row] = __ll2float_rn(v) * 2.3283064365386963e-10f;
      }
    }
  }
}

// ---- streaming kernel for matrices larger than one resident wave ---------------------------
//
// Persistent: V = gridDim.x × warps-per-CTA warps, warp v streams the contiguous unit chunk
// [v·C, (v+1)·C) of the (row tile, K unit) order, C = ceil(T/V), folding one unit while the
// next is in flight.  The CTA stages the whole activation once.  A row tile covered by one
// warp is finished by it; a row tile split between warps is finished by whichever of them
// arrives last (partial sums in the tensor's scratch, an arrival counter that resets itself).

struct StreamArgs {
  const uint8_t *pack;
  int units;          // U, units per row tile
  size_t n_rt, n_out, n_in;
  const int8_t *codes;
  const uint8_t *exps;
  const ActDesc *desc;
  long long *out_q32;
  float *out_f32;
  unsigned long long *status;
  Acc128 *partials;   // [n_rt][kmax][32]
  unsigned *counters; // [n_rt]
  long long chunk;    // C
  int kmax;           // most warps that can share a row tile
};

template <uint32_t T>
__device__ __forceinline__ void finish_row(const Acc128 &s, size_t row, size_t n_out,
                                           long long *out_q32, float *out_f32,
                                           unsigned long long *status) {
  if (row >= n_out) return;
  long long v;
  if (!acc_round_to_i64(s, v)) {
    atomicMin(status, pack_status(row, kKindOutputOverflow, 0));
  } else {
    if (out_q32) out_q32[row] = v;
    if (out_f32) out_f32[row] = __ll2float_rn(v) * 2.3283064365386963e-10f;
  }
}

template <uint32_t T>
__global__ void __launch_bounds__(256, 2) gemv_stream_kernel(StreamArgs g) {
  extern __shared__ __align__(16) unsigned char smem[];
  using F = Fam<T>;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const long long U = g.units, Ttot = (long long)g.n_rt * U;
  const long long v = (long long)blockIdx.x * nw + warp;
  const long long x0 = v * g.chunk, x1 = min(Ttot, x0 + g.chunk);

  pdl_launch_dependents();
  UnitRegs<T> cur;
  if (x0 < x1)
    load_unit(cur, g.pack + (size_t)x0 * F::unit_bytes, lane);
  pdl_wait();

  const ActDesc desc = *g.desc;
  if (desc.status != APX_OK) {
    if (blockIdx.x == 0 && threadIdx.x == 0)
      atomicMin(g.status, pack_status(0, (unsigned)desc.status, 0));
    return;
  }
  const int es = desc.emax >= 0 ? desc.emax - desc.emin : 0;
  const bool fast = bound_ok((long long)g.n_in, F::top, desc.emax) && es <= F::es_limit &&
                    !(desc.pad[0] & 1u);
  if (!fast) {
    // the warp holding a row tile's first unit runs that tile's checked rows
    for (long long x = x0; x < x1; x++)
      if (x % U == 0)
        checked_rows<T>(g.pack, g.units, (size_t)(x / U), lane, g.n_out, g.n_in, g.codes,
                        g.exps, g.out_q32, g.out_f32, g.status);
    return;
  }

  // -- the whole activation, staged once per CTA ---------------------------------------
  const int nel = (int)U * F::span;
  int *s_codes = reinterpret_cast<int *>(smem);
  int *s_e = s_codes + nel / 4;
  long long *s_xs = reinterpret_cast<long long *>(s_e + ((nel / 32 + 3) & ~3));
  const int n16 = nel / 16;
  for (int base = 0; base < n16; base += blockDim.x) {  // whole warps: the shuffle below
    const int j16 = base + threadIdx.x;
    const bool in = j16 < n16;
    const size_t j = 16 * (size_t)j16, b = j / 32;
    uint4 val = make_uint4(0, 0, 0, 0);
    unsigned e = APX_EXP_ZERO;
    if (in && j < g.n_in) {
      e = g.exps[b];
      if (j + 16 <= g.n_in && ((reinterpret_cast<uintptr_t>(g.codes + j) & 15) == 0)) {
        val = __ldg(reinterpret_cast<const uint4 *>(g.codes + j));
      } else {
        unsigned t[4] = {0, 0, 0, 0};
        for (int i = 0; i < 16; i++)
          if (j + i < g.n_in) t[i / 4] |= ((unsigned)(uint8_t)g.codes[j + i]) << (8 * (i % 4));
        val = make_uint4(t[0], t[1], t[2], t[3]);
      }
    }
    const bool zero = e == APX_EXP_ZERO;
    if (zero) val = make_uint4(0, 0, 0, 0);
    if (in) reinterpret_cast<uint4 *>(s_codes)[j16] = val;
    const int er = zero ? 0 : (int)e - desc.emin;
    int s16 = dp4a_ss((int)val.x, 0x01010101, 0);
    s16 = dp4a_ss((int)val.y, 0x01010101, s16);
    s16 = dp4a_ss((int)val.z, 0x01010101, s16);
    s16 = dp4a_ss((int)val.w, 0x01010101, s16);
    const int s32 = s16 + __shfl_xor_sync(0xFFFFFFFFu, s16, 1);
    if (!in) continue;
    if (T == kQ6_K) s_xs[j16] = (long long)s16 << er;
    if ((j16 & 1) == 0) {
      s_e[j16 / 2] = T == kQ8_0 ? (zero ? -1 : (int)e) : er;
      if (T == kQ4_K) s_xs[j16 / 2] = (long long)s32 << er;
    }
  }
  __syncthreads();

  // -- stream the chunk ---------------------------------------------------------------------
  Acc128 acc;
  acc_zero(acc);
  for (long long x = x0; x < x1; x++) {
    UnitRegs<T> nxt;
    const bool more = x + 1 < x1;
    if (more) load_unit(nxt, g.pack + (size_t)(x + 1) * F::unit_bytes, lane);
    const long long rt = x / U;
    const int u = (int)(x % U);
    if (T == kQ8_0)
      fold_unit(acc, cur, s_codes + u * 32, s_e + u * 4, nullptr, 0);
    else if (T == kQ4_K)
      fold_unit(acc, cur, s_codes + u * 64, s_e + u * 8, s_xs + u * 8, desc.emin);
    else
      fold_unit(acc, cur, s_codes + u * 64, s_e + u * 8, s_xs + u * 16, desc.emin);
    if (u == U - 1 || !more) {
      // flush this warp's share of row tile rt
      const long long first_v = (rt * U) / g.chunk;
      const long long last_v = (rt * U + U - 1) / g.chunk;
      const size_t row = (size_t)rt * 32 + lane;
      if (first_v == last_v) {
        finish_row<T>(acc, row, g.n_out, g.out_q32, g.out_f32, g.status);
      } else {
        const int k = (int)(v - first_v), count = (int)(last_v - first_v + 1);
        Acc128 *slot = g.partials + ((size_t)rt * g.kmax + k) * 32 + lane;
        slot->lo = acc.lo;
        slot->hi = acc.hi;
        __threadfence();
        __syncwarp();
        unsigned ticket = 0;
        if (lane == 0) ticket = atomicAdd(g.counters + rt, 1u);
        ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
        if (ticket == (unsigned)(count - 1)) {
          __threadfence();
          Acc128 s;
          acc_zero(s);
          for (int q = 0; q < count; q++) {
            const Acc128 *src = g.partials + ((size_t)rt * g.kmax + q) * 32 + lane;
            acc_add(s, __ldcg(&src->lo), __ldcg(&src->hi));
          }
          finish_row<T>(s, row, g.n_out, g.out_q32, g.out_f32, g.status);
          if (lane == 0) g.counters[rt] = 0u;
        }
      }
      acc_zero(acc);
    }
    if (more) cur = nxt;
  }
}

// ---- host-side launch planning -----------------------------------------------------------

static int unit_bytes_of(uint32_t t) {
  return t == kQ8_0 ? kUnitQ8_0 : (t == kQ4_K ? kUnitQ4_K : kUnitQ6_K);
}

int units_per_row_tile(uint32_t type, size_t n_in) {
  if (type == kQ8_0) return (int)((((n_in + 31) / 32) + 3) / 4);
  return (int)((n_in + 255) / 256);
}

size_t packed_bytes(uint32_t type, size_t n_out, size_t n_in) {
  size_t n_rt = (n_out + 31) / 32;
  return n_rt * (size_t)units_per_row_tile(type, n_in) * (size_t)unit_bytes_of(type);
}

cudaError_t launch_repack(const uint8_t *d_raw, uint8_t *d_pack, uint32_t type, size_t n_out,
                          size_t n_in, size_t row_bytes, cudaStream_t stream) {
  int units = units_per_row_tile(type, n_in);
  int nblk = type == kQ8_0 ? (int)((n_in + 31) / 32) : units;
  size_t total = packed_bytes(type, n_out, n_in);
  if (total == 0) return cudaSuccess;
  int threads = 256;
  size_t blocks = (total + threads - 1) / threads;
  if (blocks > 65535u * 16u) blocks = 65535u * 16u;
  repack_kernel<<<(unsigned)blocks, threads, 0, stream>>>(d_raw, d_pack, type, n_out, row_bytes,
                                                          units, nblk, total);
  return cudaGetLastError();
}

static size_t warp_act_bytes(uint32_t t) {
  return t == kQ8_0 ? sizeof(WarpAct<kQ8_0>)
                    : (t == kQ4_K ? sizeof(WarpAct<kQ4_K>) : sizeof(WarpAct<kQ6_K>));
}

GemvPlan plan_gemv(uint32_t type, size_t n_out, size_t n_in, int sm_count) {
  GemvPlan pl{};
  const int U = units_per_row_tile(type, n_in);  // 0 for n_in = 0: no loads, rows are 0
  const size_t n_rt = (n_out + 31) / 32;
  const size_t T = n_rt * (size_t)U;
  const size_t wave = (size_t)sm_count * 24;
  // One unit per warp while the whole matrix fits one resident wave (every load in flight at
  // once); otherwise warps stream several units, folding one while the next is in flight.
  pl.units = U;
  pl.n_rt = n_rt;
  if (T > wave) {
    // persistent streaming kernel: 2 CTAs of 8 warps per SM, one contiguous chunk per warp
    pl.pipe = true;
    const int span = type == kQ8_0 ? 128 : 256;
    const size_t nel = (size_t)U * span;
    pl.smem = nel + ((nel / 32 + 3) & ~(size_t)3) * 4 + nel / 16 * 8;
    const int per_sm = pl.smem * 2 <= 200 * 1024 ? 2 : 1;
    pl.block = 256;
    pl.grid = (unsigned)(sm_count * per_sm);
    const long long V = (long long)pl.grid * 8;
    pl.chunk = (long long)((T + V - 1) / V);
    pl.kmax = (int)((U + pl.chunk - 1) / pl.chunk) + 1;
    pl.R = pl.P = pl.ksplit = 1;
    return pl;
  }
  int upw = 1;
  pl.pipe = false;
  const int cap = pl.pipe ? 8 : 16;  // warps per CTA
  int w = std::max(1, (U + upw - 1) / upw);
  if (w <= cap) {
    pl.ksplit = 1;
    pl.P = w;
    pl.R = std::max(1, cap / pl.P);
    if (!pl.pipe)
      pl.R = std::max(1, std::min(pl.R, (int)std::max<size_t>(1, n_rt / sm_count)));
  } else {
    pl.ksplit = (w + cap - 1) / cap;
    pl.P = (w + pl.ksplit - 1) / pl.ksplit;
    pl.R = 1;
  }
  if ((size_t)pl.R > n_rt) pl.R = (int)(n_rt ? n_rt : 1);
  pl.units = U;
  pl.n_rt = n_rt;
  pl.grid = (unsigned)(((n_rt + pl.R - 1) / pl.R) * pl.ksplit);
  pl.block = 32 * pl.R * pl.P;
  size_t stage = (size_t)pl.R * pl.P * warp_act_bytes(type);
  size_t red = (size_t)pl.R * pl.P * 32 * sizeof(Acc128) + 64;
  pl.smem = std::max(stage, red);
  return pl;
}

size_t gemv_scratch_bytes(const GemvPlan &pl) {
  if (pl.pipe) return pl.n_rt * (size_t)pl.kmax * 32 * sizeof(Acc128) + pl.n_rt * sizeof(unsigned);
  if (pl.ksplit <= 1) return 0;
  return pl.n_rt * (size_t)pl.ksplit * 32 * sizeof(Acc128) + pl.n_rt * sizeof(unsigned);
}

// Programmatic dependent launch is on unless APX_PDL=0 in the environment (read once).
static bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("APX_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <uint32_t T>
static cudaError_t launch_stream(const GemvPlan &pl, const StreamArgs &a, cudaStream_t stream) {
  auto kern = gemv_stream_kernel<T>;
  if (pl.smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pl.smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(pl.block);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <uint32_t T>
static cudaError_t launch_t(const GemvPlan &pl, const GemvArgs &a, cudaStream_t stream) {
  auto kern = gemv_kernel<T, false>;
  if (pl.smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pl.smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(pl.block);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_gemv(const GemvPlan &pl, uint32_t type, const uint8_t *pack, void *scratch,
                        size_t n_out, size_t n_in, const int8_t *codes, const uint8_t *exps,
                        const void *desc, long long *out_q32, float *out_f32,
                        unsigned long long *status, cudaStream_t stream) {
  if (n_out == 0) return cudaSuccess;
  if (pl.ksplit > 1 && !scratch) return cudaErrorInvalidValue;
  if (pl.units > 0 && !pack) return cudaErrorInvalidValue;  // a plan that reads no payload
  if (pl.pipe) {
    if (!scratch) return cudaErrorInvalidValue;
    StreamArgs sa;
    sa.pack = pack;
    sa.units = pl.units;
    sa.n_rt = pl.n_rt;
    sa.n_out = n_out;
    sa.n_in = n_in;
    sa.codes = codes;
    sa.exps = exps;
    sa.desc = reinterpret_cast<const ActDesc *>(desc);
    sa.out_q32 = out_q32;
    sa.out_f32 = out_f32;
    sa.status = status;
    sa.partials = reinterpret_cast<Acc128 *>(scratch);
    sa.counters = reinterpret_cast<unsigned *>(reinterpret_cast<Acc128 *>(scratch) +
                                               pl.n_rt * (size_t)pl.kmax * 32);
    sa.chunk = pl.chunk;
    sa.kmax = pl.kmax;
    switch (type) {
      case kQ8_0: return launch_stream<kQ8_0>(pl, sa, stream);
      case kQ4_K: return launch_stream<kQ4_K>(pl, sa, stream);
      case kQ6_K: return launch_stream<kQ6_K>(pl, sa, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  GemvArgs a;
  a.pack = pack;
  a.units = pl.units;
  a.n_rt = pl.n_rt;
  a.n_out = n_out;
  a.n_in = n_in;
  a.codes = codes;
  a.exps = exps;
  a.desc = reinterpret_cast<const ActDesc *>(desc);
  a.out_q32 = out_q32;
  a.out_f32 = out_f32;
  a.status = status;
  a.partials = reinterpret_cast<Acc128 *>(scratch);
  a.counters = pl.ksplit > 1 ? reinterpret_cast<unsigned *>(
                                   reinterpret_cast<Acc128 *>(scratch) + pl.n_rt * pl.ksplit * 32)
                             : nullptr;
  a.R = pl.R;
  a.P = pl.P;
  a.ksplit = pl.ksplit;
  switch (type) {
    case kQ8_0: return launch_t<kQ8_0>(pl, a, stream);
    case kQ4_K: return launch_t<kQ4_K>(pl, a, stream);
    case kQ6_K: return launch_t<kQ6_K>(pl, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace apx
