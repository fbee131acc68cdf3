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
#include <cooperative_groups.h>

#include <algorithm>

#include "apx_common.cuh"
#include "apx_kernels.h"

namespace cg = cooperative_groups;

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
  int R, P, ksplit;  // row tiles per CTA, warps per row tile, CTAs per cluster along K
};

// Programmatic dependent launch: the next projection may start streaming its (constant)
// weights as soon as every CTA of this one is running; it waits for this grid's completion
// before it reads anything this grid or an earlier kernel writes.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <uint32_t T, bool PIPE>
__global__ void __launch_bounds__(PIPE ? 256 : 512) gemv_kernel(GemvArgs g) {
  extern __shared__ __align__(16) unsigned char smem[];
  using F = Fam<T>;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ks = g.ksplit > 1 ? (int)(blockIdx.x % g.ksplit) : 0;
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
  if (active && k0 + p < k1) load_unit(cur, base + (size_t)(k0 + p) * F::unit_bytes, lane);
  pdl_wait();

  const ActDesc desc = *g.desc;
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

  // -- activation prologue: codes, exponents and Σxq of units [k0, k1) ------------------
  const int nunits = k1 - k0;
  const int nel = nunits * F::span;  // multiple of 128
  const int nw4 = nel / 4;           // multiple of 32
  int *s_codes = reinterpret_cast<int *>(smem);
  int *s_e = s_codes + nw4;  // per 32-block: eabs (Q8_0) or er (K-quants)
  long long *s_xs = reinterpret_cast<long long *>(s_e + (((nel / 32) + 3) & ~3));
  const size_t e0 = (size_t)k0 * F::span;
  const size_t nb_act = (g.n_in + 31) / 32;
  for (int j4 = threadIdx.x; j4 < nw4; j4 += blockDim.x) {  // whole warps per iteration
    const size_t j = e0 + 4 * (size_t)j4;
    const size_t b = j / 32;
    const unsigned e = b < nb_act ? g.exps[b] : APX_EXP_ZERO;
    unsigned word = 0;
    if (e != APX_EXP_ZERO) {
      if (j + 4 <= g.n_in && ((reinterpret_cast<uintptr_t>(g.codes + j) & 3) == 0)) {
        word = *reinterpret_cast<const unsigned *>(g.codes + j);
      } else {
#pragma unroll
        for (int t = 0; t < 4; t++)
          if (j + t < g.n_in) word |= ((unsigned)(uint8_t)g.codes[j + t]) << (8 * t);
      }
    }
    s_codes[j4] = (int)word;
    if (T == kQ8_0) {
      if ((j4 & 7) == 0) s_e[j4 >> 3] = e == APX_EXP_ZERO ? -1 : (int)e;
    } else {
      const int er = e == APX_EXP_ZERO ? 0 : (int)e - desc.emin;
      int s4 = dp4a_ss((int)word, 0x01010101, 0);  // Σ of the four signed codes
      s4 += __shfl_xor_sync(0xFFFFFFFFu, s4, 1);
      s4 += __shfl_xor_sync(0xFFFFFFFFu, s4, 2);
      if (T == kQ6_K) {
        if ((j4 & 3) == 0) s_xs[j4 >> 2] = (long long)s4 << er;  // per 16 lanes
      }
      s4 += __shfl_xor_sync(0xFFFFFFFFu, s4, 4);
      if ((j4 & 7) == 0) {
        s_e[j4 >> 3] = er;
        if (T == kQ4_K) s_xs[j4 >> 3] = (long long)s4 << er;  // per 32 lanes
      }
    }
  }
  __syncthreads();

  // -- stream the units: fold the current registers while the next unit is in flight -----
  Acc128 acc;
  acc_zero(acc);
  if (active) {
    for (int u = k0 + p; u < k1; u += g.P) {
      UnitRegs<T> nxt;
      const bool more = u + g.P < k1;
      if (PIPE && more) load_unit(nxt, base + (size_t)(u + g.P) * F::unit_bytes, lane);
      if (!PIPE && u != k0 + p) load_unit(cur, base + (size_t)u * F::unit_bytes, lane);
      const int lu = u - k0;
      if (T == kQ8_0)
        fold_unit(acc, cur, s_codes + lu * 32, s_e + lu * 4, nullptr, 0);
      else if (T == kQ4_K)
        fold_unit(acc, cur, s_codes + lu * 64, s_e + lu * 8, s_xs + lu * 8, desc.emin);
      else
        fold_unit(acc, cur, s_codes + lu * 64, s_e + lu * 8, s_xs + lu * 16, desc.emin);
      if (PIPE && more) cur = nxt;
    }
  }

  // -- reduce: warps of a row tile, then CTAs of the cluster ------------------------------
  __syncthreads();  // the activation region is reused for the partial sums
  Acc128 *part = reinterpret_cast<Acc128 *>(smem);  // [R*P][32]
  if (r < g.R) part[warp * 32 + lane] = acc;
  __syncthreads();
  Acc128 *csum = part + g.R * g.P * 32;  // [R][32]: this CTA's sums, read by cluster rank 0
  if (p == 0 && r < g.R) {
    Acc128 s = part[(r * g.P) * 32 + lane];
    for (int q = 1; q < g.P; q++) acc_add(s, part[(r * g.P + q) * 32 + lane]);
    csum[r * 32 + lane] = s;
  }
  if (g.ksplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (ks == 0 && p == 0 && r < g.R) {
      Acc128 s = csum[r * 32 + lane];
      for (int q = 1; q < g.ksplit; q++) {
        const Acc128 *remote = cluster.map_shared_rank(csum, q);
        acc_add(s, remote[r * 32 + lane]);
      }
      csum[r * 32 + lane] = s;
    }
    cluster.sync();  // keep every CTA's shared memory alive until rank 0 has read it
  } else {
    __syncthreads();
  }
  if (ks == 0 && p == 0 && active) {
    const size_t row = rt * 32 + lane;
    if (row < g.n_out) {
      long long v;
      if (!acc_round_to_i64(csum[r * 32 + lane], v)) {
        atomicMin(g.status, pack_status(row, kKindOutputOverflow, 0));
      } else {
        if (g.out_q32) g.out_q32[row] = v;
        if (g.out_f32) g.out_f32[row] = __ll2float_rn(v) * 2.3283064365386963e-10f;
      }
    }
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

GemvPlan plan_gemv(uint32_t type, size_t n_out, size_t n_in, int sm_count) {
  GemvPlan pl{};
  const int U = units_per_row_tile(type, n_in);
  const size_t n_rt = (n_out + 31) / 32;
  const size_t T = n_rt * (size_t)U;
  const size_t wave = (size_t)sm_count * 24;
  if (T <= wave) {
    // The whole matrix fits one resident wave: one unit per warp, every load in flight at
    // once; CTAs of one row tile along K form a cluster when a row has more than 16 units.
    pl.pipe = false;
    int w = U < 1 ? 1 : U;
    if (w <= 16) {
      pl.ksplit = 1;
      pl.P = w;
      pl.R = std::max(1, std::min(16 / pl.P, (int)std::max<size_t>(1, n_rt / sm_count)));
    } else {
      pl.ksplit = std::min(8, (w + 15) / 16);
      pl.P = std::min(16, (w + pl.ksplit - 1) / pl.ksplit);
      pl.R = 1;
    }
  } else {
    // Streaming: each warp folds one unit while its next unit is in flight.
    pl.pipe = true;
    int w = std::max(1, (U + 1) / 2);
    if (w <= 8) {
      pl.ksplit = 1;
      pl.P = w;
      pl.R = std::max(1, 8 / pl.P);
    } else {
      pl.ksplit = std::min(8, (w + 7) / 8);
      pl.P = std::min(8, (w + pl.ksplit - 1) / pl.ksplit);
      pl.R = 1;
    }
  }
  if ((size_t)pl.R > n_rt) pl.R = (int)(n_rt ? n_rt : 1);
  pl.units = U;
  pl.n_rt = n_rt;
  pl.grid = (unsigned)(((n_rt + pl.R - 1) / pl.R) * pl.ksplit);
  pl.block = 32 * pl.R * pl.P;
  const int span = type == kQ8_0 ? 128 : 256;
  int kmax = (U + pl.ksplit - 1) / pl.ksplit;  // widest K-range of one CTA
  int nel = kmax * span, nblk32 = nel / 32;
  size_t act = (size_t)nel + (size_t)((nblk32 + 3) & ~3) * 4 + (size_t)nblk32 * 2 * 8;
  size_t red = (size_t)(pl.R * pl.P + pl.R) * 32 * sizeof(Acc128);
  pl.smem = act > red ? act : red;
  return pl;
}

template <uint32_t T>
static cudaError_t launch_t(const GemvPlan &pl, const GemvArgs &a, cudaStream_t stream) {
  auto kern = pl.pipe ? gemv_kernel<T, true> : gemv_kernel<T, false>;
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
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  na++;
  if (pl.ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = pl.ksplit;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_gemv(const GemvPlan &pl, uint32_t type, const uint8_t *pack, size_t n_out,
                        size_t n_in, const int8_t *codes, const uint8_t *exps,
                        const void *desc, long long *out_q32, float *out_f32,
                        unsigned long long *status, cudaStream_t stream) {
  if (n_out == 0) return cudaSuccess;
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
