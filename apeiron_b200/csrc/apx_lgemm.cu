// apx_lgemm.cu — exact k-column projection (the prefill contract) of Q8_0 / Q4_K / Q6_K tensors
// with every weight scale and activation shift inside the tensor-core operands.
//
// Contract (src/engine/kern/matmat.rs:92-134; the exact GEMMs of src/engine/kern/gemm.rs:438-580
// and src/engine/chart/kcols.rs:1406-1518): column c of the k-column projection equals
// matvec_q8act(W, qs[c]) bit for bit.  With every f16 scale split as m·2^k
// (src/engine/kern/pow2.rs:52-64), the row's smallest exponent kmin_r over its non-zero scales,
// and the token's activation scales 2^e relative to its smallest exponent emin_c (s = e − emin),
// the pre-rounding sum of every family is an integer dot product over the elements:
//     acc[r,c] = 2^(kmin_r + emin_c) · T[r,c],   T[r,c] = Σ_i W'[r,i] · X'[c,i],
//     Q8_0  W'[r,i] = m_b · q_i · 2^(k_b − kmin_r)                              (chart/mod.rs:554-628)
//     Q4_K  W'[r,i] = (m_d·sc_g) · q_i · 2^(k_d − kmin_r) − (m_m·mn_g) · 2^(k_m − kmin_r)
//                                                                            (chart/mod.rs:719-838)
//     Q6_K  W'[r,i] = (m_d·sc_g16) · q_i · 2^(k_d − kmin_r)                    (chart/mod.rs:845-938)
//     X'[c,i] = x_i · 2^(e_b − emin_c),
// and y[r,c] = round_shift_32(acc) with the i64 range check (chart/mod.rs:1746-1753).
//
// Digit planes.  W' is written once per tensor as D = 3 or 4 balanced base-256 digits (each in
// [−128, 127], W' = Σ_j 256^j·w_j; three when every weight of the tensor fits, as the benchmark's
// Q8_0 weights do) and X' per call as two (|X'| <= 128·2^7 = 2^14).  Every digit pair is one
// ordinary int8 GEMM over the whole K on the tensor cores (tcgen05.mma kind::i8, s32 accumulators
// in TMEM); pairs of equal weight 256^(j+l) share an accumulator, so D + 1 accumulators
// p = 0..D hold A_p = Σ_{j+l=p} Σ_i w_j[i]·x_l[i], and the exact combine T = Σ_p 256^p·A_p runs
// once per output instead of once per block.  Bounds:
//   |w_j·x_l| <= 128·128 (l = 0) and 128·64 (l = 1), two pairs per accumulator: |A_p| <=
//   24576·K < 2^31 for K <= 65536;
//   |W'| < 2^31 and |X'| <= 2^14, so |T| < K·2^45 < 2^62 for K <= 65536 (the finish's bound);
//   W' outside four digits (a weight exponent spread beyond about 12, 9 or 7 bits for Q8_0,
//   Q4_K or Q6_K) leaves the tensor without digit planes; a column whose activation spread
//   exceeds 7 or whose scales fail the reference's call bound (chart/mod.rs:362-383) takes the
//   checked rows (matvec_fixed), as the bound-failing columns of the reference do.
//
// Layout in HBM: the weight digits as [D][m_pad][kp] int8 (rows padded to 128, K to 64), kmin
// per row; per call the activation digits [2][n_pad][kp], emin and a route per token.
//
// Kernel: one CTA per SM; a tile is 128 rows × N tokens (N = 128 with three weight digits: four
// accumulators fill TMEM's 512 columns; 96 with four: five accumulators).  Whole tiles go in
// data-parallel waves (the CTAs of a wave share each weight row tile through L2); the tiles left
// over are split evenly in K-contiguous runs (stream-K), a split tile meeting its partial sums in
// global memory where the last CTA to arrive finishes it — no waiting.  Warp 0 issues TMA (3D
// boxes, 64-byte swizzle, no multicast) of a stage's D weight digit tiles and 2 activation digit
// tiles into a 5-stage ring; warp 1 owns TMEM and issues 2·D MMAs per 32-lane block; warps 2..17
// drain the accumulators into i64 sums (T = 256·T + A_p), release TMEM to the next tile's MMAs,
// and finish and store from registers; at the end the same CTAs take the checked columns' rows.
// Every wait is bounded; a wait that gives up reports APX_ERR_DEVICE_TIMEOUT for the call's
// columns, drains what is in flight and frees TMEM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"
#include "apx_quant.cuh"
#include "apx_tc.cuh"
#include "apx_unit.cuh"

namespace apx {

namespace {

constexpr int kLM = 128;        // weight rows per tile (MMA M)
constexpr int kLK = 64;         // K bytes per stage: two 32-lane blocks, one 64-byte swizzle row
constexpr int kLStages = 5;
constexpr int kXDig = 2;        // activation digits per pass over K
constexpr int kXPlanes = 3;     // activation digit planes written (the third for a second pass)
constexpr int kLEpiWarps = 16;  // 4 per TMEM lane quarter: 32 rows × N/4 tokens each
constexpr int kLThreads = 32 * (2 + kLEpiWarps);
constexpr int kLMaxShift = 7;   // X' = x·2^s with |x| <= 128 stays within two digits
constexpr int kLMaxShift3 = 15; // ... and within three
constexpr size_t kLMaxK = 65536;
constexpr int kLTileW = kLM * kLK;  // 8 KB: one weight digit tile
constexpr int kLNMin = 64, kLNMax = 128;  // token tile widths (workspace bounds)
constexpr int kLMinIters = 4;       // stages per stream-K CTA at least
// A column's route: refused, the GEMM with two activation digits, the checked rows, the GEMM
// with three (a tile holding such a column runs a second pass over K for the third digit), or
// the wide fold (a spread past three digits under the call bound: limb_wide_kernel).
constexpr unsigned kRouteNone = 0, kRouteGemm = 1, kRouteChecked = 2, kRouteGemm3 = 3;
constexpr unsigned kRouteWide = 4;
constexpr long long kPartSlot = (long long)kLM * kLNMax;  // i64 per partial tile

// The kernel's shape for D weight digits and N-token tiles.
template <int D, int N>
struct LShape {
  static constexpr int kAcc = D + kXDig - 1;        // accumulators (TMEM: kAcc·N columns)
  static constexpr int kTileX = N * kLK;            // one activation digit tile
  static constexpr int kStage = D * kLTileW + kXDig * kTileX;
  static constexpr int kEpt = N / 4;                // tokens per epilogue warp
  // Instruction descriptor of kind::i8: D s32 (2) at bits 4-5, A and B signed 8-bit (1) at
  // bits 7-9 and 10-12, both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
  static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) |
                                     ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kLM >> 4) << 24);
  static_assert(kAcc * N <= 512, "the accumulators fit in TMEM");
  static_assert(kStage % 1024 == 0 && kTileX % 1024 == 0, "stages keep the swizzle alignment");
  static_assert(kLStages * kStage + 4096 <= 227 * 1024, "the ring fits in shared memory");
  static_assert(kEpt % 8 == 0 && N % 16 == 0 && N <= kLNMax && N >= kLNMin, "tile shape");
};

// Shared-memory matrix descriptor of a K-major operand in the 64-byte-swizzled layout TMA writes:
// start address >> 4 in bits 0-13, leading byte offset 16 (>> 4, unused for swizzled K-major)
// in bits 16-29, 8-row groups 512 bytes apart (stride byte offset >> 4) in bits 32-45, version
// 1 in bits 46-47, layout type 4 (SWIZZLE_64B) in bits 61-63.  Only the start address varies:
// the second 32-lane block of a stage starts 32 bytes further.
constexpr uint64_t kLDescHi = ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
                              ((uint64_t)1 << 46) | ((uint64_t)4 << 61);

// bar.red.or over the epilogue warps (named barrier 1): every warp learns whether any of them
// saw `v`, so all take the same branch.
__device__ __forceinline__ bool epi_any(bool v) {
  unsigned r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((unsigned)v), "r"(kLEpiWarps * 32)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(kLEpiWarps * 32) : "memory");
}

// Balanced base-256 digits of w: w = d0 + 256·d1 + 256²·d2 + 256³·d3, each in [−128, 127];
// false when w needs more than four.
__device__ __forceinline__ bool digits4(long long w, uint32_t &d) {
  const long long d0 = (signed char)(w & 0xFF);
  w = (w - d0) >> 8;
  const long long d1 = (signed char)(w & 0xFF);
  w = (w - d1) >> 8;
  const long long d2 = (signed char)(w & 0xFF);
  w = (w - d2) >> 8;
  d = (uint32_t)(d0 & 0xFF) | ((uint32_t)(d1 & 0xFF) << 8) | ((uint32_t)(d2 & 0xFF) << 16) |
      ((uint32_t)(w & 0xFF) << 24);
  return w >= -128 && w <= 127;
}

// ---- the weight digit planes, built once per tensor from the repacked units ---------------------

// Per row: kmin = the smallest exponent k over its non-zero (finite) f16 scales (d, and dmin for
// Q4_K), 0 for a row without any.
template <uint32_t T>
__global__ void limb_row_kmin(PackGeo geo, size_t n_out, size_t n_in, int32_t *kmin) {
  const size_t row = blockIdx.x * (size_t)(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= n_out) return;
  int lo = 1 << 30;
  auto take = [&](unsigned h) {
    int m;
    unsigned k;
    f16_split(h, m, k);
    if (m != 0) lo = min(lo, (int)k);
  };
  if (T == kQ8_0) {
    const int nb = (int)((n_in + 31) / 32);
    for (int b = lane; b < nb; b += 32) {
      int l;
      const uint8_t *ub = slot_unit(geo, T, row, (size_t)b / 4, l);
      const int bi = b % 4;
      take(ub[4096 + l * 8 + 2 * bi] | (ub[4096 + l * 8 + 2 * bi + 1] << 8));
    }
  } else {
    const int ns = (int)((n_in + 255) / 256);
    for (int sb = lane; sb < ns; sb += 32) {
      int l;
      const uint8_t *ub = slot_unit(geo, T, row, (size_t)sb, l);
      if (T == kQ4_K) {
        const uint8_t *hd = ub + 4096 + l * 16;
        take(hd[0] | (hd[1] << 8));
        take(hd[2] | (hd[3] << 8));
      } else {
        take(ub[6656 + l * 2] | (ub[6656 + l * 2 + 1] << 8));
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) lo = min(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
  if (lane == 0) kmin[row] = lo == (1 << 30) ? 0 : lo;
}

// W'[row, 32g .. 32g+31] (zero past n_in and n_out) as four digit planes; bit 0 of flags[0] where
// a value needs more than four digits, bit 1 where one needs the fourth; flags[1] the largest bit
// length of |W'|.  One thread per (row, 32-lane group).
template <uint32_t T>
__global__ void limb_build_planes(PackGeo geo, size_t n_out, size_t n_in, size_t m_pad, size_t kp,
                                  const int32_t *kmin, int8_t *planes, int *flags) {
  const size_t groups = kp / 32;
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= m_pad * groups) return;
  const size_t row = idx / groups, g = idx % groups;
  uint32_t pl[4][8];  // plane j, values 4q..4q+3 in word q
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int q = 0; q < 8; q++) pl[j][q] = 0;
  bool ok = true, need4 = false;
  int wb = 0;  // bit length of the largest |W'|
  if (row < n_out && g * 32 < n_in) {
    const int km = kmin[row];
    long long w[32];
    if (T == kQ8_0) {
      int l;
      const uint8_t *ub = slot_unit(geo, T, row, g / 4, l);
      const int bi = (int)(g % 4);
      int m;
      unsigned k;
      f16_split(ub[4096 + l * 8 + 2 * bi] | (ub[4096 + l * 8 + 2 * bi + 1] << 8), m, k);
      const signed char *c0 = reinterpret_cast<const signed char *>(ub + ((2 * bi) * 32 + l) * 16);
      const signed char *c1 =
          reinterpret_cast<const signed char *>(ub + ((2 * bi + 1) * 32 + l) * 16);
      const unsigned sh = m ? k - (unsigned)km : 0u;
#pragma unroll
      for (int t = 0; t < 32; t++)
        w[t] = (long long)m * (t < 16 ? c0[t] : c1[t - 16]) * (1ll << sh);
    } else if (T == kQ4_K) {
      int l;
      const uint8_t *ub = slot_unit(geo, T, row, g / 8, l);
      const int j = (int)(g % 8);
      const uint8_t *hd = ub + 4096 + l * 16;
      int sc, mn;
      if (j < 4) {
        sc = hd[4 + j] & 63;
        mn = hd[4 + j + 4] & 63;
      } else {
        sc = (hd[4 + j + 4] & 0xF) | ((hd[4 + j - 4] >> 6) << 4);
        mn = (hd[4 + j + 4] >> 4) | ((hd[4 + j] >> 6) << 4);
      }
      int md, mm;
      unsigned kd, kmm;
      f16_split(hd[0] | (hd[1] << 8), md, kd);
      f16_split(hd[2] | (hd[3] << 8), mm, kmm);
      const unsigned shd = md ? kd - (unsigned)km : 0u, shm = mm ? kmm - (unsigned)km : 0u;
      const long long a = (long long)md * sc, b = (long long)mm * mn * (1ll << shm);
      // the group's 32 nibbles: byte 32·(j/2) + t of qs, low nibble for even j, high for odd
#pragma unroll
      for (int t = 0; t < 32; t++) {
        const int wb = 32 * (j / 2) + t;
        const unsigned byte = ub[((wb / 16) * 32 + l) * 16 + wb % 16];
        const unsigned code = (j & 1) ? (byte >> 4) : (byte & 0xF);
        w[t] = a * (long long)code * (1ll << shd) - b;
      }
    } else {
      int l;
      const uint8_t *ub = slot_unit(geo, T, row, g / 8, l);
      int md;
      unsigned kd;
      f16_split(ub[6656 + l * 2] | (ub[6656 + l * 2 + 1] << 8), md, kd);
      const unsigned shd = md ? kd - (unsigned)km : 0u;
#pragma unroll
      for (int t = 0; t < 32; t++) {
        const int p = 32 * (int)(g % 8) + t;
        const int n = p / 128, r = p % 128, quarter = r / 32, ll = r % 32;
        const int qlb = 64 * n + ll + ((quarter & 1) ? 32 : 0);
        const int qhb = 128 + 32 * n + ll;
        const unsigned qlv = ub[((qlb / 16) * 32 + l) * 16 + qlb % 16];
        const unsigned qhv = ub[((qhb / 16) * 32 + l) * 16 + qhb % 16];
        const unsigned lo = quarter < 2 ? (qlv & 0xF) : (qlv >> 4);
        const int code = (int)(lo | (((qhv >> (2 * quarter)) & 3) << 4)) - 32;
        const int sc = (int)(signed char)ub[6144 + l * 16 + p / 16];
        w[t] = (long long)md * sc * code * (1ll << shd);
      }
    }
#pragma unroll
    for (int t = 0; t < 32; t++) {
      uint32_t d;
      if (g * 32 + t >= n_in) w[t] = 0;
      ok = digits4(w[t], d) && ok;
      need4 = need4 || (d >> 24) != 0;
      const unsigned long long mag = w[t] < 0 ? 0ull - (unsigned long long)w[t] : (unsigned long long)w[t];
      wb = max(wb, mag ? 64 - __clzll((long long)mag) : 0);
#pragma unroll
      for (int j = 0; j < 4; j++) pl[j][t / 4] |= ((d >> (8 * j)) & 0xFFu) << (8 * (t % 4));
    }
  }
  const int f = (ok ? 0 : 1) | (need4 ? 2 : 0);
  if (f) atomicOr(flags, f);
  if (wb) atomicMax(flags + 1, wb);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint4 *dst = reinterpret_cast<uint4 *>(planes + ((size_t)j * m_pad + row) * kp + g * 32);
    dst[0] = make_uint4(pl[j][0], pl[j][1], pl[j][2], pl[j][3]);
    dst[1] = make_uint4(pl[j][4], pl[j][5], pl[j][6], pl[j][7]);
  }
}

// ---- per-call workspace --------------------------------------------------------------------------

// Nothing in it outlives a call: the prep kernel zeroes the tile counters and writes every
// column's route, emin and digits before the GEMM reads them.  Regions are sized for the
// narrowest token tile (most tiles) and the most padding columns any tile width gives.
struct LWork {
  int *cnt;          // [tiles] arrivals of the tiles split between CTAs (zeroed by the prep)
  long long *part;   // [2·sm_count][kPartSlot] partial sums of split tiles
  uint32_t *route;   // [n_pad]: refused / GEMM / checked rows
  int32_t *emin;     // [n_pad]
  int8_t *xp;        // [3][n_pad][kp]: the activation digits (zero off the GEMM)
  int8_t *qcodes;    // f32 path: the checked columns' codes [n_pad][kp]
  uint8_t *qexps;    // and exponent bytes [n_pad][kp / 32]
};

size_t lpad_k(size_t n_in) { return (n_in + kLK - 1) / kLK * kLK; }
size_t lpad_n(size_t n, int nt) { return (n + nt - 1) / nt * nt; }
size_t ltiles(size_t n_out, size_t n_cols, int nt) {
  return ((n_out + kLM - 1) / kLM) * ((n_cols + nt - 1) / nt);
}
size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// Columns padded to the widest any token tile pads them (96 or 128 tokens).
size_t lpad_max(size_t n_cols) { return std::max(lpad_n(n_cols, 96), lpad_n(n_cols, 128)); }

size_t lwork_bytes(size_t n_cols, size_t n_in, size_t n_out, int sm_count) {
  const size_t np = lpad_max(n_cols), kp = lpad_k(n_in);
  const size_t tiles = ltiles(n_out, n_cols, kLNMin);
  return align256(tiles * 4) + align256((size_t)2 * std::max(sm_count, 1) * kPartSlot * 8) +
         align256(np * 4) * 2 + kXPlanes * np * kp + align256(np * kp) + align256(np * (kp / 32)) +
         256;
}

LWork lwork_view(void *base, size_t n_cols, size_t n_in, size_t n_out, int sm_count) {
  const size_t np = lpad_max(n_cols), kp = lpad_k(n_in);
  const size_t tiles = ltiles(n_out, n_cols, kLNMin);
  uint8_t *p = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(base) + 255) & ~(uintptr_t)255);
  LWork w;
  w.cnt = reinterpret_cast<int *>(p);
  p += align256(tiles * 4);
  w.part = reinterpret_cast<long long *>(p);
  p += align256((size_t)2 * std::max(sm_count, 1) * kPartSlot * 8);
  w.route = reinterpret_cast<uint32_t *>(p);
  p += align256(np * 4);
  w.emin = reinterpret_cast<int32_t *>(p);
  p += align256(np * 4);
  w.xp = reinterpret_cast<int8_t *>(p);
  p += kXPlanes * np * kp;
  w.qcodes = reinterpret_cast<int8_t *>(p);
  p += align256(np * kp);
  w.qexps = p;
  return w;
}

// ---- activation prep: routes and digit planes --------------------------------------------------

// 16 codes of one 32-lane block times 2^s (s <= 15: |x·2^s| <= 2^22) as three balanced base-256
// digits; the third is zero for s <= 7.
__device__ __forceinline__ void x_digits16(uint4 v, int s, uint4 &lo, uint4 &mid, uint4 &hi) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t o0[4], o1[4], o2[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t a = 0, b = 0, c = 0;
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const int x = (int)(signed char)((in[q] >> (8 * t)) & 0xFFu) * (1 << s);
      const int d0 = (signed char)(x & 0xFF);
      const int r1 = (x - d0) >> 8;
      const int d1 = (signed char)(r1 & 0xFF);
      const int d2 = (r1 - d1) >> 8;
      a |= ((uint32_t)d0 & 0xFFu) << (8 * t);
      b |= ((uint32_t)d1 & 0xFFu) << (8 * t);
      c |= ((uint32_t)d2 & 0xFFu) << (8 * t);
    }
    o0[q] = a;
    o1[q] = b;
    o2[q] = c;
  }
  lo = make_uint4(o0[0], o0[1], o0[2], o0[3]);
  mid = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  hi = make_uint4(o2[0], o2[1], o2[2], o2[3]);
}

// The three digit planes' 16 bytes of column c at element j.
__device__ __forceinline__ void store_xdigits(int8_t *xp, size_t np, size_t kp, int c, size_t j,
                                              uint4 d0, uint4 d1, uint4 d2) {
  *reinterpret_cast<uint4 *>(xp + (size_t)c * kp + j) = d0;
  *reinterpret_cast<uint4 *>(xp + (np + c) * kp + j) = d1;
  *reinterpret_cast<uint4 *>(xp + (2 * np + c) * kp + j) = d2;
}

struct LPrepArgs {
  const int8_t *codes;   // caller codes, column c at c·ld (16-byte aligned rows)
  const uint8_t *exps;   // caller exponent bytes, column c at c·ldb
  const ActDesc *descs;  // the quantizer's descriptors (a refusal there wins), or null
  const float *x;        // f32 path: column c at x + c·ldx
  size_t ld, ldb, ldx, n_in, kp;
  size_t np;  // columns padded to the GEMM's token tile: the digit planes' rows
  int nb, n_cols, tiles;
  long long top;  // the family's call-bound constant (chart/mod.rs:1697-1706)
  int smax3;      // the largest activation spread of the three-digit route on this tensor
  LWork w;
  unsigned long long *status;  // column c's refusal word at status[c·2]
  unsigned long long *status_more[3];  // a group's other members' refusal words
  int n_more;
};

// An activation refusal goes to every member of the call.
__device__ __forceinline__ void prep_refuse(const LPrepArgs &a, int c, int kind) {
  atomicMin(a.status + (size_t)c * 2, pack_status(0, (unsigned)kind, 0));
  for (int m = 0; m < a.n_more; m++)
    atomicMin(a.status_more[m] + (size_t)c * 2, pack_status(0, (unsigned)kind, 0));
}

__device__ __forceinline__ void lzero_column(const LPrepArgs &a, int c, size_t np) {
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16)
    store_xdigits(a.w.xp, np, a.kp, c, j, z, z, z);
}

__device__ __forceinline__ void lprep_common_start(const LPrepArgs &a) {
  pdl_launch_dependents();  // the GEMM may start its weight loads now
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < a.tiles; i += blockDim.x) a.w.cnt[i] = 0;
}

// Route of a described column: the GEMM when the reference's call bound holds and the activation
// spread fits two digits (three up to the tensor's smax3); otherwise the checked rows (the GEMM's
// CTAs find the column by its route).
__device__ __forceinline__ unsigned lroute(const LPrepArgs &a, int emin, int emax) {
  if (!bound_ok((long long)a.n_in, a.top, emax)) return kRouteChecked;
  if (emax < 0 || emax - emin <= kLMaxShift) return kRouteGemm;
  return emax - emin <= a.smax3 ? kRouteGemm3 : kRouteWide;
}
__device__ __forceinline__ bool on_gemm(unsigned route) {
  return route == kRouteGemm || route == kRouteGemm3;
}

// One CTA per column (padding columns of the last tile included): describe (unless the
// quantizer's descriptor came with the call), route, activation digits.
__global__ void __launch_bounds__(256) limb_prep_kernel(LPrepArgs a) {
  __shared__ int s_emin, s_emax, s_status;
  __shared__ unsigned s_route;
  const int c = blockIdx.x;
  const size_t np = a.np;
  lprep_common_start(a);
  if (c >= a.n_cols) {
    lzero_column(a, c, np);
    if (threadIdx.x == 0) {
      a.w.emin[c] = 0;
      a.w.route[c] = kRouteNone;
    }
    return;
  }
  if (threadIdx.x == 0) {
    s_emin = 1 << 30;
    s_emax = -1;
    s_status = a.descs ? a.descs[c].status : APX_OK;
    if (a.descs && s_status == APX_OK) {
      const ActDesc d = a.descs[c];
      s_emax = d.emax;
      s_emin = d.emax >= 0 ? d.emin : 1 << 30;
    }
  }
  __syncthreads();
  const int8_t *codes = a.codes + (size_t)c * a.ld;
  const uint8_t *exps = a.exps + (size_t)c * a.ldb;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  // describe (QuantAct's Q32.32 image, chart/mod.rs:124-181) as the GEMV's descriptor does
  for (int b = warp; !a.descs && b < a.nb; b += nw) {
    const unsigned e = exps[b];
    if (e == APX_EXP_ZERO) continue;
    if (e > 62) {
      if (lane == 0) atomicMax(&s_status, (int)APX_ERR_INVALID_ARGUMENT);
      continue;
    }
    const size_t j = (size_t)b * 32 + lane;
    const int code = j < a.n_in ? codes[j] : 0;
    bool bad = false;
    if (e > 56) {
      const long long lim = 1ll << (63 - e);
      bad = code < -lim || code > lim - 1;
    }
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0)
      atomicMax(&s_status, (int)APX_ERR_FIXED_OVERFLOW);
    if (lane == 0) {
      atomicMin(&s_emin, (int)e);
      atomicMax(&s_emax, (int)e);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int emin = s_emax >= 0 ? s_emin : 0;
    unsigned route = kRouteNone;
    if (s_status != APX_OK)
      prep_refuse(a, c, s_status);
    else
      route = lroute(a, emin, s_emax);
    s_emin = emin;
    s_route = route;
    a.w.emin[c] = emin;
    a.w.route[c] = route;
  }
  __syncthreads();
  const bool gemm = on_gemm(s_route);
  const int emin = s_emin;
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16) {
    uint4 lo = make_uint4(0, 0, 0, 0), mid = lo, hi = lo;
    if (gemm && j < a.n_in) {
      const unsigned e = exps[j / 32];
      if (e != APX_EXP_ZERO) {
        uint4 v;
        if (j + 16 <= a.n_in) {
          v = *reinterpret_cast<const uint4 *>(codes + j);
        } else {
          uint8_t t[16];
          for (int i = 0; i < 16; i++) t[i] = j + i < a.n_in ? (uint8_t)codes[j + i] : 0;
          memcpy(&v, t, 16);
        }
        x_digits16(v, (int)e - emin, lo, mid, hi);
      }
    }
    store_xdigits(a.w.xp, np, a.kp, c, j, lo, mid, hi);
  }
}

constexpr int kLQChunks = 4;            // 128-lane chunks in flight per warp
constexpr size_t kLQPrepMaxIn = 32768;  // the column staged in shared memory

// The f32 prefill: f32_to_fixed + quant_act of the column into shared memory (the column
// quantizer's per-block arithmetic, apx_quant.cuh), then route and digits from there; codes and
// exponent bytes reach global memory only for a column the checked rows take.
__global__ void __launch_bounds__(256) limb_quant_prep_kernel(LPrepArgs a) {
  extern __shared__ __align__(16) uint8_t lqsm[];
  int8_t *scodes = reinterpret_cast<int8_t *>(lqsm);  // kp bytes
  uint8_t *sexps = lqsm + a.kp;                        // kp / 32 bytes
  __shared__ int s_emin, s_emax, s_status;
  __shared__ unsigned s_route;
  const int c = blockIdx.x;
  const size_t np = a.np;
  lprep_common_start(a);
  if (c >= a.n_cols) {
    lzero_column(a, c, np);
    if (threadIdx.x == 0) {
      a.w.emin[c] = 0;
      a.w.route[c] = kRouteNone;
    }
    return;
  }
  if (threadIdx.x == 0) {
    s_emin = 1 << 30;
    s_emax = -1;
    s_status = APX_OK;
  }
  __syncthreads();
  const float *x = a.x + (size_t)c * a.ldx;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const size_t chunks = a.kp / 128 + (a.kp % 128 ? 1 : 0);
  int w_emin = 1 << 30, w_emax = -1, w_status = APX_OK;
  for (size_t round = 0; round * nw * kLQChunks < chunks; round++) {
    float4 f4[kLQChunks];
#pragma unroll
    for (int u = 0; u < kLQChunks; u++) {
      const size_t j = ((round * kLQChunks + u) * nw + warp) * 128 + 4 * lane;
      f4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j + 4 <= a.n_in) {
        f4[u] = __ldg(reinterpret_cast<const float4 *>(x + j));
      } else if (j < a.n_in) {
        f4[u].x = x[j];
        if (j + 1 < a.n_in) f4[u].y = x[j + 1];
        if (j + 2 < a.n_in) f4[u].z = x[j + 2];
      }
    }
#pragma unroll
    for (int u = 0; u < kLQChunks; u++) {
      const size_t cbase = ((round * kLQChunks + u) * nw + warp) * 128;
      if (cbase >= a.kp) break;  // warp-uniform
      const size_t j = cbase + 4 * lane;
      uint32_t packed;
      int e;
      bool ok;
      quant_quad(f4[u], packed, e, ok);
      if (j < a.kp) *reinterpret_cast<uint32_t *>(scodes + j) = ok ? packed : 0u;
      if ((lane & 7) == 0 && j < a.n_in) {  // the block's leader
        if (!ok) {
          w_status = max(w_status, (int)APX_ERR_QUANT_REFUSED);
        } else {
          sexps[j / 32] = e < 0 ? (uint8_t)APX_EXP_ZERO : (uint8_t)e;
          if (e >= 0) {
            w_emin = min(w_emin, e);
            w_emax = max(w_emax, e);
          }
        }
      } else if ((lane & 7) == 0 && j < a.kp) {
        sexps[j / 32] = (uint8_t)APX_EXP_ZERO;  // a block wholly past n_in
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    w_emin = min(w_emin, __shfl_xor_sync(0xFFFFFFFFu, w_emin, o));
    w_emax = max(w_emax, __shfl_xor_sync(0xFFFFFFFFu, w_emax, o));
    w_status = max(w_status, __shfl_xor_sync(0xFFFFFFFFu, w_status, o));
  }
  if (lane == 0) {
    if (w_status != APX_OK) atomicMax(&s_status, w_status);
    if (w_emax >= 0) {
      atomicMin(&s_emin, w_emin);
      atomicMax(&s_emax, w_emax);
    }
  }
  __syncthreads();
  if (s_status != APX_OK) {  // quant_act returned None for the column
    lzero_column(a, c, np);
    if (threadIdx.x == 0) {
      prep_refuse(a, c, s_status);
      a.w.emin[c] = 0;
      a.w.route[c] = kRouteNone;
    }
    return;
  }
  if (threadIdx.x == 0) {
    const int emin = s_emax >= 0 ? s_emin : 0;
    const unsigned route = lroute(a, emin, s_emax);
    s_emin = emin;
    s_route = route;
    a.w.emin[c] = emin;
    a.w.route[c] = route;
  }
  __syncthreads();
  const bool gemm = on_gemm(s_route);
  const int emin = s_emin;
  if (!gemm) {  // the checked rows read the column from global memory
    for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16)
      *reinterpret_cast<uint4 *>(a.w.qcodes + (size_t)c * a.kp + j) =
          *reinterpret_cast<const uint4 *>(scodes + j);
    for (size_t b = threadIdx.x; b < a.kp / 32; b += blockDim.x)
      a.w.qexps[(size_t)c * (a.kp / 32) + b] = sexps[b];
  }
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16) {
    uint4 lo = make_uint4(0, 0, 0, 0), mid = lo, hi = lo;
    const unsigned e = sexps[j / 32];
    if (gemm && e != APX_EXP_ZERO)
      x_digits16(*reinterpret_cast<const uint4 *>(scodes + j), (int)e - emin, lo, mid, hi);
    store_xdigits(a.w.xp, np, a.kp, c, j, lo, mid, hi);
  }
}

// ---- the GEMM ----------------------------------------------------------------------------------

struct LArgs {
  const int32_t *kmin;   // [m_pad]
  LWork w;
  long long *out_q32;    // [n_cols][n_out] or null
  float *out_f32;        // [n_cols][n_out] or null
  unsigned long long *status;  // column c at status[c·2]
  size_t n_out;
  int n_cols, kstages, n_tiles, tiles;  // tile = mt·n_tiles + nt
  // Work split over G CTAs (one per SM at most): `waves` data-parallel waves of whole tiles (in
  // wave w CTA b takes tile w·G + (b + w) mod G: the CTAs of a wave share weight row tiles, so
  // each row tile's digits stream from HBM once, and the rotation spreads the cheaper tiles of
  // the last token tile evenly over the CTAs), then the remaining tiles' (tile, stage) space, sk_iters long,
  // split evenly in K-contiguous runs over the first Gs CTAs (stream-K: CTA b < Gs takes
  // [b·sk_iters/Gs, (b+1)·sk_iters/Gs); Gs <= sk_iters, so no run is empty and every CTA between
  // a split tile's first and last owner contributes to it).
  int G, waves, Gs;
  long long sk_iters;
  // checked route (matvec_fixed per row) of the columns the prep kernel routed there
  PackGeo geo;
  const int8_t *codes;
  const uint8_t *exps;
  size_t ld, ldb, n_in;
};

__device__ __forceinline__ long long lstart(const LArgs &g, int b) {
  return b >= g.Gs ? g.sk_iters : (long long)b * g.sk_iters / g.Gs;
}
// The CTA whose stream-K run holds iteration `it` of the remaining tiles.
__device__ __forceinline__ int lowner(const LArgs &g, long long it) {
  return (int)(((it + 1) * (long long)g.Gs - 1) / g.sk_iters);
}
// CTA b's local iteration i (its waves' stages first, then its stream-K run from s0): tile, stage.
__device__ __forceinline__ void lat(const LArgs &g, int b, long long s0, int i, int &tile,
                                    int &ks) {
  const int dp = g.waves * g.kstages;
  if (i < dp) {
    const int w = i / g.kstages;
    tile = w * g.G + (b + w) % g.G;
    ks = i % g.kstages;
  } else {
    const long long it = s0 + (i - dp);
    tile = g.waves * g.G + (int)(it / g.kstages);
    ks = (int)(it % g.kstages);
  }
}

// The checked rows (matvec_fixed per row) of every column the prep kernel routed there, by the
// GEMM's CTAs once their tiles are done: they read the routes a CTA-width at a time (one load
// per thread), gather that chunk's checked columns in shared memory and split each one's rows
// between all their threads.
template <uint32_t T>
__device__ __forceinline__ void lchecked_columns(const LArgs &g) {
  __shared__ int s_cols[kLThreads];
  __shared__ int s_n;
  const size_t first = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)g.G * blockDim.x;
  for (int base = 0; base < g.n_cols; base += blockDim.x) {
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    const int c = base + (int)threadIdx.x;
    if (c < g.n_cols && __ldcg(g.w.route + c) == kRouteChecked) s_cols[atomicAdd(&s_n, 1)] = c;
    __syncthreads();
    for (int i = 0; i < s_n; i++) {
      const int cc = s_cols[i];
      for (size_t row = first; row < g.n_out; row += stride)
        checked_row<T>(g.geo, row, g.n_out, g.n_in, g.codes + (size_t)cc * g.ld,
                       g.exps + (size_t)cc * g.ldb,
                       g.out_q32 ? g.out_q32 + (size_t)cc * g.n_out : nullptr,
                       g.out_f32 ? g.out_f32 + (size_t)cc * g.n_out : nullptr,
                       g.status + (size_t)cc * 2);
    }
    __syncthreads();
  }
}

// ---- the wide route -----------------------------------------------------------------------------
// Columns whose activation spread is past the three-digit route while the call bound holds
// (typically an FFN's hidden activations, whose exp tails spread far) fold exactly on the integer
// pipes with the GEMV's wide fold (apx_unit.cuh), from the tensor's GEMV layout: a warp takes one
// row tile and up to kWideCols such columns, copies each unit into its shared memory once and
// folds it against every column's staged activation chunk.  Work items (row tile, column group)
// are ordered row tile first, so the warps in flight share a few row tiles and the weights come
// from HBM about once.  Every CTA lists the wide columns of a chunk of the call in column order
// (warp ballots), so all CTAs agree on the groups.
constexpr int kWideCols = 4;      // columns folded against one staged unit
constexpr int kWideWarps = 8;     // warps per CTA, two CTAs per SM
constexpr int kWideChunk = 2048;  // columns listed at a time

struct WideArgs {
  PackGeo geo;            // the tensor's GEMV layout
  size_t n_out, n_in;
  int n_cols, n_rt;       // n_rt: row tiles of 32 / L rows
  const int8_t *codes;    // column c at codes + c·ld (f32 path: the prep's copies)
  const uint8_t *exps;    // and exps + c·ldb
  size_t ld, ldb;
  const uint32_t *route;  // the prep's routes and emin
  const int32_t *emin;
  long long *out_q32;     // [n_cols][n_out] or null
  float *out_f32;
  unsigned long long *status;  // column c at status[c·2]
};

template <uint32_t T>
__host__ __device__ constexpr size_t wide_smem_bytes() {
  return (size_t)kWideWarps * (Fam<T>::unit_bytes + kWideCols * sizeof(WarpAct<T>)) +
         kWideChunk * 4 + 64;
}

template <uint32_t T>
__global__ void __launch_bounds__(32 * kWideWarps, 2) limb_wide_kernel(WideArgs g) {
  using F = Fam<T>;
  extern __shared__ __align__(16) uint8_t wsm[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint8_t *unit_s = wsm + (size_t)warp * F::unit_bytes;
  WarpAct<T> *wa = reinterpret_cast<WarpAct<T> *>(wsm + (size_t)kWideWarps * F::unit_bytes) +
                   (size_t)warp * kWideCols;
  int *s_cols = reinterpret_cast<int *>(wsm + (size_t)kWideWarps *
                                                  (F::unit_bytes + kWideCols * sizeof(WarpAct<T>)));
  int *s_n = s_cols + kWideChunk;  // [kWideWarps + 1]
  pdl_launch_dependents();
  pdl_wait();  // routes, codes and the GEMM's outputs of this call are final
  const int L = g.geo.L, H = 32 / L, slot = lane % L, U = g.geo.units;
  const int nch = L * F::span / 16;
  for (int base = 0; base < g.n_cols; base += kWideChunk) {
    const int span = min(kWideChunk, g.n_cols - base);
    // the chunk's wide columns in column order: each warp counts a stripe, then places it
    const int per = (span + kWideWarps - 1) / kWideWarps;
    const int c0 = base + warp * per, c1 = min(base + span, c0 + per);
    int cnt = 0;
    for (int c = c0; c < c1; c += 32) {
      const bool w = c + lane < c1 && __ldcg(g.route + c + lane) == kRouteWide;
      cnt += __popc(__ballot_sync(0xFFFFFFFFu, w));
    }
    if (lane == 0) s_n[warp] = cnt;
    __syncthreads();
    int off = 0, n_w = 0;
    for (int k = 0; k < kWideWarps; k++) {
      if (k < warp) off += s_n[k];
      n_w += s_n[k];
    }
    for (int c = c0; c < c1; c += 32) {
      const bool w = c + lane < c1 && __ldcg(g.route + c + lane) == kRouteWide;
      const unsigned m = __ballot_sync(0xFFFFFFFFu, w);
      if (w) s_cols[off + __popc(m & ((1u << lane) - 1))] = c + lane;
      off += __popc(m);
    }
    __syncthreads();
    const int n_grp = (n_w + kWideCols - 1) / kWideCols;
    const long long items = (long long)g.n_rt * n_grp;
    for (long long it = (long long)blockIdx.x * kWideWarps + warp; it < items;
         it += (long long)gridDim.x * kWideWarps) {
      const int rt = (int)(it / n_grp), grp = (int)(it % n_grp);
      const int nc = min(kWideCols, n_w - grp * kWideCols);
      int col[kWideCols], em[kWideCols];
#pragma unroll
      for (int j = 0; j < kWideCols; j++) {
        col[j] = j < nc ? s_cols[grp * kWideCols + j] : 0;
        em[j] = j < nc ? __ldcg(g.emin + col[j]) : 0;
      }
      Acc128 acc[kWideCols];
#pragma unroll
      for (int j = 0; j < kWideCols; j++) acc_zero(acc[j]);
      const uint8_t *src = g.geo.pack + (size_t)rt * U * F::unit_bytes;
      for (int u = 0; u < U; u++, src += F::unit_bytes) {
        // the unit into shared memory and every column's chunks, all loads in flight together
        __syncwarp();  // the previous unit's folds are done with unit_s and the staging
        constexpr int kV = F::unit_bytes / 16;
        for (int i = lane; i < kV; i += 32)  // 16-byte asynchronous copies, no registers held
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                           smem_addr(unit_s + (size_t)i * 16)),
                       "l"(src + (size_t)i * 16)
                       : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
        Chunk ch[kWideCols][2];
#pragma unroll
        for (int j = 0; j < kWideCols; j++) {
          ch[j][0] = ch[j][1] = Chunk{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
          if (j < nc) {
            const int8_t *cc = g.codes + (size_t)col[j] * g.ld;
            const uint8_t *ce = g.exps + (size_t)col[j] * g.ldb;
            if (lane < nch) ch[j][0] = load_chunk_cg(cc, ce, g.n_in, chunk_first<T>(u, L, lane));
            if (lane + 32 < nch)
              ch[j][1] = load_chunk_cg(cc, ce, g.n_in, chunk_first<T>(u, L, lane + 32));
          }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
#pragma unroll
        for (int j = 0; j < kWideCols; j++) {
          store_chunk<T>(wa[j], ch[j][0], lane, lane < nch, em[j], true);
          if (nch > 32) store_chunk<T>(wa[j], ch[j][1], lane + 32, lane + 32 < nch, em[j], true);
        }
        __syncwarp();
        // one copy of the (large) wide fold in the loop, not one per column: the unrolled
        // copies overflowed the instruction cache
#pragma unroll 1
        for (int j = 0; j < nc; j++) {
          Acc128 t;
          acc_zero(t);
          int emj = em[0];
#pragma unroll
          for (int k = 1; k < kWideCols; k++)
            if (k == j) emj = em[k];
          fold_unit_smem<T>(t, unit_s, lane, wa[j].codes + slot * slot_ints<T>(),
                            wa[j].e + slot * (F::span / 32), wa[j].xs + slot * F::nxs, emj, true);
#pragma unroll
          for (int k = 0; k < kWideCols; k++)
            if (k == j) acc_add(acc[k], t);
        }
      }
#pragma unroll
      for (int j = 0; j < kWideCols; j++) {
        for (int o = 1; o < L; o <<= 1) {  // the L lanes of a row combine
          const unsigned long long lo = __shfl_xor_sync(0xFFFFFFFFu, acc[j].lo, o);
          const unsigned long long hi = __shfl_xor_sync(0xFFFFFFFFu, acc[j].hi, o);
          acc_add(acc[j], lo, hi);
        }
        if (j < nc && slot == 0) {
          const size_t c = (size_t)col[j];
          finish_row(acc[j], (size_t)rt * H + lane / L, g.n_out,
                     g.out_q32 ? g.out_q32 + c * g.n_out : nullptr,
                     g.out_f32 ? g.out_f32 + c * g.n_out : nullptr, g.status + c * 2,
                     PeerRows{});
        }
      }
    }
    __syncthreads();  // s_cols and s_n are rewritten for the next chunk
  }
}

// 18 warps, one CTA per SM: the warps spread 5/5/4/4 over the SM's four 16,384-register
// sub-partitions, which caps them at 96 registers each.
template <uint32_t T, int D, int N>
__global__ void __launch_bounds__(kLThreads, 1)
    limb_gemm_kernel(const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_x, LArgs g) {
  using S = LShape<D, N>;
  constexpr int kAcc = S::kAcc, kEpt = S::kEpt, kStage = S::kStage;
  extern __shared__ uint8_t lsmem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(lsmem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kLStages * kStage);
  uint64_t *full = bars, *empty = bars + kLStages;
  uint64_t *tfull = bars + 2 * kLStages, *tempty = tfull + 1, *mdone = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
  int *timeout = reinterpret_cast<int *>(tmem_slot + 1);
  int *slast = timeout + 1;  // split tile: this CTA arrived last
  int *tok_e = slast + 3;    // [N]: the tile's token exponents emin_c, -1 off the GEMM route

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = (int)blockIdx.x;
  const long long s0 = lstart(g, b), s1 = lstart(g, b + 1);
  const int dp = g.waves * g.kstages;
  const int nit = dp + (int)(s1 - s0);

  if (threadIdx.x == 0) {
    for (int st = 0; st < kLStages; st++) {
      mbar_init(full + st, 1);
      mbar_init(empty + st, 1);  // released by the stage's MMA commit
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kLEpiWarps);
    mbar_init(mdone, 1);
    *timeout = 0;
    prefetch_map(&map_w);
    prefetch_map(&map_x);
  }
  if (warp == 1) {  // TMEM: kAcc × N columns of 32-bit accumulators (a 512-column allocation)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto stage_w = [&](int st) { return smem + st * kStage; };
  auto stage_x = [&](int st) { return smem + st * kStage + D * kLTileW; };
  // The weight digits are the tensor's, constant since the layout was built: the first stages'
  // loads of them (the first piece's first pass) go out before the wait for the prep kernel
  // (programmatic dependent launch).  Everything the prep kernel writes is read after the wait.
  int pre;
  {
    int tile0, ks00;
    lat(g, b, s0, 0, tile0, ks00);
    pre = nit > 0 ? min(min(g.kstages - ks00, nit), kLStages) : 0;
    if (threadIdx.x == 0)
      for (int i = 0; i < pre; i++) {
        mbar_expect_tx(full + i, kStage);
        tma_load_3d(stage_w(i), &map_w, (ks00 + i) * kLK, (tile0 / g.n_tiles) * kLM, 0,
                    full + i);
      }
  }
  pdl_wait();
  // Whether token tile nt holds a column of the three-digit route (a second pass over K for the
  // third activation digit), read by a whole warp: the same answer in every role.
  auto needs3 = [&](int nt) {
    bool any = false;
    for (int t = lane; t < N; t += 32) {
      const int c = nt * N + t;
      any = any || (c < g.n_cols && __ldcg(g.w.route + c) == kRouteGemm3);
    }
    return __any_sync(0xFFFFFFFFu, any);
  };

  if (warp == 0) {
    // ---- TMA producer (lane 0): per stage the D weight digit tiles and 2 activation digit tiles
    // (digits 0 and 1 on a piece's first pass; digit 2 and a zero plane on its second) ----
    int i = 0, issued = 0;
    bool stop = false;
    for (int pi = 0; !stop && pi < nit;) {
      int tile, ks0;
      lat(g, b, s0, pi, tile, ks0);
      const int nk = min(g.kstages - ks0, nit - pi);
      const int passes = needs3(tile % g.n_tiles) ? 2 : 1;
      for (int pass = 0; !stop && pass < passes; pass++) {
        for (int k = 0; k < nk; k++, i++) {
          const int st = i % kLStages, use = i / kLStages;
          int bad = 0;
          if (lane == 0) {
            if (use > 0 && !mbar_wait(empty + st, (use - 1) & 1)) {
              atomicExch(timeout, 1);
              bad = 1;
            } else {
              if (i >= pre) {
                mbar_expect_tx(full + st, kStage);
                tma_load_3d(stage_w(st), &map_w, (ks0 + k) * kLK, (tile / g.n_tiles) * kLM, 0,
                            full + st);
              }
              tma_load_3d(stage_x(st), &map_x, (ks0 + k) * kLK, (tile % g.n_tiles) * N,
                          pass == 0 ? 0 : 2, full + st);
              issued = i + 1;
            }
          }
          if (__shfl_sync(0xFFFFFFFFu, bad, 0)) {
            stop = true;
            break;
          }
        }
      }
      pi += nk;
    }
    // every copy this thread started has landed before the CTA may exit
    if (lane == 0) {
      const int last = max(issued, pre);
      for (int j = last > kLStages ? last - kLStages : 0; j < last; j++)
        mbar_wait(full + j % kLStages, (j / kLStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer (lane 0): a piece's first pass takes 2·D MMAs per 32-lane block into D + 1
    // accumulators (accumulator p the pairs (p, 0) and (p − 1, 1)); a second pass, for a tile with
    // a three-digit column, D MMAs (weight digit p against activation digit 2 into accumulator
    // p).  One commit per stage (frees it) and one per pass (its accumulators are complete). ----
    const uint64_t w0 = kLDescHi | (smem_addr(stage_w(0)) >> 4);
    const uint64_t x0 = kLDescHi | (smem_addr(stage_x(0)) >> 4);
    int ok = 1;
    int i = 0, npass = 0;
    for (int pi = 0; ok && pi < nit;) {
      int tile, ks0;
      lat(g, b, s0, pi, tile, ks0);
      const int nk = min(g.kstages - ks0, nit - pi);
      const int passes = needs3(tile % g.n_tiles) ? 2 : 1;
      // The last token tile's MMAs cover only its live tokens, rounded up to the 16 the
      // instruction takes (512 tokens in 96-token tiles: 32 of the last tile's 96).  The columns
      // past them keep whatever TMEM held; they belong to padding tokens, which are never stored.
      const int live_tok = g.n_cols - (tile % g.n_tiles) * N;
      const int neff = live_tok >= N ? N : max(16, (live_tok + 15) & ~15);
      const uint32_t idesc = (S::kIdesc & ~(0x3Fu << 17)) | ((uint32_t)(neff >> 3) << 17);
      for (int pass = 0; ok && pass < passes; pass++, npass++) {
        if (lane == 0) {
          if (npass > 0 && !mbar_wait(tempty, (npass - 1) & 1)) ok = 0;
          tc_fence_after();
          for (int k = 0; ok && k < nk; k++, i++) {
            const int st = i % kLStages;
            if (!mbar_wait(full + st, (i / kLStages) & 1)) {
              ok = 0;
              break;
            }
            tc_fence_after();
            const uint64_t wd = w0 + (uint64_t)(st * (kStage >> 4));
            const uint64_t xd = x0 + (uint64_t)(st * (kStage >> 4));
#pragma unroll
            for (int q = 0; q < kLK / 32; q++) {
              const bool first = k == 0 && q == 0;
              if (pass == 0) {
#pragma unroll
                for (int p = 0; p < kAcc; p++) {
                  const uint32_t acc = tmem + (uint32_t)(p * N);
                  if (p < D)  // (p, 0)
                    mma_i8(acc, wd + (uint64_t)(p * (kLTileW >> 4) + 2 * q),
                           xd + (uint64_t)(2 * q), idesc, first ? 0u : 1u);
                  if (p >= 1)  // (p − 1, 1)
                    mma_i8(acc, wd + (uint64_t)((p - 1) * (kLTileW >> 4) + 2 * q),
                           xd + (uint64_t)((S::kTileX >> 4) + 2 * q), idesc,
                           (first && p == D) ? 0u : 1u);
                }
              } else {
#pragma unroll
                for (int p = 0; p < D; p++)  // (p, 2): the stage's first activation tile
                  mma_i8(tmem + (uint32_t)(p * N), wd + (uint64_t)(p * (kLTileW >> 4) + 2 * q),
                         xd + (uint64_t)(2 * q), idesc, first ? 0u : 1u);
              }
            }
            mma_commit(empty + st);
          }
          if (ok) mma_commit(tfull);
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      }
      pi += nk;
    }
    if (lane == 0) {
      if (!ok) atomicExch(timeout, 1);
      mma_commit(mdone);
      if (!mbar_wait(mdone, 0)) atomicExch(timeout, 1);
    }
  } else {
    // ---- epilogue: 32 rows × kEpt tokens per warp ----
    const int ew = warp - 2;
    const int lq = warp % 4;  // the TMEM lane quarter this warp may read
    const int tq = ew / 4;    // token quarter
    const int rl = 32 * lq + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(kEpt * tq);
    constexpr int kChunk = kEpt % 16 == 0 ? 16 : 8;
    int npass = 0;
    bool failed = false;
    for (int pi = 0; !failed && pi < nit;) {
      int tile, ks0;
      lat(g, b, s0, pi, tile, ks0);
      const int nk = min(g.kstages - ks0, nit - pi);
      const int mt = tile / g.n_tiles, nt = tile % g.n_tiles;
      const bool two = needs3(nt);
      // The piece's sums T = Σ_p 256^p·A_p go to this CTA's partial slot in global memory (they
      // stay in L2) a chunk of kChunk tokens at a time, so that a warp holds no more than kChunk
      // 64-bit sums in registers (all kEpt of them spilled to local memory, and the finish then
      // waited on those loads one after another).  A split tile's slot is read by the CTA that
      // finishes the tile; a whole tile's (slot 2b + 1, which only this CTA's last stream-K
      // piece uses after it) by the same thread right after.
      const bool split = !(ks0 == 0 && nk == g.kstages);  // stream-K: other CTAs hold the rest
      const int slot = 2 * b + (split && pi == dp ? 0 : 1);
      long long *mine = g.w.part + (size_t)slot * kPartSlot + (size_t)ew * (kEpt * 32);
      for (int pass = 0; pass < (two ? 2 : 1); pass++, npass++) {
        const bool got = mbar_wait_long(tfull, npass & 1);
        // every epilogue warp is done with the previous piece (tok_e included) past this barrier
        if (epi_any(!got)) {
          if (lane == 0) atomicExch(timeout, 1);
          failed = true;
          break;
        }
        tc_fence_after();
        if (pass == 0 && ew == 0)
          for (int t = lane; t < N; t += 32) {
            const int c = nt * N + t;
            // coherent loads: the prep kernel wrote these while this grid was already resident
            // (programmatic dependent launch), so the read-only path could serve a stale line
            tok_e[t] = c < g.n_cols && on_gemm(__ldcg(g.w.route + c)) ? __ldcg(g.w.emin + c) : -1;
          }
#pragma unroll 1
        for (int c = 0; c < kEpt / kChunk; c++) {
          long long acc[kChunk];
          if (pass == 0) {
            // drain: T by Horner from the top accumulator
#pragma unroll
            for (int p = kAcc - 1; p >= 0; p--) {
              uint32_t v[kChunk];
#pragma unroll
              for (int h = 0; h < kChunk / 8; h++)
                tmem_ld8_nowait(trow + (uint32_t)(p * N + kChunk * c + 8 * h), v, h);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < kChunk; j++)
                acc[j] = p == kAcc - 1 ? (long long)(int)v[j] : acc[j] * 256 + (long long)(int)v[j];
            }
          } else {
            // the third digit's pass: T += Σ_p 2^(16 + 8p)·A_p
#pragma unroll
            for (int j = 0; j < kChunk; j++) acc[j] = mine[(kChunk * c + j) * 32 + lane];
#pragma unroll
            for (int p = 0; p < D; p++) {
              uint32_t v[kChunk];
#pragma unroll
              for (int h = 0; h < kChunk / 8; h++)
                tmem_ld8_nowait(trow + (uint32_t)(p * N + kChunk * c + 8 * h), v, h);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < kChunk; j++)
                acc[j] += (long long)(int)v[j] * (1ll << (16 + 8 * p));
            }
          }
#pragma unroll
          for (int j = 0; j < kChunk; j++) mine[(kChunk * c + j) * 32 + lane] = acc[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty);  // the next pass's MMAs may overwrite TMEM
      }
      if (failed) break;
      bool finish = !split;  // this CTA holds the whole tile
      int bf = b, bl = b;
      long long tbeg = 0;
      if (split) {
        // the partial sums are stored: arrive; the last to arrive adds the others'.  Slot 2b
        // holds CTA b's first run piece, 2b + 1 its last.
        tbeg = (long long)(tile - g.waves * g.G) * g.kstages;
        __threadfence();
        epi_sync();
        bf = lowner(g, tbeg);
        bl = lowner(g, tbeg + g.kstages - 1);
        if (ew == 0 && lane == 0) {
          const int old = atomicAdd(g.w.cnt + tile, 1);
          const int last = old == bl - bf;
          if (last) g.w.cnt[tile] = 0;  // every contributor has arrived: ready for the next call
          *slast = last;
        }
        epi_sync();
        finish = *slast != 0;
        if (finish) __threadfence();
      } else {
        epi_sync();  // tok_e is written
      }
      if (finish) {
        // y = round_shift_32(T·2^(kmin_r + emin_c)) and its f32 image, stored from registers:
        // for each token the warp's 32 lanes hold 32 consecutive rows (one coalesced segment)
        const size_t row = (size_t)mt * kLM + rl;
        const bool live = row < g.n_out;
        const unsigned kmin = live ? (unsigned)__ldg(g.kmin + row) : 0u;
#pragma unroll 1
        for (int c = 0; c < kEpt / kChunk; c++) {
          long long acc[kChunk];
#pragma unroll
          for (int j = 0; j < kChunk; j++) acc[j] = mine[(kChunk * c + j) * 32 + lane];
          for (int b2 = bf; b2 <= bl; b2++) {
            if (b2 == b) continue;
            const int slot2 = 2 * b2 + ((b2 == bf && lstart(g, b2) < tbeg) ? 1 : 0);
            const long long *other =
                g.w.part + (size_t)slot2 * kPartSlot + (size_t)ew * (kEpt * 32);
#pragma unroll
            for (int j = 0; j < kChunk; j++) acc[j] += __ldcg(other + (kChunk * c + j) * 32 + lane);
          }
          const int t0 = kEpt * tq + kChunk * c, c0 = nt * N + t0;
          float *of = g.out_f32 ? g.out_f32 + (size_t)c0 * g.n_out + row : nullptr;
          long long *oq = g.out_q32 ? g.out_q32 + (size_t)c0 * g.n_out + row : nullptr;
          // the tokens' exponents: when every live token's shift kmin + e lies in [32, 64) the
          // loop has no call in it (the general case is out of line)
          int emn = 1 << 20, emx = -1;
#pragma unroll
          for (int j = 0; j < kChunk; j++) {
            const int e = tok_e[t0 + j];
            if (e >= 0) {
              emn = min(emn, e);
              emx = max(emx, e);
            }
          }
          uint32_t bad = 0;  // bit j: token j's output leaves i64
          if (emx < 0 || ((int)kmin + emn >= 32 && (int)kmin + emx < 64)) {
            // v = T·2^t, t = kmin + e − 32 in [0, 32), its f32 image RN(T)·2^(t − 32)
#pragma unroll
            for (int j = 0; j < kChunk; j++) {
              const int e = tok_e[t0 + j];
              const unsigned t = kmin + (unsigned)e - 32u;
              const int hi = (int)(acc[j] >> 32);
              const bool fits = (hi >> (31 - (t & 31))) == (hi >> 31);
              if (e >= 0 && live) {
                if (of)
                  *of = fits ? __ll2float_rn(acc[j]) * __int_as_float((int)(t + 95) << 23)
                             : __int_as_float(0x7FC00000);
                if (oq) *oq = fits ? (long long)((unsigned long long)acc[j] << (t & 31)) : 0;
              }
              bad |= (e >= 0 && live && !fits) ? 1u << j : 0u;
              if (of) of += g.n_out;
              if (oq) oq += g.n_out;
            }
          } else {
#pragma unroll
            for (int j = 0; j < kChunk; j++) {
              const int e = tok_e[t0 + j];
              if (e < 0 || !live) continue;
              long long v;
              float f;
              const bool fits = finish_fast(acc[j], kmin + (unsigned)e, v, f);
              if (of) of[(size_t)j * g.n_out] = fits ? f : __int_as_float(0x7FC00000);
              if (oq) oq[(size_t)j * g.n_out] = fits ? v : 0;
              bad |= fits ? 0u : 1u << j;
            }
          }
          while (bad) {  // output overflow: rare, one refusal per token
            const int j = __ffs(bad) - 1;
            bad &= bad - 1;
            atomicMin(g.status + (size_t)(c0 + j) * 2, pack_status(row, kKindOutputOverflow, 0));
          }
        }
      }
      pi += nk;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*timeout)  // a bounded wait gave up: the whole call refuses
    for (int c = threadIdx.x; c < g.n_cols; c += blockDim.x)
      atomicMin(g.status + (size_t)c * 2, pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0));
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
  lchecked_columns<T>(g);  // the routes and codes are the prep kernel's (read after its wait)
}

// ---- host side ---------------------------------------------------------------------------------

// A 3D int8 map over `planes` planes of `rows` rows of `inner` bytes (rows `inner` bytes apart,
// planes rows·inner apart), boxes of 64 bytes × box_rows × box_planes, 64-byte swizzle; reads
// past an extent (a plane past the last one included) fill zeros.
bool make_plane_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                    uint32_t planes, uint32_t box_planes, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {inner, rows, planes};
  const cuuint64_t strides[2] = {inner, inner * rows};
  const cuuint32_t box[3] = {(cuuint32_t)kLK, box_rows, box_planes};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, int N>
size_t limb_smem_bytes() {
  return 1024 + (size_t)kLStages * LShape<D, N>::kStage + (2 * kLStages + 3) * 8 + 32 + N * 4;
}

long long family_top(uint32_t type) {
  return type == kQ8_0 ? Fam<kQ8_0>::top : type == kQ4_K ? Fam<kQ4_K>::top : Fam<kQ6_K>::top;
}

// The token tile of a tensor with D weight digits: four accumulators of N = 128 tokens fill
// TMEM; with five, 96 tokens.
int tile_tokens(int digits) { return digits <= 3 ? 128 : 96; }
static_assert(kLNMax == 128, "lpad_max covers every token tile width");

template <uint32_t T, int D, int N>
cudaError_t launch_main(const GemvPlan &pl, const uint8_t *pack, const LimbLayout &lay,
                        size_t n_out, size_t n_in, size_t n_cols, const int8_t *codes, size_t ld,
                        const uint8_t *exps, size_t ldb, const LWork &w, long long *out_q32,
                        float *out_f32, unsigned long long *status, int sm_count,
                        cudaStream_t stream) {
  CUtensorMap map_x;
  const size_t np = lpad_n(n_cols, N);
  if (!make_plane_map(&map_x, w.xp, lay.kp, np, kXPlanes, kXDig, N)) return cudaErrorInvalidValue;
  LArgs a;
  a.kmin = lay.kmin;
  a.w = w;
  a.out_q32 = out_q32;
  a.out_f32 = out_f32;
  a.status = status;
  a.n_out = n_out;
  a.n_cols = (int)n_cols;
  a.kstages = (int)(lay.kp / kLK);
  a.n_tiles = (int)(np / N);
  a.tiles = (int)ltiles(n_out, n_cols, N);
  const long long iters = (long long)a.tiles * a.kstages;
  a.G = (int)std::max<long long>(
      1, std::min<long long>(sm_count, (iters + kLMinIters - 1) / kLMinIters));
  // Waves keep each weight row tile's digits streaming from HBM once; digit planes that sit in
  // L2 anyway (up to 64 MB) gain nothing from them, and an even split of all the work spares
  // such a call a long tail of one extra short round.
  const bool l2_resident = (size_t)D * lay.m_pad * lay.kp <= ((size_t)64 << 20);
  a.waves = l2_resident ? 0 : a.tiles / a.G;
  a.sk_iters = (long long)(a.tiles - a.waves * a.G) * a.kstages;
  a.Gs = (int)std::min<long long>(a.G, (a.sk_iters + kLMinIters - 1) / kLMinIters);
  a.geo = PackGeo{pack, pl.units, pl.L};
  a.codes = codes;
  a.exps = exps;
  a.ld = ld;
  a.ldb = ldb;
  a.n_in = n_in;
  const size_t smem = limb_smem_bytes<D, N>();
  cudaError_t e = cudaFuncSetAttribute(limb_gemm_kernel<T, D, N>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.G);
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, limb_gemm_kernel<T, D, N>,
                            *reinterpret_cast<const CUtensorMap *>(lay.map), map_x, a);
}

template <uint32_t T>
cudaError_t launch_family(const GemvPlan &pl, const uint8_t *pack, const LimbLayout &lay,
                          size_t n_out, size_t n_in, size_t n_cols, const int8_t *codes,
                          size_t ld, const uint8_t *exps, size_t ldb, const LWork &w,
                          long long *out_q32, float *out_f32, unsigned long long *status,
                          int sm_count, cudaStream_t stream) {
  if (lay.digits == 3)
    return launch_main<T, 3, 128>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                  out_q32, out_f32, status, sm_count, stream);
  return launch_main<T, 4, 96>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                               out_q32, out_f32, status, sm_count, stream);
}

cudaError_t launch_main_any(uint32_t type, const GemvPlan &pl, const uint8_t *pack,
                            const LimbLayout &lay, size_t n_out, size_t n_in, size_t n_cols,
                            const int8_t *codes, size_t ld, const uint8_t *exps, size_t ldb,
                            const LWork &w, long long *out_q32, float *out_f32,
                            unsigned long long *status, int sm_count, cudaStream_t stream) {
  switch (type) {
    case kQ8_0:
      return launch_family<kQ8_0>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                  out_q32, out_f32, status, sm_count, stream);
    case kQ4_K:
      return launch_family<kQ4_K>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                  out_q32, out_f32, status, sm_count, stream);
    case kQ6_K:
      return launch_family<kQ6_K>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                  out_q32, out_f32, status, sm_count, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

// The wide route's launch after a GEMM of the call: a programmatic dependent of it (its CTAs
// wait for the GEMM, and through it the prep, before reading a route), two CTAs per SM.
template <uint32_t T>
cudaError_t launch_wide_t(const WideArgs &a, int sm_count, cudaStream_t stream) {
  const size_t smem = wide_smem_bytes<T>();
  cudaError_t e = cudaFuncSetAttribute(limb_wide_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * std::max(sm_count, 1)));
  cfg.blockDim = dim3(32 * kWideWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_allowed() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, limb_wide_kernel<T>, a);
}

cudaError_t launch_wide(uint32_t type, const GemvPlan &pl, const uint8_t *pack, size_t n_out,
                        size_t n_in, size_t n_cols, const int8_t *codes, size_t ld,
                        const uint8_t *exps, size_t ldb, const LWork &w, long long *out_q32,
                        float *out_f32, unsigned long long *status, int sm_count,
                        cudaStream_t stream) {
  WideArgs a;
  a.geo = PackGeo{pack, pl.units, pl.L};
  a.n_out = n_out;
  a.n_in = n_in;
  a.n_cols = (int)n_cols;
  a.n_rt = (int)((n_out + 32 / pl.L - 1) / (32 / pl.L));
  a.codes = codes;
  a.exps = exps;
  a.ld = ld;
  a.ldb = ldb;
  a.route = w.route;
  a.emin = w.emin;
  a.out_q32 = out_q32;
  a.out_f32 = out_f32;
  a.status = status;
  switch (type) {
    case kQ8_0: return launch_wide_t<kQ8_0>(a, sm_count, stream);
    case kQ4_K: return launch_wide_t<kQ4_K>(a, sm_count, stream);
    case kQ6_K: return launch_wide_t<kQ6_K>(a, sm_count, stream);
    default: return cudaErrorInvalidValue;
  }
}

// The largest activation spread s of the three-digit route on a tensor whose weights have
// wbits bits: every sum T = Σ W'·X' and each of its two passes' parts stay below 2^61 when
// kp·2^(wbits + 8 + s) <= 2^61 (|W'| < 2^wbits, |X'| <= 2^(7 + s), and the parts' digits add at
// most one more bit), so the finish's i64 bound holds; at most 15 (three digits).
int three_digit_limit(const LimbLayout &lay) {
  int lg = 0;
  while (((size_t)1 << lg) < lay.kp) lg++;
  return std::min(kLMaxShift3, 53 - lay.wbits - lg);
}

LPrepArgs prep_args(uint32_t type, const LimbLayout &lay, size_t n_out, size_t n_in,
                    size_t n_cols, const LWork &w, unsigned long long *status) {
  const int nt = tile_tokens(lay.digits);
  LPrepArgs pa{};
  pa.n_in = n_in;
  pa.kp = lay.kp;
  pa.np = lpad_n(n_cols, nt);
  pa.nb = (int)((n_in + 31) / 32);
  pa.n_cols = (int)n_cols;
  pa.tiles = (int)ltiles(n_out, n_cols, nt);
  pa.top = family_top(type);
  pa.smax3 = three_digit_limit(lay);
  pa.w = w;
  pa.status = status;
  pa.n_more = 0;
  return pa;
}

// The prep kernels run right before the GEMM on the same SMs: giving them the GEMM's carveout
// (the most shared memory) spares the SMs a reconfiguration between the two launches.
bool set_prep_carveout() {
  cudaFuncSetAttribute(limb_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  cudaFuncSetAttribute(limb_quant_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  cudaGetLastError();  // a hint: a refusal leaves the default
  return true;
}

}  // namespace

// ---- entry points (apx_kernels.h) ------------------------------------------------------------

bool limb_shape_ok(size_t n_in) { return n_in > 0 && lpad_k(n_in) <= kLMaxK; }

size_t limb_work_bytes(size_t n_cols, size_t n_in, size_t n_out, int sm_count) {
  return lwork_bytes(n_cols, n_in, n_out, sm_count);
}

cudaError_t build_limb_layout(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                              size_t n_out, size_t n_in, LimbLayout *lay, cudaStream_t stream) {
  *lay = LimbLayout{};
  if (!limb_shape_ok(n_in) || n_out == 0 || (type != kQ8_0 && type != kQ4_K && type != kQ6_K))
    return cudaErrorInvalidValue;
  const size_t kp = lpad_k(n_in), m_pad = (n_out + kLM - 1) / kLM * kLM;
  // four planes first; a tensor whose weights all fit three digits then keeps three
  const size_t plane = m_pad * kp;
  void *base = nullptr;
  cudaError_t e = cudaMalloc(&base, 4 * plane + m_pad * 4 + 16);
  if (e != cudaSuccess) return e;
  int8_t *planes = reinterpret_cast<int8_t *>(base);
  int32_t *kmin = reinterpret_cast<int32_t *>(planes + 4 * plane);
  int *flags = reinterpret_cast<int *>(kmin + m_pad);
  e = cudaMemsetAsync(kmin, 0, m_pad * 4 + 16, stream);
  const PackGeo geo{pack, pl.units, pl.L};
  const size_t items = m_pad * (kp / 32);
  const unsigned rows_grid = (unsigned)((n_out + 7) / 8);
  const unsigned items_grid = (unsigned)((items + 127) / 128);
  if (e == cudaSuccess) {
    switch (type) {
      case kQ8_0:
        limb_row_kmin<kQ8_0><<<rows_grid, 256, 0, stream>>>(geo, n_out, n_in, kmin);
        limb_build_planes<kQ8_0><<<items_grid, 128, 0, stream>>>(geo, n_out, n_in, m_pad, kp,
                                                                 kmin, planes, flags);
        break;
      case kQ4_K:
        limb_row_kmin<kQ4_K><<<rows_grid, 256, 0, stream>>>(geo, n_out, n_in, kmin);
        limb_build_planes<kQ4_K><<<items_grid, 128, 0, stream>>>(geo, n_out, n_in, m_pad, kp,
                                                                 kmin, planes, flags);
        break;
      default:
        limb_row_kmin<kQ6_K><<<rows_grid, 256, 0, stream>>>(geo, n_out, n_in, kmin);
        limb_build_planes<kQ6_K><<<items_grid, 128, 0, stream>>>(geo, n_out, n_in, m_pad, kp,
                                                                 kmin, planes, flags);
        break;
    }
    e = cudaGetLastError();
  }
  int fl[2] = {1, 0};
  if (e == cudaSuccess) e = cudaMemcpyAsync(fl, flags, 8, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  const int f = fl[0];
  if (e != cudaSuccess || (f & 1)) {  // a weight needs more than four digits: no digit planes
    cudaFree(base);
    return e;
  }
  int digits = 4;
  if (!(f & 2)) {  // every fourth digit is zero: keep planes 0..2 and kmin in a smaller buffer
    void *b3 = nullptr;
    if (cudaMalloc(&b3, 3 * plane + m_pad * 4 + 16) == cudaSuccess) {
      e = cudaMemcpyAsync(b3, planes, 3 * plane, cudaMemcpyDeviceToDevice, stream);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(static_cast<int8_t *>(b3) + 3 * plane, kmin, m_pad * 4,
                            cudaMemcpyDeviceToDevice, stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) {
        cudaFree(b3);
        cudaFree(base);
        return e;
      }
      cudaFree(base);
      base = b3;
      planes = static_cast<int8_t *>(b3);
      kmin = reinterpret_cast<int32_t *>(planes + 3 * plane);
      digits = 3;
    } else {
      cudaGetLastError();  // keep the four planes
    }
  }
  if (!make_plane_map(reinterpret_cast<CUtensorMap *>(lay->map), planes, kp, m_pad,
                      (uint32_t)digits, (uint32_t)digits, kLM)) {
    cudaFree(base);
    return cudaErrorInvalidValue;
  }
  lay->base = base;
  lay->planes = planes;
  lay->kmin = kmin;
  lay->kp = kp;
  lay->m_pad = m_pad;
  lay->digits = digits;
  lay->wbits = fl[1];
  lay->ok = true;
  return cudaSuccess;
}

void free_limb_layout(LimbLayout *lay) {
  if (lay->base) cudaFree(lay->base);
  *lay = LimbLayout{};
}

cudaError_t launch_limb_gemm(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                             const LimbLayout &lay, size_t n_out, size_t n_in, size_t n_cols,
                             const int8_t *codes, size_t ld, const uint8_t *exps, size_t ldb,
                             const void *descs, void *work, long long *out_q32, float *out_f32,
                             unsigned long long *status, int sm_count, cudaStream_t stream) {
  if (n_cols == 0 || n_out == 0) return cudaSuccess;
  if (!lay.ok || ld % 16 || (reinterpret_cast<uintptr_t>(codes) & 15)) return cudaErrorInvalidValue;
  const LWork w = lwork_view(work, n_cols, n_in, n_out, sm_count);
  LPrepArgs pa = prep_args(type, lay, n_out, n_in, n_cols, w, status);
  pa.codes = codes;
  pa.exps = exps;
  pa.descs = static_cast<const ActDesc *>(descs);
  pa.ld = ld;
  pa.ldb = ldb;
  static const bool carve = set_prep_carveout();
  (void)carve;
  limb_prep_kernel<<<(unsigned)pa.np, 256, 0, stream>>>(pa);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess)
    e = launch_main_any(type, pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                        out_q32, out_f32, status, sm_count, stream);
  if (e == cudaSuccess)
    e = launch_wide(type, pl, pack, n_out, n_in, n_cols, codes, ld, exps, ldb, w, out_q32,
                    out_f32, status, sm_count, stream);
  return e;
}

bool limb_f32_ok(size_t n_in, const float *x, size_t ldx) {
  return lpad_k(n_in) <= kLQPrepMaxIn && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
         ldx % 4 == 0;
}

cudaError_t launch_limb_gemm_f32(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                                 const LimbLayout &lay, size_t n_out, size_t n_in, size_t n_cols,
                                 const float *x, size_t ldx, void *work, long long *out_q32,
                                 float *out_f32, unsigned long long *status, int sm_count,
                                 cudaStream_t stream) {
  if (n_cols == 0 || n_out == 0) return cudaSuccess;
  if (!lay.ok || !limb_f32_ok(n_in, x, ldx)) return cudaErrorInvalidValue;
  const LWork w = lwork_view(work, n_cols, n_in, n_out, sm_count);
  LPrepArgs pa = prep_args(type, lay, n_out, n_in, n_cols, w, status);
  pa.x = x;
  pa.ldx = ldx;
  const size_t smem = lay.kp + lay.kp / 32 + 16;
  static const bool carve = set_prep_carveout();
  (void)carve;
  limb_quant_prep_kernel<<<(unsigned)pa.np, 256, smem, stream>>>(pa);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess)
    e = launch_main_any(type, pl, pack, lay, n_out, n_in, n_cols, w.qcodes, lay.kp, w.qexps,
                        lay.kp / 32, w, out_q32, out_f32, status, sm_count, stream);
  if (e == cudaSuccess)
    e = launch_wide(type, pl, pack, n_out, n_in, n_cols, w.qcodes, lay.kp, w.qexps, lay.kp / 32,
                    w, out_q32, out_f32, status, sm_count, stream);
  return e;
}

cudaError_t launch_limb_gemm_f32_group(uint32_t type, const LimbMember *m, int count,
                                       size_t n_in, size_t n_cols, const float *x, size_t ldx,
                                       void *work, int sm_count, cudaStream_t stream) {
  if (count < 1 || count > 4) return cudaErrorInvalidValue;
  if (n_cols == 0) return cudaSuccess;
  size_t n_out_max = 0;
  int smax3 = kLMaxShift3, tiles = 0;
  for (int i = 0; i < count; i++) {
    const LimbLayout &lay = *m[i].lay;
    if (!lay.ok || lay.digits != m[0].lay->digits || lay.kp != m[0].lay->kp || m[i].n_out == 0)
      return cudaErrorInvalidValue;
    n_out_max = std::max(n_out_max, m[i].n_out);
    smax3 = std::min(smax3, three_digit_limit(lay));
  }
  if (!limb_f32_ok(n_in, x, ldx)) return cudaErrorInvalidValue;
  // one view of the workspace for every member: sized for the most rows
  const LWork w = lwork_view(work, n_cols, n_in, n_out_max, sm_count);
  LPrepArgs pa = prep_args(type, *m[0].lay, n_out_max, n_in, n_cols, w, m[0].status);
  pa.smax3 = smax3;  // a column takes the three-digit route only where every member allows it
  for (int i = 0; i < count; i++)
    tiles = std::max(tiles, (int)ltiles(m[i].n_out, n_cols, tile_tokens(m[i].lay->digits)));
  pa.tiles = tiles;
  pa.n_more = count - 1;
  for (int i = 1; i < count; i++) pa.status_more[i - 1] = m[i].status;
  pa.x = x;
  pa.ldx = ldx;
  const size_t smem = m[0].lay->kp + m[0].lay->kp / 32 + 16;
  static const bool carve = set_prep_carveout();
  (void)carve;
  limb_quant_prep_kernel<<<(unsigned)pa.np, 256, smem, stream>>>(pa);
  cudaError_t e = cudaGetLastError();
  for (int i = 0; e == cudaSuccess && i < count; i++)
    e = launch_main_any(type, *m[i].pl, m[i].pack, *m[i].lay, m[i].n_out, n_in, n_cols, w.qcodes,
                        m[i].lay->kp, w.qexps, m[i].lay->kp / 32, w, m[i].out_q32,
                        m[i].out_f32, m[i].status, sm_count, stream);
  for (int i = 0; e == cudaSuccess && i < count; i++)
    e = launch_wide(type, *m[i].pl, m[i].pack, m[i].n_out, n_in, n_cols, w.qcodes,
                    m[i].lay->kp, w.qexps, m[i].lay->kp / 32, w, m[i].out_q32, m[i].out_f32,
                    m[i].status, sm_count, stream);
  return e;
}

}  // namespace apx
