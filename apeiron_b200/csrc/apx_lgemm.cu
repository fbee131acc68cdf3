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
// Digit planes.  W' is written once per tensor as four balanced base-256 digits (each in
// [−128, 127], W' = Σ_j 256^j·w_j) and X' per call as two (|X'| <= 128·2^7 = 2^14).  Every digit
// pair is one ordinary int8 GEMM over the whole K on the tensor cores (tcgen05.mma kind::i8,
// s32 accumulators in TMEM); pairs of equal weight 256^(j+l) share an accumulator, so five
// accumulators p = 0..4 hold A_p = Σ_{j+l=p} Σ_i w_j[i]·x_l[i], and the exact combine
// T = Σ_p 256^p·A_p runs once per output instead of once per block.  Bounds:
//   |w_j·x_l| <= 128·128 (l = 0) and 128·64 (l = 1), two pairs per accumulator: |A_p| <=
//   24576·K < 2^31 for K <= 65536;
//   |W'| < 2^31 and |X'| <= 2^14, so |T| < K·2^45 < 2^62 for K <= 65536 (the finish's bound);
//   W' outside four digits (a weight exponent spread beyond about 12, 9 or 7 bits for Q8_0,
//   Q4_K or Q6_K) leaves the tensor without digit planes; a column whose activation spread
//   exceeds 7 or whose scales fail the reference's call bound (chart/mod.rs:362-383) takes the
//   checked rows (matvec_fixed), as the bound-failing columns of the reference do.
//
// Layout in HBM: the weight digits as [4][m_pad][kp] int8 (rows padded to 128, K to 64), kmin
// per row; per call the activation digits [2][n_pad][kp], emin and a route per token.
//
// Kernel: one CTA per SM (stream-K: every CTA takes an equal run of the (tile, K stage) space;
// a tile of 128 rows × 64 tokens split between CTAs meets its partial sums in global memory and
// the last to arrive finishes it — no waiting).  Warp 0 issues TMA (3D boxes, 64-byte swizzle,
// no multicast) of the stage's 4 weight digit tiles and 2 activation digit tiles into a 5-stage
// ring; warp 1 owns TMEM and issues 8 MMAs per 32-lane block; warps 2..9 drain the five
// accumulators into i64 sums (T = 256·T + A_p), release TMEM to the next tile's MMAs, and finish
// and store from registers.  Every wait is bounded; a wait that gives up reports
// APX_ERR_DEVICE_TIMEOUT for the call's columns, drains what is in flight and frees TMEM.
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

namespace apx {

namespace {

constexpr int kLM = 128;        // weight rows per tile (MMA M)
constexpr int kLN = 64;         // tokens per tile (MMA N)
constexpr int kLK = 64;         // K bytes per stage: two 32-lane blocks, one 64-byte swizzle row
constexpr int kLStages = 5;
constexpr int kWDig = 4, kXDig = 2, kAccs = kWDig + kXDig - 1;
constexpr int kLEpiWarps = 8;   // 2 per TMEM lane quarter: 32 rows × 32 tokens each
constexpr int kLThreads = 32 * (2 + kLEpiWarps);
constexpr int kLMaxShift = 7;   // X' = x·2^s with |x| <= 128 stays within two digits
constexpr size_t kLMaxK = 65536;
constexpr int kLTileW = kLM * kLK;                  // 8 KB: one weight digit tile
constexpr int kLTileX = kLN * kLK;                  // 4 KB: one activation digit tile
constexpr int kLStageBytes = kWDig * kLTileW + kXDig * kLTileX;  // 40 KB
constexpr int kLFallbackCtas = 32;  // extra CTAs of each launch for the checked columns
constexpr int kLMinIters = 4;       // stages per stream-K CTA at least
constexpr unsigned kRouteNone = 0, kRouteGemm = 1, kRouteChecked = 2;
constexpr long long kPartSlot = (long long)kLEpiWarps * 32 * 32;  // i64 per partial tile

static_assert(kLStageBytes % 1024 == 0 && kLTileW % 1024 == 0 && kLTileX % 1024 == 0,
              "stages keep the alignment of the swizzled tiles");
static_assert(kAccs * kLN <= 512, "the accumulators fit in TMEM");

// Instruction descriptor of kind::i8: D s32 (2) at bits 4-5, A and B signed 8-bit (1) at bits
// 7-9 and 10-12, both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
constexpr uint32_t kLIdesc = (2u << 4) | (1u << 7) | (1u << 10) |
                             ((uint32_t)(kLN >> 3) << 17) | ((uint32_t)(kLM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major operand in the 64-byte-swizzled layout TMA writes:
// start address >> 4 in bits 0-13, leading byte offset 16 (>> 4, unused for swizzled K-major)
// in bits 16-29, 8-row groups 512 bytes apart (stride byte offset >> 4) in bits 32-45, version
// 1 in bits 46-47, layout type 4 (SWIZZLE_64B) in bits 61-63.  Only the start address varies:
// the second 32-lane block of a stage starts 32 bytes further.
constexpr uint64_t kLDescHi = ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(512 >> 4) << 32) |
                              ((uint64_t)1 << 46) | ((uint64_t)4 << 61);

// The eight digit pairs (j, l) in issue order, accumulator j + l; `init` marks the first pair
// of each accumulator (it overwrites on the first block of a tile).
struct Pair {
  int j, l, init;
};
__device__ constexpr Pair kPairs[8] = {{0, 0, 1}, {1, 0, 1}, {0, 1, 0}, {2, 0, 1},
                                       {1, 1, 0}, {3, 0, 1}, {2, 1, 0}, {3, 1, 1}};

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

// W'[row, 32g .. 32g+31] (zero past n_in and n_out) as four digit planes; *bad = 1 where a value
// needs more than four digits.  One thread per (row, 32-lane group).
template <uint32_t T>
__global__ void limb_build_planes(PackGeo geo, size_t n_out, size_t n_in, size_t m_pad, size_t kp,
                                  const int32_t *kmin, int8_t *planes, int *bad) {
  const size_t groups = kp / 32;
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= m_pad * groups) return;
  const size_t row = idx / groups, g = idx % groups;
  uint32_t pl[4][8];  // plane j, values 4q..4q+3 in word q
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int q = 0; q < 8; q++) pl[j][q] = 0;
  bool ok = true;
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
#pragma unroll
      for (int j = 0; j < 4; j++) pl[j][t / 4] |= ((d >> (8 * j)) & 0xFFu) << (8 * (t % 4));
    }
  }
  if (!ok) atomicOr(bad, 1);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    uint4 *dst = reinterpret_cast<uint4 *>(planes + ((size_t)j * m_pad + row) * kp + g * 32);
    dst[0] = make_uint4(pl[j][0], pl[j][1], pl[j][2], pl[j][3]);
    dst[1] = make_uint4(pl[j][4], pl[j][5], pl[j][6], pl[j][7]);
  }
}

// ---- per-call workspace --------------------------------------------------------------------------

// Nothing in it outlives a call: the prep kernel zeroes the tile counters and writes every
// column's route, emin and digits before the GEMM reads them.
struct LWork {
  int *cnt;          // [tiles] arrivals of the tiles split between CTAs (zeroed by the prep)
  long long *part;   // [2·sm_count][kPartSlot] partial sums of split tiles
  uint32_t *route;   // [n_pad]: refused / GEMM / checked rows
  int32_t *emin;     // [n_pad]
  int8_t *xp;        // [2][n_pad][kp]: the activation digits (zero off the GEMM)
  int8_t *qcodes;    // f32 path: the checked columns' codes [n_pad][kp]
  uint8_t *qexps;    // and exponent bytes [n_pad][kp / 32]
};

__host__ __device__ size_t lpad_cols(size_t n) { return (n + kLN - 1) / kLN * kLN; }
size_t lpad_k(size_t n_in) { return (n_in + kLK - 1) / kLK * kLK; }
size_t ltiles(size_t n_out, size_t n_cols) {
  return ((n_out + kLM - 1) / kLM) * ((n_cols + kLN - 1) / kLN);
}
size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t lwork_bytes(size_t n_cols, size_t n_in, size_t n_out, int sm_count) {
  const size_t np = lpad_cols(n_cols), kp = lpad_k(n_in), tiles = ltiles(n_out, n_cols);
  return align256(tiles * 4) + align256((size_t)2 * std::max(sm_count, 1) * kPartSlot * 8) +
         align256(np * 4) * 2 + 2 * np * kp + align256(np * kp) + align256(np * (kp / 32)) + 256;
}

LWork lwork_view(void *base, size_t n_cols, size_t n_in, size_t n_out, int sm_count) {
  const size_t np = lpad_cols(n_cols), kp = lpad_k(n_in), tiles = ltiles(n_out, n_cols);
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
  p += 2 * np * kp;
  w.qcodes = reinterpret_cast<int8_t *>(p);
  p += align256(np * kp);
  w.qexps = p;
  return w;
}

// ---- activation prep: routes and digit planes --------------------------------------------------

// 16 codes of one 32-lane block times 2^s as balanced base-256 digits (|x·2^s| <= 2^14).
__device__ __forceinline__ void x_digits16(uint4 v, int s, uint4 &lo, uint4 &hi) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t o0[4], o1[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t a = 0, b = 0;
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const int x = (int)(signed char)((in[q] >> (8 * t)) & 0xFFu) * (1 << s);
      const int d0 = (signed char)(x & 0xFF);
      const int d1 = (x - d0) >> 8;
      a |= ((uint32_t)d0 & 0xFFu) << (8 * t);
      b |= ((uint32_t)d1 & 0xFFu) << (8 * t);
    }
    o0[q] = a;
    o1[q] = b;
  }
  lo = make_uint4(o0[0], o0[1], o0[2], o0[3]);
  hi = make_uint4(o1[0], o1[1], o1[2], o1[3]);
}

struct LPrepArgs {
  const int8_t *codes;   // caller codes, column c at c·ld (16-byte aligned rows)
  const uint8_t *exps;   // caller exponent bytes, column c at c·ldb
  const ActDesc *descs;  // the quantizer's descriptors (a refusal there wins), or null
  const float *x;        // f32 path: column c at x + c·ldx
  size_t ld, ldb, ldx, n_in, kp;
  int nb, n_cols, tiles;
  long long top;  // the family's call-bound constant (chart/mod.rs:1697-1706)
  LWork w;
  unsigned long long *status;  // column c's refusal word at status[c·2]
};

__device__ __forceinline__ void lzero_column(const LPrepArgs &a, int c, size_t np) {
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16) {
    *reinterpret_cast<uint4 *>(a.w.xp + (size_t)c * a.kp + j) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4 *>(a.w.xp + (np + c) * a.kp + j) = make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void lprep_common_start(const LPrepArgs &a) {
  pdl_launch_dependents();  // the GEMM may start its weight loads now
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < a.tiles; i += blockDim.x) a.w.cnt[i] = 0;
}

// Route of a described column: GEMM when the reference's call bound holds and the activation
// spread fits two digits; otherwise the checked rows (the GEMM's extra CTAs find the column by
// its route).
__device__ __forceinline__ unsigned lroute(const LPrepArgs &a, int emin, int emax) {
  return bound_ok((long long)a.n_in, a.top, emax) && (emax < 0 || emax - emin <= kLMaxShift)
             ? kRouteGemm
             : kRouteChecked;
}

// One CTA per column (padding columns of the last tile included): describe (unless the
// quantizer's descriptor came with the call), route, activation digits.
__global__ void __launch_bounds__(256) limb_prep_kernel(LPrepArgs a) {
  __shared__ int s_emin, s_emax, s_status;
  __shared__ unsigned s_route;
  const int c = blockIdx.x;
  const size_t np = lpad_cols((size_t)a.n_cols);
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
      atomicMin(a.status + (size_t)c * 2, pack_status(0, (unsigned)s_status, 0));
    else
      route = lroute(a, emin, s_emax);
    s_emin = emin;
    s_route = route;
    a.w.emin[c] = emin;
    a.w.route[c] = route;
  }
  __syncthreads();
  const bool gemm = s_route == kRouteGemm;
  const int emin = s_emin;
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16) {
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
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
        x_digits16(v, (int)e - emin, lo, hi);
      }
    }
    *reinterpret_cast<uint4 *>(a.w.xp + (size_t)c * a.kp + j) = lo;
    *reinterpret_cast<uint4 *>(a.w.xp + (np + c) * a.kp + j) = hi;
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
  const size_t np = lpad_cols((size_t)a.n_cols);
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
      atomicMin(a.status + (size_t)c * 2, pack_status(0, (unsigned)s_status, 0));
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
  const bool gemm = s_route == kRouteGemm;
  const int emin = s_emin;
  if (!gemm) {  // the checked rows read the column from global memory
    for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16)
      *reinterpret_cast<uint4 *>(a.w.qcodes + (size_t)c * a.kp + j) =
          *reinterpret_cast<const uint4 *>(scodes + j);
    for (size_t b = threadIdx.x; b < a.kp / 32; b += blockDim.x)
      a.w.qexps[(size_t)c * (a.kp / 32) + b] = sexps[b];
  }
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16) {
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    const unsigned e = sexps[j / 32];
    if (gemm && e != APX_EXP_ZERO)
      x_digits16(*reinterpret_cast<const uint4 *>(scodes + j), (int)e - emin, lo, hi);
    *reinterpret_cast<uint4 *>(a.w.xp + (size_t)c * a.kp + j) = lo;
    *reinterpret_cast<uint4 *>(a.w.xp + (np + c) * a.kp + j) = hi;
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
  int n_cols, kstages, n_tiles, tiles;
  long long iters;  // tiles · kstages: the stream-K space, tile-major (tile = mt·n_tiles + nt)
  int G;            // stream-K CTAs; CTA b takes [b·iters/G, (b+1)·iters/G)
  // checked route (matvec_fixed per row) of the columns the prep kernel listed
  PackGeo geo;
  const int8_t *codes;
  const uint8_t *exps;
  size_t ld, ldb, n_in;
};

__device__ __forceinline__ long long lstart(const LArgs &g, int b) {
  return (long long)b * g.iters / g.G;
}
// The stream-K CTA whose run holds iteration `it`.
__device__ __forceinline__ int lowner(const LArgs &g, long long it) {
  return (int)(((it + 1) * (long long)g.G - 1) / g.iters);
}

// The checked rows (matvec_fixed per row) of every column the prep kernel routed there: the
// extra CTAs walk the columns in order and split each one's rows between their threads.
template <uint32_t T>
__device__ __forceinline__ void lchecked_columns(const LArgs &g) {
  const size_t first = (size_t)(blockIdx.x - g.G) * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)kLFallbackCtas * blockDim.x;
  for (int c = 0; c < g.n_cols; c++) {
    if (__ldg(g.w.route + c) != kRouteChecked) continue;  // uniform over the CTA
    for (size_t row = first; row < g.n_out; row += stride)
      checked_row<T>(g.geo, row, g.n_out, g.n_in, g.codes + (size_t)c * g.ld,
                     g.exps + (size_t)c * g.ldb,
                     g.out_q32 ? g.out_q32 + (size_t)c * g.n_out : nullptr,
                     g.out_f32 ? g.out_f32 + (size_t)c * g.n_out : nullptr,
                     g.status + (size_t)c * 2);
  }
}

template <uint32_t T>
__global__ void __launch_bounds__(kLThreads, 1)
    limb_gemm_kernel(const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_x, LArgs g) {
  if ((int)blockIdx.x >= g.G) {
    pdl_wait();  // the prep kernel's routes and codes
    lchecked_columns<T>(g);
    return;
  }
  extern __shared__ uint8_t lsmem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(lsmem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kLStages * kLStageBytes);
  uint64_t *full = bars, *empty = bars + kLStages;
  uint64_t *tfull = bars + 2 * kLStages, *tempty = tfull + 1, *mdone = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
  int *timeout = reinterpret_cast<int *>(tmem_slot + 1);
  int *slast = timeout + 1;  // split tile: this CTA arrived last

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = (int)blockIdx.x;
  const long long it0 = lstart(g, b), it1 = lstart(g, b + 1);
  const int nit = (int)(it1 - it0);

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
  if (warp == 1) {  // TMEM: kAccs × kLN columns of 32-bit accumulators (a 512-column allocation)
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
  auto stage_w = [&](int st) { return smem + st * kLStageBytes; };
  auto stage_x = [&](int st) { return smem + st * kLStageBytes + kWDig * kLTileW; };
  // The weight digits are the tensor's, constant since the layout was built: the first stages'
  // loads of them go out before the wait for the prep kernel (programmatic dependent launch).
  // Everything the prep kernel writes is read after the wait.
  const int pre = min(nit, kLStages);
  if (threadIdx.x == 0) {
    for (int i = 0; i < pre; i++) {
      const long long it = it0 + i;
      const int tile = (int)(it / g.kstages), ks = (int)(it % g.kstages);
      mbar_expect_tx(full + i, kLStageBytes);
      tma_load_3d(stage_w(i), &map_w, ks * kLK, (tile / g.n_tiles) * kLM, 0, full + i);
    }
  }
  pdl_wait();

  if (warp == 0) {
    // ---- TMA producer (lane 0): per stage the 4 weight digit tiles and the 2 activation ones
    int issued = 0;
    for (int i = 0; i < nit; i++) {
      const long long it = it0 + i;
      const int tile = (int)(it / g.kstages), ks = (int)(it % g.kstages);
      const int st = i % kLStages, use = i / kLStages;
      int stop = 0;
      if (lane == 0) {
        if (use > 0 && !mbar_wait(empty + st, (use - 1) & 1)) {
          atomicExch(timeout, 1);
          stop = 1;
        } else {
          if (i >= pre) {
            mbar_expect_tx(full + st, kLStageBytes);
            tma_load_3d(stage_w(st), &map_w, ks * kLK, (tile / g.n_tiles) * kLM, 0, full + st);
          }
          tma_load_3d(stage_x(st), &map_x, ks * kLK, (tile % g.n_tiles) * kLN, 0, full + st);
          issued++;
        }
      }
      if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
    }
    // every copy this thread started has landed before the CTA may exit
    if (lane == 0) {
      for (int i = max(issued, pre) > kLStages ? max(issued, pre) - kLStages : 0;
           i < max(issued, pre); i++)
        mbar_wait(full + i % kLStages, (i / kLStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer (lane 0): 8 MMAs per 32-lane block, one commit per stage (frees it) and
    // one per tile piece (its accumulators are complete) ----
    if (lane == 0) {
      const uint64_t w0 = kLDescHi | (smem_addr(stage_w(0)) >> 4);
      const uint64_t x0 = kLDescHi | (smem_addr(stage_x(0)) >> 4);
      bool ok = true;
      int i = 0, piece = 0;
      for (long long it = it0; ok && it < it1; piece++) {
        const int ks0 = (int)(it % g.kstages);
        const int nk = (int)min((long long)(g.kstages - ks0), it1 - it);
        if (piece > 0 && !mbar_wait(tempty, (piece - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int k = 0; k < nk; k++, i++) {
          const int st = i % kLStages;
          if (!mbar_wait(full + st, (i / kLStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t wd = w0 + (uint64_t)(st * (kLStageBytes >> 4));
          const uint64_t xd = x0 + (uint64_t)(st * (kLStageBytes >> 4));
#pragma unroll
          for (int q = 0; q < kLK / 32; q++) {
#pragma unroll
            for (int pp = 0; pp < 8; pp++) {
              const Pair pr = kPairs[pp];
              const uint32_t accumulate = (k == 0 && q == 0 && pr.init) ? 0u : 1u;
              mma_i8(tmem + (uint32_t)((pr.j + pr.l) * kLN),
                     wd + (uint64_t)(pr.j * (kLTileW >> 4) + 2 * q),
                     xd + (uint64_t)(pr.l * (kLTileX >> 4) + 2 * q), kLIdesc, accumulate);
            }
          }
          mma_commit(empty + st);
        }
        if (!ok) break;
        mma_commit(tfull);
        it += nk;
      }
      if (!ok) atomicExch(timeout, 1);
      mma_commit(mdone);
      if (!mbar_wait(mdone, 0)) atomicExch(timeout, 1);
    }
  } else {
    // ---- epilogue: 32 rows × 32 tokens per warp ----
    const int ew = warp - 2;
    const int lq = warp % 4;  // the TMEM lane quarter this warp may read
    const int th = ew / 4;    // token half
    const int rl = 32 * lq + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(32 * th);
    int piece = 0;
    for (long long it = it0; it < it1; piece++) {
      const int tile = (int)(it / g.kstages), ks0 = (int)(it % g.kstages);
      const int nk = (int)min((long long)(g.kstages - ks0), it1 - it);
      const int mt = tile / g.n_tiles, nt = tile % g.n_tiles;
      const bool got = mbar_wait(tfull, piece & 1);
      if (epi_any(!got)) {
        if (lane == 0) atomicExch(timeout, 1);
        break;
      }
      tc_fence_after();
      // drain: T = Σ_p 256^p·A_p by Horner from the top accumulator
      long long acc[32];
#pragma unroll
      for (int p = kAccs - 1; p >= 0; p--) {
        uint32_t v[32];
        tmem_ld32_nowait(trow + (uint32_t)(p * kLN), v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j++)
          acc[j] = p == kAccs - 1 ? (long long)(int)v[j] : acc[j] * 256 + (long long)(int)v[j];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);  // the next piece's MMAs may overwrite TMEM
      const long long tbeg = (long long)tile * g.kstages;
      bool finish = ks0 == 0 && nk == g.kstages;  // this CTA holds the whole tile
      if (!finish) {
        // split tile: store the partial sums, arrive; the last to arrive adds the others'
        const int slot = 2 * b + (it == it0 ? 0 : 1);
        long long *mine = g.w.part + (size_t)slot * kPartSlot + (size_t)ew * 1024;
#pragma unroll
        for (int j = 0; j < 32; j++) mine[j * 32 + lane] = acc[j];
        __threadfence();
        epi_sync();
        const int bf = lowner(g, tbeg), bl = lowner(g, tbeg + g.kstages - 1);
        if (ew == 0 && lane == 0) {
          const int old = atomicAdd(g.w.cnt + tile, 1);
          const int last = old == bl - bf;
          if (last) g.w.cnt[tile] = 0;  // every contributor has arrived: ready for the next call
          *slast = last;
        }
        epi_sync();
        finish = *slast != 0;
        if (finish) {
          __threadfence();
          for (int b2 = bf; b2 <= bl; b2++) {
            if (b2 == b) continue;
            const int slot2 = 2 * b2 + ((b2 == bf && lstart(g, b2) < tbeg) ? 1 : 0);
            const long long *other = g.w.part + (size_t)slot2 * kPartSlot + (size_t)ew * 1024;
#pragma unroll
            for (int j = 0; j < 32; j++) acc[j] += __ldcg(other + j * 32 + lane);
          }
        }
      }
      if (finish) {
        // y = round_shift_32(T·2^(kmin_r + emin_c)) and its f32 image, stored from registers:
        // for each token the warp's 32 lanes hold 32 consecutive rows (one coalesced segment)
        const size_t row = (size_t)mt * kLM + rl;
        const bool live = row < g.n_out;
        const unsigned kmin = live ? (unsigned)__ldg(g.kmin + row) : 0u;
        const int c0 = nt * kLN + 32 * th;
        int ev[32];
        int emn = 1 << 20, emx = -1;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int c = c0 + j;
          const bool on = c < g.n_cols && __ldg(g.w.route + c) == kRouteGemm;
          ev[j] = on ? __ldg(g.w.emin + c) : -1;
          if (ev[j] >= 0) {
            emn = min(emn, ev[j]);
            emx = max(emx, ev[j]);
          }
        }
        float *of = g.out_f32 ? g.out_f32 + (size_t)c0 * g.n_out + row : nullptr;
        long long *oq = g.out_q32 ? g.out_q32 + (size_t)c0 * g.n_out + row : nullptr;
        uint32_t bad = 0;  // bit j: token j's output leaves i64
        if (emx < 0 || ((int)kmin + emn >= 32 && (int)kmin + emx < 64)) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int e = ev[j];
            const unsigned t = kmin + (unsigned)e - 32u;  // in [0, 32) for e >= 0
            const int hi = (int)(acc[j] >> 32);
            const long long v = (long long)((unsigned long long)acc[j] << (t & 31));
            const float f = __ll2float_rn(acc[j]) * __int_as_float((int)(t + 95) << 23);
            const bool fits = (hi >> (31 - (t & 31))) == (hi >> 31);
            if (e >= 0 && live) {
              if (of) of[(size_t)j * g.n_out] = fits ? f : __int_as_float(0x7FC00000);
              if (oq) oq[(size_t)j * g.n_out] = fits ? v : 0;
            }
            bad |= (e >= 0 && live && !fits) ? 1u << j : 0u;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int e = ev[j];
            long long v;
            float f;
            const bool fits = finish_fast(acc[j], kmin + (unsigned)e, v, f);
            if (e >= 0 && live) {
              if (of) of[(size_t)j * g.n_out] = fits ? f : __int_as_float(0x7FC00000);
              if (oq) oq[(size_t)j * g.n_out] = fits ? v : 0;
            }
            bad |= (e >= 0 && live && !fits) ? 1u << j : 0u;
          }
        }
        while (bad) {  // output overflow: rare, one refusal per token
          const int j = __ffs(bad) - 1;
          bad &= bad - 1;
          atomicMin(g.status + (size_t)(c0 + j) * 2, pack_status(row, kKindOutputOverflow, 0));
        }
      }
      it += nk;
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
}

// ---- host side ---------------------------------------------------------------------------------

// A 3D int8 map over `planes` planes of `rows` rows of `inner` bytes (rows `inner` bytes apart,
// planes rows·inner apart), boxes of 64 bytes × box_rows × planes, 64-byte swizzle; reads past
// an extent fill zeros.
bool make_plane_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                    uint32_t planes, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {inner, rows, planes};
  const cuuint64_t strides[2] = {inner, inner * rows};
  const cuuint32_t box[3] = {(cuuint32_t)kLK, box_rows, planes};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t limb_smem_bytes() {
  return 1024 + (size_t)kLStages * kLStageBytes + (2 * kLStages + 3) * 8 + 16;
}

long long family_top(uint32_t type) {
  return type == kQ8_0 ? Fam<kQ8_0>::top : type == kQ4_K ? Fam<kQ4_K>::top : Fam<kQ6_K>::top;
}

template <uint32_t T>
cudaError_t launch_main(const GemvPlan &pl, const uint8_t *pack, const LimbLayout &lay,
                        size_t n_out, size_t n_in, size_t n_cols, const int8_t *codes, size_t ld,
                        const uint8_t *exps, size_t ldb, const LWork &w, long long *out_q32,
                        float *out_f32, unsigned long long *status, int sm_count,
                        cudaStream_t stream) {
  CUtensorMap map_x;
  const size_t np = lpad_cols(n_cols);
  if (!make_plane_map(&map_x, w.xp, lay.kp, np, kXDig, kLN)) return cudaErrorInvalidValue;
  LArgs a;
  a.kmin = lay.kmin;
  a.w = w;
  a.out_q32 = out_q32;
  a.out_f32 = out_f32;
  a.status = status;
  a.n_out = n_out;
  a.n_cols = (int)n_cols;
  a.kstages = (int)(lay.kp / kLK);
  a.n_tiles = (int)(np / kLN);
  a.tiles = (int)ltiles(n_out, n_cols);
  a.iters = (long long)a.tiles * a.kstages;
  a.G = (int)std::max<long long>(
      1, std::min<long long>(sm_count, (a.iters + kLMinIters - 1) / kLMinIters));
  a.geo = PackGeo{pack, pl.units, pl.L};
  a.codes = codes;
  a.exps = exps;
  a.ld = ld;
  a.ldb = ldb;
  a.n_in = n_in;
  cudaError_t e = cudaFuncSetAttribute(limb_gemm_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)limb_smem_bytes());
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.G + kLFallbackCtas));
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = limb_smem_bytes();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, limb_gemm_kernel<T>,
                            *reinterpret_cast<const CUtensorMap *>(lay.map), map_x, a);
}

cudaError_t launch_main_any(uint32_t type, const GemvPlan &pl, const uint8_t *pack,
                            const LimbLayout &lay, size_t n_out, size_t n_in, size_t n_cols,
                            const int8_t *codes, size_t ld, const uint8_t *exps, size_t ldb,
                            const LWork &w, long long *out_q32, float *out_f32,
                            unsigned long long *status, int sm_count, cudaStream_t stream) {
  switch (type) {
    case kQ8_0:
      return launch_main<kQ8_0>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                out_q32, out_f32, status, sm_count, stream);
    case kQ4_K:
      return launch_main<kQ4_K>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                out_q32, out_f32, status, sm_count, stream);
    case kQ6_K:
      return launch_main<kQ6_K>(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                                out_q32, out_f32, status, sm_count, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

LPrepArgs prep_args(uint32_t type, const LimbLayout &lay, size_t n_out, size_t n_in,
                    size_t n_cols, const LWork &w, unsigned long long *status) {
  LPrepArgs pa{};
  pa.n_in = n_in;
  pa.kp = lay.kp;
  pa.nb = (int)((n_in + 31) / 32);
  pa.n_cols = (int)n_cols;
  pa.tiles = (int)ltiles(n_out, n_cols);
  pa.top = family_top(type);
  pa.w = w;
  pa.status = status;
  return pa;
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
  lay->kp = lpad_k(n_in);
  lay->m_pad = (n_out + kLM - 1) / kLM * kLM;
  const size_t planes_bytes = (size_t)kWDig * lay->m_pad * lay->kp;
  const size_t total = planes_bytes + lay->m_pad * 4 + 16;
  cudaError_t e = cudaMalloc(&lay->base, total);
  if (e != cudaSuccess) {
    lay->base = nullptr;
    return e;
  }
  lay->planes = reinterpret_cast<int8_t *>(lay->base);
  lay->kmin = reinterpret_cast<int32_t *>(static_cast<uint8_t *>(lay->base) + planes_bytes);
  int *bad = reinterpret_cast<int *>(lay->kmin + lay->m_pad);
  e = cudaMemsetAsync(lay->kmin, 0, lay->m_pad * 4 + 16, stream);
  const PackGeo geo{pack, pl.units, pl.L};
  const size_t items = lay->m_pad * (lay->kp / 32);
  const unsigned rows_grid = (unsigned)((n_out + 7) / 8);
  const unsigned items_grid = (unsigned)((items + 127) / 128);
  if (e == cudaSuccess) {
    switch (type) {
      case kQ8_0:
        limb_row_kmin<kQ8_0><<<rows_grid, 256, 0, stream>>>(geo, n_out, n_in, lay->kmin);
        limb_build_planes<kQ8_0><<<items_grid, 128, 0, stream>>>(
            geo, n_out, n_in, lay->m_pad, lay->kp, lay->kmin, lay->planes, bad);
        break;
      case kQ4_K:
        limb_row_kmin<kQ4_K><<<rows_grid, 256, 0, stream>>>(geo, n_out, n_in, lay->kmin);
        limb_build_planes<kQ4_K><<<items_grid, 128, 0, stream>>>(
            geo, n_out, n_in, lay->m_pad, lay->kp, lay->kmin, lay->planes, bad);
        break;
      default:
        limb_row_kmin<kQ6_K><<<rows_grid, 256, 0, stream>>>(geo, n_out, n_in, lay->kmin);
        limb_build_planes<kQ6_K><<<items_grid, 128, 0, stream>>>(
            geo, n_out, n_in, lay->m_pad, lay->kp, lay->kmin, lay->planes, bad);
        break;
    }
    e = cudaGetLastError();
  }
  int h = 1;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h, bad, 4, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess &&
      !make_plane_map(reinterpret_cast<CUtensorMap *>(lay->map), lay->planes, lay->kp,
                      lay->m_pad, kWDig, kLM))
    e = cudaErrorInvalidValue;
  if (e != cudaSuccess) {
    cudaFree(lay->base);
    *lay = LimbLayout{};
    return e;
  }
  lay->ok = h == 0;
  if (!lay->ok) {  // some weight needs more than four digits: no digit planes for this tensor
    cudaFree(lay->base);
    *lay = LimbLayout{};
  }
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
  limb_prep_kernel<<<(unsigned)lpad_cols(n_cols), 256, 0, stream>>>(pa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_main_any(type, pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w,
                         out_q32, out_f32, status, sm_count, stream);
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
  limb_quant_prep_kernel<<<(unsigned)lpad_cols(n_cols), 256, smem, stream>>>(pa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_main_any(type, pl, pack, lay, n_out, n_in, n_cols, w.qcodes, lay.kp, w.qexps,
                         lay.kp / 32, w, out_q32, out_f32, status, sm_count, stream);
}

}  // namespace apx
