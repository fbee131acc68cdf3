// apx_gemm.cu — exact Q8_0 prefill projection on the 5th-generation tensor cores (tcgen05).
//
// Contract (src/engine/kern/matmat.rs:92-134, the exact GEMM of src/engine/kern/gemm.rs:1-31,
// 438-580): column c of the k-column projection equals matvec_q8act(W, qs[c]) bit for bit.
// For Q8_0 every term of the sum is a scaled int32 block dot: with the f16 weight scale
// split as d_{r,b} = m_{r,b}·2^k_{r,b} (src/engine/kern/pow2.rs:52-64) and the activation
// scale S_{c,b} = 2^e_{c,b},
//     y[r,c] = round_shift_32( Σ_b m_{r,b}·2^(k_{r,b}+e_{c,b}) · D_b[r,c] ),
//     D_b[r,c] = Σ_{i<32} q_{r,b,i}·x_{c,b,i}.
// The tensor cores form every block's dot D_b exactly (kind::i8, one MMA per block with K = 32,
// s32 accumulators in TMEM).  The epilogue folds each block relative to the token's smallest
// activation exponent emin_c and the row's smallest weight exponent kmin_r, the way the
// reference's gemm_q8_0 shift-accumulates (gemm.rs:99-102 spread_limit, 470-486):
//     acc += (D_b · 2^s) · M_{r,b},   s = e_{c,b} − emin_c,   M = m·2^(k − kmin_r)
// one shift and one widening multiply-add per output and block.  |D| < 2^19, so D·2^s stays in
// int32 for s <= 11, and the sum stays exact in i64 while nb terms below 2^(30 + s + kspread)
// stay below 2^62 (gemm_max_shift bounds s per tensor).  y = round_shift_32(acc·2^(kmin_r +
// emin_c)) (pow2.rs:76-96 `finish`).  Columns whose activation spread exceeds that bound, outside
// the reference's i128 call bound (chart/mod.rs:362-383) or holding a code of -128 take
// matvec_fixed instead: the checked row path, by extra CTAs of the same launch.
//
// Layout in HBM (built once per tensor, on its first multi-column call): the int8 codes
// row-major, K padded to 128 bytes and rows to 128, for 2D TMA; M_{r,b} as int32 [block][row];
// kmin per row.  Per call, the prep kernel writes the activation codes row-major per token
// (zero for zero-scale blocks, past n_in and off the GEMM), s as int32 [block][token], emin and
// a per-token route (refused / GEMM / checked rows).
//
// Pipeline (one CTA per 128-row × 64-token tile and K range):
//   warp 0      TMA producer: 128-byte K slabs of W (128 rows) and of the codes (64 tokens),
//               128B-swizzled, and the slab's M and s tables, into an 8-stage ring
//               (cp.async.bulk.tensor, no multicast);
//   warp 1      TMEM owner and MMA issuer: a slab's 4 blocks into one of 2 TMEM buffers of
//               4 × 64 columns, one tcgen05.commit per slab;
//   warps 2..9  epilogue: tcgen05.ld of 32 rows × 32 tokens per block (two blocks' loads in
//               flight), the shift-and-fold per output and block.
// Every wait is bounded (kWaitLimit); a wait that gives up records APX_ERR_DEVICE_TIMEOUT,
// drains what the CTA has in flight and frees its TMEM before returning.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"
#include "apx_quant.cuh"
#include "apx_tc.cuh"

namespace apx {

constexpr int kTileM = 128;
constexpr int kTileN = 64;
constexpr int kSlab = 128;  // K bytes per stage (4 blocks): one 128B swizzle atom per row
constexpr int kStages = 8;
constexpr int kBufs = 2;    // TMEM buffers of one stage: 4 blocks × kTileN columns (512 in all)
constexpr int kBufCols = (kSlab / 32) * kTileN;
constexpr int kEpiWarps = 16;  // 4 per SM sub-partition: 32 rows × kEpiTok tokens each
constexpr int kEpiTok = kTileN * 4 / kEpiWarps;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kMaxShift = 11;  // s = e − emin_c <= 11: |D·2^s| < 2^30 stays in int32
constexpr int kStageA = kTileM * kSlab;           // 16 KB of weight codes
constexpr int kStageB = kTileN * kSlab;           // 8 KB of activation codes
constexpr int kStageM = kTileM * (kSlab / 32) * 4;  // 2 KB: M of 4 blocks × 128 rows
constexpr int kStageS = kTileN * (kSlab / 32) * 4;  // 1 KB: s of 4 blocks × 64 tokens
constexpr int kStageBytes = 27 * 1024;            // one stage, 1024-aligned
constexpr int kFallbackCtas = 32;        // extra CTAs of each launch for the checked columns
constexpr int kSpreadLimit = 20;         // weight exponent spread: M stays in int32
constexpr int kMaxBlocks = (1 << 13) - 1;  // the i64 fold's bound on the block count
constexpr unsigned kRouteNone = 0, kRouteGemm = 1, kRouteChecked = 2;

static_assert(kEpiWarps % 4 == 0 && (kEpiTok == 16 || kEpiTok == 32), "epilogue split");
static_assert(kStageA % 1024 == 0 && kStageB % 1024 == 0 && kStageBytes % 1024 == 0 &&
                  kStageA + kStageB + kStageM + kStageS <= kStageBytes,
              "stages keep the 1024-byte alignment of the swizzled tiles");

// ---- descriptors ---------------------------------------------------------------------------

// Instruction descriptor of kind::i8: D s32 (2) at bits 4-5, A and B signed 8-bit (1) at
// bits 7-9 and 10-12, both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kTileM >> 4) << 24);
}
constexpr uint32_t kIdesc64 = idesc_i8(kTileN);

// Shared-memory matrix descriptor of a K-major operand in the 128B-swizzled layout TMA
// writes: start address >> 4 in bits 0-13, leading byte offset 16 (>> 4) in bits 16-29,
// 8-row groups 1024 bytes apart (stride byte offset >> 4) in bits 32-45, version 1 in bits
// 46-47, layout type 2 (SWIZZLE_128B) in bits 61-63.  Only the start address varies.
constexpr uint64_t kDescHi = ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
                             ((uint64_t)1 << 46) | ((uint64_t)2 << 61);

// This warp's kEpiTok columns of 32 TMEM lanes.
template <int N>
__device__ __forceinline__ void tmem_ld_tok(uint32_t taddr, uint32_t (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld_tok<16>(uint32_t taddr, uint32_t (&v)[16]) {
  tmem_ld16_nowait(taddr, v);
}
template <>
__device__ __forceinline__ void tmem_ld_tok<32>(uint32_t taddr, uint32_t (&v)[32]) {
  tmem_ld32_nowait(taddr, v);
}

// acc += a·b, a 32×32 → 64-bit product added to a 64-bit sum.  Written in C++ so the compiler
// schedules the fold's 32 independent sums with the TMEM loads around them: in this kernel that
// measured faster than a fixed `mad.wide.s32` per output (49.7 → 46.0 us on 4864x896x512).
__device__ __forceinline__ void mad_wide(long long &acc, int a, int b) {
  acc += (long long)a * (long long)b;
}

// acc[j] += (D[j]·2^s[j])·M for the warp's tokens: the block dot D from the tensor cores, the
// token's shift s for this block from shared memory (the same 32 words for every lane: one
// broadcast read per 4 tokens), one shift and one widening multiply-add each.  |D| < 2^19 and
// s <= 11, so D·2^s stays in int32; |M| < 2^31.
__device__ __forceinline__ void fold(long long (&acc)[kEpiTok], const uint32_t (&d)[kEpiTok],
                                     const int *s, int32_t m) {
#pragma unroll
  for (int j4 = 0; j4 < kEpiTok / 4; j4++) {
    const int4 s4 = reinterpret_cast<const int4 *>(s)[j4];
    mad_wide(acc[4 * j4 + 0], (int)(d[4 * j4 + 0] << s4.x), m);
    mad_wide(acc[4 * j4 + 1], (int)(d[4 * j4 + 1] << s4.y), m);
    mad_wide(acc[4 * j4 + 2], (int)(d[4 * j4 + 2] << s4.z), m);
    mad_wide(acc[4 * j4 + 3], (int)(d[4 * j4 + 3] << s4.w), m);
  }
}

// ---- per-call workspace ------------------------------------------------------------------------

struct WorkView {
  int *cnt;          // split-K arrival counters, one per tile (a fixed 4 KB at the start)
  long long *part;   // split-K partial sums
  int8_t *bcodes;    // [n_cols_pad][kp]: the GEMM columns' codes (zero elsewhere)
  int32_t *shift;    // [kp / 32][n_cols_pad]: s = e − emin_c of block b of token c (0 elsewhere)
  int32_t *emin;     // [n_cols_pad]
  uint32_t *route;   // [n_cols_pad]
  int32_t *fb;       // [0] count, [1] CTAs done, [2..] checked-route columns
  int8_t *qcodes;    // f32 path: the checked columns' codes [n_cols_pad][kp]
  uint8_t *qexps;    // and exponent bytes [n_cols_pad][kp / 32]
};

static __host__ __device__ size_t cols_pad(size_t n_cols) {
  return (n_cols + kTileN - 1) / kTileN * kTileN;
}

size_t gemm_work_head_bytes(size_t n_cols) { return (n_cols + 2 + 63) / 64 * 256; }

constexpr size_t kCntBytes = 4096;  // split-K counters: at most 1024 split tiles

// The launch's work split: tiles [0, full) whole, one CTA each, in whole rounds of one CTA per
// SM; each remaining tile over `ks` CTAs (split K) so that the short last round fills the SMs.
// With fewer tiles than SMs every tile is split: the largest split that keeps one wave.
struct Split {
  int full, ks;
  int pieces(int tiles) const { return full + (tiles - full) * ks; }
};

static Split gemm_split(size_t tiles, int kslabs, int sm_count) {
  if (tiles == 0 || sm_count <= 0) return Split{(int)tiles, 1};
  const size_t rem = tiles % (size_t)sm_count;
  if (rem == 0 || rem > kCntBytes / 4) return Split{(int)tiles, 1};
  const int ks = (int)std::min<size_t>({(size_t)sm_count / rem, (size_t)kslabs, (size_t)8});
  if (ks <= 1) return Split{(int)tiles, 1};
  return Split{(int)(tiles - rem), ks};
}

// The split tiles' partial sums: one tile's worth per split CTA, and a launch has at most
// sm_count of them.
static size_t part_bytes(int sm_count) {
  return (size_t)std::max(sm_count, 1) * kTileM * kTileN * sizeof(long long);
}

static WorkView work_view(void *base, size_t n_cols, int nb, size_t kp, int sm_count) {
  uint8_t *p = static_cast<uint8_t *>(base);
  const size_t np = cols_pad(n_cols);
  WorkView w;
  w.cnt = reinterpret_cast<int *>(p);
  p += kCntBytes;
  w.part = reinterpret_cast<long long *>(p);
  p += part_bytes(sm_count);
  w.fb = reinterpret_cast<int32_t *>(p);
  p += gemm_work_head_bytes(n_cols);
  w.route = reinterpret_cast<uint32_t *>(p);
  p += np * 4;
  w.emin = reinterpret_cast<int32_t *>(p);
  p += np * 4;
  w.bcodes =
      reinterpret_cast<int8_t *>((reinterpret_cast<uintptr_t>(p) + 255) & ~(uintptr_t)255);
  p = reinterpret_cast<uint8_t *>(w.bcodes) + np * kp;
  w.shift =
      reinterpret_cast<int32_t *>((reinterpret_cast<uintptr_t>(p) + 255) & ~(uintptr_t)255);
  p = reinterpret_cast<uint8_t *>(w.shift + (kp / 32) * np);
  w.qcodes = reinterpret_cast<int8_t *>(p);
  p += np * kp;
  w.qexps = p;
  (void)nb;
  return w;
}

static size_t gemm_tiles(size_t n_out, size_t n_cols) {
  return ((n_out + kTileM - 1) / kTileM) * ((n_cols + kTileN - 1) / kTileN);
}

// The layout of work_view: counters, split accumulators, head, route and emin, the B operand,
// the shift table, the checked columns' codes and exponent bytes (with alignment slack).
size_t gemm_work_bytes(size_t n_cols, size_t n_in, size_t n_out, int sm_count) {
  const size_t kp = (n_in + kSlab - 1) / kSlab * kSlab;
  const size_t np = cols_pad(n_cols);
  (void)n_out;
  return kCntBytes + part_bytes(sm_count) + gemm_work_head_bytes(n_cols) + 2 * np * 4 + 256 +
         np * kp + 256 + (kp / 32) * np * 4 + np * kp + np * (kp / 32);
}

// ---- activation prep: describe, route, B operand, shift table --------------------------------

// The GEMM's split-K arrival counters, zero before every launch.
__device__ __forceinline__ void zero_counters(const WorkView &w) {
  for (int i = threadIdx.x; i < (int)(kCntBytes / 4); i += blockDim.x) w.cnt[i] = 0;
}

// A column the GEMM does not take (padding token, refused or checked): zero codes and shifts.
__device__ __forceinline__ void zero_column(const WorkView &w, int c, size_t np, size_t kp) {
  for (size_t j = (size_t)threadIdx.x * 16; j < kp; j += (size_t)blockDim.x * 16)
    *reinterpret_cast<uint4 *>(w.bcodes + (size_t)c * kp + j) = make_uint4(0, 0, 0, 0);
  for (size_t b = threadIdx.x; b < kp / 32; b += blockDim.x) w.shift[b * np + c] = 0;
}

struct PrepArgs {
  const int8_t *codes;  // caller codes, column c at c·ld
  const uint8_t *exps;  // caller exponent bytes, column c at c·ldb
  const ActDesc *descs; // the quantizer's descriptors (a refusal there wins), or null
  size_t ld, ldb, n_in, kp;
  int nb, n_cols;
  int max_shift;  // the largest spread e − emin a GEMM column may have on this tensor
  WorkView w;
  unsigned long long *status;  // column c's refusal word at status[c·2]
};

__global__ void __launch_bounds__(256) gemm_prep_kernel(PrepArgs a) {
  __shared__ int s_emin, s_emax, s_status;
  __shared__ unsigned s_m128, s_route;
  const int c = blockIdx.x;
  const size_t np = cols_pad((size_t)a.n_cols);
  pdl_launch_dependents();  // the GEMM may start its weight loads now
  if (c == 0) zero_counters(a.w);
  if (c >= a.n_cols) {  // padding tokens of the last tile: zero codes and shifts
    zero_column(a.w, c, np, a.kp);
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
    s_m128 = 0;
    if (a.descs && s_status == APX_OK) {  // the quantizer's descriptor: no re-scan
      const ActDesc d = a.descs[c];
      s_emax = d.emax;
      s_emin = d.emax >= 0 ? d.emin : 1 << 30;
      s_m128 = d.pad[0] & 1u;
    }
  }
  __syncthreads();
  if (s_status != APX_OK) {  // refused by the quantizer: its codes and exponents are not set
    zero_column(a.w, c, np, a.kp);
    if (threadIdx.x == 0) {
      atomicMin(a.status + (size_t)c * 2, pack_status(0, (unsigned)s_status, 0));
      a.w.emin[c] = 0;
      a.w.route[c] = kRouteNone;
    }
    return;
  }
  const int8_t *codes = a.codes + (size_t)c * a.ld;
  const uint8_t *exps = a.exps + (size_t)c * a.ldb;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  // describe (QuantAct's Q32.32 image, chart/mod.rs:124-181), as the GEMV's descriptor does,
  // unless the quantizer's descriptor came with the call
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
    if (__any_sync(0xFFFFFFFFu, code == -128) && lane == 0) atomicOr(&s_m128, 1u);
    if (lane == 0) {
      atomicMin(&s_emin, (int)e);
      atomicMax(&s_emax, (int)e);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int emin = s_emax >= 0 ? s_emin : 0;
    unsigned route = kRouteNone;
    if (s_status != APX_OK) {
      atomicMin(a.status + (size_t)c * 2, pack_status(0, (unsigned)s_status, 0));
    } else if (!s_m128 && bound_ok((long long)a.n_in, Fam<kQ8_0>::top, s_emax) &&
               (s_emax < 0 || s_emax - emin <= a.max_shift)) {
      route = kRouteGemm;
    } else {
      route = kRouteChecked;
      const int slot = atomicAdd(a.w.fb, 1);
      a.w.fb[2 + slot] = c;
    }
    s_emin = emin;
    s_route = route;
    a.w.emin[c] = emin;
    a.w.route[c] = route;
  }
  __syncthreads();
  const bool gemm = s_route == kRouteGemm;
  const int emin = s_emin;
  // the B operand (the codes; zero for zero-scale blocks, past n_in and off the GEMM) and
  // every block's shift s = e − emin
  int8_t *dst = a.w.bcodes + (size_t)c * a.kp;
  for (size_t b = threadIdx.x; b < a.kp / 32; b += blockDim.x) {
    const unsigned e = b < (size_t)a.nb ? exps[b] : APX_EXP_ZERO;
    a.w.shift[b * np + c] = gemm && e != APX_EXP_ZERO ? (int)e - emin : 0;
  }
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (gemm && j < a.n_in && exps[j / 32] != APX_EXP_ZERO) {
      if (j + 16 <= a.n_in) {
        v = *reinterpret_cast<const uint4 *>(codes + j);
      } else {
        uint8_t t[16];
        for (int i = 0; i < 16; i++) t[i] = j + i < a.n_in ? (uint8_t)codes[j + i] : 0;
        memcpy(&v, t, 16);
      }
    }
    *reinterpret_cast<uint4 *>(dst + j) = v;
  }
}

// ---- fused quantize-and-prep of f32 columns (the prefill's f32 boundary) ------------------
//
// One CTA per column: f32_to_fixed + quant_act of the column into shared memory (the same
// per-block arithmetic as the column quantizer, apx_quant.cuh), its descriptor, route and
// planes, in one pass over the f32 input.  Codes and exponent bytes leave shared memory only
// for a column the checked rows take.

struct QPrepArgs {
  const float *x;  // column c at x + c·ldx (16-byte aligned, ldx a multiple of 4)
  size_t ldx, n_in, kp;
  int nb, n_cols;
  int max_shift;  // as PrepArgs::max_shift
  WorkView w;
  unsigned long long *status;  // column c's refusal word at status[c·2]
};

constexpr int kQPrepChunks = 4;      // 128-lane chunks in flight per warp
constexpr size_t kQPrepMaxIn = 16384;  // the column staged in shared memory

__global__ void __launch_bounds__(256) gemm_quant_prep_kernel(QPrepArgs a) {
  extern __shared__ __align__(16) uint8_t qsm[];
  int8_t *scodes = reinterpret_cast<int8_t *>(qsm);  // kp bytes
  uint8_t *sexps = qsm + a.kp;                        // kp / 32 bytes
  __shared__ int s_emin, s_emax, s_status;
  __shared__ unsigned s_route;
  const int c = blockIdx.x;
  const size_t np = cols_pad((size_t)a.n_cols);
  pdl_launch_dependents();  // the GEMM may start its weight loads now
  if (c == 0) zero_counters(a.w);
  if (c >= a.n_cols) {  // padding tokens of the last tile: zero codes and shifts
    zero_column(a.w, c, np, a.kp);
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
  const size_t chunks = a.kp / 128;  // lanes past n_in read as zero: zero codes
  int w_emin = 1 << 30, w_emax = -1, w_status = APX_OK;
  for (size_t round = 0; round * nw * kQPrepChunks < chunks; round++) {
    float4 f4[kQPrepChunks];
#pragma unroll
    for (int u = 0; u < kQPrepChunks; u++) {
      const size_t j = ((round * kQPrepChunks + u) * nw + warp) * 128 + 4 * lane;
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
    for (int u = 0; u < kQPrepChunks; u++) {
      const size_t cbase = ((round * kQPrepChunks + u) * nw + warp) * 128;
      if (cbase >= a.kp) break;  // warp-uniform
      const size_t j = cbase + 4 * lane;
      uint32_t packed;
      int e;
      bool ok;
      quant_quad(f4[u], packed, e, ok);
      *reinterpret_cast<uint32_t *>(scodes + j) = ok ? packed : 0u;
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
      } else if ((lane & 7) == 0 && j / 32 < a.kp / 32) {
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
    zero_column(a.w, c, np, a.kp);
    if (threadIdx.x == 0) {
      atomicMin(a.status + (size_t)c * 2, pack_status(0, (unsigned)s_status, 0));
      a.w.emin[c] = 0;
      a.w.route[c] = kRouteNone;
    }
    return;
  }
  if (threadIdx.x == 0) {  // the route, as gemm_prep_kernel decides it (no code is -128 here)
    const int emin = s_emax >= 0 ? s_emin : 0;
    unsigned route;
    if (bound_ok((long long)a.n_in, Fam<kQ8_0>::top, s_emax) &&
        (s_emax < 0 || s_emax - emin <= a.max_shift)) {
      route = kRouteGemm;
    } else {
      route = kRouteChecked;
      const int slot = atomicAdd(a.w.fb, 1);
      a.w.fb[2 + slot] = c;
    }
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
  // the B operand (zero codes for zero blocks and past n_in already) and the shifts
  int8_t *dst = a.w.bcodes + (size_t)c * a.kp;
  for (size_t j = (size_t)threadIdx.x * 16; j < a.kp; j += (size_t)blockDim.x * 16)
    *reinterpret_cast<uint4 *>(dst + j) =
        gemm ? *reinterpret_cast<const uint4 *>(scodes + j) : make_uint4(0, 0, 0, 0);
  for (size_t b = threadIdx.x; b < a.kp / 32; b += blockDim.x) {
    const unsigned e = sexps[b];
    a.w.shift[b * np + c] = gemm && e != APX_EXP_ZERO ? (int)e - emin : 0;
  }
}

// ---- the GEMM --------------------------------------------------------------------------------

struct GemmArgs {
  const int32_t *wmul;  // [nb_pad][m_pad]
  const int32_t *kmin;  // [m_pad]
  WorkView w;
  long long *out_q32;   // [n_cols][n_out] or null
  float *out_f32;       // [n_cols][n_out] or null
  unsigned long long *status;  // column c at status[c·2]
  size_t n_out, m_pad;
  int n_cols, nb, kslabs, m_tiles, tiles;
  // tiles [0, full) one CTA each; every later tile over ksplit CTAs (split K), each over a
  // contiguous range of slabs: their exact i64 partial sums meet in `part`, and the last to
  // arrive (per split tile counter) finishes.  pieces = full + (tiles - full)·ksplit.
  int full, ksplit, pieces;
  long long *part;  // [tiles - full][ksplit][kEpiWarps][kEpiTok tokens][32 lanes]
  int *cnt;         // [tiles - full] arrivals, zeroed by the prep kernel
  // checked route (matvec_fixed per row) of the columns the prep kernel listed
  PackGeo geo;
  const int8_t *codes;
  const uint8_t *exps;
  size_t ld, ldb, n_in;
};

// Bounded wait until *p >= target (acquire at GPU scope): kWaitLimit polls or about one
// second, like mbar_wait; false when it gives up.
__device__ __forceinline__ bool wait_count(const int *p, int target) {
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int it = 0; it < kWaitLimit; it++) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    __nanosleep(64);
    if ((it & 63) == 63) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - t0 > 1000000000ull) return false;
    }
  }
  return false;
}

__device__ __forceinline__ void checked_columns(const GemmArgs g) {
  volatile int32_t *fb = g.w.fb;
  const long long n = fb[0];
  const long long items = n * (long long)g.n_out;
  const long long first =
      (long long)(blockIdx.x - g.pieces) * blockDim.x + threadIdx.x;
  for (long long i = first; i < items; i += (long long)kFallbackCtas * blockDim.x) {
    const int c = fb[2 + i / (long long)g.n_out];
    const size_t row = (size_t)(i % (long long)g.n_out);
    checked_row<kQ8_0>(g.geo, row, g.n_out, g.n_in, g.codes + (size_t)c * g.ld,
                       g.exps + (size_t)c * g.ldb,
                       g.out_q32 ? g.out_q32 + (size_t)c * g.n_out : nullptr,
                       g.out_f32 ? g.out_f32 + (size_t)c * g.n_out : nullptr,
                       g.status + (size_t)c * 2);
  }
  // every checked CTA reads the list; the last to finish resets it for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(g.w.fb + 1, 1) == kFallbackCtas - 1) {
      g.w.fb[0] = 0;
      g.w.fb[1] = 0;
      __threadfence();
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_q8_0_kernel(const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_x,
                     const __grid_constant__ CUtensorMap map_m,
                     const __grid_constant__ CUtensorMap map_s, GemmArgs g) {
  if ((int)blockIdx.x >= g.pieces) {
    pdl_wait();  // the prep kernel's list and codes
    checked_columns(g);
    return;
  }
  // stage st: weight codes (16 KB, 128B-swizzled), activation codes (8 KB, swizzled), M of
  // its 4 blocks × 128 rows and s of its 4 blocks × 64 tokens (int32)
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
  uint64_t *full = bars, *empty = bars + kStages, *dfull = bars + 2 * kStages;
  uint64_t *dempty = dfull + kBufs, *mdone = dempty + kBufs;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
  int *timeout = reinterpret_cast<int *>(tmem_slot + 1);
  // per token of the tile: the finish shift emin_c, or -1 where the token is not the GEMM's
  // (16-byte aligned for vector reads)
  int *stok = reinterpret_cast<int *>((reinterpret_cast<uintptr_t>(timeout + 1) + 15) &
                                      ~(uintptr_t)15);
  int *sflag = stok + kTileN;  // split K: this CTA is the tile's last split
  auto stage_a = [&](int st) { return smem + st * kStageBytes; };
  auto stage_m = [&](int st) {
    return reinterpret_cast<const int32_t *>(smem + st * kStageBytes + kStageA + kStageB);
  };
  auto stage_s = [&](int st) {
    return reinterpret_cast<const int *>(smem + st * kStageBytes + kStageA + kStageB + kStageM);
  };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // this CTA's tile, and its share of the tile's slabs [kt0, kt0 + nk) of ks
  int tile, split = 0, ks = 1;
  if ((int)blockIdx.x < g.full) {
    tile = (int)blockIdx.x;
  } else {
    const int i = (int)blockIdx.x - g.full, r = g.tiles - g.full;
    tile = g.full + i % r;
    split = i / r;
    ks = g.ksplit;
  }
  const int stile = tile - g.full;  // index among the split tiles
  const int mt = tile % g.m_tiles, nt = tile / g.m_tiles;
  const int kt0 = (int)((long long)split * g.kslabs / ks);
  const int nk = (int)((long long)(split + 1) * g.kslabs / ks) - kt0;
  const int m0 = mt * kTileM, n0 = nt * kTileN;
  const int np = (int)cols_pad((size_t)g.n_cols);

  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; st++) {
      mbar_init(full + st, 1);
      // released by the epilogue warps: each has seen the stage's MMAs complete (dfull)
      mbar_init(empty + st, kEpiWarps);
    }
    for (int b = 0; b < kBufs; b++) {
      mbar_init(dfull + b, 1);
      mbar_init(dempty + b, kEpiWarps);
    }
    mbar_init(mdone, 1);
    *timeout = 0;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_m)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_s)) : "memory");
  }
  if (warp == 1) {  // TMEM: kBufs × kBufCols columns of 32-bit accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kBufs * kBufCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The weight codes and their M table are the tensor's, constant since its upload: the first
  // stages' loads of them go out before the wait for the prep kernel (programmatic dependent
  // launch).  Everything the prep kernel writes is read after the wait.
  constexpr uint32_t kStageTx = kStageA + kStageB + kStageM + kStageS;
  const int pre = min(nk, kStages);
  if (threadIdx.x == 0) {
    for (int lk = 0; lk < pre; lk++) {
      uint8_t *base = stage_a(lk);
      mbar_expect_tx(full + lk, kStageTx);
      tma_load_2d(base, &map_w, (kt0 + lk) * kSlab, m0, full + lk);
      tma_load_2d(base + kStageA + kStageB, &map_m, m0, (kt0 + lk) * (kSlab / 32), full + lk);
    }
  }
  pdl_wait();
  if (threadIdx.x >= 64 && threadIdx.x < 64 + kTileN) {
    const int c = n0 + (int)threadIdx.x - 64;
    const unsigned rw = c < g.n_cols ? g.w.route[c] : kRouteNone;
    const bool gemm_col = (rw & 0xFFu) == kRouteGemm;
    stok[threadIdx.x - 64] = gemm_col ? g.w.emin[c] : -1;
  }
  __syncthreads();

  if (warp == 0) {
    // ---- TMA producer (lane 0 issues): per slab W, the codes, M and s ----
    int issued = 0;
    for (int lk = 0; lk < nk; lk++) {
      const int kt = kt0 + lk, st = lk % kStages, use = lk / kStages;
      int stop = 0;
      if (lane == 0) {
        if (use > 0 && !mbar_wait(empty + st, (use - 1) & 1)) {
          atomicExch(timeout, 1);
          stop = 1;
        } else {
          uint8_t *base = stage_a(st);
          if (lk >= pre) {  // the first stages' W and M went out before the wait
            mbar_expect_tx(full + st, kStageTx);
            tma_load_2d(base, &map_w, kt * kSlab, m0, full + st);
            tma_load_2d(base + kStageA + kStageB, &map_m, m0, kt * (kSlab / 32), full + st);
          }
          tma_load_2d(base + kStageA, &map_x, kt * kSlab, n0, full + st);
          tma_load_2d(base + kStageA + kStageB + kStageM, &map_s, n0, kt * (kSlab / 32),
                      full + st);
          issued++;
        }
      }
      if (__shfl_sync(0xFFFFFFFFu, stop, 0)) break;
    }
    // every copy this thread started has landed before the CTA may exit
    if (lane == 0)
      for (int lk = issued > kStages ? issued - kStages : 0; lk < issued; lk++)
        mbar_wait(full + lk % kStages, (lk / kStages) & 1);
  } else if (warp == 1) {
    // ---- MMA issuer: one MMA per block (its dot D, K = 32); a stage's 4 blocks into one
    // TMEM buffer, one commit per stage ----
    if (lane == 0) {
      const uint64_t a0 = kDescHi | (smem_addr(stage_a(0)) >> 4);
      const uint64_t b0 = kDescHi | (smem_addr(stage_a(0) + kStageA) >> 4);
      bool ok = true;
      for (int lk = 0; lk < nk; lk++) {
        const int kt = kt0 + lk, st = lk % kStages, buf = lk % kBufs;
        if (!mbar_wait(full + st, (lk / kStages) & 1) ||
            (lk >= kBufs && !mbar_wait(dempty + buf, ((lk / kBufs) - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a0 + (uint64_t)(st * (kStageBytes >> 4));
        const uint64_t bd = b0 + (uint64_t)(st * (kStageBytes >> 4));
        const int nq = min(4, g.nb - 4 * kt);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (q >= nq) break;
          mma_i8(tmem + (uint32_t)(buf * kBufCols + q * kTileN), ad + 2 * q, bd + 2 * q,
                 kIdesc64, 0u);
        }
        mma_commit(dfull + buf);
      }
      if (!ok) atomicExch(timeout, 1);
      mma_commit(mdone);
      if (!mbar_wait(mdone, 0)) atomicExch(timeout, 1);
    }
  } else {
    // ---- epilogue: 32 rows × 32 tokens per warp; one wake-up per stage (4 blocks) ----
    const int lg = warp % 4;  // the TMEM lane quarter this warp may read
    const int tq = (warp - 2) / 4;
    const int rl = 32 * lg + lane;
    const size_t row = (size_t)m0 + rl;
    const int c0 = kEpiTok * tq;
    const uint32_t trow = tmem + ((uint32_t)(32 * lg) << 16) + (uint32_t)c0;
    long long acc[kEpiTok];
#pragma unroll
    for (int j = 0; j < kEpiTok; j++) acc[j] = 0;
    // the row's finish exponent, fetched now so the finish does not wait for it
    const unsigned kmin_row = row < g.m_pad ? (unsigned)__ldg(g.kmin + row) : 0u;
    bool ok = true;
    for (int lk = 0; lk < nk; lk++) {
      const int kt = kt0 + lk, st = lk % kStages, buf = lk % kBufs;
      // the stage's M table (TMA) and its dots (MMA commit)
      if (!mbar_wait(full + st, (lk / kStages) & 1) ||
          !mbar_wait(dfull + buf, (lk / kBufs) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int nq = min(4, g.nb - 4 * kt);
      const int32_t *sm = stage_m(st) + rl;
      const int *ss = stage_s(st) + c0;  // [4 blocks][64 tokens]: this warp's 32 tokens
      const uint32_t t = trow + (uint32_t)(buf * kBufCols);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        if (2 * h >= nq) break;
        uint32_t d0[kEpiTok], d1[kEpiTok];
        const bool two = 2 * h + 1 < nq;
        tmem_ld_tok(t + (uint32_t)(2 * h * kTileN), d0);
        if (two) tmem_ld_tok(t + (uint32_t)((2 * h + 1) * kTileN), d1);
        tmem_wait_ld();
        fold(acc, d0, ss + 2 * h * kTileN, sm[2 * h * kTileM]);
        if (two) fold(acc, d1, ss + (2 * h + 1) * kTileN, sm[(2 * h + 1) * kTileM]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dempty + buf);  // the dots are folded
        mbar_arrive(empty + st);    // and the stage's table read
      }
    }
    if (!ok) atomicExch(timeout, 1);
    // ---- finish: acc·2^(kmin_r + emin_c) rounded to Q32.32 and to f32, stored by each thread
    // (a split tile first meets its partial sums in L2) ----
    const int ew = warp - 2;
    bool all_ok = __all_sync(0xFFFFFFFFu, ok);
    if (ks > 1) {
      // Split K: every split stores its partial sums (coalesced), arrives on the tile's
      // counter and waits (bounded) until all ks have; then the splits share the finish: split
      // p takes the token quarters q with q % ks == p and adds the other splits' partials to
      // its own (exact: i64 addition wraps and the true sum fits).  The splits of a launch
      // never outnumber the SMs and a CTA fills its SM, so they are all resident together.
      // The prep kernel zeroes the counters before every launch.
      long long *mine =
          g.part + (((size_t)stile * ks + split) * kEpiWarps + ew) * (kEpiTok * 32);
#pragma unroll
      for (int j = 0; j < kEpiTok; j++) mine[j * 32 + lane] = acc[j];
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");
      if (threadIdx.x == 64) {
        atomicAdd(g.cnt + stile, 1);
        const bool all_in = wait_count(g.cnt + stile, ks);
        if (!all_in) atomicExch(timeout, 1);
        *sflag = all_in;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");
      if (*sflag == 0 || tq % ks != split) {
        all_ok = false;  // another split finishes these tokens (or the wait gave up)
      } else {
        __threadfence();
        for (int sp = 0; sp < ks; sp++) {
          if (sp == split) continue;
          const long long *other =
              g.part + (((size_t)stile * ks + sp) * kEpiWarps + ew) * (kEpiTok * 32);
#pragma unroll
          for (int j = 0; j < kEpiTok; j++) acc[j] += __ldcg(other + j * 32 + lane);
        }
      }
    }
    if (all_ok) {
      // The outputs straight from registers: for each token the warp's 32 lanes hold 32
      // consecutive rows, so each token's store is one coalesced segment of the column-major
      // output (128 bytes of f32, 256 of Q32.32).  The tokens' exponents are read up front.
      const unsigned kmin = kmin_row;
      const bool live = row < g.n_out;
      uint32_t bad = 0;  // bit j: token j's output leaves i64
      int ev[kEpiTok];
#pragma unroll
      for (int j = 0; j < kEpiTok; j += 4) {
        const int4 e4 = *reinterpret_cast<const int4 *>(stok + c0 + j);
        ev[j] = e4.x;
        ev[j + 1] = e4.y;
        ev[j + 2] = e4.z;
        ev[j + 3] = e4.w;
      }
      float *of = g.out_f32 ? g.out_f32 + (size_t)(n0 + c0) * g.n_out + row : nullptr;
      long long *oq = g.out_q32 ? g.out_q32 + (size_t)(n0 + c0) * g.n_out + row : nullptr;
      // Tokens off the GEMM route (e < 0) are never stored.  When every other token's shift
      // kmin + e lies in [32, 64), the loop below has no call in it (the general case is out of
      // line, and a call site would keep the chains from interleaving).
      int emn = 1 << 20, emx = -1;
#pragma unroll
      for (int j = 0; j < kEpiTok; j++)
        if (ev[j] >= 0) {
          emn = min(emn, ev[j]);
          emx = max(emx, ev[j]);
        }
      if (emx < 0 || ((int)kmin + emn >= 32 && (int)kmin + emx < 64)) {
#pragma unroll
        for (int j = 0; j < kEpiTok; j++) {
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
        for (int j = 0; j < kEpiTok; j++) {
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
        atomicMin(g.status + (size_t)(n0 + c0 + j) * 2, pack_status(row, kKindOutputOverflow, 0));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*timeout && threadIdx.x < kTileN && n0 + (int)threadIdx.x < g.n_cols)
    atomicMin(g.status + (size_t)(n0 + threadIdx.x) * 2,
              pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0));
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kBufs * kBufCols)
                 : "memory");
  }
}

// ---- the weight layout of the GEMM, from the packed units --------------------------------------

// Per row: kmin = the smallest f16 exponent k of its block scales, and the largest spread.
__global__ void gemm_row_exponents(PackGeo geo, size_t n_out, int nb, int32_t *kmin,
                                   int *spread) {
  const size_t row = blockIdx.x * (size_t)(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= n_out) return;
  int lo = 1 << 30, hi = -1;
  for (int b = lane; b < nb; b += 32) {
    int l;
    const uint8_t *ub = slot_unit(geo, kQ8_0, row, (size_t)b / 4, l);
    const int bi = b % 4;
    int m;
    unsigned k;
    f16_split(ub[4096 + l * 8 + 2 * bi] | (ub[4096 + l * 8 + 2 * bi + 1] << 8), m, k);
    lo = min(lo, (int)k);
    hi = max(hi, (int)k);
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xFFFFFFFFu, hi, o));
  }
  if (lane == 0) {
    kmin[row] = nb ? lo : 0;
    if (nb) atomicMax(spread, hi - lo);
  }
}

// Row-major int8 codes [m_pad][kp] and M_{r,b} = m·2^(k − kmin_r) as int32 [nb_pad][m_pad];
// zero for padding rows and blocks, and M = 0 where the spread leaves int32 (such a tensor
// never takes the GEMM route).
__global__ void gemm_build_layout(PackGeo geo, size_t n_out, int nb, int nb_pad, size_t m_pad,
                                  size_t kp, const int32_t *kmin, int8_t *codes, int32_t *wmul) {
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;  // (row, block)
  if (idx >= m_pad * (size_t)nb_pad) return;
  const size_t row = idx / nb_pad;
  const int b = (int)(idx % nb_pad);
  int32_t mul = 0;
  uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0;
  if (row < n_out && b < nb) {
    int l;
    const uint8_t *ub = slot_unit(geo, kQ8_0, row, (size_t)b / 4, l);
    const int bi = b % 4;
    int m;
    unsigned k;
    f16_split(ub[4096 + l * 8 + 2 * bi] | (ub[4096 + l * 8 + 2 * bi + 1] << 8), m, k);
    const unsigned sh = k - (unsigned)kmin[row];
    mul = sh <= (unsigned)kSpreadLimit ? m * (1 << sh) : 0;
    c0 = *reinterpret_cast<const uint4 *>(ub + ((2 * bi) * 32 + l) * 16);
    c1 = *reinterpret_cast<const uint4 *>(ub + ((2 * bi + 1) * 32 + l) * 16);
  }
  wmul[(size_t)b * m_pad + row] = mul;
  uint4 *dst = reinterpret_cast<uint4 *>(codes + row * kp + 32 * (size_t)b);
  dst[0] = c0;
  dst[1] = c1;
}

// ---- host side ---------------------------------------------------------------------------------

// A 2D uint8 map over `rows` rows of `inner` bytes (row stride `stride`), boxes of
// 128 bytes × box_rows, 128-byte swizzle; reads past either extent fill zeros.
static bool make_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                     uint64_t stride, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {(cuuint32_t)kSlab, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A 2D int32 table [rows][inner] (row stride inner·4 bytes), boxes of box_inner × 4 rows
// (one stage's blocks), no swizzle; rows past the extent fill zeros.
static bool make_table_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t rows,
                           uint32_t box_inner) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * 4};
  const cuuint32_t box[2] = {box_inner, (cuuint32_t)(kSlab / 32)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static_assert(sizeof(CUtensorMap) == sizeof(GemmLayout::map), "tensor map storage");

cudaError_t build_gemm_layout(const GemvPlan &pl, const uint8_t *pack, size_t n_out,
                              size_t n_in, GemmLayout *lay, cudaStream_t stream) {
  *lay = GemmLayout{};
  lay->nb = (int)((n_in + 31) / 32);
  lay->kp = (n_in + kSlab - 1) / kSlab * kSlab;
  lay->nb_pad = (int)(lay->kp / 32);
  lay->m_pad = (n_out + kTileM - 1) / kTileM * kTileM;
  const size_t codes_bytes = lay->m_pad * lay->kp;
  const size_t mul_bytes = (size_t)lay->nb_pad * lay->m_pad * 4;
  const size_t kmin_bytes = lay->m_pad * 4;
  const size_t total = codes_bytes + mul_bytes + kmin_bytes + 16;
  cudaError_t e = cudaMalloc(&lay->base, total);
  if (e != cudaSuccess) {
    lay->base = nullptr;
    return e;
  }
  lay->codes = reinterpret_cast<int8_t *>(lay->base);
  lay->wmul = reinterpret_cast<int32_t *>(static_cast<uint8_t *>(lay->base) + codes_bytes);
  lay->kmin = lay->wmul + (size_t)lay->nb_pad * lay->m_pad;
  int *spread = reinterpret_cast<int *>(lay->kmin + lay->m_pad);
  e = cudaMemsetAsync(lay->base, 0, total, stream);
  const PackGeo geo{pack, pl.units, pl.L};
  if (e == cudaSuccess && n_out && lay->nb) {
    gemm_row_exponents<<<(unsigned)((n_out + 7) / 8), 256, 0, stream>>>(geo, n_out, lay->nb,
                                                                        lay->kmin, spread);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && lay->nb) {
    const size_t items = lay->m_pad * (size_t)lay->nb_pad;
    gemm_build_layout<<<(unsigned)((items + 255) / 256), 256, 0, stream>>>(
        geo, n_out, lay->nb, lay->nb_pad, lay->m_pad, lay->kp, lay->kmin, lay->codes,
        lay->wmul);
    e = cudaGetLastError();
  }
  int h = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h, spread, 4, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  lay->kspread = h;
  if (e == cudaSuccess &&
      (!make_map(reinterpret_cast<CUtensorMap *>(lay->map), lay->codes, lay->kp, lay->m_pad,
                 lay->kp, kTileM) ||
       !make_table_map(reinterpret_cast<CUtensorMap *>(lay->map_m), lay->wmul, lay->m_pad,
                       (uint64_t)lay->nb_pad, kTileM)))
    e = cudaErrorInvalidValue;
  if (e != cudaSuccess) {
    cudaFree(lay->base);
    *lay = GemmLayout{};
  }
  return e;
}

void free_gemm_layout(GemmLayout *lay) {
  if (lay->base) cudaFree(lay->base);
  *lay = GemmLayout{};
}

static size_t gemm_smem_bytes() {
  return 1024 + (size_t)kStages * kStageBytes + (2 * kStages + 2 * kBufs + 1) * 8 + 32 +
         kTileN * 4 + 16;
}

bool gemm_shape_ok(size_t n_in) { return n_in && (n_in + 31) / 32 <= (size_t)kMaxBlocks; }

// The largest activation spread s = e − emin of a GEMM column on this tensor: every term
// |D·2^s·M| < 2^(30 + s + kspread) (|D| < 2^19, |M| < 2^(11 + kspread)), and nb <= 2^lg of
// them stay below 2^62.  gemm_supported keeps it at 2 or more.
static int gemm_max_shift(const GemmLayout &lay) {
  int lg = 0;
  while ((1 << lg) < lay.nb) lg++;
  return std::max(0, std::min(kMaxShift, 32 - lay.kspread - lg));
}

bool gemm_supported(const GemmLayout &lay) {
  // |D·2^s·M| < 2^(33 + kspread) per block; nb of them stay inside i64
  int lg = 0;
  while ((1 << lg) < lay.nb) lg++;
  return lay.base && lay.nb > 0 && lay.nb <= kMaxBlocks && lay.kspread <= kSpreadLimit &&
         lay.kspread <= 30 - lg;
}

static cudaError_t launch_gemm_main(const GemvPlan &pl, const uint8_t *pack,
                                    const GemmLayout &lay, size_t n_out, size_t n_in,
                                    size_t n_cols, const int8_t *codes, size_t ld,
                                    const uint8_t *exps, size_t ldb, const WorkView &w,
                                    Split sp, long long *out_q32, float *out_f32,
                                    unsigned long long *status, cudaStream_t stream);

cudaError_t launch_gemm_q8_0(const GemvPlan &pl, const uint8_t *pack, const GemmLayout &lay,
                             size_t n_out, size_t n_in, size_t n_cols, const int8_t *codes,
                             size_t ld, const uint8_t *exps, size_t ldb, const void *descs,
                             void *work, long long *out_q32, float *out_f32,
                             unsigned long long *status, int sm_count, cudaStream_t stream) {
  if (n_cols == 0 || n_out == 0) return cudaSuccess;
  const size_t tiles = gemm_tiles(n_out, n_cols);
  const Split ksplit = gemm_split(tiles, (int)(lay.kp / kSlab), sm_count);
  const WorkView w = work_view(work, n_cols, lay.nb, lay.kp, sm_count);
  PrepArgs pa;
  pa.codes = codes;
  pa.exps = exps;
  pa.descs = static_cast<const ActDesc *>(descs);
  pa.ld = ld;
  pa.ldb = ldb;
  pa.n_in = n_in;
  pa.kp = lay.kp;
  pa.nb = lay.nb;
  pa.n_cols = (int)n_cols;
  pa.w = w;
  pa.status = status;
  pa.max_shift = gemm_max_shift(lay);
  gemm_prep_kernel<<<(unsigned)cols_pad(n_cols), 256, 0, stream>>>(pa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_gemm_main(pl, pack, lay, n_out, n_in, n_cols, codes, ld, exps, ldb, w, ksplit,
                          out_q32, out_f32, status, stream);
}

// The GEMM launch after a prep: planes, routes and the checked-column list in `w`.
static cudaError_t launch_gemm_main(const GemvPlan &pl, const uint8_t *pack,
                                    const GemmLayout &lay, size_t n_out, size_t n_in,
                                    size_t n_cols, const int8_t *codes, size_t ld,
                                    const uint8_t *exps, size_t ldb, const WorkView &w,
                                    Split sp, long long *out_q32, float *out_f32,
                                    unsigned long long *status, cudaStream_t stream) {
  cudaError_t e;
  CUtensorMap map_x, map_s;
  if (!make_map(&map_x, w.bcodes, lay.kp, cols_pad(n_cols), lay.kp, kTileN) ||
      !make_table_map(&map_s, w.shift, cols_pad(n_cols), lay.kp / 32, kTileN))
    return cudaErrorInvalidValue;
  GemmArgs a;
  a.wmul = lay.wmul;
  a.kmin = lay.kmin;
  a.w = w;
  a.out_q32 = out_q32;
  a.out_f32 = out_f32;
  a.status = status;
  a.n_out = n_out;
  a.m_pad = lay.m_pad;
  a.n_cols = (int)n_cols;
  a.nb = lay.nb;
  a.kslabs = (int)(lay.kp / kSlab);
  a.m_tiles = (int)((n_out + kTileM - 1) / kTileM);
  a.tiles = a.m_tiles * (int)((n_cols + kTileN - 1) / kTileN);
  a.full = sp.full;
  a.ksplit = sp.ks;
  a.pieces = sp.pieces(a.tiles);
  a.part = w.part;
  a.cnt = w.cnt;
  a.geo = PackGeo{pack, pl.units, pl.L};
  a.codes = codes;
  a.exps = exps;
  a.ld = ld;
  a.ldb = ldb;
  a.n_in = n_in;
  const size_t smem = gemm_smem_bytes();
  e = cudaFuncSetAttribute(gemm_q8_0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
  if (e != cudaSuccess) return e;
  // programmatic dependent launch after the prep kernel (unless APX_PDL=0)
  static const bool pdl = [] {
    const char *v = std::getenv("APX_PDL");
    return !(v && v[0] == '0');
  }();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.pieces + kFallbackCtas));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_q8_0_kernel,
                            *reinterpret_cast<const CUtensorMap *>(lay.map), map_x,
                            *reinterpret_cast<const CUtensorMap *>(lay.map_m), map_s, a);
}

bool gemm_f32_ok(size_t n_in, const float *x, size_t ldx) {
  const size_t kp = (n_in + kSlab - 1) / kSlab * kSlab;
  return kp <= kQPrepMaxIn && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0;
}

cudaError_t launch_gemm_q8_0_f32(const GemvPlan &pl, const uint8_t *pack, const GemmLayout &lay,
                                 size_t n_out, size_t n_in, size_t n_cols, const float *x,
                                 size_t ldx, void *work, long long *out_q32, float *out_f32,
                                 unsigned long long *status, int sm_count, cudaStream_t stream) {
  if (n_cols == 0 || n_out == 0) return cudaSuccess;
  if (!gemm_f32_ok(n_in, x, ldx)) return cudaErrorInvalidValue;
  const size_t tiles = gemm_tiles(n_out, n_cols);
  const Split ksplit = gemm_split(tiles, (int)(lay.kp / kSlab), sm_count);
  const WorkView w = work_view(work, n_cols, lay.nb, lay.kp, sm_count);
  QPrepArgs qa;
  qa.x = x;
  qa.ldx = ldx;
  qa.n_in = n_in;
  qa.kp = lay.kp;
  qa.nb = lay.nb;
  qa.n_cols = (int)n_cols;
  qa.w = w;
  qa.status = status;
  qa.max_shift = gemm_max_shift(lay);
  const size_t smem = lay.kp + lay.kp / 32;
  gemm_quant_prep_kernel<<<(unsigned)cols_pad(n_cols), 256, smem, stream>>>(qa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_gemm_main(pl, pack, lay, n_out, n_in, n_cols, w.qcodes, lay.kp, w.qexps,
                          lay.kp / 32, w, ksplit, out_q32, out_f32, status, stream);
}

}  // namespace apx
