// apx_common.cuh — device helpers shared by the projection kernels.
//
// Exact integer arithmetic only: every kernel accumulates the reference's
// `Σ_b S_b·(w_scale·D − w_min·Σxq)` (src/engine/chart/mod.rs:497-514) as a two's-complement
// 128-bit integer held in two 64-bit words, and finishes with the reference's single
// `round_shift_32` (src/engine/num/value.rs:10-12).
#pragma once

#include <cstddef>
#include <cstdint>

#include "../../include/apeiron_cuda.h"

namespace apx {

constexpr int kLanes = 32;       // rows per tile: one row per lane
constexpr int kActQK = 32;       // activation block (chart/mod.rs:63)
constexpr int kQK_K = 256;       // k-quant super-block (format/quant.rs:18)
constexpr uint32_t kQ8_0 = APX_GGML_TYPE_Q8_0;
constexpr uint32_t kQ4_K = APX_GGML_TYPE_Q4_K;
constexpr uint32_t kQ6_K = APX_GGML_TYPE_Q6_K;

// Repacked unit sizes (bytes per 32-row tile per unit): the same bytes as 32 rows of the
// GGUF payload for that unit, regrouped so lane l's 16-byte chunk c sits at (c*32+l)*16.
constexpr int kQ8Blocks = 4;                       // Q8_0 blocks per unit
constexpr int kUnitQ8_0 = 32 * kQ8Blocks * 34;     // 4352: codes 4096 + f16 scales 256
constexpr int kUnitQ4_K = 32 * 144;                // 4608: qs 4096 + headers 512
constexpr int kUnitQ6_K = 32 * 210;                // 6720: ql|qh 6144 + scales 512 + d 64

// Kinds in the refusal word.
constexpr unsigned kKindOutputOverflow = APX_ERR_OUTPUT_OVERFLOW;
constexpr unsigned kKindAccOverflow = APX_ERR_ACCUMULATOR_OVERFLOW;

// Device view of apx_act_desc (include/apeiron_cuda.h): written by the quant / describe
// kernels or uploaded by the host, read by every projection kernel of the call.
struct ActDesc {
  int32_t status;   // APX_OK, APX_ERR_FIXED_OVERFLOW (a product S·xq leaves i64) or
                    // APX_ERR_QUANT_REFUSED (quant_act returned None)
  int32_t emin;     // smallest exponent over non-zero scales (0 when all are zero)
  int32_t emax;     // largest exponent over non-zero scales (-1 when all are zero)
  int32_t n_in;     // activation length the descriptor was built for
  uint32_t nz;      // number of non-zero scales
  uint32_t pad[3];
};
static_assert(sizeof(ActDesc) == sizeof(apx_act_desc), "descriptor layout");

// ---- 128-bit two's-complement accumulator ------------------------------------------

struct Acc128 {
  unsigned long long lo, hi;
};

__device__ __forceinline__ void acc_zero(Acc128 &a) { a.lo = 0ull; a.hi = 0ull; }

__device__ __forceinline__ void acc_add(Acc128 &a, unsigned long long lo, unsigned long long hi) {
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;"
      : "+l"(a.lo), "+l"(a.hi)
      : "l"(lo), "l"(hi));
}

__device__ __forceinline__ void acc_add(Acc128 &a, const Acc128 &b) { acc_add(a, b.lo, b.hi); }

__device__ __forceinline__ void acc_sub(Acc128 &a, unsigned long long lo, unsigned long long hi) {
  asm("sub.cc.u64 %0, %0, %2;\n\tsubc.u64 %1, %1, %3;"
      : "+l"(a.lo), "+l"(a.hi)
      : "l"(lo), "l"(hi));
}

// v * 2^s as a 128-bit value, 0 <= s < 128.
__device__ __forceinline__ void shl128(long long v, unsigned s, unsigned long long &lo,
                                       unsigned long long &hi) {
  if (s < 64) {
    lo = (unsigned long long)v << s;
    hi = (unsigned long long)((v >> 1) >> (63 - s));
  } else {
    lo = 0ull;
    hi = (unsigned long long)v << (s - 64);
  }
}

// a += v * 2^s
__device__ __forceinline__ void acc_add_shl(Acc128 &a, long long v, unsigned s) {
  unsigned long long lo, hi;
  shl128(v, s, lo, hi);
  acc_add(a, lo, hi);
}

// a -= v * 2^s
__device__ __forceinline__ void acc_sub_shl(Acc128 &a, long long v, unsigned s) {
  unsigned long long lo, hi;
  shl128(v, s, lo, hi);
  acc_sub(a, lo, hi);
}

// round_shift_32 (src/engine/num/value.rs:10-12) and the i64 range check of round_to_i64
// (src/engine/chart/mod.rs:1746-1753).  Returns false when the result leaves i64.
__device__ __forceinline__ bool acc_round_to_i64(const Acc128 &a, long long &out) {
  // v = q*2^32 + r; result = q + [r >= 2^31]; q = v >> 32 (arithmetic, 96 bits).
  unsigned long long qlo = (a.lo >> 32) | (a.hi << 32);
  long long qhi = (long long)a.hi >> 32;  // sign-extended top 32 bits of q
  unsigned long long r = a.lo & 0xFFFFFFFFull;
  unsigned long long inc = r >= 0x80000000ull ? 1ull : 0ull;
  unsigned long long lo = qlo + inc;
  long long hi = qhi + (lo < qlo ? 1 : 0);
  // fits i64 iff hi equals the sign extension of lo
  if (hi != ((long long)lo >> 63)) return false;
  out = (long long)lo;
  return true;
}

// ---- f16 scale split (src/engine/kern/pow2.rs:52-64) ---------------------------------
// finite f16 h = m * 2^k in Q32.32 with |m| <= 2047, k in [8, 37].  A non-finite word
// (exponent 31) decodes to m = 0: its row is refused from the upload-time scan.
__device__ __forceinline__ void f16_split(unsigned h, int &m, unsigned &k) {
  unsigned e = (h >> 10) & 31u;
  int f = (int)(h & 1023u);
  int mm = e == 0 ? f : (e == 31 ? 0 : f + 1024);
  k = e == 0 ? 8u : e + 7u;
  m = (h & 0x8000u) ? -mm : mm;
}

__device__ __forceinline__ unsigned long long pack_status(unsigned long long row, unsigned kind,
                                                          unsigned bits) {
  return (row << 24) | ((unsigned long long)kind << 16) | (bits & 0xFFFFu);
}

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// unsigned bytes of a times signed bytes of b
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Streaming 16-byte load of weight bytes: read once per call, kept out of L1.
__device__ __forceinline__ uint4 ld_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ld_stream8(const void *p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

// ---- TMA bulk copies into shared memory, completion on an mbarrier --------------------------
// One-dimensional bulk copies (cp.async.bulk, no tensor map, no multicast): 16-byte aligned
// addresses, sizes a multiple of 16.  Waits are bounded: a wait that gives up reports
// APX_ERR_DEVICE_TIMEOUT through the call's refusal word instead of spinning forever.

constexpr int kWaitLimit = 1 << 22;  // try_wait rounds before a wait gives up

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Wait for phase `parity` of the barrier; false if the bounded wait gave up (after
// kWaitLimit polls or about one second of %globaltimer, whichever comes first).  A poll
// that finds the phase open backs off with a short sleep, so that waiting warps leave the
// issue slots to the warps they wait for (a producer or an MMA thread sharing the same
// SM sub-partition).
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int it = 0; it < kWaitLimit; it++) {
    __nanosleep(32);
    if (mbar_try(bar, parity)) return true;
    if ((it & 63) == 63) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - t0 > 1000000000ull) return false;
    }
  }
  return false;
}

// 16-byte asynchronous copy from global into shared memory (no register staging); complete after
// cp_async_wait_all in the issuing thread (and __syncwarp for the warp's other lanes).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// A release/acquire fence at GPU scope: with a relaxed atomic after it (writer) or before it
// (reader) it orders the writer's earlier stores before the reader's later loads, which is all
// the hand-offs through arrival counters need.  Lighter than __threadfence (sequentially
// consistent).
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// ---- thread-block clusters ------------------------------------------------------------------
// The CTAs of a cluster are co-scheduled, and each can store into the others' shared memory
// (distributed shared memory).  barrier.cluster completes when every non-exited thread of the
// cluster has arrived: a hardware barrier like __syncthreads, not a poll.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The address of `p` (in this CTA's shared memory) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(const void *p, unsigned rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_acc(uint32_t addr, unsigned long long lo,
                                               unsigned long long hi) {
  asm volatile("st.shared::cluster.v2.u64 [%0], {%1, %2};" ::"r"(addr), "l"(lo), "l"(hi)
               : "memory");
}

}  // namespace apx
