// apx_tc.cuh — tcgen05 / TMA / TMEM building blocks shared by the tensor-core GEMMs
// (apx_gemm.cu: the per-block fold; apx_lgemm.cu: the digit-plane GEMM), and the exact
// finish of one output from its pre-rounding accumulator.
//
// Only the forms this project runs: cta_group::1 MMAs of kind::i8 with both operands in shared
// memory, TMA tiled loads without multicast, 32x32b TMEM loads.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "apx_common.cuh"

namespace apx {

// ---- TMA (no multicast) ----------------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y,
                                            int z, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const void *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- MMA and its completion --------------------------------------------------------------------

// D (+)= A·B for one K = 32 step of kind::i8; `accumulate` 0 overwrites D.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  const uint32_t zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(zero), "r"(zero), "r"(zero),
      "r"(zero));
}

// Arrive on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// mbar_wait for waits that usually last microseconds (a whole tile's MMAs): a longer back-off
// leaves the issue slots to the producer and MMA threads sharing the sub-partitions.  Bounded
// like mbar_wait (about one second).
__device__ __forceinline__ bool mbar_wait_long(uint64_t *bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int it = 0; it < kWaitLimit; it++) {
    __nanosleep(256);
    if (mbar_try(bar, parity)) return true;
    if ((it & 15) == 15) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - t0 > 1000000000ull) return false;
    }
  }
  return false;
}

// ---- TMEM loads (32 lanes × n columns of 32-bit words per warp) --------------------------------

__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
}

// 8 columns into v[8h .. 8h + 7] (h a compile-time index after unrolling).
template <int N>
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t (&v)[N], int h) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(v[8 * h + 0]), "=r"(v[8 * h + 1]), "=r"(v[8 * h + 2]), "=r"(v[8 * h + 3]),
        "=r"(v[8 * h + 4]), "=r"(v[8 * h + 5]), "=r"(v[8 * h + 6]), "=r"(v[8 * h + 7])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- the exact finish of one output ----------------------------------------------------------
//
// v = round_shift_32(acc·2^s) (value.rs:10-12 on the 128-bit product) with the i64 range check
// of chart/mod.rs:1746-1753, and its f32 image F32::from_q32(v).  For s >= 32 the product has
// no fractional part: v = acc·2^(s−32) when that fits, and f32(v·2^-32) = RN(acc)·2^(s−64) (a
// power-of-two scaling commutes with the one rounding).  For s < 32, v = (acc + 2^(31−s)) >>
// (32−s), which always fits (|acc| < 2^62 is the caller's bound), and its f32 image is
// RN(v)·2^-32.  One conversion either way.
struct FinishOut {
  long long v;
  float f;
  bool fits;
};

// The general case, out of line: finishes unroll many outputs per thread, and an inlined copy
// of this per output would crowd the instruction cache.
static __device__ __noinline__ FinishOut finish_one(long long acc, unsigned s) {
  long long v;
  float f;
  bool fits = true;
  long long x;  // the integer whose rounding gives the f32 image
  int k;        // its power-of-two scale
  if (s >= 32) {
    const unsigned t = s - 32;
    v = (long long)((unsigned long long)acc << (t & 63));
    fits = t > 63 ? acc == 0 : (acc >> (63 - t)) == (acc >> 63);
    x = acc;
    k = (int)s - 64;
  } else {
    const unsigned t = 32 - s;
    v = (acc + (1ll << (t - 1))) >> t;
    x = v;
    k = -32;
  }
  f = __ll2float_rn(x) * __int_as_float((127 + k) << 23);
  return FinishOut{v, f, fits};
}

// finish_one for the common case 32 <= s < 64 with the range check on the accumulator's high
// word alone: acc·2^t fits i64 iff acc >> (63 − t) is 0 or -1, and for t < 32 that shift reads
// only the high 32 bits.
__device__ __forceinline__ bool finish_fast(long long acc, unsigned s, long long &v, float &f) {
  if (s >= 32 && s < 64) {
    const unsigned t = s - 32;
    const int hi = (int)(acc >> 32);
    v = (long long)((unsigned long long)acc << t);
    f = __ll2float_rn(acc) * __int_as_float((int)(s + 63) << 23);  // 2^(s − 64)
    return (hi >> (31 - t)) == (hi >> 31);
  }
  const FinishOut o = finish_one(acc, s);
  v = o.v;
  f = o.f;
  return o.fits;
}

// ---- host: the driver's tensor-map encoder -------------------------------------------------

static inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace apx
