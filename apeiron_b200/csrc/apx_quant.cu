// apx_quant.cu — device activation quantization and the per-call activation descriptor.
//
// quant_act (src/engine/chart/mod.rs:258-334): per 32-lane block the smallest power of two
// S = 2^e with 127·S >= absmax (act_scale, src/engine/kern/pow2.rs:22-39, e <= 62), codes
// sign(x)·floor((2|x| + S) / (2S)) (round to nearest, ties away from zero), and refusal
// exactly where QuantAct::dequantizes fails (chart/mod.rs:124-146).  f32 inputs first take
// f32_to_fixed (src/engine/num/f32_convert.rs:44-49 → F32::to_q32, src/engine/num/fp.rs:186).
//
// One CTA per activation vector: the vectors are at most a few tens of thousands of lanes,
// and the descriptor (min/max exponent, refusal) must be complete before the projection
// kernel that follows on the same stream reads it.
#include "apx_common.cuh"
#include "apx_kernels.h"

namespace apx {

__device__ __forceinline__ unsigned long long uabs64(long long v) {
  return v < 0 ? 0ull - (unsigned long long)v : (unsigned long long)v;
}

// act_scale exponent, or -1 for a zero block, or 99 when the reference returns None: the
// smallest e >= 0 with 127·2^e >= absmax (pow2.rs:22-39).  With bl the bit length of absmax
// and e0 = max(0, bl − 7), 127·2^(e0−1) < 2^(bl−1) <= absmax, so e is e0 or e0 + 1; 127·2^e0
// stays below 2^64 for every absmax <= 2^63.  No division.
__device__ __forceinline__ int act_scale_exp(unsigned long long absmax) {
  if (absmax == 0) return -1;
  const int bl = 64 - __clzll((long long)absmax);
  const int e0 = bl > 7 ? bl - 7 : 0;
  const int e = (127ull << e0) >= absmax ? e0 : e0 + 1;
  return e > 62 ? 99 : e;
}

// S·code fits i64 for S = 2^e (QuantAct::dequant's checked product).
__device__ __forceinline__ bool product_fits(int code, int e) {
  if (e <= 56) return true;  // 128·2^56 = 2^63: every int8 code fits except -128·2^56 = i64::MIN
  long long lim = 1ll << (63 - e);
  return code >= -lim && code <= lim - 1;
}

struct DescAcc {
  int emin, emax, status;
  unsigned nz, m128;
};

__device__ void desc_init(DescAcc *d) {
  if (threadIdx.x == 0) {
    d->emin = 1 << 30;
    d->emax = -1;
    d->status = APX_OK;
    d->nz = 0;
    d->m128 = 0;
  }
}

__device__ void desc_write(const DescAcc *d, ActDesc *out, size_t n) {
  if (threadIdx.x == 0) {
    ActDesc r;
    r.status = d->status;
    r.emin = d->emax >= 0 ? d->emin : 0;
    r.emax = d->emax;
    r.n_in = (int32_t)n;
    r.nz = d->nz;
    r.pad[0] = d->m128 ? 1u : 0u;
    r.pad[1] = 0;
    r.pad[2] = 0;
    *out = r;
  }
}

// Validate caller-supplied codes/exponents (the QuantAct invariant and its Q32.32 image).
__global__ void describe_kernel(const int8_t *codes, const uint8_t *exps, size_t n, size_t ld,
                                size_t ldb, ActDesc *desc) {
  __shared__ DescAcc acc;
  const int col = blockIdx.x;
  codes += (size_t)col * ld;
  exps += (size_t)col * ldb;
  desc_init(&acc);
  __syncthreads();
  const size_t nb = (n + 31) / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  for (size_t b = warp; b < nb; b += nw) {
    unsigned e = exps[b];
    if (e == APX_EXP_ZERO) continue;
    if (e > 62) {
      if (lane == 0) atomicMax(&acc.status, (int)APX_ERR_INVALID_ARGUMENT);
      continue;
    }
    size_t j = b * 32 + lane;
    int code = j < n ? codes[j] : 0;
    bool bad = !product_fits(code, (int)e);
    bool m128 = code == -128;
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicMax(&acc.status, (int)APX_ERR_FIXED_OVERFLOW);
    if (__any_sync(0xFFFFFFFFu, m128) && lane == 0) atomicOr(&acc.m128, 1u);
    if (lane == 0) {
      atomicMin(&acc.emin, (int)e);
      atomicMax(&acc.emax, (int)e);
      atomicAdd(&acc.nz, 1u);
    }
  }
  __syncthreads();
  // an invalid exponent byte outranks the overflow refusal: report it as such
  desc_write(&acc, desc + col, n);
}

// F32::to_q32 (src/engine/num/fp.rs:186-230): round(v·2^32), ties away from zero.
__device__ __forceinline__ bool f32_to_q32(float f, long long &out) {
  unsigned bits = __float_as_uint(f);
  unsigned e = (bits >> 23) & 0xFFu;
  if (e == 0xFFu) return false;
  unsigned frac = bits & 0x007FFFFFu;
  unsigned long long m = e == 0 ? frac : (frac | 0x00800000u);
  bool neg = (bits & 0x80000000u) != 0;
  unsigned ee = e == 0 ? 1 : e;
  unsigned long long mag;
  if (ee >= 118) {
    unsigned k = ee - 118;
    if (k > 40) return false;
    if (k >= 40 && m >= (1ull << 23)) {
      // m·2^k >= 2^63: the positive side refuses, the negative side only at exactly 2^63
      if (neg && m == (1ull << 23)) {
        out = (long long)(1ull << 63);
        return true;
      }
      return false;
    }
    mag = m << k;
  } else {
    unsigned sh = 118 - ee;
    mag = sh > 24 ? 0ull : (m + (1ull << (sh - 1))) >> sh;
  }
  const unsigned long long lim = 1ull << 63;
  if (neg) {
    if (mag > lim) return false;
    out = mag == lim ? (long long)lim : -(long long)mag;
    return true;
  }
  if (mag >= lim) return false;
  out = (long long)mag;
  return true;
}

// One CTA per activation vector: vector c reads x at c·ldx elements and writes its codes at
// c·ld, its exponent bytes at c·ldb and its descriptor at desc[c].
template <bool F32>
__global__ void quant_kernel(const void *xin, size_t n, size_t ldx, int8_t *codes, size_t ld,
                             uint8_t *exps, size_t ldb, ActDesc *desc) {
  __shared__ DescAcc acc;
  {
    const size_t c = blockIdx.x;
    xin = F32 ? (const void *)(reinterpret_cast<const float *>(xin) + c * ldx)
              : (const void *)(reinterpret_cast<const long long *>(xin) + c * ldx);
    codes += c * ld;
    exps += c * ldb;
    desc += c;
  }
  desc_init(&acc);
  __syncthreads();
  const size_t nb = (n + 31) / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  // per-warp descriptor statistics, merged once at the end
  int w_emin = 1 << 30, w_emax = -1, w_status = APX_OK;
  unsigned w_nz = 0;
  for (size_t b = warp; b < nb; b += nw) {
    size_t j = b * 32 + lane;
    long long v = 0;
    bool ok = true;
    unsigned long long mx;
    if (F32) {
      const float f = j < n ? reinterpret_cast<const float *>(xin)[j] : 0.0f;
      ok = f32_to_q32(f, v);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        w_status = max(w_status, (int)APX_ERR_QUANT_REFUSED);
        continue;
      }
      // |f| orders like round(|f|·2^32): the block absmax from the f32 bit patterns
      const unsigned amax = __reduce_max_sync(0xFFFFFFFFu, __float_as_uint(f) & 0x7FFFFFFFu);
      long long vm;
      // every lane converted, so the only |f| without a positive image is 2^31 (a lane
      // holding -2^31 = i64::MIN in Q32.32): its magnitude is 2^63
      mx = f32_to_q32(__uint_as_float(amax), vm) ? (unsigned long long)vm : 1ull << 63;
    } else {
      if (j < n) v = reinterpret_cast<const long long *>(xin)[j];
      mx = uabs64(v);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        mx = t > mx ? t : mx;
      }
    }
    const unsigned long long m = uabs64(v);
    int e = act_scale_exp(mx);  // warp-uniform
    if (e == 99) {
      w_status = max(w_status, (int)APX_ERR_QUANT_REFUSED);
      continue;
    }
    int code = 0;
    if (e >= 0) {
      unsigned long long S = 1ull << e, q = m >> e, r = m & (S - 1);
      unsigned long long mag = q + (2 * r >= S ? 1ull : 0ull);
      code = v < 0 ? -(int)mag : (int)mag;
      bool bad = mag > 127 || !product_fits(code, e);
      if (__any_sync(0xFFFFFFFFu, bad)) {
        w_status = max(w_status, (int)APX_ERR_QUANT_REFUSED);
        continue;
      }
      w_emin = min(w_emin, e);
      w_emax = max(w_emax, e);
      w_nz++;
    }
    if (j < n) codes[j] = (int8_t)code;
    if (lane == 0) exps[b] = e < 0 ? (uint8_t)APX_EXP_ZERO : (uint8_t)e;
  }
  if (lane == 0) {
    if (w_status != APX_OK) atomicMax(&acc.status, w_status);
    if (w_emax >= 0) {
      atomicMin(&acc.emin, w_emin);
      atomicMax(&acc.emax, w_emax);
      atomicAdd(&acc.nz, w_nz);
    }
  }
  __syncthreads();
  desc_write(&acc, desc, n);
}

// Round-half-up right shift of a value below 2^25 (0 for shifts past its bit length).
__device__ __forceinline__ unsigned rshift_round(unsigned x, unsigned s) {
  return s == 0 ? x : s > 25 ? 0u : (x + (1u << (s - 1))) >> s;
}

// Largest |f| bit pattern the 32-bit route takes: 127·2^24.  Below it every lane converts,
// act_scale gives e <= 56 and every code times 2^e fits i64, so nothing refuses.
constexpr unsigned kFastAbsMax = 0x4EFE0000u;

// act_scale exponent of a block whose largest |f| has bit pattern A <= kFastAbsMax, from the
// f32 fields: with M the 24-bit significand and E the biased exponent, round(A·2^32) is
// M·2^(E−118) for E >= 118 (bit length E − 94, so e = E − 101 or one more when M > 127·2^17),
// and below that a value under 2^25 formed by one rounding shift.
__device__ __forceinline__ int fast_scale_exp(unsigned A) {
  const unsigned E = A >> 23, M = (A & 0x7FFFFFu) | (E ? 0x800000u : 0u);
  if (E >= 118) return (int)E - 101 + (M > 0xFE0000u ? 1 : 0);
  const unsigned vm = rshift_round(M, 118 - (E ? E : 1));
  if (vm == 0) return -1;
  const int bl = 32 - __clz((int)vm);
  const int e0 = bl > 7 ? bl - 7 : 0;
  return (127u << e0) >= vm ? e0 : e0 + 1;
}

// Code of one lane (f32 bits) under block exponent e >= 0: round(|f|·2^32) then round by 2^e,
// ties away from zero both times.  Where round(|f|·2^32) is exact (E >= 118) the two
// roundings are one shift of the significand.
__device__ __forceinline__ int fast_code(unsigned bits, int e) {
  const unsigned b = bits & 0x7FFFFFFFu, E = b >> 23, M = (b & 0x7FFFFFu) | (E ? 0x800000u : 0u);
  const unsigned mag = E >= 118 ? rshift_round(M, (unsigned)e + 118 - E)
                                : rshift_round(rshift_round(M, 118 - (E ? E : 1)), (unsigned)e);
  return (bits >> 31) ? -(int)mag : (int)mag;
}

// f32 vectors, bandwidth-shaped: a warp takes 128 lanes (4 blocks) per chunk, each thread 4
// consecutive lanes (one 16-byte load, one 4-byte store of codes), with kQuantChunks chunks'
// loads in flight per thread.  The block absmax reduces over its 8 threads on the f32 bit
// patterns (|f| orders like round(|f|·2^32)).  Blocks whose absmax is at most kFastAbsMax take
// 32-bit arithmetic on the f32 fields; a warp holding any other block takes the Q32.32 route
// of quant_kernel for all its lanes.  Same codes, exponents and descriptor as
// quant_kernel<true>; vector c at x + c·ldx, ldx a multiple of 4.
constexpr int kQuantChunks = 4;

__global__ void __launch_bounds__(256) quant_f32_vec_kernel(const float *x, size_t n, size_t ldx,
                                                           int8_t *codes, size_t ld,
                                                           uint8_t *exps, size_t ldb,
                                                           ActDesc *desc) {
  __shared__ DescAcc acc;
  const size_t c = blockIdx.x;
  x += c * ldx;
  codes += c * ld;
  exps += c * ldb;
  desc_init(&acc);
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  int w_emin = 1 << 30, w_emax = -1, w_status = APX_OK;
  unsigned w_nz = 0;
  const size_t chunks = (n + 127) / 128;
  for (size_t round = 0; round * nw * kQuantChunks < chunks; round++) {
    float4 f4[kQuantChunks];
#pragma unroll
    for (int u = 0; u < kQuantChunks; u++) {
      const size_t j = ((round * kQuantChunks + u) * nw + warp) * 128 + 4 * lane;
      f4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j + 4 <= n) {
        f4[u] = __ldg(reinterpret_cast<const float4 *>(x + j));
      } else if (j < n) {
        f4[u].x = x[j];
        if (j + 1 < n) f4[u].y = x[j + 1];
        if (j + 2 < n) f4[u].z = x[j + 2];
      }
    }
#pragma unroll
    for (int u = 0; u < kQuantChunks; u++) {
      const size_t cbase = ((round * kQuantChunks + u) * nw + warp) * 128;
      if (cbase >= n) break;  // warp-uniform
      const size_t j = cbase + 4 * lane;
      const unsigned bits[4] = {__float_as_uint(f4[u].x), __float_as_uint(f4[u].y),
                                __float_as_uint(f4[u].z), __float_as_uint(f4[u].w)};
      unsigned amax = 0;
#pragma unroll
      for (int k = 0; k < 4; k++) amax = max(amax, bits[k] & 0x7FFFFFFFu);
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
      int e = -1;
      uint32_t packed = 0;
      bool blk_ok = true;
      if (__all_sync(0xFFFFFFFFu, amax <= kFastAbsMax)) {
        e = fast_scale_exp(amax);
        if (e >= 0) {
#pragma unroll
          for (int k = 0; k < 4; k++)
            packed |= ((uint32_t)(uint8_t)(int8_t)fast_code(bits[k], e)) << (8 * k);
        }
      } else {
        // Q32.32 route (f32_to_q32, act_scale, checked product) for every lane of the warp
        long long v[4];
        bool ok = true;
#pragma unroll
        for (int k = 0; k < 4; k++) ok &= f32_to_q32(__uint_as_float(bits[k]), v[k]);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) ok &= __shfl_xor_sync(0xFFFFFFFFu, (int)ok, o) != 0;
        blk_ok = ok;
        if (blk_ok) {
          long long vm;
          const unsigned long long mx =
              f32_to_q32(__uint_as_float(amax), vm) ? (unsigned long long)vm : 1ull << 63;
          e = act_scale_exp(mx);
          if (e == 99) blk_ok = false;
        }
        bool bad = false;
        if (blk_ok && e >= 0) {
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const unsigned long long m = uabs64(v[k]);
            const unsigned long long S = 1ull << e, q = m >> e, r = m & (S - 1);
            const unsigned long long mag = q + (2 * r >= S ? 1ull : 0ull);
            const int code = v[k] < 0 ? -(int)mag : (int)mag;
            bad |= mag > 127 || !product_fits(code, e);
            packed |= ((uint32_t)(uint8_t)(int8_t)code) << (8 * k);
          }
        }
        // every lane takes part in the group reduction (the branch above is group-dependent)
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) bad |= __shfl_xor_sync(0xFFFFFFFFu, (int)bad, o) != 0;
        if (bad) blk_ok = false;
      }
      const bool leader = (lane & 7) == 0 && j < n;
      if (!blk_ok) {
        if (leader) w_status = max(w_status, (int)APX_ERR_QUANT_REFUSED);
        continue;
      }
      if (j + 4 <= n) {
        *reinterpret_cast<uint32_t *>(codes + j) = packed;
      } else {
        for (int k = 0; k < 4; k++)
          if (j + k < n) codes[j + k] = (int8_t)(packed >> (8 * k));
      }
      if (leader) {
        exps[j / 32] = e < 0 ? (uint8_t)APX_EXP_ZERO : (uint8_t)e;
        if (e >= 0) {
          w_emin = min(w_emin, e);
          w_emax = max(w_emax, e);
          w_nz++;
        }
      }
    }
  }
  // merge the leaders' statistics
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    w_emin = min(w_emin, __shfl_xor_sync(0xFFFFFFFFu, w_emin, o));
    w_emax = max(w_emax, __shfl_xor_sync(0xFFFFFFFFu, w_emax, o));
    w_status = max(w_status, __shfl_xor_sync(0xFFFFFFFFu, w_status, o));
    w_nz += __shfl_xor_sync(0xFFFFFFFFu, w_nz, o);
  }
  if (lane == 0) {
    if (w_status != APX_OK) atomicMax(&acc.status, w_status);
    if (w_emax >= 0) {
      atomicMin(&acc.emin, w_emin);
      atomicMax(&acc.emax, w_emax);
      atomicAdd(&acc.nz, w_nz);
    }
  }
  __syncthreads();
  desc_write(&acc, desc + c, n);
}

cudaError_t launch_describe(const int8_t *codes, const uint8_t *exps, size_t n, int cols,
                            size_t ld, size_t ldb, void *desc, cudaStream_t stream) {
  if (cols <= 0) return cudaSuccess;
  describe_kernel<<<cols, 512, 0, stream>>>(codes, exps, n, ld, ldb,
                                            reinterpret_cast<ActDesc *>(desc));
  return cudaGetLastError();
}

cudaError_t launch_quant_q32(const long long *x, size_t n, int8_t *codes, uint8_t *exps,
                             void *desc, cudaStream_t stream) {
  quant_kernel<false><<<1, 1024, 0, stream>>>(x, n, 0, codes, 0, exps, 0,
                                              reinterpret_cast<ActDesc *>(desc));
  return cudaGetLastError();
}

cudaError_t launch_quant_f32(const float *x, size_t n, int8_t *codes, uint8_t *exps, void *desc,
                             cudaStream_t stream) {
  quant_kernel<true><<<1, 1024, 0, stream>>>(x, n, 0, codes, 0, exps, 0,
                                             reinterpret_cast<ActDesc *>(desc));
  return cudaGetLastError();
}

cudaError_t launch_quant_f32_cols(const float *x, size_t n, size_t ldx, int cols, int8_t *codes,
                                  size_t ld, uint8_t *exps, size_t ldb, void *desc,
                                  cudaStream_t stream) {
  if (cols <= 0) return cudaSuccess;
  // 16-byte loads need 16-byte aligned vectors; the codes, 4-byte aligned rows
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(codes) & 3) == 0 && ld % 4 == 0;
  if (vec) {
    quant_f32_vec_kernel<<<cols, 256, 0, stream>>>(x, n, ldx, codes, ld, exps, ldb,
                                                   reinterpret_cast<ActDesc *>(desc));
  } else {
    const int threads = n <= 4096 ? 256 : 1024;
    quant_kernel<true><<<cols, threads, 0, stream>>>(x, n, ldx, codes, ld, exps, ldb,
                                                     reinterpret_cast<ActDesc *>(desc));
  }
  return cudaGetLastError();
}

}  // namespace apx
