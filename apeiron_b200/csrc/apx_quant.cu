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

// act_scale exponent, or -1 for a zero block, or 99 when the reference returns None.
__device__ __forceinline__ int act_scale_exp(unsigned long long absmax) {
  if (absmax == 0) return -1;
  unsigned long long need = absmax / 127ull + (absmax % 127ull != 0 ? 1ull : 0ull);
  if (need <= 1) return 0;
  int e = 64 - __clzll((long long)(need - 1));
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
  for (size_t b = warp; b < nb; b += nw) {
    size_t j = b * 32 + lane;
    long long v = 0;
    bool ok = true;
    if (j < n) {
      if (F32)
        ok = f32_to_q32(reinterpret_cast<const float *>(xin)[j], v);
      else
        v = reinterpret_cast<const long long *>(xin)[j];
    }
    if (__any_sync(0xFFFFFFFFu, !ok)) {
      if (lane == 0) atomicMax(&acc.status, (int)APX_ERR_QUANT_REFUSED);
      continue;
    }
    unsigned long long m = uabs64(v), mx = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
      mx = t > mx ? t : mx;
    }
    int e = act_scale_exp(mx);  // warp-uniform
    if (e == 99) {
      if (lane == 0) atomicMax(&acc.status, (int)APX_ERR_QUANT_REFUSED);
      continue;
    }
    int code = 0;
    if (e >= 0) {
      unsigned long long S = 1ull << e, q = m >> e, r = m & (S - 1);
      unsigned long long mag = q + (2 * r >= S ? 1ull : 0ull);
      code = v < 0 ? -(int)mag : (int)mag;
      bool bad = mag > 127 || !product_fits(code, e);
      if (__any_sync(0xFFFFFFFFu, bad)) {
        if (lane == 0) atomicMax(&acc.status, (int)APX_ERR_QUANT_REFUSED);
        continue;
      }
      if (lane == 0) {
        atomicMin(&acc.emin, e);
        atomicMax(&acc.emax, e);
        atomicAdd(&acc.nz, 1u);
      }
    }
    if (j < n) codes[j] = (int8_t)code;
    if (lane == 0) exps[b] = e < 0 ? (uint8_t)APX_EXP_ZERO : (uint8_t)e;
  }
  __syncthreads();
  desc_write(&acc, desc, n);
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
  const int threads = n <= 4096 ? 256 : 1024;
  quant_kernel<true><<<cols, threads, 0, stream>>>(x, n, ldx, codes, ld, exps, ldb,
                                                   reinterpret_cast<ActDesc *>(desc));
  return cudaGetLastError();
}

}  // namespace apx
