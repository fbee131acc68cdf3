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
#include "apx_quant.cuh"

namespace apx {

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
      uint32_t packed;
      int e;
      bool blk_ok;
      quant_quad(f4[u], packed, e, blk_ok);
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
