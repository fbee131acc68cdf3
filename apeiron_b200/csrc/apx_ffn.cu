// apx_ffn.cu — the FFN hidden activation on the device: h = SwiGLU(gate, up) under the engine's
// carrier, then quant_act(h) for the down projection (the SwiGLU and quantization stages of
// fused_ffn_task, src/engine/chart/ffn.rs:1577-1594), so the projections of a decode step chain
// on the GPU without a host round trip.
//
// Carriers (swiglu_one_carrier, ffn.rs:246-284):
//   F32 (the engine's default): g = from_q32(gate), u = from_q32(up) (RN(x)/2^32, fp.rs:176-178),
//       h = to_q32(silu(g)·u) with silu(x) = x / (1 + exp(-x)) in binary32 and exp the reference's
//       Cephes-style polynomial (mixer/f32_carrier.rs:262-375); every operation one IEEE binary32
//       rounding (the __f*_rn intrinsics: never contracted), Overflow where h leaves Q32.32;
//   Q32: h = round_shift_32(silu_fixed(gate)·up) (ops/silu.rs:53-100 on fixed_exp,
//       numeric/fixed_exp.rs:1-184), Overflow where h leaves i64.
// quant_act (chart/mod.rs:258-334) then runs per 32-lane block as in the column quantizer.
//
// One warp per 32-lane block, eight blocks per CTA; each CTA leaves its descriptor statistics in
// a small workspace and a one-CTA kernel merges them into the descriptor, so no state outlives
// the call.  The lowest refusing lane reaches the status word by atomicMin (lane in the row
// field), which is the reference's first-refusal order.
#include <algorithm>
#include <climits>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"
#include "apx_quant.cuh"
#include "apx_swiglu.cuh"

namespace apx {

constexpr int kFfnWarps = 8;

// ---- kernels -------------------------------------------------------------------------------

// Row shards: copies of a one-column call's codes, exponent bytes and descriptor at n other places
// (other GPUs' buffers), element 0 of the call at codes[i][0] / exps[i][0].
struct ShardDests {
  int n;
  int8_t *codes[7];
  uint8_t *exps[7];
  ActDesc *desc[7];
};

// Column c (blockIdx.y) of a multi-column call: gate, up and h at c·ldg, codes at c·ldc, exponent
// bytes at c·lde, the status word at status[2c], CTA statistics at part[c·gridDim.x + x].
struct FfnArgs {
  const long long *gate, *up;
  long long *h;  // or null
  int8_t *codes;
  uint8_t *exps;
  size_t n, ldg, ldc, lde;
  int carrier;
  int4 *part;                  // per CTA: emin, emax, status, nz
  unsigned long long *status;  // the first refusing lane
  ShardDests dst;              // one-column calls: where else the codes and exponents go
};

__global__ void __launch_bounds__(32 * kFfnWarps) swiglu_quant_kernel(FfnArgs a) {
  __shared__ int s_emin, s_emax, s_status;
  __shared__ unsigned s_nz;
  // a programmatic dependent of the projections that wrote gate and up: nothing is read or
  // written before their grids complete
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) {
    s_emin = 1 << 30;
    s_emax = -1;
    s_status = APX_OK;
    s_nz = 0;
  }
  __syncthreads();
  const size_t col = blockIdx.y;
  if (col) {  // this CTA's column of a multi-column call
    a.gate += col * a.ldg;
    a.up += col * a.ldg;
    if (a.h) a.h += col * a.ldg;
    a.codes += col * a.ldc;
    a.exps += col * a.lde;
    a.status += col * 2;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const size_t nb = (a.n + 31) / 32;
  const size_t b = (size_t)blockIdx.x * kFfnWarps + warp;
  if (b < nb) {  // warp-uniform
    const size_t j = b * 32 + lane;
    long long v = 0;
    bool ok = true;
    if (j < a.n) {
      const int rc = swiglu_dev(__ldg(a.gate + j), __ldg(a.up + j), a.carrier, v);
      if (rc) {
        ok = false;
        v = 0;
        atomicMin(a.status, pack_status(j, APX_ERR_SWIGLU_REFUSED, (unsigned)rc));
      }
      if (a.h) a.h[j] = v;
    }
    // quant_act of the block: absmax, S = 2^e, codes rounded half away from zero
    unsigned long long mx = uabs64(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
      mx = t > mx ? t : mx;
    }
    const int e = act_scale_exp(mx);  // warp-uniform
    // a refused SwiGLU lane leaves h undefined: the activation is refused as a whole
    int w_status = __any_sync(0xFFFFFFFFu, !ok) ? (int)APX_ERR_QUANT_REFUSED : (int)APX_OK;
    int code = 0;
    if (e == 99) {
      w_status = APX_ERR_QUANT_REFUSED;
    } else if (e >= 0) {
      const unsigned long long m = uabs64(v);
      const unsigned long long S = 1ull << e, q = m >> e, r = m & (S - 1);
      const unsigned long long mag = q + (2 * r >= S ? 1ull : 0ull);
      code = v < 0 ? -(int)mag : (int)mag;
      if (__any_sync(0xFFFFFFFFu, mag > 127 || !product_fits(code, e)))
        w_status = APX_ERR_QUANT_REFUSED;
    }
    const uint8_t eb = e < 0 || e == 99 ? (uint8_t)APX_EXP_ZERO : (uint8_t)e;
    if (j < a.n) a.codes[j] = (int8_t)code;
#pragma unroll 1
    for (int i = 0; i < a.dst.n; i++) {
      if (j < a.n) a.dst.codes[i][j] = (int8_t)code;
      if (lane == 0) a.dst.exps[i][b] = eb;
    }
    if (lane == 0) {
      a.exps[b] = eb;
      if (w_status != APX_OK) atomicMax(&s_status, w_status);
      if (e >= 0 && e != 99) {
        atomicMin(&s_emin, e);
        atomicMax(&s_emax, e);
        atomicAdd(&s_nz, 1u);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0)
    a.part[col * gridDim.x + blockIdx.x] = make_int4(s_emin, s_emax, s_status, (int)s_nz);
}

// The descriptor from the CTAs' statistics (one CTA per column).
__global__ void __launch_bounds__(256) ffn_desc_kernel(const int4 *part, int nparts, size_t n,
                                                       ActDesc *desc, ShardDests dst) {
  pdl_launch_dependents();
  pdl_wait();
  part += (size_t)blockIdx.x * nparts;
  desc += blockIdx.x;
  int emin = 1 << 30, emax = -1, status = APX_OK;
  unsigned nz = 0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    const int4 p = part[i];
    emin = min(emin, p.x);
    emax = max(emax, p.y);
    status = max(status, p.z);
    nz += (unsigned)p.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    emin = min(emin, __shfl_xor_sync(0xFFFFFFFFu, emin, o));
    emax = max(emax, __shfl_xor_sync(0xFFFFFFFFu, emax, o));
    status = max(status, __shfl_xor_sync(0xFFFFFFFFu, status, o));
    nz += __shfl_xor_sync(0xFFFFFFFFu, nz, o);
  }
  __shared__ int4 w[8];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) w[warp] = make_int4(emin, emax, status, (int)nz);
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x / 32); i++) {
      emin = min(emin, w[i].x);
      emax = max(emax, w[i].y);
      status = max(status, w[i].z);
      nz += (unsigned)w[i].w;
    }
    ActDesc r;
    r.status = status;
    r.emin = emax >= 0 ? emin : 0;
    r.emax = emax;
    r.n_in = (int32_t)n;
    r.nz = nz;
    r.pad[0] = 0;  // quant_act codes are never -128
    r.pad[1] = 0;
    r.pad[2] = 0;
    *desc = r;
    for (int i = 0; i < dst.n; i++) *dst.desc[i] = r;
  }
}

size_t swiglu_work_bytes(size_t n, size_t cols) {
  return ((n + 31) / 32 + kFfnWarps - 1) / kFfnWarps * sizeof(int4) * std::max<size_t>(cols, 1);
}

cudaError_t launch_swiglu_quant(const long long *gate, const long long *up, size_t n, int carrier,
                                long long *h, int8_t *codes, uint8_t *exps, void *desc,
                                unsigned long long *status, void *work, cudaStream_t stream,
                                const SwigluDests *dests) {
  return launch_swiglu_quant_cols(gate, up, n, 1, 0, carrier, h, codes, 0, exps, 0, desc, status,
                                  work, stream, dests);
}

cudaError_t launch_swiglu_quant_cols(const long long *gate, const long long *up, size_t n,
                                     size_t cols, size_t ldg, int carrier, long long *h,
                                     int8_t *codes, size_t ldc, uint8_t *exps, size_t lde,
                                     void *desc, unsigned long long *status, void *work,
                                     cudaStream_t stream, const SwigluDests *dests) {
  if (n == 0 || cols == 0) return cudaSuccess;
  const size_t nb = (n + 31) / 32;
  const unsigned grid = (unsigned)((nb + kFfnWarps - 1) / kFfnWarps);
  FfnArgs a;
  a.gate = gate;
  a.up = up;
  a.h = h;
  a.codes = codes;
  a.exps = exps;
  a.n = n;
  a.ldg = ldg;
  a.ldc = ldc;
  a.lde = lde;
  a.carrier = carrier;
  a.part = static_cast<int4 *>(work);
  a.status = status;
  a.dst = ShardDests{};
  if (dests) {
    if (cols != 1 || dests->n < 0 || dests->n > 7) return cudaErrorInvalidValue;
    a.dst.n = dests->n;
    for (int i = 0; i < dests->n; i++) {
      a.dst.codes[i] = dests->codes[i];
      a.dst.exps[i] = dests->exps[i];
      a.dst.desc[i] = static_cast<ActDesc *>(dests->desc[i]);
    }
  }
  // both as programmatic dependents: each launches while its predecessor finishes
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, (unsigned)cols);
  cfg.blockDim = dim3(32 * kFfnWarps);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_allowed() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, a);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3((unsigned)cols);
  cfg.blockDim = dim3(256);
  return cudaLaunchKernelEx(&cfg, ffn_desc_kernel, static_cast<const int4 *>(a.part), (int)grid,
                            n, static_cast<ActDesc *>(desc), a.dst);
}

}  // namespace apx
