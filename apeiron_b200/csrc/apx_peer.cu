// apx_peer.cu — row shards' outputs between the GPUs of one node over NVLink peer stores.
//
// A row-sharded projection leaves each rank with its own rows; every rank needs the whole
// vector.  apx_matvec_gather_async runs the projection with its finish storing every output
// row into this rank's slice of every rank's gather buffer (mapped through CUDA IPC), so the
// transfer is spread over all SMs and overlaps the projection's tail.  The publication kernel
// that follows (one warp; it starts once those grids have completed) writes this
// rank's refusal keys into every buffer and releases this rank's epoch flag there, then waits,
// bounded in time, until every rank's flag has reached the epoch in its own buffer and reduces
// the keys to the first refusal in whole-tensor row order (src/engine/chart/ffn.rs:659-661).
//
// The epoch is a counter in each rank's own buffer, read at the start of the publication and
// advanced at its end, so a replayed CUDA graph publishes fresh epochs.  No remote atomics, no
// multicast: the only cross-GPU traffic is stores and the flag loads of the waiting thread.
// The wait gives up after gd.timeout_us and reports APX_ERR_DEVICE_TIMEOUT in the merged word.
#include <cuda_runtime.h>

#include <cstring>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"

namespace apx {
int context_device(const apx_ctx *ctx);
bool tensor_launch_info(apx_ctx *ctx, uint64_t handle, uint32_t *type, const uint8_t **pack,
                        void **scratch, size_t *n_out, size_t *n_in, GemvPlan *plan,
                        int *device);

namespace {

constexpr long long kNoKey = 0x7FFFFFFFFFFFFFFFll;  // "no refusal" sorts after every row
constexpr unsigned kRowShift = 24;

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ long long ld_relaxed_sys(const long long *p) {
  long long v;
  asm volatile("ld.relaxed.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(32) gather_publish_kernel(const __grid_constant__
                                                            apx_gather_desc g) {
  pdl_launch_dependents();
  pdl_wait();  // the projections that stored this rank's rows everywhere are done
  uint8_t *own = static_cast<uint8_t *>(g.peer[g.rank]);
  unsigned long long *ctr = reinterpret_cast<unsigned long long *>(own + g.ctr_off);
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long *>(ctr) + 1;
  const int q = threadIdx.x;  // thread q: rank q's buffer
  if (q < g.world) {
    uint8_t *dst = static_cast<uint8_t *>(g.peer[q]);
    for (int j = 0; j < g.nproj; j++) {  // this rank's refusal keys
      const unsigned long long w = g.status[j]->first;
      long long key =
          w == ~0ull ? kNoKey : (long long)(w + ((unsigned long long)g.row0[j] << kRowShift));
      key = min(key, g.nf_key[j]);
      reinterpret_cast<long long *>(dst + g.key_off)[g.rank * g.nproj + j] = key;
    }
    // the rows the projections stored (their grids completed before this one passed its
    // wait: their stores happen before it) and these keys precede the flag: the fence and
    // the release are cumulative
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned long long *>(dst + g.flag_off) + g.rank, epoch);
  }
  __syncwarp();  // every thread has read the epoch and the refusal words
  if (q != 0) return;

  // every rank's flag in this buffer (bounded wait), then the first refusal over the ranks
  const unsigned long long *flags = reinterpret_cast<const unsigned long long *>(own + g.flag_off);
  const unsigned long long t0 = now_ns(), limit = (unsigned long long)g.timeout_us * 1000ull;
  bool ok = true;
  // One thread of one warp polls: short sleeps (at most 64 ns) keep the hand-off's latency,
  // which every step of a sharded chain pays twice, close to the last flag's arrival.
  for (int r = 0; r < g.world && ok; r++) {
    unsigned ns = 16;
    while (ld_acquire_sys(flags + r) < epoch) {
      if (now_ns() - t0 > limit) {
        ok = false;
        break;
      }
      __nanosleep(ns);
      if (ns < 64) ns *= 2;
    }
  }
  const long long *keys = reinterpret_cast<const long long *>(own + g.key_off);
  for (int j = 0; j < g.nproj; j++) {
    long long m = kNoKey;
    for (int r = 0; ok && r < g.world; r++) m = min(m, ld_relaxed_sys(keys + r * g.nproj + j));
    g.out_status[j]->first = !ok ? pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0)
                                 : (m == kNoKey ? ~0ull : (unsigned long long)m);
    g.out_status[j]->spare = 0;
    g.status[j]->first = ~0ull;  // ready for the next projection into it
  }
  if (g.desc_off) {  // the ranks' slice descriptors of a sharded activation, merged
    const ActDesc *sl = reinterpret_cast<const ActDesc *>(own + g.desc_off);
    int status = APX_OK, emin = 1 << 30, emax = -1, n = 0;
    unsigned nz = 0;
    for (int r = 0; r < g.world; r++) {
      const ActDesc d = sl[r];  // stored before rank r's flag, read after its acquire
      status = max(status, d.status);
      if (d.emax >= 0) {
        emin = min(emin, d.emin);
        emax = max(emax, d.emax);
      }
      nz += d.nz;
      n += d.n_in;
    }
    ActDesc m;
    m.status = ok ? status : (int)APX_ERR_DEVICE_TIMEOUT;
    m.emin = emax >= 0 ? emin : 0;
    m.emax = emax;
    m.n_in = n;
    m.nz = nz;
    m.pad[0] = m.pad[1] = m.pad[2] = 0;  // quant_act codes are never -128
    *reinterpret_cast<ActDesc *>(own + g.merged_off) = m;
  }
  *reinterpret_cast<volatile unsigned long long *>(ctr) = epoch;
}

int fail(apx_err *err, int code, cudaError_t e = cudaSuccess) {
  if (err) {
    std::memset(err, 0, sizeof(*err));
    err->code = code;
    err->cuda_error = (int32_t)e;
  }
  return code;
}

}  // namespace
}  // namespace apx

using apx::fail;

extern "C" {

APX_API int apx_peer_alloc(apx_ctx *ctx, size_t bytes, void **d_ptr,
                           unsigned char handle[APX_PEER_HANDLE_BYTES], apx_err *err) {
  if (!ctx || !d_ptr || !handle || !bytes) return fail(err, APX_ERR_INVALID_ARGUMENT);
  static_assert(sizeof(cudaIpcMemHandle_t) == APX_PEER_HANDLE_BYTES, "IPC handle size");
  cudaError_t e = cudaSetDevice(apx::context_device(ctx));
  void *p = nullptr;
  if (e == cudaSuccess) e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return fail(err, APX_ERR_CUDA, e);
  }
  std::memcpy(handle, &h, sizeof(h));
  *d_ptr = p;
  return fail(err, APX_OK);
}

APX_API int apx_peer_open(apx_ctx *ctx, const unsigned char handle[APX_PEER_HANDLE_BYTES],
                          void **d_ptr, apx_err *err) {
  if (!ctx || !d_ptr || !handle) return fail(err, APX_ERR_INVALID_ARGUMENT);
  cudaError_t e = cudaSetDevice(apx::context_device(ctx));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  if (e == cudaSuccess) e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(err, APX_ERR_CUDA, e);
  *d_ptr = p;
  return fail(err, APX_OK);
}

APX_API int apx_peer_close(apx_ctx *ctx, void *d_ptr, int opened) {
  if (!ctx || !d_ptr) return APX_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaSetDevice(apx::context_device(ctx));
  if (e == cudaSuccess) e = opened ? cudaIpcCloseMemHandle(d_ptr) : cudaFree(d_ptr);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

APX_API int apx_device_read(apx_ctx *ctx, const void *d_src, void *host_dst, size_t bytes,
                            apx_err *err) {
  if (!ctx || (bytes && (!d_src || !host_dst))) return fail(err, APX_ERR_INVALID_ARGUMENT);
  cudaError_t e = cudaSetDevice(apx::context_device(ctx));
  if (e == cudaSuccess && bytes) e = cudaMemcpy(host_dst, d_src, bytes, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? fail(err, APX_OK) : fail(err, APX_ERR_CUDA, e);
}

APX_API int apx_device_write(apx_ctx *ctx, void *d_dst, const void *host_src, size_t bytes,
                             apx_err *err) {
  if (!ctx || (bytes && (!d_dst || !host_src))) return fail(err, APX_ERR_INVALID_ARGUMENT);
  cudaError_t e = cudaSetDevice(apx::context_device(ctx));
  if (e == cudaSuccess && bytes) e = cudaMemcpy(d_dst, host_src, bytes, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? fail(err, APX_OK) : fail(err, APX_ERR_CUDA, e);
}

namespace {
// [off, off + len) inside a buffer of `bytes` (no wrap-around).
bool inside(size_t off, size_t len, size_t bytes) { return off <= bytes && len <= bytes - off; }
// len = a·b without overflow.
bool mul_ok(size_t a, size_t b, size_t &len) { return !__builtin_mul_overflow(a, b, &len); }
}  // namespace

APX_API int apx_matvec_gather_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                                    const int8_t *d_codes, const uint8_t *d_exps,
                                    const apx_act_desc *d_desc, const apx_gather_desc *gd,
                                    int j, void *stream) {
  if (!ctx || !gd || gd->world < 1 || gd->world > APX_MAX_PEERS || gd->rank < 0 ||
      gd->rank >= gd->world || j < 0 || j >= gd->nproj || gd->nproj > APX_MAX_GATHER_PROJ ||
      !gd->status[j] || n_out != gd->rows[j] || (gd->out_off & 7))
    return APX_ERR_INVALID_ARGUMENT;
  {  // this projection's rows of the output area lie inside every rank's buffer
    size_t first, len;
    if (!mul_ok(gd->rows_off[j], 8, first) || !mul_ok(gd->rows[j], 8, len) ||
        !inside(gd->out_off, first, gd->bytes) || !inside(gd->out_off + first, len, gd->bytes))
      return APX_ERR_INVALID_ARGUMENT;
  }
  for (int r = 0; r < gd->world; r++)
    if (!gd->peer[r]) return APX_ERR_INVALID_ARGUMENT;
  uint32_t type;
  const uint8_t *pack;
  void *tscratch;
  size_t t_out, t_in;
  apx::GemvPlan plan;
  int device;
  if (!apx::tensor_launch_info(ctx, tensor, &type, &pack, &tscratch, &t_out, &t_in, &plan,
                               &device))
    return APX_ERR_INVALID_ARGUMENT;
  if (n_in != t_in || n_out != t_out) return APX_ERR_LAYOUT_MISMATCH;
  if (n_out == 0) return APX_OK;
  if (!d_codes || !d_exps || !d_desc) return APX_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(device) != cudaSuccess) return APX_ERR_CUDA;
  auto rows_in = [&](int r) {
    return reinterpret_cast<long long *>(static_cast<uint8_t *>(gd->peer[r]) + gd->out_off) +
           gd->rows_off[j];
  };
  apx::PeerRows pr{};
  for (int r = 0; r < gd->world; r++)
    if (r != gd->rank) pr.dst[pr.n++] = rows_in(r);
  const cudaError_t e =
      apx::launch_gemv(plan, type, pack, tscratch, n_out, n_in, d_codes, d_exps, d_desc,
                       rows_in(gd->rank), nullptr, &gd->status[j]->first,
                       static_cast<cudaStream_t>(stream), &pr);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

APX_API int apx_gather_publish_async(apx_ctx *ctx, const apx_gather_desc *gd, void *stream) {
  if (!ctx || !gd || gd->world < 1 || gd->world > APX_MAX_PEERS || gd->rank < 0 ||
      gd->rank >= gd->world || gd->nproj < 1 || gd->nproj > APX_MAX_GATHER_PROJ ||
      (gd->out_off & 15) || (gd->key_off & 7) || (gd->flag_off & 7) || (gd->ctr_off & 7))
    return APX_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < gd->world; r++)
    if (!gd->peer[r]) return APX_ERR_INVALID_ARGUMENT;
  for (int j = 0; j < gd->nproj; j++)
    if (!gd->status[j] || !gd->out_status[j]) return APX_ERR_INVALID_ARGUMENT;
  // the keys ([world][nproj] int64), the flags ([world] uint64) and this rank's epoch and
  // check-in count (2 uint64) lie inside every rank's buffer
  if ((gd->desc_off && (gd->desc_off % 16 || gd->merged_off % 16 ||
                        !inside(gd->desc_off, sizeof(apx_act_desc) * (size_t)gd->world, gd->bytes) ||
                        !inside(gd->merged_off, sizeof(apx_act_desc), gd->bytes))) ||
      !inside(gd->key_off, 8 * (size_t)gd->world * (size_t)gd->nproj, gd->bytes) ||
      !inside(gd->flag_off, 8 * (size_t)gd->world, gd->bytes) ||
      !inside(gd->ctr_off, 16, gd->bytes))
    return APX_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(apx::context_device(ctx)) != cudaSuccess) return APX_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, apx::gather_publish_kernel, *gd);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

}  // extern "C"
