// apx_peer.cu — row shards' outputs between the GPUs of one node over NVLink peer stores.
//
// A row-sharded projection leaves each rank with its own rows; every rank needs the whole
// vector.  The publication kernel below moves the rows with plain stores into the other ranks'
// gather buffers (mapped through CUDA IPC), so the transfer is one short kernel on each rank
// rather than a collective library call: one CTA per destination rank copies this rank's rows
// of each projection (16-byte stores), writes this rank's refusal keys, fences at system scope
// and releases this rank's epoch flag in the destination.  The CTA of this rank's own buffer
// then waits, bounded in time, until every rank's flag has reached the epoch and reduces the
// keys to the first refusal in whole-tensor row order (src/engine/chart/ffn.rs:659-661).
//
// The epoch is a counter in each rank's own buffer: every CTA reads it (plus one) at its start,
// the CTAs that write to other ranks check in on a second counter, and the CTA of the own
// buffer stores the new epoch only after every rank's flag and every local check-in have
// arrived.  So a replayed CUDA graph publishes fresh epochs, and no CTA of a launch can see
// the epoch its own launch has already advanced.
//
// No remote atomics, no multicast: the only cross-GPU traffic is stores and the flag loads of
// the waiting thread.  The wait gives up after gd.timeout_us and reports
// APX_ERR_DEVICE_TIMEOUT in the merged refusal word.
#include <cuda_runtime.h>

#include <cstring>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"

namespace apx {
int context_device(const apx_ctx *ctx);

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

__global__ void __launch_bounds__(512) gather_publish_kernel(const __grid_constant__
                                                             apx_gather_desc g) {
  pdl_launch_dependents();
  pdl_wait();  // the projections that wrote this rank's rows and refusal words are done
  const int q = blockIdx.x;  // destination rank
  uint8_t *dst = static_cast<uint8_t *>(g.peer[q]);
  uint8_t *src = static_cast<uint8_t *>(g.peer[g.rank]);
  unsigned long long *ctr = reinterpret_cast<unsigned long long *>(src + g.ctr_off);
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long *>(ctr) + 1;
  if (q != g.rank) {
    for (int j = 0; j < g.nproj; j++) {
      const size_t a = g.out_off + g.rows_off[j] * 8, n = g.rows[j] * 8;  // a: 16-aligned
      const uint4 *s4 = reinterpret_cast<const uint4 *>(src + a);
      uint4 *d4 = reinterpret_cast<uint4 *>(dst + a);
      const size_t n16 = n / 16;
      for (size_t i = threadIdx.x; i < n16; i += blockDim.x) d4[i] = s4[i];
      if ((n & 15) && threadIdx.x == 0)
        *reinterpret_cast<unsigned long long *>(dst + a + n16 * 16) =
            *reinterpret_cast<const unsigned long long *>(src + a + n16 * 16);
    }
  }
  if (threadIdx.x < (unsigned)g.nproj) {  // this rank's refusal keys
    const int j = threadIdx.x;
    const unsigned long long w = g.status[j]->first;
    long long key = w == ~0ull ? kNoKey
                               : (long long)(w + ((unsigned long long)g.row0[j] << kRowShift));
    key = min(key, g.nf_key[j]);
    reinterpret_cast<long long *>(dst + g.key_off)[g.rank * g.nproj + j] = key;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned long long *>(dst + g.flag_off) + g.rank, epoch);
    if (q != g.rank) atomicAdd(ctr + 1, 1ull);  // check in: this CTA has read the epoch
  }
  if (q != g.rank || threadIdx.x != 0) return;

  // every rank's flag in this buffer and every local check-in (bounded wait), then the first
  // refusal over the ranks
  const unsigned long long *flags = reinterpret_cast<const unsigned long long *>(src + g.flag_off);
  const unsigned long long t0 = now_ns(), limit = (unsigned long long)g.timeout_us * 1000ull;
  bool ok = true;
  for (int r = 0; r <= g.world && ok; r++) {
    // r < world: rank r's flag; r == world: the check-ins, (world - 1) per epoch so far
    const unsigned long long *at = r < g.world ? flags + r : ctr + 1;
    const unsigned long long want = r < g.world ? epoch : (unsigned long long)(g.world - 1) * epoch;
    unsigned ns = 32;
    while (ld_acquire_sys(at) < want) {
      if (now_ns() - t0 > limit) {
        ok = false;
        break;
      }
      __nanosleep(ns);
      if (ns < 1024) ns *= 2;
    }
  }
  const long long *keys = reinterpret_cast<const long long *>(src + g.key_off);
  for (int j = 0; j < g.nproj; j++) {
    long long m = kNoKey;
    for (int r = 0; ok && r < g.world; r++) m = min(m, ld_relaxed_sys(keys + r * g.nproj + j));
    g.out_status[j]->first = !ok ? pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0)
                                 : (m == kNoKey ? ~0ull : (unsigned long long)m);
    g.out_status[j]->spare = 0;
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

APX_API int apx_gather_publish_async(apx_ctx *ctx, const apx_gather_desc *gd, void *stream) {
  if (!ctx || !gd || gd->world < 1 || gd->world > APX_MAX_PEERS || gd->rank < 0 ||
      gd->rank >= gd->world || gd->nproj < 1 || gd->nproj > APX_MAX_GATHER_PROJ ||
      (gd->out_off & 15) || (gd->key_off & 7) || (gd->flag_off & 7) || (gd->ctr_off & 7))
    return APX_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < gd->world; r++)
    if (!gd->peer[r]) return APX_ERR_INVALID_ARGUMENT;
  for (int j = 0; j < gd->nproj; j++)
    if ((gd->rows_off[j] & 1) || !gd->status[j] || !gd->out_status[j])
      return APX_ERR_INVALID_ARGUMENT;  // rows start 16-byte aligned
  if (cudaSetDevice(apx::context_device(ctx)) != cudaSuccess) return APX_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gd->world);
  cfg.blockDim = dim3(512);
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
