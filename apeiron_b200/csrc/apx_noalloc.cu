// apx_noalloc.cu — the allocation-free f32 projection entry point.
//
// apx_matvec_f32 stages the quantized activation (int8 codes, exponent bytes, descriptor) in
// device buffers the context allocates and grows on demand.  Some callers cannot allocate
// device memory once they are running: an engine that reserves its whole HBM budget at start-up
// and forbids later cudaMalloc, a process that shares the GPU under a fixed quota, a real-time
// decode loop where an allocation's latency or failure is not acceptable.  For them this file
// keeps that staging in one fixed array compiled into the library, so the call path allocates
// nothing: the caller passes the input and output device buffers and the refusal word.
//
// The array is a file-scope __device__ variable: every GPU that loads the library holds its
// APX_NOALLOC_SCRATCH_BYTES until the process exits.  Its address is looked up once per
// device (cudaGetSymbolAddress, with that device current) on the first call on that device and
// kept for the life of the process: a host application that resets a device (cudaDeviceReset)
// invalidates it, as it invalidates every context, stream and tensor of this library there.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "apx_common.cuh"
#include "apx_kernels.h"

namespace {

constexpr size_t kMaxN = APX_NOALLOC_MAX_N_IN;
constexpr size_t kDescOff = 0;                       // 32-byte activation descriptor
constexpr size_t kExpsOff = 256;                     // one exponent byte per 32 lanes
constexpr size_t kCodesOff = kExpsOff + kMaxN / 32;  // int8 codes
constexpr size_t kScratchBytes = kCodesOff + kMaxN;
static_assert(kScratchBytes == APX_NOALLOC_SCRATCH_BYTES, "scratch size in the header");

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_addr[kMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current), looked up once.
cudaError_t scratch_address(int device, void **out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_addr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return cudaSuccess;
}

}  // namespace

// Defined in apx_runtime.cu: the tensor's device payload, launch plan and geometry.
namespace apx {
bool tensor_launch_info(apx_ctx *ctx, uint64_t handle, uint32_t *type, const uint8_t **pack,
                        void **scratch, size_t *n_out, size_t *n_in, GemvPlan *plan,
                        int *device);
}

extern "C" APX_API int apx_matvec_f32_noalloc(apx_ctx *ctx, uint64_t tensor, size_t n_out,
                                              size_t n_in, const float *d_x, float *d_y,
                                              apx_call_status *d_status, void *stream) {
  if (!ctx || !d_status || (n_in && !d_x) || (n_out && !d_y)) return APX_ERR_INVALID_ARGUMENT;
  if (n_in > kMaxN) return APX_ERR_TOO_LARGE;
  uint32_t type;
  const uint8_t *pack;
  void *tscratch;
  size_t t_out, t_in;
  apx::GemvPlan plan;
  int device;
  if (!apx::tensor_launch_info(ctx, tensor, &type, &pack, &tscratch, &t_out, &t_in, &plan,
                               &device))
    return APX_ERR_INVALID_ARGUMENT;
  if (n_in != t_in || n_out > t_out) return APX_ERR_LAYOUT_MISMATCH;
  // the launches need the context's device current; the caller's current device is restored
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
  void *base = nullptr;
  if (e == cudaSuccess) e = scratch_address(device, &base);
  if (e != cudaSuccess) {
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return APX_ERR_CUDA;
  }
  unsigned char *s = static_cast<unsigned char *>(base);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the refusal word must start at all ones (no refusal); the scratch itself is fully
  // rewritten by the quantizer before the projection reads it
  e = cudaMemsetAsync(d_status, 0xFF, sizeof(apx_call_status), st);
  if (e == cudaSuccess)
    e = apx::launch_quant_f32(d_x, n_in, reinterpret_cast<int8_t *>(s + kCodesOff),
                              s + kExpsOff, s + kDescOff, st);
  if (e == cudaSuccess)
    e = apx::launch_gemv(plan, type, pack, tscratch, n_out, n_in,
                         reinterpret_cast<const int8_t *>(s + kCodesOff), s + kExpsOff,
                         s + kDescOff, nullptr, d_y, &d_status->first, st);
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}
