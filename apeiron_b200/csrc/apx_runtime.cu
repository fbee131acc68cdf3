// apx_runtime.cu — the C ABI (include/apeiron_cuda.h): contexts, weight uploads, validation
// in the reference's order, staging, launches and refusal decoding.
//
// Validation order follows the reference exactly:
//   matvec_q8act (src/engine/chart/mod.rs:1887-1925): plan first (an activation product
//     S·xq outside i64 refuses with Dequant(FixedOverflow)), then ShapeMismatch,
//     LengthOverflow, ShortPayload, then the rows;
//   matvec_q8act_quant_chunked (src/engine/chart/ffn.rs:667-745): with more than one chunk,
//     LengthOverflow and ShortPayload, then ShapeMismatch, then the plan;
//   matmat_q8act (src/engine/kern/matmat.rs:92-134): the lowest refusing column.
// Row refusals: the first row in row order wins (ffn.rs:659-661); a row whose block scale
// is Inf/NaN refuses with that scale's bits (num/dequant.rs:25-42), found once at upload.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "apx_common.cuh"
#include "apx_kernels.h"

using namespace apx;

namespace {

struct Tensor {
  uint32_t type = 0;      // the family the kernels run (Q5_0 runs as Q8_0)
  uint32_t src_type = 0;  // the uploaded ggml type: geometry and payload checks follow it
  size_t n_out = 0, n_in = 0, raw_len = 0, row_bytes = 0;
  uint8_t *d_pack = nullptr;
  size_t pack_bytes = 0;
  void *d_scratch = nullptr;  // K-split partial sums and arrival counters (zeroed once)
  size_t nonfinite_row = SIZE_MAX;  // first row holding an Inf/NaN block scale
  uint16_t nonfinite_bits = 0;
  GemvPlan plan{};
  GemmLayout gemm;          // tcgen05 fold GEMM view (Q8_0), built when the digit planes fail
  bool gemm_tried = false;
  LimbLayout limb;          // tcgen05 digit-plane view, built on the first multi-column call
  bool limb_tried = false;
  // The synchronous GEMV call as one CUDA graph [H2D, GEMV, D2H], captured on the context's
  // staging buffers for one (n_out, q_len) and rebuilt when they change.
  cudaGraphExec_t sync_exec = nullptr;
  const void *sync_dev = nullptr, *sync_host = nullptr;
  size_t sync_n_out = 0, sync_q_len = 0;
  bool sync_graph_off = false;  // a capture failed: eager launches from then on
  void release() {
    cudaFree(d_pack);
    if (d_scratch) cudaFree(d_scratch);
    free_gemm_layout(&gemm);
    free_limb_layout(&limb);
    if (sync_exec) cudaGraphExecDestroy(sync_exec);
    sync_exec = nullptr;
  }
};

struct DevBuf {
  void *p = nullptr;
  size_t cap = 0;
  cudaError_t ensure(size_t n) {
    if (n <= cap) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    size_t want = std::max(n, (size_t)1 << 16);
    cudaError_t e = cudaMalloc(&p, want);
    if (e == cudaSuccess) cap = want;
    return e;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
};

struct HostBuf {
  void *p = nullptr;
  size_t cap = 0;
  cudaError_t ensure(size_t n) {
    if (n <= cap) return cudaSuccess;
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
    size_t want = std::max(n, (size_t)1 << 16);
    cudaError_t e = cudaHostAlloc(&p, want, cudaHostAllocDefault);
    if (e == cudaSuccess) cap = want;
    return e;
  }
  void release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
  }
};

size_t align16(size_t n) { return (n + 15) & ~(size_t)15; }

bool geom(uint32_t t, size_t &qk, size_t &bb) {
  switch (t) {
    case APX_GGML_TYPE_Q8_0: qk = 32; bb = 34; return true;
    case APX_GGML_TYPE_Q5_0: qk = 32; bb = 22; return true;
    case APX_GGML_TYPE_Q4_K: qk = 256; bb = 144; return true;
    case APX_GGML_TYPE_Q6_K: qk = 256; bb = 210; return true;
    default: return false;
  }
}

int set_err(apx_err *err, int code) {
  if (err) {
    std::memset(err, 0, sizeof *err);
    err->code = code;
  }
  return code;
}

int cuda_err(apx_err *err, cudaError_t e) {
  set_err(err, APX_ERR_CUDA);
  if (err) err->cuda_error = (int32_t)e;
  return APX_ERR_CUDA;
}

}  // namespace

struct apx_ctx {
  int device = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::unordered_map<uint64_t, Tensor> tensors;
  uint64_t next = 1;
  DevBuf dev;      // [out | status | desc | exps | codes] of the synchronous calls
  DevBuf scratch;  // device-side quantization scratch of the f32 path
  DevBuf gwork;    // fold GEMM per-call workspace (its head zeroed whenever it is reallocated)
  DevBuf lwork;    // digit-plane GEMM per-call workspace (no state kept between calls)
  DevBuf ascratch; // codes / exps / descriptors of apx_matmat_f32_async off the fused route
  DevBuf fwork;    // per-CTA statistics of apx_swiglu_quant_async
  int gemm_route = APX_GEMM_AUTO;  // apx_ctx_set_gemm_route
  HostBuf host;    // pinned mirror of `dev`
};

namespace {

// Refusal of an activation that has no Q32.32 image (QuantAct::magnitude's NoQ32 case,
// chart/mod.rs:159-181), plus the descriptor the kernels read.
struct HostAct {
  int status = APX_OK;
  ActDesc desc{};
};

HostAct describe_host(const int8_t *codes, size_t q_len, const uint8_t *exps) {
  HostAct h;
  int emin = 1 << 30, emax = -1;
  unsigned nz = 0, m128 = 0;
  const size_t nb = (q_len + 31) / 32;
  // a code of -128 anywhere (one vectorised byte search): then look at the blocks it is in
  const bool any128 = q_len && std::memchr(codes, 0x80, q_len) != nullptr;
  for (size_t b = 0; b < nb; b++) {
    unsigned e = exps[b];
    if (e == APX_EXP_ZERO) continue;
    if (e > 62) {
      h.status = APX_ERR_INVALID_ARGUMENT;
      continue;
    }
    if (e >= 57 || any128) {  // codes whose product with 2^e may leave i64, or a -128
      size_t end = std::min(q_len, b * 32 + 32);
      for (size_t j = b * 32; j < end; j++) {
        int c = codes[j];
        if (c == -128) m128 = 1;
        if (e >= 57) {
          long long lim = 1ll << (63 - e);
          if (c < -lim || c > lim - 1) {
            if (h.status == APX_OK) h.status = APX_ERR_FIXED_OVERFLOW;
          }
        }
      }
    }
    emin = std::min(emin, (int)e);
    emax = std::max(emax, (int)e);
    nz++;
  }
  h.desc.status = h.status;
  h.desc.emin = emax >= 0 ? emin : 0;
  h.desc.emax = emax;
  h.desc.n_in = (int32_t)q_len;
  h.desc.nz = nz;
  h.desc.pad[0] = m128;
  return h;
}

// ShapeMismatch / LengthOverflow / ShortPayload / layout checks of one call.
int check_geometry(const Tensor &t, size_t n_out, size_t n_in, size_t q_len, bool chunked_order,
                   apx_err *err) {
  size_t qk, bb, row_bytes, need;
  geom(t.src_type, qk, bb);
  auto shape = [&]() {
    set_err(err, APX_ERR_SHAPE_MISMATCH);
    if (err) {
      err->a = q_len;
      err->b = n_in;
    }
    return APX_ERR_SHAPE_MISMATCH;
  };
  if (!chunked_order && q_len != n_in) return shape();
  if (__builtin_mul_overflow((n_in + qk - 1) / qk, bb, &row_bytes) ||
      __builtin_mul_overflow(n_out, row_bytes, &need))
    return set_err(err, APX_ERR_LENGTH_OVERFLOW);
  if (t.raw_len < need) {
    set_err(err, APX_ERR_SHORT_PAYLOAD);
    if (err) {
      err->a = need;
      err->b = t.raw_len;
    }
    return APX_ERR_SHORT_PAYLOAD;
  }
  if (chunked_order && q_len != n_in) return shape();
  if (n_in != t.n_in || n_out > t.n_out) return set_err(err, APX_ERR_LAYOUT_MISMATCH);
  return APX_OK;
}

bool is_activation_kind(unsigned kind) {
  return kind == APX_ERR_FIXED_OVERFLOW || kind == APX_ERR_QUANT_REFUSED ||
         kind == APX_ERR_INVALID_ARGUMENT;
}

// Merge the kernel's refusal word with the upload-time non-finite finding.
int decode_status(const Tensor &t, size_t n_out, unsigned long long word, apx_err *err) {
  unsigned kind = (unsigned)((word >> 16) & 0xFF);
  size_t krow = word == ~0ull ? SIZE_MAX : (size_t)(word >> 24);
  if (word != ~0ull && is_activation_kind(kind)) return set_err(err, (int)kind);
  size_t nrow = t.nonfinite_row < n_out ? t.nonfinite_row : SIZE_MAX;
  if (nrow == SIZE_MAX && krow == SIZE_MAX) return set_err(err, APX_OK);
  if (nrow <= krow) {
    set_err(err, APX_ERR_NONFINITE_SCALE);
    if (err) {
      err->bits = t.nonfinite_bits;
      err->row = nrow;
    }
    return APX_ERR_NONFINITE_SCALE;
  }
  set_err(err, (int)kind);
  if (err) err->row = krow;
  return (int)kind;
}

Tensor *find(apx_ctx *ctx, uint64_t h) {
  auto it = ctx->tensors.find(h);
  return it == ctx->tensors.end() ? nullptr : &it->second;
}

uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

bool nonfinite(uint16_t h) { return ((h >> 10) & 0x1F) == 0x1F; }

// First Inf/NaN block scale in row order, in each row's dequantization order
// (num/dequant.rs: Q8_0 d per block; Q4_K d then dmin per super-block; Q6_K d).
void scan_nonfinite(Tensor &t, const uint8_t *raw) {
  size_t qk, bb;
  geom(t.type, qk, bb);
  const size_t blocks = (t.n_in + qk - 1) / qk;
  for (size_t r = 0; r < t.n_out; r++) {
    const uint8_t *row = raw + r * t.row_bytes;
    for (size_t b = 0; b < blocks; b++) {
      const uint8_t *blk = row + b * bb;
      uint16_t cand[2];
      int nc = 0;
      if (t.type == APX_GGML_TYPE_Q8_0) {
        cand[nc++] = rd16(blk);
      } else if (t.type == APX_GGML_TYPE_Q4_K) {
        cand[nc++] = rd16(blk);
        cand[nc++] = rd16(blk + 2);
      } else {
        cand[nc++] = rd16(blk + 208);
      }
      for (int i = 0; i < nc; i++) {
        if (nonfinite(cand[i])) {
          t.nonfinite_row = r;
          t.nonfinite_bits = cand[i];
          return;
        }
      }
    }
  }
}

// Synchronous single-column projection of host activations.
// ha: the caller's describe_host of (codes, exps).
// A Q5_0 block [f16 d][qh: 4 bytes][qs: 16 bytes] as the Q8_0 block [f16 d][32 int8 codes] of the
// same weights (quant.rs:261-299 q5_0_codes): lane j < 16 is the low nibble of qs[j] with bit j of
// qh as its fifth bit, lane 16 + j the high nibble with bit 16 + j, each offset by -16.  The
// dequantized weights d·code are unchanged, so the Q8_0 kernels serve Q5_0 exactly.
void widen_q5_0(const uint8_t *q5, uint8_t *q8) {
  q8[0] = q5[0];
  q8[1] = q5[1];
  const uint32_t qh = (uint32_t)q5[2] | ((uint32_t)q5[3] << 8) | ((uint32_t)q5[4] << 16) |
                      ((uint32_t)q5[5] << 24);
  for (int j = 0; j < 16; j++) {
    const unsigned nib = q5[6 + j];
    const int lo = (int)((nib & 0xFu) | (((qh >> j) & 1u) << 4)) - 16;
    const int hi = (int)((nib >> 4) | (((qh >> (16 + j)) & 1u) << 4)) - 16;
    q8[2 + j] = (uint8_t)(int8_t)lo;
    q8[2 + 16 + j] = (uint8_t)(int8_t)hi;
  }
}

int matvec_sync(apx_ctx *ctx, Tensor &t, size_t n_out, size_t n_in, const int8_t *codes,
                size_t q_len, const uint8_t *exps, const HostAct &ha, int64_t *out,
                apx_err *err) {
  const size_t nb = (q_len + 31) / 32;
  const size_t out_sz = align16(n_out * 8);
  const size_t head = 16 + 32;  // status + desc
  const size_t exps_sz = align16(nb), codes_sz = align16(q_len);
  const size_t in_sz = head + exps_sz + codes_sz;
  cudaError_t e;
  if ((e = ctx->dev.ensure(out_sz + in_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->host.ensure(out_sz + in_sz)) != cudaSuccess) return cuda_err(err, e);
  uint8_t *h = (uint8_t *)ctx->host.p, *d = (uint8_t *)ctx->dev.p;
  std::memset(h + out_sz, 0xFF, 16);
  std::memcpy(h + out_sz + 16, &ha.desc, sizeof(ActDesc));
  std::memcpy(h + out_sz + head, exps, nb);
  std::memcpy(h + out_sz + head + exps_sz, codes, q_len);
  auto enqueue = [&]() -> cudaError_t {
    cudaError_t q = cudaMemcpyAsync(d + out_sz, h + out_sz, in_sz, cudaMemcpyHostToDevice,
                                    ctx->stream);
    if (q == cudaSuccess)
      q = launch_gemv(t.plan, t.type, t.d_pack, t.d_scratch, n_out, n_in,
                      (const int8_t *)(d + out_sz + head + exps_sz), d + out_sz + head,
                      d + out_sz + 16, (long long *)d, nullptr,
                      (unsigned long long *)(d + out_sz), ctx->stream);
    if (q == cudaSuccess)
      q = cudaMemcpyAsync(h, d, out_sz + 16, cudaMemcpyDeviceToHost, ctx->stream);
    return q;
  };
  // One graph launch instead of three stream operations: the copies and the kernel read and
  // write the same staging addresses on every call with this shape.
  const bool fresh = t.sync_exec && t.sync_dev == d && t.sync_host == h &&
                     t.sync_n_out == n_out && t.sync_q_len == q_len;
  if (!fresh && !t.sync_graph_off) {
    if (t.sync_exec) cudaGraphExecDestroy(t.sync_exec);
    t.sync_exec = nullptr;
    cudaGraph_t gr = nullptr;
    cudaError_t ce = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
    if (ce == cudaSuccess) {
      set_pdl_suppressed(true);
      const cudaError_t qe = enqueue();
      set_pdl_suppressed(false);
      ce = cudaStreamEndCapture(ctx->stream, &gr);
      if (qe != cudaSuccess) ce = qe;
    }
    if (ce == cudaSuccess) ce = cudaGraphInstantiate(&t.sync_exec, gr, 0);
    if (gr) cudaGraphDestroy(gr);
    if (ce == cudaSuccess) {
      t.sync_dev = d;
      t.sync_host = h;
      t.sync_n_out = n_out;
      t.sync_q_len = q_len;
    } else {
      t.sync_exec = nullptr;
      t.sync_graph_off = true;
      cudaGetLastError();
    }
  }
  e = t.sync_exec ? cudaGraphLaunch(t.sync_exec, ctx->stream) : enqueue();
  if (e != cudaSuccess) return cuda_err(err, e);
  if ((e = cudaStreamSynchronize(ctx->stream)) != cudaSuccess) return cuda_err(err, e);
  unsigned long long word;
  std::memcpy(&word, h + out_sz, 8);
  int rc = decode_status(t, n_out, word, err);
  if (rc == APX_OK && n_out) std::memcpy(out, h, n_out * 8);
  return rc;
}

// ---- multi-column calls on the tensor cores ---------------------------------------------------

constexpr size_t kGemmMinCols = 4;  // fewer columns run as separate GEMVs

// Whether a Q8_0 k-column call can take the fold GEMM (apx_gemm.cu): enough columns, a width the
// kernel takes, and a weight exponent spread that leaves room for its i64 fold.  Its view of the
// tensor is built on the first such call.
bool gemm_route(apx_ctx *ctx, Tensor &t, size_t n_out, size_t n_in, size_t k_cols) {
  if (t.type != APX_GGML_TYPE_Q8_0 || k_cols < kGemmMinCols || n_out == 0 ||
      !gemm_shape_ok(n_in) || !t.d_pack)
    return false;
  if (!t.gemm_tried) {
    t.gemm_tried = true;
    if (build_gemm_layout(t.plan, t.d_pack, t.n_out, t.n_in, &t.gemm, ctx->stream) !=
        cudaSuccess)
      cudaGetLastError();  // no GEMM view: the call runs as GEMVs
  }
  return gemm_supported(t.gemm);
}

// The tensor-core route of a k-column call: a Q8_0 call below kFoldMaxMacs on the fold GEMM
// (apx_gemm.cu); otherwise the digit-plane GEMM (apx_lgemm.cu) for every family whose weights
// fit four digits, else the fold GEMM for Q8_0, else one GEMV per column.
enum TcRoute { kTcNone = 0, kTcLimb = 1, kTcFold = 2 };

// Below this many multiply-adds a Q8_0 call runs faster on the per-block fold GEMM than on the
// digit planes (B200, 512 tokens: 4864x896 38.6 vs 47.2 us, 896x4864 37.5 vs 59.7 us; above it
// 8192x8192 277 vs 222 us, 28672x8192 918 vs 697 us): the fold's work per MMA is one int8 dot
// against the digit planes' six, but its exact per-block epilogue grows with the call.
constexpr double kFoldMaxMacs = 6e9;

TcRoute tc_route(apx_ctx *ctx, Tensor &t, size_t n_out, size_t n_in, size_t k_cols) {
  if (k_cols < kGemmMinCols || n_out == 0 || !t.d_pack) return kTcNone;
  const bool small = (double)n_out * (double)n_in * (double)k_cols < kFoldMaxMacs;
  if (t.type == kQ8_0 && ctx->gemm_route != APX_GEMM_DIGITS &&
      (small || ctx->gemm_route == APX_GEMM_FOLD) && gemm_route(ctx, t, n_out, n_in, k_cols))
    return kTcFold;
  if (limb_shape_ok(n_in)) {
    if (!t.limb_tried) {
      t.limb_tried = true;
      if (build_limb_layout(t.plan, t.type, t.d_pack, t.n_out, t.n_in, &t.limb, ctx->stream) !=
          cudaSuccess)
        cudaGetLastError();  // no digit planes: the next route
    }
    if (t.limb.ok) return kTcLimb;
  }
  return gemm_route(ctx, t, n_out, n_in, k_cols) ? kTcFold : kTcNone;
}

// The route's own workspace: the fold GEMM keeps self-resetting counters in a layout of its
// own, so the two never share one buffer.
cudaError_t ensure_gwork(apx_ctx *ctx, TcRoute route, size_t n_cols, size_t n_in, size_t n_out) {
  DevBuf &b = route == kTcLimb ? ctx->lwork : ctx->gwork;
  const size_t need = route == kTcLimb ? limb_work_bytes(n_cols, n_in, n_out, ctx->sm_count)
                                       : gemm_work_bytes(n_cols, n_in, n_out, ctx->sm_count);
  if (need <= b.cap) return cudaSuccess;
  cudaError_t e = b.ensure(need);
  if (e == cudaSuccess) e = cudaMemset(b.p, 0, b.cap);
  return e;
}

// One tensor-core k-column launch of device codes (column c at codes + c·ld) on the route.
cudaError_t launch_tc(apx_ctx *ctx, Tensor &t, TcRoute route, size_t n_out, size_t n_in,
                      size_t k, const int8_t *codes, size_t ld, const uint8_t *exps, size_t ldb,
                      const void *descs, long long *out_q32, float *out_f32,
                      unsigned long long *status, cudaStream_t stream) {
  if (route == kTcLimb)
    return launch_limb_gemm(t.plan, t.type, t.d_pack, t.limb, n_out, n_in, k, codes, ld, exps,
                            ldb, descs, ctx->lwork.p, out_q32, out_f32, status, ctx->sm_count,
                            stream);
  return launch_gemm_q8_0(t.plan, t.d_pack, t.gemm, n_out, n_in, k, codes, ld, exps, ldb, descs,
                          ctx->gwork.p, out_q32, out_f32, status, ctx->sm_count, stream);
}

// The fused f32 route (quantization inside the GEMM's prep kernel), when the input allows it.
bool tc_f32_ok(TcRoute route, size_t n_in, const float *x, size_t ldx) {
  return route == kTcLimb ? limb_f32_ok(n_in, x, ldx) : gemm_f32_ok(n_in, x, ldx);
}

cudaError_t launch_tc_f32(apx_ctx *ctx, Tensor &t, TcRoute route, size_t n_out, size_t n_in,
                          size_t k, const float *x, size_t ldx, long long *out_q32,
                          float *out_f32, unsigned long long *status, cudaStream_t stream) {
  if (route == kTcLimb)
    return launch_limb_gemm_f32(t.plan, t.type, t.d_pack, t.limb, n_out, n_in, k, x, ldx,
                                ctx->lwork.p, out_q32, out_f32, status, ctx->sm_count, stream);
  return launch_gemm_q8_0_f32(t.plan, t.d_pack, t.gemm, n_out, n_in, k, x, ldx, ctx->gwork.p,
                              out_q32, out_f32, status, ctx->sm_count, stream);
}

// Synchronous k-column projection of host activations through the GEMM: one H2D of
// [status | exps | codes (rows padded to 128 bytes)], one D2H of [outputs | status].
int matmat_gemm_sync(apx_ctx *ctx, Tensor &t, TcRoute route, size_t n_out, size_t n_in, size_t k,
                     const int8_t *codes, const uint8_t *exps, int64_t *out, apx_err *err) {
  const size_t nb = (n_in + 31) / 32, ld = (n_in + 127) / 128 * 128;
  const size_t out_sz = align16(k * n_out * 8), st_sz = align16(k * 16);
  const size_t ex_sz = align16(k * nb), cd_sz = k * ld;
  const size_t in_sz = st_sz + ex_sz + cd_sz;
  cudaError_t e;
  if ((e = ctx->dev.ensure(out_sz + in_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->host.ensure(out_sz + in_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ensure_gwork(ctx, route, k, n_in, n_out)) != cudaSuccess) return cuda_err(err, e);
  uint8_t *h = (uint8_t *)ctx->host.p, *d = (uint8_t *)ctx->dev.p;
  uint8_t *hs = h + out_sz, *he = hs + st_sz, *hc = he + ex_sz;
  std::memset(hs, 0xFF, k * 16);
  std::memcpy(he, exps, k * nb);
  for (size_t c = 0; c < k; c++) {
    std::memcpy(hc + c * ld, codes + c * n_in, n_in);
    std::memset(hc + c * ld + n_in, 0, ld - n_in);
  }
  uint8_t *ds = d + out_sz, *de = ds + st_sz, *dc = de + ex_sz;
  e = cudaMemcpyAsync(ds, hs, in_sz, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess)
    e = launch_tc(ctx, t, route, n_out, n_in, k, (const int8_t *)dc, ld, de, nb, nullptr,
                  (long long *)d, nullptr, (unsigned long long *)ds, ctx->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h, d, out_sz + k * 16, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_err(err, e);
  for (size_t c = 0; c < k; c++) {
    unsigned long long word;
    std::memcpy(&word, hs + c * 16, 8);
    const int rc = decode_status(t, n_out, word, err);
    if (rc != APX_OK) {
      if (err) err->col = c;
      return rc;
    }
  }
  std::memcpy(out, h, k * n_out * 8);
  return set_err(err, APX_OK);
}

}  // namespace

namespace apx {
// The launch view of an uploaded tensor, for entry points defined in other files.
bool tensor_launch_info(apx_ctx *ctx, uint64_t handle, uint32_t *type, const uint8_t **pack,
                        void **scratch, size_t *n_out, size_t *n_in, GemvPlan *plan,
                        int *device) {
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, handle);
  if (!t) return false;
  *type = t->type;
  *pack = t->d_pack;
  *scratch = t->d_scratch;
  *n_out = t->n_out;
  *n_in = t->n_in;
  *plan = t->plan;
  *device = ctx->device;
  return true;
}

int context_device(const apx_ctx *ctx) { return ctx->device; }
}  // namespace apx

extern "C" {

const char *apx_version(void) { return "apeiron_b200 0.1 (sm_100a)"; }

apx_ctx *apx_open(int device, apx_err *err) {
  set_err(err, APX_OK);
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || device < 0 || device >= n) {
    set_err(err, e != cudaSuccess ? APX_ERR_CUDA : APX_ERR_INVALID_ARGUMENT);
    if (err) err->cuda_error = (int32_t)e;
    return nullptr;
  }
  if ((e = cudaSetDevice(device)) != cudaSuccess) {
    cuda_err(err, e);
    return nullptr;
  }
  apx_ctx *ctx = new apx_ctx();
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if ((e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking)) != cudaSuccess) {
    delete ctx;
    cuda_err(err, e);
    return nullptr;
  }
  return ctx;
}

void apx_close(apx_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (auto &kv : ctx->tensors) kv.second.release();
  ctx->dev.release();
  ctx->scratch.release();
  ctx->gwork.release();
  ctx->lwork.release();
  ctx->ascratch.release();
  ctx->fwork.release();
  ctx->host.release();
  cudaStreamDestroy(ctx->stream);
  delete ctx;
}

int apx_tensor_upload(apx_ctx *ctx, uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                      size_t n_out, size_t n_in, uint64_t *handle, apx_err *err) {
  if (!ctx || !handle || (!raw && raw_len)) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  size_t qk, bb, row_bytes, need;
  if (!geom(ggml_type, qk, bb)) {
    set_err(err, APX_ERR_UNSUPPORTED_QUANT);
    if (err) err->ggml_type = ggml_type;
    return APX_ERR_UNSUPPORTED_QUANT;
  }
  if (__builtin_mul_overflow((n_in + qk - 1) / qk, bb, &row_bytes) ||
      __builtin_mul_overflow(n_out, row_bytes, &need))
    return set_err(err, APX_ERR_LENGTH_OVERFLOW);
  if (raw_len < need) {
    set_err(err, APX_ERR_SHORT_PAYLOAD);
    if (err) {
      err->a = need;
      err->b = raw_len;
    }
    return APX_ERR_SHORT_PAYLOAD;
  }
  if (n_in > ((size_t)1 << 28) || n_out > ((size_t)1 << 36))
    return set_err(err, APX_ERR_TOO_LARGE);
  // Q5_0 is served as Q8_0: its blocks widen to Q8_0 blocks of the same weights on the host
  std::vector<uint8_t> widened;
  uint32_t exec_type = ggml_type;
  if (ggml_type == APX_GGML_TYPE_Q5_0) {
    const size_t nb = (n_in + 31) / 32, wrow = nb * 34;
    try {
      widened.resize(n_out * wrow);
    } catch (const std::bad_alloc &) {
      return set_err(err, APX_ERR_OUT_OF_MEMORY);
    }
    for (size_t r = 0; r < n_out; r++)
      for (size_t b = 0; b < nb; b++)
        widen_q5_0(raw + r * row_bytes + b * 22, widened.data() + r * wrow + b * 34);
    raw = widened.data();
    row_bytes = wrow;
    need = n_out * wrow;
    exec_type = APX_GGML_TYPE_Q8_0;
  }
  Tensor t;
  t.type = exec_type;
  t.src_type = ggml_type;
  t.n_out = n_out;
  t.n_in = n_in;
  t.raw_len = raw_len;
  t.row_bytes = row_bytes;
  scan_nonfinite(t, raw);
  ggml_type = exec_type;
  t.plan = plan_gemv(ggml_type, n_out, n_in, ctx->sm_count);
  t.pack_bytes = packed_bytes(t.plan, ggml_type);
  cudaError_t e;
  uint8_t *d_raw = nullptr;
  if (t.pack_bytes) {
    if ((e = cudaMalloc(&t.d_pack, t.pack_bytes)) != cudaSuccess) {
      set_err(err, APX_ERR_OUT_OF_MEMORY);
      if (err) err->cuda_error = (int32_t)e;
      return APX_ERR_OUT_OF_MEMORY;
    }
    if ((e = cudaMalloc(&d_raw, std::max(need, (size_t)1))) != cudaSuccess) {
      cudaFree(t.d_pack);
      set_err(err, APX_ERR_OUT_OF_MEMORY);
      if (err) err->cuda_error = (int32_t)e;
      return APX_ERR_OUT_OF_MEMORY;
    }
    e = cudaMemcpyAsync(d_raw, raw, need, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
      e = launch_repack(t.plan, d_raw, t.d_pack, ggml_type, n_out, n_in, row_bytes, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(d_raw);
    if (e != cudaSuccess) {
      cudaFree(t.d_pack);
      return cuda_err(err, e);
    }
  }
  const size_t sb = gemv_scratch_bytes(t.plan);
  if (sb) {
    if ((e = cudaMalloc(&t.d_scratch, sb)) != cudaSuccess ||
        (e = cudaMemset(t.d_scratch, 0, sb)) != cudaSuccess) {
      cudaFree(t.d_pack);
      if (t.d_scratch) cudaFree(t.d_scratch);
      set_err(err, APX_ERR_OUT_OF_MEMORY);
      if (err) err->cuda_error = (int32_t)e;
      return APX_ERR_OUT_OF_MEMORY;
    }
  }
  uint64_t h = ctx->next++;
  ctx->tensors[h] = t;
  *handle = h;
  return set_err(err, APX_OK);
}

int apx_tensor_free(apx_ctx *ctx, uint64_t handle) {
  if (!ctx) return APX_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, handle);
  if (!t) return APX_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  t->release();
  ctx->tensors.erase(handle);
  return APX_OK;
}

size_t apx_tensor_device_bytes(apx_ctx *ctx, uint64_t handle) {
  if (!ctx) return 0;
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, handle);
  if (!t) return 0;
  // the repacked payload, plus the tensor-core views once a multi-column call has built them
  size_t n = t->pack_bytes;
  if (t->limb.ok)
    n += (size_t)t->limb.digits * t->limb.m_pad * t->limb.kp + 4 * t->limb.m_pad;
  if (t->gemm.base)
    n += t->gemm.m_pad * t->gemm.kp + (size_t)t->gemm.nb_pad * t->gemm.m_pad * 4 + t->gemm.m_pad * 4;
  return n;
}

int apx_matvec_q8act(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                     const int8_t *codes, size_t q_len, const uint8_t *exps, int64_t *out,
                     apx_err *err) {
  if (!ctx || (!codes && q_len) || (!exps && q_len) || (!out && n_out))
    return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  cudaSetDevice(ctx->device);
  HostAct ha = describe_host(codes, q_len, exps);  // the plan runs first (chart/mod.rs:1893)
  if (ha.status != APX_OK) return set_err(err, ha.status);
  int rc = check_geometry(*t, n_out, n_in, q_len, false, err);
  if (rc != APX_OK) return rc;
  return matvec_sync(ctx, *t, n_out, n_in, codes, q_len, exps, ha, out, err);
}

int apx_matvec_q8act_chunked(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                             const int8_t *codes, size_t q_len, const uint8_t *exps,
                             size_t chunks, int64_t *out, apx_err *err) {
  size_t upper = n_out == 0 ? 1 : n_out;
  size_t actual = std::min(std::max(std::min(chunks, (size_t)8), (size_t)1), upper);
  if (actual == 1)
    return apx_matvec_q8act(ctx, tensor, n_out, n_in, codes, q_len, exps, out, err);
  if (!ctx || (!codes && q_len) || (!exps && q_len) || (!out && n_out))
    return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  cudaSetDevice(ctx->device);
  int rc = check_geometry(*t, n_out, n_in, q_len, true, err);
  if (rc != APX_OK) return rc;
  HostAct ha = describe_host(codes, q_len, exps);
  if (ha.status != APX_OK) return set_err(err, ha.status);
  return matvec_sync(ctx, *t, n_out, n_in, codes, q_len, exps, ha, out, err);
}

int apx_matmat_q8act(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in, size_t k_cols,
                     const int8_t *codes, size_t q_len, const uint8_t *exps, int64_t *out,
                     apx_err *err) {
  if (!ctx || (k_cols && ((!codes && q_len) || (!exps && q_len) || (!out && n_out))))
    return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  cudaSetDevice(ctx->device);
  const size_t nb = (q_len + 31) / 32;
  if (k_cols && check_geometry(*t, n_out, n_in, q_len, false, nullptr) == APX_OK) {
    const TcRoute route = tc_route(ctx, *t, n_out, n_in, k_cols);
    if (route != kTcNone)
      return matmat_gemm_sync(ctx, *t, route, n_out, n_in, k_cols, codes, exps, out, err);
  }
  for (size_t c = 0; c < k_cols; c++) {
    HostAct ha = describe_host(codes + c * q_len, q_len, exps + c * nb);
    int rc = ha.status;
    if (rc == APX_OK) rc = check_geometry(*t, n_out, n_in, q_len, false, err);
    else set_err(err, rc);
    if (rc == APX_OK)
      rc = matvec_sync(ctx, *t, n_out, n_in, codes + c * q_len, q_len, exps + c * nb, ha,
                       out + c * n_out, err);
    if (rc != APX_OK) {
      if (err) err->col = c;
      return rc;
    }
  }
  return set_err(err, APX_OK);
}

int apx_quant_act(apx_ctx *ctx, const int64_t *x, size_t n, int8_t *codes, uint8_t *exps,
                  apx_err *err) {
  if (!ctx || (n && (!x || !codes || !exps))) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  const size_t nb = (n + 31) / 32;
  const size_t x_sz = align16(n * 8), c_sz = align16(n), e_sz = align16(nb), d_sz = 32;
  cudaError_t e;
  if ((e = ctx->dev.ensure(x_sz + c_sz + e_sz + d_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->host.ensure(x_sz + c_sz + e_sz + d_sz)) != cudaSuccess) return cuda_err(err, e);
  uint8_t *h = (uint8_t *)ctx->host.p, *d = (uint8_t *)ctx->dev.p;
  std::memcpy(h, x, n * 8);
  e = cudaMemcpyAsync(d, h, n * 8, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess)
    e = launch_quant_q32((const long long *)d, n, (int8_t *)(d + x_sz), d + x_sz + c_sz,
                         d + x_sz + c_sz + e_sz, ctx->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h + x_sz, d + x_sz, c_sz + e_sz + d_sz, cudaMemcpyDeviceToHost,
                        ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_err(err, e);
  ActDesc desc;
  std::memcpy(&desc, h + x_sz + c_sz + e_sz, sizeof desc);
  if (desc.status != APX_OK) return set_err(err, desc.status);
  std::memcpy(codes, h + x_sz, n);
  std::memcpy(exps, h + x_sz + c_sz, nb);
  return set_err(err, APX_OK);
}

int apx_matvec_f32(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in, const float *x,
                   float *y, apx_err *err) {
  if (!ctx || (n_in && !x) || (n_out && !y)) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  cudaSetDevice(ctx->device);
  int rc = check_geometry(*t, n_out, n_in, n_in, false, err);
  if (rc != APX_OK) return rc;
  const size_t nb = (n_in + 31) / 32;
  const size_t out_sz = align16(n_out * 4), x_sz = align16(n_in * 4);
  const size_t c_sz = align16(n_in), e_sz = align16(nb);
  cudaError_t e;
  if ((e = ctx->dev.ensure(out_sz + 16 + x_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->host.ensure(out_sz + 16 + x_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->scratch.ensure(32 + e_sz + c_sz)) != cudaSuccess) return cuda_err(err, e);
  uint8_t *h = (uint8_t *)ctx->host.p, *d = (uint8_t *)ctx->dev.p;
  uint8_t *s = (uint8_t *)ctx->scratch.p;
  std::memset(h + out_sz, 0xFF, 16);
  std::memcpy(h + out_sz + 16, x, n_in * 4);
  e = cudaMemcpyAsync(d + out_sz, h + out_sz, 16 + n_in * 4, cudaMemcpyHostToDevice,
                      ctx->stream);
  if (e == cudaSuccess)
    e = launch_quant_f32((const float *)(d + out_sz + 16), n_in, (int8_t *)(s + 32 + e_sz),
                         s + 32, s, ctx->stream);
  if (e == cudaSuccess)
    e = launch_gemv(t->plan, t->type, t->d_pack, t->d_scratch, n_out, n_in, (const int8_t *)(s + 32 + e_sz),
                    s + 32, s, nullptr, (float *)d, (unsigned long long *)(d + out_sz),
                    ctx->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h, d, out_sz + 16, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_err(err, e);
  unsigned long long word;
  std::memcpy(&word, h + out_sz, 8);
  rc = decode_status(*t, n_out, word, err);
  if (rc == APX_OK && n_out) std::memcpy(y, h, n_out * 4);
  return rc;
}

int apx_matmat_f32(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in, size_t k_cols,
                   const float *x, float *y, apx_err *err) {
  if (!ctx || (k_cols && ((n_in && !x) || (n_out && !y))))
    return set_err(err, APX_ERR_INVALID_ARGUMENT);
  if (k_cols > (size_t)INT32_MAX) return set_err(err, APX_ERR_TOO_LARGE);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  cudaSetDevice(ctx->device);
  int rc = check_geometry(*t, n_out, n_in, n_in, false, err);
  if (rc != APX_OK || k_cols == 0) return rc;
  const size_t ld = apx_act_padded_len(n_in), ldb = ld / 32;
  const size_t y_sz = align16(k_cols * n_out * 4), st_sz = align16(k_cols * 16);
  const size_t x_sz = align16(k_cols * n_in * 4);
  const size_t ds_sz = align16(k_cols * sizeof(ActDesc)), ex_sz = align16(k_cols * ldb);
  cudaError_t e;
  if ((e = ctx->dev.ensure(y_sz + st_sz + x_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->host.ensure(y_sz + st_sz + x_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->scratch.ensure(ds_sz + ex_sz + k_cols * ld)) != cudaSuccess)
    return cuda_err(err, e);
  const TcRoute route = tc_route(ctx, *t, n_out, n_in, k_cols);
  const bool gemm = route != kTcNone;
  if (gemm && (e = ensure_gwork(ctx, route, k_cols, n_in, n_out)) != cudaSuccess)
    return cuda_err(err, e);
  uint8_t *h = (uint8_t *)ctx->host.p, *d = (uint8_t *)ctx->dev.p;
  uint8_t *sc = (uint8_t *)ctx->scratch.p;
  uint8_t *descs = sc, *dexp = sc + ds_sz;
  int8_t *dcod = (int8_t *)(sc + ds_sz + ex_sz);
  std::memset(h + y_sz, 0xFF, k_cols * 16);
  std::memcpy(h + y_sz + st_sz, x, k_cols * n_in * 4);
  e = cudaMemcpyAsync(d + y_sz, h + y_sz, st_sz + k_cols * n_in * 4, cudaMemcpyHostToDevice,
                      ctx->stream);
  unsigned long long *status = (unsigned long long *)(d + y_sz);
  const float *dx = (const float *)(d + y_sz + st_sz);
  if (e == cudaSuccess && gemm && tc_f32_ok(route, n_in, dx, n_in)) {
    // quantize inside the GEMM's prep kernel: one pass over the f32 columns
    e = launch_tc_f32(ctx, *t, route, n_out, n_in, k_cols, dx, n_in, nullptr, (float *)d, status,
                      ctx->stream);
  } else if (e == cudaSuccess && gemm) {
    e = launch_quant_f32_cols(dx, n_in, n_in, (int)k_cols, dcod, ld, dexp, ldb, descs,
                              ctx->stream);
    if (e == cudaSuccess)
      e = launch_tc(ctx, *t, route, n_out, n_in, k_cols, dcod, ld, dexp, ldb, descs, nullptr,
                    (float *)d, status, ctx->stream);
  } else {
    if (e == cudaSuccess)
      e = launch_quant_f32_cols(dx, n_in, n_in, (int)k_cols, dcod, ld, dexp, ldb, descs,
                                ctx->stream);
    for (size_t c = 0; e == cudaSuccess && c < k_cols; c++)
      e = launch_gemv(t->plan, t->type, t->d_pack, t->d_scratch, n_out, n_in, dcod + c * ld,
                      dexp + c * ldb, descs + c * sizeof(ActDesc), nullptr,
                      (float *)d + c * n_out, status + 2 * c, ctx->stream);
  }
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h, d, y_sz + k_cols * 16, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_err(err, e);
  for (size_t c = 0; c < k_cols; c++) {
    unsigned long long word;
    std::memcpy(&word, h + y_sz + c * 16, 8);
    rc = decode_status(*t, n_out, word, err);
    if (rc != APX_OK) {
      if (err) err->col = c;
      return rc;
    }
  }
  std::memcpy(y, h, k_cols * n_out * 4);
  return set_err(err, APX_OK);
}

int apx_debug_block_dots(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                         const int8_t *codes, int32_t *dots, apx_err *err) {
  if (!ctx || !codes || !dots) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t || n_in != t->n_in || n_out > t->n_out) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  cudaSetDevice(ctx->device);
  const int units = units_per_row_tile(t->type, n_in);
  const size_t span = t->type == APX_GGML_TYPE_Q8_0 ? 128 : 256;
  const size_t padded = units * span;
  const size_t per_row = t->type == APX_GGML_TYPE_Q8_0 ? (n_in + 31) / 32
                                                       : (size_t)units * (t->type == APX_GGML_TYPE_Q6_K ? 16 : 8);
  const size_t c_sz = align16(padded), d_sz = n_out * per_row * 4;
  cudaError_t e;
  if ((e = ctx->dev.ensure(c_sz + d_sz)) != cudaSuccess) return cuda_err(err, e);
  if ((e = ctx->host.ensure(c_sz + d_sz)) != cudaSuccess) return cuda_err(err, e);
  uint8_t *h = (uint8_t *)ctx->host.p, *d = (uint8_t *)ctx->dev.p;
  std::memset(h, 0, c_sz);
  std::memcpy(h, codes, n_in);
  e = cudaMemcpyAsync(d, h, c_sz, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess)
    e = launch_block_dots(t->plan, t->type, t->d_pack, n_out, n_in, (const int8_t *)d,
                          (int32_t *)(d + c_sz), ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(h + c_sz, d + c_sz, d_sz, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_err(err, e);
  std::memcpy(dots, h + c_sz, d_sz);
  return set_err(err, APX_OK);
}

// ---- asynchronous device-buffer entry points ------------------------------------------------

size_t apx_act_padded_len(size_t n_in) { return (n_in + 255) / 256 * 256; }

int apx_act_describe_async(apx_ctx *ctx, const int8_t *d_codes, const uint8_t *d_exps,
                           size_t n_in, apx_act_desc *d_desc, void *stream) {
  if (!ctx || !d_desc) return APX_ERR_INVALID_ARGUMENT;
  cudaError_t e = launch_describe(d_codes, d_exps, n_in, 1, 0, 0, d_desc, (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_quant_q32_async(apx_ctx *ctx, const int64_t *d_x, size_t n, int8_t *d_codes,
                        uint8_t *d_exps, apx_act_desc *d_desc, void *stream) {
  if (!ctx || !d_desc) return APX_ERR_INVALID_ARGUMENT;
  cudaError_t e = launch_quant_q32((const long long *)d_x, n, d_codes, d_exps, d_desc,
                                   (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_quant_f32_async(apx_ctx *ctx, const float *d_x, size_t n, int8_t *d_codes,
                        uint8_t *d_exps, apx_act_desc *d_desc, void *stream) {
  if (!ctx || !d_desc) return APX_ERR_INVALID_ARGUMENT;
  cudaError_t e = launch_quant_f32(d_x, n, d_codes, d_exps, d_desc, (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_quant_f32_cols_async(apx_ctx *ctx, const float *d_x, size_t n, size_t k_cols,
                             int8_t *d_codes, uint8_t *d_exps, apx_act_desc *d_descs,
                             void *stream) {
  if (!ctx || (k_cols && (!d_descs || (n && (!d_x || !d_codes || !d_exps)))))
    return APX_ERR_INVALID_ARGUMENT;
  if (k_cols > (size_t)INT32_MAX) return APX_ERR_TOO_LARGE;
  const size_t ld = apx_act_padded_len(n);
  cudaError_t e = launch_quant_f32_cols(d_x, n, n, (int)k_cols, d_codes, ld, d_exps, ld / 32,
                                        d_descs, (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_matvec_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                     const int8_t *d_codes, const uint8_t *d_exps, const apx_act_desc *d_desc,
                     int64_t *d_out_q32, float *d_out_f32, apx_call_status *d_status,
                     void *stream) {
  if (!ctx || !d_desc || !d_status) return APX_ERR_INVALID_ARGUMENT;
  Tensor *t;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    t = find(ctx, tensor);
  }
  if (!t || n_in != t->n_in || n_out > t->n_out) return APX_ERR_LAYOUT_MISMATCH;
  cudaError_t e = launch_gemv(t->plan, t->type, t->d_pack, t->d_scratch, n_out, n_in, d_codes, d_exps, d_desc,
                              (long long *)d_out_q32, d_out_f32,
                              (unsigned long long *)&d_status->first, (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

static_assert(APX_MAX_GROUP == kMaxGroup, "group size in the header");

int apx_matvec_group_async(apx_ctx *ctx, const uint64_t *tensors, int count, size_t n_in,
                           const int8_t *d_codes, const uint8_t *d_exps,
                           const apx_act_desc *d_desc, int64_t *const *d_out_q32,
                           float *const *d_out_f32, apx_call_status *const *d_status,
                           void *stream) {
  if (!ctx || !tensors || count < 1 || !d_desc || !d_status) return APX_ERR_INVALID_ARGUMENT;
  Tensor *ts[APX_MAX_GROUP];
  bool one_launch = count <= APX_MAX_GROUP;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    for (int i = 0; i < count; i++) {
      Tensor *t = find(ctx, tensors[i]);
      if (!t || t->n_in != n_in || !d_status[i]) return APX_ERR_LAYOUT_MISMATCH;
      if (i < APX_MAX_GROUP) ts[i] = t;
    }
  }
  // one launch when every member is a one-wave tensor of the first one's family and layout and
  // the concatenated row tiles still plan as one wave without a K split
  GemvPlan pl{};
  if (one_launch) {
    size_t n_rt = 0;
    for (int i = 0; i < count; i++) {
      const Tensor &t = *ts[i];
      one_launch = one_launch && t.d_pack && t.n_out > 0 && !t.plan.pipe &&
                   t.type == ts[0]->type && t.plan.L == ts[0]->plan.L &&
                   t.plan.units == ts[0]->plan.units;
      n_rt += t.plan.n_rt;
    }
    if (one_launch) {
      pl = plan_gemv(ts[0]->type, n_rt * (size_t)(32 / ts[0]->plan.L), n_in, ctx->sm_count);
      one_launch = !pl.pipe && (pl.ksplit == 1 || pl.cluster == pl.ksplit) &&
                   pl.L == ts[0]->plan.L &&
                   pl.units == ts[0]->plan.units && pl.n_rt == n_rt;
    }
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (!one_launch) {  // one launch per tensor
    for (int i = 0; i < count; i++) {
      Tensor *t;
      {
        std::lock_guard<std::mutex> g(ctx->mu);
        t = find(ctx, tensors[i]);
      }
      cudaError_t e = launch_gemv(t->plan, t->type, t->d_pack, t->d_scratch, t->n_out, n_in,
                                  d_codes, d_exps, d_desc,
                                  d_out_q32 ? (long long *)d_out_q32[i] : nullptr,
                                  d_out_f32 ? d_out_f32[i] : nullptr,
                                  (unsigned long long *)&d_status[i]->first, st);
      if (e != cudaSuccess) return APX_ERR_CUDA;
    }
    return APX_OK;
  }
  GemvGroup grp{};
  grp.n = count;
  size_t end = 0;
  for (int i = 0; i < count; i++) {
    end += ts[i]->plan.n_rt;
    grp.pack[i] = ts[i]->d_pack;
    grp.rt_end[i] = end;
    grp.n_out[i] = ts[i]->n_out;
    grp.out_q32[i] = d_out_q32 ? (long long *)d_out_q32[i] : nullptr;
    grp.out_f32[i] = d_out_f32 ? d_out_f32[i] : nullptr;
    grp.status[i] = (unsigned long long *)&d_status[i]->first;
  }
  cudaError_t e = launch_gemv_group(pl, ts[0]->type, grp, n_in, d_codes, d_exps, d_desc, st);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_matmat_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in, size_t k_cols,
                     const int8_t *d_codes, const uint8_t *d_exps, const apx_act_desc *d_descs,
                     int64_t *d_out_q32, float *d_out_f32, apx_call_status *d_status,
                     void *stream) {
  if (!ctx || !d_descs || !d_status) return APX_ERR_INVALID_ARGUMENT;
  Tensor *t;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    t = find(ctx, tensor);
  }
  if (!t || n_in != t->n_in || n_out > t->n_out) return APX_ERR_LAYOUT_MISMATCH;
  const size_t ld = apx_act_padded_len(n_in), ldb = ld / 32;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    const TcRoute route = tc_route(ctx, *t, n_out, n_in, k_cols);
    if (route != kTcNone) {
      if (ensure_gwork(ctx, route, k_cols, n_in, n_out) != cudaSuccess)
        return APX_ERR_OUT_OF_MEMORY;
      cudaError_t e = launch_tc(ctx, *t, route, n_out, n_in, k_cols, d_codes, ld, d_exps, ldb,
                                d_descs, (long long *)d_out_q32, d_out_f32,
                                (unsigned long long *)d_status, (cudaStream_t)stream);
      return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
    }
  }
  for (size_t c = 0; c < k_cols; c++) {
    cudaError_t e = launch_gemv(t->plan, t->type, t->d_pack, t->d_scratch, n_out, n_in, d_codes + c * ld,
                                d_exps + c * ldb, d_descs + c,
                                d_out_q32 ? (long long *)d_out_q32 + c * n_out : nullptr,
                                d_out_f32 ? d_out_f32 + c * n_out : nullptr,
                                (unsigned long long *)&d_status[c].first, (cudaStream_t)stream);
    if (e != cudaSuccess) return APX_ERR_CUDA;
  }
  return APX_OK;
}

int apx_matmat_f32_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                         size_t k_cols, const float *d_x, size_t ldx, int64_t *d_out_q32,
                         float *d_out_f32, apx_call_status *d_status, void *stream) {
  if (!ctx || !d_status || (k_cols && n_in && !d_x) || ldx < n_in)
    return APX_ERR_INVALID_ARGUMENT;
  if (k_cols > (size_t)INT32_MAX) return APX_ERR_TOO_LARGE;
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t || n_in != t->n_in || n_out > t->n_out) return APX_ERR_LAYOUT_MISMATCH;
  if (k_cols == 0) return APX_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const TcRoute route = tc_route(ctx, *t, n_out, n_in, k_cols);
  const bool gemm = route != kTcNone;
  if (gemm && ensure_gwork(ctx, route, k_cols, n_in, n_out) != cudaSuccess)
    return APX_ERR_OUT_OF_MEMORY;
  cudaError_t e;
  if (gemm && tc_f32_ok(route, n_in, d_x, ldx)) {
    e = launch_tc_f32(ctx, *t, route, n_out, n_in, k_cols, d_x, ldx, (long long *)d_out_q32,
                      d_out_f32, (unsigned long long *)d_status, st);
    return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
  }
  const size_t ld = apx_act_padded_len(n_in), ldb = ld / 32;
  const size_t ds_sz = align16(k_cols * sizeof(ActDesc)), ex_sz = align16(k_cols * ldb);
  if (ctx->ascratch.ensure(ds_sz + ex_sz + k_cols * ld) != cudaSuccess)
    return APX_ERR_OUT_OF_MEMORY;
  uint8_t *sc = (uint8_t *)ctx->ascratch.p;
  const ActDesc *descs = (const ActDesc *)sc;
  uint8_t *dexp = sc + ds_sz;
  int8_t *dcod = (int8_t *)(sc + ds_sz + ex_sz);
  e = launch_quant_f32_cols(d_x, n_in, ldx, (int)k_cols, dcod, ld, dexp, ldb, sc, st);
  if (e == cudaSuccess && gemm) {
    e = launch_tc(ctx, *t, route, n_out, n_in, k_cols, dcod, ld, dexp, ldb, descs,
                  (long long *)d_out_q32, d_out_f32, (unsigned long long *)d_status, st);
  } else {
    for (size_t c = 0; e == cudaSuccess && c < k_cols; c++)
      e = launch_gemv(t->plan, t->type, t->d_pack, t->d_scratch, n_out, n_in, dcod + c * ld,
                      dexp + c * ldb, descs + c,
                      d_out_q32 ? (long long *)d_out_q32 + c * n_out : nullptr,
                      d_out_f32 ? d_out_f32 + c * n_out : nullptr,
                      (unsigned long long *)&d_status[c].first, st);
  }
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_swiglu_quant_async(apx_ctx *ctx, const int64_t *d_gate, const int64_t *d_up, size_t n,
                           int carrier, int64_t *d_h, int8_t *d_codes, uint8_t *d_exps,
                           apx_act_desc *d_desc, apx_call_status *d_status, void *stream) {
  if (!ctx || !d_desc || !d_status || (n && (!d_gate || !d_up || !d_codes || !d_exps)) ||
      (carrier != APX_CARRIER_F32 && carrier != APX_CARRIER_Q32))
    return APX_ERR_INVALID_ARGUMENT;
  if (n > (size_t)INT32_MAX) return APX_ERR_TOO_LARGE;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (ctx->fwork.ensure(swiglu_work_bytes(n)) != cudaSuccess) return APX_ERR_OUT_OF_MEMORY;
  if (n == 0) {
    // the empty activation: an all-zero descriptor, as the quantizers write it
    ActDesc d{};
    d.emax = -1;
    return cudaMemcpyAsync(d_desc, &d, sizeof d, cudaMemcpyHostToDevice, (cudaStream_t)stream) ==
                   cudaSuccess && cudaStreamSynchronize((cudaStream_t)stream) == cudaSuccess
               ? APX_OK
               : APX_ERR_CUDA;
  }
  const cudaError_t e = launch_swiglu_quant(
      (const long long *)d_gate, (const long long *)d_up, n, carrier, (long long *)d_h, d_codes,
      d_exps, d_desc, (unsigned long long *)&d_status->first, ctx->fwork.p, (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_matmat_f32_group_async(apx_ctx *ctx, const uint64_t *tensors, int count, size_t n_in,
                               size_t k_cols, const float *d_x, size_t ldx,
                               int64_t *const *d_out_q32, float *const *d_out_f32,
                               apx_call_status *const *d_status, void *stream) {
  if (!ctx || !tensors || count < 1 || count > APX_MAX_GROUP || !d_status ||
      (k_cols && n_in && !d_x) || ldx < n_in)
    return APX_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < count; i++)
    if (!d_status[i]) return APX_ERR_INVALID_ARGUMENT;
  if (k_cols > (size_t)INT32_MAX) return APX_ERR_TOO_LARGE;
  if (k_cols == 0) return APX_OK;
  bool grouped = true;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    Tensor *ts[APX_MAX_GROUP];
    size_t n_out_max = 0;
    for (int i = 0; i < count; i++) {
      ts[i] = find(ctx, tensors[i]);
      if (!ts[i] || ts[i]->n_in != n_in) return APX_ERR_LAYOUT_MISMATCH;
      n_out_max = std::max(n_out_max, ts[i]->n_out);
    }
    // one prep over the activation when every member runs the digit-plane GEMM alike
    for (int i = 0; grouped && i < count; i++) {
      Tensor &t = *ts[i];
      grouped = t.type == ts[0]->type && k_cols >= kGemmMinCols && t.d_pack && t.n_out &&
                limb_shape_ok(n_in);
      if (grouped && !t.limb_tried) {
        t.limb_tried = true;
        if (build_limb_layout(t.plan, t.type, t.d_pack, t.n_out, t.n_in, &t.limb, ctx->stream) !=
            cudaSuccess)
          cudaGetLastError();
      }
      grouped = grouped && t.limb.ok && t.limb.digits == ts[0]->limb.digits;
    }
    grouped = grouped && limb_f32_ok(n_in, d_x, ldx) &&
              ensure_gwork(ctx, kTcLimb, k_cols, n_in, n_out_max) == cudaSuccess;
    if (grouped) {
      LimbMember m[APX_MAX_GROUP];
      for (int i = 0; i < count; i++)
        m[i] = LimbMember{&ts[i]->plan, ts[i]->d_pack, &ts[i]->limb, ts[i]->n_out,
                          d_out_q32 ? (long long *)d_out_q32[i] : nullptr,
                          d_out_f32 ? d_out_f32[i] : nullptr,
                          (unsigned long long *)d_status[i]};
      const cudaError_t e = launch_limb_gemm_f32_group(ts[0]->type, m, count, n_in, k_cols, d_x,
                                                       ldx, ctx->lwork.p, ctx->sm_count,
                                                       (cudaStream_t)stream);
      return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
    }
  }
  // otherwise each member on its own route
  for (int i = 0; i < count; i++) {
    Tensor *t;
    {
      std::lock_guard<std::mutex> g(ctx->mu);
      t = find(ctx, tensors[i]);
    }
    const int rc = apx_matmat_f32_async(ctx, tensors[i], t->n_out, n_in, k_cols, d_x, ldx,
                                        d_out_q32 ? d_out_q32[i] : nullptr,
                                        d_out_f32 ? d_out_f32[i] : nullptr, d_status[i], stream);
    if (rc != APX_OK) return rc;
  }
  return APX_OK;
}

int apx_swiglu_quant_shard_async(apx_ctx *ctx, const int64_t *d_gate, const int64_t *d_up,
                                 size_t n, int carrier, int64_t *d_h, int8_t *d_codes,
                                 uint8_t *d_exps, apx_act_desc *d_desc, int n_peers,
                                 int8_t *const *d_peer_codes, uint8_t *const *d_peer_exps,
                                 apx_act_desc *const *d_peer_desc, apx_call_status *d_status,
                                 void *stream) {
  if (!ctx || !d_desc || !d_status || n == 0 || !d_gate || !d_up || !d_codes || !d_exps ||
      (carrier != APX_CARRIER_F32 && carrier != APX_CARRIER_Q32) || n_peers < 0 ||
      n_peers > APX_PLAN_MAX_PEERS || (n_peers && (!d_peer_codes || !d_peer_exps || !d_peer_desc)))
    return APX_ERR_INVALID_ARGUMENT;
  if (n > (size_t)INT32_MAX) return APX_ERR_TOO_LARGE;
  SwigluDests dests{};
  dests.n = n_peers;
  for (int i = 0; i < n_peers; i++) {
    if (!d_peer_codes[i] || !d_peer_exps[i] || !d_peer_desc[i]) return APX_ERR_INVALID_ARGUMENT;
    dests.codes[i] = d_peer_codes[i];
    dests.exps[i] = d_peer_exps[i];
    dests.desc[i] = d_peer_desc[i];
  }
  std::lock_guard<std::mutex> g(ctx->mu);
  if (ctx->fwork.ensure(swiglu_work_bytes(n)) != cudaSuccess) return APX_ERR_OUT_OF_MEMORY;
  const cudaError_t e = launch_swiglu_quant(
      (const long long *)d_gate, (const long long *)d_up, n, carrier, (long long *)d_h, d_codes,
      d_exps, d_desc, (unsigned long long *)&d_status->first, ctx->fwork.p, (cudaStream_t)stream,
      &dests);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_swiglu_quant_cols_async(apx_ctx *ctx, const int64_t *d_gate, const int64_t *d_up,
                                size_t n, size_t k_cols, int carrier, int64_t *d_h,
                                int8_t *d_codes, uint8_t *d_exps, apx_act_desc *d_descs,
                                apx_call_status *d_status, void *stream) {
  if (!ctx || (k_cols && (!d_descs || !d_status ||
                          (n && (!d_gate || !d_up || !d_codes || !d_exps)))) ||
      (carrier != APX_CARRIER_F32 && carrier != APX_CARRIER_Q32))
    return APX_ERR_INVALID_ARGUMENT;
  if (n > (size_t)INT32_MAX || k_cols > 65535) return APX_ERR_TOO_LARGE;
  if (k_cols == 0) return APX_OK;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (n == 0) {  // empty activations: all-zero descriptors, as the quantizers write them
    std::vector<ActDesc> d(k_cols);
    for (auto &x : d) {
      x = ActDesc{};
      x.emax = -1;
    }
    return cudaMemcpyAsync(d_descs, d.data(), k_cols * sizeof(ActDesc), cudaMemcpyHostToDevice,
                           (cudaStream_t)stream) == cudaSuccess &&
                   cudaStreamSynchronize((cudaStream_t)stream) == cudaSuccess
               ? APX_OK
               : APX_ERR_CUDA;
  }
  if (ctx->fwork.ensure(swiglu_work_bytes(n, k_cols)) != cudaSuccess) return APX_ERR_OUT_OF_MEMORY;
  const size_t ld = apx_act_padded_len(n);
  const cudaError_t e = launch_swiglu_quant_cols(
      (const long long *)d_gate, (const long long *)d_up, n, k_cols, n, carrier,
      (long long *)d_h, d_codes, ld, d_exps, ld / 32, d_descs,
      (unsigned long long *)&d_status->first, ctx->fwork.p, (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_act_describe_cols_async(apx_ctx *ctx, const int8_t *d_codes, const uint8_t *d_exps,
                                size_t n_in, size_t k_cols, apx_act_desc *d_descs,
                                void *stream) {
  if (!ctx || (k_cols && (!d_descs || (n_in && (!d_codes || !d_exps)))))
    return APX_ERR_INVALID_ARGUMENT;
  if (k_cols > (size_t)INT32_MAX) return APX_ERR_TOO_LARGE;
  if (k_cols == 0) return APX_OK;
  const size_t ld = apx_act_padded_len(n_in);
  cudaError_t e = launch_describe(d_codes, d_exps, n_in, (int)k_cols, ld, ld / 32, d_descs,
                                  (cudaStream_t)stream);
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

int apx_ffn_status_decode(const apx_call_status *status, apx_err *err) {
  if (!status) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  const unsigned long long w = status->first;
  if (w == ~0ull) return set_err(err, APX_OK);
  const int code = (int)((w >> 16) & 0xFF);
  set_err(err, code);
  if (err) {
    err->row = w >> 24;
    err->bits = (uint32_t)(w & 0xFFFF);
  }
  return code;
}

int apx_status_decode(apx_ctx *ctx, uint64_t tensor, const apx_call_status *status,
                      apx_err *err) {
  if (!ctx || !status) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  return decode_status(*t, t->n_out, status->first, err);
}

int apx_ctx_set_gemm_route(apx_ctx *ctx, int route) {
  if (!ctx || (route != APX_GEMM_AUTO && route != APX_GEMM_DIGITS && route != APX_GEMM_FOLD))
    return APX_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> g(ctx->mu);
  ctx->gemm_route = route;
  return APX_OK;
}

int apx_status_decode_rows(apx_ctx *ctx, uint64_t tensor, size_t n_out,
                           const apx_call_status *status, apx_err *err) {
  if (!ctx || !status) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> g(ctx->mu);
  Tensor *t = find(ctx, tensor);
  if (!t || n_out > t->n_out) return set_err(err, APX_ERR_INVALID_ARGUMENT);
  return decode_status(*t, n_out, status->first, err);
}

// ---- step plans ------------------------------------------------------------------------------

struct apx_plan {
  apx_ctx *ctx = nullptr;
  PlanHost *host = nullptr;
  std::vector<void *> own;  // the gate / up Q32.32 outputs the caller did not provide
  ~apx_plan() {
    plan_free(host);
    for (void *p : own) cudaFree(p);
  }
};

apx_plan *apx_plan_create(apx_ctx *ctx, const apx_plan_proj *projs, size_t n_proj,
                          const apx_plan_act *acts, size_t n_act, const apx_plan_ffn *ffns,
                          size_t n_ffn, apx_err *err) {
  set_err(err, APX_OK);
  if (!ctx || !projs || n_proj == 0 || (n_act && !acts) || (n_ffn && !ffns) || n_act == 0 ||
      n_proj > (size_t)kPlanMaxProj || n_ffn > (size_t)kPlanMaxFfn || n_act > (size_t)INT32_MAX) {
    set_err(err, APX_ERR_INVALID_ARGUMENT);
    return nullptr;
  }
  auto *plan = new (std::nothrow) apx_plan;
  if (!plan) {
    set_err(err, APX_ERR_OUT_OF_MEMORY);
    return nullptr;
  }
  plan->ctx = ctx;
  PlanSpec s;
  int rc = APX_OK;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    for (size_t i = 0; i < n_proj && rc == APX_OK; i++) {
      const apx_plan_proj &q = projs[i];
      Tensor *t = find(ctx, q.tensor);
      if (!t || !t->d_pack || q.n_in != t->n_in || q.n_out > t->n_out) {
        rc = APX_ERR_LAYOUT_MISMATCH;
        break;
      }
      PlanSpec::Proj p;
      p.type = t->type;
      p.pack = t->d_pack;
      p.plan = t->plan;
      p.n_out = q.n_out;
      p.n_in = q.n_in;
      p.act = q.act;
      p.ffn = q.ffn;
      p.role = q.role;
      p.out_q32 = (long long *)q.d_out_q32;
      p.out_f32 = q.d_out_f32;
      p.status = q.d_status ? (unsigned long long *)&q.d_status->first : nullptr;
      if (q.ffn >= 0 && !p.out_q32 && q.n_out) {  // SwiGLU reads gate and up in Q32.32
        void *buf = nullptr;
        if (cudaMalloc(&buf, q.n_out * sizeof(long long)) != cudaSuccess) {
          cudaGetLastError();
          rc = APX_ERR_OUT_OF_MEMORY;
          break;
        }
        plan->own.push_back(buf);
        p.out_q32 = static_cast<long long *>(buf);
      }
      s.projs.push_back(p);
    }
    for (size_t f = 0; f < n_ffn && rc == APX_OK; f++) {
      PlanSpec::Ffn x;
      x.carrier = ffns[f].carrier;
      x.out_act = ffns[f].out_act;
      x.h = (long long *)ffns[f].d_h;
      x.status = ffns[f].d_status ? (unsigned long long *)&ffns[f].d_status->first : nullptr;
      x.refused = false;
      x.n_peers = ffns[f].n_peers;
      if (x.n_peers < 0 || x.n_peers > APX_PLAN_MAX_PEERS) {
        rc = APX_ERR_INVALID_ARGUMENT;
        break;
      }
      for (int p = 0; p < x.n_peers; p++) {
        x.peer_codes[p] = ffns[f].d_peer_codes[p];
        x.peer_exps[p] = ffns[f].d_peer_exps[p];
        x.peer_desc[p] = ffns[f].d_peer_desc[p];
      }
      if ((x.carrier != APX_CARRIER_F32 && x.carrier != APX_CARRIER_Q32) || !x.status) {
        rc = APX_ERR_INVALID_ARGUMENT;
        break;
      }
      for (size_t i = 0; i < n_proj; i++)  // a non-finite weight row leaves h undefined
        if (projs[i].ffn == (int32_t)f) {
          const Tensor *t = find(ctx, projs[i].tensor);
          x.refused = x.refused || (t && t->nonfinite_row < projs[i].n_out);
        }
      s.ffns.push_back(x);
    }
  }
  for (size_t a = 0; a < n_act && rc == APX_OK; a++) {
    const apx_plan_act &x = acts[a];
    s.acts.push_back(PlanSpec::Act{x.d_codes, x.d_exps, x.d_desc, x.ffn});
    if (x.ffn >= 0 && (size_t)x.ffn < n_ffn && x.d_codes && x.d_exps &&
        !(x.flags & APX_PLAN_ACT_UNPADDED)) {
      // the FFN writes codes [0, n) and exponent bytes [0, ceil(n/32)): the rest of the
      // padded buffers reads as zero blocks
      size_t n = 0;
      for (size_t i = 0; i < n_proj; i++)
        if (projs[i].ffn == x.ffn) n = projs[i].n_out;
      const size_t pad = apx_act_padded_len(n), nb = (n + 31) / 32;
      if (cudaMemset(x.d_codes + n, 0, pad - n) != cudaSuccess ||
          cudaMemset(x.d_exps + nb, 0xFF, pad / 32 - nb) != cudaSuccess) {
        cudaGetLastError();
        rc = APX_ERR_CUDA;
      }
    }
  }
  if (rc == APX_OK) rc = plan_build(s, ctx->sm_count, &plan->host);
  if (rc != APX_OK) {
    delete plan;
    set_err(err, rc);
    return nullptr;
  }
  return plan;
}

int apx_plan_run_async(apx_plan *plan, void *stream) {
  if (!plan || !plan->host) return APX_ERR_INVALID_ARGUMENT;
  const cudaError_t e = plan_run(*plan->host, (cudaStream_t)stream, pdl_allowed());
  return e == cudaSuccess ? APX_OK : APX_ERR_CUDA;
}

void apx_plan_destroy(apx_plan *plan) { delete plan; }

}  // extern "C"
