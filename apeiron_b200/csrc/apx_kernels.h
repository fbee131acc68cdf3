// apx_kernels.h — internal launch interface between the C-ABI runtime and the kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace apx {

struct GemvPlan {
  int units;       // units per row tile
  int L;           // lanes per row (1, 2 or 4); a row tile is 32/L rows
  size_t n_rt;     // row tiles
  int R, P;        // row tiles per CTA, warps per row tile
  int ksplit;      // CTAs per row tile along K
  bool pipe;       // persistent streaming kernel (matrices beyond one resident wave)
  long long chunk; // streaming: units per warp
  int kmax;        // streaming: most warps sharing one row tile
  int act_bytes;   // one-wave: shared bytes of activation staging / partial sums
  unsigned grid;
  int block;
  size_t smem;
};

// K-slots per row: quads of Q8_0 blocks, or k-quant super-blocks.
int units_per_row_tile(uint32_t type, size_t n_in);
size_t packed_bytes(const GemvPlan &pl, uint32_t type);
cudaError_t launch_repack(const GemvPlan &pl, const uint8_t *d_raw, uint8_t *d_pack,
                          uint32_t type, size_t n_out, size_t n_in, size_t row_bytes,
                          cudaStream_t stream);
GemvPlan plan_gemv(uint32_t type, size_t n_out, size_t n_in, int sm_count);
// Per-tensor device scratch of a K-split plan (partial sums + arrival counters, zeroed once).
size_t gemv_scratch_bytes(const GemvPlan &pl);
cudaError_t launch_gemv(const GemvPlan &pl, uint32_t type, const uint8_t *pack, void *scratch,
                        size_t n_out, size_t n_in, const int8_t *codes, const uint8_t *exps,
                        const void *desc, long long *out_q32, float *out_f32,
                        unsigned long long *status, cudaStream_t stream);

// Activation kernels (apx_quant.cu).  `cols` activation vectors of width n laid out with
// stride `ld` codes and `ldb` exponent bytes; one descriptor per column.
cudaError_t launch_describe(const int8_t *codes, const uint8_t *exps, size_t n, int cols,
                            size_t ld, size_t ldb, void *desc, cudaStream_t stream);
cudaError_t launch_quant_q32(const long long *x, size_t n, int8_t *codes, uint8_t *exps,
                             void *desc, cudaStream_t stream);
cudaError_t launch_quant_f32(const float *x, size_t n, int8_t *codes, uint8_t *exps, void *desc,
                             cudaStream_t stream);

// Debug: exact int32 group dots from the repacked layout (apx_gemv.cu).
cudaError_t launch_block_dots(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                              size_t n_out, size_t n_in, const int8_t *codes, int32_t *dots,
                              cudaStream_t stream);

}  // namespace apx
