// apx_kernels.h — internal launch interface between the C-ABI runtime and the kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

namespace apx {

struct GemvPlan {
  int units;       // units per row tile
  int L;           // lanes per row (1, 2 or 4); a row tile is 32/L rows
  size_t n_rt;     // row tiles
  int R, P;        // row tiles per CTA, warps per row tile
  int ksplit;      // CTAs per row tile along K
  int cluster;     // ksplit when those CTAs form a thread-block cluster (their partial sums
                   // meet in distributed shared memory), else 0: scratch and arrival counters
  bool pipe;       // persistent streaming kernel (matrices beyond one resident wave)
  long long chunk; // streaming: units per warp
  int kmax;        // streaming: most warps sharing one row tile
  int act_bytes;   // one-wave: shared bytes of activation staging / partial sums
  int w_off;       // one-wave: shared offset of the warps' weight slots (one unit each)
  bool smem_w;     // one-wave: weights in those slots (gemv_kernel_smem), not in registers
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
// Where a row-sharded projection also stores its Q32.32 outputs: this rank's rows in each
// other rank's gather buffer (row 0 of the call at dst[i][0]); n = 0 for an ordinary call.
struct PeerRows {
  int n;
  long long *dst[7];
};
// Up to kMaxGroup tensors of one family and width read by one launch (projections that share
// an activation): row tile rt of the launch is row tile rt - rt_begin(t) of tensor t, where
// rt_end holds the cumulative row-tile counts.  n = 0 for an ordinary launch.
constexpr int kMaxGroup = 4;
struct GemvGroup {
  int n;
  const uint8_t *pack[kMaxGroup];
  size_t rt_end[kMaxGroup];
  size_t n_out[kMaxGroup];
  long long *out_q32[kMaxGroup];
  float *out_f32[kMaxGroup];
  unsigned long long *status[kMaxGroup];
};
// One launch over a group (every tensor planned one-wave with the same lanes per row and units
// per row tile; `pl` planned for the concatenated row tiles, with ksplit 1).
cudaError_t launch_gemv_group(const GemvPlan &pl, uint32_t type, const GemvGroup &grp,
                              size_t n_in, const int8_t *codes, const uint8_t *exps,
                              const void *desc, cudaStream_t stream);
cudaError_t launch_gemv(const GemvPlan &pl, uint32_t type, const uint8_t *pack, void *scratch,
                        size_t n_out, size_t n_in, const int8_t *codes, const uint8_t *exps,
                        const void *desc, long long *out_q32, float *out_f32,
                        unsigned long long *status, cudaStream_t stream,
                        const PeerRows *peers = nullptr);

// Activation kernels (apx_quant.cu).  `cols` activation vectors of width n laid out with
// stride `ld` codes and `ldb` exponent bytes; one descriptor per column.
cudaError_t launch_describe(const int8_t *codes, const uint8_t *exps, size_t n, int cols,
                            size_t ld, size_t ldb, void *desc, cudaStream_t stream);
cudaError_t launch_quant_q32(const long long *x, size_t n, int8_t *codes, uint8_t *exps,
                             void *desc, cudaStream_t stream);
cudaError_t launch_quant_f32(const float *x, size_t n, int8_t *codes, uint8_t *exps, void *desc,
                             cudaStream_t stream);
// `cols` f32 vectors, vector c at x + c·ldx, one CTA each.
cudaError_t launch_quant_f32_cols(const float *x, size_t n, size_t ldx, int cols, int8_t *codes,
                                  size_t ld, uint8_t *exps, size_t ldb, void *desc,
                                  cudaStream_t stream);

// The tcgen05 GEMM's view of a Q8_0 tensor (apx_gemm.cu): row-major codes for TMA, the
// per-(block, row) integer multipliers and per-row smallest exponents, and the 2D tensor
// maps of the codes and the multipliers (CUtensorMap, kept opaque here).
struct GemmLayout {
  void *base = nullptr;
  int8_t *codes = nullptr;  // [m_pad][kp]
  int32_t *wmul = nullptr;  // [nb_pad][m_pad]
  int32_t *kmin = nullptr;  // [m_pad]
  int nb = 0, nb_pad = 0;
  size_t kp = 0, m_pad = 0;
  int kspread = 0;  // largest exponent spread of one row's block scales
  alignas(64) unsigned char map[128];    // the codes, 128-byte boxes × 128 rows
  alignas(64) unsigned char map_m[128];  // wmul, 128 rows × 4 blocks
};

cudaError_t build_gemm_layout(const GemvPlan &pl, const uint8_t *pack, size_t n_out,
                              size_t n_in, GemmLayout *lay, cudaStream_t stream);
void free_gemm_layout(GemmLayout *lay);
// Whether the GEMM can take a tensor of this width / this layout at all.
bool gemm_shape_ok(size_t n_in);
bool gemm_supported(const GemmLayout &lay);
// Device workspace of one call (zeroed once at allocation; its list counters reset themselves).
size_t gemm_work_bytes(size_t n_cols, size_t n_in, size_t n_out, int sm_count);
size_t gemm_work_head_bytes(size_t n_cols);
// Exact k-column Q8_0 projection: column c's codes at codes + c·ld (16-byte aligned, ld a
// multiple of 16, readable up to the 128-byte-padded width), exponent bytes at exps + c·ldb,
// refusal word at status[2c] (initialised to all ones by the caller).  `descs` (one
// ActDesc per column, or null) carries the quantizer's refusals.
cudaError_t launch_gemm_q8_0(const GemvPlan &pl, const uint8_t *pack, const GemmLayout &lay,
                             size_t n_out, size_t n_in, size_t n_cols, const int8_t *codes,
                             size_t ld, const uint8_t *exps, size_t ldb, const void *descs,
                             void *work, long long *out_q32, float *out_f32,
                             unsigned long long *status, int sm_count, cudaStream_t stream);
// The fused f32 prefill: f32_to_fixed + quant_act of every column and the GEMM's prep in one
// kernel, then the GEMM.  gemm_f32_ok: the width and the input's alignment allow it.
bool gemm_f32_ok(size_t n_in, const float *x, size_t ldx);
cudaError_t launch_gemm_q8_0_f32(const GemvPlan &pl, const uint8_t *pack, const GemmLayout &lay,
                                 size_t n_out, size_t n_in, size_t n_cols, const float *x,
                                 size_t ldx, void *work, long long *out_q32, float *out_f32,
                                 unsigned long long *status, int sm_count, cudaStream_t stream);

// The digit-plane GEMM's view of a Q8_0 / Q4_K / Q6_K tensor (apx_lgemm.cu): every weight
// W'[r,i] = w_{r,i} / 2^kmin_r (its Q32.32 value over the row's smallest scale exponent, an
// integer) as three or four balanced base-256 int8 digits [digits][m_pad][kp], kmin per row, and
// the 3D tensor map of the digits.  ok = false when some weight needs more than four digits
// (the tensor then has no such view).
struct LimbLayout {
  void *base = nullptr;
  int8_t *planes = nullptr;  // [digits][m_pad][kp]
  int32_t *kmin = nullptr;   // [m_pad]
  size_t kp = 0, m_pad = 0;
  int digits = 0;  // 3 when every weight fits three digits, else 4
  int wbits = 0;   // bit length of the largest |W'|
  bool ok = false;
  alignas(64) unsigned char map[128];  // the digits, 64-byte boxes × 128 rows × `digits` planes
};

bool limb_shape_ok(size_t n_in);
cudaError_t build_limb_layout(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                              size_t n_out, size_t n_in, LimbLayout *lay, cudaStream_t stream);
void free_limb_layout(LimbLayout *lay);
// Device workspace of one call (nothing in it outlives the call).
size_t limb_work_bytes(size_t n_cols, size_t n_in, size_t n_out, int sm_count);
// Exact k-column projection on the digit planes: the arguments of launch_gemm_q8_0 plus the
// family (the checked columns' rows and the call bound follow it).
cudaError_t launch_limb_gemm(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                             const LimbLayout &lay, size_t n_out, size_t n_in, size_t n_cols,
                             const int8_t *codes, size_t ld, const uint8_t *exps, size_t ldb,
                             const void *descs, void *work, long long *out_q32, float *out_f32,
                             unsigned long long *status, int sm_count, cudaStream_t stream);
// The f32 prefill on the digit planes: f32_to_fixed + quant_act + the digits in one prep kernel.
bool limb_f32_ok(size_t n_in, const float *x, size_t ldx);
cudaError_t launch_limb_gemm_f32(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                                 const LimbLayout &lay, size_t n_out, size_t n_in, size_t n_cols,
                                 const float *x, size_t ldx, void *work, long long *out_q32,
                                 float *out_f32, unsigned long long *status, int sm_count,
                                 cudaStream_t stream);

// Several tensors of one family, each with digit planes of the same digit count, reading one
// activation (q/k/v; gate/up): one quantize-and-digits prep, then each member's GEMM over it.
struct LimbMember {
  const GemvPlan *pl;
  const uint8_t *pack;
  const LimbLayout *lay;
  size_t n_out;
  long long *out_q32;
  float *out_f32;
  unsigned long long *status;
};
cudaError_t launch_limb_gemm_f32_group(uint32_t type, const LimbMember *m, int count,
                                       size_t n_in, size_t n_cols, const float *x, size_t ldx,
                                       void *work, int sm_count, cudaStream_t stream);

// The FFN hidden activation (apx_ffn.cu): SwiGLU under the carrier, then quant_act; `work` holds
// swiglu_work_bytes(n).
size_t swiglu_work_bytes(size_t n, size_t cols = 1);
// Row shards: where else a one-column call's codes, exponent bytes and descriptor go.
struct SwigluDests {
  int n;
  int8_t *codes[7];
  uint8_t *exps[7];
  void *desc[7];  // ActDesc
};
cudaError_t launch_swiglu_quant(const long long *gate, const long long *up, size_t n, int carrier,
                                long long *h, int8_t *codes, uint8_t *exps, void *desc,
                                unsigned long long *status, void *work, cudaStream_t stream,
                                const SwigluDests *dests = nullptr);
// `cols` columns in one launch: gate/up/h of column c at c·ldg, codes at c·ldc, exponent bytes at
// c·lde, descriptor desc[c], status word at status[2c]; `work` holds swiglu_work_bytes(n, cols).
cudaError_t launch_swiglu_quant_cols(const long long *gate, const long long *up, size_t n,
                                     size_t cols, size_t ldg, int carrier, long long *h,
                                     int8_t *codes, size_t ldc, uint8_t *exps, size_t lde,
                                     void *desc, unsigned long long *status, void *work,
                                     cudaStream_t stream, const SwigluDests *dests = nullptr);

// Step plans (apx_plan.cu): the projections of a decode step, and the FFNs among them whose
// finish runs SwiGLU + quant_act, in one persistent launch.  All projections of one plan share a
// family; each reads its tensor in the tensor's own repacked layout (plan = its GemvPlan).
constexpr int kPlanMaxProj = 4096, kPlanMaxFfn = 64;
struct PlanCtl {  // zero between launches (the launch's last warp resets it)
  unsigned queue, exit, abort, pad;
  unsigned ready[kPlanMaxFfn];   // blocks of the FFN's h quantized
  unsigned flag[kPlanMaxFfn];    // the FFN's descriptor published
  int stats[kPlanMaxFfn][4];     // [2]: the FFN's refusal (max); the rest spare
};
struct PlanSpec {
  struct Proj {
    uint32_t type;
    const uint8_t *pack;
    GemvPlan plan;
    size_t n_out, n_in;
    int act, ffn, role;  // ffn: -1 or the FFN this projection feeds as gate (0) or up (1)
    long long *out_q32;
    float *out_f32;
    unsigned long long *status;
  };
  struct Act {
    const int8_t *codes;
    const uint8_t *exps;
    const void *desc;  // ActDesc
    int ffn;           // -1: ready when the launch starts; else the FFN that writes it
  };
  struct Ffn {
    int carrier, out_act;
    long long *h;                // or null
    unsigned long long *status;  // the first refusing SwiGLU lane
    bool refused;                // gate or up holds a non-finite scale below the width
    int n_peers;                 // copies of the quantized blocks and the descriptor
    int8_t *peer_codes[7];
    uint8_t *peer_exps[7];
    void *peer_desc[7];          // ActDesc
  };
  std::vector<Proj> projs;
  std::vector<Act> acts;
  std::vector<Ffn> ffns;
};
struct PlanHost;
int plan_build(const PlanSpec &s, int sm_count, PlanHost **out);  // an APX_ERR_* code
cudaError_t plan_run(const PlanHost &h, cudaStream_t stream, bool pdl);
void plan_free(PlanHost *h);

// GEMV launches from the calling thread go without programmatic dependent launch while set.
void set_pdl_suppressed(bool on);
// Whether a launch from this thread may carry programmatic dependent launch now.
bool pdl_allowed();

// Debug: exact int32 group dots from the repacked layout (apx_gemv.cu).
cudaError_t launch_block_dots(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                              size_t n_out, size_t n_in, const int8_t *codes, int32_t *dots,
                              cudaStream_t stream);

}  // namespace apx
