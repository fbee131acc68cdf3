/*
 * apeiron_cuda.h — C ABI of the B200 (sm_100a) backend for apeiron's integer
 * Q8-activation projection: the decode GEMV `matvec_q8act` and the prefill GEMM
 * `matmat_q8act` over GGUF Q8_0 / Q5_0 / Q4_K / Q6_K weight payloads (Q5_0 runs as Q8_0:
 * its five-bit codes widen exactly at upload), and the FFN hidden activation between them.
 *
 * Every exact entry point returns, bit for bit, what the reference's CPU kernel
 * returns: `matvec_fixed(W, dequant(q))` in Q32.32 (`i64` words worth v / 2^32),
 * or the same refusal.  Plain pointers and sizes only; no torch or CUDA types.
 *
 * Reference interfaces (paths inside the apeiron tree):
 *   matvec_q8act                src/engine/chart/mod.rs:1887-1925
 *   matvec_q8act_quant_chunked  src/engine/chart/ffn.rs:667-745
 *   matmat_q8act                src/engine/kern/matmat.rs:134-200
 *   quant_act / QuantAct        src/engine/chart/mod.rs:67-334
 *   MatvecError                 src/engine/ops/matvec.rs:11-48
 *   f32_to_fixed                src/engine/num/f32_convert.rs:44-49
 *   PayloadRef / resident()     src/engine/loader.rs:421-434, :1469
 *
 * Activation encoding.  A reference `QuantAct` is `{scales: Vec<i64>, codes: Vec<i8>}`
 * with every scale 0 or a power of two 2^e, e <= 62 (`act_scale`,
 * src/engine/kern/pow2.rs:22-39).  Across this ABI a scale travels as its
 * exponent byte: `exps[b] = e` for S_b = 2^e and `exps[b] = APX_EXP_ZERO` for S_b = 0.
 *
 * Threading.  One context per thread of control: calls on one context are
 * serialised by an internal mutex (the engine calls from its pool's dispatching
 * thread, src/engine/chart/pool.rs:895-905).  Synchronous entry points return
 * after the result is in the caller's host buffer.
 */
#ifndef APEIRON_CUDA_H
#define APEIRON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define APX_API __attribute__((visibility("default")))
#else
#define APX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids the backend serves (src/format/quant.rs:27-37). */
#define APX_GGML_TYPE_Q8_0 8u
#define APX_GGML_TYPE_Q5_0 6u  /* served as Q8_0: its codes widen exactly at upload */
#define APX_GGML_TYPE_Q4_K 12u
#define APX_GGML_TYPE_Q6_K 14u

/* Exponent byte of a zero activation scale. */
#define APX_EXP_ZERO 0xFFu

/* Status codes.  1..9 mirror `MatvecError` (src/engine/ops/matvec.rs:11-48). */
typedef enum apx_status {
  APX_OK = 0,
  APX_ERR_SHAPE_MISMATCH = 1,       /* ShapeMismatch { x = a, n_in = b }            */
  APX_ERR_ROW_LENGTH = 2,           /* RowLength (unreachable for served families)  */
  APX_ERR_SHORT_PAYLOAD = 3,        /* ShortPayload { need = a, have = b }          */
  APX_ERR_LENGTH_OVERFLOW = 4,      /* LengthOverflow                               */
  APX_ERR_UNSUPPORTED_QUANT = 5,    /* UnsupportedQuant { ggml_type }               */
  APX_ERR_NONFINITE_SCALE = 6,      /* Dequant(NonFiniteScale { bits })             */
  APX_ERR_FIXED_OVERFLOW = 7,       /* Dequant(FixedOverflow)                       */
  APX_ERR_ACCUMULATOR_OVERFLOW = 8, /* AccumulatorOverflow                          */
  APX_ERR_OUTPUT_OVERFLOW = 9,      /* OutputOverflow                               */
  APX_ERR_QUANT_REFUSED = 10,       /* quant_act / f32_to_fixed returned None       */
  APX_ERR_SWIGLU_REFUSED = 11,      /* SwiGLU refused lane `row` (bits: FfnError kind, 3 = Overflow) */
  /* Backend conditions with no reference counterpart. */
  APX_ERR_INVALID_ARGUMENT = 20,    /* null pointer, unknown handle, bad size       */
  APX_ERR_LAYOUT_MISMATCH = 21,     /* call geometry differs from the upload's      */
  APX_ERR_CUDA = 22,                /* CUDA runtime error, code in cuda_error       */
  APX_ERR_OUT_OF_MEMORY = 23,
  APX_ERR_TOO_LARGE = 24,           /* a size beyond a documented backend maximum   */
  APX_ERR_DEVICE_TIMEOUT = 25       /* a bounded device-side wait gave up            */
} apx_status;

/* Refusal detail.  Field meaning depends on `code` as noted in apx_status. */
typedef struct apx_err {
  int32_t code;       /* apx_status */
  uint32_t ggml_type; /* UnsupportedQuant                                  */
  uint64_t a;         /* ShapeMismatch.x, ShortPayload.need                */
  uint64_t b;         /* ShapeMismatch.n_in, ShortPayload.have             */
  uint64_t row;       /* first refusing output row (kernel-side refusals)  */
  uint64_t col;       /* refusing column of a matmat call                  */
  uint32_t bits;      /* NonFiniteScale.bits                               */
  int32_t cuda_error; /* cudaError_t when code == APX_ERR_CUDA             */
} apx_err;

typedef struct apx_ctx apx_ctx;

/* Per-call activation descriptor, produced on the device by apx_act_describe_async /
 * apx_quant_*_async and read by the projection kernels.  Layout is part of the ABI
 * so callers can allocate it; its contents are private. */
typedef struct apx_act_desc {
  uint32_t words[8];
} apx_act_desc;

/* Per-call refusal word written by the asynchronous projections (device memory).
 * Decode with apx_status_decode after the stream is synchronised. */
typedef struct apx_call_status {
  unsigned long long first; /* (row << 24) | (kind << 16) | bits, minimum over rows */
  unsigned long long spare;
} apx_call_status;

/* ---- context ---------------------------------------------------------------- */

/* Which tensor-core GEMM a Q8_0 multi-column call takes.  APX_GEMM_AUTO (the default): the
 * per-block fold GEMM below 6e9 multiply-adds per call (faster there on B200), the digit-plane
 * GEMM above; APX_GEMM_DIGITS / APX_GEMM_FOLD: that GEMM whenever the tensor has its view.  The
 * results are the same bits on every route; K-quant tensors always take the digit planes. */
#define APX_GEMM_AUTO 0
#define APX_GEMM_DIGITS 1
#define APX_GEMM_FOLD 2
APX_API int apx_ctx_set_gemm_route(apx_ctx *ctx, int route);

/* Open a backend context on CUDA device `device`.  Returns NULL on failure. */
APX_API apx_ctx *apx_open(int device, apx_err *err);
/* Free every device buffer the context owns. */
APX_API void apx_close(apx_ctx *ctx);
/* The backend's version string. */
APX_API const char *apx_version(void);

/* ---- weights ------------------------------------------------------------------ */

/* Upload one projection's weight payload and repack it once for the kernels.
 * `raw` is the borrowed `&resident()[at.off .. at.off + at.len]` slice the engine
 * passes to matvec_q8act (src/engine/step.rs:346-378).  Validation follows
 * matvec_fixed (src/engine/ops/matvec.rs:149-178): UnsupportedQuant, LengthOverflow,
 * ShortPayload { need = n_out * row_bytes, have = raw_len }.  Non-finite block
 * scales are found here, once, and reported by every later call exactly where the
 * reference reports them. */
APX_API int apx_tensor_upload(apx_ctx *ctx, uint32_t ggml_type, const uint8_t *raw,
                      size_t raw_len, size_t n_out, size_t n_in, uint64_t *handle,
                      apx_err *err);
/* Release an uploaded tensor. */
APX_API int apx_tensor_free(apx_ctx *ctx, uint64_t handle);
/* Device bytes held by an uploaded tensor: the repacked payload and row metadata, plus the
 * tensor-core views a multi-column call builds (the weight digit planes: 4 bytes per weight;
 * or the Q8_0 fold view). */
APX_API size_t apx_tensor_device_bytes(apx_ctx *ctx, uint64_t handle);

/* ---- synchronous drop-in entry points (host buffers) ----------------------------- */

/* The decode contract (replaces matvec_q8act, src/engine/chart/mod.rs:1887).
 * codes: q_len int8 activation codes; exps: ceil(q_len/32) exponent bytes;
 * out: n_out Q32.32 words.  Refusals in the reference's order. */
APX_API int apx_matvec_q8act(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                     const int8_t *codes, size_t q_len, const uint8_t *exps,
                     int64_t *out, apx_err *err);

/* Same result as apx_matvec_q8act with the validation order of the chunked caller
 * (replaces matvec_q8act_quant_chunked, src/engine/chart/ffn.rs:667-745).  `chunks`
 * is the CPU row-task count; the device kernel's decomposition does not depend on it. */
APX_API int apx_matvec_q8act_chunked(apx_ctx *ctx, uint64_t tensor, size_t n_out,
                             size_t n_in, const int8_t *codes, size_t q_len,
                             const uint8_t *exps, size_t chunks, int64_t *out,
                             apx_err *err);

/* The prefill contract (replaces matmat_q8act, src/engine/kern/matmat.rs:134).
 * k_cols activation columns; column c has codes[c*q_len ..] and exps[c*ceil(q_len/32) ..].
 * out is column-major: out[c*n_out + r].  The call refuses with the lowest refusing
 * column's refusal (err->col). */
APX_API int apx_matmat_q8act(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                     size_t k_cols, const int8_t *codes, size_t q_len,
                     const uint8_t *exps, int64_t *out, apx_err *err);

/* quant_act on the device (src/engine/chart/mod.rs:258-334): Q32.32 in, codes and
 * exponent bytes out.  APX_ERR_QUANT_REFUSED where the reference returns None. */
APX_API int apx_quant_act(apx_ctx *ctx, const int64_t *x, size_t n, int8_t *codes,
                  uint8_t *exps, apx_err *err);

/* f32 boundary: y = from_q32(matvec_q8act(W, quant_act(f32_to_fixed(x)))).
 * x: n_in floats, y: n_out floats, each the Q32.32 result rounded once to f32. */
APX_API int apx_matvec_f32(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                   const float *x, float *y, apx_err *err);

/* f32 boundary of the prefill contract: k_cols columns of n_in floats (column c at
 * x[c*n_in ..]) to column-major y[c*n_out + r]; column c of y equals apx_matvec_f32 of
 * column c.  Q8_0 tensors with at least 4 columns run on the int8 tensor cores.  Refuses
 * with the lowest refusing column (err->col). */
APX_API int apx_matmat_f32(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                   size_t k_cols, const float *x, float *y, apx_err *err);

/* Parity hook: the exact int32 group dots the kernels form, one per (row, group)
 * in group order (32-lane groups for Q8_0/Q4_K, 16-lane groups for Q6_K). */
APX_API int apx_debug_block_dots(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                         const int8_t *codes, int32_t *dots, apx_err *err);

/* ---- asynchronous device-buffer entry points ----------------------------------- */

/* Validate device-resident codes/exps and fill the descriptor (device kernel). */
APX_API int apx_act_describe_async(apx_ctx *ctx, const int8_t *d_codes,
                           const uint8_t *d_exps, size_t n_in, apx_act_desc *d_desc,
                           void *stream);
/* Device quant_act of a Q32.32 vector. */
APX_API int apx_quant_q32_async(apx_ctx *ctx, const int64_t *d_x, size_t n, int8_t *d_codes,
                        uint8_t *d_exps, apx_act_desc *d_desc, void *stream);
/* Device f32_to_fixed + quant_act of an f32 vector. */
APX_API int apx_quant_f32_async(apx_ctx *ctx, const float *d_x, size_t n, int8_t *d_codes,
                        uint8_t *d_exps, apx_act_desc *d_desc, void *stream);
/* Exact projection of device activations; d_out_q32 and/or d_out_f32 may be NULL.
 * d_status receives the refusal word (apx_status_decode).  Buffers padded by the
 * caller: d_codes holds apx_act_padded_len(n_in) bytes (zero beyond n_in). */
APX_API int apx_matvec_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                     const int8_t *d_codes, const uint8_t *d_exps,
                     const apx_act_desc *d_desc, int64_t *d_out_q32, float *d_out_f32,
                     apx_call_status *d_status, void *stream);
/* Device f32_to_fixed + quant_act of k_cols f32 vectors (vector c at d_x[c*n ..]);
 * codes of column c at d_codes[c*apx_act_padded_len(n) ..], exponent bytes at
 * d_exps[c*apx_act_padded_len(n)/32 ..], descriptor d_descs[c]. */
APX_API int apx_quant_f32_cols_async(apx_ctx *ctx, const float *d_x, size_t n, size_t k_cols,
                             int8_t *d_codes, uint8_t *d_exps, apx_act_desc *d_descs,
                             void *stream);
/* Exact k-column projection of device activations (column-major outputs), column c
 * laid out as apx_quant_f32_cols_async writes it; d_status[c] is column c's refusal
 * word, set to all ones by the caller.  Q8_0 tensors with at least 4 columns run on
 * the int8 tensor cores; those calls share a context workspace, so calls on one
 * context must not overlap in time. */
APX_API int apx_matmat_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                     size_t k_cols, const int8_t *d_codes, const uint8_t *d_exps,
                     const apx_act_desc *d_descs, int64_t *d_out_q32,
                     float *d_out_f32, apx_call_status *d_status, void *stream);
/* The f32 prefill on device buffers: k_cols columns of n_in floats (column c at
 * d_x[c*ldx ..]) through f32_to_fixed + quant_act and the exact projection, column c equal
 * to apx_matvec_f32 of column c; d_status[c] as for apx_matmat_async.  Q8_0 tensors with
 * at least 4 columns, d_x 16-byte aligned, ldx a multiple of 4 and n_in <= 16384 quantize
 * inside the GEMM's prep kernel; other calls quantize into a context buffer first.  Shares
 * the context workspace as apx_matmat_async does. */
APX_API int apx_matmat_f32_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                                 size_t k_cols, const float *d_x, size_t ldx,
                                 int64_t *d_out_q32, float *d_out_f32,
                                 apx_call_status *d_status, void *stream);
/* The FFN hidden activation between gate/up and down (replaces the SwiGLU and quantization
 * stages of fused_ffn_task, src/engine/chart/ffn.rs:1577-1594): h_i = swiglu(gate_i, up_i) under
 * the carrier (APX_CARRIER_F32: SiLU in binary32 with the reference's exp, the engine's default,
 * mixer/f32_carrier.rs:262-375; APX_CARRIER_Q32: silu_fixed on fixed_exp in Q32.32,
 * ops/silu.rs:53), then quant_act(h) into codes / exponent bytes / descriptor laid out as
 * apx_quant_f32_async writes them (d_codes zero beyond n, as for the other quantizers).  d_h
 * (optional) receives h.  d_status (all ones on entry) receives the lowest refusing lane
 * (decode with apx_ffn_status_decode); the descriptor then refuses the activation, so a
 * projection that reads it refuses too.  Shares a context workspace with the other calls of
 * its context, which must not overlap in time. */
#define APX_CARRIER_F32 0
#define APX_CARRIER_Q32 1
APX_API int apx_swiglu_quant_async(apx_ctx *ctx, const int64_t *d_gate, const int64_t *d_up,
                                   size_t n, int carrier, int64_t *d_h, int8_t *d_codes,
                                   uint8_t *d_exps, apx_act_desc *d_desc,
                                   apx_call_status *d_status, void *stream);
/* apx_swiglu_quant_async over k_cols columns in one launch (the prefill side of the FFN: the
 * hidden activation of every token between the gate/up and down projections): column c of gate,
 * up and d_h (optional) at c*n (the column-major outputs of apx_matmat_async), codes at
 * d_codes[c*apx_act_padded_len(n) ..], exponent bytes at d_exps[c*apx_act_padded_len(n)/32 ..],
 * descriptor d_descs[c], status word d_status[c] (all ones on entry) — the layout
 * apx_quant_f32_cols_async writes, which apx_matmat_async reads.  Each column equals
 * apx_swiglu_quant_async of that column. */
APX_API int apx_swiglu_quant_cols_async(apx_ctx *ctx, const int64_t *d_gate, const int64_t *d_up,
                                        size_t n, size_t k_cols, int carrier, int64_t *d_h,
                                        int8_t *d_codes, uint8_t *d_exps, apx_act_desc *d_descs,
                                        apx_call_status *d_status, void *stream);
/* apx_act_describe_async over k_cols device columns laid out as apx_quant_f32_cols_async writes
 * them (codes of column c at d_codes[c*apx_act_padded_len(n_in) ..], exponent bytes at
 * d_exps[c*apx_act_padded_len(n_in)/32 ..]): for activations assembled on the device, e.g. the
 * slices of a row-sharded hidden activation gathered from every rank. */
APX_API int apx_act_describe_cols_async(apx_ctx *ctx, const int8_t *d_codes,
                                        const uint8_t *d_exps, size_t n_in, size_t k_cols,
                                        apx_act_desc *d_descs, void *stream);
/* A host copy of apx_swiglu_quant_async's status word into err (APX_OK, or
 * APX_ERR_SWIGLU_REFUSED with the lane in err->row and the FfnError kind in err->bits). */
APX_API int apx_ffn_status_decode(const apx_call_status *status, apx_err *err);
/* Several projections that read the same device activation (q/k/v of a layer, gate/up of a
 * FFN), each over its whole tensor: out[i] = matvec(tensors[i], x), refusal word in
 * d_status[i] (all ones on entry).  Up to APX_MAX_GROUP tensors of one family whose layout
 * allows it run as ONE launch over their concatenated row tiles; otherwise one launch each.
 * d_out_q32 / d_out_f32 are arrays of `count` device pointers (either array may be NULL). */
#define APX_MAX_GROUP 4
APX_API int apx_matvec_group_async(apx_ctx *ctx, const uint64_t *tensors, int count,
                                   size_t n_in, const int8_t *d_codes, const uint8_t *d_exps,
                                   const apx_act_desc *d_desc, int64_t *const *d_out_q32,
                                   float *const *d_out_f32, apx_call_status *const *d_status,
                                   void *stream);
/* Activation buffer length (bytes of codes) the async kernels read for width n_in. */
APX_API size_t apx_act_padded_len(size_t n_in);
/* Decode a refusal word (host copy of *d_status) together with the tensor's
 * upload-time findings into err; returns err->code.  For a call over all of the tensor's
 * rows; a call over its first n_out rows decodes with apx_status_decode_rows. */
APX_API int apx_status_decode(apx_ctx *ctx, uint64_t tensor, const apx_call_status *status,
                      apx_err *err);
/* apx_status_decode for a call that projected the tensor's first n_out rows: an Inf/NaN
 * block scale found at upload counts only when its row is below n_out (the rows the call
 * computed), as apx_matvec_q8act decides for the same n_out. */
APX_API int apx_status_decode_rows(apx_ctx *ctx, uint64_t tensor, size_t n_out,
                                   const apx_call_status *status, apx_err *err);

/* The prefill of several tensors reading one activation (q/k/v; gate/up: gemm_q8_0_group,
 * src/engine/kern/gemm.rs:818, for every family): member i's whole rows, k_cols f32 columns of
 * d_x as apx_matmat_f32_async takes them, outputs d_out_q32[i] / d_out_f32[i] (either array may
 * be NULL, or hold NULL) and refusal words d_status[i][c] (all ones on entry).  When every
 * member has digit planes of one family and digit count, the activation is quantized into its
 * digits once and each member's GEMM reads them; otherwise the members run one by one.  Each
 * member's results equal its own apx_matmat_f32_async.  count <= APX_MAX_GROUP. */
APX_API int apx_matmat_f32_group_async(apx_ctx *ctx, const uint64_t *tensors, int count,
                                       size_t n_in, size_t k_cols, const float *d_x, size_t ldx,
                                       int64_t *const *d_out_q32, float *const *d_out_f32,
                                       apx_call_status *const *d_status, void *stream);

/* apx_swiglu_quant_async for one slice of a row-sharded FFN's h: the codes, exponent bytes and
 * descriptor also go to n_peers other places (other GPUs' buffers, mapped with apx_peer_open),
 * element 0 of the slice at d_peer_codes[i][0] / d_peer_exps[i][0]; a publication
 * (apx_gather_publish_async with desc_off) makes them visible and merges the slices'
 * descriptors.  n_peers <= APX_PLAN_MAX_PEERS. */
APX_API int apx_swiglu_quant_shard_async(apx_ctx *ctx, const int64_t *d_gate,
                                         const int64_t *d_up, size_t n, int carrier,
                                         int64_t *d_h, int8_t *d_codes, uint8_t *d_exps,
                                         apx_act_desc *d_desc, int n_peers,
                                         int8_t *const *d_peer_codes,
                                         uint8_t *const *d_peer_exps,
                                         apx_act_desc *const *d_peer_desc,
                                         apx_call_status *d_status, void *stream);

/* ---- step plans: the projections of a decode step in one launch -------------------- */
/* A plan lists projections in dependency order, each reading one activation record, and
 * optionally FFNs: the gate and up projections of one activation (role APX_PLAN_GATE /
 * APX_PLAN_UP) whose finish runs SwiGLU + quant_act into an activation record that later
 * projections (down) read.  apx_plan_run_async runs the whole plan as one persistent launch;
 * every projection's outputs and refusal word are those of apx_matvec_async on the same inputs,
 * every FFN's activation and refusal word those of apx_swiglu_quant_async on the gate and up
 * outputs.  The plan replaces the per-projection calls of a decode step's projection schedule
 * (step_proj_sched, src/engine/step.rs:1458; ffn_q8act_prepared_into, chart/ffn.rs:1609): same
 * results, one launch, each projection's weights streaming while earlier ones finish.
 *
 * All tensors of a plan share a family (Q5_0 counts as Q8_0).  Records hold device pointers
 * that must stay valid while the plan exists; activation buffers follow apx_act_padded_len.
 * Status words (projections and FFNs) are set to all ones by the caller before each run.  A
 * projection reading an FFN's activation comes after both of that FFN's projections; it waits
 * for the activation on the device (bounded: about one second, then APX_ERR_DEVICE_TIMEOUT).
 * Runs of one plan must not overlap in time (the plan owns its counters and scratch). */
typedef struct apx_plan apx_plan;
#define APX_PLAN_GATE 0
#define APX_PLAN_UP 1
#define APX_PLAN_MAX_PEERS 7
#define APX_PLAN_ACT_UNPADDED 1 /* apx_plan_act.flags: an FFN's slice inside a larger buffer */
typedef struct apx_plan_act {
  int8_t *d_codes;      /* apx_act_padded_len(n) code bytes */
  uint8_t *d_exps;      /* apx_act_padded_len(n) / 32 exponent bytes */
  apx_act_desc *d_desc; /* its descriptor */
  int32_t ffn;          /* -1: written before the run; else the FFN that writes it (the plan
                         * then sets the pad bytes past n once, at creation, unless flags
                         * holds APX_PLAN_ACT_UNPADDED) */
  int32_t flags;
} apx_plan_act;
typedef struct apx_plan_proj {
  uint64_t tensor;
  size_t n_out, n_in;        /* the first n_out rows (decode with apx_status_decode_rows) */
  int32_t act;               /* the activation record it reads */
  int32_t ffn;               /* -1, or the FFN it feeds */
  int32_t role;              /* APX_PLAN_GATE or APX_PLAN_UP when ffn >= 0 */
  int32_t reserved;
  int64_t *d_out_q32;        /* optional (an FFN's gate and up get plan-owned ones) */
  float *d_out_f32;          /* optional */
  apx_call_status *d_status; /* required */
} apx_plan_proj;
typedef struct apx_plan_ffn {
  int32_t carrier;           /* APX_CARRIER_F32 or APX_CARRIER_Q32 */
  int32_t out_act;           /* the activation record it writes */
  int64_t *d_h;              /* optional: h in Q32.32 */
  apx_call_status *d_status; /* the first refusing SwiGLU lane (apx_ffn_status_decode) */
  /* Row shards: copies of every quantized block of h and of the descriptor also go to
   * n_peers other places (other GPUs' buffers, mapped with apx_peer_open): codes at
   * d_peer_codes[i][row], exponent bytes at d_peer_exps[i][row / 32], the descriptor of this
   * slice to d_peer_desc[i].  A publication (apx_gather_publish_async with desc_off) makes
   * them visible and merges the slices' descriptors. */
  int32_t n_peers;
  int32_t reserved;
  int8_t *d_peer_codes[APX_PLAN_MAX_PEERS];
  uint8_t *d_peer_exps[APX_PLAN_MAX_PEERS];
  apx_act_desc *d_peer_desc[APX_PLAN_MAX_PEERS];
} apx_plan_ffn;
/* NULL with err set on failure: APX_ERR_LAYOUT_MISMATCH (a tensor or width), APX_ERR_
 * INVALID_ARGUMENT (records: families differ, an FFN without one gate and one up of equal
 * shape and activation, a reader before its FFN, more than 4096 projections or 64 FFNs). */
APX_API apx_plan *apx_plan_create(apx_ctx *ctx, const apx_plan_proj *projs, size_t n_proj,
                                  const apx_plan_act *acts, size_t n_act,
                                  const apx_plan_ffn *ffns, size_t n_ffn, apx_err *err);
APX_API int apx_plan_run_async(apx_plan *plan, void *stream);
APX_API void apx_plan_destroy(apx_plan *plan);

/* ---- allocation-free entry point ------------------------------------------------ */

/* Widest activation the allocation-free entry point accepts, and the size of the fixed
 * device array it stages in (descriptor, exponent bytes, int8 codes). */
#define APX_NOALLOC_MAX_N_IN 65536u
#define APX_NOALLOC_SCRATCH_BYTES (256u + APX_NOALLOC_MAX_N_IN / 32u + APX_NOALLOC_MAX_N_IN)

/* apx_matvec_f32 for callers that cannot allocate device memory on the call path: an engine
 * that reserves its whole HBM budget at start-up, a process held to a fixed GPU memory
 * quota, a decode loop that cannot take an allocation's latency or failure.  It has no
 * counterpart in the reference (whose CPU kernels allocate freely).
 *
 * Same result as apx_matvec_f32 (f32_to_fixed + quant_act on the device, the exact
 * projection, one rounding to f32), on device buffers: d_x holds n_in floats, d_y receives
 * n_out floats, *d_status the refusal word (decode with apx_status_decode_rows for the same
 * n_out after the stream has finished).  The call is asynchronous on `stream` and allocates nothing: the quantized
 * activation is staged in one array of APX_NOALLOC_SCRATCH_BYTES compiled into the library,
 * which every GPU that loads the library holds until the process exits.
 *   - n_in above APX_NOALLOC_MAX_N_IN is refused with APX_ERR_TOO_LARGE.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress);
 *     make that first call before any stream capture.  The address is kept until the process
 *     exits: a cudaDeviceReset of that device invalidates it (with every context on it).
 *   - The caller's current device is left as it was.
 *   - Every call on a device shares the one array and it keeps the last call's contents:
 *     calls whose kernels overlap on the GPU (other streams, other host threads) race.
 *     Serialise them on one stream.
 * The tensor itself is uploaded beforehand with apx_tensor_upload (which does allocate). */
APX_API int apx_matvec_f32_noalloc(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                                   const float *d_x, float *d_y, apx_call_status *d_status,
                                   void *stream);

/* ---- row-sharded projections across the GPUs of one node ------------------------------
 *
 * A projection's rows are independent, so P processes (one per GPU) can each hold a row range
 * of W and project it; every rank then needs the whole output vector.  These calls move it
 * over NVLink with plain peer stores, without a collective library: each rank owns one gather
 * buffer that every other rank maps (CUDA IPC); apx_matvec_gather_async projects this rank's
 * rows and its kernel stores every output row into this rank's slice of every rank's buffer;
 * apx_gather_publish_async then posts this rank's refusal keys and an epoch flag in every
 * buffer and waits (bounded) for every rank's flag.  The output area and the keys are
 * double-buffered by epoch parity, so a rank that runs ahead never overwrites what another is
 * still reading.  The epoch (1, 2, ...) lives in each rank's
 * own buffer and advances on the device, so the calls can be captured in a CUDA graph and
 * replayed.  The caller (apeiron_b200/shard.py) owns the buffer layout and alternates the
 * parity; every rank must make the same calls in the same order. */

#define APX_MAX_PEERS 8
#define APX_MAX_GATHER_PROJ 4
#define APX_PEER_HANDLE_BYTES 64

/* A zeroed device buffer of `bytes` on ctx's GPU that other processes can map; *d_ptr gets
 * its address, `handle` the bytes to pass to apx_peer_open in those processes. */
APX_API int apx_peer_alloc(apx_ctx *ctx, size_t bytes, void **d_ptr,
                           unsigned char handle[APX_PEER_HANDLE_BYTES], apx_err *err);
/* Map another process's apx_peer_alloc buffer on ctx's GPU (peer access over NVLink). */
APX_API int apx_peer_open(apx_ctx *ctx, const unsigned char handle[APX_PEER_HANDLE_BYTES],
                          void **d_ptr, apx_err *err);
/* Release a buffer: one this process allocated (opened = 0) or mapped (opened = 1). */
APX_API int apx_peer_close(apx_ctx *ctx, void *d_ptr, int opened);
/* Synchronous copy of `bytes` from device memory on ctx's GPU to host memory. */
APX_API int apx_device_read(apx_ctx *ctx, const void *d_src, void *host_dst, size_t bytes,
                            apx_err *err);
/* Synchronous copy of `bytes` from host memory to device memory on ctx's GPU. */
APX_API int apx_device_write(apx_ctx *ctx, void *d_dst, const void *host_src, size_t bytes,
                             apx_err *err);

/* One publication: rank `rank` of `world` makes its rows of `nproj` projections visible in
 * every rank's gather buffer and collects every rank's refusal.  Offsets are bytes from each
 * buffer's base (the same layout on every rank); the refusal words are this rank's
 * apx_call_status words of the projections (device; reset to all ones here). */
typedef struct apx_gather_desc {
  int world, rank, nproj;
  unsigned timeout_us;                   /* bound on the wait for the other ranks' flags  */
  void *peer[APX_MAX_PEERS];             /* every rank's gather buffer (own one included)  */
  size_t out_off;                        /* this parity's output area (int64 elements)     */
  size_t key_off;                        /* this parity's keys: [world][nproj] int64       */
  size_t flag_off;                       /* the flags: [world] uint64, epoch of each rank  */
  size_t ctr_off;                        /* this rank's epoch and check-in count (2 uint64,
                                            read only in its own buffer; zero at alloc)    */
  size_t rows_off[APX_MAX_GATHER_PROJ];  /* element of this rank's first row of proj. j   */
  size_t rows[APX_MAX_GATHER_PROJ];      /* this rank's rows of projection j               */
  long long row0[APX_MAX_GATHER_PROJ];   /* whole-tensor row of this rank's first row      */
  long long nf_key[APX_MAX_GATHER_PROJ]; /* this rank's first non-finite scale as a word,
                                            INT64_MAX for none                              */
  apx_call_status *status[APX_MAX_GATHER_PROJ];     /* this rank's refusal words (device)  */
  apx_call_status *out_status[APX_MAX_GATHER_PROJ]; /* the first refusal over all ranks, in
                                                       whole-tensor rows; APX_ERR_DEVICE_TIMEOUT
                                                       when a rank's flag did not arrive    */
  size_t bytes;                          /* size of every rank's gather buffer: the rows, keys,
                                            flags and counters of the offsets above must lie
                                            inside it (else APX_ERR_INVALID_ARGUMENT)        */
  size_t desc_off;                       /* 0, or this parity's [world] apx_act_desc: each
                                            rank's descriptor of its slice of a sharded
                                            activation (stored by an apx_plan_ffn's peer
                                            destinations); after the wait the publication
                                            merges them into one descriptor at merged_off   */
  size_t merged_off;                     /* (16-byte aligned, as desc_off)                  */
} apx_gather_desc;

/* Projection j of the publication on `stream`: this rank's gd->rows[j] rows (the tensor holds
 * exactly them) from device activations, each Q32.32 output stored into every rank's buffer at
 * element rows_off[j] + row of the area at out_off, the refusal word into gd->status[j]. */
APX_API int apx_matvec_gather_async(apx_ctx *ctx, uint64_t tensor, size_t n_out, size_t n_in,
                                    const int8_t *d_codes, const uint8_t *d_exps,
                                    const apx_act_desc *d_desc, const apx_gather_desc *gd,
                                    int j, void *stream);
/* Queue the publication on `stream` after the group's apx_matvec_gather_async calls (it waits
 * for them on the device).  Work that follows on `stream` sees every rank's rows. */
APX_API int apx_gather_publish_async(apx_ctx *ctx, const apx_gather_desc *gd, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* APEIRON_CUDA_H */
