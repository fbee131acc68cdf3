/*
 * apx_oracle.h — CPU restatement of apeiron's integer Q8-activation projection.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker of the CUDA backend:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / `--impl reference`
 * leg load it.  The product library (apeiron_b200/csrc) never links or calls it.
 *
 * Parity pin: tests/test_oracle_golden.py checks these functions against every
 * known-answer value the reference's own tests assert for this path (chart/tests.rs,
 * kern/pow2.rs tests, kern/native_gpu_probe.rs populations and counts).
 *
 * Activation arguments use the reference's `QuantAct` form: scales as int64
 * (0 or 2^e) and codes as int8 (src/engine/chart/mod.rs:67-81).
 */
#ifndef APX_ORACLE_H
#define APX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/apeiron_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* round_shift_32 of a 128-bit value given as (hi, lo); src/engine/num/value.rs:10-12. */
void apxo_round_shift_32(int64_t hi, uint64_t lo, int64_t *out_hi, uint64_t *out_lo);
/* f16 -> Q32.32, 0 ok / APX_ERR_NONFINITE_SCALE; src/engine/num/dequant.rs:25-42. */
int apxo_f16_to_fixed(uint16_t h, int64_t *out);
/* f16 -> (m, k) with value m * 2^k; 0 ok / 1 non-finite; src/engine/kern/pow2.rs:52-64. */
int apxo_f16_split(uint16_t h, int32_t *m, uint32_t *k);
/* Smallest power of two S with 127*S >= absmax; 0 ok / 1 None; pow2.rs:22-39. */
int apxo_act_scale(uint64_t absmax, uint64_t *s);
/* round_shift_32(acc * 2^s) in i64; 0 ok / 1 None; pow2.rs:76-96. */
int apxo_finish(int64_t acc, uint32_t s, int64_t *out);
/* round(v * 2^32) half away from zero; 0 ok / 1 None; src/engine/num/fp.rs:186-230. */
int apxo_f32_to_q32(uint32_t bits, int64_t *out);

/* quant_act: 0 ok / 1 None.  codes[n], scales[ceil(n/32)]; chart/mod.rs:258-334. */
int apxo_quant_act(const int64_t *x, size_t n, int8_t *codes, int64_t *scales);
/* QuantAct::dequant: 0 ok / 1 None; chart/mod.rs:188-212. */
int apxo_dequant_act(const int8_t *codes, size_t n, const int64_t *scales,
                     size_t n_scales, int64_t *out);

/* Row dequantizer to Q32.32 (src/engine/num/dequant.rs:99-129 dispatch). */
int apxo_dequant_row(uint32_t ggml_type, const uint8_t *row, size_t row_len,
                     size_t n_elems, int64_t *out, apx_err *err);

/* matvec_fixed (src/engine/ops/matvec.rs:149-222). */
int apxo_matvec_fixed(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                      size_t n_out, size_t n_in, const int64_t *x, size_t x_len,
                      int64_t *out, apx_err *err);

/* matvec_q8act (src/engine/chart/mod.rs:1887-1925), the fused-row restatement. */
int apxo_matvec_q8act(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                      size_t n_out, size_t n_in, const int8_t *codes, size_t q_len,
                      const int64_t *scales, size_t n_scales, int64_t *out,
                      apx_err *err);

/* matvec_q8act_quant_chunked's validation order (src/engine/chart/ffn.rs:667-745). */
int apxo_matvec_q8act_chunked(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                              size_t n_out, size_t n_in, const int8_t *codes,
                              size_t q_len, const int64_t *scales, size_t n_scales,
                              size_t chunks, int64_t *out, apx_err *err);

/* matmat_q8act: per-column contract, lowest refusing column (kern/matmat.rs:92-134). */
int apxo_matmat_q8act(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                      size_t n_out, size_t n_in, size_t k_cols, const int8_t *codes,
                      size_t q_len, const int64_t *scales, int64_t *out, apx_err *err);

/* exact_dot (src/engine/kern/gemm.rs:470-486): Q8_0 row of `blocks` blocks against a
 * whole-block activation; 0 ok / 1 None. */
int apxo_exact_dot_q8_0(const uint8_t *row, size_t blocks, const int8_t *codes,
                        const int64_t *scales, int64_t *out);

/* Exact int32 group dots per (row, group), group order as the decoders emit them
 * (chart/mod.rs:554-938): 32-lane groups for Q8_0/Q4_K, 16-lane for Q6_K.
 * codes must hold ceil(n_in/qk)*qk entries (zero beyond n_in). */
int apxo_block_dots(uint32_t ggml_type, const uint8_t *raw, size_t n_out,
                    size_t n_in, const int8_t *codes, int32_t *dots);

/* CPU baseline: matvec_q8act over `threads` contiguous row chunks (ffn.rs:667-745). */
int apxo_matvec_q8act_mt(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                         size_t n_out, size_t n_in, const int8_t *codes,
                         const int64_t *scales, int threads, int64_t *out,
                         apx_err *err);
/* CPU baseline: matmat_q8act over `threads` contiguous row chunks. */
int apxo_matmat_q8act_mt(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                         size_t n_out, size_t n_in, size_t k_cols,
                         const int8_t *codes, const int64_t *scales, int threads,
                         int64_t *out, apx_err *err);

/* The timed CPU baseline's vector rows (apx_oracle_x86.c, the reference's AVX2 / AVX-VNNI
 * row cores, src/engine/chart/x86.rs:782-1200): the same results as the *_mt calls above,
 * with Q8_0 (whole blocks) and Q4_K (whole super-blocks) rows two at a time in vector code
 * when the CPU has AVX2; every other shape takes the scalar fast rows. */
int apxo_matvec_q8act_simd_mt(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                              size_t n_out, size_t n_in, const int8_t *codes,
                              const int64_t *scales, int threads, int64_t *out,
                              apx_err *err);
int apxo_matmat_q8act_simd_mt(uint32_t ggml_type, const uint8_t *raw, size_t raw_len,
                              size_t n_out, size_t n_in, size_t k_cols,
                              const int8_t *codes, const int64_t *scales, int threads,
                              int64_t *out, apx_err *err);
/* Bit 0: AVX2 (the vector rows run); bit 1: AVX-VNNI (they use vpdpbusd, and Q8_0 matmats
 * run the k-column GEMM of src/engine/kern/gemm.rs:498-580). */
int apxo_simd_features(void);
/* Matmat calls the k-column GEMM completed, and (row, group) pairs it sent to the exact i128
 * dot, since the library loaded (for the tests). */
void apxo_gemm_counts(uint64_t *calls, uint64_t *exact_groups);
/* The same for the k-column Q4_K kernel (src/engine/chart/kcols.rs:1406-1464), which Q4_K
 * matmats on whole super-blocks run with AVX2. */
void apxo_q4k_counts(uint64_t *calls, uint64_t *exact_groups);
/* And for the k-column Q6_K kernel (kcols.rs:1466-1518). */
void apxo_q6k_counts(uint64_t *calls, uint64_t *exact_groups);
/* Matmat calls the Q8_0 column runs of 16 (kern/matmat.rs:198-206, the path without AVX-VNNI)
 * completed. */
void apxo_kcols_counts(uint64_t *calls);

/* The FFN hidden activation (src/engine/chart/ffn.rs:246-284, ops/silu.rs:53-100,
 * numeric/fixed_exp.rs:1-184, mixer/f32_carrier.rs:262-375). */
int apxo_fixed_exp(int64_t x, int64_t *out);
int apxo_silu_fixed(int64_t v, int64_t *out);
uint32_t apxo_exp_f32(uint32_t x);
uint32_t apxo_silu_f32(uint32_t x);
int apxo_swiglu(int64_t gate, int64_t up, int carrier, int64_t *out);

#ifdef __cplusplus
}
#endif

#endif
