/*
 * iq_oracle.h -- CPU restatement of inferq's speculative-verify arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA path in inferq_b200/csrc.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it; the product never links or calls it.
 *
 * Every function names the reference file:line it restates (paths relative
 * to the ybrs/inferq tree).  Arithmetic that lives in the unvendored
 * candle-core 0.11.0 crate (activation quantization, block decode) is
 * restated from the published GGML block formats and pinned against
 * gguf-py 0.19.0's decoder (tests/golden).
 *
 * Dtype ids are GGML's: F32=0, F16=1, Q8_0=8, Q4_K=12, Q5_K=13, Q6_K=14,
 * Q8_K=15.
 */
#ifndef IQ_ORACLE_H
#define IQ_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q5_K = 13,
       OR_Q6_K = 14, OR_Q8_K = 15, OR_BF16 = 30 };

/* Bytes of one GGUF row of `cols` weights (cols a multiple of the block). */
int64_t or_row_bytes(int dtype, int64_t cols);

/* Exact f16 <-> f32 (round to nearest even). */
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);

/* Block decode of `rows` GGUF rows into f32 (candle to_float order). */
int or_dequant_rows(int dtype, const void* w, int64_t rows, int64_t cols, float* out);

/* candle BlockQ8K::from_float: 292-byte blocks {f32 d; i8 qs[256]; i16 bsums[16]}. */
void or_quant_q8k(const float* x, int64_t cols, void* blocks);
/* candle BlockQ8_0::from_float: 34-byte blocks {f16 d; i8 qs[32]}. */
void or_quant_q80(const float* x, int64_t cols, void* blocks);

/* y[i*rows + r] = row r of w dotted with input row i (x is [k][cols]).
 * order 0: the reference's AVX2 lane order (src/qgemm.rs:175-397).
 * order 1: the device order: exact integer block sums, one f32 FMA per
 *          block inside each of `ksplit` contiguous block chunks, chunks
 *          summed left to right. */
int or_qmatvec(int dtype, const void* w, int64_t rows, int64_t cols,
               const float* x, int k, float* y, int order, int ksplit);

/* Greedy argmax: non-finite skipped, ties to the LAST max index
 * (src/sampling.rs:104-112).  Returns -1 when nothing is finite. */
int64_t or_argmax(const float* v, int64_t n);

/* the wide pass's chunked DeltaNet recurrence over <= 32 rows of one head */
int or_delta_chunk(const float* q, const float* k, const float* v, const float* beta, const float* lg, int C, int dk,
                   int dv, float* S, float* o);
#ifdef __cplusplus
}
#endif
#endif
