/*
 * iq.h -- C ABI of libiq, the B200 (sm_100a) speculative-verify path of
 * inferq.  Every entry point returns 0 on success or a negative IQ_E* code;
 * iq_last_error() then describes the failure (thread-local, mirroring the
 * reference's anyhow messages).  No entry point aborts the process.
 *
 * Plain C types only: pointers, sizes, and opaque handles.  Weight bytes are
 * GGUF blocks exactly as they sit in the file; the library owns every device
 * allocation behind a handle and frees it in the matching *_destroy.
 */
#ifndef IQ_H
#define IQ_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes. */
#define IQ_OK 0
#define IQ_EINVAL (-1)     /* bad argument or shape */
#define IQ_ECUDA (-2)      /* CUDA runtime error */
#define IQ_ENOMEM (-3)     /* device allocation failed */
#define IQ_EUNSUPPORTED (-4)
#define IQ_ESTATE (-5)     /* call order / state violation */
#define IQ_ETIMEDOUT (-6)  /* a bounded device wait gave up */

/* GGML dtype ids accepted by the library. */
#define IQ_F32 0
#define IQ_F16 1
#define IQ_Q8_0 8
#define IQ_Q4_K 12
#define IQ_Q5_K 13
#define IQ_Q6_K 14

/* Where a caller-supplied buffer lives. */
#define IQ_HOST 0
#define IQ_DEVICE 1

/* Message of the last failure on this thread ("" when none). */
const char* iq_last_error(void);

/* Library version string. */
const char* iq_version(void);

/* ------------------------------------------------------------------ */
/* Operator level: one quantized matrix (replaces QuantizedMatrix,     */
/* src/gguf.rs:159-785).                                               */
/* ------------------------------------------------------------------ */
typedef struct iq_matrix iq_matrix;

/* Upload `rows` GGUF rows of `cols` weights (bytes at `data`, in host or
 * device memory per `location`) to the current device in the device layout.
 * Replaces GgufCheckpoint::load_matrix -> QuantizedMatrix::new
 * (src/gguf.rs:1234-1253, :305-330): same dtype set minus BF16. */
int iq_matrix_create(int dtype, const void* data, int64_t rows, int64_t cols, int location,
                     iq_matrix** out);
/* A matrix of the first `rows` rows sharing storage with `m`
 * (QuantizedMatrix::leading_rows, src/gguf.rs:352-377). */
int iq_matrix_leading_rows(const iq_matrix* m, int64_t rows, iq_matrix** out);
void iq_matrix_destroy(iq_matrix* m);
int iq_matrix_shape(const iq_matrix* m, int64_t* rows, int64_t* cols, int* dtype);

/* y[i*rows + r] = row r of m . x[i]   for i < input_rows, host buffers.
 * Replaces QuantizedMatrix::forward_rows (src/gguf.rs:433-456): same
 * argument meaning (row-major f32 in, row-major f32 out), same arithmetic
 * (activations quantized to Q8_K / Q8_0 as candle does, exact integer
 * block dots).  Any input_rows >= 1. */
int iq_matrix_forward_rows(const iq_matrix* m, const float* x, int64_t input_rows, float* y);

/* As iq_matrix_forward_rows with device buffers, enqueued on `stream`
 * (a cudaStream_t, or NULL for the legacy stream).  Input rows <= 8. */
int iq_matrix_forward_device(const iq_matrix* m, const float* x, int input_rows, float* y, void* stream);

/* One-shot form over GGUF bytes in host memory (uploads, multiplies,
 * frees): int iq_qgemv of the boundary table, mirroring forward_rows. */
int iq_qgemv(int dtype, const void* w, int64_t rows, int64_t cols, const float* x, int k, float* y,
             void* stream);

/* The number of contiguous block chunks a row of this shape is split into
 * (a function of the shape only; documents the f32 accumulation order). */
int iq_qgemv_ksplit(int dtype, int64_t rows, int64_t cols);

/* Decode rows of m to f32 (candle to_float order), device -> host copy.
 * `ids` (host, may be NULL) selects rows, as the embedding lookup does
 * (src/gguf.rs:288-290). */
int iq_matrix_dequantize(const iq_matrix* m, const int32_t* ids, int64_t n, float* out);

#ifdef __cplusplus
}
#endif
#endif
