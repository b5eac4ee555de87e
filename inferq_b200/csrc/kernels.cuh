// kernels.cuh -- declarations shared across the .cu files of libiq.
#pragma once
#include <algorithm>
#include "iq_common.cuh"
#include "qmv.cuh"

namespace iq {

struct PrepArgs {
  const float* x;        // [rows][ldx]
  int ldx;
  int cols;
  const float* norm_w;   // optional RMSNorm weight [cols]
  float eps;
  float inv_cols;
  float* xn_out;         // optional normalized f32 rows
  int ldxn;
  uint8_t* q8k;          // optional Q8_K activation rows
  uint8_t* q80;          // optional Q8_0 activation rows
  int q8k_stride;        // row strides in bytes (0: packed for `cols`)
  int q80_stride;
  // Optional MoE combine applied to x first, written back to x (the hidden
  // rows): x += sum_route y[row*topk + q] * w[row*topk + q] + y_shared[row] *
  // sigmoid(selector logit), in route order (src/qwen/quantized_moe.rs:384-400).
  const float* comb_y;   // [slot][comb_y_ld]: routed slots row*topk+q, shared slot rows*topk+row
  int comb_y_ld;
  const float* comb_w;   // [rows][topk] route weights
  const float* comb_logits;  // selector logit at [row * comb_logits_ld + comb_experts]
  int comb_logits_ld, comb_experts, comb_topk, comb_rows;
};


cudaError_t gguf_to_device(int dt, const uint8_t* src, uint8_t* dst, int64_t rows, int cols, cudaStream_t st);
cudaError_t dequant_rows(int dt, const uint8_t* w, int64_t row_bytes, int cols, const int32_t* ids,
                         int64_t rows, float* out, cudaStream_t st);
cudaError_t prep_rows(const PrepArgs& a, int rows, cudaStream_t st, bool pdl);

// f32 matrix rows (router): y[i*ld + r] = dot(w[r], x[i]); fixed lane order.
// With norm_w set, the input rows are first RMS-normalized (GGUF RMSNorm),
// and with q8k_out also written as Q8_K activation rows (row stride
// q8k_stride bytes) for the quantized matrices that take the same input.
// y[t*ldy + r] = w row r . x row t for n input rows (any n), the f32_matvec
// arithmetic per row (the wide pass's router)
cudaError_t f32_rows(const float* w, int rows, int cols, const float* x, int ldx, int n, float* y, int ldy,
                     cudaStream_t st);
cudaError_t f32_matvec(const float* w, int rows, int cols, const float* x, int ldx, int k, float* y,
                       int ldy, cudaStream_t st, bool pdl, const float* norm_w = nullptr, float eps = 0.f,
                       uint8_t* q8k_out = nullptr, int q8k_stride = 0);

// BF16 matrix rows (row-major bf16 bits): y[i*ldy + r] = sum_c w[r][c] *
// bf16(x[i][c]) with exact products summed in f32; k <= 8, cols % 8 == 0.
cudaError_t bf16_matvec(const uint16_t* w, int rows, int cols, const float* x, int ldx, int k, float* y, int ldy,
                        cudaStream_t st);

// Wide Q8_0 product on the tensor cores (wide.cu): y[t*out_ld + r] for
// ntok input rows x[t*ldx ..]; qx (ntok x cols f16), dT (cols/32 x
// wide_ldd(ntok) f32) and wx (rows x cols f16) are scratch.  cols % 128 == 0.
int wide_ldd(int ntok);
int* wide_timeout_flag();  // device flag: a wide-product wait gave up
// Q4_K / Q5_K x Q8_K wide product (wide.cu); cols % 256 == 0.  Scratch
// carved from one buffer by wide_q4k_scratch_bytes (base NULL: size only;
// q5: with the Q5_K centring tiles).
struct WideQ4kScratch {
  __half* qx;
  float* dT;
  uint8_t* bm;
  __half* wx;
  uint8_t* am;
  uint8_t* ac;  // Q5_K only
};
size_t wide_q4k_scratch_bytes(int64_t rows, int64_t cols, int ntok, WideQ4kScratch* sc, uint8_t* base,
                              bool q5 = false);
// The Q5_K wide product is enabled by the environment variable IQ_WIDE_Q5K.
bool wide_q5k_enabled();
// Q6_K x Q8_K wide product; cols % 256 == 0.
struct WideQ6kScratch {
  __half* qx;
  float* dT;
  __half* lo;
  __half* hi;
};
size_t wide_q6k_scratch_bytes(int64_t rows, int64_t cols, int ntok, WideQ6kScratch* sc, uint8_t* base);
cudaError_t wide_q6k_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, const WideQ6kScratch& sc, cudaStream_t st);
cudaError_t wide_q4k_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, const WideQ4kScratch& sc, cudaStream_t st);
cudaError_t wide_q5k_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, const WideQ4kScratch& sc, cudaStream_t st);
cudaError_t wide_q80_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, __half* qx, float* dT, __half* wx,
                             cudaStream_t st);

}  // namespace iq
