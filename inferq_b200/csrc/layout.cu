// layout.cu -- GGUF -> device layout conversion, device block decode, and
// activation quantization (Q8_K / Q8_0) with an optional fused RMSNorm.
#include "layout.cuh"
#include "kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__global__ void gguf_to_dev_kernel(int dt, const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                   int64_t rows, int cols) {
  const int nb = cols / gguf_block_elems(dt);
  const int64_t total = rows * nb;
  const int64_t srb = gguf_row_bytes(dt, cols), drb = dev_row_bytes(dt, cols);
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / nb;
    const int b = (int)(t % nb);
    const uint8_t* s = src + r * srb + (int64_t)b * gguf_block_bytes(dt);
    uint8_t* d = dst + r * drb;
    switch (dt) {
      case Q4_K: {
        uint8_t* o = d + (int64_t)b * 144;
        for (int i = 0; i < 16; i++) o[i] = s[i];
        for (int i = 0; i < 128; i++) o[16 + q4k_qs_perm(i)] = s[16 + i];
      } break;
      case Q5_K: {
        uint8_t* o = d + (int64_t)b * 176;
        for (int i = 0; i < 16; i++) o[i] = s[i];
        for (int i = 0; i < 32; i++) o[16 + q5k_qh_perm(i)] = s[16 + i];
        for (int i = 0; i < 128; i++) o[48 + q4k_qs_perm(i)] = s[48 + i];
      } break;
      case Q6_K: {
        uint8_t* o = d + (int64_t)b * 208;
        for (int tig = 0; tig < 4; tig++)
          for (int g = 0; g < 4; g++)
            for (int e = 0; e < 4; e++) {
              const int v3 = q6k_value(s, 16 * (4 * g + 3) + 4 * tig + e);
              for (int j = 0; j < 3; j++)
                o[tig * 48 + g * 12 + 4 * j + e] =
                    (uint8_t)((q6k_value(s, 16 * (4 * g + j) + 4 * tig + e) << 2) | ((v3 >> (2 * j)) & 3));
            }
        for (int i = 0; i < 16; i++) o[192 + i] = s[192 + i];
        d[(int64_t)nb * 208 + 2 * b] = s[208];
        d[(int64_t)nb * 208 + 2 * b + 1] = s[209];
      } break;
      case Q8_0: {
        uint8_t* o = d + (int64_t)(b / 4) * 128;
        for (int i = 0; i < 32; i++) o[q80_perm(b % 4, i)] = s[2 + i];
        d[(int64_t)nb * 32 + 2 * b] = s[0];
        d[(int64_t)nb * 32 + 2 * b + 1] = s[1];
      } break;
      default: {  // F32 / F16: unchanged bytes
        const int bb = gguf_block_bytes(dt);
        for (int i = 0; i < bb; i++) d[(int64_t)b * bb + i] = s[i];
      } break;
    }
  }
}

}  // namespace

namespace {

__global__ void dequant_rows_kernel(int dt, const uint8_t* __restrict__ w, int64_t row_bytes, int cols,
                                    const int32_t* __restrict__ ids, int64_t rows, float* __restrict__ out) {
  const int nb = cols / gguf_block_elems(dt);
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const int64_t src = ids ? ids[r] : r;
    const uint8_t* row = w + src * row_bytes;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < cols; e += gridDim.x * blockDim.x)
      out[r * cols + e] = dev_weight(dt, row, nb, e);
  }
}

}  // namespace

namespace {

// One CTA per input row: optional GGUF RMSNorm (x / sqrt(mean(x^2)+eps) * w,
// src/qwen/quantized_layer.rs:230-236), then quantization to the requested
// activation layouts, and optionally the normalized f32 row itself.
__global__ void __launch_bounds__(256) prep_rows_kernel(PrepArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float xs[];
  const int row = blockIdx.x;
  const float* x = a.x + (int64_t)row * a.ldx;
  const int cols = a.cols;
  if (a.norm_w) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum_256(ss);
    const float var = __fmul_rn(ss, a.inv_cols);
    const float den = sqrtf(__fadd_rn(var, a.eps));
    for (int i = threadIdx.x; i < cols; i += blockDim.x)
      xs[i] = __fmul_rn(__fdiv_rn(x[i], den), a.norm_w[i]);
  } else {
    for (int i = threadIdx.x; i < cols; i += blockDim.x) xs[i] = x[i];
  }
  __syncthreads();
  if (a.xn_out)
    for (int i = threadIdx.x; i < cols; i += blockDim.x) a.xn_out[(int64_t)row * a.ldxn + i] = xs[i];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a.q8k) {
    const int nb = cols / 256;
    uint8_t* ar = a.q8k + (int64_t)row * (a.q8k_stride ? a.q8k_stride : act_row_bytes_q8k(cols));
    for (int b = warp; b < nb; b += 8) quant_q8k_block_warp(xs, ar, nb, b, lane);
  }
  if (a.q80) {
    const int nb = cols / 32;
    uint8_t* ar = a.q80 + (int64_t)row * (a.q80_stride ? a.q80_stride : act_row_bytes_q80(cols));
    for (int g = warp; g < nb / 4; g += 8) quant_q80_group_warp(xs, ar, nb, g, lane);
  }
}

}  // namespace

cudaError_t gguf_to_device(int dt, const uint8_t* src, uint8_t* dst, int64_t rows, int cols, cudaStream_t st) {
  const int64_t total = rows * (cols / gguf_block_elems(dt));
  int grid = (int)std::min<int64_t>(ceil_div(total, 256), 148 * 16);
  if (grid < 1) grid = 1;
  gguf_to_dev_kernel<<<grid, 256, 0, st>>>(dt, src, dst, rows, cols);
  return cudaGetLastError();
}

cudaError_t dequant_rows(int dt, const uint8_t* w, int64_t row_bytes, int cols, const int32_t* ids,
                         int64_t rows, float* out, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(cols, 256), (unsigned)std::min<int64_t>(rows, 65535));
  dequant_rows_kernel<<<grid, 256, 0, st>>>(dt, w, row_bytes, cols, ids, rows, out);
  return cudaGetLastError();
}

cudaError_t prep_rows(const PrepArgs& a, int rows, cudaStream_t st, bool pdl) {
  if (rows <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = a.cols * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, prep_rows_kernel, a);
}

}  // namespace iq
