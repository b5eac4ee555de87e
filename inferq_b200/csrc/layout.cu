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
// activation layouts, and optionally the normalized f32 row itself.  Every
// load of the row (and of the norm weight) is issued before the reduction.
template <int MAXB>
__global__ void __launch_bounds__(256) prep_rows_kernel(PrepArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[8];
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* x = a.x + (int64_t)row * a.ldx;
  const int nb = (a.cols + 255) / 256;
  float v[MAXB][8], w[MAXB][8];
#pragma unroll
  for (int j = 0; j < MAXB; j++)
    if (warp + 8 * j < nb) {
      ld_q8k_lane(x, warp + 8 * j, lane, v[j], a.cols);
      if (a.norm_w) ld_q8k_lane(a.norm_w, warp + 8 * j, lane, w[j], a.cols);
    }
  if (a.comb_y) {
    // the MoE combine of this row, element by element as moe_combine does:
    // r = sum_q y_q * w_q (route order), h += r + y_shared * sigmoid(sel)
    const float sl = a.comb_logits[(int64_t)row * a.comb_logits_ld + a.comb_experts];
    const float selector = __fdiv_rn(1.f, __fadd_rn(1.f, exp_ref(-sl)));
    const float* ysh = a.comb_y + (int64_t)(a.comb_rows * a.comb_topk + row) * a.comb_y_ld;
#pragma unroll
    for (int j = 0; j < MAXB; j++) {
      const int b = warp + 8 * j;
      if (b >= nb) continue;
      // every route's values requested before the ordered sum
      constexpr int kMaxTopk = 16;
      float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, ys[8], yq[kMaxTopk][8], wq[kMaxTopk];
#pragma unroll
      for (int q = 0; q < kMaxTopk; q++)
        if (q < a.comb_topk) {
          wq[q] = a.comb_w[row * a.comb_topk + q];
          ld_q8k_lane(a.comb_y + (int64_t)(row * a.comb_topk + q) * a.comb_y_ld, b, lane, yq[q], a.cols);
        }
      ld_q8k_lane(ysh, b, lane, ys, a.cols);
#pragma unroll
      for (int q = 0; q < kMaxTopk; q++)
        if (q < a.comb_topk)
#pragma unroll
          for (int i = 0; i < 8; i++) r[i] = __fadd_rn(r[i], __fmul_rn(yq[q][i], wq[q]));
#pragma unroll
      for (int i = 0; i < 8; i++) v[j][i] = __fadd_rn(v[j][i], __fadd_rn(r[i], __fmul_rn(ys[i], selector)));
      if (b * 256 + 32 * (lane & 7) < a.cols) {
        float* p = const_cast<float*>(x) + b * 256 + 32 * (lane & 7) + 4 * (lane >> 3);
        *reinterpret_cast<float4*>(p) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
        *reinterpret_cast<float4*>(p + 16) = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
      }
    }
  }
  if (a.norm_w) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < MAXB; j++)
      if (warp + 8 * j < nb)
#pragma unroll
        for (int i = 0; i < 8; i++) ss = fmaf(v[j][i], v[j][i], ss);
    ss = cta_sum256(ss, red);
    const float den = sqrtf(__fadd_rn(__fmul_rn(ss, a.inv_cols), a.eps));
#pragma unroll
    for (int j = 0; j < MAXB; j++)
#pragma unroll
      for (int i = 0; i < 8; i++) v[j][i] = __fmul_rn(__fdiv_rn(v[j][i], den), w[j][i]);
  }
  uint8_t* q8k = a.q8k ? a.q8k + (int64_t)row * (a.q8k_stride ? a.q8k_stride : act_row_bytes_q8k(a.cols)) : nullptr;
  uint8_t* q80 = a.q80 ? a.q80 + (int64_t)row * (a.q80_stride ? a.q80_stride : act_row_bytes_q80(a.cols)) : nullptr;
  finish_row<MAXB>(v, nb, a.cols, q8k, q80, a.xn_out ? a.xn_out + (int64_t)row * a.ldxn : nullptr, xs);
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
  cfg.dynamicSmemBytes = (a.q80 || a.xn_out) ? a.cols * sizeof(float) : 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  // 16-byte row vectors: Q8_K rows of 256-element blocks, Q8_0 / f32 rows of 128
  const int nb = (a.cols + 255) / 256;
  auto a16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (a.cols % (a.q8k ? 256 : 128) || a.ldx % 4 || !a16(a.x) || (a.norm_w && !a16(a.norm_w)) ||
      (a.xn_out && (a.ldxn % 4 || !a16(a.xn_out))) ||
      (a.comb_y && (a.comb_y_ld % 4 || !a16(a.comb_y) || a.comb_topk > 16 || a.cols % 256)))
    return cudaErrorInvalidValue;
  if (nb <= 8) return cudaLaunchKernelEx(&cfg, prep_rows_kernel<1>, a);
  if (nb <= 16) return cudaLaunchKernelEx(&cfg, prep_rows_kernel<2>, a);
  if (nb <= 32) return cudaLaunchKernelEx(&cfg, prep_rows_kernel<4>, a);
  if (nb <= 64) return cudaLaunchKernelEx(&cfg, prep_rows_kernel<8>, a);
  return cudaErrorInvalidValue;
}

}  // namespace iq
