// dense.cu -- f32 matrix rows against up to eight input rows (the router,
// whose GGUF tensor is F32 and which the reference multiplies in f32,
// src/qwen/quantized_moe.rs:253).  One warp per weight row; lane l sums the
// float4 at columns 4l + 128t in order of t, then a butterfly over lanes.
#include <cuda_bf16.h>
#include "kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__global__ void __launch_bounds__(256) f32_matvec_kernel(const float* __restrict__ w, int rows, int cols,
                                                         const float* __restrict__ x, int ldx, int k,
                                                         float* __restrict__ y, int ldy, const float* norm_w,
                                                         float eps, float inv_cols, uint8_t* q8k_out,
                                                         int q8k_stride) {
  // the weight rows do not depend on the previous kernel: request them first
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  const int c4 = cols / 4;
  constexpr int kMaxPer = 32;  // float4 per lane: cols <= 4096
  float4 wv[kMaxPer];
  if (r < rows) {
    const float4* wr = reinterpret_cast<const float4*>(w + (int64_t)r * cols);
#pragma unroll
    for (int j = 0; j < kMaxPer; j++)
      if (lane + 32 * j < c4) wv[j] = __ldg(wr + lane + 32 * j);
  }
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 xs4[];  // [k][cols/4]
#pragma unroll 4
  for (int i = threadIdx.x; i < k * c4; i += 256) {
    const int rr = i / c4, c = i % c4;
    xs4[i] = *reinterpret_cast<const float4*>(x + (int64_t)rr * ldx + 4 * c);
  }
  __syncthreads();
  if (norm_w) {  // GGUF RMSNorm of the staged rows (same order as the GEMV prologue)
    __shared__ float den[8];
    const float* xs = reinterpret_cast<const float*>(xs4);
    if (warp < k) {
      float ss = 0.f;
      for (int i = lane; i < cols; i += 32) ss = fmaf(xs[warp * cols + i], xs[warp * cols + i], ss);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0) den[warp] = sqrtf(__fadd_rn(__fmul_rn(ss, inv_cols), eps));
    }
    __syncthreads();
    float* xw = reinterpret_cast<float*>(xs4);
    for (int i = threadIdx.x; i < k * cols; i += 256)
      xw[i] = __fmul_rn(__fdiv_rn(xw[i], den[i / cols]), norm_w[i % cols]);
    __syncthreads();
    if (q8k_out) {
      // the normalized rows quantized to Q8_K for the matrices that follow
      // (the (row, block) pairs shared out over every warp of the grid)
      const int nb = cols / 256;
      for (int p = blockIdx.x * 8 + warp; p < k * nb; p += gridDim.x * 8) {
        const int row = p / nb, b = p % nb;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = xw[row * cols + b * 256 + q8k_lane_pos(lane, i)];
        quant_q8k_block_warp_v(v, q8k_out + (int64_t)row * q8k_stride, nb, b, lane);
      }
    }
  }
  if (r >= rows) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPer; j++) {
    if (lane + 32 * j >= c4) break;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (i < k) {
        const float4 xv = xs4[i * c4 + lane + 32 * j];
        float t = acc[i];
        t = fmaf(wv[j].x, xv.x, t);
        t = fmaf(wv[j].y, xv.y, t);
        t = fmaf(wv[j].z, xv.z, t);
        t = fmaf(wv[j].w, xv.w, t);
        acc[i] = t;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (i >= k) break;
    float v = acc[i];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    if (lane == 0) y[(int64_t)i * ldy + r] = v;
  }
}

// Many input rows (the wide pass): the same per-row arithmetic as
// f32_matvec_kernel (lane l sums the float4 at columns 4l + 128t in order of
// t with fused multiply-adds, then the butterfly), with a CTA's 8 weight rows
// held in registers while its 64 input rows pass through shared memory in
// groups of 8.  Grid: (weight rows / 8, input rows / 64).
__global__ void __launch_bounds__(256) f32_rows_kernel(const float* __restrict__ w, int rows, int cols,
                                                      const float* __restrict__ x, int ldx, int n,
                                                      float* __restrict__ y, int ldy) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  const int c4 = cols / 4;
  constexpr int kMaxPer = 32;  // float4 per lane: cols <= 4096
  float4 wv[kMaxPer];
  if (r < rows) {
    const float4* wr = reinterpret_cast<const float4*>(w + (int64_t)r * cols);
#pragma unroll
    for (int j = 0; j < kMaxPer; j++)
      if (lane + 32 * j < c4) wv[j] = __ldg(wr + lane + 32 * j);
  }
  extern __shared__ float4 xs4[];  // [8][cols/4]
  const int g1 = min(n, (int)(blockIdx.y + 1) * 64);
  for (int g = blockIdx.y * 64; g < g1; g += 8) {
    const int k = min(8, g1 - g);
    __syncthreads();
    // eight loads in flight per thread before their stores
    for (int i0 = threadIdx.x; i0 < k * c4; i0 += 256 * 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = i0 + 256 * u;
        if (i < k * c4) v[u] = *reinterpret_cast<const float4*>(x + (int64_t)(g + i / c4) * ldx + 4 * (i % c4));
      }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (i0 + 256 * u < k * c4) xs4[i0 + 256 * u] = v[u];
    }
    __syncthreads();
    if (r >= rows) continue;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPer; j++) {
      if (lane + 32 * j >= c4) break;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        if (i < k) {
          const float4 xv = xs4[i * c4 + lane + 32 * j];
          float t = acc[i];
          t = fmaf(wv[j].x, xv.x, t);
          t = fmaf(wv[j].y, xv.y, t);
          t = fmaf(wv[j].z, xv.z, t);
          t = fmaf(wv[j].w, xv.w, t);
          acc[i] = t;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (i >= k) break;
      float v = acc[i];
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
      if (lane == 0) y[(int64_t)(g + i) * ldy + r] = v;
    }
  }
}

// One warp per weight row; the k input rows are staged rounded to bf16 (as
// f32); each lane sums its columns' exact products in column order, then the
// lanes combine in a fixed tree.
__global__ void __launch_bounds__(256) bf16_matvec_kernel(const uint16_t* __restrict__ w, int rows, int cols,
                                                         const float* __restrict__ x, int ldx, int k,
                                                         float* __restrict__ y, int ldy) {
  extern __shared__ float xb[];  // [k][cols]
  for (int i = threadIdx.x; i < k * cols; i += 256) {
    const int rr = i / cols, c = i % cols;
    xb[i] = __bfloat162float(__float2bfloat16_rn(x[(int64_t)rr * ldx + c]));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= rows) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const uint16_t* wr = w + (int64_t)r * cols;
  for (int c = 8 * lane; c < cols; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(wr + c);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const float wf = __uint_as_float(e & 1 ? (u[e / 2] & 0xffff0000u) : (u[e / 2] << 16));
#pragma unroll
      for (int i = 0; i < 8; i++)
        if (i < k) acc[i] = fmaf(wf, xb[i * cols + c + e], acc[i]);  // the product is exact
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    if (i >= k) break;
    float v = acc[i];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    if (lane == 0) y[(int64_t)i * ldy + r] = v;
  }
}

}  // namespace

cudaError_t bf16_matvec(const uint16_t* w, int rows, int cols, const float* x, int ldx, int k, float* y, int ldy,
                        cudaStream_t st) {
  if (cols % 8 || k < 1 || k > 8 || (size_t)k * cols * sizeof(float) > 200 * 1024 || ((uintptr_t)w & 15))
    return cudaErrorInvalidValue;
  static bool configured[64] = {};
  static std::mutex mu;
  const cudaError_t e = once_per_device(configured, mu, [] {
    return cudaFuncSetAttribute(bf16_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (e != cudaSuccess) return e;
  bf16_matvec_kernel<<<(unsigned)ceil_div(rows, 8), 256, (size_t)k * cols * sizeof(float), st>>>(w, rows, cols, x,
                                                                                                ldx, k, y, ldy);
  return cudaGetLastError();
}

cudaError_t f32_matvec(const float* w, int rows, int cols, const float* x, int ldx, int k, float* y, int ldy,
                       cudaStream_t st, bool pdl, const float* norm_w, float eps, uint8_t* q8k_out, int q8k_stride) {
  if (cols % 4 || cols > 4096 || k < 1 || k > 8 || (q8k_out && (!norm_w || cols % 256))) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  static std::mutex mu;
  const cudaError_t e = once_per_device(configured, mu, [] {
    return cudaFuncSetAttribute(f32_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 4096 * 4);
  });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.dynamicSmemBytes = (size_t)k * cols * sizeof(float);
  cfg.gridDim = dim3((unsigned)ceil_div(rows, 8));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, f32_matvec_kernel, w, rows, cols, x, ldx, k, y, ldy, norm_w, eps,
                            (float)(1.0 / (double)cols), q8k_out, q8k_stride);
}

cudaError_t f32_rows(const float* w, int rows, int cols, const float* x, int ldx, int n, float* y, int ldy,
                     cudaStream_t st) {
  if (cols % 4 || cols > 4096 || n < 1 || rows < 1 || ((uintptr_t)x & 15) || ldx % 4) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  static std::mutex mu;
  const cudaError_t e = once_per_device(configured, mu, [] {
    return cudaFuncSetAttribute(f32_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 4096 * 4);
  });
  if (e != cudaSuccess) return e;
  f32_rows_kernel<<<dim3((unsigned)ceil_div(rows, 8), (unsigned)ceil_div(n, 64)), 256, (size_t)8 * cols * 4, st>>>(
      w, rows, cols, x, ldx, n, y, ldy);
  return cudaGetLastError();
}

}  // namespace iq
