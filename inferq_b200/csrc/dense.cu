// dense.cu -- f32 matrix rows against up to eight input rows (the router,
// whose GGUF tensor is F32 and which the reference multiplies in f32,
// src/qwen/quantized_moe.rs:253).  One warp per weight row; lane l sums the
// float4 at columns 4l + 128t in order of t, then a butterfly over lanes.
#include "kernels.cuh"

namespace iq {
namespace {

__global__ void __launch_bounds__(256) f32_matvec_kernel(const float* __restrict__ w, int rows, int cols,
                                                         const float* __restrict__ x, int ldx, int k,
                                                         float* __restrict__ y, int ldy) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 xs4[];  // [k][cols/4]
  const int c4 = cols / 4;
  for (int i = threadIdx.x; i < k * c4; i += 256) {
    const int r = i / c4, c = i % c4;
    xs4[i] = *reinterpret_cast<const float4*>(x + (int64_t)r * ldx + 4 * c);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= rows) return;
  const float4* wr = reinterpret_cast<const float4*>(w + (int64_t)r * cols);
  constexpr int kMaxPer = 32;  // float4 per lane: cols <= 4096
  float4 wv[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; j++)
    if (lane + 32 * j < c4) wv[j] = __ldg(wr + lane + 32 * j);
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

}  // namespace

cudaError_t f32_matvec(const float* w, int rows, int cols, const float* x, int ldx, int k, float* y, int ldy,
                       cudaStream_t st, bool pdl) {
  if (cols % 4 || cols > 4096 || k < 1 || k > 8) return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(f32_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 4096 * 4);
    configured = true;
  }
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
  return cudaLaunchKernelEx(&cfg, f32_matvec_kernel, w, rows, cols, x, ldx, k, y, ldy);
}

}  // namespace iq
