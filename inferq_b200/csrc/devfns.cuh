// devfns.cuh -- device functions shared by several kernels (header-inline so
// every caller can inline them; libiq is built without relocatable code).
#pragma once
#include "layout.cuh"

namespace iq {

// Deterministic CTA-wide sum for 256 threads (fixed tree order).
__device__ __forceinline__ float block_sum_256(float v) {
  __shared__ float red[8];
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  const int warp = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int i = 1; i < 8; i++) t = __fadd_rn(t, red[i]);
  return t;
}

// Element `e` of a device-layout row, decoded as candle's to_float does
// (d*sc first, then *q, then -dmin*m: two roundings, never fused).
__device__ __forceinline__ float dev_weight(int dt, const uint8_t* row, int nb, int e) {
  switch (dt) {
    case Q4_K:
    case Q5_K: {
      const int BB = dt == Q4_K ? 144 : 176;
      const int b = e / 256, i = e % 256;
      const uint8_t* blk = row + (int64_t)b * BB;
      int sc[8], mn[8];
      unpack_k_scales(blk + 4, sc, mn);
      const int j = i / 64, w = i % 64, hi = w / 32, ii = w % 32;
      const uint8_t* qs = blk + (dt == Q4_K ? 16 : 48);
      int q = (qs[q4k_qs_perm(32 * j + ii)] >> (4 * hi)) & 15;
      if (dt == Q5_K) q |= ((blk[16 + q5k_qh_perm(ii)] >> (2 * j + hi)) & 1) << 4;
      const int s = 2 * j + hi;
      const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
      const float dmin = h2f(*reinterpret_cast<const uint16_t*>(blk + 2));
      const float d1 = __fmul_rn(d, (float)sc[s]), m1 = __fmul_rn(dmin, (float)mn[s]);
      return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case Q6_K: {
      const int b = e / 256, i = e % 256;
      const uint8_t* blk = row + (int64_t)b * 208;
      const int q = q6k_dev_value(blk, i) - 32;
      const float d = h2f(*reinterpret_cast<const uint16_t*>(row + (int64_t)nb * 208 + 2 * b));
      const float sc = (float)reinterpret_cast<const int8_t*>(blk + 192)[i / 16];
      return __fmul_rn(__fmul_rn(d, sc), (float)q);
    }
    case Q8_0: {
      const int b = e / 32, i = e % 32;
      const int8_t q = reinterpret_cast<const int8_t*>(row)[(int64_t)(b / 4) * 128 + q80_perm(b % 4, i)];
      const float d = h2f(*reinterpret_cast<const uint16_t*>(row + (int64_t)nb * 32 + 2 * b));
      return __fmul_rn((float)q, d);
    }
    case F32: return reinterpret_cast<const float*>(row)[e];
    case BF16: return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(row)[e] << 16);
    default: return __half2float(reinterpret_cast<const __half*>(row)[e]);
  }
}

// ---------------------------------------------------------------- quantizers
// One warp per Q8_K block.  Lane l = tig*8 + s holds elements
// 32s + 16h + tig*4 + e (h, e in order), which is exactly the 8 contiguous
// bytes it writes to the permuted layout.  Semantics: candle
// BlockQ8K::from_float (first value of largest magnitude sets the scale).
// v[4h + e] is element 32s + 16h + 4tig + e of block b (s = lane & 7,
// tig = lane >> 3): two runs of four contiguous floats.
__device__ __forceinline__ void quant_q8k_block_warp_v(const float (&v)[8], uint8_t* act_row, int nb, int b,
                                                       int lane) {
  const int s = lane & 7, tig = lane >> 3;
  float amax = 0.f, vmax = 0.f;
  int imax = 1 << 30;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float a = fabsf(v[i]);
    if (amax < a) { amax = a; vmax = v[i]; imax = 32 * s + 16 * (i / 4) + tig * 4 + (i % 4); }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    float oa = __shfl_xor_sync(0xffffffffu, amax, m);
    float ov = __shfl_xor_sync(0xffffffffu, vmax, m);
    int oi = __shfl_xor_sync(0xffffffffu, imax, m);
    if (oa > amax || (oa == amax && oi < imax)) { amax = oa; vmax = ov; imax = oi; }
  }
  int8_t q[8];
  float d = 0.f;
  if (amax != 0.f) {
    const float iscale = __fdiv_rn(-128.f, vmax);
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = (int8_t)fminf(roundf(__fmul_rn(iscale, v[i])), 127.f);
    d = __fdiv_rn(1.f, iscale);
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) q[i] = 0;
  }
  int sum[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; i++) sum[i / 4] += q[i];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 8);
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 16);
  }
  uint2 packed;
  packed.x = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) | ((uint32_t)(uint8_t)q[2] << 16) |
             ((uint32_t)(uint8_t)q[3] << 24);
  packed.y = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) | ((uint32_t)(uint8_t)q[6] << 16) |
             ((uint32_t)(uint8_t)q[7] << 24);
  *reinterpret_cast<uint2*>(act_row + (int64_t)b * 256 + q8k_act_perm(32 * s + tig * 4)) = packed;
  int16_t* bs = reinterpret_cast<int16_t*>(act_row + q8k_bs_offset(nb) + b * 16);
  if (tig == 0) bs[s] = (int16_t)(sum[0] + sum[1]);
  if (lane == 0) reinterpret_cast<float*>(act_row + (int64_t)nb * 256)[b] = d;
}

// One warp per group of four Q8_0 blocks.  Lane l = tig*8 + bb*2 + h holds
// the 4 elements it writes at byte 4l of the group.  Semantics: candle
// BlockQ8_0::from_float (d = amax/127 kept as f16; q from the f32 d).
// v[e] is element q80_lane_base(g, lane) + e: four contiguous floats.
__device__ __forceinline__ int q80_lane_base(int g, int lane) {
  return 32 * (4 * g + ((lane & 7) >> 1)) + 16 * (lane & 1) + (lane >> 3) * 4;
}
__device__ __forceinline__ void quant_q80_group_warp_v(const float (&v)[4], uint8_t* act_row, int nb, int g,
                                                       int lane) {
  const int tig = lane >> 3, bb = (lane & 7) >> 1, h = lane & 1;
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < 4; e++) amax = fmaxf(amax, fabsf(v[e]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 8));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 16));
  const float d = __fdiv_rn(amax, 127.f);
  const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < 4; e++) packed |= (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(v[e], id)) << (8 * e);
  *reinterpret_cast<uint32_t*>(act_row + (int64_t)g * 128 + lane * 4) = packed;
  if (tig == 0 && h == 0)
    reinterpret_cast<float*>(act_row + (int64_t)nb * 32)[4 * g + bb] = __half2float(__float2half_rn(d));
}

__device__ __forceinline__ void quant_q8k_block_warp(const float* x, uint8_t* act_row, int nb, int b, int lane) {
  const int s = lane & 7, tig = lane >> 3;
  float v[8];
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int e = 0; e < 4; e++) v[h * 4 + e] = x[b * 256 + 32 * s + 16 * h + tig * 4 + e];
  quant_q8k_block_warp_v(v, act_row, nb, b, lane);
}
__device__ __forceinline__ void quant_q80_group_warp(const float* x, uint8_t* act_row, int nb, int g, int lane) {
  const int base = q80_lane_base(g, lane);
  float v[4];
#pragma unroll
  for (int e = 0; e < 4; e++) v[e] = x[base + e];
  quant_q80_group_warp_v(v, act_row, nb, g, lane);
}

// ------------------------------------------------- row transforms (one CTA per row)
// Warp w of a 256-thread CTA owns the Q8_K blocks b = w + 8j (j < MAXB) of a
// row and keeps their elements in registers: lane l holds element
// b*256 + q8k_lane_pos(l, i) in v[j][i], i.e. the order quant_q8k_block_warp_v
// consumes, loaded as two 16-byte vectors.
__device__ __forceinline__ int q8k_lane_pos(int lane, int i) {
  return 32 * (lane & 7) + 16 * (i / 4) + 4 * (lane >> 3) + (i % 4);
}
__device__ __forceinline__ void ld_q8k_lane(const float* row, int b, int lane, float (&v)[8], int cols = 1 << 30) {
  if (b * 256 + 32 * (lane & 7) >= cols) {  // a trailing half block (cols % 256 == 128)
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = 0.f;
    return;
  }
  const float* p = row + b * 256 + 32 * (lane & 7) + 4 * (lane >> 3);
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 c = *reinterpret_cast<const float4*>(p + 16);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
}
// Deterministic CTA-wide sum of one value per thread (256 threads): lane
// tree, then the eight warp partials in warp order.
__device__ __forceinline__ float cta_sum256(float v, float* red8) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  if ((threadIdx.x & 31) == 0) red8[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red8[0];
#pragma unroll
  for (int i = 1; i < 8; i++) t = __fadd_rn(t, red8[i]);
  return t;
}
// Write a row held as above (nb = ceil(cols / 256) blocks, cols a multiple of
// 128): Q8_K straight from registers (cols a multiple of 256); the Q8_0
// layout and the f32 copy go through the shared row `xs` (cols floats).
template <int MAXB>
__device__ __forceinline__ void finish_row(const float (&v)[MAXB][8], int nb, int cols, uint8_t* q8k, uint8_t* q80,
                                           float* xn, float* xs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (q8k) {
#pragma unroll
    for (int j = 0; j < MAXB; j++)
      if (warp + 8 * j < nb) quant_q8k_block_warp_v(v[j], q8k, nb, warp + 8 * j, lane);
  }
  if (!q80 && !xn) return;
#pragma unroll
  for (int j = 0; j < MAXB; j++) {
    const int b = warp + 8 * j;
    if (b < nb && b * 256 + 32 * (lane & 7) < cols) {
      float* p = xs + b * 256 + 32 * (lane & 7) + 4 * (lane >> 3);
      *reinterpret_cast<float4*>(p) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      *reinterpret_cast<float4*>(p + 16) = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
    }
  }
  __syncthreads();
  if (q80)
    for (int g = warp; g < cols / 128; g += 8) quant_q80_group_warp(xs, q80, cols / 32, g, lane);
  if (xn)
    for (int i = 4 * threadIdx.x; i < cols; i += 1024)
      *reinterpret_cast<float4*>(xn + i) = *reinterpret_cast<const float4*>(xs + i);
}

}  // namespace iq
