// attn.cu -- gated full attention over the f32 KV cache for a pass of k rows.
//
// Restates src/qwen/quantized_attention.rs:409-507: per head [q | gate]
// projections; Q/K RMSNorm with the converted weight (:833-839); partial
// NeoX RoPE with f64 angles (:841-851); f32 KV append [pos][kv_head][hd];
// causal GQA softmax attention scaled by 1/sqrt(hd); output times
// sigmoid(gate).
//
// The scan is split over fixed position chunks of kAttnChunk: chunk c covers
// absolute positions [c*64, c*64+64) for every pass, each chunk keeps an
// online-softmax partial per query, and a row merges its chunks in order.
// A row's output therefore depends only on its own context length.
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__device__ __forceinline__ float sigmoidf_ref(float v) { return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-v))); }

// converted_norm + apply_rope on one head vector held in smem `v` (hd floats).
__device__ void norm_rope(float* v, const float* w, int hd, int rd, double theta, float eps, int position) {
  float x = threadIdx.x < hd ? v[threadIdx.x] : 0.f;
  float ss = block_sum_256(threadIdx.x < hd ? __fmul_rn(x, x) : 0.f);
  const float var = __fdiv_rn(ss, (float)hd);
  const float scale = __fdiv_rn(1.f, sqrtf(__fadd_rn(var, eps)));
  if (threadIdx.x < hd) v[threadIdx.x] = __fmul_rn(__fmul_rn(x, scale), w[threadIdx.x]);
  __syncthreads();
  const int half = rd / 2;
  float a = 0.f, b = 0.f;
  const int i = threadIdx.x;
  if (i < half) {
    const double freq = 1.0 / pow(theta, (double)(2 * i) / (double)rd);
    const double ang = (double)position * freq;
    double s, c;
    sincos(ang, &s, &c);
    const float cf = (float)c, sf = (float)s;
    const float o0 = v[i], o1 = v[half + i];
    a = __fsub_rn(__fmul_rn(o0, cf), __fmul_rn(o1, sf));
    b = __fadd_rn(__fmul_rn(o1, cf), __fmul_rn(o0, sf));
  }
  __syncthreads();
  if (i < half) {
    v[i] = a;
    v[half + i] = b;
  }
  __syncthreads();
}

// grid (rows, nh + nkv): one head vector per CTA.
__global__ void __launch_bounds__(256) attn_prep_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float v[256];
  const int t = blockIdx.x, h = blockIdx.y;
  const int position = *a.pos + t;
  if (h < a.nh) {
    const float* src = a.qg + (int64_t)t * a.qg_ld + (int64_t)h * 2 * a.hd;
    if (threadIdx.x < a.hd) v[threadIdx.x] = src[threadIdx.x];
    __syncthreads();
    norm_rope(v, a.q_norm, a.hd, a.rotary_dim, a.theta, a.eps, position);
    if (threadIdx.x < a.hd) a.qbuf[((int64_t)t * a.nh + h) * a.hd + threadIdx.x] = v[threadIdx.x];
  } else {
    const int kh = h - a.nh;
    const float* src = a.kp + (int64_t)t * a.kp_ld + (int64_t)kh * a.hd;
    if (threadIdx.x < a.hd) v[threadIdx.x] = src[threadIdx.x];
    __syncthreads();
    norm_rope(v, a.k_norm, a.hd, a.rotary_dim, a.theta, a.eps, position);
    const int64_t o = ((int64_t)position * a.nkv + kh) * a.hd;
    if (threadIdx.x < a.hd) {
      a.kcache[o + threadIdx.x] = v[threadIdx.x];
      a.vcache[o + threadIdx.x] = a.vp[(int64_t)t * a.vp_ld + (int64_t)kh * a.hd + threadIdx.x];
    }
  }
}

// grid (nkv, query groups of 8, chunk_ctas).  Warp w owns query
// q = group*8 + w (q = t*G + g over the rows and the G query heads of this kv
// head); lane l holds dims [l*D, l*D+D) with D = hd/32.  Each CTA walks chunks
// c = blockIdx.z, +chunk_ctas, ... and writes one partial {m, l, acc[hd]}.
template <int D>
__global__ void __launch_bounds__(256) attn_scan_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int kvh = blockIdx.x;
  const int G = a.nh / a.nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = blockIdx.y * 8 + warp;
  const int nq = a.rows * G;
  if (q >= nq) return;
  const int t = q / G, g = q % G;
  const int h = kvh * G + g;
  const int pos0 = *a.pos;
  const int attend = pos0 + t + 1;  // positions 0 .. pos0+t
  const int nchunks = (attend + kAttnChunk - 1) / kAttnChunk;
  const float scale = __fdiv_rn(1.f, sqrtf((float)a.hd));
  float qv[D];
  const float* qsrc = a.qbuf + ((int64_t)t * a.nh + h) * a.hd + lane * D;
#pragma unroll
  for (int d = 0; d < D; d++) qv[d] = qsrc[d];
  const int max_chunks = (pos0 + a.rows + kAttnChunk - 1) / kAttnChunk;
  for (int c = blockIdx.z; c < max_chunks; c += gridDim.z) {
    float* part = a.part + (((int64_t)t * a.nh + h) * max_chunks + c) * (a.hd + 2);
    if (c >= nchunks) {
      if (lane == 0) { part[0] = -INFINITY; part[1] = 0.f; }
      continue;
    }
    const int p0 = c * kAttnChunk, p1 = min(attend, p0 + kAttnChunk);
    float m = -INFINITY, l = 0.f, acc[D];
#pragma unroll
    for (int d = 0; d < D; d++) acc[d] = 0.f;
    for (int p = p0; p < p1; p++) {
      const float* kr = a.kcache + ((int64_t)p * a.nkv + kvh) * a.hd + lane * D;
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < D; d++) s = fmaf(qv[d], kr[d], s);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      s = __fmul_rn(s, scale);
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float e = expf(s - mn);
      l = fmaf(l, corr, e);
      const float* vr = a.vcache + ((int64_t)p * a.nkv + kvh) * a.hd + lane * D;
#pragma unroll
      for (int d = 0; d < D; d++) acc[d] = fmaf(acc[d], corr, __fmul_rn(e, vr[d]));
      m = mn;
    }
    if (lane == 0) { part[0] = m; part[1] = l; }
#pragma unroll
    for (int d = 0; d < D; d++) part[2 + lane * D + d] = acc[d];
  }
}

// grid (rows * nh): merge a row's chunk partials in order, apply the gate.
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x / a.nh, h = blockIdx.x % a.nh;
  const int pos0 = *a.pos;
  const int nchunks = (pos0 + t + 1 + kAttnChunk - 1) / kAttnChunk;
  const int max_chunks = (pos0 + a.rows + kAttnChunk - 1) / kAttnChunk;
  const float* part = a.part + ((int64_t)t * a.nh + h) * max_chunks * (a.hd + 2);
  float M = -INFINITY;
  for (int c = 0; c < nchunks; c++) M = fmaxf(M, part[c * (a.hd + 2)]);
  const int i = threadIdx.x;
  if (i >= a.hd) return;
  float L = 0.f, o = 0.f;
  for (int c = 0; c < nchunks; c++) {
    const float* pc = part + c * (a.hd + 2);
    const float w = expf(pc[0] - M);
    L = fmaf(pc[1], w, L);
    o = fmaf(pc[2 + i], w, o);
  }
  o = __fdiv_rn(o, L);
  const float gate = a.qg[(int64_t)t * a.qg_ld + (int64_t)h * 2 * a.hd + a.hd + i];
  a.out[(int64_t)t * a.out_ld + (int64_t)h * a.hd + i] = __fmul_rn(o, sigmoidf_ref(gate));
}

}  // namespace

cudaError_t attn_prep_launch(const AttnArgs& a, cudaStream_t st, bool pdl) {
  return launch_pdl(attn_prep_kernel, dim3(a.rows, a.nh + a.nkv), dim3(256), 0, st, pdl, a);
}

cudaError_t attn_scan_launch(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int G = a.nh / a.nkv;
  dim3 grid(a.nkv, (unsigned)ceil_div(a.rows * G, 8), a.chunk_ctas);
  switch (a.hd / 32) {
    case 2: return launch_pdl(attn_scan_kernel<2>, grid, dim3(256), 0, st, pdl, a);
    case 4: return launch_pdl(attn_scan_kernel<4>, grid, dim3(256), 0, st, pdl, a);
    case 8: return launch_pdl(attn_scan_kernel<8>, grid, dim3(256), 0, st, pdl, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t attn_combine_launch(const AttnArgs& a, cudaStream_t st, bool pdl) {
  return launch_pdl(attn_combine_kernel, dim3(a.rows * a.nh), dim3(256), 0, st, pdl, a);
}

}  // namespace iq
