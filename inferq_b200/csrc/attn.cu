// attn.cu -- gated full attention over the f32 KV cache for a pass of k rows.
//
// Restates src/qwen/quantized_attention.rs:409-507: per head [q | gate]
// projections; Q/K RMSNorm with the converted weight (:833-839); partial
// NeoX RoPE with f64 angles (:841-851); f32 KV append [pos][kv_head][hd];
// causal GQA softmax attention scaled by 1/sqrt(hd); output times
// sigmoid(gate).
//
// The scan is split over fixed position chunks of kAttnChunk: chunk c covers
// absolute positions [c*32, c*32+32) for every pass, each chunk keeps an
// online-softmax partial per query, and a row merges its chunks in order.
// A row's output therefore depends only on its own context length.
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__device__ __forceinline__ float sigmoidf_ref(float v) { return __fdiv_rn(1.f, __fadd_rn(1.f, exp_ref(-v))); }

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

// grid (nkv, chunks): CTA (h, c) stages K and V of positions
// [c*32, c*32+32) of kv head h in shared memory, then every warp takes the
// queries q = t*G + g of this kv head in turn: lane p scores position p,
// the warp forms the chunk's softmax partial {m, l} with butterflies, and
// lane l accumulates dims [l*D, l*D+D) of sum_p e_p V[p].  A chunk's partial
// depends only on the query and the positions inside it.
template <int D>
__global__ void __launch_bounds__(256) attn_scan_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int HD = 32 * D;
  extern __shared__ float sm[];
  float* Ks = sm;                       // [32][HD + 1]
  float* Vs = Ks + 32 * (HD + 1);       // [32][HD]
  float* Qs = Vs + 32 * HD;             // [rows * G][HD]: this KV head's query rows
  const int kvh = blockIdx.x, c = blockIdx.y;
  const int G = a.nh / a.nkv;
  // blockIdx.z picks this CTA's share of the KV head's query heads
  const int gpc = G / gridDim.z, g0 = blockIdx.z * gpc;
  const int pos0 = *a.pos;
  const int last = pos0 + a.rows - 1;   // last position any row attends to
  const int p0 = c * kAttnChunk;
  if (p0 > last) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // stage K (padded rows) and V of the chunk
  for (int i = threadIdx.x; i < 32 * HD / 4; i += 256) {
    const int p = i / (HD / 4), d4 = i % (HD / 4);
    const int pp = min(p0 + p, last);
    const float4 kv = *reinterpret_cast<const float4*>(a.kcache + ((int64_t)pp * a.nkv + kvh) * HD + 4 * d4);
    const float4 vv = *reinterpret_cast<const float4*>(a.vcache + ((int64_t)pp * a.nkv + kvh) * HD + 4 * d4);
    float* kr = Ks + p * (HD + 1) + 4 * d4;
    kr[0] = kv.x; kr[1] = kv.y; kr[2] = kv.z; kr[3] = kv.w;
    *reinterpret_cast<float4*>(Vs + p * HD + 4 * d4) = vv;
  }
  const int nq = a.rows * gpc;  // (row, query head) items of this CTA
#pragma unroll 4
  for (int i = threadIdx.x; i < nq * HD / 4; i += 256) {
    const int q = i / (HD / 4), d4 = i % (HD / 4);
    const int t = q / gpc, h = kvh * G + g0 + q % gpc;
    *reinterpret_cast<float4*>(Qs + q * HD + 4 * d4) =
        *reinterpret_cast<const float4*>(a.qbuf + ((int64_t)t * a.nh + h) * HD + 4 * d4);
  }
  __syncthreads();
  const float scale = __fdiv_rn(1.f, sqrtf((float)HD));
  const int nchunks_total = (last + kAttnChunk) / kAttnChunk;
  // a warp takes its queries q = warp + 8 j in groups of QG: each K element
  // a lane loads feeds QG score chains and each V element QG accumulators;
  // every query keeps exactly its own operation order
  constexpr int QG = 4;
  for (int q0 = warp; q0 < nq; q0 += 8 * QG) {
    bool live[QG];
    int tq[QG], hq[QG];
    bool anyl = false;
#pragma unroll
    for (int g = 0; g < QG; g++) {
      const int q = q0 + 8 * g;
      tq[g] = q / gpc;
      hq[g] = kvh * G + g0 + q % gpc;
      live[g] = q < nq && p0 <= pos0 + tq[g];  // else: past the queries, or the chunk is in row t's future
      anyl |= live[g];
    }
    if (!anyl) continue;
    const float* kr = Ks + lane * (HD + 1);
    float s[QG][4];
#pragma unroll
    for (int g = 0; g < QG; g++) s[g][0] = s[g][1] = s[g][2] = s[g][3] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
      const float k0 = kr[d], k1 = kr[d + 1], k2 = kr[d + 2], k3 = kr[d + 3];
#pragma unroll
      for (int g = 0; g < QG; g++) {
        if (!live[g]) continue;
        const float* qs = Qs + (q0 + 8 * g) * HD;
        s[g][0] = fmaf(qs[d], k0, s[g][0]);
        s[g][1] = fmaf(qs[d + 1], k1, s[g][1]);
        s[g][2] = fmaf(qs[d + 2], k2, s[g][2]);
        s[g][3] = fmaf(qs[d + 3], k3, s[g][3]);
      }
    }
    float e[QG], m[QG], l[QG];
#pragma unroll
    for (int g = 0; g < QG; g++) {
      const bool valid = live[g] && p0 + lane <= pos0 + tq[g];
      const float sc = valid ? __fmul_rn(__fadd_rn(__fadd_rn(s[g][0], s[g][1]), __fadd_rn(s[g][2], s[g][3])), scale)
                             : -INFINITY;
      float mm = sc;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
      e[g] = valid ? exp_ref(sc - mm) : 0.f;
      float ll = e[g];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ll = __fadd_rn(ll, __shfl_xor_sync(0xffffffffu, ll, o));
      m[g] = mm;
      l[g] = ll;
    }
    float acc[QG][D];
#pragma unroll
    for (int g = 0; g < QG; g++)
#pragma unroll
      for (int d = 0; d < D; d++) acc[g][d] = 0.f;
    for (int p = 0; p < 32; p++) {
      float ep[QG];
#pragma unroll
      for (int g = 0; g < QG; g++) ep[g] = __shfl_sync(0xffffffffu, e[g], p);
      const float* vr = Vs + p * HD + lane;
#pragma unroll
      for (int d = 0; d < D; d++) {
        const float v = vr[32 * d];
#pragma unroll
        for (int g = 0; g < QG; g++) acc[g][d] = fmaf(ep[g], v, acc[g][d]);
      }
    }
#pragma unroll
    for (int g = 0; g < QG; g++) {
      if (!live[g]) continue;
      float* part = a.part + (((int64_t)tq[g] * a.nh + hq[g]) * nchunks_total + c) * (HD + 2);
      if (lane == 0) { part[0] = m[g]; part[1] = l[g]; }
#pragma unroll
      for (int d = 0; d < D; d++) part[2 + 32 * d + lane] = acc[g][d];
    }
  }
}

// grid (rows * nh): merge a row's chunk partials in order, apply the gate.
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x / a.nh, h = blockIdx.x % a.nh;
  const int pos0 = *a.pos;
  const int nchunks = (pos0 + t + 1 + kAttnChunk - 1) / kAttnChunk;
  const int nchunks_total = (pos0 + a.rows - 1 + kAttnChunk) / kAttnChunk;
  const float* part = a.part + ((int64_t)t * a.nh + h) * nchunks_total * (a.hd + 2);
  const int i = threadIdx.x;
  // M = the chunks' largest max (exact in any order)
  __shared__ float red[8];
  float mx = -INFINITY;
  for (int c = i; c < nchunks; c += 256) mx = fmaxf(mx, part[c * (a.hd + 2)]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((i & 31) == 0) red[i >> 5] = mx;
  __syncthreads();
  float M = red[0];
#pragma unroll
  for (int w = 1; w < 8; w++) M = fmaxf(M, red[w]);
  // the chunks in order, 256 at a time: their weights exp(m_c - M) once per
  // CTA, then L = sum l_c w_c and o = sum o_c w_c as ordered chains
  __shared__ float wc[256];
  __shared__ float ys[256];
  float L = 0.f, o = 0.f;
  for (int c0 = 0; c0 < nchunks; c0 += 256) {
    const int nc = min(256, nchunks - c0);
    __syncthreads();  // the previous weights are read
    if (i < nc) wc[i] = exp_ref(part[(c0 + i) * (a.hd + 2)] - M);
    __syncthreads();
    if (i < a.hd) {
#pragma unroll 8
      for (int c = 0; c < nc; c++) {
        const float* pc = part + (c0 + c) * (a.hd + 2);
        const float w = wc[c];
        L = fmaf(pc[1], w, L);
        o = fmaf(pc[2 + i], w, o);
      }
    }
  }
  if (i < a.hd) {
    o = __fdiv_rn(o, L);
    const float gate = a.qg[(int64_t)t * a.qg_ld + (int64_t)h * 2 * a.hd + a.hd + i];
    const float y = __fmul_rn(o, sigmoidf_ref(gate));
    if (a.q8k_out || a.q80_out) ys[i] = y;
    else a.out[(int64_t)t * a.out_ld + (int64_t)h * a.hd + i] = y;
  }
  if (!a.q8k_out && !a.q80_out) return;
  // the output projection's activation row, quantized here: a head of 256 is
  // one Q8_K block (block h of the row), a head of 128k is k Q8_0 groups
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cols = a.nh * a.hd;
  if (a.q8k_out) {
    if (warp == 0) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = ys[q8k_lane_pos(lane, e)];
      quant_q8k_block_warp_v(v, a.q8k_out + (int64_t)t * a.q8k_stride, cols / 256, h, lane);
    }
  } else if (warp < a.hd / 128) {
    const int g = h * (a.hd / 128) + warp;
    const int base = q80_lane_base(g, lane) - h * a.hd;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = ys[base + e];
    quant_q80_group_warp_v(v, a.q80_out + (int64_t)t * a.q80_stride, cols / 32, g, lane);
  }
}

template <int D>
cudaError_t launch_scan(dim3 grid, size_t smem, cudaStream_t st, bool pdl, const AttnArgs& a) {
  static bool configured[64] = {};
  static std::mutex mu;
  const cudaError_t e = once_per_device(configured, mu, [] {
    return cudaFuncSetAttribute(attn_scan_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_scan_kernel<D>, grid, dim3(256), smem, st, pdl, a);
}

}  // namespace

cudaError_t attn_prep_launch(const AttnArgs& a, cudaStream_t st, bool pdl) {
  return launch_pdl(attn_prep_kernel, dim3(a.rows, a.nh + a.nkv), dim3(256), 0, st, pdl, a);
}

namespace {
int scan_split(const AttnArgs& a) {
  const int G = a.nh / a.nkv;
  int split = 1;  // query-head groups per KV head: at least ~2 CTAs per SM's worth of work
  while (split * 2 <= G && G % (split * 2) == 0 && a.nkv * a.chunk_ctas * split < 2 * 148) split *= 2;
  return split;
}
size_t scan_smem(const AttnArgs& a, int rows) {
  const int gpc = a.nh / a.nkv / scan_split(a);
  return (size_t)(32 * (a.hd + 1) + 32 * a.hd + rows * gpc * a.hd) * sizeof(float);
}
}  // namespace

int attn_scan_max_rows(const AttnArgs& a, int want) {
  int rows = want;
  while (rows > 1 && scan_smem(a, rows) > 200 * 1024) rows /= 2;
  return rows;
}

cudaError_t attn_scan_launch(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int split = scan_split(a);
  dim3 grid(a.nkv, a.chunk_ctas, split);
  const size_t smem = scan_smem(a, a.rows);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  switch (a.hd / 32) {
    case 2: return launch_scan<2>(grid, smem, st, pdl, a);
    case 4: return launch_scan<4>(grid, smem, st, pdl, a);
    case 8: return launch_scan<8>(grid, smem, st, pdl, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t attn_combine_launch(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.hd > 256 || (a.q8k_out && a.hd != 256) || (a.q80_out && a.hd % 128)) return cudaErrorInvalidValue;
  return launch_pdl(attn_combine_kernel, dim3(a.rows * a.nh), dim3(256), 0, st, pdl, a);
}

}  // namespace iq
