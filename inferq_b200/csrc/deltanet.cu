// deltanet.cu -- Gated DeltaNet mixer step for a pass of k rows.
//
// Restates src/qwen/quantized_deltanet.rs:517-703 (per-row causal depthwise
// conv + SiLU, per-key-head L2 norm, beta = sigmoid(b),
// g = ssm_a * softplus(a + dt_bias)) and the recurrence of
// src/qwen/deltanet.rs:122-217 (S *= exp(g); pred = S^T k;
// delta = (v - pred) * beta; S += k delta^T; o = S^T q / sqrt(dk)).
//
// Grid: one CTA per (value head, 32-column slice of the value dimension).
// The delta rule is separable over value columns, so a slice's 128 x 32
// state block lives in registers for the whole pass (8 warps x 16 key rows,
// lane = column) and is read and written exactly once.  Rows are processed
// serially inside the CTA, so a row's result never depends on how many rows
// the pass holds.
//
// Rollback: the pass reads state buffer `sel` and writes buffer `1-sel`.
// A pass that commits only c < k rows is rolled back by running the same
// kernel again over the first c rows of the same projections (replay mode),
// which reproduces bit for bit the state c sequential rows would leave.
#include "kernels.cuh"
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__device__ __forceinline__ float sigmoid_ref(float v) { return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-v))); }

__device__ __forceinline__ float softplus_ref(float v) {
  if (v > 20.f) return v;
  if (v < -20.f) return expf(v);
  return log1pf(expf(v));
}

// Fixed-order sum across the 8 warps of a column: red[warp][lane].
__device__ __forceinline__ float warp8_col_sum(float v, float (*red)[33], int warp, int lane) {
  red[warp][lane] = v;
  __syncthreads();
  float s = red[0][lane];
#pragma unroll
  for (int w = 1; w < 8; w++) s = __fadd_rn(s, red[w][lane]);
  __syncthreads();
  return s;
}

__global__ void __launch_bounds__(256) deltanet_kernel(DeltaNetArgs a) {
  pdl_wait();
  pdl_trigger();
  const int layer = blockIdx.y;
  const DeltaNetLayer& L = a.layers[layer];
  const int slices = a.dv / 32;
  const int vh = blockIdx.x / slices;
  const int slice = blockIdx.x % slices;
  const int ratio = a.nv / a.nk;
  const int kh = a.tiled_heads ? vh % a.nk : vh / ratio;
  const int rep = a.tiled_heads ? vh / a.nk : vh % ratio;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int key_dim = a.nk * a.dk;
  const int conv_dim = 2 * key_dim + a.nv * a.dv;
  const int K = a.conv_k;  // conv kernel width (<= 4)
  const int rows_i = a.dk / 8;  // key rows per warp
  const int j = slice * 32 + lane;  // value column
  const int sel = *a.sel;
  const int rows = a.replay ? *a.committed : a.rows;
  if (a.replay && rows >= a.rows) return;  // a fully accepted pass needs no replay

  __shared__ float qk[2][256];  // normalized q, k of this key head (dk <= 256)
  __shared__ float red[8][33];
  __shared__ float bg[2];
  // conv channels this CTA computes: q and k of key head kh, and its v columns
  const int nqk = 2 * a.dk;
  const int nch = nqk + 32;
  // channel id -> global conv channel
  auto chan = [&](int c) {
    if (c < a.dk) return kh * a.dk + c;
    if (c < nqk) return key_dim + kh * a.dk + (c - a.dk);
    return 2 * key_dim + vh * a.dv + slice * 32 + (c - nqk);
  };
  // conv history (K-1 taps) of this thread's channels in registers:
  // thread t owns channels t and t+256 (nch <= 512 covers dk <= 240).
  float hist[2][3];
  const float* cin = L.conv_state[sel];
#pragma unroll
  for (int u = 0; u < 2; u++) {
    const int c = threadIdx.x + 256 * u;
#pragma unroll
    for (int tp = 0; tp < 3; tp++) hist[u][tp] = (c < nch && tp < K - 1) ? cin[(int64_t)chan(c) * (K - 1) + tp] : 0.f;
  }
  // state block
  float S[16];
  const float* sin_ = L.rec_state[sel] + (int64_t)vh * a.dk * a.dv;
#pragma unroll
  for (int r = 0; r < 16; r++) S[r] = r < rows_i ? sin_[(int64_t)(warp * rows_i + r) * a.dv + j] : 0.f;
  const float qscale = __fdiv_rn(1.f, sqrtf((float)a.dk));

  for (int t = 0; t < rows; t++) {
    const float* proj = a.qkv + (int64_t)t * a.qkv_ld;
    float vcol = 0.f;
    // causal depthwise conv + SiLU (src/qwen/quantized_deltanet.rs:733-759)
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int c = threadIdx.x + 256 * u;
      if (c < nch) {
        const int g = chan(c);
        const float* w = L.conv_w + (int64_t)g * K;
        const float x = proj[g];
        float sum = __fmul_rn(w[K - 1], x);
        for (int tp = 0; tp < K - 1; tp++) sum = __fadd_rn(sum, __fmul_rn(w[tp], hist[u][tp]));
        const float out = __fmul_rn(sum, sigmoid_ref(sum));
        for (int tp = 0; tp + 1 < K - 1; tp++) hist[u][tp] = hist[u][tp + 1];
        if (K > 1) hist[u][K - 2] = x;
        if (c < nqk) qk[c / a.dk][c % a.dk] = out;
        else red[0][c - nqk] = out;  // v staged through red row 0
      }
    }
    // beta / decay for this value head
    if (threadIdx.x == 0) {
      const float* ba = a.ba + (int64_t)t * a.ba_ld;
      float b, al;
      if (a.ba_interleaved) {
        const int base = kh * 2 * ratio;
        b = ba[base + rep];
        al = ba[base + ratio + rep];
      } else {
        b = ba[vh];
        al = ba[a.nv + vh];
      }
      bg[0] = sigmoid_ref(b);
      bg[1] = __fmul_rn(L.ssm_a[vh], softplus_ref(__fadd_rn(al, L.dt_bias[vh])));
    }
    __syncthreads();
    vcol = red[0][lane];
    // L2 norm of q and k (x * (sum x^2 + 1e-6)^-1/2), warp 0 -> q, warp 1 -> k
    if (warp < 2) {
      float ss = 0.f;
      for (int i = lane; i < a.dk; i += 32) ss = fmaf(qk[warp][i], qk[warp][i], ss);
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
      const float scale = __fdiv_rn(1.f, sqrtf(__fadd_rn(ss, 1e-6f)));
      __syncwarp();
      for (int i = lane; i < a.dk; i += 32) qk[warp][i] = __fmul_rn(qk[warp][i], scale);
    }
    __syncthreads();
    const float beta = bg[0], decay = expf(bg[1]);
    // recurrence
    float pred = 0.f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
      if (r < rows_i) {
        S[r] = __fmul_rn(S[r], decay);
        pred = fmaf(S[r], qk[1][warp * rows_i + r], pred);
      }
    }
    pred = warp8_col_sum(pred, red, warp, lane);
    const float delta = __fmul_rn(__fsub_rn(vcol, pred), beta);
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
      if (r < rows_i) {
        S[r] = fmaf(qk[1][warp * rows_i + r], delta, S[r]);
        o = fmaf(S[r], qk[0][warp * rows_i + r], o);
      }
    }
    o = warp8_col_sum(o, red, warp, lane);
    if (!a.replay && warp == 0) a.out[(int64_t)t * a.out_ld + vh * a.dv + j] = __fmul_rn(o, qscale);
  }
  // write back the state after `rows` rows
  float* sout = L.rec_state[1 - sel] + (int64_t)vh * a.dk * a.dv;
#pragma unroll
  for (int r = 0; r < 16; r++)
    if (r < rows_i) sout[(int64_t)(warp * rows_i + r) * a.dv + j] = S[r];
  float* cout_ = L.conv_state[1 - sel];
  const bool qk_writer = rep == 0 && slice == 0;
#pragma unroll
  for (int u = 0; u < 2; u++) {
    const int c = threadIdx.x + 256 * u;
    if (c < nch && (c >= nqk || qk_writer))
      for (int tp = 0; tp < K - 1; tp++) cout_[(int64_t)chan(c) * (K - 1) + tp] = hist[u][tp];
  }
}

// Gated RMSNorm of every value head (src/qwen/norm.rs:16-25:
// x / sqrt(mean(x^2) + eps) * w * silu(z)), then quantization of the row for
// the output projection.  One CTA per row; warp w normalizes heads w, w+8, ...
template <int MAXB>
__global__ void __launch_bounds__(256) gated_norm_kernel(GatedNormArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float xs[];
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cols = a.heads * a.dv, nb = cols / 256;
  const float* o = a.o + (int64_t)row * a.o_ld;
  const float* z = a.z + (int64_t)row * a.z_ld;
  // a lane's elements of block b lie in one head (dv >= 32): 32s .. 32s+31
  float v[MAXB][8], zv[MAXB][8], wv[MAXB][8];
#pragma unroll
  for (int j = 0; j < MAXB; j++) {
    const int b = warp + 8 * j;
    if (b < nb) {
      ld_q8k_lane(o, b, lane, v[j]);
      ld_q8k_lane(z, b, lane, zv[j]);
      const int e0 = b * 256 + 32 * (lane & 7);
      const float* wp = a.w + (e0 % a.dv) + 4 * (lane >> 3);
      const float4 w0 = *reinterpret_cast<const float4*>(wp), w1 = *reinterpret_cast<const float4*>(wp + 16);
      wv[j][0] = w0.x; wv[j][1] = w0.y; wv[j][2] = w0.z; wv[j][3] = w0.w;
      wv[j][4] = w1.x; wv[j][5] = w1.y; wv[j][6] = w1.z; wv[j][7] = w1.w;
    }
  }
  // per head: sum of squares over the lanes of the head (s bits below
  // log2(dv/32), and the tig bits), then x / sqrt(mean + eps) * w * silu(z)
  const int smask = a.dv / 32 - 1;
#pragma unroll
  for (int j = 0; j < MAXB; j++) {
    if (warp + 8 * j >= nb) continue;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) ss = fmaf(v[j][i], v[j][i], ss);
    for (int m = 1; m <= smask; m <<= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
    ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, 8));
    ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, 16));
    const float den = sqrtf(__fadd_rn(__fmul_rn(ss, a.inv_dv), a.eps));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float silu = __fdiv_rn(zv[j][i], __fadd_rn(1.f, expf(-zv[j][i])));
      v[j][i] = __fmul_rn(__fmul_rn(__fdiv_rn(v[j][i], den), wv[j][i]), silu);
    }
  }
  finish_row<MAXB>(v, nb, cols, a.q8k ? a.q8k + (int64_t)row * a.q8k_stride : nullptr,
                   a.q80 ? a.q80 + (int64_t)row * a.q80_stride : nullptr, nullptr, xs);
}

}  // namespace

cudaError_t deltanet_launch(const DeltaNetArgs& a, int nlayers, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nv * (a.dv / 32), nlayers);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, deltanet_kernel, a);
}

cudaError_t gated_norm_launch(const GatedNormArgs& a, int rows, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  const int cols = a.heads * a.dv, nb = cols / 256;
  // lanes own 32 contiguous elements of one head; Q8_K rows need 256-blocks
  if (a.dv < 32 || a.dv > 256 || (a.dv & (a.dv - 1)) || cols % 256 || a.o_ld % 4 || a.z_ld % 4 ||
      ((uintptr_t)a.o | (uintptr_t)a.z | (uintptr_t)a.w) & 15)
    return cudaErrorInvalidValue;
  cfg.dynamicSmemBytes = a.q80 ? cols * sizeof(float) : 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (nb <= 8) return cudaLaunchKernelEx(&cfg, gated_norm_kernel<1>, a);
  if (nb <= 16) return cudaLaunchKernelEx(&cfg, gated_norm_kernel<2>, a);
  if (nb <= 32) return cudaLaunchKernelEx(&cfg, gated_norm_kernel<4>, a);
  return cudaErrorInvalidValue;
}

}  // namespace iq
