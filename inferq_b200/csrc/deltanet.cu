// deltanet.cu -- Gated DeltaNet mixer step for a pass of k rows.
//
// Restates src/qwen/quantized_deltanet.rs:517-703 (per-row causal depthwise
// conv + SiLU, per-key-head L2 norm, beta = sigmoid(b),
// g = ssm_a * softplus(a + dt_bias)) and the recurrence of
// src/qwen/deltanet.rs:122-217 (S *= exp(g); pred = S^T k;
// delta = (v - pred) * beta; S += k delta^T; o = S^T q / sqrt(dk)).
//
// Grid: one CTA per (value head, 16-column slice of the value dimension).
// The delta rule is separable over value columns, so a slice's dk x 16 state
// block lives in registers for the whole pass: warp w owns columns 2w, 2w+1,
// lane = (column, group of dk/16 key rows), and the sums over key rows are
// shuffles inside the warp.  The conv outputs of a row are shared through a
// double-buffered shared row, so a row costs one CTA barrier.  Rows are
// processed serially inside the CTA, so a row's result never depends on how
// many rows the pass holds.
//
// Rollback: the state lives in a ring of kStateRing buffers.  A pass reads
// buffer `cur` and writes the state after its row t to buffer cur+1+t, so
// committing c rows (any c <= rows) only moves `cur` by c.
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

constexpr int kMaxRowsDn = 8;

template <int K, int COLS>  // conv kernel width; value columns per CTA (32 or 16)
__global__ void __launch_bounds__(256) deltanet_kernel(DeltaNetArgs a) {
  pdl_wait();
  pdl_trigger();
  const int layer = blockIdx.y;
  const DeltaNetLayer& L = a.layers[layer];
  constexpr int CPW = COLS / 8;        // columns per warp
  constexpr int GROUPS = 32 / CPW;     // key-row groups per column (lanes)
  const int slices = a.dv / COLS;
  const int vh = blockIdx.x / slices;
  const int slice = blockIdx.x % slices;
  const int ratio = a.nv / a.nk;
  const int kh = a.tiled_heads ? vh % a.nk : vh / ratio;
  const int rep = a.tiled_heads ? vh / a.nk : vh % ratio;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int key_dim = a.nk * a.dk;
  const int rows_i = a.dk / GROUPS;  // key rows per lane
  const int c4 = lane % CPW, rg = lane / CPW;
  const int j = slice * COLS + CPW * warp + c4;  // value column of this lane
  const int kr0 = rg * rows_i;               // first key row of this lane
  const int cur = *a.cur;
  const int rows = a.rows;

  // per row t (double-buffered by t & 1): conv outputs q | k | v(32 columns)
  __shared__ float qkv[2][2 * 128 + 32];
  __shared__ float bg[2][2];
  const int nqk = 2 * a.dk;
  const int nch = nqk + COLS;
  auto chan = [&](int c) {
    if (c < a.dk) return kh * a.dk + c;
    if (c < nqk) return key_dim + kh * a.dk + (c - a.dk);
    return 2 * key_dim + vh * a.dv + slice * COLS + (c - nqk);
  };
  // every input of the pass, requested before any arithmetic and parked in
  // shared memory: thread t owns conv channels t and t+256; thread 0 also
  // reads beta/alpha
  __shared__ float xin_s[kMaxRowsDn][2 * 128 + 32];
  __shared__ float ba_s[kMaxRowsDn][2];
  float cw[2][4], hist[2][3];
  const float* cin = L.conv_state[cur];
  {
    float xin[kMaxRowsDn][2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int c = threadIdx.x + 256 * u;
      const bool own = c < nch;
      const int g = own ? chan(c) : 0;
#pragma unroll
      for (int t = 0; t < kMaxRowsDn; t++) xin[t][u] = (own && t < rows) ? a.qkv[(int64_t)t * a.qkv_ld + g] : 0.f;
#pragma unroll
      for (int tp = 0; tp < 4; tp++) cw[u][tp] = (own && tp < K) ? L.conv_w[(int64_t)g * K + tp] : 0.f;
#pragma unroll
      for (int tp = 0; tp < 3; tp++) hist[u][tp] = (own && tp < K - 1) ? cin[(int64_t)g * (K - 1) + tp] : 0.f;
    }
    if (threadIdx.x < 2 * kMaxRowsDn) {
      const int t = threadIdx.x >> 1;
      int idx = (threadIdx.x & 1) ? a.nv + vh : vh;
      if (a.ba_interleaved) idx = kh * 2 * ratio + ((threadIdx.x & 1) ? ratio : 0) + rep;
      if (t < rows) ba_s[t][threadIdx.x & 1] = a.ba[(int64_t)t * a.ba_ld + idx];
    }
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int c = threadIdx.x + 256 * u;
      if (c < nch)
#pragma unroll
        for (int t = 0; t < kMaxRowsDn; t++) xin_s[t][c] = xin[t][u];
    }
  }
  const float ssm_a = L.ssm_a[vh], dt_bias = L.dt_bias[vh];
  float S[16];
  const float* sin_ = L.rec_state[cur] + (int64_t)vh * a.dk * a.dv;
#pragma unroll
  for (int r = 0; r < 16; r++) S[r] = r < rows_i ? sin_[(int64_t)(kr0 + r) * a.dv + j] : 0.f;
  const float qscale = __fdiv_rn(1.f, sqrtf((float)a.dk));
  const bool qk_writer = rep == 0 && slice == 0;
  __syncthreads();  // ba_s is written by threads 0..15 and read by thread 0

  for (int t = 0; t < rows; t++) {
    const int buf = t & 1;
    const int snap = (cur + 1 + t) % kStateRing;
    // causal depthwise conv + SiLU (src/qwen/quantized_deltanet.rs:733-759)
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int c = threadIdx.x + 256 * u;
      if (c < nch) {
        const float x = xin_s[t][c];
        float sum = __fmul_rn(cw[u][K - 1], x);
#pragma unroll
        for (int tp = 0; tp < K - 1; tp++) sum = __fadd_rn(sum, __fmul_rn(cw[u][tp], hist[u][tp]));
        qkv[buf][c] = __fmul_rn(sum, sigmoid_ref(sum));
#pragma unroll
        for (int tp = 0; tp + 1 < K - 1; tp++) hist[u][tp] = hist[u][tp + 1];
        if (K > 1) hist[u][K - 2] = x;
        if (c >= nqk || qk_writer) {
          float* co = L.conv_state[snap] + (int64_t)chan(c) * (K - 1);
#pragma unroll
          for (int tp = 0; tp < K - 1; tp++) co[tp] = hist[u][tp];
        }
      }
    }
    if (threadIdx.x == 0) {
      bg[buf][0] = sigmoid_ref(ba_s[t][0]);
      bg[buf][1] = __fmul_rn(ssm_a, softplus_ref(__fadd_rn(ba_s[t][1], dt_bias)));
    }
    __syncthreads();
    // L2 norms of q and k (x * (sum x^2 + 1e-6)^-1/2), every warp for itself
    const float* q = qkv[buf];
    const float* kk = qkv[buf] + a.dk;
    float sq = 0.f, sk = 0.f;
    for (int i = lane; i < a.dk; i += 32) {
      sq = fmaf(q[i], q[i], sq);
      sk = fmaf(kk[i], kk[i], sk);
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, m));
      sk = __fadd_rn(sk, __shfl_xor_sync(0xffffffffu, sk, m));
    }
    const float nq = __fdiv_rn(1.f, sqrtf(__fadd_rn(sq, 1e-6f)));
    const float nk = __fdiv_rn(1.f, sqrtf(__fadd_rn(sk, 1e-6f)));
    const float beta = bg[buf][0], decay = expf(bg[buf][1]);
    const float vcol = qkv[buf][nqk + CPW * warp + c4];
    // recurrence over this lane's key rows, reduced across the 8 row groups
    float kv[16], pred = 0.f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
      if (r < rows_i) {
        kv[r] = __fmul_rn(kk[kr0 + r], nk);
        S[r] = __fmul_rn(S[r], decay);
        pred = fmaf(S[r], kv[r], pred);
      }
    }
#pragma unroll
    for (int m = CPW; m <= 16; m <<= 1) pred = __fadd_rn(pred, __shfl_xor_sync(0xffffffffu, pred, m));
    const float delta = __fmul_rn(__fsub_rn(vcol, pred), beta);
    float o = 0.f;
    float* sout = L.rec_state[snap] + (int64_t)vh * a.dk * a.dv;
#pragma unroll
    for (int r = 0; r < 16; r++) {
      if (r < rows_i) {
        S[r] = fmaf(kv[r], delta, S[r]);
        o = fmaf(S[r], __fmul_rn(q[kr0 + r], nq), o);
        sout[(int64_t)(kr0 + r) * a.dv + j] = S[r];
      }
    }
#pragma unroll
    for (int m = CPW; m <= 16; m <<= 1) o = __fadd_rn(o, __shfl_xor_sync(0xffffffffu, o, m));
    if (rg == 0) a.out[(int64_t)t * a.out_ld + vh * a.dv + j] = __fmul_rn(o, qscale);
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
  if (a.rows < 1 || a.rows > kMaxRowsDn || a.rows >= kStateRing || a.dk > 128 || a.dk % 32 || a.dv % 32 ||
      a.conv_k > 4 || a.conv_k < 1)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  // 16 value columns per CTA: 2 CTAs per SM at 35B shapes, 8 key rows a lane
  const int cols = 16;
  cfg.gridDim = dim3(a.nv * (a.dv / cols), nlayers);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cols == 16) switch (a.conv_k) {
      case 1: return cudaLaunchKernelEx(&cfg, deltanet_kernel<1, 16>, a);
      case 2: return cudaLaunchKernelEx(&cfg, deltanet_kernel<2, 16>, a);
      case 3: return cudaLaunchKernelEx(&cfg, deltanet_kernel<3, 16>, a);
      default: return cudaLaunchKernelEx(&cfg, deltanet_kernel<4, 16>, a);
    }
  switch (a.conv_k) {
    case 1: return cudaLaunchKernelEx(&cfg, deltanet_kernel<1, 32>, a);
    case 2: return cudaLaunchKernelEx(&cfg, deltanet_kernel<2, 32>, a);
    case 3: return cudaLaunchKernelEx(&cfg, deltanet_kernel<3, 32>, a);
    default: return cudaLaunchKernelEx(&cfg, deltanet_kernel<4, 32>, a);
  }
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
