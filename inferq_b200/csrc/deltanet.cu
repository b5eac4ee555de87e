// deltanet.cu -- Gated DeltaNet mixer step for a pass of k rows.
//
// Restates src/qwen/quantized_deltanet.rs:517-703 (per-row causal depthwise
// conv + SiLU, per-key-head L2 norm, beta = sigmoid(b),
// g = ssm_a * softplus(a + dt_bias)) and the recurrence of
// src/qwen/deltanet.rs:122-217 (S *= exp(g); pred = S^T k;
// delta = (v - pred) * beta; S += k delta^T; o = sum_i S[i,:] q[i] / sqrt(dk)).
//
// Summation order is the reference's: every sum over key rows (pred, o) and
// over a head's elements (the L2 norms) runs sequentially from element 0,
// each product rounded before it is added (deltanet.rs:187-216,
// quantized_deltanet.rs:724-731).  So one thread owns one value column j and
// walks the dk key rows of S[:, j] in order, with the column in registers.
//
// Grid: one CTA per value head, 2 * dv threads: two walkers per value column
// j, each holding column j of the head's dk x dv state in registers (the
// key-row walks are fully unrolled) and applying the same updates.  Rows run
// in blocks of up to 8: the conv, the norms and beta/g of a block's rows are
// computed first by the whole CTA (they do not depend on the state); then,
// per row t, the output walker sums o(t) while the prediction walker sums
// pred(t+1) and hands delta(t+1) to its partner through shared memory (one
// CTA barrier per row).  Each scheduler thus holds two independent chains.
// A pass may hold any number of rows (the wide prefill hands a whole chunk
// to one launch); only its final block is kept for rollback.
//
// Rollback without state copies: the recurrent state is one buffer per layer
// (the state before the last pass) plus, per row of the last pass, an update
// record {normalized k, delta, decay} per value head.  A row's update is
// S = (S * decay) + k delta^T (two roundings per element), so replaying the
// first `pending` records reproduces the state after those rows bit for bit.
// The next pass replays the committed rows of the previous one into the base
// buffer before its own rows (ahead of the programmatic-dependency wait, so
// it overlaps the projection GEMV).  The conv state (small) keeps a ring of
// kStateRing buffers: a pass reads slot `cur` and writes the state after its
// row t to slot cur+1+t, and committing c rows moves `cur` by c.
#include <mutex>
#include "kernels.cuh"
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__device__ __forceinline__ float sigmoid_ref(float v) { return __fdiv_rn(1.f, __fadd_rn(1.f, exp_ref(-v))); }

__device__ __forceinline__ float softplus_ref(float v) {
  if (v > 20.f) return v;
  if (v < -20.f) return exp_ref(v);
  return log1p_ref(exp_ref(v));
}

// DK key rows, DV value columns per head (32 * warps), conv width K.
template <int DK, int DV, int K>
__global__ void __launch_bounds__(2 * DV) deltanet_kernel(DeltaNetArgs a) {
  constexpr int NT = 2 * DV;           // threads: the output and the prediction walker of each column
  constexpr int NCH = 2 * DK + DV;     // conv channels of this head: q | k | v
  constexpr int CPT = (NCH + NT - 1) / NT;
  constexpr int QS = DK + 4;           // padded row of q/k in shared memory
  constexpr int B = kMaxRowsDelta;     // rows per block
  const DeltaNetLayer& L = *a.layers;
  const int vh = blockIdx.x;
  const int ratio = a.nv / a.nk;
  const int kh = a.tiled_heads ? vh % a.nk : vh / ratio;
  const int rep = a.tiled_heads ? vh / a.nk : vh % ratio;
  const int tid = threadIdx.x, lane = tid & 31;
  const int j = tid % DV;              // value column of this thread
  const bool walker_o = tid < DV;      // the output walker (else the prediction walker)
  const int key_dim = a.nk * DK;
  const int rows = a.rows;
  const int rec_stride = a.rec_stride;
  float* rec_head = L.rec_log + (int64_t)vh * B * rec_stride;  // [row][k DK | delta DV | decay]
  float* base = L.rec_state + (int64_t)vh * DK * DV + j;

  // ---- before the dependency wait: state column, replay of the committed
  // rows of the previous pass, conv weights and history (none of them is
  // written by the kernels this pass runs before this one)
  extern __shared__ __align__(16) float rec_s[];  // [B][rec_stride]
  const int pend = *a.pending;
  float S[DK];  // column j of the head's state, key rows in order
#pragma unroll
  for (int i = 0; i < DK; i++) S[i] = base[(int64_t)i * DV];
  for (int e = tid; e < pend * rec_stride; e += NT) rec_s[e] = rec_head[e];
  __syncthreads();
  for (int r = 0; r < pend; r++) {
    const float* rc = rec_s + r * rec_stride;
    const float decay = rc[DK + DV], delta = rc[DK + j];
    const float4* k4 = reinterpret_cast<const float4*>(rc);
#pragma unroll
    for (int i4 = 0; i4 < DK / 4; i4++) {
      const float4 kv = k4[i4];
      const float kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int e = 0; e < 4; e++) S[4 * i4 + e] = __fadd_rn(__fmul_rn(S[4 * i4 + e], decay), __fmul_rn(kk[e], delta));
    }
  }
  const int cur = *a.cur;
  auto chan = [&](int c) {
    if (c < DK) return kh * DK + c;
    if (c < 2 * DK) return key_dim + kh * DK + (c - DK);
    return 2 * key_dim + vh * DV + (c - 2 * DK);
  };
  float cw[CPT][4], hist[CPT][3];
  const float* cin = L.conv_state[cur];
#pragma unroll
  for (int u = 0; u < CPT; u++) {
    const int c = tid + NT * u;
    const bool own = c < NCH;
    const int g = own ? chan(c) : 0;
#pragma unroll
    for (int tp = 0; tp < 4; tp++) cw[u][tp] = (own && tp < K) ? L.conv_w[(int64_t)g * K + tp] : 0.f;
#pragma unroll
    for (int tp = 0; tp < 3; tp++) hist[u][tp] = (own && tp < K - 1) ? cin[(int64_t)g * (K - 1) + tp] : 0.f;
  }
  const float ssm_a = L.ssm_a[vh], dt_bias = L.dt_bias[vh];
  // (the replay's reads of this head's records precede the record writes
  // below: every thread passes the CTA barriers in between)

  pdl_wait();
  pdl_trigger();

  __shared__ __align__(16) float qk[B][2][QS];  // conv outputs, then normalized q and k
  __shared__ float vs[B][DV];
  __shared__ float beta_s[B], decay_s[B];
  __shared__ __align__(16) float os[B][DV];  // recurrent outputs (fused gated norm)
  __shared__ float nscale[B][2];
  __shared__ float den_s[B];
  __shared__ float dsm[B][DV];  // delta of each row, from the prediction walker
  const bool qk_writer = rep == 0;
  const bool gated = a.q80 || a.g_out;
  const float qscale = __fdiv_rn(1.f, sqrtf((float)DK));
  // The final block of up to B rows keeps update records and conv slots so
  // that the pass can be rolled back inside it; the rows before it (a wide
  // pass's prefix) advance the state directly.  Conv slots: the history
  // after the prefix in slot0, after final row t in slot0 + 1 + t; slot0 is
  // cur + 1 when there is a prefix (never cur itself, which other heads may
  // still be reading: the ring holds cur, slot0 and B rows).
  const int last = rows > 0 ? (rows - 1) % B + 1 : 0;
  const int pre = rows - last;
  const int slot0 = pre > 0 ? (cur + 1) % kStateRing : cur;
  const int col = vh * DV + j;  // column of the gated output row

  for (int b0 = 0; b0 < rows; b0 += B) {
    const int nb = min(B, rows - b0);
    const bool fin = b0 == pre;
    if (fin && (pre > 0 || pend > 0) && walker_o) {
      // the state before the final block becomes the base the records apply to
#pragma unroll
      for (int i = 0; i < DK; i++) base[(int64_t)i * DV] = S[i];
    }
    if (fin && pre > 0) {
#pragma unroll
      for (int u = 0; u < CPT; u++) {
        const int c = tid + NT * u;
        if (c < NCH && (c >= 2 * DK || qk_writer)) {
          float* co = L.conv_state[slot0] + (int64_t)chan(c) * (K - 1);
#pragma unroll
          for (int tp = 0; tp < K - 1; tp++) co[tp] = hist[u][tp];
        }
      }
    }
    float zin[B];  // gate projections of this column (fused gated norm)
#pragma unroll
    for (int t = 0; t < B; t++) zin[t] = (gated && walker_o && t < nb) ? a.z[(int64_t)(b0 + t) * a.z_ld + col] : 0.f;
    // every input of the block requested before any arithmetic
    float xin[CPT][B];
#pragma unroll
    for (int u = 0; u < CPT; u++) {
      const int c = tid + NT * u;
      const bool own = c < NCH;
      const int g = own ? chan(c) : 0;
#pragma unroll
      for (int t = 0; t < B; t++) xin[u][t] = (own && t < nb) ? a.qkv[(int64_t)(b0 + t) * a.qkv_ld + g] : 0.f;
    }
    float bin = 0.f, ain = 0.f;
    if (tid < nb) {
      int bi = vh, ai = a.nv + vh;
      if (a.ba_interleaved) {
        bi = kh * 2 * ratio + rep;
        ai = kh * 2 * ratio + ratio + rep;
      }
      bin = a.ba[(int64_t)(b0 + tid) * a.ba_ld + bi];
      ain = a.ba[(int64_t)(b0 + tid) * a.ba_ld + ai];
    }
    // causal depthwise conv + SiLU per channel and row (quantized_deltanet.rs:733-759)
#pragma unroll
    for (int u = 0; u < CPT; u++) {
      const int c = tid + NT * u;
      if (c >= NCH) continue;
#pragma unroll
      for (int t = 0; t < B; t++) {
        if (t >= nb) break;
        const float x = xin[u][t];
        float sum = __fmul_rn(cw[u][K - 1], x);
#pragma unroll
        for (int tp = 0; tp < K - 1; tp++) sum = __fadd_rn(sum, __fmul_rn(cw[u][tp], hist[u][tp]));
        const float y = __fmul_rn(sum, sigmoid_ref(sum));
        if (c < 2 * DK) qk[t][c / DK][c % DK] = y;
        else vs[t][c - 2 * DK] = y;
#pragma unroll
        for (int tp = 0; tp + 1 < K - 1; tp++) hist[u][tp] = hist[u][tp + 1];
        if (K > 1) hist[u][K - 2] = x;
        if (fin && (c >= 2 * DK || qk_writer)) {
          float* co = L.conv_state[(slot0 + 1 + t) % kStateRing] + (int64_t)chan(c) * (K - 1);
#pragma unroll
          for (int tp = 0; tp < K - 1; tp++) co[tp] = hist[u][tp];
        }
      }
    }
    if (tid < nb) {
      beta_s[tid] = sigmoid_ref(bin);
      decay_s[tid] = exp_ref(__fmul_rn(ssm_a, softplus_ref(__fadd_rn(ain, dt_bias))));
    }
    __syncthreads();
    // L2 norms: x * (sum x^2 + 1e-6)^-1/2 with the sum in element order
    // (quantized_deltanet.rs:724-731); one thread per (row, q|k)
    if (tid < 2 * nb) {
      const float4* v4 = reinterpret_cast<const float4*>(qk[tid >> 1][tid & 1]);
      float ss = 0.f;
#pragma unroll 8
      for (int i4 = 0; i4 < DK / 4; i4++) {
        const float4 v = v4[i4];
        ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
        ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
        ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
        ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
      }
      nscale[tid >> 1][tid & 1] = __fdiv_rn(1.f, sqrtf(__fadd_rn(ss, 1e-6f)));
    }
    __syncthreads();
    for (int e = tid; e < nb * 2 * DK; e += NT) {
      const int t = e / (2 * DK), w = (e / DK) & 1, i = e % DK;
      qk[t][w][i] = __fmul_rn(qk[t][w][i], nscale[t][w]);
    }
    __syncthreads();
    if (fin) {
      // update records of the final block: normalized k and decay (delta below)
      for (int e = tid; e < nb * DK; e += NT) rec_head[(int64_t)(e / DK) * rec_stride + e % DK] = qk[e / DK][1][e % DK];
      if (tid < nb) rec_head[(int64_t)tid * rec_stride + DK + DV] = decay_s[tid];
    }

    // ---- the recurrence, state in registers.  Both walkers of column j hold
    // the column and apply the same updates (bitwise the same state); the
    // output walker sums row t's output, the prediction walker row t+1's
    // pred and hands delta(t+1) over through shared memory, one CTA barrier
    // per row.
    {
      const float decay = decay_s[0];
      const float4* k4 = reinterpret_cast<const float4*>(qk[0][1]);
      float pred = 0.f;
#pragma unroll
      for (int i4 = 0; i4 < DK / 4; i4++) {
        const float4 kv = k4[i4];
        const float kk[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          S[4 * i4 + e] = __fmul_rn(S[4 * i4 + e], decay);
          if (!walker_o) pred = __fadd_rn(pred, __fmul_rn(S[4 * i4 + e], kk[e]));
        }
      }
      if (!walker_o) {
        const float delta = __fmul_rn(__fsub_rn(vs[0][j], pred), beta_s[0]);
        dsm[0][j] = delta;
        if (fin) rec_head[DK + j] = delta;
      }
    }
    __syncthreads();
    for (int t = 0; t < nb; t++) {
      const float delta = dsm[t][j];
      // S += k delta^T, then the decay of row t+1 (the block's last row:
      // decay 1, an exact multiply)
      const bool more = t + 1 < nb;
      const float4* k4 = reinterpret_cast<const float4*>(qk[t][1]);
      const float decay = more ? decay_s[t + 1] : 1.f;
      // one instruction stream for both walkers (half the unrolled code):
      // sv = S + k delta, S' = sv decay; the output walker sums
      // (sv q) qscale, the prediction walker (S' n) * 1 -- multiplying by
      // one is exact, so each sum is bitwise its own formula
      const float4* w4 = reinterpret_cast<const float4*>(walker_o ? qk[t][0] : qk[more ? t + 1 : t][1]);
      const float s2 = walker_o ? qscale : 1.f;
      float acc = 0.f;
#pragma unroll
      for (int i4 = 0; i4 < DK / 4; i4++) {
        const float4 kv = k4[i4], wv = w4[i4];
        const float kk[4] = {kv.x, kv.y, kv.z, kv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float sv = __fadd_rn(S[4 * i4 + e], __fmul_rn(kk[e], delta));
          const float sn = __fmul_rn(sv, decay);
          acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(walker_o ? sv : sn, ww[e]), s2));
          S[4 * i4 + e] = sn;
        }
      }
      if (walker_o) {
        if (gated) os[t][j] = acc;
        else a.out[(int64_t)(b0 + t) * a.out_ld + col] = acc;
      } else if (more) {
        const float dn = __fmul_rn(__fsub_rn(vs[t + 1][j], acc), beta_s[t + 1]);
        dsm[t + 1][j] = dn;
        if (fin) rec_head[(int64_t)(t + 1) * rec_stride + DK + j] = dn;
      }
      __syncthreads();
    }
    if (gated) {
      // gated RMSNorm of this value head (src/qwen/norm.rs:16-25): the sum
      // of squares in element order, then norm(o) * w * silu(z),
      // z = g / (1 + e^-g); then Q8_0 quantization of each 32-column block
      // (one warp), as BlockQ8_0::from_float: d = amax / 127 (kept as f16),
      // q = round(x / d).
      __syncthreads();
      if (tid < nb) {
        const float4* o4 = reinterpret_cast<const float4*>(os[tid]);
        float ss = 0.f;
#pragma unroll 8
        for (int i4 = 0; i4 < DV / 4; i4++) {
          const float4 v = o4[i4];
          ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
          ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
          ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
          ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
        }
        den_s[tid] = sqrtf(__fadd_rn(__fmul_rn(ss, a.inv_dv), a.eps));
      }
      __syncthreads();
      if (walker_o) {
      const int grp = col >> 7, ig = col & 127;   // 128-element group, index inside it
      const int bb = ig >> 5, tq = ig & 31;
      const int qlane = ((tq & 15) >> 2) * 8 + bb * 2 + (tq >> 4);
      const int nbq = a.nv * DV / 32;
      const float wj = a.norm_w[j];
#pragma unroll
      for (int t = 0; t < B; t++) {
        if (t >= nb) break;
        const float zz = zin[t];
        const float silu = __fdiv_rn(zz, __fadd_rn(1.f, exp_ref(-zz)));
        const float g = __fmul_rn(__fmul_rn(__fdiv_rn(os[t][j], den_s[t]), wj), silu);
        if (a.g_out) {
          a.g_out[(int64_t)(b0 + t) * a.g_ld + col] = g;
          continue;
        }
        float amax = fabsf(g);
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        const float d = __fdiv_rn(amax, 127.f);
        const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
        uint8_t* row = a.q80 + (int64_t)(b0 + t) * a.q80_stride;
        row[grp * 128 + qlane * 4 + (tq & 3)] = (uint8_t)(int8_t)roundf(__fmul_rn(g, id));
        if (lane == 0) reinterpret_cast<float*>(row + (int64_t)nbq * 32)[col >> 5] = __half2float(__float2half_rn(d));
      }
      }
    }
    __syncthreads();  // the block's shared rows are read before the next block writes them
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
      const float silu = __fdiv_rn(zv[j][i], __fadd_rn(1.f, exp_ref(-zv[j][i])));
      v[j][i] = __fmul_rn(__fmul_rn(__fdiv_rn(v[j][i], den), wv[j][i]), silu);
    }
  }
  finish_row<MAXB>(v, nb, cols, a.q8k ? a.q8k + (int64_t)row * a.q8k_stride : nullptr,
                   a.q80 ? a.q80 + (int64_t)row * a.q80_stride : nullptr, nullptr, xs);
}

int deltanet_smem_bytes(int dk, int dv) {
  return kMaxRowsDelta * ((dk + dv + 1 + 3) / 4 * 4) * (int)sizeof(float);
}

template <int DK, int DV, int K>
cudaError_t deltanet_launch_one(const DeltaNetArgs& a, cudaLaunchConfig_t& cfg) {
  // the update records and the static rows exceed the default 48 KB at
  // 128 x 128: opt in once per device
  static std::mutex mu;
  static bool done[64] = {};
  const cudaError_t e = once_per_device(done, mu, [] {
    return cudaFuncSetAttribute(deltanet_kernel<DK, DV, K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                deltanet_smem_bytes(DK, DV));
  });
  if (e != cudaSuccess) return e;
  cfg.dynamicSmemBytes = deltanet_smem_bytes(DK, DV);
  return cudaLaunchKernelEx(&cfg, deltanet_kernel<DK, DV, K>, a);
}

template <int DK, int DV>
cudaError_t deltanet_launch_k(const DeltaNetArgs& a, cudaLaunchConfig_t& cfg) {
  switch (a.conv_k) {
    case 1: return deltanet_launch_one<DK, DV, 1>(a, cfg);
    case 2: return deltanet_launch_one<DK, DV, 2>(a, cfg);
    case 3: return deltanet_launch_one<DK, DV, 3>(a, cfg);
    default: return deltanet_launch_one<DK, DV, 4>(a, cfg);
  }
}

}  // namespace

int deltanet_rec_stride(int dk, int dv) { return (int)align_up(dk + dv + 1, 4); }

bool deltanet_supported(int dk, int dv) {
  // (dk 128 with dv 32 would hold too many conv inputs per thread)
  return (dk == 32 || dk == 64 || dk == 128) && (dv == 32 || dv == 64 || dv == 128) && !(dk == 128 && dv == 32);
}

cudaError_t deltanet_launch(const DeltaNetArgs& a, cudaStream_t st, bool pdl) {
  // any number of rows: the final block of up to kMaxRowsDelta keeps its
  // conv slots after cur and the slot of the prefix
  static_assert(kStateRing >= kMaxRowsDelta + 2, "the conv ring holds cur, the prefix slot and a final block");
  if (a.rows < 1 || !deltanet_supported(a.dk, a.dv) ||
      a.conv_k > 4 || a.conv_k < 1 || a.rec_stride != deltanet_rec_stride(a.dk, a.dv) ||
      (a.q80 && (!a.z || !a.norm_w || (a.nv * a.dv) % 128)) || (a.g_out && (a.q80 || !a.z || !a.norm_w)) ||
      !a.timeout_flag ||
      ((uintptr_t)a.layers & 7))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nv);
  cfg.blockDim = dim3(2 * a.dv);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
#define IQ_DN_CASE(dk_, dv_) \
  if (a.dk == dk_ && a.dv == dv_) return deltanet_launch_k<dk_, dv_>(a, cfg);
  IQ_DN_CASE(128, 128) IQ_DN_CASE(128, 64)
  IQ_DN_CASE(64, 128) IQ_DN_CASE(64, 64) IQ_DN_CASE(64, 32)
  IQ_DN_CASE(32, 128) IQ_DN_CASE(32, 64) IQ_DN_CASE(32, 32)
#undef IQ_DN_CASE
  return cudaErrorInvalidValue;
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
