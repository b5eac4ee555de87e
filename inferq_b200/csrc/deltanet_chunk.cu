// deltanet_chunk.cu -- the chunked Gated DeltaNet recurrence for the rows of
// a wide pass that precede its final block.
//
// The sequential rule (src/qwen/deltanet.rs:122-217, per value head, state
// S [dk][dv]): S *= g_t; pred = S^T k_t; delta_t = beta_t (v_t - pred);
// S += k_t delta_t^T; o_t = S^T q_t / sqrt(dk).  Over a chunk of C rows
// starting from S0, with L_t = sum_{s<=t} log g_s and r(t,s) = exp(L_t - L_s):
//
//   delta_t = beta_t (v_t - e^{L_t} S0^T k_t) - sum_{s<t} beta_t r(t,s) (k_t.k_s) delta_s
//   o_t     = (e^{L_t} S0^T q_t + sum_{s<=t} r(t,s) (q_t.k_s) delta_s) / sqrt(dk)
//   S_C     = e^{L_{C-1}} S0 + sum_s r(C-1,s) k_s delta_s^T
//
// (the WY / UT form: the lower-triangular solve for delta runs as forward
// substitution).  This is the same arithmetic up to f32 rounding order, so
// the wide pass uses it where the reference's own prefill is not bitwise
// its split passes either (src/runtime.rs:740-747); decays enter only as
// exp of differences of the cumulative log-decay, never as a product that
// could underflow.  Every sum below has a fixed order, restated by the CPU
// oracle's wide order:
//   * dots over the key dimension (k_t.k_s, q_t.k_s): sequential in i;
//   * U_t = beta_t v_t - sum_{s<t} A[t][s] U_s and W_t = (beta_t e_t) k_t -
//     sum_{s<t} A[t][s] W_s (so delta = U - W S0), each sum in s order;
//   * W_t S0 and S0^T q_t per column: eight parts, part p the key rows
//     [p dk/8, (p+1) dk/8) in ascending order, combined as
//     ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7));
//   * the output sum over s: part p takes s = p (mod 8) in ascending order,
//     the parts combined by the same tree;
//   * the state update: e^{L_{C-1}} S0, then + (r k_s[i]) delta_s in s order.
//
// Four launches: per-row conv + SiLU, L2 norms, beta and log-decay (the
// sequential kernel's formulas, so these values are bitwise its own); per
// (head, 32-row chunk) at once, everything that does not depend on the state
// (A, M, the decays and the substitutions for U and W); the chunks in order
// per (head, 16 columns), only the state-dependent products; the gated
// RMSNorm of the rows.
#include <mutex>
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

constexpr int kChunk = 32;

__device__ __forceinline__ float sigmoid_c(float v) { return __fdiv_rn(1.f, __fadd_rn(1.f, exp_ref(-v))); }
__device__ __forceinline__ float softplus_c(float v) {
  if (v > 20.f) return v;
  if (v < -20.f) return exp_ref(v);
  return log1p_ref(exp_ref(v));
}

// grid (rows): conv + SiLU of every channel of row t (quantized_deltanet.rs:
// 733-759), L2 norms of its q and k heads (:724-731), beta = sigmoid(b) and
// log g = ssm_a * softplus(a + dt_bias) per value head.  The CTA of the last
// row also stores the conv history after the rows in conv slot cur + 1.
template <int K>
__global__ void __launch_bounds__(256) dn_prep_kernel(DeltaChunkArgs a) {
  extern __shared__ float y[];  // [conv_dim]
  __shared__ float nscale[64];
  const DeltaNetLayer& L = *a.layers;
  const int t = blockIdx.x;
  const int key_dim = a.nk * a.dk, conv_dim = 2 * key_dim + a.nv * a.dv;
  const int cur = *a.cur;
  const float* cin = L.conv_state[cur];
  for (int g = threadIdx.x; g < conv_dim; g += 256) {
    float w[4], h[3];
#pragma unroll
    for (int tp = 0; tp < K; tp++) w[tp] = L.conv_w[(int64_t)g * K + tp];
#pragma unroll
    for (int tp = 0; tp < K - 1; tp++) {
      const int r = t - (K - 1) + tp;  // the input row this history tap holds
      h[tp] = r >= 0 ? a.qkv[(int64_t)r * a.qkv_ld + g] : cin[(int64_t)g * (K - 1) + t + tp];
    }
    const float x = a.qkv[(int64_t)t * a.qkv_ld + g];
    float sum = __fmul_rn(w[K - 1], x);
#pragma unroll
    for (int tp = 0; tp < K - 1; tp++) sum = __fadd_rn(sum, __fmul_rn(w[tp], h[tp]));
    y[g] = __fmul_rn(sum, sigmoid_c(sum));
    if (t == a.rows - 1) {
      // the history after the last row: inputs t-K+2 .. t
      float* co = L.conv_state[(cur + 1) % kStateRing] + (int64_t)g * (K - 1);
#pragma unroll
      for (int tp = 0; tp < K - 1; tp++) {
        const int r = t - (K - 2) + tp;
        co[tp] = r >= 0 ? a.qkv[(int64_t)r * a.qkv_ld + g] : cin[(int64_t)g * (K - 1) + t + 1 + tp];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < 2 * a.nk) {  // q heads, then k heads
    const float* v = y + (threadIdx.x < a.nk ? threadIdx.x * a.dk : key_dim + (threadIdx.x - a.nk) * a.dk);
    float ss = 0.f;
    for (int i = 0; i < a.dk; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    nscale[threadIdx.x] = __fdiv_rn(1.f, sqrtf(__fadd_rn(ss, 1e-6f)));
  }
  __syncthreads();
  float* out = a.cv + (int64_t)t * conv_dim;
  for (int g = threadIdx.x; g < conv_dim; g += 256)
    out[g] = g < 2 * key_dim ? __fmul_rn(y[g], nscale[g / a.dk]) : y[g];
  const int ratio = a.nv / a.nk;
  for (int vh = threadIdx.x; vh < a.nv; vh += 256) {
    const int kh = a.tiled_heads ? vh % a.nk : vh / ratio;
    const int rep = a.tiled_heads ? vh / a.nk : vh % ratio;
    int bi = vh, ai = a.nv + vh;
    if (a.ba_interleaved) {
      bi = kh * 2 * ratio + rep;
      ai = kh * 2 * ratio + ratio + rep;
    }
    const float b = a.ba[(int64_t)t * a.ba_ld + bi], al = a.ba[(int64_t)t * a.ba_ld + ai];
    a.bl[(int64_t)t * 2 * a.nv + vh] = sigmoid_c(b);
    a.bl[(int64_t)t * 2 * a.nv + a.nv + vh] = __fmul_rn(L.ssm_a[vh], softplus_c(__fadd_rn(al, L.dt_bias[vh])));
  }
}

// Sum of the eight parts of a column (lanes 8c .. 8c+7):
// ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)); every lane of the group gets it.
__device__ __forceinline__ float parts_sum(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
  return v;
}

// Per (value head, chunk), independent of the state (every chunk of every
// head at once): the cumulative log-decay L, e_t = e^{L_t},
// w_s = r(C-1, s), M[t][s] = r(t,s) q_t.k_s (s <= t), A[t][s] =
// beta_t r(t,s) k_t.k_s (s < t), and the forward substitutions
//   U_t = beta_t v_t - sum_{s<t} A[t][s] U_s      (dv columns)
//   W_t = (beta_t e_t) k_t - sum_{s<t} A[t][s] W_s (dk columns)
// so that the chunk's deltas are U - W S0.  grid (nv, chunks), 256 threads.
template <int DK>
__global__ void __launch_bounds__(256) dn_wy_kernel(DeltaChunkArgs a) {
  constexpr int KS = DK + 1;
  extern __shared__ float sm[];
  float* Ks = sm;                   // [kChunk][KS]
  float* Qs = Ks + kChunk * KS;     // [kChunk][KS]
  float* A = Qs + kChunk * KS;      // [kChunk][kChunk]
  float* Ls = A + kChunk * kChunk;  // [kChunk]
  float* Bs = Ls + kChunk;          // [kChunk] beta
  float* Es = Bs + kChunk;          // [kChunk]
  const int vh = blockIdx.x, ch = blockIdx.y, DV = a.dv;
  const int c0 = ch * kChunk, C = min(kChunk, a.rows - c0);
  const int ratio = a.nv / a.nk;
  const int kh = a.tiled_heads ? vh % a.nk : vh / ratio;
  const int key_dim = a.nk * DK, conv_dim = 2 * key_dim + a.nv * DV;
  const int64_t hc = (int64_t)vh * gridDim.y + ch;  // (head, chunk) record
  for (int e = threadIdx.x; e < C * DK; e += 256) {
    const int t = e / DK, i = e % DK;
    const float* row = a.cv + (int64_t)(c0 + t) * conv_dim;
    Qs[t * KS + i] = row[kh * DK + i];
    Ks[t * KS + i] = row[key_dim + kh * DK + i];
  }
  if (threadIdx.x == 0) {
    float l = 0.f;
    for (int t = 0; t < C; t++) {
      l = __fadd_rn(l, a.bl[(int64_t)(c0 + t) * 2 * a.nv + a.nv + vh]);
      Ls[t] = l;
      Es[t] = exp_ref(l);
      Bs[t] = a.bl[(int64_t)(c0 + t) * 2 * a.nv + vh];
    }
  }
  __syncthreads();
  float* ew = a.wy_ew + hc * 2 * kChunk;  // [e | w]
  if (threadIdx.x < C) {
    ew[threadIdx.x] = Es[threadIdx.x];
    ew[kChunk + threadIdx.x] = exp_ref(__fsub_rn(Ls[C - 1], Ls[threadIdx.x]));
  }
  float* Mg = a.wy_m + hc * kChunk * kChunk;
  {
    // q_t.k_s and k_t.k_s for a 2 x 2 tile of (t, s) per thread, each sum
    // over i in order
    const int tt = (threadIdx.x >> 4) * 2, ss = (threadIdx.x & 15) * 2;
    float qk[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, kk[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    if (tt < C && ss <= tt + 1 && ss < C) {
#pragma unroll 8
      for (int i = 0; i < DK; i++) {
        const float q0 = Qs[tt * KS + i], q1 = Qs[(tt + 1) * KS + i];
        const float k0 = Ks[tt * KS + i], k1 = Ks[(tt + 1) * KS + i];
        const float s0 = Ks[ss * KS + i], s1 = Ks[(ss + 1) * KS + i];
        qk[0][0] = __fadd_rn(qk[0][0], __fmul_rn(q0, s0));
        qk[0][1] = __fadd_rn(qk[0][1], __fmul_rn(q0, s1));
        qk[1][0] = __fadd_rn(qk[1][0], __fmul_rn(q1, s0));
        qk[1][1] = __fadd_rn(qk[1][1], __fmul_rn(q1, s1));
        kk[0][0] = __fadd_rn(kk[0][0], __fmul_rn(k0, s0));
        kk[0][1] = __fadd_rn(kk[0][1], __fmul_rn(k0, s1));
        kk[1][0] = __fadd_rn(kk[1][0], __fmul_rn(k1, s0));
        kk[1][1] = __fadd_rn(kk[1][1], __fmul_rn(k1, s1));
      }
    }
#pragma unroll
    for (int x = 0; x < 2; x++)
#pragma unroll
      for (int y = 0; y < 2; y++) {
        const int t = tt + x, s2 = ss + y;
        float m = 0.f, aa = 0.f;
        if (t < C && s2 <= t) {
          const float r = exp_ref(__fsub_rn(Ls[t], Ls[s2]));
          m = __fmul_rn(r, qk[x][y]);
          if (s2 < t) aa = __fmul_rn(__fmul_rn(Bs[t], r), kk[x][y]);
        }
        Mg[t * kChunk + s2] = m;
        A[t * kChunk + s2] = aa;
      }
  }
  __syncthreads();
  // forward substitution, one column per thread: U (dv) then W (dk)
  float* Xs = Es + kChunk;  // [kChunk][dv + dk]
  const int XW = DV + DK;
  for (int col = threadIdx.x; col < XW; col += 256) {
    const bool isu = col < DV;
    for (int t = 0; t < C; t++) {
      const float y = isu ? __fmul_rn(Bs[t], a.cv[(int64_t)(c0 + t) * conv_dim + 2 * key_dim + vh * DV + col])
                          : __fmul_rn(__fmul_rn(Bs[t], Es[t]), Ks[t * KS + col - DV]);
      float acc = 0.f;
      for (int s2 = 0; s2 < t; s2++) acc = __fadd_rn(acc, __fmul_rn(A[t * kChunk + s2], Xs[s2 * XW + col]));
      Xs[t * XW + col] = __fsub_rn(y, acc);
    }
  }
  __syncthreads();
  float* X = a.wy_x + hc * kChunk * XW;  // [t][dv | dk]
  for (int e = threadIdx.x; e < C * XW; e += 256) X[e] = Xs[e];
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kSeqCols = 16;  // value columns per CTA of the in-order kernel
// A staged q / k / W row, part-major: part p (key rows [p dk/8, (p+1) dk/8))
// at p * (dk/8 + 4), so a lane reads its part as 16-byte words and the eight
// parts of a column fall in distinct bank groups.
__host__ __device__ constexpr int seq_row_floats(int dk) { return 8 * (dk / 8 + 4); }
// shared floats of one staged chunk: q, k, W rows, M, e | w, U columns
__host__ __device__ constexpr int seq_buf_floats(int dk) {
  return 3 * kChunk * seq_row_floats(dk) + kChunk * kChunk + 2 * kChunk + kChunk * kSeqCols;
}

// The chunks in order, CTA (value head, 16 columns), 128 threads: warp w owns
// columns 4w .. 4w+3 of the CTA's 16; lane = 8 * column + part.  Part p
// holds key rows [p dk/8, (p+1) dk/8) of its column of the state in
// registers (S[ii] is row p dk/8 + ii).  Per chunk: delta_t = U_t - W_t S0 and
// S0^T q_t (eight parts), o_t = (e_t S0^T q_t + sum_{s<=t} M[t][s] delta_s)
// / sqrt(dk), then the state update.  A chunk's rows are staged by cp.async
// (one buffer, so two CTAs fit per SM).
template <int DK>
__global__ void __launch_bounds__(128, 2) dn_seq_kernel(DeltaChunkArgs a) {
  constexpr int KP = DK / 8;
  constexpr int KS = seq_row_floats(DK);  // staged row stride
  constexpr int PS = KP + 4;              // part stride within a row
  constexpr int CW = kSeqCols;
  constexpr int BUF = seq_buf_floats(DK);
  extern __shared__ __align__(16) float sm[];
  float* D = sm + BUF;         // [kChunk][CW] delta
  float* Rs = D + kChunk * CW; // [kChunk][CW] S0^T q
  const DeltaNetLayer& L = *a.layers;
  const int vh = blockIdx.x, DV = a.dv;
  const int ratio = a.nv / a.nk;
  const int kh = a.tiled_heads ? vh % a.nk : vh / ratio;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = lane & 7, cl = 4 * warp + (lane >> 3);
  const int col0 = blockIdx.y * CW, col = col0 + cl;
  const int key_dim = a.nk * DK, conv_dim = 2 * key_dim + a.nv * DV;
  const int nch = (a.rows + kChunk - 1) / kChunk;
  const int XW = DV + DK;
  auto stage = [&](int ch) {
    float* b = sm;
    float *Qs = b, *Ks = Qs + kChunk * KS, *Wr = Ks + kChunk * KS, *M = Wr + kChunk * KS;
    float *Ew = M + kChunk * kChunk, *Us = Ew + 2 * kChunk;
    const int c0 = ch * kChunk, C = min(kChunk, a.rows - c0);
    const int64_t hc = (int64_t)vh * nch + ch;
    const float* X = a.wy_x + hc * kChunk * XW;
    for (int e = threadIdx.x; e < C * (DK / 4); e += 128) {
      const int t = e / (DK / 4), i = 4 * (e % (DK / 4));
      const int d = t * KS + (i / KP) * PS + i % KP;  // part-major position of element i
      const float* row = a.cv + (int64_t)(c0 + t) * conv_dim;
      cp_async16(Qs + d, row + kh * DK + i);
      cp_async16(Ks + d, row + key_dim + kh * DK + i);
      cp_async16(Wr + d, X + (int64_t)t * XW + DV + i);
    }
    for (int e = threadIdx.x; e < kChunk * kChunk / 4; e += 128)
      cp_async16(M + 4 * e, a.wy_m + hc * kChunk * kChunk + 4 * e);
    if (threadIdx.x < 2 * kChunk / 4) cp_async16(Ew + 4 * threadIdx.x, a.wy_ew + hc * 2 * kChunk + 4 * threadIdx.x);
    for (int e = threadIdx.x; e < C * (CW / 4); e += 128) {
      const int t = e / (CW / 4), c = 4 * (e % (CW / 4));
      cp_async16(Us + t * CW + c, X + (int64_t)t * XW + col0 + c);
    }
    cp_async_commit();
  };
  float* base = L.rec_state + (int64_t)vh * DK * DV + col;
  float S[KP];
#pragma unroll
  for (int ii = 0; ii < KP; ii++) S[ii] = base[(int64_t)(p * KP + ii) * DV];
  // replay the committed rows of the previous pass (S = S g + k delta)
  const int pend = *a.pending;
  const float* rec_head = L.rec_log + (int64_t)vh * kMaxRowsDelta * a.rec_stride;
  for (int r = 0; r < pend; r++) {
    const float* rc = rec_head + (int64_t)r * a.rec_stride;
    const float decay = rc[DK + DV], delta = rc[DK + col];
#pragma unroll
    for (int ii = 0; ii < KP; ii++) S[ii] = __fadd_rn(__fmul_rn(S[ii], decay), __fmul_rn(rc[p * KP + ii], delta));
  }
  const float qscale = __fdiv_rn(1.f, sqrtf((float)DK));
  for (int ch = 0; ch < nch; ch++) {
    const int c0 = ch * kChunk, C = min(kChunk, a.rows - c0);
    stage(ch);
    cp_async_wait<0>();
    __syncthreads();
    const float* b = sm;
    const float *Qs = b, *Ks = Qs + kChunk * KS, *Wr = Ks + kChunk * KS, *M = Wr + kChunk * KS;
    const float *Ew = M + kChunk * kChunk, *Us = Ew + 2 * kChunk;
#pragma unroll 4
    for (int t = 0; t < C; t++) {
      const float4* wt = reinterpret_cast<const float4*>(Wr + t * KS + p * PS);
      const float4* qt = reinterpret_cast<const float4*>(Qs + t * KS + p * PS);
      float pw = 0.f, pq = 0.f;
#pragma unroll
      for (int i4 = 0; i4 < KP / 4; i4++) {
        const float4 w4 = wt[i4], q4 = qt[i4];
        const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          pw = __fadd_rn(pw, __fmul_rn(S[4 * i4 + e], wv[e]));
          pq = __fadd_rn(pq, __fmul_rn(S[4 * i4 + e], qv[e]));
        }
      }
      pw = parts_sum(pw);
      pq = parts_sum(pq);
      if (p == 0) {
        D[t * CW + cl] = __fsub_rn(Us[t * CW + cl], pw);
        Rs[t * CW + cl] = pq;
      }
    }
    __syncwarp();
#pragma unroll 4
    for (int t = 0; t < C; t++) {
      float os = 0.f;
      for (int s2 = p; s2 <= t; s2 += 8) os = __fadd_rn(os, __fmul_rn(M[t * kChunk + s2], D[s2 * CW + cl]));
      const float o = __fmul_rn(qscale, __fadd_rn(__fmul_rn(Ew[t], Rs[t * CW + cl]), parts_sum(os)));
      if (p == 0) a.o[(int64_t)(c0 + t) * a.o_ld + vh * DV + col] = o;
    }
    // S = e^{L_{C-1}} S + sum_s (r(C-1,s) k_s[i]) delta_s
    const float eC = Ew[C - 1];
#pragma unroll
    for (int ii = 0; ii < KP; ii++) S[ii] = __fmul_rn(eC, S[ii]);
    for (int s2 = 0; s2 < C; s2++) {
      const float ws = Ew[kChunk + s2], ds = D[s2 * CW + cl];
      const float4* ks = reinterpret_cast<const float4*>(Ks + s2 * KS + p * PS);
#pragma unroll
      for (int i4 = 0; i4 < KP / 4; i4++) {
        const float4 k4 = ks[i4];
        const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; e++) S[4 * i4 + e] = __fadd_rn(S[4 * i4 + e], __fmul_rn(__fmul_rn(ws, kv[e]), ds));
      }
    }
    __syncthreads();  // the staged rows are read before the next chunk's copies land
  }
#pragma unroll
  for (int ii = 0; ii < KP; ii++) base[(int64_t)(p * KP + ii) * DV] = S[ii];
}

// grid (rows): the gated RMSNorm of every value head of row t
// (src/qwen/norm.rs:16-25), the sequential kernel's formula.
__global__ void __launch_bounds__(256) dn_gated_kernel(DeltaChunkArgs a) {
  __shared__ float den[128];
  const int t = blockIdx.x;
  const float* o = a.o + (int64_t)t * a.o_ld;
  for (int vh = threadIdx.x; vh < a.nv; vh += 256) {
    float ss = 0.f;
    for (int i = 0; i < a.dv; i++) ss = __fadd_rn(ss, __fmul_rn(o[vh * a.dv + i], o[vh * a.dv + i]));
    den[vh] = sqrtf(__fadd_rn(__fmul_rn(ss, a.inv_dv), a.eps));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.nv * a.dv; e += 256) {
    const float zz = a.z[(int64_t)t * a.z_ld + e];
    const float silu = __fdiv_rn(zz, __fadd_rn(1.f, exp_ref(-zz)));
    a.g_out[(int64_t)t * a.g_ld + e] =
        __fmul_rn(__fmul_rn(__fdiv_rn(o[e], den[e / a.dv]), a.norm_w[e % a.dv]), silu);
  }
}

size_t wy_smem(int dk) {
  return (size_t)(2 * kChunk * (dk + 1) + kChunk * kChunk + 3 * kChunk + kChunk * (128 + dk)) * sizeof(float);
}
size_t seq_smem(int dk) { return (size_t)(seq_buf_floats(dk) + 2 * kChunk * kSeqCols) * sizeof(float); }

template <int DK>
cudaError_t launch_chunk(const DeltaChunkArgs& a, cudaStream_t st) {
  static std::mutex mu;
  static bool done[64] = {};
  const cudaError_t e = once_per_device(done, mu, [] {
    cudaError_t r = cudaFuncSetAttribute(dn_wy_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)wy_smem(DK));
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(dn_seq_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)seq_smem(DK));
  });
  if (e != cudaSuccess) return e;
  const int nch = (a.rows + kChunk - 1) / kChunk;
  dn_wy_kernel<DK><<<dim3(a.nv, nch), 256, wy_smem(DK), st>>>(a);
  cudaError_t r = cudaGetLastError();
  if (r != cudaSuccess) return r;
  dn_seq_kernel<DK><<<dim3(a.nv, a.dv / kSeqCols), 128, seq_smem(DK), st>>>(a);
  return cudaGetLastError();
}

template <int K>
cudaError_t launch_prep(const DeltaChunkArgs& a, size_t smem, cudaStream_t st) {
  static std::mutex mu;
  static bool done[64] = {};
  const cudaError_t e = once_per_device(done, mu, [] {
    return cudaFuncSetAttribute(dn_prep_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (e != cudaSuccess) return e;
  dn_prep_kernel<K><<<a.rows, 256, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool deltanet_chunk_supported(int nk, int nv, int dk, int dv, int conv_k) {
  return (dk == 64 || dk == 128) && dv % 16 == 0 && dv >= 16 && dv <= 128 && nv <= 128 && 2 * nk <= 64 && conv_k >= 2 &&
         conv_k <= 4 && (size_t)(2 * nk * dk + nv * dv) * 4 <= 200 * 1024;
}

cudaError_t deltanet_chunk_launch(const DeltaChunkArgs& a, cudaStream_t st) {
  if (a.rows < 1 || !deltanet_chunk_supported(a.nk, a.nv, a.dk, a.dv, a.conv_k) ||
      a.rec_stride != deltanet_rec_stride(a.dk, a.dv) || !a.cv || !a.bl || !a.o || !a.g_out || !a.z || !a.norm_w ||
      !a.wy_x || !a.wy_m || !a.wy_ew)
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)(2 * a.nk * a.dk + a.nv * a.dv) * sizeof(float);
  cudaError_t e;
  switch (a.conv_k) {
    case 2: e = launch_prep<2>(a, smem, st); break;
    case 3: e = launch_prep<3>(a, smem, st); break;
    default: e = launch_prep<4>(a, smem, st); break;
  }
  if (e != cudaSuccess) return e;
  e = a.dk == 128 ? launch_chunk<128>(a, st) : launch_chunk<64>(a, st);
  if (e != cudaSuccess) return e;
  dn_gated_kernel<<<a.rows, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace iq
