// head.cu -- token embedding, greedy argmax over the LM-head logits, the
// on-device speculative accept, and the end-of-pass commit.
//
// argmax restates src/sampling.rs:104-112: non-finite logits are skipped and
// ties resolve to the LAST maximal index (Iterator::max_by).  The accept
// restates src/runtime.rs:2225-2236 (accepted_draft_prefix) and :1753-1755:
// the longest prefix of drafts equal to the argmax of the row before them,
// then the authoritative token = argmax of row `accepted`.
// The MTP confidence of row 0 restates top1_with_scores (:2245-2265): the
// top-1/top-2 logit margin and p(top1) = 1 / sum(exp(l - peak)).
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

__global__ void __launch_bounds__(256) embed_kernel(int dt, const uint8_t* __restrict__ w, int64_t row_bytes,
                                                    int cols, const int32_t* __restrict__ tokens, float* out,
                                                    int out_ld) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const uint8_t* row = w + (int64_t)tokens[t] * row_bytes;
  const int nb = cols / gguf_block_elems(dt);
  for (int e = threadIdx.x; e < cols; e += blockDim.x) out[(int64_t)t * out_ld + e] = dev_weight(dt, row, nb, e);
}

struct Best {
  float v;    // best value (-inf when nothing finite)
  int i;      // its index (-1 when none)
  float v2;   // best value at any other index
  float se;   // sum over finite values of exp(l - v)
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i > bi);
}

__device__ __forceinline__ Best merge(Best a, Best b, bool scores) {
  Best r;
  if (b.i >= 0 && (a.i < 0 || better(b.v, b.i, a.v, a.i))) {
    r.v = b.v; r.i = b.i;
    r.v2 = fmaxf(b.v2, a.v);
  } else {
    r.v = a.v; r.i = a.i;
    r.v2 = fmaxf(a.v2, b.i >= 0 ? b.v : -INFINITY);
  }
  if (scores) {
    const float ea = a.i >= 0 ? __fmul_rn(a.se, exp_ref(a.v - r.v)) : 0.f;
    const float eb = b.i >= 0 ? __fmul_rn(b.se, exp_ref(b.v - r.v)) : 0.f;
    r.se = __fadd_rn(ea, eb);
  } else {
    r.se = 0.f;
  }
  return r;
}

__device__ Best block_best(Best b, bool scores) {
  __shared__ Best red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    Best x;
    x.v = __shfl_xor_sync(0xffffffffu, b.v, o);
    x.i = __shfl_xor_sync(0xffffffffu, b.i, o);
    x.v2 = __shfl_xor_sync(0xffffffffu, b.v2, o);
    x.se = __shfl_xor_sync(0xffffffffu, b.se, o);
    b = (lane & o) ? merge(x, b, scores) : merge(b, x, scores);
  }
  __syncthreads();
  if (lane == 0) red[warp] = b;
  __syncthreads();
  Best r = red[0];
  for (int w = 1; w < 8; w++) r = merge(r, red[w], scores);
  return r;
}

// grid (rows, nparts): each CTA reduces a contiguous slice of one row.
__global__ void __launch_bounds__(256) argmax_part_kernel(HeadArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, part = blockIdx.y;
  const bool scores = a.scores != nullptr && t == 0;
  const int64_t per = (a.vocab + a.nparts - 1) / a.nparts;
  const int64_t lo = part * per, hi = lo + per < a.vocab ? lo + per : (int64_t)a.vocab;
  const float* l = a.logits + (int64_t)t * a.logits_ld;
  Best b = {-INFINITY, -1, -INFINITY, 0.f};
  for (int64_t i = lo + threadIdx.x; i < hi; i += 256) {
    const float v = l[i];
    if (!isfinite(v)) continue;
    Best x = {v, (int)i, -INFINITY, 1.f};
    b = merge(b, x, scores);
  }
  b = block_best(b, scores);
  if (threadIdx.x == 0) {
    a.part_val[(t * a.nparts + part) * 3 + 0] = b.v;
    a.part_val[(t * a.nparts + part) * 3 + 1] = b.v2;
    a.part_val[(t * a.nparts + part) * 3 + 2] = b.se;
    a.part_idx[t * a.nparts + part] = b.i;
  }
}

// grid (rows): the argmax of each of many rows (the wide pass), one CTA per
// row with the same comparison (better(): the tie rule) as the split form.
__global__ void __launch_bounds__(256) rows_argmax_kernel(const float* __restrict__ logits, int64_t ld, int vocab,
                                                          int* __restrict__ out) {
  const int t = blockIdx.x;
  const float* l = logits + (int64_t)t * ld;
  Best b = {-INFINITY, -1, -INFINITY, 0.f};
  const bool vec = ((ld | vocab) & 3) == 0 && (((uintptr_t)logits & 15) == 0);
  const int n4 = vec ? vocab / 4 : 0;
  for (int i0 = threadIdx.x; i0 < n4; i0 += 256 * 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (i0 + 256 * u < n4) v[u] = reinterpret_cast<const float4*>(l)[i0 + 256 * u];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      if (i0 + 256 * u >= n4) break;
      const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        if (!isfinite(e[q])) continue;
        Best x = {e[q], 4 * (i0 + 256 * u) + q, -INFINITY, 1.f};
        b = merge(b, x, false);
      }
    }
  }
  for (int i = 4 * n4 + threadIdx.x; i < vocab; i += 256) {
    const float v = l[i];
    if (!isfinite(v)) continue;
    Best x = {v, i, -INFINITY, 1.f};
    b = merge(b, x, false);
  }
  b = block_best(b, false);
  if (threadIdx.x == 0) out[t] = b.i < 0 ? 0 : b.i;  // no finite logit: token 0, a valid id
}

// One CTA: final argmax per row, then accept and the authoritative token.
__global__ void __launch_bounds__(256) accept_kernel(HeadArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ int am[8];
  for (int t = 0; t < a.rows; t++) {
    const bool scores = a.scores != nullptr && t == 0;
    Best b = {-INFINITY, -1, -INFINITY, 0.f};
    for (int p = threadIdx.x; p < a.nparts; p += 256) {
      Best x;
      x.v = a.part_val[(t * a.nparts + p) * 3 + 0];
      x.v2 = a.part_val[(t * a.nparts + p) * 3 + 1];
      x.se = a.part_val[(t * a.nparts + p) * 3 + 2];
      x.i = a.part_idx[t * a.nparts + p];
      b = merge(b, x, scores);
    }
    b = block_best(b, scores);
    if (threadIdx.x == 0) {
      const int bi = b.i < 0 ? 0 : b.i;  // no finite logit: token 0, a valid id
      am[t] = bi;
      a.argmax[t] = bi;
      if (scores) {
        a.scores[0] = b.v - b.v2;
        a.scores[1] = __fdiv_rn(1.f, b.se);
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int accepted = 0;
    if (a.verify)
      while (accepted + 1 < a.rows && am[accepted] == a.tokens[accepted + 1]) accepted++;
    const int last = a.verify ? accepted : a.rows - 1;
    a.result[0] = accepted;
    a.result[1] = am[last];
    a.result[2] = a.verify ? accepted + 1 : a.rows;
  }
}

// Keep the first result[2] rows of the pass: advance the DeltaNet state ring
// to the state after that row and the KV position past it.
__global__ void commit_kernel(int* cur, int* pos, int* pending, const int* result) {
  pdl_wait();
  pdl_trigger();
  *cur = (*cur + result[2]) % kStateRing;
  *pos += result[2];
  *pending = result[2];
}

// One MTP draft step's bookkeeping: the drafted token (row 0's argmax)
// becomes the next step's input token, its scores and token are recorded at
// slot `i`, and the normalized hidden row becomes the next step's hidden
// input (the block itself already advanced the MTP KV position).
__global__ void __launch_bounds__(256) mtp_step_kernel(MtpStepArgs a) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    const int tok = a.result[1];
    a.tokens[0] = tok;
    a.out_tok[a.i] = tok;
    a.out_margin[a.i] = a.scores[0];
    a.out_prob[a.i] = a.scores[1];
  }
  for (int j = threadIdx.x; j < a.hidden; j += 256) a.hin[j] = a.xn[j];
}

__global__ void set_int_kernel(int* p, int v, int add) {
  pdl_wait();
  pdl_trigger();
  *p = add ? *p + v : v;
}

}  // namespace

cudaError_t mtp_step_launch(const MtpStepArgs& a, cudaStream_t st, bool pdl) {
  return launch_pdl(mtp_step_kernel, dim3(1), dim3(256), 0, st, pdl, a);
}

cudaError_t set_int_launch(int* p, int v, bool add, cudaStream_t st, bool pdl) {
  return launch_pdl(set_int_kernel, dim3(1), dim3(1), 0, st, pdl, p, v, add ? 1 : 0);
}

cudaError_t embed_launch(int dt, const uint8_t* w, int64_t row_bytes, int cols, const int32_t* tokens, int rows,
                         float* out, int out_ld, cudaStream_t st, bool pdl) {
  return launch_pdl(embed_kernel, dim3(rows), dim3(256), 0, st, pdl, dt, w, row_bytes, cols, tokens, out, out_ld);
}

cudaError_t argmax_launch(const HeadArgs& a, cudaStream_t st, bool pdl) {
  return launch_pdl(argmax_part_kernel, dim3(a.rows, a.nparts), dim3(256), 0, st, pdl, a);
}

cudaError_t rows_argmax_launch(const float* logits, int64_t ld, int rows, int vocab, int* out, cudaStream_t st) {
  if (rows < 1 || vocab < 1) return cudaErrorInvalidValue;
  rows_argmax_kernel<<<rows, 256, 0, st>>>(logits, ld, vocab, out);
  return cudaGetLastError();
}

cudaError_t accept_launch(const HeadArgs& a, cudaStream_t st, bool pdl) {
  if (a.rows > 8) return cudaErrorInvalidValue;
  return launch_pdl(accept_kernel, dim3(1), dim3(256), 0, st, pdl, a);
}

cudaError_t commit_launch(int* cur, int* pos, int* pending, const int* result, cudaStream_t st, bool pdl) {
  return launch_pdl(commit_kernel, dim3(1), dim3(1), 0, st, pdl, cur, pos, pending, result);
}

}  // namespace iq
