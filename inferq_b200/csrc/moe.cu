// moe.cu -- router softmax/top-k, expert-union job tables, SwiGLU activation
// and the ordered combine of the sparse MoE block.
//
// Restates src/qwen/moe.rs:21-54 (softmax over the router logits, top-k by
// probability, renormalised weights) and src/qwen/quantized_moe.rs:237-460
// (grouped-by-expert execution: each distinct expert's weights are read once
// for every row routed to it; silu(g)*u with g/(1+exp(-g)); weighted sum in
// row -> route order, multiply then add; shared expert times
// sigmoid(x . selector) added after the routed sum).
#include <cstddef>
#include <mutex>
#include "model_kernels.cuh"
#include "devfns.cuh"

namespace iq {
namespace {

constexpr int kMaxRows = 8;
constexpr int kMaxExperts = 1024;

static_assert(offsetof(QmvJob, rowmap) % 8 == 0 && offsetof(QmvJob, outrow) % 8 == 0, "packed job maps");

// Write a job record straight to global memory (no local-memory staging):
// rowmap / outrow arrive packed, 8 bytes / 2 x 8 bytes.
__device__ __forceinline__ void put_job(QmvJob* j, const uint8_t* w, const void* tm, const void* tm_tail,
                                        int row_base, int64_t w_row_bytes, int dt, int rows, int cols, int ks,
                                        const uint8_t* act, int act_bytes, float* out, int out_ld, int n, int tile0,
                                        int act_nrows, uint64_t rowmap, uint64_t out_lo, uint64_t out_hi,
                                        int act_mode = kActQuantized) {
  j->w = w;
  j->tmap = tm;
  j->tmap_tail = tm_tail;
  j->row_base = row_base;
  j->act_mode = act_mode;
  j->act = act;
  j->out = out;
  j->resid = nullptr;
  j->w_row_bytes = w_row_bytes;
  j->act_row_bytes = act_bytes;
  j->out_ld = out_ld;
  j->dtype = dt;
  j->rows = rows;
  j->cols = cols;
  j->ksplit = ks;
  j->n = n;
  j->tile0 = tile0;
  j->act_nrows = act_nrows;
  j->epi = kEpiStore;
  *reinterpret_cast<uint64_t*>(j->rowmap) = rowmap;
  reinterpret_cast<uint64_t*>(j->outrow)[0] = out_lo;
  reinterpret_cast<uint64_t*>(j->outrow)[1] = out_hi;
}
__device__ __forceinline__ void pack_out(uint64_t& lo, uint64_t& hi, int n, int v) {
  const uint64_t x = (uint64_t)(uint16_t)v;
  if (n < 4) lo |= x << (16 * n);
  else hi |= x << (16 * (n - 4));
}

// Top-k routing of one row by one warp (moe.rs:21-54): softmax over the E
// logits (lane l holds experts l, l+32, ...), then top-k by repeated warp
// arg-max with equal probabilities ranking the lower expert first; lane 0
// leaves the experts in sel_e and their weights in sel_w (renormalized to sum
// to one when norm_topk).
template <int kPerLane>
__device__ __forceinline__ void route_row_warp(const float* lg, int E, int topk, int norm_topk, int lane, int* sel_e,
                                               float* sel_w) {
    float p[kPerLane];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPerLane; i++) {
      const int e = lane + 32 * i;
      // from L2 (the fused router's other CTAs wrote them during this launch)
      p[i] = e < E ? __ldcg(lg + e) : -INFINITY;
      mx = fmaxf(mx, p[i]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float den = 0.f;
#pragma unroll
    for (int i = 0; i < kPerLane; i++) {
      p[i] = lane + 32 * i < E ? exp_ref(p[i] - mx) : 0.f;
      den = __fadd_rn(den, p[i]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) den = __fadd_rn(den, __shfl_xor_sync(0xffffffffu, den, o));
#pragma unroll
    for (int i = 0; i < kPerLane; i++) {
      p[i] = lane + 32 * i < E ? __fdiv_rn(p[i], den) : -1.f;
      // a NaN probability (non-finite logits) ranks below every real one but
      // above the taken marker, so the selection always names valid experts
      if (p[i] != p[i]) p[i] = -0.5f;
    }
    for (int r = 0; r < topk; r++) {
      float best = -1.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < kPerLane; i++) {
        const int e = lane + 32 * i;
        if (p[i] > best) { best = p[i]; bi = e; }  // ascending e: ties keep the lower
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
#pragma unroll
      for (int i = 0; i < kPerLane; i++)
        if (lane + 32 * i == bi) p[i] = -1.f;
      if (lane == 0) { sel_e[r] = bi; sel_w[r] = best; }
    }
    __syncwarp();
    if (lane == 0) {
      float sum = 0.f;
      for (int r = 0; r < topk; r++) sum = __fadd_rn(sum, sel_w[r]);
      for (int r = 0; r < topk; r++) sel_w[r] = norm_topk ? __fdiv_rn(sel_w[r], sum) : sel_w[r];
    }
    __syncwarp();
}

// Routes of `rows` rows (warp per row): route_e / route_w [row][topk].
template <int kPerLane>
__global__ void __launch_bounds__(256) route_rows_kernel(const float* logits, int ld, int rows, int E, int topk,
                                                         int norm_topk, int* route_e, float* route_w) {
  __shared__ int se[8][16];
  __shared__ float sw[8][16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;
  route_row_warp<kPerLane>(logits + (int64_t)row * ld, E, topk, norm_topk, lane, se[warp], sw[warp]);
  if (lane < topk) {
    route_e[row * topk + lane] = se[warp][lane];
    route_w[row * topk + lane] = sw[warp][lane];
  }
}

// One CTA.  Warp t < rows routes row t with its probabilities in registers
// (lane l holds experts l, l+32, ...): top-k by repeated warp arg-max, equal
// probabilities ranking the lower expert first.  Then thread e owns experts
// [e*per, e*per+per), finds their rank in the ascending union with warp
// ballots, and writes the gate, up and down jobs of its resident ones.
template <int kPerLane>  // experts per lane: ceil(E / 32) rounded up to 8, 16 or 32
__device__ __forceinline__ void route_body(const MoeRouteArgs& a, const MoeRouteStatic& s) {
  __shared__ int sel_e[kMaxRows][16];
  __shared__ float sel_w[kMaxRows][16];
  __shared__ unsigned used[kMaxExperts / 32];
  __shared__ int wcount[2][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.experts;
  for (int i = threadIdx.x; i < kMaxExperts / 32; i += 256) used[i] = 0;
  __syncthreads();
  if (warp < a.rows) {
    route_row_warp<kPerLane>(a.logits + (int64_t)warp * a.logits_ld, E, a.topk, a.norm_topk, lane, sel_e[warp],
                             sel_w[warp]);
    if (lane == 0) {
      for (int r = 0; r < a.topk; r++) {
        a.route_expert[warp * a.topk + r] = sel_e[warp][r];
        a.route_weight[warp * a.topk + r] = sel_w[warp][r];
        atomicOr(&used[sel_e[warp][r] / 32], 1u << (sel_e[warp][r] % 32));
      }
    }
  }
  __syncthreads();
  // union ranks: thread-contiguous experts, warp ballots, then warp prefix
  const int per = (E + 255) / 256;
  int mine = 0, rmine = 0;
  for (int q = 0; q < per; q++) {
    const int e = threadIdx.x * per + q;
    if (e < E && ((used[e / 32] >> (e % 32)) & 1)) {
      mine++;
      if (e >= s.expert_lo && e < s.expert_hi) rmine++;
    }
  }
  int inc = mine, rinc = rmine;  // inclusive warp scans
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o), rv = __shfl_up_sync(0xffffffffu, rinc, o);
    if (lane >= o) { inc += v; rinc += rv; }
  }
  if (lane == 31) { wcount[0][warp] = inc; wcount[1][warp] = rinc; }
  __syncthreads();
  int base = 0, rbase = 0, total_union = 0, n_res = 0;
  for (int w = 0; w < 8; w++) {
    if (w < warp) { base += wcount[0][w]; rbase += wcount[1][w]; }
    total_union += wcount[0][w];
    n_res += wcount[1][w];
  }
  int rank = base + inc - mine;
  int res_rank = rbase + rinc - rmine;
  const int slots_routed = a.rows * a.topk;
  for (int q = 0; q < per; q++) {
    const int e = threadIdx.x * per + q;
    if (!(e < E && ((used[e / 32] >> (e % 32)) & 1))) continue;
    a.union_list[rank++] = e;
    if (e < s.expert_lo || e >= s.expert_hi) continue;
    const int le = e - s.expert_lo;
    const int ri = res_rank++;
    const bool q80 = s.gate_dt == Q8_0;
    const uint8_t* ain = q80 ? a.act_in80 : a.act_in8k;
    const int ab = q80 ? a.act_in80_bytes : a.act_in8k_bytes;
    uint64_t gmap = 0, dmap = 0, olo = 0, ohi = 0;
    int n = 0;
    for (int t = 0; t < a.rows; t++)
      for (int r = 0; r < a.topk; r++)
        if (sel_e[t][r] == e) {
          const int slot = t * a.topk + r;
          gmap |= (uint64_t)t << (8 * n);
          dmap |= (uint64_t)slot << (8 * n);
          pack_out(olo, ohi, n, slot);
          n++;
        }
    put_job(&a.gu_jobs[2 * ri], s.gate + le * s.gate_stride, s.gate_tm, s.gate_tm_tail, le * a.ffn,
            s.gate_row_bytes, s.gate_dt, a.ffn, a.hidden, s.ks_gate, ain, ab, a.gu_out, a.gu_ld, n,
            2 * ri * s.tiles_gate, a.rows, gmap, olo, ohi);
    put_job(&a.gu_jobs[2 * ri + 1], s.up + le * s.up_stride, s.up_tm, s.up_tm_tail, le * a.ffn, s.gate_row_bytes,
            s.gate_dt, a.ffn, a.hidden, s.ks_gate, ain, ab, a.gu_out + a.ffn, a.gu_ld, n,
            (2 * ri + 1) * s.tiles_gate, a.rows, gmap, olo, ohi);
    // down: staged from this expert's gate|up rows as quant(silu(g) * u)
    if (a.swiglu_down)
      put_job(&a.down_jobs[ri], s.down + le * s.down_stride, s.down_tm, s.down_tm_tail, le * a.hidden,
              s.down_row_bytes, s.down_dt, a.hidden, a.ffn, s.ks_down, reinterpret_cast<const uint8_t*>(a.gu_out),
              a.gu_ld * 4, a.y, a.y_ld, n, ri * s.tiles_down, slots_routed + a.rows, dmap, olo, ohi, kActSwiGLU);
    else
      put_job(&a.down_jobs[ri], s.down + le * s.down_stride, s.down_tm, s.down_tm_tail, le * a.hidden,
              s.down_row_bytes, s.down_dt, a.hidden, a.ffn, s.ks_down, a.act_mid, a.act_mid_bytes, a.y, a.y_ld, n,
              ri * s.tiles_down, slots_routed + a.rows, dmap, olo, ohi);
  }
  if (threadIdx.x == 0) {
    // shared expert: every row, slots rows*topk + t
    const bool q80 = s.sh_gate_dt == Q8_0;
    const uint8_t* ain = q80 ? a.act_in80 : a.act_in8k;
    const int ab = q80 ? a.act_in80_bytes : a.act_in8k_bytes;
    uint64_t gmap = 0, dmap = 0, olo = 0, ohi = 0;
    for (int t = 0; t < a.rows; t++) {
      gmap |= (uint64_t)t << (8 * t);
      dmap |= (uint64_t)(slots_routed + t) << (8 * t);
      pack_out(olo, ohi, t, slots_routed + t);
    }
    put_job(&a.gu_jobs[2 * n_res], s.sh_gate, s.sh_gate_tm, s.sh_gate_tm_tail, 0, s.sh_gate_row_bytes,
            s.sh_gate_dt, a.sh_ffn, a.hidden, s.ks_sh_gate, ain, ab, a.gu_out, a.gu_ld, a.rows,
            2 * n_res * s.tiles_gate, a.rows, gmap, olo, ohi);
    put_job(&a.gu_jobs[2 * n_res + 1], s.sh_up, s.sh_up_tm, s.sh_up_tm_tail, 0, s.sh_gate_row_bytes, s.sh_gate_dt,
            a.sh_ffn, a.hidden, s.ks_sh_gate, ain, ab, a.gu_out + a.sh_ffn, a.gu_ld, a.rows,
            2 * n_res * s.tiles_gate + s.tiles_sh_gate, a.rows, gmap, olo, ohi);
    if (a.swiglu_down)
      put_job(&a.down_jobs[n_res], s.sh_down, s.sh_down_tm, s.sh_down_tm_tail, 0, s.sh_down_row_bytes,
              s.sh_down_dt, a.hidden, a.sh_ffn, s.ks_sh_down, reinterpret_cast<const uint8_t*>(a.gu_out),
              a.gu_ld * 4, a.y, a.y_ld, a.rows, n_res * s.tiles_down, slots_routed + a.rows, dmap, olo, ohi,
              kActSwiGLU);
    else
      put_job(&a.down_jobs[n_res], s.sh_down, s.sh_down_tm, s.sh_down_tm_tail, 0, s.sh_down_row_bytes,
              s.sh_down_dt, a.hidden, a.sh_ffn, s.ks_sh_down, a.act_mid, a.act_mid_bytes, a.y, a.y_ld, a.rows,
              n_res * s.tiles_down, slots_routed + a.rows, dmap, olo, ohi);
    *a.gu_count = s.with_shared ? 2 * n_res + 2 : 2 * n_res;
    *a.down_count = s.with_shared ? n_res + 1 : n_res;
    *a.union_size = total_union;
  }
}

template <int kPerLane>
__global__ void __launch_bounds__(256) moe_route_kernel(MoeRouteArgs a, MoeRouteStatic s) {
  pdl_wait();
  pdl_trigger();
  route_body<kPerLane>(a, s);
}

// The F32 router and the routing in one launch: CTA b computes router rows
// [8b, 8b+8) for the pass's rows with f32_matvec's arithmetic (lane l sums
// the float4 at columns 4l + 128t in order of t with fused multiply-adds,
// then the butterfly), and the last CTA to finish (device counter, reset by
// that CTA) routes every row and writes the job tables as moe_route_kernel.
template <int kPerLane>
__global__ void __launch_bounds__(256) router_route_kernel(RouterRouteArgs r, MoeRouteArgs a, MoeRouteStatic s) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  const int c4 = r.cols / 4;
  constexpr int kMaxPer = 32;  // float4 per lane: cols <= 4096
  float4 wv[kMaxPer];
  if (row < r.rows) {
    const float4* wr = reinterpret_cast<const float4*>(r.w + (int64_t)row * r.cols);
#pragma unroll
    for (int j = 0; j < kMaxPer; j++)
      if (lane + 32 * j < c4) wv[j] = __ldg(wr + lane + 32 * j);
  }
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 xs4[];  // [k][cols/4]
  const int k = a.rows;
#pragma unroll 4
  for (int i = threadIdx.x; i < k * c4; i += 256) {
    const int rr = i / c4, c = i % c4;
    xs4[i] = *reinterpret_cast<const float4*>(r.x + (int64_t)rr * r.ldx + 4 * c);
  }
  __syncthreads();
  if (row < r.rows) {
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
      if (lane == 0) r.y[(int64_t)i * a.logits_ld + row] = v;
    }
  }
  // the last CTA to finish routes (every CTA's logits are visible to it)
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) is_last = atomicAdd(r.counter, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x == 0) *r.counter = 0;  // ready for the next launch
  route_body<kPerLane>(a, s);
}

// One CTA per slot: silu(gate) * up (candle's elementwise silu,
// g / (1 + exp(-g))), quantized for the down projection.
template <int MAXB>
__global__ void __launch_bounds__(256) moe_act_kernel(MoeActArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) float xs[];
  const int slot = blockIdx.x;
  const int routed = a.rows * a.topk;
  if (slot >= routed + a.rows) return;
  int ffn = a.sh_ffn;
  bool q80 = a.sh_down_q80;
  if (slot < routed) {
    const int e = a.route_expert[slot];
    if (e < a.expert_lo || e >= a.expert_hi) return;
    ffn = a.ffn;
    q80 = a.down_q80;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = (ffn + 255) / 256;
  const float* g = a.gu + (int64_t)slot * a.gu_ld;
  float v[MAXB][8], u[MAXB][8];
#pragma unroll
  for (int j = 0; j < MAXB; j++)
    if (warp + 8 * j < nb) {
      ld_q8k_lane(g, warp + 8 * j, lane, v[j], ffn);
      ld_q8k_lane(g + ffn, warp + 8 * j, lane, u[j], ffn);
    }
#pragma unroll
  for (int j = 0; j < MAXB; j++)
#pragma unroll
    for (int i = 0; i < 8; i++) v[j][i] = __fmul_rn(__fdiv_rn(v[j][i], __fadd_rn(1.f, exp_ref(-v[j][i]))), u[j][i]);
  uint8_t* ar = a.act + (int64_t)slot * a.act_bytes;
  finish_row<MAXB>(v, nb, ffn, q80 ? nullptr : ar, q80 ? ar : nullptr, nullptr, xs);
}

// hidden += (sum_route y*w) + shared * sigmoid(selector); one thread per four
// consecutive columns of a row, every load issued before the sums.
__global__ void __launch_bounds__(256) moe_combine_kernel(MoeCombineArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int kMaxTopk = 16;
  const int t = blockIdx.y;
  const int i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= a.dim) return;
  const float sl = a.logits[(int64_t)t * a.logits_ld + a.experts];
  float w[kMaxTopk];
  float4 y[kMaxTopk];
#pragma unroll
  for (int q = 0; q < kMaxTopk; q++)
    if (q < a.topk) {
      w[q] = a.route_weight[t * a.topk + q];
      y[q] = *reinterpret_cast<const float4*>(a.y + (int64_t)(t * a.topk + q) * a.y_ld + i);
    }
  const float4 ysh = *reinterpret_cast<const float4*>(a.y + (int64_t)(a.rows * a.topk + t) * a.y_ld + i);
  float4* hp = reinterpret_cast<float4*>(a.hidden + (int64_t)t * a.hidden_ld + i);
  const float4 h = *hp;
  const float selector = __fdiv_rn(1.f, __fadd_rn(1.f, exp_ref(-sl)));
  float r[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < kMaxTopk; q++)
    if (q < a.topk) {
      r[0] = __fadd_rn(r[0], __fmul_rn(y[q].x, w[q]));
      r[1] = __fadd_rn(r[1], __fmul_rn(y[q].y, w[q]));
      r[2] = __fadd_rn(r[2], __fmul_rn(y[q].z, w[q]));
      r[3] = __fadd_rn(r[3], __fmul_rn(y[q].w, w[q]));
    }
  float4 o;
  o.x = __fadd_rn(h.x, __fadd_rn(r[0], __fmul_rn(ysh.x, selector)));
  o.y = __fadd_rn(h.y, __fadd_rn(r[1], __fmul_rn(ysh.y, selector)));
  o.z = __fadd_rn(h.z, __fadd_rn(r[2], __fmul_rn(ysh.z, selector)));
  o.w = __fadd_rn(h.w, __fadd_rn(r[3], __fmul_rn(ysh.w, selector)));
  *hp = o;
}

}  // namespace

cudaError_t moe_route_launch(const MoeRouteArgs& a, const MoeRouteStatic& s, cudaStream_t st, bool pdl) {
  if (a.rows > kMaxRows || a.experts > kMaxExperts || a.topk > 16) return cudaErrorInvalidValue;
  if (a.experts <= 256) return launch_pdl(moe_route_kernel<8>, dim3(1), dim3(256), 0, st, pdl, a, s);
  if (a.experts <= 512) return launch_pdl(moe_route_kernel<16>, dim3(1), dim3(256), 0, st, pdl, a, s);
  return launch_pdl(moe_route_kernel<32>, dim3(1), dim3(256), 0, st, pdl, a, s);
}

template <int kPerLane>
cudaError_t launch_router_route(const RouterRouteArgs& r, const MoeRouteArgs& a, const MoeRouteStatic& s,
                                cudaStream_t st, bool pdl) {
  static std::mutex mu;
  static bool done[64] = {};
  const cudaError_t e = once_per_device(done, mu, [] {
    return cudaFuncSetAttribute(router_route_kernel<kPerLane>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                8 * 4096 * 4);
  });
  if (e != cudaSuccess) return e;
  return launch_pdl(router_route_kernel<kPerLane>, dim3((unsigned)ceil_div(r.rows, 8)), dim3(256),
                    (size_t)a.rows * r.cols * sizeof(float), st, pdl, r, a, s);
}

cudaError_t router_route_launch(const RouterRouteArgs& r, const MoeRouteArgs& a, const MoeRouteStatic& s,
                                cudaStream_t st, bool pdl) {
  if (a.rows > kMaxRows || a.rows > 8 || a.experts > kMaxExperts || a.topk > 16 || r.cols % 4 || r.cols > 4096 ||
      r.y != a.logits || !r.counter)
    return cudaErrorInvalidValue;
  if (a.experts <= 256) return launch_router_route<8>(r, a, s, st, pdl);
  if (a.experts <= 512) return launch_router_route<16>(r, a, s, st, pdl);
  return launch_router_route<32>(r, a, s, st, pdl);
}

cudaError_t moe_route_rows_launch(const float* logits, int ld, int rows, int E, int topk, int norm_topk,
                                  int* route_e, float* route_w, cudaStream_t st) {
  if (E > kMaxExperts || topk > 16 || rows < 1) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)ceil_div(rows, 8));
  if (E <= 256) route_rows_kernel<8><<<grid, 256, 0, st>>>(logits, ld, rows, E, topk, norm_topk, route_e, route_w);
  else if (E <= 512) route_rows_kernel<16><<<grid, 256, 0, st>>>(logits, ld, rows, E, topk, norm_topk, route_e, route_w);
  else route_rows_kernel<32><<<grid, 256, 0, st>>>(logits, ld, rows, E, topk, norm_topk, route_e, route_w);
  return cudaGetLastError();
}

cudaError_t moe_act_launch(const MoeActArgs& a, cudaStream_t st, bool pdl) {
  const int ffn = a.ffn > a.sh_ffn ? a.ffn : a.sh_ffn;
  const bool any80 = a.down_q80 || a.sh_down_q80;
  if (a.ffn % (a.down_q80 ? 128 : 256) || a.sh_ffn % (a.sh_down_q80 ? 128 : 256) || a.gu_ld % 4)
    return cudaErrorInvalidValue;
  const dim3 grid(a.rows * a.topk + a.rows);
  const size_t smem = any80 ? ffn * sizeof(float) : 0;
  const int nb = (ffn + 255) / 256;
  if (nb <= 8) return launch_pdl(moe_act_kernel<1>, grid, dim3(256), smem, st, pdl, a);
  if (nb <= 16) return launch_pdl(moe_act_kernel<2>, grid, dim3(256), smem, st, pdl, a);
  if (nb <= 32) return launch_pdl(moe_act_kernel<4>, grid, dim3(256), smem, st, pdl, a);
  return cudaErrorInvalidValue;
}

cudaError_t moe_combine_launch(const MoeCombineArgs& a, cudaStream_t st, bool pdl) {
  if (a.topk > 16 || a.dim % 4 || a.y_ld % 4 || a.hidden_ld % 4) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)ceil_div(a.dim / 4, 128), a.rows);
  return launch_pdl(moe_combine_kernel, grid, dim3(128), 0, st, pdl, a);
}

}  // namespace iq
