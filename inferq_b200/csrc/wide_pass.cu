// wide_pass.cu -- the wide prefill pass: many tokens through every layer at
// once, the form of the reference's prefill in 512-row passes
// (prefill_in_passes, src/runtime.rs:748-771; QuantizedModel::forward over a
// pass's rows, src/qwen/quantized_model.rs:654-752).
//
// Per chunk of up to kWideRows rows and per layer:
//   * the dense projections (DeltaNet qkv / gate / beta / alpha / out,
//     attention q / k / v / o, the shared expert, the quantized router and the
//     LM head) run on the tcgen05 wide products, each weight read once for
//     the whole chunk;
//   * the DeltaNet recurrence runs in its exact sequential kernel over all
//     the chunk's rows in one launch (rows in order, the final block of up
//     to 8 kept for rollback); the causal attention scan runs over 8-row
//     slices of the chunk (as consecutive 8-row passes would);
//   * the routed experts run as one grouped GEMV launch: after the routes
//     are read back, every (expert, up to 8 of its rows) group becomes one
//     job, so an expert's weights are read once per 8 of its rows; the down
//     projection stages silu(g) * u itself; the ordered combine adds each
//     row's routes in route order.
// Rows therefore compute the reference's arithmetic up to f32 summation
// order (the wide products sum a row's blocks in one chunk), not bitwise the
// 8-row decode path; the state they leave behind is used by later passes as
// any other.  Supported when every dense matrix has a wide product (Q8_0,
// Q4_K, Q6_K) and the experts are resident on one GPU (wide_capable).
#include <algorithm>
#include <cstring>
#include <nccl.h>
#include "state.h"

namespace iq {
namespace {

#define TRY_IQ(x)           \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

// ----------------------------------------------------------- small kernels
__global__ void add_rows_kernel(float* __restrict__ h, const float* __restrict__ y, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(h)[i];
    const float4 b = reinterpret_cast<const float4*>(y)[i];
    a.x = __fadd_rn(a.x, b.x);
    a.y = __fadd_rn(a.y, b.y);
    a.z = __fadd_rn(a.z, b.z);
    a.w = __fadd_rn(a.w, b.w);
    reinterpret_cast<float4*>(h)[i] = a;
  }
}

// out[r][i] = silu(g) * u with g = in[r][i], u = in[r][F + i] (candle's
// elementwise silu, g / (1 + exp(-g)))
__global__ void swiglu_rows_kernel(const float* __restrict__ in, int ld, int F, int rows, float* __restrict__ out,
                                   int out_ld) {
  const int64_t n = (int64_t)rows * F;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / F, i = e % F;
    const float g = in[r * ld + i], u = in[r * ld + F + i];
    out[r * out_ld + i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, exp_ref(-g))), u);
  }
}

// dst[j] = src[idx[j]] (rows of `cols` floats); idx < 0 leaves a zero row
__global__ void gather_rows_kernel(const float* __restrict__ src, const int* __restrict__ idx, int n, int cols,
                                   float* __restrict__ dst) {
  const int j = blockIdx.x;
  if (j >= n) return;
  const int r = idx[j];
  for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[(int64_t)j * cols + c] = r >= 0 ? src[(int64_t)r * cols + c] : 0.f;
}

// hidden[r] += (sum_q y[map[r][q]] * w[r][q], in route order) + ysh[r] *
// sigmoid(selector logit), element by element as moe_combine does
__global__ void wide_combine_kernel(float* __restrict__ hidden, int H, int topk, const int* __restrict__ map,
                                    const float* __restrict__ yg, const float* __restrict__ rw,
                                    const float* __restrict__ ysh, const float* __restrict__ lg, int lg_ld,
                                    int experts) {
  const int r = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H) return;
  const float sl = lg[(int64_t)r * lg_ld + experts];
  const float selector = __fdiv_rn(1.f, __fadd_rn(1.f, exp_ref(-sl)));
  float acc = 0.f;
  for (int q = 0; q < topk; q++)
    acc = __fadd_rn(acc, __fmul_rn(yg[(int64_t)map[r * topk + q] * H + i], rw[r * topk + q]));
  float* h = hidden + (int64_t)r * H + i;
  *h = __fadd_rn(*h, __fadd_rn(acc, __fmul_rn(ysh[(int64_t)r * H + i], selector)));
}

// [0] the conv ring index and [1] the pending records (none) of the
// sequential DeltaNet launch over a chunk's final block (the chunked launch
// before it leaves the history after the prefix in slot cur + 1); [2 + j]
// the first position of attention slice j of `rows` rows
__global__ void wide_ctrl_kernel(const int* __restrict__ ctrl, int* __restrict__ wc, int slices, int rows) {
  const int j = threadIdx.x;
  if (j == 0) {
    wc[0] = (ctrl[1] + 1) % kStateRing;
    wc[1] = 0;
  }
  if (j >= slices) return;
  wc[2 + j] = ctrl[0] + rows * j;
}

// The chunk's rows before its final block are committed for good: the conv
// history after them sits in slot cur + 1 (deltanet_kernel), the final
// block's rows after it, so the ring index moves by one for the prefix plus
// the final rows, and rollback_kernel can step back inside the final block.
__global__ void wide_commit_kernel(int* ctrl, int rows, int last) {
  ctrl[0] += rows;
  ctrl[1] = (ctrl[1] + (rows > last ? 1 : 0) + last) % kStateRing;
  ctrl[6] = last;
}


bool wide_dtype(int dt) { return dt == Q8_0 || dt == Q4_K || dt == Q6_K || (dt == Q5_K && wide_q5k_enabled()); }

// y[t*ldy + r] = row r of w (rows [0, w.rows)) . x[t*ldx ..] for n input rows
int wide_project(iq_state* s, const Weight& w, const float* x, int ldx, int n, float* y, int ldy) {
  cudaStream_t st = s->st;
  DevBuf& sc = s->wide.scratch;
  if (w.dt == Q8_0) {
    const size_t qx = align_up((int64_t)n * w.cols * 2, 256);
    const size_t dT = align_up((int64_t)(w.cols / 32) * wide_ldd(n) * 4, 256);
    const size_t wx = (size_t)w.rows * w.cols * 2;
    IQ_CUDA(sc.reserve(qx + dT + wx));
    uint8_t* b = sc.as<uint8_t>();
    IQ_CUDA(wide_q80_forward(w.p(), w.rows, w.cols, w.row_bytes, x, ldx, n, y, ldy, reinterpret_cast<__half*>(b),
                             reinterpret_cast<float*>(b + qx), reinterpret_cast<__half*>(b + qx + dT), st));
  } else if (w.dt == Q4_K || w.dt == Q5_K) {
    const bool q5 = w.dt == Q5_K;
    IQ_CUDA(sc.reserve(wide_q4k_scratch_bytes(w.rows, w.cols, n, nullptr, nullptr, q5)));
    WideQ4kScratch k;
    wide_q4k_scratch_bytes(w.rows, w.cols, n, &k, sc.as<uint8_t>(), q5);
    IQ_CUDA((q5 ? wide_q5k_forward : wide_q4k_forward)(w.p(), w.rows, w.cols, w.row_bytes, x, ldx, n, y, ldy, k,
                                                       st));
  } else if (w.dt == Q6_K) {
    IQ_CUDA(sc.reserve(wide_q6k_scratch_bytes(w.rows, w.cols, n, nullptr, nullptr)));
    WideQ6kScratch k;
    wide_q6k_scratch_bytes(w.rows, w.cols, n, &k, sc.as<uint8_t>());
    IQ_CUDA(wide_q6k_forward(w.p(), w.rows, w.cols, w.row_bytes, x, ldx, n, y, ldy, k, st));
  } else {
    set_error("wide pass: matrix dtype %d has no wide product", w.dt);
    return IQ_EUNSUPPORTED;
  }
  return IQ_OK;
}

int add_rows(iq_state* s, float* h, const float* y, int64_t n) {
  const int64_t n4 = n / 4;
  add_rows_kernel<<<(unsigned)std::min<int64_t>(ceil_div(n4, 256), 148 * 8), 256, 0, s->st>>>(h, y, n4);
  IQ_CUDA(cudaGetLastError());
  return IQ_OK;
}

// RMSNorm of n rows (f32 out, no quantization), the row-prep kernel
int norm_rows(iq_state* s, const float* x, const float* w, int n, int H, float* out, uint8_t* q8k = nullptr,
              int q8k_stride = 0, uint8_t* q80 = nullptr, int q80_stride = 0) {
  const iq_config& c = s->m->cfg;
  PrepArgs a = {};
  a.x = x;
  a.ldx = H;
  a.cols = H;
  a.norm_w = w;
  a.eps = c.rms_norm_eps;
  a.inv_cols = (float)(1.0 / (double)H);
  a.xn_out = out;
  a.ldxn = H;
  a.q8k = q8k;
  a.q8k_stride = q8k_stride;
  a.q80 = q80;
  a.q80_stride = q80_stride;
  IQ_CUDA(prep_rows(a, n, s->st, false));
  return IQ_OK;
}

int wide_delta(iq_state* s, const Layer& L, int li, int n) {
  const iq_config& c = s->m->cfg;
  auto& W = s->wide;
  const DeltaWeights& D = L.dn;
  const int nv = c.linear_num_value_heads, vdim = nv * c.linear_value_head_dim;
  const int conv_dim = 2 * c.linear_num_key_heads * c.linear_key_head_dim + vdim;
  float* qkv = W.big.as<float>();
  TRY_IQ(wide_project(s, D.qkv, W.xn.as<float>(), c.hidden_size, n, qkv, conv_dim));
  TRY_IQ(wide_project(s, D.z, W.xn.as<float>(), c.hidden_size, n, W.z.as<float>(), vdim));
  if (D.ba_fused) {
    TRY_IQ(wide_project(s, D.ba, W.xn.as<float>(), c.hidden_size, n, W.ba.as<float>(), 2 * nv));
  } else {
    TRY_IQ(wide_project(s, D.beta, W.xn.as<float>(), c.hidden_size, n, W.ba.as<float>(), 2 * nv));
    TRY_IQ(wide_project(s, D.alpha, W.xn.as<float>(), c.hidden_size, n, W.ba.as<float>() + nv, 2 * nv));
  }
  // The rows before the final block of up to 8 run in the chunked form; the
  // final block runs in the sequential kernel, which keeps its update
  // records for rollback (when the chunked form does not fit the head
  // shapes, the sequential kernel takes every row).
  const int dk = c.linear_key_head_dim, dv = c.linear_value_head_dim;
  const int last = (n - 1) % kMaxRowsDelta + 1, pre = n - last;
  const bool chunked = pre > 0 && deltanet_chunk_supported(c.linear_num_key_heads, nv, dk, dv,
                                                           c.linear_conv_kernel_dim);
  const int r0 = chunked ? pre : 0;
  if (chunked) {
    DeltaChunkArgs h = {};
    h.layers = s->dn_layers.as<DeltaNetLayer>() + li;
    h.qkv = qkv;
    h.qkv_ld = conv_dim;
    h.ba = W.ba.as<float>();
    h.ba_ld = 2 * nv;
    h.rows = pre;
    h.nk = c.linear_num_key_heads;
    h.nv = nv;
    h.dk = dk;
    h.dv = dv;
    h.conv_k = c.linear_conv_kernel_dim;
    h.tiled_heads = c.value_heads_tiled;
    h.ba_interleaved = D.ba_fused;
    h.rec_stride = deltanet_rec_stride(dk, dv);
    h.cur = s->ctrl.as<int>() + 1;
    h.pending = s->ctrl.as<int>() + 6;
    IQ_CUDA(W.cv.reserve((size_t)n * conv_dim * 4));
    IQ_CUDA(W.bl.reserve((size_t)n * 2 * nv * 4));
    IQ_CUDA(W.dno.reserve((size_t)n * vdim * 4));
    const int64_t nch = ceil_div(pre, 32);  // the chunked kernels' 32-row chunks
    IQ_CUDA(W.wyx.reserve((size_t)nv * nch * 32 * (dk + dv) * 4));
    IQ_CUDA(W.wym.reserve((size_t)nv * nch * 32 * 32 * 4));
    IQ_CUDA(W.wyew.reserve((size_t)nv * nch * 64 * 4));
    h.wy_x = W.wyx.as<float>();
    h.wy_m = W.wym.as<float>();
    h.wy_ew = W.wyew.as<float>();
    h.cv = W.cv.as<float>();
    h.bl = W.bl.as<float>();
    h.o = W.dno.as<float>();
    h.o_ld = vdim;
    h.z = W.z.as<float>();
    h.z_ld = vdim;
    h.norm_w = D.norm.p();
    h.eps = c.rms_norm_eps;
    h.inv_dv = (float)(1.0 / dv);
    h.g_out = W.o.as<float>();
    h.g_ld = vdim;
    IQ_CUDA(deltanet_chunk_launch(h, s->st));
  }
  DeltaNetArgs a = {};
  a.layers = s->dn_layers.as<DeltaNetLayer>() + li;
  a.qkv = qkv + (int64_t)r0 * conv_dim;
  a.qkv_ld = conv_dim;
  a.ba = W.ba.as<float>() + (int64_t)r0 * 2 * nv;
  a.ba_ld = 2 * nv;
  a.out = nullptr;
  a.out_ld = vdim;
  a.rows = n - r0;
  a.nk = c.linear_num_key_heads;
  a.nv = nv;
  a.dk = dk;
  a.dv = dv;
  a.conv_k = c.linear_conv_kernel_dim;
  a.tiled_heads = c.value_heads_tiled;
  a.ba_interleaved = D.ba_fused;
  a.rec_stride = deltanet_rec_stride(a.dk, a.dv);
  a.timeout_flag = qmv_timeout_flag();
  // after the chunked prefix: the history in slot cur + 1, nothing to replay
  a.cur = chunked ? W.ctrl.as<int>() : s->ctrl.as<int>() + 1;
  a.pending = chunked ? W.ctrl.as<int>() + 1 : s->ctrl.as<int>() + 6;
  a.z = W.z.as<float>() + (int64_t)r0 * vdim;
  a.z_ld = vdim;
  a.norm_w = D.norm.p();
  a.eps = c.rms_norm_eps;
  a.inv_dv = (float)(1.0 / c.linear_value_head_dim);
  a.g_out = W.o.as<float>() + (int64_t)r0 * vdim;
  a.g_ld = vdim;
  IQ_CUDA(deltanet_launch(a, s->st, false));
  TRY_IQ(wide_project(s, D.out, W.o.as<float>(), vdim, n, W.y.as<float>(), c.hidden_size));
  return add_rows(s, W.hidden.as<float>(), W.y.as<float>(), (int64_t)n * c.hidden_size);
}

int wide_attention(iq_state* s, const Layer& L, int fi, int n) {
  const iq_config& c = s->m->cfg;
  auto& W = s->wide;
  const AttnWeights& A = L.at;
  const int nhd = c.num_attention_heads * c.head_dim, kvd = c.num_key_value_heads * c.head_dim;
  TRY_IQ(wide_project(s, A.q, W.xn.as<float>(), c.hidden_size, n, W.big.as<float>(), 2 * nhd));
  TRY_IQ(wide_project(s, A.k, W.xn.as<float>(), c.hidden_size, n, W.kp.as<float>(), kvd));
  TRY_IQ(wide_project(s, A.v, W.xn.as<float>(), c.hidden_size, n, W.vp.as<float>(), kvd));
  // slices of W.attn_rows rows: every row's arithmetic is its own (fixed
  // 32-position chunks merged in order), so the slice size changes no result
  const int R = W.attn_rows;
  for (int j = 0, r0 = 0; r0 < n; j++, r0 += R) {
    const int k = std::min(R, n - r0);
    AttnArgs a = {};
    a.qg = W.big.as<float>() + (int64_t)r0 * 2 * nhd;
    a.qg_ld = 2 * nhd;
    a.kp = W.kp.as<float>() + (int64_t)r0 * kvd;
    a.kp_ld = kvd;
    a.vp = W.vp.as<float>() + (int64_t)r0 * kvd;
    a.vp_ld = kvd;
    a.q_norm = A.q_norm.p();
    a.k_norm = A.k_norm.p();
    a.kcache = s->kc[fi].as<float>();
    a.vcache = s->vc[fi].as<float>();
    a.qbuf = W.qbuf.as<float>();
    a.part = W.part.as<float>();
    a.out = W.o.as<float>() + (int64_t)r0 * nhd;
    a.out_ld = nhd;
    a.rows = k;
    a.nh = c.num_attention_heads;
    a.nkv = c.num_key_value_heads;
    a.hd = c.head_dim;
    a.rotary_dim = c.rotary_dim;
    a.theta = c.rope_theta;
    a.eps = c.rms_norm_eps;
    a.pos = W.ctrl.as<int>() + 2 + j;
    a.chunk_ctas = s->max_chunks;
    IQ_CUDA(attn_prep_launch(a, s->st, false));
    IQ_CUDA(attn_scan_launch(a, s->st, false));
    IQ_CUDA(attn_combine_launch(a, s->st, false));
  }
  TRY_IQ(wide_project(s, A.o, W.o.as<float>(), nhd, n, W.y.as<float>(), c.hidden_size));
  return add_rows(s, W.hidden.as<float>(), W.y.as<float>(), (int64_t)n * c.hidden_size);
}

int wide_moe(iq_state* s, const Layer& L, int n) {
  const iq_config& c = s->m->cfg;
  auto& W = s->wide;
  const MoeWeights& M = L.moe;
  const int H = c.hidden_size, E = c.num_experts, topk = c.num_experts_per_tok;
  const int F = c.moe_intermediate_size, Fs = c.shared_expert_intermediate_size;
  cudaStream_t st = s->st;
  TRY_IQ(norm_rows(s, W.hidden.as<float>(), L.post_norm.p(), n, H, W.xn.as<float>()));
  // router logits [n][E + 1]: column E is the shared expert's selector
  float* lg = W.lg.as<float>();
  if (M.router.present()) {
    TRY_IQ(wide_project(s, M.router, W.xn.as<float>(), H, n, lg, E + 1));
    IQ_CUDA(f32_rows(M.selector.p(), 1, H, W.xn.as<float>(), H, n, lg + E, E + 1, st));
  } else {
    IQ_CUDA(f32_rows(M.router_sel.p(), E + 1, H, W.xn.as<float>(), H, n, lg, E + 1, st));
  }
  IQ_CUDA(moe_route_rows_launch(lg, E + 1, n, E, topk, c.norm_topk_prob, W.re.as<int>(), W.rw.as<float>(), st));
  IQ_CUDA(cudaMemcpyAsync(W.h_routes, W.re.p, (size_t)n * topk * 4, cudaMemcpyDeviceToHost, st));
  // the shared expert over every row meanwhile
  TRY_IQ(wide_project(s, M.sh_gate, W.xn.as<float>(), H, n, W.gush.as<float>(), 2 * Fs));
  TRY_IQ(wide_project(s, M.sh_up, W.xn.as<float>(), H, n, W.gush.as<float>() + Fs, 2 * Fs));
  swiglu_rows_kernel<<<(unsigned)std::min<int64_t>(ceil_div((int64_t)n * Fs, 256), 148 * 8), 256, 0, st>>>(
      W.gush.as<float>(), 2 * Fs, Fs, n, W.o.as<float>(), Fs);
  IQ_CUDA(cudaGetLastError());
  TRY_IQ(wide_project(s, M.sh_down, W.o.as<float>(), Fs, n, W.ysh.as<float>(), H));
  IQ_CUDA(cudaStreamSynchronize(st));
  // Expert parallelism: this rank runs only the slots of its own experts
  // [e_lo, e_hi) (its expert tensors hold just those); after the down
  // projection every slot's output goes to a dense [slot][H] buffer, zero on
  // the ranks that do not own it, and one sum over the ranks leaves each slot
  // its owner's value (x + 0 = x), so the ordered combine is the one-GPU one.
  const bool ep = s->m->ep_world > 1;
  const int e_lo = ep ? M.expert_lo : 0, e_hi = ep ? M.expert_hi : E;
  // groups of at most 8 rows per expert, experts ascending, rows in order;
  // gathered row g*8+i is member i of group g
  std::vector<std::vector<int>> by_e(E);
  for (int r = 0; r < n; r++)
    for (int q = 0; q < topk; q++) {
      const int e = W.h_routes[r * topk + q];
      IQ_CHECK(e >= 0 && e < E, IQ_ESTATE, "wide pass: route %d of row %d names expert %d of %d", q, r, e, E);
      if (e >= e_lo && e < e_hi) by_e[e].push_back(r * topk + q);
    }
  int groups = 0;
  for (int e = 0; e < E; e++) groups += (int)ceil_div((int64_t)by_e[e].size(), 8);
  const int ng_rows = 8 * groups;
  IQ_CHECK(ng_rows < 32768, IQ_EUNSUPPORTED, "wide pass: %d expert slots exceed the GEMV's row index", ng_rows);
  const bool q80 = M.gate.dt == Q8_0;
  const int arb = (int)(q80 ? act_row_bytes_q80(H) : act_row_bytes_q8k(H));
  const int gu_ld = 2 * F;
  IQ_CUDA(W.xg.reserve((size_t)ng_rows * H * 4));
  IQ_CUDA(W.actg.reserve((size_t)ng_rows * arb));
  IQ_CUDA(W.gu.reserve((size_t)ng_rows * gu_ld * 4));
  IQ_CUDA(W.yg.reserve((size_t)ng_rows * H * 4));
  IQ_CUDA(W.jobs.reserve((size_t)3 * groups * sizeof(QmvJob)));
  IQ_CUDA(W.map.reserve(((size_t)n * topk * (ep ? 2 : 1) + ng_rows) * 4));
  std::vector<int> gather((size_t)ng_rows, -1);  // source row per gathered slot (-1 padding)
  W.map_host.assign((size_t)n * topk, ep ? -1 : 0);  // (EP: -1 for the slots of other ranks' experts)
  const int ks_gate = qmv_ksplit(M.gate.dt, F, H, true), ks_down = qmv_ksplit(M.down.dt, H, F, true);
  const int tg = (int)ceil_div(F, qmv_rows_per_cta(ks_gate)), td = (int)ceil_div(H, qmv_rows_per_cta(ks_down));
  std::vector<QmvJob>& jt = W.job_table;
  jt.clear();
  std::vector<QmvJob> down;
  int gt = 0, dtiles = 0, g = 0;
  for (int e = e_lo; e < e_hi; e++) {
    const std::vector<int>& sl = by_e[e];
    const int64_t el = e - e_lo;  // the expert's index in this rank's tensors
    for (size_t g0 = 0; g0 < sl.size(); g0 += 8, g++) {
      const int ng = (int)std::min<size_t>(8, sl.size() - g0);
      const int base = 8 * g;
      for (int i = 0; i < ng; i++) {
        gather[base + i] = sl[g0 + i] / topk;
        W.map_host[sl[g0 + i]] = base + i;
      }
      QmvJob j;
      memset(&j, 0, sizeof j);
      j.dtype = M.gate.dt;
      j.rows = F;
      j.cols = H;
      j.ksplit = ks_gate;
      j.n = ng;
      j.act_nrows = ng;
      j.epi = kEpiStore;
      j.w_row_bytes = M.gate.row_bytes;
      j.act = W.actg.as<uint8_t>() + (int64_t)base * arb;
      j.act_row_bytes = arb;
      j.out_ld = gu_ld;
      for (int i = 0; i < 8; i++) {
        j.rowmap[i] = (uint8_t)(i < ng ? i : 0);
        j.outrow[i] = (int16_t)(base + i);
      }
      j.row_base = (int)(el * F);
      j.w = M.gate.p() + el * F * M.gate.row_bytes;
      j.tmap = M.gate.tmap();
      j.tmap_tail = M.gate.tmap_tail();
      j.out = W.gu.as<float>();
      j.tile0 = gt;
      jt.push_back(j);
      gt += tg;
      j.w = M.up.p() + el * F * M.up.row_bytes;
      j.tmap = M.up.tmap();
      j.tmap_tail = M.up.tmap_tail();
      j.out = W.gu.as<float>() + F;
      j.tile0 = gt;
      jt.push_back(j);
      gt += tg;
      QmvJob d;
      memset(&d, 0, sizeof d);
      d.dtype = M.down.dt;
      d.rows = H;
      d.cols = F;
      d.ksplit = ks_down;
      d.n = ng;
      d.act_nrows = ng;
      d.epi = kEpiStore;
      d.w_row_bytes = M.down.row_bytes;
      d.act = reinterpret_cast<const uint8_t*>(W.gu.as<float>() + (int64_t)base * gu_ld);
      d.act_row_bytes = gu_ld * 4;
      d.act_mode = kActSwiGLU;
      d.out = W.yg.as<float>();
      d.out_ld = H;
      for (int i = 0; i < 8; i++) {
        d.rowmap[i] = (uint8_t)(i < ng ? i : 0);
        d.outrow[i] = (int16_t)(base + i);
      }
      d.row_base = (int)(el * H);
      d.w = M.down.p() + el * H * M.down.row_bytes;
      d.tmap = M.down.tmap();
      d.tmap_tail = M.down.tmap_tail();
      d.tile0 = dtiles;
      down.push_back(d);
      dtiles += td;
    }
  }
  const int njobs = (int)jt.size();
  for (auto& d : down) jt.push_back(d);
  int* d_map = W.map.as<int>();
  int* d_gather = d_map + (size_t)n * topk;
  if (!jt.empty())
    IQ_CUDA(cudaMemcpyAsync(W.jobs.p, jt.data(), jt.size() * sizeof(QmvJob), cudaMemcpyHostToDevice, st));
  IQ_CUDA(cudaMemcpyAsync(d_map, W.map_host.data(), (size_t)n * topk * 4, cudaMemcpyHostToDevice, st));
  if (ng_rows > 0)
    IQ_CUDA(cudaMemcpyAsync(d_gather, gather.data(), gather.size() * 4, cudaMemcpyHostToDevice, st));
  // (host vectors stay alive until the stream synchronizes at the end of the chunk)
  if (ng_rows > 0) {  // (zero only under expert parallelism: none of this rank's experts routed)
    gather_rows_kernel<<<ng_rows, 256, 0, st>>>(W.xn.as<float>(), d_gather, ng_rows, H, W.xg.as<float>());
    IQ_CUDA(cudaGetLastError());
    PrepArgs pa = {};
    pa.x = W.xg.as<float>();
    pa.ldx = H;
    pa.cols = H;
    pa.inv_cols = (float)(1.0 / (double)H);
    if (q80) { pa.q80 = W.actg.as<uint8_t>(); pa.q80_stride = arb; }
    else { pa.q8k = W.actg.as<uint8_t>(); pa.q8k_stride = arb; }
    IQ_CUDA(prep_rows(pa, ng_rows, st, false));
    IQ_CUDA(qmv_launch(W.jobs.as<QmvJob>(), njobs, nullptr, gt, 8 * arb, st, false));
    const int mid = (int)std::max(act_row_bytes_q8k(F), act_row_bytes_q80(F));
    IQ_CUDA(qmv_launch(W.jobs.as<QmvJob>() + njobs, (int)down.size(), nullptr, dtiles, 8 * mid, st, false));
  }
  const int* comb_map = d_map;
  const float* comb_y = W.yg.as<float>();
  if (ep) {
    const int slots = n * topk;
    IQ_CUDA(W.yslot.reserve((size_t)slots * H * 4));
    // slot s <- gathered row map[s] (zero where another rank owns the expert)
    gather_rows_kernel<<<slots, 256, 0, st>>>(W.yg.as<float>(), d_map, slots, H, W.yslot.as<float>());
    IQ_CUDA(cudaGetLastError());
    const ncclResult_t r = ncclAllReduce(W.yslot.p, W.yslot.p, (size_t)slots * H, ncclFloat, ncclSum,
                                         static_cast<ncclComm_t>(s->m->nccl_comm), st);
    IQ_CHECK(r == ncclSuccess, IQ_ECUDA, "wide pass expert exchange (ncclAllReduce): %s", ncclGetErrorString(r));
    std::vector<int> ident((size_t)slots);
    for (int i = 0; i < slots; i++) ident[i] = i;
    int* d_ident = d_gather + ng_rows;
    // (pageable source: the call returns once `ident` has been staged)
    IQ_CUDA(cudaMemcpyAsync(d_ident, ident.data(), (size_t)slots * 4, cudaMemcpyHostToDevice, st));
    comb_map = d_ident;
    comb_y = W.yslot.as<float>();
  }
  const dim3 grid((unsigned)ceil_div(H, 256), (unsigned)n);
  wide_combine_kernel<<<grid, 256, 0, st>>>(W.hidden.as<float>(), H, topk, comb_map, comb_y, W.rw.as<float>(),
                                            W.ysh.as<float>(), lg, E + 1, E);
  IQ_CUDA(cudaGetLastError());
  return IQ_OK;
}

int alloc_wide(iq_state* s, int n) {
  const iq_config& c = s->m->cfg;
  auto& W = s->wide;
  const int64_t H = c.hidden_size, vdim = (int64_t)c.linear_num_value_heads * c.linear_value_head_dim;
  const int64_t conv_dim = 2 * (int64_t)c.linear_num_key_heads * c.linear_key_head_dim + vdim;
  const int64_t nhd = (int64_t)c.num_attention_heads * c.head_dim, kvd = (int64_t)c.num_key_value_heads * c.head_dim;
  const int64_t E = c.num_experts, topk = c.num_experts_per_tok, Fs = c.shared_expert_intermediate_size;
  IQ_CUDA(W.hidden.reserve(n * H * 4));
  IQ_CUDA(W.xn.reserve(n * H * 4));
  IQ_CUDA(W.big.reserve(n * std::max(conv_dim, 2 * nhd) * 4));
  IQ_CUDA(W.z.reserve(n * std::max<int64_t>(vdim, 1) * 4));
  IQ_CUDA(W.ba.reserve(n * 2 * std::max(c.linear_num_value_heads, 1) * 4));
  IQ_CUDA(W.o.reserve(n * std::max({vdim, nhd, Fs}) * 4));
  IQ_CUDA(W.y.reserve(n * H * 4));
  IQ_CUDA(W.kp.reserve(n * kvd * 4));
  IQ_CUDA(W.vp.reserve(n * kvd * 4));
  IQ_CUDA(W.tokens.reserve(n * 4));
  IQ_CUDA(W.ctrl.reserve((2 + ceil_div(n, 8)) * 4));
  if (c.num_attention_heads > 0 && s->m->n_linear < c.num_hidden_layers) {
    // attention slices: as many rows as the scan's shared memory and a
    // partials buffer of at most 512 MB hold
    AttnArgs g = {};
    g.nh = c.num_attention_heads;
    g.nkv = c.num_key_value_heads;
    g.hd = c.head_dim;
    g.chunk_ctas = s->max_chunks;
    int R = attn_scan_max_rows(g, 32);
    while (R > 8 && (int64_t)R * nhd * s->max_chunks * 4 > (int64_t)512 << 20) R /= 2;
    W.attn_rows = R;
    IQ_CUDA(W.qbuf.reserve(R * nhd * 4));
    IQ_CUDA(W.part.reserve((size_t)R * c.num_attention_heads * s->max_chunks * (c.head_dim + 2) * 4));
  }
  IQ_CUDA(W.lg.reserve(n * (E + 1) * 4));
  IQ_CUDA(W.re.reserve(n * topk * 4));
  IQ_CUDA(W.rw.reserve(n * topk * 4));
  IQ_CUDA(W.ysh.reserve(n * H * 4));
  IQ_CUDA(W.gush.reserve(n * 2 * Fs * 4));
  IQ_CUDA(W.argres.reserve(n * 4));
  if (!W.h_routes) IQ_CUDA(cudaMallocHost(&W.h_routes, (size_t)kWideRows * topk * 4));
  return IQ_OK;
}

// One chunk of n <= kWideRows rows.
int wide_chunk(iq_state* s, const uint32_t* tokens, int n, float* logits, float* hidden, int32_t* argmax, int row0) {
  iq_model* m = s->m;
  const iq_config& c = m->cfg;
  auto& W = s->wide;
  cudaStream_t st = s->st;
  const int H = c.hidden_size, V = c.vocab_size;
  std::vector<int32_t> tk(tokens, tokens + n);
  IQ_CUDA(cudaMemcpyAsync(W.tokens.p, tk.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st));
  wide_ctrl_kernel<<<1, 256, 0, st>>>(s->ctrl.as<int>(), W.ctrl.as<int>(), (int)ceil_div(n, W.attn_rows),
                                      W.attn_rows);
  IQ_CUDA(cudaGetLastError());
  IQ_CUDA(embed_launch(m->embed.dt, m->embed.p(), m->embed.row_bytes, H, W.tokens.as<int32_t>(), n,
                       W.hidden.as<float>(), H, st, false));
  int li = 0, fi = 0;
  for (int l = 0; l < c.num_hidden_layers; l++) {
    const Layer& L = m->layers[l];
    TRY_IQ(norm_rows(s, W.hidden.as<float>(), L.attn_norm.p(), n, H, W.xn.as<float>()));
    if (L.type == kLinear) TRY_IQ(wide_delta(s, L, li++, n));
    else TRY_IQ(wide_attention(s, L, fi++, n));
    TRY_IQ(wide_moe(s, L, n));
  }
  TRY_IQ(norm_rows(s, W.hidden.as<float>(), m->out_norm.p(), n, H, W.xn.as<float>()));
  if (hidden)
    IQ_CUDA(cudaMemcpyAsync(hidden + (int64_t)row0 * H, W.xn.p, (size_t)n * H * 4, cudaMemcpyDeviceToHost, st));
  if (logits || argmax) {
    IQ_CUDA(W.logits.reserve((size_t)n * V * 4));
    TRY_IQ(wide_project(s, m->lm_head, W.xn.as<float>(), H, n, W.logits.as<float>(), V));
    if (logits)
      IQ_CUDA(cudaMemcpyAsync(logits + (int64_t)row0 * V, W.logits.p, (size_t)n * V * 4, cudaMemcpyDeviceToHost, st));
    if (argmax) {
      IQ_CUDA(rows_argmax_launch(W.logits.as<float>(), V, n, V, W.argres.as<int>(), st));
      IQ_CUDA(cudaMemcpyAsync(argmax + row0, W.argres.p, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    }
  }
  const int last = (n - 1) % kMaxRowsDelta + 1;  // the final block the DeltaNet kernels keep
  wide_commit_kernel<<<1, 1, 0, st>>>(s->ctrl.as<int>(), n, last);
  IQ_CUDA(cudaGetLastError());
  IQ_CUDA(cudaStreamSynchronize(st));
  s->position += n;
  s->last_rows = last;
  return IQ_OK;
}

}  // namespace

bool wide_capable(const iq_model* m) {
  // under expert parallelism only with IQ_WIDE_EP set, until its two-GPU
  // test has passed on hardware (tests/test_ep_gpu.py sets it)
  static const bool wide_ep = getenv("IQ_WIDE_EP") != nullptr;
  if (m->ep_world > 1 && !wide_ep) return false;
  const iq_config& c = m->cfg;
  if (c.num_hidden_layers < 1 || c.num_experts_per_tok > 16 || c.hidden_size % 256) return false;
  auto ok = [](const Weight& w) { return wide_dtype(w.dt); };
  if (!ok(m->lm_head)) return false;
  for (const Layer& L : m->layers) {
    if (L.type == kLinear) {
      const DeltaWeights& D = L.dn;
      if (!ok(D.qkv) || !ok(D.z) || !ok(D.out) || (D.ba_fused ? !ok(D.ba) : (!ok(D.beta) || !ok(D.alpha)))) return false;
    } else {
      const AttnWeights& A = L.at;
      if (!ok(A.q) || !ok(A.k) || !ok(A.v) || !ok(A.o)) return false;
    }
    const MoeWeights& M = L.moe;
    if (!ok(M.sh_gate) || !ok(M.sh_up) || !ok(M.sh_down)) return false;
    if (M.router.present() && !ok(M.router)) return false;
    if (M.gate.dt == F32 || M.down.dt == F32) return false;
  }
  return true;
}

int wide_forward(iq_state* s, const uint32_t* tokens, int rows, float* logits, float* hidden, int32_t* argmax) {
  TRY_IQ(alloc_wide(s, std::min(rows, kWideRows)));
  for (int r0 = 0; r0 < rows; r0 += kWideRows)
    TRY_IQ(wide_chunk(s, tokens + r0, std::min(kWideRows, rows - r0), logits, hidden, argmax, r0));
  return IQ_OK;
}

}  // namespace iq
