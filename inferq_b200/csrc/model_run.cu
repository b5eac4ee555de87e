// model_run.cu -- decode state, the k-row pass, verify/accept/rollback.
//
// One pass (QuantizedModel::forward_inner, src/qwen/quantized_model.rs:654-752):
//   embed -> per layer { RMSNorm -> DeltaNet | gated attention -> residual
//                        -> RMSNorm -> MoE -> residual }
//   -> final RMSNorm -> LM head -> argmax -> accept -> commit
// Every launch is enqueued on the state's stream with programmatic dependent
// launch, and the whole pass is captured once per row count into a CUDA graph.
#include <algorithm>
#include <map>
#include <cstring>
#include <cstdlib>
#include <string>
#include <nccl.h>
#include "state.h"

namespace iq {
namespace {

#define TRY(x)              \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

int64_t arb_for(int dt, int64_t cols) { return dt == Q8_0 ? act_row_bytes_q80(cols) : act_row_bytes_q8k(cols); }

QmvJob make_job(const Weight& w, const uint8_t* act, int64_t arb, float* out, int out_ld, int k, int epi,
                const float* resid) {
  QmvJob j;
  memset(&j, 0, sizeof j);
  j.w = w.p();
  j.tmap = w.tmap();
  j.tmap_tail = w.tmap_tail();
  j.act = act;
  j.out = out;
  j.resid = resid;
  j.w_row_bytes = w.row_bytes;
  j.act_row_bytes = (int)arb;
  j.out_ld = out_ld;
  j.dtype = w.dt;
  j.rows = (int)w.rows;
  j.cols = (int)w.cols;
  j.ksplit = qmv_ksplit(w.dt, w.rows, w.cols);
  j.n = k;
  j.act_nrows = k;
  j.epi = epi;
  for (int i = 0; i < 8; i++) {
    j.rowmap[i] = (uint8_t)(i < k ? i : 0);
    j.outrow[i] = (int16_t)i;
  }
  return j;
}

// Append a multi-job launch to `table`, assigning tile0 prefixes.
QmvRec add_launch(std::vector<QmvJob>& table, std::vector<QmvJob> jobs) {
  QmvRec r;
  r.job = (int)table.size();
  r.njobs = (int)jobs.size();
  int tiles = 0, smem = 0;
  for (auto& j : jobs) {
    j.tile0 = tiles;
    tiles += qmv_tiles(j);
    smem = std::max(smem, j.n * j.act_row_bytes);
    r.slot = std::max(r.slot, qmv_slot_bytes(j.dtype));
    table.push_back(j);
  }
  r.ntiles = tiles;
  r.smem = smem;
  return r;
}

struct Ctx {
  iq_state* s;
  iq_model* m;
  const iq_config& c;
  cudaStream_t st;
  bool pdl;
  // IQ_NO_PDL=1 turns programmatic dependent launch off (kernel timing,
  // debugging); results are identical either way.
  // Kernel fusions (IQ_FUSE=<bitmask>; results are bitwise the same either
  // way).  Default 1|2|4|16, measured faster at k = 1, 4 and 8 (35B shapes);
  // 8 puts redundant normalization on every router CTA and measured slower;
  // 32 (not a fusion, off by default: measured 1% slower at k = 4) sizes
  // GEMV ring slots per launch:
  // 1 MoE combine into the next RMSNorm, 2 gated norm + Q8_0 into the
  // DeltaNet kernel, 4 SwiGLU into the down GEMV, 8 RMSNorm + Q8_K into the
  // f32 router, 16 output-projection quantization into the attention combine,
  // 64 the f32 router and the routing kernel in one launch (off by default:
  // 1% slower at k = 4 -- the routing then waits for the slowest router CTA,
  // where as its own launch it overlaps the router's tail).
  int fuse;
  Ctx(iq_state* s_) : s(s_), m(s_->m), c(s_->m->cfg), st(s_->st), pdl(!s_->profiling && !getenv("IQ_NO_PDL")) {
    const char* f = getenv("IQ_FUSE");
    fuse = f ? atoi(f) : 23;
  }
  // ring slots sized for the launch's dtypes (fuse bit 32), else the largest
  int slot(int bytes) const { return (fuse & 32) ? bytes : 0; }
  // Stage timer: under profiling every stage is bracketed by CUDA events.
  void mark(const char* name) {
    if (!s->profiling) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, st);
    s->marks.emplace_back(name, e);
  }
  int* pos() const { return s->ctrl.as<int>(); }
  int* attn_pos = nullptr;  // KV position the attention layers use (default pos())
  // The MoE combine of the last MoE block, applied by the next kernel that
  // normalizes the hidden rows (one launch fewer per layer).
  bool comb_pending = false;
  MoeCombineArgs comb = {};
  int* cur() const { return s->ctrl.as<int>() + 1; }  // DeltaNet conv ring index
  int* pending() const { return s->ctrl.as<int>() + 6; }  // DeltaNet records to replay
  int* result() const { return s->ctrl.as<int>() + 2; }
  const uint8_t* act(int dt) const { return dt == Q8_0 ? s->act80.as<uint8_t>() : s->act8k.as<uint8_t>(); }
  int64_t arb(int dt) const { return dt == Q8_0 ? s->act80_bytes : s->act8k_bytes; }
};

bool needs(int dt, bool q80) { return dt >= 0 && (q80 ? dt == Q8_0 : dt != Q8_0 && dt != F32); }

int flush_combine(Ctx& x);

int prep(Ctx& x, const float* in, int ld, int cols, const float* norm, int k, bool q8k, bool q80, float* xn,
         int ldxn = 0) {
  if (x.comb_pending && in != x.s->hidden.as<float>()) TRY(flush_combine(x));
  PrepArgs a = {};
  a.x = in;
  a.ldx = ld;
  a.cols = cols;
  a.norm_w = norm;
  a.eps = x.c.rms_norm_eps;
  a.inv_cols = (float)(1.0 / (double)cols);
  a.xn_out = xn;
  a.ldxn = ldxn ? ldxn : cols;
  a.q8k = q8k ? x.s->act8k.as<uint8_t>() : nullptr;
  a.q80 = q80 ? x.s->act80.as<uint8_t>() : nullptr;
  a.q8k_stride = (int)x.s->act8k_bytes;
  a.q80_stride = (int)x.s->act80_bytes;
  if (x.comb_pending && in == x.s->hidden.as<float>()) {
    a.comb_y = x.comb.y;
    a.comb_y_ld = x.comb.y_ld;
    a.comb_w = x.comb.route_weight;
    a.comb_logits = x.comb.logits;
    a.comb_logits_ld = x.comb.logits_ld;
    a.comb_experts = x.comb.experts;
    a.comb_topk = x.comb.topk;
    a.comb_rows = x.comb.rows;
    x.comb_pending = false;
  }
  ++x.s->launch_count;
  IQ_CUDA(prep_rows(a, k, x.st, x.pdl));
  return IQ_OK;
}

// Launch a pending MoE combine on its own (when no normalizing kernel follows).
int flush_combine(Ctx& x) {
  if (!x.comb_pending) return IQ_OK;
  x.comb_pending = false;
  ++x.s->launch_count;
  IQ_CUDA(moe_combine_launch(x.comb, x.st, x.pdl));
  return IQ_OK;
}

// The activation rows a projection needs (row prep or gated norm kernel).
int pre(Ctx& x, const QmvPrologue& p) {
  if (p.mode == kProGated) {
    GatedNormArgs g = {};
    g.o = p.x;
    g.o_ld = p.ldx;
    g.z = p.z;
    g.z_ld = p.ldz;
    g.w = p.w;
    g.heads = p.heads;
    g.dv = p.dv;
    g.eps = p.eps;
    g.inv_dv = p.inv_n;
    g.q8k = p.want8k ? x.s->act8k.as<uint8_t>() : nullptr;
    g.q80 = p.want80 ? x.s->act80.as<uint8_t>() : nullptr;
    g.q8k_stride = (int)x.s->act8k_bytes;
    g.q80_stride = (int)x.s->act80_bytes;
    ++x.s->launch_count;
    IQ_CUDA(gated_norm_launch(g, p.rows, x.st, x.pdl));
    return IQ_OK;
  }
  return prep(x, p.x, p.ldx, p.cols, p.mode == kProRmsNorm ? p.w : nullptr, p.rows, p.want8k, p.want80, p.xn_out,
              p.ldxn);
}

int qmv(Ctx& x, const QmvRec& r, const QmvPrologue* pro = nullptr) {
  if (pro) {
    TRY(pre(x, *pro));
    x.mark("act.prep");
  }
  ++x.s->launch_count;
  IQ_CUDA(qmv_launch(x.s->jobs.as<QmvJob>() + r.job, r.njobs, nullptr, r.ntiles, r.smem, x.st, x.pdl, x.slot(r.slot)));
  return IQ_OK;
}

// Prologue that RMS-normalizes (or, norm == null, just quantizes) `k` f32
// rows of `cols` into the layouts the launch's matrices need.
QmvPrologue row_pro(Ctx& x, const float* in, int ld, int cols, const float* norm, int k, bool q8k, bool q80,
                    float* xn = nullptr) {
  QmvPrologue p = {};
  p.mode = norm ? kProRmsNorm : kProQuant;
  p.rows = k;
  p.cols = cols;
  p.x = in;
  p.ldx = ld;
  p.w = norm;
  p.eps = x.c.rms_norm_eps;
  p.inv_n = (float)(1.0 / (double)cols);
  p.want8k = q8k;
  p.want80 = q80;
  p.stride8k = (int)act_row_bytes_q8k(cols);
  p.stride80 = (int)act_row_bytes_q80(cols);
  p.xn_out = xn;
  p.ldxn = cols;
  return p;
}

// ------------------------------------------------------------ plan building
int build_plans(iq_state* s) {
  iq_model* m = s->m;
  const iq_config& c = m->cfg;
  const int H = c.hidden_size;
  const int vdim = c.linear_num_value_heads * c.linear_value_head_dim;
  const int conv_dim = 2 * c.linear_num_key_heads * c.linear_key_head_dim + vdim;
  const int nhd = c.num_attention_heads * c.head_dim;
  std::vector<QmvJob> table;
  s->plans.assign(kMaxK, KPlan());
  float* hidden = s->hidden.as<float>();
  for (int k = 1; k <= kMaxK; k++) {
    KPlan& P = s->plans[k - 1];
    P.layers.resize(c.num_hidden_layers);
    int li = 0;
    for (int l = 0; l < c.num_hidden_layers; l++) {
      const Layer& L = m->layers[l];
      LayerRec& R = P.layers[l];
      auto J = [&](const Weight& w, float* out, int ld, int epi = kEpiStore) {
        return make_job(w, w.dt == Q8_0 ? s->act80.as<uint8_t>() : s->act8k.as<uint8_t>(),
                        w.dt == Q8_0 ? s->act80_bytes : s->act8k_bytes, out, ld, k, epi, out);
      };
      if (L.type == kLinear) {
        std::vector<QmvJob> js;
        js.push_back(J(L.dn.qkv, s->dn_qkv[li].as<float>(), conv_dim));
        js.push_back(J(L.dn.z, s->z.as<float>(), vdim));
        if (L.dn.ba_fused) {
          js.push_back(J(L.dn.ba, s->dn_ba[li].as<float>(), 2 * c.linear_num_value_heads));
        } else {
          js.push_back(J(L.dn.beta, s->dn_ba[li].as<float>(), 2 * c.linear_num_value_heads));
          js.push_back(J(L.dn.alpha, s->dn_ba[li].as<float>() + c.linear_num_value_heads, 2 * c.linear_num_value_heads));
        }
        R.proj = add_launch(table, js);
        R.out = add_launch(table, {J(L.dn.out, hidden, H, kEpiResidual)});
        li++;
      } else {
        R.proj = add_launch(table, {J(L.at.q, s->qg.as<float>(), 2 * nhd),
                                    J(L.at.k, s->kp.as<float>(), c.num_key_value_heads * c.head_dim),
                                    J(L.at.v, s->vp.as<float>(), c.num_key_value_heads * c.head_dim)});
        R.out = add_launch(table, {J(L.at.o, hidden, H, kEpiResidual)});
      }
      if (L.moe.router.present())
        R.router = add_launch(table, {J(L.moe.router, s->logits_moe.as<float>(), c.num_experts + 1)});
    }
    if (m->has_mtp) {
      auto J = [&](const Weight& w, float* out, int ld, int epi = kEpiStore) {
        return make_job(w, w.dt == Q8_0 ? s->act80.as<uint8_t>() : s->act8k.as<uint8_t>(),
                        w.dt == Q8_0 ? s->act80_bytes : s->act8k_bytes, out, ld, k, epi, out);
      };
      const Layer& L = m->mtp_layer;
      P.mtp_eh = add_launch(table, {J(m->mtp_eh_proj, hidden, H)});
      P.mtp.proj = add_launch(table, {J(L.at.q, s->qg.as<float>(), 2 * nhd),
                                      J(L.at.k, s->kp.as<float>(), c.num_key_value_heads * c.head_dim),
                                      J(L.at.v, s->vp.as<float>(), c.num_key_value_heads * c.head_dim)});
      P.mtp.out = add_launch(table, {J(L.at.o, hidden, H, kEpiResidual)});
      if (L.moe.router.present())
        P.mtp.router = add_launch(table, {J(L.moe.router, s->logits_moe.as<float>(), c.num_experts + 1)});
    }
    P.lm_head = add_launch(table, {make_job(m->lm_head, m->lm_head.dt == Q8_0 ? s->act80.as<uint8_t>() : s->act8k.as<uint8_t>(),
                                            m->lm_head.dt == Q8_0 ? s->act80_bytes : s->act8k_bytes,
                                            s->logits.as<float>(), c.vocab_size, k, kEpiStore, nullptr)});
  }
  IQ_CUDA(s->jobs.reserve(table.size() * sizeof(QmvJob)));
  IQ_CUDA(cudaMemcpy(s->jobs.p, table.data(), table.size() * sizeof(QmvJob), cudaMemcpyHostToDevice));
  return IQ_OK;
}

// ------------------------------------------------------------------- layers
int run_moe(Ctx& x, const Layer& L, const LayerRec& R, int k, int layer_index) {
  iq_state* s = x.s;
  const iq_config& c = x.c;
  const MoeWeights& W = L.moe;
  const int H = c.hidden_size, E = c.num_experts;
  const bool q8k = needs(W.gate.dt, false) || needs(W.sh_gate.dt, false) || needs(W.router.dt, false);
  const bool q80 = needs(W.gate.dt, true) || needs(W.sh_gate.dt, true) || needs(W.router.dt, true);
  float* lg = s->logits_moe.as<float>();
  bool fused_router = false;
  const float* router_in = nullptr;
  if ((x.fuse & 8) && !W.router.present() && !q80 && !x.comb_pending && H % 256 == 0) {
    // f32 router: it normalizes the rows itself and writes their Q8_K form
    // for the expert matrices (one launch for norm, quantization and router)
    ++x.s->launch_count;
    IQ_CUDA(f32_matvec(W.router_sel.p(), E + 1, H, s->hidden.as<float>(), H, k, lg, E + 1, x.st, x.pdl,
                       L.post_norm.p(), c.rms_norm_eps, s->act8k.as<uint8_t>(), (int)s->act8k_bytes));
    x.mark("moe.router");
  } else {
  TRY(pre(x, row_pro(x, s->hidden.as<float>(), H, H, L.post_norm.p(), k, q8k, q80, s->xn.as<float>())));
  x.mark("act.prep");
  const float* rin = s->xn.as<float>();
  const float* rnorm = nullptr;
  if (W.router.present()) {
    ++x.s->launch_count;
    IQ_CUDA(qmv_launch(x.s->jobs.as<QmvJob>() + R.router.job, R.router.njobs, nullptr, R.router.ntiles, R.router.smem,
                       x.st, x.pdl, x.slot(R.router.slot)));
    x.mark("moe.router");
    ++x.s->launch_count;
    IQ_CUDA(f32_matvec(W.selector.p(), 1, H, rin, H, k, lg + E, E + 1, x.st, x.pdl, rnorm, c.rms_norm_eps));
    x.mark("moe.router");
  } else if (x.fuse & 64) {
    // F32 router fused with the routing kernel below (one launch)
    fused_router = true;
    router_in = rin;
  } else {
    ++x.s->launch_count;
    IQ_CUDA(f32_matvec(W.router_sel.p(), E + 1, H, rin, H, k, lg, E + 1, x.st, x.pdl, rnorm, c.rms_norm_eps));
    x.mark("moe.router");
  }
  }
  MoeRouteArgs a = {};
  a.logits = lg;
  a.logits_ld = E + 1;
  a.rows = k;
  a.experts = E;
  a.topk = c.num_experts_per_tok;
  a.norm_topk = c.norm_topk_prob;
  a.hidden = H;
  a.ffn = c.moe_intermediate_size;
  a.sh_ffn = c.shared_expert_intermediate_size;
  a.route_expert = s->route_e.as<int>() + (int64_t)layer_index * kMaxK * c.num_experts_per_tok;
  a.route_weight = s->route_w.as<float>();
  a.gu_jobs = s->gu_jobs.as<QmvJob>();
  a.down_jobs = s->down_jobs.as<QmvJob>();
  int* cnt = s->counts.as<int>();
  a.gu_count = cnt;
  a.down_count = cnt + 1;
  a.union_size = cnt + 4 + layer_index;
  a.union_list = s->union_list.as<int>();
  a.act_in8k = s->act8k.as<uint8_t>();
  a.act_in8k_bytes = (int)s->act8k_bytes;
  a.act_in80 = s->act80.as<uint8_t>();
  a.act_in80_bytes = (int)s->act80_bytes;
  a.gu_out = s->gu_out.as<float>();
  a.gu_ld = s->gu_ld;
  a.act_mid = s->act_mid.as<uint8_t>();
  a.act_mid_bytes = (int)s->act_mid_bytes;
  a.y = s->y.as<float>();
  a.y_ld = H;
  a.swiglu_down = (x.fuse & 4) ? 1 : 0;
  MoeRouteStatic t = {};
  const int F = c.moe_intermediate_size, Fs = c.shared_expert_intermediate_size;
  t.gate = W.gate.p();
  t.up = W.up.p();
  t.down = W.down.p();
  t.gate_tm = W.gate.tmap();
  t.up_tm = W.up.tmap();
  t.down_tm = W.down.tmap();
  t.down_tm_tail = W.down.tmap_tail();
  t.gate_tm_tail = W.gate.tmap_tail();
  t.up_tm_tail = W.up.tmap_tail();
  t.sh_gate_tm = W.sh_gate.tmap();
  t.sh_up_tm = W.sh_up.tmap();
  t.sh_down_tm = W.sh_down.tmap();
  t.sh_gate_tm_tail = W.sh_gate.tmap_tail();
  t.sh_up_tm_tail = W.sh_up.tmap_tail();
  t.sh_down_tm_tail = W.sh_down.tmap_tail();
  t.gate_stride = (int64_t)F * W.gate.row_bytes;
  t.up_stride = (int64_t)F * W.up.row_bytes;
  t.down_stride = (int64_t)H * W.down.row_bytes;
  t.gate_row_bytes = W.gate.row_bytes;
  t.down_row_bytes = W.down.row_bytes;
  t.gate_dt = W.gate.dt;
  t.down_dt = W.down.dt;
  t.ks_gate = qmv_ksplit(W.gate.dt, F, H, true);
  t.ks_down = qmv_ksplit(W.down.dt, H, F, true);
  t.tiles_gate = (int)ceil_div(F, qmv_rows_per_cta(t.ks_gate));
  t.tiles_down = (int)ceil_div(H, qmv_rows_per_cta(t.ks_down));
  t.sh_gate = W.sh_gate.p();
  t.sh_up = W.sh_up.p();
  t.sh_down = W.sh_down.p();
  t.sh_gate_row_bytes = W.sh_gate.row_bytes;
  t.sh_down_row_bytes = W.sh_down.row_bytes;
  t.sh_gate_dt = W.sh_gate.dt;
  t.sh_down_dt = W.sh_down.dt;
  t.ks_sh_gate = qmv_ksplit(W.sh_gate.dt, Fs, H, true);
  t.ks_sh_down = qmv_ksplit(W.sh_down.dt, H, Fs, true);
  t.tiles_sh_gate = (int)ceil_div(Fs, qmv_rows_per_cta(t.ks_sh_gate));
  t.with_shared = 1;
  t.expert_lo = W.expert_lo;
  t.expert_hi = W.expert_hi;
  ++x.s->launch_count;
  if (fused_router) {
    RouterRouteArgs rr = {};
    rr.w = W.router_sel.p();
    rr.rows = E + 1;
    rr.cols = H;
    rr.x = router_in;
    rr.ldx = H;
    rr.y = lg;
    rr.counter = cnt + 2;  // counts word 2: the fused router's finish counter
    IQ_CUDA(router_route_launch(rr, a, t, x.st, x.pdl));
  } else {
    IQ_CUDA(moe_route_launch(a, t, x.st, x.pdl));
  }
  x.mark("moe.route");
  // upper bounds on the dynamic job tables' tiles
  const int max_union = std::min(W.expert_hi - W.expert_lo, k * c.num_experts_per_tok);
  const int gu_tiles = 2 * max_union * t.tiles_gate + 2 * t.tiles_sh_gate;
  const int tiles_sh_down = (int)ceil_div(H, qmv_rows_per_cta(t.ks_sh_down));
  const int down_tiles = max_union * t.tiles_down + tiles_sh_down;
  const int gu_smem = k * (int)std::max(s->act8k_bytes, s->act80_bytes);
  ++x.s->launch_count;
  IQ_CUDA(qmv_launch(a.gu_jobs, 0, a.gu_count, gu_tiles, gu_smem, x.st, x.pdl,
                     x.slot(std::max(qmv_slot_bytes(W.gate.dt), qmv_slot_bytes(W.sh_gate.dt)))));
  x.mark("moe.gate_up");
  MoeActArgs b = {};
  b.gu = a.gu_out;
  b.gu_ld = a.gu_ld;
  b.ffn = F;
  b.sh_ffn = Fs;
  b.rows = k;
  b.topk = c.num_experts_per_tok;
  b.route_expert = a.route_expert;
  b.expert_lo = W.expert_lo;
  b.expert_hi = W.expert_hi;
  b.act = s->act_mid.as<uint8_t>();
  b.act_bytes = (int)s->act_mid_bytes;
  b.down_q80 = W.down.dt == Q8_0;
  b.sh_down_q80 = W.sh_down.dt == Q8_0;
  if (!(x.fuse & 4)) {  // else SwiGLU and its quantization run inside the down GEMV (kActSwiGLU jobs)
    ++x.s->launch_count;
    IQ_CUDA(moe_act_launch(b, x.st, x.pdl));
    x.mark("moe.act");
  }
  // Expert parallelism: this rank computes only the routed slots of its own
  // experts; the others stay exactly zero, and one sum over the ranks then
  // leaves every slot with the value its owner computed (x + 0 = x), so the
  // ordered combine below is bitwise the single-GPU one.  The shared expert
  // is replicated and stays local.
  const bool ep = x.m->ep_world > 1;
  const size_t routed = (size_t)k * c.num_experts_per_tok * H;
  if (ep) IQ_CUDA(cudaMemsetAsync(a.y, 0, routed * sizeof(float), x.st));
  ++x.s->launch_count;
  IQ_CUDA(qmv_launch(a.down_jobs, 0, a.down_count, down_tiles,
                     ((x.fuse & 4) ? k : k * c.num_experts_per_tok + k) * (int)s->act_mid_bytes, x.st, x.pdl,
                     x.slot(std::max(qmv_slot_bytes(W.down.dt), qmv_slot_bytes(W.sh_down.dt)))));
  x.mark("moe.down");
  if (ep) {
    const ncclResult_t r =
        ncclAllReduce(a.y, a.y, routed, ncclFloat, ncclSum, static_cast<ncclComm_t>(x.m->nccl_comm), x.st);
    IQ_CHECK(r == ncclSuccess, IQ_ECUDA, "expert exchange (ncclAllReduce): %s", ncclGetErrorString(r));
    x.mark("moe.exchange");
  }
  MoeCombineArgs cb = {};
  cb.y = a.y;
  cb.y_ld = H;
  cb.route_weight = a.route_weight;
  cb.logits = lg;
  cb.logits_ld = E + 1;
  cb.experts = E;
  cb.hidden = s->hidden.as<float>();
  cb.hidden_ld = H;
  cb.rows = k;
  cb.topk = c.num_experts_per_tok;
  cb.dim = H;
  x.comb = cb;
  x.comb_pending = true;  // applied by the next normalization of the hidden rows
  if (!(x.fuse & 1)) TRY(flush_combine(x));
  return IQ_OK;
}

int run_delta(Ctx& x, const Layer& L, const LayerRec& R, int k, int li) {
  iq_state* s = x.s;
  const iq_config& c = x.c;
  const DeltaWeights& D = L.dn;
  const int H = c.hidden_size;
  const int vdim = c.linear_num_value_heads * c.linear_value_head_dim;
  const int conv_dim = 2 * c.linear_num_key_heads * c.linear_key_head_dim + vdim;
  const int bdt = D.ba_fused ? D.ba.dt : D.beta.dt;
  const bool q8k = needs(D.qkv.dt, false) || needs(D.z.dt, false) || needs(bdt, false);
  const bool q80 = needs(D.qkv.dt, true) || needs(D.z.dt, true) || needs(bdt, true);
  const QmvPrologue in_pro = row_pro(x, s->hidden.as<float>(), H, H, L.attn_norm.p(), k, q8k, q80);
  TRY(qmv(x, R.proj, &in_pro));
  x.mark("dn.proj");
  DeltaNetArgs a = {};
  a.layers = s->dn_layers.as<DeltaNetLayer>() + li;
  a.qkv = s->dn_qkv[li].as<float>();
  a.qkv_ld = conv_dim;
  a.ba = s->dn_ba[li].as<float>();
  a.ba_ld = 2 * c.linear_num_value_heads;
  a.out = s->dn_out.as<float>();
  a.out_ld = vdim;
  a.rows = k;
  a.nk = c.linear_num_key_heads;
  a.nv = c.linear_num_value_heads;
  a.dk = c.linear_key_head_dim;
  a.dv = c.linear_value_head_dim;
  a.conv_k = c.linear_conv_kernel_dim;
  a.tiled_heads = c.value_heads_tiled;
  a.ba_interleaved = D.ba_fused;
  a.rec_stride = deltanet_rec_stride(a.dk, a.dv);
  a.timeout_flag = qmv_timeout_flag();
  a.cur = x.cur();
  a.pending = x.pending();
  // a Q8_0 output projection takes its activations straight from the
  // recurrence kernel (gated norm and quantization fused)
  const bool fuse = (x.fuse & 2) && D.out.dt == Q8_0 && vdim % 128 == 0;
  if (fuse) {
    a.q80 = s->act80.as<uint8_t>();
    a.q80_stride = (int)s->act80_bytes;
    a.z = s->z.as<float>();
    a.z_ld = vdim;
    a.norm_w = D.norm.p();
    a.eps = c.rms_norm_eps;
    a.inv_dv = (float)(1.0 / c.linear_value_head_dim);
  }
  ++x.s->launch_count;
  IQ_CUDA(deltanet_launch(a, x.st, x.pdl));
  x.mark("dn.recurrence");
  if (fuse) {
    TRY(qmv(x, R.out));
    x.mark("dn.out");
    return IQ_OK;
  }
  GatedNormArgs g = {};
  g.o = s->dn_out.as<float>();
  g.o_ld = vdim;
  g.z = s->z.as<float>();
  g.z_ld = vdim;
  g.w = D.norm.p();
  g.heads = c.linear_num_value_heads;
  g.dv = c.linear_value_head_dim;
  g.eps = c.rms_norm_eps;
  g.inv_dv = (float)(1.0 / c.linear_value_head_dim);
  g.q8k = D.out.dt == Q8_0 ? nullptr : s->act8k.as<uint8_t>();
  g.q80 = D.out.dt == Q8_0 ? s->act80.as<uint8_t>() : nullptr;
  g.q8k_stride = (int)s->act8k_bytes;
  g.q80_stride = (int)s->act80_bytes;
  QmvPrologue gp = {};
  gp.mode = kProGated;
  gp.rows = k;
  gp.cols = vdim;
  gp.x = g.o;
  gp.ldx = g.o_ld;
  gp.z = g.z;
  gp.ldz = g.z_ld;
  gp.w = g.w;
  gp.heads = g.heads;
  gp.dv = g.dv;
  gp.eps = g.eps;
  gp.inv_n = g.inv_dv;
  gp.want8k = D.out.dt != Q8_0;
  gp.want80 = D.out.dt == Q8_0;
  gp.stride8k = (int)act_row_bytes_q8k(vdim);
  gp.stride80 = (int)act_row_bytes_q80(vdim);
  TRY(qmv(x, R.out, &gp));
  x.mark("dn.out");
  return IQ_OK;
}

int run_attention(Ctx& x, const Layer& L, const LayerRec& R, int k, int fi) {
  iq_state* s = x.s;
  const iq_config& c = x.c;
  const AttnWeights& A = L.at;
  const int H = c.hidden_size;
  const int nhd = c.num_attention_heads * c.head_dim;
  const bool q8k = needs(A.q.dt, false) || needs(A.k.dt, false) || needs(A.v.dt, false);
  const bool q80 = needs(A.q.dt, true) || needs(A.k.dt, true) || needs(A.v.dt, true);
  const QmvPrologue in_pro = row_pro(x, s->hidden.as<float>(), H, H, L.attn_norm.p(), k, q8k, q80);
  TRY(qmv(x, R.proj, &in_pro));
  x.mark("attn.proj");
  AttnArgs a = {};
  a.qg = s->qg.as<float>();
  a.qg_ld = 2 * nhd;
  a.kp = s->kp.as<float>();
  a.kp_ld = c.num_key_value_heads * c.head_dim;
  a.vp = s->vp.as<float>();
  a.vp_ld = a.kp_ld;
  a.q_norm = A.q_norm.p();
  a.k_norm = A.k_norm.p();
  a.kcache = s->kc[fi].as<float>();
  a.vcache = s->vc[fi].as<float>();
  a.qbuf = s->qbuf.as<float>();
  a.part = s->part.as<float>();
  a.out = s->attn_out.as<float>();
  a.out_ld = nhd;
  a.rows = k;
  a.nh = c.num_attention_heads;
  a.nkv = c.num_key_value_heads;
  a.hd = c.head_dim;
  a.rotary_dim = c.rotary_dim;
  a.theta = c.rope_theta;
  a.eps = c.rms_norm_eps;
  a.pos = x.attn_pos ? x.attn_pos : x.pos();
  a.chunk_ctas = s->max_chunks;
  // the combine quantizes the output projection's input itself when a head
  // is whole blocks of that projection's activation format
  const bool o8k = needs(A.o.dt, false), o80 = needs(A.o.dt, true);
  const bool fuse_out = (x.fuse & 16) && ((o8k && c.head_dim == 256) || (o80 && c.head_dim % 128 == 0));
  if (fuse_out && o8k) {
    a.q8k_out = s->act8k.as<uint8_t>();
    a.q8k_stride = (int)s->act8k_bytes;
  } else if (fuse_out) {
    a.q80_out = s->act80.as<uint8_t>();
    a.q80_stride = (int)s->act80_bytes;
  }
  ++x.s->launch_count;
  IQ_CUDA(attn_prep_launch(a, x.st, x.pdl));
  x.mark("attn.prep");
  ++x.s->launch_count;
  IQ_CUDA(attn_scan_launch(a, x.st, x.pdl));
  x.mark("attn.scan");
  ++x.s->launch_count;
  IQ_CUDA(attn_combine_launch(a, x.st, x.pdl));
  x.mark("attn.combine");
  const QmvPrologue out_pro = row_pro(x, s->attn_out.as<float>(), nhd, nhd, nullptr, k, needs(A.o.dt, false),
                                     needs(A.o.dt, true));
  TRY(qmv(x, R.out, fuse_out ? nullptr : &out_pro));
  x.mark("attn.out");
  return IQ_OK;
}

// Undo the last pass down to `committed` of its `rows` rows: the DeltaNet
// conv state after that row is already in the ring, the recurrent state is
// the base plus that many update records, the KV cache is truncated.
__global__ void rollback_kernel(int* ctrl, int rows, int committed) {
  ctrl[1] = (ctrl[1] - rows + committed + 2 * kStateRing) % kStateRing;
  ctrl[0] -= rows - committed;
  ctrl[6] = committed;
}

// The pass body shared by forward and verify.
int run_pass(iq_state* s, int k, bool verify) {
  Ctx x(s);
  iq_model* m = s->m;
  const iq_config& c = m->cfg;
  const KPlan& P = s->plans[k - 1];
  const int H = c.hidden_size;
  IQ_CUDA(cudaMemcpyAsync(s->tokens.p, s->h_tokens, k * sizeof(int32_t), cudaMemcpyHostToDevice, x.st));
  ++s->launch_count;
  IQ_CUDA(embed_launch(m->embed.dt, m->embed.p(), m->embed.row_bytes, H, s->tokens.as<int32_t>(), k,
                       s->hidden.as<float>(), H, x.st, x.pdl));
  x.mark("embed");
  int li = 0, fi = 0;
  for (int l = 0; l < c.num_hidden_layers; l++) {
    const Layer& L = m->layers[l];
    if (L.type == kLinear) TRY(run_delta(x, L, P.layers[l], k, li++));
    else TRY(run_attention(x, L, P.layers[l], k, fi++));
    TRY(run_moe(x, L, P.layers[l], k, l));
  }
  const QmvPrologue head_pro = row_pro(x, s->hidden.as<float>(), H, H, m->out_norm.p(), k,
                                      needs(m->lm_head.dt, false), needs(m->lm_head.dt, true), s->xn.as<float>());
  TRY(qmv(x, P.lm_head, &head_pro));
  x.mark("head.lm_head");
  HeadArgs h = {};
  h.logits = s->logits.as<float>();
  h.logits_ld = c.vocab_size;
  h.rows = k;
  h.vocab = c.vocab_size;
  h.part_val = s->pval.as<float>();
  h.part_idx = s->pidx.as<int>();
  h.nparts = kArgmaxParts;
  h.argmax = s->argmax.as<int>();
  h.tokens = s->tokens.as<int32_t>();
  h.verify = verify ? 1 : 0;
  h.result = x.result();
  h.scores = nullptr;
  TRY(flush_combine(x));
  ++x.s->launch_count;
  IQ_CUDA(argmax_launch(h, x.st, x.pdl));
  x.mark("head.argmax");
  ++x.s->launch_count;
  IQ_CUDA(accept_launch(h, x.st, x.pdl));
  x.mark("head.accept");
  ++x.s->launch_count;
  IQ_CUDA(commit_launch(x.cur(), x.pos(), x.pending(), x.result(), x.st, x.pdl));
  x.mark("head.commit");
  IQ_CUDA(cudaMemcpyAsync(s->h_result, x.result(), 4 * sizeof(int), cudaMemcpyDeviceToHost, x.st));
  // the GEMVs' bounded-wait status travels back with the result
  if (int* f = qmv_timeout_flag()) IQ_CUDA(cudaMemcpyAsync(s->h_result + 4, f, sizeof(int), cudaMemcpyDeviceToHost, x.st));
  return IQ_OK;
}

// ---------------------------------------------------------------- MTP
// The MTP predictor block over k rows (quantized_mtp.rs:175-227): tokens in
// s->tokens, hidden inputs in s->mtp_hin.  x = eh_proj(enorm(embed(token)) |
// hnorm(hidden)); the block's attention (its own KV cache, position ctrl[5])
// and MoE; then shared_head_norm -> s->xn, quantized for the LM head.  The
// KV position advances by k.
int run_mtp_block(iq_state* s, int k) {
  Ctx x(s);
  x.attn_pos = s->ctrl.as<int>() + 5;
  iq_model* m = s->m;
  const iq_config& c = m->cfg;
  const KPlan& P = s->plans[k - 1];
  const int H = c.hidden_size;
  float* xcat = s->mtp_xcat.as<float>();
  ++s->launch_count;
  IQ_CUDA(embed_launch(m->embed.dt, m->embed.p(), m->embed.row_bytes, H, s->tokens.as<int32_t>(), k,
                       s->hidden.as<float>(), H, x.st, x.pdl));
  QmvPrologue e = row_pro(x, s->hidden.as<float>(), H, H, m->mtp_enorm.p(), k, false, false, xcat);
  e.ldxn = 2 * H;
  TRY(pre(x, e));
  QmvPrologue hh = row_pro(x, s->mtp_hin.as<float>(), H, H, m->mtp_hnorm.p(), k, false, false, xcat + H);
  hh.ldxn = 2 * H;
  TRY(pre(x, hh));
  const int edt = m->mtp_eh_proj.dt;
  QmvPrologue q = row_pro(x, xcat, 2 * H, 2 * H, nullptr, k, needs(edt, false), needs(edt, true));
  TRY(qmv(x, P.mtp_eh, &q));
  x.mark("mtp.eh_proj");
  TRY(run_attention(x, m->mtp_layer, P.mtp, k, m->n_full));
  TRY(run_moe(x, m->mtp_layer, P.mtp, k, c.num_hidden_layers));
  TRY(pre(x, row_pro(x, s->hidden.as<float>(), H, H, m->mtp_head_norm.p(), k, needs(m->lm_head.dt, false),
                     needs(m->lm_head.dt, true), s->xn.as<float>())));
  TRY(flush_combine(x));
  ++s->launch_count;
  IQ_CUDA(set_int_launch(x.attn_pos, k, true, x.st, x.pdl));
  x.mark("mtp.block");
  return IQ_OK;
}

// The vocabulary-prefix LM head job (first `vocab` rows, leading_rows).
int mtp_head_job(iq_state* s, int vocab) {
  if (s->mtp_head_vocab == vocab) return IQ_OK;
  iq_model* m = s->m;
  QmvJob j = make_job(m->lm_head, m->lm_head.dt == Q8_0 ? s->act80.as<uint8_t>() : s->act8k.as<uint8_t>(),
                      m->lm_head.dt == Q8_0 ? s->act80_bytes : s->act8k_bytes, s->logits.as<float>(), vocab, 1,
                      kEpiStore, nullptr);
  j.rows = vocab;
  j.ksplit = qmv_ksplit(m->lm_head.dt, vocab, m->lm_head.cols);
  IQ_CUDA(s->mtp_head_job.reserve(sizeof j));
  IQ_CUDA(cudaMemcpy(s->mtp_head_job.p, &j, sizeof j, cudaMemcpyHostToDevice));
  s->mtp_head_vocab = vocab;
  return IQ_OK;
}

// `depth` draft steps from s->tokens[0] / s->mtp_hin[0]; step i's token,
// probability and margin land in s->mtp_out.
int run_mtp_draft(iq_state* s, int depth, int vocab) {
  iq_model* m = s->m;
  const int H = m->cfg.hidden_size;
  int* out = s->mtp_out.as<int>();
  for (int i = 0; i < depth; i++) {
    TRY(run_mtp_block(s, 1));
    Ctx x(s);
    ++s->launch_count;
    IQ_CUDA(qmv_launch(s->mtp_head_job.as<QmvJob>(), 1, nullptr,
                       (int)ceil_div(vocab, qmv_rows_per_cta(qmv_ksplit(m->lm_head.dt, vocab, m->lm_head.cols))),
                       (int)(m->lm_head.dt == Q8_0 ? s->act80_bytes : s->act8k_bytes), x.st, x.pdl,
                       x.slot(qmv_slot_bytes(m->lm_head.dt))));
    x.mark("mtp.head");
    HeadArgs h = {};
    h.logits = s->logits.as<float>();
    h.logits_ld = vocab;
    h.rows = 1;
    h.vocab = vocab;
    h.part_val = s->pval.as<float>();
    h.part_idx = s->pidx.as<int>();
    h.nparts = kArgmaxParts;
    h.argmax = s->argmax.as<int>();
    h.tokens = s->tokens.as<int32_t>();
    h.verify = 0;
    h.result = s->mtp_res.as<int>();
    h.scores = s->scores.as<float>();
    ++s->launch_count;
    IQ_CUDA(argmax_launch(h, x.st, x.pdl));
    ++s->launch_count;
    IQ_CUDA(accept_launch(h, x.st, x.pdl));
    MtpStepArgs a = {};
    a.tokens = s->tokens.as<int32_t>();
    a.result = s->mtp_res.as<int>();
    a.scores = s->scores.as<float>();
    a.out_tok = out;
    a.out_prob = reinterpret_cast<float*>(out + kMaxDraft);
    a.out_margin = reinterpret_cast<float*>(out + 2 * kMaxDraft);
    a.i = i;
    a.xn = s->xn.as<float>();
    a.hin = s->mtp_hin.as<float>();
    a.hidden = H;
    ++s->launch_count;
    IQ_CUDA(mtp_step_launch(a, x.st, x.pdl));
    x.mark("mtp.pick");
  }
  return IQ_OK;
}

// Replay `ge` if it exists; otherwise run `body` eagerly once (so lazily set
// kernel attributes are configured outside any capture) and capture it into
// `ge` on the next call.  Under profiling the body always runs eagerly.
template <class F>
int run_captured(iq_state* s, cudaGraphExec_t& ge, int& eager, F body) {
  if (s->profiling) return body();
  if (!ge) {
    if (eager++ == 0) return body();
    cudaGraph_t g = nullptr;
    IQ_CUDA(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    const int64_t before = s->launch_count;
    int rc = body();
    const int64_t n = s->launch_count - before;
    s->launch_count = before;
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    IQ_CUDA(e);
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    IQ_CUDA(e);
    s->mtp_graph_launches[&ge] = n;
  }
  IQ_CUDA(cudaGraphLaunch(ge, s->st));
  s->launch_count += s->mtp_graph_launches[&ge];
  return IQ_OK;
}

// Run a pass through its CUDA graph: the first call of each (mode, rows)
// runs eagerly (so lazily configured kernel attributes are set outside any
// capture), the second captures the launch sequence, later calls replay it.
int run_pass_graph(iq_state* s, int k, bool verify) {
  if (s->profiling) {
    Ctx x(s);
    x.mark("start");
    return run_pass(s, k, verify);
  }
  const int v = verify ? 1 : 0;
  cudaGraphExec_t& ge = s->graphs[v][k - 1];
  if (!ge) {
    if (s->eager_runs[v][k - 1]++ == 0) return run_pass(s, k, verify);
    cudaGraph_t g = nullptr;
    IQ_CUDA(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
    const int64_t before = s->launch_count;
    int rc = run_pass(s, k, verify);
    s->graph_launches[v][k - 1] = (int)(s->launch_count - before);
    s->launch_count = before;
    cudaError_t e = cudaStreamEndCapture(s->st, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    IQ_CUDA(e);
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    IQ_CUDA(e);
  }
  IQ_CUDA(cudaGraphLaunch(ge, s->st));
  s->launch_count += s->graph_launches[v][k - 1];
  return IQ_OK;
}

// Fold the recorded stage events into per-stage totals (call after a sync).
void collect_marks(iq_state* s) {
  for (size_t i = 1; i < s->marks.size(); i++) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, s->marks[i - 1].second, s->marks[i].second);
    const std::string& name = s->marks[i].first == "start" ? std::string("host.gap") : s->marks[i].first;
    auto it = std::find_if(s->prof.begin(), s->prof.end(), [&](auto& p) { return p.first == name; });
    if (it == s->prof.end()) s->prof.push_back({name, {1, ms * 1000.0}});
    else { it->second.first++; it->second.second += ms * 1000.0; }
  }
  for (auto& m : s->marks) cudaEventDestroy(m.second);
  s->marks.clear();
}

int alloc_state(iq_state* s) {
  iq_model* m = s->m;
  const iq_config& c = m->cfg;
  const int K = kMaxK;
  const int64_t H = c.hidden_size;
  const int64_t vdim = (int64_t)c.linear_num_value_heads * c.linear_value_head_dim;
  const int64_t conv_dim = 2 * (int64_t)c.linear_num_key_heads * c.linear_key_head_dim + vdim;
  const int64_t nhd = (int64_t)c.num_attention_heads * c.head_dim;
  const int64_t kvd = (int64_t)c.num_key_value_heads * c.head_dim;
  const int64_t E = c.num_experts, topk = c.num_experts_per_tok;
  const int64_t F = c.moe_intermediate_size, Fs = c.shared_expert_intermediate_size;
  IQ_CUDA(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  IQ_CUDA(cudaMallocHost(&s->h_result, 8 * sizeof(int)));
  memset(s->h_result, 0, 8 * sizeof(int));
  IQ_CUDA(cudaMallocHost(&s->h_tokens, kMaxK * sizeof(int32_t)));
  IQ_CUDA(s->ctrl.reserve(8 * sizeof(int)));
  IQ_CUDA(cudaMemset(s->ctrl.p, 0, 8 * sizeof(int)));
  IQ_CUDA(s->tokens.reserve(kMaxK * sizeof(int32_t)));
  const int64_t K_conv = c.linear_conv_kernel_dim - 1;
  std::vector<DeltaNetLayer> dl;
  static_assert(kStateRing > kMaxK, "the conv ring holds a pass's rows plus the state before it");
  static_assert(kMaxRowsDelta >= kMaxK, "update records cover every row of a pass");
  IQ_CHECK(m->n_linear == 0 || deltanet_supported(c.linear_key_head_dim, c.linear_value_head_dim), IQ_EUNSUPPORTED,
           "DeltaNet head dims %d x %d (supported: 32, 64, 128 each)", c.linear_key_head_dim,
           c.linear_value_head_dim);
  const int rec_stride = deltanet_rec_stride(c.linear_key_head_dim, c.linear_value_head_dim);
  s->conv.resize(kStateRing * m->n_linear);
  s->rec.resize(m->n_linear);
  s->rec_log.resize(m->n_linear);
  s->dn_qkv.resize(m->n_linear);
  s->dn_ba.resize(m->n_linear);
  int li = 0;
  for (const Layer& L : m->layers) {
    if (L.type != kLinear) continue;
    DeltaNetLayer d = {};
    for (int b = 0; b < kStateRing; b++) {
      DevBuf& cb = s->conv[kStateRing * li + b];
      IQ_CUDA(cb.reserve(std::max<int64_t>(1, conv_dim * K_conv) * 4));
      d.conv_state[b] = cb.as<float>();
    }
    IQ_CUDA(s->rec[li].reserve((size_t)c.linear_num_value_heads * c.linear_key_head_dim * c.linear_value_head_dim * 4));
    IQ_CUDA(s->rec_log[li].reserve((size_t)c.linear_num_value_heads * kMaxRowsDelta * rec_stride * 4));
    d.rec_state = s->rec[li].as<float>();
    d.rec_log = s->rec_log[li].as<float>();
    d.conv_w = L.dn.conv_w.p();
    d.ssm_a = L.dn.ssm_a.p();
    d.dt_bias = L.dn.dt_bias.p();
    IQ_CUDA(s->dn_qkv[li].reserve((size_t)(K * conv_dim * 4)));
    IQ_CUDA(s->dn_ba[li].reserve((size_t)(K * 2 * c.linear_num_value_heads * 4)));
    dl.push_back(d);
    li++;
  }
  if (!dl.empty()) {
    IQ_CUDA(s->dn_layers.reserve(dl.size() * sizeof(DeltaNetLayer)));
    IQ_CUDA(cudaMemcpy(s->dn_layers.p, dl.data(), dl.size() * sizeof(DeltaNetLayer), cudaMemcpyHostToDevice));
  }
  s->kc.resize(m->n_full + (m->has_mtp ? 1 : 0));
  s->vc.resize(s->kc.size());
  for (size_t i = 0; i < s->kc.size(); i++) {
    IQ_CUDA(s->kc[i].reserve((size_t)(align_up(s->max_pos + kMaxK, kAttnChunk) * kvd * 4)));
    IQ_CUDA(s->vc[i].reserve((size_t)(align_up(s->max_pos + kMaxK, kAttnChunk) * kvd * 4)));
  }
  const int64_t maxcols = std::max({H, vdim, nhd, 2 * H});
  s->act8k_bytes = act_row_bytes_q8k(maxcols);
  s->act80_bytes = act_row_bytes_q80(maxcols);
  IQ_CUDA(s->hidden.reserve(K * H * 4));
  IQ_CUDA(s->xn.reserve(K * H * 4));
  IQ_CUDA(s->act8k.reserve(K * s->act8k_bytes));
  IQ_CUDA(s->act80.reserve(K * s->act80_bytes));
  IQ_CUDA(s->z.reserve(K * std::max<int64_t>(vdim, 1) * 4));
  IQ_CUDA(s->dn_out.reserve(K * std::max<int64_t>(vdim, 1) * 4));
  IQ_CUDA(s->qg.reserve(K * 2 * nhd * 4));
  IQ_CUDA(s->kp.reserve(K * kvd * 4));
  IQ_CUDA(s->vp.reserve(K * kvd * 4));
  IQ_CUDA(s->qbuf.reserve(K * nhd * 4));
  IQ_CUDA(s->attn_out.reserve(K * nhd * 4));
  s->max_chunks = (int)ceil_div(s->max_pos + kMaxK, kAttnChunk);
  IQ_CUDA(s->part.reserve((size_t)K * c.num_attention_heads * s->max_chunks * (c.head_dim + 2) * 4));
  const int64_t slots = K * topk + K;
  IQ_CUDA(s->logits_moe.reserve(K * (E + 1) * 4));
  IQ_CUDA(s->route_e.reserve((c.num_hidden_layers + 1) * K * topk * 4));
  IQ_CUDA(s->route_w.reserve(K * topk * 4));
  IQ_CUDA(s->gu_jobs.reserve((2 * E + 2) * sizeof(QmvJob)));
  IQ_CUDA(s->down_jobs.reserve((E + 1) * sizeof(QmvJob)));
  IQ_CUDA(s->counts.reserve((4 + c.num_hidden_layers + 2) * 4));
  IQ_CUDA(cudaMemset(s->counts.p, 0, (4 + c.num_hidden_layers + 2) * 4));
  IQ_CUDA(s->union_list.reserve(E * 4));
  s->gu_ld = (int)(2 * std::max(F, Fs));
  IQ_CUDA(s->gu_out.reserve(slots * s->gu_ld * 4));
  s->act_mid_bytes = std::max(act_row_bytes_q8k(std::max(F, Fs)), act_row_bytes_q80(std::max(F, Fs)));
  IQ_CUDA(s->act_mid.reserve(slots * s->act_mid_bytes));
  IQ_CUDA(s->y.reserve(slots * H * 4));
  IQ_CUDA(s->logits.reserve((size_t)K * c.vocab_size * 4));
  IQ_CUDA(s->pval.reserve(K * kArgmaxParts * 3 * 4));
  IQ_CUDA(s->pidx.reserve(K * kArgmaxParts * 4));
  IQ_CUDA(s->argmax.reserve(K * 4));
  IQ_CUDA(s->scores.reserve(4 * 4));
  if (m->has_mtp) {
    IQ_CUDA(s->mtp_xcat.reserve(K * 2 * H * 4));
    IQ_CUDA(s->mtp_hin.reserve(K * H * 4));
    IQ_CUDA(s->mtp_res.reserve(4 * 4));
    IQ_CUDA(s->mtp_out.reserve(3 * kMaxDraft * 4));
    IQ_CUDA(cudaMallocHost(&s->h_mtp, (size_t)(K * H + 3 * kMaxDraft) * 4));
  }
  return build_plans(s);
}

// After a synchronized pass: a GEMV that gave up waiting for its weights
// (bounded wait) fails the call with IQ_ETIMEDOUT; the flag is cleared.
int check_device_waits(iq_state* s) {
  if (!s->h_result[4]) return IQ_OK;
  s->h_result[4] = 0;
  if (int* f = qmv_timeout_flag()) IQ_CUDA(cudaMemset(f, 0, sizeof(int)));
  set_error("a GEMV gave up waiting for its weight tiles (bounded device wait); results of this pass are invalid");
  return IQ_ETIMEDOUT;
}

int reset_state(iq_state* s) {
  for (auto& b : s->conv) IQ_CUDA(cudaMemsetAsync(b.p, 0, b.bytes, s->st));
  for (auto& b : s->rec) IQ_CUDA(cudaMemsetAsync(b.p, 0, b.bytes, s->st));
  for (auto& b : s->rec_log) IQ_CUDA(cudaMemsetAsync(b.p, 0, b.bytes, s->st));
  IQ_CUDA(cudaMemsetAsync(s->ctrl.p, 0, 8 * sizeof(int), s->st));
  IQ_CUDA(cudaStreamSynchronize(s->st));
  s->position = 0;
  s->mtp_position = 0;
  s->can_rollback = false;
  return IQ_OK;
}

int copy_out(iq_state* s, int k, int row0, float* logits, float* hidden, int32_t* argmax) {
  const iq_config& c = s->m->cfg;
  if (logits)
    IQ_CUDA(cudaMemcpyAsync(logits + (int64_t)row0 * c.vocab_size, s->logits.p, (size_t)k * c.vocab_size * 4,
                            cudaMemcpyDeviceToHost, s->st));
  if (hidden)
    IQ_CUDA(cudaMemcpyAsync(hidden + (int64_t)row0 * c.hidden_size, s->xn.p, (size_t)k * c.hidden_size * 4,
                            cudaMemcpyDeviceToHost, s->st));
  if (argmax)
    IQ_CUDA(cudaMemcpyAsync(argmax + row0, s->argmax.p, (size_t)k * 4, cudaMemcpyDeviceToHost, s->st));
  return IQ_OK;
}

}  // namespace
}  // namespace iq

using namespace iq;

extern "C" {

int iq_state_create(iq_model* m, int64_t max_positions, iq_state** out) {
  clear_error();
  IQ_CHECK(m && out, IQ_EINVAL, "iq_state_create: null argument");
  IQ_CHECK(max_positions > 0 && max_positions <= m->cfg.max_position_embeddings, IQ_EINVAL,
           "max_positions %lld outside 1..%d", (long long)max_positions, m->cfg.max_position_embeddings);
  std::unique_ptr<iq_state> s(new iq_state);
  s->m = m;
  s->max_pos = max_positions;
  int rc = alloc_state(s.get());
  if (rc) return rc;
  rc = reset_state(s.get());
  if (rc) return rc;
  *out = s.release();
  return IQ_OK;
}

void iq_state_destroy(iq_state* s) {
  if (s && s->st) cudaStreamSynchronize(s->st);
  delete s;
}

int iq_state_reset(iq_state* s) {
  clear_error();
  IQ_CHECK(s, IQ_EINVAL, "iq_state_reset: null state");
  return reset_state(s);
}

// ------------------------------------------------------------ state image
// A self-contained copy of a sequence's state (SessionImage / QuantizedStateImage,
// src/runtime.rs:566-592, src/qwen/quantized_model.rs:59-100): a header, then
// per decoder layer in order either the KV rows [pos][kv_head][head_dim]
// (keys, then values) or the DeltaNet conv state [channel][K-1] and recurrent
// state [head][key][value], then the MTP block's KV rows.  All f32.
struct StateImageHeader {
  char magic[8];
  int32_t version, layers;
  int64_t position, mtp_position;
  int32_t has_mtp, kv_dim, conv_dim, conv_taps, rec_size, pad;
};
static_assert(sizeof(StateImageHeader) == 56, "image header layout");

namespace {
const char kImageMagic[8] = {'I', 'Q', 'S', 'T', 'A', 'T', 'E', '1'};

StateImageHeader image_header(const iq_state* s) {
  const iq_config& c = s->m->cfg;
  StateImageHeader h = {};
  memcpy(h.magic, kImageMagic, 8);
  h.version = 1;
  h.layers = c.num_hidden_layers;
  h.position = s->position;
  h.mtp_position = s->m->has_mtp ? s->mtp_position : 0;
  h.has_mtp = s->m->has_mtp ? 1 : 0;
  h.kv_dim = c.num_key_value_heads * c.head_dim;
  const int vdim = c.linear_num_value_heads * c.linear_value_head_dim;
  h.conv_dim = 2 * c.linear_num_key_heads * c.linear_key_head_dim + vdim;
  h.conv_taps = c.linear_conv_kernel_dim - 1;
  h.rec_size = c.linear_num_value_heads * c.linear_key_head_dim * c.linear_value_head_dim;
  return h;
}

int64_t image_bytes(const iq_state* s, const StateImageHeader& h) {
  int64_t b = sizeof(StateImageHeader);
  for (const Layer& L : s->m->layers)
    b += L.type == kFull ? 2 * h.position * h.kv_dim * 4 : ((int64_t)h.conv_dim * h.conv_taps + h.rec_size) * 4;
  if (h.has_mtp) b += 2 * h.mtp_position * h.kv_dim * 4;
  return b;
}
}  // namespace

int iq_state_image_size(const iq_state* s, int64_t* bytes) {
  IQ_CHECK(s && bytes, IQ_EINVAL, "iq_state_image_size: null argument");
  *bytes = image_bytes(s, image_header(s));
  return IQ_OK;
}

int iq_state_export(iq_state* s, void* out, int64_t bytes) {
  clear_error();
  IQ_CHECK(s && out, IQ_EINVAL, "iq_state_export: null argument");
  const StateImageHeader h = image_header(s);
  const int64_t need = image_bytes(s, h);
  IQ_CHECK(bytes >= need, IQ_EINVAL, "state image needs %lld bytes, buffer holds %lld", (long long)need,
           (long long)bytes);
  IQ_CUDA(cudaStreamSynchronize(s->st));
  int ctrl[8];
  IQ_CUDA(cudaMemcpy(ctrl, s->ctrl.p, sizeof ctrl, cudaMemcpyDeviceToHost));
  const int cur = ctrl[1], pending = ctrl[6];
  const iq_config& c = s->m->cfg;
  const int dk = c.linear_key_head_dim, dv = c.linear_value_head_dim, nv = c.linear_num_value_heads;
  const int rec_stride = deltanet_rec_stride(dk, dv);
  std::vector<float> log;
  uint8_t* p = static_cast<uint8_t*>(out);
  memcpy(p, &h, sizeof h);
  p += sizeof h;
  int li = 0, fi = 0;
  for (const Layer& L : s->m->layers) {
    if (L.type == kFull) {
      const size_t n = (size_t)h.position * h.kv_dim * 4;
      IQ_CUDA(cudaMemcpy(p, s->kc[fi].p, n, cudaMemcpyDeviceToHost));
      IQ_CUDA(cudaMemcpy(p + n, s->vc[fi].p, n, cudaMemcpyDeviceToHost));
      p += 2 * n;
      fi++;
    } else {
      const size_t nc = (size_t)h.conv_dim * h.conv_taps * 4, nr = (size_t)h.rec_size * 4;
      if (nc) IQ_CUDA(cudaMemcpy(p, s->conv[kStateRing * li + cur].p, nc, cudaMemcpyDeviceToHost));
      IQ_CUDA(cudaMemcpy(p + nc, s->rec[li].p, nr, cudaMemcpyDeviceToHost));
      if (pending > 0) {
        // the committed rows of the last pass: replay their update records
        // (S = S * decay + k delta, each product rounded; the host build
        // does not contract these into fused multiply-adds), as the next
        // pass would on the device
        log.resize((size_t)nv * kMaxRowsDelta * rec_stride);
        IQ_CUDA(cudaMemcpy(log.data(), s->rec_log[li].p, log.size() * 4, cudaMemcpyDeviceToHost));
        float* S = reinterpret_cast<float*>(p + nc);
        for (int h = 0; h < nv; h++)
          for (int r = 0; r < pending; r++) {
            const float* rc = log.data() + ((size_t)h * kMaxRowsDelta + r) * rec_stride;
            const float decay = rc[dk + dv];
            float* Sh = S + (size_t)h * dk * dv;
            for (int i = 0; i < dk; i++)
              for (int j = 0; j < dv; j++) {
                const float a = Sh[(size_t)i * dv + j] * decay;
                const float b = rc[i] * rc[dk + j];
                Sh[(size_t)i * dv + j] = a + b;
              }
          }
      }
      p += nc + nr;
      li++;
    }
  }
  if (h.has_mtp) {
    const size_t n = (size_t)h.mtp_position * h.kv_dim * 4;
    IQ_CUDA(cudaMemcpy(p, s->kc[s->m->n_full].p, n, cudaMemcpyDeviceToHost));
    IQ_CUDA(cudaMemcpy(p + n, s->vc[s->m->n_full].p, n, cudaMemcpyDeviceToHost));
  }
  return IQ_OK;
}

int iq_state_import(iq_state* s, const void* in, int64_t bytes) {
  clear_error();
  IQ_CHECK(s && in, IQ_EINVAL, "iq_state_import: null argument");
  IQ_CHECK(bytes >= (int64_t)sizeof(StateImageHeader), IQ_EINVAL, "state image of %lld bytes has no header",
           (long long)bytes);
  StateImageHeader h;
  memcpy(&h, in, sizeof h);
  const StateImageHeader mine = image_header(s);
  IQ_CHECK(memcmp(h.magic, kImageMagic, 8) == 0 && h.version == 1, IQ_EINVAL, "not a version-1 state image");
  IQ_CHECK(h.layers == mine.layers && h.kv_dim == mine.kv_dim && h.conv_dim == mine.conv_dim &&
               h.conv_taps == mine.conv_taps && h.rec_size == mine.rec_size && h.has_mtp == mine.has_mtp,
           IQ_EINVAL, "state image shapes do not match the loaded model");
  IQ_CHECK(h.position >= 0 && h.position <= s->max_pos && h.mtp_position >= 0 && h.mtp_position <= s->max_pos,
           IQ_EINVAL, "state image at position %lld exceeds the state's %lld positions", (long long)h.position,
           (long long)s->max_pos);
  const int64_t need = image_bytes(s, h);
  IQ_CHECK(bytes == need, IQ_EINVAL, "state image holds %lld bytes, its header describes %lld", (long long)bytes,
           (long long)need);
  IQ_CUDA(cudaStreamSynchronize(s->st));
  const uint8_t* p = static_cast<const uint8_t*>(in) + sizeof h;
  int li = 0, fi = 0;
  for (const Layer& L : s->m->layers) {
    if (L.type == kFull) {
      const size_t n = (size_t)h.position * h.kv_dim * 4;
      IQ_CUDA(cudaMemcpy(s->kc[fi].p, p, n, cudaMemcpyHostToDevice));
      IQ_CUDA(cudaMemcpy(s->vc[fi].p, p + n, n, cudaMemcpyHostToDevice));
      p += 2 * n;
      fi++;
    } else {
      const size_t nc = (size_t)h.conv_dim * h.conv_taps * 4, nr = (size_t)h.rec_size * 4;
      if (nc) IQ_CUDA(cudaMemcpy(s->conv[kStateRing * li].p, p, nc, cudaMemcpyHostToDevice));
      IQ_CUDA(cudaMemcpy(s->rec[li].p, p + nc, nr, cudaMemcpyHostToDevice));
      p += nc + nr;
      li++;
    }
  }
  if (h.has_mtp) {
    const size_t n = (size_t)h.mtp_position * h.kv_dim * 4;
    IQ_CUDA(cudaMemcpy(s->kc[s->m->n_full].p, p, n, cudaMemcpyHostToDevice));
    IQ_CUDA(cudaMemcpy(s->vc[s->m->n_full].p, p + n, n, cudaMemcpyHostToDevice));
  }
  // the imported DeltaNet state is conv ring slot 0 and the recurrent base
  // with no records pending; positions from the header
  int ctrl[8] = {(int)h.position, 0, 0, 0, 0, (int)h.mtp_position, 0, 0};
  IQ_CUDA(cudaMemcpy(s->ctrl.p, ctrl, sizeof ctrl, cudaMemcpyHostToDevice));
  s->position = h.position;
  s->mtp_position = h.mtp_position;
  s->can_rollback = false;
  return IQ_OK;
}

int iq_state_position(const iq_state* s, int64_t* position) {
  IQ_CHECK(s && position, IQ_EINVAL, "iq_state_position: null argument");
  *position = s->position;
  return IQ_OK;
}

int iq_state_stream(const iq_state* s, void** stream) {
  IQ_CHECK(s && stream, IQ_EINVAL, "iq_state_stream: null argument");
  *stream = s->st;
  return IQ_OK;
}

int iq_forward(iq_state* s, const uint32_t* tokens, int rows, float* logits, float* hidden, int32_t* argmax) {
  clear_error();
  IQ_CHECK(s && tokens, IQ_EINVAL, "iq_forward: null argument");
  IQ_CHECK(rows >= 1, IQ_EINVAL, "forward requires at least one token");
  IQ_CHECK(s->position + rows <= s->max_pos, IQ_EINVAL, "sequence exceeds the state's %lld positions",
           (long long)s->max_pos);
  const int V = s->m->cfg.vocab_size;
  for (int i = 0; i < rows; i++)
    IQ_CHECK(tokens[i] < (uint32_t)V, IQ_EINVAL, "token %u outside the vocabulary of %d", tokens[i], V);
  if (rows >= kWideMin && !s->profiling && !getenv("IQ_NO_WIDE") && wide_capable(s->m)) {
    // prefill-sized: the wide pass (tensor-core projections, grouped experts)
    IQ_CUDA(cudaStreamSynchronize(s->st));
    int rc = wide_forward(s, tokens, rows, logits, hidden, argmax);
    if (rc) return rc;
    int wflag = 0;
    if (int* f = wide_timeout_flag()) {
      IQ_CUDA(cudaMemcpy(&wflag, f, sizeof(int), cudaMemcpyDeviceToHost));
      if (wflag) IQ_CUDA(cudaMemset(f, 0, sizeof(int)));
    }
    if (int* f = qmv_timeout_flag()) IQ_CUDA(cudaMemcpy(s->h_result + 4, f, sizeof(int), cudaMemcpyDeviceToHost));
    TRY(check_device_waits(s));
    IQ_CHECK(!wflag, IQ_ETIMEDOUT, "a wide product gave up a bounded device wait; results of this call are invalid");
    s->can_rollback = true;
    return IQ_OK;
  }
  for (int r0 = 0; r0 < rows; r0 += kMaxK) {
    const int k = std::min(kMaxK, rows - r0);
    IQ_CUDA(cudaStreamSynchronize(s->st));  // h_tokens is reused
    for (int i = 0; i < k; i++) s->h_tokens[i] = (int32_t)tokens[r0 + i];
    int rc = run_pass_graph(s, k, false);
    if (rc) return rc;
    rc = copy_out(s, k, r0, logits, hidden, argmax);
    if (rc) return rc;
    s->position += k;
    s->last_rows = k;
  }
  IQ_CUDA(cudaStreamSynchronize(s->st));
  if (s->profiling) collect_marks(s);
  TRY(check_device_waits(s));
  s->can_rollback = true;
  return IQ_OK;
}

int iq_verify(iq_state* s, const uint32_t* tokens, int rows, iq_verify_result* out, float* logits, float* hidden) {
  clear_error();
  IQ_CHECK(s && tokens && out, IQ_EINVAL, "iq_verify: null argument");
  IQ_CHECK(rows >= 1 && rows <= kMaxK, IQ_EINVAL, "verify takes 1..%d rows, got %d", kMaxK, rows);
  IQ_CHECK(s->position + rows <= s->max_pos, IQ_EINVAL, "sequence exceeds the state's %lld positions",
           (long long)s->max_pos);
  const int V = s->m->cfg.vocab_size;
  for (int i = 0; i < rows; i++)
    IQ_CHECK(tokens[i] < (uint32_t)V, IQ_EINVAL, "token %u outside the vocabulary of %d", tokens[i], V);
  IQ_CUDA(cudaStreamSynchronize(s->st));
  for (int i = 0; i < rows; i++) s->h_tokens[i] = (int32_t)tokens[i];
  int rc = run_pass_graph(s, rows, true);
  if (rc) return rc;
  rc = copy_out(s, rows, 0, logits, hidden, nullptr);
  if (rc) return rc;
  IQ_CUDA(cudaStreamSynchronize(s->st));
  if (s->profiling) collect_marks(s);
  TRY(check_device_waits(s));
  out->accepted = s->h_result[0];
  out->authoritative = s->h_result[1];
  out->committed = s->h_result[2];
  s->position += out->committed;
  s->can_rollback = false;
  return IQ_OK;
}

// Row r of the MTP inputs takes the target's hidden row of the position
// before it: prev_hidden (or zeros at position 0) for the first, then rows
// 0..rows-2 of target_hidden (shifted_hidden_inputs, src/runtime.rs:2184-2223).
static void shifted_row(const float* prev_hidden, const float* target_hidden, int r, int H, float* dst) {
  if (r > 0) memcpy(dst, target_hidden + (int64_t)(r - 1) * H, (size_t)H * 4);
  else if (prev_hidden) memcpy(dst, prev_hidden, (size_t)H * 4);
  else memset(dst, 0, (size_t)H * 4);
}

int iq_mtp_shifted_inputs(const float* prev_hidden, const float* target_hidden, int rows, int hidden, float* out) {
  clear_error();
  IQ_CHECK(target_hidden && out && rows >= 0 && hidden > 0, IQ_EINVAL, "iq_mtp_shifted_inputs: bad argument");
  for (int r = 0; r < rows; r++) shifted_row(prev_hidden, target_hidden, r, hidden, out + (int64_t)r * hidden);
  return IQ_OK;
}

int iq_mtp_sync(iq_state* s, int64_t position, const float* prev_hidden, const uint32_t* tokens, int rows,
                const float* target_hidden) {
  clear_error();
  IQ_CHECK(s && tokens && target_hidden, IQ_EINVAL, "iq_mtp_sync: null argument");
  IQ_CHECK(s->m->has_mtp, IQ_EUNSUPPORTED, "the model has no MTP block");
  IQ_CHECK(rows >= 1, IQ_EINVAL, "MTP catch-up needs at least one row");
  IQ_CHECK(position >= 0 && position <= s->mtp_position, IQ_EINVAL,
           "MTP state at position %lld is behind target position %lld", (long long)s->mtp_position,
           (long long)position);
  IQ_CHECK(prev_hidden || position == 0, IQ_EINVAL, "previous target hidden row is required after position zero");
  IQ_CHECK(position + rows <= s->max_pos, IQ_EINVAL, "MTP catch-up exceeds the state's %lld positions",
           (long long)s->max_pos);
  const iq_config& c = s->m->cfg;
  const int H = c.hidden_size;
  for (int i = 0; i < rows; i++)
    IQ_CHECK(tokens[i] < (uint32_t)c.vocab_size, IQ_EINVAL, "token %u outside the vocabulary of %d", tokens[i],
             c.vocab_size);
  IQ_CUDA(cudaStreamSynchronize(s->st));
  IQ_CUDA(set_int_launch(s->ctrl.as<int>() + 5, (int)position, false, s->st, false));
  s->mtp_position = position;
  for (int r0 = 0; r0 < rows; r0 += kMaxK) {
    const int k = std::min(kMaxK, rows - r0);
    IQ_CUDA(cudaStreamSynchronize(s->st));  // pinned staging is reused
    for (int i = 0; i < k; i++) {
      s->h_tokens[i] = (int32_t)tokens[r0 + i];
      shifted_row(prev_hidden, target_hidden, r0 + i, H, s->h_mtp + (int64_t)i * H);
    }
    IQ_CUDA(cudaMemcpyAsync(s->tokens.p, s->h_tokens, k * 4, cudaMemcpyHostToDevice, s->st));
    IQ_CUDA(cudaMemcpyAsync(s->mtp_hin.p, s->h_mtp, (size_t)k * H * 4, cudaMemcpyHostToDevice, s->st));
    int rc = run_captured(s, s->mtp_sync_graphs[k - 1], s->mtp_sync_eager[k - 1], [&] { return run_mtp_block(s, k); });
    if (rc) return rc;
  }
  IQ_CUDA(cudaStreamSynchronize(s->st));
  if (s->profiling) collect_marks(s);
  s->mtp_position = position + rows;
  return IQ_OK;
}

int iq_mtp_draft(iq_state* s, uint32_t seed, const float* hidden, int depth, int draft_vocab, float min_conf,
                 uint32_t* tokens, float* probs, float* margins, int* n) {
  clear_error();
  IQ_CHECK(s && hidden && tokens && n, IQ_EINVAL, "iq_mtp_draft: null argument");
  IQ_CHECK(s->m->has_mtp, IQ_EUNSUPPORTED, "the model has no MTP block");
  const iq_config& c = s->m->cfg;
  const int H = c.hidden_size;
  IQ_CHECK(depth >= 1 && depth <= kMaxDraft, IQ_EINVAL, "MTP drafts 1..%d tokens per call, got %d", kMaxDraft,
           depth);
  IQ_CHECK(draft_vocab >= 1 && draft_vocab <= c.vocab_size, IQ_EINVAL,
           "draft vocabulary %d outside 1..%d", draft_vocab, c.vocab_size);
  IQ_CHECK(seed < (uint32_t)c.vocab_size, IQ_EINVAL, "token %u outside the vocabulary of %d", seed, c.vocab_size);
  IQ_CHECK(s->mtp_position + depth <= s->max_pos, IQ_EINVAL, "MTP drafting exceeds the state's %lld positions",
           (long long)s->max_pos);
  IQ_CUDA(cudaStreamSynchronize(s->st));
  s->h_tokens[0] = (int32_t)seed;
  memcpy(s->h_mtp, hidden, (size_t)H * 4);
  IQ_CUDA(cudaMemcpyAsync(s->tokens.p, s->h_tokens, 4, cudaMemcpyHostToDevice, s->st));
  IQ_CUDA(cudaMemcpyAsync(s->mtp_hin.p, s->h_mtp, (size_t)H * 4, cudaMemcpyHostToDevice, s->st));
  int rc = mtp_head_job(s, draft_vocab);
  if (rc) return rc;
  if (s->profiling) {
    Ctx x(s);
    x.mark("start");
  }
  const auto key = std::make_pair(depth, draft_vocab);
  rc = run_captured(s, s->mtp_draft_graphs[key], s->mtp_draft_eager[key],
                    [&] { return run_mtp_draft(s, depth, draft_vocab); });
  if (rc) return rc;
  float* ho = s->h_mtp + (int64_t)kMaxK * H;
  IQ_CUDA(cudaMemcpyAsync(ho, s->mtp_out.p, 3 * kMaxDraft * 4, cudaMemcpyDeviceToHost, s->st));
  IQ_CUDA(cudaStreamSynchronize(s->st));
  if (s->profiling) collect_marks(s);
  s->mtp_position += depth;
  const int* ot = reinterpret_cast<const int*>(ho);
  int m = 0;
  // draft_mtp stops before a token whose top-1 probability is below min_conf
  while (m < depth && ho[kMaxDraft + m] >= min_conf) m++;
  for (int i = 0; i < depth; i++) {
    tokens[i] = (uint32_t)ot[i];
    if (probs) probs[i] = ho[kMaxDraft + i];
    if (margins) margins[i] = ho[2 * kMaxDraft + i];
  }
  *n = m;
  return IQ_OK;
}

int iq_mtp_position(const iq_state* s, int64_t* position) {
  IQ_CHECK(s && position, IQ_EINVAL, "iq_mtp_position: null argument");
  *position = s->mtp_position;
  return IQ_OK;
}

int iq_rollback(iq_state* s, int committed_rows) {
  clear_error();
  IQ_CHECK(s, IQ_EINVAL, "iq_rollback: null state");
  IQ_CHECK(s->can_rollback, IQ_ESTATE, "no forward pass to roll back");
  IQ_CHECK(committed_rows >= 0 && committed_rows < s->last_rows, IQ_EINVAL,
           "cannot roll back to %d of %d committed rows", committed_rows, s->last_rows);
  rollback_kernel<<<1, 1, 0, s->st>>>(s->ctrl.as<int>(), s->last_rows, committed_rows);
  IQ_CUDA(cudaGetLastError());
  IQ_CUDA(cudaStreamSynchronize(s->st));
  s->position -= s->last_rows - committed_rows;
  s->can_rollback = false;
  return IQ_OK;
}

int iq_state_union_sizes(const iq_state* s, int32_t* per_layer) {
  IQ_CHECK(s && per_layer, IQ_EINVAL, "iq_state_union_sizes: null argument");
  IQ_CUDA(cudaStreamSynchronize(s->st));
  IQ_CUDA(cudaMemcpy(per_layer, s->counts.as<int>() + 4, s->m->cfg.num_hidden_layers * 4, cudaMemcpyDeviceToHost));
  return IQ_OK;
}

int iq_state_set_profiling(iq_state* s, int on) {
  IQ_CHECK(s, IQ_EINVAL, "iq_state_set_profiling: null state");
  IQ_CUDA(cudaStreamSynchronize(s->st));
  for (auto& m : s->marks) cudaEventDestroy(m.second);
  s->marks.clear();
  s->prof.clear();
  s->profiling = on != 0;
  return IQ_OK;
}

int iq_state_profile(const iq_state* s, char* buf, int len) {
  IQ_CHECK(s && buf && len > 0, IQ_EINVAL, "iq_state_profile: null argument");
  std::string out;
  char line[256];
  for (auto& p : s->prof) {
    snprintf(line, sizeof line, "%s %d %.3f\n", p.first.c_str(), p.second.first, p.second.second);
    out += line;
  }
  snprintf(buf, (size_t)len, "%s", out.c_str());
  return (int)out.size();
}

int iq_state_routes(const iq_state* s, int rows, int32_t* experts) {
  IQ_CHECK(s && experts, IQ_EINVAL, "iq_state_routes: null argument");
  IQ_CHECK(rows >= 1 && rows <= kMaxK, IQ_EINVAL, "rows must be 1..%d", kMaxK);
  const iq_config& c = s->m->cfg;
  IQ_CUDA(cudaStreamSynchronize(s->st));
  for (int l = 0; l < c.num_hidden_layers; l++)
    IQ_CUDA(cudaMemcpy(experts + (int64_t)l * rows * c.num_experts_per_tok,
                       s->route_e.as<int>() + (int64_t)l * kMaxK * c.num_experts_per_tok,
                       (size_t)rows * c.num_experts_per_tok * 4, cudaMemcpyDeviceToHost));
  return IQ_OK;
}

int iq_state_launch_count(const iq_state* s, int64_t* count) {
  IQ_CHECK(s && count, IQ_EINVAL, "iq_state_launch_count: null argument");
  *count = s->launch_count;
  return IQ_OK;
}

}  // extern "C"
