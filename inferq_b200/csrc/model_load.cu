// model_load.cu -- iq_model_create: GGUF tensor views -> device weights.
//
// Tensor names and shape checks follow the reference loaders:
// src/qwen/quantized_layer.rs:73-76 (norms), quantized_deltanet.rs:399-451,
// quantized_attention.rs:348-382, quantized_moe.rs:147-201,
// quantized_mtp.rs:104-120, quantized_model.rs:512-539.
#include <cstring>
#include <unordered_map>
#include <nccl.h>
#include "model.h"

namespace iq {
namespace {

struct Loader {
  std::unordered_map<std::string, const iq_tensor_view*> by_name;
  cudaStream_t st = nullptr;

  const iq_tensor_view* find(const std::string& n) const {
    auto it = by_name.find(n);
    return it == by_name.end() ? nullptr : it->second;
  }
  int missing(const std::string& n) const {
    set_error("GGUF is missing tensor \"%s\"", n.c_str());
    return IQ_EINVAL;
  }
  static int64_t elems(const iq_tensor_view* v) {
    int64_t e = 1;
    for (int i = 0; i < v->ndim; i++) e *= v->shape[i];
    return e;
  }

  // The TMA tensor maps the GEMV streams a quantized weight through.
  static int maps_for(const std::string& n, Weight& w) {
    if (w.dt != Q4_K && w.dt != Q5_K && w.dt != Q6_K && w.dt != Q8_0) return IQ_OK;
    IQ_CHECK(qmv_tensor_maps(w.dt, w.p(), w.rows, w.cols, w.maps) == cudaSuccess, IQ_ECUDA,
             "cannot describe tensor \"%s\" for the TMA unit", n.c_str());
    return IQ_OK;
  }

  // A 2-D matrix [rows, cols] (a 3-D [a, b, cols] counts as a*b rows).
  int matrix(const std::string& n, int64_t rows, int64_t cols, Weight& w) const {
    const iq_tensor_view* v = find(n);
    if (!v) return missing(n);
    IQ_CHECK(v->ndim >= 2 && v->shape[v->ndim - 1] == cols && elems(v) == rows * cols, IQ_EINVAL,
             "invalid GGUF shape for \"%s\": expected [%lld, %lld]", n.c_str(), (long long)rows, (long long)cols);
    IQ_CHECK(v->dtype != BF16, IQ_EUNSUPPORTED,
             "tensor \"%s\" is BF16: the model pass takes quantized or F32 matrices (BF16 matrices run through "
             "the operator entry points)", n.c_str());
    int rc = validate_matrix_shape(v->dtype, rows, cols);
    if (rc) {
      set_error("tensor \"%s\": %s", n.c_str(), iq_last_error());
      return rc;
    }
    rc = upload_rows(v->dtype, v->data, rows, cols, v->location, w.buf, st);
    if (rc) return rc;
    w.dt = v->dtype;
    w.rows = rows;
    w.cols = cols;
    w.row_bytes = dev_row_bytes(v->dtype, cols);
    return maps_for(n, w);
  }

  // Rows [r0, r1) of a stacked-expert tensor [E, rows_per, cols].
  int expert_rows(const std::string& n, int64_t E, int64_t rows_per, int64_t cols, int64_t e0, int64_t e1,
                  Weight& w) const {
    const iq_tensor_view* v = find(n);
    if (!v) return missing(n);
    IQ_CHECK(v->ndim == 3 && v->shape[0] == E && v->shape[1] == rows_per && v->shape[2] == cols, IQ_EINVAL,
             "invalid expert shape for \"%s\": expected [%lld, %lld, %lld]", n.c_str(), (long long)E,
             (long long)rows_per, (long long)cols);
    IQ_CHECK(v->dtype != BF16, IQ_EUNSUPPORTED, "expert tensor \"%s\" is BF16 (quantized experts only)",
             n.c_str());
    int rc = validate_matrix_shape(v->dtype, rows_per, cols);
    if (rc) return rc;
    const uint8_t* base = static_cast<const uint8_t*>(v->data) + e0 * rows_per * gguf_row_bytes(v->dtype, cols);
    rc = upload_rows(v->dtype, base, (e1 - e0) * rows_per, cols, v->location, w.buf, st);
    if (rc) return rc;
    w.dt = v->dtype;
    w.rows = (e1 - e0) * rows_per;
    w.cols = cols;
    w.row_bytes = dev_row_bytes(v->dtype, cols);
    return maps_for(n, w);
  }

  // An F32 (or F16) tensor of n elements as f32 on the device.
  int vec(const std::string& name, int64_t n, Vec& out) const {
    const iq_tensor_view* v = find(name);
    if (!v) return missing(name);
    IQ_CHECK(elems(v) == n, IQ_EINVAL, "invalid length for \"%s\": %lld elements, expected %lld", name.c_str(),
             (long long)elems(v), (long long)n);
    IQ_CHECK(v->dtype == F32 || v->dtype == F16 || v->dtype == BF16, IQ_EUNSUPPORTED,
             "tensor \"%s\" must be F32, F16 or BF16", name.c_str());
    IQ_CUDA(out.buf.reserve((size_t)n * 4));
    out.n = n;
    if (v->dtype == F32) {
      IQ_CUDA(cudaMemcpy(out.buf.p, v->data, (size_t)n * 4,
                         v->location == IQ_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice));
      return IQ_OK;
    }
    IQ_CHECK(v->location == IQ_HOST, IQ_EUNSUPPORTED, "F16 / BF16 vector \"%s\" must be in host memory",
             name.c_str());
    std::vector<float> tmp(n);
    if (v->dtype == BF16) {  // exact widening (src/gguf.rs:1487-1495 loads BF16 vectors as f32)
      const uint16_t* h = static_cast<const uint16_t*>(v->data);
      for (int64_t i = 0; i < n; i++) {
        const uint32_t u = (uint32_t)h[i] << 16;
        memcpy(&tmp[i], &u, 4);
      }
    } else {
      const __half* h = static_cast<const __half*>(v->data);
      for (int64_t i = 0; i < n; i++) tmp[i] = __half2float(h[i]);
    }
    IQ_CUDA(cudaMemcpy(out.buf.p, tmp.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
    return IQ_OK;
  }
};

#define TRY(x)              \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

int load_moe(const Loader& L, const iq_config& c, const std::string& p, int rank, int world, MoeWeights& m) {
  const int64_t E = c.num_experts, H = c.hidden_size, F = c.moe_intermediate_size;
  const int64_t Fs = c.shared_expert_intermediate_size;
  TRY(iq_ep_expert_range(E, rank, world, &m.expert_lo, &m.expert_hi));
  const std::string rn = p + ".ffn_gate_inp.weight";
  const iq_tensor_view* rv = L.find(rn);
  if (!rv) return L.missing(rn);
  TRY(L.vec(p + ".ffn_gate_inp_shexp.weight", H, m.selector));
  if (rv->dtype == F32) {
    IQ_CHECK(Loader::elems(rv) == E * H, IQ_EINVAL, "invalid router shape for \"%s\"", rn.c_str());
    IQ_CUDA(m.router_sel.buf.reserve((size_t)((E + 1) * H * 4)));
    m.router_sel.n = (E + 1) * H;
    IQ_CUDA(cudaMemcpy(m.router_sel.buf.p, rv->data, (size_t)(E * H * 4),
                       rv->location == IQ_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice));
    IQ_CUDA(cudaMemcpy(m.router_sel.p() + E * H, m.selector.p(), (size_t)(H * 4), cudaMemcpyDeviceToDevice));
  } else {
    TRY(L.matrix(rn, E, H, m.router));
  }
  TRY(L.expert_rows(p + ".ffn_gate_exps.weight", E, F, H, m.expert_lo, m.expert_hi, m.gate));
  TRY(L.expert_rows(p + ".ffn_up_exps.weight", E, F, H, m.expert_lo, m.expert_hi, m.up));
  IQ_CHECK(m.up.dt == m.gate.dt, IQ_EUNSUPPORTED, "layer %s: gate and up experts differ in dtype", p.c_str());
  TRY(L.expert_rows(p + ".ffn_down_exps.weight", E, H, F, m.expert_lo, m.expert_hi, m.down));
  TRY(L.matrix(p + ".ffn_gate_shexp.weight", Fs, H, m.sh_gate));
  TRY(L.matrix(p + ".ffn_up_shexp.weight", Fs, H, m.sh_up));
  IQ_CHECK(m.sh_up.dt == m.sh_gate.dt, IQ_EUNSUPPORTED, "layer %s: shared gate and up differ in dtype", p.c_str());
  TRY(L.matrix(p + ".ffn_down_shexp.weight", H, Fs, m.sh_down));
  return IQ_OK;
}

int load_attention(const Loader& L, const iq_config& c, const std::string& p, AttnWeights& a) {
  const int64_t H = c.hidden_size, hd = c.head_dim;
  TRY(L.matrix(p + ".attn_q.weight", (int64_t)c.num_attention_heads * hd * 2, H, a.q));
  TRY(L.matrix(p + ".attn_k.weight", (int64_t)c.num_key_value_heads * hd, H, a.k));
  TRY(L.matrix(p + ".attn_v.weight", (int64_t)c.num_key_value_heads * hd, H, a.v));
  TRY(L.matrix(p + ".attn_output.weight", H, (int64_t)c.num_attention_heads * hd, a.o));
  TRY(L.vec(p + ".attn_q_norm.weight", hd, a.q_norm));
  TRY(L.vec(p + ".attn_k_norm.weight", hd, a.k_norm));
  return IQ_OK;
}

int load_delta(const Loader& L, const iq_config& c, const std::string& p, DeltaWeights& d) {
  const int64_t H = c.hidden_size;
  const int64_t key_dim = (int64_t)c.linear_num_key_heads * c.linear_key_head_dim;
  const int64_t value_dim = (int64_t)c.linear_num_value_heads * c.linear_value_head_dim;
  const int64_t conv_dim = key_dim * 2 + value_dim;
  const int64_t nv = c.linear_num_value_heads;
  TRY(L.matrix(p + ".attn_qkv.weight", conv_dim, H, d.qkv));
  TRY(L.matrix(p + ".attn_gate.weight", value_dim, H, d.z));
  if (L.find(p + ".ssm_ba.weight")) {
    d.ba_fused = true;
    TRY(L.matrix(p + ".ssm_ba.weight", nv * 2, H, d.ba));
  } else {
    TRY(L.matrix(p + ".ssm_beta.weight", nv, H, d.beta));
    TRY(L.matrix(p + ".ssm_alpha.weight", nv, H, d.alpha));
  }
  TRY(L.matrix(p + ".ssm_out.weight", H, value_dim, d.out));
  TRY(L.vec(p + ".ssm_conv1d.weight", conv_dim * c.linear_conv_kernel_dim, d.conv_w));
  TRY(L.vec(p + ".ssm_a", nv, d.ssm_a));
  TRY(L.vec(p + ".ssm_dt.bias", nv, d.dt_bias));
  TRY(L.vec(p + ".ssm_norm.weight", c.linear_value_head_dim, d.norm));
  return IQ_OK;
}

int validate_config(const iq_config& c) {
  IQ_CHECK(c.hidden_size > 0 && c.num_hidden_layers > 0 && c.vocab_size > 0, IQ_EINVAL, "invalid config sizes");
  IQ_CHECK(c.hidden_size % 256 == 0, IQ_EUNSUPPORTED, "hidden_size must be a multiple of 256");
  IQ_CHECK(c.head_dim % 32 == 0 && c.head_dim <= 256 && c.head_dim >= 64, IQ_EUNSUPPORTED,
           "head_dim %d unsupported (64..256, multiple of 32)", c.head_dim);
  IQ_CHECK(c.rotary_dim > 0 && c.rotary_dim <= c.head_dim && c.rotary_dim % 2 == 0, IQ_EINVAL, "invalid rotary_dim");
  IQ_CHECK(c.num_key_value_heads > 0 && c.num_attention_heads % c.num_key_value_heads == 0, IQ_EINVAL,
           "attention heads must be a multiple of KV heads");
  IQ_CHECK(c.linear_num_key_heads > 0 && c.linear_num_value_heads % c.linear_num_key_heads == 0, IQ_EINVAL,
           "linear value heads must be a multiple of key heads");
  IQ_CHECK(c.linear_key_head_dim % 8 == 0 && c.linear_key_head_dim <= 128, IQ_EUNSUPPORTED,
           "linear_key_head_dim must be a multiple of 8 and <= 128");
  IQ_CHECK(c.linear_value_head_dim % 32 == 0, IQ_EUNSUPPORTED, "linear_value_head_dim must be a multiple of 32");
  IQ_CHECK(c.linear_conv_kernel_dim >= 1 && c.linear_conv_kernel_dim <= 4, IQ_EUNSUPPORTED,
           "linear_conv_kernel_dim must be 1..4");
  IQ_CHECK(c.num_experts_per_tok > 0 && c.num_experts_per_tok <= 16 && c.num_experts_per_tok <= c.num_experts &&
               c.num_experts <= 1024,
           IQ_EINVAL, "invalid top-k %d for %d experts", c.num_experts_per_tok, c.num_experts);
  IQ_CHECK(c.full_attention_interval > 0, IQ_EINVAL, "full_attention_interval must be positive");
  IQ_CHECK(c.mtp_num_hidden_layers == 0 || c.mtp_num_hidden_layers == 1, IQ_EUNSUPPORTED,
           "Qwen MTP requires exactly one configured predictor layer");
  return IQ_OK;
}

int create(const iq_tensor_view* tensors, int n, const iq_config* cfg, int rank, int world, const void* nccl_id,
           iq_model** out) {
  clear_error();
  IQ_CHECK(tensors && cfg && out && n > 0, IQ_EINVAL, "iq_model_create: null argument");
  IQ_CHECK(world >= 1 && rank >= 0 && rank < world, IQ_EINVAL, "invalid rank %d of %d", rank, world);
  TRY(validate_config(*cfg));
  Loader L;
  for (int i = 0; i < n; i++) {
    IQ_CHECK(tensors[i].name && tensors[i].data, IQ_EINVAL, "tensor view %d has no name or data", i);
    L.by_name[tensors[i].name] = &tensors[i];
  }
  std::unique_ptr<iq_model> m(new iq_model);
  m->cfg = *cfg;
  m->ep_rank = rank;
  m->ep_world = world;
  IQ_CUDA(cudaGetDevice(&m->device));
  if (world > 1) {
    IQ_CHECK(nccl_id, IQ_EINVAL, "expert parallelism over %d ranks needs an NCCL unique id", world);
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof id);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = ncclCommInitRank(&comm, world, id, rank);
    IQ_CHECK(r == ncclSuccess, IQ_ECUDA, "ncclCommInitRank (rank %d of %d): %s", rank, world,
             ncclGetErrorString(r));
    m->nccl_comm = comm;
  }
  const iq_config& c = *cfg;
  const int64_t H = c.hidden_size;
  TRY(L.matrix("token_embd.weight", c.vocab_size, H, m->embed));
  TRY(L.vec("output_norm.weight", H, m->out_norm));
  TRY(L.matrix("output.weight", c.vocab_size, H, m->lm_head));
  m->layers.resize(c.num_hidden_layers);
  for (int l = 0; l < c.num_hidden_layers; l++) {
    Layer& ly = m->layers[l];
    const std::string p = "blk." + std::to_string(l);
    ly.type = ((l + 1) % c.full_attention_interval == 0) ? kFull : kLinear;
    TRY(L.vec(p + ".attn_norm.weight", H, ly.attn_norm));
    TRY(L.vec(p + ".post_attention_norm.weight", H, ly.post_norm));
    if (ly.type == kFull) {
      TRY(load_attention(L, c, p, ly.at));
      m->n_full++;
    } else {
      TRY(load_delta(L, c, p, ly.dn));
      m->n_linear++;
    }
    TRY(load_moe(L, c, p, rank, world, ly.moe));
  }
  if (c.mtp_num_hidden_layers == 1) {
    const std::string p = "blk." + std::to_string(c.num_hidden_layers);
    m->has_mtp = true;
    TRY(L.vec(p + ".nextn.enorm.weight", H, m->mtp_enorm));
    TRY(L.vec(p + ".nextn.hnorm.weight", H, m->mtp_hnorm));
    TRY(L.vec(p + ".nextn.shared_head_norm.weight", H, m->mtp_head_norm));
    TRY(L.matrix(p + ".nextn.eh_proj.weight", H, 2 * H, m->mtp_eh_proj));
    Layer& ly = m->mtp_layer;
    ly.type = kFull;
    TRY(L.vec(p + ".attn_norm.weight", H, ly.attn_norm));
    TRY(L.vec(p + ".post_attention_norm.weight", H, ly.post_norm));
    TRY(load_attention(L, c, p, ly.at));
    TRY(load_moe(L, c, p, rank, world, ly.moe));
  }
  IQ_CUDA(cudaDeviceSynchronize());
  *out = m.release();
  return IQ_OK;
}

int64_t wbytes(const Weight& w) { return w.present() ? w.rows * w.row_bytes : 0; }
int64_t vbytes(const Vec& v) { return v.n * 4; }
int64_t layer_bytes(const Layer& l) {
  int64_t b = vbytes(l.attn_norm) + vbytes(l.post_norm);
  b += wbytes(l.dn.qkv) + wbytes(l.dn.z) + wbytes(l.dn.ba) + wbytes(l.dn.beta) + wbytes(l.dn.alpha) + wbytes(l.dn.out);
  b += vbytes(l.dn.conv_w) + vbytes(l.dn.ssm_a) + vbytes(l.dn.dt_bias) + vbytes(l.dn.norm);
  b += wbytes(l.at.q) + wbytes(l.at.k) + wbytes(l.at.v) + wbytes(l.at.o) + vbytes(l.at.q_norm) + vbytes(l.at.k_norm);
  const MoeWeights& m = l.moe;
  b += wbytes(m.router) + vbytes(m.router_sel) + vbytes(m.selector) + wbytes(m.gate) + wbytes(m.up) + wbytes(m.down);
  b += wbytes(m.sh_gate) + wbytes(m.sh_up) + wbytes(m.sh_down);
  return b;
}

}  // namespace
}  // namespace iq

using namespace iq;

extern "C" {

int iq_model_create(const iq_tensor_view* tensors, int n, const iq_config* cfg, iq_model** out) {
  return create(tensors, n, cfg, 0, 1, nullptr, out);
}

int iq_model_create_ep(const iq_tensor_view* tensors, int n, const iq_config* cfg, int rank, int world,
                       const void* nccl_unique_id, iq_model** out) {
  return create(tensors, n, cfg, rank, world, nccl_unique_id, out);
}

int iq_ep_expert_range(int64_t num_experts, int rank, int world, int32_t* lo, int32_t* hi) {
  clear_error();
  IQ_CHECK(lo && hi, IQ_EINVAL, "iq_ep_expert_range: null argument");
  IQ_CHECK(world >= 1 && rank >= 0 && rank < world, IQ_EINVAL, "invalid rank %d of %d", rank, world);
  IQ_CHECK(num_experts > 0 && num_experts <= INT32_MAX && num_experts % world == 0, IQ_EINVAL,
           "%lld experts do not divide over %d ranks", (long long)num_experts, world);
  const int64_t per = num_experts / world;
  *lo = (int32_t)(per * rank);
  *hi = (int32_t)(per * (rank + 1));
  return IQ_OK;
}

int iq_nccl_unique_id(void* out) {
  clear_error();
  IQ_CHECK(out, IQ_EINVAL, "iq_nccl_unique_id: null argument");
  ncclUniqueId id;
  const ncclResult_t r = ncclGetUniqueId(&id);
  IQ_CHECK(r == ncclSuccess, IQ_ECUDA, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  memcpy(out, &id, sizeof id);
  return IQ_OK;
}

void iq_model_destroy(iq_model* m) {
  if (m && m->nccl_comm) ncclCommDestroy(static_cast<ncclComm_t>(m->nccl_comm));
  delete m;
}

int iq_model_weight_bytes(const iq_model* m, int64_t* bytes) {
  IQ_CHECK(m && bytes, IQ_EINVAL, "iq_model_weight_bytes: null argument");
  int64_t b = wbytes(m->embed) + vbytes(m->out_norm) + wbytes(m->lm_head);
  for (const Layer& l : m->layers) b += layer_bytes(l);
  if (m->has_mtp)
    b += layer_bytes(m->mtp_layer) + wbytes(m->mtp_eh_proj) + vbytes(m->mtp_enorm) + vbytes(m->mtp_hnorm) +
         vbytes(m->mtp_head_norm);
  *bytes = b;
  return IQ_OK;
}

}  // extern "C"
