// model.h -- host-side structures of a loaded model and its decode state.
#pragma once
#include <memory>
#include <string>
#include <vector>
#include "api_util.h"
#include "model_kernels.cuh"

namespace iq {

int validate_matrix_shape(int dtype, int64_t rows, int64_t cols);
int upload_rows(int dtype, const void* data, int64_t rows, int64_t cols, int location, DevBuf& out,
                cudaStream_t st);

// A weight matrix resident in the device layout.
struct Weight {
  int dt = -1;
  int64_t rows = 0, cols = 0, row_bytes = 0;
  DevBuf buf;
  DevBuf maps;  // TMA tensor maps over buf (quantized weights): unit box, tail box
  uint8_t* p() const { return buf.as<uint8_t>(); }
  const void* tmap() const { return maps.p; }
  const void* tmap_tail() const { return maps.p ? static_cast<const uint8_t*>(maps.p) + 128 : nullptr; }
  bool present() const { return dt >= 0; }
};

struct Vec {  // f32 vector / small dense tensor on the device
  DevBuf buf;
  int64_t n = 0;
  float* p() const { return buf.as<float>(); }
};

struct DeltaWeights {
  Weight qkv, z, ba, beta, alpha, out;
  bool ba_fused = false;  // Qwen3-Next ssm_ba (interleaved per key head)
  Vec conv_w, ssm_a, dt_bias, norm;
};

struct AttnWeights {
  Weight q, k, v, o;
  Vec q_norm, k_norm;
};

struct MoeWeights {
  Weight router;       // [E, H] (F32 or quantized)
  Vec router_sel;      // F32 routers: [E+1, H] with the shared selector as row E
  Vec selector;        // [H]
  Weight gate, up, down;  // resident experts stacked: rows = n_res * ffn (down: n_res * H)
  Weight sh_gate, sh_up, sh_down;
  int expert_lo = 0, expert_hi = 0;
};

enum LayerType { kLinear = 0, kFull = 1 };

struct Layer {
  int type = kLinear;
  Vec attn_norm, post_norm;
  DeltaWeights dn;
  AttnWeights at;
  MoeWeights moe;
};

}  // namespace iq

struct iq_model {
  iq_config cfg;
  int device = 0;
  int ep_rank = 0, ep_world = 1;
  std::vector<iq::Layer> layers;
  iq::Weight embed;
  iq::Vec out_norm;
  iq::Weight lm_head;
  bool has_mtp = false;
  iq::Vec mtp_enorm, mtp_hnorm, mtp_head_norm;
  iq::Weight mtp_eh_proj;
  iq::Layer mtp_layer;
  int n_linear = 0, n_full = 0;
  void* nccl_comm = nullptr;  // expert-parallel exchange (ncclComm_t, owned), or null
};
