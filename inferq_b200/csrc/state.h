// state.h -- the decode state behind iq_state (shared by the k-row pass in
// model_run.cu and the wide prefill pass in wide_pass.cu).
#pragma once
#include <map>
#include <string>
#include <vector>
#include "model.h"

namespace iq {

constexpr int kMaxK = 8;
constexpr int kArgmaxParts = 128;

struct QmvRec {
  int job = 0;    // index of the first job in the state's job table for this k
  int njobs = 0;
  int ntiles = 0;
  int smem = 0;
  int slot = 0;   // ring slot bytes: the largest unit of the launch's dtypes
};

struct LayerRec {
  QmvRec proj, out, router;
};

struct KPlan {
  std::vector<LayerRec> layers;
  QmvRec lm_head;
  LayerRec mtp;    // the MTP block (a full-attention layer + MoE)
  QmvRec mtp_eh;   // eh_proj: [enorm(embed) | hnorm(hidden)] -> hidden
};

constexpr int kMaxDraft = 16;  // MTP draft steps per call

}  // namespace iq

struct iq_state {
  iq_model* m = nullptr;
  int64_t max_pos = 0;
  int64_t position = 0;  // host mirror of d_ctrl[0]
  int last_rows = 0;     // rows of the last iq_forward pass (rollback bound)
  bool can_rollback = false;
  cudaStream_t st = nullptr;
  // control words: [0]=pos [1]=DeltaNet conv ring index [2..4]=result
  // [5]=MTP pos [6]=DeltaNet update records still to replay (pending)
  iq::DevBuf ctrl;
  int* h_result = nullptr;   // pinned [4]
  int32_t* h_tokens = nullptr;  // pinned [8]
  iq::DevBuf tokens;
  // DeltaNet
  std::vector<iq::DevBuf> conv;       // kStateRing per linear layer
  std::vector<iq::DevBuf> rec, rec_log;  // per linear layer: base state, update records
  std::vector<iq::DevBuf> dn_qkv, dn_ba;  // per linear layer pass projections
  iq::DevBuf dn_layers;  // DeltaNetLayer[n_linear]
  // attention
  std::vector<iq::DevBuf> kc, vc;
  // scratch
  iq::DevBuf hidden, xn, act8k, act80, z, dn_out, qg, kp, vp, qbuf, part, attn_out;
  iq::DevBuf logits_moe, route_e, route_w, gu_jobs, down_jobs, counts, union_list, gu_out, act_mid, y;
  iq::DevBuf logits, pval, pidx, argmax, scores;
  // MTP predictor: position of its KV cache (host mirror of ctrl[5]), inputs,
  // per-step outputs and the cached vocabulary-prefix head job
  int64_t mtp_position = 0;
  iq::DevBuf mtp_xcat, mtp_hin, mtp_res, mtp_out, mtp_head_job;
  int mtp_head_vocab = 0;
  // captured MTP launch sequences: draft per (depth, vocabulary), catch-up per rows
  std::map<std::pair<int, int>, cudaGraphExec_t> mtp_draft_graphs;
  std::map<std::pair<int, int>, int> mtp_draft_eager;
  cudaGraphExec_t mtp_sync_graphs[8] = {};
  int mtp_sync_eager[8] = {};
  std::map<cudaGraphExec_t*, int64_t> mtp_graph_launches;
  float* h_mtp = nullptr;  // pinned: staging of hidden rows and outputs
  int64_t act8k_bytes = 0, act80_bytes = 0, act_mid_bytes = 0;
  int gu_ld = 0;
  int max_chunks = 0;
  // job tables for k = 1..8
  iq::DevBuf jobs;
  std::vector<iq::KPlan> plans;  // index k-1
  int* union_dev = nullptr;      // counts + 4*layer + 2
  // stage profiling (iq_state_set_profiling): events and accumulated times
  bool profiling = false;
  int64_t launch_count = 0;  // kernels enqueued by passes (graph replays count theirs too)
  int graph_launches[2][8] = {};
  std::vector<std::pair<std::string, cudaEvent_t>> marks;
  std::vector<std::pair<std::string, std::pair<int, double>>> prof;
  // the wide prefill pass's buffers (allocated on its first use)
  struct Wide {
    iq::DevBuf hidden, xn, big, z, ba, o, y, kp, vp, logits, tokens, ctrl, lg, re, rw, xg, actg, gu, yg, ysh, gush,
        map, jobs, argres, scratch, qbuf, part, cv, bl, dno, wyx, wym, wyew, yslot;
    int attn_rows = 8;  // rows per attention slice of the chunk
    int32_t* h_routes = nullptr;  // pinned [rows][topk]
    std::vector<iq::QmvJob> job_table;
    std::vector<int32_t> map_host;
    ~Wide() {
      if (h_routes) cudaFreeHost(h_routes);
    }
  } wide;
  // one captured graph per (mode, rows): [verify][k-1]
  cudaGraphExec_t graphs[2][8] = {};
  int eager_runs[2][8] = {};
  ~iq_state() {
    for (auto& row : graphs)
      for (auto& g : row)
        if (g) cudaGraphExecDestroy(g);
    for (auto& g : mtp_draft_graphs)
      if (g.second) cudaGraphExecDestroy(g.second);
    for (auto& g : mtp_sync_graphs)
      if (g) cudaGraphExecDestroy(g);
    if (h_result) cudaFreeHost(h_result);
    if (h_tokens) cudaFreeHost(h_tokens);
    if (h_mtp) cudaFreeHost(h_mtp);
    if (st) cudaStreamDestroy(st);
  }
};


namespace iq {
// The wide prefill pass (wide_pass.cu): `rows` tokens at the state's
// position through every layer in chunks of kWideRows; outputs as iq_forward.
constexpr int kWideRows = 512;
constexpr int kWideMin = 64;  // iq_forward takes the wide pass from this many rows
bool wide_capable(const iq_model* m);
int wide_forward(iq_state* s, const uint32_t* tokens, int rows, float* logits, float* hidden, int32_t* argmax);
}  // namespace iq
