// model_kernels.cuh -- argument blocks and launchers of the layer kernels.
#pragma once
#include "kernels.cuh"

namespace iq {

// ----------------------------------------------------------------- DeltaNet
// DeltaNet state per layer: the conv state in a ring holding the state
// before a pass and after each of its rows (so it must exceed the rows of a
// pass); the recurrent state as one base buffer plus the update records of
// the last pass's rows (see deltanet.cu).
constexpr int kStateRing = 10;  // cur, the state after a prefix, 8 rows
constexpr int kMaxRowsDelta = 8;

struct DeltaNetLayer {
  float* conv_state[kStateRing];  // [conv_dim][K-1]
  float* rec_state;       // [nv][dk][dv]: the state before the `pending` records
  float* rec_log;         // [nv][kMaxRowsDelta][rec_stride]: k[dk] | delta[dv] | decay per row
  const float* conv_w;    // [conv_dim][K]
  const float* ssm_a;     // [nv]  (already -exp(A_log))
  const float* dt_bias;   // [nv]
};

struct DeltaNetArgs {
  const DeltaNetLayer* layers;  // device pointer to this layer's entry
  const float* qkv;             // projections [rows][qkv_ld] (first conv_dim cols)
  int qkv_ld;
  const float* ba;              // beta/alpha projections [rows][ba_ld]
  int ba_ld;
  float* out;                   // recurrent outputs [rows][out_ld]
  int out_ld;
  int rows;
  int nk, nv, dk, dv, conv_k;
  int tiled_heads;              // value head layout: 1 TiledByRepeat, 0 GroupedByKeyHead
  int ba_interleaved;           // 1: ssm_ba per key head, 0: beta rows then alpha rows
  int rec_stride;               // deltanet_rec_stride(dk, dv)
  const int* cur;               // device: conv ring index of the current state
  const int* pending;           // device: records of the last pass still to replay
  // Optional fused gated RMSNorm + Q8_0 quantization of the output rows (for
  // a Q8_0 output projection): q80 = quant(norm(o) * w * silu(z)); `out` is
  // then not written.
  uint8_t* q80;                 // [rows][q80_stride] Q8_0 activation rows, or null
  int q80_stride;
  const float* z;  int z_ld;    // gate projections [rows][z_ld]
  const float* norm_w;          // [dv]
  float eps, inv_dv;
  int* timeout_flag;            // device flag set when a bounded wait gave up
  // Or: the gated norm's f32 rows (not quantized) [rows][g_ld]; needs z,
  // norm_w, eps, inv_dv as above.
  float* g_out;  int g_ld;
};
int deltanet_rec_stride(int dk, int dv);
bool deltanet_supported(int dk, int dv);
cudaError_t deltanet_launch(const DeltaNetArgs& a, cudaStream_t st, bool pdl);

// The chunked recurrence over the rows of a wide pass before its final block
// (deltanet_chunk.cu): advances the layer's base state over `rows` rows
// (after replaying `pending` records), writes the conv history after them to
// conv slot cur + 1, and the gated-norm output rows to g_out.
struct DeltaChunkArgs {
  const DeltaNetLayer* layers;
  const float* qkv;  int qkv_ld;
  const float* ba;   int ba_ld;
  int rows;
  int nk, nv, dk, dv, conv_k;
  int tiled_heads, ba_interleaved, rec_stride;
  const int* cur;
  const int* pending;
  float* cv;                    // scratch [rows][conv_dim]: normalized q, k, then v
  float* bl;                    // scratch [rows][2 nv]: beta, then log-decay
  float* o;  int o_ld;          // scratch: recurrent outputs [rows][o_ld]
  // scratch per (value head, 32-row chunk): wy_x [kChunk][dv + dk] (U | W),
  // wy_m [kChunk][kChunk], wy_ew [2][kChunk] (e_t, then w_s)
  float* wy_x;
  float* wy_m;
  float* wy_ew;
  const float* z;  int z_ld;
  const float* norm_w;
  float eps, inv_dv;
  float* g_out;  int g_ld;
};
bool deltanet_chunk_supported(int nk, int nv, int dk, int dv, int conv_k);
cudaError_t deltanet_chunk_launch(const DeltaChunkArgs& a, cudaStream_t st);

struct GatedNormArgs {
  const float* o;  int o_ld;
  const float* z;  int z_ld;
  const float* w;  // [dv]
  int heads, dv;
  float eps, inv_dv;
  uint8_t* q8k;
  uint8_t* q80;
  int q8k_stride, q80_stride;  // activation row strides in bytes
};
cudaError_t gated_norm_launch(const GatedNormArgs& a, int rows, cudaStream_t st, bool pdl);

// ---------------------------------------------------------------- attention
struct AttnArgs {
  const float* qg;  int qg_ld;   // [rows][nh][2*hd] (q then gate per head)
  const float* kp;  int kp_ld;   // [rows][nkv*hd]
  const float* vp;  int vp_ld;
  const float* q_norm;           // [hd]
  const float* k_norm;           // [hd]
  float* kcache;                 // [max_pos][nkv][hd]
  float* vcache;
  float* qbuf;                   // [rows][nh][hd]  normalized + roped queries
  float* part;                   // split-K partials
  float* out;  int out_ld;       // [rows][nh*hd]
  int rows, nh, nkv, hd, rotary_dim;
  double theta;
  float eps;
  const int* pos;                // device: position of row 0
  int chunk_ctas;                // chunks the grid covers: ceil(max positions / kAttnChunk)
  // Optional: the combine writes the output projection's quantized input
  // rows (Q8_K when hd == 256, Q8_0 when hd % 128 == 0) instead of `out`.
  uint8_t* q8k_out; int q8k_stride;
  uint8_t* q80_out; int q80_stride;
};
// Positions per split of the scan.  Chunk c always covers absolute positions
// [c*kAttnChunk, (c+1)*kAttnChunk), and a row combines its chunks in order, so
// a row's output depends only on its own context, never on the pass it ran in.
constexpr int kAttnChunk = 32;
cudaError_t attn_prep_launch(const AttnArgs& a, cudaStream_t st, bool pdl);
cudaError_t attn_scan_launch(const AttnArgs& a, cudaStream_t st, bool pdl);
// The most rows (a power-of-two fraction of `want`) one scan launch holds
// with this geometry (the query rows share the CTA's shared memory).
int attn_scan_max_rows(const AttnArgs& a, int want);
cudaError_t attn_combine_launch(const AttnArgs& a, cudaStream_t st, bool pdl);

// ---------------------------------------------------------------------- MoE
// Per-layer constants of the routed and shared experts (device layout).
struct MoeRouteStatic {
  const uint8_t* gate; const uint8_t* up; const uint8_t* down;  // expert-stacked, resident experts only
  int64_t gate_stride, up_stride, down_stride;                 // bytes per expert
  int64_t gate_row_bytes, down_row_bytes;
  int gate_dt, down_dt;
  int ks_gate, ks_down, tiles_gate, tiles_down;
  const uint8_t* sh_gate; const uint8_t* sh_up; const uint8_t* sh_down;
  int64_t sh_gate_row_bytes, sh_down_row_bytes;
  int sh_gate_dt, sh_down_dt;
  int ks_sh_gate, ks_sh_down, tiles_sh_gate;
  int with_shared;
  int expert_lo, expert_hi;  // experts resident on this rank: [lo, hi)
  // TMA tensor maps (device) over the stacked tensors; expert e's rows start
  // at row (e - expert_lo) * rows_per_expert of its map
  const void *gate_tm, *up_tm, *down_tm, *gate_tm_tail, *up_tm_tail, *down_tm_tail;
  const void *sh_gate_tm, *sh_up_tm, *sh_down_tm, *sh_gate_tm_tail, *sh_up_tm_tail, *sh_down_tm_tail;
};

struct MoeRouteArgs {
  const float* logits;  int logits_ld;  // [rows][E (+1 shared selector)]
  int rows, experts, topk, norm_topk;
  int hidden, ffn, sh_ffn;
  // outputs
  int* route_expert;     // [rows][topk]
  float* route_weight;   // [rows][topk]
  QmvJob* gu_jobs;       // gate/up job table
  int* gu_count;
  QmvJob* down_jobs;
  int* down_count;
  int* union_size;       // number of distinct experts (stat)
  int* union_list;       // [experts] distinct experts, ascending
  // buffers the jobs point at
  const uint8_t* act_in8k; int act_in8k_bytes;  // normalized hidden rows, Q8_K layout
  const uint8_t* act_in80; int act_in80_bytes;  // the same rows, Q8_0 layout
  float* gu_out;                               // [slot][2*ffn_max]
  int gu_ld;
  const uint8_t* act_mid; int act_mid_bytes;   // silu(g)*u rows per slot, in the down matrix's layout
  float* y;  int y_ld;                         // [slot][hidden]
  int swiglu_down;  // 1: down jobs stage silu(g)*u from gu_out themselves (kActSwiGLU)
};
cudaError_t moe_route_launch(const MoeRouteArgs& a, const MoeRouteStatic& s, cudaStream_t st, bool pdl);
// The F32 router (rows x cols, f32_matvec's arithmetic) and the routing in
// one launch: y [k][ld] must be a.logits; `counter` is a device int that
// starts at 0 (the launch leaves it at 0).
struct RouterRouteArgs {
  const float* w;  int rows, cols;
  const float* x;  int ldx;
  float* y;
  int* counter;
};
cudaError_t router_route_launch(const RouterRouteArgs& r, const MoeRouteArgs& a, const MoeRouteStatic& s,
                                cudaStream_t st, bool pdl);
// Routes only (any number of rows): route_e / route_w [row][topk], the same
// arithmetic as moe_route's per-row routing.
cudaError_t moe_route_rows_launch(const float* logits, int ld, int rows, int E, int topk, int norm_topk,
                                  int* route_e, float* route_w, cudaStream_t st);

struct MoeActArgs {
  const float* gu; int gu_ld;  // [slot][gate ffn | up ffn]
  int ffn, sh_ffn;
  int rows, topk;
  const int* route_expert;     // slots whose expert is not resident are skipped
  int expert_lo, expert_hi;
  uint8_t* act; int act_bytes;  // rows per slot
  int down_q80, sh_down_q80;    // 1: quantize to Q8_0 (Q8_0 down matrix), else Q8_K
};
cudaError_t moe_act_launch(const MoeActArgs& a, cudaStream_t st, bool pdl);

struct MoeCombineArgs {
  const float* y; int y_ld;     // [slot][hidden]: routed slots row*topk+route, shared at rows*topk+row
  const float* route_weight;
  const float* logits; int logits_ld;  // shared selector logit at column `experts`
  int experts;
  float* hidden; int hidden_ld;
  int rows, topk, dim;
};
cudaError_t moe_combine_launch(const MoeCombineArgs& a, cudaStream_t st, bool pdl);

// -------------------------------------------------------- embed / head / accept
cudaError_t embed_launch(int dt, const uint8_t* w, int64_t row_bytes, int cols, const int32_t* tokens, int rows,
                         float* out, int out_ld, cudaStream_t st, bool pdl);

struct HeadArgs {
  const float* logits; int logits_ld;  // [rows][vocab]
  int rows, vocab;
  float* part_val; int* part_idx;      // [rows][nparts]
  int nparts;
  int* argmax;                          // [rows]
  // speculative accept (verify mode)
  const int32_t* tokens;                // [rows]: seed then drafts
  int verify;                           // 1: accept the longest matching draft prefix
  int* result;                          // [0]=accepted [1]=authoritative [2]=committed rows
  // MTP scores of row 0: margin and top-1 probability
  float* scores;                        // [2] or null
};
cudaError_t argmax_launch(const HeadArgs& a, cudaStream_t st, bool pdl);

struct MtpStepArgs {
  int32_t* tokens;        // [0] <- drafted token (next step's input)
  const int* result;      // accept result of the draft row: [1] = argmax
  const float* scores;    // [0] margin, [1] top-1 probability
  int* out_tok; float* out_prob; float* out_margin;  // [depth]
  int i;                  // this step's slot
  const float* xn;        // normalized hidden row of the step
  float* hin;             // next step's hidden input
  int hidden;
};
cudaError_t mtp_step_launch(const MtpStepArgs& a, cudaStream_t st, bool pdl);
// *p = v (add = false) or *p += v, in stream order
cudaError_t set_int_launch(int* p, int v, bool add, cudaStream_t st, bool pdl);
cudaError_t accept_launch(const HeadArgs& a, cudaStream_t st, bool pdl);
// out[t] = argmax of logits row t (ld apart) for `rows` rows, the accept
// kernel's tie rule; one CTA per row.
cudaError_t rows_argmax_launch(const float* logits, int64_t ld, int rows, int vocab, int* out, cudaStream_t st);

// cur = (cur + committed) mod kStateRing; pos += committed;
// pending = committed (the DeltaNet records the next pass replays)
cudaError_t commit_launch(int* cur, int* pos, int* pending, const int* result, cudaStream_t st, bool pdl);

template <class K, class... Args>
inline cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace iq
