/*
 * iq.h -- C ABI of libiq, the B200 (sm_100a) speculative-verify path of
 * inferq.  Every entry point returns 0 on success or a negative IQ_E* code;
 * iq_last_error() then describes the failure (thread-local, mirroring the
 * reference's anyhow messages).  No entry point aborts the process.
 *
 * Plain C types only: pointers, sizes, and opaque handles.  Weight bytes are
 * GGUF blocks exactly as they sit in the file; the library owns every device
 * allocation behind a handle and frees it in the matching *_destroy.
 */
#ifndef IQ_H
#define IQ_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes. */
#define IQ_OK 0
#define IQ_EINVAL (-1)     /* bad argument or shape */
#define IQ_ECUDA (-2)      /* CUDA runtime error */
#define IQ_ENOMEM (-3)     /* device allocation failed */
#define IQ_EUNSUPPORTED (-4)
#define IQ_ESTATE (-5)     /* call order / state violation */
#define IQ_ETIMEDOUT (-6)  /* a bounded device wait gave up */

/* GGML dtype ids accepted by the library. */
#define IQ_F32 0
#define IQ_F16 1
#define IQ_Q8_0 8
#define IQ_Q4_K 12
#define IQ_Q5_K 13
#define IQ_Q6_K 14
#define IQ_BF16 30

/* Where a caller-supplied buffer lives. */
#define IQ_HOST 0
#define IQ_DEVICE 1

/* Message of the last failure on this thread ("" when none). */
const char* iq_last_error(void);

/* Library version string. */
const char* iq_version(void);

/* ------------------------------------------------------------------ */
/* Operator level: one quantized matrix (replaces QuantizedMatrix,     */
/* src/gguf.rs:159-785).                                               */
/* ------------------------------------------------------------------ */
typedef struct iq_matrix iq_matrix;

/* Upload `rows` GGUF rows of `cols` weights (bytes at `data`, in host or
 * device memory per `location`) to the current device in the device layout.
 * Replaces GgufCheckpoint::load_matrix -> QuantizedMatrix::new
 * (src/gguf.rs:1234-1253, :305-330): the same dtype set, Q4_K, Q5_K, Q6_K,
 * Q8_0, F32 and BF16 (cols a multiple of 8).  A BF16 matrix multiplies its
 * input rows rounded to bf16 (candle's BF16 vec-dot input type) with exact
 * products summed in f32; the model loader takes BF16 only for 1-D
 * tensors, and the wide form takes quantized matrices only. */
int iq_matrix_create(int dtype, const void* data, int64_t rows, int64_t cols, int location,
                     iq_matrix** out);
/* A matrix of the first `rows` rows sharing storage with `m`
 * (QuantizedMatrix::leading_rows, src/gguf.rs:352-377). */
int iq_matrix_leading_rows(const iq_matrix* m, int64_t rows, iq_matrix** out);
void iq_matrix_destroy(iq_matrix* m);
int iq_matrix_shape(const iq_matrix* m, int64_t* rows, int64_t* cols, int* dtype);

/* y[i*rows + r] = row r of m . x[i]   for i < input_rows, host buffers.
 * Replaces QuantizedMatrix::forward_rows (src/gguf.rs:433-456): same
 * argument meaning (row-major f32 in, row-major f32 out), same arithmetic
 * (activations quantized to Q8_K / Q8_0 as candle does, exact integer
 * block dots).  Any input_rows >= 1. */
int iq_matrix_forward_rows(const iq_matrix* m, const float* x, int64_t input_rows, float* y);

/* As iq_matrix_forward_rows with device buffers, enqueued on `stream`
 * (a cudaStream_t, or NULL for the legacy stream).  Input rows <= 8. */
int iq_matrix_forward_device(const iq_matrix* m, const float* x, int input_rows, float* y, void* stream);

/* As iq_matrix_forward_device, but allocating no device memory at all: the
 * quantized input rows and the launch record go to a fixed 37.6 KB scratch
 * array built into the library (one per GPU, held until the process exits).
 * No counterpart in the reference.  For callers that may not allocate while
 * they run -- a host whose device memory is carved up in advance by its own
 * pool, or a decode thread that cannot take cudaMalloc's implicit device
 * synchronization.  Limits: 1..8 input rows, at most 4096 columns; larger
 * requests fail with IQ_EINVAL.  The first call on a device looks up the
 * array's device address, so make that first call before any stream
 * capture.  All calls on a device share the one array: calls whose work
 * overlaps on the GPU (different streams, or threads) race and must be
 * serialized by the caller. */
int iq_matrix_forward_device_noalloc(const iq_matrix* m, const float* x, int input_rows, float* y, void* stream);

/* Wide form for many input rows at once, device buffers, enqueued on
 * `stream`.  The reference runs prefill through QuantizedMatrix::forward in
 * 512-row passes (src/runtime.rs:748-771, src/gguf.rs:406-456); this is that
 * call for Q8_0, Q4_K and Q6_K matrices on the tensor cores, and for Q5_K
 * when the environment variable IQ_WIDE_Q5K is set (other dtypes:
 * IQ_EUNSUPPORTED); 1 <= input_rows <= 65535; y[i*rows + r] as above.
 * Arithmetic: input rows quantized as in iq_matrix_forward_device (Q8_0,
 * or Q8_K for the K-quants), exact integer block dots, one f32 FMA per
 * block (and per block min term for Q4_K/Q5_K) in ascending block order -- bitwise the
 * narrow path's result whenever iq_qgemv_ksplit() is 1 for the shape.
 * Scratch (about 2 B per input element and per matrix element) is held per
 * thread between calls. */
int iq_matrix_forward_wide(const iq_matrix* m, const float* x, int input_rows, float* y, void* stream);

/* Synchronize `stream` and report whether any matrix product on this
 * device gave up a bounded device wait since the last check (IQ_ETIMEDOUT;
 * the results of that call are invalid), clearing the record.  The record
 * is per device and shared with the model passes' GEMVs, which report their
 * own timeouts from iq_forward / iq_verify.  No counterpart in the
 * reference (its CPU kernels have no device waits). */
int iq_matrix_status(void* stream);

/* One-shot form over GGUF bytes in host memory (uploads, multiplies,
 * frees): int iq_qgemv of the boundary table, mirroring forward_rows. */
int iq_qgemv(int dtype, const void* w, int64_t rows, int64_t cols, const float* x, int k, float* y,
             void* stream);

/* The number of contiguous block chunks a row of this shape is split into
 * (a function of the shape only; documents the f32 accumulation order). */
int iq_qgemv_ksplit(int dtype, int64_t rows, int64_t cols);

/* Decode rows of m to f32 (candle to_float order), device -> host copy.
 * `ids` (host, may be NULL) selects rows, as the embedding lookup does
 * (src/gguf.rs:288-290). */
int iq_matrix_dequantize(const iq_matrix* m, const int32_t* ids, int64_t n, float* out);


/* ------------------------------------------------------------------ */
/* Model level: the verify pass, greedy accept and rollback            */
/* (QuantizedModel / QuantizedModelState, src/qwen/quantized_model.rs). */
/* ------------------------------------------------------------------ */

/* The fields of Qwen3NextConfig (src/config.rs:40-93) the pass reads. */
typedef struct iq_config {
  int32_t hidden_size;
  int32_t num_hidden_layers;
  int32_t vocab_size;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;
  int32_t rotary_dim;               /* head_dim * partial_rotary_factor (config.rs:253-255) */
  int32_t linear_num_key_heads;
  int32_t linear_num_value_heads;
  int32_t linear_key_head_dim;
  int32_t linear_value_head_dim;
  int32_t linear_conv_kernel_dim;
  int32_t num_experts;
  int32_t num_experts_per_tok;
  int32_t moe_intermediate_size;
  int32_t shared_expert_intermediate_size;
  int32_t full_attention_interval;  /* layer l is full attention iff (l+1) % interval == 0 */
  int32_t mtp_num_hidden_layers;    /* 0 or 1 */
  int32_t norm_topk_prob;
  int32_t value_heads_tiled;        /* 1 for model_type qwen3_5_moe_text (TiledByRepeat) */
  int32_t max_position_embeddings;
  float rms_norm_eps;
  double rope_theta;
} iq_config;

/* One GGUF tensor: its GGUF name (e.g. "blk.3.attn_qkv.weight"), dtype,
 * row-major shape (outermost first, as candle reports it) and bytes. */
typedef struct iq_tensor_view {
  const char* name;
  int32_t dtype;
  int32_t ndim;
  int64_t shape[4];
  const void* data;
  int32_t location; /* IQ_HOST or IQ_DEVICE */
} iq_tensor_view;

typedef struct iq_model iq_model;
typedef struct iq_state iq_state;

/* Upload every tensor the pass needs to the current device (all experts
 * resident in HBM).  Replaces QuantizedModel::load (quantized_model.rs:511-564)
 * with the expert cache of src/residency.rs made fully resident.  Tensor
 * names and shape checks follow the reference's loaders; a missing or
 * misshapen tensor fails with its name in iq_last_error(). */
int iq_model_create(const iq_tensor_view* tensors, int n, const iq_config* cfg, iq_model** out);
/* Expert-parallel variant (no reference counterpart: the reference runs on
 * one CPU): this rank keeps experts [rank*E/world, (rank+1)*E/world) on the
 * current device; dense, DeltaNet, attention, LM head and MTP weights are
 * replicated.  All `world` ranks (one process per GPU) call it together
 * with the same 128-byte NCCL unique id (from iq_nccl_unique_id on one rank,
 * shared by the host); the library creates and owns the communicator.
 * After every MoE layer the routed expert outputs are summed over the ranks
 * (each slot is nonzero on its owner only), so every rank's results are
 * bitwise those of a single GPU. */
int iq_model_create_ep(const iq_tensor_view* tensors, int n, const iq_config* cfg, int rank, int world,
                       const void* nccl_unique_id, iq_model** out);
/* 128 bytes: an NCCL unique id for iq_model_create_ep. */
int iq_nccl_unique_id(void* out);
/* The experts [*lo, *hi) that iq_model_create_ep keeps on `rank` of
 * `world` (host only; IQ_EINVAL when num_experts does not divide). */
int iq_ep_expert_range(int64_t num_experts, int rank, int world, int32_t* lo, int32_t* hi);
void iq_model_destroy(iq_model* m);
int iq_model_weight_bytes(const iq_model* m, int64_t* bytes);

/* Decode state: per-layer KV cache (f32 [pos][kv_head][head_dim]) and
 * DeltaNet conv/recurrent state, double-buffered for rollback. */
int iq_state_create(iq_model* m, int64_t max_positions, iq_state** out);
void iq_state_destroy(iq_state* s);
int iq_state_reset(iq_state* s);
int iq_state_position(const iq_state* s, int64_t* position);
/* The cudaStream_t every pass of this state is enqueued on. */
int iq_state_stream(const iq_state* s, void** stream);

/* Evaluate `rows` tokens at the state's position and commit all of them
 * (QuantizedModel::forward_detailed, quantized_model.rs:599-621).  Up to 63
 * rows run as passes of at most 8 rows, bitwise the verify path.  From 64
 * rows, when every dense matrix is Q8_0, Q4_K or Q6_K and the experts sit on
 * one GPU, the call takes the wide prefill pass instead (the reference's
 * prefill_in_passes, src/runtime.rs:748-771: 512-row chunks; projections on
 * the tensor cores, the DeltaNet recurrence in its chunked form up to each
 * chunk's final block of up to 8 rows, attention in its sequential kernels,
 * experts grouped by expert): the reference's arithmetic up to f32 rounding
 * order, not bitwise the 8-row passes.  Outputs are host buffers or NULL:
 * logits [rows][vocab], normalized hidden [rows][hidden], argmax [rows]
 * (ties to the last index, sampling.rs:104-112).  The state before the last
 * pass (for the wide pass: before its final block of up to 8 rows) is kept,
 * so iq_rollback may follow. */
int iq_forward(iq_state* s, const uint32_t* tokens, int rows, float* logits, float* hidden, int32_t* argmax);

typedef struct iq_verify_result {
  int32_t accepted;       /* drafts accepted (accepted_draft_prefix, runtime.rs:2225) */
  int32_t authoritative;  /* argmax of row `accepted` */
  int32_t committed;      /* rows kept: accepted + 1 */
} iq_verify_result;

/* One speculative verification pass: tokens = [seed, draft_1..draft_{rows-1}],
 * rows <= 8.  Runs the rows (verify_rows, runtime.rs:2102-2114), takes the
 * greedy argmax of every row on the device, accepts the longest matching
 * draft prefix, rolls the DeltaNet state back to the committed boundary and
 * truncates the KV cache (QuantizedModelState::rollback,
 * quantized_model.rs:177-204) -- all before the single host synchronization.
 * logits [rows][vocab] / hidden [rows][hidden] are optional host outputs. */
int iq_verify(iq_state* s, const uint32_t* tokens, int rows, iq_verify_result* out, float* logits, float* hidden);

/* Roll the last iq_forward pass back to its first `committed_rows` rows
 * (QuantizedModelState::rollback).  committed_rows < rows of that pass; after
 * a wide pass the rows counted are those of its final block of up to 8
 * (rows before it are committed for good). */
int iq_rollback(iq_state* s, int committed_rows);

/* ---------------------------------------------------------------- MTP draft
 * The MTP predictor block (blk.N.nextn.* plus block N's attention and MoE)
 * keeps its own KV cache inside the state; `iq_mtp_position` reports it.
 *
 * Catch-up (replaces synchronize_mtp + shifted_hidden_inputs,
 * src/runtime.rs:2058-2088, :2184-2223): truncate the MTP cache to
 * `position` (<= its current position) and run the block over `rows`
 * committed tokens, token i paired with the target's normalized hidden row
 * of the position before it: `prev_hidden` (H floats) for the first, NULL
 * only at position 0 (zeros), then rows 0..rows-2 of `target_hidden`
 * ([rows][H], host).  No logits.
 */
int iq_mtp_sync(iq_state* s, int64_t position, const float* prev_hidden, const uint32_t* tokens, int rows,
                const float* target_hidden);

/* The MTP input rows iq_mtp_sync builds, on the host only (no device work):
 * out[r] = target_hidden[r-1] for r >= 1, out[0] = prev_hidden (zeros when
 * NULL).  Replaces shifted_hidden_inputs (src/runtime.rs:2184-2223). */
int iq_mtp_shifted_inputs(const float* prev_hidden, const float* target_hidden, int rows, int hidden, float* out);

/* Drafting (replaces draft_mtp, src/runtime.rs:1995-2056, with
 * top1_with_scores :2245-2265 and QuantizedMtpHead::forward_with_head,
 * src/qwen/quantized_mtp.rs:175-227): from `seed` and the target's
 * normalized hidden row (H floats), run `depth` (1..16) MTP steps, each
 * followed by the first `draft_vocab` rows of the LM head (the vocabulary
 * prefix head, leading_rows); step i+1 takes step i's top-1 token and
 * normalized hidden row.  tokens/probs/margins receive all `depth` steps
 * (probs, margins may be NULL); *n is the number of leading drafts whose
 * top-1 probability is >= min_conf (draft_mtp stops before the first that is
 * not).  Stop tokens are the caller's, as in the reference.  The MTP cache
 * advances by `depth`; the next iq_mtp_sync truncates it. */
int iq_mtp_draft(iq_state* s, uint32_t seed, const float* hidden, int depth, int draft_vocab, float min_conf,
                 uint32_t* tokens, float* probs, float* margins, int* n);

int iq_mtp_position(const iq_state* s, int64_t* position);

/* ---------------------------------------------------------------- images
 * A self-contained host copy of a sequence's state, the device form of
 * SessionImage / QuantizedStateImage (src/runtime.rs:566-592,
 * src/qwen/quantized_model.rs:59-100, restore_image :225-252): a 56-byte
 * header (magic "IQSTATE1", version, layer count, position, MTP position,
 * shapes), then per decoder layer in order the KV rows [pos][kv_head][head_dim]
 * (keys, then values) of a full-attention layer or the conv [channel][K-1]
 * and recurrent [head][key][value] state of a DeltaNet layer, then the MTP
 * block's KV rows; all f32.  Import checks the header against the loaded
 * model and the exact byte count, and replaces the state (rollback of the
 * last pass is no longer available). */
int iq_state_image_size(const iq_state* s, int64_t* bytes);
int iq_state_export(iq_state* s, void* out, int64_t bytes);
int iq_state_import(iq_state* s, const void* in, int64_t bytes);

/* Distinct experts each MoE layer ran in the last pass (one int per layer);
 * the measured expert union that sets the pass's algorithmic bytes. */
int iq_state_union_sizes(const iq_state* s, int32_t* per_layer);

/* Routed experts of the last pass: [layer][row][top_k], `rows` = that
 * pass's rows (the routes of QuantizedMoeOutput, quantized_moe.rs:227-281). */
int iq_state_routes(const iq_state* s, int rows, int32_t* experts);

/* Stage timers (the reference threads wall-clock stage timers through every
 * layer, QuantizedForwardTimings, quantized_model.rs:305-401).  With
 * profiling on, passes run without graphs or programmatic overlap and every
 * stage is bracketed by CUDA events.  iq_state_profile writes
 * "stage count total_us" lines into buf and returns their length. */
int iq_state_set_profiling(iq_state* s, int on);
/* Kernels this state has launched so far (graph replays included). */
int iq_state_launch_count(const iq_state* s, int64_t* count);
int iq_state_profile(const iq_state* s, char* buf, int len);

#ifdef __cplusplus
}
#endif
#endif
