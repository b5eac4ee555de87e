// qmv.cuh -- skinny quantized matrix x multi-row product (k <= 8 input rows).
//
// Replaces the reference's fused multi-row kernels (src/qgemm.rs:175-397,
// dispatched by QuantizedMatrix::forward / forward_rows, src/gguf.rs:406-456).
//
// One launch runs a table of jobs.  A job is one weight matrix (or a row
// range of one) against up to eight quantized input rows.  A CTA of eight
// warps owns (8 / ksplit) tiles of 16 weight rows; the ksplit warps of a tile
// each take a contiguous chunk of the row's blocks.  Integer sub-block dot
// products run on the tensor cores (int8 mma.sync, exact int32); each warp
// then folds one f32 FMA per block into its chunk partial, and the chunk
// partials are added left to right.  ksplit depends only on the matrix
// shape, so an output row never depends on how many input rows ran with it.
#pragma once
#include <cstdlib>
#include "iq_common.cuh"

namespace iq {

enum QmvActMode : int {
  kActQuantized = 0,  // act rows are quantized activation rows (Q8_K / Q8_0 layout)
  kActSwiGLU = 1,     // act rows are f32 gate|up projections: stage quant(silu(g) * u)
};

enum QmvEpilogue : int {
  kEpiStore = 0,     // out = y
  kEpiResidual = 1,  // out = resid + y   (resid may alias out)
};

struct QmvJob {
  const uint8_t* w;      // device-layout row 0
  const uint8_t* act;    // quantized activation rows (Q8_K or Q8_0 layout)
  float* out;
  const float* resid;
  const void* tmap;      // device CUtensorMap over the weight tensor: box = one unit x 16 rows
  const void* tmap_tail; // Q6_K / Q8_0: box = 16 bytes x 16 rows over the scale tails
  int64_t w_row_bytes;
  int act_row_bytes;
  int out_ld;
  int dtype, rows, cols, ksplit;
  int n;                 // input rows used, 1..8
  int act_nrows;         // rows of `act` staged into shared memory (> every rowmap entry)
  int tile0;             // first global tile of this job
  int epi;
  int row_base;          // row of the tensor map where this job's row 0 lies
  int act_mode;          // kActQuantized, or kActSwiGLU: `act` holds f32 rows
                         // [gate cols | up cols] (act_row_bytes apart, selected by
                         // rowmap) staged as the quantized silu(gate) * up
  uint8_t rowmap[8];     // activation row of input column i
  int16_t outrow[8];     // output row (of out) of input column i
};

// Two persistent CTAs per SM; each of their warps streams 16 weight rows.
constexpr int kQmvWarps = 8;
constexpr int kQmvThreads = 32 * kQmvWarps;
constexpr int kQmvMaxDepth = 8;  // weight units in flight per warp (at most)
// Rows one CTA covers for a job.
__host__ __device__ inline int qmv_rows_per_cta(int ksplit) { return 16 * (kQmvWarps / ksplit); }
__host__ __device__ inline int qmv_units(int dt, int cols) {
  return dt == Q8_0 ? cols / 128 : cols / 256;
}

// The chunk count of a matrix: a function of its shape only (never of the
// number of input rows), so a row's f32 accumulation order is fixed.
// Expert matrices (`expert`: one of many small matrices in the same launch)
// split less, so each warp streams several blocks.
inline int qmv_ksplit(int dt, int64_t rows, int64_t cols, bool expert = false) {
  int units = qmv_units(dt, (int)cols);
  const int64_t target = expert ? 32 : 148 * 32;
  int ks = 1;
  while (ks < 8 && units % (ks * 2) == 0 && (rows / 16) * ks < target) ks *= 2;
  return ks;
}
inline int qmv_tiles(const QmvJob& j) {
  return (int)ceil_div(j.rows, qmv_rows_per_cta(j.ksplit));
}

// The activation rows a projection needs, as produced by the row-prep or
// gated-norm kernel that precedes it (host-side description).
enum QmvProMode : int {
  kProNone = 0,
  kProRmsNorm = 1,  // x / sqrt(mean(x^2) + eps) * w         (GGUF RMSNorm)
  kProGated = 2,    // per head: x / sqrt(mean(x^2) + eps) * w * silu(z)
  kProQuant = 3,    // x as is
};

struct QmvPrologue {
  int mode;
  int rows;          // activation rows produced (<= 8)
  int cols;          // elements per row (a multiple of 256)
  const float* x;    // [rows][ldx] (Gated: the recurrent output o)
  int ldx;
  const float* w;    // RmsNorm: [cols]; Gated: [dv]
  const float* z;    // Gated: [rows][ldz]
  int ldz;
  int heads, dv;     // Gated
  float eps, inv_n;  // inv_n = 1/cols (RmsNorm) or 1/dv (Gated)
  int want8k, want80;  // layouts to produce
  int stride8k, stride80;  // row strides of the two layouts (bytes)
  float* xn_out;     // RmsNorm: the normalized f32 rows are also written here (or null)
  int ldxn;
};

// Launch `ntiles` CTAs over `jobs` (device memory, sorted by tile0).
// When `dyn_count` is non-null the job count is read on the device after the
// programmatic-dependency wait (jobs written by the previous kernel), and
// CTAs past the last job's tiles exit.
// `smem_bytes` must cover n * act_row_bytes of every job in the table; the
// rest of the CTA's shared memory holds the weight ring (2..4 units per warp).
// `slot_bytes` (0: the largest of any dtype) sizes each ring slot for the
// largest unit the launch streams (qmv_slot_bytes of its dtypes), so launches
// of smaller units keep more of them in flight.
cudaError_t qmv_launch(const QmvJob* jobs, int njobs, const int* dyn_count, int ntiles, int smem_bytes,
                       cudaStream_t stream, bool pdl, int slot_bytes = 0);
// Ring slot bytes of one unit of dtype `dt` (16 rows, plus the scale-tail
// piece of Q6_K / Q8_0), a multiple of 128.
inline int qmv_slot_bytes(int dt) {
  return dt == Q4_K ? 16 * 144 : dt == Q5_K ? 16 * 176 : dt == Q6_K ? 16 * 208 + 256 : 16 * 128 + 256;
}

// Encode the tensor maps the kernel loads a weight tensor through (device
// layout, `rows` x `cols`) into `maps`: [0] the unit box, [1] the tail box
// (Q6_K / Q8_0).  Jobs point at them (tmap = maps, tmap_tail = maps + 128 B).
// Device address of the flag a GEMV sets when a bounded wait for its weight
// slots gave up (0 = never); the caller clears it.
int* qmv_timeout_flag();

struct DevBuf;
cudaError_t qmv_tensor_maps(int dt, const uint8_t* base, int64_t rows, int64_t cols, DevBuf& maps);

}  // namespace iq
