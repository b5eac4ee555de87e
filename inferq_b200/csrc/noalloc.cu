// noalloc.cu -- a GEMV entry point that allocates no device memory.
//
// iq_matrix_forward_device quantizes its input rows into a scratch buffer and
// uploads a one-job table, and both of those live in device memory it obtains
// with cudaMalloc on first use.  iq_matrix_forward_device_noalloc does the
// same work with that scratch placed in a fixed array compiled into the
// library instead, for callers that must not allocate while they run.
#include <cstring>
#include <mutex>
#include "matrix.h"
#include "kernels.cuh"

namespace iq {
namespace {

// Largest problem the fixed scratch holds: 8 input rows of up to 4096
// columns (a quantized activation row is 4416 bytes in the Q8_K layout and
// 4608 bytes in the Q8_0 layout at 4096 columns; the checks below tie the
// size to the layout functions).
constexpr int kNoAllocMaxRows = 8;
constexpr int kNoAllocMaxCols = 4096;
constexpr int kNoAllocActBytes = 8 * 4672;
static_assert(kNoAllocMaxRows * act_row_bytes_q8k(kNoAllocMaxCols) <= kNoAllocActBytes,
              "the scratch holds the largest Q8_K activation rows");
static_assert(kNoAllocMaxRows * act_row_bytes_q80(kNoAllocMaxCols) <= kNoAllocActBytes,
              "the scratch holds the largest Q8_0 activation rows");
constexpr int kNoAllocJobOffset = kNoAllocActBytes;            // 256-aligned
constexpr int kNoAllocBytes = kNoAllocJobOffset + 256;

// One copy per GPU that loads the library, alive until the process exits.
// Host code must not pass `g_scratch` itself to a kernel: on the host it is a
// stand-in symbol, not a device address.  Its device address is looked up
// once per device below.
static __device__ __align__(256) uint8_t g_scratch[kNoAllocBytes];

std::mutex g_mu;
uint8_t* g_addr[64] = {};

// Device address of g_scratch on the current device (set up on first use).
int scratch_address(uint8_t** out) {
  int dev = 0;
  IQ_CUDA(cudaGetDevice(&dev));
  IQ_CHECK(dev >= 0 && dev < 64, IQ_EUNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    IQ_CUDA(cudaGetSymbolAddress(&p, g_scratch));
    g_addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_addr[dev];
  return IQ_OK;
}

// Writes the launch record into the scratch array from a kernel parameter, so
// no host staging copy is involved.
__global__ void store_job_kernel(QmvJob j, QmvJob* dst) { *dst = j; }

}  // namespace
}  // namespace iq

using namespace iq;

extern "C" int iq_matrix_forward_device_noalloc(const iq_matrix* m, const float* x, int input_rows, float* y,
                                                void* stream) {
  clear_error();
  IQ_CHECK(m && x && y, IQ_EINVAL, "iq_matrix_forward_device_noalloc: null argument");
  IQ_CHECK(input_rows >= 1 && input_rows <= kNoAllocMaxRows, IQ_EINVAL,
           "the no-allocation forward takes 1..%d input rows, got %d", kNoAllocMaxRows, input_rows);
  IQ_CHECK(m->cols <= kNoAllocMaxCols, IQ_EINVAL,
           "the no-allocation forward takes matrices of at most %d columns, this one has %lld", kNoAllocMaxCols,
           (long long)m->cols);
  IQ_CHECK(((uintptr_t)x & 15) == 0, IQ_EINVAL,
           "the no-allocation forward needs 16-byte aligned input rows (it cannot stage a copy)");
  IQ_CHECK(m->dtype != BF16, IQ_EUNSUPPORTED, "the no-allocation forward takes quantized or F32 matrices");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m->dtype == F32) {
    IQ_CUDA(f32_matvec(reinterpret_cast<const float*>(m->base), (int)m->rows, (int)m->cols, x, (int)m->cols,
                       input_rows, y, (int)m->rows, st, false));
    return IQ_OK;
  }
  uint8_t* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  const bool kq = m->dtype != Q8_0;
  const int64_t arb = kq ? act_row_bytes_q8k(m->cols) : act_row_bytes_q80(m->cols);
  PrepArgs pa = {};
  pa.x = x;
  pa.ldx = (int)m->cols;
  pa.cols = (int)m->cols;
  pa.inv_cols = 1.f / (float)m->cols;
  if (kq) pa.q8k = scratch;
  else pa.q80 = scratch;
  IQ_CUDA(prep_rows(pa, input_rows, st, false));
  QmvJob j;
  memset(&j, 0, sizeof j);  // every byte of the job record is rewritten each call
  j.w = m->base;
  j.tmap = m->tmap();
  j.tmap_tail = m->tmap_tail();
  j.act = scratch;
  j.out = y;
  j.w_row_bytes = m->row_bytes;
  j.act_row_bytes = (int)arb;
  j.out_ld = (int)m->rows;
  j.dtype = m->dtype;
  j.rows = (int)m->rows;
  j.cols = (int)m->cols;
  j.ksplit = qmv_ksplit(m->dtype, m->rows, m->cols);
  j.n = input_rows;
  j.act_nrows = input_rows;
  j.epi = kEpiStore;
  for (int i = 0; i < 8; i++) {
    j.rowmap[i] = (uint8_t)(i < input_rows ? i : 0);
    j.outrow[i] = (int16_t)i;
  }
  QmvJob* dj = reinterpret_cast<QmvJob*>(scratch + kNoAllocJobOffset);
  store_job_kernel<<<1, 1, 0, st>>>(j, dj);
  IQ_CUDA(cudaGetLastError());
  IQ_CUDA(qmv_launch(dj, 1, nullptr, qmv_tiles(j), (int)(arb * input_rows), st, false));
  return IQ_OK;
}
