// api_matrix.cu -- operator-level C ABI: iq_matrix_* and iq_qgemv.
#include <memory>
#include <vector>
#include <cstring>
#include "api_util.h"
#include "kernels.cuh"
#include "matrix.h"

namespace iq {

static thread_local std::string g_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
}
void clear_error() { g_error.clear(); }

static bool supported_dtype(int dt) {
  return dt == F32 || dt == BF16 || dt == Q8_0 || dt == Q4_K || dt == Q5_K || dt == Q6_K;
}

// Checks shared by every upload: the reference accepts Q4_K, Q5_K, Q6_K, Q8_0,
// F32 (and BF16) matrices (src/gguf.rs:307-321); the device kernels also need
// whole blocks, and for Q8_0 whole groups of four blocks.
int validate_matrix_shape(int dtype, int64_t rows, int64_t cols) {
  IQ_CHECK(supported_dtype(dtype), IQ_EUNSUPPORTED,
           "unsupported executable GGUF matrix dtype %d; expected Q4_K, Q5_K, Q6_K, Q8_0, F32, or BF16", dtype);
  IQ_CHECK(rows > 0 && cols > 0, IQ_EINVAL, "matrix shape [%lld, %lld] is empty", (long long)rows,
           (long long)cols);
  const int64_t unit = dtype == Q8_0 ? 128 : dtype == F32 ? 4 : dtype == BF16 ? 8 : 256;
  IQ_CHECK(cols % unit == 0, IQ_EINVAL, "matrix with %lld columns is not a multiple of %lld for dtype %d",
           (long long)cols, (long long)unit, dtype);
  IQ_CHECK(rows < (1ll << 31), IQ_EINVAL, "matrix has too many rows (%lld)", (long long)rows);
  return IQ_OK;
}

// Upload GGUF rows into a fresh device-layout buffer.
int upload_rows(int dtype, const void* data, int64_t rows, int64_t cols, int location, DevBuf& out,
                cudaStream_t st) {
  const int64_t src_bytes = gguf_row_bytes(dtype, cols) * rows;
  const int64_t dst_bytes = dev_row_bytes(dtype, cols) * rows;
  IQ_CUDA(out.reserve((size_t)dst_bytes));
  if (dtype == F32 || dtype == BF16) {  // used as stored
    IQ_CUDA(cudaMemcpyAsync(out.p, data, (size_t)src_bytes,
                            location == IQ_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, st));
    return IQ_OK;
  }
  const uint8_t* src = static_cast<const uint8_t*>(data);
  DevBuf staging;
  if (location == IQ_HOST) {
    IQ_CUDA(staging.reserve((size_t)src_bytes));
    IQ_CUDA(cudaMemcpyAsync(staging.p, data, (size_t)src_bytes, cudaMemcpyHostToDevice, st));
    src = staging.as<uint8_t>();
  }
  IQ_CUDA(gguf_to_device(dtype, src, out.as<uint8_t>(), rows, (int)cols, st));
  IQ_CUDA(cudaStreamSynchronize(st));
  return IQ_OK;
}

struct Scratch {
  DevBuf x, y, act, jobs, wide_w;
};
// Operator scratch: one set per thread and per device, so a thread that calls
// on several GPUs never hands one GPU's buffer to another's kernel.
Scratch& scratch() {
  static thread_local Scratch per_device[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  return per_device[dev];
}

// y[i*rows + r] for i < k <= 8; x, y device pointers.
int matrix_forward_dev(const iq_matrix* m, const float* x, int k, float* y, cudaStream_t st) {
  if (m->dtype == F32) {
    IQ_CUDA(f32_matvec(reinterpret_cast<const float*>(m->base), (int)m->rows, (int)m->cols, x, (int)m->cols, k, y,
                       (int)m->rows, st, false));
    return IQ_OK;
  }
  if (m->dtype == BF16) {
    IQ_CUDA(bf16_matvec(reinterpret_cast<const uint16_t*>(m->base), (int)m->rows, (int)m->cols, x, (int)m->cols, k,
                        y, (int)m->rows, st));
    return IQ_OK;
  }
  const bool kq = m->dtype != Q8_0;
  const int64_t arb = kq ? act_row_bytes_q8k(m->cols) : act_row_bytes_q80(m->cols);
  IQ_CUDA(scratch().act.reserve((size_t)(arb * 8)));
  if ((uintptr_t)x & 15) {  // the quantizer reads 16-byte vectors
    IQ_CUDA(scratch().x.reserve((size_t)(m->cols * k * sizeof(float))));
    IQ_CUDA(cudaMemcpyAsync(scratch().x.p, x, (size_t)(m->cols * k * sizeof(float)), cudaMemcpyDeviceToDevice, st));
    x = scratch().x.as<float>();
  }
  PrepArgs pa = {};
  pa.x = x;
  pa.ldx = (int)m->cols;
  pa.cols = (int)m->cols;
  pa.inv_cols = 1.f / (float)m->cols;
  if (kq) pa.q8k = scratch().act.as<uint8_t>();
  else pa.q80 = scratch().act.as<uint8_t>();
  IQ_CUDA(prep_rows(pa, k, st, false));
  QmvJob j;
  memset(&j, 0, sizeof j);
  j.w = m->base;
  j.tmap = m->tmap();
  j.tmap_tail = m->tmap_tail();
  j.act = scratch().act.as<uint8_t>();
  j.out = y;
  j.w_row_bytes = m->row_bytes;
  j.act_row_bytes = (int)arb;
  j.out_ld = (int)m->rows;
  j.dtype = m->dtype;
  j.rows = (int)m->rows;
  j.cols = (int)m->cols;
  j.ksplit = qmv_ksplit(m->dtype, m->rows, m->cols);
  j.n = k;
  j.act_nrows = k;
  j.tile0 = 0;
  j.epi = kEpiStore;
  for (int i = 0; i < 8; i++) { j.rowmap[i] = (uint8_t)(i < k ? i : 0); j.outrow[i] = (int16_t)i; }
  iq_matrix* mm = const_cast<iq_matrix*>(m);
  if (!mm->job_cache->p || memcmp(&mm->last_job, &j, sizeof j) != 0) {
    IQ_CUDA(mm->job_cache->reserve(sizeof(QmvJob)));
    IQ_CUDA(cudaMemcpyAsync(mm->job_cache->p, &j, sizeof j, cudaMemcpyHostToDevice, st));
    mm->last_job = j;
  }
  IQ_CUDA(qmv_launch(mm->job_cache->as<QmvJob>(), 1, nullptr, qmv_tiles(j), (int)(arb * k), st, false));
  return IQ_OK;
}

}  // namespace iq

using namespace iq;

extern "C" {

const char* iq_last_error(void) { return g_error.c_str(); }
const char* iq_version(void) { return "inferq-b200 0.1 (sm_100a)"; }

int iq_matrix_create(int dtype, const void* data, int64_t rows, int64_t cols, int location, iq_matrix** out) {
  clear_error();
  IQ_CHECK(out && data, IQ_EINVAL, "iq_matrix_create: null argument");
  IQ_CHECK(location == IQ_HOST || location == IQ_DEVICE, IQ_EINVAL, "bad location %d", location);
  int rc = validate_matrix_shape(dtype, rows, cols);
  if (rc) return rc;
  auto buf = std::make_shared<DevBuf>();
  rc = upload_rows(dtype, data, rows, cols, location, *buf, nullptr);
  if (rc) return rc;
  auto maps = std::make_shared<DevBuf>();
  if (dtype != F32 && dtype != F16 && dtype != BF16)
    IQ_CHECK(qmv_tensor_maps(dtype, buf->as<uint8_t>(), rows, cols, *maps) == cudaSuccess, IQ_ECUDA,
             "cannot describe the matrix for the TMA unit");
  auto* m = new iq_matrix;
  m->dtype = dtype;
  m->rows = rows;
  m->cols = cols;
  m->row_bytes = dev_row_bytes(dtype, cols);
  m->storage = buf;
  m->base = buf->as<uint8_t>();
  m->maps = maps;
  *out = m;
  return IQ_OK;
}

int iq_matrix_leading_rows(const iq_matrix* m, int64_t rows, iq_matrix** out) {
  clear_error();
  IQ_CHECK(m && out, IQ_EINVAL, "iq_matrix_leading_rows: null argument");
  IQ_CHECK(rows > 0 && rows <= m->rows, IQ_EINVAL, "cannot take %lld leading rows of a %lld-row matrix",
           (long long)rows, (long long)m->rows);
  auto* r = new iq_matrix(*m);
  r->rows = rows;
  r->job_cache = std::make_shared<DevBuf>();
  r->last_job = {};
  *out = r;
  return IQ_OK;
}

void iq_matrix_destroy(iq_matrix* m) { delete m; }

int iq_matrix_shape(const iq_matrix* m, int64_t* rows, int64_t* cols, int* dtype) {
  IQ_CHECK(m, IQ_EINVAL, "iq_matrix_shape: null matrix");
  if (rows) *rows = m->rows;
  if (cols) *cols = m->cols;
  if (dtype) *dtype = m->dtype;
  return IQ_OK;
}

int iq_matrix_forward_device(const iq_matrix* m, const float* x, int input_rows, float* y, void* stream) {
  clear_error();
  IQ_CHECK(m && x && y, IQ_EINVAL, "iq_matrix_forward_device: null argument");
  IQ_CHECK(input_rows >= 1 && input_rows <= 8, IQ_EINVAL,
           "device forward takes 1..8 input rows, got %d", input_rows);
  return matrix_forward_dev(m, x, input_rows, y, static_cast<cudaStream_t>(stream));
}

int iq_matrix_forward_wide(const iq_matrix* m, const float* x, int input_rows, float* y, void* stream) {
  clear_error();
  IQ_CHECK(m && x && y, IQ_EINVAL, "iq_matrix_forward_wide: null argument");
  IQ_CHECK(m->dtype == Q8_0 || m->dtype == Q4_K || m->dtype == Q6_K || (m->dtype == Q5_K && wide_q5k_enabled()),
           IQ_EUNSUPPORTED, "the wide product takes Q8_0, Q4_K or Q6_K matrices (Q5_K with IQ_WIDE_Q5K), got dtype %d",
           m->dtype);
  IQ_CHECK(input_rows >= 1 && input_rows <= 65535, IQ_EINVAL, "expected 1..65535 input rows, got %d", input_rows);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m->dtype == Q6_K) {
    const size_t need = wide_q6k_scratch_bytes(m->rows, m->cols, input_rows, nullptr, nullptr);
    IQ_CUDA(scratch().wide_w.reserve(need));
    WideQ6kScratch sc;
    wide_q6k_scratch_bytes(m->rows, m->cols, input_rows, &sc, scratch().wide_w.as<uint8_t>());
    IQ_CUDA(wide_q6k_forward(m->base, m->rows, m->cols, m->row_bytes, x, (int)m->cols, input_rows, y, (int)m->rows,
                             sc, st));
    return IQ_OK;
  }
  if (m->dtype == Q4_K || m->dtype == Q5_K) {
    const bool q5 = m->dtype == Q5_K;
    const size_t need = wide_q4k_scratch_bytes(m->rows, m->cols, input_rows, nullptr, nullptr, q5);
    IQ_CUDA(scratch().wide_w.reserve(need));
    WideQ4kScratch sc;
    wide_q4k_scratch_bytes(m->rows, m->cols, input_rows, &sc, scratch().wide_w.as<uint8_t>(), q5);
    IQ_CUDA((q5 ? wide_q5k_forward : wide_q4k_forward)(m->base, m->rows, m->cols, m->row_bytes, x, (int)m->cols,
                                                       input_rows, y, (int)m->rows, sc, st));
    return IQ_OK;
  }
  IQ_CHECK(m->cols % 128 == 0, IQ_EINVAL, "the wide product needs cols %% 128 == 0, got %lld", (long long)m->cols);
  const int64_t nb = m->cols / 32;
  IQ_CUDA(scratch().x.reserve((size_t)(input_rows * m->cols * 2)));
  IQ_CUDA(scratch().act.reserve((size_t)(nb * wide_ldd(input_rows) * 4)));
  IQ_CUDA(scratch().wide_w.reserve((size_t)(m->rows * m->cols * 2)));
  IQ_CUDA(wide_q80_forward(m->base, m->rows, m->cols, m->row_bytes, x, (int)m->cols, input_rows, y, (int)m->rows,
                           scratch().x.as<__half>(), scratch().act.as<float>(), scratch().wide_w.as<__half>(), st));
  return IQ_OK;
}

int iq_matrix_status(void* stream) {
  clear_error();
  IQ_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  bool hit = false;
  for (int* f : {qmv_timeout_flag(), wide_timeout_flag()}) {
    if (!f) continue;
    int v = 0;
    IQ_CUDA(cudaMemcpy(&v, f, sizeof v, cudaMemcpyDeviceToHost));
    if (v) {
      hit = true;
      IQ_CUDA(cudaMemset(f, 0, sizeof v));
    }
  }
  IQ_CHECK(!hit, IQ_ETIMEDOUT,
           "a matrix product gave up a bounded device wait since the last check; its results are invalid");
  return IQ_OK;
}

int iq_matrix_forward_rows(const iq_matrix* m, const float* x, int64_t input_rows, float* y) {
  clear_error();
  IQ_CHECK(m && x && y, IQ_EINVAL, "iq_matrix_forward_rows: null argument");
  IQ_CHECK(input_rows >= 1, IQ_EINVAL, "expected at least one input row, got %lld", (long long)input_rows);
  cudaStream_t st = nullptr;
  IQ_CUDA(scratch().x.reserve((size_t)(8 * m->cols * 4)));
  IQ_CUDA(scratch().y.reserve((size_t)(8 * m->rows * 4)));
  for (int64_t r0 = 0; r0 < input_rows; r0 += 8) {
    const int k = (int)std::min<int64_t>(8, input_rows - r0);
    IQ_CUDA(cudaMemcpyAsync(scratch().x.p, x + r0 * m->cols, (size_t)(k * m->cols * 4), cudaMemcpyHostToDevice, st));
    int rc = matrix_forward_dev(m, scratch().x.as<float>(), k, scratch().y.as<float>(), st);
    if (rc) return rc;
    IQ_CUDA(cudaMemcpyAsync(y + r0 * m->rows, scratch().y.p, (size_t)(k * m->rows * 4), cudaMemcpyDeviceToHost, st));
  }
  IQ_CUDA(cudaStreamSynchronize(st));
  return IQ_OK;
}

int iq_qgemv(int dtype, const void* w, int64_t rows, int64_t cols, const float* x, int k, float* y, void* stream) {
  (void)stream;
  iq_matrix* m = nullptr;
  int rc = iq_matrix_create(dtype, w, rows, cols, IQ_HOST, &m);
  if (rc) return rc;
  rc = iq_matrix_forward_rows(m, x, k, y);
  iq_matrix_destroy(m);
  return rc;
}

int iq_qgemv_ksplit(int dtype, int64_t rows, int64_t cols) {
  if (validate_matrix_shape(dtype, rows, cols)) return IQ_EINVAL;
  return dtype == F32 || dtype == BF16 ? 1 : qmv_ksplit(dtype, rows, cols);
}

int iq_matrix_dequantize(const iq_matrix* m, const int32_t* ids, int64_t n, float* out) {
  clear_error();
  IQ_CHECK(m && out, IQ_EINVAL, "iq_matrix_dequantize: null argument");
  const int64_t rows = ids ? n : m->rows;
  DevBuf dids, dout;
  if (ids) {
    for (int64_t i = 0; i < n; i++)
      IQ_CHECK(ids[i] >= 0 && ids[i] < m->rows, IQ_EINVAL, "row id %d out of range", ids[i]);
    IQ_CUDA(dids.reserve((size_t)n * 4));
    IQ_CUDA(cudaMemcpy(dids.p, ids, (size_t)n * 4, cudaMemcpyHostToDevice));
  }
  IQ_CUDA(dout.reserve((size_t)(rows * m->cols * 4)));
  IQ_CUDA(dequant_rows(m->dtype, m->base, m->row_bytes, (int)m->cols, dids.as<int32_t>(), rows,
                       dout.as<float>(), nullptr));
  IQ_CUDA(cudaMemcpy(out, dout.p, (size_t)(rows * m->cols * 4), cudaMemcpyDeviceToHost));
  return IQ_OK;
}

}  // extern "C"
