// api_util.h -- error reporting and small RAII helpers behind the C ABI.
#pragma once
#include <cstdarg>
#include <cstdio>
#include <string>
#include <cuda_runtime.h>
#include "../../include/iq.h"

namespace iq {

void set_error(const char* fmt, ...);
void clear_error();

// Evaluate a CUDA call; on failure record the error and return IQ_ECUDA.
#define IQ_CUDA(expr)                                                                       \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    if (_e != cudaSuccess) {                                                                \
      ::iq::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
      return IQ_ECUDA;                                                                      \
    }                                                                                       \
  } while (0)

#define IQ_CHECK(cond, code, ...) \
  do {                            \
    if (!(cond)) {                \
      ::iq::set_error(__VA_ARGS__); \
      return (code);              \
    }                             \
  } while (0)

// Device buffer owned by a handle.
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) {
      release();
      p = o.p; bytes = o.bytes;
      o.p = nullptr; o.bytes = 0;
    }
    return *this;
  }
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  // Grow to at least n bytes (contents not preserved).
  cudaError_t reserve(size_t n) {
    if (n <= bytes) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&p, n);
    if (e == cudaSuccess) bytes = n;
    else p = nullptr;
    return e;
  }
  template <class T>
  T* as() const { return reinterpret_cast<T*>(p); }
};

}  // namespace iq
