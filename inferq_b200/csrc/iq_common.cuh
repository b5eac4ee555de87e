// iq_common.cuh -- shared device helpers for the sm_100a verify path.
//
// Build rules that matter for numerics: no --use_fast_math, and every
// multiply-add that the reference rounds twice is written with __fmul_rn /
// __fadd_rn so the compiler cannot contract it into an FMA.
#pragma once
#include <cstdint>
#include <mutex>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace iq {

// GGML dtype ids.
enum Dtype : int { F32 = 0, F16 = 1, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15, BF16 = 30 };

constexpr int kWarp = 32;

__host__ __device__ constexpr inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr inline int64_t align_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// ------------------------------------------------------------ layouts
// GGUF block sizes (bytes per block, weights per block).
__host__ __device__ inline int gguf_block_bytes(int dt) {
  return dt == Q4_K ? 144 : dt == Q5_K ? 176 : dt == Q6_K ? 210 : dt == Q8_0 ? 34 : dt == F32 ? 4 : 2;
}
__host__ __device__ inline int gguf_block_elems(int dt) {
  return (dt == Q4_K || dt == Q5_K || dt == Q6_K) ? 256 : dt == Q8_0 ? 32 : 1;
}
__host__ __device__ inline int64_t gguf_row_bytes(int dt, int64_t cols) {
  return cols / gguf_block_elems(dt) * gguf_block_bytes(dt);
}
// Device row layout (see layout.cu): Q4_K and Q5_K keep their block size;
// Q6_K and Q8_0 move the f16 block scale into a 16-byte-padded row tail.
__host__ __device__ inline int64_t dev_row_bytes(int dt, int64_t cols) {
  int64_t nb = cols / gguf_block_elems(dt);
  switch (dt) {
    case Q4_K: return nb * 144;
    case Q5_K: return nb * 176;
    case Q6_K: return nb * 208 + align_up(nb * 2, 16);
    case Q8_0: return nb * 32 + align_up(nb * 2, 16);
    case F32: return cols * 4;
    default: return cols * 2;
  }
}
// Quantized-activation row bytes: Q8_K {qs[256] permuted, f32 d, i16 bsums[16]}
// as three planes; Q8_0 {qs[32] permuted, f32 d} as two planes.
// Q8_K activation row: nb x 256 quants, nb f32 d (padded to 16 B), then
// nb x 16 B of eight i16 sums of 32 quants.
__host__ __device__ constexpr inline int64_t q8k_bs_offset(int64_t nb) { return nb * 256 + align_up(nb * 4, 16); }
__host__ __device__ constexpr inline int64_t act_row_bytes_q8k(int64_t cols) {
  int64_t nb = cols / 256;
  return q8k_bs_offset(nb) + nb * 16;
}
__host__ __device__ constexpr inline int64_t act_row_bytes_q80(int64_t cols) {
  int64_t nb = cols / 32;
  return align_up(nb * 32 + nb * 4, 16);
}

// --------------------------------------------------------- small PTX
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// Per-device one-time setup (a kernel's shared-memory opt-in attribute and
// the like): runs `setup()` on the current device until it first succeeds
// (one flag per device, guarded by one lock per flag set), and returns its
// result, or cudaSuccess once it has succeeded.
template <class F>
inline cudaError_t once_per_device(bool (&done)[64], std::mutex& mu, F setup) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev]) return cudaSuccess;
  e = setup();
  if (e == cudaSuccess) done[dev] = true;
  return e;
}

// exp and log1p of an f32 argument evaluated in double precision and rounded
// once to f32.  That is the correctly rounded f32 result except in
// vanishingly rare near-halfway cases, which is what the reference's libm
// expf / log1pf return in practice (within about half an ulp), so the model
// kernels and the reference agree on these to the bit.  (CUDA's single-
// precision expf may differ from it by an ulp or two, and a last-bit
// difference can flip a later activation rounding.)
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log1p_ref(float x) { return (float)log1p((double)x); }

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// D = A(16x32 u8, row) * B(32x8 s8, col) + C, exact int32.
__device__ __forceinline__ void mma_u8s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A(16x32 s8) * B(32x8 s8) + C.
__device__ __forceinline__ void mma_s8s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D = A(16x16 s8) * B(16x8 s8) + C.
__device__ __forceinline__ void mma_s8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Eight 6-bit scales (sc) and mins (mn) of a Q4_K/Q5_K header; the byte
// sequence of the reference's unpack_k_scales (src/qgemm.rs:153-167).
__device__ __forceinline__ void unpack_k_scales(const uint8_t* s, int sc[8], int mn[8]) {
#pragma unroll
  for (int j = 0; j < 4; j++) {
    sc[j] = s[j] & 63;
    mn[j] = s[j + 4] & 63;
    sc[j + 4] = (s[j + 8] & 0xf) | ((s[j] >> 6) << 4);
    mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
  }
}

}  // namespace iq
