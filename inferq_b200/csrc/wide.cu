// wide.cu -- the wide quantized matrix product: many input rows at once (the
// reference's prefill passes, src/runtime.rs:748-771 prefill_in_passes, 512
// rows per pass through QuantizedMatrix::forward, src/gguf.rs:406-456) for
// Q8_0 weights, on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// Arithmetic.  Every 32-element block contributes one f32 term per output,
// as in the per-block device order of the narrow GEMV with one K chunk:
//     acc = fmaf(d_w * d_x, (float)isum, acc),   blocks in ascending order,
// where isum = sum_e q_w[e] * q_x[e] is the exact integer dot
// (src/qgemm.rs:369-397 forms the same integer dots).  The tensor cores form
// isum exactly: q_w and q_x (|q| <= 128) are exact in f16, each product is
// exact in f32, and a block's sum stays below 2^20, so an M=128 N=128 K=16
// f16 MMA pair with a fresh f32 accumulator per block yields isum itself.
// The epilogue then applies the scale product and the FMA in block order,
// so outputs are bitwise those of the per-block device order.
//
// Two kernels per call besides the input quantizer: wide_expand_q80_kernel
// writes the weights once as f16 integers (row-major, a bandwidth-bound
// pass), and wide_q80_kernel multiplies.  Expanding inside the product
// kernel was measured slower: its converter warps took issue slots and
// shared-memory bandwidth from the epilogue, which paces the kernel.
//
// Tiles.  One CTA computes 128 weight rows x 128 input rows.  An operand
// stage covers one group of four Q8_0 blocks (128 K elements):
//   A  32 KB  weights, f16, K-major, 128-byte swizzle (two 64-element atoms)
//   B  32 KB  input rows, f16 integers, same layout
// both by TMA, released as soon as the MMAs that read the stage complete.
// The scales the epilogue needs go to a deeper side ring that the epilogue
// releases:
//   D   2 KB  input-row block scales [4 blocks][128 rows] f32
//   S   2 KB  the weight rows' f16 scale tail, 16 B per row (the group's
//             four scales are one half of it)
// Three operand stages (192 KB) and six side entries (24 KB).  TMEM holds
// four 128-column f32 buffers, one per block of a stage.
//
// Warp roles: 0-15 epilogue (warp w reads TMEM lanes 32*(w%4).. and 32 of the
// 128 columns, in two 16-column halves with one load in flight while the
// previous half is scaled), 16 TMA loads (one lane), 17 MMAs (one lane).
// The two issuers sit in different warps: a lane suspended in an mbarrier
// wait holds its whole warp, so issuers that wait on each other's progress
// must not share one.  Every wait is bounded; a wait that runs out sets the
// wide product's timeout flag (reported by iq_matrix_status) and the CTA
// winds down (copies and MMAs drained, TMEM freed) without storing.
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <cstdlib>
#include <cstring>
#include "iq_common.cuh"
#include "layout.cuh"
#include "kernels.cuh"
#include "qmv.cuh"
#include "wide_expand.cuh"

namespace iq {
namespace {

constexpr int kRows = 128, kToks = 128, kStageK = 128;
constexpr int kStages = 3;
constexpr int kEpiWarps = 16;
constexpr int kTmaWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1;
constexpr int kThreads = (kMmaWarp + 1) * 32;
// registers per thread: 18 warps spread 5/5/4/4 over the SM's four register
// files of 16384, so at most 16384 / (5 * 32) -> 96
constexpr int kBoundThreads = 640;
constexpr int kAtom = 128 * 128;  // one 64-element f16 atom of 128 rows
constexpr int kOffA = 0, kOffB = 2 * kAtom;
constexpr int kStageBytes = 4 * kAtom;
constexpr int kSide = 6, kSideBytes = 4096, kOffS = 2048;  // D at 0, S at 2048
constexpr int kSmemBytes = kStages * kStageBytes + kSide * kSideBytes + 1024;
constexpr int kTmemCols = 512;
constexpr int kWaitLimit = 1 << 20;
// Waits that only let work already in flight finish before the CTA winds
// down (copies landing, MMAs completing) always use this longer bound, also
// when a test shortens the other waits: no async operation may outlive the
// CTA's shared memory or TMEM.
constexpr int kDrainLimit = 1 << 24;
static_assert(kStageBytes % 1024 == 0, "swizzled atoms stay 1024-byte aligned");

// f32 D, f16 A and B, both K-major, N = 128, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kToks >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

__device__ int g_wide_timeout;  // set when a bounded wait gave up

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int limit) {
  const uint32_t a = su32(b);
  for (int i = 0; i < limit; i++) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok)
                 : "r"(a), "r"(parity)
                 : "memory");
    if (ok) return true;
  }
  return false;
}
// 2-D TMA tile load from this GPU's memory (no multicast).
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* m, int x, int y, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(su32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(su32(b))
      : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (leading offset unused for this layout), sm_100 version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
               : "memory");
}
// Start a 16-column TMEM load (lanes of this warp's quarter); the registers
// are valid only after tmem_wait16 on the same array.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
// Wait for this thread's TMEM loads; the array is an in/out operand so no
// use of it can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15])
               :
               : "memory");
}

// (a0, a1) = fma(dw * d0, v0, a0), fma(dw * d1, v1, a1), each lane rounded
// as the scalar mul and fma (packed f32x2 forms of sm_100).
__device__ __forceinline__ void scale_fma2(float& a0, float& a1, float dw, float d0, float d1, uint32_t v0,
                                           uint32_t v1) {
  asm("{ .reg .b64 t, w, v, a;\n"
      "mov.b64 t, {%2, %3};\n"
      "mov.b64 w, {%4, %4};\n"
      "mul.rn.f32x2 t, t, w;\n"
      "mov.b64 v, {%5, %6};\n"
      "mov.b64 a, {%0, %1};\n"
      "fma.rn.f32x2 a, t, v, a;\n"
      "mov.b64 {%0, %1}, a; }"
      : "+f"(a0), "+f"(a1)
      : "f"(d0), "f"(d1), "f"(dw), "r"(v0), "r"(v1));
}
// acc[0..15] += the 16 scaled block dots v of columns d[0..15].
__device__ __forceinline__ void scale_half(float* acc, float dw, const float* d, const uint32_t (&v)[16]) {
  const float4* d4 = reinterpret_cast<const float4*>(d);
#pragma unroll
  for (int i4 = 0; i4 < 4; i4++) {
    const float4 x = d4[i4];
    scale_fma2(acc[4 * i4], acc[4 * i4 + 1], dw, x.x, x.y, v[4 * i4], v[4 * i4 + 1]);
    scale_fma2(acc[4 * i4 + 2], acc[4 * i4 + 3], dw, x.z, x.w, v[4 * i4 + 2], v[4 * i4 + 3]);
  }
}

// Four signed bytes -> four f16 (exact): 0x6400 | (q ^ 0x80) is 1024 + q + 128.
__device__ __forceinline__ uint2 s8x4_to_f16x4(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t lo = __byte_perm(u, 0x64646464u, 0x4140), hi = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&lo), off);
  __half2 b = __hsub2(*reinterpret_cast<const __half2*>(&hi), off);
  return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

__global__ void __launch_bounds__(kBoundThreads, 1)
    wide_q80_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_d, const __grid_constant__ CUtensorMap tm_s,
                    int scale_x0, int rows, int nb, int ntok, float* __restrict__ y, int out_ld,
                    int* timeout_flag, int test_skip) {
  __shared__ __align__(8) uint64_t full_op[kStages], empty_op[kStages];
  __shared__ __align__(8) uint64_t full_side[kSide], empty_side[kSide];
  __shared__ __align__(8) uint64_t tfull[4], tempty[4], drained;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (su32(smem_raw) & 1023)) & 1023);
  uint8_t* side = smem + kStages * kStageBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * kToks, row0 = blockIdx.y * kRows;
  const int nst = nb / 4;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      bar_init(&full_op[s], 1);
      bar_init(&empty_op[s], 1);
    }
    for (int e = 0; e < kSide; e++) {
      bar_init(&full_side[e], 1);
      bar_init(&empty_side[e], kEpiWarps);
    }
    for (int j = 0; j < 4; j++) {
      bar_init(&tfull[j], 1);
      bar_init(&tempty[j], kEpiWarps);
    }
    bar_init(&drained, 1);
    abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_s)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;
  // test_skip (tests only): the MMA thread skips the first stage, so the
  // epilogue's first TMEM wait runs out and the CTA takes the wind-down path
  const int lim = test_skip ? 256 : kWaitLimit;
  auto give_up = [&]() {
    atomicExch(timeout_flag, 1);
    *abort_v = 1;
  };

  if (warp < kEpiWarps) {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3, cb = 32 * (warp >> 2), r = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)cb;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; i++) acc[i] = 0.f;
    uint32_t va[16], vb[16];
    bool ok = true;
    for (int it = 0; it < nst && ok; it++) {
      const int e = it % kSide;
      const uint8_t* sd = side + e * kSideBytes;
      // warp-uniform outcomes: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, bar_wait(&full_side[e], (it / kSide) & 1, lim)) ||
          !__all_sync(0xffffffffu, bar_wait(&tfull[0], it & 1, lim))) {
        give_up();
        ok = false;
        break;
      }
      tc_after();
      tmem_ld16(lane_base, va);
      tmem_wait16(va);
      const float* ds = reinterpret_cast<const float*>(sd);
      const __half* ws = reinterpret_cast<const __half*>(sd + kOffS + r * 16 + 8 * (it & 1));
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float dw = __half2float(ws[j]);
        tmem_ld16(lane_base + (uint32_t)(j * 128 + 16), vb);  // second half, in flight
        scale_half(acc, dw, ds + j * 128 + cb, va);
        tmem_wait16(vb);
        tc_before();
        __syncwarp();
        if (lane == 0) bar_arrive(&tempty[j]);
        if (j < 3) {
          if (!__all_sync(0xffffffffu, bar_wait(&tfull[j + 1], it & 1, lim))) {
            give_up();
            ok = false;
            break;
          }
          tc_after();
          tmem_ld16(lane_base + (uint32_t)((j + 1) * 128), va);  // next block's first half, in flight
        }
        scale_half(acc + 16, dw, ds + j * 128 + cb + 16, vb);
        if (j < 3) tmem_wait16(va);
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&empty_side[e]);
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");  // nothing in flight past this point
    if (ok && !*abort_v) {
      const int row = row0 + r;
      if (row < rows) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int t = tok0 + cb + i;
          if (t < ntok) y[(int64_t)t * out_ld + row] = acc[i];
        }
      }
    }
  } else if (warp == kTmaWarp && lane == 0) {
    // ------------------------------------------------------ TMA producer
    int issued = 0;
    for (int it = 0; it < nst && !*abort_v; it++) {
      const int s = it % kStages, e = it % kSide;
      if (it >= kStages && !bar_wait(&empty_op[s], ((it / kStages) + 1) & 1, lim)) { give_up(); break; }
      uint8_t* st = smem + s * kStageBytes;
      bar_expect(&full_op[s], kStageBytes);
      tma2d(st + kOffA, &tm_w, it * kStageK, row0, &full_op[s]);
      tma2d(st + kOffA + kAtom, &tm_w, it * kStageK + 64, row0, &full_op[s]);
      tma2d(st + kOffB, &tm_x, it * kStageK, tok0, &full_op[s]);
      tma2d(st + kOffB + kAtom, &tm_x, it * kStageK + 64, tok0, &full_op[s]);
      if (it >= kSide && !bar_wait(&empty_side[e], ((it / kSide) + 1) & 1, lim)) {
        issued = it + 1;
        give_up();
        break;
      }
      uint8_t* sd = side + e * kSideBytes;
      bar_expect(&full_side[e], kSideBytes);
      tma2d(sd, &tm_d, tok0, it * 4, &full_side[e]);
      tma2d(sd + kOffS, &tm_s, scale_x0 + 16 * (it >> 1), row0, &full_side[e]);
      issued = it + 1;
    }
    if (*abort_v) {  // let the copies in flight land before the CTA exits
      for (int it = issued > kStages ? issued - kStages : 0; it < issued; it++)
        bar_wait(&full_op[it % kStages], (it / kStages) & 1, kDrainLimit);
      for (int it = issued > kSide ? issued - kSide : 0; it < issued; it++)
        bar_wait(&full_side[it % kSide], (it / kSide) & 1, kDrainLimit);
    }
  } else if (warp == kMmaWarp && lane == 0) {
    // ------------------------------------------------------- MMA issuer
    for (int it = 0; it < nst && !*abort_v; it++) {
      const int s = it % kStages;
      if (!bar_wait(&full_op[s], (it / kStages) & 1, lim)) {
        give_up();
        break;
      }
      if (test_skip && it == 0) continue;
      tc_after();
      const uint32_t a0 = su32(smem + s * kStageBytes + kOffA), b0 = su32(smem + s * kStageBytes + kOffB);
      bool ok = true;
      for (int j = 0; j < 4; j++) {
        if (it > 0 && !bar_wait(&tempty[j], (it - 1) & 1, lim)) {
          give_up();
          ok = false;
          break;
        }
        tc_after();
        const uint32_t off = (uint32_t)((j >> 1) * kAtom + (j & 1) * 64);
#pragma unroll
        for (int kk = 0; kk < 2; kk++)
          mma_f16(tmem + (uint32_t)(j * 128), sw128_desc(a0 + off + 32 * kk), sw128_desc(b0 + off + 32 * kk),
                  (uint32_t)kk);
        mma_commit(&tfull[j]);
      }
      if (!ok) break;
      mma_commit(&empty_op[s]);
    }
    mma_commit(&drained);  // every MMA issued above has completed when this fires
    bar_wait(&drained, 0, kDrainLimit);
  }
  __syncwarp();
  tc_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Input rows -> f16 integers q (row-major, cols wide) and the f16-rounded
// block scales transposed, dT[b * ldd + t].  Same arithmetic as the narrow
// path's Q8_0 quantizer (candle BlockQ8_0::from_float: d = amax / 127 kept
// as f16, q = round(x / d) from the f32 d).  One warp per (row, block).
__global__ void wide_act_kernel(const float* __restrict__ x, int ldx, int cols, __half* __restrict__ q,
                                float* __restrict__ dT, int ldd) {
  const int t = blockIdx.y, b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b * 32 >= cols) return;
  const float v = x[(int64_t)t * ldx + b * 32 + lane];
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float d = __fdiv_rn(amax, 127.f);
  const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
  const int qi = (int)(int8_t)roundf(__fmul_rn(v, id));
  q[(int64_t)t * cols + b * 32 + lane] = __int2half_rn(qi);
  if (lane == 0) dT[(int64_t)b * ldd + t] = __half2float(__float2half_rn(d));
}

// Device-layout Q8_0 rows -> f16 integers, row-major (the weight operand of
// the product).  One thread per 16-byte chunk of a four-block group: byte
// tig*32 + bb*8 + h*4 + e holds element 16h + 4tig + e of block bb.
__global__ void wide_expand_q80_kernel(const uint8_t* __restrict__ w, int64_t w_row_bytes, int rows, int cols,
                                       __half* __restrict__ out) {
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int groups = cols / 128;
  const int64_t r = id / (groups * 8);
  if (r >= rows) return;
  const int g = (int)(id / 8 % groups), cc = (int)(id & 7), tig = cc >> 1;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(w + r * w_row_bytes + g * 128 + cc * 16));
  const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const int bb = 2 * (cc & 1) + (q >> 1), h = q & 1;
    const int k = g * 128 + bb * 32 + 16 * h + 4 * tig;
    *reinterpret_cast<uint2*>(out + r * cols + k) = s8x4_to_f16x4(wd[q]);
  }
}

// ----------------------------------------------------------------- Q4_K
// The same product for Q4_K weights x Q8_K input rows, bitwise the
// per-block device order (src/qgemm.rs:153-240 forms the same integers):
//     isum = sum_s sc[s] * sum_{e in s} q_e x_e,  msum = sum_s mn[s] * bsum_s
//     acc  = fmaf(d_x * d_w, (float)isum, acc),  accm = fmaf(d_x * dmin, (float)msum, accm)
//     y    = acc - accm
// The sub-block scales are folded into the weight operand, A = sc[s] * q
// (<= 63 * 15, exact in f16), so the tensor cores form isum directly.  A
// whole block can reach 256 * 945 * 128 > 2^24, so each block's two halves
// go to separate TMEM accumulators (each below 2^24, exact) and
// (float)isum is their f32 sum (one rounding of the exact integer).  msum is
// one more K=16 MMA per block: A_m = (mn[0..7], 64 * mn[0..7]) against
// B_m = (bsum mod 64, bsum div 64), all exact in f16.  Tiles: 128 weight
// rows x 64 input rows, one 256-element block per stage; TMEM holds two
// blocks' three 64-column accumulators.
constexpr int kQ4Toks = 64;
constexpr int kQ4AtomA = 128 * 128, kQ4AtomB = kQ4Toks * 128;
constexpr int kQ4OffB = 4 * kQ4AtomA, kQ4OffAm = kQ4OffB + 4 * kQ4AtomB, kQ4OffBm = kQ4OffAm + 4096;
constexpr int kQ4StageBytes = kQ4OffBm + 2048;  // 102 KB
constexpr int kQ4Stages = 2;
constexpr int kQ4Side = 4, kQ4SideBytes = 2560, kQ4OffH = 256;  // input-row d (64 f32), then 16-B row headers
constexpr int kQ4SmemBytes = kQ4Stages * kQ4StageBytes + kQ4Side * kQ4SideBytes + 1024;
static_assert(kQ4StageBytes % 1024 == 0, "swizzled atoms stay 1024-byte aligned");
// Q5_K, the same kernel: A = sc[s] * (q - 16), |.| <= 63 * 16, so each
// half block stays below 128 * 1008 * 128 < 2^24 (exact), and one more
// K=16 MMA forms the centring term c = sum_s sc[s] * bsum_s from
// A_c = (sc[0..7], 64 * sc[0..7]) against the same B_m, exact below 2^22;
// isum = a + b + 16 c, summed as integers.  The stage gains the 4 KB A_c
// tile and TMEM holds four accumulators per block (two blocks: 512 columns).
constexpr int kQ5OffAc = kQ4StageBytes, kQ5StageBytes = kQ4StageBytes + 4096;  // 106 KB
constexpr int kQ5SmemBytes = kQ4Stages * kQ5StageBytes + kQ4Side * kQ4SideBytes + 1024;
static_assert(kQ5StageBytes % 1024 == 0, "swizzled atoms stay 1024-byte aligned");
static_assert(kQ5SmemBytes + 1024 <= 227 * 1024, "Q5_K stages and the 1 KB of static shared memory fit the opt-in");
constexpr uint32_t kQ4Idesc = (1u << 4) | ((uint32_t)(kQ4Toks >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void mma_f16_n64(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kQ4Idesc), "r"(accumulate)
      : "memory");
}
// K-major operand without swizzle: 8-row x 16-byte core matrices, the two
// 16-byte K halves 128 bytes apart, 8-row groups 256 bytes apart.
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         ((uint64_t)1 << 46);
}
// 1-D bulk copy global -> shared (this GPU's memory, no multicast).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(b))
               : "memory");
}

template <bool kQ5>
__global__ void __launch_bounds__(kBoundThreads, 1)
    wide_q4k_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_d, const __grid_constant__ CUtensorMap tm_h,
                    const uint8_t* __restrict__ am, const uint8_t* __restrict__ bm, const uint8_t* __restrict__ ac,
                    int rows, int nb, int ntok, float* __restrict__ y, int out_ld, int* timeout_flag,
                    int test_skip) {
  constexpr int kStage = kQ5 ? kQ5StageBytes : kQ4StageBytes;
  constexpr int kBlkBytes = kQ5 ? 176 : 144;        // device block bytes; its header starts it
  constexpr uint32_t kBufCols = kQ5 ? 256u : 192u;  // TMEM columns per block buffer
  __shared__ __align__(8) uint64_t full_op[kQ4Stages], empty_op[kQ4Stages];
  __shared__ __align__(8) uint64_t full_side[kQ4Side], empty_side[kQ4Side];
  __shared__ __align__(8) uint64_t tfull[2], tempty[2], drained;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (su32(smem_raw) & 1023)) & 1023);
  uint8_t* side = smem + kQ4Stages * kStage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * kQ4Toks, row0 = blockIdx.y * 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQ4Stages; s++) {
      bar_init(&full_op[s], 1);
      bar_init(&empty_op[s], 1);
    }
    for (int e = 0; e < kQ4Side; e++) {
      bar_init(&full_side[e], 1);
      bar_init(&empty_side[e], kEpiWarps);
    }
    for (int j = 0; j < 2; j++) {
      bar_init(&tfull[j], 1);
      bar_init(&tempty[j], kEpiWarps);
    }
    bar_init(&drained, 1);
    abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_s)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;
  const int lim = test_skip ? 256 : kWaitLimit;
  auto give_up = [&]() {
    atomicExch(timeout_flag, 1);
    *abort_v = 1;
  };

  if (warp < kEpiWarps) {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3, cb = 16 * (warp >> 2), r = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)cb;
    float acc[16], accm[16];
#pragma unroll
    for (int i = 0; i < 16; i++) acc[i] = accm[i] = 0.f;
    bool ok = true;
    for (int it = 0; it < nb && ok; it++) {
      const int e = it % kQ4Side, buf = it & 1;
      const uint8_t* sd = side + e * kQ4SideBytes;
      if (!__all_sync(0xffffffffu, bar_wait(&full_side[e], (it / kQ4Side) & 1, lim)) ||
          !__all_sync(0xffffffffu, bar_wait(&tfull[buf], (it >> 1) & 1, lim))) {
        give_up();
        ok = false;
        break;
      }
      tc_after();
      uint32_t va[16], vb[16], vm[16];
      tmem_ld16(lane_base + buf * kBufCols, va);
      tmem_ld16(lane_base + buf * kBufCols + 64u, vb);
      if constexpr (kQ5) {
        // isum = a + b + 16 c: exact integers (each below 2^24) summed as
        // int32, then one rounding, as (float)isum in the block order
        tmem_ld16(lane_base + buf * kBufCols + 192u, vm);
        tmem_wait16(va);
        tmem_wait16(vb);
        tmem_wait16(vm);
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int is = __float2int_rn(__uint_as_float(va[i])) + __float2int_rn(__uint_as_float(vb[i])) +
                         16 * __float2int_rn(__uint_as_float(vm[i]));
          va[i] = __float_as_uint(__int2float_rn(is));
          vb[i] = 0u;  // +0.0f, so the sum below is isum itself
        }
      }
      tmem_ld16(lane_base + buf * kBufCols + 128u, vm);
      if constexpr (!kQ5) {
        tmem_wait16(va);
        tmem_wait16(vb);
      }
      tmem_wait16(vm);
      tc_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&tempty[buf]);
      const float* dx = reinterpret_cast<const float*>(sd) + cb;
      const __half* hd = reinterpret_cast<const __half*>(sd + kQ4OffH + r * 16);
      const float dw = __half2float(hd[0]), dmin = __half2float(hd[1]);
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const float isum = __fadd_rn(__uint_as_float(va[i]), __uint_as_float(vb[i]));
        acc[i] = __fmaf_rn(__fmul_rn(dx[i], dw), isum, acc[i]);
        accm[i] = __fmaf_rn(__fmul_rn(dx[i], dmin), __uint_as_float(vm[i]), accm[i]);
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&empty_side[e]);
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (ok && !*abort_v) {
      const int row = row0 + r;
      if (row < rows) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int t = tok0 + cb + i;
          if (t < ntok) y[(int64_t)t * out_ld + row] = __fsub_rn(acc[i], accm[i]);
        }
      }
    }
  } else if (warp == kTmaWarp && lane == 0) {
    // ------------------------------------------------------ TMA producer
    const uint8_t* am_tile = am + (int64_t)blockIdx.y * nb * 4096;
    const uint8_t* bm_tile = bm + (int64_t)blockIdx.x * nb * 2048;
    const uint8_t* ac_tile = kQ5 ? ac + (int64_t)blockIdx.y * nb * 4096 : nullptr;
    int issued = 0;
    for (int it = 0; it < nb && !*abort_v; it++) {
      const int s = it % kQ4Stages, e = it % kQ4Side;
      if (it >= kQ4Stages && !bar_wait(&empty_op[s], ((it / kQ4Stages) + 1) & 1, lim)) { give_up(); break; }
      uint8_t* st = smem + s * kStage;
      bar_expect(&full_op[s], kStage);
#pragma unroll
      for (int a = 0; a < 4; a++) {
        tma2d(st + a * kQ4AtomA, &tm_w, it * 256 + 64 * a, row0, &full_op[s]);
        tma2d(st + kQ4OffB + a * kQ4AtomB, &tm_x, it * 256 + 64 * a, tok0, &full_op[s]);
      }
      bulk_load(st + kQ4OffAm, am_tile + (int64_t)it * 4096, 4096, &full_op[s]);
      bulk_load(st + kQ4OffBm, bm_tile + (int64_t)it * 2048, 2048, &full_op[s]);
      if constexpr (kQ5) bulk_load(st + kQ5OffAc, ac_tile + (int64_t)it * 4096, 4096, &full_op[s]);
      if (it >= kQ4Side && !bar_wait(&empty_side[e], ((it / kQ4Side) + 1) & 1, lim)) {
        issued = it + 1;
        give_up();
        break;
      }
      uint8_t* sd = side + e * kQ4SideBytes;
      bar_expect(&full_side[e], kQ4OffH + 2048);
      tma2d(sd, &tm_d, tok0, it, &full_side[e]);
      tma2d(sd + kQ4OffH, &tm_h, it * kBlkBytes, row0, &full_side[e]);
      issued = it + 1;
    }
    if (*abort_v) {
      for (int it = issued > kQ4Stages ? issued - kQ4Stages : 0; it < issued; it++)
        bar_wait(&full_op[it % kQ4Stages], (it / kQ4Stages) & 1, kDrainLimit);
      for (int it = issued > kQ4Side ? issued - kQ4Side : 0; it < issued; it++)
        bar_wait(&full_side[it % kQ4Side], (it / kQ4Side) & 1, kDrainLimit);
    }
  } else if (warp == kMmaWarp && lane == 0) {
    // ------------------------------------------------------- MMA issuer
    for (int it = 0; it < nb && !*abort_v; it++) {
      const int s = it % kQ4Stages, buf = it & 1;
      if (!bar_wait(&full_op[s], (it / kQ4Stages) & 1, lim)) {
        give_up();
        break;
      }
      if (test_skip && it == 0) continue;
      if (it >= 2 && !bar_wait(&tempty[buf], ((it >> 1) + 1) & 1, lim)) {
        give_up();
        break;
      }
      tc_after();
      const uint32_t a0 = su32(smem + s * kStage), b0 = a0 + kQ4OffB;
      const uint32_t d0 = tmem + buf * kBufCols;
#pragma unroll
      for (int kk = 0; kk < 16; kk++) {  // K steps of 16: halves 0..127 -> a, 128..255 -> b
        const uint32_t off_a = (uint32_t)((kk >> 2) * kQ4AtomA + (kk & 3) * 32);
        const uint32_t off_b = (uint32_t)((kk >> 2) * kQ4AtomB + (kk & 3) * 32);
        mma_f16_n64(d0 + (kk < 8 ? 0u : 64u), sw128_desc(a0 + off_a), sw128_desc(b0 + off_b),
                    (uint32_t)((kk & 7) != 0));
      }
      mma_f16_n64(d0 + 128u, plain_desc(a0 + kQ4OffAm), plain_desc(a0 + kQ4OffBm), 0u);
      if constexpr (kQ5) mma_f16_n64(d0 + 192u, plain_desc(a0 + kQ5OffAc), plain_desc(a0 + kQ4OffBm), 0u);
      mma_commit(&tfull[buf]);
      mma_commit(&empty_op[s]);
    }
    mma_commit(&drained);
    bar_wait(&drained, 0, kDrainLimit);
  }
  __syncwarp();
  tc_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Input rows -> Q8_K integers as f16 (row-major), the block scales d
// transposed (dT[b * ldd + t]) and the min operand tiles: per 64 input
// rows and block, core-matrix order, (bsum_s mod 64, bsum_s div 64) for the
// eight 32-element sub-block sums.  The arithmetic is the narrow path's Q8_K
// quantizer (candle BlockQ8K::from_float: the first value of largest
// magnitude sets iscale = -128 / v, q = min(round(iscale * x), 127),
// d = 1 / iscale).  One warp per (row, block); lane tig*8 + s holds elements
// 32s + 16h + 4tig + e.
__global__ void wide_act_q8k_kernel(const float* __restrict__ x, int ldx, int cols, __half* __restrict__ q,
                                    float* __restrict__ dT, int ldd, uint8_t* __restrict__ bm) {
  const int t = blockIdx.y, b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int nb = cols / 256;
  if (b >= nb) return;
  const int s = lane & 7, tig = lane >> 3;
  const float* xr = x + (int64_t)t * ldx + b * 256;
  float v[8];
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int e = 0; e < 4; e++) v[4 * h + e] = xr[32 * s + 16 * h + 4 * tig + e];
  float amax = 0.f, vmax = 0.f;
  int imax = 1 << 30;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float a = fabsf(v[i]);
    if (amax < a) { amax = a; vmax = v[i]; imax = 32 * s + 16 * (i / 4) + tig * 4 + (i % 4); }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, amax, m);
    const float ov = __shfl_xor_sync(0xffffffffu, vmax, m);
    const int oi = __shfl_xor_sync(0xffffffffu, imax, m);
    if (oa > amax || (oa == amax && oi < imax)) { amax = oa; vmax = ov; imax = oi; }
  }
  int qi[8];
  float d = 0.f;
  if (amax != 0.f) {
    const float iscale = __fdiv_rn(-128.f, vmax);
#pragma unroll
    for (int i = 0; i < 8; i++) qi[i] = (int)(int8_t)fminf(roundf(__fmul_rn(iscale, v[i])), 127.f);
    d = __fdiv_rn(1.f, iscale);
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) qi[i] = 0;
  }
  __half* qr = q + (int64_t)t * cols + b * 256;
  int sum = 0;
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      qr[32 * s + 16 * h + 4 * tig + e] = __int2half_rn(qi[4 * h + e]);
      sum += qi[4 * h + e];
    }
  sum += __shfl_xor_sync(0xffffffffu, sum, 8);
  sum += __shfl_xor_sync(0xffffffffu, sum, 16);  // lanes s, s+8, ...: the sum of sub-block s
  if (lane == 0) dT[(int64_t)b * ldd + t] = d;
  if (bm && tig == 0) {
    const int lo = sum & 63, hi = (sum - lo) / 64;  // sum = 64 * hi + lo, 0 <= lo < 64
    __half* tile = reinterpret_cast<__half*>(bm + ((int64_t)(t / kQ4Toks) * nb + b) * 2048);
    const int tt = t % kQ4Toks;
    tile[plain_off(tt, 0) / 2 + s] = __int2half_rn(lo);
    tile[plain_off(tt, 1) / 2 + s] = __int2half_rn(hi);
  }
}

// Device-layout Q4_K / Q5_K rows -> the f16 operand A (row-major) and the
// min (and, Q5_K, centring) operand tiles per 128 rows and block: one
// thread per 16-byte quant chunk, the arithmetic in expand_qk_chunk
// (wide_expand.cuh).
template <bool kQ5>
__global__ void wide_expand_q4k_kernel(const uint8_t* __restrict__ w, int64_t w_row_bytes, int rows, int cols,
                                       __half* __restrict__ out, uint8_t* __restrict__ am,
                                       uint8_t* __restrict__ ac) {
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nb = cols / 256;
  const int64_t r = id / (nb * 8);
  if (r >= rows) return;
  const int b = (int)(id / 8 % nb), c = (int)(id & 7), tig = c >> 1;
  const uint8_t* blk = w + r * w_row_bytes + (int64_t)b * (kQ5 ? 176 : 144);
  const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(blk + (kQ5 ? 48 : 16) + c * 16));
  uint2 qh = make_uint2(0u, 0u);
  if constexpr (kQ5) qh = __ldg(reinterpret_cast<const uint2*>(blk + 16 + tig * 8));
  const int64_t tile = ((r / 128) * nb + b) * 4096;
  expand_qk_chunk<kQ5>(hdr, v, qh, c, b, out + r * cols, reinterpret_cast<__half*>(am + tile),
                       kQ5 ? reinterpret_cast<__half*>(ac + tile) : nullptr, (int)(r % 128));
}

// ----------------------------------------------------------------- Q6_K
// Q6_K weights x Q8_K input rows, bitwise the per-block device order:
//     isum = sum_s sc[s] * sum_{e in s} (q_e - 32) x_e   (16-element s, int8 sc)
//     acc  = fmaf(d_x * d_w, (float)isum, acc)
// sc * (q - 32) reaches 4096, not exact in f16, so the scale is split,
// sc = 16 * sh + sl (sl = sc & 15, sh = sc >> 4), into two operands
// A_lo = sl * (q - 32) (|.| <= 480) and A_hi = sh * (q - 32) (|.| <= 256),
// each with its own TMEM accumulator over the whole block (at most
// 256 * 480 * 128 < 2^24, exact); (float)isum = fmaf(16, hi, lo), one
// rounding of the exact integer.  Tiles: 128 weight rows x 128 input rows,
// a quarter block (64 K elements) per stage, two blocks in TMEM.
constexpr int kQ6Atom = 128 * 128;
constexpr int kQ6StageBytes = 3 * kQ6Atom;  // A_lo, A_hi, B
constexpr int kQ6Stages = 4;
constexpr int kQ6Side = 4, kQ6SideBytes = 2560, kQ6OffT = 512;  // input-row d (128 f32), then the d tail box
constexpr int kQ6SmemBytes = kQ6Stages * kQ6StageBytes + kQ6Side * kQ6SideBytes + 1024;

__global__ void __launch_bounds__(kBoundThreads, 1)
    wide_q6k_kernel(const __grid_constant__ CUtensorMap tm_lo, const __grid_constant__ CUtensorMap tm_hi,
                    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_d,
                    const __grid_constant__ CUtensorMap tm_t, int tail_x0, int rows, int nb, int ntok,
                    float* __restrict__ y, int out_ld, int* timeout_flag, int test_skip) {
  __shared__ __align__(8) uint64_t full_op[kQ6Stages], empty_op[kQ6Stages];
  __shared__ __align__(8) uint64_t full_side[kQ6Side], empty_side[kQ6Side];
  __shared__ __align__(8) uint64_t tfull[2], tempty[2], drained;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (su32(smem_raw) & 1023)) & 1023);
  uint8_t* side = smem + kQ6Stages * kQ6StageBytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * 128, row0 = blockIdx.y * 128;
  const int nst = nb * 4;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQ6Stages; s++) {
      bar_init(&full_op[s], 1);
      bar_init(&empty_op[s], 1);
    }
    for (int e = 0; e < kQ6Side; e++) {
      bar_init(&full_side[e], 1);
      bar_init(&empty_side[e], kEpiWarps);
    }
    for (int j = 0; j < 2; j++) {
      bar_init(&tfull[j], 1);
      bar_init(&tempty[j], kEpiWarps);
    }
    bar_init(&drained, 1);
    abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_s)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;
  const int lim = test_skip ? 256 : kWaitLimit;
  auto give_up = [&]() {
    atomicExch(timeout_flag, 1);
    *abort_v = 1;
  };

  if (warp < kEpiWarps) {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3, cb = 32 * (warp >> 2), r = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)cb;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; i++) acc[i] = 0.f;
    bool ok = true;
    for (int blk = 0; blk < nb && ok; blk++) {
      const int e = blk % kQ6Side, buf = blk & 1;
      const uint8_t* sd = side + e * kQ6SideBytes;
      if (!__all_sync(0xffffffffu, bar_wait(&full_side[e], (blk / kQ6Side) & 1, lim)) ||
          !__all_sync(0xffffffffu, bar_wait(&tfull[buf], (blk >> 1) & 1, lim))) {
        give_up();
        ok = false;
        break;
      }
      tc_after();
      const float* dx = reinterpret_cast<const float*>(sd) + cb;
      const float dw = __half2float(*reinterpret_cast<const __half*>(sd + kQ6OffT + r * 16 + 2 * (blk & 7)));
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t vl[16], vh[16];
        tmem_ld16(lane_base + (uint32_t)(buf * 256 + 16 * h), vl);
        tmem_ld16(lane_base + (uint32_t)(buf * 256 + 128 + 16 * h), vh);
        tmem_wait16(vl);
        tmem_wait16(vh);
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const float isum = __fmaf_rn(16.f, __uint_as_float(vh[i]), __uint_as_float(vl[i]));
          acc[16 * h + i] = __fmaf_rn(__fmul_rn(dx[16 * h + i], dw), isum, acc[16 * h + i]);
        }
      }
      tc_before();
      __syncwarp();
      if (lane == 0) {
        bar_arrive(&tempty[buf]);
        bar_arrive(&empty_side[e]);
      }
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (ok && !*abort_v) {
      const int row = row0 + r;
      if (row < rows) {
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int t = tok0 + cb + i;
          if (t < ntok) y[(int64_t)t * out_ld + row] = acc[i];
        }
      }
    }
  } else if (warp == kTmaWarp && lane == 0) {
    // ------------------------------------------------------ TMA producer
    int issued = 0, sides = 0;
    for (int it = 0; it < nst && !*abort_v; it++) {
      const int s = it % kQ6Stages, blk = it >> 2;
      if (it >= kQ6Stages && !bar_wait(&empty_op[s], ((it / kQ6Stages) + 1) & 1, lim)) { give_up(); break; }
      uint8_t* st = smem + s * kQ6StageBytes;
      bar_expect(&full_op[s], kQ6StageBytes);
      tma2d(st, &tm_lo, it * 64, row0, &full_op[s]);
      tma2d(st + kQ6Atom, &tm_hi, it * 64, row0, &full_op[s]);
      tma2d(st + 2 * kQ6Atom, &tm_x, it * 64, tok0, &full_op[s]);
      issued = it + 1;
      if ((it & 3) == 0) {
        const int e = blk % kQ6Side;
        if (blk >= kQ6Side && !bar_wait(&empty_side[e], ((blk / kQ6Side) + 1) & 1, lim)) { give_up(); break; }
        uint8_t* sd = side + e * kQ6SideBytes;
        bar_expect(&full_side[e], kQ6OffT + 2048);
        tma2d(sd, &tm_d, tok0, blk, &full_side[e]);
        tma2d(sd + kQ6OffT, &tm_t, tail_x0 + 16 * (blk >> 3), row0, &full_side[e]);
        sides = blk + 1;
      }
    }
    if (*abort_v) {
      for (int it = issued > kQ6Stages ? issued - kQ6Stages : 0; it < issued; it++)
        bar_wait(&full_op[it % kQ6Stages], (it / kQ6Stages) & 1, kDrainLimit);
      for (int b = sides > kQ6Side ? sides - kQ6Side : 0; b < sides; b++)
        bar_wait(&full_side[b % kQ6Side], (b / kQ6Side) & 1, kDrainLimit);
    }
  } else if (warp == kMmaWarp && lane == 0) {
    // ------------------------------------------------------- MMA issuer
    for (int it = 0; it < nst && !*abort_v; it++) {
      const int s = it % kQ6Stages, blk = it >> 2, quarter = it & 3, buf = blk & 1;
      if (!bar_wait(&full_op[s], (it / kQ6Stages) & 1, lim)) {
        give_up();
        break;
      }
      if (test_skip && blk == 0) continue;
      if (quarter == 0 && blk >= 2 && !bar_wait(&tempty[buf], ((blk >> 1) + 1) & 1, lim)) {
        give_up();
        break;
      }
      tc_after();
      const uint32_t a_lo = su32(smem + s * kQ6StageBytes), a_hi = a_lo + kQ6Atom, bx = a_lo + 2 * kQ6Atom;
      const uint32_t d0 = tmem + (uint32_t)(buf * 256);
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const uint32_t acc_in = (uint32_t)((quarter | kk) != 0);
        mma_f16(d0, sw128_desc(a_lo + 32 * kk), sw128_desc(bx + 32 * kk), acc_in);
        mma_f16(d0 + 128u, sw128_desc(a_hi + 32 * kk), sw128_desc(bx + 32 * kk), acc_in);
      }
      mma_commit(&empty_op[s]);
      if (quarter == 3) mma_commit(&tfull[buf]);
    }
    mma_commit(&drained);
    bar_wait(&drained, 0, kDrainLimit);
  }
  __syncwarp();
  tc_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Device-layout Q6_K rows -> the two scale-split operands A_lo = sl * (q - 32)
// and A_hi = sh * (q - 32) as f16 (row-major).  One thread per 16-element
// sub-block; the 6-bit values come from the device re-pack (q6k_dev_value),
// the int8 scales from the 16 bytes after the quants.
__global__ void wide_expand_q6k_kernel(const uint8_t* __restrict__ w, int64_t w_row_bytes, int rows, int cols,
                                       __half* __restrict__ lo, __half* __restrict__ hi) {
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nb = cols / 256;
  const int64_t r = id / (nb * 16);
  if (r >= rows) return;
  const int b = (int)(id / 16 % nb), sb = (int)(id & 15);
  const uint8_t* blk = w + r * w_row_bytes + (int64_t)b * 208;
  const int sc = (int)(int8_t)blk[192 + sb];
  const int sh = sc >> 4, sl = sc & 15;  // sc = 16 * sh + sl
  __half vl[16], vh[16];
#pragma unroll
  for (int e = 0; e < 16; e++) {
    const int v = q6k_dev_value(blk, 16 * sb + e) - 32;
    vl[e] = __int2half_rn(sl * v);
    vh[e] = __int2half_rn(sh * v);
  }
  const int64_t k = r * cols + (int64_t)b * 256 + 16 * sb;
  uint4* dl = reinterpret_cast<uint4*>(lo + k);
  uint4* dh = reinterpret_cast<uint4*>(hi + k);
  dl[0] = *reinterpret_cast<const uint4*>(&vl[0]);
  dl[1] = *reinterpret_cast<const uint4*>(&vl[8]);
  dh[0] = *reinterpret_cast<const uint4*>(&vh[0]);
  dh[1] = *reinterpret_cast<const uint4*>(&vh[8]);
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool encode2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t stride_bytes, uint32_t box_in, uint32_t box_out, CUtensorMapSwizzle sw) {
  auto fn = encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_in, box_out};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int wide_ldd(int ntok) { return (ntok + 3) & ~3; }

int* wide_timeout_flag() {
  static int* ptr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_wide_timeout) == cudaSuccess) ptr[dev] = static_cast<int*>(p);
  }
  return ptr[dev];
}

cudaError_t wide_q80_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, __half* qx, float* dT, __half* wx,
                             cudaStream_t st) {
  if (cols % kStageK || ntok < 1 || ntok > 65535 || rows < 1 || rows > INT32_MAX || ((uintptr_t)w & 15) ||
      ((uintptr_t)qx & 15) || ((uintptr_t)dT & 15) || ((uintptr_t)wx & 15) || w_row_bytes % 16)
    return cudaErrorInvalidValue;
  const int nb = (int)(cols / 32), ldd = wide_ldd(ntok);
  wide_act_kernel<<<dim3((unsigned)((nb + 7) / 8), (unsigned)ntok), 256, 0, st>>>(x, ldx, (int)cols, qx, dT, ldd);
  const int64_t chunks = rows * (cols / 128) * 8;
  wide_expand_q80_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(w, w_row_bytes, (int)rows, (int)cols, wx);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  alignas(64) CUtensorMap mw, mx, md, ms;
  if (!encode2d(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wx, (uint64_t)cols, (uint64_t)rows, (uint64_t)cols * 2, 64,
                kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)w_row_bytes, (uint64_t)rows, (uint64_t)w_row_bytes,
                16, kRows, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qx, (uint64_t)cols, (uint64_t)ntok, (uint64_t)cols * 2, 64,
                kToks, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dT, (uint64_t)ntok, (uint64_t)nb, (uint64_t)ldd * 4, kToks, 4,
                CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool attr[64] = {};  // the shared-memory opt-in is per device
  static std::mutex mu;
  e = once_per_device(attr, mu, [] {
    return cudaFuncSetAttribute(wide_q80_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  if (e != cudaSuccess) return e;
  int* flag = wide_timeout_flag();
  if (!flag) return cudaErrorInvalidDevice;
  static const int test_skip = getenv("IQ_WIDE_TEST_TIMEOUT") ? 1 : 0;
  const dim3 grid((unsigned)((ntok + kToks - 1) / kToks), (unsigned)((rows + kRows - 1) / kRows));
  wide_q80_kernel<<<grid, kThreads, kSmemBytes, st>>>(mw, mx, md, ms, nb * 32, (int)rows, nb, ntok, y, out_ld, flag,
                                                      test_skip);
  return cudaGetLastError();
}

template <bool kQ5>
cudaError_t wide_qk_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                            int ldx, int ntok, float* y, int out_ld, const WideQ4kScratch& sc, cudaStream_t st) {
  if (cols % 256 || ntok < 1 || ntok > 65535 || rows < 1 || rows > INT32_MAX || ((uintptr_t)w & 15) ||
      w_row_bytes % 16 || (kQ5 && !sc.ac))
    return cudaErrorInvalidValue;
  const int nb = (int)(cols / 256), ldd = wide_ldd(ntok);
  const int ttiles = (ntok + kQ4Toks - 1) / kQ4Toks, rtiles = (int)((rows + 127) / 128);
  cudaError_t e = cudaMemsetAsync(sc.bm, 0, (size_t)ttiles * nb * 2048, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(sc.am, 0, (size_t)rtiles * nb * 4096, st);
  if (e == cudaSuccess && kQ5) e = cudaMemsetAsync(sc.ac, 0, (size_t)rtiles * nb * 4096, st);
  if (e != cudaSuccess) return e;
  wide_act_q8k_kernel<<<dim3((unsigned)((nb + 7) / 8), (unsigned)ntok), 256, 0, st>>>(x, ldx, (int)cols, sc.qx,
                                                                                       sc.dT, ldd, sc.bm);
  const int64_t chunks = rows * nb * 8;
  wide_expand_q4k_kernel<kQ5><<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(w, w_row_bytes, (int)rows,
                                                                                (int)cols, sc.wx, sc.am, sc.ac);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  alignas(64) CUtensorMap mw, mx, md, mh;
  if (!encode2d(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc.wx, (uint64_t)cols, (uint64_t)rows, (uint64_t)cols * 2, 64,
                128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc.qx, (uint64_t)cols, (uint64_t)ntok, (uint64_t)cols * 2, 64,
                kQ4Toks, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sc.dT, (uint64_t)ntok, (uint64_t)nb, (uint64_t)ldd * 4,
                kQ4Toks, 1, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode2d(&mh, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)w_row_bytes, (uint64_t)rows, (uint64_t)w_row_bytes,
                16, 128, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool attr[64] = {};  // the shared-memory opt-in is per device
  static std::mutex mu;
  constexpr int kSmem = kQ5 ? kQ5SmemBytes : kQ4SmemBytes;
  e = once_per_device(attr, mu, [] {
    return cudaFuncSetAttribute(wide_q4k_kernel<kQ5>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (e != cudaSuccess) return e;
  int* flag = wide_timeout_flag();
  if (!flag) return cudaErrorInvalidDevice;
  static const int test_skip = getenv("IQ_WIDE_TEST_TIMEOUT") ? 1 : 0;
  const dim3 grid((unsigned)ttiles, (unsigned)rtiles);
  wide_q4k_kernel<kQ5><<<grid, kThreads, kSmem, st>>>(mw, mx, md, mh, sc.am, sc.bm, sc.ac, (int)rows, nb, ntok, y,
                                                       out_ld, flag, test_skip);
  return cudaGetLastError();
}

cudaError_t wide_q4k_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, const WideQ4kScratch& sc, cudaStream_t st) {
  return wide_qk_forward<false>(w, rows, cols, w_row_bytes, x, ldx, ntok, y, out_ld, sc, st);
}

cudaError_t wide_q5k_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, const WideQ4kScratch& sc, cudaStream_t st) {
  return wide_qk_forward<true>(w, rows, cols, w_row_bytes, x, ldx, ntok, y, out_ld, sc, st);
}

size_t wide_q4k_scratch_bytes(int64_t rows, int64_t cols, int ntok, WideQ4kScratch* sc, uint8_t* base, bool q5) {
  const int nb = (int)(cols / 256);
  const int ttiles = (ntok + kQ4Toks - 1) / kQ4Toks, rtiles = (int)((rows + 127) / 128);
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t o = off;
    off += (n + 255) & ~(size_t)255;
    return base ? base + o : nullptr;
  };
  uint8_t* qx = take((size_t)ntok * cols * 2);
  uint8_t* dT = take((size_t)nb * wide_ldd(ntok) * 4);
  uint8_t* bm = take((size_t)ttiles * nb * 2048);
  uint8_t* wx = take((size_t)rows * cols * 2);
  uint8_t* am = take((size_t)rtiles * nb * 4096);
  uint8_t* ac = q5 ? take((size_t)rtiles * nb * 4096) : nullptr;
  if (sc) {
    sc->qx = reinterpret_cast<__half*>(qx);
    sc->dT = reinterpret_cast<float*>(dT);
    sc->bm = bm;
    sc->wx = reinterpret_cast<__half*>(wx);
    sc->am = am;
    sc->ac = ac;
  }
  return off;
}

// Q5_K takes the Q4_K kernel's instance with the centred operand; it is
// off unless IQ_WIDE_Q5K is set, until its bitwise test has passed on a
// B200 (tests/test_wide_gpu.py runs it under that variable).
bool wide_q5k_enabled() {
  static const bool on = getenv("IQ_WIDE_Q5K") != nullptr;
  return on;
}

size_t wide_q6k_scratch_bytes(int64_t rows, int64_t cols, int ntok, WideQ6kScratch* sc, uint8_t* base) {
  const int nb = (int)(cols / 256);
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t o = off;
    off += (n + 255) & ~(size_t)255;
    return base ? base + o : nullptr;
  };
  uint8_t* qx = take((size_t)ntok * cols * 2);
  uint8_t* dT = take((size_t)nb * wide_ldd(ntok) * 4);
  uint8_t* lo = take((size_t)rows * cols * 2);
  uint8_t* hi = take((size_t)rows * cols * 2);
  if (sc) {
    sc->qx = reinterpret_cast<__half*>(qx);
    sc->dT = reinterpret_cast<float*>(dT);
    sc->lo = reinterpret_cast<__half*>(lo);
    sc->hi = reinterpret_cast<__half*>(hi);
  }
  return off;
}

cudaError_t wide_q6k_forward(const uint8_t* w, int64_t rows, int64_t cols, int64_t w_row_bytes, const float* x,
                             int ldx, int ntok, float* y, int out_ld, const WideQ6kScratch& sc, cudaStream_t st) {
  if (cols % 256 || ntok < 1 || ntok > 65535 || rows < 1 || rows > INT32_MAX || ((uintptr_t)w & 15) ||
      w_row_bytes % 16)
    return cudaErrorInvalidValue;
  const int nb = (int)(cols / 256), ldd = wide_ldd(ntok);
  wide_act_q8k_kernel<<<dim3((unsigned)((nb + 7) / 8), (unsigned)ntok), 256, 0, st>>>(x, ldx, (int)cols, sc.qx,
                                                                                       sc.dT, ldd, nullptr);
  const int64_t subs = rows * nb * 16;
  wide_expand_q6k_kernel<<<(unsigned)((subs + 255) / 256), 256, 0, st>>>(w, w_row_bytes, (int)rows, (int)cols, sc.lo,
                                                                         sc.hi);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  alignas(64) CUtensorMap mlo, mhi, mx, md, mt;
  if (!encode2d(&mlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc.lo, (uint64_t)cols, (uint64_t)rows, (uint64_t)cols * 2, 64,
                128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&mhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc.hi, (uint64_t)cols, (uint64_t)rows, (uint64_t)cols * 2, 64,
                128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sc.qx, (uint64_t)cols, (uint64_t)ntok, (uint64_t)cols * 2, 64,
                128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode2d(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sc.dT, (uint64_t)ntok, (uint64_t)nb, (uint64_t)ldd * 4, 128, 1,
                CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode2d(&mt, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)w_row_bytes, (uint64_t)rows, (uint64_t)w_row_bytes,
                16, 128, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  static bool attr[64] = {};  // the shared-memory opt-in is per device
  static std::mutex mu;
  e = once_per_device(attr, mu, [] {
    return cudaFuncSetAttribute(wide_q6k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQ6SmemBytes);
  });
  if (e != cudaSuccess) return e;
  int* flag = wide_timeout_flag();
  if (!flag) return cudaErrorInvalidDevice;
  static const int test_skip = getenv("IQ_WIDE_TEST_TIMEOUT") ? 1 : 0;
  const dim3 grid((unsigned)((ntok + 127) / 128), (unsigned)((rows + 127) / 128));
  wide_q6k_kernel<<<grid, kThreads, kQ6SmemBytes, st>>>(mlo, mhi, mx, md, mt, nb * 208, (int)rows, nb, ntok, y,
                                                        out_ld, flag, test_skip);
  return cudaGetLastError();
}

}  // namespace iq
