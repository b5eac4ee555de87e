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
#include "kernels.cuh"
#include "qmv.cuh"

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
        bar_wait(&full_op[it % kStages], (it / kStages) & 1, lim);
      for (int it = issued > kSide ? issued - kSide : 0; it < issued; it++)
        bar_wait(&full_side[it % kSide], (it / kSide) & 1, lim);
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
    bar_wait(&drained, 0, lim);
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
  if (first_on_device(attr)) {
    e = cudaFuncSetAttribute(wide_q80_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
  }
  int* flag = wide_timeout_flag();
  if (!flag) return cudaErrorInvalidDevice;
  static const int test_skip = getenv("IQ_WIDE_TEST_TIMEOUT") ? 1 : 0;
  const dim3 grid((unsigned)((ntok + kToks - 1) / kToks), (unsigned)((rows + kRows - 1) / kRows));
  wide_q80_kernel<<<grid, kThreads, kSmemBytes, st>>>(mw, mx, md, ms, nb * 32, (int)rows, nb, ntok, y, out_ld, flag,
                                                      test_skip);
  return cudaGetLastError();
}

}  // namespace iq
