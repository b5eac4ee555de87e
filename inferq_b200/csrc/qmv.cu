// qmv.cu -- skinny quantized GEMV kernels (see qmv.cuh).
//
// Persistent CTAs walk the launch's tiles (tile = blockIdx.x + i*gridDim.x).
// Inside a tile, warp w owns 16 weight rows and one chunk of their blocks
// (units); its units form one stream across tiles and jobs.  Each warp keeps
// the next `depth` units of its stream in flight in a ring of shared-memory
// slots: one 2-D TMA load (tensor map over the weight tensor, box = one unit
// x 16 rows) per unit, completing on the slot's mbarrier.  The warp waits for
// a slot, copies the unit's fragments to registers, computes, then refills
// the slot with the unit `depth` ahead.  Activations are staged into shared memory
// once per change of input rows, not once per tile.
#include <algorithm>
#include <type_traits>
#include <mutex>
#include <cstdlib>
#include <climits>
#include <cstring>
#include <cudaTypedefs.h>
#include "qmv.cuh"
#include "layout.cuh"
#include "devfns.cuh"
#include "api_util.h"


namespace iq {
namespace {

struct Frag {  // per-thread accumulators for rows (gid, gid+8) x cols (2tig, 2tig+1)
  float acc[4];
  float accm[4];
};

__device__ __forceinline__ uint32_t w32(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

struct ActCols {  // the two C-fragment columns of this thread (shared memory)
  const uint8_t* c[2];
};

// Raw weight words of one block for rows (gid, gid+8), any dtype.
struct WRegs {
  uint4 r[8];
  uint32_t e;
};

__device__ __forceinline__ void load_b_words(uint4 (&bw)[4], const uint8_t* bact, int b, int tig) {
  if (bact) {
#pragma unroll
    for (int i = 0; i < 4; i++)
      bw[i] = *reinterpret_cast<const uint4*>(bact + (int64_t)b * 256 + tig * 64 + ((i ^ tig) & 3) * 16);
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) bw[i] = make_uint4(0, 0, 0, 0);
  }
}

// ------------------------------------------------------------------ slots
// A slot holds one unit of a warp's 16 rows as the TMA box lands: row r's
// unit bytes at r * unit_bytes, then (Q6_K / Q8_0) the 16-byte piece of each
// row's f16 scale tail that covers the unit, at 16 * unit_bytes + 16 r.
constexpr int kSlotBytes = 16 * 208 + 16 * 16;
static_assert(kSlotBytes % 128 == 0, "TMA destinations stay 128-byte aligned");

__device__ __forceinline__ int unit_bytes(int dt) {
  return dt == Q4_K ? 144 : dt == Q5_K ? 176 : dt == Q6_K ? 208 : 128;
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// The words of unit b for rows (gid, gid+8) from a filled slot.
__device__ __forceinline__ void load_slot(int dt, const uint8_t* slot, int b, int gid, int tig, WRegs& r) {
  switch (dt) {
    case Q4_K:
    case Q5_K: {
      const int BB = dt == Q4_K ? 144 : 176, QS = dt == Q4_K ? 16 : 48;
      const uint8_t* ba = slot + gid * BB;
      const uint8_t* bb = slot + (gid + 8) * BB;
      r.r[0] = lds128(ba);
      r.r[1] = lds128(bb);
      r.r[2] = lds128(ba + QS + tig * 32);
      r.r[3] = lds128(ba + QS + tig * 32 + 16);
      r.r[4] = lds128(bb + QS + tig * 32);
      r.r[5] = lds128(bb + QS + tig * 32 + 16);
      if (dt == Q5_K) {
        const uint2 x = *reinterpret_cast<const uint2*>(ba + 16 + tig * 8);
        const uint2 y = *reinterpret_cast<const uint2*>(bb + 16 + tig * 8);
        r.r[6] = make_uint4(x.x, x.y, y.x, y.y);
      }
    } break;
    case Q6_K: {
      const uint8_t* ba = slot + gid * 208;
      const uint8_t* bb = slot + (gid + 8) * 208;
      r.r[0] = lds128(ba + tig * 48);
      r.r[1] = lds128(ba + tig * 48 + 16);
      r.r[2] = lds128(ba + tig * 48 + 32);
      r.r[3] = lds128(bb + tig * 48);
      r.r[4] = lds128(bb + tig * 48 + 16);
      r.r[5] = lds128(bb + tig * 48 + 32);
      r.r[6] = lds128(ba + 192);
      r.r[7] = lds128(bb + 192);
      const uint8_t* tail = slot + 16 * 208 + 2 * (b & 7);
      const uint32_t da = *reinterpret_cast<const uint16_t*>(tail + gid * 16);
      const uint32_t db = *reinterpret_cast<const uint16_t*>(tail + (gid + 8) * 16);
      r.e = da | (db << 16);
    } break;
    default: {  // Q8_0: b indexes groups of four blocks
      const uint8_t* ba = slot + gid * 128;
      const uint8_t* bb = slot + (gid + 8) * 128;
      r.r[0] = lds128(ba + tig * 32);
      r.r[1] = lds128(ba + tig * 32 + 16);
      r.r[2] = lds128(bb + tig * 32);
      r.r[3] = lds128(bb + tig * 32 + 16);
      const uint8_t* tail = slot + 16 * 128 + 8 * (b & 1);
      const uint2 x = *reinterpret_cast<const uint2*>(tail + gid * 16);
      const uint2 y = *reinterpret_cast<const uint2*>(tail + (gid + 8) * 16);
      r.r[4] = make_uint4(x.x, x.y, y.x, y.y);
    } break;
  }
}

// -------------------------------------------------------------- mbarriers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Bounded wait for the phase of the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int limit = 1 << 20) {
  const uint32_t a = smem_u32(bar);
  for (int i = 0; i < limit; i++) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
// 2-D TMA tile load (this GPU's memory, no multicast) into this CTA's shared
// memory, completing on `bar`; weights are read once per pass (evict-first).
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// ---------------------------------------------------------------- compute
// The eight 6-bit scales and mins of a Q4_K/Q5_K header (words w0..w2 =
// bytes 0..11 of the reference's packed scales, src/qgemm.rs:153-167) as
// four words of bytes: sc0-3, sc4-7, mn0-3, mn4-7.
__device__ __forceinline__ void k_scale_bytes(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t& s_lo,
                                              uint32_t& s_hi, uint32_t& m_lo, uint32_t& m_hi) {
  s_lo = w0 & 0x3F3F3F3Fu;
  m_lo = w1 & 0x3F3F3F3Fu;
  s_hi = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
  m_hi = ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
}
__device__ __forceinline__ int byte_of(uint32_t w, int i) { return (int)__byte_perm(w, 0u, 0x4440u + i); }

// Q4_K / Q5_K: 8 sub-blocks of 32, u8 x s8 MMA (k32); mins term separately.
// Q4_K's odd sub-blocks use the high nibble in place (16q): their scaled sums
// are multiples of 16 and are folded back with one exact shift.
template <int DT>
__device__ __forceinline__ void compute_q45(const WRegs& r, const uint8_t* bact, ActCols ac, int nb, int b, int tig,
                                            Frag& f) {
  uint4 bw[4];
  load_b_words(bw, bact, b, tig);
  const uint4 ha = r.r[0], hb = r.r[1];
  uint32_t sAl, sAh, mAl, mAh, sBl, sBh, mBl, mBh;
  k_scale_bytes(ha.y, ha.z, ha.w, sAl, sAh, mAl, mAh);
  k_scale_bytes(hb.y, hb.z, hb.w, sBl, sBh, mBl, mBh);
  int isum[4] = {0, 0, 0, 0}, iodd[4] = {0, 0, 0, 0};
#pragma unroll
  for (int s = 0; s < 8; s++) {
    const int j = s / 2, hi = s & 1;
    const uint4& qa = j < 2 ? r.r[2] : r.r[3];
    const uint4& qb = j < 2 ? r.r[4] : r.r[5];
    const uint32_t mask = (DT == Q4_K && hi) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
    const int sh = DT == Q4_K ? 0 : 4 * hi;
    uint32_t a0 = (w32(qa, (j % 2) * 2) >> sh) & mask;
    uint32_t a2 = (w32(qa, (j % 2) * 2 + 1) >> sh) & mask;
    uint32_t a1 = (w32(qb, (j % 2) * 2) >> sh) & mask;
    uint32_t a3 = (w32(qb, (j % 2) * 2 + 1) >> sh) & mask;
    if (DT == Q5_K) {
      a0 |= ((r.r[6].x >> s) & 0x01010101u) << 4;
      a2 |= ((r.r[6].y >> s) & 0x01010101u) << 4;
      a1 |= ((r.r[6].z >> s) & 0x01010101u) << 4;
      a3 |= ((r.r[6].w >> s) & 0x01010101u) << 4;
    }
    int p[4] = {0, 0, 0, 0};
    mma_u8s8_k32(p, a0, a1, a2, a3, w32(bw[s / 2], (s % 2) * 2), w32(bw[s / 2], (s % 2) * 2 + 1));
    const int scA = byte_of(s < 4 ? sAl : sAh, s % 4), scB = byte_of(s < 4 ? sBl : sBh, s % 4);
    int* acc = (DT == Q4_K && hi) ? iodd : isum;
    acc[0] += scA * p[0];
    acc[1] += scA * p[1];
    acc[2] += scB * p[2];
    acc[3] += scB * p[3];
  }
  if (DT == Q4_K) {
#pragma unroll
    for (int i = 0; i < 4; i++) isum[i] += iodd[i] >> 4;
  }
  const float wdA = h2f(ha.x & 0xffff), wdminA = h2f(ha.x >> 16);
  const float wdB = h2f(hb.x & 0xffff), wdminB = h2f(hb.x >> 16);
#pragma unroll
  for (int c = 0; c < 2; c++) {
    float yd = 0.f;
    int msA = 0, msB = 0;
    if (ac.c[c]) {
      yd = *reinterpret_cast<const float*>(ac.c[c] + (int64_t)nb * 256 + b * 4);
      // the eight 32-element activation sums, as 16-bit pairs
      const uint4 bs = *reinterpret_cast<const uint4*>(ac.c[c] + q8k_bs_offset(nb) + b * 16);
      msA = __dp2a_lo((int)bs.x, (int)mAl, msA);
      msA = __dp2a_hi((int)bs.y, (int)mAl, msA);
      msA = __dp2a_lo((int)bs.z, (int)mAh, msA);
      msA = __dp2a_hi((int)bs.w, (int)mAh, msA);
      msB = __dp2a_lo((int)bs.x, (int)mBl, msB);
      msB = __dp2a_hi((int)bs.y, (int)mBl, msB);
      msB = __dp2a_lo((int)bs.z, (int)mBh, msB);
      msB = __dp2a_hi((int)bs.w, (int)mBh, msB);
    }
    f.acc[c] = fmaf(__fmul_rn(yd, wdA), __int2float_rn(isum[c]), f.acc[c]);
    f.accm[c] = fmaf(__fmul_rn(yd, wdminA), __int2float_rn(msA), f.accm[c]);
    f.acc[2 + c] = fmaf(__fmul_rn(yd, wdB), __int2float_rn(isum[2 + c]), f.acc[2 + c]);
    f.accm[2 + c] = fmaf(__fmul_rn(yd, wdminB), __int2float_rn(msB), f.accm[2 + c]);
  }
}

// Q6_K: 16 sub-blocks of 16, A = 4*(q-32) as s8 (k16 MMA).  Words j = 0..2
// of a set carry 4q in their top six bits (A = word & 0xFC.. ^ 0x80..); the
// fourth sub-block of the set is rebuilt from the three low bit pairs.
__device__ __forceinline__ uint32_t q6_a3(uint32_t w0, uint32_t w1, uint32_t w2) {
  return ((w0 & 0x03030303u) << 2) + ((w1 & 0x03030303u) << 4) + (((w2 & 0x03030303u) ^ 0x02020202u) << 6);
}

__device__ __forceinline__ void compute_q6(const WRegs& r, const uint8_t* bact, ActCols ac, int nb, int b, int tig,
                                           Frag& f) {
  uint4 bw[4];
  load_b_words(bw, bact, b, tig);
  const uint32_t WA[12] = {r.r[0].x, r.r[0].y, r.r[0].z, r.r[0].w, r.r[1].x, r.r[1].y,
                           r.r[1].z, r.r[1].w, r.r[2].x, r.r[2].y, r.r[2].z, r.r[2].w};
  const uint32_t WB[12] = {r.r[3].x, r.r[3].y, r.r[3].z, r.r[3].w, r.r[4].x, r.r[4].y,
                           r.r[4].z, r.r[4].w, r.r[5].x, r.r[5].y, r.r[5].z, r.r[5].w};
  const uint32_t SA[4] = {r.r[6].x, r.r[6].y, r.r[6].z, r.r[6].w};
  const uint32_t SB[4] = {r.r[7].x, r.r[7].y, r.r[7].z, r.r[7].w};
  int isum[4] = {0, 0, 0, 0};
#pragma unroll
  for (int s16 = 0; s16 < 16; s16++) {
    const int g = s16 / 4, j = s16 % 4;
    uint32_t a0, a1;
    if (j < 3) {
      a0 = (WA[3 * g + j] & 0xFCFCFCFCu) ^ 0x80808080u;
      a1 = (WB[3 * g + j] & 0xFCFCFCFCu) ^ 0x80808080u;
    } else {
      a0 = q6_a3(WA[3 * g], WA[3 * g + 1], WA[3 * g + 2]);
      a1 = q6_a3(WB[3 * g], WB[3 * g + 1], WB[3 * g + 2]);
    }
    int p[4] = {0, 0, 0, 0};
    mma_s8s8_k16(p, a0, a1, w32(bw[s16 / 4], s16 % 4));
    const int scA = (int)(int8_t)(SA[s16 / 4] >> (8 * (s16 % 4)));
    const int scB = (int)(int8_t)(SB[s16 / 4] >> (8 * (s16 % 4)));
    isum[0] += scA * p[0];
    isum[1] += scA * p[1];
    isum[2] += scB * p[2];
    isum[3] += scB * p[3];
  }
  const float wdA = h2f(r.e & 0xffff), wdB = h2f(r.e >> 16);
#pragma unroll
  for (int c = 0; c < 2; c++) {
    const float yd = ac.c[c] ? *reinterpret_cast<const float*>(ac.c[c] + (int64_t)nb * 256 + b * 4) : 0.f;
    f.acc[c] = fmaf(__fmul_rn(yd, wdA), __int2float_rn(isum[c] >> 2), f.acc[c]);
    f.acc[2 + c] = fmaf(__fmul_rn(yd, wdB), __int2float_rn(isum[2 + c] >> 2), f.acc[2 + c]);
  }
}

// Q8_0: a group of four 32-blocks, s8 x s8 MMA (k32), one FMA per block.
__device__ __forceinline__ void compute_q80(const WRegs& r, const uint8_t* bact, ActCols ac, int nb, int g, int tig,
                                            Frag& f) {
  uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
  if (bact) {
    x0 = *reinterpret_cast<const uint4*>(bact + (int64_t)g * 128 + tig * 32);
    x1 = *reinterpret_cast<const uint4*>(bact + (int64_t)g * 128 + tig * 32 + 16);
  }
  float4 yd[2];
#pragma unroll
  for (int c = 0; c < 2; c++)
    yd[c] = ac.c[c] ? *reinterpret_cast<const float4*>(ac.c[c] + (int64_t)nb * 32 + 16 * g)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int bb = 0; bb < 4; bb++) {
    const uint4& qa = bb < 2 ? r.r[0] : r.r[1];
    const uint4& qb = bb < 2 ? r.r[2] : r.r[3];
    const uint4& xx = bb < 2 ? x0 : x1;
    const int o = (bb % 2) * 2;
    int p[4] = {0, 0, 0, 0};
    mma_s8s8_k32(p, w32(qa, o), w32(qb, o), w32(qa, o + 1), w32(qb, o + 1), w32(xx, o), w32(xx, o + 1));
    const uint32_t hwa = bb < 2 ? r.r[4].x : r.r[4].y, hwb = bb < 2 ? r.r[4].z : r.r[4].w;
    const float wdA = h2f((bb & 1) ? hwa >> 16 : hwa & 0xffff);
    const float wdB = h2f((bb & 1) ? hwb >> 16 : hwb & 0xffff);
#pragma unroll
    for (int c = 0; c < 2; c++) {
      const float y = bb == 0 ? yd[c].x : bb == 1 ? yd[c].y : bb == 2 ? yd[c].z : yd[c].w;
      f.acc[c] = fmaf(__fmul_rn(wdA, y), __int2float_rn(p[c]), f.acc[c]);
      f.acc[2 + c] = fmaf(__fmul_rn(wdB, y), __int2float_rn(p[2 + c]), f.acc[2 + c]);
    }
  }
}

__device__ __forceinline__ void compute_block(int dt, const WRegs& r, const uint8_t* bact, ActCols ac, int nb, int b,
                                              int tig, Frag& f) {
  switch (dt) {
    case Q4_K: compute_q45<Q4_K>(r, bact, ac, nb, b, tig, f); break;
    case Q5_K: compute_q45<Q5_K>(r, bact, ac, nb, b, tig, f); break;
    case Q6_K: compute_q6(r, bact, ac, nb, b, tig, f); break;
    default: compute_q80(r, bact, ac, nb, b, tig, f); break;
  }
}

// ------------------------------------------------------------ tile geometry
struct WarpTile {
  int job;                 // job index (-1: no tile)
  int row0;                // first weight row of this warp's 16
  int u0, u1;              // block (unit) range of this warp's chunk
  int dt, nb, ks, chunk;
  int y0;                  // tensor-map row of row0
  const void *tm, *tmt;    // the job's tensor maps
  __device__ bool live() const { return job >= 0 && u0 < u1; }
};

constexpr int kSmemJobTable = 64;  // whole job records kept in shared memory
constexpr int kSmemJobs = kSmemJobTable * (int)(sizeof(QmvJob) / sizeof(int));  // tile offsets only

// The last job with tile0 <= tile.  `t0` is the shared-memory copy of the
// jobs' tile0 when the table fits, else null (read from global memory).
__device__ __forceinline__ int find_job(const QmvJob* jobs, const int* t0, int njobs, int tile) {
  int lo = 0, hi = njobs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    const int v = t0 ? t0[mid] : jobs[mid].tile0;
    if (v <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ WarpTile warp_tile(const QmvJob* jobs, const int* t0, int njobs, int total, int tile,
                                              int warp) {
  WarpTile w;
  w.job = -1;
  w.u0 = w.u1 = 0;
  if (tile >= total) return w;
  const int j = find_job(jobs, t0, njobs, tile);
  const QmvJob& jb = jobs[j];
  w.job = j;
  w.tm = jb.tmap;
  w.tmt = jb.tmap_tail;
  w.ks = jb.ksplit;
  w.dt = jb.dtype;
  w.nb = jb.cols / gguf_block_elems(w.dt);
  const int rt = warp / w.ks;
  w.chunk = warp % w.ks;
  w.row0 = (tile - jb.tile0) * qmv_rows_per_cta(w.ks) + rt * 16;
  w.y0 = jb.row_base + w.row0;
  if (w.row0 < jb.rows) {
    const int units = qmv_units(w.dt, jb.cols);
    w.u0 = w.chunk * units / w.ks;
    w.u1 = (w.chunk + 1) * units / w.ks;
  }
  return w;
}

__device__ __forceinline__ int act_used_bytes(int dt, int cols) {
  return (int)(dt == Q8_0 ? act_row_bytes_q80(cols) : act_row_bytes_q8k(cols));
}

__device__ int g_qmv_timeout;  // set when a slot wait gave up (not expected to happen)

// A warp's position in its stream of units.
struct StreamPos {
  int tile, b;
  WarpTile t;
};

__device__ __forceinline__ void stream_settle(const QmvJob* jobs, const int* t0, int njobs, int total, int warp,
                                              StreamPos& p) {
  while (p.tile < total && p.b >= p.t.u1) {
    p.tile += gridDim.x;
    if (p.tile >= total) break;
    p.t = warp_tile(jobs, t0, njobs, total, p.tile, warp);
    p.b = p.t.u0;
  }
}

// Lane 0: start the TMA load of unit p.b of the warp's 16 rows into `slot`.
__device__ __forceinline__ void issue_unit(const StreamPos& p, uint8_t* slot, uint64_t* bar, uint64_t pol) {
  const int dt = p.t.dt, ub = unit_bytes(dt);
  const bool tail = dt == Q6_K || dt == Q8_0;
  mbar_expect_tx(bar, 16 * ub + (tail ? 256 : 0));
  tma_load_2d(slot, p.t.tm, p.b * ub, p.t.y0, bar, pol);
  if (tail) {
    const int x = dt == Q6_K ? p.t.nb * 208 + 16 * (p.b >> 3) : p.t.nb * 32 + 16 * (p.b >> 1);
    tma_load_2d(slot + 16 * ub, p.t.tmt, x, p.t.y0, bar, pol);
  }
}

// Dynamic shared memory: [activation rows (act_bytes, rounded up to 128)]
// [kQmvWarps x depth slots of slot_bytes] (slot_bytes: the largest unit of the
// launch's dtypes, a multiple of 128 up to kSlotBytes).
__global__ void __launch_bounds__(kQmvThreads, 2) qmv_kernel(const QmvJob* jobs, int njobs,
                                                             const int* __restrict__ dyn_count, int total_hint,
                                                             int act_bytes, int depth, int slot_bytes,
                                                             int flags) {
  const bool test_skip = flags & 1;
  __shared__ float part[kQmvWarps][32][4];
  // the job table in shared memory when it is small (one parallel copy, no
  // dependent global reads later); otherwise just the jobs' tile offsets
  __shared__ union {
    QmvJob jobs[kSmemJobTable];
    int tile0[kSmemJobs];
  } tab;
  __shared__ __align__(8) uint64_t bars[kQmvWarps][kQmvMaxDepth];
  extern __shared__ __align__(128) uint8_t act_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  // TMA destinations: 128-byte aligned (the launch adds 128 bytes of slack)
  const uint32_t ring0 = (smem_u32(act_smem) + (uint32_t)act_bytes + 127u) & ~127u;
  uint8_t* ring = act_smem + (ring0 - smem_u32(act_smem)) + warp * depth * slot_bytes;
  uint64_t* wbars = bars[warp];
  if (lane == 0) {
    for (int i = 0; i < depth; i++) mbar_init(&wbars[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));

  if (dyn_count) {
    pdl_wait();
    njobs = *dyn_count;
  }
  if (njobs <= 0) {
    pdl_wait();
    return;
  }
  const int* t0 = nullptr;
  if (njobs <= kSmemJobTable) {
    constexpr int kWords = sizeof(QmvJob) / 16;
#pragma unroll 2
    for (int i = threadIdx.x; i < njobs * kWords; i += kQmvThreads)
      reinterpret_cast<uint4*>(tab.jobs)[i] = reinterpret_cast<const uint4*>(jobs)[i];
    __syncthreads();
    jobs = tab.jobs;
  } else if (njobs <= kSmemJobs) {
    for (int i = threadIdx.x; i < njobs; i += kQmvThreads) tab.tile0[i] = jobs[i].tile0;
    __syncthreads();
    t0 = tab.tile0;
  }
  int total = total_hint;
  if (total <= 0) {
    const QmvJob& last = jobs[njobs - 1];
    total = last.tile0 + (int)ceil_div(last.rows, qmv_rows_per_cta(last.ksplit));
  }

  // fill the ring before waiting on the previous kernel: weights do not depend on it
  StreamPos pp;
  pp.tile = blockIdx.x;
  pp.t = warp_tile(jobs, t0, njobs, total, pp.tile, warp);
  pp.b = pp.t.u0;
  stream_settle(jobs, t0, njobs, total, warp, pp);
  // test_skip (tests only): CTA 0's warp 0 never requests its first unit, so
  // its first slot wait must run out and take the timeout path below
  const bool skip_first = test_skip && blockIdx.x == 0 && warp == 0;
  const int wait_limit = test_skip ? 256 : 1 << 20;
  uint32_t issued = 0;
  for (int i = 0; i < depth && pp.tile < total; i++) {
    if (lane == 0 && !(skip_first && i == 0)) issue_unit(pp, ring + i * slot_bytes, &wbars[i], pol);
    issued++;
    pp.b++;
    stream_settle(jobs, t0, njobs, total, warp, pp);
  }
  pdl_wait();
  pdl_trigger();

  // staged activation key: every row of one activation buffer (or, for a
  // SwiGLU job, the job itself)
  const uint8_t* staged_act = nullptr;
  int staged_rows = -1, staged_stride = 0, staged_job = -1;
  uint32_t n = 0;  // units consumed by this warp
  uint32_t si = 0, phase = 0;  // its ring slot (n mod depth) and that slot's parity (n / depth mod 2)
  bool ok = true;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const WarpTile ct = warp_tile(jobs, t0, njobs, total, tile, warp);
    const QmvJob& jb = jobs[ct.job];
    const int nin = jb.n;
    const int used = act_used_bytes(jb.dtype, jb.cols);
    const bool swiglu = jb.act_mode == kActSwiGLU;
    if (swiglu && ct.job != staged_job) {
      // silu(g) * u of the job's input rows (g / (1 + exp(-g)), times u;
      // src/qwen/quantized_moe.rs:446), quantized as the activation row of the
      // job's matrix (Q8_K blocks of 256 or Q8_0 groups of 128 per warp);
      // staged as rows 0..n-1
      __syncthreads();  // no warp still reads the previous staging
      const float* gu = reinterpret_cast<const float*>(jb.act);
      const int gl = jb.act_row_bytes / 4, F = jb.cols;
      if (jb.dtype == Q8_0) {
        const int ng = F / 128;
        for (int i = warp; i < nin * ng; i += kQmvWarps) {
          const int c = i / ng, g = i % ng;
          const float* gr = gu + (int64_t)jb.rowmap[c] * gl;
          const int e0 = q80_lane_base(g, lane);
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float x = gr[e0 + e];
            v[e] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.f, exp_ref(-x))), gr[F + e0 + e]);
          }
          quant_q80_group_warp_v(v, act_smem + c * used, F / 32, g, lane);
        }
      } else {
        const int nbk = F / 256;
        for (int i = warp; i < nin * nbk; i += kQmvWarps) {
          const int c = i / nbk, b = i % nbk;
          const float* gr = gu + (int64_t)jb.rowmap[c] * gl;
          float g8[8], u8[8];
          ld_q8k_lane(gr, b, lane, g8);
          ld_q8k_lane(gr + F, b, lane, u8);
#pragma unroll
          for (int e = 0; e < 8; e++) g8[e] = __fmul_rn(__fdiv_rn(g8[e], __fadd_rn(1.f, exp_ref(-g8[e]))), u8[e]);
          quant_q8k_block_warp_v(g8, act_smem + c * used, nbk, b, lane);
        }
      }
      __syncthreads();
      staged_job = ct.job;
      staged_act = nullptr;
    } else if (!swiglu && (jb.act != staged_act || jb.act_nrows != staged_rows || used != staged_stride)) {
      __syncthreads();  // no warp still reads the previous staging
      const int words = used / 16;
#pragma unroll 4
      for (int i = threadIdx.x; i < jb.act_nrows * words; i += kQmvThreads) {
        const int r = i / words, w = i % words;
        reinterpret_cast<uint4*>(act_smem)[i] =
            *reinterpret_cast<const uint4*>(jb.act + (int64_t)r * jb.act_row_bytes + 16 * w);
      }
      __syncthreads();
      staged_act = jb.act;
      staged_rows = jb.act_nrows;
      staged_stride = used;
      staged_job = -1;
    }
    // staged row of input column i: rowmap[i], or i for a SwiGLU job
    auto srow = [&](int i) { return swiglu ? i : (int)jb.rowmap[i]; };
    const uint8_t* bact = gid < nin ? act_smem + srow(gid) * used : nullptr;
    ActCols ac;
    ac.c[0] = 2 * tig < nin ? act_smem + srow(2 * tig) * used : nullptr;
    ac.c[1] = 2 * tig + 1 < nin ? act_smem + srow(2 * tig + 1) * used : nullptr;

    Frag f;
#pragma unroll
    for (int i = 0; i < 4; i++) { f.acc[i] = 0.f; f.accm[i] = 0.f; }
    // the tile's units, with the dtype fixed per tile so each loop body holds
    // only its own dtype's unpack and arithmetic
    auto units = [&](auto dtc) {
      constexpr int DT = decltype(dtc)::value;
      for (int b = ct.u0; b < ct.u1; b++, n++) {
        uint8_t* slot = ring + si * slot_bytes;
        if (!mbar_wait(&wbars[si], phase, wait_limit)) {
          if (lane == 0) atomicExch(&g_qmv_timeout, 1);
          ok = false;
          // let this warp's other copies land (bounded) before it stops using the ring
          for (uint32_t j = n + 1; j < issued; j++) mbar_wait(&wbars[j % depth], (j / depth) & 1);
          break;
        }
        WRegs cur;
        load_slot(DT, slot, b, gid, tig, cur);
        compute_block(DT, cur, bact, ac, ct.nb, b, tig, f);
        // refill the slot once the unit's words have been used: every lane's
        // reads of it have completed before lane 0 hands it to the copy engine
        __syncwarp();
        if (pp.tile < total) {
          if (lane == 0) issue_unit(pp, slot, &wbars[si], pol);
          issued++;
          pp.b++;
          stream_settle(jobs, t0, njobs, total, warp, pp);
        }
        if (++si == (uint32_t)depth) {
          si = 0;
          phase ^= 1u;
        }
      }
    };
    if (ct.live() && ok) {
      switch (ct.dt) {
        case Q4_K: units(std::integral_constant<int, Q4_K>{}); break;
        case Q5_K: units(std::integral_constant<int, Q5_K>{}); break;
        case Q6_K: units(std::integral_constant<int, Q6_K>{}); break;
        default: units(std::integral_constant<int, Q8_0>{}); break;
      }
    }

    const bool has_min = jb.dtype == Q4_K || jb.dtype == Q5_K;
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; i++) y[i] = has_min ? __fsub_rn(f.acc[i], f.accm[i]) : f.acc[i];
    const int ks = jb.ksplit;
    bool store = ok && ct.row0 < jb.rows;
    if (ks > 1) {
      float(*pb)[32][4] = part;
#pragma unroll
      for (int i = 0; i < 4; i++) pb[warp][lane][i] = y[i];
      __syncthreads();
      store = store && ct.chunk == 0;
      if (store) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          float v = pb[warp][lane][i];
          for (int c = 1; c < ks; c++) v = __fadd_rn(v, pb[warp + c][lane][i]);
          y[i] = v;
        }
      }
      __syncthreads();  // part[] is free again before any later tile writes it
    }
    if (store) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int row = ct.row0 + gid + (i >= 2 ? 8 : 0);
        const int col = 2 * tig + (i & 1);
        if (row >= jb.rows || col >= nin) continue;
        const int64_t o = (int64_t)jb.outrow[col] * jb.out_ld + row;
        float v = y[i];
        if (jb.epi == kEpiResidual) v = __fadd_rn(jb.resid[o], v);
        jb.out[o] = v;
      }
    }
  }
}

}  // namespace

int* qmv_timeout_flag() {
  static int* ptr[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qmv_timeout) == cudaSuccess) ptr[dev] = static_cast<int*>(p);
  }
  return ptr[dev];
}

int qmv_persistent_ctas() {
  static int n[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lk(mu);
  if (!n[dev]) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = sms * 2;
  }
  return n[dev];
}

namespace {
// Dynamic shared memory per CTA: with two CTAs resident on an SM ([0]) and
// with one ([1]).  Per device: the opt-in attribute is set on each device
// the first time a GEMV launches there.
struct SmemLimits {
  int two = 0, one = 0;
};
// Limits of the current device, set up (with the opt-in attribute) the first
// time they are asked for there; zeros while the setup fails.
SmemLimits qmv_dyn_smem_limits() {
  static SmemLimits lims[64];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SmemLimits();
  std::lock_guard<std::mutex> lk(mu);
  SmemLimits& lim = lims[dev];
  if (!lim.one) {
    int per_sm = 0, optin = 0;
    cudaFuncAttributes fa = {};
    if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, qmv_kernel) != cudaSuccess)
      return SmemLimits();
    // each resident block also reserves 1 KB of shared memory for the system
    SmemLimits l;
    l.two = std::min(optin, per_sm / 2 - 1024) - (int)fa.sharedSizeBytes;
    l.one = optin - (int)fa.sharedSizeBytes;
    if (cudaFuncSetAttribute(qmv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, l.one) != cudaSuccess)
      return SmemLimits();
    lim = l;
  }
  return lim;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool encode_rows(CUtensorMap* m, const uint8_t* base, int64_t rows, int64_t row_bytes, uint32_t box_bytes) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {box_bytes, 16};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t qmv_tensor_maps(int dt, const uint8_t* base, int64_t rows, int64_t cols, DevBuf& maps) {
  if (dt != Q4_K && dt != Q5_K && dt != Q6_K && dt != Q8_0) return cudaErrorInvalidValue;
  const int64_t rb = dev_row_bytes(dt, (int)cols);
  const uint32_t ub = dt == Q4_K ? 144 : dt == Q5_K ? 176 : dt == Q6_K ? 208 : 128;
  if (((uintptr_t)base & 15) || rb % 16 || rows > INT32_MAX || rb > INT32_MAX) return cudaErrorInvalidValue;
  alignas(64) CUtensorMap h[2];
  memset(h, 0, sizeof h);
  if (!encode_rows(&h[0], base, rows, rb, ub)) return cudaErrorInvalidValue;
  if ((dt == Q6_K || dt == Q8_0) && !encode_rows(&h[1], base, rows, rb, 16)) return cudaErrorInvalidValue;
  cudaError_t e = maps.reserve(sizeof h);
  if (e != cudaSuccess) return e;
  return cudaMemcpy(maps.p, h, sizeof h, cudaMemcpyHostToDevice);
}

cudaError_t qmv_launch(const QmvJob* jobs, int njobs, const int* dyn_count, int ntiles, int smem_bytes,
                       cudaStream_t stream, bool pdl, int slot_bytes) {
  if (ntiles <= 0) return cudaSuccess;
  const SmemLimits lim = qmv_dyn_smem_limits();
  if (!lim.one) return cudaErrorInvalidValue;
  if (slot_bytes <= 0) slot_bytes = kSlotBytes;
  if (slot_bytes % 128 || slot_bytes > kSlotBytes) return cudaErrorInvalidValue;
  const int act = ((smem_bytes + 127) & ~127) + 128;  // + alignment slack of the ring
  const int ring_unit = kQmvWarps * slot_bytes;
  int depth = std::min(kQmvMaxDepth, (lim.two - act) / ring_unit);
  int ctas = qmv_persistent_ctas();
  if (depth < 2) {  // many activation rows: one CTA per SM
    depth = std::min(kQmvMaxDepth, (lim.one - act) / ring_unit);
    ctas /= 2;
  }
  if (depth < 2) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(ntiles, ctas));
  cfg.blockDim = dim3(kQmvThreads);
  cfg.dynamicSmemBytes = act + depth * ring_unit;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  // bit 0 (tests only): one first slot is never requested
  static const int flags = getenv("IQ_QMV_TEST_TIMEOUT") ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qmv_kernel, jobs, njobs, dyn_count, dyn_count ? 0 : ntiles, smem_bytes, depth,
                            slot_bytes, flags);
}

}  // namespace iq
