// qmv.cu -- skinny quantized GEMV kernels (see qmv.cuh).
//
// Persistent CTAs walk the launch's tiles (tile = blockIdx.x + i*gridDim.x).
// Inside a tile, warp w owns 16 weight rows and one chunk of their blocks;
// its blocks form one stream across tiles, and the next block of that stream
// (possibly the first block of the next tile, possibly of another job) is
// always loaded while the current one is computed.  Activations are staged
// into shared memory once per change of input rows, not once per tile.
#include <algorithm>
#include "qmv.cuh"
#include "layout.cuh"
#include "devfns.cuh"


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
    for (int i = 0; i < 4; i++) bw[i] = *reinterpret_cast<const uint4*>(bact + (int64_t)b * 256 + tig * 64 + i * 16);
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) bw[i] = make_uint4(0, 0, 0, 0);
  }
}

// ------------------------------------------------------------------ loads
__device__ __forceinline__ void load_block(int dt, const uint8_t* wa, const uint8_t* wb, int nb, int b, int tig,
                                           WRegs& r) {
  switch (dt) {
    case Q4_K:
    case Q5_K: {
      const int BB = dt == Q4_K ? 144 : 176, QS = dt == Q4_K ? 16 : 48;
      const uint8_t* ba = wa + (int64_t)b * BB;
      const uint8_t* bb = wb + (int64_t)b * BB;
      r.r[0] = ld_stream(ba);
      r.r[1] = ld_stream(bb);
      r.r[2] = ld_stream(ba + QS + tig * 32);
      r.r[3] = ld_stream(ba + QS + tig * 32 + 16);
      r.r[4] = ld_stream(bb + QS + tig * 32);
      r.r[5] = ld_stream(bb + QS + tig * 32 + 16);
      if (dt == Q5_K) {
        const uint2 x = *reinterpret_cast<const uint2*>(ba + 16 + tig * 8);
        const uint2 y = *reinterpret_cast<const uint2*>(bb + 16 + tig * 8);
        r.r[6] = make_uint4(x.x, x.y, y.x, y.y);
      }
    } break;
    case Q6_K: {
      const uint8_t* ba = wa + (int64_t)b * 208;
      const uint8_t* bb = wb + (int64_t)b * 208;
      r.r[0] = ld_stream(ba + tig * 48);
      r.r[1] = ld_stream(ba + tig * 48 + 16);
      r.r[2] = ld_stream(ba + tig * 48 + 32);
      r.r[3] = ld_stream(bb + tig * 48);
      r.r[4] = ld_stream(bb + tig * 48 + 16);
      r.r[5] = ld_stream(bb + tig * 48 + 32);
      r.r[6] = ld_stream(ba + 192);
      r.r[7] = ld_stream(bb + 192);
      const uint32_t da = *reinterpret_cast<const uint16_t*>(wa + (int64_t)nb * 208 + 2 * b);
      const uint32_t db = *reinterpret_cast<const uint16_t*>(wb + (int64_t)nb * 208 + 2 * b);
      r.e = da | (db << 16);
    } break;
    default: {  // Q8_0: b indexes groups of four blocks
      r.r[0] = ld_stream(wa + (int64_t)b * 128 + tig * 32);
      r.r[1] = ld_stream(wa + (int64_t)b * 128 + tig * 32 + 16);
      r.r[2] = ld_stream(wb + (int64_t)b * 128 + tig * 32);
      r.r[3] = ld_stream(wb + (int64_t)b * 128 + tig * 32 + 16);
      const uint2 x = *reinterpret_cast<const uint2*>(wa + (int64_t)nb * 32 + 8 * b);
      const uint2 y = *reinterpret_cast<const uint2*>(wb + (int64_t)nb * 32 + 8 * b);
      r.r[4] = make_uint4(x.x, x.y, y.x, y.y);
    } break;
  }
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
  const uint8_t *wa, *wb;  // the rows (gid, gid+8), clamped
  int dt, nb, ks, chunk;
  __device__ bool live() const { return job >= 0 && u0 < u1; }
};

constexpr int kSmemJobs = 1152;  // job tile offsets kept in shared memory

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
                                              int warp, int gid) {
  WarpTile w;
  w.job = -1;
  w.u0 = w.u1 = 0;
  if (tile >= total) return w;
  const int j = find_job(jobs, t0, njobs, tile);
  const QmvJob& jb = jobs[j];
  w.job = j;
  w.ks = jb.ksplit;
  w.dt = jb.dtype;
  w.nb = jb.cols / gguf_block_elems(w.dt);
  const int rt = warp / w.ks;
  w.chunk = warp % w.ks;
  w.row0 = (tile - jb.tile0) * qmv_rows_per_cta(w.ks) + rt * 16;
  if (w.row0 < jb.rows) {
    const int units = qmv_units(w.dt, jb.cols);
    w.u0 = w.chunk * units / w.ks;
    w.u1 = (w.chunk + 1) * units / w.ks;
  }
  const int ra = min(w.row0 + gid, jb.rows - 1), rb = min(w.row0 + gid + 8, jb.rows - 1);
  w.wa = jb.w + (int64_t)ra * jb.w_row_bytes;
  w.wb = jb.w + (int64_t)rb * jb.w_row_bytes;
  return w;
}

// Build the launch's activation rows in shared memory from f32 inputs
// (every CTA does it; the inputs are a few KB per row and L2-resident).
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Four transformed inputs starting at element i (a multiple of 4) of row r.
__device__ __forceinline__ void pro_values(const QmvPrologue& p, const float* den, int r, int i, float* v) {
  const float4 xv = ld4(p.x + (int64_t)r * p.ldx + i);
  const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
  if (p.mode == kProRmsNorm) {
    const float4 wv = ld4(p.w + i);
    const float ws[4] = {wv.x, wv.y, wv.z, wv.w};
    const float d = den[r];
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = __fmul_rn(__fdiv_rn(xs[e], d), ws[e]);
  } else if (p.mode == kProGated) {
    const int h = i / p.dv;
    const float4 wv = ld4(p.w + (i - h * p.dv));
    const float4 zv = ld4(p.z + (int64_t)r * p.ldz + i);
    const float ws[4] = {wv.x, wv.y, wv.z, wv.w}, zs[4] = {zv.x, zv.y, zv.z, zv.w};
    const float d = den[r * p.heads + h];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float silu = __fdiv_rn(zs[e], __fadd_rn(1.f, expf(-zs[e])));
      v[e] = __fmul_rn(__fmul_rn(__fdiv_rn(xs[e], d), ws[e]), silu);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = xs[e];
  }
}

// Every CTA builds the launch's activation rows in shared memory from the f32
// inputs: the norm statistics first (one warp per row, or eight lanes per
// head), then one warp per Q8_K block / group of four Q8_0 blocks, two items
// in flight per warp.  All loads are 16-byte vectors; the inputs were written
// by the previous kernel and are read from L2.
__device__ __noinline__ void run_prologue(const QmvPrologue& p, uint8_t* smem) {
  __shared__ float den[kProMaxDen];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* r8k = smem;
  uint8_t* r80 = smem + (p.want8k ? p.rows * p.stride8k : 0);
  if (p.mode == kProRmsNorm) {
    for (int r = warp; r < p.rows; r += kQmvWarps) {
      const float* x = p.x + (int64_t)r * p.ldx;
      float ss = 0.f;
#pragma unroll 4
      for (int i = 4 * lane; i < p.cols; i += 128) {
        const float4 v = ld4(x + i);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0) den[r] = sqrtf(__fadd_rn(__fmul_rn(ss, p.inv_n), p.eps));
    }
  } else if (p.mode == kProGated) {
    const int sub = lane & 7;
    for (int q0 = warp * 4; q0 < p.rows * p.heads; q0 += 4 * kQmvWarps) {
      const int q = q0 + (lane >> 3);
      float ss = 0.f;
      if (q < p.rows * p.heads) {
        const int r = q / p.heads, h = q % p.heads;
        const float* o = p.x + (int64_t)r * p.ldx + h * p.dv;
#pragma unroll 4
        for (int i = 4 * sub; i < p.dv; i += 32) {
          const float4 v = ld4(o + i);
          ss = fmaf(v.x, v.x, ss);
          ss = fmaf(v.y, v.y, ss);
          ss = fmaf(v.z, v.z, ss);
          ss = fmaf(v.w, v.w, ss);
        }
      }
#pragma unroll
      for (int m = 4; m >= 1; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
      if (sub == 0 && q < p.rows * p.heads) den[q] = sqrtf(__fadd_rn(__fmul_rn(ss, p.inv_n), p.eps));
    }
  }
  __syncthreads();
  if (p.want8k) {
    const int nb = p.cols / 256, n = p.rows * nb;
    const int s = lane & 7, tig = lane >> 3;
    for (int it = warp; it < n; it += 2 * kQmvWarps) {
      const int it2 = it + kQmvWarps;
      const bool two = it2 < n;
      float va[8], vb[8];
      {
        const int r = it / nb, b = it % nb;
        pro_values(p, den, r, b * 256 + 32 * s + tig * 4, va);
        pro_values(p, den, r, b * 256 + 32 * s + 16 + tig * 4, va + 4);
      }
      if (two) {
        const int r = it2 / nb, b = it2 % nb;
        pro_values(p, den, r, b * 256 + 32 * s + tig * 4, vb);
        pro_values(p, den, r, b * 256 + 32 * s + 16 + tig * 4, vb + 4);
      }
      quant_q8k_block_warp_v(va, r8k + (it / nb) * p.stride8k, nb, it % nb, lane);
      if (two) quant_q8k_block_warp_v(vb, r8k + (it2 / nb) * p.stride8k, nb, it2 % nb, lane);
    }
  }
  if (p.want80) {
    const int nb = p.cols / 32, ng = nb / 4, n = p.rows * ng;
    for (int it = warp; it < n; it += 2 * kQmvWarps) {
      const int it2 = it + kQmvWarps;
      const bool two = it2 < n;
      float va[4], vb[4];
      pro_values(p, den, it / ng, q80_lane_base(it % ng, lane), va);
      if (two) pro_values(p, den, it2 / ng, q80_lane_base(it2 % ng, lane), vb);
      quant_q80_group_warp_v(va, r80 + (it / ng) * p.stride80, nb, it % ng, lane);
      if (two) quant_q80_group_warp_v(vb, r80 + (it2 / ng) * p.stride80, nb, it2 % ng, lane);
    }
  }
  if (p.xn_out && blockIdx.x == 0)
    for (int it = 4 * threadIdx.x; it < p.rows * p.cols; it += 4 * kQmvThreads) {
      const int r = it / p.cols, i = it % p.cols;
      float v[4];
      pro_values(p, den, r, i, v);
      *reinterpret_cast<float4*>(p.xn_out + (int64_t)r * p.ldxn + i) = make_float4(v[0], v[1], v[2], v[3]);
    }
  __syncthreads();
}

__device__ __forceinline__ int act_used_bytes(int dt, int cols) {
  return (int)(dt == Q8_0 ? act_row_bytes_q80(cols) : act_row_bytes_q8k(cols));
}

__global__ void __launch_bounds__(kQmvThreads, 2) qmv_kernel(const QmvJob* __restrict__ jobs, int njobs,
                                                             const int* __restrict__ dyn_count, QmvPrologue pro) {
  __shared__ float part[2][kQmvWarps][32][4];
  __shared__ int tile0s[kSmemJobs];
  extern __shared__ __align__(16) uint8_t act_smem[];
  if (dyn_count) {
    pdl_wait();
    njobs = *dyn_count;
  }
  if (njobs <= 0) {
    pdl_wait();
    return;
  }
  const QmvJob& last = jobs[njobs - 1];
  const int total = last.tile0 + (int)ceil_div(last.rows, qmv_rows_per_cta(last.ksplit));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;

  const int* t0 = nullptr;
  if (njobs <= kSmemJobs) {
    for (int i = threadIdx.x; i < njobs; i += kQmvThreads) tile0s[i] = jobs[i].tile0;
    __syncthreads();
    t0 = tile0s;
  }
  // the first block of this warp's stream, requested before the wait
  WarpTile cur_t = warp_tile(jobs, t0, njobs, total, blockIdx.x, warp, gid);
  WRegs cur;
  if (cur_t.live()) load_block(cur_t.dt, cur_t.wa, cur_t.wb, cur_t.nb, cur_t.u0, tig, cur);
  pdl_wait();
  pdl_trigger();
  if (pro.mode != kProNone) run_prologue(pro, act_smem);
  uint8_t* pro8k = act_smem;
  uint8_t* pro80 = act_smem + (pro.want8k ? pro.rows * pro.stride8k : 0);

  // staged activation key: every row of one activation buffer
  const uint8_t* staged_act = nullptr;
  int staged_rows = -1, staged_stride = 0;
  int it = 0;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x, it++) {
    const QmvJob& jb = jobs[cur_t.job >= 0 ? cur_t.job : find_job(jobs, t0, njobs, tile)];
    const int n = jb.n;
    const int used = act_used_bytes(jb.dtype, jb.cols);
    if (pro.mode == kProNone && (jb.act != staged_act || jb.act_nrows != staged_rows || used != staged_stride)) {
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
    }
    const uint8_t* base = act_smem;
    int stride = used;
    if (pro.mode != kProNone) {
      base = jb.dtype == Q8_0 ? pro80 : pro8k;
      stride = jb.dtype == Q8_0 ? pro.stride80 : pro.stride8k;
    }
    const uint8_t* bact = gid < n ? base + jb.rowmap[gid] * stride : nullptr;
    ActCols ac;
    ac.c[0] = 2 * tig < n ? base + jb.rowmap[2 * tig] * stride : nullptr;
    ac.c[1] = 2 * tig + 1 < n ? base + jb.rowmap[2 * tig + 1] * stride : nullptr;

    // this tile's blocks, with the next block of the stream always in flight
    const WarpTile nxt_t = warp_tile(jobs, t0, njobs, total, tile + gridDim.x, warp, gid);
    Frag f;
#pragma unroll
    for (int i = 0; i < 4; i++) { f.acc[i] = 0.f; f.accm[i] = 0.f; }
    if (cur_t.live()) {
      for (int b = cur_t.u0; b < cur_t.u1; b++) {
        WRegs nx;
        const bool more = b + 1 < cur_t.u1;
        if (more) load_block(cur_t.dt, cur_t.wa, cur_t.wb, cur_t.nb, b + 1, tig, nx);
        else if (nxt_t.live()) load_block(nxt_t.dt, nxt_t.wa, nxt_t.wb, nxt_t.nb, nxt_t.u0, tig, nx);
        compute_block(cur_t.dt, cur, bact, ac, cur_t.nb, b, tig, f);
        if (more || nxt_t.live()) cur = nx;
      }
    } else if (nxt_t.live()) {
      load_block(nxt_t.dt, nxt_t.wa, nxt_t.wb, nxt_t.nb, nxt_t.u0, tig, cur);
    }

    const bool has_min = jb.dtype == Q4_K || jb.dtype == Q5_K;
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; i++) y[i] = has_min ? __fsub_rn(f.acc[i], f.accm[i]) : f.acc[i];
    const int ks = jb.ksplit;
    bool store = cur_t.job >= 0 && cur_t.row0 < jb.rows;
    if (ks > 1) {
      float(*pb)[32][4] = part[it & 1];
#pragma unroll
      for (int i = 0; i < 4; i++) pb[warp][lane][i] = y[i];
      __syncthreads();
      store = store && cur_t.chunk == 0;
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
        const int row = cur_t.row0 + gid + (i >= 2 ? 8 : 0);
        const int col = 2 * tig + (i & 1);
        if (row >= jb.rows || col >= n) continue;
        const int64_t o = (int64_t)jb.outrow[col] * jb.out_ld + row;
        float v = y[i];
        if (jb.epi == kEpiResidual) v = __fadd_rn(jb.resid[o], v);
        jb.out[o] = v;
      }
    }
    cur_t = nxt_t;
  }
}

}  // namespace

int qmv_persistent_ctas() {
  static int n = 0;
  if (!n) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n = sms * 2;
  }
  return n;
}

cudaError_t qmv_launch(const QmvJob* jobs, int njobs, const int* dyn_count, int ntiles, int smem_bytes,
                       cudaStream_t stream, bool pdl, const QmvPrologue* pro) {
  QmvPrologue p = {};
  if (pro) {
    p = *pro;
    auto a16 = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
    const bool gated = p.mode == kProGated;
    if (p.rows < 1 || p.rows > 8 || p.cols % 256 || p.ldx % 4 || !a16(p.x) ||
        (p.mode == kProRmsNorm && !a16(p.w)) || (p.xn_out && (p.ldxn % 4 || !a16(p.xn_out))) ||
        (gated && (p.dv % 32 || p.ldz % 4 || !a16(p.z) || !a16(p.w) || p.rows * p.heads > kProMaxDen)))
      return cudaErrorInvalidValue;
    smem_bytes = std::max(smem_bytes, qmv_prologue_smem(p));
  }
  if (smem_bytes > kQmvMaxActSmem) return cudaErrorInvalidValue;
  if (ntiles <= 0) return cudaSuccess;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(qmv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQmvMaxActSmem);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(ntiles, qmv_persistent_ctas()));
  cfg.blockDim = dim3(kQmvThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qmv_kernel, jobs, njobs, dyn_count, p);
}

}  // namespace iq
