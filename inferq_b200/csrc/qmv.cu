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

#ifndef QMV_MIN_BLOCKS
#define QMV_MIN_BLOCKS 2
#endif

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
      r.r[0] = ld_stream(ba + tig * 32);
      r.r[1] = ld_stream(ba + tig * 32 + 16);
      r.r[2] = ld_stream(bb + tig * 32);
      r.r[3] = ld_stream(bb + tig * 32 + 16);
      r.r[4] = ld_stream(ba + 128 + tig * 16);
      r.r[5] = ld_stream(bb + 128 + tig * 16);
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
// Q4_K / Q5_K: 8 sub-blocks of 32, u8 x s8 MMA (k32); mins term separately.
template <int DT>
__device__ __forceinline__ void compute_q45(const WRegs& r, const uint8_t* bact, ActCols ac, int nb, int b, int tig,
                                            Frag& f) {
  uint4 bw[4];
  load_b_words(bw, bact, b, tig);
  const uint4 ha = r.r[0], hb = r.r[1];
  int scA[8], mnA[8], scB[8], mnB[8];
  unpack_k_scales(reinterpret_cast<const uint8_t*>(&ha) + 4, scA, mnA);
  unpack_k_scales(reinterpret_cast<const uint8_t*>(&hb) + 4, scB, mnB);
  int isum[4] = {0, 0, 0, 0};
#pragma unroll
  for (int s = 0; s < 8; s++) {
    const int j = s / 2, hi = s & 1;
    const uint4& qa = j < 2 ? r.r[2] : r.r[3];
    const uint4& qb = j < 2 ? r.r[4] : r.r[5];
    uint32_t a0 = (w32(qa, (j % 2) * 2) >> (4 * hi)) & 0x0F0F0F0Fu;
    uint32_t a2 = (w32(qa, (j % 2) * 2 + 1) >> (4 * hi)) & 0x0F0F0F0Fu;
    uint32_t a1 = (w32(qb, (j % 2) * 2) >> (4 * hi)) & 0x0F0F0F0Fu;
    uint32_t a3 = (w32(qb, (j % 2) * 2 + 1) >> (4 * hi)) & 0x0F0F0F0Fu;
    if (DT == Q5_K) {
      a0 |= ((r.r[6].x >> s) & 0x01010101u) << 4;
      a2 |= ((r.r[6].y >> s) & 0x01010101u) << 4;
      a1 |= ((r.r[6].z >> s) & 0x01010101u) << 4;
      a3 |= ((r.r[6].w >> s) & 0x01010101u) << 4;
    }
    int p[4] = {0, 0, 0, 0};
    mma_u8s8_k32(p, a0, a1, a2, a3, w32(bw[s / 2], (s % 2) * 2), w32(bw[s / 2], (s % 2) * 2 + 1));
    isum[0] += scA[s] * p[0];
    isum[1] += scA[s] * p[1];
    isum[2] += scB[s] * p[2];
    isum[3] += scB[s] * p[3];
  }
  const float wdA = h2f(ha.x & 0xffff), wdminA = h2f(ha.x >> 16);
  const float wdB = h2f(hb.x & 0xffff), wdminB = h2f(hb.x >> 16);
#pragma unroll
  for (int c = 0; c < 2; c++) {
    float yd = 0.f;
    int msA = 0, msB = 0;
    if (ac.c[c]) {
      yd = *reinterpret_cast<const float*>(ac.c[c] + (int64_t)nb * 256 + b * 4);
      const int16_t* bs = reinterpret_cast<const int16_t*>(ac.c[c] + (int64_t)nb * 260 + b * 32);
#pragma unroll
      for (int s = 0; s < 8; s++) {
        const int b32 = bs[2 * s] + bs[2 * s + 1];
        msA += mnA[s] * b32;
        msB += mnB[s] * b32;
      }
    }
    f.acc[c] = fmaf(__fmul_rn(yd, wdA), __int2float_rn(isum[c]), f.acc[c]);
    f.accm[c] = fmaf(__fmul_rn(yd, wdminA), __int2float_rn(msA), f.accm[c]);
    f.acc[2 + c] = fmaf(__fmul_rn(yd, wdB), __int2float_rn(isum[2 + c]), f.acc[2 + c]);
    f.accm[2 + c] = fmaf(__fmul_rn(yd, wdminB), __int2float_rn(msB), f.accm[2 + c]);
  }
}

// Q6_K: 16 sub-blocks of 16, A = 4*(q-32) as s8 (k16 MMA).
__device__ __forceinline__ uint32_t q6_a(uint32_t qlw, uint32_t qhw, int q) {
  const uint32_t nib = (q / 4) ? (qlw >> 2) & 0x3C3C3C3Cu : (qlw << 2) & 0x3C3C3C3Cu;
  const int sh = 2 * (q / 2);
  const uint32_t hb = (qhw << (6 - sh)) & 0xC0C0C0C0u;
  return (nib | hb) ^ 0x80808080u;
}

__device__ __forceinline__ void compute_q6(const WRegs& r, const uint8_t* bact, ActCols ac, int nb, int b, int tig,
                                           Frag& f) {
  uint4 bw[4];
  load_b_words(bw, bact, b, tig);
  const int8_t* scA = reinterpret_cast<const int8_t*>(&r.r[6]);
  const int8_t* scB = reinterpret_cast<const int8_t*>(&r.r[7]);
  int isum[4] = {0, 0, 0, 0};
#pragma unroll
  for (int s16 = 0; s16 < 16; s16++) {
    const int half = s16 / 8, q = s16 % 8, c = q % 4, c2 = q % 2;
    const uint4& la = half ? r.r[1] : r.r[0];
    const uint4& lb = half ? r.r[3] : r.r[2];
    const uint32_t a0 = q6_a(w32(la, c), w32(r.r[4], half * 2 + c2), q);
    const uint32_t a1 = q6_a(w32(lb, c), w32(r.r[5], half * 2 + c2), q);
    int p[4] = {0, 0, 0, 0};
    mma_s8s8_k16(p, a0, a1, w32(bw[s16 / 4], s16 % 4));
    isum[0] += scA[s16] * p[0];
    isum[1] += scA[s16] * p[1];
    isum[2] += scB[s16] * p[2];
    isum[3] += scB[s16] * p[3];
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

__device__ __forceinline__ int find_job(const QmvJob* jobs, int njobs, int tile) {
  int lo = 0, hi = njobs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (jobs[mid].tile0 <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ WarpTile warp_tile(const QmvJob* jobs, int njobs, int total, int tile, int warp, int gid) {
  WarpTile w;
  w.job = -1;
  w.u0 = w.u1 = 0;
  if (tile >= total) return w;
  const int j = find_job(jobs, njobs, tile);
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

__device__ __forceinline__ int act_used_bytes(int dt, int cols) {
  return (int)(dt == Q8_0 ? act_row_bytes_q80(cols) : act_row_bytes_q8k(cols));
}

__global__ void __launch_bounds__(256, QMV_MIN_BLOCKS) qmv_kernel(const QmvJob* __restrict__ jobs, int njobs,
                                                                  const int* __restrict__ dyn_count) {
  __shared__ float part[2][8][32][4];
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

  // the first block of this warp's stream, requested before the wait
  WarpTile cur_t = warp_tile(jobs, njobs, total, blockIdx.x, warp, gid);
  WRegs cur;
  if (cur_t.live()) load_block(cur_t.dt, cur_t.wa, cur_t.wb, cur_t.nb, cur_t.u0, tig, cur);
  pdl_wait();
  pdl_trigger();

  // staged activation key: every row of one activation buffer
  const uint8_t* staged_act = nullptr;
  int staged_rows = -1, staged_stride = 0;
  int it = 0;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x, it++) {
    const QmvJob& jb = jobs[find_job(jobs, njobs, tile)];
    const int n = jb.n;
    const int used = act_used_bytes(jb.dtype, jb.cols);
    if (jb.act != staged_act || jb.act_nrows != staged_rows || used != staged_stride) {
      __syncthreads();  // no warp still reads the previous staging
      const int words = used / 16;
      for (int i = threadIdx.x; i < jb.act_nrows * words; i += 256) {
        const int r = i / words, w = i % words;
        reinterpret_cast<uint4*>(act_smem)[i] =
            *reinterpret_cast<const uint4*>(jb.act + (int64_t)r * jb.act_row_bytes + 16 * w);
      }
      __syncthreads();
      staged_act = jb.act;
      staged_rows = jb.act_nrows;
      staged_stride = used;
    }
    const uint8_t* bact = gid < n ? act_smem + jb.rowmap[gid] * used : nullptr;
    ActCols ac;
    ac.c[0] = 2 * tig < n ? act_smem + jb.rowmap[2 * tig] * used : nullptr;
    ac.c[1] = 2 * tig + 1 < n ? act_smem + jb.rowmap[2 * tig + 1] * used : nullptr;

    // this tile's blocks, with the next block of the stream always in flight
    const WarpTile nxt_t = warp_tile(jobs, njobs, total, tile + gridDim.x, warp, gid);
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
    n = sms * QMV_MIN_BLOCKS;
  }
  return n;
}

cudaError_t qmv_launch(const QmvJob* jobs, int njobs, const int* dyn_count, int ntiles, int smem_bytes,
                       cudaStream_t stream, bool pdl) {
  if (ntiles <= 0) return cudaSuccess;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(qmv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQmvMaxActSmem);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(ntiles, qmv_persistent_ctas()));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qmv_kernel, jobs, njobs, dyn_count);
}

}  // namespace iq
