// qmv.cu -- skinny quantized GEMV kernels (see qmv.cuh).
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

// Activation helpers ---------------------------------------------------------
struct ActCols {  // the two C-fragment columns of this thread
  const uint8_t* c[2];
};

__device__ __forceinline__ void load_act(uint4 (&bw)[4], const uint8_t* bact, int b, int tig) {
  if (bact) {
#pragma unroll
    for (int i = 0; i < 4; i++)
      bw[i] = *reinterpret_cast<const uint4*>(bact + (int64_t)b * 256 + tig * 64 + i * 16);
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) bw[i] = make_uint4(0, 0, 0, 0);
  }
}

// Software pipeline over a chunk: the weights of block b+1 are in flight
// while block b is computed.  The first block's weights are requested before
// the programmatic-dependency wait (weights never depend on the previous
// kernel; the activations do).
template <class Ops, class Stage>
__device__ __forceinline__ void run_chunk(const Ops& ops, int b0, int b1, bool live, Stage& stage, Frag& f) {
  typename Ops::Regs cur;
  if (live) cur = ops.load(b0);
  stage();  // every thread: wait for the producer kernel, stage activations
  if (!live) return;
  for (int b = b0; b < b1; b++) {
    typename Ops::Regs nxt;
    if (b + 1 < b1) nxt = ops.load(b + 1);
    ops.compute(cur, b, f);
    cur = nxt;
  }
}

// ---------------------------------------------------------------- Q4_K / Q5_K
template <int DT>
struct OpsQ45 {
  static constexpr int BB = DT == Q4_K ? 144 : 176;
  static constexpr int QS = DT == Q4_K ? 16 : 48;
  struct Regs {
    uint4 ha, hb, qa0, qa1, qb0, qb1;
    uint2 hha, hhb;
  };
  const uint8_t *wa, *wb, *bact;
  ActCols ac;
  int nb, tig;
  __device__ __forceinline__ Regs load(int b) const {
    Regs r;
    const uint8_t* ba = wa + (int64_t)b * BB;
    const uint8_t* bb = wb + (int64_t)b * BB;
    r.ha = ld_stream(ba);
    r.hb = ld_stream(bb);
    r.qa0 = ld_stream(ba + QS + tig * 32);
    r.qa1 = ld_stream(ba + QS + tig * 32 + 16);
    r.qb0 = ld_stream(bb + QS + tig * 32);
    r.qb1 = ld_stream(bb + QS + tig * 32 + 16);
    if (DT == Q5_K) {
      r.hha = *reinterpret_cast<const uint2*>(ba + 16 + tig * 8);
      r.hhb = *reinterpret_cast<const uint2*>(bb + 16 + tig * 8);
    } else {
      r.hha = r.hhb = make_uint2(0, 0);
    }
    return r;
  }
  __device__ __forceinline__ void compute(const Regs& r, int b, Frag& f) const {
    uint4 bw[4];
    load_act(bw, bact, b, tig);
    int scA[8], mnA[8], scB[8], mnB[8];
    unpack_k_scales(reinterpret_cast<const uint8_t*>(&r.ha) + 4, scA, mnA);
    unpack_k_scales(reinterpret_cast<const uint8_t*>(&r.hb) + 4, scB, mnB);
    int isum[4] = {0, 0, 0, 0};
#pragma unroll
    for (int s = 0; s < 8; s++) {
      const int j = s / 2, hi = s & 1;
      const uint4& qa = j < 2 ? r.qa0 : r.qa1;
      const uint4& qb = j < 2 ? r.qb0 : r.qb1;
      uint32_t wa0 = w32(qa, (j % 2) * 2), wa1 = w32(qa, (j % 2) * 2 + 1);
      uint32_t wb0 = w32(qb, (j % 2) * 2), wb1 = w32(qb, (j % 2) * 2 + 1);
      uint32_t a0 = (wa0 >> (4 * hi)) & 0x0F0F0F0Fu, a2 = (wa1 >> (4 * hi)) & 0x0F0F0F0Fu;
      uint32_t a1 = (wb0 >> (4 * hi)) & 0x0F0F0F0Fu, a3 = (wb1 >> (4 * hi)) & 0x0F0F0F0Fu;
      if (DT == Q5_K) {
        a0 |= ((r.hha.x >> s) & 0x01010101u) << 4;
        a2 |= ((r.hha.y >> s) & 0x01010101u) << 4;
        a1 |= ((r.hhb.x >> s) & 0x01010101u) << 4;
        a3 |= ((r.hhb.y >> s) & 0x01010101u) << 4;
      }
      int p[4] = {0, 0, 0, 0};
      mma_u8s8_k32(p, a0, a1, a2, a3, w32(bw[s / 2], (s % 2) * 2), w32(bw[s / 2], (s % 2) * 2 + 1));
      isum[0] += scA[s] * p[0];
      isum[1] += scA[s] * p[1];
      isum[2] += scB[s] * p[2];
      isum[3] += scB[s] * p[3];
    }
    const float wdA = h2f(r.ha.x & 0xffff), wdminA = h2f(r.ha.x >> 16);
    const float wdB = h2f(r.hb.x & 0xffff), wdminB = h2f(r.hb.x >> 16);
#pragma unroll
    for (int c = 0; c < 2; c++) {
      float yd = 0.f;
      int msA = 0, msB = 0;
      if (ac.c[c]) {
        yd = *reinterpret_cast<const float*>(ac.c[c] + (int64_t)nb * 256 + b * 4);
        const int16_t* bs = reinterpret_cast<const int16_t*>(ac.c[c] + (int64_t)nb * 260 + b * 32);
#pragma unroll
        for (int s = 0; s < 8; s++) {
          int b32 = bs[2 * s] + bs[2 * s + 1];
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
};

// ---------------------------------------------------------------------- Q6_K
__device__ __forceinline__ uint32_t q6_a(uint32_t qlw, uint32_t qhw, int q) {
  // 4*(q6 - 32) as four s8: low 4 bits from ql (nibble q/4), top 2 from qh.
  uint32_t nib = (q / 4) ? (qlw >> 2) & 0x3C3C3C3Cu : (qlw << 2) & 0x3C3C3C3Cu;
  const int sh = 2 * (q / 2);
  uint32_t hb = (qhw << (6 - sh)) & 0xC0C0C0C0u;
  return (nib | hb) ^ 0x80808080u;
}

struct OpsQ6 {
  struct Regs {
    uint4 la0, la1, lb0, lb1, hA, hB, sA, sB;
    uint16_t dA, dB;
  };
  const uint8_t *wa, *wb, *bact;
  ActCols ac;
  int nb, tig;
  __device__ __forceinline__ Regs load(int b) const {
    Regs r;
    const uint8_t* ba = wa + (int64_t)b * 208;
    const uint8_t* bb = wb + (int64_t)b * 208;
    r.la0 = ld_stream(ba + tig * 32);
    r.la1 = ld_stream(ba + tig * 32 + 16);
    r.lb0 = ld_stream(bb + tig * 32);
    r.lb1 = ld_stream(bb + tig * 32 + 16);
    r.hA = ld_stream(ba + 128 + tig * 16);
    r.hB = ld_stream(bb + 128 + tig * 16);
    r.sA = ld_stream(ba + 192);
    r.sB = ld_stream(bb + 192);
    r.dA = *reinterpret_cast<const uint16_t*>(wa + (int64_t)nb * 208 + 2 * b);
    r.dB = *reinterpret_cast<const uint16_t*>(wb + (int64_t)nb * 208 + 2 * b);
    return r;
  }
  __device__ __forceinline__ void compute(const Regs& r, int b, Frag& f) const {
    uint4 bw[4];
    load_act(bw, bact, b, tig);
    const int8_t* scA = reinterpret_cast<const int8_t*>(&r.sA);
    const int8_t* scB = reinterpret_cast<const int8_t*>(&r.sB);
    int isum[4] = {0, 0, 0, 0};
#pragma unroll
    for (int s16 = 0; s16 < 16; s16++) {
      const int half = s16 / 8, q = s16 % 8, c = q % 4, c2 = q % 2;
      const uint4& la = half ? r.la1 : r.la0;
      const uint4& lb = half ? r.lb1 : r.lb0;
      uint32_t a0 = q6_a(w32(la, c), w32(r.hA, half * 2 + c2), q);
      uint32_t a1 = q6_a(w32(lb, c), w32(r.hB, half * 2 + c2), q);
      int p[4] = {0, 0, 0, 0};
      mma_s8s8_k16(p, a0, a1, w32(bw[s16 / 4], s16 % 4));
      isum[0] += scA[s16] * p[0];
      isum[1] += scA[s16] * p[1];
      isum[2] += scB[s16] * p[2];
      isum[3] += scB[s16] * p[3];
    }
    const float wdA = h2f(r.dA), wdB = h2f(r.dB);
#pragma unroll
    for (int c = 0; c < 2; c++) {
      float yd = ac.c[c] ? *reinterpret_cast<const float*>(ac.c[c] + (int64_t)nb * 256 + b * 4) : 0.f;
      f.acc[c] = fmaf(__fmul_rn(yd, wdA), __int2float_rn(isum[c] >> 2), f.acc[c]);
      f.acc[2 + c] = fmaf(__fmul_rn(yd, wdB), __int2float_rn(isum[2 + c] >> 2), f.acc[2 + c]);
    }
  }
};

// ---------------------------------------------------------------------- Q8_0
struct OpsQ80 {
  struct Regs {
    uint4 qa0, qa1, qb0, qb1;
    uint2 dwa, dwb;
  };
  const uint8_t *wa, *wb, *bact;
  ActCols ac;
  int nb, tig;
  __device__ __forceinline__ Regs load(int g) const {
    Regs r;
    r.qa0 = ld_stream(wa + (int64_t)g * 128 + tig * 32);
    r.qa1 = ld_stream(wa + (int64_t)g * 128 + tig * 32 + 16);
    r.qb0 = ld_stream(wb + (int64_t)g * 128 + tig * 32);
    r.qb1 = ld_stream(wb + (int64_t)g * 128 + tig * 32 + 16);
    r.dwa = *reinterpret_cast<const uint2*>(wa + (int64_t)nb * 32 + 8 * g);
    r.dwb = *reinterpret_cast<const uint2*>(wb + (int64_t)nb * 32 + 8 * g);
    return r;
  }
  __device__ __forceinline__ void compute(const Regs& r, int g, Frag& f) const {
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
      const uint4& qa = bb < 2 ? r.qa0 : r.qa1;
      const uint4& qb = bb < 2 ? r.qb0 : r.qb1;
      const uint4& xx = bb < 2 ? x0 : x1;
      const int o = (bb % 2) * 2;
      int p[4] = {0, 0, 0, 0};
      mma_s8s8_k32(p, w32(qa, o), w32(qb, o), w32(qa, o + 1), w32(qb, o + 1), w32(xx, o), w32(xx, o + 1));
      const uint32_t hwa = bb < 2 ? r.dwa.x : r.dwa.y, hwb = bb < 2 ? r.dwb.x : r.dwb.y;
      const float wdA = h2f((bb & 1) ? hwa >> 16 : hwa & 0xffff);
      const float wdB = h2f((bb & 1) ? hwb >> 16 : hwb & 0xffff);
#pragma unroll
      for (int c = 0; c < 2; c++) {
        float y = bb == 0 ? yd[c].x : bb == 1 ? yd[c].y : bb == 2 ? yd[c].z : yd[c].w;
        f.acc[c] = fmaf(__fmul_rn(wdA, y), __int2float_rn(p[c]), f.acc[c]);
        f.acc[2 + c] = fmaf(__fmul_rn(wdB, y), __int2float_rn(p[2 + c]), f.acc[2 + c]);
      }
    }
  }
};

__global__ void __launch_bounds__(256, QMV_MIN_BLOCKS) qmv_kernel(const QmvJob* __restrict__ jobs, int njobs,
                                                                  const int* __restrict__ dyn_count) {
  __shared__ float part[8][32][4];
  extern __shared__ __align__(16) uint8_t act_smem[];
  if (dyn_count) {
    pdl_wait();
    njobs = *dyn_count;
  }
  const int tile = blockIdx.x;
  // locate the job: the last one with tile0 <= tile
  int lo = 0, hi = njobs - 1;
  if (njobs <= 0) {
    pdl_wait();  // every CTA waits once, so completion order stays transitive
    return;
  }
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (jobs[mid].tile0 <= tile) lo = mid; else hi = mid - 1;
  }
  const QmvJob& jb = jobs[lo];
  const int ks = jb.ksplit;
  const int local = tile - jb.tile0;
  if (local * qmv_rows_per_cta(ks) >= jb.rows) {  // past the job table's end
    pdl_wait();
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int rt = warp / ks, chunk = warp % ks;
  const int row0 = local * qmv_rows_per_cta(ks) + rt * 16;
  const bool warp_live = row0 < jb.rows;
  const int dt = jb.dtype;
  const int nb = jb.cols / gguf_block_elems(dt);
  const int units = qmv_units(dt, jb.cols);
  const int u0 = chunk * units / ks, u1 = (chunk + 1) * units / ks;
  const int arb = jb.act_row_bytes;
  const int n = jb.n;

  Frag f;
#pragma unroll
  for (int i = 0; i < 4; i++) { f.acc[i] = 0.f; f.accm[i] = 0.f; }
  const int ra = min(row0 + gid, jb.rows - 1), rb = min(row0 + gid + 8, jb.rows - 1);
  const uint8_t* wa = jb.w + (int64_t)ra * jb.w_row_bytes;
  const uint8_t* wb = jb.w + (int64_t)rb * jb.w_row_bytes;
  // The activation rows this job reads, staged once per CTA after the wait.
  auto stage = [&]() {
    pdl_wait();
    const int words = arb / 16;
    for (int i = threadIdx.x; i < n * words; i += 256) {
      const int r = i / words, w = i % words;
      reinterpret_cast<uint4*>(act_smem)[i] =
          *reinterpret_cast<const uint4*>(jb.act + (int64_t)jb.rowmap[r] * arb + 16 * w);
    }
    __syncthreads();
  };
  const uint8_t* bact = gid < n ? act_smem + gid * arb : nullptr;
  ActCols ac;
  ac.c[0] = 2 * tig < n ? act_smem + 2 * tig * arb : nullptr;
  ac.c[1] = 2 * tig + 1 < n ? act_smem + (2 * tig + 1) * arb : nullptr;
  const bool live = warp_live && u0 < u1;
  switch (dt) {
    case Q4_K: run_chunk(OpsQ45<Q4_K>{wa, wb, bact, ac, nb, tig}, u0, u1, live, stage, f); break;
    case Q5_K: run_chunk(OpsQ45<Q5_K>{wa, wb, bact, ac, nb, tig}, u0, u1, live, stage, f); break;
    case Q6_K: run_chunk(OpsQ6{wa, wb, bact, ac, nb, tig}, u0, u1, live, stage, f); break;
    default: run_chunk(OpsQ80{wa, wb, bact, ac, nb, tig}, u0, u1, live, stage, f); break;
  }
  pdl_trigger();
  const bool has_min = dt == Q4_K || dt == Q5_K;
#pragma unroll
  for (int i = 0; i < 4; i++) part[warp][lane][i] = has_min ? __fsub_rn(f.acc[i], f.accm[i]) : f.acc[i];
  __syncthreads();
  if (!warp_live || chunk != 0) return;
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    y[i] = part[warp][lane][i];
    for (int c = 1; c < ks; c++) y[i] = __fadd_rn(y[i], part[warp + c][lane][i]);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int row = row0 + gid + (i >= 2 ? 8 : 0);
    const int col = 2 * tig + (i & 1);
    if (row >= jb.rows || col >= n) continue;
    const int64_t o = (int64_t)jb.outrow[col] * jb.out_ld + row;
    float v = y[i];
    if (jb.epi == kEpiResidual) v = __fadd_rn(jb.resid[o], v);
    jb.out[o] = v;
  }
}

}  // namespace

cudaError_t qmv_launch(const QmvJob* jobs, int njobs, const int* dyn_count, int ntiles, int smem_bytes,
                       cudaStream_t stream, bool pdl) {
  if (ntiles <= 0) return cudaSuccess;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(qmv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQmvMaxActSmem);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ntiles);
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
