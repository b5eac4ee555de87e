// wide_expand.cuh -- the per-thread arithmetic of the Q4_K / Q5_K weight
// expansion for the wide product (wide.cu, wide_expand_q4k_kernel), as a
// host-and-device function over one 16-byte chunk of quant bytes that the
// caller has already loaded, so the same source also runs on the host.
//
// Device block layouts (layout.cuh): Q4_K [header 16 B][qs' 128 B], Q5_K
// [header 16 B][qh' 32 B][qs' 128 B]; qs' byte tig*32 + j*8 + h*4 + e holds
// GGUF qs byte 32j + 16h + 4tig + e (low nibble: element 64j + 16h + 4tig + e,
// high nibble: that element + 32); qh' byte tig*8 + h*4 + e holds GGUF
// qh[16h + 4tig + e], whose bit 2j is the fifth bit of the low-nibble
// element and bit 2j+1 that of the high-nibble element.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace iq {

// Byte offset of (row, K half) in a core-matrix tile of the 16-wide min /
// centring operands: 8-row x 16-byte core matrices, K halves 128 bytes
// apart, 8-row groups 256 bytes apart.
__host__ __device__ __forceinline__ int plain_off(int row, int half) {
  return (row >> 3) * 256 + half * 128 + (row & 7) * 16;
}

// Chunk c (0..7) of block b of one weight row: hdr = the block's 16-byte
// header, v = quant bytes 16c..16c+15, qh = (Q5_K) qh' bytes 8*(c/2)..+7.
// Writes the 32 operand values it covers into out_row (the row's f16
// operand, K-major): A = sc[s] * q (Q4_K) or sc[s] * (q - 16) (Q5_K).
// Chunk 0 also writes the row's line `rr` of the block's min tile
// (mn[0..7], 64 * mn[0..7]) and, for Q5_K, of its centring tile
// (sc[0..7], 64 * sc[0..7]).
template <bool kQ5>
__host__ __device__ __forceinline__ void expand_qk_chunk(uint4 hdr, uint4 v, uint2 qh, int c, int b,
                                                         __half* out_row, __half* min_tile, __half* ctr_tile,
                                                         int rr) {
  constexpr int kCentre = kQ5 ? 16 : 0;
  const int tig = c >> 1;
  // six-bit scales and mins as bytes: sc0-3, sc4-7, mn0-3, mn4-7
  const uint32_t s_lo = hdr.y & 0x3F3F3F3Fu, m_lo = hdr.z & 0x3F3F3F3Fu;
  const uint32_t s_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
  const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int qw = 0; qw < 4; qw++) {
    const int j = 2 * (c & 1) + (qw >> 1), h = qw & 1;
    const int slo = 2 * j, shi = 2 * j + 1;
    const int sc_lo = (int)(((slo < 4 ? s_lo : s_hi) >> (8 * (slo & 3))) & 0xFF);
    const int sc_hi = (int)(((shi < 4 ? s_lo : s_hi) >> (8 * (shi & 3))) & 0xFF);
    const int k = b * 256 + 64 * j + 16 * h + 4 * tig;
    __half2 lo[2], hi[2];
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int b0 = (int)((wd[qw] >> (8 * e)) & 0xFF), b1 = (int)((wd[qw] >> (8 * (e + 1))) & 0xFF);
      int l0 = b0 & 15, l1 = b1 & 15, h0 = b0 >> 4, h1 = b1 >> 4;
      if constexpr (kQ5) {
        const uint32_t qw32 = h ? qh.y : qh.x;
        const uint32_t q0 = qw32 >> (8 * e + 2 * j), q1 = qw32 >> (8 * (e + 1) + 2 * j);
        l0 |= (int)(q0 & 1) << 4;
        l1 |= (int)(q1 & 1) << 4;
        h0 |= (int)((q0 >> 1) & 1) << 4;
        h1 |= (int)((q1 >> 1) & 1) << 4;
      }
      lo[e / 2] = __halves2half2(__int2half_rn(sc_lo * (l0 - kCentre)), __int2half_rn(sc_lo * (l1 - kCentre)));
      hi[e / 2] = __halves2half2(__int2half_rn(sc_hi * (h0 - kCentre)), __int2half_rn(sc_hi * (h1 - kCentre)));
    }
    *reinterpret_cast<uint2*>(out_row + k) =
        make_uint2(*reinterpret_cast<uint32_t*>(&lo[0]), *reinterpret_cast<uint32_t*>(&lo[1]));
    *reinterpret_cast<uint2*>(out_row + k + 32) =
        make_uint2(*reinterpret_cast<uint32_t*>(&hi[0]), *reinterpret_cast<uint32_t*>(&hi[1]));
  }
  if (c == 0) {
#pragma unroll
    for (int s = 0; s < 8; s++) {
      const int mn = (int)(((s < 4 ? m_lo : m_hi) >> (8 * (s & 3))) & 0xFF);
      min_tile[plain_off(rr, 0) / 2 + s] = __int2half_rn(mn);
      min_tile[plain_off(rr, 1) / 2 + s] = __int2half_rn(64 * mn);
    }
    if constexpr (kQ5) {
#pragma unroll
      for (int s = 0; s < 8; s++) {
        const int sc = (int)(((s < 4 ? s_lo : s_hi) >> (8 * (s & 3))) & 0xFF);
        ctr_tile[plain_off(rr, 0) / 2 + s] = __int2half_rn(sc);
        ctr_tile[plain_off(rr, 1) / 2 + s] = __int2half_rn(64 * sc);
      }
    }
  }
}

}  // namespace iq
