// layout.cuh -- device row layouts of GGUF weights and quantized activations.
//
// GGUF stores each weight row as consecutive blocks (src/qgemm.rs:46-65
// mirrors them).  On the device the bytes of each block are permuted so that
// one lane of an mma.sync fragment finds everything it needs for a block in
// 16-byte-aligned, contiguous words:
//
//   Q4_K (144 B/block): [d,dmin,scales 16 B][qs' 128 B]
//        qs'[tig*32 + j*8 + h*4 + e] = qs[32j + 16h + tig*4 + e]
//   Q5_K (176 B/block): [header 16 B][qh' 32 B][qs' 128 B]
//        qh'[tig*8 + h*4 + e] = qh[16h + tig*4 + e]
//   Q6_K: row = nb x [ql' 128 | qh' 64 | scales 16] then nb f16 d, padded to 16 B
//        ql'[tig*32 + half*16 + c*4 + e] = ql[half*64 + 16c + tig*4 + e]
//        qh'[tig*16 + half*8 + c*4 + e]  = qh[half*32 + 16c + tig*4 + e]
//   Q8_0: row = (nb/4) x 128 B of qs' then nb f16 d, padded to 16 B
//        qs'[g*128 + tig*32 + bb*8 + h*4 + e] = qs[block 4g+bb][16h + tig*4 + e]
//   F32:  unchanged.
//
// Rows stay contiguous and row-major, so a leading-row prefix (the MTP
// vocabulary-prefix head, src/gguf.rs:352-377) is still a byte prefix.
//
// Quantized activations (one row per input row):
//   Q8_K: [nb x 256 B qs'][nb x f32 d][nb x 16 i16 bsums], padded to 16 B
//        qs'[b*256 + tig*64 + s*8 + h*4 + e] = q[b*256 + 32s + 16h + tig*4 + e]
//   Q8_0: [nb/4 x 128 B qs' (as the weights)][nb x f32 d (the f16-rounded d)]
#pragma once
#include "iq_common.cuh"

namespace iq {

// Position of GGUF byte `i` of a block inside the device block / row.
__host__ __device__ inline int q4k_qs_perm(int i) {  // i in [0,128)
  int j = i / 32, ii = i % 32, h = ii / 16, tig = (ii % 16) / 4, e = ii % 4;
  return tig * 32 + j * 8 + h * 4 + e;
}
__host__ __device__ inline int q5k_qh_perm(int i) {  // i in [0,32)
  int h = i / 16, tig = (i % 16) / 4, e = i % 4;
  return tig * 8 + h * 4 + e;
}
__host__ __device__ inline int q6k_ql_perm(int i) {  // i in [0,128)
  int half = i / 64, q = i % 64, c = q / 16, tig = (q % 16) / 4, e = q % 4;
  return tig * 32 + half * 16 + c * 4 + e;
}
__host__ __device__ inline int q6k_qh_perm(int i) {  // i in [0,64)
  int half = i / 32, q = i % 32, c = q / 16, tig = (q % 16) / 4, e = q % 4;
  return tig * 16 + half * 8 + c * 4 + e;
}
// byte i (0..31) of Q8_0 block bb (0..3) within a group of four blocks
__host__ __device__ inline int q80_perm(int bb, int i) {
  int h = i / 16, tig = (i % 16) / 4, e = i % 4;
  return tig * 32 + bb * 8 + h * 4 + e;
}
// element i (0..255) of a Q8_K activation block
__host__ __device__ inline int q8k_act_perm(int i) {
  int s = i / 32, ii = i % 32, h = ii / 16, tig = (ii % 16) / 4, e = ii % 4;
  return tig * 64 + s * 8 + h * 4 + e;
}

}  // namespace iq
