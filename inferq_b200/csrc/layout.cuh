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
//   Q6_K: row = nb x [q' 192 | scales 16] then nb f16 d, padded to 16 B.
//        q' holds the 256 6-bit values v(i) (0..63) re-packed for the k16
//        MMA: lane tig owns 48 B at tig*48, four sets g of three words; byte
//        e of word j (0..2) of set g is
//            v(16(4g+j) + 4tig + e) << 2  |  (v(16(4g+3) + 4tig + e) >> 2j) & 3
//        so A = 4(v-32) of sub-blocks 4g..4g+2 is one AND/XOR per word and
//        sub-block 4g+3 is reassembled from the three low bit pairs.
//   Q8_0: row = (nb/4) x 128 B of qs' then nb f16 d, padded to 16 B
//        qs'[g*128 + tig*32 + bb*8 + h*4 + e] = qs[block 4g+bb][16h + tig*4 + e]
//   F32:  unchanged.
//
// Rows stay contiguous and row-major, so a leading-row prefix (the MTP
// vocabulary-prefix head, src/gguf.rs:352-377) is still a byte prefix.
//
// Quantized activations (one row per input row):
//   Q8_K: [nb x 256 B qs'][nb x f32 d, padded to 16 B][nb x 8 i16 sums of 32 elements]
//        qs'[b*256 + tig*64 + (((s>>1) ^ tig) & 3)*16 + (s&1)*8 + h*4 + e]
//            = q[b*256 + 32s + 16h + tig*4 + e]
//        (the XOR spreads the four lanes of a row group over distinct banks)
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
// The 6-bit value (0..63) of element i of a GGUF Q6_K block (ql, qh as in
// ggml's block_q6_K: element 128h + 32c + l takes its low nibble from
// ql[64h + l + 32(c&1)] (high nibble when c >= 2) and bits 2c..2c+1 of
// qh[32h + l]).
__host__ __device__ inline int q6k_value(const uint8_t* blk, int i) {
  const int h = i / 128, c = (i % 128) / 32, l = i % 32;
  const int nib = (blk[64 * h + l + 32 * (c & 1)] >> (4 * (c >> 1))) & 15;
  const int hb = (blk[128 + 32 * h + l] >> (2 * c)) & 3;
  return nib | (hb << 4);
}
// The value of element i from a device Q6_K block (layout above).
__host__ __device__ inline int q6k_dev_value(const uint8_t* blk, int i) {
  const int s16 = i / 16, k = i % 16, tig = k / 4, e = k % 4, g = s16 / 4, j = s16 % 4;
  const uint8_t* w = blk + tig * 48 + g * 12 + e;
  if (j < 3) return w[4 * j] >> 2;
  return (w[0] & 3) | ((w[4] & 3) << 2) | ((w[8] & 3) << 4);
}
// byte i (0..31) of Q8_0 block bb (0..3) within a group of four blocks
__host__ __device__ inline int q80_perm(int bb, int i) {
  int h = i / 16, tig = (i % 16) / 4, e = i % 4;
  return tig * 32 + bb * 8 + h * 4 + e;
}
// element i (0..255) of a Q8_K activation block
__host__ __device__ inline int q8k_act_perm(int i) {
  int s = i / 32, ii = i % 32, h = ii / 16, tig = (ii % 16) / 4, e = ii % 4;
  return tig * 64 + (((s >> 1) ^ tig) & 3) * 16 + (s & 1) * 8 + h * 4 + e;
}

}  // namespace iq
