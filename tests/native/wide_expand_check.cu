// Host check of the wide product's Q4_K / Q5_K weight expansion: runs the
// kernel's own per-thread arithmetic (expand_qk_chunk, wide_expand.cuh) on
// the CPU over random GGUF blocks put into the device layout (layout.cuh),
// and compares every operand value and every min / centring tile entry with
// an independent decode of the GGUF bytes (6-bit scale unpack and 4/5-bit
// quants as the GGML block formats define them, src/qgemm.rs:153-167).
// Built and run by tests/test_wide_expand_host.py; exits 0 when all match.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>
#include "layout.cuh"
#include "wide_expand.cuh"

using namespace iq;

static uint32_t g_rng = 12345u;
static uint8_t rnd() {
  g_rng = g_rng * 1664525u + 1013904223u;
  return (uint8_t)(g_rng >> 24);
}

static void scale_min(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

template <bool kQ5>
static int check(int rows, int nb) {
  const int BB = kQ5 ? 176 : 144, QS = kQ5 ? 48 : 16, cols = nb * 256;
  std::vector<uint8_t> gguf((size_t)rows * nb * BB), dev(gguf.size());
  for (auto& x : gguf) x = rnd();
  for (int i = 0; i < rows * nb && i < 4; i++) {  // a few blocks at the extremes
    uint8_t* g = &gguf[(size_t)i * BB];
    memset(g + 4, i & 1 ? 0xFF : 0x00, 12);
    memset(g + 16, i & 2 ? 0xFF : 0x00, BB - 16);
  }
  for (int blk = 0; blk < rows * nb; blk++) {
    const uint8_t* g = &gguf[(size_t)blk * BB];
    uint8_t* d = &dev[(size_t)blk * BB];
    memcpy(d, g, 16);
    if (kQ5)
      for (int i = 0; i < 32; i++) d[16 + q5k_qh_perm(i)] = g[16 + i];
    for (int i = 0; i < 128; i++) d[QS + q4k_qs_perm(i)] = g[QS + i];
  }
  const int rtiles = (rows + 127) / 128;
  std::vector<__half> out((size_t)rows * cols, __float2half(NAN));
  std::vector<__half> am((size_t)rtiles * nb * 2048, __float2half(NAN)), ac(am.size(), __float2half(NAN));
  for (int r = 0; r < rows; r++)
    for (int b = 0; b < nb; b++)
      for (int c = 0; c < 8; c++) {
        const uint8_t* blk = &dev[((size_t)r * nb + b) * BB];
        uint4 hdr, v;
        uint2 qh = make_uint2(0u, 0u);
        memcpy(&hdr, blk, 16);
        memcpy(&v, blk + QS + c * 16, 16);
        if (kQ5) memcpy(&qh, blk + 16 + (c >> 1) * 8, 8);
        const size_t tile = ((size_t)(r / 128) * nb + b) * 2048;
        expand_qk_chunk<kQ5>(hdr, v, qh, c, b, &out[(size_t)r * cols], &am[tile], &ac[tile], r % 128);
      }
  int bad = 0;
  for (int r = 0; r < rows; r++)
    for (int b = 0; b < nb; b++) {
      const uint8_t* g = &gguf[((size_t)r * nb + b) * BB];
      int sc[8], mn[8];
      for (int j = 0; j < 8; j++) scale_min(g + 4, j, sc[j], mn[j]);
      for (int e = 0; e < 256; e++) {
        const int j = e / 64, i = e % 64;
        int q = i < 32 ? (g[QS + 32 * j + i] & 15) : (g[QS + 32 * j + i - 32] >> 4);
        if (kQ5) q |= ((g[16 + e % 32] >> (e / 32)) & 1) << 4;
        const float want = (float)(sc[e / 32] * (q - (kQ5 ? 16 : 0)));
        const float got = __half2float(out[(size_t)r * cols + b * 256 + e]);
        if (got != want && bad++ < 5)
          printf("Q%d_K row %d block %d element %d: got %g want %g\n", kQ5 ? 5 : 4, r, b, e, got, want);
      }
      const size_t tile = ((size_t)(r / 128) * nb + b) * 2048;
      const int rr = r % 128;
      for (int s = 0; s < 8; s++) {
        const float m0 = __half2float(am[tile + plain_off(rr, 0) / 2 + s]);
        const float m1 = __half2float(am[tile + plain_off(rr, 1) / 2 + s]);
        if ((m0 != mn[s] || m1 != 64 * mn[s]) && bad++ < 5)
          printf("min tile row %d block %d s %d: %g %g want %d\n", r, b, s, m0, m1, mn[s]);
        if (kQ5) {
          const float c0 = __half2float(ac[tile + plain_off(rr, 0) / 2 + s]);
          const float c1 = __half2float(ac[tile + plain_off(rr, 1) / 2 + s]);
          if ((c0 != sc[s] || c1 != 64 * sc[s]) && bad++ < 5)
            printf("centring tile row %d block %d s %d: %g %g want %d\n", r, b, s, c0, c1, sc[s]);
        }
      }
    }
  printf("Q%d_K expansion: %d rows x %d blocks, %d mismatches\n", kQ5 ? 5 : 4, rows, nb, bad);
  return bad;
}

int main() {
  int bad = check<false>(131, 3) + check<true>(131, 3) + check<true>(7, 1);
  return bad ? 1 : 0;
}
