/*
 * CPU restatement of the reference's GGUF weight decode (the checker, NOT the product).
 *
 * TEST INFRASTRUCTURE ONLY. This file is compiled into oracle/_build/liboracle.so and is loaded only by
 * tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg, always as the checker of the CUDA
 * path, never as the thing that is measured or shipped.
 *
 * What it restates (reference paths relative to the reference repository root):
 *   - engine/gpu/loom/tools/gen_gemm_decode.py:1338-1378  Q8_0 decode: w = f16(f32(d) * f32(q))
 *   - engine/gpu/loom/tools/gen_gemm_decode.py:837-1069   Q4_K decode: w = f16(fma(d*sc, q, -dmin*m)), the 6-bit
 *                                                          sc/m unpack of :946-967 (Q4_SEL), Q4DFMA :54-56
 *   - engine/gpu/loom/tools/gen_gemm_decode.py:1243-1335  Q6_K decode: w = f16((d*sc) * (code - 32))
 *   - engine/gpu/loom/tools/gen_gemm_decode.py:897-899, :1713-1716  Q5_K decode: Q4_K plus a fifth bit from the
 *                                                          qh plane, qs at 48: w = f16((d*sc)*q - dmin*m)
 *   - engine/gpu/loom/tools/gen_gemm_decode.py:1497-1546  Q3_K decode: q = (low | hbit << 2) - 4, the 6-bit signed
 *                                                          scales, w = f16((d*(sc-32)) * q)
 *   - engine/gpu/loom/tools/gen_gemm_decode.py:125-169    IQ4_XS decode: w = f16((d*(sc-32)) * kvalues[nibble])
 *   - engine/core/gguf.cpp:27-35                           block sizes (Q8_0 32/34, Q3_K 256/110, Q4_K 256/144,
 *                                                          Q5_K 256/176, Q6_K 256/210, IQ4_XS 256/136)
 * The arithmetic matches gguf-py 0.19.0 (gguf/quants.py <format>.dequantize_blocks) followed by
 * astype(float16), which is the reference's own dequant oracle (engine/gpu/loom/tools/dq_bfp16_check.py:65).
 * Parity of this file with gguf-py is pinned by the committed vectors in tests/golden/.
 *
 * Two outputs are offered per format:
 *   *_f16: the value rounded once to f16 (the tile GEMM's weights; bit-exact target of the CUDA dequant);
 *   *_f32: the f32 value before that rounding (what gguf-py's dequantize returns; the reference GEMV's oracle,
 *          engine/gpu/loom/tools/gemv_check.py:161-162).
 */
#include <stdint.h>
#include <string.h>

enum { T_Q8_0 = 8, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ4_XS = 23 };

static float h2f(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static uint16_t f2h(float f) {
  _Float16 v = (_Float16)f; /* IEEE round-to-nearest-even, subnormals kept */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

/* ---- one 256-element super-block of each format, into 256 f32 values ---- */

/* Q8_0: 8 blocks of (f16 d, int8 q[32]) = 272 bytes (gen_gemm_decode.py:1338-1339 treats 8 blocks as one). */
static void sb_q8_0(const uint8_t* b, float* out) {
  for (int blk = 0; blk < 8; ++blk) {
    const uint8_t* p = b + 34 * blk;
    uint16_t dh = (uint16_t)(p[0] | (p[1] << 8));
    float d = h2f(dh);
    for (int j = 0; j < 32; ++j) out[32 * blk + j] = d * (float)(int8_t)p[2 + j];
  }
}

/* Q4_K sub-block scale/min unpack (gguf.hpp layout; gen_gemm_decode.py:946-967). */
static void q4k_scale_min(const uint8_t* s, int g, int* sc, int* m) {
  if (g < 4) {
    *sc = s[g] & 63;
    *m = s[g + 4] & 63;
  } else {
    *sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
    *m = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
  }
}

/* Q4_K: d f16 @0, dmin f16 @2, scales[12] @4, qs[128] @16. Group g (32 values) reads qs[32*(g/2)+j], the low
 * nibble for even g and the high nibble for odd g. d*sc*q is exact in f32, so one rounding at the subtraction. */
static void sb_q4_k(const uint8_t* b, float* out) {
  float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
  float dmin = h2f((uint16_t)(b[2] | (b[3] << 8)));
  const uint8_t* s = b + 4;
  const uint8_t* qs = b + 16;
  for (int g = 0; g < 8; ++g) {
    int sc, m;
    q4k_scale_min(s, g, &sc, &m);
    float dsc = d * (float)sc;
    float dm = dmin * (float)m;
    for (int j = 0; j < 32; ++j) {
      int byte = qs[32 * (g / 2) + j];
      int q = (g & 1) ? (byte >> 4) : (byte & 15);
      volatile float prod = dsc * (float)q; /* exact; volatile keeps gcc from contracting into another form */
      out[32 * g + j] = prod - dm;
    }
  }
}

/* Q6_K: ql[128] @0, qh[64] @128, int8 scales[16] @192, d f16 @208.
 * element e = 128*h + 32*seg + j: low 4 bits from ql[64h + 32*(seg&1) + j] (low nibble if seg < 2), high 2 bits
 * from (qh[32h + j] >> 2*seg) & 3, scale index e/16. (d*sc) and (d*sc)*(code-32) are exact in f32. */
static void sb_q6_k(const uint8_t* b, float* out) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = (const int8_t*)(b + 192);
  float d = h2f((uint16_t)(b[208] | (b[209] << 8)));
  for (int e = 0; e < 256; ++e) {
    int h = e / 128, seg = (e % 128) / 32, j = e % 32;
    int lb = ql[64 * h + 32 * (seg & 1) + j];
    int lo = seg < 2 ? (lb & 15) : (lb >> 4);
    int hi = (qh[32 * h + j] >> (2 * seg)) & 3;
    int code = lo | (hi << 4);
    volatile float dsc = d * (float)sc[e / 16];
    out[e] = dsc * (float)(code - 32);
  }
}

/* Q5_K: d f16 @0, dmin f16 @2, scales[12] @4 (the Q4_K unpack), qh[32] @16, qs[128] @48. Group g (32 values):
 * q = nibble of qs[32*(g/2)+j] (low for even g) | ((qh[j] >> g) & 1) << 4. d*sc*q is exact, one rounding at the
 * subtraction. */
static void sb_q5_k(const uint8_t* b, float* out) {
  float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
  float dmin = h2f((uint16_t)(b[2] | (b[3] << 8)));
  const uint8_t* s = b + 4;
  const uint8_t* qh = b + 16;
  const uint8_t* qs = b + 48;
  for (int g = 0; g < 8; ++g) {
    int sc, m;
    q4k_scale_min(s, g, &sc, &m);
    float dsc = d * (float)sc;
    float dm = dmin * (float)m;
    for (int j = 0; j < 32; ++j) {
      int byte = qs[32 * (g / 2) + j];
      int q = ((g & 1) ? (byte >> 4) : (byte & 15)) | (((qh[j] >> g) & 1) << 4);
      volatile float prod = dsc * (float)q;
      out[32 * g + j] = prod - dm;
    }
  }
}

/* Q3_K: hmask[32] @0, qs[64] @32, scales[12] @96, d f16 @108. Element e = 128h + 32s + l (h < 2, s < 4, l < 32):
 * low = (qs[32h + l] >> 2s) & 3, hbit = (hmask[l] >> (4h + s)) & 1, q = low - 4 * (1 - hbit). Sub-block i = e/16:
 * sc = ((scales[i % 8] >> 4*(i / 8)) & 15 | ((scales[8 + i % 4] >> 2*(i / 4)) & 3) << 4) - 32. (d*sc)*q exact. */
static void sb_q3_k(const uint8_t* b, float* out) {
  const uint8_t* hm = b;
  const uint8_t* qs = b + 32;
  const uint8_t* sc = b + 96;
  float d = h2f((uint16_t)(b[108] | (b[109] << 8)));
  for (int e = 0; e < 256; ++e) {
    int h = e / 128, s = (e % 128) / 32, l = e % 32, i = e / 16;
    int low = (qs[32 * h + l] >> (2 * s)) & 3;
    int hbit = (hm[l] >> (4 * h + s)) & 1;
    int q = low - 4 * (1 - hbit);
    int scale = (((sc[i % 8] >> (4 * (i / 8))) & 15) | (((sc[8 + i % 4] >> (2 * (i / 4))) & 3) << 4)) - 32;
    volatile float dl = d * (float)scale;
    out[e] = dl * (float)q;
  }
}

/* IQ4_XS: d f16 @0, scales_h u16 @2, scales_l[4] @4, qs[128] @8. Group g (32 values): value w < 16 is the low nibble
 * of qs[16g + w], w >= 16 the high nibble of qs[16g + w - 16]; sc = ((scales_l[g/2] >> 4*(g%2)) & 15 |
 * ((scales_h >> 2g) & 3) << 4) - 32; w = (d*sc) * kvalues[nibble] (exact in f32). */
static const int8_t kIq4Values[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
static void sb_iq4_xs(const uint8_t* b, float* out) {
  float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
  int sh = b[2] | (b[3] << 8);
  const uint8_t* sl = b + 4;
  const uint8_t* qs = b + 8;
  for (int g = 0; g < 8; ++g) {
    int scale = (((sl[g / 2] >> (4 * (g % 2))) & 15) | (((sh >> (2 * g)) & 3) << 4)) - 32;
    volatile float dl = d * (float)scale;
    for (int w = 0; w < 32; ++w) {
      int byte = qs[16 * g + (w & 15)];
      int nib = w < 16 ? (byte & 15) : (byte >> 4);
      out[32 * g + w] = dl * (float)kIq4Values[nib];
    }
  }
}

static int sb_bytes(int type) {
  switch (type) {
    case T_Q8_0: return 272;
    case T_Q3_K: return 110;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_IQ4_XS: return 136;
    default: return 0;
  }
}

static void sb_decode(int type, const uint8_t* b, float* out) {
  switch (type) {
    case T_Q8_0: sb_q8_0(b, out); break;
    case T_Q3_K: sb_q3_k(b, out); break;
    case T_Q4_K: sb_q4_k(b, out); break;
    case T_Q5_K: sb_q5_k(b, out); break;
    case T_Q6_K: sb_q6_k(b, out); break;
    case T_IQ4_XS: sb_iq4_xs(b, out); break;
  }
}

/* Public: bytes of one 256-element super-block (0 for an unsupported type). */
int yah_oracle_superblock_bytes(int type) { return sb_bytes(type); }

/* Public: decode rows x K values of a GGUF weight (rows at row_stride bytes; K a multiple of 256; the K window
 * starts at super-block kb_off of each row) to f32. out is [rows][K]. Returns 0, or -1 on bad arguments. */
int yah_oracle_dequant_f32(int type, const void* w, int64_t rows, int64_t K, int64_t row_stride, int64_t kb_off,
                           float* out) {
  int bb = sb_bytes(type);
  if (!bb || K % 256) return -1;
  for (int64_t r = 0; r < rows; ++r) {
    const uint8_t* row = (const uint8_t*)w + r * row_stride + kb_off * bb;
    for (int64_t sb = 0; sb < K / 256; ++sb) sb_decode(type, row + sb * bb, out + r * K + sb * 256);
  }
  return 0;
}

/* Public: as yah_oracle_dequant_f32, each value rounded once to f16 (bit patterns). */
int yah_oracle_dequant_f16(int type, const void* w, int64_t rows, int64_t K, int64_t row_stride, int64_t kb_off,
                           uint16_t* out) {
  int bb = sb_bytes(type);
  float tmp[256];
  if (!bb || K % 256) return -1;
  for (int64_t r = 0; r < rows; ++r) {
    const uint8_t* row = (const uint8_t*)w + r * row_stride + kb_off * bb;
    for (int64_t sb = 0; sb < K / 256; ++sb) {
      sb_decode(type, row + sb * bb, tmp);
      for (int i = 0; i < 256; ++i) out[r * K + sb * 256 + i] = f2h(tmp[i]);
    }
  }
  return 0;
}

/* Public: f32 -> f16 bit pattern (round to nearest even), for tests of the host-side helpers. */
uint16_t yah_oracle_f32_to_f16(float f) { return f2h(f); }
