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
 *   - engine/core/gguf.cpp:27-35                           block sizes (Q8_0 32/34, Q4_K 256/144, Q6_K 256/210)
 * The arithmetic matches gguf-py 0.19.0 (gguf/quants.py Q8_0/Q4_K/Q6_K.dequantize_blocks) followed by
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

enum { T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

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

static int sb_bytes(int type) {
  switch (type) {
    case T_Q8_0: return 272;
    case T_Q4_K: return 144;
    case T_Q6_K: return 210;
    default: return 0;
  }
}

static void sb_decode(int type, const uint8_t* b, float* out) {
  switch (type) {
    case T_Q8_0: sb_q8_0(b, out); break;
    case T_Q4_K: sb_q4_k(b, out); break;
    case T_Q6_K: sb_q6_k(b, out); break;
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
