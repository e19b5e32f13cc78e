// Bit-exact decode of one 64-value K block of a GGUF super-block into 32 packed f16 pairs.
//
// Output convention (shared by every caller): out[c], c = 0..31, holds the values at K offsets 2c (low half) and
// 2c + 1 (high half) of the 64-value block. This is also the TMEM layout of an A-operand stage for
// tcgen05.mma kind::f16: one 32-bit column holds two consecutive K elements of a row.
//
// Arithmetic (reference: engine/gpu/loom/tools/gen_gemm_decode.py; every value is the f32 value of the
// reference dequant rounded once to f16, bit-identical to gguf-py dequantize(...).astype(float16)):
//   Q8_0 (:1338-1378)  w = f16(d * q). d * q is exact (11 x 8 bits), so one f16 multiply (mul.rn.f16x2) of the
//                      exact f16 integer q gives the same single rounding.
//   Q4_K (:837-1069)   w = f16(fma(d*sc, q, -dmin*m)). d*sc and dmin*m are exact in f32, d*sc*q is exact, so
//                      the f32 fma rounds once and the f16 conversion once, exactly as gguf-py's d*q - dm.
//                      q comes from a "magic float": (nibble << s) | 0x4B000000 is the float 2^23 + q*2^s, and
//                      subtracting 2^23 leaves q*2^s exactly; the matching scale d*sc*2^-s is exact too.
//   Q6_K (:1243-1335)  w = f16((d*sc) * (code - 32)) with d*sc and the product exact in f32 (int8 scales make
//                      sc*(code - 32) too wide for exact f16 arithmetic, so this one stays in f32).
//   Q5_K (:897-899, :1713-1716)  the Q4_K arithmetic with a 5-bit q (a fifth bit from the qh plane).
//   Q3_K (:1497-1546)  w = f16((d*sc) * q), sc = 6-bit scale - 32, q = (2-bit low | hmask bit << 2) - 4; exact f32.
//   IQ4_XS (:125-169)  w = f16((d*sc) * kvalues[nibble]), sc = 6-bit scale - 32; exact f32.
// Pairs of f32 values go through the sm_100 packed-FP32 instructions (fma/add/mul .rn.f32x2): the same IEEE
// operations, two per instruction.
#pragma once
#include "ptx.cuh"

namespace yah {

constexpr float kMagic23 = 8388608.0f;  // 2^23

__device__ __forceinline__ float magic_q(uint32_t bits) { return __uint_as_float(bits | 0x4B000000u) - kMagic23; }

__device__ __forceinline__ float h2f_bits(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// ------------------------------------------------------------------------------------------------ Q4_K
// hdr: the 16-byte block header (d | dmin << 16, scales[0..11]); qs: the 32 qs bytes of K block j (qs[32j..32j+31]).
__device__ __forceinline__ void q4k_scales(const uint4& hdr, int j, float& dsa, float& dma, float& dsb, float& dmb) {
  const float d = h2f_bits(hdr.x & 0xFFFFu);
  const float dmin = h2f_bits(hdr.x >> 16);
  // groups 2j (low nibbles) and 2j + 1 (high nibbles); s = scales bytes, w1 = s0..3, w2 = s4..7, w3 = s8..11
  int sc[2], m[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int g = 2 * j + u;
    const int gg = g & 3;
    const uint32_t b1 = (hdr.y >> (8 * gg)) & 0xFFu;
    const uint32_t b2 = (hdr.z >> (8 * gg)) & 0xFFu;
    const uint32_t b3 = (hdr.w >> (8 * gg)) & 0xFFu;
    if (g < 4) {
      sc[u] = b1 & 63;
      m[u] = b2 & 63;
    } else {
      sc[u] = (b3 & 15) | ((b1 >> 6) << 4);
      m[u] = (b3 >> 4) | ((b2 >> 6) << 4);
    }
  }
  dsa = d * (float)sc[0];
  dma = dmin * (float)m[0];
  dsb = d * (float)sc[1];
  dmb = dmin * (float)m[1];
}

// Two f32 lanes at once (sm_100 packed FP32): d = a * b + c and d = a + b on register pairs.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 A, B, C, D;\n\tmov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\tmov.b64 C, {%6, %7};\n\t"
      "fma.rn.f32x2 D, A, B, C;\n\tmov.b64 {%0, %1}, D;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 A, B, D;\n\tmov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\t"
      "add.rn.f32x2 D, A, B;\n\tmov.b64 {%0, %1}, D;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 A, B, D;\n\tmov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\t"
      "mul.rn.f32x2 D, A, B;\n\tmov.b64 {%0, %1}, D;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Two nibble-magic floats: (bits & m) | 0x4B000000 for two masks, minus 2^23 each (exact).
__device__ __forceinline__ float2 magic_pair(uint32_t w, uint32_t m0, uint32_t m1) {
  const float2 f = make_float2(__uint_as_float(lop_and_or(w, m0, 0x4B000000u)),
                               __uint_as_float(lop_and_or(w, m1, 0x4B000000u)));
  return fadd2(f, make_float2(-kMagic23, -kMagic23));
}

__device__ __forceinline__ uint32_t pack2(float2 v) { return pack_f16x2_rn(v.x, v.y); }

__device__ __forceinline__ void q4k_decode_kblock(const uint4& hdr, const uint32_t (&qs)[8], int j,
                                                  uint32_t (&out)[32]) {
  float dsa, dma, dsb, dmb;
  q4k_scales(hdr, j, dsa, dma, dsb, dmb);
  // group 2j (low nibbles at bits 0 / 8 of a half-word) and 2j+1 (high nibbles at bits 4 / 12)
  const float2 sa = make_float2(dsa, dsa * 0.00390625f);
  const float2 sb = make_float2(dsb * 0.0625f, dsb * 2.44140625e-4f);
  const float2 na = make_float2(-dma, -dma), nb = make_float2(-dmb, -dmb);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w = qs[i];
    const uint32_t v = w >> 16;
    // low nibbles: bytes 0,1 -> column 2i; bytes 2,3 -> column 2i+1; high nibbles -> columns 16+2i, 17+2i
    out[2 * i] = pack2(ffma2(sa, magic_pair(w, 0xFu, 0xF00u), na));
    out[2 * i + 1] = pack2(ffma2(sa, magic_pair(v, 0xFu, 0xF00u), na));
    out[16 + 2 * i] = pack2(ffma2(sb, magic_pair(w, 0xF0u, 0xF000u), nb));
    out[16 + 2 * i + 1] = pack2(ffma2(sb, magic_pair(v, 0xF0u, 0xF000u), nb));
  }
}

// ------------------------------------------------------------------------------------------------ Q8_0
// W[0..16]: the 68 bytes of K block j (blocks 2j and 2j+1 of the 272-byte super-block), starting 4-byte aligned.
__device__ __forceinline__ void q80_decode_kblock(const uint32_t (&W)[17], uint32_t (&out)[32]) {
  const uint32_t dA = W[0] & 0xFFFFu;
  const uint32_t dB = W[8] >> 16;
  const uint32_t dA2 = dA | (dA << 16), dB2 = dB | (dB << 16);
  constexpr uint32_t kBias = 0x64806480u;  // f16 (1152, 1152)
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    // block A value pair (2c, 2c+1) at region bytes 2 + 2c
    const int wa = (1 + c) >> 1;
    const uint32_t sela = (c & 1) ? 0x4140u : 0x4342u;
    const uint32_t pa = prmt(W[wa] ^ 0x80808080u, 0x64646464u, sela);
    out[c] = hmul2_u32(hsub2_u32(pa, kBias), dA2);
    // block B value pair at region bytes 36 + 2c
    const int wb = 9 + (c >> 1);
    const uint32_t selb = (c & 1) ? 0x4342u : 0x4140u;
    const uint32_t pb = prmt(W[wb] ^ 0x80808080u, 0x64646464u, selb);
    out[16 + c] = hmul2_u32(hsub2_u32(pb, kBias), dB2);
  }
}

// ------------------------------------------------------------------------------------------------ Q6_K
// QL: ql bytes [64h, 64h+64); QH: qh bytes [32h, 32h+32); SC: the 4 int8 scales sc[8h + 4(j&1) ...]; dbits: d.
// j = 2h + (j&1) is the K block within the super-block.
// Arithmetic in f32, as the reference: ds = d * sc (exact), q = code - 32 (exact), w = f16(ds * q) with the
// product exact (<= 23 bits) and IEEE zero signs identical to gguf-py's (d * scales) * q. The code byte is moved
// to bits 16..21 of the magic float 2^23 (one prmt); subtracting 2^23 + 32 * 2^16 leaves (code - 32) * 2^16, and
// the matching scale ds * 2^-16 is exact.
__device__ __forceinline__ void q6k_decode_kblock(const uint32_t (&QL)[16], const uint32_t (&QH)[8], uint32_t SC,
                                                  uint32_t dbits, int jodd, uint32_t (&out)[32]) {
  const float d = h2f_bits(dbits & 0xFFFFu);
  float ds[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int s = (int)(int8_t)((SC >> (8 * u)) & 0xFFu);
    ds[u] = (d * (float)s) * 1.52587890625e-05f;  // * 2^-16, exact
  }
  constexpr float kOff = 10485760.0f;  // 2^23 + 32 * 2^16
  const float2 off = make_float2(-kOff, -kOff);
  const int lsh = 4 * jodd;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t lo4 = (QL[i] >> lsh) & 0x0F0F0F0Fu;
    const uint32_t hi2 = (QH[i & 7] >> (lsh + 2 * (i >> 3))) & 0x03030303u;
    const uint32_t code = lo4 | (hi2 << 4);
    const float2 s2 = make_float2(ds[i >> 2], ds[i >> 2]);
    const float2 c01 = fadd2(make_float2(__uint_as_float(prmt(code, 0x4B000000u, 0x7044u)),
                                         __uint_as_float(prmt(code, 0x4B000000u, 0x7144u))), off);
    const float2 c23 = fadd2(make_float2(__uint_as_float(prmt(code, 0x4B000000u, 0x7244u)),
                                         __uint_as_float(prmt(code, 0x4B000000u, 0x7344u))), off);
    out[2 * i] = pack2(fmul2(s2, c01));
    out[2 * i + 1] = pack2(fmul2(s2, c23));
  }
}

// ------------------------------------------------------------------------------------------------ Q5_K
// hdr: the Q4_K header (d, dmin, scales[12]); qs: qs bytes [32j, 32j + 32); qh: the 32 qh bytes. Group 2j takes the
// low nibbles and qh bit 2j, group 2j + 1 the high nibbles and qh bit 2j + 1 (gguf-py Q5_K: q = ql | qh_bit << 4).
__device__ __forceinline__ void q5k_decode_kblock(const uint4& hdr, const uint32_t (&qs)[8], const uint32_t (&qh)[8],
                                                  int j, uint32_t (&out)[32]) {
  float dsa, dma, dsb, dmb;
  q4k_scales(hdr, j, dsa, dma, dsb, dmb);
  // 5-bit q of bytes 0 / 1 (or 2 / 3) as magic floats q and 256 q, so the scales are (d*sc, d*sc / 256)
  const float2 sa = make_float2(dsa, dsa * 0.00390625f), sb = make_float2(dsb, dsb * 0.00390625f);
  const float2 na = make_float2(-dma, -dma), nb = make_float2(-dmb, -dmb);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t hb = qh[i] >> (2 * j);
    const uint32_t lo = (qs[i] & 0x0F0F0F0Fu) | ((hb << 4) & 0x10101010u);
    const uint32_t hi = ((qs[i] >> 4) & 0x0F0F0F0Fu) | ((hb << 3) & 0x10101010u);
    out[2 * i] = pack2(ffma2(sa, magic_pair(lo, 0x1Fu, 0x1F00u), na));
    out[2 * i + 1] = pack2(ffma2(sa, magic_pair(lo >> 16, 0x1Fu, 0x1F00u), na));
    out[16 + 2 * i] = pack2(ffma2(sb, magic_pair(hi, 0x1Fu, 0x1F00u), nb));
    out[16 + 2 * i + 1] = pack2(ffma2(sb, magic_pair(hi >> 16, 0x1Fu, 0x1F00u), nb));
  }
}

// A byte b of `code` (b = 0..3) as the f32 2^23 + code_b * 2^16.
__device__ __forceinline__ float magic_hi_byte(uint32_t code, int b) {
  return __uint_as_float(prmt(code, 0x4B000000u, 0x7044u | ((uint32_t)b << 8)));
}

// Four bytes c_b < 128 (+ a bias folded into `off`) times a scale, as two f16 pairs: values (c_b * 2^16 - off) * s,
// with s = ds * 2^-16 (exact: the products are exact in f32, so one rounding to f16 as the reference). c_b must stay
// below 128: bit 7 would land in the magic float's exponent.
__device__ __forceinline__ void scaled_bytes(uint32_t code, float2 s, float off, uint32_t& p01, uint32_t& p23) {
  const float2 o = make_float2(-off, -off);
  const float2 c01 = fadd2(make_float2(magic_hi_byte(code, 0), magic_hi_byte(code, 1)), o);
  const float2 c23 = fadd2(make_float2(magic_hi_byte(code, 2), magic_hi_byte(code, 3)), o);
  p01 = pack2(fmul2(s, c01));
  p23 = pack2(fmul2(s, c23));
}

// ------------------------------------------------------------------------------------------------ Q3_K
// QS: qs bytes [32h, 32h + 32) (h = j / 2); HM: the 32 hmask bytes; LW: scale bytes [4(j % 2), 4(j % 2) + 4); HW:
// scale bytes [8, 12); dbits: d. Values c = 32t + l (t = 0, 1; l < 32) of K block j: shift s = 2(j % 2) + t, hmask
// bit 4h + s, sub-block 4j + 2t + l / 16.
__device__ __forceinline__ void q3k_decode_kblock(const uint32_t (&QS)[8], const uint32_t (&HM)[8], uint32_t LW,
                                                  uint32_t HW, uint32_t dbits, int j, uint32_t (&out)[32]) {
  const float d = h2f_bits(dbits & 0xFFFFu);
  const uint32_t sc = ((LW >> (4 * (j >> 1))) & 0x0F0F0F0Fu) | (((HW >> (2 * j)) & 0x03030303u) << 4);
  float ds[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) ds[u] = (d * (float)((int)((sc >> (8 * u)) & 0xFFu) - 32)) * 1.52587890625e-05f;
  constexpr float kOff = 8650752.0f;  // 2^23 + 4 * 2^16: byte (q + 4) -> q * 2^16
  const int h = j >> 1;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int s = 2 * (j & 1) + t;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t code = ((QS[i] >> (2 * s)) & 0x03030303u) | (((HM[i] >> (4 * h + s)) & 0x01010101u) << 2);
      const float f = ds[2 * t + (i >> 2)];
      scaled_bytes(code, make_float2(f, f), kOff, out[16 * t + 2 * i], out[16 * t + 2 * i + 1]);
    }
  }
}

// ------------------------------------------------------------------------------------------------ IQ4_XS
// Four nibbles (the low 4 bits of each byte of n) to the bytes kvalues[nibble] + 128 of the IQ4_NL level table
// {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113}: two 8-entry byte permutes, chosen per
// byte by the nibble's bit 3.
__device__ __forceinline__ uint32_t iq4_levels(uint32_t n) {
  constexpr uint32_t kT0 = 0x3F2D1801u, kT1 = 0x766A5D4Fu, kT2 = 0xA6998D81u, kT3 = 0xF1D9C5B5u;
  const uint32_t y = n | (n >> 4);                        // byte 0: n0 | n1 << 4, byte 2: n2 | n3 << 4
  const uint32_t sel = prmt(y, 0u, 0x4420u) & 0x7777u;    // n0 | n1 << 4 | n2 << 8 | n3 << 12, each mod 8
  const uint32_t lo = prmt(kT0, kT1, sel), hi = prmt(kT2, kT3, sel);
  const uint32_t m = prmt(n << 4, 0u, 0xBA98u);           // 0xFF in the bytes whose nibble has bit 3 set
  return (hi & m) | (lo & ~m);
}

// Four bytes (level + 128, up to 241: too wide for the 2^23 magic float's byte slot) times the group scale ds, as
// two f16 pairs: each level is an exact f16 (1024 + byte - 1152), widened to f32, and ds * level is exact in f32.
__device__ __forceinline__ void scaled_levels(uint32_t u, float2 ds, uint32_t& p01, uint32_t& p23) {
  const uint32_t a = hsub2_u32(prmt(u, 0x64646464u, 0x4140u), 0x64806480u);  // bytes 0, 1
  const uint32_t b = hsub2_u32(prmt(u, 0x64646464u, 0x4342u), 0x64806480u);  // bytes 2, 3
  p01 = pack2(fmul2(ds, __half22float2(*reinterpret_cast<const __half2*>(&a))));
  p23 = pack2(fmul2(ds, __half22float2(*reinterpret_cast<const __half2*>(&b))));
}

// H: bytes [0, 8) of the super-block (d, scales_h, scales_l[4]); QS: qs bytes [32j, 32j + 32) (groups 2j, 2j + 1).
// Group g = 2j + t: values 0..15 the low nibbles of its 16 bytes, 16..31 the high nibbles.
__device__ __forceinline__ void iq4xs_decode_kblock(uint2 H, const uint32_t (&QS)[8], int j, uint32_t (&out)[32]) {
  const float d = h2f_bits(H.x & 0xFFFFu);
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int g = 2 * j + t;
    const int sl = (int)((H.y >> (8 * j + 4 * t)) & 15u), sh = (int)((H.x >> (16 + 2 * g)) & 3u);
    const float f = d * (float)((sl | (sh << 4)) - 32);
    const float2 s2 = make_float2(f, f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t w = QS[4 * t + i];
      scaled_levels(iq4_levels(w & 0x0F0F0F0Fu), s2, out[16 * t + 2 * i], out[16 * t + 2 * i + 1]);
      scaled_levels(iq4_levels((w >> 4) & 0x0F0F0F0Fu), s2, out[16 * t + 8 + 2 * i], out[16 * t + 9 + 2 * i]);
    }
  }
}

// ------------------------------------------------------------------------------------------------ shared-memory
// Readers of one weight row of a staged super-block (the tile GEMM's TMA weight stage). `rb` is the shared address
// of the row's first staged byte (16-byte aligned).

__device__ __forceinline__ void q4k_decode_smem(uint32_t rb, int j, uint32_t (&out)[32]) {
  const uint4 hdr = lds128(rb);
  const uint4 a = lds128(rb + 16 + 32 * j);
  const uint4 b = lds128(rb + 32 + 32 * j);
  const uint32_t qs[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  q4k_decode_kblock(hdr, qs, j, out);
}

template <int J>
__device__ __forceinline__ void q80_decode_smem_j(uint32_t rb, uint32_t (&out)[32]) {
  uint32_t L[20];
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    const uint4 v = lds128(rb + 64 * J + 16 * c);
    L[4 * c] = v.x;
    L[4 * c + 1] = v.y;
    L[4 * c + 2] = v.z;
    L[4 * c + 3] = v.w;
  }
  uint32_t W[17];
#pragma unroll
  for (int i = 0; i < 17; ++i) W[i] = L[i + J];
  q80_decode_kblock(W, out);
}

__device__ __forceinline__ void q80_decode_smem(uint32_t rb, int j, uint32_t (&out)[32]) {
  switch (j) {
    case 0: q80_decode_smem_j<0>(rb, out); break;
    case 1: q80_decode_smem_j<1>(rb, out); break;
    case 2: q80_decode_smem_j<2>(rb, out); break;
    default: q80_decode_smem_j<3>(rb, out); break;
  }
}

// Q6_K rows are staged as a 224-byte window starting at the 16-byte boundary at or below the super-block, which
// then begins at byte o = 4*OW + 2*odd2 of the window (o even, 0..14). The row's stage slot is followed by at least
// 16 readable bytes (the stage is padded), so the one-word over-read at the window's end stays in shared memory.
template <int OW>
__device__ __forceinline__ void q6k_decode_smem_o(uint32_t rb, int j, uint32_t sel, uint32_t (&out)[32]) {
  const int h = j >> 1, jodd = j & 1;
  uint32_t L[20];
#pragma unroll
  for (int c = 0; c < 5; ++c) {
    const uint4 v = lds128(rb + 64 * h + 16 * c);
    L[4 * c] = v.x;
    L[4 * c + 1] = v.y;
    L[4 * c + 2] = v.z;
    L[4 * c + 3] = v.w;
  }
  uint32_t QL[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) QL[i] = prmt(L[OW + i], L[OW + i + 1], sel);
  uint32_t M[12];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const uint4 v = lds128(rb + 128 + 32 * h + 16 * c);
    M[4 * c] = v.x;
    M[4 * c + 1] = v.y;
    M[4 * c + 2] = v.z;
    M[4 * c + 3] = v.w;
  }
  uint32_t QH[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) QH[i] = prmt(M[OW + i], M[OW + i + 1], sel);
  const int ws = OW + 2 * h + jodd;  // word of the 4 scales, relative to byte 192
  const uint32_t SC = prmt(lds32(rb + 192 + 4 * ws), lds32(rb + 196 + 4 * ws), sel);
  const uint32_t D = prmt(lds32(rb + 208 + 4 * OW), lds32(rb + 212 + 4 * OW), sel);
  q6k_decode_kblock(QL, QH, SC, D, jodd, out);
}

__device__ __forceinline__ void q6k_decode_smem(uint32_t rb, int j, int o, uint32_t (&out)[32]) {
  const uint32_t sel = (o & 2) ? 0x5432u : 0x3210u;
  switch (o >> 2) {
    case 0: q6k_decode_smem_o<0>(rb, j, sel, out); break;
    case 1: q6k_decode_smem_o<1>(rb, j, sel, out); break;
    case 2: q6k_decode_smem_o<2>(rb, j, sel, out); break;
    default: q6k_decode_smem_o<3>(rb, j, sel, out); break;
  }
}

__device__ __forceinline__ void q5k_decode_smem(uint32_t rb, int j, uint32_t (&out)[32]) {
  const uint4 hdr = lds128(rb);
  const uint4 h0 = lds128(rb + 16), h1 = lds128(rb + 32);
  const uint4 a = lds128(rb + 48 + 32 * j), b = lds128(rb + 64 + 32 * j);
  const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint32_t qs[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  q5k_decode_kblock(hdr, qs, qh, j, out);
}

// Q3_K rows are staged as a 128-byte window from the 16-byte boundary at or below the super-block, which begins at
// byte o = 4*OW + 2*odd2 of the window (o even, 0..14; o + 110 <= 124). Words at even byte offsets come from two
// aligned words and one prmt (sel picks the half-word shift).
template <int OW>
__device__ __forceinline__ void q3k_decode_smem_o(uint32_t rb, int j, uint32_t sel, uint32_t (&out)[32]) {
  const int h = j >> 1;
  uint32_t L[12];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const uint4 v = lds128(rb + 32 + 32 * h + 16 * c);  // qs bytes 32h .. at window byte 32 + 32h + o
    L[4 * c] = v.x;
    L[4 * c + 1] = v.y;
    L[4 * c + 2] = v.z;
    L[4 * c + 3] = v.w;
  }
  uint32_t QS[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) QS[i] = prmt(L[OW + i], L[OW + i + 1], sel);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const uint4 v = lds128(rb + 16 * c);  // hmask bytes 0..31
    L[4 * c] = v.x;
    L[4 * c + 1] = v.y;
    L[4 * c + 2] = v.z;
    L[4 * c + 3] = v.w;
  }
  uint32_t HM[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) HM[i] = prmt(L[OW + i], L[OW + i + 1], sel);
  const uint32_t lw = prmt(lds32(rb + 96 + 4 * (OW + (j & 1))), lds32(rb + 100 + 4 * (OW + (j & 1))), sel);
  const uint32_t hw = prmt(lds32(rb + 104 + 4 * OW), lds32(rb + 108 + 4 * OW), sel);
  const uint32_t D = prmt(lds32(rb + 108 + 4 * OW), lds32(rb + 112 + 4 * OW), sel);
  q3k_decode_kblock(QS, HM, lw, hw, D, j, out);
}

__device__ __forceinline__ void q3k_decode_smem(uint32_t rb, int j, int o, uint32_t (&out)[32]) {
  const uint32_t sel = (o & 2) ? 0x5432u : 0x3210u;
  switch (o >> 2) {
    case 0: q3k_decode_smem_o<0>(rb, j, sel, out); break;
    case 1: q3k_decode_smem_o<1>(rb, j, sel, out); break;
    case 2: q3k_decode_smem_o<2>(rb, j, sel, out); break;
    default: q3k_decode_smem_o<3>(rb, j, sel, out); break;
  }
}

// IQ4_XS rows are staged as a 144-byte window from the 16-byte boundary at or below the super-block, which begins
// at byte o = 0 or 8 of the window (super-blocks are 8-byte aligned).
__device__ __forceinline__ void iq4xs_decode_smem(uint32_t rb, int j, int o, uint32_t (&out)[32]) {
  const uint32_t b = rb + o;
  const uint2 H = lds64(b);
  uint32_t QS[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint2 v = lds64(b + 8 + 32 * j + 8 * i);
    QS[2 * i] = v.x;
    QS[2 * i + 1] = v.y;
  }
  iq4xs_decode_kblock(H, QS, j, out);
}

// ------------------------------------------------------------------------------------------------ global memory
// A 32-bit little-endian word at a 2-byte aligned global address (read-only path).
__device__ __forceinline__ uint32_t ldg_word2(const uint8_t* p) {
  const unsigned short lo = __ldg(reinterpret_cast<const unsigned short*>(p));
  const unsigned short hi = __ldg(reinterpret_cast<const unsigned short*>(p + 2));
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// Decode K block j of the super-block at `sb` (global, 2-byte aligned) of format T.
template <int T>
__device__ __forceinline__ void decode_global(const uint8_t* sb, int j, uint32_t (&out)[32]);

template <>
__device__ __forceinline__ void decode_global<12>(const uint8_t* sb, int j, uint32_t (&out)[32]) {
  uint4 hdr;
  hdr.x = ldg_word2(sb);
  hdr.y = ldg_word2(sb + 4);
  hdr.z = ldg_word2(sb + 8);
  hdr.w = ldg_word2(sb + 12);
  uint32_t qs[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) qs[i] = ldg_word2(sb + 16 + 32 * j + 4 * i);
  q4k_decode_kblock(hdr, qs, j, out);
}

template <>
__device__ __forceinline__ void decode_global<8>(const uint8_t* sb, int j, uint32_t (&out)[32]) {
  uint32_t W[17];
#pragma unroll
  for (int i = 0; i < 17; ++i) W[i] = ldg_word2(sb + 68 * j + 4 * i);
  q80_decode_kblock(W, out);
}

template <>
__device__ __forceinline__ void decode_global<14>(const uint8_t* sb, int j, uint32_t (&out)[32]) {
  const int h = j >> 1, jodd = j & 1;
  uint32_t QL[16], QH[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) QL[i] = ldg_word2(sb + 64 * h + 4 * i);
#pragma unroll
  for (int i = 0; i < 8; ++i) QH[i] = ldg_word2(sb + 128 + 32 * h + 4 * i);
  const uint32_t SC = ldg_word2(sb + 192 + 8 * h + 4 * jodd);
  const uint32_t D = __ldg(reinterpret_cast<const unsigned short*>(sb + 208));
  q6k_decode_kblock(QL, QH, SC, D, jodd, out);
}

template <>
__device__ __forceinline__ void decode_global<13>(const uint8_t* sb, int j, uint32_t (&out)[32]) {
  uint4 hdr;
  hdr.x = ldg_word2(sb);
  hdr.y = ldg_word2(sb + 4);
  hdr.z = ldg_word2(sb + 8);
  hdr.w = ldg_word2(sb + 12);
  uint32_t qh[8], qs[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) qh[i] = ldg_word2(sb + 16 + 4 * i), qs[i] = ldg_word2(sb + 48 + 32 * j + 4 * i);
  q5k_decode_kblock(hdr, qs, qh, j, out);
}

template <>
__device__ __forceinline__ void decode_global<11>(const uint8_t* sb, int j, uint32_t (&out)[32]) {
  const int h = j >> 1;
  uint32_t QS[8], HM[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) QS[i] = ldg_word2(sb + 32 + 32 * h + 4 * i), HM[i] = ldg_word2(sb + 4 * i);
  const uint32_t lw = ldg_word2(sb + 96 + 4 * (j & 1)), hw = ldg_word2(sb + 104);
  const uint32_t D = __ldg(reinterpret_cast<const unsigned short*>(sb + 108));
  q3k_decode_kblock(QS, HM, lw, hw, D, j, out);
}

template <>
__device__ __forceinline__ void decode_global<23>(const uint8_t* sb, int j, uint32_t (&out)[32]) {
  const uint2 H = make_uint2(ldg_word2(sb), ldg_word2(sb + 4));
  uint32_t QS[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) QS[i] = ldg_word2(sb + 8 + 32 * j + 4 * i);
  iq4xs_decode_kblock(H, QS, j, out);
}

__host__ __device__ constexpr int superblock_bytes(int T) {
  return T == 8 ? 272 : T == 11 ? 110 : T == 12 ? 144 : T == 13 ? 176 : T == 14 ? 210 : T == 23 ? 136 : 0;
}

}  // namespace yah
