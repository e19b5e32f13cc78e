// Decode GEMV for M <= 32 tokens: y[t][n] (+)= sum_k W[n][k] x[t][k], GGUF weights, f16 activations.
// Formats: Q8_0, Q4_K, Q6_K, and on the same kernel Q5_K (the Q4_K form with a fifth bit per quant from the qh
// plane), Q3_K (the Q6_K form: exact small integers per 16-value sub-block) and IQ4_XS (levels of its non-linear
// table as exact f16 integers, one scale per 32 values); reference GEMV lane setups gen_gemv.py:137-230.
//
// Reference: engine/gpu/loom/tools/gen_gemv.py (kinds plain / resid, :96-754). Like the reference GEMV, this
// kernel never rounds a dequantised weight: it computes with the f32 weight values of the reference dequant
// (gguf-py dequantize, the reference GEMV's oracle, gemv_check.py:112, 161) through the algebra
// `scale * dot(q, x) - offset * sum(x)` (gen_gemv.py:7-9), with small integers on the tensor cores:
//   Q4_K  w = d*sc*q - dmin*m. A nibble masked in place is an exact f16 subnormal (q * 2^-24 or q * 2^-20);
//         per 32-value group the MMA gives sum(q x), scaled back together with d * sc in one f32 FMA; the min
//         term - dmin * sum_g m_g X_g is one more MMA, X_g (the group's activation sum) in two f16 parts.
//   Q6_K  w = (d*sc)*(code - 32): one MMA per 16-value sub-block on the exact integers code - 32, then
//         y += (d*sc) * acc.
//   Q8_0  w = d*q: two MMAs per 32-value block on the exact int8 q, then y += d * acc.
// The reference GEMV is judged on bandwidth; so is this one.
//
// B200 design. mma.sync.m16n8k16 with the weights as A (16 rows per warp; a lane applies the scales of its rows
// g and g + 8) and the tokens as B. A stage holds RB weight rows x S super-blocks (one TMA copy per <= P
// super-blocks) plus the matching activations (one 3-D TMA copy: 4S 64-K chunks x M token rows, 128-byte
// swizzle); a TMA warp keeps up to 8 stages in flight. Compute warp w works on row group w % rgp (16 rows) and
// super-block slot (w / rgp) % S of every stage, and on its share of the tokens. For Q4_K a helper warp permutes
// each stage's activations to the order the nibble pairs come in ((x0, x2), (x1, x3)) and forms the group sums.
// Two ways to split the work over the GPU:
//   row ranges (N >= 16 * #SMs and M * K small enough that all activations stay in shared memory): CTA b owns a
//     contiguous range of ~N / #SMs rows (4-row granularity) and all of K; the slots of a row group are added
//     through shared memory. No scratch, balanced within 4 rows per SM.
//   stream-K (otherwise): 128-row blocks x super-blocks, cut into equal ranges per CTA; a row block shared by
//     several CTAs is summed through a workspace by the last CTA to arrive, in CTA order (deterministic).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "decode.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace yah {
namespace {

constexpr int kGvBlock = 128;    // stream-K row block
constexpr int kGvEarlyStages = 2;  // weight copies a programmatic launch issues before the preceding kernel ends
constexpr int kGvMaxStages = 16;
constexpr int kGvSmemBudget = 225 * 1024;

// Bytes per super-block and the most super-blocks one TMA copy of a row holds (box width <= 256 elements:
// u64 elements for Q4_K / Q8_0, u16 for Q6_K, whose super-blocks are not 8-byte aligned).
__host__ __device__ constexpr int gv_sb_bytes(int t) { return superblock_bytes(t); }
// Q4_K and Q5_K share the nibble-pair algebra: permuted activations and per-group activation sums.
__host__ __device__ constexpr bool gv_q4like(int t) { return t == 12 || t == 13; }
// Formats whose super-blocks are not all 16-byte aligned (Q6_K 210, Q3_K 110, IQ4_XS 136 bytes) are copied as u16
// windows from the 16-byte boundary at or below them; the others as whole u64 super-blocks.
__host__ __device__ constexpr bool gv_windowed(int t) { return t == 14 || t == 11 || t == 23; }
// Super-blocks per weight copy: a power of two (a stage of sst super-blocks, itself a power of two, is ops whole
// copies), and at most 256 box elements (u64 for whole super-blocks, u16 for windows of up to P * bytes + 14).
__host__ __device__ constexpr int gv_pmax(int t) { return t == 8 ? 4 : gv_q4like(t) ? 8 : t == 11 ? 4 : 2; }
// Shared-memory row width of one W copy of P super-blocks (Q6_K: a 16-byte aligned window around them), padded to
// an odd number of 16-byte units. TMA lays the copied rows out at this pitch; row g starts in 16-byte bank slot
// (g * units) mod 8, so gcd(units, 8) of the 8 rows a warp's lane groups read (g = 0..7) share a slot: none for an odd
// count, all 8 for 1152 bytes = 72 units (measured: half of all shared-load wavefronts were conflicts). The extra bytes
// are the start of the next super-block, or zero fill past the end of the row.
__host__ __device__ constexpr int gv_opw_raw(int t, int P) {
  return gv_windowed(t) ? ((P * gv_sb_bytes(t) + 14 + 15) / 16) * 16 : ((P * gv_sb_bytes(t) + 15) / 16) * 16;
}
__host__ __device__ constexpr int gv_opw(int t, int P) {
  return (gv_opw_raw(t, P) / 16) % 2 ? gv_opw_raw(t, P) : gv_opw_raw(t, P) + 16;
}

template <int T, int CW>
struct GvRoles {
  static constexpr int kThreads = (CW + (gv_q4like(T) ? 2 : 1)) * 32;  // compute warps + TMA warp (+ Q4_K helper)
};

struct GvParams {
  int N, M, kb_off, nsb;
  int mode;                  // 0 row ranges, 1 stream-K
  int rb, rgp, slots, tsplit, sst, P, ops, opw;  // sst: super-blocks per stage (a divisor of slots)
  int turns, ringst;         // stage rings: stage k of a segment goes to ring k % turns, ringst stages each
  int wreg, xoff, sumoff, stage_bytes, stages, redoff, baroff;
  int xres, resoff, ressum;  // activations resident for the whole launch (row ranges, small M * K)
  int xstride, sstride;      // resident layout: bytes per token of activations / of group sums
  int sbstride;              // resident layout: bytes per super-block of activations (512, or padded)
  const __half* x;
  const float* xf;           // f32 activations (xf32: M counts the hi / lo token rows, two per f32 token)
  int xf32;
  int64_t ldx;
  int K;
  int64_t units;             // row ranges: ceil(N / 4)
  int64_t items;             // stream-K: row blocks x super-blocks
  void* y;
  int64_t ldy;
  int y_f16, epi;
  const float* aux;
  int64_t ldaux;
  float* ws;                 // stream-K: [G][2][M][128] partial sums
  int* counters;             // stream-K: [row blocks][8], zero between launches
  int* status;
};

// ------------------------------------------------------------------------------------------------ small helpers
__device__ __forceinline__ uint32_t lds_word(uint32_t addr) {  // 4 bytes at an even byte address
  const uint32_t a = addr & ~3u;
  return prmt(lds32(a), lds32(a + 4), (addr & 2) ? 0x5432u : 0x3210u);
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  return (lds32(addr & ~3u) >> (8 * (addr & 3))) & 0xFFFFu;
}

// A pure register operation: plain asm, so the compiler may schedule it among the shared-memory loads.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Activations of a stage: 128-byte rows, row = chunk * rows_per_chunk + token, the 16-byte pieces of a row
// swizzled by (row mod 8) (TMA 128-byte swizzle; the stage's activation region is 1024-byte aligned).
// Address of 16-byte piece q of row `row`:
__device__ __forceinline__ uint32_t xpiece(uint32_t xs, int row, int q) {
  return xs + row * 128 + ((q ^ (row & 7)) << 4);
}

// u >> 8 as the high word of u * 2^24: a multiply, so it issues on the FMA pipe and leaves the integer/logic
// pipe (the busiest one in the Q4_K decode) to the nibble masks.
__device__ __forceinline__ uint32_t shr8_fma(uint32_t u) {
  uint32_t r;
  asm("mul.hi.u32 %0, %1, 16777216;" : "=r"(r) : "r"(u));
  return r;
}

// 4-byte word at an even offset, as f32 2^23 + byte (for the scale bytes of Q4_K)
__device__ __forceinline__ float magic_byte(uint32_t word, int byte) {
  return __uint_as_float(prmt(word, 0x4B000000u, (uint32_t)byte | 0x7650u));
}

// Where a super-block's activations and Q4_K group sums sit, seen from one lane (g = lane / 4, c = lane % 4).
// x(n, j, cb): byte cb of this lane's part of 64-K chunk j, token tile n; the lane part is 16c (Q4_K, pieces c and
// c + 4 = bytes 0 / 64) or 8c (Q6_K, Q8_0). shi / slo: the lane's two hi / lo group sums (groups 2c, 2c + 1).
// Token rows past M read token M - 1: they only feed D columns that are never stored.
//
// XStage: a stage written by TMA (row = chunk * xrows + token, 128-byte swizzle; sums [hi, lo][xrows][8] f16).
template <int NTW>
struct XStage {
  uint32_t xs, sums;
  int xrows, c0, lane_b, lane_s;
  int tok[NTW];
  __device__ __forceinline__ uint32_t x(int n, int j, int cb) const {
    const int row = (c0 + j) * xrows + tok[n], byte = cb + lane_b;
    return xs + row * 128 + ((((byte >> 4) ^ row) & 7) << 4) + (byte & 15);
  }
  __device__ __forceinline__ uint32_t shi(int n) const { return sums + tok[n] * 16 + lane_s; }
  __device__ __forceinline__ uint32_t slo(int n) const { return sums + (xrows + tok[n]) * 16 + lane_s; }
};

// XRes: resident activations in the launch-wide layout (token row t at t * xstride, chunk ch at ch * 128, no
// swizzle: xstride = 2K + 64 puts consecutive tokens in opposite bank halves; sums [token][super-block][hi 8, lo 8]).
// xu / su already hold this lane's offsets and this super-block's position, so every access is register + constant.
template <int NTW>
struct XRes {
  uint32_t xu[NTW], su[NTW];
  __device__ __forceinline__ uint32_t x(int n, int j, int cb) const { return xu[n] + j * 128 + cb; }
  __device__ __forceinline__ uint32_t shi(int n) const { return su[n]; }
  __device__ __forceinline__ uint32_t slo(int n) const { return su[n] + 16; }
};

// ------------------------------------------------------------------------------------------------ one super-block
// A warp's 16 weight rows x one 256-K super-block, accumulated into y (rows g / g + 8, tokens 8n + 2c + e of the
// warp's token tiles). w0 / w1: shared addresses of the super-block in rows g and g + 8; xa: its activations.
// The loads of a super-block are issued before its arithmetic (all of them for one token tile).
template <int T, int NTW, class XA>
__device__ __forceinline__ void gv_superblock(uint32_t w0, uint32_t w1, const XA& xa, float (&y)[NTW][4], int c) {
  if (gv_q4like(T)) {
    // Q5_K: the same header, qs at 48 and the qh plane at 16 (bit g of qh byte p: the fifth bit of position p of
    // group g); this lane's positions 8c .. 8c + 7 of every 32-value group read qh bytes 8c .. 8c + 7
    constexpr int kQs = T == 13 ? 48 : 16;
    const uint4 h0 = lds128(w0), h1 = lds128(w1);
    uint2 q0[4], q1[4], qh0 = make_uint2(0u, 0u), qh1 = make_uint2(0u, 0u);
#pragma unroll
    for (int j = 0; j < 4; ++j) q0[j] = lds64(w0 + kQs + 32 * j + 8 * c), q1[j] = lds64(w1 + kQs + 32 * j + 8 * c);
    if (T == 13) qh0 = lds64(w0 + 16 + 8 * c), qh1 = lds64(w1 + 16 + 8 * c);
    constexpr int PJ = NTW == 1 ? 4 : 1;  // 64-K chunks of activations loaded ahead
    uint4 xl[PJ][NTW], xh[PJ][NTW];
    uint32_t bh[NTW], bl[NTW];
    if (NTW == 1) {
#pragma unroll
      for (int j = 0; j < PJ; ++j) xl[j][0] = lds128(xa.x(0, j, 0)), xh[j][0] = lds128(xa.x(0, j, 64));
      bh[0] = lds32(xa.shi(0));
      bl[0] = lds32(xa.slo(0));
    }
    // 6-bit scales of groups 0-3 / 4-7 and mins of groups 0-3 / 4-7, one per byte
    const uint32_t sc0a = h0.y & 0x3F3F3F3Fu, sc0b = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t sc1a = h1.y & 0x3F3F3F3Fu, sc1b = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    // Low nibble q masked in place reads as q * 2^-24, high nibble as q * 2^-20 (exact f16 subnormals). The group
    // factor F = (2^23 + sc) * D - 2^23 * D = sc * D (one rounding) with D = d * 2^24 or d * 2^20 undoes that.
    const float d0 = h2f_bits(h0.x & 0xFFFFu), d1 = h2f_bits(h1.x & 0xFFFFu);
    const float dl0 = d0 * 16777216.0f, dh0 = d0 * 1048576.0f, dl1 = d1 * 16777216.0f, dh1 = d1 * 1048576.0f;
    const float bl0 = dl0 * -8388608.0f, bh0 = dh0 * -8388608.0f, bl1 = dl1 * -8388608.0f, bh1 = dh1 * -8388608.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int jx = NTW == 1 ? j : 0;
      if (NTW > 1) {
#pragma unroll
        for (int n = 0; n < NTW; ++n) xl[0][n] = lds128(xa.x(n, j, 0)), xh[0][n] = lds128(xa.x(n, j, 64));
      }
      // lane bytes 8c .. 8c + 7 of the 64-K block: low nibbles at positions 8c + (0..7) (group 2j), high nibbles
      // at 32 + 8c + (0..7) (group 2j + 1)
      const uint32_t s0 = j < 2 ? sc0a : sc0b, s1 = j < 2 ? sc1a : sc1b;
      const float fl0 = __fmaf_rn(magic_byte(s0, (2 * j) & 3), dl0, bl0);
      const float fh0 = __fmaf_rn(magic_byte(s0, (2 * j + 1) & 3), dh0, bh0);
      const float fl1 = __fmaf_rn(magic_byte(s1, (2 * j) & 3), dl1, bl1);
      const float fh1 = __fmaf_rn(magic_byte(s1, (2 * j + 1) & 3), dh1, bh1);
      // A registers: word wi, bytes (0, 2) and (1, 3) of rows g and g + 8, low / high nibbles
      uint32_t lo[2][4], hi[2][4];
#pragma unroll
      for (int wi = 0; wi < 2; ++wi) {
        const uint32_t u0 = wi ? q0[j].y : q0[j].x, u1 = wi ? q1[j].y : q1[j].x;
        const uint32_t v0 = shr8_fma(u0), v1 = shr8_fma(u1);
        lo[wi][0] = u0 & 0x000F000Fu, lo[wi][1] = u1 & 0x000F000Fu, lo[wi][2] = v0 & 0x000F000Fu,
        lo[wi][3] = v1 & 0x000F000Fu;
        hi[wi][0] = u0 & 0x00F000F0u, hi[wi][1] = u1 & 0x00F000F0u, hi[wi][2] = v0 & 0x00F000F0u,
        hi[wi][3] = v1 & 0x00F000F0u;
        if (T == 13) {
          // fifth bits: group 2j (low nibbles, q * 2^-24 -> bit 4 of the half) and 2j + 1 (high, bit 8);
          // bytes 0 / 2 of the word in halves 0 / 1 of lo[.][0..1], bytes 1 / 3 in lo[.][2..3]
          const uint32_t e0 = (wi ? qh0.y : qh0.x) >> (2 * j), e1 = (wi ? qh1.y : qh1.x) >> (2 * j);
          lo[wi][0] |= (e0 << 4) & 0x00100010u, lo[wi][1] |= (e1 << 4) & 0x00100010u;
          lo[wi][2] |= (e0 >> 4) & 0x00100010u, lo[wi][3] |= (e1 >> 4) & 0x00100010u;
          hi[wi][0] |= (e0 << 7) & 0x01000100u, hi[wi][1] |= (e1 << 7) & 0x01000100u;
          hi[wi][2] |= (e0 >> 1) & 0x01000100u, hi[wi][3] |= (e1 >> 1) & 0x01000100u;
        }
      }
#pragma unroll
      for (int n = 0; n < NTW; ++n) {
        // permuted activations: 16-byte piece c = units 2c, 2c + 1 (low nibbles), piece 4 + c (high nibbles)
        const uint4 a = xl[jx][NTW == 1 ? 0 : n], b = xh[jx][NTW == 1 ? 0 : n];
        float alo[4] = {0.f, 0.f, 0.f, 0.f}, ahi[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(alo, lo[0][0], lo[0][1], lo[0][2], lo[0][3], a.x, a.y);
        mma16816(ahi, hi[0][0], hi[0][1], hi[0][2], hi[0][3], b.x, b.y);
        mma16816(alo, lo[1][0], lo[1][1], lo[1][2], lo[1][3], a.z, a.w);
        mma16816(ahi, hi[1][0], hi[1][1], hi[1][2], hi[1][3], b.z, b.w);
        y[n][0] = __fmaf_rn(fh0, ahi[0], __fmaf_rn(fl0, alo[0], y[n][0]));
        y[n][1] = __fmaf_rn(fh0, ahi[1], __fmaf_rn(fl0, alo[1], y[n][1]));
        y[n][2] = __fmaf_rn(fh1, ahi[2], __fmaf_rn(fl1, alo[2], y[n][2]));
        y[n][3] = __fmaf_rn(fh1, ahi[3], __fmaf_rn(fl1, alo[3], y[n][3]));
      }
    }
    // - dmin * sum_g m_g X_g: A row g / g + 8 = mins of groups 2c, 2c + 1 (repeated at k + 8), B = X hi / lo
    const uint32_t m0a = h0.z & 0x3F3F3F3Fu, m0b = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t m1a = h1.z & 0x3F3F3F3Fu, m1b = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    const int mb = (2 * c) & 3;
    const uint32_t msel = (uint32_t)mb | 0x40u | ((uint32_t)(mb + 1) << 8) | 0x4000u;
    const uint32_t am0 = hsub2_u32(prmt(c < 2 ? m0a : m0b, 0x64646464u, msel), 0x64006400u);
    const uint32_t am1 = hsub2_u32(prmt(c < 2 ? m1a : m1b, 0x64646464u, msel), 0x64006400u);
    const float n0 = -h2f_bits(h0.x >> 16), n1 = -h2f_bits(h1.x >> 16);
#pragma unroll
    for (int n = 0; n < NTW; ++n) {
      if (NTW > 1) bh[n] = lds32(xa.shi(n)), bl[n] = lds32(xa.slo(n));
      float acc2[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(acc2, am0, am1, am0, am1, bh[n], bl[n]);
      y[n][0] = __fmaf_rn(n0, acc2[0], y[n][0]);
      y[n][1] = __fmaf_rn(n0, acc2[1], y[n][1]);
      y[n][2] = __fmaf_rn(n1, acc2[2], y[n][2]);
      y[n][3] = __fmaf_rn(n1, acc2[3], y[n][3]);
    }
  } else if (T == 14) {
    // ql[128], qh[64], int8 scales[16], d; x in natural order: unit 4u + c of a 64-K chunk = 16-byte piece
    // 2u + (c >> 1), half c & 1 (byte 32u + 8c)
    const float dd0 = h2f_bits(lds_u16(w0 + 208)), dd1 = h2f_bits(lds_u16(w1 + 208));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int h = j >> 1, jo = j & 1;  // 128-value half, which 64 of it
      const uint32_t scw0 = lds_word(w0 + 192 + 8 * h + 4 * jo), scw1 = lds_word(w1 + 192 + 8 * h + 4 * jo);
      const uint32_t qh0[2] = {lds_word(w0 + 128 + 32 * h + 4 * c), lds_word(w0 + 144 + 32 * h + 4 * c)};
      const uint32_t qh1[2] = {lds_word(w1 + 128 + 32 * h + 4 * c), lds_word(w1 + 144 + 32 * h + 4 * c)};
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // 16-value sub-block u of the 64-K block (scale index 8h + 4jo + u)
        const uint32_t ql0 = lds_word(w0 + 64 * h + 16 * u + 4 * c), ql1 = lds_word(w1 + 64 * h + 16 * u + 4 * c);
        const int hs = 4 * jo + 2 * (u >> 1);
        const uint32_t c0w = ((ql0 >> (4 * jo)) & 0x0F0F0F0Fu) | (((qh0[u & 1] >> hs) & 0x03030303u) << 4);
        const uint32_t c1w = ((ql1 >> (4 * jo)) & 0x0F0F0F0Fu) | (((qh1[u & 1] >> hs) & 0x03030303u) << 4);
        constexpr uint32_t kB = 0x64206420u;  // f16 (1056, 1056) = 1024 + 32
        const uint32_t a0 = hsub2_u32(prmt(c0w, 0x64646464u, 0x4140u), kB);
        const uint32_t a2 = hsub2_u32(prmt(c0w, 0x64646464u, 0x4342u), kB);
        const uint32_t a1 = hsub2_u32(prmt(c1w, 0x64646464u, 0x4140u), kB);
        const uint32_t a3 = hsub2_u32(prmt(c1w, 0x64646464u, 0x4342u), kB);
        const float f0 = dd0 * (float)(int)(int8_t)((scw0 >> (8 * u)) & 0xFFu);
        const float f1 = dd1 * (float)(int)(int8_t)((scw1 >> (8 * u)) & 0xFFu);
#pragma unroll
        for (int n = 0; n < NTW; ++n) {
          const uint2 b = lds64(xa.x(n, j, 32 * u));
          float t4[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816(t4, a0, a1, a2, a3, b.x, b.y);
          y[n][0] = __fmaf_rn(f0, t4[0], y[n][0]);
          y[n][1] = __fmaf_rn(f0, t4[1], y[n][1]);
          y[n][2] = __fmaf_rn(f1, t4[2], y[n][2]);
          y[n][3] = __fmaf_rn(f1, t4[3], y[n][3]);
        }
      }
    }
  } else if (T == 11) {
    // Q3_K: hmask[32] @0, qs[64] @32, scales[12] @96, d @108 (a window: w0 / w1 at even offsets). Sub-block 4j + u
    // (16 values) of 64-K chunk j: 2-bit quants at shift s = 2(j % 2) + u / 2 of qs bytes 32h + 16(u % 2) + p
    // (h = j / 2), hmask bit 4h + s; q = (low | hbit << 2) - 4 as an exact f16, then y += d * (sc - 32) * acc.
    const float dd0 = h2f_bits(lds_u16(w0 + 108)), dd1 = h2f_bits(lds_u16(w1 + 108));
    const uint32_t hw0 = lds_word(w0 + 104), hw1 = lds_word(w1 + 104);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int h = j >> 1;
      const uint32_t lw0 = lds_word(w0 + 96 + 4 * (j & 1)), lw1 = lds_word(w1 + 96 + 4 * (j & 1));
      const uint32_t sc0 = ((lw0 >> (4 * h)) & 0x0F0F0F0Fu) | (((hw0 >> (2 * j)) & 0x03030303u) << 4);
      const uint32_t sc1 = ((lw1 >> (4 * h)) & 0x0F0F0F0Fu) | (((hw1 >> (2 * j)) & 0x03030303u) << 4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int s = 2 * (j & 1) + (u >> 1), lo16 = 16 * (u & 1) + 4 * c;
        const uint32_t c0w = ((lds_word(w0 + 32 + 32 * h + lo16) >> (2 * s)) & 0x03030303u) |
                             (((lds_word(w0 + lo16) >> (4 * h + s)) & 0x01010101u) << 2);
        const uint32_t c1w = ((lds_word(w1 + 32 + 32 * h + lo16) >> (2 * s)) & 0x03030303u) |
                             (((lds_word(w1 + lo16) >> (4 * h + s)) & 0x01010101u) << 2);
        constexpr uint32_t kB = 0x64046404u;  // f16 (1028, 1028) = 1024 + 4
        const uint32_t a0 = hsub2_u32(prmt(c0w, 0x64646464u, 0x4140u), kB);
        const uint32_t a2 = hsub2_u32(prmt(c0w, 0x64646464u, 0x4342u), kB);
        const uint32_t a1 = hsub2_u32(prmt(c1w, 0x64646464u, 0x4140u), kB);
        const uint32_t a3 = hsub2_u32(prmt(c1w, 0x64646464u, 0x4342u), kB);
        const float f0 = dd0 * (float)((int)((sc0 >> (8 * u)) & 0xFFu) - 32);
        const float f1 = dd1 * (float)((int)((sc1 >> (8 * u)) & 0xFFu) - 32);
#pragma unroll
        for (int n = 0; n < NTW; ++n) {
          const uint2 b = lds64(xa.x(n, j, 32 * u));
          float t4[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816(t4, a0, a1, a2, a3, b.x, b.y);
          y[n][0] = __fmaf_rn(f0, t4[0], y[n][0]);
          y[n][1] = __fmaf_rn(f0, t4[1], y[n][1]);
          y[n][2] = __fmaf_rn(f1, t4[2], y[n][2]);
          y[n][3] = __fmaf_rn(f1, t4[3], y[n][3]);
        }
      }
    }
  } else if (T == 23) {
    // IQ4_XS: d @0, scales_h u16 @2, scales_l[4] @4, qs[128] @8 (a window: w0 / w1 8-byte aligned). Group g (32
    // values) = sub-blocks of 16: the low nibbles of qs bytes 16g + p, then the high nibbles; each nibble becomes its
    // level (an exact f16 integer), then y += d * (sc - 32) * acc per group.
    const uint2 H0 = lds64(w0), H1 = lds64(w1);
    const float dd0 = h2f_bits(H0.x & 0xFFFFu), dd1 = h2f_bits(H1.x & 0xFFFFu);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int g = 2 * j + t;
        const float f0 = dd0 * (float)((int)(((H0.y >> (4 * g)) & 15u) | (((H0.x >> (16 + 2 * g)) & 3u) << 4)) - 32);
        const float f1 = dd1 * (float)((int)(((H1.y >> (4 * g)) & 15u) | (((H1.x >> (16 + 2 * g)) & 3u) << 4)) - 32);
        const uint32_t q0 = lds32(w0 + 8 + 16 * g + 4 * c), q1 = lds32(w1 + 8 + 16 * g + 4 * c);
        float t4[NTW][4];
#pragma unroll
        for (int n = 0; n < NTW; ++n) t4[n][0] = t4[n][1] = t4[n][2] = t4[n][3] = 0.f;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t l0 = iq4_levels((q0 >> (4 * hf)) & 0x0F0F0F0Fu);
          const uint32_t l1 = iq4_levels((q1 >> (4 * hf)) & 0x0F0F0F0Fu);
          constexpr uint32_t kB = 0x64806480u;  // f16 (1152, 1152) = 1024 + 128
          const uint32_t a0 = hsub2_u32(prmt(l0, 0x64646464u, 0x4140u), kB);
          const uint32_t a2 = hsub2_u32(prmt(l0, 0x64646464u, 0x4342u), kB);
          const uint32_t a1 = hsub2_u32(prmt(l1, 0x64646464u, 0x4140u), kB);
          const uint32_t a3 = hsub2_u32(prmt(l1, 0x64646464u, 0x4342u), kB);
#pragma unroll
          for (int n = 0; n < NTW; ++n) {
            const uint2 b = lds64(xa.x(n, j, 32 * (2 * t + hf)));
            mma16816(t4[n], a0, a1, a2, a3, b.x, b.y);
          }
        }
#pragma unroll
        for (int n = 0; n < NTW; ++n) {
          y[n][0] = __fmaf_rn(f0, t4[n][0], y[n][0]);
          y[n][1] = __fmaf_rn(f0, t4[n][1], y[n][1]);
          y[n][2] = __fmaf_rn(f1, t4[n][2], y[n][2]);
          y[n][3] = __fmaf_rn(f1, t4[n][3], y[n][3]);
        }
      }
    }
  } else {  // Q8_0: eight 34-byte blocks (d f16, 32 int8); unit 8(bk & 1) + 4hb + c of chunk bk >> 1 (byte 8 * unit)
#pragma unroll
    for (int bk = 0; bk < 8; ++bk) {
      const float d0 = h2f_bits(lds_u16(w0 + 34 * bk)), d1 = h2f_bits(lds_u16(w1 + 34 * bk));
      float t4[NTW][4];
#pragma unroll
      for (int n = 0; n < NTW; ++n) t4[n][0] = t4[n][1] = t4[n][2] = t4[n][3] = 0.f;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const uint32_t q0 = lds_word(w0 + 34 * bk + 2 + 16 * hb + 4 * c) ^ 0x80808080u;
        const uint32_t q1 = lds_word(w1 + 34 * bk + 2 + 16 * hb + 4 * c) ^ 0x80808080u;
        constexpr uint32_t kB = 0x64806480u;  // f16 (1152, 1152) = 1024 + 128
        const uint32_t a0 = hsub2_u32(prmt(q0, 0x64646464u, 0x4140u), kB);
        const uint32_t a2 = hsub2_u32(prmt(q0, 0x64646464u, 0x4342u), kB);
        const uint32_t a1 = hsub2_u32(prmt(q1, 0x64646464u, 0x4140u), kB);
        const uint32_t a3 = hsub2_u32(prmt(q1, 0x64646464u, 0x4342u), kB);
#pragma unroll
        for (int n = 0; n < NTW; ++n) {
          const uint2 b = lds64(xa.x(n, bk >> 1, 64 * (bk & 1) + 32 * hb));
          mma16816(t4[n], a0, a1, a2, a3, b.x, b.y);
        }
      }
#pragma unroll
      for (int n = 0; n < NTW; ++n) {
        y[n][0] = __fmaf_rn(d0, t4[n][0], y[n][0]);
        y[n][1] = __fmaf_rn(d0, t4[n][1], y[n][1]);
        y[n][2] = __fmaf_rn(d1, t4[n][2], y[n][2]);
        y[n][3] = __fmaf_rn(d1, t4[n][3], y[n][3]);
      }
    }
  }
}
// ------------------------------------------------------------------------------------------------ Q4_K helper
__device__ __forceinline__ void gv_store_sum(uint32_t ss, int M, int t, int grp, float v) {
  const __half hv = __float2half_rn(v);
  const __half lv = __float2half_rn(v - __half2float(hv));
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(ss + (t * 8 + grp) * 2), "h"(__half_as_ushort(hv)) : "memory");
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(ss + (M * 8 + t * 8 + grp) * 2), "h"(__half_as_ushort(lv)) : "memory");
}

// One stage's activation prep for Q4_K, by one warp: (1) the group sums X_g (hi, lo f16) of each slot's
// super-block; (2) every 4 activations (x0, x1, x2, x3) become (x0, x2, x1, x3), the order in which a weight
// word yields its nibble pairs (bytes 0, 2 and 1, 3).
// Sums for up to 4 tokens: lane l adds the 8 values at positions 8l .. 8l + 7 of the super-block in f32 and
// two shuffles finish group l / 4. For more tokens: MMAs D[group][token] += Sel[group][k] * x[k][token] over the
// 16 k16 slices of a super-block, Sel = 1 where slice k lies in the group (lane row g: ones on slices 2g, 2g + 1).
__device__ __forceinline__ void gv_prep_q4k(uint32_t xs, int slots, int M, uint32_t sums, int lane) {
  const int g = lane >> 2, c = lane & 3;
  if (M <= 4) {
    for (int s = 0; s < slots; ++s) {
      const uint32_t ss = sums + s * 32 * M;
      for (int t = 0; t < M; ++t) {
        const uint4 q = lds128(xpiece(xs, (4 * s + (lane >> 3)) * M + t, lane & 7));
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
        const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&q.z));
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q.w));
        float v = ((a.x + a.y) + (b.x + b.y)) + ((e.x + e.y) + (f.x + f.y));
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (c == 0) gv_store_sum(ss, M, t, g, v);
      }
    }
  } else {
    const int ntiles = (M + 7) >> 3;
    for (int s = 0; s < slots; ++s) {
      const uint32_t ss = sums + s * 32 * M;
      for (int nt = 0; nt < ntiles; ++nt) {
        const int tau = 8 * nt + g < M ? 8 * nt + g : M - 1;  // columns past M are never stored
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ch = 0; ch < 16; ch += 2) {
          const uint32_t a = (g == (ch >> 1)) ? 0x3C003C00u : 0u;
          const int v0 = 4 * (ch & 3) + c, v1 = 4 * ((ch + 1) & 3) + c;
          const uint2 b0 = lds64(xpiece(xs, (4 * s + (ch >> 2)) * M + tau, v0 >> 1) + 8 * (v0 & 1));
          const uint2 b1 = lds64(xpiece(xs, (4 * s + ((ch + 1) >> 2)) * M + tau, v1 >> 1) + 8 * (v1 & 1));
          mma16816(d0, a, 0u, a, 0u, b0.x, b0.y);
          mma16816(d1, a, 0u, a, 0u, b1.x, b1.y);
        }
        // d[0], d[1]: group g, tokens 8nt + 2c, 8nt + 2c + 1
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = 8 * nt + 2 * c + e;
          if (t < M) gv_store_sum(ss, M, t, g, d0[e] + d1[e]);
        }
      }
    }
  }
  __syncwarp();
  const int units = 4 * slots * M * 16;
  for (int u = lane; u < units; u += 32) {
    const int row = u >> 4, v = u & 15;
    const uint32_t a = xpiece(xs, row, v >> 1) + 8 * (v & 1);
    const uint2 q = lds64(a);
    asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(a), "r"(prmt(q.x, q.y, 0x5410u)), "r"(prmt(q.x, q.y, 0x7632u))
                 : "memory");
  }
}

// ------------------------------------------------------------------------------------------------ outputs
// silu(g) * v for the swiglu kind (the arithmetic of the tile GEMM's swiglu epilogue; aux may be the output itself:
// each element is read before it is written, by the same thread).
__device__ __forceinline__ float gv_silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ void gv_store(const GvParams& p, int t, int row, float v) {
  if (p.epi == kEpiResid) v += p.aux[(int64_t)t * p.ldaux + row];
  if (p.epi == kEpiSwiglu) v = gv_silu(p.aux[(int64_t)t * p.ldaux + row]) * v;
  if (p.y_f16) reinterpret_cast<__half*>(p.y)[(int64_t)t * p.ldy + row] = __float2half_rn(v);
  else reinterpret_cast<float*>(p.y)[(int64_t)t * p.ldy + row] = v;
}

// ------------------------------------------------------------------------------------------------ stream-K split
// First item of CTA b: floor(b * items / G).
__device__ __forceinline__ int64_t gv_lo(int b, int64_t items, int G) { return (int64_t)b * items / G; }

// The CTA whose range holds `item`.
__device__ __forceinline__ int gv_owner(int64_t item, int64_t items, int G) {
  int b = (int)(item * G / items);
  while (b + 1 < G && gv_lo(b + 1, items, G) <= item) ++b;
  while (b > 0 && gv_lo(b, items, G) > item) --b;
  return b;
}

// A CTA's item range [lo, hi) in processing order: the partial row block it starts in (head), then the partial
// row block it ends in (tail, when that differs), then the whole row blocks between. Both partial blocks are
// exchanged with the neighbouring CTAs early, behind the stream.
struct GvRange {
  int64_t lo, hi, head_end, tail_start;
  int n_head, n_tail;
};

__device__ __forceinline__ GvRange gv_range(int b, const GvParams& p) {
  GvRange r;
  r.lo = gv_lo(b, p.items, gridDim.x);
  r.hi = gv_lo(b + 1, p.items, gridDim.x);
  const int64_t block_end = (r.lo / p.nsb + 1) * p.nsb;
  r.head_end = block_end < r.hi ? block_end : r.hi;
  r.n_head = (int)(r.head_end - r.lo);
  const int64_t ts = ((r.hi - 1) / p.nsb) * p.nsb;
  const bool tail = (r.hi % p.nsb) != 0 && ts >= r.head_end;
  r.tail_start = tail ? ts : r.hi;
  r.n_tail = tail ? (int)(r.hi - ts) : 0;
  return r;
}

// A CTA's work as segments: weight rows [row0, row0 + rows) x super-blocks [sb_begin, sb_end), flushed at the
// end. Row ranges: one segment per chunk of rb rows, all of K. Stream-K: head, tail, then the whole row blocks.
struct GvSeg {
  int64_t row0;
  int sb_begin, sb_end;
};

struct GvWork {
  int64_t rs, re;  // row ranges: this CTA's rows
  GvRange r;       // stream-K
  int nseg;
};

template <bool RANGES>
__device__ __forceinline__ GvWork gv_work(const GvParams& p) {
  GvWork w;
  const int G = gridDim.x;
  if (RANGES) {
    w.rs = 4 * ((int64_t)blockIdx.x * p.units / G);
    w.re = 4 * ((int64_t)(blockIdx.x + 1) * p.units / G);
    if (w.re > p.N) w.re = p.N;
    w.nseg = (int)((w.re - w.rs + p.rb - 1) / p.rb);
  } else {
    w.rs = w.re = 0;
    w.r = gv_range(blockIdx.x, p);
    w.nseg = (w.r.n_head > 0 ? 1 : 0) + (w.r.n_tail > 0 ? 1 : 0) +
             (int)(((w.r.tail_start < w.r.hi ? w.r.tail_start : w.r.hi) - w.r.head_end) / p.nsb);
  }
  return w;
}

template <bool RANGES>
__device__ __forceinline__ GvSeg gv_seg(const GvParams& p, const GvWork& w, int si) {
  GvSeg s;
  if (RANGES) {
    s.row0 = w.rs + (int64_t)si * p.rb;
    s.sb_begin = 0;
    s.sb_end = p.nsb;
    return s;
  }
  int64_t first, last;  // items
  if (si == 0) {
    first = w.r.lo;
    last = w.r.head_end;
  } else if (si == 1 && w.r.n_tail > 0) {
    first = w.r.tail_start;
    last = w.r.hi;
  } else {
    first = w.r.head_end + (int64_t)(si - 1 - (w.r.n_tail > 0 ? 1 : 0)) * p.nsb;
    last = first + p.nsb;
  }
  const int64_t rb = first / p.nsb;
  s.row0 = rb * kGvBlock;
  s.sb_begin = (int)(first - rb * p.nsb);
  s.sb_end = (int)(last - rb * p.nsb);
  return s;
}

// Stream-K: a warp's 16 x (8 * NT) results for row block rb. Stored directly when the CTA covered the whole block,
// otherwise parked in the CTA's workspace slot (2b for the row block CTA b starts in, 2b + 1 for the one it ends
// in); the last of the block's CTAs to arrive adds the slots in CTA order, so the sum is deterministic.
template <int NT>
__device__ __forceinline__ void gv_flush_streamk(const GvParams& p, const GvRange& r, float (&y)[NT][4], int rb,
                                                 int warp, int lane) {
  const int g = lane >> 2, c = lane & 3;
  const int G = gridDim.x;
  const int64_t first = (int64_t)rb * p.nsb;
  const int bf = gv_owner(first, p.items, G), bl = gv_owner(first + p.nsb - 1, p.items, G);
  const int rloc = warp * 16 + g;
  if (bl > bf) {
    const int64_t slot = (int64_t)blockIdx.x * 2 + (rb == (int)(r.lo / p.nsb) ? 0 : 1);
    float* wsb = p.ws + slot * p.M * kGvBlock + rloc;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = 8 * n + 2 * c + (e & 1);
        if (t < p.M) __stcg(wsb + (int64_t)t * kGvBlock + 8 * (e >> 1), y[n][e]);
      }
    // Release the warp's stores and count this CTA in (the last arrival acquires everyone's).
    __syncwarp();
    int prev = 0;
    if (lane == 0)
      asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                   : "=r"(prev)
                   : "l"(p.counters + (int64_t)rb * 8 + warp)
                   : "memory");
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != bl - bf) return;
    __syncwarp();
    // CTA bf's slot is 2bf + 1 when its range started before this row block; every later CTA starts inside it.
    const int64_t lo_bf = gv_lo(bf, p.items, G);
    constexpr int kBatch = NT == 1 ? 8 : (NT == 2 ? 4 : 2);
#pragma unroll
    for (int n = 0; n < NT; ++n) y[n][0] = y[n][1] = y[n][2] = y[n][3] = 0.f;
    for (int b0 = bf; b0 <= bl; b0 += kBatch) {
      float part[kBatch][NT][4];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int b = b0 + u;
        const int64_t sl = (int64_t)b * 2 + ((b == bf && lo_bf < first) ? 1 : 0);
        const float* src = p.ws + sl * p.M * kGvBlock + rloc;
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 8 * n + 2 * c + (e & 1);
            part[u][n][e] = (b <= bl && t < p.M) ? __ldcg(src + (int64_t)t * kGvBlock + 8 * (e >> 1)) : 0.f;
          }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) y[n][e] += part[u][n][e];
    }
    if (lane == 0) p.counters[(int64_t)rb * 8 + warp] = 0;
  }
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = 8 * n + 2 * c + (e & 1), row = rb * kGvBlock + rloc + 8 * (e >> 1);
      if (t < p.M && row < p.N) gv_store(p, t, row, y[n][e]);
    }
}

// Row ranges: the slots of each row group are added in slot order through shared memory (red[warp][lane][...]),
// then the slot-0 warps store. rfull: all compute warps have parked their sums; rdone: the readers are done,
// so the next chunk may overwrite red. Returns false when a bounded wait ran out.
template <int NTW, int CW>
__device__ __forceinline__ bool gv_flush_rows(const GvParams& p, float (&y)[NTW][4], float* red, uint64_t* rfull,
                                              uint64_t* rdone, int chunk, int64_t row0, int64_t row_end, int rgi,
                                              int slot, int tp, int warp, int lane) {
  const int g = lane >> 2, c = lane & 3, tok0 = tp * NTW * 8;
  if (p.slots > 1) {
    if (chunk > 0 && !mbar_wait(rdone, (chunk - 1) & 1, p.status, kStatusTimeoutFull)) return false;
    float* mine = red + (warp * 32 + lane) * NTW * 4;
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) mine[n * 4 + e] = y[n][e];
    mbar_arrive(rfull);
    if (slot != 0) return true;
    if (!mbar_wait(rfull, chunk & 1, p.status, kStatusTimeoutFull)) return false;
    for (int s = 1; s < p.slots; ++s) {
      const float* other = red + ((rgi + p.rgp * (s + p.slots * tp)) * 32 + lane) * NTW * 4;
#pragma unroll
      for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) y[n][e] += other[n * 4 + e];
    }
  }
#pragma unroll
  for (int n = 0; n < NTW; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = tok0 + 8 * n + 2 * c + (e & 1);
      const int64_t row = row0 + rgi * 16 + g + 8 * (e >> 1);
      if (p.xf32) {  // token rows t (hi) and t + 1 (lo) of one f32 token, both in this thread
        if ((e & 1) == 0 && t < p.M && row < row_end) gv_store(p, t >> 1, (int)row, y[n][e] + y[n][e + 1]);
      } else if (t < p.M && row < row_end) {
        gv_store(p, t, (int)row, y[n][e]);
      }
    }
  if (p.slots > 1) mbar_arrive(rdone);
  return true;
}

// One 16-byte piece (8 f16 activations, piece kp of token row t) into the resident layout; for Q4_K / Q5_K also the
// group sum (hi, lo f16) and the (x0, x2, x1, x3) permutation of every 4. All 32 lanes of the warp take part (the
// group sum is finished by two shuffles over the 4 pieces of a group).
template <int T>
__device__ __forceinline__ void gv_store_piece(const GvParams& p, uint32_t res, uint32_t ressum, int t, int kp,
                                               uint4 v) {
  if (gv_q4like(T)) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
    float sum = ((a.x + a.y) + (b.x + b.y)) + ((e.x + e.y) + (f.x + f.y));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((kp & 3) == 0) {  // group kp / 4 = super-block kp / 32, group (kp / 4) % 8: hi at + 0, lo at + 16
      const uint32_t ss = ressum + t * p.sstride + (kp >> 5) * 32 + ((kp >> 2) & 7) * 2;
      const __half hv = __float2half_rn(sum);
      const __half lv = __float2half_rn(sum - __half2float(hv));
      asm volatile("st.shared.b16 [%0], %1;" ::"r"(ss), "h"(__half_as_ushort(hv)) : "memory");
      asm volatile("st.shared.b16 [%0], %1;" ::"r"(ss + 16), "h"(__half_as_ushort(lv)) : "memory");
    }
    v = make_uint4(prmt(v.x, v.y, 0x5410u), prmt(v.x, v.y, 0x7632u), prmt(v.z, v.w, 0x5410u),
                   prmt(v.z, v.w, 0x7632u));
  }
  const uint32_t a = res + t * p.xstride + (kp >> 5) * p.sbstride + (kp & 31) * 16;
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// f32 activations (the reference GEMV's x f32 operand): each value splits exactly enough into hi = f16(x) and
// lo = f16(x - hi) (22 significant bits; |x| < 65504), token t becoming the kernel's token rows 2t (hi) and 2t + 1
// (lo); the two rows' products are added in the flush.
__device__ __forceinline__ void gv_split_f32(const float4& a, const float4& b, uint4& hi, uint4& lo) {
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    const float2 hf = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&hh);
    l[i] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Resident activations (row ranges with small M * K): the compute warps copy all of x into shared memory once,
// token t at t * xstride (Q4_K already permuted), with the Q4_K group sums at ressum + t * sstride
// ([super-block][hi 8, lo 8] f16). A thread takes one 16-byte piece (8 values); four consecutive pieces
// are one group, added in f32 by two shuffles. f32 activations: a thread takes 8 values (32 bytes) of one token
// and writes the hi and lo pieces of both of its token rows.
template <int T>
__device__ __forceinline__ void gv_prep_resident(const GvParams& p, uint32_t res, uint32_t ressum, int tid,
                                                 int nthreads) {
  const int kp_total = p.K / 8;  // pieces per token, a multiple of 32
  if (p.xf32) {
    const int total = (p.M / 2) * kp_total;
    for (int L0 = tid; L0 < total; L0 += 2 * nthreads) {
      float4 va[2], vb[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int L = L0 + u * nthreads, t = L / kp_total, kp = L - t * kp_total;
        if (L < total) {
          const float4* src = reinterpret_cast<const float4*>(p.xf + (int64_t)t * p.ldx + (int64_t)kp * 8);
          va[u] = __ldg(src);
          vb[u] = __ldg(src + 1);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int L = L0 + u * nthreads, t = L / kp_total, kp = L - t * kp_total;
        if (L >= total) break;  // uniform across a warp: total and nthreads are multiples of 32
        uint4 hi, lo;
        gv_split_f32(va[u], vb[u], hi, lo);
        gv_store_piece<T>(p, res, ressum, 2 * t, kp, hi);
        gv_store_piece<T>(p, res, ressum, 2 * t + 1, kp, lo);
      }
    }
    return;
  }
  const int total = p.M * kp_total;
  // four loads in flight per thread before any is used: the prep costs one L2 round trip, not one per piece
  for (int L0 = tid; L0 < total; L0 += 4 * nthreads) {
    uint4 vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int L = L0 + u * nthreads, t = L / kp_total, kp = L - t * kp_total;
      if (L < total) vv[u] = __ldg(reinterpret_cast<const uint4*>(p.x + (int64_t)t * p.ldx + (int64_t)kp * 8));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int L = L0 + u * nthreads, t = L / kp_total, kp = L - t * kp_total;
      if (L >= total) break;  // uniform across a warp: total and nthreads are multiples of 32
      gv_store_piece<T>(p, res, ressum, t, kp, vv[u]);
    }
  }
}

template <int T, int NTW, int CW, bool RANGES>
__global__ void __launch_bounds__(GvRoles<T, CW>::kThreads, (CW == 8 && NTW == 1) ? 2 : 1)
    qgemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 const GvParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.baroff);
  uint64_t* empty = full + kGvMaxStages;
  uint64_t* sready = empty + kGvMaxStages;
  uint64_t* rfull = sready + kGvMaxStages;
  uint64_t* rdone = rfull + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  constexpr bool ranges = RANGES;

  const GvWork W = gv_work<RANGES>(p);

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.turns * p.ringst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW / p.turns + (gv_q4like(T) && !p.xres ? 1 : 0));
      mbar_init(&sready[i], 32);
    }
    mbar_init(rfull, CW * 32);
    mbar_init(rdone, p.rgp * p.tsplit * 32);
    fence_barrier_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  if (warp == CW) {
    // ---------------------------------------------------------------- TMA producer
    if (lane != 0) return;
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
    const uint32_t bytes = (uint32_t)(p.ops * p.rb * p.opw + (p.xres ? 0 : 4 * p.sst * p.M * 128));
    int cnt[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // stages issued per ring
    // Under a programmatic launch the weights (which no kernel in flight writes) start streaming while the
    // preceding kernel finishes; the activation copies of the first pass over the rings are held back until it
    // has completed (griddepcontrol.wait), and issued before any stage is reused.
    bool dep = p.xres != 0;  // resident activations: the producer copies none
    int npend = 0, pend_st[kGvMaxStages], pend_k[kGvMaxStages], issued = 0;
    bool ok = true;
    for (int si = 0; si < W.nseg && ok; ++si) {
      const GvSeg sg = gv_seg<RANGES>(p, W, si);
      const int64_t row0 = sg.row0;
      int r = 0;
      for (int sb0 = sg.sb_begin; sb0 < sg.sb_end; sb0 += p.sst) {
      const int q = cnt[r]++;
      const int st = r * p.ringst + q % p.ringst, ph = (q / p.ringst) & 1;
      if (++r == p.turns) r = 0;
      if (p.xres && ++issued == kGvEarlyStages + 1) griddep_wait();  // see qgemv_q4k_m1_kernel's producer
      if (!dep && q >= p.ringst) {
        griddep_wait();
        dep = true;
        for (int i = 0; i < npend; ++i)
          tma_load_3d(smem + pend_st[i] * p.stage_bytes + p.xoff, &tmap_x, &full[pend_st[i]], 0, 0, pend_k[i]);
      }
      if (!mbar_wait(&empty[st], ph ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
      uint8_t* base = smem + st * p.stage_bytes;
      mbar_arrive_expect_tx(&full[st], bytes);
      for (int op = 0; op < p.ops; ++op) {
        const int64_t sbg = (int64_t)p.kb_off + sb0 + op * p.P;
        const int xw = gv_windowed(T) ? (int)(((sbg * gv_sb_bytes(T)) & ~int64_t(15)) >> 1)
                                      : (int)(sbg * (gv_sb_bytes(T) / 8));
        tma_load_2d(base + op * p.wreg, &tmap_w, &full[st], xw, (int)row0);
      }
      if (!p.xres) {
        if (dep) {
          tma_load_3d(base + p.xoff, &tmap_x, &full[st], 0, 0, 4 * sb0);
        } else {
          pend_st[npend] = st;
          pend_k[npend++] = 4 * sb0;
        }
      }
      }
    }
    if (!dep) {
      griddep_wait();
      for (int i = 0; i < npend; ++i)
        tma_load_3d(smem + pend_st[i] * p.stage_bytes + p.xoff, &tmap_x, &full[pend_st[i]], 0, 0, pend_k[i]);
    }
    for (int r = 0; r < p.turns; ++r)
      for (int q = (cnt[r] > p.ringst ? cnt[r] - p.ringst : 0); q < cnt[r]; ++q)
        mbar_wait(&full[r * p.ringst + q % p.ringst], (q / p.ringst) & 1, p.status, kStatusTimeoutDrain, false);
    return;
  }

  if (warp == CW + 1) {
    // ---------------------------------------------------------------- Q4_K activation prep
    if (p.xres) return;
    int cnt[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    bool ok = true;
    for (int si = 0; si < W.nseg && ok; ++si) {
      const GvSeg sg = gv_seg<RANGES>(p, W, si);
      int r = 0;
      for (int sb0 = sg.sb_begin; sb0 < sg.sb_end; sb0 += p.sst) {
      const int q = cnt[r]++;
      const int st = r * p.ringst + q % p.ringst, ph = (q / p.ringst) & 1;
      if (++r == p.turns) r = 0;
      if (!mbar_wait(&full[st], ph, p.status, kStatusTimeoutFull)) { ok = false; break; }
      const uint32_t base = smem_u32(smem + st * p.stage_bytes);
      gv_prep_q4k(base + p.xoff, p.sst, p.M, base + p.sumoff, lane);
      fence_proxy_async();  // the permuted activations are overwritten by a later copy into this stage
      __syncwarp();
      mbar_arrive(&sready[st]);
      if (lane == 0) mbar_arrive(&empty[st]);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ compute warps
  const int rgi = warp % p.rgp, rest = warp / p.rgp, slot = rest % p.slots, tp = rest / p.slots;
  const int tok0 = tp * NTW * 8;
  // Stage k of a segment holds super-blocks k * sst .. + sst - 1; this warp takes super-block slot (mod slots),
  // i.e. position slot % sst of the stages k with k % (slots / sst) == slot / sst.
  const int pos = slot % p.sst, turn = slot / p.sst;
  const int op = pos / p.P, within = pos % p.P;
  const bool has_rows = rgi * 16 < p.rb;
  float* red = reinterpret_cast<float*>(smem + p.redoff);
  const uint32_t res = smem_u32(smem + p.resoff), ressum = smem_u32(smem + p.ressum);
  griddep_wait();  // activations are read, and outputs written, only after the preceding kernel has completed
  if (p.xres) {
    gv_prep_resident<T>(p, res, ressum, threadIdx.x, CW * 32);
    named_bar(1, CW * 32);
  }
  // This lane's activation rows (token rows past M read token M - 1; those D columns are never stored) and its
  // offsets in the resident layout.
  const int lane_b = (gv_q4like(T) ? 16 : 8) * c;
  int tokl[NTW];
  uint32_t xlane[NTW], slane[NTW];
#pragma unroll
  for (int n = 0; n < NTW; ++n) {
    tokl[n] = tok0 + 8 * n + g < p.M ? tok0 + 8 * n + g : p.M - 1;
    xlane[n] = res + tokl[n] * p.xstride + lane_b;
    slane[n] = ressum + tokl[n] * p.sstride + 4 * c;
  }
  float y[NTW][4];
#pragma unroll
  for (int n = 0; n < NTW; ++n) y[n][0] = y[n][1] = y[n][2] = y[n][3] = 0.f;
  int lslot = 0, lph = 0;  // this warp's ring: next stage slot and its phase parity
  for (int si = 0; si < W.nseg; ++si) {
    const GvSeg sg = gv_seg<RANGES>(p, W, si);
    bool ok = true;
    for (int sb0 = sg.sb_begin + turn * p.sst; sb0 < sg.sb_end; sb0 += p.slots) {
      const int st = turn * p.ringst + lslot, ph = lph;
      if (++lslot == p.ringst) lslot = 0, lph ^= 1;
      if (!mbar_wait(&full[st], ph, p.status, kStatusTimeoutFull) ||
          (gv_q4like(T) && !p.xres && !mbar_wait(&sready[st], ph, p.status, kStatusTimeoutFull))) {
        ok = false;
        break;
      }
      if (has_rows && sb0 + pos < sg.sb_end) {
        const uint32_t base = smem_u32(smem + st * p.stage_bytes);
        uint32_t off = (uint32_t)(within * gv_sb_bytes(T));
        if (gv_windowed(T))
          off = (uint32_t)((((int64_t)p.kb_off + sb0 + op * p.P) * gv_sb_bytes(T)) & 15) + within * gv_sb_bytes(T);
        const uint32_t w0 = base + op * p.wreg + (rgi * 16 + g) * p.opw + off;
        if (p.xres) {
          XRes<NTW> xa;
#pragma unroll
          for (int n = 0; n < NTW; ++n) xa.xu[n] = xlane[n] + (sb0 + pos) * 512, xa.su[n] = slane[n] + (sb0 + pos) * 32;
          gv_superblock<T, NTW>(w0, w0 + 8 * p.opw, xa, y, c);
        } else {
          XStage<NTW> xa;
          xa.xs = base + p.xoff;
          xa.sums = base + p.sumoff + pos * 32 * p.M;
          xa.xrows = p.M;
          xa.c0 = 4 * pos;
          xa.lane_b = lane_b;
          xa.lane_s = 4 * c;
#pragma unroll
          for (int n = 0; n < NTW; ++n) xa.tok[n] = tokl[n];
          gv_superblock<T, NTW>(w0, w0 + 8 * p.opw, xa, y, c);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (!ok) break;
    if constexpr (ranges) {
      const int64_t row_end = sg.row0 + p.rb < W.re ? sg.row0 + p.rb : W.re;
      if (!gv_flush_rows<NTW, CW>(p, y, red, rfull, rdone, si, sg.row0, row_end, rgi, slot, tp, warp, lane)) break;
    } else {
      gv_flush_streamk<NTW>(p, W.r, y, (int)(sg.row0 / kGvBlock), warp, lane);
    }
#pragma unroll
    for (int n = 0; n < NTW; ++n) y[n][0] = y[n][1] = y[n][2] = y[n][3] = 0.f;
  }
}

// ------------------------------------------------------------------------------------------------ Q4_K, one token
// One decode token against Q4_K weights, activations resident, row ranges. With a single token, seven of the eight
// B columns of an m16n8k16 would be idle; this form spends them. The 16 A rows of an MMA are 4 weight rows x 4
// super-blocks (lane row g: row g % 4 at super-block g / 4, lane row g + 8: the same row at super-block 2 + g / 4)
// and B column n holds the activations of super-block n, so D[g][g / 4] and D[g + 8][2 + g / 4] are the products
// of the right pairs (the other D entries mix a row with another super-block's activations and are dropped). Each
// lane owns one (row, super-block) product: lanes c = 0 that of its row g, lanes c = 1 that of row g + 8, so a lane
// forms the group scales of one super-block instead of two, and 28-row ranges split into 4-row quads with no padded
// rows. A unit (4 rows x 4 super-blocks) ends with the lane values added across the unit by two shuffles and
// stored per (row quad, super-block quad); the rows are summed in a fixed order at the end (deterministic). Warps
// take units from a shared counter in stage order, so whichever warp runs ahead takes more of them (which warp
// computes a unit does not change its result).
struct Gv1Params {
  int N, nsb, kb_off, S, ringst, stage_bytes, opw, rb;
  int units;                  // ceil(N / 4)
  int resoff, ressum, partoff, baroff, xstride, sstride;
  const __half* x;
  int64_t ldx;
  int K;
  void* y;
  int64_t ldy;
  int y_f16, epi;
  const float* aux;
  int64_t ldaux;
  int* status;
};

constexpr int kGv1Warps = 16;  // compute warps; warp 16 issues the weight copies
// Bank layout of the one-token form. Activations: super-blocks 576 bytes apart, so the four columns of an MMA
// (super-blocks n = 0..3 at n * 576 + 16 c) fill both halves of the 128-byte bank line. Weights: a copy pitch of
// 2 mod 8 16-byte units, so the 8 (row, super-block) pairs of a lane group (rows 0..3 x offsets 0 / 144 bytes) start
// in 8 different 16-byte bank slots.
constexpr int kGv1SbStride = 576;
__host__ __device__ constexpr int gv1_pitch(int S) { return (9 * S + ((2 - 9 * S) % 8 + 8) % 8) * 16; }

__device__ __forceinline__ void gv1_store(const Gv1Params& p, int row, float v) {
  if (p.epi == kEpiResid) v += p.aux[row];
  if (p.epi == kEpiSwiglu) v = gv_silu(p.aux[row]) * v;
  if (p.y_f16) reinterpret_cast<__half*>(p.y)[row] = __float2half_rn(v);
  else reinterpret_cast<float*>(p.y)[row] = v;
}

// One unit: weight rows at wg (lane row g) and wg + 288 (lane row g + 8), this lane's own header at wg + own,
// activations xu (+ 128 j, + 64 for the high-nibble pieces) and group sums su of super-block column g % 4.
// Returns the lane's product (zero for lanes c >= 2) before the cross-lane sum.
__device__ __forceinline__ float gv1_unit(uint32_t wg, uint32_t own, uint32_t xu, uint32_t su, int c,
                                          const float (&sel)[4]) {
  const uint32_t wg8 = wg + 288;
  const uint4 ho = lds128(wg + own), h0 = lds128(wg), h1 = lds128(wg8);
  uint2 q0[4], q1[4];
  uint4 xl[4], xh[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    q0[j] = lds64(wg + 16 + 32 * j + 8 * c);
    q1[j] = lds64(wg8 + 16 + 32 * j + 8 * c);
    xl[j] = lds128(xu + 128 * j);
    xh[j] = lds128(xu + 128 * j + 64);
  }
  const uint32_t bh = lds32(su), bl = lds32(su + 16);
  // this lane's group factors (see gv_superblock): F = (2^23 + sc) * D - 2^23 * D, D = d * 2^24 (low nibbles)
  // or d * 2^20 (high nibbles)
  const uint32_t sca = ho.y & 0x3F3F3F3Fu, scb = (ho.w & 0x0F0F0F0Fu) | ((ho.y >> 2) & 0x30303030u);
  const float d = h2f_bits(ho.x & 0xFFFFu);
  const float dl = d * 16777216.0f, dh = d * 1048576.0f, bl0 = dl * -8388608.0f, bh0 = dh * -8388608.0f;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t s = j < 2 ? sca : scb;
    const float fl = __fmaf_rn(magic_byte(s, (2 * j) & 3), dl, bl0);
    const float fh = __fmaf_rn(magic_byte(s, (2 * j + 1) & 3), dh, bh0);
    uint32_t lo[2][4], hi[2][4];
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
      const uint32_t u0 = wi ? q0[j].y : q0[j].x, u1 = wi ? q1[j].y : q1[j].x;
      const uint32_t v0 = shr8_fma(u0), v1 = shr8_fma(u1);
      lo[wi][0] = u0 & 0x000F000Fu, lo[wi][1] = u1 & 0x000F000Fu, lo[wi][2] = v0 & 0x000F000Fu,
      lo[wi][3] = v1 & 0x000F000Fu;
      hi[wi][0] = u0 & 0x00F000F0u, hi[wi][1] = u1 & 0x00F000F0u, hi[wi][2] = v0 & 0x00F000F0u,
      hi[wi][3] = v1 & 0x00F000F0u;
    }
    float alo[4] = {0.f, 0.f, 0.f, 0.f}, ahi[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(alo, lo[0][0], lo[0][1], lo[0][2], lo[0][3], xl[j].x, xl[j].y);
    mma16816(ahi, hi[0][0], hi[0][1], hi[0][2], hi[0][3], xh[j].x, xh[j].y);
    mma16816(alo, lo[1][0], lo[1][1], lo[1][2], lo[1][3], xl[j].z, xl[j].w);
    mma16816(ahi, hi[1][0], hi[1][1], hi[1][2], hi[1][3], xh[j].z, xh[j].w);
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = __fmaf_rn(fh, ahi[e], __fmaf_rn(fl, alo[e], y[e]));
  }
  // - dmin * sum_g m_g X_g, the mins of lane rows g / g + 8 from their own headers
  const uint32_t m0a = h0.z & 0x3F3F3F3Fu, m0b = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
  const uint32_t m1a = h1.z & 0x3F3F3F3Fu, m1b = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
  const int mb = (2 * c) & 3;
  const uint32_t msel = (uint32_t)mb | 0x40u | ((uint32_t)(mb + 1) << 8) | 0x4000u;
  const uint32_t am0 = hsub2_u32(prmt(c < 2 ? m0a : m0b, 0x64646464u, msel), 0x64006400u);
  const uint32_t am1 = hsub2_u32(prmt(c < 2 ? m1a : m1b, 0x64646464u, msel), 0x64006400u);
  float acc2[4] = {0.f, 0.f, 0.f, 0.f};
  mma16816(acc2, am0, am1, am0, am1, bh, bl);
  const float nd = -h2f_bits(ho.x >> 16);
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = __fmaf_rn(nd, acc2[e], y[e]);
  return sel[0] * y[0] + sel[1] * y[1] + sel[2] * y[2] + sel[3] * y[3];
}

__global__ void __launch_bounds__((kGv1Warps + 1) * 32, 1)
    qgemv_q4k_m1_kernel(const __grid_constant__ CUtensorMap tmap_w, const Gv1Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.baroff);
  uint64_t* empty = full + kGvMaxStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int G = gridDim.x;
  const int rs = 4 * (int)((int64_t)blockIdx.x * p.units / G);
  int re = 4 * (int)((int64_t)(blockIdx.x + 1) * p.units / G);
  if (re > p.N) re = p.N;
  const int nq = (re - rs + 3) / 4;   // row quads of this CTA
  const int nst = p.nsb / p.S;        // stages (S divides the super-blocks)
  const int sq = p.S / 4;             // super-block quads per stage
  const int nsq = p.nsb / 4;
  int* next_unit = reinterpret_cast<int*>(empty + kGvMaxStages);  // the CTA's unit counter, stage-major order
  if (threadIdx.x == 0) {
    for (int i = 0; i < p.ringst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGv1Warps);
    }
    *next_unit = 0;
    fence_barrier_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  if (warp == kGv1Warps) {
    // ---------------------------------------------------------------- TMA producer (weights only)
    if (lane != 0) return;
    tma_prefetch_desc(&tmap_w);
    // the activation row into L2 ahead of the compute warps' loads (issued before the weights)
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) bulk_prefetch_l2(p.x, (uint32_t)p.K * 2);
    const uint32_t bytes = (uint32_t)(p.rb * p.opw);
    int slot = 0, ph = 0;
    for (int k = 0; k < nst; ++k) {
      // Under a programmatic launch, no more than kGvEarlyStages copies go out before the preceding kernel has
      // completed: a deeper early prefetch from every CTA queues ahead of the activation loads in the memory
      // system and delays the start of the arithmetic (measured: 3.3 us of activation prep behind 5 early stages).
      if (k == kGvEarlyStages) griddep_wait();
      if (!mbar_wait(&empty[slot], ph ^ 1, p.status, kStatusTimeoutEmpty)) break;
      mbar_arrive_expect_tx(&full[slot], bytes);
      tma_load_2d(smem + slot * p.stage_bytes, &tmap_w, &full[slot], (int)((int64_t)(p.kb_off + k * p.S) * 18), rs);
      if (++slot == p.ringst) slot = 0, ph ^= 1;
    }
    slot = 0, ph = 0;
    for (int k = 0; k < nst; ++k) {  // exit drain: the last copies of the ring land before the CTA leaves
      if (k >= nst - p.ringst) mbar_wait(&full[slot], ph, p.status, kStatusTimeoutDrain, false);
      if (++slot == p.ringst) slot = 0, ph ^= 1;
    }
    return;
  }

  // ------------------------------------------------------------------ compute warps
  const uint32_t res = smem_u32(smem + p.resoff), ressum = smem_u32(smem + p.ressum);
  float* part = reinterpret_cast<float*>(smem + p.partoff);  // [row quad][super-block quad][4]
  griddep_wait();  // activations are read, and outputs written, only after the preceding kernel has completed
  {
    // The token's activations into shared memory (see gv_prep_resident; one token, so piece kp of thread
    // tid + 512 u needs no division): group sums (hi, lo f16) and the (x0, x2, x1, x3) permutation of every 4.
    const int np = p.K / 8;
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kp = threadIdx.x + u * kGv1Warps * 32;
      if (kp < np) v[u] = __ldg(reinterpret_cast<const uint4*>(p.x) + kp);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kp = threadIdx.x + u * kGv1Warps * 32;
      if (u * kGv1Warps * 32 >= np) break;  // uniform: np is a multiple of 32
      const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(&v[u].x));
      const float2 a1 = __half22float2(*reinterpret_cast<const __half2*>(&v[u].y));
      const float2 a2 = __half22float2(*reinterpret_cast<const __half2*>(&v[u].z));
      const float2 a3 = __half22float2(*reinterpret_cast<const __half2*>(&v[u].w));
      float sum = ((a0.x + a0.y) + (a1.x + a1.y)) + ((a2.x + a2.y) + (a3.x + a3.y));
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (kp < np) {
        if ((kp & 3) == 0) {
          const uint32_t ss = ressum + (kp >> 5) * 32 + ((kp >> 2) & 7) * 2;
          const __half hv = __float2half_rn(sum);
          const __half lv = __float2half_rn(sum - __half2float(hv));
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(ss), "h"(__half_as_ushort(hv)) : "memory");
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(ss + 16), "h"(__half_as_ushort(lv)) : "memory");
        }
        const uint32_t a = res + (kp >> 5) * kGv1SbStride + (kp & 31) * 16;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(prmt(v[u].x, v[u].y, 0x5410u)),
                     "r"(prmt(v[u].x, v[u].y, 0x7632u)), "r"(prmt(v[u].z, v[u].w, 0x5410u)),
                     "r"(prmt(v[u].z, v[u].w, 0x7632u))
                     : "memory");
      }
    }
  }
  named_bar(1, kGv1Warps * 32);
  // lane constants: which D element is this lane's product, whose header holds its scales, its activation column
  float sel[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) sel[e] = (c == 0 && e == (g >> 2)) || (c == 1 && e == 2 + (g >> 2)) ? 1.f : 0.f;
  const uint32_t own = c == 1 ? 288u : 0u;
  const uint32_t xcol = res + (g & 3) * kGv1SbStride + 16 * c, scol = ressum + (g & 3) * 32 + 4 * c;
  const int U = nq * sq;  // units per stage
  // This warp's stage kw (ring slot, phase), whether it has waited for that stage's copy, and its next unit u
  // (stage-major index). A warp releases a stage (arrives on its empty barrier) once it takes a unit of a later
  // stage or the units run out, so a warp waiting for stage s has released every stage before s.
  int slot = 0, ph = 0, kw = 0, kbase = 0;
  bool ok = true, waited = false;
  int u = lane == 0 ? atomicAdd(next_unit, 1) : 0;
  u = __shfl_sync(0xffffffffu, u, 0);
  while (u < nst * U) {
    while (u >= kbase + U) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == p.ringst) slot = 0, ph ^= 1;
      ++kw, kbase += U, waited = false;
    }
    if (!waited) {
      if (!mbar_wait(&full[slot], ph, p.status, kStatusTimeoutFull)) { ok = false; break; }
      waited = true;
    }
    const int un = lane == 0 ? atomicAdd(next_unit, 1) : 0;  // the next unit, fetched ahead of this one
    const uint32_t base = smem_u32(smem + slot * p.stage_bytes);
    const int i = u - kbase;
    const int rq = i / sq, sl = i - rq * sq;  // row quad, super-block quad within the stage
    const int sbq = kw * sq + sl;             // super-block quad of the row
    const uint32_t wg = base + (4 * rq + (g & 3)) * p.opw + (4 * sl + (g >> 2)) * 144;
    float v = gv1_unit(wg, own, xcol + sbq * 4 * kGv1SbStride, scol + sbq * 128, c, sel);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    if (lane < 16 && c == 0) part[(rq * nsq + sbq) * 4 + g] = v;
    u = __shfl_sync(0xffffffffu, un, 0);
  }
  if (ok) {
    for (; kw < nst; ++kw) {  // release the stages this warp took no unit of
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == p.ringst) slot = 0, ph ^= 1;
    }
  }
  // a wait that gave up in any warp of this CTA leaves the CTA's outputs unwritten (the status word says why); the
  // CTA-wide test is a barrier reduction, not a read of the status word, which would cost a global-memory round
  // trip at the end of every CTA
  if (named_bar_or(1, kGv1Warps * 32, !ok)) return;
  for (int r = threadIdx.x; r < re - rs; r += kGv1Warps * 32) {
    const float* pr = part + (r >> 2) * nsq * 4 + (r & 3);
    float acc = 0.f;
    for (int s = 0; s < nsq; ++s) acc += pr[s * 4];
    gv1_store(p, rs + r, acc);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn gv_encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int pow2_ceil(int v) {
  int r = 1;
  while (r < v) r <<= 1;
  return r;
}

template <int T, int NTW, int CW, bool RANGES>
cudaError_t gv_launch(const QGemvArgs& a, const GemvPlan& pl, float* ws, int* counters, cudaStream_t stream) {
  EncodeTiledFn enc = gv_encoder();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw, mx;
  {
    // weights: u64 elements for Q4_K / Q8_0 (whole super-blocks), u16 for Q6_K (a 16-byte aligned window)
    const int64_t window_bytes = (a.kb_off + a.K / 256) * gv_sb_bytes(T);
    const int es = gv_windowed(T) ? 2 : 8;
    cuuint64_t dims[2] = {(cuuint64_t)((window_bytes + es - 1) / es), (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)a.w_row_stride};
    cuuint32_t box[2] = {(cuuint32_t)(pl.opw / es), (cuuint32_t)pl.rb};
    cuuint32_t ones[2] = {1, 1};
    if (enc(&mw, gv_windowed(T) ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(a.w),
            dims, strides, box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    // activations as [K / 64][M][64]: one copy brings the 4 * sst 64-K chunks of a stage, all M tokens
    cuuint64_t dims[3] = {64, (cuuint64_t)a.M, (cuuint64_t)(a.K / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)a.ldx * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)a.M, (cuuint32_t)(4 * pl.sst)};
    cuuint32_t ones[3] = {1, 1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(a.x), dims, strides, box, ones,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  GvParams p;
  p.N = (int)a.N;
  p.M = (int)a.M;
  p.kb_off = (int)a.kb_off;
  p.nsb = (int)(a.K / 256);
  p.mode = pl.mode;
  p.rb = pl.rb;
  p.rgp = pl.rgp;
  p.slots = pl.slots;
  p.sst = pl.sst;
  p.turns = pl.slots / pl.sst;
  p.ringst = pl.ringst;
  p.tsplit = pl.tsplit;
  p.P = pl.P;
  p.ops = pl.ops;
  p.opw = pl.opw;
  p.wreg = pl.wreg;
  p.xoff = pl.xoff;
  p.sumoff = pl.sumoff;
  p.stage_bytes = pl.stage_bytes;
  p.stages = pl.stages;
  p.redoff = pl.redoff;
  p.baroff = pl.baroff;
  p.xres = pl.xres;
  p.resoff = pl.resoff;
  p.ressum = pl.ressum;
  p.x = static_cast<const __half*>(a.x);
  p.xf = static_cast<const float*>(a.x);
  p.xf32 = a.x_f32;
  if (a.x_f32) p.M = 2 * (int)a.M;
  p.ldx = a.ldx;
  p.K = (int)a.K;
  p.units = (a.N + 3) / 4;
  p.items = ((a.N + kGvBlock - 1) / kGvBlock) * (a.K / 256);
  p.y = a.y;
  p.ldy = a.ldy;
  p.y_f16 = a.y_f16;
  p.epi = a.epilogue;
  p.aux = a.aux;
  p.ldaux = a.ldaux;
  p.ws = ws;
  p.counters = counters;
  p.status = a.status;
  p.xstride = (int)(a.K * 2 + 64);
  p.sstride = (int)((a.K / 256) * 32 + 16);
  p.sbstride = 512;
  auto kern = qgemv_kernel<T, NTW, CW, RANGES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(GvRoles<T, CW>::kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, mw, mx, p);
}

template <int T>
cudaError_t gv_fmt(const QGemvArgs& a, const GemvPlan& pl, float* ws, int* counters, cudaStream_t s) {
  if (pl.mode == 0) {
    if (pl.cw == 16) return gv_launch<T, 1, 16, true>(a, pl, ws, counters, s);
    if (pl.ntw == 1) return gv_launch<T, 1, 8, true>(a, pl, ws, counters, s);
    if (pl.ntw == 2) return gv_launch<T, 2, 8, true>(a, pl, ws, counters, s);
    return gv_launch<T, 4, 8, true>(a, pl, ws, counters, s);
  }
  if (pl.ntw == 1) return gv_launch<T, 1, 8, false>(a, pl, ws, counters, s);
  if (pl.ntw == 2) return gv_launch<T, 2, 8, false>(a, pl, ws, counters, s);
  return gv_launch<T, 4, 8, false>(a, pl, ws, counters, s);
}

cudaError_t gv_launch_m1(const QGemvArgs& a, const GemvPlan& pl, cudaStream_t stream) {
  EncodeTiledFn enc = gv_encoder();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw;
  const int64_t window_bytes = (a.kb_off + a.K / 256) * 144;
  cuuint64_t dims[2] = {(cuuint64_t)(window_bytes / 8), (cuuint64_t)a.N};
  cuuint64_t strides[1] = {(cuuint64_t)a.w_row_stride};
  cuuint32_t box[2] = {(cuuint32_t)(pl.opw / 8), (cuuint32_t)pl.rb};
  cuuint32_t ones[2] = {1, 1};
  if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(a.w), dims, strides, box, ones,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  Gv1Params p{};
  p.N = (int)a.N;
  p.nsb = (int)(a.K / 256);
  p.kb_off = (int)a.kb_off;
  p.S = pl.sst;
  p.ringst = pl.ringst;
  p.stage_bytes = pl.stage_bytes;
  p.opw = pl.opw;
  p.rb = pl.rb;
  p.units = (int)((a.N + 3) / 4);
  p.resoff = pl.resoff;
  p.ressum = pl.ressum;
  p.partoff = pl.redoff;
  p.baroff = pl.baroff;
  p.xstride = (int)((a.K / 256) * kGv1SbStride + 64);
  p.sstride = (int)((a.K / 256) * 32 + 16);
  p.x = static_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.K = (int)a.K;
  p.y = a.y;
  p.ldy = a.ldy;
  p.y_f16 = a.y_f16;
  p.epi = a.epilogue;
  p.aux = a.aux;
  p.ldaux = a.ldaux;
  p.status = a.status;
  cudaError_t e = cudaFuncSetAttribute(qgemv_q4k_m1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3((kGv1Warps + 1) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qgemv_q4k_m1_kernel, mw, p);
}

// Plan of the one-token Q4_K form (mode 2), or false when the shape does not fit it.
bool plan_m1(GemvPlan& pl, int64_t N, int64_t K, int num_sms) {
  const int64_t units = (N + 3) / 4, nsb = K / 256;
  if (nsb % 4 || K * 2 > 32 * 1024 || units < 4 * (int64_t)num_sms) return false;
  const int64_t per_cta = (units + num_sms - 1) / num_sms;
  if (4 * per_cta > 128) return false;
  pl = GemvPlan{};
  pl.mode = 2;
  pl.grid = num_sms;
  pl.rb = (int)(4 * per_cta);
  pl.cw = kGv1Warps;
  pl.ntw = 1;
  // super-blocks per stage: a multiple of 4 dividing the row, one copy of at most ~36 KB (box <= 2048 bytes)
  pl.sst = 4;
  for (int S : {12, 8})
    if (nsb % S == 0 && (int64_t)pl.rb * S * 144 <= 36 * 1024) { pl.sst = S; break; }
  pl.P = pl.sst;
  pl.ops = 1;
  pl.opw = gv1_pitch(pl.sst);
  pl.wreg = pl.rb * pl.opw;
  pl.stage_bytes = (pl.wreg + 1023) / 1024 * 1024;
  const int res_bytes = (int)((nsb * kGv1SbStride + 64 + 1023) / 1024 * 1024);
  const int ressum_bytes = (int)((nsb * 32 + 16 + 1023) / 1024 * 1024);
  const int part_bytes = (int)(((pl.rb / 4) * (nsb / 4) * 16 + 1023) / 1024 * 1024);
  const int bar_bytes = 2 * kGvMaxStages * 8 + 16;  // full and empty barriers, the unit counter
  int fit = (kGvSmemBudget - res_bytes - ressum_bytes - part_bytes - bar_bytes) / pl.stage_bytes;
  if (fit > kGvMaxStages) fit = kGvMaxStages;
  if (fit < 2) return false;
  pl.ringst = fit;
  pl.stages = fit;
  pl.resoff = pl.stages * pl.stage_bytes;
  pl.ressum = pl.resoff + res_bytes;
  pl.redoff = pl.ressum + ressum_bytes;
  pl.baroff = pl.redoff + part_bytes;
  pl.smem = pl.baroff + bar_bytes + 1024;
  pl.xres = 1;
  return true;
}

}  // namespace

namespace {
std::atomic<int> g_launch_overlap{1};
}  // namespace
bool launch_overlap() { return g_launch_overlap.load(std::memory_order_relaxed) != 0; }
void set_launch_overlap(bool on) { g_launch_overlap.store(on ? 1 : 0, std::memory_order_relaxed); }

GemvPlan qgemv_plan_limit(int type, int64_t N, int64_t K, int64_t M, int num_sms, int64_t res_limit,
                          bool force_ranges = false);

GemvPlan qgemv_plan_xf32(int type, int64_t N, int64_t K, int64_t M, int num_sms) {
  // Row ranges with resident activations for the 2M hi / lo token rows, however few the rows (small N takes fewer
  // CTAs); ringst < 2 means the rows do not fit beside two weight stages.
  return qgemv_plan_limit(type, N, K, 2 * M, num_sms, int64_t(1) << 40, true);
}

GemvPlan qgemv_plan(int type, int64_t N, int64_t K, int64_t M, int num_sms) {
  GemvPlan pl{};
  if (type == 12 && M == 1 && plan_m1(pl, N, K, num_sms)) return pl;
  // resident activations when they leave a ring of >= 2 weight stages, else stream-K
  pl = qgemv_plan_limit(type, N, K, M, num_sms, 128 * 1024);
  if (pl.mode == 0 && pl.ringst < 2) pl = qgemv_plan_limit(type, N, K, M, num_sms, 0);
  return pl;
}

GemvPlan qgemv_plan_limit(int type, int64_t N, int64_t K, int64_t M, int num_sms, int64_t res_limit,
                          bool force_ranges) {
  GemvPlan pl{};
  const int nt = pow2_ceil((int)((M + 7) / 8));  // token tiles of 8: 1, 2 or 4
  const int64_t units = (N + 3) / 4, nsb = K / 256;
  // Row ranges need >= 16 rows per CTA and pay off when the activations stay resident (no per-stage activation
  // copies, permutes and group sums); otherwise stream-K over 128-row blocks shares each stage's activations
  // among 128 rows.
  // Resident activations (and Q4_K group sums) up to 128 KB, which leaves >= 2 weight stages of 32 KB beside them
  // (measured on B200, Q4_K 4096 x 14336: M = 2 21.2 -> 15.2 us, M = 4 23.3 -> 17.5 us against the 32 KB limit;
  // 14336 x 4096 M = 8 22.7 -> 16.2 us).
  const int64_t res_need = M * (K * 2 + 64) + (gv_q4like(type) ? M * ((K / 256) * 32 + 16) : 0);
  const bool ranges = force_ranges || (units >= 4 * (int64_t)num_sms && res_need <= res_limit);
  pl.mode = ranges ? 0 : 1;
  if (ranges) {
    pl.grid = units < num_sms ? (int)units : num_sms;
    const int64_t per_cta = (units + pl.grid - 1) / pl.grid;
    pl.rb = (int)(4 * per_cta < 128 ? 4 * per_cta : 128);
    pl.rgp = pow2_ceil((pl.rb + 15) / 16);
    pl.cw = nt == 1 ? 16 : 8;
    const int room = pl.cw / pl.rgp;
    pl.tsplit = nt > 1 ? (nt / 2 < room ? nt / 2 : room) : 1;
    if (pl.tsplit < 1) pl.tsplit = 1;
    pl.ntw = nt / pl.tsplit;
    pl.slots = room / pl.tsplit;
  } else {
    pl.rb = kGvBlock;
    pl.rgp = 8;
    pl.cw = 8;
    pl.tsplit = 1;
    pl.ntw = nt;
    pl.slots = 1;
  }
  pl.xres = ranges;  // all activations fit beside the weight stages
  const int red_bytes = (ranges && pl.slots > 1) ? pl.cw * 32 * pl.ntw * 4 * 4 : 0;
  const int bar_bytes = (3 * kGvMaxStages + 2) * 8;
  const bool two_per_sm = !ranges && pl.ntw == 1;
  // resident layout: M token rows of 2K + 64 bytes, M rows of group sums of 32 bytes per super-block + 16
  const int res_bytes = pl.xres ? (int)((M * (K * 2 + 64) + 1023) / 1024 * 1024) : 0;
  const int ressum_bytes =
      pl.xres && gv_q4like(type) ? (int)((M * ((K / 256) * 32 + 16) + 1023) / 1024 * 1024) : 0;
  const int budget = (two_per_sm ? 104 * 1024 : kGvSmemBudget) - red_bytes - bar_bytes - res_bytes - ressum_bytes;
  // Stage size: a TMA engine completes about one copy per ~0.27 us per SM whatever its size up to ~16 KB, so the
  // weight copies of resident-activation launches are 16-32 KB (8 KB copies cap the stream near 4 TB/s); launches
  // that also copy and permute activations per stage keep ~8 KB stages. The warps of one super-block turn
  // (slots / sst turns) consume a ring of their own of >= 2 stages, as many as fit.
  const int stage_cap = pl.xres ? 32 * 1024 : 8 * 1024;
  pl.sst = 1;
  while (pl.sst < pl.slots && 2 * pl.sst * pl.rb * gv_sb_bytes(type) <= stage_cap) pl.sst *= 2;
  for (;;) {
    pl.P = pl.sst < gv_pmax(type) ? pl.sst : gv_pmax(type);
    pl.ops = pl.sst / pl.P;
    pl.opw = gv_opw(type, pl.P);
    pl.wreg = ((pl.rgp * 16 * pl.opw) + 127) / 128 * 128;
    pl.xoff = (pl.ops * pl.wreg + 1023) / 1024 * 1024;
    pl.sumoff = pl.xoff + (pl.xres ? 0 : 4 * pl.sst * (int)M * 128);
    const int sum_bytes = gv_q4like(type) && !pl.xres ? pl.sst * 32 * (int)M : 0;
    pl.stage_bytes = (pl.sumoff + sum_bytes + 1023) / 1024 * 1024;
    const int turns = pl.slots / pl.sst;
    int fit = budget / pl.stage_bytes;
    if (fit > kGvMaxStages) fit = kGvMaxStages;
    pl.ringst = fit / turns;
    if (pl.ringst >= 2 || pl.sst == pl.slots) break;
    pl.sst *= 2;
  }
  pl.stages = (pl.slots / pl.sst) * pl.ringst;
  pl.resoff = pl.stages * pl.stage_bytes;
  pl.ressum = pl.resoff + res_bytes;
  pl.redoff = pl.ressum + ressum_bytes;
  pl.baroff = (pl.redoff + red_bytes + 7) / 8 * 8;
  pl.smem = pl.baroff + bar_bytes + 1024;  // + alignment of the dynamic shared memory base
  if (!ranges) {
    const int64_t items = ((N + kGvBlock - 1) / kGvBlock) * nsb;
    const int64_t ctas = (int64_t)num_sms * (two_per_sm ? 2 : 1);
    pl.grid = (int)(items < ctas ? items : ctas);
    if (pl.grid < 1) pl.grid = 1;
    bool split = false;  // does any CTA range start inside a row block?
    for (int b = 1; b < pl.grid && !split; ++b) split = ((int64_t)b * items / pl.grid) % nsb != 0;
    pl.ws_floats = split ? (int64_t)pl.grid * 2 * M * kGvBlock : 0;
    pl.counters = split ? ((N + kGvBlock - 1) / kGvBlock) * 8 : 0;
  }
  return pl;
}

cudaError_t launch_qgemv_ws(const QGemvArgs& a, const GemvPlan& plan, float* ws, int* counters,
                            cudaStream_t stream) {
  if (plan.ringst < 2) return cudaErrorInvalidConfiguration;
  if (plan.mode == 2) return a.type == 12 && a.M == 1 ? gv_launch_m1(a, plan, stream) : cudaErrorInvalidValue;
  switch (a.type) {
    case 8: return gv_fmt<8>(a, plan, ws, counters, stream);
    case 12: return gv_fmt<12>(a, plan, ws, counters, stream);
    case 14: return gv_fmt<14>(a, plan, ws, counters, stream);
    case 11: return gv_fmt<11>(a, plan, ws, counters, stream);
    case 13: return gv_fmt<13>(a, plan, ws, counters, stream);
    case 23: return gv_fmt<23>(a, plan, ws, counters, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace yah

// ------------------------------------------------------------------------------------------------ static scratch
// A variant of the decode GEMV for callers that cannot allocate device memory at call time: code that runs
// where cudaMalloc is not available or not allowed (inside a CUDA-graph capture region, in a real-time decode loop
// with a fixed memory budget, or in a host process whose allocator is owned by someone else). Its split-K
// workspace, split counters and status word live in one file-scope device array that every GPU loading this
// library holds until the process exits. Host code cannot use the array's name as a device address, so the
// first call on each device looks the address up with cudaGetSymbolAddress (with that device current) and keeps
// it; later calls reuse it.
namespace yah {
namespace {

constexpr size_t kStaticStatusBytes = 256;                 // status word (padded)
constexpr size_t kStaticCounters = 32768;                  // 8 per 128-row block: N <= 524288
constexpr size_t kStaticPartials = (size_t)1 << 21;        // partial sums: 2 x 32 x 128 floats per CTA, 256 CTAs
constexpr size_t kStaticBytes = kStaticStatusBytes + kStaticCounters * sizeof(int) + kStaticPartials * sizeof(float);

static __device__ __align__(256) unsigned char g_qgemv_static[kStaticBytes];

constexpr int kStaticMaxDev = 64;
void* g_static_addr[kStaticMaxDev] = {};
std::mutex g_static_mu;

}  // namespace

size_t qgemv_static_partials() { return kStaticPartials; }
size_t qgemv_static_counters() { return kStaticCounters; }

cudaError_t qgemv_static_setup(int device, void** base) {
  if (device < 0 || device >= kStaticMaxDev) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_qgemv_static);
    if (e != cudaSuccess) return e;
    g_static_addr[device] = p;
  }
  *base = g_static_addr[device];
  return cudaSuccess;
}

cudaError_t launch_qgemv_static(const QGemvArgs& a_in, const GemvPlan& plan, void* base, cudaStream_t stream) {
  QGemvArgs a = a_in;
  unsigned char* b = static_cast<unsigned char*>(base);
  int* status = reinterpret_cast<int*>(b);
  int* counters = reinterpret_cast<int*>(b + kStaticStatusBytes);
  float* partials = reinterpret_cast<float*>(b + kStaticStatusBytes + kStaticCounters * sizeof(int));
  a.status = status;
  if (plan.counters > 0) {
    // The counters must start at zero; a previous call leaves them at zero unless it was interrupted.
    const cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)plan.counters * sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  return launch_qgemv_ws(a, plan, partials, counters, stream);
}

int* qgemv_static_status_word(void* base) { return reinterpret_cast<int*>(base); }

cudaError_t qgemv_static_status(void* base, int* code, bool clear) {
  cudaError_t e = cudaMemcpy(code, base, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && *code) e = cudaMemset(base, 0, sizeof(int));
  return e;
}

}  // namespace yah
