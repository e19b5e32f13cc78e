// Decode GEMV on the 5th-generation tensor cores (tcgen05): y[t][n] (+)= sum_k W[n][k] x[t][k] for M <= 32 tokens,
// GGUF Q4_K weights, f16 activations, with the f32 weight values of the reference dequant (no f16 rounding of a
// weight), as the reference GEMV computes them (engine/gpu/loom/tools/gen_gemv.py:7-9, kinds :16-19).
//
// Arithmetic. A Q4_K weight is w = d*sc*q - dmin*m (d, dmin f16; 6-bit sc, m per 32-value group; 4-bit q). Per
// super-block s and output row n:
//   y += d_s * D1_s - D2,   D1_s = sum_k f16(sc*q)_k x_k,   D2 = sum_{s,g} (dmin*m_g)_s X_{s,g}
// where X_{s,g} = sum of the group's 32 activations. sc*q <= 945 is an exact f16 integer, so D1_s is a sum of exact
// products (f32 accumulation in TMEM); dmin*m is a 17-bit multiple of ulp(dmin) >= 2^-24 and splits exactly into two
// f16 parts hi + lo, X into an f32-accurate pair Xhi + Xlo, and the four exact products (hi + lo)(Xhi + Xlo) go through
// two more MMAs per super-block that accumulate D2 over the whole K range. So the only rounding is the f32
// accumulation; the epilogue applies d_s (one FMA per token and super-block) and subtracts D2.
//
// B200 design. Weight rows are the MMA's M side (128 TMEM lanes; a tile holds RT <= 128 rows), the tokens its N
// side (16 or 32 columns; rows past M are zero), one 16 x 16 f16 K step per MMA:
//   warp 18       weight producer: TMA of raw super-blocks, RT rows x SW (1 or 2) super-blocks per stage, rows
//                 padded to an odd number of 16-byte units (no shared-memory bank conflicts for thread = row);
//   warp 0        activation producer: per super-block one 3-D TMA copy of its 4 64-K chunks x TP token rows in
//                 the 128-byte swizzle the MMA's K-major B descriptor expects;
//   warps 2-13    decode, groups of 4 warps (one per A buffer) taking super-blocks in turn: thread = row = TMEM lane, warp =
//                 lane quarter. Per super-block a thread turns 128 nibble bytes into 128 cells of f16(sc*q) pairs
//                 (2 prmt + 4 and + 4 fma.rn.f16x2 per 8 weights) and its eight groups' (hi, lo) min factors, and
//                 tcgen05.st's them into an A buffer in TMEM;
//   warp 1        MMA issuer (one thread): 16 MMAs into a D1 slot (A buffer x activation tile) and 2 into the tile's
//                 D2 region (min factors x group sums), then commits that free the A buffer, the activation stage
//                 and hand D1 to the epilogue;
//   warps 14-17   epilogue: per super-block tcgen05.ld of D1, acc += d_s * D1; per tile acc -= D2, the cluster
//                 reduction, the kind (plain / resid / swiglu) and the stores.
// The group sums of this CTA's K range (Xhi, Xlo in f16, 4 per group: Xhi Xlo Xhi Xlo against the A side's hi hi lo
// lo) are formed once, on the first tile, by the decode warps of each super-block from its activation stage in shared
// memory (thread = token row x group), so no warp reads the activations from global memory.
// Work split: the K range is cut into KS equal parts (thread-block clusters of KS = 1, 2 or 4 CTAs, CTA rank = part)
// and the rows into tiles of RT rows; persistent clusters walk the tiles. The KS partial sums of a tile meet in
// distributed shared memory: every CTA stores its partial of each row into the shared memory of the CTA that owns
// the row (RT / KS rows per CTA), which adds the KS partials in rank order (deterministic) and stores them. No global scratch.
// Launch overlap: programmatic dependent launch as in the other GEMV (weights stream before griddepcontrol.wait;
// activations are read and outputs written after it).
// Every mbarrier wait is bounded (ptx.cuh); a wait that runs out records a status code and the CTA leaves its
// loops, drains its own copies and MMAs, and frees TMEM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "decode.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace yah {
namespace {

constexpr int kTcThreads = 608;  // 19 warps
// One MMA issuer. Measured on B200: a thread that issues tcgen05.mma waits ~45 cycles per instruction whatever its
// size up to N = 64, and ~100 while other warps store to TMEM, so the small-N MMAs of a GEMV are issue-bound;
// MMAs issued by two warps at once gave wrong results in whole 32-lane quarters, so the issue stays single.
constexpr int kTcWarpX = 0, kTcWarpMma = 1, kTcWarpDq0 = 2, kTcWarpEpi0 = 14, kTcWarpW = 18;
constexpr int kTcACols = 144;         // an A buffer: 128 columns of f16(sc*q) pairs + 16 of min factors
constexpr int kTcNP = 8;              // per-row d ring (decode -> epilogue)
constexpr int kTcWPitch2 = 304;       // weight stage row pitch for 2 super-blocks (19 x 16 B: odd)
constexpr int kTcWPitch1 = 176;       // ... for 1 super-block (11 x 16 B)
constexpr int kTcWStage = 128 * kTcWPitch2;  // 38912 bytes, a multiple of 1024

// TMEM (512 columns): NA A buffers, two D2 regions (alternate tiles), ND D1 slots. A super-block's A buffer and its
// activation stage share ring index and are released together by one MMA commit.
template <int TP>
struct TcCfg {
  static constexpr int kNA = TP == 16 ? 3 : 2;          // A buffers = activation stages
  static constexpr int kD2Col = kNA * kTcACols;         // D2 regions [2][TP]
  static constexpr int kD1Col = kD2Col + 2 * TP;        // D1 slots [kND][TP]
  static constexpr int kND = (512 - kD1Col) / TP > 8 ? 8 : (512 - kD1Col) / TP;
  static_assert(kND >= 2, "TMEM columns");
  static constexpr int kNSW = TP == 16 ? 4 : 3;         // weight stages
  static constexpr int kXStage = TP * 512;              // 4 chunks x TP rows x 128 B
  static constexpr int kMaxRange = TP == 16 ? 32 : 16;  // super-blocks per CTA (group sums kept for all of them)
  static constexpr int kB2Tile = TP * 128;              // two super-blocks' 32 entries per 128-byte token row
  static constexpr int kXOff = kTcWStage * kNSW;
  static constexpr int kB2Off = kXOff + kNA * kXStage;
  static constexpr int kParOff = kB2Off + (kMaxRange / 2) * kB2Tile;
  static constexpr int kExOff = kParOff + kTcNP * 128 * 4;
  static constexpr int kBarOff = kExOff + TP * 128 * 4;
  // wfull/wempty [NSW], xfull/sbempty/afull [NA], dfull/dempty [ND], d2full/d2empty [2], pfull/pempty [NP],
  // exfull, exempty, drain
  static constexpr int kNumBars = 2 * kNSW + 3 * kNA + 2 * kND + 4 + 2 * kTcNP + 3;
  static constexpr int kSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kSlotOff + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 227 * 1024, "shared memory");
};

struct TcParams {
  int N, M, K, kb_off;
  int rt;          // weight rows per tile (<= 128)
  int tiles;       // ceil(N / rt)
  int ks;          // CTAs per cluster = K parts
  int srange;      // super-blocks per CTA (K / 256 / ks)
  int sw;          // super-blocks per weight stage (1 or 2; divides srange)
  int pitch;       // weight stage row pitch in bytes
  const __half* x;
  int64_t ldx;
  void* y;
  int64_t ldy;
  const float* aux;
  int64_t ldaux;
  int* status;
};

// Two groups' min factors dmin * m (m given as f32 integers): cells (hi, hi), (lo, lo) for each, hi + lo ==
// dmin * m exactly (a 17-bit multiple of ulp(dmin) >= 2^-24).
__device__ __forceinline__ void min_cells2(float dmin, float ma, float mb, uint32_t* out) {
  const float2 p = fmul2(make_float2(dmin, dmin), make_float2(ma, mb));  // exact
  const uint32_t hi = pack_f16x2_rn(p.x, p.y);
  const float2 hf = make_float2(__half2float(__ushort_as_half((unsigned short)(hi & 0xFFFFu))),
                                __half2float(__ushort_as_half((unsigned short)(hi >> 16))));
  const float2 rest = fadd2(p, make_float2(-hf.x, -hf.y));  // exact
  const uint32_t lo = pack_f16x2_rn(rest.x, rest.y);
  out[0] = prmt(hi, 0, 0x1010u);  // (hi_a, hi_a)
  out[1] = prmt(lo, 0, 0x1010u);  // (lo_a, lo_a)
  out[2] = prmt(hi, 0, 0x3232u);  // (hi_b, hi_b)
  out[3] = prmt(lo, 0, 0x3232u);  // (lo_b, lo_b)
}

// One thread's half of a staged Q4_K super-block (its row, groups 4h .. 4h + 3; `rb` the row's super-block in shared
// memory): 64 A cells of f16(sc * q) pairs in K order into TMEM columns at `ta` (two stores of 32), the 8 min-factor
// cells of its 4 groups at `tm`, and d.
// The scales of the 4 groups come out as packed bytes in two vector operations (gen_gemm_decode.py:946-967). The byte
// pair (b0, b1) of a qs word goes through prmt next to 0x64 bytes: f16 (1024 + b0, 1024 + b1); masking keeps
// 1024 + low nibble or 1024 + 16 * high nibble, and one fma.rn.f16x2 gives sc * q exactly ((1024 + q) sc - 1024 sc
// and (1024 + 16 q) (sc / 16) - 64 sc; every term is an exact f16).
__device__ __forceinline__ float q4k_tc_decode_half(uint32_t rb, int h, uint32_t ta, uint32_t tm) {
  const uint4 hdr = lds128(rb);
  uint32_t SC, MM;
  if (h == 0) {
    SC = hdr.y & 0x3F3F3F3Fu;
    MM = hdr.z & 0x3F3F3F3Fu;
  } else {
    SC = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    MM = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  }
  const float d = h2f_bits(hdr.x & 0xFFFFu);
  const float dmin = h2f_bits(hdr.x >> 16);
  {
    uint32_t a2[8];
    // byte k of MM as the f32 2^23 + m, minus 2^23: m of group 4h + k
    const float2 mlo = fadd2(make_float2(__uint_as_float(prmt(MM, 0x4B000000u, 0x7650u)),
                                         __uint_as_float(prmt(MM, 0x4B000000u, 0x7651u))),
                             make_float2(-kMagic23, -kMagic23));
    const float2 mhi = fadd2(make_float2(__uint_as_float(prmt(MM, 0x4B000000u, 0x7652u)),
                                         __uint_as_float(prmt(MM, 0x4B000000u, 0x7653u))),
                             make_float2(-kMagic23, -kMagic23));
    min_cells2(dmin, mlo.x, mlo.y, a2);
    min_cells2(dmin, mhi.x, mhi.y, a2 + 4);
    tmem_st8(tm, a2);
  }
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    // groups 4h + 2pr (low nibbles) and 4h + 2pr + 1 (high nibbles): qs bytes [64h + 32pr, +32)
    const uint32_t se = hsub2_u32(prmt(SC, 0x64646464u, 0x4040u + 0x0101u * (2 * pr)), 0x64006400u);
    const uint32_t so = hsub2_u32(prmt(SC, 0x64646464u, 0x4040u + 0x0101u * (2 * pr + 1)), 0x64006400u);
    const uint32_t s0 = se, c0 = hmul2_u32(se, 0xE400E400u);       // sc, -1024 sc
    const uint32_t s1 = hmul2_u32(so, 0x2C002C00u), c1 = hmul2_u32(so, 0xD400D400u);  // sc / 16, -64 sc
    const uint4 qa = lds128(rb + 16 + 64 * h + 32 * pr);
    const uint4 qb = lds128(rb + 32 + 64 * h + 32 * pr);
    const uint32_t qs[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint32_t v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t r01 = prmt(qs[i], 0x64646464u, 0x4140u);
      const uint32_t r23 = prmt(qs[i], 0x64646464u, 0x4342u);
      v[2 * i] = hfma2_u32(r01 & 0xFF0FFF0Fu, s0, c0);
      v[2 * i + 1] = hfma2_u32(r23 & 0xFF0FFF0Fu, s0, c0);
      v[16 + 2 * i] = hfma2_u32(r01 & 0xFFF0FFF0u, s1, c1);
      v[17 + 2 * i] = hfma2_u32(r23 & 0xFFF0FFF0u, s1, c1);
    }
    tmem_st32(ta + 32 * pr, v);
  }
  return d;
}

__device__ __forceinline__ float silu_tc(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// The warps that execute warp-aligned tcgen05 instructions (decode, epilogue) wait with every lane and take the
// result by a warp vote, so that a bounded wait that runs out sends the whole warp down the same path: a
// .sync.aligned instruction must never be reached by only part of a warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  return __all_sync(0xFFFFFFFFu, mbar_wait(bar, parity, status, code));
}
__device__ __forceinline__ bool warp_wait_cluster(uint64_t* bar, uint32_t parity, int* status, int code) {
  return __all_sync(0xFFFFFFFFu, mbar_wait_cluster(bar, parity, status, code));
}

template <int EPI, bool OUT_F16>
__device__ __forceinline__ void tc_store(const TcParams& p, int t, int row, float v) {
  if (EPI == kEpiResid) v = p.aux[(int64_t)t * p.ldaux + row] + v;
  if (EPI == kEpiSwiglu) v = silu_tc(p.aux[(int64_t)t * p.ldaux + row]) * v;
  if (OUT_F16) reinterpret_cast<__half*>(p.y)[(int64_t)t * p.ldy + row] = __float2half_rn(v);
  else reinterpret_cast<float*>(p.y)[(int64_t)t * p.ldy + row] = v;
}

// Byte offset of f16 entry e (0..63) of token row t in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int t, int e) {
  const int b = 2 * e;
  return (uint32_t)(t * 128 + ((((b >> 4) ^ t) & 7) << 4) + (b & 15));
}

template <int TP, int EPI, bool OUT_F16>
__global__ void __launch_bounds__(kTcThreads, 1)
    qgemv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const TcParams p) {
  using C = TcCfg<TP>;
  constexpr int NA = C::kNA, ND = C::kND, NSW = C::kNSW;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* wfull = bars;
  uint64_t* wempty = wfull + NSW;
  uint64_t* xfull = wempty + NSW;
  uint64_t* sbempty = xfull + NA;   // A buffer + activation stage of a super-block free again (MMA commit)
  uint64_t* afull = sbempty + NA;   // the super-block's A buffer decoded (and its activations seen)
  uint64_t* dfull = afull + NA;
  uint64_t* dempty = dfull + ND;
  uint64_t* d2full = dempty + ND;
  uint64_t* d2empty = d2full + 2;
  uint64_t* pfull = d2empty + 2;
  uint64_t* pempty = pfull + kTcNP;
  uint64_t* exfull = pempty + kTcNP;
  uint64_t* exempty = exfull + 1;
  uint64_t* drain = exempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kSlotOff);
  float* params = reinterpret_cast<float*>(smem + C::kParOff);
  float* ex = reinterpret_cast<float*>(smem + C::kExOff);

  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = p.ks;
  const uint32_t rank = ks > 1 ? cluster_rank() : 0;
  const int G = gridDim.x / ks, cid = blockIdx.x / ks;  // clusters, this cluster
  const int sr = p.srange;
  const int sbx0 = (int)rank * sr;                      // first super-block of this CTA's K range (in the window)
  const int sb0 = p.kb_off + sbx0;                      // ... in the weight rows

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSW; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 4 * p.sw);  // the decode warps that read the stage: one group per super-block
    }
    for (int i = 0; i < NA; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&sbempty[i], 1);
      mbar_init(&afull[i], 4);
    }
    for (int i = 0; i < ND; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&d2full[i], 1);
      mbar_init(&d2empty[i], 4);
    }
    for (int i = 0; i < kTcNP; ++i) {
      mbar_init(&pfull[i], 4);
      mbar_init(&pempty[i], 4);
    }
    mbar_init(exfull, 4 * ks);
    mbar_init(exempty, 4 * ks);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == kTcWarpMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  if (ks > 1) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTcWarpW) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      uint32_t s = 0;
      bool ok = true;
      const int nst = sr / p.sw;
      const uint32_t bytes = (uint32_t)(p.rt * p.pitch);
      for (int tile = cid; ok && tile < p.tiles; tile += G) {
        for (int js = 0; js < nst; ++js, ++s) {
          const uint32_t ws = s % NSW, ph = (s / NSW) & 1;
          if (!mbar_wait(&wempty[ws], ph ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&wfull[ws], bytes);
          tma_load_2d(smem + ws * kTcWStage, &tmap_w, &wfull[ws], (sb0 + js * p.sw) * 18, tile * p.rt);
        }
      }
      for (uint32_t i = (s > (uint32_t)NSW ? s - NSW : 0); i < s; ++i)
        mbar_wait(&wfull[i % NSW], (i / NSW) & 1, p.status, kStatusTimeoutDrain, false);
    }
  } else if (warp == kTcWarpX) {
    // ------------------------------------------------------------------ activation producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      griddep_wait();  // the activations may come from the preceding kernel
      uint32_t s = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < p.tiles; tile += G) {
        for (int j = 0; j < sr; ++j, ++s) {
          const uint32_t xs = s % NA, ph = (s / NA) & 1;
          if (!mbar_wait(&sbempty[xs], ph ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&xfull[xs], C::kXStage);
          tma_load_3d(smem + C::kXOff + xs * C::kXStage, &tmap_x, &xfull[xs], 0, 0, (sbx0 + j) * 4);
        }
      }
      for (uint32_t i = (s > (uint32_t)NA ? s - NA : 0); i < s; ++i)
        mbar_wait(&xfull[i % NA], (i / NA) & 1, p.status, kStatusTimeoutDrain, false);
    }
  } else if (warp == kTcWarpMma) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, TP);
      const uint64_t bx0 = sdesc_sw128(smem_u32(smem + C::kXOff));
      const uint64_t bb0 = sdesc_sw128(smem_u32(smem + C::kB2Off));
      uint32_t i = 0, tc = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < p.tiles; tile += G, ++tc) {
        const uint32_t r2 = tc & 1;
        if (!mbar_wait(&d2empty[r2], ((tc >> 1) & 1) ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
        const uint32_t d2 = tmem + C::kD2Col + r2 * TP;
        for (int j = 0; j < sr; ++j, ++i) {
          const uint32_t as = i % NA, ds = i % ND;
          if (!mbar_wait(&afull[as], (i / NA) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
          if (!mbar_wait(&xfull[as], (i / NA) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
          if (!mbar_wait(&dempty[ds], ((i / ND) & 1) ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = tmem + as * kTcACols;
          const uint32_t dt = tmem + C::kD1Col + ds * TP;
          const uint64_t bx = bx0 + (uint64_t)((as * C::kXStage) >> 4);
#pragma unroll
          for (int c = 0; c < 16; ++c)
            mma_f16_ts(dt, a + 8 * c, bx + (uint64_t)(((c >> 2) * TP * 128) >> 4) + (uint64_t)(2 * (c & 3)), idesc,
                       c > 0 ? 1u : 0u);
          const uint64_t bb = bb0 + (uint64_t)(((j >> 1) * C::kB2Tile) >> 4) + (uint64_t)(4 * (j & 1));
          mma_f16_ts(d2, a + 128, bb, idesc, j > 0 ? 1u : 0u);
          mma_f16_ts(d2, a + 136, bb + 2, idesc, 1u);
          mma_commit(&sbempty[as]);
          mma_commit(&dfull[ds]);
        }
        if (!ok) break;
        mma_commit(&d2full[r2]);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, p.status, kStatusTimeoutDrain, false);
    }
  } else if (warp < kTcWarpEpi0 + 4) {
    if (warp < kTcWarpEpi0) {
      // ---------------------------------------------------------------- decode
      // NA groups of 4 warps (3 or 2; the third group idles when NA = 2) take super-blocks in turn, so group g always
      // fills A buffer g and waits only for its own previous super-block's MMAs; in a group, the warp of lane
      // quarter q decodes the whole super-block of its 32 rows (both halves). Fewer decode warps leave the MMA
      // issuer's SM sub-partition less contended.
      const int q = warp & 3, par = (warp - kTcWarpDq0) >> 2;
      const int r = q * 32 + lane;
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      const int gt0 = (((warp - kTcWarpDq0) & 3) * 32 + lane) >> 3, gg = lane & 7;  // group-sum entries: token, group
      uint32_t i = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < p.tiles; tile += G) {
        for (int j = 0; j < sr; ++j, ++i) {
          if ((int)(i % NA) != par) continue;
          const uint32_t st = i / p.sw, ws = st % NSW, wph = (st / NSW) & 1;
          const int sbw = (int)(i % p.sw);
          const uint32_t as = i % NA;
          if (!warp_wait(&wfull[ws], wph, p.status, kStatusTimeoutFull)) { ok = false; break; }
          if (!warp_wait(&sbempty[as], ((i / NA) & 1) ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
          const bool sums = tile == cid;  // the first tile forms the group sums of super-block j
          if (sums && !warp_wait(&xfull[as], (i / NA) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();  // the MMAs that read this A buffer are complete: order the stores after them
          // Every lane decodes and stores (the stores are warp-aligned): rows past the tile read the stage's
          // unused rows, and the epilogue never reads their results.
          const uint32_t rb = smem_u32(smem + ws * kTcWStage) + r * p.pitch + sbw * 144;
          const uint32_t ta = tl + as * kTcACols, tm = tl + as * kTcACols + 128;
          const float d = q4k_tc_decode_half(rb, 0, ta, tm);
          q4k_tc_decode_half(rb, 1, ta + 64, tm + 8);
          __syncwarp();
          if (lane == 0) mbar_arrive(&wempty[ws]);  // this warp's only read of the stage
          if (sums) {
            // X of group gg, token row gt: the group's 32 activations are 4 16-byte units of the 128-byte-swizzled
            // row gt of 64-K chunk gg / 2 (rows past M are zero); written as (Xhi, Xlo, Xhi, Xlo) into the group-sum
            // tile (async proxy: fenced before the arrive below)
            for (int gt = gt0; gt < TP; gt += 16) {
              const uint32_t xrow = smem_u32(smem + C::kXOff + as * C::kXStage) + (gg >> 1) * (TP * 128) + gt * 128;
              float part[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint4 v = lds128(xrow + ((((gg & 1) * 4 + u) ^ gt) & 7) * 16);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                float a = 0.f;
#pragma unroll
                for (int k = 0; k < 4; ++k) a += h2f_bits(w[k] & 0xFFFFu) + h2f_bits(w[k] >> 16);
                part[u] = a;
              }
              const float sx = (part[0] + part[1]) + (part[2] + part[3]);
              const __half hi = __float2half_rn(sx);
              const __half lo = __float2half_rn(sx - __half2float(hi));
              const uint32_t pair = (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
              uint8_t* b2 = smem + C::kB2Off + (j >> 1) * C::kB2Tile;
              *reinterpret_cast<uint2*>(b2 + sw128_off(gt, 32 * (j & 1) + 4 * gg)) = make_uint2(pair, pair);
            }
            fence_proxy_async();  // the MMA (async proxy) reads these
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[as]);
          {  // the row's d for the epilogue
            const uint32_t ps = i % kTcNP;
            if (!warp_wait(&pempty[ps], ((i / kTcNP) & 1) ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
            params[ps * 128 + r] = d;
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfull[ps]);
          }
        }
      }
    } else {
      // ---------------------------------------------------------------- epilogue
      griddep_wait();  // outputs are written (and aux read) only after the preceding kernel has completed
      const int q = warp & 3;
      const int r = q * 32 + lane;
      const int et = threadIdx.x - kTcWarpEpi0 * 32;  // 0..127
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      const uint32_t ex_local = smem_u32(ex);
      uint32_t i = 0, tc = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < p.tiles; tile += G, ++tc) {
        float acc[TP];
#pragma unroll
        for (int t = 0; t < TP; ++t) acc[t] = 0.f;
        for (int j = 0; j < sr; ++j, ++i) {
          const uint32_t ds = i % ND;
          if (!warp_wait(&dfull[ds], (i / ND) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ps = i % kTcNP;
          if (!warp_wait(&pfull[ps], (i / kTcNP) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
          const float d = params[ps * 128 + r];
#pragma unroll
          for (int h16 = 0; h16 < TP / 16; ++h16) {  // 16 columns at a time (registers)
            uint32_t v[16];
            tmem_ld16(tl + C::kD1Col + ds * TP + 16 * h16, v);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 16; ++t) acc[16 * h16 + t] = fmaf(d, __uint_as_float(v[t]), acc[16 * h16 + t]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&dempty[ds]);
            mbar_arrive(&pempty[ps]);
          }
        }
        if (!ok) break;
        {
          const uint32_t r2 = tc & 1;
          if (!warp_wait(&d2full[r2], (tc >> 1) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int h16 = 0; h16 < TP / 16; ++h16) {
            uint32_t v[16];
            tmem_ld16(tl + C::kD2Col + r2 * TP + 16 * h16, v);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 16; ++t) acc[16 * h16 + t] = acc[16 * h16 + t] - __uint_as_float(v[t]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&d2empty[r2]);
        }
        const int row0 = tile * p.rt;
        if (ks == 1) {
          const int row = row0 + r;
          if (r < p.rt && row < p.N) {
#pragma unroll
            for (int t = 0; t < TP; ++t)
              if (t < p.M) tc_store<EPI, OUT_F16>(p, t, row, acc[t]);
          }
          continue;
        }
        // cluster reduction: the rows are split in rank order, `per` rows per CTA; every CTA stores its partial sum
        // of each row into the owner CTA's shared memory (slot [rank][t][row - owner's first row]; remote stores,
        // so nothing waits on a remote load), and the owner adds the KS slots of its rows in rank order (deterministic)
        if (!warp_wait_cluster(exempty, (tc & 1) ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
        const int per = (p.rt + ks - 1) / ks;
        if (r < p.rt) {  // owner o = r / per < ks
          const int o = r / per;
          const uint32_t dst = mapa_shared(ex_local + (uint32_t)((int)rank * TP * per + r - o * per) * 4, (uint32_t)o);
#pragma unroll
          for (int t = 0; t < TP; ++t)
            if (t < p.M) st_cluster_f32(dst + (uint32_t)(t * per) * 4, acc[t]);
        }
        __syncwarp();
        if (lane == 0)
          for (int c = 0; c < ks; ++c) mbar_arrive_cluster_release(mapa_shared(smem_u32(exfull), (uint32_t)c));
        if (!warp_wait_cluster(exfull, tc & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
        const int r0 = (int)rank * per, r1 = min(p.rt, r0 + per);
        const int nr = r1 - r0;
        for (int e = et; e < nr * p.M; e += 128) {
          const int t = e / nr, rr = e % nr;
          float s = ex[t * per + rr];
          for (int c = 1; c < ks; ++c) s = s + ex[(c * TP + t) * per + rr];
          if (row0 + r0 + rr < p.N) tc_store<EPI, OUT_F16>(p, t, row0 + r0 + rr, s);
        }
        __syncwarp();
        if (lane == 0)
          for (int c = 0; c < ks; ++c) mbar_arrive_cluster_release(mapa_shared(smem_u32(exempty), (uint32_t)c));
      }
    }
  }

  tc_fence_before();
  if (ks > 1) cluster_sync(); else __syncthreads();
  if (warp == kTcWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tc_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(q);
  });
  return fn;
}

template <int TP, int EPI, bool OUT_F16>
cudaError_t tc_launch(const QGemvArgs& a, const GemvTcPlan& pl, cudaStream_t stream) {
  using C = TcCfg<TP>;
  EncodeTiledFn enc = tc_encoder();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw, mx;
  {
    const int64_t window_u64 = (a.kb_off + a.K / 256) * 18;  // 144-byte super-blocks as u64 elements
    cuuint64_t dims[2] = {(cuuint64_t)window_u64, (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)a.w_row_stride};
    cuuint32_t box[2] = {(cuuint32_t)(pl.pitch / 8), (cuuint32_t)pl.rt};
    cuuint32_t ones[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(a.w), dims, strides, box, ones,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    // activations as [K / 64][M][64]: one copy brings a super-block's 4 64-K chunks of TP token rows (rows past M
    // are zero-filled)
    cuuint64_t dims[3] = {64, (cuuint64_t)a.M, (cuuint64_t)(a.K / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)a.ldx * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)TP, 4};
    cuuint32_t ones[3] = {1, 1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(a.x), dims, strides, box, ones,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  TcParams p;
  p.N = (int)a.N;
  p.M = (int)a.M;
  p.K = (int)a.K;
  p.kb_off = (int)a.kb_off;
  p.rt = pl.rt;
  p.tiles = pl.tiles;
  p.ks = pl.ks;
  p.srange = pl.srange;
  p.sw = pl.sw;
  p.pitch = pl.pitch;
  p.x = static_cast<const __half*>(a.x);
  p.ldx = a.ldx;
  p.y = a.y;
  p.ldy = a.ldy;
  p.aux = a.aux;
  p.ldaux = a.ldaux;
  p.status = a.status;
  auto kern = qgemv_tc_kernel<TP, EPI, OUT_F16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
  if (e != cudaSuccess) return e;
  if (pl.ks > 1) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    (void)e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = C::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  int n = 0;
  at[n].id = cudaLaunchAttributeClusterDimension;
  at[n].val.clusterDim.x = pl.ks;
  at[n].val.clusterDim.y = 1;
  at[n].val.clusterDim.z = 1;
  ++n;
  if (launch_overlap()) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, mw, mx, p);
}

template <int TP>
cudaError_t tc_epi(const QGemvArgs& a, const GemvTcPlan& pl, cudaStream_t s) {
  if (a.epilogue == kEpiResid) return tc_launch<TP, kEpiResid, false>(a, pl, s);
  if (a.epilogue == kEpiSwiglu)
    return a.y_f16 ? tc_launch<TP, kEpiSwiglu, true>(a, pl, s) : tc_launch<TP, kEpiSwiglu, false>(a, pl, s);
  return a.y_f16 ? tc_launch<TP, kEpiStore, true>(a, pl, s) : tc_launch<TP, kEpiStore, false>(a, pl, s);
}

// Resident clusters of `ks` CTAs of this kernel (one CTA per SM); 0 when the device cannot place them.
int tc_max_clusters(int tp, int ks) {
  const void* k = tp == 16 ? (const void*)qgemv_tc_kernel<16, kEpiStore, false>
                           : (const void*)qgemv_tc_kernel<32, kEpiStore, false>;
  const int smem = tp == 16 ? TcCfg<16>::kAlloc : TcCfg<32>::kAlloc;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

struct ClusterCaps {
  int dev = -1;
  int n[2][5] = {};  // [tp == 32][ks]
};

}  // namespace

GemvTcPlan qgemv_tc_plan(int type, int64_t N, int64_t K, int64_t M, int num_sms, int device) {
  GemvTcPlan pl = {};
  if (type != 12 || M < 1 || M > 32 || K % 256 || N < 1) return pl;
  static std::mutex mu;
  static ClusterCaps caps[64];
  if (device < 0 || device >= 64) return pl;
  const int tp = M <= 16 ? 16 : 32;
  const int maxr = tp == 16 ? TcCfg<16>::kMaxRange : TcCfg<32>::kMaxRange;
  int clusters[5] = {0, 0, 0, 0, 0};
  {
    std::lock_guard<std::mutex> lk(mu);
    ClusterCaps& c = caps[device];
    if (c.dev != device) {
      for (int t = 0; t < 2; ++t)
        for (int k : {1, 2, 4}) c.n[t][k] = k == 1 ? 0 : tc_max_clusters(t ? 32 : 16, k);
      c.dev = device;
    }
    for (int k : {2, 4}) clusters[k] = c.n[tp == 32][k];
  }
  clusters[1] = num_sms;
  const int S = (int)(K / 256);
  double best = 0;
  for (int ks : {1, 2, 4}) {
    if (S % ks) continue;
    const int sr = S / ks;
    if (sr > maxr) continue;
    int slots = clusters[ks];
    if (ks > 1 && slots * ks > num_sms) slots = num_sms / ks;
    if (slots < 1) continue;
    // fewest rounds of tiles with rows <= 128, then the smallest tile that keeps that round count
    const int64_t tiles128 = (N + 127) / 128;
    const int64_t rounds = (tiles128 + slots - 1) / slots;
    int rt = (int)((N + rounds * slots - 1) / (rounds * slots));
    if (rt < 1) rt = 1;
    if (rt > 128) rt = 128;
    const int64_t tiles = (N + rt - 1) / rt;
    // per-CTA cost (cycles per super-block and tile): weight bytes at twice the fair share of HBM, the decode
    // (one 16-warp pass per 32-row quarter), the 18 MMAs; plus the cross-CTA reduction per tile
    const double mem = rt * 3.0;
    const double dec = ((rt + 31) / 32) * 115.0 * (rt <= 64 ? 1.5 : 1.0);
    const double mma = 9.0 * tp;
    double cost = (double)rounds * sr * (mem > dec ? (mem > mma ? mem : mma) : (dec > mma ? dec : mma));
    if (ks > 1) cost += (double)rounds * 300.0 * ks;
    if (!pl.ok || cost < best) {
      best = cost;
      pl.ok = 1;
      pl.tp = tp;
      pl.ks = ks;
      pl.rt = rt;
      pl.tiles = (int)tiles;
      pl.grid = (int)(tiles < slots ? tiles : slots) * ks;
      pl.srange = sr;
      pl.sw = sr % 2 == 0 ? 2 : 1;
      pl.pitch = pl.sw == 2 ? kTcWPitch2 : kTcWPitch1;
    }
  }
  return pl;
}

cudaError_t launch_qgemv_tc(const QGemvArgs& a, const GemvTcPlan& pl, cudaStream_t stream) {
  if (!pl.ok || a.type != 12) return cudaErrorInvalidValue;
  return pl.tp == 16 ? tc_epi<16>(a, pl, stream) : tc_epi<32>(a, pl, stream);
}

}  // namespace yah
