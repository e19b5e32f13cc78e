// Quantised tile GEMM for sm_100a: GGUF Q8_0 / Q3_K / Q4_K / Q5_K / Q6_K / IQ4_XS weights x f16 activations, f32 accumulation in TMEM.
//
// Reference: engine/gpu/loom/tools/gen_gemm_tile.py (the tile GEMM, kinds kstore / kres / swiglu :309-322, store
// :1229-1245) with the decoders of engine/gpu/loom/tools/gen_gemm_decode.py. Like the reference, the weight tile
// is decoded inside the K loop to exactly the f16 values of the reference dequant, multiplied in f16 with f32
// accumulation, and written token-major: out[t][r] at t * ldy + r (gen_gemm_tile.py:1230-1231).
//
// B200 design (one persistent CTA per SM, 23 warps). The K loop advances in stages of 128 K (two 64-K blocks):
//   warp 0      activation producer: per stage two TMA loads of 64-K activation tiles (BN tokens x 128 B,
//               128-byte swizzle) into one of 3 shared-memory slots.
//   warp 22     weight producer: TMA loads of the raw super-blocks of 128 weight rows (one 256-K super-block per
//               slot), decoupled from the activation ring so weights stream ahead on their own.
//   warp 1      MMA issuer (one thread): per stage one barrier wait, one fence, 8 x tcgen05.mma.kind::f16
//               (A = weights from TMEM, B = activations from shared memory, D = f32 in TMEM) and the commits
//               that free the stage. tcgen05.mma issue is serialised with everything else the issuing thread
//               executes, so its instruction stream is kept to that minimum: descriptors precomputed, the
//               activation-ready check folded into the A-stage barrier.
// 2-SM pairs (default): a cluster of 2 CTAs runs tcgen05.mma.cta_group::2 with M = 256: each CTA decodes its
// own 128 weight rows into its TMEM and stages half of the tile's tokens, so each SM's shared memory carries half
// of the activation traffic; the first CTA issues the MMAs and commits to both CTAs' barriers.
// TMEM layout: NACC accumulator regions of BN columns (2 for BN <= 192, so an epilogue overlaps the next
// accumulation; 1 for BN = 256) and then the A stages of 128 K (64 columns each, up to 4).
//   warps 2-17  four dequant warpgroups: (first / second 64-K block of a stage) x (even / odd stages), so each
//               warp has two stages of MMA time for its decode. Thread = weight row (= TMEM lane): it decodes its
//               row's 64 values to f16 pairs in registers and tcgen05.st's them into the A stage in TMEM (after
//               the accumulators), so the dequantised tile never touches shared memory. Before marking the A
//               stage full it also waits for the stage's activation tile, so the MMA issuer waits on one
//               barrier per stage.
//   warps 18-21 epilogue: tcgen05.ld of the accumulator, kstore / kres / swiglu, token-major global stores.
// Accuracy: the tensor core's f32 accumulation truncates (round toward zero), which at K = 14336 costs ~0.04
// absolute on |y| ~ 2000. For K above 4096 each tile is accumulated in chunks of `kcb` 64-K blocks, each chunk
// starting from zero in the free accumulator region; the epilogue sums the chunk results in f32 round-to-nearest
// in a per-CTA scratch buffer (L2-resident) while the MMA fills the other region.
// Tiles are 128 weight rows x up to BN tokens. The persistent schedule splits the (row tile, 16-token unit) space
// into equal contiguous ranges per CTA, so every SM gets the same MMA work (no wave-quantisation tail).
// Split K (few tokens, so too few tiles for the SMs): every accumulation chunk of a tile is a work unit of its own;
// a CTA writes its chunk's f32 result to a workspace and split_reduce_kernel adds the chunks of each output in
// chunk order and applies the epilogue, the same additions in the same order as the single-CTA chunk sum, so the
// result is bit-identical to the unsplit GEMM with the same chunk length.
// Every mbarrier wait is bounded (ptx.cuh mbar_wait); on a timeout the kernel records a status code, drains its
// own in-flight TMA copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <type_traits>

#include "decode.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace yah {
namespace {

constexpr int kThreads = 736;
constexpr int kBM = 128;  // weight rows per tile = TMEM lanes
constexpr int kDqGroups = 4;  // dequant warpgroups: (64-K block of the stage) x (stage parity)
constexpr int kWarpX = 0, kWarpMma = 1, kWarpDq0 = 2, kWarpEpi0 = 2 + 4 * kDqGroups, kWarpW = kWarpEpi0 + 4;

template <int T>
struct Fmt;
template <>
struct Fmt<8> {  // Q8_0: 8 blocks of 34 B as one 272-B super-block
  static constexpr int kSB = 272, kBox = 272, kNSW = 2;
};
template <>
struct Fmt<12> {  // Q4_K
  static constexpr int kSB = 144, kBox = 144, kNSW = 3;
};
template <>
struct Fmt<14> {  // Q6_K: a 224-B window from the 16-B boundary at or below the super-block
  static constexpr int kSB = 210, kBox = 224, kNSW = 2;
};
template <>
struct Fmt<13> {  // Q5_K (176-B super-blocks stay 16-B aligned)
  static constexpr int kSB = 176, kBox = 176, kNSW = 2;
};
template <>
struct Fmt<11> {  // Q3_K: a 128-B window from the 16-B boundary at or below the super-block
  static constexpr int kSB = 110, kBox = 128, kNSW = 3;
};
template <>
struct Fmt<23> {  // IQ4_XS: a 144-B window (super-blocks are 8-B aligned)
  static constexpr int kSB = 136, kBox = 144, kNSW = 3;
};
// Formats whose super-blocks do not all start 16-byte aligned: TMA copies a window from the boundary below.
__host__ __device__ constexpr bool windowed(int T) { return T == 14 || T == 11 || T == 23; }

// TMEM (512 columns) holds NACC accumulator regions of BN columns, then NA A stages of 128 K (64 columns).
// NACC = 2 overlaps an epilogue with the next accumulation and is needed for chunked accumulation; NACC = 1
// (BN = 256) trades that for four A stages.
template <int BN, int NACC>
struct TCfg {
  static constexpr int kACol0 = NACC * BN;
  static constexpr int kNA = (512 - NACC * BN) / 64 > 4 ? 4 : (512 - NACC * BN) / 64;
  static_assert(kNA >= 2, "TMEM columns");
};

// Activation slots of 128 K: a CTA stages XR token rows (all of the tile's, or half in a pair).
template <int XR>
struct XCfg {
  static constexpr int kSub = XR * 128;     // one 64-K tile: XR rows x 64 f16
  static constexpr int kStage = 2 * kSub;   // a stage holds two
  static constexpr int kNSX = XR <= 128 ? 4 : 3;
};

struct KParams {
  int N, K, M, kb_off;
  int kcb;  // 64-K blocks per accumulation chunk (>= K / 64: one chunk)
  void* y;
  int64_t ldy;
  const float* aux;
  int64_t ldaux;
  float* scratch;       // [grid][BN][128] f32 chunk sums (chunked accumulation only)
  int* status;
  int64_t total_units;  // row tiles (of 128 rows, or 256 for a pair) x 16-token units
  int upr;              // 16-token units per row tile
  int ncta;             // CTAs per tile: 1, or 2 for a 2-SM pair
  int nsplit;           // 1, or the accumulation chunks of a tile when each is its own unit (split K)
  int tma_store;        // 1: the output is written with TMA stores through shared memory (tmap_y is valid)
  int aux_tma;          // 1: the epilogue's aux operand is prefetched by TMA (tmap_aux is valid)
  int help;             // 1: the dequant warps help drain the accumulator (drain_share; one chunk per unit)
  int whole;            // 1: the schedule hands out whole tiles (see Sched)
  int64_t total_tiles;  // row tiles x chunks (split K) x token tiles of BN
  int tpr;              // token tiles of BN per row tile
  int nsl;              // > 0: token slices (output token t at ysl[t / slice_rows] + (t % slice_rows) * ldy)
  int64_t slice_rows;
  void* ysl[kMaxSlices];
};

template <int T, int XR, int AUXB = 0>  // XR: activation rows a CTA stages (the tile's tokens, or half in a pair)
struct Smem {
  static constexpr int kWStage = ((kBM * Fmt<T>::kBox + 16) + 127) / 128 * 128;
  static constexpr int kXBytes = XCfg<XR>::kNSX * XCfg<XR>::kStage;
  static constexpr int kWOff = kXBytes;
  static constexpr int kOutOff = kWOff + Fmt<T>::kNSW * kWStage;  // 2 output staging buffers (TMA stores)
  static constexpr int kOutBuf = 4096;                            // 128 rows x 16 f16 or 8 f32 tokens
  static constexpr int kAuxOff = kOutOff + 2 * kOutBuf;             // aux prefetch ring (AUXB bytes)
  static constexpr int kBarOff = kAuxOff + AUXB;
  // barriers: xfull, xempty [NSX]; wfull, wempty [NSW]; afull, aempty [4]; accfull, accempty [2]; drain;
  // auxfull [4]
  static constexpr int kNumBars = 2 * XCfg<XR>::kNSX + 2 * Fmt<T>::kNSW + 2 * 4 + 5 + 4;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kTmemSlotOff + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment of the base
};

// Tokens the epilogue drains per step: 16 for f16 outputs, 8 for f32, and 8 for the swiglu epilogue (its gate
// values and silu on 16 tokens per step spilled registers under the 80-register cap of 736 threads).
__host__ __device__ constexpr int epi_chunk(int epi, bool out_f16) { return out_f16 && epi != kEpiSwiglu ? 16 : 8; }

// The epilogue's aux operand (residual, or the swiglu gate; f32 [M][ldaux]) is prefetched by TMA into a ring of
// kDepth slots of 128 rows x CH tokens, ahead of the accumulator it is combined with, so the epilogue does not wait
// one global round trip per CH tokens. The ring takes what shared memory the stages leave (4, 2 or no slots).
constexpr int kSmemLimit = 227 * 1024;
template <int T, int XR, int EPI, bool OUT_F16>
struct AuxCfg {
  static constexpr int kCH = epi_chunk(EPI, OUT_F16);
  static constexpr int kSlot = kCH * 128 * 4;
  static constexpr int kBase = Smem<T, XR, 0>::kAlloc;
  static constexpr int kDepth = (EPI == kEpiStore || EPI == kEpiFfn) ? 0
                                : kBase + 4 * kSlot <= kSmemLimit ? 4
                                : kBase + 2 * kSlot <= kSmemLimit ? 2 : 0;
  static constexpr int kBytes = kDepth * kSlot;
};

// The persistent schedule: CTA b owns units [b * total / G, (b + 1) * total / G) of the (row tile, chunk, 16-token
// unit) space, walked row tile by row tile, at most BN / 16 units per tile. kp is the accumulation chunk under
// split K (0 otherwise).
// Whole tiles instead (p.whole, chosen on the host when it needs fewer K loops on the busiest CTA): CTA b owns tiles
// [b * T / G, (b + 1) * T / G) of the (row tile, chunk, BN-token tile) space. A tile's K loop costs about the same
// at any token count up to BN (per-stage issue time, measured), so a range that ends inside a row tile pays a second
// K loop for its last units; with few tiles per CTA (small shards) that doubled the busiest CTAs' time.
template <int BN>
struct Sched {
  int64_t u, end;
  int upr, M, nsplit, whole, tpr;
  __device__ Sched(const KParams& p) : upr(p.upr), M(p.M), nsplit(p.nsplit), whole(p.whole), tpr(p.tpr) {
    const int64_t G = gridDim.x / p.ncta, b = blockIdx.x / p.ncta;  // a pair shares one range
    const int64_t total = whole ? p.total_tiles : p.total_units;
    u = b * total / G;
    end = (b + 1) * total / G;
  }
  __device__ bool next(int& rt, int& kp, int& t0, int& nt) {
    if (u >= end) return false;
    if (whole) {
      const int vt = (int)(u / tpr);
      rt = vt / nsplit;
      kp = vt - rt * nsplit;
      t0 = (int)(u % tpr) * BN;
      nt = min(BN, M - t0);
      ++u;
      return true;
    }
    const int vt = (int)(u / upr);
    rt = vt / nsplit;
    kp = vt - rt * nsplit;
    const int tu = (int)(u % upr);
    int nu = min(BN / 16, upr - tu);
    if ((int64_t)nu > end - u) nu = (int)(end - u);
    t0 = tu * 16;
    nt = min(nu * 16, M - t0);
    u += nu;
    return true;
  }
};

// silu(g) = g / (1 + e^-g) with CUDA's fast exponential and fast division (__fdividef: ~2 ulp; a divisor that has
// overflowed to infinity, g below about -88, gives g * 0 = -0, the limit). The IEEE division it replaces took its
// slow path whenever e^-g overflowed, frequent with gate values of a few hundred, and halved the swiglu epilogue's
// rate (914-1117 us against 535 us for the residual epilogue at 4096 x 14336 x 4096).
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Shared drain of a single accumulator region (NACC = 1, plain store): while a full accumulator is drained the MMAs
// wait for it, and so do the dequant warps, whose A ring is full by then. So the epilogue warp and the four dequant
// warps of each TMEM lane quarter drain it together: warp slot k (0 the epilogue warp, 1 + g the dequant warp of
// group g) takes the 8-token chunks c with c % kDrainWarps == k and stores them straight to global memory (the 32
// lanes of a warp are 32 consecutive output rows of one token: one coalesced store per token). tq: the TMEM address
// of lane quarter q's accumulator.
constexpr int kDrainWarps = 5;
template <bool OUT_F16, int NCTA>
__device__ __forceinline__ void drain_share(const KParams& p, uint32_t tq, int q, int lane, int slot, int rt,
                                            uint32_t rank, int t0, int nt, int64_t tsplit) {
  constexpr int CH = 8;  // 8 tokens per chunk: up to 32 chunks over the 20 warps of a CTA
  const int row = (rt * NCTA + (int)rank) * kBM + q * 32 + lane;
  const bool row_ok = row < p.N;
  using E = typename std::conditional<OUT_F16, __half, float>::type;
  E* yp = reinterpret_cast<E*>(p.y) + (tsplit + t0 + slot * CH) * p.ldy + row;
  const int64_t step = (int64_t)kDrainWarps * CH * p.ldy;
  for (int j0 = slot * CH; j0 < nt; j0 += kDrainWarps * CH, yp += step) {  // the same trip count for every lane
    uint32_t v[CH];
    tmem_ld8(tq + j0, v);
    tmem_wait_ld();
    const int jn = min(CH, nt - j0);
    if (row_ok) {
      E* o = yp;
      if (p.nsl > 0) {  // token slices: a chunk of 8 tokens never crosses one (slice_rows % 16 == 0)
        const int64_t t = t0 + j0;
        o = reinterpret_cast<E*>(p.ysl[t / p.slice_rows]) + (t % p.slice_rows) * p.ldy + row;
      }
#pragma unroll
      for (int jj = 0; jj < CH; ++jj, o += p.ldy) {
        if (jj >= jn) break;
        if (OUT_F16) *reinterpret_cast<__half*>(o) = __float2half_rn(__uint_as_float(v[jj]));
        else *reinterpret_cast<float*>(o) = __uint_as_float(v[jj]);
      }
    }
  }

}

template <int T, int BN, int NACC, int EPI, bool OUT_F16, bool PAIR, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ CUtensorMap tmap_aux,
                    const KParams p) {
  constexpr int XROWS = PAIR ? BN / 2 : BN;  // a CTA of a pair stages half of the tokens
  using AC = AuxCfg<T, XROWS, EPI, OUT_F16>;
  using S = Smem<T, XROWS, AC::kBytes>;
  constexpr int XSUB = XCfg<XROWS>::kSub;
  constexpr int XST = XCfg<XROWS>::kStage;
  constexpr int kNSX = XCfg<XROWS>::kNSX;
  constexpr int kNA = TCfg<BN, NACC>::kNA;
  constexpr int ACOL = TCfg<BN, NACC>::kACol0;
  constexpr int NSW = Fmt<T>::kNSW;
  constexpr int WBOX = Fmt<T>::kBox;
  constexpr int NCTA = PAIR ? 2 : 1;
  // weight rows whose outputs a CTA produces per tile: 128 (TMEM lanes), or 64 under kEpiFfn (lanes 0-63 gate,
  // 64-127 the same rows of up)
  constexpr int kTileRows = EPI == kEpiFfn ? 64 : kBM;
  // one accumulator region, a plain store and one accumulation chunk per unit: the dequant warps help drain it
  // (drain_share; the host sets p.help)
  constexpr bool HELP_T = NACC == 1 && EPI == kEpiStore;
  const bool HELP = HELP_T && p.help != 0;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* xfull = bars;
  uint64_t* xempty = xfull + kNSX;
  uint64_t* wfull = xempty + kNSX;
  uint64_t* wempty = wfull + NSW;
  uint64_t* afull = wempty + NSW;    // the pair's first CTA counts both CTAs' dequant warps
  uint64_t* aempty = afull + 4;
  uint64_t* accfull = aempty + 4;    // [2]
  uint64_t* accempty = accfull + 2;  // [2], counts both CTAs' epilogue warps
  uint64_t* drain = accempty + 2;
  uint64_t* auxfull = drain + 1;     // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kTmemSlotOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0;  // 0 issues the pair's MMAs
  const int nst = p.K / 128;                  // 128-K stages per tile
  const int sch = p.kcb / 2;                  // stages per accumulation chunk
  const int nch = (nst + sch - 1) / sch;      // accumulation chunks per tile
  constexpr bool split = SPLIT;               // one chunk per work unit (then p.nsplit == nch)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNSX; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], 1);
    }
    for (int i = 0; i < NSW; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 4 * kDqGroups);  // every dequant warp reads one 64-K block of each super-block
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&afull[i], 8 * NCTA);   // every dequant warp (each also saw its activation tile land)
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], (HELP ? 4 + 4 * kDqGroups : 4) * NCTA);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&auxfull[i], 1);
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Barriers the pair's first CTA owns, as addresses the second CTA can arrive on.
  const uint32_t afull_lead = PAIR ? mapa_shared(smem_u32(afull), 0) : smem_u32(afull);
  const uint32_t accempty_lead = PAIR ? mapa_shared(smem_u32(accempty), 0) : smem_u32(accempty);

  if (warp == kWarpX) {
    // ------------------------------------------------------------------ activation producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      Sched<BN> sc(p);
      int rt, kp, t0, nt;
      uint32_t s = 0;  // stages issued
      bool ok = true;
      while (ok && sc.next(rt, kp, t0, nt)) {
        // a pair splits the tile's tokens: CTA r holds columns [r * n / 2, (r + 1) * n / 2) of the MMA's N
        const int ty = PAIR ? t0 + (int)rank * (((nt + 31) & ~31) / 2) : t0;
        const int st0 = split ? kp * sch : 0, st1 = split ? min(nst, st0 + sch) : nst;
        for (int st = st0; st < st1; ++st, ++s) {
          const uint32_t xs = s % kNSX, xph = (s / kNSX) & 1;
          if (!mbar_wait(&xempty[xs], xph ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&xfull[xs], XST);
          tma_load_2d(smem + xs * XST, &tmap_x, &xfull[xs], st * 128, ty);
          tma_load_2d(smem + xs * XST + XSUB, &tmap_x, &xfull[xs], st * 128 + 64, ty);
        }
      }
      for (uint32_t i = (s > (uint32_t)kNSX ? s - kNSX : 0); i < s; ++i)
        mbar_wait(&xfull[i % kNSX], (i / kNSX) & 1, p.status, kStatusTimeoutDrain, false);
    }
  } else if (warp == kWarpW) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      Sched<BN> sc(p);
      int rt, kp, t0, nt;
      uint32_t s = 0;
      bool ok = true;
      while (ok && sc.next(rt, kp, t0, nt)) {
        const int row0 = (rt * NCTA + (int)rank) * kTileRows;
        const int sb0 = split ? kp * sch / 2 : 0, sb1 = split ? min(nst, (kp + 1) * sch) / 2 : p.K / 256;
        for (int sb = sb0; sb < sb1; ++sb, ++s) {
          const uint32_t ws = s % NSW, wph = (s / NSW) & 1;
          if (!mbar_wait(&wempty[ws], wph ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&wfull[ws], kBM * WBOX);
          const int64_t sbg = (int64_t)p.kb_off + sb;
          int xw;
          if (windowed(T)) xw = (int)(((sbg * Fmt<T>::kSB) & ~int64_t(15)) >> 1);
          else xw = (int)(sbg * (Fmt<T>::kSB / 2));
          if constexpr (EPI == kEpiFfn) {  // gate rows to stage rows 0-63, the same up rows to 64-127
            tma_load_2d(smem + S::kWOff + ws * S::kWStage, &tmap_w, &wfull[ws], xw, row0);
            tma_load_2d(smem + S::kWOff + ws * S::kWStage + 64 * WBOX, &tmap_aux, &wfull[ws], xw, row0);
          } else {
            tma_load_2d(smem + S::kWOff + ws * S::kWStage, &tmap_w, &wfull[ws], xw, row0);
          }
        }
      }
      for (uint32_t i = (s > (uint32_t)NSW ? s - NSW : 0); i < s; ++i)
        mbar_wait(&wfull[i % NSW], (i / NSW) & 1, p.status, kStatusTimeoutDrain, false);
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------------ MMA issuer (pair: first CTA only)
    if (lane == 0 && rank == 0) {
      Sched<BN> sc(p);
      int rt, kp, t0, nt;
      uint32_t s = 0, u = 0;  // stage and accumulation-unit counters
      bool ok = true;
      const uint64_t bd0 = sdesc_sw128(smem_u32(smem));
      const uint64_t bstep = (uint64_t)(XST >> 4), bsub = (uint64_t)(XSUB >> 4);
      const uint32_t a0 = tmem + ACOL;
      while (ok && sc.next(rt, kp, t0, nt)) {
        const uint32_t idesc = PAIR ? idesc_f16_f32(2 * kBM, (nt + 31) & ~31) : idesc_f16_f32(kBM, (nt + 15) & ~15);
        const int ch0 = split ? kp : 0, ch1 = split ? kp + 1 : nch;
        for (int ch = ch0; ok && ch < ch1; ++ch, ++u) {
          const uint32_t r = u % NACC, rph = (u / NACC) & 1;
          const bool acc_free = mbar_wait(&accempty[r], rph ^ 1, p.status, kStatusTimeoutEmpty);
          if (!acc_free) { ok = false; break; }
          tc_fence_after();
          const uint32_t dt = tmem + r * BN;
          const int st1 = min(nst, (ch + 1) * sch);
          for (int st = ch * sch; st < st1; ++st, ++s) {
            const uint32_t as = s % kNA, xs = s % kNSX;
            const bool ready = mbar_wait(&afull[as], (s / kNA) & 1, p.status, kStatusTimeoutFull);
            if (!ready) { ok = false; break; }
            tc_fence_after();
            const uint32_t a = a0 + as * 64;
            const uint64_t b = bd0 + xs * bstep;
            const uint32_t acc0 = st == ch * sch ? 0u : 1u;
            if (PAIR) {
              mma_f16_ts_pair(dt, a, b, idesc, acc0);
              mma_f16_ts_pair(dt, a + 8, b + 2, idesc, 1u);
              mma_f16_ts_pair(dt, a + 16, b + 4, idesc, 1u);
              mma_f16_ts_pair(dt, a + 24, b + 6, idesc, 1u);
              mma_f16_ts_pair(dt, a + 32, b + bsub, idesc, 1u);
              mma_f16_ts_pair(dt, a + 40, b + bsub + 2, idesc, 1u);
              mma_f16_ts_pair(dt, a + 48, b + bsub + 4, idesc, 1u);
              mma_f16_ts_pair(dt, a + 56, b + bsub + 6, idesc, 1u);
              mma_commit_pair(&aempty[as], 3);
              mma_commit_pair(&xempty[xs], 3);
            } else {
              mma_f16_ts(dt, a, b, idesc, acc0);
              mma_f16_ts(dt, a + 8, b + 2, idesc, 1u);
              mma_f16_ts(dt, a + 16, b + 4, idesc, 1u);
              mma_f16_ts(dt, a + 24, b + 6, idesc, 1u);
              mma_f16_ts(dt, a + 32, b + bsub, idesc, 1u);
              mma_f16_ts(dt, a + 40, b + bsub + 2, idesc, 1u);
              mma_f16_ts(dt, a + 48, b + bsub + 4, idesc, 1u);
              mma_f16_ts(dt, a + 56, b + bsub + 6, idesc, 1u);
              mma_commit(&aempty[as]);
              mma_commit(&xempty[xs]);
            }
          }
          if (!ok) break;
          if (PAIR) mma_commit_pair(&accfull[r], 3); else mma_commit(&accfull[r]);
        }
      }
      // Drain: every MMA issued by this thread completes before TMEM is released.
      if (PAIR) mma_commit_pair(drain, 1); else mma_commit(drain);
      mbar_wait(drain, 0, p.status, kStatusTimeoutDrain, false);
    }
  } else if (warp < kWarpEpi0) {
    // ------------------------------------------------------------------ dequant warpgroups
    const int g = (warp - kWarpDq0) >> 2;
    const int half = g & 1;                   // 0: first 64-K block of the stage, 1: second
    const uint32_t parity = (uint32_t)(g >> 1);  // stages this warpgroup handles: s % 2 == parity
    const int q = warp & 3;                   // TMEM lane quarter
    const int r = q * 32 + lane;              // row within the CTA's 128 rows
    Sched<BN> sc(p);
    int rt, kp, t0, nt;
    uint32_t s = 0;
    bool ok = true;
    const uint32_t wbase = smem_u32(smem + S::kWOff);
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + ACOL + 32 * half;
    // HELP: the unit (tile) whose drain this warp still owes, helped once the warp has decoded the stages whose A
    // slots the MMAs can refill only after that drain, or at the latest at the end of the next unit
    int h_rt = -1, h_t0 = 0, h_nt = 0, h_kp = 0;
    uint32_t h_u = 0, units = 0;
    auto help = [&]() -> bool {
      // warp-uniform: the drain's tcgen05.ld must never run on part of the warp
      if (!__all_sync(0xffffffffu, mbar_wait(&accfull[0], h_u & 1, p.status, kStatusTimeoutFull))) return false;
      tc_fence_after();
      drain_share<OUT_F16, NCTA>(p, tmem + ((uint32_t)(q * 32) << 16), q, lane, 1 + g, h_rt, rank, h_t0, h_nt,
                                 split ? (int64_t)h_kp * p.M : 0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(accempty_lead);
        else mbar_arrive(&accempty[0]);
      }
      h_rt = -1;
      return true;
    };
    while (ok && sc.next(rt, kp, t0, nt)) {
      const int st0 = split ? kp * sch : 0, st1 = split ? min(nst, st0 + sch) : nst;
      const uint32_t unit_start = s;
      for (int st = st0; st < st1; ++st, ++s) {
        if ((s & 1) != parity) continue;
        if (HELP && h_rt >= 0 && s >= unit_start + kNA && !help()) { ok = false; break; }
        const int kb = 2 * st + half;              // 64-K block within the tile
        const uint32_t sbc = (s >> 1), ws = sbc % NSW, wph = (sbc / NSW) & 1;  // super-block = 2 stages
        const uint32_t as = s % kNA, aph = (s / kNA) & 1;
        if (!mbar_wait(&wfull[ws], wph, p.status, kStatusTimeoutFull)) { ok = false; break; }
        if (!mbar_wait(&aempty[as], aph ^ 1, p.status, kStatusTimeoutEmpty)) { ok = false; break; }
        const int j = kb & 3;
        const uint32_t rb = wbase + ws * S::kWStage + r * WBOX;
        uint32_t v[32];
        const int o = windowed(T) ? (int)((((int64_t)p.kb_off + (kb >> 2)) * Fmt<T>::kSB) & 15) : 0;
        if (T == 12) {
          q4k_decode_smem(rb, j, v);
        } else if (T == 8) {
          q80_decode_smem(rb, j, v);
        } else if (T == 13) {
          q5k_decode_smem(rb, j, v);
        } else if (T == 11) {
          q3k_decode_smem(rb, j, o, v);
        } else if (T == 23) {
          iq4xs_decode_smem(rb, j, o, v);
        } else {
          q6k_decode_smem(rb, j, o, v);
        }
        __syncwarp();  // the warp's only read of this weight slot is done
        if (lane == 0) mbar_arrive(&wempty[ws]);
        tmem_st32(tl + as * 64, v);
        tmem_wait_st();
        tc_fence_before();
        if (!mbar_wait(&xfull[s % kNSX], (s / kNSX) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
        __syncwarp();
        if (lane == 0) {
          if (PAIR) mbar_arrive_cluster(afull_lead + as * 8);
          else mbar_arrive(&afull[as]);
        }
      }
      if (HELP && ok) {
        if (h_rt >= 0 && !help()) { ok = false; break; }  // a unit too short to have triggered it
        h_rt = rt, h_t0 = t0, h_nt = nt, h_kp = kp, h_u = units;
      }
      ++units;
    }
    if (HELP && ok && h_rt >= 0) help();
    if (p.nsl > 0) __threadfence_system();  // token slices: see the epilogue's end
  } else if (warp < kWarpW) {
    // ------------------------------------------------------------------ epilogue
    // Accumulator columns are drained CH at a time (CH = 16 f16 / 8 f32 tokens); the final values go to a
    // [CH tokens][128 rows] shared-memory buffer (double-buffered) written out by one TMA store, or, when the
    // output layout does not allow TMA, by direct stores.
    constexpr int CH = epi_chunk(EPI, OUT_F16);
    constexpr int ES = OUT_F16 ? 2 : 4;
    const int q = warp & 3;
    const int rloc = q * 32 + lane;
    const bool leader = warp == kWarpEpi0 && lane == 0;  // issues the TMA stores
    Sched<BN> sc(p);
    int rt, kp, t0, nt;
    uint32_t u = 0, nbuf = 0;
    bool ok = true;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    float* part = p.scratch ? p.scratch + (size_t)blockIdx.x * BN * kBM + rloc : nullptr;
    uint8_t* obuf = smem + S::kOutOff;
    constexpr int AD = AC::kDepth;
    const bool atma = AD > 0 && p.aux_tma;
    uint8_t* abuf = smem + S::kAuxOff;
    uint32_t aux_used = 0;  // aux chunks consumed so far (slot aux_used % AD)
    if (HELP_T && HELP) {  // this warp's share of each drain (drain_share, slot 0)
      while (ok && sc.next(rt, kp, t0, nt)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&accfull[0], u & 1, p.status, kStatusTimeoutFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        drain_share<OUT_F16, NCTA>(p, tl, q, lane, 0, rt, rank, t0, nt, split ? (int64_t)kp * p.M : 0);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR) mbar_arrive_cluster(accempty_lead);
          else mbar_arrive(&accempty[0]);
        }
        ++u;
      }
      ok = false;  // done: skip the staged epilogue below
    }
    while (ok && sc.next(rt, kp, t0, nt)) {
      const int row0 = (rt * NCTA + (int)rank) * kTileRows;
      const int row = row0 + (EPI == kEpiFfn ? (rloc & 63) : rloc);  // the output row of this lane's accumulator
      const bool row_ok = row < p.N;
      const int ncks = (nt + CH - 1) / CH;  // aux chunks of this tile (its last accumulation chunk)
      const int ch0 = split ? kp : 0, ch1 = split ? kp + 1 : nch;
      // split K: this chunk's result goes to rows kp * M + t of the [nsplit * M][N] workspace (p.y)
      const int64_t tsplit = split ? (int64_t)kp * p.M : 0;
      for (int ch = ch0; ch < ch1; ++ch, ++u) {
        const uint32_t r = u % NACC;
        if (atma && ch == ch1 - 1 && leader) {  // prefetch the first aux chunks while the MMAs finish
          for (int k = 0; k < ncks && k < AD; ++k) {
            const uint32_t sl = (aux_used + k) % AD;
            mbar_arrive_expect_tx(&auxfull[sl], AC::kSlot);
            tma_load_2d(abuf + sl * AC::kSlot, &tmap_aux, &auxfull[sl], row0, t0 + k * CH);
          }
        }
        if (!mbar_wait(&accfull[r], (u / NACC) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
        tc_fence_after();
        const bool first = ch == ch0, last = ch == ch1 - 1;
        for (int j0 = 0; j0 < nt; j0 += CH) {
          uint32_t v[CH];
          if constexpr (CH == 16) tmem_ld16(tl + r * BN + j0, v); else tmem_ld8(tl + r * BN + j0, v);
          tmem_wait_ld();
          const int jn = min(CH, nt - j0);
          float val[CH];
          float prev[CH];
          if (!first && row_ok) {  // all partial-sum loads first: one L2 round trip per chunk
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) prev[jj] = jj < jn ? __ldcg(part + (size_t)(j0 + jj) * kBM) : 0.f;
          }
#pragma unroll
          for (int jj = 0; jj < CH; ++jj) {
            float acc = __uint_as_float(v[jj]);
            if (!first && row_ok) acc = prev[jj] + acc;
            val[jj] = acc;
          }
          if (!last) {
            if (row_ok) {
#pragma unroll
              for (int jj = 0; jj < CH; ++jj)
                if (jj < jn) __stcg(part + (size_t)(j0 + jj) * kBM, val[jj]);
            }
            continue;
          }
          if constexpr (EPI == kEpiFfn) {
            // lanes 64-127 hand their up values to lanes 0-63 (same output rows) through shared memory; those
            // store f16(silu(gate) * up), the arithmetic of the swiglu epilogue
            // (obuf: the f32 exchange [CH tokens][64 rows] in its first 4 KB, then two f16 [CH][64] staging tiles
            // for the TMA stores)
            float* ub = reinterpret_cast<float*>(obuf);
            __half* sb = reinterpret_cast<__half*>(obuf + 4096 + (nbuf & 1) * 2048);
            if (rloc >= 64) {
#pragma unroll
              for (int jj = 0; jj < CH; ++jj) ub[jj * 64 + rloc - 64] = val[jj];
            }
            if (p.tma_store && leader) bulk_wait_read<1>();  // the store that last used this staging tile read it
            named_bar(1, 128);
            if (rloc < 64) {
              if (p.tma_store) {
#pragma unroll
                for (int jj = 0; jj < CH; ++jj) sb[jj * 64 + rloc] = __float2half_rn(silu_f(val[jj]) * ub[jj * 64 + rloc]);
                fence_proxy_async();
              } else if (row_ok) {
#pragma unroll
                for (int jj = 0; jj < CH; ++jj) {
                  if (jj >= jn) break;
                  reinterpret_cast<__half*>(p.y)[(int64_t)(t0 + j0 + jj) * p.ldy + row] =
                      __float2half_rn(silu_f(val[jj]) * ub[jj * 64 + rloc]);
                }
              }
            }
            named_bar(1, 128);  // the exchange buffer takes the next CH tokens; the staging tile is complete
            if (p.tma_store) {
              if (leader) {
                tma_store_2d(&tmap_y, sb, row0, t0 + j0);
                bulk_commit();
              }
              ++nbuf;
            }
            continue;
          }
          if (EPI != kEpiStore && atma) {
            const uint32_t sl = aux_used % AD;
            if (!mbar_wait(&auxfull[sl], (aux_used / AD) & 1, p.status, kStatusTimeoutFull)) { ok = false; break; }
            const float* ab = reinterpret_cast<const float*>(abuf + sl * AC::kSlot);
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) {
              const float ax = ab[jj * kBM + rloc];
              val[jj] = EPI == kEpiResid ? ax + val[jj] : silu_f(ax) * val[jj];
            }
            ++aux_used;
            named_bar(1, 128);  // every thread has read this slot: refill it with the chunk AD ahead
            const int k = j0 / CH + AD;
            if (leader && k < ncks) {
              mbar_arrive_expect_tx(&auxfull[sl], AC::kSlot);
              tma_load_2d(abuf + sl * AC::kSlot, &tmap_aux, &auxfull[sl], row0, t0 + k * CH);
            }
          } else if (EPI != kEpiStore && row_ok) {
            float ax[CH];
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) ax[jj] = jj < jn ? __ldg(p.aux + (int64_t)(t0 + j0 + jj) * p.ldaux + row) : 0.f;
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) val[jj] = EPI == kEpiResid ? ax[jj] + val[jj] : silu_f(ax[jj]) * val[jj];
          }
          if (p.tma_store) {
            uint8_t* buf = obuf + (nbuf & 1) * S::kOutBuf;
            if (leader) bulk_wait_read<1>();  // the store that last used this buffer has read it
            named_bar(1, 128);
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) {
              if (OUT_F16)
                reinterpret_cast<__half*>(buf)[jj * kBM + rloc] = __float2half_rn(val[jj]);
              else
                reinterpret_cast<float*>(buf)[jj * kBM + rloc] = val[jj];
            }
            fence_proxy_async();
            named_bar(1, 128);
            if (leader) {
              tma_store_2d(&tmap_y, buf, row0, t0 + j0);
              bulk_commit();
            }
            ++nbuf;
          } else if (row_ok) {
#pragma unroll
            for (int jj = 0; jj < CH; ++jj) {
              if (jj >= jn) break;
              const int64_t t = tsplit + t0 + j0 + jj;
              void* yb = p.y;
              int64_t tt = t;
              if (p.nsl > 0) yb = p.ysl[t / p.slice_rows], tt = t % p.slice_rows;
              if (OUT_F16)
                reinterpret_cast<__half*>(yb)[tt * p.ldy + row] = __float2half_rn(val[jj]);
              else
                reinterpret_cast<float*>(yb)[tt * p.ldy + row] = val[jj];
            }
          }
          (void)ES;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR) mbar_arrive_cluster(accempty_lead + r * 8);
          else mbar_arrive(&accempty[r]);
        }
      }
    }
    if (leader) bulk_wait_all();  // stores complete before the CTA (and its shared memory) goes away
    // token slices may be other GPUs' memory: each storing thread's last stores are visible system-wide before the
    // kernel ends (the launch that signals their completion follows in stream order); once per thread, at the end
    if (p.nsl > 0) __threadfence_system();
  }

  tc_fence_before();
  if (PAIR) cluster_sync(); else __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem, 512); else tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Dynamic shared memory is at least this much, so that one CTA (which owns all 512 TMEM columns) fills an SM.
constexpr int kMinSmem = 120 * 1024;

template <int T, int BN, int NACC, int EPI, bool OUT_F16, bool PAIR, bool SPLIT = false>
cudaError_t launch_t(const QGemmArgs& a, cudaStream_t stream) {
  constexpr int XROWS = PAIR ? BN / 2 : BN;
  using AC = AuxCfg<T, XROWS, EPI, OUT_F16>;
  using S = Smem<T, XROWS, AC::kBytes>;
  EncodeTiledFn enc = encoder();
  if (!enc) return cudaErrorNotSupported;
  constexpr int kTileRows = EPI == kEpiFfn ? 64 : kBM;  // weight rows per CTA tile (per box, per tensor)
  CUtensorMap mw, mx, mw2;
  for (int k = 0; k < (EPI == kEpiFfn ? 2 : 1); ++k) {  // kEpiFfn: the gate and the up weights, 64-row boxes
    const int64_t window_bytes = (a.kb_off + a.K / 256) * Fmt<T>::kSB;
    cuuint64_t dims[2] = {(cuuint64_t)((window_bytes + 1) / 2), (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)a.w_row_stride};
    cuuint32_t box[2] = {(cuuint32_t)(Fmt<T>::kBox / 2), (cuuint32_t)kTileRows};
    cuuint32_t es[2] = {1, 1};
    if (enc(k ? &mw2 : &mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(k ? a.w2 : a.w), dims, strides,
            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)a.ldx * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)XROWS};  // one 64-K tile of this CTA's tokens; a stage loads two
    cuuint32_t es[2] = {1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  CUtensorMap my;
  const int esz = a.y_f16 ? 2 : 4;
  // (split K writes the workspace with plain stores: its rows kp * M + t are not the output tensor's rows)
  // a single accumulator region with a plain store and one accumulation chunk per unit is drained by 20 warps with
  // direct stores (drain_share)
  const bool help = NACC == 1 && EPI == kEpiStore && (SPLIT || a.kchunk <= 0 || a.kchunk >= a.K);
  const bool tma_store = !help && !SPLIT && a.nsl == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 &&
                         (a.ldy * esz) % 16 == 0;
  if (tma_store) {
    cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)(a.ldy * esz)};
    cuuint32_t box[2] = {(cuuint32_t)kTileRows, (cuuint32_t)epi_chunk(EPI, OUT_F16)};
    cuuint32_t es[2] = {1, 1};
    if (enc(&my, a.y_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.y, dims, strides,
            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else {
    my = mx;  // unused
  }
  CUtensorMap maux = EPI == kEpiFfn ? mw2 : mx;  // the up weights (kEpiFfn), or the aux prefetch, else unused
  const bool aux_tma = AC::kDepth > 0 && a.aux && (reinterpret_cast<uintptr_t>(a.aux) & 15) == 0 && a.ldaux % 4 == 0;
  if (aux_tma) {
    cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)(a.ldaux * 4)};
    cuuint32_t box[2] = {(cuuint32_t)kBM, (cuuint32_t)AC::kCH};
    cuuint32_t es[2] = {1, 1};
    if (enc(&maux, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.aux), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  KParams p;
  p.tma_store = tma_store ? 1 : 0;
  p.aux_tma = aux_tma ? 1 : 0;
  p.help = help ? 1 : 0;
  p.nsl = SPLIT ? 0 : a.nsl;
  p.slice_rows = a.slice_rows;
  for (int i = 0; i < kMaxSlices; ++i) p.ysl[i] = a.ysl[i];
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.M = (int)a.M;
  p.kb_off = (int)a.kb_off;
  p.kcb = (a.kchunk > 0 && a.kchunk < a.K) ? (int)(a.kchunk / 64) : (int)(a.K / 64);  // even: whole stages
  p.scratch = a.scratch;
  p.y = a.y;
  p.ldy = a.ldy;
  p.aux = a.aux;
  p.ldaux = a.ldaux;
  p.status = a.status;
  p.upr = (int)((a.M + 15) / 16);
  p.ncta = PAIR ? 2 : 1;
  p.nsplit = SPLIT ? a.nsplit : 1;
  const int64_t rtiles = (a.N + kTileRows * p.ncta - 1) / (kTileRows * p.ncta);
  p.total_units = rtiles * p.nsplit * p.upr;
  const int grid = qgemm_grid(a);
  // whole tiles when that gives the busiest CTA (pair) fewer K loops than the equal unit ranges
  p.tpr = (int)((a.M + BN - 1) / BN);
  p.total_tiles = rtiles * p.nsplit * p.tpr;
  {
    const int64_t G = grid / p.ncta, upt = BN / 16;
    int64_t max_units = 0;
    for (int64_t b = 0; b < G; ++b) {  // K loops of CTA b under the unit ranges (Sched::next without whole)
      int64_t u = b * p.total_units / G, end = (b + 1) * p.total_units / G, loops = 0;
      while (u < end) {
        const int64_t tu = u % p.upr;
        int64_t nu = upt < p.upr - tu ? upt : p.upr - tu;
        if (nu > end - u) nu = end - u;
        u += nu;
        ++loops;
      }
      if (loops > max_units) max_units = loops;
    }
    const int64_t max_whole = (p.total_tiles + G - 1) / G;
    p.whole = max_whole < max_units ? 1 : 0;
  }
  auto kern = qgemm_tc_kernel<T, BN, NACC, EPI, OUT_F16, PAIR, SPLIT>;
  const int smem_bytes = S::kAlloc > kMinSmem ? S::kAlloc : kMinSmem;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  if (!PAIR) {
    kern<<<grid, kThreads, smem_bytes, stream>>>(mw, mx, my, maux, p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mw, mx, my, maux, p);
}

template <int T, int BN, int NACC, bool PAIR>
cudaError_t launch_epi(const QGemmArgs& a, cudaStream_t s) {
  if (a.epilogue == kEpiFfn) return a.w2 ? launch_t<T, BN, NACC, kEpiFfn, true, PAIR>(a, s) : cudaErrorInvalidValue;
  if (a.epilogue == kEpiResid) return launch_t<T, BN, NACC, kEpiResid, false, PAIR>(a, s);
  if (a.epilogue == kEpiSwiglu) return launch_t<T, BN, NACC, kEpiSwiglu, true, PAIR>(a, s);
  return a.y_f16 ? launch_t<T, BN, NACC, kEpiStore, true, PAIR>(a, s)
                 : launch_t<T, BN, NACC, kEpiStore, false, PAIR>(a, s);
}

// Split K: out[t][r] = epilogue(sum of the nsplit chunk results part[c][t][r], added in chunk order); the additions,
// and the epilogue's arithmetic, are those of the single-CTA chunked epilogue above.
template <int EPI, bool OUT_F16>
__global__ void split_reduce_kernel(const float* __restrict__ part, int nsplit, int M, int N, void* y, int64_t ldy,
                                    const float* __restrict__ aux, int64_t ldaux) {
  const int64_t total = (int64_t)M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / N, r = i - t * N;
    float acc = __ldcs(part + i);
    for (int c = 1; c < nsplit; ++c) acc = acc + __ldcs(part + (int64_t)c * total + i);
    if (EPI == kEpiResid) acc = aux[t * ldaux + r] + acc;
    if (EPI == kEpiSwiglu) acc = silu_f(aux[t * ldaux + r]) * acc;
    if (OUT_F16) reinterpret_cast<__half*>(y)[t * ldy + r] = __float2half_rn(acc);
    else reinterpret_cast<float*>(y)[t * ldy + r] = acc;
  }
}

template <int EPI, bool OUT_F16>
cudaError_t launch_split_reduce(const QGemmArgs& a, cudaStream_t stream) {
  const int64_t total = a.M * a.N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 8LL * a.num_sms) blocks = 8LL * a.num_sms;
  split_reduce_kernel<EPI, OUT_F16><<<(int)blocks, 256, 0, stream>>>(a.kpart, a.nsplit, (int)a.M, (int)a.N, a.y,
                                                                     a.ldy, a.aux, a.ldaux);
  return cudaGetLastError();
}

// Split K: the tile kernel (plain f32 stores into the workspace) and then the ordered reduction with the epilogue.
template <int T>
cudaError_t launch_split(const QGemmArgs& a, cudaStream_t s);

// Instantiated tiles: pairs at BN 256 (one accumulator region, 4 A stages), 160 and 128 (two regions); single
// CTAs at BN 192, 128 and 64 (two regions). The C ABI only passes these combinations.
template <int T>
cudaError_t launch_fmt(const QGemmArgs& a, cudaStream_t s) {
  if (a.pair) {
    if (a.bn == 256) return launch_epi<T, 256, 1, true>(a, s);
    if (a.bn == 160) return launch_epi<T, 160, 2, true>(a, s);
    if (a.bn == 128) return launch_epi<T, 128, 2, true>(a, s);
    return cudaErrorInvalidValue;
  }
  if (a.bn == 192) return launch_epi<T, 192, 2, false>(a, s);
  if (a.bn == 128) return launch_epi<T, 128, 2, false>(a, s);
  if (a.bn == 64) return launch_epi<T, 64, 2, false>(a, s);
  return cudaErrorInvalidValue;
}

template <int T>
cudaError_t launch_split(const QGemmArgs& a, cudaStream_t s) {
  QGemmArgs b = a;  // the tile kernel writes the chunk results: f32, plain store, [nsplit * M][N]
  b.y = a.kpart;
  b.y_f16 = 0;
  b.ldy = a.N;
  b.epilogue = kEpiStore;
  b.aux = nullptr;
  b.ldaux = 0;
  cudaError_t e = cudaErrorInvalidValue;
  if (b.pair) {
    if (b.bn == 256) e = launch_t<T, 256, 1, kEpiStore, false, true, true>(b, s);
    if (b.bn == 160) e = launch_t<T, 160, 2, kEpiStore, false, true, true>(b, s);
    if (b.bn == 128) e = launch_t<T, 128, 2, kEpiStore, false, true, true>(b, s);
  } else {
    if (b.bn == 192) e = launch_t<T, 192, 2, kEpiStore, false, false, true>(b, s);
    if (b.bn == 128) e = launch_t<T, 128, 2, kEpiStore, false, false, true>(b, s);
    if (b.bn == 64) e = launch_t<T, 64, 2, kEpiStore, false, false, true>(b, s);
  }
  if (e != cudaSuccess) return e;
  if (a.epilogue == kEpiResid) return launch_split_reduce<kEpiResid, false>(a, s);
  if (a.epilogue == kEpiSwiglu) return launch_split_reduce<kEpiSwiglu, true>(a, s);
  return a.y_f16 ? launch_split_reduce<kEpiStore, true>(a, s) : launch_split_reduce<kEpiStore, false>(a, s);
}

}  // namespace

bool tensor_map_encoder_available() { return encoder() != nullptr; }

int qgemm_grid(const QGemmArgs& a) {
  const int ncta = a.pair ? 2 : 1;
  const int rows = (a.epilogue == kEpiFfn ? 64 : kBM) * ncta;  // output rows per tile
  const int64_t units = (a.N + rows - 1) / rows * ((a.M + 15) / 16) * (a.nsplit > 1 ? a.nsplit : 1);
  int64_t grid = a.grid > 0 ? a.grid : a.num_sms;
  if (a.pair) {
    grid = grid / 2 < a.max_pairs ? grid / 2 : a.max_pairs;  // pairs that can be resident at once
    if (grid > units) grid = units;
    if (grid < 1) grid = 1;
    return (int)(2 * grid);
  }
  if (grid > units) grid = units;
  return (int)grid;
}

int qgemm_max_pairs(int type, int bn) {
  // Clusters of 2 that the device can hold at once with this kernel's resources (one CTA per SM).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kMinSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const void* k = (const void*)qgemm_tc_kernel<12, 256, 1, kEpiStore, true, true, false>;
  (void)type;
  (void)bn;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMinSmem) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) return 0;
  return n;
}

cudaError_t launch_qgemm_tc(const QGemmArgs& a, cudaStream_t stream) {
  if (a.nsplit > 1 && a.epilogue == kEpiFfn) return cudaErrorInvalidValue;  // the fused gate+up does not split
  // token slices: plain stores of unsplit tiles, whole 16-token units per slice
  if (a.nsl > 0 && (a.nsplit > 1 || a.epilogue != kEpiStore || a.nsl > kMaxSlices || a.slice_rows <= 0 ||
                    a.slice_rows % 16 || a.slice_rows * a.nsl < a.M))
    return cudaErrorInvalidValue;
  if (a.nsplit > 1) {
    if (!a.kpart) return cudaErrorInvalidValue;
    switch (a.type) {
      case 8: return launch_split<8>(a, stream);
      case 12: return launch_split<12>(a, stream);
      case 14: return launch_split<14>(a, stream);
      case 11: return launch_split<11>(a, stream);
      case 13: return launch_split<13>(a, stream);
      case 23: return launch_split<23>(a, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (a.type) {
    case 8: return launch_fmt<8>(a, stream);
    case 12: return launch_fmt<12>(a, stream);
    case 14: return launch_fmt<14>(a, stream);
    case 11: return launch_fmt<11>(a, stream);
    case 13: return launch_fmt<13>(a, stream);
    case 23: return launch_fmt<23>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace yah
