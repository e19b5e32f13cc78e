// Decode GEMV for M <= 32 tokens: y[t][n] (+)= sum_k W[n][k] x[t][k], GGUF weights, f16 activations.
//
// Reference: engine/gpu/loom/tools/gen_gemv.py (kinds plain / resid :96-754, the per-row decode :365-526, the
// butterfly reduction :679-690) and its call site engine/model/loom_decoder.hpp:415-439. The reference GEMV is
// judged purely on bandwidth; so is this one. Its weights are the f16 values of the tile GEMM's decode (the
// reference dequant, bit-exact), so decode and prefill compute the same products.
//
// B200 design. A CTA owns 128 weight rows and a contiguous range of K super-blocks (split-K over CTAs when there
// are fewer row blocks than SMs). Warp 16 streams the range with TMA: per stage one 256-K super-block of the 128
// rows plus the matching 4 x 64-K activation tiles (tokens x 128 B, 128-byte swizzle), 4 stages in flight.
// Warps 0-15 each own 8 rows: lane t decodes 16 values of row t/4 (quarter t%4 of every 64-K block) into f16 pairs,
// which are exactly the B fragment of mma.sync.m16n8k16 (tokens = M side, rows = N side) under a K permutation
// that the activation fragments follow. Split-K partials go to a workspace; the last CTA of a row block to finish
// (atomic counter) sums them in split order, so results are deterministic.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "decode.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace yah {
namespace {

constexpr int kGvWarps = 16;
constexpr int kGvThreads = (kGvWarps + 1) * 32;
constexpr int kGvRows = 128;
constexpr int kGvStages = 4;

template <int T>
struct GvFmt;
template <>
struct GvFmt<8> { static constexpr int kSB = 272, kBox = 272; };
template <>
struct GvFmt<12> { static constexpr int kSB = 144, kBox = 144; };
template <>
struct GvFmt<14> { static constexpr int kSB = 210, kBox = 224; };

template <int T, int MT>
struct GvSmem {
  static constexpr int kTP = 16 * MT;                  // token rows per activation tile
  static constexpr int kXTile = kTP * 128;             // one 64-K activation tile
  static constexpr int kW = ((kGvRows * GvFmt<T>::kBox + 16) + 1023) / 1024 * 1024;
  static constexpr int kStage = kW + 4 * kXTile;
  static constexpr int kBarOff = kGvStages * kStage;
  static constexpr int kBytes = kBarOff + 2 * kGvStages * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
};

struct GvParams {
  int N, K, M, kb_off, nsb, S;
  void* y;
  int64_t ldy;
  int y_f16, epi;
  const float* aux;
  int64_t ldaux;
  float* ws;      // [S][M][N] split-K partials (S > 1)
  int* counters;  // one per row block, zero between launches
  int* status;
};

// 4 words at an even byte offset `off` of a shared-memory row (reads 5 aligned words).
__device__ __forceinline__ void lds_words4(uint32_t rb, int off, uint32_t (&w)[4]) {
  const uint32_t a = rb + (off & ~3);
  const uint32_t sel = (off & 2) ? 0x5432u : 0x3210u;
  uint32_t L[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) L[i] = lds32(a + 4 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = prmt(L[i], L[i + 1], sel);
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t rb, int off) {
  return (lds32(rb + (off & ~3)) >> (8 * (off & 3))) & 0xFFFFu;
}

// Decode 16 values (quarter c of 64-K block j) of a staged row into 8 f16 pairs: out[i] = values (2i, 2i + 1)
// of the quarter. Same arithmetic as decode.cuh's 64-value decoders.
template <int T>
__device__ __forceinline__ void decode16(uint32_t rb, int j, int c, int o, uint32_t (&out)[8]);

template <>
__device__ __forceinline__ void decode16<12>(uint32_t rb, int j, int c, int, uint32_t (&out)[8]) {
  const uint4 hdr = lds128(rb);
  const uint4 q = lds128(rb + 16 + 32 * j + 16 * (c & 1));
  const int hi = c >> 1;  // quarters 2, 3: group 2j + 1, high nibbles
  float dsa, dma, dsb, dmb;
  q4k_scales(hdr, j, dsa, dma, dsb, dmb);
  const float ds = hi ? dsb : dsa;
  const float nd = hi ? -dmb : -dma;
  const int sh = 4 * hi;
  const float s0 = hi ? ds * 0.0625f : ds;                      // nibble at bit sh
  const float s8 = hi ? ds * 2.44140625e-4f : ds * 0.00390625f;  // nibble at bit 8 + sh
  const uint32_t m0 = 0xFu << sh, m8 = 0xF00u << sh;
  const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = qw[i], v = w >> 16;
    out[2 * i] = pack_f16x2_rn(__fmaf_rn(s0, magic_q(w & m0), nd), __fmaf_rn(s8, magic_q(w & m8), nd));
    out[2 * i + 1] = pack_f16x2_rn(__fmaf_rn(s0, magic_q(v & m0), nd), __fmaf_rn(s8, magic_q(v & m8), nd));
  }
}

template <>
__device__ __forceinline__ void decode16<8>(uint32_t rb, int j, int c, int, uint32_t (&out)[8]) {
  const int b = 2 * j + (c >> 1);
  uint32_t W[4];
  lds_words4(rb, 34 * b + 2 + 16 * (c & 1), W);
  const uint32_t d = lds_u16(rb, 34 * b);
  const uint32_t d2 = d | (d << 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t x = W[i] ^ 0x80808080u;
    out[2 * i] = hmul2_u32(hsub2_u32(prmt(x, 0x64646464u, 0x4140u), 0x64806480u), d2);
    out[2 * i + 1] = hmul2_u32(hsub2_u32(prmt(x, 0x64646464u, 0x4342u), 0x64806480u), d2);
  }
}

template <>
__device__ __forceinline__ void decode16<14>(uint32_t rb, int j, int c, int o, uint32_t (&out)[8]) {
  const int h = j >> 1, jodd = j & 1;
  uint32_t QL[4], QH[4];
  lds_words4(rb, o + 64 * h + 16 * c, QL);
  lds_words4(rb, o + 128 + 32 * h + 16 * (c & 1), QH);
  const int sy = o + 192 + 8 * h + 4 * jodd + c;
  const int s = (int)(int8_t)((lds32(rb + (sy & ~3)) >> (8 * (sy & 3))) & 0xFFu);
  const float d = h2f_bits(lds_u16(rb, o + 208));
  const float ds = (d * (float)s) * 1.52587890625e-05f;
  const int lsh = 4 * jodd, hsh = 4 * jodd + 2 * (c >> 1);
  constexpr float kOff = 10485760.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t code = ((QL[i] >> lsh) & 0x0F0F0F0Fu) | (((QH[i] >> hsh) & 0x03030303u) << 4);
    const float v0 = __fmul_rn(ds, __uint_as_float(prmt(code, 0x4B000000u, 0x7044u)) - kOff);
    const float v1 = __fmul_rn(ds, __uint_as_float(prmt(code, 0x4B000000u, 0x7144u)) - kOff);
    const float v2 = __fmul_rn(ds, __uint_as_float(prmt(code, 0x4B000000u, 0x7244u)) - kOff);
    const float v3 = __fmul_rn(ds, __uint_as_float(prmt(code, 0x4B000000u, 0x7344u)) - kOff);
    out[2 * i] = pack_f16x2_rn(v0, v1);
    out[2 * i + 1] = pack_f16x2_rn(v2, v3);
  }
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

template <int T, int MT>
__global__ void __launch_bounds__(kGvThreads, 1)
    qgemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 const GvParams p) {
  using S = GvSmem<T, MT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + kGvStages;
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x / p.S, split = blockIdx.x % p.S;
  const int sb0 = (int)((int64_t)split * p.nsb / p.S), sb1 = (int)((int64_t)(split + 1) * p.nsb / p.S);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGvStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGvWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  float acc[MT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;

  if (warp == kGvWarps) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_x);
      int i = 0;
      for (int sb = sb0; sb < sb1; ++sb, ++i) {
        const int st = i % kGvStages, ph = (i / kGvStages) & 1;
        if (!mbar_wait(&empty[st], ph ^ 1, p.status, kStatusTimeoutEmpty)) break;
        uint8_t* base = smem + st * S::kStage;
        mbar_arrive_expect_tx(&full[st], kGvRows * GvFmt<T>::kBox + 4 * S::kXTile);
        const int64_t sbg = (int64_t)p.kb_off + sb;
        const int xw = (T == 14) ? (int)(((sbg * 210) & ~int64_t(15)) >> 1) : (int)(sbg * (GvFmt<T>::kSB / 2));
        tma_load_2d(base, &tmap_w, &full[st], xw, rb * kGvRows);
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_load_2d(base + S::kW + j * S::kXTile, &tmap_x, &full[st], sb * 256 + 64 * j, 0);
      }
      // drain the last copies
      const int n = sb1 - sb0;
      for (int k = (n > kGvStages ? n - kGvStages : 0); k < i; ++k)
        mbar_wait(&full[k % kGvStages], (k / kGvStages) & 1, p.status, kStatusTimeoutDrain, false);
    }
  } else {
    const int g = lane >> 2, c = lane & 3;
    const int row_local = warp * 8 + g;
    int i = 0;
    for (int sb = sb0; sb < sb1; ++sb, ++i) {
      const int st = i % kGvStages, ph = (i / kGvStages) & 1;
      if (!mbar_wait(&full[st], ph, p.status, kStatusTimeoutFull)) break;
      const uint32_t base = smem_u32(smem + st * S::kStage);
      const uint32_t rbase = base + row_local * GvFmt<T>::kBox;
      const int o = (T == 14) ? (int)((((int64_t)p.kb_off + sb) * 210) & 15) : 0;
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        uint32_t b[8];
        decode16<T>(rbase, j, c, o, b);
        const uint32_t xb = base + S::kW + j * S::kXTile;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int t0 = 16 * m + g, t1 = t0 + 8;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const int ch = 2 * c + (s >> 1), lo8 = 8 * (s & 1);
            const uint2 x0 = lds64(xb + t0 * 128 + ((ch ^ (t0 & 7)) << 4) + lo8);
            const uint2 x1 = lds64(xb + t1 * 128 + ((ch ^ (t1 & 7)) << 4) + lo8);
            mma16816(acc[m], x0.x, x1.x, x0.y, x1.y, b[2 * s], b[2 * s + 1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }

  // ---------------------------------------------------------------- results
  const bool compute = warp < kGvWarps;
  const int g = lane >> 2, c = lane & 3;
  const int row0 = rb * kGvRows + warp * 8 + 2 * c;
  if (p.S == 1) {
    if (compute) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * m + g + 8 * (e >> 1), n = row0 + (e & 1);
          if (t < p.M && n < p.N) {
            float v = acc[m][e];
            if (p.epi == kEpiResid) v += p.aux[(int64_t)t * p.ldaux + n];
            if (p.y_f16) reinterpret_cast<__half*>(p.y)[(int64_t)t * p.ldy + n] = __float2half_rn(v);
            else reinterpret_cast<float*>(p.y)[(int64_t)t * p.ldy + n] = v;
          }
        }
    }
    return;
  }
  if (compute) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = 16 * m + g + 8 * (e >> 1), n = row0 + (e & 1);
        if (t < p.M && n < p.N) p.ws[((int64_t)split * p.M + t) * p.N + n] = acc[m][e];
      }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&p.counters[rb], 1) == p.S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int rows = min(kGvRows, p.N - rb * kGvRows);
  for (int idx = threadIdx.x; idx < p.M * kGvRows; idx += blockDim.x) {
    const int t = idx / kGvRows, r = idx % kGvRows;
    if (r >= rows) continue;
    const int n = rb * kGvRows + r;
    float v = 0.f;
    for (int s = 0; s < p.S; ++s) v += __ldcg(p.ws + ((int64_t)s * p.M + t) * p.N + n);
    if (p.epi == kEpiResid) v += p.aux[(int64_t)t * p.ldaux + n];
    if (p.y_f16) reinterpret_cast<__half*>(p.y)[(int64_t)t * p.ldy + n] = __float2half_rn(v);
    else reinterpret_cast<float*>(p.y)[(int64_t)t * p.ldy + n] = v;
  }
  if (threadIdx.x == 0) p.counters[rb] = 0;
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

template <int T, int MT>
cudaError_t gv_launch(const QGemvArgs& a, float* ws, int* counters, int S, cudaStream_t stream) {
  using SM = GvSmem<T, MT>;
  EncodeTiledFn enc = gv_encoder();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw, mx;
  {
    const int64_t window_bytes = (a.kb_off + a.K / 256) * GvFmt<T>::kSB;
    cuuint64_t dims[2] = {(cuuint64_t)((window_bytes + 1) / 2), (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)a.w_row_stride};
    cuuint32_t box[2] = {(cuuint32_t)(GvFmt<T>::kBox / 2), (cuuint32_t)kGvRows};
    cuuint32_t es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(a.w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)a.ldx * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)SM::kTP};
    cuuint32_t es[2] = {1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  GvParams p;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.M = (int)a.M;
  p.kb_off = (int)a.kb_off;
  p.nsb = (int)(a.K / 256);
  p.S = S;
  p.y = a.y;
  p.ldy = a.ldy;
  p.y_f16 = a.y_f16;
  p.epi = a.epilogue;
  p.aux = a.aux;
  p.ldaux = a.ldaux;
  p.ws = ws;
  p.counters = counters;
  p.status = a.status;
  const int rblocks = (int)((a.N + kGvRows - 1) / kGvRows);
  auto kern = qgemv_kernel<T, MT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kAlloc);
  if (e != cudaSuccess) return e;
  kern<<<rblocks * S, kGvThreads, SM::kAlloc, stream>>>(mw, mx, p);
  return cudaGetLastError();
}

template <int T>
cudaError_t gv_fmt(const QGemvArgs& a, float* ws, int* counters, int S, cudaStream_t s) {
  return a.M <= 16 ? gv_launch<T, 1>(a, ws, counters, S, s) : gv_launch<T, 2>(a, ws, counters, S, s);
}

}  // namespace

// Split-K factor and workspace need of a GEMV launch (host helpers for the C ABI).
int qgemv_splits(int64_t N, int64_t K, int num_sms) {
  const int64_t rblocks = (N + kGvRows - 1) / kGvRows;
  int64_t S = num_sms / rblocks;
  if (S < 1) S = 1;
  if (S > K / 256) S = K / 256;
  return (int)S;
}

cudaError_t launch_qgemv_ws(const QGemvArgs& a, float* ws, int* counters, int S, cudaStream_t stream) {
  switch (a.type) {
    case 8: return gv_fmt<8>(a, ws, counters, S, stream);
    case 12: return gv_fmt<12>(a, ws, counters, S, stream);
    case 14: return gv_fmt<14>(a, ws, counters, S, stream);
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
constexpr size_t kStaticCounters = 4096;                   // one per 128-row block: N <= 524288
constexpr size_t kStaticPartials = (size_t)1 << 20;        // split-K partial sums: S * M * N <= 1M floats
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

cudaError_t launch_qgemv_static(const QGemvArgs& a_in, void* base, int S, cudaStream_t stream) {
  QGemvArgs a = a_in;
  unsigned char* b = static_cast<unsigned char*>(base);
  int* status = reinterpret_cast<int*>(b);
  int* counters = reinterpret_cast<int*>(b + kStaticStatusBytes);
  float* partials = reinterpret_cast<float*>(b + kStaticStatusBytes + kStaticCounters * sizeof(int));
  a.status = status;
  if (S > 1) {
    // The counters must start at zero; a previous call leaves them at zero unless it was interrupted.
    const size_t nrb = (size_t)((a.N + 127) / 128);
    const cudaError_t e = cudaMemsetAsync(counters, 0, nrb * sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  return launch_qgemv_ws(a, partials, counters, S, stream);
}

cudaError_t qgemv_static_status(void* base, int* code, bool clear) {
  cudaError_t e = cudaMemcpy(code, base, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && *code) e = cudaMemset(base, 0, sizeof(int));
  return e;
}

}  // namespace yah
