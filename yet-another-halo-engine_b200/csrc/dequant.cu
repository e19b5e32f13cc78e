// Standalone dequant: GGUF rows -> f16 [rows][ldo], with exactly the decode the tile GEMM uses.
// Reference: the "dequant" kind of engine/gpu/loom/tools/gen_gemm_tile.py:314-327, :627-802 (W -> f16 [rows][K]
// with the GEMM's own decode), checked bit for bit as engine/gpu/loom/tools/dq_bfp16_check.py:87-92 does.
// One thread decodes one 64-value K block of one row (reads 2-byte aligned words from global memory, writes
// 128 contiguous bytes); consecutive threads walk a row's K blocks, so loads and stores are coalesced.
#include <cuda_runtime.h>

#include "decode.cuh"
#include "kernels.h"

namespace yah {
namespace {

template <int T>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w, int64_t rows, int64_t nsb,
                                                      int64_t row_stride, int64_t kb_off, uint16_t* __restrict__ out,
                                                      int64_t ldo) {
  constexpr int SB = superblock_bytes(T);
  const int64_t total = rows * nsb * 4;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / (nsb * 4);
    const int64_t rem = idx - r * nsb * 4;
    const int64_t sb = rem >> 2;
    const int j = (int)(rem & 3);
    const uint8_t* p = w + r * row_stride + (kb_off + sb) * SB;
    uint32_t v[32];
    decode_global<T>(p, j, v);
    uint4* dst = reinterpret_cast<uint4*>(out + r * ldo + sb * 256 + j * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

}  // namespace

cudaError_t launch_dequant(const void* w, int type, int64_t rows, int64_t K, int64_t row_stride, int64_t kb_off,
                           uint16_t* out, int64_t ldo, int num_sms, cudaStream_t stream) {
  const int64_t nsb = K / 256;
  const int64_t work = rows * nsb * 4;
  if (work == 0) return cudaSuccess;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  switch (type) {
    case 8: dequant_kernel<8><<<(int)blocks, 256, 0, stream>>>(wb, rows, nsb, row_stride, kb_off, out, ldo); break;
    case 12: dequant_kernel<12><<<(int)blocks, 256, 0, stream>>>(wb, rows, nsb, row_stride, kb_off, out, ldo); break;
    case 14: dequant_kernel<14><<<(int)blocks, 256, 0, stream>>>(wb, rows, nsb, row_stride, kb_off, out, ldo); break;
    case 11: dequant_kernel<11><<<(int)blocks, 256, 0, stream>>>(wb, rows, nsb, row_stride, kb_off, out, ldo); break;
    case 13: dequant_kernel<13><<<(int)blocks, 256, 0, stream>>>(wb, rows, nsb, row_stride, kb_off, out, ldo); break;
    case 23: dequant_kernel<23><<<(int)blocks, 256, 0, stream>>>(wb, rows, nsb, row_stride, kb_off, out, ldo); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace yah
