// Tensor-parallel quantised linears over NCCL, and the residual-stream RMSNorm of the layer stack.
//
// The reference engine runs on one GPU and has no sharding layer; this is the one the B200 build adds. A stack
// of Llama-shaped layers is split over the GPUs of one box the Megatron way:
//   column-parallel (QKV, gate, up): each rank holds a row range of the GGUF tensor (no re-quantisation) and
//     computes its slice of the outputs; no collective.
//   row-parallel (o_proj, down): each rank holds a K window of all rows (whole super-blocks) and computes a
//     partial sum of every output; one ncclAllReduce(sum) of the f32 partials makes the result. Rank 0 adds the
//     residual in its GEMM epilogue, the other ranks store plain partials, so the allreduce yields
//     residual + W x on every rank.
// NCCL is loaded at run time (dlopen of libnccl.so.2): a process that already holds an NCCL (for example through
// a framework) shares it, and the library itself loads on hosts without NCCL.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "../../include/yah_qgemm.h"
#include "kernels.h"

namespace yah {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*get_error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi* nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.get_error_string = reinterpret_cast<decltype(api.get_error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.get_error_string;
  });
  return &api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  return set_error(YAH_ERR_NCCL, "%s: %s", what, nccl()->get_error_string ? nccl()->get_error_string(r) : "?");
}

// One row per CTA: out = f16(h * gain / sqrt(mean(h^2) + eps)). ADD: first h += d (the allreduced partial sums,
// f16 in the speed mode or f32 in the parity mode), stored back to h in f32; NORM false: the add alone (the last
// layer's update).
constexpr int kNormThreads = 256;

template <bool ADD, bool NORM, bool DF16>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(float* __restrict__ h, int64_t ldh, int H,
                                                               const void* __restrict__ d, int64_t ldd, float eps,
                                                               float gain, __half* __restrict__ out, int64_t ldo) {
  float* row = h + (int64_t)blockIdx.x * ldh;
  float ss = 0.f;
  for (int i = 4 * threadIdx.x; i < H; i += 4 * kNormThreads) {
    float4 v = *reinterpret_cast<const float4*>(row + i);
    if (ADD) {
      float4 a;
      if (DF16) {
        const uint2 dd = *reinterpret_cast<const uint2*>(static_cast<const __half*>(d) + (int64_t)blockIdx.x * ldd + i);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&dd.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&dd.y));
        a = make_float4(lo.x, lo.y, hi.x, hi.y);
      } else {
        a = *reinterpret_cast<const float4*>(static_cast<const float*>(d) + (int64_t)blockIdx.x * ldd + i);
      }
      v.x += a.x, v.y += a.y, v.z += a.z, v.w += a.w;
      *reinterpret_cast<float4*>(row + i) = v;  // re-read below by this same thread
    }
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
  if (!NORM) return;
  __shared__ float part[kNormThreads / 32];
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? part[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) part[0] = t;
  }
  __syncthreads();
  const float scale = gain * rsqrtf(part[0] / (float)H + eps);
  __half* orow = out + (int64_t)blockIdx.x * ldo;
  for (int i = 4 * threadIdx.x; i < H; i += 4 * kNormThreads) {
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    const __half2 a = __floats2half2_rn(v.x * scale, v.y * scale), b = __floats2half2_rn(v.z * scale, v.w * scale);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&a);
    packed.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(orow + i) = packed;
  }
}

}  // namespace
}  // namespace yah

struct yah_tp_comm {
  ncclComm_t nc;
  int rank, nranks, device;
};

extern "C" {

int yah_tp_available(void) { return yah::nccl()->ok ? 1 : 0; }

int yah_tp_unique_id(void* id) {
  if (!id) return yah::set_error(YAH_ERR_ARG, "null id");
  if (!yah::nccl()->ok) return yah::set_error(YAH_ERR_NCCL, "NCCL (libnccl.so.2) could not be loaded");
  ncclUniqueId u;
  const ncclResult_t r = yah::nccl()->get_unique_id(&u);
  if (r != ncclSuccess) return yah::nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof(u));
  return YAH_OK;
}

int yah_tp_init(yah_tp_comm** comm, int nranks, int rank, const void* id) {
  if (!comm || !id) return yah::set_error(YAH_ERR_ARG, "null comm or id");
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return yah::set_error(YAH_ERR_ARG, "rank %d of %d ranks", rank, nranks);
  if (!yah::nccl()->ok) return yah::set_error(YAH_ERR_NCCL, "NCCL (libnccl.so.2) could not be loaded");
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return yah::set_error(YAH_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t nc;
  const ncclResult_t r = yah::nccl()->comm_init_rank(&nc, nranks, u, rank);
  if (r != ncclSuccess) return yah::nccl_fail(r, "ncclCommInitRank");
  *comm = new yah_tp_comm{nc, rank, nranks, dev};
  return YAH_OK;
}

int yah_tp_destroy(yah_tp_comm* comm) {
  if (!comm) return YAH_OK;
  const ncclResult_t r = yah::nccl()->comm_destroy(comm->nc);
  delete comm;
  return r == ncclSuccess ? YAH_OK : yah::nccl_fail(r, "ncclCommDestroy");
}

int yah_tp_rank(const yah_tp_comm* comm, int* rank, int* nranks) {
  if (!comm || !rank || !nranks) return yah::set_error(YAH_ERR_ARG, "null argument");
  *rank = comm->rank;
  *nranks = comm->nranks;
  return YAH_OK;
}

int yah_tp_allreduce_f32(yah_tp_comm* comm, float* buf, int64_t count, void* stream) {
  if (!comm || (!buf && count > 0) || count < 0) return yah::set_error(YAH_ERR_ARG, "bad allreduce arguments");
  if (count == 0) return YAH_OK;
  const ncclResult_t r = yah::nccl()->all_reduce(buf, buf, (size_t)count, ncclFloat32, ncclSum, comm->nc,
                                                 static_cast<cudaStream_t>(stream));
  return r == ncclSuccess ? YAH_OK : yah::nccl_fail(r, "ncclAllReduce");
}

int yah_tp_linear_col(yah_tp_comm* comm, const void* w_shard, int ggml_type, int64_t N_local, int64_t K,
                      int64_t w_row_stride, const void* x, int64_t M, int64_t ldx, void* y, int y_dtype,
                      int64_t ldy, int epilogue, const void* aux, int64_t ldaux, void* stream) {
  if (!comm) return yah::set_error(YAH_ERR_ARG, "null comm");
  if (M <= 32 && epilogue != YAH_EPI_SWIGLU)
    return yah_qgemv(w_shard, ggml_type, N_local, K, w_row_stride, 0, x, M, ldx, y, y_dtype, ldy, epilogue, aux,
                     ldaux, stream);
  return yah_qgemm(w_shard, ggml_type, N_local, K, w_row_stride, 0, x, M, ldx, y, y_dtype, ldy, epilogue, aux,
                   ldaux, stream);
}

int yah_tp_linear_row(yah_tp_comm* comm, const void* w_shard, int ggml_type, int64_t N, int64_t K_local,
                      int64_t w_row_stride, int64_t kb_off, const void* x, int64_t M, int64_t ldx, float* y,
                      const float* resid, void* stream) {
  if (!comm) return yah::set_error(YAH_ERR_ARG, "null comm");
  // y is the contiguous f32 [M][N] the allreduce sums; rank 0 adds resid (which may be y itself)
  const bool add = comm->rank == 0 && resid != nullptr;
  const int epi = add ? YAH_EPI_RESID : YAH_EPI_STORE;
  int rc = M <= 32 ? yah_qgemv(w_shard, ggml_type, N, K_local, w_row_stride, kb_off, x, M, ldx, y, YAH_F32, N, epi,
                               add ? resid : nullptr, add ? N : 0, stream)
                   : yah_qgemm(w_shard, ggml_type, N, K_local, w_row_stride, kb_off, x, M, ldx, y, YAH_F32, N, epi,
                               add ? resid : nullptr, add ? N : 0, stream);
  if (rc) return rc;
  return yah_tp_allreduce_f32(comm, y, M * N, stream);
}

int yah_rmsnorm(const float* h, int64_t ldh, int64_t M, int64_t H, float eps, float gain, void* out, int64_t ldo,
                void* stream) {
  if (!h || !out || M < 0 || H <= 0) return yah::set_error(YAH_ERR_ARG, "bad rmsnorm arguments");
  if (H % 4 || ldh % 4 || ldo % 4 || ldh < H || ldo < H || (reinterpret_cast<uintptr_t>(h) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 7))
    return yah::set_error(YAH_ERR_UNSUPPORTED, "rmsnorm needs H and strides multiples of 4, 16-byte aligned h, "
                                               "8-byte aligned out");
  if (M > 0x7fffffff) return yah::set_error(YAH_ERR_ARG, "M too large");
  if (M == 0) return YAH_OK;
  yah::rmsnorm_kernel<false, true, true><<<(unsigned)M, yah::kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      const_cast<float*>(h), ldh, (int)H, nullptr, 0, eps, gain, static_cast<__half*>(out), ldo);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? YAH_OK : yah::set_error(YAH_ERR_CUDA, "rmsnorm launch: %s", cudaGetErrorString(e));
}

int yah_add_rmsnorm(float* h, int64_t ldh, const void* d, int d_dtype, int64_t ldd, int64_t M, int64_t H, float eps,
                    float gain, void* out, int64_t ldo, void* stream) {
  if (!h || !d || M < 0 || H <= 0 || (d_dtype != YAH_F16 && d_dtype != YAH_F32))
    return yah::set_error(YAH_ERR_ARG, "bad add_rmsnorm arguments");
  const uintptr_t dalign = d_dtype == YAH_F16 ? 7 : 15;
  if (H % 4 || ldh % 4 || ldd % 4 || ldh < H || ldd < H || (reinterpret_cast<uintptr_t>(h) & 15) ||
      (reinterpret_cast<uintptr_t>(d) & dalign) ||
      (out && (ldo % 4 || ldo < H || (reinterpret_cast<uintptr_t>(out) & 7))))
    return yah::set_error(YAH_ERR_UNSUPPORTED, "add_rmsnorm needs H and strides multiples of 4, 16-byte aligned h, "
                                               "d aligned to 4 of its elements, 8-byte aligned out");
  if (M > 0x7fffffff) return yah::set_error(YAH_ERR_ARG, "M too large");
  if (M == 0) return YAH_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  __half* o = static_cast<__half*>(out);
  const dim3 grid((unsigned)M), block(yah::kNormThreads);
  if (d_dtype == YAH_F16) {
    if (o) yah::rmsnorm_kernel<true, true, true><<<grid, block, 0, s>>>(h, ldh, (int)H, d, ldd, eps, gain, o, ldo);
    else yah::rmsnorm_kernel<true, false, true><<<grid, block, 0, s>>>(h, ldh, (int)H, d, ldd, eps, gain, o, 0);
  } else {
    if (o) yah::rmsnorm_kernel<true, true, false><<<grid, block, 0, s>>>(h, ldh, (int)H, d, ldd, eps, gain, o, ldo);
    else yah::rmsnorm_kernel<true, false, false><<<grid, block, 0, s>>>(h, ldh, (int)H, d, ldd, eps, gain, o, 0);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? YAH_OK : yah::set_error(YAH_ERR_CUDA, "add_rmsnorm launch: %s", cudaGetErrorString(e));
}

int yah_tp_allreduce_f16(yah_tp_comm* comm, void* buf, int64_t count, void* stream) {
  if (!comm || (!buf && count > 0) || count < 0) return yah::set_error(YAH_ERR_ARG, "bad allreduce arguments");
  if (count == 0) return YAH_OK;
  const ncclResult_t r = yah::nccl()->all_reduce(buf, buf, (size_t)count, ncclFloat16, ncclSum, comm->nc,
                                                 static_cast<cudaStream_t>(stream));
  return r == ncclSuccess ? YAH_OK : yah::nccl_fail(r, "ncclAllReduce");
}

}  // extern "C"
