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
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "../../include/yah_qgemm.h"
#include "kernels.h"
#include "ptx.cuh"

namespace yah {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
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
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.get_error_string = reinterpret_cast<decltype(api.get_error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
             api.get_error_string;
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

// ---------------------------------------------------------------- fused row-parallel reduce (peer memory)
// The row-parallel GEMM writes each rank's f32 partial of token t straight into the memory of the rank that owns t
// (yah_qgemm_sliced, stores over NVLink); these kernels finish the exchange: a signal (a flag in every rank's memory,
// release at system scope after the writes), a bounded wait for all ranks' flags, and the reduce of a rank's token
// slice with the RMSNorm whose f16 output is written into every rank's activation buffer (the all-gather).
struct PtrTable {
  void* p[kMaxSlices];
};

__global__ void tp_signal_kernel(PtrTable flags, int n, int slot, int value) {
  const int i = threadIdx.x;
  if (i >= n) return;
  int* f = static_cast<int*>(flags.p[i]) + slot;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f), "r"(value) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread i waits until flags[i] >= value (flags carry increasing epochs). Bounded: after budget_ns it records
// kStatusTimeoutPeer and returns; it also leaves as soon as another wait has failed.
__global__ void tp_wait_kernel(const int* flags, int count, int value, int* status, unsigned long long budget_ns) {
  const int i = threadIdx.x;
  if (i >= count) return;
  const int* f = flags + i;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v >= value) return;
    if ((it & 255) == 255) {
      if (*(volatile int*)status != 0) return;
      if (global_ns() - t0 > budget_ns) {
        set_status(status, kStatusTimeoutPeer);
        return;
      }
      __nanosleep(64);
    }
  }
}

// Signal and wait in one launch: thread i < n stores value into slot (base + rank) of rank i's flags (release,
// system scope), then waits, bounded as tp_wait_kernel, until this rank's flag base + i is >= value.
__global__ void tp_barrier_kernel(PtrTable flags, int n, int base, int rank, int value, const int* own, int* status,
                                  unsigned long long budget_ns) {
  const int i = threadIdx.x;
  if (i >= n) return;
  int* f = static_cast<int*>(flags.p[i]) + base + rank;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f), "r"(value) : "memory");
  const int* w = own + base + i;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(w) : "memory");
    if (v >= value) return;
    if ((it & 255) == 255) {
      if (*(volatile int*)status != 0) return;
      if (global_ns() - t0 > budget_ns) {
        set_status(status, kStatusTimeoutPeer);
        return;
      }
      __nanosleep(64);
    }
  }
}

// One row per CTA of this rank's token slice: h += parts[0] + parts[1] + ... (in slot order; the parts are the
// other ranks' writes, read through L2), then (NORM) out = f16(h * gain / sqrt(mean(h^2) + eps)) written to row
// out_row0 + row of every rank's output buffer.
template <bool ADD, bool NORM>
__global__ void __launch_bounds__(kNormThreads)
    tp_reduce_norm_kernel(float* __restrict__ h, int64_t ldh, int H, const float* __restrict__ parts, int nparts,
                          int64_t part_stride, int64_t ldp, float eps, float gain, PtrTable outs, int nout,
                          int64_t out_row0, int64_t ldo) {
  float* row = h + (int64_t)blockIdx.x * ldh;
  float ss = 0.f;
  for (int i = 4 * threadIdx.x; i < H; i += 4 * kNormThreads) {
    float4 v = *reinterpret_cast<const float4*>(row + i);
    if (ADD) {
      const float* pr = parts + (int64_t)blockIdx.x * ldp + i;
      for (int s = 0; s < nparts; ++s) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(pr + s * part_stride));
        v.x += a.x, v.y += a.y, v.z += a.z, v.w += a.w;
      }
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
  const int64_t orow = (out_row0 + blockIdx.x) * ldo;
  for (int i = 4 * threadIdx.x; i < H; i += 4 * kNormThreads) {
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    const __half2 a = __floats2half2_rn(v.x * scale, v.y * scale), b = __floats2half2_rn(v.z * scale, v.w * scale);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&a);
    packed.y = *reinterpret_cast<const uint32_t*>(&b);
    for (int r = 0; r < nout; ++r) *reinterpret_cast<uint2*>(static_cast<__half*>(outs.p[r]) + orow + i) = packed;
  }
  // (the writes to other ranks' memory are ordered before the signal by the kernel boundary: the signal kernel,
  // next in stream order, fences at system scope before its release store)
}

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<MemGetAddressRangeFn>(p);
  });
  return fn;
}

constexpr int kMaxPeerBufs = 8;
constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait

}  // namespace
}  // namespace yah

// Device buffers of every rank of a communicator, as addresses this process can use (CUDA IPC mappings of the
// other ranks' allocations, exchanged with one ncclAllGather).
struct yah_tp_peers {
  int rank = 0, nranks = 0, nbufs = 0;
  void* ptr[yah::kMaxPeerBufs][yah::kMaxSlices] = {};
  void* mapped[yah::kMaxPeerBufs][yah::kMaxSlices] = {};  // IPC mappings to close (allocation bases)
};

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

int yah_tp_allgather_f32(yah_tp_comm* comm, const float* send, float* recv, int64_t count, void* stream) {
  if (!comm || count < 0 || (count > 0 && (!send || !recv))) return yah::set_error(YAH_ERR_ARG, "bad allgather arguments");
  if (count == 0) return YAH_OK;
  const ncclResult_t r = yah::nccl()->all_gather(send, recv, (size_t)count, ncclFloat32, comm->nc,
                                                 static_cast<cudaStream_t>(stream));
  return r == ncclSuccess ? YAH_OK : yah::nccl_fail(r, "ncclAllGather");
}

int yah_tp_peers_create(yah_tp_comm* comm, void* const* bufs, int nbufs, void* stream, yah_tp_peers** out) {
  if (!comm || !bufs || !out || nbufs < 1 || nbufs > yah::kMaxPeerBufs)
    return yah::set_error(YAH_ERR_ARG, "bad peers arguments (1..%d buffers)", yah::kMaxPeerBufs);
  *out = nullptr;
  if (comm->nranks > yah::kMaxSlices)
    return yah::set_error(YAH_ERR_UNSUPPORTED, "%d ranks; peer buffers take at most %d", comm->nranks,
                          yah::kMaxSlices);
  auto range = yah::address_range_fn();
  if (!range) return yah::set_error(YAH_ERR_DEVICE, "the driver does not provide cuMemGetAddressRange");
  struct Rec {
    cudaIpcMemHandle_t h;
    uint64_t offset;
  };
  const int P = comm->nranks, me = comm->rank;
  const size_t per = sizeof(Rec) * (size_t)nbufs;
  Rec* recs = new Rec[(size_t)P * nbufs]();
  yah_tp_peers* pe = new yah_tp_peers;
  pe->rank = me;
  pe->nranks = P;
  pe->nbufs = nbufs;
  auto bail = [&](int rc) {
    delete[] recs;
    yah_tp_peers_destroy(pe);
    return rc;
  };
  for (int b = 0; b < nbufs; ++b) {
    if (!bufs[b]) return bail(yah::set_error(YAH_ERR_ARG, "null buffer %d", b));
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(bufs[b])) != CUDA_SUCCESS)
      return bail(yah::set_error(YAH_ERR_ARG, "buffer %d is not device memory", b));
    Rec& r = recs[(size_t)me * nbufs + b];
    const cudaError_t e = cudaIpcGetMemHandle(&r.h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return bail(yah::set_error(YAH_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e)));
    r.offset = reinterpret_cast<CUdeviceptr>(bufs[b]) - base;
    pe->ptr[b][me] = bufs[b];
  }
  if (P > 1) {
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* d = nullptr;
    cudaError_t e = cudaMalloc(&d, per * P);
    if (e != cudaSuccess) return bail(yah::set_error(YAH_ERR_CUDA, "cudaMalloc: %s", cudaGetErrorString(e)));
    char* dme = static_cast<char*>(d) + per * me;
    e = cudaMemcpyAsync(dme, recs + (size_t)me * nbufs, per, cudaMemcpyHostToDevice, st);
    ncclResult_t nr = ncclSuccess;
    if (e == cudaSuccess) nr = yah::nccl()->all_gather(dme, d, per, ncclUint8, comm->nc, st);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaMemcpyAsync(recs, d, per * P, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(st);
    cudaFree(d);
    if (nr != ncclSuccess) return bail(yah::nccl_fail(nr, "ncclAllGather (peer handles)"));
    if (e != cudaSuccess) return bail(yah::set_error(YAH_ERR_CUDA, "peer handle exchange: %s", cudaGetErrorString(e)));
    for (int r = 0; r < P; ++r) {
      if (r == me) continue;
      for (int b = 0; b < nbufs; ++b) {
        const Rec& rec = recs[(size_t)r * nbufs + b];
        void* base = nullptr;
        e = cudaIpcOpenMemHandle(&base, rec.h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
          return bail(yah::set_error(YAH_ERR_CUDA, "cudaIpcOpenMemHandle (rank %d, buffer %d): %s", r, b,
                                     cudaGetErrorString(e)));
        pe->mapped[b][r] = base;
        pe->ptr[b][r] = static_cast<char*>(base) + rec.offset;
      }
    }
  }
  delete[] recs;
  *out = pe;
  return YAH_OK;
}

int yah_tp_peers_ptr(const yah_tp_peers* pe, int rank, int buf, void** ptr) {
  if (!pe || !ptr || rank < 0 || rank >= pe->nranks || buf < 0 || buf >= pe->nbufs)
    return yah::set_error(YAH_ERR_ARG, "bad peers query");
  *ptr = pe->ptr[buf][rank];
  return YAH_OK;
}

int yah_tp_peers_destroy(yah_tp_peers* pe) {
  if (!pe) return YAH_OK;
  int rc = YAH_OK;
  for (int b = 0; b < yah::kMaxPeerBufs; ++b)
    for (int r = 0; r < yah::kMaxSlices; ++r)
      if (pe->mapped[b][r] && cudaIpcCloseMemHandle(pe->mapped[b][r]) != cudaSuccess)
        rc = yah::set_error(YAH_ERR_CUDA, "cudaIpcCloseMemHandle");
  delete pe;
  return rc;
}

int yah_tp_signal(const yah_tp_peers* pe, int flag_buf, int slot, int value, void* stream) {
  if (!pe || flag_buf < 0 || flag_buf >= pe->nbufs || slot < 0) return yah::set_error(YAH_ERR_ARG, "bad signal");
  yah::PtrTable t{};
  for (int r = 0; r < pe->nranks; ++r) t.p[r] = pe->ptr[flag_buf][r];
  yah::tp_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(t, pe->nranks, slot, value);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? YAH_OK : yah::set_error(YAH_ERR_CUDA, "signal launch: %s", cudaGetErrorString(e));
}

int yah_tp_wait(const yah_tp_peers* pe, int flag_buf, int first, int count, int value, void* stream) {
  if (!pe || flag_buf < 0 || flag_buf >= pe->nbufs || first < 0 || count < 1 || count > 32)
    return yah::set_error(YAH_ERR_ARG, "bad wait");
  int* status = nullptr;
  const int rc = yah::device_status_word(&status);
  if (rc) return rc;
  const int* flags = static_cast<const int*>(pe->ptr[flag_buf][pe->rank]) + first;
  yah::tp_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, count, value, status, yah::kPeerWaitNs);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? YAH_OK : yah::set_error(YAH_ERR_CUDA, "wait launch: %s", cudaGetErrorString(e));
}

int yah_tp_reduce_norm(const yah_tp_peers* pe, float* h, int64_t ldh, int64_t rows, int64_t H, const float* parts,
                       int nparts, int64_t part_stride, int64_t ldp, float eps, float gain, int out_buf,
                       int64_t out_row0, int64_t ldo, void* stream) {
  if (!pe || !h || rows < 0 || H <= 0 || nparts < 0 || (nparts > 0 && !parts) || out_buf >= pe->nbufs)
    return yah::set_error(YAH_ERR_ARG, "bad reduce_norm arguments");
  if (H % 4 || ldh % 4 || ldh < H || (reinterpret_cast<uintptr_t>(h) & 15) ||
      (nparts > 0 && (ldp % 4 || part_stride % 4 || (reinterpret_cast<uintptr_t>(parts) & 15))) ||
      (out_buf >= 0 && (ldo % 4 || ldo < H)))
    return yah::set_error(YAH_ERR_UNSUPPORTED, "reduce_norm needs H and strides multiples of 4, 16-byte aligned h "
                                               "and parts");
  if (rows > 0x7fffffff) return yah::set_error(YAH_ERR_ARG, "too many rows");
  if (rows == 0) return YAH_OK;
  yah::PtrTable t{};
  const int nout = out_buf >= 0 ? pe->nranks : 0;
  for (int r = 0; r < nout; ++r) t.p[r] = pe->ptr[out_buf][r];
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)rows), block(yah::kNormThreads);
  if (nparts > 0 && nout > 0)
    yah::tp_reduce_norm_kernel<true, true><<<grid, block, 0, s>>>(h, ldh, (int)H, parts, nparts, part_stride, ldp,
                                                                   eps, gain, t, nout, out_row0, ldo);
  else if (nparts > 0)
    yah::tp_reduce_norm_kernel<true, false><<<grid, block, 0, s>>>(h, ldh, (int)H, parts, nparts, part_stride, ldp,
                                                                    eps, gain, t, 0, 0, 0);
  else if (nout > 0)
    yah::tp_reduce_norm_kernel<false, true><<<grid, block, 0, s>>>(h, ldh, (int)H, nullptr, 0, 0, 0, eps, gain, t,
                                                                    nout, out_row0, ldo);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? YAH_OK : yah::set_error(YAH_ERR_CUDA, "reduce_norm launch: %s", cudaGetErrorString(e));
}

int yah_tp_linear_row_scatter(const yah_tp_peers* pe, const void* w_shard, int ggml_type, int64_t N,
                              int64_t K_local, int64_t w_row_stride, int64_t kb_off, const void* x, int64_t M,
                              int64_t ldx, int recv_buf, void* stream) {
  if (!pe || recv_buf < 0 || recv_buf >= pe->nbufs) return yah::set_error(YAH_ERR_ARG, "bad scatter arguments");
  const int P = pe->nranks;
  if (M % P || (M / P) % 16)
    return yah::set_error(YAH_ERR_ARG, "M=%lld does not split into %d token slices of a multiple of 16 rows",
                          (long long)M, P);
  const int64_t ms = M / P;
  void* ys[yah::kMaxSlices] = {};
  for (int o = 0; o < P; ++o)  // rank o's buffer, slot of this rank: [P][ms][N] f32
    ys[o] = static_cast<char*>(pe->ptr[recv_buf][o]) + (size_t)pe->rank * ms * N * sizeof(float);
  return yah_qgemm_sliced(w_shard, ggml_type, N, K_local, w_row_stride, kb_off, x, M, ldx, ys, P, ms, N, stream);
}

int yah_tp_barrier(const yah_tp_peers* pe, int flag_buf, int base, int value, void* stream) {
  if (!pe || flag_buf < 0 || flag_buf >= pe->nbufs || base < 0) return yah::set_error(YAH_ERR_ARG, "bad barrier");
  int* status = nullptr;
  const int rc = yah::device_status_word(&status);
  if (rc) return rc;
  yah::PtrTable t{};
  for (int r = 0; r < pe->nranks; ++r) t.p[r] = pe->ptr[flag_buf][r];
  const int* own = static_cast<const int*>(pe->ptr[flag_buf][pe->rank]);
  yah::tp_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(t, pe->nranks, base, pe->rank, value, own,
                                                                          status, yah::kPeerWaitNs);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? YAH_OK : yah::set_error(YAH_ERR_CUDA, "barrier launch: %s", cudaGetErrorString(e));
}

}  // extern "C"
