// The C ABI of libyah_b200.so (declared in include/yah_qgemm.h): argument and footprint checks, per-device
// state (SM count, the kernel status word, the GEMV split-K workspace), and the CUDA runtime wrappers that play
// the role of the reference's LoomDevice (engine/model/loom_runtime.hpp:153-325). Every entry point returns a
// status code; nothing throws across the boundary.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <vector>
#include <string>

#include "../../include/yah_qgemm.h"
#include "kernels.h"
#include "ptx.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

}  // namespace

namespace yah {
int set_error(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
}  // namespace yah

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  return fail(YAH_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define CK(call)                                   \
  do {                                             \
    cudaError_t e_ = (call);                       \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

// Which decode GEMV runs (yah_set_gemv_impl): 0 the tcgen05 form where it covers the call, else the mma.sync form;
// 1 only the tcgen05 form; 2 only the mma.sync form.
std::atomic<int> g_gemv_impl{0};

// SMs the GEMM / GEMV plans may use (0: all). A process that overlaps collectives with these kernels leaves the
// rest to the collective's kernels.
std::atomic<int> g_sm_budget{0};

struct DevState {
  bool ready = false;
  int sms = 0;
  int cc_major = 0, cc_minor = 0;
  int* status = nullptr;  // device status word
  float* ws = nullptr;    // GEMV split-K partials
  size_t ws_bytes = 0;
  int* counters = nullptr;
  size_t counters_n = 0;
  float* gemm_scratch = nullptr;  // chunked-accumulation sums of the tile GEMM
  size_t gemm_scratch_bytes = 0;
  float* gemm_kpart = nullptr;    // split-K chunk results of the tile GEMM
  size_t gemm_kpart_bytes = 0;
  int max_pairs = -1;             // resident 2-CTA clusters of the tile GEMM (-1: not queried yet)
};

// Grow a per-device buffer to at least `need` bytes (cudaFree synchronises the device, so no launch still uses
// the old one).
int grow(void** buf, size_t* have, size_t need) {
  if (need <= *have) return YAH_OK;
  if (*buf) CK(cudaFree(*buf));
  *buf = nullptr;
  *have = 0;
  CK(cudaMalloc(buf, need));
  *have = need;
  return YAH_OK;
}

constexpr int kMaxDev = 64;
DevState g_dev[kMaxDev];
std::mutex g_mu;

// State of the current device, created on first use (status word allocated and zeroed).
int dev_state(DevState** out) {
  int d = 0;
  CK(cudaGetDevice(&d));
  if (d < 0 || d >= kMaxDev) return fail(YAH_ERR_DEVICE, "device ordinal %d out of range", d);
  std::lock_guard<std::mutex> lk(g_mu);
  DevState& s = g_dev[d];
  if (!s.ready) {
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, d));
    s.sms = prop.multiProcessorCount;
    s.cc_major = prop.major;
    s.cc_minor = prop.minor;
    if (s.cc_major != 10) return fail(YAH_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", d,
                                      s.cc_major, s.cc_minor);
    if (!yah::tensor_map_encoder_available())
      return fail(YAH_ERR_DEVICE, "the driver does not provide cuTensorMapEncodeTiled");
    CK(cudaMalloc(&s.status, sizeof(int)));
    CK(cudaMemset(s.status, 0, sizeof(int)));
    s.ready = true;
  }
  *out = &s;
  return YAH_OK;
}

int sms_of(const DevState* s) {
  const int b = g_sm_budget.load(std::memory_order_relaxed);
  return b > 0 && b < s->sms ? b : s->sms;
}

int sb_bytes(int type) {
  switch (type) {
    case YAH_Q8_0: return 272;
    case YAH_Q3_K: return 110;
    case YAH_Q4_K: return 144;
    case YAH_Q5_K: return 176;
    case YAH_Q6_K: return 210;
    case YAH_IQ4_XS: return 136;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

constexpr int64_t kMaxDim = (int64_t)1 << 30;

// Shared checks of yah_qgemm / yah_qgemv.
// gemv: the decode GEMV's rules (its swiglu kind also writes f32, in place over the gate when aux == y).
int check_linear(const void* w, int type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                 int64_t M, int64_t ldx, const void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux,
                 int64_t ldaux, bool gemv = false) {
  const int sb = sb_bytes(type);
  if (!sb) return fail(YAH_ERR_UNSUPPORTED, "unsupported GGML type %d (supported: Q8_0=8, Q3_K=11, Q4_K=12, Q5_K=13, Q6_K=14, IQ4_XS=23)", type);
  if (!w || !x || !y) return fail(YAH_ERR_ARG, "null weight, input or output pointer");
  if (N < 1 || M < 1 || K < 256 || N > kMaxDim || M > kMaxDim || K > kMaxDim)
    return fail(YAH_ERR_ARG, "bad shape N=%lld K=%lld M=%lld", (long long)N, (long long)K, (long long)M);
  if (K % 256) return fail(YAH_ERR_ARG, "K=%lld is not a multiple of 256", (long long)K);
  if (kb_off < 0) return fail(YAH_ERR_ARG, "negative kb_off");
  if (w_row_stride < (kb_off + K / 256) * sb)
    return fail(YAH_ERR_ARG, "w_row_stride %lld is shorter than the K window (%lld bytes)", (long long)w_row_stride,
                (long long)((kb_off + K / 256) * sb));
  if (!aligned16(w) || w_row_stride % 16)
    return fail(YAH_ERR_UNSUPPORTED,
                "weight rows must start 16-byte aligned (pointer %p, row stride %lld); Q6_K and Q3_K rows are aligned "
                "when their super-block count is a multiple of 8, IQ4_XS rows when it is even",
                w, (long long)w_row_stride);
  if (!aligned16(x) || ldx < K || ldx % 8)
    return fail(YAH_ERR_ARG, "activations must be 16-byte aligned with ldx >= K and ldx %% 8 == 0 (ldx=%lld)",
                (long long)ldx);
  if (ldy < N) return fail(YAH_ERR_ARG, "ldy %lld < N %lld", (long long)ldy, (long long)N);
  if (y_dtype != YAH_F32 && y_dtype != YAH_F16) return fail(YAH_ERR_UNSUPPORTED, "y_dtype %d", y_dtype);
  if (epilogue == YAH_EPI_RESID) {
    if (!aux || ldaux < N) return fail(YAH_ERR_ARG, "YAH_EPI_RESID needs aux f32 [M][ldaux >= N]");
    if (y_dtype != YAH_F32) return fail(YAH_ERR_UNSUPPORTED, "YAH_EPI_RESID writes f32");
  } else if (epilogue == YAH_EPI_SWIGLU) {
    if (!aux || ldaux < N) return fail(YAH_ERR_ARG, "YAH_EPI_SWIGLU needs aux f32 gate [M][ldaux >= N]");
    if (y_dtype != YAH_F16 && !gemv) return fail(YAH_ERR_UNSUPPORTED, "YAH_EPI_SWIGLU of the tile GEMM writes f16");
    if (y_dtype == YAH_F16 && aux == y)
      return fail(YAH_ERR_ARG, "YAH_EPI_SWIGLU in place (aux == y) needs an f32 output");
  } else if (epilogue != YAH_EPI_STORE) {
    return fail(YAH_ERR_UNSUPPORTED, "epilogue %d", epilogue);
  }
  return YAH_OK;
}

int after_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return cuda_fail(e, what);
  return YAH_OK;
}

}  // namespace

namespace {
constexpr int kNotTaken = -1;

// The kernel the GEMV dispatch picks. Automatic choice, measured on B200 (Q4_K 4096 x 14336 and 14336 x 4096): the
// tcgen05 form takes 23-31 us at 1..32 tokens, its MMA issue the limit; the mma.sync form 12 us at one token and
// 15-24 us while its activations stay resident (row ranges), but 24 us at 8 and 39-74 us at 12..32 tokens when it
// has to run stream-K. Returns the tcgen05 plan (ok = false: the mma.sync kernel runs); refuses (YAH_ERR_UNSUPPORTED
// through *rc) a forced tcgen05 choice the kernel does not cover.
yah::GemvTcPlan gemv_tc_choice(int t, int64_t N, int64_t K, int64_t M, int sms, int dev, int* rc) {
  *rc = YAH_OK;
  const int impl = g_gemv_impl.load(std::memory_order_relaxed);
  if (impl == 2) return yah::GemvTcPlan{};
  if (impl == 0 && (M <= 8 || yah::qgemv_plan(t, N, K, M, sms).mode != 1)) return yah::GemvTcPlan{};
  const yah::GemvTcPlan pl = yah::qgemv_tc_plan(t, N, K, M, sms, dev);
  if (!pl.ok && impl == 1)
    *rc = fail(YAH_ERR_UNSUPPORTED, "the tcgen05 decode GEMV does not cover type %d, N=%lld, K=%lld, M=%lld", t,
               (long long)N, (long long)K, (long long)M);
  return pl;
}

// The tcgen05 decode GEMV for a call it covers (per the impl switch): its launch status, or kNotTaken when the call
// goes to the mma.sync form. a.status must be set.
int launch_gemv_tc(const yah::QGemvArgs& a, int dev, cudaStream_t stream) {
  int rc;
  const yah::GemvTcPlan pl = gemv_tc_choice(a.type, a.N, a.K, a.M, a.num_sms, dev, &rc);
  if (rc) return rc;
  if (!pl.ok) return kNotTaken;
  return after_launch(yah::launch_qgemv_tc(a, pl, stream), "qgemv (tcgen05) launch");
}

yah::QGemvArgs gemv_args(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                         const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                         const void* aux, int64_t ldaux, int* status, int sms) {
  yah::QGemvArgs a;
  a.w = w;
  a.type = t;
  a.N = N;
  a.K = K;
  a.w_row_stride = w_row_stride;
  a.kb_off = kb_off;
  a.x = x;
  a.M = M;
  a.ldx = ldx;
  a.y = y;
  a.y_f16 = y_dtype == YAH_F16;
  a.ldy = ldy;
  a.epilogue = epilogue;
  a.aux = static_cast<const float*>(aux);
  a.ldaux = ldaux;
  a.status = status;
  a.num_sms = sms;
  return a;
}

// Caller workspace of the mma.sync GEMV: the split partial sums, then the split counters, each 256-byte aligned.
size_t gemv_ws_floats_bytes(const yah::GemvPlan& p) {
  return ((size_t)p.ws_floats * sizeof(float) + 255) & ~size_t(255);
}
size_t gemv_ws_bytes(const yah::GemvPlan& p) {
  if (p.ws_floats <= 0) return 0;
  return gemv_ws_floats_bytes(p) + (((size_t)p.counters * sizeof(int) + 255) & ~size_t(255));
}
}  // namespace

namespace yah {
int device_status_word(int** status) {
  DevState* s;
  const int rc = dev_state(&s);
  if (rc) return rc;
  *status = s->status;
  return YAH_OK;
}

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return fail(code, "%s", buf);
}
}  // namespace yah

extern "C" {

const char* yah_version(void) { return "yah_b200 0.1 (sm_100a)"; }

const char* yah_last_error(void) { return g_err.c_str(); }

int yah_block_elements(int t) { return t == YAH_Q8_0 ? 32 : sb_bytes(t) ? 256 : 0; }

int yah_block_bytes(int t) { return t == YAH_Q8_0 ? 34 : sb_bytes(t); }

int64_t yah_row_bytes(int t, int64_t K) {
  const int be = yah_block_elements(t);
  if (!be || K < 0 || K % be) return -1;
  return K / be * yah_block_bytes(t);
}

int yah_device_count(int* count) {
  if (!count) return fail(YAH_ERR_ARG, "null count");
  CK(cudaGetDeviceCount(count));
  return YAH_OK;
}

int yah_set_device(int device) {
  CK(cudaSetDevice(device));
  return YAH_OK;
}

int yah_get_device(int* device) {
  if (!device) return fail(YAH_ERR_ARG, "null device");
  CK(cudaGetDevice(device));
  return YAH_OK;
}

int yah_device_info(int device, int* sm_count, int* cc_major, int* cc_minor, int64_t* total_mem) {
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (sm_count) *sm_count = prop.multiProcessorCount;
  if (cc_major) *cc_major = prop.major;
  if (cc_minor) *cc_minor = prop.minor;
  if (total_mem) *total_mem = (int64_t)prop.totalGlobalMem;
  return YAH_OK;
}

int yah_malloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(YAH_ERR_ARG, "null ptr");
  CK(cudaMalloc(ptr, bytes));
  return YAH_OK;
}

int yah_free(void* ptr) {
  CK(cudaFree(ptr));
  return YAH_OK;
}

int yah_host_alloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(YAH_ERR_ARG, "null ptr");
  CK(cudaHostAlloc(ptr, bytes, cudaHostAllocDefault));
  return YAH_OK;
}

int yah_host_free(void* ptr) {
  CK(cudaFreeHost(ptr));
  return YAH_OK;
}

int yah_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_memset(void* ptr, int value, size_t bytes, void* stream) {
  CK(cudaMemsetAsync(ptr, value, bytes, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_stream_create(void** stream) {
  if (!stream) return fail(YAH_ERR_ARG, "null stream");
  cudaStream_t s;
  CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return YAH_OK;
}

int yah_stream_destroy(void* stream) {
  CK(cudaStreamDestroy((cudaStream_t)stream));
  return YAH_OK;
}

int yah_stream_synchronize(void* stream) {
  CK(cudaStreamSynchronize((cudaStream_t)stream));
  return YAH_OK;
}

int yah_device_synchronize(void) {
  CK(cudaDeviceSynchronize());
  return YAH_OK;
}

int yah_event_create(void** event) {
  if (!event) return fail(YAH_ERR_ARG, "null event");
  cudaEvent_t e;
  CK(cudaEventCreate(&e));
  *event = e;
  return YAH_OK;
}

int yah_event_destroy(void* event) {
  CK(cudaEventDestroy((cudaEvent_t)event));
  return YAH_OK;
}

int yah_event_record(void* event, void* stream) {
  CK(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_event_synchronize(void* event) {
  CK(cudaEventSynchronize((cudaEvent_t)event));
  return YAH_OK;
}

int yah_event_elapsed_ms(void* start, void* end, float* ms) {
  if (!ms) return fail(YAH_ERR_ARG, "null ms");
  CK(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return YAH_OK;
}

int yah_stream_begin_capture(void* stream) {
  if (!stream) return fail(YAH_ERR_ARG, "capture needs a non-default stream");
  CK(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal));
  return YAH_OK;
}

int yah_stream_end_capture(void* stream, void** graph_exec) {
  if (!stream || !graph_exec) return fail(YAH_ERR_ARG, "null stream or graph");
  *graph_exec = nullptr;
  cudaGraph_t g = nullptr;
  CK(cudaStreamEndCapture((cudaStream_t)stream, &g));
  cudaGraphExec_t ge = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
  *graph_exec = ge;
  return YAH_OK;
}

int yah_graph_launch(void* graph_exec, void* stream) {
  if (!graph_exec) return fail(YAH_ERR_ARG, "null graph");
  CK(cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_graph_destroy(void* graph_exec) {
  if (graph_exec) CK(cudaGraphExecDestroy((cudaGraphExec_t)graph_exec));
  return YAH_OK;
}

int yah_set_launch_overlap(int on) {
  yah::set_launch_overlap(on != 0);
  return YAH_OK;
}

int yah_realign_rows(const void* src, int64_t rows, int64_t row_bytes, int64_t src_stride, void* dst,
                     int64_t dst_stride, void* stream) {
  if (!src || !dst) return fail(YAH_ERR_ARG, "null pointer");
  if (rows < 0 || row_bytes <= 0 || src_stride < row_bytes || dst_stride < row_bytes)
    return fail(YAH_ERR_ARG, "bad sizes: rows %lld, row bytes %lld, strides %lld / %lld", (long long)rows,
                (long long)row_bytes, (long long)src_stride, (long long)dst_stride);
  if (!aligned16(dst) || dst_stride % 16)
    return fail(YAH_ERR_ARG, "the destination rows must start 16-byte aligned (stride %lld)", (long long)dst_stride);
  if (rows == 0) return YAH_OK;
  CK(cudaMemcpy2DAsync(dst, (size_t)dst_stride, src, (size_t)src_stride, (size_t)row_bytes, (size_t)rows,
                       cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return YAH_OK;
}

int yah_set_sm_budget(int sms) {
  if (sms < 0) return fail(YAH_ERR_ARG, "SM budget %d < 0", sms);
  g_sm_budget.store(sms, std::memory_order_relaxed);
  return YAH_OK;
}

int yah_stream_wait_event(void* stream, void* event) {
  if (!event) return fail(YAH_ERR_ARG, "null event");
  CK(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0));
  return YAH_OK;
}

namespace {
// Self-test of the failure path: one warp waits on an mbarrier that nothing arrives on, through the kernels' own
// bounded wait with a short budget, so the wait runs out, records kStatusTimeoutFull in the status word and returns.
__global__ void selftest_wait_kernel(int* status, long long budget) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    yah::mbar_init(&bar, 1);
    yah::fence_barrier_init();
  }
  __syncthreads();
  yah::mbar_wait(&bar, 0, status, yah::kStatusTimeoutFull, false, budget);
}
}  // namespace

int yah_selftest_bounded_wait(int64_t budget_cycles, int* code) {
  if (!code) return fail(YAH_ERR_ARG, "null code");
  if (budget_cycles < 1000 || budget_cycles > (int64_t(1) << 31))
    return fail(YAH_ERR_ARG, "budget %lld cycles outside [1000, 2^31]", (long long)budget_cycles);
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  CK(cudaMemset(s->status, 0, sizeof(int)));
  selftest_wait_kernel<<<1, 32>>>(s->status, (long long)budget_cycles);
  CK(cudaGetLastError());
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(code, s->status, sizeof(int), cudaMemcpyDeviceToHost));
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (s->counters && s->counters_n) CK(cudaMemset(s->counters, 0, s->counters_n * sizeof(int)));
  }
  CK(cudaMemset(s->status, 0, sizeof(int)));
  CK(cudaDeviceSynchronize());
  return YAH_OK;
}

int yah_status_word(int* code) {
  if (!code) return fail(YAH_ERR_ARG, "null code");
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  CK(cudaMemcpy(code, s->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (*code) {
    // A launch whose wait ran out left early, possibly before adding itself to the GEMV's split counters (the last
    // CTA of a row block resets them only when every CTA arrived). Clear them, so that later calls count from
    // zero again, then the word itself.
    CK(cudaDeviceSynchronize());
    {
      std::lock_guard<std::mutex> lk(g_mu);
      if (s->counters && s->counters_n) CK(cudaMemset(s->counters, 0, s->counters_n * sizeof(int)));
    }
    CK(cudaMemset(s->status, 0, sizeof(int)));
    CK(cudaDeviceSynchronize());
  }
  return YAH_OK;
}

int yah_qgemm_limits(int* sm_count, int* max_pairs) {
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (s->max_pairs < 0) s->max_pairs = yah::qgemm_max_pairs(YAH_Q4_K, 192);
  }
  if (sm_count) *sm_count = s->sms;
  if (max_pairs) *max_pairs = s->max_pairs;
  return YAH_OK;
}

int yah_qgemm_footprint(int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, int64_t M, int64_t ldx,
                        int y_dtype, int64_t ldy, int64_t* w_bytes, int64_t* x_bytes, int64_t* y_bytes) {
  const int sb = sb_bytes(t);
  if (!sb || K % 256 || N < 1 || M < 1) return fail(YAH_ERR_ARG, "bad footprint query");
  if (w_bytes) *w_bytes = (N - 1) * w_row_stride + (kb_off + K / 256) * sb;
  if (x_bytes) *x_bytes = ((M - 1) * ldx + K) * 2;
  if (y_bytes) *y_bytes = ((M - 1) * ldy + N) * (y_dtype == YAH_F16 ? 2 : 4);
  return YAH_OK;
}

int yah_dequant(const void* w, int t, int64_t rows, int64_t K, int64_t w_row_stride, int64_t kb_off, void* out,
                int64_t ldo, void* stream) {
  const int sb = sb_bytes(t);
  if (!sb) return fail(YAH_ERR_UNSUPPORTED, "unsupported GGML type %d", t);
  if (!w || !out) return fail(YAH_ERR_ARG, "null pointer");
  if (rows < 1 || K < 256 || K % 256 || kb_off < 0) return fail(YAH_ERR_ARG, "bad shape rows=%lld K=%lld",
                                                                 (long long)rows, (long long)K);
  if (w_row_stride < (kb_off + K / 256) * sb) return fail(YAH_ERR_ARG, "w_row_stride shorter than the K window");
  if ((reinterpret_cast<uintptr_t>(w) & 1) || (w_row_stride & 1))
    return fail(YAH_ERR_ARG, "weight rows must be 2-byte aligned");
  if (!aligned16(out) || ldo < K || ldo % 8) return fail(YAH_ERR_ARG, "out must be 16-byte aligned, ldo >= K, %% 8");
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  return after_launch(yah::launch_dequant(w, t, rows, K, w_row_stride, kb_off, static_cast<uint16_t*>(out), ldo,
                                          s->sms, (cudaStream_t)stream),
                      "dequant launch");
}

}  // extern "C"

namespace {

// Workspace of a tile-GEMM call: the chunked-accumulation sums, then (split K) the chunk results, 256-byte aligned.
struct GemmNeed {
  size_t scratch = 0, kpart = 0;
  size_t total() const { return scratch + kpart; }
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Checks, tile choice and workspace needs of yah_qgemm_tile / yah_qgemm_ws. `sized` only: the pointers may be null
// (a workspace-size query).
int qgemm_prepare(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                  int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux,
                  int64_t ldaux, int bn, int grid, int64_t kchunk, int cta_pair, bool sized, yah::QGemmArgs& a,
                  GemmNeed& need) {
  // a size query checks the shape with stand-in pointers (aux distinct from y)
  static const char kDummy[32] __attribute__((aligned(16))) = {};
  int rc = sized ? check_linear(kDummy, t, N, K, w_row_stride, kb_off, kDummy, M, ldx, kDummy, y_dtype, ldy,
                                epilogue, epilogue == YAH_EPI_STORE ? nullptr : kDummy + 16, ldaux)
                 : check_linear(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux);
  if (rc) return rc;
  if (grid < 0) return fail(YAH_ERR_ARG, "negative grid");
  if (kchunk == 0) kchunk = K > 4096 ? 2048 : K;  // see the accuracy note in qgemm_tc.cu
  if (kchunk < 0 || kchunk >= K) kchunk = K;
  if (kchunk % 128) return fail(YAH_ERR_ARG, "kchunk %lld is not a multiple of 128", (long long)kchunk);
  DevState* s;
  rc = dev_state(&s);
  if (rc) return rc;
  a.w = w;
  a.type = t;
  a.N = N;
  a.K = K;
  a.w_row_stride = w_row_stride;
  a.kb_off = kb_off;
  a.x = x;
  a.M = M;
  a.ldx = ldx;
  a.y = y;
  a.y_f16 = y_dtype == YAH_F16;
  a.ldy = ldy;
  a.epilogue = epilogue;
  a.aux = static_cast<const float*>(aux);
  a.ldaux = ldaux;
  a.status = s->status;
  a.num_sms = sms_of(s);
  a.grid = grid > a.num_sms ? a.num_sms : grid;
  a.kchunk = kchunk;
  a.scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (s->max_pairs < 0) s->max_pairs = yah::qgemm_max_pairs(t, bn);
  }
  a.max_pairs = s->max_pairs;
  a.pair = (cta_pair != 0 && a.max_pairs > 0) ? 1 : 0;
  if (cta_pair == 1 && !a.pair) return fail(YAH_ERR_UNSUPPORTED, "2-CTA clusters are not available on this device");
  if (bn == 0) bn = a.pair ? (kchunk < K ? 160 : 256) : 192;
  if (a.pair ? (bn != 256 && bn != 160 && bn != 128) : (bn != 192 && bn != 128 && bn != 64))
    return fail(YAH_ERR_ARG, "bn %d is not a %s tile width (pairs: 256, 160, 128; single CTAs: 192, 128, 64)", bn,
                a.pair ? "2-SM pair" : "single-CTA");
  a.bn = bn;
  // Split K: with an automatic grid, when the (row tile, 16-token unit) space is smaller than the CTAs (pairs) the
  // device holds, every accumulation chunk of a tile becomes its own unit (chunks of whole super-blocks). The
  // result is bit-identical to the unsplit GEMM with the same chunk length.
  a.nsplit = 1;
  if (grid == 0 && kchunk < K && kchunk % 256 == 0) {
    const int ncta = a.pair ? 2 : 1;
    const int64_t units = (N + 128 * ncta - 1) / (128 * ncta) * ((M + 15) / 16);
    int64_t slots = a.num_sms / ncta;
    if (a.pair && slots > a.max_pairs) slots = a.max_pairs;
    if (units < slots) a.nsplit = (int)((K + kchunk - 1) / kchunk);
  }
  need = GemmNeed{};
  if (kchunk < K) {
    need.scratch = align256((size_t)yah::qgemm_grid(a) * bn * 128 * sizeof(float));
    if (a.nsplit > 1) need.kpart = align256((size_t)a.nsplit * (size_t)M * (size_t)N * sizeof(float));
  }
  return YAH_OK;
}

}  // namespace

extern "C" {

int yah_qgemm_tile(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                   int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux,
                   int64_t ldaux, int bn, int grid, int64_t kchunk, int cta_pair, void* stream) {
  yah::QGemmArgs a;
  GemmNeed need;
  int rc = qgemm_prepare(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, bn, grid,
                         kchunk, cta_pair, false, a, need);
  if (rc) return rc;
  if (need.scratch) {
    DevState* s;
    rc = dev_state(&s);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    rc = grow(reinterpret_cast<void**>(&s->gemm_scratch), &s->gemm_scratch_bytes, need.scratch);
    if (rc) return rc;
    a.scratch = s->gemm_scratch;
    if (need.kpart) {
      rc = grow(reinterpret_cast<void**>(&s->gemm_kpart), &s->gemm_kpart_bytes, need.kpart);
      if (rc) return rc;
      a.kpart = s->gemm_kpart;
    }
  }
  return after_launch(yah::launch_qgemm_tc(a, (cudaStream_t)stream), "qgemm launch");
}

int yah_qgemm_workspace_size(int t, int64_t N, int64_t K, int64_t M, int y_dtype, int epilogue, int bn, int grid,
                             int64_t kchunk, int cta_pair, size_t* bytes) {
  if (!bytes) return fail(YAH_ERR_ARG, "null bytes");
  yah::QGemmArgs a;
  GemmNeed need;
  const int64_t rs = yah_row_bytes(t, K);
  int rc = qgemm_prepare(nullptr, t, N, K, rs > 0 ? (rs + 15) / 16 * 16 : 0, 0, nullptr, M, (K + 7) / 8 * 8, nullptr,
                         y_dtype, N, epilogue, nullptr, N, bn, grid, kchunk, cta_pair, true, a, need);
  if (rc) return rc;
  *bytes = need.total();
  return YAH_OK;
}

int yah_qgemm_sliced(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                     int64_t M, int64_t ldx, void* const* ys, int nslices, int64_t slice_rows, int64_t ldy,
                     void* stream) {
  if (!ys || nslices < 1 || nslices > yah::kMaxSlices)
    return fail(YAH_ERR_ARG, "%d token slices (1..%d)", nslices, yah::kMaxSlices);
  if (slice_rows < 16 || slice_rows % 16 || slice_rows * nslices < M)
    return fail(YAH_ERR_ARG, "slice_rows %lld: a multiple of 16 with nslices * slice_rows >= M",
                (long long)slice_rows);
  for (int i = 0; i < nslices; ++i)
    if (!ys[i] || (reinterpret_cast<uintptr_t>(ys[i]) & 3)) return fail(YAH_ERR_ARG, "slice %d: null or unaligned", i);
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  yah::QGemmArgs a;
  GemmNeed need;
  // an explicit grid: split K writes its chunks elsewhere first, so slices never split; up to K = 8192 one
  // accumulation chunk (the shared-drain tile; chunked tiles store scalar-wise here, without TMA stores)
  rc = qgemm_prepare(w, t, N, K, w_row_stride, kb_off, x, M, ldx, ys[0], YAH_F32, ldy, YAH_EPI_STORE, nullptr, 0, 0,
                     sms_of(s), K <= 8192 ? -1 : 0, -1, false, a, need);
  if (rc) return rc;
  a.nsl = nslices;
  a.slice_rows = slice_rows;
  for (int i = 0; i < nslices; ++i) a.ysl[i] = ys[i];
  if (need.scratch) {
    std::lock_guard<std::mutex> lk(g_mu);
    rc = grow(reinterpret_cast<void**>(&s->gemm_scratch), &s->gemm_scratch_bytes, need.scratch);
    if (rc) return rc;
    a.scratch = s->gemm_scratch;
  }
  return after_launch(yah::launch_qgemm_tc(a, (cudaStream_t)stream), "qgemm (token slices) launch");
}

int yah_qgemm_ws(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                 int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux,
                 int64_t ldaux, int bn, int grid, int64_t kchunk, int cta_pair, void* workspace,
                 size_t workspace_bytes, void* stream) {
  yah::QGemmArgs a;
  GemmNeed need;
  int rc = qgemm_prepare(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, bn, grid,
                         kchunk, cta_pair, false, a, need);
  if (rc) return rc;
  if (need.total() > 0) {
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
      return fail(YAH_ERR_ARG, "this call needs a 256-byte aligned workspace of %zu bytes", need.total());
    if (workspace_bytes < need.total())
      return fail(YAH_ERR_SIZE, "workspace of %zu bytes; this call needs %zu (yah_qgemm_workspace_size)",
                  workspace_bytes, need.total());
    a.scratch = static_cast<float*>(workspace);
    if (need.kpart) a.kpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + need.scratch);
  }
  return after_launch(yah::launch_qgemm_tc(a, (cudaStream_t)stream), "qgemm launch");
}

int yah_qgemm_ffn(const void* w_gate, const void* w_up, int t, int64_t N, int64_t K, int64_t w_row_stride,
                  int64_t kb_off, const void* x, int64_t M, int64_t ldx, void* y, int64_t ldy, int bn, int cta_pair,
                  void* stream) {
  int rc = check_linear(w_gate, t, N, K, w_row_stride, kb_off, x, M, ldx, y, YAH_F16, ldy, YAH_EPI_STORE, nullptr, 0);
  if (rc) return rc;
  rc = check_linear(w_up, t, N, K, w_row_stride, kb_off, x, M, ldx, y, YAH_F16, ldy, YAH_EPI_STORE, nullptr, 0);
  if (rc) return rc;
  DevState* s;
  rc = dev_state(&s);
  if (rc) return rc;
  const int64_t kchunk = K > 4096 ? 2048 : K;  // the automatic chunk of yah_qgemm_tile
  yah::QGemmArgs a;
  a.w = w_gate;
  a.w2 = w_up;
  a.type = t;
  a.N = N;
  a.K = K;
  a.w_row_stride = w_row_stride;
  a.kb_off = kb_off;
  a.x = x;
  a.M = M;
  a.ldx = ldx;
  a.y = y;
  a.y_f16 = 1;
  a.ldy = ldy;
  a.epilogue = yah::kEpiFfn;
  a.aux = nullptr;
  a.ldaux = 0;
  a.status = s->status;
  a.num_sms = sms_of(s);
  a.grid = 0;
  a.kchunk = kchunk;
  a.scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (s->max_pairs < 0) s->max_pairs = yah::qgemm_max_pairs(t, bn);
  }
  a.max_pairs = s->max_pairs;
  // automatic tile: single CTAs at 192 tokens with two accumulator regions (measured fastest for this epilogue:
  // 1014 us against 1136 for pairs at 256 at M = 4096, N = 14336, K = 4096)
  a.pair = (cta_pair == 1 && a.max_pairs > 0) ? 1 : 0;
  if (cta_pair == 1 && !a.pair) return fail(YAH_ERR_UNSUPPORTED, "2-CTA clusters are not available on this device");
  if (bn == 0) bn = a.pair ? (kchunk < K ? 160 : 256) : 192;
  if (a.pair ? (bn != 256 && bn != 160 && bn != 128) : (bn != 192 && bn != 128 && bn != 64))
    return fail(YAH_ERR_ARG, "bn %d is not a %s tile width (pairs: 256, 160, 128; single CTAs: 192, 128, 64)", bn,
                a.pair ? "2-SM pair" : "single-CTA");
  a.bn = bn;
  if (kchunk < K) {
    std::lock_guard<std::mutex> lk(g_mu);
    const size_t need = (size_t)yah::qgemm_grid(a) * bn * 128 * sizeof(float);
    rc = grow(reinterpret_cast<void**>(&s->gemm_scratch), &s->gemm_scratch_bytes, need);
    if (rc) return rc;
    a.scratch = s->gemm_scratch;
  }
  return after_launch(yah::launch_qgemm_tc(a, (cudaStream_t)stream), "qgemm_ffn launch");
}

// The opt-in tile table (yah_tile_rules_set): the only mutable process-wide configuration of the library.
std::vector<yah_tile_rule> g_rules;

int yah_tile_rules_set(const yah_tile_rule* rules, int n) {
  if (n < 0 || (n > 0 && !rules)) return fail(YAH_ERR_ARG, "bad rule list");
  for (int i = 0; i < n; ++i) {
    const yah_tile_rule& r = rules[i];
    if (sb_bytes(r.ggml_type) == 0) return fail(YAH_ERR_ARG, "rule %d: unsupported type %d", i, r.ggml_type);
    if (r.epilogue < YAH_EPI_STORE || r.epilogue > YAH_EPI_SWIGLU || (r.y_dtype != YAH_F32 && r.y_dtype != YAH_F16))
      return fail(YAH_ERR_ARG, "rule %d: bad epilogue or output type", i);
    if (r.N < 1 || r.K < 256 || r.m_max < 1 || r.grid < 0)
      return fail(YAH_ERR_ARG, "rule %d: bad shape, token bound or grid", i);
    const bool pair_ok = r.cta_pair == 1 && (r.bn == 256 || r.bn == 160 || r.bn == 128);
    const bool single_ok = r.cta_pair == 0 && (r.bn == 192 || r.bn == 128 || r.bn == 64);
    if (!pair_ok && !single_ok) return fail(YAH_ERR_ARG, "rule %d: bn %d is not a tile of cta_pair %d", i, r.bn, r.cta_pair);
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_rules.assign(rules, rules + n);
  return YAH_OK;
}

int yah_tile_rules_clear(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_rules.clear();
  return YAH_OK;
}

int yah_tile_rules_count(int* n) {
  if (!n) return fail(YAH_ERR_ARG, "null count");
  std::lock_guard<std::mutex> lk(g_mu);
  *n = (int)g_rules.size();
  return YAH_OK;
}

int yah_qgemm(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
              int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux, int64_t ldaux,
              void* stream) {
  // A tuned rule for this GEMM (the smallest token bound >= M, else the largest bound); otherwise the built-in
  // choice: 2-SM pairs for plain stores, single CTAs with two accumulator regions when the epilogue reads an
  // operand (its latency then overlaps the next tile's MMAs).
  int bn = 0, grid = 0, pair = epilogue == YAH_EPI_STORE ? -1 : 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    const yah_tile_rule* best = nullptr;
    for (const yah_tile_rule& r : g_rules) {
      if (r.ggml_type != t || r.epilogue != epilogue || r.y_dtype != y_dtype || r.N != N || r.K != K) continue;
      const bool fits = r.m_max >= M, best_fits = best && best->m_max >= M;
      if (!best || (fits && (!best_fits || r.m_max < best->m_max)) || (!fits && !best_fits && r.m_max > best->m_max))
        best = &r;
    }
    if (best) {
      bn = best->bn;
      grid = best->grid;
      pair = best->cta_pair;
    }
  }
  return yah_qgemm_tile(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, bn, grid,
                        0, pair, stream);
}

int yah_qgemv(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
              int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux, int64_t ldaux,
              void* stream) {
  int rc = check_linear(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, true);
  if (rc) return rc;
  if (M > 32) return fail(YAH_ERR_ARG, "yah_qgemv takes at most 32 tokens (M=%lld); use yah_qgemm", (long long)M);
  DevState* s;
  rc = dev_state(&s);
  if (rc) return rc;
  const yah::QGemvArgs a = gemv_args(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux,
                                     ldaux, s->status, sms_of(s));
  {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    rc = launch_gemv_tc(a, dev, (cudaStream_t)stream);
    if (rc != kNotTaken) return rc;
  }
  const yah::GemvPlan plan = yah::qgemv_plan(t, N, K, M, sms_of(s));
  if (plan.ws_floats > 0) {
    std::lock_guard<std::mutex> lk(g_mu);
    rc = grow(reinterpret_cast<void**>(&s->ws), &s->ws_bytes, (size_t)plan.ws_floats * sizeof(float));
    if (rc) return rc;
    if ((size_t)plan.counters > s->counters_n) {
      size_t have = s->counters_n * sizeof(int);
      rc = grow(reinterpret_cast<void**>(&s->counters), &have, (size_t)plan.counters * sizeof(int));
      if (rc) return rc;
      CK(cudaMemset(s->counters, 0, (size_t)plan.counters * sizeof(int)));
      s->counters_n = (size_t)plan.counters;
    }
  }
  return after_launch(yah::launch_qgemv_ws(a, plan, s->ws, s->counters, (cudaStream_t)stream), "qgemv launch");
}

int yah_qgemv_x(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                int x_dtype, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux,
                int64_t ldaux, void* stream) {
  if (x_dtype == YAH_F16)
    return yah_qgemv(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, stream);
  if (x_dtype != YAH_F32) return fail(YAH_ERR_UNSUPPORTED, "x_dtype %d (YAH_F16 or YAH_F32)", x_dtype);
  int rc = check_linear(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, true);
  if (rc) return rc;
  if (M > 32) return fail(YAH_ERR_ARG, "yah_qgemv_x takes at most 32 tokens (M=%lld)", (long long)M);
  if (g_gemv_impl.load(std::memory_order_relaxed) == 1)
    return fail(YAH_ERR_UNSUPPORTED, "the tcgen05 decode GEMV takes f16 activations only");
  DevState* s;
  rc = dev_state(&s);
  if (rc) return rc;
  const int sms = sms_of(s);
  // tokens per launch: as many as stay resident (hi and lo rows) beside two weight stages
  int64_t mc = M;
  while (mc > 0 && yah::qgemv_plan_xf32(t, N, K, mc, sms).ringst < 2) --mc;
  if (mc == 0)
    return fail(YAH_ERR_UNSUPPORTED, "f32 activations of K=%lld do not fit in shared memory", (long long)K);
  const int ysz = y_dtype == YAH_F16 ? 2 : 4;
  for (int64_t m0 = 0; m0 < M; m0 += mc) {
    const int64_t m = M - m0 < mc ? M - m0 : mc;
    yah::QGemvArgs a = gemv_args(w, t, N, K, w_row_stride, kb_off, static_cast<const float*>(x) + m0 * ldx, m, ldx,
                                 static_cast<char*>(y) + m0 * ldy * ysz, y_dtype, ldy, epilogue,
                                 aux ? static_cast<const float*>(aux) + m0 * ldaux : nullptr, ldaux, s->status, sms);
    a.x_f32 = 1;
    const yah::GemvPlan plan = yah::qgemv_plan_xf32(t, N, K, m, sms);
    rc = after_launch(yah::launch_qgemv_ws(a, plan, nullptr, nullptr, (cudaStream_t)stream), "qgemv (f32 x) launch");
    if (rc) return rc;
  }
  return YAH_OK;
}

int yah_qgemv_swiglu_x(const void* w_gate, int gate_type, int64_t gate_row_stride, const void* w_up, int up_type,
                       int64_t up_row_stride, int64_t N, int64_t K, const void* x, int x_dtype, int64_t M,
                       int64_t ldx, float* y, int64_t ldy, void* stream) {
  if (!y) return fail(YAH_ERR_ARG, "null output");
  int rc = yah_qgemv_x(w_gate, gate_type, N, K, gate_row_stride, 0, x, x_dtype, M, ldx, y, YAH_F32, ldy,
                       YAH_EPI_STORE, nullptr, 0, stream);
  if (rc) return rc;
  return yah_qgemv_x(w_up, up_type, N, K, up_row_stride, 0, x, x_dtype, M, ldx, y, YAH_F32, ldy, YAH_EPI_SWIGLU, y,
                     ldy, stream);
}

int yah_qgemv_workspace_size(int t, int64_t N, int64_t K, int64_t M, size_t* bytes) {
  if (!bytes) return fail(YAH_ERR_ARG, "null bytes");
  if (!sb_bytes(t) || N < 1 || K < 256 || K % 256 || M < 1 || M > 32) return fail(YAH_ERR_ARG, "bad GEMV shape");
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const yah::GemvTcPlan pl = gemv_tc_choice(t, N, K, M, sms_of(s), dev, &rc);
  if (rc) return rc;
  *bytes = pl.ok ? 0 : gemv_ws_bytes(yah::qgemv_plan(t, N, K, M, sms_of(s)));
  return YAH_OK;
}

int yah_qgemv_ws(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, const void* x,
                 int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue, const void* aux,
                 int64_t ldaux, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_linear(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, true);
  if (rc) return rc;
  if (M > 32) return fail(YAH_ERR_ARG, "yah_qgemv_ws takes at most 32 tokens (M=%lld); use yah_qgemm", (long long)M);
  DevState* s;
  rc = dev_state(&s);
  if (rc) return rc;
  const yah::QGemvArgs a = gemv_args(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux,
                                     ldaux, s->status, sms_of(s));
  {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    rc = launch_gemv_tc(a, dev, (cudaStream_t)stream);
    if (rc != kNotTaken) return rc;
  }
  const yah::GemvPlan plan = yah::qgemv_plan(t, N, K, M, sms_of(s));
  const size_t need = gemv_ws_bytes(plan);
  float* part = nullptr;
  int* counters = nullptr;
  if (need > 0) {
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
      return fail(YAH_ERR_ARG, "this call needs a 256-byte aligned workspace of %zu bytes", need);
    if (workspace_bytes < need)
      return fail(YAH_ERR_SIZE, "workspace of %zu bytes; this call needs %zu (yah_qgemv_workspace_size)",
                  workspace_bytes, need);
    part = static_cast<float*>(workspace);
    counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + gemv_ws_floats_bytes(plan));
    // the split counters start at zero on every call (the caller's buffer holds anything)
    CK(cudaMemsetAsync(counters, 0, (size_t)plan.counters * sizeof(int), (cudaStream_t)stream));
  }
  return after_launch(yah::launch_qgemv_ws(a, plan, part, counters, (cudaStream_t)stream), "qgemv launch");
}

int yah_qgemv_noalloc(const void* w, int t, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                      const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                      const void* aux, int64_t ldaux, void* stream) {
  int rc = check_linear(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux, ldaux, true);
  if (rc) return rc;
  if (M > 32) return fail(YAH_ERR_ARG, "yah_qgemv_noalloc takes at most 32 tokens (M=%lld)", (long long)M);
  // No call below allocates: device attributes, the driver's tensor-map encoder and the static scratch address.
  int dev = 0, sms = 0, major = 0;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major != 10) return fail(YAH_ERR_DEVICE, "device %d is not an sm_100 device", dev);
  if (!yah::tensor_map_encoder_available())
    return fail(YAH_ERR_DEVICE, "the driver does not provide cuTensorMapEncodeTiled");
  {
    // the tcgen05 form needs no scratch: only the variant's own status word
    void* base = nullptr;
    CK(yah::qgemv_static_setup(dev, &base));
    const yah::QGemvArgs a = gemv_args(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux,
                                       ldaux, yah::qgemv_static_status_word(base), sms);
    rc = launch_gemv_tc(a, dev, (cudaStream_t)stream);
    if (rc != kNotTaken) return rc;
  }
  const yah::GemvPlan plan = yah::qgemv_plan(t, N, K, M, sms);
  if ((size_t)plan.ws_floats > yah::qgemv_static_partials() || (size_t)plan.counters > yah::qgemv_static_counters())
    return fail(YAH_ERR_SIZE,
                "yah_qgemv_noalloc: partial sums of %lld floats (%lld tokens, %lld rows, %d CTAs) exceed the "
                "static %zu-float scratch; call yah_qgemv instead",
                (long long)plan.ws_floats, (long long)M, (long long)N, plan.grid, yah::qgemv_static_partials());
  void* base = nullptr;
  CK(yah::qgemv_static_setup(dev, &base));
  // status set by the launcher: the variant's own status word
  const yah::QGemvArgs a = gemv_args(w, t, N, K, w_row_stride, kb_off, x, M, ldx, y, y_dtype, ldy, epilogue, aux,
                                     ldaux, nullptr, sms);
  return after_launch(yah::launch_qgemv_static(a, plan, base, (cudaStream_t)stream), "qgemv_noalloc launch");
}

int yah_qgemv_describe(int t, int64_t N, int64_t K, int64_t M, char* buf, int64_t cap) {
  if (!buf || cap < 1) return fail(YAH_ERR_ARG, "null or empty buffer");
  if (!sb_bytes(t) || N < 1 || K < 256 || K % 256 || M < 1 || M > 32) return fail(YAH_ERR_ARG, "bad GEMV shape");
  DevState* s;
  int rc = dev_state(&s);
  if (rc) return rc;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const yah::GemvTcPlan pl = gemv_tc_choice(t, N, K, M, sms_of(s), dev, &rc);
  if (rc) return rc;
  if (pl.ok) {
    snprintf(buf, (size_t)cap,
             "tcgen05: clusters of %d CTAs (K parts of %d super-blocks), %d tiles of %d rows, grid %d, %d MMA "
             "columns, %d super-block(s) per weight stage",
             pl.ks, pl.srange, pl.tiles, pl.rt, pl.grid, pl.tp, pl.sw);
  } else {
    const yah::GemvPlan g = yah::qgemv_plan(t, N, K, M, sms_of(s));
    snprintf(buf, (size_t)cap, "mma.sync: mode %d (%s), grid %d, %lld partial floats, %lld counters", g.mode,
             g.mode == 0 ? "row ranges" : g.mode == 1 ? "stream-K" : "one-token row ranges", g.grid,
             (long long)g.ws_floats, (long long)g.counters);
  }
  return YAH_OK;
}

int yah_set_gemv_impl(int impl) {
  if (impl < 0 || impl > 2) return fail(YAH_ERR_ARG, "gemv impl %d (0 auto, 1 tcgen05, 2 mma.sync)", impl);
  g_gemv_impl.store(impl, std::memory_order_relaxed);
  return YAH_OK;
}

int yah_qgemv_swiglu(const void* w_gate, int gate_type, int64_t gate_row_stride, const void* w_up, int up_type,
                     int64_t up_row_stride, int64_t N, int64_t K, const void* x, int64_t M, int64_t ldx, float* y,
                     int64_t ldy, void* stream) {
  if (!y) return fail(YAH_ERR_ARG, "null output");
  // the gate GEMV into y (f32), then the up GEMV whose swiglu kind reads each gate value and overwrites it
  int rc = yah_qgemv(w_gate, gate_type, N, K, gate_row_stride, 0, x, M, ldx, y, YAH_F32, ldy, YAH_EPI_STORE, nullptr,
                     0, stream);
  if (rc) return rc;
  return yah_qgemv(w_up, up_type, N, K, up_row_stride, 0, x, M, ldx, y, YAH_F32, ldy, YAH_EPI_SWIGLU, y, ldy, stream);
}

int yah_qgemv_noalloc_status(int* code) {
  if (!code) return fail(YAH_ERR_ARG, "null code");
  int dev = 0;
  CK(cudaGetDevice(&dev));
  void* base = nullptr;
  CK(yah::qgemv_static_setup(dev, &base));
  CK(yah::qgemv_static_status(base, code, true));
  return YAH_OK;
}

}  // extern "C"
