// Internal launch interface between the C ABI (capi.cu) and the kernel translation units. Host-only types.
// Every launcher assumes its arguments were validated by the C ABI and returns a cudaError_t.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <stdint.h>

namespace yah {

// Records the calling thread's last error message (yah_last_error) and returns `code` (capi.cu).
int set_error(int code, const std::string& msg);

// kEpiFfn (tile GEMM only): y = f16(silu(x W^T) * (x w2^T)), the gate and up weights in one GEMM.
enum Epilogue : int { kEpiStore = 0, kEpiResid = 1, kEpiSwiglu = 2, kEpiFfn = 3 };

// Tile-GEMM problem (token-major): y[M][ldy] (+)= x[M][ldx] (f16) * W[N][K]^T, W in GGUF rows.
constexpr int kMaxSlices = 8;

struct QGemmArgs {
  const void* w;        // weight rows (GGUF block layout)
  int type;             // GGML type id (8, 12, 14)
  int64_t N, K;         // weight rows, reduction length (K window length)
  int64_t w_row_stride; // bytes between weight rows
  int64_t kb_off;       // first 256-element super-block of the K window within each row
  const void* x;        // f16 activations [M][ldx]
  int64_t M, ldx;
  void* y;              // output [M][ldy], f32 or f16
  int y_f16;            // 1: f16 output, 0: f32
  int64_t ldy;
  int epilogue;         // kEpiStore / kEpiResid / kEpiSwiglu
  const float* aux;     // resid (kres) or gate (swiglu), f32 [M][ldaux]
  int64_t ldaux;
  int* status;          // device status word (bounded-wait failures)
  int num_sms;          // SMs of the device
  int grid;             // persistent CTAs (0: one per SM)
  int bn;               // max tokens per tile (64, 128, 192)
  int64_t kchunk;       // K per accumulation chunk (multiple of 64; 0: the whole K in one chunk)
  float* scratch;       // grid * bn * 128 f32 chunk sums when kchunk < K, else unused
  int pair;             // 1: 2-SM pairs (tcgen05 cta_group::2, clusters of 2), 0: one CTA per tile
  int max_pairs;        // resident 2-CTA clusters the device holds (pair mode)
  const void* w2 = nullptr;  // kEpiFfn: the up weights (same type, shape and row stride as w, the gate weights)
  int nsplit = 1;       // > 1: each accumulation chunk of a tile is its own work unit (split K, one chunk each)
  float* kpart = nullptr;  // nsplit * M * N f32 chunk results when nsplit > 1, summed in chunk order afterwards
  // Token slices (kEpiStore only, no split): output token t goes to ysl[t / slice_rows] + (t % slice_rows) * ldy
  // instead of y (slices of other GPUs' memory: a reduce-scatter written by the epilogue). 0: y.
  int nsl = 0;
  int64_t slice_rows = 0;
  void* ysl[kMaxSlices] = {};
};

// Resident 2-CTA clusters of the tile-GEMM kernel on the current device (0 if clusters are unavailable).
int qgemm_max_pairs(int type, int bn);

// Largest persistent grid and the chunk scratch a launch needs.
int qgemm_grid(const QGemmArgs& a);

cudaError_t launch_qgemm_tc(const QGemmArgs& a, cudaStream_t stream);

// Standalone dequant: out[rows][ldo] f16 = decode(W).
cudaError_t launch_dequant(const void* w, int type, int64_t rows, int64_t K, int64_t row_stride, int64_t kb_off,
                           uint16_t* out, int64_t ldo, int num_sms, cudaStream_t stream);

// Decode GEMV (M <= 32 tokens).
struct QGemvArgs {
  const void* w;
  int type;
  int64_t N, K, w_row_stride, kb_off;
  const void* x;   // f16 [M][ldx], or f32 [M][ldx] when x_f32
  int64_t M, ldx;
  int x_f32 = 0;   // GEMV only: f32 activations (row-range form with resident activations; see qgemv_plan_xf32)
  void* y;         // [M][ldy], f32 or f16
  int y_f16;
  int64_t ldy;
  int epilogue;    // kEpiStore / kEpiResid
  const float* aux;
  int64_t ldaux;
  int* status;
  int num_sms;
};

// Work split and shared-memory layout of a GEMV launch. Stream-K launches whose row blocks are split between CTAs
// need `ws_floats` floats of partial sums and `counters` zeroed ints (both 0 otherwise).
struct GemvPlan {
  int mode;    // 0: each CTA owns a row range (no scratch); 1: stream-K over 128-row blocks (scratch when split);
               // 2: one Q4_K token, row ranges, 4-row x 4-super-block MMA units (no scratch)
  int grid;
  int rb, rgp, slots, tsplit, ntw, cw;  // stage rows, row groups, super-block slots, token split, tiles per warp
  int sst, ringst;                      // super-blocks per stage (divides slots), stages per ring
  int P, ops, opw;                      // super-blocks per weight copy, copies per stage, copy row width
  int wreg, xoff, sumoff, stage_bytes, stages, redoff, baroff, smem;
  int xres, resoff, ressum;             // activations resident for the whole launch (small M * K)
  int64_t ws_floats, counters;
};
GemvPlan qgemv_plan(int type, int64_t N, int64_t K, int64_t M, int num_sms);
// Plan of an f32-activation GEMV of M tokens (2M hi / lo token rows, resident, row ranges); ringst < 2: too many
// tokens to keep resident (the caller splits the tokens).
GemvPlan qgemv_plan_xf32(int type, int64_t N, int64_t K, int64_t M, int num_sms);
cudaError_t launch_qgemv_ws(const QGemvArgs& a, const GemvPlan& plan, float* ws, int* counters,
                            cudaStream_t stream);

// Decode GEMV on tcgen05 (qgemv_tc.cu; Q4_K, M <= 32): clusters of ks CTAs split K, tiles of rt <= 128 weight rows,
// tp MMA columns (16 or 32 token rows, the rest zero). No scratch: the K parts meet in distributed shared memory.
struct GemvTcPlan {
  int ok;      // 0: the tcgen05 form does not cover this call
  int tp, ks, rt, tiles, grid, srange, sw, pitch;
};
GemvTcPlan qgemv_tc_plan(int type, int64_t N, int64_t K, int64_t M, int num_sms, int device);
cudaError_t launch_qgemv_tc(const QGemvArgs& a, const GemvTcPlan& plan, cudaStream_t stream);

// The allocation-free GEMV: its scratch is a file-scope device array in qgemv.cu. setup looks up its address on
// `device` (which must be current) once and caches it; the launcher clears the split counters it needs and runs
// the GEMV on that scratch; status reads (and optionally clears) the variant's own status word.
size_t qgemv_static_partials();
size_t qgemv_static_counters();
cudaError_t qgemv_static_setup(int device, void** base);
cudaError_t launch_qgemv_static(const QGemvArgs& a, const GemvPlan& plan, void* base, cudaStream_t stream);
cudaError_t qgemv_static_status(void* base, int* code, bool clear);
int* qgemv_static_status_word(void* base);

// Programmatic dependent launch of the GEMV kernels (on by default): a launch may start while the preceding kernel
// on its stream finishes, streaming its weights early; activations and outputs wait for that kernel to complete.
bool launch_overlap();
void set_launch_overlap(bool on);

// Records an error for yah_last_error() and returns `code` (shared by the C ABI translation units).
int set_error(int code, const char* fmt, ...);

// Tensor-map encoder resolved from the driver at first use (no libcuda link dependency).
bool tensor_map_encoder_available();

// The current device's status word (the device state is created on first use): for kernels outside capi.cu.
int device_status_word(int** status);

}  // namespace yah
