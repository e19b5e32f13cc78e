/*
 * yah_qgemm.h - C ABI of the B200 (sm_100a) quantised-linear library libyah_b200.so.
 *
 * The reference engine has no C-ABI GEMM: its operator is a compiled Loom kernel dispatched through
 * LoomDevice::Dispatch / LoomGraph::Dispatch (engine/model/loom_runtime.hpp:276-290, :384-410) with the binding
 * order weight, input, [gate | resid], ..., output (engine/gpu/loom/tools/gen_gemm_tile.py:319-320) and the
 * GEMV's weights, x, y (engine/gpu/loom/tools/gen_gemv.py:729). Each entry point below names the reference
 * interface it replaces. Conventions:
 *   - plain pointers and sizes only; every function returns a status (YAH_OK = 0) and never throws;
 *     yah_last_error() returns the calling thread's last message;
 *   - all tensors are caller-owned device memory; the library writes only the outputs it is given
 *     (engine/model/loom_prefill.hpp:647-657);
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); calls are stream-ordered;
 *   - shapes are runtime values (the reference bakes them per kernel, gen_gemm_tile.py:347-348);
 *   - layouts are the engine's: weights are GGUF rows [N][K / block * block bytes] as loaded from the file
 *     (engine/model/weights.hpp:140-152), activations token-major [M][ldx] f16, outputs token-major [M][ldy]
 *     (gen_gemm_tile.py:1230-1231);
 *   - K is a multiple of 256 (Q8_0 is taken 8 blocks at a time, gen_gemm_decode.py:1338-1339); a K window of
 *     longer rows starts at super-block kb_off of each row (the reference's KWIN, gen_gemm_tile.py:262-264);
 *     a row range at a full output stride is a weight pointer offset plus ldy (OSTRIDE, gen_gemm_tile.py:246-250).
 */
#ifndef YAH_QGEMM_H_
#define YAH_QGEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; exactly the functions declared here are exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes (the reference throws LoomError, engine/model/loom_runtime.hpp:25-40). */
#define YAH_OK 0
#define YAH_ERR_ARG 1         /* null pointer, bad shape, misaligned pointer or stride */
#define YAH_ERR_UNSUPPORTED 2 /* format / dtype / epilogue / layout the kernels do not cover */
#define YAH_ERR_SIZE 3        /* a buffer is smaller than the operation's footprint */
#define YAH_ERR_CUDA 4        /* a CUDA runtime or driver call failed */
#define YAH_ERR_DEVICE 5      /* no sm_100 device, or a kernel reported a bounded-wait timeout */
#define YAH_ERR_NCCL 6        /* a collective failed (tensor-parallel layer) */
#define YAH_ERR_IO 7          /* a file could not be opened or mapped, or is not a well-formed GGUF file */

/* GGML type ids (engine/core/gguf.hpp GgmlType). Q8_0, Q4_K and Q6_K are the benchmark configurations' formats;
 * Q3_K, Q5_K and IQ4_XS (the reference's FMTS entries q3k / q5k / iq4xs, gen_gemm_decode.py:1707-1727) run on the
 * same kernels. Weight rows must start 16-byte aligned: Q3_K rows when their super-block count is a multiple of 8,
 * IQ4_XS rows when it is even (as Q6_K rows, a multiple of 8), Q5_K / Q4_K / Q8_0 rows always. */
#define YAH_Q8_0 8
#define YAH_Q3_K 11
#define YAH_Q4_K 12
#define YAH_Q5_K 13
#define YAH_Q6_K 14
#define YAH_IQ4_XS 23

/* Element types of activations / outputs. */
#define YAH_F32 0
#define YAH_F16 1

/* Epilogues: the reference kernel kinds (gen_gemm_tile.py:309-322, gen_gemv.py:16-19). */
#define YAH_EPI_STORE 0  /* kstore / plain:  y = W x                                  */
#define YAH_EPI_RESID 1  /* kres / resid:    y = aux + W x   (aux, y f32; y may be aux) */
#define YAH_EPI_SWIGLU 2 /* swiglu:          y = silu(aux) * W x   (aux f32 gate; tile GEMM: y f16,
                          * decode GEMV: y f32 or f16)                                                   */

/* ---- library ----------------------------------------------------------------------------------------- */
const char* yah_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char* yah_last_error(void);

/* ---- format traits (engine/core/gguf.hpp:49-50 BlockElements / BlockBytes, gguf.cpp:27-35) ------------- */
int yah_block_elements(int ggml_type);
int yah_block_bytes(int ggml_type);
/* Bytes of one row of K values; -1 if K is not a whole number of blocks or the type is unsupported. */
int64_t yah_row_bytes(int ggml_type, int64_t K);

/* ---- device runtime (LoomDevice Allocate / H2D / D2H / Synchronize, loom_runtime.hpp:153-325) -------- */
int yah_device_count(int* count);
int yah_set_device(int device);
int yah_get_device(int* device);
/* sm count, compute capability and global memory of a device. */
int yah_device_info(int device, int* sm_count, int* cc_major, int* cc_minor, int64_t* total_mem);
int yah_malloc(void** ptr, size_t bytes);
int yah_free(void* ptr);
/* Page-locked host memory (for host<->device copies that overlap and run at full PCIe rate). */
int yah_host_alloc(void** ptr, size_t bytes);
int yah_host_free(void* ptr);
int yah_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int yah_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int yah_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int yah_memset(void* ptr, int value, size_t bytes, void* stream);
int yah_stream_create(void** stream);
int yah_stream_destroy(void* stream);
int yah_stream_synchronize(void* stream);
int yah_device_synchronize(void);
int yah_event_create(void** event);
int yah_event_destroy(void* event);
int yah_event_record(void* event, void* stream);
int yah_event_synchronize(void* event);
int yah_event_elapsed_ms(void* start, void* end, float* ms);
/* CUDA graphs of library calls (decode loops are launch-bound): capture on a non-default stream (thread-local
 * mode; make every call once before capturing it, so that its scratch is already allocated), instantiate, launch. */
int yah_stream_begin_capture(void* stream);
int yah_stream_end_capture(void* stream, void** graph_exec);
int yah_graph_launch(void* graph_exec, void* stream);
int yah_graph_destroy(void* graph_exec);
/* Row realignment at load time. TMA copies need 16-byte aligned row starts, but a GGUF tensor's rows are packed:
 * Q6_K rows of K = 5120 (the reference's lm head, yah_gemv_q6k_f32.loom:1-16) are 4200 bytes. A loader copies such a
 * tensor once into rows `dst_stride` bytes apart (a multiple of 16, >= row_bytes; e.g. 4208) and passes that stride
 * as w_row_stride; the blocks inside a row are untouched. Stream-ordered device-to-device copy; dst 16-byte aligned.
 * Replaces: the byte-offset tensor view of the reference loader (engine/model/weights.hpp:142-152), which needs no
 * alignment on its hardware. */
int yah_realign_rows(const void* src, int64_t rows, int64_t row_bytes, int64_t src_stride, void* dst,
                     int64_t dst_stride, void* stream);
/* Programmatic dependent launch of the decode GEMV (on by default). A GEMV launch may then begin while the kernel
 * before it on the stream is finishing: it streams its weight tensor early and reads its activations, and writes
 * its outputs, only after that kernel has completed. Contract: no kernel still in flight on the stream writes the
 * weight tensor (weights are loaded, then only read). yah_set_launch_overlap(0) restores plain stream order. */
int yah_set_launch_overlap(int on);
/* SMs the GEMM and GEMV launches may use on each device (0, the default: all). A caller that runs collectives
 * concurrently with these kernels (the tensor-parallel stack overlaps its allreduces with the next token chunk's
 * GEMMs) leaves the remaining SMs to the collectives' kernels, which otherwise wait for a persistent GEMM to end. */
int yah_set_sm_budget(int sms);
/* Self-test of the failure path (no counterpart in the reference): a one-warp kernel waits on an mbarrier that
 * nothing arrives on, through the same bounded wait every kernel here uses, with a budget of `budget_cycles` SM
 * cycles (1000 .. 2^31). The wait runs out, the kernel records its code in the device status word and returns; the
 * call synchronises, reports the code (1 = a consumer's wait for data ran out) and clears the word. The device
 * stays usable: no trap, no fault. */
int yah_selftest_bounded_wait(int64_t budget_cycles, int* code);
/* Make `stream` wait for the last work recorded on `event` (cudaStreamWaitEvent). */
int yah_stream_wait_event(void* stream, void* event);
/* Read and clear the current device's kernel status word: 0, or the code of a bounded wait that ran out
 * (1 data wait, 2 free-stage wait, 3 exit drain, 4 a wait for another GPU's signal). A non-zero word means the
 * output of that launch is invalid.
 * The read is a blocking copy on the legacy default stream, which does not wait for work on streams created with
 * cudaStreamNonBlocking (yah_stream_create makes such streams): synchronise the stream the kernels ran on first.
 * When the word is non-zero the call also resets the GEMV's split-K arrival counters, which a CTA that left early
 * may have left partly counted (it synchronises the device to do so); later calls then start from a clean state.
 * The library keeps per-device state (this word, workspaces, the noalloc scratch address) for the life of the
 * process: do not use it across cudaDeviceReset. */
int yah_status_word(int* code);

/* ---- kernels ------------------------------------------------------------------------------------------ */

/* Footprints in bytes of the buffers a yah_qgemm / yah_qgemv call touches (the reference's bounds gate,
 * engine/gpu/loom/tools/footprint_gate.py:57-79 and gen_gemv.py:856-862); callers that know their buffer sizes
 * refuse a call whose buffer is smaller (as engine/run/hal_run.cc:107-111 does). */
int yah_qgemm_footprint(int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off, int64_t M,
                        int64_t ldx, int y_dtype, int64_t ldy, int64_t* w_bytes, int64_t* x_bytes, int64_t* y_bytes);

/* Launch limits of the tile GEMM on the current device: SMs, and the 2-CTA clusters that can be resident at
 * once (0 when the device offers no clusters; the tuner's search space, engine/tune/tune.py:77). */
int yah_qgemm_limits(int* sm_count, int* max_pairs);

/* Dequantise rows x K values of a GGUF weight to f16 out[rows][ldo] with the tile GEMM's own decode,
 * bit-identical to the reference dequant (gen_gemm_tile.py kind "dequant", :314-327; checked as
 * dq_bfp16_check.py:87-92). w: rows at w_row_stride bytes (2-byte aligned), K window from super-block kb_off.
 * out: 16-byte aligned, ldo a multiple of 8. */
int yah_dequant(const void* w, int ggml_type, int64_t rows, int64_t K, int64_t w_row_stride, int64_t kb_off,
                void* out, int64_t ldo, void* stream);

/* Tile GEMM (prefill): y[M][ldy] = epilogue(x[M][ldx] * W[N][K]^T), f32 accumulation.
 * Replaces the yah_ffn_gemm_<fmt>[_kres|_swiglu] kernels (gen_gemm_tile.py:221-238, :309-322) and their
 * dispatch sites LoomPrefill::RunKstore / RunResidual / RunSwiglu (engine/model/loom_prefill.hpp:1954-2110).
 *   w        weight rows, 16-byte aligned, w_row_stride a multiple of 16 bytes (Q6_K: K window rows of a
 *            multiple of 8 super-blocks, or padded rows);
 *   x        f16 activations, 16-byte aligned, ldx >= K and a multiple of 8;
 *   y        output; y_dtype YAH_F32 or YAH_F16 (YAH_EPI_RESID: f32; YAH_EPI_SWIGLU: f16); ldy >= N;
 *   aux      f32 [M][ldaux] residual (YAH_EPI_RESID) or gate (YAH_EPI_SWIGLU), else NULL. */
int yah_qgemm(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
              const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
              const void* aux, int64_t ldaux, void* stream);

/* yah_qgemm with an explicit tile choice (the tuner's knob set, engine/tune/tune.py:77):
 *   bn      tokens per tile: 256, 160 or 128 for 2-SM pairs, 192, 128 or 64 for single CTAs (0 = auto:
 *           256, or 160 when accumulating in chunks, for pairs; 192 for single CTAs);
 *   grid    persistent CTAs (0 = one per SM);
 *   kchunk  K per f32 accumulation chunk, a multiple of 128 (0 = auto: 2048 when K > 4096, else all of K;
 *           -1 = never chunk). Chunk results are summed in f32 round-to-nearest; see the accuracy note in
 *           csrc/qgemm_tc.cu. Chunking uses a library-owned per-device scratch buffer (grid * bn * 512 bytes),
 *           so chunked calls on different streams of one device must not overlap;
 *   cta_pair  1: 2-SM pairs (256 weight rows per tile, tcgen05 cta_group::2 over clusters of 2 CTAs),
 *           0: one CTA per 128-row tile, -1: auto (pairs where the device supports clusters).
 * Split K: with grid = 0, chunked accumulation (kchunk a multiple of 256) and fewer (row tile, 16-token unit)
 * pieces than the device holds CTAs (pairs), every accumulation chunk of a tile runs on its own CTA and the chunk
 * results are added in chunk order by a second kernel that also applies the epilogue (a library-owned per-device
 * workspace of chunks * M * N * 4 bytes, same stream rule as the scratch). An explicit grid never splits.
 * Every (bn, grid, cta_pair) choice, split or not, gives identical results for a given kchunk. */
int yah_qgemm_tile(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                   const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                   const void* aux, int64_t ldaux, int bn, int grid, int64_t kchunk, int cta_pair, void* stream);

/* Caller-owned workspace (no counterpart in the reference, whose kernels need none: its GEMMs never split K). The
 * library-owned buffers of yah_qgemm / yah_qgemm_tile / yah_qgemv are shared by every call on a device; these
 * variants take the workspace from the caller instead, so calls on different streams with different workspaces
 * may overlap, and the call itself never allocates device memory.
 * yah_qgemm_workspace_size: the bytes yah_qgemm_ws needs for (type, N, K, M, y_dtype, epilogue) and a tile choice
 * (bn, grid, kchunk, cta_pair as in yah_qgemm_tile; 0 / -1 for the automatic ones); 0 when the call needs none
 * (no chunked accumulation). yah_qgemm_ws: yah_qgemm_tile on that workspace (256-byte aligned, at least the queried
 * size; NULL allowed when the size is 0; too small: YAH_ERR_SIZE). Same results, bit for bit, as yah_qgemm_tile
 * with the same arguments. The workspace holds no state between calls. */
int yah_qgemm_workspace_size(int ggml_type, int64_t N, int64_t K, int64_t M, int y_dtype, int epilogue, int bn,
                             int grid, int64_t kchunk, int cta_pair, size_t* bytes);
int yah_qgemm_ws(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                 const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                 const void* aux, int64_t ldaux, int bn, int grid, int64_t kchunk, int cta_pair, void* workspace,
                 size_t workspace_bytes, void* stream);

/* The fused gate+up SwiGLU of the feed-forward block (the reference's ffn kind, gen_gemm_tile.py:316-318, :1675):
 * y[M][ldy] = f16(silu(x W_gate^T) * (x W_up^T)), both weight tensors of the same type, shape and row stride. One
 * tile GEMM: each CTA decodes 64 gate rows and the same 64 up rows into its 128 TMEM lanes and its epilogue
 * combines them, so the f32 gate tensor never goes through memory. Results are identical to yah_qgemm of the gate
 * (f32 out) followed by yah_qgemm of the up weights with YAH_EPI_SWIGLU on that gate, for the same accumulation
 * chunks (2048 when K > 4096, else none). bn / cta_pair as in yah_qgemm_tile (0 / -1 = automatic: single CTAs,
 * 192 tokens). */
int yah_qgemm_ffn(const void* w_gate, const void* w_up, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride,
                  int64_t kb_off, const void* x, int64_t M, int64_t ldx, void* y, int64_t ldy, int bn, int cta_pair,
                  void* stream);

/* Tile table (opt-in): tuned tiles for yah_qgemm's automatic choice, the counterpart of the reference's tuned
 * tables consumed by LoomPrefill::PickGemm (engine/model/loom_prefill.hpp:908-949; engine/tune/tune.py). A call
 * (ggml_type, epilogue, y_dtype, N, K, M) uses the matching rule with the smallest m_max >= M (else the largest
 * m_max); bn / grid / cta_pair as in yah_qgemm_tile. Tiles never change results (same accumulation chunks). The
 * table is process-wide; yah_tile_rules_set replaces it. */
typedef struct {
  int ggml_type, epilogue, y_dtype;
  int64_t N, K, m_max;
  int bn, grid, cta_pair;
} yah_tile_rule;
int yah_tile_rules_set(const yah_tile_rule* rules, int n);
int yah_tile_rules_clear(void);
int yah_tile_rules_count(int* n);

/* Decode GEMV, 1 <= M <= 32 tokens (replaces gen_gemv.py's gv_{plain,resid,swiglu}_<fmt>_<M>_<K> kernels and the
 * LoomDecoder::Gemv call site, engine/model/loom_decoder.hpp:415-439). Same layouts and alignment rules as
 * yah_qgemm; epilogue YAH_EPI_STORE, YAH_EPI_RESID, or YAH_EPI_SWIGLU (y = silu(aux) * W x with y f32 or f16; aux
 * may be y itself when y is f32: each gate value is read before it is overwritten). Computes with the f32 weight
 * values of the GGUF dequant, as the reference GEMV does (no f16 rounding of weights). Results are deterministic.
 * Two kernels: an mma.sync kernel, and for Q4_K with more than 8 tokens whose activations are too many to keep in
 * shared memory (the mma.sync kernel would then run stream-K) a tcgen05 kernel (thread-block clusters split K and
 * add their partial sums in distributed shared memory; no scratch). The mma.sync kernel's stream-K form sums the row
 * blocks shared by two CTAs through a library-owned per-device workspace (allocated on first use, grown on demand),
 * so concurrent calls on different streams of one device must not overlap. */
int yah_qgemv(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
              const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
              const void* aux, int64_t ldaux, void* stream);

/* yah_qgemv with the activations' element type chosen (x_dtype YAH_F16 or YAH_F32). The reference GEMV binds
 * x f32[K] and y f32 (gen_gemv.py:4, :729; LoomDecoder::Gemv, engine/model/loom_decoder.hpp:432-434): with
 * YAH_F32 this is that binding, with no conversion step. Each f32 value is split in the kernel's activation load
 * into hi = f16(x) and lo = f16(x - hi) (22 significant bits; values need |x| < 65504), both multiplied with the
 * f32 weight values and the two products added, so results stay within the reference checker's bar
 * (max |y - ref| / max |ref| <= 1e-4, gemv_check.py:176-183). f32 activations always run the mma.sync kernel in
 * its row-range form with the activations resident in shared memory (no workspace); tokens beyond what fits run
 * as further launches (Q4_K at K = 14336: 2 tokens per launch). ldx counts elements of x_dtype. */
int yah_qgemv_x(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                const void* x, int x_dtype, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                const void* aux, int64_t ldaux, void* stream);
/* yah_qgemv_swiglu with the activations' element type chosen, as yah_qgemv_x. */
int yah_qgemv_swiglu_x(const void* w_gate, int gate_type, int64_t gate_row_stride, const void* w_up, int up_type,
                       int64_t up_row_stride, int64_t N, int64_t K, const void* x, int x_dtype, int64_t M,
                       int64_t ldx, float* y, int64_t ldy, void* stream);

/* yah_qgemv on a caller-owned workspace (see yah_qgemm_ws): yah_qgemv_workspace_size gives the bytes for (type, N,
 * K, M) under the current kernel choice (yah_set_gemv_impl), 0 where the chosen form needs none (the tcgen05
 * kernel and the row-range forms of the mma.sync kernel). yah_qgemv_ws clears the workspace's split counters on
 * `stream` before its launch, so the workspace holds no state between calls. Same results, bit for bit, as
 * yah_qgemv. */
int yah_qgemv_workspace_size(int ggml_type, int64_t N, int64_t K, int64_t M, size_t* bytes);
int yah_qgemv_ws(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                 const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                 const void* aux, int64_t ldaux, void* workspace, size_t workspace_bytes, void* stream);

/* The reference GEMV's swiglu kind (gen_gemv.py:18, :97-98; called per layer at engine/model/loom_decoder.hpp:294):
 * y[M][ldy] (f32) = silu(x W_gate^T) * (x W_up^T). The two weight tensors may differ in format and row stride (same
 * N and K). Runs the gate GEMV into y, then the up GEMV with the swiglu kind over y in place: no other memory. */
int yah_qgemv_swiglu(const void* w_gate, int gate_type, int64_t gate_row_stride, const void* w_up, int up_type,
                     int64_t up_row_stride, int64_t N, int64_t K, const void* x, int64_t M, int64_t ldx, float* y,
                     int64_t ldy, void* stream);

/* Which decode GEMV kernel yah_qgemv and yah_qgemv_noalloc run (process-wide; for tests and measurements, no
 * counterpart in the reference): 0 (default) the tcgen05 kernel for Q4_K above 8 tokens where the mma.sync kernel
 * would run stream-K, else the mma.sync kernel;
 * 1 only the tcgen05 kernel (calls it does not cover fail with YAH_ERR_UNSUPPORTED); 2 only the mma.sync kernel. */
int yah_set_gemv_impl(int impl);
/* Which kernel and work split yah_qgemv would use on the current device for (type, N, K, M), as text (no
 * counterpart in the reference; for logs and measurements). */
int yah_qgemv_describe(int ggml_type, int64_t N, int64_t K, int64_t M, char* buf, int64_t cap);

/* Decode GEMV that allocates nothing. This entry point has no counterpart in the reference engine.
 * For callers that cannot call cudaMalloc when they run the GEMV: code inside a CUDA-graph capture region, a
 * decode loop with a fixed device-memory budget, or a host process whose device allocator belongs to another
 * framework. Same arguments, layouts and results as yah_qgemv; the difference is where the split-K scratch
 * lives: a fixed 8 MiB + 128 KiB device array inside this library (every GPU that loads the library holds it
 * until the process exits), holding the partial sums (at most 2^21 floats: 2 x tokens x 128 per CTA), eight
 * counters per 128-row block (N <= 524288) and the variant's own status word. A call whose scratch would exceed
 * that is refused with YAH_ERR_SIZE (1..32 tokens always fit on devices of up to 256 SMs).
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
 * current); make that first call before any stream capture. Every call shares the one array and leaves the last
 * call's contents in it (each call clears the counters it uses first), so calls whose executions overlap on the
 * GPU (different streams, or different host threads on one device) race: serialise them. */
int yah_qgemv_noalloc(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                      const void* x, int64_t M, int64_t ldx, void* y, int y_dtype, int64_t ldy, int epilogue,
                      const void* aux, int64_t ldaux, void* stream);
/* Read and clear the status word of yah_qgemv_noalloc on the current device (same codes as yah_status_word). */
int yah_qgemv_noalloc_status(int* code);

/* ------------------------------------------------------------------ tensor-parallel layer (NCCL over NVLink)
 * The reference engine runs on one GPU and has no counterpart; this is the sharding layer the B200 build adds for
 * the Llama-shaped stack (one process per GPU). Column-parallel linears (QKV, gate, up) use a row range of the GGUF
 * tensor and need no collective; row-parallel linears (o_proj, down) use a K window of whole super-blocks and end
 * in one ncclAllReduce(sum) of f32 partials. NCCL is loaded at run time (libnccl.so.2). */
#define YAH_TP_ID_BYTES 128
typedef struct yah_tp_comm yah_tp_comm;

/* 1 when NCCL could be loaded, else 0. */
int yah_tp_available(void);
/* A new NCCL unique id (YAH_TP_ID_BYTES bytes) for yah_tp_init; create it on one rank and share it. */
int yah_tp_unique_id(void* id);
/* Join a communicator of nranks processes as `rank`, on the current device. */
int yah_tp_init(yah_tp_comm** comm, int nranks, int rank, const void* id);
int yah_tp_destroy(yah_tp_comm* comm);
int yah_tp_rank(const yah_tp_comm* comm, int* rank, int* nranks);
/* In-place sum of an f32 device buffer over the ranks, on `stream`. */
int yah_tp_allreduce_f32(yah_tp_comm* comm, float* buf, int64_t count, void* stream);
/* Column-parallel linear: y[M][N_local] = x W_shard^T for this rank's row range (w_shard points at its first row);
 * same arguments as yah_qgemm (yah_qgemv for M <= 32). No collective. */
int yah_tp_linear_col(yah_tp_comm* comm, const void* w_shard, int ggml_type, int64_t N_local, int64_t K,
                      int64_t w_row_stride, const void* x, int64_t M, int64_t ldx, void* y, int y_dtype,
                      int64_t ldy, int epilogue, const void* aux, int64_t ldaux, void* stream);
/* Row-parallel linear: this rank's K window (K_local values from super-block kb_off of rows of w_row_stride bytes)
 * times its x slice [M][K_local]; y (f32, contiguous [M][N]) becomes resid + sum over ranks of the partials,
 * on every rank (rank 0 adds resid in its GEMM epilogue; resid may be y; NULL adds nothing). */
int yah_tp_linear_row(yah_tp_comm* comm, const void* w_shard, int ggml_type, int64_t N, int64_t K_local,
                      int64_t w_row_stride, int64_t kb_off, const void* x, int64_t M, int64_t ldx, float* y,
                      const float* resid, void* stream);
/* RMSNorm of the f32 residual stream into f16: out[m][i] = h[m][i] * gain / sqrt(mean_i h[m][i]^2 + eps). The
 * layer stack's norm before QKV and gate/up (the reference normalises every layer input, docs/architecture.md:68);
 * weightless, with one gain (H and strides multiples of 4, h 16-byte and out 8-byte aligned). */
int yah_rmsnorm(const float* h, int64_t ldh, int64_t M, int64_t H, float eps, float gain, void* out, int64_t ldo,
                void* stream);
/* The residual update of the row-parallel linears: h += d (d [M][ldd] of d_dtype YAH_F16 or YAH_F32, the allreduced
 * partial sums, added in f32 and stored back to h), then, when out is not null, out = f16 RMSNorm of the new h as
 * yah_rmsnorm. One pass over h instead of an add kernel and a norm kernel. */
int yah_add_rmsnorm(float* h, int64_t ldh, const void* d, int d_dtype, int64_t ldd, int64_t M, int64_t H, float eps,
                    float gain, void* out, int64_t ldo, void* stream);
/* ncclAllReduce(sum) of f16 in place (the speed mode's partials: half the bytes of yah_tp_allreduce_f32). */
int yah_tp_allreduce_f16(yah_tp_comm* comm, void* buf, int64_t count, void* stream);
/* ncclAllGather of count f32 from every rank into recv ([nranks][count]). */
int yah_tp_allgather_f32(yah_tp_comm* comm, const float* send, float* recv, int64_t count, void* stream);

/* ---- fused row-parallel reduce over peer memory (no counterpart in the single-GPU reference) ----
 * The row-parallel linear's reduction written by its own GEMM: rank q's f32 partial of token t is stored by the
 * GEMM's epilogue straight into the memory of the rank owning t (tokens split into nranks equal slices), over
 * NVLink, so the transfer overlaps the GEMM tile by tile; the owner adds the nranks slots of its slice in rank order
 * into its slice of the residual stream and writes the RMSNorm of it (f16) into every rank's activation buffer.
 * Cross-GPU order uses flags in each rank's memory (release / acquire at system scope, epochs that only grow);
 * every wait is bounded (2 s, then code 4 in the status word). Plain stores and flags: no multicast.
 *
 * yah_qgemm_sliced: yah_qgemm (plain store, f32) with output token t written to ys[t / slice_rows] + (t % slice_rows)
 * * ldy (1..8 slices, slice_rows a multiple of 16; the slices may be other GPUs' memory).
 * yah_tp_peers_create: device buffers of this rank (any device pointers; the allocations are shared through CUDA
 * IPC, exchanged with one ncclAllGather) and the same buffers of every other rank as addresses usable here;
 * yah_tp_peers_ptr gives buffer b of rank r. Collective: every rank calls it with the same nbufs.
 * yah_tp_signal: after the preceding work on `stream`, int slot `slot` of buffer flag_buf on every rank := value.
 * yah_tp_wait: later work on `stream` waits until this rank's ints [first, first + count) of flag_buf are >= value.
 * yah_tp_reduce_norm: for rows r < rows of this rank's slice: h[r] += parts[0][r] + ... + parts[nparts-1][r]
 * (slots part_stride floats apart, rows ldp apart; nparts 0: no add); then, unless out_buf < 0,
 * f16(h[r] * gain / sqrt(mean(h[r]^2) + eps)) at row out_row0 + r (stride ldo) of buffer out_buf on every rank.
 * yah_tp_linear_row_scatter: the row-parallel GEMM of this rank's K window with its partials scattered as above
 * into slot `rank` of buffer recv_buf ([nranks][M / nranks][N] f32) on every rank; M must split into nranks slices
 * of a multiple of 16 tokens. */
typedef struct yah_tp_peers yah_tp_peers;
int yah_qgemm_sliced(const void* w, int ggml_type, int64_t N, int64_t K, int64_t w_row_stride, int64_t kb_off,
                     const void* x, int64_t M, int64_t ldx, void* const* ys, int nslices, int64_t slice_rows,
                     int64_t ldy, void* stream);
int yah_tp_peers_create(yah_tp_comm* comm, void* const* bufs, int nbufs, void* stream, yah_tp_peers** out);
int yah_tp_peers_ptr(const yah_tp_peers* pe, int rank, int buf, void** ptr);
int yah_tp_peers_destroy(yah_tp_peers* pe);
int yah_tp_signal(const yah_tp_peers* pe, int flag_buf, int slot, int value, void* stream);
int yah_tp_wait(const yah_tp_peers* pe, int flag_buf, int first, int count, int value, void* stream);
/* yah_tp_signal of slot base + rank followed by yah_tp_wait on [base, base + nranks), in one launch. */
int yah_tp_barrier(const yah_tp_peers* pe, int flag_buf, int base, int value, void* stream);
int yah_tp_reduce_norm(const yah_tp_peers* pe, float* h, int64_t ldh, int64_t rows, int64_t H, const float* parts,
                       int nparts, int64_t part_stride, int64_t ldp, float eps, float gain, int out_buf,
                       int64_t out_row0, int64_t ldo, void* stream);
int yah_tp_linear_row_scatter(const yah_tp_peers* pe, const void* w_shard, int ggml_type, int64_t N,
                              int64_t K_local, int64_t w_row_stride, int64_t kb_off, const void* x, int64_t M,
                              int64_t ldx, int recv_buf, void* stream);

/* ---- GGUF files: the quant-block loader (engine/core/gguf.hpp:74-105 core::Gguf, engine/core/gguf.cpp) ----
 * yah_gguf_open maps a GGUF (version 2 or 3) file read-only and parses its metadata and tensor table; the tensor
 * bytes are not copied. Every read is bounds-checked: a truncated or malformed file is refused with YAH_ERR_IO, a
 * tensor type of unknown block size with YAH_ERR_UNSUPPORTED. Tensors are described as the reference's TensorRef
 * (engine/model/weights.hpp:15-25): dims in GGUF order, dims[0] = ne0 = the row length (K of a linear weight),
 * dims[1] = ne1 = the row count (N); `offset` is from the start of the tensor-data region (aligned to
 * general.alignment, default 32). A weight tensor's rows are then exactly the layout the GEMM / GEMV take. */
typedef struct yah_gguf yah_gguf;
typedef struct {
  char name[128];   /* NUL-terminated (GGUF names of up to 127 bytes) */
  int ggml_type;
  int n_dims;       /* 1..4; unused dims are 1 */
  int64_t dims[4];
  uint64_t offset;  /* bytes from the start of the tensor-data region */
  uint64_t bytes;   /* dims product / block elements * block bytes */
} yah_gguf_tensor;
int yah_gguf_open(const char* path, yah_gguf** out);
int yah_gguf_close(yah_gguf* g);
int yah_gguf_version(const yah_gguf* g, uint32_t* version);
int yah_gguf_tensor_count(const yah_gguf* g, int64_t* n);
int yah_gguf_tensor_info(const yah_gguf* g, int64_t index, yah_gguf_tensor* out);
/* index of the tensor called `name` (core::Gguf::Find); YAH_ERR_ARG and index -1 when there is none. */
int yah_gguf_find(const yah_gguf* g, const char* name, int64_t* index);
/* host view of the tensor-data region (core::Gguf::tensor_data_base / tensor_data_size). */
int yah_gguf_data(const yah_gguf* g, const void** base, uint64_t* bytes);
/* Metadata (core::Gguf::Meta): the GGUF value kind of `key` (0 u8, 1 i8, 2 u16, 3 i16, 4 u32, 5 i32, 6 f32,
 * 7 bool, 8 string, 9 array, 10 u64, 11 i64, 12 f64) and, for arrays, the element count (1 otherwise); the value of
 * an integer or bool key (signed keys sign-extended, u64 keys as their two's complement bits); of a numeric key as a
 * double; of a string key (copied NUL-terminated into buf of cap bytes, truncated to fit; *len = its full length). */
int yah_gguf_meta_kind(const yah_gguf* g, const char* key, int* kind, uint64_t* count);
int yah_gguf_meta_int(const yah_gguf* g, const char* key, int64_t* value);
int yah_gguf_meta_float(const yah_gguf* g, const char* key, double* value);
int yah_gguf_meta_string(const yah_gguf* g, const char* key, char* buf, int64_t cap, int64_t* len);

/* Device copies of the tensor-data region (LoomWeights, engine/model/loom_runtime.hpp:487-516): device buffers of
 * at most chunk_bytes (0 = 1 GiB, a single larger tensor gets a chunk of its own) cut at tensor boundaries, each
 * followed by 64 KB of zeros, on the current device; the copy is complete when the call returns. yah_weights_ref
 * returns the device address of [offset, offset + bytes) of the region (a tensor's offset and bytes), which must lie
 * in one chunk: the tensor's rows as the GEMM / GEMV take them, no repacking. */
typedef struct yah_weights yah_weights;
int yah_weights_upload(const yah_gguf* g, uint64_t chunk_bytes, void* stream, yah_weights** out);
int yah_weights_ref(const yah_weights* w, uint64_t offset, uint64_t bytes, const void** dev);
int yah_weights_chunk_count(const yah_weights* w, int64_t* n);
int yah_weights_free(yah_weights* w);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* YAH_QGEMM_H_ */
