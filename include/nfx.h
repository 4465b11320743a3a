/*
 * nfx.h -- C-ABI of the B200 (sm_100a) quantized neural-operator inference library
 * (libnfx.so).  Plain pointers, sizes and status codes; no C++ or torch types.
 *
 * Every entry point replaces one interface of the reference NeuroFlow C++ runtime
 * (AITree69/neuroflow, paths relative to that project) and is cited beside it.  The
 * return value of every int-returning function is a reference StatusCode
 * (cpp/include/neuroflow/tensor.h:29-37): 0 Ok, 1 InvalidArg, 2 FileNotFound,
 * 3 ParseError, 4 ShapeMismatch, 5 UnsupportedOp, 99 Internal (CUDA failures and
 * device-side timeouts are reported as Internal with a message).
 *
 * Threading: a runtime handle is single-threaded, like the reference runtime
 * (cpp/include/neuroflow/fno.h:192-209).  Different handles may be used from
 * different threads.  Each handle is bound to one CUDA device chosen at creation.
 */
#ifndef NFX_H_
#define NFX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    NFX_OK = 0,
    NFX_INVALID_ARG = 1,
    NFX_FILE_NOT_FOUND = 2,
    NFX_PARSE_ERROR = 3,
    NFX_SHAPE_MISMATCH = 4,
    NFX_UNSUPPORTED_OP = 5,
    NFX_INTERNAL = 99
};

typedef struct nfx_runtime nfx_runtime;

/* ---- InferenceRuntime (cpp/include/neuroflow/runtime.h:69-135) ---------------- */

/* InferenceRuntime::Create (runtime.h:72-74, runtime.cpp:79-83): load a NeuroIR v0
 * binary (.nneuroir, with the optional NIRQ block) and upload the weights to
 * `device`.  On failure *out is NULL and nfx_last_error() holds the message. */
int nfx_runtime_create(const char* ir_path, int device, nfx_runtime** out);

/* LoadNeuroIr (runtime.h:66, runtime.cpp:16-19): parse a NeuroIR v0 binary on the
 * host only (no device work).  Writes the op name (NUL-terminated, truncated to
 * op_cap), the 8-int32 config block (unused slots 0), the number of weight tensors
 * read, and whether a NIRQ block was present.  Any output pointer may be NULL. */
int nfx_load_neuroir(const char* ir_path, char* op_out, int op_cap, int32_t* cfg_out8,
                     int* n_weights_out, int* quant_enabled_out);

/* Destructor of InferenceRuntime. */
void nfx_runtime_destroy(nfx_runtime* rt);

/* InferenceRuntime::op (runtime.h:114): "FNO1d", "FNO2d", ... */
const char* nfx_runtime_op(const nfx_runtime* rt);

/* InferenceRuntime::EnableInt8Gemm (runtime.h:116-124, runtime.cpp:155-166).  FNO1d:
 * the reference's semantics (the flag is set; layers whose input key has per-tensor
 * qparams and whose weight has per-channel qparams run through the INT8 GEMM).  On
 * this runtime it also enables INT8 executors the reference does not have: FNO2d
 * (with a NIRQ block: each layer input snapped with its key's per-tensor qparams, and
 * locs.i / proj_q through the INT8 GEMM where the weight has per-channel qparams and
 * the input key per-tensor ones) and TokenMixer2D / TokenMixer (per-channel weight
 * qparams of q/k/v/o/ffn0/ffn1, per-token activation qparams computed at run time);
 * without those qparams it is a no-op like the reference. */
void nfx_runtime_enable_int8_gemm(nfx_runtime* rt);

/* InferenceRuntime::IsInt8GemmEnabled (runtime.h:126-128). */
int nfx_runtime_is_int8_gemm_enabled(const nfx_runtime* rt);

/* Enable the FP8 E4M3 executor of FNO3d (per-tensor E4M3 weights, E4M3 activation codes
 * between layers, E4M3 fake-quant at the ".output" boundaries; the scales are the
 * NIRQ kind-3 entries of every Linear weight and ".output" key).  No counterpart in
 * the reference (its FNO3d has no quantised path; the switch mirrors EnableInt8Gemm and
 * is likewise a no-op when the IR lacks the scales). */
void nfx_runtime_enable_fp8(nfx_runtime* rt);
int nfx_runtime_is_fp8_enabled(const nfx_runtime* rt);

/* InferenceRuntime::Run (runtime.h:76-79, runtime.cpp:85-101).  x and y are HOST
 * float32 row-major buffers owned by the caller; shapes as the reference's
 * FNO*::Forward checks them (batch first, channels last).  Synchronous. */
int nfx_runtime_run(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                    float* y, const int64_t* y_shape, int y_rank);

/* Device-resident variant of Run: x and y are DEVICE pointers on the runtime's device;
 * the work is enqueued on `stream` (a cudaStream_t, NULL = legacy default stream)
 * and the call returns without synchronising.  Device-side errors surface at the
 * next nfx_runtime_check() or synchronous call.  No counterpart in the reference
 * (its runtime is host-only); it is the timing/multi-GPU entry of the same work. */
int nfx_runtime_run_device(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                           int x_rank, float* y, const int64_t* y_shape, int y_rank,
                           void* stream);

/* InferenceRuntime::RunTokenMixer2D (runtime.h:98-99, runtime.cpp:135-143): x
 * (batch, h, w, in_dim) -> y (batch, h, w, out_dim), HOST buffers, synchronous.  On a
 * runtime whose op is not TokenMixer2D it returns NFX_INTERNAL "TokenMixer2D not
 * initialized" as the reference does; nfx_runtime_run on a TokenMixer2D runtime returns
 * NFX_INTERNAL "runtime does not support op" (runtime.cpp:97-100). */
int nfx_runtime_run_tokenmixer2d(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                                 int x_rank, float* y, const int64_t* y_shape, int y_rank);

/* Device-resident variant of nfx_runtime_run_tokenmixer2d (asynchronous on `stream`,
 * like nfx_runtime_run_device).  No counterpart in the reference. */
int nfx_runtime_run_tokenmixer2d_device(nfx_runtime* rt, const float* x,
                                        const int64_t* x_shape, int x_rank, float* y,
                                        const int64_t* y_shape, int y_rank, void* stream);

/* InferenceRuntime::RunTokenMixer (runtime.h:88-89, runtime.cpp:115-123): the 1D
 * TokenMixer, x (batch, n_points, in_dim) -> y (batch, n_points, out_dim), HOST
 * buffers, synchronous; the TokenMixer2D executor on a 1 x n_points grid (the same
 * network, fno.cpp:1460-1644).  Another op: NFX_INTERNAL "TokenMixer not initialized". */
int nfx_runtime_run_tokenmixer(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                               int x_rank, float* y, const int64_t* y_shape, int y_rank);
int nfx_runtime_run_tokenmixer_device(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                                      int x_rank, float* y, const int64_t* y_shape, int y_rank,
                                      void* stream);

/* InferenceRuntime::RunGraphOp (runtime.h:93-94, runtime.cpp:125-133): x (batch,
 * n_nodes, in_dim) -> y (batch, n_nodes, out_dim), HOST buffers, synchronous
 * (GraphOp::Forward, fno.cpp:1653-1741).  The reference's shape checks and messages; a
 * graph whose CSR indices or offsets leave the node range (the reference reads outside
 * its buffers) returns NFX_INVALID_ARG.  Another op: NFX_INTERNAL "GraphOp not
 * initialized". */
int nfx_runtime_run_graphop(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                            float* y, const int64_t* y_shape, int y_rank);
int nfx_runtime_run_graphop_device(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                                   int x_rank, float* y, const int64_t* y_shape, int y_rank,
                                   void* stream);

/* InferenceRuntime::RunGraphOp2D (runtime.h:103-104, runtime.cpp:145-153): x (batch, h,
 * w, in_dim) -> y (batch, h, w, out_dim), as nfx_runtime_run_graphop (GraphOp2D::Forward,
 * fno.cpp:1969-2060).  Another op: NFX_INTERNAL "GraphOp2D not initialized". */
int nfx_runtime_run_graphop2d(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                              float* y, const int64_t* y_shape, int y_rank);
int nfx_runtime_run_graphop2d_device(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                                     int x_rank, float* y, const int64_t* y_shape, int y_rank,
                                     void* stream);

/* InferenceRuntime::RunDeepONet (runtime.h:82-84, runtime.cpp:103-113): u (batch,
 * n_sensor, in_branch), y (batch, n_query, in_trunk) -> out (batch, n_query,
 * out_channels), HOST buffers, synchronous (DeepONet::Forward, fno.cpp:1289-1406).  The
 * reference's shape checks and messages, plus NFX_SHAPE_MISMATCH when u and y hold
 * different batch sizes (the reference reads y with u's batch).  Layer weights whose
 * shapes disagree with the widths the loader derives give NFX_UNSUPPORTED_OP (the
 * reference reads past them).  Another op: NFX_INTERNAL "DeepONet not initialized". */
int nfx_runtime_run_deeponet(nfx_runtime* rt, const float* u, const int64_t* u_shape, int u_rank,
                             const float* y, const int64_t* y_shape, int y_rank, float* out,
                             const int64_t* out_shape, int out_rank);
int nfx_runtime_run_deeponet_device(nfx_runtime* rt, const float* u, const int64_t* u_shape,
                                    int u_rank, const float* y, const int64_t* y_shape, int y_rank,
                                    float* out, const int64_t* out_shape, int out_rank,
                                    void* stream);

/* Allocation-free variant of nfx_runtime_run_device, for callers that cannot call
 * cudaMalloc while they run inference (their device memory belongs to another
 * allocator, or allocation is forbidden or too slow on their inference path).  It
 * runs the same FNO2d INT8 kernels, with bit-identical results, but keeps all scratch
 * (activation codes, spectra, transform tables, error word) in one fixed 32 MiB device
 * array inside libnfx.so; a batch that needs more returns NFX_INVALID_ARG (2,465,792 B
 * per 128x128 sample at width 64, so at most 13 such samples per call).  With CUDA's
 * lazy module loading (the default) the 32 MiB is reserved on a device by the first
 * call there, which looks up the array's device address and uploads the transform
 * tables; it is then held until the process exits.  Make that first call at start-up
 * and before any stream capture; a call whose grid differs from the previous call's on
 * that device uploads the tables again (synchronously).  Other calls allocate nothing on
 * the device or the host.  Calls share the array: calls that overlap on the GPU race
 * and must be serialised by the caller.  x and y are device pointers; the call returns
 * after the work on `stream` has finished.  No counterpart in the reference. */
int nfx_runtime_run_device_noalloc(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                                   int x_rank, float* y, const int64_t* y_shape, int y_rank,
                                   void* stream);

/* Parity taps of the FNO2d INT8 executor: while `device_buffer` is set (NULL turns the
 * taps off), every FNO2d INT8 forward on this handle also copies the int8 activation
 * codes of each layer input -- the lift's output, then every Fourier layer's output,
 * the last being the projection's input -- into it as n_layers + 1 consecutive
 * (batch*h*w, width) channel-last blocks, on the launch stream after the kernel that
 * wrote them.  A forward whose taps do not fit in `capacity_bytes` fails with
 * NFX_INVALID_ARG.  The host-buffer Run of a large batch runs in chunks, so its taps
 * hold the last chunk only; use nfx_runtime_run_device for whole-batch taps.  No
 * counterpart in the reference runtime: it exposes, for layer-wise parity checks, the
 * activations between the iterations of FNO2d::Forward's layer loop
 * (cpp/src/fno.cpp:900-945) in their int8 form.  The FNO3d FP8 variant writes its E4M3
 * activation codes the same way, as n_layers + 1 channel-first (batch, width, h, w, d)
 * blocks on the padded grid (FNO3d::Forward's layer loop, cpp/src/fno.cpp:1182-1228);
 * an FNO3d forward without FP8 fails with NFX_UNSUPPORTED_OP while taps are set. */
int nfx_runtime_set_code_taps(nfx_runtime* rt, int8_t* device_buffer, int64_t capacity_bytes);

/* Synchronise the runtime's work and report device-side errors (bounded waits that
 * timed out inside a kernel) as NFX_INTERNAL. */
int nfx_runtime_check(nfx_runtime* rt);

/* Per-kernel device timing (tracing): when enabled, every kernel the executor launches
 * is bracketed by CUDA events recorded on its launch stream.  profile_count returns
 * the number of distinct kernels seen since enabling (waiting for the recorded events);
 * profile_entry returns a kernel's name, launch count and summed device time in ms.
 * Enabling again resets the totals.  No counterpart in the reference, whose only
 * timing is ad-hoc std::chrono in cpp/tests/bench_int8_gemm.cpp:144-178. */
int nfx_runtime_profile_enable(nfx_runtime* rt, int enable);
int nfx_runtime_profile_count(nfx_runtime* rt);
int nfx_runtime_profile_entry(nfx_runtime* rt, int index, const char** name, int* launches,
                              double* total_ms);

/* Message of the last failing call on this handle ("" when none). */
const char* nfx_runtime_last_error(const nfx_runtime* rt);

/* Message of the last failing handle-less call of this thread. */
const char* nfx_last_error(void);

/* ---- Batch partitioned across the GPUs of one node ------------------------------
 * Samples are independent, so a batch of B runs as contiguous slices of ceil(B / G)
 * samples on G GPUs with replicated weights; the only communication is moving inputs
 * to and outputs from the GPU that holds the caller's buffers (NCCL, loaded at run time
 * from libnccl.so.2 or $NFX_NCCL_LIB).  The reference runs one batch per Run on one
 * host (cpp/src/runtime.cpp:85-101); these entry points keep that call shape. */

/* The slice [first, first + count) of a batch of `batch` samples that rank `rank` of
 * `world` computes (count may be 0 for the last ranks). */
void nfx_batch_slice(int64_t batch, int world, int rank, int64_t* first, int64_t* count);

/* One process driving several GPUs: InferenceRuntime::Create (runtime.h:72-74) with a
 * device list.  Every device gets its own runtime (weights uploaded to each). */
typedef struct nfx_group nfx_group;
int nfx_group_create(const char* ir_path, const int* devices, int n_devices, nfx_group** out);
void nfx_group_destroy(nfx_group* g);
int nfx_group_size(const nfx_group* g);
/* The member runtime on the i-th listed device (owned by the group). */
nfx_runtime* nfx_group_member(nfx_group* g, int i);
const char* nfx_group_last_error(const nfx_group* g);
/* EnableInt8Gemm / IsInt8GemmEnabled / enable_fp8 on every member (runtime.h:116-128). */
void nfx_group_enable_int8_gemm(nfx_group* g);
int nfx_group_is_int8_gemm_enabled(const nfx_group* g);
void nfx_group_enable_fp8(nfx_group* g);
/* InferenceRuntime::Run (runtime.h:76-79) over the group: HOST x and y; every device
 * copies its own slice in and its outputs out (one host thread per device, each
 * overlapping its copies with its compute).  Synchronous. */
int nfx_group_run(nfx_group* g, const float* x, const int64_t* x_shape, int x_rank, float* y,
                  const int64_t* y_shape, int y_rank);
/* Device-buffer Run over the group: x and y are DEVICE buffers on the first listed
 * device.  NCCL point-to-point transfers (over NVLink) scatter the input slices to the
 * other devices and gather their outputs into y; ordered after the work queued on
 * `stream` (a stream of the first device) before the call, and work queued on it after
 * the call waits for the gathered outputs.  Asynchronous; nfx_group_check reports
 * device-side errors.  No counterpart in the reference. */
int nfx_group_run_device(nfx_group* g, const float* x, const int64_t* x_shape, int x_rank,
                         float* y, const int64_t* y_shape, int y_rank, void* stream);
int nfx_group_check(nfx_group* g);

/* One process per GPU (torchrun style): an NCCL communicator of `world` ranks.  Rank 0
 * creates the 128-byte unique id, the caller distributes it (e.g. over its own process
 * group's store), and every rank creates its communicator on its runtime's device. */
typedef struct nfx_comm nfx_comm;
int nfx_comm_unique_id(unsigned char* id_out, int id_bytes);
int nfx_comm_create(const unsigned char* id, int id_bytes, int world, int rank, int device,
                    nfx_comm** out);
void nfx_comm_destroy(nfx_comm* comm);
/* Run over a batch partitioned across the communicator's ranks: every rank passes the
 * WHOLE batch (x, y device buffers of the full shape on its own device), computes its
 * slice and writes it into y, then the slices are gathered with NCCL -- into every
 * rank's y (root < 0: an all-gather) or into `root`'s y only (the other ranks' y then
 * hold just their own slice).  Every rank must make the same call.  Asynchronous on
 * `stream`, like nfx_runtime_run_device.  No counterpart in the reference. */
int nfx_runtime_run_sharded(nfx_runtime* rt, nfx_comm* comm, const float* x,
                            const int64_t* x_shape, int x_rank, float* y,
                            const int64_t* y_shape, int y_rank, int root, void* stream);
/* The same with HOST buffers (InferenceRuntime::Run's contract, runtime.h:76-79): each
 * rank copies only its own input slice to its GPU; after the gather, y is written on
 * every rank (root < 0) or on `root` only.  Synchronous. */
int nfx_runtime_run_sharded_host(nfx_runtime* rt, nfx_comm* comm, const float* x,
                                 const int64_t* x_shape, int x_rank, float* y,
                                 const int64_t* y_shape, int y_rank, int root);

/* ---- Calibration on the GPU (neuroflow/quant/static_quant.py:609-741) ------------
 * The reference calibrates by running its FP32 PyTorch model over a calibration set with
 * hooks on every Linear and reducing the outputs on the host.  Here an FNO2d handle
 * created from the FP32 IR (no EnableInt8Gemm) runs its FP32 executor over the batches
 * with observers in the kernels, without fake-quant, and reduces on the GPU:
 *   begin(keep_values)    reset; keep_values != 0 also keeps every value (percentiles)
 *   observe(x)            one HOST batch (batch, h, w, in_ch), synchronous
 *   count()               observed tensors: lift, locs.0 .. locs.L-1, proj_q, proj_out
 *   result(i, pct, ...)   the tensor's ".output" key, its INT8 (scale, zero point) --
 *                         compute_tensor_qparams (:480-533) for pct = 100, else the
 *                         percentile rule of calibrate (:699-716) with numpy's linear
 *                         percentiles of all kept values -- its FP8 E4M3 scale
 *                         (compute_fp8_e4m3_qparams, :338-352), and the [lo, hi] used;
 *                         a NaN value gives scale 1 and zero point 0
 *   end()                 release the statistics and kept values. */
int nfx_calibrate_begin(nfx_runtime* rt, int keep_values);
int nfx_calibrate_observe(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank);
int nfx_calibrate_count(const nfx_runtime* rt);
int nfx_calibrate_result(nfx_runtime* rt, int index, double percentile, char* name_out, int name_cap,
                         float* scale_out, int32_t* zero_point_out, float* fp8_scale_out,
                         double* lo_out, double* hi_out);
int nfx_calibrate_end(nfx_runtime* rt);

/* ---- nflow-quant GEMM (cpp/include/neuroflow/int8_gemm.h) ----------------------- */

/* W8A8 GEMM over activation CODES with one (scale, zero point) per row, per-channel
 * weight codes, and the reference LinearForwardBatched epilogue
 * (int8_gemm.cpp:559-578) evaluated with the row's qparams, then + bias[o]
 * (fno.cpp:541-548) and an optional activation (act: 0 none, 1 GELU tanh form,
 * 2 ReLU; fno.cpp:36-48).  Replaces int8_gemm::LinearForwardBatched
 * (int8_gemm.h:95-97) for inputs that are already quantised per token.
 * All pointers are DEVICE pointers on the current device:
 *   A (M,K) int8; scale_a/zp_a (M,) or NULL to use scale_a_t/zp_a_t for every row;
 *   W (N,K) int8 in (out, in) layout; scale_w, zp_w, sum_w, bias (N,) (bias may be
 *   NULL); C (M,N) float32.  sum_w[o] = sum_k (W[o,k] - zp_w[o]) (int8_gemm.h:67-77).
 * K, N in {32, 64, 128, 256}; M >= 0.  Asynchronous on `stream`. */
int nfx_int8_gemm(const int8_t* A, const float* scale_a, const int32_t* zp_a, float scale_a_t,
                  int32_t zp_a_t, int M, int K, const int8_t* W, const float* scale_w,
                  const int32_t* zp_w, const int32_t* sum_w, const float* bias, int N, int act,
                  float* C, void* stream);

/* Failure-path test hook: the budget, in nanoseconds, of the pipeline waits inside the
 * INT8 GEMM kernel (nfx_int8_gemm and the GEMM layers of the FNO1d / TokenMixer2D
 * executors) for launches made after the call; 0 restores the default of 2 s.  With a
 * budget far below the kernel's latency the waits run out: the kernel raises its abort
 * flag, records the timeout in the device error word, waits (with the default budget)
 * for its own loads and MMAs in flight, releases its tensor memory and returns, and the
 * next nfx_device_errors / nfx_runtime_check reports it (NFX_INTERNAL); the context
 * stays usable.  Process-wide; not for production use.  No counterpart in the reference
 * (its errors are host-side Status codes, cpp/include/neuroflow/tensor.h:29-60). */
void nfx_debug_set_wait_budget_ns(unsigned long long ns);

/* ---- FP8 E4M3 (cpp/include/neuroflow/fp8_e4m3.h) -------------------------------
 * The reference's bit-level encoder and decoder on the GPU: fp32_array_to_e4m3_bits
 * (fp8_e4m3.h:286, RNE with saturation to +-448, NaN -> 0x7F, its subnormal rule),
 * e4m3_bits_to_fp32_array (:295) and fp8_e4m3_per_tensor_fake_quant (:312-334;
 * scale 0 acts as 1 for the division).  The plain names take DEVICE pointers of the
 * current device and run asynchronously on `stream`; the _host names take host
 * pointers (the neuroflow_cpp module's fp8_e4m3_* helpers, fp8_e4m3_pybind.h:24-66)
 * and return when the result is in `out`. */
int nfx_fp8_e4m3_to_bits(const float* x, uint8_t* bits, int64_t n, void* stream);
int nfx_fp8_e4m3_from_bits(const uint8_t* bits, float* y, int64_t n, void* stream);
int nfx_fp8_e4m3_fake_quant(const float* x, float scale, float* y, int64_t n, void* stream);
int nfx_fp8_e4m3_to_bits_host(const float* x, uint8_t* bits, int64_t n);
int nfx_fp8_e4m3_from_bits_host(const uint8_t* bits, float* y, int64_t n);
int nfx_fp8_e4m3_fake_quant_host(const float* x, float scale, float* y, int64_t n);
/* No reference counterpart: the FP8 executors and nfx_fp8_e4m3_fake_quant encode and
 * decode with the hardware E4M3 conversions, patched to the reference's subnormal and
 * NaN rules and relying on the conversion's saturation for the clamp to +-448.  This
 * runs every fp32 bit pattern (the reference form clamped) and every code through both
 * forms on the current device and returns the number of disagreements in *mismatches
 * (0 expected).  Synchronous. */
int nfx_fp8_e4m3_selfcheck(unsigned long long* mismatches);

/* Read and clear the device error word of the current device (bit flags of waits
 * that timed out inside kernels).  Synchronises the device. */
int nfx_device_errors(unsigned* flags_out);

#ifdef __cplusplus
}
#endif

#endif /* NFX_H_ */
