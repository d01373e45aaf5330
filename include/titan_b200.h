/*
 * titan_b200.h — C ABI of libtitan_b200.so, the B200 (sm_100a) backend for the
 * titan.rs operator hot path: fp32 row softmax, bf16 GEMM, causal bf16
 * scaled-dot-product attention and bf16 NHWC conv2d, plus the reference's own
 * f32 operator ABIs.
 *
 * The library mirrors three titan.rs contracts so that a titan-backend-cuda
 * host (Rust FFI, or any C caller) can swap it in:
 *   - the HAL `DeviceSession` / `BackendDriver` traits
 *       (projects/titan-hal/src/lib.rs:200-237),
 *   - the Kernel ABI payload codec and launch metadata
 *       (projects/titan-kernel/src/lib.rs:158-256, projects/titan-types/src/lib.rs:80-104),
 *   - the runtime's per-operator entry `Runtime::execute(OpRequest)`
 *       (projects/titan-runtime/src/lib.rs:1171-1256) for "softmax", "gemm",
 *       "scaled_dot_product_attention" and "conv2d",
 * and one distributed contract, `Collective::all_gather`
 *       (projects/titan-distributed/src/lib.rs:95-99).
 *
 * Conventions
 *   - Every function returns tb_status; TB_OK is 0. On failure the calling
 *     thread's last error carries an `operation` name taken from the
 *     reference's HalError vocabulary ("allocate", "upload", "download",
 *     "launch", "buffer", "stream", "event", "load", "contract", ...) and a
 *     detail string that keeps the reference's message keywords.
 *   - Handles are reference counted; *_release drops one reference. A buffer,
 *     stream, event or kernel handle belongs to the session that created it and
 *     is rejected by any other session ("foreign buffer", "foreign stream", ...).
 *   - No function synchronises the whole device.
 *   - The CUDA driver is opened with dlopen("libcuda.so.1") on first use; on a
 *     machine without a driver tb_driver_open returns TB_ERR_DRIVER_UNAVAILABLE
 *     with operation "load_driver" (the reference's `no_cuda_environment` case,
 *     projects/titan-runtime/tests/cuda_gemm.rs:32-35).
 */
#ifndef TITAN_B200_H
#define TITAN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_API_VERSION 1

typedef enum tb_status {
  TB_OK = 0,
  TB_ERR_DRIVER_UNAVAILABLE = 1, /* no libcuda / no device (reference: load_driver, status 100) */
  TB_ERR_INVALID = 2,            /* contract or ABI violation */
  TB_ERR_FOREIGN = 3,            /* handle from another session, or cross-device */
  TB_ERR_CUDA = 4,               /* a CUDA driver call failed */
  TB_ERR_UNSUPPORTED = 5,        /* valid request this backend does not implement */
  TB_ERR_TIMEOUT = 6,            /* a bounded device-side wait gave up; context stays usable */
  TB_ERR_NCCL = 7,               /* an NCCL call failed or the communicator was aborted */
  TB_ERR_OUT_OF_MEMORY = 8,
  TB_ERR_IO = 9                  /* a file-system call failed; the detail names the path and errno */
} tb_status;

/* titan_types::DType order (projects/titan-types/src/lib.rs:42-49). */
typedef enum tb_dtype { TB_F32 = 0, TB_F16 = 1, TB_BF16 = 2, TB_I32 = 3, TB_I64 = 4 } tb_dtype;

/* Last error of the calling thread (HalError{operation, detail}, titan-hal/src/lib.rs:9-14). */
const char* tb_last_error_operation(void);
const char* tb_last_error_detail(void);
const char* tb_version(void);

typedef struct tb_session tb_session;
typedef struct tb_buffer tb_buffer;
typedef struct tb_stream tb_stream;
typedef struct tb_event tb_event;
typedef struct tb_kernel tb_kernel;
typedef struct tb_comm tb_comm;
typedef struct tb_graph_exec tb_graph_exec;

/* DeviceFingerprint (titan-types/src/lib.rs:28-38); capability_revision is
 * "sm_<major><minor>" as in CudaDiscovery (titan-backend-cuda/src/lib.rs:221-226). */
typedef struct tb_fingerprint {
  uint32_t ordinal;
  char model[128];
  char driver[32];
  char capability_revision[16];
  uint32_t sm_count;
  uint64_t total_memory;
} tb_fingerprint;

/* ---------------- Driver (BackendDriver, titan-hal/src/lib.rs:233-237) ---------------- */

/* CudaDiscovery::open (titan-backend-cuda/src/lib.rs:190-230): dlopen + cuInit. Idempotent. */
tb_status tb_driver_open(void);
/* BackendDriver::enumerate (titan-backend-cuda/src/lib.rs:1544-1546). */
tb_status tb_driver_enumerate(tb_fingerprint* out, uint32_t capacity, uint32_t* count);
/* BackendDriver::open -> DeviceSession on the primary context (titan-backend-cuda/src/lib.rs:1548-1565). */
tb_status tb_session_open(uint32_t ordinal, tb_session** out);
void tb_session_retain(tb_session* session);
void tb_session_release(tb_session* session);
/* DeviceSession::fingerprint (titan-hal/src/lib.rs:202). */
tb_status tb_session_fingerprint(const tb_session* session, tb_fingerprint* out);

/* ---------------- DeviceSession (titan-hal/src/lib.rs:200-230) ---------------- */

/* DeviceSession::allocate (titan-backend-cuda/src/lib.rs:1255-1262); zero bytes are refused
 * ("zero-byte CUDA allocations are unsupported", :122-125). */
tb_status tb_allocate(tb_session* session, size_t bytes, size_t alignment, tb_buffer** out);
/* Registers device memory owned by someone else (e.g. a torch tensor) as a
 * non-owning buffer of this session. No reference counterpart; it lets callers
 * that allocate elsewhere use the op entry points. */
tb_status tb_buffer_wrap(tb_session* session, uint64_t device_ptr, size_t bytes, tb_buffer** out);
void tb_buffer_retain(tb_buffer* buffer);
void tb_buffer_release(tb_buffer* buffer);
/* Buffer::byte_len / Buffer::identity (titan-hal/src/lib.rs:44-49). */
size_t tb_buffer_byte_len(const tb_buffer* buffer);
uint64_t tb_buffer_identity(const tb_buffer* buffer);
/* Backend-private native handle (the reference's CudaBuffer downcast). */
uint64_t tb_buffer_device_ptr(const tb_buffer* buffer);

/* DeviceSession::create_stream / create_event (titan-hal/src/lib.rs:206-207). */
tb_status tb_create_stream(tb_session* session, tb_stream** out);
void tb_stream_release(tb_stream* stream);
tb_status tb_create_event(tb_session* session, tb_event** out);
void tb_event_release(tb_event* event);

/* DeviceSession::upload (titan-backend-cuda/src/lib.rs:1264-1288): `src` is copied
 * to a staging area kept alive until the returned event completes, so the
 * caller may reuse `src` immediately. */
tb_status tb_upload(tb_session* session, tb_stream* stream, tb_buffer* dst, const void* src, size_t len,
                    tb_event** out);
/* DeviceSession::download (titan-backend-cuda/src/lib.rs:1290-1306): finishes
 * before returning because `dst` is only borrowed for the call. */
tb_status tb_download(tb_session* session, tb_stream* stream, tb_buffer* src, void* dst, size_t len,
                      tb_event** out);
/* DeviceSession::copy (titan-backend-cuda/src/lib.rs:1308-1320). */
tb_status tb_copy(tb_session* session, tb_stream* stream, tb_buffer* dst, tb_buffer* src, size_t bytes,
                  tb_event** out);

/* Launch-argument kinds (LaunchArgKind, titan-types/src/lib.rs:80-88). */
typedef enum tb_arg_kind { TB_ARG_BUFFER = 0, TB_ARG_SCALAR = 1, TB_ARG_SHAPE = 2 } tb_arg_kind;
typedef struct tb_launch_arg {
  uint32_t kind;  /* tb_arg_kind */
  uint32_t width; /* scalar byte_len, or shape rank; 0 for buffers */
} tb_launch_arg;
/* KernelLaunchMetadata (titan-types/src/lib.rs:90-104). */
typedef struct tb_launch_metadata {
  uint32_t version;
  const char* entry;
  const tb_launch_arg* arguments;
  uint32_t num_arguments;
  uint32_t block[3];
  uint32_t shared_bytes;
} tb_launch_metadata;
/* BufferBinding (titan-hal/src/lib.rs:53-70): `owner` is the session the caller
 * claims owns the buffer (the reference's DeviceId). */
typedef struct tb_binding {
  uint32_t slot;
  tb_buffer* buffer;
  const tb_session* owner;
} tb_binding;
/* EncodedLaunchArgs (titan-hal/src/lib.rs:110): payload encoded per
 * KernelAbi::encode (titan-kernel/src/lib.rs:158-207), slot bindings, and the
 * canonical ABI bytes (KernelAbi::canonical_bytes, titan-kernel/src/lib.rs:130-132). */
typedef struct tb_encoded_args {
  const uint8_t* payload;
  size_t payload_len;
  const tb_binding* bindings;
  uint32_t num_bindings;
  const uint8_t* canonical_abi;
  size_t canonical_abi_len;
} tb_encoded_args;
/* LaunchGeometry (titan-hal/src/lib.rs:193-197). */
typedef struct tb_launch_geometry {
  uint32_t grid[3];
  uint32_t block[3];
  uint32_t shared_bytes;
} tb_launch_geometry;

/* DeviceSession::load (titan-backend-cuda/src/lib.rs:1339-1411). Accepts an
 * sm_100a cubin (ELF) or NUL-terminated PTX text; modules are cached per
 * session by content, so repeated loads of one artifact do not re-JIT. */
tb_status tb_load(tb_session* session, const void* artifact, size_t len, const char* abi_hash,
                  const tb_launch_metadata* metadata, tb_kernel** out);
void tb_kernel_release(tb_kernel* kernel);
/* The precompiled sm_100a cubins embedded in this library, by module name
 * ("softmax", "gemm_bf16", ...): the artifact bytes a titan-runtime would pass
 * to tb_load in place of its PTX (CudaCompiler::compile_artifact,
 * titan-backend-cuda/src/lib.rs:970-980). */
tb_status tb_builtin_cubin(const char* module, const void** data, size_t* len);
/* DeviceSession::launch (titan-backend-cuda/src/lib.rs:1413-1507): decodes the
 * payload against the kernel's metadata, substitutes device pointers and
 * launches. Rejects an ABI mismatch, a foreign kernel, truncated or trailing
 * payload bytes, scalar width mismatches and missing or cross-session bindings. */
tb_status tb_launch(tb_session* session, tb_stream* stream, tb_kernel* kernel, const tb_encoded_args* args,
                    const tb_launch_geometry* geometry, tb_event** out);
/* DeviceSession::poll / wait / wait_event (titan-backend-cuda/src/lib.rs:1509-1536).
 * tb_poll sets *ready to 1 or 0. tb_wait also reports TB_ERR_TIMEOUT if a kernel
 * of this session gave up a bounded device-side wait. */
tb_status tb_poll(tb_session* session, tb_event* event, int* ready);
tb_status tb_wait(tb_session* session, tb_event* event);
tb_status tb_wait_event(tb_session* session, tb_stream* stream, tb_event* event);

/* Extensions used for timing (titan-profiler's event-based design intent): */
tb_status tb_record(tb_session* session, tb_stream* stream, tb_event** out);
tb_status tb_event_elapsed_ms(tb_session* session, tb_event* start, tb_event* end, float* ms);
tb_status tb_stream_synchronize(tb_session* session, tb_stream* stream);
/* Raw CUstream of a session stream (for interop with other CUDA users). */
uint64_t tb_stream_handle(const tb_stream* stream);

/* CUDA graphs (no counterpart in the reference, which launches every kernel from the
 * host, titan-backend-cuda/src/lib.rs:1413-1507). The device work enqueued on `stream`
 * by this thread between tb_capture_begin and tb_capture_end (operators, device
 * copies, event records) becomes a graph that tb_graph_exec_launch replays on any
 * stream of the session with one launch, on the same device buffers. Host-staged
 * uploads/downloads, host waits and an operator's first use of per-stream scratch
 * (split-K, the persistent attention candidate: run it once first) cannot be
 * captured: tb_capture_end then returns the driver's error and no graph. */
tb_status tb_capture_begin(tb_session* session, tb_stream* stream);
tb_status tb_capture_end(tb_session* session, tb_stream* stream, tb_graph_exec** out);
tb_status tb_graph_exec_launch(tb_session* session, tb_graph_exec* graph, tb_stream* stream);
void tb_graph_exec_release(tb_graph_exec* graph);

/* Page-locked host memory and copies that use it directly (no staging): the
 * caller keeps `src`/`dst` alive until the returned event completes. */
tb_status tb_host_alloc(tb_session* session, size_t bytes, void** out);
tb_status tb_host_free(tb_session* session, void* ptr);
tb_status tb_upload_pinned(tb_session* session, tb_stream* stream, tb_buffer* dst, size_t dst_offset,
                           const void* src, size_t len, tb_event** out);
tb_status tb_download_pinned(tb_session* session, tb_stream* stream, tb_buffer* src, size_t src_offset, void* dst,
                             size_t len, tb_event** out);

/* ---------------- Operators (Runtime::execute, titan-runtime/src/lib.rs:1171-1256) ---------------- */

/* A tensor argument: the TensorHandle / TensorSpec pair of an OpRequest
 * (titan-graph/src/graph.rs:313-327, titan-tensor/src/lib.rs:17-123). Strides
 * are in elements; a tensor is contiguous when they are row-major. */
#define TB_MAX_RANK 6
typedef struct tb_tensor {
  tb_buffer* buffer;
  uint32_t dtype; /* tb_dtype */
  uint32_t rank;
  uint64_t shape[TB_MAX_RANK];
  int64_t strides[TB_MAX_RANK];
} tb_tensor;

/* An operator attribute (AttrValue Int/Bool, or String when `str` is non-NULL). */
typedef struct tb_attr {
  const char* key;
  int64_t value;
  const char* str;
} tb_attr;

/* "softmax" — execute_cuda_softmax (titan-runtime/src/lib.rs:1504-1596):
 * last axis only, F32 (or BF16 in and out, fp32 arithmetic), contiguous, output the
 * same shape. */
tb_status tb_op_softmax(tb_session* session, tb_stream* stream, const tb_tensor* input, const tb_tensor* output,
                        const tb_attr* attrs, uint32_t num_attrs, tb_event** out);

/* "gemm" — execute_cuda_gemm (titan-runtime/src/lib.rs:2289-2404) and the CPU
 * contract (titan-runtime/src/lib.rs:955-989). C[M,N] = op(A)·op(B) with the
 * attributes transpose_lhs / transpose_rhs. F32 in/out (reference ABI,
 * titan-backend-cuda/src/lib.rs:663-677) or BF16 in/out with f32 accumulation;
 * transpose_rhs=1 with rhs [N,K] is the column-major B of the B200 path. */
tb_status tb_op_gemm(tb_session* session, tb_stream* stream, const tb_tensor* lhs, const tb_tensor* rhs,
                     const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs, tb_event** out);

/* "scaled_dot_product_attention" — execute_cuda_attention
 * (titan-runtime/src/lib.rs:2575-2705): Q[B,H,Tq,D], K/V[B,H,Tk,D] -> O[B,H,Tq,D],
 * scale 1/sqrt(D). F32 rejects "mask"/"causal" as the reference does
 * (titan-backend-cuda/src/lib.rs:753-757); BF16 accepts causal=1 (query i sees
 * keys j <= i) and rejects masks. */
tb_status tb_op_sdpa(tb_session* session, tb_stream* stream, const tb_tensor* q, const tb_tensor* k,
                     const tb_tensor* v, const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs,
                     tb_event** out);

/* "conv2d" — execute_cuda_conv2d (titan-runtime/src/lib.rs:2406-2573). Attributes
 * stride_h/w, pad_h/w, dilation_h/w, groups are required as in the reference.
 * F32: NCHW input, OIHW weight, optional bias. BF16 (attribute layout="NHWC"):
 * NHWC input, KRSC weight [Cout,R,S,Cin], optional f32 bias, NHWC output. */
tb_status tb_op_conv2d(tb_session* session, tb_stream* stream, const tb_tensor* input, const tb_tensor* weight,
                       const tb_tensor* bias, const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs,
                       tb_event** out);

/* Runtime::execute (titan-runtime/src/lib.rs:1171-1256) by operator name, for a host
 * that routes OpRequests without naming each entry: "softmax" (1 input),
 * "gemm" (2), "scaled_dot_product_attention" (3), "conv2d" (2 or 3: input, weight,
 * optional bias) and "gemm.bias_act" (2 or 3: A, B, optional bias) go to the entries
 * above with the same checks; "attention.fused" (3: contiguous [Tq, D] Q, [Tk, D] K and
 * V, [Tq, D] output, the graph compiler's gemm -> softmax -> gemm node) runs tb_op_sdpa
 * on [1, 1, T, D] views of the same buffers. Another name is TB_ERR_UNSUPPORTED ("does not
 * implement"); a wrong input count is TB_ERR_INVALID with the operator's arity message.
 * Both report operation "contract", as ExecutionError{phase: "contract"} does. */
tb_status tb_execute(tb_session* session, tb_stream* stream, const char* op, const tb_tensor* inputs,
                     uint32_t num_inputs, const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs,
                     tb_event** out);

/* Runtime::compile (titan-runtime/src/lib.rs:3472-3483) over the Graph IR
 * (titan-graph/src/graph.rs:72-105), shaped like the core pipeline
 * (titan-graph/src/optimize.rs:23-60): validate, dead-code elimination, the GEMM-epilogue
 * fusion (bf16 gemm -> broadcast.add of an F32 [N] bias -> gelu/silu becomes
 * "gemm.bias_act") and the attention fusion (gemm(Q, K; transpose_rhs) -> softmax(last
 * axis) -> gemm(P, V) on bf16 [T, D] values becomes "attention.fused" with scale 1.0),
 * validate, and a non-empty check. The graph is JSON:
 *   {"inputs": [ids], "outputs": [ids], "values": {"<id>": {"dtype": "BF16", "shape": [..]}},
 *    "nodes": [{"id": n, "operator": "...", "inputs": [ids], "outputs": [ids], "attrs": {..}}]}
 * `passes` is "compile" (or NULL) for the whole pipeline, or a comma-separated list of
 * "validate", "check" (validate without a report), "dce", "fusion.gemm_epilogue",
 * "fusion.attention", "nonempty". On success `out` holds {"graph": {inputs, outputs,
 * values: [ids kept], nodes}, "reports": [{"name", "changed", "notes"}]}; a failing graph
 * returns TB_ERR_INVALID with {"error": {"operator", "phase": "compile", "message"}} in
 * `out`. Text output follows the tune store's convention (*len always set; retry with
 * cap > *len). */
tb_status tb_graph_compile(const char* graph_json, const char* passes, char* out, size_t cap, size_t* len);

/* Which kernel the last successful op on this thread launched (the candidate id
 * the runtime reports in ExecutionHandle, titan-runtime/src/lib.rs:2403). */
const char* tb_last_candidate(void);
/* Number of kernels this thread has launched through the library. */
uint64_t tb_launch_count(void);

/* ---------------- Collective (Collective trait, titan-distributed/src/lib.rs:95-99) ---------------- */

#define TB_COMM_ID_BYTES 128
/* ncclGetUniqueId; rank 0 creates it and the caller distributes it. */
tb_status tb_comm_unique_id(uint8_t id[TB_COMM_ID_BYTES]);
/* Non-blocking communicator (watchdog-aborted after `timeout_ms` of no progress). */
tb_status tb_comm_init(tb_session* session, const uint8_t id[TB_COMM_ID_BYTES], int nranks, int rank,
                       uint32_t timeout_ms, tb_comm** out);
void tb_comm_release(tb_comm* comm);
int tb_comm_rank(const tb_comm* comm);
int tb_comm_size(const tb_comm* comm);
/* Collective::all_gather (titan-distributed/src/lib.rs:98, LocalRing :129-134):
 * concatenates each rank's `bytes_per_rank` of `send` into `recv` in rank order. */
tb_status tb_comm_all_gather(tb_comm* comm, tb_stream* stream, tb_buffer* send, tb_buffer* recv,
                             size_t bytes_per_rank, tb_event** out);
/* Device-side barrier across the communicator (a 1-element all-reduce). */
tb_status tb_comm_barrier(tb_comm* comm, tb_stream* stream);

/* No counterpart in the reference, whose all_gather concatenates host vectors
 * (titan-distributed/src/lib.rs:95-99). Collective: every rank calls it with its own
 * buffer, in the same order. Maps each rank's buffer, and a 128-byte signal block
 * of flags, into every other rank's address space (CUDA IPC, peer access over
 * NVLink) so that operators such as tb_op_gemm_sharded can store into the peers'
 * copies directly and synchronise inside their kernels. Fails with
 * TB_ERR_UNSUPPORTED when two ranks share a GPU. Synchronizes `stream`. The buffer
 * stays retained until tb_comm_deregister_buffer or tb_comm_release; all ranks must
 * deregister before any rank frees its buffer. */
tb_status tb_comm_register_buffer(tb_comm* comm, tb_stream* stream, tb_buffer* buffer);
tb_status tb_comm_deregister_buffer(tb_comm* comm, tb_buffer* buffer);

/* N-sharded GEMM: this rank owns output columns [rank*N/p, (rank+1)*N/p).
 * lhs is the full A[M,K]; rhs_shard is B's shard as [N/p, K] (column-major B);
 * output is the full C[M,N] on every rank after the call.
 * When the output buffer is registered (tb_comm_register_buffer) on every rank,
 * one fused kernel (gemm_bf16_tn_allgather) stores this rank's columns into all
 * ranks' C over NVLink; it waits at its start until every rank has reached the call
 * and completes only when every rank's stores have landed (flags in the signal
 * blocks, each wait bounded at ~1 s with an error status), and `workspace` may be NULL.
 * Otherwise `workspace` holds p*M*(N/p) elements of the output dtype: the GEMM
 * fills this rank's slot, NCCL all-gathers the slots and a layout kernel writes C.
 * Every rank must take the same form. */
tb_status tb_op_gemm_sharded(tb_comm* comm, tb_stream* stream, const tb_tensor* lhs, const tb_tensor* rhs_shard,
                             const tb_tensor* output, tb_buffer* workspace, tb_event** out);

/* ---------------- Fused GEMM epilogue ---------------- */

/* "gemm.bias_act": C = act(A B^T + bias) in one launch. Fuses the reference's gemm
 * (titan-runtime/src/lib.rs:955-989) with broadcast.add of a per-column bias and its
 * gelu (:625-640, erf by Abramowitz & Stegun 7.1.26) or silu (:3064) operators:
 * the bias is added and the activation applied to the fp32 accumulator, which is
 * rounded to bf16 once. A BF16 [M,K] (or stored [K,M] with transpose_lhs = 1), B BF16
 * [K,N] (or stored [N,K] with transpose_rhs = 1), C BF16 [M,N]; bias F32 [N] or NULL;
 * attributes activation ("none" | "gelu" | "silu"), transpose_lhs, transpose_rhs,
 * candidate ("gemm_bf16_tn_bias_act[_2sm]" for A row-major and B stored [N,K];
 * "gemm_bf16_nn_2sm", "gemm_bf16_ta_2sm", "gemm_bf16_ta_nn_2sm" for the other storage
 * orders). The contiguous extents of A and B must be multiples of 8 and the tensors
 * 16-byte aligned, else TB_ERR_UNSUPPORTED. */
tb_status tb_op_gemm_bias_act(tb_session* session, tb_stream* stream, const tb_tensor* lhs, const tb_tensor* rhs,
                              const tb_tensor* bias, const tb_tensor* output, const tb_attr* attrs,
                              uint32_t num_attrs, tb_event** out);

/* ---------------- Allocation-free split-K GEMM ---------------- */

/* No counterpart in the reference. The split-K bf16 GEMM of tb_op_gemm
 * (C[M,N] = A[M,K] x B^T, A row-major, B stored [N,K], C row-major, fp32
 * accumulation) for callers that must not let a library allocate device memory,
 * such as a server that plans all of HBM up front. Its fp32 partials live in a
 * fixed 32 MiB device array inside the library instead of memory allocated per
 * stream, so it rejects splits*M*N above 8,388,608 partials (TB_ERR_INVALID) and
 * calls no allocator. `stream` is a CUstream of the current device; a, b, c are
 * 16-byte-aligned device pointers; K % 8 == 0; splits = 0 chooses as tb_op_gemm
 * does. The first call on a device fetches the array's address (do it before any
 * stream capture). All calls share the array: calls that can overlap on the GPU
 * race and must be serialised by the caller. */
tb_status tb_gemm_bf16_splitk_noalloc(uint64_t stream, const void* a, const void* b, void* c, int m, int n, int k,
                                      int splits);

/* No counterpart in the reference. The device-side result of the calls above:
 * synchronises `stream` (a CUstream of the current device), then reads and clears
 * the device's status word, which a split-K kernel sets when one of its bounded
 * waits (~1 s each) runs out and it returns early, leaving that call's C invalid.
 * The word is sticky until read, so TB_ERR_TIMEOUT (operation "wait", the code in
 * `*code` and in the error detail) means some call on this device since the
 * previous query failed; TB_OK with *code == 0 means none did. Allocates nothing. */
tb_status tb_gemm_bf16_splitk_noalloc_status(uint64_t stream, uint32_t* code);

/* ---------------- Seeded synthetic inputs (host side) ---------------- */

/* Counter-based generator: element i depends only on (seed, i), so any slice is
 * reproducible independently and the fill can run on many threads. `dtype` is
 * TB_F32 or TB_BF16 (round to nearest even). threads <= 0 uses all cores. */
tb_status tb_fill_normal(void* dst, uint32_t dtype, size_t count, uint64_t seed, double mean, double stddev,
                         int threads);
tb_status tb_fill_uniform(void* dst, uint32_t dtype, size_t count, uint64_t seed, double low, double high,
                          int threads);

/* ---------------- Tuning store (`.tune` version 2) ---------------- */

/* The autotuner's persistent cache (projects/titan-autotune/src/lib.rs:46-82, Autotuner::
 * open/get/insert/flush) with the persistence rules of docs/architecture/autotune-v2.md:9.
 * The file is `# titan.tune version=2` followed by one canonical JSON line per record,
 * {"checksum": C, "entry": E, "key": K}: K and E are JSON objects, C is the lowercase hex
 * SHA-256 of the canonical {"entry": E, "key": K}. Canonical JSON is byte-identical to
 * Python's json.dumps(obj, sort_keys=True, separators=(",", ":")). Keys are exact: two
 * keys are the same decision when their canonical texts are equal. Lines that are not
 * JSON, lack a field or fail their checksum are skipped and counted; a file without the
 * version-2 header contributes no records. The store does not interpret key or entry
 * fields, so records written by hosts with other fields survive a flush.
 *
 * Text outputs: *len receives the length without the terminating NUL; the text and a
 * NUL are copied when cap > *len, otherwise the call fails with TB_ERR_INVALID and the
 * caller retries with a larger buffer. A store handle may be used from several threads. */
typedef struct tb_tune_store tb_tune_store;

/* Opens the store at `path` (the full file name, e.g. "kernels.tune") and reads it
 * without locking; a missing or unreadable file gives an empty store. */
tb_status tb_tune_open(const char* path, tb_tune_store** out);
void tb_tune_release(tb_tune_store* store);
/* Records `entry_json` for `key_json` in memory (both JSON objects, any formatting). */
tb_status tb_tune_insert(tb_tune_store* store, const char* key_json, const char* entry_json);
/* Canonical entry for `key_json`; *len = 0 when the key has no record. */
tb_status tb_tune_get(const tb_tune_store* store, const char* key_json, char* entry, size_t cap, size_t* len);
/* Takes an exclusive flock on `<path>.lock`, merges with the records on disk (the
 * store's own records win), writes `<path>.tmp`, fsyncs it, renames it over `path` and
 * fsyncs the directory. The store then holds the merged records. TB_ERR_IO on failure. */
tb_status tb_tune_flush(tb_tune_store* store);
/* Number of records, and lines the last read of the file (open or flush) skipped. */
tb_status tb_tune_stats(const tb_tune_store* store, size_t* records, size_t* ignored_lines);
/* Record `index` (0 <= index < records) in canonical key order. */
tb_status tb_tune_record(const tb_tune_store* store, size_t index, char* key, size_t key_cap, size_t* key_len,
                         char* entry, size_t entry_cap, size_t* entry_len);
/* Canonical form of any JSON text (the form records are keyed and checksummed in). */
tb_status tb_tune_canonical_json(const char* json, char* out, size_t cap, size_t* len);
/* One timed candidate for the selection rule. */
typedef struct tb_tune_measurement {
  const char* candidate;
  uint64_t median_ns;
  uint64_t p95_ns;
  uint64_t workspace_bytes;
} tb_tune_measurement;
/* The v2 selection rule (docs/architecture/autotune-v2.md): the lowest median wins;
 * among candidates whose median is within 2% of it, the lower p95, then the smaller
 * workspace, then the smaller name (byte order) decide. *winner is an index into ms. */
tb_status tb_tune_select(const tb_tune_measurement* ms, size_t n, size_t* winner);
/* SHA-256 (FIPS 180-4) of `len` bytes as 64 lowercase hex digits and a NUL in out[65]. */
tb_status tb_sha256_hex(const void* data, size_t len, char* out);

#ifdef __cplusplus
}
#endif
#endif /* TITAN_B200_H */
