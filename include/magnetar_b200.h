/*
 * magnetar_b200.h — C ABI of the B200-native packed-weight matmul Provider.
 *
 * A drop-in for the quantized-matmul Kernels of the reference CPU Provider
 * (astorise/Magnetar-provider-CPU, `NativeCpuProvider` / `NativeCpuExecutor`,
 * src/native/mod.rs).  The entry points mirror the Rust traits `Provider` and
 * `ProviderExecutionApi` (defined in the crate `magnetar-provider-api`,
 * implemented by the reference at src/native/mod.rs:565-947) with plain
 * pointers and sizes, so a thin Rust `extern "C"` adapter can implement those
 * traits over this library (the integration guide beside this header shows
 * the binding).
 *
 * All entry points are thread-safe.  Tensors cross the boundary as host f32
 * buffers (copied in and out; the caller keeps ownership) or, for the
 * low-level `mgb_qmatmul*` family, as device pointers.  Every status other
 * than MGB_OK leaves a reason in `mgb_last_error()` (thread-local).
 */
#ifndef MAGNETAR_B200_H
#define MAGNETAR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MGB_ABI_VERSION 3
#define MGB_MAX_RANK 8

/* Status codes.  The kernel errors follow `KernelError` (src/lib.rs:2193-2230,
 * :2445-2456, :3052-3057); MGB_DECLINED is `PackedWeightWrite::Declined`
 * (src/native/mod.rs:638-653); MGB_MEMORY_DENIED is
 * `MemoryError::AllocationDenied` (src/lib.rs:1769-1771). */
typedef enum mgb_status {
    MGB_OK = 0,
    MGB_DECLINED = 1,
    MGB_EXECUTION_FAILED = 2,
    MGB_DTYPE_UNSUPPORTED = 3,
    MGB_ATTRIBUTE_UNSUPPORTED = 4,
    MGB_KERNEL_NOT_FOUND = 5,
    MGB_TIMEOUT = 6,
    MGB_MEMORY_DENIED = 7,
    MGB_UNKNOWN_HANDLE = 8,
    MGB_NOT_FOUND = 9,
    MGB_INVALID_ARGUMENT = 10,
    MGB_CUDA_ERROR = 11,
    MGB_NCCL_ERROR = 12,
    MGB_UNSUPPORTED = 13
} mgb_status;

/* Packed block formats.  Codes follow the reference's `FORMATS` order
 * (src/native/quant.rs:71-87).  This Provider stores Q8_0, Q4_K, Q5_K, Q6_K,
 * IQ4_NL and Q4_0 and declines the rest (the Runtime then loads those weights
 * as f32). */
enum {
    MGB_FORMAT_Q8_0 = 0,
    MGB_FORMAT_Q4_K = 1,
    MGB_FORMAT_Q6_K = 2,
    MGB_FORMAT_Q2_K = 3,
    MGB_FORMAT_Q3_K = 4,
    MGB_FORMAT_IQ4_NL = 5,
    MGB_FORMAT_IQ4_XS = 6,
    MGB_FORMAT_IQ2_XXS = 7,
    MGB_FORMAT_IQ2_XS = 8,
    MGB_FORMAT_IQ2_S = 9,
    MGB_FORMAT_IQ3_XXS = 10,
    MGB_FORMAT_IQ3_S = 11,
    MGB_FORMAT_Q5_K = 12,
    MGB_FORMAT_Q4_0 = 13
};

enum { MGB_DTYPE_F32 = 0, MGB_DTYPE_F16 = 1, MGB_DTYPE_BF16 = 2 };
enum { MGB_KERNEL_AUTO = 0, MGB_KERNEL_GEMV = 1, MGB_KERNEL_GEMM = 2 };
enum { MGB_CANCELLATION_TIMEOUT_ONLY = 1 };
enum { MGB_HEALTH_AVAILABLE = 0, MGB_HEALTH_UNAVAILABLE = 1 };
enum { MGB_VALUE_ABSENT = 0, MGB_VALUE_OPAQUE = 1 };

/* Observation kinds (`KernelObservationKind`, src/lib.rs:2367-2402, :3387-3401). */
enum {
    MGB_OBS_PROVIDER_REGISTERED = 0,
    MGB_OBS_DEVICE_DETECTED = 1,
    MGB_OBS_DISPATCH_STARTED = 2,
    MGB_OBS_DISPATCH_COMPLETED = 3,
    MGB_OBS_DISPATCH_FAILED = 4,
    MGB_OBS_TIMEOUT = 5
};

typedef struct mgb_provider mgb_provider;

/* Provider controls, read once per Provider like the reference's environment
 * controls (src/native/mod.rs:8-31, :505-522). */
typedef struct mgb_settings {
    int32_t packed_weights;   /* MAGNETAR_B200_PACKED_WEIGHTS (0 declines packed weights), default 1 */
    int32_t int8_activations; /* MAGNETAR_B200_INT8_ACTIVATIONS, default 0 (f32 activations) */
    int32_t device;           /* MAGNETAR_B200_DEVICE, CUDA ordinal, default 0 */
    int32_t profile;          /* MAGNETAR_B200_PROFILE=1 times every Kernel by name */
    int32_t kernel;           /* MAGNETAR_B200_KERNEL=auto|gemv|gemm (MGB_KERNEL_*) */
} mgb_settings;

typedef struct mgb_provider_metadata {
    const char *name;         /* "magnetar:provider/b200-native" */
    const char *version;
    const char *vendor;
    const char *description;
} mgb_provider_metadata;

/* `native_cpu_device()` counterpart (src/native/mod.rs:825-842). */
typedef struct mgb_device_descriptor {
    char id[64];              /* "cuda-b200:<ordinal>" */
    char name[128];
    char architecture[32];    /* "sm_100a" */
    uint32_t compute_units;   /* SMs */
    uint64_t memory_bytes;
    uint32_t max_concurrent_operations;
    uint64_t max_workspace_bytes;
} mgb_device_descriptor;

/* `KernelAdvertisement` for the Kernels this Provider executes
 * (`baseline_advertisement`, src/lib.rs:1350-1373): rank 2, f32 in and out,
 * contiguous, cancellation TimeoutOnly. */
typedef struct mgb_kernel_advertisement {
    const char *name;         /* "matmul", "matmul-bias", "matmul-residual" */
    const char *operator_family;
    int32_t rank;
    int32_t input_dtype;
    int32_t output_dtype;
    int32_t cancellation;
} mgb_kernel_advertisement;

/* Attributes of one Kernel invocation (`KernelInvocation::attributes`). */
typedef struct mgb_kernel_attrs {
    int32_t transpose_a;
    int32_t transpose_b;
    int32_t accumulation_dtype; /* MGB_DTYPE_F32; any other value is rejected (src/lib.rs:2445-2456) */
    int64_t deadline_ms;        /* < 0 none; 0 already elapsed -> MGB_TIMEOUT (src/lib.rs:2372-2380) */
    int32_t has_scale;          /* `embedding`'s optional "scale" attribute (src/native/mod.rs:439-447) */
    float scale;
} mgb_kernel_attrs;

/* `KernelResult` of a completed invocation. */
typedef struct mgb_kernel_result {
    int32_t status;           /* MGB_OK or the kernel's error code */
    char reason[256];
} mgb_kernel_result;

typedef struct mgb_observation {
    uint64_t sequence;
    int32_t kind;             /* MGB_OBS_* */
    char kernel[48];
    char detail[112];
} mgb_observation;

/* ---- errors -------------------------------------------------------------------------- */

/* The last failure's reason on this thread (reference wording where one exists). */
const char *mgb_last_error(void);
const char *mgb_status_name(int32_t status);

/* ---- identity / lifecycle (`Provider`, src/native/mod.rs:901-947) -------------------- */

int32_t mgb_abi_version(void);
/* `native_cpu_provider_metadata()` counterpart (src/native/mod.rs:813-821). */
void mgb_provider_get_metadata(mgb_provider_metadata *out);
/* `NativeCpuExecutor::new()` environment parsing (src/native/mod.rs:505-522). */
mgb_status mgb_settings_from_env(mgb_settings *out);
/* `NativeCpuExecutor::with_settings` (src/native/mod.rs:525-544); settings NULL = from env. */
mgb_status mgb_provider_create(const mgb_settings *settings, mgb_provider **out);
/* Releases every device allocation; prints the profile when enabled (mod.rs:476-496). */
void mgb_provider_destroy(mgb_provider *provider);
/* `Provider::initialize` (src/native/mod.rs:928-938): records ProviderRegistered
 * and DeviceDetected observations. */
mgb_status mgb_provider_initialize(mgb_provider *provider);
/* `Provider::shutdown` (src/native/mod.rs:940-942). */
mgb_status mgb_provider_shutdown(mgb_provider *provider);
/* `Provider::health` (src/native/mod.rs:909-911). */
int32_t mgb_provider_health(mgb_provider *provider);
/* `Provider::devices` (src/native/mod.rs:919-921). */
mgb_status mgb_provider_device(mgb_provider *provider, mgb_device_descriptor *out);
/* `Provider::kernel_advertisements` (src/native/mod.rs:848-864): the matmul
 * family and `embedding`. */
size_t mgb_kernel_advertisement_count(void);
mgb_status mgb_kernel_advertisement_get(size_t index, mgb_kernel_advertisement *out);

/* ---- tensor storage (`ProviderExecutionApi`, src/native/mod.rs:629-811) -------------- */

/* `write_tensor` (mod.rs:629-636): stores an f32 tensor, forgetting any packed
 * weight under `id`.  Returns once `data` has been copied (the caller may reuse
 * it).  The values go to a new device buffer and the old one is freed after
 * the work queued before it, so a kernel submitted meanwhile from another
 * thread reads the old or the new tensor, never a mixture; the upload runs on
 * its own stream with the Provider's lock released while the host waits. */
mgb_status mgb_write_tensor(mgb_provider *provider, const char *id, const uint64_t *shape,
                            int32_t rank, const float *data);
/* `write_packed_weight_tensor` (mod.rs:638-653): copies the checkpoint's block
 * bytes to the device.  *stored = 1 (Stored) or 0 (Declined: packed weights
 * disabled, or a format this Provider does not execute).  `transposed` = 1 when
 * the stored rows are the output columns (logical [stored_cols, stored_rows]). */
mgb_status mgb_write_packed_weight(mgb_provider *provider, const char *id, int32_t format,
                                   uint64_t stored_rows, uint64_t stored_cols,
                                   int32_t transposed, const void *bytes, uint64_t len,
                                   int32_t *stored);
/* `read_tensor` (src/lib.rs:1615-1620): f32 values in logical shape; a packed
 * weight reads back dequantised (bit-exact to the reference `decode`).  The
 * download runs on its own stream after the work queued before the call, with
 * the Provider's lock released while the host waits (a release or overwrite of
 * `id` meanwhile waits for the download before freeing its buffer).
 * shape_out has room for MGB_MAX_RANK entries; MGB_NOT_FOUND when absent. */
mgb_status mgb_read_tensor(mgb_provider *provider, const char *id, float *out,
                           uint64_t capacity, uint64_t *shape_out, int32_t *rank_out);
/* `resident_shape` (src/lib.rs:1748-1753): logical shape. */
mgb_status mgb_resident_shape(mgb_provider *provider, const char *id, uint64_t *shape_out,
                              int32_t *rank_out);
/* `release_tensor` (mod.rs:659-662). */
mgb_status mgb_release_tensor(mgb_provider *provider, const char *id, int32_t *was_present);
/* `NativeCpuExecutor::is_packed` (mod.rs:556-558). */
int32_t mgb_is_packed(mgb_provider *provider, const char *id);
/* `read_tensor_value` (mod.rs:695-702): MGB_VALUE_OPAQUE for resident ids. */
mgb_status mgb_read_tensor_value(mgb_provider *provider, const char *id, int32_t *kind);
/* `write_tensor_value(id, Opaque)` (mod.rs:704-721): stores nothing; a packed
 * weight stays resident. */
mgb_status mgb_write_tensor_value_opaque(mgb_provider *provider, const char *id);
/* `copy_tensor_admitted` (mod.rs:746-765): `to` takes a copy of `from`,
 * replacing whatever `to` held, a packed weight included. */
mgb_status mgb_copy_tensor(mgb_provider *provider, const char *from, const char *to);
/* Free / total device bytes, for the caller's admission ledger
 * (`write_tensor_admitted`, src/lib.rs:1713-1738). */
mgb_status mgb_device_memory(mgb_provider *provider, uint64_t *free_bytes,
                             uint64_t *total_bytes);
/* Packed weights expanded to f32 (count), as the reference's profile reports
 * (`NativeState::expand`, mod.rs:196-204). */
uint64_t mgb_materialization_count(mgb_provider *provider);

/* ---- execution (`submit_kernel` / `complete_kernel`, mod.rs:598-627,
 *      src/lib.rs:2301-2356) --------------------------------------------------------- */

/* Validates and enqueues one Kernel invocation on the Provider's stream and
 * returns its handle.  inputs[0] = activations [m, k] (f32 tensor id),
 * inputs[1] = weight (packed or f32 id), inputs[2] = bias ("matmul-bias") or
 * residual ("matmul-residual").  The result (success or the Kernel's error) is
 * observed exactly once through mgb_complete_kernel. */
mgb_status mgb_submit_kernel(mgb_provider *provider, const char *kernel,
                             const mgb_kernel_attrs *attrs, const char *const *inputs,
                             int32_t n_inputs, const char *output, uint64_t *handle);
/* Waits for the invocation and consumes its result; a second call for the
 * same handle returns MGB_UNKNOWN_HANDLE (single consumption, src/lib.rs:2337-2356). */
mgb_status mgb_complete_kernel(mgb_provider *provider, uint64_t handle,
                               mgb_kernel_result *result);

/* ---- observations (`observations`, src/lib.rs:1848-1868) ---------------------------- */

size_t mgb_observation_count(mgb_provider *provider);
/* Oldest first, at most 4096 kept (KERNEL_OBSERVATION_LOG_CAPACITY, src/lib.rs:171). */
mgb_status mgb_observations(mgb_provider *provider, mgb_observation *out, size_t capacity,
                            size_t *written);

/* ---- low-level device entry points (the kernels behind the Provider) ---------------- */

/* The kernels read a packed matrix in its *device layout*: the checkpoint's
 * ggml blocks rearranged into a quant plane (each 32-value run's quants in 16
 * or 32 aligned bytes, value pairs adjacent) followed by a scale plane (Q4_K:
 * the 16-byte d/dmin/scales header per super-block; Q8_0, IQ4_NL, Q4_0: the
 * f16 scale per block; Q5_K: Q4_K's header followed by each run's 32 fifth
 * bits, 48 bytes per 256 values; Q6_K: the quant plane holds 48 bytes per 64 values,
 * the two runs' low-nibble pairs then their high 2-bit fields, and the scale
 * plane a 32-byte header per 256 values, the 16 int8 scales then d).  Same
 * bits and byte count as the ggml blocks, except Q6_K's padded header (224
 * bytes per 256 values against 210).  `mgb_write_packed_weight` performs this
 * rearrangement itself. */
uint64_t mgb_packed_bytes(int32_t format, uint64_t stored_rows, uint64_t stored_cols);
/* ggml blocks (device memory, `stored_rows` rows of `stored_cols` values) ->
 * device layout in `out` (device memory of mgb_packed_bytes bytes). */
mgb_status mgb_repack(int32_t format, const void *ggml_blocks, uint64_t stored_rows,
                      uint64_t stored_cols, void *out, void *stream);
/* Scratch bytes `mgb_qmatmul` wants for this shape (0 when none): the bf16
 * copy of x and, for a shape whose tiles would be narrow (up to 128 rows: one
 * wave of tiles at most 112 columns wide with K split s ways; past 128 rows:
 * unsplit tiles under 64 columns wide or K >= 8192, split tiles at most 128
 * wide; s = 2, 4 or 8, k a multiple of 256 s, the planes within 256 MB), s f32
 * [m, n] planes: each of s CTAs per tile computes
 * 1/s of K into its plane and a sum pass adds them in plane order (a
 * different f32 summation order than one pass, same tolerance, deterministic).
 * Any workspace of at least mgb_qmatmul_min_workspace_bytes (the bf16 copy
 * alone) also takes the tensor-core path, in one K pass (a workspace in
 * between splits fewer ways).  The tensor-parallel call (mgb_qmatmul_tp)
 * follows the same rule for its shard. */
uint64_t mgb_qmatmul_workspace_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k);
uint64_t mgb_qmatmul_min_workspace_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k);
/* y[m, n] = x[m, k] * W^T on `stream`, W (device layout, 16-byte aligned)
 * with its n stored rows the output columns (`packed_matmul`,
 * src/native/mod.rs:109-152).  Device pointers.  `addend` (may be NULL) is added to y:
 * addend_len == n broadcasts one row (matmul-bias), == m*n adds elementwise
 * (matmul-residual).  Replaces `matmul_columns` (src/native/quant.rs:430-598). */
mgb_status mgb_qmatmul(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                       uint64_t m, float *y, const float *addend, uint64_t addend_len,
                       void *workspace, uint64_t workspace_bytes, void *stream);
/* mgb_qmatmul for callers that must not allocate device memory.  No
 * counterpart in the reference (its CPU kernels allocate host buffers freely).
 * Who needs it: a runtime that reserves the whole GPU for its own arena up
 * front (a cudaMalloc would fail or bypass its accounting), or a latency-
 * critical path that must stay out of the driver's allocator (cudaFree
 * synchronises the device).  Same arguments and results as mgb_qmatmul
 * without the workspace: the tensor-core path stages its bf16 activations in a
 * fixed array inside this library's device image, MGB_STATIC_SCRATCH_BYTES
 * (8 MiB) on every GPU that loads the library, held until the process exits.
 * Limits and rules:
 *  - m * k must be <= MGB_STATIC_SCRATCH_BYTES / 2 whenever m > 2 and
 *    k % 256 == 0 (the tensor-core path); larger shapes are rejected with
 *    MGB_INVALID_ARGUMENT and a message naming the limit;
 *  - the array is shared by every call on a device and keeps the last call's
 *    bytes: calls that may overlap on the GPU (different streams without
 *    ordering between them) race on it and corrupt each other's results;
 *  - the first call on a device resolves the device addresses of the array
 *    and of its error word (once, with that device current); make that first
 *    call before any stream capture.  The addresses belong to the device's
 *    CUDA context: after cudaDeviceReset, or from another driver-API context
 *    on the same device, they are stale, so do not call this entry point
 *    there;
 *  - nothing is allocated.  A bounded device wait that expires leaves y
 *    unspecified and records 1 in a second fixed device word beside the
 *    array, which mgb_take_device_error(device) reads and clears (that call
 *    allocates nothing either). */
#define MGB_STATIC_SCRATCH_BYTES (8u << 20)
mgb_status mgb_qmatmul_static_scratch(int32_t format, const void *w, uint64_t n, uint64_t k,
                                      const float *x, uint64_t m, float *y, const float *addend,
                                      uint64_t addend_len, void *stream);
/* The tensor-core GEMM alone for activations already in bf16: y[m, n] =
 * xb[m, k] (bf16, 16-byte aligned) * W^T, f32 accumulation, no scratch.
 * Needs k % 256 == 0.  For callers whose producer emits bf16 (no counterpart
 * in the reference, which only takes f32 activations). */
mgb_status mgb_qmatmul_bf16(int32_t format, const void *w, uint64_t n, uint64_t k,
                            const void *xb, uint64_t m, float *y, const float *addend,
                            uint64_t addend_len, void *stream);
/* Stored-order f32 values of a packed matrix (device layout), bit-exact to the reference
 * `dequantize_row` (src/native/quant.rs:1700-1711) on every stored row. */
mgb_status mgb_dequantize(int32_t format, const void *w, uint64_t stored_rows,
                          uint64_t stored_cols, float *out, void *stream);
/* y[m, stored_cols] = x[m, stored_rows] * W (device layout) for a weight whose
 * stored rows are the input rows (`packed_axpy`, src/native/mod.rs:154-194; `axpy_columns`,
 * src/native/quant.rs:1658-1689). */
mgb_status mgb_qmatmul_input_major(int32_t format, const void *w, uint64_t stored_rows,
                                   uint64_t stored_cols, const float *x, uint64_t m, float *y,
                                   void *stream);
/* Dense f32 y = op(a) * op(b) with the reference matmul's transposes
 * (`matmul`, src/lib.rs:262-318). */
mgb_status mgb_matmul_f32(const float *a, uint64_t a_rows, uint64_t a_cols, const float *b,
                          uint64_t b_rows, uint64_t b_cols, int32_t transpose_a,
                          int32_t transpose_b, float *out, void *stream);
/* Reads and clears the device error code the low-level kernels of `device`
 * record instead of trapping (1 = a bounded wait expired; 0 = none), both the
 * word of the calls that take a workspace and the word of
 * mgb_qmatmul_static_scratch.  Synchronises with the device; allocates
 * nothing.  No counterpart in the reference (its kernels run synchronously on
 * the calling thread). */
mgb_status mgb_take_device_error(int32_t device, int32_t *code);
/* The `embedding` lookup in a packed table (`NativeState::embedding`,
 * src/native/mod.rs:389-417): out[count, dim] = the dequantised rows of the
 * tokens `ids` (f32 device values, count of them), times `scale` when
 * has_scale (src/native/mod.rs:439-447).  An untransposed table is stored
 * [vocab = stored_rows, dim = stored_cols]; a transposed one [dim =
 * stored_rows, vocab = stored_cols] (the token's value in every stored row).
 * Values are bit-exact to the reference's `dequantize_row` / `element`.  Ids
 * are checked on the device: `bad` (device u32, may be NULL) receives the
 * position of the first id that is not a whole number below the vocabulary
 * size, 0xFFFFFFFF when all are valid (that row of out is zeros). */
mgb_status mgb_embedding(int32_t format, const void *w, uint64_t stored_rows, uint64_t stored_cols,
                         int32_t transposed, const float *ids, uint64_t count, int32_t has_scale,
                         float scale, float *out, uint32_t *bad, void *stream);
/* Int8 activation quantisation (`quantize_rows`, src/native/quant.rs:350-378):
 * values[len], scales[len/32], sums[len/32][2]. */
mgb_status mgb_quantize_rows(const float *x, uint64_t len, int8_t *values, float *scales,
                             int32_t *sums, void *stream);

/* ---- tensor parallelism over output columns (one process per GPU) ------------------ */

/* Rank g of G holds stored rows [g n/G, (g+1) n/G) of a packed weight, the
 * unit the reference's CPU pool splits a packed matmul on (`packed_matmul`,
 * src/native/mod.rs:135-150).  `mgb_qmatmul_tp` computes this rank's columns
 * and writes each one straight into every rank's full y over NVLink (the
 * all-gather fused into the kernel's output stores; peers' buffers are mapped
 * with CUDA IPC).  No counterpart in the reference, which runs on one host. */
#define MGB_MAX_TP 8
/* Bytes of a rank's synchronisation words: done[MGB_MAX_TP] (u32 at offset 0,
 * word r written by rank r), a reserved word at offset 128 (`cta_counter`
 * points at it) and, for device epochs, the rank's epoch word (u32 at offset
 * 132, the word after it). */
#define MGB_TP_SYNC_BYTES 256u
#define MGB_TP_COUNTER_OFFSET 128u
#define MGB_TP_EPOCH_OFFSET 132u

/* Where one rank's tensor-parallel call writes.  All pointers are valid on the
 * calling GPU (this rank's own buffers or IPC mappings of the peers').  Output
 * element (row, col) of the call goes to y[r] + row * ldy + col0 + col for
 * every r < world, with plain stores.  After the call's last launch, a
 * one-CTA kernel of the call waits for that launch's grid to complete (its
 * stores performed at every rank's memory) and then stores the epoch (system
 * scope) into done[r][rank] for every r.  `cta_counter` locates this rank's
 * synchronisation words: the word itself is reserved (zero; the call does not
 * write it) and the epoch word follows it.  The epoch is `epoch` (host epochs, counting from 1),
 * or, when `epoch` is 0 (device epochs), the value of this rank's epoch word
 * (the word after `cta_counter`) plus one, and the call advances the word to
 * it as it publishes: a sequence of calls and waits captured in a CUDA graph
 * then publishes fresh epochs on every replay.  One synchronisation buffer
 * uses one mode; with device epochs every rank's epoch word starts at zero,
 * and an op alternating between two y buffers per call captures an even
 * number of its calls in a graph, so that consecutive calls (across replays
 * too) alternate buffers.
 *
 * Input wait (optional; `wait_done` NULL: none).  Before the call reads x, its
 * first kernel waits, bounded by wait_timeout_ms (0: 2000; giving up records
 * device error 1), until every one of `wait_world` ranks has published
 * `wait_epoch` (0: device epochs, the current value of that buffer's epoch
 * word) into `wait_done`: this rank's synchronisation words of an earlier
 * fused call on this stream, normally the one whose gathered y is this call's
 * x.  It does what an mgb_tp_wait for that call would do, inside the next
 * call instead of as a kernel of its own between the two. */
typedef struct mgb_tp_out {
    float *y[MGB_MAX_TP];
    uint32_t *done[MGB_MAX_TP];
    uint32_t *cta_counter;
    uint64_t ldy;
    uint64_t col0;
    uint32_t epoch;
    int32_t world;
    int32_t rank;
    const uint32_t *wait_done;
    uint32_t wait_epoch;
    int32_t wait_world;
    uint32_t wait_timeout_ms;
} mgb_tp_out;

/* cudaMalloc'd, zero-filled device memory on the current device, whole
 * allocations so a CUDA IPC handle maps exactly them. */
mgb_status mgb_device_alloc(uint64_t bytes, void **out);
mgb_status mgb_device_free(void *ptr);
/* The 64-byte CUDA IPC handle of an mgb_device_alloc allocation, and its
 * mapping in another process (peer access enabled on demand). */
#define MGB_IPC_HANDLE_BYTES 64
mgb_status mgb_ipc_handle(void *ptr, uint8_t *handle_out);
mgb_status mgb_ipc_open(const uint8_t *handle, void **out);
mgb_status mgb_ipc_close(void *mapped);
/* This rank's shard product x[m, k] * W_shard^T (n = the shard's stored rows)
 * written into every rank's y as `out` says, then the completion published.
 * Same kernels, workspace and addend rules as mgb_qmatmul (the addend is this
 * rank's [n] or [m, n] slice).  The caller must not overwrite a peer's y while
 * the peer still reads it: alternate between two y buffers per rank (a call
 * starts writing only after the previous work on its stream, which includes
 * the wait for the previous call's peers, has finished). */
mgb_status mgb_qmatmul_tp(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                          uint64_t m, const mgb_tp_out *out, const float *addend,
                          uint64_t addend_len, void *workspace, uint64_t workspace_bytes,
                          void *stream);
/* Stream-ordered wait until done[r] has reached `epoch` for every r < world
 * (`done` = this rank's synchronisation words).  Work queued after it on
 * `stream` sees every rank's columns.  `epoch` 0: device epochs, the current
 * value of the rank's epoch word (which the last call on that buffer advanced
 * as it published).  A wait longer than timeout_ms (0: 2000) gives up and
 * records device error 1 (see mgb_take_device_error).  After such an error the
 * ranks' epochs disagree (the rank that gave up may be behind its peers, or
 * ahead of one that never published), so every later wait may expire too:
 * before the next call,
 * every rank synchronises its stream, then all ranks zero their whole
 * synchronisation area (MGB_TP_SYNC_BYTES: counter, epoch word and done
 * words) and meet at a host barrier, and host epochs restart from 1. */
mgb_status mgb_tp_wait(const uint32_t *done, int32_t world, uint32_t epoch, uint32_t timeout_ms,
                       void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MAGNETAR_B200_H */
