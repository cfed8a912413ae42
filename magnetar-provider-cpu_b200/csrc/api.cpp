// C ABI: errors, identity and the low-level device entry points
// (include/magnetar_b200.h).  The Provider object lives in provider.cpp.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/magnetar_b200.h"
#include "api_internal.h"
#include "kernels.h"

namespace mgb {

namespace {
thread_local std::string g_last_error;
}

mgb_status fail(mgb_status status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

mgb_status cuda_fail(cudaError_t e, const char *what) {
  return fail(MGB_CUDA_ERROR, "%s: %s", what, cudaGetErrorString(e));
}

void clear_error() { g_last_error.clear(); }

bool format_supported(int32_t format) {
  return format == MGB_FORMAT_Q8_0 || format == MGB_FORMAT_Q4_K || format == MGB_FORMAT_Q6_K ||
         format == MGB_FORMAT_Q5_K || format == MGB_FORMAT_IQ4_NL || format == MGB_FORMAT_Q4_0;
}

uint64_t format_block_elements(int32_t format) {
  return format == MGB_FORMAT_Q4_K || format == MGB_FORMAT_Q6_K || format == MGB_FORMAT_Q5_K ? 256
                                                                                             : 32;
}

uint64_t ggml_bytes(int32_t format, uint64_t rows, uint64_t cols) {
  if (!format_supported(format)) return 0;
  const uint64_t bb = format == MGB_FORMAT_Q4_K   ? 144
                      : format == MGB_FORMAT_Q6_K ? 210
                      : format == MGB_FORMAT_Q5_K ? 176
                      : format == MGB_FORMAT_Q8_0 ? 34
                                                  : 18;
  return rows * (cols / format_block_elements(format)) * bb;
}

uint64_t device_bytes(int32_t format, uint64_t rows, uint64_t cols) {
  // the ggml byte count, except Q6_K's 32-byte (not 18-byte) scale header per
  // 256 values
  if (format == MGB_FORMAT_Q6_K) return rows * (cols / 256) * 224;
  return ggml_bytes(format, rows, cols);
}

mgb_status check_packed_shape(int32_t format, uint64_t rows, uint64_t cols) {
  if (!format_supported(format))
    return fail(MGB_DECLINED, "packed format %d is not executed by this Provider", format);
  const uint64_t be = format_block_elements(format);
  if (cols == 0 || cols % be)
    return fail(MGB_INVALID_ARGUMENT, "stored columns %llu are not a multiple of the block size %llu",
                (unsigned long long)cols, (unsigned long long)be);
  return MGB_OK;
}

namespace {
std::mutex g_err_mu;
int *g_err_flags[64] = {};

// The flag of `device` if one was allocated (reading never allocates).
int *existing_error_flag(int device) {
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_err_mu);
  return g_err_flags[device];
}
}  // namespace

int *device_error_flag(int device) {
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_err_mu);
  if (!g_err_flags[device]) {
    int *p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    g_err_flags[device] = p;
  }
  return g_err_flags[device];
}

// Picks the kernel for m activation rows: GEMV (f32, m <= 2 per launch) or the
// tensor-core GEMM.  kernel_pref: MGB_KERNEL_AUTO / GEMV / GEMM.
mgb_status run_qmatmul(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                       uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                       void *workspace, uint64_t workspace_bytes, int *err, int kernel_pref,
                       cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = device_sms(dev);
  if (m == 0 || n == 0) return MGB_OK;
  const bool gemm_ok = gemm_supported(format, m, n, k) &&
                       workspace_bytes >= gemm_workspace_bytes(format, m, n, k) && workspace;
  const bool use_gemm = kernel_pref == MGB_KERNEL_GEMM ? gemm_ok
                        : kernel_pref == MGB_KERNEL_GEMV ? false
                                                         : (m > 2 && gemm_ok);
  if (kernel_pref == MGB_KERNEL_GEMM && !gemm_ok)
    return fail(MGB_UNSUPPORTED, "tensor-core GEMM needs k %% 256 == 0 and %llu workspace bytes",
                (unsigned long long)gemm_workspace_bytes(format, m, n, k));
  cudaError_t e;
  if (use_gemm) {
    e = launch_gemm(format, w, n, k, x, m, out, addend, addend_mode, workspace, workspace_bytes,
                    err, sms, stream);
    if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
    return MGB_OK;
  }
  // row pairs
  for (uint64_t r = 0; r < m; r += 2) {
    const uint64_t rows = m - r < 2 ? m - r : 2;
    const float *add = addend_mode == 2 ? addend + r * n : addend;
    OutSpec sub = rows_from(out, r);
    if (r > 0) sub = without_input_wait(sub);  // the first launch waited
    e = launch_gemv(format, w, n, k, x + r * k, rows, sub, add, addend_mode, err, sms, stream);
    if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
  }
  return MGB_OK;
}

// Scratch the dispatch above uses for m rows: the GEMM's bf16 activations,
// plus its split-K partial planes where those apply (the GEMV needs none).
uint64_t qmatmul_scratch_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k) {
  if (!format_supported(format)) return 0;
  if (m > 2 && gemm_supported(format, m, n, k))
    return gemm_workspace_bytes_preferred(format, m, n, k);
  return 0;
}

// The least scratch with which the dispatch still takes the GEMM.
uint64_t qmatmul_min_scratch_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k) {
  if (!format_supported(format)) return 0;
  if (m > 2 && gemm_supported(format, m, n, k)) return gemm_workspace_bytes(format, m, n, k);
  return 0;
}

mgb_status validate_qmatmul(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                            uint64_t m, float *y) {
  if (!format_supported(format))
    return fail(MGB_UNSUPPORTED, "packed format %d is not executed by this Provider", format);
  if (k == 0 || k % format_block_elements(format))
    return fail(MGB_EXECUTION_FAILED,
                "packed matmul: activations have %llu columns, not a whole number of blocks",
                (unsigned long long)k);
  if ((m && n) && (!w || !x || !y)) return fail(MGB_INVALID_ARGUMENT, "null device pointer");
  if (reinterpret_cast<uintptr_t>(w) & 15)
    return fail(MGB_INVALID_ARGUMENT, "packed weight pointer is not 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(x) & 15)
    return fail(MGB_INVALID_ARGUMENT, "activation pointer is not 16-byte aligned");
  return MGB_OK;
}

}  // namespace mgb

using namespace mgb;

extern "C" {

const char *mgb_last_error(void) { return g_last_error.c_str(); }

const char *mgb_status_name(int32_t status) {
  switch (status) {
    case MGB_OK: return "ok";
    case MGB_DECLINED: return "declined";
    case MGB_EXECUTION_FAILED: return "kernel-execution-failed";
    case MGB_DTYPE_UNSUPPORTED: return "kernel-dtype-unsupported";
    case MGB_ATTRIBUTE_UNSUPPORTED: return "kernel-attribute-unsupported";
    case MGB_KERNEL_NOT_FOUND: return "kernel-not-found";
    case MGB_TIMEOUT: return "kernel-timeout";
    case MGB_MEMORY_DENIED: return "allocation-denied";
    case MGB_UNKNOWN_HANDLE: return "unknown-handle";
    case MGB_NOT_FOUND: return "not-found";
    case MGB_INVALID_ARGUMENT: return "invalid-argument";
    case MGB_CUDA_ERROR: return "cuda-error";
    case MGB_NCCL_ERROR: return "nccl-error";
    case MGB_UNSUPPORTED: return "unsupported";
    default: return "unknown";
  }
}

int32_t mgb_abi_version(void) { return MGB_ABI_VERSION; }

uint64_t mgb_packed_bytes(int32_t format, uint64_t stored_rows, uint64_t stored_cols) {
  return device_bytes(format, stored_rows, stored_cols);
}

mgb_status mgb_repack(int32_t format, const void *ggml_blocks, uint64_t stored_rows,
                      uint64_t stored_cols, void *out, void *stream) {
  mgb_status s = check_packed_shape(format, stored_rows, stored_cols);
  if (s != MGB_OK) return s == MGB_DECLINED ? fail(MGB_UNSUPPORTED, "%s", mgb_last_error()) : s;
  if (!ggml_blocks || !out) return fail(MGB_INVALID_ARGUMENT, "null device pointer");
  if (reinterpret_cast<uintptr_t>(out) & 15)
    return fail(MGB_INVALID_ARGUMENT, "device-layout pointer is not 16-byte aligned");
  cudaError_t e = launch_repack(format, ggml_blocks, stored_rows, stored_cols, out,
                                static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "repack launch");
}

uint64_t mgb_qmatmul_workspace_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k) {
  return qmatmul_scratch_bytes(format, m, n, k);
}

uint64_t mgb_qmatmul_min_workspace_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k) {
  return qmatmul_min_scratch_bytes(format, m, n, k);
}

mgb_status mgb_qmatmul(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                       uint64_t m, float *y, const float *addend, uint64_t addend_len,
                       void *workspace, uint64_t workspace_bytes, void *stream) {
  mgb_status s = validate_qmatmul(format, w, n, k, x, m, y);
  if (s != MGB_OK) return s;
  int mode = 0;
  if (addend) {
    if (addend_len == n) mode = 1;
    else if (addend_len == m * n) mode = 2;
    else return fail(MGB_INVALID_ARGUMENT, "addend has %llu values, expected %llu or %llu",
                     (unsigned long long)addend_len, (unsigned long long)n,
                     (unsigned long long)(m * n));
  }
  int dev = 0;
  cudaGetDevice(&dev);
  return run_qmatmul(format, w, n, k, x, m, plain_out(y, n), addend, mode, workspace,
                     workspace_bytes, device_error_flag(dev), MGB_KERNEL_AUTO,
                     static_cast<cudaStream_t>(stream));
}

mgb_status mgb_qmatmul_bf16(int32_t format, const void *w, uint64_t n, uint64_t k, const void *xb,
                            uint64_t m, float *y, const float *addend, uint64_t addend_len,
                            void *stream) {
  if (!format_supported(format))
    return fail(MGB_UNSUPPORTED, "packed format %d is not executed by this Provider", format);
  if (!gemm_supported(format, m, n, k))
    return fail(MGB_UNSUPPORTED, "tensor-core GEMM needs k %% 256 == 0 (got %llu)",
                (unsigned long long)k);
  if (!w || !xb || !y) return fail(MGB_INVALID_ARGUMENT, "null device pointer");
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(xb) & 15))
    return fail(MGB_INVALID_ARGUMENT, "weight and activation pointers must be 16-byte aligned");
  int mode = 0;
  if (addend) {
    if (addend_len == n) mode = 1;
    else if (addend_len == m * n) mode = 2;
    else return fail(MGB_INVALID_ARGUMENT, "addend has %llu values, expected %llu or %llu",
                     (unsigned long long)addend_len, (unsigned long long)n,
                     (unsigned long long)(m * n));
  }
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = launch_gemm_bf16(format, w, n, k, xb, m, plain_out(y, n), addend, mode,
                                   device_error_flag(dev), device_sms(dev),
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "GEMM launch");
}

mgb_status mgb_embedding(int32_t format, const void *w, uint64_t stored_rows, uint64_t stored_cols,
                         int32_t transposed, const float *ids, uint64_t count, int32_t has_scale,
                         float scale, float *out, uint32_t *bad, void *stream) {
  mgb_status s = check_packed_shape(format, stored_rows, stored_cols);
  if (s != MGB_OK) return s == MGB_DECLINED ? fail(MGB_UNSUPPORTED, "%s", mgb_last_error()) : s;
  if (count && (!w || !ids || !out)) return fail(MGB_INVALID_ARGUMENT, "null device pointer");
  cudaError_t e = launch_embedding(format, w, stored_rows, stored_cols, transposed != 0, ids, count,
                                   has_scale != 0, scale, out, bad,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "embedding launch");
}

mgb_status mgb_dequantize(int32_t format, const void *w, uint64_t stored_rows, uint64_t stored_cols,
                          float *out, void *stream) {
  mgb_status s = check_packed_shape(format, stored_rows, stored_cols);
  if (s != MGB_OK) return s == MGB_DECLINED ? fail(MGB_UNSUPPORTED, "%s", mgb_last_error()) : s;
  if (!w || !out) return fail(MGB_INVALID_ARGUMENT, "null device pointer");
  cudaError_t e = launch_dequantize(format, w, stored_rows, stored_cols, out,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "dequantize launch");
}

mgb_status mgb_qmatmul_input_major(int32_t format, const void *w, uint64_t stored_rows,
                                   uint64_t stored_cols, const float *x, uint64_t m, float *y,
                                   void *stream) {
  mgb_status s = check_packed_shape(format, stored_rows, stored_cols);
  if (s != MGB_OK) return s == MGB_DECLINED ? fail(MGB_UNSUPPORTED, "%s", mgb_last_error()) : s;
  if ((m && stored_cols) && (!w || !x || !y)) return fail(MGB_INVALID_ARGUMENT, "null device pointer");
  cudaError_t e = launch_input_major(format, w, stored_rows, stored_cols, x, m, y,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "input-major launch");
}

mgb_status mgb_matmul_f32(const float *a, uint64_t a_rows, uint64_t a_cols, const float *b,
                          uint64_t b_rows, uint64_t b_cols, int32_t transpose_a,
                          int32_t transpose_b, float *out, void *stream) {
  const uint64_t k = transpose_a ? a_rows : a_cols, k2 = transpose_b ? b_cols : b_rows;
  if (k != k2)
    return fail(MGB_EXECUTION_FAILED, "matmul inner dimension mismatch: %llu vs %llu",
                (unsigned long long)k, (unsigned long long)k2);
  cudaError_t e = launch_matmul_f32(a, a_rows, a_cols, b, b_rows, b_cols, transpose_a, transpose_b,
                                    out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "matmul launch");
}

mgb_status mgb_quantize_rows(const float *x, uint64_t len, int8_t *values, float *scales,
                             int32_t *sums, void *stream) {
  if (len % 32) return fail(MGB_INVALID_ARGUMENT, "length %llu is not a multiple of 32", (unsigned long long)len);
  cudaError_t e = launch_quantize_rows(x, len, values, scales, sums, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "quantize launch");
}

mgb_status mgb_take_device_error(int32_t device, int32_t *code) {
  if (!code) return fail(MGB_INVALID_ARGUMENT, "null code pointer");
  *code = 0;
  if (device < 0 || device >= 64) return fail(MGB_INVALID_ARGUMENT, "device %d out of range", device);
  int prev = 0;
  mgb_status s = take_static_scratch_error(device, &prev);
  if (s != MGB_OK) return s;
  if (int *flag = existing_error_flag(device)) {
    int word = 0;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMemcpy(&word, flag, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error flag");
    if (word) cudaMemset(flag, 0, sizeof(int));
    if (!prev) prev = word;
  }
  *code = prev;
  return MGB_OK;
}

}  // extern "C"
