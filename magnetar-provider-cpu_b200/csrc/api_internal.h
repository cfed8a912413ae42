// Host-side helpers shared by api.cpp and provider.cpp.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/magnetar_b200.h"
#include "outspec.h"

namespace mgb {

// Records `fmt` as this thread's last error and returns `status`.
mgb_status fail(mgb_status status, const char *fmt, ...);
mgb_status cuda_fail(cudaError_t e, const char *what);
void clear_error();

bool format_supported(int32_t format);
uint64_t format_block_elements(int32_t format);
uint64_t ggml_bytes(int32_t format, uint64_t rows, uint64_t cols);
// bytes of the device layout (quant plane + scale plane)
uint64_t device_bytes(int32_t format, uint64_t rows, uint64_t cols);
mgb_status check_packed_shape(int32_t format, uint64_t rows, uint64_t cols);
int *device_error_flag(int device);
// the error word of mgb_qmatmul_static_scratch on `device` (read and cleared)
mgb_status take_static_scratch_error(int device, int *code);

mgb_status validate_qmatmul(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                            uint64_t m, float *y);
uint64_t qmatmul_scratch_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k);
uint64_t qmatmul_min_scratch_bytes(int32_t format, uint64_t m, uint64_t n, uint64_t k);
// y = x W^T (+ addend) written where `out` says: one rank's y[m, n] or, for a
// tensor-parallel call, columns col0.. of every rank's y[m, ldy].
mgb_status run_qmatmul(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                       uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                       void *workspace, uint64_t workspace_bytes, int *err, int kernel_pref,
                       cudaStream_t stream);

}  // namespace mgb
