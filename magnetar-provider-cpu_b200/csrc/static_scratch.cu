// mgb_qmatmul_static_scratch: the packed-weight matmul for callers that must
// not allocate device memory.  The tensor-core GEMM stages its bf16 copy of
// the activations in scratch memory; here that scratch is a fixed array in the
// library's own device image instead of a caller-provided or cudaMalloc'd
// buffer.  Every GPU that loads the library holds the array until the process
// exits.
#include <mutex>

#include "../../include/magnetar_b200.h"
#include "api_internal.h"
#include "common.cuh"
#include "kernels.h"

namespace mgb {
namespace {

// MGB_STATIC_SCRATCH_BYTES bytes: room for the bf16 activations of any m x k
// with m * k <= 4,194,304 (e.g. 512 x 8192 or 1024 x 4096).
__device__ __align__(256) static unsigned char g_static_scratch[MGB_STATIC_SCRATCH_BYTES];

std::mutex g_mu;
void *g_scratch_ptr[64] = {};

// The array's device address for `device` (the current device), resolved once
// per device; host code may not use the symbol itself as a device address.
mgb_status scratch_address(int device, void **out) {
  if (device < 0 || device >= 64) return fail(MGB_INVALID_ARGUMENT, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return MGB_OK;
}

}  // namespace
}  // namespace mgb

using namespace mgb;

extern "C" mgb_status mgb_qmatmul_static_scratch(int32_t format, const void *w, uint64_t n,
                                                 uint64_t k, const float *x, uint64_t m,
                                                 float *y, const float *addend,
                                                 uint64_t addend_len, void *stream) {
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
  const uint64_t need = qmatmul_min_scratch_bytes(format, m, n, k);
  if (need > MGB_STATIC_SCRATCH_BYTES)
    return fail(MGB_INVALID_ARGUMENT,
                "m=%llu x k=%llu needs %llu bytes of scratch; the static scratch holds %llu "
                "(m * k must be <= %llu)",
                (unsigned long long)m, (unsigned long long)k, (unsigned long long)need,
                (unsigned long long)MGB_STATIC_SCRATCH_BYTES,
                (unsigned long long)(MGB_STATIC_SCRATCH_BYTES / 2));
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  void *scratch = nullptr;
  s = scratch_address(dev, &scratch);
  if (s != MGB_OK) return s;
  // The scratch is fully rewritten by each call before it is read (nothing in
  // it has to start at zero).  No error word is passed: a bounded device wait
  // that expires leaves y unspecified and is not reported through this call.
  return run_qmatmul(format, w, n, k, x, m, plain_out(y, n), addend, mode, scratch,
                     MGB_STATIC_SCRATCH_BYTES, nullptr, MGB_KERNEL_AUTO,
                     static_cast<cudaStream_t>(stream));
}
