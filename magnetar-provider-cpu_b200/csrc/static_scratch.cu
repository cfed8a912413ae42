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

// The device error word of the calls above (1 = a bounded device wait gave
// up), beside the array: read and cleared by mgb_take_device_error.
__device__ static int g_static_error;

std::mutex g_mu;
void *g_scratch_ptr[64] = {};
int *g_error_ptr[64] = {};

// The device addresses of the array and of the error word for `device` (the
// current device), resolved once per device; host code may not use the
// symbols themselves as device addresses.
mgb_status scratch_address(int device, void **out, int **err) {
  if (device < 0 || device >= 64) return fail(MGB_INVALID_ARGUMENT, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[device]) {
    void *p = nullptr, *q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    e = cudaGetSymbolAddress(&q, g_static_error);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static error word)");
    g_error_ptr[device] = static_cast<int *>(q);
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  *err = g_error_ptr[device];
  return MGB_OK;
}

}  // namespace

// Reads and clears the error word of the static-scratch calls on `device`
// (0 when that device has made none).  Allocates nothing.
mgb_status take_static_scratch_error(int device, int *code) {
  *code = 0;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (device < 0 || device >= 64 || !g_error_ptr[device]) return MGB_OK;
  }
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(code, g_static_error, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "reading the static scratch error word");
  if (*code) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_static_error, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the static scratch error word");
  }
  return MGB_OK;
}

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
  int *err = nullptr;
  s = scratch_address(dev, &scratch, &err);
  if (s != MGB_OK) return s;
  // The scratch is fully rewritten by each call before it is read (nothing in
  // it has to start at zero).  A bounded device wait that expires records 1 in
  // the static error word (mgb_take_device_error reads it).
  return run_qmatmul(format, w, n, k, x, m, plain_out(y, n), addend, mode, scratch,
                     MGB_STATIC_SCRATCH_BYTES, err, MGB_KERNEL_AUTO,
                     static_cast<cudaStream_t>(stream));
}
