// Tensor parallelism over output columns: the C ABI of the fused all-gather.
//
// Each rank's packed matmul stores its columns into every rank's y (IPC
// mappings of the peers' buffers over NVLink) with plain stores; a one-CTA
// kernel after the call's last launch publishes the call's epoch into every
// rank's done words (OutSpec).  A rank then waits for all ranks' epochs with
// one small stream-ordered kernel, or inside the first kernel of its next
// call.  The
// column split is the reference's per-thread unit of `packed_matmul`
// (src/native/mod.rs:135-150): whole stored rows, so no block is cut.

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/magnetar_b200.h"
#include "api_internal.h"
#include "common.cuh"
#include "kernels.h"

namespace mgb {

static_assert(MGB_MAX_TP == MAX_TP, "C ABI and kernel rank limits differ");
static_assert(sizeof(cudaIpcMemHandle_t) == MGB_IPC_HANDLE_BYTES, "IPC handle size");
static_assert(MGB_TP_EPOCH_OFFSET == 4 * TP_EPOCH_WORD, "epoch word offset");

// One warp waits until every rank's done word has reached the epoch
// (poll_epoch); with epoch_word set (device epochs) the epoch is the word's
// current value, which the call it waits for advanced as it published.
__global__ void mgb_tp_wait_kernel(const uint32_t *done, int world, uint32_t epoch,
                               const uint32_t *epoch_word, uint64_t timeout_ns, int *err) {
  // The next kernel on the stream (a programmatic dependent, e.g. the next
  // projection's GEMV) may launch now and stream its weights while this wait
  // polls; its griddepcontrol.wait still holds its reads of x until this grid
  // has completed.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x;
  if (epoch_word) epoch = *(volatile const uint32_t *)epoch_word;
  const bool reached = poll_epoch(done, world, epoch, timeout_ns, lane);
  if (!__all_sync(0xffffffffu, reached) && lane == 0) record_error(err, ERR_WAIT_TIMEOUT);
}

// Publishes a tensor-parallel call: a programmatic dependent of the call's last
// launch.  Its griddepcontrol.wait returns once that grid has completed and its
// memory operations, the stores into every rank's y included, have been
// performed (each launch of the call waited for the one before it in the same
// way).  Thread 0 then advances the device epoch (if used) and stores the
// epoch into word `rank` of every rank's done words.  Those stores are
// relaxed (system scope): they are issued only after the data they announce
// has been performed at every rank's memory, so no peer can see an epoch
// before its columns.  Publishing at the kernel boundary replaces a
// system-scope fence in every CTA of the call (each such fence on the critical
// path cost ~5 us per call on B200), and the relaxed store a release (another
// ~1 to 2.6 us per call, one GPU / two GPUs).
__global__ void mgb_tp_publish_kernel(const OutSpec o) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x != 0) return;
  uint32_t epoch = o.epoch;
  if (o.epoch_word) {
    epoch = *(volatile const uint32_t *)o.epoch_word + 1u;
    *(volatile uint32_t *)o.epoch_word = epoch;  // the next call publishes epoch + 1
  }
  for (int r = 0; r < o.world; ++r)
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(o.done_ranks[r] + o.rank), "r"(epoch)
                 : "memory");
}

static cudaError_t launch_publish(const OutSpec &spec, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mgb_tp_publish_kernel, spec);
}

static mgb_status to_outspec(const mgb_tp_out *o, uint64_t n, OutSpec &spec) {
  if (!o) return fail(MGB_INVALID_ARGUMENT, "null tensor-parallel output");
  if (o->world < 1 || o->world > MGB_MAX_TP || o->rank < 0 || o->rank >= o->world)
    return fail(MGB_INVALID_ARGUMENT, "rank %d of world %d (at most %d ranks)", o->rank, o->world,
                MGB_MAX_TP);
  if (!o->cta_counter) return fail(MGB_INVALID_ARGUMENT, "null CTA counter");
  if (o->col0 + n > o->ldy)
    return fail(MGB_INVALID_ARGUMENT, "columns %llu..%llu exceed the output row of %llu",
                (unsigned long long)o->col0, (unsigned long long)(o->col0 + n),
                (unsigned long long)o->ldy);
  spec = OutSpec{};
  for (int r = 0; r < o->world; ++r) {
    if (!o->y[r] || !o->done[r])
      return fail(MGB_INVALID_ARGUMENT, "null output or done pointer of rank %d", r);
    spec.y_ranks[r] = o->y[r];
    spec.done_ranks[r] = o->done[r];
  }
  spec.cta_counter = o->cta_counter;
  // epoch 0: device epochs, from this rank's epoch word (the word after the
  // reserved word `cta_counter` points at)
  spec.epoch_word = o->epoch == 0 ? o->cta_counter + 1 : nullptr;
  if (o->wait_done) {
    if (o->wait_world < 1 || o->wait_world > MGB_MAX_TP)
      return fail(MGB_INVALID_ARGUMENT, "input wait over %d ranks (1..%d)", o->wait_world,
                  MGB_MAX_TP);
    spec.wait_done = o->wait_done;
    spec.wait_epoch = o->wait_epoch;
    spec.wait_world = o->wait_world;
    spec.wait_timeout_ns = (uint64_t)(o->wait_timeout_ms ? o->wait_timeout_ms : 2000) * 1000000ull;
  }
  spec.ldy = o->ldy;
  spec.col0 = o->col0;
  spec.epoch = o->epoch;
  spec.world = o->world;
  spec.rank = o->rank;
  return MGB_OK;
}

}  // namespace mgb

using namespace mgb;

extern "C" {

mgb_status mgb_device_alloc(uint64_t bytes, void **out) {
  if (!out) return fail(MGB_INVALID_ARGUMENT, "null output pointer");
  *out = nullptr;
  if (bytes == 0) return fail(MGB_INVALID_ARGUMENT, "zero-byte allocation");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "zero-filling an allocation");
  }
  *out = p;
  return MGB_OK;
}

mgb_status mgb_device_free(void *ptr) {
  if (!ptr) return MGB_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "cudaFree");
}

mgb_status mgb_ipc_handle(void *ptr, uint8_t *handle_out) {
  if (!ptr || !handle_out) return fail(MGB_INVALID_ARGUMENT, "null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  return MGB_OK;
}

mgb_status mgb_ipc_open(const uint8_t *handle, void **out) {
  if (!handle || !out) return fail(MGB_INVALID_ARGUMENT, "null pointer");
  *out = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *out = p;
  return MGB_OK;
}

mgb_status mgb_ipc_close(void *mapped) {
  if (!mapped) return MGB_OK;
  cudaError_t e = cudaIpcCloseMemHandle(mapped);
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

mgb_status mgb_qmatmul_tp(int32_t format, const void *w, uint64_t n, uint64_t k, const float *x,
                          uint64_t m, const mgb_tp_out *out, const float *addend,
                          uint64_t addend_len, void *workspace, uint64_t workspace_bytes,
                          void *stream) {
  OutSpec spec;
  mgb_status s = to_outspec(out, n, spec);
  if (s != MGB_OK) return s;
  s = validate_qmatmul(format, w, n, k, x, m, spec.y_ranks[spec.rank]);
  if (s != MGB_OK) return s;
  if (m == 0 || n == 0)
    return fail(MGB_INVALID_ARGUMENT, "an empty tensor-parallel call publishes nothing");
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
  s = run_qmatmul(format, w, n, k, x, m, spec, addend, mode, workspace, workspace_bytes,
                  device_error_flag(dev), MGB_KERNEL_AUTO, static_cast<cudaStream_t>(stream));
  if (s != MGB_OK) return s;
  cudaError_t e = launch_publish(spec, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "publish launch");
}

mgb_status mgb_tp_wait(const uint32_t *done, int32_t world, uint32_t epoch, uint32_t timeout_ms,
                       void *stream) {
  if (!done) return fail(MGB_INVALID_ARGUMENT, "null done words");
  if (world < 1 || world > MGB_MAX_TP)
    return fail(MGB_INVALID_ARGUMENT, "world %d (at most %d ranks)", world, MGB_MAX_TP);
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t ns = (uint64_t)(timeout_ms ? timeout_ms : 2000) * 1000000ull;
  // epoch 0: device epochs (this rank's epoch word in its synchronisation words)
  const uint32_t *epoch_word = epoch == 0 ? done + TP_EPOCH_WORD : nullptr;
  mgb_tp_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(done, world, epoch, epoch_word,
                                                                  ns, device_error_flag(dev));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MGB_OK : cuda_fail(e, "wait launch");
}

}  // extern "C"
