// The B200 Provider object behind the C ABI: a counterpart of the reference's
// `NativeCpuExecutor` / `NativeCpuProvider` (src/native/mod.rs:465-947) with
// device-resident storage.
//
// - f32 tensors and packed weights live in device memory, keyed by resource
//   id; a packed weight is held in the device layout (same bytes as its ggml
//   blocks, rearranged at write time).
// - `submit_kernel` validates an invocation, enqueues it on the Provider's
//   stream and records an event; `complete_kernel` waits for that event and
//   hands the result out exactly once (src/lib.rs:2301-2356).
// - Observations are kept like the reference's bounded log (capacity 4096,
//   trimmed at twice that, src/lib.rs:171, :1848-1868).
// Every entry point takes the Provider's mutex, so they are thread-safe (the
// reference's trait takes `&self` everywhere: calls may come from several
// threads).  Tensor uploads and downloads run on copy streams of their own and
// release the mutex while the host waits for them, so one thread's download
// overlaps another thread's upload and kernels (PCIe carries both directions
// at once); kernels stay on the one compute stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/magnetar_b200.h"
#include "api_internal.h"
#include "kernels.h"

namespace {

using namespace mgb;

constexpr const char *PROVIDER_NAME = "magnetar:provider/b200-native";
constexpr const char *PROVIDER_VERSION = "0.1.0";
constexpr const char *PROVIDER_VENDOR = "magnetar";
constexpr size_t OBS_CAPACITY = 4096;

struct DevBuf {
  void *ptr = nullptr;
  uint64_t bytes = 0;
};

struct Tensor {
  std::vector<uint64_t> shape;
  DevBuf buf;
  uint64_t elems() const {
    uint64_t e = 1;
    for (uint64_t d : shape) e *= d;
    return e;
  }
};

struct Packed {
  int32_t format = 0;
  uint64_t stored_rows = 0, stored_cols = 0;
  bool transposed = false;
  DevBuf buf;  // device layout
  std::vector<uint64_t> logical_shape() const {
    return transposed ? std::vector<uint64_t>{stored_cols, stored_rows}
                      : std::vector<uint64_t>{stored_rows, stored_cols};
  }
};

struct Execution {
  int32_t status = MGB_OK;
  std::string reason;
  std::string kernel;
  cudaEvent_t start = nullptr, stop = nullptr;
};

struct ProfileEntry {
  uint64_t count = 0;
  double ms = 0.0;
};

}  // namespace

struct mgb_provider {
  mgb_settings settings{};
  int sms = 148;
  cudaStream_t stream = nullptr;  // kernels, allocations and frees
  cudaStream_t h2d = nullptr;     // tensor uploads
  cudaStream_t d2h = nullptr;     // tensor downloads
  std::mutex mu;
  // Buffers that a download reads with the mutex released, with the number of
  // such downloads; freeing one of them waits in `deferred` until the last
  // download ends.
  std::map<void *, int> reading;
  std::vector<DevBuf> deferred;
  std::map<std::string, Tensor> storage;
  std::map<std::string, Packed> packed;
  std::map<uint64_t, Execution> executions;
  uint64_t next_handle = 1;
  std::deque<mgb_observation> observations;
  uint64_t obs_seq = 0;
  DevBuf workspace;
  cudaMemPool_t pool = nullptr;  // this Provider's stream-ordered device memory
  int *dev_err = nullptr;
  uint32_t *dev_bad = nullptr;  // first invalid token position of an embedding lookup
  uint64_t materializations = 0;
  double materialize_ms = 0.0;
  std::map<std::string, ProfileEntry> profile;
  bool shut_down = false;
};

namespace {

void observe(mgb_provider *p, int32_t kind, const std::string &kernel, const std::string &detail) {
  if (p->observations.size() >= 2 * OBS_CAPACITY)
    p->observations.erase(p->observations.begin(), p->observations.begin() + OBS_CAPACITY);
  mgb_observation o{};
  o.sequence = p->obs_seq++;
  o.kind = kind;
  snprintf(o.kernel, sizeof o.kernel, "%s", kernel.c_str());
  snprintf(o.detail, sizeof o.detail, "%s", detail.c_str());
  p->observations.push_back(o);
}

// Device buffers come from the Provider's own memory pool, in the order of its
// stream: a free is queued behind the work that still reads the buffer (no
// host synchronisation), and the pool keeps freed memory for the next
// allocation of the step (no cudaMalloc / cudaFree per tensor).
void free_buf(mgb_provider *p, DevBuf &b) {
  if (b.ptr && p->reading.count(b.ptr)) p->deferred.push_back(b);
  else if (b.ptr) cudaFreeAsync(b.ptr, p->stream);
  b.ptr = nullptr;
  b.bytes = 0;
}

// Ends one download of `ptr` (mutex held): the last one frees the buffer if it
// was released meanwhile.  The copy has completed (the host waited for it),
// so the free needs no ordering against the download stream.
void end_read(mgb_provider *p, void *ptr) {
  auto r = p->reading.find(ptr);
  if (r == p->reading.end() || --r->second > 0) return;
  p->reading.erase(r);
  for (size_t i = 0; i < p->deferred.size();) {
    if (p->deferred[i].ptr == ptr) {
      cudaFreeAsync(ptr, p->stream);
      p->deferred.erase(p->deferred.begin() + i);
    } else {
      ++i;
    }
  }
}

// One host<->device copy on `copy_stream`, ordered after everything already
// queued on the compute stream (the buffer's stream-ordered allocation, the
// kernel that produced it, kernels that still read it).  The mutex is released
// while the host waits for the copy and held again on return.
cudaError_t copy_unlocked(mgb_provider *p, std::unique_lock<std::mutex> &lock,
                          cudaStream_t copy_stream, void *dst, const void *src, uint64_t bytes,
                          cudaMemcpyKind kind) {
  cudaEvent_t ready = nullptr, done = nullptr;
  cudaError_t e = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventRecord(ready, p->stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(copy_stream, ready, 0);
  bool queued = false;
  if (e == cudaSuccess) {
    e = cudaMemcpyAsync(dst, src, bytes, kind, copy_stream);
    queued = e == cudaSuccess;
  }
  if (e == cudaSuccess) e = cudaEventRecord(done, copy_stream);
  lock.unlock();
  if (e == cudaSuccess) e = cudaEventSynchronize(done);
  else if (queued) cudaStreamSynchronize(copy_stream);  // nothing may outlive the call
  lock.lock();
  if (ready) cudaEventDestroy(ready);
  if (done) cudaEventDestroy(done);
  return e;
}

// Reuses `b` when it already holds `bytes`, else reallocates; fallible.  An
// allocation the device cannot satisfy returns the pool's idle memory to the
// device and tries once more before it is denied.
mgb_status ensure_buf(mgb_provider *p, DevBuf &b, uint64_t bytes) {
  if (b.ptr && b.bytes == bytes) return MGB_OK;
  if (b.ptr) free_buf(p, b);
  if (!bytes) return MGB_OK;
  void *ptr = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&ptr, bytes, p->pool, p->stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaStreamSynchronize(p->stream);
    cudaMemPoolTrimTo(p->pool, 0);
    e = cudaMallocFromPoolAsync(&ptr, bytes, p->pool, p->stream);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MGB_MEMORY_DENIED, "device allocation of %llu bytes denied: %s",
                (unsigned long long)bytes, cudaGetErrorString(e));
  }
  b.ptr = ptr;
  b.bytes = bytes;
  return MGB_OK;
}

bool forget_packed(mgb_provider *p, const std::string &id) {
  auto it = p->packed.find(id);
  if (it == p->packed.end()) return false;
  free_buf(p, it->second.buf);
  p->packed.erase(it);
  return true;
}

bool forget_tensor(mgb_provider *p, const std::string &id) {
  auto it = p->storage.find(id);
  if (it == p->storage.end()) return false;
  free_buf(p, it->second.buf);
  p->storage.erase(it);
  return true;
}

// Stores a device buffer of f32 values under `id` (taking the buffer).
void put_tensor(mgb_provider *p, const std::string &id, std::vector<uint64_t> shape, DevBuf buf) {
  forget_tensor(p, id);
  Tensor t;
  t.shape = std::move(shape);
  t.buf = buf;
  p->storage[id] = t;
}

// A packed weight's logical f32 values in a new device buffer (`expand`,
// src/native/mod.rs:196-204, counted as a materialisation).
mgb_status expand(mgb_provider *p, const Packed &w, DevBuf &out) {
  const auto t0 = std::chrono::steady_clock::now();
  const uint64_t elems = w.stored_rows * w.stored_cols;
  DevBuf stored;
  mgb_status s = ensure_buf(p, stored, elems * 4);
  if (s != MGB_OK) return s;
  cudaError_t e = launch_dequantize(w.format, w.buf.ptr, w.stored_rows, w.stored_cols,
                                    static_cast<float *>(stored.ptr), p->stream);
  if (e != cudaSuccess) {
    free_buf(p, stored);
    return cuda_fail(e, "dequantize launch");
  }
  if (!w.transposed) {
    out = stored;
  } else {
    // logical [stored_cols, stored_rows]: the transpose of the stored rows
    s = ensure_buf(p, out, elems * 4);
    if (s != MGB_OK) {
      free_buf(p, stored);
      return s;
    }
    e = launch_transpose(static_cast<const float *>(stored.ptr), w.stored_rows, w.stored_cols,
                         static_cast<float *>(out.ptr), p->stream);
    free_buf(p, stored);
    if (e != cudaSuccess) return cuda_fail(e, "transpose launch");
  }
  p->materializations++;
  p->materialize_ms +=
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  return MGB_OK;
}

struct Operand {
  const float *ptr = nullptr;
  uint64_t rows = 0, cols = 0;
  std::vector<uint64_t> shape;
  DevBuf owned;  // set when the operand was materialised for this call
};

mgb_status input_f32(mgb_provider *p, const char *id, size_t index, Operand &out) {
  if (!id) return fail(MGB_EXECUTION_FAILED, "missing input at index %zu", index);
  auto it = p->storage.find(id);
  if (it != p->storage.end()) {
    out.ptr = static_cast<const float *>(it->second.buf.ptr);
    out.shape = it->second.shape;
  } else {
    auto pk = p->packed.find(id);
    if (pk == p->packed.end())
      return fail(MGB_EXECUTION_FAILED, "no materialized data for input resource %s", id);
    mgb_status s = expand(p, pk->second, out.owned);
    if (s != MGB_OK) return s;
    out.ptr = static_cast<const float *>(out.owned.ptr);
    out.shape = pk->second.logical_shape();
  }
  if (out.shape.size() == 2) {
    out.rows = out.shape[0];
    out.cols = out.shape[1];
  } else if (out.shape.size() == 1) {
    out.rows = 1;
    out.cols = out.shape[0];
  }
  return MGB_OK;
}

mgb_status ensure_workspace(mgb_provider *p, uint64_t bytes) {
  if (p->workspace.bytes >= bytes) return MGB_OK;
  return ensure_buf(p, p->workspace, bytes);
}

std::string shape_str(const std::vector<uint64_t> &s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

// The matmul family on the Provider's stream (`NativeState::matmul`,
// src/native/mod.rs:206-236).  Writes the output tensor on success.
mgb_status run_matmul(mgb_provider *p, const std::string &kernel, const mgb_kernel_attrs &attrs,
                      const char *const *inputs, int32_t n_inputs, const char *output) {
  Operand a;
  mgb_status s = input_f32(p, n_inputs > 0 ? inputs[0] : nullptr, 0, a);
  if (s != MGB_OK) return s;
  if (a.shape.size() != 2)
    return fail(MGB_EXECUTION_FAILED, "matmul expects rank-2 activations, got %s",
                shape_str(a.shape).c_str());
  if (attrs.accumulation_dtype != MGB_DTYPE_F32)
    return fail(MGB_DTYPE_UNSUPPORTED,
                "the B200 Provider only accumulates in f32; requested dtype %d",
                attrs.accumulation_dtype);
  const char *wid = n_inputs > 1 ? inputs[1] : nullptr;
  if (!wid) return fail(MGB_EXECUTION_FAILED, "missing input at index 1");
  DevBuf product;
  std::vector<uint64_t> out_shape;
  auto pk = p->packed.find(wid);
  int kernel_pref = p->settings.kernel;

  // int8 activations: the rows as the reference's int8 path sees them.
  DevBuf rounded;
  const float *act = a.ptr;
  if (p->settings.int8_activations && a.rows * a.cols % 32 == 0) {
    s = ensure_buf(p, rounded, a.rows * a.cols * 4);
    if (s != MGB_OK) return s;
    cudaError_t e = launch_int8_rounded(a.ptr, a.rows * a.cols, static_cast<float *>(rounded.ptr),
                                        p->stream);
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    act = static_cast<const float *>(rounded.ptr);
  }

  if (pk != p->packed.end() && !attrs.transpose_a && pk->second.transposed != (bool)attrs.transpose_b) {
    const Packed &w = pk->second;
    const uint64_t m = a.rows, k = a.cols, n = w.stored_rows;
    if (k != w.stored_cols || k % 32)
      return fail(MGB_EXECUTION_FAILED,
                  "packed matmul: activations have %llu columns, the weight's stored rows %llu",
                  (unsigned long long)k, (unsigned long long)w.stored_cols);
    s = ensure_buf(p, product, m * n * 4);
    if (s != MGB_OK) return s;
    // scratch for the GEMM's bf16 activations (and its split-K partials)
    uint64_t ws = qmatmul_scratch_bytes(w.format, m, n, k);
    if (gemm_supported(w.format, m, n, k) && kernel_pref == MGB_KERNEL_GEMM)
      ws = gemm_workspace_bytes_preferred(w.format, m, n, k);
    if (kernel_pref == MGB_KERNEL_GEMV) ws = 0;
    if (ws) {
      s = ensure_workspace(p, ws);
      if (s != MGB_OK) return s;
    }
    s = run_qmatmul(w.format, w.buf.ptr, n, k, act, m,
                    plain_out(static_cast<float *>(product.ptr), n), nullptr, 0, p->workspace.ptr,
                    p->workspace.bytes, p->dev_err, kernel_pref, p->stream);
    if (s != MGB_OK) {
      free_buf(p, product);
      return s;
    }
    out_shape = {m, n};
  } else if (pk != p->packed.end() && !attrs.transpose_a) {
    // stored rows are the input rows: the input-major branch (packed_axpy)
    const Packed &w = pk->second;
    const uint64_t m = a.rows, k = a.cols, n = w.stored_cols;
    if (k != w.stored_rows)
      return fail(MGB_EXECUTION_FAILED,
                  "packed matmul: activations have %llu columns, the weight %llu stored rows",
                  (unsigned long long)k, (unsigned long long)w.stored_rows);
    s = ensure_buf(p, product, m * n * 4);
    if (s != MGB_OK) return s;
    cudaError_t e = launch_input_major(w.format, w.buf.ptr, w.stored_rows, w.stored_cols, act, m,
                                       static_cast<float *>(product.ptr), p->stream);
    if (e != cudaSuccess) {
      free_buf(p, product);
      return cuda_fail(e, "input-major launch");
    }
    out_shape = {m, n};
  } else {
    // an f32 weight, or transpose_a on an expanded packed weight: dense matmul
    Operand b;
    s = input_f32(p, wid, 1, b);
    if (s != MGB_OK) return s;
    if (b.shape.size() != 2)
      return fail(MGB_EXECUTION_FAILED, "matmul expects a rank-2 weight, got %s",
                  shape_str(b.shape).c_str());
    const uint64_t m = attrs.transpose_a ? a.cols : a.rows, k = attrs.transpose_a ? a.rows : a.cols;
    const uint64_t k2 = attrs.transpose_b ? b.cols : b.rows, n = attrs.transpose_b ? b.rows : b.cols;
    if (k != k2) {
      free_buf(p, b.owned);
      return fail(MGB_EXECUTION_FAILED, "matmul inner dimension mismatch: %llu vs %llu",
                  (unsigned long long)k, (unsigned long long)k2);
    }
    s = ensure_buf(p, product, m * n * 4);
    if (s == MGB_OK) {
      cudaError_t e = launch_matmul_f32(act, a.rows, a.cols, b.ptr, b.rows, b.cols,
                                        attrs.transpose_a, attrs.transpose_b,
                                        static_cast<float *>(product.ptr), p->stream);
      if (e != cudaSuccess) s = cuda_fail(e, "matmul launch");
    }
    if (b.owned.ptr) {
      free_buf(p, b.owned);
    }
    if (s != MGB_OK) {
      free_buf(p, product);
      return s;
    }
    out_shape = {m, n};
  }
  if (a.owned.ptr) {
    free_buf(p, a.owned);
  }
  if (rounded.ptr) {
    free_buf(p, rounded);
  }

  // matmul-bias: add(product, bias); matmul-residual: add(residual, product)
  if (kernel == "matmul-bias" || kernel == "matmul-residual") {
    Operand c;
    s = input_f32(p, n_inputs > 2 ? inputs[2] : nullptr, 2, c);
    if (s != MGB_OK) {
      free_buf(p, product);
      return s;
    }
    const uint64_t len = out_shape[0] * out_shape[1], cols = out_shape[1];
    uint64_t clen = 1;
    for (uint64_t d : c.shape) clen *= d;
    const bool same = c.shape == out_shape;
    const bool row = c.shape == std::vector<uint64_t>{cols} ||
                     c.shape == std::vector<uint64_t>{1, cols};
    if (kernel == "matmul-bias" && !same && !row) {
      free_buf(p, product);
      return fail(MGB_EXECUTION_FAILED,
                  "add expects b to match a's shape %s or broadcast as [%llu]/[1, %llu], got %s",
                  shape_str(out_shape).c_str(), (unsigned long long)cols,
                  (unsigned long long)cols, shape_str(c.shape).c_str());
    }
    if (kernel == "matmul-residual" && !same) {
      free_buf(p, product);
      return fail(MGB_EXECUTION_FAILED, "shape mismatch: %s vs %s", shape_str(c.shape).c_str(),
                  shape_str(out_shape).c_str());
    }
    cudaError_t e = launch_add(static_cast<float *>(product.ptr), len, c.ptr, clen, cols, p->stream);
    if (c.owned.ptr) {
      free_buf(p, c.owned);
    }
    if (e != cudaSuccess) {
      free_buf(p, product);
      return cuda_fail(e, "epilogue launch");
    }
  }
  forget_packed(p, output);
  put_tensor(p, output, out_shape, product);
  return MGB_OK;
}

// An f32 as Rust's `Display` writes it: the shortest digits that read back to
// the same value, in positional notation ("3", "-0", "2.5", "0.0001",
// "NaN", "inf").  The reference formats token ids in its errors this way.
std::string rust_f32(float v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v < 0 ? "-inf" : "inf";
  const std::string sign = std::signbit(v) ? "-" : "";
  const float a = std::fabs(v);
  if (a == 0.0f) return sign + "0";
  char buf[64];
  for (int prec = 0; prec < 9; ++prec) {
    snprintf(buf, sizeof buf, "%.*e", prec, (double)a);
    if (strtof(buf, nullptr) == a) break;
  }
  std::string digits;
  const char *c = buf;
  for (; *c && *c != 'e'; ++c)
    if (*c >= '0' && *c <= '9') digits += *c;
  const int exp10 = atoi(c + 1);  // value = d.ddd x 10^exp10
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string r;
  if (exp10 >= 0) {
    const size_t int_len = (size_t)exp10 + 1;
    if (digits.size() <= int_len) r = digits + std::string(int_len - digits.size(), '0');
    else r = digits.substr(0, int_len) + "." + digits.substr(int_len);
  } else {
    r = "0." + std::string((size_t)(-exp10 - 1), '0') + digits;
  }
  return sign + r;
}

// `embedding` (src/native/mod.rs:389-417, dispatch and "scale" :432-450):
// inputs [table, ids]; a packed table is read in place (`NativeState::
// embedding`), an f32 one gathered (`f32_embedding`, :238-263).  Output
// [ids count, dim].
mgb_status run_embedding(mgb_provider *p, const mgb_kernel_attrs &attrs, const char *const *inputs,
                         int32_t n_inputs, const char *output) {
  const char *tid = n_inputs > 0 ? inputs[0] : nullptr;
  if (!tid) return fail(MGB_EXECUTION_FAILED, "missing input at index 0");
  Operand ids;
  mgb_status s = input_f32(p, n_inputs > 1 ? inputs[1] : nullptr, 1, ids);
  if (s != MGB_OK) return s;
  uint64_t count = 1;
  for (uint64_t d : ids.shape) count *= d;
  uint64_t vocab = 0, dim = 0;
  DevBuf product;
  cudaError_t e = cudaSuccess;
  auto pk = p->packed.find(tid);
  if (pk != p->packed.end()) {
    const Packed &w = pk->second;
    const std::vector<uint64_t> ls = w.logical_shape();
    vocab = ls[0];
    dim = ls[1];
    s = ensure_buf(p, product, count * dim * 4);
    if (s == MGB_OK)
      e = launch_embedding(w.format, w.buf.ptr, w.stored_rows, w.stored_cols, w.transposed ? 1 : 0,
                           ids.ptr, count, attrs.has_scale, attrs.scale,
                           static_cast<float *>(product.ptr), p->dev_bad, p->stream);
  } else {
    auto st = p->storage.find(tid);
    if (st == p->storage.end()) s = fail(MGB_EXECUTION_FAILED, "no materialized data for input resource %s", tid);
    else if (st->second.shape.size() != 2)
      s = fail(MGB_EXECUTION_FAILED, "embedding table %s has shape %s, not [vocab, dim]", tid,
               shape_str(st->second.shape).c_str());
    else {
      vocab = st->second.shape[0];
      dim = st->second.shape[1];
      s = ensure_buf(p, product, count * dim * 4);
      if (s == MGB_OK)
        e = launch_embedding_f32(static_cast<const float *>(st->second.buf.ptr), vocab, dim, ids.ptr,
                                 count, attrs.has_scale, attrs.scale,
                                 static_cast<float *>(product.ptr), p->dev_bad, p->stream);
    }
  }
  uint32_t bad = 0xFFFFFFFFu;
  float raw = 0.0f;
  if (s == MGB_OK && e == cudaSuccess)
    e = cudaMemcpyAsync(&bad, p->dev_bad, sizeof(bad), cudaMemcpyDeviceToHost, p->stream);
  if (s == MGB_OK && e == cudaSuccess) e = cudaStreamSynchronize(p->stream);
  if (s == MGB_OK && e == cudaSuccess && bad != 0xFFFFFFFFu)
    e = cudaMemcpy(&raw, ids.ptr + bad, sizeof(raw), cudaMemcpyDeviceToHost);
  if (ids.owned.ptr) free_buf(p, ids.owned);
  if (s == MGB_OK && e != cudaSuccess) s = cuda_fail(e, "embedding");
  if (s == MGB_OK && bad != 0xFFFFFFFFu)
    s = fail(MGB_EXECUTION_FAILED, "token id %s is not below the vocabulary size %llu",
             rust_f32(raw).c_str(), (unsigned long long)vocab);
  if (s != MGB_OK) {
    free_buf(p, product);
    return s;
  }
  forget_packed(p, output);
  put_tensor(p, output, {count, dim}, product);
  return MGB_OK;
}

const mgb_kernel_advertisement ADS[] = {
    {"matmul", "linear-algebra", 2, MGB_DTYPE_F32, MGB_DTYPE_F32, MGB_CANCELLATION_TIMEOUT_ONLY},
    {"matmul-bias", "linear-algebra", 2, MGB_DTYPE_F32, MGB_DTYPE_F32, MGB_CANCELLATION_TIMEOUT_ONLY},
    {"matmul-residual", "linear-algebra", 2, MGB_DTYPE_F32, MGB_DTYPE_F32,
     MGB_CANCELLATION_TIMEOUT_ONLY},
    {"embedding", "lookup", 2, MGB_DTYPE_F32, MGB_DTYPE_F32, MGB_CANCELLATION_TIMEOUT_ONLY},
};

int env_flag(const char *name, int dflt) {
  const char *v = getenv(name);
  if (!v) return dflt;
  return strcmp(v, "0") != 0;
}

}  // namespace

extern "C" {

void mgb_provider_get_metadata(mgb_provider_metadata *out) {
  if (!out) return;
  out->name = PROVIDER_NAME;
  out->version = PROVIDER_VERSION;
  out->vendor = PROVIDER_VENDOR;
  out->description =
      "B200-native implementation of packed quantized-weight matmul: sm_100a GEMV and "
      "tcgen05 GEMM kernels over device-resident packed weights";
}

mgb_status mgb_settings_from_env(mgb_settings *out) {
  if (!out) return fail(MGB_INVALID_ARGUMENT, "null settings");
  out->packed_weights = env_flag("MAGNETAR_B200_PACKED_WEIGHTS", 1);
  const char *i8 = getenv("MAGNETAR_B200_INT8_ACTIVATIONS");
  out->int8_activations = i8 && strcmp(i8, "1") == 0;
  const char *dev = getenv("MAGNETAR_B200_DEVICE");
  out->device = dev ? atoi(dev) : 0;
  const char *prof = getenv("MAGNETAR_B200_PROFILE");
  out->profile = prof && strcmp(prof, "1") == 0;
  const char *k = getenv("MAGNETAR_B200_KERNEL");
  out->kernel = !k ? MGB_KERNEL_AUTO
                   : (strcmp(k, "gemv") == 0 ? MGB_KERNEL_GEMV
                                             : (strcmp(k, "gemm") == 0 ? MGB_KERNEL_GEMM
                                                                       : MGB_KERNEL_AUTO));
  return MGB_OK;
}

mgb_status mgb_provider_create(const mgb_settings *settings, mgb_provider **out) {
  if (!out) return fail(MGB_INVALID_ARGUMENT, "null output pointer");
  *out = nullptr;
  mgb_settings st{};
  if (settings) st = *settings;
  else mgb_settings_from_env(&st);
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(MGB_CUDA_ERROR, "no CUDA device is available%s%s",
                e != cudaSuccess ? ": " : "", e != cudaSuccess ? cudaGetErrorString(e) : "");
  }
  if (st.device < 0 || st.device >= count)
    return fail(MGB_INVALID_ARGUMENT, "device %d is not one of the %d visible devices", st.device,
                count);
  e = cudaSetDevice(st.device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  auto *p = new mgb_provider();
  p->settings = st;
  p->sms = device_sms(st.device);
  e = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking);
  if (e == cudaSuccess) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = st.device;
    e = cudaMemPoolCreate(&p->pool, &props);
  }
  if (e == cudaSuccess) {
    // freed memory stays in the pool until an allocation needs it elsewhere
    uint64_t keep = UINT64_MAX;
    e = cudaMemPoolSetAttribute(p->pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  if (e == cudaSuccess) e = cudaMalloc(&p->dev_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(p->dev_err, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&p->dev_bad, sizeof(uint32_t));
  if (e != cudaSuccess) {
    if (p->dev_err) cudaFree(p->dev_err);
    if (p->dev_bad) cudaFree(p->dev_bad);
    if (p->pool) cudaMemPoolDestroy(p->pool);
    if (p->stream) cudaStreamDestroy(p->stream);
    if (p->h2d) cudaStreamDestroy(p->h2d);
    if (p->d2h) cudaStreamDestroy(p->d2h);
    delete p;
    return cuda_fail(e, "provider set-up");
  }
  *out = p;
  return MGB_OK;
}

void mgb_provider_destroy(mgb_provider *p) {
  if (!p) return;
  cudaSetDevice(p->settings.device);
  cudaStreamSynchronize(p->stream);
  if (p->settings.profile) {
    fprintf(stderr, "[b200 profile] packed weights expanded to f32: %llu, %.1f ms\n",
            (unsigned long long)p->materializations, p->materialize_ms);
    std::vector<std::pair<std::string, ProfileEntry>> rows(p->profile.begin(), p->profile.end());
    std::sort(rows.begin(), rows.end(),
              [](const auto &a, const auto &b) { return a.second.ms > b.second.ms; });
    for (auto &r : rows)
      fprintf(stderr, "[b200 profile] %s: %llu calls, %.1f ms total, %.3f ms each\n",
              r.first.c_str(), (unsigned long long)r.second.count, r.second.ms,
              r.second.ms / (double)r.second.count);
  }
  for (auto &kv : p->executions) {
    if (kv.second.start) cudaEventDestroy(kv.second.start);
    if (kv.second.stop) cudaEventDestroy(kv.second.stop);
  }
  for (auto &kv : p->storage) free_buf(p, kv.second.buf);
  for (auto &kv : p->packed) free_buf(p, kv.second.buf);
  free_buf(p, p->workspace);
  p->reading.clear();  // no call may be in flight while the Provider is destroyed
  for (auto &b : p->deferred) free_buf(p, b);
  if (p->stream) cudaStreamSynchronize(p->stream);
  if (p->pool) cudaMemPoolDestroy(p->pool);
  if (p->dev_err) cudaFree(p->dev_err);
  if (p->dev_bad) cudaFree(p->dev_bad);
  if (p->stream) cudaStreamDestroy(p->stream);
  if (p->h2d) cudaStreamDestroy(p->h2d);
  if (p->d2h) cudaStreamDestroy(p->d2h);
  delete p;
}

mgb_status mgb_provider_initialize(mgb_provider *p) {
  if (!p) return fail(MGB_INVALID_ARGUMENT, "null provider");
  std::lock_guard<std::mutex> lock(p->mu);
  observe(p, MGB_OBS_PROVIDER_REGISTERED, "", std::string("provider=") + PROVIDER_NAME);
  observe(p, MGB_OBS_DEVICE_DETECTED, "", "device=cuda-b200:" + std::to_string(p->settings.device));
  return MGB_OK;
}

mgb_status mgb_provider_shutdown(mgb_provider *p) {
  if (!p) return fail(MGB_INVALID_ARGUMENT, "null provider");
  std::lock_guard<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  cudaStreamSynchronize(p->stream);
  return MGB_OK;
}

int32_t mgb_provider_health(mgb_provider *p) {
  if (!p) return MGB_HEALTH_UNAVAILABLE;
  std::lock_guard<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  cudaError_t e = cudaStreamQuery(p->stream);
  return (e == cudaSuccess || e == cudaErrorNotReady) ? MGB_HEALTH_AVAILABLE
                                                      : MGB_HEALTH_UNAVAILABLE;
}

mgb_status mgb_provider_device(mgb_provider *p, mgb_device_descriptor *out) {
  if (!p || !out) return fail(MGB_INVALID_ARGUMENT, "null argument");
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, p->settings.device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  memset(out, 0, sizeof *out);
  snprintf(out->id, sizeof out->id, "cuda-b200:%d", p->settings.device);
  snprintf(out->name, sizeof out->name, "%s", prop.name);
  snprintf(out->architecture, sizeof out->architecture, "sm_%d%da", prop.major, prop.minor);
  out->compute_units = (uint32_t)prop.multiProcessorCount;
  out->memory_bytes = prop.totalGlobalMem;
  out->max_concurrent_operations = 1;  // one stream per Provider
  out->max_workspace_bytes = prop.totalGlobalMem;
  return MGB_OK;
}

size_t mgb_kernel_advertisement_count(void) { return sizeof ADS / sizeof ADS[0]; }

mgb_status mgb_kernel_advertisement_get(size_t index, mgb_kernel_advertisement *out) {
  if (!out || index >= mgb_kernel_advertisement_count())
    return fail(MGB_INVALID_ARGUMENT, "no advertisement %zu", index);
  *out = ADS[index];
  return MGB_OK;
}

mgb_status mgb_write_tensor(mgb_provider *p, const char *id, const uint64_t *shape, int32_t rank,
                            const float *data) {
  if (!p || !id || (rank > 0 && !shape) || rank < 0 || rank > MGB_MAX_RANK)
    return fail(MGB_INVALID_ARGUMENT, "invalid tensor arguments");
  std::unique_lock<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  std::vector<uint64_t> sh(shape, shape + rank);
  uint64_t elems = 1;
  for (uint64_t d : sh) elems *= d;
  if (elems && !data) return fail(MGB_INVALID_ARGUMENT, "null tensor data");
  // A new buffer (the pool hands back the memory of the previous one, in
  // stream order): the resource keeps its old value until the upload is done,
  // so a kernel submitted meanwhile from another thread reads old or new,
  // never a half-written tensor.
  DevBuf buf;
  mgb_status s = ensure_buf(p, buf, elems * 4);
  if (s != MGB_OK) return s;
  if (elems) {
    cudaError_t e = copy_unlocked(p, lock, p->h2d, buf.ptr, data, elems * 4,
                                  cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      free_buf(p, buf);
      return cuda_fail(e, "tensor upload");
    }
  }
  forget_packed(p, id);
  put_tensor(p, id, sh, buf);
  return MGB_OK;
}

mgb_status mgb_write_packed_weight(mgb_provider *p, const char *id, int32_t format,
                                   uint64_t stored_rows, uint64_t stored_cols, int32_t transposed,
                                   const void *bytes, uint64_t len, int32_t *stored) {
  if (!p || !id || !stored) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  *stored = 0;
  if (!p->settings.packed_weights || !format_supported(format)) return MGB_OK;  // Declined
  mgb_status s = check_packed_shape(format, stored_rows, stored_cols);
  if (s != MGB_OK) return s;
  const uint64_t expect = ggml_bytes(format, stored_rows, stored_cols);
  if (len != expect)
    return fail(MGB_INVALID_ARGUMENT, "packed weight holds %llu bytes, its shape needs %llu",
                (unsigned long long)len, (unsigned long long)expect);
  if (len && !bytes) return fail(MGB_INVALID_ARGUMENT, "null weight bytes");
  std::lock_guard<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  DevBuf staging, layout;
  s = ensure_buf(p, staging, len);
  if (s != MGB_OK) return s;
  s = ensure_buf(p, layout, device_bytes(format, stored_rows, stored_cols));
  if (s != MGB_OK) {
    free_buf(p, staging);
    return s;
  }
  cudaError_t e = cudaMemcpyAsync(staging.ptr, bytes, len, cudaMemcpyHostToDevice, p->stream);
  if (e == cudaSuccess) e = launch_repack(format, staging.ptr, stored_rows, stored_cols, layout.ptr, p->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(p->stream);
  free_buf(p, staging);
  if (e != cudaSuccess) {
    free_buf(p, layout);
    return cuda_fail(e, "packed weight upload");
  }
  forget_tensor(p, id);
  forget_packed(p, id);
  Packed w;
  w.format = format;
  w.stored_rows = stored_rows;
  w.stored_cols = stored_cols;
  w.transposed = transposed != 0;
  w.buf = layout;
  p->packed[id] = w;
  *stored = 1;
  return MGB_OK;
}

mgb_status mgb_read_tensor(mgb_provider *p, const char *id, float *out, uint64_t capacity,
                           uint64_t *shape_out, int32_t *rank_out) {
  if (!p || !id) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  std::unique_lock<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  const void *src = nullptr;
  std::vector<uint64_t> shape;
  DevBuf owned;
  auto it = p->storage.find(id);
  if (it != p->storage.end()) {
    src = it->second.buf.ptr;
    shape = it->second.shape;
  } else {
    auto pk = p->packed.find(id);
    if (pk == p->packed.end()) return fail(MGB_NOT_FOUND, "no tensor %s", id);
    mgb_status s = expand(p, pk->second, owned);
    if (s != MGB_OK) return s;
    src = owned.ptr;
    shape = pk->second.logical_shape();
  }
  uint64_t elems = 1;
  for (uint64_t d : shape) elems *= d;
  if (rank_out) *rank_out = (int32_t)shape.size();
  if (shape_out)
    for (size_t i = 0; i < shape.size(); ++i) shape_out[i] = shape[i];
  mgb_status s = MGB_OK;
  if (out) {
    if (capacity < elems) {
      s = fail(MGB_INVALID_ARGUMENT, "output capacity %llu < %llu values",
               (unsigned long long)capacity, (unsigned long long)elems);
    } else if (elems) {
      // the buffer stays allocated while the mutex is released: a release or
      // overwrite of the resource meanwhile defers its free to `end_read`
      void *key = const_cast<void *>(src);
      if (!owned.ptr) p->reading[key]++;
      cudaError_t e = copy_unlocked(p, lock, p->d2h, out, src, elems * 4, cudaMemcpyDeviceToHost);
      if (!owned.ptr) end_read(p, key);
      if (e != cudaSuccess) s = cuda_fail(e, "tensor download");
    }
  }
  if (owned.ptr) {
    free_buf(p, owned);
  }
  return s;
}

mgb_status mgb_resident_shape(mgb_provider *p, const char *id, uint64_t *shape_out,
                              int32_t *rank_out) {
  if (!p || !id || !shape_out || !rank_out) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  std::vector<uint64_t> shape;
  auto it = p->storage.find(id);
  if (it != p->storage.end()) shape = it->second.shape;
  else {
    auto pk = p->packed.find(id);
    if (pk == p->packed.end()) return fail(MGB_NOT_FOUND, "no tensor %s", id);
    shape = pk->second.logical_shape();
  }
  *rank_out = (int32_t)shape.size();
  for (size_t i = 0; i < shape.size(); ++i) shape_out[i] = shape[i];
  return MGB_OK;
}

mgb_status mgb_release_tensor(mgb_provider *p, const char *id, int32_t *was_present) {
  if (!p || !id) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  const bool a = forget_packed(p, id);
  const bool b = forget_tensor(p, id);
  if (was_present) *was_present = (a || b) ? 1 : 0;
  return MGB_OK;
}

int32_t mgb_is_packed(mgb_provider *p, const char *id) {
  if (!p || !id) return 0;
  std::lock_guard<std::mutex> lock(p->mu);
  return p->packed.count(id) ? 1 : 0;
}

mgb_status mgb_read_tensor_value(mgb_provider *p, const char *id, int32_t *kind) {
  if (!p || !id || !kind) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  *kind = (p->packed.count(id) || p->storage.count(id)) ? MGB_VALUE_OPAQUE : MGB_VALUE_ABSENT;
  return MGB_OK;
}

mgb_status mgb_write_tensor_value_opaque(mgb_provider *p, const char *id) {
  if (!p || !id) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  return MGB_OK;  // an Opaque value stores nothing; a packed weight stays resident
}

mgb_status mgb_copy_tensor(mgb_provider *p, const char *from, const char *to) {
  if (!p || !from || !to) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  Operand src;
  mgb_status s = input_f32(p, from, 0, src);
  if (s != MGB_OK) return s == MGB_EXECUTION_FAILED ? fail(MGB_NOT_FOUND, "no tensor %s", from) : s;
  uint64_t elems = 1;
  for (uint64_t d : src.shape) elems *= d;
  DevBuf copy;
  if (src.owned.ptr && std::string(from) != to) {
    copy = src.owned;
    src.owned = DevBuf{};
  } else {
    s = ensure_buf(p, copy, elems * 4);
    if (s != MGB_OK) return s;
    cudaError_t e = cudaMemcpyAsync(copy.ptr, src.ptr, elems * 4, cudaMemcpyDeviceToDevice, p->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(p->stream);
    if (e != cudaSuccess) {
      free_buf(p, copy);
      return cuda_fail(e, "tensor copy");
    }
    if (src.owned.ptr) free_buf(p, src.owned);
  }
  forget_packed(p, to);
  put_tensor(p, to, src.shape, copy);
  return MGB_OK;
}

mgb_status mgb_device_memory(mgb_provider *p, uint64_t *free_bytes, uint64_t *total_bytes) {
  if (!p || !free_bytes || !total_bytes) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  cudaSetDevice(p->settings.device);
  size_t f = 0, t = 0;
  cudaError_t e = cudaMemGetInfo(&f, &t);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemGetInfo");
  // memory the pool holds for reuse is free for this Provider's tensors
  uint64_t reserved = 0, used = 0;
  if (p->pool &&
      cudaMemPoolGetAttribute(p->pool, cudaMemPoolAttrReservedMemCurrent, &reserved) == cudaSuccess &&
      cudaMemPoolGetAttribute(p->pool, cudaMemPoolAttrUsedMemCurrent, &used) == cudaSuccess &&
      reserved > used)
    f += reserved - used;
  *free_bytes = f;
  *total_bytes = t;
  return MGB_OK;
}

uint64_t mgb_materialization_count(mgb_provider *p) {
  if (!p) return 0;
  std::lock_guard<std::mutex> lock(p->mu);
  return p->materializations;
}

mgb_status mgb_submit_kernel(mgb_provider *p, const char *kernel, const mgb_kernel_attrs *attrs,
                             const char *const *inputs, int32_t n_inputs, const char *output,
                             uint64_t *handle) {
  if (!p || !kernel || !handle || (n_inputs > 0 && !inputs) || n_inputs < 0)
    return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  mgb_kernel_attrs at{0, 0, MGB_DTYPE_F32, -1, 0, 1.0f};
  if (attrs) at = *attrs;
  std::lock_guard<std::mutex> lock(p->mu);
  cudaSetDevice(p->settings.device);
  const uint64_t h = p->next_handle++;
  Execution ex;
  ex.kernel = kernel;
  observe(p, MGB_OBS_DISPATCH_STARTED, kernel, "handle=" + std::to_string(h));
  const std::string name = kernel;
  if (at.deadline_ms == 0) {
    ex.status = MGB_TIMEOUT;
    ex.reason = "the invocation's deadline elapsed before dispatch";
    observe(p, MGB_OBS_TIMEOUT, kernel, "handle=" + std::to_string(h));
  } else if (name != "matmul" && name != "matmul-bias" && name != "matmul-residual" &&
             name != "embedding") {
    ex.status = MGB_KERNEL_NOT_FOUND;
    ex.reason = "no Kernel named " + name + " is advertised by this Provider";
    observe(p, MGB_OBS_DISPATCH_FAILED, kernel, ex.reason);
  } else if (!output) {
    ex.status = MGB_EXECUTION_FAILED;
    ex.reason = "missing output at index 0";
    observe(p, MGB_OBS_DISPATCH_FAILED, kernel, ex.reason);
  } else {
    if (p->settings.profile) {
      cudaEventCreate(&ex.start);
      cudaEventRecord(ex.start, p->stream);
    }
    mgb_status s = name == "embedding" ? run_embedding(p, at, inputs, n_inputs, output)
                                       : run_matmul(p, name, at, inputs, n_inputs, output);
    if (s != MGB_OK) {
      ex.status = s;
      ex.reason = mgb_last_error();
      observe(p, MGB_OBS_DISPATCH_FAILED, kernel, ex.reason);
    } else {
      cudaEventCreateWithFlags(&ex.stop, p->settings.profile ? cudaEventDefault
                                                              : cudaEventDisableTiming);
      cudaEventRecord(ex.stop, p->stream);
      observe(p, MGB_OBS_DISPATCH_COMPLETED, kernel, "handle=" + std::to_string(h));
    }
  }
  p->executions[h] = ex;
  *handle = h;
  clear_error();
  return MGB_OK;
}

mgb_status mgb_complete_kernel(mgb_provider *p, uint64_t handle, mgb_kernel_result *result) {
  if (!p || !result) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  Execution ex;
  {
    std::lock_guard<std::mutex> lock(p->mu);
    auto it = p->executions.find(handle);
    if (it == p->executions.end())
      return fail(MGB_UNKNOWN_HANDLE,
                  "no Kernel execution is associated with this handle: it was never submitted "
                  "through submit_kernel, or has already been completed once");
    ex = it->second;
    p->executions.erase(it);
  }
  cudaSetDevice(p->settings.device);
  if (ex.stop) {
    cudaError_t e = cudaEventSynchronize(ex.stop);
    int flag = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&flag, p->dev_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
      ex.status = MGB_CUDA_ERROR;
      ex.reason = std::string("device error: ") + cudaGetErrorString(e);
    } else if (flag) {
      cudaMemset(p->dev_err, 0, sizeof(int));
      ex.status = MGB_TIMEOUT;
      ex.reason = "a bounded device wait expired before the kernel's data arrived";
      std::lock_guard<std::mutex> lock(p->mu);
      observe(p, MGB_OBS_TIMEOUT, ex.kernel, ex.reason);
    }
    if (ex.start && e == cudaSuccess) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ex.start, ex.stop);
      std::lock_guard<std::mutex> lock(p->mu);
      auto &pe = p->profile[ex.kernel];
      pe.count++;
      pe.ms += ms;
    }
  }
  if (ex.start) cudaEventDestroy(ex.start);
  if (ex.stop) cudaEventDestroy(ex.stop);
  result->status = ex.status;
  snprintf(result->reason, sizeof result->reason, "%s", ex.reason.c_str());
  return MGB_OK;
}

size_t mgb_observation_count(mgb_provider *p) {
  if (!p) return 0;
  std::lock_guard<std::mutex> lock(p->mu);
  return std::min(p->observations.size(), OBS_CAPACITY);
}

mgb_status mgb_observations(mgb_provider *p, mgb_observation *out, size_t capacity,
                            size_t *written) {
  if (!p || !written || (capacity && !out)) return fail(MGB_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  const size_t n = std::min(p->observations.size(), OBS_CAPACITY);
  const size_t start = p->observations.size() - n;
  size_t w = 0;
  for (size_t i = start; i < p->observations.size() && w < capacity; ++i) out[w++] = p->observations[i];
  *written = w;
  return MGB_OK;
}

}  // extern "C"
