// Shared device-side definitions of the B200 packed-weight matmul Provider:
// format codes, the device layout of packed matrices, exact f16 decoding and
// the bounded mbarrier / bulk-copy PTX wrappers the kernels are built on.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "outspec.h"

namespace mgb {

// Format codes: the reference's `FORMATS` order (src/native/quant.rs:71-87).
enum Format : int { Q8_0 = 0, Q4_K = 1, Q6_K = 2, IQ4_NL = 5, Q5_K = 12, Q4_0 = 13 };

constexpr int RUN = 32;  // values per run (src/native/quant.rs:19)

__host__ __device__ inline bool supported(int f) {
  return f == Q8_0 || f == Q4_K || f == Q6_K || f == Q5_K || f == IQ4_NL || f == Q4_0;
}
__host__ __device__ inline int block_elements(int f) {
  return f == Q4_K || f == Q6_K || f == Q5_K ? 256 : 32;
}
__host__ __device__ inline int block_bytes(int f) {
  return f == Q4_K ? 144 : f == Q6_K ? 210 : f == Q5_K ? 176 : (f == Q8_0 ? 34 : 18);
}
// Super-block formats whose header holds d, dmin and Q4_K's 6-bit scale fields.
__host__ __device__ inline bool k_scale_min(int f) { return f == Q4_K || f == Q5_K; }

// Device layout of an [n stored rows x k stored cols] packed matrix: the
// quant plane (n rows of `qs_row` bytes: one 16-byte run of nibble pairs for
// the 4-bit formats, 32 bytes per run for Q8_0; Q6_K: 48 bytes per 64 values,
// the two runs' low-nibble pairs then their high 2-bit fields, 8 bytes per
// run) followed by the scale plane (n rows of `sc_row` bytes: Q4_K's 16-byte
// d/dmin/scales header per 256 values; Q6_K's 32-byte header per 256 values,
// its 16 int8 scales then d; Q5_K's 48-byte header per 256 values, Q4_K's 16
// bytes then each run's 32 fifth bits as one word; or one f16 scale per 32
// values).  The byte count equals the ggml blocks' except Q6_K's (224 bytes
// per 256 values against 210: the header is padded so every copy stays
// 16-byte aligned).
struct Layout {
  uint64_t n, k, qs_row, sc_row, qs_bytes, total;
  __host__ __device__ Layout(int f, uint64_t n_, uint64_t k_) : n(n_), k(k_) {
    qs_row = f == Q8_0 ? k : f == Q6_K ? k / 4 * 3 : k / 2;
    sc_row = f == Q6_K ? k / 8 : f == Q5_K ? k / 256 * 48 : k / 16;
    qs_bytes = n * qs_row;
    total = qs_bytes + n * sc_row;
  }
};

// The reference's run quant value for a 4-bit index (IQ4_NL's non-linear
// codebook; Q4_0's q - 8).  The IQ4_NL values are the ggml format constant.
__host__ __device__ inline int iq4nl_value(int i) {
#ifdef __CUDA_ARCH__
  // the same 16 values as the bytes of four words, picked with byte permutes:
  // a run-time index into a local array would go through local memory
  const uint32_t lo = __byte_perm(0xBFAD9881u, 0xF6EADDCFu, (uint32_t)(i & 7));
  const uint32_t hi = __byte_perm(0x26190D01u, 0x71594535u, (uint32_t)(i & 7));
  return (int)(int8_t)((i & 8 ? hi : lo) & 0xFFu);
#else
  const int8_t t[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                        1,    13,   25,  38,  53,  69,  89,  113};
  return t[i & 15];
#endif
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
  // cvt.f32.f16 is exact for every finite and infinite f16.
  return __half2float(__ushort_as_half((unsigned short)(bits & 0xffffu)));
}

// get_scale_min_k4 (src/native/quant.rs:46-57): sub-block j's 6-bit scale and
// min in a ggml Q4_K super-block's 12 scale bytes `q`.
__host__ __device__ inline void scale_min_k4_bytes(int j, const uint8_t *q, uint8_t &sc,
                                                   uint8_t &m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

// The device layout's Q4_K header keeps d and dmin (bytes 0..3) and stores the
// same eight (scale, min) pairs as 16 contiguous 6-bit fields over bytes
// 4..15: scale j at bits 6j, min j at bits 48 + 6j.  h1, h2, h3 are bytes
// 4..7, 8..11, 12..15 as little-endian words.  Two shifts per value, the same
// for every sub-block (no branch on j).
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t h1, uint32_t h2, uint32_t h3,
                                              uint32_t &sc, uint32_t &m) {
  const uint64_t a = ((uint64_t)h2 << 32) | h1;
  const uint64_t b = ((uint64_t)h3 << 32) | h2;
  sc = (uint32_t)(a >> (6 * j)) & 63;
  m = (uint32_t)(b >> (16 + 6 * j)) & 63;
}

// Q6_K: the quant plane offsets of run u's nibble pairs (16 bytes) and high
// 2-bit fields (8 bytes) within its row.
__host__ __device__ inline uint64_t q6k_nib_offset(uint64_t u) { return (u / 2) * 48 + (u % 2) * 16; }
__host__ __device__ inline uint64_t q6k_high_offset(uint64_t u) { return (u / 2) * 48 + 32 + (u % 2) * 8; }

// Q6_K: the 6-bit codes (q + 32) of the 8 values of nibble word wd of a run,
// in the nibble-pair order: ev = values 8 wd + 0, 2, 4, 6, od = values
// 8 wd + 1, 3, 5, 7, one per byte.  hw is the run's high word for wd's half
// (wd / 2): its byte j holds the high bits of values 16 a + 8 b + 2 j (bits
// 4 b, 4 b + 1) and 16 a + 8 b + 2 j + 1 (bits 4 b + 2, 4 b + 3), b = wd % 2.
__device__ __forceinline__ void q6k_codes(uint32_t nib_word, uint32_t hw, int wd, uint32_t &ev,
                                          uint32_t &od) {
  const int b = wd & 1;
  ev = (nib_word & 0x0F0F0F0Fu) | (((hw >> (4 * b)) & 0x03030303u) << 4);
  od = ((nib_word >> 4) & 0x0F0F0F0Fu) | (((hw >> (4 * b + 2)) & 0x03030303u) << 4);
}

// Q5_K: the 5-bit codes of the 8 values of nibble word wd of a run (nibble-pair
// order, as q6k_codes).  hb is the run's fifth-bit word: byte j holds the
// fifth bits of values 8 wd + 2 j (bit 2 wd) and 8 wd + 2 j + 1 (bit 2 wd + 1)
// for wd = 0..3.
__device__ __forceinline__ void q5k_codes(uint32_t nib_word, uint32_t hb, int wd, uint32_t &ev,
                                          uint32_t &od) {
  ev = (nib_word & 0x0F0F0F0Fu) | (((hb >> (2 * wd)) & 0x01010101u) << 4);
  od = ((nib_word >> 4) & 0x0F0F0F0Fu) | (((hb >> (2 * wd + 1)) & 0x01010101u) << 4);
}

// ---- device error flag -------------------------------------------------------------
// Kernels never trap: a bounded wait that gives up records a code here and the
// kernel returns; the host maps it to MGB_TIMEOUT.
enum DeviceError : int { ERR_NONE = 0, ERR_WAIT_TIMEOUT = 1, ERR_BAD_SHAPE = 2 };

__device__ __forceinline__ void record_error(int *flag, int code) {
  if (flag) atomicCAS(flag, 0, code);
}

// ---- shared-memory addresses, mbarriers and bulk copies (PTX) -----------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` with an iteration bound (each try_wait
// itself suspends for a hardware time slice).  Returns false, after recording
// ERR_WAIT_TIMEOUT, when the bound is exceeded; the caller then returns.
constexpr uint32_t WAIT_BOUND = 1u << 22;

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
  for (uint32_t i = 0; i < WAIT_BOUND; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (err && (i & 1023) == 1023 && *(volatile int *)err != 0) return false;
  }
  record_error(err, ERR_WAIT_TIMEOUT);
  return false;
}

// mbar_wait for waits that are not on a critical path (or that share the SM
// with another kernel's busy warps): after a few polls the thread sleeps
// between polls (32 ns doubling to `max_ns`), leaving the issue slots to
// warps with work.  Same iteration bound (at most ~WAIT_BOUND * max_ns).
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t *bar, uint32_t parity, int *err,
                                                  uint32_t max_ns = 256) {
  uint32_t ns = 32;
  for (uint32_t i = 0; i < WAIT_BOUND; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 4) {
      __nanosleep(ns);
      if (ns < max_ns) ns <<= 1;
    }
    if (err && (i & 1023) == 1023 && *(volatile int *)err != 0) return false;
  }
  record_error(err, ERR_WAIT_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared, completing `bytes` on `bar`.  Both addresses
// 16-byte aligned, bytes a multiple of 16 (this CTA's shared memory only).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__host__ __device__ inline uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

// ---- output fan-out and completion of a tensor-parallel call ----------------------

// Output element (m, col) of this call, written to every rank's y.  The rank
// loop is unrolled over MAX_TP so y_ranks is only indexed by constants: a
// runtime index into the kernel parameter would make every thread copy the
// whole OutSpec into local memory at entry.
__device__ __forceinline__ void out_store(const OutSpec &o, int m, uint64_t col, float v) {
  const uint64_t off = (uint64_t)m * o.ldy + o.col0 + col;
#pragma unroll
  for (int r = 0; r < MAX_TP; ++r)
    if (r < o.world) o.y_ranks[r][off] = v;
}

// ---- waits on the ranks of a tensor-parallel group ------------------------------------

// Word index of the epoch word in a rank's synchronisation buffer
// (MGB_TP_EPOCH_OFFSET / 4: after the done words and the reserved word).
constexpr int TP_EPOCH_WORD = 33;

// Lane r (< world) of one warp polls done[r] until it reaches `epoch` (serial
// number arithmetic, so epochs may wrap), sleeping 32 to 128 ns between polls,
// giving up after `timeout_ns` of the global timer or an iteration cap.  The
// load is an acquire at system scope, so this thread's later loads are not
// satisfied before it (the columns an epoch announces were performed before
// the epoch was stored).  Returns whether this lane's rank got there; lanes
// >= world return true.
__device__ __forceinline__ bool poll_epoch(const uint32_t *done, int world, uint32_t epoch,
                                           uint64_t timeout_ns, int lane) {
  if (lane >= world) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  uint32_t ns = 32;
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(done + lane) : "memory");
    if ((int32_t)(v - epoch) >= 0) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > timeout_ns) break;
    __nanosleep(ns);
    if (ns < 128) ns <<= 1;
  }
  return false;
}

// The input wait of a call (OutSpec::wait_done): one whole warp, after the
// kernel's griddepcontrol.wait (so the earlier call on this stream, which
// advanced the epoch word, has finished), before a barrier that precedes every
// read of x in the CTA.  A wait that gives up records ERR_WAIT_TIMEOUT.
__device__ __forceinline__ void out_wait_input(const OutSpec &o, int lane, int *err) {
  if (!o.wait_done) return;
  const uint32_t epoch =
      o.wait_epoch ? o.wait_epoch : *(volatile const uint32_t *)(o.wait_done + TP_EPOCH_WORD);
  const bool reached = poll_epoch(o.wait_done, o.wait_world, epoch, o.wait_timeout_ns, lane);
  if (!__all_sync(0xffffffffu, reached) && lane == 0) record_error(err, ERR_WAIT_TIMEOUT);
}
}  // namespace mgb
