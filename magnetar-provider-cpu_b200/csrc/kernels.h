// Internal launch entry points of the B200 kernels (host side, C++).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "outspec.h"

namespace mgb {

// layout.cu
cudaError_t launch_repack(int fmt, const void *ggml, uint64_t n, uint64_t k, void *dst,
                          cudaStream_t stream);
cudaError_t launch_dequantize(int fmt, const void *w, uint64_t n, uint64_t k, float *out,
                              cudaStream_t stream);
cudaError_t launch_input_major(int fmt, const void *w, uint64_t k_rows, uint64_t n_cols,
                               const float *x, uint64_t m, float *y, cudaStream_t stream);
// Packed / f32 table lookups; *bad (when given) receives the position of the
// first invalid id, 0xFFFFFFFF when every id is valid.
cudaError_t launch_embedding(int fmt, const void *w, uint64_t stored_rows, uint64_t stored_cols,
                             int transposed, const float *ids, uint64_t count, int has_scale,
                             float scale, float *out, uint32_t *bad, cudaStream_t stream);
cudaError_t launch_embedding_f32(const float *table, uint64_t vocab, uint64_t dim, const float *ids,
                                 uint64_t count, int has_scale, float scale, float *out,
                                 uint32_t *bad, cudaStream_t stream);

// gemv.cu: m <= 2.  addend_mode 0 none, 1 row broadcast addend[n], 2 addend[m, n].
// Launched with programmatic stream serialization (it may start while the
// previous kernel on the stream drains; it waits for it before reading x).
// No scratch: each CTA packs its activations into shared memory.
cudaError_t launch_gemv(int fmt, const void *w, uint64_t n, uint64_t k, const float *x,
                        uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                        int *err, int sms, cudaStream_t stream);

// gemm.cu: tensor-core path (bf16 operands, f32 accumulation) for m > 2.
// The minimum scratch is the bf16 activation copy; the preferred size adds the
// 2, 4 or 8 f32 [m, n] planes with which a call of narrow tiles splits K.
uint64_t gemm_workspace_bytes(int fmt, uint64_t m, uint64_t n, uint64_t k);
uint64_t gemm_workspace_bytes_preferred(int fmt, uint64_t m, uint64_t n, uint64_t k);
bool gemm_supported(int fmt, uint64_t m, uint64_t n, uint64_t k);
cudaError_t launch_gemm(int fmt, const void *w, uint64_t n, uint64_t k, const float *x,
                        uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                        void *workspace, uint64_t workspace_bytes, int *err, int sms,
                        cudaStream_t stream);

// the GEMM alone on bf16 activations xb[m, k] (no conversion pass)
cudaError_t launch_gemm_bf16(int fmt, const void *w, uint64_t n, uint64_t k, const void *xb,
                             uint64_t m, const OutSpec &out, const float *addend, int addend_mode, int *err,
                             int sms, cudaStream_t stream);

// dense.cu
cudaError_t launch_matmul_f32(const float *a, uint64_t a_rows, uint64_t a_cols, const float *b,
                              uint64_t b_rows, uint64_t b_cols, int transpose_a, int transpose_b,
                              float *out, cudaStream_t stream);
// out[cols, rows] = in[rows, cols]^T
cudaError_t launch_transpose(const float *in, uint64_t rows, uint64_t cols, float *out,
                             cudaStream_t stream);
cudaError_t launch_add(float *y, uint64_t len, const float *addend, uint64_t addend_len,
                       uint64_t cols, cudaStream_t stream);
cudaError_t launch_quantize_rows(const float *x, uint64_t len, int8_t *values, float *scales,
                                 int32_t *sums, cudaStream_t stream);
cudaError_t launch_int8_rounded(const float *x, uint64_t len, float *out, cudaStream_t stream);

int device_sms(int device);

}  // namespace mgb
