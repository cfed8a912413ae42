// Small kernels around the packed path: the dense f32 matmul (an f32 weight,
// or `transpose_a` on an expanded packed weight, src/native/mod.rs:221-222),
// the bias / residual epilogue (src/lib.rs:1028-1133) and the int8
// activation quantiser (`quantize_rows`, src/native/quant.rs:350-378).
#include "common.cuh"
#include "kernels.h"

namespace mgb {

// out[m, n] = op(a)[m, k] * op(b)[k, n], strides as src/lib.rs:291-302.
// 64x64 output tile per 256-thread CTA, 4x4 per thread, k in steps of 16.
__global__ void __launch_bounds__(256) mgb_matmul_f32_kernel(
    const float *__restrict__ a, const float *__restrict__ b, uint64_t m, uint64_t n, uint64_t k,
    uint64_t a_row_stride, uint64_t a_inner_stride, uint64_t b_inner_stride,
    uint64_t b_col_stride, float *__restrict__ out) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const uint64_t row0 = (uint64_t)blockIdx.y * 64, col0 = (uint64_t)blockIdx.x * 64;
  float acc[4][4] = {};
  for (uint64_t k0 = 0; k0 < k; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, rr = i % 64;
      const uint64_t gr = row0 + rr, gk = k0 + kk;
      As[kk][rr] = (gr < m && gk < k) ? a[gr * a_row_stride + gk * a_inner_stride] : 0.f;
      const uint64_t gc = col0 + rr;
      Bs[kk][rr] = (gc < n && gk < k) ? b[gk * b_inner_stride + gc * b_col_stride] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t r = row0 + ty * 4 + i, c = col0 + tx * 4 + j;
      if (r < m && c < n) out[r * n + c] = acc[i][j];
    }
}

cudaError_t launch_matmul_f32(const float *a, uint64_t a_rows, uint64_t a_cols, const float *b,
                              uint64_t b_rows, uint64_t b_cols, int transpose_a, int transpose_b,
                              float *out, cudaStream_t stream) {
  const uint64_t m = transpose_a ? a_cols : a_rows, k = transpose_a ? a_rows : a_cols;
  const uint64_t n = transpose_b ? b_rows : b_cols;
  const uint64_t a_row_stride = transpose_a ? 1 : a_cols, a_inner = transpose_a ? a_cols : 1;
  const uint64_t b_inner = transpose_b ? 1 : b_cols, b_col = transpose_b ? b_cols : 1;
  if (!m || !n) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(n, 64), (unsigned)ceil_div(m, 64));
  mgb_matmul_f32_kernel<<<grid, 256, 0, stream>>>(a, b, m, n, k, a_row_stride, a_inner, b_inner,
                                              b_col, out);
  return cudaGetLastError();
}

__global__ void mgb_transpose_kernel(const float *__restrict__ in, uint64_t rows, uint64_t cols,
                                 float *__restrict__ out) {
  __shared__ float tile[32][33];
  const uint64_t c0 = (uint64_t)blockIdx.x * 32, r0 = (uint64_t)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const uint64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const uint64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
  }
}

cudaError_t launch_transpose(const float *in, uint64_t rows, uint64_t cols, float *out,
                             cudaStream_t stream) {
  if (!rows || !cols) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32));
  mgb_transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(in, rows, cols, out);
  return cudaGetLastError();
}

// y = y + addend, addend of y's length or one row of `cols` broadcast.
__global__ void mgb_add_kernel(float *__restrict__ y, uint64_t len, const float *__restrict__ addend,
                           uint64_t addend_len, uint64_t cols) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < len;
       i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = y[i] + (addend_len == len ? addend[i] : addend[i % cols]);
}

cudaError_t launch_add(float *y, uint64_t len, const float *addend, uint64_t addend_len,
                       uint64_t cols, cudaStream_t stream) {
  if (!len) return cudaSuccess;
  const uint64_t blocks = ceil_div(len, 256);
  mgb_add_kernel<<<(unsigned)(blocks > 4096 ? 4096 : blocks), 256, 0, stream>>>(y, len, addend,
                                                                           addend_len, cols);
  return cudaGetLastError();
}

// One warp per 32-value block: amax, d = amax / 127 (a division, as the
// reference), q = round-half-even(x / d), per-16 sums.
__global__ void mgb_quantize_rows_kernel(const float *__restrict__ x, uint64_t blocks,
                                     int8_t *__restrict__ values, float *__restrict__ scales,
                                     int32_t *__restrict__ sums, float *__restrict__ rounded) {
  const int lane = threadIdx.x & 31;
  for (uint64_t b = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) / 32; b < blocks;
       b += (uint64_t)gridDim.x * blockDim.x / 32) {
    const float v = x[b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float d = __fdiv_rn(amax, 127.0f);
    int q = 0;
    if (amax != 0.0f) q = (int)rintf(__fdiv_rn(v, d));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    if (values) values[b * 32 + lane] = (int8_t)q;
    if (rounded) rounded[b * 32 + lane] = __fmul_rn((float)q, d);
    int s = q;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      if (scales) scales[b] = d;
      if (sums) sums[2 * b] = s;
    }
    if (lane == 16 && sums) sums[2 * b + 1] = s;
  }
}

cudaError_t launch_quantize_rows(const float *x, uint64_t len, int8_t *values, float *scales,
                                 int32_t *sums, cudaStream_t stream) {
  const uint64_t blocks = len / 32;
  if (!blocks) return cudaSuccess;
  const uint64_t ctas = ceil_div(blocks, 8);
  mgb_quantize_rows_kernel<<<(unsigned)(ctas > 8192 ? 8192 : ctas), 256, 0, stream>>>(
      x, blocks, values, scales, sums, nullptr);
  return cudaGetLastError();
}

cudaError_t launch_int8_rounded(const float *x, uint64_t len, float *out, cudaStream_t stream) {
  const uint64_t blocks = len / 32;
  if (!blocks) return cudaSuccess;
  const uint64_t ctas = ceil_div(blocks, 8);
  mgb_quantize_rows_kernel<<<(unsigned)(ctas > 8192 ? 8192 : ctas), 256, 0, stream>>>(
      x, blocks, nullptr, nullptr, nullptr, out);
  return cudaGetLastError();
}

int device_sms(int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return 148;
  return sms > 0 ? sms : 148;
}

}  // namespace mgb
