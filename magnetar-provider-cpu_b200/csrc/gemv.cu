// Decode GEMV for packed weights on sm_100a: y[m, n] = x[m, k] * W^T for
// m <= 2 activation rows, f32 activations, f32 accumulation.
// Replaces the reference's `columns_q4k_avx2` / `columns_avx2` /
// `columns_iq4nl_avx2` (src/native/quant.rs:604-744, :1438-1483) with the f32
// semantics of its scalar path (:559-597).
//
// Work split: one CTA owns a contiguous range of output rows (stored rows of
// W).  Thread t owns run t of K (32 values) for the whole kernel: its
// activations live in registers, so the only memory stream is W itself, read
// once with 128-bit loads (each warp reads 512 contiguous quant bytes per
// row).  Per row every thread produces a partial dot product; warps reduce with
// shuffles and a fixed-order shared-memory pass produces y (deterministic).
//
// Quant -> f32 without integer-to-float conversions:
//   4-bit q: prmt places q in bits 16..19 of 0x3F000000, i.e. the float
//            0.5 + q/256.  With t = sum((0.5 + q/256) x) over the run and
//            X = sum(x) over the run (computed once per thread),
//            sum(q x) = 256 t - 128 X.
//   8-bit q: prmt places (q + 128) in the low byte of 0x4B000000, the float
//            2^23 + q + 128; subtracting 2^23 + 128 is exact.
// Products accumulate with the packed fma.rn.f32x2 (two values per issue).
#include "common.cuh"
#include "kernels.h"

namespace mgb {

__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ld_nc_u16(const void *p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// 0.5 + q/256 for the 4-bit value in byte i of `v` (bits 0..3 of that byte).
__device__ __forceinline__ float nib_f(uint32_t v, int i) {
  return __uint_as_float(__byte_perm(v, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
}

// 2^23 + b for byte i of `v`.
__device__ __forceinline__ float byte_f(uint32_t v, int i) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7650u | (uint32_t)i));
}

// sum over a 32-value run of (0.5 + q/256) * x for 4-bit quants stored as
// nibble pairs (byte i = values 2i, 2i+1).
__device__ __forceinline__ float dot_nib_run(const uint4 &qs, const float *xr) {
  const uint32_t words[4] = {qs.x, qs.y, qs.z, qs.w};
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    const uint32_t lo = words[wd] & 0x0F0F0F0Fu;
    const uint32_t hi = (words[wd] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 q = make_float2(nib_f(lo, i), nib_f(hi, i));
      const float2 xv = make_float2(xr[8 * wd + 2 * i], xr[8 * wd + 2 * i + 1]);
      acc = __ffma2_rn(q, xv, acc);
    }
  }
  return acc.x + acc.y;
}

// sum over a run of (b + 128) * x for the biased bytes of 8 words (byte
// order = value order); returns sum(b * x) exactly shifted back.
__device__ __forceinline__ float dot_byte_words(const uint32_t *u, const float *xr) {
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int wd = 0; wd < 8; ++wd) {
#pragma unroll
    for (int i = 0; i < 4; i += 2) {
      float2 q = make_float2(byte_f(u[wd], i), byte_f(u[wd], i + 1));
      q = __fadd2_rn(q, bias);
      const float2 xv = make_float2(xr[4 * wd + i], xr[4 * wd + i + 1]);
      acc = __ffma2_rn(q, xv, acc);
    }
  }
  return acc.x + acc.y;
}

// IQ4_NL codebook lookup: the 8 indices of word `v` (nibble order = value
// order) -> two words of codebook values biased by +128 (u8).
__device__ __forceinline__ void iq4_lookup(uint32_t v, const uint32_t t[4], uint32_t &o0,
                                           uint32_t &o1) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t s = (v >> (16 * h)) & 0xFFFFu;
    const uint32_t sel = s & 0x7777u;
    const uint32_t low = __byte_perm(t[0], t[1], sel);
    const uint32_t high = __byte_perm(t[2], t[3], sel);
    const uint32_t pick = 0x3210u | ((s & 0x8888u) >> 1);
    const uint32_t r = __byte_perm(low, high, pick);
    if (h == 0) o0 = r; else o1 = r;
  }
}

template <int FMT, int MR, int R, int MAXT>
__global__ void __launch_bounds__(MAXT, 1)
    gemv_kernel(const uint8_t *__restrict__ w, int n, int k, const float *__restrict__ x,
                float *__restrict__ y, const float *__restrict__ addend, int addend_mode,
                int rows_per_cta) {
  __shared__ float red[2][32][R * MR];
  const Layout L(FMT, (uint64_t)n, (uint64_t)k);
  const int runs = k / RUN;
  const int u = threadIdx.x;
  const bool active = u < runs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;

  float xr[MR][32];
  float X[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    X[m] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (active) v = __ldg(reinterpret_cast<const float4 *>(x + (size_t)m * k + (size_t)u * 32) + i);
      xr[m][4 * i] = v.x;
      xr[m][4 * i + 1] = v.y;
      xr[m][4 * i + 2] = v.z;
      xr[m][4 * i + 3] = v.w;
      X[m] += (v.x + v.y) + (v.z + v.w);
    }
  }

  uint32_t lut[4] = {0, 0, 0, 0};
  if (FMT == IQ4_NL) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t v = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) v |= (uint32_t)((iq4nl_value(4 * i + b) + 128) & 0xff) << (8 * b);
      lut[i] = v;
    }
  }

  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(n, r0 + rows_per_cta);
  const uint8_t *scale_plane = w + L.qs_bytes;
  int buf = 0;
  for (int r = r0; r < r1; r += R) {
    uint4 qa[R], qb[R], hd[R];
    uint32_t dh[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int row = r + i;
      qa[i] = qb[i] = hd[i] = make_uint4(0, 0, 0, 0);
      dh[i] = 0;
      if (active && row < r1) {
        const uint8_t *qrow = w + (size_t)row * L.qs_row;
        const uint8_t *srow = scale_plane + (size_t)row * L.sc_row;
        if (FMT == Q8_0) {
          qa[i] = ld_stream_v4(qrow + (size_t)u * 32);
          qb[i] = ld_stream_v4(qrow + (size_t)u * 32 + 16);
          dh[i] = ld_nc_u16(srow + (size_t)u * 2);
        } else {
          qa[i] = ld_stream_v4(qrow + (size_t)u * 16);
          if (FMT == Q4_K)
            hd[i] = __ldg(reinterpret_cast<const uint4 *>(srow + (size_t)(u >> 3) * 16));
          else
            dh[i] = ld_nc_u16(srow + (size_t)u * 2);
        }
      }
    }
    float part[R][MR];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (FMT == Q4_K) {
        const float d = f16_bits_to_f32(hd[i].x), dmin = f16_bits_to_f32(hd[i].x >> 16);
        uint32_t sc, mn;
        scale_min_k4(u & 7, hd[i].y, hd[i].z, hd[i].w, sc, mn);
        const float s = d * (float)sc, mv = dmin * (float)mn;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const float t = dot_nib_run(qa[i], xr[m]);
          part[i][m] = (256.f * s) * t - (128.f * s + mv) * X[m];
        }
      } else if (FMT == Q4_0) {
        const float d = f16_bits_to_f32(dh[i]);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const float t = dot_nib_run(qa[i], xr[m]);
          part[i][m] = d * (256.f * t - 136.f * X[m]);
        }
      } else if (FMT == Q8_0) {
        const float d = f16_bits_to_f32(dh[i]);
        const uint32_t ub[8] = {qa[i].x ^ 0x80808080u, qa[i].y ^ 0x80808080u,
                                qa[i].z ^ 0x80808080u, qa[i].w ^ 0x80808080u,
                                qb[i].x ^ 0x80808080u, qb[i].y ^ 0x80808080u,
                                qb[i].z ^ 0x80808080u, qb[i].w ^ 0x80808080u};
#pragma unroll
        for (int m = 0; m < MR; ++m) part[i][m] = d * dot_byte_words(ub, xr[m]);
      } else {  // IQ4_NL
        const float d = f16_bits_to_f32(dh[i]);
        uint32_t ub[8];
        const uint32_t words[4] = {qa[i].x, qa[i].y, qa[i].z, qa[i].w};
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) iq4_lookup(words[wd], lut, ub[2 * wd], ub[2 * wd + 1]);
#pragma unroll
        for (int m = 0; m < MR; ++m) part[i][m] = d * dot_byte_words(ub, xr[m]);
      }
    }
    // reduce every partial over the warp, then over the warps in fixed order
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        float v = active ? part[i][m] : 0.f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[buf][warp][i * MR + m] = v;
      }
    __syncthreads();
    if (threadIdx.x < R * MR) {
      const int i = threadIdx.x / MR, m = threadIdx.x % MR;
      const int row = r + i;
      if (row < r1) {
        float s = 0.f;
        for (int wi = 0; wi < nwarps; ++wi) s += red[buf][wi][threadIdx.x];
        if (addend_mode == 1) s = s + addend[row];
        else if (addend_mode == 2) s = s + addend[(size_t)m * n + row];
        y[(size_t)m * n + row] = s;
      }
    }
    buf ^= 1;
  }
}

template <int FMT, int MR, int R, int MAXT>
static cudaError_t launch_t(const void *w, int n, int k, const float *x, float *y,
                            const float *addend, int addend_mode, int sms, cudaStream_t stream) {
  const int runs = k / RUN;
  const int threads = ((runs + 31) / 32) * 32;
  int per_sm = 2048 / threads;
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 8) per_sm = 8;
  const int target = sms * per_sm;
  int rows = (int)ceil_div((uint64_t)n, (uint64_t)target);
  if (rows < 1) rows = 1;
  const int grid = (int)ceil_div((uint64_t)n, (uint64_t)rows);
  gemv_kernel<FMT, MR, R, MAXT><<<grid, threads, 0, stream>>>(
      static_cast<const uint8_t *>(w), n, k, x, y, addend, addend_mode, rows);
  return cudaGetLastError();
}

template <int FMT, int MR>
static cudaError_t launch_fmt(const void *w, int n, int k, const float *x, float *y,
                              const float *addend, int addend_mode, int sms, cudaStream_t stream) {
  if (k <= 256 * 32) return launch_t<FMT, MR, 4, 256>(w, n, k, x, y, addend, addend_mode, sms, stream);
  // 1024-thread CTAs have 64 registers per thread: one activation row per launch
  cudaError_t e = launch_t<FMT, 1, 2, 1024>(w, n, k, x, y, addend, addend_mode, sms, stream);
  if (MR == 2 && e == cudaSuccess)
    e = launch_t<FMT, 1, 2, 1024>(w, n, k, x + k, y + n,
                                  addend_mode == 2 ? addend + n : addend, addend_mode, sms, stream);
  return e;
}

cudaError_t launch_gemv(int fmt, const void *w, uint64_t n, uint64_t k, const float *x,
                        uint64_t m, float *y, const float *addend, int addend_mode, int sms,
                        cudaStream_t stream) {
  // m <= 2 per launch; larger m is split into row pairs by the caller.
  const int N = (int)n, K = (int)k;
#define MGB_GEMV_CASE(F)                                                                      \
  case F:                                                                                     \
    return m == 1 ? launch_fmt<F, 1>(w, N, K, x, y, addend, addend_mode, sms, stream)         \
                  : launch_fmt<F, 2>(w, N, K, x, y, addend, addend_mode, sms, stream);
  switch (fmt) {
    MGB_GEMV_CASE(Q4_K)
    MGB_GEMV_CASE(Q8_0)
    MGB_GEMV_CASE(IQ4_NL)
    MGB_GEMV_CASE(Q4_0)
    default:
      return cudaErrorInvalidValue;
  }
#undef MGB_GEMV_CASE
}

}  // namespace mgb
