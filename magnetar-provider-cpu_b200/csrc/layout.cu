// Device layout of packed matrices: ggml blocks -> (quant plane, scale plane),
// and the bit-exact dequantisation of that layout back to f32.
//
// Dequantised values equal the reference `decode` + `dequantize_row`
// (src/native/quant.rs:100-195, Q6_K :136-149, :1700-1711) bit for bit: every product and
// difference is rounded on its own (__fmul_rn / __fsub_rn, never an FMA), as
// Rust evaluates `scale * q - min` with `scale = d * sc`, `min = dmin * m`.
#include "common.cuh"
#include "kernels.h"

namespace mgb {

// The 16-byte device header of a Q4_K / Q5_K super-block: d, dmin as they are,
// then the eight 6-bit (scale, min) pairs of get_scale_min_k4 (the 12 bytes at
// blk + 4) rearranged as 16 contiguous 6-bit fields.
__device__ void write_k_header(const uint8_t *blk, uint8_t *out) {
  for (int i = 0; i < 4; ++i) out[i] = blk[i];
  uint64_t lo = 0, hi = 0;  // bits 0..63 and 64..95 of the 96-bit field array
  for (int jj = 0; jj < 8; ++jj) {
    uint8_t s, m;
    scale_min_k4_bytes(jj, blk + 4, s, m);
    const int bs = 6 * jj, bm = 48 + 6 * jj;
    lo |= (uint64_t)s << bs;
    if (bm < 64) {
      lo |= (uint64_t)m << bm;
      if (bm + 6 > 64) hi |= (uint64_t)m >> (64 - bm);
    } else {
      hi |= (uint64_t)m << (bm - 64);
    }
  }
  for (int i = 0; i < 8; ++i) out[4 + i] = (uint8_t)(lo >> (8 * i));
  for (int i = 0; i < 4; ++i) out[12 + i] = (uint8_t)(hi >> (8 * i));
}

// One thread per 32-value run: gathers the run's quants from its ggml block and
// writes them as 16 (or 32) bytes holding values (2i, 2i+1) in byte i.
__global__ void mgb_repack_kernel(int fmt, const uint8_t *__restrict__ src, uint64_t n, uint64_t k,
                              uint8_t *__restrict__ dst) {
  const uint64_t runs_per_row = k / RUN;
  const uint64_t total = n * runs_per_row;
  const Layout L(fmt, n, k);
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = t / runs_per_row, u = t % runs_per_row;
    const uint64_t row_bytes = k / block_elements(fmt) * block_bytes(fmt);
    const uint8_t *row_src = src + row * row_bytes;
    uint8_t *qs = dst + row * L.qs_row;
    uint8_t *sc = dst + L.qs_bytes + row * L.sc_row;
    if (fmt == Q4_K) {
      const uint64_t b = u / 8;
      const int j = (int)(u % 8);
      const uint8_t *blk = row_src + b * 144;
      const uint8_t *chunk = blk + 16 + 32 * (j / 2);
      const int shift = 4 * (j % 2);
      uint32_t words[4];
      for (int w = 0; w < 4; ++w) {
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
          const int e = 2 * (4 * w + i);
          const uint32_t lo = (chunk[e] >> shift) & 0xF, hi = (chunk[e + 1] >> shift) & 0xF;
          v |= (lo | (hi << 4)) << (8 * i);
        }
        words[w] = v;
      }
      *reinterpret_cast<uint4 *>(qs + u * 16) = make_uint4(words[0], words[1], words[2], words[3]);
      if (j == 0) write_k_header(blk, sc + b * 16);
    } else if (fmt == Q5_K) {
      // as Q4_K with the quants at blk + 48 and each value's fifth bit at bit j
      // of byte i of the 32 bytes at blk + 16 (value i of run j)
      const uint64_t b = u / 8;
      const int j = (int)(u % 8);
      const uint8_t *blk = row_src + b * 176;
      const uint8_t *chunk = blk + 48 + 32 * (j / 2);
      const int shift = 4 * (j % 2);
      uint32_t words[4];
      for (int w = 0; w < 4; ++w) {
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
          const int e = 2 * (4 * w + i);
          const uint32_t lo = (chunk[e] >> shift) & 0xF, hi = (chunk[e + 1] >> shift) & 0xF;
          v |= (lo | (hi << 4)) << (8 * i);
        }
        words[w] = v;
      }
      *reinterpret_cast<uint4 *>(qs + u * 16) = make_uint4(words[0], words[1], words[2], words[3]);
      // the run's fifth bits: byte jj bit 2 wd = value 8 wd + 2 jj, bit 2 wd + 1
      // = value 8 wd + 2 jj + 1
      uint32_t hb = 0;
      for (int wd = 0; wd < 4; ++wd)
        for (int jj = 0; jj < 4; ++jj) {
          const int v = 8 * wd + 2 * jj;
          hb |= (uint32_t)((blk[16 + v] >> j) & 1) << (8 * jj + 2 * wd);
          hb |= (uint32_t)((blk[16 + v + 1] >> j) & 1) << (8 * jj + 2 * wd + 1);
        }
      *reinterpret_cast<uint32_t *>(sc + b * 48 + 16 + 4 * j) = hb;
      if (j == 0) write_k_header(blk, sc + b * 48);
    } else if (fmt == Q6_K) {
      // run r = 4 h + g of the block: low nibbles in the 32 bytes at
      // 64 h + 32 (g % 2) (shift 4 (g / 2)), high 2 bits in the 32 bytes at
      // 128 + 32 h (shift 2 g); codes c = q + 32 in 0..63
      const uint64_t b = u / 8;
      const int r = (int)(u % 8), h = r / 4, g = r % 4;
      const uint8_t *blk = row_src + b * 210;
      const uint8_t *low = blk + 64 * h + 32 * (g % 2), *high = blk + 128 + 32 * h;
      uint8_t c[32];
      for (int i = 0; i < 32; ++i)
        c[i] = (uint8_t)(((low[i] >> (4 * (g / 2))) & 0xF) | (((high[i] >> (2 * g)) & 3) << 4));
      uint8_t *nib = qs + q6k_nib_offset(u);
      for (int i = 0; i < 16; ++i) nib[i] = (uint8_t)((c[2 * i] & 0xF) | ((c[2 * i + 1] & 0xF) << 4));
      uint32_t hw[2] = {0, 0};
      for (int a = 0; a < 2; ++a)
        for (int bb = 0; bb < 2; ++bb)
          for (int j = 0; j < 4; ++j) {
            const int v = 16 * a + 8 * bb + 2 * j;
            hw[a] |= (uint32_t)(c[v] >> 4) << (8 * j + 4 * bb);
            hw[a] |= (uint32_t)(c[v + 1] >> 4) << (8 * j + 4 * bb + 2);
          }
      *reinterpret_cast<uint2 *>(qs + q6k_high_offset(u)) = make_uint2(hw[0], hw[1]);
      if (r == 0) {
        // header: the 16 int8 scales (scale 2 r + p covers values 16 p .. of
        // run r), then d, then zeros
        for (int i = 0; i < 16; ++i) sc[b * 32 + i] = blk[192 + i];
        sc[b * 32 + 16] = blk[208];
        sc[b * 32 + 17] = blk[209];
        for (int i = 18; i < 32; ++i) sc[b * 32 + i] = 0;
      }
    } else if (fmt == Q8_0) {
      const uint8_t *blk = row_src + u * 34;
      for (int i = 0; i < 32; ++i) qs[u * 32 + i] = blk[2 + i];
      sc[u * 2] = blk[0];
      sc[u * 2 + 1] = blk[1];
    } else {  // IQ4_NL, Q4_0: ggml byte l holds indices l (low) and l + 16 (high)
      const uint8_t *blk = row_src + u * 18;
      for (int i = 0; i < 16; ++i) {
        const int e0 = 2 * i, e1 = 2 * i + 1;
        const uint32_t v0 = e0 < 16 ? (blk[2 + e0] & 0xF) : (blk[2 + e0 - 16] >> 4);
        const uint32_t v1 = e1 < 16 ? (blk[2 + e1] & 0xF) : (blk[2 + e1 - 16] >> 4);
        qs[u * 16 + i] = (uint8_t)(v0 | (v1 << 4));
      }
      sc[u * 2] = blk[0];
      sc[u * 2 + 1] = blk[1];
    }
  }
}

// The 32 quant values of run `u` of `row` (as ints) and the run's scale and
// min of each 16-value half (the same for both halves except Q6_K's scales).
__device__ __forceinline__ void decode_run(int fmt, const uint8_t *__restrict__ w, const Layout &L,
                                           uint64_t row, uint64_t u, int q[32], float scale[2],
                                           float min[2]) {
  const uint8_t *sc = w + L.qs_bytes + row * L.sc_row;
  if (fmt == Q6_K) {
    const uint8_t *qrow = w + row * L.qs_row;
    const uint4 v = *reinterpret_cast<const uint4 *>(qrow + q6k_nib_offset(u));
    const uint2 hh = *reinterpret_cast<const uint2 *>(qrow + q6k_high_offset(u));
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
    for (int wd = 0; wd < 4; ++wd) {
      uint32_t ev, od;
      q6k_codes(words[wd], wd < 2 ? hh.x : hh.y, wd, ev, od);
      for (int j = 0; j < 4; ++j) {
        q[8 * wd + 2 * j] = (int)((ev >> (8 * j)) & 0xFF) - 32;
        q[8 * wd + 2 * j + 1] = (int)((od >> (8 * j)) & 0xFF) - 32;
      }
    }
    const uint8_t *hd = sc + (u / 8) * 32;
    const float d = f16_bits_to_f32(hd[16] | (hd[17] << 8));
    const int r = (int)(u % 8);
    for (int p = 0; p < 2; ++p) {
      scale[p] = __fmul_rn(d, (float)(int8_t)hd[2 * r + p]);
      min[p] = 0.0f;
    }
    return;
  }
  if (fmt == Q8_0) {
    const uint4 a = *reinterpret_cast<const uint4 *>(w + row * L.qs_row + u * 32);
    const uint4 b = *reinterpret_cast<const uint4 *>(w + row * L.qs_row + u * 32 + 16);
    const uint32_t words[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    for (int i = 0; i < 32; ++i) q[i] = (int)(int8_t)((words[i / 4] >> (8 * (i % 4))) & 0xff);
    scale[0] = scale[1] = f16_bits_to_f32(sc[u * 2] | (sc[u * 2 + 1] << 8));
    min[0] = min[1] = 0.0f;
    return;
  }
  const uint4 v = *reinterpret_cast<const uint4 *>(w + row * L.qs_row + u * 16);
  const uint32_t words[4] = {v.x, v.y, v.z, v.w};
  if (fmt == Q5_K) {
    const uint8_t *hd = sc + (u / 8) * 48;
    const uint32_t hb = *reinterpret_cast<const uint32_t *>(hd + 16 + 4 * (u % 8));
    for (int wd = 0; wd < 4; ++wd) {
      uint32_t ev, od;
      q5k_codes(words[wd], hb, wd, ev, od);
      for (int j = 0; j < 4; ++j) {
        q[8 * wd + 2 * j] = (int)((ev >> (8 * j)) & 0xFF);
        q[8 * wd + 2 * j + 1] = (int)((od >> (8 * j)) & 0xFF);
      }
    }
    const uint4 h = *reinterpret_cast<const uint4 *>(hd);
    const float d = f16_bits_to_f32(h.x), dmin = f16_bits_to_f32(h.x >> 16);
    uint32_t s, m;
    q4k_scale_min((int)(u % 8), h.y, h.z, h.w, s, m);
    scale[0] = scale[1] = __fmul_rn(d, (float)s);
    min[0] = min[1] = __fmul_rn(dmin, (float)m);
    return;
  }
  for (int i = 0; i < 32; ++i) {
    const uint32_t nib = (words[i / 8] >> (4 * (i % 8))) & 0xF;
    q[i] = fmt == Q4_K ? (int)nib : (fmt == Q4_0 ? (int)nib - 8 : iq4nl_value((int)nib));
  }
  if (fmt == Q4_K) {
    const uint4 h = *reinterpret_cast<const uint4 *>(sc + (u / 8) * 16);
    const float d = f16_bits_to_f32(h.x), dmin = f16_bits_to_f32(h.x >> 16);
    uint32_t s, m;
    q4k_scale_min((int)(u % 8), h.y, h.z, h.w, s, m);
    scale[0] = scale[1] = __fmul_rn(d, (float)s);
    min[0] = min[1] = __fmul_rn(dmin, (float)m);
  } else {
    scale[0] = scale[1] = f16_bits_to_f32(sc[u * 2] | (sc[u * 2 + 1] << 8));
    min[0] = min[1] = 0.0f;
  }
}

// One element of decode_run: value i of run u of stored row `row`, as
// scale[i / 16] * q[i] - min[i / 16] with the same roundings, decoding only
// that element's code and its run's factors (the input-major product and the
// embedding lookup use one value of a run at a time).
__device__ __forceinline__ float decode_value(int fmt, const uint8_t *__restrict__ w,
                                              const Layout &L, uint64_t row, uint64_t u, int i) {
  const uint8_t *sc = w + L.qs_bytes + row * L.sc_row;
  const uint8_t *qrow = w + row * L.qs_row;
  int q;
  float scale, mn = 0.0f;
  if (fmt == Q6_K) {
    const int wd = i / 8;
    const uint32_t word = *reinterpret_cast<const uint32_t *>(qrow + q6k_nib_offset(u) + 4 * wd);
    const uint32_t hw = *reinterpret_cast<const uint32_t *>(qrow + q6k_high_offset(u) + 4 * (wd >> 1));
    uint32_t ev, od;
    q6k_codes(word, hw, wd, ev, od);
    q = (int)((((i & 1) ? od : ev) >> (8 * ((i % 8) / 2))) & 0xFF) - 32;
    const uint8_t *hd = sc + (u / 8) * 32;
    const float d = f16_bits_to_f32(hd[16] | (hd[17] << 8));
    scale = __fmul_rn(d, (float)(int8_t)hd[2 * (int)(u % 8) + i / 16]);
  } else if (fmt == Q8_0) {
    q = (int)(int8_t)qrow[u * 32 + i];
    scale = f16_bits_to_f32(sc[u * 2] | (sc[u * 2 + 1] << 8));
  } else {
    const uint32_t word = *reinterpret_cast<const uint32_t *>(qrow + u * 16 + 4 * (i / 8));
    if (fmt == Q5_K || fmt == Q4_K) {
      const uint8_t *hd = sc + (u / 8) * (fmt == Q5_K ? 48 : 16);
      if (fmt == Q5_K) {
        const uint32_t hb = *reinterpret_cast<const uint32_t *>(hd + 16 + 4 * (u % 8));
        uint32_t ev, od;
        q5k_codes(word, hb, i / 8, ev, od);
        q = (int)((((i & 1) ? od : ev) >> (8 * ((i % 8) / 2))) & 0xFF);
      } else {
        q = (int)((word >> (4 * (i % 8))) & 0xF);
      }
      const uint4 h = *reinterpret_cast<const uint4 *>(hd);
      const float d = f16_bits_to_f32(h.x), dmin = f16_bits_to_f32(h.x >> 16);
      uint32_t s, m;
      q4k_scale_min((int)(u % 8), h.y, h.z, h.w, s, m);
      scale = __fmul_rn(d, (float)s);
      mn = __fmul_rn(dmin, (float)m);
    } else {
      const int nib = (int)((word >> (4 * (i % 8))) & 0xF);
      q = fmt == Q4_0 ? nib - 8 : iq4nl_value(nib);
      scale = f16_bits_to_f32(sc[u * 2] | (sc[u * 2 + 1] << 8));
    }
  }
  return __fsub_rn(__fmul_rn(scale, (float)q), mn);
}

__global__ void mgb_dequantize_kernel(int fmt, const uint8_t *__restrict__ w, uint64_t n, uint64_t k,
                                  float *__restrict__ out) {
  const Layout L(fmt, n, k);
  const uint64_t runs_per_row = k / RUN, total = n * runs_per_row;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = t / runs_per_row, u = t % runs_per_row;
    int q[32];
    float scale[2], min[2];
    decode_run(fmt, w, L, row, u, q, scale, min);
    float4 *o = reinterpret_cast<float4 *>(out + row * k + u * RUN);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v[4];
      for (int e = 0; e < 4; ++e)
        v[e] = __fsub_rn(__fmul_rn(scale[i / 4], (float)q[4 * i + e]), min[i / 4]);
      o[i] = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

// Input-major product (`axpy_columns`, src/native/quant.rs:1658-1689): W's
// stored rows are the k input rows, y[m, n_cols].  One thread per (output row
// r, output column c); sums x[r, j] * value(j, c) over j in order, skipping
// x == 0 like the reference.
__global__ void mgb_input_major_kernel(int fmt, const uint8_t *__restrict__ w, uint64_t k_rows,
                                   uint64_t n_cols, const float *__restrict__ x, uint64_t m,
                                   float *__restrict__ y) {
  const Layout L(fmt, k_rows, n_cols);
  const uint64_t total = m * n_cols;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = t / n_cols, c = t % n_cols;
    const uint64_t u = c / RUN;
    const int i = (int)(c % RUN);
    // eight input rows' loads in flight at a time; the products are still
    // added one by one in row order, zero activations skipped
    float acc = 0.0f;
    uint64_t j = 0;
    for (; j + 8 <= k_rows; j += 8) {
      float a[8], v[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        a[t] = x[r * k_rows + j + t];
        v[t] = decode_value(fmt, w, L, j + t, u, i);
      }
#pragma unroll
      for (int t = 0; t < 8; ++t)
        if (a[t] != 0.0f) acc = __fadd_rn(acc, __fmul_rn(a[t], v[t]));
    }
    for (; j < k_rows; ++j) {
      const float a = x[r * k_rows + j];
      if (a == 0.0f) continue;
      acc = __fadd_rn(acc, __fmul_rn(a, decode_value(fmt, w, L, j, u, i)));
    }
    y[t] = acc;
  }
}

// A token id is valid when it is a whole number in [0, vocab) (the
// reference's `raw_id < 0.0 || raw_id.fract() != 0.0 || raw_id as u64 >=
// vocab` check; NaN and infinities fail it).
__device__ __forceinline__ bool valid_token(float raw, uint64_t vocab) {
  return raw >= 0.0f && floorf(raw) == raw && (double)raw < (double)vocab;
}

// Packed-table embedding (`NativeState::embedding`, src/native/mod.rs:389-417):
// out[t, j] = value(token_t, j) (* scale), with value the dequantised
// element: stored row token_t, column j of an untransposed [vocab, dim] table,
// or stored row j, column token_t of a transposed [dim, vocab] one.  One
// thread per output element.  An invalid id writes zeros for its row and
// records its position (the smallest one wins) in *bad.
__global__ void mgb_embedding_kernel(int fmt, const uint8_t *__restrict__ w, uint64_t stored_rows,
                                 uint64_t stored_cols, int transposed, const float *__restrict__ ids,
                                 uint64_t count, int has_scale, float scale, float *__restrict__ out,
                                 uint32_t *bad) {
  const Layout L(fmt, stored_rows, stored_cols);
  const uint64_t vocab = transposed ? stored_cols : stored_rows;
  const uint64_t dim = transposed ? stored_rows : stored_cols;
  const uint64_t total = count * dim;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t t = e / dim, j = e % dim;
    const float raw = ids[t];
    if (!valid_token(raw, vocab)) {
      out[e] = 0.0f;
      if (j == 0 && bad) atomicMin(bad, (uint32_t)(t < 0xFFFFFFFEull ? t : 0xFFFFFFFEull));
      continue;
    }
    const uint64_t token = (uint64_t)raw;
    const uint64_t row = transposed ? j : token, col = transposed ? token : j;
    float v = decode_value(fmt, w, L, row, col / RUN, (int)(col % RUN));
    if (has_scale) v = __fmul_rn(v, scale);
    out[e] = v;
  }
}

// The same lookup in an f32 table [vocab, dim] (`f32_embedding`,
// src/native/mod.rs:238-263), with the optional scale.
__global__ void mgb_embedding_f32_kernel(const float *__restrict__ table, uint64_t vocab, uint64_t dim,
                                     const float *__restrict__ ids, uint64_t count, int has_scale,
                                     float scale, float *__restrict__ out, uint32_t *bad) {
  const uint64_t total = count * dim;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t t = e / dim, j = e % dim;
    const float raw = ids[t];
    if (!valid_token(raw, vocab)) {
      out[e] = 0.0f;
      if (j == 0 && bad) atomicMin(bad, (uint32_t)(t < 0xFFFFFFFEull ? t : 0xFFFFFFFEull));
      continue;
    }
    const float v = table[(uint64_t)raw * dim + j];
    out[e] = has_scale ? __fmul_rn(v, scale) : v;
  }
}

static int grid_for(uint64_t work, int threads) {
  uint64_t blocks = ceil_div(work, threads);
  return (int)(blocks > 65535 * 4 ? 65535 * 4 : (blocks ? blocks : 1));
}

cudaError_t launch_repack(int fmt, const void *src, uint64_t n, uint64_t k, void *dst,
                          cudaStream_t stream) {
  mgb_repack_kernel<<<grid_for(n * (k / RUN), 256), 256, 0, stream>>>(
      fmt, static_cast<const uint8_t *>(src), n, k, static_cast<uint8_t *>(dst));
  return cudaGetLastError();
}

cudaError_t launch_dequantize(int fmt, const void *w, uint64_t n, uint64_t k, float *out,
                              cudaStream_t stream) {
  mgb_dequantize_kernel<<<grid_for(n * (k / RUN), 256), 256, 0, stream>>>(
      fmt, static_cast<const uint8_t *>(w), n, k, out);
  return cudaGetLastError();
}

cudaError_t launch_embedding(int fmt, const void *w, uint64_t stored_rows, uint64_t stored_cols,
                             int transposed, const float *ids, uint64_t count, int has_scale,
                             float scale, float *out, uint32_t *bad, cudaStream_t stream) {
  if (bad) {
    cudaError_t e = cudaMemsetAsync(bad, 0xFF, sizeof(uint32_t), stream);
    if (e != cudaSuccess) return e;
  }
  const uint64_t dim = transposed ? stored_rows : stored_cols;
  if (count * dim == 0) return cudaSuccess;
  mgb_embedding_kernel<<<grid_for(count * dim, 256), 256, 0, stream>>>(
      fmt, static_cast<const uint8_t *>(w), stored_rows, stored_cols, transposed, ids, count,
      has_scale, scale, out, bad);
  return cudaGetLastError();
}

cudaError_t launch_embedding_f32(const float *table, uint64_t vocab, uint64_t dim, const float *ids,
                                 uint64_t count, int has_scale, float scale, float *out,
                                 uint32_t *bad, cudaStream_t stream) {
  if (bad) {
    cudaError_t e = cudaMemsetAsync(bad, 0xFF, sizeof(uint32_t), stream);
    if (e != cudaSuccess) return e;
  }
  if (count * dim == 0) return cudaSuccess;
  mgb_embedding_f32_kernel<<<grid_for(count * dim, 256), 256, 0, stream>>>(table, vocab, dim, ids, count,
                                                                      has_scale, scale, out, bad);
  return cudaGetLastError();
}

cudaError_t launch_input_major(int fmt, const void *w, uint64_t k_rows, uint64_t n_cols,
                               const float *x, uint64_t m, float *y, cudaStream_t stream) {
  mgb_input_major_kernel<<<grid_for(m * n_cols, 256), 256, 0, stream>>>(
      fmt, static_cast<const uint8_t *>(w), k_rows, n_cols, x, m, y);
  return cudaGetLastError();
}

}  // namespace mgb
