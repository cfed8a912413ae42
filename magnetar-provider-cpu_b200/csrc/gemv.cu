// Decode GEMV for packed weights on sm_100a: y[m, n] = x[m, k] * W^T for
// m <= 2 activation rows.  Replaces the reference's `columns_q4k_avx2` /
// `columns_avx2` / `columns_iq4nl_avx2` (src/native/quant.rs:604-744,
// :1438-1483) at the accuracy of its f32 path (:559-597).
//
// Main kernel (k % 256 == 0), persistent and bulk-copy staged:
//   warp 0      one thread streams the CTA's rows of both planes of W (the
//               quant plane and the scale plane; consecutive rows are
//               contiguous, so one cp.async.bulk per plane per stage) into a
//               ring of shared-memory stages, starting before anything else:
//               the bytes in flight cost no registers.
//   warps 1..   consumer teams of ceil(k / 1024) warps; thread u of a team owns
//               run u of K (32 values) for the whole kernel and reads its 16
//               (Q8_0: 32) quant bytes of each staged row from shared memory.
//               Per row the team reduces its partial sums with shuffles and a
//               fixed-order pass over its warps (deterministic).
// Programmatic dependent launch: the producer starts streaming weights at
// once (they never depend on an earlier kernel); consumers execute
// griddepcontrol.wait before reading x or writing y.
//
// Arithmetic: each thread holds its run of x as 16-bit integers
// x ~= dx * v, dx = max|x| / 32767 over the run (|error| <= dx / 2, i.e.
// <= 2^-16 of the run's largest value), split into a signed high byte and an
// unsigned low byte.  Integer dot products with the quants (dp4a, exact,
// int32) give sum(q v) = 256 sum(q hi) + sum(q lo); the run then contributes
// dx * scale * sum(q v) - min * sum(x) in f32, sum(x) taken from the exact f32
// values.  Relative error ~1e-5, against the 1e-3 tolerance of the GEMV.
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

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Four-way byte dot products, accumulating into c (dp4a; u = unsigned bytes,
// s = signed bytes; first operand a, second b).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One thread's run of one activation row as 16-bit integers: dx, the exact
// f32 sum, and the high / low bytes packed four to a word in the order the
// format's quant words use (pair order for the linear 4-bit formats: word 2w
// holds values 8w+0,2,4,6 and word 2w+1 values 8w+1,3,5,7; value order
// otherwise).
struct XRun {
  float dx, sum;
  float hs[2];  // sums of values 0..15 and 16..31 (Q6_K: one scale per half)
  uint32_t hi[8], lo[8];
};

// Quantises one run: q = round(v / dx) with dx = max|v| / 32767, so |q| <=
// 32767.  The rounding adds 1.5 * 2^23 in one fused multiply-add, which leaves
// 0x4B400000 + q in the float's bits: byte 0 is q's low byte and byte 1 its
// high byte (two's complement, |q| < 2^22), so byte permutes build the words.
__device__ __forceinline__ void pack_run(const float (&v)[32], bool pair_order, XRun &r) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i += 4) s += (v[i] + v[i + 1]) + (v[i + 2] + v[i + 3]);
  float mx[16];  // max |v| as a tree (depth 5, not a chain of 32)
#pragma unroll
  for (int i = 0; i < 16; ++i) mx[i] = fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1]));
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
  const float amax = mx[0];
  r.sum = s;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float t = 0.f;
#pragma unroll
    for (int i = 16 * h; i < 16 * h + 16; i += 4) t += (v[i] + v[i + 1]) + (v[i + 2] + v[i + 3]);
    r.hs[h] = t;
  }
  r.dx = amax / 32767.f;
  const float inv = amax > 0.f ? 32767.f / amax : 0.f;
  uint32_t b[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) b[i] = __float_as_uint(fmaf(v[i], inv, 12582912.f));
#pragma unroll
  for (int wd = 0; wd < 8; ++wd) {
    // pair order: word 2w -> values 8w + 2j, word 2w + 1 -> values 8w + 2j + 1
    int e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = pair_order ? 8 * (wd / 2) + 2 * j + (wd & 1) : 4 * wd + j;
    const uint32_t l01 = __byte_perm(b[e[0]], b[e[1]], 0x0040u), l23 = __byte_perm(b[e[2]], b[e[3]], 0x0040u);
    const uint32_t h01 = __byte_perm(b[e[0]], b[e[1]], 0x0051u), h23 = __byte_perm(b[e[2]], b[e[3]], 0x0051u);
    r.lo[wd] = __byte_perm(l01, l23, 0x5410u);
    r.hi[wd] = __byte_perm(h01, h23, 0x5410u);
  }
}

// sum(q v) for a run of 4-bit quants in nibble pairs (byte i = values 2i, 2i+1).
__device__ __forceinline__ int dot_nib(const uint4 &qs, const XRun &x) {
  const uint32_t words[4] = {qs.x, qs.y, qs.z, qs.w};
  int sh = 0, sl = 0;
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    const uint32_t ev = words[wd] & 0x0F0F0F0Fu;         // values 8wd + 0, 2, 4, 6
    const uint32_t od = (words[wd] >> 4) & 0x0F0F0F0Fu;  // values 8wd + 1, 3, 5, 7
    sh = dp4a_us(ev, x.hi[2 * wd], sh);
    sh = dp4a_us(od, x.hi[2 * wd + 1], sh);
    sl = dp4a_uu(ev, x.lo[2 * wd], sl);
    sl = dp4a_uu(od, x.lo[2 * wd + 1], sl);
  }
  return sh * 256 + sl;
}

// sum(q v) for a run of signed byte quants in value order.
__device__ __forceinline__ int dot_s8(const uint32_t (&q)[8], const XRun &x) {
  int sh = 0, sl = 0;
#pragma unroll
  for (int wd = 0; wd < 8; ++wd) {
    sh = dp4a_ss(q[wd], x.hi[wd], sh);
    sl = dp4a_su(q[wd], x.lo[wd], sl);
  }
  return sh * 256 + sl;
}

// IQ4_NL codebook lookup: the 8 indices of word `v` (nibble order = value
// order) -> two words of signed codebook bytes.
__device__ __forceinline__ void iq4_lookup(uint32_t v, const uint32_t t[4], uint32_t &o0,
                                           uint32_t &o1) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t s = (v >> (16 * h)) & 0xFFFFu;
    const uint32_t sel = s & 0x7777u;
    const uint32_t low = __byte_perm(t[0], t[1], sel);
    const uint32_t high = __byte_perm(t[2], t[3], sel);
    const uint32_t r = __byte_perm(low, high, 0x3210u | ((s & 0x8888u) >> 1));
    if (h == 0) o0 = r; else o1 = r;
  }
}

__device__ __forceinline__ void iq4_table(uint32_t lut[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) v |= (uint32_t)(iq4nl_value(4 * i + b) & 0xff) << (8 * b);
    lut[i] = v;
  }
}

// The partial dot products of one run of one weight row with MR activation
// rows.  qa (and qb for Q8_0) hold the run's quant bytes; hd the Q4_K header
// of its super-block; dh the f16 scale of the other formats; j the run's index
// in its super-block.
template <int FMT, int MR>
__device__ __forceinline__ void run_partials(const uint4 &qa, const uint4 &qb, const uint4 &hd,
                                             uint32_t dh, int j, const XRun (&x)[MR],
                                             const uint32_t lut[4], float (&part)[MR]) {
  if (FMT == Q6_K) {
    // qa: nibble pairs; qb.x, qb.y: the two high words; hd: the 16 int8
    // scales of the super-block; dh: d
    const float d = f16_bits_to_f32(dh);
    const uint32_t sw = (j < 2 ? hd.x : j < 4 ? hd.y : j < 6 ? hd.z : hd.w) >> (16 * (j & 1));
    const float s0 = d * (float)(int8_t)(sw & 0xFF), s1 = d * (float)(int8_t)((sw >> 8) & 0xFF);
    const uint32_t words[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      int sh[2] = {0, 0}, sl[2] = {0, 0};
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) {
        uint32_t ev, od;
        q6k_codes(words[wd], wd < 2 ? qb.x : qb.y, wd, ev, od);
        sh[wd >> 1] = dp4a_us(ev, x[m].hi[2 * wd], sh[wd >> 1]);
        sh[wd >> 1] = dp4a_us(od, x[m].hi[2 * wd + 1], sh[wd >> 1]);
        sl[wd >> 1] = dp4a_uu(ev, x[m].lo[2 * wd], sl[wd >> 1]);
        sl[wd >> 1] = dp4a_uu(od, x[m].lo[2 * wd + 1], sl[wd >> 1]);
      }
      part[m] = ((s0 * x[m].dx) * (float)(sh[0] * 256 + sl[0]) - (32.f * s0) * x[m].hs[0]) +
                ((s1 * x[m].dx) * (float)(sh[1] * 256 + sl[1]) - (32.f * s1) * x[m].hs[1]);
    }
  } else if (FMT == Q4_K || FMT == Q5_K) {
    const float d = f16_bits_to_f32(hd.x), dmin = f16_bits_to_f32(hd.x >> 16);
    uint32_t sc, mn;
    q4k_scale_min(j, hd.y, hd.z, hd.w, sc, mn);
    const float s = d * (float)sc, mv = dmin * (float)mn;
    uint4 q = qa;
    if (FMT == Q5_K) {  // 5-bit codes in the nibble-pair order (qb.x: the fifth bits)
      uint32_t e[4], o[4];
      const uint32_t words[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
      for (int wd = 0; wd < 4; ++wd) q5k_codes(words[wd], qb.x, wd, e[wd], o[wd]);
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        int sh = 0, sl = 0;
#pragma unroll
        for (int wd = 0; wd < 4; ++wd) {
          sh = dp4a_us(e[wd], x[m].hi[2 * wd], sh);
          sh = dp4a_us(o[wd], x[m].hi[2 * wd + 1], sh);
          sl = dp4a_uu(e[wd], x[m].lo[2 * wd], sl);
          sl = dp4a_uu(o[wd], x[m].lo[2 * wd + 1], sl);
        }
        part[m] = (s * x[m].dx) * (float)(sh * 256 + sl) - mv * x[m].sum;
      }
    } else {
#pragma unroll
      for (int m = 0; m < MR; ++m)
        part[m] = (s * x[m].dx) * (float)dot_nib(q, x[m]) - mv * x[m].sum;
    }
  } else if (FMT == Q4_0) {
    const float d = f16_bits_to_f32(dh);
#pragma unroll
    for (int m = 0; m < MR; ++m)
      part[m] = d * (x[m].dx * (float)dot_nib(qa, x[m]) - 8.f * x[m].sum);
  } else if (FMT == Q8_0) {
    const float d = f16_bits_to_f32(dh);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int m = 0; m < MR; ++m) part[m] = (d * x[m].dx) * (float)dot_s8(q, x[m]) + 0.f * x[m].sum;
  } else {  // IQ4_NL
    const float d = f16_bits_to_f32(dh);
    uint32_t q[8];
    const uint32_t words[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) iq4_lookup(words[wd], lut, q[2 * wd], q[2 * wd + 1]);
#pragma unroll
    for (int m = 0; m < MR; ++m) part[m] = (d * x[m].dx) * (float)dot_s8(q, x[m]) + 0.f * x[m].sum;
  }
}

// A run's two f32 factors, decoded once from the scale plane: the multiplier
// of its integer dot product and the multiplier of its activation sum, so that
// the run contributes (s * dx) * dot - m * sum.  Q4_K: s = d * scale_j,
// m = dmin * min_j; Q4_0: s = d, m = 8 d (q - 8); Q8_0, IQ4_NL: s = d, m = 0.
// Q6_K: the two halves' scales d * sc (each half contributes
// (s * dx) * dot - 32 s * sum over its 16 values).
template <int FMT>
__device__ __forceinline__ float2 decode_run_scale(const uint8_t *srow, int uu) {
  if (FMT == Q6_K) {  // the scales of the run's two halves (q - 32: no separate min)
    const uint8_t *hd = srow + (uu >> 3) * 32;
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(hd + 16));
    const uint16_t sp = *reinterpret_cast<const uint16_t *>(hd + 2 * (uu & 7));
    return make_float2(d * (float)(int8_t)(sp & 0xFF), d * (float)(int8_t)(sp >> 8));
  } else if (FMT == Q4_K || FMT == Q5_K) {
    const uint4 hd = *reinterpret_cast<const uint4 *>(srow + (uu >> 3) * (FMT == Q5_K ? 48 : 16));
    const float d = f16_bits_to_f32(hd.x), dmin = f16_bits_to_f32(hd.x >> 16);
    uint32_t sc, mn;
    q4k_scale_min(uu & 7, hd.y, hd.z, hd.w, sc, mn);
    return make_float2(d * (float)sc, dmin * (float)mn);
  } else {
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(srow + uu * 2));
    return make_float2(d, FMT == Q4_0 ? 8.f * d : 0.f);
  }
}

// Partial dot products of one run (uu) of RPT weight rows with MR activation
// rows.  The rows' quant words and decoded factors are loaded first; the
// integer dot products then run word by word across all rows, so 2 * RPT * MR
// independent dp4a chains interleave instead of two per row.  Row i's quants
// start at q + i * q_stride, its scale-plane bytes at sc + i * sc_stride; its
// factors are decoded here (`fused`) or were decoded earlier into
// dec[i * dec_stride] (the stages that land before the dependency wait).
template <int FMT, int MR, int RPT>
__device__ __forceinline__ void rows_partials(const uint8_t *q, size_t q_stride, const float2 *dec,
                                              size_t dec_stride, int uu, const XRun (&x)[MR],
                                              const uint32_t lut[4], float (&part)[RPT * MR],
                                              const uint8_t *sc = nullptr, size_t sc_stride = 0,
                                              bool fused = false) {
  int sh[RPT][MR], sl[RPT][MR];
  float2 sm[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    sm[i] = fused ? decode_run_scale<FMT>(sc + (size_t)i * sc_stride, uu) : dec[(size_t)i * dec_stride];
#pragma unroll
    for (int m = 0; m < MR; ++m) sh[i][m] = sl[i][m] = 0;
  }
  if (FMT == Q6_K) {
    uint4 qa[RPT];
    uint2 qh[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      qa[i] = *reinterpret_cast<const uint4 *>(q + (size_t)i * q_stride + q6k_nib_offset(uu));
      qh[i] = *reinterpret_cast<const uint2 *>(q + (size_t)i * q_stride + q6k_high_offset(uu));
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {  // the run's halves: one scale each
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int m = 0; m < MR; ++m) sh[i][m] = sl[i][m] = 0;
#pragma unroll
      for (int wd = 2 * hf; wd < 2 * hf + 2; ++wd)
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const uint32_t v = wd == 0 ? qa[i].x : wd == 1 ? qa[i].y : wd == 2 ? qa[i].z : qa[i].w;
          uint32_t ev, od;
          q6k_codes(v, hf == 0 ? qh[i].x : qh[i].y, wd, ev, od);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            sh[i][m] = dp4a_us(ev, x[m].hi[2 * wd], sh[i][m]);
            sh[i][m] = dp4a_us(od, x[m].hi[2 * wd + 1], sh[i][m]);
            sl[i][m] = dp4a_uu(ev, x[m].lo[2 * wd], sl[i][m]);
            sl[i][m] = dp4a_uu(od, x[m].lo[2 * wd + 1], sl[i][m]);
          }
        }
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const float sc = hf == 0 ? sm[i].x : sm[i].y;
          const float c = (sc * x[m].dx) * (float)(sh[i][m] * 256 + sl[i][m]) - (32.f * sc) * x[m].hs[hf];
          part[i * MR + m] = hf == 0 ? c : part[i * MR + m] + c;
        }
    }
    return;
  }
  if (FMT == Q8_0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // 16 bytes of each row's run at a time
      uint4 qa[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i)
        qa[i] = *reinterpret_cast<const uint4 *>(q + (size_t)i * q_stride + uu * 32 + 16 * h);
#pragma unroll
      for (int wd = 0; wd < 4; ++wd)
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const uint32_t v = wd == 0 ? qa[i].x : wd == 1 ? qa[i].y : wd == 2 ? qa[i].z : qa[i].w;
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            sh[i][m] = dp4a_ss(v, x[m].hi[4 * h + wd], sh[i][m]);
            sl[i][m] = dp4a_su(v, x[m].lo[4 * h + wd], sl[i][m]);
          }
        }
    }
  } else {
    uint4 qa[RPT];
    uint32_t hb[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      qa[i] = *reinterpret_cast<const uint4 *>(q + (size_t)i * q_stride + uu * 16);
      hb[i] = FMT == Q5_K ? *reinterpret_cast<const uint32_t *>(sc + (size_t)i * sc_stride +
                                                                 (uu >> 3) * 48 + 16 + (uu & 7) * 4)
                          : 0u;
    }
#pragma unroll
    for (int wd = 0; wd < 4; ++wd)
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const uint32_t v = wd == 0 ? qa[i].x : wd == 1 ? qa[i].y : wd == 2 ? qa[i].z : qa[i].w;
        if (FMT == IQ4_NL) {
          uint32_t c0, c1;  // codebook bytes of values 8wd + 0..3 and 8wd + 4..7
          iq4_lookup(v, lut, c0, c1);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            sh[i][m] = dp4a_ss(c0, x[m].hi[2 * wd], sh[i][m]);
            sh[i][m] = dp4a_ss(c1, x[m].hi[2 * wd + 1], sh[i][m]);
            sl[i][m] = dp4a_su(c0, x[m].lo[2 * wd], sl[i][m]);
            sl[i][m] = dp4a_su(c1, x[m].lo[2 * wd + 1], sl[i][m]);
          }
        } else {  // Q4_K, Q4_0: nibble pairs; Q5_K: plus each value's fifth bit
          uint32_t ev = v & 0x0F0F0F0Fu;         // values 8wd + 0, 2, 4, 6
          uint32_t od = (v >> 4) & 0x0F0F0F0Fu;  // values 8wd + 1, 3, 5, 7
          if (FMT == Q5_K) q5k_codes(v, hb[i], wd, ev, od);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            sh[i][m] = dp4a_us(ev, x[m].hi[2 * wd], sh[i][m]);
            sh[i][m] = dp4a_us(od, x[m].hi[2 * wd + 1], sh[i][m]);
            sl[i][m] = dp4a_uu(ev, x[m].lo[2 * wd], sl[i][m]);
            sl[i][m] = dp4a_uu(od, x[m].lo[2 * wd + 1], sl[i][m]);
          }
        }
      }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const float dot = (float)(sh[i][m] * 256 + sl[i][m]);
      if (FMT == Q4_K || FMT == Q4_0 || FMT == Q5_K)
        part[i * MR + m] = (sm[i].x * x[m].dx) * dot - sm[i].y * x[m].sum;
      else
        part[i * MR + m] = (sm[i].x * x[m].dx) * dot + 0.f * x[m].sum;  // NaN / Inf in x reach y
    }
}

template <int FMT, int MR>
__device__ __forceinline__ void load_x(const float *__restrict__ x, int k, int u, bool active,
                                       XRun (&xr)[MR]) {
  constexpr bool pair = FMT == Q4_K || FMT == Q4_0 || FMT == Q6_K || FMT == Q5_K;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      // Ordinary (L1-cacheable) loads, never the non-coherent read-only path
      // (ld.global.nc): under programmatic dependent launch the kernel starts
      // while the previous one may still write x, and with ld.global.nc, one
      // warp waiting and the others released by a barrier, only the waiting
      // warp was seen to read fresh values.  L2-only loads (ld.global.cg)
      // were 3.5 us slower per config-0 link than these.
      if (active) {
        const float *src = x + (size_t)m * k + (size_t)u * 32 + 4 * i;
        asm volatile("ld.global.ca.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                     : "l"(src));
      }
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
    pack_run(v, pair, xr[m]);
  }
}

// Sums NV per-lane values (NV a power of two <= 32) over the warp with a
// transposing butterfly: each step halves the values a lane keeps and sends
// the other half to its partner, so NV values cost NV - 1 + log2(32 / NV)
// shuffles instead of 5 NV.  Returns the total of value lane / (32 / NV).
template <int NV>
__device__ __forceinline__ float warp_sum_transpose(float (&v)[NV], int lane) {
#pragma unroll
  for (int c = NV, o = 16; c > 1; c >>= 1, o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < c / 2; ++j) {
      const float send = upper ? v[j] : v[j + c / 2];
      const float keep = upper ? v[j + c / 2] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float s = v[0];
#pragma unroll
  for (int o = 16 / NV; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// ---- main kernel: bulk-copy staged, persistent ----------------------------------------

// Rows per team per stage: 8 for one activation row of a 4-bit format in a
// 288-thread CTA (16 independent integer dot chains per thread), otherwise 4
// (two activation rows; Q8_0's twice larger rows, which would leave room for
// one ring slot; or the 64 registers of a 1024-thread CTA).
template <int FMT, int MR, int MAXT>
__host__ __device__ constexpr int rows_per_team() {
  return MR == 1 && FMT != Q8_0 && MAXT <= 288 ? 8 : 4;
}

struct GemvStaged {
  int n, k;
  int teams, team_warps;  // consumer geometry
  int stages;             // ring slots (never more than a CTA's stages of work)
  int chunk;              // stages per reduction pass
  int rows_per_cta;
  uint32_t stage_bytes, qs_stage_bytes;
  uint32_t dec_stage_bytes;  // decoded run factors of one stage: rows * runs * 8
  int addend_mode;
  const float *addend;
  OutSpec out;
  int *err;
};

template <int FMT, int MR, int MAXT, int MINB>
__global__ void __launch_bounds__(MAXT, MINB)
    mgb_gemv_staged_kernel(const uint8_t *__restrict__ w, const float *__restrict__ x,
                       const GemvStaged p) {
  constexpr int RPT = rows_per_team<FMT, MR, MAXT>();
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L(FMT, (uint64_t)p.n, (uint64_t)p.k);
  const int S = p.stages;
  const int TR = p.teams * RPT;  // rows per stage
  const int runs = p.k / RUN;
  float2 *dec = reinterpret_cast<float2 *>(smem + (size_t)S * p.stage_bytes);  // [S][TR][runs]
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * (p.stage_bytes + p.dec_stage_bytes));
  uint64_t *empty = full + S;
  float *red = reinterpret_cast<float *>(empty + S);  // [teams][chunk][RPT][team_warps][MR]
  const int consumer_warps = p.teams * p.team_warps;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(p.n, r0 + p.rows_per_cta);
  const int nstages = r1 > r0 ? (r1 - r0 + TR - 1) / TR : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], consumer_warps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      grid_launch_dependents();
      int issued = 0;
      for (int g = 0; g < nstages; ++g) {
        const int s = g % S;
        if (g >= S && !mbar_wait_backoff(&empty[s], ((g / S) - 1) & 1, p.err, 64)) break;
        const int row = r0 + g * TR;
        const int rows = min(TR, r1 - row);
        uint8_t *st = smem + (size_t)s * p.stage_bytes;
        const uint32_t qb = (uint32_t)(rows * L.qs_row), sb = (uint32_t)(rows * L.sc_row);
        mbar_arrive_expect_tx(&full[s], qb + sb);
        bulk_g2s(st, w + (size_t)row * L.qs_row, qb, &full[s]);
        bulk_g2s(st + p.qs_stage_bytes, w + L.qs_bytes + (size_t)row * L.sc_row, sb, &full[s]);
        issued = g + 1;
      }
      // every copy issued has landed before the CTA may exit
      for (int g = (issued > S ? issued - S : 0); g < issued; ++g)
        mbar_wait_backoff(&full[g % S], (g / S) & 1, nullptr);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  const int team = cw / p.team_warps, tw = cw % p.team_warps;
  const int u = tw * 32 + lane;  // this thread's run of K
  const bool active = u < runs;
  const int uu = active ? u : 0;  // idle lanes read a valid run; their result is dropped
  const int team_threads = p.team_warps * 32;
  float *red_team = red + (size_t)team * p.chunk * RPT * p.team_warps * MR;

  // A wait that gives up records the error and the thread stops waiting, but
  // it keeps stepping through every stage so its team's named barriers match.
  bool ok = true;
  auto wait_stage = [&](int g, uint32_t max_ns) {
    // lane 0 polls (sleeping between polls: a co-resident kernel may be
    // computing); once the phase is complete every lane's own try_wait
    // succeeds at once and acquires the bulk-copied bytes for that lane
    if (lane == 0) ok = ok && mbar_wait_backoff(&full[g % S], (g / S) & 1, p.err, max_ns);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) ok = mbar_try_wait(&full[g % S], (g / S) & 1);
  };
  // Each thread decodes the factors of its own run of its team's rows of
  // stage g into its own slots (no other thread reads them: no barrier).
  auto decode_stage = [&](int g) {
    const int s = g % S;
    const uint8_t *sc = smem + (size_t)s * p.stage_bytes + p.qs_stage_bytes;
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int lr = team * RPT + i;
      if (active) dec[((size_t)s * TR + lr) * runs + u] = decode_run_scale<FMT>(sc + (size_t)lr * L.sc_row, u);
    }
  };

  // Before the activations can be read: decode the run factors of the stages
  // already in flight (they land while the previous kernel drains).
  const int pre = min(S, nstages);
  for (int g = 0; g < pre; ++g) {
    wait_stage(g, 256);
    decode_stage(g);
  }

  // x may be the previous kernel's output; the weight stream above never
  // waits.  Every consumer warp waits for the previous grid itself (its
  // completion, its memory made visible to this grid; a hardware wait, nothing
  // spins), so its own loads of x are ordered after that grid's writes.  Each
  // thread then loads and quantises its own run of x.
  grid_dependency_wait();
  if (cw == 0 && p.out.wait_done) {
    // a tensor-parallel call's wait on the call before (peers' writes, which
    // the grid dependency does not cover): the acquire and the barrier below
    // order the other warps' loads after it
    out_wait_input(p.out, lane, p.err);
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  named_barrier(14, consumer_warps * 32);
  XRun xr[MR];
  load_x<FMT, MR>(x, p.k, u, active, xr);
  uint32_t lut[4] = {0, 0, 0, 0};
  if (FMT == IQ4_NL) iq4_table(lut);

  for (int g = 0; g < nstages; ++g) {
    const int s = g % S;
    if (g >= pre) wait_stage(g, 64);  // (its run factors are decoded in rows_partials)
    const uint8_t *st = smem + (size_t)s * p.stage_bytes;
    const int row0 = r0 + g * TR;
    // branch-free over the team's RPT rows (rows past the end of a partial
    // stage read stale stage bytes and are dropped), so their loads and
    // integer dot products interleave
    float part[RPT * MR];
    rows_partials<FMT, MR, RPT>(st + (size_t)team * RPT * L.qs_row, L.qs_row,
                                dec + ((size_t)s * TR + team * RPT) * runs + uu, runs, uu, xr, lut,
                                part, st + p.qs_stage_bytes + (size_t)team * RPT * L.sc_row,
                                L.sc_row, g >= pre);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const bool keep = ok && active && row0 + team * RPT + i < r1;
#pragma unroll
      for (int m = 0; m < MR; ++m) part[i * MR + m] = keep ? part[i * MR + m] : 0.f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage's bytes
    // warp totals of this stage's rows -> red[stage in chunk][row][warp][m]
    constexpr int NV = RPT * MR;
    const int c = g % p.chunk;
    const float tot = warp_sum_transpose<NV>(part, lane);
    if ((lane & (32 / NV - 1)) == 0) {
      const int v = lane / (32 / NV);
      red_team[((c * RPT + v / MR) * p.team_warps + tw) * MR + v % MR] = tot;
    }
    // every `chunk` stages (and after the last) the team sums its warps in a
    // fixed order and writes y
    if (c == p.chunk - 1 || g == nstages - 1) {
      named_barrier(1 + team, team_threads);
      const int g0 = g - c;
      for (int t = tw * 32 + lane; t < (c + 1) * NV; t += team_threads) {
        const int cc = t / NV, i = (t % NV) / MR, m = t % MR;
        const int row = r0 + (g0 + cc) * TR + team * RPT + i;
        if (row < r1) {
          float sum = 0.f;
          for (int wi = 0; wi < p.team_warps; ++wi)
            sum += red_team[((cc * RPT + i) * p.team_warps + wi) * MR + m];
          if (p.addend_mode == 1) sum = sum + __ldcg(p.addend + row);
          else if (p.addend_mode == 2) sum = sum + __ldcg(p.addend + (size_t)m * p.n + row);
          out_store(p.out, m, row, sum);
        }
      }
      named_barrier(1 + team, team_threads);
    }
  }
}

// ---- fallback kernel for k % 256 != 0 (ragged scale planes): direct loads -------------
//
// Thread u owns run u.  With more runs than threads (K > 32 * MAXT, MULTI) each
// thread takes runs u, u + blockDim, ... in turn and loads each run's x inside
// the row loop: slower, but no K is refused (a 405B-class down projection has
// K = 53,248).

template <int FMT, int MR, int R, int MAXT, bool MULTI>
__global__ void __launch_bounds__(MAXT, 1)
    mgb_gemv_simple_kernel(const uint8_t *__restrict__ w, int n, int k, const float *__restrict__ x,
                       const OutSpec out, const float *__restrict__ addend, int addend_mode,
                       int rows_per_cta, int *err) {
  __shared__ float red[2][32][R * MR];
  const Layout L(FMT, (uint64_t)n, (uint64_t)k);
  const int runs = k / RUN;
  const int u = threadIdx.x;
  const bool active = u < runs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  if (out.wait_done) {  // a tensor-parallel call's wait on the call before
    if (warp == 0) out_wait_input(out, lane, err);
    __syncthreads();
  }
  XRun xr[MR];
  if (!MULTI) load_x<FMT, MR>(x, k, u, active, xr);
  uint32_t lut[4] = {0, 0, 0, 0};
  if (FMT == IQ4_NL) iq4_table(lut);
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(n, r0 + rows_per_cta);
  const uint8_t *scale_plane = w + L.qs_bytes;
  const int groups = MULTI ? (runs + (int)blockDim.x - 1) / (int)blockDim.x : 1;
  int buf = 0;
  for (int r = r0; r < r1; r += R) {
    float part[R * MR];
#pragma unroll
    for (int i = 0; i < R * MR; ++i) part[i] = 0.f;
    for (int gi = 0; gi < groups; ++gi) {
      const int uu = MULTI ? u + gi * (int)blockDim.x : u;
      const bool act = MULTI ? uu < runs : active;
      if (MULTI) load_x<FMT, MR>(x, k, uu, act, xr);
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int row = r + i;
        if (act && row < r1) {
          const uint8_t *qrow = w + (size_t)row * L.qs_row;
          const uint8_t *srow = scale_plane + (size_t)row * L.sc_row;
          uint4 qa, qb = make_uint4(0, 0, 0, 0), hd = make_uint4(0, 0, 0, 0);
          uint32_t dh = 0;
          if (FMT == Q8_0) {
            qa = ld_stream_v4(qrow + (size_t)uu * 32);
            qb = ld_stream_v4(qrow + (size_t)uu * 32 + 16);
          } else if (FMT == Q6_K) {
            qa = ld_stream_v4(qrow + q6k_nib_offset((uint64_t)uu));
            const uint2 h2 = __ldg(reinterpret_cast<const uint2 *>(qrow + q6k_high_offset((uint64_t)uu)));
            qb = make_uint4(h2.x, h2.y, 0, 0);
          } else {
            qa = ld_stream_v4(qrow + (size_t)uu * 16);
          }
          if (FMT == Q4_K) hd = __ldg(reinterpret_cast<const uint4 *>(srow + (size_t)(uu >> 3) * 16));
          else if (FMT == Q5_K) {
            hd = __ldg(reinterpret_cast<const uint4 *>(srow + (size_t)(uu >> 3) * 48));
            qb.x = __ldg(reinterpret_cast<const uint32_t *>(srow + (size_t)(uu >> 3) * 48 + 16 + (uu & 7) * 4));
          } else if (FMT == Q6_K) {
            hd = __ldg(reinterpret_cast<const uint4 *>(srow + (size_t)(uu >> 3) * 32));
            dh = ld_nc_u16(srow + (size_t)(uu >> 3) * 32 + 16);
          } else dh = ld_nc_u16(srow + (size_t)uu * 2);
          float pm[MR];
          run_partials<FMT, MR>(qa, qb, hd, dh, uu & 7, xr, lut, pm);
#pragma unroll
          for (int m = 0; m < MR; ++m) part[i * MR + m] = gi == 0 ? pm[m] : part[i * MR + m] + pm[m];
        }
      }
    }
    {
      constexpr int NV = R * MR;
      const float tot = warp_sum_transpose<NV>(part, lane);
      if ((lane & (32 / NV - 1)) == 0) red[buf][warp][lane / (32 / NV)] = tot;
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
        out_store(out, m, row, s);
      }
    }
    buf ^= 1;
  }
}

// ---- launch --------------------------------------------------------------------------

template <typename K, typename... Args>
static cudaError_t launch_dependent(K kern, dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// The staged GEMV: a programmatic dependent of whatever precedes it on the
// stream (its weight stream starts at once; it waits before reading x).
constexpr size_t MAX_SMEM = 227 * 1024;
// Shared memory of one CTA when two kernels' CTAs are to share an SM (the next
// GEMV on the stream streams its weights while this one computes).
constexpr size_t CORESIDENT_SMEM = 112 * 1024;

// Geometry and shared-memory size of a staged launch.  One CTA per SM with 8
// consumer warps (k <= 8192) or one team of up to 31 warps (larger k); rows
// split evenly; a CTA's last stage may hold fewer than TR rows; the ring
// never has more slots than a CTA has stages.
template <int FMT, int MR, int MAXT>
static size_t staged_config(int n, int k, int sms, GemvStaged &p, int &grid, int &threads) {
  constexpr int RPT = rows_per_team<FMT, MR, MAXT>();
  const Layout L(FMT, (uint64_t)n, (uint64_t)k);
  const int runs = k / RUN;
  p.n = n;
  p.k = k;
  p.team_warps = (runs + 31) / 32;
  p.teams = p.team_warps >= 8 ? 1 : 8 / p.team_warps;
  const int TR = p.teams * RPT;
  p.qs_stage_bytes = (uint32_t)ceil_div((uint64_t)TR * L.qs_row, 128) * 128;
  p.stage_bytes = p.qs_stage_bytes + (uint32_t)ceil_div((uint64_t)TR * L.sc_row, 128) * 128;
  p.dec_stage_bytes = (uint32_t)(TR * runs * 8);
  threads = 32 * (1 + p.teams * p.team_warps);
  const int units = (int)ceil_div((uint64_t)n, (uint64_t)TR);
  // One CTA per SM, or two for long 288-thread launches (at least 16 stages
  // of rows per SM): twice the warps to hide the dot products' latency, at the
  // cost of the next kernel's CTAs finding no free slot until these finish
  // (graph-replayed chains, one B200: N = 65,536, K = 4,096: 43.5 -> 39.4 us;
  // N = 28,672, K = 8,192: 39.9 -> 38.4 us; shorter launches keep one).
  grid = (MAXT == 288 && units >= 16 * sms) ? 2 * sms : sms;
  if (grid > units) grid = units;
  p.rows_per_cta = (int)ceil_div((uint64_t)n, (uint64_t)grid);
  grid = (int)ceil_div((uint64_t)n, (uint64_t)p.rows_per_cta);
  const int nst = (int)ceil_div((uint64_t)p.rows_per_cta, (uint64_t)TR);
  // reduction buffer: as many stages as fit in 16 KB (usually all of a CTA's)
  const size_t red_stage = sizeof(float) * (size_t)p.teams * RPT * p.team_warps * MR;
  int chunk = (int)(16384 / red_stage);
  if (chunk > nst) chunk = nst;
  if (chunk < 1) chunk = 1;
  p.chunk = chunk;
  const size_t fixed = red_stage * chunk;
  const size_t per_stage = (size_t)p.stage_bytes + p.dec_stage_bytes + 16;
  // The 288-thread form stays within half an SM so the next GEMV's CTA can
  // stream its weights beside it; the 1024-thread form (k > 8192) takes the
  // whole SM's shared memory instead: its deeper ring is worth more than the
  // overlap (K = 28,672, N = 8,192: 47.6 -> 34.4 us).
  const size_t cap = MAXT > 288 ? MAX_SMEM - 1024 : CORESIDENT_SMEM;
  const size_t budget = cap > fixed ? cap - fixed : 0;
  int stages = (int)(budget / per_stage);
  if (stages > 8) stages = 8;
  if (stages > nst) stages = nst;
  if (stages < 1) stages = 1;
  p.stages = stages;
  return (size_t)stages * per_stage + fixed;
}

template <int FMT, int MR, int MAXT>
static bool staged_fits(int n, int k, int sms) {
  GemvStaged p;
  int grid, threads;
  return staged_config<FMT, MR, MAXT>(n, k, sms, p, grid, threads) <= MAX_SMEM;
}

// The staged GEMV: a programmatic dependent of whatever precedes it on the
// stream (its weight stream starts at once; it waits before reading x).
template <int FMT, int MR, int MAXT, int MINB>
static cudaError_t launch_staged(const void *w, int n, int k, const float *x, const OutSpec &out,
                                 const float *addend, int addend_mode, int *err, int sms,
                                 cudaStream_t stream) {
  GemvStaged p;
  int grid, threads;
  const size_t smem = staged_config<FMT, MR, MAXT>(n, k, sms, p, grid, threads);
  p.addend_mode = addend_mode;
  p.addend = addend;
  p.out = out;
  p.err = err;
  auto kern = mgb_gemv_staged_kernel<FMT, MR, MAXT, MINB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_dependent(kern, dim3((unsigned)grid), dim3((unsigned)threads), smem, stream,
                          static_cast<const uint8_t *>(w), x, p);
}

template <int FMT, int MR, int R, int MAXT>
static cudaError_t launch_simple(const void *w, int n, int k, const float *x, const OutSpec &out,
                                 const float *addend, int addend_mode, int *err, int sms,
                                 cudaStream_t stream) {
  const int runs = k / RUN;
  const bool multi = runs > MAXT;  // more runs than threads: each thread takes several
  const int threads = multi ? MAXT : ((runs + 31) / 32) * 32;
  int per_sm = 2048 / threads;
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 8) per_sm = 8;
  const int target = sms * per_sm;
  int rows = (int)ceil_div((uint64_t)n, (uint64_t)target);
  if (rows < 1) rows = 1;
  const int grid = (int)ceil_div((uint64_t)n, (uint64_t)rows);
  if (multi)
    mgb_gemv_simple_kernel<FMT, MR, R, MAXT, true><<<grid, threads, 0, stream>>>(
        static_cast<const uint8_t *>(w), n, k, x, out, addend, addend_mode, rows, err);
  else
    mgb_gemv_simple_kernel<FMT, MR, R, MAXT, false><<<grid, threads, 0, stream>>>(
        static_cast<const uint8_t *>(w), n, k, x, out, addend, addend_mode, rows, err);
  return cudaGetLastError();
}

static bool staged_ok(uint64_t k) { return k % 256 == 0 && k / RUN <= 31 * 32; }

template <int FMT, int MR>
static cudaError_t launch_fmt(const void *w, int n, int k, const float *x, const OutSpec &out,
                              const float *addend, int addend_mode, int *err, int sms,
                              cudaStream_t stream) {
  // (Two activation rows in the 1,024-thread forms: two launches, one per row.)
  const float *addend1 = addend_mode == 2 ? addend + n : addend;
  if (staged_ok((uint64_t)k)) {  // a team of at most 31 warps plus the producer
    // 288 threads with at most 112 registers each: two kernels' CTAs fit on an SM
    if (k <= 8192 && staged_fits<FMT, MR, 288>(n, k, sms))
      return launch_staged<FMT, MR, 288, 2>(w, n, k, x, out, addend, addend_mode, err, sms, stream);
    if (k > 8192 && staged_fits<FMT, 1, 1024>(n, k, sms)) {
      // 1024-thread CTAs have 64 registers per thread: one activation row per launch
      if (MR == 1)
        return launch_staged<FMT, 1, 1024, 1>(w, n, k, x, out, addend, addend_mode, err, sms, stream);
      cudaError_t e = launch_staged<FMT, 1, 1024, 1>(w, n, k, x, out, addend, addend_mode, err,
                                                     sms, stream);
      if (e == cudaSuccess)
        e = launch_staged<FMT, 1, 1024, 1>(w, n, k, x + k, without_input_wait(rows_from(out, 1)),
                                           addend1, addend_mode, err, sms, stream);
      return e;
    }
  }
  if (k <= 256 * 32)
    return launch_simple<FMT, MR, 4, 256>(w, n, k, x, out, addend, addend_mode, err, sms, stream);
  if (MR == 1)
    return launch_simple<FMT, 1, 2, 1024>(w, n, k, x, out, addend, addend_mode, err, sms, stream);
  cudaError_t e = launch_simple<FMT, 1, 2, 1024>(w, n, k, x, out, addend, addend_mode, err, sms,
                                                 stream);
  if (e == cudaSuccess)
    e = launch_simple<FMT, 1, 2, 1024>(w, n, k, x + k, without_input_wait(rows_from(out, 1)),
                                       addend1, addend_mode, err, sms, stream);
  return e;
}

cudaError_t launch_gemv(int fmt, const void *w, uint64_t n, uint64_t k, const float *x,
                        uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                        int *err, int sms, cudaStream_t stream) {
  // m <= 2 per launch; larger m is split into row pairs by the caller.
  const int N = (int)n, K = (int)k;
#define MGB_GEMV_CASE(F)                                                                      \
  case F:                                                                                     \
    return m == 1 ? launch_fmt<F, 1>(w, N, K, x, out, addend, addend_mode, err, sms, stream)  \
                  : launch_fmt<F, 2>(w, N, K, x, out, addend, addend_mode, err, sms, stream);
  switch (fmt) {
    MGB_GEMV_CASE(Q4_K)
    MGB_GEMV_CASE(Q6_K)
    MGB_GEMV_CASE(Q5_K)
    MGB_GEMV_CASE(Q8_0)
    MGB_GEMV_CASE(IQ4_NL)
    MGB_GEMV_CASE(Q4_0)
    default:
      return cudaErrorInvalidValue;
  }
#undef MGB_GEMV_CASE
}

}  // namespace mgb
