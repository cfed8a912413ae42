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
  uint32_t hi[8], lo[8];
};

__device__ __forceinline__ void pack_run(const float (&v)[32], bool pair_order, XRun &r) {
  float amax = 0.f, s = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i += 4) s += (v[i] + v[i + 1]) + (v[i + 2] + v[i + 3]);
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  r.sum = s;
  r.dx = amax / 32767.f;
  const float inv = amax > 0.f ? 32767.f / amax : 0.f;
#pragma unroll
  for (int wd = 0; wd < 8; ++wd) {
    uint32_t h = 0, l = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      // pair order: word 2w -> values 8w + 2b, word 2w + 1 -> values 8w + 2b + 1
      const int e = pair_order ? 8 * (wd / 2) + 2 * b + (wd & 1) : 4 * wd + b;
      int q = __float2int_rn(v[e] * inv);
      q = max(-32767, min(32767, q));
      h |= (uint32_t)((q >> 8) & 0xff) << (8 * b);
      l |= (uint32_t)(q & 0xff) << (8 * b);
    }
    r.hi[wd] = h;
    r.lo[wd] = l;
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
  if (FMT == Q4_K) {
    const float d = f16_bits_to_f32(hd.x), dmin = f16_bits_to_f32(hd.x >> 16);
    uint32_t sc, mn;
    q4k_scale_min(j, hd.y, hd.z, hd.w, sc, mn);
    const float s = d * (float)sc, mv = dmin * (float)mn;
#pragma unroll
    for (int m = 0; m < MR; ++m)
      part[m] = (s * x[m].dx) * (float)dot_nib(qa, x[m]) - mv * x[m].sum;
  } else if (FMT == Q4_0) {
    const float d = f16_bits_to_f32(dh);
#pragma unroll
    for (int m = 0; m < MR; ++m)
      part[m] = d * (x[m].dx * (float)dot_nib(qa, x[m]) - 8.f * x[m].sum);
  } else if (FMT == Q8_0) {
    const float d = f16_bits_to_f32(dh);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int m = 0; m < MR; ++m) part[m] = (d * x[m].dx) * (float)dot_s8(q, x[m]);
  } else {  // IQ4_NL
    const float d = f16_bits_to_f32(dh);
    uint32_t q[8];
    const uint32_t words[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) iq4_lookup(words[wd], lut, q[2 * wd], q[2 * wd + 1]);
#pragma unroll
    for (int m = 0; m < MR; ++m) part[m] = (d * x[m].dx) * (float)dot_s8(q, x[m]);
  }
}

template <int FMT, int MR>
__device__ __forceinline__ void load_x(const float *__restrict__ x, int k, int u, bool active,
                                       XRun (&xr)[MR]) {
  constexpr bool pair = FMT == Q4_K || FMT == Q4_0;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (active) f = __ldg(reinterpret_cast<const float4 *>(x + (size_t)m * k + (size_t)u * 32) + i);
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
    pack_run(v, pair, xr[m]);
  }
}

// ---- activation packing, once per CTA into shared memory ------------------------------
// Layout for m rows of runs = k/32: hi words [m][8][runs], lo words [m][8][runs],
// dx [m][runs], sum [m][runs] (72 bytes per run; consecutive runs are
// consecutive words, so a team's reads are conflict-free).

__host__ __device__ inline uint64_t xpack_bytes(uint64_t m, uint64_t k) {
  return m * (k / RUN) * 72;
}

// The consumer threads (ct of nthreads, a multiple of 32) pack the m rows of x:
// four lanes per run, each packing 8 of its values into 2 high and 2 low words
// (words 2p, 2p+1 hold values 8p..8p+7 in either order); the run's max |x|
// and sum come from a 4-lane shuffle.
template <bool PAIR>
__device__ __forceinline__ void pack_x_to_smem(const float *__restrict__ x, int m, int k, int ct,
                                               int nthreads, uint32_t *xs) {
  const int runs = k / RUN;
  const int total = m * runs * 4;
  uint32_t *hi = xs, *lo = xs + (size_t)m * 8 * runs;
  float *dx = reinterpret_cast<float *>(xs + (size_t)m * 16 * runs), *sum = dx + (size_t)m * runs;
  for (int base = 0; base < total; base += nthreads) {
    const int t = base + ct;
    const int p = t & 3, ru = t >> 2;
    const bool live = t < total;  // whole 4-lane groups are live or not
    const int row = live ? ru / runs : 0, u = live ? ru % runs : 0;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
      const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)row * k + (size_t)u * 32 + 8 * p);
      const float4 a = __ldg(src), b = __ldg(src + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    float amax = 0.f, s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      s += __shfl_xor_sync(0xffffffffu, s, off);
    }
    if (!live) continue;
    const float inv = amax > 0.f ? 32767.f / amax : 0.f;
    uint32_t h[2] = {0, 0}, l[2] = {0, 0};
#pragma unroll
    for (int wd = 0; wd < 2; ++wd)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int e = PAIR ? 2 * b + wd : 4 * wd + b;
        int q = __float2int_rn(v[e] * inv);
        q = max(-32767, min(32767, q));
        h[wd] |= (uint32_t)((q >> 8) & 0xff) << (8 * b);
        l[wd] |= (uint32_t)(q & 0xff) << (8 * b);
      }
#pragma unroll
    for (int wd = 0; wd < 2; ++wd) {
      hi[((size_t)row * 8 + 2 * p + wd) * runs + u] = h[wd];
      lo[((size_t)row * 8 + 2 * p + wd) * runs + u] = l[wd];
    }
    if (p == 0) {
      dx[(size_t)row * runs + u] = amax / 32767.f;
      sum[(size_t)row * runs + u] = s;
    }
  }
}

template <int MR>
__device__ __forceinline__ void load_packed_x(const uint32_t *xs, int k, int u, bool active,
                                              XRun (&xr)[MR]) {
  const int runs = k / RUN;
  const uint32_t *hi = xs, *lo = xs + (size_t)MR * 8 * runs;
  const float *dx = reinterpret_cast<const float *>(xs + (size_t)MR * 16 * runs);
  const float *sum = dx + (size_t)MR * runs;
  const int uu = active ? u : 0;
#pragma unroll
  for (int m = 0; m < MR; ++m) {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      xr[m].hi[w] = active ? hi[((size_t)m * 8 + w) * runs + uu] : 0u;
      xr[m].lo[w] = active ? lo[((size_t)m * 8 + w) * runs + uu] : 0u;
    }
    xr[m].dx = active ? dx[(size_t)m * runs + uu] : 0.f;
    xr[m].sum = active ? sum[(size_t)m * runs + uu] : 0.f;
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

constexpr int RPT = 4;  // rows per team per stage

struct GemvStaged {
  int n, k;
  int teams, team_warps;  // consumer geometry
  int stages;
  int chunk;              // stages per reduction pass
  int rows_per_cta;
  uint32_t stage_bytes, qs_stage_bytes;
  int addend_mode;
  const float *addend;
  float *y;
  int *err;
};

template <int FMT, int MR, int MAXT>
__global__ void __launch_bounds__(MAXT, 1)
    gemv_staged_kernel(const uint8_t *__restrict__ w, const float *__restrict__ x,
                       const GemvStaged p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Layout L(FMT, (uint64_t)p.n, (uint64_t)p.k);
  const int S = p.stages;
  const int TR = p.teams * RPT;  // rows per stage
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * p.stage_bytes);
  uint64_t *empty = full + S;
  uint32_t *xs = reinterpret_cast<uint32_t *>(empty + S);  // packed activations (xpack_bytes)
  float *red = reinterpret_cast<float *>(xs + xpack_bytes(MR, p.k) / 4);  // [teams][chunk][RPT][team_warps][MR]
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
        if (g >= S && !mbar_wait(&empty[s], ((g / S) - 1) & 1, p.err)) break;
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
        mbar_wait(&full[g % S], (g / S) & 1, nullptr);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  const int team = cw / p.team_warps, tw = cw % p.team_warps;
  const int u = tw * 32 + lane;  // this thread's run of K
  const int runs = p.k / RUN;
  const bool active = u < runs;
  const int team_threads = p.team_warps * 32;
  float *red_team = red + (size_t)team * p.chunk * RPT * p.team_warps * MR;

  // x may be the previous kernel's output; the weight stream above never waits
  grid_dependency_wait();
  constexpr bool pair = FMT == Q4_K || FMT == Q4_0;
  pack_x_to_smem<pair>(x, MR, p.k, threadIdx.x - 32, consumer_warps * 32, xs);
  named_barrier(15, consumer_warps * 32);
  XRun xr[MR];
  load_packed_x<MR>(xs, p.k, u, active, xr);
  uint32_t lut[4] = {0, 0, 0, 0};
  if (FMT == IQ4_NL) iq4_table(lut);
  const int uu = active ? u : 0;  // idle lanes read a valid run; their result is dropped

  // A wait that gives up records the error and the thread stops waiting, but
  // it keeps stepping through every stage so its team's named barriers match.
  bool ok = true;
  for (int g = 0; g < nstages; ++g) {
    const int s = g % S;
    // lane 0 polls; once the phase is complete every lane's own try_wait
    // succeeds at once and acquires the bulk-copied bytes for that lane
    if (lane == 0) ok = ok && mbar_wait(&full[s], (g / S) & 1, p.err);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) ok = mbar_try_wait(&full[s], (g / S) & 1);
    const uint8_t *st = smem + (size_t)s * p.stage_bytes;
    const int row0 = r0 + g * TR;
    // branch-free over the team's RPT rows (rows past the end of a partial
    // stage read stale stage bytes and are dropped), so their loads and
    // integer dot products interleave
    float part[RPT * MR];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int lr = team * RPT + i;  // row within the stage
      const uint8_t *qrow = st + (size_t)lr * L.qs_row;
      const uint8_t *srow = st + p.qs_stage_bytes + (size_t)lr * L.sc_row;
      uint4 qa, qb = make_uint4(0, 0, 0, 0), hd = make_uint4(0, 0, 0, 0);
      uint32_t dh = 0;
      if (FMT == Q8_0) {
        qa = *reinterpret_cast<const uint4 *>(qrow + uu * 32);
        qb = *reinterpret_cast<const uint4 *>(qrow + uu * 32 + 16);
      } else {
        qa = *reinterpret_cast<const uint4 *>(qrow + uu * 16);
      }
      if (FMT == Q4_K) hd = *reinterpret_cast<const uint4 *>(srow + (uu >> 3) * 16);
      else dh = *reinterpret_cast<const uint16_t *>(srow + uu * 2);
      float pm[MR];
      run_partials<FMT, MR>(qa, qb, hd, dh, uu & 7, xr, lut, pm);
      const bool keep = ok && active && row0 + lr < r1;
#pragma unroll
      for (int m = 0; m < MR; ++m) part[i * MR + m] = keep ? pm[m] : 0.f;
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
          if (p.addend_mode == 1) sum = sum + p.addend[row];
          else if (p.addend_mode == 2) sum = sum + p.addend[(size_t)m * p.n + row];
          p.y[(size_t)m * p.n + row] = sum;
        }
      }
      named_barrier(1 + team, team_threads);
    }
  }
}

// ---- fallback kernel for k % 256 != 0 (ragged scale planes): direct loads -------------

template <int FMT, int MR, int R, int MAXT>
__global__ void __launch_bounds__(MAXT, 1)
    gemv_simple_kernel(const uint8_t *__restrict__ w, int n, int k, const float *__restrict__ x,
                       float *__restrict__ y, const float *__restrict__ addend, int addend_mode,
                       int rows_per_cta) {
  __shared__ float red[2][32][R * MR];
  const Layout L(FMT, (uint64_t)n, (uint64_t)k);
  const int runs = k / RUN;
  const int u = threadIdx.x;
  const bool active = u < runs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  XRun xr[MR];
  load_x<FMT, MR>(x, k, u, active, xr);
  uint32_t lut[4] = {0, 0, 0, 0};
  if (FMT == IQ4_NL) iq4_table(lut);
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(n, r0 + rows_per_cta);
  const uint8_t *scale_plane = w + L.qs_bytes;
  int buf = 0;
  for (int r = r0; r < r1; r += R) {
    float part[R * MR];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int row = r + i;
#pragma unroll
      for (int m = 0; m < MR; ++m) part[i * MR + m] = 0.f;
      if (active && row < r1) {
        const uint8_t *qrow = w + (size_t)row * L.qs_row;
        const uint8_t *srow = scale_plane + (size_t)row * L.sc_row;
        uint4 qa, qb = make_uint4(0, 0, 0, 0), hd = make_uint4(0, 0, 0, 0);
        uint32_t dh = 0;
        if (FMT == Q8_0) {
          qa = ld_stream_v4(qrow + (size_t)u * 32);
          qb = ld_stream_v4(qrow + (size_t)u * 32 + 16);
        } else {
          qa = ld_stream_v4(qrow + (size_t)u * 16);
        }
        if (FMT == Q4_K) hd = __ldg(reinterpret_cast<const uint4 *>(srow + (size_t)(u >> 3) * 16));
        else dh = ld_nc_u16(srow + (size_t)u * 2);
        float pm[MR];
        run_partials<FMT, MR>(qa, qb, hd, dh, u & 7, xr, lut, pm);
#pragma unroll
        for (int m = 0; m < MR; ++m) part[i * MR + m] = pm[m];
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
        y[(size_t)m * n + row] = s;
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
template <int FMT, int MR, int MAXT>
static cudaError_t launch_staged(const void *w, int n, int k, const float *x, float *y,
                                 const float *addend, int addend_mode, int *err, int sms,
                                 cudaStream_t stream) {
  const Layout L(FMT, (uint64_t)n, (uint64_t)k);
  const int runs = k / RUN;
  GemvStaged p;
  p.n = n;
  p.k = k;
  p.team_warps = (runs + 31) / 32;
  p.teams = p.team_warps >= 8 ? 1 : 8 / p.team_warps;
  const int TR = p.teams * RPT;
  p.qs_stage_bytes = (uint32_t)ceil_div((uint64_t)TR * L.qs_row, 128) * 128;
  p.stage_bytes = p.qs_stage_bytes + (uint32_t)ceil_div((uint64_t)TR * L.sc_row, 128) * 128;
  // Two CTAs per SM when they fit (more consumer warps to hide latency), each
  // within ~110 KB of shared memory.  Rows split evenly; a CTA's last stage
  // may hold fewer than TR rows.
  const uint64_t fixed = xpack_bytes(MR, (uint64_t)k) + 2048;
  const uint64_t budget = 110 * 1024 > fixed ? 110 * 1024 - fixed : 0;
  int stages = (int)(budget / p.stage_bytes);
  if (stages > 8) stages = 8;
  if (stages < 2) stages = 2;
  p.stages = stages;
  const int threads = 32 * (1 + p.teams * p.team_warps);
  const int per_sm = threads <= 512 ? 2 : 1;
  const int units = (int)ceil_div((uint64_t)n, (uint64_t)TR);
  int grid = sms * per_sm;
  if (grid > units) grid = units;
  p.rows_per_cta = (int)ceil_div((uint64_t)n, (uint64_t)grid);
  grid = (int)ceil_div((uint64_t)n, (uint64_t)p.rows_per_cta);
  // reduction buffer: as many stages as fit in 16 KB (usually all of a CTA's)
  const int nst = (int)ceil_div((uint64_t)p.rows_per_cta, (uint64_t)TR);
  const size_t red_stage = sizeof(float) * (size_t)p.teams * RPT * p.team_warps * MR;
  int chunk = (int)(16384 / red_stage);
  if (chunk > nst) chunk = nst;
  if (chunk < 1) chunk = 1;
  p.chunk = chunk;
  p.addend_mode = addend_mode;
  p.addend = addend;
  p.y = y;
  p.err = err;
  const size_t smem = (size_t)stages * p.stage_bytes + 2 * 8 * (size_t)stages +
                      xpack_bytes(MR, (uint64_t)k) + red_stage * chunk;
  auto kern = gemv_staged_kernel<FMT, MR, MAXT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_dependent(kern, dim3((unsigned)grid), dim3((unsigned)threads), smem, stream,
                          static_cast<const uint8_t *>(w), x, p);
}

template <int FMT, int MR, int R, int MAXT>
static cudaError_t launch_simple(const void *w, int n, int k, const float *x, float *y,
                                 const float *addend, int addend_mode, int sms,
                                 cudaStream_t stream) {
  const int runs = k / RUN;
  const int threads = ((runs + 31) / 32) * 32;
  int per_sm = 2048 / threads;
  if (per_sm < 1) per_sm = 1;
  if (per_sm > 8) per_sm = 8;
  const int target = sms * per_sm;
  int rows = (int)ceil_div((uint64_t)n, (uint64_t)target);
  if (rows < 1) rows = 1;
  const int grid = (int)ceil_div((uint64_t)n, (uint64_t)rows);
  gemv_simple_kernel<FMT, MR, R, MAXT><<<grid, threads, 0, stream>>>(
      static_cast<const uint8_t *>(w), n, k, x, y, addend, addend_mode, rows);
  return cudaGetLastError();
}

static bool staged_ok(uint64_t k) { return k % 256 == 0 && k / RUN <= 31 * 32; }

template <int FMT, int MR>
static cudaError_t launch_fmt(const void *w, int n, int k, const float *x, float *y,
                              const float *addend, int addend_mode, int *err, int sms,
                              cudaStream_t stream) {
  if (staged_ok((uint64_t)k)) {  // a team of at most 31 warps plus the producer
    if (k <= 8192)
      return launch_staged<FMT, MR, 288>(w, n, k, x, y, addend, addend_mode, err, sms, stream);
    // 1024-thread CTAs have 64 registers per thread: one activation row per launch
    cudaError_t e = launch_staged<FMT, 1, 1024>(w, n, k, x, y, addend, addend_mode, err, sms, stream);
    if (MR == 2 && e == cudaSuccess)
      e = launch_staged<FMT, 1, 1024>(w, n, k, x + k, y + n, addend_mode == 2 ? addend + n : addend,
                                      addend_mode, err, sms, stream);
    return e;
  }
  if (k <= 256 * 32) return launch_simple<FMT, MR, 4, 256>(w, n, k, x, y, addend, addend_mode, sms, stream);
  cudaError_t e = launch_simple<FMT, 1, 2, 1024>(w, n, k, x, y, addend, addend_mode, sms, stream);
  if (MR == 2 && e == cudaSuccess)
    e = launch_simple<FMT, 1, 2, 1024>(w, n, k, x + k, y + n,
                                       addend_mode == 2 ? addend + n : addend, addend_mode, sms,
                                       stream);
  return e;
}

cudaError_t launch_gemv(int fmt, const void *w, uint64_t n, uint64_t k, const float *x,
                        uint64_t m, float *y, const float *addend, int addend_mode, int *err,
                        int sms, cudaStream_t stream) {
  // m <= 2 per launch; larger m is split into row pairs by the caller.
  const int N = (int)n, K = (int)k;
#define MGB_GEMV_CASE(F)                                                                      \
  case F:                                                                                     \
    return m == 1 ? launch_fmt<F, 1>(w, N, K, x, y, addend, addend_mode, err, sms, stream)    \
                  : launch_fmt<F, 2>(w, N, K, x, y, addend, addend_mode, err, sms, stream);
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
