// Prefill GEMM for packed weights on sm_100a (tcgen05 + TMEM + TMA):
// y[m, n] = x[m, k] * W^T, W in the device layout (quant plane + scale plane),
// bf16 operands, f32 accumulation in tensor memory.  Replaces the reference's
// packed matmul for many activation rows (`packed_matmul`,
// src/native/mod.rs:109-152 -> `columns_q4k_avx2`, src/native/quant.rs:673-744).
//
// CTA tile: BM activation rows (1 or 2 accumulators of 128 rows) x BN weight
// rows (the MMA N, <= 256, a multiple of 16), K in steps of 64 (one 128-byte
// swizzle atom of bf16).  Two shared-memory rings: operand stages (the
// activation tile and the bf16 W tile of a K step, 3 to 6 deep), each with one
// `full` barrier (the activation TMA bytes + one arrival per dequantising
// warp of the step) and one `empty` barrier (the MMAs' commit), so the MMA
// issuer waits and commits once per step; and packed-W stages (quant and scale
// boxes from HBM, 3+ deep, released by the dequantising warps).  Launched as a
// programmatic dependent: everything but the activation loads (TMEM, barriers,
// the weight stream, dequantisation) overlaps the previous kernel on the
// stream.  Warp roles, 96 + 32 * DQW threads (DQW = 16 dequantising warps;
// 128-row tiles up to 128 columns wide hold two 64-value K atoms per stage):
//   warp 0     TMA producer of the bf16 activation boxes (SWIZZLE_128B,
//              straight into the UMMA operand layout) on full[s], after
//              griddepcontrol.wait.  Owns the TMEM allocation.
//   warp 1     one thread issues tcgen05.mma (kind::f16, bf16 x bf16 -> f32)
//              per 16-wide K slice and commits each step to empty[s].
//   warp 2     TMA producer of the packed W quant and scale boxes (no
//              swizzle) on p_full[s].
//   warps 3.. dequantise the staged packed W into the bf16 B operand
//              (K-major, SWIZZLE_128B written by hand), fence the async proxy
//              and arrive on full[s] and p_empty[s] (on narrow tiles as 2 or 4
//              groups that take K steps in turn); after the last stage they
//              drain TMEM with tcgen05.ld and write y (+ the addend): for one
//              output of wide tiles, 32 x 32 blocks staged SWIZZLE_128B in
//              shared memory and written by TMA stores; otherwise straight from
//              registers, or, when every rank's y receives the tile (fused
//              all-gather over NVLink), through shared memory in whole row
//              segments.
// A call with narrow tiles (choose_split) may split K over 2, 4 or 8 CTAs per
// tile (blockIdx.z), each writing an f32 partial plane that mgb_splitk_sum_kernel
// adds.
// Every CTA loads its own tiles from this GPU's HBM (no cluster-shared loads).
// Every wait is bounded; on expiry the kernel records ERR_WAIT_TIMEOUT, skips
// the remaining work, waits (bounded) for its own copies and MMAs, frees TMEM
// and returns.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace mgb {

namespace {

constexpr int KSTEP = 64;                    // bf16 values per 128-byte row of a stage
// warps 3 .. 3 + DQW - 1 dequantise, then run the epilogue: 16 warps, as many
// as the registers allow (608 threads x <= 104 registers); against 8 they took
// config 1's 256-row tiles from 70.2 to 58.4 us and a 128-row M = 16 tile from
// 37.4 to 35.8 us
constexpr int dq_warps_for(int) { return 16; }
constexpr int EPI_SQUARE_BYTES = 4352;  // a warp's 32 x 33 f32 square, rounded up
constexpr int EPI_TMA_BYTES = 8192;     // a warp's two 4 KB TMA-store buffers

struct GemmParams {
  int m, n, k;
  int bn;               // weight rows per CTA (MMA N)
  int astages;          // activation-tile ring
  int bstages;          // bf16 W-tile ring
  int pstages;          // packed-W ring
  int qbytes;           // packed quant bytes per weight row per K step (32, 48 or 64)
  int wsw;              // scale-plane bytes per weight row per 256 values (16, 32 or 48)
  int dq_groups;        // dequant warp groups taking K steps in turn (1, 2 or 4)
  int ksplit;           // K parts computed by separate CTAs (blockIdx.z), summed after
  int atoms;            // 64-value K atoms per pipeline stage (the kernel's AT)
  uint32_t b_atom;      // bytes of one atom's bf16 W tile
  uint32_t a_bytes;     // per activation stage
  uint32_t b_bytes;     // per W-tile stage
  uint32_t wq_bytes;    // per packed stage
  uint32_t ws_bytes;
  uint32_t pstage_bytes;
  uint32_t ptx_bytes;   // bytes the two packed boxes of one step deliver
  int addend_mode;
  const float *addend;
  OutSpec out;          // y of this rank, or of every rank (fused all-gather)
  int vec_out;          // every output row start is 16-byte aligned: float4 stores
  int tma_out;          // one output, no addend, 16-byte rows: TMA stores of 32x32 blocks
  int *err;
};

// ---- tcgen05 / TMA PTX ---------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major, SWIZZLE_128B: 8-row groups 1024 bytes apart (SBO), LBO unused (1),
  // version 1 (sm_100), layout type 2.
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ uint32_t instr_desc_bf16(int m, int n) {
  // D f32 (bits 4-5 = 1), A bf16 (7-9 = 1), B bf16 (10-12 = 1), both K-major,
  // N >> 3 at bits 17-22, M >> 4 at bits 24-28.
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float v[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 8 columns summed over `accs` accumulators `stride` columns apart.
__device__ __forceinline__ void tmem_ld8_sum(uint32_t taddr, int accs, uint32_t stride, float v[8]) {
  tmem_ld8(taddr, v);
  if (accs == 2) {
    float w[8];
    tmem_ld8(taddr + stride, w);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] + w[i];
  }
}

// 32 consecutive columns of this warp's 32 TMEM lanes: lane i gets row i.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float v[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32_sum(uint32_t taddr, int accs, uint32_t stride,
                                              float v[32]) {
  tmem_ld32(taddr, v);
  if (accs == 2) {
    float w[32];
    tmem_ld32(taddr + stride, w);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = v[i] + w[i];
  }
}

// ---- TMA stores (shared -> this GPU's global memory) -----------------------------------

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, const void *src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory source of all but the newest `n` committed groups has been read
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- dequantisation of one 32-value run into 64 bytes of bf16 ----------------------

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// 4-bit nibble pairs (byte i = values 2i, 2i+1) with value = s * q - mn,
// written as 4 uint4 (8 bf16 each) into out[].  f = 0.5 + q/256 (one prmt
// per value) and s*q - mn = f * 256 s - (128 s + mn): one packed f32x2 FMA
// per value pair, one cvt.rn.bf16x2 per pair.
__device__ __forceinline__ void dq_nib_linear(const uint4 &qs, float s, float mn, uint4 out[4]) {
  const float a = 256.f * s, c = -(128.f * s + mn);
  const float2 a2 = make_float2(a, a), c2 = make_float2(c, c);
  const uint32_t words[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    const uint32_t lo = words[wd] & 0x0F0F0F0Fu, hi = (words[wd] >> 4) & 0x0F0F0F0Fu;
    uint32_t p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float f0 = __uint_as_float(__byte_perm(lo, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
      const float f1 = __uint_as_float(__byte_perm(hi, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
      const float2 v = __ffma2_rn(make_float2(f0, f1), a2, c2);
      p[i] = pack_bf16(v.x, v.y);
    }
    out[wd] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

// Q6_K: 6-bit codes c (nibble pairs plus the high 2-bit fields of the two
// halves, hw[0] and hw[1]) with value = s_h * (c - 32), s_h the scale of the
// value's 16-value half: the nibble formula with the code in the mantissa.
__device__ __forceinline__ void dq_q6k(const uint4 &qs, const uint2 &hw, float s0, float s1,
                                       uint4 out[4]) {
  const uint32_t words[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    const float s = wd < 2 ? s0 : s1;
    const float a = 256.f * s, c = -(128.f * s + 32.f * s);
    const float2 a2 = make_float2(a, a), c2 = make_float2(c, c);
    uint32_t ev, od;
    q6k_codes(words[wd], wd < 2 ? hw.x : hw.y, wd, ev, od);
    uint32_t p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float f0 = __uint_as_float(__byte_perm(ev, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
      const float f1 = __uint_as_float(__byte_perm(od, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
      const float2 v = __ffma2_rn(make_float2(f0, f1), a2, c2);
      p[i] = pack_bf16(v.x, v.y);
    }
    out[wd] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

// Q5_K: nibble pairs plus the run's fifth-bit word; value = s * c - mn with
// the 5-bit code c, by the nibble formula with the code in the mantissa.
__device__ __forceinline__ void dq_q5k(const uint4 &qs, uint32_t hb, float s, float mn,
                                       uint4 out[4]) {
  const float a = 256.f * s, c = -(128.f * s + mn);
  const float2 a2 = make_float2(a, a), c2 = make_float2(c, c);
  const uint32_t words[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
  for (int wd = 0; wd < 4; ++wd) {
    uint32_t ev, od;
    q5k_codes(words[wd], hb, wd, ev, od);
    uint32_t p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float f0 = __uint_as_float(__byte_perm(ev, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
      const float f1 = __uint_as_float(__byte_perm(od, 0x3F000000u, 0x7054u | ((uint32_t)i << 8)));
      const float2 v = __ffma2_rn(make_float2(f0, f1), a2, c2);
      p[i] = pack_bf16(v.x, v.y);
    }
    out[wd] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

// Biased bytes (b + 128, byte order = value order) times d.
__device__ __forceinline__ void dq_bytes(const uint32_t u[8], float d, uint4 out[4]) {
#pragma unroll
  for (int wd = 0; wd < 8; wd += 2) {
    uint32_t p[4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        const float f0 = __uint_as_float(__byte_perm(u[wd + h], 0x4B000000u, 0x7650u | (uint32_t)i)) - 8388736.0f;
        const float f1 = __uint_as_float(__byte_perm(u[wd + h], 0x4B000000u, 0x7650u | (uint32_t)(i + 1))) - 8388736.0f;
        p[2 * h + i / 2] = pack_bf16(f0 * d, f1 * d);
      }
    out[wd / 2] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

__device__ __forceinline__ void iq4_lookup2(uint32_t v, const uint32_t t[4], uint32_t &o0,
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

template <int FMT>
__device__ __forceinline__ void dequant_run(const uint8_t *wq_row, const uint8_t *ws_row, int kt,
                                            int j, const uint32_t lut[4], uint4 out[4]) {
  const int sub = (kt & 3) * 2 + j;  // run index within the 8 runs the scale box covers
  if (FMT == Q6_K) {
    // this K step's 48 bytes: the two runs' nibble pairs, then their high words
    const uint4 qs = *reinterpret_cast<const uint4 *>(wq_row + j * 16);
    const uint2 hw = *reinterpret_cast<const uint2 *>(wq_row + 32 + j * 8);
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(ws_row + 16));
    const uint16_t sp = *reinterpret_cast<const uint16_t *>(ws_row + 2 * sub);
    dq_q6k(qs, hw, d * (float)(int8_t)(sp & 0xFF), d * (float)(int8_t)(sp >> 8), out);
  } else if (FMT == Q4_K || FMT == Q5_K) {
    const uint4 qs = *reinterpret_cast<const uint4 *>(wq_row + j * 16);
    const uint4 h = *reinterpret_cast<const uint4 *>(ws_row);
    const float d = f16_bits_to_f32(h.x), dmin = f16_bits_to_f32(h.x >> 16);
    uint32_t sc, mn;
    q4k_scale_min(sub, h.y, h.z, h.w, sc, mn);
    if (FMT == Q5_K)
      dq_q5k(qs, *reinterpret_cast<const uint32_t *>(ws_row + 16 + 4 * sub), d * (float)sc,
             dmin * (float)mn, out);
    else
      dq_nib_linear(qs, d * (float)sc, dmin * (float)mn, out);
  } else if (FMT == Q4_0) {
    const uint4 qs = *reinterpret_cast<const uint4 *>(wq_row + j * 16);
    const uint32_t hb = *reinterpret_cast<const uint16_t *>(ws_row + 2 * sub);
    const float d = f16_bits_to_f32(hb);
    dq_nib_linear(qs, d, 8.f * d, out);
  } else if (FMT == Q8_0) {
    const uint4 a = *reinterpret_cast<const uint4 *>(wq_row + j * 32);
    const uint4 b = *reinterpret_cast<const uint4 *>(wq_row + j * 32 + 16);
    const uint32_t hb = *reinterpret_cast<const uint16_t *>(ws_row + 2 * sub);
    const uint32_t u[8] = {a.x ^ 0x80808080u, a.y ^ 0x80808080u, a.z ^ 0x80808080u,
                           a.w ^ 0x80808080u, b.x ^ 0x80808080u, b.y ^ 0x80808080u,
                           b.z ^ 0x80808080u, b.w ^ 0x80808080u};
    dq_bytes(u, f16_bits_to_f32(hb), out);
  } else {  // IQ4_NL
    const uint4 qs = *reinterpret_cast<const uint4 *>(wq_row + j * 16);
    const uint32_t hb = *reinterpret_cast<const uint16_t *>(ws_row + 2 * sub);
    uint32_t u[8];
    const uint32_t words[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) iq4_lookup2(words[wd], lut, u[2 * wd], u[2 * wd + 1]);
    dq_bytes(u, f16_bits_to_f32(hb), out);
  }
}

// ---- the kernel ----------------------------------------------------------------------

// ---- epilogue ------------------------------------------------------------------------

// Drains this warp's 32 TMEM lanes (lane quarter `quarter`) of `nsub`
// accumulator blocks into y; with accs == 2 each block is the sum of two
// accumulators 256 columns apart (even and odd K slices).  Block b holds output rows row0 + 128 b + 32
// quarter + lane at TMEM columns b * sub_stride + c for tile columns c <
// tile_cols (output columns n0 + c); `half` (0 .. parts-1) picks this warp's
// share of the column chunks, taken in turn by the `parts` warps of a quarter
// column chunks (two warps per quarter).  One output rank: each lane stores
// its row's 8-column pieces directly (the L2 merges the warp's row segments).
// Several ranks: 32-column chunks go through a padded 32 x 33 square of
// shared memory (`square`, this warp's own) so that the warp's stores cover
// whole 128-byte row segments: full-size writes over NVLink.
__device__ __forceinline__ void drain_accumulators(const GemmParams &p, const CUtensorMap *map_y,
                                                   uint32_t tmem_base,
                                                   int nsub, int sub_stride, int row0, int n0,
                                                   int tile_cols, int quarter, int half, int parts,
                                                   int accs, int lane,
                                                   float *square) {
  const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
  if (p.tma_out) {
    // 32 x 32 blocks: lane = row; written SWIZZLE_128B into one of this warp's
    // two 4 KB buffers (16-byte chunk q of row r at r * 128 + ((q ^ (r & 7)) << 4))
    // and stored by one TMA copy (rows past m, columns past n are clipped); a
    // partial last block of the tile (tile_cols % 32) is stored directly
    uint8_t *buf = reinterpret_cast<uint8_t *>(square);
    int nb = 0;
    for (int sub = 0; sub < nsub; ++sub) {
      const int rb = row0 + sub * 128 + quarter * 32;
      for (int c0 = 32 * half; c0 < tile_cols; c0 += 32 * parts) {
        float v[32];
        tmem_ld32_sum(lane_base + (uint32_t)(sub * sub_stride + c0), accs, 256, v);
        if (c0 + 32 <= tile_cols) {
          uint8_t *b = buf + (nb & 1) * 4096;
          if (lane == 0) bulk_wait_read<1>();  // the buffer's previous store has read it
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4 *>(b + lane * 128 + ((q ^ (lane & 7)) << 4)) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(map_y, n0 + c0, rb, b);
            bulk_commit();
          }
          ++nb;
        } else {
          const int row = rb + lane;
          if (row < p.m) {
            float *yr = p.out.y_ranks[0] + (size_t)row * p.out.ldy;
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (e < tile_cols - c0 && n0 + c0 + e < p.n) yr[n0 + c0 + e] = v[e];
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    return;
  }
  if (p.out.world == 1) {
    // (a split-K CTA writes its partial sums: plane blockIdx.z of [ksplit][m][ldy])
    float *y = p.out.y_ranks[0] + (size_t)blockIdx.z * p.m * p.out.ldy;
    for (int sub = 0; sub < nsub; ++sub) {
      const int row = row0 + sub * 128 + quarter * 32 + lane;
      for (int c = 8 * half; c < tile_cols; c += 8 * parts) {
        float v[8];
        tmem_ld8_sum(lane_base + (uint32_t)(sub * sub_stride + c), accs, 256, v);
        if (row >= p.m) continue;
        const int col = n0 + c;
        float *yr = y + (size_t)row * p.out.ldy + p.out.col0;
        if (col + 8 <= p.n && p.addend_mode == 0 && p.vec_out) {
          reinterpret_cast<float4 *>(yr + col)[0] = make_float4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<float4 *>(yr + col)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (col + e < p.n) {
              float o = v[e];
              if (p.addend_mode == 1) o = o + __ldcg(p.addend + col + e);
              else if (p.addend_mode == 2) o = o + __ldcg(p.addend + (size_t)row * p.n + col + e);
              yr[col + e] = o;
            }
          }
        }
      }
    }
    return;
  }
  const int sub_lane = lane >> 3, c4 = (lane & 7) * 4;  // store lanes: 4 rows x 8 float4
  for (int sub = 0; sub < nsub; ++sub) {
    const int rbase = row0 + sub * 128 + quarter * 32;
    for (int c = 32 * half; c < tile_cols; c += 32 * parts) {
      float v[32];
      tmem_ld32_sum(lane_base + (uint32_t)(sub * sub_stride + c), accs, 256, v);
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) square[lane * 33 + j] = v[j];
      __syncwarp();
      const int col = n0 + c + c4;  // this lane's first column (a multiple of 4)
#pragma unroll 2
      for (int r0 = 0; r0 < 32; r0 += 4) {
        const int rr = r0 + sub_lane;
        const int row = rbase + rr;
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = square[rr * 33 + c4 + e];
        if (row >= p.m || c + c4 >= tile_cols || col >= p.n) continue;
        if (p.addend_mode == 1) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (col + e < p.n) o[e] = o[e] + __ldcg(p.addend + col + e);
        } else if (p.addend_mode == 2) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (col + e < p.n) o[e] = o[e] + __ldcg(p.addend + (size_t)row * p.n + col + e);
        }
        // this call's column col lands at col0 + col of every output rank's y
        const size_t off = (size_t)row * p.out.ldy + p.out.col0 + col;
        if (p.vec_out && col + 4 <= p.n) {
          for (int r = 0; r < p.out.world; ++r)
            *reinterpret_cast<float4 *>(p.out.y_ranks[r] + off) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
          for (int r = 0; r < p.out.world; ++r)
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (col + e < p.n) p.out.y_ranks[r][off + e] = o[e];
        }
      }
    }
  }
}

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// AT: 64-value K atoms per pipeline stage (1 or 2).
template <int FMT, int SUBS, int DQW, int AT>
__global__ void __launch_bounds__(96 + 32 * DQW, 1)
    mgb_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_wq,
                const __grid_constant__ CUtensorMap map_ws, const __grid_constant__ CUtensorMap map_y,
                const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte align the operand area (SWIZZLE_128B atoms).
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.astages, SP = p.pstages;
  uint8_t *a0 = smem;                                    // S activation tiles
  uint8_t *b0 = a0 + (size_t)S * p.a_bytes;              // S bf16 W tiles
  uint8_t *pk0 = b0 + (size_t)S * p.b_bytes;             // SP packed W (quant box, scale box)
  uint64_t *bars = reinterpret_cast<uint64_t *>(pk0 + (size_t)SP * p.pstage_bytes);
  // A stage is its activation tile and its bf16 W tile: one barrier says both
  // are ready (the TMA bytes + one arrival per dequantising warp), one says
  // the MMAs finished reading both.  The MMA issuer waits and commits once per
  // K step: its own instruction stream is what keeps the tensor pipe fed.
  uint64_t *full = bars;
  uint64_t *empty = full + S;
  uint64_t *p_full = empty + S;         // packed W boxes landed (TMA bytes)
  uint64_t *p_empty = p_full + SP;      // every dequant warp finished reading them
  uint64_t *done = p_empty + SP;        // all MMAs finished
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * p.bn;
  const int m0 = blockIdx.y * (128 * SUBS);
  const int KT = p.k / (KSTEP * AT) / p.ksplit;   // this CTA's stages
  const int kt0 = (int)blockIdx.z * KT;                // its first stage
  // 128-row tiles alternate two accumulators over the K slices (columns 0 and
  // 256): consecutive MMAs into one accumulator wait on each other
  constexpr int ACCS = SUBS == 1 ? 2 : 1;
  constexpr uint32_t TMEM_COLS = 512;

  if (threadIdx.x == 0) {
    // each K step is dequantised by one group of DQW / dq_groups warps
    const int gw = DQW / p.dq_groups;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1 + gw);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < SP; ++s) {
      mbar_init(&p_full[s], 1);
      mbar_init(&p_empty[s], gw);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_map(&map_a);
    prefetch_map(&map_wq);
    prefetch_map(&map_ws);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- activation tiles (TMA, SWIZZLE_128B) ----------------
    if (lane == 0) {
      grid_launch_dependents();
      grid_dependency_wait();  // the activations may be the previous kernel's output
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % S;
        if (kt >= S && !mbar_wait(&empty[s], ((kt / S) - 1) & 1, p.err)) {
          *(volatile int *)abort_flag = 1;
          break;
        }
        if (*(volatile int *)abort_flag) break;
        uint8_t *st = a0 + (size_t)s * p.a_bytes;
        mbar_arrive_expect_tx(&full[s], p.a_bytes);
#pragma unroll
        for (int a = 0; a < AT; ++a)
          for (int sub = 0; sub < SUBS; ++sub)
            tma_load_2d(st + (a * SUBS + sub) * 16384, &map_a, ((kt0 + kt) * AT + a) * KSTEP,
                        m0 + sub * 128, &full[s]);
      }
      // (every activation copy has landed before the MMAs that read it, and
      // the epilogue waits for those)
    }
  } else if (warp == 2) {
    // ---------------- packed W boxes, prefetched SP steps ahead ----------------
    // (weights never depend on an earlier kernel: no grid-dependency wait)
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % SP;
        if (kt >= SP && !mbar_wait(&p_empty[s], ((kt / SP) - 1) & 1, p.err)) {
          *(volatile int *)abort_flag = 1;
          break;
        }
        if (*(volatile int *)abort_flag) break;
        uint8_t *st = pk0 + (size_t)s * p.pstage_bytes;
        mbar_arrive_expect_tx(&p_full[s], p.ptx_bytes);
        // (a stage's atoms lie in one 256-value block: one scale box)
        tma_load_2d(st, &map_wq, (kt0 + kt) * p.qbytes * AT, n0, &p_full[s]);
        tma_load_2d(st + p.wq_bytes, &map_ws, ((kt0 + kt) * AT / 4) * p.wsw, n0, &p_full[s]);
        issued = kt + 1;
      }
      for (int kt = (issued > SP ? issued - SP : 0); kt < issued; ++kt)
        mbar_wait(&p_full[kt % SP], (kt / SP) & 1, nullptr);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = instr_desc_bf16(128, p.bn);
      // The descriptors' start address is bits 0..13 (address >> 4) and every
      // shared-memory address is below 256 KB: a stage's descriptors are the
      // first stage's plus the offset >> 4, with no carry out of the field.
      const uint64_t a_desc0 = smem_desc_sw128(smem_u32(a0));
      const uint64_t b_desc0 = smem_desc_sw128(smem_u32(b0));
      int s = 0, round = 0;
      for (int kt = 0; kt < KT; ++kt) {
        if (!mbar_wait(&full[s], round & 1, p.err)) {
          *(volatile int *)abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_desc0 + (((uint64_t)s * p.a_bytes) >> 4);
        const uint64_t bd = b_desc0 + (((uint64_t)s * p.b_bytes) >> 4);
#pragma unroll
        for (int a = 0; a < AT; ++a)
#pragma unroll
          for (int sub = 0; sub < SUBS; ++sub)
#pragma unroll
            for (int kk = 0; kk < KSTEP / 16; ++kk)
              mma_bf16(tmem_base + (ACCS == 2 ? (kk & 1) : sub) * 256,
                       ad + (uint64_t)(((a * SUBS + sub) * 16384 + kk * 32) >> 4),
                       bd + (uint64_t)((a * p.b_atom + kk * 32) >> 4), idesc,
                       (kt | a | (ACCS == 2 ? kk >> 1 : kk)) != 0);
        mma_commit(&empty[s]);
        if (++s == S) {
          s = 0;
          ++round;
        }
      }
      mma_commit(done);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---------------- dequantise W, then the epilogue ----------------
    const int t = threadIdx.x - 96;  // 0 .. 32 * DQW - 1
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
    const int items1 = p.bn * 2;              // (weight row, run) pairs per atom
    const int items = items1 * AT;            // ... per stage
    const int pk_row = p.qbytes * AT;         // a weight row's packed bytes per stage
    // Narrow tiles have little dequantisation per step, and one warp's pass
    // through a step (two barrier waits, the proxy fence, two arrivals) is
    // what bounds them: the warps split into groups that take K steps in
    // turn, so several steps are in flight.
    const int gw = DQW / p.dq_groups;
    const int grp = (warp - 3) / gw;
    const int gt = t - grp * gw * 32;  // thread index within the group
    bool ok = true;
    for (int kt = grp; kt < KT && ok; kt += p.dq_groups) {
      const int sb = kt % S, sp = kt % SP;
      if (*(volatile int *)abort_flag) break;
      // the stage is free once the MMAs of round (kt / S) - 1 released it, and
      // the packed boxes of this step have landed
      ok = (kt < S || mbar_wait(&empty[sb], ((kt / S) - 1) & 1, p.err)) &&
           mbar_wait(&p_full[sp], (kt / SP) & 1, p.err);
      if (!ok) {
        *(volatile int *)abort_flag = 1;
        break;
      }
      uint8_t *bt = b0 + (size_t)sb * p.b_bytes;
      const uint8_t *wq = pk0 + (size_t)sp * p.pstage_bytes;
      const uint8_t *ws = wq + p.wq_bytes;
      for (int it = gt; it < items; it += gw * 32) {
        const int a = AT == 2 && it >= items1 ? 1 : 0;
        const int r = it - a * items1;
        const int row = r >> 1, j = r & 1;
        uint4 out[4];
        dequant_run<FMT>(wq + row * pk_row + a * p.qbytes, ws + row * p.wsw,
                         (kt0 + kt) * AT + a, j, lut, out);
        uint8_t *dst_row = bt + a * p.b_atom + row * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = j * 4 + c;
          *reinterpret_cast<uint4 *>(dst_row + ((chunk ^ (row & 7)) << 4)) = out[c];
        }
      }
      // each thread's writes reach the async proxy; the warp syncs and one
      // lane arrives for it
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&full[sb]);
        mbar_arrive(&p_empty[sp]);
      }
    }
    // epilogue: TMEM lanes of this warp's quarter -> y rows
    const bool finished = mbar_wait(done, 0, p.err);
    tc_fence_after();
    // tcgen05.ld is warp-collective: the whole warp drains TMEM or none of it
    const bool drain = __all_sync(0xffffffffu, finished && !*(volatile int *)abort_flag);
    if (drain)
      drain_accumulators(p, &map_y, tmem_base, SUBS, 256, m0, n0, p.bn, warp & 3, (warp - 3) / 4,
                         DQW / 4, ACCS, lane,
                         reinterpret_cast<float *>(
                             smem + (size_t)(warp - 3) * (p.tma_out ? EPI_TMA_BYTES : EPI_SQUARE_BYTES)));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---- host side ---------------------------------------------------------------------------

// f32 -> bf16 activations; lets the dependent GEMM launch at once (its weight
// stream and dequantisation overlap this pass; its activation loads wait).
// A tensor-parallel call with an input wait (OutSpec::wait_done) waits here,
// warp 0 of every CTA, before any thread of the CTA reads x.
__global__ void mgb_f32_to_bf16_kernel(const float *__restrict__ x, __nv_bfloat16 *__restrict__ out,
                                   uint64_t n, const OutSpec spec, int *err) {
  grid_launch_dependents();
  grid_dependency_wait();
  if (spec.wait_done) {
    if (threadIdx.x < 32) out_wait_input(spec, threadIdx.x, err);
    __syncthreads();
  }
  const uint64_t n4 = n / 4;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
       i += (uint64_t)gridDim.x * blockDim.x) {
    // coherent loads: x may have been written by the kernel this one overlaps
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(x) + i);
    uint2 o;
    o.x = pack_bf16(v.x, v.y);
    o.y = pack_bf16(v.z, v.w);
    reinterpret_cast<uint2 *>(out)[i] = o;
  }
}

// Split-K: y = the partial planes summed in plane order (+ the addend); a
// programmatic dependent of the GEMM that wrote them.
__global__ void mgb_splitk_sum_kernel(const float *__restrict__ part, int planes, uint64_t m,
                                  uint64_t n, const OutSpec out,
                                  const float *__restrict__ addend, int addend_mode) {
  grid_launch_dependents();
  grid_dependency_wait();
  const uint64_t total = m * n;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    // coherent loads: the planes are the overlapped GEMM's output
    float v = __ldcg(part + i);
    for (int z = 1; z < planes; ++z) v = v + __ldcg(part + z * total + i);
    if (addend_mode == 1) v = v + __ldcg(addend + i % n);
    else if (addend_mode == 2) v = v + __ldcg(addend + i);
    out_store(out, (int)(i / n), i % n, v);  // every rank's y for a tensor-parallel call
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_map_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct TileChoice {
  int subs, bn;
};

TileChoice choose_tiles(uint64_t m, uint64_t n, int sms) {
  TileChoice t;
  t.subs = m > 128 ? 2 : 1;
  const uint64_t mt = ceil_div(m, 128 * (uint64_t)t.subs);
  // columns per tile so that mt rows of tiles fit one wave of `sms` CTAs
  const uint64_t per_row = (uint64_t)sms / mt > 0 ? (uint64_t)sms / mt : 1;
  uint64_t bn = ceil_div(n, per_row);
  bn = ceil_div(bn, 16) * 16;
  if (bn < 32) bn = 32;
  if (bn > 256 && mt * ceil_div(n, 256) <= 4 * (uint64_t)sms) {
    // one to four waves even at the widest tile: the width with the least
    // waves x (fixed + width), a tile's time being about 256 columns' worth of
    // fixed per-step cost plus its width (measured at M = 512: 60.5, 52.5, 42.3
    // and 37.2 us for 208, 112, 64 and 32 columns over the same K).  A nearly
    // empty last wave costs a whole tile time here (M = 2,048, K = 8,192, one
    // B200: N 14,336 at 208 columns 542 -> 458 us, N 8,192 at 224 290 -> 282 us,
    // and N 8,192, K 28,672 985 -> 940 us); over more waves the CTAs drift apart
    // and the widest tile stays best (N 28,672: 973 us at 256 against 982 at 224).
    uint64_t best = 256, best_cost = ~0ull;
    for (uint64_t w = 256; w >= 128; w -= 16) {
      const uint64_t waves = ceil_div(mt * ceil_div(n, w), (uint64_t)sms);
      const uint64_t cost = waves * (256 + w);
      if (cost < best_cost) {
        best = w;
        best_cost = cost;
      }
    }
    bn = best;
  }
  if (bn > 256) bn = 256;
  t.bn = (int)bn;
  return t;
}

template <typename K, typename... Args>
cudaError_t launch_dependent(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args... args) {
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

}  // namespace

uint64_t gemm_workspace_bytes(int, uint64_t m, uint64_t, uint64_t k) {
  return ceil_div(m * k * 2, 256) * 256;
}

// Split-K.  A pipeline stage of a tile up to ~112 columns wide costs about the
// same whatever its width (a copy of the kernel with no loads, no
// dequantisation and no MMAs keeps most of it), so fewer stages per CTA is
// what shortens such a call: s CTAs per tile (s = 2, 4 or 8) each take 1/s of
// K and a sum pass adds the s partial planes.  s is the largest that keeps
// tiles at most 112 columns wide (128 past 128 rows), each part whole
// 256-value blocks, one wave of one CTA per SM, and the planes within 256 MB.
// Up to 128 rows (128-row tiles) that is the rule.  Past 128 rows (256-row
// tiles) a split pays only where the unsplit tiles would be under 64 columns
// wide or K is 8,192 or longer; one B200, against one pass: M = 512, N 1,792,
// K 4,096 37.2 -> 30.5 us; M = 512, N 1,024, K 8,192 67.6 -> 30.6 us; M = 256,
// N 1,792 35.8 -> 23.8 us; M = 2,048, K 8,192, N 128 / 512 / 1,024 78.6 / 80.0
// / 86.8 -> 33.8 / 54.2 / 78.4 us; M = 2,048, N 1,024, K 28,672 285.7 -> 218.3
// us; while M = 512, N 3,584, K 4,096 stays one pass (42.3 against 43.0 us
// split).  These are the narrow shards of tensor-parallel prefill.
static int choose_split(uint64_t m, uint64_t n, uint64_t k, int sms) {
  int best = 1;
  if (m > 128 && choose_tiles(m, n, sms).bn >= 64 && k < 8192) return best;
  const uint64_t mt = ceil_div(m, m > 128 ? 256 : 128);  // row tiles
  for (int s = 2; s <= 8; s *= 2) {
    if (k % (256ull * s) != 0 || (uint64_t)s * m * n * 4 > (256ull << 20)) break;
    const TileChoice t = choose_tiles(m, n, sms / s);
    if (t.bn > (m > 128 ? 128 : 112) || (uint64_t)s * mt * ceil_div(n, (uint64_t)t.bn) > (uint64_t)sms)
      break;
    best = s;
  }
  return best;
}

// B200's SM count: the size a caller is told to provide (a launch on a device
// with fewer SMs splits less when the workspace is short).
constexpr int kB200Sms = 148;

uint64_t gemm_workspace_bytes_preferred(int fmt, uint64_t m, uint64_t n, uint64_t k) {
  const uint64_t base = gemm_workspace_bytes(fmt, m, n, k);
  const int s = choose_split(m, n, k, kB200Sms);
  return s > 1 ? base + (uint64_t)s * m * n * 4 : base;
}

bool gemm_supported(int fmt, uint64_t m, uint64_t n, uint64_t k) {
  return supported(fmt) && m >= 1 && n >= 1 && k % 256 == 0 && k >= 256 && m < (1u << 30) &&
         n < (1u << 30) && k < (1u << 24);
}

cudaError_t launch_gemm_core(int fmt, const void *w, uint64_t n, uint64_t k, const void *xb,
                             uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                             int *err, int sms, cudaStream_t stream, int ksplit);

cudaError_t launch_gemm(int fmt, const void *w, uint64_t n, uint64_t k, const float *x, uint64_t m,
                        const OutSpec &out, const float *addend, int addend_mode, void *workspace,
                        uint64_t workspace_bytes, int *err, int sms, cudaStream_t stream) {
  if (!gemm_supported(fmt, m, n, k) || workspace_bytes < gemm_workspace_bytes(fmt, m, n, k) ||
      (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return cudaErrorInvalidValue;
  __nv_bfloat16 *xb = static_cast<__nv_bfloat16 *>(workspace);
  const uint64_t n4 = m * k / 4;
  uint64_t blocks = ceil_div(n4, 256);
  if (blocks > (uint64_t)sms * 16) blocks = (uint64_t)sms * 16;
  // same shared-memory carveout as the GEMM: no SM reconfiguration between them
  cudaError_t e = cudaFuncSetAttribute(mgb_f32_to_bf16_kernel,
                                       cudaFuncAttributePreferredSharedMemoryCarveout,
                                       (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  e = launch_dependent(mgb_f32_to_bf16_kernel, dim3((unsigned)blocks), dim3(256), 0,
                                   stream, x, xb, m * k, out, err);
  if (e != cudaSuccess) return e;
  // room for the partial planes: split K (the sum pass writes every rank's y
  // of a tensor-parallel call; the call publishes after it)
  const uint64_t base = gemm_workspace_bytes(fmt, m, n, k);
  int s = choose_split(m, n, k, sms);
  while (s > 1 && workspace_bytes < base + (uint64_t)s * m * n * 4) s /= 2;
  if (s > 1) {
    float *part = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + base);
    e = launch_gemm_core(fmt, w, n, k, xb, m, plain_out(part, n), nullptr, 0, err, sms, stream, s);
    if (e == cudaSuccess) {
      uint64_t sblocks = ceil_div(m * n, 256);
      if (sblocks > (uint64_t)sms * 8) sblocks = (uint64_t)sms * 8;
      e = launch_dependent(mgb_splitk_sum_kernel, dim3((unsigned)sblocks), dim3(256), 0, stream,
                           (const float *)part, s, m, n, out, addend, addend_mode);
    }
    return e;
  }
  return launch_gemm_core(fmt, w, n, k, xb, m, out, addend, addend_mode, err, sms, stream, 1);
}

cudaError_t launch_gemm_bf16(int fmt, const void *w, uint64_t n, uint64_t k, const void *xb,
                             uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                             int *err, int sms, cudaStream_t stream) {
  return launch_gemm_core(fmt, w, n, k, xb, m, out, addend, addend_mode, err, sms, stream, 1);
}

// The GEMM kernel launch; ksplit = 2, 4 or 8 writes the K parts' partial sums
// into planes 0 .. ksplit-1 of out (one output, ldy = n, no addend).
cudaError_t launch_gemm_core(int fmt, const void *w, uint64_t n, uint64_t k, const void *xb,
                             uint64_t m, const OutSpec &out, const float *addend, int addend_mode,
                             int *err, int sms, cudaStream_t stream, int ksplit) {
  if (!gemm_supported(fmt, m, n, k) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(xb) & 15) ||
      (ksplit != 1 && ksplit != 2 && ksplit != 4 && ksplit != 8) ||
      k % (256ull * ksplit) != 0 ||
      (ksplit > 1 && (out.world != 1 || out.cta_counter || addend_mode != 0)))
    return cudaErrorInvalidValue;
  const Layout L(fmt, n, k);
  const TileChoice t = choose_tiles(m, n, sms / ksplit);
  GemmParams p = {};
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.qbytes = fmt == Q8_0 ? 64 : fmt == Q6_K ? 48 : 32;
  p.wsw = fmt == Q6_K ? 32 : fmt == Q5_K ? 48 : 16;
  p.bn = t.bn;
  const dim3 grid((unsigned)ceil_div(n, (uint64_t)t.bn), (unsigned)ceil_div(m, 128ull * t.subs),
                  (unsigned)ksplit);
  p.ksplit = ksplit;
  const uint32_t budget = 225 * 1024 - 1024 /*align slack*/ - 512 /*barriers*/;
  const int dqw = dq_warps_for(t.subs);
  // Stage geometry and ring depths for `atoms` K atoms per stage; false when
  // not even the shallowest rings fit.
  //
  // Narrow tiles (few weight rows per CTA) run their K loop faster with more
  // operand stages in flight: as many as fit (up to 6), then packed stages (up
  // to 8).  Dequant warp groups for narrow tiles (see the kernel): a group
  // waits on the slots of its own steps only, and an mbarrier parity wait
  // cannot tell phase q from phase q - 2, so the previous use of every slot a
  // group waits on must be a step that group waited on itself.  That holds for
  // the packed ring when its depth is a multiple of the group count, and for
  // the operand ring (released in K order by the MMA commits) when it is at
  // least that deep.
  int groups = 1, sa = 2, sp = 3;
  uint32_t ab = 0;
  auto size_rings = [&](int atoms) -> bool {
    p.atoms = atoms;
    p.a_bytes = 16384u * t.subs * atoms;
    p.b_atom = (uint32_t)ceil_div((uint64_t)t.bn * 128u, 1024) * 1024;
    p.b_bytes = p.b_atom * atoms;
    p.wq_bytes = (uint32_t)ceil_div((uint64_t)t.bn * p.qbytes * atoms, 1024) * 1024;
    p.ws_bytes = (uint32_t)ceil_div((uint64_t)t.bn * p.wsw, 1024) * 1024;
    p.pstage_bytes = p.wq_bytes + p.ws_bytes;
    p.ptx_bytes = (uint32_t)t.bn * (uint32_t)(p.qbytes * atoms + p.wsw);
    ab = p.a_bytes + p.b_bytes;
    auto fits = [&](int a, int q) { return (uint32_t)a * ab + (uint32_t)q * p.pstage_bytes <= budget; };
    groups = dqw == 16 ? (t.bn <= 128 ? 4 : 2) : (t.bn <= 64 ? 4 : t.bn <= 128 ? 2 : 1);
    sa = 2;
    sp = 2 * groups;
    while (groups > 1) {
      sp = 2 * groups;
      sa = 2;
      while (sa < 6 && fits(sa + 1, sp)) ++sa;
      if (fits(sa, sp) && sa >= groups) break;
      groups /= 2;
    }
    if (groups == 1) {
      sa = 2;
      sp = 3;
      if (!fits(sa, sp)) return false;
      while (sa < 6 && fits(sa + 1, sp)) ++sa;
      while (sp < 8 && fits(sa, sp + 1)) ++sp;
    }
    return true;
  };
  // 128-row tiles up to 128 columns wide take two K atoms per pipeline stage:
  // half the barrier rounds per K (wider tiles would be left with too shallow
  // rings)
  const bool two = t.subs == 1 && t.bn <= 128 && size_rings(2);
  if (!two && !size_rings(1)) return cudaErrorInvalidValue;
  p.dq_groups = groups;
  p.astages = sa;
  p.bstages = sa;
  p.pstages = sp;
  p.addend_mode = addend_mode;
  p.addend = addend;
  p.out = out;
  p.vec_out = ((out.ldy | out.col0) & 3) == 0;
  for (int r = 0; r < out.world; ++r)
    if (reinterpret_cast<uintptr_t>(out.y_ranks[r]) & 15) p.vec_out = 0;
  p.err = err;

  CUtensorMap map_a, map_wq, map_ws, map_y;
  if (!make_map_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xb, k, m, k * 2, KSTEP, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&map_wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, L.qs_row, n, L.qs_row,
                   (uint32_t)(p.qbytes * p.atoms), (uint32_t)t.bn, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&map_ws, CU_TENSOR_MAP_DATA_TYPE_UINT8,
                   static_cast<const uint8_t *>(w) + L.qs_bytes, L.sc_row, n, L.sc_row,
                   (uint32_t)p.wsw, (uint32_t)t.bn, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  // one output, no addend, 16-byte rows: the epilogue stores 32 x 32 blocks by TMA
  // (wide tiles only: for narrow ones the per-block waits outweigh the gain)
  // (the epilogue's per-warp scratch lies in the operand ring)
  const uint64_t ring_bytes = (uint64_t)sa * ab;
  p.tma_out = out.world == 1 && addend_mode == 0 && p.vec_out && out.col0 == 0 && t.bn >= 192 &&
              ksplit == 1 && ring_bytes >= (uint64_t)dqw * EPI_TMA_BYTES;
  if (out.world > 1 && ring_bytes < (uint64_t)dqw * EPI_SQUARE_BYTES) return cudaErrorInvalidValue;
  if (p.tma_out && !make_map_2d(&map_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, out.y_ranks[0], n, m,
                                out.ldy * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
    p.tma_out = 0;
  if (!p.tma_out) map_y = map_a;  // unused

  const size_t smem = (size_t)sa * ab + (size_t)sp * p.pstage_bytes + 1024 + 512;
  cudaError_t e = cudaSuccess;
#define MGB_GEMM_LAUNCH(KERN)                                                                  \
  do {                                                                                         \
    auto kern = KERN;                                                                          \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    if (e != cudaSuccess) return e;                                                            \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,             \
                             (int)cudaSharedmemCarveoutMaxShared);                             \
    if (e != cudaSuccess) return e;                                                            \
    e = launch_dependent(kern, grid, dim3(96 + 32 * dqw), smem, stream, map_a, map_wq, map_ws,   \
                         map_y, p);                                                            \
  } while (0)
#define MGB_GEMM_FMT(F)                                     \
  case F:                                                   \
    if (t.subs == 2) MGB_GEMM_LAUNCH((mgb_gemm_kernel<F, 2, 16, 1>));       \
    else if (two) MGB_GEMM_LAUNCH((mgb_gemm_kernel<F, 1, 16, 2>));         \
    else MGB_GEMM_LAUNCH((mgb_gemm_kernel<F, 1, 16, 1>));                  \
    break;
  switch (fmt) {
    MGB_GEMM_FMT(Q4_K)
    MGB_GEMM_FMT(Q6_K)
    MGB_GEMM_FMT(Q5_K)
    MGB_GEMM_FMT(Q8_0)
    MGB_GEMM_FMT(IQ4_NL)
    MGB_GEMM_FMT(Q4_0)
    default:
      return cudaErrorInvalidValue;
  }
#undef MGB_GEMM_FMT
#undef MGB_GEMM_LAUNCH
  return e;
}

}  // namespace mgb
