/*
 * CPU oracle for the packed-weight matmul path — TEST INFRASTRUCTURE ONLY.
 * See oracle.h for the contract; every function cites the reference
 * (astorise/Magnetar-provider-CPU) file:line it restates.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- format table (block_elements / block_bytes as src/native/quant.rs uses them:
 *      Q8_0 34 B/32, Q4_K 144 B/256, IQ4_NL and Q4_0 18 B/32) ---------------------- */

int orc_supported(int format) {
    return format == ORC_Q8_0 || format == ORC_Q4_K || format == ORC_IQ4_NL ||
           format == ORC_Q4_0 || format == ORC_Q6_K || format == ORC_Q5_K;
}

int orc_block_elements(int format) {
    switch (format) {
    case ORC_Q8_0: case ORC_IQ4_NL: case ORC_Q4_0: return 32;
    case ORC_Q4_K: case ORC_Q6_K: case ORC_Q5_K: return 256;
    default: return 0;
    }
}

int orc_block_bytes(int format) {
    switch (format) {
    case ORC_Q8_0: return 34;
    case ORC_Q4_K: return 144;
    case ORC_Q6_K: return 210;
    case ORC_Q5_K: return 176;
    case ORC_IQ4_NL: case ORC_Q4_0: return 18;
    default: return 0;
    }
}

/* ---- f16 -> f32, exact (src/native/quant.rs:30-40 tabulates `f16_to_f32`) --------- */

static float bits_to_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    if (exp == 0) {
        if (man == 0) return bits_to_f32(sign);
        /* subnormal: man * 2^-24, exact in f32 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (exp == 31) return bits_to_f32(sign | 0x7f800000u | (man << 13));
    return bits_to_f32(sign | ((exp + 112) << 23) | (man << 13));
}

static float half_at(const uint8_t *b, int at) {
    return orc_f16_to_f32((uint16_t)(b[at] | (b[at + 1] << 8)));
}

/* ---- get_scale_min_k4 (src/native/quant.rs:46-57) --------------------------------- */

void orc_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* ---- codebooks: the ggml IQ4_NL non-linear table (checked against gguf-py's
 *      `IQ4_NL.kvalues` by tests/test_oracle.py) and Q4_0's `q - 8` ------------------ */

static const int8_t IQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                 1,    13,   25,  38,  53,  69,  89,  113};
static const int8_t Q40[16] = {-8, -7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7};

const int8_t *orc_iq4nl_values(void) { return IQ4NL; }
const int8_t *orc_q4_0_values(void) { return Q40; }

/* ---- decode (src/native/quant.rs:100-280: Q8_0 :102-109, Q4_K :110-121,
 *      Q5_K :122-135, Q6_K :136-149, IQ4_NL / Q4_0 :180-195) --------------------------- */

int orc_decode_run(int format, const uint8_t *block, int run, orc_run *out) {
    switch (format) {
    case ORC_Q8_0: {
        float d = half_at(block, 0);
        for (int i = 0; i < ORC_RUN; i++) out->q[i] = (int8_t)block[2 + i];
        out->scale[0] = out->scale[1] = d;
        out->min[0] = out->min[1] = 0.0f;
        return 0;
    }
    case ORC_Q4_K: {
        float d = half_at(block, 0);
        float dmin = half_at(block, 2);
        uint8_t sc, m;
        orc_scale_min_k4(run, block + 4, &sc, &m);
        int chunk = run / 2, shift = 4 * (run % 2);
        const uint8_t *qs = block + 16 + 32 * chunk;
        for (int i = 0; i < ORC_RUN; i++) out->q[i] = (int8_t)((qs[i] >> shift) & 0xF);
        out->scale[0] = out->scale[1] = d * (float)sc;
        out->min[0] = out->min[1] = dmin * (float)m;
        return 0;
    }
    case ORC_Q5_K: {
        /* d, dmin; scales as Q4_K; run r's low nibbles in the 32 bytes at
           48 + 32 (r / 2) (shift 4 (r % 2)), its fifth bits at bit r of the
           32 bytes at 16 */
        float d = half_at(block, 0);
        float dmin = half_at(block, 2);
        uint8_t sc, m;
        orc_scale_min_k4(run, block + 4, &sc, &m);
        int chunk = run / 2, shift = 4 * (run % 2);
        const uint8_t *low = block + 48 + 32 * chunk, *high = block + 16;
        for (int i = 0; i < ORC_RUN; i++)
            out->q[i] = (int8_t)(((low[i] >> shift) & 0xF) | (((high[i] >> run) & 1) << 4));
        out->scale[0] = out->scale[1] = d * (float)sc;
        out->min[0] = out->min[1] = dmin * (float)m;
        return 0;
    }
    case ORC_Q6_K: {
        /* d at 208; run r = 4 h + g: low nibbles in the 32 bytes at
           64 h + 32 (g % 2) (shift 4 (g / 2)), high 2 bits in the 32 bytes at
           128 + 32 h (shift 2 g), q - 32; one int8 scale per 16 values at
           192 + 8 h + 2 g + p; no min */
        float d = half_at(block, 208);
        int h = run / 4, g = run % 4;
        const uint8_t *low = block + 64 * h + 32 * (g % 2), *high = block + 128 + 32 * h;
        int ls = 4 * (g / 2), hs = 2 * g;
        for (int i = 0; i < ORC_RUN; i++)
            out->q[i] = (int8_t)((((low[i] >> ls) & 0xF) | (((high[i] >> hs) & 3) << 4)) - 32);
        for (int p = 0; p < 2; p++) {
            out->scale[p] = d * (float)(int8_t)block[192 + 8 * h + 2 * g + p];
            out->min[p] = 0.0f;
        }
        return 0;
    }
    case ORC_IQ4_NL:
    case ORC_Q4_0: {
        const int8_t *table = format == ORC_Q4_0 ? Q40 : IQ4NL;
        float d = half_at(block, 0);
        for (int l = 0; l < 16; l++) {
            uint8_t byte = block[2 + l];
            out->q[l] = table[byte & 0xF];
            out->q[l + 16] = table[byte >> 4];
        }
        out->scale[0] = out->scale[1] = d;
        out->min[0] = out->min[1] = 0.0f;
        return 0;
    }
    default:
        return -1;
    }
}

/* ---- RunReader (src/native/quant.rs:282-338) -------------------------------------- */

int orc_read_run(int format, const uint8_t *bytes, uint64_t stored_cols, uint64_t row,
                 uint64_t run, orc_run *out) {
    int be = orc_block_elements(format), bb = orc_block_bytes(format);
    if (!be) return -1;
    uint64_t row_bytes = stored_cols / (uint64_t)be * (uint64_t)bb;
    uint64_t runs_per_block = (uint64_t)be / ORC_RUN;
    uint64_t block = run / runs_per_block;
    const uint8_t *start = bytes + row * row_bytes + block * (uint64_t)bb;
    return orc_decode_run(format, start, (int)(run % runs_per_block), out);
}

static inline float run_value(const orc_run *r, int i) {
    int p = i / 16;
    return r->scale[p] * (float)r->q[i] - r->min[p];
}

/* ---- element / dequantize_row (src/native/quant.rs:1691-1711) --------------------- */

float orc_element(int format, const uint8_t *bytes, uint64_t stored_cols, uint64_t row,
                  uint64_t index) {
    orc_run r;
    if (orc_read_run(format, bytes, stored_cols, row, index / ORC_RUN, &r)) return NAN;
    return run_value(&r, (int)(index % ORC_RUN));
}

int orc_dequantize_row(int format, const uint8_t *bytes, uint64_t stored_cols, uint64_t row,
                       float *out) {
    orc_run r;
    for (uint64_t u = 0; u < stored_cols / ORC_RUN; u++) {
        if (orc_read_run(format, bytes, stored_cols, row, u, &r)) return -1;
        for (int i = 0; i < ORC_RUN; i++) out[u * ORC_RUN + i] = run_value(&r, i);
    }
    return 0;
}

int orc_dequantize(int format, const uint8_t *bytes, uint64_t stored_rows,
                   uint64_t stored_cols, float *out) {
    for (uint64_t r = 0; r < stored_rows; r++)
        if (orc_dequantize_row(format, bytes, stored_cols, r, out + r * stored_cols)) return -1;
    return 0;
}

/* ---- dense f32 matmul (src/lib.rs:262-318) ---------------------------------------- */

int orc_matmul(const float *a, uint64_t a_rows, uint64_t a_cols, const float *b,
               uint64_t b_rows, uint64_t b_cols, int transpose_a, int transpose_b,
               float *out) {
    uint64_t m = transpose_a ? a_cols : a_rows, k = transpose_a ? a_rows : a_cols;
    uint64_t k2 = transpose_b ? b_cols : b_rows, n = transpose_b ? b_rows : b_cols;
    if (k != k2) return -1;
    uint64_t a_row_stride = transpose_a ? 1 : a_cols, a_inner_stride = transpose_a ? a_cols : 1;
    uint64_t b_inner_stride = transpose_b ? 1 : b_cols, b_col_stride = transpose_b ? b_cols : 1;
    memset(out, 0, sizeof(float) * m * n);
    for (uint64_t row = 0; row < m; row++) {
        float *o = out + row * n;
        for (uint64_t inner = 0; inner < k; inner++) {
            float av = a[row * a_row_stride + inner * a_inner_stride];
            uint64_t base = inner * b_inner_stride;
            for (uint64_t col = 0; col < n; col++) o[col] += av * b[base + col * b_col_stride];
        }
    }
    return 0;
}

/* ---- add with row broadcast (src/lib.rs:1028-1075) -------------------------------- */

int orc_add(const float *a, uint64_t a_len, uint64_t cols, const float *b, uint64_t b_len,
            float *out) {
    if (b_len == a_len) {
        for (uint64_t i = 0; i < a_len; i++) out[i] = a[i] + b[i];
        return 0;
    }
    if (b_len != cols || cols == 0 || a_len % cols) return -1;
    for (uint64_t i = 0; i < a_len; i++) out[i] = a[i] + b[i % cols];
    return 0;
}

/* ---- quantize_rows (src/native/quant.rs:350-378) ---------------------------------- */

void orc_quantize_rows(const float *rows, uint64_t len, int8_t *values, float *scales,
                       int32_t *sums) {
    uint64_t blocks = len / ORC_RUN;
    for (uint64_t b = 0; b < blocks; b++) {
        const float *x = rows + b * ORC_RUN;
        float amax = 0.0f;
        for (int i = 0; i < ORC_RUN; i++) amax = fmaxf(amax, fabsf(x[i]));
        float d = amax / 127.0f;
        int32_t s[2] = {0, 0};
        for (int i = 0; i < ORC_RUN; i++) {
            int8_t q = 0;
            if (amax != 0.0f) {
                float r = nearbyintf(x[i] / d); /* default rounding: ties to even */
                /* Rust's `as i8` saturates and maps NaN to 0 */
                q = isnan(r) ? 0 : (int8_t)(r > 127.0f ? 127 : (r < -128.0f ? -128 : r));
            }
            values[b * ORC_RUN + i] = q;
            s[i / 16] += q;
        }
        scales[b] = d;
        sums[2 * b] = s[0];
        sums[2 * b + 1] = s[1];
    }
}

/* ---- scalar columns (src/native/quant.rs:559-597, dot_halves_scalar :382-388) ----- */

typedef struct {
    int8_t *values;
    float *scales;
    int32_t *sums;
} quantized_rows;

static int quantize_alloc(const float *x, uint64_t n, quantized_rows *q) {
    q->values = (int8_t *)malloc(n ? n : 1);
    q->scales = (float *)malloc(sizeof(float) * (n / ORC_RUN + 1));
    q->sums = (int32_t *)malloc(sizeof(int32_t) * 2 * (n / ORC_RUN + 1));
    if (!q->values || !q->scales || !q->sums) return -1;
    orc_quantize_rows(x, n, q->values, q->scales, q->sums);
    return 0;
}

static void quantize_free(quantized_rows *q) {
    free(q->values);
    free(q->scales);
    free(q->sums);
}

static int columns_impl(int format, const uint8_t *bytes, uint64_t stored_cols, const float *x,
                        const quantized_rows *qa, uint64_t m, uint64_t k, uint64_t first,
                        uint64_t count, float *acc, float *out) {
    uint64_t runs = k / ORC_RUN;
    orc_run run;
    for (uint64_t c = 0; c < count; c++) {
        for (uint64_t r = 0; r < m; r++) acc[r] = 0.0f;
        for (uint64_t u = 0; u < runs; u++) {
            if (orc_read_run(format, bytes, stored_cols, first + c, u, &run)) return -1;
            for (uint64_t r = 0; r < m; r++) {
                uint64_t block = r * runs + u;
                if (qa) {
                    int32_t dots[2] = {0, 0};
                    const int8_t *a = qa->values + block * ORC_RUN;
                    for (int i = 0; i < ORC_RUN; i++) dots[i / 16] += (int32_t)run.q[i] * a[i];
                    float d = qa->scales[block];
                    const int32_t *sm = qa->sums + 2 * block;
                    acc[r] += d * (run.scale[0] * (float)dots[0] + run.scale[1] * (float)dots[1] -
                                   run.min[0] * (float)sm[0] - run.min[1] * (float)sm[1]);
                } else {
                    const float *xv = x + block * ORC_RUN;
                    for (int i = 0; i < ORC_RUN; i++) {
                        int p = i / 16;
                        acc[r] += (run.scale[p] * (float)run.q[i] - run.min[p]) * xv[i];
                    }
                }
            }
        }
        for (uint64_t r = 0; r < m; r++) out[r * count + c] = acc[r];
    }
    return 0;
}

int orc_columns(int format, const uint8_t *bytes, uint64_t stored_cols, const float *x,
                uint64_t m, uint64_t k, uint64_t first, uint64_t count, int int8,
                float *out) {
    quantized_rows q = {0, 0, 0};
    float *acc = (float *)malloc(sizeof(float) * (m ? m : 1));
    int rc = acc ? 0 : -1;
    if (!rc && int8) rc = quantize_alloc(x, m * k, &q);
    if (!rc) rc = columns_impl(format, bytes, stored_cols, x, int8 ? &q : 0, m, k, first, count,
                               acc, out);
    if (int8) quantize_free(&q);
    free(acc);
    return rc;
}

/* ---- NativeState::packed_matmul (src/native/mod.rs:109-152) ----------------------- */

int orc_packed_matmul(int format, const uint8_t *bytes, uint64_t stored_rows,
                      uint64_t stored_cols, const float *x, uint64_t m, uint64_t k, int int8,
                      float *y) {
    if (k != stored_cols || k % ORC_RUN || !orc_supported(format)) return -1;
    uint64_t n = stored_rows;
    quantized_rows q = {0, 0, 0};
    float *acc = (float *)malloc(sizeof(float) * (m ? m : 1));
    float *local = (float *)malloc(sizeof(float) * (m ? m : 1));
    int rc = (acc && local) ? 0 : -1;
    if (!rc && int8) rc = quantize_alloc(x, m * k, &q);
    /* every column is independent: the reference's chunked pool partition
       (mod.rs:135-150) writes the same values as this sequential sweep */
    for (uint64_t c = 0; !rc && c < n; c++) {
        rc = columns_impl(format, bytes, stored_cols, x, int8 ? &q : 0, m, k, c, 1, acc, local);
        for (uint64_t r = 0; !rc && r < m; r++) y[r * n + c] = local[r];
    }
    if (int8) quantize_free(&q);
    free(acc);
    free(local);
    return rc;
}

/* ---- axpy_columns (src/native/quant.rs:1658-1689) over all runs ------------------- */

int orc_packed_axpy(int format, const uint8_t *bytes, uint64_t stored_rows,
                    uint64_t stored_cols, const float *x, uint64_t m, uint64_t k, float *y) {
    if (k != stored_rows) return -1;
    uint64_t n = stored_cols, runs = n / ORC_RUN;
    memset(y, 0, sizeof(float) * m * n);
    orc_run run;
    float values[ORC_RUN];
    for (uint64_t j = 0; j < k; j++) {
        for (uint64_t u = 0; u < runs; u++) {
            if (orc_read_run(format, bytes, stored_cols, j, u, &run)) return -1;
            for (int i = 0; i < ORC_RUN; i++) values[i] = run_value(&run, i);
            for (uint64_t r = 0; r < m; r++) {
                float w = x[r * k + j];
                if (w == 0.0f) continue;
                float *o = y + r * n + u * ORC_RUN;
                for (int i = 0; i < ORC_RUN; i++) o[i] += w * values[i];
            }
        }
    }
    return 0;
}

/* ---- the reference's test generators (src/native/tests.rs:23-75) ------------------ */

static uint32_t xorshift32(uint32_t *s) {
    uint32_t v = *s;
    v ^= v << 13;
    v ^= v >> 17;
    v ^= v << 5;
    *s = v;
    return v;
}

static int half_offsets(int format, int *out) {
    switch (format) {
    case ORC_Q4_K: case ORC_Q5_K: out[0] = 0; out[1] = 2; return 2;
    case ORC_Q6_K: out[0] = 208; return 1;
    case ORC_Q2_K: out[0] = 80; out[1] = 82; return 2;
    case ORC_Q3_K: out[0] = 108; return 1;
    default: out[0] = 0; return 1;
    }
}

void orc_test_packed(int format, uint64_t rows, uint64_t cols, uint32_t seed, uint8_t *out) {
    uint32_t s = seed * 2654435761u + 1u;
    int bb = orc_block_bytes(format), be = orc_block_elements(format);
    uint64_t blocks = rows * cols / (uint64_t)be;
    int offs[2];
    int nh = half_offsets(format, offs);
    for (uint64_t b = 0; b < blocks; b++) {
        uint8_t *blk = out + b * (uint64_t)bb;
        for (int i = 0; i < bb; i++) blk[i] = (uint8_t)(xorshift32(&s) % 256);
        for (int h = 0; h < nh; h++) {
            uint16_t exponent = (uint16_t)(3 + xorshift32(&s) % 5);
            uint16_t bits = (uint16_t)((exponent << 10) | (xorshift32(&s) % 1024));
            blk[offs[h]] = (uint8_t)(bits & 0xff);
            blk[offs[h] + 1] = (uint8_t)(bits >> 8);
        }
    }
}

void orc_test_activations(uint64_t rows, uint64_t cols, uint32_t seed, float *out) {
    uint32_t s = seed + 7u;
    for (uint64_t i = 0; i < rows * cols; i++)
        out[i] = (float)(xorshift32(&s) % 2001) / 1000.0f - 1.0f;
}
