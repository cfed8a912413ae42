/*
 * CPU oracle for the packed-weight matmul path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference CPU Provider's packed-weight
 * arithmetic (astorise/Magnetar-provider-CPU, `src/native/quant.rs`,
 * `src/native/mod.rs`, `src/lib.rs`).  Only `tests/`, `__graft_entry__.smoke()`
 * and `bench.py`'s CPU-baseline leg may load this library, and only as the
 * checker or the timed CPU baseline.  The B200 product path never calls it.
 *
 * Compiled with `-ffp-contract=off` so every f32 operation rounds on its own,
 * as Rust (which never contracts `a * b + c` into an FMA) does.
 *
 * Parity pin: the dequantisation the reference calls lives in the absent
 * crate `magnetar-provider-api` 1.0.0 (ggml block formats).  This restatement
 * is pinned against gguf-py 0.19.0's dequantisation (an independent
 * implementation of the same ggml formats) by the committed fixtures in
 * `tests/golden/`, bit for bit.
 */
#ifndef MGB_ORACLE_H
#define MGB_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Format codes: the reference's `FORMATS` order (src/native/quant.rs:71-87). */
enum {
    ORC_Q8_0 = 0,
    ORC_Q4_K = 1,
    ORC_Q6_K = 2,
    ORC_Q2_K = 3,
    ORC_Q3_K = 4,
    ORC_IQ4_NL = 5,
    ORC_IQ4_XS = 6,
    ORC_IQ2_XXS = 7,
    ORC_IQ2_XS = 8,
    ORC_IQ2_S = 9,
    ORC_IQ3_XXS = 10,
    ORC_IQ3_S = 11,
    ORC_Q5_K = 12,
    ORC_Q4_0 = 13,
};

#define ORC_RUN 32

/* A decoded run (src/native/quant.rs:21-28): value i = scale[i/16]*q[i] - min[i/16]. */
typedef struct orc_run {
    int8_t q[ORC_RUN];
    float scale[2];
    float min[2];
} orc_run;

/* 1 when the oracle decodes `format` (Q8_0, Q4_K, Q5_K, Q6_K, IQ4_NL, Q4_0), else 0. */
int orc_supported(int format);
/* Weights per block (32 or 256) and bytes per block; 0 for unknown formats. */
int orc_block_elements(int format);
int orc_block_bytes(int format);

/* Exact IEEE binary16 -> binary32 (the reference's `half` table, quant.rs:30-40). */
float orc_f16_to_f32(uint16_t bits);

/* ggml get_scale_min_k4 (quant.rs:46-57). */
void orc_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m);

/* The IQ4_NL codebook and Q4_0's q-8 table (16 entries each). */
const int8_t *orc_iq4nl_values(void);
const int8_t *orc_q4_0_values(void);

/* `decode` (quant.rs:100-280) for the supported formats; returns 0 on success. */
int orc_decode_run(int format, const uint8_t *block, int run, orc_run *out);

/* `RunReader::read` (quant.rs:313-321): run `run` of stored row `row`. */
int orc_read_run(int format, const uint8_t *bytes, uint64_t stored_cols, uint64_t row,
                 uint64_t run, orc_run *out);

/* `dequantize_row` (quant.rs:1700-1711). */
int orc_dequantize_row(int format, const uint8_t *bytes, uint64_t stored_cols, uint64_t row,
                       float *out);

/* Every stored row dequantised: out[stored_rows * stored_cols], stored order. */
int orc_dequantize(int format, const uint8_t *bytes, uint64_t stored_rows,
                   uint64_t stored_cols, float *out);

/* `element` (quant.rs:1691-1698). */
float orc_element(int format, const uint8_t *bytes, uint64_t stored_cols, uint64_t row,
                  uint64_t index);

/*
 * Correctness-first dense matmul (src/lib.rs:262-318): a is [a_rows, a_cols],
 * b is [b_rows, b_cols], both row-major; logical transposes by stride swap;
 * loop order row -> inner -> col, `+=`, no zero-skip.  Returns 0, or -1 on an
 * inner-dimension mismatch.
 */
int orc_matmul(const float *a, uint64_t a_rows, uint64_t a_cols, const float *b,
               uint64_t b_rows, uint64_t b_cols, int transpose_a, int transpose_b,
               float *out);

/* `add` with the row broadcast of src/lib.rs:1028-1075 (b is [cols] or same shape). */
int orc_add(const float *a, uint64_t a_len, uint64_t cols, const float *b, uint64_t b_len,
            float *out);

/* `quantize_rows` (quant.rs:350-378): per 32-value block. */
void orc_quantize_rows(const float *rows, uint64_t len, int8_t *values, float *scales,
                       int32_t *sums /* [blocks][2] */);

/*
 * The scalar `columns` (quant.rs:559-597): out[r*count + c] for columns
 * first..first+count of x[m,k] times the packed W (stored rows = output
 * columns).  int8 != 0 takes the quantised-activation branch.
 */
int orc_columns(int format, const uint8_t *bytes, uint64_t stored_cols, const float *x,
                uint64_t m, uint64_t k, uint64_t first, uint64_t count, int int8,
                float *out);

/*
 * `NativeState::packed_matmul` (src/native/mod.rs:109-152), single threaded:
 * y[m, n] with n = stored_rows.  Returns 0, or -1 with the reference's shape
 * error when k != stored_cols or k % 32 != 0.
 */
int orc_packed_matmul(int format, const uint8_t *bytes, uint64_t stored_rows,
                      uint64_t stored_cols, const float *x, uint64_t m, uint64_t k, int int8,
                      float *y);

/*
 * `axpy_columns` (quant.rs:1658-1689) over every run: the input-major branch,
 * W's stored rows are the k input rows, y[m, stored_cols].
 */
int orc_packed_axpy(int format, const uint8_t *bytes, uint64_t stored_rows,
                    uint64_t stored_cols, const float *x, uint64_t m, uint64_t k, float *y);

/* The reference's test generators (src/native/tests.rs:34-75), for mirrored tests. */
void orc_test_packed(int format, uint64_t rows, uint64_t cols, uint32_t seed, uint8_t *out);
void orc_test_activations(uint64_t rows, uint64_t cols, uint32_t seed, float *out);

#ifdef __cplusplus
}
#endif

#endif
