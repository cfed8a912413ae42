/*
 * CPU baseline — TEST AND BENCHMARK INFRASTRUCTURE ONLY.
 *
 * A C restatement of the reference CPU Provider's default packed-matmul path
 * (astorise/Magnetar-provider-CPU `NativeState::packed_matmul`,
 * src/native/mod.rs:109-152): activations quantised to int8 per 32-value
 * block (`quantize_rows`, src/native/quant.rs:350-378), output columns split
 * into tasks of `max(8, ceil(n / (4 * threads)))` (mod.rs:134-136) across a
 * persistent worker pool in which the calling thread also works
 * (src/native/pool.rs:58-155), and the AVX2 column kernels:
 *   Q4_K   `columns_q4k_avx2`   src/native/quant.rs:673-744
 *   Q8_0   `columns_avx2`       src/native/quant.rs:604-664 (+ `vector_run` :1546-1650)
 *   IQ4_NL `columns_iq4nl_avx2` src/native/quant.rs:1438-1483 (+ `iq4_pair` :1364-1384,
 *   Q4_0    `accumulate_signed` :956-984, `hsum` :909-917)
 * The instruction choice follows the reference because the same algorithm on
 * the same ISA has one natural spelling; this file is the timed CPU arm and a
 * second checker, never part of the B200 product.
 *
 * `cpb_packed_matmul_f32` times the f32-activation scalar path (quant.rs:559-597),
 * the one numerically equal to the parity oracle.
 */
#include <immintrin.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

/* ---------------------------------------------------------------- pool ---- */

typedef void (*task_fn)(void *ctx, uint64_t index);

typedef struct {
    pthread_mutex_t lock;
    pthread_cond_t wake, done;
    pthread_t *workers;
    int threads;
    uint64_t generation;
    int shutdown;
    /* current job */
    task_fn fn;
    void *ctx;
    uint64_t tasks;
    atomic_uint_fast64_t next, pending;
    int finished;
} pool_t;

static void pool_work(pool_t *p) {
    for (;;) {
        uint64_t i = atomic_fetch_add(&p->next, 1);
        if (i >= p->tasks) return;
        p->fn(p->ctx, i);
        if (atomic_fetch_sub(&p->pending, 1) == 1) {
            pthread_mutex_lock(&p->lock);
            p->finished = 1;
            pthread_cond_broadcast(&p->done);
            pthread_mutex_unlock(&p->lock);
        }
    }
}

static void *pool_worker(void *arg) {
    pool_t *p = (pool_t *)arg;
    uint64_t seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->lock);
        while (!p->shutdown && p->generation == seen) pthread_cond_wait(&p->wake, &p->lock);
        if (p->shutdown) {
            pthread_mutex_unlock(&p->lock);
            return 0;
        }
        seen = p->generation;
        pthread_mutex_unlock(&p->lock);
        pool_work(p);
    }
}

static pool_t *pool_new(int threads) {
    pool_t *p = (pool_t *)calloc(1, sizeof(pool_t));
    pthread_mutex_init(&p->lock, 0);
    pthread_cond_init(&p->wake, 0);
    pthread_cond_init(&p->done, 0);
    p->threads = threads < 1 ? 1 : threads;
    p->workers = (pthread_t *)calloc((size_t)p->threads, sizeof(pthread_t));
    for (int i = 1; i < p->threads; i++) pthread_create(&p->workers[i], 0, pool_worker, p);
    return p;
}

static void pool_free(pool_t *p) {
    pthread_mutex_lock(&p->lock);
    p->shutdown = 1;
    pthread_cond_broadcast(&p->wake);
    pthread_mutex_unlock(&p->lock);
    for (int i = 1; i < p->threads; i++) pthread_join(p->workers[i], 0);
    free(p->workers);
    free(p);
}

static void pool_run(pool_t *p, uint64_t tasks, task_fn fn, void *ctx) {
    if (!tasks) return;
    if (tasks == 1 || p->threads == 1) {
        for (uint64_t i = 0; i < tasks; i++) fn(ctx, i);
        return;
    }
    pthread_mutex_lock(&p->lock);
    p->fn = fn;
    p->ctx = ctx;
    p->tasks = tasks;
    atomic_store(&p->next, 0);
    atomic_store(&p->pending, tasks);
    p->finished = 0;
    p->generation++;
    pthread_cond_broadcast(&p->wake);
    pthread_mutex_unlock(&p->lock);
    pool_work(p);
    pthread_mutex_lock(&p->lock);
    while (!p->finished) pthread_cond_wait(&p->done, &p->lock);
    pthread_mutex_unlock(&p->lock);
}

/* ------------------------------------------------------------- helpers ---- */

static inline float half_f16c(const uint8_t *b, int at) {
    int bits = b[at] | (b[at + 1] << 8);
    return _mm_cvtss_f32(_mm_cvtph_ps(_mm_cvtsi32_si128(bits)));
}

static inline float hsum(__m256 lanes) {
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(lanes), _mm256_extractf128_ps(lanes, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    return _mm_cvtss_f32(_mm_add_ss(h, _mm_shuffle_ps(h, h, 1)));
}

typedef struct {
    const int8_t *values;
    const float *scales;
    const int32_t *sums;
} qrows;

/* Q4_K: one pass per super-block, both nibble runs of each 32-byte chunk. */
static void columns_q4k(const uint8_t *w, uint64_t row_bytes, const qrows *q, uint64_t m,
                        uint64_t k, uint64_t first, uint64_t count, __m256 *acc, float *mins,
                        float *out) {
    const uint64_t runs = k / 32, blocks = k / 256;
    const __m256i low_mask = _mm256_set1_epi8(0xF);
    const __m256i ones = _mm256_set1_epi16(1);
    for (uint64_t c = 0; c < count; c++) {
        for (uint64_t r = 0; r < m; r++) {
            acc[r] = _mm256_setzero_ps();
            mins[r] = 0.0f;
        }
        const uint8_t *row = w + (first + c) * row_bytes;
        for (uint64_t b = 0; b < blocks; b++) {
            const uint8_t *block = row + b * 144;
            float d = half_f16c(block, 0), dmin = half_f16c(block, 2);
            float scale[8], min[8];
            for (int j = 0; j < 8; j++) {
                uint8_t sc, mn;
                orc_scale_min_k4(j, block + 4, &sc, &mn);
                scale[j] = d * (float)sc;
                min[j] = dmin * (float)mn;
            }
            for (int chunk = 0; chunk < 4; chunk++) {
                __m256i bytes = _mm256_loadu_si256((const __m256i *)(block + 16 + 32 * chunk));
                __m256i nib[2] = {_mm256_and_si256(bytes, low_mask),
                                  _mm256_and_si256(_mm256_srli_epi16(bytes, 4), low_mask)};
                for (int half = 0; half < 2; half++) {
                    int j = 2 * chunk + half;
                    uint64_t u = b * 8 + (uint64_t)j;
                    for (uint64_t r = 0; r < m; r++) {
                        uint64_t index = r * runs + u;
                        __m256i x = _mm256_loadu_si256((const __m256i *)(q->values + index * 32));
                        __m256 sums = _mm256_cvtepi32_ps(
                            _mm256_madd_epi16(_mm256_maddubs_epi16(nib[half], x), ones));
                        float da = q->scales[index];
                        acc[r] = _mm256_fmadd_ps(sums, _mm256_set1_ps(da * scale[j]), acc[r]);
                        mins[r] += da * min[j] * (float)(q->sums[2 * index] + q->sums[2 * index + 1]);
                    }
                }
            }
        }
        for (uint64_t r = 0; r < m; r++) out[r * count + c] = hsum(acc[r]) - mins[r];
    }
}

/* Signed 32-value run times every row's int8 activations (sign trick). */
static inline void accumulate_signed(__m256i w, float scale, const qrows *q, uint64_t runs,
                                     uint64_t u, uint64_t m, __m256 *acc) {
    const __m256i ones = _mm256_set1_epi16(1);
    __m256i mag = _mm256_sign_epi8(w, w);
    for (uint64_t r = 0; r < m; r++) {
        uint64_t index = r * runs + u;
        __m256i x = _mm256_loadu_si256((const __m256i *)(q->values + index * 32));
        __m256 sums = _mm256_cvtepi32_ps(
            _mm256_madd_epi16(_mm256_maddubs_epi16(mag, _mm256_sign_epi8(x, w)), ones));
        acc[r] = _mm256_fmadd_ps(sums, _mm256_set1_ps(q->scales[index] * scale), acc[r]);
    }
}

/* Q8_0 through the generic kernel: one run = one block, loaded as is. */
static void columns_q8_0(const uint8_t *w, uint64_t row_bytes, const qrows *q, uint64_t m,
                         uint64_t k, uint64_t first, uint64_t count, __m256 *acc, float *out) {
    const uint64_t runs = k / 32;
    for (uint64_t c = 0; c < count; c++) {
        for (uint64_t r = 0; r < m; r++) acc[r] = _mm256_setzero_ps();
        const uint8_t *row = w + (first + c) * row_bytes;
        for (uint64_t u = 0; u < runs; u++) {
            const uint8_t *block = row + u * 34;
            __m256i v = _mm256_loadu_si256((const __m256i *)(block + 2));
            accumulate_signed(v, half_f16c(block, 0), q, runs, u, m, acc);
        }
        for (uint64_t r = 0; r < m; r++) out[r * count + c] = hsum(acc[r]);
    }
}

/* IQ4_NL / Q4_0: two blocks' index bytes per register, codebook by vpshufb. */
static void columns_iq4(const uint8_t *w, uint64_t row_bytes, const qrows *q, uint64_t m,
                        uint64_t k, uint64_t first, uint64_t count, __m256 *acc,
                        const int8_t *table, float *out) {
    const uint64_t runs = k / 32;
    const __m256i mask = _mm256_set1_epi8(0xF);
    __m128i t = _mm_loadu_si128((const __m128i *)table);
    const __m256i tab = _mm256_set_m128i(t, t);
    for (uint64_t c = 0; c < count; c++) {
        for (uint64_t r = 0; r < m; r++) acc[r] = _mm256_setzero_ps();
        const uint8_t *row = w + (first + c) * row_bytes;
        for (uint64_t u = 0; u < runs; u += 2) {
            int pair = u + 1 < runs;
            const uint8_t *b0 = row + u * 18;
            __m128i lo = _mm_loadu_si128((const __m128i *)(b0 + 2));
            __m128i hi = pair ? _mm_loadu_si128((const __m128i *)(row + (u + 1) * 18 + 2))
                              : _mm_setzero_si128();
            __m256i bytes = _mm256_set_m128i(hi, lo);
            __m256i low = _mm256_and_si256(bytes, mask);
            __m256i high = _mm256_and_si256(_mm256_srli_epi16(bytes, 4), mask);
            __m256i w0 = _mm256_shuffle_epi8(tab, _mm256_permute2x128_si256(low, high, 0x20));
            __m256i w1 = _mm256_shuffle_epi8(tab, _mm256_permute2x128_si256(low, high, 0x31));
            accumulate_signed(w0, half_f16c(b0, 0), q, runs, u, m, acc);
            if (pair) accumulate_signed(w1, half_f16c(row + (u + 1) * 18, 0), q, runs, u + 1, m, acc);
        }
        for (uint64_t r = 0; r < m; r++) out[r * count + c] = hsum(acc[r]);
    }
}

/* ---------------------------------------------------------- entry points -- */

typedef struct {
    int format, int8;
    const uint8_t *w;
    uint64_t row_bytes, n, m, k, chunk;
    const float *x;
    qrows q;
    float *y;
} job_t;

static void task(void *ctx, uint64_t index) {
    job_t *j = (job_t *)ctx;
    uint64_t first = index * j->chunk;
    uint64_t count = j->n - first < j->chunk ? j->n - first : j->chunk;
    float *local = (float *)malloc(sizeof(float) * j->m * count);
    if (j->int8) {
        __m256 *acc = (__m256 *)_mm_malloc(sizeof(__m256) * j->m, 32);
        float *mins = (float *)malloc(sizeof(float) * j->m);
        switch (j->format) {
        case ORC_Q4_K: columns_q4k(j->w, j->row_bytes, &j->q, j->m, j->k, first, count, acc, mins, local); break;
        case ORC_Q8_0: columns_q8_0(j->w, j->row_bytes, &j->q, j->m, j->k, first, count, acc, local); break;
        case ORC_IQ4_NL: columns_iq4(j->w, j->row_bytes, &j->q, j->m, j->k, first, count, acc, orc_iq4nl_values(), local); break;
        default: columns_iq4(j->w, j->row_bytes, &j->q, j->m, j->k, first, count, acc, orc_q4_0_values(), local); break;
        }
        _mm_free(acc);
        free(mins);
    } else {
        orc_columns(j->format, j->w, j->k, j->x, j->m, j->k, first, count, 0, local);
    }
    for (uint64_t r = 0; r < j->m; r++)
        for (uint64_t c = 0; c < count; c++) j->y[r * j->n + first + c] = local[r * count + c];
    free(local);
}

static pool_t *g_pool;
static int g_threads;

/* Creates (or resizes) the persistent pool; returns the thread count in use. */
int cpb_set_threads(int threads) {
    if (threads < 1) threads = 1;
    if (g_pool && g_threads == threads) return threads;
    if (g_pool) pool_free(g_pool);
    g_pool = pool_new(threads);
    g_threads = threads;
    return threads;
}

static int run(int format, const uint8_t *w, uint64_t stored_rows, uint64_t stored_cols,
               const float *x, uint64_t m, uint64_t k, int int8, float *y) {
    if (k != stored_cols || k % 32 || !orc_supported(format)) return -1;
    if (format == ORC_Q4_K && k % 256) return -1;
    if (!g_pool) cpb_set_threads(1);
    job_t j;
    memset(&j, 0, sizeof j);
    j.format = format;
    j.int8 = int8;
    j.w = w;
    j.row_bytes = stored_cols / (uint64_t)orc_block_elements(format) * (uint64_t)orc_block_bytes(format);
    j.n = stored_rows;
    j.m = m;
    j.k = k;
    j.x = x;
    j.y = y;
    uint64_t per = (j.n + (uint64_t)g_threads * 4 - 1) / ((uint64_t)g_threads * 4);
    j.chunk = per < 8 ? 8 : per;
    int8_t *values = 0;
    float *scales = 0;
    int32_t *sums = 0;
    if (int8) {
        values = (int8_t *)malloc(m * k);
        scales = (float *)malloc(sizeof(float) * (m * k / 32));
        sums = (int32_t *)malloc(sizeof(int32_t) * 2 * (m * k / 32));
        orc_quantize_rows(x, m * k, values, scales, sums);
        j.q.values = values;
        j.q.scales = scales;
        j.q.sums = sums;
    }
    pool_run(g_pool, (j.n + j.chunk - 1) / j.chunk, task, &j);
    free(values);
    free(scales);
    free(sums);
    return 0;
}

/* The reference's default path: int8 activations, AVX2 kernels, pool. */
int cpb_packed_matmul(int format, const uint8_t *w, uint64_t stored_rows, uint64_t stored_cols,
                      const float *x, uint64_t m, uint64_t k, float *y) {
    return run(format, w, stored_rows, stored_cols, x, m, k, 1, y);
}

/* The f32-activation scalar path (MAGNETAR_CPU_INT8_ACTIVATIONS=0), pooled. */
int cpb_packed_matmul_f32(int format, const uint8_t *w, uint64_t stored_rows,
                          uint64_t stored_cols, const float *x, uint64_t m, uint64_t k, float *y) {
    return run(format, w, stored_rows, stored_cols, x, m, k, 0, y);
}
