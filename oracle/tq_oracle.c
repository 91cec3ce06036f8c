/*
 * tq_oracle.c — CPU restatement of tensai's weight-only quantized path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle the CUDA library is checked
 * against and the CPU baseline it is timed beside. Nothing in the product
 * (tensai_b200/, include/) links, loads or calls it.
 *
 * Every function restates one function of github.com/mattn/tensai (Go); the
 * citation is given as file:line within that project. The Go toolchain is not
 * available, so the reference itself cannot be built; parity of the codes is
 * pinned by restating the algorithm text exactly and by the reference's own
 * known-answer tests (quant_test.go, quant4_test.go), which the Python tests
 * port shape for shape.
 *
 * Numerics: build with -ffp-contract=off so the "generic" bodies round every
 * multiply and add separately, as gc does at GOAMD64=v1; the AVX2 bodies use
 * explicit _mm256_fmadd_ps where the Go kernels call MulAdd.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define TQO_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* Synthetic inputs. The same generator is implemented bit-for-bit on the   */
/* GPU (tensai_b200/csrc/tq_quantize.cu) so weights never have to ship.    */
/*   key   = splitmix64 state derived from (seed, stream)                   */
/*   elem i: h_j = mix(key + (3i+j)*gamma), j = 0..2                         */
/*           S   = sum of the twelve 16-bit fields of h_0..h_2              */
/*           v   = float(2S - 786420) * (sigma * 2^-17)                     */
/* 2S - 786420 is an exact integer below 2^20, so v takes a single IEEE     */
/* rounding (the multiply) on every device. The distribution is the         */
/* Irwin-Hall sum of 12 uniforms: mean 0, standard deviation sigma.         */
/* ------------------------------------------------------------------------ */
#define TQ_GAMMA 0x9E3779B97F4A7C15ull

static inline uint64_t tq_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

TQO_EXPORT uint64_t tqo_synth_key(uint64_t seed, uint64_t stream) {
    return tq_mix64(seed * TQ_GAMMA + 0x632BE59BD9B4E019ull) ^ tq_mix64((stream + 1) * 0xD1B54A32D192ED03ull);
}

static inline float tq_synth_one(uint64_t key, uint64_t i, float c) {
    int32_t s = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = tq_mix64(key + (3 * i + (uint64_t)j + 1) * TQ_GAMMA);
        s += (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
             (int32_t)(h >> 48);
    }
    return (float)(2 * s - 786420) * c;
}

/* ------------------------------------------------------------------------ */
/* A small persistent thread pool, standing in for the goroutine fan-out of */
/* quant.go:88-101 / quant4.go:107-117. The caller thread takes tasks too,  */
/* as a Go caller's P runs goroutines while it sits in wg.Wait().           */
/* ------------------------------------------------------------------------ */
typedef void (*tqo_task_fn)(void *arg, int idx);

static struct {
    int n; /* total threads including the caller */
    pthread_t th[256];
    pthread_mutex_t mu;
    pthread_cond_t cv;
    pthread_cond_t done_cv;
    tqo_task_fn fn;
    void *arg;
    int ntasks;
    atomic_int next;
    atomic_int done;
    unsigned gen;
    int started;
} g_pool = {.mu = PTHREAD_MUTEX_INITIALIZER, .cv = PTHREAD_COND_INITIALIZER, .done_cv = PTHREAD_COND_INITIALIZER};

static void pool_drain(void) {
    for (;;) {
        int idx = atomic_fetch_add(&g_pool.next, 1);
        if (idx >= g_pool.ntasks) break;
        g_pool.fn(g_pool.arg, idx);
        if (atomic_fetch_add(&g_pool.done, 1) + 1 == g_pool.ntasks) {
            pthread_mutex_lock(&g_pool.mu);
            pthread_cond_broadcast(&g_pool.done_cv);
            pthread_mutex_unlock(&g_pool.mu);
        }
    }
}

static void *pool_worker(void *unused) {
    (void)unused;
    unsigned seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_pool.mu);
        while (g_pool.gen == seen) pthread_cond_wait(&g_pool.cv, &g_pool.mu);
        seen = g_pool.gen;
        pthread_mutex_unlock(&g_pool.mu);
        pool_drain();
    }
    return NULL;
}

/* Sets the worker count (runtime.NumCPU() in the reference). 0 = nproc. */
TQO_EXPORT int tqo_set_threads(int n) {
    if (n <= 0) n = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (n > 256) n = 256;
    pthread_mutex_lock(&g_pool.mu);
    if (g_pool.started < n - 1) {
        for (int t = g_pool.started; t < n - 1; t++) pthread_create(&g_pool.th[t], NULL, pool_worker, NULL);
        g_pool.started = n - 1;
    }
    g_pool.n = n;
    pthread_mutex_unlock(&g_pool.mu);
    return n;
}

TQO_EXPORT int tqo_get_threads(void) {
    if (g_pool.n == 0) tqo_set_threads(0);
    return g_pool.n;
}

static void pool_run(tqo_task_fn fn, void *arg, int ntasks) {
    if (g_pool.n == 0) tqo_set_threads(0);
    if (ntasks <= 1 || g_pool.n <= 1) {
        for (int i = 0; i < ntasks; i++) fn(arg, i);
        return;
    }
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = fn;
    g_pool.arg = arg;
    g_pool.ntasks = ntasks;
    atomic_store(&g_pool.next, 0);
    atomic_store(&g_pool.done, 0);
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.cv);
    pthread_mutex_unlock(&g_pool.mu);
    pool_drain();
    pthread_mutex_lock(&g_pool.mu);
    while (atomic_load(&g_pool.done) < ntasks) pthread_cond_wait(&g_pool.done_cv, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
}

/* The pool for the model restatements (tq_model.c). */
TQO_EXPORT void tqo_pool_run(void (*fn)(void *arg, int idx), void *arg, int ntasks) { pool_run(fn, arg, ntasks); }

/* Fills out[0..n) from (seed, stream) with standard deviation sigma. The   */
/* value of element i depends only on (seed, stream, i), never on threads.  */
struct synth_job { float *out; size_t n; uint64_t key; float c; size_t per; };
static void synth_task(void *a, int t) {
    struct synth_job *j = a;
    size_t lo = (size_t)t * j->per, hi = lo + j->per;
    if (hi > j->n) hi = j->n;
    for (size_t i = lo; i < hi; i++) j->out[i] = tq_synth_one(j->key, i, j->c);
}
TQO_EXPORT void tqo_synth_fill(float *out, size_t n, uint64_t seed, uint64_t stream, float sigma) {
    struct synth_job j = {out, n, tqo_synth_key(seed, stream), sigma * 0x1p-17f, 1 << 16};
    int tasks = (int)((n + j.per - 1) / j.per);
    pool_run(synth_task, &j, tasks);
}

/* ------------------------------------------------------------------------ */
/* Quantizers.                                                              */
/* ------------------------------------------------------------------------ */

/* QuantizeMatrix, quant.go:37-72, for columns [lo, hi). Columns are        */
/* independent, so splitting them over threads cannot change a code.        */
static void quantize8_cols(const float *w, int rows, int cols, int8_t *q, float *scale, int lo, int hi) {
    for (int j = lo; j < hi; j++) {
        float maxAbs = 0;
        for (int i = 0; i < rows; i++) {
            float v = w[(size_t)i * cols + j];
            if (v < 0) v = -v;
            if (v > maxAbs) maxAbs = v;
        }
        float s = maxAbs / 127;
        scale[j] = s;
        if (s == 0) continue;
        float inv = 1 / s;
        for (int i = 0; i < rows; i++) {
            float v = w[(size_t)i * cols + j] * inv;
            if (v >= 0)
                v += 0.5f;
            else
                v -= 0.5f;
            q[(size_t)i * cols + j] = (int8_t)(int32_t)v; /* int8(v): truncation toward zero */
        }
    }
}

struct qz_job { const float *w; int rows, cols; void *q; float *scale; int per, limit; };
static void quantize8_task(void *a, int t) {
    struct qz_job *j = a;
    int lo = t * j->per, hi = lo + j->per < j->limit ? lo + j->per : j->limit;
    quantize8_cols(j->w, j->rows, j->cols, j->q, j->scale, lo, hi);
}

/* q must hold rows*cols+16 bytes (the pad of quant.go:41) and is zeroed     */
/* here; scale holds cols floats.                                           */
TQO_EXPORT void tqo_quantize8(const float *w, int rows, int cols, int8_t *q, float *scale) {
    memset(q, 0, (size_t)rows * cols + 16);
    struct qz_job j = {w, rows, cols, q, scale, 64, cols};
    pool_run(quantize8_task, &j, (cols + 63) / 64);
}

#define Q4_GROUP 64 /* q4Group, quant4.go:12 */

/* QuantizeMatrix4, quant4.go:28-89, for the column pairs [lo, hi): column  */
/* p and column half+p share byte column p, so one worker owns both.         */
static void quantize4_col(const float *w, int rows, int cols, uint8_t *q, float *scale, int j, uint8_t *nib) {
    int half = cols / 2;
    int groups = (rows + Q4_GROUP - 1) / Q4_GROUP;
    for (int g = 0; g < groups; g++) {
        int rlo = g * Q4_GROUP;
        int rhi = rlo + Q4_GROUP < rows ? rlo + Q4_GROUP : rows;
        float maxAbs = 0;
        for (int i = rlo; i < rhi; i++) {
            float v = w[(size_t)i * cols + j];
            if (v < 0) v = -v;
            if (v > maxAbs) maxAbs = v;
        }
        float s = maxAbs / 7;
        scale[(size_t)g * cols + j] = s;
        if (s == 0) {
            for (int i = rlo; i < rhi; i++) nib[i] = 8;
            continue;
        }
        float inv = 1 / s;
        for (int i = rlo; i < rhi; i++) {
            float v = w[(size_t)i * cols + j] * inv;
            if (v >= 0)
                v += 0.5f;
            else
                v -= 0.5f;
            int64_t n = (int64_t)v; /* int(v): truncation toward zero */
            if (n < -8)
                n = -8;
            else if (n > 7)
                n = 7;
            nib[i] = (uint8_t)(n + 8);
        }
    }
    for (int i = 0; i < rows; i++) {
        if (j < half)
            q[(size_t)i * half + j] |= nib[i];
        else
            q[(size_t)i * half + j - half] |= (uint8_t)(nib[i] << 4);
    }
}

static void quantize4_task(void *a, int t) {
    struct qz_job *j = a;
    int lo = t * j->per, hi = lo + j->per < j->limit ? lo + j->per : j->limit;
    uint8_t *nib = malloc(j->rows > 0 ? (size_t)j->rows : 1);
    int half = j->cols / 2;
    for (int p = lo; p < hi; p++) {
        quantize4_col(j->w, j->rows, j->cols, j->q, j->scale, p, nib);
        quantize4_col(j->w, j->rows, j->cols, j->q, j->scale, half + p, nib);
    }
    free(nib);
}

/* Returns -1 for an odd column count (quant4.go:29-31). q must hold         */
/* rows*cols/2+16 bytes (quant4.go:37); scale holds ceil(rows/64)*cols      */
/* floats, group-major (quant4.go:38).                                      */
TQO_EXPORT int tqo_quantize4(const float *w, int rows, int cols, uint8_t *q, float *scale) {
    if (cols % 2 != 0) return -1;
    memset(q, 0, (size_t)rows * (cols / 2) + 16);
    struct qz_job j = {w, rows, cols, q, scale, 32, cols / 2};
    pool_run(quantize4_task, &j, (cols / 2 + 31) / 32);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* int8 matvec bodies.                                                      */
/* ------------------------------------------------------------------------ */

/* qmatvecColsGeneric, quant.go:108-122: zero skip, separately rounded      */
/* multiply and add, column scale after all rows.                           */
static void q8_cols_generic(float *out, const float *x, int rows, const int8_t *qw, const float *scale, int cols,
                            int lo, int hi) {
    memset(out + lo, 0, sizeof(float) * (size_t)(hi - lo));
    for (int i = 0; i < rows; i++) {
        float xi = x[i];
        if (xi == 0) continue;
        const int8_t *row = qw + (size_t)i * cols;
        for (int j = lo; j < hi; j++) out[j] += xi * (float)row[j];
    }
    for (int j = lo; j < hi; j++) out[j] *= scale[j];
}

/* qmatvecCols (AVX2), quant_simd.go:12-48: per row, 8 int8 codes widened   */
/* and converted, fma(w, x[i], out) with no zero skip; 32- then 8-column    */
/* blocks; the column scale multiplies after all rows; the last (hi-lo)%8   */
/* columns go through the generic body (quant_simd.go:45-47).               */
static void q8_cols_avx2(float *out, const float *x, int rows, const int8_t *qw, const float *scale, int cols,
                         int lo, int hi) {
    int wide = lo + ((hi - lo) & ~31);
    int vecEnd = lo + ((hi - lo) & ~7);
    memset(out + lo, 0, sizeof(float) * (size_t)(hi - lo));
    if (vecEnd > lo) {
        for (int i = 0; i < rows; i++) {
            __m256 xv = _mm256_set1_ps(x[i]);
            const int8_t *row = qw + (size_t)i * cols;
            int j = lo;
            for (; j < wide; j += 32) {
                for (int u = 0; u < 32; u += 8) {
                    __m256 w = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(row + j + u))));
                    _mm256_storeu_ps(out + j + u, _mm256_fmadd_ps(w, xv, _mm256_loadu_ps(out + j + u)));
                }
            }
            for (; j < vecEnd; j += 8) {
                __m256 w = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(row + j))));
                _mm256_storeu_ps(out + j, _mm256_fmadd_ps(w, xv, _mm256_loadu_ps(out + j)));
            }
        }
        for (int j = lo; j < vecEnd; j += 8)
            _mm256_storeu_ps(out + j, _mm256_mul_ps(_mm256_loadu_ps(out + j), _mm256_loadu_ps(scale + j)));
    }
    if (vecEnd < hi) q8_cols_generic(out, x, rows, qw, scale, cols, vecEnd, hi);
}

/* ------------------------------------------------------------------------ */
/* int4 matvec bodies (column pairs [lo,hi) and [half+lo, half+hi)).        */
/* ------------------------------------------------------------------------ */

/* q4matvecColsGeneric, quant4.go:126-154. */
static void q4_cols_generic(float *out, const float *x, int rows, const uint8_t *qw, const float *scale, int cols,
                            int lo, int hi, float *tmp) {
    int half = cols / 2;
    memset(out + lo, 0, sizeof(float) * (size_t)(hi - lo));
    memset(out + half + lo, 0, sizeof(float) * (size_t)(hi - lo));
    int groups = (rows + Q4_GROUP - 1) / Q4_GROUP;
    for (int g = 0; g < groups; g++) {
        int rlo = g * Q4_GROUP;
        int rhi = rlo + Q4_GROUP < rows ? rlo + Q4_GROUP : rows;
        memset(tmp + lo, 0, sizeof(float) * (size_t)(hi - lo));
        memset(tmp + half + lo, 0, sizeof(float) * (size_t)(hi - lo));
        for (int i = rlo; i < rhi; i++) {
            float xi = x[i];
            if (xi == 0) continue;
            const uint8_t *row = qw + (size_t)i * half;
            for (int j = lo; j < hi; j++) {
                uint8_t b = row[j];
                tmp[j] += xi * (float)((int)(b & 0x0F) - 8);
                tmp[half + j] += xi * (float)((int)(b >> 4) - 8);
            }
        }
        const float *srow = scale + (size_t)g * cols;
        for (int j = lo; j < hi; j++) {
            out[j] += tmp[j] * srow[j];
            out[half + j] += tmp[half + j] * srow[half + j];
        }
    }
}

/* q4matvecCols (AVX2), quant4_simd.go:17-57: 8 column pairs per step, low  */
/* nibble by mask, high nibble by a 16-bit shift then mask, each widened,   */
/* converted and reduced by 8.0; fma into tmp; at each group end            */
/* out = fma(tmp, scale, out); the last (hi-lo)%8 pairs go generic.         */
static void q4_cols_avx2(float *out, const float *x, int rows, const uint8_t *qw, const float *scale, int cols,
                         int lo, int hi, float *tmp) {
    int half = cols / 2;
    int vecEnd = lo + ((hi - lo) & ~7);
    if (vecEnd > lo) {
        const __m128i mask = _mm_set1_epi8(0x0F);
        const __m256 eight = _mm256_set1_ps(8);
        memset(out + lo, 0, sizeof(float) * (size_t)(vecEnd - lo));
        memset(out + half + lo, 0, sizeof(float) * (size_t)(vecEnd - lo));
        int groups = (rows + Q4_GROUP - 1) / Q4_GROUP;
        for (int g = 0; g < groups; g++) {
            int rlo = g * Q4_GROUP;
            int rhi = rlo + Q4_GROUP < rows ? rlo + Q4_GROUP : rows;
            memset(tmp + lo, 0, sizeof(float) * (size_t)(vecEnd - lo));
            memset(tmp + half + lo, 0, sizeof(float) * (size_t)(vecEnd - lo));
            for (int i = rlo; i < rhi; i++) {
                __m256 xv = _mm256_set1_ps(x[i]);
                const uint8_t *row = qw + (size_t)i * half;
                for (int j = lo; j < vecEnd; j += 8) {
                    __m128i v = _mm_loadl_epi64((const __m128i *)(row + j));
                    __m256 loN = _mm256_sub_ps(_mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_and_si128(v, mask))), eight);
                    __m256 hiN = _mm256_sub_ps(
                        _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_and_si128(_mm_srli_epi16(v, 4), mask))), eight);
                    _mm256_storeu_ps(tmp + j, _mm256_fmadd_ps(loN, xv, _mm256_loadu_ps(tmp + j)));
                    _mm256_storeu_ps(tmp + half + j, _mm256_fmadd_ps(hiN, xv, _mm256_loadu_ps(tmp + half + j)));
                }
            }
            const float *srow = scale + (size_t)g * cols;
            for (int j = lo; j < vecEnd; j += 8) {
                _mm256_storeu_ps(out + j, _mm256_fmadd_ps(_mm256_loadu_ps(tmp + j), _mm256_loadu_ps(srow + j),
                                                          _mm256_loadu_ps(out + j)));
                _mm256_storeu_ps(out + half + j,
                                 _mm256_fmadd_ps(_mm256_loadu_ps(tmp + half + j), _mm256_loadu_ps(srow + half + j),
                                                 _mm256_loadu_ps(out + half + j)));
            }
        }
    }
    if (vecEnd < hi) q4_cols_generic(out, x, rows, qw, scale, cols, vecEnd, hi, tmp);
}

/* ------------------------------------------------------------------------ */
/* MatVec drivers: shape is checked by the caller (the Python/host mirror   */
/* returns the reference's error); here only the worker split.              */
/* ------------------------------------------------------------------------ */

/* matvecWorkerCount, quant.go:13-22. */
static int worker_count(int cols, int rows) {
    if ((long long)cols * rows < (1 << 20)) return 1;
    int w = tqo_get_threads();
    if (w > cols) w = cols;
    return w;
}

enum { TQO_GENERIC = 0, TQO_AVX2 = 1 };

struct mv_job {
    int bits, variant, rows, cols, chunk, limit;
    const float *x;
    float *out;
    const void *q;
    const float *scale;
};

static void mv_task(void *a, int t) {
    struct mv_job *j = a;
    int lo = t * j->chunk, hi = lo + j->chunk;
    if (hi > j->limit) hi = j->limit;
    if (j->bits == 8) {
        if (j->variant == TQO_AVX2)
            q8_cols_avx2(j->out, j->x, j->rows, j->q, j->scale, j->cols, lo, hi);
        else
            q8_cols_generic(j->out, j->x, j->rows, j->q, j->scale, j->cols, lo, hi);
    } else {
        /* quant4.go:101 gives every worker a fresh zeroed tmp of Cols floats. */
        float *tmp = calloc((size_t)j->cols > 0 ? (size_t)j->cols : 1, sizeof(float));
        if (j->variant == TQO_AVX2)
            q4_cols_avx2(j->out, j->x, j->rows, j->q, j->scale, j->cols, lo, hi, tmp);
        else
            q4_cols_generic(j->out, j->x, j->rows, j->q, j->scale, j->cols, lo, hi, tmp);
        free(tmp);
    }
}

static void matvec(int bits, int variant, const void *q, const float *scale, int rows, int cols, const float *x,
                   float *out) {
    /* int8 splits columns (quant.go:82-101); int4 splits column pairs      */
    /* (quant4.go:99-117). Chunks are rounded up to a multiple of 8.        */
    int limit = bits == 8 ? cols : cols / 2;
    int workers = worker_count(limit, rows);
    struct mv_job j = {bits, variant, rows, cols, limit, limit, x, out, q, scale};
    if (workers == 1) {
        mv_task(&j, 0);
        return;
    }
    j.chunk = ((limit + workers - 1) / workers + 7) & ~7;
    int tasks = (limit + j.chunk - 1) / j.chunk;
    pool_run(mv_task, &j, tasks);
}

/* (*QMatrix).MatVec, quant.go:77-103, applied to m activation rows in turn */
/* (the reference has no batched call: m rows are m MatVec calls).          */
TQO_EXPORT void tqo_q8_matmul(const int8_t *q, const float *scale, int rows, int cols, const float *x, float *out,
                              int m, int variant) {
    for (int r = 0; r < m; r++)
        matvec(8, variant, q, scale, rows, cols, x + (size_t)r * rows, out + (size_t)r * cols);
}

/* (*Q4Matrix).MatVec, quant4.go:93-119, applied to m rows in turn. */
TQO_EXPORT void tqo_q4_matmul(const uint8_t *q, const float *scale, int rows, int cols, const float *x, float *out,
                              int m, int variant) {
    for (int r = 0; r < m; r++)
        matvec(4, variant, q, scale, rows, cols, x + (size_t)r * rows, out + (size_t)r * cols);
}
