/*
 * tq_model.c — CPU restatement of tensai's GPT-2 example decode loop with
 * int8 weights (_example/gpt2/model.go, main.go).
 *
 * TEST INFRASTRUCTURE ONLY: it produces the golden greedy token ids the GPU
 * decode engine must reproduce, and is never linked by the product.
 *
 * Numerics follow the Go source statement by statement, built with
 * -ffp-contract=off (gc at GOAMD64=v1 fuses nothing): layer norm statistics,
 * attention scores, softmax and GELU in float64; residual, bias and the
 * attention-weighted sum in float32 with separate multiply and add; prefill
 * matmuls as tensai's AVX2 dotRows (one fused multiply-add chain per output
 * element over k in order, zero activations skipped); decode matvecs as
 * (*QMatrix).MatVec on the AVX2 kernel (tq_oracle.c); greedy argmax with a
 * strict > (ties to the lowest id).
 *
 * Random-init model (no checkpoint): every matrix and embedding is drawn
 * from the shared seeded generator with standard deviation sigma; layer norm
 * weights are 1 and every bias is 0. Generator streams: wte 1, wpe 2, layer
 * l: c_attn 16+8l, attn c_proj 17+8l, mlp c_fc 18+8l, mlp c_proj 19+8l.
 */
#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "tq_oracle.h"

enum { TQO_AVX2_VARIANT = 1 };

typedef struct {
    int n_layer, n_head, d, ffn, vocab, ctx;
} tqo_gpt2_cfg;

typedef struct {
    float *w;      /* fp32 [rows][cols] (prefill) */
    int8_t *q;     /* QuantizeMatrix codes (+16 pad bytes) */
    float *scale;  /* per column */
    int rows, cols;
} qmat;

typedef struct {
    qmat attn, proj, fc, fc2;
    float *ln1w, *ln1b, *ln2w, *ln2b, *attnB, *projB, *fcB, *fc2B;
    float *kc, *vc; /* [ctx][d] */
} g2block;

typedef struct {
    tqo_gpt2_cfg c;
    float *wte, *wpe, *lnfw, *lnfb;
    qmat wteT;
    g2block *b;
} gpt2;

static float *zeros(size_t n) { return calloc(n ? n : 1, sizeof(float)); }
static float *ones(size_t n) {
    float *p = malloc((n ? n : 1) * sizeof(float));
    for (size_t i = 0; i < n; i++) p[i] = 1.0f;
    return p;
}

static void qmat_init(qmat *m, float *w, int rows, int cols) {
    m->w = w;
    m->rows = rows;
    m->cols = cols;
    m->q = calloc((size_t)rows * cols + 16, 1);
    m->scale = zeros((size_t)cols);
    tqo_quantize8(w, rows, cols, m->q, m->scale); /* gpt2.quantize, model.go:51-60 */
}

static void qmat_free(qmat *m) {
    free(m->w);
    free(m->q);
    free(m->scale);
}

/* layernorm, model.go:135-153. */
static void layernorm(const float *x, const float *w, const float *b, int n, float *out) {
    double mean = 0;
    for (int i = 0; i < n; i++) mean += (double)x[i];
    mean /= (double)n;
    double var = 0;
    for (int i = 0; i < n; i++) {
        double d = (double)x[i] - mean;
        var += d * d;
    }
    var /= (double)n;
    double inv = 1 / sqrt(var + 1e-5);
    for (int i = 0; i < n; i++) out[i] = (float)(((double)x[i] - mean) * inv) * w[i] + b[i];
}

/* geluNew, model.go:170-175. */
static void gelu_new(float *x, int n) {
    for (int i = 0; i < n; i++) {
        double f = x[i];
        x[i] = (float)(0.5 * f * (1 + tanh(0.7978845608028654 * (f + 0.044715 * f * f * f))));
    }
}

/* dotRows (dot_simd.go:23-79): out[r][c] = fma chain over k in order with */
/* the activation a[r][k] broadcast; zero activations are skipped; the     */
/* first product is a plain multiply. Rows are split over the pool as     */
/* DotInto (tensor.go:106-136) does; the split never changes results.     */
struct dot_job {
    const float *a, *b;
    float *out;
    int inner, cols;
};
static void dot_row_task(void *arg, int r) {
    struct dot_job *j = arg;
    const float *ar = j->a + (size_t)r * j->inner;
    float *o = j->out + (size_t)r * j->cols;
    int init = 0;
    for (int k = 0; k < j->inner; k++) {
        if (ar[k] == 0.0f) continue;
        const float *br = j->b + (size_t)k * j->cols;
        const __m256 vv = _mm256_set1_ps(ar[k]);
        int c = 0;
        if (!init) {
            for (; c + 8 <= j->cols; c += 8) _mm256_storeu_ps(o + c, _mm256_mul_ps(_mm256_loadu_ps(br + c), vv));
            for (; c < j->cols; c++) o[c] = br[c] * ar[k];
            init = 1;
            continue;
        }
        for (; c + 8 <= j->cols; c += 8)
            _mm256_storeu_ps(o + c, _mm256_fmadd_ps(_mm256_loadu_ps(br + c), vv, _mm256_loadu_ps(o + c)));
        for (; c < j->cols; c++) o[c] = fmaf(br[c], ar[k], o[c]);
    }
    if (!init) memset(o, 0, sizeof(float) * (size_t)j->cols);
}
static void dot(const float *a, int rows, int inner, const float *b, int cols, float *out) {
    struct dot_job j = {a, b, out, inner, cols};
    tqo_pool_run(dot_row_task, &j, rows);
}

static void add_bias(float *x, const float *b, int n) {
    for (int i = 0; i < n; i++) x[i] += b[i];
}

/* One query row over cached positions 0..steps-1 of one block's KV cache   */
/* (step attention, model.go:195-227; cpuCausalMHA row, model.go:289-322). */
struct attn_job {
    const float *q; /* [d] */
    const float *kc, *vc; /* [steps][kv stride] */
    float *out; /* [d], zeroed */
    int steps, d, hd, stride;
};
static void attn_head_task(void *arg, int h) {
    struct attn_job *j = arg;
    const int off = h * j->hd;
    double *scores = malloc(sizeof(double) * (size_t)(j->steps > 0 ? j->steps : 1));
    double maxs = -INFINITY;
    for (int t = 0; t < j->steps; t++) {
        double s = 0;
        const float *kt = j->kc + (size_t)t * j->stride;
        for (int i = 0; i < j->hd; i++) s += (double)j->q[off + i] * (double)kt[off + i];
        s /= 8; /* sqrt(headSz) */
        scores[t] = s;
        if (s > maxs) maxs = s;
    }
    double sum = 0;
    for (int t = 0; t < j->steps; t++) {
        scores[t] = exp(scores[t] - maxs);
        sum += scores[t];
    }
    for (int t = 0; t < j->steps; t++) {
        const float p = (float)(scores[t] / sum);
        const float *vt = j->vc + (size_t)t * j->stride;
        for (int i = 0; i < j->hd; i++) j->out[off + i] += p * vt[off + i];
    }
    free(scores);
}

static void attention(const gpt2 *m, const float *q, const float *kc, const float *vc, int steps, float *out) {
    const int d = m->c.d;
    memset(out, 0, sizeof(float) * (size_t)d);
    struct attn_job j = {q, kc, vc, out, steps, d, d / m->c.n_head, d};
    tqo_pool_run(attn_head_task, &j, m->c.n_head);
}

/* step, model.go:179-245 (int8 decode). */
static void gpt2_step(gpt2 *m, int token, int pos, float *logits) {
    const int d = m->c.d, ffn = m->c.ffn;
    float *x = malloc(sizeof(float) * d), *xn = malloc(sizeof(float) * d), *qkv = malloc(sizeof(float) * 3 * d);
    float *attn = malloc(sizeof(float) * d), *proj = malloc(sizeof(float) * d), *h = malloc(sizeof(float) * ffn);
    for (int i = 0; i < d; i++) x[i] = m->wte[(size_t)token * d + i] + m->wpe[(size_t)pos * d + i];
    for (int l = 0; l < m->c.n_layer; l++) {
        g2block *b = &m->b[l];
        layernorm(x, b->ln1w, b->ln1b, d, xn);
        tqo_q8_matmul(b->attn.q, b->attn.scale, d, 3 * d, xn, qkv, 1, TQO_AVX2_VARIANT);
        add_bias(qkv, b->attnB, 3 * d);
        memcpy(b->kc + (size_t)pos * d, qkv + d, sizeof(float) * d);
        memcpy(b->vc + (size_t)pos * d, qkv + 2 * d, sizeof(float) * d);
        attention(m, qkv, b->kc, b->vc, pos + 1, attn);
        tqo_q8_matmul(b->proj.q, b->proj.scale, d, d, attn, proj, 1, TQO_AVX2_VARIANT);
        add_bias(proj, b->projB, d);
        for (int i = 0; i < d; i++) x[i] += proj[i];
        layernorm(x, b->ln2w, b->ln2b, d, xn);
        tqo_q8_matmul(b->fc.q, b->fc.scale, d, ffn, xn, h, 1, TQO_AVX2_VARIANT);
        add_bias(h, b->fcB, ffn);
        gelu_new(h, ffn);
        tqo_q8_matmul(b->fc2.q, b->fc2.scale, ffn, d, h, proj, 1, TQO_AVX2_VARIANT);
        add_bias(proj, b->fc2B, d);
        for (int i = 0; i < d; i++) x[i] += proj[i];
    }
    layernorm(x, m->lnfw, m->lnfb, d, xn);
    tqo_q8_matmul(m->wteT.q, m->wteT.scale, d, m->c.vocab, xn, logits, 1, TQO_AVX2_VARIANT);
    free(x), free(xn), free(qkv), free(attn), free(proj), free(h);
}

/* prefill, model.go:361-401 (fp32 weights, one batched pass). */
static void gpt2_prefill(gpt2 *m, const int *tokens, int T, float *logits) {
    const int d = m->c.d, ffn = m->c.ffn;
    float *x = malloc(sizeof(float) * (size_t)T * d), *xn = malloc(sizeof(float) * (size_t)T * d);
    float *qkv = malloc(sizeof(float) * (size_t)T * 3 * d), *q = malloc(sizeof(float) * (size_t)T * d);
    float *attn = malloc(sizeof(float) * (size_t)T * d), *y = malloc(sizeof(float) * (size_t)T * d);
    float *h = malloc(sizeof(float) * (size_t)T * ffn);
    for (int t = 0; t < T; t++)
        for (int i = 0; i < d; i++) x[(size_t)t * d + i] = m->wte[(size_t)tokens[t] * d + i] + m->wpe[(size_t)t * d + i];
    for (int l = 0; l < m->c.n_layer; l++) {
        g2block *b = &m->b[l];
        for (int t = 0; t < T; t++) layernorm(x + (size_t)t * d, b->ln1w, b->ln1b, d, xn + (size_t)t * d);
        dot(xn, T, d, b->attn.w, 3 * d, qkv);
        for (int t = 0; t < T; t++) {
            float *row = qkv + (size_t)t * 3 * d;
            add_bias(row, b->attnB, 3 * d);
            memcpy(q + (size_t)t * d, row, sizeof(float) * d);
            memcpy(b->kc + (size_t)t * d, row + d, sizeof(float) * d);
            memcpy(b->vc + (size_t)t * d, row + 2 * d, sizeof(float) * d);
        }
        for (int t = 0; t < T; t++) attention(m, q + (size_t)t * d, b->kc, b->vc, t + 1, attn + (size_t)t * d);
        dot(attn, T, d, b->proj.w, d, y);
        for (int t = 0; t < T; t++) add_bias(y + (size_t)t * d, b->projB, d);
        for (size_t i = 0; i < (size_t)T * d; i++) x[i] += y[i];
        for (int t = 0; t < T; t++) layernorm(x + (size_t)t * d, b->ln2w, b->ln2b, d, xn + (size_t)t * d);
        dot(xn, T, d, b->fc.w, ffn, h);
        for (int t = 0; t < T; t++) add_bias(h + (size_t)t * ffn, b->fcB, ffn);
        gelu_new(h, T * ffn);
        dot(h, T, ffn, b->fc2.w, d, y);
        for (int t = 0; t < T; t++) add_bias(y + (size_t)t * d, b->fc2B, d);
        for (size_t i = 0; i < (size_t)T * d; i++) x[i] += y[i];
    }
    layernorm(x + (size_t)(T - 1) * d, m->lnfw, m->lnfb, d, xn);
    dot(xn, 1, d, m->wteT.w, m->c.vocab, logits);
    free(x), free(xn), free(qkv), free(q), free(attn), free(y), free(h);
}

/* sample at temperature 0, main.go:69-77: strict >, ties to the lowest id. */
static int argmax(const float *v, int n, float *margin) {
    int best = 0;
    for (int i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    float second = -INFINITY;
    for (int i = 0; i < n; i++)
        if (i != best && v[i] > second) second = v[i];
    if (margin) *margin = v[best] - second;
    return best;
}

/* The examples' sample step (_example/gpt2/main.go:78-105 and
 * _example/qwen/main.go:115-150 are the same function): temp <= 0 is the
 * greedy scan; otherwise p_i = exp(float64(v_i - maxl) / temp) (the
 * difference in float32, as Go evaluates v-maxl), the sum in index order,
 * the candidates sorted by p descending, r = u * sum and the first
 * candidate at which r -= p reaches <= 0, else the first candidate. u is
 * the caller's rng.Float64(). Go's sort.Slice is not stable: among equal p
 * it leaves the order to its pattern-defeating quicksort, so here ties go to
 * the lower id (a choice, not Go's). */
typedef struct {
    double p;
    int id;
} tqo_cand;
static int cand_cmp(const void *a, const void *b) {
    const tqo_cand *x = a, *y = b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->id > y->id) - (x->id < y->id);
}
TQO_EXPORT int tqo_sample(const float *logits, int n, double temp, double u) {
    if (n <= 0) return -1;
    if (temp <= 0) {
        int best = 0;
        for (int i = 0; i < n; i++)
            if (logits[i] > logits[best]) best = i;
        return best;
    }
    tqo_cand *c = malloc(sizeof(tqo_cand) * (size_t)n);
    float maxl = logits[0];
    for (int i = 0; i < n; i++)
        if (logits[i] > maxl) maxl = logits[i];
    double sum = 0;
    for (int i = 0; i < n; i++) {
        const float d = logits[i] - maxl;
        c[i].p = exp((double)d / temp);
        c[i].id = i;
        sum += c[i].p;
    }
    qsort(c, (size_t)n, sizeof(tqo_cand), cand_cmp);
    double r = u * sum;
    int id = c[0].id;
    for (int i = 0; i < n; i++) {
        r -= c[i].p;
        if (r <= 0) {
            id = c[i].id;
            break;
        }
    }
    free(c);
    return id;
}

static float *synth(size_t n, uint64_t seed, uint64_t stream, float sigma) {
    float *p = malloc(sizeof(float) * (n ? n : 1));
    tqo_synth_fill(p, n, seed, stream, sigma);
    return p;
}

static gpt2 *gpt2_new(const tqo_gpt2_cfg *c, uint64_t seed, float sigma) {
    gpt2 *m = calloc(1, sizeof(gpt2));
    m->c = *c;
    const int d = c->d, ffn = c->ffn;
    m->wte = synth((size_t)c->vocab * d, seed, 1, sigma);
    m->wpe = synth((size_t)c->ctx * d, seed, 2, sigma);
    m->lnfw = ones(d);
    m->lnfb = zeros(d);
    float *wt = malloc(sizeof(float) * (size_t)d * c->vocab); /* wteT = wte^T, model.go:122 */
    for (int v = 0; v < c->vocab; v++)
        for (int i = 0; i < d; i++) wt[(size_t)i * c->vocab + v] = m->wte[(size_t)v * d + i];
    qmat_init(&m->wteT, wt, d, c->vocab);
    m->b = calloc((size_t)c->n_layer, sizeof(g2block));
    for (int l = 0; l < c->n_layer; l++) {
        g2block *b = &m->b[l];
        const uint64_t s0 = 16 + 8 * (uint64_t)l;
        qmat_init(&b->attn, synth((size_t)d * 3 * d, seed, s0, sigma), d, 3 * d);
        qmat_init(&b->proj, synth((size_t)d * d, seed, s0 + 1, sigma), d, d);
        qmat_init(&b->fc, synth((size_t)d * ffn, seed, s0 + 2, sigma), d, ffn);
        qmat_init(&b->fc2, synth((size_t)ffn * d, seed, s0 + 3, sigma), ffn, d);
        b->ln1w = ones(d), b->ln2w = ones(d);
        b->ln1b = zeros(d), b->ln2b = zeros(d);
        b->attnB = zeros(3 * d), b->projB = zeros(d), b->fcB = zeros(ffn), b->fc2B = zeros(d);
        b->kc = zeros((size_t)c->ctx * d);
        b->vc = zeros((size_t)c->ctx * d);
    }
    return m;
}

static void gpt2_free(gpt2 *m) {
    free(m->wte), free(m->wpe), free(m->lnfw), free(m->lnfb);
    qmat_free(&m->wteT);
    for (int l = 0; l < m->c.n_layer; l++) {
        g2block *b = &m->b[l];
        qmat_free(&b->attn), qmat_free(&b->proj), qmat_free(&b->fc), qmat_free(&b->fc2);
        free(b->ln1w), free(b->ln2w), free(b->ln1b), free(b->ln2b);
        free(b->attnB), free(b->projB), free(b->fcB), free(b->fc2B), free(b->kc), free(b->vc);
    }
    free(m->b);
    free(m);
}

/*
 * The generation loop of main.go:163-170 at temperature 0: prefill the
 * prompt, then n_gen times pick the argmax and feed it back. tokens[i] is
 * the i-th generated id; margins[i] its logit lead over the runner-up;
 * first_logits (optional, vocab floats) the prefill logits; seconds
 * (optional, 2 doubles) the wall time of the prefill and of the n_gen - 1
 * decode steps. Returns 0, or -1 on bad arguments.
 */
static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

TQO_EXPORT int tqo_gpt2_generate(const tqo_gpt2_cfg *c, uint64_t seed, float sigma, const int *prompt, int n_prompt,
                                 int n_gen, int *tokens, float *margins, float *first_logits, double *seconds) {
    /* the attention scale is the reference's literal 1/8 = 1/sqrt(64) */
    if (!c || n_prompt < 1 || n_prompt + n_gen > c->ctx + 1 || c->d % c->n_head || c->d / c->n_head != 64) return -1;
    gpt2 *m = gpt2_new(c, seed, sigma);
    float *logits = malloc(sizeof(float) * (size_t)c->vocab);
    const double t0 = now_s();
    gpt2_prefill(m, prompt, n_prompt, logits);
    const double t1 = now_s();
    if (first_logits) memcpy(first_logits, logits, sizeof(float) * (size_t)c->vocab);
    int pos = n_prompt;
    for (int i = 0; i < n_gen; i++) {
        const int next = argmax(logits, c->vocab, margins ? &margins[i] : NULL);
        tokens[i] = next;
        if (i + 1 < n_gen) gpt2_step(m, next, pos++, logits);
    }
    if (seconds) seconds[0] = t1 - t0, seconds[1] = now_s() - t1; /* prefill, decode steps */
    free(logits);
    gpt2_free(m);
    return 0;
}

/* Seeded uniform token ids in [0, vocab): id i = mix64(key + (i+1)*gamma) %
 * vocab, key from (seed, stream 3); the same rule as tq_synth_tokens in the
 * CUDA library. Stands in for a tokenized prompt. */
TQO_EXPORT void tqo_synth_tokens(int *out, int n, int vocab, uint64_t seed) {
    uint64_t key = tqo_synth_key(seed, 3);
    for (int i = 0; i < n; i++) {
        uint64_t z = key + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        out[i] = (int)(z % (uint64_t)vocab);
    }
}

/* ======================================================================== */
/* Qwen2 (_example/qwen/model.go:182-307, main.go:225-240) with int4        */
/* (QuantizeMatrix4) weights: RMSNorm, half-split RoPE, grouped-query       */
/* attention, SwiGLU, untied lm head; the prompt is fed token by token      */
/* through step, as main.go:229-231 does. Random init: matrices in the     */
/* reference's [in, out] orientation from the shared generator (embed 1,    */
/* lm head 2, layer l: q 32+16l, k +1, v +2, o +3, gate +4, up +5, down +6),  */
/* norm weights 1, biases 0.                                                */
/* ======================================================================== */

typedef struct {
    int n_layer, n_head, n_kv, d, ffn, vocab, ctx;
    double eps, theta;
} tqo_qwen_cfg;

typedef struct {
    uint8_t *q; /* QuantizeMatrix4 codes (+16 pad) */
    float *scale;
    int rows, cols;
} q4mat;

typedef struct {
    q4mat wq, wk, wv, wo, gate, up, down;
    float *ln1, *ln2, *bq, *bk, *bv;
    float *kc, *vc; /* [ctx][n_kv * hd] */
} qwblock;

typedef struct {
    tqo_qwen_cfg c;
    int hd, kvd;
    float *embed, *normw;
    q4mat lm;
    qwblock *b;
} qwen;

static void q4_init(q4mat *m, uint64_t seed, uint64_t stream, float sigma, int rows, int cols) {
    float *w = synth((size_t)rows * cols, seed, stream, sigma);
    m->rows = rows, m->cols = cols;
    m->q = calloc((size_t)rows * (cols / 2) + 16, 1);
    m->scale = zeros((size_t)((rows + 63) / 64) * cols);
    tqo_quantize4(w, rows, cols, m->q, m->scale); /* quantizeMat(.., 4), model.go:40-52 */
    free(w);
}

static void q4_mv(const q4mat *m, const float *x, float *out) {
    tqo_q4_matmul(m->q, m->scale, m->rows, m->cols, x, out, 1, TQO_AVX2_VARIANT);
}

/* rmsnorm, model.go:182-193. */
static void rmsnorm(const float *x, const float *w, int n, double eps, float *out) {
    double ss = 0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    double inv = 1 / sqrt(ss / (double)n + eps);
    for (int i = 0; i < n; i++) out[i] = (float)((double)x[i] * inv) * w[i];
}

/* rope, model.go:219-229: rotate pairs (i, i + hd/2) of one head. */
static void rope(float *h, int hd, int pos, double theta) {
    const int half = hd / 2;
    for (int i = 0; i < half; i++) {
        double freq = pow(theta, -2 * (double)i / (double)hd);
        double s = sin((double)pos * freq), c = cos((double)pos * freq);
        double a = h[i], b = h[i + half];
        h[i] = (float)(a * c - b * s);
        h[i + half] = (float)(b * c + a * s);
    }
}

struct gqa_job {
    const float *q, *kc, *vc;
    float *out;
    int steps, hd, kvd, group;
    double scale;
};
static void gqa_head_task(void *arg, int h) {
    struct gqa_job *j = arg;
    const int qoff = h * j->hd, kvoff = (h / j->group) * j->hd;
    double *scores = malloc(sizeof(double) * (size_t)(j->steps > 0 ? j->steps : 1));
    double maxs = -INFINITY;
    for (int t = 0; t < j->steps; t++) {
        double s = 0;
        const float *kt = j->kc + (size_t)t * j->kvd;
        for (int i = 0; i < j->hd; i++) s += (double)j->q[qoff + i] * (double)kt[kvoff + i];
        s *= j->scale;
        scores[t] = s;
        if (s > maxs) maxs = s;
    }
    double sum = 0;
    for (int t = 0; t < j->steps; t++) {
        scores[t] = exp(scores[t] - maxs);
        sum += scores[t];
    }
    for (int t = 0; t < j->steps; t++) {
        const float p = (float)(scores[t] / sum);
        const float *vt = j->vc + (size_t)t * j->kvd;
        for (int i = 0; i < j->hd; i++) j->out[qoff + i] += p * vt[kvoff + i];
    }
    free(scores);
}

/* step, model.go:232-307. */
static void qwen_step(qwen *m, int token, int pos, float *logits) {
    const tqo_qwen_cfg *c = &m->c;
    const int d = c->d, hd = m->hd, kvd = m->kvd, ffn = c->ffn;
    float *x = malloc(sizeof(float) * d), *a = malloc(sizeof(float) * d), *q = malloc(sizeof(float) * d);
    float *k = malloc(sizeof(float) * kvd), *v = malloc(sizeof(float) * kvd), *attn = malloc(sizeof(float) * d);
    float *proj = malloc(sizeof(float) * d), *gate = malloc(sizeof(float) * ffn), *up = malloc(sizeof(float) * ffn);
    memcpy(x, m->embed + (size_t)token * d, sizeof(float) * d);
    for (int l = 0; l < c->n_layer; l++) {
        qwblock *b = &m->b[l];
        rmsnorm(x, b->ln1, d, c->eps, a);
        q4_mv(&b->wq, a, q), add_bias(q, b->bq, d);
        q4_mv(&b->wk, a, k), add_bias(k, b->bk, kvd);
        q4_mv(&b->wv, a, v), add_bias(v, b->bv, kvd);
        for (int h = 0; h < c->n_head; h++) rope(q + h * hd, hd, pos, c->theta);
        for (int h = 0; h < c->n_kv; h++) rope(k + h * hd, hd, pos, c->theta);
        memcpy(b->kc + (size_t)pos * kvd, k, sizeof(float) * kvd);
        memcpy(b->vc + (size_t)pos * kvd, v, sizeof(float) * kvd);
        memset(attn, 0, sizeof(float) * d);
        struct gqa_job j = {q, b->kc, b->vc, attn, pos + 1, hd, kvd, c->n_head / c->n_kv, 1 / sqrt((double)hd)};
        tqo_pool_run(gqa_head_task, &j, c->n_head);
        q4_mv(&b->wo, attn, proj);
        for (int i = 0; i < d; i++) x[i] += proj[i];
        rmsnorm(x, b->ln2, d, c->eps, a);
        q4_mv(&b->gate, a, gate);
        q4_mv(&b->up, a, up);
        for (int i = 0; i < ffn; i++) {
            double g = gate[i];
            gate[i] = (float)(g / (1 + exp(-g))) * up[i]; /* silu(gate) * up */
        }
        q4_mv(&b->down, gate, proj);
        for (int i = 0; i < d; i++) x[i] += proj[i];
    }
    rmsnorm(x, m->normw, d, c->eps, a);
    q4_mv(&m->lm, a, logits);
    free(x), free(a), free(q), free(k), free(v), free(attn), free(proj), free(gate), free(up);
}

static qwen *qwen_new(const tqo_qwen_cfg *c, uint64_t seed, float sigma) {
    qwen *m = calloc(1, sizeof(qwen));
    m->c = *c;
    m->hd = c->d / c->n_head;
    m->kvd = c->n_kv * m->hd;
    const int d = c->d, kvd = m->kvd, ffn = c->ffn;
    m->embed = synth((size_t)c->vocab * d, seed, 1, sigma);
    m->normw = ones(d);
    q4_init(&m->lm, seed, 2, sigma, d, c->vocab);
    m->b = calloc((size_t)c->n_layer, sizeof(qwblock));
    for (int l = 0; l < c->n_layer; l++) {
        qwblock *b = &m->b[l];
        const uint64_t s0 = 32 + 16 * (uint64_t)l;
        q4_init(&b->wq, seed, s0, sigma, d, d);
        q4_init(&b->wk, seed, s0 + 1, sigma, d, kvd);
        q4_init(&b->wv, seed, s0 + 2, sigma, d, kvd);
        q4_init(&b->wo, seed, s0 + 3, sigma, d, d);
        q4_init(&b->gate, seed, s0 + 4, sigma, d, ffn);
        q4_init(&b->up, seed, s0 + 5, sigma, d, ffn);
        q4_init(&b->down, seed, s0 + 6, sigma, ffn, d);
        b->ln1 = ones(d), b->ln2 = ones(d);
        b->bq = zeros(d), b->bk = zeros(kvd), b->bv = zeros(kvd);
        b->kc = zeros((size_t)c->ctx * kvd);
        b->vc = zeros((size_t)c->ctx * kvd);
    }
    return m;
}

static void q4_free(q4mat *m) { free(m->q), free(m->scale); }

static void qwen_free(qwen *m) {
    free(m->embed), free(m->normw);
    q4_free(&m->lm);
    for (int l = 0; l < m->c.n_layer; l++) {
        qwblock *b = &m->b[l];
        q4_free(&b->wq), q4_free(&b->wk), q4_free(&b->wv), q4_free(&b->wo);
        q4_free(&b->gate), q4_free(&b->up), q4_free(&b->down);
        free(b->ln1), free(b->ln2), free(b->bq), free(b->bk), free(b->bv), free(b->kc), free(b->vc);
    }
    free(m->b);
    free(m);
}

/*
 * main.go:225-240 at temperature 0 without the end-of-turn stop: the
 * prompt through step one token at a time, then n_gen greedy picks, each fed
 * back. tokens/margins as tqo_gpt2_generate; seconds (optional): wall time of
 * the prompt steps and of the n_gen - 1 decode steps; prompt_logits
 * (optional, vocab floats): the logits after the last prompt token.
 * Returns 0 or -1.
 */
TQO_EXPORT int tqo_qwen_generate(const tqo_qwen_cfg *c, uint64_t seed, float sigma, const int *prompt, int n_prompt,
                                 int n_gen, int *tokens, float *margins, double *seconds, float *prompt_logits) {
    if (!c || n_prompt < 1 || n_prompt + n_gen > c->ctx + 1 || c->n_head % c->n_kv || c->d % c->n_head ||
        (c->d / c->n_head) % 2 || c->ffn % 2 || c->vocab % 2 || c->d % 2)
        return -1;
    qwen *m = qwen_new(c, seed, sigma);
    float *logits = malloc(sizeof(float) * (size_t)c->vocab);
    const double t0 = now_s();
    for (int p = 0; p < n_prompt; p++) qwen_step(m, prompt[p], p, logits);
    const double t1 = now_s();
    if (prompt_logits) memcpy(prompt_logits, logits, sizeof(float) * (size_t)c->vocab);
    int pos = n_prompt;
    for (int i = 0; i < n_gen; i++) {
        const int next = argmax(logits, c->vocab, margins ? &margins[i] : NULL);
        tokens[i] = next;
        if (i + 1 < n_gen) qwen_step(m, next, pos++, logits);
    }
    if (seconds) seconds[0] = t1 - t0, seconds[1] = now_s() - t1;
    free(logits);
    qwen_free(m);
    return 0;
}

/* ---- bounded timing of the decode step at a long context ------------------- */

/* Fills n bytes (fill_job) with a seeded xorshift stream, in parallel chunks:
 * the timed model's codes and its float buffers, whose values do not change
 * the cost of a step. */
struct fill_job {
    uint8_t *p;
    size_t n;
    uint64_t seed;
    int floats; /* fill floats in [-1, 1) instead of bytes */
};
#define FILL_CHUNK ((size_t)1 << 22)
static void fill_task(void *arg, int idx) {
    struct fill_job *j = arg;
    const size_t a = (size_t)idx * FILL_CHUNK, b = a + FILL_CHUNK < j->n ? a + FILL_CHUNK : j->n;
    uint64_t x = j->seed ^ (0x9E3779B97F4A7C15ull * (uint64_t)(idx + 1));
    for (size_t i = a; i < b; i += 4) {
        x ^= x << 13, x ^= x >> 7, x ^= x << 17;
        if (j->floats) {
            ((float *)j->p)[i / 4] = (float)((int32_t)(x >> 32)) * (1.0f / 2147483648.0f);
        } else {
            for (size_t k = 0; k < 4 && i + k < b; k++) j->p[i + k] = (uint8_t)(x >> (8 * k));
        }
    }
}
static void fill(void *p, size_t bytes, uint64_t seed, int floats) {
    struct fill_job j = {p, bytes, seed, floats};
    tqo_pool_run(fill_task, &j, (int)((bytes + FILL_CHUNK - 1) / FILL_CHUNK));
}
static void q4_timing(q4mat *m, int rows, int cols, uint64_t seed) {
    m->rows = rows, m->cols = cols;
    const size_t qb = (size_t)rows * (cols / 2) + 16, sf = (size_t)((rows + 63) / 64) * cols;
    m->q = malloc(qb);
    m->scale = malloc(sizeof(float) * sf);
    fill(m->q, qb, seed, 0);
    for (size_t i = 0; i < sf; i++) m->scale[i] = 0.01f;
}

/*
 * Wall time of n_steps decode steps (step, model.go:232-307) at cached
 * positions pos0 .. pos0 + n_steps - 1 of a Qwen2 of shape c: the bounded CPU
 * baseline of a long-context decode, extrapolated per token by the caller.
 * The model's codes, embeddings and caches are seeded filler (the cost of a
 * step does not depend on their values, and building real weights of the 7B
 * shape takes minutes). seconds[0]: the timed steps; seconds[1]: the build.
 * Returns 0 or -1.
 */
TQO_EXPORT int tqo_qwen_time_steps(const tqo_qwen_cfg *c, int pos0, int n_steps, double *seconds) {
    if (!c || !seconds || pos0 < 0 || n_steps < 1 || pos0 + n_steps > c->ctx || c->n_head % c->n_kv ||
        c->d % c->n_head || (c->d / c->n_head) % 2 || c->ffn % 2 || c->vocab % 2)
        return -1;
    const double t0 = now_s();
    qwen *m = calloc(1, sizeof(qwen));
    m->c = *c;
    m->hd = c->d / c->n_head;
    m->kvd = c->n_kv * m->hd;
    const int d = c->d, kvd = m->kvd, ffn = c->ffn;
    m->embed = malloc(sizeof(float) * (size_t)c->vocab * d);
    fill(m->embed, sizeof(float) * (size_t)c->vocab * d, 1, 1);
    m->normw = ones(d);
    q4_timing(&m->lm, d, c->vocab, 2);
    m->b = calloc((size_t)c->n_layer, sizeof(qwblock));
    for (int l = 0; l < c->n_layer; l++) {
        qwblock *b = &m->b[l];
        const uint64_t s0 = 32 + 16 * (uint64_t)l;
        q4_timing(&b->wq, d, d, s0);
        q4_timing(&b->wk, d, kvd, s0 + 1);
        q4_timing(&b->wv, d, kvd, s0 + 2);
        q4_timing(&b->wo, d, d, s0 + 3);
        q4_timing(&b->gate, d, ffn, s0 + 4);
        q4_timing(&b->up, d, ffn, s0 + 5);
        q4_timing(&b->down, ffn, d, s0 + 6);
        b->ln1 = ones(d), b->ln2 = ones(d);
        b->bq = zeros(d), b->bk = zeros(kvd), b->bv = zeros(kvd);
        b->kc = malloc(sizeof(float) * (size_t)c->ctx * kvd);
        b->vc = malloc(sizeof(float) * (size_t)c->ctx * kvd);
        fill(b->kc, sizeof(float) * (size_t)c->ctx * kvd, s0 + 7, 1);
        fill(b->vc, sizeof(float) * (size_t)c->ctx * kvd, s0 + 8, 1);
    }
    float *logits = malloc(sizeof(float) * (size_t)c->vocab);
    const double t1 = now_s();
    int tok = 0;
    for (int i = 0; i < n_steps; i++) {
        qwen_step(m, tok, pos0 + i, logits);
        tok = argmax(logits, c->vocab, NULL);
    }
    seconds[0] = now_s() - t1;
    seconds[1] = t1 - t0;
    free(logits);
    qwen_free(m);
    return 0;
}
