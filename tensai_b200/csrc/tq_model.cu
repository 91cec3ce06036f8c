// tq_model.cu — decode engine of tensai's GPT-2 example
// (_example/gpt2/model.go, main.go) on one B200: fp32 prefill with the
// unquantized weights, then int8 weight-only decode, weights and the fp32 KV
// cache resident in HBM, one CUDA graph per generated token.
//
// Numerics follow the Go code operation by operation (no FMA contraction
// where Go at GOAMD64=v1 has none): layer norm statistics, attention scores,
// softmax and GELU in float64; residual and bias adds and the
// attention-weighted value sum in float32 with separately rounded multiply
// and add, positions in order; prefill matmuls as tensai's dotRows (one fused
// multiply-add chain per output over k in order, zero activations skipped);
// decode matvecs on the library's int8 kernels; argmax with a strict > (ties
// to the lowest id), or the sample step with the caller's draws
// (tq_gpt2_set_sampling, main.go:78-105). Only reduction orders of the
// float64 sums differ from the sequential Go loops.
//
// Device state (int[3]): the token to feed, its position, tokens generated.
// Every kernel of a decode step reads the position from there, so one
// captured graph serves every step; the pick (argmax or sample) writes the
// next token and advances the state.
#include <cstdio>
#include <memory>
#include <string>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/tensai_cuda.h"
#define TQD_NS tqd_gpt2
// Programmatic dependent launch for every GPT-2 step kernel: measured 11% more
// tokens/s (1069 vs 960) on B200.
#define TQ_DECODE_PDL 1
#include "tq_decode.cuh"
#include "tq_internal.h"

namespace {

using namespace tqd_gpt2;

// ---- elementwise / normalisation kernels -------------------------------------
// x = wte[token] + wpe[pos] (model.go:181-184); decode: token and position
// from the state; prefill: row r takes tokens[r] at position r.
__global__ void embed_kernel(const float *wte, const float *wpe, const int *state, const int *tokens, float *x,
                             int d) {
    step_entry();
    const int r = blockIdx.x;
    const int tok = tokens ? tokens[r] : state[0];
    const int pos = tokens ? r : state[1];
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        x[(size_t)r * d + i] = __fadd_rn(wte[(size_t)tok * d + i], wpe[(size_t)pos * d + i]);
}

// layernorm (model.go:135-153) of row blockIdx.x. With y (decode, one row):
// first the residual add x += y + yb (model.go:229-231 / 242-244), then the
// norm of the new x, in one launch.
__global__ void layernorm_kernel(float *x, const float *w, const float *b, float *out, int n, const float *y = nullptr,
                                 const float *yb = nullptr) {
    step_entry();
    __shared__ double sh[32];
    float *xr = x + (size_t)blockIdx.x * n;
    float *o = out + (size_t)blockIdx.x * n;
    if (y) { // loads in batches of 4 per thread ahead of the stores (xr may alias y as far as nvcc knows)
        const int bd = blockDim.x;
        for (int i0 = threadIdx.x; i0 < n; i0 += 4 * bd) {
            float a[4], c[4], e[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + u * bd;
                a[u] = i < n ? xr[i] : 0.f;
                c[u] = i < n ? y[i] : 0.f;
                e[u] = i < n ? yb[i] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (i0 + u * bd < n) xr[i0 + u * bd] = __fadd_rn(a[u], __fadd_rn(c[u], e[u]));
        }
        __syncthreads();
    }
    double s = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = __dadd_rn(s, (double)xr[i]);
    const double mean = __ddiv_rn(block_reduce_d(s, sh, 0), (double)n);
    double v = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double d = __dsub_rn((double)xr[i], mean);
        v = __dadd_rn(v, __dmul_rn(d, d));
    }
    const double var = __ddiv_rn(block_reduce_d(v, sh, 0), (double)n);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(var, 1e-5)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        o[i] = __fadd_rn(__fmul_rn((float)__dmul_rn(__dsub_rn((double)xr[i], mean), inv), w[i]), b[i]);
}

// h = geluNew(h + b) (model.go:170-175, 239-240).
__global__ void bias_gelu_kernel(float *h, const float *b, int n, size_t total) {
    step_entry();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const double f = (double)__fadd_rn(h[i], b[i % n]);
        const double c = __dmul_rn(__dmul_rn(__dmul_rn(0.044715, f), f), f);
        const double t = tanh(__dmul_rn(0.7978845608028654, __dadd_rn(f, c)));
        h[i] = (float)__dmul_rn(__dmul_rn(0.5, f), __dadd_rn(1.0, t));
    }
}

// qkv rows (+ bias): q stays in place, k and v go to the cache at the row's
// position (decode: the state's position; prefill: row r at position r).
__global__ void qkv_post_kernel(float *qkv, const float *bias, float *kc, float *vc, const int *state, int d,
                                int prefill) {
    step_entry();
    const int r = blockIdx.x;
    const int pos = prefill ? r : state[1];
    float *row = qkv + (size_t)r * 3 * d;
    for (int i = threadIdx.x; i < 3 * d; i += blockDim.x) {
        const float v = __fadd_rn(row[i], bias[i]);
        if (i < d)
            row[i] = v;
        else if (i < 2 * d)
            kc[(size_t)pos * d + (i - d)] = v;
        else
            vc[(size_t)pos * d + (i - 2 * d)] = v;
    }
}

// C[M][N] = A[M][K] @ B[K][N], every element one fused multiply-add chain
// over k in order with zero A entries skipped: tensai's dotRows
// (dot_simd.go:23-79). 64 x 64 tile per block, 4 x 4 per thread.
__global__ void __launch_bounds__(256) sgemm_chain_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                          float *__restrict__ C, int M, int N, int K) {
    step_entry();
    __shared__ float As[16][64];
    __shared__ float Bs[16][64];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            const int kk = e & 15, rr = e >> 4; // A: 64 rows x 16 k
            const int r = r0 + rr, k = k0 + kk;
            As[kk][rr] = (r < M && k < K) ? A[(size_t)r * K + k] : 0.f;
            const int cc = e & 63, kb = e >> 6; // B: 16 k x 64 cols
            const int c = c0 + cc, k2 = k0 + kb;
            Bs[kb][cc] = (c < N && k2 < K) ? B[(size_t)k2 * N + c] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (a[i] != 0.f)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(b[j], a[i], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int r = r0 + ty * 4 + i, c = c0 + tx * 4 + j;
            if (r < M && c < N) C[(size_t)r * N + c] = acc[i][j];
        }
}

__global__ void transpose_kernel(const float *in, float *out, int rows, int cols) {
    step_entry();
    __shared__ float t[32][33];
    const int c = blockIdx.x * 32 + threadIdx.x, r0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y)
        if (r0 + j < rows && c < cols) t[j][threadIdx.x] = in[(size_t)(r0 + j) * cols + c];
    __syncthreads();
    const int r = r0 + threadIdx.x, cb = blockIdx.x * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y)
        if (cb + j < cols && r < rows) out[(size_t)(cb + j) * rows + r] = t[threadIdx.x][j];
}

// ---- engine -------------------------------------------------------------------

struct Weight {
    float *w = nullptr; // fp32 [rows][cols] (prefill)
    TqMatrixDev q{};    // int8 twin (decode)
    int rows = 0, cols = 0;
};

struct Block {
    Weight attn, proj, fc, fc2;
    float *ln1w, *ln1b, *ln2w, *ln2b, *attnB, *projB, *fcB, *fc2B;
    float *kc, *vc; // [ctx][d]
};

struct Gpt2 {
    int device = 0;
    tq_gpt2_config c{};
    cudaStream_t st = nullptr;
    TqScratch scr{};
    float *wte = nullptr, *wpe = nullptr, *lnfw = nullptr, *lnfb = nullptr;
    Weight wteT;
    std::vector<Block> b;
    // decode buffers
    float *x, *xn, *qkv, *att, *y, *h, *logits;
    // prefill buffers (max_prompt rows)
    int max_prompt = 0;
    float *X = nullptr, *XN = nullptr, *QKV = nullptr, *ATT = nullptr, *Y = nullptr, *H = nullptr;
    int *state = nullptr, *tokens = nullptr, *d_prompt = nullptr, *cand = nullptr, *part = nullptr;
    AttScratch att_scr;
    cudaGraphExec_t graph = nullptr;
    std::vector<void *> allocs;
    bool loaded = false; // tq_gpt2_create_empty: weights come from tq_gpt2_load_tensor
    // tq_gpt2_set_sampling: temp > 0 draws generated token k with draws[k]
    double temp = 0;
    double *draws = nullptr;
    int n_draws = 0;
    TqSampler smp;
};

std::mutex g_models_mu;
std::unordered_map<uint64_t, std::shared_ptr<Gpt2>> g_models;
uint64_t g_next_model = 1;

cudaError_t dalloc(Gpt2 &m, void **p, size_t bytes) {
    cudaError_t e = tq_dev_malloc(p, bytes);
    if (e == cudaSuccess) m.allocs.push_back(*p);
    return e;
}

unsigned grid_for(size_t n) {
    size_t g = (n + kThreads - 1) / kThreads;
    return (unsigned)(g < 148 * 16 ? (g ? g : 1) : 148 * 16);
}

cudaError_t fill(float *p, float v, size_t n, cudaStream_t st) {
    fill_kernel<<<grid_for(n), kThreads, 0, st>>>(p, v, n);
    return cudaGetLastError();
}

void destroy(Gpt2 &m) {
    if (m.graph) cudaGraphExecDestroy(m.graph);
    m.graph = nullptr;
    if (m.st) cudaStreamSynchronize(m.st);
    for (auto &bl : m.b)
        for (Weight *w : {&bl.attn, &bl.proj, &bl.fc, &bl.fc2}) tq_release_matrix(&w->q);
    tq_release_matrix(&m.wteT.q);
    for (void *p : m.allocs) cudaFree(p);
    m.allocs.clear();
    tq_sampler_free(&m.smp);
    if (m.draws) cudaFree(m.draws);
    m.draws = nullptr;
    if (m.st) tq_scratch_release(m.device, m.st);
    if (m.st) cudaStreamDestroy(m.st);
    m.st = nullptr;
}

#define TRY(expr)                                                                                                      \
    do {                                                                                                               \
        cudaError_t e_ = (expr);                                                                                       \
        if (e_ != cudaSuccess) return e_;                                                                              \
    } while (0)

size_t attn_smem(const Gpt2 &m) { return attention_smem(m.c.ctx); }

// A random-init weight: fp32 from the shared generator, then its int8 twin.
cudaError_t make_weight(Gpt2 &m, Weight &w, int rows, int cols, uint64_t seed, uint64_t stream, float sigma, int *rc) {
    w.rows = rows, w.cols = cols;
    TRY(dalloc(m, (void **)&w.w, sizeof(float) * (size_t)rows * cols));
    if (m.loaded) // filled by tq_gpt2_load_tensor
        TRY(cudaMemsetAsync(w.w, 0, sizeof(float) * (size_t)rows * cols, m.st));
    else
        TRY(tq_launch_synth(w.w, (size_t)rows * cols, seed, stream, sigma, m.st));
    if ((*rc = tq_alloc_matrix(8, rows, cols, &w.q, m.st)) != TQ_OK) return cudaErrorMemoryAllocation;
    return tq_launch_quantize(w.q, w.w, m.st);
}

cudaError_t build(Gpt2 &m, uint64_t seed, float sigma, int *rc) {
    const tq_gpt2_config &c = m.c;
    const int d = c.d, ffn = c.ffn;
    TRY(cudaStreamCreateWithFlags(&m.st, cudaStreamNonBlocking));
    TRY(dalloc(m, (void **)&m.wte, sizeof(float) * (size_t)c.vocab * d));
    TRY(dalloc(m, (void **)&m.wpe, sizeof(float) * (size_t)c.ctx * d));
    if (m.loaded) {
        TRY(cudaMemsetAsync(m.wte, 0, sizeof(float) * (size_t)c.vocab * d, m.st));
        TRY(cudaMemsetAsync(m.wpe, 0, sizeof(float) * (size_t)c.ctx * d, m.st));
    } else {
        TRY(tq_launch_synth(m.wte, (size_t)c.vocab * d, seed, 1, sigma, m.st));
        TRY(tq_launch_synth(m.wpe, (size_t)c.ctx * d, seed, 2, sigma, m.st));
    }
    // wteT = wte^T (model.go:122), fp32 for the prefill head and its int8 twin.
    m.wteT.rows = d, m.wteT.cols = c.vocab;
    TRY(dalloc(m, (void **)&m.wteT.w, sizeof(float) * (size_t)d * c.vocab));
    transpose_kernel<<<dim3((d + 31) / 32, (c.vocab + 31) / 32), dim3(32, 8), 0, m.st>>>(m.wte, m.wteT.w, c.vocab, d);
    TRY(cudaGetLastError());
    if ((*rc = tq_alloc_matrix(8, d, c.vocab, &m.wteT.q, m.st)) != TQ_OK) return cudaErrorMemoryAllocation;
    TRY(tq_launch_quantize(m.wteT.q, m.wteT.w, m.st));
    // ones / zeros for the layer norms and biases of a random-init model
    float *ones, *zeros;
    const size_t vec = (size_t)(3 * d > ffn ? 3 * d : ffn);
    TRY(dalloc(m, (void **)&ones, sizeof(float) * vec));
    TRY(dalloc(m, (void **)&zeros, sizeof(float) * vec));
    TRY(fill(ones, 1.f, vec, m.st));
    TRY(fill(zeros, 0.f, vec, m.st));
    m.lnfw = ones, m.lnfb = zeros;
    // a checkpoint model gets its own norm weights and biases (1 and 0 until loaded)
    auto vec_of = [&](float v, size_t n, float **out) -> cudaError_t {
        TRY(dalloc(m, (void **)out, sizeof(float) * n));
        return fill(*out, v, n, m.st);
    };
    if (m.loaded) {
        TRY(vec_of(1.f, d, &m.lnfw));
        TRY(vec_of(0.f, d, &m.lnfb));
    }
    m.b.resize(c.n_layer);
    for (int l = 0; l < c.n_layer; l++) {
        Block &bl = m.b[l];
        const uint64_t s0 = 16 + 8 * (uint64_t)l;
        TRY(make_weight(m, bl.attn, d, 3 * d, seed, s0, sigma, rc));
        TRY(make_weight(m, bl.proj, d, d, seed, s0 + 1, sigma, rc));
        TRY(make_weight(m, bl.fc, d, ffn, seed, s0 + 2, sigma, rc));
        TRY(make_weight(m, bl.fc2, ffn, d, seed, s0 + 3, sigma, rc));
        bl.ln1w = bl.ln2w = ones;
        bl.ln1b = bl.ln2b = bl.attnB = bl.projB = bl.fcB = bl.fc2B = zeros;
        if (m.loaded) {
            TRY(vec_of(1.f, d, &bl.ln1w));
            TRY(vec_of(1.f, d, &bl.ln2w));
            TRY(vec_of(0.f, d, &bl.ln1b));
            TRY(vec_of(0.f, d, &bl.ln2b));
            TRY(vec_of(0.f, 3 * (size_t)d, &bl.attnB));
            TRY(vec_of(0.f, d, &bl.projB));
            TRY(vec_of(0.f, ffn, &bl.fcB));
            TRY(vec_of(0.f, d, &bl.fc2B));
        }
        TRY(dalloc(m, (void **)&bl.kc, sizeof(float) * (size_t)c.ctx * d));
        TRY(dalloc(m, (void **)&bl.vc, sizeof(float) * (size_t)c.ctx * d));
    }
    TRY(dalloc(m, (void **)&m.x, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.xn, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.qkv, sizeof(float) * 3 * d));
    TRY(dalloc(m, (void **)&m.att, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.y, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.h, sizeof(float) * ffn));
    TRY(dalloc(m, (void **)&m.logits, sizeof(float) * c.vocab));
    TRY(dalloc(m, (void **)&m.state, sizeof(int) * 4));
    TRY(dalloc(m, (void **)&m.cand, sizeof(int) * 2));
    TRY(dalloc(m, (void **)&m.part, sizeof(int) * 2 * kArgBlocks));
    void *ab = nullptr;
    TRY(dalloc(m, &ab, att_scratch_bytes(c.n_head, c.ctx, d / c.n_head)));
    TRY(att_scratch(ab, c.n_head, c.ctx, d / c.n_head, m.st, &m.att_scr));
    TRY(att_setup(d / c.n_head, 1));
    TRY(dalloc(m, (void **)&m.tokens, sizeof(int) * (size_t)(c.ctx + 1)));
    if ((*rc = tq_scratch_for(m.device, m.st, &m.scr, 1)) != TQ_OK) return cudaErrorMemoryAllocation;
    const size_t smem = attn_smem(m);
    if (smem > 48 * 1024) TRY(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    return cudaStreamSynchronize(m.st);
}

cudaError_t ensure_prefill(Gpt2 &m, int T) {
    if (T <= m.max_prompt) return cudaSuccess;
    const int d = m.c.d, ffn = m.c.ffn;
    TRY(dalloc(m, (void **)&m.X, sizeof(float) * (size_t)T * d));
    TRY(dalloc(m, (void **)&m.XN, sizeof(float) * (size_t)T * d));
    TRY(dalloc(m, (void **)&m.QKV, sizeof(float) * (size_t)T * 3 * d));
    TRY(dalloc(m, (void **)&m.ATT, sizeof(float) * (size_t)T * d));
    TRY(dalloc(m, (void **)&m.Y, sizeof(float) * (size_t)T * d));
    TRY(dalloc(m, (void **)&m.H, sizeof(float) * (size_t)T * ffn));
    TRY(dalloc(m, (void **)&m.d_prompt, sizeof(int) * (size_t)T));
    m.max_prompt = T;
    return cudaSuccess;
}

cudaError_t sgemm(const float *A, const float *B, float *C, int M, int N, int K, cudaStream_t st) {
    sgemm_chain_kernel<<<dim3((N + 63) / 64, (M + 63) / 64), 256, 0, st>>>(A, B, C, M, N, K);
    return cudaGetLastError();
}


// prefill (model.go:361-401) of T prompt tokens, then the first pick.
cudaError_t prefill(Gpt2 &m, const int *prompt, int T) {
    const int d = m.c.d, ffn = m.c.ffn, hd = d / m.c.n_head;
    TRY(ensure_prefill(m, T));
    TRY(cudaMemcpyAsync(m.d_prompt, prompt, sizeof(int) * T, cudaMemcpyHostToDevice, m.st));
    set_state_kernel<<<1, 1, 0, m.st>>>(m.state, 0, 0, 0);
    embed_kernel<<<T, kThreads, 0, m.st>>>(m.wte, m.wpe, m.state, m.d_prompt, m.X, d);
    TRY(cudaGetLastError());
    for (Block &bl : m.b) {
        layernorm_kernel<<<T, kThreads, 0, m.st>>>(m.X, bl.ln1w, bl.ln1b, m.XN, d);
        TRY(sgemm(m.XN, bl.attn.w, m.QKV, T, 3 * d, d, m.st));
        qkv_post_kernel<<<T, kThreads, 0, m.st>>>(m.QKV, bl.attnB, bl.kc, bl.vc, m.state, d, 1);
        attention_kernel<<<dim3(m.c.n_head, T), kThreads, attn_smem(m), m.st>>>(
            m.QKV, 3 * d, bl.kc, bl.vc, d, m.ATT, d, m.state, hd, 1, 0.125 /* 1/sqrt(64) */, 1, m.c.ctx, 0);
        TRY(cudaGetLastError());
        TRY(sgemm(m.ATT, bl.proj.w, m.Y, T, d, d, m.st));
        residual_kernel<<<grid_for((size_t)T * d), kThreads, 0, m.st>>>(m.X, m.Y, bl.projB, d, (size_t)T * d);
        layernorm_kernel<<<T, kThreads, 0, m.st>>>(m.X, bl.ln2w, bl.ln2b, m.XN, d);
        TRY(sgemm(m.XN, bl.fc.w, m.H, T, ffn, d, m.st));
        bias_gelu_kernel<<<grid_for((size_t)T * ffn), kThreads, 0, m.st>>>(m.H, bl.fcB, ffn, (size_t)T * ffn);
        TRY(sgemm(m.H, bl.fc2.w, m.Y, T, d, ffn, m.st));
        residual_kernel<<<grid_for((size_t)T * d), kThreads, 0, m.st>>>(m.X, m.Y, bl.fc2B, d, (size_t)T * d);
        TRY(cudaGetLastError());
    }
    layernorm_kernel<<<1, kThreads, 0, m.st>>>(m.X + (size_t)(T - 1) * d, m.lnfw, m.lnfb, m.xn, d);
    TRY(sgemm(m.xn, m.wteT.w, m.logits, 1, m.c.vocab, d, m.st));
    if (m.temp > 0) { // main.go:78-105 with the caller's draw for generated token state[2]
        TRY(tq_launch_sample(m.smp, m.logits, m.c.vocab, m.temp, m.draws, m.state + 2, m.cand + 1, m.st));
        pick_kernel<<<1, 32, 0, m.st>>>(m.cand, 1, m.state, m.tokens, T);
    } else {
        argmax_kernel<<<1, 1024, 0, m.st>>>(m.logits, m.c.vocab, 0, m.cand, m.state, m.tokens, T, 1);
    }
    return cudaGetLastError();
}

// step (model.go:179-245) on the int8 weights: feeds the state's token at
// the state's position, then picks the next token.
cudaError_t decode_step(Gpt2 &m) {
    const int d = m.c.d, ffn = m.c.ffn, hd = d / m.c.n_head;
    TRY(step_launch(embed_kernel, dim3(1), dim3(kThreads), 0, m.st, m.wte, m.wpe, m.state, nullptr, m.x, d));
    const float *pend = nullptr, *pendb = nullptr; // residual still to be added to x
    for (Block &bl : m.b) {
        TRY(step_launch(layernorm_kernel, dim3(1), dim3(kThreads), 0, m.st, m.x, bl.ln1w, bl.ln1b, m.xn, d, pend, pendb));
        TRY(tq_launch_matmul(bl.attn.q, m.xn, m.qkv, 1, m.scr, m.st));
        TRY(step_launch(qkv_post_kernel, dim3(1), dim3(kThreads), 0, m.st, m.qkv, bl.attnB, bl.kc, bl.vc, m.state, d, 0));
        TRY(decode_attention(m.qkv, bl.kc, bl.vc, d, m.att, m.state, m.c.n_head, hd, 1, 0.125 /* 1/sqrt(64) */,
                             m.att_scr, m.st));
        TRY(tq_launch_matmul(bl.proj.q, m.att, m.y, 1, m.scr, m.st));
        TRY(step_launch(layernorm_kernel, dim3(1), dim3(kThreads), 0, m.st, m.x, bl.ln2w, bl.ln2b, m.xn, d, m.y, bl.projB));
        TRY(tq_launch_matmul(bl.fc.q, m.xn, m.h, 1, m.scr, m.st));
        TRY(step_launch(bias_gelu_kernel, dim3(grid_for(ffn)), dim3(kThreads), 0, m.st, m.h, bl.fcB, ffn, (size_t)ffn));
        TRY(tq_launch_matmul(bl.fc2.q, m.h, m.y, 1, m.scr, m.st));
        pend = m.y, pendb = bl.fc2B;
        TRY(cudaGetLastError());
    }
    TRY(step_launch(layernorm_kernel, dim3(1), dim3(kThreads), 0, m.st, m.x, m.lnfw, m.lnfb, m.xn, d, pend, pendb));
    TRY(tq_launch_matmul(m.wteT.q, m.xn, m.logits, 1, m.scr, m.st));
    if (m.temp > 0) {
        TRY(tq_launch_sample(m.smp, m.logits, m.c.vocab, m.temp, m.draws, m.state + 2, m.cand + 1, m.st));
        return step_launch(pick_kernel, dim3(1), dim3(32), 0, m.st, (const int *)m.cand, 1, m.state, m.tokens, -1);
    }
    return greedy_pick(m.logits, m.c.vocab, 0, m.part, m.cand, m.state, m.tokens, -1, 1, m.st);
}

cudaError_t capture_step(Gpt2 &m) {
    if (m.graph) return cudaSuccess;
    cudaGraph_t g = nullptr;
    TRY(cudaStreamBeginCapture(m.st, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = decode_step(m);
    cudaError_t e2 = cudaStreamEndCapture(m.st, &g);
    if (e == cudaSuccess) e = e2;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&m.graph, g, 0);
    if (g) cudaGraphDestroy(g);
    return e;
}

std::shared_ptr<Gpt2> find_model(uint64_t h, int *rc) {
    std::lock_guard<std::mutex> lk(g_models_mu);
    auto it = g_models.find(h);
    if (it == g_models.end()) {
        *rc = tq_fail(TQ_ERR_HANDLE, "tensai: invalid or freed model handle %llu", (unsigned long long)h);
        return nullptr;
    }
    return it->second;
}

} // namespace

extern "C" {

static int gpt2_create(const tq_gpt2_config *cfg, uint64_t seed, float sigma, bool loaded, uint64_t *model) {
    if (!cfg || !model) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    const tq_gpt2_config &c = *cfg;
    if (c.n_layer < 1 || c.n_head < 1 || c.d < 1 || c.ffn < 1 || c.vocab < 1 || c.ctx < 1 || c.d % c.n_head ||
        c.d / c.n_head != 64)
        return tq_fail(TQ_ERR_ARG, "tensai: bad GPT-2 configuration (the attention scale is the example's 1/8: "
                                   "head size must be 64)");
    if (c.ctx > 8192) return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: context %d exceeds 8192", c.ctx);
    auto m = std::make_shared<Gpt2>();
    m->c = c;
    m->loaded = loaded;
    cudaError_t e = cudaGetDevice(&m->device);
    int rc = TQ_OK;
    if (e == cudaSuccess) e = build(*m, seed, sigma, &rc);
    if (e != cudaSuccess || rc != TQ_OK) {
        destroy(*m);
        return rc != TQ_OK ? rc : tq_cuda_fail(e, "GPT-2 model build");
    }
    std::lock_guard<std::mutex> lk(g_models_mu);
    *model = g_next_model++;
    g_models[*model] = m;
    return TQ_OK;
}

int tq_gpt2_create(const tq_gpt2_config *cfg, uint64_t seed, float sigma, uint64_t *model) {
    return gpt2_create(cfg, seed, sigma, false, model);
}

int tq_gpt2_create_empty(const tq_gpt2_config *cfg, uint64_t *model) { return gpt2_create(cfg, 0, 0.f, true, model); }

int tq_gpt2_load_tensor(uint64_t model, const char *name, const void *data, int dtype, int rows, int cols) {
    if (!name || !data) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    if (dtype != TQ_LINEAR_F32 && dtype != TQ_LINEAR_F16 && dtype != TQ_LINEAR_BF16)
        return tq_fail(TQ_ERR_ARG, "tensai: unknown tensor type %d", dtype);
    int rc = TQ_OK;
    auto m = find_model(model, &rc);
    if (!m) return rc;
    if (!m->loaded) return tq_fail(TQ_ERR_ARG, "tensai: %s: the model holds random-init weights", name);
    const tq_gpt2_config &c = m->c;
    const int d = c.d, ffn = c.ffn;
    cudaError_t e = cudaSetDevice(m->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "tensor load");
    auto shape = [&](int r, int cc) {
        return rows == r && cols == cc ? TQ_OK
                                       : tq_fail(TQ_ERR_SHAPE, "tensai: %s is %d x %d, expected %d x %d", name, rows,
                                                 cols, r, cc);
    };
    auto widen = [&](float *dst, size_t n) {
        widen_kernel<<<grid_for(n), kThreads, 0, m->st>>>(data, dtype, dst, n);
        return cudaGetLastError();
    };
    // a Conv1D weight [in, out] (model.go:126-129): the fp32 prefill copy and its int8 twin
    auto weight = [&](Weight &w) {
        if ((rc = shape(w.rows, w.cols)) != TQ_OK) return rc;
        cudaError_t err = widen(w.w, (size_t)w.rows * w.cols);
        if (err == cudaSuccess) err = tq_launch_quantize(w.q, w.w, m->st);
        return err == cudaSuccess ? TQ_OK : tq_cuda_fail(err, "tensor quantize");
    };
    auto vec = [&](float *dst, int n) {
        if ((rc = shape(1, n)) != TQ_OK) return rc;
        const cudaError_t err = widen(dst, (size_t)n);
        return err == cudaSuccess ? TQ_OK : tq_cuda_fail(err, "tensor load");
    };
    const std::string n(name);
    int l = -1, used = 0;
    char rest[96] = {};
    if (n == "wte.weight") { // the embedding and the tied head wte^T (model.go:106-119)
        if ((rc = shape(c.vocab, d)) != TQ_OK) return rc;
        e = widen(m->wte, (size_t)c.vocab * d);
        if (e == cudaSuccess) {
            transpose_kernel<<<dim3((d + 31) / 32, (c.vocab + 31) / 32), dim3(32, 8), 0, m->st>>>(m->wte, m->wteT.w,
                                                                                                   c.vocab, d);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = tq_launch_quantize(m->wteT.q, m->wteT.w, m->st);
        if (e != cudaSuccess) rc = tq_cuda_fail(e, "embedding");
    } else if (n == "wpe.weight") { // positions beyond the model's context are not kept
        if (cols != d || rows < c.ctx)
            return tq_fail(TQ_ERR_SHAPE, "tensai: %s is %d x %d, expected at least %d x %d", name, rows, cols, c.ctx, d);
        if ((e = widen(m->wpe, (size_t)c.ctx * d)) != cudaSuccess) rc = tq_cuda_fail(e, "positions");
    } else if (n == "ln_f.weight") {
        rc = vec(m->lnfw, d);
    } else if (n == "ln_f.bias") {
        rc = vec(m->lnfb, d);
    } else if (std::sscanf(name, "h.%d.%95s%n", &l, rest, &used) == 2 && (size_t)used == n.size() && l >= 0 &&
               l < c.n_layer) {
        Block &b = m->b[l];
        const std::string r(rest);
        if (r == "ln_1.weight") rc = vec(b.ln1w, d);
        else if (r == "ln_1.bias") rc = vec(b.ln1b, d);
        else if (r == "ln_2.weight") rc = vec(b.ln2w, d);
        else if (r == "ln_2.bias") rc = vec(b.ln2b, d);
        else if (r == "attn.c_attn.weight") rc = weight(b.attn);
        else if (r == "attn.c_attn.bias") rc = vec(b.attnB, 3 * d);
        else if (r == "attn.c_proj.weight") rc = weight(b.proj);
        else if (r == "attn.c_proj.bias") rc = vec(b.projB, d);
        else if (r == "mlp.c_fc.weight") rc = weight(b.fc);
        else if (r == "mlp.c_fc.bias") rc = vec(b.fcB, ffn);
        else if (r == "mlp.c_proj.weight") rc = weight(b.fc2);
        else if (r == "mlp.c_proj.bias") rc = vec(b.fc2B, d);
        else rc = tq_fail(TQ_ERR_ARG, "tensai: unknown GPT-2 tensor %s", name);
    } else {
        rc = tq_fail(TQ_ERR_ARG, "tensai: unknown GPT-2 tensor %s", name);
    }
    if (rc != TQ_OK) return rc;
    if ((e = cudaStreamSynchronize(m->st)) != cudaSuccess) return tq_cuda_fail(e, "tensor load");
    return TQ_OK;
}

int tq_gpt2_generate(uint64_t model, const int *prompt, int n_prompt, int n_gen, int *tokens, float *times_ms) {
    int rc = TQ_OK;
    auto m = find_model(model, &rc);
    if (!m) return rc;
    if (!prompt || !tokens || n_prompt < 1 || n_gen < 1) return tq_fail(TQ_ERR_ARG, "tensai: bad generate arguments");
    if (n_prompt + n_gen - 1 > m->c.ctx)
        return tq_fail(TQ_ERR_ARG, "tensai: %d prompt + %d generated tokens exceed the context of %d", n_prompt, n_gen,
                       m->c.ctx);
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= m->c.vocab)
            return tq_fail(TQ_ERR_ARG, "tensai: prompt token %d out of range [0, %d)", prompt[i], m->c.vocab);
    if (m->temp > 0 && n_gen > m->n_draws)
        return tq_fail(TQ_ERR_ARG, "tensai: %d tokens to sample but %d draws set", n_gen, m->n_draws);
    cudaError_t e = cudaSetDevice(m->device);
    cudaEvent_t ev[3] = {};
    for (int i = 0; i < 3 && e == cudaSuccess; i++) e = cudaEventCreate(&ev[i]);
    if (e == cudaSuccess) e = cudaEventRecord(ev[0], m->st);
    if (e == cudaSuccess) e = prefill(*m, prompt, n_prompt);
    if (e == cudaSuccess) e = cudaEventRecord(ev[1], m->st);
    // The first step runs eagerly (it configures the kernels), the rest replay one graph.
    if (e == cudaSuccess && n_gen > 1) e = decode_step(*m);
    if (e == cudaSuccess && n_gen > 2) e = capture_step(*m);
    for (int i = 2; i < n_gen && e == cudaSuccess; i++) e = cudaGraphLaunch(m->graph, m->st);
    if (e == cudaSuccess) e = cudaEventRecord(ev[2], m->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tokens, m->tokens, sizeof(int) * n_gen, cudaMemcpyDeviceToHost, m->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
    if (e == cudaSuccess && times_ms) {
        e = cudaEventElapsedTime(&times_ms[0], ev[0], ev[1]);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&times_ms[1], ev[1], ev[2]);
    }
    for (auto &x : ev)
        if (x) cudaEventDestroy(x);
    if (e != cudaSuccess) return tq_cuda_fail(e, "GPT-2 generate");
    unsigned status = 0;
    if ((e = tq_read_status(m->scr, m->st, &status)) != cudaSuccess) return tq_cuda_fail(e, "status read");
    if (status & TQ_STATUS_TIMEOUT) return tq_fail(TQ_ERR_TIMEOUT, "tensai: a kernel timed out during decode");
    return TQ_OK;
}

int tq_gpt2_set_sampling(uint64_t model, double temp, const double *draws, int n_draws) {
    int rc = TQ_OK;
    auto m = find_model(model, &rc);
    if (!m) return rc;
    if ((rc = tq_check_draws(temp, draws, n_draws)) != TQ_OK) return rc;
    cudaError_t e = cudaSetDevice(m->device);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
    if (m->graph) cudaGraphExecDestroy(m->graph); // the graph holds the previous pick
    m->graph = nullptr;
    if (m->draws) cudaFree(m->draws);
    m->draws = nullptr;
    m->n_draws = 0;
    m->temp = 0;
    if (e == cudaSuccess && temp > 0) {
        e = tq_dev_malloc((void **)&m->draws, sizeof(double) * n_draws);
        if (e == cudaSuccess) e = cudaMemcpy(m->draws, draws, sizeof(double) * n_draws, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = tq_sampler_alloc(&m->smp, m->c.vocab);
        if (e == cudaSuccess) m->temp = temp, m->n_draws = n_draws;
    }
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "sampling set-up");
}

int tq_gpt2_free(uint64_t model) {
    std::shared_ptr<Gpt2> m;
    {
        std::lock_guard<std::mutex> lk(g_models_mu);
        auto it = g_models.find(model);
        if (it == g_models.end()) return TQ_OK;
        m = it->second;
        g_models.erase(it);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    destroy(*m);
    cudaSetDevice(prev);
    return TQ_OK;
}

} // extern "C"
