// tq_qwen.cu — greedy decode engine of tensai's Qwen2 example
// (_example/qwen/model.go:182-307, main.go:225-240) with int4 group-64
// weights, tensor-parallel over 1, 2, 4 or 8 GPUs of one node, one process
// per GPU.
//
// Sharding (weights re-quantized per shard give the same codes and scales
// as the unsharded QuantizeMatrix4, which is per column and per 64-row group):
//   q/k/v     column shards by attention head, fused into one [d x (q|k|v)]
//             matrix; with more GPUs than KV heads the attention shards are
//             duplicated across GPU groups (8 GPUs, 4 KV heads: pairs);
//   o_proj    row shard of d/world rows (whole 64-row groups), inside this
//             GPU's attention shard;
//   gate/up   column shards of ffn/world, fused into one [d x (gate|up)];
//   down      row shard of ffn/world rows;
//   lm head   column shard of vocab/world, greedy pick per shard, then the
//             candidates (value, id) of all GPUs gathered, ties to the lower id.
// The o_proj and down partial sums meet in an NCCL all-reduce (sum), the only
// exchange of the step; NCCL is resolved at run time from the process (the
// library torch loaded), so the whole step, collectives included, is one
// CUDA graph replayed per token.
//
// The prompt goes through the same step one token at a time (main.go:229-231):
// the step's last kernel feeds the next prompt id while the prompt lasts and
// the greedy pick after it.
//
// Numerics as the Go code: RMSNorm, RoPE, attention scores, softmax and SiLU
// in float64, residuals and the value sum in float32, products unfused.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/tensai_cuda.h"
#define TQD_NS tqd_qwen
// Plain launches for the Qwen2 step: letting each step's matvec become resident
// early beside the small kernels (TQ_DECODE_PDL 1) measured 10% fewer tokens/s
// at the 7B shape on B200 (277 vs 310), though it helps GPT-2.
#define TQ_DECODE_PDL 0
#include "tq_decode.cuh"
#include "tq_internal.h"

namespace {

using namespace tqd_qwen;

// ---- NCCL, resolved at run time -----------------------------------------------
struct Nccl {
    bool ok = false;
    ncclResult_t (*getUniqueId)(ncclUniqueId *);
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*commDestroy)(ncclComm_t);
    const char *(*errorString)(ncclResult_t);
};
std::mutex g_nccl_mu;
Nccl g_nccl;

int load_nccl() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.ok) return TQ_OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD); // the copy already in the process (torch's)
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: libnccl.so.2 not found: %s", dlerror());
    auto sym = [&](const char *n) { return dlsym(h, n); };
    g_nccl.getUniqueId = (decltype(g_nccl.getUniqueId))sym("ncclGetUniqueId");
    g_nccl.commInitRank = (decltype(g_nccl.commInitRank))sym("ncclCommInitRank");
    g_nccl.allReduce = (decltype(g_nccl.allReduce))sym("ncclAllReduce");
    g_nccl.allGather = (decltype(g_nccl.allGather))sym("ncclAllGather");
    g_nccl.commDestroy = (decltype(g_nccl.commDestroy))sym("ncclCommDestroy");
    g_nccl.errorString = (decltype(g_nccl.errorString))sym("ncclGetErrorString");
    if (!g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.allReduce || !g_nccl.allGather || !g_nccl.commDestroy ||
        !g_nccl.errorString)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: libnccl.so.2 lacks an expected symbol");
    g_nccl.ok = true;
    return TQ_OK;
}

// ---- kernels ------------------------------------------------------------------
// Loads go in batches of kNormBatch per thread, issued before the batch's
// stores (x may alias y as far as the compiler knows); the elements keep the
// per-thread order of a plain strided loop.
constexpr int kNormBatch = 8;
// x = embed[token] and out = rmsnorm(x) * w (model.go:239-240, 182-193), and
// the step's RoPE table cs for the state's position, one launch.
__global__ void embed_norm_kernel(const float *embed, const int *state, float *x, const float *w, float *out, int d,
                                  double eps, double *cs, int hd, double theta) {
    step_entry();
    __shared__ double sh[32];
    rope_table(cs, state[1], hd, theta);
    const float *row = embed + (size_t)state[0] * d;
    constexpr int B = kNormBatch;
    const int bd = blockDim.x;
    double ss = 0;
    for (int i0 = threadIdx.x; i0 < d; i0 += B * bd) {
        float a[B];
#pragma unroll
        for (int u = 0; u < B; u++) a[u] = i0 + u * bd < d ? row[i0 + u * bd] : 0.f;
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            if (i < d) {
                x[i] = a[u];
                ss = __dadd_rn(ss, __dmul_rn((double)a[u], (double)a[u]));
            }
        }
    }
    ss = block_reduce_d(ss, sh, 0);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)d), eps)));
    for (int i0 = threadIdx.x; i0 < d; i0 += B * bd) {
        float a[B], c[B];
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            a[u] = i < d ? row[i] : 0.f;
            c[u] = i < d ? w[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            if (i < d) out[i] = __fmul_rn((float)__dmul_rn((double)a[u], inv), c[u]);
        }
    }
}

// rmsnorm (model.go:182-193): sum of squares in float64, out = float32(v *
// inv) * w. With y: first the residual add x += y (model.go:276-278 /
// 301-303), then the norm of the new x, in one launch.
__global__ void rmsnorm_kernel(float *x, const float *y, const float *w, float *out, int n, double eps) {
    step_entry();
    __shared__ double sh[32];
    constexpr int B = kNormBatch;
    const int bd = blockDim.x;
    double ss = 0;
    for (int i0 = threadIdx.x; i0 < n; i0 += B * bd) {
        float a[B], b[B];
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            a[u] = i < n ? x[i] : 0.f;
            b[u] = i < n && y ? y[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            if (i < n) {
                const float v = y ? __fadd_rn(a[u], b[u]) : a[u];
                if (y) x[i] = v;
                ss = __dadd_rn(ss, __dmul_rn((double)v, (double)v));
            }
        }
    }
    ss = block_reduce_d(ss, sh, 0);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)n), eps)));
    for (int i0 = threadIdx.x; i0 < n; i0 += B * bd) {
        float a[B], c[B];
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            a[u] = i < n ? x[i] : 0.f;
            c[u] = i < n ? w[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = i0 + u * bd;
            if (i < n) out[i] = __fmul_rn((float)__dmul_rn((double)a[u], inv), c[u]);
        }
    }
}

// The next token of the sequence: the next prompt id while the prompt lasts
// (main.go:229-231), else the best candidate of the w shards (value, id;
// ties to the lower id), recorded as generated. Position + 1.
__global__ void advance_kernel(const int *cands, int w, int *state, int *tokens, const int *prompt, int n_prompt) {
    step_entry();
    if (threadIdx.x != 0) return;
    const int pos = state[1];
    if (pos + 1 < n_prompt) {
        state[0] = prompt[pos + 1];
    } else {
        float best = __int_as_float(cands[0]);
        int idx = cands[1];
        for (int k = 1; k < w; k++) {
            const float v = __int_as_float(cands[2 * k]);
            const int i = cands[2 * k + 1];
            if (v > best || (v == best && i < idx)) best = v, idx = i;
        }
        tokens[state[2]] = idx;
        state[0] = idx;
        state[2] += 1;
    }
    state[1] = pos + 1;
}

// out[r][out_col0 + j] = in[r][in_col0 + j] for j < ncols.
__global__ void copy_cols_kernel(const float *in, int in_cols, int in_col0, float *out, int out_cols, int out_col0,
                                 int rows, int ncols) {
    step_entry();
    const size_t total = (size_t)rows * ncols;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / ncols), j = (int)(e % ncols);
        out[(size_t)r * out_cols + out_col0 + j] = in[(size_t)r * in_cols + in_col0 + j];
    }
}

// ---- engine -------------------------------------------------------------------
struct Layer {
    TqMatrixDev qkv{}, o{}, gu{}, down{};
    float *kc = nullptr, *vc = nullptr; // [ctx][kvd]
};

struct Qwen {
    int device = 0, rank = 0, world = 1;
    tq_qwen_config c{};
    int hd = 0, group = 0, wa = 1, ashard = 0, nq = 0, nkv = 0, qd = 0, kvd = 0;
    int orow0 = 0, orows = 0, arow = 0, fcols = 0, vcols = 0, voff = 0;
    cudaStream_t st = nullptr;
    TqScratch scr{};
    ncclComm_t comm = nullptr;
    float *embed = nullptr, *ones = nullptr, *zeros = nullptr;
    std::vector<Layer> L;
    TqMatrixDev lm{};
    float *x, *a, *qkv, *att, *y, *h, *logits;
    double *rope = nullptr; // the step's RoPE table [hd/2][2]
    int *state = nullptr, *tokens = nullptr, *cand = nullptr, *cands = nullptr, *prompt = nullptr, *part = nullptr;
    AttScratch att_scr;
    int prompt_cap = 0;
    cudaGraphExec_t graph = nullptr;
    int graph_prompt = -1; // the prompt length baked into the graph (advance_kernel)
    std::vector<void *> allocs;
};

std::mutex g_q_mu;
std::unordered_map<uint64_t, std::shared_ptr<Qwen>> g_qwens;
uint64_t g_next_qwen = 1;

#define TRY(expr)                                                                                                      \
    do {                                                                                                               \
        cudaError_t e_ = (expr);                                                                                       \
        if (e_ != cudaSuccess) return e_;                                                                              \
    } while (0)

cudaError_t dalloc(Qwen &m, void **p, size_t bytes) {
    cudaError_t e = tq_dev_malloc(p, bytes);
    if (e == cudaSuccess) m.allocs.push_back(*p);
    return e;
}

unsigned grid_for(size_t n) {
    size_t g = (n + kThreads - 1) / kThreads;
    return (unsigned)(g < 148 * 16 ? (g ? g : 1) : 148 * 16);
}

void destroy(Qwen &m) {
    if (m.st) cudaStreamSynchronize(m.st);
    if (m.graph) cudaGraphExecDestroy(m.graph); // before the communicator it holds
    m.graph = nullptr;
    if (m.comm) g_nccl.commDestroy(m.comm);
    m.comm = nullptr;
    for (Layer &l : m.L)
        for (TqMatrixDev *w : {&l.qkv, &l.o, &l.gu, &l.down}) tq_release_matrix(w);
    tq_release_matrix(&m.lm);
    for (void *p : m.allocs) cudaFree(p);
    m.allocs.clear();
    if (m.st) tq_scratch_release(m.device, m.st);
    if (m.st) cudaStreamDestroy(m.st);
    m.st = nullptr;
}

// Quantizes the fp32 shard buf [rows x cols] into *w (int4).
cudaError_t quantize_shard(Qwen &m, const float *buf, int rows, int cols, TqMatrixDev *w, int *rc) {
    if ((*rc = tq_alloc_matrix(4, rows, cols, w, m.st)) != TQ_OK) return cudaErrorMemoryAllocation;
    return tq_launch_quantize(*w, buf, m.st);
}

cudaError_t copy_cols(Qwen &m, const float *in, int in_cols, int in_col0, float *out, int out_cols, int out_col0,
                      int rows, int ncols) {
    copy_cols_kernel<<<grid_for((size_t)rows * ncols), kThreads, 0, m.st>>>(in, in_cols, in_col0, out, out_cols,
                                                                            out_col0, rows, ncols);
    return cudaGetLastError();
}

cudaError_t build(Qwen &m, uint64_t seed, float sigma, int *rc) {
    const tq_qwen_config &c = m.c;
    const int d = c.d, ffn = c.ffn;
    const int kv_full = c.n_kv * m.hd;
    TRY(cudaStreamCreateWithFlags(&m.st, cudaStreamNonBlocking));
    TRY(dalloc(m, (void **)&m.embed, sizeof(float) * (size_t)c.vocab * d));
    TRY(tq_launch_synth(m.embed, (size_t)c.vocab * d, seed, 1, sigma, m.st));
    const size_t vec = (size_t)(d > m.qd + 2 * m.kvd ? d : m.qd + 2 * m.kvd);
    TRY(dalloc(m, (void **)&m.ones, sizeof(float) * vec));
    TRY(dalloc(m, (void **)&m.zeros, sizeof(float) * vec));
    fill_kernel<<<grid_for(vec), kThreads, 0, m.st>>>(m.ones, 1.f, vec);
    fill_kernel<<<grid_for(vec), kThreads, 0, m.st>>>(m.zeros, 0.f, vec);
    TRY(cudaGetLastError());
    // fp32 scratch: the largest full matrix, and the largest (fused) shard
    size_t full = (size_t)d * c.vocab, shard = (size_t)d * m.vcols;
    for (size_t n : {(size_t)d * d, (size_t)d * kv_full, (size_t)d * ffn}) full = n > full ? n : full;
    for (size_t n : {(size_t)d * (m.qd + 2 * m.kvd), (size_t)d * 2 * m.fcols}) shard = n > shard ? n : shard;
    float *wfull, *wshard;
    TRY(tq_dev_malloc((void **)&wfull, sizeof(float) * full));
    cudaError_t e = tq_dev_malloc((void **)&wshard, sizeof(float) * shard);
    if (e != cudaSuccess) {
        cudaFree(wfull);
        return e;
    }
    auto run = [&]() -> cudaError_t {
        m.L.resize(c.n_layer);
        for (int l = 0; l < c.n_layer; l++) {
            Layer &ly = m.L[l];
            const uint64_t s0 = 32 + 16 * (uint64_t)l;
            const int qkvc = m.qd + 2 * m.kvd;
            // q | k | v columns of this GPU's attention heads
            TRY(tq_launch_synth(wfull, (size_t)d * d, seed, s0, sigma, m.st));
            TRY(copy_cols(m, wfull, d, m.ashard * m.qd, wshard, qkvc, 0, d, m.qd));
            TRY(tq_launch_synth(wfull, (size_t)d * kv_full, seed, s0 + 1, sigma, m.st));
            TRY(copy_cols(m, wfull, kv_full, m.ashard * m.kvd, wshard, qkvc, m.qd, d, m.kvd));
            TRY(tq_launch_synth(wfull, (size_t)d * kv_full, seed, s0 + 2, sigma, m.st));
            TRY(copy_cols(m, wfull, kv_full, m.ashard * m.kvd, wshard, qkvc, m.qd + m.kvd, d, m.kvd));
            TRY(quantize_shard(m, wshard, d, qkvc, &ly.qkv, rc));
            // o_proj rows [orow0, orow0 + orows)
            TRY(tq_launch_synth(wfull, (size_t)d * d, seed, s0 + 3, sigma, m.st));
            TRY(quantize_shard(m, wfull + (size_t)m.orow0 * d, m.orows, d, &ly.o, rc));
            // gate | up columns [rank * fcols, + fcols)
            TRY(tq_launch_synth(wfull, (size_t)d * ffn, seed, s0 + 4, sigma, m.st));
            TRY(copy_cols(m, wfull, ffn, m.rank * m.fcols, wshard, 2 * m.fcols, 0, d, m.fcols));
            TRY(tq_launch_synth(wfull, (size_t)d * ffn, seed, s0 + 5, sigma, m.st));
            TRY(copy_cols(m, wfull, ffn, m.rank * m.fcols, wshard, 2 * m.fcols, m.fcols, d, m.fcols));
            TRY(quantize_shard(m, wshard, d, 2 * m.fcols, &ly.gu, rc));
            // down rows [rank * fcols, + fcols)
            TRY(tq_launch_synth(wfull, (size_t)ffn * d, seed, s0 + 6, sigma, m.st));
            TRY(quantize_shard(m, wfull + (size_t)m.rank * m.fcols * d, m.fcols, d, &ly.down, rc));
            TRY(dalloc(m, (void **)&ly.kc, sizeof(float) * (size_t)c.ctx * m.kvd));
            TRY(dalloc(m, (void **)&ly.vc, sizeof(float) * (size_t)c.ctx * m.kvd));
            TRY(cudaStreamSynchronize(m.st)); // wfull / wshard are reused by the next matrix
        }
        // lm head columns [voff, voff + vcols)
        TRY(tq_launch_synth(wfull, (size_t)d * c.vocab, seed, 2, sigma, m.st));
        TRY(copy_cols(m, wfull, c.vocab, m.voff, wshard, m.vcols, 0, d, m.vcols));
        TRY(quantize_shard(m, wshard, d, m.vcols, &m.lm, rc));
        return cudaStreamSynchronize(m.st);
    };
    e = run();
    cudaFree(wfull);
    cudaFree(wshard);
    TRY(e);
    TRY(dalloc(m, (void **)&m.x, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.a, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.qkv, sizeof(float) * (m.qd + 2 * m.kvd)));
    TRY(dalloc(m, (void **)&m.att, sizeof(float) * m.qd));
    TRY(dalloc(m, (void **)&m.y, sizeof(float) * d));
    TRY(dalloc(m, (void **)&m.h, sizeof(float) * m.fcols));
    TRY(dalloc(m, (void **)&m.logits, sizeof(float) * m.vcols));
    TRY(dalloc(m, (void **)&m.state, sizeof(int) * 4));
    TRY(dalloc(m, (void **)&m.tokens, sizeof(int) * (size_t)(c.ctx + 1)));
    TRY(dalloc(m, (void **)&m.cand, sizeof(int) * 2));
    TRY(dalloc(m, (void **)&m.cands, sizeof(int) * 2 * m.world));
    TRY(dalloc(m, (void **)&m.part, sizeof(int) * 2 * kArgBlocks));
    void *ab = nullptr;
    TRY(dalloc(m, &ab, att_scratch_bytes(m.nq, c.ctx, m.hd)));
    TRY(att_scratch(ab, m.nq, c.ctx, m.hd, m.st, &m.att_scr));
    TRY(dalloc(m, (void **)&m.rope, sizeof(double) * m.hd));
    if ((*rc = tq_scratch_for(m.device, m.st, &m.scr, 1)) != TQ_OK) return cudaErrorMemoryAllocation;
    return cudaSuccess;
}

cudaError_t nccl_err(ncclResult_t r) { return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown; }

// One step (model.go:232-307) for the state's token at the state's position.
// The gate|up matvec ends with SiLU(gate) * up; the attention's scores pass
// applies RoPE and fills the caches. A residual add and the RMSNorm after it
// are one launch (measured on B200 at the 7B shape: 401 tokens/s, against 391
// with that norm done by the matvec's last CTA and 326 when the next matvec
// was also let in early beside it).
cudaError_t step(Qwen &m, int n_prompt) {
    const int d = m.c.d;
    TRY(step_launch(embed_norm_kernel, dim3(1), dim3(1024), 0, m.st, m.embed, m.state, m.x, m.ones, m.a, d, m.c.eps,
                    m.rope, m.hd, m.c.theta));
    AttRope rope;
    rope.cs = m.rope;
    rope.k = m.qkv + m.qd;
    rope.v = m.qkv + m.qd + m.kvd;
    rope.qbias = m.zeros;
    rope.kbias = m.zeros + m.qd;
    rope.vbias = m.zeros + m.qd + m.kvd;
    const float *pending = nullptr; // residual still to be added to x (the previous down_proj output)
    for (Layer &ly : m.L) {
        if (pending)
            TRY(step_launch(rmsnorm_kernel, dim3(1), dim3(1024), 0, m.st, m.x, pending, m.ones, m.a, d, m.c.eps));
        TRY(tq_launch_matmul(ly.qkv, m.a, m.qkv, 1, m.scr, m.st));
        rope.kc = ly.kc;
        rope.vc = ly.vc;
        TRY(decode_attention(m.qkv, ly.kc, ly.vc, m.kvd, m.att, m.state, m.nq, m.hd, m.group,
                             1.0 / sqrt((double)m.hd), m.att_scr, m.st, rope));
        TRY(tq_launch_matmul(ly.o, m.att + m.arow, m.y, 1, m.scr, m.st));
        if (m.world > 1) TRY(nccl_err(g_nccl.allReduce(m.y, m.y, d, ncclFloat32, ncclSum, m.comm, m.st)));
        TRY(step_launch(rmsnorm_kernel, dim3(1), dim3(1024), 0, m.st, m.x, m.y, m.ones, m.a, d, m.c.eps)); // x += o_proj, then norm
        TRY(tq_launch_cmv_epi(ly.gu, m.a, m.h, m.scr, m.st, TQ_EPI_SWIGLU, tq_matvec_uses_tmv()));
        TRY(tq_launch_matmul(ly.down, m.h, m.y, 1, m.scr, m.st));
        if (m.world > 1) TRY(nccl_err(g_nccl.allReduce(m.y, m.y, d, ncclFloat32, ncclSum, m.comm, m.st)));
        pending = m.y;
        TRY(cudaGetLastError());
    }
    if (pending) TRY(step_launch(rmsnorm_kernel, dim3(1), dim3(1024), 0, m.st, m.x, pending, m.ones, m.a, d, m.c.eps));
    TRY(tq_launch_matmul(m.lm, m.a, m.logits, 1, m.scr, m.st));
    TRY(greedy_pick(m.logits, m.vcols, m.voff, m.part, m.cand, m.state, m.tokens, -1, 0, m.st));
    if (m.world > 1)
        TRY(nccl_err(g_nccl.allGather(m.cand, m.cands, 2, ncclInt32, m.comm, m.st)));
    else
        TRY(cudaMemcpyAsync(m.cands, m.cand, sizeof(int) * 2, cudaMemcpyDeviceToDevice, m.st));
    TRY(step_launch(advance_kernel, dim3(1), dim3(32), 0, m.st, m.cands, m.world, m.state, m.tokens, m.prompt, n_prompt));
    return cudaGetLastError();
}

// How rank `rank` of `world` GPUs shards a model (the header's
// tq_qwen_shard_plan): attention ways wa (world when it divides the KV heads,
// else the KV heads, repeated over world / n_kv GPUs), this rank's attention
// shard, its o_proj rows, MLP columns (= down rows) and lm-head columns.
struct ShardPlan {
    int wa, ashard, nq, nkv, orow0, orows, fcols, vcols, voff;
};
int shard_plan(const tq_qwen_config &c, int world, int rank, ShardPlan *p) {
    if (c.n_layer < 1 || c.n_head < 1 || c.n_kv < 1 || c.d < 1 || c.ffn < 1 || c.vocab < 1 || c.ctx < 1 ||
        c.n_head % c.n_kv || c.d % c.n_head || (c.d / c.n_head) % 2)
        return tq_fail(TQ_ERR_ARG, "tensai: bad Qwen2 configuration");
    if (world < 1 || rank < 0 || rank >= world)
        return tq_fail(TQ_ERR_ARG, "tensai: bad rank %d of world %d", rank, world);
    if (c.n_kv % world == 0)
        p->wa = world;
    else if (world % c.n_kv == 0)
        p->wa = c.n_kv;
    else
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: %d GPUs do not split %d KV heads", world, c.n_kv);
    if (c.d % world || (c.d / world) % TQ_GROUP || c.ffn % world || (c.ffn / world) % TQ_GROUP || c.vocab % world ||
        (c.vocab / world) % 2)
        return tq_fail(TQ_ERR_UNSUPPORTED,
                       "tensai: d/world and ffn/world must be whole 64-row groups and vocab/world even");
    p->ashard = rank * p->wa / world;
    p->nq = c.n_head / p->wa;
    p->nkv = c.n_kv / p->wa;
    p->orows = c.d / world;
    p->orow0 = rank * p->orows;
    p->fcols = c.ffn / world;
    p->vcols = c.vocab / world;
    p->voff = rank * p->vcols;
    return TQ_OK;
}

std::shared_ptr<Qwen> find(uint64_t h, int *rc) {
    std::lock_guard<std::mutex> lk(g_q_mu);
    auto it = g_qwens.find(h);
    if (it == g_qwens.end()) {
        *rc = tq_fail(TQ_ERR_HANDLE, "tensai: invalid or freed model handle %llu", (unsigned long long)h);
        return nullptr;
    }
    return it->second;
}

} // namespace

extern "C" {

int tq_nccl_unique_id(void *id) {
    if (!id) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId u;
    ncclResult_t r = g_nccl.getUniqueId(&u);
    if (r != ncclSuccess) return tq_fail(TQ_ERR_CUDA, "tensai: ncclGetUniqueId: %s", g_nccl.errorString(r));
    static_assert(sizeof(ncclUniqueId) == TQ_NCCL_ID_BYTES, "NCCL unique id size");
    std::memcpy(id, &u, sizeof u);
    return TQ_OK;
}

int tq_qwen_create(const tq_qwen_config *cfg, uint64_t seed, float sigma, int rank, int world, const void *nccl_id,
                   uint64_t *model) {
    if (!cfg || !model) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    const tq_qwen_config &c = *cfg;
    ShardPlan sp;
    int rc0 = shard_plan(c, world, rank, &sp);
    if (rc0) return rc0;
    if (world > 1 && !nccl_id)
        return tq_fail(TQ_ERR_ARG, "tensai: bad rank %d of world %d (world > 1 needs an NCCL id)", rank, world);
    if (c.ctx > 6144) return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: context %d exceeds 6144", c.ctx);
    auto m = std::make_shared<Qwen>();
    m->c = c;
    m->rank = rank;
    m->world = world;
    m->hd = c.d / c.n_head;
    m->group = c.n_head / c.n_kv;
    m->wa = sp.wa;
    m->ashard = sp.ashard;
    m->nq = sp.nq;
    m->nkv = sp.nkv;
    m->qd = m->nq * m->hd;
    m->kvd = m->nkv * m->hd;
    m->orows = sp.orows;
    m->orow0 = sp.orow0;
    m->arow = m->orow0 - m->ashard * m->qd;
    m->fcols = sp.fcols;
    m->vcols = sp.vcols;
    m->voff = sp.voff;
    int rc = TQ_OK;
    cudaError_t e = cudaGetDevice(&m->device);
    if (e == cudaSuccess && world > 1) {
        if ((rc = load_nccl()) != TQ_OK) return rc;
        ncclUniqueId u;
        std::memcpy(&u, nccl_id, sizeof u);
        ncclResult_t r = g_nccl.commInitRank(&m->comm, world, u, rank);
        if (r != ncclSuccess) return tq_fail(TQ_ERR_CUDA, "tensai: ncclCommInitRank: %s", g_nccl.errorString(r));
    }
    if (e == cudaSuccess) e = build(*m, seed, sigma, &rc);
    if (e != cudaSuccess || rc != TQ_OK) {
        destroy(*m);
        return rc != TQ_OK ? rc : tq_cuda_fail(e, "Qwen2 model build");
    }
    std::lock_guard<std::mutex> lk(g_q_mu);
    *model = g_next_qwen++;
    g_qwens[*model] = m;
    return TQ_OK;
}

int tq_qwen_generate(uint64_t model, const int *prompt, int n_prompt, int n_gen, int *tokens, float *times_ms) {
    int rc = TQ_OK;
    auto m = find(model, &rc);
    if (!m) return rc;
    if (!prompt || !tokens || n_prompt < 1 || n_gen < 1) return tq_fail(TQ_ERR_ARG, "tensai: bad generate arguments");
    if (n_prompt + n_gen - 1 > m->c.ctx)
        return tq_fail(TQ_ERR_ARG, "tensai: %d prompt + %d generated tokens exceed the context of %d", n_prompt, n_gen,
                       m->c.ctx);
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= m->c.vocab)
            return tq_fail(TQ_ERR_ARG, "tensai: prompt token %d out of range [0, %d)", prompt[i], m->c.vocab);
    cudaError_t e = cudaSetDevice(m->device);
    if (e == cudaSuccess && n_prompt > m->prompt_cap) {
        if (m->graph) cudaGraphExecDestroy(m->graph); // the graph holds the old prompt buffer
        m->graph = nullptr;
        e = dalloc(*m, (void **)&m->prompt, sizeof(int) * (size_t)n_prompt);
        if (e == cudaSuccess) m->prompt_cap = n_prompt;
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->prompt, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, m->st);
    cudaEvent_t ev[3] = {};
    for (int i = 0; i < 3 && e == cudaSuccess; i++) e = cudaEventCreate(&ev[i]);
    if (e == cudaSuccess) {
        set_state_kernel<<<1, 1, 0, m->st>>>(m->state, prompt[0], 0, 0);
        e = cudaGetLastError();
    }
    // The graph bakes in n_prompt through advance_kernel: rebuild it when it changes.
    if (e == cudaSuccess && m->graph && m->graph_prompt != n_prompt) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    if (e == cudaSuccess && !m->graph) {
        e = step(*m, n_prompt); // eager first step: kernel set-up outside the capture
        if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
        set_state_kernel<<<1, 1, 0, m->st>>>(m->state, prompt[0], 0, 0); // start the sequence over
        cudaGraph_t g = nullptr;
        if (e == cudaSuccess) e = cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal);
        if (e == cudaSuccess) {
            cudaError_t e1 = step(*m, n_prompt);
            cudaError_t e2 = cudaStreamEndCapture(m->st, &g);
            e = e1 != cudaSuccess ? e1 : e2;
        }
        if (e == cudaSuccess) e = cudaGraphInstantiate(&m->graph, g, 0);
        if (g) cudaGraphDestroy(g);
        m->graph_prompt = n_prompt;
    }
    if (e == cudaSuccess) e = cudaEventRecord(ev[0], m->st);
    for (int i = 0; i < n_prompt && e == cudaSuccess; i++) e = cudaGraphLaunch(m->graph, m->st);
    if (e == cudaSuccess) e = cudaEventRecord(ev[1], m->st);
    for (int i = 1; i < n_gen && e == cudaSuccess; i++) e = cudaGraphLaunch(m->graph, m->st);
    if (e == cudaSuccess) e = cudaEventRecord(ev[2], m->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tokens, m->tokens, sizeof(int) * n_gen, cudaMemcpyDeviceToHost, m->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->st);
    if (e == cudaSuccess && times_ms) {
        e = cudaEventElapsedTime(&times_ms[0], ev[0], ev[1]);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&times_ms[1], ev[1], ev[2]);
    }
    for (auto &x : ev)
        if (x) cudaEventDestroy(x);
    if (e != cudaSuccess) return tq_cuda_fail(e, "Qwen2 generate");
    unsigned status = 0;
    if ((e = tq_read_status(m->scr, m->st, &status)) != cudaSuccess) return tq_cuda_fail(e, "status read");
    if (status & TQ_STATUS_TIMEOUT) return tq_fail(TQ_ERR_TIMEOUT, "tensai: a kernel timed out during decode");
    return TQ_OK;
}

int tq_qwen_shard_plan(const tq_qwen_config *cfg, int world, int rank, int *plan) {
    if (!cfg || !plan) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    ShardPlan sp;
    int rc = shard_plan(*cfg, world, rank, &sp);
    if (rc) return rc;
    const int hd = cfg->d / cfg->n_head;
    const int v[12] = {sp.ashard * sp.nq,    (sp.ashard + 1) * sp.nq,    sp.ashard * sp.nkv,
                       (sp.ashard + 1) * sp.nkv, sp.orow0,             sp.orow0 + sp.orows,
                       sp.ashard * sp.nq * hd, (sp.ashard + 1) * sp.nq * hd, rank * sp.fcols,
                       (rank + 1) * sp.fcols, sp.voff,               sp.voff + sp.vcols};
    std::memcpy(plan, v, sizeof v);
    return TQ_OK;
}

int tq_qwen_free(uint64_t model) {
    std::shared_ptr<Qwen> m;
    {
        std::lock_guard<std::mutex> lk(g_q_mu);
        auto it = g_qwens.find(model);
        if (it == g_qwens.end()) return TQ_OK;
        m = it->second;
        g_qwens.erase(it);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    destroy(*m);
    cudaSetDevice(prev);
    return TQ_OK;
}

} // extern "C"
