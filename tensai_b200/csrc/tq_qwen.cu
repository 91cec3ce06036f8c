// tq_qwen.cu — decode engine of tensai's Qwen2 example
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
// The o_proj and down partial sums meet in the step's exchanges: one kernel
// each that stores this GPU's partial into every peer's memory over NVLink
// and adds all ranks' partials in rank order, fused with the residual add and
// RMSNorm after it (the candidates likewise, in the advance kernel); NCCL's
// all-reduce where peer memory cannot be mapped, and for the batched
// prefill. NCCL is resolved at run time from the process (the library torch
// loaded). The whole step is one CUDA graph replayed per token.
//
// The prompt goes through the same step one token at a time (main.go:229-231):
// the step's last kernel feeds the next prompt id while the prompt lasts and
// the picked token after it (greedy, or the sample step with the caller's
// draws: tq_qwen_set_sampling); tq_qwen_set_prefill batches it instead.
//
// Numerics as the Go code: RMSNorm, RoPE, attention scores, softmax and SiLU
// in float64, residuals and the value sum in float32, products unfused.
#include <cuda_fp16.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
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
#include "tq_ptx.cuh"

namespace {

using namespace tqd_qwen;
using tqp::global_ns;
using tqp::kWaitNs;

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
    step_release_next();
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
// 301-303), then the norm of the new x, in one launch. Block b takes row b
// of [gridDim.x][n] x, y and out (one row in the decode step).
__global__ void rmsnorm_kernel(float *x, const float *y, const float *w, float *out, int n, double eps) {
    step_entry();
    step_wait_prev(); // launched early in the decode step (step_launch_early)
    step_release_next();
    __shared__ double sh[32];
    x += (size_t)blockIdx.x * n;
    out += (size_t)blockIdx.x * n;
    if (y) y += (size_t)blockIdx.x * n;
    constexpr int B = kNormBatch;
    const int bd = blockDim.x;
    double ss = 0;
    if (n <= B * bd) { // one batch per thread: the new x stays in registers, w comes with the first loads
        float a[B], b[B], c[B];
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = threadIdx.x + u * bd;
            a[u] = i < n ? x[i] : 0.f;
            b[u] = i < n && y ? y[i] : 0.f;
            c[u] = i < n ? w[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = threadIdx.x + u * bd;
            if (i < n) {
                if (y) a[u] = __fadd_rn(a[u], b[u]);
                if (y) x[i] = a[u];
                ss = __dadd_rn(ss, __dmul_rn((double)a[u], (double)a[u]));
            }
        }
        ss = block_reduce_d(ss, sh, 0);
        const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)n), eps)));
#pragma unroll
        for (int u = 0; u < B; u++) {
            const int i = threadIdx.x + u * bd;
            if (i < n) out[i] = __fmul_rn((float)__dmul_rn((double)a[u], inv), c[u]);
        }
        return;
    }
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

// ---- batched prefill (rows of a prompt chunk at once) ----

// Row r of a chunk: x[r] = embed[prompt[pos0 + r]] (model.go:239-240) and
// a[r] = rmsnorm(x[r]) * w, one block per row.
__global__ void embed_rows_kernel(const float *embed, const int *prompt, int pos0, float *x, const float *w, float *a,
                                  int d, double eps) {
    __shared__ double sh[32];
    const int r = blockIdx.x;
    const float *row = embed + (size_t)prompt[pos0 + r] * d;
    float *xr = x + (size_t)r * d, *ar = a + (size_t)r * d;
    double ss = 0;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = row[i];
        xr[i] = v;
        ss = __dadd_rn(ss, __dmul_rn((double)v, (double)v));
    }
    ss = block_reduce_d(ss, sh, 0);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)d), eps)));
    for (int i = threadIdx.x; i < d; i += blockDim.x) ar[i] = __fmul_rn((float)__dmul_rn((double)row[i], inv), w[i]);
}

// Row r of a chunk's fused q|k|v (position pos0 + r): the biases added, q and
// k rotated (model.go:244-250, 219-229: half-split pairs, float64), q in place,
// k and the biased v stored in the caches at the row's position.
__global__ void rope_rows_kernel(float *qkv, int qkvc, int nq, int nkv, int hd, int pos0, double theta,
                                 const float *qbias, const float *kbias, const float *vbias, float *kc, float *vc) {
    __shared__ double cs[kAttMaxHd];
    const int r = blockIdx.x, pos = pos0 + r, half = hd / 2, kvd = nkv * hd;
    rope_table(cs, pos, hd, theta);
    __syncthreads();
    float *q = qkv + (size_t)r * qkvc, *k = q + nq * hd, *v = k + kvd;
    for (int e = threadIdx.x; e < nq * half; e += blockDim.x) {
        const int h = e / half, i = e % half, j = h * hd + i;
        float r0, r1;
        rope_pair(cs, i, __fadd_rn(q[j], qbias[j]), __fadd_rn(q[j + half], qbias[j + half]), r0, r1);
        q[j] = r0;
        q[j + half] = r1;
    }
    float *kd = kc + (size_t)pos * kvd, *vd = vc + (size_t)pos * kvd;
    for (int e = threadIdx.x; e < nkv * half; e += blockDim.x) {
        const int h = e / half, i = e % half, j = h * hd + i;
        float r0, r1;
        rope_pair(cs, i, __fadd_rn(k[j], kbias[j]), __fadd_rn(k[j + half], kbias[j + half]), r0, r1);
        kd[j] = r0;
        kd[j + half] = r1;
    }
    for (int j = threadIdx.x; j < kvd; j += blockDim.x) vd[j] = __fadd_rn(v[j], vbias[j]);
}

// Causal attention of a prompt chunk's rows (model.go:262-293 per row):
// block (head h, rows r0 .. r0 + kPfRows - 1 of the chunk, positions pos0 +
// r) stages 64-position tiles of the head's cached k, then v, in shared
// memory with coalesced loads and uses each tile for all its rows, instead
// of every row reading the whole cache. Scores s_t = (q . k_t, float64
// products added in dimension order) * scale stay in shared memory; the
// softmax is float64 (max, then sum exp(s - max) per row over two warps),
// p_t = float32(exp(s_t - max) / sum) as the Go code forms it, and out = the
// sum over positions in order of p_t * v_t in float32.
constexpr int kPfRows = 4;   // query rows per block
constexpr int kPfTile = 64;  // cached positions per shared tile
constexpr int kPfThreads = 256;
__global__ void __launch_bounds__(kPfThreads) prefill_attention_kernel(const float *qkv, int qkvc, const float *kc,
                                                                      const float *vc, int kvd, float *out, int outc,
                                                                      int hd, int group, double scale, int pos0,
                                                                      int rows, int ctx /* scores row stride: >= the last position + 1 */) {
    extern __shared__ __align__(16) double pfd[];
    double *sc = pfd;                                               // [kPfRows][ctx]: scores, then p
    double *qs = sc + (size_t)kPfRows * ctx;                        // [kPfRows][hd], widened once
    const int TS = hd + 1;                                          // tile row stride: conflict-free rows
    float *ts = reinterpret_cast<float *>(qs + kPfRows * hd);      // [kPfTile][TS]: k, then v
    float *ps = ts + kPfTile * TS;                                  // [kPfRows][kPfTile]: the tile's p
    const int h = blockIdx.x, kvh = h / group, r0 = blockIdx.y * kPfRows;
    const int nr = min(kPfRows, rows - r0);
    const int tmax = pos0 + r0 + nr - 1; // the block's last position
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < kPfRows * hd; e += kPfThreads)
        qs[e] = e / hd < nr ? (double)qkv[(size_t)(r0 + e / hd) * qkvc + h * hd + e % hd] : 0.0;
    auto load_tile = [&](const float *cache, int k0, int nk) { // coalesced 16-byte loads, padded rows
        for (int e = threadIdx.x; e < nk * hd / 4; e += kPfThreads) {
            const int t = e / (hd / 4), i = 4 * (e % (hd / 4));
            const float4 v = *reinterpret_cast<const float4 *>(cache + (size_t)(k0 + t) * kvd + kvh * hd + i);
            float *d = ts + t * TS + i;
            d[0] = v.x;
            d[1] = v.y;
            d[2] = v.z;
            d[3] = v.w;
        }
    };
    // ---- scores: thread (position t of the tile, row rb) ----
    const int tt = threadIdx.x % kPfTile, rb = threadIdx.x / kPfTile;
    for (int k0 = 0; k0 <= tmax; k0 += kPfTile) {
        const int nk = min(kPfTile, tmax - k0 + 1);
        __syncthreads(); // the previous tile is no longer read
        load_tile(kc, k0, nk);
        __syncthreads();
        if (tt < nk && rb < nr && k0 + tt <= pos0 + r0 + rb) {
            const float *kt = ts + tt * TS;
            const double *qr = qs + rb * hd;
            double acc = 0;
            for (int i = 0; i < hd; i++) acc = __dadd_rn(acc, __dmul_rn(qr[i], (double)kt[i]));
            sc[(size_t)rb * ctx + k0 + tt] = __dmul_rn(acc, scale);
        }
    }
    __syncthreads();
    // ---- softmax per row, in shared memory: warps 2r and 2r + 1 take row r ----
    {
        const int r = warp >> 1, half = warp & 1;
        __shared__ double red[kPfThreads / 32][2];
        double mx = -INFINITY, sum = 0;
        const int pos = pos0 + r0 + r;
        double *srow = sc + (size_t)r * ctx;
        if (r < nr)
            for (int t = half * 32 + lane; t <= pos; t += 64) mx = fmax(mx, srow[t]);
        mx = warp_max_d(mx);
        if (lane == 0) red[warp][0] = mx;
        __syncthreads();
        mx = fmax(red[2 * r][0], red[2 * r + 1][0]);
        if (r < nr)
            for (int t = half * 32 + lane; t <= pos; t += 64) sum = __dadd_rn(sum, exp(__dsub_rn(srow[t], mx)));
        sum = warp_sum_d(sum);
        if (lane == 0) red[warp][1] = sum;
        __syncthreads();
        sum = __dadd_rn(red[2 * r][1], red[2 * r + 1][1]);
        if (r < nr)
            for (int t = half * 32 + lane; t <= pos; t += 64)
                srow[t] = (double)(float)__ddiv_rn(exp(__dsub_rn(srow[t], mx)), sum);
    }
    // ---- out = sum over positions in order of p_t v_t: thread (dimension, rows rsl, rsl + nsl, ..) ----
    const int dsl = threadIdx.x % hd, rsl = threadIdx.x / hd, nsl = kPfThreads / hd;
    float acc[kPfRows];
#pragma unroll
    for (int k = 0; k < kPfRows; k++) acc[k] = 0.f;
    for (int k0 = 0; k0 <= tmax; k0 += kPfTile) {
        const int nk = min(kPfTile, tmax - k0 + 1);
        __syncthreads();
        load_tile(vc, k0, nk);
        for (int e = threadIdx.x; e < kPfRows * kPfTile; e += kPfThreads) { // the tile's p, as float, once
            const int r = e / kPfTile, t = e % kPfTile;
            ps[e] = (r < nr && t < nk && k0 + t <= pos0 + r0 + r) ? (float)sc[(size_t)r * ctx + k0 + t] : 0.f;
        }
        __syncthreads();
        if (rsl < nsl) {
#pragma unroll
            for (int k = 0; k < kPfRows; k++) {
                const int r = rsl + k * nsl;
                if (k * nsl >= kPfRows || r >= nr) break;
                const int lim = min(nk, pos0 + r0 + r - k0 + 1); // this row's positions in the tile
                const float *pr = ps + r * kPfTile;
                float a = acc[k];
                for (int t = 0; t < lim; t++) a = __fadd_rn(a, __fmul_rn(pr[t], ts[t * TS + dsl]));
                acc[k] = a;
            }
        }
    }
    if (rsl < nsl)
#pragma unroll
        for (int k = 0; k < kPfRows; k++) {
            const int r = rsl + k * nsl;
            if (k * nsl < kPfRows && r < nr) out[(size_t)(r0 + r) * outc + h * hd + dsl] = acc[k];
        }
}

inline size_t prefill_attention_smem(int hd, int ctx) {
    return sizeof(double) * ((size_t)kPfRows * ctx + (size_t)kPfRows * hd) +
           sizeof(float) * ((size_t)kPfTile * (hd + 1) + (size_t)kPfRows * kPfTile);
}

// h[r][c] = float32(silu(gate)) * up of the fused [gate | up] rows (model.go:296-299).
__global__ void swiglu_rows_kernel(const float *gu, float *h, int f, int rows) {
    const size_t total = (size_t)rows * f;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const size_t r = e / f, c = e % f;
        const double g = (double)gu[r * 2 * f + c];
        h[e] = __fmul_rn((float)__ddiv_rn(g, __dadd_rn(1.0, exp(-g))), gu[r * 2 * f + f + c]);
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

// ---- one-shot exchange over NVLink peer memory -----------------------------------
// Each rank owns a slot area of [2 parities][world][cap] 8-byte words in its
// own HBM, mapped into every other rank by CUDA IPC. Exchange call e (1, 2, …
// counted per rank in ctl[0]; every rank makes the same calls) stores the
// rank's words (e << 32 | payload) into slot[e & 1][rank] of every peer, then
// waits in its own area for the words of epoch e from every peer. A 64-bit
// store arrives whole, so the epoch half vouches for the payload half: no
// fence or flag round trip. Two parities suffice: a rank stores into parity
// (e + 2) & 1 only after it has every peer's words of call e + 1, which a peer
// sends only after it has finished reading call e.
// Every wait is bounded (kWaitNs): a wait that runs out sets TQ_STATUS_TIMEOUT
// and ctl[1], after which later calls wait no more (their sums are garbage;
// the status fails the generate call).
constexpr int kArMaxWorld = 8;
constexpr int kArBatch = 8; // words loaded per thread before the first check
struct ArLink {
    unsigned long long *slot[kArMaxWorld]; // rank r's slot area as mapped here (own included)
    unsigned *ctl;                         // [0] calls done, [1] a wait ran out
    int world, rank, cap;
};

__device__ __forceinline__ void st_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool ar_is(unsigned long long w, unsigned e) { return (unsigned)(w >> 32) == e; }

// One thread: bounded wait for the word at p to carry epoch e.
__device__ __noinline__ unsigned long long ar_wait(const unsigned long long *p, unsigned e, volatile int *abort,
                                                   unsigned *ctl, unsigned *status) {
    unsigned long long v = ld_sys_u64(p);
    if (ar_is(v, e) || *abort) return v;
    const unsigned long long t0 = global_ns();
    for (unsigned it = 1;; it++) {
        __nanosleep(32);
        v = ld_sys_u64(p);
        if (ar_is(v, e) || *abort) return v;
        if ((it & 63) == 0 && global_ns() - t0 > kWaitNs) {
            atomicOr(status, TQ_STATUS_TIMEOUT);
            *abort = 1;
            ctl[1] = 1;
            return v;
        }
    }
}

// x += the sum over ranks of y (rank order, so every rank holds the same
// bits), then out = RMSNorm(x) * w: the o_proj / down_proj all-reduce fused
// with the residual add and norm after it (rmsnorm_kernel's numerics). One
// block; peers' words are staged in dynamic shared memory ((world-1) x n floats).
__global__ void __launch_bounds__(1024) ar_rmsnorm_kernel(ArLink L, float *x, const float *y, const float *w,
                                                          float *out, int n, double eps, unsigned *status) {
    step_entry();
    extern __shared__ float recv[]; // [world-1][n], peers in the order rank+1, rank+2, …
    __shared__ double sh[32];
    __shared__ unsigned long long *slot[kArMaxWorld];
    __shared__ unsigned s_e;
    __shared__ volatile int abort;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int r = 0; r < kArMaxWorld; r++) slot[r] = L.slot[r]; // constant indexes: no local copy
    }
    if (threadIdx.x == 0) {
        s_e = L.ctl[0] + 1;
        abort = L.ctl[1] != 0;
    }
    __syncthreads();
    const unsigned e = s_e;
    const int bd = blockDim.x, np = L.world - 1;
    const size_t par = (size_t)(e & 1) * L.world * L.cap;
    // n <= kArKeep * blockDim.x: x and w are loaded before the wait and the new x kept in registers
    constexpr int kArKeep = 4;
    const bool keep = n <= kArKeep * bd;
    float xs[kArKeep], ws[kArKeep];
    if (keep) {
#pragma unroll
        for (int u = 0; u < kArKeep; u++) {
            const int i = threadIdx.x + u * bd;
            xs[u] = i < n ? x[i] : 0.f;
            ws[u] = i < n ? w[i] : 0.f;
        }
    }
    for (int i = threadIdx.x; i < n; i += bd) {
        const unsigned long long wd = ((unsigned long long)e << 32) | __float_as_uint(y[i]);
        for (int k = 1; k <= np; k++) {
            const int r = L.rank + k < L.world ? L.rank + k : L.rank + k - L.world;
            st_sys_u64(slot[r] + par + (size_t)L.rank * L.cap + i, wd);
        }
    }
    const unsigned long long *mine = slot[L.rank] + par;
    const int total = np * n;
    for (int f0 = threadIdx.x; f0 < total; f0 += kArBatch * bd) {
        unsigned long long v[kArBatch];
#pragma unroll
        for (int u = 0; u < kArBatch; u++) {
            const int f = f0 + u * bd;
            if (f < total) {
                const int k = f / n, i = f - k * n;
                const int r = L.rank + 1 + k < L.world ? L.rank + 1 + k : L.rank + 1 + k - L.world;
                v[u] = ld_sys_u64(mine + (size_t)r * L.cap + i);
            }
        }
#pragma unroll
        for (int u = 0; u < kArBatch; u++) {
            const int f = f0 + u * bd;
            if (f < total) {
                const int k = f / n, i = f - k * n;
                const int r = L.rank + 1 + k < L.world ? L.rank + 1 + k : L.rank + 1 + k - L.world;
                if (!ar_is(v[u], e)) v[u] = ar_wait(mine + (size_t)r * L.cap + i, e, &abort, L.ctl, status);
                recv[f] = __uint_as_float((unsigned)v[u]);
            }
        }
    }
    __syncthreads();
    // the rank-order sum of element i, own partial y[i] included
    auto total_at = [&](int i) {
        float s = 0.f;
        for (int r = 0; r < L.world; r++) {
            const int k = r > L.rank ? r - L.rank - 1 : r + L.world - L.rank - 1;
            const float t = r == L.rank ? y[i] : recv[(size_t)k * n + i];
            s = r == 0 ? t : __fadd_rn(s, t);
        }
        return s;
    };
    double ss = 0;
    if (keep) {
#pragma unroll
        for (int u = 0; u < kArKeep; u++) {
            const int i = threadIdx.x + u * bd;
            if (i < n) {
                xs[u] = __fadd_rn(xs[u], total_at(i));
                x[i] = xs[u];
                ss = __dadd_rn(ss, __dmul_rn((double)xs[u], (double)xs[u]));
            }
        }
    } else {
        for (int i = threadIdx.x; i < n; i += bd) {
            const float xv = __fadd_rn(x[i], total_at(i));
            x[i] = xv;
            ss = __dadd_rn(ss, __dmul_rn((double)xv, (double)xv));
        }
    }
    ss = block_reduce_d(ss, sh, 0);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)n), eps)));
    if (keep) {
#pragma unroll
        for (int u = 0; u < kArKeep; u++) {
            const int i = threadIdx.x + u * bd;
            if (i < n) out[i] = __fmul_rn((float)__dmul_rn((double)xs[u], inv), ws[u]);
        }
    } else {
        for (int i = threadIdx.x; i < n; i += bd) out[i] = __fmul_rn((float)__dmul_rn((double)x[i], inv), w[i]);
    }
    if (threadIdx.x == 0) L.ctl[0] = e; // every thread read s_e before block_reduce_d's barriers
}

// The lm-head candidates (value, id) of every rank gathered over the same
// slots, then advance_kernel's pick: one launch for the gather and the step's
// last kernel.
__global__ void ar_advance_kernel(ArLink L, const int *cand, int *cands, int *state, int *tokens, const int *prompt,
                                  int n_prompt, unsigned *status) {
    step_entry();
    __shared__ unsigned long long *slot[kArMaxWorld];
    __shared__ unsigned s_e;
    __shared__ volatile int abort;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int r = 0; r < kArMaxWorld; r++) slot[r] = L.slot[r]; // constant indexes: no local copy
    }
    if (threadIdx.x == 0) {
        s_e = L.ctl[0] + 1;
        abort = L.ctl[1] != 0;
    }
    __syncthreads();
    const unsigned e = s_e;
    const size_t par = (size_t)(e & 1) * L.world * L.cap;
    const int t = threadIdx.x;
    if (t < 2) {
        const unsigned long long wd = ((unsigned long long)e << 32) | (unsigned)cand[t];
        for (int r = 0; r < L.world; r++)
            if (r != L.rank) st_sys_u64(slot[r] + par + (size_t)L.rank * L.cap + t, wd);
        cands[2 * L.rank + t] = cand[t];
    }
    if (t < 2 * L.world && t / 2 != L.rank) {
        const unsigned long long *p = slot[L.rank] + par + (size_t)(t / 2) * L.cap + (t & 1);
        unsigned long long v = ld_sys_u64(p);
        if (!ar_is(v, e)) v = ar_wait(p, e, &abort, L.ctl, status);
        cands[t] = (int)(unsigned)v;
    }
    __syncthreads();
    if (t != 0) return;
    __threadfence_block();
    const int pos = state[1];
    if (pos + 1 < n_prompt) {
        state[0] = prompt[pos + 1];
    } else {
        float best = __int_as_float(cands[0]);
        int idx = cands[1];
        for (int k = 1; k < L.world; k++) {
            const float v = __int_as_float(cands[2 * k]);
            const int i = cands[2 * k + 1];
            if (v > best || (v == best && i < idx)) best = v, idx = i;
        }
        tokens[state[2]] = idx;
        state[0] = idx;
        state[2] += 1;
    }
    state[1] = pos + 1;
    L.ctl[0] = e;
}

// ---- engine -------------------------------------------------------------------
struct Layer {
    TqMatrixDev qkv{}, o{}, gu{}, down{};
    float *kc = nullptr, *vc = nullptr; // [ctx][kvd]
    // norm weights (input, post-attention) and the q|k|v bias of this GPU's
    // heads: the engine's ones / zeros for random-init weights
    float *ln1 = nullptr, *ln2 = nullptr, *qkvb = nullptr;
    // checkpoint loading: q|k|v and gate|up rows staged until all parts came
    void *stage_qkv = nullptr, *stage_gu = nullptr;
    int got_qkv = 0, got_gu = 0, stage_dtype = -1;
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
    float *normw = nullptr; // the final norm's weight
    bool loaded = false;          // tq_qwen_create_empty: weights come from tq_qwen_load_tensor
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
    int prefill_rows = 0; // tq_qwen_set_prefill: 0 = token by token (the reference's), else rows per chunk
    float *px = nullptr, *pa = nullptr, *pqkv = nullptr, *patt = nullptr, *py = nullptr, *pgu = nullptr, *ph = nullptr;
    // the decode step's exchange: over peer memory (ar_on) or NCCL
    bool ar_on = false;
    ArLink ar{};
    unsigned long long *ar_area = nullptr; // this rank's slot area (exported by IPC)
    size_t ar_smem = 0;                    // ar_rmsnorm_kernel's dynamic shared memory
    // tq_qwen_set_sampling (one GPU): temp > 0 draws generated token k with draws[k]
    double temp = 0;
    double *draws = nullptr;
    int n_draws = 0;
    TqSampler smp;
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
    for (int r = 0; r < kArMaxWorld; r++)
        if (r != m.rank && m.ar.slot[r]) cudaIpcCloseMemHandle(m.ar.slot[r]);
    if (m.ar_area) cudaFree(m.ar_area);
    m.ar = ArLink{};
    m.ar_area = nullptr;
    m.ar_on = false;
    if (m.comm) g_nccl.commDestroy(m.comm);
    m.comm = nullptr;
    for (Layer &l : m.L) {
        for (TqMatrixDev *w : {&l.qkv, &l.o, &l.gu, &l.down}) tq_release_matrix(w);
        for (void *p : {l.stage_qkv, l.stage_gu})
            if (p) cudaFree(p);
        l.stage_qkv = l.stage_gu = nullptr;
    }
    tq_release_matrix(&m.lm);
    for (void *p : m.allocs) cudaFree(p);
    m.allocs.clear();
    tq_sampler_free(&m.smp);
    if (m.draws) cudaFree(m.draws);
    m.draws = nullptr;
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

cudaError_t buffers(Qwen &m, int *rc);

cudaError_t build(Qwen &m, uint64_t seed, float sigma, int *rc) {
    const tq_qwen_config &c = m.c;
    const int d = c.d, ffn = c.ffn;
    const int kv_full = c.n_kv * m.hd;
    TRY(cudaStreamCreateWithFlags(&m.st, cudaStreamNonBlocking));
    TRY(dalloc(m, (void **)&m.embed, sizeof(float) * (size_t)c.vocab * d));
    if (m.loaded)
        TRY(cudaMemsetAsync(m.embed, 0, sizeof(float) * (size_t)c.vocab * d, m.st));
    else
        TRY(tq_launch_synth(m.embed, (size_t)c.vocab * d, seed, 1, sigma, m.st));
    const size_t vec = (size_t)(d > m.qd + 2 * m.kvd ? d : m.qd + 2 * m.kvd);
    TRY(dalloc(m, (void **)&m.ones, sizeof(float) * vec));
    TRY(dalloc(m, (void **)&m.zeros, sizeof(float) * vec));
    fill_kernel<<<grid_for(vec), kThreads, 0, m.st>>>(m.ones, 1.f, vec);
    fill_kernel<<<grid_for(vec), kThreads, 0, m.st>>>(m.zeros, 0.f, vec);
    TRY(cudaGetLastError());
    m.normw = m.ones;
    if (m.loaded) { // checkpoint weights: zeroed matrices, per-layer norm weights (1) and biases (0) to fill
        const int qkvc = m.qd + 2 * m.kvd;
        auto vec_of = [&](float v, int n, float **out) -> cudaError_t {
            float *p = nullptr;
            TRY(dalloc(m, (void **)&p, sizeof(float) * n));
            fill_kernel<<<grid_for(n), kThreads, 0, m.st>>>(p, v, (size_t)n);
            *out = p;
            return cudaGetLastError();
        };
        TRY(vec_of(1.f, d, &m.normw));
        m.L.resize(c.n_layer);
        for (Layer &ly : m.L) {
            if ((*rc = tq_alloc_matrix(4, d, qkvc, &ly.qkv, m.st)) != TQ_OK ||
                (*rc = tq_alloc_matrix(4, m.orows, d, &ly.o, m.st)) != TQ_OK ||
                (*rc = tq_alloc_matrix(4, d, 2 * m.fcols, &ly.gu, m.st)) != TQ_OK ||
                (*rc = tq_alloc_matrix(4, m.fcols, d, &ly.down, m.st)) != TQ_OK)
                return cudaErrorMemoryAllocation;
            TRY(vec_of(1.f, d, &ly.ln1));
            TRY(vec_of(1.f, d, &ly.ln2));
            TRY(vec_of(0.f, qkvc, &ly.qkvb));
            TRY(dalloc(m, (void **)&ly.kc, sizeof(float) * (size_t)c.ctx * m.kvd));
            TRY(dalloc(m, (void **)&ly.vc, sizeof(float) * (size_t)c.ctx * m.kvd));
        }
        if ((*rc = tq_alloc_matrix(4, d, m.vcols, &m.lm, m.st)) != TQ_OK) return cudaErrorMemoryAllocation;
        TRY(cudaStreamSynchronize(m.st));
        return buffers(m, rc);
    }
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
            ly.ln1 = ly.ln2 = m.ones;
            ly.qkvb = m.zeros;
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
    return buffers(m, rc);
}

// The step's activation, state and scratch buffers (after the weights).
cudaError_t buffers(Qwen &m, int *rc) {
    const tq_qwen_config &c = m.c;
    const int d = c.d;
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
    TRY(att_setup(m.hd, m.group));
    TRY(dalloc(m, (void **)&m.rope, sizeof(double) * m.hd));
    if ((*rc = tq_scratch_for(m.device, m.st, &m.scr, 1)) != TQ_OK) return cudaErrorMemoryAllocation;
    return cudaSuccess;
}

cudaError_t nccl_err(ncclResult_t r) { return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown; }

// This rank's candidate (value, id) for the next token into cand: the greedy
// pick of its logits, or (one GPU, tq_qwen_set_sampling) the sample step of
// main.go:115-150 with the draw of generated token state[2] (the id only).
cudaError_t pick_next(Qwen &m) {
    if (m.temp > 0) return tq_launch_sample(m.smp, m.logits, m.vcols, m.temp, m.draws, m.state + 2, m.cand + 1, m.st);
    return greedy_pick(m.logits, m.vcols, m.voff, m.part, m.cand, m.state, m.tokens, -1, 0, m.st);
}

// Each rank's value of v gathered over NCCL (host ints, a few bytes each).
cudaError_t gather_host(Qwen &m, const void *v, size_t bytes, void *all) {
    void *dv = nullptr;
    cudaError_t e = cudaMalloc(&dv, bytes * (m.world + 1));
    if (e != cudaSuccess) return e;
    char *mine = (char *)dv + bytes * m.world;
    e = cudaMemcpyAsync(mine, v, bytes, cudaMemcpyHostToDevice, m.st);
    if (e == cudaSuccess) e = nccl_err(g_nccl.allGather(mine, dv, bytes, ncclInt8, m.comm, m.st));
    if (e == cudaSuccess) e = cudaMemcpyAsync(all, dv, bytes * m.world, cudaMemcpyDeviceToHost, m.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m.st);
    cudaFree(dv);
    return e;
}

// Sets up the decode step's exchange over peer memory (world > 1): the slot
// area, its IPC handle gathered over NCCL, every peer's area opened here. All
// ranks take the same steps and agree (a rank that cannot, or whose
// TENSAI_QWEN_EXCHANGE is "nccl", makes every rank keep the NCCL
// all-reduce). Errors of the agreement itself fail the model build.
cudaError_t ar_setup(Qwen &m) {
    const char *env = getenv("TENSAI_QWEN_EXCHANGE");
    const int cap = ((m.c.d > 2 ? m.c.d : 2) + 31) & ~31;
    const size_t smem = sizeof(float) * (size_t)(m.world - 1) * m.c.d;
    int ok = m.world <= kArMaxWorld && smem <= 200 * 1024 && !(env && !strcmp(env, "nccl"));
    const size_t bytes = sizeof(unsigned long long) * 2 * m.world * cap;
    if (ok) ok = cudaMalloc((void **)&m.ar_area, bytes) == cudaSuccess;
    if (ok) ok = cudaMemsetAsync(m.ar_area, 0, bytes, m.st) == cudaSuccess;
    if (ok && smem > 48 * 1024)
        ok = cudaFuncSetAttribute(ar_rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
             cudaSuccess;
    struct Rec {
        cudaIpcMemHandle_t h;
        int ok, pad[15];
    } rec{};
    if (ok) ok = cudaIpcGetMemHandle(&rec.h, m.ar_area) == cudaSuccess;
    if (ok) ok = cudaStreamSynchronize(m.st) == cudaSuccess; // zeroed before any peer can see it
    rec.ok = ok;
    cudaGetLastError(); // a failed optional step above leaves no sticky error
    std::vector<Rec> all(m.world);
    TRY(gather_host(m, &rec, sizeof rec, all.data()));
    for (const Rec &r : all) ok = ok && r.ok;
    for (int r = 0; r < m.world && ok; r++) {
        if (r == m.rank) {
            m.ar.slot[r] = m.ar_area;
            continue;
        }
        void *p = nullptr;
        ok = cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        if (ok) m.ar.slot[r] = (unsigned long long *)p;
    }
    cudaGetLastError();
    std::vector<int> okv(m.world);
    TRY(gather_host(m, &ok, sizeof ok, okv.data()));
    for (int v : okv) ok = ok && v;
    if (ok) {
        unsigned *ctl = nullptr;
        TRY(dalloc(m, (void **)&ctl, sizeof(unsigned) * 2));
        TRY(cudaMemsetAsync(ctl, 0, sizeof(unsigned) * 2, m.st));
        m.ar.ctl = ctl;
        m.ar.world = m.world;
        m.ar.rank = m.rank;
        m.ar.cap = cap;
        m.ar_smem = smem;
        m.ar_on = true;
        return cudaStreamSynchronize(m.st);
    }
    for (int r = 0; r < kArMaxWorld; r++)
        if (r != m.rank && m.ar.slot[r]) cudaIpcCloseMemHandle(m.ar.slot[r]);
    if (m.ar_area) cudaFree(m.ar_area);
    m.ar = ArLink{};
    m.ar_area = nullptr;
    return cudaSuccess;
}

// One step (model.go:232-307) for the state's token at the state's position.
// The gate|up matvec ends with SiLU(gate) * up; the attention's scores pass
// applies RoPE and fills the caches. A residual add and the RMSNorm after it
// are one launch (measured on B200 at the 7B shape: 401 tokens/s, against 391
// with that norm done by the matvec's last CTA and 326 when the next matvec
// was also let in early beside it).
cudaError_t step(Qwen &m, int n_prompt) {
    const int d = m.c.d;
    TRY(step_launch(embed_norm_kernel, dim3(1), dim3(1024), 0, m.st, m.embed, m.state, m.x, m.L[0].ln1, m.a, d,
                    m.c.eps, m.rope, m.hd, m.c.theta));
    AttRope rope;
    rope.cs = m.rope;
    rope.k = m.qkv + m.qd;
    rope.v = m.qkv + m.qd + m.kvd;
    // x += the all-reduced y (an o_proj or down_proj output), then a = RMSNorm(x) * w
    auto add_norm = [&](const float *w) -> cudaError_t {
        if (m.ar_on)
            return step_launch(ar_rmsnorm_kernel, dim3(1), dim3(1024), m.ar_smem, m.st, m.ar, m.x, m.y, w, m.a, d,
                               m.c.eps, m.scr.status);
        if (m.world > 1) {
            TRY(nccl_err(g_nccl.allReduce(m.y, m.y, d, ncclFloat32, ncclSum, m.comm, m.st)));
            return step_launch(rmsnorm_kernel, dim3(1), dim3(1024), 0, m.st, m.x, m.y, w, m.a, d, m.c.eps);
        }
        // 512 threads: small enough to be resident beside the matvec before it, ready when it completes
        return step_launch_early(rmsnorm_kernel, dim3(1), dim3(512), 0, m.st, m.x, m.y, w, m.a, d, m.c.eps);
    };
    bool pending = false; // the previous down_proj output is still to be added to x
    for (Layer &ly : m.L) {
        if (pending) TRY(add_norm(ly.ln1));
        TRY(tq_launch_matmul(ly.qkv, m.a, m.qkv, 1, m.scr, m.st));
        rope.qbias = ly.qkvb;
        rope.kbias = ly.qkvb + m.qd;
        rope.vbias = ly.qkvb + m.qd + m.kvd;
        rope.kc = ly.kc;
        rope.vc = ly.vc;
        TRY(decode_attention(m.qkv, ly.kc, ly.vc, m.kvd, m.att, m.state, m.nq, m.hd, m.group,
                             1.0 / sqrt((double)m.hd), m.att_scr, m.st, rope, m.world == 1));
        TRY(tq_launch_matmul(ly.o, m.att + m.arow, m.y, 1, m.scr, m.st));
        TRY(add_norm(ly.ln2)); // x += o_proj, then norm
        TRY(tq_launch_cmv_epi(ly.gu, m.a, m.h, m.scr, m.st, TQ_EPI_SWIGLU, tq_matvec_uses_tmv()));
        TRY(tq_launch_matmul(ly.down, m.h, m.y, 1, m.scr, m.st));
        pending = true;
        TRY(cudaGetLastError());
    }
    if (pending) TRY(add_norm(m.normw));
    TRY(tq_launch_matmul(m.lm, m.a, m.logits, 1, m.scr, m.st));
    TRY(pick_next(m));
    if (m.ar_on)
        return step_launch(ar_advance_kernel, dim3(1), dim3(32), 0, m.st, m.ar, m.cand, m.cands, m.state, m.tokens,
                           m.prompt, n_prompt, m.scr.status);
    if (m.world > 1)
        TRY(nccl_err(g_nccl.allGather(m.cand, m.cands, 2, ncclInt32, m.comm, m.st)));
    else
        TRY(cudaMemcpyAsync(m.cands, m.cand, sizeof(int) * 2, cudaMemcpyDeviceToDevice, m.st));
    TRY(step_launch(advance_kernel, dim3(1), dim3(32), 0, m.st, m.cands, m.world, m.state, m.tokens, m.prompt, n_prompt));
    return cudaGetLastError();
}

// The prompt in chunks of m.prefill_rows rows: each layer's matvecs as M-row
// matmuls (tq_launch_matmul: the tf32 tensor-core kernel from 16 rows), RoPE
// and the KV caches per row, the causal attention of each row over the
// cached positions, the same norms and epilogues as the step; then the last
// row's logits give the first generated token, and the state ends as the
// token-by-token prompt leaves it (the prompt's last position, one token
// generated).
cudaError_t prefill(Qwen &m, int n_prompt) {
    const int d = m.c.d, R = m.prefill_rows, qkvc = m.qd + 2 * m.kvd;
    const double scale = 1.0 / sqrt((double)m.hd);
    // rows of scores are as long as the prompt (not the context), so that two
    // blocks fit per SM for prompts up to about 2,600 positions
    const size_t pf_smem = prefill_attention_smem(m.hd, n_prompt);
    for (int c0 = 0; c0 < n_prompt; c0 += R) {
        const int rows = n_prompt - c0 < R ? n_prompt - c0 : R;
        embed_rows_kernel<<<rows, 1024, 0, m.st>>>(m.embed, m.prompt, c0, m.px, m.L[0].ln1, m.pa, d, m.c.eps);
        TRY(cudaGetLastError());
        for (size_t l = 0; l < m.L.size(); l++) {
            Layer &ly = m.L[l];
            if (l > 0) { // x += the previous layer's down_proj, then the norm
                rmsnorm_kernel<<<rows, 1024, 0, m.st>>>(m.px, m.py, ly.ln1, m.pa, d, m.c.eps);
                TRY(cudaGetLastError());
            }
            TRY(tq_launch_matmul(ly.qkv, m.pa, m.pqkv, rows, m.scr, m.st));
            rope_rows_kernel<<<rows, 256, 0, m.st>>>(m.pqkv, qkvc, m.nq, m.nkv, m.hd, c0, m.c.theta, ly.qkvb,
                                                     ly.qkvb + m.qd, ly.qkvb + m.qd + m.kvd, ly.kc, ly.vc);
            prefill_attention_kernel<<<dim3(m.nq, (rows + kPfRows - 1) / kPfRows), kPfThreads, pf_smem, m.st>>>(
                m.pqkv, qkvc, ly.kc, ly.vc, m.kvd, m.patt, m.qd, m.hd, m.group, scale, c0, rows, n_prompt);
            TRY(cudaGetLastError());
            TRY(tq_launch_matmul(ly.o, m.patt, m.py, rows, m.scr, m.st));
            if (m.world > 1)
                TRY(nccl_err(g_nccl.allReduce(m.py, m.py, (size_t)rows * d, ncclFloat32, ncclSum, m.comm, m.st)));
            rmsnorm_kernel<<<rows, 1024, 0, m.st>>>(m.px, m.py, ly.ln2, m.pa, d, m.c.eps); // x += o_proj, then norm
            TRY(cudaGetLastError());
            TRY(tq_launch_matmul(ly.gu, m.pa, m.pgu, rows, m.scr, m.st));
            swiglu_rows_kernel<<<grid_for((size_t)rows * m.fcols), kThreads, 0, m.st>>>(m.pgu, m.ph, m.fcols, rows);
            TRY(cudaGetLastError());
            TRY(tq_launch_matmul(ly.down, m.ph, m.py, rows, m.scr, m.st));
            if (m.world > 1)
                TRY(nccl_err(g_nccl.allReduce(m.py, m.py, (size_t)rows * d, ncclFloat32, ncclSum, m.comm, m.st)));
        }
    }
    // the prompt's last row: its final residual add and norm, the lm head, the pick
    const int last = (n_prompt - 1) % R;
    set_state_kernel<<<1, 1, 0, m.st>>>(m.state, 0, n_prompt - 1, 0);
    rmsnorm_kernel<<<1, 1024, 0, m.st>>>(m.px + (size_t)last * d, m.py + (size_t)last * d, m.normw, m.a, d, m.c.eps);
    TRY(cudaGetLastError());
    TRY(tq_launch_matmul(m.lm, m.a, m.logits, 1, m.scr, m.st));
    TRY(pick_next(m));
    if (m.world > 1)
        TRY(nccl_err(g_nccl.allGather(m.cand, m.cands, 2, ncclInt32, m.comm, m.st)));
    else
        TRY(cudaMemcpyAsync(m.cands, m.cand, sizeof(int) * 2, cudaMemcpyDeviceToDevice, m.st));
    advance_kernel<<<1, 32, 0, m.st>>>(m.cands, m.world, m.state, m.tokens, m.prompt, n_prompt);
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

static int qwen_create(const tq_qwen_config *cfg, uint64_t seed, float sigma, int rank, int world,
                       const void *nccl_id, bool loaded, uint64_t *model) {
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
    m->loaded = loaded;
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
    if (e == cudaSuccess && rc == TQ_OK && world > 1) e = ar_setup(*m);
    if (e != cudaSuccess || rc != TQ_OK) {
        destroy(*m);
        return rc != TQ_OK ? rc : tq_cuda_fail(e, "Qwen2 model build");
    }
    std::lock_guard<std::mutex> lk(g_q_mu);
    *model = g_next_qwen++;
    g_qwens[*model] = m;
    return TQ_OK;
}

int tq_qwen_create(const tq_qwen_config *cfg, uint64_t seed, float sigma, int rank, int world, const void *nccl_id,
                   uint64_t *model) {
    return qwen_create(cfg, seed, sigma, rank, world, nccl_id, false, model);
}

int tq_qwen_create_empty(const tq_qwen_config *cfg, uint64_t *model) {
    return qwen_create(cfg, 0, 0.f, 0, 1, nullptr, true, model);
}

int tq_qwen_load_tensor(uint64_t model, const char *name, const void *data, int dtype, int rows, int cols) {
    if (!name || !data) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    if (dtype != TQ_LINEAR_F32 && dtype != TQ_LINEAR_F16 && dtype != TQ_LINEAR_BF16)
        return tq_fail(TQ_ERR_ARG, "tensai: unknown tensor type %d", dtype);
    int rc = TQ_OK;
    auto m = find(model, &rc);
    if (!m) return rc;
    if (!m->loaded) return tq_fail(TQ_ERR_ARG, "tensai: %s: the model holds random-init weights", name);
    const tq_qwen_config &c = m->c;
    const int d = c.d, qd = m->qd, kvd = m->kvd, ffn = c.ffn;
    const size_t es = dtype == TQ_LINEAR_F32 ? 4 : 2;
    cudaError_t e = cudaSetDevice(m->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "tensor load");
    auto shape = [&](int r, int cc) {
        return rows == r && cols == cc ? TQ_OK
                                       : tq_fail(TQ_ERR_SHAPE, "tensai: %s is %d x %d, expected %d x %d", name, rows,
                                                 cols, r, cc);
    };
    auto widen = [&](float *dst) {
        widen_kernel<<<grid_for((size_t)rows * cols), kThreads, 0, m->st>>>(data, dtype, dst, (size_t)rows * cols);
        return cudaGetLastError();
    };
    // rows [row0, row0 + rows) of a fused [total x d] matrix staged in *stage;
    // once every part (bit) arrived, quantized into w and the stage freed
    auto stage = [&](Layer &ly, void **st, int *got, int bit, int all, int row0, int total, TqMatrixDev &w) {
        if (ly.stage_dtype >= 0 && ly.stage_dtype != dtype)
            return tq_fail(TQ_ERR_ARG, "tensai: %s: the parts of a fused matrix differ in type", name);
        cudaError_t err = cudaSuccess;
        if (!*st) err = tq_dev_malloc(st, es * (size_t)total * d);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(static_cast<char *>(*st) + es * (size_t)row0 * d, data, es * (size_t)rows * cols,
                                  cudaMemcpyDeviceToDevice, m->st);
        if (err != cudaSuccess) return tq_cuda_fail(err, "tensor staging");
        ly.stage_dtype = dtype;
        *got |= bit;
        if (*got == all) {
            err = tq_launch_quantize_linear(w, *st, dtype, m->st);
            if (err == cudaSuccess) err = cudaStreamSynchronize(m->st);
            cudaFree(*st);
            *st = nullptr;
            *got = 0;
            if (err != cudaSuccess) return tq_cuda_fail(err, "tensor quantize");
        }
        return TQ_OK;
    };
    auto linear = [&](TqMatrixDev &w) {
        cudaError_t err = tq_launch_quantize_linear(w, data, dtype, m->st);
        return err == cudaSuccess ? TQ_OK : tq_cuda_fail(err, "tensor quantize");
    };
    const std::string n(name);
    int l = -1, used = 0;
    char rest[96] = {};
    if (n == "model.embed_tokens.weight") {
        if ((rc = shape(c.vocab, d)) == TQ_OK && (e = widen(m->embed)) != cudaSuccess) rc = tq_cuda_fail(e, "embed");
    } else if (n == "model.norm.weight") {
        if ((rc = shape(1, d)) == TQ_OK && (e = widen(m->normw)) != cudaSuccess) rc = tq_cuda_fail(e, "norm");
    } else if (n == "lm_head.weight") {
        if ((rc = shape(c.vocab, d)) == TQ_OK) rc = linear(m->lm);
    } else if (std::sscanf(name, "model.layers.%d.%95s%n", &l, rest, &used) == 2 && (size_t)used == n.size() &&
               l >= 0 && l < c.n_layer) {
        Layer &ly = m->L[l];
        const std::string r(rest);
        const int qkvc = qd + 2 * kvd;
        if (r == "self_attn.q_proj.weight") {
            if ((rc = shape(qd, d)) == TQ_OK) rc = stage(ly, &ly.stage_qkv, &ly.got_qkv, 1, 7, 0, qkvc, ly.qkv);
        } else if (r == "self_attn.k_proj.weight") {
            if ((rc = shape(kvd, d)) == TQ_OK) rc = stage(ly, &ly.stage_qkv, &ly.got_qkv, 2, 7, qd, qkvc, ly.qkv);
        } else if (r == "self_attn.v_proj.weight") {
            if ((rc = shape(kvd, d)) == TQ_OK)
                rc = stage(ly, &ly.stage_qkv, &ly.got_qkv, 4, 7, qd + kvd, qkvc, ly.qkv);
        } else if (r == "self_attn.q_proj.bias" || r == "self_attn.k_proj.bias" || r == "self_attn.v_proj.bias") {
            const int off = r[10] == 'q' ? 0 : r[10] == 'k' ? qd : qd + kvd, len = r[10] == 'q' ? qd : kvd;
            if ((rc = shape(1, len)) == TQ_OK && (e = widen(ly.qkvb + off)) != cudaSuccess)
                rc = tq_cuda_fail(e, "bias");
        } else if (r == "self_attn.o_proj.weight") {
            if ((rc = shape(d, qd)) == TQ_OK) rc = linear(ly.o);
        } else if (r == "mlp.gate_proj.weight") {
            if ((rc = shape(ffn, d)) == TQ_OK) rc = stage(ly, &ly.stage_gu, &ly.got_gu, 1, 3, 0, 2 * ffn, ly.gu);
        } else if (r == "mlp.up_proj.weight") {
            if ((rc = shape(ffn, d)) == TQ_OK) rc = stage(ly, &ly.stage_gu, &ly.got_gu, 2, 3, ffn, 2 * ffn, ly.gu);
        } else if (r == "mlp.down_proj.weight") {
            if ((rc = shape(d, ffn)) == TQ_OK) rc = linear(ly.down);
        } else if (r == "input_layernorm.weight") {
            if ((rc = shape(1, d)) == TQ_OK && (e = widen(ly.ln1)) != cudaSuccess) rc = tq_cuda_fail(e, "norm");
        } else if (r == "post_attention_layernorm.weight") {
            if ((rc = shape(1, d)) == TQ_OK && (e = widen(ly.ln2)) != cudaSuccess) rc = tq_cuda_fail(e, "norm");
        } else {
            rc = tq_fail(TQ_ERR_ARG, "tensai: unknown Qwen2 tensor %s", name);
        }
    } else {
        rc = tq_fail(TQ_ERR_ARG, "tensai: unknown Qwen2 tensor %s", name);
    }
    if (rc != TQ_OK) return rc;
    if ((e = cudaStreamSynchronize(m->st)) != cudaSuccess) return tq_cuda_fail(e, "tensor load");
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
    if (m->temp > 0 && n_gen > m->n_draws)
        return tq_fail(TQ_ERR_ARG, "tensai: %d tokens to sample but %d draws set", n_gen, m->n_draws);
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
    if (m->prefill_rows > 0) {
        if (e == cudaSuccess) e = prefill(*m, n_prompt);
    } else {
        for (int i = 0; i < n_prompt && e == cudaSuccess; i++) e = cudaGraphLaunch(m->graph, m->st);
    }
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

int tq_qwen_set_sampling(uint64_t model, double temp, const double *draws, int n_draws) {
    int rc = TQ_OK;
    auto m = find(model, &rc);
    if (!m) return rc;
    if ((rc = tq_check_draws(temp, draws, n_draws)) != TQ_OK) return rc;
    if (temp > 0 && m->world > 1)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: sampling needs the whole vocabulary on one GPU (world %d)",
                       m->world);
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
        if (e == cudaSuccess) e = tq_sampler_alloc(&m->smp, m->vcols);
        if (e == cudaSuccess) m->temp = temp, m->n_draws = n_draws;
    }
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "sampling set-up");
}

int tq_qwen_exchange(uint64_t model, int *kind) {
    if (!kind) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    int rc = TQ_OK;
    auto m = find(model, &rc);
    if (!m) return rc;
    *kind = m->world == 1 ? TQ_EXCHANGE_NONE : m->ar_on ? TQ_EXCHANGE_PEER : TQ_EXCHANGE_NCCL;
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

int tq_qwen_set_prefill(uint64_t model, int rows) {
    int rc = TQ_OK;
    auto m = find(model, &rc);
    if (!m) return rc;
    if (rows != 0 && (rows < TQ_MM_MIN_ROWS || rows > TQ_MM_MAX_ROWS))
        return tq_fail(TQ_ERR_ARG, "tensai: prefill rows must be 0 or %d..%d, got %d", TQ_MM_MIN_ROWS, TQ_MM_MAX_ROWS,
                       rows);
    if (rows == 0) {
        m->prefill_rows = 0;
        return TQ_OK;
    }
    if (m->arow != 0 || m->orows != m->qd)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: batched prefill needs each GPU's attention heads to be its own "
                                           "(this shard repeats the attention: more GPUs than KV heads)");
    if (m->hd % 4 || m->hd > kAttMaxHd || kPfThreads % m->hd)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: batched prefill attention takes head sizes dividing %d",
                       kPfThreads);
    const size_t smem = prefill_attention_smem(m->hd, m->c.ctx);
    if (smem > 227 * 1024)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: batched prefill attention keeps %d rows of scores per block in "
                                           "shared memory: a context of %d positions is too long", kPfRows, m->c.ctx);
    cudaError_t e = cudaSetDevice(m->device);
    if (e == cudaSuccess && smem > 48 * 1024)
        e = cudaFuncSetAttribute(prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return tq_cuda_fail(e, "prefill set-up");
    if (rows > m->prefill_rows) {
        const int d = m->c.d, qkvc = m->qd + 2 * m->kvd;
        const std::pair<float **, size_t> bufs[] = {
            {&m->px, (size_t)d}, {&m->pa, (size_t)d}, {&m->pqkv, (size_t)qkvc}, {&m->patt, (size_t)m->qd},
            {&m->py, (size_t)d}, {&m->pgu, 2 * (size_t)m->fcols}, {&m->ph, (size_t)m->fcols}};
        for (const auto &b : bufs)
            if ((e = dalloc(*m, (void **)b.first, sizeof(float) * rows * b.second)) != cudaSuccess)
                return tq_cuda_fail(e, "prefill buffers");
        if ((rc = tq_scratch_for(m->device, m->st, &m->scr, rows)) != TQ_OK) return rc; // the matmul's partials
    }
    m->prefill_rows = rows;
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
