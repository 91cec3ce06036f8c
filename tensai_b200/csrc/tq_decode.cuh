// tq_decode.cuh — kernels shared by the greedy decode engines (tq_model.cu:
// GPT-2; tq_qwen.cu: Qwen2). Each restates one operation of tensai's example
// decode loops in the same float64 / float32 arithmetic as the Go code, with
// explicitly rounded intrinsics so that nvcc contracts nothing into an FMA
// that the Go code (gc at GOAMD64=v1) does not fuse.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

// Each including file names the namespace (TQD_NS) so that every
// translation unit gets its own, distinctly named copy of the kernels.
#ifndef TQD_NS
#error "define TQD_NS before including tq_decode.cuh"
#endif
namespace TQD_NS {

constexpr int kThreads = 256;

// ---- programmatic dependent launch -------------------------------------------
// With TQ_DECODE_PDL set by the including engine, every kernel of a decode step
// is launched with programmatic stream serialization and starts with
// step_entry: it lets the next kernel on the stream be scheduled at once, then
// waits until its predecessor has completed and its memory is visible
// (griddepcontrol.wait) before touching anything. A step's matvec is then
// resident and streams its weights while the small kernels before it run. A
// dependent grid is scheduled only after every CTA of its predecessor has
// started, so waiting CTAs never block an unscheduled predecessor. Without
// TQ_DECODE_PDL, launches are plain and step_entry is empty.
#ifndef TQ_DECODE_PDL
#error "define TQ_DECODE_PDL (0 or 1) before including tq_decode.cuh"
#endif
__device__ __forceinline__ void step_entry() {
#if TQ_DECODE_PDL
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
// For grids of hundreds of CTAs (the attention passes): wait only, so the
// successor is scheduled when this grid completes rather than early, and its
// CTAs do not sit resident beside this grid's.
__device__ __forceinline__ void step_entry_wait() {
#if TQ_DECODE_PDL
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
template <typename... KArgs, typename... Args>
inline cudaError_t step_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               Args... args) {
#if TQ_DECODE_PDL
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
#else
    kernel<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
    return cudaGetLastError();
#endif
}

// ---- reductions ---------------------------------------------------------------
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Block-wide sum (kind 0) or max (kind 1) of one double per thread; every
// thread gets the result. sh: 32 doubles of shared memory.
__device__ inline double block_reduce_d(double v, double *sh, int kind) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = kind ? warp_max_d(v) : warp_sum_d(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        double u = lane < nw ? sh[lane] : (kind ? -INFINITY : 0.0);
        u = kind ? warp_max_d(u) : warp_sum_d(u);
        if (lane == 0) sh[0] = u;
    }
    __syncthreads();
    return sh[0];
}

// ---- elementwise ------------------------------------------------------------------
// x += y + b (bias into the matvec output, then the residual add; b may be null).
__global__ void residual_kernel(float *x, const float *y, const float *b, int n, size_t total) {
    step_entry();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], b ? __fadd_rn(y[i], b[i % n]) : y[i]);
}

__global__ void fill_kernel(float *p, float v, size_t n) {
    step_entry();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}

// state = {token to feed, its position, tokens generated}
__global__ void set_state_kernel(int *state, int token, int pos, int generated) {
    step_entry();
    state[0] = token;
    state[1] = pos;
    state[2] = generated;
}

// ---- attention ----------------------------------------------------------------------
// One query row over cached positions 0..pos, query head blockIdx.x (its KV
// head: blockIdx.x / group), query row blockIdx.y: scores in float64 times
// `scale`, softmax in float64, p = float32(score / sum), out += p * v in
// float32 over positions in order (_example/gpt2/model.go:195-227;
// _example/qwen/model.go:262-293). Decode: pos from the state; prefill: the
// row index. Shared memory: ctx doubles + ctx floats.
__global__ void attention_kernel(const float *q, int qstride, const float *kc, const float *vc, int kvstride,
                                 float *out, int outstride, const int *state, int hd, int group, double scale,
                                 int prefill, int ctx) {
    step_entry();
    extern __shared__ double sc[];
    __shared__ double sh[32];
    const int h = blockIdx.x, r = blockIdx.y, kvh = h / group;
    const int pos = prefill ? r : state[1];
    const float *qr = q + (size_t)r * qstride + h * hd;
    double mx = -INFINITY;
    for (int t = threadIdx.x; t <= pos; t += blockDim.x) {
        const float *kt = kc + (size_t)t * kvstride + kvh * hd;
        double s = 0;
        for (int i = 0; i < hd; i++) s = __dadd_rn(s, __dmul_rn((double)qr[i], (double)kt[i]));
        s = __dmul_rn(s, scale);
        sc[t] = s;
        mx = fmax(mx, s);
    }
    mx = block_reduce_d(mx, sh, 1);
    double sum = 0;
    for (int t = threadIdx.x; t <= pos; t += blockDim.x) {
        const double e = exp(__dsub_rn(sc[t], mx));
        sc[t] = e;
        sum = __dadd_rn(sum, e);
    }
    sum = block_reduce_d(sum, sh, 0);
    float *p = reinterpret_cast<float *>(sc + ctx);
    for (int t = threadIdx.x; t <= pos; t += blockDim.x) p[t] = (float)__ddiv_rn(sc[t], sum);
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.f;
        for (int t = 0; t <= pos; t++) acc = __fadd_rn(acc, __fmul_rn(p[t], vc[(size_t)t * kvstride + kvh * hd + i]));
        out[(size_t)r * outstride + h * hd + i] = acc;
    }
}

inline size_t attention_smem(int ctx) { return (sizeof(double) + sizeof(float)) * (size_t)ctx; }

// ---- split-K decode attention -------------------------------------------------------
// The same attention for the decode step's single query row, spread over
// chunks of kAttChunk cached positions so that long contexts use every SM:
//   scores:   per (head, chunk): s_t = (q . k_t in float64) * scale, and the
//             chunk's max m_b and sum l_b = sum exp(s_t - m_b);
//   weights:  per (head, chunk): the softmax's global max M and sum
//             L = sum_b l_b exp(m_b - M) (chunks in order), p_t = float32(
//             exp(s_t - M) / L) as the Go code forms it, and the chunk's
//             float32 partial sum_t p_t * v_t (positions in order);
//   combine:  per head: the chunk partials summed in chunk order.
// Scratch (per engine): scores [heads][ctx] doubles, stats [heads][chunks][2]
// doubles, partials [heads][chunks][hd] floats.
constexpr int kAttChunk = 128;

__global__ void __launch_bounds__(128) att_scores_kernel(const float *q, const float *kc, int kvstride, const int *state,
                                                         int hd, int group, double scale, double *scores,
                                                         double *stats, int ctx, int nchunks) {
    step_entry_wait();
    __shared__ double ss[kAttChunk];
    __shared__ double sh[32];
    const int h = blockIdx.x, b = blockIdx.y, pos = state[1], t0 = b * kAttChunk;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, kvh = h / group;
    if (t0 > pos) return;
    const int t1 = min(t0 + kAttChunk, pos + 1);
    const float *qh = q + h * hd;
    for (int t = t0 + warp; t < t1; t += 4) {
        const float *kt = kc + (size_t)t * kvstride + kvh * hd;
        double s = 0;
        for (int i = lane; i < hd; i += 32) s = __dadd_rn(s, __dmul_rn((double)qh[i], (double)kt[i]));
        s = warp_sum_d(s);
        if (lane == 0) ss[t - t0] = __dmul_rn(s, scale);
    }
    __syncthreads();
    double mx = -INFINITY;
    for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) mx = fmax(mx, ss[t - t0]);
    mx = block_reduce_d(mx, sh, 1);
    double l = 0;
    for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) {
        l = __dadd_rn(l, exp(__dsub_rn(ss[t - t0], mx)));
        scores[(size_t)h * ctx + t] = ss[t - t0];
    }
    l = block_reduce_d(l, sh, 0);
    if (threadIdx.x == 0) {
        stats[((size_t)h * nchunks + b) * 2] = mx;
        stats[((size_t)h * nchunks + b) * 2 + 1] = l;
    }
}

__global__ void __launch_bounds__(128) att_weighted_kernel(const float *vc, int kvstride, const int *state, int hd,
                                                           int group, const double *scores, const double *stats,
                                                           float *partial, int ctx, int nchunks) {
    step_entry_wait();
    __shared__ float ps[kAttChunk];
    const int h = blockIdx.x, b = blockIdx.y, pos = state[1], t0 = b * kAttChunk, kvh = h / group;
    if (t0 > pos) return;
    const int t1 = min(t0 + kAttChunk, pos + 1), nb = pos / kAttChunk + 1;
    const double *st = stats + (size_t)h * nchunks * 2;
    double M = -INFINITY;
    for (int c = 0; c < nb; c++) M = fmax(M, st[2 * c]);
    double L = 0;
    for (int c = 0; c < nb; c++) L = __dadd_rn(L, __dmul_rn(st[2 * c + 1], exp(__dsub_rn(st[2 * c], M))));
    for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x)
        ps[t - t0] = (float)__ddiv_rn(exp(__dsub_rn(scores[(size_t)h * ctx + t], M)), L);
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        const float *v = vc + kvh * hd + i;
        float acc = 0.f;
#pragma unroll 8
        for (int t = t0; t < t1; t++) acc = __fadd_rn(acc, __fmul_rn(ps[t - t0], v[(size_t)t * kvstride]));
        partial[((size_t)h * nchunks + b) * hd + i] = acc;
    }
}

__global__ void att_combine_kernel(const float *partial, const int *state, int hd, float *out, int nchunks) {
    step_entry();
    const int h = blockIdx.x, nb = state[1] / kAttChunk + 1;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.f;
        for (int c = 0; c < nb; c++) acc = __fadd_rn(acc, partial[((size_t)h * nchunks + c) * hd + i]);
        out[h * hd + i] = acc;
    }
}

struct AttScratch {
    double *scores = nullptr, *stats = nullptr;
    float *partial = nullptr;
    int ctx = 0, nchunks = 0;
};

inline size_t att_scratch_bytes(int heads, int ctx, int hd) {
    const int nc = (ctx + kAttChunk - 1) / kAttChunk;
    return sizeof(double) * (size_t)heads * ctx + sizeof(double) * 2 * (size_t)heads * nc +
           sizeof(float) * (size_t)heads * nc * hd;
}

// Carves the scratch out of one device buffer of att_scratch_bytes().
inline AttScratch att_scratch(void *buf, int heads, int ctx, int hd) {
    AttScratch a;
    a.ctx = ctx;
    a.nchunks = (ctx + kAttChunk - 1) / kAttChunk;
    a.scores = static_cast<double *>(buf);
    a.stats = a.scores + (size_t)heads * ctx;
    a.partial = reinterpret_cast<float *>(a.stats + 2 * (size_t)heads * a.nchunks);
    return a;
}

// The decode-step attention of q (heads x hd) over cached positions 0..state[1].
inline cudaError_t decode_attention(const float *q, const float *kc, const float *vc, int kvstride, float *out,
                                    const int *state, int heads, int hd, int group, double scale, const AttScratch &a,
                                    cudaStream_t st) {
    cudaError_t e = step_launch(att_scores_kernel, dim3(heads, a.nchunks), dim3(128), 0, st, q, kc, kvstride, state, hd, group,
                        scale, a.scores, a.stats, a.ctx, a.nchunks);
    if (e == cudaSuccess)
        e = step_launch(att_weighted_kernel, dim3(heads, a.nchunks), dim3(128), 0, st, vc, kvstride, state, hd, group, a.scores,
                a.stats, a.partial, a.ctx, a.nchunks);
    if (e == cudaSuccess) e = step_launch(att_combine_kernel, dim3(heads), dim3(128), 0, st, a.partial, state, hd, out, a.nchunks);
    return e;
}

// ---- greedy pick ------------------------------------------------------------------------
// The first index of the largest of n logits (main.go:69-77: strict >), as
// the candidate (value, offset + index) in cand[0..1] (value bits, index).
// final != 0: also take it as the next token and advance the state
// (position = set_pos if >= 0, else + 1).
__global__ void argmax_kernel(const float *logits, int n, int offset, int *cand, int *state, int *tokens,
                              int set_pos, int final) {
    step_entry();
    __shared__ float bv[32];
    __shared__ int bi[32];
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (v > best) best = v, idx = i; // increasing i per thread: keeps the first maximum
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) bv[w] = best, bi[w] = idx;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); k++)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) best = bv[k], idx = bi[k];
        if (idx == 0x7fffffff) idx = 0;
        idx += offset;
        cand[0] = __float_as_int(best);
        cand[1] = idx;
        if (final) {
            tokens[state[2]] = idx;
            state[0] = idx;
            state[1] = set_pos >= 0 ? set_pos : state[1] + 1;
            state[2] += 1;
        }
    }
}

// Two-stage greedy pick for long logit vectors: block b finds the first
// maximum of its contiguous slice (argmax_part_kernel), then one block takes
// the best of the slices in order (argmax_final_kernel, same outputs as
// argmax_kernel). Ties resolve to the lowest index either way.
constexpr int kArgBlocks = 128;

__global__ void argmax_part_kernel(const float *logits, int n, int *part) {
    step_entry();
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int per = (n + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per, hi = min(n, lo + per);
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = logits[i];
        if (v > best) best = v, idx = i;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) best = ov, idx = oi;
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) bv[w] = best, bi[w] = idx;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); k++)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) best = bv[k], idx = bi[k];
        part[2 * blockIdx.x] = __float_as_int(best);
        part[2 * blockIdx.x + 1] = idx;
    }
}

__global__ void argmax_final_kernel(const int *part, int nparts, int offset, int *cand, int *state, int *tokens,
                                    int set_pos, int final) {
    step_entry();
    if (threadIdx.x != 0) return;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int k = 0; k < nparts; k++) {
        const float v = __int_as_float(part[2 * k]);
        const int i = part[2 * k + 1];
        if (v > best || (v == best && i < idx)) best = v, idx = i;
    }
    if (idx == 0x7fffffff) idx = 0;
    idx += offset;
    cand[0] = __float_as_int(best);
    cand[1] = idx;
    if (final) {
        tokens[state[2]] = idx;
        state[0] = idx;
        state[1] = set_pos >= 0 ? set_pos : state[1] + 1;
        state[2] += 1;
    }
}

// argmax over n logits into cand (and the state when final), part: 2 *
// kArgBlocks ints of scratch.
inline cudaError_t greedy_pick(const float *logits, int n, int offset, int *part, int *cand, int *state, int *tokens,
                               int set_pos, int final, cudaStream_t st) {
    cudaError_t e = step_launch(argmax_part_kernel, dim3(kArgBlocks), dim3(256), 0, st, logits, n, part);
    if (e == cudaSuccess)
        e = step_launch(argmax_final_kernel, dim3(1), dim3(32), 0, st, part, kArgBlocks, offset, cand, state, tokens, set_pos,
                final);
    return e;
}

// The best of w candidates (value, global index) from the shards of a
// column-split head: larger value, ties to the lower index. Advances the
// state like argmax_kernel's final form.
__global__ void pick_kernel(const int *cands, int w, int *state, int *tokens, int set_pos) {
    step_entry();
    if (threadIdx.x != 0) return;
    float best = __int_as_float(cands[0]);
    int idx = cands[1];
    for (int k = 1; k < w; k++) {
        const float v = __int_as_float(cands[2 * k]);
        const int i = cands[2 * k + 1];
        if (v > best || (v == best && i < idx)) best = v, idx = i;
    }
    tokens[state[2]] = idx;
    state[0] = idx;
    state[1] = set_pos >= 0 ? set_pos : state[1] + 1;
    state[2] += 1;
}

} // namespace TQD_NS
