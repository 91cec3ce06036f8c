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
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fadd_rn(x[i], b ? __fadd_rn(y[i], b[i % n]) : y[i]);
}

__global__ void fill_kernel(float *p, float v, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}

// state = {token to feed, its position, tokens generated}
__global__ void set_state_kernel(int *state, int token, int pos, int generated) {
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

// ---- greedy pick ------------------------------------------------------------------------
// The first index of the largest of n logits (main.go:69-77: strict >), as
// the candidate (value, offset + index) in cand[0..1] (value bits, index).
// final != 0: also take it as the next token and advance the state
// (position = set_pos if >= 0, else + 1).
__global__ void argmax_kernel(const float *logits, int n, int offset, int *cand, int *state, int *tokens,
                              int set_pos, int final) {
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

// The best of w candidates (value, global index) from the shards of a
// column-split head: larger value, ties to the lower index. Advances the
// state like argmax_kernel's final form.
__global__ void pick_kernel(const int *cands, int w, int *state, int *tokens, int set_pos) {
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
