// tq_decode.cuh — kernels shared by the greedy decode engines (tq_model.cu:
// GPT-2; tq_qwen.cu: Qwen2). Each restates one operation of tensai's example
// decode loops in the same float64 / float32 arithmetic as the Go code, with
// explicitly rounded intrinsics so that nvcc contracts nothing into an FMA
// that the Go code (gc at GOAMD64=v1) does not fuse.
#pragma once

#include <cuda_fp16.h>
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
// Lets the next kernel on the stream be scheduled now when it is launched
// with programmatic stream serialization (the matvecs are): its CTAs stream
// their weights while this kernel runs and wait on griddepcontrol.wait before
// reading anything this kernel writes. For the small kernels right before a
// matvec (norms, the attention's value pass).
__device__ __forceinline__ void step_release_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the previous kernel on the stream has completed and its writes
// are visible; returns at once for a kernel launched without programmatic
// stream serialization.
__device__ __forceinline__ void step_wait_prev() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// A launch with programmatic stream serialization whatever TQ_DECODE_PDL is:
// for a small kernel that starts with step_wait_prev, so that it is resident
// (and its launch latency spent) when its predecessor completes.
template <typename... KArgs, typename... Args>
inline cudaError_t step_launch_early(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                     Args... args) {
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
// row index plus pos0 (the chunk's first position). Shared memory: ctx
// doubles + ctx floats.
__global__ void attention_kernel(const float *q, int qstride, const float *kc, const float *vc, int kvstride,
                                 float *out, int outstride, const int *state, int hd, int group, double scale,
                                 int prefill, int ctx, int pos0 = 0) {
    step_entry();
    extern __shared__ double sc[];
    __shared__ double sh[32];
    const int h = blockIdx.x, r = blockIdx.y, kvh = h / group;
    const int pos = prefill ? pos0 + r : state[1];
    const float *qr = q + (size_t)r * qstride + h * hd;
    double mx = -INFINITY;
    const bool vec = (hd & 31) == 0 && ((uintptr_t)qr & 15) == 0 && ((uintptr_t)(kc + kvh * hd) & 15) == 0 &&
                     (kvstride & 3) == 0;
    for (int t = threadIdx.x; t <= pos; t += blockDim.x) {
        const float *kt = kc + (size_t)t * kvstride + kvh * hd;
        double s = 0;
        if (vec) { // 8 float4 loads in flight, then the products in dimension order
            for (int i0 = 0; i0 < hd; i0 += 32) {
                float4 kv[8], qv[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    kv[u] = *reinterpret_cast<const float4 *>(kt + i0 + 4 * u);
                    qv[u] = *reinterpret_cast<const float4 *>(qr + i0 + 4 * u);
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    s = __dadd_rn(s, __dmul_rn((double)qv[u].x, (double)kv[u].x));
                    s = __dadd_rn(s, __dmul_rn((double)qv[u].y, (double)kv[u].y));
                    s = __dadd_rn(s, __dmul_rn((double)qv[u].z, (double)kv[u].z));
                    s = __dadd_rn(s, __dmul_rn((double)qv[u].w, (double)kv[u].w));
                }
            }
        } else {
            for (int i = 0; i < hd; i++) s = __dadd_rn(s, __dmul_rn((double)qr[i], (double)kt[i]));
        }
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
        const float *v = vc + kvh * hd + i;
        for (int t0 = 0; t0 <= pos; t0 += 8) { // 8 loads in flight, then the sum over positions in order
            float vv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) vv[u] = t0 + u <= pos ? v[(size_t)(t0 + u) * kvstride] : 0.f;
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (t0 + u <= pos) acc = __fadd_rn(acc, __fmul_rn(p[t0 + u], vv[u]));
        }
        out[(size_t)r * outstride + h * hd + i] = acc;
    }
}

inline size_t attention_smem(int ctx) { return (sizeof(double) + sizeof(float)) * (size_t)ctx; }

// dst[i] = float32 of src[i], a checkpoint tensor of type dtype (0 float32,
// 1 float16, 2 bfloat16: TQ_LINEAR_*); both widenings are exact.
__global__ void widen_kernel(const void *src, int dtype, float *dst, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v;
        if (dtype == 0)
            v = static_cast<const float *>(src)[i];
        else if (dtype == 1)
            v = __half2float(static_cast<const __half *>(src)[i]);
        else
            v = __uint_as_float((unsigned)static_cast<const unsigned short *>(src)[i] << 16);
        dst[i] = v;
    }
}

// ---- split-K decode attention -------------------------------------------------------
// The attention of the decode step's single query row, spread over chunks of
// cached positions so that long contexts use every SM. A block serves one KV
// head and all `group` query heads that share it (grouped-query attention),
// so each cached k and v row is read once per step, not once per query head.
// Two passes:
//   scores:   per KV head and chunk of kAttSChunk positions, one warp per
//             query head and one lane per position: s_t = (q . k_t, the
//             float64 products added in dimension order) * scale, then the
//             head's chunk max m_b and sum l_b = sum exp(s_t - m_b). The
//             chunk's k rows are staged in shared memory by coalesced 16-byte
//             copies. A float32 x float32 product is exact in float64, so
//             fma(q, k, acc) rounds once exactly as acc + q*k does. With RoPE
//             (Qwen2) the pass first rotates the group's q heads (and, in the
//             chunk holding the position, the KV head's k) from the fused row
//             with the step's cos/sin table, and stores the rotated k and the
//             biased v in the caches;
//   weights:  per KV head and chunk of kAttChunk positions: each head's
//             softmax max M and sum L = sum_b l_b exp(m_b - M) over the score
//             chunks, p_t = float32(exp(s_t - M) / L) as the Go code forms
//             it, and for every head the float32 sums p_t * v_t over the
//             chunk's positions in order (in sub-chunks added in order), each
//             v row read once for all heads; the last chunk of a KV head to
//             finish adds the chunk sums in chunk order.
// Scratch (per engine): scores [heads][ctx] doubles, stats [heads][score
// chunks][2] doubles, partials [heads][chunks][hd] floats, arrival counters
// [heads].
constexpr int kAttChunk = 128;    // positions per value-pass block
constexpr int kAttSChunk = 32;    // positions per scores block (a lane each)
constexpr int kAttMaxHd = 256;
constexpr int kAttMaxGroup = 16;  // query heads per KV head (a warp each in the scores pass)
constexpr int kAttWThreads = 512; // value pass

// RoPE of the scores pass (Qwen2, model.go:219-229: half-split pairs (i, i +
// hd/2)); cs == nullptr for none (GPT-2, whose q, k and v are stored already).
struct AttRope {
    const double *cs = nullptr; // [hd/2][2]: cos, sin of pos * theta^(-2i/hd)
    const float *k = nullptr;   // this position's raw k heads [n_kv][hd] and v heads
    const float *v = nullptr;
    const float *qbias = nullptr, *kbias = nullptr, *vbias = nullptr;
    float *kc = nullptr, *vc = nullptr; // caches [ctx][kvstride]
};

// cs[2i], cs[2i + 1] = cos, sin of pos * theta^(-2i/hd), i < hd/2 (model.go:221-224).
__device__ __forceinline__ void rope_table(double *cs, int pos, int hd, double theta) {
    for (int i = threadIdx.x; i < hd / 2; i += blockDim.x) {
        const double freq = pow(theta, __ddiv_rn(-2.0 * (double)i, (double)hd));
        double s, c;
        sincos(__dmul_rn((double)pos, freq), &s, &c);
        cs[2 * i] = c;
        cs[2 * i + 1] = s;
    }
}

// Rotated pair (a, b) of dimension i with the table: (a c - b s, b c + a s).
__device__ __forceinline__ void rope_pair(const double *cs, int i, float a, float b, float &r0, float &r1) {
    const double c = cs[2 * i], s = cs[2 * i + 1], ad = (double)a, bd = (double)b;
    r0 = (float)__dsub_rn(__dmul_rn(ad, c), __dmul_rn(bd, s));
    r1 = (float)__dadd_rn(__dmul_rn(bd, c), __dmul_rn(ad, s));
}

// Shared memory of the scores pass: the chunk's k rows (stride hd + 4 floats:
// 16-byte rows whose float4 reads by 8 lanes fall in distinct banks) and the
// group's q heads.
inline size_t att_scores_smem(int hd, int group) {
    return sizeof(float) * ((size_t)kAttSChunk * (hd + 4) + (size_t)group * hd);
}
// Shared memory of the value pass: p [group][chunk] and the sub-chunk sums
// [sub-chunks][group][hd].
inline size_t att_weighted_smem(int hd, int group) {
    return sizeof(float) * ((size_t)group * kAttChunk + (size_t)(kAttWThreads / hd) * group * hd);
}

__device__ __forceinline__ void att_cp16(float *dst, const float *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

// Block (KV head, score chunk) of 32 x group threads.
__global__ void __launch_bounds__(32 * kAttMaxGroup) att_scores_kernel(const float *q, const float *kc, int kvstride,
                                                                       const int *state, int hd, int group,
                                                                       double scale, double *scores, double *stats,
                                                                       int ctx, int nschunks, AttRope rope) {
    step_entry_wait();
    extern __shared__ __align__(16) float att_sm[];
    __shared__ __align__(16) float kp[kAttMaxHd];
    const int kvh = blockIdx.x, b = blockIdx.y, pos = state[1], t0 = b * kAttSChunk;
    if (t0 > pos) return;
    const int tid = threadIdx.x, bd = blockDim.x, ld = hd + 4, f4 = hd / 4, half = hd / 2;
    float *ks = att_sm;                       // [kAttSChunk][ld]
    float *qs = ks + (size_t)kAttSChunk * ld; // [group][hd]
    const int nrows = min(kAttSChunk, pos + 1 - t0);
    const bool own = rope.cs && pos < t0 + kAttSChunk; // this chunk holds the step's own (new) k row
    {   // the chunk's cached k rows, in flight while q is prepared (the new
        // row comes from kp instead)
        const float *src = kc + (size_t)kvh * hd;
        for (int f = tid; f < nrows * f4; f += bd) {
            const int r = f / f4, c4 = f - r * f4;
            if (!(own && t0 + r == pos))
                att_cp16(ks + (size_t)r * ld + 4 * c4, src + (size_t)(t0 + r) * kvstride + 4 * c4);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (rope.cs) {
        for (int e = tid; e < group * half; e += bd) {
            const int j = e / half, i = e - j * half, hq = (kvh * group + j) * hd;
            rope_pair(rope.cs, i, __fadd_rn(q[hq + i], rope.qbias[hq + i]),
                      __fadd_rn(q[hq + i + half], rope.qbias[hq + i + half]), qs[j * hd + i], qs[j * hd + i + half]);
        }
        if (own) { // this position's k and v: into the caches and the staged rows (this block alone reads them)
            for (int i = tid; i < half; i += bd) {
                const int kj = kvh * hd + i;
                rope_pair(rope.cs, i, __fadd_rn(rope.k[kj], rope.kbias[kj]),
                          __fadd_rn(rope.k[kj + half], rope.kbias[kj + half]), kp[i], kp[i + half]);
            }
            __syncthreads();
            float *kd = rope.kc + (size_t)pos * kvstride + kvh * hd;
            float *vd = rope.vc + (size_t)pos * kvstride + kvh * hd;
            float *kr = ks + (size_t)(pos - t0) * ld;
            for (int i = tid; i < hd; i += bd) {
                kd[i] = kp[i];
                kr[i] = kp[i];
                vd[i] = __fadd_rn(rope.v[kvh * hd + i], rope.vbias[kvh * hd + i]);
            }
        }
    } else {
        for (int e = tid; e < group * hd; e += bd) qs[e] = q[(size_t)kvh * group * hd + e];
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads(); // q and the k rows
    const int j = tid >> 5, r = tid & 31, h = kvh * group + j;
    double sv = -INFINITY;
    if (r < nrows) {
        const float *kt = ks + (size_t)r * ld, *qr = qs + (size_t)j * hd;
        double acc = 0;
        for (int i0 = 0; i0 < hd; i0 += 32) { // products added in dimension order
            float4 kv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) kv[u] = *reinterpret_cast<const float4 *>(kt + i0 + 4 * u);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float4 qv = *reinterpret_cast<const float4 *>(qr + i0 + 4 * u);
                acc = __fma_rn((double)qv.x, (double)kv[u].x, acc);
                acc = __fma_rn((double)qv.y, (double)kv[u].y, acc);
                acc = __fma_rn((double)qv.z, (double)kv[u].z, acc);
                acc = __fma_rn((double)qv.w, (double)kv[u].w, acc);
            }
        }
        sv = __dmul_rn(acc, scale);
        scores[(size_t)h * ctx + t0 + r] = sv;
    }
    const double mx = warp_max_d(sv);
    const double l = warp_sum_d(r < nrows ? exp(__dsub_rn(sv, mx)) : 0.0);
    if (r == 0) {
        const size_t o = ((size_t)h * nschunks + b) * 2;
        stats[o] = mx;
        stats[o + 1] = l;
    }
}

// One CTA's arrival at a counter after a barrier that ordered the CTA's
// stores; acq_rel at gpu scope, the last of n arrivals re-arms the counter.
__device__ __forceinline__ bool att_arrive_last(unsigned *counter, unsigned n) {
    unsigned prev;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
    const bool last = prev == n - 1;
    if (last) asm volatile("st.relaxed.gpu.u32 [%0], %1;" ::"l"(counter), "r"(0u) : "memory");
    return last;
}

__global__ void __launch_bounds__(kAttWThreads) att_weighted_kernel(const float *vc, int kvstride, const int *state,
                                                                    int hd, int group, const double *scores,
                                                                    const double *stats, float *partial,
                                                                    unsigned *count, float *out, int ctx,
                                                                    int nchunks, int nschunks, int release) {
    step_entry_wait();
    if (release) step_release_next(); // the o_proj matvec streams its weights meanwhile
    extern __shared__ __align__(16) float att_sm[];
    __shared__ double ml[kAttMaxGroup][2];
    __shared__ int last;
    const int kvh = blockIdx.x, b = blockIdx.y, pos = state[1], t0 = b * kAttChunk;
    if (t0 > pos) return;
    const int tid = threadIdx.x, bd = blockDim.x;
    const int t1 = min(t0 + kAttChunk, pos + 1), nb = pos / kAttChunk + 1, nbs = pos / kAttSChunk + 1;
    float *ps = att_sm;                              // [group][kAttChunk]
    float *sub = att_sm + (size_t)group * kAttChunk; // [nsub][group][hd]
    // sub-chunk sq of sz positions, dimension i: the first 32 values and the
    // thread's scores are loaded before the softmax statistics
    const int nsub = bd / hd, sz = kAttChunk / nsub, sq = tid / hd, i = tid - sq * hd;
    const int ta = t0 + sq * sz, tb = min(ta + sz, t1);
    const float *v = vc + (size_t)kvh * hd + i;
    float vv[32];
    auto load_v = [&](int tt) {
#pragma unroll
        for (int u = 0; u < 32; u++) vv[u] = tt + u < tb ? v[(size_t)(tt + u) * kvstride] : 0.f;
    };
    load_v(ta);
    constexpr int kPs = kAttMaxGroup * kAttChunk / kAttWThreads; // p entries per thread
    const int nit = group * kAttChunk;
    double my_s[kPs];
#pragma unroll
    for (int k = 0; k < kPs; k++) {
        const int it = tid + k * bd, j = it / kAttChunk, r = it - j * kAttChunk;
        my_s[k] = it < nit && t0 + r < t1 ? scores[(size_t)(kvh * group + j) * ctx + t0 + r] : 0.0;
    }
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < group) { // head `warp`: the softmax's max and sum over the score chunks' stats
        const double *st = stats + (size_t)(kvh * group + warp) * nschunks * 2;
        double M = -INFINITY;
        for (int c = lane; c < nbs; c += 32) M = fmax(M, st[2 * c]);
        M = warp_max_d(M);
        double L = 0;
        for (int c = lane; c < nbs; c += 32) L = __dadd_rn(L, __dmul_rn(st[2 * c + 1], exp(__dsub_rn(st[2 * c], M))));
        L = warp_sum_d(L);
        if (lane == 0) ml[warp][0] = M, ml[warp][1] = L;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kPs; k++) {
        const int it = tid + k * bd, j = it / kAttChunk, r = it - j * kAttChunk;
        if (it < nit && t0 + r < t1) ps[it] = (float)__ddiv_rn(exp(__dsub_rn(my_s[k], ml[j][0])), ml[j][1]);
    }
    __syncthreads();
    // per head, the sub-chunk's positions in order; the running sums live in sub
    for (int tt = ta; tt < tb; tt += 32) {
        if (tt != ta) load_v(tt);
        for (int j = 0; j < group; j++) {
            float *sj = sub + ((size_t)sq * group + j) * hd + i;
            float a = tt == ta ? 0.f : *sj;
            const float *pj = ps + (size_t)j * kAttChunk + (tt - t0);
            if (tb - tt >= 32) { // a whole batch: p by float4 (16-byte aligned: tt - t0 is a multiple of 32)
#pragma unroll
                for (int u0 = 0; u0 < 32; u0 += 4) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(pj + u0);
                    a = __fadd_rn(a, __fmul_rn(p4.x, vv[u0]));
                    a = __fadd_rn(a, __fmul_rn(p4.y, vv[u0 + 1]));
                    a = __fadd_rn(a, __fmul_rn(p4.z, vv[u0 + 2]));
                    a = __fadd_rn(a, __fmul_rn(p4.w, vv[u0 + 3]));
                }
            } else {
#pragma unroll
                for (int u = 0; u < 32; u++)
                    if (tt + u < tb) a = __fadd_rn(a, __fmul_rn(pj[u], vv[u]));
            }
            *sj = a;
        }
    }
    if (ta >= tb) // an empty sub-chunk adds zeros
        for (int j = 0; j < group; j++) sub[((size_t)sq * group + j) * hd + i] = 0.f;
    __syncthreads();
    const int ne = group * hd;
    for (int e = tid; e < ne; e += bd) { // the chunk's sums: sub-chunks in order
        const int j = e / hd, ii = e - j * hd;
        float a = 0.f;
        for (int c = 0; c < nsub; c++) a = __fadd_rn(a, sub[((size_t)c * group + j) * hd + ii]);
        partial[((size_t)(kvh * group + j) * nchunks + b) * hd + ii] = a;
    }
    __syncthreads(); // every thread's partial store before the arrival
    if (tid == 0) last = att_arrive_last(count + kvh, (unsigned)nb) ? 1 : 0;
    __syncthreads();
    if (!last) return;
    for (int e = tid; e < ne; e += bd) { // chunk sums in chunk order, 16 loads in flight
        const int j = e / hd, ii = e - j * hd;
        const float *pp = partial + (size_t)(kvh * group + j) * nchunks * hd + ii;
        float a = 0.f;
        for (int c0 = 0; c0 < nb; c0 += 16) {
            float pv[16];
#pragma unroll
            for (int u = 0; u < 16; u++) pv[u] = c0 + u < nb ? __ldcg(pp + (size_t)(c0 + u) * hd) : 0.f;
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (c0 + u < nb) a = __fadd_rn(a, pv[u]);
        }
        out[(size_t)(kvh * group + j) * hd + ii] = a;
    }
}

struct AttScratch {
    double *scores = nullptr, *stats = nullptr;
    float *partial = nullptr;
    unsigned *count = nullptr;
    int ctx = 0, nchunks = 0, nschunks = 0;
};

inline size_t att_scratch_bytes(int heads, int ctx, int hd) {
    const int nc = (ctx + kAttChunk - 1) / kAttChunk, ns = (ctx + kAttSChunk - 1) / kAttSChunk;
    return sizeof(double) * (size_t)heads * ctx + sizeof(double) * 2 * (size_t)heads * ns +
           sizeof(float) * (size_t)heads * nc * hd + sizeof(unsigned) * (size_t)heads;
}

// Carves the scratch out of one device buffer of att_scratch_bytes() and
// zeroes the arrival counters on stream st.
inline cudaError_t att_scratch(void *buf, int heads, int ctx, int hd, cudaStream_t st, AttScratch *a) {
    a->ctx = ctx;
    a->nchunks = (ctx + kAttChunk - 1) / kAttChunk;
    a->nschunks = (ctx + kAttSChunk - 1) / kAttSChunk;
    a->scores = static_cast<double *>(buf);
    a->stats = a->scores + (size_t)heads * ctx;
    a->partial = reinterpret_cast<float *>(a->stats + 2 * (size_t)heads * a->nschunks);
    a->count = reinterpret_cast<unsigned *>(a->partial + (size_t)heads * a->nchunks * hd);
    return cudaMemsetAsync(a->count, 0, sizeof(unsigned) * heads, st);
}

// Lets both passes take their shared memory on the current device (once per
// engine build); fails for shapes the kernels do not take.
inline cudaError_t att_setup(int hd, int group) {
    if (hd % 32 || hd > kAttMaxHd || kAttWThreads % hd || group < 1 || group > kAttMaxGroup)
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(att_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)att_scores_smem(hd, group));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(att_weighted_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)att_weighted_smem(hd, group));
    return e;
}

// The decode-step attention of q (heads x hd) over cached positions 0..state[1].
// release: let the next kernel (the o_proj matvec) be scheduled as the value
// pass starts (measured faster on one GPU; the tensor-parallel step keeps it off).
inline cudaError_t decode_attention(const float *q, const float *kc, const float *vc, int kvstride, float *out,
                                    const int *state, int heads, int hd, int group, double scale, const AttScratch &a,
                                    cudaStream_t st, const AttRope &rope = AttRope(), bool release = true) {
    if (hd % 32 || hd > kAttMaxHd || kAttWThreads % hd || group < 1 || group > kAttMaxGroup || heads % group)
        return cudaErrorInvalidValue;
    cudaError_t e = step_launch(att_scores_kernel, dim3(heads / group, a.nschunks), dim3(32 * group),
                                att_scores_smem(hd, group), st, q, kc, kvstride, state, hd, group, scale, a.scores,
                                a.stats, a.ctx, a.nschunks, rope);
    if (e == cudaSuccess)
        e = step_launch(att_weighted_kernel, dim3(heads / group, a.nchunks), dim3(kAttWThreads),
                        att_weighted_smem(hd, group), st, vc, kvstride, state, hd, group, a.scores, a.stats,
                        a.partial, a.count, out, a.ctx, a.nchunks, a.nschunks, release ? 1 : 0);
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
