// tq_sample.cu — the examples' sample step (_example/gpt2/main.go:78-105,
// the same function as _example/qwen/main.go:115-150) on the GPU:
//   temp <= 0: the first index of the largest logit (the greedy scan: strict
//              >, a NaN never wins, a NaN at index 0 stays);
//   temp > 0:  p_i = exp(float64(v_i - maxl) / temp) (the difference rounded
//              to float32, as Go evaluates v-maxl), the candidates sorted by p
//              descending, r = u * sum(p) and the first candidate at which
//              r -= p reaches <= 0, else the first candidate.
// Four launches: the max (one block, exact), the weights with fixed-order
// block sums (a fixed grid, so the sum's bits do not depend on timing), a
// stable radix sort by weight (CUB; equal weights keep ascending ids) and one
// warp that walks the sorted weights with the reference's sequential
// subtractions. Differences from the Go code, all in the last bits: the sum
// is added in a fixed tree instead of index order, exp is CUDA's, and Go's
// unstable sort may order equal weights differently.
#include <cub/device/device_radix_sort.cuh>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdint>
#include <mutex>
#include <unordered_map>

#include "../../include/tensai_cuda.h"
#include "tq_internal.h"

namespace {

constexpr int kMaxThreads = 1024; // max pass: one block
constexpr int kPBlocks = 296;     // weight pass: a fixed grid (two blocks per SM)
constexpr int kPThreads = 256;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// *maxl, *arg = the largest logit and the first index holding it; NaNs never
// win, and a NaN at index 0 is kept (value and index), as in the Go scans
// that start from element 0.
__global__ void __launch_bounds__(kMaxThreads) sample_max_kernel(const float *v, int n, float *maxl, int *arg) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = v[i];
        if (better(x, i, bv, bi)) bv = x, bi = i;
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) sv[warp] = bv, si[warp] = bi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 0; w < nw; w++)
            if (better(sv[w], si[w], bv, bi)) bv = sv[w], bi = si[w];
        const float v0 = v[0];
        if (v0 != v0) bv = v0, bi = 0;
        *maxl = bv;
        *arg = bi;
    }
}

// keys[i] = p_i, ids[i] = i; partial[b] = block b's sum of its threads' p
// (each thread in index order, then a fixed tree).
__global__ void __launch_bounds__(kPThreads) sample_weights_kernel(const float *v, int n, const float *maxl,
                                                                   double temp, double *keys, int *ids,
                                                                   double *partial) {
    __shared__ double sh[kPThreads / 32];
    const float m = *maxl;
    double s = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const double p = exp(__ddiv_rn((double)__fsub_rn(v[i], m), temp));
        keys[i] = p;
        ids[i] = i;
        s = __dadd_rn(s, p);
    }
    for (int o = 16; o; o >>= 1) s = __dadd_rn(s, __shfl_down_sync(0xffffffffu, s, o));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0;
        for (int w = 0; w < kPThreads / 32; w++) t = __dadd_rn(t, sh[w]);
        partial[blockIdx.x] = t;
    }
}

// One warp: the total of the block sums, r = u * total with u = draws[*at]
// (draws[0] without at), then r -= p over the sorted weights until r <= 0
// (every lane holds the same r: the weights are broadcast one at a time, the
// next 32 loaded while the current are walked).
__global__ void sample_pick_kernel(const double *keys, const int *ids, int n, const double *partial, int np,
                                   const double *draws, const int *at, int *token) {
    const int lane = threadIdx.x;
    const double u = draws[at ? *at : 0];
    double s = 0;
    for (int b = lane; b < np; b += 32) s = __dadd_rn(s, partial[b]);
    for (int o = 16; o; o >>= 1) s = __dadd_rn(s, __shfl_down_sync(0xffffffffu, s, o));
    s = __shfl_sync(0xffffffffu, s, 0);
    double r = __dmul_rn(u, s);
    int found = -1;
    double cur = lane < n ? keys[lane] : 0.0;
    for (int j0 = 0; j0 < n && found < 0; j0 += 32) {
        const double next = j0 + 32 + lane < n ? keys[j0 + 32 + lane] : 0.0;
        const int kn = n - j0 < 32 ? n - j0 : 32;
        for (int k = 0; k < kn; k++) {
            r = __dsub_rn(r, __shfl_sync(0xffffffffu, cur, k));
            if (r <= 0) {
                found = j0 + k;
                break;
            }
        }
        cur = next;
    }
    if (lane == 0) *token = ids[found >= 0 ? found : 0];
}

} // namespace

cudaError_t tq_sampler_alloc(TqSampler *s, int n) {
    if (n <= s->cap) return cudaSuccess;
    tq_sampler_free(s);
    cudaError_t e = cudaSuccess;
    auto get = [&](void **p, size_t bytes) {
        if (e == cudaSuccess) e = tq_dev_malloc(p, bytes);
    };
    get((void **)&s->kin, sizeof(double) * n);
    get((void **)&s->kout, sizeof(double) * n);
    get((void **)&s->iin, sizeof(int) * n);
    get((void **)&s->iout, sizeof(int) * n);
    get((void **)&s->partial, sizeof(double) * kPBlocks);
    get((void **)&s->maxl, sizeof(float));
    if (e == cudaSuccess)
        e = cub::DeviceRadixSort::SortPairsDescending(nullptr, s->tmp_bytes, s->kin, s->kout, s->iin, s->iout, n);
    get(&s->tmp, s->tmp_bytes);
    if (e != cudaSuccess) {
        tq_sampler_free(s);
        return e;
    }
    s->cap = n;
    return cudaSuccess;
}

void tq_sampler_free(TqSampler *s) {
    for (void *p : {(void *)s->kin, (void *)s->kout, (void *)s->iin, (void *)s->iout, (void *)s->partial,
                    (void *)s->maxl, s->tmp})
        if (p) cudaFree(p);
    *s = TqSampler{};
}

cudaError_t tq_launch_sample(const TqSampler &s, const float *logits, int n, double temp, const double *draws,
                             const int *at, int *id_out, cudaStream_t st) {
    if (n < 1 || n > s.cap) return cudaErrorInvalidValue;
    if (temp <= 0) { // the greedy scan
        sample_max_kernel<<<1, kMaxThreads, 0, st>>>(logits, n, s.maxl, id_out);
        return cudaGetLastError();
    }
    sample_max_kernel<<<1, kMaxThreads, 0, st>>>(logits, n, s.maxl, s.iout);
    sample_weights_kernel<<<kPBlocks, kPThreads, 0, st>>>(logits, n, s.maxl, temp, s.kin, s.iin, s.partial);
    cudaError_t e = cudaGetLastError();
    size_t bytes = s.tmp_bytes;
    if (e == cudaSuccess)
        e = cub::DeviceRadixSort::SortPairsDescending(s.tmp, bytes, s.kin, s.kout, s.iin, s.iout, n, 0,
                                                      (int)sizeof(double) * 8, st);
    if (e == cudaSuccess) {
        sample_pick_kernel<<<1, 32, 0, st>>>(s.kout, s.iout, n, s.partial, kPBlocks, draws, at, id_out);
        e = cudaGetLastError();
    }
    return e;
}

namespace {
// Per-device state of the host-pointer call.
struct SampleDev {
    TqSampler smp;
    float *v = nullptr;
    int vcap = 0;
    double *u = nullptr;
    int *tok = nullptr;
    cudaStream_t st = nullptr;
};
std::mutex g_sample_mu;
std::unordered_map<int, SampleDev> g_sample;
} // namespace

int tq_check_draws(double temp, const double *draws, int n_draws) {
    if (temp != temp) return tq_fail(TQ_ERR_ARG, "tensai: sampling temperature is NaN");
    if (temp <= 0) return TQ_OK;
    if (!draws || n_draws < 1) return tq_fail(TQ_ERR_ARG, "tensai: temperature %g needs at least one draw", temp);
    for (int i = 0; i < n_draws; i++)
        if (!(draws[i] >= 0 && draws[i] <= 1))
            return tq_fail(TQ_ERR_ARG, "tensai: draw %d (%g) outside [0, 1]", i, draws[i]);
    return TQ_OK;
}

extern "C" int tq_sample(const float *logits, int n, double temp, double u, int *token) {
    if (!logits || !token) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    if (n < 1) return tq_fail(TQ_ERR_ARG, "tensai: sample needs at least one logit, got %d", n);
    if (temp != temp) return tq_fail(TQ_ERR_ARG, "tensai: sample temperature is NaN");
    if (temp > 0 && !(u >= 0 && u <= 1)) return tq_fail(TQ_ERR_ARG, "tensai: sample draw %g outside [0, 1]", u);
    std::lock_guard<std::mutex> lk(g_sample_mu);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return tq_cuda_fail(e, "sample");
    SampleDev &b = g_sample[dev];
    if (!b.st && (e = cudaStreamCreateWithFlags(&b.st, cudaStreamNonBlocking)) != cudaSuccess)
        return tq_cuda_fail(e, "sample stream");
    if (!b.u && (e = tq_dev_malloc((void **)&b.u, sizeof(double))) != cudaSuccess) return tq_cuda_fail(e, "sample");
    if (!b.tok && (e = tq_dev_malloc((void **)&b.tok, sizeof(int))) != cudaSuccess) return tq_cuda_fail(e, "sample");
    if (n > b.vcap) {
        if (b.v) cudaFree(b.v);
        b.v = nullptr;
        b.vcap = 0;
        if ((e = tq_dev_malloc((void **)&b.v, sizeof(float) * n)) != cudaSuccess) return tq_cuda_fail(e, "sample");
        b.vcap = n;
    }
    if ((e = tq_sampler_alloc(&b.smp, n)) != cudaSuccess) return tq_cuda_fail(e, "sample buffers");
    e = cudaMemcpyAsync(b.v, logits, sizeof(float) * n, cudaMemcpyHostToDevice, b.st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b.u, &u, sizeof(double), cudaMemcpyHostToDevice, b.st);
    if (e == cudaSuccess) e = tq_launch_sample(b.smp, b.v, n, temp, b.u, nullptr, b.tok, b.st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(token, b.tok, sizeof(int), cudaMemcpyDeviceToHost, b.st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.st);
    if (e != cudaSuccess) return tq_cuda_fail(e, "sample");
    return TQ_OK;
}
