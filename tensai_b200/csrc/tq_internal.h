// tq_internal.h — helpers shared by the library's host-side translation units
// (not part of the public ABI).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>

#include "tq_common.cuh"

struct Handle {
    int device;
    TqMatrixDev m;
};

// Records a formatted message for tq_last_error() and returns code.
int tq_fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
// Records a CUDA failure (TQ_ERR_NOMEM for allocation failures, else TQ_ERR_CUDA).
int tq_cuda_fail(cudaError_t e, const char *what);
// cudaMalloc that honours tq_debug_fail_allocs().
cudaError_t tq_dev_malloc(void **p, size_t bytes);
// Looks a handle up; on failure *rc holds TQ_ERR_HANDLE and the message is set.
std::shared_ptr<Handle> tq_lookup_checked(uint64_t h, int *rc);
// The matvec scratch of (device, stream), created on first use (with the
// M >= 16 matmul partials when m >= TQ_MM_MIN_ROWS). Not inside a capture.
int tq_scratch_for(int device, cudaStream_t st, TqScratch *out, int m);
// Frees and forgets the scratch of (device, stream); before destroying a stream
// whose scratch tq_scratch_for created, after its work has finished.
void tq_scratch_release(int device, cudaStream_t st);
// out[M][cols] = x @ W with the kernel the library would pick for M rows.
// Whether the selected matvec kernel runs int4 rows on the tensor cores (tq_set_matvec_kernel).
bool tq_matvec_uses_tmv();
cudaError_t tq_launch_matmul(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                             cudaStream_t st);
// A zeroed device matrix (shape checked) on the current device / its release.
int tq_alloc_matrix(int bits, int rows, int cols, TqMatrixDev *m, cudaStream_t st);
void tq_release_matrix(TqMatrixDev *m);
// Reads and clears a scratch's status word, ORing it into *out (synchronous on st).
cudaError_t tq_read_status(const TqScratch &scr, cudaStream_t st, unsigned *out);
// Temperature sampling of device logits (tq_sample.cu): the examples' sample
// step (tq_sample in the header). Buffers for up to cap logits.
struct TqSampler {
    int cap = 0;
    double *kin = nullptr, *kout = nullptr, *partial = nullptr;
    int *iin = nullptr, *iout = nullptr;
    float *maxl = nullptr;
    void *tmp = nullptr;
    size_t tmp_bytes = 0;
};
cudaError_t tq_sampler_alloc(TqSampler *s, int n);
void tq_sampler_free(TqSampler *s);
// The token picked from logits[0..n) into *id_out (device), with the draw
// draws[*at] (draws[0] when at is null) for temp > 0; asynchronous on st.
cudaError_t tq_launch_sample(const TqSampler &s, const float *logits, int n, double temp, const double *draws,
                             const int *at, int *id_out, cudaStream_t st);
// Checks sampling settings: a NaN temperature, or temp > 0 without n_draws >= 1
// draws in [0, 1], fail with TQ_ERR_ARG (message set).
int tq_check_draws(double temp, const double *draws, int n_draws);
// Seeded uniform token ids on the host (tq_quantize.cu).
void tq_host_synth_tokens(int *out, int n, int vocab, uint64_t seed);
