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
