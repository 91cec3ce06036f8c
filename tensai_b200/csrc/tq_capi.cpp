// tq_capi.cpp — the C ABI of libtensai_cuda.so (declared in
// include/tensai_cuda.h): handle table, argument checks with the reference's
// error wording, per-thread streams and staging, and dispatch to the kernels.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <map>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/tensai_cuda.h"
#include "tq_common.cuh"
#include "tq_internal.h"

namespace {

thread_local std::string t_err;
thread_local int t_device = 0;
std::atomic<int> g_fail_allocs{0};

std::mutex g_mu;
std::unordered_map<uint64_t, std::shared_ptr<Handle>> g_handles;
uint64_t g_next_handle = 1;

// Matvec chains (tq_chain_create) and the device they live on.
struct ChainEntry {
    TqChain *chain = nullptr;
    int device = 0;
};
std::mutex g_chain_mu;
std::unordered_map<uint64_t, std::shared_ptr<ChainEntry>> g_chains;
uint64_t g_next_chain = 1;

// Per-thread, per-device context for the host-pointer entry points.
// The output block d_blk / h_blk is [status word, 3 pad words | out]: the
// call's kernels report into its first word, which travels back with out.
struct ThreadCtx {
    cudaStream_t stream = nullptr;
    float *d_x = nullptr, *d_blk = nullptr;
    size_t d_x_cap = 0, d_blk_cap = 0;
    float *h_x = nullptr, *h_blk = nullptr; // pinned staging
    size_t h_x_cap = 0, h_blk_cap = 0;
    // Single-row calls replayed as one graph (x in, the matvec, status and
    // out back) per (matrix handle, kernel selection); built on a matrix's
    // second call, dropped when the staging buffers move.
    std::unordered_map<uint64_t, cudaGraphExec_t> graphs;
};
constexpr size_t kBlkHead = 4; // floats before out in the output block
constexpr size_t kMaxGraphs = 64;
thread_local std::unordered_map<int, ThreadCtx> t_ctx;

// Matvec scratch, one per (device, stream): kernels on one stream run in
// order, so they may share it; kernels on different streams never do.
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, TqScratch> g_scratch;

} // namespace

int tq_fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

int tq_cuda_fail(cudaError_t e, const char *what) {
    cudaGetLastError(); // clear a sticky-free error so the next call starts clean
    return tq_fail(e == cudaErrorMemoryAllocation ? TQ_ERR_NOMEM : TQ_ERR_CUDA, "tensai: %s: %s (%s)", what,
                   cudaGetErrorString(e), cudaGetErrorName(e));
}

cudaError_t tq_dev_malloc(void **p, size_t bytes) {
    int f = g_fail_allocs.load();
    while (f > 0) {
        if (g_fail_allocs.compare_exchange_weak(f, f - 1)) {
            *p = nullptr;
            return cudaErrorMemoryAllocation;
        }
    }
    return cudaMalloc(p, bytes ? bytes : 1);
}

static ThreadCtx *ctx_for(int device) { return &t_ctx[device]; }

// The partial-sum buffer of the M >= 16 matmul, added to a stream's scratch
// on the first such call.
static int add_mm_partial(int device, TqScratch *s) {
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = tq_dev_malloc((void **)&s->mm_partial, tq_mm_partial_floats(sms) * sizeof(float));
    if (e != cudaSuccess) {
        s->mm_partial = nullptr;
        return tq_cuda_fail(e, "matmul scratch allocation");
    }
    return TQ_OK;
}

// The scratch of (device, stream), created and cleared on first use (and
// widened on the first call with m >= TQ_MM_MIN_ROWS); those first calls on a
// stream must therefore not be inside a CUDA-graph capture.
static int scratch_for(int device, cudaStream_t st, TqScratch *out, int m = 1) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    auto key = std::make_pair(device, st);
    auto it = g_scratch.find(key);
    if (it != g_scratch.end()) {
        if (m >= TQ_MM_MIN_ROWS && !it->second.mm_partial) {
            int rc = add_mm_partial(device, &it->second);
            if (rc) return rc;
        }
        *out = it->second;
        return TQ_OK;
    }
    TqScratch s{nullptr, nullptr, nullptr, nullptr, nullptr};
    const size_t words = TQ_MAX_TILES + 32; // arrival counters, then the status word
    cudaError_t e = tq_dev_malloc((void **)&s.partial, TQ_SCRATCH_PARTIAL_FLOATS * sizeof(float));
    if (e == cudaSuccess) e = tq_dev_malloc((void **)&s.counters, words * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemsetAsync(s.counters, 0, words * sizeof(unsigned), st);
    if (e == cudaSuccess) e = tq_dev_malloc((void **)&s.planes, TQ_SCRATCH_PLANES_BYTES);
    s.status = s.counters + TQ_MAX_TILES;
    if (e != cudaSuccess) {
        if (s.partial) cudaFree(s.partial);
        if (s.counters) cudaFree(s.counters);
        if (s.planes) cudaFree(s.planes);
        return tq_cuda_fail(e, "matvec scratch allocation");
    }
    if (m >= TQ_MM_MIN_ROWS) {
        int rc = add_mm_partial(device, &s);
        if (rc) {
            cudaFree(s.partial);
            cudaFree(s.counters);
            cudaFree(s.planes);
            return rc;
        }
    }
    g_scratch[key] = s;
    *out = s;
    return TQ_OK;
}

// Reads and clears a scratch's status word (synchronous on st).
cudaError_t tq_read_status(const TqScratch &scr, cudaStream_t st, unsigned *out);
static cudaError_t read_status(const TqScratch &scr, cudaStream_t st, unsigned *out) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, scr.status, sizeof v, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && v) e = cudaMemsetAsync(scr.status, 0, sizeof v, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    *out |= v;
    return e;
}

// Matvec kernel for M <= 15 rows (tq_set_matvec_kernel):
//   0 (default): int4 single rows on the tensor cores by mma.sync (tq_cmv.cu,
//                K-packed copy), otherwise the single-launch CUDA-core matvec
//                (tq_cmv.cu) for M <= 2 and the tcgen05 matvec (tq_igemv.cu)
//                for 3 <= M <= 15;
//   1: CUDA-core matvec with per-warp copies (tq_matvec.cu);
//   2: retired (a single-launch tensor-core variant, never the fastest);
//   3: single-launch CUDA-core matvec (tq_cmv.cu), 2 rows per launch;
//   4: tensor-core matvec with a digit-plane launch (tq_igemv.cu);
//   5: int4 on the tensor cores by mma.sync (tq_cmv.cu), one row per launch;
//      int8 as 3.
std::atomic<int> g_matvec_kernel{0};

// M >= TQ_MM_MIN_ROWS: the tf32 tensor-core matmul; fewer rows: the matvec
// kernel chosen by tq_set_matvec_kernel.
static cudaError_t launch_matvec(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                                 cudaStream_t st) {
    if (M >= TQ_MM_MIN_ROWS) return tq_launch_mm(m, x, out, M, scr, st);
    switch (g_matvec_kernel.load()) {
    case 1: return tq_launch_matvec(m, x, out, M, scr, st);
    case 3: return tq_launch_cmv(m, x, out, M, scr, st);
    case 4: return tq_launch_igemv(m, x, out, M, scr, st);
    case 5: return tq_launch_tmv(m, x, out, M, scr, st);
    default:
        if (M == 1 && m.bits == 4 && m.kpack) return tq_launch_tmv(m, x, out, M, scr, st);
        return M <= 2 ? tq_launch_cmv(m, x, out, M, scr, st) : tq_launch_igemv(m, x, out, M, scr, st);
    }
}

int tq_scratch_for(int device, cudaStream_t st, TqScratch *out, int m) { return scratch_for(device, st, out, m); }

// Frees the scratch of (device, stream) and forgets it; for owners of a
// stream (the decode engines) before they destroy it, with its work finished.
void tq_scratch_release(int device, cudaStream_t st) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    auto it = g_scratch.find(std::make_pair(device, st));
    if (it == g_scratch.end()) return;
    TqScratch &s = it->second;
    for (void *p : {(void *)s.partial, (void *)s.counters, (void *)s.planes, (void *)s.mm_partial})
        if (p) cudaFree(p);
    g_scratch.erase(it);
}

cudaError_t tq_read_status(const TqScratch &scr, cudaStream_t st, unsigned *out) { return read_status(scr, st, out); }

bool tq_matvec_uses_tmv() {
    const int k = g_matvec_kernel.load();
    return k == 0 || k == 5;
}

cudaError_t tq_launch_matmul(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                             cudaStream_t st) {
    return launch_matvec(m, x, out, M, scr, st);
}

static int ensure_stream(ThreadCtx *c) {
    if (!c->stream) {
        cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) return tq_cuda_fail(e, "stream create");
    }
    return TQ_OK;
}

static void drop_graphs(ThreadCtx *c) {
    for (auto &kv : c->graphs)
        if (kv.second) cudaGraphExecDestroy(kv.second);
    c->graphs.clear();
}

static int grow_dev(float **p, size_t *cap, size_t floats) {
    if (*cap >= floats) return TQ_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = tq_dev_malloc((void **)p, floats * sizeof(float));
    if (e != cudaSuccess) return tq_cuda_fail(e, "device staging allocation");
    *cap = floats;
    return TQ_OK;
}

static int grow_host(float **p, size_t *cap, size_t floats) {
    if (*cap >= floats) return TQ_OK;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMallocHost((void **)p, floats * sizeof(float));
    if (e != cudaSuccess) return tq_cuda_fail(e, "pinned staging allocation");
    *cap = floats;
    return TQ_OK;
}

static std::shared_ptr<Handle> lookup(uint64_t h) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_handles.find(h);
    return it == g_handles.end() ? nullptr : it->second;
}

std::shared_ptr<Handle> tq_lookup_checked(uint64_t h, int *rc) {
    auto p = lookup(h);
    *rc = p ? TQ_OK : tq_fail(TQ_ERR_HANDLE, "tensai: invalid or freed matrix handle %llu", (unsigned long long)h);
    return p;
}

static int check_dims(int bits, int rows, int cols) {
    if (rows < 0 || cols < 0) return tq_fail(TQ_ERR_ARG, "tensai: negative matrix shape %dx%d", rows, cols);
    if (bits == 4 && cols % 2 != 0)
        return tq_fail(TQ_ERR_ARG, "tensai: quantize4 needs an even column count, got %d", cols);
    if (tq_tiles(bits, cols) > TQ_MAX_TILES)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: %d columns exceed the supported %d", cols,
                       TQ_MAX_TILES * TQ_TILE_BYTES * (bits == 8 ? 1 : 2));
    if ((long long)rows * tq_row_bytes(bits, cols) > (1ll << 40))
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: matrix %dx%d too large", rows, cols);
    return TQ_OK;
}

static void release_matrix(TqMatrixDev *m) {
    for (void *p : {(void *)m->codes, (void *)m->scale, (void *)m->kpack})
        if (p) cudaFree(p);
    m->codes = m->kpack = nullptr;
    m->scale = nullptr;
}

// Allocates a device matrix on the calling thread's device and clears it on
// stream st (ordered before whatever the caller enqueues next on st).
static int alloc_matrix(int bits, int rows, int cols, TqMatrixDev *m, cudaStream_t st) {
    std::memset(m, 0, sizeof *m);
    m->bits = bits;
    m->rows = rows;
    m->cols = cols;
    m->tiles = tq_tiles(bits, cols);
    m->units = tq_units(rows);
    const size_t cbytes = tq_code_bytes(bits, rows, cols);
    const size_t sfloats = tq_scale_floats(bits, rows, cols);
    // int4 matrices also hold a K-packed copy of codes and scales for the
    // tensor-core matvecs (filled by the quantize / upload launchers)
    cudaError_t e = tq_dev_malloc((void **)&m->codes, cbytes);
    if (e == cudaSuccess) e = tq_dev_malloc((void **)&m->scale, sfloats * sizeof(float));
    if (e == cudaSuccess) e = cudaMemsetAsync(m->codes, 0, cbytes, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->scale, 0, sfloats * sizeof(float), st);
    if (bits == 4) {
        const size_t kbytes = cbytes / TQ_ITEM_BYTES * TQ_KPACK_BYTES;
        if (e == cudaSuccess) e = tq_dev_malloc((void **)&m->kpack, kbytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(m->kpack, 0, kbytes, st);
    }
    if (e != cudaSuccess) {
        release_matrix(m);
        return tq_cuda_fail(e, "matrix allocation");
    }
    return TQ_OK;
}

int tq_alloc_matrix(int bits, int rows, int cols, TqMatrixDev *m, cudaStream_t st) {
    int rc = check_dims(bits, rows, cols);
    return rc ? rc : alloc_matrix(bits, rows, cols, m, st);
}
void tq_release_matrix(TqMatrixDev *m) { release_matrix(m); }

static uint64_t register_handle(int device, const TqMatrixDev &m) {
    auto h = std::make_shared<Handle>();
    h->device = device;
    h->m = m;
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t id = g_next_handle++;
    g_handles[id] = h;
    return id;
}

// Host reference layout <-> tiled device layout: one copy into a temporary
// device buffer in the reference layout, then a re-layout kernel (and the
// reverse for downloads). Synchronous.
static size_t ref_scale_floats(const TqMatrixDev &m) { return m.bits == 8 ? (size_t)m.cols : (size_t)m.units * m.cols; }

static cudaError_t copy_in(const TqMatrixDev &m, const void *q, const float *scale) {
    const size_t qb = (size_t)m.rows * tq_row_bytes(m.bits, m.cols), sf = ref_scale_floats(m);
    if (qb == 0) return cudaSuccess;
    uint8_t *tmp = nullptr;
    cudaError_t e = tq_dev_malloc((void **)&tmp, qb + sf * sizeof(float) + 16);
    if (e != cudaSuccess) return e;
    float *tscale = reinterpret_cast<float *>(tmp + ((qb + 15) & ~(size_t)15));
    e = cudaMemcpy(tmp, q, qb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(tscale, scale, sf * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = tq_launch_to_tiled(m, tmp, tscale, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(tmp);
    return e;
}

static cudaError_t copy_out(const TqMatrixDev &m, void *q, float *scale) {
    const size_t qb = (size_t)m.rows * tq_row_bytes(m.bits, m.cols), sf = ref_scale_floats(m);
    std::memset((uint8_t *)q + qb, 0, 16); // the reference's pad bytes
    if (qb == 0) {
        if (sf) std::memset(scale, 0, sf * sizeof(float));
        return cudaSuccess;
    }
    uint8_t *tmp = nullptr;
    cudaError_t e = tq_dev_malloc((void **)&tmp, qb + sf * sizeof(float) + 16);
    if (e != cudaSuccess) return e;
    float *tscale = reinterpret_cast<float *>(tmp + ((qb + 15) & ~(size_t)15));
    e = tq_launch_from_tiled(m, tmp, tscale, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(q, tmp, qb, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(scale, tscale, sf * sizeof(float), cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    return e;
}

static int set_thread_device() {
    cudaError_t e = cudaSetDevice(t_device);
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "set device");
}

extern "C" {

int tq_version(void) { return TQ_ABI_VERSION; }

const char *tq_last_error(void) { return t_err.c_str(); }

int tq_device_count(int *n) {
    if (!n) return tq_fail(TQ_ERR_ARG, "tensai: null output pointer");
    cudaError_t e = cudaGetDeviceCount(n);
    if (e != cudaSuccess) {
        *n = 0;
        return tq_cuda_fail(e, "device count");
    }
    return TQ_OK;
}

int tq_set_device(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return tq_cuda_fail(e, "device count");
    if (device < 0 || device >= n) return tq_fail(TQ_ERR_ARG, "tensai: device %d out of range (have %d)", device, n);
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return tq_cuda_fail(e, "device properties");
    if (prop.major != 10)
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: device %d is sm_%d%d; this library is built for sm_100a", device,
                       prop.major, prop.minor);
    t_device = device;
    return set_thread_device();
}

static int upload(int bits, const void *q, const float *scale, int rows, int cols, uint64_t *handle) {
    if (!handle || (!q && rows && cols) || (!scale && cols)) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    int rc = check_dims(bits, rows, cols);
    if (rc) return rc;
    if ((rc = set_thread_device())) return rc;
    TqMatrixDev m;
    if ((rc = alloc_matrix(bits, rows, cols, &m, nullptr))) return rc;
    cudaError_t e = copy_in(m, q, scale);
    if (e != cudaSuccess) {
        release_matrix(&m);
        return tq_cuda_fail(e, "upload");
    }
    *handle = register_handle(t_device, m);
    return TQ_OK;
}

int tq_q8_upload(const int8_t *q, const float *scale, int rows, int cols, uint64_t *handle) {
    return upload(8, q, scale, rows, cols, handle);
}

int tq_q4_upload(const uint8_t *q, const float *scale, int rows, int cols, uint64_t *handle) {
    return upload(4, q, scale, rows, cols, handle);
}

static int quantize_dev(int bits, const float *w, int rows, int cols, void *stream, uint64_t *handle) {
    if (!handle || (!w && rows && cols)) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    int rc = check_dims(bits, rows, cols);
    if (rc) return rc;
    if ((rc = set_thread_device())) return rc;
    TqMatrixDev m;
    if ((rc = alloc_matrix(bits, rows, cols, &m, (cudaStream_t)stream))) return rc;
    cudaError_t e = tq_launch_quantize(m, w, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        release_matrix(&m);
        return tq_cuda_fail(e, "quantize launch");
    }
    *handle = register_handle(t_device, m);
    return TQ_OK;
}

int tq_quantize8_dev(const float *w, int rows, int cols, void *stream, uint64_t *handle) {
    return quantize_dev(8, w, rows, cols, stream, handle);
}

int tq_quantize4_dev(const float *w, int rows, int cols, void *stream, uint64_t *handle) {
    return quantize_dev(4, w, rows, cols, stream, handle);
}

static int quantize_linear_dev(int bits, const void *w, int dtype, int out_features, int in_features, void *stream,
                               uint64_t *handle) {
    if (!handle || (!w && out_features && in_features)) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    if (dtype != TQ_LINEAR_F32 && dtype != TQ_LINEAR_F16 && dtype != TQ_LINEAR_BF16)
        return tq_fail(TQ_ERR_ARG, "tensai: unknown Linear weight type %d", dtype);
    const int rows = in_features, cols = out_features; // the transpose the loader quantizes
    int rc = check_dims(bits, rows, cols);
    if (rc) return rc;
    if ((rc = set_thread_device())) return rc;
    TqMatrixDev m;
    if ((rc = alloc_matrix(bits, rows, cols, &m, (cudaStream_t)stream))) return rc;
    cudaError_t e = tq_launch_quantize_linear(m, w, dtype, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        release_matrix(&m);
        return tq_cuda_fail(e, "quantize launch");
    }
    *handle = register_handle(t_device, m);
    return TQ_OK;
}

int tq_quantize8_linear_dev(const void *w, int dtype, int out_features, int in_features, void *stream,
                            uint64_t *handle) {
    return quantize_linear_dev(8, w, dtype, out_features, in_features, stream, handle);
}

int tq_quantize4_linear_dev(const void *w, int dtype, int out_features, int in_features, void *stream,
                            uint64_t *handle) {
    return quantize_linear_dev(4, w, dtype, out_features, in_features, stream, handle);
}

static int quantize_host(int bits, const float *w, int rows, int cols, void *q, float *scale) {
    if (!q || !scale || (!w && rows && cols)) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    int rc = check_dims(bits, rows, cols);
    if (rc) return rc;
    if ((rc = set_thread_device())) return rc;
    float *dw = nullptr;
    cudaError_t e = tq_dev_malloc((void **)&dw, sizeof(float) * (size_t)rows * cols);
    if (e != cudaSuccess) return tq_cuda_fail(e, "weight staging allocation");
    if (rows && cols) e = cudaMemcpy(dw, w, sizeof(float) * (size_t)rows * cols, cudaMemcpyHostToDevice);
    uint64_t h = 0;
    if (e == cudaSuccess) {
        rc = quantize_dev(bits, dw, rows, cols, nullptr, &h);
    } else {
        rc = tq_cuda_fail(e, "weight upload");
    }
    if (rc == TQ_OK) {
        auto p = lookup(h);
        e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = copy_out(p->m, q, scale);
        if (e != cudaSuccess) rc = tq_cuda_fail(e, "quantize");
        tq_free(h);
    }
    cudaFree(dw);
    return rc;
}

int tq_quantize8(const float *w, int rows, int cols, int8_t *q, float *scale) {
    return quantize_host(8, w, rows, cols, q, scale);
}

int tq_quantize4(const float *w, int rows, int cols, uint8_t *q, float *scale) {
    return quantize_host(4, w, rows, cols, q, scale);
}

int tq_matrix_info(uint64_t handle, int *bits, int *rows, int *cols) {
    int rc;
    auto p = tq_lookup_checked(handle, &rc);
    if (!p) return rc;
    if (bits) *bits = p->m.bits;
    if (rows) *rows = p->m.rows;
    if (cols) *cols = p->m.cols;
    return TQ_OK;
}

int tq_download(uint64_t handle, void *q, float *scale) {
    if (!q || !scale) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    int rc;
    auto p = tq_lookup_checked(handle, &rc);
    if (!p) return rc;
    cudaError_t e = cudaSetDevice(p->device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = copy_out(p->m, q, scale);
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "download");
}

int tq_free(uint64_t handle) {
    std::shared_ptr<Handle> p;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_handles.find(handle);
        if (it == g_handles.end()) return TQ_OK;
        p = it->second;
        g_handles.erase(it);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaDeviceSynchronize(); // no kernel of any stream may still read the codes
    release_matrix(&p->m);
    cudaSetDevice(prev);
    return TQ_OK;
}

int tq_matmul_dev(uint64_t handle, const float *x, float *out, int m, void *stream) {
    int rc;
    auto p = tq_lookup_checked(handle, &rc);
    if (!p) return rc;
    if (m < 0) return tq_fail(TQ_ERR_ARG, "tensai: negative row count %d", m);
    if (m && ((!x && p->m.rows) || (!out && p->m.cols))) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    cudaError_t e = cudaSetDevice(p->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "set device");
    TqScratch scr;
    if ((rc = scratch_for(p->device, (cudaStream_t)stream, &scr, m))) return rc;
    e = launch_matvec(p->m, x, out, m, scr, (cudaStream_t)stream);
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "matmul launch");
}

int tq_matmul_dev_fixed(uint64_t handle, const float *x, float *out, int m, void *stream) {
    int rc;
    auto p = tq_lookup_checked(handle, &rc);
    if (!p) return rc;
    if (m < 0) return tq_fail(TQ_ERR_ARG, "tensai: negative row count %d", m);
    if (m && ((!x && p->m.rows) || (!out && p->m.cols))) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    cudaError_t e = cudaSetDevice(p->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "set device");
    switch (tq_launch_matvec_fixed(p->m, x, out, m, (cudaStream_t)stream, &e)) {
    case TQ_FIXED_OK: return TQ_OK;
    case TQ_FIXED_DEVICE: return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: fixed-scratch matvec serves devices 0-63 only");
    case TQ_FIXED_SMS:
        return tq_fail(TQ_ERR_UNSUPPORTED, "tensai: fixed-scratch matvec serves GPUs with at most %d SMs",
                       TQ_FIXED_MAX_SMS);
    case TQ_FIXED_TILES:
        return tq_fail(TQ_ERR_UNSUPPORTED,
                       "tensai: matrix of %d columns exceeds the fixed-scratch limit of %d column tiles "
                       "(%d int8 / %d int4 columns); use tq_matmul_dev",
                       p->m.cols, TQ_FIXED_MAX_TILES, TQ_FIXED_MAX_TILES * TQ_TILE_BYTES,
                       2 * TQ_FIXED_MAX_TILES * TQ_TILE_BYTES);
    default: return tq_cuda_fail(e, "fixed-scratch matmul launch");
    }
}

int tq_matmul(uint64_t handle, const float *x, float *out, int m) {
    int rc;
    auto p = tq_lookup_checked(handle, &rc);
    if (!p) return rc;
    if (m < 0) return tq_fail(TQ_ERR_ARG, "tensai: negative row count %d", m);
    if (m == 0) return TQ_OK;
    if ((!x && p->m.rows) || (!out && p->m.cols)) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    cudaError_t e = cudaSetDevice(p->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "set device");
    ThreadCtx *c = ctx_for(p->device);
    if ((rc = ensure_stream(c))) return rc;
    const size_t nx = (size_t)m * p->m.rows, no = (size_t)m * p->m.cols;
    const float *old_x = c->d_x, *old_blk = c->d_blk, *old_hx = c->h_x, *old_hb = c->h_blk;
    if ((rc = grow_dev(&c->d_x, &c->d_x_cap, nx)) || (rc = grow_dev(&c->d_blk, &c->d_blk_cap, kBlkHead + no)) ||
        (rc = grow_host(&c->h_x, &c->h_x_cap, nx)) || (rc = grow_host(&c->h_blk, &c->h_blk_cap, kBlkHead + no)))
        return rc;
    if (c->d_blk != old_blk && (e = cudaMemsetAsync(c->d_blk, 0, kBlkHead * sizeof(float), c->stream)) != cudaSuccess)
        return tq_cuda_fail(e, "status word reset");
    if (c->d_x != old_x || c->d_blk != old_blk || c->h_x != old_hx || c->h_blk != old_hb) drop_graphs(c);
    TqScratch scr;
    if ((rc = scratch_for(p->device, c->stream, &scr, m))) return rc;
    scr.status = reinterpret_cast<unsigned *>(c->d_blk); // this call's status word travels back with out
    // x in, the launch, then status and out back in one copy; one synchronization.
    auto enqueue = [&]() {
        cudaError_t r = cudaMemcpyAsync(c->d_x, c->h_x, nx * sizeof(float), cudaMemcpyHostToDevice, c->stream);
        if (r == cudaSuccess) r = launch_matvec(p->m, c->d_x, c->d_blk + kBlkHead, m, scr, c->stream);
        if (r == cudaSuccess)
            r = cudaMemcpyAsync(c->h_blk, c->d_blk, (kBlkHead + no) * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
        return r;
    };
    const uint64_t key = handle * 8 + (uint64_t)g_matvec_kernel.load();
    auto it = m == 1 ? c->graphs.find(key) : c->graphs.end();
    const bool known = it != c->graphs.end(), cached = known && it->second; // null: capture failed once
    std::memcpy(c->h_x, x, nx * sizeof(float));
    e = cached ? cudaGraphLaunch(it->second, c->stream) : enqueue();
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return tq_cuda_fail(e, "matmul");
    const unsigned status = *reinterpret_cast<const unsigned *>(c->h_blk);
    if (status) { // rare: re-arm the status word before reporting
        e = cudaMemsetAsync(c->d_blk, 0, sizeof(unsigned), c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) return tq_cuda_fail(e, "status reset");
        if (status & TQ_STATUS_TIMEOUT)
            return tq_fail(TQ_ERR_TIMEOUT, "tensai: a kernel timed out waiting for its weight copies");
    }
    std::memcpy(out, c->h_blk + kBlkHead, no * sizeof(float));
    if (m == 1 && !known) { // the next call on this matrix replays the same work as one graph
        if (c->graphs.size() >= kMaxGraphs) drop_graphs(c);
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ge = nullptr;
        cudaError_t r = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal);
        if (r == cudaSuccess) {
            const cudaError_t q = enqueue();
            r = cudaStreamEndCapture(c->stream, &g);
            if (q != cudaSuccess) r = q;
        }
        if (r == cudaSuccess) r = cudaGraphInstantiate(&ge, g, 0);
        if (g) cudaGraphDestroy(g);
        if (r != cudaSuccess) cudaGetLastError(); // the call itself succeeded: stay on plain launches
        c->graphs[key] = r == cudaSuccess ? ge : nullptr;
    }
    return TQ_OK;
}

int tq_matvec(uint64_t handle, const float *x, size_t x_len, float *out, size_t out_len) {
    int rc;
    auto p = tq_lookup_checked(handle, &rc);
    if (!p) return rc;
    if (x_len != (size_t)p->m.rows || out_len != (size_t)p->m.cols)
        return tq_fail(TQ_ERR_SHAPE, "tensai: %s shape mismatch: x=%zu out=%zu, want %dx%d",
                       p->m.bits == 8 ? "qmatvec" : "q4matvec", x_len, out_len, p->m.rows, p->m.cols);
    return tq_matmul(handle, x, out, 1);
}

int tq_synth_dev(float *out, size_t n, uint64_t seed, uint64_t stream_id, float sigma, void *cuda_stream) {
    if (!out && n) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    cudaError_t e = tq_launch_synth(out, n, seed, stream_id, sigma, (cudaStream_t)cuda_stream);
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "synth launch");
}

int tq_synth_tokens(int *out, int n, int vocab, uint64_t seed) {
    if (n < 0 || vocab < 1 || (n && !out)) return tq_fail(TQ_ERR_ARG, "tensai: bad token synthesis arguments");
    tq_host_synth_tokens(out, n, vocab, seed);
    return TQ_OK;
}

int tq_device_status(unsigned *bits) {
    if (!bits) return tq_fail(TQ_ERR_ARG, "tensai: null output pointer");
    *bits = 0;
    cudaError_t e = cudaSetDevice(t_device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return tq_cuda_fail(e, "device synchronize");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    for (auto &kv : g_scratch) {
        if (kv.first.first != t_device) continue;
        // after the device synchronize: plain synchronous copies, so no
        // registered stream handle is used (a caller's stream may be gone)
        unsigned v = 0;
        e = cudaMemcpy(&v, kv.second.status, sizeof v, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && v) e = cudaMemset(kv.second.status, 0, sizeof v);
        if (e != cudaSuccess) return tq_cuda_fail(e, "status read");
        *bits |= v;
    }
    unsigned fixed = 0; // the allocation-free entry point's own status word
    if ((e = tq_fixed_status(&fixed)) != cudaSuccess) return tq_cuda_fail(e, "fixed status read");
    *bits |= fixed;
    return TQ_OK;
}

int tq_chain_create(const tq_chain_op *ops, int n, uint64_t *chain) {
    if (!chain || (!ops && n > 0)) return tq_fail(TQ_ERR_ARG, "tensai: null pointer argument");
    if (n < 1 || n > TQ_CHAIN_MAX_OPS)
        return tq_fail(TQ_ERR_ARG, "tensai: a chain takes 1 to %d ops, got %d", TQ_CHAIN_MAX_OPS, n);
    std::vector<std::shared_ptr<Handle>> hs(n);
    std::vector<TqChainSpec> spec(n);
    int rc;
    for (int j = 0; j < n; j++) {
        if (!(hs[j] = tq_lookup_checked(ops[j].matrix, &rc))) return rc;
        if (hs[j]->device != hs[0]->device)
            return tq_fail(TQ_ERR_ARG, "tensai: chain op %d is on device %d, op 0 on device %d", j, hs[j]->device,
                           hs[0]->device);
        spec[j].m = &hs[j]->m;
        spec[j].x = ops[j].x;
        spec[j].out = ops[j].out;
        spec[j].epi = ops[j].epilogue;
        spec[j].resid = ops[j].resid;
        spec[j].norm_w = ops[j].norm_w;
        spec[j].norm_from = ops[j].norm_from;
        spec[j].eps = ops[j].eps;
    }
    cudaError_t e = cudaSetDevice(hs[0]->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "set device");
    TqChain *ch = nullptr;
    int why = TQ_CHAIN_OK, bad = 0;
    e = tq_chain_build(spec.data(), n, &ch, &why, &bad);
    if (why != TQ_CHAIN_OK) {
        static const char *what[] = {"",
                                     "op count out of range",
                                     "int8 and int4 matrices in one chain",
                                     "a matrix without rows or columns",
                                     "an int4 matrix without its tensor-core copy",
                                     "a null or not 16-byte aligned input, or a null output",
                                     "an unknown epilogue, or one the matrix cannot take (SwiGLU: int4, even "
                                     "columns; residual: a resid pointer)",
                                     "too many columns (int8: more than 8192 column tiles; int4: more than 256 "
                                     "columns per SM)",
                                     "a normalised input that is not the output of an earlier residual op of "
                                     "matching width",
                                     "too many rows for its column count: a GPU's share of the matrix covers "
                                     "more than 64 groups of 64 rows",
                                     "an input or residual that overlaps an earlier op's output without being "
                                     "exactly that output (or an int4 output overlapping its own external input)"};
        return tq_fail(TQ_ERR_ARG, "tensai: chain op %d: %s", bad, what[why]);
    }
    if (e != cudaSuccess) return tq_cuda_fail(e, "chain build");
    auto ent = std::make_shared<ChainEntry>();
    ent->chain = ch;
    ent->device = hs[0]->device;
    std::lock_guard<std::mutex> lk(g_chain_mu);
    *chain = g_next_chain++;
    g_chains[*chain] = ent;
    return TQ_OK;
}

static std::shared_ptr<ChainEntry> find_chain(uint64_t h, int *rc) {
    std::lock_guard<std::mutex> lk(g_chain_mu);
    auto it = g_chains.find(h);
    if (it == g_chains.end()) {
        *rc = tq_fail(TQ_ERR_HANDLE, "tensai: invalid or freed chain handle %llu", (unsigned long long)h);
        return nullptr;
    }
    *rc = TQ_OK;
    return it->second;
}

int tq_chain_run(uint64_t chain, void *stream) {
    int rc;
    auto c = find_chain(chain, &rc);
    if (!c) return rc;
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return tq_cuda_fail(e, "set device");
    TqScratch scr;
    if ((rc = scratch_for(c->device, (cudaStream_t)stream, &scr, 1))) return rc;
    e = tq_chain_launch(c->chain, scr, (cudaStream_t)stream);
    return e == cudaSuccess ? TQ_OK : tq_cuda_fail(e, "chain launch");
}

int tq_chain_free(uint64_t chain) {
    std::shared_ptr<ChainEntry> c;
    {
        std::lock_guard<std::mutex> lk(g_chain_mu);
        auto it = g_chains.find(chain);
        if (it == g_chains.end()) return TQ_OK;
        c = it->second;
        g_chains.erase(it);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    cudaDeviceSynchronize(); // no launch may still read the descriptors
    tq_chain_destroy(c->chain);
    cudaSetDevice(prev);
    return TQ_OK;
}

int tq_set_matvec_kernel(int which) {
    if (which < 0 || which > 5 || which == 2)
        return tq_fail(TQ_ERR_ARG, "tensai: matvec kernel must be 0, 1, 3, 4 or 5, got %d", which);
    g_matvec_kernel.store(which);
    return TQ_OK;
}

int tq_debug_fail_allocs(int n) {
    g_fail_allocs.store(n < 0 ? 0 : n);
    return TQ_OK;
}

} // extern "C"
