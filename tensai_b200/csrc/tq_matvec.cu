// tq_matvec.cu — weight-only int8 / int4 dequantize-fused matvec for M <= 8
// activation rows on the CUDA cores (HBM-bound).
//
// Computes out[m][j] = sum_i x[m][i] * W[i][j], the product the reference
// computes one activation row at a time in qmatvecCols (quant_simd.go:12-48,
// quant.go:108-122) and q4matvecCols (quant4_simd.go:17-57, quant4.go:126-154):
//   int8: acc_j = sum_i x_i * q_ij, then out_j = acc_j * scale_j;
//   int4: per 64-row group g, tmp_j = sum_{i in g} x_i * (nib_ij - 8), then
//         out_j = fma(tmp_j, scale_gj, out_j), the group fold of
//         quant4_simd.go:46-50.
//
// Data movement (bulk async copies, latency tolerant by construction):
//   The codes sit in HBM tiled (tq_common.cuh): an item, the 64-row x
//   128-byte block of one column tile and one 64-row unit (an int4 unit is
//   exactly one scale group), is 8 KB of contiguous memory, and items are
//   stored tile-major. Every warp owns two 8 KB shared-memory buffers; its
//   lane 0 loads a whole item with one cp.async.bulk, completion signalled
//   through an mbarrier transaction count, and keeps the next item in flight
//   while the warp unpacks the current one. 8 warps x 2 buffers keep 128 KB
//   per SM in flight. The activations of each item (64 rows x M) arrive by
//   cp.async one item ahead.
//
// Work split (stream-K, balanced to +-1 item per SM):
//   One persistent CTA per SM takes an equal contiguous slice of the
//   tile-major item list, i.e. one contiguous range of HBM. A slice crosses at most a few tile boundaries; the
//   CTA reduces its 8 warps in shared memory per tile segment. A tile wholly
//   inside one CTA is written directly; a tile shared by several CTAs gets
//   their partial sums through a scratch buffer and a per-tile arrival
//   counter: the last CTA to arrive adds the partials in CTA order and writes
//   the tile. Every sum therefore runs in a fixed order: results are
//   bit-reproducible run to run.
//
// Unpack: each 32-bit word of codes is spread into floats with byte_perm under
// the exponent of 2^23 (2^23 + byte, exact), one packed f32x2 add removes the
// offset, and packed f32x2 FMAs accumulate against the activation.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "tq_common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = TQ_TILE_BYTES;  // bytes of a code row per item
constexpr int kUnit = TQ_GROUP;       // rows per item
constexpr int kBuf = kTile * kUnit;   // 8 KB
constexpr unsigned long long kWaitNs = 2000000000ull; // mbarrier wait limit: 2 s

struct QmvParams {
    const uint8_t *codes;
    const float *scale;
    const float *x; // [M][rows]
    float *out;     // [M][cols]
    float *partial; // scratch: [2*ctas][M*TWC]
    unsigned *counters;
    unsigned *status;
    long long items;
    int rows, cols, half, units, tiles;
};

// ---- PTX helpers ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for phase `parity` of an mbarrier; gives up after kWaitNs, records
// TQ_STATUS_TIMEOUT and returns false (the caller then skips the item).
__device__ __noinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) {
            atomicOr(status, TQ_STATUS_TIMEOUT);
            return false;
        }
    }
}

// One contiguous global -> shared bulk copy (bytes a multiple of 16, both
// addresses 16-byte aligned), completing on the mbarrier's transaction count.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void cp_async_f32(float *dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- unpack -------------------------------------------------------------------
// Byte e of t placed under the exponent of 2^23: the float 2^23 + byte, exact.
__device__ __forceinline__ float tq_magic(uint32_t t, int e) {
    return __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7440 + e));
}

// NP float2 pairs per lane per activation row: int8 -> 4 columns (2 pairs);
// int4 -> 4 low-nibble columns then 4 high-nibble columns (4 pairs).
template <int BITS> __host__ __device__ constexpr int kPairs() { return BITS == 8 ? 2 : 4; }

template <int BITS, int M>
__device__ __forceinline__ void qmv_row(uint32_t w, const float (&xv)[M], float2 (&acc)[M][kPairs<BITS>()]) {
    if (BITS == 8) {
        const uint32_t t = w ^ 0x80808080u;                       // signed byte b -> b + 128
        const float2 off = make_float2(-8388736.0f, -8388736.0f); // 2^23 + 128
        const float2 c0 = __fadd2_rn(make_float2(tq_magic(t, 0), tq_magic(t, 1)), off);
        const float2 c1 = __fadd2_rn(make_float2(tq_magic(t, 2), tq_magic(t, 3)), off);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const float2 xx = make_float2(xv[m], xv[m]);
            acc[m][0] = __ffma2_rn(c0, xx, acc[m][0]);
            acc[m][1] = __ffma2_rn(c1, xx, acc[m][1]);
        }
    } else {
        const uint32_t l = w & 0x0F0F0F0Fu, h = (w >> 4) & 0x0F0F0F0Fu;
        const float2 off = make_float2(-8388616.0f, -8388616.0f); // 2^23 + 8
        const float2 c0 = __fadd2_rn(make_float2(tq_magic(l, 0), tq_magic(l, 1)), off);
        const float2 c1 = __fadd2_rn(make_float2(tq_magic(l, 2), tq_magic(l, 3)), off);
        const float2 c2 = __fadd2_rn(make_float2(tq_magic(h, 0), tq_magic(h, 1)), off);
        const float2 c3 = __fadd2_rn(make_float2(tq_magic(h, 2), tq_magic(h, 3)), off);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const float2 xx = make_float2(xv[m], xv[m]);
            acc[m][0] = __ffma2_rn(c0, xx, acc[m][0]);
            acc[m][1] = __ffma2_rn(c1, xx, acc[m][1]);
            acc[m][2] = __ffma2_rn(c2, xx, acc[m][2]);
            acc[m][3] = __ffma2_rn(c3, xx, acc[m][3]);
        }
    }
}

// Shared-memory layout (bytes):
//   bufs [kWarps][ST][kBuf]                code boxes (TMA destination); ST = 3
//                                          buffers per warp for M <= 2, else 2
//   xs   [kWarps][2][M][kUnit] floats      activations of the current/next item
//   red  [kWarps][M][2NP][32] floats       warp partials of a tile segment
//   flag [4] ints, mbar [kWarps][ST] u64
template <int BITS, int M> struct Smem {
    static constexpr int NP = kPairs<BITS>();
    static constexpr int ST = M <= 2 ? 3 : 2;
    static constexpr size_t bufs = (size_t)kWarps * ST * kBuf;
    static constexpr size_t xs = (size_t)kWarps * 2 * M * kUnit * sizeof(float);
    static constexpr size_t red = (size_t)kWarps * M * 2 * NP * 32 * sizeof(float);
    static constexpr size_t flag = 16;
    static constexpr size_t mbar = (size_t)kWarps * ST * sizeof(uint64_t);
    static constexpr size_t total = bufs + xs + red + flag + mbar;
};


template <int BITS, int M>
__global__ void __launch_bounds__(kThreads, 1) qmv_kernel(QmvParams p) {
    using S = Smem<BITS, M>;
    constexpr int NP = S::NP;
    constexpr int kStages = S::ST;
    constexpr int SLOTS = M * 2 * NP * 32; // partial entries per tile segment (M x tile columns)
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *bufs = smem;
    float *xs_all = reinterpret_cast<float *>(smem + S::bufs);
    float *red = reinterpret_cast<float *>(smem + S::bufs + S::xs);
    int *flag = reinterpret_cast<int *>(smem + S::bufs + S::xs + S::red);
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + S::bufs + S::xs + S::red + S::flag);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const TqSplit split(p.items, G);
    const long long i0 = split.start(c), i1 = split.start(c + 1);
    uint8_t *wbuf = bufs + (size_t)warp * kStages * kBuf;
    float *wx = xs_all + (size_t)warp * 2 * M * kUnit;
    uint64_t *wbar = mbar + warp * kStages;

    if (lane == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(&wbar[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();

    // This warp's items: i0 + warp + kWarps*k, k = 0 .. nk-1.
    const long long first = i0 + warp;
    const int nk = first < i1 ? (int)((i1 - first + kWarps - 1) / kWarps) : 0;
    bool ok = true; // false once a wait timed out: the warp stops issuing copies

    auto issue_codes = [&](int k) {
        const long long it = first + (long long)k * kWarps;
        uint64_t *bar = &wbar[k % kStages];
        mbar_arrive_expect_tx(bar, kBuf);
        bulk_load(wbuf + (size_t)(k % kStages) * kBuf, p.codes + it * kBuf, kBuf, bar);
    };
    auto issue_x = [&](int k) {
        const long long it = first + (long long)k * kWarps;
        const int unit = (int)(it % p.units);
        float *dst = wx + (k & 1) * M * kUnit;
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int r = lane; r < kUnit; r += 32) {
                const int row = unit * kUnit + r;
                const bool v = row < p.rows;
                cp_async_f32(dst + m * kUnit + r, p.x + (size_t)m * p.rows + (v ? row : 0), v);
            }
    };

    if (lane == 0)
        for (int k = 0; k < kStages && k < nk; k++) issue_codes(k);
    if (nk > 0) issue_x(0);
    cp_async_commit();

    int k = 0; // next item of this warp
    // Tile segments of [i0, i1), in order.
    for (long long seg0 = i0; seg0 < i1;) {
        const int tile = (int)(seg0 / p.units);
        const long long seg1 = min(i1, (long long)(tile + 1) * p.units);

        float2 acc[M][NP];
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int q = 0; q < NP; q++) acc[m][q] = make_float2(0.f, 0.f);

        for (; k < nk; k++) {
            const long long it = first + (long long)k * kWarps;
            if (it >= seg1) break;
            const int unit = (int)(it % p.units);
            const int nrows = min(kUnit, p.rows - unit * kUnit);

            if (k + 1 < nk) issue_x(k + 1);
            cp_async_commit();
            float4 slo = make_float4(0.f, 0.f, 0.f, 0.f), shi = slo;
            if (BITS == 4) {
                const float *sp = p.scale + it * (2 * kTile) + lane * 4;
                slo = __ldg(reinterpret_cast<const float4 *>(sp));
                shi = __ldg(reinterpret_cast<const float4 *>(sp + kTile));
            }
            const bool ready = ok && mbar_wait(&wbar[k % kStages], (uint32_t)((k / kStages) & 1), p.status);
            ok = ok && ready;
            cp_async_wait<1>();
            __syncwarp();
            if (ready) {
                // Lane l reads bytes 4l..4l+3 of each row: chunk l/4, stored at chunk (l/4) ^ (r%8).
                const uint32_t *codes = reinterpret_cast<const uint32_t *>(wbuf + (size_t)(k % kStages) * kBuf) + (lane & 3);
                const float *xk = wx + (k & 1) * M * kUnit;
                float2 tmp[M][NP];
#pragma unroll
                for (int m = 0; m < M; m++)
#pragma unroll
                    for (int q = 0; q < NP; q++) tmp[m][q] = make_float2(0.f, 0.f);
                if (nrows == kUnit) {
#pragma unroll 16
                    for (int r = 0; r < kUnit; r++) {
                        float xv[M];
#pragma unroll
                        for (int m = 0; m < M; m++) xv[m] = xk[m * kUnit + r];
                        qmv_row<BITS, M>(codes[r * (kTile / 4) + (((lane >> 2) ^ (r & 7)) << 2)], xv, BITS == 8 ? acc : tmp);
                    }
                } else {
                    for (int r = 0; r < nrows; r++) {
                        float xv[M];
#pragma unroll
                        for (int m = 0; m < M; m++) xv[m] = xk[m * kUnit + r];
                        qmv_row<BITS, M>(codes[r * (kTile / 4) + (((lane >> 2) ^ (r & 7)) << 2)], xv, BITS == 8 ? acc : tmp);
                    }
                }
                if (BITS == 4) {
                    const float2 sl0 = make_float2(slo.x, slo.y), sl1 = make_float2(slo.z, slo.w);
                    const float2 sh0 = make_float2(shi.x, shi.y), sh1 = make_float2(shi.z, shi.w);
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        acc[m][0] = __ffma2_rn(tmp[m][0], sl0, acc[m][0]);
                        acc[m][1] = __ffma2_rn(tmp[m][1], sl1, acc[m][1]);
                        acc[m][2] = __ffma2_rn(tmp[m][2], sh0, acc[m][2]);
                        acc[m][3] = __ffma2_rn(tmp[m][3], sh1, acc[m][3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && ok && k + kStages < nk) {
                fence_proxy_async(); // generic-proxy reads of this buffer happen before the TMA overwrite
                issue_codes(k + kStages);
            }
        }

        // ---- reduce the tile segment over the 8 warps ------------------------
        // Entry (m, e, lane) of warp w at red[((w*M + m)*2NP + e)*32 + lane].
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int q = 0; q < NP; q++) {
                red[((warp * M + m) * 2 * NP + 2 * q) * 32 + lane] = acc[m][q].x;
                red[((warp * M + m) * 2 * NP + 2 * q + 1) * 32 + lane] = acc[m][q].y;
            }
        __syncthreads();
        for (int idx = threadIdx.x; idx < SLOTS; idx += kThreads) {
            float s = red[idx];
#pragma unroll
            for (int w = 1; w < kWarps; w++) s += red[w * SLOTS + idx];
            red[idx] = s;
        }

        // Which CTAs contribute to this tile, and is this one the last to arrive?
        const long long t0 = (long long)tile * p.units, t1 = t0 + p.units;
        const int cf = split.owner(t0), cl = split.owner(t1 - 1);
        const bool shared_tile = cf != cl;
        const float *src = red;
        if (shared_tile) {
            float *dst = p.partial + (size_t)split.slot(c, t0) * SLOTS;
            __syncthreads();
            for (int idx = threadIdx.x; idx < SLOTS; idx += kThreads) dst[idx] = red[idx];
            __syncthreads();
            if (threadIdx.x == 0) flag[0] = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1));
            __syncthreads();
            if (!flag[0]) src = nullptr;
        } else {
            __syncthreads();
        }

        if (src) {
            for (int idx = threadIdx.x; idx < SLOTS; idx += kThreads) {
                float s;
                if (shared_tile) {
                    // contributors in CTA order, four loads in flight
                    s = 0.f;
                    const int slot_f = split.slot(cf, t0);
                    for (int cc = cf; cc <= cl; cc += 4) {
                        float pv[4];
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const int c2 = cc + u;
                            const int slot = c2 == cf ? slot_f : 2 * c2;
                            pv[u] = c2 <= cl ? __ldcg(p.partial + (size_t)slot * SLOTS + idx) : 0.f;
                        }
#pragma unroll
                        for (int u = 0; u < 4; u++) s += pv[u];
                    }
                } else {
                    s = src[idx];
                }
                const int l = idx & 31, e = (idx >> 5) % (2 * NP), m = (idx >> 5) / (2 * NP);
                const int b = tile * kTile + l * 4; // this lane's first byte in the row
                if (BITS == 8) {
                    const int col = b + e;
                    if (col < p.cols) p.out[(size_t)m * p.cols + col] = s * p.scale[col];
                } else {
                    const int pr = b + (e & 3); // column pair
                    const int col = e < 4 ? pr : p.half + pr;
                    if (pr < p.half) p.out[(size_t)m * p.cols + col] = s;
                }
            }
        }
        __syncthreads(); // red is rewritten by the next segment
        seg0 = seg1;
    }
    cp_async_wait<0>();
}

// Per-device set-up of qmv_kernel<BITS, M>: its shared-memory attribute, which
// also loads the kernel's code onto the device.
template <int BITS, int M> TqDeviceOnce g_qmv_once;
template <int BITS, int M> cudaError_t qmv_setup(int dev) {
    using S = Smem<BITS, M>;
    return tq_device_once(g_qmv_once<BITS, M>, dev, [] {
        return cudaFuncSetAttribute(qmv_kernel<BITS, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::total);
    });
}

template <int BITS, int M>
cudaError_t launch_qmv(const TqMatrixDev &mat, const float *x, float *out, const TqScratch &scr, cudaStream_t st) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if ((e = qmv_setup<BITS, M>(dev)) != cudaSuccess) return e;
    const int sms = g_qmv_once<BITS, M>.sms[dev];
    QmvParams prm;
    prm.codes = mat.codes;
    prm.scale = mat.scale;
    prm.x = x;
    prm.out = out;
    prm.partial = scr.partial;
    prm.counters = scr.counters;
    prm.status = scr.status;
    prm.rows = mat.rows;
    prm.cols = mat.cols;
    prm.half = mat.cols / 2;
    prm.units = mat.units;
    prm.tiles = mat.tiles;
    prm.items = (long long)prm.tiles * prm.units;
    if (prm.tiles > TQ_MAX_TILES || sms > TQ_MAX_CTAS) return cudaErrorInvalidValue;
    const int ctas = (int)(prm.items < sms ? prm.items : sms);
    qmv_kernel<BITS, M><<<ctas, kThreads, Smem<BITS, M>::total, st>>>(prm);
    return cudaGetLastError();
}

template <int BITS>
cudaError_t dispatch_m(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                       cudaStream_t st) {
    switch (M) {
    case 1: return launch_qmv<BITS, 1>(mat, x, out, scr, st);
    case 2: return launch_qmv<BITS, 2>(mat, x, out, scr, st);
    case 3: return launch_qmv<BITS, 3>(mat, x, out, scr, st);
    case 4: return launch_qmv<BITS, 4>(mat, x, out, scr, st);
    case 5: return launch_qmv<BITS, 5>(mat, x, out, scr, st);
    case 6: return launch_qmv<BITS, 6>(mat, x, out, scr, st);
    case 7: return launch_qmv<BITS, 7>(mat, x, out, scr, st);
    default: return launch_qmv<BITS, 8>(mat, x, out, scr, st);
    }
}

} // namespace

// out[M][cols] = x[M][rows] @ W. M > 8 runs as consecutive 8-row launches.
cudaError_t tq_launch_matvec(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                             cudaStream_t st) {
    if (M <= 0 || mat.cols == 0) return cudaSuccess;
    if (mat.rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
    for (int m0 = 0; m0 < M; m0 += 8) {
        const int mm = M - m0 < 8 ? M - m0 : 8;
        const float *xm = x + (size_t)m0 * mat.rows;
        float *om = out + (size_t)m0 * mat.cols;
        cudaError_t e =
            mat.bits == 8 ? dispatch_m<8>(mat, xm, om, mm, scr, st) : dispatch_m<4>(mat, xm, om, mm, scr, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}


// ---------------------------------------------------------------------------
// Allocation-free variant (tq_matmul_dev_fixed in the C ABI): the same kernel
// with its cross-CTA scratch in fixed device arrays of this file instead of
// the per-stream scratch the library allocates on first use.
// ---------------------------------------------------------------------------
namespace {

constexpr int kFixedRows = TQ_FIXED_ROWS_PER_LAUNCH; // activation rows per launch (more: consecutive launches)
constexpr int kFixedCtas = TQ_FIXED_MAX_SMS;          // largest grid served (one CTA per SM; a B200 has 148)
constexpr int kFixedTiles = TQ_FIXED_MAX_TILES;       // column tiles: 524,288 int8 / 1,048,576 int4 columns
// Partial sums: two slots per CTA of up to kFixedRows x 256 floats (int4, the
// larger case): 1.25 MiB.
constexpr size_t kFixedPartialFloats = (size_t)2 * kFixedCtas * kFixedRows * 2 * kPairs<4>() * 32;

// Must be zero before the first launch: the tile arrival counters and the
// status word. Static device memory is zero when the module loads, and every
// launch leaves each counter it used at zero again (the last CTA to arrive at
// a tile re-arms it). The partial sums need no initial value.
static __device__ __align__(256) float g_fixed_partial[kFixedPartialFloats];
static __device__ __align__(256) unsigned g_fixed_words[kFixedTiles + 32]; // counters, then status

struct FixedScratch {
    bool ready;
    int sms;
    TqScratch scr;
};
FixedScratch g_fixed[64];
std::mutex g_fixed_mu;

// Loads and configures every kernel the fixed path can launch (int8 and int4,
// 1..kFixedRows rows), so that no later call loads code onto the device.
cudaError_t fixed_kernels_setup(int dev) {
    const cudaError_t es[] = {qmv_setup<8, 1>(dev), qmv_setup<8, 2>(dev), qmv_setup<8, 3>(dev), qmv_setup<8, 4>(dev),
                              qmv_setup<4, 1>(dev), qmv_setup<4, 2>(dev), qmv_setup<4, 3>(dev), qmv_setup<4, 4>(dev)};
    static_assert(kFixedRows == 4, "one set-up per row count");
    for (cudaError_t e : es)
        if (e != cudaSuccess) return e;
    return cudaSuccess;
}

} // namespace

// Launches out = x @ W for M rows with the fixed scratch. Set-up runs once per
// device, with that device current: the symbol addresses of the fixed arrays
// (cudaGetSymbolAddress), the SM count, and the kernels' code and attributes.
// Returns TQ_FIXED_OK or the limit that was exceeded; *err holds a CUDA error
// for TQ_FIXED_CUDA.
int tq_launch_matvec_fixed(const TqMatrixDev &mat, const float *x, float *out, int M, cudaStream_t st,
                           cudaError_t *err) {
    *err = cudaSuccess;
    int dev = 0;
    if ((*err = cudaGetDevice(&dev)) != cudaSuccess) return TQ_FIXED_CUDA;
    if (dev < 0 || dev >= 64) return TQ_FIXED_DEVICE;
    TqScratch scr;
    {
        std::lock_guard<std::mutex> lk(g_fixed_mu);
        FixedScratch &f = g_fixed[dev];
        if (!f.ready) {
            void *partial = nullptr, *words = nullptr;
            if ((*err = cudaGetSymbolAddress(&partial, g_fixed_partial)) != cudaSuccess) return TQ_FIXED_CUDA;
            if ((*err = cudaGetSymbolAddress(&words, g_fixed_words)) != cudaSuccess) return TQ_FIXED_CUDA;
            if ((*err = cudaDeviceGetAttribute(&f.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
                return TQ_FIXED_CUDA;
            if ((*err = fixed_kernels_setup(dev)) != cudaSuccess) return TQ_FIXED_CUDA;
            f.scr.partial = static_cast<float *>(partial);
            f.scr.counters = static_cast<unsigned *>(words);
            f.scr.status = static_cast<unsigned *>(words) + kFixedTiles;
            f.scr.planes = nullptr;
            f.scr.mm_partial = nullptr;
            f.ready = true;
        }
        if (f.sms > kFixedCtas) return TQ_FIXED_SMS;
        scr = f.scr;
    }
    if (mat.tiles > kFixedTiles) return TQ_FIXED_TILES;
    if (M <= 0 || mat.cols == 0) return TQ_FIXED_OK;
    if (mat.rows == 0) {
        *err = cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
        return *err == cudaSuccess ? TQ_FIXED_OK : TQ_FIXED_CUDA;
    }
    for (int m0 = 0; m0 < M; m0 += kFixedRows) {
        const int mm = M - m0 < kFixedRows ? M - m0 : kFixedRows;
        const float *xm = x + (size_t)m0 * mat.rows;
        float *om = out + (size_t)m0 * mat.cols;
        *err = mat.bits == 8 ? dispatch_m<8>(mat, xm, om, mm, scr, st) : dispatch_m<4>(mat, xm, om, mm, scr, st);
        if (*err != cudaSuccess) return TQ_FIXED_CUDA;
    }
    return TQ_FIXED_OK;
}

// The fixed scratch's status bits on the current device (0 before its first
// call), with the device idle. A timeout may have left tile counters
// mid-count, so when the status is set the counters and the status word are
// zeroed again (plain memsets of the fixed array; nothing is allocated).
cudaError_t tq_fixed_status(unsigned *bits) {
    *bits = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return e;
    std::lock_guard<std::mutex> lk(g_fixed_mu);
    const FixedScratch &f = g_fixed[dev];
    if (!f.ready) return cudaSuccess;
    if ((e = cudaMemcpy(bits, f.scr.status, sizeof *bits, cudaMemcpyDeviceToHost)) != cudaSuccess) return e;
    if (*bits) e = cudaMemset(f.scr.counters, 0, sizeof(unsigned) * (kFixedTiles + 32));
    return e;
}
