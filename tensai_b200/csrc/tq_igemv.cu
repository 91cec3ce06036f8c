// tq_igemv.cu — weight-only int8 / int4 matvec (M <= 8 activation rows) on the
// 5th-generation tensor cores with exact integer products.
//
// Computes out[m][j] = sum_i x[m][i] * W[i][j], the product of qmatvecCols
// (quant_simd.go:12-48) and q4matvecCols (quant4_simd.go:17-57), without
// dequantizing the weights:
//
//   * The codes are the UMMA A operand as stored: int8 codes are signed 8-bit
//     integers already; int4 codes expand to unsigned bytes n = nibble
//     (0..15) by one mask (low run) or shift+mask (high run), in place.
//   * Per 64-row unit (an int4 scale group) and activation row m, x is scaled
//     by a power of two 2^e_m (exact) so |x|/2^e < 64, and split into four
//     signed 7-bit digits: x/2^e = b0 + b1/128 + b2/128^2 + b3/128^3 + r with
//     |r| <= 2^-22. The digits are the UMMA B operand (N = 4M columns,
//     padded to 16 or 32).
//   * tcgen05.mma.kind::i8 forms D_p = sum_i code_i * b_p,i exactly in int32
//     in tensor memory (128 weight columns x N, one MMA per 32 rows).
//   * The epilogue rebuilds each unit's dot product in fp32:
//       int8: v = 2^e * sum_p D_p 128^-p                  (acc += v)
//       int4: v = 2^e * sum_p (D_p - 8 sum_i b_p,i) 128^-p (acc = fma(v, scale_g, acc))
//     and int8 multiplies by the column scale at the end (quant.go:120).
//   Only the digit truncation (<= 2^-22 of the unit's largest |x|) and the
//   fp32 rebuild round, so the result is at least as accurate as the
//   reference's fp32 accumulation.
//
// Two launches per call, chained with programmatic dependent launch:
//   planes_kernel  one CTA per 64-row unit: the unit's digit planes in the
//                  UMMA B layout plus its 2^e and digit sums, into scratch.
//   igemv_kernel   starts streaming weights at once (they depend on nothing),
//                  and waits for the planes (griddepcontrol.wait) only before
//                  loading them, touching scratch or writing the output.
//
// igemv schedule. The codes sit in HBM as 8 KB items (128 code bytes x 64
// rows), tile-major. One persistent CTA per SM takes an equal contiguous
// slice of the item list (stream-K, balanced to +-1 item). The slice is walked
// as batches of up to NU consecutive units of one column tile (contiguous in
// HBM): one bulk copy of the codes and one of the B planes per batch, one
// MMA-issuer wait and one commit per batch, so the tensor-core control cost is
// amortized over 8 MMAs. Warp roles (14 warps):
//   warp 0      producer: bulk copies into a ring of code stages
//   warp 1      owns the tensor memory; lane 0 issues the MMAs
//   warps 2-5   int4 only: nibble -> byte expansion into operand stages
//   warps 6-13  epilogue, two warpgroups taking alternate batches: tcgen05.ld
//               of the accumulators, scale folding, per-tile output. Tiles
//               shared with other CTAs reduce through scratch partials; the
//               last CTA to arrive adds them in CTA order, so results are
//               bit-reproducible.
// One commit per batch lands on done[b % DR]; the producer (stage reuse), the
// expansion warps (operand-stage reuse) and the epilogue (accumulators ready)
// all wait on it for their own batch index.
// Every mbarrier wait is bounded (2 s); a timeout sets TQ_STATUS_TIMEOUT and a
// CTA-wide abort flag that turns all later waits into no-ops, so a fault
// ends the kernel instead of hanging it.
#include <cuda.h>

#include "tq_common.cuh"

namespace {

constexpr int kItem = TQ_ITEM_BYTES; // 8192
constexpr int kRows = TQ_GROUP;      // 64
constexpr int kCols = TQ_TILE_BYTES; // 128
constexpr int kExpWarps = 4;         // warps 2..5
constexpr int kEpiWarp0 = 2 + kExpWarps;
constexpr int kEpiThreads = 128; // one epilogue warpgroup
constexpr int kThreads = (kEpiWarp0 + 8) * 32;
constexpr unsigned long long kWaitNs = 2000000000ull;

// Planes buffer of one call: B blocks [units][BBYTES], then meta [units][MB]
// (2^e per row m, then the four digit sums per row m, as ints).
template <int M> struct Planes {
    static constexpr int N = 4 * M <= 16 ? 16 : 32;    // UMMA N: digit planes, padded
    static constexpr int KSTEP_B = (N / 8) * 256;      // B bytes per 32-row MMA step
    static constexpr int BBYTES = 2 * KSTEP_B;         // B bytes per unit
    static constexpr int MB = (M * 20 + 15) / 16 * 16; // meta bytes per unit
};

template <int BITS, int M> struct Cfg {
    using PL = Planes<M>;
    static constexpr int N = PL::N;
    static constexpr int KSTEP_B = PL::KSTEP_B;
    static constexpr int BB = PL::BBYTES;
    static constexpr int NU = BITS == 8 ? 4 : 2;    // units per batch
    static constexpr int H = BITS == 8 ? 1 : 2;     // column runs per unit (int4: low, high nibbles)
    static constexpr int ACC = H * N;               // accumulator columns per unit
    static constexpr int BACC = NU * ACC;           // per batch
    static constexpr int NBUF = 4 * BACC <= 512 ? 4 : 2; // accumulator buffers
    static constexpr int TCOLS = NBUF * BACC <= 128 ? 128 : (NBUF * BACC <= 256 ? 256 : 512);
    // code stage    [codes NU x 8 KB | B planes NU x BB]; int8: the codes are the A operand.
    // operand stage [NU x (A lo 8 KB | A hi 8 KB)] (int4 only).
    static constexpr int CSTRIDE = (NU * (kItem + BB) + 1023) & ~1023;
    static constexpr int OSTRIDE = NU * 2 * kItem;
    static constexpr int OST = BITS == 8 ? 0 : 2;
    static constexpr int RED_BYTES = 2 * M * kCols * 4;   // warpgroup 1 -> 0 partial sums
    static constexpr int MSLOTS = 6;                      // prefetched meta batches per warpgroup
    static constexpr int META_BYTES = 2 * MSLOTS * NU * PL::MB;
    static constexpr int FIXED = RED_BYTES + META_BYTES + 512 + 1024;
    static constexpr int BUDGET = 227 * 1024 - FIXED - OST * OSTRIDE;
    static constexpr int CST = BUDGET / CSTRIDE < 12 ? BUDGET / CSTRIDE : 12; // code stages
    static constexpr int DR = (CST > NBUF ? CST : NBUF) + 2;                  // done-barrier ring
    static constexpr int O_OFF = 0;
    static constexpr int C_OFF = OST * OSTRIDE;
    static constexpr int RED_OFF = C_OFF + CST * CSTRIDE;
    static constexpr int META_OFF = RED_OFF + RED_BYTES;
    static constexpr int BAR_OFF = (META_OFF + META_BYTES + 15) & ~15;
    static constexpr int NBARS = CST + OST + DR + NBUF;
    static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
    static constexpr int SMEM = MISC_OFF + 32 + 1024;
    static_assert(NBUF * BACC <= TCOLS && TCOLS <= 512, "accumulators must fit tensor memory");
    static_assert(CST >= 4, "too few code stages");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct IgParams {
    const uint8_t *codes;
    const float *scale;
    const uint8_t *planes; // B blocks [units][BB], then meta [units][MB]
    float *out;
    float *partial;
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
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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
// Bounded wait on phase `parity`; on timeout (or if the CTA already aborted)
// sets the abort flag and returns false.
__device__ __noinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *status) {
    if (*abort) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_ns() - t0 > kWaitNs) {
            atomicOr(status, TQ_STATUS_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
}
// Fast path inline (phase already complete), bounded slow path out of line.
__device__ __forceinline__ bool wait_fast(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *status) {
    return mbar_try_wait(bar, parity) || wait_bar(bar, parity, abort, status);
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor: start, leading/stride byte offsets, version 1
// (sm_100), layout type (0 = no swizzle, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 columns of 32-bit accumulators (this warp's lane quarter).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// Instruction descriptor of tcgen05.mma.kind::i8: D s32, A = codes (s8 for
// int8, u8 for int4; MN-major), B = digits (s8, K-major), M = 128, N.
template <int BITS, int N> __device__ __forceinline__ uint32_t idesc_i8() {
    return (2u << 4) | ((BITS == 8 ? 1u : 0u) << 7) | (1u << 10) | (1u << 15) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// ---------------------------------------------------------------------------
// planes_kernel: digit planes of x for one 64-row unit per CTA (64 threads,
// thread t = row t of the unit). For activation row m: 2^e_m with
// max_i |x_m,i| in [2^(e_m+5), 2^(e_m+6)), digits b_q of x/2^e_m (round to
// nearest even, remainder times 128), written as B[n = 4m+q][k = t] in the
// UMMA K-major no-swizzle layout: byte (n, k) of 32-row step j sits at
// j*KSTEP_B + (n/8)*256 + (k%32/16)*128 + (n%8)*16 + k%16.
// ---------------------------------------------------------------------------
template <int M>
__global__ void __launch_bounds__(64) planes_kernel(const float *__restrict__ x, int rows, int units,
                                                   uint8_t *__restrict__ planes) {
    using PL = Planes<M>;
    __shared__ float red_max[2][M];
    __shared__ int red_bad[2][M];
    __shared__ int red_sum[2][M][4];
    pdl_trigger();
    pdl_wait(); // x is produced by the previous kernel on the stream
    const int u = blockIdx.x, t = threadIdx.x, w = t >> 5, lane = t & 31;
    uint8_t *B = planes + (size_t)u * PL::BBYTES;
    float *meta = reinterpret_cast<float *>(planes + (size_t)units * PL::BBYTES + (size_t)u * PL::MB);
    const int row = u * kRows + t;
    float v[M];
#pragma unroll
    for (int m = 0; m < M; m++) {
        v[m] = row < rows ? x[(size_t)m * rows + row] : 0.f;
        float mx = fabsf(v[m]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // fmaxf skips NaN: a NaN or infinity is flagged on its own
        const int bad = __any_sync(0xffffffffu, !(fabsf(v[m]) <= 3.402823466e38f));
        if (lane == 0) {
            red_max[w][m] = mx;
            red_bad[w][m] = bad;
        }
    }
    __syncthreads();
    const int kk = t & 31, j = t >> 5;
#pragma unroll
    for (int m = 0; m < M; m++) {
        const bool bad = red_bad[0][m] | red_bad[1][m];
        const float mx = bad ? 0.f : fmaxf(red_max[0][m], red_max[1][m]);
        int e = 0;
        if (mx > 0.f) frexpf(mx, &e); // mx = f * 2^e, f in [0.5, 1)
        float r = mx > 0.f ? ldexpf(v[m], 6 - e) : 0.f; // exact: |r| < 64
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const float di = rintf(r);
            const int d = (int)di;
            r = (r - di) * 128.0f; // exact
            const int n = m * 4 + q;
            B[j * PL::KSTEP_B + (n >> 3) * 256 + (kk >> 4) * 128 + (n & 7) * 16 + (kk & 15)] = (uint8_t)(int8_t)d;
            int sum = d;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) red_sum[w][m][q] = sum;
        }
        // a NaN or infinity in the unit: no digits, and its sums become NaN
        if (t == 0) meta[m] = bad ? __uint_as_float(0x7FC00000u) : mx > 0.f ? ldexpf(1.0f, e - 6) : 0.f;
    }
    __syncthreads();
    if (t < 4 * M) {
        const int m = t >> 2, q = t & 3;
        reinterpret_cast<int *>(meta)[M + m * 4 + q] = red_sum[0][m][q] + red_sum[1][m][q];
    }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The batch sequence of one CTA: up to NU consecutive units of one tile.
struct BatchWalk {
    int tile, unit, left, units;
    __device__ __forceinline__ int next(int NU) { // units in the next batch (0 = done)
        int n = units - unit;
        if (n > NU) n = NU;
        if (n > left) n = left;
        return n;
    }
    __device__ __forceinline__ bool advance(int n) { // true if the tile segment ended
        unit += n;
        left -= n;
        if (unit == units) {
            unit = 0;
            tile++;
            return true;
        }
        return left == 0;
    }
};

template <int BITS, int M>
__global__ void __launch_bounds__(kThreads, 1) igemv_kernel(IgParams p) {
    using C = Cfg<BITS, M>;
    using PL = Planes<M>;
    constexpr int CS = C::CST, OS = C::OST, DR = C::DR, NB = C::NBUF, NU = C::NU, H = C::H, N = C::N;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *cfull = bars, *ofull = bars + CS, *done = ofull + OS, *accempty = done + DR;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);
    volatile int *lastflag = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 8);
    auto cstage = [&](int k) { return smem + C::C_OFF + (k % CS) * C::CSTRIDE; };
    auto ostage = [&](int k) { return smem + C::O_OFF + (k % (OS ? OS : 1)) * C::OSTRIDE; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const TqSplit split(p.items, G);
    const long long i0 = split.start(c), i1 = split.start(c + 1);
    const BatchWalk walk0{(int)(i0 / p.units), (int)(i0 % p.units), (int)(i1 - i0), p.units};
    int nbatches = 0;
    {
        BatchWalk w = walk0;
        for (int n; (n = w.next(NU)) > 0; w.advance(n)) nbatches++;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < CS; s++) mbar_init(&cfull[s], 1);
        for (int s = 0; s < OS; s++) mbar_init(&ofull[s], 1);
        for (int s = 0; s < DR; s++) mbar_init(&done[s], 1);
        for (int b = 0; b < NB; b++) mbar_init(&accempty[b], 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            // The first CS batches' codes depend on nothing: stream them before
            // the planes (written by the preceding kernel) are known to be ready.
            BatchWalk w = walk0;
            const int pre = nbatches < CS ? nbatches : CS;
            for (int k = 0; k < pre; k++) {
                const int n = w.next(NU);
                const long long it = (long long)w.tile * p.units + w.unit;
                mbar_arrive_expect_tx(&cfull[k], n * (kItem + C::BB));
                bulk_load(cstage(k), p.codes + it * kItem, n * kItem, &cfull[k]);
                w.advance(n);
            }
            pdl_wait();
            w = walk0;
            for (int k = 0; k < nbatches; k++) {
                const int n = w.next(NU);
                const long long it = (long long)w.tile * p.units + w.unit;
                if (k >= pre) {
                    // stage k % CS last held batch k - CS
                    if (!wait_fast(&done[(k - CS) % DR], ((k - CS) / DR) & 1, abort, p.status)) {
                        w.advance(n);
                        continue;
                    }
                    mbar_arrive_expect_tx(&cfull[k % CS], n * (kItem + C::BB));
                    bulk_load(cstage(k), p.codes + it * kItem, n * kItem, &cfull[k % CS]);
                }
                bulk_load(cstage(k) + NU * kItem, p.planes + (size_t)w.unit * C::BB, n * C::BB, &cfull[k % CS]);
                w.advance(n);
            }
            pdl_trigger(); // every load is issued: the next kernel may start its prologue
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_i8<BITS, N>();
            BatchWalk w = walk0;
            for (int k = 0; k < nbatches; k++) {
                const int n = w.next(NU);
                w.advance(n);
                const int buf = k % NB;
                const bool ok_a = BITS == 8 ? wait_fast(&cfull[k % CS], (k / CS) & 1, abort, p.status)
                                            : wait_fast(&ofull[k % (OS ? OS : 1)], (k / (OS ? OS : 1)) & 1, abort, p.status);
                const bool ok_c = wait_fast(&accempty[buf], ((k / NB) & 1) ^ 1, abort, p.status);
                if (!(ok_a && ok_c)) continue;
                tc_fence_after();
                const uint32_t asb = smem_u32(BITS == 8 ? cstage(k) : ostage(k));
                const uint32_t bsb = smem_u32(cstage(k) + NU * kItem);
                const uint32_t d0 = tbase + (uint32_t)(buf * C::BACC);
                for (int j = 0; j < n; j++) {
#pragma unroll
                    for (int ks = 0; ks < 2; ks++) { // two 32-row K steps per unit
                        const uint64_t bd = umma_desc(bsb + j * C::BB + ks * C::KSTEP_B, 128, 256, 0);
#pragma unroll
                        for (int h = 0; h < H; h++)
                            umma_i8(d0 + j * C::ACC + h * N,
                                    umma_desc(asb + (j * H + h) * kItem + ks * 4096, kItem, 1024, 2), bd, idesc, ks);
                    }
                }
                umma_commit(&done[k % DR]);
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------- int4: nibbles -> bytes (position for position) ----------------
        if (BITS == 4) {
            const int t = threadIdx.x - 64;
            constexpr int NT = kExpWarps * 32;
            BatchWalk w = walk0;
            for (int k = 0; k < nbatches; k++) {
                const int n = w.next(NU);
                w.advance(n);
                bool ok = wait_fast(&cfull[k % CS], (k / CS) & 1, abort, p.status);
                if (k >= OS) ok = wait_fast(&done[(k - OS) % DR], ((k - OS) / DR) & 1, abort, p.status) && ok;
                if (ok) {
                    const uint4 *P = reinterpret_cast<const uint4 *>(cstage(k));
                    uint4 *A = reinterpret_cast<uint4 *>(ostage(k));
                    for (int j = 0; j < n; j++) {
#pragma unroll
                        for (int q = t; q < kItem / 16; q += NT) {
                            const uint4 v = P[j * (kItem / 16) + q];
                            A[(2 * j) * (kItem / 16) + q] =
                                make_uint4(v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu);
                            A[(2 * j + 1) * (kItem / 16) + q] =
                                make_uint4((v.x >> 4) & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                           (v.w >> 4) & 0x0F0F0F0Fu);
                        }
                    }
                }
                fence_proxy_async(); // generic-proxy writes become visible to the tensor cores
                named_sync(1, NT);
                if (t == 0) mbar_arrive(&ofull[k % (OS ? OS : 1)]);
            }
        }
    } else {
        // ---------------- epilogue: two warpgroups take alternate batches ----------------
        // Warp w reads TMEM lanes 32*(w%4)..+31, i.e. tile columns of that range.
        pdl_wait(); // planes, scratch and the output belong to the previous kernel until here
        const int g = (warp - kEpiWarp0) >> 2;
        const int q4 = warp & 3;
        const int col = q4 * 32 + lane; // tile column of this thread (int4: pair index in each run)
        const int et = threadIdx.x - kEpiWarp0 * 32 - g * kEpiThreads; // 0..127 within the warpgroup
        const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
        float *red = reinterpret_cast<float *>(smem + C::RED_OFF); // [H][M][128] from warpgroup 1
        uint8_t *mring = smem + C::META_OFF + g * C::MSLOTS * NU * PL::MB;
        const uint8_t *meta_g = p.planes + (size_t)p.units * PL::BBYTES;
        // Meta prefetch: this warpgroup's j-th batch is batch 2j + g; cp.async
        // one group per batch, MSLOTS - 2 batches ahead.
        constexpr int PD = C::MSLOTS - 2;
        BatchWalk pw = walk0; // prefetch walker: positioned at batch index pk
        int pk = 0;
        auto skip_to_mine = [&]() {
            while (pk < nbatches && (pk & 1) != g) {
                pw.advance(pw.next(NU));
                pk++;
            }
        };
        auto prefetch = [&]() {
            skip_to_mine();
            if (pk < nbatches) {
                const int n = pw.next(NU);
                const int slot = (pk >> 1) % C::MSLOTS;
                for (int q = et; q < n * PL::MB / 16; q += kEpiThreads)
                    cp_async16(mring + slot * NU * PL::MB + q * 16, meta_g + (size_t)pw.unit * PL::MB + q * 16);
                pw.advance(n);
                pk++;
            }
            cp_async_commit();
        };
        for (int i = 0; i < PD; i++) prefetch();

        BatchWalk w = walk0;
        int k = 0;
        while (k < nbatches) {
            const int tile = w.tile;
            float acc[H][M];
#pragma unroll
            for (int h = 0; h < H; h++)
#pragma unroll
                for (int m = 0; m < M; m++) acc[h][m] = 0.f;
            bool seg_end = false;
            while (!seg_end) {
                const int n = w.next(NU);
                const long long it0 = (long long)w.tile * p.units + w.unit;
                seg_end = w.advance(n);
                if ((k & 1) == g) {
                    const int buf = k % NB;
                    float wsc[NU][H];
                    if (BITS == 4) {
#pragma unroll
                        for (int j = 0; j < NU; j++)
#pragma unroll
                            for (int h = 0; h < H; h++)
                                wsc[j][h] = j < n ? __ldg(p.scale + (it0 + j) * (2 * kCols) + h * kCols + col) : 0.f;
                    }
                    prefetch(); // batch (k >> 1) + PD of this warpgroup
                    cp_async_wait<C::MSLOTS - 2>(); // this thread's part of batch k's meta has landed
                    bool ok = wait_fast(&done[k % DR], (k / DR) & 1, abort, p.status);
                    ok = __all_sync(0xffffffffu, ok);
                    named_sync(2 + g, kEpiThreads); // publishes batch k's meta to the warpgroup
                    tc_fence_after();
                    const uint8_t *mb = mring + ((k >> 1) % C::MSLOTS) * NU * PL::MB;
                    for (int j = 0; j < n; j++) {
                        int d[H][N];
                        if (ok) {
#pragma unroll
                            for (int h = 0; h < H; h++)
#pragma unroll
                                for (int c0 = 0; c0 < N; c0 += 16)
                                    tmem_ld16(lane_base + (uint32_t)(buf * C::BACC + j * C::ACC + h * N + c0),
                                              *reinterpret_cast<int(*)[16]>(&d[h][c0]));
                            tmem_wait_ld();
                        } else {
#pragma unroll
                            for (int h = 0; h < H; h++)
#pragma unroll
                                for (int q = 0; q < N; q++) d[h][q] = 0;
                        }
                        const float *meta = reinterpret_cast<const float *>(mb + j * PL::MB);
#pragma unroll
                        for (int h = 0; h < H; h++)
#pragma unroll
                            for (int m = 0; m < M; m++) {
                                const int o = BITS == 4 ? 8 : 0; // int4 codes carry +8: subtract 8 * digit sum
                                const int *bsum = reinterpret_cast<const int *>(meta) + M + m * 4;
                                float v = (float)(d[h][m * 4 + 3] - o * bsum[3]);
#pragma unroll
                                for (int q = 2; q >= 0; q--)
                                    v = fmaf(v, 0.0078125f, (float)(d[h][m * 4 + q] - o * bsum[q]));
                                if (BITS == 4) {
                                    float ws = 0.f;
#pragma unroll
                                    for (int jj = 0; jj < NU; jj++)
                                        if (jj == j) ws = wsc[jj][h];
                                    acc[h][m] = fmaf(v * meta[m], ws, acc[h][m]);
                                } else {
                                    acc[h][m] = fmaf(v, meta[m], acc[h][m]);
                                }
                            }
                    }
                    tc_fence_before();
                    named_sync(2 + g, kEpiThreads);
                    if (et == 0) mbar_arrive(&accempty[buf]);
                }
                k++;
            }
            // ---- tile segment end: warpgroup 1 hands its sums to warpgroup 0 ----
            if (g == 1) {
#pragma unroll
                for (int h = 0; h < H; h++)
#pragma unroll
                    for (int m = 0; m < M; m++) red[(h * M + m) * kCols + col] = acc[h][m];
            }
            named_sync(4, 2 * kEpiThreads);
            if (g == 0) {
#pragma unroll
                for (int h = 0; h < H; h++)
#pragma unroll
                    for (int m = 0; m < M; m++) acc[h][m] += red[(h * M + m) * kCols + col];
                const long long t0 = (long long)tile * p.units, t1 = t0 + p.units;
                const int cf = split.owner(t0), cl = split.owner(t1 - 1);
                constexpr int SL = H * M * kCols; // partial entries per tile
                bool write = true;
                if (cf != cl) {
                    float *dst = p.partial + (size_t)split.slot(c, t0) * SL;
#pragma unroll
                    for (int h = 0; h < H; h++)
#pragma unroll
                        for (int m = 0; m < M; m++) dst[(h * M + m) * kCols + col] = acc[h][m];
                    named_sync(2, kEpiThreads);
                    if (et == 0) *lastflag = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1));
                    named_sync(2, kEpiThreads);
                    write = *lastflag != 0;
                    if (write) {
                        const int slot_f = split.slot(cf, t0);
#pragma unroll
                        for (int h = 0; h < H; h++)
#pragma unroll
                            for (int m = 0; m < M; m++) acc[h][m] = 0.f;
                        // contributors in CTA order, up to four loads in flight per entry
                        for (int cc = cf; cc <= cl; cc += 4) {
                            float pv[4][H][M];
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const int c2 = cc + u;
                                const int sl = c2 == cf ? slot_f : 2 * c2;
                                const float *src = p.partial + (size_t)sl * SL;
#pragma unroll
                                for (int h = 0; h < H; h++)
#pragma unroll
                                    for (int m = 0; m < M; m++)
                                        pv[u][h][m] = c2 <= cl ? __ldcg(src + (h * M + m) * kCols + col) : 0.f;
                            }
#pragma unroll
                            for (int u = 0; u < 4; u++)
#pragma unroll
                                for (int h = 0; h < H; h++)
#pragma unroll
                                    for (int m = 0; m < M; m++) acc[h][m] += pv[u][h][m];
                        }
                    }
                }
                if (write) {
                    const int base = tile * kCols + col; // byte index in the reference row
                    if (BITS == 8) {
                        if (base < p.cols) {
                            const float sc = __ldg(p.scale + base);
#pragma unroll
                            for (int m = 0; m < M; m++) p.out[(size_t)m * p.cols + base] = acc[0][m] * sc;
                        }
                    } else if (base < p.half) {
#pragma unroll
                        for (int m = 0; m < M; m++) {
                            p.out[(size_t)m * p.cols + base] = acc[0][m];
                            p.out[(size_t)m * p.cols + p.half + base] = acc[H - 1][m];
                        }
                    }
                }
            }
            named_sync(4, 2 * kEpiThreads); // red and lastflag are reused by the next segment
        }
        cp_async_wait<0>();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(C::TCOLS) : "memory");
    }
}

template <int BITS, int M>
cudaError_t launch_ig(const TqMatrixDev &mat, const float *x, float *out, const TqScratch &scr, cudaStream_t st) {
    using C = Cfg<BITS, M>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static TqDeviceOnce once;
    e = tq_device_once(once, dev, [] {
        return cudaFuncSetAttribute(igemv_kernel<BITS, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (e != cudaSuccess) return e;
    IgParams prm;
    prm.codes = mat.codes;
    prm.scale = mat.scale;
    prm.planes = scr.planes;
    prm.out = out;
    prm.partial = scr.partial;
    prm.counters = scr.counters;
    prm.status = scr.status;
    prm.rows = mat.rows;
    prm.cols = mat.cols;
    prm.half = mat.cols / 2;
    prm.units = mat.units;
    prm.tiles = mat.tiles;
    prm.items = (long long)mat.tiles * mat.units;
    const int sms = once.sms[dev];
    if (mat.tiles > TQ_MAX_TILES || sms > TQ_MAX_CTAS) return cudaErrorInvalidValue;
    if ((size_t)mat.units * (Planes<M>::BBYTES + Planes<M>::MB) > TQ_SCRATCH_PLANES_BYTES) return cudaErrorInvalidValue;
    const int ctas = (int)(prm.items < sms ? prm.items : sms);
    // Both launches may begin before their predecessor on the stream ends
    // (programmatic dependent launch); each waits on griddepcontrol.wait
    // before touching data the predecessor produces.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(mat.units);
    cfg.blockDim = dim3(64);
    e = cudaLaunchKernelEx(&cfg, planes_kernel<M>, x, mat.rows, mat.units, scr.planes);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    return cudaLaunchKernelEx(&cfg, igemv_kernel<BITS, M>, prm);
}

template <int BITS>
cudaError_t ig_dispatch(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                        cudaStream_t st) {
    switch (M) {
    case 1: return launch_ig<BITS, 1>(mat, x, out, scr, st);
    case 2: return launch_ig<BITS, 2>(mat, x, out, scr, st);
    case 3: return launch_ig<BITS, 3>(mat, x, out, scr, st);
    case 4: return launch_ig<BITS, 4>(mat, x, out, scr, st);
    case 5: return launch_ig<BITS, 5>(mat, x, out, scr, st);
    case 6: return launch_ig<BITS, 6>(mat, x, out, scr, st);
    case 7: return launch_ig<BITS, 7>(mat, x, out, scr, st);
    default: return launch_ig<BITS, 8>(mat, x, out, scr, st);
    }
}

} // namespace

// Tensor-core matvec for up to 8 activation rows (larger M in 8-row launches).
cudaError_t tq_launch_igemv(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                            cudaStream_t st) {
    if (M <= 0 || mat.cols == 0) return cudaSuccess;
    if (mat.rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
    for (int m0 = 0; m0 < M; m0 += 8) {
        const int mm = M - m0 < 8 ? M - m0 : 8;
        const float *xm = x + (size_t)m0 * mat.rows;
        float *om = out + (size_t)m0 * mat.cols;
        cudaError_t e =
            mat.bits == 8 ? ig_dispatch<8>(mat, xm, om, mm, scr, st) : ig_dispatch<4>(mat, xm, om, mm, scr, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
