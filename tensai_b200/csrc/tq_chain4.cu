// tq_chain4.cu — int4 chains of dependent single-row matvecs in ONE
// persistent launch, with every output column owned by one CTA: op j reads
// what earlier ops wrote, as the decode loops call MatVec one after another
// (_example/qwen/model.go:196-217, 232-307; quant4.go:93-119 per call).
//
// Why column owners. A matvec split over the K rows needs a reduction across
// CTAs, and in a chain of dependent ops every such reduction is a round trip
// through L2 on the critical path (partials out, arrival counter, the last
// arriver's reads, its release, the next op's acquire). Here a CTA owns whole
// 32-column blocks (16 code bytes: 16 low-nibble columns c and their 16
// high-nibble partners c + cols/2) over ALL rows, so an output value is final
// the moment its owner has it. It is published in 8-byte words carrying an
// epoch: a reader polls the words themselves and takes them when the epoch is
// the op's, so no fence, flag or counter sits between producer and consumer.
//
// What is published. The tensor cores multiply the codes by activation
// digits (below); every CTA of the next op needs the digits of every row, so
// the owner of 16 consecutive outputs makes their digits once, in its
// epilogue, and publishes them (13 words per 16 values, "digit words"); the
// readers load their mma.sync B fragments straight from those words. A value
// also read as a residual, or by a reader that cannot take digits, is
// published as a float word {value, epoch}.
//
// Layout (made once by chain4_pack_kernel from the tiled codes and scales):
// op j's column blocks are dealt to the grid's CTAs in contiguous runs (CTA c
// owns blocks [P c / C, P (c + 1) / C)), and CTA c's run is stored unit-major,
// one 1152-byte block-group per (64-row group u, block) in the order
// (u, block), so the CTA streams one contiguous HBM range per op and a
// shared-memory slot holds whole groups of all its blocks. A block-group:
//   [0, 512)     rows 0..31:  lane l = (g, t) holds 16 bytes, the mma.sync
//                m16n8k32 A fragment {A[g][4t..], A[g+8][4t..], A[g][16+4t..],
//                A[g+8][16+4t..]}: A[m][k] is the raw code byte of byte column
//                16 b + m at row k (low nibble column 16 b + m, high nibble its
//                partner); rows past K hold 0x88 (code 8 = weight 0);
//   [512, 1024)  the same for rows 32..63;
//   [1024, 1152) float4 per g: scales of low columns g, g + 8 and high
//                columns g, g + 8 of group u.
// Math (one activation row). Activations are cut into three signed byte
// digits, X = round(x 2^s) = d0 + 256 d1 + 65536 d2 (|X| <= 2^22, s from the
// largest |x| of the digit group). With the raw code bytes as A the tensor
// cores give D_raw = sum (lo + 16 hi) d and, with the bytes masked to their
// high nibbles, D_hi = 16 sum hi d: sum lo d = D_raw - D_hi and sum hi d =
// D_hi / 16, exact integers. Lane t of a quad holds D columns 2t, 2t + 1 and
// adds (D_2t + 256 D_2t+1) K_t + O_t; with the code offset 8 folded into O
// (-8 sum(X) 2^-s), then the 64-row group fold scale * sum, as
// quant4_simd.go:46-50 (fma(tmp, scale, out) per group).
//   * digit words (16-row groups): in each 32-row MMA the first 16 rows'
//     digits are B columns 0..2 and the second 16 rows' columns 4..6, so lane
//     t = 0, 1 folds the first group (K_0 = 2^-s, K_1 = 2^(16-s), O_1) and
//     t = 2, 3 the second. Words of a group: plane p (0..2), rows 4w..4w+3 at
//     word 4p + w (digit bytes in the high half), then {O, s} at word 12; the
//     low 24 bits of each word hold the epoch.
//   * own digits (the first op's external input, or a reader of float
//     words): 64-row groups made by each warp (tq_items.cuh tmv_digits), B
//     columns 0..2, lanes t = 0, 1.
// RMSNorm prologue: with digit words, the writer makes the digits of x * w
// (w the reader's norm weight) and the reader scales its sums by inv =
// 1 / sqrt(sum(x^2) / n + eps) (model.go:182-193; sum(x^2) added in float64
// from the writer's per-CTA sums); with own digits x is normalised first.
//
// Ordering. A value an op reads from an earlier op is always read from that
// op's words (never from the plain output), so it is the value of this
// launch. An op whose input is the previous op's whole output cannot store
// before every CTA has finished the previous op; any other op first waits
// until every CTA has counted the previous op done. Together with the
// build-time alias rules the chain computes what n consecutive calls compute.
//
// Epochs: a launch of a chain of n ops uses epochs seq * n + j + 1 (op j),
// seq counted on the device by the last CTA to leave; words of an earlier
// launch never match. Every wait is bounded (tqp::kWaitNs): a timeout sets
// TQ_STATUS_TIMEOUT and the chain's abort word, which ends every other CTA's
// waits; the last CTA to leave re-arms the counters.
#include <cstring>
#include <vector>

#include "tq_internal.h"
#include "tq_items.cuh"

namespace {

using namespace tqi;

constexpr int QW = 8;                     // consumer warps
constexpr int kQThreads = (QW + 1) * 32;  // + the producer warp
constexpr int kBlkB = 1152;               // one 32-column block of one 64-row group
constexpr int kSlotBlks = 16;             // block-groups per ring slot
constexpr int kSlotB = kSlotBlks * kBlkB; // 18432: one bulk copy
constexpr int kNP = TQ_CHAIN4_MAX_BLOCKS; // blocks per CTA and op
constexpr int kDgW = 13;                  // digit words per 16 values
constexpr int kQSmemCap = 226 * 1024;
constexpr int kRedB = QW * kNP * 32 * 4;       // warp sums per block column
constexpr int kPlB = QW * 2 * 256;             // per warp: two digit-plane buffers
constexpr int kXD = 4;                         // digit-word batches in flight per warp
constexpr int kXB = 4 * 4 * kDgW * 8;          // words of a batch of 4 groups (1664 bytes)
constexpr int kXrB = QW * kXD * kXB;           // per warp: a ring of kXD batches
constexpr int kQR = (kQSmemCap - kRedB - kPlB - kXrB - 1024) / kSlotB;
constexpr int kRedOff = kQR * kSlotB;
constexpr int kPlOff = kRedOff + kRedB;
constexpr int kXrOff = kPlOff + kPlB;
constexpr int kBarOff = kXrOff + kXrB; // full[kQR], empty[kQR]
constexpr int kMiscOff = kBarOff + 2 * kQR * 8;
constexpr int kQSmem = kMiscOff + 128;
static_assert(kQR >= 6, "ring too shallow");
static_assert(kQSmem <= kQSmemCap, "shared memory budget");
static_assert(kNP * 32 == QW * 32, "one epilogue entry per consumer thread");

struct Q4Op {
    const uint8_t *w;              // this op's block-groups (layout above)
    const float *x;                // external input (xsrc < 0)
    const unsigned long long *xw;  // float words of op xsrc (own digits)
    const unsigned long long *xd;  // digit words of op xsrc (digit path)
    float *out;
    unsigned long long *ow;        // this op's float words, or null
    unsigned long long *od;        // this op's digit words, or null
    const float *dw;               // weights the digit words are made of x * dw with, or null
    const float *resid;            // external residual (rsrc < 0)
    const unsigned long long *rw;  // words of op rsrc
    const float *norm_w;           // RMSNorm prologue weights, or null
    const unsigned long long *nss; // sums-of-squares words of op xsrc: [ctas][2]
    unsigned long long *ss_out;    // this op's sums-of-squares words, or null
    double eps;
    int rows, units, blocks, half; // K, 64-row groups, 32-column blocks, cols / 2
    int epi, xsrc, rsrc, digit_in; // digit_in: read op xsrc's digit words
    int wait_prev;                 // wait for every CTA to finish op j - 1 before storing
    int count_done;                // count this op done (op j + 1 waits for it)
};

struct Q4Params {
    const Q4Op *ops;
    int nops;
    unsigned *done;   // [nops] CTAs that finished op j (ops with count_done)
    unsigned *ctl;    // [0] CTAs that left, [1] abort word, [2] launch sequence
    unsigned *status;
};

__device__ __forceinline__ unsigned ld_relaxed(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ld_word2(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void st_u64(unsigned long long *p, unsigned long long w) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_word(unsigned long long *p, float v, unsigned e) {
    st_u64(p, ((unsigned long long)e << 32) | __float_as_uint(v));
}
__device__ __forceinline__ bool word_is(unsigned long long w, unsigned e) { return (unsigned)(w >> 32) == e; }
__device__ __forceinline__ float word_val(unsigned long long w) { return __uint_as_float((unsigned)w); }
// digit words: the epoch in the low 24 bits
__device__ __forceinline__ bool dword_is(unsigned long long w, unsigned e) { return (((unsigned)w ^ e) & 0xFFFFFFu) == 0; }

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-groups per ring slot's units, and units per batch of the digit path:
// a slot holds whole batches.
__device__ __forceinline__ int op_batch(int nb) { return nb <= 4 ? 4 : 2; }
__device__ __forceinline__ int op_ub(int nb) {
    const int ub = op_batch(nb);
    return ub * (kSlotBlks / (ub * nb));
}

// Called by a waiter that gave up (timed_out) or saw the chain's abort word.
__device__ __noinline__ void chain4_abort(const Q4Params &p, volatile int *abort, bool timed_out) {
    if (timed_out) {
        atomicOr(p.status, TQ_STATUS_TIMEOUT);
        st_relaxed(p.ctl + 1, 1u);
    }
    *abort = 1;
}

// One thread: bounded wait for a float word of epoch e; returns its value.
__device__ __noinline__ float wait_word(const Q4Params &p, const unsigned long long *w, unsigned e, volatile int *abort) {
    unsigned long long v = ld_word(w);
    if (word_is(v, e)) return word_val(v);
    const unsigned long long t0 = global_ns();
    for (unsigned it = 1;; it++) {
        __nanosleep(64);
        v = ld_word(w);
        if (word_is(v, e) || *abort) break;
        if ((it & 63) == 0) {
            if (ld_relaxed(p.ctl + 1)) { chain4_abort(p, abort, false); break; }
            if (global_ns() - t0 > kWaitNs) { chain4_abort(p, abort, true); break; }
        }
    }
    return word_val(v);
}

// One thread: bounded wait until *cnt >= target, then acquire.
__device__ void wait_count(const Q4Params &p, const unsigned *cnt, unsigned target, volatile int *abort) {
    if (ld_relaxed(cnt) < target) {
        const unsigned long long t0 = global_ns();
        while (ld_relaxed(cnt) < target) {
            if (*abort || ld_relaxed(p.ctl + 1)) { chain4_abort(p, abort, false); return; }
            if (global_ns() - t0 > kWaitNs) { chain4_abort(p, abort, true); return; }
            __nanosleep(128);
        }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// A warp's bounded poll step: true when the warp should stop waiting.
__device__ __forceinline__ bool poll_stop(const Q4Params &p, volatile int *abort, unsigned it,
                                          unsigned long long t0, int lane) {
    int stop = 0;
    if (lane == 0) {
        if (*abort) stop = 1;
        else if ((it & 63) == 0) {
            if (ld_relaxed(p.ctl + 1)) { chain4_abort(p, abort, false); stop = 1; }
            else if (global_ns() - t0 > kWaitNs) { chain4_abort(p, abort, true); stop = 1; }
        }
    }
    return __shfl_sync(0xffffffffu, stop, 0) != 0;
}

__device__ __forceinline__ int blk_start(int blocks, int c, int ctas) { return (int)((long long)blocks * c / ctas); }

// Bounded wait until ring slot k is full (the producer issued it, its copy landed).
__device__ __forceinline__ bool slot_ready(const Q4Params &p, uint64_t *full, volatile int *issued, int k,
                                           volatile int *abort) {
    if (*issued <= k) {
        const unsigned long long t0 = global_ns();
        while (*issued <= k && !*abort)
            if (global_ns() - t0 > kWaitNs) chain4_abort(p, abort, true);
    }
    return wait_bar(&full[k % kQR], (k / kQR) & 1, abort, p.status);
}

// One block-group into the lane's sums acc = {low g, low g + 8, high g, high
// g + 8}: b = B fragments of the two 32-row MMAs, (K, O) their lane folds.
__device__ __forceinline__ void block_group(const uint8_t *blk, int lane, const uint32_t (&b)[4], float K0, float O0,
                                            float K1, float O1, float (&acc)[4]) {
    constexpr uint32_t HI = 0xF0F0F0F0u;
    const uint4 a0 = *reinterpret_cast<const uint4 *>(blk + 16 * lane);
    const uint4 a1 = *reinterpret_cast<const uint4 *>(blk + 512 + 16 * lane);
    const float4 sc = *reinterpret_cast<const float4 *>(blk + 1024 + 16 * (lane >> 2));
    int r0[4] = {0, 0, 0, 0}, h0[4] = {0, 0, 0, 0}, r1[4] = {0, 0, 0, 0}, h1[4] = {0, 0, 0, 0};
    mma_u8s8(r0, a0.x, a0.y, a0.z, a0.w, b[0], b[1]);
    mma_u8s8(h0, a0.x & HI, a0.y & HI, a0.z & HI, a0.w & HI, b[0], b[1]);
    mma_u8s8(r1, a1.x, a1.y, a1.z, a1.w, b[2], b[3]);
    mma_u8s8(h1, a1.x & HI, a1.y & HI, a1.z & HI, a1.w & HI, b[2], b[3]);
    // low nibbles: D_raw - D_hi; high nibbles: D_hi / 16 (exact: a multiple of 16)
    const float l0 = fmaf((float)((r0[0] - h0[0]) + ((r0[1] - h0[1]) << 8)), K0,
                          fmaf((float)((r1[0] - h1[0]) + ((r1[1] - h1[1]) << 8)), K1, O0 + O1));
    const float l8 = fmaf((float)((r0[2] - h0[2]) + ((r0[3] - h0[3]) << 8)), K0,
                          fmaf((float)((r1[2] - h1[2]) + ((r1[3] - h1[3]) << 8)), K1, O0 + O1));
    const float u0 = fmaf((float)((h0[0] + (h0[1] << 8)) >> 4), K0, fmaf((float)((h1[0] + (h1[1] << 8)) >> 4), K1, O0 + O1));
    const float u8 = fmaf((float)((h0[2] + (h0[3] << 8)) >> 4), K0, fmaf((float)((h1[2] + (h1[3] << 8)) >> 4), K1, O0 + O1));
    acc[0] = fmaf(l0, sc.x, acc[0]);
    acc[1] = fmaf(l8, sc.y, acc[1]);
    acc[2] = fmaf(u0, sc.z, acc[2]);
    acc[3] = fmaf(u8, sc.w, acc[3]);
}

// UBT block-groups of one block (consecutive groups, stride apart in the
// slot) into the lane's sums, two groups at a time: both groups' A fragments
// loaded, their 8 MMAs issued, then the folds. Groups past the slot's last
// (n <= k < UBT) are skipped.
template <int UBT>
__device__ __forceinline__ void block_groups(const uint8_t *blk, size_t stride, int n, int lane,
                                             const uint32_t (&b)[UBT][4], const float (&K)[UBT][2],
                                             const float (&O)[UBT][2], float (&acc)[4]) {
    constexpr uint32_t HI = 0xF0F0F0F0u;
#pragma unroll
    for (int k0 = 0; k0 < UBT; k0 += 2) {
        if (k0 >= n) break;
        uint4 a[2][2];
        float4 sc[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint8_t *bk = blk + (k0 + k < n ? k0 + k : k0) * stride;
            a[k][0] = *reinterpret_cast<const uint4 *>(bk + 16 * lane);
            a[k][1] = *reinterpret_cast<const uint4 *>(bk + 512 + 16 * lane);
            sc[k] = *reinterpret_cast<const float4 *>(bk + 1024 + 16 * (lane >> 2));
        }
        int d[2][4][4];
#pragma unroll
        for (int k = 0; k < 2; k++) {
#pragma unroll
            for (int m = 0; m < 4; m++) d[k][m][0] = d[k][m][1] = d[k][m][2] = d[k][m][3] = 0;
            const uint32_t *bb = b[k0 + k];
            mma_u8s8(d[k][0], a[k][0].x, a[k][0].y, a[k][0].z, a[k][0].w, bb[0], bb[1]);
            mma_u8s8(d[k][1], a[k][0].x & HI, a[k][0].y & HI, a[k][0].z & HI, a[k][0].w & HI, bb[0], bb[1]);
            mma_u8s8(d[k][2], a[k][1].x, a[k][1].y, a[k][1].z, a[k][1].w, bb[2], bb[3]);
            mma_u8s8(d[k][3], a[k][1].x & HI, a[k][1].y & HI, a[k][1].z & HI, a[k][1].w & HI, bb[2], bb[3]);
        }
#pragma unroll
        for (int k = 0; k < 2; k++) {
            if (k0 + k >= n) break;
            const int(&r0)[4] = d[k][0];
            const int(&h0)[4] = d[k][1];
            const int(&r1)[4] = d[k][2];
            const int(&h1)[4] = d[k][3];
            const float K0 = K[k0 + k][0], K1 = K[k0 + k][1], o = O[k0 + k][0] + O[k0 + k][1];
            const float l0 = fmaf((float)((r0[0] - h0[0]) + ((r0[1] - h0[1]) << 8)), K0,
                                  fmaf((float)((r1[0] - h1[0]) + ((r1[1] - h1[1]) << 8)), K1, o));
            const float l8 = fmaf((float)((r0[2] - h0[2]) + ((r0[3] - h0[3]) << 8)), K0,
                                  fmaf((float)((r1[2] - h1[2]) + ((r1[3] - h1[3]) << 8)), K1, o));
            const float u0 = fmaf((float)((h0[0] + (h0[1] << 8)) >> 4), K0, fmaf((float)((h1[0] + (h1[1] << 8)) >> 4), K1, o));
            const float u8 = fmaf((float)((h0[2] + (h0[3] << 8)) >> 4), K0, fmaf((float)((h1[2] + (h1[3] << 8)) >> 4), K1, o));
            acc[0] = fmaf(l0, sc[k].x, acc[0]);
            acc[1] = fmaf(l8, sc[k].y, acc[1]);
            acc[2] = fmaf(u0, sc[k].z, acc[2]);
            acc[3] = fmaf(u8, sc[k].w, acc[3]);
        }
    }
}

// ---- own digits: activations fetched per 64-row group ----

// Activations of group u, lane l: rows 64u + 2l and + 1 (raw: floats or words).
__device__ __forceinline__ void x_fetch(const Q4Op &op, int u, int lane, unsigned long long &a, unsigned long long &b) {
    const int r = u * kRows + 2 * lane;
    a = b = 0;
    if (op.xsrc < 0) {
        if (r + 1 < op.rows) {
            const float2 v = __ldcg(reinterpret_cast<const float2 *>(op.x + r));
            a = __float_as_uint(v.x);
            b = __float_as_uint(v.y);
        } else if (r < op.rows) {
            a = __float_as_uint(__ldcg(op.x + r));
        }
    } else if (r < op.rows) {
        ld_word2(op.xw + r, a, b); // the word buffer holds an even number of words
    }
}

// The fetched activations as floats, once every word of the warp carries epoch
// e (bounded polling); rows past K are zero.
__device__ __forceinline__ float2 x_resolve(const Q4Op &op, const Q4Params &p, int u, int lane, unsigned long long a,
                                            unsigned long long b, unsigned e, volatile int *abort) {
    const int r = u * kRows + 2 * lane;
    if (op.xsrc < 0) return make_float2(__uint_as_float((unsigned)a), __uint_as_float((unsigned)b));
    bool ok0 = r >= op.rows || word_is(a, e), ok1 = r + 1 >= op.rows || word_is(b, e);
    if (!__all_sync(0xffffffffu, ok0 && ok1)) {
        const unsigned long long t0 = global_ns();
        for (unsigned it = 1;; it++) {
            __nanosleep(32);
            if (!ok0) { a = ld_word(op.xw + r); ok0 = word_is(a, e); }
            if (!ok1) { b = ld_word(op.xw + r + 1); ok1 = word_is(b, e); }
            if (__all_sync(0xffffffffu, ok0 && ok1)) break;
            if (poll_stop(p, abort, it, t0, lane)) break;
        }
    }
    return make_float2(r < op.rows ? word_val(a) : 0.f, r + 1 < op.rows ? word_val(b) : 0.f);
}

// B fragments of lane (g, t) from a 64-row group's digit planes ([3][64]
// bytes): plane g at rows 4t.., 16 + 4t.. (first 32 rows) and 32 + 4t.., 48 + 4t...
__device__ __forceinline__ void bfrag4(const uint8_t *pl, int lane, uint32_t (&b)[4]) {
    const int g = lane >> 2, t = lane & 3;
    if (g < 3) {
        const uint8_t *q = pl + g * 64 + 4 * t;
#pragma unroll
        for (int i = 0; i < 4; i++) b[i] = *reinterpret_cast<const uint32_t *>(q + 16 * i);
    } else {
        b[0] = b[1] = b[2] = b[3] = 0u;
    }
}

// This warp's groups u = cw, cw + 8, ... with digits it makes itself:
// activations fetched two groups ahead, digits one group ahead.
__device__ __forceinline__ void own_digit_loop(const Q4Op &op, const Q4Params &p, uint8_t *smem, uint64_t *full,
                                               uint64_t *empty, volatile int *issued, volatile int *abort, int cw,
                                               int lane, int nb, int slot_base, unsigned ex, double inv,
                                               float (&acc)[kNP][4]) {
    const int U = op.units, UB = op_ub(nb);
    uint8_t *pl0 = smem + kPlOff + cw * 512;
    auto digits = [&](unsigned long long a, unsigned long long b, int u, uint8_t *pl, float &Kf, float &Of) {
        float2 xv = x_resolve(op, p, u, lane, a, b, ex, abort);
        if (op.norm_w) {
            const int r = u * kRows + 2 * lane;
            if (r < op.rows) xv.x = __fmul_rn((float)__dmul_rn((double)xv.x, inv), __ldg(op.norm_w + r));
            if (r + 1 < op.rows) xv.y = __fmul_rn((float)__dmul_rn((double)xv.y, inv), __ldg(op.norm_w + r + 1));
        }
        float K0, K1, O1;
        tmv_digits(xv, pl, lane, K0, K1, O1);
        tmv_fold(lane, K0, K1, O1, Kf, Of);
    };
    unsigned long long a1 = 0, b1 = 0, a2 = 0, b2 = 0, a0, bb0;
    x_fetch(op, cw, lane, a0, bb0);
    if (cw + QW < U) x_fetch(op, cw + QW, lane, a1, b1);
    if (cw + 2 * QW < U) x_fetch(op, cw + 2 * QW, lane, a2, b2);
    float Kc, Oc;
    digits(a0, bb0, cw, pl0, Kc, Oc);
    __syncwarp();
    uint32_t bc[4];
    bfrag4(pl0, lane, bc);
    int i = 0;
    for (int u = cw; u < U; u += QW, i++) {
        const int un = u + QW;
        uint8_t *pln = pl0 + ((i + 1) & 1) * 256;
        float Kn = 0.f, On = 0.f;
        if (un < U) digits(a1, b1, un, pln, Kn, On);
        a1 = a2;
        b1 = b2;
        if (un + 2 * QW < U) x_fetch(op, un + 2 * QW, lane, a2, b2);
        const int k = slot_base + u / UB;
        if (slot_ready(p, full, issued, k, abort)) {
            const uint8_t *blk = smem + (size_t)(k % kQR) * kSlotB + (size_t)(u % UB) * nb * kBlkB;
#pragma unroll
            for (int q = 0; q < kNP; q++)
                if (q < nb) block_group(blk + q * kBlkB, lane, bc, Kc, 0.f, Kc, Oc, acc[q]);
        }
        __syncwarp();
        if (lane == 0) {
            const int first = u - u % UB, nu = U - first < UB ? U - first : UB;
            mbar_arrive_cnt(&empty[k % kQR], u == first ? 1 + (kSlotBlks - nu) : 1);
        }
        if (un < U) bfrag4(pln, lane, bc);
        __syncwarp(); // the planes just read are rewritten two groups on
        Kc = Kn;
        Oc = On;
    }
}

// ---- digit words: B fragments read from the writer's words ----
//
// Each warp copies the words of its next kXD batches into its own shared
// ring (cp.async through L2), so the L2 latency of a batch's words is hidden
// behind the batches before it; words of an earlier launch are copied again
// (bounded polling) until they carry this launch's epoch.

// Copies the words of groups 4 u0 .. 4 (u0 + UBT) - 1 (those below ng) to xs;
// one cp.async group per lane.
template <int UBT>
__device__ __forceinline__ void dg_issue(const Q4Op &op, int u0, int ng, uint8_t *xs, int lane) {
    constexpr int NW = UBT * 4 * kDgW; // words of a batch (an even count)
    const int g0 = 4 * u0;
    int nw = (ng - g0) * kDgW;
    nw = nw < 0 ? 0 : nw > NW ? NW : nw;
    const uint8_t *src = reinterpret_cast<const uint8_t *>(op.xd + (size_t)g0 * kDgW); // 16-byte aligned: 416 u0
    for (int c = lane; c < NW / 2; c += 32) {
        const int bytes = 2 * c + 2 <= nw ? 16 : 2 * c < nw ? 8 : 0;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(xs + 16 * c)),
                     "l"(src + (bytes ? 16 * c : 0)), "r"(bytes)
                     : "memory");
    }
}

// Lane (g, t)'s words of unit k of a batch in xs: per 32-row half h its plane
// word (g = 0..2: first 16 rows' plane g; g = 4..6: second 16 rows' plane
// g - 4) and the {O, s} word of the 16-row group lane t folds; 0 past ng.
__device__ __forceinline__ void dg_words(const uint8_t *xs, int k, int u, int lane, int ng, unsigned long long (&w)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const unsigned long long *xw = reinterpret_cast<const unsigned long long *>(xs);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int rp = 4 * k + 2 * h + (g >> 2), rc = 4 * k + 2 * h + (t >> 1);
        w[h] = ((g & 3) != 3 && 4 * u - 4 * k + rp < ng) ? xw[rp * kDgW + (g & 3) * 4 + t] : 0ull;
        w[2 + h] = 4 * u - 4 * k + rc < ng ? xw[rc * kDgW + 12] : 0ull;
    }
}

__device__ __forceinline__ bool dg_ok(const unsigned long long (&w)[4], int u, int lane, int ng, unsigned e) {
    const int g = lane >> 2, t = lane & 3;
    bool ok = true;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int gp = 4 * u + 2 * h + (g >> 2), gc = 4 * u + 2 * h + (t >> 1);
        ok = ok && ((g & 3) == 3 || gp >= ng || dword_is(w[h], e)) && (gc >= ng || dword_is(w[2 + h], e));
    }
    return ok;
}

// B fragments and lane folds of one 64-row group from its words.
__device__ __forceinline__ void dg_decode(const unsigned long long (&w)[4], int u, int lane, int ng, uint32_t (&b)[4],
                                          float (&K)[2], float (&O)[2]) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t d = (uint32_t)(w[h] >> 32);
        b[2 * h] = g < 3 ? d : 0u;
        b[2 * h + 1] = (g >= 4 && g < 7) ? d : 0u;
        const int gc = 4 * u + 2 * h + (t >> 1);
        if (gc < ng) {
            const unsigned s = ((unsigned)w[2 + h] >> 24) & 0xFFu;
            const float o = __uint_as_float((unsigned)(w[2 + h] >> 32));
            K[h] = __uint_as_float((127u - s + ((t & 1) ? 16u : 0u)) << 23);
            O[h] = ((t & 1) || o != o) ? o : 0.f;
        } else {
            K[h] = 0.f;
            O[h] = 0.f;
        }
    }
}

// This warp's batches of UBT consecutive groups (batches cw, cw + 8, ...).
template <int UBT>
__device__ __forceinline__ void digit_loop(const Q4Op &op, const Q4Params &p, uint8_t *smem, uint64_t *full,
                                           uint64_t *empty, volatile int *issued, volatile int *abort, int cw,
                                           int lane, int nb, int slot_base, unsigned ex, float (&acc)[kNP][4]) {
    const int U = op.units, UB = op_ub(nb), ng = (op.rows + 15) / 16;
    const int nbat = (U + UBT - 1) / UBT;
    const int nloc = cw < nbat ? (nbat - 1 - cw) / QW + 1 : 0;
    const unsigned e24 = ex & 0xFFFFFFu;
    uint8_t *xr = smem + kXrOff + cw * kXD * kXB;
#pragma unroll
    for (int i = 0; i < kXD; i++) {
        if (i < nloc) dg_issue<UBT>(op, (cw + QW * i) * UBT, ng, xr + i * kXB, lane);
        cp_async_commit();
    }
    for (int i = 0; i < nloc; i++) {
        const int u0 = (cw + QW * i) * UBT;
        uint8_t *xs = xr + (i % kXD) * kXB;
        cp_async_wait<kXD - 1>();
        __syncwarp();
        unsigned long long w[UBT][4];
        bool ok = true;
#pragma unroll
        for (int k = 0; k < UBT; k++) {
            dg_words(xs, k, u0 + k, lane, ng, w[k]);
            ok = ok && dg_ok(w[k], u0 + k, lane, ng, e24);
        }
        if (!__all_sync(0xffffffffu, ok)) { // copied before the writers were done: again (bounded)
            const unsigned long long t0 = global_ns();
            for (unsigned it = 1;; it++) {
                __nanosleep(64);
                dg_issue<UBT>(op, u0, ng, xs, lane);
                cp_async_commit();
                cp_async_wait<0>();
                __syncwarp();
                ok = true;
#pragma unroll
                for (int k = 0; k < UBT; k++) {
                    dg_words(xs, k, u0 + k, lane, ng, w[k]);
                    ok = ok && dg_ok(w[k], u0 + k, lane, ng, e24);
                }
                if (__all_sync(0xffffffffu, ok)) break;
                if (poll_stop(p, abort, it, t0, lane)) break;
            }
        }
        uint32_t b[UBT][4];
        float K[UBT][2], O[UBT][2];
#pragma unroll
        for (int k = 0; k < UBT; k++) dg_decode(w[k], u0 + k, lane, ng, b[k], K[k], O[k]);
        __syncwarp(); // every lane has read xs before it is refilled
        if (i + kXD < nloc) dg_issue<UBT>(op, (cw + QW * (i + kXD)) * UBT, ng, xs, lane);
        cp_async_commit();
        const int k = slot_base + u0 / UB, ub = u0 % UB;
        if (slot_ready(p, full, issued, k, abort)) {
            const uint8_t *slot = smem + (size_t)(k % kQR) * kSlotB;
            const int nu = U - u0 < UBT ? U - u0 : UBT;
#pragma unroll
            for (int q = 0; q < kNP; q++)
                if (q < nb)
                    block_groups<UBT>(slot + ((size_t)ub * nb + q) * kBlkB, (size_t)nb * kBlkB, nu, lane, b, K, O, acc[q]);
        }
        __syncwarp();
        if (lane == 0) {
            const int nu = U - u0 < UBT ? U - u0 : UBT;
            const int first = u0 - ub, nus = U - first < UB ? U - first : UB;
            mbar_arrive_cnt(&empty[k % kQR], nu + (ub == 0 ? kSlotBlks - nus : 0));
        }
    }
    cp_async_wait<0>(); // no copy lands in the ring after the warp moves on
    __syncwarp();
}

__global__ void __launch_bounds__(kQThreads, 1) chain4_kernel(Q4Params p) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kBarOff);
    uint64_t *empty = full + kQR;
    volatile int *abort = reinterpret_cast<volatile int *>(smem + kMiscOff);
    // Ring slots issued so far (a running count over the ops). Warps take slots
    // out of ring order, so before the parity wait for slot k they check that k
    // was issued: k is issued only after k - R was consumed, so the barrier
    // cannot still be two phases behind.
    volatile int *issued = reinterpret_cast<volatile int *>(smem + kMiscOff + 4);
    double *inv_s = reinterpret_cast<double *>(smem + kMiscOff + 8);
    double *ssw = reinterpret_cast<double *>(smem + kMiscOff + 16); // [QW]
    float *red = reinterpret_cast<float *>(smem + kRedOff);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x, C = gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kQR; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSlotBlks);
        }
        *abort = 0;
        *issued = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer: the weights depend on nothing ----------------
        if (lane == 0) {
            pdl_trigger();
            int seq = 0;
            bool stop = false;
            for (int j = 0; j < p.nops && !stop; j++) {
                const Q4Op *op = p.ops + j;
                const int b0 = blk_start(op->blocks, c, C), nb = blk_start(op->blocks, c + 1, C) - b0;
                if (nb == 0) continue;
                const int U = op->units, UB = op_ub(nb);
                const uint8_t *src = op->w + (size_t)b0 * U * kBlkB;
                for (int u0 = 0; u0 < U; u0 += UB, seq++) {
                    const int s = seq % kQR;
                    if (seq >= kQR && !wait_bar(&empty[s], ((seq / kQR) & 1) ^ 1, abort, p.status)) {
                        stop = true;
                        break;
                    }
                    if (*abort) {
                        stop = true;
                        break;
                    }
                    const int nu = U - u0 < UB ? U - u0 : UB;
                    const uint32_t bytes = (uint32_t)(nu * nb * kBlkB);
                    mbar_arrive_expect_tx(&full[s], bytes);
                    bulk_load(smem + (size_t)s * kSlotB, src + (size_t)u0 * nb * kBlkB, bytes, &full[s]);
                    *issued = seq + 1;
                }
            }
            // no copy may still be landing when the CTA leaves (bounded wait)
            const int n = *issued;
            const unsigned long long t0 = global_ns();
            for (int k = n - kQR > 0 ? n - kQR : 0; k < n; k++)
                while (!mbar_try_wait_hint(&full[k % kQR], (k / kQR) & 1, 100000u))
                    if (global_ns() - t0 > kWaitNs) break;
        }
    } else {
        // ---------------- consumers ----------------
        const int cw = warp - 1, ct = threadIdx.x - 32;
        pdl_wait(); // inputs and outputs belong to the previous kernel until here
        const unsigned seq = ld_relaxed(p.ctl + 2);
        const unsigned ep0 = seq * (unsigned)p.nops + 1u;
        int slot_base = 0; // ring sequence number of this CTA's first slot of op j
        for (int j = 0; j < p.nops; j++) {
            const Q4Op &op = p.ops[j];
            const int U = op.units;
            const int b0 = blk_start(op.blocks, c, C), nb = blk_start(op.blocks, c + 1, C) - b0;
            const unsigned ej = ep0 + (unsigned)j;
            const unsigned ex = op.xsrc >= 0 ? ep0 + (unsigned)op.xsrc : 0u;
            // RMSNorm: every CTA adds the source op's per-CTA sums of squares in
            // CTA order (own digits: before the digits; digit words: the sums
            // are scaled at the end, so the wait overlaps the groups)
            auto norm_inv = [&]() {
                if (cw == 0) { // all of a lane's words in flight at once, then bounded polling of stale ones
                    constexpr int MC = TQ_MAX_CTAS / 32;
                    unsigned long long w[MC][2];
                    bool ok = true;
#pragma unroll
                    for (int i = 0; i < MC; i++) {
                        const int cc = lane + 32 * i;
                        w[i][0] = w[i][1] = 0;
                        if (cc < C) ld_word2(op.nss + 2 * cc, w[i][0], w[i][1]);
                    }
#pragma unroll
                    for (int i = 0; i < MC; i++) ok = ok && (lane + 32 * i >= C || (word_is(w[i][0], ex) && word_is(w[i][1], ex)));
                    if (!__all_sync(0xffffffffu, ok)) {
                        const unsigned long long t0 = global_ns();
                        for (unsigned it = 1;; it++) {
                            __nanosleep(32);
                            ok = true;
#pragma unroll
                            for (int i = 0; i < MC; i++) {
                                const int cc = lane + 32 * i;
                                if (cc < C && !(word_is(w[i][0], ex) && word_is(w[i][1], ex))) ld_word2(op.nss + 2 * cc, w[i][0], w[i][1]);
                                ok = ok && (cc >= C || (word_is(w[i][0], ex) && word_is(w[i][1], ex)));
                            }
                            if (__all_sync(0xffffffffu, ok)) break;
                            if (poll_stop(p, abort, it, t0, lane)) break;
                        }
                    }
                    double s = 0.0;
#pragma unroll
                    for (int i = 0; i < MC; i++)
                        if (lane + 32 * i < C) s = __dadd_rn(s, __hiloint2double((int)(unsigned)w[i][0], (int)(unsigned)w[i][1]));
                    s = warp_sum_d(s);
                    if (lane == 0) *inv_s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s, (double)op.rows), op.eps)));
                }
            };
            double inv = 1.0;
            if (op.norm_w && !op.digit_in) {
                norm_inv();
                named_sync(1, QW * 32);
                inv = *inv_s;
            }
            float acc[kNP][4];
#pragma unroll
            for (int i = 0; i < kNP; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
            if (nb > 0) {
                if (!op.digit_in) {
                    if (cw < U) own_digit_loop(op, p, smem, full, empty, issued, abort, cw, lane, nb, slot_base, ex, inv, acc);
                } else if (op_batch(nb) == 4) {
                    digit_loop<4>(op, p, smem, full, empty, issued, abort, cw, lane, nb, slot_base, ex, acc);
                } else {
                    digit_loop<2>(op, p, smem, full, empty, issued, abort, cw, lane, nb, slot_base, ex, acc);
                }
            }
            if (op.norm_w && op.digit_in) norm_inv(); // read after the barrier below
            // ---- epilogue: warp sums in warp order, then one thread per column ----
#pragma unroll
            for (int q = 0; q < kNP; q++) {
                if (q < nb) {
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        float v = acc[q][h];
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        v += __shfl_xor_sync(0xffffffffu, v, 2);
                        if ((lane & 3) == 0) red[(cw * kNP + q) * 32 + (h >> 1) * 16 + (h & 1) * 8 + (lane >> 2)] = v;
                    }
                }
            }
            named_sync(1, QW * 32);
            if (op.norm_w && op.digit_in) inv = *inv_s;
            if (op.wait_prev) {
                if (ct == 0) wait_count(p, p.done + j - 1, (unsigned)C, abort);
                named_sync(1, QW * 32);
            }
            double ss = 0.0;
            if (ct < nb * 32) { // warp q: block b0 + q, lanes 0..15 low columns, 16..31 high
                const int q = ct >> 5, e = ct & 31;
                const int bc = (b0 + q) * 16 + (e & 15); // code byte column
                auto wsum = [&](int en) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < QW; w++) v += red[(w * kNP + q) * 32 + en];
                    if (op.norm_w && op.digit_in) v = (float)__dmul_rn((double)v, inv);
                    return v;
                };
                const bool sw = op.epi == TQ_EPI_SWIGLU;
                const bool has = bc < op.half && (!sw || e < 16);
                const int col = (sw || e < 16) ? bc : op.half + bc;
                float v = 0.f;
                if (has) {
                    if (sw) {
                        v = swiglu(wsum(e), wsum(e + 16));
                    } else {
                        v = wsum(e);
                        if (op.epi == TQ_EPI_RESID)
                            v = __fadd_rn(op.rsrc >= 0 ? wait_word(p, op.rw + col, ep0 + (unsigned)op.rsrc, abort)
                                                       : __ldcg(op.resid + col),
                                          v);
                    }
                    op.out[col] = v;
                    if (op.ow) st_word(op.ow + col, v, ej);
                    ss = __dmul_rn((double)v, (double)v);
                }
                if (op.od) { // the digits of 16 consecutive outputs (a half warp), once for every reader
                    const float dv = has ? (op.dw ? __fmul_rn(v, __ldg(op.dw + col)) : v) : 0.f;
                    uint32_t amax = __float_as_uint(dv) & 0x7FFFFFFFu;
#pragma unroll
                    for (int o = 1; o < 16; o <<= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                    int sh = 148 - (int)(amax >> 23); // |X| <= 2^22
                    sh = sh > 126 ? 126 : sh;
                    const float up = __uint_as_float((uint32_t)(127 + sh) << 23);
                    const float dn = __uint_as_float((uint32_t)(127 - sh) << 23);
                    const int X = __float2int_rn(dv * up);
                    int sx = X;
#pragma unroll
                    for (int o = 1; o < 16; o <<= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
                    const uint32_t dg = (uint32_t)(X + 0x808080) ^ 0x808080u;
                    const int i = e & 15;
                    const bool live = (b0 + q) * 16 < op.half && (!sw || e < 16);
                    const int grp = (sw || e < 16) ? b0 + q : op.half / 16 + b0 + q;
                    unsigned long long *gw = op.od + (size_t)grp * kDgW;
                    const unsigned e24 = ej & 0xFFFFFFu;
#pragma unroll
                    for (int pl = 0; pl < 3; pl++) {
                        const uint32_t by = (dg >> (8 * pl)) & 0xFFu;
                        const uint32_t wd = by | (__shfl_down_sync(0xffffffffu, by, 1, 16) << 8) |
                                            (__shfl_down_sync(0xffffffffu, by, 2, 16) << 16) |
                                            (__shfl_down_sync(0xffffffffu, by, 3, 16) << 24);
                        if (live && (i & 3) == 0) st_u64(gw + pl * 4 + (i >> 2), ((unsigned long long)wd << 32) | e24);
                    }
                    if (live && i == 0) {
                        const float o = amax >= 0x7F800000u ? __uint_as_float(0x7FC00000u) : -8.f * (float)sx * dn;
                        st_u64(gw + 12, ((unsigned long long)__float_as_uint(o) << 32) | ((unsigned)sh << 24) | e24);
                    }
                }
            }
            if (op.ss_out) { // this CTA's sum of squares of what it wrote, warp order
                ss = warp_sum_d(ss);
                if (lane == 0) ssw[cw] = ss;
            }
            named_sync(1, QW * 32);
            if (ct == 0) {
                if (op.ss_out) {
                    double t = 0.0;
                    for (int w = 0; w < QW; w++) t = __dadd_rn(t, ssw[w]);
                    st_word(op.ss_out + 2 * c, __uint_as_float((unsigned)__double2hiint(t)), ej);
                    st_word(op.ss_out + 2 * c + 1, __uint_as_float((unsigned)__double2loint(t)), ej);
                }
                if (op.count_done) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.done + j) : "memory");
            }
            if (nb > 0) {
                const int UB = op_ub(nb);
                slot_base += (U + UB - 1) / UB;
            }
        }
    }
    __syncthreads();
    // ---- exit: the last CTA to leave re-arms the counters and moves the epoch on ----
    if (threadIdx.x == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.ctl) : "memory");
        if (prev == gridDim.x - 1) {
            for (int j = 0; j < p.nops; j++) st_relaxed(p.done + j, 0u);
            st_relaxed(p.ctl + 1, 0u);
            st_relaxed(p.ctl + 2, ld_relaxed(p.ctl + 2) + 1u);
            st_relaxed(p.ctl, 0u);
        }
    }
}

// Packs op j's blocks for a grid of `ctas` CTAs (layout at the top of the
// file): one thread per (block, group, lane).
__global__ void chain4_pack_kernel(const uint8_t *codes, const float *scale, int rows, int units, int half, int blocks,
                                   int ctas, uint8_t *dst) {
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (long long)blocks * units * 32) return;
    const int lane = (int)(gid & 31);
    const long long bu = gid >> 5;
    const int u = (int)(bu % units), b = (int)(bu / units);
    int cc = (int)(((long long)(b + 1) * ctas - 1) / blocks);
    while (cc > 0 && blk_start(blocks, cc, ctas) > b) cc--;
    while (cc + 1 < ctas && blk_start(blocks, cc + 1, ctas) <= b) cc++;
    const int b0 = blk_start(blocks, cc, ctas), nb = blk_start(blocks, cc + 1, ctas) - b0;
    uint8_t *blk = dst + ((size_t)b0 * units + (size_t)u * nb + (b - b0)) * kBlkB;
    const int g = lane >> 2, t = lane & 3;
    // padding (rows past K, columns past the matrix) holds code 8: weight 0
    auto code = [&](int col, int r) -> uint32_t {
        return (col < half && r < rows) ? (uint32_t)codes[tq_code_offset(units, r, col)] : 0x88u;
    };
#pragma unroll
    for (int ks = 0; ks < 2; ks++) {
        uint32_t wv[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int col = b * 16 + g + (q & 1) * 8;
            const int r = u * kRows + ks * 32 + (q >> 1) * 16 + 4 * t;
            wv[q] = code(col, r) | code(col, r + 1) << 8 | code(col, r + 2) << 16 | code(col, r + 3) << 24;
        }
        *reinterpret_cast<uint4 *>(blk + ks * 512 + lane * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    if (lane < 8) {
        const int col = b * 16 + lane;
        auto sc = [&](int hi, int cl) { return cl < half ? scale[tq_scale4_offset(units, u, hi, cl)] : 0.f; };
        *reinterpret_cast<float4 *>(blk + 1024 + lane * 16) = make_float4(sc(0, col), sc(0, col + 8), sc(1, col), sc(1, col + 8));
    }
}

} // namespace

// ---- host side ------------------------------------------------------------------

struct TqChain4 {
    int device = 0, nops = 0, ctas = 0;
    void *mem = nullptr; // descriptors, counters, words
    std::vector<void *> packs;
    Q4Op *ops = nullptr;
    unsigned *done = nullptr, *ctl = nullptr;
};

static bool overlaps(const void *a, size_t na, const void *b, size_t nb) {
    const uintptr_t x = (uintptr_t)a, y = (uintptr_t)b;
    return x < y + nb && y < x + na;
}

void tq_chain4_destroy(TqChain4 *ch) {
    if (!ch) return;
    for (void *q : ch->packs)
        if (q) cudaFree(q);
    if (ch->mem) cudaFree(ch->mem);
    delete ch;
}

cudaError_t tq_chain4_build(const TqChainSpec *spec, int n, int sms, TqChain4 **out, int *why, int *bad_op) {
    *out = nullptr;
    auto fail = [&](int j, int w) {
        *why = w;
        *bad_op = j;
        return cudaErrorInvalidValue;
    };
    // output count of op k, and the latest op before j whose output is exactly p
    auto nout = [&](int k) { return spec[k].epi == TQ_EPI_SWIGLU ? spec[k].m->cols / 2 : spec[k].m->cols; };
    std::vector<int> xsrc(n, -1), rsrc(n, -1);
    for (int j = 0; j < n; j++) {
        const TqChainSpec &s = spec[j];
        const TqMatrixDev &m = *s.m;
        if (m.rows < 1 || m.cols < 1) return fail(j, TQ_CHAIN_EMPTY);
        if (!s.x || !s.out || ((uintptr_t)s.x & 15) || ((uintptr_t)s.out & 3)) return fail(j, TQ_CHAIN_X_ALIGN);
        if (s.epi != TQ_EPI_NONE && s.epi != TQ_EPI_SWIGLU && s.epi != TQ_EPI_RESID) return fail(j, TQ_CHAIN_EPI);
        if (s.epi == TQ_EPI_SWIGLU && m.cols % 2) return fail(j, TQ_CHAIN_EPI);
        if (s.epi == TQ_EPI_RESID && !s.resid) return fail(j, TQ_CHAIN_EPI);
        const int half = (m.cols + 1) / 2, blocks = (half + 15) / 16;
        if (blocks > (long long)sms * TQ_CHAIN4_MAX_BLOCKS) return fail(j, TQ_CHAIN_TOO_WIDE);
        const size_t xb = sizeof(float) * (size_t)m.rows, ob = sizeof(float) * (size_t)nout(j);
        const size_t rb = sizeof(float) * (size_t)m.cols;
        for (int k = j - 1; k >= 0; k--) { // the latest earlier writer of x / resid
            const size_t kb = sizeof(float) * (size_t)nout(k);
            if (xsrc[j] < 0 && overlaps(s.x, xb, spec[k].out, kb)) {
                if (s.x != spec[k].out || m.rows > nout(k)) return fail(j, TQ_CHAIN_ALIAS);
                xsrc[j] = k;
            }
            if (s.epi == TQ_EPI_RESID && rsrc[j] < 0 && overlaps(s.resid, rb, spec[k].out, kb)) {
                if (s.resid != spec[k].out || m.cols > nout(k)) return fail(j, TQ_CHAIN_ALIAS);
                rsrc[j] = k;
            }
        }
        // an op's own output may only coincide with its residual (in place)
        if (overlaps(s.out, ob, s.x, xb) && xsrc[j] < 0) return fail(j, TQ_CHAIN_ALIAS);
        if (s.epi == TQ_EPI_RESID && overlaps(s.out, ob, s.resid, rb) && s.out != s.resid) return fail(j, TQ_CHAIN_ALIAS);
        if (s.norm_w) {
            const int f = s.norm_from;
            if (f < 0 || f >= j || spec[f].epi != TQ_EPI_RESID || xsrc[j] != f || spec[f].m->cols != m.rows)
                return fail(j, TQ_CHAIN_NORM);
        }
    }
    // Who publishes what: digit words for readers of a writer whose 16-value
    // groups are whole (SwiGLU outputs, or cols / 2 a multiple of 16), all with
    // the same norm weight (the first reader's); float words for the others
    // and for residual reads; sums of squares for norms.
    std::vector<char> fw(n, 0), dg(n, 0), ssk(n, 0), din(n, 0);
    std::vector<const float *> dwt(n, nullptr);
    for (int j = 0; j < n; j++) {
        const int k = xsrc[j];
        if (k >= 0) {
            const bool whole = spec[k].epi == TQ_EPI_SWIGLU || (spec[k].m->cols / 2) % 16 == 0;
            if (whole && (!dg[k] || dwt[k] == spec[j].norm_w)) {
                dg[k] = 1;
                dwt[k] = spec[j].norm_w;
                din[j] = 1;
            } else {
                fw[k] = 1;
            }
        }
        if (rsrc[j] >= 0) fw[rsrc[j]] = 1;
        if (spec[j].norm_w) ssk[spec[j].norm_from] = 1;
    }
    // descriptors | done[n] + ctl[4] | per op: float words (even count), digit words, sums-of-squares words
    const size_t ops_b = sizeof(Q4Op) * n;
    const size_t cnt_at = (ops_b + 255) & ~(size_t)255, cnt_b = sizeof(unsigned) * ((size_t)n + 4);
    size_t at = (cnt_at + cnt_b + 255) & ~(size_t)255;
    std::vector<size_t> w_at(n, 0), d_at(n, 0), s_at(n, 0);
    auto take = [&](size_t bytes) {
        const size_t r = at;
        at = (at + bytes + 255) & ~(size_t)255;
        return r;
    };
    for (int j = 0; j < n; j++) {
        if (fw[j]) w_at[j] = take(sizeof(unsigned long long) * (size_t)((spec[j].m->cols + 1) & ~1));
        if (dg[j]) d_at[j] = take(sizeof(unsigned long long) * kDgW * (size_t)((nout(j) + 15) / 16));
        if (ssk[j]) s_at[j] = take(sizeof(unsigned long long) * 2 * (size_t)sms);
    }
    TqChain4 *ch = new TqChain4();
    cudaError_t e = cudaGetDevice(&ch->device);
    if (e == cudaSuccess) e = tq_dev_malloc(&ch->mem, at);
    if (e != cudaSuccess) {
        tq_chain4_destroy(ch);
        return e;
    }
    uint8_t *base = static_cast<uint8_t *>(ch->mem);
    auto words = [&](size_t off) { return reinterpret_cast<unsigned long long *>(base + off); };
    ch->ops = reinterpret_cast<Q4Op *>(base);
    ch->done = reinterpret_cast<unsigned *>(base + cnt_at);
    ch->ctl = ch->done + n;
    ch->nops = n;
    ch->ctas = sms;
    ch->packs.assign(n, nullptr);
    std::vector<Q4Op> h(n);
    for (int j = 0; j < n && e == cudaSuccess; j++) {
        const TqChainSpec &s = spec[j];
        const TqMatrixDev &m = *s.m;
        Q4Op &o = h[j];
        std::memset(&o, 0, sizeof o);
        o.rows = m.rows;
        o.units = m.units;
        o.half = m.cols / 2;
        o.blocks = (o.half + 15) / 16;
        const size_t pb = (size_t)o.blocks * o.units * kBlkB;
        if ((e = tq_dev_malloc(&ch->packs[j], pb)) != cudaSuccess) break;
        const long long threads = (long long)o.blocks * o.units * 32;
        chain4_pack_kernel<<<(unsigned)((threads + 255) / 256), 256>>>(m.codes, m.scale, m.rows, m.units, o.half,
                                                                       o.blocks, sms, static_cast<uint8_t *>(ch->packs[j]));
        if ((e = cudaGetLastError()) != cudaSuccess) break;
        o.w = static_cast<const uint8_t *>(ch->packs[j]);
        o.x = s.x;
        o.xsrc = xsrc[j];
        o.digit_in = din[j];
        if (xsrc[j] >= 0) {
            if (din[j]) o.xd = words(d_at[xsrc[j]]);
            else o.xw = words(w_at[xsrc[j]]);
        }
        o.out = s.out;
        if (fw[j]) o.ow = words(w_at[j]);
        if (dg[j]) {
            o.od = words(d_at[j]);
            o.dw = dwt[j];
        }
        o.epi = s.epi;
        o.rsrc = rsrc[j];
        if (s.epi == TQ_EPI_RESID) {
            o.resid = s.resid;
            if (rsrc[j] >= 0) o.rw = words(w_at[rsrc[j]]);
        }
        if (s.norm_w) {
            o.norm_w = s.norm_w;
            o.nss = words(s_at[s.norm_from]);
        }
        if (ssk[j]) o.ss_out = words(s_at[j]);
        o.eps = s.eps;
        // an op fed by the whole output of op j - 1 cannot store before every
        // CTA has finished op j - 1; any other op waits for the count
        o.wait_prev = j > 0 && !(xsrc[j] == j - 1 && m.rows == nout(j - 1));
    }
    for (int j = 0; j + 1 < n; j++) h[j].count_done = h[j + 1].wait_prev;
    if (e == cudaSuccess) e = cudaMemcpy(ch->ops, h.data(), ops_b, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(base + cnt_at, 0, at - cnt_at); // counters, epochs 0: never an op's
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        tq_chain4_destroy(ch);
        return e;
    }
    *out = ch;
    return cudaSuccess;
}

static TqDeviceOnce g_chain4_once;

cudaError_t tq_chain4_launch(const TqChain4 *ch, unsigned *status, cudaStream_t st) {
    cudaError_t e = tq_device_once(g_chain4_once, ch->device, [] {
        return cudaFuncSetAttribute(chain4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQSmem);
    });
    if (e != cudaSuccess) return e;
    Q4Params prm;
    prm.ops = ch->ops;
    prm.nops = ch->nops;
    prm.done = ch->done;
    prm.ctl = ch->ctl;
    prm.status = status;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(ch->ctas);
    cfg.blockDim = dim3(kQThreads);
    cfg.dynamicSmemBytes = kQSmem;
    return cudaLaunchKernelEx(&cfg, chain4_kernel, prm);
}
