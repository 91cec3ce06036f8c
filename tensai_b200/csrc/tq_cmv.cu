// tq_cmv.cu — weight-only int8 / int4 matvec for M <= 2 activation rows on the
// CUDA cores, one launch per call, HBM-bound.
//
// Computes out[m][j] = sum_i x[m][i] * W[i][j], the product of qmatvecCols
// (quant_simd.go:12-48) and q4matvecCols (quant4_simd.go:17-57):
//   int8: acc_j = sum_i x_i * q_ij, out_j = acc_j * scale_j (quant.go:120);
//   int4: per 64-row group g, tmp_j = sum_{i in g} x_i * (nib_ij - 8), then
//         acc_j = fma(tmp_j, scale_gj, acc_j), the fold of quant4_simd.go:46-50.
//
// Why the CUDA cores: a tcgen05.mma of M = 128 rows costs about 170 cycles
// whatever its N, so a matvec (N = one activation row) pays 170 cycles per
// 4 KB of codes on the tensor cores, more than HBM needs to deliver them. Here
// a code costs about 2.3 instructions:
//   int4: each nibble becomes a float with one LOP3 by OR-ing it, in place,
//         under the exponent of 2^23 (the float 2^23 + 16^k n for the nibble at
//         bits 4k..4k+3, k < 5; the top three nibbles after one shift), one
//         packed f32x2 add removes 2^23 + 16^k * 8 exactly, and packed f32x2
//         FMAs accumulate 16^k (n - 8) x. The power of two 16^k is taken out
//         exactly by folding 16^-k into the group scale: fma(16^k tmp,
//         scale * 16^-k, acc) == fma(tmp, scale, acc) bit for bit.
//   int8: byte_perm puts each signed byte (xor 0x80) under the exponent of
//         2^23; a packed add removes 2^23 + 128.
//
// Schedule. One persistent CTA per SM takes an equal contiguous slice of the
// tile-major item list (8 KB items: 64 rows x 128 code bytes; stream-K,
// balanced to +-1 item). A producer warp streams the slice's items (int4:
// with their 1 KB of scales) through a ring of up to 24 slots by bulk copies,
// from kernel start: the weights do not depend on the previous kernel, so the
// ring fills while it finishes (programmatic dependent launch). Eight
// consumer warps take the slice's items round robin, warps 2i and 2i + 1 the
// two halves of one item (CUDA cores: 32-row halves; tensor cores: 128-column
// halves); lane l owns code bytes 4l..4l+3 of every row (int4: 8 columns,
// int8: 4). Activations of an item go through a per-warp ring of shared slots
// by cp.async, three items ahead.
//
// Reductions, all in a fixed order (results are bit-reproducible run to run):
//   * per tile segment (the slice's items of one column tile), each warp
//     deposits its sums in a shared buffer; the last warp to deposit adds the
//     deposits in warp order;
//   * a tile wholly inside the slice is written at once; a tile shared with
//     other CTAs goes through scratch partials and an acq_rel arrival counter,
//     and the last CTA to arrive adds all partials in CTA order. The slice's
//     first segment, when shared and not also its last, is published by a
//     fixup warp so the consumers do not wait on global memory ordering.
// Every wait is bounded (tqp::kWaitNs); a timeout sets TQ_STATUS_TIMEOUT and an
// abort flag that turns later waits into no-ops.
#include "tq_items.cuh"

namespace {

using namespace tqi;

constexpr int W = 8;                 // consumer warps
constexpr int WI = W / 2;            // item streams: warps 2i and 2i + 1 take the two 32-row halves of an item
constexpr int kThreads = (W + 2) * 32;
// Shared memory per CTA, small enough for two CTAs per SM: the next kernel on
// the stream (programmatic dependent launch) is resident while this one
// computes and reduces, and fills its ring meanwhile.
constexpr int kSmemCap = 113 * 1024; // 2 x (113 + 1 reserved) KB <= 228 KB per SM
// The tensor-core variant needs a quarter of the CUDA-core variant's issue
// slots per code, so it runs one CTA per SM instead, with a ring deep enough to
// have its whole stream-K slice in flight at once.
constexpr int kSmemCapTc = 226 * 1024;

template <int BITS, int M, bool TC = false> struct CCfg {
    static constexpr int NP = BITS == 8 ? 4 : 8;       // columns per lane
    static constexpr int E = M * NP * 32;              // sums of one tile segment
    static constexpr int SLOT = BITS == 4 ? kItem + 1024 : kItem; // codes (+ int4 scales)
    static constexpr int XD = 4;                      // per-warp activation ring (half items; TC: whole items)
    static constexpr int XROWS = TC ? kRows : kHalf;
    static constexpr int XSLOT = XD * XROWS * M * 4;  // [XD][M][XROWS] floats per warp
    static constexpr int PLANES = TC ? 3 * kRows : 0;  // TC: per-warp activation digit planes [3][64] bytes
    static constexpr int RED = 2 * W * E * 4;          // two deposit buffers
    static constexpr int HAND = E * 4;
    static constexpr int FIXED = W * XSLOT + W * PLANES + RED + HAND + 1024;
    static constexpr int CAP = TC ? kSmemCapTc : kSmemCap;
    static constexpr int RMAX = TC ? 24 : 16;
    static constexpr int R0 = (CAP - FIXED) / SLOT;
    static constexpr int R = R0 < RMAX ? R0 : RMAX;   // ring slots
    static constexpr int RING_OFF = 0;
    static constexpr int X_OFF = R * SLOT;
    static constexpr int PL_OFF = X_OFF + W * XSLOT;
    static constexpr int RED_OFF = PL_OFF + W * PLANES;
    static constexpr int HAND_OFF = RED_OFF + RED;
    static constexpr int BAR_OFF = HAND_OFF + HAND;
    static constexpr int MISC_OFF = BAR_OFF + (2 * R + 1) * 8;
    static constexpr int SMEM = MISC_OFF + 64;
    static_assert(R >= 6, "ring too shallow");
    static_assert(SMEM <= CAP, "shared memory budget");
};

struct CmvParams {
    const uint8_t *codes;
    const float *scale;
    const float *x;
    float *out;
    float *partial;
    unsigned *counters;
    unsigned *status;
    long long items;
    int rows, cols, half, units, tiles;
    uint32_t magic; // 0x4B000000 (2^23), passed in so it sits in a register: one LOP3 per nibble
    int k;          // cluster split: CTAs per column tile (kcmv_kernel)
    int epi;        // TQ_EPI_* (M = 1)
};


// Output column of sum j of lane `lane` in tile `tile` (int4: -1 if beyond N/2 pairs).
template <int BITS>
__device__ __forceinline__ int out_col(const CmvParams &p, int tile, int lane, int j) {
    if (BITS == 8) {
        const int col = tile * kCols + 4 * lane + j;
        return col < p.cols ? col : -1;
    }
    const int e = j & 3, hi = j >> 2;
    const int pair = tile * kCols + 4 * lane + e;
    if (pair >= p.half) return -1;
    return hi ? p.half + pair : pair;
}

// Entry e = (m*NP + q)*32 + l of a finished tile to the output. With the
// SwiGLU epilogue (int4, M = 1) the gate entries (q < 4) write silu(v) * u,
// u being the sum of their up partner e + kUp, and the up entries nothing.
constexpr int kUp = 4 * 32;
template <int BITS>
__device__ __forceinline__ void write_entry(const CmvParams &p, int tile, int e, float v, float u) {
    constexpr int NP = BITS == 8 ? 4 : 8;
    const int l = e & 31, q = (e >> 5) % NP, m = (e >> 5) / NP;
    if (BITS == 4 && p.epi == TQ_EPI_SWIGLU) {
        const int c = tile * kCols + 4 * l + q;
        if (q < 4 && c < p.half) p.out[c] = swiglu(v, u);
        return;
    }
    const int col = out_col<BITS>(p, tile, l, q);
    if (col >= 0) p.out[(size_t)m * p.cols + col] = BITS == 8 ? v * __ldg(p.scale + col) : v;
}
// Whether entry e needs its up partner's sum too (SwiGLU gate entries).
template <int BITS> __device__ __forceinline__ bool needs_up(const CmvParams &p, int e) {
    return BITS == 4 && p.epi == TQ_EPI_SWIGLU && e < kUp;
}

// Sums of a finished tile (entry (m, j, lane) in the order [m][j][lane]) to the output.
template <int BITS, int M>
__device__ __forceinline__ void write_out(const CmvParams &p, int tile, int lane, const float (&v)[M][BITS == 8 ? 4 : 8]) {
    constexpr int NP = BITS == 8 ? 4 : 8;
    if constexpr (BITS == 4 && M == 1) {
        if (p.epi == TQ_EPI_SWIGLU) { // sums e (gate column c) and 4 + e (up column c)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int c = tile * kCols + 4 * lane + e;
                if (c < p.half) p.out[c] = swiglu(v[0][e], v[0][4 + e]);
            }
            return;
        }
    }
#pragma unroll
    for (int j = 0; j < NP; j++) {
        const int col = out_col<BITS>(p, tile, lane, j);
        if (col < 0) continue;
        const float sc = BITS == 8 ? __ldg(p.scale + col) : 1.f;
#pragma unroll
        for (int m = 0; m < M; m++) p.out[(size_t)m * p.cols + col] = BITS == 8 ? v[m][j] * sc : v[m][j];
    }
}

// A shared tile, by one warp (lane holds entries [m][j][lane]): publish this
// CTA's sums, count in, and if last add every contributor in CTA order.
template <int BITS, int M>
__device__ void publish_shared(const CmvParams &p, const TqSplit &split, int c, int tile, int lane,
                               const float (&v)[M][BITS == 8 ? 4 : 8]) {
    constexpr int NP = BITS == 8 ? 4 : 8;
    constexpr int E = M * NP * 32;
    const long long t0 = (long long)tile * p.units;
    const int cf = split.owner(t0), cl = split.owner(t0 + p.units - 1);
    float *dst = p.partial + (size_t)split.slot(c, t0) * E + lane;
#pragma unroll
    for (int m = 0; m < M; m++)
#pragma unroll
        for (int j = 0; j < NP; j++) dst[(m * NP + j) * 32] = v[m][j];
    // __syncwarp orders the lanes' stores before lane 0's cumulative acq_rel
    // arrival; for the last CTA its acquire, then __syncwarp, orders the other
    // CTAs' partials before the lanes' loads.
    __syncwarp();
    int last = 0;
    if (lane == 0) last = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1)) ? 1 : 0;
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) return;
    const int slot_f = split.slot(cf, t0);
    float s[M][NP];
#pragma unroll
    for (int m = 0; m < M; m++)
#pragma unroll
        for (int j = 0; j < NP; j++) s[m][j] = 0.f;
    constexpr int CH = 32 / (M * NP) > 0 ? 32 / (M * NP) : 1; // contributors per round of loads
    for (int cc = cf; cc <= cl; cc += CH) {
        float pv[CH][M][NP];
#pragma unroll
        for (int u = 0; u < CH; u++) {
            const int c2 = cc + u;
            const float *src = p.partial + (size_t)(c2 == cf ? slot_f : 2 * c2) * E + lane;
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int j = 0; j < NP; j++) pv[u][m][j] = c2 <= cl ? __ldcg(src + (m * NP + j) * 32) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < CH; u++)
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int j = 0; j < NP; j++) s[m][j] += pv[u][m][j];
    }
    write_out<BITS, M>(p, tile, lane, s);
}


template <int BITS, int M, bool TC = false>
__global__ void __launch_bounds__(kThreads, TC ? 1 : 2) cmv_kernel(CmvParams p) {
    using C = CCfg<BITS, M, TC>;
    static_assert(!TC || (BITS == 4 && M == 1), "the tensor-core variant is int4, one row");
    constexpr int R = C::R, NP = C::NP, E = C::E;
    // 16-byte alignment is all the bulk copies and vector loads need; indexing
    // the array directly keeps every access in the shared state space.
    extern __shared__ __align__(16) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + R;
    uint64_t *hand_full = empty + R;
    volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF);
    int *cnt = reinterpret_cast<int *>(smem + C::MISC_OFF + 16);             // [2] deposits per buffer
    volatile int *ready = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 32); // [2] next segment a buffer takes
    // Items issued by the producer so far. Consumers take items out of ring
    // order (warp cw takes items cw, cw + W, ...), so before the parity wait
    // on full[j % R] for item j a consumer checks that item j was issued: the
    // producer issues it only after item j - R was consumed, so the barrier's
    // previous phase is complete and the parity test cannot pass on it.
    volatile int *issued = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 48);
    volatile int *lastflag = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 52);
    volatile int *first_last = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 56);
    float *red = reinterpret_cast<float *>(smem + C::RED_OFF);
    float *hand = reinterpret_cast<float *>(smem + C::HAND_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const TqSplit split(p.items, G);
    const long long i0 = split.start(c), i1 = split.start(c + 1);
    const int nitems = (int)(i1 - i0);
    // Tile segments of the slice: segment s holds slice items [sb(s), sb(s + 1)).
    const int tile0 = (int)(i0 / p.units);
    auto seg_begin = [&](int s) { // slice-relative first item of segment s
        return s == 0 ? 0 : (int)((long long)(tile0 + s) * p.units - i0);
    };
    const int nseg = (int)((i1 - 1) / p.units) - tile0 + 1;
    const long long ft0 = (long long)tile0 * p.units;
    const bool first_shared = split.owner(ft0) != split.owner(ft0 + p.units - 1);
    const bool handoff = first_shared && nseg > 1;
    // The slice's last tile segment: its owners and this CTA's partial slot,
    // worked out now rather than on the reduction's critical path at the end.
    const int last_tile = tile0 + nseg - 1;
    const long long lt0 = (long long)last_tile * p.units;
    const int last_cf = split.owner(lt0), last_cl = split.owner(lt0 + p.units - 1);
    const int last_slot = split.slot(c, lt0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2); // both halves consumed
        }
        mbar_init(hand_full, 1);
        *abort = 0;
        cnt[0] = cnt[1] = 0;
        ready[0] = 0;
        ready[1] = 1;
        *issued = 0;
        *first_last = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer: the weights depend on nothing ----------------
        if (lane == 0) {
            // The next kernel on the stream may be scheduled now: its CTAs fit
            // beside this one and only stream their weights until this kernel
            // completes (griddepcontrol.wait).
            pdl_trigger();
            for (int j = 0; j < nitems; j++) {
                const int s = j % R;
                if (j >= R && !wait_bar(&empty[s], ((j / R) & 1) ^ 1, abort, p.status)) continue;
                const long long it = i0 + j;
                uint8_t *dst = smem + C::RING_OFF + s * C::SLOT;
                mbar_arrive_expect_tx(&full[s], C::SLOT);
                if (TC) { // one K-packed item: codes then scales, contiguous
                    bulk_load(dst, p.codes + it * TQ_KPACK_BYTES, TQ_KPACK_BYTES, &full[s]);
                } else {
                    bulk_load(dst, p.codes + it * kItem, kItem, &full[s]);
                    if (BITS == 4) bulk_load(dst + kItem, p.scale + it * (2 * kCols), 1024, &full[s]);
                }
                *issued = j + 1;
            }
        }
    } else if (warp <= W) {
        // ---------------- consumers ----------------
        const int cw = warp - 1;
        const uint32_t mg = p.magic;
        pdl_wait(); // x, the output and the scratch belong to the previous kernel until here
        // Warp cw takes half h = cw % 2 (rows 32h..32h+31) of items js, js + WI,
        // ... with js = cw / 2: the work units k = 2j + h with k = cw (mod W).
        const int hf = cw & 1, js = cw >> 1;
        // Activations of this warp's half items: ring slot t % XD holds item t's
        // rows 32h..32h+31 for every m ([m][32] floats), copied by cp.async
        // XD - 1 items ahead; lane l copies row 32h + l and reads all rows
        // after cp.async.wait_group and __syncwarp.
        float *xs = reinterpret_cast<float *>(smem + C::X_OFF + cw * C::XSLOT);
        int unit_x = (int)((i0 + js) % p.units); // unit (64-row group) of the next item to copy activations for
        int tx = 0;                            // items of this warp whose activations were issued
        const int nmine = js < nitems ? (nitems - 1 - js) / WI + 1 : 0;
        const float *xrow = p.x + hf * kHalf + lane; // + unit * 64 + m * rows
        auto issue_x = [&]() { // one cp.async group per call (empty past this warp's last item)
            if (tx < nmine) {
                if constexpr (TC) { // all 64 rows: lane l copies rows l and 32 + l
                    float *dst = xs + (tx & (C::XD - 1)) * kRows + lane;
                    const int r0 = unit_x * kRows + lane, r1 = r0 + kHalf;
                    cp_async_f32(dst, p.x + (r0 < p.rows ? r0 : 0), r0 < p.rows);
                    cp_async_f32(dst + kHalf, p.x + (r1 < p.rows ? r1 : 0), r1 < p.rows);
                } else {
                    float *dst = xs + (tx & (C::XD - 1)) * M * kHalf + lane;
                    const int row = unit_x * kRows + hf * kHalf + lane;
                    const bool v = row < p.rows;
                    const float *src = xrow + (v ? unit_x * kRows : -(hf * kHalf + lane));
#pragma unroll
                    for (int m = 0; m < M; m++) cp_async_f32(dst + m * kHalf, src + (size_t)m * p.rows, v);
                }
                unit_x += WI; // next item of this warp: WI units on, modulo the units of a tile
                while (unit_x >= p.units) unit_x -= p.units;
            }
            cp_async_commit();
            tx++;
        };
        static_assert((C::XD & (C::XD - 1)) == 0, "XD must be a power of two");
        for (int i = 0; i < C::XD - 1; i++) issue_x();
        // byte offset of this lane's code word (bytes 4l..4l+3) in row k of an
        // 8-row group: chunk l/4 of row r sits at chunk (l/4) ^ (r % 8)
        uint32_t ofs[8];
#pragma unroll
        for (int k = 0; k < 8; k++) ofs[k] = k * kCols + 4 * (lane ^ (k << 2));

        float acc[M][NP];
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int j = 0; j < NP; j++) acc[m][j] = 0.f;
        // TC: the lane's partial sums per MMA block and row half, moved into
        // acc (quad-added, the lane's own columns) before each deposit
        float accp[TC ? 8 : 1][2];
#pragma unroll
        for (int cb = 0; cb < (TC ? 8 : 1); cb++) accp[cb][0] = accp[cb][1] = 0.f;
        auto flush = [&]() {
            if constexpr (TC) tmv_flush(accp, acc, lane, hf);
        };

        // Deposits this warp's sums of segment s; the last warp to deposit
        // reduces the segment and hands it on.
        auto deposit = [&](int s) {
            const int sb = 2 * seg_begin(s), se = 2 * (s + 1 < nseg ? seg_begin(s + 1) : nitems); // work units
            const int len = se - sb;
            const int parts = len < W ? len : W; // warps with work in the segment
            // warps with work: cw = (sb + i) % W, i < len
            const bool mine = len >= W || ((cw - sb % W + W) % W) < len;
            if (!mine) return;
            const int b = s & 1;
            // buffer b is free once segment s - 2 was reduced
            if (ready[b] < s) {
                const unsigned long long t0 = global_ns();
                while (ready[b] < s) {
                    if (*abort) break;
                    if (global_ns() - t0 > kWaitNs) {
                        atomicOr(p.status, TQ_STATUS_TIMEOUT);
                        *abort = 1;
                        break;
                    }
                }
            }
            float *rb = red + (size_t)(b * W + cw) * E + lane;
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int j = 0; j < NP; j++) rb[(m * NP + j) * 32] = acc[m][j];
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                __threadfence_block(); // this warp's deposit before its count
                last = atomicAdd(&cnt[b], 1) == parts - 1;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) return;
            __threadfence_block(); // every other warp's deposit before the reads below
            // reduce the deposits in warp order
            float v[M][NP];
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int j = 0; j < NP; j++) v[m][j] = 0.f;
            for (int i = 0; i < parts; i++) { // warps in a fixed order
                const int w = len >= W ? i : (sb + i) % W;
                const float *src = red + (size_t)(b * W + w) * E + lane;
#pragma unroll
                for (int m = 0; m < M; m++)
#pragma unroll
                    for (int j = 0; j < NP; j++) v[m][j] += src[(m * NP + j) * 32];
            }
            __syncwarp();
            if (lane == 0) {
                cnt[b] = 0;
                __threadfence_block();
                ready[b] = s + 2;
            }
            const int tile = tile0 + s;
            const long long t0 = (long long)tile * p.units;
            if (split.owner(t0) == split.owner(t0 + p.units - 1)) {
                write_out<BITS, M>(p, tile, lane, v);
            } else if (s == 0 && handoff) {
                float *hb = hand + lane;
#pragma unroll
                for (int m = 0; m < M; m++)
#pragma unroll
                    for (int j = 0; j < NP; j++) hb[(m * NP + j) * 32] = v[m][j];
                __syncwarp();
                if (lane == 0) mbar_arrive(hand_full);
            } else {
                publish_shared<BITS, M>(p, split, c, tile, lane, v);
            }
        };

        int s = 0;                                   // segment of the next item
        int next_sb = nseg > 1 ? seg_begin(1) : nitems; // first item of segment s + 1
        const uint8_t *ring = smem + C::RING_OFF;
        static_assert(R >= WI, "ring shorter than the item streams");
        int slot = js % R, ph = (js / R) & 1; // ring slot and full-barrier parity of item j
        for (int j = js, t_it = 0; j < nitems; j += WI, t_it++) {
            while (j >= next_sb) {
                flush();
                deposit(s);
#pragma unroll
                for (int m = 0; m < M; m++)
#pragma unroll
                    for (int q = 0; q < NP; q++) acc[m][q] = 0.f;
                s++;
                next_sb = s + 1 < nseg ? next_sb + p.units : nitems;
            }
            issue_x(); // activations of this warp's item t_it + XD - 1
            cp_async_wait<C::XD - 1>(); // this item's have landed (this lane's copies)
            if (*issued <= j) { // bounded: the producer is normally far ahead
                const unsigned long long t0 = global_ns();
                while (*issued <= j && !*abort) {
                    if (global_ns() - t0 > kWaitNs) {
                        atomicOr(p.status, TQ_STATUS_TIMEOUT);
                        *abort = 1;
                    }
                }
            }
            const bool ok = wait_bar(&full[slot], ph, abort, p.status);
            __syncwarp(); // every lane's activation copies visible to the whole warp
            const uint8_t *item = ring + slot * C::SLOT;
            if constexpr (TC) {
                const float *xr = xs + (t_it & (C::XD - 1)) * kRows;
                if (ok) tmv_item(item, hf, xr, smem + C::PL_OFF + cw * C::PLANES, lane, accp);
            } else {
                const float *xr = xs + (t_it & (C::XD - 1)) * M * kHalf;
                if (ok) half_item<BITS, M>(item, hf, xr, ofs, mg, lane, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            __syncwarp(); // the x slot is reused XD - 1 items later
            slot += WI;
            if (slot >= R) {
                slot -= R;
                ph ^= 1;
            }
        }
        // segments before the last one that this warp has not deposited yet
        flush();
        for (; s < nseg - 1; s++) {
            deposit(s);
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int q = 0; q < NP; q++) acc[m][q] = 0.f;
        }
        // The last CTA to arrive at a shared tile adds every contributor's sums
        // in CTA order, one entry per thread, all contributor loads in flight.
        auto reduce_all = [&](int tile) {
            const long long t0 = (long long)tile * p.units;
            const int cf = split.owner(t0), cl = split.owner(t0 + p.units - 1);
            const int slot_f = split.slot(cf, t0);
            auto sum_entry = [&](int e) {
                constexpr int CH = 16; // contributor loads in flight per thread
                float v = 0.f;
                for (int cc = cf; cc <= cl; cc += CH) {
                    float pv[CH];
#pragma unroll
                    for (int u = 0; u < CH; u++) {
                        const int c2 = cc + u;
                        pv[u] = c2 <= cl ? __ldcg(p.partial + (size_t)(c2 == cf ? slot_f : 2 * c2) * E + e) : 0.f;
                    }
#pragma unroll
                    for (int u = 0; u < CH; u++) v += pv[u];
                }
                return v;
            };
            for (int e = threadIdx.x - 32; e < E; e += W * 32) {
                if (BITS == 4 && p.epi == TQ_EPI_SWIGLU && e >= kUp) continue; // taken by its gate entry
                const float v = sum_entry(e);
                write_entry<BITS>(p, tile, e, v, needs_up<BITS>(p, e) ? sum_entry(e + kUp) : 0.f);
            }
        };
        // The slice's last segment, by all consumer warps: every warp's sums
        // (zero if it had no item there) are added in warp order, one entry per
        // thread, and a shared tile is published and, by the last CTA to
        // arrive, reduced with every contributor's load in flight at once.
        {
            const int sl = nseg - 1, b = sl & 1;
            if (ready[b] < sl) { // buffer b is free once segment sl - 2 was reduced
                const unsigned long long t0 = global_ns();
                while (ready[b] < sl && !*abort) {
                    if (global_ns() - t0 > kWaitNs) {
                        atomicOr(p.status, TQ_STATUS_TIMEOUT);
                        *abort = 1;
                    }
                }
            }
            float *rb = red + (size_t)(b * W + cw) * E + lane;
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int q = 0; q < NP; q++) rb[(m * NP + q) * 32] = acc[m][q];
            named_sync(1, W * 32);
            const int tile = last_tile, cf = last_cf, cl = last_cl;
            const int ct = threadIdx.x - 32; // 0 .. W*32-1
            float *part = p.partial + (size_t)last_slot * E;
            auto warp_sum = [&](int e) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < W; w++) v += red[(size_t)(b * W + w) * E + e];
                return v;
            };
            for (int e = ct; e < E; e += W * 32) { // entry e = (m*NP + q)*32 + l
                const float v = warp_sum(e);
                if (cf == cl) {
                    if (!(BITS == 4 && p.epi == TQ_EPI_SWIGLU && e >= kUp))
                        write_entry<BITS>(p, tile, e, v, needs_up<BITS>(p, e) ? warp_sum(e + kUp) : 0.f);
                } else {
                    part[e] = v;
                }
            }
            if (cf != cl) {
                // The barrier orders every thread's partial stores before thread
                // 0's acq_rel arrival, whose release is cumulative over them; for
                // the last CTA its acquire, followed by the second barrier,
                // orders the other CTAs' partials before every thread's loads.
                named_sync(1, W * 32);
                if (ct == 0) *lastflag = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1)) ? 1 : 0;
                named_sync(1, W * 32);
                if (*lastflag) reduce_all(tile);
            }
        }
        if (handoff) { // the first segment, published by the fixup warp
            named_sync(2, W * 32 + 32);
            if (*first_last) reduce_all(tile0);
        }
    } else {
        // ---------------- fixup: the first segment, when shared and not last ----------------
        if (handoff) {
            pdl_wait();
            wait_bar(hand_full, 0, abort, p.status);
            float v[M][NP];
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int j = 0; j < NP; j++) v[m][j] = hand[(m * NP + j) * 32 + lane];
            // publish this CTA's sums; if it is the last to arrive, the
            // consumer warps add the contributors (all loads in flight)
            const int cf = split.owner(ft0), cl = split.owner(ft0 + p.units - 1);
            float *dst = p.partial + (size_t)split.slot(c, ft0) * E + lane;
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int j = 0; j < NP; j++) dst[(m * NP + j) * 32] = v[m][j];
            __syncwarp(); // the lanes' stores before lane 0's cumulative acq_rel arrival
            if (lane == 0) *first_last = tq_arrive_last(&p.counters[tile0], (unsigned)(cl - cf + 1)) ? 1 : 0;
            __syncwarp();
            named_arrive(2, W * 32 + 32);
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Cluster split, for matrices with fewer column tiles than SMs: column tile t
// goes to cluster t of k CTAs (k <= 8, k * tiles <= SMs), and CTA rank r of
// the cluster takes the tile's 64-row units [r*units/k, (r+1)*units/k). Each
// CTA runs the same item pipeline as cmv_kernel (producer ring filled before
// griddepcontrol.wait, eight consumer warps on half items) and adds its warps'
// sums in warp order in shared memory; the k CTAs' sums then meet in
// distributed shared memory: after a cluster barrier, CTA r adds the k CTAs'
// sums of its 1/k of the tile's entries in rank order and writes them, and a
// second cluster barrier keeps every CTA's shared memory alive until all
// reads are done. No global scratch and no atomics: the reduction costs two
// cluster barriers instead of global round trips.
// ---------------------------------------------------------------------------
template <int BITS, int M, bool TC = false> struct KCfg {
    static constexpr int NP = BITS == 8 ? 4 : 8;
    static constexpr int E = M * NP * 32;
    static constexpr int SLOT = BITS == 4 ? kItem + 1024 : kItem;
    static constexpr int XD = 4;
    static constexpr int XSLOT = XD * (TC ? kRows : kHalf) * M * 4;
    static constexpr int PLANES = TC ? 3 * kRows : 0;
    static constexpr int RED = W * E * 4;  // per-warp sums
    static constexpr int CPART = E * 4;    // this CTA's sums, read across the cluster
    static constexpr int FIXED = W * XSLOT + W * PLANES + RED + CPART + 1024;
    static constexpr int CAP = TC ? kSmemCapTc : kSmemCap;
    static constexpr int RMAX = TC ? 24 : 16;
    static constexpr int R0 = (CAP - FIXED) / SLOT;
    static constexpr int R = R0 < RMAX ? R0 : RMAX; // ring slots
    static constexpr int RING_OFF = 0;
    static constexpr int X_OFF = R * SLOT;
    static constexpr int PL_OFF = X_OFF + W * XSLOT;
    static constexpr int RED_OFF = PL_OFF + W * PLANES;
    static constexpr int CPART_OFF = RED_OFF + RED;
    static constexpr int BAR_OFF = CPART_OFF + CPART;
    static constexpr int MISC_OFF = BAR_OFF + 2 * R * 8;
    static constexpr int SMEM = MISC_OFF + 32;
    static_assert(R >= 6, "ring too shallow");
    static_assert(SMEM <= CAP, "shared memory budget");
};
constexpr int kKThreads = (W + 1) * 32; // producer warp + consumer warps
constexpr int kMaxCluster = 8;

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A float of the shared memory of cluster CTA `rank` at this CTA's address p.
__device__ __forceinline__ float ld_cluster(const float *p, uint32_t rank) {
    uint32_t remote;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

template <int BITS, int M, bool TC = false>
__global__ void __launch_bounds__(kKThreads, TC ? 1 : 2) kcmv_kernel(CmvParams p) {
    using C = KCfg<BITS, M, TC>;
    static_assert(!TC || (BITS == 4 && M == 1), "the tensor-core variant is int4, one row");
    constexpr int R = C::R, NP = C::NP, E = C::E;
    extern __shared__ __align__(16) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + R;
    volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF);
    volatile int *issued = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4); // see cmv_kernel
    float *red = reinterpret_cast<float *>(smem + C::RED_OFF);
    float *cpart = reinterpret_cast<float *>(smem + C::CPART_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k = p.k;
    const int tile = blockIdx.x / k, r = blockIdx.x % k; // r is the cluster rank: clusters are k consecutive CTAs
    const int u0 = (int)((long long)r * p.units / k), u1 = (int)((long long)(r + 1) * p.units / k);
    const int nitems = u1 - u0;
    const long long i0 = (long long)tile * p.units + u0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2); // both halves consumed
        }
        *abort = 0;
        *issued = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer: the weights depend on nothing ----------------
        if (lane == 0) {
            pdl_trigger(); // the next kernel on the stream may be scheduled beside this one
            for (int j = 0; j < nitems; j++) {
                const int s = j % R;
                if (j >= R && !wait_bar(&empty[s], ((j / R) & 1) ^ 1, abort, p.status)) continue;
                const long long it = i0 + j;
                uint8_t *dst = smem + C::RING_OFF + s * C::SLOT;
                mbar_arrive_expect_tx(&full[s], C::SLOT);
                if (TC) { // one K-packed item: codes then scales, contiguous
                    bulk_load(dst, p.codes + it * TQ_KPACK_BYTES, TQ_KPACK_BYTES, &full[s]);
                } else {
                    bulk_load(dst, p.codes + it * kItem, kItem, &full[s]);
                    if (BITS == 4) bulk_load(dst + kItem, p.scale + it * (2 * kCols), 1024, &full[s]);
                }
                *issued = j + 1;
            }
        }
    } else {
        // ---------------- consumers: warp cw takes half h = cw % 2 of items cw/2, cw/2 + WI, ... ----------------
        const int cw = warp - 1;
        const uint32_t mg = p.magic;
        const int hf = cw & 1, js = cw >> 1;
        pdl_wait(); // x belongs to the previous kernel until here
        float *xs = reinterpret_cast<float *>(smem + C::X_OFF + cw * C::XSLOT);
        int unit_x = u0 + js; // unit of the next item to copy activations for
        int tx = 0;
        const int nmine = js < nitems ? (nitems - 1 - js) / WI + 1 : 0;
        const float *xrow = p.x + hf * kHalf + lane;
        auto issue_x = [&]() {
            if (tx < nmine) {
                if constexpr (TC) { // all 64 rows: lane l copies rows l and 32 + l
                    float *dst = xs + (tx & (C::XD - 1)) * kRows + lane;
                    const int r0 = unit_x * kRows + lane, r1 = r0 + kHalf;
                    cp_async_f32(dst, p.x + (r0 < p.rows ? r0 : 0), r0 < p.rows);
                    cp_async_f32(dst + kHalf, p.x + (r1 < p.rows ? r1 : 0), r1 < p.rows);
                } else {
                    float *dst = xs + (tx & (C::XD - 1)) * M * kHalf + lane;
                    const int row = unit_x * kRows + hf * kHalf + lane;
                    const bool v = row < p.rows;
                    const float *src = xrow + (v ? unit_x * kRows : -(hf * kHalf + lane));
#pragma unroll
                    for (int m = 0; m < M; m++) cp_async_f32(dst + m * kHalf, src + (size_t)m * p.rows, v);
                }
                unit_x += WI;
            }
            cp_async_commit();
            tx++;
        };
        for (int i = 0; i < C::XD - 1; i++) issue_x();
        uint32_t ofs[8];
#pragma unroll
        for (int q = 0; q < 8; q++) ofs[q] = q * kCols + 4 * (lane ^ (q << 2));
        float acc[M][NP];
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int q = 0; q < NP; q++) acc[m][q] = 0.f;
        float accp[TC ? 8 : 1][2]; // TC: partial sums per MMA block and row half (see tmv_flush)
#pragma unroll
        for (int cb = 0; cb < (TC ? 8 : 1); cb++) accp[cb][0] = accp[cb][1] = 0.f;
        const uint8_t *ring = smem + C::RING_OFF;
        int slot = js % R, ph = (js / R) & 1;
        for (int j = js, t_it = 0; j < nitems; j += WI, t_it++) {
            issue_x();
            cp_async_wait<C::XD - 1>();
            if (*issued <= j) {
                const unsigned long long t0 = global_ns();
                while (*issued <= j && !*abort) {
                    if (global_ns() - t0 > kWaitNs) {
                        atomicOr(p.status, TQ_STATUS_TIMEOUT);
                        *abort = 1;
                    }
                }
            }
            const bool ok = wait_bar(&full[slot], ph, abort, p.status);
            __syncwarp();
            const uint8_t *item = ring + slot * C::SLOT;
            if constexpr (TC) {
                if (ok) tmv_item(item, hf, xs + (t_it & (C::XD - 1)) * kRows, smem + C::PL_OFF + cw * C::PLANES, lane, accp);
            } else {
                if (ok) half_item<BITS, M>(item, hf, xs + (t_it & (C::XD - 1)) * M * kHalf, ofs, mg, lane, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            __syncwarp();
            slot += WI;
            if (slot >= R) {
                slot -= R;
                ph ^= 1;
            }
        }
        cp_async_wait<0>();
        if constexpr (TC) tmv_flush(accp, acc, lane, hf);
        float *rb = red + (size_t)cw * E + lane;
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int q = 0; q < NP; q++) rb[(m * NP + q) * 32] = acc[m][q];
    }
    __syncthreads(); // every warp's sums are in red
    pdl_wait();      // the output belongs to the previous kernel until here (consumers waited already)
    // this CTA's sums: entries e = (m*NP + q)*32 + l, warps added in order
    for (int e = threadIdx.x; e < E; e += kKThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < W; w++) v += red[w * E + e];
        cpart[e] = v;
    }
    // entries written: with SwiGLU the gate entries, each taking its up partner
    const bool sw = BITS == 4 && p.epi == TQ_EPI_SWIGLU;
    const int EW = sw ? kUp : E;
    if (k == 1) {
        __syncthreads();
        for (int e = threadIdx.x; e < EW; e += kKThreads) write_entry<BITS>(p, tile, e, cpart[e], sw ? cpart[e + kUp] : 0.f);
    } else {
        cluster_sync_all(); // every CTA's cpart is complete and visible to the cluster
        const int lo = r * EW / k, hi = (r + 1) * EW / k;
        for (int e = lo + threadIdx.x; e < hi; e += kKThreads) {
            float v = 0.f, u = 0.f;
            for (int q = 0; q < k; q++) v += ld_cluster(cpart + e, (uint32_t)q);
            if (sw)
                for (int q = 0; q < k; q++) u += ld_cluster(cpart + e + kUp, (uint32_t)q);
            write_entry<BITS>(p, tile, e, v, u);
        }
        cluster_sync_all(); // no CTA leaves (and frees its shared memory) while others still read it
    }
}

template <int BITS, int M>
cudaError_t launch_kcmv(const TqMatrixDev &mat, const float *x, float *out, const TqScratch &scr, cudaStream_t st,
                        int k, int epi, bool tc = false) {
    using C = KCfg<BITS, M>;
    constexpr bool kHasTc = BITS == 4 && M == 1;
    using CT = KCfg<4, 1, true>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static TqDeviceOnce once;
    e = tq_device_once(once, dev, [] {
        cudaError_t r = cudaFuncSetAttribute(kcmv_kernel<BITS, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if constexpr (kHasTc) {
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(kcmv_kernel<4, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CT::SMEM);
        }
        return r;
    });
    if (e != cudaSuccess) return e;
    CmvParams prm = {};
    prm.codes = tc ? mat.kpack : mat.codes;
    prm.scale = tc ? nullptr : mat.scale;
    prm.x = x;
    prm.out = out;
    prm.status = scr.status;
    prm.rows = mat.rows;
    prm.cols = mat.cols;
    prm.half = mat.cols / 2;
    prm.units = mat.units;
    prm.tiles = mat.tiles;
    prm.items = (long long)mat.tiles * mat.units;
    prm.magic = 0x4B000000u;
    prm.k = k;
    prm.epi = epi;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = k;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cfg.gridDim = dim3(mat.tiles * k);
    cfg.blockDim = dim3(kKThreads);
    if constexpr (kHasTc) {
        if (tc) {
            cfg.dynamicSmemBytes = CT::SMEM;
            return cudaLaunchKernelEx(&cfg, kcmv_kernel<4, 1, true>, prm);
        }
    }
    cfg.dynamicSmemBytes = C::SMEM;
    return cudaLaunchKernelEx(&cfg, kcmv_kernel<BITS, M>, prm);
}

// Cluster size for the cluster split, or 0 for the stream-K kernel. With
// fewer column tiles than SMs each tile gets k = min(8, SMs / tiles, units)
// CTAs, so k * tiles <= SMs: the reduction is cheap but up to a few SMs idle
// and each CTA takes a little more. Measured on B200, that wins for int8 (the
// unpack is cheap, the call is latency-bound) and for small int4 matrices,
// and loses for int4 matrices of more than 12 items per SM under stream-K
// (the unpack is ALU-bound): 4096 x 11008 took 14.3 us per call split by
// clusters against 10.0 us by stream-K.
inline int cluster_split(const TqMatrixDev &mat, int sms) {
    if (mat.tiles >= sms) return 0;
    if (mat.bits == 4 && (long long)mat.tiles * mat.units > 12LL * sms) return 0;
    int k = sms / mat.tiles;
    if (k > kMaxCluster) k = kMaxCluster;
    if (k > mat.units) k = mat.units;
    return k < 1 ? 1 : k;
}

// Cluster size for the tensor-core variant: with fewer column tiles than SMs
// and at most 12 items per SM, k = min(8, SMs / tiles, units) CTAs per tile;
// 0 = stream-K. Measured on B200: the 4096 x 11008 / 11008 x 4096 pair (19
// items per SM) took 11.7 us per call by clusters and 9.4 by stream-K.
inline int cluster_split_tc(const TqMatrixDev &mat, int sms) {
    if (mat.tiles >= sms || (long long)mat.tiles * mat.units > 12LL * sms) return 0;
    int k = sms / mat.tiles;
    if (k > kMaxCluster) k = kMaxCluster;
    if (k > mat.units) k = mat.units;
    return k < 1 ? 1 : k;
}

template <int BITS, int M>
cudaError_t launch_cmv(const TqMatrixDev &mat, const float *x, float *out, const TqScratch &scr, cudaStream_t st,
                       int epi, bool tc = false) {
    using C = CCfg<BITS, M>;
    constexpr bool kHasTc = BITS == 4 && M == 1;
    using CT = CCfg<4, 1, true>;
    tc = tc && kHasTc && mat.kpack;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static TqDeviceOnce once;
    e = tq_device_once(once, dev, [] {
        cudaError_t r = cudaFuncSetAttribute(cmv_kernel<BITS, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if constexpr (kHasTc) {
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(cmv_kernel<4, 1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, CT::SMEM);
        }
        return r;
    });
    if (e != cudaSuccess) return e;
    CmvParams prm = {};
    prm.codes = tc ? mat.kpack : mat.codes;
    prm.scale = tc ? nullptr : mat.scale;
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
    prm.items = (long long)mat.tiles * mat.units;
    prm.magic = 0x4B000000u;
    prm.epi = epi;
    const int sms = once.sms[dev];
    if (mat.tiles > TQ_MAX_TILES || sms > TQ_MAX_CTAS) return cudaErrorInvalidValue;
    if (const int k = tc ? cluster_split_tc(mat, sms) : cluster_split(mat, sms))
        return launch_kcmv<BITS, M>(mat, x, out, scr, st, k, epi, tc);
    if ((size_t)2 * sms * C::E > TQ_SCRATCH_PARTIAL_FLOATS) return cudaErrorInvalidValue;
    const int ctas = (int)(prm.items < sms ? prm.items : sms);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    if constexpr (kHasTc) {
        if (tc) {
            cfg.dynamicSmemBytes = CT::SMEM;
            return cudaLaunchKernelEx(&cfg, cmv_kernel<4, 1, true>, prm);
        }
    }
    cfg.dynamicSmemBytes = C::SMEM;
    return cudaLaunchKernelEx(&cfg, cmv_kernel<BITS, M>, prm);
}

// Item column of MMA row rho of block cb in warp half hf (tensor-core variant).
TQ_HD int tmv_col(int hf, int cb, int rho) { return 128 * hf + 4 * (4 * (rho & 7) + (cb & 3)) + 2 * (cb >> 2) + (rho >> 3); }

// The K-packed copy of an int4 matrix (see the tensor-core variant above):
// one thread per 4-byte word of an item's K-packed codes (8 codes of one item
// column), then one per scale float; item it occupies kpack[it * TQ_KPACK_BYTES ..].
__global__ void repack4_kernel(const uint8_t *__restrict__ codes, const float *__restrict__ scale,
                               uint8_t *__restrict__ kpack, long long items) {
    const long long words = items * (kItem / 4), stride = (long long)gridDim.x * blockDim.x;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < words; i += stride) {
        const long long it = i / (kItem / 4);
        const int wi = (int)(i % (kItem / 4));
        const int q = wi & 3, lane = (wi >> 2) & 31, cb = (wi >> 7) & 7, hf = wi >> 10;
        const int rho = (lane >> 2) + 8 * (q & 1), kb = (lane & 3) + 4 * (q >> 1);
        const int j = tmv_col(hf, cb, rho), b = j & 127, hi = j >> 7;
        const uint8_t *src = codes + it * kItem;
        uint32_t w = 0;
#pragma unroll
        for (int r = 0; r < 8; r++) {
            const uint32_t byte = src[tq_item_offset(8 * kb + r, b)];
            w |= (hi ? byte >> 4 : byte & 15u) << (4 * r);
        }
        reinterpret_cast<uint32_t *>(kpack + it * TQ_KPACK_BYTES)[wi] = w;
    }
    const long long nsc = items * 256;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nsc; i += stride) {
        const long long it = i / 256;
        const int ks = (int)(i % 256);
        const int hf = ks >> 7, tq = (ks >> 5) & 3, g = (ks >> 2) & 7, e = ks & 3;
        reinterpret_cast<float *>(kpack + it * TQ_KPACK_BYTES + kItem)[ks] =
            scale[it * 256 + tmv_col(hf, tq + 4 * (e >> 1), g + 8 * (e & 1))];
    }
}

} // namespace

cudaError_t tq_launch_repack4(const TqMatrixDev &m, cudaStream_t st) {
    if (m.bits != 4 || !m.kpack) return cudaSuccess;
    const long long items = (long long)m.tiles * m.units;
    if (items == 0) return cudaSuccess;
    const long long words = items * (kItem / 4);
    const unsigned grid = (unsigned)(words / 256 < 148 * 8 ? (words + 255) / 256 : 148 * 8);
    repack4_kernel<<<grid, 256, 0, st>>>(m.codes, m.scale, m.kpack, items);
    return cudaGetLastError();
}

// int4, one row per launch, on the tensor cores (the K-packed copy).
cudaError_t tq_launch_tmv(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                          cudaStream_t st) {
    if (mat.bits != 4 || !mat.kpack) return tq_launch_cmv(mat, x, out, M, scr, st);
    if (M <= 0 || mat.cols == 0) return cudaSuccess;
    if (mat.rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
    for (int m0 = 0; m0 < M; m0++) {
        const cudaError_t e = launch_cmv<4, 1>(mat, x + (size_t)m0 * mat.rows, out + (size_t)m0 * mat.cols, scr, st,
                                               TQ_EPI_NONE, true);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// CUDA-core matvec for M <= 2 rows per launch (more rows: consecutive 2-row launches).
cudaError_t tq_launch_cmv(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                          cudaStream_t st) {
    if (M <= 0 || mat.cols == 0) return cudaSuccess;
    if (mat.rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
    for (int m0 = 0; m0 < M; m0 += 2) {
        const int mm = M - m0 < 2 ? M - m0 : 2;
        const float *xm = x + (size_t)m0 * mat.rows;
        float *om = out + (size_t)m0 * mat.cols;
        cudaError_t e;
        if (mat.bits == 8)
            e = mm == 1 ? launch_cmv<8, 1>(mat, xm, om, scr, st, TQ_EPI_NONE) : launch_cmv<8, 2>(mat, xm, om, scr, st, TQ_EPI_NONE);
        else
            e = mm == 1 ? launch_cmv<4, 1>(mat, xm, om, scr, st, TQ_EPI_NONE) : launch_cmv<4, 2>(mat, xm, om, scr, st, TQ_EPI_NONE);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// One activation row with an epilogue (TQ_EPI_*): the decode steps' matvecs.
cudaError_t tq_launch_cmv_epi(const TqMatrixDev &mat, const float *x, float *out, const TqScratch &scr, cudaStream_t st,
                              int epi, bool tc) {
    if (epi == TQ_EPI_NONE) return tc ? tq_launch_tmv(mat, x, out, 1, scr, st) : tq_launch_cmv(mat, x, out, 1, scr, st);
    if (epi != TQ_EPI_SWIGLU || mat.bits != 4 || mat.cols % 2 || mat.rows == 0) return cudaErrorInvalidValue;
    return launch_cmv<4, 1>(mat, x, out, scr, st, epi, tc);
}
