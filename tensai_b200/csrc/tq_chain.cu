// tq_chain.cu — a chain of dependent weight-only matvecs (one activation row
// each) in ONE persistent launch: op j reads what op j - 1 wrote, as the
// decode loops call MatVec one after another (_example/qwen/model.go:196-217,
// 232-307; quant4.go:93-119 and quant.go:77-103 per call).
//
// Why: a matvec launch pays a fixed cost the weights cannot hide. The next
// launch's CTAs only become resident as this one's leave their SMs, its
// activations are only released when this grid has fully completed, and its
// cross-CTA reduction leaves HBM idle at the end. Here one CTA per SM serves
// every op of the chain:
//   * a producer warp streams the weights of op 0, op 1, ... through one
//     shared-memory ring of 8 KB items without ever waiting on data: the
//     weights of later ops land while earlier ops compute and reduce;
//   * consumer warps take op j's items once op j - 1 is complete, which they
//     learn from a device-side counter of finished column tiles (bounded
//     wait), then reduce the op exactly as the single-call kernel does
//     (tq_cmv.cu: tile segments added in warp order, tiles shared between CTAs
//     through scratch partials added in CTA order by the last CTA to arrive);
//   * whoever writes a column tile's final values bumps op j's counter.
// Ops therefore run strictly in order (op j starts reading its input only
// after op j - 1 wrote all of its output), so any aliasing between inputs and
// outputs behaves as it would with one launch per op.
//
// Per op, fused into the loads and the final write:
//   * prologue (norm_w set): x is replaced by float32(float64(x) * inv) * w,
//     inv = 1 / sqrt(sum(x^2) / n + eps), the RMSNorm of
//     _example/qwen/model.go:182-193, sum(x^2) added in float64 from the
//     per-tile sums of squares that the op which wrote x kept;
//   * epilogue TQ_EPI_SWIGLU (int4 [gate | up]): silu(gate) * up, as tq_cmv.cu;
//   * epilogue TQ_EPI_RESID: out = resid + x W (model.go:276-278, 301-303),
//     keeping the tile's float64 sum of squares of what it wrote when a later
//     op normalises it.
// int4 ops multiply on the tensor cores (mma.sync over the K-packed copy,
// tmv_item), int8 ops on the CUDA cores (half_item); a chain is one or the
// other.
//
// Counters: op j's tile counter, and the chain's exit counter, are zeroed by
// the last CTA to leave, so every launch starts from zero. Every wait is
// bounded (tqp::kWaitNs): a timeout sets TQ_STATUS_TIMEOUT and a chain-wide
// abort word that turns every other CTA's waits into no-ops; the last CTA to
// leave then clears the tile-arrival counters a broken launch may have left.
#include <cstring>
#include <mutex>
#include <vector>

#include "tq_internal.h"
#include "tq_items.cuh"

namespace {

using namespace tqi;

constexpr int CW = 8;          // consumer warps
constexpr int CWI = CW / 2;    // item streams: warps 2i and 2i + 1 take the two halves (TC: column halves) of an item
constexpr int kChainThreads = (CW + 2) * 32; // producer warp, consumers, reducer warp
constexpr int kChainSmemCap = 226 * 1024;
constexpr int kUp = 4 * 32; // SwiGLU: entry e (gate) pairs with entry e + kUp (up)
// Activations staged per op and CTA: the 64-row groups its slice touches, at
// most TQ_CHAIN_MAX_GROUPS of them, 256 bytes each (int4: their digits in place).
constexpr int XU = TQ_CHAIN_MAX_GROUPS;

struct ChainOp {
    const uint8_t *codes; // int4: the K-packed items (codes and scales); int8: the tiled codes
    const float *scale;   // int8: per-column scales
    const float *x;       // rows floats, 16-byte aligned
    float *out;
    const float *resid;   // TQ_EPI_RESID
    const float *norm_w;  // non-null: RMSNorm prologue
    const double *norm_ss; // per-tile sums of squares of x (norm_nss of them)
    double *ss_out;       // non-null: keep the per-tile sums of squares of out
    double eps;
    long long items;
    int rows, cols, half, units, tiles, ctas;
    int epi, norm_nss;
};

struct ChainParams {
    const ChainOp *ops;
    int nops;
    unsigned *done;   // [nops] finished column tiles per op
    unsigned *ctl;    // [0] CTAs that left, [1] abort word
    float *partial;   // stream scratch: tile partials
    unsigned *counters; // stream scratch: tile arrival counters
    unsigned *status;
};

template <int BITS> struct ChCfg {
    static constexpr bool TC = BITS == 4;
    static constexpr int NP = BITS == 8 ? 4 : 8; // sums per lane
    static constexpr int E = NP * 32;            // sums of a tile segment
    // A ring slot holds G consecutive items of a slice, moved by ONE bulk copy:
    // a copy has a fixed cost per SM of about 0.4 us whatever its size, so one
    // thread issuing 8 KB copies streams about 3.2 TB/s over 148 SMs, 16 KB
    // copies 6.2 TB/s and 32 KB copies 7.0 TB/s (measured on B200).
    static constexpr int ITEMB = TC ? TQ_KPACK_BYTES : kItem; // int4: codes and scales of a K-packed item
    static constexpr int G = TC ? 2 : 4;
    static constexpr int SLOT = G * ITEMB;
    static constexpr int XS = XU * 256;          // staged activation groups
    static constexpr int RED = 2 * CW * E * 4;   // two deposit buffers
    static constexpr int HAND = E * 4;           // the first segment, handed to the reducer warp
    static constexpr int FIXED = XS + RED + HAND + 2048;
    static constexpr int R0 = (kChainSmemCap - FIXED) / SLOT;
    static constexpr int R = R0 < 24 ? R0 : 24;
    static constexpr int RING_OFF = 0;
    static constexpr int XS_OFF = R * SLOT;
    static constexpr int RED_OFF = XS_OFF + XS;
    static constexpr int HAND_OFF = RED_OFF + RED;
    static constexpr int BAR_OFF = HAND_OFF + HAND;     // full[R], empty[R], hand_full, hand_empty
    static constexpr int SSR_OFF = BAR_OFF + (2 * R + 2) * 8; // CW doubles
    static constexpr int MISC_OFF = SSR_OFF + CW * 8;
    static constexpr int SMEM = MISC_OFF + 64;
    static_assert(R >= 4, "ring too shallow");
    static_assert(SMEM <= kChainSmemCap, "shared memory budget");
    static_assert(E <= CW * 32, "one entry per consumer thread");
};

__device__ __forceinline__ unsigned ld_relaxed(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(unsigned *p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// 16-byte global -> shared copy through L2 only (the source may have been
// written by another SM during this launch); bytes < 16 zero-fill the rest.
__device__ __forceinline__ void cp_async16_cg(void *dst, const void *src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sets the abort state after a timeout (or on seeing another CTA's).
__device__ __forceinline__ void chain_abort(const ChainParams &p, volatile int *abort, bool timed_out) {
    if (timed_out) {
        atomicOr(p.status, TQ_STATUS_TIMEOUT);
        st_relaxed(p.ctl + 1, 1u);
    }
    *abort = 1;
}

// Bounded wait until *cnt >= target, then acquire. One thread.
__device__ void wait_count(const ChainParams &p, const unsigned *cnt, unsigned target, volatile int *abort) {
    if (ld_relaxed(cnt) < target) {
        const unsigned long long t0 = global_ns();
        while (ld_relaxed(cnt) < target) {
            if (*abort || ld_relaxed(p.ctl + 1)) {
                chain_abort(p, abort, false);
                return;
            }
            if (global_ns() - t0 > kWaitNs) {
                chain_abort(p, abort, true);
                return;
            }
        }
    }
    fence_gpu(); // acquire: the writers' tiles before this CTA's loads
}

// Output column of sum j of lane `lane` in tile `tile` (int4: -1 beyond the pairs).
template <int BITS> __device__ __forceinline__ int out_col(const ChainOp &op, int tile, int lane, int j) {
    if (BITS == 8) {
        const int col = tile * kCols + 4 * lane + j;
        return col < op.cols ? col : -1;
    }
    const int e = j & 3, hi = j >> 2;
    const int pair = tile * kCols + 4 * lane + e;
    if (pair >= op.half) return -1;
    return hi ? op.half + pair : pair;
}

// The final value of sum j of a lane, written with the op's epilogue; returns
// what was written, for the tile's sum of squares.
template <int BITS> __device__ __forceinline__ float put(const ChainOp &op, int col, float v) {
    if (BITS == 8) v = __fmul_rn(v, __ldg(op.scale + col)); // acc_j * scale_j (quant.go:120)
    if (op.epi == TQ_EPI_RESID) v = __fadd_rn(__ldcg(op.resid + col), v);
    op.out[col] = v;
    return v;
}

// A finished tile held by one warp (lane: its NP sums): written, its sum of
// squares kept, and the op's tile counter bumped.
template <int BITS>
__device__ void finish_tile_warp(const ChainOp &op, unsigned *done, int tile, int lane, const float (&v)[BITS == 8 ? 4 : 8]) {
    constexpr int NP = BITS == 8 ? 4 : 8;
    double ss = 0.0;
    if (BITS == 4 && op.epi == TQ_EPI_SWIGLU) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int c = tile * kCols + 4 * lane + e;
            if (c < op.half) op.out[c] = swiglu(v[e], v[4 + e]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < NP; j++) {
            const int col = out_col<BITS>(op, tile, lane, j);
            if (col >= 0) {
                const float w = put<BITS>(op, col, v[j]);
                ss = __dadd_rn(ss, __dmul_rn((double)w, (double)w));
            }
        }
    }
    if (op.ss_out) {
        ss = warp_sum_d(ss);
        if (lane == 0) op.ss_out[tile] = ss;
    }
    // the warp's stores, then one cumulative release of the tile count
    __syncwarp();
    if (lane == 0) red_release(done, 1u);
}

// A tile shared with other CTAs, by one warp: publish this CTA's sums, count
// in, and if last add every contributor in CTA order and finish the tile.
template <int BITS>
__device__ void publish_shared_warp(const ChainOp &op, const ChainParams &p, unsigned *done, const TqSplit &split,
                                    int c, int tile, int lane, const float (&v)[BITS == 8 ? 4 : 8]) {
    constexpr int NP = BITS == 8 ? 4 : 8;
    constexpr int E = NP * 32;
    const long long t0 = (long long)tile * op.units;
    const int cf = split.owner(t0), cl = split.owner(t0 + op.units - 1);
    float *dst = p.partial + (size_t)split.slot(c, t0) * E + lane;
#pragma unroll
    for (int j = 0; j < NP; j++) dst[j * 32] = v[j];
    __syncwarp();
    int last = 0;
    if (lane == 0) last = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1)) ? 1 : 0;
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) return;
    const int slot_f = split.slot(cf, t0);
    float s[NP];
#pragma unroll
    for (int j = 0; j < NP; j++) s[j] = 0.f;
    constexpr int CH = 32 / NP; // contributors per round of loads
    for (int cc = cf; cc <= cl; cc += CH) {
        float pv[CH][NP];
#pragma unroll
        for (int u = 0; u < CH; u++) {
            const int c2 = cc + u;
            const float *src = p.partial + (size_t)(c2 == cf ? slot_f : 2 * c2) * E + lane;
#pragma unroll
            for (int j = 0; j < NP; j++) pv[u][j] = c2 <= cl ? __ldcg(src + j * 32) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < CH; u++)
#pragma unroll
            for (int j = 0; j < NP; j++) s[j] += pv[u][j];
    }
    finish_tile_warp<BITS>(op, done, tile, lane, s);
}

// Entry e = q * 32 + l of a finished tile, by the consumer thread holding it
// (u: the up partner's sum for SwiGLU gate entries). Returns the written value
// (0 if none) for the tile's sum of squares.
template <int BITS> __device__ __forceinline__ float put_entry(const ChainOp &op, int tile, int e, float v, float u) {
    const int l = e & 31, q = e >> 5;
    if (BITS == 4 && op.epi == TQ_EPI_SWIGLU) {
        const int cg = tile * kCols + 4 * l + q;
        if (q < 4 && cg < op.half) op.out[cg] = swiglu(v, u);
        return 0.f;
    }
    const int col = out_col<BITS>(op, tile, l, q);
    return col >= 0 ? put<BITS>(op, col, v) : 0.f;
}

// Where a CTA's slice of op j lies: items [i0, i1) of the tile-major list,
// tile segments, and whether its first segment (a tile shared with earlier
// CTAs, when the slice goes on past it) is handed to the reducer warp.
struct Slice {
    long long i0, i1;
    int nitems, tile0, nseg;
    bool handoff;
    __device__ __forceinline__ Slice(const TqSplit &split, int c, int units) {
        i0 = split.start(c);
        i1 = split.start(c + 1);
        nitems = (int)(i1 - i0);
        tile0 = (int)(i0 / units);
        nseg = (int)((i1 - 1) / units) - tile0 + 1;
        const long long t0 = (long long)tile0 * units;
        handoff = nseg > 1 && split.owner(t0) != split.owner(t0 + units - 1);
    }
};

template <int BITS>
__global__ void __launch_bounds__(kChainThreads, 1) chain_kernel(ChainParams p) {
    using C = ChCfg<BITS>;
    constexpr bool TC = C::TC;
    constexpr int R = C::R, NP = C::NP, E = C::E;
    extern __shared__ __align__(16) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + R;
    uint64_t *hand_full = empty + R, *hand_empty = hand_full + 1;
    double *ssred = reinterpret_cast<double *>(smem + C::SSR_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF);
    int *cnt = reinterpret_cast<int *>(smem + C::MISC_OFF + 8);                    // [2] deposits per buffer
    volatile int *ready = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 16); // [2] next segment a buffer takes
    // Items issued by the producer so far (a running count over the chain's
    // ops). Consumers take items out of ring order, so before the parity wait
    // for item k they check that k was issued: the producer issues k only after
    // k - R was consumed, so the barrier cannot still be two phases behind.
    volatile int *issued = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 24);
    volatile int *lastflag = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 28);
    double *inv_s = reinterpret_cast<double *>(smem + C::MISC_OFF + 32);
    float *red = reinterpret_cast<float *>(smem + C::RED_OFF);
    float *hand = reinterpret_cast<float *>(smem + C::HAND_OFF);
    uint8_t *xs = smem + C::XS_OFF; // staged groups, 256 bytes each

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < R; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2 * C::G); // both halves of each item consumed
        }
        mbar_init(hand_full, 1);
        mbar_init(hand_empty, 1);
        *abort = 0;
        *issued = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer: weights depend on nothing ----------------
        if (lane == 0) {
            pdl_trigger(); // the next kernel on the stream may be scheduled; it waits for this grid
            int seq = 0;
            bool stop = false;
            for (int j = 0; j < p.nops && !stop; j++) {
                const ChainOp *op = p.ops + j;
                const int ctas = op->ctas;
                if (c >= ctas) continue;
                const TqSplit split(op->items, ctas);
                const long long i0 = split.start(c), i1 = split.start(c + 1);
                const uint8_t *codes = op->codes;
                for (long long it = i0; it < i1; it += C::G, seq++) { // one group of up to G items per slot
                    const int s = seq % R;
                    if (seq >= R && !wait_bar(&empty[s], ((seq / R) & 1) ^ 1, abort, p.status)) {
                        stop = true;
                        break;
                    }
                    if (*abort) {
                        stop = true;
                        break;
                    }
                    const uint32_t bytes = (uint32_t)(i1 - it < C::G ? i1 - it : C::G) * C::ITEMB;
                    uint8_t *dst = smem + C::RING_OFF + s * C::SLOT;
                    mbar_arrive_expect_tx(&full[s], bytes);
                    bulk_load(dst, codes + it * C::ITEMB, bytes, &full[s]);
                    *issued = seq + 1;
                }
            }
            // No copy may still be landing in shared memory when the CTA
            // leaves: wait (bounded, whatever the abort state) for the last
            // issue of every slot. Normally the consumers have already.
            const int n = *issued;
            const unsigned long long t0 = global_ns();
            for (int k = n - R > 0 ? n - R : 0; k < n; k++)
                while (!mbar_try_wait_hint(&full[k % R], (k / R) & 1, 100000u))
                    if (global_ns() - t0 > kWaitNs) break;
        }
    } else if (warp == CW + 1) {
        // ---------------- reducer: a shared first segment, off the consumers' path ----------------
        pdl_wait(); // it may write op 0's outputs, which the previous kernel owns until here
        int nh = 0;
        for (int j = 0; j < p.nops; j++) {
            const ChainOp &op = p.ops[j];
            if (c >= op.ctas) continue;
            const TqSplit split(op.items, op.ctas);
            const Slice sl(split, c, op.units);
            if (!sl.handoff) continue;
            const bool ok = wait_bar(hand_full, nh & 1, abort, p.status);
            float v[NP];
#pragma unroll
            for (int q = 0; q < NP; q++) v[q] = hand[q * 32 + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(hand_empty);
            nh++;
            if (ok) publish_shared_warp<BITS>(op, p, p.done + j, split, c, sl.tile0, lane, v);
        }
    } else {
        // ---------------- consumers ----------------
        const int cw = warp - 1, ct = threadIdx.x - 32;
        const int hf = cw & 1, jsub = cw >> 1;
        const uint32_t mg = 0x4B000000u;
        const uint8_t *ring = smem + C::RING_OFF;
        int seq_base = 0; // sequence number of the ring group holding this CTA's first item of op j
        int nh = 0;       // first segments handed to the reducer so far
        unsigned prev_tiles = 0;
        for (int j = 0; j < p.nops; j++) {
            const ChainOp &op = p.ops[j];
            unsigned *done = p.done + j;
            // ---- op boundary: the previous op's bookkeeping is over ----
            named_sync(1, CW * 32);
            if (ct == 0) {
                cnt[0] = cnt[1] = 0;
                ready[0] = 0;
                ready[1] = 1;
            }
            if (j == 0) {
                pdl_wait(); // x and out belong to the previous kernel until here
            } else if (ct == 0) {
                wait_count(p, p.done + j - 1, prev_tiles, abort); // op j - 1 wrote all of its tiles
            }
            const bool norm = op.norm_w != nullptr;
            if (norm && ct == 0) {
                double ss = 0.0;
                for (int t = 0; t < op.norm_nss; t++) ss = __dadd_rn(ss, __ldcg(op.norm_ss + t));
                *inv_s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)op.rows), op.eps)));
            }
            named_sync(1, CW * 32);
            prev_tiles = (unsigned)op.tiles;
            const int ctas = op.ctas;
            if (c >= ctas) continue;
            const int units = op.units;
            const TqSplit split(op.items, ctas);
            const Slice sl(split, c, units);
            const long long i0 = sl.i0;
            const int nitems = sl.nitems, tile0 = sl.tile0, nseg = sl.nseg;
            auto seg_begin = [&](int s) { return s == 0 ? 0 : (int)((long long)(tile0 + s) * units - i0); };
            const int last_tile = tile0 + nseg - 1;
            const long long lt0 = (long long)last_tile * units;
            const int last_cf = split.owner(lt0), last_cl = split.owner(lt0 + units - 1);
            const int last_slot = split.slot(c, lt0);

            // ---- the slice's activations, all at once: groups u0, u0 + 1, ...
            // (mod units) into slots 0.. (item jj's group is slot jj % units) ----
            const int u0 = (int)(i0 % units);
            const int ngroups = nitems < units ? nitems : units; // <= XU (checked when the chain was built)
            for (int ci = ct; ci < ngroups * 16; ci += CW * 32) {
                const int k = ci >> 4, ch = ci & 15;
                int unit = u0 + k;
                if (unit >= units) unit -= units;
                const int r0 = unit * kRows + 4 * ch;
                const int nv = op.rows - r0;
                const int bytes = nv >= 4 ? 16 : nv > 0 ? 4 * nv : 0;
                cp_async16_cg(xs + k * 256 + 16 * ch, op.x + (bytes ? r0 : 0), bytes);
            }
            cp_async_commit();
            cp_async_wait<0>();
            if (norm) { // the same chunks, RMS-normalised in place by the thread that copied them
                const double inv = *inv_s;
                for (int ci = ct; ci < ngroups * 16; ci += CW * 32) {
                    const int k = ci >> 4, ch = ci & 15;
                    int unit = u0 + k;
                    if (unit >= units) unit -= units;
                    const int r0 = unit * kRows + 4 * ch;
                    float4 *v4 = reinterpret_cast<float4 *>(xs + k * 256 + 16 * ch);
                    float4 v = *v4;
                    float *f = reinterpret_cast<float *>(&v);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (r0 + q < op.rows)
                            f[q] = __fmul_rn((float)__dmul_rn((double)f[q], inv), __ldg(op.norm_w + r0 + q));
                    *v4 = v;
                }
            }
            named_sync(1, CW * 32);
            if constexpr (TC) { // each group's digits, once, in place
                for (int k = cw; k < ngroups; k += CW) tmv_digits_unit(xs + k * 256, lane);
                named_sync(1, CW * 32);
            }

            uint32_t ofs[8];
#pragma unroll
            for (int k = 0; k < 8; k++) ofs[k] = k * kCols + 4 * (lane ^ (k << 2));
            float acc[1][NP];
#pragma unroll
            for (int q = 0; q < NP; q++) acc[0][q] = 0.f;
            float accp[TC ? 8 : 1][2];
#pragma unroll
            for (int cb = 0; cb < (TC ? 8 : 1); cb++) accp[cb][0] = accp[cb][1] = 0.f;
            auto flush = [&]() {
                if constexpr (TC) tmv_flush(accp, acc, lane, hf);
            };

            // Deposits this warp's sums of segment s (not the slice's last);
            // the last warp to deposit reduces the segment in warp order and
            // finishes its tile, or hands a shared first segment to the
            // reducer warp.
            auto deposit = [&](int s) {
                const int sb = 2 * seg_begin(s), se = 2 * seg_begin(s + 1); // work units
                const int len = se - sb;
                const int parts = len < CW ? len : CW;
                const bool mine = len >= CW || ((cw - sb % CW + CW) % CW) < len;
                if (!mine) return;
                const int b = s & 1;
                if (ready[b] < s) { // buffer b is free once segment s - 2 was reduced
                    const unsigned long long t0 = global_ns();
                    while (ready[b] < s && !*abort)
                        if (global_ns() - t0 > kWaitNs) chain_abort(p, abort, true);
                }
                float *rb = red + (size_t)(b * CW + cw) * E + lane;
#pragma unroll
                for (int q = 0; q < NP; q++) rb[q * 32] = acc[0][q];
                __syncwarp();
                int last = 0;
                if (lane == 0) {
                    __threadfence_block();
                    last = atomicAdd(&cnt[b], 1) == parts - 1;
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) return;
                __threadfence_block();
                float v[NP];
#pragma unroll
                for (int q = 0; q < NP; q++) v[q] = 0.f;
                for (int i = 0; i < parts; i++) {
                    const int w = len >= CW ? i : (sb + i) % CW;
                    const float *src = red + (size_t)(b * CW + w) * E + lane;
#pragma unroll
                    for (int q = 0; q < NP; q++) v[q] += src[q * 32];
                }
                __syncwarp();
                if (lane == 0) {
                    cnt[b] = 0;
                    __threadfence_block();
                    ready[b] = s + 2;
                }
                if (s == 0 && sl.handoff) {
                    if (nh > 0) wait_bar(hand_empty, (nh - 1) & 1, abort, p.status); // the previous handoff was taken
#pragma unroll
                    for (int q = 0; q < NP; q++) hand[q * 32 + lane] = v[q];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(hand_full);
                } else {
                    finish_tile_warp<BITS>(op, done, tile0 + s, lane, v); // a whole tile inside the slice
                }
            };

            int s = 0;
            int next_sb = nseg > 1 ? seg_begin(1) : nitems;
            for (int jj = jsub; jj < nitems; jj += CWI) {
                while (jj >= next_sb) {
                    flush();
                    deposit(s);
#pragma unroll
                    for (int q = 0; q < NP; q++) acc[0][q] = 0.f;
                    s++;
                    next_sb = s + 1 < nseg ? next_sb + units : nitems;
                }
                const int gi = jj / C::G;  // the item's group within the slice
                const int k = seq_base + gi; // and its ring sequence number
                if (*issued <= k) {
                    const unsigned long long t0 = global_ns();
                    while (*issued <= k && !*abort)
                        if (global_ns() - t0 > kWaitNs) chain_abort(p, abort, true);
                }
                const int slot = k % R;
                const bool ok = wait_bar(&full[slot], (k / R) & 1, abort, p.status);
                const uint8_t *item = ring + slot * C::SLOT + (jj - gi * C::G) * C::ITEMB;
                const uint8_t *grp = xs + (jj % units) * 256;
                if constexpr (TC) {
                    if (ok) tmv_item_pre(item, hf, grp, lane, accp);
                } else {
                    if (ok) half_item<BITS, 1>(item, hf, reinterpret_cast<const float *>(grp) + hf * kHalf, ofs, mg, lane, acc);
                }
                __syncwarp();
                if (lane == 0) {
                    // a group short of G items (a slice's last) is completed by
                    // its first item's first half for the missing items
                    const int geff = nitems - gi * C::G < C::G ? nitems - gi * C::G : C::G;
                    const int n = (jj == gi * C::G && hf == 0) ? 1 + 2 * (C::G - geff) : 1;
                    mbar_arrive_cnt(&empty[slot], n);
                }
            }
            flush();
            for (; s < nseg - 1; s++) {
                deposit(s);
#pragma unroll
                for (int q = 0; q < NP; q++) acc[0][q] = 0.f;
            }
            if (sl.handoff) nh++;
            // ---- the slice's last segment, by all consumer threads ----
            {
                const int sg = nseg - 1, b = sg & 1;
                if (ready[b] < sg) {
                    const unsigned long long t0 = global_ns();
                    while (ready[b] < sg && !*abort)
                        if (global_ns() - t0 > kWaitNs) chain_abort(p, abort, true);
                }
                float *rb = red + (size_t)(b * CW + cw) * E + lane;
#pragma unroll
                for (int q = 0; q < NP; q++) rb[q * 32] = acc[0][q];
                named_sync(1, CW * 32);
                const int tile = last_tile, cf = last_cf, cl = last_cl;
                const bool sw = BITS == 4 && op.epi == TQ_EPI_SWIGLU;
                auto warp_sum = [&](int e) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < CW; w++) v += red[(size_t)(b * CW + w) * E + e];
                    return v;
                };
                // the tile's sum of squares over the consumer threads in a fixed
                // order, then one cumulative release of the tile count
                auto finish_all = [&](double ss) {
                    if (op.ss_out) {
                        ss = warp_sum_d(ss);
                        if (lane == 0) ssred[cw] = ss;
                    }
                    named_sync(1, CW * 32);
                    if (ct == 0) {
                        if (op.ss_out) {
                            double t = 0.0;
                            for (int w = 0; w < CW; w++) t = __dadd_rn(t, ssred[w]);
                            op.ss_out[tile] = t;
                        }
                        red_release(done, 1u);
                    }
                };
                const int e = ct;
                if (cf == cl) {
                    double ss = 0.0;
                    if (e < E && !(sw && e >= kUp)) {
                        const float w = put_entry<BITS>(op, tile, e, warp_sum(e), sw ? warp_sum(e + kUp) : 0.f);
                        ss = __dmul_rn((double)w, (double)w);
                    }
                    finish_all(ss);
                } else {
                    float *part = p.partial + (size_t)last_slot * E;
                    if (e < E) part[e] = warp_sum(e);
                    // the barrier orders every thread's partial stores before
                    // thread 0's cumulative acq_rel arrival; for the last CTA
                    // its acquire, then the second barrier, orders the other
                    // CTAs' partials before every thread's loads
                    named_sync(1, CW * 32);
                    if (ct == 0) *lastflag = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1)) ? 1 : 0;
                    named_sync(1, CW * 32);
                    if (*lastflag) {
                        const long long t0 = (long long)tile * units;
                        const int slot_f = split.slot(cf, t0);
                        auto sum_entry = [&](int en) {
                            constexpr int CH = 16; // contributor loads in flight per thread
                            float v = 0.f;
                            for (int cc = cf; cc <= cl; cc += CH) {
                                float pv[CH];
#pragma unroll
                                for (int u = 0; u < CH; u++) {
                                    const int c2 = cc + u;
                                    pv[u] = c2 <= cl ? __ldcg(p.partial + (size_t)(c2 == cf ? slot_f : 2 * c2) * E + en) : 0.f;
                                }
#pragma unroll
                                for (int u = 0; u < CH; u++) v += pv[u];
                            }
                            return v;
                        };
                        double ss = 0.0;
                        if (e < E && !(sw && e >= kUp)) {
                            const float w = put_entry<BITS>(op, tile, e, sum_entry(e), sw ? sum_entry(e + kUp) : 0.f);
                            ss = __dmul_rn((double)w, (double)w);
                        }
                        finish_all(ss);
                    }
                }
            }
            seq_base += (nitems + C::G - 1) / C::G;
        }
    }
    __syncthreads();
    // ---- exit: the last CTA to leave re-arms the chain's counters ----
    if (threadIdx.x == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.ctl) : "memory");
        if (prev == gridDim.x - 1) {
            for (int j = 0; j < p.nops; j++) st_relaxed(p.done + j, 0u);
            if (ld_relaxed(p.ctl + 1)) { // a broken launch: tile counters may be mid-count
                for (int t = 0; t < TQ_MAX_TILES; t++) st_relaxed(p.counters + t, 0u);
                st_relaxed(p.ctl + 1, 0u);
            }
            st_relaxed(p.ctl, 0u);
        }
    }
}

} // namespace

// ---- host side ------------------------------------------------------------------

// 64-row groups the busiest CTA's slice of m touches (one CTA per SM, at most
// one per item): what the kernel stages per op.
static int chain_groups(const TqMatrixDev &m, int sms) {
    const long long items = (long long)m.tiles * m.units;
    const long long ctas = items < sms ? items : sms;
    const long long per = (items + ctas - 1) / ctas;
    return (int)(per < m.units ? per : m.units);
}

struct TqChain {
    int device = 0;
    int bits = 0;
    int nops = 0;
    int ctas = 0;          // grid: one CTA per SM
    void *mem = nullptr;   // device: ops, done counters, ctl words, sums of squares
    ChainOp *ops = nullptr;
    unsigned *done = nullptr, *ctl = nullptr;
    TqChain4 *c4 = nullptr; // int4 chains
};

cudaError_t tq_chain_build(const TqChainSpec *spec, int n, TqChain **out, int *why, int *bad_op) {
    *out = nullptr;
    *why = TQ_CHAIN_OK;
    *bad_op = 0;
    if (n < 1 || n > TQ_CHAIN_MAX_OPS) {
        *why = TQ_CHAIN_BAD_COUNT;
        return cudaErrorInvalidValue;
    }
    int device = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess && (sms < 1 || sms > TQ_MAX_CTAS)) e = cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
    const int bits = spec[0].m->bits;
    for (int j = 0; j < n; j++)
        if (spec[j].m->bits != bits) {
            *why = TQ_CHAIN_MIXED_BITS;
            *bad_op = j;
            return cudaErrorInvalidValue;
        }
    if (bits == 4) {
        TqChain4 *c4 = nullptr;
        e = tq_chain4_build(spec, n, sms, &c4, why, bad_op);
        if (e != cudaSuccess) return e;
        TqChain *ch = new TqChain();
        ch->device = device;
        ch->bits = 4;
        ch->nops = n;
        ch->ctas = sms;
        ch->c4 = c4;
        *out = ch;
        return cudaSuccess;
    }
    for (int j = 0; j < n; j++) {
        const TqChainSpec &s = spec[j];
        const TqMatrixDev &m = *s.m;
        int bad = TQ_CHAIN_OK;
        if (m.bits != bits) bad = TQ_CHAIN_MIXED_BITS;
        else if (m.rows < 1 || m.cols < 1) bad = TQ_CHAIN_EMPTY;
        else if (bits == 4 && !m.kpack) bad = TQ_CHAIN_NO_KPACK;
        else if (!s.x || !s.out || ((uintptr_t)s.x & 15)) bad = TQ_CHAIN_X_ALIGN;
        else if (s.epi != TQ_EPI_NONE && s.epi != TQ_EPI_SWIGLU && s.epi != TQ_EPI_RESID) bad = TQ_CHAIN_EPI;
        else if (s.epi == TQ_EPI_SWIGLU && (bits != 4 || m.cols % 2)) bad = TQ_CHAIN_EPI;
        else if (s.epi == TQ_EPI_RESID && !s.resid) bad = TQ_CHAIN_EPI;
        else if (m.tiles > TQ_MAX_TILES) bad = TQ_CHAIN_TOO_WIDE;
        else if (chain_groups(m, sms) > TQ_CHAIN_MAX_GROUPS) bad = TQ_CHAIN_TOO_DEEP;
        else if (s.norm_w) {
            const int f = s.norm_from;
            if (f < 0 || f >= j || spec[f].epi != TQ_EPI_RESID || spec[f].out != s.x || spec[f].m->cols != m.rows)
                bad = TQ_CHAIN_NORM;
        }
        if (bad != TQ_CHAIN_OK) {
            *why = bad;
            *bad_op = j;
            return cudaErrorInvalidValue;
        }
    }
    TqChain *ch = new TqChain();
    ch->device = device;
    // sums of squares: one double per column tile of every op a later op normalises
    std::vector<size_t> ss_off(n, 0);
    size_t ss_doubles = 0;
    for (int j = 0; j < n; j++) {
        bool kept = false;
        for (int k = j + 1; k < n; k++) kept = kept || (spec[k].norm_w && spec[k].norm_from == j);
        if (kept) {
            ss_off[j] = ss_doubles + 1; // + 1: 0 means none
            ss_doubles += (size_t)spec[j].m->tiles;
        }
    }
    const size_t ops_b = sizeof(ChainOp) * n, cnt_b = sizeof(unsigned) * ((size_t)n + 2);
    const size_t ss_at = (ops_b + cnt_b + 255) & ~(size_t)255;
    const size_t total = ss_at + sizeof(double) * ss_doubles;
    e = tq_dev_malloc(&ch->mem, total);
    if (e != cudaSuccess) {
        delete ch;
        return e;
    }
    uint8_t *base = static_cast<uint8_t *>(ch->mem);
    ch->ops = reinterpret_cast<ChainOp *>(base);
    ch->done = reinterpret_cast<unsigned *>(base + ops_b);
    ch->ctl = ch->done + n;
    double *ss = reinterpret_cast<double *>(base + ss_at);
    std::vector<ChainOp> h(n);
    for (int j = 0; j < n; j++) {
        const TqChainSpec &s = spec[j];
        const TqMatrixDev &m = *s.m;
        ChainOp &o = h[j];
        std::memset(&o, 0, sizeof o);
        o.codes = bits == 4 ? m.kpack : m.codes;
        o.scale = bits == 4 ? nullptr : m.scale;
        o.x = s.x;
        o.out = s.out;
        o.resid = s.epi == TQ_EPI_RESID ? s.resid : nullptr;
        o.epi = s.epi;
        o.rows = m.rows;
        o.cols = m.cols;
        o.half = m.cols / 2;
        o.units = m.units;
        o.tiles = m.tiles;
        o.items = (long long)m.tiles * m.units;
        o.ctas = (int)(o.items < sms ? o.items : sms);
        o.eps = s.eps;
        if (ss_off[j]) o.ss_out = ss + (ss_off[j] - 1);
        if (s.norm_w) {
            o.norm_w = s.norm_w;
            o.norm_ss = ss + (ss_off[s.norm_from] - 1);
            o.norm_nss = spec[s.norm_from].m->tiles;
        }
    }
    ch->bits = bits;
    ch->nops = n;
    ch->ctas = sms;
    e = cudaMemcpy(ch->ops, h.data(), ops_b, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(ch->done, 0, cnt_b);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        tq_chain_destroy(ch);
        return e;
    }
    *out = ch;
    return cudaSuccess;
}

void tq_chain_destroy(TqChain *ch) {
    if (!ch) return;
    tq_chain4_destroy(ch->c4);
    if (ch->mem) cudaFree(ch->mem);
    delete ch;
}

int tq_chain_device(const TqChain *ch) { return ch->device; }

template <int BITS> static cudaError_t launch_chain(const TqChain &ch, const TqScratch &scr, cudaStream_t st) {
    using C = ChCfg<BITS>;
    static std::once_flag once[64];
    static cudaError_t set_err[64];
    if (ch.device < 0 || ch.device >= 64) return cudaErrorInvalidDevice;
    std::call_once(once[ch.device], [&]() {
        set_err[ch.device] = cudaFuncSetAttribute(chain_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (set_err[ch.device] != cudaSuccess) return set_err[ch.device];
    if ((size_t)2 * ch.ctas * C::E > TQ_SCRATCH_PARTIAL_FLOATS) return cudaErrorInvalidValue;
    ChainParams prm;
    prm.ops = ch.ops;
    prm.nops = ch.nops;
    prm.done = ch.done;
    prm.ctl = ch.ctl;
    prm.partial = scr.partial;
    prm.counters = scr.counters;
    prm.status = scr.status;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(ch.ctas);
    cfg.blockDim = dim3(kChainThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    return cudaLaunchKernelEx(&cfg, chain_kernel<BITS>, prm);
}

cudaError_t tq_chain_launch(const TqChain *ch, const TqScratch &scr, cudaStream_t st) {
    return ch->c4 ? tq_chain4_launch(ch->c4, scr.status, st) : launch_chain<8>(*ch, scr, st);
}
