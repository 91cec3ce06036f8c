// tq_gemv.cu — weight-only int8 / int4 matvec (M <= 8 activation rows) on the
// 5th-generation tensor cores, one launch per call.
//
// Computes out[m][j] = sum_i x[m][i] * W[i][j], the product of qmatvecCols
// (quant_simd.go:12-48) and q4matvecCols (quant4_simd.go:17-57), with exact
// integer products on tcgen05.mma.kind::i8:
//
//   * Per 64-row unit (an int4 scale group) and activation row m, x is scaled
//     by a power of two 2^e_m (exact) so |x|/2^e < 64 and split into four
//     signed 7-bit digits, x/2^e = b0 + b1/128 + b2/128^2 + b3/128^3 + r with
//     |r| <= 2^-22 (the B operand, N = 4M columns padded to 16 or 32).
//   * int8 codes are the A operand as stored (s8). An int4 code byte holds
//     column j in its low nibble and column j + N/2 in its high nibble; the
//     raw byte (u8) and the byte masked to its high nibble are two A operands
//     over the same B: D_raw = sum (lo + 16 hi) b and D_hi = sum 16 hi b, so
//     sum lo b = D_raw - D_hi and sum hi b = D_hi / 16, exactly, in int32.
//   * The epilogue rebuilds each unit's dot product in fp32:
//       int8: v = 2^e * sum_p D_p 128^-p                 (acc += v; out = acc * scale)
//       int4: v = 2^e * sum_p (S_p - 8 sum_i b_p,i) 128^-p (acc = fma(v, scale_g, acc))
//     the int4 group fold of quant4_simd.go:46-50 (nibble n encodes n - 8).
//
// Schedule. Codes sit in HBM as 8 KB items (64 rows x 128 code bytes, the
// UMMA 128-byte-swizzled MN-major operand layout), tile-major. One persistent
// CTA per SM takes an equal contiguous slice of the item list (stream-K,
// balanced to +-1 item), walked as batches of up to NU consecutive units of one
// column tile. Nothing that depends on x happens before griddepcontrol.wait,
// and everything else does: the code ring (up to 160 KB per SM) fills and the
// int4 high-nibble copies of the first batches are made while the previous
// kernel on the stream is still finishing. Warp roles (11 warps):
//   warp 0      producer: one bulk copy per batch into the code ring
//   warp 1      owns the tensor memory; lane 0 issues the MMAs, one commit per batch
//   warps 2-5   prep: digit planes and digit sums of the batch's units from x
//               (loaded a batch ahead), int4 high-nibble operand copies
//   warps 6-9   epilogue: tcgen05.ld of the accumulators, fold into the tile
//               segment's fp32 sums, output
//   warp 10     fixup: publishes the first tile segment's partial sums when
//               that tile is shared with earlier CTAs, off the epilogue's path
// A column tile shared by several CTAs is reduced through scratch partials:
// each contributor stores its sums, fences and counts itself in with an
// acq_rel atomic; the last to arrive adds all partials in CTA order, so results
// are bit-reproducible run to run.
// Every mbarrier wait is bounded (tqp::kWaitNs); a timeout sets
// TQ_STATUS_TIMEOUT and a CTA-wide abort flag that turns all later waits into
// no-ops, so a fault ends the kernel instead of hanging it.
#include "tq_ptx.cuh"

namespace {

using namespace tqp;

constexpr int kItem = TQ_ITEM_BYTES; // 8192
constexpr int kRows = TQ_GROUP;      // 64
constexpr int kCols = TQ_TILE_BYTES; // 128
constexpr int kPrepWarp0 = 2;
constexpr int kPrepThreads = 128;
constexpr int kEpiWarp0 = 6;
constexpr int kEpiThreads = 128;
constexpr int kFixWarp = 10;
constexpr int kThreads = 11 * 32;
constexpr int kBarPrep = 1, kBarEpi = 2, kBarFix = 3; // named barrier ids

template <int M> struct Planes {
    static constexpr int N = 4 * M <= 16 ? 16 : 32; // UMMA N: digit planes, padded
    static constexpr int KSTEP_B = (N / 8) * 256;   // B bytes per 32-row MMA step
    static constexpr int BB = 2 * KSTEP_B;          // B bytes per unit
    static constexpr int MB = (M * 20 + 15) / 16 * 16; // meta bytes per unit: 2^e[M] floats, digit sums[4M] ints
};

template <int BITS, int M> struct Cfg {
    using PL = Planes<M>;
    static constexpr int N = PL::N, BB = PL::BB, MB = PL::MB, KSTEP_B = PL::KSTEP_B;
    static constexpr int NU = BITS == 8 ? 4 : 2;  // units per batch
    static constexpr int H = BITS == 8 ? 1 : 2;   // A operands per unit (int4: raw, high nibbles)
    static constexpr int ACC = H * N;             // TMEM columns per unit
    static constexpr int BACC = NU * ACC;         // per batch
    static constexpr int NB = 4;                  // accumulator buffers
    static constexpr int TCOLS = NB * BACC <= 256 ? 256 : 512;
    static constexpr int SL = H * M * kCols;      // partial floats of one tile segment
    // operand stage: [high-nibble codes NU x 8 KB (int4) | B planes NU x BB]
    static constexpr int AH = BITS == 4 ? NU * kItem : 0;
    static constexpr int OSTR = (AH + NU * BB + 1023) & ~1023;
    static constexpr int OS = BITS == 4 ? 3 : 4;
    static constexpr int CSTR = NU * kItem; // code stage
    static constexpr int MR = 8;            // meta ring
    static constexpr int META = MR * NU * MB;
    static constexpr int HAND = SL * 4;     // epilogue -> fixup warp hand-off
    static constexpr int XR = 4;            // x staging ring (prep), XR - 1 batches ahead
    static constexpr int XSLOT = NU * M * kRows * 4;
    static constexpr int SR = BITS == 4 ? 4 : 1; // int4 scale ring (epilogue), SR - 1 batches ahead
    static constexpr int SSLOT = NU * 2 * kCols * 4;
    static constexpr int XS = XR * XSLOT + SR * SSLOT;
    static constexpr int FIXED = OS * OSTR + META + HAND + XS + 1024;
    static constexpr int BUDGET = 227 * 1024 - 1024 - FIXED;
    static constexpr int CS = BUDGET / CSTR < 12 ? BUDGET / CSTR : 12; // code stages
    static constexpr int DR = (CS > NB ? CS : NB) + 2;                 // done ring
    static constexpr int O_OFF = 0;
    static constexpr int C_OFF = OS * OSTR;
    static constexpr int META_OFF = C_OFF + CS * CSTR;
    static constexpr int HAND_OFF = META_OFF + META;
    static constexpr int X_OFF = HAND_OFF + HAND;
    static constexpr int S_OFF = X_OFF + XR * XSLOT;
    static constexpr int BAR_OFF = (S_OFF + SR * SSLOT + 15) & ~15;
    static constexpr int NBARS = CS + OS + DR + NB + 2 * MR + 1;
    static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
    static constexpr int SMEM = MISC_OFF + 32 + 1024; // + alignment slack of the 1024-aligned base
    static_assert(NB * BACC <= TCOLS && TCOLS <= 512, "accumulators must fit tensor memory");
    static_assert(CS >= 4, "too few code stages");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct GvParams {
    const uint8_t *codes;
    const float *scale;
    const float *x;
    float *out;
    float *partial;
    unsigned *counters;
    unsigned *status;
    long long items;
    int rows, cols, half, units, tiles;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void named_arrive(int id, int n) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// 4-byte global -> shared async copy; src_size 0 writes a zero.
__device__ __forceinline__ void cp_async_f32(float *dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void umma_i8(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// Instruction descriptor of tcgen05.mma.kind::i8: D s32; A = codes (s8 for
// int8, u8 for int4), MN-major; B = digits, s8, K-major; M = 128; N.
template <int BITS, int N> __device__ __forceinline__ uint32_t idesc_i8() {
    return (2u << 4) | ((BITS == 8 ? 1u : 0u) << 7) | (1u << 10) | (1u << 15) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// The batch sequence of one CTA: up to NU consecutive units of one tile.
struct BatchWalk {
    int tile, unit, left, units;
    __device__ __forceinline__ int next(int NU) const { // units in the next batch (0 = done)
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

// Output of one finished tile: sums v[h][m] of this thread's tile column.
template <int BITS, int M>
__device__ __forceinline__ void write_tile(const GvParams &p, int tile, int col, const float (&v)[BITS == 8 ? 1 : 2][M]) {
    const int base = tile * kCols + col; // byte index in the reference row
    if (BITS == 8) {
        if (base < p.cols) {
            const float sc = __ldg(p.scale + base);
#pragma unroll
            for (int m = 0; m < M; m++) p.out[(size_t)m * p.cols + base] = v[0][m] * sc;
        }
    } else if (base < p.half) {
#pragma unroll
        for (int m = 0; m < M; m++) {
            p.out[(size_t)m * p.cols + base] = v[0][m];
            p.out[(size_t)m * p.cols + p.half + base] = v[1][m];
        }
    }
}

// The last CTA to arrive at a shared tile adds every contributor's partial
// sums for this thread's column in CTA order (cf first), with up to 32 loads in
// flight per thread, and writes the tile.
template <int BITS, int M>
__device__ __forceinline__ void reduce_tile(const GvParams &p, const TqSplit &split, int tile, int col) {
    constexpr int H = BITS == 8 ? 1 : 2;
    constexpr int V = H * M;
    constexpr int CH = 32 / V > 0 ? 32 / V : 1;
    constexpr int SL = V * kCols;
    const long long t0 = (long long)tile * p.units;
    const int cf = split.owner(t0), cl = split.owner(t0 + p.units - 1);
    const int slot_f = split.slot(cf, t0);
    float s[H][M];
#pragma unroll
    for (int h = 0; h < H; h++)
#pragma unroll
        for (int m = 0; m < M; m++) s[h][m] = 0.f;
    for (int cc = cf; cc <= cl; cc += CH) {
        float pv[CH][H][M];
#pragma unroll
        for (int u = 0; u < CH; u++) {
            const int c2 = cc + u;
            const float *src = p.partial + (size_t)(c2 == cf ? slot_f : 2 * c2) * SL + col;
#pragma unroll
            for (int h = 0; h < H; h++)
#pragma unroll
                for (int m = 0; m < M; m++) pv[u][h][m] = c2 <= cl ? __ldcg(src + (h * M + m) * kCols) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < CH; u++)
#pragma unroll
            for (int h = 0; h < H; h++)
#pragma unroll
                for (int m = 0; m < M; m++) s[h][m] += pv[u][h][m];
    }
    write_tile<BITS, M>(p, tile, col, s);
}

template <int BITS, int M>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(GvParams p) {
    using C = Cfg<BITS, M>;
    constexpr int CS = C::CS, OS = C::OS, DR = C::DR, NB = C::NB, NU = C::NU, H = C::H, N = C::N, MR = C::MR;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *cfull = bars, *ofull = cfull + CS, *done = ofull + OS, *accempty = done + DR;
    uint64_t *mfull = accempty + NB, *mempty = mfull + MR, *hand_full = mempty + MR;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::MISC_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 4);
    volatile int *lastflag = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 8);
    volatile int *first_last = reinterpret_cast<volatile int *>(smem + C::MISC_OFF + 12);
    auto cstage = [&](int k) { return smem + C::C_OFF + (k % CS) * C::CSTR; };
    auto ostage = [&](int k) { return smem + C::O_OFF + (k % OS) * C::OSTR; };
    auto mslot = [&](int k) { return smem + C::META_OFF + (k % MR) * NU * C::MB; };
    float *hand = reinterpret_cast<float *>(smem + C::HAND_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const TqSplit split(p.items, G);
    const long long i0 = split.start(c), i1 = split.start(c + 1);
    const BatchWalk walk0{(int)(i0 / p.units), (int)(i0 % p.units), (int)(i1 - i0), p.units};
    int nb = 0;
    {
        BatchWalk w = walk0;
        for (int n; (n = w.next(NU)) > 0; w.advance(n)) nb++;
    }
    // The first tile segment is handed to the fixup warp when it is shared and
    // is not also the slice's last segment.
    const int tile0 = walk0.tile;
    const long long ft0 = (long long)tile0 * p.units;
    const bool first_shared = split.owner(ft0) != split.owner(ft0 + p.units - 1);
    const bool handoff = first_shared && ft0 + p.units < i1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < CS; s++) mbar_init(&cfull[s], 1);
        for (int s = 0; s < OS; s++) mbar_init(&ofull[s], 1);
        for (int s = 0; s < DR; s++) mbar_init(&done[s], 1);
        for (int b = 0; b < NB; b++) mbar_init(&accempty[b], 4);
        for (int s = 0; s < MR; s++) mbar_init(&mfull[s], 1);
        for (int s = 0; s < MR; s++) mbar_init(&mempty[s], 4);
        mbar_init(hand_full, 4);
        *abort = 0;
        *first_last = 0;
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
        // ---------------- producer: codes depend on nothing ----------------
        if (lane == 0) {
            BatchWalk w = walk0;
            for (int k = 0; k < nb; k++) {
                const int n = w.next(NU);
                const long long it = (long long)w.tile * p.units + w.unit;
                w.advance(n);
                // stage k % CS last held batch k - CS
                if (k >= CS && !wait_bar(&done[(k - CS) % DR], ((k - CS) / DR) & 1, abort, p.status)) continue;
                mbar_arrive_expect_tx(&cfull[k % CS], n * kItem);
                bulk_load(cstage(k), p.codes + it * kItem, n * kItem, &cfull[k % CS]);
            }
            pdl_trigger(); // every load is issued: the next kernel may be scheduled
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_i8<BITS, N>();
            BatchWalk w = walk0;
            for (int k = 0; k < nb; k++) {
                const int n = w.next(NU);
                w.advance(n);
                const int buf = k % NB;
                bool ok = wait_bar(&ofull[k % OS], (k / OS) & 1, abort, p.status);
                ok = wait_bar(&cfull[k % CS], (k / CS) & 1, abort, p.status) && ok;
                ok = wait_bar(&accempty[buf], ((k / NB) & 1) ^ 1, abort, p.status) && ok;
                if (!ok) continue;
                tc_fence_after();
                const uint32_t asb = smem_u32(cstage(k));
                const uint32_t hsb = smem_u32(ostage(k));
                const uint32_t bsb = hsb + C::AH;
                const uint32_t d0 = tbase + (uint32_t)(buf * C::BACC);
                for (int j = 0; j < n; j++) {
#pragma unroll
                    for (int ks = 0; ks < 2; ks++) { // two 32-row K steps per unit
                        const uint64_t bd = umma_desc(bsb + j * C::BB + ks * C::KSTEP_B, 128, 256, 0);
                        umma_i8(d0 + j * C::ACC, umma_desc(asb + j * kItem + ks * 4096, kItem, 1024, 2), bd, idesc, ks);
                        if (BITS == 4)
                            umma_i8(d0 + j * C::ACC + N, umma_desc(hsb + j * kItem + ks * 4096, kItem, 1024, 2), bd,
                                    idesc, ks);
                    }
                }
                umma_commit(&done[k % DR]);
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------- prep: high-nibble copies and digit planes ----------------
        const int t = threadIdx.x - kPrepWarp0 * 32; // 0..127
        const int pw = t >> 5;                       // unit of the batch this warp plans
        // int4: operand stage k % OS gets batch k's codes masked to the high
        // nibble (position for position), made as soon as the codes landed.
        auto hi_copy = [&](int k, int n) {
            if (!wait_bar(&cfull[k % CS], (k / CS) & 1, abort, p.status)) return;
            const uint4 *src = reinterpret_cast<const uint4 *>(cstage(k));
            uint4 *dst = reinterpret_cast<uint4 *>(ostage(k));
            constexpr int PER = NU * kItem / 16 / kPrepThreads; // 8 uint4 per thread for a full batch
            uint4 v[PER];
#pragma unroll
            for (int r = 0; r < PER; r++) {
                const int q = t + r * kPrepThreads;
                v[r] = q < n * (kItem / 16) ? src[q] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int r = 0; r < PER; r++) {
                const int q = t + r * kPrepThreads;
                if (q < n * (kItem / 16))
                    dst[q] = make_uint4(v[r].x & 0xF0F0F0F0u, v[r].y & 0xF0F0F0F0u, v[r].z & 0xF0F0F0F0u,
                                        v[r].w & 0xF0F0F0F0u);
            }
        };
        BatchWalk wh = walk0; // hi-copy walker
        int kh = 0;           // next batch to copy
        if (BITS == 4) {
            for (; kh < nb && kh < OS; kh++) {
                const int n = wh.next(NU);
                hi_copy(kh, n);
                wh.advance(n);
            }
        }
        pdl_wait(); // x is produced by the previous kernel on the stream

        // x staging: slot k % XR holds batch k's [NU][M][64] floats. Unit j of
        // a batch is planned by warps j, j + NU, ... (int4: two warps per unit,
        // alternate rows m); lane l copies rows l and l + 32 of the unit for its
        // rows m (cp.async, XR - 1 batches ahead) and reads back exactly those.
        constexpr int XR = C::XR;
        constexpr int MSTEP = 4 / NU;
        const int pj = pw % NU, m0 = pw / NU;
        float *xs = reinterpret_cast<float *>(smem + C::X_OFF);
        BatchWalk wx = walk0;
        auto issue_x = [&](int kx) { // one cp.async group per batch (empty past the end)
            if (kx < nb) {
                const int n = wx.next(NU);
                if (pj < n) {
                    const int u = wx.unit + pj;
                    float *dst = xs + (size_t)((kx % XR) * NU + pj) * M * kRows;
                    for (int m = m0; m < M; m += MSTEP)
#pragma unroll
                        for (int hh = 0; hh < 2; hh++) {
                            const int row = u * kRows + hh * 32 + lane;
                            const bool v = row < p.rows;
                            cp_async_f32(dst + m * kRows + hh * 32 + lane, p.x + (size_t)m * p.rows + (v ? row : 0), v);
                        }
                }
                wx.advance(n);
            }
            cp_async_commit();
        };
        for (int kx = 0; kx < XR - 1; kx++) issue_x(kx);
        BatchWalk w = walk0;
        for (int k = 0; k < nb; k++) {
            const int n = w.next(NU);
            w.advance(n);
            issue_x(k + XR - 1); // into the slot batch k - 1 used (read by this lane already)
            cp_async_wait<XR - 1>(); // batch k's copies have landed
            bool ok = true;
            if (BITS == 8 && k >= OS) ok = wait_bar(&done[(k - OS) % DR], ((k - OS) / DR) & 1, abort, p.status);
            if (k >= MR) ok = wait_bar(&mempty[k % MR], ((k / MR) & 1) ^ 1, abort, p.status) && ok;
            if (ok && pj < n) {
                const float *xr = xs + (size_t)((k % XR) * NU + pj) * M * kRows;
                uint8_t *B = ostage(k) + C::AH + pj * C::BB;
                uint8_t *meta = mslot(k) + pj * C::MB;
                for (int m = m0; m < M; m += MSTEP) {
                    const float v0 = xr[m * kRows + lane], v1 = xr[m * kRows + 32 + lane];
                    // largest |x| of the unit: non-negative floats order like their bits
                    const unsigned amax = __reduce_max_sync(
                        0xffffffffu, max(__float_as_uint(fabsf(v0)), __float_as_uint(fabsf(v1))));
                    float r0 = 0.f, r1 = 0.f, unit_scale = 0.f;
                    if (amax != 0u) {
                        int e; // amax = f * 2^e, f in [0.5, 1)
                        const int ex = (int)(amax >> 23);
                        if (ex != 0) e = ex - 126;
                        else frexpf(__uint_as_float(amax), &e);
                        if (e >= -121) { // 2^(6 - e) is a normal float: scaling is one exact multiply
                            const float sc = __uint_as_float((uint32_t)(133 - e) << 23);
                            r0 = v0 * sc;
                            r1 = v1 * sc;
                        } else {
                            r0 = ldexpf(v0, 6 - e);
                            r1 = ldexpf(v1, 6 - e);
                        }
                        unit_scale = e >= -120 ? __uint_as_float((uint32_t)(e + 121) << 23) : ldexpf(1.0f, e - 6);
                    }
                    if (amax >= 0x7F800000u) { // a NaN or infinity: no digits; the unit's sums become NaN
                        r0 = r1 = 0.f;
                        unit_scale = __uint_as_float(0x7FC00000u);
                    }
                    // |r| < 64: four signed 7-bit digits, round to nearest even, remainder x128 (exact)
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float d0 = rintf(r0), d1 = rintf(r1);
                        r0 = (r0 - d0) * 128.0f;
                        r1 = (r1 - d1) * 128.0f;
                        const int nn = m * 4 + q;
                        // byte (n, k) of 32-row step s: s*KSTEP_B + (n/8)*256 + (k%32/16)*128 + (n%8)*16 + k%16
                        const int off = (nn >> 3) * 256 + (lane >> 4) * 128 + (nn & 7) * 16 + (lane & 15);
                        B[off] = (uint8_t)(int8_t)(int)d0;
                        B[C::KSTEP_B + off] = (uint8_t)(int8_t)(int)d1;
                        const int sum = __reduce_add_sync(0xffffffffu, (int)d0 + (int)d1);
                        if (lane == 0) reinterpret_cast<int *>(meta)[M + nn] = sum;
                    }
                    if (lane == 0) reinterpret_cast<float *>(meta)[m] = unit_scale;
                }
            }
            fence_proxy_async(); // generic-proxy writes become visible to the tensor cores
            named_sync(kBarPrep, kPrepThreads);
            if (t == 0) {
                mbar_arrive(&ofull[k % OS]);
                mbar_arrive(&mfull[k % MR]);
            }
            // int4: the high-nibble copy of batch kh = k + OS - 1 goes into the
            // stage batch k - 1 used, once that batch's MMAs are done.
            if (BITS == 4 && k >= 1 && kh < nb) {
                const int n2 = wh.next(NU);
                if (wait_bar(&done[(k - 1) % DR], ((k - 1) / DR) & 1, abort, p.status)) hi_copy(kh, n2);
                wh.advance(n2);
                kh++;
            }
        }
        cp_async_wait<0>();
    } else if (warp < kFixWarp) {
        // ---------------- epilogue ----------------
        const int q4 = warp & 3; // TMEM lane quarter of this warp
        const int col = q4 * 32 + lane;
        // int4 scales of this thread's column (both runs) for each batch, by
        // cp.async into ring slot k % SR, SR - 1 batches ahead; each thread
        // reads back only what it copied.
        float *ss = reinterpret_cast<float *>(smem + C::S_OFF);
        BatchWalk wsw = walk0;
        int ks = 0;
        auto issue_s = [&]() {
            if (BITS == 4) {
                if (ks < nb) {
                    const int n = wsw.next(NU);
                    const long long it = (long long)wsw.tile * p.units + wsw.unit;
                    float *dst = ss + (size_t)(ks % C::SR) * NU * 2 * kCols;
                    for (int j = 0; j < n; j++)
#pragma unroll
                        for (int h = 0; h < 2; h++)
                            cp_async_f32(dst + (j * 2 + h) * kCols + col, p.scale + (it + j) * (2 * kCols) + h * kCols + col,
                                         true);
                    wsw.advance(n);
                }
                cp_async_commit();
                ks++;
            }
        };
        for (int i = 0; i < C::SR - 1; i++) issue_s(); // weights: no need to wait for the previous kernel
        pdl_wait(); // the output and the scratch belong to the previous kernel until here
        const int et = threadIdx.x - kEpiWarp0 * 32;
        const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
        BatchWalk w = walk0;
        int k = 0;
        bool first_seg = true;
        while (k < nb) {
            const int tile = w.tile;
            float acc[H][M];
#pragma unroll
            for (int h = 0; h < H; h++)
#pragma unroll
                for (int m = 0; m < M; m++) acc[h][m] = 0.f;
            bool seg_end = false;
            while (!seg_end) {
                const int n = w.next(NU);
                seg_end = w.advance(n);
                const int buf = k % NB;
                float wsc[NU][H];
                if (BITS == 4) {
                    issue_s(); // batch k + SR - 1
                    cp_async_wait<C::SR - 1>();
                    const float *sb = ss + (size_t)(k % C::SR) * NU * 2 * kCols;
#pragma unroll
                    for (int j = 0; j < NU; j++)
#pragma unroll
                        for (int h = 0; h < H; h++) wsc[j][h] = j < n ? sb[(j * 2 + h) * kCols + col] : 0.f;
                }
                bool ok = wait_bar(&mfull[k % MR], (k / MR) & 1, abort, p.status);
                ok = wait_bar(&done[k % DR], (k / DR) & 1, abort, p.status) && ok;
                ok = __all_sync(0xffffffffu, ok);
                tc_fence_after();
                const uint8_t *mb = mslot(k);
#pragma unroll
                for (int j = 0; j < NU; j++) {
                    if (j >= n) break;
                    uint32_t d[H][N];
                    if (ok) {
#pragma unroll
                        for (int h = 0; h < H; h++)
#pragma unroll
                            for (int c0 = 0; c0 < N; c0 += 16)
                                tmem_ld16(lane_base + (uint32_t)(buf * C::BACC + j * C::ACC + h * N + c0),
                                          *reinterpret_cast<uint32_t(*)[16]>(&d[h][c0]));
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int h = 0; h < H; h++)
#pragma unroll
                            for (int q = 0; q < N; q++) d[h][q] = 0;
                    }
                    const float *meta = reinterpret_cast<const float *>(mb + j * C::MB);
                    const int *bsum = reinterpret_cast<const int *>(meta) + M;
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        if (BITS == 8) {
                            float v = (float)(int)d[0][m * 4 + 3];
#pragma unroll
                            for (int q = 2; q >= 0; q--) v = fmaf(v, 0.0078125f, (float)(int)d[0][m * 4 + q]);
                            acc[0][m] = fmaf(v, meta[m], acc[0][m]);
                        } else {
                            // low nibbles: D_raw - D_hi; high nibbles: D_hi / 16; codes carry +8
                            auto lo = [&](int q) { return (int)d[0][m * 4 + q] - (int)d[1][m * 4 + q] - 8 * bsum[m * 4 + q]; };
                            auto hi = [&](int q) { return ((int)d[1][m * 4 + q] >> 4) - 8 * bsum[m * 4 + q]; };
                            float vl = (float)lo(3), vh = (float)hi(3);
#pragma unroll
                            for (int q = 2; q >= 0; q--) {
                                vl = fmaf(vl, 0.0078125f, (float)lo(q));
                                vh = fmaf(vh, 0.0078125f, (float)hi(q));
                            }
                            float ws0 = 0.f, ws1 = 0.f;
#pragma unroll
                            for (int jj = 0; jj < NU; jj++)
                                if (jj == j) {
                                    ws0 = wsc[jj][0];
                                    ws1 = wsc[jj][H - 1];
                                }
                            acc[0][m] = fmaf(vl * meta[m], ws0, acc[0][m]);
                            acc[H - 1][m] = fmaf(vh * meta[m], ws1, acc[H - 1][m]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&accempty[buf]);
                    mbar_arrive(&mempty[k % MR]);
                }
                k++;
            }
            // ---- tile segment end ----
            const long long t0 = (long long)tile * p.units;
            const int cf = split.owner(t0), cl = split.owner(t0 + p.units - 1);
            if (cf == cl) {
                write_tile<BITS, M>(p, tile, col, acc);
            } else if (first_seg && handoff) {
                // shared with earlier CTAs, more segments follow: the fixup warp publishes it
#pragma unroll
                for (int h = 0; h < H; h++)
#pragma unroll
                    for (int m = 0; m < M; m++) hand[(h * M + m) * kCols + col] = acc[h][m];
                __syncwarp();
                if (lane == 0) mbar_arrive(hand_full);
            } else {
                // the slice's last segment, shared: publish, count in, reduce if last
                float *dst = p.partial + (size_t)split.slot(c, t0) * C::SL + col;
#pragma unroll
                for (int h = 0; h < H; h++)
#pragma unroll
                    for (int m = 0; m < M; m++) dst[(h * M + m) * kCols] = acc[h][m];
                __threadfence();
                named_sync(kBarEpi, kEpiThreads);
                if (et == 0) *lastflag = tq_arrive_last(&p.counters[tile], (unsigned)(cl - cf + 1));
                named_sync(kBarEpi, kEpiThreads);
                if (*lastflag) reduce_tile<BITS, M>(p, split, tile, col);
            }
            first_seg = false;
        }
        cp_async_wait<0>();
        if (handoff) {
            // the fixup warp has counted the first segment in; reduce it here if it was last
            named_sync(kBarFix, kEpiThreads + 32);
            if (*first_last) reduce_tile<BITS, M>(p, split, tile0, col);
        }
    } else {
        // ---------------- fixup: the first segment's partial sums ----------------
        if (handoff) {
            pdl_wait();
            wait_bar(hand_full, 0, abort, p.status);
            float *dst = p.partial + (size_t)split.slot(c, ft0) * C::SL;
            for (int e = lane; e < C::SL; e += 32) dst[e] = hand[e];
            __threadfence();
            __syncwarp();
            if (lane == 0) {
                const int cf = split.owner(ft0), cl = split.owner(ft0 + p.units - 1);
                *first_last = tq_arrive_last(&p.counters[tile0], (unsigned)(cl - cf + 1)) ? 1 : 0;
            }
            __syncwarp();
            named_arrive(kBarFix, kEpiThreads + 32);
        }
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
cudaError_t launch_gv(const TqMatrixDev &mat, const float *x, float *out, const TqScratch &scr, cudaStream_t st) {
    using C = Cfg<BITS, M>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static int configured[64] = {};
    static int sm_count[64] = {};
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(gemv_kernel<BITS, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    GvParams prm;
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
    prm.items = (long long)mat.tiles * mat.units;
    const int sms = sm_count[dev];
    if (mat.tiles > TQ_MAX_TILES || sms > TQ_MAX_CTAS) return cudaErrorInvalidValue;
    const int ctas = (int)(prm.items < sms ? prm.items : sms);
    // May begin before its predecessor on the stream ends (programmatic
    // dependent launch): only weight loads and their high-nibble copies run
    // before griddepcontrol.wait.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<BITS, M>, prm);
}

template <int BITS>
cudaError_t gv_dispatch(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                        cudaStream_t st) {
    switch (M) {
    case 1: return launch_gv<BITS, 1>(mat, x, out, scr, st);
    case 2: return launch_gv<BITS, 2>(mat, x, out, scr, st);
    case 3: return launch_gv<BITS, 3>(mat, x, out, scr, st);
    case 4: return launch_gv<BITS, 4>(mat, x, out, scr, st);
    case 5: return launch_gv<BITS, 5>(mat, x, out, scr, st);
    case 6: return launch_gv<BITS, 6>(mat, x, out, scr, st);
    case 7: return launch_gv<BITS, 7>(mat, x, out, scr, st);
    default: return launch_gv<BITS, 8>(mat, x, out, scr, st);
    }
}

} // namespace

// Single-launch tensor-core matvec for up to 8 activation rows (larger M in
// 8-row launches).
cudaError_t tq_launch_gemv(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                           cudaStream_t st) {
    if (M <= 0 || mat.cols == 0) return cudaSuccess;
    if (mat.rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
    for (int m0 = 0; m0 < M; m0 += 8) {
        const int mm = M - m0 < 8 ? M - m0 : 8;
        const float *xm = x + (size_t)m0 * mat.rows;
        float *om = out + (size_t)m0 * mat.cols;
        cudaError_t e =
            mat.bits == 8 ? gv_dispatch<8>(mat, xm, om, mm, scr, st) : gv_dispatch<4>(mat, xm, om, mm, scr, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
