// tq_mm.cu — weight-only int8 / int4 matmul for M >= 16 activation rows on
// the 5th-generation tensor cores, kind::tf32 with fp32 accumulators in
// tensor memory.
//
// out[m][j] = sum_i x[m][i] * W[i][j] with W[i][j] = code * scale: the same
// product as M calls of qmatvecCols (quant_simd.go:12-48) or q4matvecCols
// (quant4_simd.go:17-57), computed as one contraction. int8/int4 codes are
// exact in tf32; the dequantized weight code*scale (fp32, one rounding) and
// x are rounded to tf32 (round to nearest, ties away) before the MMA, so
// every product carries at most 2 x 2^-11 relative error and the sum is
// accumulated in fp32: well inside a 2e-3 relative-L2 budget. int8 codes go
// into the MMA as they are and the column scale multiplies the finished sum,
// as the reference does (quant.go:120).
//
// Mapping: the UMMA M dimension is 128 weight columns (one run of a column
// tile: int8 tiles have one run, int4 tiles two, the low-nibble columns
// j and the high-nibble columns j+N/2), N is the activation rows padded to
// NP in {16, 32, 64}, K is 8 rows of W per MMA. One 8 KB item (64 rows
// x 128 code bytes, tq_common.cuh) feeds 8 K-steps per run.
//
// Operands in shared memory, both K-major in the canonical UMMA layout with
// 128-byte swizzle (kind::tf32 with an MN-major operand returned zeros on
// B200, so the dequantizing warps transpose W while they expand it):
//   A (W^T, 128 weight columns x 64 rows per run): [K atom: 2][col group: 16]
//     blocks of 8 columns x 128 B; element (n, k) at (k/32)*16384 +
//     (n/8)*1024 + (n%8)*128 + (((k%32)/4) ^ (n%8))*16 + (k%4)*4.
//   B (x, NP rows x 64): [K atom: 2][row group: NP/8] blocks of 8 rows x
//     128 B; element (m, k) at (k/32)*NP*128 + (m/8)*1024 + (m%8)*128 +
//     (((k%32)/4) ^ (m%8))*16 + (k%4)*4.
// Descriptors: SBO = 1024 (8-row groups); K-step s (8 rows of W) starts at
// (s/4) * K-atom bytes + (s%4)*32.
//
// Schedule: one persistent CTA per SM takes an equal contiguous slice of the
// tile-major item list (stream-K). Warp roles (14 warps):
//   warp 0       producer: one bulk copy per item (codes) plus its scales
//   warp 1       owns tensor memory; lane 0 issues 8 x runs MMAs per item
//   warps 2-9    dequantize the item into A, convert x into B (tf32); two
//                groups of four warps, alternate items
//   warps 10-13  epilogue: tcgen05.ld of a finished tile segment, written to
//                the output (tile wholly inside the CTA) or to the CTA's
//                partial slot in scratch (tile shared with other CTAs)
// mm_reduce_kernel then sums the partials of every shared tile over its CTAs
// in CTA order (a fixed order: results are bit-reproducible), all SMs at
// once, so the split-K reduction runs at L2 bandwidth.
// Accumulators are double-buffered in tensor memory, so the epilogue of one
// tile segment overlaps the MMAs of the next. All waits are bounded (2 s);
// a timeout sets TQ_STATUS_TIMEOUT and the CTA drains.
#include "tq_ptx.cuh"

namespace {
using namespace tqp;

constexpr int kItem = TQ_ITEM_BYTES; // 8192
constexpr int kRows = TQ_GROUP;      // 64 rows per item
constexpr int kCols = TQ_TILE_BYTES; // 128 code bytes per item row
constexpr int kDqWarp0 = 2, kDqWarps = 8, kEpiWarp0 = kDqWarp0 + kDqWarps;
constexpr int kThreads = (kEpiWarp0 + 4) * 32;
constexpr int kDqThreads = kDqWarps * 32;

template <int BITS, int NP> struct MmCfg {
    static constexpr int H = BITS == 8 ? 1 : 2;            // runs of 128 weight columns per tile
    static constexpr int RUN = kCols * kRows * 4;          // A bytes per run: 32 KB
    static constexpr int A_BYTES = H * RUN;
    static constexpr int B_BYTES = NP * kRows * 4;         // NP rows x 64 K x 4 B
    static constexpr int OSTRIDE = A_BYTES + B_BYTES;      // multiple of 1024
    static constexpr int OS = 2;                           // operand stages
    static constexpr int SC_BYTES = BITS == 8 ? 0 : H * kCols * 4; // int4 group scales per item (1 KB)
    static constexpr int CSTRIDE = kItem + SC_BYTES;       // code stage: codes, then scales
    static constexpr int ACC = H * NP;                     // tensor-memory columns per accumulator
    static constexpr int NB = 2;                           // accumulator buffers
    static constexpr int TCOLS = NB * ACC <= 32 ? 32 : NB * ACC <= 64 ? 64 : NB * ACC <= 128 ? 128
                                : NB * ACC <= 256 ? 256 : 512;
    static constexpr int MISC_BYTES = 256;
    static constexpr int CS_FIT = (227 * 1024 - 1024 - MISC_BYTES - OS * OSTRIDE) / CSTRIDE;
    static constexpr int CS = CS_FIT < 6 ? CS_FIT : 6;     // code stages
    static constexpr int O_OFF = 0;
    static constexpr int C_OFF = OS * OSTRIDE;
    static constexpr int BAR_OFF = C_OFF + CS * CSTRIDE;
    static constexpr int SMEM = BAR_OFF + MISC_BYTES + 1024;
    static_assert(OSTRIDE % 1024 == 0, "operand stages must keep 1024-byte alignment");
    static_assert(CS >= 2, "too few code stages");
    static_assert(NB * ACC <= 512, "accumulators must fit tensor memory");
    static_assert((2 * CS + 2 * OS + 2 * NB) * 8 + 16 <= MISC_BYTES, "barrier area");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

struct MmParams {
    const uint8_t *codes;
    const float *scale;
    const float *x; // [m][rows]
    float *out;     // [m][cols]
    float *partial; // [2 * ctas][H][NP][128]
    unsigned *status;
    long long items;
    int rows, cols, half, units, tiles, m;
    int xvec; // x rows are 16-byte aligned (rows % 4 == 0, aligned base): 128-bit loads
};

// Instruction descriptor of tcgen05.mma.kind::tf32: D f32, A and B tf32
// K-major, M = 128, N.
template <int N> __device__ __forceinline__ uint32_t idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// Byte e (0..3) of w0..w3 gathered into one word, byte i taken from w_i.
__device__ __forceinline__ uint32_t gather_byte(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, int e) {
    const uint32_t sel = (uint32_t)e | ((uint32_t)(4 + e) << 4);
    return __byte_perm(__byte_perm(w0, w1, sel), __byte_perm(w2, w3, sel), 0x5410);
}

// 2^23 + byte e of t, exactly (byte placed under the exponent of 2^23).
__device__ __forceinline__ float magic_byte(uint32_t t, int e) {
    return __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7440 + e));
}

// The contributing CTAs [cf, cl] of the tile whose items are [t0, t1).
__device__ __forceinline__ void tile_ctas(const TqSplit &split, long long t0, long long t1, int &cf, int &cl) {
    cf = split.owner(t0);
    cl = split.owner(t1 - 1);
}

template <int BITS, int NP>
__global__ void __launch_bounds__(kThreads, 1) mm_kernel(MmParams p) {
    using C = MmCfg<BITS, NP>;
    constexpr int H = C::H, CS = C::CS, OS = C::OS, NB = C::NB, ACC = C::ACC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *cfull = bars, *cempty = cfull + CS, *ofull = cempty + CS, *oempty = ofull + OS, *accfull = oempty + OS,
             *accempty = accfull + NB;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accempty + NB);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    auto ostage = [&](int j) { return smem + C::O_OFF + (j % OS) * C::OSTRIDE; };
    auto cstage = [&](int j) { return smem + C::C_OFF + (j % CS) * C::CSTRIDE; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const TqSplit split(p.items, G);
    const long long i0 = split.start(c), i1 = split.start(c + 1);
    const int n = (int)(i1 - i0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < CS; s++) {
            mbar_init(&cfull[s], 1);
            mbar_init(&cempty[s], 1);
        }
        for (int s = 0; s < OS; s++) {
            mbar_init(&ofull[s], 1);
            mbar_init(&oempty[s], 1);
        }
        for (int b = 0; b < NB; b++) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], 1);
        }
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
        // ---------------- producer: codes + scales of each item ----------------
        if (lane == 0) {
            for (int j = 0; j < n; j++) {
                const long long it = i0 + j;
                if (j >= CS && !wait_bar(&cempty[j % CS], ((j / CS) - 1) & 1, abort, p.status)) continue;
                uint8_t *dst = cstage(j);
                mbar_arrive_expect_tx(&cfull[j % CS], C::CSTRIDE);
                bulk_load(dst, p.codes + it * kItem, kItem, &cfull[j % CS]);
                if (BITS == 4) bulk_load(dst + kItem, p.scale + it * (2 * kCols), C::SC_BYTES, &cfull[j % CS]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32<NP>();
            int seg = 0;
            for (int j = 0; j < n; j++) {
                const long long it = i0 + j;
                const int unit = (int)(it % p.units);
                const bool first = j == 0 || unit == 0;                     // first item of a tile segment
                const bool last = j == n - 1 || unit == p.units - 1;        // last item of a tile segment
                const int b = seg % NB;
                bool ok = true;
                if (first) ok = wait_bar(&accempty[b], ((seg / NB) & 1) ^ 1, abort, p.status);
                ok = wait_bar(&ofull[j % OS], (j / OS) & 1, abort, p.status) && ok;
                if (ok) {
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(ostage(j)), b0 = a0 + C::A_BYTES;
#pragma unroll
                    for (int h = 0; h < H; h++)
#pragma unroll
                        for (int ks = 0; ks < 8; ks++) {
                            const uint64_t ad = umma_desc(a0 + h * C::RUN + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, 2);
                            const uint64_t bd = umma_desc(b0 + (ks >> 2) * (NP * 128) + (ks & 3) * 32, 16, 1024, 2);
                            umma_tf32(tbase + (uint32_t)(b * ACC + h * NP), ad, bd, idesc, (first && ks == 0) ? 0u : 1u);
                        }
                }
                umma_commit(&oempty[j % OS]);
                if (last) {
                    umma_commit(&accfull[b]);
                    seg++;
                }
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------- dequantize A, convert B ----------------
        // Two groups of four warps take alternate items (group g: items g, g+2,
        // ...; operand stage g), so two items are being expanded at once. In a
        // group, thread t owns two blocks of rows 4kq..4kq+3 x code bytes
        // 8co..8co+7 of its items: kq = 8*(warp%2) + lane%8, co = 4*(warp/2 + 2*pass)
        // + lane/8, so the 16-byte stores of a warp (eight K-chunks x four column
        // groups) hit every bank position once per wavefront.
        static_assert(OS == 2, "one operand stage per dequantizing group");
        constexpr int GT = kDqThreads / 2; // threads per group
        const int g = (threadIdx.x - kDqWarp0 * 32) / GT;
        const int t = (threadIdx.x - kDqWarp0 * 32) % GT;
        const int dw = t >> 5, dl = t & 31;
        const int kq = 8 * (dw & 1) + (dl & 7);
        const int k0 = 4 * kq;                        // first W row of the blocks
        const int kch = (k0 & 31) >> 2;               // its 16-byte K-chunk within the 32-row atom
        const int kofs = (k0 >> 5) * 16384;           // its K atom
        // x of the group's next item is loaded one item ahead, into registers.
        constexpr int BCH = NP * 16 / GT > 0 ? NP * 16 / GT : 1; // 16-byte chunks per thread
        float xv[BCH][4];
        auto load_x = [&](int unit) {
#pragma unroll
            for (int i = 0; i < BCH; i++) {
                const int idx = i * GT + t, m = idx >> 4, kc = idx & 15;
                const int row = unit * kRows + kc * 4;
                const bool mv = idx < NP * 16 && m < p.m;
                if (p.xvec && mv && row + 3 < p.rows) {
                    const float4 v = __ldg(reinterpret_cast<const float4 *>(p.x + (size_t)m * p.rows + row));
                    xv[i][0] = v.x, xv[i][1] = v.y, xv[i][2] = v.z, xv[i][3] = v.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        xv[i][e] = (mv && row + e < p.rows) ? __ldg(p.x + (size_t)m * p.rows + row + e) : 0.f;
                }
            }
        };
        if (g < n) load_x((int)((i0 + g) % p.units));
        for (int j = g; j < n; j += 2) {
            bool ok = wait_bar(&cfull[j % CS], (j / CS) & 1, abort, p.status);
            if (j >= OS) ok = wait_bar(&oempty[j % OS], ((j / OS) - 1) & 1, abort, p.status) && ok;
            uint8_t *A = ostage(j);
            uint8_t *B = A + C::A_BYTES;
            if (ok) {
                const uint8_t *cs = cstage(j);
                const float *sc = reinterpret_cast<const float *>(cs + kItem);
#pragma unroll 1
                for (int pass = 0; pass < 2; pass++) {
                const int co = 4 * ((dw >> 1) + 2 * pass) + (dl >> 3);
                float s_lo[8], s_hi[8];
                if (BITS == 4) {
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const float4 a = reinterpret_cast<const float4 *>(sc + co * 8)[q];
                        s_lo[4 * q] = a.x, s_lo[4 * q + 1] = a.y, s_lo[4 * q + 2] = a.z, s_lo[4 * q + 3] = a.w;
                        const float4 b = reinterpret_cast<const float4 *>(sc + kCols + co * 8)[q];
                        s_hi[4 * q] = b.x, s_hi[4 * q + 1] = b.y, s_hi[4 * q + 2] = b.z, s_hi[4 * q + 3] = b.w;
                    }
                }
                // rows k0..k0+3, bytes 8co..8co+7: chunk co/2 (swizzled by row), half co%2
                uint32_t w[4][2];
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    const int k = k0 + r;
                    const uint2 v = *reinterpret_cast<const uint2 *>(cs + k * kCols + (((co >> 1) ^ (k & 7)) << 4) +
                                                                     ((co & 1) << 3));
                    w[r][0] = v.x;
                    w[r][1] = v.y;
                }
#pragma unroll
                for (int jc = 0; jc < 8; jc++) { // code byte column 8co + jc = weight column nn of each run
                    const int nn = 8 * co + jc;
                    const uint32_t g = gather_byte(w[0][jc >> 2], w[1][jc >> 2], w[2][jc >> 2], w[3][jc >> 2], jc & 3);
                    const int adr = kofs + (nn >> 3) * 1024 + (nn & 7) * 128 + ((kch ^ (nn & 7)) << 4);
                    uint4 o;
                    if (BITS == 8) {
                        // the code itself (exact in tf32); the column scale is applied to the sum
                        const uint32_t tt = g ^ 0x80808080u; // signed byte b -> b + 128
                        const float2 off = make_float2(-8388736.0f, -8388736.0f); // 2^23 + 128
                        const float2 c01 = __fadd2_rn(make_float2(magic_byte(tt, 0), magic_byte(tt, 1)), off);
                        const float2 c23 = __fadd2_rn(make_float2(magic_byte(tt, 2), magic_byte(tt, 3)), off);
                        o = make_uint4(__float_as_uint(c01.x), __float_as_uint(c01.y), __float_as_uint(c23.x),
                                       __float_as_uint(c23.y));
                        *reinterpret_cast<uint4 *>(A + adr) = o;
                    } else {
                        // (nibble - 8) * group scale, rounded to tf32
                        const uint32_t lo = g & 0x0F0F0F0Fu, hi = (g >> 4) & 0x0F0F0F0Fu;
                        const float2 off = make_float2(-8388616.0f, -8388616.0f); // 2^23 + 8
                        const float2 sl = make_float2(s_lo[jc], s_lo[jc]), sh = make_float2(s_hi[jc], s_hi[jc]);
                        float2 a = __fmul2_rn(__fadd2_rn(make_float2(magic_byte(lo, 0), magic_byte(lo, 1)), off), sl);
                        float2 b = __fmul2_rn(__fadd2_rn(make_float2(magic_byte(lo, 2), magic_byte(lo, 3)), off), sl);
                        o = make_uint4(tf32_rna_bits(a.x), tf32_rna_bits(a.y), tf32_rna_bits(b.x), tf32_rna_bits(b.y));
                        *reinterpret_cast<uint4 *>(A + adr) = o;
                        a = __fmul2_rn(__fadd2_rn(make_float2(magic_byte(hi, 0), magic_byte(hi, 1)), off), sh);
                        b = __fmul2_rn(__fadd2_rn(make_float2(magic_byte(hi, 2), magic_byte(hi, 3)), off), sh);
                        o = make_uint4(tf32_rna_bits(a.x), tf32_rna_bits(a.y), tf32_rna_bits(b.x), tf32_rna_bits(b.y));
                        *reinterpret_cast<uint4 *>(A + C::RUN + adr) = o;
                    }
                }
                } // pass
#pragma unroll
                for (int i = 0; i < BCH; i++) {
                    const int idx = i * GT + t, m = idx >> 4, kc = idx & 15;
                    if (idx < NP * 16) {
                        const int r = m & 7;
                        uint4 o;
                        o.x = tf32_rna_bits(xv[i][0]);
                        o.y = tf32_rna_bits(xv[i][1]);
                        o.z = tf32_rna_bits(xv[i][2]);
                        o.w = tf32_rna_bits(xv[i][3]);
                        *reinterpret_cast<uint4 *>(B + (kc >> 3) * (NP * 128) + (m >> 3) * 1024 + r * 128 +
                                                   (((kc & 7) ^ r) << 4)) = o;
                    }
                }
            }
            if (j + 2 < n) load_x((int)((i0 + j + 2) % p.units)); // in flight across the next item's waits
            fence_proxy_async(); // generic-proxy writes of A and B become visible to the tensor cores
            named_sync(1 + 2 * g, GT); // barriers 1 and 3 (2 is the epilogue's)
            if (t == 0) {
                mbar_arrive(&ofull[j % OS]);
                mbar_arrive(&cempty[j % CS]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int et = threadIdx.x - kEpiWarp0 * 32; // 0..127
        const int q4 = warp & 3;                     // tensor-memory lane quarter of this warp
        const int col = q4 * 32 + lane;              // weight column of this thread within a run
        const uint32_t lane_base = tbase + ((uint32_t)(q4 * 32) << 16);
        constexpr int SL = H * NP * kCols; // partial entries per tile
        int seg = 0;
        for (long long s0 = i0; s0 < i1; seg++) {
            const int tile = (int)(s0 / p.units);
            const long long t0 = (long long)tile * p.units, t1 = t0 + p.units;
            const long long s1 = t1 < i1 ? t1 : i1;
            const int b = seg % NB;
            int cf, cl;
            tile_ctas(split, t0, t1, cf, cl);
            const bool shared = cf != cl;
            const bool ok = wait_bar(&accfull[b], (seg / NB) & 1, abort, p.status);
            tc_fence_after();
            float *dst = p.partial + (size_t)split.slot(c, t0) * SL;
            const int base = tile * kCols + col; // byte column of this thread in the reference row
            // int8: sum x*code, then times the column scale (quant.go:120); shared
            // tiles are scaled after their cross-CTA sum.
            const float cscale = BITS == 8 && base < p.cols ? __ldg(p.scale + base) : 1.f;
#pragma unroll
            for (int h = 0; h < H; h++) {
                const int gcol = BITS == 8 ? base : (h == 0 ? base : p.half + base);
                const bool cvalid = BITS == 8 ? base < p.cols : base < p.half;
#pragma unroll 1
                for (int c0 = 0; c0 < NP; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(lane_base + (uint32_t)(b * ACC + h * NP + c0), v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float f = ok ? __uint_as_float(v[i]) : 0.f;
                        const int m = c0 + i;
                        if (shared)
                            dst[(h * NP + m) * kCols + col] = f;
                        else if (cvalid && m < p.m)
                            p.out[(size_t)m * p.cols + gcol] = BITS == 8 ? f * cscale : f;
                    }
                }
            }
            tc_fence_before();
            named_sync(2, 128);
            if (et == 0) mbar_arrive(&accempty[b]); // accumulator buffer b is free again
            s0 = s1;
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

// Sums the partial slots of every tile shared by several CTAs of mm_kernel,
// contributors in CTA order, and writes those output columns (int8: times the
// column scale). Block (tile, run h, rows 4z..4z+3), thread = tile column.
template <int BITS, int NP>
__global__ void __launch_bounds__(128) mm_reduce_kernel(MmParams p, int ctas) {
    constexpr int H = BITS == 8 ? 1 : 2;
    constexpr int SL = H * NP * kCols;
    constexpr int RB = 4; // rows per block
    const int tile = blockIdx.x, h = blockIdx.y, m0 = blockIdx.z * RB, col = threadIdx.x;
    const long long t0 = (long long)tile * p.units, t1 = t0 + p.units;
    int cf, cl;
    const TqSplit split(p.items, ctas);
    tile_ctas(split, t0, t1, cf, cl);
    if (cf == cl) return; // written by the tile's only CTA
    const int b = tile * kCols + col;
    if (!(BITS == 8 ? b < p.cols : b < p.half)) return;
    const float cscale = BITS == 8 ? __ldg(p.scale + b) : 1.f;
    float sum[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) sum[r] = 0.f;
    const int slot_f = split.slot(cf, t0);
    for (int c2 = cf; c2 <= cl; c2 += 8) { // contributors in CTA order, 8 x RB loads in flight
        float pv[8][RB];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int cu = c2 + u;
            const int sl = cu == cf ? slot_f : 2 * cu;
            const float *src = p.partial + (size_t)sl * SL + (size_t)(h * NP + m0) * kCols + col;
#pragma unroll
            for (int r = 0; r < RB; r++) pv[u][r] = cu <= cl && m0 + r < p.m ? __ldcg(src + r * kCols) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++)
#pragma unroll
            for (int r = 0; r < RB; r++) sum[r] += pv[u][r];
    }
    const int gcol = BITS == 8 || h == 0 ? b : p.half + b;
#pragma unroll
    for (int r = 0; r < RB; r++)
        if (m0 + r < p.m) p.out[(size_t)(m0 + r) * p.cols + gcol] = BITS == 8 ? sum[r] * cscale : sum[r];
}

template <int BITS, int NP>
cudaError_t launch_mm(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                      cudaStream_t st) {
    using C = MmCfg<BITS, NP>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static TqDeviceOnce once;
    e = tq_device_once(once, dev, [] {
        return cudaFuncSetAttribute(mm_kernel<BITS, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    });
    if (e != cudaSuccess) return e;
    MmParams prm;
    prm.codes = mat.codes;
    prm.scale = mat.scale;
    prm.x = x;
    prm.out = out;
    prm.partial = scr.mm_partial;
    prm.status = scr.status;
    prm.rows = mat.rows;
    prm.cols = mat.cols;
    prm.half = mat.cols / 2;
    prm.units = mat.units;
    prm.tiles = mat.tiles;
    prm.m = M;
    prm.xvec = (mat.rows % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    prm.items = (long long)mat.tiles * mat.units;
    const int sms = once.sms[dev];
    if (mat.tiles > TQ_MAX_TILES || sms > TQ_MAX_CTAS || !scr.mm_partial) return cudaErrorInvalidValue;
    const int ctas = (int)(prm.items < sms ? prm.items : sms);
    mm_kernel<BITS, NP><<<ctas, kThreads, C::SMEM, st>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess || ctas == 1) return e;
    mm_reduce_kernel<BITS, NP><<<dim3(mat.tiles, C::H, (M + 3) / 4), 128, 0, st>>>(prm, ctas);
    return cudaGetLastError();
}

template <int BITS>
cudaError_t mm_dispatch(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                        cudaStream_t st) {
    if (M <= 16) return launch_mm<BITS, 16>(mat, x, out, M, scr, st);
    if (M <= 32) return launch_mm<BITS, 32>(mat, x, out, M, scr, st);
    return launch_mm<BITS, 64>(mat, x, out, M, scr, st);
}

} // namespace

// out[M][cols] = x[M][rows] @ W on the tf32 tensor-core path, 64 activation
// rows per launch.
cudaError_t tq_launch_mm(const TqMatrixDev &mat, const float *x, float *out, int M, const TqScratch &scr,
                         cudaStream_t st) {
    if (M <= 0 || mat.cols == 0) return cudaSuccess;
    if (mat.rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * mat.cols, st);
    for (int m0 = 0; m0 < M; m0 += TQ_MM_MAX_ROWS) {
        const int mm = M - m0 < TQ_MM_MAX_ROWS ? M - m0 : TQ_MM_MAX_ROWS;
        const float *xm = x + (size_t)m0 * mat.rows;
        float *om = out + (size_t)m0 * mat.cols;
        cudaError_t e = mat.bits == 8 ? mm_dispatch<8>(mat, xm, om, mm, scr, st) : mm_dispatch<4>(mat, xm, om, mm, scr, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
