// tq_items.cuh — the per-item arithmetic shared by the single-call matvec
// (tq_cmv.cu) and the chained matvec (tq_chain.cu): one 8 KB item (64 rows x
// 128 code bytes, the tiled layout of tq_common.cuh) multiplied into a lane's
// column sums, on the CUDA cores (half_item) or on the tensor cores by
// mma.sync over the K-packed int4 copy (tmv_item), plus the small PTX helpers
// both kernels use.
#pragma once

#include "tq_ptx.cuh"

namespace tqi {

using namespace tqp;

constexpr int kItem = TQ_ITEM_BYTES; // 8192
constexpr int kRows = TQ_GROUP;      // 64
constexpr int kCols = TQ_TILE_BYTES; // 128
constexpr int kHalf = TQ_GROUP / 2;  // rows per half item

// silu(g) * u as the Go code forms it (model.go:296-299): silu in float64,
// the product in float32.
__device__ __forceinline__ float swiglu(float g, float u) {
    const double gd = (double)g;
    return __fmul_rn((float)__ddiv_rn(gd, __dadd_rn(1.0, exp(-gd))), u);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ void named_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// 4-byte global -> shared async copy; src_size 0 writes a zero.
__device__ __forceinline__ void cp_async_f32(float *dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// The float 2^23 + (w & mask), exact for a mask inside bits 0..22 (magic = 2^23's bits).
__device__ __forceinline__ float mag(uint32_t w, uint32_t mask, uint32_t magic) { return __uint_as_float((w & mask) | magic); }
// Byte e of t under the exponent of 2^23: the float 2^23 + byte, exact.
__device__ __forceinline__ float mag_byte(uint32_t t, int e) { return __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7440 + e)); }

// int4 column order of a lane's 8 sums: pairs (lo0, lo1), (lo2, lo3),
// (hi0, hi1), (hi2, hi3); lo e = low nibble of byte e (column pair 4l + e),
// hi e = its high nibble. The nibble at bits 4k..4k+3 carries 16^k:
//   lo0 k=0, hi0 k=1, lo1 k=2, hi1 k=3, lo2 k=4 (bits 0..19 of w), then
//   w >> 20: hi2 k=0, lo3 k=1, hi3 k=2.
__device__ __forceinline__ float pos_scale(int j) { // 16^-k of sum j (j = 0..7 in the order above)
    // lo0 lo1 lo2 lo3 hi0 hi1 hi2 hi3
    constexpr float s[8] = {1.f, 1.f / 256.f, 1.f / 65536.f, 1.f / 16.f, 1.f / 16.f, 1.f / 4096.f, 1.f, 1.f / 256.f};
    return s[j];
}

// Code rows r and r + 1 of a lane (words w0, w1) into its column sums:
// t[m][j] = (sum over even rows, sum over odd rows) of column j, packed so
// that one f32x2 FMA takes both rows against (x_r, x_r+1). int4: 8 columns in
// the order lo0 lo1 lo2 lo3 hi0 hi1 hi2 hi3; int8: 4 columns (bytes 0..3).
template <int BITS, int M>
__device__ __forceinline__ void row_pair(uint32_t w0, uint32_t w1, const float2 (&xp)[M],
                                         float2 (&t)[M][BITS == 8 ? 4 : 8], uint32_t mg) {
    if (BITS == 4) {
        const uint32_t v0 = w0 >> 20, v1 = w1 >> 20;
        float2 c[8];
        c[0] = __fadd2_rn(f2(mag(w0, 0xFu, mg), mag(w1, 0xFu, mg)), f2(-8388616.0f, -8388616.0f));          // 2^23 + n
        c[1] = __fadd2_rn(f2(mag(w0, 0xF00u, mg), mag(w1, 0xF00u, mg)), f2(-8390656.0f, -8390656.0f));      // 2^23 + 256 n
        c[2] = __fadd2_rn(f2(mag(w0, 0xF0000u, mg), mag(w1, 0xF0000u, mg)), f2(-8912896.0f, -8912896.0f));  // 2^23 + 65536 n
        c[3] = __fadd2_rn(f2(mag(v0, 0xF0u, mg), mag(v1, 0xF0u, mg)), f2(-8388736.0f, -8388736.0f));        // 2^23 + 16 n
        c[4] = __fadd2_rn(f2(mag(w0, 0xF0u, mg), mag(w1, 0xF0u, mg)), f2(-8388736.0f, -8388736.0f));        // 2^23 + 16 n
        c[5] = __fadd2_rn(f2(mag(w0, 0xF000u, mg), mag(w1, 0xF000u, mg)), f2(-8421376.0f, -8421376.0f));    // 2^23 + 4096 n
        c[6] = __fadd2_rn(f2(mag(v0, 0xFu, mg), mag(v1, 0xFu, mg)), f2(-8388616.0f, -8388616.0f));          // 2^23 + n
        c[7] = __fadd2_rn(f2(mag(v0, 0xF00u, mg), mag(v1, 0xF00u, mg)), f2(-8390656.0f, -8390656.0f));      // 2^23 + 256 n
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int j = 0; j < 8; j++) t[m][j] = __ffma2_rn(c[j], xp[m], t[m][j]);
    } else {
        const uint32_t u0 = w0 ^ 0x80808080u, u1 = w1 ^ 0x80808080u; // signed byte b -> b + 128
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float2 c = __fadd2_rn(f2(mag_byte(u0, e), mag_byte(u1, e)), f2(-8388736.0f, -8388736.0f));
#pragma unroll
            for (int m = 0; m < M; m++) t[m][e] = __ffma2_rn(c, xp[m], t[m][e]);
        }
    }
}

// One warp's half item (rows 32h..32h+31 of a 64-row item in shared memory)
// into the lane's column sums acc (int4: through the group fold).
template <int BITS, int M>
__device__ __forceinline__ void half_item(const uint8_t *item, int hf, const float *xr, const uint32_t (&ofs)[8],
                                          uint32_t mg, int lane, float (&acc)[M][BITS == 8 ? 4 : 8]) {
    constexpr int NP = BITS == 8 ? 4 : 8;
    float2 t[M][NP];
#pragma unroll
    for (int m = 0; m < M; m++)
#pragma unroll
        for (int q = 0; q < NP; q++) t[m][q] = f2(0.f, 0.f);
    // all 32 rows of the half: rows past the matrix have zero codes and zero activations
    const uint8_t *half = item + hf * kHalf * kCols;
#pragma unroll
    for (int g = 0; g < kHalf / 8; g++) {
#pragma unroll
        for (int k = 0; k < 8; k += 4) {
            const int r = 8 * g + k; // row within the half
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; i++) w[i] = *reinterpret_cast<const uint32_t *>(half + g * 8 * kCols + ofs[k + i]);
            float2 xa[M], xb[M];
#pragma unroll
            for (int m = 0; m < M; m++) {
                const float4 v = *reinterpret_cast<const float4 *>(xr + m * kHalf + r);
                xa[m] = f2(v.x, v.y);
                xb[m] = f2(v.z, v.w);
            }
            row_pair<BITS, M>(w[0], w[1], xa, t, mg);
            row_pair<BITS, M>(w[2], w[3], xb, t, mg);
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        float tmp[NP];
#pragma unroll
        for (int q = 0; q < NP; q++) tmp[q] = t[m][q].x + t[m][q].y;
        if (BITS == 4) {
            // group fold with 16^-k taken into the scale (exact)
            const float4 slo = *reinterpret_cast<const float4 *>(item + kItem + 16 * lane);
            const float4 shi = *reinterpret_cast<const float4 *>(item + kItem + 512 + 16 * lane);
            const float sc[8] = {slo.x, slo.y, slo.z, slo.w, shi.x, shi.y, shi.z, shi.w};
#pragma unroll
            for (int q = 0; q < NP; q++) acc[m][q] = fmaf(tmp[q], sc[q] * pos_scale(q), acc[m][q]);
        } else {
#pragma unroll
            for (int q = 0; q < NP; q++) acc[m][q] += tmp[q];
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-core variant (int4, one activation row): the same schedule, with each
// item's codes multiplied on the tensor cores by mma.sync m16n8k32 (u8 codes x
// s8 activation digits, exact s32 sums), which issues about four times more
// codes per SM cycle than the CUDA-core unpack above.
//
// Activations: per 64-row group, X = round(x * 2^s) with |X| <= 2^22 (s from
// the group's largest |x|), cut into three signed byte digits, X = d0 + 256 d1
// + 65536 d2 (bytes of X + 0x808080, each xor 0x80). The digits are the MMA's
// B columns n = 0, 1, 2 (n = 3..7 zero).
// Codes: a second, K-packed copy of the matrix (tq_launch_repack4): in item
// (tile, unit), warp half hf (item columns 128hf..), MMA block cb (0..7) and
// lane (g, t) = (lane / 4, lane % 4) hold 16 bytes: the words of MMA rows g and
// g + 8 for rows 8t..8t+7 and 32+8t..32+8t+7 of the group. Word (j, k) packs
// rows 8k..8k+7 of item column j, byte r = code(8k + 2r) | code(8k + 2r + 1) << 4,
// so w & 0x0F0F0F0F (even rows) and (w >> 4) & 0x0F0F0F0F (odd rows) are A
// fragments as they stand. MMA row rho of block cb is item column
//   128 hf + 4 (4 (rho % 8) + cb % 4) + 2 (cb / 4) + rho / 8,
// which puts every sum in the lane that owns it in the CUDA-core layout
// (lane l: item columns 4l + e, 128 + 4l + e), so deposits and reductions are
// shared. Scales: per item, [hf][cb % 4][g][2 (cb / 4) + rho / 8].
// Per group and block the D fragment holds, in lane t = 0, sum n*d0 and sum
// n*d1 (n the unsigned code) and in lane t = 1 sum n*d2; each lane adds
//   scale * ((D_a + 256 D_b) * K_t + O_t),  K_0 = 2^-s, K_1 = 2^(16-s),
//   O_1 = -8 * sum(X) * 2^-s (the code offset 8), K and O zero for t >= 2,
// and the four lanes of a quad are added when a tile segment is deposited.
// The integer sums are exact; |X| <= 2^22 keeps 22 bits of every group.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The MMA part of one 64-row item, item columns of half hf, into this lane's
// partial sums accp[cb][rh] (MMA rows g + 8 rh of block cb): B fragments be0,
// bo0 (digit g at the even / odd rows of the first 32-row half), be1, bo1 (the
// second half), and the lane's K and O of the group fold (see below).
__device__ __forceinline__ void tmv_mma(const uint8_t *item, int hf, uint32_t be0, uint32_t bo0, uint32_t be1,
                                        uint32_t bo1, float K, float O, int lane, float (&accp)[8][2]) {
    const int g = lane >> 2;
    const uint8_t *cw = item + hf * (kItem / 2) + lane * 16;
    const float *scl = reinterpret_cast<const float *>(item + kItem) + hf * 128 + g * 4;
    float4 sc[4];
#pragma unroll
    for (int u = 0; u < 4; u++) sc[u] = *reinterpret_cast<const float4 *>(scl + u * 32);
    constexpr uint32_t LO = 0x0F0F0F0Fu;
    // In phases over the eight blocks (all loads, all first-half MMAs, all
    // second-half MMAs, then the sums), so that eight independent chains
    // hide the shared-memory and MMA latencies of each.
    uint4 w[8];
#pragma unroll
    for (int cb = 0; cb < 8; cb++) w[cb] = *reinterpret_cast<const uint4 *>(cw + cb * 512);
    int d[8][4];
#pragma unroll
    for (int cb = 0; cb < 8; cb++) {
        d[cb][0] = d[cb][1] = d[cb][2] = d[cb][3] = 0;
        mma_u8s8(d[cb], w[cb].x & LO, w[cb].y & LO, (w[cb].x >> 4) & LO, (w[cb].y >> 4) & LO, be0, bo0);
    }
#pragma unroll
    for (int cb = 0; cb < 8; cb++)
        mma_u8s8(d[cb], w[cb].z & LO, w[cb].w & LO, (w[cb].z >> 4) & LO, (w[cb].w >> 4) & LO, be1, bo1);
#pragma unroll
    for (int cb = 0; cb < 8; cb++) {
        const float vg = fmaf((float)(d[cb][0] + (d[cb][1] << 8)), K, O);
        const float vg8 = fmaf((float)(d[cb][2] + (d[cb][3] << 8)), K, O);
        const float4 s4 = sc[cb & 3];
        accp[cb][0] = fmaf(vg, cb < 4 ? s4.x : s4.z, accp[cb][0]);
        accp[cb][1] = fmaf(vg8, cb < 4 ? s4.y : s4.w, accp[cb][1]);
    }
}

// The group's activation digits, by one warp: lane l holds rows 2l, 2l + 1
// (xv). X = round(x 2^s) with 2^s from the group's largest |x| (|X| <= 2^22)
// is cut into three signed byte digits (bytes of X + 0x808080, each xor 0x80),
// written as planes [3][64] bytes at pl. K0 = 2^-s, K1 = 2^(16-s) and
// O1 = -8 sum(X) 2^-s are the fold constants of lanes t = 0 and 1; O1 is NaN
// for a group holding a NaN or an infinity, which has no digits (its
// columns become NaN).
__device__ __forceinline__ void tmv_digits(float2 xv, uint8_t *pl, int lane, float &K0, float &K1, float &O1) {
    const uint32_t ax = max(__float_as_uint(xv.x) & 0x7FFFFFFFu, __float_as_uint(xv.y) & 0x7FFFFFFFu);
    uint32_t amax;
    asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(amax) : "r"(ax));
    // |x| < 2^(e - 126) for the largest biased exponent e: 2^s with s = 148 - e
    // keeps |X| <= 2^22 (s at most 126 so that 2^-s is a normal float)
    int sh = 148 - (int)(amax >> 23);
    sh = sh > 126 ? 126 : sh;
    const float up = __uint_as_float((uint32_t)(127 + sh) << 23), dn = __uint_as_float((uint32_t)(127 - sh) << 23);
    const int X0 = __float2int_rn(xv.x * up), X1 = __float2int_rn(xv.y * up);
    int sx;
    asm volatile("redux.sync.add.s32 %0, %1, 0xffffffff;" : "=r"(sx) : "r"(X0 + X1));
    const uint32_t dg0 = (uint32_t)(X0 + 0x808080) ^ 0x808080u, dg1 = (uint32_t)(X1 + 0x808080) ^ 0x808080u;
    uint16_t *pl16 = reinterpret_cast<uint16_t *>(pl);
    pl16[lane] = (uint16_t)__byte_perm(dg0, dg1, 0x0040); // plane p, bytes 2l, 2l + 1
    pl16[32 + lane] = (uint16_t)__byte_perm(dg0, dg1, 0x0051);
    pl16[64 + lane] = (uint16_t)__byte_perm(dg0, dg1, 0x0062);
    K0 = dn;
    K1 = dn * 65536.f;
    O1 = amax >= 0x7F800000u ? __uint_as_float(0x7FC00000u) : -8.f * (float)sx * dn;
}

// The B fragments of lane (g, t) from a group's digit planes.
__device__ __forceinline__ void tmv_bfrag(const uint8_t *pl, int lane, uint32_t &be0, uint32_t &bo0, uint32_t &be1,
                                          uint32_t &bo1) {
    const int g = lane >> 2, t = lane & 3;
    be0 = bo0 = be1 = bo1 = 0;
    if (g < 3) {
        const uint2 q0 = *reinterpret_cast<const uint2 *>(pl + g * 64 + 8 * t);
        const uint2 q1 = *reinterpret_cast<const uint2 *>(pl + g * 64 + 32 + 8 * t);
        be0 = __byte_perm(q0.x, q0.y, 0x6420);
        bo0 = __byte_perm(q0.x, q0.y, 0x7531);
        be1 = __byte_perm(q1.x, q1.y, 0x6420);
        bo1 = __byte_perm(q1.x, q1.y, 0x7531);
    }
}

// Lane t's K and O of the group fold: the D fragment holds, in lane t = 0,
// sum n*d0 and sum n*d1 (n the unsigned code) and in lane t = 1 sum n*d2, so
// lane t adds scale * ((D_a + 256 D_b) * K_t + O_t) with K_0 = 2^-s,
// K_1 = 2^(16-s), O_1 = -8 * sum(X) * 2^-s (the code offset 8), K and O zero
// for t >= 2; O is NaN for every lane of a non-finite group.
__device__ __forceinline__ void tmv_fold(int lane, float K0, float K1, float O1, float &K, float &O) {
    const int t = lane & 3;
    K = t == 0 ? K0 : t == 1 ? K1 : 0.f;
    O = (t == 1 || O1 != O1) ? O1 : 0.f;
}

// One 64-row item, item columns of half hf, into this lane's partial sums
// accp[cb][rh]. xr: the group's 64 activations; pl: this warp's 192 bytes of
// digit planes.
__device__ __forceinline__ void tmv_item(const uint8_t *item, int hf, const float *xr, uint8_t *pl, int lane,
                                         float (&accp)[8][2]) {
    float K0, K1, O1;
    tmv_digits(*reinterpret_cast<const float2 *>(xr + 2 * lane), pl, lane, K0, K1, O1); // rows 2l, 2l + 1
    __syncwarp();
    uint32_t be0, bo0, be1, bo1;
    tmv_bfrag(pl, lane, be0, bo0, be1, bo1);
    __syncwarp(); // the planes are read before the next item writes them
    float K, O;
    tmv_fold(lane, K0, K1, O1, K, O);
    tmv_mma(item, hf, be0, bo0, be1, bo1, K, O, lane, accp);
}

// A group's digits prepared once in shared memory (unit slot u: planes
// [3][64] bytes, then float4 {K0, K1, O1, 0} at byte 192): the digits of the
// 64 floats at u, written over them in place, by one warp.
__device__ __forceinline__ void tmv_digits_unit(uint8_t *u, int lane) {
    const float2 xv = *reinterpret_cast<const float2 *>(reinterpret_cast<const float *>(u) + 2 * lane);
    __syncwarp(); // every lane has its activations before the planes overwrite them
    float K0, K1, O1;
    tmv_digits(xv, u, lane, K0, K1, O1);
    if (lane == 0) *reinterpret_cast<float4 *>(u + 192) = make_float4(K0, K1, O1, 0.f);
}

// One 64-row item with its group's digits prepared in unit slot u.
__device__ __forceinline__ void tmv_item_pre(const uint8_t *item, int hf, const uint8_t *u, int lane,
                                             float (&accp)[8][2]) {
    uint32_t be0, bo0, be1, bo1;
    tmv_bfrag(u, lane, be0, bo0, be1, bo1);
    const float4 kc = *reinterpret_cast<const float4 *>(u + 192);
    float K, O;
    tmv_fold(lane, kc.x, kc.y, kc.z, K, O);
    tmv_mma(item, hf, be0, bo0, be1, bo1, K, O, lane, accp);
}

// The lane's partial sums accp (all lanes of a quad hold parts of the same
// columns) into its sums acc in the CUDA-core layout: quad-added, blocks t and
// t + 4 kept (item columns 4l + 2k + rh of half hf), the other half zero.
// accp is zeroed.
__device__ __forceinline__ void tmv_flush(float (&accp)[8][2], float (&acc)[1][8], int lane, int hf) {
    const int t = lane & 3;
    float tot[8][2];
#pragma unroll
    for (int cb = 0; cb < 8; cb++)
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            float v = accp[cb][rh];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            tot[cb][rh] = v;
            accp[cb][rh] = 0.f;
        }
#pragma unroll
    for (int k = 0; k < 2; k++)
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            const float v = t == 0 ? tot[4 * k][rh] : t == 1 ? tot[4 * k + 1][rh] : t == 2 ? tot[4 * k + 2][rh] : tot[4 * k + 3][rh];
            acc[0][2 * k + rh] = hf ? 0.f : v;
            acc[0][4 + 2 * k + rh] = hf ? v : 0.f;
        }
}

} // namespace tqi
