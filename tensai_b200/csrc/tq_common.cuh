// tq_common.cuh — shared definitions for the tensai B200 library.
//
// Device layout of a quantized matrix (one per handle, resident in HBM).
// rowBytes = cols (int8) or cols/2 (int4): the length of a row of the
// reference's Q (quant.go:31, quant4.go:144). The matrix is cut into column
// tiles of 128 bytes and units of 64 rows (an int4 unit is one scale group);
// tiles = ceil(rowBytes/128), units = ceil(rows/64).
//   codes : tiled. Item (t, u) = the 64 x 128 byte block of rows 64u.. and row
//           bytes 128t.., stored contiguously at byte offset (t*units + u)*8192.
//           Inside an item, row r occupies bytes [128r, 128r+128) with its
//           sixteen 16-byte chunks permuted: chunk c sits at chunk position
//           c ^ (r % 8). That is the tensor cores' 128-byte-swizzled,
//           MN-major shared-memory operand layout, so an item copied verbatim
//           into shared memory is a ready UMMA A operand (128 columns x 64 K).
//           Padding rows and bytes are zero. Each item is one 8 KB contiguous
//           read, and a run of consecutive items is one contiguous range of
//           HBM.
//   scale : int8 -> [tiles*128] floats, scale[j] = Scale[j] (quant.go:32).
//           int4 -> per item 256 floats at (t*units + u)*256: [0,128) hold the
//           reference's Scale[u*cols + 128t + c] (low-nibble columns) and
//           [128,256) hold Scale[u*cols + cols/2 + 128t + c] (high-nibble
//           columns), c < 128 (quant4.go:38, :56).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#define TQ_GROUP 64        // rows per int4 scale group (q4Group, quant4.go:12)
#define TQ_TILE_BYTES 128  // bytes of a code row per item
#define TQ_ITEM_BYTES (TQ_TILE_BYTES * TQ_GROUP)
#define TQ_KPACK_BYTES (TQ_ITEM_BYTES + 1024) // a K-packed int4 item: codes, then 256 float scales
#define TQ_MAX_TILES 8192  // rowBytes <= 1 MiB
#define TQ_MAX_CTAS 256    // persistent matvec grid <= 256 CTAs
#define TQ_STATUS_TIMEOUT 1u // a kernel gave up waiting on an mbarrier

// Scratch for the matvec's cross-CTA tile reduction: partial sums of tiles
// shared by several CTAs, and one arrival counter per column tile (zero at
// rest; the last arriving CTA re-arms it). One scratch per stream.
struct TqScratch {
    float *partial;     // TQ_SCRATCH_PARTIAL_FLOATS
    unsigned *counters; // TQ_MAX_TILES
    unsigned *status;   // TQ_STATUS_* bits set by kernels on this stream
    uint8_t *planes;    // TQ_SCRATCH_PLANES_BYTES: activation digit planes of a matvec
    float *mm_partial;  // tq_mm_partial_floats(SMs): tile partials of the M >= 16 matmul (or null)
};
#define TQ_SCRATCH_PARTIAL_FLOATS ((size_t)2 * TQ_MAX_CTAS * 8 * 8 * 32)
#define TQ_SCRATCH_PLANES_BYTES ((size_t)8 << 20) // 2304 B per 64 rows: K <= 233,000
#define TQ_MM_MIN_ROWS 16  // activation rows from which tq_matmul* use the tf32 tensor-core matmul
#define TQ_MM_MAX_ROWS 64  // activation rows per matmul launch
// Two partial slots per CTA of up to 2 runs x 128 rows x 128 columns.
static inline size_t tq_mm_partial_floats(int sms) { return (size_t)2 * sms * 2 * TQ_MM_MAX_ROWS * TQ_TILE_BYTES; }

// One-time set-up of a kernel launcher on each device (kernel attributes, SM
// count), safe when several host threads launch at once: the first caller on
// a device runs it, concurrent callers wait for it, later calls read the
// cached result. Devices 0..63.
struct TqDeviceOnce {
    std::once_flag flag[64];
    cudaError_t err[64] = {};
    int sms[64] = {};
};
template <class F> inline cudaError_t tq_device_once(TqDeviceOnce &o, int dev, F &&setup) {
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::call_once(o.flag[dev], [&] {
        cudaError_t e = cudaDeviceGetAttribute(&o.sms[dev], cudaDevAttrMultiProcessorCount, dev);
        o.err[dev] = e == cudaSuccess ? setup() : e;
    });
    return o.err[dev];
}

struct TqMatrixDev {
    int bits;       // 8 or 4
    int rows;       // K
    int cols;       // N
    int tiles;      // ceil(rowBytes/128)
    int units;      // ceil(rows/64) (= scale groups for int4)
    uint8_t *codes; // tiles*units*8192 bytes, tiled (see above)
    float *scale;   // see above
    // int4: the same items K-packed for the tensor-core matvecs (tq_cmv.cu,
    // tq_chain.cu), TQ_KPACK_BYTES each: 8 KB of codes then the item's 256
    // scales in that kernel's order, so that one bulk copy moves an item and
    // consecutive items are one contiguous range. Null for int8.
    uint8_t *kpack;
};

#ifdef __CUDACC__
#define TQ_HD __host__ __device__ __forceinline__
#else
#define TQ_HD inline
#endif

// Byte position of (row r, byte c) inside an item: 128-byte swizzle.
TQ_HD int tq_item_offset(int r, int c) { return r * TQ_TILE_BYTES + ((((c >> 4) ^ (r & 7)) << 4) | (c & 15)); }
// Byte b of code row i in the tiled layout.
TQ_HD size_t tq_code_offset(int units, int i, int b) {
    return ((size_t)(b / TQ_TILE_BYTES) * units + i / TQ_GROUP) * TQ_ITEM_BYTES +
           tq_item_offset(i % TQ_GROUP, b % TQ_TILE_BYTES);
}
// int4 scale of group u, run hi (0 = low-nibble columns, 1 = high), column pair p.
TQ_HD size_t tq_scale4_offset(int units, int u, int hi, int p) {
    return ((size_t)(p / TQ_TILE_BYTES) * units + u) * (2 * TQ_TILE_BYTES) + hi * TQ_TILE_BYTES + (p % TQ_TILE_BYTES);
}

#ifdef __CUDACC__
// Stream-K split of `items` work items (column tile, 64-row unit), tile-major,
// over G <= items persistent CTAs: CTA c owns [start(c), start(c + 1)) with
// start(c) = floor(items * c / G), so column tile t (items [t0, t1)) is shared
// by CTAs owner(t0) .. owner(t1 - 1). 32-bit division whenever items * G < 2^32.
struct TqSplit {
    long long items;
    int G;
    bool narrow;
    __device__ __forceinline__ TqSplit(long long n, int g)
        : items(n), G(g), narrow((unsigned long long)n * (unsigned)g < (1ull << 32)) {}
    __device__ __forceinline__ long long start(int c) const {
        return narrow ? (long long)((unsigned)items * (unsigned)c / (unsigned)G) : items * c / G;
    }
    // The largest c with start(c) <= it: floor(((it + 1) * G - 1) / items).
    __device__ __forceinline__ int owner(long long it) const {
        return narrow ? (int)(((unsigned)(it + 1) * (unsigned)G - 1u) / (unsigned)items)
                      : (int)(((it + 1) * G - 1) / items);
    }
    // Partial-sum slot of contributor c to the tile starting at item t0: 2c for
    // a slice that starts inside the tile (its first segment), 2c + 1 for one
    // that started before it (its last segment). Only owner(t0) can be the latter.
    __device__ __forceinline__ int slot(int c, long long t0) const { return 2 * c + (start(c) >= t0 ? 0 : 1); }
};

// One CTA's arrival at a shared tile's counter, by one thread after a barrier
// that orders the CTA's partial-sum stores before it. acq_rel at gpu scope
// publishes those stores and, for the last of n arrivals, acquires every other
// contributor's; a barrier after this call extends that to the whole CTA. The
// last arrival re-arms the counter for the next launch on the stream.
__device__ __forceinline__ bool tq_arrive_last(unsigned *counter, unsigned n) {
    unsigned prev;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
    const bool last = prev == n - 1;
    if (last) asm volatile("st.relaxed.gpu.u32 [%0], %1;" ::"l"(counter), "r"(0u) : "memory");
    return last;
}
#endif

static inline int tq_row_bytes(int bits, int cols) { return bits == 8 ? cols : cols / 2; }
static inline int tq_tiles(int bits, int cols) { return (tq_row_bytes(bits, cols) + TQ_TILE_BYTES - 1) / TQ_TILE_BYTES; }
static inline int tq_units(int rows) { return (rows + TQ_GROUP - 1) / TQ_GROUP; }
static inline size_t tq_code_bytes(int bits, int rows, int cols) {
    return (size_t)tq_tiles(bits, cols) * tq_units(rows) * TQ_ITEM_BYTES;
}
static inline size_t tq_scale_floats(int bits, int rows, int cols) {
    const size_t t = (size_t)tq_tiles(bits, cols);
    return bits == 8 ? t * TQ_TILE_BYTES : t * tq_units(rows) * 2 * TQ_TILE_BYTES;
}

// Kernel launchers (defined in the .cu files). All return cudaError_t of the
// launch; none synchronizes.
cudaError_t tq_launch_synth(float *out, size_t n, uint64_t seed, uint64_t stream, float sigma, cudaStream_t st);
cudaError_t tq_launch_quantize(const TqMatrixDev &m, const float *w, cudaStream_t st);
// Quantizes the transpose of a Linear weight [m.cols][m.rows] of element type
// dtype (TQ_LINEAR_*): W[i][j] = w[j][i] widened to f32 exactly.
cudaError_t tq_launch_quantize_linear(const TqMatrixDev &m, const void *w, int dtype, cudaStream_t st);
// Reference layout (rows x rowBytes codes, reference Scale) <-> device layout,
// both sides in device memory.
cudaError_t tq_launch_to_tiled(const TqMatrixDev &m, const uint8_t *ref_q, const float *ref_scale, cudaStream_t st);
cudaError_t tq_launch_from_tiled(const TqMatrixDev &m, uint8_t *ref_q, float *ref_scale, cudaStream_t st);
cudaError_t tq_launch_matvec(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                             cudaStream_t st);

// What a single-row (M = 1) CUDA-core matvec does with its output, for the
// decode steps:
//   TQ_EPI_NONE    out = x W;
//   TQ_EPI_SWIGLU  int4 [gate | up] matrix of 2F columns (column c and F + c
//                  share a code byte): out[c] = float32(silu(gate_c)) * up_c,
//                  c < F, silu in float64 (_example/qwen/model.go:296-299).
//   TQ_EPI_RESID   (chains only) out = resid + x W, resid may be out itself
//                  (the residual adds of _example/qwen/model.go:276-278, 301-303).
#define TQ_EPI_NONE 0
#define TQ_EPI_SWIGLU 1
#define TQ_EPI_RESID 2
cudaError_t tq_launch_cmv_epi(const TqMatrixDev &m, const float *x, float *out, const TqScratch &scr, cudaStream_t st,
                              int epi, bool tc);
// int4 matvec on the tensor cores (mma.sync over the K-packed copy), one row
// per launch; matrices without the copy go to tq_launch_cmv.
cudaError_t tq_launch_tmv(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                          cudaStream_t st);
// Fills kcodes / kscale of an int4 matrix from its codes and scales (no-op
// without them); the quantize and upload launchers end with it.
cudaError_t tq_launch_repack4(const TqMatrixDev &m, cudaStream_t st);
cudaError_t tq_launch_igemv(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                            cudaStream_t st);
// CUDA-core matvec for M <= 2 rows per launch (tq_cmv.cu).
cudaError_t tq_launch_cmv(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                          cudaStream_t st);
// Matmul for M >= 16 rows on tcgen05 kind::tf32 (needs scr.mm_partial).
cudaError_t tq_launch_mm(const TqMatrixDev &m, const float *x, float *out, int M, const TqScratch &scr,
                         cudaStream_t st);
// Allocation-free CUDA-core matvec (fixed device scratch in tq_matvec.cu).
enum { TQ_FIXED_OK = 0, TQ_FIXED_CUDA, TQ_FIXED_DEVICE, TQ_FIXED_SMS, TQ_FIXED_TILES };
#define TQ_FIXED_MAX_TILES 4096
#define TQ_FIXED_MAX_SMS 160
#define TQ_FIXED_ROWS_PER_LAUNCH 4
int tq_launch_matvec_fixed(const TqMatrixDev &m, const float *x, float *out, int M, cudaStream_t st,
                           cudaError_t *err);
// Status bits of the fixed scratch on the current device (device idle); when
// set, the fixed counters are re-armed.
cudaError_t tq_fixed_status(unsigned *bits);

// A chain of dependent single-row matvecs in one persistent launch
// (tq_chain.cu). Op j reads its input only after op j - 1 has written all of
// its output. Every op of a chain has the same bit width; x is 16-byte aligned.
// norm_w != null: x (the output of op norm_from, a TQ_EPI_RESID op earlier in
// the chain) is RMS-normalised with weight norm_w and epsilon eps first.
#define TQ_CHAIN_MAX_OPS 4096
// 64-row groups of activations a CTA stages per op: an op whose per-CTA slice
// (items / SMs, rounded up) covers more distinct groups is not chainable.
#define TQ_CHAIN_MAX_GROUPS 64
struct TqChainSpec {
    const TqMatrixDev *m;
    const float *x;
    float *out;
    int epi;
    const float *resid;
    const float *norm_w;
    int norm_from;
    double eps;
};
struct TqChain;
enum {
    TQ_CHAIN_OK = 0,
    TQ_CHAIN_BAD_COUNT,  // no ops, or more than TQ_CHAIN_MAX_OPS
    TQ_CHAIN_MIXED_BITS, // int8 and int4 ops in one chain
    TQ_CHAIN_EMPTY,      // a matrix without rows or columns
    TQ_CHAIN_NO_KPACK,   // an int4 matrix without its K-packed copy
    TQ_CHAIN_X_ALIGN,    // a null or not 16-byte aligned input, or a null output
    TQ_CHAIN_EPI,        // an unknown epilogue or one the matrix cannot take
    TQ_CHAIN_TOO_WIDE,   // more than TQ_MAX_TILES column tiles
    TQ_CHAIN_NORM,       // a normalised input that is not an earlier residual op's output
    TQ_CHAIN_TOO_DEEP,   // a per-CTA slice covering more than TQ_CHAIN_MAX_GROUPS row groups
    TQ_CHAIN_ALIAS,      // an input or residual overlapping an earlier op's output other than exactly
};
// Validates the ops and copies their descriptors to the current device
// (synchronous); *why names the first problem found and *bad_op its op.
cudaError_t tq_chain_build(const TqChainSpec *spec, int n, TqChain **out, int *why, int *bad_op);
void tq_chain_destroy(TqChain *ch);
int tq_chain_device(const TqChain *ch);
cudaError_t tq_chain_launch(const TqChain *ch, const TqScratch &scr, cudaStream_t st);
// int4 chains (tq_chain4.cu): column-owner CTAs, at most TQ_CHAIN4_MAX_BLOCKS
// 32-column blocks per CTA and op (cols <= 256 x SMs).
#define TQ_CHAIN4_MAX_BLOCKS 8
struct TqChain4;
cudaError_t tq_chain4_build(const TqChainSpec *spec, int n, int sms, TqChain4 **out, int *why, int *bad_op);
void tq_chain4_destroy(TqChain4 *ch);
cudaError_t tq_chain4_launch(const TqChain4 *ch, unsigned *status, cudaStream_t st);
