// tq_quantize.cu — device quantizers, bit-exact with tensai's Go quantizers,
// and the seeded synthetic-input generator.
//
// Bit-exactness: every floating-point step of quant.go:37-72 and
// quant4.go:28-89 is written with an explicitly rounded intrinsic so nvcc
// cannot contract `w*inv + 0.5` into an FMA (that would change the code at
// exact half-way points): __fdiv_rn for maxAbs/127 and 1/s, __fmul_rn for
// w*inv, __fadd_rn/__fsub_rn for the +/-0.5, and __float2int_rz for Go's
// truncating int8()/int() conversion.
#include <cuda_fp16.h>
#include "../../include/tensai_cuda.h"
#include "tq_common.cuh"

// ---------------------------------------------------------------------------
// Synthetic inputs: element i of (seed, stream) is
//   S = sum of the twelve 16-bit fields of mix(key + (3i+j+1)*gamma), j=0..2
//   v = float(2S - 786420) * (sigma * 2^-17)
// with one IEEE rounding (the multiply), identical to the host generator.
// ---------------------------------------------------------------------------
#define TQ_GAMMA 0x9E3779B97F4A7C15ull

__host__ __device__ static inline uint64_t tq_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t tq_synth_key(uint64_t seed, uint64_t stream) {
    return tq_mix64(seed * TQ_GAMMA + 0x632BE59BD9B4E019ull) ^ tq_mix64((stream + 1) * 0xD1B54A32D192ED03ull);
}

__global__ void tq_synth_kernel(float *__restrict__ out, size_t n, uint64_t key, float c) {
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        int32_t s = 0;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            uint64_t h = tq_mix64(key + (3 * (uint64_t)i + (uint64_t)j + 1) * TQ_GAMMA);
            s += (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
                 (int32_t)(h >> 48);
        }
        out[i] = __fmul_rn((float)(2 * s - 786420), c);
    }
}

// Seeded uniform token ids (host): id i = mix64(key + (i+1)*gamma) % vocab.
void tq_host_synth_tokens(int *out, int n, int vocab, uint64_t seed) {
    const uint64_t key = tq_synth_key(seed, 3);
    for (int i = 0; i < n; i++) out[i] = (int)(tq_mix64(key + (uint64_t)(i + 1) * TQ_GAMMA) % (uint64_t)vocab);
}

cudaError_t tq_launch_synth(float *out, size_t n, uint64_t seed, uint64_t stream, float sigma, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    // sigma * 2^-17 is exact in float (a power-of-two scaling).
    tq_synth_kernel<<<(unsigned)blocks, 256, 0, st>>>(out, n, tq_synth_key(seed, stream), sigma * 0x1p-17f);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// int8: QuantizeMatrix (quant.go:37-72). Block = 32 columns x 8 row lanes.
// Pass 1 takes maxAbs per column with the reference's comparisons (v<0 -> -v;
// keep v if v > maxAbs), pass 2 writes the codes. The max is order-free, so
// the row-lane split cannot change it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tq_absmax_step(float maxAbs, float v) {
    if (v < 0) v = -v;
    return v > maxAbs ? v : maxAbs;
}

__device__ __forceinline__ int tq_round_away(float w, float inv) {
    float v = __fmul_rn(w, inv);
    v = v >= 0 ? __fadd_rn(v, 0.5f) : __fsub_rn(v, 0.5f);
    return __float2int_rz(v);
}

// Where the kernels read W[i][j] (K = m.rows, N = m.cols): a row-major f32
// [K][N] matrix, or a [N][K] Linear weight ([out][in], the checkpoint layout)
// read transposed and widened to f32 exactly (BF16: bits << 16 as
// safetensors.go:187-190; F16: IEEE widening), which is the loader's
// Matrix().T() (_example/qwen/model.go:126-140) fused into the quantizer.
struct SrcRowMajor {
    const float *w;
    int cols;
    __device__ __forceinline__ float operator()(int i, int j) const { return w[(size_t)i * cols + j]; }
};
struct SrcLinear {
    const void *w;
    int rows, dtype;
    __device__ __forceinline__ float operator()(int i, int j) const {
        const size_t k = (size_t)j * rows + i;
        if (dtype == TQ_LINEAR_BF16) return __uint_as_float((uint32_t)static_cast<const uint16_t *>(w)[k] << 16);
        if (dtype == TQ_LINEAR_F16) return __half2float(static_cast<const __half *>(w)[k]);
        return static_cast<const float *>(w)[k];
    }
};

template <class Src>
__global__ void __launch_bounds__(256) tq_quantize8_kernel(TqMatrixDev m, Src w) {
    __shared__ float red[8][33];
    const int j = blockIdx.x * 32 + threadIdx.x;
    const bool valid = j < m.cols;
    float maxAbs = 0.f;
    if (valid)
        for (int i = threadIdx.y; i < m.rows; i += 8) maxAbs = tq_absmax_step(maxAbs, w(i, j));
    red[threadIdx.y][threadIdx.x] = maxAbs;
    __syncthreads();
    maxAbs = red[0][threadIdx.x];
#pragma unroll
    for (int r = 1; r < 8; r++) maxAbs = tq_absmax_step(maxAbs, red[r][threadIdx.x]);
    const float s = __fdiv_rn(maxAbs, 127.0f);
    if (valid && threadIdx.y == 0) m.scale[j] = s;
    if (!valid || s == 0) return; // codes stay 0 (quant.go:57-59); buffer is pre-zeroed
    const float inv = __fdiv_rn(1.0f, s);
    for (int i = threadIdx.y; i < m.rows; i += 8)
        m.codes[tq_code_offset(m.units, i, j)] = (uint8_t)(int8_t)tq_round_away(w(i, j), inv);
}

// ---------------------------------------------------------------------------
// int4: QuantizeMatrix4 (quant4.go:28-89). One thread per (column pair p,
// group g) owns the byte column p of that group: it quantizes column p (low
// nibble) and column half+p (high nibble) and writes whole bytes, so no two
// threads touch one byte. s==0 gives nibble 8 (quant4.go:57-62).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t tq_nibble(float w, float s, float inv) {
    if (s == 0) return 8u;
    int n = tq_round_away(w, inv);
    n = n < -8 ? -8 : (n > 7 ? 7 : n);
    return (uint32_t)(n + 8);
}

template <class Src>
__global__ void __launch_bounds__(128) tq_quantize4_kernel(TqMatrixDev m, Src w) {
    const int half = m.cols / 2;
    const int p = blockIdx.x * 128 + threadIdx.x;
    const int g = blockIdx.y;
    if (p >= half) return;
    const int rlo = g * TQ_GROUP;
    const int rhi = min(rlo + TQ_GROUP, m.rows);
    float mlo = 0.f, mhi = 0.f;
    for (int i = rlo; i < rhi; i++) {
        mlo = tq_absmax_step(mlo, w(i, p));
        mhi = tq_absmax_step(mhi, w(i, half + p));
    }
    const float slo = __fdiv_rn(mlo, 7.0f), shi = __fdiv_rn(mhi, 7.0f);
    m.scale[tq_scale4_offset(m.units, g, 0, p)] = slo;
    m.scale[tq_scale4_offset(m.units, g, 1, p)] = shi;
    const float ilo = slo == 0 ? 0.f : __fdiv_rn(1.0f, slo);
    const float ihi = shi == 0 ? 0.f : __fdiv_rn(1.0f, shi);
    for (int i = rlo; i < rhi; i++) {
        uint32_t lo = tq_nibble(w(i, p), slo, ilo);
        uint32_t hi = tq_nibble(w(i, half + p), shi, ihi);
        m.codes[tq_code_offset(m.units, i, p)] = (uint8_t)(lo | (hi << 4));
    }
}

template <class Src> static cudaError_t launch_quantize(const TqMatrixDev &m, Src w, cudaStream_t st) {
    if (m.rows == 0 || m.cols == 0) return cudaSuccess;
    if (m.bits == 8) {
        dim3 grid((m.cols + 31) / 32), block(32, 8);
        tq_quantize8_kernel<<<grid, block, 0, st>>>(m, w);
    } else {
        int half = m.cols / 2;
        if (half == 0) return cudaSuccess;
        dim3 grid((half + 127) / 128, m.units);
        tq_quantize4_kernel<<<grid, 128, 0, st>>>(m, w);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        return tq_launch_repack4(m, st); // the tensor-core matvec's K-packed copy
    }
    return cudaGetLastError();
}

cudaError_t tq_launch_quantize(const TqMatrixDev &m, const float *w, cudaStream_t st) {
    return launch_quantize(m, SrcRowMajor{w, m.cols}, st);
}

cudaError_t tq_launch_quantize_linear(const TqMatrixDev &m, const void *w, int dtype, cudaStream_t st) {
    return launch_quantize(m, SrcLinear{w, m.rows, dtype}, st);
}

// ---------------------------------------------------------------------------
// Reference layout <-> tiled device layout (see tq_common.cuh).
// ---------------------------------------------------------------------------
__global__ void tq_codes_layout_kernel(TqMatrixDev m, uint8_t *ref, bool to_tiled) {
    const int rb = m.bits == 8 ? m.cols : m.cols / 2;
    const size_t n = (size_t)m.rows * rb;
    for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (size_t)gridDim.x * blockDim.x) {
        const int i = (int)(k / rb), b = (int)(k % rb);
        if (to_tiled)
            m.codes[tq_code_offset(m.units, i, b)] = ref[k];
        else
            ref[k] = m.codes[tq_code_offset(m.units, i, b)];
    }
}

__global__ void tq_scale4_layout_kernel(TqMatrixDev m, float *ref, bool to_tiled) {
    const int half = m.cols / 2;
    const size_t n = (size_t)m.units * m.cols; // reference Scale[g*cols + j]
    for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (size_t)gridDim.x * blockDim.x) {
        const int g = (int)(k / m.cols), j = (int)(k % m.cols);
        const int hi = j >= half, pr = hi ? j - half : j;
        if (to_tiled)
            m.scale[tq_scale4_offset(m.units, g, hi, pr)] = ref[k];
        else
            ref[k] = m.scale[tq_scale4_offset(m.units, g, hi, pr)];
    }
}

static cudaError_t layout(const TqMatrixDev &m, uint8_t *ref_q, float *ref_scale, bool to_tiled, cudaStream_t st) {
    if (m.rows == 0 || m.cols == 0) return cudaSuccess;
    const unsigned blocks = 148 * 8;
    tq_codes_layout_kernel<<<blocks, 256, 0, st>>>(m, ref_q, to_tiled);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (m.bits == 8) {
        return to_tiled ? cudaMemcpyAsync(m.scale, ref_scale, sizeof(float) * m.cols, cudaMemcpyDeviceToDevice, st)
                        : cudaMemcpyAsync(ref_scale, m.scale, sizeof(float) * m.cols, cudaMemcpyDeviceToDevice, st);
    }
    if (m.cols / 2 == 0) return cudaSuccess;
    tq_scale4_layout_kernel<<<blocks, 256, 0, st>>>(m, ref_scale, to_tiled);
    return cudaGetLastError();
}

cudaError_t tq_launch_to_tiled(const TqMatrixDev &m, const uint8_t *ref_q, const float *ref_scale, cudaStream_t st) {
    const cudaError_t e = layout(m, const_cast<uint8_t *>(ref_q), const_cast<float *>(ref_scale), true, st);
    return e != cudaSuccess ? e : tq_launch_repack4(m, st);
}

cudaError_t tq_launch_from_tiled(const TqMatrixDev &m, uint8_t *ref_q, float *ref_scale, cudaStream_t st) {
    return layout(m, ref_q, ref_scale, false, st);
}
