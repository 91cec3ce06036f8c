/*
 * tensai_cuda.h — C ABI of libtensai_cuda.so, the B200 (sm_100a) backend for
 * tensai's weight-only quantized inference path (github.com/mattn/tensai).
 *
 * The Go package reaches this library the way wgpu.go reaches wgpu-native:
 * purego.Dlopen + RegisterLibFunc (wgpu_dlopen.go:9-11, wgpu.go:292-357),
 * no cgo. Every entry point therefore takes only scalars and plain pointers,
 * returns an int status (0 = success, negative = error), never aborts the
 * process, and leaves a human-readable message in tq_last_error() on the
 * calling thread. Messages for argument errors repeat the reference's own
 * wording ("tensai: ..."), so the Go shim can return them unchanged.
 *
 * Threading: every entry point is thread-safe. Host-pointer calls run on a
 * per-thread, per-device CUDA stream with per-thread staging buffers; matrix
 * handles are read-only after creation and may be shared across threads.
 * Freeing a handle while another thread computes with it is a caller error,
 * as using a freed GPUTensor is in the reference (wgputensor.go:676-686).
 *
 * Ownership: the library copies codes and scales into device memory at
 * upload/quantize time and keeps them resident in HBM until tq_free.
 */
#ifndef TENSAI_CUDA_H
#define TENSAI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TQ_EXPORT __attribute__((visibility("default")))
#else
#define TQ_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TQ_ABI_VERSION 1

/* Status codes. */
#define TQ_OK 0
#define TQ_ERR_ARG (-1)         /* bad argument (null pointer, negative size, odd int4 column count) */
#define TQ_ERR_SHAPE (-2)       /* x/out lengths do not match the matrix */
#define TQ_ERR_HANDLE (-3)      /* unknown or freed handle */
#define TQ_ERR_CUDA (-4)        /* a CUDA runtime call failed; message has the CUDA error string */
#define TQ_ERR_NOMEM (-5)       /* device or pinned allocation failed */
#define TQ_ERR_UNSUPPORTED (-6) /* no sm_100 device, or a size beyond a documented limit */
#define TQ_ERR_TIMEOUT (-7)     /* a kernel gave up a bounded wait (see tq_device_status) */

/* Library version gate, as wgpu.go:292-313 checks wgpu-native's version. */
TQ_EXPORT int tq_version(void);

/* Message of the last failing call on this thread ("" if none). */
TQ_EXPORT const char *tq_last_error(void);

/* Number of visible CUDA devices; selects the device that later calls on
 * this thread create handles on (default 0). */
TQ_EXPORT int tq_device_count(int *n);
TQ_EXPORT int tq_set_device(int device);

/* ---- quantized matrices ------------------------------------------------- */

/* Uploads an int8 QMatrix: q = QMatrix.Q (rows*cols bytes, row-major; the
 * reference's 16 pad bytes are not read), scale = QMatrix.Scale (cols).
 * Replaces: type QMatrix (quant.go:29-33), made resident for MatVec. */
TQ_EXPORT int tq_q8_upload(const int8_t *q, const float *scale, int rows, int cols, uint64_t *handle);

/* Uploads an int4 Q4Matrix: q = Q4Matrix.Q (rows*cols/2 bytes, byte (i,j)
 * holding column j in its low nibble and column j+cols/2 in its high one),
 * scale = Q4Matrix.Scale (ceil(rows/64)*cols, group-major).
 * Replaces: type Q4Matrix (quant4.go:20-24). cols must be even. */
TQ_EXPORT int tq_q4_upload(const uint8_t *q, const float *scale, int rows, int cols, uint64_t *handle);

/* Quantizes a host float32 matrix [rows][cols] on the device and writes the
 * reference's exact byte layout back: q gets rows*cols (+16 zero pad) bytes,
 * scale gets cols floats. Bit-exact with QuantizeMatrix (quant.go:37-72). */
TQ_EXPORT int tq_quantize8(const float *w, int rows, int cols, int8_t *q, float *scale);

/* As tq_quantize8 for QuantizeMatrix4 (quant4.go:28-89): q gets
 * rows*cols/2 (+16 zero pad) bytes, scale gets ceil(rows/64)*cols floats.
 * Odd cols -> TQ_ERR_ARG, "tensai: quantize4 needs an even column count, got N"
 * (quant4.go:29-31). */
TQ_EXPORT int tq_quantize4(const float *w, int rows, int cols, uint8_t *q, float *scale);

/* Quantizes a DEVICE float32 matrix [rows][cols] (row-major, on the current
 * device) straight into a new resident handle, with no host round trip:
 * the quantize-on-load path of _example/qwen/model.go:126-140 kept on the GPU.
 * stream: a cudaStream_t (NULL = legacy default stream). The handle is ready
 * for use on that stream; the call does not synchronize. */
TQ_EXPORT int tq_quantize8_dev(const float *w, int rows, int cols, void *stream, uint64_t *handle);
TQ_EXPORT int tq_quantize4_dev(const float *w, int rows, int cols, void *stream, uint64_t *handle);

/* Quantize-on-load from a checkpoint tensor: w is a DEVICE Linear weight
 * [out_features][in_features], row-major, of element type dtype (BF16: the
 * upper half of an f32, widened by a 16-bit shift as safetensors.go:187-190;
 * F16: IEEE half, widened exactly; F32). The new handle holds the matrix the
 * loader builds with Matrix().T() (_example/qwen/model.go:126-140),
 * rows = in_features and cols = out_features, quantized bit for bit as
 * QuantizeMatrix / QuantizeMatrix4 quantize that transpose; the transpose and
 * the widening are fused into the quantizer (no f32 copy is made). int4 with
 * odd out_features -> TQ_ERR_ARG as tq_quantize4. Asynchronous on stream. */
#define TQ_LINEAR_F32 0
#define TQ_LINEAR_F16 1
#define TQ_LINEAR_BF16 2
TQ_EXPORT int tq_quantize8_linear_dev(const void *w, int dtype, int out_features, int in_features, void *stream,
                                      uint64_t *handle);
TQ_EXPORT int tq_quantize4_linear_dev(const void *w, int dtype, int out_features, int in_features, void *stream,
                                      uint64_t *handle);

/* bits (8 or 4), rows, cols of a handle. Any output pointer may be NULL. */
TQ_EXPORT int tq_matrix_info(uint64_t handle, int *bits, int *rows, int *cols);

/* Copies a handle's codes and scales back in the reference layout (the same
 * sizes tq_quantize8/4 write, including the 16 zero pad bytes). */
TQ_EXPORT int tq_download(uint64_t handle, void *q, float *scale);

/* Releases the device copy. Freeing 0 or an already freed handle is a no-op,
 * as GPUTensor.Free is idempotent (wgputensor.go:676-686). */
TQ_EXPORT int tq_free(uint64_t handle);

/* ---- compute ------------------------------------------------------------ */

/* out = x @ W for one activation row, host buffers, synchronous.
 * Replaces: (*QMatrix).MatVec (quant.go:77-103) and (*Q4Matrix).MatVec
 * (quant4.go:93-119). x_len must equal rows and out_len cols, else
 * TQ_ERR_SHAPE with the reference's message
 * "tensai: qmatvec shape mismatch: x=%d out=%d, want %dx%d" (quant.go:79)
 * or "tensai: q4matvec ..." (quant4.go:95). out is overwritten. */
TQ_EXPORT int tq_matvec(uint64_t handle, const float *x, size_t x_len, float *out, size_t out_len);

/* out[m][cols] = x[m][rows] @ W for m activation rows, host buffers,
 * synchronous. The reference has no batched call: this equals m MatVec calls
 * (quant.go:77, applied per row). m <= 8 runs on the CUDA-core kernels. */
TQ_EXPORT int tq_matmul(uint64_t handle, const float *x, float *out, int m);

/* As tq_matmul with DEVICE pointers (x: m*rows floats, out: m*cols floats,
 * on the handle's device), enqueued on stream (a cudaStream_t; NULL = legacy
 * default stream). Does not synchronize. The library keeps a small scratch
 * per (device, stream), created on the first call on that stream, so that
 * first call must not happen inside a CUDA-graph capture; graphs holding
 * these launches must not be replayed concurrently with each other. */
TQ_EXPORT int tq_matmul_dev(uint64_t handle, const float *x, float *out, int m, void *stream);

/* As tq_matmul_dev, but allocates nothing: no device or pinned memory, on
 * any call. No counterpart in the reference (its Go MatVec allocates no GPU
 * memory at all); it exists for callers that must not have the library
 * allocate at run time, e.g. a serving process that has handed all free HBM
 * to its own weight and KV-cache pool, where a library cudaMalloc could fail
 * mid-decode or stall the device.
 * Runs the CUDA-core kernel (tq_set_matvec_kernel does not apply) with its
 * cross-CTA scratch in fixed device arrays inside the library: 1.25 MiB of
 * partial sums plus 4096 tile counters, zero at load and left at zero by
 * every call. Limits: matrices of at most 4096 column tiles (524,288 int8 /
 * 1,048,576 int4 columns) and GPUs of at most 160 SMs, else
 * TQ_ERR_UNSUPPORTED with a message naming the limit; activation rows run 4
 * per launch, any m. The first call on each device does the set-up (looks up
 * the fixed arrays' device addresses and loads every kernel this entry point
 * can launch, so no later call loads code) and should come before any stream
 * capture. All callers on one device share the fixed scratch: calls that may
 * overlap on the device (other streams, other threads) race and corrupt each
 * other's results, so issue them in order on one stream. A bounded-wait
 * timeout inside the kernel sets the fixed scratch's status word:
 * tq_device_status reports it (TQ_STATUS_TIMEOUT) and re-arms the fixed
 * counters; results since the timeout are invalid. The set-up holds device
 * addresses for the life of the process: after a cudaDeviceReset of a device,
 * do not use this entry point on that device again. */
TQ_EXPORT int tq_matmul_dev_fixed(uint64_t handle, const float *x, float *out, int m, void *stream);

/* ---- chains of dependent matvecs ----------------------------------------- */

/* One op of a chain: out = x @ W (one activation row, DEVICE pointers on the
 * matrix's device). epilogue: TQ_CHAIN_EPI_NONE; TQ_CHAIN_EPI_SWIGLU (int4,
 * even cols: W is [gate | up], out[c] = float32(silu(gate_c)) * up_c for
 * c < cols/2, silu in float64, _example/qwen/model.go:296-299);
 * TQ_CHAIN_EPI_RESID (out = resid + x @ W, resid may equal out: the residual
 * adds of model.go:276-278 / 301-303). norm_w non-NULL: x is first replaced
 * by its RMSNorm, float32(float64(x) * inv) * norm_w with inv =
 * 1/sqrt(sum(x^2)/rows + eps) in float64 (model.go:182-193); x must then be
 * the output of op norm_from, an earlier TQ_CHAIN_EPI_RESID op of the same
 * chain. x must be 16-byte aligned. */
typedef struct {
    uint64_t matrix;
    const float *x;
    float *out;
    int epilogue;
    const float *resid;
    const float *norm_w;
    int norm_from;
    double eps;
} tq_chain_op;

#define TQ_CHAIN_EPI_NONE 0
#define TQ_CHAIN_EPI_SWIGLU 1
#define TQ_CHAIN_EPI_RESID 2

/* Builds a chain of n (1..4096) dependent matvecs, all int8 or all int4,
 * on the device of their matrices: op j reads x only after op j - 1 has
 * written all of its output, so the chain computes exactly what n
 * consecutive MatVec calls (quant.go:77-103 / quant4.go:93-119) with the
 * fused norms and epilogues compute, in the order the decode loops make them
 * (_example/qwen/model.go:232-307). No counterpart call exists in the
 * reference: it is the device-side form of that sequence, so that the
 * weights of later ops stream while earlier ops finish. The matrices must
 * outlive the chain. Synchronous; TQ_ERR_ARG names the first bad op. */
TQ_EXPORT int tq_chain_create(const tq_chain_op *ops, int n, uint64_t *chain);

/* Enqueues the whole chain as ONE kernel launch on stream (a cudaStream_t;
 * NULL = legacy default stream). Does not synchronize. Uses the same
 * per-(device, stream) scratch as tq_matmul_dev (so the first call on a
 * stream must not be inside a capture); capturable in CUDA graphs
 * afterwards. Launches of one chain on different streams must not overlap. */
TQ_EXPORT int tq_chain_run(uint64_t chain, void *stream);

/* Releases a chain (waits for the device first; a second call is a no-op). */
TQ_EXPORT int tq_chain_free(uint64_t chain);

/* Selects the GPU kernel behind tq_matvec / tq_matmul / tq_matmul_dev for
 * m <= 15 rows (process-wide). 0 (default) = the fastest measured choice per
 * row count: int4 single rows as 5 below, otherwise single-launch CUDA-core
 * fp32 FMA for m <= 2 and tensor-core integer MMA (weights used as stored,
 * activations split into exact int8 digit planes) for 3 <= m <= 15. 1 = CUDA-core fp32 FMA with per-warp copies;
 * 2 is retired (TQ_ERR_ARG); 3 = single-launch CUDA-core fp32
 * FMA, 2 rows per launch; 4 = tensor-core integer MMA with a digit-plane
 * launch; 5 = int4 on the tensor cores by mma.sync (codes from a K-packed
 * device copy that every int4 matrix holds, activations as exact int8 digits
 * per 64-row group), one row per launch, int8 as 3. All are GPU
 * implementations with the same contract; there is no CPU path. */
TQ_EXPORT int tq_set_matvec_kernel(int which);

/* ---- synthetic inputs ----------------------------------------------------- */

/* Fills n floats on the current device with the seeded generator the CPU
 * oracle uses (Irwin-Hall(12) normal with standard deviation sigma; element i
 * depends only on (seed, stream_id, i)). Stand-in for RandomMatrix
 * (tensor.go:269-277) and NormFloat64 activations, bit-identical on host and
 * device. cuda_stream: a cudaStream_t or NULL. */
TQ_EXPORT int tq_synth_dev(float *out, size_t n, uint64_t seed, uint64_t stream_id, float sigma, void *cuda_stream);

/* Waits for all work on the current device, then returns and clears its
 * status bits: bit 0 (TQ_STATUS_TIMEOUT = 1) means a kernel gave up waiting
 * for a weight copy (bounded at 2 s) and its output is invalid. The host-
 * pointer calls check this themselves and return TQ_ERR_TIMEOUT. */
TQ_EXPORT int tq_device_status(unsigned *bits);

/* ---- whole-model decode: GPT-2 (int8 decode weights) ----------------------- */

/* Shape of a GPT-2 model (_example/gpt2/model.go:17-24): layers, heads,
 * embedding width d (head size d/n_head must be 64: the example divides the
 * scores by 8), MLP width, vocabulary, context length. */
typedef struct {
    int n_layer, n_head, d, ffn, vocab, ctx;
} tq_gpt2_config;

/* Builds a random-init GPT-2 on the current device: every matrix and
 * embedding drawn from the tq_synth_dev generator with standard deviation
 * sigma (streams: wte 1, wpe 2, layer l: c_attn 16+8l, attn c_proj 17+8l,
 * mlp c_fc 18+8l, mlp c_proj 19+8l), layer-norm weights 1, biases 0. Keeps
 * the fp32 weights for the prefill and their QuantizeMatrix int8 twins for
 * decode (gpt2.quantize, model.go:51-60), plus a fp32 KV cache of ctx
 * positions, all resident. Replaces loadModel + quantize (model.go:79-133)
 * for synthetic weights. */
TQ_EXPORT int tq_gpt2_create(const tq_gpt2_config *cfg, uint64_t seed, float sigma, uint64_t *model);

/* Greedy generation (main.go:163-170 at temperature 0): prefill of the
 * n_prompt ids with the fp32 weights (model.go:361-401), then n_gen - 1 int8
 * decode steps (model.go:179-245); tokens[0..n_gen) receives the generated
 * ids (argmax, ties to the lowest id, main.go:69-77). times_ms (optional,
 * 2 floats): device time of the prefill and of the decode steps. Starts a
 * fresh sequence every call. n_prompt + n_gen - 1 must not exceed ctx. */
TQ_EXPORT int tq_gpt2_generate(uint64_t model, const int *prompt, int n_prompt, int n_gen, int *tokens,
                               float *times_ms);

/* A GPT-2 model whose weights come from a checkpoint instead of the
 * random-init generator: zeros, layer-norm weights 1, biases 0, until
 * tq_gpt2_load_tensor fills them (the example's loader, _example/gpt2/model.go:
 * 83-131). */
TQ_EXPORT int tq_gpt2_create_empty(const tq_gpt2_config *cfg, uint64_t *model);

/* One checkpoint tensor by the example's name, from device memory as stored
 * (TQ_LINEAR_F32 / F16 / BF16; matrices rows x cols, vectors 1 x n): wte.weight
 * (the embedding; the tied head wte^T is rebuilt from it, fp32 and int8),
 * wpe.weight (the first ctx positions kept), ln_f.{weight,bias}, and per
 * layer h.N. + ln_1.{weight,bias}, ln_2.{weight,bias},
 * attn.c_attn.{weight,bias}, attn.c_proj.{weight,bias}, mlp.c_fc.{weight,bias},
 * mlp.c_proj.{weight,bias}: Conv1D weights [in, out] kept in fp32 for the
 * prefill and quantized to int8 (QuantizeMatrix) for the decode steps.
 * Synchronous. TQ_ERR_SHAPE for a wrong shape, TQ_ERR_ARG for an unknown
 * name or a model made by tq_gpt2_create. */
TQ_EXPORT int tq_gpt2_load_tensor(uint64_t model, const char *name, const void *data, int dtype, int rows, int cols);

/* How tq_gpt2_generate picks each generated token: temp <= 0 (the default)
 * greedy; temp > 0 the examples' sample step (main.go:78-105, tq_sample)
 * with draws[k], the caller's rng.Float64() for generated token k, so
 * tq_gpt2_generate then needs n_gen <= n_draws (the draws are copied; every
 * generate call starts again from draws[0]). TQ_ERR_ARG for a NaN
 * temperature or temp > 0 without draws in [0, 1]. */
TQ_EXPORT int tq_gpt2_set_sampling(uint64_t model, double temp, const double *draws, int n_draws);

/* Releases a model (a second call is a no-op). */
TQ_EXPORT int tq_gpt2_free(uint64_t model);

/* ---- whole-model decode: Qwen2 (int4 weights), tensor parallel ------------- */

/* Shape of a Qwen2 model (_example/qwen/model.go:20-32): layers, query and
 * KV heads (grouped-query attention; head size d/n_head, even), hidden
 * width d, MLP width, vocabulary, context length, RMSNorm epsilon, RoPE
 * theta. The lm head is untied. */
typedef struct {
    int n_layer, n_head, n_kv, d, ffn, vocab, ctx;
    double eps, theta;
} tq_qwen_config;

#define TQ_NCCL_ID_BYTES 128

/* Writes a fresh NCCL unique id (TQ_NCCL_ID_BYTES bytes) for
 * tq_qwen_create: rank 0 makes it and every rank receives a copy. */
TQ_EXPORT int tq_nccl_unique_id(void *id);

/* Builds this rank's shard of a random-init Qwen2 on the current device
 * (one process per GPU; all ranks call it together when world > 1): every
 * matrix in the reference's [in, out] orientation drawn from the
 * tq_synth_dev generator with standard deviation sigma (streams: embedding
 * 1, lm head 2, layer l: q 32+16l, k +1, v +2, o +3, gate +4, up +5,
 * down +6), norm weights 1, biases 0, quantized with QuantizeMatrix4 per
 * shard (quantizeMat, model.go:40-52). q/k/v and gate/up are column-sharded,
 * o_proj and down row-sharded on 64-row groups, the lm head column-sharded;
 * world must divide or be a multiple of n_kv, and d/world, ffn/world be
 * multiples of 64. nccl_id: from tq_nccl_unique_id (NULL when world == 1).
 * Replaces loadQwen (model.go:95-177) for synthetic weights. */
TQ_EXPORT int tq_qwen_create(const tq_qwen_config *cfg, uint64_t seed, float sigma, int rank, int world,
                             const void *nccl_id, uint64_t *model);

/* Greedy generation (main.go:225-240 at temperature 0, no end-of-turn
 * stop): the prompt through the decode step one token at a time, then n_gen
 * greedy tokens into tokens[0..n_gen). Collective over the ranks of a
 * tensor-parallel model. times_ms (optional, 2 floats): device time of the
 * prompt steps and of the n_gen - 1 later steps. */
TQ_EXPORT int tq_qwen_generate(uint64_t model, const int *prompt, int n_prompt, int n_gen, int *tokens,
                               float *times_ms);

/* A one-GPU Qwen2 model whose weights come from a checkpoint instead of the
 * random-init generator: matrices zeroed, norm weights 1, biases 0, until
 * tq_qwen_load_tensor fills them (loadQwen, _example/qwen/model.go:95-177). */
TQ_EXPORT int tq_qwen_create_empty(const tq_qwen_config *cfg, uint64_t *model);

/* One checkpoint tensor, by its Hugging Face name, from device memory in its
 * stored layout and type (TQ_LINEAR_F32 / F16 / BF16; Linear weights
 * [out, in] = rows x cols, vectors 1 x n): model.embed_tokens.weight (widened
 * to float32), lm_head.weight (a tied checkpoint passes the embedding under
 * this name), model.norm.weight, and per layer model.layers.N. +
 * self_attn.{q,k,v}_proj.{weight,bias}, self_attn.o_proj.weight,
 * mlp.{gate,up,down}_proj.weight, input_layernorm.weight,
 * post_attention_layernorm.weight. Linear weights are quantized on the device
 * as QuantizeMatrix4 of Matrix().T() (the q|k|v and gate|up parts once all of
 * a fused matrix arrived). Synchronous; the caller may free data on return.
 * TQ_ERR_SHAPE for a wrong shape, TQ_ERR_ARG for an unknown name or a model
 * made by tq_qwen_create. */
TQ_EXPORT int tq_qwen_load_tensor(uint64_t model, const char *name, const void *data, int dtype, int rows, int cols);

/* How tq_qwen_generate processes the prompt. rows = 0 (the default) feeds it
 * token by token through the decode step, as the reference does
 * (_example/qwen/main.go:229-231): the parity mode. rows in 16..64 runs it in
 * chunks of that many prompt positions, each layer's matvecs as rows-row
 * matmuls on the tf32 tensor-core kernel (2e-3 relative L2 per matmul against
 * the float32 products), RoPE, caches and attention row by row with the
 * step's numerics; the generated ids may then differ from the parity mode's.
 * TQ_ERR_UNSUPPORTED when a GPU's shard repeats the attention (more GPUs
 * than KV heads) or the context exceeds the batched attention's shared
 * memory. */
TQ_EXPORT int tq_qwen_set_prefill(uint64_t model, int rows);

/* tq_gpt2_set_sampling for a Qwen2 model (main.go:115-150); one GPU only
 * (TQ_ERR_UNSUPPORTED when world > 1: the lm head is split by vocabulary).
 * During a token-by-token prompt every step runs the sample step too (its
 * result is discarded until the prompt's last position). */
TQ_EXPORT int tq_qwen_set_sampling(uint64_t model, double temp, const double *draws, int n_draws);

/* How the ranks of a tensor-parallel model exchange partial sums in the
 * decode step: *kind = TQ_EXCHANGE_NONE (world 1), TQ_EXCHANGE_NCCL (NCCL
 * all-reduce and all-gather) or TQ_EXCHANGE_PEER (one kernel per exchange
 * that stores this rank's partial into every peer's memory over NVLink,
 * sums all ranks' partials in rank order and applies the residual add and
 * RMSNorm after it; the candidates of the lm head likewise). tq_qwen_create
 * picks PEER when every rank can map every other rank's memory (CUDA IPC,
 * at most 8 GPUs) unless the environment variable TENSAI_QWEN_EXCHANGE is
 * "nccl" on a rank. A peer that does not arrive within 2 s fails
 * tq_qwen_generate with TQ_ERR_TIMEOUT. The batched prefill's all-reduces
 * use NCCL either way. */
#define TQ_EXCHANGE_NONE 0
#define TQ_EXCHANGE_NCCL 1
#define TQ_EXCHANGE_PEER 2
TQ_EXPORT int tq_qwen_exchange(uint64_t model, int *kind);

/* Releases a model and its NCCL communicator (a second call is a no-op). */
TQ_EXPORT int tq_qwen_free(uint64_t model);

/* The shard of the model that rank `rank` of `world` GPUs holds, as
 * tq_qwen_create computes it: plan[0..11] = query heads [a, b), KV heads
 * [a, b), o_proj rows [a, b), attention output dims [a, b), MLP columns
 * (gate/up, = down rows) [a, b), lm-head columns [a, b). The Go loader of a
 * sharded checkpoint slices its tensors with it (loadQwen, model.go:95-177,
 * per rank). Errors as tq_qwen_create's for configurations that do not split
 * over world GPUs. Needs no GPU. */
TQ_EXPORT int tq_qwen_shard_plan(const tq_qwen_config *cfg, int world, int rank, int *plan);

/* The examples' sample step (_example/gpt2/main.go:78-105, the same
 * function as _example/qwen/main.go:115-150) on the current device, for the
 * host logits[0..n): temp <= 0 gives the first index of the largest logit;
 * otherwise p_i = exp(float64(logits_i - max) / temp), the candidates sorted
 * by p descending, r = u * sum(p), and *token = the first candidate at which
 * r -= p reaches <= 0 (else the first candidate). u is the caller's uniform
 * draw, rng.Float64() in the Go code (used only when temp > 0; must lie in
 * [0, 1]). Equal weights are taken in ascending id order (Go's unstable sort
 * leaves them unspecified); the sum of p is added in a fixed tree order, not
 * index order, so r can differ from the Go code's in the last bits.
 * Synchronous. TQ_ERR_ARG for n < 1, a NaN temperature or u out of range. */
TQ_EXPORT int tq_sample(const float *logits, int n, double temp, double u, int *token);

/* Seeded uniform token ids in [0, vocab) on the host: id i =
 * mix64(key + (i+1)*0x9E3779B97F4A7C15) % vocab with the generator key of
 * (seed, stream 3). A stand-in for a tokenized prompt. */
TQ_EXPORT int tq_synth_tokens(int *out, int n, int vocab, uint64_t seed);

/* ---- host-side fault injection (tests) ------------------------------------ */

/* Makes the next n device allocations made by this library fail with
 * TQ_ERR_NOMEM, so error paths can be tested without touching the GPU. */
TQ_EXPORT int tq_debug_fail_allocs(int n);

#ifdef __cplusplus
}
#endif

#endif /* TENSAI_CUDA_H */
