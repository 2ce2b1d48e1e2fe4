/*
 * smallm_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for smallm-engine.
 *
 * Two levels, both plain C (pointers, sizes, status codes; no C++ or CUDA
 * types in the signatures, streams are passed as void*):
 *
 *  1. Op level -- the six operations of smallm::Backend
 *     (include/smallm/backend/common/backend.h:12-38 in smallm-engine), with
 *     the same argument meaning.  The smallm_backend_* calls take HOST
 *     pointers exactly like the reference interface (each call copies its
 *     operands to the GPU and the result back).  The device-pointer calls
 *     (smallm_qmatrix_*, smallm_gemv) are the same math on device-resident
 *     operands, for callers that keep their activations on the GPU.
 *
 *  2. Model level -- a device-resident Qwen2/Llama decoder behind the
 *     smallm::Model contract (include/smallm/model/common/model.h:16-43):
 *     forward(token, pos) -> logits, reset_cache, truncate_cache,
 *     cached_length.  Weights are read once from the GGUF file, repacked for
 *     coalesced 128-bit loads and kept in HBM with an f32 KV cache; the
 *     whole per-token step is one CUDA graph.
 *
 * Conventions
 *  - Every function returns SMALLM_OK (0) or a positive SMALLM_ERR_* code;
 *    smallm_last_error() returns the message of the calling thread's last
 *    failure.  The reference throws std::runtime_error at the same points.
 *  - There is no CPU fallback: without a usable sm_100 device every call
 *    fails with SMALLM_ERR_CUDA.
 *  - A context or model is used by one host thread at a time.
 *
 * GGML tensor type ids (include/smallm/core/tensor.h:14-20, plus Q4_K = 12,
 * which the reference does not implement): F32 = 0, Q4_0 = 2, Q8_0 = 8,
 * Q4_K = 12, Q6_K = 14.  Any other type is rejected with
 * SMALLM_ERR_UNSUPPORTED_TYPE (the reference's GEMV instead reads unknown
 * types as F32, src/core/ops.cpp:289-299).
 */
#ifndef SMALLM_CUDA_H
#define SMALLM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SMALLM_OK 0
#define SMALLM_ERR_INVALID 1          /* bad argument or shape */
#define SMALLM_ERR_UNSUPPORTED_TYPE 2 /* tensor type not in {0, 2, 8, 12, 14} */
#define SMALLM_ERR_CUDA 3             /* CUDA runtime error / no device */
#define SMALLM_ERR_IO 4               /* cannot open / map the GGUF file */
#define SMALLM_ERR_FORMAT 5           /* malformed GGUF, missing key or tensor */
#define SMALLM_ERR_NCCL 6             /* tensor-parallel communication failed */
#define SMALLM_ERR_RANGE 7            /* position beyond the context length */

#define SMALLM_TYPE_F32 0u
#define SMALLM_TYPE_Q4_0 2u
#define SMALLM_TYPE_Q8_0 8u
#define SMALLM_TYPE_Q4_K 12u
#define SMALLM_TYPE_Q6_K 14u

/* Message of the calling thread's last failure ("" if none). */
const char* smallm_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int smallm_version(void);

/* ------------------------------------------------------------------ */
/* Op level                                                            */
/* ------------------------------------------------------------------ */

typedef struct smallm_ctx smallm_ctx;

/* A context owns one CUDA stream on `device` and a cache of device copies of
 * host weight matrices keyed by host pointer (the reference hands the
 * backend the same stable mmap pointer for a weight on every call,
 * src/model/qwen2_model.cpp:93-95). */
int smallm_ctx_create(int device, smallm_ctx** out);
int smallm_ctx_destroy(smallm_ctx* ctx);
/* The context's cudaStream_t. */
void* smallm_ctx_stream(smallm_ctx* ctx);
int smallm_ctx_synchronize(smallm_ctx* ctx);

/* Backend::matmul (backend.h:17-18): y[rows] = W[rows, cols] . x[cols], f32,
 * host pointers, any cols (cols == 0 gives zeros; rows == 0 does nothing). */
int smallm_backend_matmul(smallm_ctx* ctx, const float* W, const float* x, uint32_t rows,
                          uint32_t cols, float* y);

/* Backend::matmul_quantized (backend.h:21-23; ops.cpp:97-300): W is `rows`
 * rows of GGUF blocks of `type` (row-major [out][in], as the reference
 * consumes GGUF weights), x f32[cols], y f32[rows], host pointers.  The
 * first call with a given W uploads and repacks it; later calls reuse the
 * device copy (the caller must not change the bytes behind W).  As in the
 * reference, a quantized row holds only whole blocks (cols / 32, or cols / 256
 * for the K types), so columns past the last whole block are ignored and a
 * row with no whole block gives 0.  Unlike the reference, whose fallback reads
 * any type other than Q8_0 / Q4_0 / Q6_K as F32 (ops.cpp:283-293), Q4_K is
 * computed as Q4_K and unknown types return SMALLM_ERR_UNSUPPORTED_TYPE. */
int smallm_backend_matmul_quantized(smallm_ctx* ctx, const uint8_t* W, uint32_t type,
                                    const float* x, uint32_t rows, uint32_t cols, float* y);

/* Backend::rmsnorm (backend.h:26-27; ops.cpp:29-40): y = x / rms(x) * w. */
int smallm_backend_rmsnorm(smallm_ctx* ctx, const float* x, const float* weight, uint32_t size,
                           float eps, float* y);

/* Backend::softmax (backend.h:30; ops.cpp:43-57), in place. */
int smallm_backend_softmax(smallm_ctx* ctx, float* x, uint32_t size);

/* Backend::silu (backend.h:33; ops.cpp:60-65), in place. */
int smallm_backend_silu(smallm_ctx* ctx, float* x, uint32_t size);

/* Backend::rope (backend.h:36-37; ops.cpp:68-92): NeoX rotation of pairs
 * (i, i + head_dim/2) of each head, in place. */
int smallm_backend_rope(smallm_ctx* ctx, float* x, uint32_t n_heads, uint32_t head_dim,
                        uint32_t pos, float freq_base);

/* Forget every cached weight copy of the context. */
int smallm_ctx_clear_weights(smallm_ctx* ctx);

/* ---- device-resident operands ---- */

typedef struct smallm_qmatrix smallm_qmatrix;

/* Upload a quantized (or F32) matrix from host memory and repack it into the
 * device layout the GEMV kernels stream (src/core/tensor.cpp:140-152 is the
 * view the reference keeps instead). */
int smallm_qmatrix_upload(smallm_ctx* ctx, const uint8_t* W, uint32_t type, uint32_t rows,
                          uint32_t cols, smallm_qmatrix** out);
int smallm_qmatrix_free(smallm_qmatrix* m);
/* Bytes of the GGUF encoding of the matrix (the algorithmic bytes a GEMV
 * reads) and bytes it occupies on the device. */
int smallm_qmatrix_bytes(const smallm_qmatrix* m, uint64_t* gguf_bytes, uint64_t* device_bytes);

/* y_dev[rows] = W . x_dev[cols] on `stream` (NULL = the context stream).
 * Asynchronous; device pointers. */
int smallm_gemv(smallm_ctx* ctx, const smallm_qmatrix* W, const float* x_dev, float* y_dev,
                void* stream);

/* Tensor-core GEMM (tcgen05, sm_100a) of the batched prefill on device
 * operands: y_dev[t * ldy + n] = sum_k x_dev[t * K + k] * w_dev[n * K + k]
 * for t < T, n < N.  w_dev [N][K] and x_dev [T][K] are row-major IEEE half
 * (uint16 bit patterns, 16-byte aligned, K a positive multiple of 8); the
 * products are exact and accumulate in f32.  This is the contraction the
 * reference performs as matmul_quantized once per prompt token
 * (src/core/ops.cpp:103-184 via src/runtime/generator.cpp:47-51), here over T
 * tokens at once on dequantized (f16-rounded) weights.  A bounded wait that
 * gives up raises bit 6 of the device error word (smallm_ctx_device_errors).
 * Asynchronous on `stream` (NULL = the context stream). */
int smallm_gemm_f16(smallm_ctx* ctx, const uint16_t* w_dev, const uint16_t* x_dev, uint32_t N, uint32_t K,
                    uint32_t T, float* y_dev, uint32_t ldy, void* stream);

/* The tensor-parallel residual step of the decode path as one call (what the
 * decode step's QKV, gate/up and lm_head GEMVs do under tensor parallelism):
 *   x_out = x_res + parts[0] + ... + parts[n_parts-1]   (f32, in that order)
 *   y     = W . (x_out * norm_w / rms(x_out))           (ops::rmsnorm, src/core/ops.cpp:29-40)
 * once every arrival flag flags[r] equals *epoch + 1 (the value a sender
 * stores after its part is complete).  parts is [n_parts][cols] f32,
 * n_parts in 1..8; x_out may be written by any one CTA.  The flag wait is
 * bounded (about one second): when it gives up, bit 3 of the device error
 * word is raised and y / x_out are not valid (smallm_ctx_device_errors).
 * Asynchronous on `stream` (NULL = the context stream); device pointers. */
int smallm_gemv_residual_sum(smallm_ctx* ctx, const smallm_qmatrix* W, const float* x_res_dev,
                             const float* parts_dev, uint32_t n_parts, const uint32_t* flags_dev,
                             const uint32_t* epoch_dev, const float* norm_w_dev, float eps, float* x_out_dev,
                             float* y_dev, void* stream);

/* The device error word that the bounded waits of the GEMV and attention
 * kernels raise when they give up (0 = none): bit 0 a GEMV producer's stage
 * wait, bits 1-2 a GEMV or attention pipeline wait, bit 3 a residual part's
 * arrival flag, bit 5 the decode position changed during a step.  Waits for
 * the device; clear != 0 resets the word. */
int smallm_ctx_device_errors(smallm_ctx* ctx, uint32_t* flags, int clear);

/* Dequantize the matrix from its device layout into y_dev[rows * cols]
 * (row-major), bit-identical to the reference's dequantize_tensor
 * (src/core/tensor.cpp:115-138). */
int smallm_qmatrix_dequantize(smallm_ctx* ctx, const smallm_qmatrix* W, float* y_dev, void* stream);

/* Dequantize `count` elements of GGUF blocks of `type` (host in, host out),
 * bit-identical to dequantize_tensor. */
int smallm_dequantize(smallm_ctx* ctx, uint32_t type, const uint8_t* src, uint64_t count, float* out);

/* Decode attention that allocates nothing.  No counterpart in the reference
 * (there, attention is a loop inside each model's forward,
 * src/model/qwen2_model.cpp:111-133).
 *
 * out_dev[n_heads * head_dim] = softmax(q . K^T / sqrt(head_dim)) . V over
 * positions 0..pos, query head h reading KV head h / (n_heads / n_kv_heads):
 * a split-K decode-attention kernel (partials merged by the last CTA of each
 * KV head; a loaded model runs a cluster variant), on caller-owned device buffers
 * q_dev[n_heads * head_dim] and kcache_dev / vcache_dev laid out
 * [n_kv_heads][max_ctx][head_dim] (f32; kcache_dev and vcache_dev 16-byte
 * aligned, since their rows are bulk-copied, else SMALLM_ERR_INVALID).
 * Asynchronous on `stream` (NULL = the context stream).
 *
 * For callers that cannot let the library allocate device memory (a serving
 * engine whose memory all belongs to its own KV pool; a loop that cannot absorb
 * the device synchronisation cudaMalloc / cudaFree may cause): the kernel's
 * scratch (split-K partials, per-KV-head tickets) is one static 4 MiB + 1 KiB
 * array inside the library, not a buffer; pos travels as a kernel parameter.
 *   - The first call on each device does one-time set-up on that device (looks
 *     up the array's address and zeroes the tickets on `stream`); make it
 *     before any stream capture begins.
 *   - Calls on one device share the array: calls whose kernels overlap in time
 *     (different streams or threads) race and must be ordered by the caller.
 *   - Limits: n_kv_heads <= 256; n_heads / n_kv_heads <= 8 and a whole
 *     number; head_dim 32, 64 or 128; pos < max_ctx; and the partials,
 *     4 * n_heads * (head_dim + 2) bytes per split, fit in 4 MiB (about
 *     max_ctx 16128 at 32 heads of 128).  Beyond them the call returns
 *     SMALLM_ERR_RANGE (or SMALLM_ERR_INVALID for an unsupported shape) and
 *     launches nothing. */
int smallm_attention_noalloc(smallm_ctx* ctx, const float* q_dev, const float* kcache_dev,
                             const float* vcache_dev, uint32_t n_heads, uint32_t n_kv_heads,
                             uint32_t head_dim, uint32_t max_ctx, uint32_t pos, float* out_dev,
                             void* stream);

/* Samplers (src/runtime/sampler/*.cpp): one token from `n` HOST logits.
 * kind 0 = GreedySampler (first maximum), 1 = TemperatureSampler(temperature),
 * 2 = TopKSampler(k, temperature), 3 = TopPSampler(p, temperature).  `u` is
 * the uniform the reference sampler would draw for this call
 * (std::uniform_real_distribution<float>(0, 1) on its std::mt19937; ignored
 * for greedy), so the caller owns the random stream.  k must be >= 1 for
 * top-k (the reference's k = 0 reads out of bounds). */
#define SMALLM_SAMPLE_GREEDY 0u
#define SMALLM_SAMPLE_TEMPERATURE 1u
#define SMALLM_SAMPLE_TOP_K 2u
#define SMALLM_SAMPLE_TOP_P 3u
int smallm_sample(smallm_ctx* ctx, const float* logits, uint32_t n, uint32_t kind, uint32_t k, float p,
                  float temperature, float u, uint32_t* token);

/* ------------------------------------------------------------------ */
/* Model level                                                         */
/* ------------------------------------------------------------------ */

typedef struct smallm_model smallm_model;

typedef struct smallm_model_opts {
    int device;            /* CUDA device ordinal */
    uint32_t max_ctx;      /* KV capacity in positions; 0 = GGUF <arch>.context_length */
    int tp_rank;           /* tensor-parallel rank (0 when tp_size == 1) */
    int tp_size;           /* tensor-parallel degree: 1, 2, 4 or 8 */
    const void* nccl_id;   /* 128-byte ncclUniqueId shared by all ranks (tp_size > 1) */
    uint32_t flags;        /* reserved, 0 */
} smallm_model_opts;

typedef struct smallm_model_info {
    char arch[16];         /* "qwen2" or "llama" */
    uint32_t n_layers, embd, ffn, n_heads, n_kv_heads, head_dim, vocab, context_length;
    uint32_t max_ctx;      /* KV capacity actually allocated */
    float rope_freq_base, rms_eps;
    uint64_t weight_bytes_per_token; /* GGUF bytes of every matrix a decode step reads
                                        (this rank's share under tensor parallelism) */
    uint64_t device_bytes; /* device memory held by the model */
    uint32_t step_launches; /* kernel launches of one decode step: 1 when the whole
                               step runs as one persistent kernel, else one per op */
    uint32_t reserved;
} smallm_model_info;

/* Parse `gguf_path` (src/core/gguf.cpp:116-183, src/config/common/config.cpp
 * :14-48) and build a device-resident model: Qwen2Model / LlamaModel
 * (src/model/qwen2_model.cpp:28-65, llama_model.cpp:17-49).  Same required
 * keys and tensors as the reference; output.weight is required. */
int smallm_model_load(const char* gguf_path, const smallm_model_opts* opts, smallm_model** out);
int smallm_model_free(smallm_model* m);
int smallm_model_get_info(const smallm_model* m, smallm_model_info* out);
/* The model's cudaStream_t (all model work is ordered on it). */
void* smallm_model_stream(smallm_model* m);

/* Model::forward (model.h:22): one token at `pos`; writes vocab logits to
 * host memory `logits` (may be NULL to skip the copy) and, when `argmax` is
 * not NULL, the first index of the maximum logit (greedy_sampler.cpp:8-14).
 * Updates cached_length to pos + 1 like qwen2_model.cpp:196. */
int smallm_model_forward(smallm_model* m, uint32_t token, uint32_t pos, float* logits,
                         uint32_t* argmax);

/* Model::reset_cache / truncate_cache / cached_length (model.h:25-34). */
int smallm_model_reset_cache(smallm_model* m);
int smallm_model_truncate_cache(smallm_model* m, uint32_t n);
uint32_t smallm_model_cached_length(const smallm_model* m);

/* Greedy decode entirely on the device: step i feeds the argmax of step i-1
 * (the first step feeds `token`) at positions pos, pos+1, ...  Enqueues
 * n_steps graph launches without host synchronisation; ids of the n_steps
 * generated tokens are read back with smallm_model_decode_ids. */
int smallm_model_decode_greedy_async(smallm_model* m, uint32_t token, uint32_t pos,
                                     uint32_t n_steps);
/* Wait for the decode and copy the `n` ids it produced to host `ids`. */
int smallm_model_decode_ids(smallm_model* m, uint32_t* ids, uint32_t n);

/* Batched prefill: tokens[0..n) at positions start_pos .. start_pos + n - 1
 * in one pass per layer (GEMMs over the n tokens; the reference calls
 * Model::forward once per prompt token, src/runtime/generator.cpp:47-51).
 * Fills the KV cache like n forward calls and returns the last token's
 * logits (host `logits`, may be NULL) and greedy id (`argmax`, may be NULL);
 * cached_length becomes start_pos + n.  Single GPU (tp_size 1).  The GEMMs
 * run on the backend's own tcgen05 tensor-core kernel (smallm_gemm_f16) over
 * f16 copies of the layer weights (2 bytes per weight, made at the first
 * call from the exactly dequantized values) and f16-rounded activations
 * (11-bit significands; f16 range, |x| < 65504), with f32 accumulation.
 * flags: 0, or SMALLM_PREFILL_TC (the same path, named); any other bit is
 * SMALLM_ERR_INVALID. */
#define SMALLM_PREFILL_TC 2u
int smallm_model_prefill(smallm_model* m, const uint32_t* tokens, uint32_t n, uint32_t start_pos, float* logits,
                         uint32_t* argmax, uint32_t flags);

/* The same samplers on the last step's logits, on the device (no logits
 * copy); under tensor parallelism the vocabulary shards are gathered first. */
int smallm_model_sample(smallm_model* m, uint32_t kind, uint32_t k, float p, float temperature, float u,
                        uint32_t* token);

/* Device address of the last step's logits (f32[vocab] on this rank's
 * device; this rank's vocabulary shard under tensor parallelism), valid
 * until the next step is enqueued. */
const float* smallm_model_logits_device(smallm_model* m);

/* Tracing (the reference only times the decode loop with steady_clock,
 * src/runtime/generator.cpp:57-68): run one step like smallm_model_forward
 * (no logits copy) through a copy of the step graph whose kernels stamp the
 * GPU global timer.  Writes up to `cap` records of 4 uint64 each to `out`:
 * start of the kernel's first CTA, first CTA past its wait on the previous
 * kernel, end of its last CTA (ns, relative to the first record's start),
 * and a kind code (1 embed, 2 QKV, 3 V, 4 attention, 5 O, 6 gate/up,
 * 7 down, 8 lm_head, 9 finalize).  *n receives the number of kernels.
 * When the model runs the persistent step (one kernel per step), there is one
 * record per op of that kernel instead (earliest CTA at the op, earliest CTA
 * past its barrier, latest CTA done), followed by CTA 0's weight pieces: kind
 * 1000 records hold (copy started, data seen in shared memory, piece
 * retired) and the kind 1001 record after each holds, as its start, the time
 * the piece's last warp finished it. */
int smallm_model_trace_step(smallm_model* m, uint32_t token, uint32_t pos, uint64_t* out, uint32_t cap,
                            uint32_t* n);

/* ------------------------------------------------------------------ */
/* Helpers (no counterpart in the reference, which is single-process)   */
/* ------------------------------------------------------------------ */

/* Write a fresh 128-byte ncclUniqueId to `out` (rank 0 creates it and shares
 * it with the other ranks out of band, e.g. over torch.distributed). */
int smallm_nccl_unique_id(void* out);

/* Page-locked host memory for inputs/outputs that cross the PCIe/C2C link
 * every step. */
int smallm_host_alloc(size_t bytes, void** out);
int smallm_host_free(void* p);

#ifdef __cplusplus
}
#endif

#endif /* SMALLM_CUDA_H */
