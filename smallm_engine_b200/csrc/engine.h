// Internal host-side interface of the CUDA backend (not part of the C ABI).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "trace.h"

namespace smallm {

// Error carrying one of the SMALLM_ERR_* codes of include/smallm_cuda.h.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void cuda_check(cudaError_t e, const char* what);
#define SM_CUDA(call) ::smallm::cuda_check((call), #call)

// Elements per block and bytes per block of a GGUF type; 0 when unsupported.
uint32_t type_block_elems(uint32_t type);
uint32_t type_block_bytes(uint32_t type);
bool type_supported(uint32_t type);
uint64_t type_row_bytes(uint32_t type, uint64_t cols);

// A matrix repacked into the device layout the GEMV kernels stream: every
// storage row is one contiguous record of row_stride bytes (a multiple of
// 16), so any run of consecutive rows is one contiguous range:
//   F32   [cols][f32]
//   Q4_0  [units][16 B nibbles] [units][f16 d]          (+ pad)   unit = 32 elements
//   Q8_0  [units][32 B int8]    [units][f16 d]          (+ pad)   unit = 32
//   Q4_K  [nsb][144 B GGUF super-block]                           unit = 64
//   Q6_K  [units][48 B codes]   [units][4 x i8 scales] [nsb][f16 d] (+ pad)  unit = 64
struct QMat {
    uint32_t type = 0;
    uint32_t rows = 0;        // logical rows
    uint32_t rows_pad = 0;    // storage rows (multiple of 32; the extra rows are zero)
    uint32_t cols = 0;
    uint32_t units = 0;       // cols / elements-per-unit of the format
    uint32_t row_stride = 0;  // bytes per storage row
    uint8_t* base = nullptr;  // rows_pad * row_stride bytes
    uint64_t dev_bytes = 0;
    uint64_t gguf_bytes = 0;  // bytes of the same rows in GGUF encoding
};

// Where the rows of a QMat come from: `src` holds GGUF rows of `src_cols`
// elements (device memory, any alignment); physical row p of the QMat is
// source row row_map[p] (UINT32_MAX = zero row), columns
// [col0, col0 + cols) of it.
struct RepackSource {
    const uint8_t* src = nullptr;
    uint64_t src_cols = 0;
    uint64_t col0 = 0;
    const uint32_t* row_map = nullptr;  // device array of rows_pad entries, or null = identity
};

// Allocate `m` for (type, rows, cols) and fill it from `s` on `stream`.
void qmat_alloc(QMat& m, uint32_t type, uint32_t rows, uint32_t cols);
void qmat_repack(QMat& m, const RepackSource& s, cudaStream_t stream);
void qmat_free(QMat& m);

// Upload host GGUF rows (rows x src_cols, row-major) and repack them; the
// helper stages through a temporary device buffer.  row_map (host, may be
// empty = identity) has one entry per storage row.
void qmat_upload(QMat& m, const uint8_t* host, uint32_t type, uint32_t rows, uint32_t cols,
                 uint64_t src_cols, uint64_t col0, const std::vector<uint32_t>& row_map,
                 cudaStream_t stream);

enum GemvPro { GEMV_PRO_PLAIN = 0, GEMV_PRO_RMS = 1, GEMV_PRO_RMS_SUM = 2, GEMV_PRO_MERGE = 3 };
enum GemvEpi { GEMV_EPI_STORE = 0, GEMV_EPI_RESIDUAL = 1, GEMV_EPI_QKV = 2, GEMV_EPI_SWIGLU = 3,
               GEMV_EPI_LOGITS = 4, GEMV_EPI_PEER = 5 };
constexpr int kMaxTPRanks = 8;

// Everything a GEMV launch needs besides the matrix (see gemv.cuh).
struct GemvArgs {
    const float* x = nullptr;
    const float* norm_w = nullptr;
    float eps = 0.f;
    float* y = nullptr;
    const float* bias = nullptr;
    uint32_t q_rows = 0, k_rows = 0, head_dim = 0, max_ctx = 0;
    float* qout = nullptr;
    float* kcache = nullptr;
    float* vcache = nullptr;
    const float2* rope = nullptr;
    const uint32_t* pos = nullptr;
    unsigned long long* argmax = nullptr;
    uint32_t row_offset = 0;  // LOGITS: global index of storage row 0 (vocab-parallel shards)
    TraceSlot* trace = nullptr;  // traced steps only
    // tensor-parallel residual through peer memory (gemv.cuh, GemvParams)
    const float* x_res = nullptr;
    float* x_out = nullptr;
    const float* rx = nullptr;
    const unsigned int* rx_flag = nullptr;
    float* peer_out[kMaxTPRanks] = {};
    unsigned int* peer_flag[kMaxTPRanks] = {};
    unsigned int* done_ctr = nullptr;
    const unsigned int* epoch = nullptr;
    uint32_t tp = 1;
    // Shared memory the launch may use (0: the 227 KB limit).  The decode
    // step caps the QKV and O GEMVs so the attention kernel's CTAs fit next
    // to theirs (it stages cached K/V while the QKV GEMV runs, and the O
    // GEMV prefetches weights while attention runs).
    size_t smem_cap = 0;
    // GEMV_PRO_MERGE: x is the merge of merge_parts attention partials
    // (x + k * cols, weighted per head of merge_hd elements by merge_ml)
    uint32_t merge_parts = 1, merge_hd = 0;
    const float* merge_ml = nullptr;
};

void launch_gemv(const QMat& m, int pro, int epi, const GemvArgs& a, cudaStream_t stream, bool pdl = false);

// cudaFuncAttributeMaxDynamicSharedMemorySize of `fn` on the current device,
// set once per (device, kernel, size) under a lock.
void set_smem_limit_once(const void* fn, int bytes);

// Pipeline shape the GEMV uses for a matrix: rows per tile, stages of the
// shared-memory ring, bytes of staged x, total dynamic shared memory.
struct GemvPlan {
    uint32_t rt = 0, stages = 0, ngroups = 0, gsize = 0, kring = 0, warps = 0;
    size_t xbytes = 0, smem = 0;
};
GemvPlan gemv_plan(const QMat& m, size_t smem_cap = 0);

// Error bits raised by GEMV kernels whose bounded waits gave up (0 = none).
unsigned int gemv_error_flags(bool clear);

// Dequantize a QMat to f32 [rows][cols] (bit-identical to the reference).
void launch_qmat_dequant(const QMat& m, float* y, cudaStream_t stream);
// Dequantize raw GGUF blocks on the device (bit-identical to the reference).
void launch_dequant_raw(uint32_t type, const uint8_t* src, uint64_t count, float* out, cudaStream_t stream);

// Decode-step state kept in device memory so a captured graph can replay.
struct DecodeState {
    uint32_t token;
    uint32_t pos;
    uint32_t step;        // ids written so far by finalize
    uint32_t pad;
    unsigned long long argmax;
};

// x[embd] = dequantized row state->token of the embedding matrix; resets the
// argmax slot.
void launch_embed(const QMat& emb, DecodeState* st, float* x, cudaStream_t stream, bool pdl = false,
                  TraceSlot* trace = nullptr);
// state->token = argmax, ids[state->step++] = token, state->pos += 1.
void launch_finalize(DecodeState* st, uint32_t* ids, uint32_t ids_cap, cudaStream_t stream, bool pdl = false,
                     TraceSlot* trace = nullptr);
// Same, taking the maximum of the `n` gathered per-rank argmax keys.
// Also counts the step in *epoch (the tensor-parallel flags carry it).
void launch_finalize_tp(DecodeState* st, const unsigned long long* keys, int n, uint32_t* ids,
                        uint32_t ids_cap, unsigned int* epoch, cudaStream_t stream, bool pdl = false);

// Split-K GQA decode attention over the head-major f32 KV cache, with the
// per-head combine done by the last CTA of each KV head.
struct AttnArgs {
    const float* q;        // [n_heads * hd] (after RoPE)
    const float* kcache;   // [n_kv][max_ctx][hd]
    const float* vcache;
    float* out;            // [n_heads * hd]
    float* partial;        // scratch: [n_kv][n_split][group][hd + 2]
    unsigned int* counter; // scratch: [n_kv], zero between launches
    const uint32_t* pos;   // attend over positions 0..*pos (null: 0..pos_value)
    uint32_t pos_value = 0;
    uint32_t n_heads, n_kv, hd, max_ctx, n_split;
    unsigned int* err = nullptr;  // raised if a bounded wait gives up
    TraceSlot* trace = nullptr;   // traced steps only
    uint32_t chunk = 32;          // cluster kernel: positions per chunk (attention_cluster_chunk)
    // cluster kernel, parts > 1 clusters per KV head (attention_cluster_parts):
    // part k writes its normalised output to part_out [parts][n_heads * hd]
    // and its (max, sum) per head to part_ml [parts][n_heads][2]; the next
    // GEMV merges them while it stages x (GemvArgs::merge_*)
    uint32_t parts = 1;
    float* part_out = nullptr;
    float* part_ml = nullptr;
};
uint32_t attention_splits(uint32_t n_kv, uint32_t max_ctx, int sm_count);
size_t attention_partial_floats(uint32_t n_heads, uint32_t hd, uint32_t n_split);
size_t attention_smem(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t max_ctx, uint32_t n_split);
void launch_attention(const AttnArgs& a, cudaStream_t stream, bool pdl = false);
// Cluster attention (the decode step's): one cluster of C CTAs per KV head,
// partials merged through distributed shared memory.  attention_cluster_size
// picks the largest C <= 16 the device can schedule (and sets the kernel's
// attributes on the current device) for chunks of `chunk` positions;
// attention_cluster_chunk sizes them for contexts up to max_ctx.
uint32_t attention_cluster_size(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t chunk);
uint32_t attention_cluster_chunk(uint32_t max_ctx, uint32_t C, uint32_t hd, uint32_t parts);
uint32_t attention_cluster_parts(uint32_t n_kv, uint32_t C, uint32_t max_ctx, int sm_count);
// Dynamic shared memory of one cluster-attention CTA.
size_t attention_cluster_smem(uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t chunk);
void launch_attention_cluster(const AttnArgs& a, uint32_t C, cudaStream_t stream, bool pdl);
// The split-K kernel with its scratch in a static array of attention.cu (no
// allocation; calls that overlap in time race on it).
void launch_attention_static(const float* q, const float* kcache, const float* vcache, uint32_t n_heads,
                             uint32_t n_kv, uint32_t hd, uint32_t max_ctx, uint32_t pos, float* out,
                             cudaStream_t stream);

// cudaLaunchKernelExC with optional programmatic dependent launch.
void launch_kernel_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      void** args);
// Device address of the current device's kernel error word (see
// gemv_error_flags).
unsigned int* device_error_flag();

// Batched prefill (prefill.cu and the embedding in kernels.cu): rows are
// tokens, T of them at positions pos0 .. pos0 + T - 1.
void launch_embed_rows(const QMat& emb, const uint32_t* tokens, uint32_t T, float* X, cudaStream_t stream);
// The *_rows kernels and the attention write f16 to the last argument instead
// of f32 when it is set (the tensor-core GEMM's input).
void launch_rmsnorm_rows(const float* X, const float* w, uint32_t n, uint32_t T, float eps, float* Y,
                         cudaStream_t s, __half* Yh = nullptr);
void launch_qkv_post(const float* Y, uint32_t rows, uint32_t T, uint32_t q_rows, uint32_t k_rows, uint32_t hd,
                     const float* bias, const float2* rope, uint32_t pos0, uint32_t max_ctx, float* Q, float* kc,
                     float* vc, cudaStream_t s);
// Causal attention over the prompt; when the grid is small the keys of each
// token block are split over prefill_attention_splits() CTAs whose partials
// go to `part` (prefill_attention_scratch_floats() floats) and are merged.
void launch_attention_prefill(const float* Q, const float* kc, const float* vc, uint32_t n_heads, uint32_t n_kv,
                              uint32_t hd, uint32_t max_ctx, uint32_t pos0, uint32_t T, float* out, cudaStream_t s,
                              __half* out_h = nullptr, float* part = nullptr);
uint32_t prefill_attention_tokens(uint32_t T, uint32_t n_kv);
uint32_t prefill_attention_splits(uint32_t T, uint32_t n_kv, uint32_t pos0);
size_t prefill_attention_scratch_floats(uint32_t T, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t pos0);
void launch_swiglu_rows(const float* Y, uint32_t ffn, uint32_t T, float* H, cudaStream_t s, __half* Hh = nullptr);
void launch_add_rows(float* X, const float* Y, uint64_t n, cudaStream_t s);

// Tensor-core GEMM of the batched prefill (tc_gemm.cu, tcgen05 + TMA):
// Y[t * ldy + n] = sum_k X[t][k] * W[n][k] for t < T, n < N; X [T][K] and
// W [N][K] row-major f16 (16-byte aligned, K a multiple of 8), f32 result.
// A bounded wait that gives up raises bit 6 of the device error word.
void launch_tc_gemm(const __half* W, uint32_t N, uint32_t K, const __half* X, uint32_t T, float* Y, uint32_t ldy,
                    cudaStream_t s);
// Token-tile width (64, 128 or 256) the GEMM uses for an N x T output.
uint32_t tc_gemm_token_tile(uint32_t N, uint32_t T);
// dst[i] = (f16) src[i], round to nearest even (src 16-byte, dst 8-byte aligned).
void launch_f32_to_f16(const float* src, __half* dst, uint64_t n, cudaStream_t s);

// One sample from n logits on the device (sampler.cu): kind 0 greedy, 1
// temperature, 2 top-k, 3 top-p; r is the host's uniform draw; scratch holds
// 4 * n u32; the token is written to *out (device).
void launch_sample(const float* logits, uint32_t n, uint32_t kind, uint32_t k, float p, float temp, float r,
                   uint32_t* scratch, uint32_t* out, cudaStream_t stream);

// Op-level kernels (Backend semantics on device pointers).
void launch_rmsnorm(const float* x, const float* w, uint32_t n, float eps, float* y, cudaStream_t s);
void launch_softmax(float* x, uint32_t n, cudaStream_t s);
void launch_silu(float* x, uint32_t n, cudaStream_t s);
// cs: [head_dim/2] (cos, sin) computed on the host exactly as ops::rope does.
void launch_rope(float* x, uint32_t n_heads, uint32_t head_dim, const float2* cs, cudaStream_t s);

// Host-side rotary table, identical to ops::rope's arithmetic
// (src/core/ops.cpp:77-82): out[p * hd/2 + i] = (cos, sin)(p * 1/powf(base, 2i/hd)).
void rope_table(uint32_t head_dim, uint32_t positions, float base, std::vector<float2>& out,
                uint32_t first_pos = 0);

int device_sm_count();

}  // namespace smallm
