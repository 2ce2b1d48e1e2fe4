// Device-resident decoder model (internal).
#pragma once

#include <nccl.h>

#include <string>
#include <vector>

#include "engine.h"
#include "smallm_cuda.h"

namespace smallm {

class GGUFFile;
struct StepOp;

struct LayerW {
    QMat qkv;              // Q pairs | K pairs | V rows (V only when it shares Q's type)
    QMat v;                // V rows when attn_v has another type than attn_q
    bool fused_v = true;
    QMat o, gu, down;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* bias = nullptr;  // Qwen2: [q_local | k_local | v_local]
};

struct Model {
    // configuration (src/config/common/config.h:15-46)
    std::string arch;
    uint32_t n_layers = 0, embd = 0, ffn = 0, n_heads = 0, n_kv = 0, hd = 0, vocab = 0, ctx = 0, max_ctx = 0;
    float rope_base = 10000.f, eps = 1e-5f;
    // placement
    int device = 0, sm_count = 0, tp_rank = 0, tp_size = 1;
    uint32_t nh_l = 0, nkv_l = 0, ffn_l = 0, vocab_l = 0, v0 = 0;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;
    // weights
    QMat embd_m, out_m;
    float* out_norm = nullptr;
    std::vector<LayerW> layers;
    // state
    float* kv = nullptr;        // [layer][k|v][n_kv_local][max_ctx][hd]
    float2* rope = nullptr;     // [max_ctx][hd/2]
    float *x = nullptr, *q = nullptr, *att = nullptr, *hbuf = nullptr;
    float *logits = nullptr, *logits_local = nullptr;
    uint32_t attn_cluster = 1;  // CTAs per KV head in the cluster attention
    uint32_t attn_chunk = 32;   // its positions per chunk (sized for max_ctx)
    uint32_t attn_parts = 1;    // clusters per KV head (long contexts, few KV heads)
    float* attn_part_out = nullptr;  // [parts][n_heads * hd] when attn_parts > 1
    float* attn_part_ml = nullptr;   // [parts][n_heads][2]
    size_t gemv_cap_attn = 0;   // shared-memory cap of the QKV / O GEMVs (room for an attention CTA)
    // Tensor parallelism (tp_size > 1): the residual is all-reduced through
    // peer memory by the GEMVs themselves (gemv.cuh EPI_PEER / PRO_RMS_SUM).
    // xchg (this rank's, mapped into every peer) holds the receive buffers
    // [op][sender][embd] f32 then the flags [op][sender]; op 2i is layer i's
    // O projection, op 2i+1 its down projection.
    float* xbuf[2] = {nullptr, nullptr};  // residual before / after each add (op k reads xbuf[k % 2])
    uint8_t* xchg = nullptr;
    size_t xchg_rx_bytes = 0;
    uint8_t* peer_xchg[kMaxTPRanks] = {};  // every rank's xchg as mapped here (own at tp_rank)
    unsigned int* done = nullptr;          // [op] finished-CTA counters
    unsigned int* epoch = nullptr;         // steps run, identical on every rank
    DecodeState* st = nullptr;
    DecodeState* h_st = nullptr;
    unsigned int* h_err = nullptr;  // pinned copy of the device error word after a step
    unsigned long long* keys = nullptr;
    uint32_t* ids = nullptr;
    uint32_t ids_cap = 0;
    uint32_t pending_steps = 0;
    cudaGraphExec_t exec = nullptr;
    cudaGraphExec_t trace_exec = nullptr;  // copy of the step that stamps trace slots
    TraceSlot* trace_dev = nullptr;
    std::vector<uint32_t> trace_kinds;
    uint32_t cached = 0;
    uint64_t weight_bytes = 0, dev_bytes = 0;
    std::vector<void*> allocs;

    Model() = default;
    ~Model();
    Model(const Model&) = delete;
    Model& operator=(const Model&) = delete;

    void load(const std::string& path, const smallm_model_opts& opts);
    void forward(uint32_t token, uint32_t pos, float* logits, uint32_t* argmax);
    void decode_async(uint32_t token, uint32_t pos, uint32_t n_steps);
    void decode_ids(uint32_t* out, uint32_t n);
    // One sample (sampler.cu) from the last step's logits.
    uint32_t sample(uint32_t kind, uint32_t k, float p, float temperature, float u);
    uint32_t* samp_scratch = nullptr;  // 4 * vocab + 4 u32
    // Batched prefill: f16 copies of the layer matrices in storage row order
    // (made at the first prefill from the bit-exact dequantized values), GEMMs
    // over the T tokens on the tcgen05 kernel.
    void prefill(const uint32_t* tokens, uint32_t T, uint32_t pos0, float* out_logits, uint32_t* out_argmax,
                 uint32_t flags);
    struct LayerF16 {
        __half *qkv = nullptr, *v = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
    };
    std::vector<LayerF16> layers_f16;
    __half* pre_xh = nullptr;  // f16 copy of a GEMM's input rows
    uint64_t pre_xh_cap = 0;   // elements pre_xh holds
    float* pre_part = nullptr; // key-split partials of the prefill attention
    size_t pre_part_cap = 0;   // floats pre_part holds
    uint32_t pre_cap = 0;  // tokens the prefill buffers hold
    float *pre_x = nullptr, *pre_xn = nullptr, *pre_y = nullptr, *pre_q = nullptr, *pre_a = nullptr,
          *pre_h = nullptr;
    uint32_t* pre_tok = nullptr;
    std::vector<void*> pre_allocs;
    void enqueue_step(cudaStream_t s, TraceSlot* trace = nullptr);
    // The persistent decode step (step.cu): the whole token step as one
    // cooperative kernel when the model's shapes and formats allow it
    // (step_on; otherwise step_why says why and the per-op kernels run).
    bool step_on = false;
    std::string step_why;
    StepOp* step_ops = nullptr;
    uint32_t step_nops = 0, step_nsig = 0, step_xbytes = 0, step_ring = 0, step_grid = 0;
    size_t step_smem = 0;
    const void* step_fn = nullptr;
    unsigned int* step_bar = nullptr;    // grid barrier counter; step_bar + 1 is the abort flag
    unsigned int* step_abort = nullptr;
    float* step_part = nullptr;          // attention item partials
    unsigned int* step_tickets = nullptr;
    std::string step_unsupported() const;
    void alloc_step_buffers();
    void build_step();
    void launch_step(cudaStream_t s, TraceSlot* trace = nullptr, unsigned long long* pieces = nullptr,
                     uint32_t piece_cap = 0);
    void trace_step_persistent(uint32_t token, uint32_t pos, std::vector<TraceSlot>& out);
    TraceSlot* trace_dev_step = nullptr;
    unsigned long long* trace_dev_pieces = nullptr;
    void reset_step_state();
    uint32_t step_launch_count() const;
    void trace_step(uint32_t token, uint32_t pos, std::vector<TraceSlot>& out);

private:
    void* dalloc(size_t bytes);
    float* upload_vector(const GGUFFile& f, const std::string& name, uint64_t expect, uint64_t first, uint64_t count);
    std::vector<QMat*> all_mats();
    void capture(cudaGraphExec_t* out, TraceSlot* trace);
    void set_state(uint32_t token, uint32_t pos);
    // After a synchronised step: raise if a bounded device wait gave up (the
    // step's results are then invalid).
    void check_step_errors();
};

}  // namespace smallm
