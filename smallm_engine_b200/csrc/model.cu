// Device-resident Qwen2/Llama decoder (host orchestration).
//
// Mirrors Qwen2Model / LlamaModel (src/model/qwen2_model.cpp:28-198,
// src/model/llama_model.cpp:17-177) behind the Model contract
// (include/smallm/model/common/model.h:16-43), with the per-token step
//
//   embed -> L x [ QKV GEMV (fused RMSNorm, bias, RoPE, KV append)
//                -> split-K attention -> O GEMV (+ residual)
//                -> gate/up GEMV (fused RMSNorm, SwiGLU) -> down GEMV (+ residual) ]
//         -> lm_head GEMV (fused final RMSNorm, logits, greedy argmax) -> finalize
//
// captured once as a CUDA graph whose inputs (token, position) live in
// device memory, so a decode step is one graph launch.
//
// Tensor parallelism (tp_size > 1): query/KV heads and FFN rows are split
// across ranks (column-parallel Q/K/V and gate/up, row-parallel O and down),
// lm_head is split by vocabulary rows.  The residual all-reduce after O and
// after down is fused into the GEMVs over peer memory: the row-parallel GEMV
// stores each finished row of its partial W_r.h into every rank's receive
// buffer (CUDA IPC mappings, NVLink stores) and its last CTA raises this
// rank's flag there; the next GEMV waits for every rank's flag and adds the
// partials to the residual in rank order in its prologue (no collective
// launch between them).  The greedy argmax is merged with an ncclAllGather of
// 8-byte keys.
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "engine.h"
#include "gguf.h"
#include "model.h"

namespace smallm {

static void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw Error(6, std::string(what) + ": " + ncclGetErrorString(r));
}

void* Model::dalloc(size_t bytes) {
    void* p = nullptr;
    SM_CUDA(cudaMalloc(&p, bytes ? bytes : 16));
    allocs.push_back(p);
    dev_bytes += bytes;
    return p;
}

Model::~Model() {
    if (stream) cudaStreamSynchronize(stream);
    for (void* p : pre_allocs) cudaFree(p);
    for (int r = 0; r < tp_size && r < kMaxTPRanks; ++r)
        if (peer_xchg[r] && peer_xchg[r] != xchg) cudaIpcCloseMemHandle(peer_xchg[r]);
    if (exec) cudaGraphExecDestroy(exec);
    if (trace_exec) cudaGraphExecDestroy(trace_exec);
    if (comm) ncclCommDestroy(comm);
    for (QMat* m : all_mats()) qmat_free(*m);
    for (void* p : allocs) cudaFree(p);
    if (h_st) cudaFreeHost(h_st);
    if (h_err) cudaFreeHost(h_err);
    if (stream) cudaStreamDestroy(stream);
}

std::vector<QMat*> Model::all_mats() {
    std::vector<QMat*> v{&embd_m, &out_m};
    for (auto& l : layers) {
        v.push_back(&l.qkv);
        v.push_back(&l.v);
        v.push_back(&l.o);
        v.push_back(&l.gu);
        v.push_back(&l.down);
    }
    return v;
}

namespace {

// Staging for uploads: host segments are concatenated into one device
// buffer and repacked through a row map.
struct Stager {
    uint8_t* buf = nullptr;
    size_t cap = 0;
    uint32_t* map = nullptr;
    size_t map_cap = 0;
    ~Stager() {
        if (buf) cudaFree(buf);
        if (map) cudaFree(map);
    }
    void need(size_t bytes, size_t map_entries) {
        if (bytes > cap) {
            if (buf) cudaFree(buf);
            buf = nullptr;
            SM_CUDA(cudaMalloc(&buf, bytes));
            cap = bytes;
        }
        if (map_entries > map_cap) {
            if (map) cudaFree(map);
            map = nullptr;
            SM_CUDA(cudaMalloc(&map, map_entries * 4));
            map_cap = map_entries;
        }
    }
};

struct Seg {
    const uint8_t* host;
    uint64_t rows;
};

// Upload `segs` (each full GGUF rows of src_cols elements of `type`) and
// repack rows `row_map` (indices into the concatenation; padded with
// UINT32_MAX to a multiple of 8) into `m` of rows x cols taking columns
// [col0, col0 + cols).
void upload(QMat& m, uint32_t type, uint32_t rows, uint32_t cols, uint64_t src_cols, uint64_t col0,
            const std::vector<Seg>& segs, std::vector<uint32_t> row_map, Stager& stg, cudaStream_t s) {
    const uint64_t rb = type_row_bytes(type, src_cols);
    uint64_t total = 0;
    for (const Seg& g : segs) total += g.rows;
    qmat_alloc(m, type, rows, cols);
    row_map.resize(m.rows_pad, 0xFFFFFFFFu);
    stg.need(total * rb, row_map.size());
    uint64_t off = 0;
    for (const Seg& g : segs) {
        SM_CUDA(cudaMemcpyAsync(stg.buf + off, g.host, g.rows * rb, cudaMemcpyHostToDevice, s));
        off += g.rows * rb;
    }
    SM_CUDA(cudaMemcpyAsync(stg.map, row_map.data(), row_map.size() * 4, cudaMemcpyHostToDevice, s));
    RepackSource src{stg.buf, src_cols, col0, stg.map};
    qmat_repack(m, src, s);
    SM_CUDA(cudaStreamSynchronize(s));
}

std::vector<uint32_t> iota_map(uint32_t n, uint32_t first = 0) {
    std::vector<uint32_t> v(n);
    for (uint32_t i = 0; i < n; ++i) v[i] = first + i;
    return v;
}

}  // namespace

// f32 vector from a 1-D GGUF tensor, dequantised on the device exactly as
// dequantize_tensor does (src/core/tensor.cpp:115-138).
float* Model::upload_vector(const GGUFFile& f, const std::string& name, uint64_t expect, uint64_t first,
                            uint64_t count) {
    const GGUFTensor& t = f.tensor(name);
    if (!type_supported(t.type)) throw Error(2, "unsupported tensor type: " + std::to_string(t.type));
    if (t.numel() != expect) throw Error(5, "tensor " + name + " has an unexpected size");
    const uint64_t n = t.numel();
    const uint64_t bytes = type_row_bytes(t.type, n);
    uint8_t* raw = nullptr;
    float* full = nullptr;
    SM_CUDA(cudaMalloc(&raw, bytes));
    SM_CUDA(cudaMalloc(&full, n * 4));
    SM_CUDA(cudaMemcpyAsync(raw, f.data(t), bytes, cudaMemcpyHostToDevice, stream));
    launch_dequant_raw(t.type, raw, n, full, stream);
    float* out = static_cast<float*>(dalloc(count * 4));
    SM_CUDA(cudaMemcpyAsync(out, full + first, count * 4, cudaMemcpyDeviceToDevice, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    cudaFree(raw);
    cudaFree(full);
    return out;
}

void Model::load(const std::string& path, const smallm_model_opts& o) {
    device = o.device;
    SM_CUDA(cudaSetDevice(device));
    int major = 0;
    SM_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    if (major < 10) throw Error(3, "smallm: an sm_100 (Blackwell) device is required");
    sm_count = device_sm_count();
    tp_rank = o.tp_size > 1 ? o.tp_rank : 0;
    tp_size = o.tp_size > 1 ? o.tp_size : 1;
    if (tp_size != 1 && tp_size != 2 && tp_size != 4 && tp_size != 8)
        throw Error(1, "tp_size must be 1, 2, 4 or 8");
    if (tp_rank < 0 || tp_rank >= tp_size) throw Error(1, "tp_rank out of range");
    SM_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));

    GGUFFile f(path);
    // src/config/common/config.cpp:14-48
    arch = f.get_str("general.architecture");
    if (arch != "qwen2" && arch != "llama") throw Error(5, "config: unsupported architecture: " + arch);
    const std::string& p = arch;
    n_layers = f.get_u32(p + ".block_count");
    embd = f.get_u32(p + ".embedding_length");
    ffn = f.get_u32(p + ".feed_forward_length");
    n_heads = f.get_u32(p + ".attention.head_count");
    ctx = f.get_u32(p + ".context_length");
    n_kv = f.get_u32_or(p + ".attention.head_count_kv", n_heads);
    rope_base = f.get_f32_or(p + ".rope.freq_base", 10000.0f);
    eps = f.get_f32_or(p + ".attention.layer_norm_rms_epsilon", 1e-5f);
    vocab = (uint32_t)f.str_array_len("tokenizer.ggml.tokens");
    if (n_heads == 0 || n_kv == 0 || n_heads % n_kv) throw Error(5, "config: bad head counts");
    hd = embd / n_heads;
    if (hd != 32 && hd != 64 && hd != 128) throw Error(5, "config: head_dim must be 32, 64 or 128");
    if (vocab == 0) throw Error(5, "config: empty vocabulary (tokenizer.ggml.tokens)");
    max_ctx = o.max_ctx ? o.max_ctx : ctx;
    if (max_ctx == 0) throw Error(5, "config: context_length is 0");
    const bool bias = arch == "qwen2";

    if (n_heads % tp_size || n_kv % tp_size || ffn % tp_size)
        throw Error(1, "tensor parallel degree does not divide the head / FFN counts");
    nh_l = n_heads / tp_size;
    nkv_l = n_kv / tp_size;
    ffn_l = ffn / tp_size;
    vocab_l = (vocab + tp_size - 1) / tp_size;
    v0 = tp_rank * vocab_l;
    const uint32_t vrows = std::min(vocab_l, vocab - std::min(vocab, v0));
    const uint32_t qd = n_heads * hd, kvd = n_kv * hd;
    const uint32_t h0 = tp_rank * nh_l, g0 = tp_rank * nkv_l, f0 = tp_rank * ffn_l;

    Stager stg;
    auto weight = [&](const std::string& name, uint64_t in, uint64_t out) -> const GGUFTensor& {
        const GGUFTensor& t = f.tensor(name);
        if (!type_supported(t.type)) throw Error(2, "unsupported tensor type: " + std::to_string(t.type));
        if (t.dims.size() != 2 || t.dims[0] != in || t.dims[1] != out)
            throw Error(5, "tensor " + name + " has an unexpected shape");
        return t;
    };
    auto col_aligned = [&](uint32_t type, uint64_t c) {
        const uint32_t be = type_block_elems(type);
        const uint32_t ue = (type == SMALLM_TYPE_Q4_K || type == SMALLM_TYPE_Q6_K) ? 256 : 32;
        return c % (be > ue ? be : ue) == 0;
    };

    // embeddings and output (qwen2_model.cpp:36-42)
    {
        const GGUFTensor& te = weight("token_embd.weight", embd, vocab);
        upload(embd_m, te.type, vocab, embd, embd, 0, {{f.data(te), vocab}}, iota_map(vocab), stg, stream);
        const GGUFTensor& to = weight("output.weight", embd, vocab);
        upload(out_m, to.type, vrows, embd, embd, 0, {{f.data(to) + (uint64_t)v0 * type_row_bytes(to.type, embd), vrows}},
               iota_map(vrows), stg, stream);
        out_norm = upload_vector(f, "output_norm.weight", embd, 0, embd);
        weight_bytes += out_m.gguf_bytes + type_row_bytes(te.type, embd);
    }

    layers.resize(n_layers);
    for (uint32_t i = 0; i < n_layers; ++i) {
        LayerW& L = layers[i];
        const std::string b = "blk." + std::to_string(i) + ".";
        L.attn_norm = upload_vector(f, b + "attn_norm.weight", embd, 0, embd);
        L.ffn_norm = upload_vector(f, b + "ffn_norm.weight", embd, 0, embd);
        const GGUFTensor& tq = weight(b + "attn_q.weight", embd, qd);
        const GGUFTensor& tk = weight(b + "attn_k.weight", embd, kvd);
        const GGUFTensor& tv = weight(b + "attn_v.weight", embd, kvd);
        const GGUFTensor& to = weight(b + "attn_output.weight", qd, embd);
        const GGUFTensor& tg = weight(b + "ffn_gate.weight", embd, ffn);
        const GGUFTensor& tu = weight(b + "ffn_up.weight", embd, ffn);
        const GGUFTensor& td = weight(b + "ffn_down.weight", ffn, embd);
        if (tq.type != tk.type) throw Error(2, "attn_q and attn_k must share a tensor type");
        if (tg.type != tu.type) throw Error(2, "ffn_gate and ffn_up must share a tensor type");
        if (!col_aligned(to.type, (uint64_t)nh_l * hd) || !col_aligned(td.type, ffn_l))
            throw Error(1, "tensor parallel split is not aligned to quantization blocks");

        // Q/K/V rows: rotary pairs (i, i + hd/2) of every local head adjacent
        // so the epilogue can rotate them; V rows in natural order.
        std::vector<uint32_t> map;
        const uint32_t half = hd / 2;
        for (uint32_t h = 0; h < nh_l; ++h)
            for (uint32_t k = 0; k < half; ++k) {
                map.push_back((h0 + h) * hd + k);
                map.push_back((h0 + h) * hd + k + half);
            }
        for (uint32_t g = 0; g < nkv_l; ++g)
            for (uint32_t k = 0; k < half; ++k) {
                map.push_back(qd + (g0 + g) * hd + k);
                map.push_back(qd + (g0 + g) * hd + k + half);
            }
        L.fused_v = tv.type == tq.type;
        if (L.fused_v) {
            for (uint32_t g = 0; g < nkv_l; ++g)
                for (uint32_t k = 0; k < hd; ++k) map.push_back(qd + kvd + (g0 + g) * hd + k);
            const uint32_t rows = (nh_l + 2 * nkv_l) * hd;
            upload(L.qkv, tq.type, rows, embd, embd, 0, {{f.data(tq), qd}, {f.data(tk), kvd}, {f.data(tv), kvd}},
                   map, stg, stream);
        } else {
            const uint32_t rows = (nh_l + nkv_l) * hd;
            upload(L.qkv, tq.type, rows, embd, embd, 0, {{f.data(tq), qd}, {f.data(tk), kvd}}, map, stg, stream);
            upload(L.v, tv.type, nkv_l * hd, embd, embd, 0, {{f.data(tv), kvd}}, iota_map(nkv_l * hd, g0 * hd),
                   stg, stream);
        }
        if (bias) {
            // [q_local | k_local | v_local] in logical order
            float* qb = upload_vector(f, b + "attn_q.bias", qd, (uint64_t)h0 * hd, (uint64_t)nh_l * hd);
            float* kb = upload_vector(f, b + "attn_k.bias", kvd, (uint64_t)g0 * hd, (uint64_t)nkv_l * hd);
            float* vb = upload_vector(f, b + "attn_v.bias", kvd, (uint64_t)g0 * hd, (uint64_t)nkv_l * hd);
            L.bias = static_cast<float*>(dalloc(4ull * (nh_l + 2 * nkv_l) * hd));
            SM_CUDA(cudaMemcpyAsync(L.bias, qb, 4ull * nh_l * hd, cudaMemcpyDeviceToDevice, stream));
            SM_CUDA(cudaMemcpyAsync(L.bias + nh_l * hd, kb, 4ull * nkv_l * hd, cudaMemcpyDeviceToDevice, stream));
            SM_CUDA(cudaMemcpyAsync(L.bias + (nh_l + nkv_l) * hd, vb, 4ull * nkv_l * hd, cudaMemcpyDeviceToDevice,
                                    stream));
        }
        // O: all embd rows, this rank's head columns (row-parallel)
        upload(L.o, to.type, embd, nh_l * hd, qd, (uint64_t)h0 * hd, {{f.data(to), embd}}, iota_map(embd), stg,
               stream);
        // gate/up interleaved so the epilogue sees (gate_j, up_j) together
        std::vector<uint32_t> gm;
        for (uint32_t j = 0; j < ffn_l; ++j) {
            gm.push_back(f0 + j);
            gm.push_back(ffn + f0 + j);
        }
        upload(L.gu, tg.type, 2 * ffn_l, embd, embd, 0, {{f.data(tg), ffn}, {f.data(tu), ffn}}, gm, stg, stream);
        upload(L.down, td.type, embd, ffn_l, ffn, f0, {{f.data(td), embd}}, iota_map(embd), stg, stream);
        weight_bytes += L.qkv.gguf_bytes + L.v.gguf_bytes + L.o.gguf_bytes + L.gu.gguf_bytes + L.down.gguf_bytes;
    }
    for (QMat* m : all_mats()) dev_bytes += m->dev_bytes;

    // activations, KV cache, rotary table, scratch
    const size_t kv_per = (size_t)nkv_l * max_ctx * hd;
    kv = static_cast<float*>(dalloc(4ull * kv_per * 2 * n_layers));
    SM_CUDA(cudaMemsetAsync(kv, 0, 4ull * kv_per * 2 * n_layers, stream));
    std::vector<float2> rt;
    rope_table(hd, max_ctx, rope_base, rt);
    rope = static_cast<float2*>(dalloc(rt.size() * sizeof(float2)));
    SM_CUDA(cudaMemcpy(rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice));
    x = static_cast<float*>(dalloc(4ull * embd));
    q = static_cast<float*>(dalloc(4ull * nh_l * hd));
    att = static_cast<float*>(dalloc(4ull * nh_l * hd));
    hbuf = static_cast<float*>(dalloc(4ull * ffn_l));
    logits = static_cast<float*>(dalloc(4ull * vocab_l * tp_size));
    logits_local = tp_size > 1 ? static_cast<float*>(dalloc(4ull * vocab_l)) : logits;
    // cluster size and chunk depend on each other (the chunk's shared memory
    // decides which cluster sizes schedule): size the chunk for the largest
    // cluster, then settle on the cluster that fits it
    // models with at most 2 KV heads at short contexts (<= 512 positions):
    // 8-CTA clusters, whose merge moves half the partials of a 16-CTA one
    // (measured on the Qwen2-0.5B shape, same box: 1690 -> 1749 tok/s; on
    // Llama-8B's 8 KV heads it lost 3%)
    const uint32_t c_cap = (nkv_l <= 2 && max_ctx <= 512) ? 8u : 16u;
    attn_cluster = std::min(c_cap, attention_cluster_size(nh_l, nkv_l, hd, 32));
    for (int it = 0; it < 3; ++it) {
        attn_parts = attention_cluster_parts(nkv_l, attn_cluster, max_ctx, device_sm_count());
        attn_chunk = attention_cluster_chunk(max_ctx, attn_cluster, hd, attn_parts);
        const uint32_t c = std::min(c_cap, attention_cluster_size(nh_l, nkv_l, hd, attn_chunk));
        if (c == attn_cluster) break;
        attn_cluster = c;
    }
    if (attn_parts > 1) {
        attn_part_out = static_cast<float*>(dalloc(4ull * attn_parts * nh_l * hd));
        attn_part_ml = static_cast<float*>(dalloc(8ull * attn_parts * nh_l));
    }
    {
        // an attention CTA (dynamic + a little static shared memory) next to a
        // GEMV CTA on one SM, each with the per-CTA reservation
        int dev = 0, per_sm = 0, reserved = 0;
        SM_CUDA(cudaGetDevice(&dev));
        SM_CUDA(cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
        SM_CUDA(cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
        const size_t attn = attention_cluster_smem(nh_l, nkv_l, hd, attn_chunk) + 256;
        const size_t need = attn + 2 * (size_t)reserved;
        gemv_cap_attn = (size_t)per_sm > need ? (size_t)per_sm - need : 0;
    }
    st = static_cast<DecodeState*>(dalloc(sizeof(DecodeState)));
    SM_CUDA(cudaMemsetAsync(st, 0, sizeof(DecodeState), stream));
    keys = static_cast<unsigned long long*>(dalloc(8ull * tp_size));
    ids_cap = max_ctx;
    ids = static_cast<uint32_t*>(dalloc(4ull * ids_cap));
    SM_CUDA(cudaHostAlloc(&h_st, sizeof(DecodeState), cudaHostAllocDefault));
    std::memset(h_st, 0, sizeof(DecodeState));
    SM_CUDA(cudaHostAlloc(&h_err, 4, cudaHostAllocDefault));
    *h_err = 0;

    if (tp_size > 1) {
        if (!o.nccl_id) throw Error(1, "tensor parallel load needs an NCCL unique id");
        ncclUniqueId id;
        std::memcpy(&id, o.nccl_id, sizeof(id));
        nccl_check(ncclCommInitRank(&comm, tp_size, id, tp_rank), "ncclCommInitRank");
        // residual exchange buffers, mapped into every peer (CUDA IPC; the
        // 64-byte handles travel over the communicator)
        const uint32_t ops = 2 * n_layers;
        xchg_rx_bytes = 4ull * ops * tp_size * embd;
        const size_t xbytes = xchg_rx_bytes + 4ull * ops * tp_size;
        xchg = static_cast<uint8_t*>(dalloc(xbytes));
        SM_CUDA(cudaMemset(xchg, 0, xbytes));
        cudaIpcMemHandle_t mine;
        SM_CUDA(cudaIpcGetMemHandle(&mine, xchg));
        uint8_t* hbuf_dev = static_cast<uint8_t*>(dalloc(sizeof(mine) * (tp_size + 1)));
        SM_CUDA(cudaMemcpy(hbuf_dev, &mine, sizeof(mine), cudaMemcpyHostToDevice));
        nccl_check(ncclAllGather(hbuf_dev, hbuf_dev + sizeof(mine), sizeof(mine), ncclUint8, comm, stream),
                   "ncclAllGather");
        std::vector<cudaIpcMemHandle_t> handles(tp_size);
        SM_CUDA(cudaMemcpyAsync(handles.data(), hbuf_dev + sizeof(mine), sizeof(mine) * tp_size,
                                cudaMemcpyDeviceToHost, stream));
        SM_CUDA(cudaStreamSynchronize(stream));
        for (int r = 0; r < tp_size; ++r) {
            if (r == tp_rank) {
                peer_xchg[r] = xchg;
                continue;
            }
            void* pm = nullptr;
            SM_CUDA(cudaIpcOpenMemHandle(&pm, handles[r], cudaIpcMemLazyEnablePeerAccess));
            peer_xchg[r] = static_cast<uint8_t*>(pm);
        }
        done = static_cast<unsigned int*>(dalloc(4ull * ops));
        SM_CUDA(cudaMemset(done, 0, 4ull * ops));
        epoch = static_cast<unsigned int*>(dalloc(4));
        SM_CUDA(cudaMemset(epoch, 0, 4));
        xbuf[0] = x;
        xbuf[1] = static_cast<float*>(dalloc(4ull * embd));
        // every rank's buffers are zeroed and mapped before any step writes into them
        nccl_check(ncclAllGather(hbuf_dev, hbuf_dev + sizeof(mine), sizeof(mine), ncclUint8, comm, stream),
                   "ncclAllGather");
    }
    if (tp_size == 1) {
        alloc_step_buffers();
        build_step();
    }
    SM_CUDA(cudaStreamSynchronize(stream));
    capture(&exec, nullptr);
}

// One decode step: everything after the (token, pos) state is in place.
// Kind codes of the kernels of a traced step (smallm_model_trace_step).
enum TraceKind { TK_EMBED = 1, TK_QKV = 2, TK_V = 3, TK_ATTN = 4, TK_O = 5, TK_GATE_UP = 6, TK_DOWN = 7,
                 TK_LM_HEAD = 8, TK_FINALIZE = 9 };

// One decode step: everything after the (token, pos) state is in place.
// With `trace`, kernel k of the step stamps slot trace[k] and its kind is
// recorded in trace_kinds.
void Model::enqueue_step(cudaStream_t s, TraceSlot* trace) {
    if (step_on && !trace) {  // the whole step as one persistent kernel (step.cu)
        launch_step(s);
        return;
    }
    const bool pdl = true;  // programmatic dependent launch between the step's kernels
    uint32_t nslot = 0;
    if (trace) trace_kinds.clear();
    auto slot = [&](uint32_t kind) -> TraceSlot* {
        if (!trace) return nullptr;
        trace_kinds.push_back(kind);
        return trace + nslot++;
    };
    launch_embed(embd_m, st, x, s, pdl, slot(TK_EMBED));
    const uint32_t qrows = nh_l * hd, krows = nkv_l * hd;
    const bool tpx = tp_size > 1;
    // op k's receive slot for sender r in rank base's buffers, and its flag
    auto rx_at = [&](uint8_t* base, uint32_t op, int r) {
        return reinterpret_cast<float*>(base) + ((size_t)op * tp_size + r) * embd;
    };
    auto flag_at = [&](uint8_t* base, uint32_t op, int r) {
        return reinterpret_cast<unsigned int*>(base + xchg_rx_bytes) + (size_t)op * tp_size + r;
    };
    auto send = [&](GemvArgs& a, uint32_t op) {  // this rank's partial of op -> every rank
        a.tp = tp_size;
        a.epoch = epoch;
        a.done_ctr = done + op;
        for (int r = 0; r < tp_size; ++r) {
            a.peer_out[r] = rx_at(peer_xchg[r], op, tp_rank);
            a.peer_flag[r] = flag_at(peer_xchg[r], op, tp_rank);
        }
    };
    auto gather = [&](GemvArgs& a, uint32_t op) {  // residual after op = before + all partials
        a.tp = tp_size;
        a.epoch = epoch;
        a.x_res = xbuf[op % 2];
        a.x_out = xbuf[(op + 1) % 2];
        a.x = a.x_res;
        a.rx = rx_at(xchg, op, 0);
        a.rx_flag = flag_at(xchg, op, 0);
    };
    for (uint32_t i = 0; i < n_layers; ++i) {
        LayerW& L = layers[i];
        float* kc = kv + (size_t)(2 * i) * nkv_l * max_ctx * hd;
        float* vc = kv + (size_t)(2 * i + 1) * nkv_l * max_ctx * hd;
        const bool sum_in = tpx && i > 0;  // QKV completes the previous layer's down all-reduce
        GemvArgs a;
        a.x = tpx ? xbuf[0] : x;
        a.norm_w = L.attn_norm;
        a.eps = eps;
        a.bias = L.bias;
        a.q_rows = qrows;
        a.k_rows = krows;
        a.head_dim = hd;
        a.max_ctx = max_ctx;
        a.qout = q;
        a.kcache = kc;
        a.vcache = vc;
        a.rope = rope;
        a.pos = &st->pos;
        a.trace = slot(TK_QKV);
        a.smem_cap = gemv_cap_attn;
        if (sum_in) gather(a, 2 * i - 1);
        launch_gemv(L.qkv, sum_in ? GEMV_PRO_RMS_SUM : GEMV_PRO_RMS, GEMV_EPI_QKV, a, s, pdl);
        if (!L.fused_v) {
            GemvArgs av = a;
            av.q_rows = 0;
            av.k_rows = 0;
            av.bias = L.bias ? L.bias + qrows + krows : nullptr;
            av.trace = slot(TK_V);
            if (sum_in) av.x = xbuf[(2 * i) % 2];  // the residual the QKV GEMV just completed
            launch_gemv(L.v, GEMV_PRO_RMS, GEMV_EPI_QKV, av, s, pdl);
        }
        AttnArgs at;
        at.q = q;
        at.kcache = kc;
        at.vcache = vc;
        at.out = att;
        at.pos = &st->pos;
        at.n_heads = nh_l;
        at.n_kv = nkv_l;
        at.hd = hd;
        at.max_ctx = max_ctx;
        at.err = device_error_flag();
        at.trace = slot(TK_ATTN);
        at.chunk = attn_chunk;
        at.parts = attn_parts;
        at.part_out = attn_part_out;
        at.part_ml = attn_part_ml;
        launch_attention_cluster(at, attn_cluster, s, pdl);

        GemvArgs ao;
        ao.x = att;
        if (attn_parts > 1) {  // the O GEMV merges the attention's parts as it stages x
            ao.x = attn_part_out;
            ao.merge_parts = attn_parts;
            ao.merge_hd = hd;
            ao.merge_ml = attn_part_ml;
        }
        ao.y = x;
        ao.trace = slot(TK_O);
        ao.smem_cap = gemv_cap_attn;
        if (tpx) send(ao, 2 * i);
        launch_gemv(L.o, attn_parts > 1 ? GEMV_PRO_MERGE : GEMV_PRO_PLAIN, tpx ? GEMV_EPI_PEER : GEMV_EPI_RESIDUAL,
                    ao, s, pdl);

        GemvArgs ag;
        ag.x = x;
        ag.norm_w = L.ffn_norm;
        ag.eps = eps;
        ag.y = hbuf;
        ag.trace = slot(TK_GATE_UP);
        if (tpx) gather(ag, 2 * i);
        launch_gemv(L.gu, tpx ? GEMV_PRO_RMS_SUM : GEMV_PRO_RMS, GEMV_EPI_SWIGLU, ag, s, pdl);

        GemvArgs ad;
        ad.x = hbuf;
        ad.y = x;
        ad.trace = slot(TK_DOWN);
        if (tpx) send(ad, 2 * i + 1);
        launch_gemv(L.down, GEMV_PRO_PLAIN, tpx ? GEMV_EPI_PEER : GEMV_EPI_RESIDUAL, ad, s, pdl);
    }
    GemvArgs al;
    al.x = x;
    al.norm_w = out_norm;
    al.eps = eps;
    al.y = logits_local;
    al.argmax = &st->argmax;
    al.row_offset = v0;
    al.trace = slot(TK_LM_HEAD);
    if (tpx) gather(al, 2 * n_layers - 1);
    launch_gemv(out_m, tpx ? GEMV_PRO_RMS_SUM : GEMV_PRO_RMS, GEMV_EPI_LOGITS, al, s, pdl);
    if (tpx) {
        nccl_check(ncclAllGather(&st->argmax, keys, 1, ncclUint64, comm, s), "ncclAllGather");
        launch_finalize_tp(st, keys, tp_size, ids, ids_cap, epoch, s, pdl);
    } else {
        launch_finalize(st, ids, ids_cap, s, pdl, slot(TK_FINALIZE));
    }
}

void Model::capture(cudaGraphExec_t* out, TraceSlot* trace) {
    cudaGraph_t g = nullptr;
    SM_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    try {
        enqueue_step(stream, trace);
    } catch (...) {
        cudaStreamEndCapture(stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    SM_CUDA(cudaStreamEndCapture(stream, &g));
    cudaError_t e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    SM_CUDA(e);
}

// Run one step through a copy of the graph whose kernels stamp trace slots.
void Model::trace_step(uint32_t token, uint32_t pos, std::vector<TraceSlot>& out) {
    if (token >= vocab) throw Error(1, "token id out of range");
    if (pos >= max_ctx) throw Error(7, "position " + std::to_string(pos) + " is beyond the context length");
    if (step_on) {
        trace_step_persistent(token, pos, out);
        return;
    }
    const uint32_t nmax = 8 + 6 * n_layers;
    if (!trace_dev) {
        trace_dev = static_cast<TraceSlot*>(dalloc(sizeof(TraceSlot) * nmax));
        capture(&trace_exec, trace_dev);
    }
    const uint32_t n = (uint32_t)trace_kinds.size();
    std::vector<TraceSlot> init(n);
    for (uint32_t k = 0; k < n; ++k) init[k] = TraceSlot{~0ull, ~0ull, 0ull, trace_kinds[k]};
    SM_CUDA(cudaMemcpyAsync(trace_dev, init.data(), sizeof(TraceSlot) * n, cudaMemcpyHostToDevice, stream));
    set_state(token, pos);
    SM_CUDA(cudaGraphLaunch(trace_exec, stream));
    out.resize(n);
    SM_CUDA(cudaMemcpyAsync(out.data(), trace_dev, sizeof(TraceSlot) * n, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaMemcpyAsync(h_err, device_error_flag(), 4, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    check_step_errors();
    cached = pos + 1;
}

void Model::set_state(uint32_t token, uint32_t pos) {
    h_st->token = token;
    h_st->pos = pos;
    h_st->step = 0;
    h_st->argmax = 0;
    SM_CUDA(cudaMemcpyAsync(st, h_st, sizeof(DecodeState), cudaMemcpyHostToDevice, stream));
}

void Model::forward(uint32_t token, uint32_t pos, float* out_logits, uint32_t* out_argmax) {
    if (token >= vocab) throw Error(1, "token id out of range");
    if (pos >= max_ctx) throw Error(7, "position " + std::to_string(pos) + " is beyond the context length");
    set_state(token, pos);
    SM_CUDA(cudaGraphLaunch(exec, stream));
    if (out_logits) {
        if (tp_size > 1)
            nccl_check(ncclAllGather(logits_local, logits, vocab_l, ncclFloat32, comm, stream), "ncclAllGather");
        SM_CUDA(cudaMemcpyAsync(out_logits, logits, 4ull * vocab, cudaMemcpyDeviceToHost, stream));
    }
    if (out_argmax) SM_CUDA(cudaMemcpyAsync(h_st, st, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaMemcpyAsync(h_err, device_error_flag(), 4, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    check_step_errors();
    if (out_argmax) *out_argmax = h_st->token;
    cached = pos + 1;
}

void Model::check_step_errors() {
    const unsigned int e = *h_err;
    if (!e) return;
    *h_err = 0;
    gemv_error_flags(true);
    reset_step_state();
    throw Error(SMALLM_ERR_CUDA, "a bounded device wait gave up during the step (flags " + std::to_string(e) +
                                     "); its results are invalid");
}

void Model::decode_async(uint32_t token, uint32_t pos, uint32_t n_steps) {
    if (token >= vocab) throw Error(1, "token id out of range");
    if ((uint64_t)pos + n_steps > max_ctx)
        throw Error(7, "decode would run past the context length");
    if (n_steps > ids_cap) throw Error(1, "too many decode steps");
    set_state(token, pos);
    for (uint32_t i = 0; i < n_steps; ++i) SM_CUDA(cudaGraphLaunch(exec, stream));
    pending_steps = n_steps;
    cached = pos + n_steps;
}

// ------------------------------------------------------------ prefill --

// The prompt tokens[0..T) at positions pos0 .. pos0 + T - 1 in one pass per
// layer: every linear layer is a GEMM over the T tokens (the reference runs
// Model::forward once per token, generator.cpp:47-51); the KV cache receives
// all T positions and the last token's logits go through the decode lm_head
// (fused final RMSNorm, logits, argmax).
void Model::prefill(const uint32_t* tokens, uint32_t T, uint32_t pos0, float* out_logits, uint32_t* out_argmax,
                    uint32_t flags) {
    if (tp_size > 1) throw Error(1, "prefill runs on a single GPU (tp_size 1)");
    if (T == 0) throw Error(1, "prefill needs at least one token");
    for (uint32_t t = 0; t < T; ++t)
        if (tokens[t] >= vocab) throw Error(1, "token id out of range");
    if ((uint64_t)pos0 + T > max_ctx) throw Error(7, "prefill would run past the context length");
    if (flags & ~SMALLM_PREFILL_TC) throw Error(SMALLM_ERR_INVALID, "unknown prefill flags");
    auto palloc = [&](size_t bytes) {
        void* p = nullptr;
        SM_CUDA(cudaMalloc(&p, bytes));
        pre_allocs.push_back(p);
        return static_cast<float*>(p);
    };
    if (layers_f16.empty()) {
        // dequantize each matrix (bit-exact) into one f32 staging buffer, then
        // round it to f16 into its own copy (2 bytes per weight)
        uint64_t most = 0;
        for (uint32_t i = 0; i < n_layers; ++i)
            for (const QMat* q : {&layers[i].qkv, &layers[i].v, &layers[i].o, &layers[i].gu, &layers[i].down})
                if (q->base) most = std::max<uint64_t>(most, (uint64_t)q->rows * q->cols);
        float* stage = nullptr;
        SM_CUDA(cudaMalloc(&stage, 4 * most));
        std::vector<LayerF16> made(n_layers);
        auto deq16 = [&](const QMat& q) -> __half* {
            if (!q.base) return nullptr;
            __half* w = reinterpret_cast<__half*>(palloc(2ull * q.rows * q.cols));
            launch_qmat_dequant(q, stage, stream);
            launch_f32_to_f16(stage, w, (uint64_t)q.rows * q.cols, stream);
            return w;
        };
        try {
            for (uint32_t i = 0; i < n_layers; ++i) {
                LayerW& L = layers[i];
                LayerF16& F = made[i];
                F.qkv = deq16(L.qkv);
                F.v = L.fused_v ? nullptr : deq16(L.v);
                F.o = deq16(L.o);
                F.gu = deq16(L.gu);
                F.down = deq16(L.down);
            }
            SM_CUDA(cudaStreamSynchronize(stream));
        } catch (...) {
            cudaStreamSynchronize(stream);
            cudaFree(stage);
            throw;
        }
        SM_CUDA(cudaFree(stage));
        layers_f16 = std::move(made);
    }
    const uint32_t qrows = nh_l * hd, krows = nkv_l * hd;
    if (T > pre_cap) {
        for (float** b : {&pre_x, &pre_xn, &pre_y, &pre_q, &pre_a, &pre_h}) *b = nullptr;
        const uint32_t wide = std::max({layers[0].qkv.rows, layers[0].gu.rows, embd});
        pre_x = palloc(4ull * T * embd);
        pre_xn = palloc(4ull * T * embd);
        pre_y = palloc(4ull * T * wide);
        pre_q = palloc(4ull * T * qrows);
        pre_a = palloc(4ull * T * qrows);
        pre_h = palloc(4ull * T * ffn_l);
        pre_tok = reinterpret_cast<uint32_t*>(palloc(4ull * T));
        pre_cap = T;
    }
    if ((uint64_t)T * std::max({embd, qrows, ffn_l}) > pre_xh_cap) {
        pre_xh_cap = (uint64_t)T * std::max({embd, qrows, ffn_l});
        pre_xh = reinterpret_cast<__half*>(palloc(2 * pre_xh_cap));
    }
    // Y[T][rows] = X[T][cols] . W^T on the tcgen05 kernel over the f16
    // copies; X is in pre_xh, written as f16 by the kernel that produced it
    auto linear = [&](const __half* w16, uint32_t rows, uint32_t cols) {
        launch_tc_gemm(w16, rows, cols, pre_xh, T, pre_y, rows, stream);
    };
    __half* const xh = pre_xh;
    const size_t part_floats = prefill_attention_scratch_floats(T, nh_l, nkv_l, hd, pos0);
    if (part_floats > pre_part_cap) {
        pre_part = palloc(4 * part_floats);
        pre_part_cap = part_floats;
    }
    SM_CUDA(cudaMemcpyAsync(pre_tok, tokens, 4ull * T, cudaMemcpyHostToDevice, stream));
    launch_embed_rows(embd_m, pre_tok, T, pre_x, stream);
    for (uint32_t i = 0; i < n_layers; ++i) {
        LayerW& L = layers[i];
        const LayerF16& H = layers_f16[i];
        float* kc = kv + (size_t)(2 * i) * nkv_l * max_ctx * hd;
        float* vc = kv + (size_t)(2 * i + 1) * nkv_l * max_ctx * hd;
        launch_rmsnorm_rows(pre_x, L.attn_norm, embd, T, eps, pre_xn, stream, xh);
        linear(H.qkv, L.qkv.rows, embd);
        launch_qkv_post(pre_y, L.qkv.rows, T, qrows, krows, hd, L.bias, rope, pos0, max_ctx, pre_q, kc, vc, stream);
        if (!L.fused_v) {
            linear(H.v, L.v.rows, embd);
            launch_qkv_post(pre_y, L.v.rows, T, 0, 0, hd, L.bias ? L.bias + qrows + krows : nullptr, rope, pos0,
                            max_ctx, pre_q, kc, vc, stream);
        }
        launch_attention_prefill(pre_q, kc, vc, nh_l, nkv_l, hd, max_ctx, pos0, T, pre_a, stream, xh, pre_part);
        linear(H.o, embd, qrows);
        launch_add_rows(pre_x, pre_y, (uint64_t)T * embd, stream);
        launch_rmsnorm_rows(pre_x, L.ffn_norm, embd, T, eps, pre_xn, stream, xh);
        linear(H.gu, L.gu.rows, embd);
        launch_swiglu_rows(pre_y, ffn_l, T, pre_h, stream, xh);
        linear(H.down, embd, ffn_l);
        launch_add_rows(pre_x, pre_y, (uint64_t)T * embd, stream);
    }
    SM_CUDA(cudaMemsetAsync(&st->argmax, 0, sizeof(unsigned long long), stream));
    GemvArgs al;
    al.x = pre_x + (size_t)(T - 1) * embd;
    al.norm_w = out_norm;
    al.eps = eps;
    al.y = logits_local;
    al.argmax = &st->argmax;
    al.row_offset = v0;
    launch_gemv(out_m, GEMV_PRO_RMS, GEMV_EPI_LOGITS, al, stream);
    if (out_logits) SM_CUDA(cudaMemcpyAsync(out_logits, logits, 4ull * vocab, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaMemcpyAsync(h_st, st, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    if (out_argmax) {  // packed key (common.cuh argmax_key): low word = ~index
        const unsigned long long k = h_st->argmax;
        *out_argmax = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
    }
    cached = pos0 + T;
}

uint32_t Model::sample(uint32_t kind, uint32_t k, float p, float temperature, float u) {
    if (!samp_scratch) samp_scratch = static_cast<uint32_t*>(dalloc(16ull * vocab + 16));
    if (tp_size > 1)
        nccl_check(ncclAllGather(logits_local, logits, vocab_l, ncclFloat32, comm, stream), "ncclAllGather");
    launch_sample(logits, vocab, kind, k, p, temperature, u, samp_scratch, samp_scratch + 4ull * vocab, stream);
    SM_CUDA(cudaMemcpyAsync(h_st, samp_scratch + 4ull * vocab, 4, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    uint32_t tok;
    std::memcpy(&tok, h_st, 4);
    return tok;
}

void Model::decode_ids(uint32_t* out, uint32_t n) {
    if (n > pending_steps) throw Error(1, "fewer decode steps were run than ids requested");
    SM_CUDA(cudaMemcpyAsync(out, ids, 4ull * n, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaMemcpyAsync(h_err, device_error_flag(), 4, cudaMemcpyDeviceToHost, stream));
    SM_CUDA(cudaStreamSynchronize(stream));
    check_step_errors();
}

}  // namespace smallm
