// engine.cu -- GPT-2 decode engine over libb2decode (the sm_100a hot-path
// kernels) and cuBLAS (the GEMMs); the C-ABI is include/b2_engine.h.
//
// Rebuilds Engine / Engine::Impl of gpu-engine/src/engine.cu:71-388 with the
// same life cycle and the same host flow per decode step (engine.cu:309-377):
// take KV blocks at 16-token boundaries, build token ids / positions /
// seq_lens / block tables for the batch bucket (pad lanes replay the last
// real lane), upload, run the step (a captured CUDA graph per bucket, or
// direct launches), download the next tokens, synchronise.  What differs:
//   * one packed upload per step instead of four copies;
//   * the per-layer sequence fuses the reference's bias / add_one launches
//     into neighbours: LN1(+fc_proj bias of the previous layer) -> QKV GEMM ->
//     kv_append(+k,v bias, seq_lens+1) -> paged attention(+q bias) -> proj
//     GEMM -> LN2(+proj bias) -> fc GEMM -> bias+GELU -> fc_proj GEMM;
//     final LN(+fc_proj bias) -> tied lm_head GEMM -> argmax
//     (reference: engine.cu:150-204, eleven launches per layer vs eight here);
//   * f32 / f16 / bf16 storage with fp32 accumulation everywhere (the f32
//     engine uses CUBLAS_COMPUTE_32F under pedantic math: no TF32);
//   * capacity is checked before anything changes, so an exhausted pool
//     returns B2_ERR_POOL instead of throwing half-way (engine.cu:227-233).
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <nlohmann/json.hpp>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "b2_decode.h"
#include "b2_engine.h"
#include "block_pool.h"
#include "lt_gemm.h"

namespace b2 {
namespace eng {

thread_local std::string g_err;

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void cuda_ok(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(static_cast<int>(e), std::string(what) + ": " + cudaGetErrorString(e));
}
void cublas_ok(cublasStatus_t s, const char* what) {
    if (s != CUBLAS_STATUS_SUCCESS) throw Error(B2_ERR_DEVICE, std::string(what) + ": cuBLAS status " + std::to_string(s));
}
void nccl_ok(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) throw Error(B2_ERR_DEVICE, std::string(what) + ": " + ncclGetErrorString(r));
}
void b2_ok(int rc, const char* what) {
    if (rc != B2_OK) throw Error(rc, std::string(what) + ": " + b2_last_error_string());
}

int dtype_bytes(int dt) { return dt == B2_F32 ? 4 : 2; }
size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// ------------------------------------------------------ synthetic weights
// splitmix64 of (seed, tensor, index) -> two uniforms -> Box-Muller normal.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

template <typename T>
__global__ void synth_normal_kernel(T* dst, size_t n, uint64_t key, float stdev) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = mix64(key ^ mix64(i));
        const float u1 = (static_cast<float>(r >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
        const float u2 = static_cast<float>((r >> 16) & 0xffffffu) * (1.0f / 16777216.0f);
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        dst[i] = static_cast<T>(z * stdev);
    }
}

template <typename T>
__global__ void fill_kernel(T* dst, size_t n, float v) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        dst[i] = static_cast<T>(v);
}

// dst[i] = src[rows[i]] for n rows of `cols` 16-byte chunks (prefill: each
// sequence's last prompt row goes on to the lm_head).
__global__ void gather_rows_kernel(uint4* dst, const uint4* src, const int32_t* rows, int n, int cols) {
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const uint4* s = src + static_cast<size_t>(rows[i]) * cols;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[static_cast<size_t>(i) * cols + c] = s[c];
    }
}

// Block tables live on the device, one row of max_blocks_per_seq entries per
// sequence slot.  The host sends only what changed: (slot, index, block)
// triples for newly allocated blocks, scattered here.
__global__ void scatter_table_updates_kernel(int32_t* slot_tables, const int32_t* upd, int n, int mbps) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) slot_tables[static_cast<size_t>(upd[3 * i]) * mbps + upd[3 * i + 1]] = upd[3 * i + 2];
}

// The step's batch-ordered tables [bucket][mbps] from the slot rows: lane b
// copies the entries of the blocks holding positions [0, seq_lens[b]] (the
// only ones any kernel of the step reads).
__global__ void gather_step_tables_kernel(int32_t* tables, const int32_t* slot_tables, const int32_t* slots,
                                          const int32_t* seq_lens, int mbps) {
    const int b = blockIdx.x;
    const int n = min(mbps, seq_lens[b] / B2_BLOCK_TOKENS + 1);
    const int32_t* src = slot_tables + static_cast<size_t>(slots[b]) * mbps;
    for (int j = threadIdx.x; j < n; j += blockDim.x) tables[static_cast<size_t>(b) * mbps + j] = src[j];
}

// Head-sharded engines with the NCCL all-gather: ncclAllGather leaves the
// ranks' slices one after another, [rank][row][qd chunks]; the output
// projection wants each row's slices side by side, [row][rank * qd chunks].
__global__ void interleave_slices_kernel(uint4* dst, const uint4* src, int rows, int ranks, int qchunks) {
    const long long total = static_cast<long long>(rows) * ranks * qchunks;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % qchunks);
        const long long rr = i / qchunks;
        const int r = static_cast<int>(rr % ranks);
        const int row = static_cast<int>(rr / ranks);
        dst[i] = src[(static_cast<long long>(r) * rows + row) * qchunks + c];
    }
}

// The step's last launch: the device error word (the one b2_device_errors
// reads) next to the step's tokens, so one download brings both back.
__global__ void copy_error_word_kernel(int32_t* dst, const uint32_t* word) {
    if (threadIdx.x == 0) *dst = static_cast<int32_t>(*word);
}

// ------------------------------------------------------------- the engine

struct LayerW {
    const void *ln1_g, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b, *ln2_g, *ln2_b, *fc_w, *fc_b, *fc_proj_w, *fc_proj_b;
};

struct Seq {
    BlockTable table;
    int slot = -1;    // row of the device-resident block tables
    int seq_len = 0;  // positions already in the KV cache
    std::vector<int32_t> prompt;
    int prompt_pos = 0;
    int32_t last_token = 0;
};

// Tensor list in the exporter's file order (gpu-engine/src/loader.cpp:28-47).
struct TensorSpec {
    std::string name;
    std::vector<int64_t> shape;
    int init;  // 0 normal, 1 ones, 2 zeros
};

std::vector<TensorSpec> tensor_specs(const B2ModelShape& s) {
    const int64_t D = s.d_model, V = s.vocab_size;
    std::vector<TensorSpec> t = {{"wte", {V, D}, 0}, {"wpe", {s.n_ctx, D}, 0}};
    for (int i = 0; i < s.n_layer; ++i) {
        const std::string p = "layer" + std::to_string(i) + ".";
        t.push_back({p + "ln1_g", {D}, 1});
        t.push_back({p + "ln1_b", {D}, 2});
        t.push_back({p + "qkv_w", {3 * D, D}, 0});
        t.push_back({p + "qkv_b", {3 * D}, 0});
        t.push_back({p + "proj_w", {D, D}, 0});
        t.push_back({p + "proj_b", {D}, 0});
        t.push_back({p + "ln2_g", {D}, 1});
        t.push_back({p + "ln2_b", {D}, 2});
        t.push_back({p + "fc_w", {4 * D, D}, 0});
        t.push_back({p + "fc_b", {4 * D}, 0});
        t.push_back({p + "fc_proj_w", {D, 4 * D}, 0});
        t.push_back({p + "fc_proj_b", {D}, 0});
    }
    t.push_back({"lnf_g", {D}, 1});
    t.push_back({"lnf_b", {D}, 2});
    return t;
}

size_t numel(const std::vector<int64_t>& shape) {
    size_t n = 1;
    for (auto d : shape) n *= static_cast<size_t>(d);
    return n;
}

struct Engine {
    B2ModelShape shape{};
    B2EngineConfig cfg{};
    int dt = B2_F16, es = 2, device = 0, head_dim = 0, mbps = 0, bucket_cap = 0;
    void* weights = nullptr;
    std::vector<const void*> tensor_ptrs;
    const void *wte = nullptr, *wpe = nullptr, *lnf_g = nullptr, *lnf_b = nullptr;
    std::vector<LayerW> layers;
    void* pool = nullptr;
    int num_blocks = 0;
    std::unique_ptr<BlockPool> blocks;
    cudaStream_t stream = nullptr;
    cublasHandle_t cublas = nullptr;
    void* cublas_ws = nullptr;
    // Per-step buffers at fixed addresses (CUDA graphs replay them).
    // d_in: [tokens | positions | seq_lens | slots] (max_batch each) and the
    // step's gathered block tables [max_batch][mbps].
    // d_next / h_next: [max_batch] next tokens, then the device error word.
    int32_t *d_in = nullptr, *d_seq_post = nullptr, *d_next = nullptr;
    int32_t *h_in = nullptr, *h_next = nullptr;  // pinned
    uint32_t* d_err_word = nullptr;               // libb2decode's device error word
    // Device-resident block tables [num_blocks slots][mbps] (a live sequence
    // holds at least one block, so num_blocks slots always suffice), the free
    // slots, and the (slot, index, block) updates not yet on the device.
    int32_t* d_slot_tables = nullptr;
    int32_t *d_upd = nullptr, *h_upd = nullptr;  // update staging, kUpdChunk triples
    std::vector<int> free_slots;
    std::vector<int32_t> pending_upd;
    void *d_resid = nullptr, *d_x = nullptr, *d_qkv = nullptr, *d_attn = nullptr, *d_attn_out = nullptr,
         *d_ff = nullptr, *d_ff_out = nullptr, *d_logits = nullptr;
    void* attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    // b2_engine_set_lm_head_fused: the tied lm_head GEMM and the argmax as one
    // b2_lm_head_argmax launch (f16 / bf16), with its workspace (zeroed once)
    bool lm_fused = false;
    void* lm_ws = nullptr;
    size_t lm_ws_bytes = 0;
    std::unordered_map<int, Seq> seqs;
    int next_id = 0;
    bool use_graphs = true;
    std::map<int, cudaGraphExec_t> graphs;
    // Head sharding (tp > 1): this engine holds heads [tp_rank * hl, tp_rank * hl + hl)
    // (hl = ceil(n_head / tp); heads past n_head are zero padding), their QKV slice,
    // a zero-padded copy of every output projection, the gathered attention output
    // [2][max_batch, tp * hl * head_dim] (one half per layer parity: after barrier l a
    // fast rank may write layer l + 1 while a peer still reads layer l; it cannot come
    // back to a half before barrier l + 1, which that peer enters only after reading)
    // and the barrier flags [n_layer][tp] (both IPC-shared with the peers), and the
    // peers' addresses of both (d_peer_outs: [parity][rank]).
    int tp = 1, tp_rank = 0, hl = 0;  // hl: heads held here (all of them when tp == 1)
    void* tp_weights = nullptr;
    std::vector<const void*> qkv_w_loc, qkv_b_loc, proj_w_pad;
    void* d_gath = nullptr;
    uint32_t* d_flags = nullptr;
    uint32_t* d_epoch = nullptr;
    void** d_peer_outs = nullptr;
    uint32_t** d_peer_flags = nullptr;
    std::vector<void*> peer_mapped;  // IPC-opened peer bases, closed at destruction
    bool tp_connected = false;
    // cfg.tp_allgather == 1: attention writes this rank's slice to d_attn_loc
    // [max_batch][hl * head_dim], ncclAllGather collects every rank's slice
    // into d_gath's first half ([rank][row][...]) and a small kernel
    // interleaves them into the second half ([row][rank * hl * head_dim]),
    // which the output projection reads.  No peer stores, no flag barrier.
    bool tp_nccl = false;
    ncclComm_t nccl = nullptr;
    void* d_attn_loc = nullptr;
    // Batched prefill (allocated at the first b2_engine_prefill): per-row inputs
    // [tokens | positions | seq_lens | last rows (max_batch) | tables (cap x mbps)],
    // row activations, and the per-sequence tail (last rows, logits, next tokens).
    int prefill_cap = 0;
    bool prefill_tc = true;  // b2_engine_set_prefill_tensor_cores
    bool linear_tc = false;  // b2_engine_set_linear_tensor_cores
    // b2_engine_set_gemm_mode: 16-bit decode-step GEMMs on cuBLASLt with the
    // algorithm per shape chosen by timing (bit 1), the FC layer's bias + GELU
    // in that GEMM's epilogue (bit 2).
    int gemm_mode = 0;
    std::unique_ptr<LtGemm> lt;
    bool in_decode = false;  // run_step_kernels is issuing the decode step
    int32_t *d_pin = nullptr, *h_pin = nullptr, *d_pseq_post = nullptr, *d_pnext = nullptr, *h_pnext = nullptr;
    void *p_resid = nullptr, *p_x = nullptr, *p_qkv = nullptr, *p_attn = nullptr, *p_attn_out = nullptr,
         *p_ff = nullptr, *p_ff_out = nullptr, *p_last = nullptr, *p_logits = nullptr, *p_attn_ws = nullptr;
    size_t p_attn_ws_bytes = 0;

    static constexpr int kUpdChunk = 4096;  // table updates per upload
    int32_t* in_tokens() const { return d_in; }
    int32_t* in_positions() const { return d_in + cfg.max_batch; }
    int32_t* in_seq_lens() const { return d_in + 2 * cfg.max_batch; }
    int32_t* in_slots() const { return d_in + 3 * cfg.max_batch; }
    int32_t* in_tables() const { return d_in + 4 * cfg.max_batch; }

    ~Engine() {
        if (device >= 0) cudaSetDevice(device);
        for (auto& g : graphs) cudaGraphExecDestroy(g.second);  // graphs holding NCCL calls go first
        if (nccl) {
            cudaStreamSynchronize(stream);
            ncclCommDestroy(nccl);
        }
        if (cublas) cublasDestroy(cublas);
        if (stream) cudaStreamDestroy(stream);
        for (void* p : peer_mapped) cudaIpcCloseMemHandle(p);
        void* dev_ptrs[] = {weights, pool, cublas_ws, d_in, d_seq_post, d_next, d_resid, d_x, d_qkv,
                            d_attn, d_attn_out, d_ff, d_ff_out, d_logits, attn_ws, tp_weights, d_gath,
                            d_flags, d_epoch, d_peer_outs, d_peer_flags, d_pin, d_pseq_post, d_pnext,
                            p_resid, p_x, p_qkv, p_attn, p_attn_out, p_ff, p_ff_out, p_last, p_logits,
                            p_attn_ws, d_slot_tables, d_upd, d_attn_loc, lm_ws};
        for (void* p : dev_ptrs)
            if (p) cudaFree(p);
        if (h_in) cudaFreeHost(h_in);
        if (h_upd) cudaFreeHost(h_upd);
        if (h_next) cudaFreeHost(h_next);
        if (h_pin) cudaFreeHost(h_pin);
        if (h_pnext) cudaFreeHost(h_pnext);
    }

    // This rank's slices of the full weights: QKV rows of its heads (zero rows
    // for padding heads) and the output projection widened with zero input
    // columns for the padding heads, so it reads the gathered buffer as is.
    void build_tp_weights() {
        if (tp == 1) return;
        const int D = shape.d_model, L = shape.n_layer;
        const size_t QD = static_cast<size_t>(hl) * head_dim;
        const int h0 = tp_rank * hl;
        const int nreal = std::max(0, std::min(shape.n_head, h0 + hl) - h0);
        const size_t rows = static_cast<size_t>(nreal) * head_dim;
        const size_t w_qkv = align256(3 * QD * D * es), b_qkv = align256(3 * QD * es);
        const size_t w_proj = align256(static_cast<size_t>(D) * tp * QD * es);
        const size_t per = w_qkv + b_qkv + w_proj;
        cuda_ok(cudaMalloc(&tp_weights, per * L), "malloc head-sharded weights");
        cuda_ok(cudaMemsetAsync(tp_weights, 0, per * L, stream), "memset head-sharded weights");
        for (int l = 0; l < L; ++l) {
            const LayerW& w = layers[static_cast<size_t>(l)];
            char* base = static_cast<char*>(tp_weights) + static_cast<size_t>(l) * per;
            char* qw = base;
            char* qb = base + w_qkv;
            char* pw = base + w_qkv + b_qkv;
            for (int part = 0; part < 3; ++part) {  // q, k, v rows of heads [h0, h0 + nreal)
                const size_t src_row = static_cast<size_t>(part) * D + static_cast<size_t>(h0) * head_dim;
                if (rows == 0) break;
                cuda_ok(cudaMemcpyAsync(qw + part * QD * D * es, static_cast<const char*>(w.qkv_w) + src_row * D * es,
                                        rows * D * es, cudaMemcpyDeviceToDevice, stream),
                        "slice qkv_w");
                cuda_ok(cudaMemcpyAsync(qb + part * QD * es, static_cast<const char*>(w.qkv_b) + src_row * es, rows * es,
                                        cudaMemcpyDeviceToDevice, stream),
                        "slice qkv_b");
            }
            cuda_ok(cudaMemcpy2DAsync(pw, tp * QD * es, w.proj_w, static_cast<size_t>(D) * es,
                                      static_cast<size_t>(D) * es, D, cudaMemcpyDeviceToDevice, stream),
                    "pad proj_w");
            qkv_w_loc.push_back(qw);
            qkv_b_loc.push_back(qb);
            proj_w_pad.push_back(pw);
        }
        cuda_ok(cudaStreamSynchronize(stream), "head-sharded weights");
    }

    void check_shape() {
        const B2ModelShape& s = shape;
        if (s.n_layer <= 0 || s.n_head <= 0 || s.d_model <= 0 || s.d_model % s.n_head || s.vocab_size <= 0 ||
            s.n_ctx <= 0)
            throw Error(B2_ERR_SHAPE, "invalid model shape");
        head_dim = s.d_model / s.n_head;
        if (head_dim != 64 && head_dim != 128) throw Error(B2_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
        if (cfg.max_batch <= 0 || cfg.max_seq_len <= 0 || cfg.max_seq_len > s.n_ctx || cfg.kv_block_budget <= 0)
            throw Error(B2_ERR_SHAPE, "invalid engine config (max_batch, max_seq_len <= n_ctx, kv_block_budget)");
        if (cfg.dtype != B2_F32 && cfg.dtype != B2_F16 && cfg.dtype != B2_BF16) throw Error(B2_ERR_DTYPE, "unknown dtype");
        tp = cfg.tp_size <= 1 ? 1 : cfg.tp_size;
        tp_rank = tp == 1 ? 0 : cfg.tp_rank;
        if (tp > B2_MAX_GATHER || tp_rank < 0 || tp_rank >= tp)
            throw Error(B2_ERR_SHAPE, "tp_size must be 1..8 and tp_rank in [0, tp_size)");
        hl = (s.n_head + tp - 1) / tp;
        if (cfg.tp_allgather != 0 && cfg.tp_allgather != 1) throw Error(B2_ERR_SHAPE, "tp_allgather must be 0 or 1");
        tp_nccl = tp > 1 && cfg.tp_allgather == 1;
    }

    // Vocabulary rounded up to a multiple of 8: wte (the tied lm_head) gets
    // zero rows up to it and the logits rows are that long, so the lm_head GEMM
    // has 16-byte aligned rows and columns.  With the odd GPT-2 vocabulary
    // (50257) cuBLAS otherwise falls back to its slow unaligned kernels.
    int vocab_padded() const { return (shape.vocab_size + 7) / 8 * 8; }

    // Weight arena: every tensor at a 256-byte aligned offset, in file order
    // (wte sized for vocab_padded() rows).
    std::vector<size_t> layout(const std::vector<TensorSpec>& specs, size_t* total) const {
        std::vector<size_t> off;
        size_t o = 0;
        for (size_t i = 0; i < specs.size(); ++i) {
            off.push_back(o);
            const size_t n = i == 0 ? static_cast<size_t>(vocab_padded()) * shape.d_model : numel(specs[i].shape);
            o = align256(o + n * es);
        }
        *total = o;
        return off;
    }

    // The KV cache is layer-major: layer l owns a contiguous
    // [num_blocks][K|V][16][n_head][head_dim] region (the paged layout of
    // gpu-engine/include/engine/kv_cache.h:6-8 with n_layer = 1), and a block
    // id names the same slot in every layer.  With all layers inside each
    // block, the slabs one layer's attention reads sit a whole block (4.9 MB
    // for GPT-2 XL) apart, each on its own 2 MB page; over a 100 GB pool the
    // page-translation misses cost attention ~30% of its bandwidth.
    size_t layer_bytes() const {
        return static_cast<size_t>(num_blocks) * 2 * B2_BLOCK_TOKENS * hl * head_dim * es;
    }
    void* layer_pool(int l) const { return static_cast<char*>(pool) + static_cast<size_t>(l) * layer_bytes(); }
    size_t gath_half_bytes() const {
        return static_cast<size_t>(cfg.max_batch) * tp * hl * head_dim * es;
    }

    void bind_tensors(const std::vector<size_t>& off) {
        auto at = [&](size_t i) { return static_cast<const void*>(static_cast<char*>(weights) + off[i]); };
        size_t i = 0;
        wte = at(i++);
        wpe = at(i++);
        layers.resize(static_cast<size_t>(shape.n_layer));
        for (auto& l : layers) {
            l.ln1_g = at(i++);
            l.ln1_b = at(i++);
            l.qkv_w = at(i++);
            l.qkv_b = at(i++);
            l.proj_w = at(i++);
            l.proj_b = at(i++);
            l.ln2_g = at(i++);
            l.ln2_b = at(i++);
            l.fc_w = at(i++);
            l.fc_b = at(i++);
            l.fc_proj_w = at(i++);
            l.fc_proj_b = at(i++);
        }
        lnf_g = at(i++);
        lnf_b = at(i++);
    }

    void setup_device() {
        if (cfg.device >= 0) cuda_ok(cudaSetDevice(cfg.device), "cudaSetDevice");
        cuda_ok(cudaGetDevice(&device), "cudaGetDevice");
        dt = cfg.dtype;
        es = dtype_bytes(dt);
        use_graphs = cfg.use_cuda_graphs != 0;
        cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
        cublas_ok(cublasCreate(&cublas), "cublasCreate");
        cublas_ok(cublasSetStream(cublas, stream), "cublasSetStream");
        // A fixed cuBLAS workspace keeps GEMMs capturable in CUDA graphs.
        const size_t ws = 32u << 20;
        cuda_ok(cudaMalloc(&cublas_ws, ws), "malloc cublas workspace");
        cublas_ok(cublasSetWorkspace(cublas, cublas_ws, ws), "cublasSetWorkspace");
        cublas_ok(cublasSetMathMode(cublas, dt == B2_F32 ? CUBLAS_PEDANTIC_MATH : CUBLAS_DEFAULT_MATH),
                  "cublasSetMathMode");
        if (dt != B2_F32) {
            lt = std::make_unique<LtGemm>();
            lt->init(dt == B2_F16 ? CUDA_R_16F : CUDA_R_16BF, cublas_ws, ws);
        }
    }

    void setup_buffers() {
        const int B = cfg.max_batch, D = shape.d_model, V = shape.vocab_size;
        mbps = (cfg.max_seq_len + B2_BLOCK_TOKENS - 1) / B2_BLOCK_TOKENS;
        num_blocks = cfg.kv_block_budget;
        cuda_ok(cudaMalloc(&pool, layer_bytes() * shape.n_layer), "malloc KV pool");
        cuda_ok(cudaMemsetAsync(pool, 0, layer_bytes() * shape.n_layer, stream), "memset KV pool");
        blocks = std::make_unique<BlockPool>(num_blocks);
        const size_t in_ints = 4 * static_cast<size_t>(B) + static_cast<size_t>(B) * mbps;
        cuda_ok(cudaMalloc(&d_in, in_ints * 4), "malloc step inputs");
        cuda_ok(cudaMemsetAsync(d_in, 0, in_ints * 4, stream), "memset step inputs");
        cuda_ok(cudaMallocHost(&h_in, 4 * static_cast<size_t>(B) * 4), "pinned step inputs");
        std::memset(h_in, 0, 4 * static_cast<size_t>(B) * 4);
        const size_t slot_ints = static_cast<size_t>(num_blocks) * mbps;
        cuda_ok(cudaMalloc(&d_slot_tables, slot_ints * 4), "malloc block tables");
        cuda_ok(cudaMemsetAsync(d_slot_tables, 0, slot_ints * 4, stream), "memset block tables");
        cuda_ok(cudaMalloc(&d_upd, 3 * static_cast<size_t>(kUpdChunk) * 4), "malloc table updates");
        cuda_ok(cudaMallocHost(&h_upd, 3 * static_cast<size_t>(kUpdChunk) * 4), "pinned table updates");
        free_slots.resize(static_cast<size_t>(num_blocks));
        for (int i = 0; i < num_blocks; ++i) free_slots[static_cast<size_t>(i)] = num_blocks - 1 - i;
        cuda_ok(cudaMalloc(&d_seq_post, B * 4), "malloc seq_lens_post");
        cuda_ok(cudaMalloc(&d_next, (B + 1) * 4), "malloc next tokens");
        cuda_ok(cudaMallocHost(&h_next, (B + 1) * 4), "pinned next tokens");
        b2_ok(b2_device_error_word(&d_err_word), "device error word");
        auto act = [&](void** p, size_t cols, const char* what) { cuda_ok(cudaMalloc(p, static_cast<size_t>(B) * cols * es), what); };
        act(&d_resid, D, "malloc residual");
        act(&d_x, D, "malloc ln out");
        act(&d_qkv, 3 * static_cast<size_t>(hl) * head_dim, "malloc qkv");
        if (tp > 1) {
            const size_t gath = 2 * gath_half_bytes();
            cuda_ok(cudaMalloc(&d_gath, gath), "malloc gathered attention output");
            cuda_ok(cudaMemsetAsync(d_gath, 0, gath, stream), "memset gathered attention output");
            const size_t nflags = static_cast<size_t>(shape.n_layer) * tp;
            cuda_ok(cudaMalloc(&d_flags, nflags * 4), "malloc barrier flags");
            cuda_ok(cudaMemsetAsync(d_flags, 0, nflags * 4, stream), "memset barrier flags");
            cuda_ok(cudaMalloc(&d_epoch, 4), "malloc epoch");
            cuda_ok(cudaMemsetAsync(d_epoch, 0, 4, stream), "memset epoch");
            cuda_ok(cudaMalloc(&d_peer_outs, 2 * tp * sizeof(void*)), "malloc peer table");
            cuda_ok(cudaMalloc(&d_peer_flags, tp * sizeof(void*)), "malloc peer table");
            if (tp_nccl) act(&d_attn_loc, static_cast<size_t>(hl) * head_dim, "malloc local attention slice");
        }
        act(&d_attn, D, "malloc attention out");
        act(&d_attn_out, D, "malloc proj out");
        act(&d_ff, 4 * static_cast<size_t>(D), "malloc ff");
        act(&d_ff_out, D, "malloc ff out");
        act(&d_logits, static_cast<size_t>(vocab_padded()), "malloc logits");
        B2PagedAttnArgs a = attn_args(B, 0);
        attn_ws_bytes = b2_paged_attention_workspace_bytes(&a);
        if (attn_ws_bytes == 0) throw Error(B2_ERR_UNSUPPORTED, std::string("attention shape: ") + b2_last_error_string());
        cuda_ok(cudaMalloc(&attn_ws, attn_ws_bytes), "malloc attention workspace");
        cuda_ok(cudaMemsetAsync(attn_ws, 0, attn_ws_bytes, stream), "zero attention workspace");
        bucket_cap = B;
        cuda_ok(cudaStreamSynchronize(stream), "engine set-up");
    }

    B2PagedAttnArgs attn_args(int bucket, int layer) const {
        B2PagedAttnArgs a{};
        a.dtype = dt;
        a.out_dtype = dt;
        a.q = d_qkv;
        a.q_row_stride = 3 * hl * head_dim;
        a.kv_pool = layer_pool(layer);
        a.block_tables = in_tables();
        a.seq_lens = d_seq_post;
        a.out = tp > 1 ? d_gath : d_attn;
        a.batch = bucket;
        a.n_head = hl;
        a.n_kv_head = hl;
        a.head_dim = head_dim;
        a.max_blocks_per_seq = mbps;
        a.layer_idx = 0;
        a.n_layer = 1;
        a.num_blocks = num_blocks;
        return a;
    }

    // Row-major Y[batch, O] = X[batch, I] . W^T with W row-major [O, I]: the
    // convention of gpu-engine/include/engine/kernels.h:9-20.  ldy (>= O) is the
    // row stride of Y.
    // The decode step's GEMMs go to b2_linear (tcgen05, split-K over a cluster,
    // weights streamed before griddepcontrol.wait so they overlap the kernel
    // before) when switched on, for 16-bit models, batches of at most 256 rows
    // and layers whose 128-feature tiles fit the GPU in one wave; cuBLAS
    // otherwise.  With gelu_bias the caller's bias + GELU is fused into the
    // GEMM's epilogue; the return value says whether that happened.
    bool linear_ok(int batch, int O) const {
        return linear_tc && dt != B2_F32 && batch <= 256 && (O + 127) / 128 <= 148;
    }
    bool lt_on() const { return lt && (gemm_mode & 1) && in_decode; }
    bool capturing() const {
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(stream, &st);
        return st != cudaStreamCaptureStatusNone;
    }
    bool gemm_fused(int batch, int I, int O, const void* X, const void* W, void* Y, const void* gelu_bias) {
        if (!linear_ok(batch, O)) {
            if (gelu_bias && lt_on() && (gemm_mode & 2)) {
                lt->run(batch, I, O, X, W, Y, O, LtGemm::kGeluBias, gelu_bias, stream, !capturing());
                return true;
            }
            gemm(batch, I, O, X, W, Y);
            return false;
        }
        B2LinearArgs la{};
        la.dtype = dt;
        la.x = X;
        la.x_row_stride = I;
        la.w = W;
        la.bias = gelu_bias;
        la.y = Y;
        la.y_row_stride = O;
        la.batch = batch;
        la.in_features = I;
        la.out_features = O;
        la.epilogue = gelu_bias ? B2_LINEAR_GELU : B2_LINEAR_STORE;
        b2_ok(b2_linear(&la, stream), "linear");
        return gelu_bias != nullptr;
    }
    void gemm(int batch, int I, int O, const void* X, const void* W, void* Y, int ldy = 0) {
        if (ldy == 0 && linear_ok(batch, O)) {
            gemm_fused(batch, I, O, X, W, Y, nullptr);
            return;
        }
        if (lt_on()) {
            lt->run(batch, I, O, X, W, Y, ldy > 0 ? ldy : O, LtGemm::kNone, nullptr, stream, !capturing());
            return;
        }
        const float alpha = 1.0f, beta = 0.0f;
        const cudaDataType_t t = dt == B2_F32 ? CUDA_R_32F : (dt == B2_F16 ? CUDA_R_16F : CUDA_R_16BF);
        cublas_ok(cublasGemmEx(cublas, CUBLAS_OP_T, CUBLAS_OP_N, O, batch, I, &alpha, W, t, I, X, t, I, &beta, Y, t,
                               ldy > 0 ? ldy : O, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT),
                  "cublasGemmEx");
    }

    void run_step_kernels(int bucket) {
        in_decode = true;
        struct Leave {
            bool& f;
            ~Leave() { f = false; }
        } leave{in_decode};
        const int D = shape.d_model, V = shape.vocab_size, L = shape.n_layer;
        const float eps = shape.layer_norm_epsilon;
        b2_stream_t s = stream;
        const char* qkv = static_cast<const char*>(d_qkv);
        if (tp > 1 && !tp_nccl) b2_ok(b2_tp_epoch_bump(d_epoch, s), "tp_epoch_bump");  // a new step for the barriers
        // this step's block tables, gathered from the device-resident slot rows
        gather_step_tables_kernel<<<bucket, 64, 0, stream>>>(in_tables(), d_slot_tables, in_slots(), in_seq_lens(),
                                                              mbps);
        cuda_ok(cudaGetLastError(), "gather step tables");
        b2_ok(b2_embedding(dt, d_resid, wte, wpe, in_tokens(), in_positions(), bucket, D, V, shape.n_ctx, s), "embedding");
        const void* delta = nullptr;
        const void* delta_bias = nullptr;
        for (int l = 0; l < L; ++l) {
            const LayerW& w = layers[static_cast<size_t>(l)];
            b2_ok(b2_add_layernorm(dt, d_x, d_resid, delta, delta_bias, d_resid, w.ln1_g, w.ln1_b, bucket, D, eps, s), "ln1");
            // this engine's heads: all of them, or its slice when head-sharded
            const int QD = hl * head_dim;
            const void* qkv_w = tp > 1 ? qkv_w_loc[static_cast<size_t>(l)] : w.qkv_w;
            const char* qkv_b = static_cast<const char*>(tp > 1 ? qkv_b_loc[static_cast<size_t>(l)] : w.qkv_b);
            gemm(bucket, D, 3 * QD, d_x, qkv_w, d_qkv);
            B2KvAppendArgs ka{};
            ka.dtype = dt;
            ka.kv_pool = layer_pool(l);
            ka.k = qkv + static_cast<size_t>(QD) * es;
            ka.v = qkv + 2 * static_cast<size_t>(QD) * es;
            ka.kv_row_stride = 3 * QD;
            ka.k_bias = qkv_b + static_cast<size_t>(QD) * es;
            ka.v_bias = qkv_b + 2 * static_cast<size_t>(QD) * es;
            ka.block_tables = in_tables();
            ka.seq_lens = in_seq_lens();
            ka.seq_lens_post = l == 0 ? d_seq_post : nullptr;  // same for every layer
            ka.batch = bucket;
            ka.n_kv_head = hl;
            ka.head_dim = head_dim;
            ka.max_blocks_per_seq = mbps;
            ka.layer_idx = 0;
            ka.n_layer = 1;
            ka.num_blocks = num_blocks;
            b2_ok(b2_kv_append(&ka, s), "kv_append");
            B2PagedAttnArgs aa = attn_args(bucket, l);
            aa.q_bias = qkv_b;
            // Past layer 0, seq_lens_post, the block tables, q and every key row
            // but the newest were complete before kv_append started -- when the
            // QKV GEMM was cuBLAS, which lets kv_append start only once it has
            // finished.  b2_linear lets its dependents start early (kv_append
            // may begin while q is still being written), so then attention
            // waits for kv_append before reading anything.
            if (l > 0 && !linear_ok(bucket, 3 * QD)) aa.flags = B2_ATTN_NEWEST_ROW_PENDING;
            if (tp_nccl) {
                // this rank's heads, then ncclAllGather of every rank's slice and
                // the interleave into [row][rank slices] for the projection
                aa.out = d_attn_loc;
                b2_ok(b2_paged_attention(&aa, attn_ws, attn_ws_bytes, s), "paged_attention");
                const ncclDataType_t nt = dt == B2_F32 ? ncclFloat32 : (dt == B2_F16 ? ncclFloat16 : ncclBfloat16);
                nccl_ok(ncclAllGather(d_attn_loc, d_gath, static_cast<size_t>(bucket) * QD, nt, nccl, stream),
                        "ncclAllGather");
                const int qchunks = QD * es / 16;
                void* inter = static_cast<char*>(d_gath) + gath_half_bytes();
                const long long total = static_cast<long long>(bucket) * tp * qchunks;
                interleave_slices_kernel<<<static_cast<int>(std::min<long long>((total + 255) / 256, 148 * 8)), 256, 0,
                                           stream>>>(static_cast<uint4*>(inter), static_cast<const uint4*>(d_gath),
                                                     bucket, tp, qchunks);
                cuda_ok(cudaGetLastError(), "interleave gathered slices");
                gemm(bucket, tp * QD, D, inter, proj_w_pad[static_cast<size_t>(l)], d_attn_out);
            } else if (tp > 1) {
                // all-gather in the attention epilogue, then meet the peers
                const int par = l & 1;  // gathered-buffer half of this layer
                B2OutputGather g{d_peer_outs + par * tp, tp, static_cast<int64_t>(tp) * QD,
                                 static_cast<int64_t>(tp_rank) * QD};
                b2_ok(b2_paged_attention_gather(&aa, attn_ws, attn_ws_bytes, &g, s), "paged_attention_gather");
                b2_ok(b2_tp_barrier(d_flags, d_peer_flags, tp_rank, tp, d_epoch, l, s), "tp_barrier");
                gemm(bucket, tp * QD, D, static_cast<char*>(d_gath) + par * gath_half_bytes(),
                     proj_w_pad[static_cast<size_t>(l)], d_attn_out);
            } else {
                b2_ok(b2_paged_attention(&aa, attn_ws, attn_ws_bytes, s), "paged_attention");
                gemm(bucket, D, D, d_attn, w.proj_w, d_attn_out);
            }
            b2_ok(b2_add_layernorm(dt, d_x, d_resid, d_attn_out, w.proj_b, d_resid, w.ln2_g, w.ln2_b, bucket, D, eps, s), "ln2");
            if (!gemm_fused(bucket, D, 4 * D, d_x, w.fc_w, d_ff, w.fc_b))
                b2_ok(b2_bias_gelu(dt, d_ff, d_ff, w.fc_b, bucket, 4 * D, s), "bias_gelu");
            gemm(bucket, 4 * D, D, d_ff, w.fc_proj_w, d_ff_out);
            delta = d_ff_out;
            delta_bias = w.fc_proj_b;
        }
        b2_ok(b2_add_layernorm(dt, d_x, d_resid, delta, delta_bias, d_resid, lnf_g, lnf_b, bucket, D, eps, s), "ln_f");
        lm_head_argmax(bucket, d_x, d_logits, d_next);
        copy_error_word_kernel<<<1, 32, 0, stream>>>(d_next + cfg.max_batch, d_err_word);
        cuda_ok(cudaGetLastError(), "copy error word");
    }

    // Next tokens of `rows` final hidden rows x [rows][D]: the lm_head tied to
    // wte over the padded vocabulary into `logits` (pad logits are 0 and never
    // read by the argmax), then the argmax -- or, with lm_fused, both in one
    // b2_lm_head_argmax launch that writes no logits.
    void lm_head_argmax(int rows, const void* x, void* logits, int32_t* next) {
        cudaStream_t s = stream;
        const int D = shape.d_model, V = shape.vocab_size;
        if (lm_fused) {
            B2LmHeadArgmaxArgs la{};
            la.dtype = dt;
            la.x = x;
            la.x_row_stride = D;
            la.w = wte;
            la.batch = rows;
            la.d_model = D;
            la.vocab = V;
            la.out_tokens = next;
            la.workspace = lm_ws;
            la.workspace_bytes = lm_ws_bytes;
            b2_ok(b2_lm_head_argmax(&la, s), "lm_head_argmax");
            return;
        }
        gemm(rows, D, vocab_padded(), x, wte, logits, vocab_padded());
        b2_ok(b2_argmax_rows(dt, next, logits, vocab_padded(), rows, V, s), "argmax");
    }

    // After a step's synchronisation: a nonzero device error word (a bounded
    // wait that gave up, a clamped block id, seq_len or token) means the
    // step's results are invalid.  The word is per device and shared by every
    // user of libb2decode on it; it is cleared here and the step fails.
    void check_device_errors(uint32_t bits) {
        if (bits == 0) return;
        cuda_ok(cudaMemsetAsync(d_err_word, 0, 4, stream), "clear device error word");
        cuda_ok(cudaStreamSynchronize(stream), "clear device error word");
        std::string what;
        if (bits & B2_DEVERR_BLOCK_ID) what += " block id out of range;";
        if (bits & B2_DEVERR_SEQ_LEN) what += " seq_len beyond the block table;";
        if (bits & B2_DEVERR_TIMEOUT) what += " a bounded wait gave up;";
        if (bits & B2_DEVERR_TOKEN) what += " token id or position out of range;";
        char hex[16];
        std::snprintf(hex, sizeof(hex), "0x%x", bits);
        throw Error(B2_ERR_KERNEL, std::string("device-side error bits ") + hex + ":" + what +
                                       " the step's tokens are invalid and no sequence advanced");
    }

    cudaGraphExec_t graph_for(int bucket) {
        auto it = graphs.find(bucket);
        if (it != graphs.end()) return it->second;
        // cuBLASLt shapes are timed outside any capture: one eager pass of the
        // step first (the step is idempotent: same inputs, same writes).
        if (lt && (gemm_mode & 1)) run_step_kernels(bucket);
        cudaGraph_t g = nullptr;
        cuda_ok(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
        try {
            run_step_kernels(bucket);
        } catch (...) {
            cudaStreamEndCapture(stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        cuda_ok(cudaStreamEndCapture(stream, &g), "cudaStreamEndCapture");
        cudaGraphExec_t exec = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        cuda_ok(e, "cudaGraphInstantiate");
        graphs[bucket] = exec;
        return exec;
    }

    // Batch buckets 1, 2, 4, ... up to max_batch (the reference stops at 8,
    // engine.cu:52-59, and pads everything larger to max_batch).
    int pick_bucket(int batch) const {
        int b = 1;
        while (b < batch) b <<= 1;
        return b < cfg.max_batch ? b : cfg.max_batch;
    }

    // Prefill attention on the tensor cores (b2_prefill_attention) for 16-bit
    // models of head_dim 64 unless switched off; otherwise one decode-attention
    // row per prompt token.
    bool tc_prefill() const { return prefill_tc && dt != B2_F32 && head_dim == 64; }

    void setup_prefill() {
        if (prefill_cap > 0) return;
        const int cap = cfg.max_prefill_tokens > 0 ? cfg.max_prefill_tokens : 2048;
        const int B = cfg.max_batch, D = shape.d_model;
        // [tok|pos|seq_len per row][last row|pre|start|rows per sequence][block table per sequence][per row]
        const size_t in_ints = 3 * static_cast<size_t>(cap) + 4 * static_cast<size_t>(B) +
                               static_cast<size_t>(B) * mbps + static_cast<size_t>(cap) * mbps;
        cuda_ok(cudaMalloc(&d_pin, in_ints * 4), "malloc prefill inputs");
        cuda_ok(cudaMallocHost(&h_pin, in_ints * 4), "pinned prefill inputs");
        std::memset(h_pin, 0, in_ints * 4);
        cuda_ok(cudaMalloc(&d_pseq_post, static_cast<size_t>(cap) * 4), "malloc prefill seq_lens_post");
        cuda_ok(cudaMalloc(&d_pnext, static_cast<size_t>(B + 1) * 4), "malloc prefill next tokens");
        cuda_ok(cudaMallocHost(&h_pnext, static_cast<size_t>(B + 1) * 4), "pinned prefill next tokens");
        auto act = [&](void** p, size_t rows, size_t cols, const char* what) {
            cuda_ok(cudaMalloc(p, rows * cols * es), what);
        };
        const size_t QD = static_cast<size_t>(hl) * head_dim;
        act(&p_resid, cap, D, "malloc prefill residual");
        act(&p_x, cap, D, "malloc prefill ln out");
        act(&p_qkv, cap, 3 * QD, "malloc prefill qkv");
        act(&p_attn, cap, D, "malloc prefill attention out");
        act(&p_attn_out, cap, D, "malloc prefill proj out");
        act(&p_ff, cap, 4 * static_cast<size_t>(D), "malloc prefill ff");
        act(&p_ff_out, cap, D, "malloc prefill ff out");
        act(&p_last, B, D, "malloc prefill last rows");
        act(&p_logits, B, static_cast<size_t>(vocab_padded()), "malloc prefill logits");
        prefill_cap = cap;
    }

    // The decode-attention workspace of the row-per-token prefill path (f32
    // models, or tensor-core prefill switched off), made on first use: the
    // tcgen05 prefill attention needs none, so an engine that only uses it can
    // take prompt-token budgets larger than one decode-attention launch allows.
    void prefill_rows_workspace() {
        if (p_attn_ws) return;
        B2PagedAttnArgs a = attn_args(prefill_cap, 0);
        p_attn_ws_bytes = b2_paged_attention_workspace_bytes(&a);
        if (p_attn_ws_bytes == 0)
            throw Error(B2_ERR_UNSUPPORTED, std::string("prefill through decode-attention rows (max_prefill_tokens too "
                                                        "large for one launch?): ") + b2_last_error_string());
        cuda_ok(cudaMalloc(&p_attn_ws, p_attn_ws_bytes), "malloc prefill attention workspace");
        cuda_ok(cudaMemsetAsync(p_attn_ws, 0, p_attn_ws_bytes, stream), "zero prefill attention workspace");
    }

    // One pass over every remaining prompt token of the listed sequences: the
    // decode step's kernels with one row per token.  Row r of sequence s is
    // position p = seq_len(s) + t; kv_append writes its K/V at p and attention
    // reads positions [0, p]: each sequence's rows as 128-row query tiles on the
    // tensor cores (tc_prefill), or one decode-attention row per token.
    void prefill(const int32_t* ids, int n, int32_t* out) {
        if (tp > 1) throw Error(B2_ERR_UNSUPPORTED, "batched prefill is not available on head-sharded engines");
        if (n <= 0 || n > cfg.max_batch) throw Error(B2_ERR_SHAPE, "n must be in [1, max_batch]");
        setup_prefill();
        std::vector<Seq*> sv(static_cast<size_t>(n));
        int rows = 0, need = 0;
        for (int i = 0; i < n; ++i) {
            auto it = seqs.find(ids[i]);
            if (it == seqs.end()) throw Error(B2_ERR_SHAPE, "unknown sequence id " + std::to_string(ids[i]));
            Seq& q = it->second;
            for (int j = 0; j < i; ++j)
                if (sv[static_cast<size_t>(j)] == &q) throw Error(B2_ERR_SHAPE, "sequence listed twice in one call");
            const int t = static_cast<int>(q.prompt.size()) - q.prompt_pos;
            if (t <= 0) throw Error(B2_ERR_SHAPE, "sequence " + std::to_string(ids[i]) + " is past its prompt");
            if (q.seq_len + t > cfg.max_seq_len) throw Error(B2_ERR_SHAPE, "prompt longer than max_seq_len");
            sv[static_cast<size_t>(i)] = &q;
            rows += t;
            const int have = static_cast<int>(q.table.ids.size());
            const int want = (q.seq_len + t + B2_BLOCK_TOKENS - 1) / B2_BLOCK_TOKENS;
            need += std::max(0, want - have);
        }
        if (rows > prefill_cap) throw Error(B2_ERR_SHAPE, "more prompt tokens than max_prefill_tokens in one call");
        if (!tc_prefill()) prefill_rows_workspace();
        if (need > blocks->num_free()) throw Error(B2_ERR_POOL, "KV cache block pool exhausted");
        const int cap = prefill_cap, B = cfg.max_batch, D = shape.d_model, V = shape.vocab_size, L = shape.n_layer;
        const size_t seq_off = 3 * static_cast<size_t>(cap);          // last, pre, start, rows: B each
        const size_t sbt_off = seq_off + 4 * static_cast<size_t>(B);  // per-sequence block tables
        const size_t bt_off = sbt_off + static_cast<size_t>(B) * mbps;
        int32_t* tok = h_pin;
        int32_t* pos = h_pin + cap;
        int32_t* sl = h_pin + 2 * cap;
        int32_t* last = h_pin + seq_off;
        int32_t* s_pre = last + B;
        int32_t* s_start = last + 2 * B;
        int32_t* s_rows = last + 3 * B;
        int32_t* sbt = h_pin + sbt_off;
        int32_t* bt = h_pin + bt_off;
        int r = 0, max_t = 0;
        for (int i = 0; i < n; ++i) {
            Seq& q = *sv[static_cast<size_t>(i)];
            const int t = static_cast<int>(q.prompt.size()) - q.prompt_pos;
            while (static_cast<int>(q.table.ids.size()) * B2_BLOCK_TOKENS < q.seq_len + t) grow(q);
            s_pre[i] = q.seq_len;
            s_start[i] = r;
            s_rows[i] = t;
            max_t = std::max(max_t, t);
            int32_t* srow = sbt + static_cast<size_t>(i) * mbps;
            for (size_t j = 0; j < q.table.ids.size(); ++j) srow[j] = q.table.ids[j];
            for (int k = 0; k < t; ++k, ++r) {
                tok[r] = q.prompt[static_cast<size_t>(q.prompt_pos + k)];
                pos[r] = q.seq_len + k;
                sl[r] = q.seq_len + k;
                int32_t* row = bt + static_cast<size_t>(r) * mbps;
                for (size_t j = 0; j < q.table.ids.size(); ++j) row[j] = q.table.ids[j];
            }
            last[i] = r - 1;
        }
        const size_t up = (bt_off + static_cast<size_t>(rows) * mbps) * 4;
        cuda_ok(cudaMemcpyAsync(d_pin, h_pin, up, cudaMemcpyHostToDevice, stream), "upload prefill inputs");
        const int32_t* d_tok = d_pin;
        const int32_t* d_pos = d_pin + cap;
        const int32_t* d_sl = d_pin + 2 * cap;
        const int32_t* d_last = d_pin + seq_off;
        const int32_t* d_bt = d_pin + bt_off;
        const float eps = shape.layer_norm_epsilon;
        b2_stream_t s = stream;
        const char* qkv = static_cast<const char*>(p_qkv);
        b2_ok(b2_embedding(dt, p_resid, wte, wpe, d_tok, d_pos, rows, D, V, shape.n_ctx, s), "embedding");
        const void* delta = nullptr;
        const void* delta_bias = nullptr;
        for (int l = 0; l < L; ++l) {
            const LayerW& w = layers[static_cast<size_t>(l)];
            b2_ok(b2_add_layernorm(dt, p_x, p_resid, delta, delta_bias, p_resid, w.ln1_g, w.ln1_b, rows, D, eps, s), "ln1");
            gemm(rows, D, 3 * D, p_x, w.qkv_w, p_qkv);
            B2KvAppendArgs ka{};
            ka.dtype = dt;
            ka.kv_pool = layer_pool(l);
            ka.k = qkv + static_cast<size_t>(D) * es;
            ka.v = qkv + 2 * static_cast<size_t>(D) * es;
            ka.kv_row_stride = 3 * D;
            ka.k_bias = static_cast<const char*>(w.qkv_b) + static_cast<size_t>(D) * es;
            ka.v_bias = static_cast<const char*>(w.qkv_b) + 2 * static_cast<size_t>(D) * es;
            ka.block_tables = d_bt;
            ka.seq_lens = d_sl;
            ka.seq_lens_post = l == 0 ? d_pseq_post : nullptr;
            ka.batch = rows;
            ka.n_kv_head = hl;
            ka.head_dim = head_dim;
            ka.max_blocks_per_seq = mbps;
            ka.layer_idx = 0;
            ka.n_layer = 1;
            ka.num_blocks = num_blocks;
            b2_ok(b2_kv_append(&ka, s), "kv_append");
            if (tc_prefill()) {
                // causal attention of each sequence's new rows, 128-row query tiles on tcgen05
                B2PrefillAttnArgs pa{};
                pa.dtype = dt;
                pa.q = p_qkv;
                pa.q_row_stride = 3 * D;
                pa.q_bias = w.qkv_b;
                pa.kv_pool = layer_pool(l);
                pa.block_tables = d_pin + sbt_off;
                pa.seq_lens_pre = d_pin + seq_off + B;
                pa.q_start = d_pin + seq_off + 2 * B;
                pa.q_len = d_pin + seq_off + 3 * B;
                pa.out = p_attn;
                pa.out_row_stride = D;
                pa.n_seqs = n;
                pa.n_head = shape.n_head;
                pa.n_kv_head = shape.n_head;
                pa.head_dim = head_dim;
                pa.max_blocks_per_seq = mbps;
                pa.layer_idx = 0;
                pa.n_layer = 1;
                pa.num_blocks = num_blocks;
                pa.max_q_len = max_t;
                b2_ok(b2_prefill_attention(&pa, s), "prefill_attention");
            } else {
                // one decode row per prompt token: row r reads keys [0, position]
                B2PagedAttnArgs aa = attn_args(rows, l);
                aa.q = p_qkv;
                aa.q_bias = w.qkv_b;
                aa.block_tables = d_bt;
                aa.seq_lens = d_pseq_post;
                aa.out = p_attn;
                b2_ok(b2_paged_attention(&aa, p_attn_ws, p_attn_ws_bytes, s), "paged_attention");
            }
            gemm(rows, D, D, p_attn, w.proj_w, p_attn_out);
            b2_ok(b2_add_layernorm(dt, p_x, p_resid, p_attn_out, w.proj_b, p_resid, w.ln2_g, w.ln2_b, rows, D, eps, s),
                  "ln2");
            gemm(rows, D, 4 * D, p_x, w.fc_w, p_ff);
            b2_ok(b2_bias_gelu(dt, p_ff, p_ff, w.fc_b, rows, 4 * D, s), "bias_gelu");
            gemm(rows, 4 * D, D, p_ff, w.fc_proj_w, p_ff_out);
            delta = p_ff_out;
            delta_bias = w.fc_proj_b;
        }
        b2_ok(b2_add_layernorm(dt, p_x, p_resid, delta, delta_bias, p_resid, lnf_g, lnf_b, rows, D, eps, s), "ln_f");
        const int cols = D * es / 16;
        gather_rows_kernel<<<std::min(n, 1024), 128, 0, stream>>>(static_cast<uint4*>(p_last),
                                                                  static_cast<const uint4*>(p_x), d_last, n, cols);
        cuda_ok(cudaGetLastError(), "gather last rows");
        lm_head_argmax(n, p_last, p_logits, d_pnext);
        copy_error_word_kernel<<<1, 32, 0, stream>>>(d_pnext + B, d_err_word);
        cuda_ok(cudaGetLastError(), "copy error word");
        cuda_ok(cudaMemcpyAsync(h_pnext, d_pnext, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, stream),
                "download next tokens");
        cuda_ok(cudaMemcpyAsync(h_pnext + B, d_pnext + B, 4, cudaMemcpyDeviceToHost, stream), "download error word");
        cuda_ok(cudaStreamSynchronize(stream), "prefill");
        check_device_errors(static_cast<uint32_t>(h_pnext[B]));
        for (int i = 0; i < n; ++i) {
            Seq& q = *sv[static_cast<size_t>(i)];
            const int t = static_cast<int>(q.prompt.size()) - q.prompt_pos;
            q.seq_len += t;
            q.prompt_pos = static_cast<int>(q.prompt.size());
            q.last_token = h_pnext[i];
            out[i] = h_pnext[i];
        }
    }

    // ---- sequences and their device-resident block tables

    // Registers a sequence whose table already holds its first blocks: a slot,
    // and one pending table update per block.
    int32_t register_seq(Seq&& q) {
        if (free_slots.empty()) throw Error(B2_ERR_POOL, "no free block-table slot");
        q.slot = free_slots.back();
        free_slots.pop_back();
        for (size_t j = 0; j < q.table.ids.size(); ++j) note_block(q, static_cast<int>(j));
        const int32_t id = next_id++;
        seqs.emplace(id, std::move(q));
        return id;
    }

    void note_block(const Seq& q, int j) {
        pending_upd.push_back(q.slot);
        pending_upd.push_back(j);
        pending_upd.push_back(q.table.ids[static_cast<size_t>(j)]);
    }

    // One more block at the end of q's table (the caller checked the pool).
    void grow(Seq& q) {
        q.table.ids.push_back(blocks->allocate());
        note_block(q, static_cast<int>(q.table.ids.size()) - 1);
    }

    void release_seq(int32_t id) {
        auto it = seqs.find(id);
        if (it == seqs.end()) return;
        for (int blk : it->second.table.ids) blocks->free(blk);
        free_slots.push_back(it->second.slot);
        seqs.erase(it);
    }

    // Uploads the pending table updates and scatters them into the slot rows
    // (stream-ordered before the step that needs them).
    void flush_table_updates() {
        const size_t n = pending_upd.size() / 3;
        for (size_t done = 0; done < n; done += kUpdChunk) {
            const int m = static_cast<int>(std::min<size_t>(kUpdChunk, n - done));
            // the staging buffer is reused: the previous chunk's copy must have left it
            cuda_ok(cudaStreamSynchronize(stream), "table update staging");
            std::memcpy(h_upd, pending_upd.data() + 3 * done, static_cast<size_t>(m) * 12);
            cuda_ok(cudaMemcpyAsync(d_upd, h_upd, static_cast<size_t>(m) * 12, cudaMemcpyHostToDevice, stream),
                    "upload table updates");
            scatter_table_updates_kernel<<<(m + 255) / 256, 256, 0, stream>>>(d_slot_tables, d_upd, m, mbps);
            cuda_ok(cudaGetLastError(), "scatter table updates");
        }
        pending_upd.clear();
    }

    void decode_step(const int32_t* ids, int batch, int32_t* out) {
        if (batch <= 0 || batch > cfg.max_batch) throw Error(B2_ERR_SHAPE, "batch must be in [1, max_batch]");
        if (tp > 1 && !tp_connected) throw Error(B2_ERR_SHAPE, "head-sharded engine is not connected (b2_engine_tp_connect)");
        std::vector<Seq*> sv(static_cast<size_t>(batch));
        int need = 0;
        for (int i = 0; i < batch; ++i) {
            auto it = seqs.find(ids[i]);
            if (it == seqs.end()) throw Error(B2_ERR_SHAPE, "unknown sequence id " + std::to_string(ids[i]));
            Seq& q = it->second;
            if (q.seq_len >= cfg.max_seq_len) throw Error(B2_ERR_SHAPE, "sequence " + std::to_string(ids[i]) + " reached max_seq_len");
            for (int j = 0; j < i; ++j)
                if (sv[static_cast<size_t>(j)] == &q) throw Error(B2_ERR_SHAPE, "sequence listed twice in one step");
            sv[static_cast<size_t>(i)] = &q;
            if (static_cast<int>(q.table.ids.size()) * B2_BLOCK_TOKENS <= q.seq_len) ++need;
        }
        if (need > blocks->num_free()) throw Error(B2_ERR_POOL, "KV cache block pool exhausted");
        const int bucket = pick_bucket(batch);
        const int B = cfg.max_batch;
        int32_t* tok = h_in;
        int32_t* pos = h_in + B;
        int32_t* sl = h_in + 2 * B;
        int32_t* slot = h_in + 3 * B;
        for (int i = 0; i < batch; ++i) {
            Seq& q = *sv[static_cast<size_t>(i)];
            if (static_cast<int>(q.table.ids.size()) * B2_BLOCK_TOKENS <= q.seq_len) grow(q);
            tok[i] = q.prompt_pos < static_cast<int>(q.prompt.size()) ? q.prompt[static_cast<size_t>(q.prompt_pos)] : q.last_token;
            pos[i] = q.seq_len;
            sl[i] = q.seq_len;
            slot[i] = q.slot;
        }
        for (int i = batch; i < bucket; ++i) {  // pad lanes replay the last real lane
            tok[i] = tok[batch - 1];
            pos[i] = pos[batch - 1];
            sl[i] = sl[batch - 1];
            slot[i] = slot[batch - 1];
        }
        // the h_in copy of the previous step is complete: that step synchronised
        flush_table_updates();
        cuda_ok(cudaMemcpyAsync(d_in, h_in, 4 * static_cast<size_t>(B) * 4, cudaMemcpyHostToDevice, stream),
                "upload step inputs");
        if (use_graphs)
            cuda_ok(cudaGraphLaunch(graph_for(bucket), stream), "cudaGraphLaunch");
        else
            run_step_kernels(bucket);
        if (batch < B) {
            cuda_ok(cudaMemcpyAsync(h_next, d_next, static_cast<size_t>(batch) * 4, cudaMemcpyDeviceToHost, stream),
                    "download next tokens");
            cuda_ok(cudaMemcpyAsync(h_next + B, d_next + B, 4, cudaMemcpyDeviceToHost, stream), "download error word");
        } else {
            cuda_ok(cudaMemcpyAsync(h_next, d_next, static_cast<size_t>(B + 1) * 4, cudaMemcpyDeviceToHost, stream),
                    "download next tokens");
        }
        cuda_ok(cudaStreamSynchronize(stream), "decode step");
        check_device_errors(static_cast<uint32_t>(h_next[B]));
        for (int i = 0; i < batch; ++i) {
            Seq& q = *sv[static_cast<size_t>(i)];
            if (q.prompt_pos < static_cast<int>(q.prompt.size())) ++q.prompt_pos;
            ++q.seq_len;
            q.last_token = h_next[i];
            out[i] = h_next[i];
        }
    }
};

// ----------------------------------------------------------- weight files

B2ModelShape read_config(const std::string& dir) {
    std::ifstream f(dir + "/config.json");
    if (!f) throw Error(B2_ERR_IO, "cannot open " + dir + "/config.json");
    nlohmann::json j;
    f >> j;
    B2ModelShape s{};
    s.n_layer = j.at("n_layer").get<int>();
    s.n_head = j.at("n_head").get<int>();
    s.d_model = j.at("d_model").get<int>();
    s.vocab_size = j.at("vocab_size").get<int>();
    s.n_ctx = j.at("n_ctx").get<int>();
    s.layer_norm_epsilon = j.at("layer_norm_epsilon").get<float>();
    s.eos_token_id = j.at("eos_token_id").get<int>();
    if (j.at("head_dim").get<int>() * s.n_head != s.d_model) throw Error(B2_ERR_IO, "config.json: head_dim * n_head != d_model");
    return s;
}

// Reads weights.bin / manifest.json, checks them the way the reference's
// WeightsLoader does (total_bytes, byte ranges, shapes, the double
// checksum_sum to 1e-6 relative; weights_loader.cpp:28-71), converts to the
// engine dtype and uploads into the arena.
void load_weights(Engine& e, const std::string& dir) {
    std::ifstream mf(dir + "/manifest.json");
    if (!mf) throw Error(B2_ERR_IO, "cannot open " + dir + "/manifest.json");
    nlohmann::json man;
    mf >> man;
    std::ifstream wf(dir + "/weights.bin", std::ios::binary | std::ios::ate);
    if (!wf) throw Error(B2_ERR_IO, "cannot open " + dir + "/weights.bin");
    const size_t file_bytes = static_cast<size_t>(wf.tellg());
    wf.seekg(0);
    if (file_bytes != man.at("total_bytes").get<size_t>()) throw Error(B2_ERR_IO, "weights.bin size differs from manifest total_bytes");
    std::vector<char> blob(file_bytes);
    wf.read(blob.data(), static_cast<std::streamsize>(file_bytes));
    if (!wf) throw Error(B2_ERR_IO, "short read of weights.bin");
    std::unordered_map<std::string, const nlohmann::json*> by_name;
    for (const auto& t : man.at("tensors")) by_name[t.at("name").get<std::string>()] = &t;

    const auto specs = tensor_specs(e.shape);
    size_t total = 0;
    const auto off = e.layout(specs, &total);
    cuda_ok(cudaMalloc(&e.weights, total), "malloc weights");
    char* staging = nullptr;
    cuda_ok(cudaMallocHost(&staging, total), "pinned weight staging");
    std::unique_ptr<char, void (*)(char*)> guard(staging, [](char* p) { cudaFreeHost(p); });
    std::memset(staging, 0, total);  // padding, including wte's zero rows past the vocabulary
    double checksum = 0.0;
    for (size_t i = 0; i < specs.size(); ++i) {
        auto it = by_name.find(specs[i].name);
        if (it == by_name.end()) throw Error(B2_ERR_IO, "manifest lacks tensor " + specs[i].name);
        const nlohmann::json& t = *it->second;
        std::vector<int64_t> shp;
        for (auto& d : t.at("shape")) shp.push_back(d.get<int64_t>());
        if (shp != specs[i].shape) throw Error(B2_ERR_IO, "tensor " + specs[i].name + " has an unexpected shape");
        const size_t o = t.at("byte_offset").get<size_t>(), len = t.at("byte_length").get<size_t>();
        const size_t n = numel(shp);
        if (o + len > file_bytes || len != n * 4) throw Error(B2_ERR_IO, "tensor " + specs[i].name + " byte range is inconsistent");
        const float* src = reinterpret_cast<const float*>(blob.data() + o);
        char* dst = staging + off[i];
        for (size_t k = 0; k < n; ++k) checksum += static_cast<double>(src[k]);
        if (e.dt == B2_F32) {
            std::memcpy(dst, src, n * 4);
        } else if (e.dt == B2_F16) {
            __half* h = reinterpret_cast<__half*>(dst);
            for (size_t k = 0; k < n; ++k) h[k] = __float2half_rn(src[k]);
        } else {
            __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(dst);
            for (size_t k = 0; k < n; ++k) h[k] = __float2bfloat16_rn(src[k]);
        }
    }
    const double want = man.value("checksum_sum", 0.0);
    if (std::fabs(checksum - want) / std::max(1.0, std::fabs(want)) > 1e-6)
        throw Error(B2_ERR_IO, "weight checksum_sum differs from the manifest (corrupt export?)");
    cuda_ok(cudaMemcpy(e.weights, staging, total, cudaMemcpyHostToDevice), "upload weights");
    e.bind_tensors(off);
}

void synth_weights(Engine& e, uint64_t seed, float stdev) {
    const auto specs = tensor_specs(e.shape);
    size_t total = 0;
    const auto off = e.layout(specs, &total);
    cuda_ok(cudaMalloc(&e.weights, total), "malloc weights");
    cuda_ok(cudaMemsetAsync(e.weights, 0, total, e.stream), "memset weights");  // wte's zero rows past the vocabulary
    for (size_t i = 0; i < specs.size(); ++i) {
        void* dst = static_cast<char*>(e.weights) + off[i];
        const size_t n = numel(specs[i].shape);
        const uint64_t key = seed * 0x100000001b3ull + i;
        const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 148 * 32));
        if (e.dt == B2_F32) {
            if (specs[i].init == 0) synth_normal_kernel<float><<<grid, 256, 0, e.stream>>>(static_cast<float*>(dst), n, key, stdev);
            else fill_kernel<float><<<grid, 256, 0, e.stream>>>(static_cast<float*>(dst), n, specs[i].init == 1 ? 1.0f : 0.0f);
        } else if (e.dt == B2_F16) {
            if (specs[i].init == 0) synth_normal_kernel<__half><<<grid, 256, 0, e.stream>>>(static_cast<__half*>(dst), n, key, stdev);
            else fill_kernel<__half><<<grid, 256, 0, e.stream>>>(static_cast<__half*>(dst), n, specs[i].init == 1 ? 1.0f : 0.0f);
        } else {
            if (specs[i].init == 0)
                synth_normal_kernel<__nv_bfloat16><<<grid, 256, 0, e.stream>>>(static_cast<__nv_bfloat16*>(dst), n, key, stdev);
            else
                fill_kernel<__nv_bfloat16><<<grid, 256, 0, e.stream>>>(static_cast<__nv_bfloat16*>(dst), n,
                                                                        specs[i].init == 1 ? 1.0f : 0.0f);
        }
        cuda_ok(cudaGetLastError(), "synthetic weights");
    }
    cuda_ok(cudaStreamSynchronize(e.stream), "synthetic weights");
    e.bind_tensors(off);
}

// Bench hook: the KV pool of a synthetic engine holds N(0, 1) values instead
// of zeros, so cached contexts look like real keys and values.
void synth_pool(Engine& e, uint64_t seed) {
    const size_t n = e.layer_bytes() / e.es * e.shape.n_layer;
    const uint64_t key = seed * 0x9e3779b97f4a7c15ull + 0x6b7650ull;
    const int grid = 148 * 32;
    if (e.dt == B2_F32) synth_normal_kernel<float><<<grid, 256, 0, e.stream>>>(static_cast<float*>(e.pool), n, key, 1.0f);
    else if (e.dt == B2_F16) synth_normal_kernel<__half><<<grid, 256, 0, e.stream>>>(static_cast<__half*>(e.pool), n, key, 1.0f);
    else synth_normal_kernel<__nv_bfloat16><<<grid, 256, 0, e.stream>>>(static_cast<__nv_bfloat16*>(e.pool), n, key, 1.0f);
    cuda_ok(cudaGetLastError(), "synthetic KV pool");
    cuda_ok(cudaStreamSynchronize(e.stream), "synthetic KV pool");
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return B2_OK;
    } catch (const Error& err) {
        g_err = err.what();
        return err.code;
    } catch (const std::exception& ex) {
        g_err = ex.what();
        return B2_ERR_IO;
    }
}

}  // namespace eng
}  // namespace b2

struct b2_engine : b2::eng::Engine {};
struct b2_block_pool : b2::BlockPool {
    explicit b2_block_pool(int n) : b2::BlockPool(n) {}
};

using b2::eng::Error;
using b2::eng::guarded;

extern "C" {

const char* b2_engine_last_error(void) { return b2::eng::g_err.c_str(); }

int b2_engine_create(const char* weights_dir, const B2EngineConfig* cfg, b2_engine** out) {
    if (!weights_dir || !cfg || !out) {
        b2::eng::g_err = "weights_dir, cfg and out are required";
        return B2_ERR_NULL;
    }
    *out = nullptr;
    auto e = std::make_unique<b2_engine>();
    const int rc = guarded([&] {
        e->cfg = *cfg;
        e->shape = b2::eng::read_config(weights_dir);
        e->check_shape();
        e->setup_device();
        b2::eng::load_weights(*e, weights_dir);
        e->build_tp_weights();
        e->setup_buffers();
    });
    if (rc == B2_OK) *out = e.release();
    return rc;
}

int b2_engine_create_synthetic(const B2ModelShape* shape, uint64_t seed, float stdev, const B2EngineConfig* cfg,
                               b2_engine** out) {
    if (!shape || !cfg || !out) {
        b2::eng::g_err = "shape, cfg and out are required";
        return B2_ERR_NULL;
    }
    *out = nullptr;
    auto e = std::make_unique<b2_engine>();
    const int rc = guarded([&] {
        e->cfg = *cfg;
        e->shape = *shape;
        e->check_shape();
        e->setup_device();
        b2::eng::synth_weights(*e, seed, stdev);
        e->build_tp_weights();
        e->setup_buffers();
        b2::eng::synth_pool(*e, seed);
    });
    if (rc == B2_OK) *out = e.release();
    return rc;
}

void b2_engine_destroy(b2_engine* eng) { delete eng; }

int32_t b2_engine_add_sequence(b2_engine* eng, const int32_t* prompt, int32_t prompt_len) {
    if (!eng || (prompt_len > 0 && !prompt) || prompt_len < 0) {
        b2::eng::g_err = "bad arguments";
        return B2_ERR_NULL;
    }
    int32_t id = -1;
    const int rc = guarded([&] {
        for (int i = 0; i < prompt_len; ++i)
            if (prompt[i] < 0 || prompt[i] >= eng->shape.vocab_size) throw Error(B2_ERR_SHAPE, "prompt token outside the vocabulary");
        const int blk = eng->blocks->allocate();
        if (blk < 0) return;  // pool exhausted: -1, like the reference
        b2::eng::Seq q;
        q.table.ids.push_back(blk);
        q.prompt.assign(prompt, prompt + prompt_len);
        id = eng->register_seq(std::move(q));
    });
    return rc == B2_OK ? id : rc;
}

int32_t b2_engine_add_sequence_cached(b2_engine* eng, int32_t ctx_len, int32_t last_token) {
    if (!eng) return B2_ERR_NULL;
    int32_t id = -1;
    const int rc = guarded([&] {
        if (ctx_len < 0 || ctx_len >= eng->cfg.max_seq_len) throw Error(B2_ERR_SHAPE, "ctx_len must be in [0, max_seq_len)");
        if (last_token < 0 || last_token >= eng->shape.vocab_size) throw Error(B2_ERR_SHAPE, "last_token outside the vocabulary");
        const int nblk = ctx_len / B2_BLOCK_TOKENS + 1;  // covers positions [0, ctx_len]
        if (nblk > eng->blocks->num_free()) return;
        b2::eng::Seq q;
        for (int i = 0; i < nblk; ++i) q.table.ids.push_back(eng->blocks->allocate());
        q.seq_len = ctx_len;
        q.last_token = last_token;
        id = eng->register_seq(std::move(q));
    });
    return rc == B2_OK ? id : rc;
}

int b2_engine_decode_step(b2_engine* eng, const int32_t* seq_ids, int32_t batch, int32_t* out_next_tokens) {
    if (!eng || !seq_ids || !out_next_tokens) {
        b2::eng::g_err = "engine, seq_ids and out_next_tokens are required";
        return B2_ERR_NULL;
    }
    return guarded([&] {
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        eng->decode_step(seq_ids, batch, out_next_tokens);
    });
}

int b2_engine_prefill(b2_engine* eng, const int32_t* seq_ids, int32_t n, int32_t* out_next_tokens) {
    if (!eng || !seq_ids || !out_next_tokens) {
        b2::eng::g_err = "engine, seq_ids and out_next_tokens are required";
        return B2_ERR_NULL;
    }
    return guarded([&] {
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        eng->prefill(seq_ids, n, out_next_tokens);
    });
}

int b2_engine_free_sequence(b2_engine* eng, int32_t seq_id) {
    if (!eng) return B2_ERR_NULL;
    return guarded([&] { eng->release_seq(seq_id); });
}

int64_t b2_engine_free_blocks(const b2_engine* eng) { return eng ? eng->blocks->num_free() : 0; }

int b2_engine_set_use_cuda_graphs(b2_engine* eng, int32_t enabled) {
    if (!eng) return B2_ERR_NULL;
    eng->use_graphs = enabled != 0;
    return B2_OK;
}

int b2_engine_set_prefill_tensor_cores(b2_engine* eng, int32_t enabled) {
    if (!eng) return B2_ERR_NULL;
    eng->prefill_tc = enabled != 0;
    return B2_OK;
}

int b2_engine_last_step_outputs(const b2_engine* eng, int32_t rows, void* hidden_out, void* logits_out) {
    if (!eng) return B2_ERR_NULL;
    return guarded([&] {
        if (rows < 0 || rows > eng->cfg.max_batch) throw Error(B2_ERR_SHAPE, "rows must be in [0, max_batch]");
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        b2::eng::cuda_ok(cudaStreamSynchronize(eng->stream), "last step outputs");
        const size_t es = static_cast<size_t>(eng->es);
        const size_t D = static_cast<size_t>(eng->shape.d_model), V = static_cast<size_t>(eng->shape.vocab_size);
        if (hidden_out && rows > 0)
            b2::eng::cuda_ok(cudaMemcpy(hidden_out, eng->d_x, static_cast<size_t>(rows) * D * es, cudaMemcpyDeviceToHost),
                             "copy final LayerNorm rows");
        if (logits_out && rows > 0)
            b2::eng::cuda_ok(cudaMemcpy2D(logits_out, V * es, eng->d_logits, static_cast<size_t>(eng->vocab_padded()) * es,
                                          V * es, static_cast<size_t>(rows), cudaMemcpyDeviceToHost),
                             "copy logits");
    });
}

int b2_engine_set_gemm_mode(b2_engine* eng, int32_t mode) {
    if (!eng) return B2_ERR_NULL;
    return guarded([&] {
        if (mode < 0 || mode > 3) throw Error(B2_ERR_SHAPE, "gemm mode must be 0..3");
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        b2::eng::cuda_ok(cudaStreamSynchronize(eng->stream), "gemm mode switch");
        for (auto& g : eng->graphs) cudaGraphExecDestroy(g.second);
        eng->graphs.clear();
        eng->gemm_mode = eng->dt == B2_F32 ? 0 : mode;
    });
}

int b2_engine_set_lm_head_fused(b2_engine* eng, int32_t enabled) {
    if (!eng) return B2_ERR_NULL;
    return guarded([&] {
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        b2::eng::cuda_ok(cudaStreamSynchronize(eng->stream), "lm_head switch");
        for (auto& g : eng->graphs) cudaGraphExecDestroy(g.second);  // captured with the other lm_head
        eng->graphs.clear();
        const bool on = enabled != 0 && eng->dt != B2_F32;
        if (on && eng->lm_ws == nullptr) {
            eng->lm_ws_bytes = b2_lm_head_argmax_workspace_bytes(eng->cfg.max_batch);
            b2::eng::cuda_ok(cudaMalloc(&eng->lm_ws, eng->lm_ws_bytes), "malloc lm_head workspace");
            b2::eng::cuda_ok(cudaMemsetAsync(eng->lm_ws, 0, eng->lm_ws_bytes, eng->stream), "zero lm_head workspace");
        }
        eng->lm_fused = on;
    });
}

int b2_engine_set_linear_tensor_cores(b2_engine* eng, int32_t enabled) {
    if (!eng) return B2_ERR_NULL;
    return guarded([&] {
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        b2::eng::cuda_ok(cudaStreamSynchronize(eng->stream), "linear switch");
        for (auto& g : eng->graphs) cudaGraphExecDestroy(g.second);  // captured with the other GEMMs
        eng->graphs.clear();
        eng->linear_tc = enabled != 0;
    });
}

int b2_engine_shape(const b2_engine* eng, B2ModelShape* out) {
    if (!eng || !out) return B2_ERR_NULL;
    *out = eng->shape;
    return B2_OK;
}

int b2_engine_stream(const b2_engine* eng, b2_stream_t* out) {
    if (!eng || !out) return B2_ERR_NULL;
    *out = eng->stream;
    return B2_OK;
}

int b2_engine_tp_handle(const b2_engine* eng, void* out) {
    if (!eng || !out) return B2_ERR_NULL;
    static_assert(2 * sizeof(cudaIpcMemHandle_t) == B2_TP_HANDLE_BYTES, "IPC handle size");
    return guarded([&] {
        if (eng->tp <= 1) throw Error(B2_ERR_SHAPE, "not a head-sharded engine");
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        cudaIpcMemHandle_t h[2];
        b2::eng::cuda_ok(cudaIpcGetMemHandle(&h[0], eng->d_gath), "cudaIpcGetMemHandle (gathered buffer)");
        b2::eng::cuda_ok(cudaIpcGetMemHandle(&h[1], eng->d_flags), "cudaIpcGetMemHandle (flags)");
        std::memcpy(out, h, sizeof(h));
    });
}

int b2_engine_tp_connect(b2_engine* eng, const void* handles) {
    if (!eng || !handles) return B2_ERR_NULL;
    return guarded([&] {
        if (eng->tp <= 1 || eng->tp_nccl) throw Error(B2_ERR_SHAPE, "not a head-sharded engine with tp_allgather = 0");
        if (eng->tp_connected) throw Error(B2_ERR_SHAPE, "already connected");
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        std::vector<void*> outs(2 * static_cast<size_t>(eng->tp)), flags(static_cast<size_t>(eng->tp));
        const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
        for (int p = 0; p < eng->tp; ++p) {
            if (p == eng->tp_rank) {
                outs[p] = eng->d_gath;
                outs[eng->tp + p] = static_cast<char*>(eng->d_gath) + eng->gath_half_bytes();
                flags[p] = eng->d_flags;
                continue;
            }
            void* o = nullptr;
            void* f = nullptr;
            b2::eng::cuda_ok(cudaIpcOpenMemHandle(&o, h[2 * p], cudaIpcMemLazyEnablePeerAccess),
                             "cudaIpcOpenMemHandle (peer gathered buffer)");
            eng->peer_mapped.push_back(o);
            b2::eng::cuda_ok(cudaIpcOpenMemHandle(&f, h[2 * p + 1], cudaIpcMemLazyEnablePeerAccess),
                             "cudaIpcOpenMemHandle (peer flags)");
            eng->peer_mapped.push_back(f);
            outs[p] = o;
            outs[eng->tp + p] = static_cast<char*>(o) + eng->gath_half_bytes();
            flags[p] = f;
        }
        b2::eng::cuda_ok(cudaMemcpy(eng->d_peer_outs, outs.data(), outs.size() * sizeof(void*), cudaMemcpyHostToDevice),
                         "upload peer table");
        b2::eng::cuda_ok(cudaMemcpy(eng->d_peer_flags, flags.data(), flags.size() * sizeof(void*),
                                    cudaMemcpyHostToDevice),
                         "upload peer table");
        eng->tp_connected = true;
    });
}

int b2_engine_tp_nccl_id(void* out) {
    if (!out) return B2_ERR_NULL;
    static_assert(sizeof(ncclUniqueId) == B2_TP_NCCL_ID_BYTES, "NCCL id size");
    return guarded([&] {
        ncclUniqueId id;
        b2::eng::nccl_ok(ncclGetUniqueId(&id), "ncclGetUniqueId");
        std::memcpy(out, &id, sizeof(id));
    });
}

int b2_engine_tp_connect_nccl(b2_engine* eng, const void* id) {
    if (!eng || !id) return B2_ERR_NULL;
    return guarded([&] {
        if (!eng->tp_nccl) throw Error(B2_ERR_SHAPE, "not a head-sharded engine with tp_allgather = 1");
        if (eng->tp_connected) throw Error(B2_ERR_SHAPE, "already connected");
        b2::eng::cuda_ok(cudaSetDevice(eng->device), "cudaSetDevice");
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof(uid));
        b2::eng::nccl_ok(ncclCommInitRank(&eng->nccl, eng->tp, uid, eng->tp_rank), "ncclCommInitRank");
        eng->tp_connected = true;
    });
}

b2_block_pool* b2_block_pool_create(int32_t num_blocks) { return num_blocks >= 0 ? new b2_block_pool(num_blocks) : nullptr; }
void b2_block_pool_destroy(b2_block_pool* pool) { delete pool; }
int32_t b2_block_pool_allocate(b2_block_pool* pool) { return pool ? pool->allocate() : -1; }
int32_t b2_block_pool_free(b2_block_pool* pool, int32_t block_id) {
    try {
        pool->free(block_id);
        return 0;
    } catch (const std::out_of_range&) {
        return 1;
    } catch (const std::logic_error&) {
        return 2;
    }
}
int32_t b2_block_pool_num_free(const b2_block_pool* pool) { return pool ? pool->num_free() : 0; }

}  // extern "C"
