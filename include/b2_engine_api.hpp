// b2_engine_api.hpp -- the reference's Engine class over the C-ABI of
// libb2engine.so (include/b2_engine.h).
//
// Same declarations and behaviour as gpu-engine/include/engine/engine_api.h:9-48,
// so a caller such as GpuEngineGenerator (cpp-engine/src/gpu_engine_generator.h:26-49)
// switches by including this header instead of "engine/engine_api.h" and
// linking libb2engine.so:
//   - EngineConfig keeps max_batch / max_seq_len / kv_block_budget with the
//     same defaults; dtype, use_cuda_graphs and device are added after them;
//   - init() returns false on any failure; add_sequence() returns -1 when the
//     KV pool is exhausted; decode_step() throws std::runtime_error on any
//     failure (the reference throws from its CUDA / cuBLAS checks and from
//     ensure_capacity, engine.cu:40-44, 227-233);
//   - free_blocks() and set_use_cuda_graphs() as in the reference.
// CUDA-free, like the reference header: nothing here includes a CUDA header.
#pragma once

#include <cstddef>
#include <stdexcept>
#include <cstdlib>
#include <string>

#include "b2_engine.h"

namespace b2 {

// The storage dtype an EngineConfig starts with: B2_F16 (the reference engine
// is fp16), or what the B2_ENGINE_DTYPE environment variable names ("f32",
// "f16", "bf16") -- so a caller that builds its config without naming a dtype
// (the reference's GpuEngineGenerator) can still run an f32 or bf16 engine.
inline int default_engine_dtype() {
    const char* v = std::getenv("B2_ENGINE_DTYPE");
    if (v == nullptr) return B2_F16;
    const std::string s(v);
    if (s == "f32") return B2_F32;
    if (s == "bf16") return B2_BF16;
    return B2_F16;
}

struct EngineConfig {
    int max_batch = 8;
    int max_seq_len = 1024;
    int kv_block_budget = 4096;
    int dtype = default_engine_dtype();
    bool use_cuda_graphs = true;
    int device = -1;  // -1: the device current on the calling thread
    int tp_rank = 0;  // head-sharded engines (include/b2_engine.h)
    int tp_size = 1;
    int max_prefill_tokens = 0;  // 0: 2048
    int tp_allgather = 0;        // head-sharded: 0 fused peer stores, 1 ncclAllGather
};

class Engine {
public:
    Engine() = default;
    ~Engine() { b2_engine_destroy(eng_); }
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    bool init(const std::string& weights_dir, const EngineConfig& cfg) {
        b2_engine_destroy(eng_);
        eng_ = nullptr;
        const B2EngineConfig c{cfg.max_batch, cfg.max_seq_len, cfg.kv_block_budget, cfg.dtype,
                               cfg.use_cuda_graphs ? 1 : 0, cfg.device, cfg.tp_rank, cfg.tp_size,
                               cfg.max_prefill_tokens, cfg.tp_allgather};
        return b2_engine_create(weights_dir.c_str(), &c, &eng_) == B2_OK;
    }

    int add_sequence(const int* prompt_tokens, int prompt_len) {
        const int id = b2_engine_add_sequence(handle(), prompt_tokens, prompt_len);
        if (id < -1) throw std::runtime_error(b2_engine_last_error());
        return id;
    }

    void decode_step(const int* seq_ids, int batch, int* out_next_tokens) {
        if (b2_engine_decode_step(handle(), seq_ids, batch, out_next_tokens) != B2_OK)
            throw std::runtime_error(b2_engine_last_error());
    }

    // Batched prefill of the listed sequences' prompts (no reference counterpart).
    void prefill(const int* seq_ids, int n, int* out_next_tokens) {
        if (b2_engine_prefill(handle(), seq_ids, n, out_next_tokens) != B2_OK)
            throw std::runtime_error(b2_engine_last_error());
    }

    void free_sequence(int seq_id) {
        if (b2_engine_free_sequence(handle(), seq_id) != B2_OK) throw std::runtime_error(b2_engine_last_error());
    }

    size_t free_blocks() const { return static_cast<size_t>(b2_engine_free_blocks(eng_)); }

    void set_use_cuda_graphs(bool enabled) { b2_engine_set_use_cuda_graphs(handle(), enabled ? 1 : 0); }
    // Prefill attention on the tensor cores (default) or as decode-attention rows.
    void set_prefill_tensor_cores(bool enabled) { b2_engine_set_prefill_tensor_cores(handle(), enabled ? 1 : 0); }

    // Text of the failure behind the last false / exception (no reference counterpart).
    static std::string last_error() { return b2_engine_last_error(); }

private:
    b2_engine* handle() const {
        if (!eng_) throw std::runtime_error("Engine used before a successful init()");
        return eng_;
    }
    b2_engine* eng_ = nullptr;
};

}  // namespace b2

#ifndef B2_NO_GLOBAL_ENGINE_NAMES
// The reference declares these at global scope.
using b2::Engine;
using b2::EngineConfig;
#endif
