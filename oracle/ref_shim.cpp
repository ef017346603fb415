// ref_shim.cpp -- extern "C" entry points over the reference's own CPU path.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference sources where they lie (gpu-engine/src/reference/cpu_model.cpp,
// gpu-engine/src/reference/weights_loader.cpp, gpu-engine/src/model.cpp,
// gpu-engine/src/kv_cache_pool.cpp) into oracle/_ref/libref_cpu.so.  Nothing
// here restates reference code: it only calls it, so tests can pin the oracle
// (b2_oracle.c) and the engine against the reference's CPUModel, and the bench
// can time the reference's CPU forward path.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "engine/kv_cache.h"
#include "engine/model.h"
#include "reference/cpu_model.h"
#include "reference/weights_loader.h"

namespace {
thread_local std::string g_err;
}

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// CPUModel::greedy_generate (cpu_model.cpp:198-216) for one prompt.
// Returns the number of tokens written to out (<= n_new), or -1 on error.
int ref_greedy_generate(const char* model_dir, const int32_t* prompt, int prompt_len, int n_new,
                        int32_t* out) {
    try {
        GPT2Config cfg = GPT2Config::load_from_json(std::string(model_dir) + "/config.json");
        WeightsLoader weights(model_dir);
        CPUModel model(cfg, weights);
        std::vector<int32_t> p(prompt, prompt + prompt_len);
        std::vector<int32_t> gen = model.greedy_generate(p, n_new);
        for (size_t i = 0; i < gen.size(); ++i) out[i] = gen[i];
        return static_cast<int>(gen.size());
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// Many prompts, one CPUModel per host thread sharing one WeightsLoader (the
// multi-threaded CPU baseline).  prompts is a flat array; prompt i starts at
// offsets[i] and has lens[i] tokens.  out is [n_prompts, n_new]; out_counts[i]
// receives the generated count.  Returns elapsed seconds, or -1 on error.
double ref_greedy_generate_many(const char* model_dir, const int32_t* prompts, const int* offsets,
                                const int* lens, int n_prompts, int n_new, int n_threads,
                                int32_t* out, int* out_counts) {
    try {
        GPT2Config cfg = GPT2Config::load_from_json(std::string(model_dir) + "/config.json");
        WeightsLoader weights(model_dir);
        if (n_threads < 1) n_threads = 1;
        std::vector<int> next(1, 0);
        std::vector<std::string> errors(n_threads);
        auto worker = [&](int tid) {
            try {
                CPUModel model(cfg, weights);
                for (int i = tid; i < n_prompts; i += n_threads) {
                    std::vector<int32_t> p(prompts + offsets[i], prompts + offsets[i] + lens[i]);
                    std::vector<int32_t> gen = model.greedy_generate(p, n_new);
                    out_counts[i] = static_cast<int>(gen.size());
                    for (size_t j = 0; j < gen.size(); ++j) out[static_cast<size_t>(i) * n_new + j] = gen[j];
                }
            } catch (const std::exception& e) {
                errors[tid] = e.what();
            }
        };
        auto t0 = std::chrono::steady_clock::now();
        std::vector<std::thread> threads;
        for (int t = 0; t < n_threads; ++t) threads.emplace_back(worker, t);
        for (auto& th : threads) th.join();
        auto t1 = std::chrono::steady_clock::now();
        for (auto& e : errors)
            if (!e.empty()) {
                g_err = e;
                return -1.0;
            }
        return std::chrono::duration<double>(t1 - t0).count();
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1.0;
    }
}

// The reference's block_bytes (kv_cache.h:12-14).
size_t ref_block_bytes(int n_layer, int n_heads, int head_dim) {
    return block_bytes(n_layer, n_heads, head_dim);
}

int ref_block_tokens() { return BLOCK_TOKENS; }

// The reference's BlockPool (kv_cache_pool.cpp), driven through opaque handles
// so the allocator tests exercise the reference's own implementation.
void* ref_pool_create(int n) { return new BlockPool(n); }
void ref_pool_destroy(void* p) { delete static_cast<BlockPool*>(p); }
int ref_pool_allocate(void* p) { return static_cast<BlockPool*>(p)->allocate(); }
int ref_pool_num_free(void* p) { return static_cast<BlockPool*>(p)->num_free(); }
// Returns 0 on success, 1 for std::out_of_range, 2 for std::logic_error.
int ref_pool_free(void* p, int id) {
    try {
        static_cast<BlockPool*>(p)->free(id);
        return 0;
    } catch (const std::out_of_range&) {
        return 1;
    } catch (const std::logic_error&) {
        return 2;
    }
}

}  // extern "C"
