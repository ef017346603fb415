// b2_batched_generator.hpp -- a TokenGenerator over this library's Engine that
// prefills newly admitted sequences in one batched call.
//
// The reference's ContinuousBatchScheduler (cpp-engine/src/scheduler.h) drives
// any TokenGenerator (cpp-engine/src/token_generator.h:15-56): forward() gets
// every newly admitted sequence with its whole prompt (prefill_step) and, in a
// separate call, every running sequence with its last token (decode_step).
// The reference's GpuEngineGenerator (gpu_engine_generator.cpp:16-58) walks
// each new prompt token by token at batch 1 through Engine::decode_step.  This
// generator keeps the same interface and the same kv_slot -> engine sequence
// bookkeeping, but registers all new sequences and runs their prompts through
// one b2_engine_prefill (tensor-core prefill attention for 16-bit models),
// splitting only where a call would exceed the engine's prompt-token budget.
//
// Header-only.  Build with the reference's cpp-engine/src on the include path
// (for token_generator.h) and link libb2engine.so.  tokenize() is a stand-in
// (the reference has no C++ GPT-2 tokenizer either): by default one id per
// byte of the text; pass Config::tokenizer for anything else.
#pragma once

#include <algorithm>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "b2_engine_api.hpp"
#include "token_generator.h"

namespace b2 {

class BatchedPrefillGenerator : public TokenGenerator {
public:
    struct Config {
        std::string weights_dir;
        int max_batch_size = 8;
        int max_seq_len = 1024;
        int kv_block_budget = 512;
        int max_prefill_tokens = 0;  // prompt tokens per prefill call; 0 = the engine's default (2048)
        int32_t eos_token_id = -1;   // -1: never matches a generated token
        std::function<std::vector<int32_t>(const std::string&)> tokenizer;  // empty: one id per byte
    };

    explicit BatchedPrefillGenerator(Config config) : config_(std::move(config)) {
        b2::EngineConfig cfg;
        cfg.max_batch = config_.max_batch_size;
        cfg.max_seq_len = config_.max_seq_len;
        cfg.kv_block_budget = config_.kv_block_budget;
        cfg.max_prefill_tokens = config_.max_prefill_tokens;
        if (!engine_.init(config_.weights_dir, cfg))
            throw std::runtime_error("BatchedPrefillGenerator: engine init failed: " + b2::Engine::last_error());
        prefill_budget_ = config_.max_prefill_tokens > 0 ? config_.max_prefill_tokens : 2048;
    }

    BatchOutput forward(const BatchInput& input) override {
        BatchOutput out;
        out.next_tokens.assign(input.entries.size(), 0);
        std::vector<int> fresh_ids, fresh_idx, step_ids, step_idx;
        for (size_t i = 0; i < input.entries.size(); ++i) {
            const Entry& e = input.entries[i];
            auto it = slot_to_seq_.find(e.kv_slot);
            if (it == slot_to_seq_.end()) {
                if (static_cast<int>(e.tokens.size()) > prefill_budget_)
                    throw std::runtime_error("BatchedPrefillGenerator: prompt longer than max_prefill_tokens");
                const int id = engine_.add_sequence(e.tokens.data(), static_cast<int>(e.tokens.size()));
                if (id < 0) throw std::runtime_error("BatchedPrefillGenerator: KV block pool exhausted");
                slot_to_seq_[e.kv_slot] = id;
                fresh_ids.push_back(id);
                fresh_idx.push_back(static_cast<int>(i));
                fresh_len_.push_back(static_cast<int>(e.tokens.size()));
            } else {
                step_ids.push_back(it->second);
                step_idx.push_back(static_cast<int>(i));
            }
        }
        // New prompts: as few prefill calls as the prompt-token budget allows.
        size_t a = 0;
        std::vector<int> next;
        while (a < fresh_ids.size()) {
            size_t b = a;
            int tokens = 0;
            while (b < fresh_ids.size() && (b == a || tokens + fresh_len_[b] <= prefill_budget_)) tokens += fresh_len_[b++];
            next.assign(b - a, 0);
            engine_.prefill(fresh_ids.data() + a, static_cast<int>(b - a), next.data());
            for (size_t k = a; k < b; ++k) out.next_tokens[static_cast<size_t>(fresh_idx[k])] = next[k - a];
            a = b;
        }
        fresh_len_.clear();
        if (!step_ids.empty()) {
            next.assign(step_ids.size(), 0);
            engine_.decode_step(step_ids.data(), static_cast<int>(step_ids.size()), next.data());
            for (size_t k = 0; k < step_ids.size(); ++k) out.next_tokens[static_cast<size_t>(step_idx[k])] = next[k];
        }
        return out;
    }

    std::vector<int32_t> tokenize(const std::string& text) override {
        if (config_.tokenizer) return config_.tokenizer(text);
        std::vector<int32_t> ids;
        ids.reserve(text.size());
        for (unsigned char c : text) ids.push_back(static_cast<int32_t>(c));
        return ids;
    }

    std::string detokenize(int32_t token_id) override { return "<" + std::to_string(token_id) + ">"; }

    int32_t eos_token_id() const override { return config_.eos_token_id; }

    void reset_sequence(int kv_slot) override {
        auto it = slot_to_seq_.find(kv_slot);
        if (it == slot_to_seq_.end()) return;
        engine_.free_sequence(it->second);
        slot_to_seq_.erase(it);
    }

private:
    Config config_;
    b2::Engine engine_;
    int prefill_budget_ = 2048;
    std::unordered_map<int, int> slot_to_seq_;
    std::vector<int> fresh_len_;
};

}  // namespace b2
