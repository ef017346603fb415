// ref_scheduler_harness.cpp -- drives the reference's own ContinuousBatchScheduler
// (cpp-engine/src/scheduler.cpp, compiled unchanged from the reference's
// sources) on this library's engine, through either the reference's
// GpuEngineGenerator (cpp-engine/src/gpu_engine_generator.cpp, unchanged; its
// "engine/engine_api.h" resolves to include/compat/engine/engine_api.h) or
// this library's BatchedPrefillGenerator (include/b2_batched_generator.hpp).
//
// TEST AND BENCH INFRASTRUCTURE.  oracle/Makefile builds it into
// oracle/_ref/ref_scheduler_harness; tests/test_ref_scheduler_gpu.py and
// bench.py --workload serve-medium run it.
//
//   ref_scheduler_harness <weights_dir> <reference|batched> key=value ...
//     requests=N  max_batch=B  vocab=V  seed=S  static=0|1
//     prompt_lo=a prompt_hi=b  out_lo=c out_hi=d   (uniform, inclusive)
//     rate=R      Poisson arrivals at R requests/s (0: all submitted at once)
//     max_seq_len=L kv_block_budget=K max_prefill_tokens=P  per_request=0|1
//
// Prompts are token-count controlled: request i's prompt is a list of ids
// drawn from std::mt19937_64(seed) -- the harness's tokenize() override returns
// it for the text "req:<i>" (the reference's tokenize ignores the text and
// makes 4-11 ids, gpu_engine_generator.cpp:81-88).  Prints one JSON line per
// request when per_request=1 (prompt, generated ids, TTFT, finish reason), then
// one summary line (output tok/s over the makespan, TTFT p50/p99).
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "b2_batched_generator.hpp"
#include "gpu_engine_generator.h"
#include "scheduler.h"

using Clock = std::chrono::steady_clock;

namespace {

std::map<std::string, std::string> g_opt;

long opt(const std::string& k, long dflt) {
    auto it = g_opt.find(k);
    return it == g_opt.end() ? dflt : std::atol(it->second.c_str());
}
double optf(const std::string& k, double dflt) {
    auto it = g_opt.find(k);
    return it == g_opt.end() ? dflt : std::atof(it->second.c_str());
}

std::vector<std::vector<int32_t>> g_prompts;

std::vector<int32_t> prompt_for(const std::string& text) {
    const size_t i = static_cast<size_t>(std::atol(text.c_str() + 4));  // "req:<i>"
    return g_prompts.at(i);
}

// The reference generator with the prompt lookup above as its tokenizer.
class ControlledGpuEngineGenerator : public GpuEngineGenerator {
public:
    using GpuEngineGenerator::GpuEngineGenerator;
    std::vector<int32_t> tokenize(const std::string& text) override { return prompt_for(text); }
};

struct Req {
    std::vector<int32_t> tokens;
    Clock::time_point submit, first, done;
    int finish = 0;
};

double pct(std::vector<double> v, double p) {
    if (v.empty()) return 0.0;
    std::sort(v.begin(), v.end());
    const size_t k = std::min(v.size() - 1, static_cast<size_t>(p * static_cast<double>(v.size() - 1) + 0.5));
    return v[k];
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: %s <weights_dir> <reference|batched> key=value ...\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1], kind = argv[2];
    for (int i = 3; i < argc; ++i) {
        const std::string a = argv[i];
        const size_t eq = a.find('=');
        if (eq != std::string::npos) g_opt[a.substr(0, eq)] = a.substr(eq + 1);
    }
    const int n = static_cast<int>(opt("requests", 8));
    const int max_batch = static_cast<int>(opt("max_batch", 4));
    const int vocab = static_cast<int>(opt("vocab", 50257));
    const int max_seq = static_cast<int>(opt("max_seq_len", 1024));
    const double rate = optf("rate", 0.0);
    std::mt19937_64 rng(static_cast<uint64_t>(opt("seed", 1)));
    std::uniform_int_distribution<int> plen(static_cast<int>(opt("prompt_lo", 4)), static_cast<int>(opt("prompt_hi", 16)));
    std::uniform_int_distribution<int> olen(static_cast<int>(opt("out_lo", 4)), static_cast<int>(opt("out_hi", 16)));
    std::uniform_int_distribution<int> tok(0, vocab - 1);
    std::vector<int> out_len(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
        std::vector<int32_t> p(static_cast<size_t>(plen(rng)));
        for (auto& t : p) t = tok(rng);
        g_prompts.push_back(std::move(p));
        out_len[static_cast<size_t>(i)] = olen(rng);
    }
    std::vector<double> offsets(static_cast<size_t>(n), 0.0);
    if (rate > 0) {
        std::exponential_distribution<double> gap(rate);
        double t = 0.0;
        for (auto& o : offsets) o = (t += gap(rng));
    }

    std::unique_ptr<TokenGenerator> gen;
    try {
        if (kind == "reference") {
            GpuEngineGenerator::Config g;
            g.weights_dir = dir;
            g.max_batch_size = max_batch;
            g.max_seq_len = max_seq;
            g.kv_block_budget = static_cast<int>(opt("kv_block_budget", 512));
            gen = std::make_unique<ControlledGpuEngineGenerator>(g);
        } else {
            b2::BatchedPrefillGenerator::Config g;
            g.weights_dir = dir;
            g.max_batch_size = max_batch;
            g.max_seq_len = max_seq;
            g.kv_block_budget = static_cast<int>(opt("kv_block_budget", 512));
            g.max_prefill_tokens = static_cast<int>(opt("max_prefill_tokens", 0));
            g.tokenizer = prompt_for;
            gen = std::make_unique<b2::BatchedPrefillGenerator>(g);
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "generator set-up failed: %s\n", e.what());
        return 1;
    }

    ContinuousBatchScheduler::Config sc;
    sc.max_batch_size = max_batch;
    sc.max_sequence_length = max_seq;
    sc.max_queue_depth = n;
    // The scheduler's own slot allocator (cpp-engine/src/kv_cache.cpp) holds a
    // host buffer the GPU path never reads: keep it small.
    sc.num_layers = 1;
    sc.num_kv_heads = 1;
    sc.head_dim = 8;
    sc.static_batching = opt("static", 0) != 0;
    ContinuousBatchScheduler sched(sc, std::move(gen));

    std::mutex mu;
    std::vector<Req> reqs(static_cast<size_t>(n));
    int completed = 0;
    sched.set_token_callback([&](const std::string& rid, const std::string&, int32_t token, bool finished, int why) {
        const auto now = Clock::now();
        std::lock_guard<std::mutex> lock(mu);
        Req& r = reqs.at(static_cast<size_t>(std::atol(rid.c_str() + 4)));
        if (r.tokens.empty()) r.first = now;
        r.tokens.push_back(token);
        if (finished) {
            r.done = now;
            r.finish = why;
            ++completed;
        }
    });
    std::thread loop([&] {
        try {
            sched.run();
        } catch (const std::exception& e) {
            std::fprintf(stderr, "scheduler loop failed: %s\n", e.what());
            std::fflush(stderr);
            std::_Exit(1);
        }
    });
    const auto t0 = Clock::now();
    for (int i = 0; i < n; ++i) {
        if (rate > 0)
            std::this_thread::sleep_until(t0 + std::chrono::duration_cast<Clock::duration>(
                                                   std::chrono::duration<double>(offsets[static_cast<size_t>(i)])));
        const std::string rid = "req:" + std::to_string(i);
        {
            std::lock_guard<std::mutex> lock(mu);
            reqs[static_cast<size_t>(i)].submit = Clock::now();
        }
        while (!sched.submit(rid, rid, out_len[static_cast<size_t>(i)], 0.0f))
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    for (;;) {
        {
            std::lock_guard<std::mutex> lock(mu);
            if (completed >= n) break;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    const auto t1 = Clock::now();
    sched.stop();
    loop.join();

    long out_tokens = 0;
    std::vector<double> ttft;
    for (int i = 0; i < n; ++i) {
        const Req& r = reqs[static_cast<size_t>(i)];
        out_tokens += static_cast<long>(r.tokens.size());
        const double tt = std::chrono::duration<double, std::milli>(r.first - r.submit).count();
        ttft.push_back(tt);
        if (opt("per_request", 0)) {
            std::printf("{\"req\": %d, \"prompt\": [", i);
            const auto& p = g_prompts[static_cast<size_t>(i)];
            for (size_t k = 0; k < p.size(); ++k) std::printf(k ? ", %d" : "%d", p[k]);
            std::printf("], \"tokens\": [");
            for (size_t k = 0; k < r.tokens.size(); ++k) std::printf(k ? ", %d" : "%d", r.tokens[k]);
            std::printf("], \"finish\": %d, \"ttft_ms\": %.3f}\n", r.finish, tt);
        }
    }
    const double wall = std::chrono::duration<double>(t1 - t0).count();
    std::printf(
        "{\"summary\": true, \"generator\": \"%s\", \"static\": %d, \"requests\": %d, \"max_batch\": %d, "
        "\"output_tokens\": %ld, \"makespan_s\": %.4f, \"output_tok_s\": %.2f, \"ttft_p50_ms\": %.3f, "
        "\"ttft_p99_ms\": %.3f}\n",
        kind.c_str(), sc.static_batching ? 1 : 0, n, max_batch, out_tokens, wall, out_tokens / wall, pct(ttft, 0.5),
        pct(ttft, 0.99));
    return 0;
}
