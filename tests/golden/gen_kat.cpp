// gen_kat.cpp -- writes the reference's kernel known-answer cases as JSON.
//
// Restates the setup of gpu-engine/tests/test_kernels.cpp:50-228 (the same
// std::mt19937 seeds, shapes and uniform_real_distribution ranges, drawn in
// the same order, so the inputs are the reference test's inputs bit for bit)
// and the test's own CPU expectation for each case:
//   embedding    seed 0, B=4, D=16, U(-1,1), ids {3,10,40,63}, pos {0..3}  (:50-96)
//   add+LN       seed 1, B=3, D=32, U(-2,2), gamma 1+0.1u, beta 0.1u       (:98-160)
//   bias+GELU    seed 2, B=2, D=24, U(-3,3)                                (:162-199)
//   argmax       seed 3, B=2, V=100, U(-5,5), [0][42] = [1][7] = 100       (:201-228)
// The reference compares its GPU output against these within max-abs 5e-2.
// Build and run: tests/golden/make_golden.py.
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

static void dump(const char* name, const std::vector<float>& v, bool last = false) {
    std::printf("  \"%s\": [", name);
    for (size_t i = 0; i < v.size(); ++i) std::printf("%s%.9g", i ? ", " : "", v[i]);
    std::printf("]%s\n", last ? "" : ",");
}

int main() {
    std::printf("{\n");
    {  // embedding
        const int batch = 4, d = 16;
        std::mt19937 rng(0);
        std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
        std::vector<float> wte(64 * d), wpe(32 * d);
        for (auto& v : wte) v = dist(rng);
        for (auto& v : wpe) v = dist(rng);
        const int tok[4] = {3, 10, 40, 63}, pos[4] = {0, 1, 2, 3};
        std::vector<float> expected(batch * d);
        for (int b = 0; b < batch; ++b)
            for (int i = 0; i < d; ++i) expected[b * d + i] = wte[tok[b] * d + i] + wpe[pos[b] * d + i];
        std::printf(" \"embedding\": {\n");
        dump("wte", wte);
        dump("wpe", wpe);
        std::printf("  \"token_ids\": [3, 10, 40, 63], \"positions\": [0, 1, 2, 3], \"batch\": 4, \"d\": 16,\n");
        dump("expected", expected, true);
        std::printf(" },\n");
    }
    {  // add + layernorm
        const int batch = 3, d = 32;
        std::mt19937 rng(1);
        std::uniform_real_distribution<float> dist(-2.0f, 2.0f);
        std::vector<float> x(batch * d), r(batch * d), g(d), be(d);
        for (auto& v : x) v = dist(rng);
        for (auto& v : r) v = dist(rng);
        for (auto& v : g) v = 1.0f + 0.1f * dist(rng);
        for (auto& v : be) v = 0.1f * dist(rng);
        std::vector<float> expected(batch * d);
        const float eps = 1e-5f;
        for (int b = 0; b < batch; ++b) {
            double mean = 0.0;
            std::vector<float> row(d);
            for (int i = 0; i < d; ++i) {
                row[i] = x[b * d + i] + r[b * d + i];
                mean += row[i];
            }
            mean /= d;
            double var = 0.0;
            for (int i = 0; i < d; ++i) var += (row[i] - mean) * (row[i] - mean);
            var /= d;
            const float inv_std = 1.0f / std::sqrt(static_cast<float>(var) + eps);
            for (int i = 0; i < d; ++i)
                expected[b * d + i] = static_cast<float>((row[i] - mean) * inv_std) * g[i] + be[i];
        }
        std::printf(" \"add_layernorm\": {\n  \"batch\": 3, \"d\": 32, \"eps\": 1e-5,\n");
        dump("x", x);
        dump("residual", r);
        dump("gamma", g);
        dump("beta", be);
        dump("expected", expected, true);
        std::printf(" },\n");
    }
    {  // bias + gelu
        const int batch = 2, d = 24;
        std::mt19937 rng(2);
        std::uniform_real_distribution<float> dist(-3.0f, 3.0f);
        std::vector<float> x(batch * d), bias(d);
        for (auto& v : x) v = dist(rng);
        for (auto& v : bias) v = dist(rng);
        auto gelu = [](float v) {
            const float k0 = 0.7978845608028654f;
            return 0.5f * v * (1.0f + std::tanh(k0 * (v + 0.044715f * v * v * v)));
        };
        std::vector<float> expected(batch * d);
        for (int b = 0; b < batch; ++b)
            for (int i = 0; i < d; ++i) expected[b * d + i] = gelu(x[b * d + i] + bias[i]);
        std::printf(" \"bias_gelu\": {\n  \"batch\": 2, \"d\": 24,\n");
        dump("x", x);
        dump("bias", bias);
        dump("expected", expected, true);
        std::printf(" },\n");
    }
    {  // argmax
        const int batch = 2, vocab = 100;
        std::mt19937 rng(3);
        std::uniform_real_distribution<float> dist(-5.0f, 5.0f);
        std::vector<float> logits(batch * vocab);
        for (auto& v : logits) v = dist(rng);
        logits[0 * vocab + 42] = 100.0f;
        logits[1 * vocab + 7] = 100.0f;
        std::printf(" \"argmax\": {\n  \"batch\": 2, \"vocab\": 100, \"expected\": [42, 7],\n");
        dump("logits", logits, true);
        std::printf(" }\n");
    }
    std::printf("}\n");
    return 0;
}
