// lt_gemm.h -- the 16-bit engine's decode GEMMs on cuBLASLt, with the
// algorithm for each shape chosen by timing.
//
// Row-major Y[batch][O] = X[batch][I] . W^T (+ bias, GELU) with W stored
// [O][I], the convention of gpu-engine/include/engine/kernels.h:9-20; in
// cuBLASLt's column-major terms C[O x batch] = W^T[O x I] . X^T[I x batch]
// (A = W, transposed; B = X).  cublasGemmEx takes the algorithm cuBLAS's
// heuristic ranks first; at the decode step's skinny shapes (batch 128 per GPU
// at the 8-GPU GPT-2 XL shape) that is not always the fastest, so the engine
// times the heuristic's top candidates once per shape, on its own buffers and
// stream, before the step is captured, and keeps the fastest.  The FC layer's
// bias + GELU can ride in the GEMM's epilogue (CUBLASLT_EPILOGUE_GELU_BIAS),
// which removes one launch per layer.
#pragma once

#include <cublasLt.h>
#include <cuda_runtime.h>

#include <map>
#include <stdexcept>
#include <string>
#include <tuple>

namespace b2 {
namespace eng {

class LtGemm {
public:
    enum Epi { kNone = 0, kGeluBias = 1 };

    LtGemm() = default;
    LtGemm(const LtGemm&) = delete;
    LtGemm& operator=(const LtGemm&) = delete;
    ~LtGemm() {
        for (auto& kv : plans_) kv.second.release();
        if (h_) cublasLtDestroy(h_);
    }

    void init(cudaDataType_t type, void* workspace, size_t ws_bytes) {
        ok(cublasLtCreate(&h_), "cublasLtCreate");
        type_ = type;
        ws_ = workspace;
        ws_bytes_ = ws_bytes;
    }

    // Y = epi(X . W^T): the plan of this shape is made and timed on first use
    // (outside any stream capture: the caller tunes every shape of a graph
    // before capturing it).
    void run(int batch, int I, int O, const void* X, const void* W, void* Y, int ldy, Epi epi, const void* bias,
             cudaStream_t s, bool may_tune) {
        Plan& p = plan(batch, I, O, ldy, epi);
        if (epi == kGeluBias)
            ok(cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias)),
               "bias pointer");
        if (!p.tuned) {
            if (!may_tune) throw std::runtime_error("cuBLASLt shape used before it was tuned");
            tune(p, X, W, Y, s);
        }
        const float alpha = 1.0f, beta = 0.0f;
        ok(cublasLtMatmul(h_, p.op, &alpha, W, p.a, X, p.b, &beta, Y, p.c, Y, p.c, &p.algo, ws_, ws_bytes_, s),
           "cublasLtMatmul");
    }

    // Whether the shape has a timed algorithm already.
    bool tuned(int batch, int I, int O, int ldy, Epi epi) const {
        auto it = plans_.find(std::make_tuple(batch, I, O, ldy, static_cast<int>(epi)));
        return it != plans_.end() && it->second.tuned;
    }

    // The measured time of the chosen algorithm and of the heuristic's first
    // choice (what cublasGemmEx would run), in microseconds, for reports.
    std::pair<float, float> times(int batch, int I, int O, int ldy, Epi epi) const {
        auto it = plans_.find(std::make_tuple(batch, I, O, ldy, static_cast<int>(epi)));
        if (it == plans_.end()) return {0.0f, 0.0f};
        return {it->second.best_us, it->second.first_us};
    }

private:
    struct Plan {
        cublasLtMatmulDesc_t op = nullptr;
        cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
        cublasLtMatmulAlgo_t algo{};
        bool tuned = false;
        float best_us = 0.0f, first_us = 0.0f;
        void release() {
            if (op) cublasLtMatmulDescDestroy(op);
            if (a) cublasLtMatrixLayoutDestroy(a);
            if (b) cublasLtMatrixLayoutDestroy(b);
            if (c) cublasLtMatrixLayoutDestroy(c);
            op = nullptr;
            a = b = c = nullptr;
        }
    };

    static void ok(cublasStatus_t st, const char* what) {
        if (st != CUBLAS_STATUS_SUCCESS) throw std::runtime_error(std::string(what) + ": cuBLASLt status " + std::to_string(st));
    }

    Plan& plan(int batch, int I, int O, int ldy, Epi epi) {
        const auto key = std::make_tuple(batch, I, O, ldy, static_cast<int>(epi));
        auto it = plans_.find(key);
        if (it != plans_.end()) return it->second;
        Plan p;
        ok(cublasLtMatmulDescCreate(&p.op, CUBLAS_COMPUTE_32F, CUDA_R_32F), "matmul desc");
        const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
        ok(cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA)), "transa");
        ok(cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB)), "transb");
        if (epi == kGeluBias) {
            const cublasLtEpilogue_t e = CUBLASLT_EPILOGUE_GELU_BIAS;
            ok(cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_EPILOGUE, &e, sizeof(e)), "epilogue");
        }
        // W is [O][I] row-major = I x O column-major (ld I), used transposed.
        ok(cublasLtMatrixLayoutCreate(&p.a, type_, I, O, I), "layout A");
        ok(cublasLtMatrixLayoutCreate(&p.b, type_, I, batch, I), "layout B");
        ok(cublasLtMatrixLayoutCreate(&p.c, type_, O, batch, ldy), "layout C");
        return plans_.emplace(key, p).first->second;
    }

    // Times the heuristic's top candidates (a few runs each, CUDA events on
    // the caller's stream) and keeps the fastest that runs.
    void tune(Plan& p, const void* X, const void* W, void* Y, cudaStream_t s) {
        cublasLtMatmulPreference_t pref = nullptr;
        ok(cublasLtMatmulPreferenceCreate(&pref), "preference");
        ok(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes_,
                                                sizeof(ws_bytes_)),
           "preference workspace");
        constexpr int kCand = 16;
        cublasLtMatmulHeuristicResult_t res[kCand];
        int n = 0;
        const cublasStatus_t hs = cublasLtMatmulAlgoGetHeuristic(h_, p.op, p.a, p.b, p.c, p.c, pref, kCand, res, &n);
        cublasLtMatmulPreferenceDestroy(pref);
        ok(hs, "algorithm heuristic");
        if (n <= 0) throw std::runtime_error("cuBLASLt offers no algorithm for a decode GEMM shape");
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        const float alpha = 1.0f, beta = 0.0f;
        float best = 1e30f;
        int best_i = -1;
        for (int i = 0; i < n; ++i) {
            if (res[i].state != CUBLAS_STATUS_SUCCESS) continue;
            bool good = true;
            for (int r = 0; r < 2 && good; ++r)
                good = cublasLtMatmul(h_, p.op, &alpha, W, p.a, X, p.b, &beta, Y, p.c, Y, p.c, &res[i].algo, ws_,
                                      ws_bytes_, s) == CUBLAS_STATUS_SUCCESS;
            if (!good) continue;
            constexpr int kReps = 10;
            cudaEventRecord(e0, s);
            for (int r = 0; r < kReps; ++r)
                cublasLtMatmul(h_, p.op, &alpha, W, p.a, X, p.b, &beta, Y, p.c, Y, p.c, &res[i].algo, ws_, ws_bytes_, s);
            cudaEventRecord(e1, s);
            cudaEventSynchronize(e1);
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, e0, e1);
            const float us = ms * 1000.0f / kReps;
            if (i == 0) p.first_us = us;
            if (us < best) {
                best = us;
                best_i = i;
            }
        }
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        cudaGetLastError();
        if (best_i < 0) throw std::runtime_error("no cuBLASLt algorithm ran for a decode GEMM shape");
        p.algo = res[best_i].algo;
        p.best_us = best;
        p.tuned = true;
    }

    cublasLtHandle_t h_ = nullptr;
    cudaDataType_t type_ = CUDA_R_16F;
    void* ws_ = nullptr;
    size_t ws_bytes_ = 0;
    std::map<std::tuple<int, int, int, int, int>, Plan> plans_;
};

}  // namespace eng
}  // namespace b2
