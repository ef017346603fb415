// rows.cuh -- the row kernels around attention in the decode step:
// fused residual add + LayerNorm, bias + GELU(tanh), bias add, embedding
// gather, greedy argmax and the seq_lens + 1 update.  Arithmetic follows the
// reference CPU path (gpu-engine/src/reference/cpu_model.cpp) operation by
// operation, with explicit round-to-nearest intrinsics where a fused
// multiply-add would change the rounding the CPU path does.
#pragma once

#include <cfloat>

#include "b2_common.cuh"

namespace b2 {

// ------------------------------------------------------ add + LayerNorm
// r = x + bias + residual_in; residual_out = r; out = LN(r) * gamma + beta.
// One warp per row; each lane keeps up to NCH 16-byte chunks of r in
// registers, so the row is read once and written once.  Mean and variance
// are accumulated in double and the normalised value is formed as
// float((r - mean) * inv_std) * gamma + beta, the expression of
// cpu_model.cpp:33-45 (layernorm.cu:34-38 instead re-reads the half-rounded
// residual; this kernel does not).
template <typename T, int NCH>
__global__ void __launch_bounds__(128) add_layernorm_kernel(T* out, T* residual_out, const T* x, const T* bias,
                                                            const T* residual_in, const T* gamma, const T* beta,
                                                            int batch, int d, float eps) {
    constexpr int E = Elem<T>::kPer16B;
    const int row = static_cast<int>((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= batch) return;
    const int nch = d / E;
    const size_t base = static_cast<size_t>(row) * d;
    float v[NCH][E];
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
            // r = residual + (x + bias): the bias belongs to the GEMM output x,
            // as in the reference (add_bias before the residual add,
            // engine.cu:184-188; cpu_model.cpp:164-165 adds linear-with-bias).
            float r[E], xf[E];
            unpack16<T>(__ldg(reinterpret_cast<const uint4*>(residual_in + base) + c), r);
            if (x != nullptr) {
                unpack16<T>(__ldg(reinterpret_cast<const uint4*>(x + base) + c), xf);
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) xf[e] = 0.0f;
            }
            if (bias != nullptr) {
                float bf[E];
                unpack16<T>(__ldg(reinterpret_cast<const uint4*>(bias) + c), bf);
#pragma unroll
                for (int e = 0; e < E; ++e) xf[e] = __fadd_rn(xf[e], bf[e]);
            }
            if (x != nullptr || bias != nullptr) {
#pragma unroll
                for (int e = 0; e < E; ++e) r[e] = __fadd_rn(r[e], xf[e]);
            }
#pragma unroll
            for (int e = 0; e < E; ++e) {
                v[i][e] = r[e];
                sum += static_cast<double>(r[e]);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const double mean = sum / d;
    double var = 0.0;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const double df = static_cast<double>(v[i][e]) - mean;
                var = fma(df, df, var);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) var += __shfl_xor_sync(0xffffffffu, var, off);
    var /= d;
    const float inv_std = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
            float gf[E], bf[E], y[E];
            unpack16<T>(__ldg(reinterpret_cast<const uint4*>(gamma) + c), gf);
            unpack16<T>(__ldg(reinterpret_cast<const uint4*>(beta) + c), bf);
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const float nrm = static_cast<float>(__dmul_rn(static_cast<double>(v[i][e]) - mean,
                                                               static_cast<double>(inv_std)));
                y[e] = __fadd_rn(__fmul_rn(nrm, gf[e]), bf[e]);
            }
            if (residual_out != nullptr) reinterpret_cast<uint4*>(residual_out + base)[c] = pack16<T>(v[i]);
            reinterpret_cast<uint4*>(out + base)[c] = pack16<T>(y);
        }
    }
}

// ------------------------------------------------------ bias + GELU(tanh)
// gelu_new of cpu_model.cpp:49-54, evaluated in the same operation order.
__device__ __forceinline__ float gelu_tanh_ref(float x) {
    const float k = 0.7978845608028654f;
    const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    const float inner = __fmul_rn(k, __fadd_rn(x, cube));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

template <typename T>
__global__ void __launch_bounds__(256) bias_gelu_kernel(T* out, const T* x, const T* bias, long long nchunks,
                                                        int row_chunks) {
    constexpr int E = Elem<T>::kPer16B;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < nchunks;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % row_chunks);
        float f[E], bf[E];
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(x) + i), f);
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(bias) + c), bf);
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] = gelu_tanh_ref(__fadd_rn(f[e], bf[e]));
        reinterpret_cast<uint4*>(out)[i] = pack16<T>(f);
    }
}

// ------------------------------------------------------ bias add
template <typename T>
__global__ void __launch_bounds__(256) add_bias_kernel(T* out, const T* x, const T* bias, long long nchunks,
                                                       int row_chunks) {
    constexpr int E = Elem<T>::kPer16B;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < nchunks;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % row_chunks);
        float f[E], bf[E];
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(x) + i), f);
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(bias) + c), bf);
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] = __fadd_rn(f[e], bf[e]);
        reinterpret_cast<uint4*>(out)[i] = pack16<T>(f);
    }
}

// ------------------------------------------------------ embedding
template <typename T>
__global__ void __launch_bounds__(256) embedding_kernel(T* out, const T* wte, const T* wpe, const int* token_ids,
                                                        const int* positions, int batch, int row_chunks, int vocab,
                                                        int n_pos) {
    constexpr int E = Elem<T>::kPer16B;
    const long long total = static_cast<long long>(batch) * row_chunks;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(i / row_chunks);
        const int c = static_cast<int>(i - static_cast<long long>(b) * row_chunks);
        int tok = __ldg(token_ids + b);
        int pos = __ldg(positions + b);
        if (tok < 0 || tok >= vocab || pos < 0 || pos >= n_pos) {
            if (c == 0) flag_error(B2_DEVERR_TOKEN);
            tok = min(max(tok, 0), vocab - 1);
            pos = min(max(pos, 0), n_pos - 1);
        }
        float a[E], p[E];
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(wte) + static_cast<size_t>(tok) * row_chunks + c), a);
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(wpe) + static_cast<size_t>(pos) * row_chunks + c), p);
#pragma unroll
        for (int e = 0; e < E; ++e) a[e] = __fadd_rn(a[e], p[e]);
        reinterpret_cast<uint4*>(out)[i] = pack16<T>(a);
    }
}

// ------------------------------------------------------ greedy argmax
// One CTA per row; ties go to the lowest index (cpu_model.cpp:190 keeps the
// first maximum).  Rows need not be 16-byte aligned (vocab 50257 is odd), so
// loads are per element, coalesced across the CTA.
template <typename T>
__global__ void __launch_bounds__(256) argmax_kernel(int* out_tokens, const T* logits, int vocab) {
    const T* row = logits + static_cast<size_t>(blockIdx.x) * vocab;
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int v = threadIdx.x; v < vocab; v += blockDim.x) {
        const float x = Elem<T>::to_f(row[v]);
        if (x > best) {
            best = x;
            best_i = v;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
        if (ob > best || (ob == best && oi < best_i)) {
            best = ob;
            best_i = oi;
        }
    }
    __shared__ float s_best[32];
    __shared__ int s_idx[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        s_best[warp] = best;
        s_idx[warp] = best_i;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? s_best[lane] : -INFINITY;
        best_i = lane < nw ? s_idx[lane] : 0x7fffffff;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
            if (ob > best || (ob == best && oi < best_i)) {
                best = ob;
                best_i = oi;
            }
        }
        if (lane == 0) out_tokens[blockIdx.x] = best_i == 0x7fffffff ? 0 : best_i;
    }
}

__global__ void add_one_kernel(int* out, const int* in, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = in[i] + 1;
}

}  // namespace b2
