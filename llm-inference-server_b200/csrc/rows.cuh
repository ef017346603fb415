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
// r = residual_in + (x + bias); residual_out = r; out = LN(r) * gamma + beta.
// One CTA per row, each thread holding NCH 16-byte chunks of r in registers
// (the row is read once and written once).  Mean and variance are
// accumulated in double and the normalised value is formed as
// float((r - mean) * inv_std) * gamma + beta, the expression of
// cpu_model.cpp:33-45 (layernorm.cu:34-38 instead re-reads the half-rounded
// residual; this kernel does not).

// Sum over the CTA; every thread gets the result.  red needs 33 doubles.
__device__ __forceinline__ double block_sum(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        double w = lane < nw ? red[lane] : 0.0;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) w += __shfl_xor_sync(0xffffffffu, w, off);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    const double total = red[32];
    __syncthreads();  // red is reused by the next call
    return total;
}

template <typename T, int NCH>
__global__ void __launch_bounds__(1024) add_layernorm_kernel(T* out, T* residual_out, const T* x, const T* bias,
                                                             const T* residual_in, const T* gamma, const T* beta,
                                                             int d, float eps) {
    constexpr int E = Elem<T>::kPer16B;
    __shared__ double red[33];
    const int nch = d / E;
    const size_t base = static_cast<size_t>(blockIdx.x) * d;
    // gamma and beta are weights (nothing on the stream writes them): fetched
    // before waiting for the kernel that produced x and residual_in.
    uint4 graw[NCH], braw[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = threadIdx.x + i * static_cast<int>(blockDim.x);
        if (c < nch) {
            graw[i] = __ldg(reinterpret_cast<const uint4*>(gamma) + c);
            braw[i] = __ldg(reinterpret_cast<const uint4*>(beta) + c);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    float v[NCH][E];
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = threadIdx.x + i * static_cast<int>(blockDim.x);
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
    const double mean = block_sum(sum, red) / d;
    double var = 0.0;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = threadIdx.x + i * static_cast<int>(blockDim.x);
        if (c < nch) {
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const double df = static_cast<double>(v[i][e]) - mean;
                var = fma(df, df, var);
            }
        }
    }
    var = block_sum(var, red) / d;
    const float inv_std = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int c = threadIdx.x + i * static_cast<int>(blockDim.x);
        if (c < nch) {
            float gf[E], bf[E], y[E];
            unpack16<T>(graw[i], gf);
            unpack16<T>(braw[i], bf);
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
    const long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    // The first chunk's bias (a weight) is fetched before waiting for the
    // kernel that produced x.
    uint4 b0 = make_uint4(0u, 0u, 0u, 0u);
    if (i0 < nchunks) b0 = __ldg(reinterpret_cast<const uint4*>(bias) + static_cast<int>(i0 % row_chunks));
    pdl_launch_dependents();
    pdl_wait();
    for (long long i = i0; i < nchunks; i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float f[E], bf[E];
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(x) + i), f);
        unpack16<T>(i == i0 ? b0 : __ldg(reinterpret_cast<const uint4*>(bias) + static_cast<int>(i % row_chunks)), bf);
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
// first maximum).  Rows that start on a 16-byte boundary (a row stride that
// is a multiple of 16 bytes, as the engine pads its logits) are read in
// 16-byte vectors, several in flight per thread; otherwise (vocab 50257 as the
// row stride) element by element, coalesced across the CTA.
__device__ __forceinline__ void argmax_take(float x, int i, float& best, int& best_i) {
    if (x > best || (x == best && i < best_i)) {
        best = x;
        best_i = i;
    }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(512) argmax_kernel(int* out_tokens, const T* logits, int vocab, long long stride) {
    const T* row = logits + static_cast<long long>(blockIdx.x) * stride;
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    if constexpr (VEC) {
        constexpr int E = Elem<T>::kPer16B;
        constexpr int U = 4;  // vectors in flight per thread
        const int nvec = vocab / E;
        const uint4* rv = reinterpret_cast<const uint4*>(row);
        for (int base = threadIdx.x; base < nvec; base += U * blockDim.x) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int idx = base + u * static_cast<int>(blockDim.x);
                raw[u] = idx < nvec ? __ldg(rv + idx) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int idx = base + u * static_cast<int>(blockDim.x);
                if (idx < nvec) {
                    float f[E];
                    unpack16<T>(raw[u], f);
#pragma unroll
                    for (int e = 0; e < E; ++e) argmax_take(f[e], idx * E + e, best, best_i);
                }
            }
        }
        for (int v = nvec * E + static_cast<int>(threadIdx.x); v < vocab; v += blockDim.x)
            argmax_take(Elem<T>::to_f(row[v]), v, best, best_i);
    } else {
        for (int v = threadIdx.x; v < vocab; v += blockDim.x) argmax_take(Elem<T>::to_f(row[v]), v, best, best_i);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
        argmax_take(ob, oi, best, best_i);
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
            argmax_take(ob, oi, best, best_i);
        }
        if (lane == 0) out_tokens[blockIdx.x] = best_i == 0x7fffffff ? 0 : best_i;
    }
}

__global__ void add_one_kernel(int* out, const int* in, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = in[i] + 1;
}

}  // namespace b2
