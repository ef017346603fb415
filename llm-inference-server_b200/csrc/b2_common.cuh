// b2_common.cuh -- dtype traits, 16-byte vector conversion and the sm_100a
// PTX primitives (mbarrier, bulk async copy, named barriers, bounded waits)
// shared by the decode kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2_decode.h"

namespace b2 {

constexpr int kBlockTokens = B2_BLOCK_TOKENS;

// Per-device error word (see B2_DEVERR_*).  Kernels OR bits into it; the host
// reads and clears it with b2_device_errors().  Defined here: the library is
// one translation unit (b2_decode.cu), so this header is included once.
__device__ unsigned int g_device_errors = 0;

__device__ __forceinline__ void flag_error(unsigned int bits) { atomicOr(&g_device_errors, bits); }

// ------------------------------------------------------------- dtype traits

template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static constexpr int kPer16B = 4;
    static constexpr bool kIsBf16 = false;
    __device__ __forceinline__ static float to_f(float x) { return x; }
    __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <>
struct Elem<__half> {
    static constexpr int kPer16B = 8;
    static constexpr bool kIsBf16 = false;
    __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
    __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};
template <>
struct Elem<__nv_bfloat16> {
    static constexpr int kPer16B = 8;
    static constexpr bool kIsBf16 = true;
    __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Widen one 16-byte vector of T into kPer16B floats.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float* f);

template <>
__device__ __forceinline__ void unpack16<float>(const uint4& raw, float* f) {
    f[0] = __uint_as_float(raw.x);
    f[1] = __uint_as_float(raw.y);
    f[2] = __uint_as_float(raw.z);
    f[3] = __uint_as_float(raw.w);
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& raw, float* f) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
        float2 v = __half22float2(h2);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& raw, float* f) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        // bf16 -> f32 is a 16-bit shift.
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

// Round kPer16B floats to T and pack them into one 16-byte vector.
template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f);

template <>
__device__ __forceinline__ uint4 pack16<float>(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h2 = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h2);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 b2 = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&b2);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Store n (= kPer16B of the source type, 4 or 8) floats as OutT at dst,
// which is 16-byte aligned.
template <typename OutT, int N>
__device__ __forceinline__ void store_row(OutT* dst, const float* f) {
    constexpr int P = Elem<OutT>::kPer16B;
    static_assert(N % P == 0, "store width");
#pragma unroll
    for (int i = 0; i < N / P; ++i) *reinterpret_cast<uint4*>(dst + i * P) = pack16<OutT>(f + i * P);
}

// ------------------------------------------------- mixed-precision chunk math
// sm_100 has FMA-pipe instructions that take 16-bit operands with an fp32
// accumulator (fma.rn.f32.{f16,bf16}, add.rn.f32.{f16,bf16}).  A product of
// two 16-bit floats is exact in fp32, so dot16 gives the same value as
// widening both operands first -- without a separate conversion instruction
// per element (the widening cvt runs on the quarter-rate XU pipe).

// acc + sum_e q[e] * k[e] over one 16-byte chunk; q and k hold the same dtype.
template <typename T>
__device__ __forceinline__ float dot16(const uint4& q, const uint4& k, float acc);

template <>
__device__ __forceinline__ float dot16<float>(const uint4& q, const uint4& k, float acc) {
    acc = fmaf(__uint_as_float(q.x), __uint_as_float(k.x), acc);
    acc = fmaf(__uint_as_float(q.y), __uint_as_float(k.y), acc);
    acc = fmaf(__uint_as_float(q.z), __uint_as_float(k.z), acc);
    return fmaf(__uint_as_float(q.w), __uint_as_float(k.w), acc);
}

#define B2_DOT2_ASM(TY, REG)                                                                   \
    "{\n\t.reg ." REG " ql, qh, kl, kh;\n\t"                                                   \
    "mov.b32 {ql, qh}, %1;\n\t"                                                                \
    "mov.b32 {kl, kh}, %2;\n\t"                                                                \
    "fma.rn.f32." TY " %0, ql, kl, %0;\n\t"                                                    \
    "fma.rn.f32." TY " %0, qh, kh, %0;\n\t}"

__device__ __forceinline__ float dot2_f16(uint32_t q2, uint32_t k2, float acc) {
    asm(B2_DOT2_ASM("f16", "f16") : "+f"(acc) : "r"(q2), "r"(k2));
    return acc;
}
__device__ __forceinline__ float dot2_bf16(uint32_t q2, uint32_t k2, float acc) {
    asm(B2_DOT2_ASM("bf16", "b16") : "+f"(acc) : "r"(q2), "r"(k2));
    return acc;
}
#undef B2_DOT2_ASM

template <>
__device__ __forceinline__ float dot16<__half>(const uint4& q, const uint4& k, float acc) {
    // two independent chains, summed at the end, halve the dependency depth
    float a = dot2_f16(q.x, k.x, acc);
    float b = dot2_f16(q.y, k.y, 0.0f);
    a = dot2_f16(q.z, k.z, a);
    b = dot2_f16(q.w, k.w, b);
    return a + b;
}
template <>
__device__ __forceinline__ float dot16<__nv_bfloat16>(const uint4& q, const uint4& k, float acc) {
    float a = dot2_bf16(q.x, k.x, acc);
    float b = dot2_bf16(q.y, k.y, 0.0f);
    a = dot2_bf16(q.z, k.z, a);
    b = dot2_bf16(q.w, k.w, b);
    return a + b;
}

// Both halves of a packed pair widened exactly to fp32 on the FMA pipe
// (x + 0 with x a 16-bit float and the sum in fp32).
__device__ __forceinline__ float2 widen2_f16(uint32_t w) {
    float lo, hi;
    asm("{\n\t.reg .f16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "add.rn.f32.f16 %0, a, %3;\n\tadd.rn.f32.f16 %1, b, %3;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "r"(w), "f"(0.0f));
    return make_float2(lo, hi);
}

// acc[e] += p * v[e] over one 16-byte chunk of v.
template <typename T>
__device__ __forceinline__ void axpy16(float p, const uint4& v, float* acc);

template <>
__device__ __forceinline__ void axpy16<float>(float p, const uint4& v, float* acc) {
    acc[0] = fmaf(p, __uint_as_float(v.x), acc[0]);
    acc[1] = fmaf(p, __uint_as_float(v.y), acc[1]);
    acc[2] = fmaf(p, __uint_as_float(v.z), acc[2]);
    acc[3] = fmaf(p, __uint_as_float(v.w), acc[3]);
}
template <>
__device__ __forceinline__ void axpy16<__half>(float p, const uint4& v, float* acc) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = widen2_f16(w[i]);
        acc[2 * i] = fmaf(p, f.x, acc[2 * i]);
        acc[2 * i + 1] = fmaf(p, f.y, acc[2 * i + 1]);
    }
}
template <>
__device__ __forceinline__ void axpy16<__nv_bfloat16>(float p, const uint4& v, float* acc) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(p, __uint_as_float(w[i] << 16), acc[2 * i]);
        acc[2 * i + 1] = fmaf(p, __uint_as_float(w[i] & 0xffff0000u), acc[2 * i + 1]);
    }
}

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wall-clock bound on every pipeline wait: past it the wait reports failure
// and the caller flags B2_DEVERR_TIMEOUT and winds down instead of spinning.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

// Waits for the phase with the given parity to complete.  Returns false if
// the wall-clock limit passed first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// One-dimensional bulk async copy global -> shared, completing on an mbarrier
// (the TMA engine's untiled form; no tensor map; into this CTA's own shared
// memory).  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Asks the TMA engine to bring [src, src + bytes) into L2 (no destination, no
// completion): a hint that cannot change any value read later, since L2 is
// where every SM's reads and writes meet.  src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Named barrier over the first nthreads threads of the CTA (multiple of 32).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participants.
__device__ __forceinline__ bool named_sync_or(int id, int nthreads, bool pred) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred pin, pout;\n\t"
        "setp.ne.u32 pin, %1, 0;\n\t"
        "bar.red.or.pred pout, %2, %3, pin;\n\t"
        "selp.u32 %0, 1, 0, pout;\n\t}"
        : "=r"(out)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
        : "memory");
    return out != 0;
}

__device__ __forceinline__ uint4 ld_shared16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Acquire-release fence at GPU scope (lighter than the sequentially
// consistent fence __threadfence() issues).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// 2^x by the SFU in one instruction (ex2.approx.ftz: relative error ~2^-22;
// -inf gives 0).  The softmax weights and rescale factors of the attention
// kernels use it: the error is far below their 16-bit inputs' resolution and
// the 2e-3 output bar.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Programmatic dependent launch.  launch_dependents lets the next kernel on
// the stream start its prologue; pdl_wait blocks until the previous kernel
// has completed and its writes are visible (a no-op when the launch had no
// programmatic dependency).  A kernel reads nothing the previous one writes,
// and writes nothing it reads, before its pdl_wait.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace b2
