// lm_head_tc.cuh -- the decode step's tied lm_head and greedy argmax in one
// kernel on the 5th-generation tensor cores: token[b] = argmax_v T(x[b] . w[v])
// over v < vocab, ties to the lowest v.
//
// The reference runs a cuBLAS GEMM into a [batch][vocab] logits buffer and
// then one argmax block per row (gpu-engine/src/engine.cu:202-203,
// kernels/logits.cu:18-57); the CPU path takes the first maximum of the
// fp32 logits (reference/cpu_model.cpp:182-196).  Here the logits never
// leave the chip:
//
//   * work items of (VN <= 256 vocabulary rows, 128 batch rows): MMA M = the
//     batch rows (zero rows past the batch), N = VN vocabulary rows, K in
//     64-element SWIZZLE_128B TMA boxes, the fp32 logits tile D[batch][vocab]
//     in TMEM.  Weights on the N side: each tcgen05.mma instruction takes in
//     up to 8 KB of weight rows.  (With the weights as M = 128, the operand
//     order of linear_tc.cuh, per-CTA stamps showed ~0.5 us per 64-element K
//     block whatever the batch -- 16 or 256 columns -- so the instruction
//     count per weight byte, not the arithmetic, paced the stream.)  Whole K
//     per item: a max does not distribute over partial sums;
//   * VN is sized so the items spread evenly over the SMs (GPT-2's 50257 rows
//     at batch <= 128: 176 rows, 286 items, two per SM at most; 256-row items
//     left a third of the SMs with twice the weights of the rest);
//   * persistent: one CTA per SM walks its items (blockIdx.x, + grid, ...)
//     with one ring running across item boundaries and two TMEM
//     accumulators, so the argmax of one item overlaps the MMAs of the next;
//   * the weight rows stream before griddepcontrol.wait (the tied embedding
//     never depends on the previous kernel), x after it;
//   * epilogue: a thread owns one batch row (its TMEM lane) and every other
//     group of 32 of the item's columns.  Each logit is rounded to T exactly
//     as the unfused path stores it and packed into a 32-bit key
//     (order-preserving 16-bit image of the T value, then 0xFFFF - column) so
//     that the larger key is the larger logit and, among equal logits, the
//     lower index; the thread keeps the largest, the two warps of a lane
//     quadrant meet in shared memory, and one 64-bit atomic max per batch row
//     -- (order-preserving image of the value, 0xFFFFFFFF - vocabulary index)
//     -- merges the CTAs;
//   * the last CTA to finish (an acquire-release counter) turns the keys
//     into tokens and leaves keys and counter at zero for the next launch.
//
// NaN logits never win against a number (their key is the smallest one, as
// b2_argmax_rows never takes a NaN); rows past the vocabulary never count.
// Roles (320 threads): warp 0 lane 0 TMA producer, warp 1 TMEM owner and
// (lane 0) MMA issuer, warps 2-9 epilogue (two per TMEM lane quadrant).
// Every mbarrier wait is bounded.
#pragma once

#include "b2_common.cuh"
#include "tcgen05.cuh"

namespace b2 {

constexpr int kLmMaxVRows = 256;  // vocabulary rows per work item at most (MMA N)
constexpr int kLmBRows = 128;     // batch rows per work item (MMA M)
constexpr int kLmKBlock = 64;     // K elements per stage (one 128-B swizzle row)
constexpr int kLmXBytes = kLmBRows * kLmKBlock * 2;  // x box: 16 KiB
constexpr int kLmEpiWarps = 8;  // two per TMEM lane quadrant, taking alternate groups of 32 columns
constexpr int kLmThreads = 64 + 32 * kLmEpiWarps;
constexpr uint32_t kLmAccCols = kLmMaxVRows;  // TMEM columns per accumulator; the kernel holds two

struct LmParams {
    int batch, vocab;
    int vn;               // vocabulary rows per work item: a multiple of 16, 16 .. 256 (the MMA's N)
    int xrows;            // x rows each stage loads: the batch rounded up to 16 (at most 128); the
                          // A tile's rows past them hold stale bytes and feed only unused result rows
    int kb_total;         // 64-element K blocks
    int stages;           // ring slots
    int n_tiles, chunks;  // work item w: vocabulary tile w / chunks, batch chunk w % chunks
    unsigned long long* keys;  // [batch] best keys so far; zero between launches
    unsigned int* counter;     // CTAs finished; zero between launches
    int* tokens;               // [batch]
};

// Shared-memory plan (bytes from the 1024-aligned base): the ring of
// [weights | x] stages, the two column halves' keys [2][128], the last-CTA
// flag, the barriers (ring full/empty, two accumulator full/empty pairs),
// the TMEM slot.
struct LmLayout {
    // a stage: vn weight rows of 128 bytes (vn a multiple of 16, so 1 KiB-aligned), then the x box
    __host__ __device__ static constexpr int w_bytes(int vn) { return vn * kLmKBlock * 2; }
    __host__ __device__ static constexpr int stage_bytes(int vn) { return w_bytes(vn) + kLmXBytes; }
    __host__ __device__ static constexpr int off_red(int vn, int stages) { return stages * stage_bytes(vn); }
    __host__ __device__ static constexpr int off_flag(int vn, int stages) { return off_red(vn, stages) + 2 * kLmBRows * 4; }
    __host__ __device__ static constexpr int off_bars(int vn, int stages) { return off_flag(vn, stages) + 16; }
    __host__ __device__ static constexpr int off_tmem(int vn, int stages) {
        return off_bars(vn, stages) + 8 * (2 * stages + 4);
    }
    __host__ __device__ static constexpr int bytes(int vn, int stages) { return off_tmem(vn, stages) + 16 + 1024; }
};

// Order-preserving 16-bit image of an f16 / bf16 value: a larger image is a
// larger value; -0 maps like +0; NaN maps to 0, below every number.
template <typename T>
__device__ __forceinline__ uint32_t lm_ord16(uint32_t h) {
    const bool nan = Elem<T>::kIsBf16 ? ((h & 0x7F80u) == 0x7F80u && (h & 0x007Fu) != 0u)
                                      : ((h & 0x7C00u) == 0x7C00u && (h & 0x03FFu) != 0u);
    if (nan) return 0u;
    if (h == 0x8000u) h = 0u;
    return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}

// The T value behind a non-zero order image, widened to float.
template <typename T>
__device__ __forceinline__ float lm_from_ord16(uint32_t o) {
    const uint32_t h = (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu);
    if constexpr (Elem<T>::kIsBf16) return __uint_as_float(h << 16);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// Order-preserving 32-bit image of a (non-NaN) float; 0 is left for NaN.
__device__ __forceinline__ uint32_t lm_ord32(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ uint32_t lm_bits(float v) {
    if constexpr (Elem<T>::kIsBf16) return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v)));
}

// The 32-bit key of one logit (lm_ord16 of its T value, then rowkey); 0 for
// NaN.  rowkey = 0xFFFF - row; a row that does not count passes valid = false.
template <typename T>
__device__ __forceinline__ uint32_t lm_key(float v, uint32_t rowkey, bool valid) {
    uint32_t h = lm_bits<T>(v);
    if (h == 0x8000u) h = 0u;  // -0 like +0
    const bool nan = (h & 0x7FFFu) > (Elem<T>::kIsBf16 ? 0x7F80u : 0x7C00u);
    const uint32_t o = h ^ ((h & 0x8000u) ? 0xFFFFu : 0x8000u);
    return valid && !nan ? (o << 16) | rowkey : 0u;
}

template <typename T>
__global__ void __launch_bounds__(kLmThreads, 1)
    lm_head_argmax_kernel(const LmParams p, const __grid_constant__ CUtensorMap w_map,
                          const __grid_constant__ CUtensorMap x_map) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int nkb = p.kb_total;
    const int ST = p.stages;
    const int VN = p.vn;
    const int SBY = LmLayout::stage_bytes(VN);
    const int WBY = LmLayout::w_bytes(VN);
    const uint32_t TX = static_cast<uint32_t>(WBY + p.xrows * kLmKBlock * 2);  // bytes a stage receives
    const int n_items = p.n_tiles * p.chunks;
    const int G = static_cast<int>(gridDim.x);
    // this CTA's work items: blockIdx.x, + G, ... (CTAs next to each other
    // take the batch chunks of one vocabulary tile together, so its weight
    // rows come from HBM once)
    const int my_items = (n_items - static_cast<int>(blockIdx.x) + G - 1) / G;
    const int total = my_items * nkb;  // K blocks through the ring

    uint32_t* red = reinterpret_cast<uint32_t*>(smem + LmLayout::off_red(VN, ST));  // [2 halves][128 rows]
    int* last_flag = reinterpret_cast<int*>(smem + LmLayout::off_flag(VN, ST));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + LmLayout::off_bars(VN, ST));
    uint64_t* empty = full + ST;
    uint64_t* acc_full = empty + ST;     // [2] MMA -> epilogue
    uint64_t* acc_empty = acc_full + 2;  // [2] epilogue (every epilogue warp) -> MMA
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LmLayout::off_tmem(VN, ST));

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kLmEpiWarps);
        }
        *last_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * kLmAccCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    int issued = 0;  // producer: K blocks issued (their copies must land before the CTA leaves)
    if (warp == 0) {
        if (lane == 0) {
            // The weight rows never depend on the kernel ahead: the first ring
            // fills take theirs before griddepcontrol.wait, x after it.
            const int npre = min(total, ST);
            for (int i = 0; i < npre; ++i) {
                const int w = static_cast<int>(blockIdx.x) + (i / nkb) * G;
                mbar_arrive_expect_tx(&full[i], TX);
                tma_load_2d(smem + i * SBY, &w_map, (i % nkb) * kLmKBlock, (w / p.chunks) * VN, &full[i]);
            }
            pdl_wait();  // x is the previous kernel's output
            for (int i = 0; i < npre; ++i) {
                const int w = static_cast<int>(blockIdx.x) + (i / nkb) * G;
                tma_load_2d(smem + i * SBY + WBY, &x_map, (i % nkb) * kLmKBlock, (w % p.chunks) * kLmBRows,
                            &full[i]);
            }
            issued = npre;
            for (int i = npre; i < total; ++i) {
                const int s = i % ST;
                if (!mbar_wait_bounded(&empty[s], (static_cast<uint32_t>(i / ST) & 1u) ^ 1u)) {
                    flag_error(B2_DEVERR_TIMEOUT);
                    break;
                }
                const int w = static_cast<int>(blockIdx.x) + (i / nkb) * G;
                const int kc = (i % nkb) * kLmKBlock;
                mbar_arrive_expect_tx(&full[s], TX);
                tma_load_2d(smem + s * SBY, &w_map, kc, (w / p.chunks) * VN, &full[s]);
                tma_load_2d(smem + s * SBY + WBY, &x_map, kc, (w % p.chunks) * kLmBRows, &full[s]);
                issued = i + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc<T>(kLmBRows, VN, false, false);
            for (int i = 0; i < total; ++i) {
                const int j = i / nkb, kb = i - j * nkb;
                const int buf = j & 1;
                if (kb == 0) {  // the epilogue has read this accumulator's previous item
                    if (!mbar_wait_bounded(&acc_empty[buf], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u)) {
                        flag_error(B2_DEVERR_TIMEOUT);
                        break;
                    }
                    tc_fence_after();
                }
                const int s = i % ST;
                if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(i / ST) & 1u)) {
                    flag_error(B2_DEVERR_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t bw = smem_addr(smem + s * SBY);        // B: VN weight rows
                const uint32_t ax = bw + static_cast<uint32_t>(WBY);  // A: 128 batch rows
                const uint32_t d = tmem + static_cast<uint32_t>(buf) * kLmAccCols;
#pragma unroll
                for (int k = 0; k < kLmKBlock / 16; ++k)
                    umma_f16(d, sw128_desc(ax + 32 * k, 16, 1024), sw128_desc(bw + 32 * k, 16, 1024), idesc,
                             (kb | k) != 0);
                umma_commit(&empty[s]);  // the slot is free once these MMAs have read it
                if (kb == nkb - 1) umma_commit(&acc_full[buf]);
            }
        }
    } else {
        // ---- epilogue warps: TMEM lane quadrant q holds batch rows b0 + 32q ...;
        // the two warps of a quadrant take alternate groups of 32 of the VN columns
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = q * 32 + lane;  // this thread's batch row in the item
        const int t = tid - 64;
        bool ok = true;
        for (int j = 0; j < my_items && ok; ++j) {
            const int w = static_cast<int>(blockIdx.x) + j * G;
            const int n0 = (w / p.chunks) * VN;
            const int b0 = (w % p.chunks) * kLmBRows;
            const int buf = j & 1;
            ok = mbar_wait_bounded(&acc_full[buf], static_cast<uint32_t>(j >> 1) & 1u);
            if (!ok && lane == 0) flag_error(B2_DEVERR_TIMEOUT);
            __syncwarp();
            tc_fence_after();
            const uint32_t taddr =
                tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf) * kLmAccCols;
            uint32_t best = 0u;
#pragma unroll 1
            for (int c = half * 32; c < VN; c += 64) {  // columns past VN: allocated, never counted
                float v[32];
                tmem_ld32(taddr + static_cast<uint32_t>(c), v);
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    const int col = c + jj;  // vocabulary row n0 + col
                    const uint32_t key =
                        lm_key<T>(v[jj], static_cast<uint32_t>(0xFFFF - col), ok && col < VN && n0 + col < p.vocab);
                    best = key > best ? key : best;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);  // the MMAs may overwrite this accumulator
            red[half * kLmBRows + row] = best;
            named_sync(1, kLmThreads - 64);
            if (j == 0) pdl_wait();  // the keys of the launch before this one are cleared by its last CTA
            if (t < kLmBRows) {
                const uint32_t k0 = red[t], k1 = red[kLmBRows + t];
                const uint32_t k = k0 > k1 ? k0 : k1;
                if (k != 0u && b0 + t < p.batch) {
                    const uint32_t o = k >> 16;
                    const int n = n0 + static_cast<int>(0xFFFFu - (k & 0xFFFFu));
                    const uint32_t hi = o == 0u ? 0u : lm_ord32(lm_from_ord16<T>(o));
                    const unsigned long long key = (static_cast<unsigned long long>(hi) << 32) |
                                                   static_cast<unsigned long long>(0xFFFFFFFFu - n);
                    atomicMax(p.keys + b0 + t, key);
                }
            }
            named_sync(1, kLmThreads - 64);  // red is rewritten by the next item
        }
        if (!ok) pdl_wait();  // a warp that gave up still orders its counter update after the kernel ahead
        __threadfence();
        named_sync(1, kLmThreads - 64);
        if (t == 0) {
            unsigned int old;
            asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.counter) : "memory");
            *last_flag = old == gridDim.x - 1 ? 1 : 0;
        }
        named_sync(1, kLmThreads - 64);
        if (*last_flag) {
            // Every CTA's maxima are in: tokens out, keys and counter back to zero.
            for (int b = t; b < p.batch; b += kLmThreads - 64) {
                const unsigned long long key = atomicExch(p.keys + b, 0ull);
                p.tokens[b] = key == 0ull ? 0 : static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key));
            }
            if (t == 0) atomicExch(p.counter, 0u);
        }
    }

    // ---- exit: this CTA's copies have landed, its MMAs are done, TMEM freed
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < ST && s < issued; ++s) {
            const int last_use = (issued - 1 - s) / ST;  // uses of slot s: s, s + ST, ...
            if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(last_use) & 1u)) flag_error(B2_DEVERR_TIMEOUT);
        }
    }
    if (warp == 1 && lane == 0 && my_items > 0) {
        // the last item's accumulator-full phase completes after every MMA of the CTA
        const int jl = my_items - 1;
        if (!mbar_wait_bounded(&acc_full[jl & 1], static_cast<uint32_t>(jl >> 1) & 1u)) flag_error(B2_DEVERR_TIMEOUT);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 2 * kLmAccCols);
}

}  // namespace b2
