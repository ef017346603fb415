// prefill_tc.cuh -- causal prefill attention over the paged KV cache on the
// 5th-generation tensor cores (tcgen05 + TMEM + TMA), head_dim 64.
//
// The reference has no prefill kernel: GpuEngineGenerator walks every prompt
// token through Engine::decode_step at batch 1
// (cpp-engine/src/gpu_engine_generator.cpp:28-42), so each prompt row reads
// the whole key prefix again.  Here the new rows of a sequence are query
// tiles: row i of sequence b (position seq_lens_pre[b] + i) attends the keys
// at positions [0, seq_lens_pre[b] + i] -- the result the reference's decode
// attention (gpu-engine/src/kernels/attention.cu:49-127, cpu_model.cpp:131-162)
// gives that row, with every key tile read once per 128 query rows.
//
// One CTA per (sequence, query head, 128-row query tile), two CTAs per SM
// (256 TMEM columns, ~82 KB of shared memory and <= 102 registers a thread
// each): a tile's chain -- K/V lands, S, softmax, P . V -- is serial within a
// CTA, so the second CTA's chain and its set-up fill the gaps (one CTA per SM
// with S double-buffered in TMEM ran 37 us where this runs 27 us at 8 x 512
// rows x 16 heads):
//   Q tile [128 rows][64]             smem, SWIZZLE_128B K-major (threads, + bias)
//   K, V tiles [128 keys][64]         8 paged blocks x one 16-row TMA box each,
//                                      2-slot ring
//   S = Q . K^T      M=128 N=128 K=64  fp32 in TMEM columns [0, 128)
//   O += P . V       M=128 N=64  K=128 fp32 in TMEM columns [128, 192), P read
//                                      from TMEM (the A operand of the MMA)
// P is written by the softmax threads as two 16-bit halves hi = T(p) and
// lo = T(p - hi) and both are multiplied in (16 significant bits per weight).
// P(t) overwrites S(t): each thread handles its 64 S columns as two chunks of
// 32, reading a chunk's scores before writing its packed hi words into the
// chunk's first 16 columns and its lo words into the next 16.  S(t + 1) is
// issued after P(t) . V(t) (one thread's MMAs execute in order, so the product
// has read P before S overwrites it), and the softmax, which waits for S(t + 1),
// thereby also knows P(t) . V(t) has finished when it rescales O.
// Softmax in log2 units with a lazily moved reference maximum (moves only when
// a tile's row maximum exceeds it by more than 8, so weights stay <= 2^8 and
// O is rescaled only then).  Causality comes from positions: key k counts for
// query row i iff k <= seq_lens_pre + i.  Key boxes past the last needed block
// are fetched at an out-of-range slab (TMA fills zeros); rows of the last block
// past the keys in use are zeroed before the PV product, so stale values there
// (never written) cannot reach the output.
//
// Roles (320 threads): warp 0 lane 0 TMA producer, warp 1 TMEM owner and
// (lane 0) MMA issuer, warps 2-9 softmax / epilogue: two threads per query row
// (warps w and w + 4 read the same TMEM lanes 32 * (w % 4) ...), each taking 64
// of a tile's 128 keys; the two halves of a row exchange their maxima (and at
// the end their sums) through shared memory.  Every wait is bounded; a wait
// that gives up flags B2_DEVERR_TIMEOUT and the CTA winds down through the
// common exit (its copies landed, its MMAs done, TMEM freed).
#pragma once

#include "b2_common.cuh"
#include "tcgen05.cuh"

namespace b2 {

constexpr int kPfRows = 128;                    // query rows per CTA (MMA M)
constexpr int kPfKeys = 128;                    // keys per tile: 8 paged blocks
constexpr int kPfHeadDim = 64;                  // one 128-byte swizzle row per key / query
constexpr int kPfTile = kPfKeys * kPfHeadDim * 2;  // one K or V tile: 16 KiB
constexpr int kPfStages = 2;
constexpr int kPfSoftmax = 256;  // two threads per query row, 64 key columns each
constexpr int kPfThreads = 64 + kPfSoftmax;
constexpr uint32_t kPfTmemCols = 256;  // S/P [0, 128), O [128, 192): two CTAs share an SM's 512
constexpr uint32_t kPfOCol = 128;

struct PfParams {
    const void* q;
    int q_row_stride;
    const void* q_bias;
    const int* block_tables;
    const int* seq_lens_pre;
    const int* q_start;
    const int* q_len;
    void* out;
    int out_row_stride;
    int qg;  // query heads per kv head
    int mbps, layer_idx, n_layer, num_blocks;
    int oob_slab;  // a slab index past the pool: boxes there read zeros
    float scale_log2;
};

// Shared-memory plan (bytes from the 1024-aligned base).
struct PfLayout {
    static constexpr int off_q = 0;                          // [128][64] K-major
    static constexpr int off_kv = off_q + kPfRows * 128;     // [stage][K | V]
    static constexpr int off_red = off_kv + kPfStages * 2 * kPfTile;  // [2 halves][128 rows] fp32
    static constexpr int off_bars = off_red + 2 * kPfRows * 4;
    static constexpr int n_bars = 2 * kPfStages + 4;  // kv_full, kv_empty, s_full, p_ready, o_done, done
    static constexpr int off_tmem = off_bars + 8 * n_bars;
    static constexpr int bytes = off_tmem + 16 + 1024;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) tmem_st8(taddr + static_cast<uint32_t>(i), v + i);
}

// Two 16-bit values in one 32-bit word (first in the low half) and back.
__device__ __forceinline__ uint32_t pf_pack2(__half, float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pf_pack2(__nv_bfloat16, float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 pf_unpack2(__half, uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
__device__ __forceinline__ float2 pf_unpack2(__nv_bfloat16, uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// Pass 2 of NK of one thread's keys: p = 2^(s * v - m_ref) (0 for masked keys
// when MASK), accumulated into ls, and written over those keys' S columns as
// hi = T(p) (first NK / 2 columns) and lo = T(p - hi) (next NK / 2).
template <typename T, bool MASK, int NK>
__device__ __forceinline__ void pf_weights(const float* v, float scale_log2, float m_ref, int kbase, int qpos,
                                           bool valid, uint32_t s_addr, float* ls) {
#pragma unroll
    for (int j = 0; j < NK; j += 8) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float pw[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int c = j + 2 * q + e;
                pw[e] = (!MASK || (valid && kbase + c <= qpos)) ? ex2_approx(fmaf(v[c], scale_log2, -m_ref)) : 0.0f;
                ls[(2 * q + e) & 7] += pw[e];
            }
            hw[q] = pf_pack2(T(), pw[0], pw[1]);
            const float2 h = pf_unpack2(T(), hw[q]);
            lw[q] = pf_pack2(T(), pw[0] - h.x, pw[1] - h.y);
        }
        tmem_st4u(s_addr + static_cast<uint32_t>(j / 2), make_uint4(hw[0], hw[1], hw[2], hw[3]));
        tmem_st4u(s_addr + static_cast<uint32_t>(NK / 2 + j / 2), make_uint4(lw[0], lw[1], lw[2], lw[3]));
    }
}

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 2)
    prefill_attn_tc_kernel(const PfParams p, const __grid_constant__ CUtensorMap kv_map) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // swizzled tiles need 1024-B alignment
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // grid (sequence, head, query tile) with the tile index reversed in the
    // slowest dimension: CTAs are dispatched in launch order, so the tiles with
    // the most keys (the last ones) start first and the short ones fill the tail
    const int b = static_cast<int>(blockIdx.x);
    const int h = static_cast<int>(blockIdx.y);
    const int i0 = static_cast<int>(gridDim.z - 1 - blockIdx.z) * kPfRows;

    pdl_launch_dependents();
    pdl_wait();  // q comes from the QKV product, the keys from the KV append before this launch
    const int T_len = __ldg(p.q_len + b);
    if (i0 >= T_len) return;  // CTA-uniform, before any barrier or TMEM use
    const int pre = __ldg(p.seq_lens_pre + b);
    const int nq = min(kPfRows, T_len - i0);  // query rows of this tile
    int kv_end = pre + i0 + nq;              // keys [0, kv_end) are read
    if (pre < 0 || kv_end > p.mbps * kBlockTokens) {
        if (tid == 0) flag_error(B2_DEVERR_SEQ_LEN);
        kv_end = max(1, min(kv_end, p.mbps * kBlockTokens));
    }
    const int ntiles = (kv_end + kPfKeys - 1) / kPfKeys;
    const int hk = h / p.qg;
    const size_t row0 = static_cast<size_t>(__ldg(p.q_start + b)) + i0;

    unsigned char* qbuf = smem + PfLayout::off_q;
    unsigned char* kv = smem + PfLayout::off_kv;
    uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + PfLayout::off_bars);
    uint64_t* kv_empty = kv_full + kPfStages;
    uint64_t* s_full = kv_empty + kPfStages;
    uint64_t* p_ready = s_full + 1;
    uint64_t* o_done = p_ready + 1;
    uint64_t* done_bar = o_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PfLayout::off_tmem);

    if (tid == 0) {
        for (int s = 0; s < kPfStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(p_ready, 1);
        mbar_init(o_done, 1);
        mbar_init(done_bar, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kPfTmemCols);
        tmem_relinquish();
    }
    // softmax threads: query row = their TMEM lane (warp w reads lanes 32 * (w % 4) ...),
    // key columns [64 * half, 64 * half + 64) of each tile
    const int row = 32 * (warp & 3) + lane;
    const int half = (warp - 2) >> 2;
    if (warp >= 2) {
        // Q row (+ bias, rounded to T as the reference's add_bias stores it), zeros past the tile;
        // each of the row's two threads writes 4 of its 8 16-byte chunks
        const T* qsrc = static_cast<const T*>(p.q) + (row0 + row) * static_cast<size_t>(p.q_row_stride) +
                        static_cast<size_t>(h) * kPfHeadDim;
        const T* bsrc = p.q_bias != nullptr ? static_cast<const T*>(p.q_bias) + h * kPfHeadDim : nullptr;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const int c = 4 * half + cc;
            uint4 raw = make_uint4(0u, 0u, 0u, 0u);
            if (row < nq) {
                raw = __ldg(reinterpret_cast<const uint4*>(qsrc) + c);
                if (bsrc != nullptr) {
                    float f[8], bf[8];
                    unpack16<T>(raw, f);
                    unpack16<T>(__ldg(reinterpret_cast<const uint4*>(bsrc) + c), bf);
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = __fadd_rn(f[e], bf[e]);
                    raw = pack16<T>(f);
                }
            }
            *reinterpret_cast<uint4*>(qbuf + sw128_offset(row, c * 8, 2)) = raw;
        }
        fence_proxy_async_smem();  // the tensor core reads Q through the async proxy
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued = 0;  // producer: ring fills issued
    if (warp == 0) {
        // ================================================= TMA producer
        if (lane == 0) {
            const int* bt = p.block_tables + static_cast<size_t>(b) * p.mbps;
            const int nblk = (kv_end + kBlockTokens - 1) / kBlockTokens;
            for (int t = 0; t < ntiles; ++t) {
                const int st = t % kPfStages;
                if (t >= kPfStages &&
                    !mbar_wait_bounded(&kv_empty[st], (static_cast<uint32_t>(t / kPfStages) & 1u) ^ 1u)) {
                    flag_error(B2_DEVERR_TIMEOUT);
                    break;
                }
                mbar_arrive_expect_tx(&kv_full[st], 2 * kPfTile);  // every box counts, zero-filled ones too
                unsigned char* kdst = kv + st * 2 * kPfTile;
                for (int j = 0; j < kPfKeys / kBlockTokens; ++j) {
                    const int kb = t * (kPfKeys / kBlockTokens) + j;
                    int slab = p.oob_slab;
                    if (kb < nblk) {
                        int blk = __ldg(bt + kb);
                        if (blk < 0 || blk >= p.num_blocks) {
                            flag_error(B2_DEVERR_BLOCK_ID);
                            blk = 0;
                        }
                        slab = (blk * p.n_layer + p.layer_idx) * 2;
                    }
                    tma_load_4d(kdst + j * 2048, &kv_map, 0, 0, hk, slab, &kv_full[st]);
                    tma_load_4d(kdst + kPfTile + j * 2048, &kv_map, 0, 0, hk, slab == p.oob_slab ? slab : slab + 1,
                                &kv_full[st]);
                }
                issued = t + 1;
            }
        }
    } else if (warp == 1) {
        // ================================================= MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC_S = umma_idesc<T>(kPfRows, kPfKeys, false, false);
            constexpr uint32_t IDESC_O = umma_idesc<T>(kPfRows, kPfHeadDim, false, true);
            const uint32_t qa = smem_addr(qbuf);
            // S(t) = Q . K(t)^T into the S/P columns once K(t) has landed; they held P(t - 1),
            // which PV(t - 1), issued before it, has read (one thread's MMAs run in order)
            auto issue_s = [&](int t) -> bool {
                const int st = t % kPfStages;
                if (!mbar_wait_bounded(&kv_full[st], static_cast<uint32_t>(t / kPfStages) & 1u)) return false;
                tc_fence_after();
                const uint32_t ka = smem_addr(kv + st * 2 * kPfTile);
#pragma unroll
                for (int k = 0; k < kPfHeadDim / 16; ++k)
                    umma_f16(tmem, sw128_desc(qa + 32 * k, 16, 1024), sw128_desc(ka + 32 * k, 16, 1024), IDESC_S,
                             k > 0);
                umma_commit(s_full);
                return true;
            };
            bool ok = issue_s(0);
            for (int t = 0; ok && t < ntiles; ++t) {
                if (!mbar_wait_bounded(p_ready, static_cast<uint32_t>(t) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t va = smem_addr(kv + (t % kPfStages) * 2 * kPfTile) + kPfTile;
#pragma unroll
                for (int kk = 0; kk < kPfKeys / 16; ++kk) {
                    // keys [16 kk, 16 kk + 16): in the 32-key chunk kk / 2, hi words then lo words
                    const uint32_t pa = tmem + static_cast<uint32_t>((kk >> 1) * 32 + (kk & 1) * 8);
                    const uint64_t vd = sw128_desc(va + static_cast<uint32_t>(kk) * 2048u, kPfTile, 1024);
                    umma_f16_ts(tmem + kPfOCol, pa, vd, IDESC_O, t > 0 || kk > 0);
                    umma_f16_ts(tmem + kPfOCol, pa + 16u, vd, IDESC_O, true);
                }
                umma_commit(o_done);
                umma_commit(&kv_empty[t % kPfStages]);
                if (t + 1 < ntiles && !(ok = issue_s(t + 1))) break;
            }
            if (!ok) flag_error(B2_DEVERR_TIMEOUT);
        }
    } else {
        // ================================================= softmax / epilogue
        constexpr int NS = kPfSoftmax;
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const uint32_t s_base = tmem + lane_base + static_cast<uint32_t>(64 * half);
        const uint32_t o_addr = tmem + lane_base + kPfOCol + static_cast<uint32_t>(32 * half);
        float* red = reinterpret_cast<float*>(smem + PfLayout::off_red);  // [half][row]
        const bool valid = row < nq;
        const int qpos = pre + i0 + row;
        float m_ref = -INFINITY, l = 0.0f;  // l: this thread's share of the row sum
        bool ok = true;
        for (int t = 0; t < ntiles; ++t) {
            ok = mbar_wait_bounded(s_full, static_cast<uint32_t>(t) & 1u);
            if (named_sync_or(1, NS, !ok)) {
                if (!ok) flag_error(B2_DEVERR_TIMEOUT);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t s_addr = s_base;
            const int kbase = t * kPfKeys + 64 * half;  // position of this thread's first key
            float v[32];  // 32 of this thread's 64 scores of the tile at a time
            // A tile whose last key precedes the tile's first query position is
            // visible to every row (CTA-uniform): no causal mask.  Rows past nq
            // then see S = 0 (their Q rows are zero) and are never stored.
            const bool open = (t + 1) * kPfKeys - 1 <= pre + i0;
            // pass 1: the maximum over this thread's visible keys, combined with the
            // other half's; scaled once (x -> x * s is monotonic for s > 0, so
            // max(v) * s == max(v * s) exactly)
            float mxs[8];  // independent partial maxima (no 64-long dependency chain)
#pragma unroll
            for (int e = 0; e < 8; ++e) mxs[e] = -INFINITY;
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                tmem_ld32(s_addr + static_cast<uint32_t>(32 * ch), v);
                if (open) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) mxs[j & 7] = fmaxf(mxs[j & 7], v[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (valid && kbase + 32 * ch + j <= qpos) mxs[j & 7] = fmaxf(mxs[j & 7], v[j]);
                }
            }
            float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                             fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]))) *
                       p.scale_log2;
            red[half * kPfRows + row] = mx;
            named_sync(2, NS);
            mx = fmaxf(mx, red[(half ^ 1) * kPfRows + row]);
            // move the reference maximum (always on a row's first keys, which are in
            // tile 0: key 0 is visible to every row); O rows are rescaled by all
            // threads together when any row moved (tcgen05.ld/st are warp-wide)
            const bool need = mx > m_ref + 8.0f;
            float corr = 1.0f;
            if (need) {
                corr = exp2f(m_ref - mx);
                l *= corr;
                m_ref = mx;
            }
            if (named_sync_or(4, NS, need) && t > 0) {
                // PV(t - 1) has finished: S(t), whose completion the softmax waited
                // for, was issued after it
                float o[32];
                tmem_ld32(o_addr, o);
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] *= corr;
                tmem_st32(o_addr, o);
                tmem_wait_st();
            }
            // pass 2: weights, split into two 16-bit halves, over this thread's S columns,
            // 32 keys at a time (each chunk's scores are re-read before its P overwrites them)
            float ls[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};  // partial sums
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                const uint32_t ca = s_addr + static_cast<uint32_t>(32 * ch);
                tmem_ld32(ca, v);
                if (open)
                    pf_weights<T, false, 32>(v, p.scale_log2, m_ref, kbase + 32 * ch, qpos, valid, ca, ls);
                else
                    pf_weights<T, true, 32>(v, p.scale_log2, m_ref, kbase + 32 * ch, qpos, valid, ca, ls);
            }
            tmem_wait_st();
            l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
            if (t == ntiles - 1 && half == 0 && t * kPfKeys + row >= kv_end) {
                // key row past the keys in use: zero its V (P is 0 there; V may be stale)
                uint4* vrow = reinterpret_cast<uint4*>(kv + (t % kPfStages) * 2 * kPfTile + kPfTile + row * 128);
#pragma unroll
                for (int c = 0; c < 8; ++c) vrow[c] = make_uint4(0u, 0u, 0u, 0u);
            }
            fence_proxy_async_smem();  // the zeroed V rows are read by the tensor core
            tc_fence_before();
            named_sync(3, NS);
            if (tid == 64) mbar_arrive(p_ready);
        }
        // ---- O / l for the tile's rows; each thread stores its 32 of the 64 dims
        // (every lane loads: tcgen05.ld is warp-wide)
        red[half * kPfRows + row] = l;
        // PV(ntiles - 1) done (PV(ntiles - 2) is: S(ntiles - 1) was issued after it)
        const bool fin = ok && mbar_wait_bounded(o_done, static_cast<uint32_t>(ntiles - 1) & 1u);
        if (!named_sync_or(5, NS, !fin)) {
            tc_fence_after();
            const float lt = l + red[(half ^ 1) * kPfRows + row];
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
            T* dst = static_cast<T*>(p.out) + (row0 + row) * static_cast<size_t>(p.out_row_stride) +
                     static_cast<size_t>(h) * kPfHeadDim + 32 * half;
            float o[32];
            tmem_ld32(o_addr, o);
            if (valid) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) f[e] = o[j + e] * inv;
                    *reinterpret_cast<uint4*>(dst + j) = pack16<T>(f);
                }
            }
        } else if (ok) {
            flag_error(B2_DEVERR_TIMEOUT);
        }
        tc_fence_before();
    }

    // ---- common exit: copies landed, MMAs done, TMEM freed
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kPfStages && s < issued; ++s) {
            const int last_use = (issued - 1 - s) / kPfStages;
            if (!mbar_wait_bounded(&kv_full[s], static_cast<uint32_t>(last_use) & 1u)) flag_error(B2_DEVERR_TIMEOUT);
        }
    }
    if (warp == 1 && lane == 0) {
        umma_commit(done_bar);
        if (!mbar_wait_bounded(done_bar, 0)) flag_error(B2_DEVERR_TIMEOUT);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kPfTmemCols);
}

}  // namespace b2
