// attention.cuh -- paged decode attention for sm_100a.
//
// Computes what gpu-engine/src/kernels/attention.cu:49-127 computes
// (softmax(q.K^T * scale) V over the block-table KV cache, fp32 softmax
// state), organised for B200 instead of one CTA per (batch, head):
//
//  * Work split.  Every sequence b owns nb_b = ceil(seq_len_b / 16) paged
//    blocks.  All blocks of all sequences form one list of N units, and CTA i
//    of the G = min(grid, N) working CTAs (one per SM) takes units
//    [i*N/G, (i+1)*N/G).  The split is even whatever the length skew, and a
//    sequence may be cut into segments handled by several CTAs
//    (flash-decoding split-K with split points chosen by load).
//  * Data movement.  For one layer, a block's K rows of ALL kv heads are one
//    contiguous slab of 16*n_kv_head*head_dim elements (layout
//    [block][layer][K|V][16][n_kv_head][head_dim], kv_cache.h:6-7), with the V
//    slab right behind it.  A producer warp streams each unit's K and V slabs
//    (only the valid token rows) with 1-D bulk async copies (cp.async.bulk,
//    the TMA engine's untiled path) into a ring of shared-memory stages
//    guarded by mbarriers; q rows travel the same way at a segment's first
//    block.  Consumer warps never read K/V from global memory.
//  * Math.  Consumer thread (ts, c) owns 16-byte chunk c of the token row
//    (kv head c / GL, dims (c % GL) * E ...) and the tokens t = ts (mod k) of
//    every block.  The GL lanes that share a head row form a group that
//    reduces q.k with xor shuffles and keeps that head's online-softmax state
//    (m, l) and its slice of the accumulator in registers, rescaling once per
//    batch of up to four tokens.  No CTA-wide barrier is needed per block:
//    warps only meet at the stage mbarriers, and at a segment's end, where the
//    k token subgroups are merged through shared memory.
//  * Merge.  A sequence finished inside one CTA is normalised and written
//    directly.  Otherwise each CTA writes (m, l, acc) to the workspace, bumps
//    the sequence's counter, and the CTA that arrives last merges all
//    partials and resets the counter to zero (no CTA ever waits for another).
//
// Every wait is bounded (b2_common.cuh): on timeout the CTA flags
// B2_DEVERR_TIMEOUT, drains its own copies in flight and returns.
#pragma once

#include "b2_common.cuh"

namespace b2 {

struct AttnParams {
    const void* q;
    long long q_row_stride;  // elements
    const void* q_bias;
    const void* pool;
    const int* block_tables;
    const int* seq_lens;
    void* out;
    int batch, n_head, n_kv_head, mbps, layer_idx, n_layer, num_blocks;
    float scale_log2;  // scale * log2(e)
    int ksplit;        // token subgroups per block (1, 2 or 4)
    int ncons;         // consumer threads, multiple of 32
    int stages;
    int stage_bytes;
    int slab_bytes;  // 16 * n_kv_head * head_dim * sizeof(T)
    int q_bytes;     // n_head * head_dim * sizeof(T)
    int off_meta;    // within a stage
    int off_scratch, off_misc, off_bars;
    unsigned int* counters;  // [batch] merge counters, zero between launches
    float2* part_ml;         // [grid + batch][n_head] (m, l)
    float* part_acc;         // [grid + batch][n_head][head_dim]
};

// Largest working-CTA index whose range start floor(i*N/G) is <= u.  With
// G <= N every working CTA owns at least one unit.
__device__ __forceinline__ int cta_of_unit(long long u, long long N, int G) {
    return static_cast<int>(((u + 1) * G - 1) / N);
}

__device__ __forceinline__ int clamp_seq_len(int c, int mbps) {
    return c < 0 ? 0 : (c > mbps * kBlockTokens ? mbps * kBlockTokens : c);
}

// Exclusive scan of v over all threads of the CTA; *total gets the sum.
// warp_sums needs 33 ints of shared memory.  Contains __syncthreads.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    int incl = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? warp_sums[lane] : 0;
        int wi = w;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, off);
            if (lane >= off) wi += y;
        }
        warp_sums[lane] = wi - w;  // exclusive prefix of warp totals
        if (lane == 31) warp_sums[32] = wi;
    }
    __syncthreads();
    *total = warp_sums[32];
    return warp_sums[warp] + incl - v;
}

template <typename T, int DH, int QG, typename OutT, int MAXT>
__global__ void __launch_bounds__(MAXT, 1) paged_decode_kernel(const AttnParams p) {
    constexpr int E = Elem<T>::kPer16B;
    constexpr int GL = DH / E;  // lanes sharing one head row
    static_assert(GL >= 2 && GL <= 32 && (32 % GL) == 0, "head_dim / dtype combination");
    constexpr int ES = static_cast<int>(sizeof(T));
    constexpr int TB = 4;           // tokens per online-softmax rescale
    constexpr int kMaxPending = 16;  // deferred hand-offs per CTA before a flush

    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int H = p.n_head;
    const int Hkv = p.n_kv_head;
    const int C = Hkv * GL;  // 16-byte chunks per token row (all kv heads)
    const int cta = blockIdx.x;
    const int B = p.batch;
    const int S = p.stages;

    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    uint64_t* empty = full + S;
    // misc (512 B): [0..1] first sequence and its prefix, [2..34] scan, [40] pending count, [48..111] pending list
    int* misc = reinterpret_cast<int*>(smem + p.off_misc);
    float* sScratch = reinterpret_cast<float*>(smem + p.off_scratch);

    uint64_t* segbar = empty + S;  // consumer-wide sync at segment ends
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], static_cast<uint32_t>(p.ncons / 32));
        }
        mbar_init(segbar, static_cast<uint32_t>(p.ncons));
        misc[40] = 0;
        fence_mbar_init();
    }

    // Programmatic dependent launch: let the next kernel in the stream start
    // its own prologue as our CTAs retire, and wait here until the kernels
    // before us (which produce q, the pool and seq_lens) have completed.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // ---- prologue: per-sequence block counts, global prefix, this CTA's range
    const int per =(B + static_cast<int>(blockDim.x) - 1) / static_cast<int>(blockDim.x);
    const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
    int local = 0;
    for (int b = b_lo; b < b_hi; ++b) local += (clamp_seq_len(__ldg(p.seq_lens + b), p.mbps) + 15) >> 4;
    int N = 0;
    const int excl = block_exclusive_scan(local, misc + 2, &N);
    const int G = min(static_cast<int>(gridDim.x), max(N, 1));
    const long long s_unit = cta < G ? static_cast<long long>(cta) * N / G : 0;
    const long long e_unit = cta < G ? static_cast<long long>(cta + 1) * N / G : 0;
    {
        int run = excl;
        for (int b = b_lo; b < b_hi; ++b) {
            const int raw = __ldg(p.seq_lens + b);
            const int cl = clamp_seq_len(raw, p.mbps);
            const int nb = (cl + 15) >> 4;
            if (nb > 0 && run <= s_unit && s_unit < run + nb) {
                misc[0] = b;
                misc[1] = run;
            }
            run += nb;
            if (b % static_cast<int>(gridDim.x) == cta) {
                if (raw != cl) flag_error(B2_DEVERR_SEQ_LEN);
                if (nb == 0) {  // no keys: the reference writes 0 (l == 0)
                    OutT* o = reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(b) * H * DH;
                    for (int i = 0; i < H * DH; ++i) o[i] = Elem<OutT>::from_f(0.0f);
                }
            }
        }
    }
    __syncthreads();
    const int nunits = static_cast<int>(e_unit - s_unit);
    if (nunits <= 0) return;

    const size_t row_elems = static_cast<size_t>(Hkv) * DH;
    const size_t slab_elems = row_elems * kBlockTokens;
    const int row_bytes = static_cast<int>(row_elems) * ES;

    if (tid >= p.ncons) {
        // ================================================= producer warp
        const int lane = tid & 31;
        const char* pool = static_cast<const char*>(p.pool);
        const size_t block_elems = static_cast<size_t>(p.n_layer) * 2 * slab_elems;
        const size_t layer_off = static_cast<size_t>(p.layer_idx) * 2 * slab_elems;
        long long u = s_unit;
        int bb = misc[0];
        long long Pb = misc[1];
        int n = 0;
        bool failed = false;
        while (u < e_unit && !failed && bb < B) {
            const int b = bb + lane;
            int cl = 0;
            if (b < B) cl = clamp_seq_len(__ldg(p.seq_lens + b), p.mbps);
            const int nbl = (cl + 15) >> 4;
            int incl = nbl;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += y;
            }
            const int wtotal = __shfl_sync(0xffffffffu, incl, 31);
            for (int sidx = 0; sidx < 32 && u < e_unit && !failed; ++sidx) {
                const int nbs = __shfl_sync(0xffffffffu, nbl, sidx);
                const int cs = __shfl_sync(0xffffffffu, cl, sidx);
                const long long Ps = Pb + __shfl_sync(0xffffffffu, incl - nbl, sidx);
                const int bs = bb + sidx;
                if (nbs == 0 || Ps + nbs <= u) continue;
                const int j0 = static_cast<int>(u - Ps);
                const int j1 = static_cast<int>(min(e_unit, Ps + nbs) - Ps);
                const int i0 = cta_of_unit(Ps, N, G);
                const int nseg = cta_of_unit(Ps + nbs - 1, N, G) - i0 + 1;
                for (int jc = j0; jc < j1 && !failed; jc += 32) {
                    const int jj = jc + lane;
                    int blk_l = 0;
                    if (jj < j1) {
                        blk_l = __ldg(p.block_tables + static_cast<size_t>(bs) * p.mbps + jj);
                        if (blk_l < 0 || blk_l >= p.num_blocks) {
                            flag_error(B2_DEVERR_BLOCK_ID);
                            blk_l = 0;
                        }
                    }
                    const int cnt = min(32, j1 - jc);
                    for (int x = 0; x < cnt; ++x) {
                        const int blk = __shfl_sync(0xffffffffu, blk_l, x);
                        int ok = 1;
                        if (lane == 0) {
                            const int st = n % S;
                            const uint32_t ph = static_cast<uint32_t>(n / S) & 1u;
                            if (!mbar_wait_bounded(&empty[st], ph ^ 1u)) {
                                ok = 0;
                            } else {
                                const int j = jc + x;
                                const int ntok = min(kBlockTokens, cs - j * kBlockTokens);
                                const int first = (j == j0) ? 1 : 0;
                                const int lastf = (j == j1 - 1) ? 2 : 0;
                                unsigned char* stage = smem + static_cast<size_t>(st) * p.stage_bytes;
                                *reinterpret_cast<int4*>(stage + p.off_meta) =
                                    make_int4(bs, ntok | ((first | lastf) << 8), nseg, i0);
                                const uint32_t kv_bytes = static_cast<uint32_t>(ntok * row_bytes);
                                mbar_arrive_expect_tx(&full[st], 2u * kv_bytes + (first ? p.q_bytes : 0));
                                const char* src = pool + (static_cast<size_t>(blk) * block_elems + layer_off) * ES;
                                bulk_g2s(stage, src, kv_bytes, &full[st]);
                                bulk_g2s(stage + p.slab_bytes, src + slab_elems * ES, kv_bytes, &full[st]);
                                if (first) {
                                    const char* qsrc = static_cast<const char*>(p.q) +
                                                       static_cast<size_t>(bs) * p.q_row_stride * ES;
                                    bulk_g2s(stage + 2 * p.slab_bytes, qsrc, static_cast<uint32_t>(p.q_bytes),
                                             &full[st]);
                                }
                            }
                        }
                        ok = __shfl_sync(0xffffffffu, ok, 0);
                        if (!ok) {
                            failed = true;
                            break;
                        }
                        ++n;
                    }
                }
                u = Ps + j1;
            }
            bb += 32;
            Pb += wtotal;
        }
        if (lane == 0) {
            if (failed) flag_error(B2_DEVERR_TIMEOUT);
            // Never leave with copies in flight: wait (bounded) for the last
            // issue of every stage to land.
            for (int m = max(0, n - S); m < n; ++m)
                if (!mbar_wait_bounded(&full[m % S], static_cast<uint32_t>(m / S) & 1u))
                    flag_error(B2_DEVERR_TIMEOUT);
        }
        return;
    }

    // ===================================================== consumer threads
    const int ncons = p.ncons;
    const int ks = p.ksplit;
    (void)ncons;
    const int ts = tid / C;
    const int c = tid - ts * C;
    const bool active = ts < ks;
    const int hk = c / GL;
    const int dg = c - hk * GL;
    const int lane = tid & 31;
    const unsigned gmask = (GL == 32) ? 0xffffffffu : (((1u << GL) - 1u) << (lane & ~(GL - 1)));
    // All consumer threads meet on segbar (bounded): returns false on timeout.
    uint32_t seg_parity = 0;
    auto consumers_sync = [&]() -> bool {
        mbar_arrive(segbar);
        const bool ok = mbar_wait_bounded(segbar, seg_parity);
        seg_parity ^= 1u;
        return !__any_sync(0xffffffffu, !ok);
    };

    OutT* const out_ptr = static_cast<OutT*>(p.out);
    // Sequences whose partial this CTA wrote but has not yet reported
    // (b, nseg, i0, last-flag).  Reporting is batched: one fence and atomic
    // per entry at the end of the range instead of a stall per segment.
    int* npend_s = misc + 40;
    int4* pend = reinterpret_cast<int4*>(misc + 48);

    // Combines the nseg partials of sequence b (workspace slots i0 + s + b)
    // and writes its output; all consumer threads take part.
    auto merge_sequence = [&](int b, int nseg, int i0) {
        for (int idx = tid; idx < H * GL; idx += ncons) {
            const int h = idx / GL;
            const int dc = idx - h * GL;
            float mmax = -INFINITY;
            for (int s2 = 0; s2 < nseg; ++s2)
                mmax = fmaxf(mmax, __ldcg(p.part_ml + static_cast<size_t>(i0 + s2 + b) * H + h).x);
            float l = 0.0f;
            float a[E];
#pragma unroll
            for (int e = 0; e < E; ++e) a[e] = 0.0f;
            for (int s2 = 0; s2 < nseg; ++s2) {
                const size_t sl = static_cast<size_t>(i0 + s2 + b);
                const float2 ml = __ldcg(p.part_ml + sl * H + h);
                const float w = exp2f(ml.x - mmax);
                l = fmaf(ml.y, w, l);
                const float* src = p.part_acc + (sl * H + h) * DH + dc * E;
#pragma unroll
                for (int e = 0; e < E; e += 4) {
                    const float4 v4 = __ldcg(reinterpret_cast<const float4*>(src + e));
                    a[e] = fmaf(v4.x, w, a[e]);
                    a[e + 1] = fmaf(v4.y, w, a[e + 1]);
                    a[e + 2] = fmaf(v4.z, w, a[e + 2]);
                    a[e + 3] = fmaf(v4.w, w, a[e + 3]);
                }
            }
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
            for (int e = 0; e < E; ++e) a[e] *= inv;
            store_row<OutT, E>(out_ptr + (static_cast<size_t>(b) * H + h) * DH + dc * E, a);
        }
    };

    // Reports every pending partial: after the CTA-wide sync that ordered all
    // partial writes, one thread per entry fences at gpu scope (cumulative over
    // the CTA's writes) and bumps the sequence's counter; the CTA that brings a
    // counter to nseg merges that sequence and resets the counter to zero.
    auto flush_pending = [&]() -> bool {
        const int np = npend_s[0];
        if (np == 0) return true;
        for (int j = tid; j < np; j += ncons) {
            const int4 e = pend[j];
            __threadfence();
            const unsigned int prev = atomicAdd(p.counters + e.x, 1u);
            const bool is_last = prev == static_cast<unsigned int>(e.y - 1);
            if (is_last) __threadfence();
            pend[j].w = is_last ? 1 : 0;
        }
        if (!consumers_sync()) {
            if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
            return false;
        }
        for (int j = 0; j < np; ++j) {
            const int4 e = pend[j];
            if (!e.w) continue;
            merge_sequence(e.x, e.y, e.z);
            if (tid == 0) p.counters[e.x] = 0u;
        }
        if (tid == 0) npend_s[0] = 0;
        if (!consumers_sync()) {
            if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
            return false;
        }
        return true;
    };

    uint4 qraw[QG];  // this thread's q chunks, in the storage dtype (bias added)
    float acc[QG][E];
    float m_run[QG];
    float l_run[QG];
#pragma unroll
    for (int g = 0; g < QG; ++g) {
        qraw[g] = make_uint4(0u, 0u, 0u, 0u);
        m_run[g] = -INFINITY;
        l_run[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] = 0.0f;
    }
    const float scale_log2 = p.scale_log2;

    OutT* out = static_cast<OutT*>(p.out);
    for (int n = 0; n < nunits; ++n) {
        const int st = n % S;
        const uint32_t ph = static_cast<uint32_t>(n / S) & 1u;
        unsigned char* stage = smem + static_cast<size_t>(st) * p.stage_bytes;
        // A warp that gives up leaves the kernel as a whole (warp-uniform
        // decision); the others then time out on their own bounded waits.
        if (__any_sync(0xffffffffu, !mbar_wait_bounded(&full[st], ph))) {
            if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
            return;
        }
        const int4 meta = *reinterpret_cast<const int4*>(stage + p.off_meta);
        const int b = meta.x;
        const int ntok = min(meta.y & 0xff, kBlockTokens);
        const bool first = (meta.y >> 8) & 1;
        const bool last = (meta.y >> 9) & 1;

        if (active) {
            if (first) {
                const unsigned char* qs = stage + 2 * p.slab_bytes;
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    qraw[g] = ld_shared16(qs + ((hk * QG + g) * DH + dg * E) * ES);
                    if (p.q_bias != nullptr) {
                        // q + bias rounded to T, as the reference's separate
                        // add_bias launch stores it (engine.cu:158).
                        float f[E], bf[E];
                        unpack16<T>(qraw[g], f);
                        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.q_bias) +
                                                                         (hk * QG + g) * DH + dg * E)),
                                    bf);
#pragma unroll
                        for (int e = 0; e < E; ++e) f[e] = __fadd_rn(f[e], bf[e]);
                        qraw[g] = pack16<T>(f);
                    }
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[g][e] = 0.0f;
                    m_run[g] = -INFINITY;
                    l_run[g] = 0.0f;
                }
            }
            const unsigned char* K = stage;
            const unsigned char* V = stage + p.slab_bytes;
            for (int t0 = ts; t0 < ntok; t0 += TB * ks) {
                const int cnt = min(TB, (ntok - t0 + ks - 1) / ks);  // same for the whole lane group
                float s[TB][QG];
#pragma unroll
                for (int j = 0; j < TB; ++j) {
                    if (j < cnt) {
                        const uint4 kraw = ld_shared16(K + ((t0 + j * ks) * C + c) * 16);
#pragma unroll
                        for (int g = 0; g < QG; ++g) s[j][g] = dot16<T>(qraw[g], kraw, 0.0f);
                    } else {
#pragma unroll
                        for (int g = 0; g < QG; ++g) s[j][g] = 0.0f;
                    }
                }
#pragma unroll
                for (int off = GL / 2; off > 0; off >>= 1)
#pragma unroll
                    for (int j = 0; j < TB; ++j)
#pragma unroll
                        for (int g = 0; g < QG; ++g) s[j][g] += __shfl_xor_sync(gmask, s[j][g], off);
#pragma unroll
                for (int j = 0; j < TB; ++j)
#pragma unroll
                    for (int g = 0; g < QG; ++g) s[j][g] *= scale_log2;  // (q.k) * scale, in log2 units
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    float mx = m_run[g];
#pragma unroll
                    for (int j = 0; j < TB; ++j)
                        if (j < cnt) mx = fmaxf(mx, s[j][g]);
                    const float corr = exp2f(m_run[g] - mx);  // 0 on the first batch (m_run = -inf)
                    m_run[g] = mx;
                    l_run[g] *= corr;
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[g][e] *= corr;
                }
#pragma unroll
                for (int j = 0; j < TB; ++j) {
                    if (j < cnt) {
                        const uint4 vraw = ld_shared16(V + ((t0 + j * ks) * C + c) * 16);
#pragma unroll
                        for (int g = 0; g < QG; ++g) {
                            const float pw = exp2f(s[j][g] - m_run[g]);
                            l_run[g] += pw;
                            axpy16<T>(pw, vraw, acc[g]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);

        if (!last) continue;

        // ---- segment end: merge the k token subgroups, then write or hand off
        const int nseg = meta.z;
        const int i0 = meta.w;
        const bool single = nseg == 1;
        const int slot = cta + b;
        if (ks > 1) {
            float* sacc = sScratch;                                          // [ks][H][DH]
            float* sml = sScratch + static_cast<size_t>(ks) * H * DH;        // [ks][H][2]
            if (active) {
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    float* dst = sacc + (static_cast<size_t>(ts) * H + hk * QG + g) * DH + dg * E;
#pragma unroll
                    for (int e = 0; e < E; ++e) dst[e] = acc[g][e];
                    if (dg == 0) {
                        sml[(ts * H + hk * QG + g) * 2] = m_run[g];
                        sml[(ts * H + hk * QG + g) * 2 + 1] = l_run[g];
                    }
                }
            }
            if (!consumers_sync()) {
                if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
                return;
            }
            for (int idx = tid; idx < H * GL; idx += ncons) {
                const int h = idx / GL;
                const int dc = idx - h * GL;
                float mmax = -INFINITY;
                for (int s2 = 0; s2 < ks; ++s2) mmax = fmaxf(mmax, sml[(s2 * H + h) * 2]);
                float a[E], l = 0.0f;
#pragma unroll
                for (int e = 0; e < E; ++e) a[e] = 0.0f;
                for (int s2 = 0; s2 < ks; ++s2) {
                    const float ms = sml[(s2 * H + h) * 2];
                    const float w = ms == -INFINITY ? 0.0f : exp2f(ms - mmax);  // a subgroup may have had no tokens
                    l = fmaf(sml[(s2 * H + h) * 2 + 1], w, l);
                    const float* src = sacc + (static_cast<size_t>(s2) * H + h) * DH + dc * E;
#pragma unroll
                    for (int e = 0; e < E; ++e) a[e] = fmaf(src[e], w, a[e]);
                }
                if (single) {
                    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
                    for (int e = 0; e < E; ++e) a[e] *= inv;
                    store_row<OutT, E>(out + (static_cast<size_t>(b) * H + h) * DH + dc * E, a);
                } else {
                    float* dst = p.part_acc + (static_cast<size_t>(slot) * H + h) * DH + dc * E;
#pragma unroll
                    for (int e = 0; e < E; e += 4)
                        __stcg(reinterpret_cast<float4*>(dst + e), make_float4(a[e], a[e + 1], a[e + 2], a[e + 3]));
                    if (dc == 0) __stcg(p.part_ml + static_cast<size_t>(slot) * H + h, make_float2(mmax, l));
                }
            }
        } else if (active) {
#pragma unroll
            for (int g = 0; g < QG; ++g) {
                const int h = hk * QG + g;
                if (single) {
                    const float inv = l_run[g] > 0.0f ? 1.0f / l_run[g] : 0.0f;
                    float a[E];
#pragma unroll
                    for (int e = 0; e < E; ++e) a[e] = acc[g][e] * inv;
                    store_row<OutT, E>(out + (static_cast<size_t>(b) * H + h) * DH + dg * E, a);
                } else {
                    float* dst = p.part_acc + (static_cast<size_t>(slot) * H + h) * DH + dg * E;
#pragma unroll
                    for (int e = 0; e < E; e += 4)
                        __stcg(reinterpret_cast<float4*>(dst + e),
                               make_float4(acc[g][e], acc[g][e + 1], acc[g][e + 2], acc[g][e + 3]));
                    if (dg == 0) __stcg(p.part_ml + static_cast<size_t>(slot) * H + h, make_float2(m_run[g], l_run[g]));
                }
            }
        }
        if (!single && tid == 0) {
            // Hand-off deferred to the end of this CTA's range (or to a flush
            // when the list is full): the partial is written, the arrival is not.
            pend[npend_s[0]] = make_int4(b, nseg, i0, 0);
            npend_s[0] += 1;
        }
        // The scratch (and the pending list's count) are reused at the next segment end.
        if ((ks > 1 || !single) && !consumers_sync()) {
            if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
            return;
        }
        if (npend_s[0] == kMaxPending && !flush_pending()) return;
    }
    flush_pending();
}

}  // namespace b2
