// attention.cuh -- paged decode attention for sm_100a.
//
// Computes what gpu-engine/src/kernels/attention.cu:49-127 computes
// (softmax(q.K^T * scale) V over the block-table KV cache, fp32 softmax
// state), organised for B200 instead of one CTA per (batch, head):
//
//  * Work split.  The keys of all sequences form one list of N token rows
//    (sequence after sequence), and CTA i of the G = min(grid, N) working
//    CTAs (one or two per SM) takes rows [i*N/G, (i+1)*N/G).  Every CTA
//    streams the same number of bytes whatever the length skew; a sequence
//    may be cut into segments handled by several CTAs (flash-decoding split-K
//    with the split points chosen by load, down to single token rows).
//  * Data movement.  For one layer, a block's K rows of ALL kv heads are one
//    contiguous slab of 16*n_kv_head*head_dim elements (layout
//    [block][layer][K|V][16][n_kv_head][head_dim], kv_cache.h:6-7), with the V
//    slab right behind it, so any run of rows of one block is contiguous.  A
//    producer warp streams each block's run of rows (K and V) with 1-D bulk
//    async copies (cp.async.bulk, the TMA engine's untiled path) into a ring
//    of shared-memory stages guarded by mbarriers; q rows travel the same way
//    at a segment's first block.  Consumer warps never read K/V from global memory.
//  * Math.  Consumer thread (ts, c) owns one or two consecutive 16-byte
//    chunks of the token row (two for 16-bit types) and the tokens
//    t = ts (mod k) of every block.  The lanes that share a head row form a group that
//    reduces q.k with xor shuffles (16-bit operands go straight into fp32
//    FMAs, see dot16) and keeps that head's online-softmax state (m, l) and
//    its slice of the accumulator in registers, rescaling once per batch of
//    up to four tokens.  Warps meet only at the stage mbarriers.
//  * Merge.  At a segment's end the token subgroups' (m, l, acc) go to the
//    workspace -- one slot per subgroup, or, where the planner folds pieces
//    (one CTA per SM), one slot per piece after a fold in shared memory -- and
//    the piece goes to the CTA's bookkeeping warp.  The CTA holding a
//    sequence's last piece (its own first piece) merges the sequence at its
//    end; every other piece is published with one fire-and-forget release-add
//    on the sequence's counter, so those CTAs never wait for an answer.  The
//    merging CTA's bookkeeping warp waits (bounded, acquire loads) for the
//    count, then all its softmax threads merge the slots (max-rescaled sums,
//    in slot order) and write the output in the output dtype.  A sequence
//    that lies in one CTA is folded in shared memory and written out
//    directly.  One kernel per call; the counters are left at zero for the
//    next launch.
//
// Every wait is bounded (b2_common.cuh): on timeout the CTA flags
// B2_DEVERR_TIMEOUT, drains its own copies in flight and returns.
#pragma once

#include "b2_common.cuh"

namespace b2 {

// Where attention outputs go.  n == 0: one packed [batch, n_head, head_dim]
// array at `out`.  n > 0: the same values are stored into each of the n
// arrays outs[0..n) (this GPU's memory or a peer's, through its UVA
// address), row b at b * row_stride + col_offset elements -- so a
// head-sharded rank writes its heads' slice of every rank's gathered
// attention output directly (the all-gather happens in the epilogue).
struct OutSpec {
    void* out;
    void* const* outs;  // device array of n bases
    int n;
    long long row_stride, col_offset;
};

template <typename OutT, int E>
__device__ __forceinline__ void store_out(const OutSpec& o, int b, int H, int h, int DH, int dc, const float* a) {
    if (o.n == 0) {
        store_row<OutT, E>(static_cast<OutT*>(o.out) + (static_cast<size_t>(b) * H + h) * DH + dc * E, a);
        return;
    }
    const long long off = static_cast<long long>(b) * o.row_stride + o.col_offset + static_cast<long long>(h) * DH +
                          static_cast<long long>(dc) * E;
    for (int i = 0; i < o.n; ++i) store_row<OutT, E>(static_cast<OutT*>(o.outs[i]) + off, a);
    __threadfence_system();  // peers read these after the next barrier
}

struct AttnParams {
    const void* q;
    long long q_row_stride;  // elements
    const void* q_bias;
    const void* pool;
    const int* block_tables;
    const int* seq_lens;
    int batch, n_head, n_kv_head, mbps, layer_idx, n_layer, num_blocks;
    float scale_log2;  // scale * log2(e)
    int ksplit;        // token subgroups per block
    int ncons;         // consumer threads, multiple of 32
    int stages;
    int stage_bytes;
    int stage_rows;  // key rows a stage holds at most: 16 (a block), 8 or 4
    int slab_bytes;  // stage_rows * n_kv_head * head_dim * sizeof(T): K (then V) capacity of a stage
    int q_bytes;     // n_head * head_dim * sizeof(T)
    int off_meta;    // within a stage
    int off_misc, off_bars;
    int off_seqlens;  // >= 0: shared int[batch] holding the clamped seq_lens (the producer's copy); -1: none
    int fold_pieces;  // with local_merge: every piece's subgroups are folded in shared memory (one slot per piece)
    int spec_blocks;  // flags 0: paged blocks of the CTA's range the speculative pass prefetches into L2 (<= 31)
    int off_stash;    // >= 0 (early start only): shared [sk][H][head_dim] fp32 + [sk][H] (m, l), sk = fold_pieces ? 1
                      // : ksplit, holding the CTA's first mid-range piece until the bookkeeping warp writes it out
    int2* seq_info;   // [batch] (first CTA, number of segments) for the combine kernel
    float2* part_ml;  // [(grid + batch) * ksplit][n_head] (m, l); fold_pieces: one slot per piece
    float* part_acc;  // [(grid + batch) * ksplit][n_head][head_dim]
    unsigned int* counters;  // [batch] pieces finished per sequence; zero between launches
    OutSpec out;
    int early;  // 0 wait first; 1 inputs complete; 2 only each sequence's newest row pending
    int local_merge;  // 1: a sequence whose rows all lie in one CTA is merged there, in shared memory
};

struct CombineParams {
    const int2* seq_info;
    const float2* part_ml;
    const float* part_acc;
    OutSpec out;
    int n_head, ksplit;
};

// Largest working-CTA index whose range start floor(i*N/G) is <= u.  With
// G <= N every working CTA owns at least one row.
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

// Merges the partials (m, l, acc) of sequence b -- slots (i0 + b) * sk ...
// (i0 + nseg + b) * sk - 1, sk per (CTA, sequence) piece -- with a running
// maximum and writes out[b] in OutT.  Each (head, E-element chunk) item is
// taken by TPI adjacent threads, each folding E / TPI of its elements over
// all slots in slot order (the (m, l) fold is repeated in each).  So the
// result is the same to the bit whatever TPI is, and every merging path (the
// bookkeeping warp at TPI 1, the softmax threads at up to 4) writes the same
// bits: a launch is deterministic although which CTA merges a sequence can
// depend on timing.  The loads of SB slots are issued together (one L2 round
// trip per SB slots).  A partial that saw no rows has l == 0 and is skipped.
// Partials are read through L2 (__ldcg): other CTAs wrote them.  nthr must
// be a multiple of 32 and tid / nthr cover whole warps.
__device__ __forceinline__ void fold_state(float& m, float& l, float* a, int E, float m2, float l2, const float* a2) {
    if (!(l2 > 0.0f)) return;
    const float mn = fmaxf(m, m2);
    const float wo = exp2f(m - mn);  // 0 while m is -inf
    const float wn = exp2f(m2 - mn);
    m = mn;
    l = fmaf(l2, wn, l * wo);
    for (int e = 0; e < E; ++e) a[e] = fmaf(a2[e], wn, a[e] * wo);
}

// EP consecutive floats from global memory through L2, EP in {1, 2, 4, 8}.
template <int EP>
__device__ __forceinline__ void ldcg_floats(const float* src, float* d) {
    if constexpr (EP == 1) {
        d[0] = __ldcg(src);
    } else if constexpr (EP == 2) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(src));
        d[0] = v.x;
        d[1] = v.y;
    } else {
#pragma unroll
        for (int q = 0; q < EP / 4; ++q) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src) + q);
            d[4 * q] = v.x;
            d[4 * q + 1] = v.y;
            d[4 * q + 2] = v.z;
            d[4 * q + 3] = v.w;
        }
    }
}

template <int DH, int E, int TPI, typename OutT>
__device__ __forceinline__ void merge_partials(const float2* part_ml, const float* part_acc, const OutSpec& out, int H,
                                               int sk, int b, int i0, int nseg, int tid, int nthr) {
    constexpr int GL = DH / E;
    constexpr int EP = E / TPI;  // elements per thread
    constexpr int SB = 8;  // slots in flight per thread (more spill in the wider instantiations)
    static_assert(E % TPI == 0 && (EP == 1 || EP == 2 || EP % 4 == 0), "threads per merge item");
    const int nslots = nseg * sk;
    const size_t slot0 = (static_cast<size_t>(i0) + b) * sk;
    const int items = H * GL;
    const int per_round = nthr / TPI;
    const int sub = tid % TPI;
    const int iters = (items + per_round - 1) / per_round;  // the same for every thread (full-warp shuffles)
    for (int it = 0; it < iters; ++it) {
        const int item = tid / TPI + it * per_round;
        const bool valid = item < items;
        const int h = valid ? item / GL : 0;
        const int dc = valid ? item - h * GL : 0;
        float mrun = -INFINITY, l = 0.0f, a[EP];
#pragma unroll
        for (int e = 0; e < EP; ++e) a[e] = 0.0f;
        for (int s0 = 0; s0 < nslots; s0 += SB) {
            float2 ml[SB];
            float v[SB][EP];
#pragma unroll
            for (int j = 0; j < SB; ++j) {
                const int s = s0 + j;
                ml[j] = make_float2(-INFINITY, 0.0f);
                if (valid && s < nslots) {
                    const size_t sl = slot0 + s;
                    ml[j] = __ldcg(part_ml + sl * H + h);
                    ldcg_floats<EP>(part_acc + (sl * H + h) * DH + dc * E + sub * EP, v[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < SB; ++j) fold_state(mrun, l, a, EP, ml[j].x, ml[j].y, v[j]);
        }
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        float o[E];
#pragma unroll
        for (int e = 0; e < EP; ++e) o[e] = a[e] * inv;
        // thread sub == 0 collects the item's other elements (16-byte stores)
#pragma unroll
        for (int k = 1; k < TPI; ++k)
#pragma unroll
            for (int e = 0; e < EP; ++e) o[k * EP + e] = __shfl_down_sync(0xffffffffu, o[e], k);
        if (valid && sub == 0) store_out<OutT, E>(out, b, H, h, DH, dc, o);
    }
}

// Publishes one finished piece of a sequence: a release at GPU scope (the
// partials this CTA wrote before it are visible to whoever acquires the
// count), fire and forget.
__device__ __forceinline__ void publish_piece(unsigned* counter) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
}

// Waits (bounded, 1 s of %globaltimer) until *counter reaches `target`, with
// acquire loads: the partials published before each count are visible after
// it.  Returns false if the limit passed first.
__device__ __forceinline__ bool wait_count(const unsigned* counter, unsigned target) {
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
        if (v >= target) return true;
        if ((it & 15u) == 15u && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Before griddepcontrol.wait, when the inputs may still be written by the
// kernel ahead of this one (p.early == 0): runs the prologue on whatever
// seq_lens and block tables hold now and asks for this CTA's first K/V rows
// (up to two paged blocks of its first sequence) and that sequence's q row to
// be brought into L2.  Every value it reads may be stale; it only decides
// which addresses to prefetch, and a prefetch into L2 changes no value any
// thread reads afterwards (L2 is where all reads and writes meet; these loads
// bypass L1).  After the wait, the real prologue's dependent loads and the
// first stages then come from L2 instead of DRAM.  Uses misc[0..34]; ends with
// a CTA barrier.
template <int DH>
__device__ __forceinline__ void speculative_prefetch(const AttnParams& p, int* misc, int es) {
    const int tid = threadIdx.x;
    const int B = p.batch;
    const int per = (B + static_cast<int>(blockDim.x) - 1) / static_cast<int>(blockDim.x);
    const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
    int local = 0;
    for (int b = b_lo; b < b_hi; ++b) local += clamp_seq_len(__ldcg(p.seq_lens + b), p.mbps);
    if (tid == 0) misc[0] = -1;
    int N = 0;
    const int excl = block_exclusive_scan(local, misc + 2, &N);  // its barriers also order misc[0] = -1
    const int G = min(static_cast<int>(gridDim.x), max(N, 1));
    const int cta = blockIdx.x;
    const long long s_unit = cta < G ? static_cast<long long>(cta) * N / G : 0;
    const long long e_unit = cta < G ? static_cast<long long>(cta + 1) * N / G : 0;
    int run = excl;
    for (int b = b_lo; b < b_hi; ++b) {
        const int cl = clamp_seq_len(__ldcg(p.seq_lens + b), p.mbps);
        if (cl > 0 && run <= s_unit && s_unit < run + cl) {
            misc[0] = b;
            misc[1] = run;
        }
        run += cl;
    }
    __syncthreads();
    const int b0 = misc[0];
    if (tid < 32 && b0 >= 0 && e_unit > s_unit) {
        // Lane k < spec_blocks: the k-th paged block of this CTA's range (its
        // K and V runs), walking at most 8 sequences from the first one;
        // lane 31: the first sequence's q row.
        const int lane = tid;
        const size_t row_elems = static_cast<size_t>(p.n_kv_head) * DH;
        const size_t slab_elems = row_elems * kBlockTokens;
        if (lane < p.spec_blocks) {
            int k = lane;
            long long P = misc[1];  // rows before sequence b
            for (int b = b0, walked = 0; b < B && P < e_unit && walked < 8; ++b, ++walked) {
                const int cs = clamp_seq_len(__ldcg(p.seq_lens + b), p.mbps);
                const long long u = max(s_unit, P);
                const int t_lo = static_cast<int>(u - P);
                const int t_hi = static_cast<int>(min(e_unit - P, static_cast<long long>(cs)));
                if (t_hi > t_lo) {
                    const int j0 = t_lo / kBlockTokens, j1 = (t_hi - 1) / kBlockTokens + 1;
                    if (k < j1 - j0) {
                        const int j = j0 + k;
                        const int r_lo = max(t_lo - j * kBlockTokens, 0);
                        const int r_hi = min(t_hi - j * kBlockTokens, kBlockTokens);
                        const int blk = __ldcg(p.block_tables + static_cast<size_t>(b) * p.mbps + j);
                        if (blk >= 0 && blk < p.num_blocks && r_hi > r_lo) {
                            const char* src = static_cast<const char*>(p.pool) +
                                              ((static_cast<size_t>(blk) * p.n_layer + p.layer_idx) * 2 * slab_elems +
                                               static_cast<size_t>(r_lo) * row_elems) * es;
                            const uint32_t bytes = static_cast<uint32_t>((r_hi - r_lo) * row_elems * es);
                            bulk_prefetch_l2(src, bytes);
                            bulk_prefetch_l2(src + slab_elems * es, bytes);
                        }
                        break;
                    }
                    k -= j1 - j0;
                }
                P += cs;
            }
        } else if (lane == 31) {
            bulk_prefetch_l2(static_cast<const char*>(p.q) + static_cast<size_t>(b0) * p.q_row_stride * es,
                             static_cast<uint32_t>(p.n_head * DH * es));
        }
    }
    __syncthreads();
}

// Shared-memory ring between the softmax threads and the bookkeeping warp:
// one entry per finished sequence piece.
constexpr int kPieceRing = 8;

template <typename T, int DH, int QG, int MAXT, typename OutT, int CPT>
__global__ void __launch_bounds__(MAXT, 1) paged_decode_kernel(const AttnParams p) {
    constexpr int E = Elem<T>::kPer16B;
    constexpr int GL = DH / E;  // lanes sharing one head row
    static_assert(GL >= 2 && GL <= 32 && (32 % GL) == 0, "head_dim / dtype combination");
    constexpr int ES = static_cast<int>(sizeof(T));
    constexpr int TB = 4;  // tokens per online-softmax rescale
    constexpr int R = kPieceRing;

    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int H = p.n_head;
    const int Hkv = p.n_kv_head;
    const int C = Hkv * GL;  // 16-byte chunks per token row (all kv heads)
    const int cta = blockIdx.x;
    const int B = p.batch;
    const int S = p.stages;
    const int ncw = p.ncons / 32;  // softmax warps

    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    uint64_t* empty = full + S;
    uint64_t* piece_full = empty + S;  // [R], one arrival per softmax warp
    uint64_t* piece_empty = piece_full + R;  // [R]
    uint64_t* book_done = piece_empty + R;
    uint64_t* lm_bar = book_done + 1;  // [2] consumer-warp barriers of the in-CTA merge
    int* misc = reinterpret_cast<int*>(smem + p.off_misc);  // [0..1] first sequence and its row prefix, [2..34] scan
    int4* pieces = reinterpret_cast<int4*>(smem + p.off_misc + 160);  // [R] (b, i0, nseg, final)
    int* final_merge = misc + 36;  // [0] merge the final piece's sequence here, [1] b, [2] i0, [3] nseg
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], static_cast<uint32_t>(ncw));
        }
        for (int s = 0; s < R; ++s) {
            mbar_init(&piece_full[s], static_cast<uint32_t>(ncw));
            mbar_init(&piece_empty[s], 1);
        }
        mbar_init(book_done, 1);
        mbar_init(&lm_bar[0], static_cast<uint32_t>(ncw));
        mbar_init(&lm_bar[1], static_cast<uint32_t>(ncw));
        final_merge[0] = 0;
        fence_mbar_init();
    }

    // Programmatic dependent launch: the kernel behind us may be scheduled
    // right away.  Unless the caller said the inputs are already complete
    // (p.early), we wait here until the kernel before us has completed; with
    // p.early the set-up and the K/V streaming overlap its tail, and every
    // thread waits before its first global write (outputs, partials, counters)
    // -- and, with p.early == 2, the producer before reading each sequence's
    // newest key row.
    pdl_launch_dependents();
    if (p.early == 0) {
        __syncthreads();  // the barriers are initialised before misc is reused below
        speculative_prefetch<DH>(p, misc, ES);
        pdl_wait();
    }

    // ---- prologue: per-sequence row counts, global prefix, this CTA's range
    // (L2 loads: with p.early == 0 the speculative pass may have read these
    // addresses before the wait, so nothing may come from a stale L1 line)
    if (p.early != 0 && tid == 0) {
        // The producer reads the block tables only once the scan below has
        // placed this CTA; a small table is brought into L2 now, while the
        // seq_lens loads are in flight, so that read is not a second DRAM
        // round trip.  (With p.early == 0 the speculative pass has touched
        // this CTA's entries already.)  Rounded out to 16-byte granules that
        // each hold table bytes, so nothing outside mapped memory is named.
        const size_t bt_bytes = static_cast<size_t>(B) * p.mbps * sizeof(int);
        if (bt_bytes <= 32768) {
            const uintptr_t lo = reinterpret_cast<uintptr_t>(p.block_tables) & ~static_cast<uintptr_t>(15);
            const uintptr_t hi = (reinterpret_cast<uintptr_t>(p.block_tables) + bt_bytes + 15) &
                                 ~static_cast<uintptr_t>(15);
            bulk_prefetch_l2(reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo));
        }
    }
    const int per = (B + static_cast<int>(blockDim.x) - 1) / static_cast<int>(blockDim.x);
    const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
    // A thread's first kSeqLenRegs values stay in registers for the second
    // pass below (a second trip to L2 would sit on every CTA's start-up).
    constexpr int kSeqLenRegs = 4;
    int sl_raw[kSeqLenRegs];
    int local = 0;
#pragma unroll
    for (int i = 0; i < kSeqLenRegs; ++i) {
        sl_raw[i] = b_lo + i < b_hi ? __ldcg(p.seq_lens + b_lo + i) : 0;
        local += clamp_seq_len(sl_raw[i], p.mbps);
    }
    for (int b = b_lo + kSeqLenRegs; b < b_hi; ++b) local += clamp_seq_len(__ldcg(p.seq_lens + b), p.mbps);
    int N = 0;
    const int excl = block_exclusive_scan(local, misc + 2, &N);
    const int G = min(static_cast<int>(gridDim.x), max(N, 1));
    const long long s_unit = cta < G ? static_cast<long long>(cta) * N / G : 0;
    const long long e_unit = cta < G ? static_cast<long long>(cta + 1) * N / G : 0;
    {
        int run = excl;
        for (int b = b_lo; b < b_hi; ++b) {
            int raw = 0;
#pragma unroll
            for (int i = 0; i < kSeqLenRegs; ++i)
                if (b == b_lo + i) raw = sl_raw[i];
            if (b >= b_lo + kSeqLenRegs) raw = __ldcg(p.seq_lens + b);
            const int cl = clamp_seq_len(raw, p.mbps);
            if (p.off_seqlens >= 0) reinterpret_cast<int*>(smem + p.off_seqlens)[b] = cl;
            if (cl > 0 && run <= s_unit && s_unit < run + cl) {
                misc[0] = b;
                misc[1] = run;
            }
            if (b % static_cast<int>(gridDim.x) == cta) {
                if (raw != cl) flag_error(B2_DEVERR_SEQ_LEN);
                if (cl == 0) {
                    // no keys: the output is 0, like the reference (l == 0)
                    if (p.early) pdl_wait();
                    float z[E];
#pragma unroll
                    for (int e = 0; e < E; ++e) z[e] = 0.0f;
                    for (int i = 0; i < H * DH; i += E) store_out<OutT, E>(p.out, b, H, i / DH, DH, (i % DH) / E, z);
                }
            }
            run += cl;
        }
    }
    __syncthreads();
    if (e_unit <= s_unit) return;

    const size_t row_elems = static_cast<size_t>(Hkv) * DH;
    const size_t slab_elems = row_elems * kBlockTokens;
    const int row_bytes = static_cast<int>(row_elems) * ES;
    const int warp = tid >> 5;

    if (warp == ncw) {
        // ================================================= producer warp
        // Walks the sequences of [s_unit, e_unit) in windows of 32 (one lane
        // each) and issues one stage per (sequence, block) run of rows.  The
        // stage holding the range's last row carries the final flag, which
        // ends the consumers' loop.
        const int lane = tid & 31;
        const char* pool = static_cast<const char*>(p.pool);
        const size_t block_elems = static_cast<size_t>(p.n_layer) * 2 * slab_elems;
        const size_t layer_off = static_cast<size_t>(p.layer_idx) * 2 * slab_elems;
        long long u = s_unit;
        int bb = misc[0];
        long long Pb = misc[1];
        int n = 0;
        bool failed = false;
        bool newest_ok = p.early != 2;  // may the newest key rows be read yet?
        while (u < e_unit && !failed && bb < B) {
            const int b = bb + lane;
            int cl = 0;
            if (b < B)  // the prologue's copy in shared memory when there is one (no second trip to L2)
                cl = p.off_seqlens >= 0 ? reinterpret_cast<const int*>(smem + p.off_seqlens)[b]
                                        : clamp_seq_len(__ldcg(p.seq_lens + b), p.mbps);
            int incl = cl;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += y;
            }
            const int wtotal = __shfl_sync(0xffffffffu, incl, 31);
            for (int sidx = 0; sidx < 32 && u < e_unit && !failed; ++sidx) {
                const int cs = __shfl_sync(0xffffffffu, cl, sidx);
                const long long Ps = Pb + __shfl_sync(0xffffffffu, incl - cl, sidx);
                const int bs = bb + sidx;
                if (cs == 0 || Ps + cs <= u) continue;
                const int t_lo = static_cast<int>(u - Ps);                     // first row of the segment
                const int t_hi = static_cast<int>(min(e_unit, Ps + cs) - Ps);  // one past its last row
                const int j0 = t_lo / kBlockTokens, j1 = (t_hi - 1) / kBlockTokens + 1;
                // CTAs sharing this sequence: every piece computes the same pair
                const int i0 = cta_of_unit(Ps, N, G);
                const int nseg = cta_of_unit(Ps + cs - 1, N, G) - i0 + 1;
                for (int jc = j0; jc < j1 && !failed; jc += 32) {
                    const int jj = jc + lane;
                    int blk_l = 0;
                    if (jj < j1) {
                        blk_l = __ldcg(p.block_tables + static_cast<size_t>(bs) * p.mbps + jj);
                        if (blk_l < 0 || blk_l >= p.num_blocks) {
                            flag_error(B2_DEVERR_BLOCK_ID);
                            blk_l = 0;
                        }
                    }
                    const int cnt = min(32, j1 - jc);
                    for (int x = 0; x < cnt && !failed; ++x) {
                        const int blk = __shfl_sync(0xffffffffu, blk_l, x);
                        const int j = jc + x;
                        const int r_lo = max(t_lo - j * kBlockTokens, 0);
                        const int r_hi = min(t_hi - j * kBlockTokens, kBlockTokens);
                        // the block's rows [r_lo, r_hi) in stages of at most stage_rows rows
                        for (int rs = r_lo; rs < r_hi; rs += p.stage_rows) {
                            const int re = min(rs + p.stage_rows, r_hi);
                            int ok = 1;
                            if (lane == 0) {
                                const int st = n % S;
                                const uint32_t ph = static_cast<uint32_t>(n / S) & 1u;
                                if (!mbar_wait_bounded(&empty[st], ph ^ 1u)) {
                                    ok = 0;
                                } else {
                                    if (!newest_ok && j == (cs - 1) / kBlockTokens) {
                                        pdl_wait();  // this block holds the sequence's newest row
                                        newest_ok = true;
                                    }
                                    const int nrows = re - rs;
                                    const int first = (j == j0 && rs == r_lo) ? 1 : 0;
                                    const int lastf = (j == j1 - 1 && re == r_hi) ? 2 : 0;
                                    // the stage that ends at this CTA's last row ends its work
                                    const int finalf = (Ps + j * kBlockTokens + re == e_unit) ? 4 : 0;
                                    unsigned char* stage = smem + static_cast<size_t>(st) * p.stage_bytes;
                                    *reinterpret_cast<int4*>(stage + p.off_meta) =
                                        make_int4(bs, nrows | ((first | lastf | finalf) << 8), i0, nseg);
                                    const uint32_t kv_bytes = static_cast<uint32_t>(nrows * row_bytes);
                                    mbar_arrive_expect_tx(&full[st], 2u * kv_bytes + (first ? p.q_bytes : 0));
                                    const char* src = pool + (static_cast<size_t>(blk) * block_elems + layer_off +
                                                              static_cast<size_t>(rs) * row_elems) * ES;
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
                }
                u = Ps + t_hi;
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

    if (warp == ncw + 1) {
        // ============================================== bookkeeping warp
        // For each finished piece of a sequence spread over several CTAs:
        // the CTA holding the sequence's last piece (always that CTA's first
        // piece) merges the sequence at its end; every other piece is
        // published with one release-add on the sequence's counter and needs
        // no answer, so its CTA leaves as soon as its own work is done (a
        // last-arriver merge made every CTA wait for its count's round trip).
        const int lane = tid & 31;
        bool ok = true;
        int mb = -1, mi0 = 0, mn = 0;  // the sequence this CTA merges at its end
        for (int k = 0; ok; ++k) {
            const int rk = k % R;
            ok = mbar_wait_bounded(&piece_full[rk], static_cast<uint32_t>(k / R) & 1u);
            if (!ok) break;
            const int4 pc = pieces[rk];  // w: bit 0 the CTA's final piece, bit 1 its partials are in the stash
            if (p.early) pdl_wait();  // counters and outputs are written below
            __syncwarp();  // every lane has read the entry before it is released
            if (lane == 0) mbar_arrive(&piece_empty[rk]);
            if (pc.w & 2) {
                // The consumers left this piece's partials in the stash (they
                // did not wait for the kernel ahead); write them to the piece's
                // workspace slots.  Each lane fences its stores before the
                // warp barrier, so lane 0's counter update below publishes them.
                const int sk = p.fold_pieces ? 1 : p.ksplit;
                const size_t slot0 = (static_cast<size_t>(cta) + pc.x) * sk;
                const float4* sa = reinterpret_cast<const float4*>(smem + p.off_stash);
                float4* da = reinterpret_cast<float4*>(p.part_acc + slot0 * H * DH);
                const int n4 = sk * H * DH / 4;
                for (int i = lane; i < n4; i += 32) __stcg(da + i, sa[i]);
                const float2* sm = reinterpret_cast<const float2*>(sa + n4);
                for (int i = lane; i < sk * H; i += 32) __stcg(p.part_ml + slot0 * H + i, sm[i]);
                __threadfence();
                __syncwarp();
            }
            // pc.z == 0: a one-piece sequence, merged by the softmax threads
            if (pc.z > 0) {
                if (cta == pc.y + pc.z - 1) {
                    mb = pc.x;
                    mi0 = pc.y;
                    mn = pc.z;
                } else if (lane == 0) {
                    publish_piece(p.counters + pc.x);
                }
            }
            if (pc.w & 1) break;
        }
        if (!ok && lane == 0) flag_error(B2_DEVERR_TIMEOUT);
        if (ok && mb >= 0 && lane == 0) {
            // Wait (bounded) for the sequence's other pieces; the acquire
            // orders their partials before the softmax threads' merge (through
            // book_done below).
            if (wait_count(p.counters + mb, static_cast<unsigned>(mn - 1))) {
                final_merge[0] = 1;
                final_merge[1] = mb;
                final_merge[2] = mi0;
                final_merge[3] = mn;
            } else {
                flag_error(B2_DEVERR_TIMEOUT);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(book_done);  // also on failure: nobody waits on a dead warp
        return;
    }

    // ===================================================== consumer threads
    // Thread (ts, ct) of the CT = Hkv * GLT per token subgroup holds CPT
    // consecutive 16-byte chunks of one head row.  Two (16-bit types, up to two
    // query heads per kv head; more would spill) mean fewer shuffle levels and
    // the softmax bookkeeping each lane of a head repeats spread over half as
    // many lanes -- the planner picks them for the one-CTA-per-SM (wide head)
    // shapes, where the consumers' instruction count limits the stream.
    static_assert(CPT == 1 || (CPT == 2 && ES == 2 && QG <= 2), "chunks per consumer thread");
    constexpr int GLT = GL / CPT;  // lanes sharing one head row
    const int CT = Hkv * GLT;
    const int ks = p.ksplit;
    const int ts = tid / CT;
    const int ct = tid - ts * CT;
    const bool active = ts < ks;
    const int hk = ct / GLT;
    const int dgt = ct - hk * GLT;
    const int c0 = hk * GL + dgt * CPT;  // this thread's first chunk of the token row
    const int lane = tid & 31;
    const unsigned gmask = (GLT == 32) ? 0xffffffffu : (((1u << GLT) - 1u) << (lane & ~(GLT - 1)));

    uint4 qraw[QG][CPT];  // this thread's q chunks, in the storage dtype (bias added)
    float acc[QG][CPT * E];
    float m_run[QG];
    float l_run[QG];
#pragma unroll
    for (int g = 0; g < QG; ++g) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) qraw[g][i] = make_uint4(0u, 0u, 0u, 0u);
        m_run[g] = -INFINITY;
        l_run[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < CPT * E; ++e) acc[g][e] = 0.0f;
    }
    const float scale_log2 = p.scale_log2;

    int npieces = 0;
    int npieces_local = 0;  // pieces merged in shared memory (phase of lm_bar)
    for (int n = 0;; ++n) {
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
        const int nrows = min(meta.y & 0xff, kBlockTokens);
        const bool first = (meta.y >> 8) & 1;
        const bool last = (meta.y >> 9) & 1;
        const bool final_stage = (meta.y >> 10) & 1;

        if (active) {
            if (first) {
                const unsigned char* qs = stage + 2 * p.slab_bytes;
#pragma unroll
                for (int g = 0; g < QG; ++g) {
#pragma unroll
                    for (int i = 0; i < CPT; ++i) {
                        const int dofs = (hk * QG + g) * DH + (dgt * CPT + i) * E;  // element offset in the q row
                        qraw[g][i] = ld_shared16(qs + dofs * ES);
                        if (p.q_bias != nullptr) {
                            // q + bias rounded to T, as the reference's separate
                            // add_bias launch stores it (engine.cu:158).
                            float f[E], bf[E];
                            unpack16<T>(qraw[g][i], f);
                            unpack16<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.q_bias) + dofs)),
                                        bf);
#pragma unroll
                            for (int e = 0; e < E; ++e) f[e] = __fadd_rn(f[e], bf[e]);
                            qraw[g][i] = pack16<T>(f);
                        }
                    }
#pragma unroll
                    for (int e = 0; e < CPT * E; ++e) acc[g][e] = 0.0f;
                    m_run[g] = -INFINITY;
                    l_run[g] = 0.0f;
                }
            }
            const unsigned char* K = stage;
            const unsigned char* V = stage + p.slab_bytes;
            for (int t0 = ts; t0 < nrows; t0 += TB * ks) {
                const int cnt = min(TB, (nrows - t0 + ks - 1) / ks);  // same for the whole lane group
                float s[TB][QG];
#pragma unroll
                for (int j = 0; j < TB; ++j) {
                    if (j < cnt) {
                        const unsigned char* krow = K + ((t0 + j * ks) * C + c0) * 16;
                        uint4 kraw[CPT];
#pragma unroll
                        for (int i = 0; i < CPT; ++i) kraw[i] = ld_shared16(krow + i * 16);
#pragma unroll
                        for (int g = 0; g < QG; ++g) {
                            float d = dot16<T>(qraw[g][0], kraw[0], 0.0f);
#pragma unroll
                            for (int i = 1; i < CPT; ++i) d += dot16<T>(qraw[g][i], kraw[i], 0.0f);
                            s[j][g] = d;
                        }
                    } else {
#pragma unroll
                        for (int g = 0; g < QG; ++g) s[j][g] = 0.0f;
                    }
                }
#pragma unroll
                for (int off = GLT / 2; off > 0; off >>= 1)
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
                    const float corr = ex2_approx(m_run[g] - mx);  // 0 on the first batch (m_run = -inf)
                    m_run[g] = mx;
                    l_run[g] *= corr;
#pragma unroll
                    for (int e = 0; e < CPT * E; ++e) acc[g][e] *= corr;
                }
#pragma unroll
                for (int j = 0; j < TB; ++j) {
                    if (j < cnt) {
                        const unsigned char* vrow = V + ((t0 + j * ks) * C + c0) * 16;
                        uint4 vraw[CPT];
#pragma unroll
                        for (int i = 0; i < CPT; ++i) vraw[i] = ld_shared16(vrow + i * 16);
#pragma unroll
                        for (int g = 0; g < QG; ++g) {
                            const float pw = ex2_approx(s[j][g] - m_run[g]);
                            l_run[g] += pw;
#pragma unroll
                            for (int i = 0; i < CPT; ++i) axpy16<T>(pw, vraw[i], acc[g] + i * E);
                        }
                    }
                }
            }
        }
        // A piece's token subgroups can be folded right here through shared
        // memory -- the stage just consumed serves as scratch, so it is
        // released only afterwards: a sequence whose rows all lie in this CTA
        // (one piece, nseg == 1) is finished and written out; with
        // fold_pieces, any other piece leaves one partial in the workspace
        // instead of one per subgroup.
        const bool local = last && p.local_merge != 0 && meta.w == 1;
        const bool lm = local || (last && p.fold_pieces != 0);
        // An early-start launch's first piece, when it ends in mid-range,
        // leaves its partials in the stash and the consumers stream on; the
        // bookkeeping warp waits for the kernel ahead and writes them out.
        const bool stash = last && !local && !final_stage && npieces == 0 && p.early != 0 && p.off_stash >= 0;
        if (!lm) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }

        if (last && !stash) {
            if (p.early) pdl_wait();  // outputs / the workspace are written from here on
        }
        if (lm) {
            // (1) every consumer warp is done with the stage's K/V; (2) every
            // subgroup's (m, l, acc) is in the scratch; (3) item-parallel merge.
            // The barriers are mbarriers with bounded waits (no CTA barrier: a
            // warp that timed out has left).
            float* acc_s = reinterpret_cast<float*>(stage);
            float2* ml_s = reinterpret_cast<float2*>(acc_s + static_cast<size_t>(ks) * H * DH);
            const uint32_t lph = static_cast<uint32_t>(npieces_local) & 1u;
            __syncwarp();
            if (lane == 0) mbar_arrive(&lm_bar[0]);
            if (__any_sync(0xffffffffu, !mbar_wait_bounded(&lm_bar[0], lph))) {
                if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
                return;
            }
            if (active) {
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    const int h = hk * QG + g;
                    float* dst = acc_s + (static_cast<size_t>(ts) * H + h) * DH + dgt * CPT * E;
#pragma unroll
                    for (int e = 0; e < CPT * E; e += 4)
                        *reinterpret_cast<float4*>(dst + e) =
                            make_float4(acc[g][e], acc[g][e + 1], acc[g][e + 2], acc[g][e + 3]);
                    if (dgt == 0) ml_s[ts * H + h] = make_float2(m_run[g], l_run[g]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&lm_bar[1]);
            if (__any_sync(0xffffffffu, !mbar_wait_bounded(&lm_bar[1], lph))) {
                if (lane == 0) flag_error(B2_DEVERR_TIMEOUT);
                return;
            }
            constexpr int EO = Elem<OutT>::kPer16B;  // output elements per item (one 16-byte store)
            constexpr int CH = DH / EO;
            if (!local) {
                // the piece's partial, slot (cta + b) of one per piece (or the stash)
                const size_t slot = static_cast<size_t>(cta) + b;
                float* st_acc = reinterpret_cast<float*>(smem + p.off_stash);
                float2* st_ml = reinterpret_cast<float2*>(st_acc + static_cast<size_t>(H) * DH);
                for (int it = tid; it < H * (DH / 4); it += p.ncons) {
                    const int h = it / (DH / 4);
                    const int c = it - h * (DH / 4);
                    float mrun = -INFINITY, l = 0.0f, a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    for (int j = 0; j < ks; ++j) {
                        const float2 ml = ml_s[j * H + h];
                        const float4 v =
                            *reinterpret_cast<const float4*>(acc_s + (static_cast<size_t>(j) * H + h) * DH + c * 4);
                        const float a2[4] = {v.x, v.y, v.z, v.w};
                        fold_state(mrun, l, a, 4, ml.x, ml.y, a2);
                    }
                    if (stash) {
                        *reinterpret_cast<float4*>(st_acc + static_cast<size_t>(h) * DH + c * 4) =
                            make_float4(a[0], a[1], a[2], a[3]);
                        if (c == 0) st_ml[h] = make_float2(mrun, l);
                    } else {
                        __stcg(reinterpret_cast<float4*>(p.part_acc + (slot * H + h) * DH + c * 4),
                               make_float4(a[0], a[1], a[2], a[3]));
                        if (c == 0) __stcg(p.part_ml + slot * H + h, make_float2(mrun, l));
                    }
                }
            }
            for (int it = tid; local && it < H * CH; it += p.ncons) {
                const int h = it / CH;
                const int c = it - h * CH;
                float mrun = -INFINITY, l = 0.0f, a[EO];
#pragma unroll
                for (int e = 0; e < EO; ++e) a[e] = 0.0f;
                for (int j = 0; j < ks; ++j) {
                    const float2 ml = ml_s[j * H + h];
                    float a2[EO];
                    const float* src = acc_s + (static_cast<size_t>(j) * H + h) * DH + c * EO;
#pragma unroll
                    for (int e = 0; e < EO; e += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(src + e);
                        a2[e] = v.x;
                        a2[e + 1] = v.y;
                        a2[e + 2] = v.z;
                        a2[e + 3] = v.w;
                    }
                    fold_state(mrun, l, a, EO, ml.x, ml.y, a2);
                }
                const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
                for (int e = 0; e < EO; ++e) a[e] *= inv;
                store_out<OutT, EO>(p.out, b, H, h, DH, c, a);
            }
            ++npieces_local;
            // the scratch was written through the generic proxy; the producer's
            // next bulk copy into this stage writes through the async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);  // the scratch reads are done
        }
        if (last) {
            // ---- piece end: this subgroup's partial goes to the workspace.
            // Slot (cta + b) is unique per (CTA, sequence) pair: along the CTA
            // order both indices only grow, so cta + b never repeats.
            if (active && !lm && stash) {
                // the stash mirrors the slots' layout: [ts][h][head_dim], then [ts][h] (m, l)
                float* st_acc = reinterpret_cast<float*>(smem + p.off_stash);
                float2* st_ml = reinterpret_cast<float2*>(st_acc + static_cast<size_t>(ks) * H * DH);
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    const int h = hk * QG + g;
                    float* dst = st_acc + (static_cast<size_t>(ts) * H + h) * DH + dgt * CPT * E;
#pragma unroll
                    for (int e = 0; e < CPT * E; e += 4)
                        *reinterpret_cast<float4*>(dst + e) =
                            make_float4(acc[g][e], acc[g][e + 1], acc[g][e + 2], acc[g][e + 3]);
                    if (dgt == 0) st_ml[ts * H + h] = make_float2(m_run[g], l_run[g]);
                }
            } else if (active && !lm) {
                const size_t slot = (static_cast<size_t>(cta) + b) * ks + ts;
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    const int h = hk * QG + g;
                    float* dst = p.part_acc + (slot * H + h) * DH + dgt * CPT * E;
#pragma unroll
                    for (int e = 0; e < CPT * E; e += 4)
                        __stcg(reinterpret_cast<float4*>(dst + e),
                               make_float4(acc[g][e], acc[g][e + 1], acc[g][e + 2], acc[g][e + 3]));
                    if (dgt == 0) __stcg(p.part_ml + slot * H + h, make_float2(m_run[g], l_run[g]));
                }
            }
            // Hand the piece to the bookkeeping warp (ring slot npieces % R):
            // thread 0 writes the entry, and every warp arrives once its
            // partial stores are issued.  The arrivals are CTA-scope releases;
            // the bookkeeper's GPU-scope fence before its counter update then
            // publishes all of them (the release pattern of a CTA barrier
            // followed by one thread's fence and atomic).
            const int rk = npieces % R;
            if (tid == 0) {
                if (!mbar_wait_bounded(&piece_empty[rk], (static_cast<uint32_t>(npieces / R) & 1u) ^ 1u))
                    flag_error(B2_DEVERR_TIMEOUT);
                pieces[rk] = make_int4(b, meta.z, local ? 0 : meta.w, (final_stage ? 1 : 0) | (stash ? 2 : 0));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&piece_full[rk]);
            ++npieces;
        }
        if (final_stage) break;
    }

    // ---- tail: merge the final piece's sequence if this CTA completed it.
    // Every thread waits for the bookkeeper on its own (bounded); no CTA
    // barrier, since a warp that timed out above has already left.
    if (!mbar_wait_bounded(book_done, 0)) {
        if (tid == 0) flag_error(B2_DEVERR_TIMEOUT);
        return;
    }
    if (final_merge[0]) {
        // The bookkeeper's acquire on the counter, then its arrival on
        // book_done, order the other CTAs' partials before these reads.
        const int fb = final_merge[1], fi0 = final_merge[2], fn = final_merge[3];
        const int sk = p.fold_pieces ? 1 : ks;  // partial slots per piece
        const OutSpec& o = p.out;
        if (p.ncons >= 4 * H * GL)
            merge_partials<DH, E, 4, OutT>(p.part_ml, p.part_acc, o, H, sk, fb, fi0, fn, tid, p.ncons);
        else if (p.ncons >= 2 * H * GL)
            merge_partials<DH, E, 2, OutT>(p.part_ml, p.part_acc, o, H, sk, fb, fi0, fn, tid, p.ncons);
        else
            merge_partials<DH, E, 1, OutT>(p.part_ml, p.part_acc, o, H, sk, fb, fi0, fn, tid, p.ncons);
        if (tid == 0) p.counters[fb] = 0u;  // every launch leaves the counters at zero
    }
}

// Merges the partials of one sequence per CTA: thread (h, chunk dc) combines
// (m, l, acc) over the sequence's segments and token subgroups -- slots
// (i0 + b) * ks ... -- with a running max, and writes E output elements.  The
// loads of SB slots are issued together (one L2 round trip per SB slots).  A
// subgroup that saw no rows has l == 0 and is skipped; a sequence without
// keys gets zeros.
template <int DH, int E, typename OutT>
__global__ void __launch_bounds__(512) paged_decode_combine_kernel(const CombineParams c) {
    constexpr int GL = DH / E;
    constexpr int SB = 8;  // slots in flight: 48 (E = 4) or 80 (E = 8) registers of loads
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    const int idx = threadIdx.x;
    const int H = c.n_head;
    if (idx >= H * GL) return;
    const int h = idx / GL;
    const int dc = idx - h * GL;
    const int2 info = __ldcg(c.seq_info + b);
    const int ks = c.ksplit;
    const int nslots = info.y * ks;
    const size_t slot0 = (static_cast<size_t>(info.x) + b) * ks;
    float mrun = -INFINITY, l = 0.0f, a[E];
#pragma unroll
    for (int e = 0; e < E; ++e) a[e] = 0.0f;
    for (int s0 = 0; s0 < nslots; s0 += SB) {
        float2 ml[SB];
        float4 v[SB][E / 4];
#pragma unroll
        for (int j = 0; j < SB; ++j) {
            ml[j] = make_float2(-INFINITY, 0.0f);
            if (s0 + j < nslots) {
                const size_t sl = slot0 + s0 + j;
                ml[j] = __ldcg(c.part_ml + sl * H + h);
                const float4* src = reinterpret_cast<const float4*>(c.part_acc + (sl * H + h) * DH + dc * E);
#pragma unroll
                for (int q = 0; q < E / 4; ++q) v[j][q] = __ldcg(src + q);
            }
        }
#pragma unroll
        for (int j = 0; j < SB; ++j) {
            if (!(ml[j].y > 0.0f)) continue;  // no rows in that subgroup (or past the end)
            const float mn = fmaxf(mrun, ml[j].x);
            const float wo = exp2f(mrun - mn);  // 0 while mrun is -inf
            const float wn = exp2f(ml[j].x - mn);
            mrun = mn;
            l = fmaf(ml[j].y, wn, l * wo);
#pragma unroll
            for (int q = 0; q < E / 4; ++q) {
                a[4 * q] = fmaf(v[j][q].x, wn, a[4 * q] * wo);
                a[4 * q + 1] = fmaf(v[j][q].y, wn, a[4 * q + 1] * wo);
                a[4 * q + 2] = fmaf(v[j][q].z, wn, a[4 * q + 2] * wo);
                a[4 * q + 3] = fmaf(v[j][q].w, wn, a[4 * q + 3] * wo);
            }
        }
    }
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) a[e] *= inv;
    store_out<OutT, E>(c.out, b, H, h, DH, dc, a);
}

}  // namespace b2
