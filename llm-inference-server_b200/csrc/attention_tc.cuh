// attention_tc.cuh -- grouped-query paged decode attention on the 5th-generation
// tensor cores (tcgen05 + TMEM + TMA), for 8 KV heads of head_dim 128 and
// 8 * QG query heads (QG = 1, 2, 4).
//
// Same result and contract as paged_decode_kernel (attention.cuh), which
// restates gpu-engine/src/kernels/attention.cu:49-127 (softmax over the
// seq_lens[b] cached keys of kv head h / QG).  Why a second kernel: with
// grouped queries every K/V element feeds QG dot products, and on the CUDA
// cores the FMAs, conversions and shuffles of 8 * QG heads outrun the issue
// slots before HBM is saturated.  Here the two contractions of a 16-token
// block run on the tensor cores:
//
//   one block slab in shared memory, rows r = kv_head * 16 + token (128 rows):
//       K[r][0..128)   V[r][0..128)         (TMA, SWIZZLE_128B, 2 boxes each)
//   S^T[r][hq]  = sum_d K[r][d] * Q[hq][d]            M=128, N=NP, K=128
//   O^T[d][hq] += sum_r V[r][d] * P^T[hq][r]          M=128, N=NP, K=128
//
// Q holds all NP (= max(16, H)) query heads, so S^T is computed for every
// (row, head) pair and a row reads back only the QG columns of its own kv
// head.  P^T is block-diagonal: entry (hq, r) is the softmax weight when hq
// belongs to row r's kv head and 0 otherwise (the zeros are written once),
// so the second product sums over the right keys only.  Tensor work is 8x
// the useful FLOPs, far below the tensor-core roof; the kernel is HBM-bound.
//
// Softmax: scores are scaled into log2 units; each (kv head, query head)
// keeps a reference maximum m_ref that only moves when a block maximum
// exceeds it by more than 8, so weights stay <= 2^8 and O in TMEM is
// rescaled only on those (rare) moves -- exact arithmetic, not an
// approximation.  Weights p are split into hi = T(p) and lo = T(p - hi) and
// both parts are multiplied in, so O carries ~16 significant bits of each
// weight (a single 16-bit weight would carry 8 for bf16).
//
// Work split and partials are those of paged_decode_kernel, in units of
// 16-token blocks: every CTA owns an equal share of the batch's blocks and
// writes one partial (m, l, acc) per sequence piece, merged by
// paged_decode_combine_kernel.
//
// Roles (224 threads, one CTA per SM), all talking through mbarriers:
//   warps 0-3  softmax / epilogue, one TMEM lane (MMA row) per thread;
//   warp 4     K producer: walks this CTA's blocks (block tables), publishes
//              each block's (sequence, valid rows, piece flags) in a meta
//              ring, writes each new piece's q (+ bias) into one of two Q
//              buffers, and streams K slabs by TMA into a 3-slot ring;
//   warp 5     MMA issuer (one thread): S(n+2) = K . Q^T as soon as K lands,
//              O += V^T . P^T when the softmax warps publish P(n);
//   warp 6     V producer: streams V slabs by TMA into its own 3-slot ring.
// K slots free up as soon as their S product completes and V slots when
// their PV product does, so each ring keeps about three blocks of loads in
// flight ahead of its consumer.
// Every wait is bounded (b2_common.cuh); a wait that gives up flags
// B2_DEVERR_TIMEOUT and the CTA leaves through the common exit, which waits
// for its own MMAs and copies and frees its TMEM.
#pragma once

#include "attention.cuh"
#include "b2_common.cuh"
#include "tcgen05.cuh"

namespace b2 {

constexpr int kTcKvHeads = 8;
constexpr int kTcHeadDim = 128;
constexpr int kTcHalfBytes = 16 * kTcKvHeads * 64 * 2;  // one TMA box: 128 rows x 64 elements = 16 KiB
constexpr int kTcSlotBytes = 2 * kTcHalfBytes;           // one K (or V) slab: both 64-dim halves
constexpr int kTcThreads = 224;
constexpr int kTcConsumers = 128;
constexpr int kTcMetaRing = 8;

struct TcParams {
    const void* q;
    int q_row_stride;
    const void* q_bias;
    const int* block_tables;
    const int* seq_lens;
    int batch, mbps, layer_idx, n_layer, num_blocks;
    float scale_log2;
    int stages;
    int2* seq_info;
    float2* part_ml;
    float* part_acc;
};

// Barriers of the 128 softmax threads (ids 1..7; 0 is __syncthreads).  bar.red
// is warp-aligned, so the warp is reconverged first (thread 0 runs extra
// issuer code between barriers).
__device__ __forceinline__ bool tc_sync_or(int id, bool pred) {
    __syncwarp();
    return named_sync_or(id, kTcConsumers, pred);
}
__device__ __forceinline__ void tc_sync(int id) {
    __syncwarp();
    named_sync(id, kTcConsumers);
}

// Shared-memory plan shared by host and device (bytes from the 1024-aligned
// base).  S = slots of each of the K and V rings.
template <int QG>
struct TcLayout {
    static constexpr int H = kTcKvHeads * QG;
    static constexpr int NP = H < 16 ? 16 : H;  // MMA N (query heads, padded)
    static constexpr int QHALF = NP * 128;      // one 64-dim half of Q, or of one P^T part
    static constexpr int TMEM_COLS = 3 * NP <= 64 ? 64 : (3 * NP <= 128 ? 128 : 256);
    static constexpr int NBARS_FIXED = 2 * kTcMetaRing + 2 + 2 + 2 + 3;  // meta, q, s_full, p_ready/pv/done
    __host__ __device__ static constexpr int off_v(int S) { return S * kTcSlotBytes; }
    __host__ __device__ static constexpr int off_q(int S) { return 2 * S * kTcSlotBytes; }  // [buffer][dims half]
    __host__ __device__ static constexpr int off_p(int S) { return off_q(S) + 4 * QHALF; }  // [hi|lo][rows half]
    __host__ __device__ static constexpr int off_meta(int S) { return off_p(S) + 4 * QHALF; }
    __host__ __device__ static constexpr int off_corr(int S) { return off_meta(S) + 16 * kTcMetaRing; }
    __host__ __device__ static constexpr int off_bars(int S) { return off_corr(S) + 4 * NP; }
    __host__ __device__ static constexpr int off_tmem(int S) { return off_bars(S) + 8 * (4 * S + NBARS_FIXED); }
    __host__ __device__ static constexpr int off_misc(int S) { return off_tmem(S) + 16; }
    __host__ __device__ static constexpr int bytes(int S) { return off_misc(S) + 4 * 36 + 1024; }
};

// Visits this CTA's blocks [s_unit, e_unit) in order with a whole warp:
// block-table entries are read 32 at a time, one per lane, then
// fn(sequence, block j, valid rows, flags, pool block) is called by every
// lane for each block (flags: 1 first block of the piece, 2 last, 4 last of
// the CTA).  fn returns false (warp-uniformly) to stop.  Returns the number
// of blocks visited.
template <typename F>
__device__ __forceinline__ int tc_walk_blocks(const TcParams& p, long long s_unit, long long e_unit, int b_first,
                                              long long p_first, F&& fn) {
    const int lane = threadIdx.x & 31;
    const int B = p.batch;
    long long u = s_unit;
    int bb = b_first;
    long long Pb = p_first;
    int n = 0;
    bool stop = false;
    while (u < e_unit && !stop && bb < B) {
        const int b = bb + lane;
        const int cl = b < B ? clamp_seq_len(__ldg(p.seq_lens + b), p.mbps) : 0;
        const int nbk = (cl + kBlockTokens - 1) / kBlockTokens;
        int incl = nbk;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        const int wtotal = __shfl_sync(0xffffffffu, incl, 31);
        for (int sidx = 0; sidx < 32 && u < e_unit && !stop; ++sidx) {
            const int cs = __shfl_sync(0xffffffffu, cl, sidx);
            const int nbs = __shfl_sync(0xffffffffu, nbk, sidx);
            const long long Ps = Pb + __shfl_sync(0xffffffffu, incl - nbk, sidx);
            const int bs = bb + sidx;
            if (nbs == 0 || Ps + nbs <= u) continue;
            const int j0 = static_cast<int>(u - Ps);
            const int j1 = static_cast<int>(min(e_unit, Ps + nbs) - Ps);
            for (int jc = j0; jc < j1 && !stop; jc += 32) {
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
                    const int j = jc + x;
                    const int nvalid = j == nbs - 1 ? cs - j * kBlockTokens : kBlockTokens;
                    const int flags = (j == j0 ? 1 : 0) | (j == j1 - 1 ? 2 : 0) | (Ps + j + 1 == e_unit ? 4 : 0);
                    if (!fn(bs, nvalid, flags, blk)) {
                        stop = true;
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
    return n;
}

template <typename T, int QG>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_decode_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap kv_map) {
    using L = TcLayout<QG>;
    constexpr int H = L::H;
    constexpr int NP = L::NP;
    constexpr int QHALF = L::QHALF;
    constexpr uint32_t TMEM_COLS = L::TMEM_COLS;
    constexpr uint32_t IDESC_QK = umma_idesc<T>(128, NP, false, false);
    constexpr uint32_t IDESC_PV = umma_idesc<T>(128, NP, true, false);
    constexpr int SCOLS = 2 * QG;  // S columns a warp reads: the QG heads of its two kv heads
    constexpr int MR = kTcMetaRing;

    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // swizzled tiles need 1024-B alignment
    const int S = p.stages;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int cta = blockIdx.x;
    const int B = p.batch;

    unsigned char* kring = smem;
    unsigned char* vring = smem + L::off_v(S);
    unsigned char* qbuf = smem + L::off_q(S);
    unsigned char* pbuf = smem + L::off_p(S);
    int4* meta = reinterpret_cast<int4*>(smem + L::off_meta(S));
    float* corr = reinterpret_cast<float*>(smem + L::off_corr(S));
    uint64_t* k_full = reinterpret_cast<uint64_t*>(smem + L::off_bars(S));
    uint64_t* k_empty = k_full + S;
    uint64_t* v_full = k_empty + S;
    uint64_t* v_empty = v_full + S;
    uint64_t* meta_full = v_empty + S;
    uint64_t* meta_empty = meta_full + MR;
    uint64_t* q_full = meta_empty + MR;
    uint64_t* q_empty = q_full + 2;
    uint64_t* s_full = q_empty + 2;
    uint64_t* p_ready = s_full + 2;
    uint64_t* pv_bar = p_ready + 1;
    uint64_t* done_bar = pv_bar + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_tmem(S));
    int* misc = reinterpret_cast<int*>(smem + L::off_misc(S));

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int s = 0; s < MR; ++s) {
            mbar_init(&meta_full[s], 1);
            mbar_init(&meta_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&q_full[s], 1);
            mbar_init(&q_empty[s], 1);
            mbar_init(&s_full[s], 1);
        }
        mbar_init(p_ready, 1);
        mbar_init(pv_bar, 1);
        mbar_init(done_bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    // Q rows >= H and the off-diagonal P^T entries stay zero for the whole kernel.
    for (int i = tid; i < 8 * QHALF / 16; i += kTcThreads)
        reinterpret_cast<uint4*>(qbuf)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < NP; i += kTcThreads) corr[i] = 1.0f;  // padding heads are never rescaled
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    pdl_launch_dependents();
    pdl_wait();

    // ---- prologue: per-sequence block counts, global prefix, this CTA's blocks
    const int per = (B + kTcThreads - 1) / kTcThreads;
    const int b_lo = min(B, tid * per), b_hi = min(B, b_lo + per);
    int local = 0;
    for (int b = b_lo; b < b_hi; ++b)
        local += (clamp_seq_len(__ldg(p.seq_lens + b), p.mbps) + kBlockTokens - 1) / kBlockTokens;
    int N = 0;
    const int excl = block_exclusive_scan(local, misc + 2, &N);
    const int G = min(static_cast<int>(gridDim.x), max(N, 1));
    const long long s_unit = cta < G ? static_cast<long long>(cta) * N / G : 0;
    const long long e_unit = cta < G ? static_cast<long long>(cta + 1) * N / G : 0;
    {
        int run = excl;
        for (int b = b_lo; b < b_hi; ++b) {
            const int raw = __ldg(p.seq_lens + b);
            const int nbk = (clamp_seq_len(raw, p.mbps) + kBlockTokens - 1) / kBlockTokens;
            if (nbk > 0 && run <= s_unit && s_unit < run + nbk) {
                misc[0] = b;
                misc[1] = run;
            }
            if (b % static_cast<int>(gridDim.x) == cta) {
                if (raw != clamp_seq_len(raw, p.mbps)) flag_error(B2_DEVERR_SEQ_LEN);
                int2 info = make_int2(0, 0);
                if (nbk > 0) {
                    const int i0 = cta_of_unit(run, N, G);
                    info = make_int2(i0, cta_of_unit(run + nbk - 1, N, G) - i0 + 1);
                }
                p.seq_info[b] = info;
            }
            run += nbk;
        }
    }
    __syncthreads();
    const int nblocks = static_cast<int>(e_unit - s_unit);  // blocks of this CTA (0 if none)
    const int b_first = misc[0];
    const long long p_first = misc[1];

    if (warp == 4 && nblocks > 0) {
        // ================================================= K producer
        int m = 0, pc = 0;
        bool failed = false;
        const int visited = tc_walk_blocks(p, s_unit, e_unit, b_first, p_first,
                                           [&](int bs, int nvalid, int flags, int blk) -> bool {
            int ok = 1;
            if (flags & 1) {
                // new piece: q of sequence bs (+ bias, rounded to T) into Q[pc & 1]
                if (lane == 0) ok = mbar_wait_bounded(&q_empty[pc & 1], (static_cast<uint32_t>(pc >> 1) & 1u) ^ 1u);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) return false;
                const T* qsrc = static_cast<const T*>(p.q) + static_cast<size_t>(bs) * p.q_row_stride;
                unsigned char* qdst = qbuf + (pc & 1) * 2 * QHALF;
                for (int c = lane; c < H * 16; c += 32) {
                    const int hq = c >> 4, dc = c & 15;
                    uint4 raw = __ldg(reinterpret_cast<const uint4*>(qsrc + hq * kTcHeadDim + dc * 8));
                    if (p.q_bias != nullptr) {
                        // q + bias rounded to T, as the reference's separate add_bias
                        // launch stores it (engine.cu:158)
                        float f[8], bf[8];
                        unpack16<T>(raw, f);
                        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.q_bias) +
                                                                         hq * kTcHeadDim + dc * 8)),
                                    bf);
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = __fadd_rn(f[e], bf[e]);
                        raw = pack16<T>(f);
                    }
                    *reinterpret_cast<uint4*>(qdst + (dc >> 3) * QHALF + sw128_offset(hq, (dc & 7) * 8, 2)) = raw;
                }
                fence_proxy_async_smem();  // the tensor core reads Q through the async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(&q_full[pc & 1]);
                ++pc;
            }
            if (lane == 0) {
                const int mr = m % MR;
                ok = mbar_wait_bounded(&meta_empty[mr], (static_cast<uint32_t>(m / MR) & 1u) ^ 1u);
                if (ok) {
                    meta[mr] = make_int4(bs, nvalid | (flags << 8), 0, 0);
                    mbar_arrive(&meta_full[mr]);
                    const int st = m % S;
                    ok = mbar_wait_bounded(&k_empty[st], (static_cast<uint32_t>(m / S) & 1u) ^ 1u);
                    if (ok) {
                        mbar_arrive_expect_tx(&k_full[st], kTcSlotBytes);
                        const int slab = (blk * p.n_layer + p.layer_idx) * 2;
                        unsigned char* dst = kring + static_cast<size_t>(st) * kTcSlotBytes;
                        tma_load_4d(dst, &kv_map, 0, 0, 0, slab, &k_full[st]);
                        tma_load_4d(dst + kTcHalfBytes, &kv_map, 64, 0, 0, slab, &k_full[st]);
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                failed = true;
                return false;
            }
            ++m;
            return true;
        });
        (void)visited;
        if (lane == 0) {
            if (failed) flag_error(B2_DEVERR_TIMEOUT);
            for (int i = max(0, m - S); i < m; ++i)  // no copy may still be in flight at exit
                if (!mbar_wait_bounded(&k_full[i % S], static_cast<uint32_t>(i / S) & 1u)) flag_error(B2_DEVERR_TIMEOUT);
        }
    } else if (warp == 6 && nblocks > 0) {
        // ================================================= V producer
        int m = 0;
        bool failed = false;
        tc_walk_blocks(p, s_unit, e_unit, b_first, p_first, [&](int, int, int, int blk) -> bool {
            int ok = 1;
            if (lane == 0) {
                const int st = m % S;
                ok = mbar_wait_bounded(&v_empty[st], (static_cast<uint32_t>(m / S) & 1u) ^ 1u);
                if (ok) {
                    mbar_arrive_expect_tx(&v_full[st], kTcSlotBytes);
                    const int slab = (blk * p.n_layer + p.layer_idx) * 2 + 1;
                    unsigned char* dst = vring + static_cast<size_t>(st) * kTcSlotBytes;
                    tma_load_4d(dst, &kv_map, 0, 0, 0, slab, &v_full[st]);
                    tma_load_4d(dst + kTcHalfBytes, &kv_map, 64, 0, 0, slab, &v_full[st]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                failed = true;
                return false;
            }
            ++m;
            return true;
        });
        if (lane == 0) {
            if (failed) flag_error(B2_DEVERR_TIMEOUT);
            for (int i = max(0, m - S); i < m; ++i)
                if (!mbar_wait_bounded(&v_full[i % S], static_cast<uint32_t>(i / S) & 1u)) flag_error(B2_DEVERR_TIMEOUT);
        }
    } else if (warp == 5 && lane == 0 && nblocks > 0) {
        // ================================================= MMA issuer
        uint32_t first_bits = 0;  // bit m % 32: block m starts a piece (PV(m) must not accumulate)
        int qpc = 0;              // pieces whose Q has been taken
        int qcur = 0;             // Q buffer of the piece being multiplied
        // S(m) = K(m) . Q^T into S buffer m & 1
        auto issue_qk = [&](int m) -> bool {
            const int mr = m % MR;
            if (!mbar_wait_bounded(&meta_full[mr], static_cast<uint32_t>(m / MR) & 1u)) return false;
            const int flags = meta[mr].y >> 8;
            if (flags & 1) {
                qcur = qpc & 1;
                if (!mbar_wait_bounded(&q_full[qcur], static_cast<uint32_t>(qpc >> 1) & 1u)) return false;
                ++qpc;
                first_bits |= 1u << (m & 31);
            } else {
                first_bits &= ~(1u << (m & 31));
            }
            const int st = m % S;
            if (!mbar_wait_bounded(&k_full[st], static_cast<uint32_t>(m / S) & 1u)) return false;
            tc_fence_after();
            const uint32_t kb = smem_addr(kring + static_cast<size_t>(st) * kTcSlotBytes);
            const uint32_t qa = smem_addr(qbuf + qcur * 2 * QHALF);
            const uint32_t d = tmem + static_cast<uint32_t>((m & 1) * NP);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t h = static_cast<uint32_t>(kk >> 2), ko = static_cast<uint32_t>((kk & 3) * 32);
                umma_f16(d, sw128_desc(kb + h * kTcHalfBytes + ko, 16, 1024), sw128_desc(qa + h * QHALF + ko, 16, 1024),
                         IDESC_QK, kk > 0);
            }
            umma_commit(&k_empty[st]);
            umma_commit(&s_full[m & 1]);
            if (flags & 2) umma_commit(&q_empty[qcur]);  // the piece's last S product frees its Q buffer
            return true;
        };
        bool ok = issue_qk(0);
        if (ok && nblocks > 1) ok = issue_qk(1);
        for (int n = 0; ok && n < nblocks; ++n) {
            // O^T (+)= V(n)^T . P^T(n), hi then lo part
            const int st = n % S;
            if (!mbar_wait_bounded(p_ready, static_cast<uint32_t>(n) & 1u) ||
                !mbar_wait_bounded(&v_full[st], static_cast<uint32_t>(n / S) & 1u)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const bool first_blk = (first_bits >> (n & 31)) & 1u;
            const uint32_t vb = smem_addr(vring + static_cast<size_t>(st) * kTcSlotBytes);
            const uint32_t pb = smem_addr(pbuf);
#pragma unroll
            for (int part = 0; part < 2; ++part)
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t bo = static_cast<uint32_t>(part * 2 * QHALF + (kk >> 2) * QHALF + (kk & 3) * 32);
                    umma_f16(tmem + 2u * NP, sw128_desc(vb + static_cast<uint32_t>(kk) * 2048u, kTcHalfBytes, 1024),
                             sw128_desc(pb + bo, 16, 1024), IDESC_PV, !(first_blk && part == 0 && kk == 0));
                }
            umma_commit(&v_empty[st]);
            umma_commit(pv_bar);
            if (n + 2 < nblocks) ok = issue_qk(n + 2);
        }
        if (!ok) flag_error(B2_DEVERR_TIMEOUT);
    } else if (warp < 4 && nblocks > 0) {
        // ================================================ softmax warps
        const int r = tid;           // MMA row = TMEM lane of S
        const int hk = r >> 4;       // kv head of this row
        const int t = r & 15;        // token within the block
        const bool upper = (lane & 16) != 0;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        const uint32_t s_col0 = static_cast<uint32_t>(2 * warp * QG);
        const uint32_t o_col = 2u * NP;
        const float scale_log2 = p.scale_log2;
        float m_ref[QG], l_part[QG];
#pragma unroll
        for (int g = 0; g < QG; ++g) {
            m_ref[g] = -INFINITY;
            l_part[g] = 0.0f;
        }
        for (int n = 0; n < nblocks; ++n) {
            const int mr = n % MR;
            bool ok = mbar_wait_bounded(&meta_full[mr], static_cast<uint32_t>(n / MR) & 1u);
            int4 m4 = make_int4(0, 0, 0, 0);
            if (ok) m4 = meta[mr];
            const int b = m4.x;
            const int nvalid = m4.y & 0xff;
            const bool first = (m4.y >> 8) & 1;
            const bool last = (m4.y >> 9) & 1;
            if (first) {
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    m_ref[g] = -INFINITY;
                    l_part[g] = 0.0f;
                }
            }
            // ---- scores of block n: this row's QG query heads
            ok = ok && mbar_wait_bounded(&s_full[n & 1], static_cast<uint32_t>(n >> 1) & 1u);
            float sv[SCOLS];
#pragma unroll
            for (int i = 0; i < SCOLS; ++i) sv[i] = 0.0f;
            // tcgen05.ld is warp-collective: the warp loads when all its lanes may.
            if (__all_sync(0xffffffffu, ok)) {
                tc_fence_after();
                const uint32_t saddr = tmem + lane_base + static_cast<uint32_t>((n & 1) * NP) + s_col0;
                if constexpr (SCOLS == 2) {
                    tmem_ld2(saddr, sv);
                } else if constexpr (SCOLS == 4) {
                    tmem_ld4(saddr, sv);
                } else {
#pragma unroll
                    for (int c0 = 0; c0 < SCOLS; c0 += 8) tmem_ld8(saddr + c0, sv + c0);
                }
            } else {
                ok = false;
            }
            const bool valid = t < nvalid;
            float s[QG], cf[QG];
            bool need = false;
#pragma unroll
            for (int g = 0; g < QG; ++g) {
                s[g] = valid ? (upper ? sv[QG + g] : sv[g]) * scale_log2 : -INFINITY;
                float bm = s[g];
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
                cf[g] = 1.0f;
                if (bm > m_ref[g] + 8.0f) {  // the block has at least one valid row, so bm is finite
                    cf[g] = exp2f(m_ref[g] - bm);  // 0 while m_ref is -inf
                    m_ref[g] = bm;
                    l_part[g] *= cf[g];
                    need = true;
                }
            }
            // P^T(n-1) is read until PV(n-1) completes; after it, O is stable too.
            if (!first) ok = ok && mbar_wait_bounded(pv_bar, static_cast<uint32_t>(n - 1) & 1u);
            if (!valid && ok) {
                // rows past the sequence end: whatever the pool holds there (even
                // NaN) must not reach O through 0 * V.  The slab must have landed.
                ok = mbar_wait_bounded(&v_full[n % S], static_cast<uint32_t>(n / S) & 1u);
                if (ok) {
                    unsigned char* vrow = vring + static_cast<size_t>(n % S) * kTcSlotBytes + r * 128;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        reinterpret_cast<uint4*>(vrow)[i] = make_uint4(0u, 0u, 0u, 0u);
                        reinterpret_cast<uint4*>(vrow + kTcHalfBytes)[i] = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
            }
            if (ok) {
                const int kh = r >> 6, rr = r & 63;
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    const float pw = valid ? exp2f(s[g] - m_ref[g]) : 0.0f;
                    l_part[g] += pw;
                    const T hi = Elem<T>::from_f(pw);
                    const T lo = Elem<T>::from_f(pw - Elem<T>::to_f(hi));
                    const int hq = hk * QG + g;
                    const uint32_t off = static_cast<uint32_t>(kh * QHALF) + sw128_offset(hq, rr, 2);
                    *reinterpret_cast<T*>(pbuf + off) = hi;
                    *reinterpret_cast<T*>(pbuf + 2 * QHALF + off) = lo;
                    if ((lane & 15) == 0) corr[hq] = cf[g];
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            if (tc_sync_or(1, !ok)) {
                if (tid == 0) flag_error(B2_DEVERR_TIMEOUT);
                break;
            }
            if (tc_sync_or(2, need) && !first) {
                // O columns of heads whose reference max moved: O *= corr (lane = dim)
                tc_fence_after();
                const uint32_t oaddr = tmem + lane_base + o_col;
#pragma unroll
                for (int c0 = 0; c0 < NP; c0 += 8) {
                    float o[8];
                    tmem_ld8(oaddr + c0, o);
#pragma unroll
                    for (int i = 0; i < 8; ++i) o[i] *= corr[c0 + i];
                    tmem_st8(oaddr + c0, o);
                }
                tmem_wait_st();
                tc_fence_before();
                tc_sync(3);
            }
            if (tid == 0) {
                mbar_arrive(p_ready);          // P(n) written, S(n) read, O rescaled: PV(n) may go
                mbar_arrive(&meta_empty[mr]);  // every softmax thread has read meta(n)
            }
            if (last) {
                // ---- piece end: partial (m, l, acc) of sequence b, slot cta + b
                const bool got_o = mbar_wait_bounded(pv_bar, static_cast<uint32_t>(n) & 1u);
                if (tc_sync_or(4, !got_o)) {
                    if (tid == 0) flag_error(B2_DEVERR_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const size_t slot = static_cast<size_t>(cta) + b;
                const uint32_t oaddr = tmem + lane_base + o_col;
                float* acc = p.part_acc + slot * H * kTcHeadDim + r;  // lane r holds dim r
#pragma unroll
                for (int c0 = 0; c0 < NP; c0 += 8) {
                    float o[8];
                    tmem_ld8(oaddr + c0, o);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (c0 + i < H) __stcg(acc + (c0 + i) * kTcHeadDim, o[i]);
                }
#pragma unroll
                for (int g = 0; g < QG; ++g) {
                    float lt = l_part[g];
#pragma unroll
                    for (int off = 8; off > 0; off >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
                    if ((lane & 15) == 0) __stcg(p.part_ml + slot * H + hk * QG + g, make_float2(m_ref[g], lt));
                }
                // the next piece's first PV overwrites O only after the next p_ready
                tc_fence_before();
                tc_sync(5);
            }
        }
    }

    // ---- common exit: every MMA of this CTA done, every thread out of TMEM
    if (warp == 5 && lane == 0) {
        umma_commit(done_bar);
        if (!mbar_wait_bounded(done_bar, 0)) flag_error(B2_DEVERR_TIMEOUT);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace b2
