// linear_tc.cuh -- the decode step's linear layers on the 5th-generation
// tensor cores: y[b][n] = epilogue(sum_k x[b][k] * w[n][k]) for a small
// batch of rows b and a large weight matrix w (nn.Linear layout, [n][k],
// the layout gpu-engine/src/engine.cu:124-131 hands cuBLAS as op(T)).
//
// At decode batch sizes the layer is a weight stream: every weight byte is
// used for `batch` multiply-adds, so the kernel is built to read w from HBM
// once at full bandwidth and to keep the batch on chip:
//
//   * swapped operands: the MMA's M = 128 weight rows (output features), its
//     N = the batch tile (16..256 rows of x), K in blocks of 64 elements.
//     A = the weight tile [128][64] and B = the x tile [bn][64] are both
//     K-major, landed by 2-D TMA boxes in the 128-byte-swizzled layout;
//     the fp32 accumulator D^T[feature][batch] lives in TMEM;
//   * split K across a thread-block cluster: the S CTAs of a cluster share
//     one 128-feature tile and take S disjoint K ranges, so that
//     (features / 128) x S CTAs cover the GPU even for narrow layers.  The S
//     partial tiles are summed through distributed shared memory, pushed
//     rather than pulled: CTA o finishes feature rows [o * 128 / S, ...), and
//     every CTA stores its partial rows for o straight from TMEM into o's
//     receive buffer (st.shared::cluster, fire and forget; pulling them with
//     remote loads was latency-bound at ~10% of the DSMEM bandwidth).  CTA o
//     then adds the S slots in rank order (a deterministic sum) and runs the
//     epilogue;
//   * weights first: w never depends on the previous kernel on the stream,
//     so the producer issues the weight half of its first stages before
//     griddepcontrol.wait and the x half after it -- with programmatic
//     dependent launch the weight stream overlaps the previous kernel;
//   * epilogue fused: optional bias and GELU (the reference's separate
//     add_bias / bias_gelu launches, engine.cu:157-194), rounded the way the
//     unfused path rounds: T(gemm), then + bias, then GELU, then T.
//
// Roles (192 threads): warp 0 lane 0 TMA producer, warp 1 TMEM owner and
// (lane 0) MMA issuer, warps 2-5 epilogue (warp w reads TMEM lanes
// 32 * (w % 4) ...).  Every mbarrier wait is bounded; a wait that gives up
// flags B2_DEVERR_TIMEOUT and the CTA still passes both cluster barriers,
// so no CTA of the cluster is left waiting on it.
#pragma once

#include "b2_common.cuh"
#include "rows.cuh"
#include "tcgen05.cuh"

namespace b2 {

constexpr int kLinRows = 128;                          // weight rows per CTA (MMA M)
constexpr int kLinKBlock = 64;                         // K elements per stage (one 128-B swizzle row)
constexpr int kLinWBytes = kLinRows * kLinKBlock * 2;  // weight box: 16 KiB
constexpr int kLinThreads = 192;
constexpr int kLinMaxCols = 256;  // batch rows per CTA (MMA N limit)
constexpr int kLinMaxSplit = 8;   // CTAs per cluster (portable cluster size)

struct LinParams {
    const void* bias;  // [n_out] or null
    void* y;           // [batch][ldy]
    long long ldy;
    int batch, n_out;
    int bn;        // batch rows per CTA: multiple of 16, <= 256
    int kb_total;  // 64-element K blocks
    int stages;    // ring slots
};

// Shared-memory plan (bytes from the 1024-aligned base).  Once every MMA has
// completed the ring is reused by the epilogue: the split-K receive buffer
// (128 x bn fp32, S slots of 128 / S rows; S > 1 only) and after it the
// output tile this CTA stores ([bn][128 / S] of T, written by one TMA store).
struct LinLayout {
    __host__ __device__ static constexpr int stage_bytes(int bn) { return kLinWBytes + bn * 128; }
    __host__ __device__ static constexpr int off_out(int bn, int split) { return split > 1 ? kLinRows * bn * 4 : 0; }
    __host__ __device__ static constexpr int epi_bytes(int bn, int split) {
        return off_out(bn, split) + (kLinRows / split) * bn * 2;
    }
    __host__ __device__ static constexpr int ring_bytes(int bn, int stages, int split) {
        return epi_bytes(bn, split) > stages * stage_bytes(bn) ? epi_bytes(bn, split) : stages * stage_bytes(bn);
    }
    __host__ __device__ static constexpr int off_bars(int bn, int stages, int split) {
        return ring_bytes(bn, stages, split);
    }
    __host__ __device__ static constexpr int off_tmem(int bn, int stages, int split) {
        return off_bars(bn, stages, split) + 8 * (2 * stages + 1);
    }
    __host__ __device__ static constexpr int bytes(int bn, int stages, int split) {
        return off_tmem(bn, stages, split) + 16 + 1024;
    }
};

__host__ __device__ constexpr uint32_t lin_tmem_cols(int bn) {
    return bn <= 32 ? 32u : (bn <= 64 ? 64u : (bn <= 128 ? 128u : 256u));
}

// Bias of feature n as float (0 without a bias or past the last feature).
template <typename T>
__device__ __forceinline__ float lin_bias(const LinParams& p, int n) {
    return p.bias != nullptr && n < p.n_out ? Elem<T>::to_f(static_cast<const T*>(p.bias)[n]) : 0.0f;
}

// gelu_new (cpu_model.cpp:49-54, gelu.cu:7-10) in its sigmoid form:
// 0.5 x (1 + tanh(u)) = x / (1 + exp(-2u)), u = sqrt(2/pi) (x + 0.044715 x^3),
// the same function with one exponential and one division instead of tanhf.
// Within ~1e-5 relative of the tanhf form -- far below a 16-bit output's
// rounding step (this epilogue only serves f16 / bf16 outputs).  For
// x < ~-10 the denominator passes 2^126 and the result is 0 (exactly: -0).
__device__ __forceinline__ float gelu_sigmoid_form(float x) {
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return __fdividef(x, 1.0f + __expf(-2.0f * u));
}

// The epilogue of one output: acc is the fp32 dot product.  Compiled per
// (epilogue, bias) so that each kernel carries only its own arithmetic.
template <typename T, int EPI, bool BIAS>
__device__ __forceinline__ T lin_out(float acc, float bias_n) {
    float v = acc;
    if (BIAS || EPI == B2_LINEAR_GELU) {
        v = Elem<T>::to_f(Elem<T>::from_f(v));  // the GEMM's own output, rounded to T
        if (BIAS) v = __fadd_rn(v, bias_n);
        if (EPI == B2_LINEAR_GELU) v = gelu_sigmoid_form(v);
    }
    return Elem<T>::from_f(v);
}

template <typename T, int EPI, bool BIAS>
__global__ void __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const LinParams p, const __grid_constant__ CUtensorMap w_map,
                     const __grid_constant__ CUtensorMap x_map, const __grid_constant__ CUtensorMap y_map) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);  // swizzled tiles need 1024-B alignment
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int S = static_cast<int>(gridDim.x);  // CTAs of the cluster, splitting K
    const int rank = static_cast<int>(cluster_ctarank());
    const int n0 = static_cast<int>(blockIdx.y) * kLinRows;
    const int b0 = static_cast<int>(blockIdx.z) * p.bn;
    const int kb0 = rank * p.kb_total / S;
    const int nkb = (rank + 1) * p.kb_total / S - kb0;  // >= 1: the host keeps S <= kb_total
    const int ST = p.stages;
    const int SB = LinLayout::stage_bytes(p.bn);
    const uint32_t tmem_cols = lin_tmem_cols(p.bn);

    uint64_t* full = reinterpret_cast<uint64_t*>(smem + LinLayout::off_bars(p.bn, ST, S));
    uint64_t* empty = full + ST;
    uint64_t* acc_full = empty + ST;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LinLayout::off_tmem(p.bn, ST, S));

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    int issued = 0;  // producer: ring fills issued (their copies must land before the CTA leaves)
    if (warp == 0) {
        if (lane == 0) {
            const int npre = min(nkb, ST);
            for (int i = 0; i < npre; ++i) {
                mbar_arrive_expect_tx(&full[i], static_cast<uint32_t>(SB));
                tma_load_2d(smem + i * SB, &w_map, (kb0 + i) * kLinKBlock, n0, &full[i]);
            }
            issued = npre;
            pdl_wait();  // x is the previous kernel's output
            for (int i = 0; i < npre; ++i)
                tma_load_2d(smem + i * SB + kLinWBytes, &x_map, (kb0 + i) * kLinKBlock, b0, &full[i]);
            for (int i = npre; i < nkb; ++i) {
                const int s = i % ST;
                if (!mbar_wait_bounded(&empty[s], (static_cast<uint32_t>(i / ST) & 1u) ^ 1u)) {
                    flag_error(B2_DEVERR_TIMEOUT);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(SB));
                tma_load_2d(smem + s * SB, &w_map, (kb0 + i) * kLinKBlock, n0, &full[s]);
                tma_load_2d(smem + s * SB + kLinWBytes, &x_map, (kb0 + i) * kLinKBlock, b0, &full[s]);
                issued = i + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc<T>(kLinRows, p.bn, false, false);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % ST;
                if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(i / ST) & 1u)) {
                    flag_error(B2_DEVERR_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_addr(smem + s * SB);
                const uint32_t b = a + kLinWBytes;
#pragma unroll
                for (int k = 0; k < kLinKBlock / 16; ++k)
                    umma_f16(tmem, sw128_desc(a + 32 * k, 16, 1024), sw128_desc(b + 32 * k, 16, 1024), idesc,
                             (i | k) != 0);
                umma_commit(&empty[s]);  // the slot is free once these MMAs have read it
            }
            umma_commit(acc_full);
        }
    } else {
        // ---- epilogue warps: TMEM lane quadrant q holds features n0 + 32q ...
        pdl_wait();  // outputs are written below
        if (!mbar_wait_bounded(acc_full, 0)) flag_error(B2_DEVERR_TIMEOUT);
        __syncwarp();
        tc_fence_after();
        if (S == 1) {
            // thread = feature n; TMEM columns c = batch rows b0 + c, staged as
            // out[c][n - n0], 32 columns per TMEM load (32 independent outputs
            // in flight: the bias / GELU chain is latency-bound otherwise).
            constexpr int CH = 32;
            const int q = warp & 3;
            const int nl = q * 32 + lane;
            const float bias_n = lin_bias<T>(p, n0 + nl);
            T* out = reinterpret_cast<T*>(smem + LinLayout::off_out(p.bn, 1)) + nl;
            const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < p.bn; c += CH) {
                float v[CH];
                tmem_ld32(taddr + static_cast<uint32_t>(c), v);  // columns past bn: allocated, unused
#pragma unroll
                for (int j = 0; j < CH; ++j)
                    if (c + j < p.bn) out[(c + j) * kLinRows] = lin_out<T, EPI, BIAS>(v[j], bias_n);
            }
        }
    }

    // ---- split-K reduction over the cluster.  CTA o finishes feature rows
    // [o * R, (o + 1) * R); its receive buffer (over its own ring) holds one
    // slot per source CTA, [source][column / 4][row - o * R][4] fp32, so a
    // warp's stores of 32 rows land as contiguous runs of 16-byte chunks.
    if (S > 1) {
        const int lg_r = 7 - (__ffs(S) - 1);  // S is 2, 4 or 8
        const int R = 1 << lg_r;
        const int slot4 = (R * p.bn) >> 2;  // float4s per slot
        __syncwarp();
        cluster_sync_all();  // every CTA's MMAs are done: all rings are free
        if (warp >= 2) {
            const int q = warp & 3;
            const int row = q * 32 + lane;
            const uint32_t dst = dsmem_addr(smem_addr(smem) + static_cast<uint32_t>((rank * slot4 + (row & (R - 1))) * 16),
                                            static_cast<uint32_t>(row >> lg_r));
            const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
            for (int c = 0; c < p.bn; c += 32) {
                float v[32];
                tmem_ld32(taddr + static_cast<uint32_t>(c), v);
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    if (c + j < p.bn)
                        st_dsmem_f4(dst + static_cast<uint32_t>(((c + j) >> 2) * R * 16),
                                    make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
            }
        }
        __syncwarp();
        cluster_sync_all();  // every partial has landed in its owner's buffer
        if (warp >= 2) {
            // thread t: feature row t % R, column groups t / R, t / R + S, ...
            const int t = tid - 64;
            const int rr = t & (R - 1);
            const int n = n0 + rank * R + rr;
            const float bias_n = lin_bias<T>(p, n);
            T* out = reinterpret_cast<T*>(smem + LinLayout::off_out(p.bn, S)) + rr;  // [bn][R]
            const float4* in = reinterpret_cast<const float4*>(smem) + rr;
#pragma unroll 1
            for (int c4 = t >> lg_r; c4 < (p.bn >> 2); c4 += S) {
                const float4* src = in + c4 * R;
                float4 acc = src[0];
#pragma unroll
                for (int j = 1; j < kLinMaxSplit; ++j)
                    if (j < S) {  // in source order: the sum does not depend on timing
                        const float4 u = src[j * slot4];
                        acc.x += u.x;
                        acc.y += u.y;
                        acc.z += u.z;
                        acc.w += u.w;
                    }
                out[(4 * c4) * R] = lin_out<T, EPI, BIAS>(acc.x, bias_n);
                out[(4 * c4 + 1) * R] = lin_out<T, EPI, BIAS>(acc.y, bias_n);
                out[(4 * c4 + 2) * R] = lin_out<T, EPI, BIAS>(acc.z, bias_n);
                out[(4 * c4 + 3) * R] = lin_out<T, EPI, BIAS>(acc.w, bias_n);
            }
        }
    }

    // ---- the output tile leaves by one TMA store (rows past the batch and
    // features past out_features are clipped by the tensor map)
    if (warp >= 2) {
        fence_proxy_async_smem();  // the staged tile is read by the async proxy
        __syncwarp();
        named_sync(1, kLinThreads - 64);
        if (tid == 64) {
            tma_store_2d(&y_map, n0 + rank * (kLinRows / S), b0, smem + LinLayout::off_out(p.bn, S));
            bulk_commit_group();
            bulk_wait_group_all();
        }
    }
    if (warp >= 2) tc_fence_before();  // TMEM reads precede the dealloc below

    // ---- exit: this CTA's copies have landed, its MMAs are done, TMEM freed
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < ST && s < issued; ++s) {
            const int last_use = (issued - 1 - s) / ST;  // uses of slot s: s, s + ST, ...
            if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(last_use) & 1u)) flag_error(B2_DEVERR_TIMEOUT);
        }
    }
    if (warp == 1 && lane == 0) {
        // acc_full's first phase completes after every MMA of the CTA
        if (!mbar_wait_bounded(acc_full, 0)) flag_error(B2_DEVERR_TIMEOUT);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, tmem_cols);
}

}  // namespace b2
