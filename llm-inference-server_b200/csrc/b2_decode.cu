// b2_decode.cu -- extern "C" entry points of libb2decode.so (include/b2_decode.h).
//
// Host side of the kernel-launch layer: argument checks (returned as status
// codes before anything is launched), the attention launch plan (stages,
// token subgroups, grid = one CTA per SM), and dtype / head_dim dispatch.
// Nothing here allocates device memory or synchronises, except
// b2_device_errors, which reads the device error word.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "append.cuh"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "b2_common.cuh"
#include "linear_tc.cuh"
#include "lm_head_tc.cuh"
#include "prefill_tc.cuh"
#include "rows.cuh"
#include "tp.cuh"

namespace b2 {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* what) {
    g_last_error = what;
    return code;
}

int launch_status() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    return B2_OK;
}

int dtype_size(int dt) { return dt == B2_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == B2_F32 || dt == B2_F16 || dt == B2_BF16; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct DeviceInfo {
    int sms = 0;
    int max_smem_optin = 0;
    int smem_per_sm = 0;
};

DeviceInfo device_info(int* dev_out) {
    static DeviceInfo cache[64];
    static std::once_flag once[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        *dev_out = -1;
        return DeviceInfo{};
    }
    *dev_out = dev;
    std::call_once(once[dev], [dev]() {
        DeviceInfo d;
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cache[dev] = d;
    });
    return cache[dev];
}

// cudaFuncSetAttribute once per (kernel, device); `done` must be a flag word
// owned by that one kernel instantiation.
template <typename K>
int ensure_max_smem(K kernel, std::atomic<uint64_t>& done, int dev, int bytes) {
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return B2_OK;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    done.fetch_or(bit, std::memory_order_acq_rel);
    return B2_OK;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Threads per attention CTA at most (consumers + the producer warp); keeps
// the register cap at 128 per thread.
constexpr int kAttnMaxThreads = 512;
// Shared bytes of the attention kernel's misc area (first sequence, scan).
constexpr int kMiscBytes = 320;
// Batches up to this size keep their seq_lens in the attention kernel's shared memory.
constexpr int kSeqLenCache = 2048;

// ---------------------------------------------------------- attention plan

struct AttnPlan {
    int grid = 0, threads = 0, smem = 0;
    int combine_threads = 0;
    bool tensor_cores = false;  // paged_decode_tc_kernel instead of paged_decode_kernel
    int tc_stages = 0;
    int cpt = 1;  // paged_decode_kernel: 16-byte chunks per consumer thread
    AttnParams prm{};
    // workspace: [piece counters][seq_info][(m, l) partials][acc partials]
    size_t ws_cnt = 0, ws_info = 0, ws_ml = 0, ws_acc = 0, ws_total = 0;
};

// The tensor-core kernel serves 16-bit K/V with 8 kv heads of head_dim 128
// and 8, 16 or 32 query heads.  B2_ATTENTION_TENSOR_CORES=0 in the
// environment routes those shapes to the CUDA-core kernel instead (read once).
bool tc_disabled_by_env() {
    static const bool off = [] {
        const char* v = std::getenv("B2_ATTENTION_TENSOR_CORES");
        return v != nullptr && v[0] == '0';
    }();
    return off;
}

bool tc_eligible(const B2PagedAttnArgs* a) {
    const int qg = a->n_head / a->n_kv_head;
    return a->dtype != B2_F32 && a->head_dim == kTcHeadDim && a->n_kv_head == kTcKvHeads &&
           (qg == 1 || qg == 2 || qg == 4) &&
           static_cast<long long>(a->num_blocks) * a->n_layer * 2 < (1LL << 31) && !tc_disabled_by_env();
}

int tc_smem_bytes(int qg, int stages) {
    switch (qg) {
        case 1: return TcLayout<1>::bytes(stages);
        case 2: return TcLayout<2>::bytes(stages);
        default: return TcLayout<4>::bytes(stages);
    }
}

int check_attn_args(const B2PagedAttnArgs* a) {
    if (a == nullptr) return fail(B2_ERR_NULL, "args is NULL");
    if (!dtype_ok(a->dtype)) return fail(B2_ERR_DTYPE, "unknown dtype");
    if (a->out_dtype != B2_F32 && a->out_dtype != a->dtype)
        return fail(B2_ERR_DTYPE, "out_dtype must be F32 or equal to dtype");
    if (a->batch < 0) return fail(B2_ERR_SHAPE, "batch < 0");
    if (a->batch == 0) return B2_OK;
    if (!a->q || !a->kv_pool || !a->block_tables || !a->seq_lens || !a->out)
        return fail(B2_ERR_NULL, "q, kv_pool, block_tables, seq_lens and out are required");
    if (a->head_dim != 64 && a->head_dim != 128) return fail(B2_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
    if (a->n_kv_head <= 0 || a->n_head <= 0 || a->n_head % a->n_kv_head != 0)
        return fail(B2_ERR_SHAPE, "n_head must be a positive multiple of n_kv_head");
    const int qg = a->n_head / a->n_kv_head;
    const int es = dtype_size(a->dtype);
    if (!(qg == 1 || qg == 2 || qg == 4 || (qg == 8 && es == 4)))
        return fail(B2_ERR_UNSUPPORTED, "query-group size must be 1, 2 or 4 (8 for f32)");
    if (a->max_blocks_per_seq <= 0 || a->n_layer <= 0 || a->layer_idx < 0 || a->layer_idx >= a->n_layer ||
        a->num_blocks <= 0)
        return fail(B2_ERR_SHAPE, "max_blocks_per_seq, n_layer, layer_idx or num_blocks out of range");
    if (a->max_blocks_per_seq > (1 << 26) / B2_BLOCK_TOKENS) return fail(B2_ERR_SHAPE, "max_blocks_per_seq too large");
    if (static_cast<long long>(a->batch) * a->max_blocks_per_seq * B2_BLOCK_TOKENS >= (1LL << 31))
        return fail(B2_ERR_SHAPE, "batch * max_blocks_per_seq * 16 must stay below 2^31 token rows");
    if (a->q_row_stride < a->n_head * a->head_dim) return fail(B2_ERR_SHAPE, "q_row_stride < n_head*head_dim");
    if (a->flags != 0 && a->flags != B2_ATTN_INPUTS_READY && a->flags != B2_ATTN_NEWEST_ROW_PENDING)
        return fail(B2_ERR_SHAPE, "unknown flags");
    if (a->max_ctas < 0) return fail(B2_ERR_SHAPE, "max_ctas < 0");
    if (!aligned16(a->q) || !aligned16(a->kv_pool) || !aligned16(a->out) || (a->q_bias && !aligned16(a->q_bias)) ||
        (static_cast<long long>(a->q_row_stride) * es) % 16 != 0)
        return fail(B2_ERR_ALIGN, "q, q_bias, kv_pool and out must be 16-byte aligned, q_row_stride*elem 16-byte multiple");
    return B2_OK;
}

int plan_attention(const B2PagedAttnArgs* a, AttnPlan* pl) {
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    if (dev < 0 || di.sms <= 0) return fail(B2_ERR_DEVICE, "no current CUDA device");
    const int es = dtype_size(a->dtype);
    const int E = 16 / es;
    const int GL = a->head_dim / E;
    const int C = a->n_kv_head * GL;
    const int H = a->n_head;
    const int maxt = kAttnMaxThreads;
    if (tc_eligible(a)) {
        // One CTA per SM; as many 64-KiB stages as fit (3 for up to 32 heads).
        const int qg = H / a->n_kv_head;
        int stages = 4;
        while (stages > 2 && tc_smem_bytes(qg, stages) > di.max_smem_optin) --stages;
        if (tc_smem_bytes(qg, stages) <= di.max_smem_optin) {
            pl->tensor_cores = true;
            pl->tc_stages = stages;
            pl->grid = a->max_ctas > 0 ? std::min(di.sms, a->max_ctas) : di.sms;
            pl->threads = kTcThreads;
            pl->smem = tc_smem_bytes(qg, stages);
            pl->combine_threads = static_cast<int>(align_up(static_cast<size_t>(H) * GL, 32));
            pl->prm.ksplit = 1;
            const size_t slots = static_cast<size_t>(pl->grid) + a->batch;
            pl->ws_cnt = align_up(static_cast<size_t>(a->batch) * sizeof(unsigned), 256);
            pl->ws_info = align_up(static_cast<size_t>(a->batch) * sizeof(int2), 256);
            pl->ws_ml = align_up(slots * H * sizeof(float2), 256);
            pl->ws_acc = align_up(slots * H * a->head_dim * sizeof(float), 256);
            pl->ws_total = pl->ws_cnt + pl->ws_info + pl->ws_ml + pl->ws_acc;
            return B2_OK;
        }
    }
    const int qbytes = H * a->head_dim * es;
    // Plans, in order of preference:
    //  1. two CTAs per SM, a stage per paged block (16 rows), one chunk per consumer
    //     thread -- each CTA still gets a double-buffered ring, and one CTA's
    //     prologue and tail overlap the other's streaming;
    //  2. where a block does not fit that, two CTAs per SM with stages of 8 rows and
    //     two chunks per thread, if that leaves at least two token subgroups (GPT-2
    //     medium's 16 heads x 64: 48.7 -> 46.4 us per launch; with 25 heads only one
    //     subgroup fits and it is slower than plan 3);
    //  3. one CTA per SM, a stage per block, two chunks per thread (16-bit, up to two
    //     query heads per kv head): fewer shuffle levels and less repeated softmax
    //     bookkeeping, which the wide-head shapes' instruction count needs.
    // The 128-register cap limits a co-resident pair to 256 threads each.
    struct Cand {
        int cps, rows, cpt, min_k;
    };
    // The prologue leaves the clamped seq_lens in shared memory for the producer
    // warp (its first block-table read then needs no second trip to L2), for
    // batches up to kSeqLenCache.
    const int seq_cache = a->batch <= kSeqLenCache ? static_cast<int>(align_up(static_cast<size_t>(a->batch) * 4, 16)) : 0;
    const bool cpt2_ok = es == 2 && H / a->n_kv_head <= 2;
    // 4./5. last resorts for rows too wide for a ring of whole blocks (f32 with many heads, e.g. 25 x 64 fp32 =
    //    6.4 KB a row): one CTA per SM, stages of 8 or 4 rows.
    const Cand cands[5] = {{2, B2_BLOCK_TOKENS, 1, 1},
                           {2, B2_BLOCK_TOKENS / 2, 2, 2},
                           {1, B2_BLOCK_TOKENS, cpt2_ok ? 2 : 1, 1},
                           {1, B2_BLOCK_TOKENS / 2, cpt2_ok ? 2 : 1, 1},
                           {1, B2_BLOCK_TOKENS / 4, cpt2_ok ? 2 : 1, 1}};
    int best_k = 0, best_s = 0, best_cps = 0, best_cpt = 1, best_rows = 0;
    int slab = 0, off_meta = 0, stage = 0;
    for (const Cand& cd : cands) {
        if (cd.cpt == 2 && !cpt2_ok) continue;
        slab = cd.rows * a->n_kv_head * a->head_dim * es;
        off_meta = 2 * slab + qbytes;
        stage = static_cast<int>(align_up(off_meta + 16, 128));
        const int CT = C / cd.cpt;  // consumer threads per token subgroup
        const int smem_cap = cd.cps == 1 ? di.max_smem_optin : di.smem_per_sm / cd.cps - 1024;
        const int thread_cap = cd.cps == 1 ? maxt : 256;
        for (int k : {8, 6, 4, 3, 2, 1}) {  // token subgroups: more consumer warps to hide latency
            if (k < cd.min_k) break;
            const int ncons = static_cast<int>(align_up(static_cast<size_t>(k) * CT, 32));
            if (ncons + 64 > thread_cap) continue;  // + producer warp + bookkeeping warp
            if (k > 1 && k * CT > 512) continue;  // enough warps
            int s = (smem_cap - kMiscBytes - seq_cache - 512) / stage;  // 512: barriers + alignment padding
            if (s > 8) s = 8;
            if (s < 2) continue;
            best_k = k;
            best_s = s;
            best_cps = cd.cps;
            best_cpt = cd.cpt;
            best_rows = cd.rows;
            break;
        }
        if (best_k != 0) break;
    }
    if (best_k == 0) return fail(B2_ERR_UNSUPPORTED, "head shape does not fit the decode kernel's shared memory");
    const int CT = C / best_cpt;
    pl->cpt = best_cpt;
    if (a->batch > 16 * (static_cast<int>(align_up(static_cast<size_t>(best_k) * CT, 32)) + 32))
        return fail(B2_ERR_UNSUPPORTED, "batch too large for one launch");

    AttnParams& p = pl->prm;
    p.ksplit = best_k;
    p.ncons = static_cast<int>(align_up(static_cast<size_t>(best_k) * CT, 32));
    p.stages = best_s;
    p.stage_bytes = stage;
    p.stage_rows = best_rows;
    p.slab_bytes = slab;
    p.q_bytes = qbytes;
    p.off_meta = off_meta;
    // One-piece sequences are merged in shared memory, over the stage just
    // consumed: [ks][H][head_dim] fp32 states and [ks][H] (m, l) must fit it.
    p.local_merge = static_cast<long long>(best_k) * H * (a->head_dim * 4 + 8) <= stage ? 1 : 0;
    // At one CTA per SM (the wide-head shapes) every piece is folded that way
    // and leaves one partial instead of one per subgroup: a quarter of the
    // partial stores and merge loads (GPT-2 XL's 25 heads, 128 sequences:
    // 85.1 -> 80.8 us per launch).  At two CTAs per SM the consumers' wait at
    // a mid-range piece end costs more than it saves (batch 64 x 12 heads,
    // INPUTS_READY: 24.2 -> 24.7 us).
    p.fold_pieces = p.local_merge && best_cps == 1 ? 1 : 0;
    int off = best_s * stage;
    p.off_misc = off;
    off += kMiscBytes;
    p.off_seqlens = seq_cache > 0 ? off : -1;
    off += seq_cache;
    p.off_bars = off;
    off += (2 * best_s + 2 * kPieceRing + 1 + 2) * 8;  // stages full/empty, piece ring, book_done, merge barriers
    // An early-start launch writes nothing before griddepcontrol.wait, so a
    // CTA whose first piece ends in mid-range used to stall its consumers
    // there until the kernel ahead finished (median 2.5 us, up to 17 us, for
    // the quarter of the CTAs holding two pieces at batch 64 x 12 heads).  The
    // partials of that first piece go to this shared-memory stash instead,
    // and the bookkeeping warp copies them out after its own wait; the
    // consumers stream on.  Only where the stash fits next to the ring.
    // Flags 0: the speculative pass before the wait brings this CTA's first
    // two blocks into L2.  Deeper prefetches competed with the previous
    // launch's tail (batch 64 x 12 heads, back to back: 2 blocks 28.8 us,
    // 4: 29.8, 8: 31.4, 16: 31.9 per launch).
    p.spec_blocks = 2;
    p.off_stash = -1;
    if (a->flags != 0) {
        const int sk = p.fold_pieces ? 1 : best_k;
        const size_t stash = align_up(static_cast<size_t>(sk) * H * (a->head_dim * 4 + 8), 16);
        const int smem_cap = best_cps == 1 ? di.max_smem_optin : di.smem_per_sm / best_cps - 1024;
        const size_t at = align_up(static_cast<size_t>(off), 16);
        if (at + stash <= static_cast<size_t>(smem_cap)) {
            p.off_stash = static_cast<int>(at);
            off = static_cast<int>(at + stash);
        }
    }
    pl->smem = off;
    pl->threads = p.ncons + 64;
    pl->grid = a->max_ctas > 0 ? std::min(di.sms * best_cps, a->max_ctas) : di.sms * best_cps;
    // With B2_ATTN_INPUTS_READY this launch may start while the kernel before it
    // drains.  At two CTAs per SM every slot would be taken, so the next such
    // launch could not place a CTA until one of this launch's CTAs exits; leaving
    // sms / 16 slots free lets its first CTAs do their set-up and start streaming
    // during this launch's tail (back-to-back launches of batch 64 x 12 heads:
    // 24.0 -> 23.0 us; with flags 0 the smaller grid costs under 1 %).
    if (best_cps == 2 && a->flags == B2_ATTN_INPUTS_READY && a->max_ctas == 0) pl->grid -= di.sms / 16;
    pl->combine_threads = static_cast<int>(align_up(static_cast<size_t>(H) * GL, 32));

    // One partial per (CTA, sequence) pair and token subgroup; cta + b < grid + batch.
    const size_t slots = (static_cast<size_t>(pl->grid) + a->batch) * best_k;
    pl->ws_cnt = align_up(static_cast<size_t>(a->batch) * sizeof(unsigned), 256);
    pl->ws_info = align_up(static_cast<size_t>(a->batch) * sizeof(int2), 256);
    pl->ws_ml = align_up(slots * H * sizeof(float2), 256);
    pl->ws_acc = align_up(slots * H * a->head_dim * sizeof(float), 256);
    pl->ws_total = pl->ws_cnt + pl->ws_info + pl->ws_ml + pl->ws_acc;
    return B2_OK;
}

// Set while b2_paged_attention_host launches an early-start attention
// (B2_ATTN_INPUTS_READY / B2_ATTN_NEWEST_ROW_PENDING) behind the kernel that
// writes its inputs: that launch must then start only once the kernel before
// it has completed, so launch_pdl leaves the programmatic attribute off.
thread_local bool t_full_dependency = false;

// Launch with programmatic dependent launch: the kernel waits on
// griddepcontrol.wait before reading what the kernel before it wrote, so its
// launch and set-up overlap that kernel's tail.
template <typename K, typename... P>
int launch_pdl(K kern, dim3 grid, dim3 block, int smem, cudaStream_t stream, const P&... prm) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = t_full_dependency ? 0 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, prm...);
    if (e != cudaSuccess) {
        cudaGetLastError();
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    return launch_status();
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// The pool as a 4-D tensor for the tensor-core kernel's TMA boxes:
//   dim 0: head_dim elements (contiguous), box 64 (one 128-B swizzle row)
//   dim 1: 16 token rows of a slab, stride n_kv_head*head_dim elements, box 16
//   dim 2: kv head, stride head_dim elements, box 8
//   dim 3: slab index ((block * n_layer + layer) * 2 + K|V), box 1
// so one box lands as 128 rows (kv_head * 16 + token) of 128 B, swizzled.
int encode_kv_map(const B2PagedAttnArgs* a, CUtensorMap* map) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t es = 2;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kTcHeadDim), 16, static_cast<cuuint64_t>(kTcKvHeads),
                                static_cast<cuuint64_t>(a->num_blocks) * a->n_layer * 2};
    const cuuint64_t strides[3] = {kTcKvHeads * kTcHeadDim * es, kTcHeadDim * es,
                                   16 * kTcKvHeads * kTcHeadDim * es};
    const cuuint32_t box[4] = {64, 16, static_cast<cuuint32_t>(kTcKvHeads), 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, a->dtype == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           4, const_cast<void*>(a->kv_pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled rejected the KV pool layout");
    return B2_OK;
}

template <typename T, int QG>
int launch_tc_t(const AttnPlan& pl, const TcParams& tp, const CUtensorMap& map, cudaStream_t stream) {
    auto kern = paged_decode_tc_kernel<T, QG>;
    static std::atomic<uint64_t> smem_set{0};
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    const int rc = ensure_max_smem(kern, smem_set, dev, di.max_smem_optin);
    if (rc != B2_OK) return rc;
    return launch_pdl(kern, dim3(static_cast<unsigned>(pl.grid)), dim3(static_cast<unsigned>(pl.threads)), pl.smem,
                      stream, tp, map);
}

template <typename T>
int launch_tc(const AttnPlan& pl, const TcParams& tp, const CUtensorMap& map, int qg, cudaStream_t s) {
    switch (qg) {
        case 1: return launch_tc_t<T, 1>(pl, tp, map, s);
        case 2: return launch_tc_t<T, 2>(pl, tp, map, s);
        case 4: return launch_tc_t<T, 4>(pl, tp, map, s);
    }
    return fail(B2_ERR_UNSUPPORTED, "no tensor-core kernel for this head shape");
}

template <typename T, int DH, int QG, typename OutT, int CPT>
int launch_attn_c(const AttnPlan& pl, cudaStream_t stream) {
    constexpr int MAXT = kAttnMaxThreads;
    auto kern = paged_decode_kernel<T, DH, QG, MAXT, OutT, CPT>;
    static std::atomic<uint64_t> smem_set{0};  // one flag word per instantiation
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    const int rc = ensure_max_smem(kern, smem_set, dev, di.max_smem_optin);
    if (rc != B2_OK) return rc;
    return launch_pdl(kern, dim3(static_cast<unsigned>(pl.grid)), dim3(static_cast<unsigned>(pl.threads)), pl.smem,
                      stream, pl.prm);
}

template <typename T, int DH, int QG, typename OutT>
int launch_attn_o(const AttnPlan& pl, cudaStream_t stream) {
    if constexpr (sizeof(T) == 2 && QG <= 2) {
        if (pl.cpt == 2) return launch_attn_c<T, DH, QG, OutT, 2>(pl, stream);
    }
    return launch_attn_c<T, DH, QG, OutT, 1>(pl, stream);
}

// out_dtype is F32, or the input dtype (checked by check_attn_args).
template <typename T, int DH, int QG>
int launch_attn_t(const AttnPlan& pl, int out_dtype, cudaStream_t stream) {
    if (out_dtype == B2_F32) return launch_attn_o<T, DH, QG, float>(pl, stream);
    if constexpr (sizeof(T) == 2) return launch_attn_o<T, DH, QG, T>(pl, stream);
    return fail(B2_ERR_DTYPE, "16-bit output needs 16-bit inputs");
}

template <typename T>
int launch_attn_dh(const AttnPlan& pl, int dh, int qg, int out_dtype, cudaStream_t s) {
    if (dh == 64) {
        switch (qg) {
            case 1: return launch_attn_t<T, 64, 1>(pl, out_dtype, s);
            case 2: return launch_attn_t<T, 64, 2>(pl, out_dtype, s);
            case 4: return launch_attn_t<T, 64, 4>(pl, out_dtype, s);
            case 8:
                if constexpr (sizeof(T) == 4) return launch_attn_t<T, 64, 8>(pl, out_dtype, s);
                break;
        }
    } else {
        switch (qg) {
            case 1: return launch_attn_t<T, 128, 1>(pl, out_dtype, s);
            case 2: return launch_attn_t<T, 128, 2>(pl, out_dtype, s);
            case 4: return launch_attn_t<T, 128, 4>(pl, out_dtype, s);
            case 8:
                if constexpr (sizeof(T) == 4) return launch_attn_t<T, 128, 8>(pl, out_dtype, s);
                break;
        }
    }
    return fail(B2_ERR_UNSUPPORTED, "no kernel for this head shape");
}

template <int DH, int E>
int launch_combine_out(const CombineParams& c, int out_dtype, int batch, int threads, cudaStream_t s) {
    const dim3 grid(static_cast<unsigned>(batch)), block(static_cast<unsigned>(threads));
    if (out_dtype == B2_F32) return launch_pdl(paged_decode_combine_kernel<DH, E, float>, grid, block, 0, s, c);
    if constexpr (E == 8) {  // 16-bit outputs only come with 16-bit inputs (8 elements per chunk)
        if (out_dtype == B2_F16) return launch_pdl(paged_decode_combine_kernel<DH, E, __half>, grid, block, 0, s, c);
        return launch_pdl(paged_decode_combine_kernel<DH, E, __nv_bfloat16>, grid, block, 0, s, c);
    }
    return fail(B2_ERR_DTYPE, "16-bit output needs 16-bit inputs");
}

int launch_combine(const CombineParams& c, int dtype, int out_dtype, int dh, int batch, int threads,
                   cudaStream_t s) {
    const int E = 16 / dtype_size(dtype);
    if (dh == 64) return E == 8 ? launch_combine_out<64, 8>(c, out_dtype, batch, threads, s)
                                : launch_combine_out<64, 4>(c, out_dtype, batch, threads, s);
    return E == 8 ? launch_combine_out<128, 8>(c, out_dtype, batch, threads, s)
                  : launch_combine_out<128, 4>(c, out_dtype, batch, threads, s);
}

// Row-kernel grid: grid-stride loops over 16-byte chunks, a few waves of CTAs.
int row_grid(long long nchunks) {
    long long g = (nchunks + 255) / 256;
    if (g > 148LL * 16) g = 148LL * 16;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {

const char* b2_version(void) { return "b2decode 0.1 (sm_100a)"; }

const char* b2_last_error_string(void) { return g_last_error.c_str(); }

int b2_device_errors(uint32_t* bits_out) {
    if (bits_out == nullptr) return fail(B2_ERR_NULL, "bits_out is NULL");
    unsigned int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_errors, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_errors, &zero, sizeof(zero));
    if (e != cudaSuccess) {
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    *bits_out = v;
    return B2_OK;
}

// ------------------------------------------------------------- kv append

int b2_kv_append(const B2KvAppendArgs* a, b2_stream_t stream) {
    if (a == nullptr) return fail(B2_ERR_NULL, "args is NULL");
    if (!dtype_ok(a->dtype)) return fail(B2_ERR_DTYPE, "unknown dtype");
    if (a->batch < 0) return fail(B2_ERR_SHAPE, "batch < 0");
    if (a->batch == 0) return B2_OK;
    if (!a->kv_pool || !a->k || !a->v || !a->block_tables || !a->seq_lens)
        return fail(B2_ERR_NULL, "kv_pool, k, v, block_tables and seq_lens are required");
    if (a->head_dim != 64 && a->head_dim != 128) return fail(B2_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
    if (a->n_kv_head <= 0 || a->max_blocks_per_seq <= 0 || a->n_layer <= 0 || a->layer_idx < 0 ||
        a->layer_idx >= a->n_layer || a->num_blocks <= 0)
        return fail(B2_ERR_SHAPE, "n_kv_head, max_blocks_per_seq, n_layer, layer_idx or num_blocks out of range");
    if (a->kv_row_stride < a->n_kv_head * a->head_dim) return fail(B2_ERR_SHAPE, "kv_row_stride < n_kv_head*head_dim");
    if (a->seq_lens_post != nullptr && a->seq_lens_post == a->seq_lens)
        return fail(B2_ERR_SHAPE, "seq_lens_post must not alias seq_lens");
    const int es = dtype_size(a->dtype);
    if (!aligned16(a->kv_pool) || !aligned16(a->k) || !aligned16(a->v) || (a->k_bias && !aligned16(a->k_bias)) ||
        (a->v_bias && !aligned16(a->v_bias)) || (static_cast<long long>(a->kv_row_stride) * es) % 16 != 0)
        return fail(B2_ERR_ALIGN, "pointers must be 16-byte aligned, kv_row_stride*elem a 16-byte multiple");
    AppendParams p;
    p.pool = a->kv_pool;
    p.k = a->k;
    p.v = a->v;
    p.kv_row_stride = a->kv_row_stride;
    p.k_bias = a->k_bias;
    p.v_bias = a->v_bias;
    p.block_tables = a->block_tables;
    p.seq_lens = a->seq_lens;
    p.seq_lens_post = a->seq_lens_post;
    p.batch = a->batch;
    p.n_kv_head = a->n_kv_head;
    p.mbps = a->max_blocks_per_seq;
    p.layer_idx = a->layer_idx;
    p.n_layer = a->n_layer;
    p.num_blocks = a->num_blocks;
    const int E = 16 / es;
    const long long total = static_cast<long long>(a->batch) * 2 * a->n_kv_head * (a->head_dim / E);
    const int grid = static_cast<int>((total + 255) / 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->dtype == B2_F32)
        return a->head_dim == 64 ? launch_pdl(kv_append_kernel<float, 64>, grid, 256, 0, s, p)
                                 : launch_pdl(kv_append_kernel<float, 128>, grid, 256, 0, s, p);
    if (a->dtype == B2_F16)
        return a->head_dim == 64 ? launch_pdl(kv_append_kernel<__half, 64>, grid, 256, 0, s, p)
                                 : launch_pdl(kv_append_kernel<__half, 128>, grid, 256, 0, s, p);
    return a->head_dim == 64 ? launch_pdl(kv_append_kernel<__nv_bfloat16, 64>, grid, 256, 0, s, p)
                             : launch_pdl(kv_append_kernel<__nv_bfloat16, 128>, grid, 256, 0, s, p);
}

// ------------------------------------------------------- paged attention

size_t b2_paged_attention_workspace_bytes(const B2PagedAttnArgs* a) {
    if (check_attn_args(a) != B2_OK || a->batch == 0) return 0;
    AttnPlan pl;
    if (plan_attention(a, &pl) != B2_OK) return 0;
    return pl.ws_total;
}

}  // extern "C"

namespace b2 {
namespace {
// b2_paged_attention with the output going to `gather`'s arrays when non-NULL.
int paged_attention_impl(const B2PagedAttnArgs* a, void* ws, size_t ws_bytes, const B2OutputGather* gather,
                         b2_stream_t stream) {
    int rc = check_attn_args(a);
    if (rc != B2_OK) return rc;
    if (gather != nullptr) {
        const long long es_out = a->out_dtype == B2_F32 ? 4 : 2;
        if (gather->n_outs < 1 || gather->n_outs > B2_MAX_GATHER || gather->outs == nullptr)
            return fail(B2_ERR_SHAPE, "gather needs 1..B2_MAX_GATHER output arrays");
        if (gather->col_offset < 0 ||
            gather->row_stride < gather->col_offset + static_cast<long long>(a->n_head) * a->head_dim)
            return fail(B2_ERR_SHAPE, "gather row_stride must cover col_offset + n_head*head_dim");
        if ((gather->row_stride * es_out) % 16 != 0 || (gather->col_offset * es_out) % 16 != 0 ||
            !aligned16(gather->outs))
            return fail(B2_ERR_ALIGN, "gather row_stride and col_offset must be 16-byte multiples");
    }
    if (a->batch == 0) return B2_OK;
    AttnPlan pl;
    rc = plan_attention(a, &pl);
    if (rc != B2_OK) return rc;
    if (ws == nullptr || ws_bytes < pl.ws_total || !aligned16(ws))
        return fail(B2_ERR_WORKSPACE, "workspace missing, misaligned or too small");
    AttnParams& p = pl.prm;
    p.q = a->q;
    p.q_row_stride = a->q_row_stride;
    p.q_bias = a->q_bias;
    p.pool = a->kv_pool;
    p.block_tables = a->block_tables;
    p.seq_lens = a->seq_lens;
    p.batch = a->batch;
    p.n_head = a->n_head;
    p.n_kv_head = a->n_kv_head;
    p.mbps = a->max_blocks_per_seq;
    p.layer_idx = a->layer_idx;
    p.n_layer = a->n_layer;
    p.num_blocks = a->num_blocks;
    const float scale = a->scale > 0.0f ? a->scale : 1.0f / std::sqrt(static_cast<float>(a->head_dim));
    p.scale_log2 = scale * 1.4426950408889634f;
    char* base = static_cast<char*>(ws);
    p.counters = reinterpret_cast<unsigned int*>(base);
    p.seq_info = reinterpret_cast<int2*>(base + pl.ws_cnt);
    p.part_ml = reinterpret_cast<float2*>(base + pl.ws_cnt + pl.ws_info);
    p.part_acc = reinterpret_cast<float*>(base + pl.ws_cnt + pl.ws_info + pl.ws_ml);
    p.out.out = a->out;
    p.out.outs = gather ? gather->outs : nullptr;
    p.out.n = gather ? gather->n_outs : 0;
    p.out.row_stride = gather ? gather->row_stride : 0;
    p.out.col_offset = gather ? gather->col_offset : 0;
    p.early = a->flags;
    const int qg = a->n_head / a->n_kv_head;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (pl.tensor_cores) {
        CUtensorMap map;
        rc = encode_kv_map(a, &map);
        if (rc != B2_OK) return rc;
        TcParams tp;
        tp.q = a->q;
        tp.q_row_stride = a->q_row_stride;
        tp.q_bias = a->q_bias;
        tp.block_tables = a->block_tables;
        tp.seq_lens = a->seq_lens;
        tp.batch = a->batch;
        tp.mbps = a->max_blocks_per_seq;
        tp.layer_idx = a->layer_idx;
        tp.n_layer = a->n_layer;
        tp.num_blocks = a->num_blocks;
        tp.scale_log2 = p.scale_log2;
        tp.stages = pl.tc_stages;
        tp.seq_info = p.seq_info;
        tp.part_ml = p.part_ml;
        tp.part_acc = p.part_acc;
        rc = a->dtype == B2_F16 ? launch_tc<__half>(pl, tp, map, qg, s) : launch_tc<__nv_bfloat16>(pl, tp, map, qg, s);
    } else {
        // The CUDA-core kernel merges each sequence's pieces itself.
        if (a->dtype == B2_F32) return launch_attn_dh<float>(pl, a->head_dim, qg, a->out_dtype, s);
        if (a->dtype == B2_F16) return launch_attn_dh<__half>(pl, a->head_dim, qg, a->out_dtype, s);
        return launch_attn_dh<__nv_bfloat16>(pl, a->head_dim, qg, a->out_dtype, s);
    }
    if (rc != B2_OK) return rc;
    CombineParams cp;
    cp.seq_info = p.seq_info;
    cp.part_ml = p.part_ml;
    cp.part_acc = p.part_acc;
    cp.out = p.out;
    cp.n_head = a->n_head;
    cp.ksplit = p.ksplit;
    return launch_combine(cp, a->dtype, a->out_dtype, a->head_dim, a->batch, pl.combine_threads, s);
}
}  // namespace
}  // namespace b2

extern "C" {

int b2_paged_attention(const B2PagedAttnArgs* a, void* ws, size_t ws_bytes, b2_stream_t stream) {
    return b2::paged_attention_impl(a, ws, ws_bytes, nullptr, stream);
}

int b2_paged_attention_gather(const B2PagedAttnArgs* a, void* ws, size_t ws_bytes, const B2OutputGather* gather,
                              b2_stream_t stream) {
    if (gather == nullptr) return fail(B2_ERR_NULL, "gather is NULL");
    return b2::paged_attention_impl(a, ws, ws_bytes, gather, stream);
}

namespace {
// Waits for the stream by polling it: the host call returns within about a
// microsecond of the GPU finishing, where cudaStreamSynchronize under the
// default blocking-sync policy can add several microseconds of wake-up.
// This host-buffer entry point is a synchronous, latency-bound call by
// design, so it spends a host core spinning.
cudaError_t wait_stream_polling(cudaStream_t s) {
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e != cudaErrorNotReady) return e;
    }
}
}  // namespace

namespace b2 {
// The uploads of one b2_paged_attention_host call when every host buffer is
// page-locked and mapped: pieces of 16-byte units (both sides 16-byte
// aligned) or of single bytes, walked as one index space.
constexpr int kMaxHostPieces = 6;
struct HostPieces {
    char* dst[kMaxHostPieces];
    const char* src[kMaxHostPieces];  // device addresses of the mapped host pages
    unsigned long long units[kMaxHostPieces];
    int wide[kMaxHostPieces];  // 16-byte units (1) or bytes (0)
    int n;
    unsigned long long total;
};

// Reads the call's inputs straight out of mapped host memory over the bus and
// stores them where the attention launch reads them: the loads of the whole
// upload are in flight at once (one unit per thread at the sizes a decode
// step uploads), with no copy-engine set-up on the call's critical path.
// ld.global.cv fetches every line again, so a host buffer refilled between
// calls is never served from a cached copy.  The attention launch after it
// may start (griddepcontrol) and waits for this grid before reading.
__global__ void __launch_bounds__(256) pull_host_inputs_kernel(HostPieces g) {
    pdl_launch_dependents();
    const unsigned long long nth = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
    for (unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < g.total;
         i += nth) {
        int s = 0;
        unsigned long long k = i;
        while (s + 1 < g.n && k >= g.units[s]) k -= g.units[s++];
        if (g.wide[s])
            reinterpret_cast<uint4*>(g.dst[s])[k] = __ldcv(reinterpret_cast<const uint4*>(g.src[s]) + k);
        else
            reinterpret_cast<unsigned char*>(g.dst[s])[k] = __ldcv(reinterpret_cast<const unsigned char*>(g.src[s]) + k);
    }
}
}  // namespace b2

namespace {

// The device address of page-locked host memory mapped into the device's
// address space, or nullptr (pageable memory, device memory, failure).
const char* mapped_host_address(const void* h) {
    cudaPointerAttributes pa;
    const char* d = nullptr;
    if (cudaPointerGetAttributes(&pa, h) == cudaSuccess && pa.type == cudaMemoryTypeHost)
        d = static_cast<const char*>(pa.devicePointer);
    cudaGetLastError();
    return d;
}
}  // namespace

int b2_paged_attention_host(const B2PagedAttnArgs* a, const B2AttnHostIO* io, void* ws, size_t ws_bytes,
                            b2_stream_t stream) {
    using namespace b2;
    if (io == nullptr) return fail(B2_ERR_NULL, "io is NULL");
    int rc = check_attn_args(a);
    if (rc != B2_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    struct Up {
        char* dst;
        const char* src;
        size_t bytes;
    } up[3];
    int n = 0;
    if (a->batch > 0) {
        const size_t es = static_cast<size_t>(dtype_size(a->dtype));
        const size_t qn = static_cast<size_t>(a->batch - 1) * a->q_row_stride + static_cast<size_t>(a->n_head) * a->head_dim;
        if (io->q) up[n++] = {static_cast<char*>(const_cast<void*>(a->q)), static_cast<const char*>(io->q), qn * es};
        if (io->block_tables)
            up[n++] = {reinterpret_cast<char*>(const_cast<int32_t*>(a->block_tables)),
                       reinterpret_cast<const char*>(io->block_tables),
                       static_cast<size_t>(a->batch) * a->max_blocks_per_seq * sizeof(int32_t)};
        if (io->seq_lens)
            up[n++] = {reinterpret_cast<char*>(const_cast<int32_t*>(a->seq_lens)),
                       reinterpret_cast<const char*>(io->seq_lens), static_cast<size_t>(a->batch) * sizeof(int32_t)};
    }
    // Every upload from mapped page-locked memory: one small kernel reads them
    // all over the bus (pull_host_inputs_kernel).  Otherwise one copy per run
    // of uploads that are contiguous on both sides.
    const char* mapped_src[3] = {nullptr, nullptr, nullptr};
    bool pull = n > 0;
    for (int i = 0; i < n && pull; ++i) pull = (mapped_src[i] = mapped_host_address(up[i].src)) != nullptr;
    if (pull) {
        HostPieces g{};
        for (int i = 0; i < n; ++i) {
            size_t head = 0;
            if (aligned16(up[i].dst) && aligned16(mapped_src[i]) && up[i].bytes >= 16) {
                head = up[i].bytes & ~static_cast<size_t>(15);
                g.dst[g.n] = up[i].dst;
                g.src[g.n] = mapped_src[i];
                g.units[g.n] = head / 16;
                g.wide[g.n++] = 1;
            }
            if (up[i].bytes > head) {
                g.dst[g.n] = up[i].dst + head;
                g.src[g.n] = mapped_src[i] + head;
                g.units[g.n] = up[i].bytes - head;
                g.wide[g.n++] = 0;
            }
        }
        for (int i = 0; i < g.n; ++i) g.total += g.units[i];
        if (g.total > 0) {
            const unsigned long long blocks = std::min<unsigned long long>((g.total + 255) / 256, 4096);
            pull_host_inputs_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(g);
            rc = launch_status();
            if (rc != B2_OK) return rc;
        }
    } else {
        for (int i = 0; i < n;) {
            Up c = up[i++];
            while (i < n && up[i].dst == c.dst + c.bytes && up[i].src == c.src + c.bytes) c.bytes += up[i++].bytes;
            const cudaError_t e = cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) {
                cudaGetLastError();
                return fail(static_cast<int>(e), cudaGetErrorString(e));
            }
        }
    }
    // Output straight into the caller's buffer when it is page-locked host
    // memory mapped into the device's address space: the stores cross PCIe
    // while the kernel runs instead of in a copy after it.
    void* mapped_out = io->out ? const_cast<char*>(mapped_host_address(io->out)) : nullptr;
    // The inputs are written by the pull kernel: a launch that reads them
    // before griddepcontrol.wait (a nonzero flags value) must not start until
    // that kernel has completed.
    struct FullDependency {
        bool prev;
        explicit FullDependency(bool on) : prev(t_full_dependency) { t_full_dependency = on; }
        ~FullDependency() { t_full_dependency = prev; }
    } full_dependency(pull && a->flags != 0);
    if (mapped_out != nullptr && aligned16(mapped_out)) {
        B2PagedAttnArgs direct = *a;
        direct.out = mapped_out;
        rc = paged_attention_impl(&direct, ws, ws_bytes, nullptr, s);
        if (rc != B2_OK) return rc;
        const cudaError_t e = wait_stream_polling(s);
        if (e != cudaSuccess) return fail(static_cast<int>(e), cudaGetErrorString(e));
        return B2_OK;
    }
    rc = paged_attention_impl(a, ws, ws_bytes, nullptr, s);
    if (rc != B2_OK) return rc;
    if (io->out && a->batch > 0) {
        const size_t out_bytes = static_cast<size_t>(a->batch) * a->n_head * a->head_dim * dtype_size(a->out_dtype);
        const cudaError_t e = cudaMemcpyAsync(io->out, a->out, out_bytes, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(static_cast<int>(e), cudaGetErrorString(e));
        }
    }
    const cudaError_t e = wait_stream_polling(s);
    if (e != cudaSuccess) return fail(static_cast<int>(e), cudaGetErrorString(e));
    return B2_OK;
}

int b2_tp_barrier_timed(uint32_t* local_flags, uint32_t* const* peer_flags, int32_t rank, int32_t n,
                        const uint32_t* epoch, int32_t slot, uint64_t limit_ns, b2_stream_t stream) {
    if (!local_flags || !peer_flags || !epoch) return fail(B2_ERR_NULL, "local_flags, peer_flags and epoch are required");
    if (n < 1 || n > B2_MAX_GATHER || rank < 0 || rank >= n || slot < 0) return fail(B2_ERR_SHAPE, "bad rank / n / slot");
    if (limit_ns == 0 || limit_ns > 60000000000ull) return fail(B2_ERR_SHAPE, "limit_ns must be in (0, 60 s]");
    tp_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(local_flags, peer_flags, rank, n, epoch, slot,
                                                                        limit_ns);
    return launch_status();
}

int b2_tp_barrier(uint32_t* local_flags, uint32_t* const* peer_flags, int32_t rank, int32_t n, const uint32_t* epoch,
                  int32_t slot, b2_stream_t stream) {
    return b2_tp_barrier_timed(local_flags, peer_flags, rank, n, epoch, slot, kTpWaitLimitNs, stream);
}

int b2_device_error_word(uint32_t** out) {
    if (out == nullptr) return fail(B2_ERR_NULL, "out is NULL");
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_device_errors);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(static_cast<int>(e), cudaGetErrorString(e));
    }
    *out = static_cast<uint32_t*>(p);
    return B2_OK;
}

int b2_raise_device_error(uint32_t bits, b2_stream_t stream) {
    raise_device_error_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(bits);
    return launch_status();
}

int b2_tp_epoch_bump(uint32_t* epoch, b2_stream_t stream) {
    if (!epoch) return fail(B2_ERR_NULL, "epoch is NULL");
    tp_epoch_bump_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(epoch);
    return launch_status();
}

}  // extern "C"

// --------------------------------------- attention with a built-in workspace
// For callers that may not allocate device memory on their decode path (a
// plugin whose host runtime owns all device memory through its own pool, a
// hard real-time loop that cannot take cudaMalloc's implicit synchronisation),
// the workspace can come from this fixed array instead.  It is part of the
// module, so every device that loads the library holds it until exit.  Host
// code must not pass `g_noalloc_scratch` itself to a kernel: on the host that
// name is only a stand-in for the symbol; the device address comes from
// cudaGetSymbolAddress, looked up once per device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[B2_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
// Per device: the array's device address once a lookup has succeeded.  A
// failed lookup is not remembered, so the next call tries again.  The cached
// address belongs to the device's primary context: after cudaDeviceReset a
// later call would use a stale address, so this entry point does not support
// a reset (the header says so).
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
    int dev = -1;
    const cudaError_t ge = cudaGetDevice(&dev);
    if (ge != cudaSuccess) {
        cudaGetLastError();
        return fail(static_cast<int>(ge), (std::string("cudaGetDevice failed: ") + cudaGetErrorString(ge)).c_str());
    }
    if (dev < 0 || dev >= kMaxDevices)
        return fail(B2_ERR_DEVICE, "b2_paged_attention_noalloc supports device ordinals 0..63 only");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        // First call on this device (it is current here): its address of the array.
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            g_last_error = std::string("cudaGetSymbolAddress for the built-in scratch failed: ") + cudaGetErrorString(e);
            return e != cudaSuccess ? static_cast<int>(e) : B2_ERR_DEVICE;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return B2_OK;
}
}  // namespace

extern "C" int b2_paged_attention_noalloc(const B2PagedAttnArgs* a, b2_stream_t stream) {
    int rc = check_attn_args(a);
    if (rc != B2_OK) return rc;
    if (a->batch == 0) return B2_OK;
    AttnPlan pl;
    rc = plan_attention(a, &pl);
    if (rc != B2_OK) return rc;
    if (pl.ws_total > B2_NOALLOC_SCRATCH_BYTES) {
        char msg[200];
        std::snprintf(msg, sizeof(msg),
                      "this shape needs a %zu-byte workspace, more than the %u-byte built-in scratch of "
                      "b2_paged_attention_noalloc; use b2_paged_attention with a caller-provided workspace",
                      pl.ws_total, static_cast<unsigned>(B2_NOALLOC_SCRATCH_BYTES));
        return fail(B2_ERR_WORKSPACE, msg);
    }
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc != B2_OK) return rc;
    // The array keeps whatever the last call left in it.  A completed call
    // leaves its piece counters at zero, but one that gave up on a bounded
    // wait (B2_DEVERR_TIMEOUT) may not, and a stale count would make a later
    // call merge a sequence too early or never.  So every call clears the
    // counter region first, on its own stream (no allocation).
    const cudaError_t me = cudaMemsetAsync(scratch, 0, pl.ws_cnt, static_cast<cudaStream_t>(stream));
    if (me != cudaSuccess) {
        cudaGetLastError();
        return fail(static_cast<int>(me), cudaGetErrorString(me));
    }
    return b2_paged_attention(a, scratch, B2_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" {

// ------------------------------------------------------------ row kernels

int b2_add_layernorm(int32_t dtype, void* out, void* residual_out, const void* x, const void* bias,
                     const void* residual_in, const void* gamma, const void* beta, int32_t batch, int32_t d_model,
                     float eps, b2_stream_t stream) {
    if (!dtype_ok(dtype)) return fail(B2_ERR_DTYPE, "unknown dtype");
    if (batch < 0 || d_model <= 0) return fail(B2_ERR_SHAPE, "batch < 0 or d_model <= 0");
    if (batch == 0) return B2_OK;
    if (!out || !residual_in || !gamma || !beta) return fail(B2_ERR_NULL, "out, residual_in, gamma, beta required");
    const int E = 16 / dtype_size(dtype);
    if (d_model % E != 0) return fail(B2_ERR_SHAPE, "d_model*elem must be a multiple of 16 bytes");
    if (!aligned16(out) || !aligned16(residual_in) || !aligned16(gamma) || !aligned16(beta) ||
        (x && !aligned16(x)) || (bias && !aligned16(bias)) || (residual_out && !aligned16(residual_out)))
        return fail(B2_ERR_ALIGN, "pointers must be 16-byte aligned");
    // One CTA per row, one to four 16-byte chunks per thread.
    const int nch = d_model / E;
    const int per_thread = nch <= 1024 ? 1 : (nch <= 2048 ? 2 : 4);
    if (nch > 4 * 1024) return fail(B2_ERR_UNSUPPORTED, "d_model too large for the one-CTA-per-row kernel");
    const int threads = static_cast<int>(align_up(static_cast<size_t>((nch + per_thread - 1) / per_thread), 32));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define B2_LN_LAUNCH(T, N)                                                                                   \
    return launch_pdl(add_layernorm_kernel<T, N>, batch, threads, 0, s, static_cast<T*>(out),                \
                      static_cast<T*>(residual_out), static_cast<const T*>(x), static_cast<const T*>(bias), \
                      static_cast<const T*>(residual_in), static_cast<const T*>(gamma),                     \
                      static_cast<const T*>(beta), static_cast<int>(d_model), eps)
#define B2_LN_DISPATCH(T)                      \
    if (per_thread == 1) B2_LN_LAUNCH(T, 1);      \
    else if (per_thread == 2) B2_LN_LAUNCH(T, 2); \
    else B2_LN_LAUNCH(T, 4);
    if (dtype == B2_F32) {
        B2_LN_DISPATCH(float)
    } else if (dtype == B2_F16) {
        B2_LN_DISPATCH(__half)
    } else {
        B2_LN_DISPATCH(__nv_bfloat16)
    }
#undef B2_LN_DISPATCH
#undef B2_LN_LAUNCH
    return launch_status();
}

static int check_rowwise(int32_t dtype, const void* out, const void* x, const void* bias, int32_t batch, int32_t dim) {
    if (!dtype_ok(dtype)) return fail(B2_ERR_DTYPE, "unknown dtype");
    if (batch < 0 || dim <= 0) return fail(B2_ERR_SHAPE, "batch < 0 or dim <= 0");
    if (batch > 0 && (!out || !x || !bias)) return fail(B2_ERR_NULL, "out, x and bias are required");
    if (dim % (16 / dtype_size(dtype)) != 0) return fail(B2_ERR_SHAPE, "dim*elem must be a multiple of 16 bytes");
    if (!aligned16(out) || !aligned16(x) || !aligned16(bias)) return fail(B2_ERR_ALIGN, "pointers must be 16-byte aligned");
    return B2_OK;
}

int b2_bias_gelu(int32_t dtype, void* out, const void* x, const void* bias, int32_t batch, int32_t d_ff,
                 b2_stream_t stream) {
    int rc = check_rowwise(dtype, out, x, bias, batch, d_ff);
    if (rc != B2_OK || batch == 0) return rc;
    const int rc_chunks = d_ff / (16 / dtype_size(dtype));
    const long long n = static_cast<long long>(batch) * rc_chunks;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int g = row_grid(n);
    if (dtype == B2_F32)
        return launch_pdl(bias_gelu_kernel<float>, g, 256, 0, s, static_cast<float*>(out),
                          static_cast<const float*>(x), static_cast<const float*>(bias), n, rc_chunks);
    if (dtype == B2_F16)
        return launch_pdl(bias_gelu_kernel<__half>, g, 256, 0, s, static_cast<__half*>(out),
                          static_cast<const __half*>(x), static_cast<const __half*>(bias), n, rc_chunks);
    return launch_pdl(bias_gelu_kernel<__nv_bfloat16>, g, 256, 0, s, static_cast<__nv_bfloat16*>(out),
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(bias), n, rc_chunks);
}

int b2_add_bias(int32_t dtype, void* out, const void* x, const void* bias, int32_t batch, int32_t dim,
                b2_stream_t stream) {
    int rc = check_rowwise(dtype, out, x, bias, batch, dim);
    if (rc != B2_OK || batch == 0) return rc;
    const int rc_chunks = dim / (16 / dtype_size(dtype));
    const long long n = static_cast<long long>(batch) * rc_chunks;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int g = row_grid(n);
    if (dtype == B2_F32)
        add_bias_kernel<float><<<g, 256, 0, s>>>(static_cast<float*>(out), static_cast<const float*>(x),
                                                 static_cast<const float*>(bias), n, rc_chunks);
    else if (dtype == B2_F16)
        add_bias_kernel<__half><<<g, 256, 0, s>>>(static_cast<__half*>(out), static_cast<const __half*>(x),
                                                  static_cast<const __half*>(bias), n, rc_chunks);
    else
        add_bias_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<__nv_bfloat16*>(out),
                                                         static_cast<const __nv_bfloat16*>(x),
                                                         static_cast<const __nv_bfloat16*>(bias), n, rc_chunks);
    return launch_status();
}

int b2_add_one(int32_t* out, const int32_t* in, int32_t batch, b2_stream_t stream) {
    if (batch < 0) return fail(B2_ERR_SHAPE, "batch < 0");
    if (batch == 0) return B2_OK;
    if (!out || !in) return fail(B2_ERR_NULL, "out and in are required");
    add_one_kernel<<<(batch + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(out, in, batch);
    return launch_status();
}

int b2_embedding(int32_t dtype, void* out, const void* wte, const void* wpe, const int32_t* token_ids,
                 const int32_t* positions, int32_t batch, int32_t d_model, int32_t vocab, int32_t n_pos,
                 b2_stream_t stream) {
    if (!dtype_ok(dtype)) return fail(B2_ERR_DTYPE, "unknown dtype");
    if (batch < 0 || d_model <= 0 || vocab <= 0 || n_pos <= 0) return fail(B2_ERR_SHAPE, "bad sizes");
    if (batch == 0) return B2_OK;
    if (!out || !wte || !wpe || !token_ids || !positions) return fail(B2_ERR_NULL, "all pointers are required");
    const int E = 16 / dtype_size(dtype);
    if (d_model % E != 0) return fail(B2_ERR_SHAPE, "d_model*elem must be a multiple of 16 bytes");
    if (!aligned16(out) || !aligned16(wte) || !aligned16(wpe)) return fail(B2_ERR_ALIGN, "pointers must be 16-byte aligned");
    const int rcn = d_model / E;
    const int g = row_grid(static_cast<long long>(batch) * rcn);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == B2_F32)
        embedding_kernel<float><<<g, 256, 0, s>>>(static_cast<float*>(out), static_cast<const float*>(wte),
                                                  static_cast<const float*>(wpe), token_ids, positions, batch, rcn,
                                                  vocab, n_pos);
    else if (dtype == B2_F16)
        embedding_kernel<__half><<<g, 256, 0, s>>>(static_cast<__half*>(out), static_cast<const __half*>(wte),
                                                   static_cast<const __half*>(wpe), token_ids, positions, batch, rcn,
                                                   vocab, n_pos);
    else
        embedding_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<__nv_bfloat16*>(out),
                                                          static_cast<const __nv_bfloat16*>(wte),
                                                          static_cast<const __nv_bfloat16*>(wpe), token_ids,
                                                          positions, batch, rcn, vocab, n_pos);
    return launch_status();
}

int b2_argmax_rows(int32_t dtype, int32_t* out_tokens, const void* logits, int64_t row_stride, int32_t batch,
                   int32_t vocab, b2_stream_t stream) {
    if (!dtype_ok(dtype)) return fail(B2_ERR_DTYPE, "unknown dtype");
    if (batch < 0 || vocab <= 0 || row_stride < vocab) return fail(B2_ERR_SHAPE, "bad sizes (row_stride < vocab?)");
    if (batch == 0) return B2_OK;
    if (!out_tokens || !logits) return fail(B2_ERR_NULL, "out_tokens and logits are required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = aligned16(logits) && (row_stride * dtype_size(dtype)) % 16 == 0;
    const long long st = row_stride;
#define B2_ARGMAX(T)                                                                                     \
    (vec ? argmax_kernel<T, true><<<batch, 512, 0, s>>>(out_tokens, static_cast<const T*>(logits), vocab, st) \
         : argmax_kernel<T, false><<<batch, 512, 0, s>>>(out_tokens, static_cast<const T*>(logits), vocab, st))
    if (dtype == B2_F32) B2_ARGMAX(float);
    else if (dtype == B2_F16) B2_ARGMAX(__half);
    else B2_ARGMAX(__nv_bfloat16);
#undef B2_ARGMAX
    return launch_status();
}

int b2_argmax(int32_t dtype, int32_t* out_tokens, const void* logits, int32_t batch, int32_t vocab,
              b2_stream_t stream) {
    return b2_argmax_rows(dtype, out_tokens, logits, vocab, batch, vocab, stream);
}

}  // extern "C"

// ------------------------------------------------------------ linear layers
namespace b2 {
namespace {

struct LinPlan {
    int split = 1;    // CTAs per cluster, splitting K
    int n_tiles = 0;  // 128-feature tiles
    int chunks = 0;   // batch chunks of bn rows
    int bn = 16;
    int kb_total = 0;
    int stages = 1;
    int smem = 0;
};

// Clusters of `split` CTAs of `kern` (smem bytes each) the device holds at
// once; cached per (kernel, device, split, smem).
int linear_max_clusters(const void* kern, int dev, int split, int smem, int* out) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, int>, int> cache;
    const auto key = std::make_tuple(kern, dev, split, smem);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return B2_OK;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(split));
    cfg.blockDim = dim3(kLinThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(split);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) {
        cudaGetLastError();
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = n;
    *out = n;
    return B2_OK;
}

// Grid = split x n_tiles x chunks: `split` CTAs (one cluster) share each
// 128-feature tile and split its K range, so narrow layers still spread their
// weight stream over the GPU.
int plan_linear(const B2LinearArgs* a, const void* kern, LinPlan* pl) {
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    if (dev < 0 || di.sms <= 0) return fail(B2_ERR_DEVICE, "no current CUDA device");
    pl->chunks = (a->batch + kLinMaxCols - 1) / kLinMaxCols;
    const int per = (a->batch + pl->chunks - 1) / pl->chunks;
    pl->bn = (std::max(per, 16) + 15) / 16 * 16;
    pl->kb_total = (a->in_features + kLinKBlock - 1) / kLinKBlock;
    pl->n_tiles = (a->out_features + kLinRows - 1) / kLinRows;
    if (pl->n_tiles > 65535 || pl->chunks > 65535) return fail(B2_ERR_SHAPE, "out_features or batch too large");
    // The split doubles while the grid is still smaller than the SM count and
    // all its clusters fit on the device at once (one wave: the cluster
    // scheduler places a cluster's CTAs on distinct SMs of one GPC, so the
    // number of resident clusters drops as they grow).
    const long long tiles = static_cast<long long>(pl->n_tiles) * pl->chunks;
    bool have = false;
    for (int split = 1; split <= kLinMaxSplit && split <= pl->kb_total; split *= 2) {
        if (split > 1 && tiles * (split / 2) >= di.sms) break;
        const int max_kb = (pl->kb_total + split - 1) / split;
        int stages = std::min(max_kb, 6);
        while (stages > 1 && LinLayout::bytes(pl->bn, stages, split) > di.max_smem_optin) --stages;
        int smem = LinLayout::bytes(pl->bn, stages, split);
        // The CTAs one SM can hold must fit in its 512 TMEM columns together:
        // a CTA left waiting in tcgen05.alloc while the CTAs holding the
        // columns wait for it at a cluster barrier would never proceed.
        // Shared memory bounds the residency (1 KiB of it is reserved per CTA).
        const int max_res = 512 / static_cast<int>(lin_tmem_cols(pl->bn));
        smem = std::max(smem, di.smem_per_sm / (max_res + 1) + 1 - 1024);
        if (smem > di.max_smem_optin) break;
        if (split > 1) {
            int fit = 0;
            const int rc = linear_max_clusters(kern, dev, split, smem, &fit);
            if (rc != B2_OK) return rc;
            if (tiles > fit) break;
        }
        pl->split = split;
        pl->stages = stages;
        pl->smem = smem;
        have = true;
    }
    if (!have) return fail(B2_ERR_UNSUPPORTED, "linear: tile does not fit in shared memory");
    return B2_OK;
}

// Row-major [rows][inner] matrix (row stride `ld` elements) as a 2-D tensor
// map with boxes of box_rows x 64 elements, 128-byte swizzled.  Boxes that
// reach past the matrix read zeros.
int encode_rows_map(CUtensorMap* map, int dtype, const void* base, long long inner, long long rows, long long ld,
                    int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kLinKBlock), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, dtype == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled rejected a linear-layer operand");
    return B2_OK;
}

// The output [batch][out_features] (row stride ld elements) as a 2-D tensor
// map for TMA stores of box_cols x box_rows tiles, unswizzled (the staged tile
// is row-major); parts of a box outside the matrix are not written.
int encode_out_map(CUtensorMap* map, int dtype, void* base, long long cols, long long rows, long long ld, int box_cols,
                   int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, dtype == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled rejected the linear-layer output");
    return B2_OK;
}

// Plans, encodes the operand maps and launches one instantiation.
template <typename T, int EPI, bool BIAS>
int linear_t(const B2LinearArgs* a, cudaStream_t stream) {
    auto kern = linear_tc_kernel<T, EPI, BIAS>;
    static std::atomic<uint64_t> smem_set{0};
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    int rc = ensure_max_smem(kern, smem_set, dev, di.max_smem_optin);
    if (rc != B2_OK) return rc;
    LinPlan pl;
    rc = plan_linear(a, reinterpret_cast<const void*>(kern), &pl);
    if (rc != B2_OK) return rc;
    CUtensorMap wm, xm, ym;
    rc = encode_rows_map(&wm, a->dtype, a->w, a->in_features, a->out_features, a->in_features, kLinRows);
    if (rc != B2_OK) return rc;
    rc = encode_rows_map(&xm, a->dtype, a->x, a->in_features, a->batch, a->x_row_stride, pl.bn);
    if (rc != B2_OK) return rc;
    rc = encode_out_map(&ym, a->dtype, a->y, a->out_features, a->batch, a->y_row_stride, kLinRows / pl.split, pl.bn);
    if (rc != B2_OK) return rc;
    LinParams lp;
    lp.bias = a->bias;
    lp.y = a->y;
    lp.ldy = a->y_row_stride;
    lp.batch = a->batch;
    lp.n_out = a->out_features;
    lp.bn = pl.bn;
    lp.kb_total = pl.kb_total;
    lp.stages = pl.stages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(pl.split), static_cast<unsigned>(pl.n_tiles),
                       static_cast<unsigned>(pl.chunks));
    cfg.blockDim = dim3(kLinThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(pl.split);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pl.split > 1 ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, lp, wm, xm, ym);
    if (e != cudaSuccess) {
        cudaGetLastError();
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    return launch_status();
}

template <typename T>
int linear_epi(const B2LinearArgs* a, cudaStream_t s) {
    const bool bias = a->bias != nullptr;
    if (a->epilogue == B2_LINEAR_GELU)
        return bias ? linear_t<T, B2_LINEAR_GELU, true>(a, s) : linear_t<T, B2_LINEAR_GELU, false>(a, s);
    return bias ? linear_t<T, B2_LINEAR_STORE, true>(a, s) : linear_t<T, B2_LINEAR_STORE, false>(a, s);
}

}  // namespace
}  // namespace b2

extern "C" int b2_linear(const B2LinearArgs* a, b2_stream_t stream) {
    using namespace b2;
    if (a == nullptr) return fail(B2_ERR_NULL, "args is NULL");
    if (a->dtype != B2_F16 && a->dtype != B2_BF16)
        return fail(B2_ERR_DTYPE, "b2_linear runs F16 and BF16 on the tensor cores (F32 callers keep cuBLAS)");
    if (a->epilogue != B2_LINEAR_STORE && a->epilogue != B2_LINEAR_GELU) return fail(B2_ERR_SHAPE, "unknown epilogue");
    if (a->batch < 0 || a->in_features <= 0 || a->out_features <= 0) return fail(B2_ERR_SHAPE, "bad sizes");
    if (a->batch == 0) return B2_OK;
    if (!a->x || !a->w || !a->y) return fail(B2_ERR_NULL, "x, w and y are required");
    if (a->x_row_stride < a->in_features || a->y_row_stride < a->out_features)
        return fail(B2_ERR_SHAPE, "row strides must cover in_features / out_features");
    if (a->in_features % 8 != 0 || a->x_row_stride % 8 != 0 || a->y_row_stride % 8 != 0 || !aligned16(a->x) ||
        !aligned16(a->w) || !aligned16(a->y))
        return fail(B2_ERR_ALIGN,
                    "x, w and y must be 16-byte aligned with in_features, x_row_stride and y_row_stride multiples of 8");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return a->dtype == B2_F16 ? linear_epi<__half>(a, s) : linear_epi<__nv_bfloat16>(a, s);
}

// ------------------------------------------------------------ lm_head + argmax
namespace b2 {
namespace {

struct LmPlan {
    int chunks = 0, vn = 0, kb_total = 0, n_tiles = 0, grid = 0, stages = 0, smem = 0;
};

size_t lm_workspace_bytes(int batch) {
    return align_up(16 + static_cast<size_t>(batch > 0 ? batch : 0) * sizeof(unsigned long long), 256);
}

// Work items of vn vocabulary rows x 128 batch rows, whole K per item; one
// persistent CTA per SM (at most one per item).
// vn (a multiple of 16, at most 256) is set by the smallest whole number of
// items per SM that keeps it within 256, so the items spread evenly (vocab
// 50257 at batch <= 128: 176 rows, 286 items on 148 SMs, none with more than
// two).
int plan_lm_head(const B2LmHeadArgmaxArgs* a, LmPlan* pl) {
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    if (dev < 0 || di.sms <= 0) return fail(B2_ERR_DEVICE, "no current CUDA device");
    pl->chunks = (a->batch + kLmBRows - 1) / kLmBRows;
    pl->kb_total = (a->d_model + kLmKBlock - 1) / kLmKBlock;
    for (long long k = 1;; ++k) {
        const long long tiles = std::max(1LL, (k * di.sms + pl->chunks - 1) / pl->chunks);
        const long long rows = (a->vocab + tiles - 1) / tiles;
        pl->vn = static_cast<int>(std::max(16LL, (rows + 15) / 16 * 16));
        if (pl->vn <= kLmMaxVRows) break;
    }
    pl->n_tiles = (a->vocab + pl->vn - 1) / pl->vn;
    const long long items = static_cast<long long>(pl->n_tiles) * pl->chunks;
    if (items > (1LL << 30)) return fail(B2_ERR_SHAPE, "vocab x batch too large");
    pl->grid = static_cast<int>(std::min<long long>(items, di.sms));
    // three ring slots: measured best at every batch (GPT-2 XL lm_head at
    // batch 128: 2 slots 43.7 us, 3: 37.2, 4: 37.8, 6: 38.2)
    int stages = 3;
    while (stages > 2 && LmLayout::bytes(pl->vn, stages) > di.max_smem_optin) --stages;
    if (LmLayout::bytes(pl->vn, stages) > di.max_smem_optin)
        return fail(B2_ERR_UNSUPPORTED, "lm_head + argmax: tile does not fit in shared memory");
    pl->stages = stages;
    pl->smem = LmLayout::bytes(pl->vn, stages);
    return B2_OK;
}

template <typename T>
int lm_head_t(const B2LmHeadArgmaxArgs* a, cudaStream_t stream) {
    auto kern = lm_head_argmax_kernel<T>;
    static std::atomic<uint64_t> smem_set{0};
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    int rc = ensure_max_smem(kern, smem_set, dev, di.max_smem_optin);
    if (rc != B2_OK) return rc;
    LmPlan pl;
    rc = plan_lm_head(a, &pl);
    if (rc != B2_OK) return rc;
    CUtensorMap wm, xm;
    rc = encode_rows_map(&wm, a->dtype, a->w, a->d_model, a->vocab, a->d_model, pl.vn);
    if (rc != B2_OK) return rc;
    // x boxes of the batch's rows (rounded to 16) while one batch chunk holds them all
    const int xrows = pl.chunks > 1 ? kLmBRows : std::max(16, (a->batch + 15) / 16 * 16);
    rc = encode_rows_map(&xm, a->dtype, a->x, a->d_model, a->batch, a->x_row_stride, xrows);
    if (rc != B2_OK) return rc;
    LmParams lp;
    lp.batch = a->batch;
    lp.vocab = a->vocab;
    lp.vn = pl.vn;
    lp.xrows = xrows;
    lp.kb_total = pl.kb_total;
    lp.stages = pl.stages;
    lp.n_tiles = pl.n_tiles;
    lp.chunks = pl.chunks;

    char* ws = static_cast<char*>(a->workspace);
    lp.counter = reinterpret_cast<unsigned int*>(ws);
    lp.keys = reinterpret_cast<unsigned long long*>(ws + 16);
    lp.tokens = a->out_tokens;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
    cfg.blockDim = dim3(kLmThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, lp, wm, xm);
    if (e != cudaSuccess) {
        cudaGetLastError();
        g_last_error = cudaGetErrorString(e);
        return static_cast<int>(e);
    }
    return launch_status();
}

}  // namespace
}  // namespace b2

extern "C" size_t b2_lm_head_argmax_workspace_bytes(int32_t batch) { return b2::lm_workspace_bytes(batch); }

extern "C" int b2_lm_head_argmax(const B2LmHeadArgmaxArgs* a, b2_stream_t stream) {
    using namespace b2;
    if (a == nullptr) return fail(B2_ERR_NULL, "args is NULL");
    if (a->dtype != B2_F16 && a->dtype != B2_BF16)
        return fail(B2_ERR_DTYPE, "b2_lm_head_argmax runs F16 and BF16 on the tensor cores");
    if (a->batch < 0 || a->d_model <= 0 || a->vocab <= 0) return fail(B2_ERR_SHAPE, "bad sizes");
    if (a->batch == 0) return B2_OK;
    if (!a->x || !a->w || !a->out_tokens || !a->workspace)
        return fail(B2_ERR_NULL, "x, w, out_tokens and workspace are required");
    if (a->x_row_stride < a->d_model) return fail(B2_ERR_SHAPE, "x_row_stride must cover d_model");
    if (a->d_model % 8 != 0 || a->x_row_stride % 8 != 0 || !aligned16(a->x) || !aligned16(a->w))
        return fail(B2_ERR_ALIGN, "x and w must be 16-byte aligned with d_model and x_row_stride multiples of 8");
    if (!aligned16(a->workspace) || a->workspace_bytes < lm_workspace_bytes(a->batch))
        return fail(B2_ERR_WORKSPACE, "workspace missing, misaligned or smaller than b2_lm_head_argmax_workspace_bytes");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return a->dtype == B2_F16 ? lm_head_t<__half>(a, s) : lm_head_t<__nv_bfloat16>(a, s);
}

// ------------------------------------------------------------ prefill attention
namespace b2 {
namespace {

// The pool as a 4-D tensor for the prefill kernel's boxes: dim 0 head_dim (64,
// one 128-byte swizzle row), dim 1 the 16 token rows of a slab (stride
// n_kv_head * head_dim), dim 2 kv head, dim 3 slab ((block * n_layer + layer)
// * 2 + K|V); box {64, 16, 1, 1} = one head's 16 rows of one slab.
int encode_prefill_kv_map(const B2PrefillAttnArgs* a, CUtensorMap* map) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc == nullptr) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t es = 2;
    const cuuint64_t hd = static_cast<cuuint64_t>(a->head_dim), hk = static_cast<cuuint64_t>(a->n_kv_head);
    const cuuint64_t dims[4] = {hd, 16, hk, static_cast<cuuint64_t>(a->num_blocks) * a->n_layer * 2};
    const cuuint64_t strides[3] = {hk * hd * es, hd * es, 16 * hk * hd * es};
    const cuuint32_t box[4] = {64, 16, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, a->dtype == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           4, const_cast<void*>(a->kv_pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2_ERR_DEVICE, "cuTensorMapEncodeTiled rejected the KV pool layout");
    return B2_OK;
}

template <typename T>
int launch_prefill_t(const B2PrefillAttnArgs* a, const PfParams& pp, const CUtensorMap& map, cudaStream_t stream) {
    auto kern = prefill_attn_tc_kernel<T>;
    static std::atomic<uint64_t> smem_set{0};
    int dev = -1;
    const DeviceInfo di = device_info(&dev);
    const int rc = ensure_max_smem(kern, smem_set, dev, di.max_smem_optin);
    if (rc != B2_OK) return rc;
    if (PfLayout::bytes > di.max_smem_optin) return fail(B2_ERR_UNSUPPORTED, "prefill attention: shared memory");
    const dim3 grid(static_cast<unsigned>(a->n_seqs), static_cast<unsigned>(a->n_head),
                    static_cast<unsigned>((a->max_q_len + kPfRows - 1) / kPfRows));
    return launch_pdl(kern, grid, dim3(kPfThreads), PfLayout::bytes, stream, pp, map);
}

}  // namespace
}  // namespace b2

extern "C" int b2_prefill_attention(const B2PrefillAttnArgs* a, b2_stream_t stream) {
    using namespace b2;
    if (a == nullptr) return fail(B2_ERR_NULL, "args is NULL");
    if (a->dtype != B2_F16 && a->dtype != B2_BF16) return fail(B2_ERR_DTYPE, "prefill attention runs F16 and BF16");
    if (a->n_seqs < 0 || a->max_q_len < 0) return fail(B2_ERR_SHAPE, "n_seqs and max_q_len must be >= 0");
    if (a->n_seqs == 0 || a->max_q_len == 0) return B2_OK;
    if (!a->q || !a->kv_pool || !a->block_tables || !a->seq_lens_pre || !a->q_start || !a->q_len || !a->out)
        return fail(B2_ERR_NULL, "q, kv_pool, block_tables, seq_lens_pre, q_start, q_len and out are required");
    if (a->head_dim != kPfHeadDim) return fail(B2_ERR_UNSUPPORTED, "prefill attention: head_dim must be 64");
    if (a->n_kv_head <= 0 || a->n_head <= 0 || a->n_head % a->n_kv_head != 0)
        return fail(B2_ERR_SHAPE, "n_head must be a positive multiple of n_kv_head");
    if (a->n_head > 65535 || (a->max_q_len + kPfRows - 1) / kPfRows > 65535)
        return fail(B2_ERR_SHAPE, "n_head and max_q_len / 128 must be <= 65535");
    if (a->max_blocks_per_seq <= 0 || a->n_layer <= 0 || a->layer_idx < 0 || a->layer_idx >= a->n_layer ||
        a->num_blocks <= 0 || static_cast<long long>(a->num_blocks) * a->n_layer * 2 >= (1LL << 31) - 1)
        return fail(B2_ERR_SHAPE, "max_blocks_per_seq, n_layer, layer_idx or num_blocks out of range");
    if (a->q_row_stride < a->n_head * a->head_dim || a->out_row_stride < a->n_head * a->head_dim)
        return fail(B2_ERR_SHAPE, "row strides must cover n_head * head_dim");
    if (!aligned16(a->q) || !aligned16(a->kv_pool) || !aligned16(a->out) || (a->q_bias && !aligned16(a->q_bias)) ||
        a->q_row_stride % 8 != 0 || a->out_row_stride % 8 != 0)
        return fail(B2_ERR_ALIGN, "q, q_bias, kv_pool and out must be 16-byte aligned, row strides multiples of 8");
    CUtensorMap map;
    int rc = encode_prefill_kv_map(a, &map);
    if (rc != B2_OK) return rc;
    PfParams pp;
    pp.q = a->q;
    pp.q_row_stride = a->q_row_stride;
    pp.q_bias = a->q_bias;
    pp.block_tables = a->block_tables;
    pp.seq_lens_pre = a->seq_lens_pre;
    pp.q_start = a->q_start;
    pp.q_len = a->q_len;
    pp.out = a->out;
    pp.out_row_stride = a->out_row_stride;
    pp.qg = a->n_head / a->n_kv_head;
    pp.mbps = a->max_blocks_per_seq;
    pp.layer_idx = a->layer_idx;
    pp.n_layer = a->n_layer;
    pp.num_blocks = a->num_blocks;
    pp.oob_slab = a->num_blocks * a->n_layer * 2;
    const float scale = a->scale != 0.0f ? a->scale : 1.0f / std::sqrt(static_cast<float>(a->head_dim));
    pp.scale_log2 = scale * 1.4426950408889634f;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return a->dtype == B2_F16 ? launch_prefill_t<__half>(a, pp, map, s) : launch_prefill_t<__nv_bfloat16>(a, pp, map, s);
}
