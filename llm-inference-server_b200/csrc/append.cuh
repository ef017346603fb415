// append.cuh -- paged KV append (reshape-and-cache) for sm_100a.
//
// Same placement rule as gpu-engine/src/kernels/attention.cu:21-47: this
// step's K and V rows of sequence b go to token slot p % 16 of block
// block_tables[b][p / 16], p = seq_lens[b] (pre-append).  One thread moves
// one 16-byte chunk (the reference moves one 2-byte element per thread), and
// the optional bias add and the seq_lens + 1 update of
// gpu-engine/src/kernels/embedding.cu:26-29 ride along in the same launch.
#pragma once

#include "b2_common.cuh"

namespace b2 {

struct AppendParams {
    void* pool;
    const void* k;
    const void* v;
    long long kv_row_stride;
    const void* k_bias;
    const void* v_bias;
    const int* block_tables;
    const int* seq_lens;
    int* seq_lens_post;
    int batch, n_kv_head, mbps, layer_idx, n_layer, num_blocks;
};

template <typename T, int DH>
__global__ void __launch_bounds__(256) kv_append_kernel(const AppendParams p) {
    constexpr int E = Elem<T>::kPer16B;
    constexpr int GL = DH / E;
    // The attention launched next may start now: with B2_ATTN_NEWEST_ROW_PENDING
    // it streams every key row but the one written here, and waits for this
    // kernel before reading that row (and with flags 0 before reading anything).
    pdl_launch_dependents();
    pdl_wait();  // k and v come from the kernel before this one
    const int chunks_per_row = p.n_kv_head * GL;  // per K (or V) row
    const long long total = static_cast<long long>(p.batch) * 2 * chunks_per_row;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int b = static_cast<int>(idx / (2 * chunks_per_row));
    const int rem = static_cast<int>(idx - static_cast<long long>(b) * 2 * chunks_per_row);
    const int kv = rem / chunks_per_row;  // 0 = K, 1 = V
    const int c = rem - kv * chunks_per_row;
    const int h = c / GL;
    const int dg = c - h * GL;

    const int pos = __ldg(p.seq_lens + b);
    if (rem == 0 && p.seq_lens_post != nullptr) p.seq_lens_post[b] = pos + 1;
    if (pos < 0 || pos >= p.mbps * kBlockTokens) {
        if (rem == 0) flag_error(B2_DEVERR_SEQ_LEN);
        return;
    }
    const int blk = __ldg(p.block_tables + static_cast<size_t>(b) * p.mbps + pos / kBlockTokens);
    if (blk < 0 || blk >= p.num_blocks) {
        if (rem == 0) flag_error(B2_DEVERR_BLOCK_ID);
        return;
    }
    const size_t row = static_cast<size_t>(p.n_kv_head) * DH;
    const size_t slab = row * kBlockTokens;
    const size_t dst_off = static_cast<size_t>(blk) * p.n_layer * 2 * slab +
                           static_cast<size_t>(p.layer_idx) * 2 * slab + static_cast<size_t>(kv) * slab +
                           static_cast<size_t>(pos % kBlockTokens) * row + static_cast<size_t>(h) * DH + dg * E;
    const T* src = static_cast<const T*>(kv ? p.v : p.k) + static_cast<size_t>(b) * p.kv_row_stride +
                   static_cast<size_t>(h) * DH + dg * E;
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
    const void* bias = kv ? p.v_bias : p.k_bias;
    if (bias != nullptr) {
        float f[E], bf[E];
        unpack16<T>(raw, f);
        unpack16<T>(__ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(bias) + h * DH + dg * E)), bf);
#pragma unroll
        for (int e = 0; e < E; ++e) f[e] += bf[e];
        raw = pack16<T>(f);
    }
    *reinterpret_cast<uint4*>(static_cast<T*>(p.pool) + dst_off) = raw;
}

}  // namespace b2
