/*
 * b2_decode.h -- C-ABI of the sm_100a decode hot path (libb2decode.so).
 *
 * Drop-in for the kernel-launch layer of kanish10/LLM-Inference-Server
 * (gpu-engine/include/engine/kernels.h:29-93): every entry point below names
 * the reference function it replaces.  Plain C: no CUDA or torch types in the
 * signatures, so cgo / ctypes / JNI can bind it directly.
 *
 * Conventions kept from the reference:
 *   - paged KV layout, one block = all layers of 16 token positions:
 *       [block][layer][2 (K,V)][16][n_kv_head][head_dim]   (kv_cache.h:6-8)
 *     (n_kv_head == n_head for multi-head attention; the reference calls it
 *     n_heads.)
 *   - seq_lens: b2_kv_append takes the PRE-append count (the slot written);
 *     b2_paged_attention takes the POST-append key count (kernels.h:22-27).
 *   - q / k / v may live inside a fused QKV row: *_row_stride is the element
 *     distance between batch rows (kernels.h:51-56, 67-70).
 *   - attention output is packed [batch, n_head, head_dim] (kernels.h:73).
 *
 * Additions over the reference (all optional to use):
 *   - dtype per call (f32 / f16 / bf16) instead of half only;
 *   - n_kv_head for grouped-query attention;
 *   - num_blocks (pool capacity) so kernels can refuse out-of-range block
 *     ids instead of reading or writing outside the pool;
 *   - status codes: 0 = OK, < 0 = argument error found on the host before
 *     any launch, > 0 = the cudaError_t seen right after the launch.
 *     The reference launchers return void and never check.
 *
 * All buffers are caller-owned device memory.  No entry point allocates or
 * frees, and none synchronises except b2_device_errors and
 * b2_paged_attention_host (a synchronous call by design), so every other
 * launch can be captured in a CUDA graph.
 * All pointers handed to the attention and append kernels must be 16-byte
 * aligned, and every row stride times the element size a multiple of 16 bytes.
 */
#ifndef B2_DECODE_H
#define B2_DECODE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2_API __attribute__((visibility("default")))
#else
#define B2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t passed as an opaque pointer; NULL is the legacy default stream. */
typedef void* b2_stream_t;

typedef enum b2_dtype { B2_F32 = 0, B2_F16 = 1, B2_BF16 = 2 } b2_dtype;

#define B2_BLOCK_TOKENS 16 /* gpu-engine/include/engine/kv_cache.h:8 */

#define B2_OK 0
#define B2_ERR_NULL (-1)        /* a required pointer is NULL */
#define B2_ERR_DTYPE (-2)       /* unknown or unsupported dtype combination */
#define B2_ERR_SHAPE (-3)       /* a size is out of range or inconsistent */
#define B2_ERR_ALIGN (-4)       /* a pointer or stride breaks the 16-byte rule */
#define B2_ERR_WORKSPACE (-5)   /* workspace missing or too small */
#define B2_ERR_UNSUPPORTED (-6) /* a shape this build has no kernel for */
#define B2_ERR_DEVICE (-7)      /* the device query failed */

/* Device-side error bits, accumulated in a per-device word (b2_device_errors). */
#define B2_DEVERR_BLOCK_ID 1u   /* a block-table entry outside [0, num_blocks) was clamped */
#define B2_DEVERR_SEQ_LEN 2u    /* a seq_len beyond max_blocks_per_seq*16 (or < 0) was clamped */
#define B2_DEVERR_TIMEOUT 4u    /* a bounded pipeline wait gave up; the output is invalid */
#define B2_DEVERR_TOKEN 8u      /* a token id or position outside its table was clamped */

/* Library version string. */
B2_API const char* b2_version(void);

/* Text of the last host-side error on the calling thread ("" if none). */
B2_API const char* b2_last_error_string(void);

/* Reads the device error word of the current device and clears it.  This
 * call synchronises the device; use it in tests and health checks, not per step. */
B2_API int b2_device_errors(uint32_t* bits_out);

/* ------------------------------------------------------------------------
 * Paged KV append (reshape-and-cache).
 * Replaces kernels::launch_kv_append (gpu-engine/include/engine/kernels.h:51-60,
 * gpu-engine/src/kernels/attention.cu:131-139).
 * pool[block_tables[b][p/16]][layer][K|V][p%16][h][:] = k|v[b][h][:], p = seq_lens[b]
 * (pre-append).  A bit copy.  When k_bias / v_bias are non-NULL the bias
 * ([n_kv_head*head_dim], same dtype) is added first (the reference adds the
 * QKV bias in a separate add_bias launch, gpu-engine/src/engine.cu:158).
 * When seq_lens_post is non-NULL it receives seq_lens[b] + 1 (the reference's
 * launch_add_one, kernels.h:62-65), so one launch does both.
 * ---------------------------------------------------------------------- */
typedef struct B2KvAppendArgs {
    int32_t dtype; /* b2_dtype of k, v, biases and pool */
    void* kv_pool;
    const void* k;
    const void* v;
    int32_t kv_row_stride; /* elements between batch rows of k and v */
    const void* k_bias;    /* optional */
    const void* v_bias;    /* optional */
    const int32_t* block_tables; /* [batch, max_blocks_per_seq] */
    const int32_t* seq_lens;     /* [batch], pre-append */
    int32_t* seq_lens_post;      /* optional [batch] output: seq_lens + 1 */
    int32_t batch;
    int32_t n_kv_head;
    int32_t head_dim;
    int32_t max_blocks_per_seq;
    int32_t layer_idx;
    int32_t n_layer;
    int32_t num_blocks; /* pool capacity in blocks (bounds check) */
} B2KvAppendArgs;

B2_API int b2_kv_append(const B2KvAppendArgs* args, b2_stream_t stream);

/* ------------------------------------------------------------------------
 * Paged decode attention.
 * Replaces kernels::launch_paged_attention and PagedAttentionArgs
 * (gpu-engine/include/engine/kernels.h:67-87, attention.cu:141-149).
 * out[b,h,:] = sum_j softmax_j(scale * q[b,h,:].k_j) v_j over the seq_lens[b]
 * keys of sequence b (post-append count), keys of kv head h / (n_head/n_kv_head).
 * A sequence with seq_lens[b] == 0 gets a zero output, like the reference.
 *
 * The work is split over the whole GPU by key rows (every CTA streams the
 * same number of K/V rows, whatever the per-sequence lengths), so one
 * sequence may be cut into pieces handled by several CTAs.  Each piece's
 * partial softmax state goes to a caller-provided workspace; the CTA that
 * finishes a sequence's last piece merges them and writes `out` (the
 * tensor-core kernel for 8 kv heads of head_dim 128 instead launches a second,
 * small merge kernel).  Size the workspace with
 * b2_paged_attention_workspace_bytes and ZERO IT ONCE before its first use
 * (cudaMemset): it holds per-sequence piece counters, and every launch that
 * completes leaves them at zero again.  After a launch that reported
 * B2_DEVERR_TIMEOUT, zero it again.  One workspace serves any number of
 * launches on one stream; launches that may run concurrently need their own.
 * The kernels use programmatic dependent launch, so each may start while the
 * kernel before it finishes.
 * ---------------------------------------------------------------------- */
typedef struct B2PagedAttnArgs {
    int32_t dtype;     /* b2_dtype of q and the pool */
    int32_t out_dtype; /* B2_F32, or the same as dtype */
    const void* q;
    int32_t q_row_stride; /* elements between batch rows of q */
    const void* q_bias;   /* optional [n_head*head_dim], added to q first */
    const void* kv_pool;
    const int32_t* block_tables; /* [batch, max_blocks_per_seq] */
    const int32_t* seq_lens;     /* [batch], post-append key counts */
    void* out;                   /* [batch, n_head, head_dim] packed */
    int32_t batch;
    int32_t n_head;
    int32_t n_kv_head;
    int32_t head_dim; /* 64 or 128 */
    int32_t max_blocks_per_seq;
    int32_t layer_idx;
    int32_t n_layer;
    int32_t num_blocks; /* pool capacity in blocks (bounds check) */
    float scale;        /* 0 selects 1/sqrt(head_dim) */
    int32_t flags;      /* 0, B2_ATTN_INPUTS_READY or B2_ATTN_NEWEST_ROW_PENDING */
    int32_t max_ctas;   /* 0: the whole GPU (one or two CTAs per SM; at two per SM with
                           B2_ATTN_INPUTS_READY, SMs / 16 slots stay free for the next
                           launch's first CTAs); n > 0: at most n CTAs, leaving SMs to
                           kernels running concurrently on other streams */
} B2PagedAttnArgs;

/* flags: what the kernel may read before the kernel launched just before it
 * on the stream has finished (programmatic dependent launch lets it start
 * early).  0: nothing -- every input waits for that kernel.
 * B2_ATTN_INPUTS_READY: nothing this call reads is written by that kernel, so
 *   the set-up and the K/V streaming overlap its tail.
 * B2_ATTN_NEWEST_ROW_PENDING: only the last key row of every sequence (its
 *   newest position, from a kv_append launched just before) may be; seq_lens,
 *   block_tables, q, q_bias and all earlier rows were complete before that
 *   kernel started.  The block holding each sequence's last row is read after
 *   the wait.
 * Outputs and the workspace are always written after the wait.  The
 * tensor-core kernel ignores flags. */
#define B2_ATTN_INPUTS_READY 1
#define B2_ATTN_NEWEST_ROW_PENDING 2

/* Workspace bytes for launches with this batch and head shape on the
 * current device (depends on the SM count). */
B2_API size_t b2_paged_attention_workspace_bytes(const B2PagedAttnArgs* args);

/* One launch on `stream` (the CUDA-core kernel merges each sequence's pieces
 * itself); the tensor-core kernel for 8 kv heads of head_dim 128 adds a small
 * merge kernel. */
B2_API int b2_paged_attention(const B2PagedAttnArgs* args, void* workspace, size_t workspace_bytes,
                              b2_stream_t stream);

/* ------------------------------------------------------------------------
 * One synchronous decode-attention call from host buffers.
 * Replaces the host side of one decode step around the attention launch in
 * Engine::decode_step (gpu-engine/src/engine.cu:343-368): upload the step's
 * inputs with cudaMemcpyAsync, launch, download the output, synchronise.
 *
 * Uploads io->q, io->block_tables and io->seq_lens (each optional: NULL
 * skips that upload) into args->q, args->block_tables and args->seq_lens, runs
 * b2_paged_attention on `stream`, copies args->out into io->out (optional),
 * and waits for the stream.  When every given host input is page-locked
 * memory mapped into the device's address space (cudaHostAlloc /
 * cudaHostRegister memory on a unified-addressing system), one small kernel
 * reads them over the bus and stores them into the device arrays -- no
 * copy-engine set-up on the call's path -- and the attention launch waits for
 * it whatever args->flags says.  Otherwise the uploads are copies, and those
 * whose host AND device ranges are both back to back (q, then block tables,
 * then seq_lens at the same offsets in one host and one device allocation) go
 * as one copy; pageable memory works but copies synchronously.
 * When io->out is page-locked memory mapped into the device's address space
 * (cudaHostAlloc / cudaHostRegister memory on a unified-addressing system)
 * and 16-byte aligned, the kernel stores the output into it directly (the
 * PCIe writes overlap the kernel) and args->out is not written.  The call
 * waits for the stream by polling it (cudaStreamQuery), spending the calling
 * thread's core until the GPU is done -- it returns within about a microsecond
 * instead of after a blocking-sync wake-up.
 * Byte counts: q ((batch-1)*q_row_stride + n_head*head_dim) elements of
 * dtype; block tables batch*max_blocks_per_seq int32; seq_lens batch int32;
 * out batch*n_head*head_dim elements of out_dtype.
 * ---------------------------------------------------------------------- */
typedef struct B2AttnHostIO {
    const void* q;
    const int32_t* block_tables;
    const int32_t* seq_lens;
    void* out;
} B2AttnHostIO;

B2_API int b2_paged_attention_host(const B2PagedAttnArgs* args, const B2AttnHostIO* io, void* workspace,
                                   size_t workspace_bytes, b2_stream_t stream);

/* ------------------------------------------------------------------------
 * Paged decode attention whose output is all-gathered in its epilogue.
 * No counterpart in the reference (its engine is single-GPU).  For
 * head-sharded decode: a rank computes attention for its own heads and stores
 * each output row straight into n_outs arrays -- its own and its peers'
 * gathered attention outputs, peers reached through their UVA (IPC-mapped)
 * addresses over NVLink -- at row b * row_stride + col_offset.  Nothing else
 * changes; use b2_tp_barrier afterwards so every rank's slice has landed
 * before the gathered array is read.
 * ---------------------------------------------------------------------- */
#define B2_MAX_GATHER 8

typedef struct B2OutputGather {
    void* const* outs;  /* device array of n_outs base pointers (local or peer) */
    int32_t n_outs;     /* 1 .. B2_MAX_GATHER */
    int64_t row_stride; /* elements between batch rows of every output array */
    int64_t col_offset; /* element column where this call's head 0 goes */
} B2OutputGather;

B2_API int b2_paged_attention_gather(const B2PagedAttnArgs* args, void* workspace, size_t workspace_bytes,
                                     const B2OutputGather* gather, b2_stream_t stream);

/* Cross-GPU barrier for head-sharded ranks, one launch of one small CTA.
 * Every rank r of n publishes `*epoch` into slot[r] of each peer's flag array
 * (peer_flags[p] + slot * n, written with release semantics at system scope
 * after a system-scope fence, so the rank's earlier stores to peers are
 * visible first) and then waits until its own local_flags[slot * n + p]
 * reach *epoch for every p.  The wait is bounded (2 s); a timeout sets
 * B2_DEVERR_TIMEOUT and returns.  While the device's error word holds
 * B2_DEVERR_TIMEOUT (a barrier earlier in the step gave up), later barriers
 * publish their flags but do not wait, so a step whose peer stopped fails in
 * one limit, not one per layer.  flag arrays start zeroed; epochs only grow. */
B2_API int b2_tp_barrier(uint32_t* local_flags, uint32_t* const* peer_flags, int32_t rank, int32_t n,
                         const uint32_t* epoch, int32_t slot, b2_stream_t stream);

/* b2_tp_barrier with the wait bounded by limit_ns (0 < limit_ns <= 60 s)
 * instead of 2 s.  No reference counterpart. */
B2_API int b2_tp_barrier_timed(uint32_t* local_flags, uint32_t* const* peer_flags, int32_t rank, int32_t n,
                               const uint32_t* epoch, int32_t slot, uint64_t limit_ns, b2_stream_t stream);

/* *epoch += 1 (one thread): the start of a new step for b2_tp_barrier. */
B2_API int b2_tp_epoch_bump(uint32_t* epoch, b2_stream_t stream);

/* Device address of the current device's error word (the one
 * b2_device_errors reads), for callers that read it without a device-wide
 * synchronisation: a stream-ordered copy of it next to a step's results.
 * No reference counterpart (its kernels report nothing). */
B2_API int b2_device_error_word(uint32_t** out);

/* Sets `bits` in the current device's error word from a one-thread kernel on
 * `stream`, for tests of error propagation: no kernel has to fail for a
 * caller's error path to run.  No reference counterpart. */
B2_API int b2_raise_device_error(uint32_t bits, b2_stream_t stream);

/* ------------------------------------------------------------------------
 * Paged decode attention without any device allocation.
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they run attention -- for example a plugin whose host
 * runtime owns all device memory through its own pool and forbids allocation
 * outside it, or a hard real-time decode loop that cannot take cudaMalloc's
 * implicit device synchronisation and unbounded latency.
 *
 * Same arguments and results as b2_paged_attention, but the workspace is a
 * fixed array of B2_NOALLOC_SCRATCH_BYTES compiled into the library: every GPU
 * that loads the library holds it until the process exits.  Shapes whose
 * workspace (b2_paged_attention_workspace_bytes) exceeds it are rejected with
 * B2_ERR_WORKSPACE before anything is launched.
 *
 * The first call on a device looks up the array's device address for that
 * device (cudaGetSymbolAddress; a failed lookup is retried by the next call);
 * make that first call before any stream capture.  The address is kept for
 * the life of the process, so this entry point does not support
 * cudaDeviceReset.  All calls share the one array, which keeps what the last
 * call left in it: each call first clears the array's piece-counter region
 * with cudaMemsetAsync on `stream` (a call that gave up on a bounded wait,
 * B2_DEVERR_TIMEOUT, may leave counts behind), then launches.  Calls whose
 * work overlaps on the GPU (different streams, no ordering between them) race
 * on the array: order them on one stream, or use b2_paged_attention with a
 * workspace per stream.
 * ---------------------------------------------------------------------- */
#define B2_NOALLOC_SCRATCH_BYTES (4u << 20) /* 4 MiB */

B2_API int b2_paged_attention_noalloc(const B2PagedAttnArgs* args, b2_stream_t stream);

/* ------------------------------------------------------------------------
 * Row kernels around attention.  All take dtype (f32 / f16 / bf16),
 * compute in fp32, and accept out == x (in place).
 * ---------------------------------------------------------------------- */

/* Fused residual add + LayerNorm.  Replaces kernels::launch_add_layernorm
 * (kernels.h:39-44, layernorm.cu:56-63):
 *   r = residual_in + (x + bias)  (x, bias optional);  residual_out = r;
 *   out = (r - mean(r)) / sqrt(var(r) + eps) * gamma + beta.
 * Statistics are taken over the unrounded fp32 r.  x may be NULL (adds zero),
 * replacing the reference's persistent zero buffer (engine.cu:97). */
B2_API int b2_add_layernorm(int32_t dtype, void* out, void* residual_out, const void* x,
                     const void* bias, const void* residual_in, const void* gamma,
                     const void* beta, int32_t batch, int32_t d_model, float eps,
                     b2_stream_t stream);

/* out = gelu_tanh(x + bias).  Replaces kernels::launch_bias_gelu (kernels.h:46-49). */
B2_API int b2_bias_gelu(int32_t dtype, void* out, const void* x, const void* bias, int32_t batch,
                 int32_t d_ff, b2_stream_t stream);

/* out = x + bias.  Replaces kernels::launch_add_bias (kernels.h:35-37). */
B2_API int b2_add_bias(int32_t dtype, void* out, const void* x, const void* bias, int32_t batch,
                int32_t dim, b2_stream_t stream);

/* out[b] = in[b] + 1.  Replaces kernels::launch_add_one (kernels.h:62-65). */
B2_API int b2_add_one(int32_t* out, const int32_t* in, int32_t batch, b2_stream_t stream);

/* out = wte[token_ids[b]] + wpe[positions[b]].  Replaces kernels::launch_embedding
 * (kernels.h:31-33).  vocab / n_pos bound the lookups (clamped and flagged). */
B2_API int b2_embedding(int32_t dtype, void* out, const void* wte, const void* wpe,
                 const int32_t* token_ids, const int32_t* positions, int32_t batch,
                 int32_t d_model, int32_t vocab, int32_t n_pos, b2_stream_t stream);

/* Greedy argmax per row, ties to the lowest index (cpu_model.cpp:186-195).
 * Replaces kernels::launch_argmax (kernels.h:89-92). */
B2_API int b2_argmax(int32_t dtype, int32_t* out_tokens, const void* logits, int32_t batch,
              int32_t vocab, b2_stream_t stream);

/* b2_argmax over rows row_stride elements apart (row_stride >= vocab).  No
 * reference counterpart: a caller that pads each logits row to a multiple of
 * 16 bytes (so GEMMs writing them stay vector-aligned) gets 16-byte vector
 * reads here. */
B2_API int b2_argmax_rows(int32_t dtype, int32_t* out_tokens, const void* logits, int64_t row_stride,
                          int32_t batch, int32_t vocab, b2_stream_t stream);

/* ------------------------------------------------------------------ prefill attention
 * Causal attention of a prefill call's new rows over the paged KV cache, on
 * the tensor cores (tcgen05), head_dim 64.  No reference counterpart: the
 * reference prefills by walking each prompt token through Engine::decode_step
 * at batch 1 (cpp-engine/src/gpu_engine_generator.cpp:28-42), i.e. through
 * kernels::launch_paged_attention (kernels.h:67-87) once per prompt row.  For
 * sequence b of the call, rows q_start[b] .. q_start[b] + q_len[b] - 1 of q and
 * out are its new tokens at positions seq_lens_pre[b] + i; row i attends the
 * keys at positions [0, seq_lens_pre[b] + i], which must already be in the pool
 * (b2_kv_append of the same rows first).  Per row this is exactly what
 * b2_paged_attention computes with seq_lens = position + 1; here each 128-row
 * query tile reads its keys once.  q_bias (optional) is added to q first and
 * rounded to the dtype, like b2_paged_attention.  F16 / BF16 only; 16-byte
 * aligned pointers, row strides multiples of 8 elements.  Each launch is
 * self-contained (no workspace).  Programmatic dependent launch as above. */
typedef struct B2PrefillAttnArgs {
    int32_t dtype;               /* B2_F16 or B2_BF16: q, pool and out */
    const void* q;               /* [rows][q_row_stride]; head h at columns h * head_dim */
    int32_t q_row_stride;
    const void* q_bias;          /* optional [n_head * head_dim] */
    const void* kv_pool;
    const int32_t* block_tables; /* [n_seqs, max_blocks_per_seq] */
    const int32_t* seq_lens_pre; /* [n_seqs] keys cached before this call's rows */
    const int32_t* q_start;      /* [n_seqs] first row of each sequence in q and out */
    const int32_t* q_len;        /* [n_seqs] new rows of each sequence */
    void* out;                   /* [rows][out_row_stride], packed [n_head][head_dim] per row */
    int32_t out_row_stride;
    int32_t n_seqs;
    int32_t n_head;
    int32_t n_kv_head;
    int32_t head_dim;            /* 64 */
    int32_t max_blocks_per_seq;
    int32_t layer_idx;
    int32_t n_layer;
    int32_t num_blocks;
    int32_t max_q_len;           /* >= every q_len[b]: sizes the grid */
    float scale;                 /* 0 selects 1/sqrt(head_dim) */
} B2PrefillAttnArgs;

B2_API int b2_prefill_attention(const B2PrefillAttnArgs* args, b2_stream_t stream);

/* ------------------------------------------------------------------ linear layers
 * y[b][n] = epilogue(sum_k x[b][k] * w[n][k]) on the tensor cores (tcgen05),
 * for the decode step's small batches.  Replaces the engine's cuBLAS call
 * gemm_rowmajor (gpu-engine/src/engine.cu:124-131: row-major Y = X * W^T, W
 * stored [out][in]) together with the launch that follows it:
 *   B2_LINEAR_STORE  y = T(x.W^T); with a bias, T(float(T(x.W^T)) + bias) --
 *                    gemm_rowmajor + kernels::launch_add_bias (kernels.h:35-37)
 *   B2_LINEAR_GELU   y = T(gelu_tanh(float(T(x.W^T)) + bias)) --
 *                    gemm_rowmajor + kernels::launch_bias_gelu (kernels.h:46-49)
 * fp32 accumulation; the sum's order differs from cuBLAS's, so results agree
 * with it to rounding, not bit for bit.  F16 and BF16 only (B2_ERR_DTYPE for
 * F32, whose callers keep cuBLAS).  x, w, y: 16-byte aligned; in_features,
 * x_row_stride and y_row_stride multiples of 8.  The
 * launch uses programmatic dependent launch: it starts streaming w while the
 * previous kernel on the stream finishes (w must not be that kernel's
 * output; x may be). */
#define B2_LINEAR_STORE 0
#define B2_LINEAR_GELU 1

typedef struct B2LinearArgs {
    int32_t dtype;        /* B2_F16 or B2_BF16, for x, w, bias and y */
    const void* x;        /* [batch][x_row_stride] */
    int64_t x_row_stride; /* elements */
    const void* w;        /* [out_features][in_features], row-major */
    const void* bias;     /* [out_features] or NULL (B2_LINEAR_GELU: NULL = no bias) */
    void* y;              /* [batch][y_row_stride] */
    int64_t y_row_stride; /* elements, >= out_features */
    int32_t batch;        /* 1 .. 65535 * 256 */
    int32_t in_features;
    int32_t out_features;
    int32_t epilogue;     /* B2_LINEAR_* */
} B2LinearArgs;

B2_API int b2_linear(const B2LinearArgs* args, b2_stream_t stream);

/* ------------------------------------------------------------------ lm_head + argmax
 * out_tokens[b] = the v < vocab that maximises T(x[b] . w[v]): the tied lm_head
 * GEMM and the greedy argmax in one kernel on the tensor cores (tcgen05), the
 * logits never written to memory.  Replaces gemm_rowmajor(bucket, D, vocab,
 * d_x, wte, d_logits) + kernels::launch_argmax (gpu-engine/src/engine.cu:202-203;
 * kernels.h:89-92, logits.cu:18-57).  Each logit is the fp32 dot product
 * rounded to the dtype, as the unfused path stores it; ties go to the lowest
 * index, like the reference CPU path's first maximum (cpu_model.cpp:182-196);
 * NaN logits never win against a number.  The dot products are summed in a
 * different order from cuBLAS's, so a near-tie can resolve differently from
 * the unfused GEMM + b2_argmax_rows.  F16 and BF16 only (B2_ERR_DTYPE for F32).
 *   x: [batch][x_row_stride], the final hidden states.
 *   w: [>= vocab rows][d_model] row-major (rows past vocab are never read
 *      into a result).
 * x and w 16-byte aligned; d_model and x_row_stride multiples of 8.
 * workspace: b2_lm_head_argmax_workspace_bytes(batch) bytes, 16-byte aligned,
 * zeroed by the caller once; every launch leaves it zeroed (the last CTA to
 * finish clears it, also after a bounded wait gave up).  Programmatic
 * dependent launch: w streams while the
 * previous kernel on the stream finishes (w must not be that kernel's output;
 * x may be).  Launches that share a workspace must not overlap on the GPU. */
typedef struct B2LmHeadArgmaxArgs {
    int32_t dtype;        /* B2_F16 or B2_BF16, for x and w */
    const void* x;        /* [batch][x_row_stride] */
    int64_t x_row_stride; /* elements */
    const void* w;        /* [vocab (or more) rows][d_model] */
    int32_t batch;        /* 0 .. 65535 * 256 */
    int32_t d_model;
    int32_t vocab;
    int32_t* out_tokens;  /* [batch] */
    void* workspace;
    size_t workspace_bytes;
} B2LmHeadArgmaxArgs;

B2_API size_t b2_lm_head_argmax_workspace_bytes(int32_t batch);
B2_API int b2_lm_head_argmax(const B2LmHeadArgmaxArgs* args, b2_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B2_DECODE_H */
