/*
 * b2_engine.h -- C-ABI of the GPT-2 decode engine (libb2engine.so).
 *
 * The decode-step orchestration of kanish10/LLM-Inference-Server's gpu-engine
 * (Engine / Engine::Impl, gpu-engine/include/engine/engine_api.h:9-48 and
 * gpu-engine/src/engine.cu:71-388), rebuilt over the sm_100a kernels of
 * libb2decode.so and cuBLAS.  The same life cycle and the same calls:
 * create (init) -> add_sequence -> decode_step ... -> free_sequence, with
 * free_blocks() for admission control and a CUDA-graph switch.  Differences:
 * a dtype per engine (f32 / f16 / bf16; the reference is f16 only), status
 * codes instead of exceptions, and two bench hooks (synthetic weights made on
 * the device, sequences whose context is treated as already cached).
 *
 * include/b2_engine_api.hpp wraps this in a C++ class with the reference's
 * Engine signatures.  Every call that takes an engine runs on that engine's
 * device and stream; one engine must not be used from two threads at once.
 */
#ifndef B2_ENGINE_H
#define B2_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "b2_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2_engine b2_engine;

/* gpu-engine/include/engine/engine_api.h:9-13 (EngineConfig) plus the dtype,
 * the graph switch (Engine::set_use_cuda_graphs) and the device. */
typedef struct B2EngineConfig {
    int32_t max_batch;       /* largest batch decode_step accepts */
    int32_t max_seq_len;     /* positions per sequence (<= n_ctx) */
    int32_t kv_block_budget; /* KV pool size in 16-token blocks */
    int32_t dtype;           /* b2_dtype of weights, activations and KV */
    int32_t use_cuda_graphs; /* 1: capture and replay one graph per batch bucket */
    int32_t device;          /* CUDA device ordinal; -1 = the current device */
    int32_t tp_rank;         /* head-sharded engines: this rank (0 .. tp_size-1) */
    int32_t tp_size;         /* 0 or 1: one engine holds every head; 2..8: head-sharded */
    int32_t max_prefill_tokens; /* prompt tokens one b2_engine_prefill call may carry; 0 = 2048 */
    int32_t tp_allgather;    /* head-sharded engines: 0 = peer stores fused into the attention
                                epilogue + flag barrier; 1 = ncclAllGather after attention */
} B2EngineConfig;

/* gpu-engine/include/engine/model.h:7-18 (GPT2Config). */
typedef struct B2ModelShape {
    int32_t n_layer;
    int32_t n_head;
    int32_t d_model;
    int32_t vocab_size;
    int32_t n_ctx;
    float layer_norm_epsilon;
    int32_t eos_token_id;
} B2ModelShape;

/* Engine::init (engine.cu:240-294): reads weights_dir/{config.json,
 * manifest.json, weights.bin} in the reference exporter's format
 * (gpu-engine/export/export_gpt2.py), checks total_bytes and checksum_sum
 * like WeightsLoader, converts to cfg->dtype and uploads. */
B2_API int b2_engine_create(const char* weights_dir, const B2EngineConfig* cfg, b2_engine** out);

/* Bench hook: weights drawn on the device, every matrix, embedding and bias
 * ~ N(0, std) from a counter-based generator keyed by seed, LayerNorm gamma 1
 * and beta 0 -- for model sizes where writing weight files is pointless.  The
 * KV pool is filled with N(0, 1) values, so sequences added with
 * b2_engine_add_sequence_cached attend over random keys and values. */
B2_API int b2_engine_create_synthetic(const B2ModelShape* shape, uint64_t seed, float std,
                                      const B2EngineConfig* cfg, b2_engine** out);

B2_API void b2_engine_destroy(b2_engine* eng);

/* Engine::add_sequence (engine.cu:296-307): registers a prompt and takes its
 * first KV block.  Returns a sequence id >= 0, -1 if the pool is exhausted,
 * or another negative status. */
B2_API int32_t b2_engine_add_sequence(b2_engine* eng, const int32_t* prompt, int32_t prompt_len);

/* Bench hook: a sequence whose first ctx_len positions count as already
 * cached (their KV is whatever the pool holds; the pool starts zeroed) and
 * whose next input token is last_token.  Takes the blocks those positions
 * need.  Returns an id, -1 when the pool is exhausted, or a status. */
B2_API int32_t b2_engine_add_sequence_cached(b2_engine* eng, int32_t ctx_len, int32_t last_token);

/* Engine::decode_step (engine.cu:309-377): one token for each listed sequence
 * -- its next prompt token while it is still inside its prompt, otherwise its
 * last generated token -- and one next-token id per entry, in order.  A new
 * block is taken when a sequence crosses a 16-token boundary; running out of
 * blocks returns B2_ERR_POOL (the reference throws) with nothing launched. */
B2_API int b2_engine_decode_step(b2_engine* eng, const int32_t* seq_ids, int32_t batch, int32_t* out_next_tokens);

/* Batched prefill (no reference counterpart: the reference walks every prompt
 * token by token through decode_step at batch 1, gpu-engine/src/engine.cu:8-18
 * and cpp-engine/src/gpu_engine_generator.cpp:28-42).  Runs the whole remaining
 * prompt of each listed sequence in one pass -- every prompt token a row of the
 * same GEMMs, each token's K/V appended at its position, each attending to the
 * positions up to its own -- and writes each sequence's first generated token,
 * as decode_step would after the last prompt token.  Afterwards the sequences
 * continue with decode_step.  Every listed sequence must still be inside its
 * prompt; the call's prompt tokens may not exceed cfg.max_prefill_tokens.
 * Blocks are taken for all prompt positions up front (B2_ERR_POOL if they do
 * not fit, with nothing changed).  Not available on head-sharded engines.
 * The attention of f16 / bf16 models of head_dim 64 runs as 128-row query
 * tiles on the tensor cores (b2_prefill_attention); f32 models and the switch
 * below use one decode-attention row per prompt token. */
B2_API int b2_engine_prefill(b2_engine* eng, const int32_t* seq_ids, int32_t n, int32_t* out_next_tokens);

/* Prefill attention on the tensor cores (default on; takes effect for f16 /
 * bf16 models of head_dim 64).  0 selects the decode-attention rows instead. */
B2_API int b2_engine_set_prefill_tensor_cores(b2_engine* eng, int32_t enabled);

/* The decode step's linear layers on b2_linear (tcgen05, weights streamed
 * while the kernel before it runs, bias + GELU fused into the FC layer) for
 * f16 / bf16 models and batches of at most 256 rows; cuBLAS otherwise (and
 * for the lm_head).  Default off.  Switching drops the captured graphs. */
B2_API int b2_engine_set_linear_tensor_cores(b2_engine* eng, int32_t enabled);

/* How the decode step's GEMMs of f16 / bf16 engines run on cuBLAS (no effect
 * on f32 engines, which keep cublasGemmEx in pedantic fp32).  Bit 1: cuBLASLt
 * with the algorithm for each (batch bucket, layer shape) chosen by timing the
 * library's top candidates once, before the bucket's graph is captured
 * (cublasGemmEx runs the heuristic's first choice).  Bit 2 (with bit 1): the
 * FC layer's bias + GELU in that GEMM's epilogue (CUBLASLT_EPILOGUE_GELU_BIAS,
 * fp32 before the one rounding) instead of a separate launch.  Switching drops
 * the captured graphs. */
B2_API int b2_engine_set_gemm_mode(b2_engine* eng, int32_t mode);

/* The tied lm_head GEMM and the greedy argmax of decode steps and prefill as
 * one b2_lm_head_argmax launch (tensor cores, no logits written) for f16 /
 * bf16 models; f32 engines keep cuBLAS + argmax.  Replaces the pair
 * gemm_rowmajor(.., wte, d_logits) + launch_argmax (gpu-engine/src/engine.cu:
 * 202-203).  Default off: on B200 (GPT-2 XL shape) it is faster than cuBLAS +
 * argmax at 128 rows and slower at 1-32 and from 256 rows up.  With it on, b2_engine_last_step_outputs has no
 * logits to copy (they are never formed).  Switching drops the captured graphs. */
B2_API int b2_engine_set_lm_head_fused(b2_engine* eng, int32_t enabled);

/* Inspection (no reference counterpart): copies the first `rows` lanes of the
 * last decode_step's final LayerNorm output ([rows][d_model]) and logits
 * ([rows][vocab_size]) into host buffers (either may be NULL), in the engine's
 * dtype.  Synchronises the engine's stream.  For parity tests: a prompt fed
 * through decode_step is a teacher-forced token stream. */
B2_API int b2_engine_last_step_outputs(const b2_engine* eng, int32_t rows, void* hidden_out, void* logits_out);

/* Engine::free_sequence: returns the sequence's blocks; unknown ids are ignored. */
B2_API int b2_engine_free_sequence(b2_engine* eng, int32_t seq_id);

/* Engine::free_blocks: blocks left in the pool. */
B2_API int64_t b2_engine_free_blocks(const b2_engine* eng);

/* Engine::set_use_cuda_graphs. */
B2_API int b2_engine_set_use_cuda_graphs(b2_engine* eng, int32_t enabled);

/* The model shape, and the stream every launch of this engine goes to (a
 * cudaStream_t), for callers that time steps with CUDA events. */
B2_API int b2_engine_shape(const b2_engine* eng, B2ModelShape* out);
B2_API int b2_engine_stream(const b2_engine* eng, b2_stream_t* out);

/* Text of the last engine error on the calling thread. */
B2_API const char* b2_engine_last_error(void);

#define B2_ERR_POOL (-8) /* the KV block pool ran out during decode_step */
#define B2_ERR_IO (-9)   /* a weight file is missing, short or inconsistent */
/* A kernel of the step set a device-side error bit (B2_DEVERR_*, named in
 * b2_engine_last_error): a bounded wait gave up (e.g. a head-sharded peer
 * that never reached the barrier), or a block id, seq_len or token was out of
 * range and clamped.  decode_step / prefill copy the device's error word next
 * to the step's tokens and check it after the step's synchronisation; on a
 * nonzero word they clear it and return this code, with no sequence advanced
 * (the step's tokens are invalid).  The word is shared by everything on the
 * device that uses libb2decode, so a bit set by another caller's kernel fails
 * this engine's next step too.  The reference throws std::runtime_error on
 * CUDA errors (gpu-engine/src/engine.cu:40-44) and has no device-side checks. */
#define B2_ERR_KERNEL (-10)

/* Head-sharded decode (no reference counterpart; the reference engine is
 * single-GPU).  tp_size engines, one per GPU (each created with its
 * tp_rank), each own ceil(n_head / tp_size) heads: their slice of the QKV
 * projection and of every layer's KV cache.  LayerNorms, the output
 * projection, the MLP and the lm_head are replicated.  Each layer's attention
 * stores its heads' output rows into every rank's gathered buffer over NVLink
 * (b2_paged_attention_gather) and the ranks meet at b2_tp_barrier before the
 * output projection reads it.  All ranks must make the same calls with the
 * same sequences in the same order; each computes the same next tokens.
 *
 * Set-up, once, after creation on every rank: exchange the
 * B2_TP_HANDLE_BYTES blob of b2_engine_tp_handle between the ranks (any
 * host transport), then pass all of them, in rank order, to
 * b2_engine_tp_connect.  decode_step before that returns B2_ERR_SHAPE. */
#define B2_TP_HANDLE_BYTES 128 /* two cudaIpcMemHandle_t: gathered buffer, barrier flags */
B2_API int b2_engine_tp_handle(const b2_engine* eng, void* out);
B2_API int b2_engine_tp_connect(b2_engine* eng, const void* handles);

/* The NCCL variant (cfg.tp_allgather = 1), the all-gather the reference's
 * multi-GPU plan would use: each layer's attention writes this rank's heads
 * locally, one ncclAllGather (captured in the step's CUDA graph) collects every
 * rank's slice and a small kernel lays the rows out for the output projection.
 * Set-up: one rank calls b2_engine_tp_nccl_id (B2_TP_NCCL_ID_BYTES), every
 * rank receives that blob (any host transport) and calls
 * b2_engine_tp_connect_nccl.  Destroying the engine destroys its graphs, then
 * its communicator. */
#define B2_TP_NCCL_ID_BYTES 128
B2_API int b2_engine_tp_nccl_id(void* out);
B2_API int b2_engine_tp_connect_nccl(b2_engine* eng, const void* id);

/* The engine's paged-block allocator, exposed so its behaviour can be checked
 * against the reference's BlockPool (gpu-engine/src/kv_cache_pool.cpp:6-28):
 * LIFO free stack, allocate() -> -1 when empty, free() refuses an id out of
 * range (returns 1) or not allocated (returns 2). */
typedef struct b2_block_pool b2_block_pool;
B2_API b2_block_pool* b2_block_pool_create(int32_t num_blocks);
B2_API void b2_block_pool_destroy(b2_block_pool* pool);
B2_API int32_t b2_block_pool_allocate(b2_block_pool* pool);
B2_API int32_t b2_block_pool_free(b2_block_pool* pool, int32_t block_id);
B2_API int32_t b2_block_pool_num_free(const b2_block_pool* pool);

#ifdef __cplusplus
}
#endif

#endif /* B2_ENGINE_H */
