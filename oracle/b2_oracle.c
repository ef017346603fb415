/*
 * b2_oracle.c -- CPU restatement of the reference decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * llm-inference-server_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it.  The product path
 * never links it and has no CPU fallback.
 *
 * Every routine restates the arithmetic of the reference (kanish10/
 * LLM-Inference-Server, gpu-engine/) on host memory:
 *
 *   oracle_paged_attention  gpu-engine/src/reference/cpu_model.cpp:131-162
 *                           (float dot in d order, dot *= scale after the dot,
 *                           running max, float std::exp, double denominator,
 *                           float weight = score/denom, float accumulation in
 *                           key order), with the keys addressed through the
 *                           paged block table exactly as
 *                           gpu-engine/src/kernels/attention.cu:64-92 does
 *                           (layout gpu-engine/include/engine/kv_cache.h:6-7).
 *                           GQA: kv head = h / (n_head / n_kv_head).
 *   oracle_kv_append        gpu-engine/src/kernels/attention.cu:21-47 (a bit copy)
 *   oracle_add_layernorm    residual add (gpu-engine/src/kernels/layernorm.cu:19-24)
 *                           + cpu_model.cpp:27-47 (double mean / variance)
 *   oracle_bias_gelu        cpu_model.cpp:49-54 on x + bias (gelu.cu:13-21)
 *   oracle_add_bias         gpu-engine/src/kernels/embedding.cu:17-24
 *   oracle_embedding        cpu_model.cpp:103-108
 *   oracle_argmax           cpu_model.cpp:182-196 (strict >, lowest index wins)
 *   oracle_linear           cpu_model.cpp:11-25
 *
 * Element storage is dtype-generic (0 = f32, 1 = f16, 2 = bf16); values are
 * widened to float on load, so the oracle sees exactly the rounded inputs
 * the GPU sees.  Parity status: pinned -- the composed forward built from
 * these routines is checked token-for-token against the reference's own
 * CPUModel::greedy_generate (compiled from the reference sources into
 * oracle/_ref) by tests/test_oracle_pin.py.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_BLOCK_TOKENS 16 /* gpu-engine/include/engine/kv_cache.h:8 */

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

static size_t dt_size(int dt) { return dt == DT_F32 ? 4u : 2u; }

/* IEEE binary16 -> binary32, exact. */
static float half_bits_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even. */
static uint16_t float_to_half_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* overflow to inf */
    if (absx < 0x33000001u) return (uint16_t)sign;              /* underflow to 0 */
    int32_t e = (int32_t)(absx >> 23) - 127 + 15;
    uint32_t man = (absx & 0x7fffffu) | 0x800000u;
    uint32_t shift;
    uint32_t hv;
    if (e <= 0) { /* subnormal result */
        shift = (uint32_t)(14 - e);
        hv = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (hv & 1u))) hv++;
        return (uint16_t)(sign | hv);
    }
    hv = ((uint32_t)e << 10) | ((man >> 13) & 0x3ffu);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (hv & 1u))) hv++;
    return (uint16_t)(sign | hv);
}

static float bf16_bits_to_float(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t float_to_bf16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

static inline float ld(const void* base, int dt, size_t i) {
    if (dt == DT_F32) return ((const float*)base)[i];
    if (dt == DT_F16) return half_bits_to_float(((const uint16_t*)base)[i]);
    return bf16_bits_to_float(((const uint16_t*)base)[i]);
}

static inline void st(void* base, int dt, size_t i, float v) {
    if (dt == DT_F32) {
        ((float*)base)[i] = v;
    } else if (dt == DT_F16) {
        ((uint16_t*)base)[i] = float_to_half_bits(v);
    } else {
        ((uint16_t*)base)[i] = float_to_bf16_bits(v);
    }
}

/* Exposed so tests can round host data exactly the way the oracle reads it. */
void oracle_round_to_dtype(int dt, const float* in, void* out, size_t n) {
    for (size_t i = 0; i < n; ++i) st(out, dt, i, in[i]);
}

void oracle_widen_from_dtype(int dt, const void* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = ld(in, dt, i);
}

/* Element offset of (block, layer, kv, token-in-block, head, 0) in the pool:
 * [block][layer][2][16][n_kv_head][head_dim], kv_cache.h:6-7. */
static size_t pool_offset(int block_id, int layer, int kv, int tok, int head, int n_layer,
                          int n_kv_head, int head_dim) {
    const size_t row = (size_t)n_kv_head * head_dim;
    const size_t slab = (size_t)ORACLE_BLOCK_TOKENS * row;
    const size_t block_elems = (size_t)n_layer * 2 * slab;
    return (size_t)block_id * block_elems + (size_t)layer * 2 * slab + (size_t)kv * slab +
           (size_t)tok * row + (size_t)head * head_dim;
}

/* ---------------------------------------------------------------- kv append */

/* attention.cu:21-47: slot seq_lens[b] (pre-append count) of the sequence's
 * block table receives this step's K and V rows.  A pure copy: the element
 * bits are moved unchanged.  Returns 0, or -1 when a block index or slot is
 * out of range (the oracle refuses rather than writing out of bounds). */
int oracle_kv_append(int dt, void* pool, const void* k, const void* v, int kv_row_stride,
                     const int* block_tables, const int* seq_lens, int batch, int n_kv_head,
                     int head_dim, int max_blocks_per_seq, int layer_idx, int n_layer,
                     int num_blocks) {
    const size_t es = dt_size(dt);
    for (int b = 0; b < batch; ++b) {
        const int pos = seq_lens[b];
        const int slot = pos / ORACLE_BLOCK_TOKENS;
        const int tok = pos % ORACLE_BLOCK_TOKENS;
        if (pos < 0 || slot >= max_blocks_per_seq) return -1;
        const int blk = block_tables[(size_t)b * max_blocks_per_seq + slot];
        if (blk < 0 || blk >= num_blocks) return -1;
        for (int h = 0; h < n_kv_head; ++h) {
            const size_t kdst = pool_offset(blk, layer_idx, 0, tok, h, n_layer, n_kv_head, head_dim);
            const size_t vdst = pool_offset(blk, layer_idx, 1, tok, h, n_layer, n_kv_head, head_dim);
            const size_t src = (size_t)b * kv_row_stride + (size_t)h * head_dim;
            memcpy((char*)pool + kdst * es, (const char*)k + src * es, (size_t)head_dim * es);
            memcpy((char*)pool + vdst * es, (const char*)v + src * es, (size_t)head_dim * es);
        }
    }
    return 0;
}

/* ---------------------------------------------------------- paged attention */

typedef struct {
    int dt;
    const void* q;
    int q_row_stride;
    const void* pool;
    const int* block_tables;
    const int* seq_lens;
    float* out;
    int batch, n_head, n_kv_head, head_dim, max_blocks_per_seq, layer_idx, n_layer;
    float scale;
    int next_item; /* shared work counter, guarded by mu */
    pthread_mutex_t mu;
} attn_job;

/* cpu_model.cpp:139-161 for one (b, h): returns 0, or -1 on a bad block index. */
static int attend_one(const attn_job* J, int b, int h, float* scores) {
    const int Dh = J->head_dim;
    const int group = J->n_head / J->n_kv_head;
    const int hk = h / group;
    const int num_keys = J->seq_lens[b];
    const size_t q_base = (size_t)b * J->q_row_stride + (size_t)h * Dh;
    float* out_head = J->out + ((size_t)b * J->n_head + h) * Dh;
    float qv[512];
    for (int d = 0; d < Dh; ++d) qv[d] = ld(J->q, J->dt, q_base + d);
    for (int d = 0; d < Dh; ++d) out_head[d] = 0.0f;
    if (num_keys <= 0) return 0; /* the reference leaves l = 0 and writes 0 */
    if ((num_keys + ORACLE_BLOCK_TOKENS - 1) / ORACLE_BLOCK_TOKENS > J->max_blocks_per_seq) return -1;

    float max_score = -INFINITY;
    for (int j = 0; j < num_keys; ++j) {
        const int blk = J->block_tables[(size_t)b * J->max_blocks_per_seq + j / ORACLE_BLOCK_TOKENS];
        if (blk < 0) return -1;
        const size_t ko = pool_offset(blk, J->layer_idx, 0, j % ORACLE_BLOCK_TOKENS, hk, J->n_layer,
                                      J->n_kv_head, Dh);
        float dot = 0.0f;
        for (int d = 0; d < Dh; ++d) dot += qv[d] * ld(J->pool, J->dt, ko + d);
        dot *= J->scale;
        scores[j] = dot;
        if (dot > max_score) max_score = dot;
    }
    double denom = 0.0;
    for (int j = 0; j < num_keys; ++j) {
        scores[j] = expf(scores[j] - max_score);
        denom += scores[j];
    }
    for (int j = 0; j < num_keys; ++j) {
        const int blk = J->block_tables[(size_t)b * J->max_blocks_per_seq + j / ORACLE_BLOCK_TOKENS];
        const float w = (float)(scores[j] / denom);
        const size_t vo = pool_offset(blk, J->layer_idx, 1, j % ORACLE_BLOCK_TOKENS, hk, J->n_layer,
                                      J->n_kv_head, Dh);
        for (int d = 0; d < Dh; ++d) out_head[d] += w * ld(J->pool, J->dt, vo + d);
    }
    return 0;
}

typedef struct {
    attn_job* job;
    int status;
    int max_keys;
} attn_worker;

static void* attn_thread(void* arg) {
    attn_worker* w = (attn_worker*)arg;
    attn_job* J = w->job;
    float* scores = (float*)malloc(sizeof(float) * (size_t)(w->max_keys > 0 ? w->max_keys : 1));
    const int total = J->batch * J->n_head;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        const int item = J->next_item++;
        pthread_mutex_unlock(&J->mu);
        if (item >= total) break;
        if (attend_one(J, item / J->n_head, item % J->n_head, scores) != 0) w->status = -1;
    }
    free(scores);
    return NULL;
}

/* out: fp32 [batch, n_head, head_dim].  seq_lens are post-append key counts
 * (gpu-engine/include/engine/kernels.h:22-27).  nthreads <= 1 runs inline. */
int oracle_paged_attention(int dt, const void* q, int q_row_stride, const void* pool,
                           const int* block_tables, const int* seq_lens, float* out, int batch,
                           int n_head, int n_kv_head, int head_dim, int max_blocks_per_seq,
                           int layer_idx, int n_layer, float scale, int nthreads) {
    if (head_dim > 512 || n_kv_head <= 0 || n_head % n_kv_head != 0) return -2;
    attn_job J;
    J.dt = dt;
    J.q = q;
    J.q_row_stride = q_row_stride;
    J.pool = pool;
    J.block_tables = block_tables;
    J.seq_lens = seq_lens;
    J.out = out;
    J.batch = batch;
    J.n_head = n_head;
    J.n_kv_head = n_kv_head;
    J.head_dim = head_dim;
    J.max_blocks_per_seq = max_blocks_per_seq;
    J.layer_idx = layer_idx;
    J.n_layer = n_layer;
    J.scale = scale > 0.0f ? scale : 1.0f / sqrtf((float)head_dim);
    J.next_item = 0;
    pthread_mutex_init(&J.mu, NULL);
    int max_keys = 1;
    for (int b = 0; b < batch; ++b)
        if (seq_lens[b] > max_keys) max_keys = seq_lens[b];
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    attn_worker workers[256];
    pthread_t tids[256];
    int status = 0;
    for (int t = 0; t < nthreads; ++t) {
        workers[t].job = &J;
        workers[t].status = 0;
        workers[t].max_keys = max_keys;
    }
    if (nthreads == 1) {
        attn_thread(&workers[0]);
    } else {
        for (int t = 0; t < nthreads; ++t) pthread_create(&tids[t], NULL, attn_thread, &workers[t]);
        for (int t = 0; t < nthreads; ++t) pthread_join(tids[t], NULL);
    }
    for (int t = 0; t < nthreads; ++t)
        if (workers[t].status) status = -1;
    pthread_mutex_destroy(&J.mu);
    return status;
}

/* ------------------------------------------------------ layer-norm and MLP */

/* residual_out = residual_in + (x + bias) (stored in dt); out = LN of that sum
 * with mean and variance accumulated in double (cpu_model.cpp:27-47) over the
 * float sum; the normalised value is computed in double, rounded to float,
 * then * gamma + beta in float -- the exact cpu_model.cpp:44 expression.
 * out is fp32 so the caller can compare before any output rounding;
 * out_dt_copy (may be NULL) receives the same values rounded to dt. */
void oracle_add_layernorm(int dt, float* out, void* out_dt_copy, void* residual_out, const void* x,
                          const void* bias, const void* residual_in, const void* gamma, const void* beta,
                          int batch, int d_model, float eps) {
    float* row = (float*)malloc(sizeof(float) * (size_t)d_model);
    for (int b = 0; b < batch; ++b) {
        const size_t base = (size_t)b * d_model;
        double mean = 0.0;
        for (int d = 0; d < d_model; ++d) {
            /* residual + (x + bias): the bias belongs to the GEMM output x
             * (engine.cu:184-188 adds it before the residual add) */
            float xb = x ? ld(x, dt, base + d) : 0.0f;
            if (bias) xb = xb + ld(bias, dt, d);
            row[d] = ld(residual_in, dt, base + d);
            if (x || bias) row[d] = row[d] + xb;
            mean += row[d];
        }
        mean /= d_model;
        double var = 0.0;
        for (int d = 0; d < d_model; ++d) {
            const double diff = row[d] - mean;
            var += diff * diff;
        }
        var /= d_model;
        const float inv_std = (float)(1.0 / sqrt(var + eps));
        for (int d = 0; d < d_model; ++d) {
            const float y = (float)((row[d] - mean) * inv_std) * ld(gamma, dt, d) + ld(beta, dt, d);
            out[base + d] = y;
            if (out_dt_copy) st(out_dt_copy, dt, base + d, y);
        }
        if (residual_out)
            for (int d = 0; d < d_model; ++d) st(residual_out, dt, base + d, row[d]);
    }
    free(row);
}

/* cpu_model.cpp:49-54, "gelu_new". */
static float gelu_tanh(float x) {
    const float k = 0.7978845608028654f;
    const float inner = k * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

/* out (fp32) = gelu_tanh(x + bias), gelu.cu:13-21. */
void oracle_bias_gelu(int dt, float* out, const void* x, const void* bias, int batch, int d_ff) {
    for (int b = 0; b < batch; ++b)
        for (int d = 0; d < d_ff; ++d) {
            const size_t i = (size_t)b * d_ff + d;
            out[i] = gelu_tanh(ld(x, dt, i) + ld(bias, dt, d));
        }
}

/* out (fp32) = x + bias, embedding.cu:17-24. */
void oracle_add_bias(int dt, float* out, const void* x, const void* bias, int batch, int dim) {
    for (int b = 0; b < batch; ++b)
        for (int d = 0; d < dim; ++d) {
            const size_t i = (size_t)b * dim + d;
            out[i] = ld(x, dt, i) + ld(bias, dt, d);
        }
}

/* out (fp32) = wte[tok] + wpe[pos], cpu_model.cpp:103-108. */
void oracle_embedding(int dt, float* out, const void* wte, const void* wpe, const int* token_ids,
                      const int* positions, int batch, int d_model) {
    for (int b = 0; b < batch; ++b)
        for (int d = 0; d < d_model; ++d)
            out[(size_t)b * d_model + d] = ld(wte, dt, (size_t)token_ids[b] * d_model + d) +
                                           ld(wpe, dt, (size_t)positions[b] * d_model + d);
}

/* cpu_model.cpp:186-195: strict '>' so the lowest index wins a tie. */
void oracle_argmax(int dt, int* out, const void* logits, int batch, int vocab) {
    for (int b = 0; b < batch; ++b) {
        int best = 0;
        float best_v = -INFINITY;
        for (int v = 0; v < vocab; ++v) {
            const float x = ld(logits, dt, (size_t)b * vocab + v);
            if (x > best_v) {
                best_v = x;
                best = v;
            }
        }
        out[b] = best;
    }
}

/* cpu_model.cpp:11-25: out[t,o] = b[o] + sum_i in[t,i] * W[o,i], float, i order. */
typedef struct {
    float* out;
    const float* in;
    int T, I, O;
    const float* W;
    const float* b;
    int o_begin, o_end;
} linear_part;

static void* linear_thread(void* arg) {
    linear_part* p = (linear_part*)arg;
    for (int t = 0; t < p->T; ++t) {
        const float* x = p->in + (size_t)t * p->I;
        float* y = p->out + (size_t)t * p->O;
        for (int o = p->o_begin; o < p->o_end; ++o) {
            const float* w = p->W + (size_t)o * p->I;
            float acc = p->b ? p->b[o] : 0.0f;
            for (int i = 0; i < p->I; ++i) acc += x[i] * w[i];
            y[o] = acc;
        }
    }
    return NULL;
}

/* The per-output sum order is the reference's, so splitting the outputs
 * over threads changes no bit of the result. */
void oracle_linear(float* out, const float* in, int T, int I, int O, const float* W, const float* b,
                   int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    linear_part parts[256];
    pthread_t tids[256];
    for (int t = 0; t < nthreads; ++t) {
        parts[t].out = out;
        parts[t].in = in;
        parts[t].T = T;
        parts[t].I = I;
        parts[t].O = O;
        parts[t].W = W;
        parts[t].b = b;
        parts[t].o_begin = (int)((long long)O * t / nthreads);
        parts[t].o_end = (int)((long long)O * (t + 1) / nthreads);
    }
    if (nthreads == 1) {
        linear_thread(&parts[0]);
        return;
    }
    for (int t = 0; t < nthreads; ++t) pthread_create(&tids[t], NULL, linear_thread, &parts[t]);
    for (int t = 0; t < nthreads; ++t) pthread_join(tids[t], NULL);
}

/* cpu_model.cpp:182-196 with the logits dot in float, d order. */
int oracle_tied_lm_head_argmax(const float* wte, const float* hidden, int vocab, int d_model) {
    int best = 0;
    float best_v = -INFINITY;
    for (int v = 0; v < vocab; ++v) {
        const float* row = wte + (size_t)v * d_model;
        float acc = 0.0f;
        for (int d = 0; d < d_model; ++d) acc += row[d] * hidden[d];
        if (acc > best_v) {
            best_v = acc;
            best = v;
        }
    }
    return best;
}

/* ------------------------------------------------------- paged bookkeeping */

/* gpu-engine/include/engine/kv_cache.h:12-14 (elements are 2 bytes there;
 * this form takes the element size so the fp32 layout is covered too). */
size_t oracle_block_bytes(int n_layer, int n_heads, int head_dim, int elem_bytes) {
    return (size_t)n_layer * 2 * ORACLE_BLOCK_TOKENS * n_heads * head_dim * (size_t)elem_bytes;
}
