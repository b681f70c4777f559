/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the flow-LM attention path.
 *
 * A plain-C restatement of the arithmetic that gradium-ai/xn-ptts runs for its flow-LM
 * transformer, used as the checker for the CUDA library and as the timed CPU baseline.
 * Nothing in the shipped library links, loads or calls this code.
 *
 * parity unpinned: the reference computes this path inside the third-party crate `xn` 0.2.15
 * (Cargo.lock:5623), which is not vendored and cannot be built without a Rust toolchain, and
 * the reference holds no numeric golden vectors for attention. The oracle is pinned only by the
 * reference's own known-answer and equivalence tests, re-expressed in tests/test_oracle.py:
 *   - ptts/src/transformer.rs:1055-1099  (with_seq_budget prefix copy, zero tail, refusal)
 *   - ptts/src/transformer.rs:1112-1164  (grouped-query == repeated heads, 1e-6)
 *   - ptts/src/transformer.rs:1169-1225  (device-position step == host step, 1e-6)
 *
 * Storage modes (`store_bf16`, a bit mask). 0 is the reference's CPU path (T = f32 everywhere).
 * ORACLE_ROUND_KV rounds the rotated k and the v rows to bf16 as they enter the cache, as the
 * CUDA library stores them. ORACLE_ROUND_OPERANDS also rounds the GEMM inputs (the normalised
 * rows, the attention output, the GELU output) to bf16, as a bf16-operand GEMM would. The rotated
 * q and the residual stream stay f32 in every mode.
 */
#ifndef PTTS_ORACLE_H
#define PTTS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORACLE_ROUND_KV 1
#define ORACLE_ROUND_OPERANDS 2

/* bf16 <-> f32, round to nearest even (NaN kept quiet). */
float oracle_bf16_to_f32(uint16_t h);
uint16_t oracle_f32_to_bf16(float f);
void oracle_round_bf16(float* x, int64_t n);

/* rope.rs:44-48: inv_freq[i] = 1 / max_period^(i / (head_dim/2)), in f32. */
void oracle_rope_inv_freq(int head_dim, float max_period, float* inv_freq);
/* rope.rs:50-57: cos/sin tables [n, head_dim/2] at f32 positions. */
void oracle_rope_table(int head_dim, const float* positions, int n, float max_period,
                       float* cos_out, float* sin_out);
/* xn `rope_i` on one head row: interleaved pairs (x[2i], x[2i+1]) turned by angle pos*inv_freq[i]. */
void oracle_rope_row(float* x, int head_dim, const float* cos_row, const float* sin_row);

/*
 * One attention call of StreamingMultiheadAttention::forward (transformer.rs:183-251) after the
 * projections, for a ragged batch of independent streams.
 *
 * q [n_rows, H, D]; k, v [n_rows, KVH, D] (un-rotated, as projected). Sequence i is stream
 * streams[i]; its rows are row_offsets[i]..row_offsets[i+1] and sit at positions
 * lengths[stream] + j. Every row's k and v are rotated (k only), repeated over the H / KVH query
 * heads that share them (transformer.rs:201-211) and written into the cache
 * [num_streams, capacity, H, D] at those positions (complete_kv, transformer.rs:84-91). Then
 * row j attends to keys 0 ..= lengths[stream] + j (materialize_causal_mask,
 * transformer.rs:94-108; one row is the sdpa_decode case). out [n_rows, H*D], f32.
 * Lengths are not advanced. Returns 0, or -2 when a sequence does not fit its capacity.
 */
int oracle_attend(const float* q, const float* k, const float* v, int num_heads, int num_kv_heads,
                  int head_dim, float* k_cache, float* v_cache, int num_streams, int capacity,
                  const int32_t* lengths, const int32_t* streams, const int32_t* row_offsets,
                  int n_seq, float max_period, int store_bf16, float* out, int n_threads);

/* y[m, n] = sum_b scale[n, b] * sum_{k in block b} x[m, k] * w[n, k]; group 0 = one block. */
void oracle_linear_i8(const float* x, const int8_t* w, const float* scale, int m, int n, int k,
                      int group, float* y, int n_threads);
/* LayerNorm over the last dim, biased variance, transformer.rs:547-548 (eps 1e-5). */
void oracle_layer_norm(const float* x, const float* gamma, const float* beta, int m, int d,
                       float eps, float* y);
/* GELU: erf form (transformer.rs:624) or tanh form x*sigmoid(2u) (transformer.rs:500-504). */
float oracle_gelu(float x, int tanh_form);

/* A flow-LM transformer with int8 per-output-channel (or block-32) weights. */
typedef struct {
    int d_model, num_heads, num_kv_heads, head_dim, num_layers, dim_feedforward;
    float max_period;
    int scale_group; /* 0: one scale per output row; else block length along K */
    int gelu_tanh;   /* 0: erf (phonon checkpoints), 1: tanh */
    /* Per-layer weights, concatenated over layers, rows = output features, K contiguous. */
    const int8_t* w_qkv;  /* [L, (H + 2 KVH) * D, d_model] */
    const float* s_qkv;   /* [L, rows, groups] */
    const int8_t* w_out;  /* [L, d_model, H * D] */
    const float* s_out;
    const int8_t* w_ff1;  /* [L, ff, d_model] */
    const float* s_ff1;
    const int8_t* w_ff2;  /* [L, d_model, ff] */
    const float* s_ff2;
    const float* ln1_g;   /* [L, d_model] */
    const float* ln1_b;
    const float* ln2_g;
    const float* ln2_b;
} oracle_model_desc;

typedef struct oracle_model oracle_model;
oracle_model* oracle_model_create(const oracle_model_desc* desc);
void oracle_model_free(oracle_model* m);

/*
 * StreamingTransformer::forward (transformer.rs:742-808) over a ragged batch: for each layer,
 * x += attn(LN1 x); x += W2 GELU(W1 LN2 x) (transformer.rs:591-634). x [n_rows, d_model] is the
 * residual stream (in: the layer-0 input, out: the last layer's output). Caches are
 * [L, num_streams, capacity, H, D]. Lengths are not advanced. Returns 0 or -2 (capacity).
 */
int oracle_model_forward(const oracle_model* m, float* x, float* k_cache, float* v_cache,
                         int num_streams, int capacity, const int32_t* lengths,
                         const int32_t* streams, const int32_t* row_offsets, int n_seq,
                         int store_bf16, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
