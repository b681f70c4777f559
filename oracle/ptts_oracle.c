/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the flow-LM attention path of gradium-ai/xn-ptts.
 * parity unpinned (no golden vectors exist for this path; see ptts_oracle.h for what pins it).
 *
 * Each function names the reference lines whose behaviour it restates. The arithmetic that
 * the reference delegates to `xn` 0.2.15 (rope_i, sdpa_decode, matmul/softmax, LayerNorm,
 * gelu_erf, the quantised linears) is restated from the published definitions of those ops.
 */
#include "ptts_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float oracle_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float rb(float f) { return oracle_bf16_to_f32(oracle_f32_to_bf16(f)); }

void oracle_round_bf16(float* x, int64_t n) {
    for (int64_t i = 0; i < n; i++) x[i] = rb(x[i]);
}

/* rope.rs:44-48 */
void oracle_rope_inv_freq(int head_dim, float max_period, float* inv_freq) {
    int half = head_dim / 2;
    for (int i = 0; i < half; i++) inv_freq[i] = 1.0f / powf(max_period, (float)i / (float)half);
}

/* rope.rs:50-57: angle = pos * freq in f32, then cos and sin of that f32 angle. */
void oracle_rope_table(int head_dim, const float* positions, int n, float max_period,
                       float* cos_out, float* sin_out) {
    int half = head_dim / 2;
    float inv_freq[512];
    oracle_rope_inv_freq(head_dim, max_period, inv_freq);
    for (int p = 0; p < n; p++) {
        for (int i = 0; i < half; i++) {
            float angle = positions[p] * inv_freq[i];
            cos_out[(int64_t)p * half + i] = cosf(angle);
            sin_out[(int64_t)p * half + i] = sinf(angle);
        }
    }
}

/* xn `rope_i` (called at rope.rs:89-90): pairs (2i, 2i+1) of one head row. */
void oracle_rope_row(float* x, int head_dim, const float* c, const float* s) {
    for (int i = 0; i < head_dim / 2; i++) {
        float x0 = x[2 * i], x1 = x[2 * i + 1];
        x[2 * i] = x0 * c[i] - x1 * s[i];
        x[2 * i + 1] = x0 * s[i] + x1 * c[i];
    }
}

static void rope_at(float* x, int head_dim, const float* inv_freq, int pos) {
    float c[256], s[256];
    for (int i = 0; i < head_dim / 2; i++) {
        float angle = (float)pos * inv_freq[i];
        c[i] = cosf(angle);
        s[i] = sinf(angle);
    }
    oracle_rope_row(x, head_dim, c, s);
}

/*
 * transformer.rs:183-251 after the in_proj: split, GQA repeat (:201-211), RoPE (:214), append
 * (complete_kv :84-91), then softmax(q k^T * 1/sqrt(d) + causal mask) v (:229-248).
 */
int oracle_attend(const float* q, const float* k, const float* v, int H, int KVH, int D,
                  float* k_cache, float* v_cache, int num_streams, int capacity,
                  const int32_t* lengths, const int32_t* streams, const int32_t* row_offsets,
                  int n_seq, float max_period, int store_bf16, float* out, int n_threads) {
    float inv_freq[256];
    oracle_rope_inv_freq(D, max_period, inv_freq);
    const int group = H / KVH;
    const int64_t row = (int64_t)H * D;
    const float scale = 1.0f / sqrtf((float)D); /* transformer.rs:215 */
    for (int i = 0; i < n_seq; i++) {
        int s = streams[i];
        if (s < 0 || s >= num_streams) return -1;
        int t = row_offsets[i + 1] - row_offsets[i];
        if (lengths[s] + t > capacity) return -2;
    }
    int n_rows = row_offsets[n_seq];
    float* qr = (float*)malloc(sizeof(float) * (size_t)n_rows * row);
    /* Rotate q; rotate, round and append k; round and append v. */
    for (int i = 0; i < n_seq; i++) {
        int s = streams[i];
        for (int r = row_offsets[i]; r < row_offsets[i + 1]; r++) {
            int pos = lengths[s] + (r - row_offsets[i]);
            for (int h = 0; h < H; h++) {
                float* qh = qr + (int64_t)r * row + (int64_t)h * D;
                memcpy(qh, q + (int64_t)r * row + (int64_t)h * D, sizeof(float) * D);
                rope_at(qh, D, inv_freq, pos); /* q stays f32 in both modes */
            }
            for (int g = 0; g < KVH; g++) {
                float kr[256], vr[256];
                memcpy(kr, k + ((int64_t)r * KVH + g) * D, sizeof(float) * D);
                memcpy(vr, v + ((int64_t)r * KVH + g) * D, sizeof(float) * D);
                rope_at(kr, D, inv_freq, pos);
                if (store_bf16 & ORACLE_ROUND_KV) {
                    oracle_round_bf16(kr, D);
                    oracle_round_bf16(vr, D);
                }
                for (int rep = 0; rep < group; rep++) {
                    int h = g * group + rep;
                    int64_t at = (((int64_t)s * capacity + pos) * H + h) * D;
                    memcpy(k_cache + at, kr, sizeof(float) * D);
                    memcpy(v_cache + at, vr, sizeof(float) * D);
                }
            }
        }
    }
    /* Attention, one (row, head) at a time. */
    int64_t work = (int64_t)n_rows * H;
#pragma omp parallel num_threads(n_threads > 0 ? n_threads : 1)
    {
        float* sc = (float*)malloc(sizeof(float) * (size_t)(capacity + 1));
#pragma omp for schedule(dynamic, 4)
        for (int64_t w = 0; w < work; w++) {
            int r = (int)(w / H), h = (int)(w % H);
            int lo = 0, hi = n_seq - 1; /* the sequence holding row r */
            while (lo < hi) {
                int mid = (lo + hi + 1) / 2;
                if (row_offsets[mid] <= r) lo = mid; else hi = mid - 1;
            }
            int i = lo;
            int s = streams[i];
            int nk = lengths[s] + (r - row_offsets[i]) + 1; /* keys k <= q + current_end */
            const float* qh = qr + (int64_t)r * row + (int64_t)h * D;
            float m = -INFINITY;
            for (int j = 0; j < nk; j++) {
                const float* kj = k_cache + (((int64_t)s * capacity + j) * H + h) * D;
                float acc = 0.f;
#pragma omp simd reduction(+ : acc)
                for (int d = 0; d < D; d++) acc += qh[d] * kj[d];
                sc[j] = acc * scale;
                if (sc[j] > m) m = sc[j];
            }
            float sum = 0.f;
            for (int j = 0; j < nk; j++) {
                sc[j] = expf(sc[j] - m);
                sum += sc[j];
            }
            float o[256];
            for (int d = 0; d < D; d++) o[d] = 0.f;
            for (int j = 0; j < nk; j++) {
                const float* vj = v_cache + (((int64_t)s * capacity + j) * H + h) * D;
                float p = sc[j];
#pragma omp simd
                for (int d = 0; d < D; d++) o[d] += p * vj[d];
            }
            float* oh = out + (int64_t)r * row + (int64_t)h * D;
            for (int d = 0; d < D; d++) oh[d] = o[d] / sum;
        }
        free(sc);
    }
    free(qr);
    return 0;
}

/* Dot products of one x row against 8 weight rows held as f32. */
static inline void dot8(const float* x, const float* w, int64_t ldw, int k, float* out) {
    float a0 = 0, a1 = 0, a2 = 0, a3 = 0, a4 = 0, a5 = 0, a6 = 0, a7 = 0;
    const float *w0 = w, *w1 = w + ldw, *w2 = w + 2 * ldw, *w3 = w + 3 * ldw;
    const float *w4 = w + 4 * ldw, *w5 = w + 5 * ldw, *w6 = w + 6 * ldw, *w7 = w + 7 * ldw;
#pragma omp simd reduction(+ : a0, a1, a2, a3, a4, a5, a6, a7)
    for (int i = 0; i < k; i++) {
        float xi = x[i];
        a0 += xi * w0[i];
        a1 += xi * w1[i];
        a2 += xi * w2[i];
        a3 += xi * w3[i];
        a4 += xi * w4[i];
        a5 += xi * w5[i];
        a6 += xi * w6[i];
        a7 += xi * w7[i];
    }
    out[0] = a0; out[1] = a1; out[2] = a2; out[3] = a3;
    out[4] = a4; out[5] = a5; out[6] = a6; out[7] = a7;
}

static inline float dot1(const float* x, const float* w, int k) {
    float a = 0;
#pragma omp simd reduction(+ : a)
    for (int i = 0; i < k; i++) a += x[i] * w[i];
    return a;
}

/*
 * y = x W^T with W = q * scale: int8 rows, f32 scales per output row (group 0) or per block of
 * `group` weights along K (the GGML q8_0 layout of ptts/examples/quantize.rs:46-47).
 * wf holds the int8 values as f32.
 */
static void linear_f32w(const float* x, const float* wf, const float* scale, int m, int n, int k,
                        int group, float* y, int n_threads) {
    int nb = (n + 7) / 8;
    int groups = group > 0 ? k / group : 1;
#pragma omp parallel for collapse(2) schedule(static) num_threads(n_threads > 0 ? n_threads : 1)
    for (int b = 0; b < nb; b++) {
        for (int mi = 0; mi < m; mi++) {
            int n0 = b * 8;
            const float* xr = x + (int64_t)mi * k;
            float* yr = y + (int64_t)mi * n;
            if (group == 0 && n0 + 8 <= n) {
                float acc[8];
                dot8(xr, wf + (int64_t)n0 * k, k, k, acc);
                for (int j = 0; j < 8; j++) yr[n0 + j] = acc[j] * scale[n0 + j];
            } else {
                for (int nn = n0; nn < n && nn < n0 + 8; nn++) {
                    const float* wr = wf + (int64_t)nn * k;
                    if (group == 0) {
                        yr[nn] = dot1(xr, wr, k) * scale[nn];
                    } else {
                        float acc = 0.f;
                        for (int g = 0; g < groups; g++)
                            acc += scale[(int64_t)nn * groups + g] *
                                   dot1(xr + g * group, wr + g * group, group);
                        yr[nn] = acc;
                    }
                }
            }
        }
    }
}

void oracle_linear_i8(const float* x, const int8_t* w, const float* scale, int m, int n, int k,
                      int group, float* y, int n_threads) {
    float* wf = (float*)malloc(sizeof(float) * (size_t)n * k);
    for (int64_t i = 0; i < (int64_t)n * k; i++) wf[i] = (float)w[i];
    linear_f32w(x, wf, scale, m, n, k, group, y, n_threads);
    free(wf);
}

/* xn LayerNorm: (x - mean) / sqrt(var + eps) * gamma + beta, biased variance. */
void oracle_layer_norm(const float* x, const float* gamma, const float* beta, int m, int d,
                       float eps, float* y) {
    for (int r = 0; r < m; r++) {
        const float* xr = x + (int64_t)r * d;
        float mean = 0.f;
        for (int i = 0; i < d; i++) mean += xr[i];
        mean /= (float)d;
        float var = 0.f;
        for (int i = 0; i < d; i++) {
            float c = xr[i] - mean;
            var += c * c;
        }
        var /= (float)d;
        float inv = 1.0f / sqrtf(var + eps);
        for (int i = 0; i < d; i++) y[(int64_t)r * d + i] = (xr[i] - mean) * inv * gamma[i] + beta[i];
    }
}

/* transformer.rs:624 (erf, exact) and :500-504 (tanh form as x * sigmoid(2u)). */
float oracle_gelu(float x, int tanh_form) {
    if (tanh_form) {
        float u2 = (x * x * 0.07135482f + 1.595769f) * x;
        return x / (1.0f + expf(-u2));
    }
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

struct oracle_model {
    oracle_model_desc d;
    float *wq, *wo, *w1, *w2; /* int8 values as f32, all layers */
};

static float* to_f32(const int8_t* w, int64_t n) {
    float* f = (float*)malloc(sizeof(float) * (size_t)n);
    for (int64_t i = 0; i < n; i++) f[i] = (float)w[i];
    return f;
}

oracle_model* oracle_model_create(const oracle_model_desc* desc) {
    oracle_model* m = (oracle_model*)calloc(1, sizeof(oracle_model));
    m->d = *desc;
    int64_t L = desc->num_layers, dm = desc->d_model, hd = (int64_t)desc->num_heads * desc->head_dim;
    int64_t qkv = (int64_t)(desc->num_heads + 2 * desc->num_kv_heads) * desc->head_dim;
    int64_t ff = desc->dim_feedforward;
    m->wq = to_f32(desc->w_qkv, L * qkv * dm);
    m->wo = to_f32(desc->w_out, L * dm * hd);
    m->w1 = to_f32(desc->w_ff1, L * ff * dm);
    m->w2 = to_f32(desc->w_ff2, L * dm * ff);
    return m;
}

void oracle_model_free(oracle_model* m) {
    if (!m) return;
    free(m->wq);
    free(m->wo);
    free(m->w1);
    free(m->w2);
    free(m);
}

/* StreamingTransformer::forward (transformer.rs:742-808) with StreamingTransformerLayer::forward
 * (transformer.rs:591-634), no layer scale (the flow LM has none). */
int oracle_model_forward(const oracle_model* m, float* x, float* k_cache, float* v_cache,
                         int num_streams, int capacity, const int32_t* lengths,
                         const int32_t* streams, const int32_t* row_offsets, int n_seq,
                         int store_bf16, int n_threads) {
    const oracle_model_desc* d = &m->d;
    const int dm = d->d_model, H = d->num_heads, KVH = d->num_kv_heads, D = d->head_dim;
    const int hd = H * D, kvd = KVH * D, nqkv = hd + 2 * kvd, ff = d->dim_feedforward;
    const int rows = row_offsets[n_seq];
    const int g = d->scale_group;
    const int64_t sq = g ? (int64_t)nqkv * (dm / g) : nqkv, so = g ? (int64_t)dm * (hd / g) : dm;
    const int64_t s1 = g ? (int64_t)ff * (dm / g) : ff, s2 = g ? (int64_t)dm * (ff / g) : dm;
    const int64_t cache_layer = (int64_t)num_streams * capacity * H * D;
    for (int i = 0; i < n_seq; i++) {
        if (lengths[streams[i]] + row_offsets[i + 1] - row_offsets[i] > capacity) return -2;
    }
    float* h = (float*)malloc(sizeof(float) * (size_t)rows * (dm > hd ? dm : hd));
    float* qkv = (float*)malloc(sizeof(float) * (size_t)rows * nqkv);
    float* q = (float*)malloc(sizeof(float) * (size_t)rows * hd);
    float* k = (float*)malloc(sizeof(float) * (size_t)rows * kvd);
    float* v = (float*)malloc(sizeof(float) * (size_t)rows * kvd);
    float* a = (float*)malloc(sizeof(float) * (size_t)rows * hd);
    float* y = (float*)malloc(sizeof(float) * (size_t)rows * (ff > dm ? ff : dm));
    float* f = (float*)malloc(sizeof(float) * (size_t)rows * ff);
    int rc = 0;
    for (int l = 0; l < d->num_layers && rc == 0; l++) {
        /* x + attn(norm1(x)) */
        oracle_layer_norm(x, d->ln1_g + (int64_t)l * dm, d->ln1_b + (int64_t)l * dm, rows, dm, 1e-5f, h);
        if (store_bf16 & ORACLE_ROUND_OPERANDS) oracle_round_bf16(h, (int64_t)rows * dm);
        linear_f32w(h, m->wq + (int64_t)l * nqkv * dm, d->s_qkv + l * sq, rows, nqkv, dm, g, qkv,
                    n_threads);
        for (int r = 0; r < rows; r++) { /* [q | k | v] on the last dim, transformer.rs:197-211 */
            memcpy(q + (int64_t)r * hd, qkv + (int64_t)r * nqkv, sizeof(float) * hd);
            memcpy(k + (int64_t)r * kvd, qkv + (int64_t)r * nqkv + hd, sizeof(float) * kvd);
            memcpy(v + (int64_t)r * kvd, qkv + (int64_t)r * nqkv + hd + kvd, sizeof(float) * kvd);
        }
        rc = oracle_attend(q, k, v, H, KVH, D, k_cache + l * cache_layer, v_cache + l * cache_layer,
                           num_streams, capacity, lengths, streams, row_offsets, n_seq,
                           d->max_period, store_bf16, a, n_threads);
        if (store_bf16 & ORACLE_ROUND_OPERANDS) oracle_round_bf16(a, (int64_t)rows * hd);
        linear_f32w(a, m->wo + (int64_t)l * dm * hd, d->s_out + l * so, rows, dm, hd, g, y, n_threads);
        for (int64_t i = 0; i < (int64_t)rows * dm; i++) x[i] += y[i];
        /* x + ff(norm2(x)) */
        oracle_layer_norm(x, d->ln2_g + (int64_t)l * dm, d->ln2_b + (int64_t)l * dm, rows, dm, 1e-5f, h);
        if (store_bf16 & ORACLE_ROUND_OPERANDS) oracle_round_bf16(h, (int64_t)rows * dm);
        linear_f32w(h, m->w1 + (int64_t)l * ff * dm, d->s_ff1 + l * s1, rows, ff, dm, g, f, n_threads);
        for (int64_t i = 0; i < (int64_t)rows * ff; i++) f[i] = oracle_gelu(f[i], d->gelu_tanh);
        if (store_bf16 & ORACLE_ROUND_OPERANDS) oracle_round_bf16(f, (int64_t)rows * ff);
        linear_f32w(f, m->w2 + (int64_t)l * dm * ff, d->s_ff2 + l * s2, rows, dm, ff, g, y, n_threads);
        for (int64_t i = 0; i < (int64_t)rows * dm; i++) x[i] += y[i];
    }
    free(h); free(qkv); free(q); free(k); free(v); free(a); free(y); free(f);
    return rc;
}
