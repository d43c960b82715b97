/*
 * floyd_oracle.c - CPU restatement of floyd's verify step (TEST
 * INFRASTRUCTURE ONLY; see floyd_oracle.h for who may use it and how its
 * parity is pinned).
 *
 * The model is the compressed-latent MLA + MoE transformer that floyd's
 * Moonlight Metal runtime executes (moonlight_metal.m:287-725), with the
 * MoE contract of moe_route.h / moe_exec.h and the acceptance rule of the
 * DS4 speculative verifier (patches/ds4/deepseek-v4-dspark-metal.patch
 * :1727-1906).  Weights come from the integer synthetic generator of
 * include/floyd_synth.h, so the CUDA backend and this file hold identical
 * weights for the same seed.
 */
#include "floyd_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../include/floyd_synth.h"

/* ---- primitives ---------------------------------------------------------- */

void orc_philox4x32_10(const uint32_t counter[4], const uint32_t key[2],
                       uint32_t out[4]) {
    fc_philox4x32_10(counter, key, out);
}

float orc_fp16_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits >> 15) << 31;
    int exponent = (bits >> 10) & 31;
    uint32_t mantissa = bits & 1023u;
    float value;
    if (exponent == 0) value = ldexpf((float)mantissa, -24);
    else if (exponent == 31) value = mantissa ? NAN : INFINITY;
    else value = ldexpf((float)(mantissa | 1024u), exponent - 25);
    uint32_t out;
    memcpy(&out, &value, 4);
    out |= sign;
    memcpy(&value, &out, 4);
    return value;
}

uint16_t orc_f32_to_fp16(float value) {
    /* IEEE round-to-nearest-even conversion, the same as __float2half_rn. */
    uint32_t x;
    memcpy(&x, &value, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) /* inf or nan */
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* overflow */
    if (absx < 0x33000001u) return (uint16_t)sign;               /* < half min subnormal */
    int exponent = (int)(absx >> 23) - 127;
    uint32_t mantissa = (absx & 0x7FFFFFu) | 0x800000u;
    int shift;
    uint32_t base;
    if (exponent < -14) { /* subnormal half */
        shift = -exponent - 14 + 13;
        base = 0;
    } else {
        shift = 13;
        base = (uint32_t)(exponent + 15) << 10;
        mantissa &= 0x7FFFFFu;
    }
    uint32_t kept = mantissa >> shift;
    uint32_t rest = mantissa & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    uint32_t result = base + kept;
    if (rest > half || (rest == half && (kept & 1u))) result += 1u;
    return (uint16_t)(sign | result);
}

float orc_e8m0_to_f32(uint8_t code) {
    if (code == 255) return NAN;
    return ldexpf(1.0f, (int)code - 127);
}

static const float orc_e2m1_table[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f
};

float orc_e2m1_to_f32(uint8_t code) { return orc_e2m1_table[code & 15]; }

static inline float value_of(int fmt, int8_t v) {
    return fmt == FC_FMT_MXFP4 ? orc_e2m1_table[(uint8_t)v & 15] : (float)v;
}

void orc_gemv(int fmt, const int8_t *values, const float *scales,
              const float *f32, int O, int K, const float *x, int S, float *y) {
    int groups = K / 32;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < O; ++o) {
        for (int s = 0; s < S; ++s) {
            const float *xs = x + (int64_t)s * K;
            float sum = 0.0f;
            if (fmt == FC_FMT_F32) {
                const float *w = f32 + (int64_t)o * K;
                for (int k = 0; k < K; ++k) sum += w[k] * xs[k];
            } else {
                const int8_t *w = values + (int64_t)o * K;
                for (int g = 0; g < groups; ++g) {
                    float partial = 0.0f;
                    for (int k = 32 * g; k < 32 * g + 32; ++k)
                        partial += value_of(fmt, w[k]) * xs[k];
                    sum += partial * scales[(int64_t)o * groups + g];
                }
            }
            y[(int64_t)s * O + o] = sum;
        }
    }
}

void orc_rmsnorm(const float *x, const float *w, int rows, int width, float eps,
                 float *out) {
    for (int r = 0; r < rows; ++r) {
        const float *src = x + (int64_t)r * width;
        float sum = 0.0f;
        for (int c = 0; c < width; ++c) sum += src[c] * src[c];
        float scale = 1.0f / sqrtf(sum / (float)width + eps);
        for (int c = 0; c < width; ++c)
            out[(int64_t)r * width + c] = src[c] * scale * w[c];
    }
}

void orc_rope(const float *in, float *out, int width, int position, float theta) {
    int half = width / 2;
    float tmp[512];
    for (int c = 0; c < width; ++c) tmp[c] = in[c];
    for (int p = 0; p < half; ++p) {
        float angle = (float)position * powf(theta, -2.0f * (float)p / (float)width);
        float cosine = cosf(angle), sine = sinf(angle);
        float first = tmp[2 * p], second = tmp[2 * p + 1];
        out[p] = first * cosine - second * sine;
        out[half + p] = second * cosine + first * sine;
    }
}

static void route_scores(const float *logits, int n, int score_fn, float *scores) {
    if (score_fn == FC_SCORE_SOFTMAX) {
        float m = logits[0];
        for (int e = 1; e < n; ++e) if (logits[e] > m) m = logits[e];
        float sum = 0.0f;
        for (int e = 0; e < n; ++e) { scores[e] = expf(logits[e] - m); sum += scores[e]; }
        for (int e = 0; e < n; ++e) scores[e] /= sum;
        return;
    }
    for (int e = 0; e < n; ++e) {
        float x = logits[e];
        if (score_fn == FC_SCORE_SQRT_SOFTPLUS) {
            float sp;
            if (x > 20.0f) sp = x;
            else if (x < -20.0f) sp = expf(x);
            else sp = log1pf(expf(x));
            scores[e] = sqrtf(sp);
        } else {
            scores[e] = 1.0f / (1.0f + expf(-x));
        }
    }
}

int orc_route(const float *logits, const float *bias, int n_experts, int top_k,
              int score_fn, int normalize, float routed_scale,
              const int *fixed, int *indices, float *weights) {
    float scores[1024], choice[1024];
    if (n_experts <= 0 || n_experts > 1024 || top_k <= 0) return 0;
    if (top_k > n_experts) top_k = n_experts;
    route_scores(logits, n_experts, score_fn, scores);
    if (fixed) { /* moe_route_fixed, moe_route.h:76-87 */
        for (int k = 0; k < top_k; ++k) {
            if (fixed[k] < 0 || fixed[k] >= n_experts) return 0;
            indices[k] = fixed[k];
            weights[k] = scores[fixed[k]];
        }
    } else { /* moe_route_select, moe_route.h:47-74 */
        for (int e = 0; e < n_experts; ++e) choice[e] = scores[e] + (bias ? bias[e] : 0.0f);
        for (int k = 0; k < top_k; ++k) {
            int best = -1;
            float best_value = -INFINITY;
            for (int e = 0; e < n_experts; ++e) {
                int taken = 0;
                for (int j = 0; j < k; ++j) if (indices[j] == e) { taken = 1; break; }
                if (!taken && choice[e] > best_value) { best = e; best_value = choice[e]; }
            }
            indices[k] = best;
            weights[k] = scores[best];
        }
    }
    /* moe_route_finalize, moe_route.h:89-99 */
    if (normalize) {
        float sum = 0.0f;
        for (int k = 0; k < top_k; ++k) sum += weights[k];
        sum += 1e-20f;
        for (int k = 0; k < top_k; ++k) weights[k] /= sum;
    }
    for (int k = 0; k < top_k; ++k) weights[k] *= routed_scale;
    return top_k;
}

int orc_argmax(const float *logits, int n) {
    int best = -1;
    for (int i = 0; i < n; ++i) {
        float v = logits[i];
        if (v != v) continue;
        if (best < 0 || v > logits[best]) best = i;
    }
    return best;
}

int orc_accept_greedy(const int *row_tops, const int *ids, int k) {
    int commit = 1;
    for (int i = 1; i <= k; ++i) {
        if (row_tops[i - 1] != ids[i]) break;
        commit++;
    }
    return commit;
}

float orc_accept_uniform(uint64_t seed, uint64_t counter, int row) {
    uint32_t c[4] = {(uint32_t)row, 0xACCE97EDu, (uint32_t)counter, (uint32_t)(counter >> 32)};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t out[4];
    fc_philox4x32_10(c, key, out);
    return (float)(out[0] >> 8) * (1.0f / 16777216.0f);
}

float orc_gumbel(uint64_t seed, uint64_t counter, int row, int v) {
    uint32_t c[4] = {(uint32_t)v >> 2, (uint32_t)row, (uint32_t)counter,
                     (uint32_t)(counter >> 32) ^ 0x9E3779B9u};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t out[4];
    fc_philox4x32_10(c, key, out);
    float u = ((float)(out[v & 3] >> 8) + 0.5f) * (1.0f / 16777216.0f);
    return -logf(-logf(u));
}

static int sample_excluding(const float *logits, int V, float temperature,
                            uint64_t seed, uint64_t counter, int row, int excluded) {
    int best = -1;
    float best_value = -INFINITY;
    for (int v = 0; v < V; ++v) {
        if (v == excluded || logits[v] != logits[v]) continue;
        float z = logits[v] / temperature + orc_gumbel(seed, counter, row, v);
        if (best < 0 || z > best_value) { best = v; best_value = z; }
    }
    return best;
}

static float softmax_prob(const float *logits, int V, float temperature, int x) {
    float m = -INFINITY;
    for (int v = 0; v < V; ++v) {
        float z = logits[v] / temperature;
        if (z > m) m = z;
    }
    float sum = 0.0f;
    for (int v = 0; v < V; ++v) sum += expf(logits[v] / temperature - m);
    return expf(logits[x] / temperature - m) / sum;
}

int orc_accept_sample(const float *logits, int V, const int *ids, int k,
                      float temperature, uint64_t seed, uint64_t counter,
                      int *next_token) {
    for (int i = 1; i <= k; ++i) {
        const float *row = logits + (int64_t)(i - 1) * V;
        float p = softmax_prob(row, V, temperature, ids[i]);
        float u = orc_accept_uniform(seed, counter, i - 1);
        if (!(u < p)) {
            *next_token = sample_excluding(row, V, temperature, seed, counter, i - 1, ids[i]);
            return i;
        }
    }
    *next_token = sample_excluding(logits + (int64_t)k * V, V, temperature, seed, counter, k, -1);
    return k + 1;
}

/* ---- model ---------------------------------------------------------------- */

typedef struct {
    int fmt, O, K;
    int8_t *values;   /* [O][K] logical (int8, int4 value, or e2m1 code)   */
    float *scales;    /* [O][K/32]                                         */
    uint16_t *scale_bits; /* fp16 bits or e8m0 byte per group              */
    float *f32;       /* [O][K] for F32                                    */
    int pending;      /* 1: not generated yet (routed experts are generated
                         on first use, so full-width configs with hundreds of
                         experts need host memory only for the ones a test
                         touches)                                           */
    uint64_t seed;
    uint32_t tid;
} Mat;

typedef struct {
    float *attn_norm, *ffn_norm, *kv_a_norm, *q_a_norm;
    Mat q_proj, q_a, q_b, kv_a, kv_b, o_proj;
    Mat router;       /* F32 [E][D] */
    float *bias;      /* [E] or NULL */
    int *hash;        /* [V][top_k] or NULL */
    Mat *gate, *up, *down;   /* [E] */
    Mat sh_gate, sh_up, sh_down;
    Mat d_gate, d_up, d_down;
    int dense;
    float *enorm, *hnorm, *head_norm;  /* MTP drafter layer only */
    Mat eh_proj;                       /* MTP: [D][2D] */
} Layer;

struct OrcModel {
    FcModelConfig c;
    uint64_t seed;
    Mat embed, lm_head;
    float *final_norm;
    Layer *layers;
};

struct OrcSession {
    OrcModel *m;
    int ctx, kv_fp16, position;
    float *latent; /* [layers (+ MTP)][ctx][L] */
    float *rope;   /* [layers (+ MTP)][ctx][R] */
    float *last_x; /* final pre-norm hidden rows of the last forward */
    float *hist;   /* final pre-norm hidden row of every position [ctx][D] */
    int *tok;      /* token id of every position [ctx]                      */
    int last_rows;
    int drafts[64], n_drafts;  /* MTP proposals of the last verify */
};

static float *alloc_f(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

static void mat_gen(Mat *m, int fmt, int O, int K, uint64_t seed, uint32_t tid) {
    m->fmt = fmt; m->O = O; m->K = K;
    size_t n = (size_t)O * K;
    if (fmt == FC_FMT_F32) {
        m->f32 = alloc_f(n);
#pragma omp parallel for schedule(static)
        for (size_t e = 0; e < n; ++e) m->f32[e] = fc_synth_f32(seed, tid, e);
        return;
    }
    int groups = K / 32;
    m->values = (int8_t *)malloc(n);
    m->scales = alloc_f((size_t)O * groups);
    m->scale_bits = (uint16_t *)malloc((size_t)O * groups * sizeof(uint16_t));
    /* One Philox block yields 8 int8 values or 32 nibbles (floyd_synth.h). */
    if (fmt == FC_FMT_Q8) {
        size_t blocks = (n + 7) / 8;
#pragma omp parallel for schedule(static)
        for (size_t b = 0; b < blocks; ++b) {
            uint32_t w[4];
            fc_synth_block(seed, tid, FC_STREAM_VALUES, b, w);
            for (int i = 0; i < 8 && b * 8 + i < n; ++i) {
                int v = (int)fc_synth_byte(w, 2 * i) + (int)fc_synth_byte(w, 2 * i + 1) - 255;
                m->values[b * 8 + i] = (int8_t)(v / 2);
            }
        }
    } else {
        size_t blocks = (n + 31) / 32;
#pragma omp parallel for schedule(static)
        for (size_t b = 0; b < blocks; ++b) {
            uint32_t w[4];
            fc_synth_block(seed, tid, FC_STREAM_VALUES, b, w);
            for (int i = 0; i < 32 && b * 32 + i < n; ++i) {
                int nib = (int)((w[i >> 3] >> (4 * (i & 7))) & 0xFu);
                m->values[b * 32 + i] = (int8_t)(fmt == FC_FMT_Q4 ? nib - 8 : nib);
            }
        }
    }
#pragma omp parallel for schedule(static)
    for (size_t g = 0; g < (size_t)O * groups; ++g) {
        if (fmt == FC_FMT_Q8) {
            m->scale_bits[g] = fc_synth_scale_q8(seed, tid, g);
            m->scales[g] = orc_fp16_to_f32(m->scale_bits[g]);
        } else if (fmt == FC_FMT_Q4) {
            m->scale_bits[g] = fc_synth_scale_q4(seed, tid, g);
            m->scales[g] = orc_fp16_to_f32(m->scale_bits[g]);
        } else {
            m->scale_bits[g] = fc_synth_scale_e8m0(seed, tid, g);
            m->scales[g] = orc_e8m0_to_f32((uint8_t)m->scale_bits[g]);
        }
    }
}

/* Deferred generation: the same values mat_gen would make, produced when
 * the matrix is first read or written. */
static void mat_defer(Mat *m, int fmt, int O, int K, uint64_t seed, uint32_t tid) {
    memset(m, 0, sizeof(*m));
    m->fmt = fmt; m->O = O; m->K = K; m->seed = seed; m->tid = tid; m->pending = 1;
}

static void mat_ensure(Mat *m) {
    if (m->pending) {
        m->pending = 0;
        mat_gen(m, m->fmt, m->O, m->K, m->seed, m->tid);
    }
}

static void mat_free(Mat *m) {
    free(m->values); free(m->scales); free(m->scale_bits); free(m->f32);
    memset(m, 0, sizeof(*m));
}

static float *norm_gen(int n, uint64_t seed, uint32_t tid) {
    float *w = alloc_f((size_t)n);
    for (int i = 0; i < n; ++i) w[i] = fc_synth_norm(seed, tid, (uint64_t)i);
    return w;
}

static void mat_apply(const Mat *m, const float *x, int S, float *y) {
    orc_gemv(m->fmt, m->values, m->scales, m->f32, m->O, m->K, x, S, y);
}

OrcModel *orc_model_create(const FcModelConfig *config, uint64_t seed) {
    if (!config || config->hidden_size % 32 || config->kv_lora_rank % 32) return NULL;
    OrcModel *m = (OrcModel *)calloc(1, sizeof(*m));
    const FcModelConfig *c = config;
    m->c = *config;
    m->seed = seed;
    int D = c->hidden_size, H = c->head_count, L = c->kv_lora_rank, R = c->qk_rope_dim;
    int qw = H * (c->qk_nope_dim + R);
    int df = c->dense_format, ef = c->expert_format;
    int hf = c->embed_f32 ? FC_FMT_F32 : df;  /* fp32 embedding / lm-head */
    mat_gen(&m->embed, hf, c->vocab_size, D, seed, fc_tensor_id(-1, FC_T_EMBED, 0));
    mat_gen(&m->lm_head, hf, c->vocab_size, D, seed, fc_tensor_id(-1, FC_T_LM_HEAD, 0));
    m->final_norm = norm_gen(D, seed, fc_tensor_id(-1, FC_T_FINAL_NORM, 0));
    m->layers = (Layer *)calloc((size_t)(c->layer_count + c->mtp_layers), sizeof(Layer));
    for (int l = 0; l < c->layer_count + c->mtp_layers; ++l) {
        Layer *y = &m->layers[l];
        if (l >= c->layer_count) { /* MTP drafter extras (DeepSeek-V3 MTP module) */
            y->enorm = norm_gen(D, seed, fc_tensor_id(l, FC_T_MTP_ENORM, 0));
            y->hnorm = norm_gen(D, seed, fc_tensor_id(l, FC_T_MTP_HNORM, 0));
            y->head_norm = norm_gen(D, seed, fc_tensor_id(l, FC_T_MTP_HEAD_NORM, 0));
            mat_gen(&y->eh_proj, df, D, 2 * D, seed, fc_tensor_id(l, FC_T_MTP_EH_PROJ, 0));
        }
        y->attn_norm = norm_gen(D, seed, fc_tensor_id(l, FC_T_ATTN_NORM, 0));
        y->ffn_norm = norm_gen(D, seed, fc_tensor_id(l, FC_T_FFN_NORM, 0));
        y->kv_a_norm = norm_gen(L, seed, fc_tensor_id(l, FC_T_KV_A_NORM, 0));
        if (c->q_lora_rank > 0) {
            y->q_a_norm = norm_gen(c->q_lora_rank, seed, fc_tensor_id(l, FC_T_Q_A_NORM, 0));
            mat_gen(&y->q_a, df, c->q_lora_rank, D, seed, fc_tensor_id(l, FC_T_Q_A, 0));
            mat_gen(&y->q_b, df, qw, c->q_lora_rank, seed, fc_tensor_id(l, FC_T_Q_B, 0));
        } else {
            mat_gen(&y->q_proj, df, qw, D, seed, fc_tensor_id(l, FC_T_Q_PROJ, 0));
        }
        mat_gen(&y->kv_a, df, L + R, D, seed, fc_tensor_id(l, FC_T_KV_A, 0));
        mat_gen(&y->kv_b, df, H * (c->qk_nope_dim + c->value_dim), L, seed,
                fc_tensor_id(l, FC_T_KV_B, 0));
        mat_gen(&y->o_proj, df, D, H * c->value_dim, seed, fc_tensor_id(l, FC_T_O_PROJ, 0));
        y->dense = l < c->first_dense_layer_count;
        if (y->dense) {
            int I = c->dense_intermediate_size;
            mat_gen(&y->d_gate, df, I, D, seed, fc_tensor_id(l, FC_T_DENSE_GATE, 0));
            mat_gen(&y->d_up, df, I, D, seed, fc_tensor_id(l, FC_T_DENSE_UP, 0));
            mat_gen(&y->d_down, df, D, I, seed, fc_tensor_id(l, FC_T_DENSE_DOWN, 0));
            continue;
        }
        int E = c->expert_count, I = c->moe_intermediate_size;
        mat_gen(&y->router, FC_FMT_F32, E, D, seed, fc_tensor_id(l, FC_T_ROUTER, 0));
        if (c->has_selection_bias) {
            y->bias = alloc_f((size_t)E);
            for (int e = 0; e < E; ++e)
                y->bias[e] = fc_synth_bias(seed, fc_tensor_id(l, FC_T_ROUTER_BIAS, 0), (uint64_t)e);
        }
        if (l < c->hash_layer_count) {
            y->hash = (int *)malloc((size_t)c->vocab_size * c->experts_per_token * sizeof(int));
            for (int t = 0; t < c->vocab_size; ++t)
                for (int k = 0; k < c->experts_per_token; ++k)
                    y->hash[(int64_t)t * c->experts_per_token + k] = fc_synth_hash_expert(
                        seed, fc_tensor_id(l, FC_T_HASH, 0), t, k, E, c->experts_per_token);
        }
        y->gate = (Mat *)calloc((size_t)E, sizeof(Mat));
        y->up = (Mat *)calloc((size_t)E, sizeof(Mat));
        y->down = (Mat *)calloc((size_t)E, sizeof(Mat));
        for (int e = 0; e < E; ++e) {
            mat_defer(&y->gate[e], ef, I, D, seed, fc_tensor_id(l, FC_T_EXP_GATE, e + 1));
            mat_defer(&y->up[e], ef, I, D, seed, fc_tensor_id(l, FC_T_EXP_UP, e + 1));
            mat_defer(&y->down[e], ef, D, I, seed, fc_tensor_id(l, FC_T_EXP_DOWN, e + 1));
        }
        if (c->shared_expert_count > 0) {
            int W = I * c->shared_expert_count;
            mat_gen(&y->sh_gate, df, W, D, seed, fc_tensor_id(l, FC_T_SH_GATE, 0));
            mat_gen(&y->sh_up, df, W, D, seed, fc_tensor_id(l, FC_T_SH_UP, 0));
            mat_gen(&y->sh_down, df, D, W, seed, fc_tensor_id(l, FC_T_SH_DOWN, 0));
        }
    }
    return m;
}

void orc_model_free(OrcModel *m) {
    if (!m) return;
    mat_free(&m->embed); mat_free(&m->lm_head); free(m->final_norm);
    for (int l = 0; l < m->c.layer_count + m->c.mtp_layers; ++l) {
        Layer *y = &m->layers[l];
        free(y->enorm); free(y->hnorm); free(y->head_norm); mat_free(&y->eh_proj);
        free(y->attn_norm); free(y->ffn_norm); free(y->kv_a_norm); free(y->q_a_norm);
        mat_free(&y->q_proj); mat_free(&y->q_a); mat_free(&y->q_b);
        mat_free(&y->kv_a); mat_free(&y->kv_b); mat_free(&y->o_proj);
        mat_free(&y->router); free(y->bias); free(y->hash);
        if (y->gate) {
            for (int e = 0; e < m->c.expert_count; ++e) {
                mat_free(&y->gate[e]); mat_free(&y->up[e]); mat_free(&y->down[e]);
            }
        }
        free(y->gate); free(y->up); free(y->down);
        mat_free(&y->sh_gate); mat_free(&y->sh_up); mat_free(&y->sh_down);
        mat_free(&y->d_gate); mat_free(&y->d_up); mat_free(&y->d_down);
    }
    free(m->layers);
    free(m);
}

/* Name lookup for the checkpoint tensor names the reference uses
 * (moonlight_metal.m:301-321, :450-466, :494-500, :580-612). */
static int lookup(OrcModel *m, const char *name, Mat **mat, float **vec, size_t *count) {
    int l = -1, e = -1;
    char rest[256];
    *mat = NULL; *vec = NULL; *count = 0;
    const FcModelConfig *c = &m->c;
    if (!strcmp(name, "model.embed_tokens.weight")) { *mat = &m->embed; return 1; }
    if (!strcmp(name, "lm_head.weight")) { *mat = &m->lm_head; return 1; }
    if (!strcmp(name, "model.norm.weight")) { *vec = m->final_norm; *count = (size_t)c->hidden_size; return 1; }
    if (sscanf(name, "model.layers.%d.%255s", &l, rest) != 2 || l < 0 || l >= c->layer_count) return 0;
    Layer *y = &m->layers[l];
    if (!strcmp(rest, "input_layernorm.weight")) { *vec = y->attn_norm; *count = (size_t)c->hidden_size; return 1; }
    if (!strcmp(rest, "post_attention_layernorm.weight")) { *vec = y->ffn_norm; *count = (size_t)c->hidden_size; return 1; }
    if (!strcmp(rest, "self_attn.kv_a_layernorm.weight")) { *vec = y->kv_a_norm; *count = (size_t)c->kv_lora_rank; return 1; }
    if (!strcmp(rest, "self_attn.q_a_layernorm.weight") && y->q_a_norm) { *vec = y->q_a_norm; *count = (size_t)c->q_lora_rank; return 1; }
    if (!strcmp(rest, "self_attn.q_proj.weight") && !c->q_lora_rank) { *mat = &y->q_proj; return 1; }
    if (!strcmp(rest, "self_attn.q_a_proj.weight") && c->q_lora_rank) { *mat = &y->q_a; return 1; }
    if (!strcmp(rest, "self_attn.q_b_proj.weight") && c->q_lora_rank) { *mat = &y->q_b; return 1; }
    if (!strcmp(rest, "self_attn.kv_a_proj_with_mqa.weight")) { *mat = &y->kv_a; return 1; }
    if (!strcmp(rest, "self_attn.kv_b_proj.weight")) { *mat = &y->kv_b; return 1; }
    if (!strcmp(rest, "self_attn.o_proj.weight")) { *mat = &y->o_proj; return 1; }
    if (y->dense) {
        if (!strcmp(rest, "mlp.gate_proj.weight")) { *mat = &y->d_gate; return 1; }
        if (!strcmp(rest, "mlp.up_proj.weight")) { *mat = &y->d_up; return 1; }
        if (!strcmp(rest, "mlp.down_proj.weight")) { *mat = &y->d_down; return 1; }
        return 0;
    }
    if (!strcmp(rest, "mlp.gate.weight")) { *mat = &y->router; return 1; }
    if (!strcmp(rest, "mlp.gate.e_score_correction_bias") && y->bias) { *vec = y->bias; *count = (size_t)c->expert_count; return 1; }
    if (!strcmp(rest, "mlp.shared_experts.gate_proj.weight")) { *mat = &y->sh_gate; return 1; }
    if (!strcmp(rest, "mlp.shared_experts.up_proj.weight")) { *mat = &y->sh_up; return 1; }
    if (!strcmp(rest, "mlp.shared_experts.down_proj.weight")) { *mat = &y->sh_down; return 1; }
    char proj[64];
    if (sscanf(rest, "mlp.experts.%d.%63s", &e, proj) == 2 && e >= 0 && e < c->expert_count) {
        if (!strcmp(proj, "gate_proj.weight")) *mat = &y->gate[e];
        if (!strcmp(proj, "up_proj.weight")) *mat = &y->up[e];
        if (!strcmp(proj, "down_proj.weight")) *mat = &y->down[e];
        if (*mat) { mat_ensure(*mat); return 1; }
    }
    return 0;
}

int orc_model_set_f32(OrcModel *m, const char *name, const float *data, size_t count) {
    Mat *mat; float *vec; size_t n;
    if (!m || !lookup(m, name, &mat, &vec, &n)) return 0;
    if (vec) {
        if (count != n) return 0;
        memcpy(vec, data, n * sizeof(float));
        return 1;
    }
    if (count != (size_t)mat->O * mat->K) return 0;
    int O = mat->O, K = mat->K;
    mat_free(mat);
    mat->fmt = FC_FMT_F32; mat->O = O; mat->K = K;
    mat->f32 = alloc_f(count);
    memcpy(mat->f32, data, count * sizeof(float));
    return 1;
}

size_t orc_model_get_tensor(const OrcModel *m, const char *name, int scales_part,
                            void *data, size_t bytes) {
    Mat *mat; float *vec; size_t n;
    if (!m || !lookup((OrcModel *)m, name, &mat, &vec, &n)) return 0;
    if (vec) {
        if (bytes < n * 4) return 0;
        memcpy(data, vec, n * 4);
        return n * 4;
    }
    size_t elems = (size_t)mat->O * mat->K;
    if (mat->fmt == FC_FMT_F32) {
        if (bytes < elems * 4) return 0;
        memcpy(data, mat->f32, elems * 4);
        return elems * 4;
    }
    size_t groups = (size_t)mat->O * (mat->K / 32);
    if (scales_part) {
        if (mat->fmt == FC_FMT_MXFP4) {
            if (bytes < groups) return 0;
            for (size_t g = 0; g < groups; ++g) ((uint8_t *)data)[g] = (uint8_t)mat->scale_bits[g];
            return groups;
        }
        if (bytes < groups * 2) return 0;
        memcpy(data, mat->scale_bits, groups * 2);
        return groups * 2;
    }
    if (mat->fmt == FC_FMT_Q8) {
        if (bytes < elems) return 0;
        memcpy(data, mat->values, elems);
        return elems;
    }
    /* packed nibbles, even element low (moonlight_kernels.metal:123-127) */
    if (bytes < elems / 2) return 0;
    uint8_t *out = (uint8_t *)data;
    for (size_t i = 0; i < elems / 2; ++i) {
        int lo = mat->values[2 * i], hi = mat->values[2 * i + 1];
        if (mat->fmt == FC_FMT_Q4) { lo += 8; hi += 8; }
        out[i] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
    }
    return elems / 2;
}

OrcSession *orc_session_create(OrcModel *m, int context_size, int kv_fp16) {
    if (!m || context_size <= 0) return NULL;
    OrcSession *s = (OrcSession *)calloc(1, sizeof(*s));
    s->m = m; s->ctx = context_size; s->kv_fp16 = kv_fp16;
    size_t rows = (size_t)(m->c.layer_count + m->c.mtp_layers) * context_size;
    s->latent = alloc_f(rows * m->c.kv_lora_rank);
    s->rope = alloc_f(rows * m->c.qk_rope_dim);
    s->hist = alloc_f((size_t)context_size * m->c.hidden_size);
    s->tok = (int *)calloc((size_t)context_size, sizeof(int));
    if (!s->latent || !s->rope) { orc_session_free(s); return NULL; }
    return s;
}

void orc_session_free(OrcSession *s) {
    if (!s) return;
    free(s->latent); free(s->rope); free(s->last_x); free(s->hist); free(s->tok); free(s);
}

int orc_session_position(const OrcSession *s) { return s ? s->position : 0; }

void orc_session_set_position(OrcSession *s, int position) {
    if (s && position >= 0 && position <= s->position) s->position = position;
}

int orc_session_seed_context(OrcSession *s, int positions, uint64_t seed) {
    const FcModelConfig *c = &s->m->c;
    if (positions < 0 || positions > s->ctx) return 0;
    int L = c->kv_lora_rank, R = c->qk_rope_dim;
    for (int l = 0; l < c->layer_count; ++l) {
        uint32_t tl = fc_tensor_id(l, FC_T_KV_LATENT, 0), tr = fc_tensor_id(l, FC_T_KV_ROPE, 0);
        float *lat = s->latent + (size_t)l * s->ctx * L;
        float *rop = s->rope + (size_t)l * s->ctx * R;
        for (size_t e = 0; e < (size_t)positions * L; ++e) lat[e] = fc_synth_kv(seed, tl, e);
        for (size_t e = 0; e < (size_t)positions * R; ++e) rop[e] = fc_synth_kv(seed, tr, e);
    }
    s->position = positions;
    return 1;
}

/* Synthetic latent KV for positions [start, end) only (the values depend on
 * the position, as in orc_session_seed_context); the position becomes end
 * when that is further.  Lets a test build a context whose leading part is
 * shared with other sequences and whose tail is its own. */
int orc_session_seed_range(OrcSession *s, int start, int end, uint64_t seed) {
    const FcModelConfig *c = &s->m->c;
    if (start < 0 || end < start || end > s->ctx) return 0;
    int L = c->kv_lora_rank, R = c->qk_rope_dim;
    for (int l = 0; l < c->layer_count; ++l) {
        uint32_t tl = fc_tensor_id(l, FC_T_KV_LATENT, 0), tr = fc_tensor_id(l, FC_T_KV_ROPE, 0);
        float *lat = s->latent + (size_t)l * s->ctx * L;
        float *rop = s->rope + (size_t)l * s->ctx * R;
        for (size_t e = (size_t)start * L; e < (size_t)end * L; ++e) lat[e] = fc_synth_kv(seed, tl, e);
        for (size_t e = (size_t)start * R; e < (size_t)end * R; ++e) rop[e] = fc_synth_kv(seed, tr, e);
    }
    if (end > s->position) s->position = end;
    return 1;
}

static float round_kv(const OrcSession *s, float v) {
    return s->kv_fp16 ? orc_fp16_to_f32(orc_f32_to_fp16(v)) : v;
}

static float silu(float x) { return x / (1.0f + expf(-x)); }

/* moe_f32_add_expert (moe_exec.h:47-63) on a quantized expert, accumulating
 * coefficient * down(swiglu(gate x, up x)) into out. */
static void add_expert(const Mat *gate, const Mat *up, const Mat *down, const float *x,
                       float coefficient, float limit, float *out, float *tmp) {
    mat_ensure((Mat *)gate); mat_ensure((Mat *)up); mat_ensure((Mat *)down);
    int I = gate->O, D = down->O;
    float *g = tmp, *u = tmp + I, *h = tmp + 2 * I, *p = tmp + 3 * I;
    mat_apply(gate, x, 1, g);
    mat_apply(up, x, 1, u);
    for (int i = 0; i < I; ++i) {
        float gv = g[i], uv = u[i];
        if (limit > 0.0f) {
            if (gv > limit) gv = limit;
            if (uv > limit) uv = limit;
            if (uv < -limit) uv = -limit;
        }
        h[i] = silu(gv) * uv;
    }
    mat_apply(down, h, 1, p);
    for (int d = 0; d < D; ++d) out[d] += coefficient * p[d];
}

/* moe_f32_forward for one token (moe_exec.h:65-114): router matvec, select or
 * fixed routes, finalize, routed experts accumulated in ascending expert id,
 * then the shared expert with coefficient 1.  y must start at zero. */
static int moe_row(const FcModelConfig *c, const Mat *router, const float *bias,
                   const int *fixed, const Mat *gate, const Mat *up, const Mat *down,
                   const Mat *sh_gate, const Mat *sh_up, const Mat *sh_down, const float *xr,
                   float *y, int *routes, float *lg, float *tmp) {
    int E = c->expert_count, K = c->experts_per_token;
    int idx[64], order[64];
    float wt[64];
    mat_apply(router, xr, 1, lg);
    if (orc_route(lg, bias, E, K, c->score_fn, c->normalize_topk, c->routed_scale, fixed, idx,
                  wt) != K)
        return 0;
    if (routes)
        for (int k = 0; k < K; ++k) routes[k] = idx[k];
    for (int k = 0; k < K; ++k) order[k] = k;
    for (int a = 1; a < K; ++a) { /* insertion sort, moe_exec.h:97-105 */
        int v = order[a], b = a - 1;
        while (b >= 0 && idx[order[b]] > idx[v]) { order[b + 1] = order[b]; b--; }
        order[b + 1] = v;
    }
    for (int k = 0; k < K; ++k) {
        int e = idx[order[k]];
        add_expert(&gate[e], &up[e], &down[e], xr, wt[order[k]], c->swiglu_limit, y, tmp);
    }
    if (sh_gate) add_expert(sh_gate, sh_up, sh_down, xr, 1.0f, c->swiglu_limit, y, tmp);
    return 1;
}

static Mat f32_mat(int O, int K, const float *p) {
    Mat m;
    memset(&m, 0, sizeof(m));
    m.fmt = FC_FMT_F32; m.O = O; m.K = K; m.f32 = (float *)p;
    return m;
}

int orc_moe_forward_f32(int hidden, int intermediate, int n_experts, int top_k, int score_fn,
                        int normalize, float routed_scale, float swiglu_limit,
                        const float *router, const float *bias, const float *expert_weights,
                        int n_shared, const float *shared_weights, const float *input,
                        int n_tokens, float *output) {
    if (n_experts > 1024 || top_k > 64 || n_shared > 1) return 0;
    FcModelConfig c;
    memset(&c, 0, sizeof(c));
    c.expert_count = n_experts; c.experts_per_token = top_k; c.score_fn = score_fn;
    c.normalize_topk = normalize; c.routed_scale = routed_scale; c.swiglu_limit = swiglu_limit;
    size_t block = (size_t)hidden * intermediate;
    Mat r = f32_mat(n_experts, hidden, router);
    Mat *g = (Mat *)calloc((size_t)n_experts, sizeof(Mat));
    Mat *u = (Mat *)calloc((size_t)n_experts, sizeof(Mat));
    Mat *d = (Mat *)calloc((size_t)n_experts, sizeof(Mat));
    for (int e = 0; e < n_experts; ++e) { /* w1 = gate, w2 = down, w3 = up */
        g[e] = f32_mat(intermediate, hidden, expert_weights + (3 * (size_t)e) * block);
        d[e] = f32_mat(hidden, intermediate, expert_weights + (3 * (size_t)e + 1) * block);
        u[e] = f32_mat(intermediate, hidden, expert_weights + (3 * (size_t)e + 2) * block);
    }
    Mat sg = f32_mat(intermediate, hidden, shared_weights);
    Mat sd = f32_mat(hidden, intermediate, n_shared ? shared_weights + block : NULL);
    Mat su = f32_mat(intermediate, hidden, n_shared ? shared_weights + 2 * block : NULL);
    float *lg = alloc_f((size_t)n_experts);
    float *tmp = alloc_f((size_t)4 * intermediate + hidden);
    int ok = 1;
    for (int t = 0; t < n_tokens && ok; ++t) {
        float *y = output + (size_t)t * hidden;
        for (int i = 0; i < hidden; ++i) y[i] = 0.0f;
        ok = moe_row(&c, &r, bias, NULL, g, u, d, n_shared ? &sg : NULL, &su, &sd,
                     input + (size_t)t * hidden, y, NULL, lg, tmp);
    }
    free(g); free(u); free(d); free(lg); free(tmp);
    return ok;
}

/* Wall time spent in the attention blocks and in the FFN / MoE blocks of
 * run_layers since the last orc_part_times call (bench.py's CPU baseline
 * splits a layer with it). */
static double g_t_attn, g_t_ffn;

void orc_part_times(double *attn_s, double *ffn_s) {
    if (attn_s) *attn_s = g_t_attn;
    if (ffn_s) *ffn_s = g_t_ffn;
    g_t_attn = g_t_ffn = 0.0;
}

/* Layers [l0, l1) over the residual rows x at positions pos .. pos+rows-1
 * (the MTP layer is layer_count; its cache follows the target's). */
static int run_layers(OrcSession *s, float *x, int rows, int pos, const int *ids, int l0, int l1,
                      float *layer_out, int *routes) {
    OrcModel *m = s->m;
    const FcModelConfig *c = &m->c;
    int D = c->hidden_size, H = c->head_count, L = c->kv_lora_rank, R = c->qk_rope_dim;
    int NP = c->qk_nope_dim, VD = c->value_dim, QW = NP + R;

    int maxI = c->moe_intermediate_size * (c->shared_expert_count > 1 ? c->shared_expert_count : 1);
    if (c->dense_intermediate_size > maxI) maxI = c->dense_intermediate_size;
    if (c->moe_intermediate_size > maxI) maxI = c->moe_intermediate_size;
    int maxO = D;
    if (H * QW > maxO) maxO = H * QW;
    if (H * (NP + VD) > maxO) maxO = H * (NP + VD);
    if (c->q_lora_rank > maxO) maxO = c->q_lora_rank;
    float *xn = alloc_f((size_t)rows * D);
    float *q = alloc_f((size_t)rows * H * QW);
    float *qa = alloc_f((size_t)rows * (c->q_lora_rank > 0 ? c->q_lora_rank : 1));
    float *ckv = alloc_f((size_t)rows * (L + R));
    float *attn = alloc_f((size_t)rows * H * VD);
    float *tmp = alloc_f((size_t)4 * maxI + (size_t)4 * maxO + (size_t)s->ctx + (size_t)8 * L + D);
    float *y = alloc_f((size_t)D);
    float *ao = alloc_f((size_t)rows * D);
    float scale = 1.0f / sqrtf((float)(NP + R));

    for (int l = l0; l < l1; ++l) {
        Layer *ly = &m->layers[l];
        float *lat = s->latent + (size_t)l * s->ctx * L;
        float *rop = s->rope + (size_t)l * s->ctx * R;
        /* attention block, moonlight_metal.m:287-440 */
        double t_a0 = omp_get_wtime();
        orc_rmsnorm(x, ly->attn_norm, rows, D, c->rms_norm_epsilon, xn);
        if (c->q_lora_rank > 0) {
            mat_apply(&ly->q_a, xn, rows, qa);
            orc_rmsnorm(qa, ly->q_a_norm, rows, c->q_lora_rank, c->rms_norm_epsilon, qa);
            mat_apply(&ly->q_b, qa, rows, q);
        } else {
            mat_apply(&ly->q_proj, xn, rows, q);
        }
        mat_apply(&ly->kv_a, xn, rows, ckv);
        for (int r = 0; r < rows; ++r) {
            /* cache_append: RMSNorm latent, RoPE rope part (:132-170) */
            float *src = ckv + (int64_t)r * (L + R);
            float *dl = lat + (int64_t)(pos + r) * L;
            orc_rmsnorm(src, ly->kv_a_norm, 1, L, c->rms_norm_epsilon, dl);
            orc_rope(src + L, rop + (int64_t)(pos + r) * R, R, pos + r, c->rope_theta);
            for (int i = 0; i < L; ++i) dl[i] = round_kv(s, dl[i]);
            for (int i = 0; i < R; ++i) rop[(int64_t)(pos + r) * R + i] = round_kv(s, rop[(int64_t)(pos + r) * R + i]);
            /* rope_query (:172-200) */
            for (int h = 0; h < H; ++h) {
                float *qh = q + ((int64_t)r * H + h) * QW;
                orc_rope(qh + NP, qh + NP, R, pos + r, c->rope_theta);
            }
        }
        for (int r = 0; r < rows; ++r) {
            int keys = pos + r + 1;
#pragma omp parallel for schedule(dynamic)
            for (int h = 0; h < H; ++h) {
                const float *qh = q + ((int64_t)r * H + h) * QW;
                float *work = alloc_f((size_t)3 * L + 2 * R + (size_t)keys);
                float *qabs = work, *qr = work + L, *ctxl = work + L + R, *sc = work + 2 * L + R;
                /* absorb_query (:218-245): q_abs = q_nope . W_UK[h] */
                for (int i = 0; i < L; ++i) qabs[i] = 0.0f;
                const Mat *kb = &ly->kv_b;
                for (int n = 0; n < NP; ++n) {
                    int row = h * (NP + VD) + n;
                    for (int i = 0; i < L; ++i) {
                        float w = kb->fmt == FC_FMT_F32 ? kb->f32[(int64_t)row * L + i]
                            : value_of(kb->fmt, kb->values[(int64_t)row * L + i]) *
                              kb->scales[(int64_t)row * (L / 32) + i / 32];
                        qabs[i] += qh[n] * w;
                    }
                }
                for (int i = 0; i < L; ++i) qabs[i] = round_kv(s, qabs[i]);
                for (int i = 0; i < R; ++i) qr[i] = round_kv(s, qh[NP + i]);
                /* scores + softmax + latent context (:247-343) */
                float mx = -INFINITY;
                for (int key = 0; key < keys; ++key) {
                    const float *cl = lat + (int64_t)key * L, *cr = rop + (int64_t)key * R;
                    float a = 0.0f;
                    for (int i = 0; i < L; ++i) a += qabs[i] * cl[i];
                    for (int i = 0; i < R; ++i) a += qr[i] * cr[i];
                    sc[key] = a * scale;
                    if (sc[key] > mx) mx = sc[key];
                }
                float den = 0.0f;
                for (int key = 0; key < keys; ++key) den += expf(sc[key] - mx);
                for (int i = 0; i < L; ++i) ctxl[i] = 0.0f;
                for (int key = 0; key < keys; ++key) {
                    float p = expf(sc[key] - mx) / den;
                    const float *cl = lat + (int64_t)key * L;
                    for (int i = 0; i < L; ++i) ctxl[i] += p * cl[i];
                }
                /* decode_value (:345-375): o = ctx_L . W_UV[h] */
                for (int v = 0; v < VD; ++v) {
                    int row = h * (NP + VD) + NP + v;
                    float a = 0.0f;
                    for (int i = 0; i < L; ++i) {
                        float w = kb->fmt == FC_FMT_F32 ? kb->f32[(int64_t)row * L + i]
                            : value_of(kb->fmt, kb->values[(int64_t)row * L + i]) *
                              kb->scales[(int64_t)row * (L / 32) + i / 32];
                        a += ctxl[i] * w;
                    }
                    attn[((int64_t)r * H + h) * VD + v] = a;
                }
                free(work);
            }
        }
        mat_apply(&ly->o_proj, attn, rows, ao);
        for (size_t i = 0; i < (size_t)rows * D; ++i) x[i] += ao[i];

        /* FFN block */
        double t_f0 = omp_get_wtime();
        g_t_attn += t_f0 - t_a0;
        orc_rmsnorm(x, ly->ffn_norm, rows, D, c->rms_norm_epsilon, xn);
        for (int r = 0; r < rows; ++r) {
            const float *xr = xn + (int64_t)r * D;
            for (int d = 0; d < D; ++d) y[d] = 0.0f;
            if (ly->dense) { /* encode_dense_residual_buffer, moonlight_metal.m:442-483 */
                add_expert(&ly->d_gate, &ly->d_up, &ly->d_down, xr, 1.0f, 0.0f, y, tmp);
                if (routes)
                    for (int k = 0; k < c->experts_per_token; ++k)
                        routes[((int64_t)l * rows + r) * c->experts_per_token + k] = -1;
            } else {
                const int *fixed = ly->hash ? ly->hash + (int64_t)ids[r] * c->experts_per_token : NULL;
                int *rt = routes ? routes + ((int64_t)l * rows + r) * c->experts_per_token : NULL;
                if (!moe_row(c, &ly->router, ly->bias, fixed, ly->gate, ly->up, ly->down,
                             c->shared_expert_count > 0 ? &ly->sh_gate : NULL, &ly->sh_up,
                             &ly->sh_down, xr, y, rt, tmp + 4 * maxI, tmp)) goto fail;
            }
            for (int d = 0; d < D; ++d) x[(int64_t)r * D + d] += y[d];
        }
        g_t_ffn += omp_get_wtime() - t_f0;
        if (layer_out) memcpy(layer_out + (size_t)l * rows * D, x, (size_t)rows * D * sizeof(float));
    }
    free(xn); free(q); free(qa); free(ckv); free(attn); free(tmp); free(y); free(ao);
    return 1;
fail:
    free(xn); free(q); free(qa); free(ckv); free(attn); free(tmp); free(y); free(ao);
    return 0;
}

static void embed_rows(const OrcModel *m, const int *ids, int rows, float *x) {
    const FcModelConfig *c = &m->c;
    int D = c->hidden_size;
    /* embedding: dequantized row (moonlight_kernels.metal:10-21) */
    for (int r = 0; r < rows; ++r) {
        const Mat *e = &m->embed;
        for (int k = 0; k < D; ++k) {
            float v = e->fmt == FC_FMT_F32 ? e->f32[(int64_t)ids[r] * D + k]
                : value_of(e->fmt, e->values[(int64_t)ids[r] * D + k]) *
                  e->scales[(int64_t)ids[r] * (D / 32) + k / 32];
            x[(int64_t)r * D + k] = v;
        }
    }

}

int orc_session_forward(OrcSession *s, const int *ids, int rows, float *logits,
                        float *layer_out, int *routes) {
    OrcModel *m = s->m;
    const FcModelConfig *c = &m->c;
    int D = c->hidden_size, V = c->vocab_size;
    int pos = s->position;
    if (rows <= 0 || pos + rows > s->ctx) return 0;
    for (int r = 0; r < rows; ++r) if (ids[r] < 0 || ids[r] >= V) return 0;
    float *x = alloc_f((size_t)rows * D);
    float *xn = alloc_f((size_t)rows * D);
    embed_rows(m, ids, rows, x);
    if (!run_layers(s, x, rows, pos, ids, 0, c->layer_count, layer_out, routes)) {
        free(x); free(xn);
        return 0;
    }
    free(s->last_x);
    s->last_x = alloc_f((size_t)rows * D);
    memcpy(s->last_x, x, (size_t)rows * D * sizeof(float));
    s->last_rows = rows;
    memcpy(s->hist + (size_t)pos * D, x, (size_t)rows * D * sizeof(float));
    memcpy(s->tok + pos, ids, (size_t)rows * sizeof(int));
    if (logits) {
        orc_rmsnorm(x, m->final_norm, rows, D, c->rms_norm_epsilon, xn);
        mat_apply(&m->lm_head, xn, rows, logits);
    }
    s->position = pos + rows;
    free(x); free(xn);
    return 1;
}

/* The MTP drafter (DeepSeek-V3 MTP module; the role of
 * deepseek_v4_forward_dspark_propose, deepseek_v4_forward.h:1873-1949):
 * step i at position start + i takes token t_i (t_0 = the target's next
 * token, then the previous proposal) and hidden h (h_0 = the target's last
 * committed row): x = eh_proj([enorm(embed(t_i)) | hnorm(h)]), the MTP
 * layer, h = x, proposal = argmax(lm_head(shared_head.norm(x))). */
static int mtp_drafts(OrcSession *s, const float *h0, int start, int first_token, int k, int *out,
                      float *conf) {
    OrcModel *m = s->m;
    const FcModelConfig *c = &m->c;
    int D = c->hidden_size, V = c->vocab_size, lm = c->layer_count;
    const Layer *y = &m->layers[lm];
    float *h = alloc_f((size_t)D), *e = alloc_f((size_t)D), *cat = alloc_f((size_t)2 * D);
    float *x = alloc_f((size_t)D), *xn = alloc_f((size_t)D), *lg = alloc_f((size_t)V);
    memcpy(h, h0, (size_t)D * sizeof(float));
    int token = first_token, ok = 1;
    for (int i = 0; i < k && ok; ++i) {
        if (start + i >= s->ctx) { ok = 0; break; }
        embed_rows(m, &token, 1, e);
        orc_rmsnorm(e, y->enorm, 1, D, c->rms_norm_epsilon, cat);
        orc_rmsnorm(h, y->hnorm, 1, D, c->rms_norm_epsilon, cat + D);
        mat_apply(&y->eh_proj, cat, 1, x);
        ok = run_layers(s, x, 1, start + i, &token, lm, lm + 1, NULL, NULL);
        memcpy(h, x, (size_t)D * sizeof(float));
        orc_rmsnorm(x, y->head_norm, 1, D, c->rms_norm_epsilon, xn);
        mat_apply(&m->lm_head, xn, 1, lg);
        token = orc_argmax(lg, V);
        out[i] = token;
        if (conf) conf[i] = lg[token];
    }
    free(h); free(e); free(cat); free(x); free(xn); free(lg);
    return ok;
}

int orc_session_drafts(const OrcSession *s, int *out, int capacity) {
    if (!s || !out) return 0;
    int n = s->n_drafts < capacity ? s->n_drafts : capacity;
    memcpy(out, s->drafts, (size_t)n * sizeof(int));
    return n;
}

int orc_session_copy_kv(const OrcSession *s, int layer, float *latent, float *rope,
                        int capacity) {
    const FcModelConfig *c = &s->m->c;
    if (layer < 0 || layer >= c->layer_count || capacity < s->position) return 0;
    int L = c->kv_lora_rank, R = c->qk_rope_dim;
    if (latent) memcpy(latent, s->latent + (size_t)layer * s->ctx * L, (size_t)s->position * L * 4);
    if (rope) memcpy(rope, s->rope + (size_t)layer * s->ctx * R, (size_t)s->position * R * 4);
    return 1;
}

int orc_session_verify(OrcSession *s, const int *ids, int k, const FcAcceptConfig *accept,
                       int *emitted, int *n_emitted, int *next_token, float *row_logits,
                       int *row_tops) {
    int V = s->m->c.vocab_size, rows = k + 1, start = s->position;
    float *logits = row_logits ? row_logits : alloc_f((size_t)rows * V);
    int tops[64];
    if (k < 0 || rows > 64) return 0;
    if (!orc_session_forward(s, ids, rows, logits, NULL, NULL)) {
        if (!row_logits) free(logits);
        return 0;
    }
    for (int r = 0; r < rows; ++r) tops[r] = orc_argmax(logits + (int64_t)r * V, V);
    if (row_tops) memcpy(row_tops, tops, (size_t)rows * sizeof(int));
    int commit, next;
    if (accept && accept->mode == FC_ACCEPT_SAMPLE) {
        commit = orc_accept_sample(logits, V, ids, k, accept->temperature, accept->seed,
                                   accept->counter, &next);
    } else {
        commit = orc_accept_greedy(tops, ids, k);
        next = tops[commit - 1];
    }
    for (int i = 0; i < commit; ++i) emitted[i] = ids[i];
    *n_emitted = commit;
    *next_token = next;
    s->position = start + commit; /* rollback: the MLA cache is append-only */
    s->n_drafts = 0;
    if (s->m->c.mtp_layers > 0 && k > 0) {
        int D = s->m->c.hidden_size;
        if (mtp_drafts(s, s->last_x + (size_t)(commit - 1) * D, start + commit, next < 0 ? 0 : next, k,
                       s->drafts, NULL))
            s->n_drafts = k;
    }
    if (!row_logits) free(logits);
    return 1;
}

/* The drafter layer over positions p0 + 1 .. p0 + r of the session's own
 * history: row i takes the final hidden row of position p0 + i and the
 * token at p0 + 1 + i (the pairing of mtp_drafts) and writes the drafter's
 * latent KV at p0 + 1 + i.  The counterpart of the reference runtime's
 * DSpark prefill / append (deepseek_v4_runtime.h:130-198) for the MTP
 * stand-in. */
int orc_dspark_rows(OrcSession *s, int p0, int r) {
    OrcModel *m = s->m;
    const FcModelConfig *c = &m->c;
    int D = c->hidden_size, lm = c->layer_count;
    if (c->mtp_layers != 1 || p0 < 0 || p0 + r >= s->ctx) return 0;
    const Layer *y = &m->layers[lm];
    float *e = alloc_f((size_t)D), *cat = alloc_f((size_t)2 * D), *x = alloc_f((size_t)D);
    int ok = 1;
    for (int i = 0; i < r && ok; ++i) {
        int q = p0 + 1 + i, token = s->tok[q];
        embed_rows(m, &token, 1, e);
        orc_rmsnorm(e, y->enorm, 1, D, c->rms_norm_epsilon, cat);
        orc_rmsnorm(s->hist + (size_t)(q - 1) * D, y->hnorm, 1, D, c->rms_norm_epsilon, cat + D);
        mat_apply(&y->eh_proj, cat, 1, x);
        ok = run_layers(s, x, 1, q, &token, lm, lm + 1, NULL, NULL);
    }
    free(e); free(cat); free(x);
    return ok;
}

/* Five greedy drafter steps from the hidden row of position p and the next
 * token: out[0..4] proposals, conf[0..4] their top-1 logits. */
int orc_dspark_propose(OrcSession *s, int p, int input_id, int *out, float *conf) {
    if (p < 0 || p + 5 >= s->ctx) return 0;
    return mtp_drafts(s, s->hist + (size_t)p * s->m->c.hidden_size, p + 1, input_id, 5, out, conf);
}

