/*
 * test_moonlight_cuda.c - floyd's Moonlight Metal test programs
 * (tests/test_moonlight_metal_primitives.c, _mla.c, _moe.c, _runtime.c)
 * rerun against the CUDA backend through the moonlight_* shim
 * (floyd_b200/shim/moonlight_cuda.c), in plain C, linked against
 * libfloyd_cuda.so.
 *
 *   test_moonlight_cuda MODEL_DIR ORACLE.safetensors
 *
 * MODEL_DIR is a Moonlight container (config.json + U8 / .qs safetensors);
 * the oracle file holds the expected intermediates (tests/golden/
 * make_container.py writes both).  Each section makes the same calls and
 * checks the same quantities as the Metal test it is named after.  Where
 * this backend's numerics differ by design the bound is widened and the
 * reason stated next to it:
 *   - row scales are stored as fp16 group scales (relative error <= 2^-12
 *     per weight row);
 *   - the latent KV cache is fp16 (relative error <= 2^-11 per element);
 *   - activations enter the tensor cores as hi + lo fp16 halves (22 bits).
 * Every bound is printed with the measured error.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "moonlight_api.h"
#include "st_lite.h"

static int failures = 0;

#define CHECK(cond)                                                                 \
    do {                                                                            \
        if (!(cond)) {                                                              \
            fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #cond); \
            failures++;                                                             \
            return 1;                                                               \
        }                                                                           \
    } while (0)

/* measured error, the Metal test's bound, this backend's bound */
#define BOUND(label, err, metal, ours)                                                          \
    do {                                                                                        \
        printf("  %-28s %.3g (metal bound %.1g, bound here %.1g)\n", label, (double)(err),      \
               (double)(metal), (double)(ours));                                                \
        CHECK((err) < (ours));                                                                  \
    } while (0)

static float max_abs(const float *a, const float *b, int64_t n) {
    float r = 0;
    for (int64_t i = 0; i < n; ++i) {
        float d = fabsf(a[i] - b[i]);
        if (d > r) r = d;
    }
    return r;
}

static int argmax(const float *v, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (v[i] > v[best]) best = i;
    return best;
}

static const char *g_model;
static StFile g_oracle;

static float *need_f32(const char *name, int64_t expect) {
    int64_t n = 0;
    float *v = st_read_f32(&g_oracle, name, &n);
    if (!v || (expect >= 0 && n != expect)) {
        fprintf(stderr, "oracle tensor %s missing or of size %lld\n", name, (long long)n);
        free(v);
        return NULL;
    }
    return v;
}

/* tests/test_moonlight_metal_primitives.c */
static int primitives(void) {
    MoonlightModel *model = NULL;
    MoonlightSession *session = NULL;
    MoonlightOptions options = {.context_size = 64, .max_batch = 32};
    char error[512] = {0};
    int64_t n = 0;
    int *ids = st_read_ids(&g_oracle, "input_ids", &n);
    CHECK(ids && n > 0 && n <= 32);
    CHECK(moonlight_model_open(&model, g_model, error, sizeof error) == 1);
    MoonlightModelInfo info = moonlight_model_info(model);
    const int D = info.hidden_size, V = info.vocab_size;
    const int Q = info.head_count * (info.qk_nope_dim + info.qk_rope_dim);
    float *embed = need_f32("embed", n * D), *final_in = need_f32("final_input", n * D);
    float *final_norm = need_f32("final_norm", n * D), *in_norm = need_f32("layer.0.input_norm", n * D);
    float *q = need_f32("layer.0.q", n * Q), *logits = need_f32("logits", n * V);
    CHECK(embed && final_in && final_norm && in_norm && q && logits);
    float *a_embed = calloc((size_t)n * D, 4), *a_norm = calloc((size_t)n * D, 4);
    float *a_q = calloc((size_t)n * Q, 4), *a_logits = calloc((size_t)n * V, 4);
    CHECK(moonlight_session_create(&session, model, &options, error, sizeof error) == 1);
    CHECK(moonlight_test_embed(session, ids, (int)n, a_embed) == 1);
    CHECK(moonlight_test_rmsnorm(session, final_in, "model.norm.weight", (int)n, D, a_norm) == 1);
    CHECK(moonlight_test_matmul(session, "model.layers.0.self_attn.q_proj.weight", in_norm, (int)n, D, Q,
                                a_q) == 1);
    CHECK(moonlight_test_matmul(session, "lm_head.weight", final_norm, (int)n, D, V, a_logits) == 1);
    printf("primitives:\n");
    BOUND("embed", max_abs(a_embed, embed, n * D), 3e-6, 3e-6);
    BOUND("final norm", max_abs(a_norm, final_norm, n * D), 3e-5, 3e-5);
    /* q8 rows: fp16 row scale (<= 2^-12 relative) on |q| up to about 8 */
    BOUND("q_proj (q8)", max_abs(a_q, q, n * Q), 3e-5, 3e-3);
    /* fp32 lm-head on hi + lo fp16 activations */
    BOUND("lm_head (f32) logits", max_abs(a_logits, logits, n * V), 3e-5, 3e-5);
    MoonlightStats st = moonlight_session_stats(session);
    CHECK(st.command_buffers == 4);
    CHECK(st.cpu_fallbacks == 0);
    moonlight_session_destroy(session);
    moonlight_model_close(model);
    free(ids); free(embed); free(final_in); free(final_norm); free(in_norm); free(q); free(logits);
    free(a_embed); free(a_norm); free(a_q); free(a_logits);
    return 0;
}

static void rope_reference(const float *in, float *out, int rows, int width, float theta) {
    int half = width / 2;
    for (int r = 0; r < rows; ++r)
        for (int p = 0; p < half; ++p) {
            float angle = r * powf(theta, -2.0f * p / width);
            float c = cosf(angle), s = sinf(angle);
            float a = in[(size_t)r * width + 2 * p], b = in[(size_t)r * width + 2 * p + 1];
            out[(size_t)r * width + p] = a * c - b * s;
            out[(size_t)r * width + half + p] = b * c + a * s;
        }
}

/* tests/test_moonlight_metal_mla.c */
static int mla(void) {
    MoonlightModel *model = NULL;
    MoonlightSession *full = NULL, *split = NULL;
    MoonlightOptions options = {.context_size = 64, .max_batch = 32};
    char error[512] = {0};
    CHECK(moonlight_model_open(&model, g_model, error, sizeof error) == 1);
    MoonlightModelInfo info = moonlight_model_info(model);
    const int D = info.hidden_size, L = info.kv_lora_rank, R = info.qk_rope_dim;
    int64_t n = st_numel(&g_oracle, "input_ids");
    CHECK(n > 1 && n <= 32);
    float *input = need_f32("layer.0.input_norm", n * D), *attn = need_f32("layer.0.attn", n * D);
    float *kv_a = need_f32("layer.0.kv_a", n * (L + R)), *latent = need_f32("layer.0.kv_norm", n * L);
    CHECK(input && attn && kv_a && latent);
    float *rope_in = malloc((size_t)n * R * 4), *rope = malloc((size_t)n * R * 4);
    for (int r = 0; r < n; ++r) memcpy(rope_in + (size_t)r * R, kv_a + (size_t)r * (L + R) + L, (size_t)R * 4);
    rope_reference(rope_in, rope, (int)n, R, info.rope_theta);
    float *prefill = calloc((size_t)n * D, 4), *prefix = calloc((size_t)(n - 1) * D, 4);
    float *decode = calloc((size_t)D, 4), *a_lat = calloc((size_t)n * L, 4), *a_rope = calloc((size_t)n * R, 4);
    CHECK(moonlight_session_create(&full, model, &options, error, sizeof error) == 1);
    CHECK(moonlight_session_create(&split, model, &options, error, sizeof error) == 1);
    CHECK(moonlight_test_attention(full, 0, input, (int)n, 0, prefill) == 1);
    CHECK(moonlight_test_kv_length(full, 0) == n);
    CHECK(moonlight_session_position(full) == n);
    CHECK(moonlight_test_copy_kv(full, 0, a_lat, a_rope, (int)n) == 1);
    CHECK(moonlight_test_attention(split, 0, input, (int)n - 1, 0, prefix) == 1);
    CHECK(moonlight_test_attention(split, 0, input + (n - 1) * D, 1, (int)n - 1, decode) == 1);
    CHECK(moonlight_test_kv_length(split, 0) == n);
    CHECK(moonlight_test_attention(split, 0, input, 1, (int)n + 1, decode) == 0);  /* not the KV length */
    printf("mla:\n");
    /* fp16 latent cache and q8 row scales under the attention */
    BOUND("attention", max_abs(prefill, attn, n * D), 3e-4, 2e-3);
    /* the split run's last row against the one-shot run's: the GEMVs and the
     * attention reduce in an order that depends only on K and the key index */
    BOUND("split vs one-shot", max_abs(decode, prefill + (n - 1) * D, D), 3e-4, 3e-4);
    /* fp16 cache: 2^-11 relative on values of order 1-4 */
    BOUND("latent (fp16 cache)", max_abs(a_lat, latent, n * L), 3e-5, 4e-3);
    BOUND("rope (fp16 cache)", max_abs(a_rope, rope, n * R), 3e-5, 4e-3);
    CHECK(moonlight_session_stats(full).cpu_fallbacks == 0);
    moonlight_session_reset(split);
    CHECK(moonlight_test_kv_length(split, 0) == 0);
    CHECK(moonlight_session_position(split) == 0);
    moonlight_session_destroy(split);
    moonlight_session_destroy(full);
    moonlight_model_close(model);
    free(input); free(attn); free(kv_a); free(latent); free(rope_in); free(rope);
    free(prefill); free(prefix); free(decode); free(a_lat); free(a_rope);
    return 0;
}

/* tests/test_moonlight_metal_moe.c */
static int moe(void) {
    MoonlightModel *model = NULL;
    MoonlightSession *session = NULL;
    MoonlightOptions options = {.context_size = 64, .max_batch = 32};
    char error[512] = {0};
    CHECK(moonlight_model_open(&model, g_model, error, sizeof error) == 1);
    MoonlightModelInfo info = moonlight_model_info(model);
    const int D = info.hidden_size, E = info.expert_count, K = info.experts_per_token;
    int64_t n = st_numel(&g_oracle, "input_ids"), nid = 0;
    CHECK(n > 0 && n <= 32);
    float *input = need_f32("layer.1.post_norm", n * D), *scores = need_f32("layer.1.router_scores", n * E);
    float *weights = need_f32("layer.1.router_weights", n * K), *routed = need_f32("layer.1.routed_mlp", n * D);
    float *shared = need_f32("layer.1.shared_mlp", n * D), *output = need_f32("layer.1.mlp", n * D);
    int *eids = st_read_ids(&g_oracle, "layer.1.router_ids", &nid);
    CHECK(input && scores && weights && routed && shared && output && eids && nid == n * K);
    int *a_ids = calloc((size_t)n * K, 4);
    float *a_w = calloc((size_t)n * K, 4), *a_sc = calloc((size_t)n * E, 4), *a_r = calloc((size_t)n * D, 4);
    float *a_s = calloc((size_t)n * D, 4), *a_o = calloc((size_t)n * D, 4);
    CHECK(moonlight_session_create(&session, model, &options, error, sizeof error) == 1);
    CHECK(moonlight_test_moe(session, 1, input, (int)n, a_ids, a_w, a_sc, a_r, a_s, a_o) == 1);
    float werr = 0;
    for (int r = 0; r < n; ++r)
        for (int k = 0; k < K; ++k) {
            int slot = -1;
            for (int c = 0; c < K; ++c)
                if (eids[r * K + c] == a_ids[r * K + k]) slot = c;
            CHECK(slot >= 0); /* the same expert set per row */
            float d = fabsf(a_w[r * K + k] - weights[r * K + slot]);
            if (d > werr) werr = d;
        }
    printf("moe:\n");
    /* raw router logits: fp32 weights, hi + lo fp16 activations */
    BOUND("router scores", max_abs(a_sc, scores, n * E), 3e-5, 3e-5);
    BOUND("route weights", werr, 3e-6, 3e-6);
    BOUND("routed (q8 experts)", max_abs(a_r, routed, n * D), 3e-4, 3e-3);
    BOUND("shared (q8)", max_abs(a_s, shared, n * D), 3e-4, 3e-3);
    BOUND("output", max_abs(a_o, output, n * D), 5e-4, 5e-3);
    MoonlightStats st = moonlight_session_stats(session);
    CHECK(st.command_buffers == 1);  /* routing and experts in one submission */
    CHECK(st.cpu_fallbacks == 0);
    moonlight_session_destroy(session);
    moonlight_model_close(model);
    free(input); free(scores); free(weights); free(routed); free(shared); free(output); free(eids);
    free(a_ids); free(a_w); free(a_sc); free(a_r); free(a_s); free(a_o);
    return 0;
}

/* tests/test_moonlight_metal_runtime.c */
static int runtime(void) {
    MoonlightModel *model = NULL;
    MoonlightSession *session = NULL;
    MoonlightOptions options = {.context_size = 64, .max_batch = 32};
    char error[512] = {0};
    CHECK(moonlight_model_open(&model, g_model, error, sizeof error) == 1);
    CHECK(model != NULL);
    CHECK(strstr(moonlight_device_name(model), "B200") != NULL);
    MoonlightModelInfo info = moonlight_model_info(model);
    CHECK(info.hidden_size > 0 && info.layer_count > 0 && info.vocab_size > 0 && info.resident_bytes > 0);
    const int D = info.hidden_size, V = info.vocab_size, K = info.experts_per_token;
    CHECK(moonlight_session_create(&session, model, &options, error, sizeof error) == 1);
    MoonlightStats before = moonlight_session_stats(session);
    CHECK(before.buffer_allocations >= 5);
    CHECK(before.resident_bytes > info.resident_bytes);
    CHECK(before.cpu_fallbacks == 0);
    CHECK(moonlight_session_position(session) == 0);
    moonlight_session_reset(session);
    MoonlightStats after = moonlight_session_stats(session);
    CHECK(after.buffer_allocations == before.buffer_allocations);
    CHECK(after.resident_bytes == before.resident_bytes);
    int64_t n = 0, ng = 0;
    int *ids = st_read_ids(&g_oracle, "input_ids", &n);
    int *greedy = st_read_ids(&g_oracle, "greedy", &ng);
    float *expected = need_f32("logits", -1);
    CHECK(ids && greedy && ng == 2 && expected && n <= options.max_batch);
    float *dense_in = need_f32("layer.0.post_norm", n * D), *dense_out = need_f32("layer.0.mlp", n * D);
    CHECK(dense_in && dense_out);
    float *a_dense = calloc((size_t)n * D, 4), *logits = calloc((size_t)V, 4);
    float *layers = calloc((size_t)info.layer_count * n * D, 4);
    printf("runtime:\n");
    CHECK(moonlight_test_dense_mlp(session, 0, dense_in, (int)n, a_dense) == 1);
    BOUND("dense MLP", max_abs(a_dense, dense_out, n * D), 3e-4, 3e-3);
    CHECK(moonlight_test_prefill_layers(session, ids, (int)n, layers, logits, error, sizeof error) == 1);
    for (int l = 0; l < info.layer_count; ++l) {
        char name[64], label[64];
        snprintf(name, sizeof name, "layer.%d.output", l);
        float *exp_l = need_f32(name, n * D);
        CHECK(exp_l);
        snprintf(label, sizeof label, "layer %d output", l);
        BOUND(label, max_abs(layers + (size_t)l * n * D, exp_l, n * D), 2e-3, 1e-2);
        free(exp_l);
    }
    int mismatches = 0;
    int *routes = calloc((size_t)n * K, 4);
    for (int l = info.first_dense_layer_count; l < info.layer_count; ++l) {
        char name[64];
        int64_t ne = 0;
        snprintf(name, sizeof name, "layer.%d.router_ids", l);
        int *er = st_read_ids(&g_oracle, name, &ne);
        CHECK(er && ne == n * K);
        CHECK(moonlight_test_copy_routes(session, l, routes, (int)n) == 1);
        for (int r = 0; r < n; ++r) {
            int match = 1;
            for (int k = 0; k < K; ++k) {
                int found = 0;
                for (int c = 0; c < K; ++c) found = found || routes[r * K + k] == er[r * K + c];
                match = match && found;
            }
            if (!match) mismatches++;
        }
        free(er);
    }
    printf("  route mismatch rows         %d\n", mismatches);
    CHECK(mismatches == 0);
    float lerr = max_abs(logits, expected + (n - 1) * V, V);
    BOUND("prefill logits", lerr, 3e-4, 1e-2);
    CHECK(argmax(logits, V) == greedy[0]);
    CHECK(moonlight_session_position(session) == n);
    CHECK(moonlight_session_decode(session, greedy[0], logits, error, sizeof error) == 1);
    CHECK(argmax(logits, V) == greedy[1]);
    CHECK(moonlight_session_position(session) == n + 1);
    after = moonlight_session_stats(session);
    CHECK(after.prefill_tokens == (uint64_t)n);
    CHECK(after.decode_tokens == 1);
    CHECK(after.cpu_fallbacks == 0);

    /* the fast path: the session's own prefill (tensor-core chunks for
     * more than 8 rows) and decode */
    moonlight_session_reset(session);
    CHECK(moonlight_session_prefill(session, ids, (int)n, logits, error, sizeof error) == 1);
    lerr = max_abs(logits, expected + (n - 1) * V, V);
    /* fp16 operands of the prefill GEMMs */
    BOUND("fast-path prefill logits", lerr, 3e-4, 3e-2);
    CHECK(argmax(logits, V) == greedy[0]);
    CHECK(moonlight_session_decode(session, greedy[0], logits, error, sizeof error) == 1);
    CHECK(argmax(logits, V) == greedy[1]);
    after = moonlight_session_stats(session);
    CHECK(after.command_buffers <= (uint64_t)(2 * info.layer_count + 2));
    CHECK(after.cpu_fallbacks == 0);
    printf("  timing: prefill %.3f ms, decode %.3f ms\n", after.prefill_ms, after.decode_ms);

    moonlight_session_reset(session);
    int split = (int)n / 2;
    CHECK(moonlight_session_prefill(session, ids, split, logits, error, sizeof error) == 1);
    CHECK(moonlight_session_append(session, ids + split, (int)n - split, logits, error, sizeof error) == 1);
    lerr = max_abs(logits, expected + (n - 1) * V, V);
    BOUND("prefill + append logits", lerr, 3e-4, 1e-2);
    CHECK(argmax(logits, V) == greedy[0]);
    CHECK(moonlight_session_position(session) == n);
    moonlight_session_destroy(session);
    moonlight_model_close(model);
    free(ids); free(greedy); free(expected); free(dense_in); free(dense_out); free(a_dense);
    free(logits); free(layers); free(routes);
    return 0;
}

int main(int argc, char **argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s MODEL_DIR ORACLE.safetensors\n", argv[0]);
        return 2;
    }
    g_model = argv[1];
    if (!st_open(&g_oracle, argv[2])) {
        fprintf(stderr, "cannot open %s\n", argv[2]);
        return 2;
    }
    primitives();
    mla();
    moe();
    runtime();
    st_close(&g_oracle);
    if (failures) {
        printf("FAILED (%d section(s))\n", failures);
        return 1;
    }
    printf("OK\n");
    return 0;
}
