/*
 * ref_harness.c - exposes floyd's own C reference headers through a small
 * C ABI so the tests can compare the oracle restatement (floyd_oracle.c) with
 * the reference on identical inputs.  TEST INFRASTRUCTURE ONLY.
 *
 * Built by oracle/Makefile into oracle/_ref/libref_harness.so from the
 * headers where they lie in the reference checkout (-I$(REF)); no reference
 * source is copied into this repository.
 *   moe_route.h:24-99        routing (scores, select, fixed, finalize)
 *   moe_exec.h:36-114        expert execution (matvec, clamped SwiGLU,
 *                            ascending-expert accumulation, shared experts)
 *   deepseek_v4_quant.h:103-139  e2m1 / ue8m0 fp4 matmul
 */
#include <stdint.h>
#include <stdlib.h>

#include "moe_exec.h"
#include "deepseek_v4_quant.h"

int ref_route_select(const float *logits, const float *bias, int n_experts,
                     int top_k, int score_fn, int normalize, float scale,
                     int *indices, float *weights) {
    float scores[1024], choices[1024];
    if (n_experts > 1024) return 0;
    int n = moe_route_select(logits, bias, n_experts, top_k, (MoeScoreFn)score_fn,
                             indices, weights, scores, choices);
    moe_route_finalize(weights, n, normalize, scale);
    return n;
}

int ref_route_fixed(const float *logits, int n_experts, const int *indices,
                    int count, int score_fn, int normalize, float scale,
                    float *weights) {
    float scores[1024];
    if (n_experts > 1024) return 0;
    int n = moe_route_fixed(logits, n_experts, indices, count, (MoeScoreFn)score_fn,
                            weights, scores);
    moe_route_finalize(weights, n, normalize, scale);
    return n;
}

/* experts: [n_experts][3] pointers (w1 = gate [I][D], w2 = down [D][I],
 * w3 = up [I][D]) laid out as gate | down | up blocks of `expert_block`
 * floats each; shared likewise (n_shared of them, width I each). */
int ref_moe_forward(int hidden, int intermediate, int n_experts, int top_k,
                    int score_fn, int normalize, float route_scale,
                    float swiglu_limit, const float *router, const float *bias,
                    const int64_t *fixed, int vocab_size, const float *expert_weights,
                    int n_shared, const float *shared_weights,
                    const float *input, const int *token_ids, int n_tokens,
                    float *output) {
    size_t block = (size_t)hidden * intermediate;
    MoeExpertF32 *experts = calloc((size_t)n_experts, sizeof(*experts));
    MoeExpertF32 *shared = calloc((size_t)(n_shared > 0 ? n_shared : 1), sizeof(*shared));
    for (int e = 0; e < n_experts; ++e) {
        experts[e].w1 = expert_weights + (3 * (size_t)e + 0) * block;
        experts[e].w2 = expert_weights + (3 * (size_t)e + 1) * block;
        experts[e].w3 = expert_weights + (3 * (size_t)e + 2) * block;
    }
    for (int e = 0; e < n_shared; ++e) {
        shared[e].w1 = shared_weights + (3 * (size_t)e + 0) * block;
        shared[e].w2 = shared_weights + (3 * (size_t)e + 1) * block;
        shared[e].w3 = shared_weights + (3 * (size_t)e + 2) * block;
    }
    MoeF32 model = {
        .hidden = hidden, .intermediate = intermediate, .n_experts = n_experts,
        .top_k = top_k, .vocab_size = vocab_size, .score_fn = (MoeScoreFn)score_fn,
        .normalize = normalize, .route_scale = route_scale,
        .swiglu_limit = swiglu_limit, .router = router, .selection_bias = bias,
        .fixed_experts = fixed, .experts = experts,
        .shared_experts = n_shared > 0 ? shared : NULL, .n_shared_experts = n_shared,
    };
    int ok = moe_f32_forward(&model, input, token_ids, n_tokens, output);
    free(experts);
    free(shared);
    return ok;
}

int ref_fp4_matmul(float *output, const float *input, int n_inputs,
                   const uint8_t *weights, const uint8_t *scales, int rows,
                   int columns) {
    return deepseek_v4_fp4_matmul_f32(output, input, n_inputs, weights, scales,
                                      rows, columns);
}

float ref_e8m0(uint8_t code) { return deepseek_v4_e8m0_to_f32(code); }
float ref_fp4_code(uint8_t code) { return deepseek_v4_fp4_code_value(code); }
