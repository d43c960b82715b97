/*
 * floyd_oracle.h - CPU restatement of floyd's verify-step algorithm.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library,
 * and only as the checker or the timed CPU baseline.  The CUDA backend never
 * calls it and has no CPU fallback.
 *
 * Each function names the reference code it restates (paths inside
 * c4pt0r/floyd).  Parity of this restatement is pinned by
 *   - the reference's own known-answer tests (tests/test_moe_route.c,
 *     tests/test_moe_exec.c, tests/test_deepseek_v4_quant.c), restated in
 *     tests/test_oracle_known_answers.py;
 *   - a harness compiled from the reference headers (oracle/ref_harness.c,
 *     built into oracle/_ref/) that the oracle is compared with on random
 *     inputs;
 *   - golden fixtures produced by transformers' DeepseekV3 (the model the
 *     reference's tools/make_oracle.py uses), tests/golden/.
 */
#ifndef FLOYD_ORACLE_H
#define FLOYD_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/floyd_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitives ---------------------------------------------------------- */

void orc_philox4x32_10(const uint32_t counter[4], const uint32_t key[2],
                       uint32_t out[4]);
float orc_fp16_to_f32(uint16_t bits);
uint16_t orc_f32_to_fp16(float value);          /* round to nearest even */
float orc_e8m0_to_f32(uint8_t code);            /* deepseek_v4_quant.h:63-66 */
float orc_e2m1_to_f32(uint8_t code);            /* deepseek_v4_quant.h:48-56 */

/* y[s][o] = sum_k x[s][k] * w[o][k] with w dequantized from `values`
 * (int8 values, int4 values -8..7, or e2m1 codes) and per-32 `scales`
 * (fp32 values of the fp16 / ue8m0 scales).  fmt = FcFormat.  For F32,
 * `f32` holds the matrix.  moonlight_kernels.metal:62-130,
 * deepseek_v4_quant.h:103-139, moe_exec.h:36-44. */
void orc_gemv(int fmt, const int8_t *values, const float *scales,
              const float *f32, int O, int K, const float *x, int S, float *y);

/* moonlight_kernels.metal:23-41 */
void orc_rmsnorm(const float *x, const float *w, int rows, int width, float eps,
                 float *out);

/* moonlight_kernels.metal:132-200: interleaved pairs in, half-split out. */
void orc_rope(const float *in, float *out, int width, int position, float theta);

/* moe_route.h:24-99: scores, selection (bias selects only, lower index wins
 * ties), fixed routes, finalize. Returns the selected count. */
int orc_route(const float *logits, const float *bias, int n_experts, int top_k,
              int score_fn, int normalize, float routed_scale,
              const int *fixed /* nullable: top_k ids */, int *indices,
              float *weights);

/* deepseek_v4_runtime.h:231-237 and fast-argmax.patch:225-233: strict >,
 * lowest index on ties, NaN never wins. */
int orc_argmax(const float *logits, int n);

/* dspark-metal.patch:1793-1797. Returns commit. */
int orc_accept_greedy(const int *row_tops, const int *ids, int k);

/* Rejection-sampling acceptance (Leviathan et al. 2023; Chen et al. 2023)
 * with a point-mass drafter; see fc_session_verify in floyd_cuda.h.
 * logits [k+1][V].  Returns commit, writes *next_token. */
int orc_accept_sample(const float *logits, int V, const int *ids, int k,
                      float temperature, uint64_t seed, uint64_t counter,
                      int *next_token);

/* Uniform in [0, 1) for the accept test of row `row`, and Gumbel noise for
 * vocab index v of row `row` (shared definitions with the CUDA kernels). */
float orc_accept_uniform(uint64_t seed, uint64_t counter, int row);
float orc_gumbel(uint64_t seed, uint64_t counter, int row, int v);

/* moe_f32_forward (moe_exec.h:65-114) on fp32 experts laid out like the
 * reference harness: per expert [w1 gate I x D][w2 down D x I][w3 up I x D]. */
int orc_moe_forward_f32(int hidden, int intermediate, int n_experts, int top_k, int score_fn,
                        int normalize, float routed_scale, float swiglu_limit,
                        const float *router, const float *bias, const float *expert_weights,
                        int n_shared, const float *shared_weights, const float *input,
                        int n_tokens, float *output);

/* ---- model ---------------------------------------------------------------- */

typedef struct OrcModel OrcModel;
typedef struct OrcSession OrcSession;

/* Builds the synthetic model of floyd_synth.h for `config`. */
OrcModel *orc_model_create(const FcModelConfig *config, uint64_t seed);
void orc_model_free(OrcModel *model);

/* Replaces a tensor with fp32 data (golden-fixture tests). `count` must be
 * the tensor's element count. Returns 1 on success. */
int orc_model_set_f32(OrcModel *model, const char *name, const float *data,
                      size_t count);

/* Copies a quantized tensor in the logical layout fc_model_get_tensor uses
 * (values or scales; `scales_part` selects). Returns bytes written or 0. */
size_t orc_model_get_tensor(const OrcModel *model, const char *name,
                            int scales_part, void *data, size_t bytes);

/* kv_fp16: round the cached latent / rope rows, the absorbed query and the
 * rotated query rope part to fp16 before the attention dot products, as the
 * CUDA backend stores them.  0 keeps the reference's fp32 cache. */
OrcSession *orc_session_create(OrcModel *model, int context_size, int kv_fp16);
void orc_session_free(OrcSession *session);
int orc_session_position(const OrcSession *session);
void orc_session_set_position(OrcSession *session, int position);
int orc_session_seed_context(OrcSession *session, int positions, uint64_t seed);
int orc_session_seed_range(OrcSession *session, int start, int end, uint64_t seed);

/* Runs `rows` tokens at the current position and advances it.
 * logits [rows][V] (nullable), layer_out [layers][rows][D] (nullable),
 * routes [layers][rows][top_k] (nullable; -1 for dense layers). */
int orc_session_forward(OrcSession *session, const int *ids, int rows,
                        float *logits, float *layer_out, int *routes);

/* Copies the cached latent / rope rows of `layer` as fp32. */
int orc_session_copy_kv(const OrcSession *session, int layer, float *latent,
                        float *rope, int capacity);

/* Full verify (forward + acceptance + rollback), the CPU counterpart of
 * fc_session_verify. */
/* Proposals of the MTP drafter made by the last orc_session_verify (models
 * with mtp_layers = 1); returns their count. */
int orc_session_drafts(const OrcSession *s, int *out, int capacity);
int orc_session_verify(OrcSession *session, const int *ids, int k,
                       const FcAcceptConfig *accept, int *emitted,
                       int *n_emitted, int *next_token, float *row_logits,
                       int *row_tops);

/* The MTP drafter over the session's history: orc_dspark_rows writes the
 * drafter's latent KV at positions p0 + 1 .. p0 + r from (hidden row q - 1,
 * token q); orc_dspark_propose makes five greedy proposals from the hidden
 * row of position p and the next token. */
int orc_dspark_rows(OrcSession *s, int p0, int r);
int orc_dspark_propose(OrcSession *s, int p, int input_id, int *out, float *conf);

/* Wall seconds spent in the attention and in the FFN / MoE blocks of the
 * forwards since the previous call; resets both. */
void orc_part_times(double *attn_s, double *ffn_s);

#ifdef __cplusplus
}
#endif

#endif
