/*
 * moonlight_cuda.c - floyd's Moonlight session API (moonlight_metal.h)
 * implemented over the B200 backend's C ABI (include/floyd_cuda.h).  Drop it
 * into floyd in place of moonlight_metal.m and link libfloyd_cuda.so:
 *
 *   cc -DFLOYD_TREE -I<floyd> -I<this repo>/include -c moonlight_cuda.c
 *   cc ... moonlight_cuda.o -L<this repo>/floyd_b200 -lfloyd_cuda
 *
 * Every call forwards to its fc_ counterpart; the handles are the backend's
 * own (a MoonlightModel * is an FcModel *, a MoonlightSession * an
 * FcSession *).  The CUDA device is FLOYD_CUDA_DEVICE (default 0).  Model
 * info and stats are copied field by field, since the backend's structs
 * carry more fields than the Metal ones.
 */
#include <stdlib.h>

#ifdef FLOYD_TREE
#include "moonlight_metal.h"
#else
#include "moonlight_api.h"
#endif
#include "floyd_cuda.h"

#define M(p) ((FcModel *)(p))
#define S(p) ((FcSession *)(p))

int moonlight_model_open(MoonlightModel **out, const char *path, char *error, size_t error_size) {
    const char *dev = getenv("FLOYD_CUDA_DEVICE");
    return fc_model_open((FcModel **)out, path, dev ? atoi(dev) : 0, error, error_size);
}

void moonlight_model_close(MoonlightModel *model) { fc_model_close(M(model)); }

const char *moonlight_device_name(const MoonlightModel *model) {
    return fc_device_name((const FcModel *)model);
}

MoonlightModelInfo moonlight_model_info(const MoonlightModel *model) {
    MoonlightModelInfo r = {0};
    if (!model) return r;
    FcModelConfig c = fc_model_info((const FcModel *)model);
    r.hidden_size = c.hidden_size;
    r.layer_count = c.layer_count;
    r.vocab_size = c.vocab_size;
    r.head_count = c.head_count;
    r.kv_lora_rank = c.kv_lora_rank;
    r.qk_nope_dim = c.qk_nope_dim;
    r.qk_rope_dim = c.qk_rope_dim;
    r.value_dim = c.value_dim;
    r.expert_count = c.expert_count;
    r.experts_per_token = c.experts_per_token;
    r.moe_intermediate_size = c.moe_intermediate_size;
    r.shared_expert_count = c.shared_expert_count;
    r.first_dense_layer_count = c.first_dense_layer_count;
    r.rms_norm_epsilon = c.rms_norm_epsilon;
    r.rope_theta = c.rope_theta;
    r.routed_scale = c.routed_scale;
    r.resident_bytes = c.resident_bytes;
    return r;
}

int moonlight_session_create(MoonlightSession **out, MoonlightModel *model,
                             const MoonlightOptions *options, char *error, size_t error_size) {
    FcOptions o = {0, 0};
    if (options) {
        o.context_size = options->context_size;
        o.max_batch = options->max_batch;
    }
    return fc_session_create((FcSession **)out, M(model), options ? &o : NULL, error, error_size);
}

void moonlight_session_destroy(MoonlightSession *session) { fc_session_destroy(S(session)); }
void moonlight_session_reset(MoonlightSession *session) { fc_session_reset(S(session)); }
int moonlight_session_position(const MoonlightSession *session) {
    return fc_session_position((const FcSession *)session);
}

MoonlightStats moonlight_session_stats(const MoonlightSession *session) {
    MoonlightStats r = {0};
    if (!session) return r;
    FcStats s = fc_session_stats((const FcSession *)session);
    r.command_buffers = s.command_buffers;
    r.prefill_tokens = s.prefill_tokens;
    r.decode_tokens = s.decode_tokens;
    r.cpu_fallbacks = s.cpu_fallbacks;
    r.buffer_allocations = s.buffer_allocations;
    r.resident_bytes = s.resident_bytes;
    r.prefill_ms = s.prefill_ms;
    r.decode_ms = s.decode_ms;
    return r;
}

int moonlight_session_prefill(MoonlightSession *session, const int *ids, int count, float *last_logits,
                              char *error, size_t error_size) {
    return fc_session_prefill(S(session), ids, count, last_logits, error, error_size);
}

int moonlight_session_append(MoonlightSession *session, const int *ids, int count, float *last_logits,
                             char *error, size_t error_size) {
    return fc_session_append(S(session), ids, count, last_logits, error, error_size);
}

int moonlight_session_decode(MoonlightSession *session, int token, float *logits, char *error,
                             size_t error_size) {
    return fc_session_decode(S(session), token, logits, error, error_size);
}

int moonlight_test_prefill_layers(MoonlightSession *session, const int *ids, int count,
                                  float *layer_outputs, float *last_logits, char *error,
                                  size_t error_size) {
    return fc_test_prefill_layers(S(session), ids, count, layer_outputs, last_logits, error, error_size);
}

int moonlight_test_embed(MoonlightSession *session, const int *ids, int count, float *output) {
    return fc_test_embed(S(session), ids, count, output);
}

int moonlight_test_rmsnorm(MoonlightSession *session, const float *input, const char *weight_name,
                           int rows, int width, float *output) {
    return fc_test_rmsnorm(S(session), input, weight_name, rows, width, output);
}

int moonlight_test_matmul(MoonlightSession *session, const char *weight_name, const float *input,
                          int rows, int input_width, int output_width, float *output) {
    return fc_test_matmul(S(session), weight_name, input, rows, input_width, output_width, output);
}

int moonlight_test_attention(MoonlightSession *session, int layer, const float *input, int rows,
                             int position, float *output) {
    return fc_test_attention(S(session), layer, input, rows, position, output);
}

int moonlight_test_kv_length(const MoonlightSession *session, int layer) {
    return fc_test_kv_length((const FcSession *)session, layer);
}

int moonlight_test_copy_kv(const MoonlightSession *session, int layer, float *latent, float *rope,
                           int capacity) {
    return fc_test_copy_kv((const FcSession *)session, layer, latent, rope, capacity);
}

int moonlight_test_moe(MoonlightSession *session, int layer, const float *input, int rows,
                       int *route_ids, float *route_weights, float *router_scores,
                       float *routed_output, float *shared_output, float *output) {
    return fc_test_moe(S(session), layer, input, rows, route_ids, route_weights, router_scores,
                       routed_output, shared_output, output);
}

int moonlight_test_dense_mlp(MoonlightSession *session, int layer, const float *input, int rows,
                             float *output) {
    return fc_test_dense_mlp(S(session), layer, input, rows, output);
}

int moonlight_test_copy_routes(const MoonlightSession *session, int layer, int *route_ids,
                               int capacity) {
    return fc_test_copy_routes((const FcSession *)session, layer, route_ids, capacity);
}
