/*
 * floyd_cuda.h - C ABI of the B200 (sm_100a) backend for floyd's
 * speculative-decode verify step.
 *
 * This header is the drop-in boundary.  It mirrors floyd's Metal session API
 * (moonlight_metal.h:1-96) function for function, with the prefix `fc_`
 * instead of `moonlight_`, and adds the verify / rollback calls that the
 * DS4 speculative loop needs (deepseek_v4_ds4.c:570-691 drives them through
 * ds4_session_eval_speculative_argmax, patches/ds4/deepseek-v4-dspark-metal.patch
 * :1727-1906).
 *
 * Conventions kept from the reference (moonlight_metal.m:97-105):
 *   - functions that can fail return int: 1 = ok, 0 = failure;
 *   - failures fill `error` (size `error_size`) via vsnprintf;
 *   - `*out` handles are set to NULL on failure;
 *   - every host array is caller-owned; logits are copied out as float[vocab];
 *   - a session is used from one host thread; a model may be shared
 *     read-only by several sessions.
 *
 * Everything runs on the GPU.  There is no CPU fallback: FcStats.cpu_fallbacks
 * exists for parity with MoonlightStats and always reads 0.
 *
 * Weights are resident on the device, in the layouts described next to
 * FcFormat.  Session buffers (latent KV cache, activations, scratch) are all
 * allocated in fc_session_create; FcStats.buffer_allocations stays flat
 * afterwards (tests/test_moonlight_metal_runtime.c:106-115).
 */
#ifndef FLOYD_CUDA_H
#define FLOYD_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct FcModel FcModel;     /* replaces MoonlightModel   (moonlight_metal.h:7) */
typedef struct FcSession FcSession; /* replaces MoonlightSession (moonlight_metal.h:8) */

/* Weight storage formats.  Quantized formats use groups of 32 along the
 * input (K) dimension; K must be a multiple of 32.
 *   FC_FMT_F32   fp32 [O][K] (router weights, norms).
 *   FC_FMT_Q8    symmetric int8, one fp16 scale per group of 32
 *                (the 34-byte Q8_0-style block of BASELINE config 1/2).
 *   FC_FMT_Q4    int4 stored with a +8 offset (value = nibble - 8), one fp16
 *                scale per 32; the even element sits in the low nibble
 *                (moonlight_kernels.metal:123-127).
 *   FC_FMT_MXFP4 e2m1 codes (deepseek_v4_quant.h:48-51) with one ue8m0 scale
 *                per 32 (deepseek_v4_quant.h:63-66).
 * On the device the values of a row are permuted so that one tensor-core
 * MMA step always covers a single scale group; fc_model_set_tensor takes the
 * plain row-major logical layout and performs that permutation. */
typedef enum {
    FC_FMT_F32 = 0,
    FC_FMT_Q8 = 1,
    FC_FMT_Q4 = 2,
    FC_FMT_MXFP4 = 3
} FcFormat;

/* Router score functions, same values and meaning as MoeScoreFn
 * (moe_route.h:6-10). */
typedef enum {
    FC_SCORE_SOFTMAX = 0,
    FC_SCORE_SIGMOID = 1,
    FC_SCORE_SQRT_SOFTPLUS = 2
} FcScoreFn;

/* Model description.  Field names follow MoonlightModelInfo
 * (moonlight_metal.h:15-33); the extra fields cover the DS4-style stand-in
 * (q-lora, hash-routed layers, swiglu clamp) and the per-family formats. */
typedef struct {
    int hidden_size;
    int layer_count;
    int vocab_size;
    int head_count;
    int q_lora_rank;             /* 0 = plain q_proj (Moonlight)        */
    int kv_lora_rank;            /* latent width L                      */
    int qk_nope_dim;
    int qk_rope_dim;             /* R, even                             */
    int value_dim;
    int expert_count;
    int experts_per_token;
    int moe_intermediate_size;
    int shared_expert_count;     /* shared experts fused into one wide MLP */
    int first_dense_layer_count;
    int dense_intermediate_size;
    int hash_layer_count;        /* layers < this use moe_route_fixed     */
    int score_fn;                /* FcScoreFn                           */
    int normalize_topk;
    int has_selection_bias;      /* e_score_correction_bias present     */
    float routed_scale;
    float swiglu_limit;          /* <= 0: no clamp (moe_exec.h:55-60)   */
    float rms_norm_epsilon;
    float rope_theta;
    int dense_format;            /* FcFormat of attention, dense, shared,
                                    embedding and lm-head matrices       */
    int expert_format;           /* FcFormat of routed experts           */
    int mtp_layers;              /* 0, or 1: a DeepSeek-V3-style MTP drafter
                                    layer (enorm / hnorm / eh_proj, one MoE
                                    layer, shared_head.norm, shared lm-head) */
    int embed_f32;               /* 1: embedding and lm-head stored as fp32
                                    [vocab][hidden] (floyd's Moonlight
                                    container keeps them unquantized,
                                    tools/convert_moonlight.py:12-17); 0: in
                                    dense_format                         */
    uint64_t resident_bytes;     /* filled by fc_model_info              */
} FcModelConfig;

/* Session sizing, same meaning as MoonlightOptions (moonlight_metal.h:10-13):
 * 0 < max_batch <= context_size. */
typedef struct {
    int context_size;
    int max_batch;
} FcOptions;

/* MoonlightStats (moonlight_metal.h:35-44) plus verify counters. */
typedef struct {
    uint64_t command_buffers;     /* graph / stream submissions          */
    uint64_t prefill_tokens;
    uint64_t decode_tokens;
    uint64_t cpu_fallbacks;       /* always 0: there is no CPU path      */
    uint64_t buffer_allocations;
    uint64_t resident_bytes;
    double prefill_ms;
    double decode_ms;
    uint64_t verify_calls;
    uint64_t proposed_tokens;     /* drafts offered to verify            */
    uint64_t accepted_tokens;     /* tokens committed by verify          */
    uint64_t graph_replays;       /* CUDA-graph launches                 */
    double verify_ms;             /* host wall time inside fc_session_verify */
    double gpu_ms;                /* device time of all graph replays
                                     (CUDA events on the session stream)  */
} FcStats;

/* Acceptance rule of fc_session_verify. */
typedef enum {
    FC_ACCEPT_GREEDY = 0,  /* dspark-metal.patch:1793-1797                */
    FC_ACCEPT_SAMPLE = 1   /* speculative rejection sampling, Philox RNG  */
} FcAcceptMode;

typedef struct {
    int mode;              /* FcAcceptMode                                */
    float temperature;     /* > 0 for FC_ACCEPT_SAMPLE                    */
    uint64_t seed;         /* Philox4x32-10 key                           */
    uint64_t counter;      /* Philox counter base; callers advance it     */
} FcAcceptConfig;

/* ---- model -------------------------------------------------------------- */

/* Creates a model on CUDA device `device` with every weight allocated and
 * resident but not yet filled.  Rejects configurations whose weights exceed
 * 95% of free device memory (moonlight_metal.m:834-843 does the same against
 * the Metal working-set budget). */
int fc_model_create(FcModel **out, const FcModelConfig *config, int device,
                    char *error, size_t error_size);

/* Expert-parallel variant: rank `rank` of `world` holds routed experts
 * [rank * E / world, (rank + 1) * E / world); attention, dense, shared,
 * router and lm-head weights are replicated.  E must divide by world. */
int fc_model_create_ep(FcModel **out, const FcModelConfig *config, int device,
                       int rank, int world, char *error, size_t error_size);

/* Opens floyd's Moonlight model directory, the counterpart of
 * moonlight_model_open (moonlight_metal.h:46-47, moonlight_model.c:41-110):
 * config.json (hidden_size, num_hidden_layers, ..., rope_theta or
 * rope_parameters.rope_theta, scoring_func with sigmoid as the default) and
 * every *.safetensors shard written by tools/convert_moonlight.py.  Int8 /
 * int4 matrices come as U8 values plus `name`.qs fp32 row scales (each row's
 * scale is rounded to fp16 for its group scales, as in
 * fc_model_set_tensor_rowscale); the embedding and lm-head stay fp32
 * (embed_f32 = 1); router weights, norms and selection biases are fp32.
 * Fails, naming the tensor, when one the model needs is missing; tensors the
 * model does not use (rotary_emb.inv_freq) are ignored.  Weights are
 * uploaded once and stay resident on CUDA device `device`. */
int fc_model_open(FcModel **out, const char *path, int device, char *error,
                  size_t error_size);

/* Fills every weight with the seeded synthetic generator of floyd_synth.h
 * (integer-only Philox mapping, identical to the CPU oracle's). */
int fc_model_fill_synthetic(FcModel *model, uint64_t seed,
                            char *error, size_t error_size);

/* Uploads one tensor by its checkpoint name
 * ("model.layers.3.self_attn.kv_b_proj.weight", moonlight_metal.m:301-321).
 * Quantized matrices take two calls: `name` with the values in logical
 * row-major layout (int8 [O][K], packed nibbles [O][K/2] with the even
 * element low, or e2m1 codes packed the same way) and `name` + ".gs" with the
 * group scales (fp16 [O][K/32], or ue8m0 bytes for MXFP4).  F32 tensors take
 * float data.  `bytes` must match exactly. */
int fc_model_set_tensor(FcModel *model, const char *name, const void *data,
                        size_t bytes, char *error, size_t error_size);

/* Weight ingest from checkpoint block formats (no counterpart in the Metal
 * session: floyd's host code reads these formats itself).
 *
 * GGUF blocks (ggml type ids): Q8_0 = {fp16 d; int8 q[32]} per 32 values,
 * MXFP4 = {ue8m0 e; uint8 q[16]} per 32 values with element j in the low
 * nibble and element j + 16 in the high nibble of q[j]
 * (patches/ds4/deepseek-v4-mxfp4-runtime.patch, block_mxfp4; the reader in
 * deepseek-v4-dspark-metal.patch:4430-4460).  Both map exactly onto the
 * q8 / MXFP4 group-32 formats. */
typedef enum { FC_BLOCKS_Q8_0 = 8, FC_BLOCKS_MXFP4 = 39 } FcBlockType;

/* Host-only conversion of rows x cols values stored as blocks (cols / 32
 * blocks per row) into the logical layout of fc_model_set_tensor: values
 * (int8 [rows][cols], or e2m1 codes packed two per byte with the even element
 * low) and group scales (fp16 bits, or ue8m0 bytes) [rows][cols / 32]. */
int fc_blocks_to_logical(int block_type, const void *blocks, size_t bytes, int rows, int cols,
                         void *values, void *scales, char *error, size_t error_size);

/* Uploads one q8 (Q8_0 blocks) or MXFP4 (MXFP4 blocks) matrix; exact. */
int fc_model_set_tensor_blocks(FcModel *model, const char *name, int block_type,
                               const void *blocks, size_t bytes, char *error,
                               size_t error_size);

/* Uploads one matrix of floyd's Moonlight container
 * (tools/convert_moonlight.py:50-75): U8 values (int8, or int4 stored as
 * q + 8 with the even element in the low nibble) and one fp32 scale per row
 * (`name` + ".qs").  Every 32-column group takes the row's scale rounded to
 * fp16 (the group-32 fp16 format of this backend; the only change). */
int fc_model_set_tensor_rowscale(FcModel *model, const char *name, const void *values,
                                 size_t value_bytes, const float *row_scales, int rows,
                                 char *error, size_t error_size);

/* Downloads a tensor in the same logical layout fc_model_set_tensor takes. */
int fc_model_get_tensor(const FcModel *model, const char *name, void *data,
                        size_t bytes, char *error, size_t error_size);

void fc_model_close(FcModel *model);                      /* moonlight_metal.h:50 */
const char *fc_device_name(const FcModel *model);         /* moonlight_metal.h:51 */
FcModelConfig fc_model_info(const FcModel *model);        /* moonlight_metal.h:52 */

/* ---- session ------------------------------------------------------------ */

int fc_session_create(FcSession **out, FcModel *model, const FcOptions *options,
                      char *error, size_t error_size);   /* moonlight_metal.h:54-56 */
void fc_session_destroy(FcSession *session);               /* moonlight_metal.h:57 */
void fc_session_reset(FcSession *session);                 /* moonlight_metal.h:58 */
int fc_session_position(const FcSession *session);         /* moonlight_metal.h:59 */
FcStats fc_session_stats(const FcSession *session);        /* moonlight_metal.h:60 */

/* Runs `count` tokens at position 0 (requires an empty session) and copies
 * the logits of the last row.  moonlight_metal.h:61-63, moonlight_metal.m:1988-2005. */
int fc_session_prefill(FcSession *session, const int *ids, int count,
                       float *last_logits, char *error, size_t error_size);

/* Runs `count` tokens at the current position (> 0).  moonlight_metal.h:64-66. */
int fc_session_append(FcSession *session, const int *ids, int count,
                      float *last_logits, char *error, size_t error_size);

/* One token.  moonlight_metal.h:67-68, moonlight_metal.m:2024-2037. */
int fc_session_decode(FcSession *session, int token, float *logits,
                      char *error, size_t error_size);

/* Speculative verify of 1 + k rows at the current position.
 *   ids[0]      the token the target already chose (the previous round's
 *               next_token, i.e. proposals[0] in the DS4 loop);
 *   ids[1..k]   the k draft tokens.
 * Greedy: row_tops[i] = argmax(logits of row i) (strict >, lowest index on
 * ties, NaN ignored); commit = 1 + the number of leading i >= 1 with
 * row_tops[i-1] == ids[i] (dspark-metal.patch:1793-1797).
 * Sample: draft ids[i] is accepted when u_i < p_{i-1}(ids[i]) with
 * p = softmax(logits / temperature); the first rejected draft is replaced
 * by a sample of p_{i-1} with ids[i] removed, and a fully accepted round
 * samples a bonus token from p_k.  Uniforms and Gumbel noise come from
 * Philox4x32-10 keyed by `seed` at counter (`counter`, row, index).
 * On return emitted[0..commit-1] = ids[0..commit-1], *n_emitted = commit,
 * *next_token = the target's token after them, the latent KV cache is
 * rolled back to position + commit and the position advances by commit.
 * `last_logits` (nullable) receives the logits row commit-1. */
int fc_session_verify(FcSession *session, const int *ids, int k,
                      const FcAcceptConfig *accept, int *emitted,
                      int *n_emitted, int *next_token, float *last_logits,
                      char *error, size_t error_size);

/* Truncates the session to `position` (clamped to <= the current one), as
 * ds4_session_rewind (dspark-metal.patch:1973).  MLA keeps no compressor
 * state, so rollback is a KV-length change. */
int fc_session_rollback(FcSession *session, int position,
                        char *error, size_t error_size);

/* Copies the logits of every row of the last forward ([rows][vocab]; for a
 * batch session, the last pass of the last verify); the Metal backend keeps
 * only the last row (moonlight_metal.m:708-725). */
int fc_session_copy_row_logits(const FcSession *session, float *logits,
                               int capacity_rows);

/* Fills latent KV positions [0, positions) of every layer with the seeded
 * synthetic generator and sets the position, so a long context exists without
 * a prefill (benchmark and test hook, like moonlight_test_* in
 * moonlight_metal.h:69-96). */
int fc_session_seed_context(FcSession *session, int positions, uint64_t seed,
                            char *error, size_t error_size);

/* ---- batched multi-sequence verify ---------------------------------------
 * A batch session holds `sequences` sequences over one paged latent cache
 * (64-row pages).  Their first `shared_prefix` positions (a multiple of 64)
 * live in pages every sequence maps: the prefix-cache snapshot of
 * deepseek_v4_prefix_cache.c:139-229, reused instead of copied.  Each
 * sequence has its own position and private pages for the rest of its
 * context.  fc_session_verify_batch runs one verify of 1 + k rows for every
 * sequence, packing floor(8 / (1 + k)) sequences into each device pass so
 * that they share the weight reads, and accepts and rolls back each sequence
 * on its own.  On one GPU the passes of a verify run concurrently, up to 4
 * at a time, each on its own stream and workspace over the shared cache
 * (environment FLOYD_BATCH_LANES=n caps that at n; 1 runs them one at a
 * time).  Each sequence gets the same result as the same verify in a
 * one-sequence session.  No reference counterpart: floyd verifies one
 * sequence at a time. */
typedef struct {
    int context_size;        /* positions per sequence                       */
    int sequences;           /* 1 .. 64                                      */
    int rows_per_sequence;   /* 1 + drafts of each verify (1 .. 8)           */
    int shared_prefix;       /* positions shared by all sequences (x64)      */
} FcBatchOptions;

int fc_session_create_batch(FcSession **out, FcModel *model, const FcBatchOptions *options,
                            char *error, size_t error_size);

/* Synthetic latent KV (the generator of fc_session_seed_context) for
 * positions [start, end) of one sequence; positions below shared_prefix are
 * the shared pages.  The sequence's position becomes end when that is
 * further.  Benchmark and test hook. */
int fc_session_batch_seed(FcSession *session, int sequence, int start, int end, uint64_t seed,
                          char *error, size_t error_size);

/* ids: [sequences][1 + k] (row 0 the last accepted token, then the drafts);
 * accept: one config per sequence (NULL: greedy).  Outputs per sequence:
 * n_emitted (1 .. k + 1, the committed prefix of its ids) and next_token.
 * Every sequence must be at a position >= shared_prefix (its rows must not
 * land in the shared pages). */
int fc_session_verify_batch(FcSession *session, const int *ids, int k, const FcAcceptConfig *accept,
                            int *n_emitted, int *next_token, char *error, size_t error_size);

int fc_session_batch_position(const FcSession *session, int sequence);
/* Truncates one sequence to `position` (clamped to <= its current one). */
int fc_session_batch_rollback(FcSession *session, int sequence, int position, char *error,
                              size_t error_size);

/* Draft proposals of the on-device MTP drafter (models with mtp_layers = 1).
 * Every fc_session_verify with k > 0 runs the drafter in the same device
 * graph after acceptance: k sequential greedy steps from the last committed
 * row's hidden state and the next token (the role of
 * deepseek_v4_forward_dspark_propose, deepseek_v4_forward.h:1873-1949, for
 * the 1-layer MTP stand-in).  Copies the k proposals of the last verify into
 * `drafts` and returns k (0 when none were made). */
int fc_session_drafts(const FcSession *session, int *drafts, int capacity);

/* Kernels launched by the last forward pass (kernel nodes of its CUDA
 * graph; 0 for eager profiled passes; for a batch session, every pass of
 * the last wave of concurrent passes).  No reference counterpart. */
int fc_session_last_kernel_count(const FcSession *session);

/* Bytes of the two host<->device copies every forward pass makes: the
 * per-pass parameter record copied to the device at the head of the pass
 * and the result record copied back at its tail (logits copies the caller
 * asks for come on top).  No reference counterpart. */
void fc_io_bytes(size_t *h2d, size_t *d2h);

/* Expert parallelism across the GPUs of one box (no reference counterpart:
 * floyd has no communication backend; the contract follows the expert
 * partitioning of moe_exec.h:97-110 with one exchange per MoE layer).
 * A session of a model made by fc_model_create_ep with world > 1 owns a
 * receive region (two buffers of every rank's routed expert outputs plus
 * epoch flags).  fc_session_ep_handle writes its CUDA IPC handle
 * (FC_EP_HANDLE_BYTES bytes); the caller gathers the handles of all ranks
 * (rank order) and passes them to fc_session_ep_connect on every rank.
 * Afterwards every rank must make the same sequence of forward calls
 * (prefill / append / decode / verify) with the same ids: each MoE layer
 * stores this rank's expert outputs into every peer's region over
 * NVLink, publishes an epoch flag, and waits (bounded, about 1 s) for the
 * peers' flags before the combine, which sums all experts in ascending id
 * exactly as on one GPU.  Forward calls fail until the session is
 * connected. */
#define FC_EP_HANDLE_BYTES 64
/* Milliseconds the MoE combines of this rank spent waiting for the peers'
 * expert outputs (the exposed part of the exchange: one timer per MoE layer,
 * on the device) since the previous call; resets the counter.  0 for a
 * single-GPU session. */
double fc_session_exchange_wait_ms(FcSession *session);
int fc_session_ep_handle(FcSession *session, void *handle, size_t handle_size,
                         char *error, size_t error_size);
int fc_session_ep_connect(FcSession *session, const void *handles, int world,
                          char *error, size_t error_size);

/* Per-kernel profiling, the CUDA counterpart of MOONLIGHT_PROFILE
 * (moonlight_metal.m:1899-1979) and ds4's kernel counters.  While enabled,
 * forwards run eagerly (no graph) with a CUDA event after every kernel, and
 * the time between events accumulates per kernel name.  fc_session_profile
 * returns entry `index` (0 past the end). */
int fc_session_set_profiling(FcSession *session, int enabled);
int fc_session_profile(const FcSession *session, int index, char *name,
                       size_t name_size, double *total_ms, uint64_t *launches);
void fc_session_profile_reset(FcSession *session);

/* ---- test hooks (moonlight_metal.h:69-96) -------------------------------- */

/* Single-primitive hooks, each the counterpart of the moonlight_test_* call
 * named beside it and returning 1 on success, 0 on failure.  Each runs the
 * same device code the forward runs, on up to options.max_batch rows, and
 * counts one submission in FcStats.command_buffers (one per hook call, the
 * MoE hook included: routing and experts run without a host round trip).
 *   embed:      output[count][hidden] = embedding rows of ids       (:73-74)
 *   rmsnorm:    output = RMSNorm(input) with the named norm vector  (:75-77)
 *   matmul:     output[rows][output_width] = input . W^T of the named
 *               matrix (quantized or fp32)                          (:78-80)
 *   attention:  the attention block of `layer` (q / kv_a, KV append, MLA,
 *               o_proj) on normalized input rows at positions position ..
 *               position + rows - 1; position must equal the session's
 *               position (the layer's KV length), which then advances
 *               by rows                                             (:81-83)
 *   moe:        the MoE block of `layer` on normalized rows: route ids and
 *               weights [rows][top-k] in selection order, the raw router
 *               logits [rows][experts], routed sum, shared experts' output
 *               and their sum [rows][hidden] (any output may be NULL
 *               except `output`)                                    (:88-92)
 *   dense_mlp:  the dense MLP of a first-k-dense layer              (:93-94)
 *   prefill_layers: prefill of `count` tokens into an empty session with
 *               the hidden state after every layer [layers][count][hidden]
 *               and the last row's logits                           (:67-70) */
int fc_test_embed(FcSession *session, const int *ids, int count, float *output);
int fc_test_rmsnorm(FcSession *session, const float *input, const char *weight_name,
                    int rows, int width, float *output);
int fc_test_matmul(FcSession *session, const char *weight_name, const float *input,
                   int rows, int input_width, int output_width, float *output);
int fc_test_attention(FcSession *session, int layer, const float *input, int rows,
                      int position, float *output);
int fc_test_moe(FcSession *session, int layer, const float *input, int rows,
                int *route_ids, float *route_weights, float *router_scores,
                float *routed_output, float *shared_output, float *output);
int fc_test_dense_mlp(FcSession *session, int layer, const float *input, int rows,
                      float *output);
int fc_test_prefill_layers(FcSession *session, const int *ids, int count,
                           float *layer_outputs, float *last_logits,
                           char *error, size_t error_size);

int fc_test_kv_length(const FcSession *session, int layer);      /* :85 */
/* The acceptance kernels of the verify graph (row argmax, softmax
 * partials, Gumbel picks, the acceptance rule of fc_session_verify) run on
 * caller-given logits [rows][vocab] with ids[0..rows-1] (ids[0] the target's
 * token, ids[1..] the drafts, k = rows - 1), once for each of `trials`
 * Philox counters accept->counter, accept->counter + 1, ...; writes each
 * trial's commit and next token.  For distribution tests of the sampling
 * rule, which has no counterpart in the reference. */
int fc_test_accept(const float *logits, int rows, int vocab, const int *ids,
                   const FcAcceptConfig *accept, int trials, int *commits,
                   int *next_tokens, char *error, size_t error_size);
/* The page table a batch session builds (host only, no GPU): fills
 * table[sequence][page] and returns the physical page count, -1 on invalid
 * options or a short buffer. */
int fc_test_batch_page_table(int context_size, int sequences, int shared_prefix, int *table,
                             int capacity);
/* latent [capacity][kv_lora_rank], rope [capacity][qk_rope_dim] as fp32. */
int fc_test_copy_kv(const FcSession *session, int layer, float *latent,
                    float *rope, int capacity);                   /* :86-87 */
/* route ids [rows][experts_per_token] of the last forward (selection order). */
int fc_test_copy_routes(const FcSession *session, int layer, int *route_ids,
                        int capacity);                            /* :95-96 */
/* Enables the per-layer hidden-state copies that fc_test_copy_layer_outputs
 * reads (off by default: they add a copy per layer to every forward). */
int fc_session_set_layer_trace(FcSession *session, int enabled);
/* hidden state after each layer of the last forward: [layers][rows][hidden];
 * needs fc_session_set_layer_trace(session, 1) before that forward. */
int fc_test_copy_layer_outputs(const FcSession *session, float *outputs,
                               int capacity_rows);

/* ---- spec-runtime contract (deepseek_v4_runtime.h:72-256) --------------- */

/* A thin owner of one session with the deepseek_v4_runtime_* call shapes. */
typedef struct {
    FcSession *session;
    float *logits;       /* last forward's last row, [vocab]           */
    int vocab_size;
    int max_context;
    int last_count;
    int last_start_position;
    int dspark_ready;    /* fc_runtime_dspark_prefill has run          */
} FcRuntime;

int fc_runtime_init(FcRuntime *runtime, FcModel *model, int max_context,
                    int max_batch);                                /* :72-97   */
int fc_runtime_forward(FcRuntime *runtime, const int *token_ids, int n_tokens,
                       const float **logits);                      /* :148-178 */
int fc_runtime_argmax(const float *logits, int vocab_size);        /* :231-237 */
int fc_runtime_verify_token(const float *logits, int vocab_size,
                            int64_t proposal, int *accepted);      /* :239-244 */
void fc_runtime_reset(FcRuntime *runtime);                         /* :99-128  */
/* The drafter of a model with an MTP layer (mtp_layers = 1), the stand-in
 * for ds4's DSpark block (deepseek_v4_runtime.h:180-223).
 * dspark_prefill: after a forward that started at position 0, runs the
 * drafter layer over the prompt (hidden row of position p with the token at
 * p + 1, for every p) so that its latent cache covers the prompt; once per
 * runtime until fc_runtime_reset.
 * dspark_propose: from the last forward's last row and the next token
 * `input_id`, five greedy drafter steps; output_ids[0] = input_id,
 * output_ids[1..5] = the proposals, confidence[i] = the drafter's top-1
 * logit of proposal i (the stand-in drafter has no learned confidence head,
 * deepseek_v4_forward.h:1935-1944).  Both return 1 on success. */
int fc_runtime_dspark_prefill(FcRuntime *runtime);
int fc_runtime_dspark_propose(FcRuntime *runtime, int input_id, int64_t output_ids[6],
                              float confidence[5]);
void fc_runtime_free(FcRuntime *runtime);                          /* :246-256 */

#ifdef __cplusplus
}
#endif

#endif /* FLOYD_CUDA_H */
