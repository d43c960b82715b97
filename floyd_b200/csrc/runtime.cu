// runtime.cu - model, session and C ABI of the B200 verify-step backend
// (include/floyd_cuda.h).
//
// The host side mirrors moonlight_metal.m: weights resident on the device,
// every session buffer allocated up front (moonlight_metal.m:938-1125), one
// submission per forward.  Where the Metal runtime records a command buffer
// per MoE layer and round-trips the route tables through the host
// (moonlight_metal.m:1892-1986), here the whole forward - embedding, every
// layer, lm-head, argmax and acceptance - is one CUDA graph per row count,
// with one H2D copy of the per-call parameters at its head and one D2H copy
// of the result at its tail.  Everything runs on the GPU; a missing or
// failing kernel is an error, never a CPU fallback.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/floyd_kernels.h"
#include "../../include/floyd_fm.h"
#include "common.cuh"
#include "container.h"
#include "gemv.cuh"
#include "head.cuh"
#include "mla.cuh"
#include "mla_tc.cuh"
#include "moe.cuh"
#include "prefill.cuh"
#include "synth.cuh"

using namespace fc;

namespace {

int set_error(char *error, size_t error_size, const char *format, ...) {
    if (error && error_size) {
        va_list args;
        va_start(args, format);
        vsnprintf(error, error_size, format, args);
        va_end(args);
    }
    return 0;
}

double now_ms() {
    return std::chrono::duration<double, std::milli>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

inline int kpad(int k) { return (k + 127) / 128 * 128; }

// A matrix (or a family of `count` equally shaped matrices) in device layout.
struct DevMat {
    int fmt = FC_FMT_F32, O = 0, K = 0, kp = 0, count = 0;
    uint8_t *w = nullptr;   // tile-major values + scales (common.cuh), or fp32 data
    size_t w_bytes = 0;     // per member
    uint32_t tid = 0;       // synthetic tensor id (slot 0)
    int slot0 = 0;          // synthetic slot of member 0
};

struct DevVec {
    float *p = nullptr;
    size_t n = 0;
    uint32_t tid = 0;
    int kind = 1;  // 0 f32 matrix, 1 norm, 2 bias
};

struct DevLayer {
    DevVec attn_norm, ffn_norm, kv_a_norm, q_a_norm, router, bias;
    DevMat q_proj, q_a, q_b, kv_a, kv_b, o_proj;
    DevMat d_gate, d_up, d_down;
    DevMat e_gate, e_up, e_down;   // routed expert families (local experts)
    DevMat s_gate, s_up, s_down;   // shared experts (one wide MLP)
    int *hash = nullptr;           // [vocab][K] or null
    uint32_t hash_tid = 0;
    bool dense = false;
    DevVec enorm, hnorm, head_norm;  // MTP drafter layer only
    DevMat eh_proj;                  // MTP: [D][2D]
};

struct TensorRef {
    DevMat *mat = nullptr;
    int member = 0;
    DevVec *vec = nullptr;
    int *ints = nullptr;
    size_t ints_n = 0;
};

}  // namespace

struct FcModel {
    FcModelConfig c{};
    int device = 0;
    int sms = 148;                     // multiprocessors of the device
    int expert_lo = 0, expert_hi = 0;  // local routed experts
    int rank = 0, world = 1;           // expert-parallel position
    std::string device_name;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    DevMat embed, lm_head;
    DevVec final_norm;
    std::vector<DevLayer> layers;
    std::map<std::string, TensorRef> names;
    uint64_t resident = 0;
};

constexpr int kMaxLanes = 4;  // concurrent passes of a batch step

struct FcSession {
    FcModel *m = nullptr;
    FcOptions opt{};
    cudaStream_t stream = nullptr;
    int rows_max = 0;        // rows per pass (<= kMaxRows)
    int position = 0;
    int last_rows = 0;
    // latent-cache paging (head.cuh PageMap): page table [sequences][pps] on
    // the device; an ordinary session maps each page to itself
    int *page_table = nullptr;
    PageMap pmap{};
    int layer_rows = 0;      // cache rows per layer
    int n_seq = 1;           // sequences (batch sessions)
    int group_rows = 0;      // rows per sequence in a batch pass (1 + drafts)
    int shared_rows = 0;     // leading positions every sequence shares (batch sessions)
    std::vector<int> seq_pos;  // position of each sequence (batch sessions)
    bool batch = false;      // created by fc_session_create_batch
    int max_slots = 0;
    int splits = 0, chunks_per_split = 1;
    // split plan of the drafter (MTP) layers: they always run one row per
    // pass against their own cache, so with the tcgen05 kernel they take
    // enough splits to fill the SMs with one query tile
    int mtp_splits = 0, mtp_chunks_per_split = 1;
    bool attn_tc = true;     // tcgen05 attention (else the mma.sync kernel)
    CUtensorMap qmap{}, kvmap{};  // TMA maps of qcat and of the latent cache
    int head_chunks = 0;
    std::vector<void *> allocs;
    FcStats stats{};
    // buffers
    __half *cache = nullptr;
    float *resid = nullptr, *xn = nullptr, *q = nullptr, *qa = nullptr, *ckv = nullptr;
    __half *xq_norm = nullptr, *qa_xq = nullptr, *qcat = nullptr, *ctx_xq = nullptr, *o_xq = nullptr;
    float *part_o = nullptr, *part_m = nullptr, *part_l = nullptr;
    float *router_logits = nullptr, *route_w = nullptr, *coef = nullptr;
    int *route_ids = nullptr, *n_active = nullptr, *active = nullptr;
    __half *h_xq = nullptr, *hsh_xq = nullptr, *hd_xq = nullptr;
    float *moe_part = nullptr, *sh_part = nullptr;
    float *logits = nullptr, *layer_out = nullptr;
    HeadPartials hp{};
    int *d_err = nullptr;    // bit 1: a bounded wait in a kernel gave up
    int *route_arrivals = nullptr;   // router block counter (zero between launches)
    Staging *d_mtp = nullptr;        // MTP drafter step parameters (device)
    float *mtp_h = nullptr;          // drafter hidden state [D]
    float *mtp_logits = nullptr;     // drafter logits [V] (the target's stay readable)
    __half *mtp_xq = nullptr;        // [enorm(embed) | hnorm(h)] as xq, [rows_max][kpad(2D)]
    float *hist = nullptr;           // final hidden row of every position [context][D] (MTP models)
    std::vector<int> tok_hist;       // token id of every position (MTP models)
    // routes of every row of the last fc_test_prefill_layers call
    // [layers][rows][top-k]; cleared by the next forward
    std::vector<int> route_trace;
    int route_trace_rows = 0;
    int last_drafts = 0;             // proposals made by the last pass
    int *n_global = nullptr, *n_before = nullptr;  // global active experts / first global slot here
    int g_slots = 0;                 // global slots (active experts of all ranks) at most
    // expert parallel (model world > 1): receive region = two buffers of the
    // routed outputs of every rank [2][g_slots][rows][D] + kMaxRanks epoch
    // flags, exported by IPC; the peers' regions opened here
    void *ep_region = nullptr;
    float *ep_xbuf = nullptr;
    int *ep_flags = nullptr, *ep_epoch = nullptr;
    unsigned long long *ep_wait_ns = nullptr;  // time the combines spent waiting for peers
    // head-parallel attention (expert-parallel single-sequence sessions):
    // this rank runs heads [head0, head0 + heads) of the MLA block; the W_UV
    // outputs of every rank meet in each rank's o_proj input, two buffers
    // (layer parity) in the receive region after the expert exchange
    bool head_shard = false;
    int head0 = 0, heads = 0;
    size_t ep_attn_off = 0, ep_oxq_bytes = 0;  // byte offsets in the region: flags, then [2] o_proj inputs
    int *ep_aepoch = nullptr;
    int *ep_adone = nullptr;     // W_UV CTAs finished (zero between launches)
    void *ep_peer_region[kMaxRanks] = {};
    bool ep_connected = false;
    Staging *d_stage = nullptr, *h_stage = nullptr;
    Result *d_res = nullptr, *h_res = nullptr;
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, int> graph_kernels;  // kernel nodes of each captured graph
    int last_kernels = 0;              // kernels launched by the last pass
    size_t attn_smem = 0;
    cudaEvent_t ev_begin = nullptr, ev_end = nullptr;   // device time of each pass
    // per-kernel profiling (eager passes with an event after every launch)
    bool profiling = false;
    bool trace = false;      // per-layer hidden-state copies (test hook)
    std::vector<cudaEvent_t> prof_events;
    // prefill chunks of more than rows_max tokens (max_batch > 8): tcgen05
    // GEMMs over up to pf_rows tokens, buffers rows padded to pf_pad (x128)
    int pf_rows = 0, pf_pad = 0, pf_slots = 0;
    int *pf_ids = nullptr, *pf_h_ids = nullptr;   // [position, ids...] device / pinned host
    float *pf_resid = nullptr, *pf_xn = nullptr, *pf_ckv = nullptr, *pf_qa = nullptr;
    float *pf_logits = nullptr, *pf_choice = nullptr, *pf_route_w = nullptr, *pf_yd = nullptr, *pf_sh = nullptr;
    float *pf_rpart = nullptr;   // router k-split partials [splits][rows][E]
    __half *pf_x16 = nullptr, *pf_q16 = nullptr, *pf_qa16 = nullptr, *pf_kvd = nullptr;
    __half *pf_o16 = nullptr, *pf_h16 = nullptr, *pf_xg = nullptr, *pf_hg = nullptr;
    int *pf_route_ids = nullptr, *pf_counts = nullptr, *pf_offsets = nullptr, *pf_cursor = nullptr;
    int *pf_slot_of = nullptr, *pf_mt_count = nullptr;
    int4 *pf_mt_table = nullptr;
    std::map<std::pair<const void *, int>, CUtensorMap> pf_wmaps;  // weight maps by (base, box tiles)
    CUtensorMap pf_map_x{}, pf_map_q{}, pf_map_qa{}, pf_map_o{}, pf_map_hd{}, pf_map_hs{}, pf_map_xg{},
        pf_map_hg{}, pf_map_kvd{}, pf_cmap{}, pf_cmap64{};
    std::vector<std::string> prof_marks;
    // batch sessions: child sessions ("lanes") with their own workspace,
    // stream and graphs over this session's latent cache and page table; the
    // passes of one batch step run on them concurrently (single GPU)
    std::vector<FcSession *> lanes;
    bool lane = false;                 // a lane (does not own the cache)
    const FcSession *last_lane = nullptr;  // the lane of the last pass (its logits)
    cudaEvent_t ev_lane = nullptr;     // end of this lane's pass
    std::vector<std::pair<std::string, std::pair<double, uint64_t>>> prof;
};

namespace {

// ---------------------------------------------------------------------------
// model construction
// ---------------------------------------------------------------------------
size_t align256(size_t n) { return (n + 255) / 256 * 256; }

void plan_mat(DevMat &m, int fmt, int O, int K, int count, uint32_t tid, int slot0) {
    m.fmt = fmt; m.O = O; m.K = K; m.count = count; m.tid = tid; m.slot0 = slot0;
    if (fmt == FC_FMT_F32) {
        m.kp = K;
        m.w_bytes = (size_t)O * K * 4;
    } else {
        m.kp = kpad(K);
        m.w_bytes = matrix_bytes(fmt, O, m.kp);
    }
}

size_t mat_bytes(const DevMat &m) {
    if (!m.count) return 0;
    return align256(m.w_bytes * m.count);
}

void place_mat(FcModel *model, DevMat &m) {
    if (!m.count) return;
    m.w = model->arena + model->arena_used;
    model->arena_used += align256(m.w_bytes * m.count);
}

void plan_vec(DevVec &v, size_t n, uint32_t tid, int kind) { v.n = n; v.tid = tid; v.kind = kind; }

void place_vec(FcModel *model, DevVec &v) {
    if (!v.n) return;
    v.p = reinterpret_cast<float *>(model->arena + model->arena_used);
    model->arena_used += align256(v.n * 4);
}

template <typename F>
void for_each_tensor(FcModel *m, F f) {
    f(&m->embed, nullptr);
    f(&m->lm_head, nullptr);
    f(nullptr, &m->final_norm);
    for (auto &y : m->layers) {
        DevVec *vecs[] = {&y.attn_norm, &y.ffn_norm, &y.kv_a_norm, &y.q_a_norm, &y.router, &y.bias,
                          &y.enorm, &y.hnorm, &y.head_norm};
        for (DevVec *v : vecs) f(nullptr, v);
        DevMat *mats[] = {&y.q_proj, &y.q_a, &y.q_b, &y.kv_a, &y.kv_b, &y.o_proj,
                          &y.d_gate, &y.d_up, &y.d_down, &y.e_gate, &y.e_up, &y.e_down,
                          &y.s_gate, &y.s_up, &y.s_down, &y.eh_proj};
        for (DevMat *mm : mats) f(mm, nullptr);
    }
}

bool config_ok(const FcModelConfig *c, char *err, size_t n) {
    if (c->hidden_size <= 0 || c->layer_count <= 0 || c->vocab_size <= 0 || c->head_count <= 0)
        return set_error(err, n, "invalid model dimensions");
    if (c->hidden_size % 32 || c->kv_lora_rank % 32 || (c->q_lora_rank % 32) ||
        c->moe_intermediate_size % 32 || c->dense_intermediate_size % 32 ||
        (c->head_count * c->value_dim) % 32)
        return set_error(err, n, "every matrix input width must be a multiple of 32");
    if (c->hidden_size % 4)
        return set_error(err, n, "hidden_size must be a multiple of 4");
    if (!(c->kv_lora_rank == 512 && c->qk_rope_dim == 64) &&
        !(c->kv_lora_rank == 256 && c->qk_rope_dim == 64))
        return set_error(err, n, "supported MLA shapes: kv_lora_rank 512 or 256 with rope 64");
    if (c->qk_rope_dim & 1) return set_error(err, n, "qk_rope_dim must be even");
    if (c->first_dense_layer_count < c->layer_count &&
        (c->expert_count <= 0 || c->expert_count > 1024 || c->experts_per_token <= 0 ||
         c->experts_per_token > c->expert_count || c->experts_per_token > 64))
        return set_error(err, n, "unsupported expert configuration");
    auto fmt_ok = [](int f) { return f == FC_FMT_Q8 || f == FC_FMT_Q4 || f == FC_FMT_MXFP4; };
    if (!fmt_ok(c->dense_format) || !fmt_ok(c->expert_format))
        return set_error(err, n, "dense and expert formats must be Q8, Q4 or MXFP4");
    if (c->first_dense_layer_count > 0 && c->dense_intermediate_size <= 0)
        return set_error(err, n, "dense layers need dense_intermediate_size");
    if (c->mtp_layers < 0 || c->mtp_layers > 1 ||
        (c->mtp_layers && c->first_dense_layer_count > c->layer_count))
        return set_error(err, n, "mtp_layers must be 0 or 1");
    return true;
}

int build_model(FcModel *m, char *err, size_t n) {
    const FcModelConfig &c = m->c;
    int D = c.hidden_size, H = c.head_count, L = c.kv_lora_rank, R = c.qk_rope_dim;
    int df = c.dense_format, ef = c.expert_format;
    const int hf = c.embed_f32 ? FC_FMT_F32 : df;
    plan_mat(m->embed, hf, c.vocab_size, D, 1, fc_tensor_id(-1, FC_T_EMBED, 0), 0);
    plan_mat(m->lm_head, hf, c.vocab_size, D, 1, fc_tensor_id(-1, FC_T_LM_HEAD, 0), 0);
    plan_vec(m->final_norm, D, fc_tensor_id(-1, FC_T_FINAL_NORM, 0), 1);
    m->layers.resize(c.layer_count + c.mtp_layers);
    int nl = m->expert_hi - m->expert_lo;
    for (int l = 0; l < c.layer_count + c.mtp_layers; ++l) {
        DevLayer &y = m->layers[l];
        if (l >= c.layer_count) {  // MTP drafter extras
            plan_vec(y.enorm, D, fc_tensor_id(l, FC_T_MTP_ENORM, 0), 1);
            plan_vec(y.hnorm, D, fc_tensor_id(l, FC_T_MTP_HNORM, 0), 1);
            plan_vec(y.head_norm, D, fc_tensor_id(l, FC_T_MTP_HEAD_NORM, 0), 1);
            plan_mat(y.eh_proj, df, D, 2 * D, 1, fc_tensor_id(l, FC_T_MTP_EH_PROJ, 0), 0);
        }
        plan_vec(y.attn_norm, D, fc_tensor_id(l, FC_T_ATTN_NORM, 0), 1);
        plan_vec(y.ffn_norm, D, fc_tensor_id(l, FC_T_FFN_NORM, 0), 1);
        plan_vec(y.kv_a_norm, L, fc_tensor_id(l, FC_T_KV_A_NORM, 0), 1);
        int qw = H * (c.qk_nope_dim + R);
        if (c.q_lora_rank > 0) {
            plan_vec(y.q_a_norm, c.q_lora_rank, fc_tensor_id(l, FC_T_Q_A_NORM, 0), 1);
            plan_mat(y.q_a, df, c.q_lora_rank, D, 1, fc_tensor_id(l, FC_T_Q_A, 0), 0);
            plan_mat(y.q_b, df, qw, c.q_lora_rank, 1, fc_tensor_id(l, FC_T_Q_B, 0), 0);
        } else {
            plan_mat(y.q_proj, df, qw, D, 1, fc_tensor_id(l, FC_T_Q_PROJ, 0), 0);
        }
        plan_mat(y.kv_a, df, L + R, D, 1, fc_tensor_id(l, FC_T_KV_A, 0), 0);
        plan_mat(y.kv_b, df, H * (c.qk_nope_dim + c.value_dim), L, 1, fc_tensor_id(l, FC_T_KV_B, 0), 0);
        plan_mat(y.o_proj, df, D, H * c.value_dim, 1, fc_tensor_id(l, FC_T_O_PROJ, 0), 0);
        y.dense = l < c.first_dense_layer_count;
        if (y.dense) {
            int I = c.dense_intermediate_size;
            plan_mat(y.d_gate, df, I, D, 1, fc_tensor_id(l, FC_T_DENSE_GATE, 0), 0);
            plan_mat(y.d_up, df, I, D, 1, fc_tensor_id(l, FC_T_DENSE_UP, 0), 0);
            plan_mat(y.d_down, df, D, I, 1, fc_tensor_id(l, FC_T_DENSE_DOWN, 0), 0);
            continue;
        }
        int E = c.expert_count, I = c.moe_intermediate_size;
        plan_vec(y.router, (size_t)E * D, fc_tensor_id(l, FC_T_ROUTER, 0), 0);
        if (c.has_selection_bias) plan_vec(y.bias, E, fc_tensor_id(l, FC_T_ROUTER_BIAS, 0), 2);
        // slot of expert e is e + 1; the local family starts at expert_lo
        plan_mat(y.e_gate, ef, I, D, nl, fc_tensor_id(l, FC_T_EXP_GATE, 0), m->expert_lo + 1);
        plan_mat(y.e_up, ef, I, D, nl, fc_tensor_id(l, FC_T_EXP_UP, 0), m->expert_lo + 1);
        plan_mat(y.e_down, ef, D, I, nl, fc_tensor_id(l, FC_T_EXP_DOWN, 0), m->expert_lo + 1);
        if (c.shared_expert_count > 0) {
            int W = I * c.shared_expert_count;
            plan_mat(y.s_gate, df, W, D, 1, fc_tensor_id(l, FC_T_SH_GATE, 0), 0);
            plan_mat(y.s_up, df, W, D, 1, fc_tensor_id(l, FC_T_SH_UP, 0), 0);
            plan_mat(y.s_down, df, D, W, 1, fc_tensor_id(l, FC_T_SH_DOWN, 0), 0);
        }
        if (l < c.hash_layer_count) y.hash_tid = fc_tensor_id(l, FC_T_HASH, 0);
    }
    // size the arena
    size_t total = 0;
    for_each_tensor(m, [&](DevMat *mm, DevVec *v) {
        if (mm) total += mat_bytes(*mm);
        if (v) total += align256(v->n * 4);
    });
    size_t hash_bytes = 0;
    for (auto &y : m->layers)
        if (y.hash_tid) hash_bytes += align256((size_t)c.vocab_size * c.experts_per_token * 4);
    total += hash_bytes;
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    if (total > free_b / 100 * 95)
        return set_error(err, n, "model requires %.2f GiB, above 95%% of free device memory %.2f GiB",
                         total / 1073741824.0, free_b / 1073741824.0);
    if (cudaMalloc(&m->arena, total) != cudaSuccess)
        return set_error(err, n, "device allocation of %.2f GiB failed", total / 1073741824.0);
    m->arena_bytes = total;
    cudaMemset(m->arena, 0, total);
    for_each_tensor(m, [&](DevMat *mm, DevVec *v) {
        if (mm) place_mat(m, *mm);
        if (v) place_vec(m, *v);
    });
    for (auto &y : m->layers)
        if (y.hash_tid) {
            y.hash = reinterpret_cast<int *>(m->arena + m->arena_used);
            m->arena_used += align256((size_t)c.vocab_size * c.experts_per_token * 4);
        }
    m->resident = total;

    // checkpoint names (moonlight_metal.m:301-321, :450-466, :494-500, :580-612)
    auto add_mat = [&](const std::string &name, DevMat &mm, int member) {
        if (mm.count) m->names[name] = TensorRef{&mm, member, nullptr, nullptr, 0};
    };
    auto add_vec = [&](const std::string &name, DevVec &v) {
        if (v.n) m->names[name] = TensorRef{nullptr, 0, &v, nullptr, 0};
    };
    add_mat("model.embed_tokens.weight", m->embed, 0);
    add_mat("lm_head.weight", m->lm_head, 0);
    add_vec("model.norm.weight", m->final_norm);
    for (int l = 0; l < c.layer_count + c.mtp_layers; ++l) {
        DevLayer &y = m->layers[l];
        std::string p = "model.layers." + std::to_string(l) + ".";
        add_vec(p + "enorm.weight", y.enorm);
        add_vec(p + "hnorm.weight", y.hnorm);
        add_vec(p + "shared_head.norm.weight", y.head_norm);
        add_mat(p + "eh_proj.weight", y.eh_proj, 0);
        add_vec(p + "input_layernorm.weight", y.attn_norm);
        add_vec(p + "post_attention_layernorm.weight", y.ffn_norm);
        add_vec(p + "self_attn.kv_a_layernorm.weight", y.kv_a_norm);
        add_vec(p + "self_attn.q_a_layernorm.weight", y.q_a_norm);
        add_mat(p + "self_attn.q_proj.weight", y.q_proj, 0);
        add_mat(p + "self_attn.q_a_proj.weight", y.q_a, 0);
        add_mat(p + "self_attn.q_b_proj.weight", y.q_b, 0);
        add_mat(p + "self_attn.kv_a_proj_with_mqa.weight", y.kv_a, 0);
        add_mat(p + "self_attn.kv_b_proj.weight", y.kv_b, 0);
        add_mat(p + "self_attn.o_proj.weight", y.o_proj, 0);
        add_mat(p + "mlp.gate_proj.weight", y.d_gate, 0);
        add_mat(p + "mlp.up_proj.weight", y.d_up, 0);
        add_mat(p + "mlp.down_proj.weight", y.d_down, 0);
        add_vec(p + "mlp.gate.weight", y.router);
        add_vec(p + "mlp.gate.e_score_correction_bias", y.bias);
        if (y.hash)
            m->names[p + "mlp.gate.tid2eid"] =
                TensorRef{nullptr, 0, nullptr, y.hash, (size_t)c.vocab_size * c.experts_per_token};
        for (int e = m->expert_lo; e < m->expert_hi && !y.dense; ++e) {
            std::string q = p + "mlp.experts." + std::to_string(e) + ".";
            add_mat(q + "gate_proj.weight", y.e_gate, e - m->expert_lo);
            add_mat(q + "up_proj.weight", y.e_up, e - m->expert_lo);
            add_mat(q + "down_proj.weight", y.e_down, e - m->expert_lo);
        }
        add_mat(p + "mlp.shared_experts.gate_proj.weight", y.s_gate, 0);
        add_mat(p + "mlp.shared_experts.up_proj.weight", y.s_up, 0);
        add_mat(p + "mlp.shared_experts.down_proj.weight", y.s_down, 0);
    }
    return 1;
}

int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, 148 * 16); }

cudaError_t fill_mat(const DevMat &mm, uint64_t seed, cudaStream_t st) {
    if (!mm.count) return cudaSuccess;
    if (mm.fmt == FC_FMT_F32) {
        size_t n = (size_t)mm.O * mm.K * mm.count;
        synth_f32_kernel<<<grid_for(n), 256, 0, st>>>(reinterpret_cast<float *>(mm.w), n, 0, seed, mm.tid);
        return cudaGetLastError();
    }
    size_t nb = (size_t)mm.O * mm.K / (mm.fmt == FC_FMT_Q8 ? 8 : 32) * mm.count;
    synth_values_kernel<<<grid_for(nb), 256, 0, st>>>(mm.fmt, mm.w, mm.O, mm.K, mm.kp, mm.count,
                                                      seed, mm.tid, mm.slot0);
    size_t ns = ((size_t)mm.O * (mm.K / 32) + 3) / 4 * mm.count;
    synth_scales_kernel<<<grid_for(ns), 256, 0, st>>>(mm.fmt, mm.w, mm.O, mm.K, mm.kp, mm.count,
                                                      seed, mm.tid, mm.slot0);
    return cudaGetLastError();
}

// Logical row-major values (int8 / packed nibbles, even element low) into
// the tile-major device image `dev` of one member (values only).
void pack_values(const DevMat &mm, const uint8_t *src, uint8_t *dev) {
    for (int o = 0; o < mm.O; ++o)
        for (int k = 0; k < mm.K; ++k) {
            int nib;
            size_t off = value_offset(mm.fmt, mm.kp, o, k, &nib);
            if (mm.fmt == FC_FMT_Q8) {
                dev[off] = src[(size_t)o * mm.K + k];
            } else {
                size_t e = (size_t)o * mm.K + k;
                uint8_t v = (src[e >> 1] >> (4 * (e & 1))) & 15;
                dev[off] = (uint8_t)((dev[off] & ~(15 << (4 * nib))) | (v << (4 * nib)));
            }
        }
}

void unpack_values(const DevMat &mm, const uint8_t *dev, uint8_t *dst) {
    if (mm.fmt != FC_FMT_Q8) memset(dst, 0, (size_t)mm.O * mm.K / 2);
    for (int o = 0; o < mm.O; ++o)
        for (int k = 0; k < mm.K; ++k) {
            int nib;
            uint8_t b = dev[value_offset(mm.fmt, mm.kp, o, k, &nib)];
            if (mm.fmt == FC_FMT_Q8) {
                dst[(size_t)o * mm.K + k] = b;
            } else {
                size_t e = (size_t)o * mm.K + k;
                uint8_t v = (b >> (4 * nib)) & 15;
                dst[e >> 1] |= (uint8_t)(v << (4 * (e & 1)));
            }
        }
}

// Group scales [O][K/32] (fp16 bits or ue8m0 bytes) <-> the device image.
void pack_scales(const DevMat &mm, const uint8_t *src, uint8_t *dev) {
    int gk = mm.K / 32, el = scale_elem_bytes(mm.fmt);
    for (int o = 0; o < mm.O; ++o)
        for (int g = 0; g < gk; ++g)
            memcpy(dev + scale_offset(mm.fmt, mm.kp, o, g), src + ((size_t)o * gk + g) * el, el);
}

void unpack_scales(const DevMat &mm, const uint8_t *dev, uint8_t *dst) {
    int gk = mm.K / 32, el = scale_elem_bytes(mm.fmt);
    for (int o = 0; o < mm.O; ++o)
        for (int g = 0; g < gk; ++g)
            memcpy(dst + ((size_t)o * gk + g) * el, dev + scale_offset(mm.fmt, mm.kp, o, g), el);
}

// ---------------------------------------------------------------------------
// session
// ---------------------------------------------------------------------------
template <typename T>
bool salloc(FcSession *s, T *&p, size_t count) {
    void *raw = nullptr;
    size_t bytes = align256(std::max<size_t>(count * sizeof(T), 16));
    if (cudaMalloc(&raw, bytes) != cudaSuccess) return false;
    cudaMemset(raw, 0, bytes);
    s->allocs.push_back(raw);
    s->stats.buffer_allocations++;
    s->stats.resident_bytes += bytes;
    p = reinterpret_cast<T *>(raw);
    return true;
}

void free_session_buffers(FcSession *s) {
    for (auto &g : s->graphs) cudaGraphExecDestroy(g.second);
    s->graphs.clear();
    for (void *&p : s->ep_peer_region)
        if (p) {
            cudaIpcCloseMemHandle(p);
            p = nullptr;
        }
    if (s->ep_region) cudaFree(s->ep_region);
    s->ep_region = nullptr;
    for (void *p : s->allocs) cudaFree(p);
    s->allocs.clear();
    if (s->h_stage) cudaFreeHost(s->h_stage);
    if (s->h_res) cudaFreeHost(s->h_res);
    if (s->pf_h_ids) cudaFreeHost(s->pf_h_ids);
    s->pf_h_ids = nullptr;
    s->h_stage = nullptr;
    s->h_res = nullptr;
    if (s->stream) cudaStreamDestroy(s->stream);
    s->stream = nullptr;
    if (s->ev_begin) cudaEventDestroy(s->ev_begin);
    if (s->ev_end) cudaEventDestroy(s->ev_end);
    if (s->ev_lane) cudaEventDestroy(s->ev_lane);
    s->ev_begin = s->ev_end = s->ev_lane = nullptr;
    for (cudaEvent_t ev : s->prof_events) cudaEventDestroy(ev);
    s->prof_events.clear();
}

GemvSeg seg_of(const DevMat &mm, const __half *xq, int epi) {
    GemvSeg g{};
    g.w = mm.w;
    g.xq = xq;
    g.O = mm.O;
    g.kp = mm.kp;
    g.epi = epi;
    g.count = 1;
    return g;
}

#define FC_TRY(expr)                                 \
    do {                                             \
        cudaError_t e_ = (expr);                     \
        if (e_ != cudaSuccess) return e_;            \
    } while (0)

cudaError_t gemv1(int fmt, GemvSeg a, int S, float limit, int *err, int sms, cudaStream_t st,
                  const GemvWork *sync = nullptr) {
    GemvBatch b{};
    b.sync = sync;
    b.seg[0] = a;
    b.nseg = 1;
    b.S = S;
    b.swiglu_limit = limit;
    b.err = err;
    return launch_gemv_batch(fmt, b, sms, st);
}

// The lm-head over S rows of xq activations: the quantized GEMV, or the fp32
// GEMV when the model keeps its lm-head unquantized.
cudaError_t head_gemv(const FcModel *m, const __half *xq, int S, float *y, int *err, cudaStream_t st) {
    const DevMat &h = m->lm_head;
    if (h.fmt == FC_FMT_F32)
        return launch_f32_gemv(reinterpret_cast<const float *>(h.w), h.O, h.K, xq, kpad(h.K), S, y, h.O,
                               m->sms, st);
    GemvSeg g = seg_of(h, xq, EPI_STORE);
    g.y = y;
    g.ldy = h.O;
    return gemv1(h.fmt, g, S, 0.0f, err, m->sms, st);
}

// 2-D fp16 tensor map [rows][inner] with a {64, box_rows} box and the
// 128-byte swizzle the tcgen05 descriptors expect.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }();
    return encode;
}

bool make_map_f16(CUtensorMap *map, void *base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D byte tensor map of a tile-major quantized matrix family (`tiles`
// 16-row tiles of padded width kp): [tiles][chunks][block_bytes / 64][64],
// box {64, block_bytes / 64, 1, box_tiles} - one chunk block of box_tiles
// consecutive tiles, landing in shared memory as consecutive blocks.
bool make_map_weights(CUtensorMap *map, const uint8_t *w, int fmt, uint64_t tiles, int kp, uint32_t box_tiles) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return false;
    const uint64_t bb = (uint64_t)block_bytes(fmt);
    cuuint64_t dims[4] = {64, bb / 64, (cuuint64_t)chunk_count(fmt, kp), tiles};
    cuuint64_t strides[3] = {64, bb, (cuuint64_t)tile_bytes(fmt, kp)};
    cuuint32_t box[4] = {64, (cuuint32_t)(bb / 64), 1, box_tiles};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(w), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Records a profiling event after the launch named `name` (eager passes only).
void mark(FcSession *s, const char *name) {
    if (!s->profiling) return;
    size_t i = s->prof_marks.size();
    if (i + 1 >= s->prof_events.size()) return;
    s->prof_marks.push_back(name);
    cudaEventRecord(s->prof_events[i + 1], s->stream);
}

// Enqueues one forward of `rows` rows (parameters already in d_stage) on the
// session stream: embedding, every layer, lm-head, argmax / acceptance.
// Enqueues layer l (target layers 0 .. layer_count - 1, the MTP layer at
// layer_count) for S rows at positions *d_pos + s, updating s->resid.
// `ids` are the rows' token ids (hash routing).
// The attention block of layer l over S rows whose normalized input is
// already in xq_norm: q / kv_a projections, KV append, absorbed attention,
// W_UV, and o_proj through epilogue `o_epi` into `o_y` (EPI_ADD into the
// residual in a forward; EPI_STORE for the attention test hook).
cudaError_t record_attention(FcSession *s, int S, int l, const Staging *dst, int o_epi, float *o_y) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size, H = c.head_count, L = c.kv_lora_rank, R = c.qk_rope_dim;
    const int NP = c.qk_nope_dim, VD = c.value_dim, QW = NP + R;
    const int kpD = kpad(D), kpL = kpad(L), kpO = kpad(H * VD);
    const int mb = s->rows_max;
    const float scale = 1.0f / sqrtf((float)(NP + R));
    const int df = c.dense_format, ef = c.expert_format;
    (void)kpL;
    (void)kpO;
    (void)ef;
    DevLayer &y = m->layers[l];
    __half *cache = s->cache + (size_t)l * s->layer_rows * (L + R);
    // head-parallel sessions run heads [h0, h0 + Hl) from q_b to W_UV
    const int Hl = s->head_shard ? s->heads : H, h0 = s->head0;
    const uint8_t *kv_b_w = y.kv_b.w + (size_t)(h0 * (NP + VD) / kTileRows) * tile_bytes(df, y.kv_b.kp);
    const __half *o_in = s->o_xq;  // o_proj input
    GemvWork o_sync{};             // o_proj's wait for the peers' heads (head-parallel)
    (void)kpD;
    {
        GemvBatch b{};
        b.S = S;
        b.err = s->d_err;
        if (c.q_lora_rank > 0) {
            b.seg[0] = seg_of(y.q_a, s->xq_norm, EPI_STORE);
            b.seg[0].y = s->qa;
            b.seg[0].ldy = c.q_lora_rank;
        } else {
            b.seg[0] = seg_of(y.q_proj, s->xq_norm, EPI_STORE);
            b.seg[0].y = s->q;
            b.seg[0].ldy = H * QW;
        }
        b.seg[1] = seg_of(y.kv_a, s->xq_norm, EPI_STORE);
        b.seg[1].y = s->ckv;
        b.seg[1].ldy = L + R;
        b.nseg = 2;
        FC_TRY(launch_gemv_batch(df, b, m->sms, st));
        mark(s, "gemv_q_kv_a");
    }
    if (c.q_lora_rank > 0) {
        FC_TRY(launch_pdl(rmsnorm_kernel, dim3(S), dim3(norm_threads(c.q_lora_rank)), 0, st, s->qa, c.q_lora_rank, y.q_a_norm.p, c.q_lora_rank,
                                          c.rms_norm_epsilon, s->qa_xq, kpad(c.q_lora_rank),
                                          nullptr, 0));
        mark(s, "rmsnorm");
        GemvSeg g = seg_of(y.q_b, s->qa_xq, EPI_STORE);
        g.w += (size_t)(h0 * QW / kTileRows) * tile_bytes(df, y.q_b.kp);
        g.O = Hl * QW;
        g.y = s->q;
        g.ldy = Hl * QW;
        FC_TRY(gemv1(df, g, S, 0.0f, s->d_err, m->sms, st));
        mark(s, "gemv_q_b");
    }
    {
        const int prep_y = 1 + (Hl * (R / 2) + 255) / 256;
        const int blocks = S * prep_y + Hl * (L / kAbsorbCols);
        FC_TRY(launch_pdl(mla_prep_absorb_kernel, dim3(blocks), dim3(256), 0, st, (const float *)s->ckv,
                          (const float *)s->q, (const float *)y.kv_a_norm.p, L, R, Hl, NP, c.rms_norm_epsilon,
                          c.rope_theta, dst, s->pmap, cache, s->qcat, S, prep_y, df, kv_b_w,
                          y.kv_b.kp, VD));
        mark(s, "mla_prep_absorb");
    }
    const bool mtp_layer = l >= c.layer_count;
    const int nsplit = mtp_layer ? s->mtp_splits : s->splits;
    if (s->attn_tc) {
        dim3 grid((S * Hl + kTcRows - 1) / kTcRows, 2, nsplit);
        const int kv_row0 = l * s->layer_rows,
                  kps = (mtp_layer ? s->mtp_chunks_per_split : s->chunks_per_split) * kAttnKeys;
        if (L == 512)
            FC_TRY(launch_pdl(mla_attention_tc_kernel<512>, grid, dim3(kTcThreads), TcAttnPlan<512>::SMEM, st,
                              s->qmap, s->kvmap, kv_row0, S, Hl, kps, dst, s->pmap, scale, s->part_o, s->part_m,
                              s->part_l, s->d_err));
        else
            FC_TRY(launch_pdl(mla_attention_tc_kernel<256>, grid, dim3(kTcThreads), TcAttnPlan<256>::SMEM, st,
                              s->qmap, s->kvmap, kv_row0, S, Hl, kps, dst, s->pmap, scale, s->part_o, s->part_m,
                              s->part_l, s->d_err));
        mark(s, "mla_attention");
    } else {
        dim3 grid((S * H + kAttnQ - 1) / kAttnQ, s->splits);
        if (L == 512)
            FC_TRY(launch_pdl(mla_attention_kernel<512, 64>, grid, dim3(kAttnThreads), s->attn_smem,
                              st, (const __half *)cache, (const __half *)s->qcat, S, H,
                              s->chunks_per_split, dst, s->pmap, scale, s->part_o, s->part_m, s->part_l));
        else
            FC_TRY(launch_pdl(mla_attention_kernel<256, 64>, grid, dim3(kAttnThreads), s->attn_smem,
                              st, (const __half *)cache, (const __half *)s->qcat, S, H,
                              s->chunks_per_split, dst, s->pmap, scale, s->part_o, s->part_m, s->part_l));
        mark(s, "mla_attention");
    }
    {
        size_t head_stride = (size_t)mb * kpL * 2;
        FC_TRY(launch_pdl(mla_combine_kernel, dim3(S * Hl, (L + kCombineThreads - 1) / kCombineThreads),
                          dim3(kCombineThreads), 0, st, (const float *)s->part_o,
                          (const float *)s->part_m, (const float *)s->part_l, nsplit, S, Hl, L,
                          s->attn_tc ? L / 2 : L, s->ctx_xq, head_stride));
        mark(s, "mla_combine");
        // W_UV: rows nope .. nope+v of each head's kv_b block (decode_value, :345-375)
        // nope and value_dim are multiples of 16, so each head's W_UV
        // block starts on a tile boundary of kv_b
        GemvSeg g = seg_of(y.kv_b, s->ctx_xq, EPI_STORE_XQ);
        size_t tb = tile_bytes(df, y.kv_b.kp);
        g.w_stride = (int64_t)((NP + VD) / kTileRows) * (int64_t)tb;
        g.w = kv_b_w + (size_t)(NP / kTileRows) * tb;
        g.O = VD;
        g.count = Hl;
        g.xq_stride = (int64_t)head_stride;
        g.yq = s->o_xq;
        g.kpy = kpO;
        g.col_off = h0 * VD;
        g.out_stride = VD;
        if (s->head_shard) {
            // this rank's heads into its own o_proj input and every peer's
            // (buffer = layer parity), then the epoch is published and the
            // peers' heads awaited (bounded) before o_proj
            const size_t off = s->ep_attn_off + 256 + (size_t)(l & 1) * s->ep_oxq_bytes;
            g.yq = reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(s->ep_region) + off);
            for (int r = 0, k = 0; r < m->world; ++r)
                if (r != m->rank)
                    g.peer_y[k++] = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(s->ep_peer_region[r]) + off);
            g.npeer = m->world - 1;
        }
        // head-parallel: the W_UV launch's last CTA publishes the epoch to
        // the peers, o_proj's producer waits for theirs (bounded)
        GemvWork hand{};
        if (s->head_shard) {
            hand.pub_done = s->ep_adone;
            hand.pub_epoch = s->ep_aepoch;
            for (int r = 0; r < m->world; ++r)
                if (r != m->rank)
                    hand.pub_flags[r] =
                        reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(s->ep_peer_region[r]) + s->ep_attn_off);
            hand.wait_flags = reinterpret_cast<const int *>(reinterpret_cast<uint8_t *>(s->ep_region) + s->ep_attn_off);
            hand.wait_epoch = s->ep_aepoch;
            hand.wait_ns = s->ep_wait_ns;
            hand.peer_world = m->world;
            hand.peer_rank = m->rank;
        }
        GemvWork pub = hand, wait = hand;
        pub.wait_flags = nullptr;
        wait.pub_done = nullptr;
        FC_TRY(gemv1(df, g, S, 0.0f, s->d_err, m->sms, st, s->head_shard ? &pub : nullptr));
        mark(s, "gemv_w_uv");
        o_in = g.yq;
        o_sync = s->head_shard ? wait : GemvWork{};
    }
    {
        GemvSeg g = seg_of(y.o_proj, o_in, o_epi);
        g.y = o_y;
        g.ldy = D;
        FC_TRY(gemv1(df, g, S, 0.0f, s->d_err, m->sms, st, s->head_shard ? &o_sync : nullptr));
        mark(s, "gemv_o_proj");
    }
    return cudaSuccess;
}

// The FFN block of layer l over S rows whose normalized input is in xq_norm
// (xq) and xn (fp32, the router's input): the dense MLP, or router + routed
// and shared experts + combine, added into `out` (the residual in a
// forward).  `routed_only`: the combine leaves out the shared expert (the
// MoE test hook reads the shared output from sh_part).
cudaError_t record_ffn(FcSession *s, int S, int l, const Staging *dst, float *out, int dense_epi,
                       bool routed_only) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size;
    const int mb = s->rows_max;
    const int df = c.dense_format, ef = c.expert_format;
    DevLayer &y = m->layers[l];
    if (y.dense) {
        int kpI = kpad(c.dense_intermediate_size);
        GemvSeg g = seg_of(y.d_gate, s->xq_norm, EPI_SWIGLU_XQ);
        g.w2 = y.d_up.w;
        g.yq = s->hd_xq;
        g.kpy = kpI;
        FC_TRY(gemv1(df, g, S, 0.0f, s->d_err, m->sms, st));
        mark(s, "gemv_dense_gate_up");
        GemvSeg d = seg_of(y.d_down, s->hd_xq, dense_epi);
        d.y = out;
        d.ldy = D;
        FC_TRY(gemv1(df, d, S, 0.0f, s->d_err, m->sms, st));
        mark(s, "gemv_dense_down");
    } else {
        int E = c.expert_count, K = c.experts_per_token;
        RouteParams rp{};
        rp.E = E; rp.K = K; rp.S = S;
        rp.score_fn = c.score_fn;
        rp.normalize = c.normalize_topk;
        rp.routed_scale = c.routed_scale;
        rp.bias = y.bias.p;
        rp.hash = y.hash;
        rp.ids = dst->ids;
        rp.expert_lo = m->expert_lo;
        rp.expert_hi = m->expert_hi;
        rp.route_ids = s->route_ids + (size_t)l * mb * K;
        rp.route_w = s->route_w + (size_t)l * mb * K;
        rp.n_active = s->n_active;
        rp.active = s->active;
        rp.coef = s->coef;
        rp.n_global = s->n_global;
        rp.choice = s->router_logits + (size_t)mb * E;
        rp.n_before = s->n_before;
        rp.arrivals = s->route_arrivals;
        FC_TRY(launch_pdl(router_kernel, dim3(E), dim3(kRouteThreads), 0, st, y.router.p, s->xn, D,
                          s->router_logits, rp));
        mark(s, "router");
        int I = c.moe_intermediate_size, kpI = kpad(I);
        int W = I * c.shared_expert_count, kpW = kpad(std::max(W, 1));
        // gate / up + SwiGLU of the active routed experts and the shared expert
        GemvWork gu{};
        gu.moe = 1;
        gu.seg[0] = seg_of(y.e_gate, s->xq_norm, EPI_SWIGLU_XQ);
        gu.seg[0].w2 = y.e_up.w;
        gu.seg[0].w_stride = (int64_t)y.e_gate.w_bytes;
        gu.seg[0].yq = s->h_xq;
        gu.seg[0].kpy = kpI;
        if (y.s_gate.count) {
            gu.seg[1] = seg_of(y.s_gate, s->xq_norm, EPI_SWIGLU_XQ);
            gu.seg[1].w2 = y.s_up.w;
            gu.seg[1].yq = s->hsh_xq;
            gu.seg[1].kpy = kpW;
        }
        gu.nseg = 2;
        gu.shared_first = y.s_gate.count ? 1 : 0;  // the shared expert overlaps the router
        gu.max_slots = s->max_slots;
        gu.expert_base = m->expert_lo;
        gu.n_active = s->n_active;
        gu.active = s->active;
        gu.in_slot_stride = 0;
        gu.out_slot_stride = (int64_t)mb * kpI * 2;
        gu.S = S;
        gu.swiglu_limit = c.swiglu_limit;
        gu.err = s->d_err;
        FC_TRY(launch_gemv_work(ef, df, gu, m->sms, st));
        mark(s, "moe_gate_up");
        // down projections
        GemvWork dn{};
        dn.moe = 1;
        dn.seg[0] = seg_of(y.e_down, s->h_xq, EPI_STORE);
        dn.seg[0].w_stride = (int64_t)y.e_down.w_bytes;
        dn.seg[0].y = s->moe_part;
        dn.seg[0].ldy = D;
        const bool ep = m->world > 1;
        const int64_t parity_stride = (int64_t)s->g_slots * mb * D;
        if (ep) {
            // routed outputs go to global slot n_before + local slot of
            // the receive buffer of every rank (this one and the peers)
            dn.seg[0].y = s->ep_xbuf;
            for (int r = 0, k = 0; r < m->world; ++r)
                if (r != m->rank) dn.seg[0].peer_y[k++] = reinterpret_cast<float *>(s->ep_peer_region[r]);
            dn.seg[0].npeer = m->world - 1;
            dn.slot_base = s->n_before;
            dn.ep_epoch = s->ep_epoch;
            dn.parity_stride = parity_stride;
        }
        if (y.s_down.count) {
            dn.seg[1] = seg_of(y.s_down, s->hsh_xq, EPI_STORE);
            dn.seg[1].y = s->sh_part;
            dn.seg[1].ldy = D;
        }
        dn.nseg = 2;
        dn.max_slots = s->max_slots;
        dn.expert_base = m->expert_lo;
        dn.n_active = s->n_active;
        dn.active = s->active;
        dn.in_slot_stride = (int64_t)mb * kpI * 2;
        dn.out_slot_stride = (int64_t)mb * D;
        dn.S = S;
        dn.err = s->d_err;
        FC_TRY(launch_gemv_work(ef, df, dn, m->sms, st));
        mark(s, "moe_down");
        EpLink link{};
        link.world = m->world;
        link.rank = m->rank;
        if (ep) {
            link.epoch = s->ep_epoch;
            link.flags = s->ep_flags;
            link.wait_ns = s->ep_wait_ns;
            for (int r = 0; r < m->world; ++r)
                if (r != m->rank)
                    link.peer_flags[r] = reinterpret_cast<int *>(
                        reinterpret_cast<uint8_t *>(s->ep_peer_region[r]) + 2 * parity_stride * sizeof(float));
            FC_TRY(launch_pdl(ep_signal_kernel, dim3(1), dim3(1), 0, st, link));
            mark(s, "ep_signal");
        }
        FC_TRY(launch_pdl(moe_combine_kernel, dim3(S * ((D + kMoeCombineThreads - 1) / kMoeCombineThreads)),
                          dim3(kMoeCombineThreads), 0, st, out, ep ? (const float *)s->ep_xbuf : s->moe_part,
                          (y.s_down.count && !routed_only) ? (const float *)s->sh_part : nullptr,
                          (const float *)s->coef, (const int *)s->n_global, S, D, mb, link, parity_stride,
                          s->d_err));
        mark(s, "moe_combine");
    }
    return cudaSuccess;
}

cudaError_t record_layer(FcSession *s, int S, int l, const Staging *dst) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size, kpD = kpad(D);
    const int mb = s->rows_max;
    DevLayer &y = m->layers[l];
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(S), dim3(norm_threads(D)), 0, st, s->resid, D, y.attn_norm.p, D, c.rms_norm_epsilon,
                                      s->xq_norm, kpD, nullptr, 0));
    mark(s, "rmsnorm");
    FC_TRY(record_attention(s, S, l, dst, EPI_ADD, s->resid));
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(S), dim3(norm_threads(D)), 0, st, s->resid, D, y.ffn_norm.p, D, c.rms_norm_epsilon,
                                      s->xq_norm, kpD, s->xn, D));
    mark(s, "rmsnorm");
    FC_TRY(record_ffn(s, S, l, dst, s->resid, EPI_ADD, false));
    if (s->trace && l < c.layer_count) {
        FC_TRY(cudaMemcpyAsync(s->layer_out + (size_t)l * mb * D, s->resid, (size_t)S * D * 4,
                               cudaMemcpyDeviceToDevice, st));
        mark(s, "layer_trace_copy");
    }

    return cudaSuccess;
}

cudaError_t record_mtp_step(FcSession *s, int i);

cudaError_t record_forward(FcSession *s, int S, int drafts) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size, kpD = kpad(D);

    FC_TRY(cudaMemcpyAsync(s->d_stage, s->h_stage, sizeof(Staging), cudaMemcpyHostToDevice, st));
    FC_TRY(launch_pdl(embed_kernel, embed_grid(S, D), dim3(kEmbedThreads), 0, st, m->embed.fmt, m->embed.w, D, m->embed.kp, s->d_stage->ids,
                                    s->resid));
    FC_TRY(cudaGetLastError());
    mark(s, "embed");
    for (int l = 0; l < c.layer_count; ++l) FC_TRY(record_layer(s, S, l, s->d_stage));
    if (s->hist) {
        FC_TRY(launch_pdl(hist_store_kernel, dim3((D + 255) / 256, S), dim3(256), 0, st, (const float *)s->resid,
                          (const Staging *)s->d_stage, s->hist, D));
        mark(s, "hist_store");
    }
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(S), dim3(norm_threads(D)), 0, st, s->resid, D, m->final_norm.p, D, c.rms_norm_epsilon,
                                      s->xq_norm, kpD, nullptr, 0));
    mark(s, "rmsnorm");
    FC_TRY(head_gemv(m, s->xq_norm, S, s->logits, s->d_err, st));
    mark(s, "gemv_lm_head");
    {
        dim3 grid(s->head_chunks, S);
        FC_TRY(launch_pdl(head_partial_kernel, dim3(grid), dim3(256), 0, st, s->logits, c.vocab_size, s->d_stage, s->hp,
                                                  s->head_chunks));
        mark(s, "head_partial");
        FC_TRY(launch_pdl(accept_kernel, dim3(1), dim3(256), 0, st, s->logits, c.vocab_size, s->d_stage, s->hp, s->head_chunks,
                                         s->d_res, s->d_err));
        mark(s, "accept");
    }
    for (int i = 0; i < drafts; ++i) FC_TRY(record_mtp_step(s, i));
    FC_TRY(cudaGetLastError());
    FC_TRY(cudaMemcpyAsync(s->h_res, s->d_res, sizeof(Result), cudaMemcpyDeviceToHost, st));
    return cudaSuccess;
}

// One greedy step of the MTP drafter (S = 1): embed the input token,
// h_in = eh_proj([enorm(embed) | hnorm(h)]), the MTP layer over its own latent
// cache, shared_head.norm, the shared lm-head, argmax -> proposal i.
cudaError_t record_mtp_step(FcSession *s, int i) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size, kpD = kpad(D), kp2 = kpad(2 * D), df = c.dense_format;
    const int lm = c.layer_count;  // the MTP layer
    DevLayer &y = m->layers[lm];
    FC_TRY(launch_pdl(mtp_prep_kernel, dim3((D + 255) / 256), dim3(256), 0, st, i, (const Staging *)s->d_stage,
                      (const Result *)s->d_res, s->d_mtp, (const float *)s->resid, s->mtp_h, D));
    mark(s, "mtp_prep");
    FC_TRY(launch_pdl(embed_kernel, embed_grid(1, D), dim3(kEmbedThreads), 0, st, m->embed.fmt, m->embed.w, D, m->embed.kp,
                      (const int *)s->d_mtp->ids, s->resid));
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(1), dim3(norm_threads(D)), 0, st, (const float *)s->resid, D,
                      (const float *)y.enorm.p, D, c.rms_norm_epsilon, s->mtp_xq, kp2, (float *)nullptr, 0));
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(1), dim3(norm_threads(D)), 0, st, (const float *)s->mtp_h, D,
                      (const float *)y.hnorm.p, D, c.rms_norm_epsilon, s->mtp_xq + (size_t)D * 2, kp2,
                      (float *)nullptr, 0));
    {
        GemvSeg g = seg_of(y.eh_proj, s->mtp_xq, EPI_STORE);
        g.y = s->resid;
        g.ldy = D;
        FC_TRY(gemv1(df, g, 1, 0.0f, s->d_err, m->sms, st));
    }
    mark(s, "mtp_input");
    FC_TRY(record_layer(s, 1, lm, s->d_mtp));
    FC_TRY(cudaMemcpyAsync(s->mtp_h, s->resid, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(1), dim3(norm_threads(D)), 0, st, (const float *)s->resid, D,
                      (const float *)y.head_norm.p, D, c.rms_norm_epsilon, s->xq_norm, kpD, (float *)nullptr, 0));
    FC_TRY(head_gemv(m, s->xq_norm, 1, s->mtp_logits, s->d_err, st));
    FC_TRY(launch_pdl(head_partial_kernel, dim3(s->head_chunks, 1), dim3(256), 0, st, (const float *)s->mtp_logits,
                      c.vocab_size, (const Staging *)s->d_mtp, s->hp, s->head_chunks));
    FC_TRY(launch_pdl(mtp_pick_kernel, dim3(1), dim3(32), 0, st, s->hp, s->head_chunks, s->d_res, s->d_mtp, i));
    mark(s, "mtp_head");
    return cudaGetLastError();
}

// Every kernel of the forward asks for the same (maximum) shared-memory
// carveout, so consecutive kernels never make an SM reconfigure its L1 split.
cudaError_t prefer_shared_carveout() {
    const void *kernels[] = {
        (const void *)embed_kernel, (const void *)rmsnorm_kernel, (const void *)mla_prep_absorb_kernel,
        (const void *)mla_attention_kernel<512, 64>,
        (const void *)mla_attention_kernel<256, 64>, (const void *)mla_combine_kernel,
        (const void *)mla_attention_tc_kernel<512>, (const void *)mla_attention_tc_kernel<256>,
        (const void *)router_kernel,
        (const void *)moe_combine_kernel, (const void *)head_partial_kernel,
        (const void *)accept_kernel, (const void *)mtp_prep_kernel, (const void *)mtp_pick_kernel,
#define FC_GEMV_PTR(A, B) (const void *)gemv_kernel<A, B>,
        FC_GEMV_FORMATS(FC_GEMV_PTR)
#undef FC_GEMV_PTR
    };
    for (const void *k : kernels) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaGraphExec_t get_graph(FcSession *s, int S, int drafts, char *err, size_t n) {
    int key = (S * 2 + (s->trace ? 1 : 0)) * 16 + drafts;
    auto it = s->graphs.find(key);
    if (it != s->graphs.end()) return it->second;
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        set_error(err, n, "cudaStreamBeginCapture failed");
        return nullptr;
    }
    cudaError_t rec = record_forward(s, S, drafts);
    cudaError_t end = cudaStreamEndCapture(s->stream, &graph);
    if (rec != cudaSuccess || end != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        set_error(err, n, "recording the forward graph failed: %s",
                  cudaGetErrorString(rec != cudaSuccess ? rec : end));
        return nullptr;
    }
    size_t nodes = 0;
    int kernels = 0;
    if (cudaGraphGetNodes(graph, nullptr, &nodes) == cudaSuccess && nodes) {
        std::vector<cudaGraphNode_t> list(nodes);
        if (cudaGraphGetNodes(graph, list.data(), &nodes) == cudaSuccess)
            for (auto nd : list) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
            }
    }
    s->graph_kernels[key] = kernels;
    cudaGraphExec_t exec = nullptr;
    cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
        set_error(err, n, "cudaGraphInstantiate failed: %s", cudaGetErrorString(inst));
        return nullptr;
    }
    s->graphs[key] = exec;
    return exec;
}

// Adds the event intervals of the last eager pass to the per-name profile.
void collect_profile(FcSession *s) {
    for (size_t i = 0; i < s->prof_marks.size(); ++i) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, s->prof_events[i], s->prof_events[i + 1]);
        bool found = false;
        for (auto &p : s->prof)
            if (p.first == s->prof_marks[i]) {
                p.second.first += ms;
                p.second.second++;
                found = true;
                break;
            }
        if (!found) s->prof.push_back({s->prof_marks[i], {ms, 1}});
    }
}

// Runs one forward pass of `rows` <= rows_max tokens at the session position.
int exec_pass(FcSession *s, int rows, int drafts, char *err, size_t n);

int run_pass(FcSession *s, const int *ids, int rows, int k, const FcAcceptConfig *accept,
             char *err, size_t n) {
    if (s->m->world > 1 && !s->ep_connected)
        return set_error(err, n, "expert-parallel session is not connected (fc_session_ep_connect)");
    Staging *st = s->h_stage;
    memset(st, 0, sizeof(*st));
    st->pos = s->position;
    st->rows = rows;
    st->k = k;
    st->mode = accept ? accept->mode : FC_ACCEPT_GREEDY;
    st->temperature = accept ? accept->temperature : 1.0f;
    st->seed = accept ? accept->seed : 0;
    st->counter = accept ? accept->counter : 0;
    for (int i = 0; i < rows; ++i) {
        st->ids[i] = ids[i];
        st->rowpos[i] = s->position + i;
        st->rowseq[i] = 0;
        if (!s->tok_hist.empty()) s->tok_hist[s->position + i] = ids[i];
    }
    st->group_rows = rows;
    st->groups = 1;
    st->gcounter[0] = st->counter;
    // the drafter runs after a verify (k > 0) of a model with an MTP layer
    const int drafts = (s->m->c.mtp_layers > 0 && k > 0) ? k : 0;
    return exec_pass(s, rows, drafts, err, n);
}

// Launches the captured graph of the pass staged in h_stage on the
// session's stream, without waiting for it.
int launch_pass(FcSession *s, int rows, int drafts, char *err, size_t n) {
    cudaGraphExec_t g = get_graph(s, rows, drafts, err, n);
    if (!g) return 0;
    s->last_kernels = s->graph_kernels[(rows * 2 + (s->trace ? 1 : 0)) * 16 + drafts];
    cudaError_t e = cudaGraphLaunch(g, s->stream);
    if (e != cudaSuccess) return set_error(err, n, "CUDA forward failed: %s", cudaGetErrorString(e));
    s->stats.graph_replays++;
    return 1;
}

// After a launched pass has completed: its kernels' error word.
int finish_pass(FcSession *s, int rows, int drafts, char *err, size_t n) {
    if (s->h_res->error) {
        // a kernel that gave up may have left the router counter mid-count
        cudaMemsetAsync(s->route_arrivals, 0, sizeof(int), s->stream);
        cudaStreamSynchronize(s->stream);
        return set_error(err, n, "a kernel wait gave up (error bits 0x%x); results are invalid",
                         s->h_res->error);
    }
    s->stats.command_buffers++;
    s->last_rows = rows;
    s->last_drafts = drafts;
    return 1;
}

// Runs the pass whose parameters are in h_stage: the captured graph for
// (rows, drafts), or an eager profiled pass.
int exec_pass(FcSession *s, int rows, int drafts, char *err, size_t n) {
    cudaSetDevice(s->m->device);
    s->route_trace_rows = 0;
    cudaError_t e;
    if (s->profiling) {
        // eager pass with an event after every kernel (MOONLIGHT_PROFILE-style
        // per-phase timing, moonlight_metal.m:1899-1979)
        s->prof_marks.clear();
        cudaEventRecord(s->prof_events[0], s->stream);
        e = record_forward(s, rows, drafts);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
        if (e == cudaSuccess) collect_profile(s);
    } else {
        cudaGraphExec_t g = get_graph(s, rows, drafts, err, n);
        if (!g) return 0;
        s->last_kernels = s->graph_kernels[(rows * 2 + (s->trace ? 1 : 0)) * 16 + drafts];
        cudaEventRecord(s->ev_begin, s->stream);
        e = cudaGraphLaunch(g, s->stream);
        cudaEventRecord(s->ev_end, s->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
        if (e == cudaSuccess) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, s->ev_begin, s->ev_end);
            s->stats.gpu_ms += ms;
        }
        s->stats.graph_replays++;
    }
    if (e != cudaSuccess) return set_error(err, n, "CUDA forward failed: %s", cudaGetErrorString(e));
    if (!s->profiling && s->h_res->error) {
        // a kernel that gave up may have left the router counter mid-count
        cudaMemsetAsync(s->route_arrivals, 0, sizeof(int), s->stream);
        cudaStreamSynchronize(s->stream);
        return set_error(err, n, "a kernel wait gave up (error bits 0x%x); results are invalid",
                         s->h_res->error);
    }
    s->stats.command_buffers++;
    s->last_rows = rows;
    s->last_drafts = drafts;
    return 1;
}

// ---------------------------------------------------------------------------
// prefill chunks on the tensor cores
// ---------------------------------------------------------------------------
#define FC_PF_VARIANTS(X, F) \
    X(F, kPfBN, PF_STORE_F32) X(F, kPfBN, PF_STORE_F16) X(F, kPfBN, PF_ADD_F32) X(F, kPfBN, PF_SWIGLU_F16)
#define FC_PF_ALL(X) FC_PF_VARIANTS(X, FC_FMT_Q8) FC_PF_VARIANTS(X, FC_FMT_Q4) FC_PF_VARIANTS(X, FC_FMT_MXFP4)

cudaError_t pf_prepare_all() {
#define FC_PF_ATTR(F, BN, EPI)                                                                       \
    {                                                                                                \
        cudaError_t e_ = cudaFuncSetAttribute(pf_gemm_kernel<F, BN, EPI>,                            \
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                                              (int)PfPlan<BN>::SMEM);                                \
        if (e_ != cudaSuccess) return e_;                                                            \
    }
    FC_PF_ALL(FC_PF_ATTR)
#undef FC_PF_ATTR
#define FC_FA_ATTR(A, B)                                                                              \
    {                                                                                                \
        cudaError_t e_ = cudaFuncSetAttribute(pf_attention_kernel<A, B>,                              \
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                                              (int)FaPlan<A, B>::SMEM);                              \
        if (e_ != cudaSuccess) return e_;                                                            \
    }
    FC_FA_ATTR(2, 1) FC_FA_ATTR(2, 2) FC_FA_ATTR(3, 1) FC_FA_ATTR(3, 2)
#undef FC_FA_ATTR
    return cudaSuccess;
}

// One tcgen05 GEMM launch (one CTA per SM) of weight format `fmt`.
cudaError_t pf_gemm(int fmt, int epi, const CUtensorMap &map, const CUtensorMap &wmap, const CUtensorMap &wmap2,
                    const PfGemm &p, int sms, cudaStream_t st) {
    constexpr int bn = kPfBN;
#define FC_PF_CASE(F, BN, EPI)                                                                       \
    if (fmt == F && bn == BN && epi == EPI)                                                          \
        return launch_pdl(pf_gemm_kernel<F, BN, EPI>, dim3(sms), dim3(kPfThreads), PfPlan<BN>::SMEM, st, map, \
                          wmap, wmap2, p);
    FC_PF_ALL(FC_PF_CASE)
#undef FC_PF_CASE
    return cudaErrorInvalidValue;
}

// The weight tensor map of a matrix family for boxes of box_tiles tiles
// (cached per session; the weights never move).
const CUtensorMap *pf_wmap(FcSession *s, const DevMat &mm, int box_tiles) {
    auto key = std::make_pair((const void *)mm.w, box_tiles);
    auto it = s->pf_wmaps.find(key);
    if (it != s->pf_wmaps.end()) return &it->second;
    CUtensorMap map{};
    const uint64_t tiles = (uint64_t)std::max(mm.count, 1) * (uint64_t)((mm.O + kTileRows - 1) / kTileRows);
    if (!make_map_weights(&map, mm.w, mm.fmt, tiles, mm.kp, (uint32_t)box_tiles)) return nullptr;
    return &(s->pf_wmaps[key] = map);
}

// Launches the prefill GEMM of matrix `w` (and the up rows `w2` for SwiGLU).
cudaError_t pf_gemm_w(FcSession *s, int epi, const CUtensorMap &amap, const DevMat &w, const DevMat *w2,
                      PfGemm p) {
    // a box never exceeds the tensor (such a copy would not complete)
    const int tiles = std::max(w.count, 1) * ((w.O + kTileRows - 1) / kTileRows);
    const int box = std::min(epi == PF_SWIGLU_F16 ? kPfBN / 32 : kPfBN / 16, tiles);
    p.box_tiles = box;
    const CUtensorMap *m1 = pf_wmap(s, w, box);
    const CUtensorMap *m2 = w2 ? pf_wmap(s, *w2, box) : m1;
    if (!m1 || !m2) return cudaErrorInvalidValue;
    return pf_gemm(w.fmt, epi, amap, *m1, *m2, p, s->m->sms, s->stream);
}

// A GEMM of matrix `mm` over `rows` rows of the A map.
PfGemm pf_plain(FcSession *s, const DevMat &mm, int rows, void *out, int64_t out_ld) {
    PfGemm p{};
    p.tiles_per_group = (mm.O + kTileRows - 1) / kTileRows;
    p.kp = mm.kp;
    p.N = mm.O;
    p.K = mm.kp;
    p.groups = 1;
    p.rows = rows;
    p.out = out;
    p.out_ld = out_ld;
    p.err = s->d_err;
    return p;
}

// Enqueues the forward of T (<= pf_rows) tokens at position pf_ids[0]:
// every layer over the whole chunk, then the final norm and lm-head of the
// last row into logits row 0.
cudaError_t record_prefill(FcSession *s, int T) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size, H = c.head_count, L = c.kv_lora_rank, R = c.qk_rope_dim;
    const int NP = c.qk_nope_dim, VD = c.value_dim, QW = NP + R;
    const int sms = m->sms;
    const float scale = 1.0f / sqrtf((float)(NP + R));
    const int *d_pos = s->pf_ids, *ids = s->pf_ids + 1;
    FC_TRY(launch_pdl(embed_kernel, embed_grid(T, D), dim3(kEmbedThreads), 0, st, m->embed.fmt, (const uint8_t *)m->embed.w, D,
                      m->embed.kp, ids, s->pf_resid));
    mark(s, "pf_embed");
    for (int l = 0; l < c.layer_count; ++l) {
        DevLayer &y = m->layers[l];
        __half *cache = s->cache + (size_t)l * s->opt.context_size * (L + R);
        FC_TRY(launch_pdl(pf_rmsnorm_kernel, dim3(T), dim3(256), 0, st, (const float *)s->pf_resid, D,
                          (const float *)y.attn_norm.p, c.rms_norm_epsilon, s->pf_x16, D, (float *)nullptr));
        mark(s, "pf_rmsnorm");
        if (c.q_lora_rank > 0) {
            PfGemm a = pf_plain(s, y.q_a, T, s->pf_qa, c.q_lora_rank);
            FC_TRY(pf_gemm_w(s, PF_STORE_F32, s->pf_map_x, y.q_a, nullptr, a));
            FC_TRY(launch_pdl(pf_rmsnorm_kernel, dim3(T), dim3(256), 0, st, (const float *)s->pf_qa, c.q_lora_rank,
                              (const float *)y.q_a_norm.p, c.rms_norm_epsilon, s->pf_qa16, c.q_lora_rank,
                              (float *)nullptr));
            PfGemm b = pf_plain(s, y.q_b, T, s->pf_q16, H * QW);
            FC_TRY(pf_gemm_w(s, PF_STORE_F16, s->pf_map_qa, y.q_b, nullptr, b));
        } else {
            PfGemm a = pf_plain(s, y.q_proj, T, s->pf_q16, H * QW);
            FC_TRY(pf_gemm_w(s, PF_STORE_F16, s->pf_map_x, y.q_proj, nullptr, a));
        }
        mark(s, "pf_gemm_q");
        {
            PfGemm a = pf_plain(s, y.kv_a, T, s->pf_ckv, L + R);
            FC_TRY(pf_gemm_w(s, PF_STORE_F32, s->pf_map_x, y.kv_a, nullptr, a));
            mark(s, "pf_gemm_kv_a");
        }
        FC_TRY(launch_pdl(pf_prep_kernel, dim3(T, 1 + (H * (R / 2) + 255) / 256), dim3(256), 0, st,
                          (const float *)s->pf_ckv, s->pf_q16, (const float *)y.kv_a_norm.p, L, R, H, NP,
                          c.rms_norm_epsilon, c.rope_theta, d_pos, cache));
        mark(s, "pf_prep");
        {
            // keys and values of every visible position: kvd[k][h*(nope+v) + j]
            // = cache_latent[k] . kv_b[h*(nope+v) + j]  (W_UK rows, then W_UV)
            PfGemm a = pf_plain(s, y.kv_b, s->position + T, s->pf_kvd, (int64_t)H * (NP + VD));
            a.a_y0 = l * s->opt.context_size;
            FC_TRY(pf_gemm_w(s, PF_STORE_F16, s->pf_cmap, y.kv_b, nullptr, a));
            mark(s, "pf_gemm_kv_b");
        }
        {
            dim3 grid((T + kFaRows - 1) / kFaRows, H);
            const int nqs = NP / 64 + 1, nvs = VD / 64;
#define FC_FA_LAUNCH(A, B)                                                                                        \
    if (nqs == A && nvs == B)                                                                                     \
        FC_TRY(launch_pdl(pf_attention_kernel<A, B>, grid, dim3(kFaThreads), FaPlan<A, B>::SMEM, st, s->pf_map_q, \
                          s->pf_map_kvd, s->pf_cmap64, l * s->opt.context_size, L, T, H, d_pos, scale, s->pf_o16, \
                          s->d_err));
            FC_FA_LAUNCH(2, 1) FC_FA_LAUNCH(2, 2) FC_FA_LAUNCH(3, 1) FC_FA_LAUNCH(3, 2)
#undef FC_FA_LAUNCH
            mark(s, "pf_attention");
        }
        {
            PfGemm a = pf_plain(s, y.o_proj, T, s->pf_resid, D);
            FC_TRY(pf_gemm_w(s, PF_ADD_F32, s->pf_map_o, y.o_proj, nullptr, a));
            mark(s, "pf_gemm_o_proj");
        }
        FC_TRY(launch_pdl(pf_rmsnorm_kernel, dim3(T), dim3(256), 0, st, (const float *)s->pf_resid, D,
                          (const float *)y.ffn_norm.p, c.rms_norm_epsilon, s->pf_x16, D, s->pf_xn));
        mark(s, "pf_rmsnorm");
        if (y.dense) {
            const int I = c.dense_intermediate_size;
            PfGemm a = pf_plain(s, y.d_gate, T, s->pf_h16, I);
            FC_TRY(pf_gemm_w(s, PF_SWIGLU_F16, s->pf_map_x, y.d_gate, &y.d_up, a));
            mark(s, "pf_gemm_dense_gate_up");
            PfGemm b = pf_plain(s, y.d_down, T, s->pf_resid, D);
            FC_TRY(pf_gemm_w(s, PF_ADD_F32, s->pf_map_hd, y.d_down, nullptr, b));
            mark(s, "pf_gemm_dense_down");
            continue;
        }
        const int E = c.expert_count, K = c.experts_per_token, I = c.moe_intermediate_size;
        // k splits: at least ~2 tiles per SM, 32-column multiples
        const int tiles = ((T + kPfRtTile - 1) / kPfRtTile) * ((E + kPfRtTile - 1) / kPfRtTile);
        int nsplit = std::min(kPfRtMaxSplits, std::max(1, (2 * sms + tiles - 1) / tiles));
        const int ksplit = ((D + nsplit - 1) / nsplit + kPfRtK - 1) / kPfRtK * kPfRtK;
        nsplit = (D + ksplit - 1) / ksplit;
        FC_TRY(launch_pdl(pf_router_logits_kernel,
                          dim3((T + kPfRtTile - 1) / kPfRtTile, (E + kPfRtTile - 1) / kPfRtTile, nsplit), dim3(256),
                          0, st, (const float *)y.router.p, (const float *)s->pf_xn, T, D, E, ksplit, s->pf_rpart));
        mark(s, "pf_router");
        RouteParams rp{};
        rp.E = E; rp.K = K; rp.S = T;
        rp.score_fn = c.score_fn;
        rp.normalize = c.normalize_topk;
        rp.routed_scale = c.routed_scale;
        rp.bias = y.bias.p;
        rp.hash = y.hash;
        rp.ids = ids;
        rp.route_ids = s->pf_route_ids;
        rp.route_w = s->pf_route_w;
        rp.choice = s->pf_choice;
        FC_TRY(launch_pdl(pf_route_kernel, dim3((T + kPfRouteWarps - 1) / kPfRouteWarps), dim3(32 * kPfRouteWarps), 0,
                          st, (const float *)s->pf_rpart, nsplit, s->pf_logits, rp, s->pf_counts));
        FC_TRY(launch_pdl(pf_group_kernel, dim3(1), dim3(1024), 0, st, s->pf_counts, E, s->pf_offsets, s->pf_cursor,
                          s->pf_mt_table, s->pf_mt_count));
        FC_TRY(launch_pdl(pf_gather_kernel, dim3((T * K + 7) / 8), dim3(256), 0, st, (const int *)s->pf_route_ids, T, K,
                          s->pf_cursor, s->pf_slot_of, (const __half *)s->pf_x16, D, s->pf_xg));
        mark(s, "pf_route_group");
        {
            PfGemm a = pf_plain(s, y.e_gate, 0, s->pf_hg, I);
            a.mt_count = s->pf_mt_count;
            a.mt_table = s->pf_mt_table;
            a.limit = c.swiglu_limit;
            FC_TRY(pf_gemm_w(s, PF_SWIGLU_F16, s->pf_map_xg, y.e_gate, &y.e_up, a));
            mark(s, "pf_gemm_moe_gate_up");
            PfGemm b = pf_plain(s, y.e_down, 0, s->pf_yd, D);
            b.mt_count = s->pf_mt_count;
            b.mt_table = s->pf_mt_table;
            FC_TRY(pf_gemm_w(s, PF_STORE_F32, s->pf_map_hg, y.e_down, nullptr, b));
            mark(s, "pf_gemm_moe_down");
        }
        if (y.s_gate.count) {
            const int W = I * c.shared_expert_count;
            PfGemm a = pf_plain(s, y.s_gate, T, s->pf_h16, W);
            a.limit = c.swiglu_limit;
            FC_TRY(pf_gemm_w(s, PF_SWIGLU_F16, s->pf_map_x, y.s_gate, &y.s_up, a));
            PfGemm b = pf_plain(s, y.s_down, T, s->pf_sh, D);
            FC_TRY(pf_gemm_w(s, PF_STORE_F32, s->pf_map_hs, y.s_down, nullptr, b));
            mark(s, "pf_gemm_shared");
        }
        FC_TRY(launch_pdl(pf_combine_kernel, dim3(T), dim3(256), 0, st, s->pf_resid, (const float *)s->pf_yd,
                          y.s_gate.count ? (const float *)s->pf_sh : (const float *)nullptr,
                          (const int *)s->pf_route_ids, (const float *)s->pf_route_w, (const int *)s->pf_slot_of, K, D));
        mark(s, "pf_moe_combine");
    }
    if (s->hist) {
        FC_TRY(launch_pdl(hist_store_rows_kernel, dim3((D + 255) / 256, T), dim3(256), 0, st,
                          (const float *)s->pf_resid, (const int *)s->pf_ids, T, s->hist, D));
        mark(s, "hist_store");
    }
    // final norm + lm-head of the last row (a one-row GEMV)
    const int kpD = kpad(D);
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(1), dim3(norm_threads(D)), 0, st, (const float *)(s->pf_resid + (size_t)(T - 1) * D),
                      D, (const float *)m->final_norm.p, D, c.rms_norm_epsilon, s->xq_norm, kpD, (float *)nullptr, 0));
    FC_TRY(head_gemv(m, s->xq_norm, 1, s->logits, s->d_err, st));
    mark(s, "pf_lm_head");
    return cudaGetLastError();
}

// Runs T tokens (rows_max < T <= pf_rows) through the prefill path.
int run_prefill_chunk(FcSession *s, const int *ids, int T, char *err, size_t n) {
    cudaSetDevice(s->m->device);
    s->pf_h_ids[0] = s->position;
    memcpy(s->pf_h_ids + 1, ids, (size_t)T * sizeof(int));
    if (!s->tok_hist.empty()) memcpy(&s->tok_hist[s->position], ids, (size_t)T * sizeof(int));
    cudaError_t e = cudaMemcpyAsync(s->pf_ids, s->pf_h_ids, (size_t)(T + 1) * sizeof(int), cudaMemcpyHostToDevice,
                                    s->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->d_err, 0, sizeof(int), s->stream);
    if (e == cudaSuccess) e = cudaEventRecord(s->ev_begin, s->stream);
    if (s->profiling) {
        s->prof_marks.clear();
        cudaEventRecord(s->prof_events[0], s->stream);
    }
    if (e == cudaSuccess) e = record_prefill(s, T);
    if (e == cudaSuccess) e = cudaEventRecord(s->ev_end, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return set_error(err, n, "CUDA prefill failed: %s", cudaGetErrorString(e));
    if (s->profiling) collect_profile(s);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, s->ev_begin, s->ev_end);
    s->stats.gpu_ms += ms;
    s->stats.command_buffers++;
    int herr = 0;
    cudaMemcpy(&herr, s->d_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (herr) return set_error(err, n, "a kernel wait gave up (error bits 0x%x); results are invalid", herr);
    s->last_rows = 1;
    s->last_drafts = 0;
    return 1;
}

// Synthetic latent KV (synth_kv_kernel's values, by logical position) for
// positions [start, end) of sequence `seq`, written through the page table.
__global__ void synth_kv_range_kernel(__half *cache, PageMap pm, int seq, int start, int end, int L, int R,
                                      uint64_t seed, uint32_t tid_latent, uint32_t tid_rope) {
    const size_t total = (size_t)(end - start) * (L + R);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t p = (size_t)start + i / (L + R);
        const int c = (int)(i % (L + R));
        const float v = c < L ? fc_synth_kv(seed, tid_latent, p * L + c) : fc_synth_kv(seed, tid_rope, p * R + (c - L));
        cache[(size_t)kv_row(pm, seq, (int)p) * (L + R) + c] = __float2half_rn(v);
    }
}

// Stages one device pass of the batch verify in s->h_stage: sequences
// seqs[0 .. ng) at positions seq_pos[...] with their rows
// ids[j * group_rows ..]; no drafter.
void stage_batch_pass(FcSession *s, const std::vector<int> &seq_pos, const int *seqs, int ng, const int *ids,
                      int k, const FcAcceptConfig *accept) {
    const int gr = s->group_rows, rows = ng * gr;
    Staging *st = s->h_stage;
    memset(st, 0, sizeof(*st));
    const FcAcceptConfig *a0 = accept ? &accept[seqs[0]] : nullptr;
    st->pos = seq_pos[seqs[0]];
    st->rows = rows;
    st->k = k;
    st->mode = a0 ? a0->mode : FC_ACCEPT_GREEDY;
    st->temperature = a0 ? a0->temperature : 1.0f;
    st->seed = a0 ? a0->seed : 0;
    st->group_rows = gr;
    st->groups = ng;
    for (int j = 0; j < ng; ++j) {
        const int q = seqs[j];
        st->gcounter[j] = accept ? accept[q].counter : 0;
        for (int i = 0; i < gr; ++i) {
            st->ids[j * gr + i] = ids[j * gr + i];
            st->rowpos[j * gr + i] = seq_pos[q] + i;
            st->rowseq[j * gr + i] = q;
        }
    }
    st->counter = st->gcounter[0];
}

// One device pass of the batch verify (see stage_batch_pass), run to completion.
int run_batch_pass(FcSession *s, const int *seqs, int ng, const int *ids, int k, const FcAcceptConfig *accept,
                   char *err, size_t n) {
    if (s->m->world > 1 && !s->ep_connected)
        return set_error(err, n, "expert-parallel session is not connected (fc_session_ep_connect)");
    stage_batch_pass(s, s->seq_pos, seqs, ng, ids, k, accept);
    return exec_pass(s, ng * s->group_rows, 0, err, n);
}

int check_ids(const FcSession *s, const int *ids, int count, char *err, size_t n) {
    for (int i = 0; i < count; ++i)
        if (ids[i] < 0 || ids[i] >= s->m->c.vocab_size)
            return set_error(err, n, "token id %d out of range", ids[i]);
    return 1;
}

// prefill / append body: chunks of rows_max, logits of the last row.
int run_tokens(FcSession *s, const int *ids, int count, float *last_logits, char *err, size_t n) {
    if (!check_ids(s, ids, count, err, n)) return 0;
    int done = 0;
    while (done < count) {
        if (s->pf_rows && count - done > s->rows_max) {
            const int rows = std::min(s->pf_rows, count - done);
            if (!run_prefill_chunk(s, ids + done, rows, err, n)) return 0;
            s->position += rows;
            done += rows;
            continue;
        }
        int rows = std::min(s->rows_max, count - done);
        if (!run_pass(s, ids + done, rows, -1, nullptr, err, n)) return 0;
        s->position += rows;
        done += rows;
    }
    if (last_logits) {
        int V = s->m->c.vocab_size;
        cudaError_t e = cudaMemcpy(last_logits, s->logits + (size_t)(s->last_rows - 1) * V,
                                   (size_t)V * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return set_error(err, n, "logits copy failed: %s", cudaGetErrorString(e));
    }
    return 1;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int fc_model_create(FcModel **out, const FcModelConfig *config, int device, char *error,
                    size_t error_size) {
    if (!out) return set_error(error, error_size, "model output is required");
    *out = nullptr;
    if (!config) return set_error(error, error_size, "config is required");
    if (!config_ok(config, error, error_size)) return 0;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0)
        return set_error(error, error_size, "no CUDA device is available");
    if (device < 0 || device >= count) return set_error(error, error_size, "invalid device %d", device);
    if (cudaSetDevice(device) != cudaSuccess)
        return set_error(error, error_size, "cannot select CUDA device %d", device);
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major < 10)
        return set_error(error, error_size, "device %s is sm_%d%d; this backend is built for sm_100a",
                         prop.name, prop.major, prop.minor);
    FcModel *m = new FcModel();
    m->c = *config;
    m->device = device;
    m->device_name = prop.name;
    m->sms = prop.multiProcessorCount;
    m->expert_lo = 0;
    m->expert_hi = config->expert_count;
    if (!build_model(m, error, error_size)) {
        fc_model_close(m);
        return 0;
    }
    *out = m;
    return 1;
}

int fc_model_create_ep(FcModel **out, const FcModelConfig *config, int device, int rank,
                       int world, char *error, size_t error_size) {
    if (!out) return set_error(error, error_size, "model output is required");
    *out = nullptr;
    if (!config || world <= 0 || world > kMaxRanks || rank < 0 || rank >= world ||
        (config->expert_count > 0 && config->expert_count % world))
        return set_error(error, error_size, "invalid expert-parallel layout");
    if (!config_ok(config, error, error_size)) return 0;
    if (cudaSetDevice(device) != cudaSuccess)
        return set_error(error, error_size, "cannot select CUDA device %d", device);
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    FcModel *m = new FcModel();
    m->c = *config;
    m->device = device;
    m->device_name = prop.name;
    m->sms = prop.multiProcessorCount;
    int per = config->expert_count / world;
    m->expert_lo = rank * per;
    m->expert_hi = rank * per + per;
    m->rank = rank;
    m->world = world;
    if (!build_model(m, error, error_size)) {
        fc_model_close(m);
        return 0;
    }
    *out = m;
    return 1;
}

int fc_model_fill_synthetic(FcModel *m, uint64_t seed, char *error, size_t error_size) {
    if (!m) return set_error(error, error_size, "model is required");
    cudaSetDevice(m->device);
    cudaStream_t st = nullptr;
    cudaError_t e = cudaSuccess;
    for_each_tensor(m, [&](DevMat *mm, DevVec *v) {
        if (e != cudaSuccess) return;
        if (mm) e = fill_mat(*mm, seed, st);
        if (v && v->n) {
            synth_f32_kernel<<<grid_for(v->n), 256, 0, st>>>(v->p, v->n, v->kind, seed, v->tid);
            e = cudaGetLastError();
        }
    });
    for (auto &y : m->layers)
        if (y.hash && e == cudaSuccess) {
            size_t cnt = (size_t)m->c.vocab_size * m->c.experts_per_token;
            synth_hash_kernel<<<grid_for(cnt), 256, 0, st>>>(y.hash, m->c.vocab_size,
                                                            m->c.experts_per_token,
                                                            m->c.expert_count, seed, y.hash_tid);
            e = cudaGetLastError();
        }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess)
        return set_error(error, error_size, "synthetic fill failed: %s", cudaGetErrorString(e));
    return 1;
}

static int tensor_io(const FcModel *m, const char *name, void *data, size_t bytes, bool upload,
                     char *error, size_t error_size) {
    if (!m || !name || !data) return set_error(error, error_size, "model, name and data are required");
    std::string key(name);
    bool scales = false;
    if (key.size() > 3 && key.compare(key.size() - 3, 3, ".gs") == 0) {
        scales = true;
        key.resize(key.size() - 3);
    }
    auto it = m->names.find(key);
    if (it == m->names.end()) return set_error(error, error_size, "unknown tensor %s", name);
    const TensorRef &r = it->second;
    cudaSetDevice(m->device);
    if (r.vec || r.ints) {
        if (scales) return set_error(error, error_size, "tensor %s has no group scales", key.c_str());
        size_t need = r.vec ? r.vec->n * 4 : r.ints_n * 4;
        void *dev = r.vec ? (void *)r.vec->p : (void *)r.ints;
        if (bytes != need)
            return set_error(error, error_size, "%s: expected %zu bytes, got %zu", name, need, bytes);
        cudaError_t e = upload ? cudaMemcpy(dev, data, need, cudaMemcpyHostToDevice)
                               : cudaMemcpy(data, dev, need, cudaMemcpyDeviceToHost);
        return e == cudaSuccess ? 1 : set_error(error, error_size, "copy failed: %s", cudaGetErrorString(e));
    }
    const DevMat &mm = *r.mat;
    uint8_t *base = mm.w + (size_t)r.member * mm.w_bytes;
    if (mm.fmt == FC_FMT_F32) {
        if (scales) return set_error(error, error_size, "tensor %s has no group scales", key.c_str());
        size_t need = (size_t)mm.O * mm.K * 4;
        if (bytes != need)
            return set_error(error, error_size, "%s: expected %zu bytes, got %zu", name, need, bytes);
        cudaError_t e = upload ? cudaMemcpy(base, data, need, cudaMemcpyHostToDevice)
                               : cudaMemcpy(data, base, need, cudaMemcpyDeviceToHost);
        return e == cudaSuccess ? 1 : set_error(error, error_size, "copy failed");
    }
    size_t need = scales ? (size_t)mm.O * (mm.K / 32) * scale_elem_bytes(mm.fmt)
                  : mm.fmt == FC_FMT_Q8 ? (size_t)mm.O * mm.K : (size_t)mm.O * mm.K / 2;
    if (bytes != need)
        return set_error(error, error_size, "%s: expected %zu bytes, got %zu", name, need, bytes);
    std::vector<uint8_t> dev(mm.w_bytes);
    if (cudaMemcpy(dev.data(), base, mm.w_bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
        return set_error(error, error_size, "copy failed");
    if (!upload) {
        if (scales) unpack_scales(mm, dev.data(), reinterpret_cast<uint8_t *>(data));
        else unpack_values(mm, dev.data(), reinterpret_cast<uint8_t *>(data));
        return 1;
    }
    if (scales) pack_scales(mm, reinterpret_cast<const uint8_t *>(data), dev.data());
    else pack_values(mm, reinterpret_cast<const uint8_t *>(data), dev.data());
    if (cudaMemcpy(base, dev.data(), mm.w_bytes, cudaMemcpyHostToDevice) != cudaSuccess)
        return set_error(error, error_size, "copy failed");
    return 1;
}

int fc_model_set_tensor(FcModel *m, const char *name, const void *data, size_t bytes, char *error,
                        size_t error_size) {
    return tensor_io(m, name, const_cast<void *>(data), bytes, true, error, error_size);
}

int fc_blocks_to_logical(int type, const void *blocks, size_t bytes, int rows, int cols, void *values,
                         void *scales, char *error, size_t error_size) {
    if (!blocks || !values || !scales || rows <= 0 || cols <= 0 || cols % 32)
        return set_error(error, error_size, "blocks need rows > 0 and cols a multiple of 32");
    const size_t nb = (size_t)rows * (cols / 32);
    const uint8_t *b = static_cast<const uint8_t *>(blocks);
    if (type == FC_BLOCKS_Q8_0) {
        if (bytes != nb * 34) return set_error(error, error_size, "Q8_0 data must be %zu bytes", nb * 34);
        int8_t *v = static_cast<int8_t *>(values);
        uint16_t *sc = static_cast<uint16_t *>(scales);
        for (size_t i = 0; i < nb; ++i, b += 34) {
            memcpy(&sc[i], b, 2);
            memcpy(v + i * 32, b + 2, 32);
        }
        return 1;
    }
    if (type == FC_BLOCKS_MXFP4) {
        if (bytes != nb * 17) return set_error(error, error_size, "MXFP4 data must be %zu bytes", nb * 17);
        uint8_t *v = static_cast<uint8_t *>(values);
        uint8_t *sc = static_cast<uint8_t *>(scales);
        for (size_t i = 0; i < nb; ++i, b += 17) {
            sc[i] = b[0];
            uint8_t code[32];
            for (int j = 0; j < 16; ++j) {
                code[j] = b[1 + j] & 15;
                code[j + 16] = b[1 + j] >> 4;
            }
            for (int m = 0; m < 16; ++m) v[i * 16 + m] = (uint8_t)(code[2 * m] | (code[2 * m + 1] << 4));
        }
        return 1;
    }
    return set_error(error, error_size, "unknown block type %d", type);
}

namespace {
const DevMat *find_mat(const FcModel *m, const std::string &name, int *member) {
    auto it = m->names.find(name);
    if (it == m->names.end() || !it->second.mat) return nullptr;
    *member = it->second.member;
    return it->second.mat;
}
}  // namespace

int fc_model_set_tensor_blocks(FcModel *m, const char *name, int type, const void *blocks, size_t bytes,
                               char *error, size_t error_size) {
    if (!m || !name) return set_error(error, error_size, "model and name are required");
    int member = 0;
    const DevMat *mm = find_mat(m, name, &member);
    if (!mm) return set_error(error, error_size, "unknown matrix %s", name);
    const int want = type == FC_BLOCKS_Q8_0 ? FC_FMT_Q8 : type == FC_BLOCKS_MXFP4 ? FC_FMT_MXFP4 : -1;
    if (mm->fmt != want)
        return set_error(error, error_size, "%s is stored as format %d; block type %d does not match", name,
                         mm->fmt, type);
    const size_t vbytes = (size_t)mm->O * mm->K / (want == FC_FMT_Q8 ? 1 : 2);
    const size_t sbytes = (size_t)mm->O * (mm->K / 32) * (want == FC_FMT_Q8 ? 2 : 1);
    std::vector<uint8_t> v(vbytes), sc(sbytes);
    if (!fc_blocks_to_logical(type, blocks, bytes, mm->O, mm->K, v.data(), sc.data(), error, error_size))
        return 0;
    return fc_model_set_tensor(m, name, v.data(), vbytes, error, error_size) &&
           fc_model_set_tensor(m, (std::string(name) + ".gs").c_str(), sc.data(), sbytes, error, error_size);
}

int fc_model_set_tensor_rowscale(FcModel *m, const char *name, const void *values, size_t value_bytes,
                                 const float *row_scales, int rows, char *error, size_t error_size) {
    if (!m || !name || !values || !row_scales) return set_error(error, error_size, "arguments are required");
    int member = 0;
    const DevMat *mm = find_mat(m, name, &member);
    if (!mm) return set_error(error, error_size, "unknown matrix %s", name);
    if (mm->fmt != FC_FMT_Q8 && mm->fmt != FC_FMT_Q4)
        return set_error(error, error_size, "%s is not an int8 / int4 matrix", name);
    if (rows != mm->O) return set_error(error, error_size, "%s has %d rows, not %d", name, mm->O, rows);
    const int G = mm->K / 32;
    std::vector<uint16_t> sc((size_t)mm->O * G);
    for (int r = 0; r < mm->O; ++r) {
        __half h = __float2half_rn(row_scales[r]);
        uint16_t bits;
        memcpy(&bits, &h, 2);
        for (int g = 0; g < G; ++g) sc[(size_t)r * G + g] = bits;
    }
    return fc_model_set_tensor(m, name, values, value_bytes, error, error_size) &&
           fc_model_set_tensor(m, (std::string(name) + ".gs").c_str(), sc.data(), sc.size() * 2, error,
                               error_size);
}

// floyd's Moonlight model directory (moonlight_model.c:41-110): config.json
// and *.safetensors shards written by tools/convert_moonlight.py.
int fc_model_open(FcModel **out, const char *path, int device, char *error, size_t error_size) {
    using namespace fc_container;
    if (!out) return set_error(error, error_size, "model output is required");
    *out = nullptr;
    if (!path || !path[0]) return set_error(error, error_size, "model path is required");
    const std::string dir(path);
    std::string text, err;
    if (!read_file(dir + "/config.json", text))
        return set_error(error, error_size, "cannot open %s/config.json", path);
    Json cfg;
    JsonParser jp(text.data(), text.data() + text.size());
    if (!jp.parse(cfg) || cfg.kind != Json::Obj)
        return set_error(error, error_size, "invalid JSON in %s/config.json", path);
    auto num = [&](const char *k, double fallback) {
        const Json *v = cfg.get(k);
        return v && v->kind == Json::Num ? v->num : fallback;
    };
    auto flag = [&](const char *k, int fallback) {
        const Json *v = cfg.get(k);
        return v && v->kind == Json::Bool ? (int)v->b : fallback;
    };
    Index idx;
    if (!idx.open_dir(dir, err)) return set_error(error, error_size, "%s", err.c_str());
    if (idx.tensors.empty()) return set_error(error, error_size, "no safetensors found in %s", path);

    FcModelConfig c{};
    c.hidden_size = (int)num("hidden_size", 0);
    c.layer_count = (int)num("num_hidden_layers", 0);
    c.vocab_size = (int)num("vocab_size", 0);
    c.head_count = (int)num("num_attention_heads", 0);
    c.q_lora_rank = (int)num("q_lora_rank", 0);  // null (Moonlight) reads as 0
    c.kv_lora_rank = (int)num("kv_lora_rank", 0);
    c.qk_nope_dim = (int)num("qk_nope_head_dim", 0);
    c.qk_rope_dim = (int)num("qk_rope_head_dim", 0);
    c.value_dim = (int)num("v_head_dim", 0);
    c.expert_count = (int)num("n_routed_experts", 0);
    c.experts_per_token = (int)num("num_experts_per_tok", 0);
    c.moe_intermediate_size = (int)num("moe_intermediate_size", 0);
    c.shared_expert_count = (int)num("n_shared_experts", 0);
    c.first_dense_layer_count = (int)num("first_k_dense_replace", 0);
    c.dense_intermediate_size = (int)num("intermediate_size", 0);
    c.normalize_topk = flag("norm_topk_prob", 1);
    c.routed_scale = (float)num("routed_scaling_factor", 1.0);
    c.rms_norm_epsilon = (float)num("rms_norm_eps", 1e-5);
    c.rope_theta = (float)num("rope_theta", 10000.0);
    if (c.rope_theta == 10000.0f) {
        const Json *rp = cfg.get("rope_parameters");
        const Json *t = rp ? rp->get("rope_theta") : nullptr;
        if (t && t->kind == Json::Num) c.rope_theta = (float)t->num;
    }
    // Moonlight routes with sigmoid scores and a selection bias (noaux_tc);
    // the Metal runtime has only that router (moonlight_kernels.metal:469-512)
    c.score_fn = FC_SCORE_SIGMOID;
    if (const Json *sf = cfg.get("scoring_func"))
        if (sf->kind == Json::Str) {
            if (sf->str == "softmax") c.score_fn = FC_SCORE_SOFTMAX;
            else if (sf->str == "sqrtsoftplus") c.score_fn = FC_SCORE_SQRT_SOFTPLUS;
            else if (sf->str != "sigmoid")
                return set_error(error, error_size, "unsupported scoring_func %s", sf->str.c_str());
        }
    c.swiglu_limit = (float)num("swiglu_limit", 0.0);
    c.mtp_layers = 0;
    if (c.hidden_size <= 0 || c.layer_count <= 0 || c.head_count <= 0 || c.vocab_size <= 0 ||
        c.kv_lora_rank <= 0 || c.qk_rope_dim <= 0 ||
        (c.first_dense_layer_count < c.layer_count && (c.expert_count <= 0 || c.experts_per_token <= 0)))
        return set_error(error, error_size, "unsupported Moonlight config in %s/config.json", path);

    // storage formats from the tensors themselves (convert_moonlight.py:56-75):
    // U8 + ".qs" is int8 when it has O*I bytes, int4 when O*ceil(I/2)
    auto row_format = [&](const std::string &name, int I, int *fmt) {
        const Tensor *t = idx.find(name), *qs = idx.find(name + ".qs");
        if (!t || !qs || t->dtype != DT_U8 || qs->dtype != DT_F32 || qs->numel() <= 0) return false;
        const uint64_t O = (uint64_t)qs->numel();
        if (t->bytes == O * (uint64_t)I) *fmt = FC_FMT_Q8;
        else if (t->bytes == O * (uint64_t)((I + 1) / 2)) *fmt = FC_FMT_Q4;
        else return false;
        return true;
    };
    if (!row_format("model.layers.0.self_attn.kv_a_proj_with_mqa.weight", c.hidden_size, &c.dense_format))
        return set_error(error, error_size, "layer 0 kv_a_proj_with_mqa is not an int8 / int4 container matrix");
    c.expert_format = c.dense_format;
    if (c.first_dense_layer_count < c.layer_count) {
        const std::string e0 = "model.layers." + std::to_string(c.first_dense_layer_count) +
                               ".mlp.experts.0.gate_proj.weight";
        if (!row_format(e0, c.hidden_size, &c.expert_format))
            return set_error(error, error_size, "%s is not an int8 / int4 container matrix", e0.c_str());
        c.has_selection_bias = idx.find("model.layers." + std::to_string(c.first_dense_layer_count) +
                                        ".mlp.gate.e_score_correction_bias") != nullptr;
    }
    const Tensor *emb = idx.find("model.embed_tokens.weight");
    if (!emb) return set_error(error, error_size, "model.embed_tokens.weight is missing");
    if (emb->dtype == DT_F32 || emb->dtype == DT_BF16 || emb->dtype == DT_F16) {
        c.embed_f32 = 1;
    } else {
        int f = 0;
        if (!row_format("model.embed_tokens.weight", c.hidden_size, &f) || f != c.dense_format)
            return set_error(error, error_size, "the embedding must be F32 or in the attention format");
    }

    FcModel *m = nullptr;
    if (!fc_model_create(&m, &c, device, error, error_size)) return 0;
    std::map<std::string, bool> pending;
    for (auto &kv : m->names) pending[kv.first] = true;
    std::vector<uint8_t> raw;
    std::vector<float> f32;
    for (auto &kv : idx.tensors) {
        const std::string &name = kv.first;
        const Tensor &t = kv.second;
        if (name.size() > 3 && name.compare(name.size() - 3, 3, ".qs") == 0) continue;
        auto it = m->names.find(name);
        if (it == m->names.end()) continue;  // e.g. rotary_emb.inv_freq: not used
        const Tensor *qs = idx.find(name + ".qs");
        int ok = 1;
        if (qs) {
            if (t.dtype != DT_U8 || !idx.read_f32(*qs, f32)) {
                ok = set_error(error, error_size, "cannot read %s / %s.qs", name.c_str(), name.c_str());
            } else {
                raw.resize(t.bytes);
                const int rows = (int)f32.size();
                const TensorRef &r = it->second;
                if (!r.mat) {
                    ok = set_error(error, error_size, "%s is a vector in this model", name.c_str());
                } else if (!idx.read(t, raw.data())) {
                    ok = set_error(error, error_size, "cannot read %s", name.c_str());
                } else {
                    // int4 rows of an odd width are padded to a whole byte on
                    // disk; the widths here are multiples of 32, so the packed
                    // rows are contiguous
                    ok = fc_model_set_tensor_rowscale(m, name.c_str(), raw.data(), raw.size(), f32.data(), rows,
                                                      error, error_size);
                }
            }
        } else {
            if (!idx.read_f32(t, f32))
                ok = set_error(error, error_size, "%s: unsupported dtype for an unquantized tensor", name.c_str());
            else
                ok = fc_model_set_tensor(m, name.c_str(), f32.data(), f32.size() * 4, error, error_size);
        }
        if (!ok) {
            fc_model_close(m);
            return 0;
        }
        pending.erase(name);
    }
    for (auto &kv : pending) {
        const TensorRef &r = m->names[kv.first];
        if (r.ints) continue;  // hash-routing tables (not in Moonlight)
        std::string missing = kv.first;
        fc_model_close(m);
        return set_error(error, error_size, "tensor %s is missing from %s", missing.c_str(), path);
    }
    cudaDeviceSynchronize();
    *out = m;
    return 1;
}

int fc_model_get_tensor(const FcModel *m, const char *name, void *data, size_t bytes, char *error,
                        size_t error_size) {
    return tensor_io(m, name, data, bytes, false, error, error_size);
}

void fc_model_close(FcModel *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->arena) cudaFree(m->arena);
    delete m;
}

const char *fc_device_name(const FcModel *m) { return m ? m->device_name.c_str() : "(none)"; }

FcModelConfig fc_model_info(const FcModel *m) {
    FcModelConfig c{};
    if (!m) return c;
    c = m->c;
    c.resident_bytes = m->resident;
    return c;
}

}  // extern "C"

namespace {

// Page table [sequences][pages per sequence] of 64-row pages: the first
// shared_rows / 64 pages of every sequence are the same physical pages, the
// rest are each sequence's own.  Returns the number of physical pages.
int build_page_table(int context_size, int sequences, int shared_rows, int *table) {
    const int pps = (context_size + kPageRows - 1) / kPageRows, shared = shared_rows / kPageRows;
    for (int q = 0; q < sequences; ++q)
        for (int p = 0; p < pps; ++p)
            table[(size_t)q * pps + p] = p < shared ? p : shared + q * (pps - shared) + (p - shared);
    return shared + sequences * (pps - shared);
}

// Session construction; `batch` (nullable) makes a multi-sequence session
// whose passes hold whole sequences of batch->rows_per_sequence rows.
int create_session(FcSession **out, FcModel *m, const FcOptions *options, const FcBatchOptions *batch,
                   char *error, size_t error_size, FcSession *share = nullptr) {
    if (!out || !m || !options)
        return set_error(error, error_size, "model and session options are required");
    *out = nullptr;
    if (options->context_size <= 0 || options->max_batch <= 0 ||
        options->max_batch > options->context_size)
        return set_error(error, error_size, "invalid context or batch size");
    cudaSetDevice(m->device);
    const FcModelConfig &c = m->c;
    FcSession *s = new FcSession();
    s->m = m;
    s->opt = *options;
    s->rows_max = std::min(options->max_batch, kMaxRows);
    if (batch) {
        s->batch = true;
        s->n_seq = batch->sequences;
        s->group_rows = batch->rows_per_sequence;
        s->shared_rows = batch->shared_prefix;
        s->seq_pos.assign(batch->sequences, 0);
    }
    s->stats.resident_bytes = m->resident;
    const int mb = s->rows_max;
    const int D = c.hidden_size, H = c.head_count, L = c.kv_lora_rank, R = c.qk_rope_dim;
    const int QW = c.qk_nope_dim + R, V = c.vocab_size;
    const int E = std::max(c.expert_count, 1), K = std::max(c.experts_per_token, 1);
    const int I = std::max(c.moe_intermediate_size, 32);
    const int W = std::max(I * c.shared_expert_count, 32);
    const int nl = std::max(m->expert_hi - m->expert_lo, 1);
    s->max_slots = std::min(nl, mb * K);
    // attention split plan: fixed per session (see mla.cuh)
    int max_chunks = (options->context_size + kAttnKeys - 1) / kAttnKeys;
    // tcgen05 attention when a verify batch fills at least one 128-query
    // tile; the choice depends only on the session shape, so decode and
    // verify rows always take the same kernel (FLOYD_ATTENTION=mma / tc
    // overrides it for measurements)
    const char *attn_env = getenv("FLOYD_ATTENTION");
    s->attn_tc = std::min(mb, 4) * H >= kTcRows;
    if (attn_env && strcmp(attn_env, "mma") == 0) s->attn_tc = false;
    if (attn_env && strcmp(attn_env, "tc") == 0) s->attn_tc = true;
    if (batch) {
        // a query tile must hold rows of one sequence only
        const int q = s->group_rows * H;
        s->attn_tc = q % kTcRows == 0;
        if (!s->attn_tc && q % kAttnQ) {
            delete s;
            return set_error(error, error_size,
                             "rows_per_sequence x heads (%d) must be a multiple of %d", q, kAttnQ);
        }
    }
    int target;
    if (s->attn_tc) {
        // one wave of (128-query tile, half) CTAs at up to 4 rows; at most
        // 64 splits (the combine's register budget)
        int qt = (std::min(mb, 4) * H + kTcRows - 1) / kTcRows;
        target = std::max(1, std::min(64, 148 / (2 * qt)));
    } else {
        int qtiles = (mb * H + kAttnQ - 1) / kAttnQ;
        target = std::max(1, 2 * 148 / qtiles);
    }
    s->chunks_per_split = (max_chunks + target - 1) / target;
    s->splits = (max_chunks + s->chunks_per_split - 1) / s->chunks_per_split;
    s->mtp_chunks_per_split = s->chunks_per_split;
    s->mtp_splits = s->splits;
    if (s->attn_tc) {
        const int qt1 = (H + kTcRows - 1) / kTcRows;  // one row's query tiles
        const int t1 = std::max(1, std::min(64, 148 / (2 * qt1)));
        s->mtp_chunks_per_split = (max_chunks + t1 - 1) / t1;
        s->mtp_splits = (max_chunks + s->mtp_chunks_per_split - 1) / s->mtp_chunks_per_split;
    }
    const int part_splits = std::max(s->splits, s->mtp_splits);  // split partial buffers hold either plan
    s->head_chunks = (V + kHeadChunk - 1) / kHeadChunk;
    s->attn_smem = AttnSmem::total(L + R);
    bool ok = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaEventCreate(&s->ev_begin) == cudaSuccess && cudaEventCreate(&s->ev_end) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&s->ev_lane, cudaEventDisableTiming) == cudaSuccess;
    const int NLc = c.layer_count + c.mtp_layers;  // cache layers (target + drafter)
    {
        // page table: an ordinary session maps page p to itself; a batch
        // session maps every sequence's first shared_rows / 64 pages to the
        // same (shared) pages and the rest to its own pages
        const int pps = (options->context_size + kPageRows - 1) / kPageRows;
        std::vector<int> table((size_t)s->n_seq * pps);
        const int pages = build_page_table(options->context_size, s->n_seq, s->shared_rows, table.data());
        s->layer_rows = batch ? pages * kPageRows : options->context_size;
        if (share) {  // a lane: the parent's cache and page table
            s->lane = true;
            s->cache = share->cache;
            s->page_table = share->page_table;
        } else {
            ok = ok && salloc(s, s->cache, (size_t)NLc * s->layer_rows * (L + R));
            ok = ok && salloc(s, s->page_table, table.size()) &&
                 cudaMemcpy(s->page_table, table.data(), table.size() * sizeof(int), cudaMemcpyHostToDevice) ==
                     cudaSuccess;
        }
        s->pmap.pt = s->page_table;
        s->pmap.pps = pps;
    }
    ok = ok && salloc(s, s->resid, (size_t)mb * D) && salloc(s, s->xn, (size_t)mb * D);
    ok = ok && salloc(s, s->xq_norm, (size_t)mb * kpad(D) * 2);
    ok = ok && salloc(s, s->q, (size_t)mb * H * QW);
    ok = ok && salloc(s, s->qa, (size_t)mb * std::max(c.q_lora_rank, 1));
    ok = ok && salloc(s, s->qa_xq, (size_t)mb * kpad(std::max(c.q_lora_rank, 1)) * 2);
    ok = ok && salloc(s, s->ckv, (size_t)mb * (L + R));
    // rows padded to whole 128-query tiles (the TMA box of the query tile)
    const int q_rows = (mb * H + kTcRows - 1) / kTcRows * kTcRows;
    ok = ok && salloc(s, s->qcat, (size_t)q_rows * (L + R));
    ok = ok && salloc(s, s->part_o, (size_t)part_splits * mb * H * L);
    ok = ok && salloc(s, s->part_m, (size_t)2 * part_splits * mb * H);  // [half][split][row] (tcgen05 attention)
    ok = ok && salloc(s, s->part_l, (size_t)2 * part_splits * mb * H);
    ok = ok && salloc(s, s->ctx_xq, (size_t)H * mb * kpad(L) * 2);
    ok = ok && salloc(s, s->o_xq, (size_t)mb * kpad(H * c.value_dim) * 2);
    ok = ok && salloc(s, s->router_logits, (size_t)2 * mb * E);  // scores, then choices
    ok = ok && salloc(s, s->route_ids, (size_t)NLc * mb * K);
    ok = ok && salloc(s, s->route_w, (size_t)NLc * mb * K);
    if (c.mtp_layers) {
        ok = ok && salloc(s, s->d_mtp, 1) && salloc(s, s->mtp_h, (size_t)D);
        ok = ok && salloc(s, s->mtp_logits, (size_t)V);
        ok = ok && salloc(s, s->mtp_xq, (size_t)mb * kpad(2 * D) * 2);
        if (!batch) {
            ok = ok && salloc(s, s->hist, (size_t)s->opt.context_size * D);
            s->tok_hist.assign((size_t)s->opt.context_size, 0);
        }
    }
    ok = ok && salloc(s, s->n_active, 1) && salloc(s, s->active, (size_t)s->max_slots + 1);
    s->g_slots = std::min(E, mb * K);
    ok = ok && salloc(s, s->coef, (size_t)(s->g_slots + 1) * 8);
    ok = ok && salloc(s, s->n_global, 1) && salloc(s, s->n_before, 1);
    ok = ok && salloc(s, s->h_xq, (size_t)s->max_slots * mb * kpad(I) * 2);
    ok = ok && salloc(s, s->hsh_xq, (size_t)mb * kpad(W) * 2);
    ok = ok && salloc(s, s->hd_xq, (size_t)mb * kpad(std::max(c.dense_intermediate_size, 32)) * 2);
    ok = ok && salloc(s, s->moe_part, (size_t)s->g_slots * mb * D);
    if (ok && m->world > 1) {
        const size_t xb = (size_t)2 * s->g_slots * mb * D * sizeof(float);
        // head-parallel attention: single-sequence sessions of models with
        // q-lora whose heads split evenly and whose last target layer and
        // drafter layers are MoE (the expert exchange between two attention
        // exchanges of the same buffer parity orders them);
        // opt-in with FLOYD_HEAD_SHARD=1 (measured slower than replicated
        // heads at 2 GPUs: the W_UV hand-off costs more than the halved MLA work)
        bool hs = !batch && c.q_lora_rank > 0 && c.head_count % m->world == 0 && s->attn_tc &&
                  (c.qk_nope_dim + c.qk_rope_dim) % kTileRows == 0 && (c.qk_nope_dim + c.value_dim) % kTileRows == 0;
        for (int l = c.layer_count - 1; hs && l < (int)m->layers.size(); ++l) hs = !m->layers[l].dense;
        const char *hs_env = getenv("FLOYD_HEAD_SHARD");
        hs = hs && hs_env && strcmp(hs_env, "1") == 0;
        s->head_shard = hs;
        s->heads = hs ? c.head_count / m->world : c.head_count;
        s->head0 = hs ? m->rank * s->heads : 0;
        s->ep_attn_off = xb + 256;
        s->ep_oxq_bytes = hs ? align256((size_t)mb * kpad(H * c.value_dim) * 2 * sizeof(__half)) : 0;
        const size_t region = s->ep_attn_off + 256 + 2 * s->ep_oxq_bytes;
        ok = cudaMalloc(&s->ep_region, region) == cudaSuccess;
        if (ok) {
            cudaMemset(s->ep_region, 0, region);
            s->ep_xbuf = reinterpret_cast<float *>(s->ep_region);
            s->ep_flags = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(s->ep_region) + xb);
        }
        ok = ok && salloc(s, s->ep_epoch, 1);
        ok = ok && salloc(s, s->ep_aepoch, 1) && salloc(s, s->ep_adone, 1);
        ok = ok && salloc(s, s->ep_wait_ns, 1);
    }
    ok = ok && salloc(s, s->sh_part, (size_t)mb * D);
    ok = ok && salloc(s, s->logits, (size_t)mb * V);
    ok = ok && salloc(s, s->layer_out, (size_t)c.layer_count * mb * D);
    size_t hc = (size_t)mb * s->head_chunks;
    ok = ok && salloc(s, s->hp.amax, hc) && salloc(s, s->hp.aidx, hc) && salloc(s, s->hp.zmax, hc) &&
         salloc(s, s->hp.zsum, hc) && salloc(s, s->hp.gval, hc) && salloc(s, s->hp.gidx, hc);
    ok = ok && salloc(s, s->d_stage, 1) && salloc(s, s->d_res, 1) && salloc(s, s->d_err, 1);
    ok = ok && salloc(s, s->route_arrivals, 1);
    ok = ok && cudaMallocHost(&s->h_stage, sizeof(Staging)) == cudaSuccess;
    ok = ok && cudaMallocHost(&s->h_res, sizeof(Result)) == cudaSuccess;
    if (ok && s->attn_tc)
        ok = make_map_f16(&s->qmap, s->qcat, (uint64_t)(L + R), (uint64_t)q_rows, kTcRows);
    // prefill chunks on the tensor cores when the caller asks for more rows
    // per pass than a verify holds (single-GPU models with quantized weights)
    auto quant = [](int f) { return f == FC_FMT_Q8 || f == FC_FMT_Q4 || f == FC_FMT_MXFP4; };
    const int NP = c.qk_nope_dim, VD = c.value_dim, DI = c.dense_intermediate_size;
    const bool pf_ok = !batch && options->max_batch > s->rows_max && m->world == 1 && quant(c.dense_format) &&
                       (c.expert_count == 0 || quant(c.expert_format)) && L % 64 == 0 && R == 64 &&
                       (NP == 64 || NP == 128) && (VD == 64 || VD == 128) && D <= 4 * kPfNormVec * 256 && c.q_lora_rank <= 4 * kPfNormVec * 256 && (size_t)NLc * options->context_size >= (size_t)kPfM && D % 32 == 0 && (H * QW) % 32 == 0 && I % 32 == 0 &&
                       W % 32 == 0 && DI % 32 == 0 && c.q_lora_rank % 32 == 0 && K <= 64 && E <= 1024;
    if (ok && pf_ok) {
        const int P = options->max_batch, Pp = (P + kPfM - 1) / kPfM * kPfM;
        const int Sp = (Pp * K + kPfM - 1) / kPfM * kPfM;
        const int QL = std::max(c.q_lora_rank, 32), HW = std::max(std::max(DI, W), 32);
        s->pf_rows = P;
        s->pf_pad = Pp;
        s->pf_slots = Sp;
        ok = ok && salloc(s, s->pf_ids, (size_t)P + 1) &&
             cudaMallocHost(&s->pf_h_ids, ((size_t)P + 1) * sizeof(int)) == cudaSuccess;
        ok = ok && salloc(s, s->pf_resid, (size_t)Pp * D) && salloc(s, s->pf_xn, (size_t)Pp * D);
        ok = ok && salloc(s, s->pf_x16, (size_t)Pp * D) && salloc(s, s->pf_q16, (size_t)Pp * H * QW);
        ok = ok && salloc(s, s->pf_qa, (size_t)Pp * QL) && salloc(s, s->pf_qa16, (size_t)Pp * QL);
        const int Kr = (options->context_size + kFaKeys - 1) / kFaKeys * kFaKeys;  // kvd rows
        ok = ok && salloc(s, s->pf_ckv, (size_t)Pp * (L + R)) && salloc(s, s->pf_kvd, (size_t)Kr * H * (NP + VD));
        ok = ok && salloc(s, s->pf_o16, (size_t)Pp * H * VD);
        ok = ok && salloc(s, s->pf_h16, (size_t)Pp * HW);
        ok = ok && salloc(s, s->pf_logits, (size_t)Pp * E) && salloc(s, s->pf_choice, (size_t)Pp * E);
        ok = ok && salloc(s, s->pf_rpart, (size_t)kPfRtMaxSplits * Pp * E);
        ok = ok && salloc(s, s->pf_route_ids, (size_t)Pp * K) && salloc(s, s->pf_route_w, (size_t)Pp * K);
        ok = ok && salloc(s, s->pf_slot_of, (size_t)Pp * K) && salloc(s, s->pf_counts, (size_t)E);
        ok = ok && salloc(s, s->pf_offsets, (size_t)E) && salloc(s, s->pf_cursor, (size_t)E);
        ok = ok && salloc(s, s->pf_mt_count, 1) && salloc(s, s->pf_mt_table, (size_t)Sp / kPfM + E + 1);
        ok = ok && salloc(s, s->pf_xg, (size_t)Sp * D) && salloc(s, s->pf_hg, (size_t)Sp * I);
        ok = ok && salloc(s, s->pf_yd, (size_t)Sp * D) && salloc(s, s->pf_sh, (size_t)Pp * D);
        ok = ok && make_map_f16(&s->pf_map_x, s->pf_x16, D, Pp, kPfM) &&
             make_map_f16(&s->pf_map_q, s->pf_q16, (uint64_t)H * QW, Pp, kPfM) &&
             make_map_f16(&s->pf_map_qa, s->pf_qa16, QL, Pp, kPfM) &&
             make_map_f16(&s->pf_map_o, s->pf_o16, (uint64_t)H * VD, Pp, kPfM) &&
             make_map_f16(&s->pf_map_hd, s->pf_h16, std::max(DI, 32), Pp, kPfM) &&
             make_map_f16(&s->pf_map_hs, s->pf_h16, W, Pp, kPfM) &&
             make_map_f16(&s->pf_map_xg, s->pf_xg, D, Sp, kPfM) &&
             make_map_f16(&s->pf_map_hg, s->pf_hg, I, Sp, kPfM) &&
             make_map_f16(&s->pf_map_kvd, s->pf_kvd, (uint64_t)H * (NP + VD), Kr, kFaKeys) &&
             make_map_f16(&s->pf_cmap, s->cache, (uint64_t)(L + R), (uint64_t)NLc * options->context_size, kPfM) &&
             make_map_f16(&s->pf_cmap64, s->cache, (uint64_t)(L + R), (uint64_t)NLc * options->context_size,
                          kFaKeys);
        ok = ok && pf_prepare_all() == cudaSuccess;
    }
    if (ok && (s->attn_tc || s->pf_rows))
        ok = make_map_f16(&s->kvmap, s->cache, (uint64_t)(L + R), (uint64_t)NLc * s->layer_rows, kTcKeys);
    if (ok) {
        cudaError_t e1 = cudaFuncSetAttribute(mla_attention_kernel<512, 64>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)AttnSmem::total(576));
        cudaError_t e2 = cudaFuncSetAttribute(mla_attention_kernel<256, 64>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)AttnSmem::total(320));
        cudaError_t e3 = cudaFuncSetAttribute(mla_attention_tc_kernel<512>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)TcAttnPlan<512>::SMEM);
        cudaError_t e4 = cudaFuncSetAttribute(mla_attention_tc_kernel<256>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)TcAttnPlan<256>::SMEM);
        ok = e1 == cudaSuccess && e2 == cudaSuccess && e3 == cudaSuccess && e4 == cudaSuccess &&
             gemv_prepare_all() == cudaSuccess && prefer_shared_carveout() == cudaSuccess;
    }
    if (!ok) {
        free_session_buffers(s);
        delete s;
        return set_error(error, error_size, "session allocation failed");
    }
    *out = s;
    return 1;
}

}  // namespace

extern "C" {

int fc_session_create(FcSession **out, FcModel *m, const FcOptions *options, char *error,
                      size_t error_size) {
    return create_session(out, m, options, nullptr, error, error_size);
}

int fc_session_create_batch(FcSession **out, FcModel *m, const FcBatchOptions *options, char *error,
                            size_t error_size) {
    if (!out || !m || !options) return set_error(error, error_size, "model and batch options are required");
    *out = nullptr;
    const FcBatchOptions &b = *options;
    if (b.sequences < 1 || b.sequences > 64 || b.rows_per_sequence < 1 || b.rows_per_sequence > kMaxRows ||
        b.context_size < b.rows_per_sequence || b.shared_prefix < 0 || b.shared_prefix % kPageRows ||
        b.shared_prefix > b.context_size)
        return set_error(error, error_size, "invalid batch options");
    FcOptions o{};
    o.context_size = b.context_size;
    o.max_batch = std::min(b.sequences, kMaxRows / b.rows_per_sequence) * b.rows_per_sequence;
    if (!create_session(out, m, &o, &b, error, error_size)) return 0;
    // one lane per pass of a batch step (at most kMaxLanes) on a single
    // GPU; FLOYD_BATCH_LANES=n caps it (1: the passes run one at a time)
    FcSession *s = *out;
    const int per_pass = o.max_batch / b.rows_per_sequence;
    int nl = std::min((b.sequences + per_pass - 1) / per_pass, kMaxLanes);
    if (const char *env = getenv("FLOYD_BATCH_LANES")) nl = std::max(1, std::min(nl, atoi(env)));
    if (m->world > 1) nl = 1;  // the expert exchange buffers belong to one session
    for (int i = 1; i < nl; ++i) {
        FcSession *c = nullptr;
        if (!create_session(&c, m, &o, &b, error, error_size, s)) {
            fc_session_destroy(s);
            *out = nullptr;
            return 0;
        }
        s->lanes.push_back(c);
    }
    return 1;
}

void fc_session_destroy(FcSession *s) {
    if (!s) return;
    cudaSetDevice(s->m->device);
    for (FcSession *c : s->lanes) {
        free_session_buffers(c);
        delete c;
    }
    s->lanes.clear();
    free_session_buffers(s);
    delete s;
}

void fc_session_reset(FcSession *s) {
    if (!s) return;
    s->position = 0;
    s->last_rows = 0;
    std::fill(s->seq_pos.begin(), s->seq_pos.end(), 0);
    uint64_t allocs = s->stats.buffer_allocations, resident = s->stats.resident_bytes;
    s->stats = FcStats{};
    s->stats.buffer_allocations = allocs;
    s->stats.resident_bytes = resident;
}

int fc_session_position(const FcSession *s) { return s ? s->position : 0; }

FcStats fc_session_stats(const FcSession *s) {
    FcStats r{};
    return s ? s->stats : r;
}

int fc_session_prefill(FcSession *s, const int *ids, int count, float *last_logits, char *error,
                       size_t error_size) {
    if (s && s->batch) return set_error(error, error_size, "batch sessions run fc_session_verify_batch");
    if (!s || !ids || !last_logits || count <= 0 || count > s->opt.max_batch ||
        count > s->opt.context_size)
        return set_error(error, error_size, "invalid prefill request");
    if (s->position != 0) return set_error(error, error_size, "prefill requires an empty session");
    double t0 = now_ms();
    if (!run_tokens(s, ids, count, last_logits, error, error_size)) return 0;
    s->stats.prefill_tokens += (uint64_t)count;
    s->stats.prefill_ms += now_ms() - t0;
    return 1;
}

int fc_session_append(FcSession *s, const int *ids, int count, float *last_logits, char *error,
                      size_t error_size) {
    if (s && s->batch) return set_error(error, error_size, "batch sessions run fc_session_verify_batch");
    if (!s || !ids || !last_logits || count <= 0 || count > s->opt.max_batch || s->position <= 0 ||
        s->position + count > s->opt.context_size)
        return set_error(error, error_size, "invalid append request");
    double t0 = now_ms();
    if (!run_tokens(s, ids, count, last_logits, error, error_size)) return 0;
    s->stats.prefill_tokens += (uint64_t)count;
    s->stats.prefill_ms += now_ms() - t0;
    return 1;
}

int fc_session_decode(FcSession *s, int token, float *logits, char *error, size_t error_size) {
    if (s && s->batch) return set_error(error, error_size, "batch sessions run fc_session_verify_batch");
    if (!s || !logits || s->position < 0 || s->position >= s->opt.context_size)
        return set_error(error, error_size, "invalid decode request");
    double t0 = now_ms();
    if (!run_tokens(s, &token, 1, logits, error, error_size)) return 0;
    s->stats.decode_tokens++;
    s->stats.decode_ms += now_ms() - t0;
    return 1;
}

int fc_session_verify(FcSession *s, const int *ids, int k, const FcAcceptConfig *accept,
                      int *emitted, int *n_emitted, int *next_token, float *last_logits,
                      char *error, size_t error_size) {
    if (s && s->batch) return set_error(error, error_size, "batch sessions run fc_session_verify_batch");
    if (!s || !ids || !emitted || !n_emitted || !next_token || k < 0)
        return set_error(error, error_size, "invalid verify request");
    int rows = k + 1;
    if (rows > s->rows_max)
        return set_error(error, error_size, "verify of %d rows exceeds the %d-row pass", rows,
                         s->rows_max);
    if (s->position + rows > s->opt.context_size)
        return set_error(error, error_size, "verify exceeds the context (%d + %d > %d)", s->position,
                         rows, s->opt.context_size);
    if (accept && accept->mode == FC_ACCEPT_SAMPLE && !(accept->temperature > 0.0f))
        return set_error(error, error_size, "sampling needs a positive temperature");
    if (!check_ids(s, ids, rows, error, error_size)) return 0;
    double t0 = now_ms();
    if (!run_pass(s, ids, rows, k, accept, error, error_size)) return 0;
    const Result &r = *s->h_res;
    int commit = r.commit;
    if (commit < 1 || commit > rows) return set_error(error, error_size, "verify produced commit %d", commit);
    for (int i = 0; i < commit; ++i) emitted[i] = ids[i];
    *n_emitted = commit;
    *next_token = r.next_token;
    if (last_logits) {  // the logits row of the last committed token
        cudaError_t e = cudaMemcpy(last_logits, s->logits + (size_t)(commit - 1) * s->m->c.vocab_size,
                                   (size_t)s->m->c.vocab_size * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return set_error(error, error_size, "logits copy failed");
    }
    s->position += commit;  // rollback of rows >= commit: the cache is append-only
    s->stats.verify_calls++;
    s->stats.proposed_tokens += (uint64_t)k;
    s->stats.accepted_tokens += (uint64_t)commit;
    s->stats.verify_ms += now_ms() - t0;
    return 1;
}

int fc_session_batch_seed(FcSession *s, int sequence, int start, int end, uint64_t seed, char *error,
                          size_t error_size) {
    if (!s || !s->batch || sequence < 0 || sequence >= s->n_seq || start < 0 || end < start ||
        end > s->opt.context_size)
        return set_error(error, error_size, "invalid batch seed request");
    const FcModelConfig &c = s->m->c;
    cudaSetDevice(s->m->device);
    const int L = c.kv_lora_rank, R = c.qk_rope_dim;
    for (int l = 0; l < c.layer_count && end > start; ++l)
        synth_kv_range_kernel<<<grid_for((size_t)(end - start) * (L + R)), 256, 0, s->stream>>>(
            s->cache + (size_t)l * s->layer_rows * (L + R), s->pmap, sequence, start, end, L, R, seed,
            fc_tensor_id(l, FC_T_KV_LATENT, 0), fc_tensor_id(l, FC_T_KV_ROPE, 0));
    cudaError_t e = cudaStreamSynchronize(s->stream);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(error, error_size, "seeding failed: %s", cudaGetErrorString(e));
    s->seq_pos[sequence] = std::max(s->seq_pos[sequence], end);
    return 1;
}

int fc_session_verify_batch(FcSession *s, const int *ids, int k, const FcAcceptConfig *accept, int *n_emitted,
                            int *next_token, char *error, size_t error_size) {
    if (!s || !s->batch || !ids || !n_emitted || !next_token || k + 1 != s->group_rows)
        return set_error(error, error_size, "invalid batch verify request (k must be rows_per_sequence - 1)");
    const int gr = s->group_rows, nseq = s->n_seq;
    for (int q = 0; q < nseq; ++q) {
        if (s->seq_pos[q] + gr > s->opt.context_size)
            return set_error(error, error_size, "sequence %d: verify exceeds the context (%d + %d > %d)", q,
                             s->seq_pos[q], gr, s->opt.context_size);
        if (s->seq_pos[q] < 1) return set_error(error, error_size, "sequence %d has no context", q);
        if (s->seq_pos[q] < s->shared_rows)  // its rows would land in pages every sequence reads
            return set_error(error, error_size, "sequence %d is inside the shared prefix (%d < %d)", q,
                             s->seq_pos[q], s->shared_rows);
        if (accept) {
            if (accept[q].mode == FC_ACCEPT_SAMPLE && !(accept[q].temperature > 0.0f))
                return set_error(error, error_size, "sampling needs a positive temperature");
            if (accept[q].mode != accept[0].mode || accept[q].temperature != accept[0].temperature ||
                accept[q].seed != accept[0].seed)
                return set_error(error, error_size, "sequences of a batch share mode, temperature and seed");
        }
    }
    if (!check_ids(s, ids, nseq * gr, error, error_size)) return 0;
    double t0 = now_ms();
    const int per_pass = s->rows_max / gr;
    // passes run in waves of one pass per lane (the session itself is lane
    // 0); eager profiled and traced passes run one at a time
    const int nl = (s->profiling || s->trace) ? 1 : 1 + (int)s->lanes.size();
    auto lane = [&](int w) { return w == 0 ? s : s->lanes[w - 1]; };
    int seqs[kMaxLanes][kMaxRows], ngs[kMaxLanes];
    for (int q0 = 0; q0 < nseq; q0 += per_pass * nl) {
        int nw = 0;
        for (; nw < nl && q0 + nw * per_pass < nseq; ++nw) {
            const int qa = q0 + nw * per_pass;
            ngs[nw] = std::min(per_pass, nseq - qa);
            for (int j = 0; j < ngs[nw]; ++j) seqs[nw][j] = qa + j;
        }
        s->last_lane = nullptr;
        if (nw == 1) {
            if (!run_batch_pass(s, seqs[0], ngs[0], ids + (size_t)q0 * gr, k, accept, error, error_size)) return 0;
        } else {
            // every pass of the wave is staged and its graph recorded before
            // any is launched; the lanes start after an event on the
            // session's stream and the session's stream waits for all of
            // them, so the events around the wave time all its passes
            for (int w = 0; w < nw; ++w) {
                FcSession *L = lane(w);
                stage_batch_pass(L, s->seq_pos, seqs[w], ngs[w], ids + (size_t)(q0 + w * per_pass) * gr, k, accept);
                if (!get_graph(L, ngs[w] * gr, 0, error, error_size)) return 0;
            }
            cudaSetDevice(s->m->device);
            cudaEventRecord(s->ev_begin, s->stream);
            for (int w = 0; w < nw; ++w) {
                FcSession *L = lane(w);
                if (w > 0) cudaStreamWaitEvent(L->stream, s->ev_begin, 0);
                if (!launch_pass(L, ngs[w] * gr, 0, error, error_size)) {
                    cudaDeviceSynchronize();
                    return 0;
                }
                if (w > 0) {
                    cudaEventRecord(L->ev_lane, L->stream);
                    cudaStreamWaitEvent(s->stream, L->ev_lane, 0);
                }
            }
            cudaEventRecord(s->ev_end, s->stream);
            cudaError_t e = cudaStreamSynchronize(s->stream);
            if (e != cudaSuccess) return set_error(error, error_size, "CUDA forward failed: %s", cudaGetErrorString(e));
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, s->ev_begin, s->ev_end);
            s->stats.gpu_ms += ms;
            int kernels = 0;
            for (int w = 0; w < nw; ++w) {
                if (!finish_pass(lane(w), ngs[w] * gr, 0, error, error_size)) return 0;
                kernels += lane(w)->last_kernels;
            }
            s->last_lane = lane(nw - 1);
            s->last_kernels = kernels;  // every pass of the wave
        }
        for (int w = 0; w < nw; ++w) {
            const Result &r = *lane(w)->h_res;
            for (int j = 0; j < ngs[w]; ++j) {
                const int q = seqs[w][j], commit = r.g_commit[j];
                if (commit < 1 || commit > gr)
                    return set_error(error, error_size, "sequence %d: verify produced commit %d", q, commit);
                n_emitted[q] = commit;
                next_token[q] = r.g_next[j];
                s->seq_pos[q] += commit;  // rows past the commit are overwritten later
                s->stats.accepted_tokens += (uint64_t)commit;
            }
        }
    }
    s->stats.verify_calls++;
    s->stats.proposed_tokens += (uint64_t)k * nseq;
    s->stats.verify_ms += now_ms() - t0;
    return 1;
}

int fc_session_batch_position(const FcSession *s, int sequence) {
    if (!s || !s->batch || sequence < 0 || sequence >= s->n_seq) return -1;
    return s->seq_pos[sequence];
}

int fc_session_batch_rollback(FcSession *s, int sequence, int position, char *error, size_t error_size) {
    if (!s || !s->batch || sequence < 0 || sequence >= s->n_seq || position < 0)
        return set_error(error, error_size, "invalid batch rollback");
    s->seq_pos[sequence] = std::min(s->seq_pos[sequence], position);
    return 1;
}

int fc_session_set_profiling(FcSession *s, int enabled) {
    if (!s) return 0;
    cudaSetDevice(s->m->device);
    if (enabled && s->prof_events.empty()) {
        size_t count = (size_t)(s->m->c.layer_count + 4 * s->m->c.mtp_layers) * 24 + 64;
        s->prof_events.resize(count);
        for (auto &ev : s->prof_events)
            if (cudaEventCreate(&ev) != cudaSuccess) return 0;
    }
    s->profiling = enabled != 0;
    return 1;
}

int fc_session_profile(const FcSession *s, int index, char *name, size_t name_size,
                       double *total_ms, uint64_t *launches) {
    if (!s || index < 0 || (size_t)index >= s->prof.size()) return 0;
    const auto &p = s->prof[(size_t)index];
    if (name && name_size) snprintf(name, name_size, "%s", p.first.c_str());
    if (total_ms) *total_ms = p.second.first;
    if (launches) *launches = p.second.second;
    return 1;
}

int fc_session_set_layer_trace(FcSession *s, int enabled) {
    if (!s) return 0;
    s->trace = enabled != 0;
    return 1;
}

void fc_session_profile_reset(FcSession *s) {
    if (s) s->prof.clear();
}

int fc_session_rollback(FcSession *s, int position, char *error, size_t error_size) {
    if (s && s->batch) return set_error(error, error_size, "batch sessions run fc_session_verify_batch");
    if (!s || position < 0) return set_error(error, error_size, "invalid rollback request");
    if (position < s->position) s->position = position;
    return 1;
}

int fc_session_copy_row_logits(const FcSession *s, float *logits, int capacity_rows) {
    if (s && s->last_lane) s = s->last_lane;  // a batch step's last pass ran on a lane
    if (!s || !logits || capacity_rows < s->last_rows || s->last_rows <= 0) return 0;
    return cudaMemcpy(logits, s->logits, (size_t)s->last_rows * s->m->c.vocab_size * 4,
                      cudaMemcpyDeviceToHost) == cudaSuccess;
}

int fc_session_last_kernel_count(const FcSession *s) { return s ? s->last_kernels : 0; }

double fc_session_exchange_wait_ms(FcSession *s) {
    if (!s || !s->ep_wait_ns) return 0.0;
    unsigned long long ns = 0;
    cudaSetDevice(s->m->device);
    cudaStreamSynchronize(s->stream);
    cudaMemcpy(&ns, s->ep_wait_ns, sizeof ns, cudaMemcpyDeviceToHost);
    cudaMemset(s->ep_wait_ns, 0, sizeof ns);
    return (double)ns * 1e-6;
}

void fc_io_bytes(size_t *h2d, size_t *d2h) {
    if (h2d) *h2d = sizeof(Staging);
    if (d2h) *d2h = sizeof(Result);
}

int fc_session_drafts(const FcSession *s, int *drafts, int capacity) {
    if (!s || !drafts) return 0;
    int n = std::min(s->last_drafts, capacity);
    for (int i = 0; i < n; ++i) drafts[i] = s->h_res->drafts[i];
    return n;
}

int fc_session_ep_handle(FcSession *s, void *handle, size_t handle_size, char *error,
                         size_t error_size) {
    if (!s || !handle || handle_size < sizeof(cudaIpcMemHandle_t))
        return set_error(error, error_size, "session and a %zu-byte handle buffer are required",
                         sizeof(cudaIpcMemHandle_t));
    if (!s->ep_region) return set_error(error, error_size, "session is not expert-parallel");
    cudaSetDevice(s->m->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, s->ep_region);
    if (e != cudaSuccess) return set_error(error, error_size, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    memcpy(handle, &h, sizeof(h));
    return 1;
}

int fc_session_ep_connect(FcSession *s, const void *handles, int world, char *error, size_t error_size) {
    if (!s || !handles) return set_error(error, error_size, "session and handles are required");
    FcModel *m = s->m;
    if (world != m->world || !s->ep_region)
        return set_error(error, error_size, "world %d does not match the model's expert-parallel world %d",
                         world, m->world);
    cudaSetDevice(m->device);
    for (int r = 0; r < world; ++r) {
        if (r == m->rank || s->ep_peer_region[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, reinterpret_cast<const uint8_t *>(handles) + (size_t)r * FC_EP_HANDLE_BYTES, sizeof(h));
        cudaError_t e = cudaIpcOpenMemHandle(&s->ep_peer_region[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(error, error_size, "cudaIpcOpenMemHandle(rank %d): %s", r, cudaGetErrorString(e));
    }
    for (auto &g : s->graphs) cudaGraphExecDestroy(g.second);
    s->graphs.clear();
    s->ep_connected = true;
    return 1;
}

int fc_session_seed_context(FcSession *s, int positions, uint64_t seed, char *error,
                            size_t error_size) {
    if (s && s->batch) return set_error(error, error_size, "batch sessions run fc_session_verify_batch");
    if (!s || positions < 0 || positions > s->opt.context_size)
        return set_error(error, error_size, "invalid seeded context");
    const FcModelConfig &c = s->m->c;
    cudaSetDevice(s->m->device);
    int L = c.kv_lora_rank, R = c.qk_rope_dim;
    for (int l = 0; l < c.layer_count && positions > 0; ++l) {
        __half *cache = s->cache + (size_t)l * s->layer_rows * (L + R);
        synth_kv_kernel<<<grid_for((size_t)positions * (L + R)), 256, 0, s->stream>>>(
            cache, positions, L, R, seed, fc_tensor_id(l, FC_T_KV_LATENT, 0),
            fc_tensor_id(l, FC_T_KV_ROPE, 0));
    }
    cudaError_t e = cudaStreamSynchronize(s->stream);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(error, error_size, "seeding failed: %s", cudaGetErrorString(e));
    s->position = positions;
    return 1;
}

int fc_test_batch_page_table(int context_size, int sequences, int shared_prefix, int *table, int capacity) {
    if (context_size <= 0 || sequences < 1 || shared_prefix < 0 || shared_prefix % kPageRows ||
        shared_prefix > context_size)
        return -1;
    const int pps = (context_size + kPageRows - 1) / kPageRows;
    if (!table || capacity < sequences * pps) return -1;
    return build_page_table(context_size, sequences, shared_prefix, table);
}

int fc_test_kv_length(const FcSession *s, int layer) {
    if (!s || layer < 0 || layer >= s->m->c.layer_count) return -1;
    return s->position;
}

int fc_test_copy_kv(const FcSession *s, int layer, float *latent, float *rope, int capacity) {
    if (!s || layer < 0 || layer >= s->m->c.layer_count || capacity < s->position) return 0;
    const FcModelConfig &c = s->m->c;
    int L = c.kv_lora_rank, R = c.qk_rope_dim, P = s->position;
    std::vector<__half> h((size_t)P * (L + R));
    if (P && cudaMemcpy(h.data(), s->cache + (size_t)layer * s->layer_rows * (L + R),
                        h.size() * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    for (int p = 0; p < P; ++p) {
        for (int i = 0; i < L; ++i)
            if (latent) latent[(size_t)p * L + i] = __half2float(h[(size_t)p * (L + R) + i]);
        for (int i = 0; i < R; ++i)
            if (rope) rope[(size_t)p * R + i] = __half2float(h[(size_t)p * (L + R) + L + i]);
    }
    return 1;
}

int fc_test_copy_routes(const FcSession *s, int layer, int *route_ids, int capacity) {
    if (!s || !route_ids) return 0;
    const FcModelConfig &c = s->m->c;
    if (layer < c.first_dense_layer_count || layer >= c.layer_count) return 0;
    int K = c.experts_per_token;
    if (s->route_trace_rows) {  // all rows of the last fc_test_prefill_layers
        if (capacity < s->route_trace_rows) return 0;
        memcpy(route_ids, s->route_trace.data() + (size_t)layer * s->route_trace_rows * K,
               (size_t)s->route_trace_rows * K * 4);
        return 1;
    }
    if (capacity < s->last_rows) return 0;
    return cudaMemcpy(route_ids, s->route_ids + (size_t)layer * s->rows_max * K,
                      (size_t)s->last_rows * K * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
}

int fc_test_copy_layer_outputs(const FcSession *s, float *outputs, int capacity_rows) {
    if (!s || !outputs || capacity_rows < s->last_rows || !s->trace) return 0;
    const FcModelConfig &c = s->m->c;
    int D = c.hidden_size;
    for (int l = 0; l < c.layer_count; ++l)
        if (cudaMemcpy(outputs + (size_t)l * s->last_rows * D,
                       s->layer_out + (size_t)l * s->rows_max * D, (size_t)s->last_rows * D * 4,
                       cudaMemcpyDeviceToHost) != cudaSuccess)
            return 0;
    return 1;
}

// ---- spec-runtime shim (deepseek_v4_runtime.h:72-256) ----
}  // extern "C"
namespace {
cudaError_t mtp_history_rows(FcSession *s, int p0, int r);
int mtp_finish(FcSession *s);
}  // namespace
extern "C" {

int fc_runtime_init(FcRuntime *rt, FcModel *m, int max_context, int max_batch) {
    if (!rt || !m || max_context <= 0) return 0;
    memset(rt, 0, sizeof(*rt));
    FcOptions o{max_context, std::max(1, std::min(max_batch, max_context))};
    char err[256];
    if (!fc_session_create(&rt->session, m, &o, err, sizeof(err))) return 0;
    rt->vocab_size = m->c.vocab_size;
    rt->max_context = max_context;
    rt->logits = (float *)malloc((size_t)rt->vocab_size * 4);
    if (!rt->logits) {
        fc_session_destroy(rt->session);
        memset(rt, 0, sizeof(*rt));
        return 0;
    }
    return 1;
}

int fc_runtime_forward(FcRuntime *rt, const int *ids, int n, const float **logits) {
    if (!rt || !rt->session || !ids || n <= 0 ||
        fc_session_position(rt->session) + n > rt->max_context)
        return 0;
    char err[256];
    int start = fc_session_position(rt->session);
    int done = 0;
    while (done < n) {
        int chunk = std::min(n - done, rt->session->opt.max_batch);
        int ok = fc_session_position(rt->session) == 0
                     ? fc_session_prefill(rt->session, ids + done, chunk, rt->logits, err, sizeof(err))
                     : fc_session_append(rt->session, ids + done, chunk, rt->logits, err, sizeof(err));
        if (!ok) return 0;
        done += chunk;
    }
    rt->last_start_position = start;
    rt->last_count = n;
    // a prefilled drafter follows the target: its cache gains the pairs
    // (hidden row q - 1, token q) of the new positions (the reference
    // appends its DSpark main KV the same way, deepseek_v4_runtime.h:171-176)
    if (rt->dspark_ready && start > 0) {
        FcSession *s = rt->session;
        for (int q0 = start; q0 < start + n; q0 += s->rows_max) {
            const int r = std::min(s->rows_max, start + n - q0);
            if (mtp_history_rows(s, q0 - 1, r) != cudaSuccess || !mtp_finish(s)) return 0;
        }
    }
    if (logits) *logits = rt->logits;
    return 1;
}

int fc_runtime_argmax(const float *logits, int vocab_size) {
    if (!logits || vocab_size <= 0) return -1;
    int best = 0;
    for (int t = 1; t < vocab_size; ++t)
        if (logits[t] > logits[best]) best = t;
    return best;
}

int fc_runtime_verify_token(const float *logits, int vocab_size, int64_t proposal, int *accepted) {
    int base = fc_runtime_argmax(logits, vocab_size);
    if (accepted) *accepted = base >= 0 && proposal == base;
    return base;
}

void fc_runtime_reset(FcRuntime *rt) {
    if (!rt || !rt->session) return;
    fc_session_reset(rt->session);
    rt->last_count = 0;
    rt->last_start_position = 0;
    rt->dspark_ready = 0;
}

void fc_runtime_free(FcRuntime *rt) {
    if (!rt) return;
    if (rt->session) fc_session_destroy(rt->session);
    free(rt->logits);
    memset(rt, 0, sizeof(*rt));
}

}  // extern "C"

namespace {

// The MTP drafter layer over `r` (<= rows_max) consecutive positions
// p0 + 1 .. p0 + r of the session's own history: row i takes the final
// hidden row of position p0 + i and the token at position p0 + 1 + i, the
// pairing the drafter's steps use during a verify (record_mtp_step), and
// writes the drafter's latent KV at position p0 + 1 + i.  Eager, on the
// session stream.
cudaError_t mtp_history_rows(FcSession *s, int p0, int r) {
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    cudaStream_t st = s->stream;
    const int D = c.hidden_size, kp2 = kpad(2 * D), lm = c.layer_count;
    DevLayer &y = m->layers[lm];
    Staging *h = s->h_stage;
    memset(h, 0, sizeof(*h));
    h->pos = p0 + 1;
    h->rows = r;
    h->k = -1;
    h->temperature = 1.0f;
    for (int i = 0; i < r; ++i) {
        h->ids[i] = s->tok_hist[p0 + 1 + i];
        h->rowpos[i] = p0 + 1 + i;
    }
    h->group_rows = r;
    h->groups = 1;
    FC_TRY(cudaMemcpyAsync(s->d_mtp, h, sizeof(Staging), cudaMemcpyHostToDevice, st));
    FC_TRY(launch_pdl(embed_kernel, embed_grid(r, D), dim3(kEmbedThreads), 0, st, m->embed.fmt, (const uint8_t *)m->embed.w, D,
                      m->embed.kp, (const int *)s->d_mtp->ids, s->resid));
    FC_TRY(cudaMemsetAsync(s->mtp_xq, 0, (size_t)r * kp2 * 4, st));
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(r), dim3(norm_threads(D)), 0, st, (const float *)s->resid, D,
                      (const float *)y.enorm.p, D, c.rms_norm_epsilon, s->mtp_xq, kp2, (float *)nullptr, 0));
    FC_TRY(launch_pdl(rmsnorm_kernel, dim3(r), dim3(norm_threads(D)), 0, st, (const float *)(s->hist + (size_t)p0 * D),
                      D, (const float *)y.hnorm.p, D, c.rms_norm_epsilon, s->mtp_xq + (size_t)D * 2, kp2,
                      (float *)nullptr, 0));
    GemvSeg g = seg_of(y.eh_proj, s->mtp_xq, EPI_STORE);
    g.y = s->resid;
    g.ldy = D;
    FC_TRY(gemv1(c.dense_format, g, r, 0.0f, s->d_err, m->sms, st));
    return record_layer(s, r, lm, s->d_mtp);
}

int mtp_finish(FcSession *s) {
    cudaError_t e = cudaStreamSynchronize(s->stream);
    int flag = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&flag, s->d_err, 4, cudaMemcpyDeviceToHost);
    if (flag) {
        cudaMemset(s->d_err, 0, 4);
        cudaMemset(s->route_arrivals, 0, sizeof(int));
    }
    return e == cudaSuccess && !flag;
}

}  // namespace

extern "C" {

int fc_runtime_dspark_prefill(FcRuntime *rt) {
    if (!rt || !rt->session || rt->dspark_ready || rt->last_count <= 0 || rt->last_start_position != 0)
        return 0;
    FcSession *s = rt->session;
    if (s->m->c.mtp_layers != 1 || !s->hist || s->m->world != 1) return 0;
    cudaSetDevice(s->m->device);
    const int pairs = rt->last_count - 1;
    for (int p0 = 0; p0 < pairs; p0 += s->rows_max) {
        const int r = std::min(s->rows_max, pairs - p0);
        if (mtp_history_rows(s, p0, r) != cudaSuccess || !mtp_finish(s)) return 0;
    }
    s->stats.command_buffers++;
    rt->dspark_ready = 1;
    return 1;
}

int fc_runtime_dspark_propose(FcRuntime *rt, int input_id, int64_t output_ids[6], float confidence[5]) {
    enum { kDraft = 5 };
    if (!rt || !rt->session || !rt->dspark_ready || rt->last_count <= 0 || input_id < 0) return 0;
    FcSession *s = rt->session;
    FcModel *m = s->m;
    if (input_id >= m->c.vocab_size) return 0;
    const int p = rt->last_start_position + rt->last_count - 1;  // the current row
    if (p + kDraft >= s->opt.context_size) return 0;
    cudaSetDevice(m->device);
    const int D = m->c.hidden_size;
    cudaStream_t st = s->stream;
    // the drafter's inputs as if a verify had just committed the current row:
    // main position p with commit 1, next token input_id, hidden row p
    Staging *h = s->h_stage;
    memset(h, 0, sizeof(*h));
    h->pos = p;
    h->rows = 1;
    h->k = -1;
    h->group_rows = 1;
    h->groups = 1;
    Result *res = s->h_res;
    memset(res, 0, sizeof(*res));
    res->commit = 1;
    res->next_token = input_id;
    cudaError_t e = cudaMemcpyAsync(s->d_stage, h, sizeof(Staging), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->d_res, res, sizeof(Result), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(s->resid, s->hist + (size_t)p * D, (size_t)D * 4, cudaMemcpyDeviceToDevice, st);
    for (int i = 0; i < kDraft && e == cudaSuccess; ++i) e = record_mtp_step(s, i);
    if (e == cudaSuccess) e = cudaMemcpyAsync(res, s->d_res, sizeof(Result), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess || !mtp_finish(s)) return 0;
    s->stats.command_buffers++;
    if (output_ids) {
        output_ids[0] = input_id;
        for (int i = 0; i < kDraft; ++i) output_ids[i + 1] = res->drafts[i];
    }
    if (confidence)
        for (int i = 0; i < kDraft; ++i) confidence[i] = res->draft_conf[i];
    return 1;
}

}  // extern "C"

// ===========================================================================
// single-kernel entry points (include/floyd_kernels.h)
// ===========================================================================
namespace {

__global__ void to_xq_kernel(const float *x, int S, int K, int kp, __half *xq) {
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= S * K) return;
    store_xq(xq, kp, idx / K, idx % K, x[idx]);
}

__global__ void to_f16_kernel(const float *x, size_t n, __half *y) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2half_rn(fminf(fmaxf(x[i], -65504.0f), 65504.0f));
}

// fc_matmul for S > 8 rows: the prefill GEMM on the tensor cores.
int matmul_gemm(int format, float *y, const float *x, const DevMat &mm, const std::vector<uint8_t> &image, int O,
                int K, int S, char *error, size_t error_size) {
    const int Sp = (S + kPfM - 1) / kPfM * kPfM;
    uint8_t *dw = nullptr;
    float *dx = nullptr, *dy = nullptr;
    __half *dx16 = nullptr;
    int *derr = nullptr;
    bool ok = cudaMalloc(&dw, image.size()) == cudaSuccess && cudaMalloc(&dx, (size_t)S * K * 4) == cudaSuccess &&
              cudaMalloc(&dy, (size_t)S * O * 4) == cudaSuccess &&
              cudaMalloc(&dx16, (size_t)Sp * K * 2) == cudaSuccess && cudaMalloc(&derr, 4) == cudaSuccess;
    cudaError_t e = cudaErrorMemoryAllocation;
    int herr = 0;
    CUtensorMap map{};
    if (ok) e = pf_prepare_all();
    if (ok && e == cudaSuccess && !make_map_f16(&map, dx16, (uint64_t)K, (uint64_t)Sp, kPfM)) e = cudaErrorInvalidValue;
    if (ok && e == cudaSuccess) {
        cudaMemcpy(dw, image.data(), image.size(), cudaMemcpyHostToDevice);
        cudaMemcpy(dx, x, (size_t)S * K * 4, cudaMemcpyHostToDevice);
        cudaMemset(dx16, 0, (size_t)Sp * K * 2);
        cudaMemset(derr, 0, 4);
        const size_t n = (size_t)S * K;
        to_f16_kernel<<<(unsigned)((n + 255) / 256), 256>>>(dx, n, dx16);
        PfGemm p{};
        p.tiles_per_group = (O + kTileRows - 1) / kTileRows;
        p.kp = mm.kp;
        p.N = O;
        p.K = mm.kp;
        p.groups = 1;
        p.rows = S;
        p.out = dy;
        p.out_ld = O;
        p.err = derr;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        CUtensorMap wmap{};
        p.box_tiles = std::min(16, p.tiles_per_group);
        if (!make_map_weights(&wmap, dw, format, (uint64_t)p.tiles_per_group, mm.kp, (uint32_t)p.box_tiles))
            e = cudaErrorInvalidValue;
        else e = pf_gemm(format, PF_STORE_F32, map, wmap, wmap, p, sms, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(y, dy, (size_t)S * O * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(dw); cudaFree(dx); cudaFree(dy); cudaFree(dx16); cudaFree(derr);
    if (e == cudaSuccess && herr) return set_error(error, error_size, "a kernel wait gave up (0x%x)", herr);
    if (e != cudaSuccess) return set_error(error, error_size, "matmul failed: %s", cudaGetErrorString(e));
    return 1;
}

}  // namespace

extern "C" int fc_matmul(int format, float *y, const float *x, const void *values,
                         const void *scales, int O, int K, int S, char *error,
                         size_t error_size) {
    if (!y || !x || !values || !scales || O <= 0 || K <= 0 || K % 32 || S < 1 || (S > kMaxRows && O % 32))
        return set_error(error, error_size, "invalid matmul shape");
    if (format != FC_FMT_Q8 && format != FC_FMT_Q4 && format != FC_FMT_MXFP4)
        return set_error(error, error_size, "unsupported format %d", format);
    DevMat mm;
    plan_mat(mm, format, O, K, 1, 0, 0);
    std::vector<uint8_t> image(mm.w_bytes, 0);
    pack_values(mm, reinterpret_cast<const uint8_t *>(values), image.data());
    pack_scales(mm, reinterpret_cast<const uint8_t *>(scales), image.data());
    if (S > kMaxRows) return matmul_gemm(format, y, x, mm, image, O, K, S, error, error_size);
    uint8_t *dw = nullptr;
    float *dx = nullptr, *dy = nullptr;
    __half *dxq = nullptr;
    int *derr = nullptr;
    size_t xq_bytes = (size_t)S * mm.kp * 2 * sizeof(__half);
    bool ok = cudaMalloc(&dw, image.size()) == cudaSuccess &&
              cudaMalloc(&dx, (size_t)S * K * 4) == cudaSuccess &&
              cudaMalloc(&dy, (size_t)S * O * 4) == cudaSuccess &&
              cudaMalloc(&dxq, xq_bytes) == cudaSuccess && cudaMalloc(&derr, 4) == cudaSuccess;
    cudaError_t e = cudaErrorMemoryAllocation;
    int herr = 0;
    if (ok) e = gemv_prepare_all();
    if (ok && e == cudaSuccess) {
        cudaMemcpy(dw, image.data(), image.size(), cudaMemcpyHostToDevice);
        cudaMemcpy(dx, x, (size_t)S * K * 4, cudaMemcpyHostToDevice);
        cudaMemset(dxq, 0, xq_bytes);
        cudaMemset(derr, 0, 4);
        to_xq_kernel<<<(S * K + 255) / 256, 256>>>(dx, S, K, mm.kp, dxq);
        GemvSeg g = seg_of(mm, dxq, EPI_STORE);
        g.w = dw;
        g.y = dy;
        g.ldy = O;
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        e = gemv1(format, g, S, 0.0f, derr, sms, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(y, dy, (size_t)S * O * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(dw); cudaFree(dx); cudaFree(dy); cudaFree(dxq); cudaFree(derr);
    if (e == cudaSuccess && herr) return set_error(error, error_size, "a kernel wait gave up");
    if (e != cudaSuccess) return set_error(error, error_size, "matmul failed: %s", cudaGetErrorString(e));
    return 1;
}

// ===========================================================================
// fc_test_accept: the acceptance kernels of the verify graph on caller-given
// logits, for `trials` consecutive Philox counters (test hook).
// ===========================================================================
extern "C" int fc_test_accept(const float *logits, int rows, int vocab, const int *ids,
                              const FcAcceptConfig *accept, int trials, int *commits,
                              int *next_tokens, char *error, size_t error_size) {
    if (!logits || !ids || !accept || !commits || !next_tokens || rows < 1 || rows > kMaxRows ||
        vocab < 1 || trials < 1)
        return set_error(error, error_size, "invalid acceptance test arguments");
    if (accept->mode == FC_ACCEPT_SAMPLE && !(accept->temperature > 0.0f))
        return set_error(error, error_size, "sampling needs a temperature > 0");
    const int chunks = (vocab + kHeadChunk - 1) / kHeadChunk;
    const size_t part = (size_t)rows * chunks;
    float *d_logits = nullptr, *d_f = nullptr;
    int *d_i = nullptr, *d_err = nullptr;
    Staging *d_st = nullptr;
    Result *d_res = nullptr;
    cudaError_t e = cudaMalloc(&d_logits, (size_t)rows * vocab * 4);
    if (e == cudaSuccess) e = cudaMalloc(&d_f, part * 4 * 4);
    if (e == cudaSuccess) e = cudaMalloc(&d_i, part * 2 * 4);
    if (e == cudaSuccess) e = cudaMalloc(&d_err, 4);
    if (e == cudaSuccess) e = cudaMalloc(&d_st, sizeof(Staging));
    if (e == cudaSuccess) e = cudaMalloc(&d_res, sizeof(Result));
    if (e == cudaSuccess) e = cudaMemcpy(d_logits, logits, (size_t)rows * vocab * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(d_err, 0, 4);
    HeadPartials hp{};
    hp.amax = d_f; hp.zmax = d_f + part; hp.zsum = d_f + 2 * part; hp.gval = d_f + 3 * part;
    hp.aidx = d_i; hp.gidx = d_i + part;
    Staging h{};
    h.rows = rows;
    h.k = rows - 1;
    h.mode = accept->mode;
    h.temperature = accept->mode == FC_ACCEPT_SAMPLE ? accept->temperature : 1.0f;
    h.seed = accept->seed;
    h.group_rows = rows;
    h.groups = 1;
    for (int r = 0; r < rows; ++r) h.ids[r] = ids[r];
    Result res{};
    for (int t = 0; t < trials && e == cudaSuccess; ++t) {
        h.counter = accept->counter + (unsigned long long)t;
        h.gcounter[0] = h.counter;
        e = cudaMemcpy(d_st, &h, sizeof(Staging), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) break;
        head_partial_kernel<<<dim3(chunks, rows), 256>>>(d_logits, vocab, d_st, hp, chunks);
        accept_kernel<<<1, 256>>>(d_logits, vocab, d_st, hp, chunks, d_res, d_err);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpy(&res, d_res, sizeof(Result), cudaMemcpyDeviceToHost);
        commits[t] = res.commit;
        next_tokens[t] = res.next_token;
    }
    cudaFree(d_logits); cudaFree(d_f); cudaFree(d_i); cudaFree(d_err); cudaFree(d_st); cudaFree(d_res);
    if (e != cudaSuccess) return set_error(error, error_size, "acceptance test failed: %s", cudaGetErrorString(e));
    return 1;
}

// ===========================================================================
// fc_matmul_noalloc: fc_matmul for callers that must not allocate device
// memory.  Its working memory is one fixed file-scope device array.
// ===========================================================================
namespace {

constexpr size_t kNoAllocImage = (size_t)6 << 20;    // tile-major weight image
constexpr size_t kNoAllocValues = (size_t)6 << 20;   // logical values as passed
constexpr size_t kNoAllocScales = (size_t)512 << 10; // logical group scales
constexpr size_t kNoAllocX = (size_t)256 << 10;      // fp32 activations
constexpr size_t kNoAllocXq = (size_t)512 << 10;     // hi/lo fp16 activations
constexpr size_t kNoAllocY = (size_t)512 << 10;      // fp32 outputs
constexpr size_t kNoAllocOffValues = kNoAllocImage;
constexpr size_t kNoAllocOffScales = kNoAllocOffValues + kNoAllocValues;
constexpr size_t kNoAllocOffX = kNoAllocOffScales + kNoAllocScales;
constexpr size_t kNoAllocOffXq = kNoAllocOffX + kNoAllocX;
constexpr size_t kNoAllocOffY = kNoAllocOffXq + kNoAllocXq;
constexpr size_t kNoAllocOffErr = kNoAllocOffY + kNoAllocY;
constexpr size_t kNoAllocBytes = kNoAllocOffErr + 256;

// Every GPU that loads this library holds this array (about 14 MiB) until
// the process exits.  Host code must not pass the symbol itself to a kernel:
// on the host it names a stand-in, not device memory.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

constexpr int kNoAllocMaxDevices = 64;
uint8_t *g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};

// Scatters logical values (int8 [O][K], or packed nibbles [O][K/2] with the
// even element low) into the zeroed tile-major image.  One thread per group
// of 4 consecutive columns: the device bytes holding those nibbles hold no
// other element, so every byte is written by exactly one thread.
__global__ void noalloc_pack_values(int fmt, int O, int K, int kp, const uint8_t *src,
                                    uint8_t *image) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t groups = (size_t)O * K / 4;
    if (idx >= groups) return;
    size_t e0 = idx * 4;
    int o = (int)(e0 / K), k0 = (int)(e0 % K);
    size_t off[4];
    int nib[4];
    uint32_t val[4];
    for (int i = 0; i < 4; ++i) {
        size_t e = e0 + i;
        off[i] = value_offset(fmt, kp, o, k0 + i, &nib[i]);
        val[i] = fmt == FC_FMT_Q8 ? src[e] : (src[e >> 1] >> (4 * (e & 1))) & 15u;
    }
    for (int i = 0; i < 4; ++i) {
        bool first = true;
        for (int jx = 0; jx < i; ++jx) first = first && off[jx] != off[i];
        if (!first) continue;
        uint32_t b = 0;
        for (int m = i; m < 4; ++m)
            if (off[m] == off[i]) b |= fmt == FC_FMT_Q8 ? val[m] : val[m] << (4 * nib[m]);
        image[off[i]] = (uint8_t)b;
    }
}

__global__ void noalloc_pack_scales(int fmt, int O, int K, int kp, const uint8_t *src,
                                    uint8_t *image) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    int gk = K / 32, el = scale_elem_bytes(fmt);
    if (idx >= (size_t)O * gk) return;
    int o = (int)(idx / gk), g = (int)(idx % gk);
    uint8_t *dst = image + scale_offset(fmt, kp, o, g);
    for (int b = 0; b < el; ++b) dst[b] = src[idx * el + b];
}

}  // namespace

extern "C" int fc_matmul_noalloc(int format, float *y, const float *x, const void *values,
                                 const void *scales, int O, int K, int S, char *error,
                                 size_t error_size) {
    if (!y || !x || !values || !scales || O <= 0 || K <= 0 || K % 32 || S < 1)
        return set_error(error, error_size, "invalid matmul shape");
    if (S > kMaxRows)
        return set_error(error, error_size,
                         "S=%d exceeds the %d-row limit of the no-allocation path "
                         "(fc_matmul takes wider inputs)", S, kMaxRows);
    if (format != FC_FMT_Q8 && format != FC_FMT_Q4 && format != FC_FMT_MXFP4)
        return set_error(error, error_size, "unsupported format %d", format);
    const int kp = kpad(K);
    const size_t image = matrix_bytes(format, O, kp);
    const size_t vbytes = format == FC_FMT_Q8 ? (size_t)O * K : (size_t)O * K / 2;
    const size_t sbytes = (size_t)O * (K / 32) * scale_elem_bytes(format);
    if (image > kNoAllocImage || vbytes > kNoAllocValues || sbytes > kNoAllocScales ||
        (size_t)S * K * 4 > kNoAllocX || (size_t)S * kp * 4 > kNoAllocXq ||
        (size_t)S * O * 4 > kNoAllocY)
        return set_error(error, error_size,
                         "matmul of %d x %d (S=%d) exceeds the fixed no-allocation workspace "
                         "(weight image <= %zu bytes, S*K*4 <= %zu, S*O*4 <= %zu)",
                         O, K, S, kNoAllocImage, kNoAllocX, kNoAllocY);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
        return set_error(error, error_size, "no usable CUDA device");
    // One-time set-up on this device: the array's device address.
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return set_error(error, error_size, "cannot resolve the workspace address: %s",
                             cudaGetErrorString(e));
        g_noalloc_ptr[dev] = reinterpret_cast<uint8_t *>(p);
    }
    uint8_t *base = g_noalloc_ptr[dev];
    uint8_t *d_image = base, *d_values = base + kNoAllocOffValues, *d_scales = base + kNoAllocOffScales;
    float *d_x = reinterpret_cast<float *>(base + kNoAllocOffX);
    __half *d_xq = reinterpret_cast<__half *>(base + kNoAllocOffXq);
    float *d_y = reinterpret_cast<float *>(base + kNoAllocOffY);
    int *d_err = reinterpret_cast<int *>(base + kNoAllocOffErr);
    int sms = 148, herr = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e = gemv_prepare_all();
    // The array keeps the previous call's contents: clear what must start at zero
    // (image padding, xq padding, error flag).
    if (e == cudaSuccess) e = cudaMemset(d_image, 0, image);
    if (e == cudaSuccess) e = cudaMemset(d_xq, 0, (size_t)S * kp * 4);
    if (e == cudaSuccess) e = cudaMemset(d_err, 0, 4);
    if (e == cudaSuccess) e = cudaMemcpy(d_values, values, vbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d_scales, scales, sbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d_x, x, (size_t)S * K * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        size_t groups = (size_t)O * K / 4;
        noalloc_pack_values<<<(unsigned)((groups + 255) / 256), 256>>>(format, O, K, kp, d_values, d_image);
        size_t ng = (size_t)O * (K / 32);
        noalloc_pack_scales<<<(unsigned)((ng + 255) / 256), 256>>>(format, O, K, kp, d_scales, d_image);
        to_xq_kernel<<<(S * K + 255) / 256, 256>>>(d_x, S, K, kp, d_xq);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        DevMat mm;
        plan_mat(mm, format, O, K, 1, 0, 0);
        GemvSeg g = seg_of(mm, d_xq, EPI_STORE);
        g.w = d_image;
        g.y = d_y;
        g.ldy = O;
        e = gemv1(format, g, S, 0.0f, d_err, sms, 0);
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(y, d_y, (size_t)S * O * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_error(error, error_size, "matmul failed: %s", cudaGetErrorString(e));
    if (herr) return set_error(error, error_size, "a kernel wait gave up");
    return 1;
}

#ifdef FC_TC_TRACE
extern "C" int fc_debug_tc_trace(unsigned long long *out, int n) {
    return cudaMemcpyFromSymbol(out, g_tc_trace, sizeof(unsigned long long) * (n < 256 ? n : 256)) == cudaSuccess;
}
#endif

#ifdef FC_GEMV_TRACE
extern "C" int fc_debug_gemv_trace(int items, unsigned long long *out, int n) {
    if (!out) {
        g_host_trace_items = items;
        return 1;
    }
    return cudaMemcpyFromSymbol(out, g_gemv_trace, sizeof(unsigned long long) * (n < 512 ? n : 512)) == cudaSuccess;
}
#endif

#include "hooks.cuh"
#include "fm.cuh"
