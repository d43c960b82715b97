// hooks.cuh - per-primitive test hooks of a session, the counterparts of
// moonlight_test_* (moonlight_metal.h:67-92): each runs one piece of the
// forward (embedding, RMSNorm, one matrix, the attention block of a layer,
// the MoE or dense MLP of a layer, the prefill with per-layer outputs) on
// the device, eagerly on the session stream, and copies the result to host
// arrays.  The reference's Metal tests (tests/test_moonlight_metal_*.c)
// assert against exactly these outputs.
//
// Included at the end of runtime.cu: the hooks reuse the forward's own
// recording functions (record_attention, record_ffn) and kernels, so they
// test the code the forward runs.  Rows beyond one pass (8) run in passes
// of 8 in position order.  Scratch buffers of a hook call are allocated and
// freed by that call (the session's own buffers stay as they were).
#pragma once

namespace {

struct HookScratch {
    std::vector<void *> ptrs;
    ~HookScratch() {
        for (void *p : ptrs) cudaFree(p);
    }
    template <typename T>
    T *get(size_t count) {
        void *p = nullptr;
        if (cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, std::max<size_t>(count, 1) * sizeof(T));
        ptrs.push_back(p);
        return reinterpret_cast<T *>(p);
    }
};

// Per-pass parameters of a hook: `rows` rows at positions pos .. pos+rows-1
// of sequence 0, no acceptance.
cudaError_t hook_stage(FcSession *s, int pos, int rows, const int *ids) {
    Staging *st = s->h_stage;
    memset(st, 0, sizeof(*st));
    st->pos = pos;
    st->rows = rows;
    st->k = -1;
    st->mode = FC_ACCEPT_GREEDY;
    st->temperature = 1.0f;
    for (int i = 0; i < rows; ++i) {
        st->ids[i] = ids ? ids[i] : 0;
        st->rowpos[i] = pos + i;
        st->rowseq[i] = 0;
    }
    st->group_rows = rows;
    st->groups = 1;
    return cudaMemcpyAsync(s->d_stage, s->h_stage, sizeof(Staging), cudaMemcpyHostToDevice, s->stream);
}

// fp32 rows [rows][K] from the host into the xq operand buffer [rows][kpad(K)].
cudaError_t hook_xq(FcSession *s, const float *host, int rows, int K, float *dev_f32, __half *xq) {
    FC_TRY(cudaMemcpyAsync(dev_f32, host, (size_t)rows * K * 4, cudaMemcpyHostToDevice, s->stream));
    FC_TRY(cudaMemsetAsync(xq, 0, (size_t)rows * kpad(K) * 4, s->stream));
    to_xq_kernel<<<(rows * K + 255) / 256, 256, 0, s->stream>>>(dev_f32, rows, K, kpad(K), xq);
    return cudaGetLastError();
}

// Waits for the hook's work and folds in the kernels' error flag.
int hook_finish(FcSession *s, cudaError_t e) {
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    int flag = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&flag, s->d_err, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && flag) {
        cudaMemset(s->d_err, 0, 4);
        cudaMemset(s->route_arrivals, 0, sizeof(int));
        return 0;
    }
    return e == cudaSuccess ? 1 : 0;
}

bool hook_ready(const FcSession *s) { return s && !s->batch && s->m->world == 1; }

}  // namespace

extern "C" {

int fc_test_embed(FcSession *s, const int *ids, int count, float *output) {
    if (!hook_ready(s) || !ids || !output || count <= 0 || count > s->opt.max_batch) return 0;
    FcModel *m = s->m;
    const int D = m->c.hidden_size;
    for (int i = 0; i < count; ++i)
        if (ids[i] < 0 || ids[i] >= m->c.vocab_size) return 0;
    cudaSetDevice(m->device);
    HookScratch hs;
    int *d_ids = hs.get<int>(count);
    float *d_x = hs.get<float>((size_t)count * D);
    if (!d_ids || !d_x) return 0;
    cudaError_t e = cudaMemcpyAsync(d_ids, ids, (size_t)count * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess)
        e = launch_pdl(embed_kernel, embed_grid(count, D), dim3(kEmbedThreads), 0, s->stream, m->embed.fmt,
                       (const uint8_t *)m->embed.w, D, m->embed.kp, (const int *)d_ids, d_x);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(output, d_x, (size_t)count * D * 4, cudaMemcpyDeviceToHost, s->stream);
    s->stats.command_buffers++;
    return hook_finish(s, e);
}

int fc_test_rmsnorm(FcSession *s, const float *input, const char *weight_name, int rows, int width,
                    float *output) {
    if (!hook_ready(s) || !input || !weight_name || !output || rows <= 0 || rows > s->opt.max_batch ||
        width <= 0 || width % 4)
        return 0;
    FcModel *m = s->m;
    auto it = m->names.find(weight_name);
    if (it == m->names.end() || !it->second.vec || it->second.vec->n != (size_t)width) return 0;
    cudaSetDevice(m->device);
    HookScratch hs;
    float *d_x = hs.get<float>((size_t)rows * width), *d_y = hs.get<float>((size_t)rows * width);
    __half *d_q = hs.get<__half>((size_t)rows * kpad(width) * 2);
    if (!d_x || !d_y || !d_q) return 0;
    cudaError_t e = cudaMemcpyAsync(d_x, input, (size_t)rows * width * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess)
        e = launch_pdl(rmsnorm_kernel, dim3(rows), dim3(norm_threads(width)), 0, s->stream, (const float *)d_x,
                       width, (const float *)it->second.vec->p, width, m->c.rms_norm_epsilon, d_q, kpad(width),
                       d_y, width);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(output, d_y, (size_t)rows * width * 4, cudaMemcpyDeviceToHost, s->stream);
    s->stats.command_buffers++;
    return hook_finish(s, e);
}

int fc_test_matmul(FcSession *s, const char *weight_name, const float *input, int rows, int input_width,
                   int output_width, float *output) {
    if (!hook_ready(s) || !weight_name || !input || !output || rows <= 0 || rows > s->opt.max_batch) return 0;
    FcModel *m = s->m;
    auto it = m->names.find(weight_name);
    if (it == m->names.end() || !it->second.mat) return 0;
    const DevMat &mm = *it->second.mat;
    if (mm.K != input_width || mm.O != output_width) return 0;
    cudaSetDevice(m->device);
    HookScratch hs;
    const int chunk = s->rows_max, K = mm.K, O = mm.O;
    float *d_x = hs.get<float>((size_t)chunk * K), *d_y = hs.get<float>((size_t)chunk * O);
    __half *d_q = hs.get<__half>((size_t)chunk * kpad(K) * 2);
    if (!d_x || !d_y || !d_q) return 0;
    cudaError_t e = cudaSuccess;
    for (int r0 = 0; r0 < rows && e == cudaSuccess; r0 += chunk) {
        const int r = std::min(chunk, rows - r0);
        e = hook_xq(s, input + (size_t)r0 * K, r, K, d_x, d_q);
        if (e != cudaSuccess) break;
        if (mm.fmt == FC_FMT_F32) {
            e = launch_f32_gemv(reinterpret_cast<const float *>(mm.w + (size_t)it->second.member * mm.w_bytes), O,
                                K, d_q, kpad(K), r, d_y, O, m->sms, s->stream);
        } else {
            GemvSeg g = seg_of(mm, d_q, EPI_STORE);
            g.w = mm.w + (size_t)it->second.member * mm.w_bytes;
            g.y = d_y;
            g.ldy = O;
            e = gemv1(mm.fmt, g, r, 0.0f, s->d_err, m->sms, s->stream);
        }
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(output + (size_t)r0 * O, d_y, (size_t)r * O * 4, cudaMemcpyDeviceToHost,
                                s->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    }
    s->stats.command_buffers++;
    return hook_finish(s, e);
}

// The attention block of `layer` for `rows` normalized input rows at
// positions position .. position+rows-1 (position must equal the session's
// current position, i.e. the layer's KV length); output = o_proj(attention)
// [rows][hidden].  Appends the rows' latent KV and advances the position.
int fc_test_attention(FcSession *s, int layer, const float *input, int rows, int position, float *output) {
    if (!hook_ready(s) || !input || !output || rows <= 0 || rows > s->opt.max_batch) return 0;
    FcModel *m = s->m;
    if (layer < 0 || layer >= m->c.layer_count || position != s->position ||
        position + rows > s->opt.context_size)
        return 0;
    cudaSetDevice(m->device);
    const int D = m->c.hidden_size, chunk = s->rows_max;
    HookScratch hs;
    float *d_x = hs.get<float>((size_t)chunk * D), *d_y = hs.get<float>((size_t)chunk * D);
    if (!d_x || !d_y) return 0;
    cudaError_t e = cudaSuccess;
    for (int r0 = 0; r0 < rows && e == cudaSuccess; r0 += chunk) {
        const int r = std::min(chunk, rows - r0);
        e = hook_stage(s, position + r0, r, nullptr);
        if (e == cudaSuccess) e = hook_xq(s, input + (size_t)r0 * D, r, D, d_x, s->xq_norm);
        if (e == cudaSuccess) e = record_attention(s, r, layer, s->d_stage, EPI_STORE, d_y);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(output + (size_t)r0 * D, d_y, (size_t)r * D * 4, cudaMemcpyDeviceToHost,
                                s->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    }
    s->stats.command_buffers++;
    if (!hook_finish(s, e)) return 0;
    s->position = position + rows;
    return 1;
}

// The MoE block of `layer` on `rows` normalized rows: route ids and weights
// [rows][top-k] (selection order), the raw router logits [rows][experts],
// the routed sum, the shared experts' output and their sum [rows][hidden].
int fc_test_moe(FcSession *s, int layer, const float *input, int rows, int *route_ids, float *route_weights,
                float *router_scores, float *routed_output, float *shared_output, float *output) {
    if (!hook_ready(s) || !input || !output || rows <= 0 || rows > s->opt.max_batch) return 0;
    FcModel *m = s->m;
    const FcModelConfig &c = m->c;
    if (layer < c.first_dense_layer_count || layer >= c.layer_count) return 0;
    cudaSetDevice(m->device);
    const int D = c.hidden_size, E = c.expert_count, K = c.experts_per_token, chunk = s->rows_max;
    const DevLayer &y = m->layers[layer];
    HookScratch hs;
    float *d_routed = hs.get<float>((size_t)chunk * D), *d_scores = hs.get<float>((size_t)chunk * E);
    if (!d_routed || !d_scores) return 0;
    std::vector<float> routed((size_t)chunk * D), shared((size_t)chunk * D);
    cudaError_t e = cudaSuccess;
    for (int r0 = 0; r0 < rows && e == cudaSuccess; r0 += chunk) {
        const int r = std::min(chunk, rows - r0);
        e = hook_stage(s, s->position, r, nullptr);
        if (e == cudaSuccess) e = hook_xq(s, input + (size_t)r0 * D, r, D, s->xn, s->xq_norm);
        if (e == cudaSuccess) e = cudaMemsetAsync(d_routed, 0, (size_t)r * D * 4, s->stream);
        if (e == cudaSuccess) e = record_ffn(s, r, layer, s->d_stage, d_routed, EPI_ADD, true);
        // raw router logits (the router kernel keeps scores, not logits)
        if (e == cudaSuccess)
            e = launch_f32_gemv(y.router.p, E, D, s->xq_norm, kpad(D), r, d_scores, E, m->sms, s->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
        if (e != cudaSuccess) break;
        if (router_scores)
            e = cudaMemcpy(router_scores + (size_t)r0 * E, d_scores, (size_t)r * E * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && route_ids)
            e = cudaMemcpy(route_ids + (size_t)r0 * K, s->route_ids + (size_t)layer * s->rows_max * K,
                           (size_t)r * K * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && route_weights)
            e = cudaMemcpy(route_weights + (size_t)r0 * K, s->route_w + (size_t)layer * s->rows_max * K,
                           (size_t)r * K * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(routed.data(), d_routed, (size_t)r * D * 4, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess && y.s_down.count)
            e = cudaMemcpy(shared.data(), s->sh_part, (size_t)r * D * 4, cudaMemcpyDeviceToHost);
        if (!y.s_down.count) std::fill(shared.begin(), shared.end(), 0.0f);
        for (size_t i = 0; e == cudaSuccess && i < (size_t)r * D; ++i) {
            const size_t o = (size_t)r0 * D + i;
            if (routed_output) routed_output[o] = routed[i];
            if (shared_output) shared_output[o] = shared[i];
            output[o] = routed[i] + shared[i];
        }
    }
    s->stats.command_buffers++;
    return hook_finish(s, e);
}

int fc_test_dense_mlp(FcSession *s, int layer, const float *input, int rows, float *output) {
    if (!hook_ready(s) || !input || !output || rows <= 0 || rows > s->opt.max_batch) return 0;
    FcModel *m = s->m;
    if (layer < 0 || layer >= m->c.first_dense_layer_count || layer >= m->c.layer_count) return 0;
    cudaSetDevice(m->device);
    const int D = m->c.hidden_size, chunk = s->rows_max;
    HookScratch hs;
    float *d_y = hs.get<float>((size_t)chunk * D);
    if (!d_y) return 0;
    cudaError_t e = cudaSuccess;
    for (int r0 = 0; r0 < rows && e == cudaSuccess; r0 += chunk) {
        const int r = std::min(chunk, rows - r0);
        e = hook_stage(s, s->position, r, nullptr);
        if (e == cudaSuccess) e = hook_xq(s, input + (size_t)r0 * D, r, D, s->xn, s->xq_norm);
        if (e == cudaSuccess) e = record_ffn(s, r, layer, s->d_stage, d_y, EPI_STORE, false);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(output + (size_t)r0 * D, d_y, (size_t)r * D * 4, cudaMemcpyDeviceToHost,
                                s->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    }
    s->stats.command_buffers++;
    return hook_finish(s, e);
}

// Prefill of `count` tokens (session at position 0) with the hidden state
// after every layer, [layers][count][hidden], and the last row's logits.
// Runs the verify-width passes (8 rows) so that every layer's output can be
// read back; the result equals fc_session_prefill's within its tolerance.
int fc_test_prefill_layers(FcSession *s, const int *ids, int count, float *layer_outputs, float *last_logits,
                           char *error, size_t error_size) {
    if (!hook_ready(s) || !ids || count <= 0) return set_error(error, error_size, "invalid arguments");
    if (s->position != 0) return set_error(error, error_size, "prefill requires an empty session");
    if (count > s->opt.context_size) return set_error(error, error_size, "prompt exceeds the context");
    if (!check_ids(s, ids, count, error, error_size)) return 0;
    FcModel *m = s->m;
    const int D = m->c.hidden_size, L = m->c.layer_count, chunk = s->rows_max;
    const bool keep_trace = s->trace;
    s->trace = true;
    double t0 = now_ms();
    int ok = 1;
    std::vector<float> buf((size_t)L * chunk * D);
    const int K = std::max(m->c.experts_per_token, 1);
    std::vector<int> trace((size_t)L * count * K, -1), rbuf((size_t)chunk * K);
    for (int r0 = 0; r0 < count && ok; r0 += chunk) {
        const int r = std::min(chunk, count - r0);
        ok = run_pass(s, ids + r0, r, -1, nullptr, error, error_size);
        if (!ok) break;
        s->position += r;
        for (int l = m->c.first_dense_layer_count; l < L && ok; ++l) {
            if (cudaMemcpy(rbuf.data(), s->route_ids + (size_t)l * s->rows_max * K, (size_t)r * K * 4,
                           cudaMemcpyDeviceToHost) != cudaSuccess)
                ok = set_error(error, error_size, "route copy failed");
            memcpy(&trace[((size_t)l * count + r0) * K], rbuf.data(), (size_t)r * K * 4);
        }
        if (layer_outputs) {
            if (cudaMemcpy(buf.data(), s->layer_out, buf.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
                ok = set_error(error, error_size, "layer output copy failed");
                break;
            }
            for (int l = 0; l < L; ++l)
                memcpy(layer_outputs + ((size_t)l * count + r0) * D, buf.data() + (size_t)l * chunk * D,
                       (size_t)r * D * 4);
        }
    }
    s->trace = keep_trace;
    if (ok) {
        s->route_trace.swap(trace);
        s->route_trace_rows = count;
    }
    if (ok && last_logits) {
        const int V = m->c.vocab_size;
        if (cudaMemcpy(last_logits, s->logits + (size_t)(s->last_rows - 1) * V, (size_t)V * 4,
                       cudaMemcpyDeviceToHost) != cudaSuccess)
            ok = set_error(error, error_size, "logits copy failed");
    }
    if (ok) {
        s->stats.prefill_tokens += (uint64_t)count;
        s->stats.prefill_ms += now_ms() - t0;
    }
    return ok;
}

}  // extern "C"
