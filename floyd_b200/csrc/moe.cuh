// moe.cuh - top-k router, device-side expert grouping and the grouped expert
// GEMVs of the MoE block.
//
// Replaces moonlight_route_sigmoid_topk (moonlight_kernels.metal:469-512),
// the host-side prepare_route_tables (moonlight_metal.m:525-559, a GPU->host
// round trip per layer in the reference) and the per-expert
// gather / gate / up / SiLU / down / scatter sequence of
// encode_moe_residual_buffer (moonlight_metal.m:561-676), under the
// moe_route.h / moe_exec.h contract:
//   - scores by MoeScoreFn; the selection bias changes selection only;
//   - top-k by repeated argmax, lower expert index on ties;
//   - weights normalized with +1e-20, then times routed_scale;
//   - routed experts summed in ascending expert id, then the shared experts
//     with coefficient 1 (moe_exec.h:97-110), no atomics.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace fc {

// Router logits, fp32 weights [E][D]: one block per expert row, the 256
// threads split D (float4 loads), per-row partial sums reduced in a fixed
// order (warp butterfly, then warps in index order).
__global__ void __launch_bounds__(256) router_logits_kernel(const float *W, const float *x, int E,
                                                            int D, int S, float *logits) {
    pdl_wait();
    pdl_release();
    __shared__ float red[8][8];
    const int e = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float acc[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) acc[s] = 0.0f;
    const float4 *w4 = reinterpret_cast<const float4 *>(W + (size_t)e * D);
    for (int k4 = threadIdx.x; k4 < D / 4; k4 += blockDim.x) {
        float4 w = __ldg(w4 + k4);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            if (s < S) {
                float4 xv = *reinterpret_cast<const float4 *>(x + (size_t)s * D + 4 * k4);
                acc[s] = fmaf(w.x, xv.x, acc[s]);
                acc[s] = fmaf(w.y, xv.y, acc[s]);
                acc[s] = fmaf(w.z, xv.z, acc[s]);
                acc[s] = fmaf(w.w, xv.w, acc[s]);
            }
        }
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        float v = warp_sum(acc[s]);
        if (lane == 0) red[warp][s] = v;
    }
    __syncthreads();
    if (threadIdx.x < S) {
        float t = 0.0f;
        for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
        logits[(size_t)threadIdx.x * E + e] = t;
    }
}

struct RouteParams {
    int E, K, S;
    int score_fn, normalize;
    float routed_scale;
    const float *bias;       // nullable
    const int *hash;         // nullable [vocab][K] (fixed routes)
    const int *ids;          // token ids [S] (hash routing)
    int expert_lo, expert_hi;  // experts owned by this rank [lo, hi)
    int *route_ids;          // [S][K] selection order
    float *route_w;          // [S][K]
    int *n_active;           // number of local active experts
    int *active;             // [max_slots] ascending expert ids (local range)
    float *coef;             // [max_slots][8] coefficient of slot for row s
};

__device__ __forceinline__ float route_score(float x, int fn) {
    if (fn == FC_SCORE_SQRT_SOFTPLUS) {
        float sp;
        if (x > 20.0f) sp = x;
        else if (x < -20.0f) sp = expf(x);
        else sp = log1pf(expf(x));
        return sqrtf(sp);
    }
    return 1.0f / (1.0f + expf(-x));
}

// One block of 256 threads; warp s handles row s (S <= 8).  Scores are
// computed lane-parallel with fixed-order warp reductions, top-k by repeated
// warp argmax (lower index on ties), finalize in slot order on lane 0; then
// the ascending list of active local experts and their per-row coefficients
// come from a block-wide scan.
constexpr int kRouteThreads = 256;

__global__ void __launch_bounds__(kRouteThreads) route_select_kernel(const float *logits, RouteParams p) {
    pdl_wait();
    pdl_release();
    extern __shared__ float rs_smem[];  // scores [8][E], choice [8][E]
    __shared__ int used_flag[1024];
    __shared__ int slot_of[1024];
    __shared__ int warp_total[kRouteThreads / 32];
    __shared__ int sel[8][64];
    __shared__ float selw[8][64];
    const int E = p.E, K = p.K;
    float *scores = rs_smem;
    float *choice = rs_smem + 8 * E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) used_flag[e] = 0;
    for (int i = threadIdx.x; i < p.S * E; i += blockDim.x) choice[i] = logits[i];
    __syncthreads();
    if (warp < p.S) {
        const int s = warp;
        float *lg = choice + s * E;
        float *sc = scores + s * E;
        float *ch = choice + s * E;
        if (p.score_fn == FC_SCORE_SOFTMAX) {  // moe_route.h:26-37
            float m = -INFINITY;
            for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e]);
            m = warp_max(m);
            float sum = 0.0f;
            for (int e = lane; e < E; e += 32) {
                float v = expf(lg[e] - m);
                sc[e] = v;
                sum += v;
            }
            sum = warp_sum(sum);
            __syncwarp();
            for (int e = lane; e < E; e += 32) sc[e] = sc[e] / sum;
        } else {
            for (int e = lane; e < E; e += 32) sc[e] = route_score(lg[e], p.score_fn);
        }
        __syncwarp();
        for (int e = lane; e < E; e += 32) ch[e] = sc[e] + (p.bias ? p.bias[e] : 0.0f);
        __syncwarp();
        if (p.hash) {
            if (lane < K) {
                int e = p.hash[(size_t)p.ids[s] * K + lane];
                sel[s][lane] = e;
                selw[s][lane] = sc[e];
            }
        } else {
            for (int k = 0; k < K; ++k) {
                float best = -INFINITY;
                int bi = 0x7fffffff;
                for (int e = lane; e < E; e += 32) {
                    bool taken = false;
                    for (int t = 0; t < k; ++t) taken |= sel[s][t] == e;
                    float v = ch[e];
                    if (!taken && v > best) { best = v; bi = e; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    float ov = __shfl_xor_sync(0xffffffffu, best, o);
                    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
                }
                if (lane == 0) {
                    sel[s][k] = bi;
                    selw[s][k] = sc[bi];
                }
                __syncwarp();
            }
        }
        __syncwarp();
        if (lane == 0) {  // moe_route_finalize, moe_route.h:89-99
            float sum = 0.0f;
            if (p.normalize) {
                for (int k = 0; k < K; ++k) sum += selw[s][k];
                sum += 1e-20f;
            }
            for (int k = 0; k < K; ++k) {
                float w = p.normalize ? selw[s][k] / sum : selw[s][k];
                w = w * p.routed_scale;
                p.route_ids[s * K + k] = sel[s][k];
                p.route_w[s * K + k] = w;
                selw[s][k] = w;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < p.S * K) {
        int s = threadIdx.x / K, k = threadIdx.x % K;
        int e = sel[s][k];
        if (e >= p.expert_lo && e < p.expert_hi) used_flag[e - p.expert_lo] = 1;
    }
    __syncthreads();
    // block scan over the local experts, 4 per thread, ascending
    const int nl = p.expert_hi - p.expert_lo;
    int cnt = 0;
    for (int i = 0; i < 4; ++i) {
        int e = 4 * threadIdx.x + i;
        if (e < nl) cnt += used_flag[e];
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_total[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += warp_total[w];
    int slot = base + incl - cnt;
    for (int i = 0; i < 4; ++i) {
        int e = 4 * threadIdx.x + i;
        if (e < nl && used_flag[e]) {
            slot_of[e] = slot;
            p.active[slot] = p.expert_lo + e;
            ++slot;
        }
    }
    int total = 0;
    for (int w = 0; w < kRouteThreads / 32; ++w) total += warp_total[w];
    if (threadIdx.x == 0) *p.n_active = total;
    for (int i = threadIdx.x; i < total * 8; i += blockDim.x) p.coef[i] = 0.0f;
    __syncthreads();
    if (threadIdx.x < p.S * K) {
        int s = threadIdx.x / K, k = threadIdx.x % K;
        int e = sel[s][k];
        if (e >= p.expert_lo && e < p.expert_hi) p.coef[slot_of[e - p.expert_lo] * 8 + s] = selw[s][k];
    }
}

// resid[s][d] += (sum over slots ascending of coef * routed[slot][s][d])
//                + shared[s][d]                           (moe_exec.h:97-110)
// Products and sums are rounded separately (no contraction), the order the
// C reference spells out.
__global__ void moe_combine_kernel(float *resid, const float *routed, const float *shared,
                                   const float *coef, const int *n_active, int S, int D,
                                   int max_batch) {
    pdl_wait();
    pdl_release();
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= S * D) return;
    int s = idx / D, d = idx % D;
    int n = *n_active;
    float y = 0.0f;
    for (int slot = 0; slot < n; ++slot) {
        float c = coef[slot * 8 + s];
        if (c != 0.0f)
            y = __fadd_rn(y, __fmul_rn(c, routed[((size_t)slot * max_batch + s) * D + d]));
    }
    if (shared) y = __fadd_rn(y, shared[(size_t)s * D + d]);
    resid[(size_t)s * D + d] = __fadd_rn(resid[(size_t)s * D + d], y);
}

}  // namespace fc
