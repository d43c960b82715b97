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

#ifdef FC_TC_TRACE
#define RT_MARK(i) g_tc_trace[(i)] = clock64()
#else
#define RT_MARK(i) \
    do {           \
    } while (0)
#endif


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
    float *coef;             // [global slots][8] coefficient of global slot g for row s
    float *choice;           // [S][E] score + selection bias (non-softmax score functions)
    int *n_global;           // active experts of all ranks (global slots)
    int *n_before;           // active experts below expert_lo (first global slot of this rank)
    int *arrivals;           // block arrival counter (zero between launches)
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

constexpr int kRouteThreads = 256;

// Scores and top-k of row s by one warp; lane l holds experts l + 32 i
// (i < PER) in registers.  Scores by MoeScoreFn (softmax: lane sums in
// ascending expert order, then a butterfly), top-k by repeated warp argmax
// over score + bias (lower index on ties), finalize in slot order on lane 0
// (moe_route.h:26-99).
template <int PER>
__device__ __forceinline__ void route_row(const float *logits, const RouteParams &p, int s,
                                          int (&sel)[64], float (&selw)[64]) {
    const int lane = threadIdx.x & 31;
    const int E = p.E, K = p.K;
    float sc[PER], ch[PER];
    const bool pre = p.score_fn != FC_SCORE_SOFTMAX;  // scores / choices came from the router blocks
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        int e = lane + 32 * i;
        sc[i] = e < E ? __ldcg(logits + (size_t)s * E + e) : -INFINITY;
        ch[i] = (pre && e < E) ? __ldcg(p.choice + (size_t)s * E + e) : -INFINITY;
    }
    if (threadIdx.x == 0) RT_MARK(220);
    if (!pre) {
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < PER; ++i) m = fmaxf(m, sc[i]);
        m = warp_max(m);
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            float v = lane + 32 * i < E ? expf(sc[i] - m) : 0.0f;
            sc[i] = v;
            sum += v;
        }
        sum = warp_sum(sum);
#pragma unroll
        for (int i = 0; i < PER; ++i) sc[i] = sc[i] / sum;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            int e = lane + 32 * i;
            ch[i] = e < E ? sc[i] + (p.bias ? p.bias[e] : 0.0f) : -INFINITY;
        }
    }
    // score of expert e (same value on every lane)
    auto score_of = [&](int e) {
        float v = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; ++i)
            if (i == (e >> 5)) v = sc[i];
        return __shfl_sync(0xffffffffu, v, e & 31);
    };
    if (threadIdx.x == 0) RT_MARK(221);
    if (p.hash) {
        int mine = lane < K ? p.hash[(size_t)p.ids[s] * K + lane] : 0;
        for (int k = 0; k < K; ++k) {
            int e = __shfl_sync(0xffffffffu, mine, k & 31);
            if (k >= 32) e = p.hash[(size_t)p.ids[s] * K + k];
            float w = score_of(e);
            if (lane == 0) {
                sel[k] = e;
                selw[k] = w;
            }
        }
    } else {
        uint32_t taken = 0;
        for (int k = 0; k < K; ++k) {
            float best = -INFINITY;
            int bi = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                int e = lane + 32 * i;
                if (e < E && !((taken >> i) & 1u) && ch[i] > best) {
                    best = ch[i];
                    bi = e;
                }
            }
            // warp argmax: the largest value (order-preserving unsigned key,
            // -0 taken as +0 so equal values compare equal), then the lowest
            // expert id among the lanes holding it (NaN never became a
            // lane's best, so it never wins)
            const float bz = best == 0.0f ? 0.0f : best;
            const uint32_t bits = __float_as_uint(bz);
            const uint32_t key = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
            const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
            bi = (int)__reduce_min_sync(0xffffffffu, (uint32_t)(key == kmax ? bi : 0x7fffffff));
            if (bi == 0x7fffffff) bi = 0;  // no finite candidate left
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            float w = score_of(bi);
            if (lane == 0) {
                sel[k] = bi;
                selw[k] = w;
            }
        }
    }
    if (threadIdx.x == 0) RT_MARK(222);
    __syncwarp();
    // moe_route_finalize (moe_route.h:89-99): every lane forms the same
    // ascending-slot sum, then lane k finishes slot k
    float sum = 0.0f;
    if (p.normalize) {
        for (int k = 0; k < K; ++k) sum += selw[k];
        sum += 1e-20f;
    }
    __syncwarp();
    for (int k = lane; k < K; k += 32) {
        float w = p.normalize ? selw[k] / sum : selw[k];
        w = w * p.routed_scale;
        p.route_ids[s * K + k] = sel[k];
        p.route_w[s * K + k] = w;
        selw[k] = w;
    }
    __syncwarp();
}

// Selection for all rows by one block (warp s = row s), then the ascending
// list of active local experts and their per-row coefficients from a
// block-wide scan (the device-side replacement of prepare_route_tables).
__device__ __forceinline__ void route_select_block(const float *logits, const RouteParams &p) {
    __shared__ int used_flag[1024];
    __shared__ int slot_of[1024];
    __shared__ int warp_total[kRouteThreads / 32];
    __shared__ int sel[8][64];
    __shared__ float selw[8][64];
    const int K = p.K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < 1024; e += blockDim.x) used_flag[e] = 0;
    if (warp < p.S) {
        const int per = (p.E + 31) / 32;
        if (per <= 2) route_row<2>(logits, p, warp, sel[warp], selw[warp]);
        else if (per <= 4) route_row<4>(logits, p, warp, sel[warp], selw[warp]);
        else if (per <= 8) route_row<8>(logits, p, warp, sel[warp], selw[warp]);
        else if (per <= 16) route_row<16>(logits, p, warp, sel[warp], selw[warp]);
        else route_row<32>(logits, p, warp, sel[warp], selw[warp]);
    }
    __syncthreads();
    if (threadIdx.x == 0) RT_MARK(213);
    if (threadIdx.x < p.S * K) {
        int s = threadIdx.x / K, k = threadIdx.x % K;
        used_flag[sel[s][k]] = 1;
    }
    __syncthreads();
    // Global slots: every selected expert of every rank in ascending id
    // (block scan, 4 experts per thread).  This rank's local slots are the
    // window [n_before, n_before + local count) of that order, so the
    // expert-parallel combine sums exactly the single-GPU sequence.
    int cnt = 0;
    for (int i = 0; i < 4; ++i) {
        int e = 4 * threadIdx.x + i;
        if (e < p.E) cnt += used_flag[e];
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
    int total = 0;
    for (int w = 0; w < kRouteThreads / 32; ++w) total += warp_total[w];
    // slots below expert_lo and below expert_hi (exclusive prefixes)
    __shared__ int pre_lo, pre_hi;
    if (threadIdx.x == 0) pre_hi = total;
    __syncthreads();
    int slot = base + incl - cnt;
    for (int i = 0; i < 4; ++i) {
        int e = 4 * threadIdx.x + i;
        if (e == p.expert_lo) pre_lo = slot;
        if (e == p.expert_hi) pre_hi = slot;
        if (e < p.E && used_flag[e]) slot_of[e] = slot++;
    }
    __syncthreads();
    if (threadIdx.x == 0) RT_MARK(214);
    if (threadIdx.x == 0) {
        *p.n_before = pre_lo;
        *p.n_active = pre_hi - pre_lo;
        *p.n_global = total;
    }
    for (int i = threadIdx.x; i < total * 8; i += blockDim.x) p.coef[i] = 0.0f;
    __syncthreads();
    if (threadIdx.x < p.S * K) {
        int s = threadIdx.x / K, k = threadIdx.x % K;
        int e = sel[s][k];
        p.coef[slot_of[e] * 8 + s] = selw[s][k];
    }
    // local active list (ascending): global slots of this rank's experts
    // minus the slots below them
    for (int e = p.expert_lo + threadIdx.x; e < p.expert_hi; e += blockDim.x)
        if (used_flag[e]) p.active[slot_of[e] - pre_lo] = e;
}

// Router: one block per expert computes its logits for every row (fp32
// weights [E][D], float4 loads, fixed-order reduction: warp butterfly, then
// warps in index order); the last block to finish runs the selection and
// the expert grouping.
__global__ void __launch_bounds__(kRouteThreads) router_kernel(const float *W, const float *x, int D,
                                                               float *logits, RouteParams p) {
    __shared__ float red[8][8];
    __shared__ int is_last;
    const int e = blockIdx.x, E = p.E, S = p.S;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float acc[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) acc[s] = 0.0f;
    const float4 *w4 = reinterpret_cast<const float4 *>(W + (size_t)e * D);
    // the weight row is constant: up to 4 float4 per thread fetched before
    // waiting for the activations
    constexpr int kPre = 4;
    float4 wpre[kPre];
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        int k4 = threadIdx.x + i * kRouteThreads;
        if (k4 < D / 4) wpre[i] = __ldg(w4 + k4);
    }
    if (threadIdx.x == 0 && blockIdx.x == 0) RT_MARK(210);
    pdl_wait();
    pdl_release();
    if (threadIdx.x == 0 && blockIdx.x == 0) RT_MARK(211);
    for (int k4 = threadIdx.x, i = 0; k4 < D / 4; k4 += blockDim.x, ++i) {
        float4 w;
        if (i < kPre) {
            w = wpre[0];
#pragma unroll
            for (int t = 1; t < kPre; ++t)
                if (i == t) w = wpre[t];
        } else {
            w = __ldg(w4 + k4);
        }
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
        if (p.score_fn == FC_SCORE_SOFTMAX) {
            logits[(size_t)threadIdx.x * E + e] = t;  // normalized over the row by the selection
        } else {
            // per-expert score functions: score and selection value here
            const float sc = route_score(t, p.score_fn);
            logits[(size_t)threadIdx.x * E + e] = sc;
            p.choice[(size_t)threadIdx.x * E + e] = sc + (p.bias ? __ldg(p.bias + e) : 0.0f);
        }
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int prev = atomicAdd(p.arrivals, 1);
        is_last = prev == E - 1;
        if (is_last) *p.arrivals = 0;
    }
    __syncthreads();
    if (!is_last) return;
    if (threadIdx.x == 0) RT_MARK(212);
    __threadfence();
    route_select_block(logits, p);
    if (threadIdx.x == 0) RT_MARK(215);
}

// resid[s][d] += (sum over slots ascending of coef * routed[slot][s][d])
//                + shared[s][d]                           (moe_exec.h:97-110)
// Products and sums are rounded separately (no contraction), the order the
// C reference spells out.
constexpr int kMoeCombineThreads = 256;
constexpr int kMaxRanks = 8;

// Expert-parallel exchange state of one session (pointers into the peers'
// receive regions; absent on a single GPU).
struct EpLink {
    int world, rank;
    int *epoch;                      // local counter, +1 per MoE layer (both sides in lockstep)
    int *flags;                      // [world] epochs published by the peers into this GPU
    int *peer_flags[kMaxRanks];      // the peers' flag arrays (index rank = this rank)
    unsigned long long *wait_ns;     // nullable: block 0 adds the time it spent waiting for the peers
};

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// After this rank's routed down projections (which stored their outputs
// into every peer's receive buffer): publish the next epoch to every peer.
__global__ void ep_signal_kernel(EpLink link) {
    pdl_wait();
    pdl_release();
    __threadfence_system();
    const int e = *link.epoch + 1;
    *link.epoch = e;
    for (int r = 0; r < link.world; ++r)
        if (r != link.rank) st_release_sys(link.peer_flags[r] + link.rank, e);
}

// resid[s][d] += (sum over global slots ascending of coef * routed[slot][s][d])
//                + shared[s][d]                           (moe_exec.h:97-110)
// Products and sums are rounded separately (no contraction), the order the
// C reference spells out.  With expert parallelism the routed outputs of
// every rank sit in this GPU's receive buffer (buffer = epoch parity) once
// every peer has published the current epoch; the wait is bounded (error
// bit 2 on timeout).
__global__ void __launch_bounds__(kMoeCombineThreads)
moe_combine_kernel(float *resid, const float *routed, const float *shared, const float *coef,
                   const int *n_active, int S, int D, int max_batch, EpLink link, int64_t parity_stride,
                   int *err) {
    pdl_wait();
    pdl_release();
    __shared__ int list[1024];
    __shared__ float lc[1024];
    __shared__ int count;
    if (link.world > 1) {
        if (threadIdx.x == 0) {
            const int e = *link.epoch;
            uint64_t t0 = 0, w0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(w0));
            for (int r = 0; r < link.world; ++r) {
                if (r == link.rank) continue;
                for (uint32_t it = 0; ld_acquire_sys(link.flags + r) < e; ++it) {
                    if ((it & 255u) == 0) {
                        uint64_t t;
                        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                        if (t0 == 0) t0 = t;
                        else if (t - t0 > 1000000000ull) {
                            atomicOr(err, 2);
                            break;
                        }
                    }
                }
            }
            count = e;  // reused below for the parity
            if (link.wait_ns && blockIdx.x == 0) {  // the exchange time this rank was exposed to
                uint64_t w1;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(w1));
                atomicAdd(link.wait_ns, (unsigned long long)(w1 - w0));
            }
        }
        __syncthreads();
        routed += (count & 1) * parity_stride;
        __syncthreads();
    }
    // blocks of one row: blockIdx.x = s * (D / 256) + column block
    const int per_row = (D + kMoeCombineThreads - 1) / kMoeCombineThreads;
    const int s = blockIdx.x / per_row;
    const int d = (blockIdx.x % per_row) * kMoeCombineThreads + threadIdx.x;
    const int n = *n_active;
    if (threadIdx.x < 32) {  // ascending list of the slots that feed row s
        int base = 0;
        for (int i0 = 0; i0 < n; i0 += 32) {
            int slot = i0 + threadIdx.x;
            float c = slot < n ? coef[slot * 8 + s] : 0.0f;
            unsigned m = __ballot_sync(0xffffffffu, c != 0.0f);
            if (c != 0.0f) {
                int at = base + __popc(m & ((1u << threadIdx.x) - 1u));
                if (at < 1024) {
                    list[at] = slot;
                    lc[at] = c;
                }
            }
            base += __popc(m);
        }
        if (threadIdx.x == 0) count = base < 1024 ? base : 1024;
    }
    __syncthreads();
    if (d >= D) return;
    const int cnt = count;
    float y = 0.0f;
    int i = 0;
    for (; i + 8 <= cnt; i += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldcg(routed + ((size_t)list[i + u] * max_batch + s) * D + d);
#pragma unroll
        for (int u = 0; u < 8; ++u) y = __fadd_rn(y, __fmul_rn(lc[i + u], v[u]));
    }
    for (; i < cnt; ++i) y = __fadd_rn(y, __fmul_rn(lc[i], __ldcg(routed + ((size_t)list[i] * max_batch + s) * D + d)));
    if (shared) y = __fadd_rn(y, shared[(size_t)s * D + d]);
    resid[(size_t)s * D + d] = __fadd_rn(resid[(size_t)s * D + d], y);
}

}  // namespace fc
