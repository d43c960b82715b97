// head.cuh - lm-head reduction and acceptance of the verify step.
//
// Replaces encode_final_logits' consumer side (moonlight_metal.m:708-725),
// deepseek_v4_runtime_argmax / _verify_token (deepseek_v4_runtime.h:231-244),
// ds4's two-pass argmax (patches/ds4/deepseek-v4-dspark-fast-argmax.patch
// :225-307: NaN never wins, the lowest index wins ties) and the commit rule
// of ds4_session_commit_dspark_speculative (dspark-metal.patch:1793-1797).
// Rejection sampling has no reference implementation (the reference rejects
// temperature > 0 with draft > 1, deepseek_v4_ds4.c:75-85); it follows
// speculative sampling (Leviathan et al. 2023, Chen et al. 2023) with a
// point-mass drafter, Philox4x32-10 uniforms and Gumbel-max sampling so the
// whole vocabulary pass is a single read of the logits.
#pragma once

#include "common.cuh"

namespace fc {

constexpr int kMaxRows = 8;       // rows per forward pass
constexpr int kHeadChunk = 2048;  // vocab entries per partial block

// Host -> device per-launch parameters (one H2D copy at the head of a graph).
// The rows of a pass form `groups` sequence groups of group_rows consecutive
// rows (one group for an ordinary session); row r sits at position
// rowpos[r] of sequence rowseq[r], and each group is accepted on its own.
struct Staging {
    int pos;
    int rows;
    int k;          // drafts per group (verify) or -1 (plain forward)
    int mode;       // FcAcceptMode
    float temperature;
    int pad;
    unsigned long long seed;
    unsigned long long counter;   // Philox counter of group 0
    int ids[kMaxRows];
    int rowpos[kMaxRows];
    int rowseq[kMaxRows];
    int group_rows;
    int groups;
    unsigned long long gcounter[kMaxRows];  // Philox counter of each group
};

// Device -> host results (one D2H copy at the tail of a graph).
struct Result {
    int commit;       // group 0 (the session's sequence)
    int next_token;
    int error;      // error bits raised by kernels of this pass
    int pad;
    int row_tops[kMaxRows];
    int drafts[kMaxRows];   // MTP drafter proposals (verify with k > 0)
    int g_commit[kMaxRows];
    int g_next[kMaxRows];
    float draft_conf[kMaxRows];  // the drafter's top-1 logit of each proposal
};

// Latent-cache paging: sequence `seq`'s position p lives at row
// pt[seq * pps + p / 64] * 64 + p % 64 of a layer's region (64-row pages, so
// a 64- or 32-key block never straddles two pages).  Ordinary sessions map
// every page to itself.
constexpr int kPageRows = 64;
struct PageMap {
    const int *pt;
    int pps;        // pages per sequence
};
__device__ __forceinline__ int kv_row(const PageMap &pm, int seq, int p) {
    return pm.pt[seq * pm.pps + (p >> 6)] * kPageRows + (p & (kPageRows - 1));
}

__device__ __forceinline__ float accept_uniform(unsigned long long seed, unsigned long long counter,
                                                int row) {
    uint32_t c[4] = {(uint32_t)row, 0xACCE97EDu, (uint32_t)counter, (uint32_t)(counter >> 32)};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t out[4];
    fc_philox4x32_10(c, key, out);
    return (float)(out[0] >> 8) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float gumbel(unsigned long long seed, unsigned long long counter, int row,
                                        int v) {
    uint32_t c[4] = {(uint32_t)v >> 2, (uint32_t)row, (uint32_t)counter,
                     (uint32_t)(counter >> 32) ^ 0x9E3779B9u};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t out[4];
    fc_philox4x32_10(c, key, out);
    float u = ((float)(out[v & 3] >> 8) + 0.5f) * (1.0f / 16777216.0f);
    return -logf(-logf(u));
}

// (value, index) better-than for argmax: strict >, then lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

struct HeadPartials {
    float *amax; int *aidx;      // argmax   [rows][chunks]
    float *zmax; float *zsum;    // softmax  [rows][chunks] of logits / T
    float *gval; int *gidx;      // Gumbel argmax [rows][chunks]
};

// grid (chunks, rows), 256 threads.
__global__ void head_partial_kernel(const float *logits, int V, const Staging *st, HeadPartials hp,
                                    int chunks) {
    pdl_wait();
    pdl_release();
    __shared__ float sv[3][8];
    __shared__ int si[2][8];
    int chunk = blockIdx.x, row = blockIdx.y;
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *lg = logits + (size_t)row * V;
    int begin = chunk * kHeadChunk, end = min(V, begin + kHeadChunk);
    bool sample = st->mode == FC_ACCEPT_SAMPLE && st->k >= 0;
    float temp = sample ? st->temperature : 1.0f;
    // row index and Philox counter within the row's sequence group
    const int grp = row / st->group_rows, local = row - grp * st->group_rows;
    const unsigned long long counter = st->gcounter[grp];
    int excluded = (sample && local < st->k) ? st->ids[row + 1] : -1;
    float bv = -INFINITY; int bi = 0x7fffffff;
    float zm = -INFINITY;
    float gv = -INFINITY; int gi = 0x7fffffff;
    for (int v = begin + threadIdx.x; v < end; v += blockDim.x) {
        float x = lg[v];
        if (x != x) continue;  // NaN never wins
        if (better(x, v, bv, bi)) { bv = x; bi = v; }
        if (sample) {
            float z = x / temp;
            zm = fmaxf(zm, z);
            if (v != excluded) {
                float t = z + gumbel(st->seed, counter, local, v);
                if (better(t, v, gv, gi)) { gv = t; gi = v; }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        float og = __shfl_xor_sync(0xffffffffu, gv, o);
        int ogi = __shfl_xor_sync(0xffffffffu, gi, o);
        if (better(og, ogi, gv, gi)) { gv = og; gi = ogi; }
        zm = fmaxf(zm, __shfl_xor_sync(0xffffffffu, zm, o));
    }
    if (lane == 0) { sv[0][warp] = bv; si[0][warp] = bi; sv[1][warp] = gv; si[1][warp] = gi; sv[2][warp] = zm; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) {
            if (better(sv[0][w], si[0][w], sv[0][0], si[0][0])) { sv[0][0] = sv[0][w]; si[0][0] = si[0][w]; }
            if (better(sv[1][w], si[1][w], sv[1][0], si[1][0])) { sv[1][0] = sv[1][w]; si[1][0] = si[1][w]; }
            sv[2][0] = fmaxf(sv[2][0], sv[2][w]);
        }
        size_t o = (size_t)row * chunks + chunk;
        hp.amax[o] = sv[0][0]; hp.aidx[o] = si[0][0];
        hp.gval[o] = sv[1][0]; hp.gidx[o] = si[1][0];
        hp.zmax[o] = sv[2][0];
    }
    if (!sample) return;
    __syncthreads();
    float m = sv[2][0];
    float sum = 0.0f;
    for (int v = begin + threadIdx.x; v < end; v += blockDim.x) {
        float x = lg[v];
        if (x != x) continue;
        sum += expf(x / temp - m);
    }
    __shared__ float ssum[8];
    sum = warp_sum(sum);
    if (lane == 0) ssum[warp] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < 8; ++w) t += ssum[w];
        hp.zsum[(size_t)row * chunks + chunk] = m == -INFINITY ? 0.0f : t;
    }
}

// One block of 256 threads.  Warp r reduces row r's per-chunk partials in
// parallel (the (value, index) order is total, so the result does not depend
// on the reduction shape); thread 0 then applies the acceptance rule and
// writes the result record.
__global__ void __launch_bounds__(256) accept_kernel(const float *logits, int V, const Staging *st,
                                                     HeadPartials hp, int chunks, Result *res,
                                                     int *err) {
    pdl_wait();
    pdl_release();
    __shared__ int tops[kMaxRows], picks[kMaxRows];
    __shared__ float zmax_row[kMaxRows], den_row[kMaxRows];
    const int rows = st->rows, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool sample = st->k >= 0 && st->mode == FC_ACCEPT_SAMPLE;
    if (warp < rows) {
        const int r = warp;
        float bv = -INFINITY, gv = -INFINITY, M = -INFINITY;
        int bi = 0x7fffffff, gi = 0x7fffffff;
        for (int c = lane; c < chunks; c += 32) {
            size_t o = (size_t)r * chunks + c;
            if (better(hp.amax[o], hp.aidx[o], bv, bi)) { bv = hp.amax[o]; bi = hp.aidx[o]; }
            if (sample) {
                if (better(hp.gval[o], hp.gidx[o], gv, gi)) { gv = hp.gval[o]; gi = hp.gidx[o]; }
                M = fmaxf(M, hp.zmax[o]);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            float og = __shfl_xor_sync(0xffffffffu, gv, off);
            int ogi = __shfl_xor_sync(0xffffffffu, gi, off);
            if (better(og, ogi, gv, gi)) { gv = og; gi = ogi; }
            M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        }
        float den = 0.0f;
        if (sample)
            for (int c = lane; c < chunks; c += 32) {
                float zm = hp.zmax[(size_t)r * chunks + c];
                if (zm != -INFINITY) den += expf(zm - M) * hp.zsum[(size_t)r * chunks + c];
            }
        den = warp_sum(den);
        if (lane == 0) {
            tops[r] = bi == 0x7fffffff ? -1 : bi;
            picks[r] = gi == 0x7fffffff ? -1 : gi;
            zmax_row[r] = M;
            den_row[r] = den;
        }
    }
    __syncthreads();
    if (threadIdx.x >= st->groups) return;
    // thread g applies the acceptance rule to sequence group g
    const int g = threadIdx.x, gr = st->group_rows, r0 = g * gr;
    if (g == 0)
        for (int r = 0; r < rows; ++r) res->row_tops[r] = tops[r];
    const int k = st->k;
    const int *ids = st->ids + r0;
    int commit = gr, next = tops[r0 + gr - 1];
    if (sample) {
        commit = k + 1;
        next = picks[r0 + k];
        for (int i = 1; i <= k; ++i) {
            const int r = r0 + i - 1, x = ids[i];
            float p = expf(logits[(size_t)r * V + x] / st->temperature - zmax_row[r]) / den_row[r];
            float u = accept_uniform(st->seed, st->gcounter[g], i - 1);
            if (!(u < p)) {
                commit = i;
                next = picks[r];
                break;
            }
        }
    } else if (k >= 0) {
        commit = 1;
        for (int i = 1; i <= k; ++i) {
            if (tops[r0 + i - 1] != ids[i]) break;
            commit++;
        }
        next = tops[r0 + commit - 1];
    }
    res->g_commit[g] = commit;
    res->g_next[g] = next;
    if (g == 0) {
        res->commit = commit;
        res->next_token = next;
        res->error = *err;
        *err = 0;
    }
}

// ---- MTP drafter glue --------------------------------------------------
// Step i of the drafter: position pos + commit + i, input token = the
// target's next token (i = 0) or the previous proposal; step 0 also takes
// the hidden state (pre-norm residual) of the last committed row.
__global__ void mtp_prep_kernel(int i, const Staging *main_st, const Result *res, Staging *mst,
                                const float *resid, float *mtp_h, int D) {
    pdl_wait();
    pdl_release();
    const int commit = res->commit;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        mst->pos = main_st->pos + commit + i;
        mst->rows = 1;
        mst->k = -1;
        mst->mode = FC_ACCEPT_GREEDY;
        mst->rowpos[0] = mst->pos;
        mst->rowseq[0] = 0;
        mst->group_rows = 1;
        mst->groups = 1;
        mst->gcounter[0] = 0;
        int t = i == 0 ? res->next_token : res->drafts[i - 1];
        mst->ids[0] = t < 0 ? 0 : t;
    }
    if (i == 0)
        for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < D; d += gridDim.x * blockDim.x)
            mtp_h[d] = resid[(size_t)(commit - 1) * D + d];
}

// Final hidden rows (pre-norm residual) of a forward, stored by position
// for the drafter's prefill (models with an MTP layer): hist[rowpos[r]] =
// resid[r].
__global__ void hist_store_kernel(const float *resid, const Staging *st, float *hist, int D) {
    pdl_wait();
    pdl_release();
    const int r = blockIdx.y;
    if (r >= st->rows) return;
    float *dst = hist + (size_t)st->rowpos[r] * D;
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < D; d += gridDim.x * blockDim.x)
        dst[d] = resid[(size_t)r * D + d];
}

// The same for T prefill rows at positions pos0 .. pos0 + T - 1, pos0 read
// from the device (the prefill parameter record's first word).
__global__ void hist_store_rows_kernel(const float *rows, const int *pos0, int T, float *hist, int D) {
    pdl_wait();
    pdl_release();
    const int t = blockIdx.y;
    if (t >= T) return;
    float *dst = hist + ((size_t)*pos0 + t) * D;
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < D; d += gridDim.x * blockDim.x)
        dst[d] = rows[(size_t)t * D + d];
}

// Greedy pick of the drafter's row (same order as the target's argmax:
// NaN never wins, lower index on ties); writes proposal i.
__global__ void __launch_bounds__(32) mtp_pick_kernel(HeadPartials hp, int chunks, Result *res,
                                                      Staging *mst, int i) {
    pdl_wait();
    pdl_release();
    const int lane = threadIdx.x;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < chunks; c += 32)
        if (better(hp.amax[c], hp.aidx[c], bv, bi)) { bv = hp.amax[c]; bi = hp.aidx[c]; }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
        const int t = bi == 0x7fffffff ? 0 : bi;
        res->drafts[i] = t;
        res->draft_conf[i] = bv;
        mst->ids[0] = t;
    }
}

}  // namespace fc
