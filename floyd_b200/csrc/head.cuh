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
struct Staging {
    int pos;
    int rows;
    int k;          // drafts (verify) or -1 (plain forward)
    int mode;       // FcAcceptMode
    float temperature;
    int pad;
    unsigned long long seed;
    unsigned long long counter;
    int ids[kMaxRows];
};

// Device -> host results (one D2H copy at the tail of a graph).
struct Result {
    int commit;
    int next_token;
    int error;      // error bits raised by kernels of this pass
    int pad;
    int row_tops[kMaxRows];
};

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
    __shared__ float sv[3][8];
    __shared__ int si[2][8];
    int chunk = blockIdx.x, row = blockIdx.y;
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *lg = logits + (size_t)row * V;
    int begin = chunk * kHeadChunk, end = min(V, begin + kHeadChunk);
    bool sample = st->mode == FC_ACCEPT_SAMPLE && st->k >= 0;
    float temp = sample ? st->temperature : 1.0f;
    int excluded = (sample && row < st->k) ? st->ids[row + 1] : -1;
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
                float t = z + gumbel(st->seed, st->counter, row, v);
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

// One block.  Final argmax per row (chunk order), acceptance, result record
// and, when `last_logits` is set, the logits row commit-1.
__global__ void accept_kernel(const float *logits, int V, const Staging *st, HeadPartials hp,
                              int chunks, Result *res, float *last_logits, int *err) {
    __shared__ int commit_s;
    int rows = st->rows;
    if (threadIdx.x == 0) {
        int tops[kMaxRows];
        for (int r = 0; r < rows; ++r) {
            float bv = -INFINITY; int bi = -1;
            for (int c = 0; c < chunks; ++c) {
                size_t o = (size_t)r * chunks + c;
                int idx = hp.aidx[o];
                if (idx == 0x7fffffff) continue;
                if (bi < 0 || better(hp.amax[o], idx, bv, bi)) { bv = hp.amax[o]; bi = idx; }
            }
            tops[r] = bi;
            res->row_tops[r] = bi;
        }
        int k = st->k;
        int commit = rows, next = tops[rows - 1];
        if (k >= 0 && st->mode == FC_ACCEPT_SAMPLE) {
            float temp = st->temperature;
            auto gumbel_pick = [&](int r) {
                float bv = -INFINITY; int bi = -1;
                for (int c = 0; c < chunks; ++c) {
                    size_t o = (size_t)r * chunks + c;
                    int idx = hp.gidx[o];
                    if (idx == 0x7fffffff) continue;
                    if (bi < 0 || better(hp.gval[o], idx, bv, bi)) { bv = hp.gval[o]; bi = idx; }
                }
                return bi;
            };
            commit = k + 1;
            next = -1;
            for (int i = 1; i <= k; ++i) {
                int r = i - 1;
                float M = -INFINITY;
                for (int c = 0; c < chunks; ++c) M = fmaxf(M, hp.zmax[(size_t)r * chunks + c]);
                float den = 0.0f;
                for (int c = 0; c < chunks; ++c) {
                    float zm = hp.zmax[(size_t)r * chunks + c];
                    if (zm != -INFINITY) den += expf(zm - M) * hp.zsum[(size_t)r * chunks + c];
                }
                int x = st->ids[i];
                float p = expf(logits[(size_t)r * V + x] / temp - M) / den;
                float u = accept_uniform(st->seed, st->counter, r);
                if (!(u < p)) {
                    commit = i;
                    next = gumbel_pick(r);
                    break;
                }
            }
            if (next < 0) next = gumbel_pick(k);
        } else if (k >= 0) {
            commit = 1;
            for (int i = 1; i <= k; ++i) {
                if (tops[i - 1] != st->ids[i]) break;
                commit++;
            }
            next = tops[commit - 1];
        }
        res->commit = commit;
        res->next_token = next;
        res->error = *err;
        *err = 0;
        commit_s = commit;
    }
    __syncthreads();
    if (last_logits) {
        const float *src = logits + (size_t)(commit_s - 1) * V;
        for (int v = threadIdx.x; v < V; v += blockDim.x) last_logits[v] = src[v];
    }
}

}  // namespace fc
