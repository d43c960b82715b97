// synth.cuh - device side of the seeded synthetic generator (floyd_synth.h)
// and the logical <-> device weight-layout conversions.
#pragma once

#include "common.cuh"

namespace fc {

// Logical column of byte `b` (and nibble `nib`) of a 64-byte row chunk `c`;
// the inverse of weight_position (common.cuh).
__host__ __device__ inline int logical_column(int fmt, int c, int b, int nib) {
    if (fmt == FC_FMT_Q8) {
        int j = b >> 4, i = (b & 15) >> 2, bb = b & 3;
        return 64 * c + 16 * i + 4 * j + bb;
    }
    int j = b >> 4, word = (b & 15) >> 2, bw = b & 3;
    int slot = 2 * bw + nib;
    int q = 4 * word + (slot & 3), e = slot >> 2;
    int i = q >> 1, h = q & 1;
    return 128 * c + 16 * i + 4 * j + 2 * h + e;
}

// Fills `count` matrices (rows O, logical K, padded kp) of a family with the
// synthetic values of tensors tid0 + slot (slot = member + slot0).
__global__ void synth_values_kernel(int fmt, uint8_t *w, int O, int K, int kp, int count,
                                    uint64_t seed, uint32_t tid_base, int slot0) {
    size_t rb = (size_t)row_bytes(fmt, kp);
    size_t per = (size_t)O * rb;
    size_t total = per * count;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        int member = (int)(idx / per);
        size_t in = idx % per;
        int o = (int)(in / rb);
        int byte = (int)(in % rb);
        int c = byte >> 6, b = byte & 63;
        uint32_t tid = tid_base | (uint32_t)(member + slot0);
        uint8_t out;
        if (fmt == FC_FMT_Q8) {
            int k = logical_column(fmt, c, b, 0);
            int v = k < K ? fc_synth_q8(seed, tid, (uint64_t)o * K + k) : 0;
            out = (uint8_t)(int8_t)v;
        } else {
            uint32_t nib[2];
            for (int n = 0; n < 2; ++n) {
                int k = logical_column(fmt, c, b, n);
                if (k < K) nib[n] = (uint32_t)fc_synth_nibble(seed, tid, (uint64_t)o * K + k);
                else nib[n] = fmt == FC_FMT_Q4 ? 8u : 0u;
            }
            out = (uint8_t)(nib[0] | (nib[1] << 4));
        }
        w[idx] = out;
    }
}

__global__ void synth_scales_kernel(int fmt, void *sc, int O, int K, int kp, int count,
                                    uint64_t seed, uint32_t tid_base, int slot0) {
    int gk = K / 32, gp = kp / 32;
    size_t per = (size_t)O * gp;
    size_t total = per * count;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        int member = (int)(idx / per);
        size_t in = idx % per;
        int o = (int)(in / gp), g = (int)(in % gp);
        uint32_t tid = tid_base | (uint32_t)(member + slot0);
        uint64_t lg = (uint64_t)o * gk + g;
        if (fmt == FC_FMT_MXFP4) {
            reinterpret_cast<uint8_t *>(sc)[idx] = g < gk ? fc_synth_scale_e8m0(seed, tid, lg) : 0;
        } else {
            uint16_t bits = 0;
            if (g < gk) bits = fmt == FC_FMT_Q8 ? fc_synth_scale_q8(seed, tid, lg)
                                                : fc_synth_scale_q4(seed, tid, lg);
            reinterpret_cast<uint16_t *>(sc)[idx] = bits;
        }
    }
}

__global__ void synth_f32_kernel(float *w, size_t n, int kind, uint64_t seed, uint32_t tid) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        if (kind == 0) w[i] = fc_synth_f32(seed, tid, i);
        else if (kind == 1) w[i] = fc_synth_norm(seed, tid, i);
        else w[i] = fc_synth_bias(seed, tid, i);
    }
}

__global__ void synth_hash_kernel(int *table, int vocab, int K, int E, uint64_t seed, uint32_t tid) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (size_t)vocab * K;
         i += (size_t)gridDim.x * blockDim.x)
        table[i] = fc_synth_hash_expert(seed, tid, (int)(i / K), (int)(i % K), E, K);
}

// Latent KV rows [0, positions) of one layer: latent from stream KV_LATENT,
// rope part from KV_ROPE (element index position * width + column).
__global__ void synth_kv_kernel(__half *cache, int positions, int L, int R, uint64_t seed,
                                uint32_t tid_latent, uint32_t tid_rope) {
    size_t total = (size_t)positions * (L + R);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        size_t p = i / (L + R);
        int c = (int)(i % (L + R));
        float v = c < L ? fc_synth_kv(seed, tid_latent, p * L + c)
                        : fc_synth_kv(seed, tid_rope, p * R + (c - L));
        cache[i] = __float2half_rn(v);
    }
}

}  // namespace fc
