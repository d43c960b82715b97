// synth.cuh - device side of the seeded synthetic generator (floyd_synth.h)
// and the logical <-> device weight-layout conversions.
#pragma once

#include "common.cuh"

namespace fc {

// Fills `count` matrices (rows O, logical K, padded kp) of a family with the
// synthetic values of tensors tid_base | (member + slot0).  One thread per
// Philox block: 8 int8 values or 32 nibbles of consecutive logical elements
// (a block never crosses a row since K % 32 == 0), scattered to their
// permuted device positions.  Both nibbles of a device byte come from the
// same block, so no two threads write one byte.  Padded columns are not
// written (the activations there are zero).
__global__ void synth_values_kernel(int fmt, uint8_t *w, int O, int K, int kp, int count,
                                    uint64_t seed, uint32_t tid_base, int slot0) {
    const int per_block = fmt == FC_FMT_Q8 ? 8 : 32;
    const size_t mb = matrix_bytes(fmt, O, kp);
    const size_t blocks_per_member = (size_t)O * K / per_block;
    const size_t total = blocks_per_member * count;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        int member = (int)(idx / blocks_per_member);
        size_t blk = idx % blocks_per_member;
        uint32_t tid = tid_base | (uint32_t)(member + slot0);
        uint32_t words[4];
        fc_synth_block(seed, tid, FC_STREAM_VALUES, blk, words);
        size_t e0 = blk * per_block;
        int o = (int)(e0 / K), k0 = (int)(e0 % K);
        uint8_t *row = w + (size_t)member * mb;
        if (fmt == FC_FMT_Q8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                int v = ((int)fc_synth_byte(words, 2 * i) + (int)fc_synth_byte(words, 2 * i + 1) - 255) / 2;
                row[value_offset(fmt, kp, o, k0 + i, nullptr)] = (uint8_t)(int8_t)v;
            }
        } else {
            // gather the 16 device bytes this block covers: byte -> two nibbles
#pragma unroll 4
            for (int i = 0; i < 32; i += 2) {
                int nib0, nib1;
                size_t byte = value_offset(fmt, kp, o, k0 + i, &nib0);
                size_t byte1 = value_offset(fmt, kp, o, k0 + i + 1, &nib1);
                uint32_t c0 = (words[i >> 3] >> (4 * (i & 7))) & 0xFu;
                uint32_t c1 = (words[(i + 1) >> 3] >> (4 * ((i + 1) & 7))) & 0xFu;
                if (byte == byte1) {
                    row[byte] = (uint8_t)((c0 << (4 * nib0)) | (c1 << (4 * nib1)));
                } else {
                    // elements k, k+1 live in different bytes; their partner
                    // nibbles are elements k+2 / k+3 (same block)
                    int nib2, nib3;
                    value_offset(fmt, kp, o, k0 + i + 2, &nib2);
                    value_offset(fmt, kp, o, k0 + i + 3, &nib3);
                    uint32_t c2 = (words[(i + 2) >> 3] >> (4 * ((i + 2) & 7))) & 0xFu;
                    uint32_t c3 = (words[(i + 3) >> 3] >> (4 * ((i + 3) & 7))) & 0xFu;
                    row[byte] = (uint8_t)((c0 << (4 * nib0)) | (c2 << (4 * nib2)));
                    row[byte1] = (uint8_t)((c1 << (4 * nib1)) | (c3 << (4 * nib3)));
                    i += 2;
                }
            }
        }
    }
}

// Group scales: one thread per Philox block of 4 scales.
__global__ void synth_scales_kernel(int fmt, uint8_t *w, int O, int K, int kp, int count,
                                    uint64_t seed, uint32_t tid_base, int slot0) {
    const int gk = K / 32;
    const size_t mb = matrix_bytes(fmt, O, kp);
    const size_t groups = (size_t)O * gk;
    const size_t blocks_per_member = (groups + 3) / 4;
    const size_t total = blocks_per_member * count;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        int member = (int)(idx / blocks_per_member);
        size_t blk = idx % blocks_per_member;
        uint32_t tid = tid_base | (uint32_t)(member + slot0);
        uint32_t words[4];
        fc_synth_block(seed, tid, FC_STREAM_SCALES, blk, words);
        for (int i = 0; i < 4; ++i) {
            size_t lg = blk * 4 + i;
            if (lg >= groups) break;
            int o = (int)(lg / gk), g = (int)(lg % gk);
            uint8_t *dst = w + (size_t)member * mb + scale_offset(fmt, kp, o, g);
            uint32_t wd = words[i];
            if (fmt == FC_FMT_MXFP4)
                *dst = (uint8_t)(119u + (wd & 1u));
            else if (fmt == FC_FMT_Q8)
                *reinterpret_cast<uint16_t *>(dst) = (uint16_t)((3u << 10) | (wd & 0x3FFu));
            else
                *reinterpret_cast<uint16_t *>(dst) = (uint16_t)((7u << 10) | (wd & 0x3FFu));
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
