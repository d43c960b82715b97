/*
 * floyd_synth.h - the seeded synthetic-model generator shared by the CUDA
 * backend (device fill) and the CPU oracle.
 *
 * The reference benchmarks on random weights drawn from N(0, 0.02) and then
 * quantized (tools/make_oracle.py:12-44 builds its tiny fixture the same way).
 * Drawing floats and quantizing them would let the host and device libm
 * differ in the last bit, so this generator produces the quantized
 * representation directly with integer arithmetic only: every value is a
 * function of (seed, tensor id, element index) through Philox4x32-10
 * (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
 * SC'11).  The host and the device therefore generate bit-identical weights.
 *
 *   int8 value  v = trunc((b0 + b1 - 255) / 2)       triangular, std ~ 52
 *   int4 value  nibble uniform in [0, 15] (value = nibble - 8)
 *   e2m1 code   uniform in [0, 15]
 *   fp16 scale  exponent fixed per format, 10 random mantissa bits, so that
 *               value * scale has a standard deviation of about 0.02
 *   ue8m0 scale 119 or 120 (2^-8 or 2^-7)
 *   fp32 matrix (b0 + b1 - 255) * 2^-13                  exact in fp32
 *   norm weight 1 + (b0 - 128) * 2^-9                     exact in fp32
 *   latent KV   (b0 + b1 - 255) * 2^-7                    exact in fp16
 *
 * Bytes b0, b1 are consecutive bytes of the Philox output for the element.
 */
#ifndef FLOYD_SYNTH_H
#define FLOYD_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define FC_HD __host__ __device__ __forceinline__
#else
#define FC_HD static inline
#endif

/* Tensor kinds.  A tensor id is (layer + 1) << 20 | kind << 12 | slot, where
 * slot is expert + 1 for routed experts and 0 otherwise; layer -1 marks the
 * global tensors. */
enum {
    FC_T_EMBED = 1, FC_T_FINAL_NORM, FC_T_LM_HEAD,
    FC_T_ATTN_NORM, FC_T_Q_PROJ, FC_T_Q_A, FC_T_Q_A_NORM, FC_T_Q_B,
    FC_T_KV_A, FC_T_KV_A_NORM, FC_T_KV_B, FC_T_O_PROJ,
    FC_T_FFN_NORM, FC_T_ROUTER, FC_T_ROUTER_BIAS, FC_T_HASH,
    FC_T_EXP_GATE, FC_T_EXP_UP, FC_T_EXP_DOWN,
    FC_T_SH_GATE, FC_T_SH_UP, FC_T_SH_DOWN,
    FC_T_DENSE_GATE, FC_T_DENSE_UP, FC_T_DENSE_DOWN,
    FC_T_KV_LATENT, FC_T_KV_ROPE,
    FC_T_MTP_ENORM, FC_T_MTP_HNORM, FC_T_MTP_EH_PROJ, FC_T_MTP_HEAD_NORM
};

/* Streams inside one tensor's counter space. */
enum { FC_STREAM_VALUES = 0, FC_STREAM_SCALES = 1 };

FC_HD uint32_t fc_tensor_id(int layer, int kind, int slot) {
    return ((uint32_t)(layer + 1) << 20) | ((uint32_t)kind << 12) | (uint32_t)slot;
}

FC_HD uint32_t fc_mulhilo32(uint32_t a, uint32_t b, uint32_t *hi) {
    uint64_t product = (uint64_t)a * (uint64_t)b;
    *hi = (uint32_t)(product >> 32);
    return (uint32_t)product;
}

/* Philox4x32 with 10 rounds (SC'11, section 3; constants from the paper). */
FC_HD void fc_philox4x32_10(const uint32_t counter[4], const uint32_t key[2],
                            uint32_t out[4]) {
    uint32_t c0 = counter[0], c1 = counter[1], c2 = counter[2], c3 = counter[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int round = 0; round < 10; ++round) {
        uint32_t hi0, hi1;
        uint32_t lo0 = fc_mulhilo32(0xD2511F53u, c0, &hi0);
        uint32_t lo1 = fc_mulhilo32(0xCD9E8D57u, c2, &hi1);
        uint32_t n0 = hi1 ^ c1 ^ k0;
        uint32_t n1 = lo1;
        uint32_t n2 = hi0 ^ c3 ^ k1;
        uint32_t n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* 16 random bytes for block `block` of (tensor, stream). */
FC_HD void fc_synth_block(uint64_t seed, uint32_t tensor, uint32_t stream,
                          uint64_t block, uint32_t out[4]) {
    uint32_t counter[4] = {(uint32_t)block, (uint32_t)(block >> 32), tensor, stream};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    fc_philox4x32_10(counter, key, out);
}

FC_HD uint32_t fc_synth_byte(const uint32_t words[4], int index) {
    return (words[index >> 2] >> (8 * (index & 3))) & 0xFFu;
}

/* Element e uses bytes 2*(e%8), 2*(e%8)+1 of block e/8. */
FC_HD int fc_synth_pair(uint64_t seed, uint32_t tensor, uint32_t stream, uint64_t e) {
    uint32_t words[4];
    fc_synth_block(seed, tensor, stream, e >> 3, words);
    int slot = (int)(e & 7);
    return (int)fc_synth_byte(words, 2 * slot) + (int)fc_synth_byte(words, 2 * slot + 1) - 255;
}

/* int8 weight value in [-127, 127]. */
FC_HD int fc_synth_q8(uint64_t seed, uint32_t tensor, uint64_t e) {
    return fc_synth_pair(seed, tensor, FC_STREAM_VALUES, e) / 2;
}

/* 4-bit code (int4 nibble or e2m1 code): nibble e%32 of block e/32. */
FC_HD int fc_synth_nibble(uint64_t seed, uint32_t tensor, uint64_t e) {
    uint32_t words[4];
    fc_synth_block(seed, tensor, FC_STREAM_VALUES, e >> 5, words);
    int slot = (int)(e & 31);
    return (int)((words[slot >> 3] >> (4 * (slot & 7))) & 0xFu);
}

/* Group scale bits for group g: fp16 bits for Q8 / Q4, a ue8m0 byte for MXFP4.
 * Word g%4 of block g/4 of the scale stream. */
FC_HD uint32_t fc_synth_scale_word(uint64_t seed, uint32_t tensor, uint64_t g) {
    uint32_t words[4];
    fc_synth_block(seed, tensor, FC_STREAM_SCALES, g >> 2, words);
    return words[g & 3];
}

FC_HD uint16_t fc_synth_scale_q8(uint64_t seed, uint32_t tensor, uint64_t g) {
    /* exponent field 3: [2^-12, 2^-11) */
    return (uint16_t)((3u << 10) | (fc_synth_scale_word(seed, tensor, g) & 0x3FFu));
}

FC_HD uint16_t fc_synth_scale_q4(uint64_t seed, uint32_t tensor, uint64_t g) {
    /* exponent field 7: [2^-8, 2^-7) */
    return (uint16_t)((7u << 10) | (fc_synth_scale_word(seed, tensor, g) & 0x3FFu));
}

FC_HD uint8_t fc_synth_scale_e8m0(uint64_t seed, uint32_t tensor, uint64_t g) {
    return (uint8_t)(119u + (fc_synth_scale_word(seed, tensor, g) & 1u));
}

/* fp32 matrix element (router weights): exact multiple of 2^-13. */
FC_HD float fc_synth_f32(uint64_t seed, uint32_t tensor, uint64_t e) {
    return (float)fc_synth_pair(seed, tensor, FC_STREAM_VALUES, e) * (1.0f / 8192.0f);
}

/* Norm weight: 1 + (b - 128) * 2^-9. */
FC_HD float fc_synth_norm(uint64_t seed, uint32_t tensor, uint64_t e) {
    uint32_t words[4];
    fc_synth_block(seed, tensor, FC_STREAM_VALUES, e >> 4, words);
    int b = (int)fc_synth_byte(words, (int)(e & 15));
    return 1.0f + (float)(b - 128) * (1.0f / 512.0f);
}

/* Selection bias: (b - 128) * 2^-10. */
FC_HD float fc_synth_bias(uint64_t seed, uint32_t tensor, uint64_t e) {
    uint32_t words[4];
    fc_synth_block(seed, tensor, FC_STREAM_VALUES, e >> 4, words);
    int b = (int)fc_synth_byte(words, (int)(e & 15));
    return (float)(b - 128) * (1.0f / 1024.0f);
}

/* Latent / rope KV element: multiple of 2^-7, |v| <= 255/128. */
FC_HD float fc_synth_kv(uint64_t seed, uint32_t tensor, uint64_t e) {
    return (float)fc_synth_pair(seed, tensor, FC_STREAM_VALUES, e) * (1.0f / 128.0f);
}

/* Hash routing table entry (layers < hash_layer_count): top_k distinct
 * experts per token, (base + slot * (E / top_k)) mod E. */
FC_HD int fc_synth_hash_expert(uint64_t seed, uint32_t tensor, int token, int slot,
                               int n_experts, int top_k) {
    uint32_t words[4];
    fc_synth_block(seed, tensor, FC_STREAM_VALUES, (uint64_t)token, words);
    int base = (int)(words[0] % (uint32_t)n_experts);
    int stride = n_experts / top_k;
    if (stride < 1) stride = 1;
    return (base + slot * stride) % n_experts;
}

#endif /* FLOYD_SYNTH_H */
