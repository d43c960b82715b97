// gemv.cuh - fused dequant-GEMV for the decode / verify regime (S <= 8 rows).
//
// Replaces moonlight_matmul_q8(_reduction) / _q4 (moonlight_kernels.metal
// :62-130), fm_matmul_q8 / q4 (backend_metal.m:124-130) and
// deepseek_v4_fp4_matmul_f32 (deepseek_v4_quant.h:103-139):
//     y[s][o] = sum_k x[s][k] * dequant(w[o][k])
// with fp32 accumulation.
//
// B200 design.  The step is HBM-bound: every weight byte is read once, so
// the kernel's only job is to keep enough bytes in flight and to spend few
// issue slots per byte.  Weights are dequantized exactly into fp16 registers
// (int8, int4 and e2m1 values are all exact in fp16) and multiplied on the
// tensor cores with mma.m16n8k16 against activations split into hi + lo fp16
// halves (about 22 significant bits), so one warp instruction covers 256
// weights.  The device weight layout is permuted (common.cuh,
// weight_position) so that each thread's 16-byte load feeds whole MMAs and
// each MMA covers one scale group; the per-group scale is applied in fp32 to
// the MMA result.  A CTA of 8 warps owns 32 output rows; warps take
// interleaved 64-byte column chunks and are reduced in a fixed order through
// shared memory, so every output row's summation order depends only on K,
// never on the number of rows S: a verify row is bit-identical to the same
// token decoded alone.
#pragma once

#include "common.cuh"

namespace fc {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * kWarp;
constexpr int kGemvRows = 32;  // two m16 tiles per CTA

enum GemvEpilogue {
    EPI_STORE = 0,      // y[s*ldy + o] = v
    EPI_ADD = 1,        // y[s*ldy + o] += v   (residual add, in place)
    EPI_STORE_XQ = 2,   // xq output at column col_off + o
    EPI_SWIGLU_XQ = 3   // tile 0 = gate rows, tile 1 = up rows -> silu(g)*u as xq
};

// One matrix (or a family of `count` equally shaped matrices laid out with
// fixed strides, e.g. the per-head W_UV blocks of kv_b) applied to one xq
// input and written through one epilogue.
struct GemvSeg {
    const uint8_t *w;       // device values, row stride row_bytes(fmt, kp)
    const void *sc;         // group scales [O][kp/32]
    const uint8_t *w2;      // SWIGLU: up-projection values
    const void *sc2;        // SWIGLU: up-projection scales
    const __half *xq;       // input rows [S][kp] in xq format
    float *y;               // EPI_STORE / EPI_ADD output
    __half *yq;             // xq outputs
    int O, kp;              // rows (per matrix), padded K
    int ldy;                // fp32 output row stride
    int kpy;                // xq output row length
    int col_off;            // xq output column offset
    int epi;
    int count;              // matrices in the family
    int64_t w_stride;       // bytes between family members
    int64_t sc_stride;      // scale elements between family members
    int64_t xq_stride;      // halves between family members' inputs
    int out_stride;         // output columns between family members
    int tiles;              // CTAs per member (filled by the launcher)
};

constexpr int kMaxSegs = 6;

struct GemvBatch {
    GemvSeg seg[kMaxSegs];
    int nseg;
    int S;
    float swiglu_limit;
};

// Accumulates the 32 x 8 output tile (two m16 tiles x one n8 tile) of rows
// [row0, row0 + 32) (tile t uses w_t, sc_t; rows >= nrows_t give zero) into
// shared memory `out` [32][8] after a fixed-order reduction over the warps.
template <int FMT>
__device__ __forceinline__ void gemv_tile(const uint8_t *w0, const void *sc0, int nrows0,
                                          const uint8_t *w1, const void *sc1, int nrows1,
                                          int kp, const __half *xq, int S, float *red,
                                          float *out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, j = lane & 3;
    const int rb = row_bytes(FMT, kp);
    const int groups = kp / 32;
    const int nchunks = rb / 64;
    constexpr int kMmas = FMT == FC_FMT_Q8 ? 4 : 8;  // MMAs per chunk
    constexpr int kGroups = kMmas / 2;               // scale groups per chunk

    const uint8_t *wp[2] = {w0, w1};
    const void *sp[2] = {sc0, sc1};
    const int nr[2] = {nrows0, nrows1};
    const bool has_b = g < S;

    float acc[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;

    for (int c = warp; c < nchunks; c += kGemvWarps) {
        // ---- loads: A (2 tiles x 2 rows x 16 bytes), scales, B (xq) ----
        uint4 a_raw[2][2];
        float scale[2][2][kGroups];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int r = g + 8 * h;
                if (r < nr[t]) {
                    a_raw[t][h] = ldg_stream(wp[t] + (size_t)r * rb + 64 * c + 16 * j);
                    if (FMT == FC_FMT_Q8) {
                        uint32_t s2 = __ldg(reinterpret_cast<const uint32_t *>(
                            reinterpret_cast<const __half *>(sp[t]) + (size_t)r * groups + 2 * c));
                        __half2 hs = *reinterpret_cast<__half2 *>(&s2);
                        scale[t][h][0] = __low2float(hs);
                        scale[t][h][1] = __high2float(hs);
                    } else if (FMT == FC_FMT_Q4) {
                        uint2 s4 = __ldg(reinterpret_cast<const uint2 *>(
                            reinterpret_cast<const __half *>(sp[t]) + (size_t)r * groups + 4 * c));
                        __half2 h0 = *reinterpret_cast<__half2 *>(&s4.x);
                        __half2 h1 = *reinterpret_cast<__half2 *>(&s4.y);
                        scale[t][h][0] = __low2float(h0);
                        scale[t][h][1] = __high2float(h0);
                        scale[t][h][kGroups > 2 ? 2 : 0] = __low2float(h1);
                        scale[t][h][kGroups > 3 ? 3 : 0] = __high2float(h1);
                    } else {
                        uint32_t s4 = __ldg(reinterpret_cast<const uint32_t *>(
                            reinterpret_cast<const uint8_t *>(sp[t]) + (size_t)r * groups + 4 * c));
#pragma unroll
                        for (int q = 0; q < kGroups; ++q)
                            scale[t][h][q] = e8m0_to_float((s4 >> (8 * q)) & 0xFFu);
                    }
                } else {
                    a_raw[t][h] = make_uint4(0, 0, 0, 0);
#pragma unroll
                    for (int q = 0; q < kGroups; ++q) scale[t][h][q] = 0.0f;
                }
            }
        }
        uint4 b_raw[kMmas];
#pragma unroll
        for (int i = 0; i < kMmas; ++i) {
            if (has_b) {
                int m = kMmas * c + i;  // global k16 step
                b_raw[i] = ldg_v4(xq + ((size_t)g * kp + 16 * m + 4 * j) * 2);
            } else {
                b_raw[i] = make_uint4(0, 0, 0, 0);
            }
        }

        // ---- dequant + MMA, one scale group (2 MMAs) at a time ----
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            uint32_t regs[2][16];  // per row h: fp16x2 registers (q index)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t words[4] = {a_raw[t][h].x, a_raw[t][h].y, a_raw[t][h].z,
                                           a_raw[t][h].w};
                if (FMT == FC_FMT_Q8) {
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi)
                        dequant_q8_word(words[wi], regs[h][2 * wi], regs[h][2 * wi + 1]);
                } else if (FMT == FC_FMT_Q4) {
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                        for (int s = 0; s < 4; ++s)
                            regs[h][4 * wi + s] = dequant_q4_pair(words[wi], 4 * s);
                } else {
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi) {
                        uint32_t o4[4];
                        dequant_e2m1_word(words[wi], o4);
#pragma unroll
                        for (int p = 0; p < 4; ++p) regs[h][4 * wi + p] = o4[p];
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < kGroups; ++q) {
                float tmp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int ii = 0; ii < 2; ++ii) {
                    int i = 2 * q + ii;
                    // A fragment: a0 = row g (k slots 2j,2j+1), a1 = row g+8,
                    // a2 = row g (slots 2j+8, 2j+9), a3 = row g+8.
                    uint32_t a[4] = {regs[0][2 * i], regs[1][2 * i], regs[0][2 * i + 1],
                                     regs[1][2 * i + 1]};
                    mma_f16(tmp, a, b_raw[i].x, b_raw[i].y, tmp);
                    mma_f16(tmp, a, b_raw[i].z, b_raw[i].w, tmp);
                }
                acc[t][0] = fmaf(scale[t][0][q], tmp[0], acc[t][0]);
                acc[t][1] = fmaf(scale[t][0][q], tmp[1], acc[t][1]);
                acc[t][2] = fmaf(scale[t][1][q], tmp[2], acc[t][2]);
                acc[t][3] = fmaf(scale[t][1][q], tmp[3], acc[t][3]);
            }
        }
    }

    // ---- fixed-order reduction over warps ----
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[((warp * 2 + t) * 32 + lane) * 4 + e] = acc[t][e];
    __syncthreads();
    {
        // 256 threads -> 256 outputs (2 tiles x 32 lanes x 4)
        int idx = threadIdx.x;
        int t = idx >> 7, l = (idx >> 2) & 31, e = idx & 3;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) sum += red[((w * 2 + t) * 32 + l) * 4 + e];
        int row = 16 * t + (l >> 2) + 8 * (e >> 1);
        int col = 2 * (l & 3) + (e & 1);
        out[row * 8 + col] = sum;
    }
    __syncthreads();
}

// Applies the epilogue of `sg` to the finished tile `out` [32][8] whose first
// row is `row0` of member matrix `member`.
__device__ __forceinline__ void gemv_epilogue(const GemvSeg &sg, int member, int row0,
                                              int S, float limit, const float *out) {
    int idx = threadIdx.x;
    if (sg.epi == EPI_SWIGLU_XQ) {
        if (idx >= 128) return;
        int r = idx >> 3, s = idx & 7;
        int o = row0 + r;
        if (s >= S || o >= sg.O) return;
        float gv = out[r * 8 + s], uv = out[(16 + r) * 8 + s];
        if (limit > 0.0f) {  // moe_exec.h:55-60
            gv = fminf(gv, limit);
            uv = fminf(fmaxf(uv, -limit), limit);
        }
        store_xq(sg.yq, sg.kpy, s, sg.col_off + member * sg.out_stride + o, silu(gv) * uv);
        return;
    }
    int r = idx >> 3, s = idx & 7;
    int o = row0 + r;
    if (s >= S || o >= sg.O) return;
    float v = out[r * 8 + s];
    int col = member * sg.out_stride + o;
    if (sg.epi == EPI_STORE) {
        sg.y[(size_t)s * sg.ldy + col] = v;
    } else if (sg.epi == EPI_ADD) {
        sg.y[(size_t)s * sg.ldy + col] += v;
    } else {
        store_xq(sg.yq, sg.kpy, s, sg.col_off + col, v);
    }
}

template <int FMT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_batch_kernel(const __grid_constant__ GemvBatch b) {
    __shared__ float red[kGemvWarps * 2 * 32 * 4];
    __shared__ float out[kGemvRows * 8];
    int block = blockIdx.x;
    int si = 0;
    while (si < b.nseg - 1 && block >= b.seg[si].tiles * b.seg[si].count) {
        block -= b.seg[si].tiles * b.seg[si].count;
        ++si;
    }
    const GemvSeg &sg = b.seg[si];
    int member = block / sg.tiles, tile = block % sg.tiles;
    const uint8_t *w = sg.w + member * sg.w_stride;
    const int rb = row_bytes(FMT, sg.kp);
    const size_t scale_elem = FMT == FC_FMT_MXFP4 ? 1 : 2;
    const uint8_t *sc = reinterpret_cast<const uint8_t *>(sg.sc) + member * sg.sc_stride * scale_elem;
    const __half *xq = sg.xq + member * sg.xq_stride;
    int row0;
    const uint8_t *w0, *w1;
    const void *s0, *s1;
    int n0, n1;
    int groups = sg.kp / 32;
    if (sg.epi == EPI_SWIGLU_XQ) {
        row0 = tile * 16;
        const uint8_t *up = sg.w2 + member * sg.w_stride;
        const uint8_t *usc = reinterpret_cast<const uint8_t *>(sg.sc2) + member * sg.sc_stride * scale_elem;
        w0 = w + (size_t)row0 * rb;
        w1 = up + (size_t)row0 * rb;
        s0 = sc + (size_t)row0 * groups * scale_elem;
        s1 = usc + (size_t)row0 * groups * scale_elem;
        n0 = n1 = min(16, sg.O - row0);
    } else {
        row0 = tile * 32;
        w0 = w + (size_t)row0 * rb;
        w1 = w + (size_t)(row0 + 16) * rb;
        s0 = sc + (size_t)row0 * groups * scale_elem;
        s1 = sc + (size_t)(row0 + 16) * groups * scale_elem;
        n0 = min(16, sg.O - row0);
        n1 = min(16, sg.O - row0 - 16);
    }
    gemv_tile<FMT>(w0, s0, n0, w1, s1, n1, sg.kp, xq, b.S, red, out);
    gemv_epilogue(sg, member, row0, b.S, b.swiglu_limit, out);
}

inline int gemv_tiles(const GemvSeg &s) {
    return s.epi == EPI_SWIGLU_XQ ? (s.O + 15) / 16 : (s.O + 31) / 32;
}

// Launches one batch of segments that share a weight format.
inline cudaError_t launch_gemv_batch(int fmt, GemvBatch &b, cudaStream_t stream) {
    int blocks = 0;
    for (int i = 0; i < b.nseg; ++i) {
        b.seg[i].tiles = gemv_tiles(b.seg[i]);
        if (b.seg[i].count <= 0) b.seg[i].count = 1;
        blocks += b.seg[i].tiles * b.seg[i].count;
    }
    if (blocks == 0) return cudaSuccess;
    switch (fmt) {
        case FC_FMT_Q8: gemv_batch_kernel<FC_FMT_Q8><<<blocks, kGemvThreads, 0, stream>>>(b); break;
        case FC_FMT_Q4: gemv_batch_kernel<FC_FMT_Q4><<<blocks, kGemvThreads, 0, stream>>>(b); break;
        case FC_FMT_MXFP4: gemv_batch_kernel<FC_FMT_MXFP4><<<blocks, kGemvThreads, 0, stream>>>(b); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace fc
