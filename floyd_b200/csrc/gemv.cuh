// gemv.cuh - fused dequant-GEMV for the decode / verify regime (S <= 8 rows).
//
// Replaces moonlight_matmul_q8(_reduction) / _q4 (moonlight_kernels.metal
// :62-130), fm_matmul_q8 / q4 (backend_metal.m:124-130) and
// deepseek_v4_fp4_matmul_f32 (deepseek_v4_quant.h:103-139):
//     y[s][o] = sum_k x[s][k] * dequant(w[o][k])
// with fp32 accumulation.
//
// B200 design.  The step is HBM-bound: every weight byte is read once, so the
// kernel's job is to keep HBM busy and to spend few issue slots per byte.
//   - A CTA owns two 16-row tiles (two tiles of one matrix, or the gate and
//     up tiles of a SwiGLU pair).  A tile is contiguous in the tile-major
//     layout (common.cuh), so one thread streams it through shared memory
//     with cp.async.bulk (TMA 1-D bulk copies) in 8-chunk stages, kStages
//     stages in flight, completion tracked by mbarriers.
//   - Each of the 8 warps takes one chunk of every stage, dequantizes it
//     exactly into fp16 registers (int8, int4 and e2m1 values are all exact
//     in fp16) and runs m16n8k16 tensor-core MMAs against the activations
//     split into hi + lo fp16 halves (about 22 significant bits), one scale
//     group per MMA pair, the group scale applied in fp32 to the MMA result.
//   - Warps are reduced in a fixed order through shared memory, so every
//     output's summation order depends only on K, never on the number of
//     rows S: a verify row is bit-identical to the same token decoded alone.
#pragma once

#include "common.cuh"

namespace fc {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * kWarp;
constexpr int kGemvRows = 32;  // two 16-row tiles per CTA
constexpr int kStages = 4;     // bulk-copy stages in flight per CTA

__host__ __device__ constexpr size_t gemv_stage_bytes(int fmt) {
    return (size_t)kGemvWarps * block_bytes(fmt);
}
__host__ __device__ constexpr size_t gemv_smem_bytes(int fmt) {
    return (size_t)kStages * 2 * gemv_stage_bytes(fmt) + kStages * 8;
}

enum GemvEpilogue {
    EPI_STORE = 0,      // y[s*ldy + o] = v
    EPI_ADD = 1,        // y[s*ldy + o] += v   (residual add, in place)
    EPI_STORE_XQ = 2,   // xq output at column col_off + o
    EPI_SWIGLU_XQ = 3   // tile 0 = gate rows, tile 1 = up rows -> silu(g)*u as xq
};

// One matrix (or a family of `count` equally shaped matrices laid out with a
// fixed stride, e.g. the per-head W_UV blocks of kv_b) applied to one xq
// input and written through one epilogue.
struct GemvSeg {
    const uint8_t *w;       // tile-major values + scales
    const uint8_t *w2;      // SWIGLU: up-projection (same shape as w)
    const __half *xq;       // input rows [S][kp] in xq format
    float *y;               // EPI_STORE / EPI_ADD output
    __half *yq;             // xq outputs
    int O, kp;              // rows (per member), padded K
    int ldy;                // fp32 output row stride
    int kpy;                // xq output row length
    int col_off;            // xq output column offset
    int epi;
    int count;              // members in the family
    int64_t w_stride;       // bytes between members
    int64_t xq_stride;      // halves between members' inputs
    int out_stride;         // output columns between members
    int tiles;              // CTAs per member (set by the launcher)
};

constexpr int kMaxSegs = 6;

struct GemvBatch {
    GemvSeg seg[kMaxSegs];
    int nseg;
    int S;
    float swiglu_limit;
    int *err;
};

// Streams tiles t0 / t1 (nullptr = absent) of padded width kp through shared
// memory and leaves the reduced 32 x 8 tile (rows 0-15 from t0, 16-31 from
// t1, columns = activation rows) in `out`.
template <int FMT>
__device__ __forceinline__ void gemv_tile(const uint8_t *t0, const uint8_t *t1, int kp,
                                          const __half *xq, int S, uint8_t *smem, float *red,
                                          float *out, int *err) {
    constexpr int kBlock = block_bytes(FMT);
    constexpr size_t kStageBytes = gemv_stage_bytes(FMT);
    constexpr int kMmas = FMT == FC_FMT_Q8 ? 4 : 8;  // MMAs per chunk
    constexpr int kGroups = kMmas / 2;               // scale groups per chunk
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, j = lane & 3;
    const int nchunks = chunk_count(FMT, kp);
    const int nstages = (nchunks + kGemvWarps - 1) / kGemvWarps;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStages * 2 * kStageBytes);
    const uint8_t *src[2] = {t0, t1};

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int s) {
        int slot = s % kStages;
        int c0 = s * kGemvWarps;
        int nc = min(kGemvWarps, nchunks - c0);
        uint32_t bytes = (uint32_t)(nc * kBlock);
        uint32_t total = bytes * ((t0 ? 1u : 0u) + (t1 ? 1u : 0u));
        mbar_expect_tx(&bars[slot], total);
        for (int t = 0; t < 2; ++t)
            if (src[t])
                bulk_g2s(smem + (slot * 2 + t) * kStageBytes, src[t] + (size_t)c0 * kBlock, bytes,
                         &bars[slot]);
    };
    if (tid == 0)
        for (int s = 0; s < min(kStages, nstages); ++s) issue(s);

    const bool has_b = g < S;
    float acc[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;

    for (int s = 0; s < nstages; ++s) {
        const int slot = s % kStages;
        const int c = s * kGemvWarps + warp;
        // B fragments (activations, L2-resident) are fetched before the wait
        uint4 b_raw[kMmas];
#pragma unroll
        for (int i = 0; i < kMmas; ++i) {
            if (has_b && c < nchunks)
                b_raw[i] = ldg_v4(xq + ((size_t)g * kp + 16 * (kMmas * c + i) + 4 * j) * 2);
            else
                b_raw[i] = make_uint4(0, 0, 0, 0);
        }
        mbar_wait_bounded(&bars[slot], (uint32_t)((s / kStages) & 1), err);
        if (c < nchunks) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                if (!src[t]) continue;
                const uint8_t *blk = smem + (slot * 2 + t) * kStageBytes + (size_t)warp * kBlock;
                uint4 a_raw[2];
                float scale[2][kGroups];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    int r = g + 8 * h;
                    a_raw[h] = *reinterpret_cast<const uint4 *>(blk + r * 64 + 16 * j);
                    const uint8_t *sp = blk + kBlockValueBytes + r * scale_row_bytes(FMT);
                    if (FMT == FC_FMT_Q8) {
                        __half2 hs = *reinterpret_cast<const __half2 *>(sp);
                        scale[h][0] = __low2float(hs);
                        scale[h][kGroups > 1 ? 1 : 0] = __high2float(hs);
                    } else if (FMT == FC_FMT_Q4) {
                        uint2 s4 = *reinterpret_cast<const uint2 *>(sp);
                        __half2 h0 = *reinterpret_cast<__half2 *>(&s4.x);
                        __half2 h1 = *reinterpret_cast<__half2 *>(&s4.y);
                        scale[h][0] = __low2float(h0);
                        scale[h][1] = __high2float(h0);
                        scale[h][kGroups > 2 ? 2 : 0] = __low2float(h1);
                        scale[h][kGroups > 3 ? 3 : 0] = __high2float(h1);
                    } else {
                        uint32_t s4 = *reinterpret_cast<const uint32_t *>(sp);
#pragma unroll
                        for (int q = 0; q < kGroups; ++q)
                            scale[h][q] = e8m0_to_float((s4 >> (8 * q)) & 0xFFu);
                    }
                }
                uint32_t regs[2][16];  // per row h: fp16x2 registers (index q)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t words[4] = {a_raw[h].x, a_raw[h].y, a_raw[h].z, a_raw[h].w};
                    if (FMT == FC_FMT_Q8) {
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi)
                            dequant_q8_word(words[wi], regs[h][2 * wi], regs[h][2 * wi + 1]);
                    } else if (FMT == FC_FMT_Q4) {
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                            for (int sh = 0; sh < 4; ++sh)
                                regs[h][4 * wi + sh] = dequant_q4_pair(words[wi], 4 * sh);
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
                        // a0 = row g (k slots 2j,2j+1), a1 = row g+8,
                        // a2 = row g (slots 2j+8, 2j+9), a3 = row g+8.
                        uint32_t a[4] = {regs[0][2 * i], regs[1][2 * i], regs[0][2 * i + 1],
                                         regs[1][2 * i + 1]};
                        mma_f16(tmp, a, b_raw[i].x, b_raw[i].y, tmp);
                        mma_f16(tmp, a, b_raw[i].z, b_raw[i].w, tmp);
                    }
                    acc[t][0] = fmaf(scale[0][q], tmp[0], acc[t][0]);
                    acc[t][1] = fmaf(scale[0][q], tmp[1], acc[t][1]);
                    acc[t][2] = fmaf(scale[1][q], tmp[2], acc[t][2]);
                    acc[t][3] = fmaf(scale[1][q], tmp[3], acc[t][3]);
                }
            }
        }
        __syncthreads();  // every warp is done with this slot
        if (tid == 0 && s + kStages < nstages) issue(s + kStages);
    }

    // ---- fixed-order reduction over warps ----
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[((warp * 2 + t) * 32 + lane) * 4 + e] = acc[t][e];
    __syncthreads();
    {
        int idx = threadIdx.x;  // 256 threads -> 2 tiles x 32 lanes x 4
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
__device__ __forceinline__ void gemv_epilogue(const GemvSeg &sg, int member, int row0, int S,
                                              float limit, const float *out) {
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

// CTA `tile` of a member matrix: the two tile streams and the first row.
template <int FMT>
__device__ __forceinline__ void seg_tiles(const GemvSeg &sg, const uint8_t *w, const uint8_t *w2,
                                          int tile, const uint8_t *&t0, const uint8_t *&t1,
                                          int &row0) {
    const size_t tb = tile_bytes(FMT, sg.kp);
    const int ntiles = (sg.O + kTileRows - 1) / kTileRows;
    if (sg.epi == EPI_SWIGLU_XQ) {
        row0 = tile * kTileRows;
        t0 = w + (size_t)tile * tb;
        t1 = w2 + (size_t)tile * tb;
    } else {
        row0 = tile * 2 * kTileRows;
        t0 = w + (size_t)(2 * tile) * tb;
        t1 = 2 * tile + 1 < ntiles ? w + (size_t)(2 * tile + 1) * tb : nullptr;
    }
}

template <int FMT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_batch_kernel(const __grid_constant__ GemvBatch b) {
    extern __shared__ __align__(128) uint8_t gemv_smem[];
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
    const uint8_t *w2 = sg.w2 ? sg.w2 + member * sg.w_stride : nullptr;
    const __half *xq = sg.xq + member * sg.xq_stride;
    const uint8_t *t0, *t1;
    int row0;
    seg_tiles<FMT>(sg, w, w2, tile, t0, t1, row0);
    gemv_tile<FMT>(t0, t1, sg.kp, xq, b.S, gemv_smem, red, out, b.err);
    gemv_epilogue(sg, member, row0, b.S, b.swiglu_limit, out);
}

inline int gemv_tiles(const GemvSeg &s) {
    int ntiles = (s.O + kTileRows - 1) / kTileRows;
    return s.epi == EPI_SWIGLU_XQ ? ntiles : (ntiles + 1) / 2;
}

// Opts the GEMV kernels into their dynamic shared memory (call once per
// device before launching or capturing).
inline cudaError_t gemv_prepare_all() {
    cudaError_t e = cudaFuncSetAttribute(gemv_batch_kernel<FC_FMT_Q8>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)gemv_smem_bytes(FC_FMT_Q8));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_batch_kernel<FC_FMT_Q4>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)gemv_smem_bytes(FC_FMT_Q4));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_batch_kernel<FC_FMT_MXFP4>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)gemv_smem_bytes(FC_FMT_MXFP4));
    return e;
}

// Launches one batch of segments that share a weight format.
inline cudaError_t launch_gemv_batch(int fmt, GemvBatch &b, cudaStream_t stream) {
    int blocks = 0;
    for (int i = 0; i < b.nseg; ++i) {
        if (b.seg[i].count <= 0) b.seg[i].count = 1;
        b.seg[i].tiles = gemv_tiles(b.seg[i]);
        blocks += b.seg[i].tiles * b.seg[i].count;
    }
    if (blocks == 0) return cudaSuccess;
    switch (fmt) {
        case FC_FMT_Q8:
            gemv_batch_kernel<FC_FMT_Q8><<<blocks, kGemvThreads, gemv_smem_bytes(FC_FMT_Q8), stream>>>(b);
            break;
        case FC_FMT_Q4:
            gemv_batch_kernel<FC_FMT_Q4><<<blocks, kGemvThreads, gemv_smem_bytes(FC_FMT_Q4), stream>>>(b);
            break;
        case FC_FMT_MXFP4:
            gemv_batch_kernel<FC_FMT_MXFP4><<<blocks, kGemvThreads, gemv_smem_bytes(FC_FMT_MXFP4), stream>>>(b);
            break;
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace fc
