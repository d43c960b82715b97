// gemv.cuh - fused dequant-GEMV for the decode / verify regime (S <= 8 rows).
//
// Replaces moonlight_matmul_q8(_reduction) / _q4 (moonlight_kernels.metal
// :62-130), fm_matmul_q8 / q4 (backend_metal.m:124-130) and
// deepseek_v4_fp4_matmul_f32 (deepseek_v4_quant.h:103-139):
//     y[s][o] = sum_k x[s][k] * dequant(w[o][k])
// with fp32 accumulation, plus the grouped expert form of
// encode_moe_residual_buffer (moonlight_metal.m:561-676).
//
// B200 design.  The step is HBM-bound: every weight byte is read once, so the
// kernel's job is to keep HBM busy and to spend few issue slots per byte.
//   - Work items are pairs of 16-row tiles (two tiles of one matrix, or the
//     gate and up tiles of a SwiGLU pair).  A tile is contiguous in the
//     tile-major layout (common.cuh).
//   - The kernel is persistent and warp-specialized: CTAs loop over work
//     items; one producer warp streams every item's tiles through a ring of
//     kStages shared-memory stages with cp.async.bulk (TMA 1-D bulk copies),
//     full / empty mbarriers between it and the consumers, so copies for the
//     next item are in flight while the current one is reduced.
//   - Each of the 8 consumer warps takes one 64-byte-per-row chunk of every
//     stage, dequantizes it exactly into fp16 registers (int8, int4 and e2m1
//     values are all exact in fp16) and runs m16n8k16 tensor-core MMAs
//     against the activations split into hi + lo fp16 halves (about 22
//     significant bits); each MMA pair covers one 32-column scale group and
//     the group scale is applied in fp32 to the MMA result.
//   - Warps are reduced in a fixed order through shared memory, so every
//     output's summation order depends only on K, never on the number of
//     rows S or on the work distribution: a verify row is bit-identical to
//     the same token decoded alone.
#pragma once

#include "common.cuh"

namespace fc {

constexpr int kGemvWarps = 8;                      // consumer warps
constexpr int kGemvThreads = (kGemvWarps + 1) * kWarp;  // + producer warp
constexpr int kGemvConsumers = kGemvWarps * kWarp;
constexpr int kGemvRows = 32;  // two 16-row tiles per work item
constexpr int kStages = 4;     // most bulk-copy stages in the ring

__host__ __device__ constexpr size_t gemv_stage_bytes(int fmt) {
    return (size_t)kGemvWarps * block_bytes(fmt);
}
__host__ __device__ constexpr size_t gemv_slot_w(int fa, int fb) {
    return gemv_stage_bytes(fa) > gemv_stage_bytes(fb) ? gemv_stage_bytes(fa) : gemv_stage_bytes(fb);
}
// Every launch stages each stage's activation rows in shared memory next to
// the weights (the producer copies them), so the consumers never wait on L2
// for B fragments (FC_GEMV_NO_SMEM_B builds the global-load variant for
// measurements).
__host__ __device__ constexpr bool gemv_smem_b(int fa, int fb) {
#if defined(FC_GEMV_NO_SMEM_B)
    return false;
#else
    return true;
#endif
}
// Bytes of one activation row of one stage (kGemvWarps chunks, hi + lo fp16,
// 4 B per column), padded so the rows start in different banks.
__host__ __device__ constexpr int gemv_b_row_bytes(int fa, int fb) {
    return kGemvWarps * (chunk_cols(fa) > chunk_cols(fb) ? chunk_cols(fa) : chunk_cols(fb)) * 4 + 64;
}
constexpr size_t kGemvDynSmemBudget = 100 * 1024;  // two CTAs per SM with the static arrays
__host__ __device__ constexpr size_t gemv_slot_bytes(int fa, int fb, int S) {
    return 2 * gemv_slot_w(fa, fb) + (gemv_smem_b(fa, fb) ? (size_t)S * gemv_b_row_bytes(fa, fb) : 0);
}
// Ring depth: as many stages as the budget holds, at least two (wide
// formats with 8 activation rows then exceed the budget and run one CTA per
// SM).
inline int gemv_stages(int fa, int fb, int S) {
    int n = (int)((kGemvDynSmemBudget - 2 * kStages * 8) / gemv_slot_bytes(fa, fb, S));
    return n > kStages ? kStages : (n < 2 ? 2 : n);
}
inline size_t gemv_smem_bytes(int fa, int fb, int S) {
    return (size_t)gemv_stages(fa, fb, S) * gemv_slot_bytes(fa, fb, S) + 2 * kStages * 8;
}
inline size_t gemv_smem_max(int fa, int fb) {  // over 1 .. 8 activation rows
    size_t m = 0;
    for (int S = 1; S <= 8; ++S) m = gemv_smem_bytes(fa, fb, S) > m ? gemv_smem_bytes(fa, fb, S) : m;
    return m;
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
    int tiles;              // work items per member (set by the launcher)
    int npeer;              // EPI_STORE / EPI_STORE_XQ copies into peer GPUs' buffers
    float *peer_y[7];       // same offsets as y (or yq, as __half *) in each peer's buffer
};

constexpr int kMaxSegs = 6;

// A launch: either a batch of static segments sharing format FA, or (moe = 1)
// the grouped routed experts (seg[0], format FA, member = active[slot] -
// expert_base, per-slot inputs / outputs) followed by the shared expert
// (seg[1], format FB).
struct GemvWork {
    GemvSeg seg[kMaxSegs];
    int nseg;
    int moe;
    int max_slots;
    int expert_base;
    const int *n_active;
    const int *active;
    int64_t in_slot_stride;   // halves between slots' xq inputs
    int64_t out_slot_stride;  // floats (EPI_STORE) or halves (xq) between slots
    const int *slot_base;     // nullable: global slot of local slot 0 (expert parallel)
    const int *ep_epoch;      // nullable: receive buffer = (epoch + 1) & 1
    int64_t parity_stride;    // floats between the two receive buffers
    int total_items;
    int S;
    float swiglu_limit;
    int *err;
    int stages;               // ring depth (set by the launcher)
    // MoE gate/up: the shared expert's items come first and run before the
    // wait on the predecessor (the router).  Its input is the RMSNorm output
    // two kernels back, complete by the time this kernel can start: the
    // router releases its dependents only after its own wait.  (This kernel
    // releases its dependents at its start, so its successor may not assume
    // the same of the router.)
    int shared_first;
    // cross-GPU hand-off (head-parallel attention), all nullable:
    // publish - the last CTA to finish (done counter, zero between launches)
    //   stores epoch + 1 into every peer's flag slot `rank` after the CTAs'
    //   peer stores are fenced;
    // wait - the producer waits (bounded, error bit 2) until every peer has
    //   published this GPU's current epoch before copying activation rows
    int *pub_done, *pub_epoch;
    int *pub_flags[8];        // each peer's flag array, by peer rank (slot = this rank)
    const int *wait_flags, *wait_epoch;
    unsigned long long *wait_ns;
    int peer_world, peer_rank;
#ifdef FC_GEMV_TRACE
    int trace;
#endif
};

__device__ __forceinline__ void gemv_peer_wait(const GemvWork &wk) {
    if (!wk.wait_flags) return;
    const int e = *wk.wait_epoch;
    uint64_t t0 = 0, w0, w1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(w0));
    for (int r = 0; r < wk.peer_world; ++r) {
        if (r == wk.peer_rank) continue;
        for (uint32_t it = 0;; ++it) {
            int v;
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];\n" : "=r"(v) : "l"(wk.wait_flags + r) : "memory");
            if (v >= e) break;
            if ((it & 255u) == 0) {
                uint64_t t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (t0 == 0) t0 = t;
                else if (t - t0 > 1000000000ull) {
                    atomicOr(wk.err, 2);
                    break;
                }
            }
        }
    }
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(w1));
    if (wk.wait_ns && blockIdx.x == 0) atomicAdd(wk.wait_ns, (unsigned long long)(w1 - w0));
}

// A resolved work item.
struct GemvItem {
    const uint8_t *t0, *t1;
    const __half *xq;
    int kp, fmt, seg, member, row0;
    int64_t out_shift;  // slot offset of the outputs
};

__device__ __forceinline__ int seg_items(const GemvSeg &s) {
    int ntiles = (s.O + kTileRows - 1) / kTileRows;
    return s.epi == EPI_SWIGLU_XQ ? ntiles : (ntiles + 1) / 2;
}

template <int FA, int FB>
__device__ __forceinline__ bool resolve_item(const GemvWork &wk, int item, GemvItem &it) {
    int si, member, tile;
    it.out_shift = 0;
    if (wk.moe) {
        const GemvSeg &r = wk.seg[0];
        int rt = r.tiles;
        int routed_items = wk.max_slots * rt;
        if (wk.shared_first) {  // shared items first, then the routed ones
            item = item < wk.seg[1].tiles ? routed_items + item : item - wk.seg[1].tiles;
        }
        if (item < routed_items) {
            int slot = item / rt;
            if (slot >= *wk.n_active) return false;
            si = 0;
            tile = item % rt;
            member = wk.active[slot] - wk.expert_base;
            it.xq = r.xq + slot * wk.in_slot_stride;
            it.out_shift = (slot + (wk.slot_base ? *wk.slot_base : 0)) * wk.out_slot_stride;
            if (wk.ep_epoch) it.out_shift += ((*wk.ep_epoch + 1) & 1) * wk.parity_stride;
            it.fmt = FA;
        } else {
            si = 1;
            tile = item - routed_items;
            member = 0;
            it.xq = wk.seg[1].xq;
            it.fmt = FB;
        }
    } else {
        si = 0;
        while (si < wk.nseg - 1 && item >= wk.seg[si].tiles * wk.seg[si].count) {
            item -= wk.seg[si].tiles * wk.seg[si].count;
            ++si;
        }
        member = item / wk.seg[si].tiles;
        tile = item % wk.seg[si].tiles;
        it.xq = wk.seg[si].xq + member * wk.seg[si].xq_stride;
        it.fmt = FA;
    }
    const GemvSeg &sg = wk.seg[si];
    it.seg = si;
    it.member = wk.moe ? 0 : member;
    it.kp = sg.kp;
    const uint8_t *w = sg.w + member * sg.w_stride;
    const size_t tb = tile_bytes(it.fmt, sg.kp);
    const int ntiles = (sg.O + kTileRows - 1) / kTileRows;
    if (sg.epi == EPI_SWIGLU_XQ) {
        it.row0 = tile * kTileRows;
        it.t0 = w + (size_t)tile * tb;
        it.t1 = sg.w2 + member * sg.w_stride + (size_t)tile * tb;
    } else {
        it.row0 = tile * 2 * kTileRows;
        it.t0 = w + (size_t)(2 * tile) * tb;
        it.t1 = 2 * tile + 1 < ntiles ? w + (size_t)(2 * tile + 1) * tb : nullptr;
    }
    return true;
}

// Consumes one chunk block per tile from shared memory and accumulates
// the 2 x (16 x 8) partial tile of this warp.  The activation fragments
// carry fp16 hi / lo halves.  PACK (at most 4 activation rows): one MMA per
// fragment, B columns 0-3 the hi halves of rows 0-3 and columns 4-7 their lo
// halves (b_raw[i].x/.y).  Otherwise hi (.x/.y) and lo (.z/.w) go to two MMAs
// with separate accumulators (acc, accl).  Each output column of an MMA is
// its own dot product, so both forms give the same bits for a row.
template <int FMT, bool PACK>
__device__ __forceinline__ void gemv_chunk(const uint8_t *blk0, const uint8_t *blk1,
                                           const uint4 (&b_raw)[8], float (&acc)[2][4],
                                           float (&accl)[2][4]) {
    constexpr int kMmas = FMT == FC_FMT_Q8 ? 4 : 8;
    constexpr int kGroups = kMmas / 2;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, j = lane & 3;
    const uint8_t *blks[2] = {blk0, blk1};
    if constexpr (FMT == FC_FMT_MXFP4) {
        // group by group: each group's 8 codes per row are decoded right
        // before its two MMAs, so few registers are live at a time (the
        // same arithmetic, in the same order, as the general path below)
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const uint8_t *blk = blks[t];
            if (!blk) continue;
            uint4 a_raw[2];
            uint32_t s4[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = g + 8 * h;
                a_raw[h] = *reinterpret_cast<const uint4 *>(blk + r * 64 + 16 * j);
                s4[h] = *reinterpret_cast<const uint32_t *>(blk + kBlockValueBytes + r * scale_row_bytes(FMT));
            }
#pragma unroll
            for (int q = 0; q < kGroups; ++q) {
                const uint32_t w0 = q == 0 ? a_raw[0].x : q == 1 ? a_raw[0].y : q == 2 ? a_raw[0].z : a_raw[0].w;
                const uint32_t w1 = q == 0 ? a_raw[1].x : q == 1 ? a_raw[1].y : q == 2 ? a_raw[1].z : a_raw[1].w;
                uint32_t r0[4], r1[4];
                dequant_e2m1_word(w0, r0);
                dequant_e2m1_word(w1, r1);
                float sc0[4], sc1[4];
                e8m0x4_to_float(s4[0], sc0);
                e8m0x4_to_float(s4[1], sc1);
                float tmp[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                float tml[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int ii = 0; ii < 2; ++ii) {
                    const int i = 2 * q + ii;
                    uint32_t a[4] = {r0[2 * ii], r1[2 * ii], r0[2 * ii + 1], r1[2 * ii + 1]};
                    mma_f16(tmp, a, b_raw[i].x, b_raw[i].y, tmp);
                    if (!PACK) mma_f16(tml, a, b_raw[i].z, b_raw[i].w, tml);
                }
                acc[t][0] = fmaf(sc0[q], tmp[0], acc[t][0]);
                acc[t][1] = fmaf(sc0[q], tmp[1], acc[t][1]);
                acc[t][2] = fmaf(sc1[q], tmp[2], acc[t][2]);
                acc[t][3] = fmaf(sc1[q], tmp[3], acc[t][3]);
                if (!PACK) {
                    accl[t][0] = fmaf(sc0[q], tml[0], accl[t][0]);
                    accl[t][1] = fmaf(sc0[q], tml[1], accl[t][1]);
                    accl[t][2] = fmaf(sc1[q], tml[2], accl[t][2]);
                    accl[t][3] = fmaf(sc1[q], tml[3], accl[t][3]);
                }
            }
        }
    } else {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const uint8_t *blk = blks[t];
        if (!blk) continue;
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
                float f4[4];
                e8m0x4_to_float(*reinterpret_cast<const uint32_t *>(sp), f4);
#pragma unroll
                for (int q = 0; q < kGroups; ++q) scale[h][q] = f4[q];
            }
        }
        uint32_t regs[2][16];  // per row h: fp16x2 registers (index q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t words[4] = {a_raw[h].x, a_raw[h].y, a_raw[h].z, a_raw[h].w};
            if (FMT == FC_FMT_Q8) {
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) dequant_q8_word(words[wi], regs[h][2 * wi], regs[h][2 * wi + 1]);
            } else if (FMT == FC_FMT_Q4) {
#pragma unroll
                for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                    for (int sh = 0; sh < 4; ++sh) regs[h][4 * wi + sh] = dequant_q4_pair(words[wi], 4 * sh);
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
            float tml[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) {
                int i = 2 * q + ii;
                // a0 = row g (k slots 2j,2j+1), a1 = row g+8,
                // a2 = row g (slots 2j+8, 2j+9), a3 = row g+8.
                uint32_t a[4] = {regs[0][2 * i], regs[1][2 * i], regs[0][2 * i + 1], regs[1][2 * i + 1]};
                mma_f16(tmp, a, b_raw[i].x, b_raw[i].y, tmp);
                if (!PACK) mma_f16(tml, a, b_raw[i].z, b_raw[i].w, tml);
            }
            acc[t][0] = fmaf(scale[0][q], tmp[0], acc[t][0]);
            acc[t][1] = fmaf(scale[0][q], tmp[1], acc[t][1]);
            acc[t][2] = fmaf(scale[1][q], tmp[2], acc[t][2]);
            acc[t][3] = fmaf(scale[1][q], tmp[3], acc[t][3]);
            if (!PACK) {
                accl[t][0] = fmaf(scale[0][q], tml[0], accl[t][0]);
                accl[t][1] = fmaf(scale[0][q], tml[1], accl[t][1]);
                accl[t][2] = fmaf(scale[1][q], tml[2], accl[t][2]);
                accl[t][3] = fmaf(scale[1][q], tml[3], accl[t][3]);
            }
        }
    }
    }
}

#ifdef FC_GEMV_TRACE
__device__ unsigned long long g_gemv_trace[512];
__device__ int g_gemv_trace_items;
static int g_host_trace_items = -1;
#define GEMV_MARK(i)                                                                                  \
    do {                                                                                              \
        if (wk.trace && blockIdx.x == 0 && (i) < 512) g_gemv_trace[(i)] = clock64(); \
    } while (0)
#else
#define GEMV_MARK(i) \
    do {             \
    } while (0)
#endif

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;\n" ::"n"(kGemvConsumers) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// Applies the epilogue of segment `sg` to the finished tile `out` [32][8].
__device__ __forceinline__ void gemv_epilogue(const GemvSeg &sg, const GemvItem &it, int S,
                                              float limit, const float *out) {
    int idx = threadIdx.x;  // consumer threads 0 .. 255
    if (sg.epi == EPI_SWIGLU_XQ) {
        if (idx >= 128) return;
        int r = idx >> 3, s = idx & 7;
        int o = it.row0 + r;
        if (s >= S || o >= sg.O) return;
        float gv = out[r * 8 + s], uv = out[(16 + r) * 8 + s];
        if (limit > 0.0f) {  // moe_exec.h:55-60
            gv = fminf(gv, limit);
            uv = fminf(fmaxf(uv, -limit), limit);
        }
        store_xq(sg.yq + it.out_shift, sg.kpy, s, sg.col_off + it.member * sg.out_stride + o,
                 silu(gv) * uv);
        return;
    }
    // plain outputs: consecutive threads take consecutive rows of one
    // activation row (coalesced, also for the stores into peer GPUs)
    const bool plain = sg.epi == EPI_STORE || sg.epi == EPI_ADD;
    int r = plain ? (idx & 31) : (idx >> 3), s = plain ? (idx >> 5) : (idx & 7);
    int o = it.row0 + r;
    if (s >= S || o >= sg.O) return;
    float v = out[r * 8 + s];
    int col = it.member * sg.out_stride + o;
    if (sg.epi == EPI_STORE) {
        const size_t at = it.out_shift + (size_t)s * sg.ldy + col;
        sg.y[at] = v;
        for (int p = 0; p < sg.npeer; ++p) sg.peer_y[p][at] = v;  // NVLink stores
    } else if (sg.epi == EPI_ADD) {
        sg.y[it.out_shift + (size_t)s * sg.ldy + col] += v;
    } else {
        store_xq(sg.yq + it.out_shift, sg.kpy, s, sg.col_off + col, v);
        // xq copies into peer GPUs' buffers (head-parallel attention: each
        // rank's W_UV heads into every rank's o_proj input); NVLink stores
        for (int p = 0; p < sg.npeer; ++p)
            store_xq(reinterpret_cast<__half *>(sg.peer_y[p]) + it.out_shift, sg.kpy, s, sg.col_off + col, v);
    }
}

// Sums the consumer warps' fragments (fixed warp order) into out8 [32][8].
__device__ __forceinline__ void reduce_warps(float *red, const float (&acc)[2][4], float *out8) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[((warp * 2 + t) * 32 + lane) * 4 + e] = acc[t][e];
    consumer_sync();
    int t = tid >> 7, l = (tid >> 2) & 31, e = tid & 3;
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) sum += red[((w * 2 + t) * 32 + l) * 4 + e];
    int row = 16 * t + (l >> 2) + 8 * (e >> 1);
    int col = 2 * (l & 3) + (e & 1);
    out8[row * 8 + col] = sum;
    consumer_sync();
}

// The consumer warps of gemv_kernel: per work item, wait for each stage,
// multiply its chunk blocks, reduce, and run the epilogue.
template <int FA, int FB, bool PACK>
__device__ __forceinline__ void gemv_consume(const GemvWork &wk, const uint8_t *smem, size_t kSlotW,
                                             size_t kSlotBytes, uint64_t *full, uint64_t *empty, float *red,
                                             float *out) {
    constexpr bool kSmemB = gemv_smem_b(FA, FB);
    constexpr int kBRow = gemv_b_row_bytes(FA, FB);
    const int stages = kSmemB ? wk.stages : kStages;  // compile-time ring for the global-B kernels
    __shared__ float out_hi[kGemvRows * 8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, j = lane & 3;
    // PACK: lane group g reads activation row g & 3, hi half (g < 4) or lo half
    const int brow = PACK ? (g & 3) : g;
    const int bhalf = PACK ? (g >> 2) * 8 : 0;
    const bool has_b = brow < wk.S;
    int idx = 0, slot = 0;
    uint32_t phase = 0;  // parity of the ring pass `slot` is in
    bool waited = !(wk.moe && wk.shared_first);
    for (int item = blockIdx.x; item < wk.total_items; item += gridDim.x) {
        if (!waited && item >= wk.seg[1].tiles) {
            pdl_wait();
            waited = true;
        }
        GemvItem it;
        if (!resolve_item<FA, FB>(wk, item, it)) continue;
        const bool fa = it.fmt == FA;
        const int blk = fa ? block_bytes(FA) : block_bytes(FB);
        const int kmmas = it.fmt == FC_FMT_Q8 ? 4 : 8;
        const int nchunks = chunk_count(it.fmt, it.kp);
        const int nst = (nchunks + kGemvWarps - 1) / kGemvWarps;
        float acc[2][4], accl[2][4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[t][e] = accl[t][e] = 0.0f;
        // activation fragments of chunk c (zeros past the end / unused rows)
        auto load_b = [&](int c, uint4 (&b)[8]) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const bool live = has_b && c < nchunks && i < kmmas;
                const __half *src = it.xq + ((size_t)brow * it.kp + 16 * (kmmas * c + i) + 4 * j) * 2;
                if (PACK) {
                    uint2 v = live ? ldg_v2(reinterpret_cast<const uint8_t *>(src) + bhalf) : make_uint2(0, 0);
                    b[i] = make_uint4(v.x, v.y, 0, 0);
                } else {
                    b[i] = live ? ldg_v4(src) : make_uint4(0, 0, 0, 0);
                }
            }
        };
        // (global B) PACK: the next stage's fragments load while this stage computes
        uint4 b_next[8];
        if (!kSmemB && PACK) load_b(warp, b_next);
        for (int s = 0; s < nst; ++s, ++idx) {
            const int c = s * kGemvWarps + warp;
            const uint8_t *sb = smem + (size_t)slot * kSlotBytes;
            uint4 b_raw[8];
            if (!kSmemB) {
                if (PACK) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) b_raw[i] = b_next[i];
                    if (s + 1 < nst) load_b(c + kGemvWarps, b_next);
                } else {
                    load_b(c, b_raw);
                }
            }
            if (warp == 0 && lane == 0) GEMV_MARK(128 + idx);
            mbar_wait_bounded(&full[slot], phase, wk.err);
            if (warp == 0 && lane == 0) GEMV_MARK(256 + idx);
            if (kSmemB) {
                // this stage's activation rows, copied by the producer
                const uint8_t *brow_p = sb + 2 * kSlotW + (size_t)brow * kBRow + warp * kmmas * 64 + 16 * j;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const bool live = has_b && c < nchunks && i < kmmas;
                    if (PACK) {
                        uint2 v = live ? *reinterpret_cast<const uint2 *>(brow_p + i * 64 + bhalf) : make_uint2(0, 0);
                        b_raw[i] = make_uint4(v.x, v.y, 0, 0);
                    } else {
                        b_raw[i] = live ? *reinterpret_cast<const uint4 *>(brow_p + i * 64) : make_uint4(0, 0, 0, 0);
                    }
                }
            }
            if (c < nchunks) {
                const uint8_t *b0 = sb + (size_t)warp * blk;
                const uint8_t *b1 = it.t1 ? sb + kSlotW + (size_t)warp * blk : nullptr;
                if (fa) gemv_chunk<FA, PACK>(b0, b1, b_raw, acc, accl);
                else gemv_chunk<FB, PACK>(b0, b1, b_raw, acc, accl);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (warp == 0 && lane == 0) GEMV_MARK(384 + idx);
            if (++slot == stages) {
                slot = 0;
                phase ^= 1u;
            }
        }
        // out[row][s] = (hi sum over warps) + (lo sum over warps), the same
        // arithmetic for both forms
        if (PACK) {
            reduce_warps(red, acc, out_hi);
            out[tid] = (tid & 7) < 4 ? out_hi[tid] + out_hi[tid + 4] : 0.0f;
        } else {
            reduce_warps(red, acc, out_hi);
            reduce_warps(red, accl, out);
            out[tid] = out_hi[tid] + out[tid];
        }
        consumer_sync();
        gemv_epilogue(wk.seg[it.seg], it, wk.S, wk.swiglu_limit, out);
        if (tid == 0) GEMV_MARK(127);
    }
    if (wk.seg[0].npeer) {
        // all of this CTA's peer stores before the epoch flag (one
        // cumulative system fence after a CTA barrier)
        consumer_sync();
        if (tid == 0) __threadfence_system();
    }
    if (wk.pub_done && tid == 0) {
        // the last CTA publishes the next epoch to every peer
        if (atomicAdd(wk.pub_done, 1) == (int)gridDim.x - 1) {
            *wk.pub_done = 0;
            __threadfence_system();
            const int e = *wk.pub_epoch + 1;
            *wk.pub_epoch = e;
            for (int r = 0; r < wk.peer_world; ++r)
                if (r != wk.peer_rank)
                    asm volatile("st.release.sys.global.s32 [%0], %1;\n" ::"l"(wk.pub_flags[r] + wk.peer_rank), "r"(e) : "memory");
        }
    }
}

template <int FA, int FB>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const __grid_constant__ GemvWork wk) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[kGemvWarps * 2 * 32 * 4];
    __shared__ float out[kGemvRows * 8];
    constexpr size_t kSlotW = gemv_slot_w(FA, FB);
    constexpr bool kSmemB = gemv_smem_b(FA, FB);
    constexpr int kBRow = gemv_b_row_bytes(FA, FB);
    const int stages = kSmemB ? wk.stages : kStages;  // compile-time ring for the global-B kernels
    const size_t kSlotBytes = 2 * kSlotW + (kSmemB ? (size_t)wk.S * kBRow : 0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + stages * kSlotBytes);
    uint64_t *empty = full + kStages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_release();

    if (tid == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kGemvWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kGemvWarps) {
        // ---------------- producer ----------------
        if (lane != 0) return;
        // Weights are constant during a forward, so the producer streams the
        // first ring of weights before the predecessor finishes; the
        // activation rows (kSmemB) and the MoE work list (written by the
        // router kernel) need the wait.
        bool waited = false;
        if (wk.moe && !wk.shared_first) {
            pdl_wait();
            waited = true;
        }
        // activation copies of stages issued before the wait
        struct BJob {
            int slot;
            const __half *xq;
            int kp, col0, cols;
        } pend[kStages];
        int npend = 0;
        int idx = 0, slot = 0;
        uint32_t phase = 0;    // parity of the ring pass `slot` is in
        bool reuse = false;    // slot already used once (wait for its release)
        for (int item = blockIdx.x; item < wk.total_items; item += gridDim.x) {
            if (wk.moe && !waited && item >= wk.seg[1].tiles) {
                pdl_wait();  // the routed items need the router's work list
                waited = true;
            }
            GemvItem it;
            if (!resolve_item<FA, FB>(wk, item, it)) continue;
            const int blk = it.fmt == FA ? block_bytes(FA) : block_bytes(FB);
            const int ccols = chunk_cols(it.fmt);
            const int nchunks = chunk_count(it.fmt, it.kp);
            const int nst = (nchunks + kGemvWarps - 1) / kGemvWarps;
            for (int s = 0; s < nst; ++s, ++idx) {
                if (kSmemB && !waited && reuse) {
                    // the ring is full: wait for the predecessor, then send
                    // the activation rows of the stages already in flight
                    pdl_wait();
                    gemv_peer_wait(wk);
                    waited = true;
                    for (int p = 0; p < npend; ++p)
                        for (int r = 0; r < wk.S; ++r)
                            bulk_g2s(smem + (size_t)pend[p].slot * kSlotBytes + 2 * kSlotW + (size_t)r * kBRow,
                                     pend[p].xq + ((size_t)r * pend[p].kp + pend[p].col0) * 2,
                                     (uint32_t)(pend[p].cols * 4), &full[pend[p].slot]);
                    npend = 0;
                }
                if (reuse) mbar_wait_bounded(&empty[slot], phase ^ 1u, wk.err);
                GEMV_MARK(idx);
                const int c0 = s * kGemvWarps;
                const int nch = min(kGemvWarps, nchunks - c0);
                const uint32_t bytes = (uint32_t)(nch * blk);
                const uint32_t bbytes = kSmemB ? (uint32_t)(wk.S * nch * ccols * 4) : 0u;
                mbar_expect_tx(&full[slot], bytes * (it.t1 ? 2u : 1u) + bbytes);
                uint8_t *sb = smem + (size_t)slot * kSlotBytes;
                bulk_g2s(sb, it.t0 + (size_t)c0 * blk, bytes, &full[slot]);
                if (it.t1) bulk_g2s(sb + kSlotW, it.t1 + (size_t)c0 * blk, bytes, &full[slot]);
                if (kSmemB) {
                    if (waited || wk.moe) {  // MoE: shared-first items read an input that is ready
                        for (int r = 0; r < wk.S; ++r)
                            bulk_g2s(sb + 2 * kSlotW + (size_t)r * kBRow, it.xq + ((size_t)r * it.kp + c0 * ccols) * 2,
                                     (uint32_t)(nch * ccols * 4), &full[slot]);
                    } else {
                        pend[npend++] = BJob{slot, it.xq, it.kp, c0 * ccols, nch * ccols};
                    }
                }
                if (++slot == stages) {
                    slot = 0;
                    phase ^= 1u;
                    reuse = true;
                }
            }
        }
        if (kSmemB && !waited) {
            pdl_wait();
            gemv_peer_wait(wk);
            for (int p = 0; p < npend; ++p)
                for (int r = 0; r < wk.S; ++r)
                    bulk_g2s(smem + (size_t)pend[p].slot * kSlotBytes + 2 * kSlotW + (size_t)r * kBRow,
                             pend[p].xq + ((size_t)r * pend[p].kp + pend[p].col0) * 2,
                             (uint32_t)(pend[p].cols * 4), &full[pend[p].slot]);
        }
        return;
    }

    // ---------------- consumers ----------------
    if (tid == 0) GEMV_MARK(125);
    if (!(wk.moe && wk.shared_first)) pdl_wait();
    if (tid == 0) GEMV_MARK(126);
    if (wk.S <= 4)
        gemv_consume<FA, FB, true>(wk, smem, kSlotW, kSlotBytes, full, empty, red, out);
    else
        gemv_consume<FA, FB, false>(wk, smem, kSlotW, kSlotBytes, full, empty, red, out);
}

inline int gemv_tiles(const GemvSeg &s) {
    int ntiles = (s.O + kTileRows - 1) / kTileRows;
    return s.epi == EPI_SWIGLU_XQ ? ntiles : (ntiles + 1) / 2;
}

#define FC_GEMV_FORMATS(X)         \
    X(FC_FMT_Q8, FC_FMT_Q8)        \
    X(FC_FMT_Q4, FC_FMT_Q4)        \
    X(FC_FMT_MXFP4, FC_FMT_MXFP4)  \
    X(FC_FMT_MXFP4, FC_FMT_Q8)     \
    X(FC_FMT_Q4, FC_FMT_Q8)        \
    X(FC_FMT_Q8, FC_FMT_Q4)

// Opts the GEMV kernels into their dynamic shared memory (once per device,
// before launching or capturing).
inline cudaError_t gemv_prepare_all() {
    cudaError_t e = cudaSuccess;
#define FC_GEMV_ATTR(A, B)                                                                    \
    if (e == cudaSuccess)                                                                     \
        e = cudaFuncSetAttribute(gemv_kernel<A, B>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 (int)gemv_smem_max(A, B));
    FC_GEMV_FORMATS(FC_GEMV_ATTR)
#undef FC_GEMV_ATTR
    return e;
}

constexpr int kGemvCtasPerSm = 2;

inline cudaError_t launch_gemv_work(int fa, int fb, GemvWork &wk, int sms, cudaStream_t stream) {
    int items = 0;
    if (wk.moe) {
        wk.seg[0].tiles = gemv_tiles(wk.seg[0]);
        wk.seg[1].tiles = wk.seg[1].w ? gemv_tiles(wk.seg[1]) : 0;
        items = wk.max_slots * wk.seg[0].tiles + wk.seg[1].tiles;
    } else {
        for (int i = 0; i < wk.nseg; ++i) {
            if (wk.seg[i].count <= 0) wk.seg[i].count = 1;
            wk.seg[i].tiles = gemv_tiles(wk.seg[i]);
            items += wk.seg[i].tiles * wk.seg[i].count;
        }
    }
    wk.total_items = items;
    wk.stages = gemv_stages(fa, fb, wk.S);
#ifdef FC_GEMV_TRACE
    wk.trace = g_host_trace_items == items;
#endif
    if (items == 0) return cudaSuccess;
    int grid = std::min(items, sms * kGemvCtasPerSm);
#define FC_GEMV_CASE(A, B)                                                               \
    if (fa == A && fb == B) {                                                            \
        return launch_pdl(gemv_kernel<A, B>, dim3(grid), dim3(kGemvThreads),               \
                          gemv_smem_bytes(A, B, wk.S), stream, wk);                        \
    }
    FC_GEMV_FORMATS(FC_GEMV_CASE)
#undef FC_GEMV_CASE
    return cudaErrorInvalidValue;
}

// Batch of static segments sharing one format.
struct GemvBatch {
    GemvSeg seg[kMaxSegs];
    int nseg;
    int S;
    float swiglu_limit;
    int *err;
    const GemvWork *sync;  // nullable: the cross-GPU hand-off fields (pub_*, wait_*, peer_*)
};

inline cudaError_t launch_gemv_batch(int fmt, GemvBatch &b, int sms, cudaStream_t stream) {
    GemvWork wk{};
    for (int i = 0; i < b.nseg; ++i) wk.seg[i] = b.seg[i];
    wk.nseg = b.nseg;
    wk.S = b.S;
    wk.swiglu_limit = b.swiglu_limit;
    wk.err = b.err;
    if (b.sync) {
        wk.pub_done = b.sync->pub_done;
        wk.pub_epoch = b.sync->pub_epoch;
        for (int r = 0; r < 8; ++r) wk.pub_flags[r] = b.sync->pub_flags[r];
        wk.wait_flags = b.sync->wait_flags;
        wk.wait_epoch = b.sync->wait_epoch;
        wk.wait_ns = b.sync->wait_ns;
        wk.peer_world = b.sync->peer_world;
        wk.peer_rank = b.sync->peer_rank;
    }
    return launch_gemv_work(fmt, fmt, wk, sms, stream);
}

// ---------------------------------------------------------------------------
// fp32-weight GEMV (an unquantized embedding-sized matrix, e.g. the fp32
// lm-head of floyd's Moonlight container; moonlight_matmul_f32 in
// moonlight_kernels.metal): y[s][o] = sum_k x[s][k] * w[o][k], w row-major
// [O][K].  HBM-bound: one warp per output row streams the row with 16-byte
// loads (the same rows for every activation row, so each weight byte is read
// once per launch), the activations (decoded from the xq hi / lo halves) sit
// in shared memory.  Each lane sums its columns in ascending k and the warp
// reduces in a fixed butterfly, so a row's result does not depend on S.
// ---------------------------------------------------------------------------
constexpr int kF32GemvThreads = 256;
constexpr int kF32MaxRows = 8;  // activation rows per launch

__global__ void __launch_bounds__(kF32GemvThreads) f32_gemv_kernel(const float *w, int O, int K,
                                                                    const __half *xq, int kp, int S,
                                                                    float *y, int ldy) {
    extern __shared__ float xs[];  // [S][K]
    pdl_wait();
    pdl_release();
    for (int i = threadIdx.x; i < S * K; i += blockDim.x) {
        const int s = i / K, k = i - s * K;
        const __half *rec = xq + ((size_t)s * kp + (k & ~3)) * 2;
        xs[i] = __half2float(rec[k & 3]) + __half2float(rec[4 + (k & 3)]);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int o = blockIdx.x * warps + (threadIdx.x >> 5); o < O; o += gridDim.x * warps) {
        const float4 *row = reinterpret_cast<const float4 *>(w + (size_t)o * K);
        float acc[kF32MaxRows];
#pragma unroll
        for (int s = 0; s < kF32MaxRows; ++s) acc[s] = 0.0f;
        for (int k4 = lane; k4 < K / 4; k4 += 32) {
            const float4 v = __ldcs(row + k4);
#pragma unroll
            for (int s = 0; s < kF32MaxRows; ++s) {
                if (s >= S) break;
                const float4 x = *reinterpret_cast<const float4 *>(xs + (size_t)s * K + 4 * k4);
                acc[s] = fmaf(v.x, x.x, acc[s]);
                acc[s] = fmaf(v.y, x.y, acc[s]);
                acc[s] = fmaf(v.z, x.z, acc[s]);
                acc[s] = fmaf(v.w, x.w, acc[s]);
            }
        }
#pragma unroll
        for (int s = 0; s < kF32MaxRows; ++s) {
            if (s >= S) break;
            float v = acc[s];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) y[(size_t)s * ldy + o] = v;
        }
    }
}

inline cudaError_t launch_f32_gemv(const float *w, int O, int K, const __half *xq, int kp, int S,
                                   float *y, int ldy, int sms, cudaStream_t stream) {
    const size_t smem = (size_t)S * K * 4;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(f32_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int warps = kF32GemvThreads / 32;
    const int grid = std::min((O + warps - 1) / warps, sms * 4);
    return launch_pdl(f32_gemv_kernel, dim3(grid), dim3(kF32GemvThreads), smem, stream, w, O, K, xq,
                      kp, S, y, ldy);
}

}  // namespace fc
