// prefill.cuh - the prefill / append path for chunks of many tokens
// (moonlight_session_prefill, moonlight_metal.m:1988-2005): every linear
// layer is a GEMM on the 5th-generation tensor cores with the quantized
// weights dequantized in shared memory, plus the row-parallel kernels around
// them (norms, KV append + rope, router, expert grouping, combine).
//
// pf_gemm_kernel: Y[m][n] = sum_k A[m][k] * W[n][k] for M = the chunk's
// tokens (or an expert's rows), W a tile-major q8 / q4 / mxfp4 matrix
// (common.cuh).  Persistent: one CTA per SM walks (m-tile, n-tile) items.
//   warps 0-3   epilogue: thread = output row = TMEM lane; reads the fp32
//               accumulator with tcgen05.ld and stores fp32 / fp16 / adds /
//               SwiGLU (moe_exec.h:55-60 clamp);
//   warp 4      producer: TMA of the fp16 A tile (128 rows x 64 columns,
//               128-byte swizzle) and bulk copies of the quantized weight
//               blocks of the n-tile;
//   warp 5      MMA issuer (one thread): tcgen05.mma kind::f16, M = 128,
//               N = BN, K = 16 steps; TMEM holds two BN-column accumulators
//               so the epilogue of one item overlaps the MMAs of the next;
//   warps 6-13  dequant: quantized block -> fp16 (value x group scale,
//               rounded once) written straight into the 128-byte-swizzled
//               K-major B tile.
// Rings: A 6 x 16 KB, dequantized B 2 x BN x 128 B, raw weights 2 x 18 KB.
// Every wait is bounded (~0.2 s); a timeout sets an error bit and makes
// every later wait of the CTA give up at once.
#pragma once

#include "mla.cuh"
#include "mla_tc.cuh"
#include "moe.cuh"

namespace fc {

constexpr int kPfThreads = 448;
constexpr int kPfWarpProducer = 4, kPfWarpMma = 5, kPfWarpDq0 = 6, kPfDqThreads = 256;
constexpr int kPfM = 128, kPfK = 64;
// m-tiles per work item: each dequantized weight tile feeds the MMAs of two
// 128-row m-tiles, so the dequant work per MMA is half of one m-tile's
constexpr int kPfMP = 2, kPfMI = kPfM * kPfMP;
constexpr int kPfBN = 128;  // weight rows (MMA N) per n-tile
constexpr int kPfSA = 4, kPfSD = 3, kPfSQ = 2;
constexpr int kPfRawBytes = 16 * 1152;

enum PfEpi : int { PF_STORE_F32 = 0, PF_STORE_F16 = 1, PF_ADD_F32 = 2, PF_SWIGLU_F16 = 3 };

struct PfGemm {
    int tiles_per_group;     // 16-row weight tiles from one group's matrix to the next
    int box_tiles;           // tiles per weight-map box (BN / 16, BN / 32 for SwiGLU, fewer for tiny matrices)
    int kp;                  // padded width of the stored matrix
    int N, K;                // outputs per group (multiple of 32); reduction length (multiple of 64)
    int groups, rows;        // arithmetic m-tiles: groups x ceil(rows / 128)
    int a_gx, a_gy;          // A coordinates of group g start at (g * a_gx, a_y0 + g * a_gy)
    int a_y0;
    const int *mt_count;     // table m-tiles (expert groups), nullable
    const int4 *mt_table;    // {group, first A row, end row, 0}
    void *out;
    int64_t out_ld, out_gstride;  // elements
    float limit;             // SwiGLU clamp (0 = none)
    int *err;
};

template <int BN>
struct PfPlan {
    static constexpr int A_BYTES = kPfMP * kPfM * 128;  // both m-tiles of a k-step
    static constexpr int D_BYTES = BN * 128;
    static constexpr int OFF_D = kPfSA * A_BYTES;
    static constexpr int OFF_Q = OFF_D + kPfSD * D_BYTES;
    static constexpr int OFF_BAR = OFF_Q + kPfSQ * kPfRawBytes;
    static constexpr size_t SMEM = (size_t)OFF_BAR + 256 + 1024;  // + base alignment
    static constexpr uint32_t TMEM_COLS = 2 * kPfMP * BN;  // (double buffer) x (m-tile)
    static_assert(SMEM <= 232448, "shared memory plan");
};

struct PfTile {
    int g, a_x, a_y, out_row0, nvalid;  // nvalid: rows of the item (m-tile mp has nvalid - 128 mp)
};

__device__ __forceinline__ PfTile pf_tile(const PfGemm &p, int mi, int mpg) {
    PfTile t;
    if (p.mt_table) {
        int4 e = p.mt_table[mi];
        t.g = e.x;
        t.a_x = e.x * p.a_gx;
        t.a_y = e.y;
        t.out_row0 = e.y;
        t.nvalid = min(kPfMI, e.z - e.y);
    } else {
        t.g = mi / mpg;
        const int m0 = (mi % mpg) * kPfMI;
        t.a_x = t.g * p.a_gx;
        t.a_y = p.a_y0 + t.g * p.a_gy + m0;
        t.out_row0 = m0;
        t.nvalid = min(kPfMI, p.rows - m0);
    }
    return t;
}

// Bounded wait (~20 ms) used on the way out: the copies and MMAs a CTA
// issued must finish before it exits, even after an abort.
__device__ __forceinline__ void pf_drain(uint64_t *bar, uint32_t parity) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return;
        if ((it & 255u) == 0) {
            const uint64_t t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > 20000000ull) return;
        }
    }
}

__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, int *err, volatile int *abort, int site) {
    if (*abort) return false;
    if (mbar_wait_timed(bar, parity, err, site)) return true;
    *abort = 1;
    return false;
}

// 16 values of one row of a quantized block: columns 16 i + 4 j + b
// (i < 4, b < 4) of the 64-column half `sub` of the chunk, as fp16 pairs
// o[2 i + b / 2] = (b even, b odd), each value x its group scale rounded
// once.  `v` is the row's 16-byte record j of the chunk, `sc` the row's
// group scales of the chunk (q8: 2 x fp16, q4: 4 x fp16, mxfp4: 4 x ue8m0).
template <int FMT>
__device__ __forceinline__ void pf_dequant_rec(uint4 v, uint2 sc, int sub, uint32_t (&o)[8]) {
    if (FMT == FC_FMT_Q8) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        const __half2 s0 = __half2half2(__ushort_as_half((unsigned short)(sc.x & 0xFFFFu)));
        const __half2 s1 = __half2half2(__ushort_as_half((unsigned short)(sc.x >> 16)));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t lo, hi;
            dequant_q8_word(w[i], lo, hi);
            const __half2 s = i < 2 ? s0 : s1;
            __half2 a = __hmul2(*reinterpret_cast<__half2 *>(&lo), s);
            __half2 b = __hmul2(*reinterpret_cast<__half2 *>(&hi), s);
            o[2 * i] = *reinterpret_cast<uint32_t *>(&a);
            o[2 * i + 1] = *reinterpret_cast<uint32_t *>(&b);
        }
    } else if (FMT == FC_FMT_Q4) {
        const uint32_t w0 = sub ? v.z : v.x, w1 = sub ? v.w : v.y, s2 = sub ? sc.y : sc.x;
        const __half2 s0 = __half2half2(__ushort_as_half((unsigned short)(s2 & 0xFFFFu)));
        const __half2 s1 = __half2half2(__ushort_as_half((unsigned short)(s2 >> 16)));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t word = i < 2 ? w0 : w1;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t pr = dequant_q4_pair(word, 4 * (2 * (i & 1) + h));
                __half2 a = __hmul2(*reinterpret_cast<__half2 *>(&pr), i < 2 ? s0 : s1);
                o[2 * i + h] = *reinterpret_cast<uint32_t *>(&a);
            }
        }
    } else {
        uint32_t c0[4], c1[4];
        dequant_e2m1_word(sub ? v.z : v.x, c0);
        dequant_e2m1_word(sub ? v.w : v.y, c1);
        const uint32_t sb = sc.x >> (16 * sub), e0 = sb & 0xFFu, e1 = (sb >> 8) & 0xFFu;
        if (e0 - 113u <= 29u && e1 - 113u <= 29u) {
            // 2^(e - 127) is a normal fp16: scaling an e2m1 value by it in
            // fp16 is exact (subnormal results included) or overflows alike
            const __half2 s0 = __half2half2(__ushort_as_half((unsigned short)((e0 - 112u) << 10)));
            const __half2 s1 = __half2half2(__ushort_as_half((unsigned short)((e1 - 112u) << 10)));
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                uint32_t cq = q < 4 ? c0[q] : c1[q - 4];
                __half2 r = __hmul2(*reinterpret_cast<__half2 *>(&cq), q < 4 ? s0 : s1);
                o[q] = *reinterpret_cast<uint32_t *>(&r);
            }
            return;
        }
        const float f0 = e8m0_to_float(e0), f1 = e8m0_to_float(e1);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float f = q < 4 ? f0 : f1;
            const uint32_t cq = q < 4 ? c0[q] : c1[q - 4];
            float2 x = __half22float2(*reinterpret_cast<const __half2 *>(&cq));
            __half2 r = __floats2half2_rn(x.x * f, x.y * f);
            o[q] = *reinterpret_cast<uint32_t *>(&r);
        }
    }
}

// Row and 16-byte record of dequant unit u (64 units per 16-row block):
// a quarter-warp's eight 16-byte record loads cover 128 distinct bytes
// modulo 128 and a half-warp's 8-byte tile stores (fixed i) 128 distinct
// bytes of the swizzled tile, so neither conflicts.
__device__ __forceinline__ void pf_unit_pos(int u, int &rho, int &j) {
    const int lane = u & 31, hw = lane >> 4, q = (lane >> 3) & 1, w = lane & 7;
    j = w & 3;
    rho = 8 * ((u >> 5) & 1) + 2 * (2 * q + ((j >> 1) ^ hw)) + (w >> 2);
}

// Byte offset of element (n, k) in a K-major 128-byte-swizzled tile of
// 64 k-columns (rows n 128 B apart, 16-byte chunks xor-ed with n % 8).
__device__ __forceinline__ uint32_t sw128_kmajor(int n, int k) {
    return (uint32_t)(n * 128 + ((((k >> 3) ^ n) & 7) << 4) + (k & 7) * 2);
}
__device__ __forceinline__ float pf_swiglu(float g, float u, float limit) {
    if (limit > 0.0f) {
        g = fminf(g, limit);
        u = fminf(fmaxf(u, -limit), limit);
    }
    return silu(g) * u;
}

// grid = SM count, kPfThreads threads, PfPlan<BN>::SMEM bytes.
// wmap / wmap2: 4-D tensor maps of the weights (and, for SwiGLU, of the up
// rows) viewed as [16-row tiles][chunks][block_bytes / 64][64 bytes], box
// {64, block_bytes / 64, 1, BN / 16} (BN / 32 tiles each for SwiGLU): one
// request brings a stage's blocks in the raw ring's layout.
template <int FMT, int BN, int EPI>
__global__ void __launch_bounds__(kPfThreads, 1)
pf_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
               const __grid_constant__ CUtensorMap wmap2, const PfGemm p) {
    using P = PfPlan<BN>;
    constexpr int KC = FMT == FC_FMT_Q8 ? 64 : 128;  // columns per stored chunk
    constexpr int KPR = KC / 64;                     // k-steps per raw stage
    constexpr int BB = block_bytes(FMT);
    constexpr int BNO = EPI == PF_SWIGLU_F16 ? BN / 2 : BN;  // outputs per n-tile
    extern __shared__ uint8_t pf_smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = sm, *sD = sm + P::OFF_D, *sQ = sm + P::OFF_Q;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P::OFF_BAR);
    uint64_t *a_full = bars, *a_empty = bars + kPfSA, *d_full = bars + 2 * kPfSA,
             *d_empty = d_full + kPfSD, *q_full = d_empty + kPfSD, *q_empty = q_full + kPfSQ,
             *acc_full = q_empty + kPfSQ, *acc_empty = acc_full + 2, *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kPfSA; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kPfSD; ++i) {
            mbar_init(&d_full[i], kPfDqThreads / 32);
            mbar_init(&d_empty[i], 1);
        }
        for (int i = 0; i < kPfSQ; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], kPfDqThreads / 32);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        mbar_fence_init();
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
        if (EPI == PF_SWIGLU_F16)
            asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&wmap2)) : "memory");
    }
    if (warp == kPfWarpMma) {
        __syncwarp();
        tmem_alloc(tmem_slot, P::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_release();

    const int mpg = (p.rows + kPfMI - 1) / kPfMI;
    const int n_mt = p.mt_table ? *p.mt_count : p.groups * mpg;
    const int n_nt = (p.N + BNO - 1) / BNO;
    const int items = n_mt * n_nt;
    const int nk = p.K / kPfK;

    if (warp == kPfWarpProducer) {
        if (lane == 0) {
            uint32_t a_slot = 0, a_ph = 0, q_slot = 0, q_ph = 0;
            int a_fill = 0, q_fill = 0;
            for (int it = blockIdx.x; it < items && !*abort; it += gridDim.x) {
                const int mi = it / n_nt, nt = it % n_nt;
                const PfTile t = pf_tile(p, mi, mpg);
                for (int ks = 0; ks < nk && !*abort; ++ks) {
                    if (ks % KPR == 0) {
                        if (q_fill >= kPfSQ && !pf_wait(&q_empty[q_slot], q_ph ^ 1, p.err, abort, 0)) break;
                        uint8_t *dst = sQ + q_slot * kPfRawBytes;
                        // BN stored rows (BN / 16 tiles) x one chunk; rows past the
                        // matrix arrive as zeros and are never stored
                        const int c = ks * kPfK / KC;
                        const int tile0 = t.g * p.tiles_per_group + nt * BNO / 16;
                        mbar_expect_tx(&q_full[q_slot], (EPI == PF_SWIGLU_F16 ? 2 : 1) * p.box_tiles * BB);
                        if (EPI == PF_SWIGLU_F16) {
                            tma_load_4d(dst, &wmap, 0, 0, c, tile0, &q_full[q_slot]);
                            tma_load_4d(dst + (BN / 32) * BB, &wmap2, 0, 0, c, tile0, &q_full[q_slot]);
                        } else {
                            tma_load_4d(dst, &wmap, 0, 0, c, tile0, &q_full[q_slot]);
                        }
                        ++q_fill;
                        if (++q_slot == kPfSQ) { q_slot = 0; q_ph ^= 1; }
                    }
                    if (a_fill >= kPfSA && !pf_wait(&a_empty[a_slot], a_ph ^ 1, p.err, abort, 1)) break;
                    mbar_expect_tx(&a_full[a_slot], P::A_BYTES);
                    // both m-tiles (rows past the tensor arrive as zeros)
                    tma_load_2d(sA + a_slot * P::A_BYTES, &amap, t.a_x + ks * kPfK, t.a_y, &a_full[a_slot]);
                    tma_load_2d(sA + a_slot * P::A_BYTES + kPfM * 128, &amap, t.a_x + ks * kPfK, t.a_y + kPfM,
                                &a_full[a_slot]);
                    ++a_fill;
                    if (++a_slot == kPfSA) { a_slot = 0; a_ph ^= 1; }
                }
            }
            // before the CTA can exit, every copy this thread issued has
            // landed: wait (bounded) for the last fill of each ring slot
            for (int i = 0; i < kPfSA && i < a_fill; ++i) {
                const int f = a_fill - 1 - ((a_fill - 1 - i) % kPfSA);  // last fill of slot i
                pf_drain(&a_full[f % kPfSA], (uint32_t)((f / kPfSA) & 1));
            }
            for (int i = 0; i < kPfSQ && i < q_fill; ++i) {
                const int f = q_fill - 1 - ((q_fill - 1 - i) % kPfSQ);
                pf_drain(&q_full[f % kPfSQ], (uint32_t)((f / kPfSQ) & 1));
            }
        }
    } else if (warp == kPfWarpMma) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kPfM, BN, false);
            const uint32_t a0 = smem_u32(sA), d0 = smem_u32(sD);
            uint32_t a_slot = 0, a_ph = 0, d_slot = 0, d_ph = 0;
            int t = 0;
            for (int it = blockIdx.x; it < items && !*abort; it += gridDim.x, ++t) {
                const int b = t & 1;
                if (t >= 2) pf_wait(&acc_empty[b], ((t >> 1) - 1) & 1, p.err, abort, 2);
                tc_fence_after();
                const uint32_t tacc = tmem + b * kPfMP * BN;
                for (int ks = 0; ks < nk; ++ks) {
                    pf_wait(&a_full[a_slot], a_ph, p.err, abort, 3);
                    pf_wait(&d_full[d_slot], d_ph, p.err, abort, 4);
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t bd = smem_desc(d0 + d_slot * P::D_BYTES + kk * 32, 16, 1024, kSmemLayoutSw128);
#pragma unroll
                        for (int mp = 0; mp < kPfMP; ++mp) {
                            const uint64_t ad = smem_desc(a0 + a_slot * P::A_BYTES + mp * kPfM * 128 + kk * 32, 16,
                                                          1024, kSmemLayoutSw128);
                            tc_mma_f16(tacc + mp * BN, ad, bd, idesc, (ks | kk) != 0);
                        }
                    }
                    tc_commit(&a_empty[a_slot]);
                    tc_commit(&d_empty[d_slot]);
                    if (++a_slot == kPfSA) { a_slot = 0; a_ph ^= 1; }
                    if (++d_slot == kPfSD) { d_slot = 0; d_ph ^= 1; }
                }
                tc_commit(&acc_full[b]);
            }
            // every MMA this thread issued completes before TMEM is freed
            tc_commit(mma_done);
            pf_drain(mma_done, 0);
        }
    } else if (warp >= kPfWarpDq0) {
        constexpr int UPT = BN * 4 / kPfDqThreads;  // dequant units per thread
        const int dt = tid - kPfWarpDq0 * 32;
        // per-thread constants: the unit's block, record and scale offsets in
        // the raw stage, and its swizzled tile offset at i = 0 (the 16-column
        // group i only flips bits 5-6 of it: offset ^ (i << 5))
        int u_blk[UPT];
        uint32_t u_rec[UPT], u_scl[UPT], u_dst[UPT];
#pragma unroll
        for (int r = 0; r < UPT; ++r) {
            const int u = dt + r * kPfDqThreads;
            int rho, j;
            pf_unit_pos(u, rho, j);
            u_blk[r] = u >> 6;
            u_rec[r] = (u >> 6) * BB + rho * 64 + 16 * j;
            u_scl[r] = (u >> 6) * BB + kBlockValueBytes + rho * scale_row_bytes(FMT);
            u_dst[r] = sw128_kmajor((u >> 6) * 16 + rho, 4 * j);
        }
        uint4 recs[UPT];
        uint2 scs[UPT];
        uint32_t q_slot = 0, q_ph = 0, d_slot = 0, d_ph = 0;
        int d_fill = 0;
        for (int it = blockIdx.x; it < items && !*abort; it += gridDim.x) {
            const int nt = it % n_nt;
            uint32_t vmask = 0;  // units whose stored rows exist
#pragma unroll
            for (int r = 0; r < UPT; ++r) {
                const int blk = u_blk[r];
                const int o0 = EPI == PF_SWIGLU_F16 ? nt * BNO + (blk % (BN / 32)) * 16 : nt * BN + blk * 16;
                if (o0 < p.N) vmask |= 1u << r;
            }
            for (int ks = 0; ks < nk; ++ks) {
                if (ks % KPR == 0) pf_wait(&q_full[q_slot], q_ph, p.err, abort, 5);
                if (d_fill >= kPfSD) pf_wait(&d_empty[d_slot], d_ph ^ 1, p.err, abort, 6);
                const uint8_t *raw = sQ + q_slot * kPfRawBytes;
                uint8_t *dst = sD + d_slot * P::D_BYTES;
                const int sub = ks % KPR;
                if (vmask == (1u << UPT) - 1u) {
                    // every unit valid (all but a matrix's last n-tile): loads,
                    // decodes and stores of the units as independent chains
                    if (sub == 0) {
#pragma unroll
                        for (int r = 0; r < UPT; ++r) {
                            recs[r] = *reinterpret_cast<const uint4 *>(raw + u_rec[r]);
                            if (FMT == FC_FMT_Q4) scs[r] = *reinterpret_cast<const uint2 *>(raw + u_scl[r]);
                            else scs[r] = make_uint2(*reinterpret_cast<const uint32_t *>(raw + u_scl[r]), 0u);
                        }
                    }
                    uint32_t o[UPT][8];
#pragma unroll
                    for (int r = 0; r < UPT; ++r) pf_dequant_rec<FMT>(recs[r], scs[r], sub, o[r]);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
#pragma unroll
                        for (int r = 0; r < UPT; ++r)
                            *reinterpret_cast<uint2 *>(dst + (u_dst[r] ^ (uint32_t)(i << 5))) =
                                make_uint2(o[r][2 * i], o[r][2 * i + 1]);
                } else
#pragma unroll
                for (int r = 0; r < UPT; ++r) {
                    if (!((vmask >> r) & 1u)) continue;
                    if (sub == 0) {  // the record and scales serve every 64-column half of the chunk
                        recs[r] = *reinterpret_cast<const uint4 *>(raw + u_rec[r]);
                        if (FMT == FC_FMT_Q4) scs[r] = *reinterpret_cast<const uint2 *>(raw + u_scl[r]);
                        else scs[r] = make_uint2(*reinterpret_cast<const uint32_t *>(raw + u_scl[r]), 0u);
                    }
                    uint32_t o[8];
                    pf_dequant_rec<FMT>(recs[r], scs[r], sub, o);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        *reinterpret_cast<uint2 *>(dst + (u_dst[r] ^ (uint32_t)(i << 5))) = make_uint2(o[2 * i], o[2 * i + 1]);
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive_cta(&d_full[d_slot]);
                ++d_fill;
                if (++d_slot == kPfSD) { d_slot = 0; d_ph ^= 1; }
                if (ks % KPR == KPR - 1 || ks == nk - 1) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cta(&q_empty[q_slot]);
                    if (++q_slot == kPfSQ) { q_slot = 0; q_ph ^= 1; }
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 0-3) ----------------
        const int row = 32 * warp + lane;
        const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
        int t = 0;
        for (int it = blockIdx.x; it < items && !*abort; it += gridDim.x, ++t) {
            const int mi = it / n_nt, nt = it % n_nt;
            const PfTile tl = pf_tile(p, mi, mpg);
            const int b = t & 1;
            pf_wait(&acc_full[b], (t >> 1) & 1, p.err, abort, 7);
            __syncwarp();
            tc_fence_after();
#pragma unroll 1
            for (int mp = 0; mp < kPfMP; ++mp) {
            const uint32_t tacc = tmem + (b * kPfMP + mp) * BN + lane_off;
            const bool ok = mp * kPfM + row < tl.nvalid;
            const int64_t orow = (int64_t)(tl.out_row0 + mp * kPfM + row) * p.out_ld + (int64_t)tl.g * p.out_gstride;
            if (EPI == PF_SWIGLU_F16) {
                __half *out = reinterpret_cast<__half *>(p.out) + orow;
#pragma unroll 1
                for (int c0 = 0; c0 < BNO; c0 += 32) {
                    const int n = nt * BNO + c0;
                    if (n >= p.N) break;
                    float g[32], u[32];
                    tmem_ld32(tacc + c0, g);
                    tmem_ld32(tacc + BNO + c0, u);
                    tmem_wait_ld();
                    if (ok) {
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            uint4 v;
                            __half2 h0 = __floats2half2_rn(pf_swiglu(g[c], u[c], p.limit), pf_swiglu(g[c + 1], u[c + 1], p.limit));
                            __half2 h1 = __floats2half2_rn(pf_swiglu(g[c + 2], u[c + 2], p.limit), pf_swiglu(g[c + 3], u[c + 3], p.limit));
                            __half2 h2 = __floats2half2_rn(pf_swiglu(g[c + 4], u[c + 4], p.limit), pf_swiglu(g[c + 5], u[c + 5], p.limit));
                            __half2 h3 = __floats2half2_rn(pf_swiglu(g[c + 6], u[c + 6], p.limit), pf_swiglu(g[c + 7], u[c + 7], p.limit));
                            v.x = *reinterpret_cast<uint32_t *>(&h0);
                            v.y = *reinterpret_cast<uint32_t *>(&h1);
                            v.z = *reinterpret_cast<uint32_t *>(&h2);
                            v.w = *reinterpret_cast<uint32_t *>(&h3);
                            *reinterpret_cast<uint4 *>(out + n + c) = v;
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    const int n = nt * BN + c0;
                    if (n >= p.N) break;
                    float v[32];
                    tmem_ld32(tacc + c0, v);
                    tmem_wait_ld();
                    if (!ok) continue;
                    if (EPI == PF_STORE_F16) {
                        __half *out = reinterpret_cast<__half *>(p.out) + orow + n;
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            uint4 q;
                            __half2 h0 = __floats2half2_rn(v[c], v[c + 1]);
                            __half2 h1 = __floats2half2_rn(v[c + 2], v[c + 3]);
                            __half2 h2 = __floats2half2_rn(v[c + 4], v[c + 5]);
                            __half2 h3 = __floats2half2_rn(v[c + 6], v[c + 7]);
                            q.x = *reinterpret_cast<uint32_t *>(&h0);
                            q.y = *reinterpret_cast<uint32_t *>(&h1);
                            q.z = *reinterpret_cast<uint32_t *>(&h2);
                            q.w = *reinterpret_cast<uint32_t *>(&h3);
                            *reinterpret_cast<uint4 *>(out + c) = q;
                        }
                    } else {
                        float *out = reinterpret_cast<float *>(p.out) + orow + n;
#pragma unroll
                        for (int c = 0; c < 32; c += 4) {
                            float4 r = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
                            if (EPI == PF_ADD_F32) {
                                const float4 o = *reinterpret_cast<const float4 *>(out + c);
                                r.x = __fadd_rn(o.x, r.x);
                                r.y = __fadd_rn(o.y, r.y);
                                r.z = __fadd_rn(o.z, r.z);
                                r.w = __fadd_rn(o.w, r.w);
                            }
                            *reinterpret_cast<float4 *>(out + c) = r;
                        }
                    }
                }
            }
            }  // m-tile
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cta(&acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPfWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, P::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Causal attention of the chunk in the decompressed form.  For a chunk of
// many queries the absorbed form (1088 MACs per query, key and head) costs
// several times the decompressed one: keys k = [c . W_UK^T | k_rope] (nope +
// rope columns) and values v = c . W_UV^T (value_dim columns) come from one
// GEMM over the latent cache (kvd[key][h * (nope + v) + j]), then
//   o[t][h] = softmax_k((q[t][h] . k[k][h]) * scale, k <= pos + t) . v[k][h]
// (the same function as moonlight_kernels.metal:247-375; the cache, the
// scale and the mask are those of the decode path).
//
// CTA = (128-query tile, head); 64-key blocks in a three-stage ring:
//   warp 0      TMA: the query tile once (q16 row t, columns h*(nope+R) ..),
//               then per block the nope slices from kvd, the rope slice from
//               the latent cache and the value slices from kvd;
//   warp 1      MMA issuer: S = Q . K^T (M = 128, N = 64) into one of two
//               TMEM score buffers, O += P . V (N = value_dim) in TMEM;
//   warp 2      TMEM allocation;
//   warps 4-7   softmax, one query row per thread (exp2 domain, lazy
//               rescale as in mla_attention_tc_kernel), P to shared memory;
//               at the end O / l as fp16 into o16[t][h * value_dim ..].
// ---------------------------------------------------------------------------
constexpr int kFaRows = 128, kFaKeys = 128, kFaStages = 2, kFaThreads = 256;

template <int NQS, int NVS>  // 64-column slices of q.k (nope + rope) and of v
struct FaPlan {
    static constexpr int Q_BYTES = NQS * kFaRows * 128;
    static constexpr int K_BYTES = NQS * kFaKeys * 128;
    static constexpr int V_BYTES = NVS * kFaKeys * 128;
    static constexpr int STAGE = K_BYTES + V_BYTES;
    static constexpr int OFF_KV = Q_BYTES;
    static constexpr int OFF_BAR = OFF_KV + kFaStages * STAGE;
    static constexpr size_t SMEM = (size_t)OFF_BAR + 256 + 1024;
    static constexpr int DV = NVS * 64;
    // TMEM: O (DV columns), two score buffers, P (fp16 pairs: kFaKeys / 2)
    static constexpr uint32_t T_P = DV + 2 * kFaKeys;
    static constexpr uint32_t TMEM_COLS = T_P + kFaKeys / 2 <= 256 ? 256 : 512;
    static_assert(T_P + kFaKeys / 2 <= 512, "TMEM plan");
    static_assert(SMEM <= 232448, "shared memory plan");
};

// grid (query tiles, heads), kFaThreads threads, FaPlan::SMEM bytes.
// qmap: q16 [rows][H * (nope + R)] box {64, 128}; kvmap: kvd
// [keys][H * (nope + v)] box {64, 64}; ropemap: the latent cache
// [layers * context][L + R] box {64, 64}, rows of this layer from rope_row0.
template <int NQS, int NVS>
__global__ void __launch_bounds__(kFaThreads, 1)
pf_attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kvmap,
                    const __grid_constant__ CUtensorMap ropemap, int rope_row0, int L, int T, int H,
                    const int *d_pos, float softmax_scale, __half *o16, int *err) {
    using P = FaPlan<NQS, NVS>;
    constexpr int NP = (NQS - 1) * 64, DV = P::DV;
    extern __shared__ uint8_t fa_smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *Qs = sm, *KVs = sm + P::OFF_KV;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P::OFF_BAR);
    uint64_t *q_full = bars, *kv_full = bars + 1, *kv_empty = kv_full + kFaStages, *s_full = kv_empty + kFaStages,
             *s_free = s_full + 2, *p_full = s_free + 2, *pv_done = p_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pv_done + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // heavier (later) query tiles first
    const int qt = gridDim.x - 1 - blockIdx.x, h = blockIdx.y;
    const int t0 = qt * kFaRows;
    if (tid == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < kFaStages; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
        }
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        mbar_fence_init();
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&qmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&kvmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&ropemap)) : "memory");
    }
    if (warp == 2) {
        __syncwarp();
        tmem_alloc(tmem_slot, P::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_release();

    const int pos = *d_pos;
    const int nkeys = pos + min(t0 + kFaRows, T);   // keys visible to the tile's last row
    const int nblk = (nkeys + kFaKeys - 1) / kFaKeys;
    const uint32_t tO = tmem, tS = tmem + DV, tP = tmem + P::T_P;

    if (warp == 0) {
        if (lane == 0) {
            mbar_expect_tx(q_full, P::Q_BYTES);
            for (int s = 0; s < NQS; ++s) tma_load_2d(Qs + s * kFaRows * 128, &qmap, h * (NP + 64) + s * 64, t0, q_full);
            for (int j = 0; j < nblk; ++j) {
                const int st = j % kFaStages;
                if (j >= kFaStages) mbar_wait_timed(&kv_empty[st], (uint32_t)(((j / kFaStages) - 1) & 1), err, 1);
                mbar_expect_tx(&kv_full[st], P::STAGE);
                uint8_t *dst = KVs + st * P::STAGE;
                const int key0 = j * kFaKeys;
                for (int s = 0; s < NQS - 1; ++s)
                    tma_load_2d(dst + s * kFaKeys * 128, &kvmap, h * (NP + DV) + s * 64, key0, &kv_full[st]);
                tma_load_2d(dst + (NQS - 1) * kFaKeys * 128, &ropemap, L, rope_row0 + key0, &kv_full[st]);
                for (int s = 0; s < NVS; ++s)
                    tma_load_2d(dst + P::K_BYTES + s * kFaKeys * 128, &kvmap, h * (NP + DV) + NP + s * 64, key0,
                                &kv_full[st]);
            }
            // every copy issued has landed before the CTA may exit
            pf_drain(q_full, 0);
            for (int j = max(nblk - kFaStages, 0); j < nblk; ++j)
                pf_drain(&kv_full[j % kFaStages], (uint32_t)((j / kFaStages) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idS = idesc_f16(kFaRows, kFaKeys, false);
            constexpr uint32_t idO = idesc_f16(kFaRows, DV, true);
            const uint32_t qa = smem_u32(Qs), kva = smem_u32(KVs);
            mbar_wait_timed(q_full, 0, err, 0);
            auto issue_scores = [&](int j) {
                const uint32_t kst = kva + (j % kFaStages) * P::STAGE;
                for (int s = 0; s < NQS; ++s)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        uint64_t a = smem_desc(qa + s * kFaRows * 128 + kk * 32, 16, 1024, kSmemLayoutSw128);
                        uint64_t b = smem_desc(kst + s * kFaKeys * 128 + kk * 32, 16, 1024, kSmemLayoutSw128);
                        tc_mma_f16(tS + (j & 1) * kFaKeys, a, b, idS, (s | kk) != 0);
                    }
                tc_commit(&s_full[j & 1]);
            };
            auto scores_ready = [&](int k) {
                return mbar_try_wait(&kv_full[k % kFaStages], (uint32_t)((k / kFaStages) & 1)) &&
                       (k < 2 || mbar_try_wait(&s_free[k & 1], (uint32_t)(((k - 2) >> 1) & 1)));
            };
            int next = 0;
            for (int j = 0; j < nblk; ++j) {
                uint64_t w0 = 0;
                for (uint32_t it = 0;; ++it) {
                    if (next <= j + 1 && next < nblk && scores_ready(next)) {
                        tc_fence_after();
                        issue_scores(next);
                        ++next;
                    }
                    if (next > j && mbar_try_wait(p_full, (uint32_t)(j & 1))) break;
                    if ((it & 255u) == 0) {
                        uint64_t t = global_ns();
                        if (w0 == 0) w0 = t;
                        else if (t - w0 > 200000000ull) {
                            atomicOr(err, 1 | (1 << 12));
                            break;
                        }
                    }
                }
                tc_fence_after();
                const uint32_t vst = kva + (j % kFaStages) * P::STAGE + P::K_BYTES;
#pragma unroll
                for (int kk = 0; kk < kFaKeys / 16; ++kk) {
                    // P from TMEM (one query row per lane, 16 keys = 8 columns per step);
                    // V: MN-major 128-byte swizzle, 64-column slices kFaKeys * 128 B apart
                    uint64_t b = smem_desc(vst + kk * 2048, kFaKeys * 128, 1024, kSmemLayoutSw128);
                    tc_mma_f16_ta(tO, tP + kk * 8, b, idO, (j | kk) != 0);
                }
                tc_commit(&kv_empty[j % kFaStages]);
                tc_commit(pv_done);
            }
        }
    } else if (warp >= 4) {
        const int row = tid - 128;
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        const int t = t0 + row;
        const int limit = t < T ? pos + t : -1;
        const float scale2 = softmax_scale * 1.4426950408889634f;
        float m_run = -INFINITY, l_run = 0.0f;
        for (int j = 0; j < nblk; ++j) {
            const int st = j & 1;
            mbar_wait_timed(&s_full[st], (uint32_t)((j >> 1) & 1), err, 5);
            __syncwarp();
            tc_fence_after();
            // pass 1: the block max; a block with every key visible (all but
            // the diagonal one) skips the mask; scaling after the max is
            // exact (scale2 > 0)
            const int nvis = min(max(limit - j * kFaKeys + 1, 0), kFaKeys);
            const uint32_t ts = tS + st * kFaKeys + lane_off;
            const bool full = nvis == kFaKeys;
            float mb = -INFINITY;
#pragma unroll 1
            for (int c0 = 0; c0 < kFaKeys; c0 += 32) {
                float sv[32];
                tmem_ld32(ts + c0, sv);
                tmem_wait_ld();
                if (full) {
#pragma unroll
                    for (int c = 0; c < 32; ++c) mb = fmaxf(mb, sv[c]);
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c) mb = fmaxf(mb, c0 + c < nvis ? sv[c] : -INFINITY);
                }
            }
            mb = mb == -INFINITY ? mb : mb * scale2;
            const float m_new = (m_run == -INFINITY || mb > m_run + kRescaleLog2) ? mb : m_run;
            const float alpha = m_new == m_run ? 1.0f : exp2f(m_run - m_new);
            const float msub = m_new == -INFINITY ? 0.0f : m_new;
            // the previous block's P . V must be done before P is rewritten
            // and before O is rescaled
            if (j > 0) {
                mbar_wait_timed(pv_done, (uint32_t)((j - 1) & 1), err, 6);
                __syncwarp();
                tc_fence_after();
            }
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                for (int c0 = 0; c0 < DV; c0 += 32) {
                    float o[32];
                    tmem_ld32(tO + c0 + lane_off, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] *= alpha;
                    tmem_st32(tO + c0 + lane_off, o);
                }
                tmem_wait_st();
            }
            // pass 2: P = 2^(s - m) as fp16 pairs into TMEM, 32 keys at a time
            float ps = 0.0f;
#pragma unroll 1
            for (int c0 = 0; c0 < kFaKeys; c0 += 32) {
                float sv[32];
                tmem_ld32(ts + c0, sv);
                tmem_wait_ld();
                uint32_t packed[16];
                if (full) {
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        float p0 = exp2f(fmaf(sv[c], scale2, -msub));
                        float p1 = exp2f(fmaf(sv[c + 1], scale2, -msub));
                        ps += p0;
                        ps += p1;
                        __half2 hp = __floats2half2_rn(p0, p1);
                        packed[c / 2] = *reinterpret_cast<uint32_t *>(&hp);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        float p0 = c0 + c < nvis ? exp2f(fmaf(sv[c], scale2, -msub)) : 0.0f;
                        float p1 = c0 + c + 1 < nvis ? exp2f(fmaf(sv[c + 1], scale2, -msub)) : 0.0f;
                        ps += p0;
                        ps += p1;
                        __half2 hp = __floats2half2_rn(p0, p1);
                        packed[c / 2] = *reinterpret_cast<uint32_t *>(&hp);
                    }
                }
                tmem_st16(tP + c0 / 2 + lane_off, packed);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive_cta(&s_free[st]);
            mbar_arrive_cta(p_full);
            l_run = l_run * alpha + ps;
            m_run = m_new;
        }
        if (nblk > 0) {
            mbar_wait_timed(pv_done, (uint32_t)((nblk - 1) & 1), err, 7);
            __syncwarp();
            tc_fence_after();
        }
        const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        __half *dst = o16 + (size_t)(t < T ? t : 0) * H * DV + (size_t)h * DV;
#pragma unroll 1
        for (int c0 = 0; c0 < DV; c0 += 32) {
            float o[32];
            tmem_ld32(tO + c0 + lane_off, o);
            tmem_wait_ld();
            if (t < T) {
#pragma unroll
                for (int c = 0; c < 32; c += 8) {
                    __half2 h0 = __floats2half2_rn(o[c] * inv, o[c + 1] * inv);
                    __half2 h1 = __floats2half2_rn(o[c + 2] * inv, o[c + 3] * inv);
                    __half2 h2 = __floats2half2_rn(o[c + 4] * inv, o[c + 5] * inv);
                    __half2 h3 = __floats2half2_rn(o[c + 6] * inv, o[c + 7] * inv);
                    *reinterpret_cast<uint4 *>(dst + c0 + c) =
                        make_uint4(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1),
                                   *reinterpret_cast<uint32_t *>(&h2), *reinterpret_cast<uint32_t *>(&h3));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, P::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Row-parallel kernels of the prefill chunk.
// ---------------------------------------------------------------------------

// RMSNorm of row blockIdx.x (moonlight_kernels.metal:23-41) -> fp16 GEMM
// operand y16[row][0..D) and, optionally, fp32 y32.  float4 loads, the row
// held in registers (D <= 8192), half4 / float4 stores.
constexpr int kPfNormVec = 8;  // float4 per thread at most
__global__ void __launch_bounds__(256) pf_rmsnorm_kernel(const float *x, int D, const float *w, float eps,
                                                         __half *y16, int ld16, float *y32) {
    pdl_wait();
    pdl_release();
    __shared__ float scratch[32];
    const int s = blockIdx.x, n4 = D / 4;
    const float4 *xs = reinterpret_cast<const float4 *>(x + (size_t)s * D);
    float4 v[kPfNormVec];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kPfNormVec; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        if (k4 < n4) {
            v[i] = xs[k4];
            ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        }
    }
    ss = block_sum(ss, scratch);
    const float scale = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < kPfNormVec; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        if (k4 >= n4) continue;
        const float4 wv = reinterpret_cast<const float4 *>(w)[k4];
        float o[4] = {v[i].x * scale * wv.x, v[i].y * scale * wv.y, v[i].z * scale * wv.z, v[i].w * scale * wv.w};
        __half2 h0 = __floats2half2_rn(fminf(fmaxf(o[0], -65504.0f), 65504.0f), fminf(fmaxf(o[1], -65504.0f), 65504.0f));
        __half2 h1 = __floats2half2_rn(fminf(fmaxf(o[2], -65504.0f), 65504.0f), fminf(fmaxf(o[3], -65504.0f), 65504.0f));
        *reinterpret_cast<uint2 *>(y16 + (size_t)s * ld16 + 4 * k4) =
            make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
        if (y32) reinterpret_cast<float4 *>(y32 + (size_t)s * D)[k4] = make_float4(o[0], o[1], o[2], o[3]);
    }
}

// KV append and query rope for row blockIdx.x at position *pos + row
// (moonlight_cache_append / _rope_query, moonlight_kernels.metal:132-216):
// block y 0 normalizes the latent (kv_a_norm) and ropes the key into the
// cache; blocks y >= 1 rope the rope columns of the fp16 queries in place
// (pairs (2p, 2p+1) -> halves (p, R/2 + p), the cache's key layout).  A
// block holds whole heads (R/2 divides 256), so reading every pair before
// the barrier and writing after it is race-free.
__global__ void __launch_bounds__(256) pf_prep_kernel(const float *ckv, __half *q16, const float *norm_w, int L,
                                                      int R, int H, int nope, float eps, float theta,
                                                      const int *d_pos, __half *cache) {
    pdl_wait();
    pdl_release();
    __shared__ float scratch[32];
    const int s = blockIdx.x, position = *d_pos + s, half = R / 2;
    if (blockIdx.y == 0) {
        const float *src = ckv + (size_t)s * (L + R);
        float ss = 0.0f;
        for (int i = threadIdx.x; i < L; i += blockDim.x) ss += src[i] * src[i];
        ss = block_sum(ss, scratch);
        const float scale = 1.0f / sqrtf(ss / (float)L + eps);
        __half *dst = cache + (size_t)position * (L + R);
        for (int i = threadIdx.x; i < L; i += blockDim.x) dst[i] = __float2half_rn(src[i] * scale * norm_w[i]);
        for (int pp = threadIdx.x; pp < half; pp += blockDim.x) {
            float a, b;
            rope_pair(src[L + 2 * pp], src[L + 2 * pp + 1], pp, R, position, theta, a, b);
            dst[L + pp] = __float2half_rn(a);
            dst[L + half + pp] = __float2half_rn(b);
        }
        return;
    }
    const int qw = nope + R;
    const int t = (blockIdx.y - 1) * blockDim.x + threadIdx.x;
    const bool on = t < H * half;
    const int h = on ? t / half : 0, pp = on ? t % half : 0;
    __half *qh = q16 + ((size_t)s * H + h) * qw + nope;
    float a = 0.0f, b = 0.0f;
    if (on) rope_pair(__half2float(qh[2 * pp]), __half2float(qh[2 * pp + 1]), pp, R, position, theta, a, b);
    __syncthreads();
    if (on) {
        qh[pp] = __float2half_rn(a);
        qh[half + pp] = __float2half_rn(b);
    }
}

// Router logits of the chunk in fp32: part[split][t][e] = sum over the
// split's k range of x[t][k] * W[e][k] (64 x 64 output tiles, 4 x 4 per
// thread, k ascending); pf_route_kernel adds the splits in split order.
// Splitting k keeps every SM busy when rows x experts make few tiles.
constexpr int kPfRtTile = 64, kPfRtK = 32, kPfRtMaxSplits = 8;
__global__ void __launch_bounds__(256) pf_router_logits_kernel(const float *W, const float *x, int T, int D, int E,
                                                               int ksplit, float *part) {
    pdl_wait();
    pdl_release();
    __shared__ __align__(16) float xs[kPfRtK][kPfRtTile + 4], ws[kPfRtK][kPfRtTile + 4];
    const int t0 = blockIdx.x * kPfRtTile, e0 = blockIdx.y * kPfRtTile, sp = blockIdx.z;
    const int kb = sp * ksplit, ke = min(D, kb + ksplit);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    // the next k-tile is loaded into registers while this one is multiplied
    constexpr int kPer = kPfRtTile * kPfRtK / 256;  // elements per thread per tile
    float xr[kPer], wr[kPer];
    auto load = [&](int k0) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = threadIdx.x + j * 256, r = i / kPfRtK, k = i % kPfRtK;
            xr[j] = t0 + r < T ? x[(size_t)(t0 + r) * D + k0 + k] : 0.0f;
            wr[j] = e0 + r < E ? W[(size_t)(e0 + r) * D + k0 + k] : 0.0f;
        }
    };
    if (kb < ke) load(kb);
    for (int k0 = kb; k0 < ke; k0 += kPfRtK) {
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = threadIdx.x + j * 256, r = i / kPfRtK, k = i % kPfRtK;
            xs[k][r] = xr[j];
            ws[k][r] = wr[j];
        }
        __syncthreads();
        if (k0 + kPfRtK < ke) load(k0 + kPfRtK);
#pragma unroll 8
        for (int k = 0; k < kPfRtK; ++k) {
            const float4 xv = *reinterpret_cast<const float4 *>(&xs[k][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4 *>(&ws[k][tx * 4]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(xa[a], wa[b], acc[a][b]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int t = t0 + ty * 4 + a;
        if (t >= T) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int e = e0 + tx * 4 + b;
            if (e < E) part[((size_t)sp * T + t) * E + e] = acc[a][b];
        }
    }
}

// Top-k selection of every row (one warp per row, route_row), then the
// rows per expert (counts[e], zero on entry).
constexpr int kPfRouteWarps = 8;
__global__ void __launch_bounds__(32 * kPfRouteWarps) pf_route_kernel(const float *part, int nsplit, float *logits,
                                                                      RouteParams p, int *counts) {
    pdl_wait();
    pdl_release();
    __shared__ int sel[kPfRouteWarps][64];
    __shared__ float selw[kPfRouteWarps][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s = blockIdx.x * kPfRouteWarps + warp;
    if (s >= p.S) return;
    // logits = the k splits in order; per-expert score functions: the score
    // and the selection value (score + bias) here
    for (int e = lane; e < p.E; e += 32) {
        float v = 0.0f;
        for (int sp = 0; sp < nsplit; ++sp) v += part[((size_t)sp * p.S + s) * p.E + e];
        if (p.score_fn == FC_SCORE_SOFTMAX) {
            logits[(size_t)s * p.E + e] = v;
        } else {
            const float sc = route_score(v, p.score_fn);
            logits[(size_t)s * p.E + e] = sc;
            p.choice[(size_t)s * p.E + e] = sc + (p.bias ? p.bias[e] : 0.0f);
        }
    }
    __syncwarp();
    const int per = (p.E + 31) / 32;
    if (per <= 2) route_row<2>(logits, p, s, sel[warp], selw[warp]);
    else if (per <= 4) route_row<4>(logits, p, s, sel[warp], selw[warp]);
    else if (per <= 8) route_row<8>(logits, p, s, sel[warp], selw[warp]);
    else if (per <= 16) route_row<16>(logits, p, s, sel[warp], selw[warp]);
    else route_row<32>(logits, p, s, sel[warp], selw[warp]);
    for (int k = lane; k < p.K; k += 32) atomicAdd(&counts[sel[warp][k]], 1);
}

// Expert row ranges (ascending expert id) and the m-tile table of the
// grouped GEMMs; clears the counts for the next layer.  One block.
__global__ void __launch_bounds__(1024) pf_group_kernel(int *counts, int E, int *offsets, int *cursor,
                                                        int4 *mt_table, int *mt_count) {
    pdl_wait();
    pdl_release();
    __shared__ int off[1025], tiles[1025];
    const int e = threadIdx.x;
    const int c = e < E ? counts[e] : 0;
    off[e + 1] = c;
    tiles[e + 1] = (c + kPfMI - 1) / kPfMI;
    if (e == 0) off[0] = tiles[0] = 0;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        int a = 0, b = 0;
        if (e + 1 > o) {
            a = off[e + 1 - o];
            b = tiles[e + 1 - o];
        }
        __syncthreads();
        off[e + 1] += a;
        tiles[e + 1] += b;
        __syncthreads();
    }
    if (e < E) {
        offsets[e] = off[e];
        cursor[e] = off[e];
        counts[e] = 0;
        for (int i = 0; i < tiles[e + 1] - tiles[e]; ++i)
            mt_table[tiles[e] + i] = make_int4(e, off[e] + i * kPfMI, off[e] + c, 0);
    }
    if (e == 0) *mt_count = tiles[E];
}

// One warp per (row, choice): takes the next row of its expert's range and
// copies the row's fp16 activations there.
__global__ void __launch_bounds__(256) pf_gather_kernel(const int *route_ids, int T, int K, int *cursor,
                                                        int *slot_of, const __half *x16, int D, __half *xg) {
    pdl_wait();
    pdl_release();
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= T * K) return;
    int slot = 0;
    if (lane == 0) {
        slot = atomicAdd(&cursor[route_ids[w]], 1);
        slot_of[w] = slot;
    }
    slot = __shfl_sync(0xffffffffu, slot, 0);
    const uint4 *src = reinterpret_cast<const uint4 *>(x16 + (size_t)(w / K) * D);
    uint4 *dst = reinterpret_cast<uint4 *>(xg + (size_t)slot * D);
    for (int i = lane; i < D / 8; i += 32) dst[i] = src[i];
}

// resid[t] += (sum over the row's experts in ascending id of w * y[slot])
// + shared[t]  (moe_exec.h:97-110 order); float4 loads and stores, each
// element's sum in the same order.
__global__ void __launch_bounds__(256) pf_combine_kernel(float *resid, const float *yd, const float *shared,
                                                         const int *route_ids, const float *route_w,
                                                         const int *slot_of, int K, int D) {
    pdl_wait();
    pdl_release();
    __shared__ int sl[64];
    __shared__ float sw[64];
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        int ids[64];
        for (int k = 0; k < K; ++k) {
            ids[k] = route_ids[t * K + k];
            sl[k] = slot_of[t * K + k];
            sw[k] = route_w[t * K + k];
        }
        for (int a = 1; a < K; ++a)  // insertion sort by expert id
            for (int b = a; b > 0 && ids[b - 1] > ids[b]; --b) {
                int ti = ids[b]; ids[b] = ids[b - 1]; ids[b - 1] = ti;
                int ts = sl[b]; sl[b] = sl[b - 1]; sl[b - 1] = ts;
                float tw = sw[b]; sw[b] = sw[b - 1]; sw[b - 1] = tw;
            }
    }
    __syncthreads();
    float4 *r4 = reinterpret_cast<float4 *>(resid + (size_t)t * D);
    for (int d4 = threadIdx.x; d4 < D / 4; d4 += blockDim.x) {
        float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < K; ++k) {
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(yd + (size_t)sl[k] * D) + d4);
            const float c = sw[k];
            y.x = __fadd_rn(y.x, __fmul_rn(c, v.x));
            y.y = __fadd_rn(y.y, __fmul_rn(c, v.y));
            y.z = __fadd_rn(y.z, __fmul_rn(c, v.z));
            y.w = __fadd_rn(y.w, __fmul_rn(c, v.w));
        }
        if (shared) {
            const float4 sh = reinterpret_cast<const float4 *>(shared + (size_t)t * D)[d4];
            y.x = __fadd_rn(y.x, sh.x);
            y.y = __fadd_rn(y.y, sh.y);
            y.z = __fadd_rn(y.z, sh.z);
            y.w = __fadd_rn(y.w, sh.w);
        }
        float4 r = r4[d4];
        r.x = __fadd_rn(r.x, y.x);
        r.y = __fadd_rn(r.y, y.y);
        r.z = __fadd_rn(r.z, y.z);
        r.w = __fadd_rn(r.w, y.w);
        r4[d4] = r;
    }
}

}  // namespace fc
