// mla_tc.cuh - latent attention of the verify rows on the 5th-generation
// tensor cores (tcgen05 + TMEM, operands staged by TMA).
//
// Same contract as mla_attention_kernel (moonlight_kernels.metal:247-330 for
// the math): for every query q = s * H + h of the batch and every key of one
// split, scores = qcat[q] . cache[key] (latent + rope, width L + 64), scaled,
// masked to key <= pos + s, online softmax, and O = P . cache[key][0:L].
// Writes the unnormalized split partials part_o [split][q][L] and, per half
// of the output columns, part_m / part_l [half][split][q] that
// mla_combine_kernel folds in split order.
//
// One CTA = (128-query tile, half of the L output columns, key split):
//   warp 0      TMA producer: the query tile once, then 32-key blocks of the
//               latent cache into a two-stage ring (128-byte swizzle).  Each
//               stage has two parts with their own barriers: the 64-column
//               slices this half's P . V reads (V slices) and the others.
//               The other slices are refilled as soon as the block's score
//               MMAs are done, the V slices once its P . V is done;
//   warp 1      MMA issuer: S = Q . K^T into one of two 32-column TMEM score
//               buffers (M=128, N=32, K=L+64; the V slices last, so the
//               V-slice load of a block overlaps its first score MMAs), then
//               O += P . V into the L/2-column TMEM accumulator (M=128,
//               N=L/2, K=32, V read MN-major straight from the key block);
//   warp 2      TMEM allocation;
//   warps 4-7   softmax: thread = query row = TMEM lane; reads its 32 scores,
//               masks, updates max / sum, rescales its O row in TMEM when the
//               max rises, writes its P row (fp16) to shared memory.
// The two halves of a query tile compute the same scores (summed in each
// half's slice order, so each half keeps its own max and sum); each keeps its
// own 256 (or 128) output columns, so O fits the 512 TMEM columns.
// Each output row depends only on its own query and the split's keys, so a
// verify row and a decode of the same token give the same bits.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "head.cuh"

namespace fc {

// ---- tcgen05 / TMA wrappers ------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// Arrives on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// D (TMEM) (+)= A (smem) . B (smem), fp16 inputs, fp32 accumulation.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 16 consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::
            "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// tcgen05.mma kind::f16 with the A operand in tensor memory: M rows, one per
// lane, 16 fp16 per row as 8 columns of pairs (k = 2c, 2c + 1 in column c).
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// Orders this thread's generic shared-memory writes before later tensor-core reads.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
// 2-D tiled TMA load of this GPU's memory into shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// 4-D tiled TMA load of this GPU's memory (no multicast).
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
    return t;
}
// Waits for phase `parity` of `bar` for at most ~0.2 s; on timeout records
// bit (8 + site) in *err (which wait gave up) and returns false.
__device__ __forceinline__ bool mbar_wait_timed(uint64_t *bar, uint32_t parity, int *err, int site) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            uint64_t t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > 200000000ull) break;
        }
    }
    if (err) atomicOr(err, 1 | (1 << (8 + site)));
    return false;
}

// Shared-memory matrix descriptor (tcgen05): start, leading / stride byte
// offsets, version 1, layout (0 = interleaved core matrices, 2 = 128-byte swizzle).
constexpr uint32_t kSmemLayoutNone = 0, kSmemLayoutSw128 = 2;
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
// Instruction descriptor of kind::f16: fp16 A and B, fp32 D, A K-major,
// B K-major or MN-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn_major) {
    return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- kernel ----------------------------------------------------------------
#ifdef FC_TC_TRACE
__device__ unsigned long long g_tc_trace[256];
#define TC_MARK(i)                                                                                   \
    do {                                                                                             \
        if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (i) < 256) g_tc_trace[(i)] = clock64(); \
    } while (0)
#else
#define TC_MARK(i) \
    do {           \
    } while (0)
#endif
constexpr int kTcThreads = 256;
constexpr int kTcRows = 128;  // queries per tile (MMA M)
constexpr int kTcKeys = 32;   // keys per block (score MMA N)
constexpr float kRescaleLog2 = 11.0f;  // lazy softmax rescale threshold (log2)

template <int L>
struct TcAttnPlan {
    static constexpr int DW = L + 64;            // score width (latent + rope)
    static constexpr int NKB = DW / 64;          // 64-column (128-byte) slices
    static constexpr int HALF = L / 2;           // output columns per CTA
    static constexpr int VS = HALF / 64;         // V slices of a half
    static constexpr int NV = NKB - VS;          // slices only the scores read
    static constexpr int Q_BYTES = NKB * kTcRows * 128;
    static constexpr int K_BYTES = NKB * kTcKeys * 128;
    static constexpr int P_BYTES = kTcRows * kTcKeys * 2;
    static constexpr int OFF_K = Q_BYTES;
    static constexpr int OFF_P = OFF_K + 2 * K_BYTES;
    static constexpr int OFF_BAR = OFF_P + P_BYTES;
    static constexpr size_t SMEM = (size_t)OFF_BAR + 128 + 1024;  // + 1 KB for base alignment
    static constexpr int S_COLS = kTcKeys;                      // one score buffer
    static constexpr uint32_t TMEM_COLS = 512;                   // O (HALF) + two score buffers
    static_assert(HALF + 2 * S_COLS <= (int)TMEM_COLS, "TMEM plan");
    static_assert(SMEM <= 232448, "shared memory plan");
};

// grid (query tiles, 2 halves, splits), 256 threads, TcAttnPlan<L>::SMEM bytes.
// kv_row0 = layer * context rows of the cache tensor map; split `z` covers
// keys [z * keys_per_split, (z + 1) * keys_per_split) (a multiple of 32).
template <int L>
__global__ void __launch_bounds__(kTcThreads, 1)
mla_attention_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kvmap,
                        int kv_row0, int S, int H, int keys_per_split, const Staging *st, PageMap pm,
                        float softmax_scale, float *part_o, float *part_m, float *part_l, int *err) {
    using P = TcAttnPlan<L>;
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *Qs = sm;
    uint8_t *Ks = sm + P::OFF_K;
    uint8_t *Ps = sm + P::OFF_P;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + P::OFF_BAR);
    // kv_*_a: the stage's non-V slices, kv_*_b: its V slices
    uint64_t *q_full = bars + 0, *kv_full_a = bars + 1, *kv_full_b = bars + 3, *kv_empty_a = bars + 5,
             *kv_empty_b = bars + 7, *s_full = bars + 9, *s_free = bars + 11, *p_full = bars + 13,
             *pv_done = bars + 14;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 15);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * kTcRows, half = blockIdx.y, split = blockIdx.z;
    if (tid == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&kv_full_a[i], 1);
            mbar_init(&kv_full_b[i], 1);
            mbar_init(&kv_empty_a[i], 1);
            mbar_init(&kv_empty_b[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
        }
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        mbar_fence_init();
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&qmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&kvmap)) : "memory");
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
    if (tid == 0) TC_MARK(0);
    pdl_wait();
    pdl_release();
    if (tid == 0) TC_MARK(1);

    // the tile's rows belong to one sequence; keys up to its last row's
    // position (causal: key <= that row's position)
    const int nq = S * H, seq = st->rowseq[q0 / H];
    const int total = st->rowpos[(min(q0 + kTcRows, nq) - 1) / H] + 1;
    const int k0 = split * keys_per_split;
    const int k1 = min(k0 + keys_per_split, total);
    const int nblk = k1 > k0 ? (k1 - k0 + kTcKeys - 1) / kTcKeys : 0;
    const uint32_t tO = tmem, tS = tmem + P::HALF;
    // i-th slice in this half's order: the non-V slices ascending, then the V slices
    auto slice = [&](int i) { return i < P::NV ? (i < half * P::VS ? i : i + P::VS) : half * P::VS + (i - P::NV); };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && nblk > 0) {
            mbar_expect_tx(q_full, P::Q_BYTES);
            for (int kb = 0; kb < P::NKB; ++kb) tma_load_2d(Qs + kb * kTcRows * 128, &qmap, kb * 64, q0, q_full);
            // the non-V slices run one block ahead of the V slices: those of
            // block j are refilled once block j - 2's scores are done, before
            // the V slices of block j - 1 (which wait for block j - 3's P . V)
            for (int j = 0; j <= nblk; ++j) {
                if (j < nblk) {
                    const int stg = j & 1;
                    if (j >= 2) mbar_wait_timed(&kv_empty_a[stg], (uint32_t)(((j - 2) >> 1) & 1), err, 1);
                    TC_MARK(136 + j);
                    const int krow = kv_row0 + kv_row(pm, seq, k0 + j * kTcKeys);
                    uint8_t *dst = Ks + stg * P::K_BYTES;
                    mbar_expect_tx(&kv_full_a[stg], P::NV * kTcKeys * 128);
                    for (int i = 0; i < P::NV; ++i) {
                        const int kb = slice(i);
                        tma_load_2d(dst + kb * kTcKeys * 128, &kvmap, kb * 64, krow, &kv_full_a[stg]);
                    }
                }
                if (j >= 1) {
                    const int k = j - 1, stg = k & 1;
                    if (k >= 2) mbar_wait_timed(&kv_empty_b[stg], (uint32_t)(((k - 2) >> 1) & 1), err, 1);
                    TC_MARK(168 + k);
                    const int krow = kv_row0 + kv_row(pm, seq, k0 + k * kTcKeys);
                    uint8_t *dst = Ks + stg * P::K_BYTES;
                    mbar_expect_tx(&kv_full_b[stg], P::VS * kTcKeys * 128);
                    for (int i = P::NV; i < P::NKB; ++i) {
                        const int kb = slice(i);
                        tma_load_2d(dst + kb * kTcKeys * 128, &kvmap, kb * 64, krow, &kv_full_b[stg]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && nblk > 0) {
            constexpr uint32_t idS = idesc_f16(kTcRows, kTcKeys, false);
            constexpr uint32_t idO = idesc_f16(kTcRows, P::HALF, true);
            const uint32_t qa = smem_u32(Qs), ka = smem_u32(Ks), pa = smem_u32(Ps);
            mbar_wait_timed(q_full, 0, err, 0);
            TC_MARK(2);
            // score MMAs of slices [i0, i1) (in this half's order) of block k.
            // K-major, 128-byte swizzle: rows 128 B apart, 8-row groups 1024 B
            // apart; the k-th 16-column step starts 32 B further into the row.
            // The descriptors are built once; a step adds its byte offset / 16
            // to the start-address field (every operand lies below 256 KB).
            const uint64_t qdesc = smem_desc(qa, 16, 1024, kSmemLayoutSw128);
            const uint64_t kdesc = smem_desc(ka, 16, 1024, kSmemLayoutSw128);
            auto issue_scores = [&](int k, int i0, int i1) {
                const uint64_t kd = kdesc + (uint64_t)(((k & 1) * P::K_BYTES) >> 4);
                const uint32_t ts = tS + (k & 1) * P::S_COLS;
#pragma unroll
                for (int i = 0; i < P::NKB; ++i) {
                    if (i < i0 || i >= i1) continue;
                    const int kb = slice(i);
                    const uint64_t ad = qdesc + (uint64_t)(kb * (kTcRows * 128 / 16));
                    const uint64_t bd = kd + (uint64_t)(kb * (kTcKeys * 128 / 16));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        tc_mma_f16(ts, ad + 2 * kk, bd + 2 * kk, idS, i > 0 || kk != 0);
                    }
                }
            };
            int next = 0;           // next score block to issue
            bool next_nv = false;   // its non-V slices are issued
            for (int j = 0; j < nblk; ++j) {
                // Issue P . V of block j as soon as its P is written; until
                // then issue the scores of block j (needed for that) and of
                // block j + 1 whenever their inputs are ready: the non-V
                // slices once they have landed and the softmax has read the
                // score buffer's previous block (k - 2), the V slices once
                // they have landed.
                uint64_t t0 = 0;
                for (uint32_t it = 0;; ++it) {
                    if (next > j && mbar_try_wait(p_full, (uint32_t)(j & 1))) break;
                    if (next <= j + 1 && next < nblk) {
                        const int stg = next & 1;
                        const uint32_t ph = (uint32_t)((next >> 1) & 1);
                        if (!next_nv && mbar_try_wait(&kv_full_a[stg], ph) &&
                            (next < 2 || mbar_try_wait(&s_free[stg], (uint32_t)(((next - 2) >> 1) & 1)))) {
                            tc_fence_after();
                            TC_MARK(8 + next);
                            issue_scores(next, 0, P::NV);
                            tc_commit(&kv_empty_a[stg]);
                            next_nv = true;
                        }
                        if (next_nv && mbar_try_wait(&kv_full_b[stg], ph)) {
                            tc_fence_after();
                            TC_MARK(24 + next);
                            issue_scores(next, P::NV, P::NKB);
                            tc_commit(&s_full[stg]);
                            ++next;
                            next_nv = false;
                            continue;
                        }
                    }
                    if ((it & 255u) == 0) {
                        uint64_t t = global_ns();
                        if (t0 == 0) t0 = t;
                        else if (t - t0 > 200000000ull) {
                            atomicOr(err, 1 | (1 << 12));
                            break;
                        }
                    }
                }
                tc_fence_after();
                TC_MARK(40 + j);
                const uint32_t vst = ka + (j & 1) * P::K_BYTES + (half * P::HALF / 64) * (kTcKeys * 128);
#pragma unroll
                for (int kk = 0; kk < kTcKeys / 16; ++kk) {
                    // P: K-major core matrices (8 rows x 16 B), K-adjacent 128 B apart, 8-row groups 512 B apart
                    uint64_t a = smem_desc(pa + kk * 256, 128, 512, kSmemLayoutNone);
                    // V: MN-major, 128-byte swizzle: 64 columns per 128-byte key row, next 64 columns
                    // in the next slice (4 KB), next 8 keys 1024 B further
                    uint64_t b = smem_desc(vst + kk * 2048, kTcKeys * 128, 1024, kSmemLayoutSw128);
                    tc_mma_f16(tO, a, b, idO, (j | kk) != 0);
                }
                tc_commit(&kv_empty_b[j & 1]);
                tc_commit(pv_done);
            }
        }
    } else if (warp >= 4) {
        // ---------------- softmax: one query row per thread ----------------
        const int row = tid - 128;                      // == 32 * (warp & 3) + lane
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        const int q = q0 + row;
        const int limit = q < nq ? st->rowpos[q / H] : -1;  // key <= limit is visible
        const float scale2 = softmax_scale * 1.4426950408889634f;  // log2(e)
        float m_run = -INFINITY, l_run = 0.0f;                      // log2 domain
        for (int j = 0; j < nblk; ++j) {
            const int stg = j & 1;
            mbar_wait_timed(&s_full[stg], (uint32_t)((j >> 1) & 1), err, 5);
            if (row == 0) TC_MARK(72 + j);
            __syncwarp();  // tcgen05.ld is warp-collective
            tc_fence_after();
            float sv[32];
            tmem_ld32(tS + stg * P::S_COLS + lane_off, sv);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive_cta(&s_free[stg]);
            // scores in the log2 domain: s2 = score * scale * log2(e)
            const int nvis = min(max(limit - (k0 + j * kTcKeys) + 1, 0), kTcKeys);
            float mb = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                float v = c < nvis ? sv[c] * scale2 : -INFINITY;
                sv[c] = v;
                mb = fmaxf(mb, v);
            }
            // The reference max moves only when the block max exceeds it by
            // more than kRescaleLog2 (P stays below 2^11 in fp16, O and l in
            // fp32), so the TMEM round trip of rescaling O is rare; the
            // decision depends on this row's scores alone.
            const float m_new = (m_run == -INFINITY || mb > m_run + kRescaleLog2) ? mb : m_run;
            const float alpha = m_new == m_run ? 1.0f : exp2f(m_run - m_new);
            const float msub = m_new == -INFINITY ? 0.0f : m_new;  // all masked: 2^-inf = 0
            float ps = 0.0f;
            uint32_t packed[16];
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
                float p0 = exp2f(sv[c] - msub);
                float p1 = exp2f(sv[c + 1] - msub);
                ps += p0;
                ps += p1;
                __half2 hp = __floats2half2_rn(p0, p1);
                packed[c / 2] = *reinterpret_cast<uint32_t *>(&hp);
            }
            // the previous block's P . V must be done before P is rewritten
            // and before O is rescaled
            if (j > 0) {
                mbar_wait_timed(pv_done, (uint32_t)((j - 1) & 1), err, 6);
                __syncwarp();
                tc_fence_after();
            }
            // warp-uniform branch (tcgen05.ld / st are warp-collective); rows
            // whose max did not rise scale by exactly 1
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                for (int c0 = 0; c0 < P::HALF; c0 += 32) {
                    float o[32];
                    tmem_ld32(tO + c0 + lane_off, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] *= alpha;
                    tmem_st32(tO + c0 + lane_off, o);
                }
                tmem_wait_st();
            }
            uint8_t *prow = Ps + (row >> 3) * 512 + (row & 7) * 16;
#pragma unroll
            for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4 *>(prow + c * 128) =
                    make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
            fence_async_smem();
            tc_fence_before();
            mbar_arrive_cta(p_full);
            if (row == 0) TC_MARK(104 + j);
            l_run = l_run * alpha + ps;
            m_run = m_new;
        }
        if (nblk > 0) {
            mbar_wait_timed(pv_done, (uint32_t)((nblk - 1) & 1), err, 7);
            __syncwarp();
            tc_fence_after();
        }
        float *dst = part_o + ((size_t)split * nq + (q < nq ? q : 0)) * L + half * P::HALF;
#pragma unroll 1
        for (int c0 = 0; c0 < P::HALF; c0 += 32) {
            float o[32];
            if (nblk > 0) {
                tmem_ld32(tO + c0 + lane_off, o);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) o[c] = 0.0f;
            }
            if (q < nq) {
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                    *reinterpret_cast<float4 *>(dst + c0 + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
            }
        }
        if (row == 0) TC_MARK(200);
        if (q < nq) {
            // back to the natural-log domain of the split combine
            const size_t at = ((size_t)half * gridDim.z + split) * nq + q;
            part_m[at] = m_run == -INFINITY ? -INFINITY : m_run * 0.6931471805599453f;
            part_l[at] = l_run;
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

}  // namespace fc

