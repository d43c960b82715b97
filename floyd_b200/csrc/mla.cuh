// mla.cuh - compressed-latent MLA attention over the resident KV cache for
// 1 + k verify rows (absorbed W_UK / W_UV, the cache is never decompressed).
//
// Replaces, from moonlight_kernels.metal: cache_append (:132-170),
// rope_query (:172-200), attention_absorb_query (:218-245),
// attention_scores (:247-282), attention_latent_context (:284-343); the
// decode_value step (:345-375) is a GEMV family in gemv.cuh.
//
// Cache layout: per layer [context][L + R] fp16 (latent row, then the rotated
// rope part), 1152 bytes per position for L=512, R=64.  The query operand is
// the same shape: qcat[s * H + h][L + R] = (q_nope . W_UK[h], rope(q_rope)).
//
// The attention kernel is flash-decoding on the tensor cores: a CTA owns 32
// query rows (heads x verify rows share one cache, MQA-like) and a fixed
// range of 64-key chunks; scores (32 x 64, K = L + R) and P . C (32 x L,
// K = 64 keys) are m16n8k16 MMAs from shared memory, with an online softmax
// across the chunks of the range.  Split boundaries are a function of the key
// index and the session's context size only, and masked keys contribute
// exact zeros, so a verify row reproduces a single-token decode bit for bit.
#pragma once

#include "common.cuh"
#include "head.cuh"

namespace fc {

// ---------------------------------------------------------------------------
// Embedding gather (moonlight_kernels.metal:10-21) of a quantized table.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float dequant_element(int fmt, const uint8_t *w, int kp, int row, int k) {
    if (fmt == FC_FMT_F32) return reinterpret_cast<const float *>(w)[(size_t)row * kp + k];
    int nib;
    uint8_t byte = w[value_offset(fmt, kp, row, k, &nib)];
    const uint8_t *sp = w + scale_offset(fmt, kp, row, k >> 5);
    if (fmt == FC_FMT_Q8) return (float)(int8_t)byte * __half2float(*reinterpret_cast<const __half *>(sp));
    uint32_t code = (byte >> (4 * nib)) & 15u;
    if (fmt == FC_FMT_Q4)
        return (float)((int)code - 8) * __half2float(*reinterpret_cast<const __half *>(sp));
    const float table[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    float v = table[code & 7];
    if (code & 8) v = -v;
    return v * e8m0_to_float(*sp);
}

// grid (rows, ceil(D / 256)), 256 threads: one element per thread, so the
// scattered weight and scale loads of a row are all in flight at once.
constexpr int kEmbedThreads = 256;
__global__ void embed_kernel(int fmt, const uint8_t *w, int D, int kp, const int *ids, float *x) {
    pdl_wait();
    pdl_release();
    const int s = blockIdx.x, k = blockIdx.y * kEmbedThreads + threadIdx.x;
    if (k < D) x[(size_t)s * D + k] = dequant_element(fmt, w, kp, ids[s], k);
}
inline dim3 embed_grid(int rows, int D) { return dim3(rows, (D + kEmbedThreads - 1) / kEmbedThreads); }

// ---------------------------------------------------------------------------
// RMSNorm (moonlight_kernels.metal:23-41): y = x / sqrt(mean(x^2) + eps) * w.
// Writes the xq operand of the next GEMV and, optionally, fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float block_sum(float v, float *scratch) {
    v = warp_sum(v);
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += scratch[i];
    return t;
}

// One block per row, one float4 per thread per pass (D / 4 <= 4 * blockDim):
// a single read of the row, the sum of squares reduced in a fixed order,
// then 16-byte xq records (and optionally fp32) written back.
constexpr int kNormThreads = 1024;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float *x, int ldx, const float *w,
                                                               int D, float eps, __half *yq, int kpy,
                                                               float *y, int ldy) {
    __shared__ float scratch[32];
    const int s = blockIdx.x, n4 = D / 4;
    // the norm weights are constant: fetch them before waiting for x
    float4 wv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int k4 = threadIdx.x + i * blockDim.x;
        if (k4 < n4) wv[i] = __ldg(reinterpret_cast<const float4 *>(w) + k4);
    }
    pdl_wait();
    pdl_release();
    const float4 *xs = reinterpret_cast<const float4 *>(x + (size_t)s * ldx);
    float4 v[4];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int k4 = threadIdx.x + i * blockDim.x;
        if (k4 < n4) {
            v[i] = xs[k4];
            ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        }
    }
    ss = block_sum(ss, scratch);
    const float scale = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int k4 = threadIdx.x + i * blockDim.x;
        if (k4 >= n4) continue;
        float o[4] = {v[i].x * scale * wv[i].x, v[i].y * scale * wv[i].y, v[i].z * scale * wv[i].z,
                      v[i].w * scale * wv[i].w};
        if (yq) {
            __half hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) split_hi_lo(o[e], hi[e], lo[e]);
            uint4 rec;
            rec.x = (uint32_t)__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
            rec.y = (uint32_t)__half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16);
            rec.z = (uint32_t)__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
            rec.w = (uint32_t)__half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16);
            *reinterpret_cast<uint4 *>(yq + ((size_t)s * kpy + 4 * k4) * 2) = rec;
        }
        if (y) *reinterpret_cast<float4 *>(y + (size_t)s * ldy + 4 * k4) = make_float4(o[0], o[1], o[2], o[3]);
    }
}

inline int norm_threads(int D) {
    int t = (D / 4 + 3) / 4;  // at most 4 float4 per thread
    t = (t + 31) / 32 * 32;
    return t < 32 ? 32 : (t > kNormThreads ? kNormThreads : t);
}

// ---------------------------------------------------------------------------
// KV append + query rope (moonlight_kernels.metal:132-200).  One block per
// verify row: RMSNorm(latent) and RoPE(rope part) into the cache at
// position pos + s; RoPE of every head's rope slice into qcat.  RoPE takes
// interleaved pairs and writes the half-split order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void rope_pair(float first, float second, int p, int R, int position,
                                          float theta, float &out_a, float &out_b) {
    float angle = (float)position * powf(theta, -2.0f * (float)p / (float)R);
    float c = cosf(angle), sn = sinf(angle);
    out_a = first * c - second * sn;
    out_b = second * c + first * sn;
}

// grid (S, 1 + ceil(H * R/2 / blockDim)): block y == 0 appends the KV row,
// blocks y >= 1 rotate a slice of the heads' query rope pairs.
__device__ __forceinline__ void mla_prep_block(int bx, int by, const float *ckv, const float *q,
                                               const float *norm_w, int L, int R, int H, int nope, float eps,
                                               float theta, const Staging *st, PageMap pm, __half *cache,
                                               __half *qcat) {
    pdl_wait();
    pdl_release();
    __shared__ float scratch[32];
    const int s = bx;
    const int position = st->rowpos[s];
    const int half = R / 2;
    if (by == 0) {
        const float *src = ckv + (size_t)s * (L + R);
        float ss = 0.0f;
        for (int i = threadIdx.x; i < L; i += blockDim.x) ss += src[i] * src[i];
        ss = block_sum(ss, scratch);
        float scale = 1.0f / sqrtf(ss / (float)L + eps);
        __half *dst = cache + (size_t)kv_row(pm, st->rowseq[s], position) * (L + R);
        for (int i = threadIdx.x; i < L; i += blockDim.x)
            dst[i] = __float2half_rn(src[i] * scale * norm_w[i]);
        for (int p = threadIdx.x; p < half; p += blockDim.x) {
            float a, b;
            rope_pair(src[L + 2 * p], src[L + 2 * p + 1], p, R, position, theta, a, b);
            dst[L + p] = __float2half_rn(a);
            dst[L + half + p] = __float2half_rn(b);
        }
        return;
    }
    const int qw = nope + R;
    const int t = (by - 1) * blockDim.x + threadIdx.x;
    if (t >= H * half) return;
    const int h = t / half, p = t % half;
    const float *qh = q + ((size_t)s * H + h) * qw + nope;
    float a, b;
    rope_pair(qh[2 * p], qh[2 * p + 1], p, R, position, theta, a, b);
    __half *qo = qcat + ((size_t)s * H + h) * (L + R) + L;
    qo[p] = __float2half_rn(a);
    qo[half + p] = __float2half_rn(b);
}

// ---------------------------------------------------------------------------
// Query absorption (moonlight_kernels.metal:218-245):
//   qcat[s*H+h][l] = fp16( sum_n q[s][h][n] * W_kvb[h*(nope+v)+n][l] )
// grid (H, L/64), 256 threads: the W_UK block [nope][64] is dequantized into
// shared memory before waiting for the queries (weights are constant), then
// each output sums over n in fp32 sequentially without contraction (the
// oracle's order).
// ---------------------------------------------------------------------------
constexpr int kAbsorbCols = 64;
constexpr int kAbsorbMaxNope = 128;

__device__ __forceinline__ void mla_absorb_block(int bx, int by, int fmt, const uint8_t *w, int kp,
                                                 const float *q, int S, int H, int nope, int vdim, int R,
                                                 int L, __half *qcat) {
    __shared__ float wsm[kAbsorbMaxNope][kAbsorbCols + 1];
    __shared__ float qs[8][kAbsorbMaxNope];
    __shared__ __align__(16) uint8_t raw[kAbsorbMaxNope / kTileRows][1152];
    const int h = bx, l0 = by * kAbsorbCols;
    const int qw = nope + R;
    const int cc = chunk_cols(fmt), blk = block_bytes(fmt);
    const int c = l0 / cc, col0 = l0 % cc;
    const int tile0 = h * (nope + vdim) / kTileRows, ntiles = nope / kTileRows;
    const int nchunks = chunk_count(fmt, kp);
    // the W_UK rows of this head and this column chunk: ntiles contiguous blocks
    for (int i = threadIdx.x; i < ntiles * (blk / 16); i += blockDim.x) {
        int t = i / (blk / 16), v = i % (blk / 16);
        const uint4 *src = reinterpret_cast<const uint4 *>(
            w + ((size_t)(tile0 + t) * nchunks + c) * blk);
        reinterpret_cast<uint4 *>(raw[t])[v] = __ldg(src + v);
    }
    __syncthreads();
    // Record-wise decode: unit (row n, record j) holds columns 16 i + 4 j + b
    // (i, b < 4) of the 64-column half `sub` of the chunk (common.cuh
    // layout); every value is the exact fp32 product value x group scale.
    const int srb = scale_row_bytes(fmt), sub = col0 / 64;
    for (int u = threadIdx.x; u < nope * 4; u += blockDim.x) {
        const int n = u >> 2, j = u & 3, g = n % kTileRows;
        const uint8_t *b = raw[n / kTileRows];
        const uint4 rec = *reinterpret_cast<const uint4 *>(b + g * 64 + 16 * j);
        const uint8_t *sp = b + kBlockValueBytes + g * srb;
        float *dst = &wsm[n][4 * j];
        if (fmt == FC_FMT_Q8) {
            const uint32_t words[4] = {rec.x, rec.y, rec.z, rec.w};
            const float s0 = __half2float(reinterpret_cast<const __half *>(sp)[0]);
            const float s1 = __half2float(reinterpret_cast<const __half *>(sp)[1]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int bb = 0; bb < 4; ++bb)
                    dst[16 * i + bb] = (float)(int8_t)((words[i] >> (8 * bb)) & 0xFFu) * (i < 2 ? s0 : s1);
        } else {
            const uint32_t w0 = sub ? rec.z : rec.x, w1 = sub ? rec.w : rec.y;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int grp = 2 * sub + (i >> 1);
                float scale;
                if (fmt == FC_FMT_Q4) scale = __half2float(reinterpret_cast<const __half *>(sp)[grp]);
                else scale = e8m0_to_float(sp[grp]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t lo, hi;
                    if (fmt == FC_FMT_Q4) {
                        const uint32_t word = i < 2 ? w0 : w1, sh = 4 * (2 * (i & 1) + h);
                        lo = (word >> sh) & 15u;
                        hi = (word >> (sh + 16)) & 15u;
                    } else {
                        const uint32_t byte = ((i < 2 ? w0 : w1) >> (8 * (2 * (i & 1) + h))) & 0xFFu;
                        lo = byte & 15u;
                        hi = byte >> 4;
                    }
                    const uint32_t codes[2] = {lo, hi};
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const uint32_t code = codes[e];
                        float v;
                        if (fmt == FC_FMT_Q4) {
                            v = (float)((int)code - 8);
                        } else {
                            // e2m1 magnitude: 0, 0.5, 1, 1.5, 2, 3, 4, 6
                            const uint32_t ex = (code >> 1) & 3u, mb = code & 1u;
                            v = ex == 0 ? 0.5f * (float)mb : (float)(2u + mb) * (float)(1u << ex) * 0.25f;
                            if (code & 8) v = -v;
                        }
                        dst[16 * i + 2 * h + e] = v * scale;
                    }
                }
            }
        }
    }
    pdl_wait();
    pdl_release();
    for (int i = threadIdx.x; i < S * nope; i += blockDim.x) {
        int s = i / nope, n = i % nope;
        qs[s][n] = q[((size_t)s * H + h) * qw + n];
    }
    __syncthreads();
    for (int o = threadIdx.x; o < S * kAbsorbCols; o += blockDim.x) {
        int s = o / kAbsorbCols, col = o % kAbsorbCols;
        float acc = 0.0f;
        for (int n = 0; n < nope; ++n) acc = __fadd_rn(acc, __fmul_rn(qs[s][n], wsm[n][col]));
        qcat[((size_t)s * H + h) * (L + R) + l0 + col] = __float2half_rn(acc);
    }
}

// KV append + query rope (blocks 0 .. S * prep_y - 1) and query absorption
// (the remaining H * L / 64 blocks) in one launch: both read only the q_b and
// kv_a outputs, so neither waits for the other.
__global__ void __launch_bounds__(256)
mla_prep_absorb_kernel(const float *ckv, const float *q, const float *norm_w, int L, int R, int H, int nope,
                       float eps, float theta, const Staging *st, PageMap pm, __half *cache, __half *qcat, int S,
                       int prep_y, int fmt, const uint8_t *w, int kp, int vdim) {
    const int b = blockIdx.x, n_prep = S * prep_y;
    if (b < n_prep) {
        mla_prep_block(b / prep_y, b % prep_y, ckv, q, norm_w, L, R, H, nope, eps, theta, st, pm, cache, qcat);
    } else {
        const int a = b - n_prep, cols = L / kAbsorbCols;
        mla_absorb_block(a / cols, a % cols, fmt, w, kp, q, S, H, nope, vdim, R, L, qcat);
    }
}

// ---------------------------------------------------------------------------
// Flash-decoding attention on the tensor cores.
// ---------------------------------------------------------------------------
constexpr int kAttnQ = 32;       // query rows per CTA
constexpr int kAttnKeys = 64;    // keys per chunk
constexpr int kAttnThreads = 256;

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *p) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
    int bytes = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(a), "l"(gmem), "r"(bytes));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Shared-memory plan (bytes) for width DW = L + R and L.
struct AttnSmem {
    static __host__ __device__ constexpr int stride(int dw) { return dw + 8; }  // halves
    static __host__ __device__ constexpr size_t q_bytes(int dw) { return (size_t)kAttnQ * stride(dw) * 2; }
    static __host__ __device__ constexpr size_t k_bytes(int dw) { return (size_t)kAttnKeys * stride(dw) * 2; }
    static __host__ __device__ constexpr size_t p_bytes() { return (size_t)kAttnQ * (kAttnKeys + 8) * 2; }
    static __host__ __device__ constexpr size_t total(int dw) {
        return q_bytes(dw) + 2 * k_bytes(dw) + p_bytes() + (size_t)(4 * kAttnQ * 2 + 3 * kAttnQ) * 4;
    }
};

// grid (query tiles, splits).  Each split covers chunks [split*G, split*G+G).
// Writes unnormalized partial outputs part_o [split][q][L], part_m / part_l
// [split][q] (m = -inf, l = 0 when no key of the split is visible).
template <int L, int R>
__global__ void __launch_bounds__(kAttnThreads, 1)
mla_attention_kernel(const __half *cache, const __half *qcat, int S, int H, int chunks_per_split,
                     const Staging *st, PageMap pm, float softmax_scale, float *part_o, float *part_m,
                     float *part_l) {
    pdl_wait();
    pdl_release();
    constexpr int DW = L + R;
    constexpr int ST = DW + 8;        // smem row stride (halves)
    constexpr int PST = kAttnKeys + 8;
    constexpr int NCB = L / 4;        // O columns per warp (4 column blocks)
    constexpr int NT_O = NCB / 8;     // n8 tiles per warp in P.C
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __half *Qs = reinterpret_cast<__half *>(smem_raw);
    __half *Ks = Qs + kAttnQ * ST;                 // 2 buffers
    __half *Ps = Ks + 2 * kAttnKeys * ST;
    float *red_max = reinterpret_cast<float *>(Ps + kAttnQ * PST);  // [4][32]
    float *red_sum = red_max + 4 * kAttnQ;                          // [4][32]
    float *m_run = red_sum + 4 * kAttnQ;
    float *l_run = m_run + kAttnQ;
    float *alpha = l_run + kAttnQ;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, j = lane & 3;
    const int nq = S * H;
    const int q0 = blockIdx.x * kAttnQ;
    // the tile's rows belong to one sequence; keys up to its last row's position
    const int seq = st->rowseq[q0 / H];
    const int total_keys = st->rowpos[(min(q0 + kAttnQ, nq) - 1) / H] + 1;
    const int chunk0 = blockIdx.y * chunks_per_split;
    int chunk1 = chunk0 + chunks_per_split;
    const int last_chunk = (total_keys + kAttnKeys - 1) / kAttnKeys;
    if (chunk1 > last_chunk) chunk1 = last_chunk;

    // Load the query tile (rows beyond nq are zero).
    for (int i = tid; i < kAttnQ * (DW / 8); i += kAttnThreads) {
        int r = i / (DW / 8), c8 = i % (DW / 8);
        bool ok = q0 + r < nq;
        cp_async16(Qs + r * ST + c8 * 8, qcat + (size_t)(ok ? q0 + r : 0) * DW + c8 * 8, ok);
    }
    if (tid < kAttnQ) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
    }
    auto load_chunk = [&](int chunk, int buf) {
        __half *dst = Ks + buf * kAttnKeys * ST;
        int base = chunk * kAttnKeys;
        const __half *src = cache + (size_t)kv_row(pm, seq, base) * DW;  // one 64-row page
        // 16-byte pieces i = tid + n * threads of the [keys][DW/8] tile;
        // (row, column) advance incrementally instead of by division
        constexpr int kCols = DW / 8;
        constexpr int kStepR = kAttnThreads / kCols, kStepC = kAttnThreads % kCols;
        int r = tid / kCols, c8 = tid % kCols;
#pragma unroll 4
        for (int i = tid; i < kAttnKeys * kCols; i += kAttnThreads) {
            bool ok = base + r < total_keys;
            cp_async16(dst + r * ST + c8 * 8, src + (size_t)(ok ? r : 0) * DW + c8 * 8, ok);
            r += kStepR;
            c8 += kStepC;
            if (c8 >= kCols) { c8 -= kCols; ++r; }
        }
    };
    if (chunk0 < chunk1) load_chunk(chunk0, 0);
    cp_async_commit();

    const int mt = warp >> 2;        // m16 tile of the query rows
    const int kq = warp & 3;         // key quarter (16 keys) in S, column block in P.C
    float o_acc[NT_O][4];
#pragma unroll
    for (int t = 0; t < NT_O; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) o_acc[t][e] = 0.0f;

    // The visible-key limit of each of this thread's two query rows.
    int row_limit[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        int q = q0 + 16 * mt + g + 8 * h2;
        row_limit[h2] = q < nq ? st->rowpos[q / H] : -1;  // key <= limit is visible
    }

    for (int chunk = chunk0; chunk < chunk1; ++chunk) {
        int buf = (chunk - chunk0) & 1;
        if (chunk + 1 < chunk1) load_chunk(chunk + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const __half *Kb = Ks + buf * kAttnKeys * ST;

        // ---- scores: rows 16*mt.., keys 16*kq .. +16 (two n8 tiles) ----
        // Four independent accumulator sets over interleaved k-steps (short
        // MMA dependency chains), fragments for 4 k-steps loaded up front;
        // summed in a fixed order, so each row's result is unchanged by the
        // number of rows in the batch.
        static_assert(DW % 64 == 0, "score width must be a multiple of 64");
        float part[4][2][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) part[u][t][e] = 0.0f;
        const __half *ap0 = Qs + (16 * mt + (lane & 15)) * ST + 8 * (lane >> 4);
        const __half *bp0 = Kb + (16 * kq + (lane & 7) + 8 * (lane >> 4)) * ST + 8 * ((lane >> 3) & 1);
#pragma unroll 1
        for (int d = 0; d < DW; d += 64) {
            uint32_t a[4][4], b[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ldmatrix_x4(a[u], ap0 + d + 16 * u);
                ldmatrix_x4(b[u], bp0 + d + 16 * u);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                mma_f16(part[u][0], a[u], b[u][0], b[u][1], part[u][0]);
                mma_f16(part[u][1], a[u], b[u][2], b[u][3], part[u][1]);
            }
        }
        float sacc[2][4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e)
                sacc[t][e] = (part[0][t][e] + part[1][t][e]) + (part[2][t][e] + part[3][t][e]);
        // scale + mask; per-row chunk max within the warp
        float rmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                int key = chunk * kAttnKeys + 16 * kq + 8 * t + 2 * j + (e & 1);
                int h2 = e >> 1;
                float v = key <= row_limit[h2] ? sacc[t][e] * softmax_scale : -INFINITY;
                sacc[t][e] = v;
                rmax[h2] = fmaxf(rmax[h2], v);
            }
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            rmax[h2] = fmaxf(rmax[h2], __shfl_xor_sync(0xffffffffu, rmax[h2], 1));
            rmax[h2] = fmaxf(rmax[h2], __shfl_xor_sync(0xffffffffu, rmax[h2], 2));
        }
        if (j == 0) {
            red_max[kq * kAttnQ + 16 * mt + g] = rmax[0];
            red_max[kq * kAttnQ + 16 * mt + g + 8] = rmax[1];
        }
        __syncthreads();
        float m_new[2], rsum[2] = {0.0f, 0.0f};
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            int r = 16 * mt + g + 8 * h2;
            float cm = fmaxf(fmaxf(red_max[r], red_max[kAttnQ + r]),
                             fmaxf(red_max[2 * kAttnQ + r], red_max[3 * kAttnQ + r]));
            m_new[h2] = fmaxf(m_run[r], cm);
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                int h2 = e >> 1;
                p[e] = m_new[h2] == -INFINITY ? 0.0f : expf(sacc[t][e] - m_new[h2]);
                rsum[h2] += p[e];
            }
            int col = 16 * kq + 8 * t + 2 * j;
            int r0 = 16 * mt + g;
            *reinterpret_cast<uint32_t *>(Ps + r0 * PST + col) = pack_half2(p[0], p[1]);
            *reinterpret_cast<uint32_t *>(Ps + (r0 + 8) * PST + col) = pack_half2(p[2], p[3]);
        }
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            rsum[h2] += __shfl_xor_sync(0xffffffffu, rsum[h2], 1);
            rsum[h2] += __shfl_xor_sync(0xffffffffu, rsum[h2], 2);
        }
        if (j == 0) {
            red_sum[kq * kAttnQ + 16 * mt + g] = rsum[0];
            red_sum[kq * kAttnQ + 16 * mt + g + 8] = rsum[1];
        }
        __syncthreads();
        if (tid < kAttnQ) {
            float cm = fmaxf(fmaxf(red_max[tid], red_max[kAttnQ + tid]),
                             fmaxf(red_max[2 * kAttnQ + tid], red_max[3 * kAttnQ + tid]));
            float mo = m_run[tid];
            float mn = fmaxf(mo, cm);
            float a = (mn == -INFINITY) ? 1.0f : expf(mo - mn);
            float cs = red_sum[tid] + red_sum[kAttnQ + tid] + red_sum[2 * kAttnQ + tid] +
                       red_sum[3 * kAttnQ + tid];
            l_run[tid] = l_run[tid] * a + cs;
            m_run[tid] = mn;
            alpha[tid] = a;
        }
        __syncthreads();

        // ---- O += P . C over this chunk: rows 16*mt.., columns kq*NCB .. ----
        {
            float a0 = alpha[16 * mt + g], a1 = alpha[16 * mt + g + 8];
#pragma unroll
            for (int t = 0; t < NT_O; ++t) {
                o_acc[t][0] *= a0; o_acc[t][1] *= a0;
                o_acc[t][2] *= a1; o_acc[t][3] *= a1;
            }
        }
#pragma unroll
        for (int ks = 0; ks < kAttnKeys; ks += 16) {
            uint32_t a[4];
            ldmatrix_x4(a, Ps + (16 * mt + (lane & 15)) * PST + ks + 8 * (lane >> 4));
#pragma unroll
            for (int t = 0; t < NT_O; t += 2) {
                // B = C[key][l]: k = keys ks..ks+15, n = columns n0..n0+15 (two n8 tiles)
                int n0 = kq * NCB + 8 * t;
                uint32_t b[4];
                const __half *bp = Kb + (ks + (lane & 7) + 8 * ((lane >> 3) & 1)) * ST + n0 + 8 * (lane >> 4);
                ldmatrix_x4_trans(b, bp);
                mma_f16(o_acc[t], a, b[0], b[1], o_acc[t]);
                mma_f16(o_acc[t + 1], a, b[2], b[3], o_acc[t + 1]);
            }
        }
        __syncthreads();  // Ps / Kb reuse
    }
    cp_async_wait<0>();

    // ---- write partials ----
    const int split = blockIdx.y;
#pragma unroll
    for (int t = 0; t < NT_O; ++t) {
        int col = kq * NCB + 8 * t + 2 * j;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            int q = q0 + 16 * mt + g + 8 * h2;
            if (q < nq) {
                float2 v = make_float2(o_acc[t][2 * h2], o_acc[t][2 * h2 + 1]);
                *reinterpret_cast<float2 *>(part_o + ((size_t)split * nq + q) * L + col) = v;
            }
        }
    }
    __syncthreads();
    if (tid < kAttnQ && q0 + tid < nq) {
        part_m[(size_t)split * nq + q0 + tid] = m_run[tid];
        part_l[(size_t)split * nq + q0 + tid] = l_run[tid];
    }
}

// Combines the split partials in split order and writes the latent context of
// each (row s, head h) in xq format at ctx_xq + h * head_stride + s * L * 2.
// grid (S*H, L/128), 128 threads.  Splits with no visible key (m = -inf)
// contribute nothing, so a verify row and a decode of the same token see the
// same sequence of terms.
constexpr int kCombineThreads = 128;
constexpr int kMaxSplits = 1024;

template <int NS>
__device__ __forceinline__ void combine_row(const float *part_o, const float *part_m, const float *part_l,
                                            int splits, int nq, int q, int L, int l, float *wts, float *red,
                                            float &out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // the partial outputs of every split, loaded together
    float o[NS > 0 ? NS : 1];
#pragma unroll
    for (int i = 0; i < NS; ++i)
        o[i] = (i < splits && l < L) ? __ldcg(part_o + ((size_t)i * nq + q) * L + l) : 0.0f;
    float m = -INFINITY, mi = -INFINITY, li = 0.0f;
    for (int i = threadIdx.x; i < splits; i += kCombineThreads) {
        mi = __ldcg(part_m + (size_t)i * nq + q);
        li = __ldcg(part_l + (size_t)i * nq + q);
        m = fmaxf(m, mi);
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float M = red[0];
    for (int w = 1; w < kCombineThreads / 32; ++w) M = fmaxf(M, red[w]);
    __syncthreads();
    float den = 0.0f;
    if (splits <= kCombineThreads) {
        if (threadIdx.x < splits) {
            float wi = mi == -INFINITY ? 0.0f : expf(mi - M);
            wts[threadIdx.x] = wi;
            if (wi != 0.0f) den = wi * li;
        }
    } else {
        for (int i = threadIdx.x; i < splits; i += kCombineThreads) {
            float mj = __ldcg(part_m + (size_t)i * nq + q);
            float wi = mj == -INFINITY ? 0.0f : expf(mj - M);
            wts[i] = wi;
            if (wi != 0.0f) den += wi * __ldcg(part_l + (size_t)i * nq + q);
        }
    }
    den = warp_sum(den);
    if (lane == 0) red[warp] = den;
    __syncthreads();
    den = 0.0f;
    for (int w = 0; w < kCombineThreads / 32; ++w) den += red[w];
    float acc = 0.0f;
    if (NS > 0) {
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            float wi = i < splits ? wts[i] : 0.0f;
            if (wi != 0.0f) acc += wi * o[i];
        }
    } else {
        for (int i = 0; i < splits; ++i) {
            float wi = wts[i];
            if (wi != 0.0f) acc += wi * __ldcg(part_o + ((size_t)i * nq + q) * L + l);
        }
    }
    out = acc / den;
}

__global__ void __launch_bounds__(kCombineThreads)
mla_combine_kernel(const float *part_o, const float *part_m, const float *part_l, int splits, int S,
                   int H, int L, int ml_cols, __half *ctx_xq, size_t head_stride) {
    pdl_wait();
    pdl_release();
    __shared__ float wts[kMaxSplits];
    __shared__ float red[kCombineThreads / 32];
    const int q = blockIdx.x, nq = S * H;
    const int l = blockIdx.y * kCombineThreads + threadIdx.x;
    // every ml_cols output columns (a multiple of the block width) have their
    // own max / sum partials [group][split][q]
    const size_t grp = (size_t)(blockIdx.y * kCombineThreads / ml_cols) * splits * nq;
    part_m += grp;
    part_l += grp;
    float v;
    if (splits <= 16) combine_row<16>(part_o, part_m, part_l, splits, nq, q, L, l, wts, red, v);
    else if (splits <= 32) combine_row<32>(part_o, part_m, part_l, splits, nq, q, L, l, wts, red, v);
    else if (splits <= 64) combine_row<64>(part_o, part_m, part_l, splits, nq, q, L, l, wts, red, v);
    else combine_row<0>(part_o, part_m, part_l, splits, nq, q, L, l, wts, red, v);
    if (l >= L) return;
    const int s = q / H, h = q % H;
    store_xq(ctx_xq + (size_t)h * head_stride, L, s, l, v);
}

}  // namespace fc
