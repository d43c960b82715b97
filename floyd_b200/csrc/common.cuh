// common.cuh - device helpers shared by the sm_100a kernels of the verify
// step: tensor-core MMA wrappers, exact int8 / int4 / e2m1 -> fp16 dequant,
// the hi/lo fp16 activation format, warp reductions and error checks.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/floyd_cuda.h"
#include "../../include/floyd_synth.h"

namespace fc {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// Activation operand format ("xq").  A row of K activations is stored as K/4
// 16-byte records {hi[4], lo[4]} of fp16 with x = hi + lo exactly to about
// 22 bits (hi = fp16(x), lo = fp16(x - hi)).  Record r holds k = 4r .. 4r+3,
// which is exactly the B fragment one thread needs for one m16n8k16 MMA.
// Values must satisfy |x| < 65504; the producers saturate.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_hi_lo(float x, __half &hi, __half &lo) {
    x = fminf(fmaxf(x, -65504.0f), 65504.0f);
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

// Writes x at (row s, column k) of an xq buffer with row length kp.
__device__ __forceinline__ void store_xq(__half *xq, int kp, int s, int k, float x) {
    __half hi, lo;
    split_hi_lo(x, hi, lo);
    __half *rec = xq + ((size_t)s * kp + (k & ~3)) * 2;
    rec[k & 3] = hi;
    rec[4 + (k & 3)] = lo;
}

// ---------------------------------------------------------------------------
// Tensor-core MMA m16n8k16, fp16 inputs, fp32 accumulate.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4],
                                        uint32_t b0, uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// ---------------------------------------------------------------------------
// Streaming loads (weights are read once per step: skip L1).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ uint2 ldg_v2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ldg_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}

// int8 x4 (one 32-bit word) -> two fp16x2 registers, exact:
// fp16(1024 + (v ^ 0x80)) - 1152 = v.  lo = bytes {0,1}, hi = bytes {2,3}.
__device__ __forceinline__ void dequant_q8_word(uint32_t w, uint32_t &lo, uint32_t &hi) {
    uint32_t u = w ^ 0x80808080u;
    lo = hsub2_bits(prmt(u, 0x64646464u, 0x5140u), 0x64806480u);
    hi = hsub2_bits(prmt(u, 0x64646464u, 0x7362u), 0x64806480u);
}

// int4 pair at nibble offset `shift` and shift+16 -> fp16x2 (nibble - 8), exact.
__device__ __forceinline__ uint32_t dequant_q4_pair(uint32_t w, int shift) {
    uint32_t t = ((w >> shift) & 0x000F000Fu) | 0x64006400u;
    return hsub2_bits(t, 0x64086408u);
}

// One 32-bit word of 4 bytes of e2m1 code pairs -> 4 fp16x2 registers with
// Blackwell's hardware conversion (exact: every e2m1 value is an fp16);
// register b holds (low nibble, high nibble) of byte b.
__device__ __forceinline__ void dequant_e2m1_word(uint32_t w, uint32_t (&out)[4]) {
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
        " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}\n"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
        : "r"(w));
}

__device__ __forceinline__ float e8m0_to_float(uint32_t code) {
    if (code == 255u) return __int_as_float(0x7FC00000);
    if (code == 0u) return __int_as_float(0x00400000);  // 2^-127, subnormal
    return __int_as_float((int)(code << 23));
}

// Four ue8m0 scale bytes -> fp32 powers of two without branches: code << 23
// (an integer multiply, issued on the FMA pipe) is the fp32 pattern of
// 2^(code - 127) for 1 <= code <= 254; an integer max maps code 0 to the
// subnormal 2^-127 exactly.  Code 255 (NaN in the format) becomes +inf, which
// is equally non-finite in every product.
__device__ __forceinline__ void e8m0x4_to_float(uint32_t s4, float (&out)[4]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t bits = ((s4 >> (8 * q)) & 0xFFu) * 8388608u;
        out[q] = __uint_as_float(max(bits, 0x00400000u));
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ---------------------------------------------------------------------------
// Device weight layout of a quantized matrix [O][K] ("tile-major"):
//   - rows are grouped in 16-row tiles (O padded up to a multiple of 16);
//   - K is cut in chunks of chunk_cols columns (64 for Q8, 128 for Q4 /
//     MXFP4), i.e. 64 bytes of values per row and chunk (K padded up to a
//     whole number of 128 columns);
//   - a tile is a sequence of chunk blocks, and a chunk block is
//       [16 rows x 64 value bytes][16 rows x scale_row_bytes group scales]
//     so one tile is contiguous and one block is what a warp consumes for
//     one chunk (1088 / 1152 bytes, a multiple of 16 for bulk copies);
//   - inside a row's 64 value bytes the columns are permuted so that the
//     16 bytes thread j of a warp loads feed whole m16n8k16 MMAs and every
//     MMA covers a single 32-column scale group:
//       q8:   column r (0..63): MMA i = r/16, thread j = (r%16)/4, b = r%4
//             byte = 16j + 4i + b
//       q4:   column r (0..127): MMA i = r/16, j = (r%16)/4, b = r%4,
//             h = b/2, e = b%2; register q = 2i + h; word = q/4;
//             nibble slot = q%4 + 4e; byte = 16j + 4*word + slot/2,
//             nibble = slot%2   (shift-and-mask decode, two values a word
//             apart land in one fp16x2 register)
//       e2m1: same i, j, h, e; byte = 16j + q, nibble = e, so each byte is
//             exactly one fp16x2 A register for cvt.rn.f16x2.e2m1x2
// ---------------------------------------------------------------------------
constexpr int kTileRows = 16;
constexpr int kBlockValueBytes = kTileRows * 64;

__host__ __device__ constexpr int chunk_cols(int fmt) { return fmt == FC_FMT_Q8 ? 64 : 128; }
__host__ __device__ constexpr int groups_per_chunk(int fmt) { return fmt == FC_FMT_Q8 ? 2 : 4; }
__host__ __device__ constexpr int scale_elem_bytes(int fmt) { return fmt == FC_FMT_MXFP4 ? 1 : 2; }
__host__ __device__ constexpr int scale_row_bytes(int fmt) {
    return groups_per_chunk(fmt) * scale_elem_bytes(fmt);
}
__host__ __device__ constexpr int block_bytes(int fmt) {
    return kBlockValueBytes + kTileRows * scale_row_bytes(fmt);
}
__host__ __device__ inline int pad_cols(int k) { return (k + 127) / 128 * 128; }
__host__ __device__ inline int chunk_count(int fmt, int kp) { return kp / chunk_cols(fmt); }
__host__ __device__ inline size_t tile_bytes(int fmt, int kp) {
    return (size_t)chunk_count(fmt, kp) * block_bytes(fmt);
}
__host__ __device__ inline size_t matrix_bytes(int fmt, int O, int kp) {
    return (size_t)((O + kTileRows - 1) / kTileRows) * tile_bytes(fmt, kp);
}

// Byte (and nibble) of column r (0 <= r < chunk_cols) inside a row's 64
// value bytes of a chunk.
__host__ __device__ inline void inner_position(int fmt, int r, int &byte, int &nibble) {
    if (fmt == FC_FMT_Q8) {
        byte = 16 * ((r & 15) >> 2) + 4 * (r >> 4) + (r & 3);
        nibble = 0;
        return;
    }
    int i = r >> 4, j = (r & 15) >> 2, b = r & 3;
    int q = 2 * i + (b >> 1), e = b & 1;
    if (fmt == FC_FMT_MXFP4) {
        byte = 16 * j + q;
        nibble = e;
        return;
    }
    int word = q >> 2;
    int slot = (q & 3) + 4 * e;
    byte = 16 * j + 4 * word + (slot >> 1);
    nibble = slot & 1;
}

// Offset of the value byte holding element (o, k) of a matrix with padded
// width kp; *nibble selects the half-byte for Q4 / MXFP4.
__host__ __device__ inline size_t value_offset(int fmt, int kp, int o, int k, int *nibble) {
    int cc = chunk_cols(fmt);
    int byte, nib;
    inner_position(fmt, k % cc, byte, nib);
    if (nibble) *nibble = nib;
    size_t blk = (size_t)(o / kTileRows) * chunk_count(fmt, kp) + (size_t)(k / cc);
    return blk * block_bytes(fmt) + (size_t)(o % kTileRows) * 64 + byte;
}

// Offset of the scale of group `grp` (32 columns) of row o.
__host__ __device__ inline size_t scale_offset(int fmt, int kp, int o, int grp) {
    int gpc = groups_per_chunk(fmt);
    size_t blk = (size_t)(o / kTileRows) * chunk_count(fmt, kp) + (size_t)(grp / gpc);
    return blk * block_bytes(fmt) + kBlockValueBytes + (size_t)(o % kTileRows) * scale_row_bytes(fmt) +
           (size_t)(grp % gpc) * scale_elem_bytes(fmt);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Kernels of the forward are launched with
// programmatic stream serialization: a kernel may start while its
// predecessor drains, waits (griddepcontrol.wait) before it reads anything
// the predecessor wrote, and releases its own dependents at once.  Without
// the launch attribute both instructions are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_release() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA 1-D) helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` with an iteration limit; on timeout
// records error bit 1 in *err and returns false (the caller carries on; the
// host reports the error after the pass).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err) {
    for (uint32_t it = 0; it < (1u << 20); ++it)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicOr(err, 1);
    return false;
}

// Global -> shared bulk copy completing on `bar` (16-byte aligned, size a
// multiple of 16).  A plain (non-multicast) copy of this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Host: launches `kernel` with programmatic stream serialization allowed.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace fc

#define FC_CUDA_OK(expr) ((expr) == cudaSuccess)
