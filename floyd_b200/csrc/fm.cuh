// fm.cuh - floyd's single-matmul offload surface (backend_metal.h:14-42) on
// the B200: fm_init, fm_device_name, fm_matmul_q8 / _q4 with one fp32 scale
// per output row and the pointer-keyed resident-weight cache, and the native
// DeepSeek V4 formats fm_matmul_deepseek_v4_fp8 (E4M3 values, one E8M0
// scale per 128 x 128 block) and _fp4 (E2M1 codes, one E8M0 per 32).
//
// q8 / q4 (kernels.metal:4-39): y[s][o] = (sum_i w[o][i] * x[s][i]) * s[o].
// The weights go into the tile-major image of the GEMV with unit group
// scales (exact in fp16), the fp32 row scale multiplies the finished dot
// product (fm_row_scale_kernel), so the result is the reference's up to
// fp32 summation order.  Any input width works: rows are padded to the
// GEMV's 32-column groups with zeros (int4 padding nibble 8 = value 0).
//
// cache = 1 (backend_metal.m:14-72): the device image of `w` (and the row
// scales `s`) is looked up by host pointer and built only on the first
// call; the caller promises that the pointer names the same tensor for its
// whole life (a hit does not compare contents).  cache = 0 builds a
// transient image for this call only, for host buffers whose contents are
// recycled.  The cache is shared by all threads (a mutex guards it).
#pragma once

#include <cuda_fp8.h>

#include <mutex>

namespace {

struct FmEntry {
    uint8_t *image = nullptr;  // tile-major values + unit scales
    int fmt = 0, O = 0, I = 0;
};

struct FmState {
    std::mutex mu;
    int device = -1;
    std::string name = "(none)";
    int sms = 148;
    std::map<std::pair<const void *, int>, FmEntry> weights;
    std::map<const void *, std::pair<float *, int>> scales;
};

FmState &fm_state() {
    static FmState st;
    return st;
}

__global__ void fm_row_scale_kernel(float *y, const float *scale, int O, int S) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)O * S) y[i] *= scale[i % O];
}

// Host image of an int8 [O][I] or int4 [O][ceil(I/2)] matrix (per-row
// layout of kernels.metal) with unit group scales, I padded to K32.
std::vector<uint8_t> fm_image(int fmt, const void *w, int O, int I, DevMat &mm) {
    const int K = (I + 31) / 32 * 32;
    plan_mat(mm, fmt, O, K, 1, 0, 0);
    std::vector<uint8_t> logical;
    if (fmt == FC_FMT_Q8) {
        logical.assign((size_t)O * K, 0);
        for (int o = 0; o < O; ++o)
            memcpy(&logical[(size_t)o * K], reinterpret_cast<const uint8_t *>(w) + (size_t)o * I, I);
    } else {
        const int rb = (I + 1) / 2;
        logical.assign((size_t)O * K / 2, 0x88);  // nibble 8 = value 0
        for (int o = 0; o < O; ++o) {
            const uint8_t *src = reinterpret_cast<const uint8_t *>(w) + (size_t)o * rb;
            uint8_t *dst = &logical[(size_t)o * K / 2];
            memcpy(dst, src, I / 2);
            if (I & 1) dst[I / 2] = (uint8_t)((src[I / 2] & 0x0F) | 0x80);
        }
    }
    std::vector<uint8_t> image(mm.w_bytes, 0);
    pack_values(mm, logical.data(), image.data());
    std::vector<uint16_t> unit((size_t)O * (K / 32), 0x3C00);  // fp16 1.0
    pack_scales(mm, reinterpret_cast<const uint8_t *>(unit.data()), image.data());
    return image;
}

int fm_ready() {
    FmState &st = fm_state();
    if (st.device >= 0) return 1;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess || prop.major < 10) return 0;
    if (gemv_prepare_all() != cudaSuccess) return 0;
    st.device = dev;
    st.name = prop.name;
    st.sms = prop.multiProcessorCount;
    return 1;
}

// q8 / q4 with per-row scales; S rows in passes of up to 8 through the GEMV.
int fm_rowscale_matmul(int fmt, float *y, const float *x, const void *w, const float *s, int O, int I, int S,
                       int cache) {
    if (!y || !x || !w || !s || O <= 0 || I <= 0 || S <= 0) return 0;
    FmState &st = fm_state();
    std::lock_guard<std::mutex> lock(st.mu);
    if (!fm_ready()) return 0;
    cudaSetDevice(st.device);
    DevMat mm;
    const uint8_t *image = nullptr;
    uint8_t *transient = nullptr;
    float *dscale = nullptr, *tscale = nullptr;
    const int K = (I + 31) / 32 * 32;
    if (cache) {
        auto key = std::make_pair((const void *)w, fmt);
        auto it = st.weights.find(key);
        if (it != st.weights.end() && it->second.O == O && it->second.I == I) {
            plan_mat(mm, fmt, O, K, 1, 0, 0);
            image = it->second.image;
        } else {
            std::vector<uint8_t> img = fm_image(fmt, w, O, I, mm);
            uint8_t *d = nullptr;
            if (cudaMalloc(&d, img.size()) != cudaSuccess) return 0;
            cudaMemcpy(d, img.data(), img.size(), cudaMemcpyHostToDevice);
            if (it != st.weights.end()) cudaFree(it->second.image);
            st.weights[key] = FmEntry{d, fmt, O, I};
            image = d;
        }
        auto sit = st.scales.find(s);
        if (sit != st.scales.end() && sit->second.second == O) {
            dscale = sit->second.first;
        } else {
            if (cudaMalloc(&dscale, (size_t)O * 4) != cudaSuccess) return 0;
            cudaMemcpy(dscale, s, (size_t)O * 4, cudaMemcpyHostToDevice);
            if (sit != st.scales.end()) cudaFree(sit->second.first);
            st.scales[s] = std::make_pair(dscale, O);
        }
    } else {
        std::vector<uint8_t> img = fm_image(fmt, w, O, I, mm);
        if (cudaMalloc(&transient, img.size()) != cudaSuccess) return 0;
        cudaMemcpy(transient, img.data(), img.size(), cudaMemcpyHostToDevice);
        image = transient;
        if (cudaMalloc(&tscale, (size_t)O * 4) != cudaSuccess) {
            cudaFree(transient);
            return 0;
        }
        cudaMemcpy(tscale, s, (size_t)O * 4, cudaMemcpyHostToDevice);
        dscale = tscale;
    }
    const int chunk = 8;
    float *dx = nullptr, *dy = nullptr;
    __half *dxq = nullptr;
    int *derr = nullptr;
    cudaError_t e = cudaMalloc(&dx, (size_t)chunk * K * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dy, (size_t)chunk * O * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dxq, (size_t)chunk * mm.kp * 4);
    if (e == cudaSuccess) e = cudaMalloc(&derr, 4);
    if (e == cudaSuccess) e = cudaMemset(derr, 0, 4);
    std::vector<float> xpad((size_t)chunk * K, 0.0f);
    for (int r0 = 0; r0 < S && e == cudaSuccess; r0 += chunk) {
        const int r = std::min(chunk, S - r0);
        for (int i = 0; i < r; ++i) memcpy(&xpad[(size_t)i * K], x + (size_t)(r0 + i) * I, (size_t)I * 4);
        e = cudaMemcpy(dx, xpad.data(), (size_t)r * K * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(dxq, 0, (size_t)r * mm.kp * 4);
        if (e != cudaSuccess) break;
        to_xq_kernel<<<(r * K + 255) / 256, 256>>>(dx, r, K, mm.kp, dxq);
        GemvSeg g = seg_of(mm, dxq, EPI_STORE);
        g.w = image;
        g.y = dy;
        g.ldy = O;
        e = gemv1(fmt, g, r, 0.0f, derr, st.sms, 0);
        if (e == cudaSuccess) {
            fm_row_scale_kernel<<<(unsigned)(((size_t)O * r + 255) / 256), 256>>>(dy, dscale, O, r);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpy(y + (size_t)r0 * O, dy, (size_t)r * O * 4, cudaMemcpyDeviceToHost);
    }
    int herr = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
    cudaFree(dx); cudaFree(dy); cudaFree(dxq); cudaFree(derr);
    cudaFree(transient); cudaFree(tscale);
    return e == cudaSuccess && !herr;
}

// E4M3 weights [O][I] with one E8M0 scale per 128 x 128 block
// (kernels.metal:41-75, deepseek_v4_quant.h:141-178): one warp per output
// row, 16 codes per lane per step decoded with the hardware fp8 -> fp16x2
// conversion; each 128-column block's dot product is formed in fp32 and
// scaled once.  Scale code 255 and the E4M3 NaN codes give NaN, as there.
constexpr int kFp8Threads = 256;

__device__ __forceinline__ float fm_e8m0(uint8_t code) {
    return code == 255 ? __int_as_float(0x7fc00000) : e8m0_to_float(code);
}

__global__ void __launch_bounds__(kFp8Threads) fm_fp8_kernel(const uint8_t *w, const uint8_t *sc, const float *x,
                                                             float *y, int O, int I, int S) {
    extern __shared__ float xs[];  // [S][I]
    for (int i = threadIdx.x; i < S * I; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int blocks = I / 128;
    for (int o = blockIdx.x * warps + (threadIdx.x >> 5); o < O; o += gridDim.x * warps) {
        const uint8_t *row = w + (size_t)o * I;
        const uint8_t *srow = sc + (size_t)(o / 128) * blocks;
        for (int s0 = 0; s0 < S; s0 += 4) {
            float tot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int b = 0; b < blocks; ++b) {
                // lane covers 4 codes of the block's 128
                const uint32_t codes = *reinterpret_cast<const uint32_t *>(row + b * 128 + 4 * lane);
                __half2_raw h01 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(codes & 0xFFFF), __NV_E4M3);
                __half2_raw h23 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(codes >> 16), __NV_E4M3);
                const float2 f01 = __half22float2(*reinterpret_cast<__half2 *>(&h01));
                const float2 f23 = __half22float2(*reinterpret_cast<__half2 *>(&h23));
                const float bs = fm_e8m0(srow[b]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int s = s0 + j;
                    if (s >= S) break;
                    const float *xr = xs + (size_t)s * I + b * 128 + 4 * lane;
                    float p = f01.x * xr[0];
                    p = fmaf(f01.y, xr[1], p);
                    p = fmaf(f23.x, xr[2], p);
                    p = fmaf(f23.y, xr[3], p);
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) p += __shfl_xor_sync(0xffffffffu, p, off);
                    tot[j] = fmaf(p, bs, tot[j]);
                }
            }
            if (lane == 0)
                for (int j = 0; j < 4 && s0 + j < S; ++j) y[(size_t)(s0 + j) * O + o] = tot[j];
        }
    }
}

}  // namespace

extern "C" {

int fm_init(void) {
    FmState &st = fm_state();
    std::lock_guard<std::mutex> lock(st.mu);
    return fm_ready();
}

const char *fm_device_name(void) { return fm_state().name.c_str(); }

void fm_matmul_q8(float *y, const float *x, const int8_t *w, const float *s, int O, int I, int S, int cache) {
    fm_rowscale_matmul(FC_FMT_Q8, y, x, w, s, O, I, S, cache);
}

void fm_matmul_q4(float *y, const float *x, const uint8_t *w, const float *s, int O, int I, int S, int cache) {
    fm_rowscale_matmul(FC_FMT_Q4, y, x, w, s, O, I, S, cache);
}

int fm_matmul_deepseek_v4_fp8(float *y, const float *x, const uint8_t *w, const uint8_t *s, int O, int I, int S,
                              int block_size) {
    if (block_size != 128 || O <= 0 || I <= 0 || O % 128 || I % 128 || S <= 0 || !y || !x || !w || !s) return 0;
    FmState &st = fm_state();
    std::lock_guard<std::mutex> lock(st.mu);
    if (!fm_ready()) return 0;
    cudaSetDevice(st.device);
    const int rows = std::min(S, 8);  // activation rows per launch (shared memory)
    const size_t wbytes = (size_t)O * I, sbytes = (size_t)(O / 128) * (I / 128);
    uint8_t *dw = nullptr, *ds = nullptr;
    float *dx = nullptr, *dy = nullptr;
    cudaError_t e = cudaMalloc(&dw, wbytes);
    if (e == cudaSuccess) e = cudaMalloc(&ds, sbytes);
    if (e == cudaSuccess) e = cudaMalloc(&dx, (size_t)rows * I * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dy, (size_t)rows * O * 4);
    if (e == cudaSuccess) e = cudaMemcpy(dw, w, wbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(ds, s, sbytes, cudaMemcpyHostToDevice);
    const size_t smem = (size_t)rows * I * 4;
    if (e == cudaSuccess && smem > 48 * 1024)
        e = cudaFuncSetAttribute(fm_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && smem > 227 * 1024) e = cudaErrorInvalidValue;
    for (int r0 = 0; r0 < S && e == cudaSuccess; r0 += rows) {
        const int r = std::min(rows, S - r0);
        e = cudaMemcpy(dx, x + (size_t)r0 * I, (size_t)r * I * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) break;
        const int grid = std::min((O + 7) / 8, st.sms * 4);
        fm_fp8_kernel<<<grid, kFp8Threads, (size_t)r * I * 4>>>(dw, ds, dx, dy, O, I, r);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpy(y + (size_t)r0 * O, dy, (size_t)r * O * 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(dw); cudaFree(ds); cudaFree(dx); cudaFree(dy);
    return e == cudaSuccess;
}

int fm_matmul_deepseek_v4_fp4(float *y, const float *x, const uint8_t *w, const uint8_t *s, int O, int I, int S) {
    if (I % 32 || O <= 0 || S <= 0) return 0;
    {
        FmState &st = fm_state();
        std::lock_guard<std::mutex> lock(st.mu);
        if (!fm_ready()) return 0;
    }
    char err[256];
    // E2M1 codes two per byte (even element low) with one E8M0 per 32: the
    // MXFP4 format of fc_matmul
    for (int r0 = 0; r0 < S; r0 += 8) {
        const int r = std::min(8, S - r0);
        if (!fc_matmul(FC_FMT_MXFP4, y + (size_t)r0 * O, x + (size_t)r0 * I, w, s, O, I, r, err, sizeof err))
            return 0;
    }
    return 1;
}

}  // extern "C"
