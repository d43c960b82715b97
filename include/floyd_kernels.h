/*
 * floyd_kernels.h - single-kernel entry points of the B200 backend, for
 * callers that offload one operation at a time (floyd's backend_metal.h
 * surface) and for per-kernel parity tests.
 *
 * These take HOST arrays, copy them to the device, run the same sm_100a
 * kernel the session path uses, and copy the result back.
 */
#ifndef FLOYD_KERNELS_H
#define FLOYD_KERNELS_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[s][o] = sum_k x[s][k] * dequant(w[o][k]) for s < S, fp32 accumulation.
 * `format` is an FcFormat (Q8, Q4 or MXFP4); `values` / `scales` are in the
 * logical layout of fc_model_set_tensor (int8 [O][K] or packed nibbles
 * [O][K/2], fp16 / ue8m0 group scales [O][K/32]).  K % 32 == 0, S >= 1.
 * S <= 8 runs the GEMV (fp32-exact activations as hi/lo fp16 pairs);
 * S > 8 runs the prefill GEMM on the tcgen05 tensor cores (activations and
 * dequantized weights rounded to fp16 once, fp32 accumulation) and needs
 * O % 32 == 0.
 * Replaces fm_matmul_q8 / fm_matmul_q4 (backend_metal.h:18-33) and the Metal
 * offload of deepseek_v4_fp4_matmul_f32 (deepseek_v4_quant.h:103-139). */
int fc_matmul(int format, float *y, const float *x, const void *values,
              const void *scales, int O, int K, int S, char *error,
              size_t error_size);

/* fc_matmul without any device allocation.  For callers that cannot call
 * cudaMalloc at all - code running under a caching allocator that owns all
 * free device memory, an embedding host whose memory policy forbids driver
 * allocations, or a path that must not fail on out-of-memory.  Same arguments
 * and result as fc_matmul for S <= 8 rows, the GEMV path (no counterpart in
 * the reference; wider inputs are rejected, fc_matmul takes them).  Its
 * working memory is one fixed device array of about 14 MiB that every GPU
 * loading this library keeps until exit, so it accepts only: weight image
 * (tile-major values + scales) <= 6 MiB, packed values <= 6 MiB,
 * S*K*4 <= 256 KiB, S*O*4 <= 512 KiB; larger shapes are rejected with an
 * error.  The array becomes resident when the library's device code is
 * loaded on a device, which under CUDA's lazy module loading may be this
 * entry point's first call: make that first call (or any other call of this
 * library on that device) before the host's allocator claims the free device
 * memory, and before any stream capture on that device, since it also looks
 * up the array's device address.  All calls share the array: calls that
 * overlap on the GPU (from several host threads) race and must not. */
int fc_matmul_noalloc(int format, float *y, const float *x, const void *values,
                      const void *scales, int O, int K, int S, char *error,
                      size_t error_size);

#ifdef __cplusplus
}
#endif

#endif
