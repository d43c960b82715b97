/*
 * floyd_fm.h - floyd's single-matmul offload surface on the B200, with the
 * reference's own entry-point names so that floyd's engine links against
 * libfloyd_cuda.so in place of its Metal backend.
 *
 * Each declaration replaces the one of backend_metal.h (line given) with the
 * same arguments and meaning.  Host arrays in, host arrays out; the device
 * work is synchronous.  There is no CPU fallback: a call that cannot run on
 * the GPU fails (returns 0, or leaves y untouched for the void calls).
 */
#ifndef FLOYD_FM_H
#define FLOYD_FM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 1 = a B200 (sm_100a) device is ready, 0 = none.  backend_metal.h:14-16 */
int fm_init(void);
/* Name of the device fm_init selected.  backend_metal.h:17 */
const char *fm_device_name(void);

/* y[S][O] = x[S][I] . w[O][I]^T with one fp32 scale per row s[O]; int8
 * values, or int4 packed two per byte (low nibble first, value = nibble - 8,
 * ceil(I/2) bytes per row).  cache = 1 keeps the device copy of w (and s)
 * by host pointer for later calls (stable, model-resident tensors); cache =
 * 0 copies them for this call only.  backend_metal.h:19-33 */
void fm_matmul_q8(float *y, const float *x, const int8_t *w, const float *s,
                  int O, int I, int S, int cache);
void fm_matmul_q4(float *y, const float *x, const uint8_t *w, const float *s,
                  int O, int I, int S, int cache);

/* DeepSeek V4 FP8: E4M3 values [O][I] with one E8M0 scale per 128 x 128
 * block, s[(O/128)][(I/128)]; block_size must be 128, O and I multiples of
 * 128.  Returns 1 on success.  backend_metal.h:35-38 */
int fm_matmul_deepseek_v4_fp8(float *y, const float *x, const uint8_t *w,
                              const uint8_t *s, int O, int I, int S,
                              int block_size);
/* DeepSeek V4 FP4: E2M1 codes [O][I/2] (even element low) with one E8M0
 * scale per 32 columns, s[O][I/32]; I a multiple of 32.
 * backend_metal.h:39-40 */
int fm_matmul_deepseek_v4_fp4(float *y, const float *x, const uint8_t *w,
                              const uint8_t *s, int O, int I, int S);

#ifdef __cplusplus
}
#endif

#endif
