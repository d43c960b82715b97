/*
 * test_fm_cuda.c - floyd's offload-backend test (tests/test_backend_metal.c)
 * against the B200 backend's fm_* entry points (include/floyd_fm.h), plus
 * the two DeepSeek V4 formats checked against an f64 dequantized reference.
 *
 * Same cases and bound as the Metal test: O = 128, I = 257 (odd: the int4
 * tail), S = 4; q8 twice through the transient path (cache = 0), q4 twice
 * through the pointer-keyed cache (cache = 1) with new activations the
 * second time; max relative error against f64 below 1e-3.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "floyd_fm.h"

static float frand(void) { return (float)rand() / RAND_MAX * 2.f - 1.f; }

static double maxrel_q(const float *y, const void *w, int q4, const float *s, const float *x, int O, int I,
                       int S) {
    double m = 0;
    int rb = (I + 1) / 2;
    for (int t = 0; t < S; ++t)
        for (int o = 0; o < O; ++o) {
            double ref = 0;
            for (int i = 0; i < I; ++i) {
                int v;
                if (q4) {
                    uint8_t b = ((const uint8_t *)w)[(size_t)o * rb + (i >> 1)];
                    v = (i & 1) ? (b >> 4) - 8 : (b & 15) - 8;
                } else {
                    v = ((const int8_t *)w)[(size_t)o * I + i];
                }
                ref += (double)v * x[(size_t)t * I + i];
            }
            ref *= s[o];
            double rel = fabs(y[(size_t)t * O + o] - ref) / (fabs(ref) + 1e-6);
            if (rel > m) m = rel;
        }
    return m;
}

static double e4m3(uint8_t c) {
    int sign = (c & 0x80) ? -1 : 1, e = (c >> 3) & 15, m = c & 7;
    double v = e == 0 ? (m / 8.0) * ldexp(1.0, -6) : (1.0 + m / 8.0) * ldexp(1.0, e - 7);
    return sign * v;
}

static const double kFp4[16] = {0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6};

int main(void) {
    if (!fm_init()) {
        fprintf(stderr, "no B200 device\n");
        return 1;
    }
    printf("device: %s\n", fm_device_name());
    srand(42);
    int O = 128, I = 257, S = 4;
    int8_t *w8 = malloc((size_t)O * I);
    float *s = malloc(O * 4), *x = malloc((size_t)S * I * 4), *y = malloc((size_t)S * O * 4);
    for (int i = 0; i < O * I; i++) w8[i] = rand() % 255 - 127;
    for (int o = 0; o < O; o++) s[o] = frand() * 0.01f + 0.02f;
    for (int i = 0; i < S * I; i++) x[i] = frand();
    fm_matmul_q8(y, x, w8, s, O, I, S, 0);
    double r = maxrel_q(y, w8, 0, s, x, O, I, S);
    printf("q8 max rel err (cache=0): %.2e\n", r);
    if (r > 1e-3) { printf("FAIL q8 cache=0\n"); return 1; }
    for (int i = 0; i < S * I; i++) x[i] = frand();
    fm_matmul_q8(y, x, w8, s, O, I, S, 0);
    r = maxrel_q(y, w8, 0, s, x, O, I, S);
    printf("q8 max rel err (cache=0, repeated): %.2e\n", r);
    if (r > 1e-3) { printf("FAIL q8 cache=0 repeated\n"); return 1; }

    int rb = (I + 1) / 2;
    uint8_t *w4 = malloc((size_t)O * rb);
    for (int i = 0; i < O * rb; i++) w4[i] = rand() & 0xFF;
    fm_matmul_q4(y, x, w4, s, O, I, S, 1);
    r = maxrel_q(y, w4, 1, s, x, O, I, S);
    printf("q4 max rel err (cache=1): %.2e\n", r);
    if (r > 1e-3) { printf("FAIL q4 cache=1\n"); return 1; }
    for (int i = 0; i < S * I; i++) x[i] = frand();
    fm_matmul_q4(y, x, w4, s, O, I, S, 1);
    r = maxrel_q(y, w4, 1, s, x, O, I, S);
    printf("q4 max rel err (cache=1, same pointer): %.2e\n", r);
    if (r > 1e-3) { printf("FAIL q4 cache=1 repeated\n"); return 1; }

    /* DeepSeek V4 FP8: O = 256, I = 512, 128 x 128 E8M0 blocks */
    {
        int O8 = 256, I8 = 512, S8 = 3;
        uint8_t *w = malloc((size_t)O8 * I8), *sc = malloc((size_t)(O8 / 128) * (I8 / 128));
        float *xx = malloc((size_t)S8 * I8 * 4), *yy = malloc((size_t)S8 * O8 * 4);
        for (int i = 0; i < O8 * I8; i++) {
            uint8_t c = rand() & 0xFF;
            if ((c & 0x7F) == 0x7F) c ^= 1;  /* no NaN codes */
            w[i] = c;
        }
        for (int i = 0; i < (O8 / 128) * (I8 / 128); i++) sc[i] = 120 + rand() % 8;
        for (int i = 0; i < S8 * I8; i++) xx[i] = frand();
        if (!fm_matmul_deepseek_v4_fp8(yy, xx, w, sc, O8, I8, S8, 128)) { printf("FAIL fp8 call\n"); return 1; }
        double m = 0;
        for (int t = 0; t < S8; t++)
            for (int o = 0; o < O8; o++) {
                double ref = 0;
                for (int i = 0; i < I8; i++)
                    ref += xx[(size_t)t * I8 + i] * e4m3(w[(size_t)o * I8 + i]) *
                           ldexp(1.0, sc[(o / 128) * (I8 / 128) + i / 128] - 127);
                double rel = fabs(yy[(size_t)t * O8 + o] - ref) / (fabs(ref) + 1e-6);
                if (rel > m) m = rel;
            }
        printf("fp8 max rel err: %.2e\n", m);
        if (m > 1e-3) { printf("FAIL fp8\n"); return 1; }
        if (fm_matmul_deepseek_v4_fp8(yy, xx, w, sc, O8, I8, S8, 64)) { printf("FAIL fp8 block 64 accepted\n"); return 1; }
        free(w); free(sc); free(xx); free(yy);
    }
    /* DeepSeek V4 FP4: E2M1 codes with an E8M0 scale per 32 */
    {
        int O4 = 96, I4 = 256, S4 = 5;
        uint8_t *w = malloc((size_t)O4 * I4 / 2), *sc = malloc((size_t)O4 * I4 / 32);
        float *xx = malloc((size_t)S4 * I4 * 4), *yy = malloc((size_t)S4 * O4 * 4);
        for (int i = 0; i < O4 * I4 / 2; i++) w[i] = rand() & 0xFF;
        for (int i = 0; i < O4 * I4 / 32; i++) sc[i] = 118 + rand() % 6;
        for (int i = 0; i < S4 * I4; i++) xx[i] = frand();
        if (!fm_matmul_deepseek_v4_fp4(yy, xx, w, sc, O4, I4, S4)) { printf("FAIL fp4 call\n"); return 1; }
        double m = 0;
        for (int t = 0; t < S4; t++)
            for (int o = 0; o < O4; o++) {
                double ref = 0;
                for (int i = 0; i < I4; i++) {
                    uint8_t b = w[(size_t)o * I4 / 2 + i / 2];
                    int code = (i & 1) ? b >> 4 : b & 15;
                    ref += xx[(size_t)t * I4 + i] * kFp4[code] * ldexp(1.0, sc[(size_t)o * I4 / 32 + i / 32] - 127);
                }
                double rel = fabs(yy[(size_t)t * O4 + o] - ref) / (fabs(ref) + 1e-6);
                if (rel > m) m = rel;
            }
        printf("fp4 max rel err: %.2e\n", m);
        if (m > 1e-3) { printf("FAIL fp4\n"); return 1; }
        free(w); free(sc); free(xx); free(yy);
    }
    printf("OK\n");
    return 0;
}
