/*
 * st_lite.h - the smallest safetensors reader the C boundary tests need:
 * one file, tensors looked up by name, read as raw bytes or as float32.
 * (floyd's tests use its st.h; this is a separate, minimal one.)
 */
#ifndef ST_LITE_H
#define ST_LITE_H

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    FILE *f;
    char *header;
    uint64_t header_len;
} StFile;

static int st_open(StFile *st, const char *path) {
    unsigned char len8[8];
    memset(st, 0, sizeof(*st));
    st->f = fopen(path, "rb");
    if (!st->f || fread(len8, 1, 8, st->f) != 8) return 0;
    for (int i = 7; i >= 0; --i) st->header_len = (st->header_len << 8) | len8[i];
    st->header = (char *)malloc(st->header_len + 1);
    if (!st->header || fread(st->header, 1, st->header_len, st->f) != st->header_len) return 0;
    st->header[st->header_len] = 0;
    return 1;
}

static void st_close(StFile *st) {
    if (st->f) fclose(st->f);
    free(st->header);
    memset(st, 0, sizeof(*st));
}

/* Finds "name": {...} in the header; fills dtype, element count and the
 * byte range.  Tensor names in these fixtures never contain quotes. */
static int st_find(const StFile *st, const char *name, char dtype[8], int64_t *numel, uint64_t *begin,
                   uint64_t *end) {
    char key[300];
    snprintf(key, sizeof key, "\"%s\"", name);
    const char *p = strstr(st->header, key);
    if (!p) return 0;
    const char *obj = strchr(p + strlen(key), '{');
    const char *close = obj ? strchr(obj, '}') : NULL;
    if (!obj || !close) return 0;
    const char *d = strstr(obj, "\"dtype\"");
    const char *s = strstr(obj, "\"shape\"");
    const char *o = strstr(obj, "\"data_offsets\"");
    if (!d || !s || !o || d > close || s > close || o > close) return 0;
    d = strchr(d + 7, '"');
    if (!d) return 0;
    int i = 0;
    for (++d; *d && *d != '"' && i < 7; ++d) dtype[i++] = *d;
    dtype[i] = 0;
    s = strchr(s, '[');
    int64_t n = 1;
    for (++s; *s && *s != ']';) {
        while (*s == ' ' || *s == ',') ++s;
        if (*s == ']') break;
        n *= strtoll(s, (char **)&s, 10);
    }
    *numel = n;
    o = strchr(o, '[');
    *begin = strtoull(o + 1, (char **)&o, 10);
    while (*o == ' ' || *o == ',') ++o;
    *end = strtoull(o, NULL, 10);
    return 1;
}

static int64_t st_numel(const StFile *st, const char *name) {
    char dt[8];
    int64_t n;
    uint64_t b, e;
    return st_find(st, name, dt, &n, &b, &e) ? n : -1;
}

static int st_read_raw(const StFile *st, const char *name, void *dst, uint64_t capacity) {
    char dt[8];
    int64_t n;
    uint64_t b, e;
    if (!st_find(st, name, dt, &n, &b, &e) || e - b > capacity) return 0;
    if (fseek(st->f, (long)(8 + st->header_len + b), SEEK_SET) != 0) return 0;
    return fread(dst, 1, e - b, st->f) == e - b;
}

/* Allocates and reads an F32 tensor; *count = its element count. */
static float *st_read_f32(const StFile *st, const char *name, int64_t *count) {
    char dt[8];
    int64_t n;
    uint64_t b, e;
    if (!st_find(st, name, dt, &n, &b, &e) || strcmp(dt, "F32") != 0) return NULL;
    float *v = (float *)malloc((size_t)n * sizeof(float));
    if (!v || !st_read_raw(st, name, v, (uint64_t)n * 4)) {
        free(v);
        return NULL;
    }
    *count = n;
    return v;
}

/* Reads an I64 tensor into ints. */
static int *st_read_ids(const StFile *st, const char *name, int64_t *count) {
    int64_t n = st_numel(st, name);
    if (n <= 0) return NULL;
    int64_t *raw = (int64_t *)malloc((size_t)n * 8);
    int *v = (int *)malloc((size_t)n * sizeof(int));
    if (!raw || !v || !st_read_raw(st, name, raw, (uint64_t)n * 8)) {
        free(raw);
        free(v);
        return NULL;
    }
    for (int64_t i = 0; i < n; ++i) v[i] = (int)raw[i];
    free(raw);
    *count = n;
    return v;
}

#endif
