/*
 * A plain C caller of the backend's C ABI (include/gcdr_cuda.h), the way a C#
 * P/Invoke binding or a C++ service would call it: no Python, no torch.
 *
 *   enhance_demo <gc.onnx> <dr.onnx> <width> <height>
 *
 * Builds a Bgra32 gradient image with a row stride of width*4 + 64 and an alpha
 * ramp, enhances it in place through the pooled enhancer, then checks the
 * contract of GcdrEnhancer.Enhance (GcdrEnhancer.cs:181-271): status OK, alpha
 * and row padding untouched, argument errors reported with the reference's
 * exception kinds, pool statistics.  Prints "ok" and exits 0 on success.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gcdr_cuda.h"

static unsigned char *read_file(const char *path, size_t *len) {
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    unsigned char *buf = (unsigned char *)malloc((size_t)n);
    if (buf && fread(buf, 1, (size_t)n, f) != (size_t)n) {
        free(buf);
        buf = NULL;
    }
    fclose(f);
    *len = (size_t)n;
    return buf;
}

#define CHECK(cond, msg)                                   \
    do {                                                   \
        if (!(cond)) {                                     \
            fprintf(stderr, "FAILED: %s (%s)\n", msg, err); \
            return 1;                                      \
        }                                                  \
    } while (0)

int main(int argc, char **argv) {
    char err[512] = "";
    if (argc != 5) {
        fprintf(stderr, "usage: %s gc.onnx dr.onnx width height\n", argv[0]);
        return 2;
    }
    size_t gc_len = 0, dr_len = 0;
    unsigned char *gc = read_file(argv[1], &gc_len), *dr = read_file(argv[2], &dr_len);
    CHECK(gc && dr, "model files");
    const int w = atoi(argv[3]), h = atoi(argv[4]), stride = w * 4 + 64;
    gcdr_enhancer *e = NULL;
    int rc = gcdr_enhancer_create(0, gc, gc_len, dr, dr_len, GCDR_PRECISION_FP16, &e, err, sizeof err);
    free(gc);
    free(dr);
    CHECK(rc == GCDR_OK && e, "gcdr_enhancer_create");

    const size_t len = (size_t)h * stride;
    uint8_t *img = (uint8_t *)malloc(len), *orig = (uint8_t *)malloc(len);
    for (int y = 0; y < h; y++)
        for (int x = 0; x < stride; x++) {
            uint8_t v = 0x5A;   /* row padding */
            if (x < w * 4) {
                const int c = x % 4, px = x / 4;
                v = (uint8_t)(c == 3 ? (px * 7 + y * 13) & 255 : 180 + ((px + y) % 60) - 20 * (c == 1));
            }
            img[(size_t)y * stride + x] = v;
        }
    memcpy(orig, img, len);

    rc = gcdr_enhancer_enhance(e, img, len, w, h, stride, img, len, stride, GCDR_BGRA32, err, sizeof err);
    CHECK(rc == GCDR_OK, "enhance in place");
    int changed = 0;
    for (int y = 0; y < h; y++)
        for (int x = 0; x < stride; x++) {
            const size_t i = (size_t)y * stride + x;
            if (x >= w * 4 || x % 4 == 3) CHECK(img[i] == orig[i], "alpha / row padding must stay untouched");
            else changed += img[i] != orig[i];
        }
    CHECK(changed > 0, "the image was enhanced");

    /* argument errors, in the reference's order and kinds */
    CHECK(gcdr_enhancer_enhance(e, img, len, 0, h, stride, img, len, stride, GCDR_BGRA32, err, sizeof err) ==
              GCDR_ERR_RANGE, "width < 1 -> ArgumentOutOfRange");
    CHECK(gcdr_enhancer_enhance(e, img, len, w, h, stride, img, len, stride, 9, err, sizeof err) == GCDR_ERR_RANGE,
          "unknown pixel format -> ArgumentOutOfRange");
    CHECK(gcdr_enhancer_enhance(e, img, len / 2, w, h, stride, img, len, stride, GCDR_BGRA32, err, sizeof err) ==
              GCDR_ERR_ARG, "short source -> Argument");

    int64_t pools = 0, workers = 0, evicted = 0;
    gcdr_enhancer_pool_stats(e, &pools, &workers, &evicted);
    CHECK(pools == 1 && workers == 1 && evicted == 0, "pool statistics");
    gcdr_enhancer_destroy(e);
    free(img);
    free(orig);
    printf("ok\n");
    return 0;
}
