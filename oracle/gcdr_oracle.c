/*
 * gcdr_oracle.c -- CPU restatement of the GCDRNet enhancement path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the CUDA
 * backend: it is linked by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline / reference legs of bench.py, as the checker.  The product
 * library (libgcdr_cuda.so) never links or calls it.
 *
 * It restates, in plain C (OpenMP over rows, loops written for the compiler's
 * auto-vectoriser), the operator semantics of the two ONNX graphs
 * tests/testdata/models/gcdrnet_{gcnet,drnet}_sim.onnx of the reference and
 * the glue around them:
 *
 *   pre    GcdrEnhancer.cs:242-243 (ImageTensor.FromPixels), spec
 *          Backends/Vulkan/Shaders/bgr2nhwc.comp:23-35, tests/GoldenDerive.cs:11-23
 *   div6   Kernels/PixelOps.cs:77-102 (DivConcatNhwc), div6.comp:14-24
 *   post   GcdrEnhancer.cs:266-268 (ImageTensor.ToPixels), nhwc2bgr.comp:23-55,
 *          Kernels/PixelOps.cs:118-135 (alpha copied from the source)
 *   shift  Extensions/GcdrKernels.cs:169-198 (ChannelShift, NHWC)
 *   resize ONNX Resize linear/half_pixel, spec uphead.glsl:190-195
 *   conv / maxpool / layernorm / gemm / depthwise / gelu: ONNX opset-18
 *          semantics of the nodes gc#22..459 / dr#22..459.
 *
 * All tensors are NHWC float32, batch 1.  Convolution weights are given in
 * ONNX order [Cout][Cin][kh][kw] and repacked here.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

static inline int reflect_index(int i, int n)
{
    /* ONNX Pad mode=reflect (edge excluded), as PyTorch ReflectionPad2d. */
    if (n <= 1) return 0;
    while (i < 0 || i >= n) i = i < 0 ? -i : 2 * n - 2 - i;
    return i;
}

ORC_API int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

ORC_API void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------ conv */

/*
 * Dense or depthwise-free 2-D convolution, NHWC.
 *   x   [H][W][Cin]
 *   w   ONNX [Cout][Cin][k][k]
 *   out [Ho][Wo][Cout], Ho = (H + 2*pad - k)/stride + 1
 * pad_mode 0: zero padding, 1: reflect padding (the graph's explicit
 * Pad(mode=reflect) followed by a pads=0 Conv, gc#22-23).
 * out = bias + sum over (ky,kx,ci) of w * x, accumulated in float in
 * tap-major, channel-ascending order.
 */
ORC_API void orc_conv2d(const float *x, int H, int W, int Cin,
                        const float *w, const float *bias, int Cout,
                        int k, int stride, int pad, int pad_mode, float *out)
{
    int Ho = (H + 2 * pad - k) / stride + 1;
    int Wo = (W + 2 * pad - k) / stride + 1;
    /* repack to [ky][kx][ci][co] so the inner loop runs over contiguous co */
    size_t K = (size_t)k * k * Cin;
    float *wp = (float *)malloc(K * Cout * sizeof(float));
    for (int co = 0; co < Cout; co++)
        for (int ci = 0; ci < Cin; ci++)
            for (int ky = 0; ky < k; ky++)
                for (int kx = 0; kx < k; kx++)
                    wp[(((size_t)ky * k + kx) * Cin + ci) * Cout + co] =
                        w[(((size_t)co * Cin + ci) * k + ky) * k + kx];

#pragma omp parallel
    {
        float *acc = (float *)malloc((size_t)Cout * 4 * sizeof(float));
#pragma omp for schedule(dynamic, 1)
        for (int oy = 0; oy < Ho; oy++) {
            for (int ox0 = 0; ox0 < Wo; ox0 += 4) {
                int np = Wo - ox0 < 4 ? Wo - ox0 : 4;
                for (int p = 0; p < 4; p++)
                    for (int co = 0; co < Cout; co++)
                        acc[p * Cout + co] = bias ? bias[co] : 0.0f;
                for (int ky = 0; ky < k; ky++) {
                    int iy = oy * stride + ky - pad;
                    int vy = 1;
                    if (iy < 0 || iy >= H) {
                        if (pad_mode == 1) iy = reflect_index(iy, H);
                        else vy = 0;
                    }
                    for (int kx = 0; kx < k; kx++) {
                        const float *xs[4];
                        for (int p = 0; p < 4; p++) {
                            int ix = (ox0 + (p < np ? p : 0)) * stride + kx - pad;
                            int vx = 1;
                            if (ix < 0 || ix >= W) {
                                if (pad_mode == 1) ix = reflect_index(ix, W);
                                else vx = 0;
                            }
                            xs[p] = (vy && vx) ? x + ((size_t)iy * W + ix) * Cin : NULL;
                        }
                        const float *wt = wp + ((size_t)ky * k + kx) * Cin * Cout;
                        for (int ci = 0; ci < Cin; ci++) {
                            const float *wr = wt + (size_t)ci * Cout;
                            for (int p = 0; p < 4; p++) {
                                if (!xs[p]) continue;
                                float xv = xs[p][ci];
                                float *a = acc + p * Cout;
                                for (int co = 0; co < Cout; co++) a[co] += xv * wr[co];
                            }
                        }
                    }
                }
                for (int p = 0; p < np; p++)
                    memcpy(out + ((size_t)oy * Wo + ox0 + p) * Cout, acc + p * Cout,
                           (size_t)Cout * sizeof(float));
            }
        }
        free(acc);
    }
    free(wp);
}

/* MaxPool 2x2 stride 2 (no padding, floor) then ReLU: gc#24-25. */
ORC_API void orc_maxpool2_relu(const float *x, int H, int W, int C, float *out)
{
    int Ho = H / 2, Wo = W / 2;
#pragma omp parallel for
    for (int oy = 0; oy < Ho; oy++)
        for (int ox = 0; ox < Wo; ox++) {
            const float *a = x + ((size_t)(2 * oy) * W + 2 * ox) * C;
            const float *b = a + C;
            const float *c = a + (size_t)W * C;
            const float *d = c + C;
            float *o = out + ((size_t)oy * Wo + ox) * C;
            for (int ch = 0; ch < C; ch++) {
                float m = a[ch];
                if (b[ch] > m) m = b[ch];
                if (c[ch] > m) m = c[ch];
                if (d[ch] > m) m = d[ch];
                o[ch] = m > 0.0f ? m : 0.0f;
            }
        }
}

ORC_API void orc_relu(float *x, size_t n)
{
#pragma omp parallel for
    for (size_t i = 0; i < n; i++) x[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

ORC_API void orc_add(const float *a, const float *b, float *out, size_t n)
{
#pragma omp parallel for
    for (size_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

ORC_API void orc_sigmoid(float *x, size_t n)
{
#pragma omp parallel for
    for (size_t i = 0; i < n; i++) x[i] = 1.0f / (1.0f + expf(-x[i]));
}

/*
 * LayerNormalization over the last axis (C), epsilon eps, stash_type=1
 * (statistics in full precision): gc#37 etc.  Mean and variance are
 * accumulated in double; y = (x - mean) / sqrt(var + eps) * g + b.
 */
ORC_API void orc_layernorm(const float *x, size_t T, int C, const float *g,
                           const float *b, float eps, float *out)
{
#pragma omp parallel for
    for (size_t t = 0; t < T; t++) {
        const float *r = x + t * C;
        double s = 0.0;
        for (int c = 0; c < C; c++) s += r[c];
        double mean = s / C;
        double v = 0.0;
        for (int c = 0; c < C; c++) {
            double d = r[c] - mean;
            v += d * d;
        }
        double inv = 1.0 / sqrt(v / C + (double)eps);
        float *o = out + t * C;
        for (int c = 0; c < C; c++)
            o[c] = (float)((r[c] - mean) * inv) * g[c] + b[c];
    }
}

/* Gemm alpha=1 beta=1 transA=0 transB=0: out[T][N] = x[T][K] @ B[K][N] + bias (gc#81). */
ORC_API void orc_gemm_bias(const float *x, size_t T, int K, const float *B,
                           const float *bias, int N, float *out)
{
#pragma omp parallel for schedule(static)
    for (size_t t = 0; t < T; t++) {
        float *o = out + t * N;
        for (int n = 0; n < N; n++) o[n] = bias ? bias[n] : 0.0f;
        const float *r = x + t * K;
        for (int k = 0; k < K; k++) {
            float xv = r[k];
            const float *br = B + (size_t)k * N;
            for (int n = 0; n < N; n++) o[n] += xv * br[n];
        }
    }
}

/*
 * Depthwise 3x3 conv, zero pad 1, stride 1, group = C (gc#85):
 * w is ONNX [C][1][3][3].
 */
ORC_API void orc_dwconv3x3(const float *x, int H, int W, int C, const float *w,
                           const float *bias, float *out)
{
    float *wp = (float *)malloc((size_t)9 * C * sizeof(float));
    for (int c = 0; c < C; c++)
        for (int t = 0; t < 9; t++) wp[(size_t)t * C + c] = w[(size_t)c * 9 + t];
#pragma omp parallel for
    for (int oy = 0; oy < H; oy++)
        for (int ox = 0; ox < W; ox++) {
            float *o = out + ((size_t)oy * W + ox) * C;
            for (int c = 0; c < C; c++) o[c] = bias[c];
            for (int ky = 0; ky < 3; ky++) {
                int iy = oy + ky - 1;
                if (iy < 0 || iy >= H) continue;
                for (int kx = 0; kx < 3; kx++) {
                    int ix = ox + kx - 1;
                    if (ix < 0 || ix >= W) continue;
                    const float *r = x + ((size_t)iy * W + ix) * C;
                    const float *wt = wp + (size_t)(ky * 3 + kx) * C;
                    for (int c = 0; c < C; c++) o[c] += wt[c] * r[c];
                }
            }
        }
    free(wp);
}

/* Exact GELU as exported (gc#88-92): x * (0.5 * (erf(x / sqrt2) + 1)). */
ORC_API void orc_gelu(float *x, size_t n)
{
    const float sqrt2 = 1.4142135381698608f;
#pragma omp parallel for
    for (size_t i = 0; i < n; i++) {
        float v = x[i];
        x[i] = v * (0.5f * (erff(v / sqrt2) + 1.0f));
    }
}

/*
 * ChannelShift, NHWC (Extensions/GcdrKernels.cs:169-198): for channel group
 * g = [ends[g-1], ends[g]) out[y,x,c] = in[y+off_g, x, c] (axis 2 = H) or
 * in[y, x+off_g, c] (axis 3 = W), zero outside the image.  Channels past the
 * last group end are copied unshifted.
 */
ORC_API void orc_shift(const float *x, int H, int W, int C, int axis,
                       const int *ends, const int *offs, int ngroups, float *out)
{
#pragma omp parallel for
    for (int y = 0; y < H; y++)
        for (int xx = 0; xx < W; xx++) {
            float *o = out + ((size_t)y * W + xx) * C;
            int g0 = 0;
            for (int g = 0; g < ngroups; g++) {
                int g1 = ends[g];
                int sy = axis == 2 ? y + offs[g] : y;
                int sx = axis == 2 ? xx : xx + offs[g];
                if (sy >= 0 && sy < H && sx >= 0 && sx < W)
                    memcpy(o + g0, x + ((size_t)sy * W + sx) * C + g0, (size_t)(g1 - g0) * sizeof(float));
                else
                    memset(o + g0, 0, (size_t)(g1 - g0) * sizeof(float));
                g0 = g1;
            }
            if (g0 < C)
                memcpy(o + g0, x + ((size_t)y * W + xx) * C + g0, (size_t)(C - g0) * sizeof(float));
        }
}

/*
 * Resize x2, mode=linear, coordinate_transformation_mode=half_pixel
 * (gc#236): src = (dst + 0.5) / 2 - 0.5, neighbours clamped to the edge.
 */
ORC_API void orc_resize2x(const float *x, int H, int W, int C, float *out)
{
    int Ho = 2 * H, Wo = 2 * W;
#pragma omp parallel for
    for (int oy = 0; oy < Ho; oy++) {
        float fy = ((float)oy + 0.5f) / 2.0f - 0.5f;
        int y0 = (int)floorf(fy);
        float dy = fy - (float)y0;
        int ya = y0 < 0 ? 0 : (y0 > H - 1 ? H - 1 : y0);
        int yb = y0 + 1 < 0 ? 0 : (y0 + 1 > H - 1 ? H - 1 : y0 + 1);
        for (int ox = 0; ox < Wo; ox++) {
            float fx = ((float)ox + 0.5f) / 2.0f - 0.5f;
            int x0 = (int)floorf(fx);
            float dx = fx - (float)x0;
            int xa = x0 < 0 ? 0 : (x0 > W - 1 ? W - 1 : x0);
            int xb = x0 + 1 < 0 ? 0 : (x0 + 1 > W - 1 ? W - 1 : x0 + 1);
            const float *p00 = x + ((size_t)ya * W + xa) * C;
            const float *p01 = x + ((size_t)ya * W + xb) * C;
            const float *p10 = x + ((size_t)yb * W + xa) * C;
            const float *p11 = x + ((size_t)yb * W + xb) * C;
            float *o = out + ((size_t)oy * Wo + ox) * C;
            for (int c = 0; c < C; c++) {
                float top = p00[c] + (p01[c] - p00[c]) * dx;
                float bot = p10[c] + (p11[c] - p10[c]) * dx;
                o[c] = top + (bot - top) * dy;
            }
        }
    }
}

/* ------------------------------------------------------------------ glue */

static inline int fmt_bpp(int fmt) { return fmt >= 2 ? 4 : 3; }
static inline int fmt_swap(int fmt) { return fmt == 1 || fmt == 3; }

/*
 * Pre: interleaved u8 (GcdrPixelFormat 0..3, row stride `stride`) to the
 * padded NHWC net input x[h+ph][w+pw][3] in B,G,R order scaled by 1/255,
 * top/left edge replicated (bgr2nhwc.comp:28-34, GoldenDerive.cs:11-23).
 */
ORC_API void orc_pre(const uint8_t *src, int w, int h, int stride, int fmt,
                     int ph, int pw, float *x)
{
    int H = h + ph, Wd = w + pw, bpp = fmt_bpp(fmt), ob = fmt_swap(fmt) ? 2 : 0;
#pragma omp parallel for
    for (int y = 0; y < H; y++) {
        int sy = y - ph < 0 ? 0 : y - ph;
        for (int xx = 0; xx < Wd; xx++) {
            int sx = xx - pw < 0 ? 0 : xx - pw;
            const uint8_t *s = src + (size_t)sy * stride + (size_t)sx * bpp;
            float *o = x + ((size_t)y * Wd + xx) * 3;
            o[0] = (float)s[ob] / 255.0f;
            o[1] = (float)s[1] / 255.0f;
            o[2] = (float)s[2 - ob] / 255.0f;
        }
    }
}

/* div6 (PixelOps.cs:81-102): out[p,0..2] = x, out[p,3..5] = clamp(x / max(s,1e-6), 0, 1). */
ORC_API void orc_div6(const float *x, const float *s, size_t npx, float *out)
{
#pragma omp parallel for
    for (size_t p = 0; p < npx; p++)
        for (int c = 0; c < 3; c++) {
            float v = x[p * 3 + c];
            float d = s[p * 3 + c] > 1e-6f ? s[p * 3 + c] : 1e-6f;
            float r = v / d;
            r = r < 0.0f ? 0.0f : (r > 1.0f ? 1.0f : r);
            out[p * 6 + c] = v;
            out[p * 6 + 3 + c] = r;
        }
}

/*
 * Post: net output y[H][W][3] (B,G,R in [0,1]) to the caller's format,
 * cropping the top/left pad, u8 = clamp(y*255 + 0.5, 0, 255) truncated
 * (nhwc2bgr.comp:23); 4-byte formats take alpha from alpha_src (same
 * format, stride alpha_stride), which may alias dst.
 */
ORC_API void orc_post(const float *y, int H, int W, int ph, int pw,
                      uint8_t *dst, int w, int h, int dst_stride, int fmt,
                      const uint8_t *alpha_src, int alpha_stride)
{
    int bpp = fmt_bpp(fmt), ob = fmt_swap(fmt) ? 2 : 0;
    (void)H;
#pragma omp parallel for
    for (int r = 0; r < h; r++)
        for (int c = 0; c < w; c++) {
            const float *v = y + ((size_t)(r + ph) * W + (c + pw)) * 3;
            uint8_t q[3];
            for (int k = 0; k < 3; k++) {
                float f = v[k] * 255.0f + 0.5f;
                f = f < 0.0f ? 0.0f : (f > 255.0f ? 255.0f : f);
                q[k] = (uint8_t)f;
            }
            uint8_t *d = dst + (size_t)r * dst_stride + (size_t)c * bpp;
            uint8_t a = bpp == 4 ? alpha_src[(size_t)r * alpha_stride + (size_t)c * 4 + 3] : 0;
            d[ob] = q[0];
            d[1] = q[1];
            d[2 - ob] = q[2];
            if (bpp == 4) d[3] = a;
        }
}
