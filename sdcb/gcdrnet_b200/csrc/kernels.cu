// kernels.cu -- the SIMT kernels of the pipeline: fp32 stem and head (with the
// pixel glue fused in), the shift-MLP depthwise stage, the decoder joins and
// the standalone glue kernels.
#include <cuda_runtime.h>

#include "kernels.h"

namespace gcdr {
namespace {

__device__ __forceinline__ int reflect1(int i, int n) {
    // ONNX Pad mode=reflect by one pixel; a dimension of size 1 mirrors onto itself
    if (n <= 1) return 0;
    if (i < 0) return -i;
    if (i >= n) return 2 * n - 2 - i;
    return i;
}

// Net input x at padded coordinates (py, px): the source pixel with the
// top/left edge replicated, channels in B,G,R order, scaled by 1/255
// (bgr2nhwc.comp:28-34, GoldenDerive.cs:11-23).
__device__ __forceinline__ float img_val(const ImgSpec &im, int py, int px, int c) {
    int sy = py - im.ph, sx = px - im.pw;
    sy = sy < 0 ? 0 : sy;
    sx = sx < 0 ? 0 : sx;
    const uint8_t *p = im.src + (size_t)sy * im.stride + (size_t)sx * im.bpp;
    const int ob = im.swap ? 2 : 0;
    const int off = c == 1 ? 1 : (c == 0 ? ob : 2 - ob);
    return (float)p[off] / 255.0f;
}

template <int CIN>
__device__ __forceinline__ void load_px(const ImgSpec &im, const float *r, int W, int py, int px, float *v) {
#pragma unroll
    for (int c = 0; c < 3; c++) v[c] = img_val(im, py, px, c);
    if (CIN == 6) {
        const float *rp = r + ((size_t)py * W + px) * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) v[3 + c] = rp[c];
    }
}

template <int CIN, int C1>
__global__ void __launch_bounds__(128) stem_kernel(const StemArgs a) {
    pdl_wait();
    __shared__ float ws[9 * CIN * C1];
    __shared__ float bs[C1];
    for (int i = threadIdx.x; i < 9 * CIN * C1; i += blockDim.x) {
        int co = i % C1, t = i / C1, ci = t % CIN, tap = t / CIN;
        ws[i] = a.w[(co * CIN + ci) * 9 + tap];
    }
    for (int i = threadIdx.x; i < C1; i += blockDim.x) bs[i] = a.b[i];
    __syncthreads();
    const int Hh = a.H / 2, Wh = a.W / 2;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= Hh * Wh) return;
    const int y2 = idx / Wh, x2 = idx - y2 * Wh;
    float patch[4][4][CIN];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int yy = reflect1(2 * y2 - 1 + i, a.H);
#pragma unroll
        for (int j = 0; j < 4; j++) load_px<CIN>(a.img, a.r, a.W, yy, reflect1(2 * x2 - 1 + j, a.W), patch[i][j]);
    }
    __align__(16) __half h[C1];
#pragma unroll 1
    for (int co = 0; co < C1; co++) {
        float acc[4];
#pragma unroll
        for (int p = 0; p < 4; p++) acc[p] = bs[co];
#pragma unroll
        for (int ky = 0; ky < 3; ky++)
#pragma unroll
            for (int kx = 0; kx < 3; kx++)
#pragma unroll
                for (int ci = 0; ci < CIN; ci++) {
                    const float w = ws[((ky * 3 + kx) * CIN + ci) * C1 + co];
#pragma unroll
                    for (int dy = 0; dy < 2; dy++)
#pragma unroll
                        for (int dx = 0; dx < 2; dx++)
                            acc[dy * 2 + dx] = fmaf(patch[dy + ky][dx + kx][ci], w, acc[dy * 2 + dx]);
                }
        const float m = fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3]));
        h[co] = __float2half_rn(fmaxf(m, 0.0f));
    }
    act_store(a.out, y2, x2, 0, h, C1);
    pdl_trigger();
}

template <int CIN, int C1, bool DR>
__global__ void __launch_bounds__(128) head_kernel(const HeadArgs a) {
    pdl_wait();
    __shared__ float ws[9 * CIN * C1];
    __shared__ float bs[C1];
    __shared__ float fw[3 * C1];
    __shared__ float fb[3];
    for (int i = threadIdx.x; i < 9 * CIN * C1; i += blockDim.x) {
        int co = i % C1, t = i / C1, ci = t % CIN, tap = t / CIN;
        ws[i] = a.w[(co * CIN + ci) * 9 + tap];
    }
    for (int i = threadIdx.x; i < C1; i += blockDim.x) bs[i] = a.b[i];
    for (int i = threadIdx.x; i < 3 * C1; i += blockDim.x) fw[i] = a.fw[i];
    if (threadIdx.x < 3) fb[threadIdx.x] = a.fb[threadIdx.x];
    __syncthreads();
    const int ow = DR ? a.img.w : a.W, oh = DR ? a.img.h : a.H;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= ow * oh) return;
    const int oy = idx / ow, ox = idx - oy * ow;
    const int py = DR ? oy + a.img.ph : oy, px = DR ? ox + a.img.pw : ox;

    // skip = relu(enc1 conv) recomputed at this pixel (uphead.glsl:200-229)
    float patch[3][3][CIN];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int yy = reflect1(py - 1 + i, a.H);
#pragma unroll
        for (int j = 0; j < 3; j++) load_px<CIN>(a.img, a.r, a.W, yy, reflect1(px - 1 + j, a.W), patch[i][j]);
    }
    // bilinear x2, half_pixel, edge clamp (Resize gc#454)
    const int Hh = a.H / 2, Wh = a.W / 2;
    const float fy = ((float)py + 0.5f) / 2.0f - 0.5f, fx = ((float)px + 0.5f) / 2.0f - 0.5f;
    const int y0 = (int)floorf(fy), x0 = (int)floorf(fx);
    const float dy = fy - (float)y0, dx = fx - (float)x0;
    const int ya = min(max(y0, 0), Hh - 1), yb = min(max(y0 + 1, 0), Hh - 1);
    const int xa = min(max(x0, 0), Wh - 1), xb = min(max(x0 + 1, 0), Wh - 1);
    const __half *p00 = a.dec5 + ((size_t)ya * Wh + xa) * C1, *p01 = a.dec5 + ((size_t)ya * Wh + xb) * C1;
    const __half *p10 = a.dec5 + ((size_t)yb * Wh + xa) * C1, *p11 = a.dec5 + ((size_t)yb * Wh + xb) * C1;
    float o0 = fb[0], o1 = fb[1], o2 = fb[2];
#pragma unroll 1
    for (int co = 0; co < C1; co++) {
        float acc = bs[co];
#pragma unroll
        for (int ky = 0; ky < 3; ky++)
#pragma unroll
            for (int kx = 0; kx < 3; kx++)
#pragma unroll
                for (int ci = 0; ci < CIN; ci++) acc = fmaf(patch[ky][kx][ci], ws[((ky * 3 + kx) * CIN + ci) * C1 + co], acc);
        const float v00 = __half2float(p00[co]), v01 = __half2float(p01[co]);
        const float v10 = __half2float(p10[co]), v11 = __half2float(p11[co]);
        const float top = v00 + (v01 - v00) * dx, bot = v10 + (v11 - v10) * dx;
        const float up = top + (bot - top) * dy;
        const float s = fmaxf(up, 0.0f) + fmaxf(acc, 0.0f);
        o0 = fmaf(s, fw[co], o0);
        o1 = fmaf(s, fw[C1 + co], o1);
        o2 = fmaf(s, fw[2 * C1 + co], o2);
    }
    float o[3] = {1.0f / (1.0f + expf(-o0)), 1.0f / (1.0f + expf(-o1)), 1.0f / (1.0f + expf(-o2))};
    if (!DR) {
        const size_t base = ((size_t)py * a.W + px) * 3;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const float d = o[c] > 1e-6f ? o[c] : 1e-6f;
            float q = patch[1][1][c] / d;
            q = q < 0.0f ? 0.0f : (q > 1.0f ? 1.0f : q);
            a.r_out[base + c] = q;
            if (a.ism_out) a.ism_out[base + c] = o[c];
        }
    } else {
        if (a.y_out) {
            const size_t base = ((size_t)py * a.W + px) * 3;
            for (int c = 0; c < 3; c++) a.y_out[base + c] = o[c];
        }
        uint8_t q[3];
#pragma unroll
        for (int c = 0; c < 3; c++) {
            float f = o[c] * 255.0f + 0.5f;
            f = f < 0.0f ? 0.0f : (f > 255.0f ? 255.0f : f);
            q[c] = (uint8_t)f;
        }
        const int bpp = a.img.bpp, ob = a.img.swap ? 2 : 0;
        uint8_t *d = a.dst + ((size_t)oy * a.img.w + ox) * bpp;
        if (bpp == 4) {
            const uint8_t al = a.img.src[(size_t)oy * a.img.stride + (size_t)ox * 4 + 3];
            uchar4 v;
            v.x = ob ? q[2] : q[0];
            v.y = q[1];
            v.z = ob ? q[0] : q[2];
            v.w = al;
            *reinterpret_cast<uchar4 *>(d) = v;
        } else {
            d[ob] = q[0];
            d[1] = q[1];
            d[2 - ob] = q[2];
        }
    }
    pdl_trigger();
}

// gc#88-92: x * (0.5 * (erf(x / 1.4142135381698608) + 1)).  erf by Abramowitz &
// Stegun, Handbook of Mathematical Functions, formula 7.1.26: for z >= 0,
// erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2), t = 1 / (1 + p z),
// |error| <= 1.5e-7 (two orders below the fp16 rounding of the stored activation).
// For x < 0 the factor 1 + erf(z) = e(z) = poly * exp(-z^2) is formed directly, so the
// small negative tail carries no cancellation.  Two values at a time: the multiplies and
// fused multiply-adds on packed fp32 pairs (FMUL2 / FFMA2, each lane rounded as its scalar
// form), the reciprocal, exponential and selects per lane.
__device__ __forceinline__ float2 gelu_exact2(float2 v) {
    const float2 z = __fmul2_rn(make_float2(fabsf(v.x), fabsf(v.y)), make_float2(0.70710678118654752f, 0.70710678118654752f));
    const float2 d = __ffma2_rn(make_float2(0.3275911f, 0.3275911f), z, make_float2(1.0f, 1.0f));
    const float2 t = make_float2(__fdividef(1.0f, d.x), __fdividef(1.0f, d.y));
    float2 poly = __ffma2_rn(t, make_float2(1.061405429f, 1.061405429f), make_float2(-1.453152027f, -1.453152027f));
    poly = __ffma2_rn(poly, t, make_float2(1.421413741f, 1.421413741f));
    poly = __ffma2_rn(poly, t, make_float2(-0.284496736f, -0.284496736f));
    poly = __ffma2_rn(poly, t, make_float2(0.254829592f, 0.254829592f));
    const float2 zz = __fmul2_rn(z, z);
    const float2 e = __fmul2_rn(__fmul2_rn(poly, t), make_float2(__expf(-zz.x), __expf(-zz.y)));   // 1 - erf(z)
    const float2 h = __fmul2_rn(make_float2(0.5f, 0.5f), v);
    return __fmul2_rn(h, make_float2(v.x >= 0.0f ? 2.0f - e.x : e.x, v.y >= 0.0f ? 2.0f - e.y : e.y));
}

// out = shiftW(gelu(dw(in))): depthwise 3x3 (zero pad 1) + bias + exact GELU,
// then the W shift that precedes fc2 (gc#95-126), applied as a gather: channel c
// of output pixel x is the activation of source pixel x + off_g(c) (zero when
// that column lies outside the row).  A thread computes one 8-channel chunk of
// two consecutive output pixels (x, x+1): the chunk's channels [0, split) belong
// to one shift group (offset offa), the rest, when the chunk straddles a group
// boundary, to the next (offb).  Each row of the 3x3 window is read as four source
// columns at offset offa and, for a straddling chunk, four more at offset offb;
// one byte permutation per 32-bit word merges the two into the columns the chunk's
// channels read, so every output chunk is one 16-byte store (a scatter splits the
// straddling chunks into per-channel stores).  Each tap's eight weights are read
// once from shared memory (tap-major [9][C] fp32) and serve both pixels.  (Four
// pixels per thread measured no faster: the kernel is bound by the latency of its
// loads, and the wider window spills registers.)  A flat grid of 128-thread blocks
// over (row, pixel pair, chunk): no partly empty block per row.  The tap sums (in
// the order ky, kx) and the GELU run on packed channel pairs (FFMA2), lane by lane
// as fmaf.
constexpr int kDwMaxC = 512;
constexpr int kDwPx = 2;   // output pixels per thread

__device__ __forceinline__ uint4 dw_col(const __half *rowp, int xx, int W, int C) {
    return (xx >= 0 && xx < W) ? *reinterpret_cast<const uint4 *>(rowp + (size_t)xx * C) : make_uint4(0, 0, 0, 0);
}

__global__ void __launch_bounds__(128, 7) dw_gelu_shift_kernel(const __half *in, int H, int W, int C, const float *wt,
                                                            const float *b, const ShiftSpec s, __half *out,
                                                            long long img_bytes) {
    constexpr int PX = kDwPx;
    extern __shared__ __align__(16) float ws[];   // [9][C]
    // the weights are constant: staged before the wait on the previous kernel
    for (int i = threadIdx.x * 4; i < 9 * C; i += blockDim.x * 4)
        *reinterpret_cast<float4 *>(ws + i) = __ldg(reinterpret_cast<const float4 *>(wt + i));
    __syncthreads();
    pdl_wait();
    const int chunks = C >> 3;
    const int Wq = (W + PX - 1) / PX;                  // pixel pairs per row
    const int per_row = Wq * chunks;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = i / per_row, t = i - y * per_row;
    if (y < H) {
        const int xq = t / chunks, ch = t - xq * chunks;
        const int x = PX * xq, c0 = ch * 8;
        // shift groups of the chunk: channels [0, split) offset offa, [split, 8) offb
        // (the launcher checks that no chunk spans three groups)
        const int ga = shift_group(s, c0), gb = shift_group(s, c0 + 7);
        const int offa = ga >= 0 ? s.offs[ga] : 0, offb = gb >= 0 ? s.offs[gb] : 0;
        const int split = ga == gb ? 8 : s.ends[ga] - c0;
        const bool straddle = split < 8;
        // per 32-bit word (a channel pair): its low and high halves from the offa
        // column (bytes 0-3 of the permutation) or the offb column (bytes 4-7)
        uint32_t sel[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            sel[k] = (2 * k < split ? 0x10u : 0x54u) | ((2 * k + 1 < split ? 0x32u : 0x76u) << 8);
        float2 acc[PX][4];   // channel pairs (c0 + 2i, c0 + 2i + 1): packed FFMA2, per lane as fmaf
        {
            const float4 b0 = __ldg(reinterpret_cast<const float4 *>(b + c0));
            const float4 b1 = __ldg(reinterpret_cast<const float4 *>(b + c0 + 4));
#pragma unroll
            for (int p = 0; p < PX; p++) {
                acc[p][0] = make_float2(b0.x, b0.y);
                acc[p][1] = make_float2(b0.z, b0.w);
                acc[p][2] = make_float2(b1.x, b1.y);
                acc[p][3] = make_float2(b1.z, b1.w);
            }
        }
        const size_t io = (size_t)blockIdx.y * (size_t)img_bytes;   // this block's image
        const __half *col = img_at(in, io) + c0;
#pragma unroll
        for (int ky = 0; ky < 3; ky++) {
            const int yy = y + ky - 1;
            if (yy < 0 || yy >= H) continue;
            float2 w[3][4];
#pragma unroll
            for (int kx = 0; kx < 3; kx++) {
                const float4 w0 = *reinterpret_cast<const float4 *>(ws + (ky * 3 + kx) * C + c0);
                const float4 w1 = *reinterpret_cast<const float4 *>(ws + (ky * 3 + kx) * C + c0 + 4);
                w[kx][0] = make_float2(w0.x, w0.y);
                w[kx][1] = make_float2(w0.z, w0.w);
                w[kx][2] = make_float2(w1.x, w1.y);
                w[kx][3] = make_float2(w1.z, w1.w);
            }
            const __half *rowp = col + (size_t)yy * W * C;
#pragma unroll
            for (int j = 0; j < PX + 2; j++) {
                // window column j: output pixel x + p reads it at tap kx = j - p, from source
                // column x + j - 1 + off (zero outside the row: the conv's zero padding)
                const uint4 ra = dw_col(rowp, x + j - 1 + offa, W, C);
                const uint4 rb = straddle ? dw_col(rowp, x + j - 1 + offb, W, C) : ra;
                uint4 raw;
                raw.x = __byte_perm(ra.x, rb.x, sel[0]);
                raw.y = __byte_perm(ra.y, rb.y, sel[1]);
                raw.z = __byte_perm(ra.z, rb.z, sel[2]);
                raw.w = __byte_perm(ra.w, rb.w, sel[3]);
                const __half2 *hv = reinterpret_cast<const __half2 *>(&raw);
                float2 f[4];
#pragma unroll
                for (int i = 0; i < 4; i++) f[i] = __half22float2(hv[i]);
#pragma unroll
                for (int p = 0; p < PX; p++) {
                    const int kx = j - p;
                    if (kx < 0 || kx > 2) continue;
#pragma unroll
                    for (int i = 0; i < 4; i++) acc[p][i] = __ffma2_rn(w[kx][i], f[i], acc[p][i]);
                }
            }
        }
        __half *rowo = img_at(out, io) + (size_t)y * W * C + c0;
#pragma unroll
        for (int p = 0; p < PX; p++) {
            if (x + p >= W) break;
            // a channel whose source column lies outside the row receives zero
            const bool va = x + p + offa >= 0 && x + p + offa < W;
            const bool vb = x + p + offb >= 0 && x + p + offb < W;
            __align__(16) __half o[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 g = gelu_exact2(acc[p][i]);
                o[2 * i] = __float2half_rn(g.x);
                o[2 * i + 1] = __float2half_rn(g.y);
            }
            if (!va || !vb) {
                const __half zero = __float2half_rn(0.0f);
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (k < split ? !va : !vb) o[k] = zero;
            }
            *reinterpret_cast<uint4 *>(rowo + (size_t)(x + p) * C) = *reinterpret_cast<const uint4 *>(o);
        }
    }
    pdl_trigger();
}

// Tiled form of the same operator: a block computes R output rows x 2*TP pixels x CS
// 8-channel chunks (TP * CS = 256 threads, two pixels of one chunk per thread and
// row).  The block's input rows y0-1 .. y0+R, the columns its gather reads (its pixels
// widened by the 3x3 halo and the layer's shift offsets) and its chunks are first
// copied into shared memory with cp.async (16 bytes a copy, zero-filled outside the
// image: the conv's zero padding), all of the block's copies in flight at once; the
// taps then read shared memory.  The direct form above reads every input row once for
// each output row that uses it, from L2, with the latency of its loads exposed.  The
// arithmetic (tap order, GELU, zero fill) is the direct form's, so both give the same
// bits.  Weights: [tap][half][chunk][4] fp32 in shared memory, so that the eight lanes
// of a shared-memory phase read 128 consecutive bytes.
struct DwTile {
    int R = 4;              // output rows per block
    int lcs = 4;            // log2 of the chunks per block (CS = 4, 8 or 16)
    int span = 0;           // tile columns: 2 * TP + 2 + (hi - lo)
    int lo = 0;             // lowest shift offset of the layer (<= 0)
    int ntx = 0, nty = 0;   // column and row tiles of one image (the slabs multiply them)
};

__global__ void __launch_bounds__(256, 3) dw_tile_kernel(const __half *in, int H, int W, int C, const float *wt,
                                                      const float *b, const ShiftSpec s, __half *out,
                                                      long long img_bytes, const DwTile tl) {
    constexpr int PX = kDwPx;
    extern __shared__ __align__(16) uint8_t dsm[];
    const int CS = 1 << tl.lcs, TW = PX * (256 >> tl.lcs);
    const int tx = blockIdx.x % tl.ntx, rest = blockIdx.x / tl.ntx;
    const int ty = rest % tl.nty, slab = rest / tl.nty;
    const int y0 = ty * tl.R, x0 = tx * TW, cs0 = slab * CS * 8;      // first channel of the slab
    float4 *ws = reinterpret_cast<float4 *>(dsm);                       // [9][2][CS] float4
    uint4 *tile = reinterpret_cast<uint4 *>(dsm + (size_t)9 * 2 * CS * sizeof(float4));   // [R+2][span][CS]
    // the weights are constant: staged before the wait on the previous kernel
    for (int i = threadIdx.x; i < 9 * 2 * CS; i += blockDim.x) {
        const int th = i >> tl.lcs, ch = i & (CS - 1);
        ws[i] = __ldg(reinterpret_cast<const float4 *>(wt + (th >> 1) * C + cs0 + ch * 8 + (th & 1) * 4));
    }
    pdl_wait();
    const size_t io = (size_t)blockIdx.y * (size_t)img_bytes;   // this block's image
    const __half *src = img_at(in, io);
    const int rowc = tl.span << tl.lcs;                          // copies per tile row
    for (int r = 0; r < tl.R + 2; r++) {
        const int gy = y0 - 1 + r;
        for (int j = threadIdx.x; j < rowc; j += blockDim.x) {
            const int gx = x0 + tl.lo - 1 + (j >> tl.lcs);
            const bool ok = gy >= 0 && gy < H && gx >= 0 && gx < W;
            const __half *g = ok ? src + ((size_t)gy * W + gx) * C + cs0 + (j & (CS - 1)) * 8 : src;
            const uint32_t d = (uint32_t)__cvta_generic_to_shared(tile + (size_t)r * rowc + j);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(g), "r"(ok ? 16 : 0)
                         : "memory");
        }
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    const int ch = threadIdx.x & (CS - 1), pr = threadIdx.x >> tl.lcs;
    const int x = x0 + PX * pr, c0 = cs0 + ch * 8;
    if (x < W) {
        const int ga = shift_group(s, c0), gb = shift_group(s, c0 + 7);
        const int offa = ga >= 0 ? s.offs[ga] : 0, offb = gb >= 0 ? s.offs[gb] : 0;
        const int split = ga == gb ? 8 : s.ends[ga] - c0;
        const bool straddle = split < 8;
        uint32_t sel[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            sel[k] = (2 * k < split ? 0x10u : 0x54u) | ((2 * k + 1 < split ? 0x32u : 0x76u) << 8);
        // tile column of window column 0 (source column x - 1 + off) for either offset
        const int ca = PX * pr + offa - tl.lo, cb = PX * pr + offb - tl.lo;
        const float4 b0 = __ldg(reinterpret_cast<const float4 *>(b + c0));
        const float4 b1 = __ldg(reinterpret_cast<const float4 *>(b + c0 + 4));
        for (int r = 0; r < tl.R; r++) {
            const int y = y0 + r;
            if (y >= H) break;
            float2 acc[PX][4];
#pragma unroll
            for (int p = 0; p < PX; p++) {
                acc[p][0] = make_float2(b0.x, b0.y);
                acc[p][1] = make_float2(b0.z, b0.w);
                acc[p][2] = make_float2(b1.x, b1.y);
                acc[p][3] = make_float2(b1.z, b1.w);
            }
#pragma unroll
            for (int ky = 0; ky < 3; ky++) {
                const int yy = y + ky - 1;
                if (yy < 0 || yy >= H) continue;
                float2 w[3][4];
#pragma unroll
                for (int kx = 0; kx < 3; kx++) {
                    const float4 w0 = ws[((ky * 3 + kx) * 2) * CS + ch];
                    const float4 w1 = ws[((ky * 3 + kx) * 2 + 1) * CS + ch];
                    w[kx][0] = make_float2(w0.x, w0.y);
                    w[kx][1] = make_float2(w0.z, w0.w);
                    w[kx][2] = make_float2(w1.x, w1.y);
                    w[kx][3] = make_float2(w1.z, w1.w);
                }
                const uint4 *trow = tile + (size_t)(r + ky) * rowc + ch;   // column c at trow[c << lcs]
#pragma unroll
                for (int j = 0; j < PX + 2; j++) {
                    const uint4 ra = trow[(ca + j) << tl.lcs];
                    const uint4 rb = straddle ? trow[(cb + j) << tl.lcs] : ra;
                    uint4 raw;
                    raw.x = __byte_perm(ra.x, rb.x, sel[0]);
                    raw.y = __byte_perm(ra.y, rb.y, sel[1]);
                    raw.z = __byte_perm(ra.z, rb.z, sel[2]);
                    raw.w = __byte_perm(ra.w, rb.w, sel[3]);
                    const __half2 *hv = reinterpret_cast<const __half2 *>(&raw);
                    float2 f[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) f[i] = __half22float2(hv[i]);
#pragma unroll
                    for (int p = 0; p < PX; p++) {
                        const int kx = j - p;
                        if (kx < 0 || kx > 2) continue;
#pragma unroll
                        for (int i = 0; i < 4; i++) acc[p][i] = __ffma2_rn(w[kx][i], f[i], acc[p][i]);
                    }
                }
            }
            __half *rowo = img_at(out, io) + (size_t)y * W * C + c0;
#pragma unroll
            for (int p = 0; p < PX; p++) {
                if (x + p >= W) break;
                const bool va = x + p + offa >= 0 && x + p + offa < W;
                const bool vb = x + p + offb >= 0 && x + p + offb < W;
                __align__(16) __half o[8];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 g = gelu_exact2(acc[p][i]);
                    o[2 * i] = __float2half_rn(g.x);
                    o[2 * i + 1] = __float2half_rn(g.y);
                }
                if (!va || !vb) {
                    const __half zero = __float2half_rn(0.0f);
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        if (k < split ? !va : !vb) o[k] = zero;
                }
                *reinterpret_cast<uint4 *>(rowo + (size_t)(x + p) * C) = *reinterpret_cast<const uint4 *>(o);
            }
        }
    }
    pdl_trigger();
}

__device__ __forceinline__ void bilin_coords(int Y, int n, int &a0, int &a1, float &f) {
    const float fy = ((float)Y + 0.5f) / 2.0f - 0.5f;
    const int y0 = (int)floorf(fy);
    f = fy - (float)y0;
    a0 = min(max(y0, 0), n - 1);
    a1 = min(max(y0 + 1, 0), n - 1);
}

// CH: 8-channel chunks per pixel when fixed at compile time (0: from the layout); the
// interpolation and the skip add run on packed fp32 pairs (FMUL2 / FFMA2 / FADD2)
template <int CH>
__global__ void __launch_bounds__(256) up_add_pad_kernel(const UpAddArgs a) {
    pdl_wait();
    const size_t io = (size_t)blockIdx.z * (size_t)a.img_bytes;   // this block's image
    const __half *dd = img_at(a.d, io);
    const int C = CH ? CH * 8 : a.out.C, H = a.out.H, W = a.out.W, chunks = CH ? CH : C / 8;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int Y = blockIdx.y;
    if (t < W * chunks) {
        const int X = t / chunks, ch = t - X * chunks;
        const int h = H / 2, w = W / 2, c0 = ch * 8;
        int ya, yb, xa, xb;
        float dy, dx;
        bilin_coords(Y, h, ya, yb, dy);
        bilin_coords(X, w, xa, xb, dx);
        const uint4 r00 = *reinterpret_cast<const uint4 *>(dd + ((size_t)ya * w + xa) * C + c0);
        const uint4 r01 = *reinterpret_cast<const uint4 *>(dd + ((size_t)ya * w + xb) * C + c0);
        const uint4 r10 = *reinterpret_cast<const uint4 *>(dd + ((size_t)yb * w + xa) * C + c0);
        const uint4 r11 = *reinterpret_cast<const uint4 *>(dd + ((size_t)yb * w + xb) * C + c0);
        const uint4 rs = *reinterpret_cast<const uint4 *>(img_at(act_ptr(a.skip, Y, X), io) + c0);
        const __half2 *h00 = reinterpret_cast<const __half2 *>(&r00), *h01 = reinterpret_cast<const __half2 *>(&r01);
        const __half2 *h10 = reinterpret_cast<const __half2 *>(&r10), *h11 = reinterpret_cast<const __half2 *>(&r11);
        const __half2 *hs = reinterpret_cast<const __half2 *>(&rs);
        const float2 wx0 = make_float2(1.0f - dx, 1.0f - dx), wx1 = make_float2(dx, dx);
        const float2 wy0 = make_float2(1.0f - dy, 1.0f - dy), wy1 = make_float2(dy, dy);
        __align__(16) __half2 o[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float2 top = __ffma2_rn(__half22float2(h01[k]), wx1, __fmul2_rn(__half22float2(h00[k]), wx0));
            const float2 bot = __ffma2_rn(__half22float2(h11[k]), wx1, __fmul2_rn(__half22float2(h10[k]), wx0));
            const float2 up = __ffma2_rn(bot, wy1, __fmul2_rn(top, wy0));
            o[k] = __float22half2_rn(__fadd2_rn(make_float2(fmaxf(up.x, 0.0f), fmaxf(up.y, 0.0f)), __half22float2(hs[k])));
        }
        act_store(a.out, Y, X, c0, reinterpret_cast<const __half *>(o), 8, io);
    }
    pdl_trigger();
}

// Lane groups for the per-pixel LayerNorm kernels: LP lanes (16 or 32) share a
// pixel (token), each lane owning NCH chunks of 8 channels (16-byte accesses).
template <int LP>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int m = LP / 2; m; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

__device__ __forceinline__ void load8f(const float *p, float *v) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p)), b = __ldg(reinterpret_cast<const float4 *>(p + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ uint4 pack8h(const float *v) {
    uint4 u;
    __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
    for (int k = 0; k < 4; k++) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
    return u;
}

__device__ __forceinline__ uint32_t word_of(const uint4 &u, int i) {
    return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}

// Halves [0, n) (0 < n < 8) of the packed chunk u to dst (16-byte aligned): one
// naturally aligned store each of 4, 2 and 1 halves, as n's bits ask.
__device__ __forceinline__ void store_prefix(__half *dst, const uint4 &u, int n) {
    int k = 0;
    if (n & 4) {
        *reinterpret_cast<uint2 *>(dst) = make_uint2(u.x, u.y);
        k = 4;
    }
    if (n & 2) {
        *reinterpret_cast<uint32_t *>(dst + k) = word_of(u, k >> 1);
        k += 2;
    }
    if (n & 1) *reinterpret_cast<unsigned short *>(dst + k) = (unsigned short)(word_of(u, k >> 1) & 0xFFFFu);
}

// Halves [n, 8) (0 < n < 8) of the packed chunk u to dst + n (dst 16-byte aligned).
__device__ __forceinline__ void store_suffix(__half *dst, const uint4 &u, int n) {
    int k = n;
    if (k & 1) {
        *reinterpret_cast<unsigned short *>(dst + k) = (unsigned short)(word_of(u, k >> 1) >> 16);
        k++;
    }
    if (k & 2) {
        *reinterpret_cast<uint32_t *>(dst + k) = word_of(u, k >> 1);
        k += 2;
    }
    if (k & 4) *reinterpret_cast<uint2 *>(dst + k) = make_uint2(u.z, u.w);
}

// H-shift scatter of channels [c0, c0+8) of token pixel (y, x) of a LAY_PLAIN
// tensor: one 16-byte store when the chunk lies in one channel group; a chunk
// across a group boundary goes out as its two parts, each in at most three
// aligned stores (groups narrower than a chunk: per channel pair).
__device__ __forceinline__ void shift_store8(const Act &a, const ShiftSpec &s, int y, int x, int c0, const float *v,
                                             size_t io) {
    const int g0 = shift_group(s, c0), g7 = shift_group(s, c0 + 7);
    const uint4 zero = make_uint4(0, 0, 0, 0);
    __half *base = img_at(a.p, io);
    if (g0 == g7) {
        int dy = y;
        bool z = false;
        if (g0 >= 0) dy = shift_dest(y, s.offs[g0], a.H, &z);
        *reinterpret_cast<uint4 *>(base + ((size_t)dy * a.W + x) * a.C + c0) = z ? zero : pack8h(v);
    } else if (!s.narrow) {
        // channels [c0, ends[g0]) in group g0 (g0 >= 0 here), the rest in g7 (-1: unshifted)
        const uint4 u = pack8h(v);
        const int split = s.ends[g0] - c0;
        bool za, zb = false;
        const int da = shift_dest(y, s.offs[g0], a.H, &za);
        const int db = g7 >= 0 ? shift_dest(y, s.offs[g7], a.H, &zb) : y;
        store_prefix(base + ((size_t)da * a.W + x) * a.C + c0, za ? zero : u, split);
        store_suffix(base + ((size_t)db * a.W + x) * a.C + c0, zb ? zero : u, split);
    } else {
#pragma unroll
        for (int k = 0; k < 4; k++) shift_store2(a, s, 2, y, x, c0 + 2 * k, v[2 * k], v[2 * k + 1], io);
    }
}

// out = relu(up(d)) + skip as tokens, then LN2(out) scattered with the H shift;
// LP lanes per output pixel, 8 channels per lane and chunk.
template <int LP, int NCH>
__global__ void __launch_bounds__(256) up_add_tok_kernel(const UpAddArgs a) {
    pdl_wait();
    const size_t io = (size_t)blockIdx.z * (size_t)a.img_bytes;   // this block's image
    const __half *dd = img_at(a.d, io);
    const int C = a.out.C, H = a.out.H, W = a.out.W, nchunk = C >> 3;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    const int p = gid / LP, l = gid - p * LP;
    const bool valid = p < H * W;              // invalid groups still join the shuffles
    const int pp = valid ? p : 0;
    const int Y = pp / W, X = pp - Y * W;
    const int h = H / 2, w = W / 2;
    int ya, yb, xa, xb;
    float dy, dx;
    bilin_coords(Y, h, ya, yb, dy);
    bilin_coords(X, w, xa, xb, dx);
    const __half *d00 = dd + ((size_t)ya * w + xa) * C, *d01 = dd + ((size_t)ya * w + xb) * C;
    const __half *d10 = dd + ((size_t)yb * w + xa) * C, *d11 = dd + ((size_t)yb * w + xb) * C;
    const __half *sk = img_at(act_ptr(a.skip, Y, X), io);
    __half *outp = img_at(a.out.p, io);
    const float2 wx0 = make_float2(1.0f - dx, 1.0f - dx), wx1 = make_float2(dx, dx);
    const float2 wy0 = make_float2(1.0f - dy, 1.0f - dy), wy1 = make_float2(dy, dy);
    float v[NCH][8];
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; k++) {
        const int ch = l + LP * k;
#pragma unroll
        for (int e = 0; e < 8; e++) v[k][e] = 0.f;
        if (ch < nchunk) {
            const int c0 = ch * 8;
            const uint4 r00 = *reinterpret_cast<const uint4 *>(d00 + c0), r01 = *reinterpret_cast<const uint4 *>(d01 + c0);
            const uint4 r10 = *reinterpret_cast<const uint4 *>(d10 + c0), r11 = *reinterpret_cast<const uint4 *>(d11 + c0);
            const uint4 rs = *reinterpret_cast<const uint4 *>(sk + c0);
            const __half2 *h00 = reinterpret_cast<const __half2 *>(&r00), *h01 = reinterpret_cast<const __half2 *>(&r01);
            const __half2 *h10 = reinterpret_cast<const __half2 *>(&r10), *h11 = reinterpret_cast<const __half2 *>(&r11);
            const __half2 *hs = reinterpret_cast<const __half2 *>(&rs);
            // the interpolation and the skip add on packed fp32 pairs
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 top = __ffma2_rn(__half22float2(h01[e]), wx1, __fmul2_rn(__half22float2(h00[e]), wx0));
                const float2 bot = __ffma2_rn(__half22float2(h11[e]), wx1, __fmul2_rn(__half22float2(h10[e]), wx0));
                const float2 up = __ffma2_rn(bot, wy1, __fmul2_rn(top, wy0));
                const float2 r = __fadd2_rn(make_float2(fmaxf(up.x, 0.0f), fmaxf(up.y, 0.0f)), __half22float2(hs[e]));
                v[k][2 * e] = r.x;
                v[k][2 * e + 1] = r.y;
                sum += r.x + r.y;
            }
            if (valid)
                *reinterpret_cast<uint4 *>(outp + a.out.row(Y, X) * C + c0) = pack8h(v[k]);
        }
    }
    const float mean = group_sum<LP>(sum) / C;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; k++)
        if (l + LP * k < nchunk)
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float dd = v[k][e] - mean;
                q += dd * dd;
            }
    const float rstd = rsqrtf(group_sum<LP>(q) / C + a.eps);
#pragma unroll
    for (int k = 0; k < NCH; k++) {
        const int ch = l + LP * k;
        if (ch < nchunk && valid) {
            const int c0 = ch * 8;
            float g[8], bb[8], o[8];
            load8f(a.g + c0, g);
            load8f(a.b + c0, bb);
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = (v[k][e] - mean) * rstd * g[e] + bb[e];
            shift_store8(a.h, a.shift, Y, X, c0, o, io);
        }
    }
    pdl_trigger();
}

// Split-K finish, LP lanes per token, 8 channels per lane and chunk: the k-split
// partials summed in order (k ascending), + bias (+ residual), LN1 -> out,
// [LN2 -> out2 with the H shift].
template <int LP, int NCH>
__global__ void __launch_bounds__(256) ln_finalize_kernel(const LnFinalizeArgs a) {
    const int N = a.N, nchunk = N >> 3;
    const int T = a.H * a.W;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    const int t = gid / LP, l = gid - t * LP;
    const bool valid = t < T;                  // invalid groups still join the shuffles
    const int tt = valid ? t : 0;
    const int y = tt / a.W, x = tt - y * a.W;
    float v[NCH][8];
#pragma unroll
    for (int k = 0; k < NCH; k++) {
        const int ch = l + LP * k;
        if (ch < nchunk) load8f(a.bias + ch * 8, v[k]);
        else
#pragma unroll
            for (int e = 0; e < 8; e++) v[k][e] = 0.f;
    }
    pdl_wait();   // (the bias is constant: read before the wait on the partials' producer)
    const size_t io = (size_t)blockIdx.z * (size_t)a.img_bytes;   // this block's image
    // (unrolled: the loads of several partials in flight at once; the sum stays in k order)
#pragma unroll 4
    for (int ks = 0; ks < a.ksplit; ks++) {
        const float *pk = img_at(a.partial, io) + ((size_t)ks * T + tt) * N;
#pragma unroll
        for (int k = 0; k < NCH; k++) {
            const int ch = l + LP * k;
            if (ch < nchunk) {
                float pv[8];
                load8f(pk + ch * 8, pv);
#pragma unroll
                for (int e = 0; e < 8; e++) v[k][e] += pv[e];
            }
        }
    }
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; k++) {
        const int ch = l + LP * k;
        if (ch < nchunk) {
            if (a.res) {
                float r[8];
                load16h8(img_at(a.res, io) + (size_t)tt * N + ch * 8, r);
#pragma unroll
                for (int e = 0; e < 8; e++) v[k][e] += r[e];
            }
#pragma unroll
            for (int e = 0; e < 8; e++) sum += v[k][e];
        }
    }
    const float mean = group_sum<LP>(sum) / N;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; k++)
        if (l + LP * k < nchunk)
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const float dd = v[k][e] - mean;
                q += dd * dd;
            }
    const float rstd = rsqrtf(group_sum<LP>(q) / N + a.eps1);
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; k++) {
        const int ch = l + LP * k;
        if (ch < nchunk) {
            const int c0 = ch * 8;
            float g[8], bb[8];
            load8f(a.g1 + c0, g);
            load8f(a.b1 + c0, bb);
#pragma unroll
            for (int e = 0; e < 8; e++) {
                v[k][e] = (v[k][e] - mean) * rstd * g[e] + bb[e];
                s2 += v[k][e];
            }
            if (valid) {
                const uint4 u = pack8h(v[k]);
                act_store(a.out, y, x, c0, reinterpret_cast<const __half *>(&u), 8, io);
            }
        }
    }
    if (a.ln2) {
        const float mean2 = group_sum<LP>(s2) / N;
        float q2 = 0.f;
#pragma unroll
        for (int k = 0; k < NCH; k++)
            if (l + LP * k < nchunk)
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float dd = v[k][e] - mean2;
                    q2 += dd * dd;
                }
        const float rstd2 = rsqrtf(group_sum<LP>(q2) / N + a.eps2);
#pragma unroll
        for (int k = 0; k < NCH; k++) {
            const int ch = l + LP * k;
            if (ch < nchunk && valid) {
                const int c0 = ch * 8;
                float g[8], bb[8], o[8];
                load8f(a.g2 + c0, g);
                load8f(a.b2 + c0, bb);
#pragma unroll
                for (int e = 0; e < 8; e++) o[e] = (v[k][e] - mean2) * rstd2 * g[e] + bb[e];
                shift_store8(a.out2, a.shift, y, x, c0, o, io);
            }
        }
    }
    pdl_trigger();
}

__global__ void bgr2nhwc_kernel(const ImgSpec im, float *x, int H, int W) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)H * W) return;
    const int py = (int)(idx / W), px = (int)(idx - (long long)py * W);
#pragma unroll
    for (int c = 0; c < 3; c++) x[idx * 3 + c] = img_val(im, py, px, c);
}

__global__ void div6_kernel(const float *x, const float *s, size_t npx, float *out) {
    const size_t p = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= npx) return;
#pragma unroll
    for (int c = 0; c < 3; c++) {
        const float v = x[p * 3 + c];
        const float d = s[p * 3 + c] > 1e-6f ? s[p * 3 + c] : 1e-6f;
        float r = v / d;
        r = r < 0.0f ? 0.0f : (r > 1.0f ? 1.0f : r);
        out[p * 6 + c] = v;
        out[p * 6 + 3 + c] = r;
    }
}

__global__ void nhwc2bgr_kernel(const float *y, int W, int ph, int pw, uint8_t *dst, int w, int h, int dst_stride,
                                int bpp, int swap, const uint8_t *alpha, int alpha_stride) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)w * h) return;
    const int r = (int)(idx / w), c = (int)(idx - (long long)r * w);
    const float *v = y + ((size_t)(r + ph) * W + (c + pw)) * 3;
    uint8_t q[3];
#pragma unroll
    for (int k = 0; k < 3; k++) {
        float f = v[k] * 255.0f + 0.5f;
        f = f < 0.0f ? 0.0f : (f > 255.0f ? 255.0f : f);
        q[k] = (uint8_t)f;
    }
    const int ob = swap ? 2 : 0;
    uint8_t *d = dst + (size_t)r * dst_stride + (size_t)c * bpp;
    uint8_t al = bpp == 4 ? alpha[(size_t)r * alpha_stride + (size_t)c * 4 + 3] : 0;
    d[ob] = q[0];
    d[1] = q[1];
    d[2 - ob] = q[2];
    if (bpp == 4) d[3] = al;
}

// One block per (row, 256-pixel segment) of the padded image.  The segment's source bytes --
// part of one row of the top/left replicate-padded image, a contiguous byte range of the
// tight device copy -- are read with aligned 16-byte loads into shared memory (the device
// copy carries 16 bytes of slack past its end, so the last word stays inside the
// allocation), then each thread builds its pixel's 16-channel row [x, x, 0] and stores it as
// two 16-byte stores (plus the reflect-border copies).
constexpr int kStemInPx = 256;

__global__ void __launch_bounds__(kStemInPx) stem_in_kernel(const ImgSpec im, Act si, int *err, long long img_bytes) {
    __shared__ __align__(16) uint8_t seg[kStemInPx * 4 + 32];
    pdl_wait();
    const size_t io = (size_t)blockIdx.z * (size_t)img_bytes;   // this block's image
    si.p = img_at(si.p, io);
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && err) *img_at(err, io) = 0;   // the enhancement's first kernel
    const int y = blockIdx.y, x0 = blockIdx.x * kStemInPx, x = x0 + (int)threadIdx.x;
    const int sy = max(y - im.ph, 0);
    const int sx_lo = max(x0 - im.pw, 0);
    const int sx_hi = max(min(x0 + kStemInPx - 1 - im.pw, im.w - 1), sx_lo);
    const uintptr_t rowp = reinterpret_cast<uintptr_t>(im.src) + io + (size_t)sy * im.stride;
    const uintptr_t a_lo = (rowp + (size_t)sx_lo * im.bpp) & ~uintptr_t(15);
    const uintptr_t a_hi = rowp + (size_t)(sx_hi + 1) * im.bpp;   // exclusive
    const int nwords = (int)((a_hi - a_lo + 15) >> 4);           // <= 66
    for (int i = threadIdx.x; i < nwords; i += kStemInPx)
        reinterpret_cast<uint4 *>(seg)[i] = reinterpret_cast<const uint4 *>(a_lo)[i];
    __syncthreads();
    if (x < si.W) {
        const int sx = max(x - im.pw, 0);
        const uint8_t *p = seg + (rowp + (size_t)sx * im.bpp - a_lo);
        const int ob = im.swap ? 2 : 0;
        const __half b = __ushort2half_rn(p[ob]), g = __ushort2half_rn(p[1]), r = __ushort2half_rn(p[2 - ob]);
        const __half z = __ushort2half_rn(0);
        __align__(16) __half v[16] = {b, g, r, b, g, r, z, z, z, z, z, z, z, z, z, z};
        act_store(si, y, x, 0, v, 16);
    }
    pdl_trigger();
}

inline int grid_for(long long n, int bs) { return (int)((n + bs - 1) / bs); }

thread_local cudaError_t t_last_launch = cudaSuccess;

inline int launch_status() {
    t_last_launch = cudaGetLastError();
    return t_last_launch == cudaSuccess ? 0 : -1;
}

}  // namespace

const char *last_launch_error() { return cudaGetErrorString(t_last_launch); }

}  // namespace gcdr
#include <cstdlib>
namespace gcdr {
bool pdl_enabled() {
    static const bool on = [] { const char *v = std::getenv("GCDR_CUDA_PDL"); return !(v && v[0] == '0'); }();
    return on;
}

int stem_in_launch(const ImgSpec &im, const Act &si, int *err, cudaStream_t st, int nimg, long long img_bytes) {
    if (si.C != 16 || si.kind != LAY_PADREFL || im.stride != im.w * im.bpp) return -2;
    if (nimg < 1 || nimg > 65535 || (nimg > 1 && (img_bytes <= 0 || img_bytes % 16))) return -2;
    launch_pdl(stem_in_kernel, dim3(grid_for(si.W, kStemInPx), si.H, nimg), dim3(kStemInPx), 0, st, im, si, err,
               img_bytes);
    return launch_status();
}

void pack_stem_conv(const float *w, int c1, int cin, __half *out) {
    for (int i = 0; i < c1 * 9 * 16; i++) out[i] = __float2half_rn(0.0f);
    for (int n = 0; n < c1; n++)
        for (int tap = 0; tap < 9; tap++)
            for (int ci = 0; ci < cin; ci++) {
                const float v = w[((size_t)n * cin + ci) * 9 + tap];
                __half *o = out + ((size_t)n * 9 + tap) * 16;
                if (ci < 3) {
                    const float s = v / 255.0f;
                    const __half hi = __float2half_rn(s);
                    o[ci] = hi;
                    o[3 + ci] = __float2half_rn(s - __half2float(hi));
                } else {
                    const int c = ci - 3;
                    const __half hi = __float2half_rn(v);
                    o[6 + c] = hi;
                    o[9 + c] = hi;
                    o[12 + c] = __float2half_rn(v - __half2float(hi));
                }
            }
}

int stem_launch(const StemArgs &a, cudaStream_t st) {
    const long long n = (long long)(a.H / 2) * (a.W / 2);
    if (a.cin == 3 && a.c1 == 16) launch_pdl(stem_kernel<3, 16>, dim3(grid_for(n, 128)), dim3(128), 0, st, a);
    else if (a.cin == 6 && a.c1 == 32) launch_pdl(stem_kernel<6, 32>, dim3(grid_for(n, 128)), dim3(128), 0, st, a);
    else if (a.cin == 3 && a.c1 == 32) launch_pdl(stem_kernel<3, 32>, dim3(grid_for(n, 128)), dim3(128), 0, st, a);
    else if (a.cin == 6 && a.c1 == 16) launch_pdl(stem_kernel<6, 16>, dim3(grid_for(n, 128)), dim3(128), 0, st, a);
    else return -2;
    return launch_status();
}

int head_launch(const HeadArgs &a, cudaStream_t st) {
    const long long n = a.is_dr ? (long long)a.img.w * a.img.h : (long long)a.H * a.W;
    const int g = grid_for(n, 128);
    if (!a.is_dr) {
        if (a.cin == 3 && a.c1 == 16) launch_pdl(head_kernel<3, 16, false>, dim3(g), dim3(128), 0, st, a);
        else if (a.cin == 3 && a.c1 == 32) launch_pdl(head_kernel<3, 32, false>, dim3(g), dim3(128), 0, st, a);
        else return -2;
    } else {
        if (a.cin == 6 && a.c1 == 32) launch_pdl(head_kernel<6, 32, true>, dim3(g), dim3(128), 0, st, a);
        else if (a.cin == 6 && a.c1 == 16) launch_pdl(head_kernel<6, 16, true>, dim3(g), dim3(128), 0, st, a);
        else return -2;
    }
    return launch_status();
}

int dw_gelu_shift_launch(const __half *in, int H, int W, int C, const float *wt, const float *b, const ShiftSpec &s,
                         __half *out, cudaStream_t st, int nimg, long long img_bytes) {
    if (C % 8 || C > kDwMaxC) return -2;
    if (nimg < 1 || nimg > 65535 || (nimg > 1 && (img_bytes <= 0 || img_bytes % 16))) return -2;
    // the kernel gives a chunk of 8 channels at most two shift groups (a group boundary
    // inside it): shift groups that put three into one chunk are rejected
    for (int c0 = 0; c0 < C; c0 += 8) {
        auto group = [&](int c) {
            for (int g = 0; g < s.ngroups; g++)
                if (c < s.ends[g]) return g;
            return -1;
        };
        const int ga = group(c0), gb = group(c0 + 7);
        for (int c = c0; c < c0 + 8; c++)
            if (group(c) != ga && group(c) != gb) return -2;
    }
    // the tiled form when the chunks split into slabs of 4, 8 or 16 and the tile fits
    const int nchunk = C / 8;
    DwTile tl;
    tl.lcs = nchunk % 16 == 0 ? 4 : nchunk % 8 == 0 ? 3 : nchunk % 4 == 0 ? 2 : -1;
    if (tl.lcs > 0) {
        int lo = 0, hi = 0;
        for (int g = 0; g < s.ngroups; g++) {
            lo = std::min(lo, s.offs[g]);
            hi = std::max(hi, s.offs[g]);
        }
        static const int nsm = [] {
            int d = 0, n = 148;
            if (cudaGetDevice(&d) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
            return n;
        }();
        const int CS = 1 << tl.lcs, TW = kDwPx * (256 >> tl.lcs);
        tl.lo = lo;
        tl.span = TW + 2 + (hi - lo);
        tl.ntx = (W + TW - 1) / TW;
        // four output rows a block (the tile's two halo rows cost half its loads) while
        // that still fills the GPU with three blocks per SM; fewer for small grids
        long long blocks = 0;
        for (tl.R = 4;; tl.R /= 2) {
            tl.nty = (H + tl.R - 1) / tl.R;
            blocks = (long long)tl.ntx * tl.nty * (nchunk / CS);
            if (tl.R == 1 || blocks * nimg >= 3LL * nsm) break;
        }
        const size_t smem = (size_t)9 * 2 * CS * 16 + (size_t)(tl.R + 2) * tl.span * CS * 16;
        if (hi - lo <= 64 && smem <= 96 * 1024 && blocks < (1ll << 31)) {
            // one cap for every launch (the attribute is per kernel and device)
            if (cudaFuncSetAttribute(dw_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024) !=
                cudaSuccess)
                return -1;
            launch_pdl(dw_tile_kernel, dim3((unsigned)blocks, nimg), dim3(256), smem, st, in, H, W, C, wt, b, s, out,
                       img_bytes, tl);
            return launch_status();
        }
    }
    const int blocks = grid_for((long long)((W + kDwPx - 1) / kDwPx) * (C / 8) * H, 128);
    launch_pdl(dw_gelu_shift_kernel, dim3(blocks, nimg), dim3(128), (size_t)9 * C * sizeof(float), st, in, H, W, C,
               wt, b, s, out, img_bytes);
    return launch_status();
}

int up_add_launch(const UpAddArgs &a, cudaStream_t st) {
    const int C = a.out.C;
    if (a.nimg < 1 || a.nimg > 65535 || (a.nimg > 1 && (a.img_bytes <= 0 || a.img_bytes % 16))) return -2;
    if (!a.tokens) {
        if (C % 8) return -2;
        const dim3 grid(grid_for((long long)a.out.W * (C / 8), 256), a.out.H, a.nimg);
        switch (C) {
            case 16: launch_pdl(up_add_pad_kernel<2>, grid, dim3(256), 0, st, a); break;
            case 32: launch_pdl(up_add_pad_kernel<4>, grid, dim3(256), 0, st, a); break;
            case 64: launch_pdl(up_add_pad_kernel<8>, grid, dim3(256), 0, st, a); break;
            default: launch_pdl(up_add_pad_kernel<0>, grid, dim3(256), 0, st, a); break;
        }
    } else {
        if (C % 8 || C > 512) return -2;
        const int nchunk = C / 8;
        const int LP = nchunk <= 16 ? 16 : 32;
        const long long n = (long long)a.out.H * a.out.W * LP;
        const dim3 grid(grid_for(n, 256), 1, a.nimg);
        if (LP == 16) launch_pdl(up_add_tok_kernel<16, 1>, grid, dim3(256), 0, st, a);
        else if (nchunk <= 32) launch_pdl(up_add_tok_kernel<32, 1>, grid, dim3(256), 0, st, a);
        else launch_pdl(up_add_tok_kernel<32, 2>, grid, dim3(256), 0, st, a);
    }
    return launch_status();
}

int ln_finalize_launch(const LnFinalizeArgs &a, cudaStream_t st) {
    if (a.N % 8 || a.N > 512 || a.ksplit < 1) return -2;
    if (a.nimg < 1 || a.nimg > 65535 || (a.nimg > 1 && (a.img_bytes <= 0 || a.img_bytes % 16))) return -2;
    const int nchunk = a.N / 8;
    const int LP = nchunk <= 16 ? 16 : 32;
    const long long n = (long long)a.H * a.W * LP;
    const dim3 grid(grid_for(n, 256), 1, a.nimg);
    if (LP == 16) launch_pdl(ln_finalize_kernel<16, 1>, grid, dim3(256), 0, st, a);
    else if (nchunk <= 32) launch_pdl(ln_finalize_kernel<32, 1>, grid, dim3(256), 0, st, a);
    else launch_pdl(ln_finalize_kernel<32, 2>, grid, dim3(256), 0, st, a);
    return launch_status();
}

int k_bgr2nhwc(const uint8_t *src, int w, int h, int stride, int fmt, float *x, int ph, int pw, cudaStream_t st) {
    ImgSpec im;
    im.src = src;
    im.w = w;
    im.h = h;
    im.stride = stride;
    im.bpp = fmt >= 2 ? 4 : 3;
    im.swap = (fmt == 1 || fmt == 3) ? 1 : 0;
    im.ph = ph;
    im.pw = pw;
    const long long n = (long long)(h + ph) * (w + pw);
    bgr2nhwc_kernel<<<grid_for(n, 256), 256, 0, st>>>(im, x, h + ph, w + pw);
    return launch_status();
}

int k_div6(const float *x, const float *s, size_t npx, float *out6, cudaStream_t st) {
    div6_kernel<<<grid_for((long long)npx, 256), 256, 0, st>>>(x, s, npx, out6);
    return launch_status();
}

int k_nhwc2bgr(const float *y, int H, int W, int ph, int pw, uint8_t *dst, int w, int h, int dst_stride, int fmt,
               const uint8_t *alpha, int alpha_stride, cudaStream_t st) {
    (void)H;
    nhwc2bgr_kernel<<<grid_for((long long)w * h, 256), 256, 0, st>>>(
        y, W, ph, pw, dst, w, h, dst_stride, fmt >= 2 ? 4 : 3, (fmt == 1 || fmt == 3) ? 1 : 0, alpha, alpha_stride);
    return launch_status();
}

}  // namespace gcdr
