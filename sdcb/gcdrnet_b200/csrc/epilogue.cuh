// epilogue.cuh -- per-pixel epilogues of the implicit-GEMM convolutions.
//
// The GEMM tile is 128 output positions x Nsub channels (a slice [n0, n0+Nsub)
// of the layer's N).  Thread `row` (0..127) of the four epilogue warps owns
// one position; its accumulators are read 32 (or 16) columns at a time through
// a Loader (TMEM for the tcgen05 kernel, global scratch for the SIMT
// reference), so the same code finishes both.  Loader loads are
// warp-synchronous (tcgen05.ld is .sync.aligned): control flow around them is
// uniform; per-thread validity only masks stores.
//
// Modes (the fusions the reference's CPU plan makes, EngineTests.cs:79-141):
//   EPI_PLAIN    y = acc + bias [relu]                        decoder convs, fc1
//   EPI_POOL     y = relu(maxpool2x2(acc + bias))             encoder conv+pool+relu (gc#23-25):
//                a unit holds the two conv rows of a pooled row in two accumulators, so a
//                thread maxes its own pair of rows and one shuffle finishes the 2x2 window
//   EPI_LN2      y0 = LN1(acc + bias) -> out (tokens);        patch embed + its norm (gc#34-37)
//                h = LN2(y0) -> out2 with the H-shift scatter  and the block's norm2 + shift (gc#38-44)
//   EPI_RESLN    y = LN(acc + bias + res) -> out              fc2 + residual + norm3 (gc#127-130)
//   EPI_PARTIAL  fp32 partial sums of one k-split -> partial[k][token][N] (no bias); a token
//                kernel (ln_finalize) sums the splits in order and applies the LN modes above,
//                for layers with too few tiles to fill the GPU.
#pragma once
#include "common.cuh"

namespace gcdr {

enum EpiMode : int { EPI_PLAIN = 0, EPI_POOL = 1, EPI_LN2 = 2, EPI_RESLN = 3, EPI_PARTIAL = 4, EPI_HEAD = 5 };

// Stem input layout: LAY_PADREFL [H+2][W+2][16] fp16 per padded image pixel,
//   GC: [xb, xg, xr, xb, xg, xr, 0 x 10]
//   DR: [xb, xg, xr, xb, xg, xr, rh x3, rl x3, rh x3, 0]
// with x the u8 pixel (exact in fp16) and r = rh + rl the division-corrected
// image.  The stem weights pair with it as [w'_hi, w'_lo, wr_hi, wr_hi, wr_lo]
// (w' = w_x / 255), so one fp16 GEMM with fp32 accumulation yields
// sum x*w_x/255 + r*w_r to fp32-level accuracy (the r_lo*wr_lo term, ~2^-22
// relative, is dropped).
constexpr int kStemInC = 16;

// UpHead epilogue (EPI_HEAD): s = relu(bilinear x2 of dec5) + relu(conv + bias),
// o = sigmoid(fb + fw . s), then GC: I_sm -> r = clamp(x / max(I_sm, 1e-6), 0, 1)
// written as the DR stem input (the div6 stage); DR: crop, round, R/B swap and
// alpha from the source into the caller's u8 image.
struct HeadParams {
    const __half *dec5 = nullptr;   // [H/2][W/2][C1] fp16 tokens
    // the 1x1 head and the stem bias by value: kernel-parameter (constant bank)
    // operands of the per-pixel FMAs instead of per-pixel loads
    float fw[3 * 32];               // 1x1 [3][C1]
    float fb[3];
    float b1[32];                   // stem conv bias [C1]
    Act si_in;                      // this net's stem input (GC reads x from it)
    Act si_out;                     // GC: the DR stem input
    float *r_out = nullptr, *ism_out = nullptr, *y_out = nullptr;   // debug [H][W][3] fp32
    ImgSpec img;                    // DR: destination format and the alpha source
    uint8_t *dst = nullptr;
    int is_dr = 0;
};

constexpr int kMaxBiasConst = 512;

struct EpiParams {
    const float *bias = nullptr;     // [N] (indexed with the slice offset)
    // the same bias by value (kernel-parameter constant bank): the epilogues read
    // these, a per-element global load being a full cache round trip per column
    float bias_c[kMaxBiasConst];
    int relu = 0;                    // EPI_PLAIN: relu after the bias
    Act out;                         // primary output (logical dims = conv or pooled output)
    // LN modes
    const float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
    // EPI_RESLN with 3 * N <= kMaxBiasConst: g1 and b1 by value in bias_c[N, 2N) and
    // bias_c[2N, 3N) (constant-bank operands instead of two loads per element)
    int ln_c = 0;
    float eps1 = 1e-5f, eps2 = 1e-5f;
    Act out2;                        // EPI_LN2: LN2 output, LAY_PLAIN tokens, H-shift scatter
    ShiftSpec shift;
    const __half *res = nullptr;     // EPI_RESLN residual tokens [T][N]
    float *partial = nullptr;        // EPI_PARTIAL: [ksplit][T][N] fp32
    HeadParams head;                 // EPI_HEAD
};

// Geometry of the output grid: q = y * pitch + x over a flat row space.
//   plain: work units of rt consecutive 128-row tiles (ntiles tiles in all);
//   pool:  work units of two conv rows (2*y2, 2*y2+1) x 128*rt pixels.
struct TileGeom {
    int pool = 0;
    int pitch = 0;        // grid rows per image row (>= out_w; extra columns are discarded)
    int conv_h = 0, conv_w = 0;   // conv output dims (valid region of the grid)
    int ntiles = 0;       // plain: 128-row tiles
};

// Work units along M for `rt` (tiles per unit, or 128-pixel segments per pooled row).
__host__ __device__ inline int m_units(const TileGeom &tg, int rt) {
    if (tg.pool) return (tg.conv_h / 2) * ((tg.conv_w + 128 * rt - 1) / (128 * rt));
    return (tg.ntiles + rt - 1) / rt;
}

// Reads columns [c0, c0 + w) (w = 32 or 16) of this thread's accumulator row.
template <class L>
__device__ __forceinline__ void load_cols(L &ld, int c0, int w, float *v) {
    if (w == 32) ld.load32(c0, v);
    else ld.load16(c0, v);
}

// t = acc + bias (+ residual `res`, this image's tokens) of columns [c0, c0+w) of the row.
template <class L>
__device__ __forceinline__ void row_vals(L &ld, const EpiParams &ep, const __half *res, int N, long long tok,
                                         bool use_res, int c0, int w, float *v) {
    load_cols(ld, c0, w, v);
    float r[32];
    if (use_res) {
        load16h(res + tok * N + c0, r);
        if (w == 32) load16h(res + tok * N + c0 + 16, r + 16);
    }
#pragma unroll
    for (int k = 0; k < 32; k++)
        if (k < w) v[k] += ep.bias_c[c0 + k] + (use_res ? r[k] : 0.0f);
}

// PLAIN epilogue of output pixel (y, x): bias [+ relu] -> fp16 store of the
// column chunks c0 = part*cw, (part + nparts)*cw, ... (several warps may share a row).
// io: byte offset of the unit's image (batched launches; 0 for image 0).
template <class L>
__device__ __forceinline__ void epilogue_plain_yx(const EpiParams &ep, const TileGeom &tg, int y, int x, int n0,
                                                  int Nsub, L &ld, int part, int nparts, const float *bias,
                                                  size_t io = 0) {
    float v[32];
    const int cw = (Nsub % 32 == 0) ? 32 : 16;
    const bool valid = y < tg.conv_h && x < tg.conv_w;
    for (int c0 = part * cw; c0 < Nsub; c0 += nparts * cw) {
        load_cols(ld, c0, cw, v);
        if (valid) {
            __align__(16) __half h[32];
#pragma unroll
            for (int k = 0; k < 32; k++) {
                if (k < cw) {
                    float t = v[k] + bias[n0 + c0 + k];
                    h[k] = __float2half_rn(ep.relu ? fmaxf(t, 0.0f) : t);
                }
            }
            act_store(ep.out, y, x, n0 + c0, h, cw, io);
        }
    }
}

// PLAIN epilogue of one warp's 32 consecutive pixels (y, x0w + lane), channels [c0, c0 + CW),
// stored through the warp's staging buffer `stg` (32 * CW * 2 bytes): one store instruction
// covers eight pixels' chunks instead of one chunk per lane.  Warp-collective (TMEM).
template <int CW, class L>
__device__ __forceinline__ void epilogue_plain_staged(const EpiParams &ep, const TileGeom &tg, int y, int x0w, int c0,
                                                      L &ld, const float *bias, uint8_t *stg, size_t io) {
    float v[32];
    load_cols(ld, c0, CW, v);
    if (y >= tg.conv_h) return;                       // (uniform over the warp: one output row)
    __align__(16) __half h[CW];
#pragma unroll
    for (int k = 0; k < CW; k++) {
        const float t = v[k] + bias[c0 + k];
        h[k] = __float2half_rn(ep.relu ? fmaxf(t, 0.0f) : t);
    }
    const int lane = threadIdx.x & 31;
    warp_store_staged<CW>(ep.out, c0, h, true, lane, 32, [&](int p, int &yy, int &xx) {
        yy = y;
        xx = x0w + p;
        return xx < tg.conv_w;
    }, stg, io);
}

// PLAIN and PARTIAL finish the column chunks c0 = part*cw, (part + nparts)*cw, ...
// (several warps may share a row); the LayerNorm modes need the whole row (nparts = 1).
template <int MODE, class L>
__device__ void epilogue_tile(const EpiParams &ep, const TileGeom &tg, int tile, int row, int n0, int Nsub, int N,
                              int ksplit_idx, L &ld, int part = 0, int nparts = 1, size_t io = 0) {
    float v[32];
    const int cw = (Nsub % 32 == 0) ? 32 : 16;
    const long long q = (long long)tile * 128 + row;
    const int y = (int)(q / tg.pitch), x = (int)(q - (long long)y * tg.pitch);
    const bool valid = y < tg.conv_h && x < tg.conv_w;
    const long long tok = valid ? (long long)y * tg.conv_w + x : 0;
    if (MODE == EPI_PLAIN) {
        epilogue_plain_yx(ep, tg, y, x, n0, Nsub, ld, part, nparts, ep.bias_c, io);
        return;
    }
    if (MODE == EPI_PARTIAL) {
        const long long T = (long long)tg.conv_h * tg.conv_w;
        float *dst = img_at(ep.partial, io) + ((long long)ksplit_idx * T + tok) * N + n0;
        for (int c0 = part * cw; c0 < Nsub; c0 += nparts * cw) {
            load_cols(ld, c0, cw, v);
            if (valid) {
#pragma unroll
                for (int k = 0; k < 32; k += 4)
                    if (k < cw) *reinterpret_cast<float4 *>(dst + c0 + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
            }
        }
        return;
    }
    // LayerNorm modes (the slice is the whole row: n0 = 0, Nsub = N): single-pass
    // statistics shifted by the row's first value.
    const bool use_res = MODE == EPI_RESLN;
    const __half *res = use_res ? img_at(ep.res, io) : nullptr;
    float shift0 = 0.f, s1 = 0.f, s2 = 0.f;
    for (int c0 = 0; c0 < N; c0 += cw) {
        row_vals(ld, ep, res, N, tok, use_res, c0, cw, v);
        if (c0 == 0) shift0 = v[0];
#pragma unroll
        for (int k = 0; k < 32; k++)
            if (k < cw) {
                const float d = v[k] - shift0;
                s1 += d;
                s2 += d * d;
            }
    }
    const float m1 = s1 / N;
    const float mean = shift0 + m1;
    const float rstd = rsqrtf(fmaxf(s2 / N - m1 * m1, 0.0f) + ep.eps1);
    if (MODE == EPI_RESLN) {
        for (int c0 = 0; c0 < N; c0 += cw) {
            row_vals(ld, ep, res, N, tok, true, c0, cw, v);
            if (valid) {
                __align__(16) __half h[32];
#pragma unroll
                for (int k = 0; k < 32; k++)
                    if (k < cw) h[k] = __float2half_rn((v[k] - mean) * rstd * ep.g1[c0 + k] + ep.b1[c0 + k]);
                act_store(ep.out, y, x, c0, h, cw, io);
            }
        }
        return;
    }
    // EPI_LN2: y0 = LN1(v) stored; LN2 statistics over the fp32 y0 (shifted by its first value).
    float t0 = 0.f, u1 = 0.f, u2 = 0.f;
    for (int c0 = 0; c0 < N; c0 += cw) {
        row_vals(ld, ep, res, N, tok, false, c0, cw, v);
        __align__(16) __half h[32];
#pragma unroll
        for (int k = 0; k < 32; k++)
            if (k < cw) {
                const float t = (v[k] - mean) * rstd * ep.g1[c0 + k] + ep.b1[c0 + k];
                if (c0 == 0 && k == 0) t0 = t;
                const float d = t - t0;
                u1 += d;
                u2 += d * d;
                h[k] = __float2half_rn(t);
            }
        if (valid) act_store(ep.out, y, x, c0, h, cw, io);
    }
    const float mu = u1 / N;
    const float mean2 = t0 + mu;
    const float rstd2 = rsqrtf(fmaxf(u2 / N - mu * mu, 0.0f) + ep.eps2);
    for (int c0 = 0; c0 < N; c0 += cw) {
        row_vals(ld, ep, res, N, tok, false, c0, cw, v);
        if (valid) {
            float o[32];
#pragma unroll
            for (int k = 0; k < 32; k++)
                if (k < cw) {
                    const float t = (v[k] - mean) * rstd * ep.g1[c0 + k] + ep.b1[c0 + k];
                    o[k] = (t - mean2) * rstd2 * ep.g2[c0 + k] + ep.b2[c0 + k];
                }
            shift_store(ep.out2, ep.shift, 2, y, x, c0, o, cw, io);
        }
    }
}

// LayerNorm modes (EPI_LN2, EPI_RESLN) with one whole row per thread (the four warps
// of one set of TMEM lane quadrants own the unit).  Exact two-pass statistics without a
// second read of the residual: the first pass writes t = acc + bias (+ res) back into
// the row's TMEM columns, and LN2 runs its two passes over the LN1 output, written back
// the same way.  Warp-collective (TMEM); stores are masked.
template <int MODE, class L>
__device__ void epilogue_ln_row(const EpiParams &ep, const TileGeom &tg, int tile, int row, int N, L &ld,
                                size_t io = 0) {
    const __half *res = MODE == EPI_RESLN ? img_at(ep.res, io) : nullptr;
    float v[32];
    const long long q = (long long)tile * 128 + row;
    const int y = (int)(q / tg.pitch), x = (int)(q - (long long)y * tg.pitch);
    const bool valid = y < tg.conv_h && x < tg.conv_w;
    const long long tok = valid ? (long long)y * tg.conv_w + x : 0;
    float s = 0.f;
    for (int c0 = 0; c0 < N; c0 += 32) {
        row_vals(ld, ep, res, N, tok, MODE == EPI_RESLN, c0, 32, v);
#pragma unroll
        for (int k = 0; k < 32; k++) s += v[k];
        ld.store32(c0, v);
    }
    L::wait_st();
    const float mean = s / N;
    float sq = 0.f;
    for (int c0 = 0; c0 < N; c0 += 32) {
        ld.load32(c0, v);
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float d = v[k] - mean;
            sq += d * d;
        }
    }
    const float rstd = rsqrtf(sq / N + ep.eps1);
    if (MODE == EPI_RESLN && ep.ln_c) {
        for (int c0 = 0; c0 < N; c0 += 32) {
            ld.load32(c0, v);
            __align__(16) __half h[32];
#pragma unroll
            for (int k = 0; k < 32; k++)
                h[k] = __float2half_rn((v[k] - mean) * rstd * ep.bias_c[N + c0 + k] + ep.bias_c[2 * N + c0 + k]);
            if (valid) act_store(ep.out, y, x, c0, h, 32, io);
        }
        return;
    }
    float s2 = 0.f;
    for (int c0 = 0; c0 < N; c0 += 32) {
        ld.load32(c0, v);
        __align__(16) __half h[32];
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float t = (v[k] - mean) * rstd * ep.g1[c0 + k] + ep.b1[c0 + k];
            s2 += t;
            h[k] = __float2half_rn(t);
            v[k] = t;
        }
        if (valid) act_store(ep.out, y, x, c0, h, 32, io);
        if (MODE == EPI_LN2) ld.store32(c0, v);
    }
    if (MODE == EPI_RESLN) return;
    // EPI_LN2: LN2 over the fp32 LN1 outputs, then the H-shift scatter
    L::wait_st();
    const float mean2 = s2 / N;
    float q2 = 0.f;
    for (int c0 = 0; c0 < N; c0 += 32) {
        ld.load32(c0, v);
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float d = v[k] - mean2;
            q2 += d * d;
        }
    }
    const float rstd2 = rsqrtf(q2 / N + ep.eps2);
    for (int c0 = 0; c0 < N; c0 += 32) {
        ld.load32(c0, v);
        if (valid) {
#pragma unroll
            for (int k = 0; k < 32; k += 2)
                shift_store2(ep.out2, ep.shift, 2, y, x, c0 + k, (v[k] - mean2) * rstd2 * ep.g2[c0 + k] + ep.b2[c0 + k],
                             (v[k + 1] - mean2) * rstd2 * ep.g2[c0 + k + 1] + ep.b2[c0 + k + 1], io);
        }
    }
}

// Pool epilogue: this thread's conv pixel (2*y2, x) is in `top`, (2*y2+1, x) in
// `bot` (same TMEM lane, two accumulators); lanes L and L^1 hold x and x^1.
template <class L>
__device__ void epilogue_pool(const EpiParams &ep, const TileGeom &tg, int y2, int x, int n0, int Nsub, L &top,
                              L &bot, int part = 0, int nparts = 1, size_t io = 0) {
    float a[32], b[32];
    const int cw = (Nsub % 32 == 0) ? 32 : 16;
    const bool writer = (x & 1) == 0 && x < tg.conv_w;
    for (int c0 = part * cw; c0 < Nsub; c0 += nparts * cw) {
        load_cols(top, c0, cw, a);
        load_cols(bot, c0, cw, b);
        __align__(16) __half h[32];
#pragma unroll
        for (int k = 0; k < 32; k++) {
            if (k < cw) {
                float v = fmaxf(a[k], b[k]);
                v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1)) + ep.bias_c[n0 + c0 + k];
                h[k] = __float2half_rn(fmaxf(v, 0.0f));
            }
        }
        if (writer) act_store(ep.out, y2, x >> 1, n0 + c0, h, cw, io);
    }
}

// The pool epilogue of one warp's 32 conv pixels (2*y2 and 2*y2+1, x0w + lane; x0w even)
// for channels [c0, c0 + CW): the 16 pooled pixels (y2, x0w/2 + p) are stored through the
// warp's staging buffer.  Warp-collective (TMEM, shuffles).
template <int CW, class L>
__device__ __forceinline__ void epilogue_pool_staged(const EpiParams &ep, const TileGeom &tg, int y2, int x0w, int c0,
                                                     L &top, L &bot, uint8_t *stg, size_t io) {
    float a[32], b[32];
    load_cols(top, c0, CW, a);
    load_cols(bot, c0, CW, b);
    __align__(16) __half h[CW];
#pragma unroll
    for (int k = 0; k < CW; k++) {
        float v = fmaxf(a[k], b[k]);
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1)) + ep.bias_c[c0 + k];
        h[k] = __float2half_rn(fmaxf(v, 0.0f));
    }
    const int lane = threadIdx.x & 31, xp0 = x0w >> 1, wp = tg.conv_w >> 1;
    warp_store_staged<CW>(ep.out, c0, h, (lane & 1) == 0, lane >> 1, 16, [&](int p, int &yy, int &xx) {
        yy = y2;
        xx = xp0 + p;
        return xx < wp;
    }, stg, io);
}

// dec5 window of one row-window unit in shared memory: a TMA box of C1 channels x
// kHeadWinCols dec5 columns x (R/2 + 2) dec5 rows, rows of C1 * 2 bytes under the
// matching swizzle (32B for 16 channels, 64B for 32: 16-byte chunk bits [5:4] XOR
// address bits [8:7]), so that the two-column gathers of a warp hit distinct banks.
constexpr int kHeadWinCols = 66;   // 128 pixels -> 64 dec5 columns + the clamp/interpolation halo

// The swizzle of a window pixel's 16-byte chunk k depends on the pixel only: its row starts
// on a multiple of C1 * 2 bytes, so chunk k's offset bits [5:4] (C1 = 32; bit 4 for 16) come
// from k alone and address bits [8:7] from the pixel.  A HeadWinPix holds the pixel's byte
// offset and its chunk XOR; chunk k then costs one XOR and one add.
struct HeadWinPix {
    uint32_t base, sw;
};

template <int C1>
__device__ __forceinline__ HeadWinPix head_win_pix(int r, int c) {
    const uint32_t b = (uint32_t)((r * kHeadWinCols + c) * (C1 * 2));
    return HeadWinPix{b, (b >> 7) & (C1 == 32 ? 3u : 1u)};
}

__device__ __forceinline__ uint4 head_win_ld(const uint8_t *win, HeadWinPix px, int k) {
    return *reinterpret_cast<const uint4 *>(win + px.base + ((((uint32_t)k) ^ px.sw) << 4));
}

__device__ __forceinline__ float sigmoid_fast(float v) { return __fdividef(1.0f, 1.0f + __expf(-v)); }

// The per-pixel tail of the head: div6 into the DR stem input (GC) or the u8 output (DR).
// xin: the pixel's first 8 stem-input channels (GC: the u8 image in channels 0-2).
__device__ __forceinline__ void head_store(const HeadParams &hp, int W, int y, int x, const float *o, const uint4 xin,
                                           size_t io) {
    const size_t pix = (size_t)y * W + x;
    if (!hp.is_dr) {
        // div6: r = clamp(x / max(I_sm, 1e-6), 0, 1) with x = u8 / 255, written as the DR stem input
        const __half *xu = reinterpret_cast<const __half *>(&xin);
        __align__(16) __half v[kStemInC];
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const __half u = xu[c];
            const float d = o[c] > 1e-6f ? o[c] : 1e-6f;
            float r = __fdividef(__half2float(u) * (1.0f / 255.0f), d);
            r = r < 0.0f ? 0.0f : (r > 1.0f ? 1.0f : r);
            const __half rh = __float2half_rn(r);
            const __half rl = __float2half_rn(r - __half2float(rh));
            v[c] = u;
            v[3 + c] = u;
            v[6 + c] = rh;
            v[9 + c] = rl;
            v[12 + c] = rh;
            if (hp.r_out) img_at(hp.r_out, io)[pix * 3 + c] = r;
            if (hp.ism_out) img_at(hp.ism_out, io)[pix * 3 + c] = o[c];
        }
        v[15] = __float2half_rn(0.0f);
        act_store(hp.si_out, y, x, 0, v, kStemInC, io);
    } else {
        if (hp.y_out)
            for (int c = 0; c < 3; c++) img_at(hp.y_out, io)[pix * 3 + c] = o[c];
        const ImgSpec &im = hp.img;
        const int oy = y - im.ph, ox = x - im.pw;
        if (oy < 0 || ox < 0) return;
        uint8_t q[3];
#pragma unroll
        for (int c = 0; c < 3; c++) {
            float f = o[c] * 255.0f + 0.5f;
            f = f < 0.0f ? 0.0f : (f > 255.0f ? 255.0f : f);
            q[c] = (uint8_t)f;
        }
        const int ob = im.swap ? 2 : 0;
        uint8_t *d = img_at(hp.dst, io) + ((size_t)oy * im.w + ox) * im.bpp;
        if (im.bpp == 4) {
            uchar4 v;
            v.x = ob ? q[2] : q[0];
            v.y = q[1];
            v.z = ob ? q[0] : q[2];
            v.w = img_at(im.src, io)[(size_t)oy * im.stride + (size_t)ox * 4 + 3];
            *reinterpret_cast<uchar4 *>(d) = v;
        } else {
            d[ob] = q[0];
            d[1] = q[1];
            d[2 - ob] = q[2];
        }
    }
}

// EPI_HEAD for the padded-image pixels (y, x) and (y + 1, x), y even: accumulator rows
// ld0 / ld1 hold their stem conv (C1 = 16 or 32 columns).  The two rows share the
// middle dec5 row of their x2 bilinear (half_pixel, edge clamp: ONNX Resize linear),
// so six window columns serve both pixels.  win holds dec5 rows wy0.. and columns
// wx0.. (window origin, may be -1).  Warp-collective (the TMEM loads); stores are masked.
// segs: the unit's stem-input row segments in the same ring stage (segment r = padded row
// y0 + r, pixel slot p = padded column x0 + p, 32-byte rows under the 32B swizzle), where the
// GC tail finds its pixels' u8 values (segments jj + 1, jj + 2, slot x - x0 + 1).
template <int C1, class L>
__device__ void epilogue_head_pair(const EpiParams &ep, const TileGeom &tg, int y, int x, L &ld0, L &ld1,
                                   const uint8_t *win, int wy0, int wx0, const uint8_t *seg0, const uint8_t *seg1,
                                   int slot, size_t io) {
    const HeadParams &hp = ep.head;
    // the TMEM loads below are warp-collective: a warp leaves only as a whole; lanes past
    // the image edge compute on in-window data and store nothing
    const bool valid = y < tg.conv_h && x < tg.conv_w;
    if (!__any_sync(0xffffffffu, valid)) return;
    const int Hh = tg.conv_h >> 1, Wh = tg.conv_w >> 1;
    const int M = y >> 1, n = x >> 1;
    const bool xodd = x & 1;
    // even output row y: dec5 rows M-1 (1/4), M (3/4); odd row y+1: rows M (3/4), M+1 (1/4)
    const int r0 = max(M - 1, 0) - wy0, r1 = M - wy0, r2 = min(M + 1, Hh - 1) - wy0;
    // even x: columns n-1 (1/4), n (3/4); odd x: n (3/4), n+1 (1/4)
    const int cA = (xodd ? n : max(n - 1, 0)) - wx0, cB = (xodd ? min(n + 1, Wh - 1) : n) - wx0;
    const HeadWinPix p0a = head_win_pix<C1>(r0, cA), p0b = head_win_pix<C1>(r0, cB);
    const HeadWinPix p1a = head_win_pix<C1>(r1, cA), p1b = head_win_pix<C1>(r1, cB);
    const HeadWinPix p2a = head_win_pix<C1>(r2, cA), p2b = head_win_pix<C1>(r2, cB);
    // the products of 1/4 and 3/4 are exact in fp16: the interpolation of the fp16 dec5
    // runs on channel pairs (HFMA2), the rest in fp32
    const float wa = xodd ? 0.75f : 0.25f, wb = 1.0f - wa;
    const __half2 q_a = __float2half2_rn(0.25f * wa), q_b = __float2half2_rn(0.25f * wb);
    const __half2 t_a = __float2half2_rn(0.75f * wa), t_b = __float2half2_rn(0.75f * wb);
    // the 1x1 on packed fp32 pairs (FFMA2: even channels in .x, odd in .y, one chain each,
    // added at the end), the relu-add of the bias likewise
    float2 oa[3], ob[3];
#pragma unroll
    for (int o = 0; o < 3; o++) oa[o] = ob[o] = make_float2(hp.fb[o], 0.0f);
    uint32_t ca[16], cb[16];   // the stem conv of both pixels, 16 channels at a time
#pragma unroll
    for (int k = 0; k < C1 / 8; k++) {
        if (k % 2 == 0) {
            // a phase boundary for the scheduler: the next phase's window loads stay below
            // this phase's arithmetic (hoisting them all would spill at 128 registers)
            if (k) asm volatile("" ::: "memory");
            ld0.load16_nw(ca, 8 * k);
            ld1.load16_nw(cb, 8 * k);
            L::wait_ld();
        }
        const uint4 u0a = head_win_ld(win, p0a, k), u0b = head_win_ld(win, p0b, k);
        const uint4 u1a = head_win_ld(win, p1a, k), u1b = head_win_ld(win, p1b, k);
        const uint4 u2a = head_win_ld(win, p2a, k), u2b = head_win_ld(win, p2b, k);
        const __half2 *h0a = reinterpret_cast<const __half2 *>(&u0a), *h0b = reinterpret_cast<const __half2 *>(&u0b);
        const __half2 *h1a = reinterpret_cast<const __half2 *>(&u1a), *h1b = reinterpret_cast<const __half2 *>(&u1b);
        const __half2 *h2a = reinterpret_cast<const __half2 *>(&u2a), *h2b = reinterpret_cast<const __half2 *>(&u2b);
#pragma unroll
        for (int p = 0; p < 4; p++) {
            __half2 ue = __hmul2(h0a[p], q_a);
            ue = __hfma2(h0b[p], q_b, ue);
            ue = __hfma2(h1a[p], t_a, ue);
            ue = __hfma2(h1b[p], t_b, ue);
            __half2 uo = __hmul2(h1a[p], t_a);
            uo = __hfma2(h1b[p], t_b, uo);
            uo = __hfma2(h2a[p], q_a, uo);
            uo = __hfma2(h2b[p], q_b, uo);
            // relu of the upsampled pair in fp16 (one max per pair; the widening is exact)
            const __half2 zero2 = __float2half2_rn(0.0f);
            const float2 fe = __half22float2(__hmax2(ue, zero2)), fo = __half22float2(__hmax2(uo, zero2));
            const int c = 8 * k + 2 * p, cl = c % 16;
            const float2 bias = make_float2(hp.b1[c], hp.b1[c + 1]);
            const float2 ta = __fadd2_rn(make_float2(__uint_as_float(ca[cl]), __uint_as_float(ca[cl + 1])), bias);
            const float2 tb = __fadd2_rn(make_float2(__uint_as_float(cb[cl]), __uint_as_float(cb[cl + 1])), bias);
            const float2 sa = __fadd2_rn(fe, make_float2(fmaxf(ta.x, 0.0f), fmaxf(ta.y, 0.0f)));
            const float2 sb = __fadd2_rn(fo, make_float2(fmaxf(tb.x, 0.0f), fmaxf(tb.y, 0.0f)));
#pragma unroll
            for (int o = 0; o < 3; o++) {
                const float2 w = make_float2(hp.fw[o * C1 + c], hp.fw[o * C1 + c + 1]);
                oa[o] = __ffma2_rn(sa, w, oa[o]);
                ob[o] = __ffma2_rn(sb, w, ob[o]);
            }
        }
    }
    const float ya[3] = {sigmoid_fast(oa[0].x + oa[0].y), sigmoid_fast(oa[1].x + oa[1].y), sigmoid_fast(oa[2].x + oa[2].y)};
    const float yb[3] = {sigmoid_fast(ob[0].x + ob[0].y), sigmoid_fast(ob[1].x + ob[1].y), sigmoid_fast(ob[2].x + ob[2].y)};
    if (valid) {
        uint4 xa = make_uint4(0, 0, 0, 0), xb = xa;
        if (!hp.is_dr) {
            // channels 0-7 of the pixel: 16-byte chunk 0 of its 32-byte row, at chunk 0 ^ address bit 7
            const uint32_t off = (uint32_t)slot * 32u;
            const uint32_t sw = ((off >> 7) & 1u) << 4;
            xa = *reinterpret_cast<const uint4 *>(seg0 + (off ^ sw));
            xb = *reinterpret_cast<const uint4 *>(seg1 + (off ^ sw));
        }
        head_store(hp, tg.conv_w, y, x, ya, xa, io);
        head_store(hp, tg.conv_w, y + 1, x, yb, xb, io);
    }
}

}  // namespace gcdr
