// epilogue.cuh -- per-pixel epilogues of the implicit-GEMM convolutions.
//
// The GEMM tile is 128 output positions x N channels.  Thread `row` (0..127)
// of the four epilogue warps owns one position; its N accumulators are read
// in chunks of 16 columns through a Loader (TMEM for the tcgen05 kernel,
// global scratch for the SIMT reference), so the same code finishes both.
// Loader::load16 is warp-synchronous (tcgen05.ld is .sync.aligned): all
// control flow around it is uniform; per-thread validity only masks stores.
//
// Modes (the fusions the reference's CPU plan makes, EngineTests.cs:79-141):
//   EPI_PLAIN  y = acc + bias                                 decoder convs, fc1
//   EPI_POOL   y = relu(maxpool2x2(acc + bias))               encoder conv+pool+relu (gc#23-25)
//   EPI_LN2    y0 = LN1(acc + bias) -> out (tokens);          patch embed + its norm (gc#34-37)
//              h = LN2(y0) -> out2 with the H-shift scatter    and the block's norm2 + shift (gc#38-44)
//   EPI_RESLN  y = LN(acc + bias + res) -> out                fc2 + residual + norm3 (gc#127-130)
#pragma once
#include "common.cuh"

namespace gcdr {

enum EpiMode : int { EPI_PLAIN = 0, EPI_POOL = 1, EPI_LN2 = 2, EPI_RESLN = 3 };

struct EpiParams {
    const float *bias = nullptr;
    int relu = 0;                    // EPI_PLAIN: relu after the bias
    Act out;                         // primary output (logical dims = conv or pooled output)
    // LN modes
    const float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
    float eps1 = 1e-5f, eps2 = 1e-5f;
    Act out2;                        // EPI_LN2: LN2 output, LAY_PLAIN tokens, H-shift scatter
    ShiftSpec shift;
    const __half *res = nullptr;     // EPI_RESLN residual tokens [T][N]
};

// Geometry of the output grid: q = y * pitch + x over a flat row space; in pool
// mode a tile is a pair of conv rows x 64 columns.
struct TileGeom {
    int pool = 0;
    int pitch = 0;        // grid rows per image row (>= out_w; extra columns are discarded)
    int conv_h = 0, conv_w = 0;   // conv output dims (valid region of the grid)
    int tiles_x = 0;      // pool mode: tiles per row pair
    int ntiles = 0;
};

struct EpiSmem {
    float x[128 * 17];    // pool exchange
};

__device__ inline void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <class L>
__device__ inline void ln_stats(L &ld, const EpiParams &ep, int N, long long tok, bool use_res, float &mean, float &rstd,
                                float eps) {
    float s = 0.f;
    float v[16], r[16];
    for (int c0 = 0; c0 < N; c0 += 16) {
        ld.load16(c0, v);
        if (use_res) load16h(ep.res + tok * N + c0, r);
#pragma unroll
        for (int k = 0; k < 16; k++) s += v[k] + ep.bias[c0 + k] + (use_res ? r[k] : 0.0f);
    }
    mean = s / N;
    float q = 0.f;
    for (int c0 = 0; c0 < N; c0 += 16) {
        ld.load16(c0, v);
        if (use_res) load16h(ep.res + tok * N + c0, r);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            float d = v[k] + ep.bias[c0 + k] + (use_res ? r[k] : 0.0f) - mean;
            q += d * d;
        }
    }
    rstd = rsqrtf(q / N + eps);
}

template <int MODE, class L>
__device__ void epilogue_tile(const EpiParams &ep, const TileGeom &tg, int tile, int row, int N, L &ld,
                              EpiSmem *sm) {
    float v[16];
    if (MODE == EPI_POOL) {
        const int y2 = tile / tg.tiles_x, xt = tile - y2 * tg.tiles_x;
        const int sub = row >> 6, xx = row & 63;
        const int cx = xt * 64 + xx;
        const bool writer = sub == 0 && (xx & 1) == 0 && cx < tg.conv_w;
        for (int c0 = 0; c0 < N; c0 += 16) {
            ld.load16(c0, v);
#pragma unroll
            for (int k = 0; k < 16; k++) {
                float t = v[k] + ep.bias[c0 + k];
                float o = __shfl_xor_sync(0xffffffffu, t, 1);
                v[k] = fmaxf(t, o);
            }
            if (sub == 1) {
#pragma unroll
                for (int k = 0; k < 16; k++) sm->x[xx * 17 + k] = v[k];
            }
            named_bar_sync(1, 128);
            if (writer) {
                __align__(16) __half h[16];
#pragma unroll
                for (int k = 0; k < 16; k++) h[k] = __float2half_rn(fmaxf(fmaxf(v[k], sm->x[xx * 17 + k]), 0.0f));
                act_store(ep.out, y2, cx >> 1, c0, h, 16);
            }
            named_bar_sync(1, 128);
        }
        return;
    }
    const long long q = (long long)tile * 128 + row;
    const int y = (int)(q / tg.pitch), x = (int)(q - (long long)y * tg.pitch);
    const bool valid = y < tg.conv_h && x < tg.conv_w;
    if (MODE == EPI_PLAIN) {
        for (int c0 = 0; c0 < N; c0 += 16) {
            ld.load16(c0, v);
            if (valid) {
                __align__(16) __half h[16];
#pragma unroll
                for (int k = 0; k < 16; k++) {
                    float t = v[k] + ep.bias[c0 + k];
                    h[k] = __float2half_rn(ep.relu ? fmaxf(t, 0.0f) : t);
                }
                act_store(ep.out, y, x, c0, h, 16);
            }
        }
        return;
    }
    // LayerNorm modes: the whole row of N channels is in this thread's lane.
    const long long tok = valid ? (long long)y * tg.conv_w + x : 0;
    const bool use_res = MODE == EPI_RESLN;
    float mean, rstd;
    ln_stats(ld, ep, N, tok, use_res, mean, rstd, ep.eps1);
    if (MODE == EPI_RESLN) {
        float r[16];
        for (int c0 = 0; c0 < N; c0 += 16) {
            ld.load16(c0, v);
            if (valid) {
                load16h(ep.res + tok * N + c0, r);
                __align__(16) __half h[16];
#pragma unroll
                for (int k = 0; k < 16; k++) {
                    int c = c0 + k;
                    float t = v[k] + ep.bias[c] + r[k];
                    h[k] = __float2half_rn((t - mean) * rstd * ep.g1[c] + ep.b1[c]);
                }
                act_store(ep.out, y, x, c0, h, 16);
            }
        }
        return;
    }
    // EPI_LN2: y0 = LN1(v) stored; LN2 statistics over the fp32 y0.
    float s2 = 0.f;
    for (int c0 = 0; c0 < N; c0 += 16) {
        ld.load16(c0, v);
        __align__(16) __half h[16];
#pragma unroll
        for (int k = 0; k < 16; k++) {
            int c = c0 + k;
            float t = (v[k] + ep.bias[c] - mean) * rstd * ep.g1[c] + ep.b1[c];
            s2 += t;
            h[k] = __float2half_rn(t);
        }
        if (valid) act_store(ep.out, y, x, c0, h, 16);
    }
    const float mean2 = s2 / N;
    float q2 = 0.f;
    for (int c0 = 0; c0 < N; c0 += 16) {
        ld.load16(c0, v);
#pragma unroll
        for (int k = 0; k < 16; k++) {
            int c = c0 + k;
            float t = (v[k] + ep.bias[c] - mean) * rstd * ep.g1[c] + ep.b1[c];
            float d = t - mean2;
            q2 += d * d;
        }
    }
    const float rstd2 = rsqrtf(q2 / N + ep.eps2);
    for (int c0 = 0; c0 < N; c0 += 16) {
        ld.load16(c0, v);
        if (valid) {
            float o[16];
#pragma unroll
            for (int k = 0; k < 16; k++) {
                int c = c0 + k;
                float t = (v[k] + ep.bias[c] - mean) * rstd * ep.g1[c] + ep.b1[c];
                o[k] = (t - mean2) * rstd2 * ep.g2[c] + ep.b2[c];
            }
            shift_store(ep.out2, ep.shift, 2, y, x, c0, o, 16);
        }
    }
}

}  // namespace gcdr
