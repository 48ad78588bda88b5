// kernels.h -- launchers of the SIMT kernels around the tensor-core convs.
#pragma once
#include <cuda_runtime.h>

#include "common.cuh"

namespace gcdr {

// Stem: enc1 conv 3x3 reflect (Cin = 3 from the image, or 6 = image + the
// division-corrected image `r`) + bias -> maxpool 2x2 -> relu, fp32 math,
// fp16 LAY_PADREFL output (gc#22-25).  w is ONNX [C1][Cin][3][3].
struct StemArgs {
    ImgSpec img;
    const float *r = nullptr;       // DR only: [H][W][3] fp32
    int H = 0, W = 0;               // padded dims
    int cin = 3, c1 = 16;
    const float *w = nullptr, *b = nullptr;
    Act out;
};
int stem_launch(const StemArgs &a, cudaStream_t st);

// Head (UpHeadOp with the skip recomputed, Extensions/UpHeadOp.cs:8-28,249-279):
//   s = relu(bilinear2x(dec5)) + relu(enc1conv(input)); o = sigmoid(fb + fw . s)
// GC: writes r = clamp(x / max(o, 1e-6), 0, 1) (div6, PixelOps.cs:81-102) and
//     optionally o itself (the shading map).
// DR: writes the caller's u8 format, cropped, alpha from the source
//     (nhwc2bgr.comp:23-55).
struct HeadArgs {
    ImgSpec img;
    const float *r = nullptr;       // DR input half (DR only)
    int H = 0, W = 0;
    int cin = 3, c1 = 16;
    const float *w = nullptr, *b = nullptr;     // enc1 conv (recomputed skip)
    const float *fw = nullptr, *fb = nullptr;   // final 1x1 conv [3][c1], [3]
    const __half *dec5 = nullptr;   // [H/2][W/2][c1] LAY_PLAIN
    float *r_out = nullptr;         // GC: [H][W][3]
    float *ism_out = nullptr;       // GC, optional: [H][W][3]
    float *y_out = nullptr;         // DR, optional: [H][W][3] net output (debug)
    uint8_t *dst = nullptr;         // DR: tight [h][w][bpp]
    int is_dr = 0;
};
int head_launch(const HeadArgs &a, cudaStream_t st);


// The stem and the head on the tensor cores are row-window convs (conv_rw.cu)
// over a 16-channel stem input; these kernels (SIMT, fp32) are the reference
// path selected by GCDR_CUDA_STEM=simt.
//
// The GC stem input (the stem-input layout of epilogue.cuh, LAY_PADREFL
// [H+2][W+2][16] fp16): [x, x, 0] with x the u8 pixel of the top/left
// replicate-padded source in B,G,R order (GcdrEnhancer.cs:242-243 pads and reads it).
// err (may be null): the device error word, cleared by the kernel (the enhancement's first).
// im.src: a tight device image (stride = w * bpp) with at least 16 bytes of slack past its
// end (the kernel reads whole aligned 16-byte words).
// Batched launches (nimg > 1): image k's source, stem input and error word lie k * img_bytes
// past image 0's (the same holds for every batched launch below).
int stem_in_launch(const ImgSpec &im, const Act &si, int *err, cudaStream_t st, int nimg = 1, long long img_bytes = 0);
// CUDA error string of this thread's last failed launch of the kernels above.
const char *last_launch_error();
// Stem conv weights for that layout: ONNX [C1][Cin][3][3] -> [C1][9 taps][16]
// with w' = w_x / 255 split hi+lo for the image channels and w_r split hi+lo
// for the r channels (DR).
void pack_stem_conv(const float *w, int c1, int cin, __half *out);

// Depthwise 3x3 (zero pad 1) + bias -> exact GELU -> W-shift scatter
// (gc#85-95 with ChannelShift along W).  wt is tap-major [9][C] fp32 (ONNX
// [C][1][3][3] transposed at upload), b [C]; both 16-byte aligned.
int dw_gelu_shift_launch(const __half *in, int H, int W, int C, const float *wt, const float *b, const ShiftSpec &s,
                         __half *out, cudaStream_t st, int nimg = 1, long long img_bytes = 0);

// Decoder join: out = relu(bilinear2x(d)) + skip  (gc#236-240, 444-446).
//   tokens=false: out is an Act (LAY_PADREFL) for the next decoder conv.
//   tokens=true : out is LAY_PLAIN tokens (the block residual) and h gets
//                 LN2(out) with the H-shift scatter (the block's norm2 + shift).
struct UpAddArgs {
    const __half *d = nullptr;      // [h][w][C] LAY_PLAIN, h = H/2
    Act skip;                       // [H][W][C]
    Act out;                        // [H][W][C]
    int tokens = 0;
    const float *g = nullptr, *b = nullptr;
    float eps = 1e-5f;
    Act h;                          // tokens [H][W][C]
    ShiftSpec shift;
    int nimg = 1;                   // images per launch (d, skip, out, h at image k's offset)
    long long img_bytes = 0;
};
int up_add_launch(const UpAddArgs &a, cudaStream_t st);

// Finishes a split-K tensor-core layer (EPI_PARTIAL): per token, sums the
// k-split partials in order, adds the bias (and the residual), then
//   ln2 = 0: out = LN1(v)                               (fc2 + residual + norm)
//   ln2 = 1: out = y0 = LN1(v) (tokens); out2 = LN2(y0) with the H shift
//            (patch embed + its norm + the block's norm2 + shift)
struct LnFinalizeArgs {
    const float *partial = nullptr;   // [ksplit][T][N]
    int ksplit = 1;
    int H = 0, W = 0, N = 0;          // token grid (T = H*W) and channels
    const float *bias = nullptr;
    const __half *res = nullptr;      // optional residual tokens [T][N]
    const float *g1 = nullptr, *b1 = nullptr;
    float eps1 = 1e-5f;
    int ln2 = 0;
    const float *g2 = nullptr, *b2 = nullptr;
    float eps2 = 1e-5f;
    ShiftSpec shift;
    Act out, out2;
    int nimg = 1;                     // images per launch (partial, res, out, out2 at image k's offset)
    long long img_bytes = 0;
};
int ln_finalize_launch(const LnFinalizeArgs &a, cudaStream_t st);

// Channel-shift groups (cumulative ends, offsets; at most 5) -> ShiftSpec (pipeline.cu).
ShiftSpec make_shift(int ngroups, const int *ends, const int *offs);

// Standalone glue kernels (the C ABI's gcdr_k_*).
int k_bgr2nhwc(const uint8_t *src, int w, int h, int stride, int fmt, float *x, int ph, int pw, cudaStream_t st);
int k_div6(const float *x, const float *s, size_t npx, float *out6, cudaStream_t st);
int k_nhwc2bgr(const float *y, int H, int W, int ph, int pw, uint8_t *dst, int w, int h, int dst_stride, int fmt,
               const uint8_t *alpha, int alpha_stride, cudaStream_t st);

}  // namespace gcdr
