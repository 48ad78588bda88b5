// conv.cuh -- the implicit-GEMM convolution shared by every tensor-core layer.
//
//   out[q][n] = epilogue( sum_tap sum_c A[q + tap_off[tap]][c] * B[n][tap*C + c] )
//
// A is a flat fp16 matrix of `a_rows` rows of C channels (an activation in
// LAY_PADREFL / LAY_PHASE / LAY_PLAIN), B the packed weights [N][taps*C]
// (K-major, k = tap*C + c, tap = ky*3 + kx), q runs over the output grid.
// A 3x3 stride-1 reflect conv is 9 taps over LAY_PADREFL with offsets
// ky*(W+2)+kx; the stride-2 patch embeds are 9 taps over LAY_PHASE; the
// shift-MLP Gemms (fc1/fc2) are 1 tap over tokens.  Rows past the end of A
// read as zeros (TMA out-of-bounds fill), which only feeds discarded outputs.
#pragma once
#include "epilogue.cuh"

namespace gcdr {

struct ConvArgs {
    int ntaps = 1;
    int tap_off[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    int C = 0;                 // channels per tap (K per tap)
    int N = 0;                 // output channels (multiple of 16, <= 512)
    int nsplit = 1;            // N slices per tile (each Nsub = N / nsplit channels)
    int ksplit = 1;            // k-block splits (EPI_PARTIAL only)
    int rw = 0;                // 3x3 stride-1 over a [H+2][W+2][C] layout (taps ky*pitch + kx):
                               // eligible for the row-window kernel (conv_rw.cu)
    long long a_rows = 0;
    const __half *A = nullptr; // for the SIMT reference path and host checks
    const __half *B = nullptr; // packed weights [N][ntaps*C]
    TileGeom tg;
    EpiParams ep;
    int *err = nullptr;        // device error flag (GCDR_ERR_FLAG_*)
    int nimg = 1;              // images per launch: work units run over every image's grid
    long long img_bytes = 0;   // byte distance between consecutive images' buffers (nimg > 1)
    long long wait_cycles = 0; // bound of each mbarrier wait in SM cycles (0: the default, ~2 s)
    int timeout_probe = 0;     // test hook: issue no copies and no MMAs, so every wait runs out
};

// The wait bound a launch uses.
__host__ __device__ inline long long wait_budget(const ConvArgs &a) {
    return a.wait_cycles > 0 ? a.wait_cycles : kWaitCycles;
}

// Byte stride of the image dimension of a tensor map over `bytes` per image: the images'
// distance in a batched launch, else the (16-byte rounded) size of the one image.
__host__ __device__ inline unsigned long long img_stride(const ConvArgs &a, unsigned long long bytes) {
    return a.nimg > 1 ? (unsigned long long)a.img_bytes : (bytes + 15) & ~15ull;
}

// Work unit u -> (m unit, n slice, k split).
__host__ __device__ inline void unit_coords(const ConvArgs &a, int u, int &tile, int &ni, int &ki) {
    const int per = a.nsplit * a.ksplit;
    tile = u / per;
    const int r = u - tile * per;
    ni = r / a.ksplit;
    ki = r - ni * a.ksplit;
}

}  // namespace gcdr
