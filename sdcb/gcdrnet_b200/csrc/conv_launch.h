// conv_launch.h -- host entry points of the implicit-GEMM convolution.
#pragma once
#include <cuda_runtime.h>

#include <string>

#include "conv.cuh"

namespace gcdr {

constexpr int kMaxStages = 32;

struct TcConfig {
    int bk = 64;           // channels per k-block (16/32/64 -> SWIZZLE_32B/64B/128B)
    int stages = 2;        // shared-memory ring depth
    int kps = 1;           // k-blocks (A tile + B tile pairs) per ring stage
    int rt = 1;            // plain: consecutive 128-row tiles per work unit; pool: 128-pixel
                           // segments per pooled row (2*rt sub-tiles); one B tile feeds them all
    int sub_bytes = 0;     // one A tile + B tile, 1 KB aligned
    int stage_bytes = 0;   // kps * sub_bytes
    int acc_cols = 32;     // TMEM columns per accumulator (power of two >= N)
    int acc_bufs = 1;      // accumulator double buffering
    int tmem_cols = 32;
};

int tc_pick_bk(int C);
int tc_plan(const ConvArgs &a, int num_sms, TcConfig &cfg, std::string &err);
// tcgen05 path (sm_100a).  mode = EpiMode.
int tc_conv_launch(const ConvArgs &a, int mode, int num_sms, cudaStream_t st, std::string &err);
// SIMT reference path: same math and epilogue, fp32 FMA, accumulators staged in
// `scratch` (ref_conv_scratch_floats: one row of N per output-grid position).
// Used by the tests to check the tensor-core path.
int ref_conv_launch(const ConvArgs &a, int mode, float *scratch, cudaStream_t st, std::string &err);
size_t ref_conv_scratch_floats(const ConvArgs &a);

}  // namespace gcdr
