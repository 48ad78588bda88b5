// conv_launch.h -- host entry points of the implicit-GEMM convolution.
#pragma once
#include <cuda.h>
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

// Row-window plan (conv_rw.cu): a unit is R output rows x 128 pixels; each ring
// stage holds the unit's R+2 input row segments (136 pixels) of one k-block, and
// all nine taps read them through shifted descriptors; weights stay resident.
struct RwConfig {
    int bk = 64;
    int R = 2;             // output rows per unit (sub-tiles, one MMA warp each)
    int segs_x = 1;        // 128-pixel segments per row
    int units = 0;
    int seg_bytes = 0;     // one input row segment (136 rows of bk channels), 1 KB aligned
    int stage_bytes = 0;   // (R + 2) * seg_bytes
    int stages = 2;
    int b_block = 0;       // one (k-block, tap) weight block: N rows x bk, 1 KB aligned
    int b_bytes = 0;       // all weights: 9 * C/bk blocks
    int acc_cols = 32, acc_bufs = 1, tmem_cols = 32;
    int win_tx = 0;        // head: bytes of the dec5 window box per stage (0 otherwise)
    int stg_bytes = 0;     // plain / pool: the epilogue warps' store staging buffers
};

// Copies the layer's bias (device, N floats) into a.ep.bias_c (synchronous; at op
// build time, never inside a stream capture).  0, or -1 if N exceeds kMaxBiasConst.
int fill_bias_consts(ConvArgs &a);

int tc_pick_bk(int C);
// fp16 tensor map of `rank` dims (dims[0] contiguous, swizzled by its width in bytes:
// 32/64/128), strides[i] = byte stride of dims[i + 1].
bool tma_encode(CUtensorMap *m, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                const uint32_t *box, int swizzle_bytes, std::string &err);
// The activation map of a conv (a.A): [nimg][a_rows][C] with the launch's image stride, a
// box of box_inner channels x box_rows rows of one image.
bool tma_encode_act(CUtensorMap *m, const ConvArgs &a, uint32_t box_inner, uint32_t box_rows, std::string &err);
// Checks a launch's image count and stride (batched launches).
bool batch_ok(const ConvArgs &a, std::string &err);
bool tma_encode_2d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                   uint32_t box_outer, int bk, std::string &err);
// 0 and a plan when the layer suits the row-window kernel, -1 otherwise.
int rw_plan(const ConvArgs &a, int mode, int num_sms, RwConfig &cfg);
int rw_conv_launch(const ConvArgs &a, int mode, const RwConfig &cfg, int num_sms, cudaStream_t st, std::string &err);
int tc_plan(const ConvArgs &a, int mode, int num_sms, TcConfig &cfg, std::string &err);
// tcgen05 path (sm_100a).  mode = EpiMode.
int tc_conv_launch(const ConvArgs &a, int mode, int num_sms, cudaStream_t st, std::string &err);
// SIMT reference path: same math and epilogue, fp32 FMA, accumulators staged in
// `scratch` (ref_conv_scratch_floats: one row of N per output-grid position).
// Used by the tests to check the tensor-core path.
int ref_conv_launch(const ConvArgs &a, int mode, float *scratch, cudaStream_t st, std::string &err);
size_t ref_conv_scratch_floats(const ConvArgs &a);

}  // namespace gcdr
