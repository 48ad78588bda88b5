// model.h -- GCDRNet weights as parsed from the two ONNX graphs.
//
// The reference delegates this to the external engine (OnnxModel.Load +
// GraphCompiler.Compile with the GCDR fusion passes,
// src/Sdcb.SimdGcdrNet/GcdrEnhancer.cs:84-124, Extensions/GcdrExtensions.cs:12-15).
// Here a small protobuf reader decodes the ModelProto and a recogniser maps
// the graph onto the UNeXt-style topology both nets share; anything else is
// rejected (GCDR_ERR_UNSUPPORTED) instead of being run wrongly.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace gcdr {

struct ConvW {
    int cout = 0, cin = 0, k = 0, stride = 1, pad = 0;
    bool reflect = false;          // explicit Pad(mode=reflect) before a pads=0 conv
    std::vector<float> w;          // ONNX order [cout][cin][k][k]
    std::vector<float> b;          // [cout]
};

struct LNW {
    int c = 0;
    float eps = 1e-5f;
    std::vector<float> g, b;
};

struct ShiftW {
    int axis = 2;                  // 2: along H (rows), 3: along W (columns)
    std::vector<int> ends;         // cumulative channel-group ends (5 groups)
    std::vector<int> offs;         // out[y] = in[y + off] per group, zero fill
};

// One shifted-MLP block plus the LayerNorm that follows it
// (UNeXt shiftedBlock: x + fc2(shiftW(gelu(dw(fc1(shiftH(LN2(x))))))), then norm).
struct BlockW {
    LNW norm2;
    ShiftW shift_a, shift_b;       // before fc1 (H) and before fc2 (W)
    std::vector<float> fc1_w, fc1_b, fc2_w, fc2_b;   // Gemm B operands [K][N]
    ConvW dw;                      // depthwise 3x3, group = C, zero pad 1
    LNW norm_out;                  // norm3 / norm4 / dnorm3 / dnorm4
};

struct NetW {
    int cin = 0;
    int c1 = 0, c2 = 0, c3 = 0, c4 = 0, c5 = 0;   // encoder / patch-embed widths
    ConvW enc[3], pe3, pe4, dec[5], fin;
    LNW pe3_norm, pe4_norm;
    BlockW blk[4];                 // block1, block2, dblock1, dblock2
};

struct Model {
    NetW gc, dr;
};

// Parses one ONNX model into `net`.  Returns 0 or a GCDR_ERR_* code with a
// message in `err`.
int parse_gcdr_net(const uint8_t *data, size_t len, NetW &net, std::string &err);
std::string describe_net(const NetW &n);

}  // namespace gcdr
