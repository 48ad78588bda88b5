// conv_ref.cu -- SIMT reference of the implicit-GEMM convolution.
//
// Computes the same sum as conv_tc.cu with fp32 FMAs straight from global
// memory, stages the accumulators in a scratch buffer laid out like the TMEM
// tile (tile, row, column), then runs the identical epilogue.  It exists to
// check the tensor-core kernel layer by layer on the GPU; the pipeline never
// uses it.
#include "conv_launch.h"

namespace gcdr {
namespace {

// Rows of the output grid the reference computes: every q = y * pitch + x the
// tensor-core kernel can touch (pool: the conv rows; plain: whole 128-row tiles).
long long ref_rows(const TileGeom &tg) {
    return tg.pool ? (long long)tg.conv_h * tg.pitch : (long long)tg.ntiles * 128;
}

__global__ void ref_gemm_kernel(const ConvArgs a, long long rows, float *scratch) {
    const long long q = (long long)blockIdx.x * 128 + threadIdx.x;
    const int n0 = blockIdx.y * 16;
    if (q >= rows) return;
    float acc[16];
#pragma unroll
    for (int k = 0; k < 16; k++) acc[k] = 0.f;
    const int K = a.ntaps * a.C;
    for (int tap = 0; tap < a.ntaps; tap++) {
        const long long ar = q + a.tap_off[tap];
        if (ar < 0 || ar >= a.a_rows) continue;   // TMA reads zeros out of bounds
        const __half *ap = a.A + ar * a.C;
        for (int c = 0; c < a.C; c++) {
            const float x = __half2float(ap[c]);
            const __half *bp = a.B + (long long)n0 * K + (long long)tap * a.C + c;
#pragma unroll
            for (int k = 0; k < 16; k++) acc[k] = fmaf(x, __half2float(bp[(long long)k * K]), acc[k]);
        }
    }
    float *o = scratch + q * a.N + n0;
#pragma unroll
    for (int k = 0; k < 16; k++) o[k] = acc[k];
}

struct ScratchLoader {
    const float *p;
    __device__ void load16(int c0, float *v) {
#pragma unroll
        for (int k = 0; k < 16; k++) v[k] = p[c0 + k];
    }
    __device__ void load32(int c0, float *v) {
#pragma unroll
        for (int k = 0; k < 32; k++) v[k] = p[c0 + k];
    }
};

template <int MODE>
__global__ void ref_epilogue_kernel(const ConvArgs a, const float *scratch) {
    const int tile = blockIdx.x, row = threadIdx.x;
    ScratchLoader ld{scratch + ((long long)tile * 128 + row) * a.N};
    epilogue_tile<MODE>(a.ep, a.tg, tile, row, 0, a.N, a.N, 0, ld);
}

// Pool: block (y2, segment of 128 conv columns); the same epilogue_pool as the
// tensor-core kernel, fed from the two conv rows in scratch.
__global__ void ref_pool_kernel(const ConvArgs a, const float *scratch) {
    const int y2 = blockIdx.x, x = blockIdx.y * 128 + threadIdx.x;
    const int xc = x < a.tg.pitch ? x : a.tg.pitch - 1;   // lanes past the row read a valid row
    ScratchLoader top{scratch + ((long long)(2 * y2) * a.tg.pitch + xc) * a.N};
    ScratchLoader bot{scratch + ((long long)(2 * y2 + 1) * a.tg.pitch + xc) * a.N};
    epilogue_pool(a.ep, a.tg, y2, x, 0, a.N, top, bot);
}

}  // namespace

size_t ref_conv_scratch_floats(const ConvArgs &a) { return (size_t)ref_rows(a.tg) * a.N; }

int ref_conv_launch(const ConvArgs &a, int mode, float *scratch, cudaStream_t st, std::string &err) {
    if (a.N % 16 || a.tg.ntiles < 1 || a.nsplit != 1 || a.ksplit != 1) { err = "ref conv: bad shape"; return -1; }
    if (a.nimg != 1) { err = "ref conv: one image per launch"; return -1; }
    if ((mode == EPI_POOL) != (a.tg.pool != 0)) { err = "ref conv: pool geometry / mode mismatch"; return -1; }
    if (a.tg.pool && (a.tg.conv_h % 2 || a.tg.conv_w % 2 || a.tg.pitch < a.tg.conv_w)) {
        err = "ref conv: bad pool geometry";
        return -1;
    }
    const long long rows = ref_rows(a.tg);
    ref_gemm_kernel<<<dim3((unsigned)((rows + 127) / 128), a.N / 16), 128, 0, st>>>(a, rows, scratch);
    switch (mode) {
        case EPI_PLAIN: ref_epilogue_kernel<EPI_PLAIN><<<a.tg.ntiles, 128, 0, st>>>(a, scratch); break;
        case EPI_POOL:
            ref_pool_kernel<<<dim3(a.tg.conv_h / 2, (a.tg.conv_w + 127) / 128), 128, 0, st>>>(a, scratch);
            break;
        case EPI_LN2: ref_epilogue_kernel<EPI_LN2><<<a.tg.ntiles, 128, 0, st>>>(a, scratch); break;
        case EPI_RESLN: ref_epilogue_kernel<EPI_RESLN><<<a.tg.ntiles, 128, 0, st>>>(a, scratch); break;
        default: err = "bad epilogue mode"; return -1;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { err = std::string("ref conv launch: ") + cudaGetErrorString(e); return -1; }
    return 0;
}

}  // namespace gcdr
