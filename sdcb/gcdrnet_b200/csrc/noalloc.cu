// noalloc.cu -- gcdr_k_conv_static: one k-split tensor-core convolution layer
// that allocates no device memory.
//
// The split-K form of the layer (gcdr_k_conv with epilogue 3) needs an fp32
// workspace of ksplit x Ho*Wo x N partial sums, which the caller normally
// allocates.  This entry keeps that workspace, and the kernels' error word, in
// one file-scope __device__ array compiled into the library, so a caller that
// may not allocate (a fixed memory budget, a memory pool that owns the whole
// device, code running where cudaMalloc is not allowed) can still run the
// layer.  The array is part of this file's device image: the driver reserves
// it on a device when the module is loaded there, which the first call on that
// device does through cudaGetSymbolAddress (every call looks the address up
// again).  That first call should therefore come before any stream capture.
// The call is synchronous: it reads the kernels' error word back before it
// returns.  Every call shares the one workspace per device, so calls that
// overlap in time (two host threads, or two streams without ordering between
// them) race on it.  The partial sums add no bias (the sum kernel adds it from
// the device bias), so no bias is read back to the host.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <string>

#include "../../../include/gcdr_cuda.h"
#include "conv_launch.h"

namespace gcdr {
int conv_args_from_desc(const gcdr_conv_desc *d, ConvArgs &a, int &mode, std::string &err);
}

using namespace gcdr;

namespace {

// 256 bytes of header (the error word at [0]), then the partial sums.
constexpr long long kHeaderFloats = 64;
constexpr long long kStaticWsFloats = GCDR_STATIC_WS_BYTES / 4;
static __device__ __align__(256) float g_static_ws[kHeaderFloats + kStaticWsFloats];

// out[t][n] = act(sum_k partial[k][t][n] + bias[n]), k summed in order; 8 channels a thread.
__global__ void splitk_sum_kernel(const float *__restrict__ partial, int ksplit, long long T, int N,
                                  const float *__restrict__ bias, int relu, __half *__restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int groups = N / 8;
    if (i >= T * groups) return;
    const long long t = i / groups;
    const int c0 = (int)(i - t * groups) * 8;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = 0.f;
    for (int k = 0; k < ksplit; k++) {
        const float4 *p = reinterpret_cast<const float4 *>(partial + ((long long)k * T + t) * N + c0);
        const float4 a = p[0], b = p[1];
        v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
        v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float y = v[j] + bias[c0 + j];
        h[j] = __float2half_rn(relu ? fmaxf(y, 0.f) : y);
    }
    *reinterpret_cast<uint4 *>(out + t * N + c0) = *reinterpret_cast<const uint4 *>(h);
}

// Device address of the current device's static workspace.  Looked up on every call (cheap
// once the module is loaded), so the address stays right after a device reset reloads the
// module at another address.
float *static_ws() {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_ws);
    if (e != cudaSuccess || !p) {
        std::fprintf(stderr, "gcdr_k_conv_static: cudaGetSymbolAddress failed: %s\n", cudaGetErrorString(e));
        return nullptr;
    }
    return static_cast<float *>(p);
}

}  // namespace

extern "C" int gcdr_k_conv_static(const gcdr_conv_desc *d, void *stream) {
    if (!d || (d->epilogue != 0 && d->epilogue != 2)) return GCDR_ERR_ARG;
    // run the layer as its split-K form: partial sums into the static workspace
    gcdr_conv_desc pd = *d;
    pd.epilogue = 3;
    pd.scratch = nullptr;
    ConvArgs a;
    int mode = 0;
    std::string err;
    if (conv_args_from_desc(&pd, a, mode, err)) {
        std::fprintf(stderr, "gcdr_k_conv_static: %s\n", err.c_str());
        return GCDR_ERR_ARG;
    }
    const long long T = (long long)a.tg.conv_h * a.tg.conv_w;
    const long long need = (long long)a.ksplit * T * a.N;
    if (need > kStaticWsFloats) {
        std::fprintf(stderr,
                     "gcdr_k_conv_static: ksplit x Ho*Wo x N = %lld floats exceeds the static workspace of %lld "
                     "floats (%d MiB); use fewer k splits or a smaller layer\n",
                     need, kStaticWsFloats, (int)(GCDR_STATIC_WS_BYTES >> 20));
        return GCDR_ERR_RANGE;
    }
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess) return GCDR_ERR_DEVICE;
    float *ws = static_ws();
    if (!ws) return GCDR_ERR_DEVICE;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int *err_word = reinterpret_cast<int *>(ws);
    float *partial = ws + kHeaderFloats;
    a.err = err_word;
    a.ep.partial = partial;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the error word must start at zero; the partials are overwritten in full
    if (cudaMemsetAsync(err_word, 0, sizeof(int), st) != cudaSuccess) return GCDR_ERR_DEVICE;
    if (tc_conv_launch(a, mode, sms, st, err)) {
        std::fprintf(stderr, "gcdr_k_conv_static: %s\n", err.c_str());
        return GCDR_ERR_DEVICE;
    }
    const long long n = T * (a.N / 8);
    splitk_sum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(partial, a.ksplit, T, a.N, d->bias,
                                                                     d->epilogue == 2, static_cast<__half *>(d->out));
    if (cudaGetLastError() != cudaSuccess) return GCDR_ERR_DEVICE;
    // the bounded waits of the conv kernel report a timeout through the error word
    int h_err = 0;
    if (cudaMemcpyAsync(&h_err, err_word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return GCDR_ERR_DEVICE;
    return h_err ? GCDR_ERR_TIMEOUT : GCDR_OK;
}
