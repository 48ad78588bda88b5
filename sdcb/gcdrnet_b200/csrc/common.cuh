// common.cuh -- activation layouts and store helpers shared by every kernel.
//
// Activations are NHWC fp16 (the tensor-core operand type) in one of three
// layouts, chosen by who reads them next:
//
//   LAY_PLAIN    [H][W][C]                       tokens, decoder conv outputs
//   LAY_PADREFL  [H+2][W+2][C] with a 1-px reflect border (ONNX Pad
//                mode=reflect, gc#22/26/30/234/...): the input of a stride-1
//                3x3 conv.  Flattened to rows of C, every conv tap is then a
//                constant row offset from the output position, so each tap's
//                operand tile is one rectangular TMA box.
//   LAY_PHASE    four planes P[dy][dx] of [(H+2)/2][(W+2)/2][C] holding the
//                zero-padded input at (2Y+dy, 2X+dx): the input of a stride-2
//                pad-1 3x3 conv (the patch embeds gc#34/134).  Tap (ky,kx)
//                reads plane (ky&1,kx&1) at a constant row offset.  The zero
//                border is written once when the arena is planned.
//   LAY_PADZERO  as LAY_PADREFL with a zero border (a zero-padded stride-1
//                conv; used by the conv microbenchmark).
//
// Producers write the interior and, for LAY_PADREFL, the mirrored border
// copies (reflect of 1 px: padded row 0 = row 1, padded row H+1 = row H-2;
// a dimension of size 1 mirrors onto itself).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

namespace gcdr {

enum LayoutKind : int { LAY_PLAIN = 0, LAY_PADREFL = 1, LAY_PHASE = 2, LAY_PADZERO = 3 };

// Programmatic dependent launch: every pipeline kernel is launched with
// launch_pdl, waits for its predecessor grid before its first access to
// activations (read or write), and lets its successor launch early: persistent
// kernels right after their setup, the others when each block is done.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();   // GCDR_CUDA_PDL=0 turns it off (kernels.cu)

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Image source / destination as the caller laid it out (GcdrPixelFormat).
struct ImgSpec {
    const uint8_t *src = nullptr;   // device copy of the source image
    int w = 0, h = 0, stride = 0;   // original dims, row stride in bytes
    int bpp = 3, swap = 0;          // bytes per pixel, R/B swapped (Rgb24/Rgba32)
    int ph = 0, pw = 0;             // top/left replicate pad to /32
};

struct Act {
    __half *p = nullptr;
    int H = 0, W = 0, C = 0;   // logical dims of the stored tensor
    int kind = LAY_PLAIN;

    __host__ __device__ int pitch() const {       // rows per padded image row
        return (kind == LAY_PADREFL || kind == LAY_PADZERO) ? W + 2 : kind == LAY_PHASE ? (W + 2) / 2 : W;
    }
    __host__ __device__ long long plane_rows() const {
        return (long long)((H + 2) / 2) * ((W + 2) / 2);
    }
    __host__ __device__ long long rows() const {  // rows of C elements allocated
        return (kind == LAY_PADREFL || kind == LAY_PADZERO) ? (long long)(H + 2) * (W + 2)
             : kind == LAY_PHASE ? 4 * plane_rows() : (long long)H * W;
    }
    __host__ __device__ size_t bytes() const { return (size_t)rows() * C * sizeof(__half); }
    // Row index of logical pixel (y, x) (its interior copy).
    __host__ __device__ long long row(int y, int x) const {
        if (kind == LAY_PADREFL || kind == LAY_PADZERO) return (long long)(y + 1) * (W + 2) + (x + 1);
        if (kind == LAY_PHASE) {
            int py = y + 1, px = x + 1;
            return ((py & 1) * 2 + (px & 1)) * plane_rows() + (long long)(py >> 1) * ((W + 2) / 2) + (px >> 1);
        }
        return (long long)y * W + x;
    }
};

// Batched launches: the buffers of image k lie k * img_bytes past image 0's (a batch plan's
// image slices, one after another in the shape's arena).  Callers test an optional pointer
// for null before they offset it.  (Byte arithmetic on the pointer itself, not through an
// integer: the compiler keeps knowing that a kernel parameter's pointer is global memory.)
template <class T>
__host__ __device__ inline T *img_at(T *p, size_t off) {
    using B = typename std::conditional<std::is_const<T>::value, const char, char>::type;
    return reinterpret_cast<T *>(reinterpret_cast<B *>(p) + off);
}

__host__ __device__ inline int refl_lo(int n) { return n > 1 ? 1 : 0; }      // source of padded index 0
__host__ __device__ inline int refl_hi(int n) { return n > 1 ? n - 2 : 0; }  // source of padded index n+1

// Calls put(r) for the row r of pixel (y, x) and, for LAY_PADREFL, for each
// border copy that mirrors it (no arrays: interior pixels return after one put).
// interior = false: the border copies only.
template <class F>
__device__ __forceinline__ void act_rows(const Act &a, int y, int x, F &&put, bool interior = true) {
    if (interior) put(a.row(y, x));
    if (a.kind != LAY_PADREFL) return;
    const bool ylo = y == refl_lo(a.H), yhi = y == refl_hi(a.H);
    const bool xlo = x == refl_lo(a.W), xhi = x == refl_hi(a.W);
    if (!(ylo || yhi || xlo || xhi)) return;
    const long long P = a.W + 2, top = 0, bot = (long long)(a.H + 1) * P, row = (long long)(y + 1) * P;
    if (ylo) put(top + x + 1);
    if (yhi) put(bot + x + 1);
    if (xlo) put(row);
    if (xhi) put(row + a.W + 1);
    if (ylo && xlo) put(top);
    if (ylo && xhi) put(top + a.W + 1);
    if (yhi && xlo) put(bot);
    if (yhi && xhi) put(bot + a.W + 1);
}

// Stores `n` halves (n multiple of 2, 4-byte aligned) at channel c0 of pixel
// (y, x), plus the reflect-border copies for LAY_PADREFL.  io: byte offset of the
// image in a batched launch (the tensor of image k lies k * img_bytes past a.p).
__device__ __forceinline__ void act_store(const Act &a, int y, int x, int c0, const __half *v, int n, size_t io = 0) {
    __half *base = img_at(a.p, io);
    act_rows(a, y, x, [&](long long r) {
        __half *d = base + r * a.C + c0;
        if ((n & 7) == 0 && ((reinterpret_cast<uintptr_t>(d) & 15) == 0)) {
            for (int k = 0; k < n; k += 8) *reinterpret_cast<uint4 *>(d + k) = *reinterpret_cast<const uint4 *>(v + k);
        } else {
            for (int k = 0; k < n; k += 2) *reinterpret_cast<__half2 *>(d + k) = *reinterpret_cast<const __half2 *>(v + k);
        }
    });
}

// The reflect-border copies of act_store alone (LAY_PADREFL; nothing for other layouts).
__device__ __forceinline__ void act_store_borders(const Act &a, int y, int x, int c0, const __half *v, int n,
                                                  size_t io) {
    if (a.kind != LAY_PADREFL) return;
    __half *base = img_at(a.p, io);
    act_rows(a, y, x, [&](long long r) {
        __half *d = base + r * a.C + c0;
        for (int k = 0; k < n; k += 8) *reinterpret_cast<uint4 *>(d + k) = *reinterpret_cast<const uint4 *>(v + k);
    }, false);
}

// A warp's store of up to 32 pixels p < npix (consecutive along a row, where the layout allows),
// channels [c0, c0 + CW) (CW = 16 or 32 halves), staged through the warp's shared-memory buffer
// `stg` (npix * CW * 2 bytes, 16-byte aligned) so that each store instruction writes contiguous
// 16-byte chunks of consecutive pixels instead of one pixel's chunk per lane: lanes write their
// pixel into the buffer (chunk j of pixel p at 16-byte slot j ^ f(p), f spreading a quarter-warp
// over all banks), then each lane stores chunks q = lane, lane + 32, ... (pixel q / (CW/8)) from
// it.  has_px: this lane holds pixel `my_p` in h; pix(p, y, x): pixel p's logical coordinates,
// false when it is not stored.  Reflect-border copies (LAY_PADREFL) go out per lane afterwards.
// Warp-collective.
template <int CW, class Pix>
__device__ __forceinline__ void warp_store_staged(const Act &a, int c0, const __half *h, bool has_px, int my_p,
                                                  int npix, Pix &&pix, uint8_t *stg, size_t io) {
    constexpr int CPP = CW / 8;                       // 16-byte chunks per pixel
    constexpr int SPREAD = 8 / CPP;                   // pixels per 128 bytes
    const int lane = threadIdx.x & 31;
    if (has_px) {
#pragma unroll
        for (int j = 0; j < CPP; j++) {
            const int slot = j ^ ((my_p / SPREAD) & (CPP - 1));
            *reinterpret_cast<uint4 *>(stg + my_p * (CW * 2) + slot * 16) = *reinterpret_cast<const uint4 *>(h + 8 * j);
        }
    }
    __syncwarp();
    __half *base = img_at(a.p, io);
#pragma unroll
    for (int i = 0; i < CPP; i++) {
        const int q = i * 32 + lane, p = q / CPP, j = q - p * CPP;
        int y, x;
        if (p < npix && pix(p, y, x)) {
            const int slot = j ^ ((p / SPREAD) & (CPP - 1));
            const uint4 d = *reinterpret_cast<const uint4 *>(stg + p * (CW * 2) + slot * 16);
            *reinterpret_cast<uint4 *>(base + a.row(y, x) * a.C + c0 + 8 * j) = d;
        }
    }
    __syncwarp();                                     // the buffer is free for the next store
    int y, x;
    if (has_px && pix(my_p, y, x)) act_store_borders(a, y, x, c0, h, CW, io);
}

// Two channels (c even) by value.
__device__ __forceinline__ void act_store2(const Act &a, int y, int x, int c, __half2 v, size_t io = 0) {
    __half *base = img_at(a.p, io);
    act_rows(a, y, x, [&](long long r) { *reinterpret_cast<__half2 *>(base + r * a.C + c) = v; });
}

__device__ inline const __half *act_ptr(const Act &a, int y, int x) { return a.p + a.row(y, x) * a.C; }

// Shift-MLP channel groups (Extensions/ChannelShiftOp.cs:8-13, GcdrKernels.cs:169-198):
// out[y,x,c] = in[y+off_g, x, c] (axis 2) or in[y, x+off_g, c] (axis 3), zero fill.
// Applied as a scatter by the producer: the value at source position s goes to
// (s - off) mod L; the |off| sources that fall off the edge carry zeros into the
// |off| vacated destinations, so every destination is written exactly once.
struct ShiftSpec {
    int ngroups = 0;
    int ends[5] = {0, 0, 0, 0, 0};
    int offs[5] = {0, 0, 0, 0, 0};
    // > 0 when group g covers [g*gs, min((g+1)*gs, C)) (ONNX Split into equal
    // ceil-sized chunks): the group of a channel is one division
    int gs = 0;
    // 1 when a group is narrower than 8 channels (a chunk of 8 may then span three
    // groups; the scatters fall back to channel pairs)
    int narrow = 0;
};

// Group of channel c (-1 past the last group).
__device__ inline int shift_group(const ShiftSpec &s, int c) {
    if (s.gs > 0) return c < s.ends[s.ngroups - 1] ? c / s.gs : -1;
    int g = 0;
    while (g < s.ngroups - 1 && c >= s.ends[g]) g++;
    return c < s.ends[s.ngroups - 1] ? g : -1;
}

// Destination of source coordinate `s` (along the shifted axis of length L)
// for offset `off`; *zero tells whether the destination receives zeros.
__device__ inline int shift_dest(int s, int off, int L, bool *zero) {
    int d = s - off;
    *zero = d < 0 || d >= L;
    if (*zero) {                        // rare: the wrapped column gets the zero (L may be 1 or 2)
        d %= L;
        if (d < 0) d += L;
    }
    return d;
}

// Stores channels c, c+1 (c even) of token pixel (y, x) of a LAY_PLAIN [H][W][C]
// tensor with the group shift along `axis` (2 = H, 3 = W) applied as a scatter;
// a pair in one group goes out as one 4-byte store.
__device__ __forceinline__ void shift_store2(const Act &a, const ShiftSpec &s, int axis, int y, int x, int c, float v0,
                                             float v1, size_t io = 0) {
    __half *base = img_at(a.p, io);
    const int g0 = shift_group(s, c), g1 = shift_group(s, c + 1);
    int dy = y, dx = x;
    bool z = false;
    if (g0 >= 0) {
        if (axis == 2) dy = shift_dest(y, s.offs[g0], a.H, &z);
        else dx = shift_dest(x, s.offs[g0], a.W, &z);
    }
    __half *d = base + ((size_t)dy * a.W + dx) * a.C + c;
    if (g0 == g1) {
        *reinterpret_cast<__half2 *>(d) = z ? __float2half2_rn(0.0f) : __floats2half2_rn(v0, v1);
    } else {
        d[0] = __float2half_rn(z ? 0.0f : v0);
        int ey = y, ex = x;
        bool z1 = false;
        if (g1 >= 0) {
            if (axis == 2) ey = shift_dest(y, s.offs[g1], a.H, &z1);
            else ex = shift_dest(x, s.offs[g1], a.W, &z1);
        }
        base[((size_t)ey * a.W + ex) * a.C + c + 1] = __float2half_rn(z1 ? 0.0f : v1);
    }
}

// Stores the channels [c0, c0+n) (n even, c0 even) of token pixel (y, x) with
// the group shift (shift_store2 per pair).
__device__ inline void shift_store(const Act &a, const ShiftSpec &s, int axis, int y, int x, int c0,
                                   const float *v, int n, size_t io = 0) {
    for (int k = 0; k < n; k += 2) shift_store2(a, s, axis, y, x, c0 + k, v[k], v[k + 1], io);
}

// Loads 8 consecutive halves (16-byte aligned) as floats.
__device__ inline void load16h8(const __half *p, float *v) {
    const uint4 a = *reinterpret_cast<const uint4 *>(p);
    const __half2 *ha = reinterpret_cast<const __half2 *>(&a);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 f = __half22float2(ha[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
    }
}

// Loads 16 consecutive halves (16-byte aligned) as floats.
__device__ inline void load16h(const __half *p, float *v) {
    const uint4 a = *reinterpret_cast<const uint4 *>(p), b = *reinterpret_cast<const uint4 *>(p + 8);
    const __half2 *ha = reinterpret_cast<const __half2 *>(&a), *hb = reinterpret_cast<const __half2 *>(&b);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float2 f = __half22float2(ha[k]), g = __half22float2(hb[k]);
        v[2 * k] = f.x; v[2 * k + 1] = f.y; v[8 + 2 * k] = g.x; v[8 + 2 * k + 1] = g.y;
    }
}

#define GCDR_ERR_FLAG_TIMEOUT 1
#define GCDR_ERR_FLAG_BOUNDS 2

// Default bound of a device-side wait: ~2 s of SM clock at 1.9 GHz.
constexpr long long kWaitCycles = 4000000000LL;

}  // namespace gcdr
