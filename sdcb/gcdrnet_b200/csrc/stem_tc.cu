// stem_tc.cu -- tensor-core stem (enc1 conv + maxpool + relu, gc#22-25) and
// head (UpHead with the stem skip recomputed, Extensions/UpHeadOp.cs:8-28,
// 249-279, then div6 or the u8 output) for sm_100a.
//
// The 3x3 stem conv over the net input is the one layer whose arithmetic the
// output is sensitive to (its result feeds the head directly), so it keeps
// fp32-level accuracy on fp16 tensor cores:
//   * the image part of the input is u8/255: the u8 values are exact in
//     fp16, so the conv runs on the integers with the weights split
//     w = w_hi + w_lo (both fp16), accumulates in fp32 and scales by 1/255
//     in the epilogue (accumulator D1);
//   * the DR input's second half r = clamp(x / I_sm, 0, 1) is split the same
//     way, r = r_hi + r_lo, and D2 = r_hi*w_hi + r_lo*w_hi + r_hi*w_lo.
// Per 128-pixel tile the four warps build the im2col rows (27 u8 taps, 27 r_hi,
// 27 r_lo, zero padded to 128 fp16 columns) straight into a SWIZZLE_128B
// K-major shared-memory tile, one thread issues the tcgen05.mma chain into
// TMEM, and each thread then finishes its own pixel from TMEM.
#include <cuda_runtime.h>

#include "kernels.h"
#include "tc_util.cuh"

namespace gcdr {
namespace {

constexpr int kABlock = 128 * 128;           // bytes of one 64-column SW128 block of the A tile
constexpr int kBBlock = 32 * 128;            // bytes of one 32-row x 64-column SW128 block of a B matrix
// Staged B blocks: GC uses x_hi and x_lo over columns 0..63; DR adds r_hi over
// columns 0..127 and r_lo over 0..63.  (matrix, 64-column block) -> slot:
__host__ __device__ constexpr int bslot(int m, int blk) { return m == 0 ? 0 : m == 1 ? 1 : m == 2 ? 2 + blk : 4; }
template <bool DR> constexpr int a_blocks() { return DR ? 2 : 1; }
template <bool DR> constexpr int b_slots() { return DR ? 5 : 2; }
template <bool DR> constexpr int tmem_cols() { return DR ? 64 : 32; }
template <bool DR> constexpr int stem_smem() { return 1024 + a_blocks<DR>() * kABlock + b_slots<DR>() * kBBlock + 1024 + 64 * 17 * 4; }

__device__ __forceinline__ int reflect1(int i, int n) {
    if (n <= 1) return 0;
    if (i < 0) return -i;
    if (i >= n) return 2 * n - 2 - i;
    return i;
}

// Byte offset of 16-byte chunk j (columns 8j..8j+7) of row r in a tile of
// 64-column SW128 blocks (`rows` rows per block).
__device__ __forceinline__ uint32_t sw_off(int r, int j, int rows) {
    return (uint32_t)((j >> 3) * rows * 128 + r * 128 + (((j & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void put_chunk(uint8_t *base, int r, int j, const __half *v8) {
    *reinterpret_cast<uint4 *>(base + sw_off(r, j, 128)) = *reinterpret_cast<const uint4 *>(v8);
}

// im2col row of pixel (py, px) of the padded image into row `row` of the A tile.
template <bool DR>
__device__ __forceinline__ void build_row(uint8_t *A, int row, const ImgSpec &im, const float *r, int H, int W, int py,
                                          int px) {
    __align__(16) __half u[32];
    __align__(16) __half rh[32];
    __align__(16) __half rl[32];
    const int ob = im.swap ? 2 : 0;
#pragma unroll
    for (int ky = 0; ky < 3; ky++) {
        const int yy = reflect1(py + ky - 1, H);
        const int sy = max(yy - im.ph, 0);
#pragma unroll
        for (int kx = 0; kx < 3; kx++) {
            const int xx = reflect1(px + kx - 1, W);
            const int sx = max(xx - im.pw, 0);
            const uint8_t *p = im.src + (size_t)sy * im.stride + (size_t)sx * im.bpp;
            const int t = (ky * 3 + kx) * 3;
            u[t + 0] = __ushort2half_rn(p[ob]);
            u[t + 1] = __ushort2half_rn(p[1]);
            u[t + 2] = __ushort2half_rn(p[2 - ob]);
            if (DR) {
                const float *rp = r + ((size_t)yy * W + xx) * 3;
#pragma unroll
                for (int c = 0; c < 3; c++) {
                    const float v = rp[c];
                    const __half hi = __float2half_rn(v);
                    rh[t + c] = hi;
                    rl[t + c] = __float2half_rn(v - __half2float(hi));
                }
            }
        }
    }
#pragma unroll
    for (int k = 27; k < 32; k++) {
        u[k] = __ushort2half_rn(0);
        rh[k] = __ushort2half_rn(0);
        rl[k] = __ushort2half_rn(0);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) put_chunk(A, row, j, u + 8 * j);
    if (DR) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            put_chunk(A, row, 4 + j, rh + 8 * j);
            put_chunk(A, row, 8 + j, rl + 8 * j);
        }
    }
}

struct StemShared {
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort_flag;
};

// D1 (cols 0..31) and D2 (cols 32..63) of this tile.
template <bool DR>
__device__ __forceinline__ void issue_mmas(uint32_t tmem, uint32_t a_s, uint32_t b_s, int c1) {
    const uint32_t idesc = (1u << 4) | ((uint32_t)(c1 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    auto ad = [&](int step) { return sdesc(a_s + (step >> 2) * kABlock + (step & 3) * 32, 1024, 2); };
    auto bd = [&](int m, int step) { return sdesc(b_s + bslot(m, step >> 2) * kBBlock + (step & 3) * 32, 1024, 2); };
    // x part: u8 columns 0..31 with w_x_hi then w_x_lo
    mma_f16(tmem, ad(0), bd(0, 0), idesc, 0u);
    mma_f16(tmem, ad(1), bd(0, 1), idesc, 1u);
    mma_f16(tmem, ad(0), bd(1, 0), idesc, 1u);
    mma_f16(tmem, ad(1), bd(1, 1), idesc, 1u);
    if (DR) {
        const uint32_t d2 = tmem + 32;
        // r_hi (cols 32..63) and r_lo (64..95) with w_r_hi; r_hi with w_r_lo
        mma_f16(d2, ad(2), bd(2, 2), idesc, 0u);
        mma_f16(d2, ad(3), bd(2, 3), idesc, 1u);
        mma_f16(d2, ad(4), bd(2, 4), idesc, 1u);
        mma_f16(d2, ad(5), bd(2, 5), idesc, 1u);
        mma_f16(d2, ad(2), bd(3, 2), idesc, 1u);
        mma_f16(d2, ad(3), bd(3, 3), idesc, 1u);
    }
}

template <int C1, bool DR>
__device__ __forceinline__ void load_c1(uint32_t taddr, int c0, const float *bias, float *c1) {
    float v1[16], v2[16];
    TmemLoader{taddr}.load16(c0, v1);
    if (DR) TmemLoader{taddr + 32}.load16(c0, v2);
#pragma unroll
    for (int k = 0; k < 16; k++) c1[k] = bias[c0 + k] + v1[k] * (1.0f / 255.0f) + (DR ? v2[k] : 0.0f);
}

// One persistent kernel per role: HEAD=false -> stem (conv + pool + relu -> t1),
// HEAD=true -> head (skip recompute + bilinear + 1x1 + sigmoid -> r or u8).
template <int C1, bool DR, bool HEAD>
__global__ void __launch_bounds__(128) stem_tc_kernel(const StemArgs sa, const HeadArgs ha, const __half *bpack,
                                                      int ntiles, int tiles_x, int *err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *A = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *B = A + a_blocks<DR>() * kABlock;
    StemShared *sh = reinterpret_cast<StemShared *>(B + b_slots<DR>() * kBBlock);
    float *xchg = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(sh) + 1024);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const ImgSpec &im = HEAD ? ha.img : sa.img;
    const float *rin = HEAD ? ha.r : sa.r;
    const int H = HEAD ? ha.H : sa.H, W = HEAD ? ha.W : sa.W;
    const float *bias = HEAD ? ha.b : sa.b;

    // zero the A tile (padding columns stay zero), stage the swizzled B blocks
    for (int i = tid; i < a_blocks<DR>() * kABlock / 16; i += 128) reinterpret_cast<uint4 *>(A)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < 4 * 32 * 16; i += 128) {
        const int m = i / (32 * 16), rem = i % (32 * 16), n = rem / 16, j = rem % 16;
        const int blk = j >> 3;
        const bool staged = m < 2 ? blk == 0 : (DR && (m == 2 || blk == 0));
        if (!staged) continue;
        *reinterpret_cast<uint4 *>(B + bslot(m, blk) * kBBlock + sw_off(n, j & 7, 32)) =
            *reinterpret_cast<const uint4 *>(bpack + ((size_t)(m * 32 + n) * 128 + j * 8));
    }
    if (tid == 0) {
        mbar_init(&sh->mma_done, 1);
        sh->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        __syncwarp();
        tmem_alloc(&sh->tmem_base, tmem_cols<DR>());
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh->tmem_base;
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t a_s = smem_u32(A), b_s = smem_u32(B);
    volatile int *abort_flag = &sh->abort_flag;

    int t = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, t++) {
        // ---- im2col rows
        int py, px, oy = 0, ox = 0;
        bool valid;
        int y2 = 0, xt = 0;
        if (!HEAD) {
            y2 = tile / tiles_x;
            xt = tile - y2 * tiles_x;
            const int sub = tid >> 6, xx = tid & 63;
            py = 2 * y2 + sub;
            px = xt * 64 + xx;
            valid = px < W;
            if (!valid) px = W - 1;
        } else {
            const int ow = DR ? im.w : W, oh = DR ? im.h : H;
            long long p = (long long)tile * 128 + tid;
            valid = p < (long long)ow * oh;
            if (!valid) p = (long long)ow * oh - 1;
            oy = (int)(p / ow);
            ox = (int)(p - (long long)oy * ow);
            py = DR ? oy + im.ph : oy;
            px = DR ? ox + im.pw : ox;
        }
        build_row<DR>(A, tid, im, rin, H, W, py, px);
        // head: relu(bilinear x2 of dec5) at this pixel (half_pixel, edge clamp), loaded
        // while the im2col loads are in flight, before waiting on the MMAs
        float up[HEAD ? C1 : 1];
        if (HEAD) {
            const int Hh = H / 2, Wh = W / 2;
            const float fy = ((float)py + 0.5f) / 2.0f - 0.5f, fx = ((float)px + 0.5f) / 2.0f - 0.5f;
            const int y0 = (int)floorf(fy), x0 = (int)floorf(fx);
            const float dy = fy - (float)y0, dx = fx - (float)x0;
            const int ya = min(max(y0, 0), Hh - 1), yb = min(max(y0 + 1, 0), Hh - 1);
            const int xa = min(max(x0, 0), Wh - 1), xb = min(max(x0 + 1, 0), Wh - 1);
            const __half *p00 = ha.dec5 + ((size_t)ya * Wh + xa) * C1, *p01 = ha.dec5 + ((size_t)ya * Wh + xb) * C1;
            const __half *p10 = ha.dec5 + ((size_t)yb * Wh + xa) * C1, *p11 = ha.dec5 + ((size_t)yb * Wh + xb) * C1;
#pragma unroll
            for (int c0 = 0; c0 < C1; c0 += 16) {
                float q00[16], q01[16], q10[16], q11[16];
                load16h(p00 + c0, q00);
                load16h(p01 + c0, q01);
                load16h(p10 + c0, q10);
                load16h(p11 + c0, q11);
#pragma unroll
                for (int k = 0; k < 16; k++) {
                    const float top = q00[k] + (q01[k] - q00[k]) * dx, bot = q10[k] + (q11[k] - q10[k]) * dx;
                    up[c0 + k] = fmaxf(top + (bot - top) * dy, 0.0f);
                }
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            issue_mmas<DR>(tmem, a_s, b_s, C1);
            mma_commit(&sh->mma_done);
        }
        const bool ok = mbar_wait(&sh->mma_done, (uint32_t)(t & 1), abort_flag, err);
        if (__syncthreads_or(!ok)) break;
        tc_fence_after();

        if (!HEAD) {
            const int sub = tid >> 6, xx = tid & 63;
            const int cx = xt * 64 + xx;
            const bool writer = sub == 0 && (xx & 1) == 0 && cx < W;
#pragma unroll
            for (int c0 = 0; c0 < C1; c0 += 16) {
                float v[16];
                load_c1<C1, DR>(taddr, c0, bias, v);
#pragma unroll
                for (int k = 0; k < 16; k++) v[k] = fmaxf(v[k], __shfl_xor_sync(0xffffffffu, v[k], 1));
                if (sub == 1) {
#pragma unroll
                    for (int k = 0; k < 16; k++) xchg[xx * 17 + k] = v[k];
                }
                __syncthreads();
                if (writer) {
                    __align__(16) __half h[16];
#pragma unroll
                    for (int k = 0; k < 16; k++) h[k] = __float2half_rn(fmaxf(fmaxf(v[k], xchg[xx * 17 + k]), 0.0f));
                    act_store(sa.out, y2, cx >> 1, c0, h, 16);
                }
                __syncthreads();
            }
        } else {
            float o0 = ha.fb[0], o1 = ha.fb[1], o2 = ha.fb[2];
#pragma unroll
            for (int c0 = 0; c0 < C1; c0 += 16) {
                float c1[16];
                load_c1<C1, DR>(taddr, c0, bias, c1);
#pragma unroll
                for (int k = 0; k < 16; k++) {
                    const float sv = (HEAD ? up[c0 + k] : 0.0f) + fmaxf(c1[k], 0.0f);
                    o0 = fmaf(sv, ha.fw[c0 + k], o0);
                    o1 = fmaf(sv, ha.fw[C1 + c0 + k], o1);
                    o2 = fmaf(sv, ha.fw[2 * C1 + c0 + k], o2);
                }
            }
            if (valid) {
                const float o[3] = {1.0f / (1.0f + expf(-o0)), 1.0f / (1.0f + expf(-o1)), 1.0f / (1.0f + expf(-o2))};
                const int ob = im.swap ? 2 : 0;
                if (!DR) {
                    const int sy = max(py - im.ph, 0), sx = max(px - im.pw, 0);
                    const uint8_t *sp = im.src + (size_t)sy * im.stride + (size_t)sx * im.bpp;
                    const float xv[3] = {(float)sp[ob] / 255.0f, (float)sp[1] / 255.0f, (float)sp[2 - ob] / 255.0f};
                    const size_t base = ((size_t)py * W + px) * 3;
#pragma unroll
                    for (int c = 0; c < 3; c++) {
                        const float d = o[c] > 1e-6f ? o[c] : 1e-6f;
                        float q = xv[c] / d;
                        q = q < 0.0f ? 0.0f : (q > 1.0f ? 1.0f : q);
                        ha.r_out[base + c] = q;
                        if (ha.ism_out) ha.ism_out[base + c] = o[c];
                    }
                } else {
                    if (ha.y_out) {
                        const size_t base = ((size_t)py * W + px) * 3;
                        for (int c = 0; c < 3; c++) ha.y_out[base + c] = o[c];
                    }
                    uint8_t q[3];
#pragma unroll
                    for (int c = 0; c < 3; c++) {
                        float f = o[c] * 255.0f + 0.5f;
                        f = f < 0.0f ? 0.0f : (f > 255.0f ? 255.0f : f);
                        q[c] = (uint8_t)f;
                    }
                    uint8_t *d = ha.dst + ((size_t)oy * im.w + ox) * im.bpp;
                    if (im.bpp == 4) {
                        uchar4 v;
                        v.x = ob ? q[2] : q[0];
                        v.y = q[1];
                        v.z = ob ? q[0] : q[2];
                        v.w = im.src[(size_t)oy * im.stride + (size_t)ox * 4 + 3];
                        *reinterpret_cast<uchar4 *>(d) = v;
                    } else {
                        d[ob] = q[0];
                        d[1] = q[1];
                        d[2 - ob] = q[2];
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (sh->abort_flag && tid == 0) {
        // the last MMA chain may still be in flight: wait for it (bounded) before freeing TMEM
        long long t0 = clock64();
        while (!mbar_try(&sh->mma_done, (uint32_t)(t & 1)) && clock64() - t0 < kWaitCycles) {}
    }
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols<DR>());
    }
}

template <int C1, bool DR, bool HEAD>
int launch_one(const StemArgs &sa, const HeadArgs &ha, const __half *bpack, int ntiles, int tiles_x, int *err,
               int num_sms, cudaStream_t st) {
    auto k = stem_tc_kernel<C1, DR, HEAD>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, stem_smem<DR>()) != cudaSuccess) return -1;
    // persistent grid: exactly the CTAs that can be resident at once, limited by
    // shared memory, registers and TMEM (512 columns per SM); a second wave of a
    // persistent kernel only adds start-up work and a tail
    cudaFuncAttributes fa;
    int dev = 0, smem_sm = 0, reserved = 0;
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess) return -1;
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    const int by_smem = smem_sm / (stem_smem<DR>() + (int)fa.sharedSizeBytes + reserved);
    const int regs_per_warp = (fa.numRegs * 32 + 255) / 256 * 256;
    const int by_regs = 65536 / (regs_per_warp * 4);
    const int per_sm = max(1, min(min(by_smem, by_regs), min(512 / tmem_cols<DR>(), 16)));
    const int grid = min(ntiles, num_sms * per_sm);
    k<<<grid, 128, stem_smem<DR>(), st>>>(sa, ha, bpack, ntiles, tiles_x, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace

int stem_tc_launch(const StemArgs &a, const __half *bpack, int num_sms, int *err, cudaStream_t st) {
    const int tiles_x = (a.W + 63) / 64, ntiles = (a.H / 2) * tiles_x;
    HeadArgs none;
    if (a.cin == 3 && a.c1 == 16) return launch_one<16, false, false>(a, none, bpack, ntiles, tiles_x, err, num_sms, st);
    if (a.cin == 6 && a.c1 == 32) return launch_one<32, true, false>(a, none, bpack, ntiles, tiles_x, err, num_sms, st);
    if (a.cin == 3 && a.c1 == 32) return launch_one<32, false, false>(a, none, bpack, ntiles, tiles_x, err, num_sms, st);
    if (a.cin == 6 && a.c1 == 16) return launch_one<16, true, false>(a, none, bpack, ntiles, tiles_x, err, num_sms, st);
    return -2;
}

int head_tc_launch(const HeadArgs &a, const __half *bpack, int num_sms, int *err, cudaStream_t st) {
    const long long n = a.is_dr ? (long long)a.img.w * a.img.h : (long long)a.H * a.W;
    const int ntiles = (int)((n + 127) / 128);
    StemArgs none;
    if (!a.is_dr && a.cin == 3 && a.c1 == 16) return launch_one<16, false, true>(none, a, bpack, ntiles, 0, err, num_sms, st);
    if (!a.is_dr && a.cin == 3 && a.c1 == 32) return launch_one<32, false, true>(none, a, bpack, ntiles, 0, err, num_sms, st);
    if (a.is_dr && a.cin == 6 && a.c1 == 32) return launch_one<32, true, true>(none, a, bpack, ntiles, 0, err, num_sms, st);
    if (a.is_dr && a.cin == 6 && a.c1 == 16) return launch_one<16, true, true>(none, a, bpack, ntiles, 0, err, num_sms, st);
    return -2;
}

// Packs the stem weights ONNX [C1][Cin][3][3] into the four B matrices the
// kernels stage: [x_hi, x_lo, r_hi, r_lo] x [32 rows][128 columns] fp16, row =
// output channel, columns matching the im2col A layout (tap*3 + ci for the
// image part at 0..26, the r part at 32..58 (r_hi) and 64..90 (r_lo)).
void pack_stem_weights(const float *w, int c1, int cin, __half *out) {
    for (int i = 0; i < 4 * 32 * 128; i++) out[i] = __float2half_rn(0.0f);
    auto at = [&](int m, int n, int col) -> __half & { return out[((size_t)m * 32 + n) * 128 + col]; };
    for (int n = 0; n < c1; n++)
        for (int tap = 0; tap < 9; tap++)
            for (int ci = 0; ci < cin; ci++) {
                const float v = w[((size_t)n * cin + ci) * 9 + tap];
                const __half hi = __float2half_rn(v);
                const __half lo = __float2half_rn(v - __half2float(hi));
                if (ci < 3) {
                    at(0, n, tap * 3 + ci) = hi;
                    at(1, n, tap * 3 + ci) = lo;
                } else {
                    const int c = tap * 3 + (ci - 3);
                    at(2, n, 32 + c) = hi;
                    at(2, n, 64 + c) = hi;
                    at(3, n, 32 + c) = lo;
                }
            }
}

}  // namespace gcdr
