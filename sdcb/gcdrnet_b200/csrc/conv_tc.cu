// conv_tc.cu -- tcgen05 (sm_100a) implicit-GEMM convolution.
//
// One persistent CTA per SM, 13 warps:
//   warp 0      TMA producer: per (tap, k-block) the unit's A rows (two boxes,
//               SWIZZLE_{32,64,128}B K-major) and the B tile (weights) into a
//               multi-stage shared-memory ring; also allocates TMEM.
//   warps 1-4   MMA issuers, one per accumulator of the unit (a 128-row
//               sub-tile, or one 256-column half of N): each issues its own
//               tcgen05.mma.kind::f16 chain (fp16 x fp16 -> fp32, M=128,
//               N<=256) and commits.  A single issuing thread spends ~100-200
//               cycles per MMA whatever N is, so thin layers (N <= 64) are
//               issue-bound with one issuer; four issuers overlap their chains.
//   warps 5-12  epilogue: tcgen05.ld 32x32b rows out of TMEM (thread = output
//               position; two warps per TMEM lane quadrant share the column
//               chunks), bias / pool / LayerNorm / residual / shift, stores.
// Accumulators are double-buffered in TMEM when both buffers fit in 512
// columns, so the epilogue of unit i overlaps the MMAs of unit i+1.
//
// Every mbarrier wait is bounded (clock64 budget): on expiry the CTA raises the
// abort flag, sets GCDR_ERR_FLAG_TIMEOUT in the global error word, drains its
// own copies in flight (bounded), frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <string>

#include "conv.cuh"
#include "conv_launch.h"
#include "tc_util.cuh"

namespace gcdr {

namespace {

constexpr int kMmaWarps = 4;
constexpr int kEpiWarps = 8;
constexpr int kTcSmemCap = 200 * 1024;   // the ring budget below plus the barriers and alignment
constexpr int kConvThreads = (2 + kMmaWarps + kEpiWarps) * 32;
constexpr int kProducer2Warp = 1 + kMmaWarps + kEpiWarps;     // the second TMA producer

struct TcShared {
    uint64_t full[kMaxStages], empty[kMaxStages], tfull[2], tempty[2], mdone[kMmaWarps];
    uint32_t tmem_base;
    int abort_flag;
    int issued[2], consumed;
};

// A work unit covers `nst` 128-row MMA sub-tiles: rt consecutive tiles (plain),
// or the two conv rows of a pooled row x 128*rt pixels (pool: nst = 2*rt, the
// top row's sub-tiles first).  Its A rows arrive as two TMA boxes of nst*64 rows.
template <int BK, int MODE>
__global__ void __launch_bounds__(kConvThreads, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ ConvArgs args, const __grid_constant__ TcConfig cfg) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    TcShared *sh = reinterpret_cast<TcShared *>(ring + (size_t)cfg.stages * cfg.stage_bytes);
    constexpr bool kLnUnits = MODE == EPI_LN2 || MODE == EPI_RESLN;   // whole rows, units split by buffer

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom &tg = args.tg;
    const int N = args.N;
    const int Ns = N / args.nsplit;                               // channels of one unit
    const int kb_per_tap = args.C / BK;
    const int kblocks = args.ntaps * kb_per_tap / args.ksplit;    // k-blocks of one unit
    const int nst = MODE == EPI_POOL ? 2 * cfg.rt : cfg.rt;      // 128-row sub-tiles per unit
    const int munits = m_units(tg, cfg.rt);
    const int segs = MODE == EPI_POOL ? (tg.conv_w + 128 * cfg.rt - 1) / (128 * cfg.rt) : 1;
    const int img_units = munits * args.nsplit * args.ksplit;   // units of one image
    const int nunits = img_units * args.nimg;                    // image-major over a batch
    const bool batched = args.nimg > 1;                          // the activation map's rank: 3, else 2
    const uint32_t a_bytes = 128u * nst * BK * 2u;
    const uint32_t b_bytes = (uint32_t)Ns * BK * 2u;
    const int nsub = (Ns + 255) / 256;
    const int nacc = nst * nsub;                                  // accumulators = active MMA warps (<= 4)

    if (threadIdx.x == 0) {
        for (int s = 0; s < cfg.stages; s++) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], (uint32_t)nacc);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sh->tfull[b], (uint32_t)nacc);
            mbar_init(&sh->tempty[b], kLnUnits ? kEpiWarps / 2 : kEpiWarps);
        }
        for (int m = 0; m < kMmaWarps; m++) mbar_init(&sh->mdone[m], 1);
        sh->abort_flag = 0;
        sh->issued[0] = sh->issued[1] = 0;
        sh->consumed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh->tmem_base)),
                     "r"((uint32_t)cfg.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = sh->tmem_base;
    volatile int *abort_flag = &sh->abort_flag;
    const long long budget = wait_budget(args);
    pdl_trigger();                          // all CTAs are resident: the next kernel may start launching
    pdl_wait();                             // activations of the previous kernels

    if (warp == 0 || warp == kProducer2Warp) {
        // two producers take the ring stages alternately: the per-stage cost of one
        // thread (barrier round trip + a few TMA issues) is what bounds thin layers
        const int p = warp == 0 ? 0 : 1;
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int g = 0, issued = 0;
            bool ok = true;
            // (the timeout probe issues nothing: every consumer's wait runs out)
            for (int u = blockIdx.x; u < nunits && ok && !args.timeout_probe; u += gridDim.x) {
                const int img = u / img_units;
                int mu, ni, ki;
                unit_coords(args, u - img * img_units, mu, ni, ki);
                long long r0, r1;
                if (MODE == EPI_POOL) {
                    const int y2 = mu / segs, x0 = (mu - y2 * segs) * 128 * cfg.rt;
                    r0 = (long long)(2 * y2) * tg.pitch + x0;
                    r1 = r0 + tg.pitch;
                } else {
                    r0 = (long long)mu * cfg.rt * 128;
                    r1 = r0 + 64 * nst;
                }
                for (int st = 0; st < kblocks / cfg.kps; st++, g++) {
                    if ((g & 1) == p) {
                        if (!mbar_wait(&sh->empty[s], ph ^ 1u, abort_flag, args.err, budget)) { ok = false; break; }
                        uint8_t *stage = ring + (size_t)s * cfg.stage_bytes;
                        mbar_expect_tx(&sh->full[s], (uint32_t)cfg.kps * (a_bytes + b_bytes));
                        for (int j = 0; j < cfg.kps; j++) {
                            const int kb = ki * kblocks + st * cfg.kps + j;
                            const int tap = kb / kb_per_tap, cb = kb - tap * kb_per_tap;
                            uint8_t *sa = stage + (size_t)j * cfg.sub_bytes;
                            uint8_t *sb = sa + a_bytes;
                            const int off = args.tap_off[tap];
                            tma_load_act(sa, &tmA, cb * BK, (int)(r0 + off), img, batched, &sh->full[s]);
                            tma_load_act(sa + a_bytes / 2, &tmA, cb * BK, (int)(r1 + off), img, batched, &sh->full[s]);
                            for (int h = 0; h < nsub; h++)
                                tma_load_2d(sb + (size_t)h * 256 * BK * 2, &tmB, tap * args.C + cb * BK,
                                            ni * Ns + h * 256, &sh->full[s]);
                        }
                        issued++;
                    }
                    if (++s == cfg.stages) { s = 0; ph ^= 1u; }
                }
            }
            sh->issued[p] = issued;
        }
    } else if (warp <= kMmaWarps) {
        const int m = warp - 1;                    // accumulator m: sub-tile m / nsub, N half m % nsub
        if (lane == 0 && m < nacc) {
            const int i = m / nsub, h = m - i * nsub;
            constexpr uint32_t layout = BK == 64 ? 2u : BK == 32 ? 4u : 6u;
            constexpr uint32_t sbo = 8u * BK * 2u;
            // descriptors are built once; per MMA only the start-address field moves
            const uint64_t desc0 = sdesc(0, sbo, layout);
            const int nh = h == 0 ? (Ns < 256 ? Ns : 256) : Ns - 256;
            const uint32_t idesc = idesc_f16(nh);
            const uint32_t a_off = (uint32_t)(i * 128 * BK * 2), b_off = a_bytes + (uint32_t)(h * 256 * BK * 2);
            int s = 0;
            uint32_t ph = 0;
            int t = 0, consumed = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, t++) {
                const int ab = cfg.acc_bufs == 2 ? (t & 1) : 0;
                const uint32_t aph = (uint32_t)((cfg.acc_bufs == 2 ? (t >> 1) : t) & 1);
                if (!mbar_wait(&sh->tempty[ab], aph ^ 1u, abort_flag, args.err, budget)) break;
                tc_fence_after();
                const uint32_t dcol = tmem_base + (uint32_t)((ab * nst + i) * cfg.acc_cols + h * 256);
                for (int st = 0; st < kblocks / cfg.kps; st++) {
                    if (!mbar_wait(&sh->full[s], ph, abort_flag, args.err, budget)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t stage = smem_u32(ring + (size_t)s * cfg.stage_bytes);
                    for (int j = 0; j < cfg.kps; j++) {
                        const uint32_t sa = stage + (uint32_t)(j * cfg.sub_bytes);
                        const uint64_t ad0 = desc0 | (uint64_t)(((sa + a_off) & 0x3FFFFu) >> 4);
                        const uint64_t bd0 = desc0 | (uint64_t)(((sa + b_off) & 0x3FFFFu) >> 4);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++)
                            mma_f16(dcol, ad0 + (uint64_t)(kk * 2), bd0 + (uint64_t)(kk * 2), idesc,
                                    (st | j | kk) ? 1u : 0u);
                    }
                    mma_commit(&sh->empty[s]);
                    consumed++;
                    if (++s == cfg.stages) { s = 0; ph ^= 1u; }
                }
                if (ok) mma_commit(&sh->tfull[ab]);
            }
            if (m == 0) sh->consumed = consumed;
            if (*abort_flag) {
                // after an abort the issuers stop at different stages: each waits (bounded)
                // for the completion of every MMA it issued before TMEM is freed
                mma_commit(&sh->mdone[m]);
                long long t0 = clock64();
                while (!mbar_try(&sh->mdone[m], 0) && clock64() - t0 < kWaitCycles) {}
            }
        }
    } else {
        const int e = warp - 1 - kMmaWarps;         // epilogue warp 0..7
        const int quad = warp & 3;                  // TMEM lane quadrant this warp may read
        const int part = e >> 2;                    // which half of the column chunks
        const int row = quad * 32 + lane;           // sub-tile row (output position) of this thread
        const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16);
        int t = 0;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, t++) {
            // LayerNorm modes: each set of four warps (one per lane quadrant) takes the units
            // of one accumulator buffer, one whole row per thread
            if (kLnUnits && (cfg.acc_bufs == 2 ? (t & 1) : 0) != part) continue;
            const int img = u / img_units;
            const size_t io = (size_t)img * (size_t)args.img_bytes;
            int mu, ni, ki;
            unit_coords(args, u - img * img_units, mu, ni, ki);
            const int ab = cfg.acc_bufs == 2 ? (t & 1) : 0;
            const uint32_t aph = (uint32_t)((cfg.acc_bufs == 2 ? (t >> 1) : t) & 1);
            bool ok = mbar_wait(&sh->tfull[ab], aph, abort_flag, args.err, budget);
            // the warps sharing this unit leave together (bar.red.or over their threads)
            uint32_t bad;
            if (kLnUnits)
                asm volatile(
                    "{\n\t.reg .pred p, q;\n\t"
                    "setp.eq.u32 p, %1, 0;\n\t"
                    "bar.red.or.pred q, %2, %3, p;\n\t"
                    "selp.u32 %0, 1, 0, q;\n\t}"
                    : "=r"(bad)
                    : "r"((uint32_t)ok), "r"(3 + part), "n"(kEpiWarps / 2 * 32));
            else
                asm volatile(
                    "{\n\t.reg .pred p, q;\n\t"
                    "setp.eq.u32 p, %1, 0;\n\t"
                    "bar.red.or.pred q, 2, %2, p;\n\t"
                    "selp.u32 %0, 1, 0, q;\n\t}"
                    : "=r"(bad)
                    : "r"((uint32_t)ok), "n"(kEpiWarps * 32));
            if (bad) break;
            tc_fence_after();
            const uint32_t acc0 = lane_base + (uint32_t)(ab * nst * cfg.acc_cols);
            if (MODE == EPI_POOL) {
                const int y2 = mu / segs, x0 = (mu - y2 * segs) * 128 * cfg.rt;
                for (int i = 0; i < cfg.rt; i++) {
                    TmemLoader top{acc0 + (uint32_t)(i * cfg.acc_cols)};
                    TmemLoader bot{acc0 + (uint32_t)((cfg.rt + i) * cfg.acc_cols)};
                    epilogue_pool(args.ep, tg, y2, x0 + 128 * i + row, ni * Ns, Ns, top, bot, part, 2, io);
                }
            } else if (kLnUnits) {
                for (int i = 0; i < cfg.rt; i++) {
                    const int tile = mu * cfg.rt + i;
                    if (tile >= tg.ntiles) break;
                    TmemLoader ld{acc0 + (uint32_t)(i * cfg.acc_cols)};
                    epilogue_ln_row<MODE>(args.ep, tg, tile, row, N, ld, io);
                }
            } else {
                for (int i = 0; i < cfg.rt; i++) {
                    const int tile = mu * cfg.rt + i;
                    if (tile >= tg.ntiles) break;
                    TmemLoader ld{acc0 + (uint32_t)(i * cfg.acc_cols)};
                    epilogue_tile<MODE>(args.ep, tg, tile, row, ni * Ns, Ns, N, ki, ld, part, 2, io);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->tempty[ab]);
        }
    }

    __syncthreads();
    if (threadIdx.x == 0) {
        // drain before the CTA's shared memory and TMEM go away: TMA copies issued
        // but never consumed (only after an abort; producer p issued stages p, p+2, ...),
        // then the asynchronous mbarrier arrivals of the last tcgen05.commit (always)
        const int issued_end = max(2 * sh->issued[0], 2 * sh->issued[1] + 1);
        for (int g = sh->consumed; g < issued_end; g++) {
            if (g / 2 >= sh->issued[g & 1]) continue;
            const int s = g % cfg.stages;
            const uint32_t ph = (uint32_t)((g / cfg.stages) & 1);
            long long t0 = clock64();
            while (!mbar_try(&sh->full[s], ph) && clock64() - t0 < kWaitCycles) {}
        }
        if (sh->consumed > 0) {
            int ls = (sh->consumed - 1) % cfg.stages;
            uint32_t lph = (uint32_t)(((sh->consumed - 1) / cfg.stages) & 1);
            long long t0 = clock64();
            while (!mbar_try(&sh->empty[ls], lph) && clock64() - t0 < kWaitCycles) {}
        }
    }
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)cfg.tmem_cols)
                     : "memory");
    }
}

// The driver entry point, looked up once (thread-safe: workers plan concurrently).
PFN_cuTensorMapEncodeTiled_v12000 get_encoder(std::string &err) {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        return (e == cudaSuccess && q == cudaDriverEntryPointSuccess) ? reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f)
                                                                        : nullptr;
    }();
    if (!fn) err = "cuTensorMapEncodeTiled not available";
    return fn;
}

bool encode_2d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint32_t box_inner,
               uint32_t box_outer, int bk, std::string &err) {
    const auto encode = get_encoder(err);
    if (!encode) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    CUtensorMapSwizzle sw = bk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : bk == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                                             : CU_TENSOR_MAP_SWIZZLE_32B;
    CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
        return false;
    }
    return true;
}

template <int BK, int MODE>
int launch_bk_mode(const ConvArgs &a, const TcConfig &cfg, const CUtensorMap &ta, const CUtensorMap &tb, int grid,
                   cudaStream_t st, std::string &err) {
    auto k = tc_conv_kernel<BK, MODE>;
    size_t smem = 1024 + (size_t)cfg.stages * cfg.stage_bytes + sizeof(TcShared);
    if (smem > (size_t)kTcSmemCap) { err = "tc_conv: shared memory plan over the cap"; return -1; }
    // one cap for every layer and thread (the attribute is per kernel): see conv_rw.cu
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemCap);
    if (e != cudaSuccess) { err = std::string("smem attribute: ") + cudaGetErrorString(e); return -1; }
    e = launch_pdl(k, dim3(grid), dim3(kConvThreads), smem, st, ta, tb, a, cfg);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { err = std::string("tc_conv launch: ") + cudaGetErrorString(e); return -1; }
    return 0;
}

template <int BK>
int launch_bk(const ConvArgs &a, int mode, const TcConfig &cfg, const CUtensorMap &ta, const CUtensorMap &tb,
              int grid, cudaStream_t st, std::string &err) {
    switch (mode) {
        case EPI_PLAIN: return launch_bk_mode<BK, EPI_PLAIN>(a, cfg, ta, tb, grid, st, err);
        case EPI_POOL: return launch_bk_mode<BK, EPI_POOL>(a, cfg, ta, tb, grid, st, err);
        case EPI_LN2: return launch_bk_mode<BK, EPI_LN2>(a, cfg, ta, tb, grid, st, err);
        case EPI_RESLN: return launch_bk_mode<BK, EPI_RESLN>(a, cfg, ta, tb, grid, st, err);
        case EPI_PARTIAL: return launch_bk_mode<BK, EPI_PARTIAL>(a, cfg, ta, tb, grid, st, err);
    }
    err = "bad epilogue mode";
    return -1;
}

}  // namespace

int tc_pick_bk(int C) { return C % 64 == 0 ? 64 : C % 32 == 0 ? 32 : C % 16 == 0 ? 16 : 0; }

int fill_bias_consts(ConvArgs &a) {
    if (!a.ep.bias) return 0;
    if (a.N > kMaxBiasConst) return -1;
    return cudaMemcpy(a.ep.bias_c, a.ep.bias, (size_t)a.N * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

// fp16 tensor of `rank` dims (dims[0] contiguous, `swizzle_bytes` = its 32/64/128-byte
// swizzle), strides[i] = byte stride of dims[i + 1]; a box of box[0..rank); out-of-range
// elements of a box read as zero
bool tma_encode(CUtensorMap *m, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                const uint32_t *box, int swizzle_bytes, std::string &err) {
    const auto encode = get_encoder(err);
    if (!encode) return false;
    if (rank < 2 || rank > 5) { err = "tma: rank must be 2..5"; return false; }
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; i++) {
        d[i] = dims[i];
        b[i] = box[i];
        es[i] = 1;
        if (i) st[i - 1] = strides[i - 1];
    }
    const CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                                       : CU_TENSOR_MAP_SWIZZLE_32B;
    CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank, const_cast<void *>(base), d, st, b, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        err = "cuTensorMapEncodeTiled (" + std::to_string(rank) + "d) failed (" + std::to_string((int)r) + ")";
        return false;
    }
    return true;
}

bool tma_encode_act(CUtensorMap *m, const ConvArgs &a, uint32_t box_inner, uint32_t box_rows, std::string &err) {
    // one image: a 2-D map (the kernels issue 2-D loads then: a 3-D box costs more to issue)
    const uint64_t dims[3] = {(uint64_t)a.C, (uint64_t)a.a_rows, (uint64_t)a.nimg};
    const uint64_t strides[2] = {(uint64_t)a.C * 2, img_stride(a, (unsigned long long)a.a_rows * a.C * 2)};
    const uint32_t box[3] = {box_inner, box_rows, 1};
    return tma_encode(m, a.A, a.nimg > 1 ? 3 : 2, dims, strides, box, (int)box_inner * 2, err);
}

bool batch_ok(const ConvArgs &a, std::string &err) {
    if (a.nimg < 1 || a.nimg > 65535) { err = "images per launch must be 1..65535"; return false; }
    if (a.nimg > 1 && (a.img_bytes <= 0 || a.img_bytes % 16 || (unsigned long long)a.img_bytes < (unsigned long long)a.a_rows * a.C * 2)) {
        err = "batched launch: the image stride must be a positive multiple of 16 bytes holding each image's input";
        return false;
    }
    return true;
}

bool tma_encode_2d(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                   uint32_t box_outer, int bk, std::string &err) {
    return encode_2d(m, base, inner, outer, box_inner, box_outer, bk, err);
}

int tc_plan(const ConvArgs &a, int mode, int num_sms, TcConfig &cfg, std::string &err) {
    const int bk = tc_pick_bk(a.C);
    if (!bk) { err = "channels per tap must be a multiple of 16"; return -1; }
    if (a.nsplit < 1 || a.ksplit < 1 || a.N % a.nsplit) { err = "bad N / k split"; return -1; }
    const int Ns = a.N / a.nsplit;
    if (Ns < 16 || Ns > 512 || Ns % 16) { err = "N slice must be a multiple of 16 in [16, 512]"; return -1; }
    if (Ns > 256 && Ns % 256) { err = "N slices above 256 must be a multiple of 256"; return -1; }
    if ((a.ntaps * (a.C / bk)) % a.ksplit) { err = "k split must divide the k-blocks"; return -1; }
    if (a.ntaps < 1 || a.ntaps > 9) { err = "1..9 taps"; return -1; }
    for (int t = 0; t < a.ntaps; t++)
        if (a.tap_off[t] < 0) { err = "negative tap offset"; return -1; }
    if (a.tg.pool && (a.tg.conv_h % 2 || a.tg.conv_w % 2)) { err = "pool needs even conv dims"; return -1; }
    cfg.bk = bk;
    int cols = 32;
    while (cols < Ns) cols <<= 1;
    // Units of several 128-row sub-tiles: one B tile and two TMA boxes feed them all.
    //   plain: up to 4 consecutive tiles;
    //   pool: the two conv rows of a pooled row x 128*rt pixels (2*rt sub-tiles).
    // Each sub-tile is its own accumulator with its own issuing warp (at most 4);
    // both TMEM accumulator buffers must fit in 512 columns, with one wave of units.
    cfg.rt = 1;
    for (int r = 4; r > 1; r >>= 1) {
        const int nst = a.tg.pool ? 2 * r : r;
        if (a.ksplit != 1 || nst > 4 || Ns > 256) continue;
        if (2 * nst * cols <= 512 && (long long)m_units(a.tg, r) * a.nsplit * a.nimg >= num_sms) { cfg.rt = r; break; }
    }
    if (mode == EPI_PLAIN && !a.tg.pool && a.ksplit == 1 && Ns <= 256) {
        // Plain layers: cost ~ waves x (rt A tiles + one B tile) per k-block.  Between one and
        // two waves, two tiles per unit (one wave, each B tile serving both) beat one: measured
        // 21.7 -> 18.7 us on the 128 -> 64 conv at 144 x 200.  A single accumulator buffer
        // only when each CTA has one unit.
        double best = 1e30;
        for (int r = 1; r <= 4; r <<= 1) {
            const long long units = (long long)m_units(a.tg, r) * a.nsplit * a.nimg;
            const int bufs = 2 * r * cols <= 512 ? 2 : 1;
            if (r * cols > 512 || (bufs == 1 && units > num_sms)) continue;
            const double cost = (double)((units + num_sms - 1) / num_sms) * (r * 128.0 + Ns);
            if (cost < 0.97 * best) {
                best = cost;
                cfg.rt = r;
            }
        }
    }
    const int nst = a.tg.pool ? 2 * cfg.rt : cfg.rt;
    cfg.sub_bytes = (128 * nst * bk * 2 + Ns * bk * 2 + 1023) & ~1023;
    // at most ~200 KB per CTA (below the 227 KB limit): one stage more than 176 KB for the
    // 256-wide layers, which measured ~1.5 % faster over the whole enhancement
    const int budget = kTcSmemCap - (int)sizeof(TcShared) - 1024;
    // several k-blocks per stage when they are small (few channels per tap): one
    // barrier round trip and one commit per stage instead of per k-block
    const int kb_unit = a.ntaps * (a.C / bk) / a.ksplit;
    cfg.kps = 1;
    for (int k = 2; k <= 9; k++)
        if (kb_unit % k == 0 && k * cfg.sub_bytes <= 64 * 1024 && budget / (k * cfg.sub_bytes) >= 3) cfg.kps = k;
    cfg.stage_bytes = cfg.kps * cfg.sub_bytes;
    cfg.stages = budget / cfg.stage_bytes;
    if (cfg.stages > kMaxStages) cfg.stages = kMaxStages;
    if (cfg.stages < 2) { err = "shared-memory ring too small"; return -1; }
    cfg.acc_cols = cols;
    cfg.acc_bufs = 2 * nst * cols <= 512 ? 2 : 1;
    cfg.tmem_cols = cols * nst * cfg.acc_bufs;
    if (cfg.tmem_cols > 512) { err = "accumulators exceed TMEM"; return -1; }
    return 0;
}

int tc_conv_launch(const ConvArgs &a, int mode, int num_sms, cudaStream_t st, std::string &err) {
    static const bool flat_only = [] { const char *v = std::getenv("GCDR_CUDA_CONV"); return v && std::string(v) == "flat"; }();
    if (!flat_only || mode == EPI_HEAD) {   // the head epilogue exists only in the row-window kernel
        RwConfig rc;
        if (rw_plan(a, mode, num_sms, rc) == 0) return rw_conv_launch(a, mode, rc, num_sms, st, err);
    }
    if ((mode == EPI_LN2 || mode == EPI_RESLN) && (a.nsplit != 1 || a.N % 32)) {
        err = "LayerNorm layers need whole rows with N % 32 == 0";
        return -1;
    }
    TcConfig cfg;
    if (!batch_ok(a, err) || tc_plan(a, mode, num_sms, cfg, err)) return -1;
    if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15)) {
        err = "operands must be 16-byte aligned";
        return -1;
    }
    CUtensorMap ta, tb;
    const int box_rows = 64 * (a.tg.pool ? 2 * cfg.rt : cfg.rt);
    if (!tma_encode_act(&ta, a, (uint32_t)cfg.bk, (uint32_t)box_rows, err)) return -1;
    const int Ns = a.N / a.nsplit;
    if (!encode_2d(&tb, a.B, (uint64_t)a.C * a.ntaps, (uint64_t)a.N, (uint32_t)cfg.bk, (uint32_t)(Ns < 256 ? Ns : 256),
                   cfg.bk, err))
        return -1;
    const long long units = (long long)m_units(a.tg, cfg.rt) * a.nsplit * a.ksplit * a.nimg;
    if (units > (1ll << 30)) { err = "too many work units"; return -1; }
    int grid = units < num_sms ? (int)units : num_sms;
    static const bool verbose = [] { const char *v = std::getenv("GCDR_CUDA_VERBOSE"); return v && v[0] == '1'; }();
    if (verbose)
        std::fprintf(stderr, "tc_conv mode %d C %d N %d taps %d tiles %d rt %d nsplit %d ksplit %d units %d grid %d | bk %d "
                             "kps %d stages %d stage_bytes %d tmem %d\n",
                     mode, a.C, a.N, a.ntaps, a.tg.ntiles, cfg.rt, a.nsplit, a.ksplit, (int)units, grid, cfg.bk, cfg.kps,
                     cfg.stages, cfg.stage_bytes, cfg.tmem_cols);
    if (grid < 1) return 0;
    switch (cfg.bk) {
        case 64: return launch_bk<64>(a, mode, cfg, ta, tb, grid, st, err);
        case 32: return launch_bk<32>(a, mode, cfg, ta, tb, grid, st, err);
        case 16: return launch_bk<16>(a, mode, cfg, ta, tb, grid, st, err);
    }
    err = "bad k-block";
    return -1;
}

}  // namespace gcdr
