// conv_rw.cu -- row-window tcgen05 convolution for 3x3 stride-1 layers.
//
// The flat implicit GEMM (conv_tc.cu) re-reads the input once per tap: nine
// ring stages per work unit, each a barrier round trip plus TMA issues by one
// thread, which is what bounds the thin layers.  Here a work unit is R output
// rows x 128 pixels of one image window:
//   * each ring stage holds the unit's R + 2 input row segments (136 pixels:
//     the 128 outputs plus the 3x3 halo) for one k-block of channels, loaded
//     once as R + 2 TMA boxes in the layer's swizzled K-major layout;
//   * the nine taps read those segments in place: tap (ky, kx) of output row j
//     starts at segment j + ky, row kx.  tcgen05 applies the shared-memory
//     swizzle on absolute addresses, so a descriptor may start on any row of a
//     swizzled tile (base offset 0);
//   * the weights (9 taps x C/bk k-blocks of N x bk) stay resident in shared
//     memory for the whole persistent CTA.
// Roles: warp 0 (and warp 13) TMA producers taking alternate stages, warps 1..4
// MMA issuers (one accumulator = one output row each; the rows j and j + 4 of
// 8-row pool units), warps 5-12 epilogue
// (bias [+ relu], the 2x2 max-pool + relu of two accumulators, or the head).
// Head units also carry their dec5 window in the ring stage (a third TMA box, read
// by the epilogue), so a head stage is released by the MMA commits and the epilogue
// warps together.
// Every mbarrier wait is bounded; on expiry the CTA raises the abort flag and the
// global error word, drains its copies in flight and its last commit, and frees TMEM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <string>

#include "conv.cuh"
#include "conv_launch.h"
#include "tc_util.cuh"

namespace gcdr {

namespace {

// Warp roles: producer 0 = warp 0, MMA issuers = warps 1..mma, epilogue = the next epi
// warps (a multiple of 4: each TMEM lane quadrant alike, `parts` warps per quadrant),
// producer 1 (when there are two) = the last warp.  The head's epilogue is long and
// latency-bound (one pixel pair per thread and unit), so its CTA trades a producer and an
// MMA warp for four more epilogue warps: 16 warps at the 128 registers a thread may keep.
template <int MODE>
struct RwRoles {
    static constexpr int prod = MODE == EPI_HEAD ? 1 : 2;
    static constexpr int mma = MODE == EPI_HEAD ? 3 : 4;
    static constexpr int epi = MODE == EPI_HEAD ? 12 : 8;
    static constexpr int parts = epi / 4;
    static constexpr int threads = (prod + mma + epi) * 32;
};
constexpr int kSegRows = 136;          // 128 outputs + 2 halo, rounded up to 8 rows
constexpr int kRwSmemCap = 210 * 1024;

struct RwShared {
    uint64_t full[kMaxStages], empty[kMaxStages], tfull[2], tempty[2], bfull, mdone[4];
    uint32_t tmem_base;
    int abort_flag;
    int issued[2], consumed;
    int b_issued;
};

__host__ __device__ inline int round1k(int b) { return (b + 1023) & ~1023; }

// The epilogue warps' store staging buffers (plain and pool): one output row chunk of
// 32 pixels x 32 halves per warp, after the shared block (128-byte aligned).
constexpr int kStgWarpBytes = 32 * 32 * 2;
constexpr int kRwSharedBytes = (int)((sizeof(RwShared) + 127) & ~size_t(127));

// HC: the head's stem channels (16 or 32; a separate instantiation each: one register
// allocation per width), 0 for the other modes.  ROWS: output rows per MMA warp (2 for the
// head and the 8-row pool units; a compile-time bound keeps the issue loop unrolled)
template <int BK, int MODE, int HC, int ROWS>
__global__ void __launch_bounds__(RwRoles<MODE>::threads, 1)
    rw_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ ConvArgs args,
                   const __grid_constant__ RwConfig cfg) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *bres = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = bres + cfg.b_bytes;
    RwShared *sh = reinterpret_cast<RwShared *>(ring + (size_t)cfg.stages * cfg.stage_bytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom &tg = args.tg;
    const int N = args.N, C = args.C, R = cfg.R;
    const int kbs = C / BK;                     // k-blocks (ring stages) per unit
    const int pitch = tg.pitch;
    using Roles = RwRoles<MODE>;
    const int issuers = min(Roles::mma, R);     // MMA warps with rows (each commits once per stage / unit)

    if (threadIdx.x == 0) {
        for (int s = 0; s < cfg.stages; s++) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], (uint32_t)(MODE == EPI_HEAD ? issuers + Roles::epi : issuers));
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&sh->tfull[b], (uint32_t)issuers);
            mbar_init(&sh->tempty[b], Roles::epi);
        }
        mbar_init(&sh->bfull, 1);
        for (int m = 0; m < 4; m++) mbar_init(&sh->mdone[m], 1);
        sh->abort_flag = 0;
        sh->issued[0] = sh->issued[1] = 0;
        sh->consumed = 0;
        sh->b_issued = 0;
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
    const bool b_loader = (warp == 0 && lane == 0);
    if (!b_loader) pdl_wait();              // activations of the previous kernels

    // unit -> (image, first output row, first pixel); pool units cover R conv rows = R/2
    // pooled rows; a batched launch runs the units of image 0, then image 1, ...
    const int nunits = cfg.units * args.nimg;
    const bool batched = args.nimg > 1;          // map ranks: activations 3 (else 2), dec5 4 (else 3)
    auto unit_origin = [&](int u, int &img, int &y0, int &x0) {
        img = u / cfg.units;
        u -= img * cfg.units;
        const int yb = u / cfg.segs_x;
        y0 = yb * R;
        x0 = (u - yb * cfg.segs_x) * 128;
    };

    if (warp == 0 || (Roles::prod == 2 && warp == Roles::mma + Roles::epi + 1)) {
        const int p = warp == 0 ? 0 : 1;
        if (lane == 0) {
            if (p == 0 && !args.timeout_probe) {
                // resident weights: block (kb, tap) = rows [0, N) x columns tap*C + kb*BK
                mbar_expect_tx(&sh->bfull, (uint32_t)(9 * kbs * N * BK * 2));
                for (int kb = 0; kb < kbs; kb++)
                    for (int tap = 0; tap < 9; tap++)
                        tma_load_2d(bres + (size_t)(kb * 9 + tap) * cfg.b_block, &tmB, tap * C + kb * BK, 0, &sh->bfull);
                sh->b_issued = 1;
            }
            if (p == 0) pdl_wait();         // the weights are constant; the activations are not
            int s = 0;
            uint32_t ph = 0;
            int g = 0, issued = 0;
            bool ok = true;
            // (the timeout probe issues nothing: every consumer's wait runs out)
            for (int u = blockIdx.x; u < nunits && ok && !args.timeout_probe; u += gridDim.x) {
                int img, y0, x0;
                unit_origin(u, img, y0, x0);
                for (int kb = 0; kb < kbs; kb++, g++) {
                    if (g % Roles::prod == p) {
                        if (!mbar_wait(&sh->empty[s], ph ^ 1u, abort_flag, args.err, budget)) { ok = false; break; }
                        uint8_t *stage = ring + (size_t)s * cfg.stage_bytes;
                        mbar_expect_tx(&sh->full[s], (uint32_t)((R + 2) * kSegRows * BK * 2 + cfg.win_tx));
                        for (int r = 0; r < R + 2; r++)
                            tma_load_act(stage + (size_t)r * cfg.seg_bytes, &tmA, kb * BK, (y0 + r) * pitch + x0, img,
                                         batched, &sh->full[s]);
                        if (MODE == EPI_HEAD) {   // dec5 rows y0/2 - 1.., columns x0/2 - 1.. (edge: zero fill, never read)
                            uint8_t *win = stage + (size_t)(R + 2) * cfg.seg_bytes;
                            if (batched) tma_load_4d(win, &tmC, 0, x0 / 2 - 1, y0 / 2 - 1, img, &sh->full[s]);
                            else tma_load_3d(win, &tmC, 0, x0 / 2 - 1, y0 / 2 - 1, &sh->full[s]);
                        }
                        issued++;
                    }
                    if (++s == cfg.stages) { s = 0; ph ^= 1u; }
                }
            }
            sh->issued[p] = issued;
        }
    } else if (warp <= Roles::mma) {
        const int j = warp - 1;                    // output rows j, j + mma, ... of the unit (one accumulator each)
        if (lane == 0 && j < R) {
            constexpr uint32_t layout = BK == 64 ? 2u : BK == 32 ? 4u : 6u;
            constexpr uint32_t sbo = 8u * BK * 2u;
            const uint64_t desc0 = sdesc(0, sbo, layout);
            const uint32_t idesc = idesc_f16(N);
            const uint32_t b_s = smem_u32(bres);
            int s = 0;
            uint32_t ph = 0;
            int t = 0, consumed = 0;
            bool ok = mbar_wait(&sh->bfull, 0, abort_flag, args.err, budget);
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, t++) {
                const int ab = cfg.acc_bufs == 2 ? (t & 1) : 0;
                const uint32_t aph = (uint32_t)((cfg.acc_bufs == 2 ? (t >> 1) : t) & 1);
                if (!mbar_wait(&sh->tempty[ab], aph ^ 1u, abort_flag, args.err, budget)) break;
                tc_fence_after();
                const uint32_t dcol0 = tmem_base + (uint32_t)(ab * R * cfg.acc_cols);
                for (int kb = 0; kb < kbs; kb++) {
                    if (!mbar_wait(&sh->full[s], ph, abort_flag, args.err, budget)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t stage = smem_u32(ring + (size_t)s * cfg.stage_bytes);
                    // taps outer, this warp's rows inner (rows j and j + mma when ROWS = 2):
                    // consecutive MMAs go to different accumulators.  The row count is a compile-time
                    // bound, the issue loop stays fully unrolled (it bounds the thin layers).
                    constexpr int kRows = ROWS;
#pragma unroll
                    for (int ky = 0; ky < 3; ky++) {
#pragma unroll
                        for (int kx = 0; kx < 3; kx++) {
                            const uint64_t bd = desc0 | (uint64_t)(((b_s + (uint32_t)((kb * 9 + ky * 3 + kx) * cfg.b_block)) & 0x3FFFFu) >> 4);
#pragma unroll
                            for (int kk = 0; kk < BK / 16; kk++)
#pragma unroll
                                for (int i = 0; i < kRows; i++) {
                                    const int jr = j + i * Roles::mma;
                                    if (kRows > 1 && jr >= R) break;
                                    const uint32_t seg = stage + (uint32_t)((jr + ky) * cfg.seg_bytes);
                                    const uint64_t ad = desc0 | (uint64_t)(((seg + (uint32_t)(kx * BK * 2)) & 0x3FFFFu) >> 4);
                                    mma_f16(dcol0 + (uint32_t)(jr * cfg.acc_cols), ad + (uint64_t)(kk * 2),
                                            bd + (uint64_t)(kk * 2), idesc, (kb | ky | kx | kk) ? 1u : 0u);
                                }
                        }
                    }
                    mma_commit(&sh->empty[s]);
                    consumed++;
                    if (++s == cfg.stages) { s = 0; ph ^= 1u; }
                }
                if (ok) mma_commit(&sh->tfull[ab]);
            }
            if (j == 0) sh->consumed = consumed;
            if (*abort_flag) {
                // after an abort the issuers stop at different stages: each waits (bounded)
                // for the completion of every MMA it issued before TMEM is freed
                mma_commit(&sh->mdone[j]);
                long long t0 = clock64();
                while (!mbar_try(&sh->mdone[j], 0) && clock64() - t0 < kWaitCycles) {}
            }
        }
    } else {
        const int e = warp - 1 - Roles::mma;        // epilogue warp 0..epi-1
        uint8_t *stg = reinterpret_cast<uint8_t *>(sh) + kRwSharedBytes + (size_t)e * kStgWarpBytes;
        const int quad = warp & 3;                  // the TMEM lane quadrant this warp may read
        const int part = e >> 2;                    // 0..parts-1
        const int row = quad * 32 + lane;           // pixel within the unit's 128
        const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16);
        int t = 0;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, t++) {
            int img, y0, x0;
            unit_origin(u, img, y0, x0);
            const size_t io = (size_t)img * (size_t)args.img_bytes;
            const int ab = cfg.acc_bufs == 2 ? (t & 1) : 0;
            const uint32_t aph = (uint32_t)((cfg.acc_bufs == 2 ? (t >> 1) : t) & 1);
            bool ok = mbar_wait(&sh->tfull[ab], aph, abort_flag, args.err, budget);
            uint32_t bad;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.eq.u32 p, %1, 0;\n\t"
                "bar.red.or.pred q, 2, %2, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(bad)
                : "r"((uint32_t)ok), "n"(Roles::epi * 32));
            if (bad) break;
            tc_fence_after();
            const uint32_t acc0 = lane_base + (uint32_t)(ab * R * cfg.acc_cols);
            const int x = x0 + row;
            // work items (output row or pooled row, 32/16-column chunk) taken in turn by the
            // warps of each TMEM lane quadrant
            const int cw = (N % 32 == 0) ? 32 : 16, nch = N / cw;
            if (MODE == EPI_POOL) {
                const int rows2 = min(R / 2, tg.conv_h / 2 - y0 / 2);   // uniform over the CTA
                for (int it = part; it < rows2 * nch; it += Roles::parts) {
                    const int q = it / nch, ch = it - q * nch;
                    TmemLoader top{acc0 + (uint32_t)(2 * q * cfg.acc_cols)};
                    TmemLoader bot{acc0 + (uint32_t)((2 * q + 1) * cfg.acc_cols)};
                    if (cw == 32)
                        epilogue_pool_staged<32>(args.ep, tg, y0 / 2 + q, x - lane, ch * 32, top, bot, stg, io);
                    else
                        epilogue_pool_staged<16>(args.ep, tg, y0 / 2 + q, x - lane, ch * 16, top, bot, stg, io);
                }
            } else if (MODE == EPI_HEAD) {
                // pixel pairs (rows 2q, 2q + 1: one shared dec5 row) taken in turn by the warps;
                // one head unit = one ring stage (C = BK), whose dec5 window the MMA commit left
                // in place: the full barrier's phase has completed (wait for visibility only)
                const int hs = t % cfg.stages;
                const uint8_t *win = ring + (size_t)hs * cfg.stage_bytes + (size_t)(R + 2) * cfg.seg_bytes;
                // (after an abort it is skipped: the next unit's vote ends all epilogue warps together)
                if (mbar_wait(&sh->full[hs], (uint32_t)((t / cfg.stages) & 1), abort_flag, args.err, budget)) {
                    for (int q = part; q < R / 2; q += Roles::parts) {
                        TmemLoader l0{acc0 + (uint32_t)(2 * q * cfg.acc_cols)};
                        TmemLoader l1{acc0 + (uint32_t)((2 * q + 1) * cfg.acc_cols)};
                        const uint8_t *segs = ring + (size_t)hs * cfg.stage_bytes;
                        epilogue_head_pair<HC>(args.ep, tg, y0 + 2 * q, x, l0, l1, win, y0 / 2 - 1, x0 / 2 - 1,
                                               segs + (size_t)(2 * q + 1) * cfg.seg_bytes,
                                               segs + (size_t)(2 * q + 2) * cfg.seg_bytes, row + 1, io);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh->empty[hs]);    // the window may be overwritten
            } else {
                for (int it = part; it < R * nch; it += Roles::parts) {
                    const int jj = it / nch, ch = it - jj * nch;
                    TmemLoader ld{acc0 + (uint32_t)(jj * cfg.acc_cols)};
                    if (cw == 32)
                        epilogue_plain_staged<32>(args.ep, tg, y0 + jj, x - lane, ch * 32, ld, args.ep.bias_c, stg, io);
                    else
                        epilogue_plain_staged<16>(args.ep, tg, y0 + jj, x - lane, ch * 16, ld, args.ep.bias_c, stg, io);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->tempty[ab]);
        }
    }

    __syncthreads();
    if (threadIdx.x == 0) {
        // drain: unconsumed TMA stages (after an abort only), the weights, the last commit
        // producer p issued the stages g = p, p + prod, ... (issued[p] of them)
        const int issued_end = max(Roles::prod * sh->issued[0], Roles::prod * sh->issued[1] + 1);
        for (int g = sh->consumed; g < issued_end; g++) {
            if (g / Roles::prod >= sh->issued[g % Roles::prod]) continue;
            const int s = g % cfg.stages;
            const uint32_t ph = (uint32_t)((g / cfg.stages) & 1);
            long long t0 = clock64();
            while (!mbar_try(&sh->full[s], ph) && clock64() - t0 < kWaitCycles) {}
        }
        if (sh->b_issued) {
            long long t0 = clock64();
            while (!mbar_try(&sh->bfull, 0) && clock64() - t0 < kWaitCycles) {}
        }
        if (sh->consumed > 0) {
            const int ls = (sh->consumed - 1) % cfg.stages;
            const uint32_t lph = (uint32_t)(((sh->consumed - 1) / cfg.stages) & 1);
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

size_t rw_smem(const RwConfig &cfg) {
    return 1024 + (size_t)cfg.b_bytes + (size_t)cfg.stages * cfg.stage_bytes + kRwSharedBytes + cfg.stg_bytes;
}

template <int BK, int MODE, int HC = 0, int ROWS = 1>
int rw_launch_bk_mode(const ConvArgs &a, const RwConfig &cfg, const CUtensorMap &ta, const CUtensorMap &tb,
                      const CUtensorMap &tc, int grid, cudaStream_t st, std::string &err) {
    auto k = rw_conv_kernel<BK, MODE, HC, ROWS>;
    const size_t smem = rw_smem(cfg);
    // the attribute is per kernel, shared by every layer (and every thread) launching it:
    // always the same cap, never a layer's own size, so concurrent workers cannot lower it
    // under one another's launches
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kRwSmemCap);
    if (e != cudaSuccess) { err = std::string("rw smem attribute: ") + cudaGetErrorString(e); return -1; }
    e = launch_pdl(k, dim3(grid), dim3(RwRoles<MODE>::threads), smem, st, ta, tb, tc, a, cfg);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { err = std::string("rw_conv launch: ") + cudaGetErrorString(e); return -1; }
    return 0;
}

}  // namespace

int rw_plan(const ConvArgs &a, int mode, int num_sms, RwConfig &cfg) {
    if (!a.rw || (mode != EPI_PLAIN && mode != EPI_POOL && mode != EPI_HEAD) || a.nsplit != 1 || a.ksplit != 1)
        return -1;
    if (mode == EPI_HEAD && (a.C != kStemInC || (a.N != 16 && a.N != 32))) return -1;
    if (a.ntaps != 9 || a.N < 16 || a.N > 256 || a.N % 16) return -1;
    // the k-block width orders the sums (taps within a k-block, k-blocks outermost): it is
    // the one-image plan's in a batched launch too, so that each image gets the same bytes;
    // the rows per unit change no sum and are sized for the whole launch
    int bk_fixed = 0;
    if (a.nimg > 1) {
        ConvArgs one = a;
        one.nimg = 1;
        RwConfig c1;
        if (rw_plan(one, mode, num_sms, c1)) return -1;
        bk_fixed = c1.bk;
    }
    const TileGeom &tg = a.tg;
    if (tg.pool && (tg.conv_h % 2 || tg.conv_w % 2)) return -1;
    int cols = 32;
    while (cols < a.N) cols <<= 1;
    const int segs_x = (tg.conv_w + 127) / 128;
    // pool: conv row pairs; head: pixel pairs of rows 2q, 2q + 1
    const int r_min = (tg.pool || mode == EPI_HEAD) ? 2 : 1;
    if (mode == EPI_HEAD && (tg.conv_h % 2 || tg.conv_w % 2)) return -1;
    // (k-block, rows per unit): the most rows that fit TMEM (two buffers), keep >= 3
    // ring stages and still fill the GPU in one wave; narrower k-blocks when the
    // widest leave too few stages.  Weights must stay resident.
    bool found = false;
    // pass 0: R = 4 or 2 (head: 6, 4 or 2: three epilogue warps per lane quadrant, one
    // pixel pair each; pool: 8 first, two rows per MMA warp, when that still leaves eight
    // units per SM: fewer handshakes and halo rows per output row) with a full wave of
    // units (pool: R = 2 always qualifies);
    // pass 1 (small layers): the fewest rows per unit that fit, for the most units
    for (int pass = 0; pass < 2 && !found; pass++) {
        for (int bk = tc_pick_bk(a.C); bk >= 16 && !found; bk >>= 1) {
            if (a.C % bk || (bk_fixed && bk != bk_fixed)) continue;
            if (mode == EPI_HEAD && bk != a.C) continue;   // one ring stage (and dec5 window) per head unit
            const int b_block = round1k(a.N * bk * 2);
            const int b_bytes = 9 * (a.C / bk) * b_block;
            if (b_bytes > 96 * 1024) continue;
            const int seg_bytes = round1k(kSegRows * bk * 2);
            const int stg_bytes = mode == EPI_HEAD ? 0 : RwRoles<EPI_PLAIN>::epi * kStgWarpBytes;
            const int avail = kRwSmemCap - 1024 - b_bytes - kRwSharedBytes - stg_bytes;
            for (int i = 0; i < 3 && !found; i++) {
                // (head R <= 6: two rows per MMA warp at most)
                const int R = mode == EPI_HEAD ? (pass == 0 ? 6 - 2 * i : 2 + 2 * i)
                              : pass == 0 ? (i == 0 ? (mode == EPI_POOL ? 8 : 4) : i == 1 ? 4 : 2) : (r_min << i);
                if (R < r_min || R > (mode == EPI_HEAD ? 6 : mode == EPI_POOL ? 8 : 4)) continue;
                const int units = ((tg.conv_h + R - 1) / R) * segs_x;   // of one image
                const long long all_units = (long long)units * a.nimg;
                // head: the unit's dec5 window (R/2 + 2 rows of kHeadWinCols columns x N channels)
                const int win_tx = mode == EPI_HEAD ? (R / 2 + 2) * kHeadWinCols * a.N * 2 : 0;
                const int stage_bytes = (R + 2) * seg_bytes + round1k(win_tx);
                const int stages = avail / stage_bytes;
                if (2 * R * cols > 512 || stages < 3) continue;
                if (pass == 0 && all_units < num_sms && !(tg.pool && R == 2)) continue;
                // (8-row units: instantiated for 16-channel k-blocks, the stems)
                if (R == 8 && (bk != 16 || (pass == 0 && all_units < 8 * num_sms))) continue;
                cfg.bk = bk;
                cfg.R = R;
                cfg.b_block = b_block;
                cfg.b_bytes = b_bytes;
                cfg.seg_bytes = seg_bytes;
                cfg.segs_x = segs_x;
                cfg.units = units;
                cfg.stage_bytes = stage_bytes;
                cfg.win_tx = win_tx;
                cfg.stg_bytes = stg_bytes;
                cfg.stages = stages > kMaxStages ? kMaxStages : stages;
                found = true;
            }
        }
    }
    if (!found) return -1;
    cfg.acc_cols = cols;
    cfg.acc_bufs = 2;
    cfg.tmem_cols = 32;   // an allocation is a power of two columns
    while (cfg.tmem_cols < cols * cfg.R * 2) cfg.tmem_cols <<= 1;
    return 0;
}

int rw_conv_launch(const ConvArgs &a, int mode, const RwConfig &cfg, int num_sms, cudaStream_t st, std::string &err) {
    if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15)) {
        err = "operands must be 16-byte aligned";
        return -1;
    }
    if (!batch_ok(a, err)) return -1;
    CUtensorMap ta, tb;
    if (!tma_encode_act(&ta, a, (uint32_t)cfg.bk, (uint32_t)kSegRows, err)) return -1;
    if (!tma_encode_2d(&tb, a.B, (uint64_t)a.C * 9, (uint64_t)a.N, (uint32_t)cfg.bk, (uint32_t)a.N, cfg.bk, err))
        return -1;
    CUtensorMap tc = tb;   // the head's dec5 window map (other modes: unused)
    if (mode == EPI_HEAD) {
        const __half *d5 = a.ep.head.dec5;
        if (!d5 || (reinterpret_cast<uintptr_t>(d5) & 15)) { err = "head: dec5 missing or misaligned"; return -1; }
        // [nimg][H/2][W/2][N] fp16: a box of N channels x kHeadWinCols columns x (R/2 + 2) rows
        const uint64_t w2 = (uint64_t)(a.tg.conv_w / 2), h2 = (uint64_t)(a.tg.conv_h / 2);
        const uint64_t dims[4] = {(uint64_t)a.N, w2, h2, (uint64_t)a.nimg};
        const uint64_t strides[3] = {(uint64_t)a.N * 2, (uint64_t)a.N * 2 * w2, img_stride(a, (unsigned long long)a.N * 2 * w2 * h2)};
        const uint32_t box[4] = {(uint32_t)a.N, (uint32_t)kHeadWinCols, (uint32_t)(cfg.R / 2 + 2), 1};
        if (!tma_encode(&tc, d5, a.nimg > 1 ? 4 : 3, dims, strides, box, a.N * 2, err)) return -1;
    }
    const long long all_units = (long long)cfg.units * a.nimg;
    if (all_units > (1ll << 30)) { err = "too many work units"; return -1; }
    const int grid = all_units < num_sms ? (int)all_units : num_sms;
    static const bool verbose = [] { const char *v = std::getenv("GCDR_CUDA_VERBOSE"); return v && v[0] == '1'; }();
    if (verbose)
        std::fprintf(stderr, "rw_conv mode %d C %d N %d H %d W %d | bk %d R %d units %d grid %d stages %d stage_bytes %d "
                             "b_bytes %d tmem %d smem %zu\n",
                     mode, a.C, a.N, a.tg.conv_h, a.tg.conv_w, cfg.bk, cfg.R, cfg.units, grid, cfg.stages,
                     cfg.stage_bytes, cfg.b_bytes, cfg.tmem_cols, rw_smem(cfg));
    if (grid < 1) return 0;
    if (rw_smem(cfg) > (size_t)kRwSmemCap) { err = "rw_conv: shared memory plan over the cap"; return -1; }
    switch (cfg.bk * 8 + mode) {
        case 64 * 8 + EPI_PLAIN: return rw_launch_bk_mode<64, EPI_PLAIN>(a, cfg, ta, tb, tc, grid, st, err);
        case 64 * 8 + EPI_POOL: return rw_launch_bk_mode<64, EPI_POOL>(a, cfg, ta, tb, tc, grid, st, err);
        case 32 * 8 + EPI_PLAIN: return rw_launch_bk_mode<32, EPI_PLAIN>(a, cfg, ta, tb, tc, grid, st, err);
        case 32 * 8 + EPI_POOL: return rw_launch_bk_mode<32, EPI_POOL>(a, cfg, ta, tb, tc, grid, st, err);
        case 16 * 8 + EPI_PLAIN: return rw_launch_bk_mode<16, EPI_PLAIN>(a, cfg, ta, tb, tc, grid, st, err);
        case 16 * 8 + EPI_POOL:
            return cfg.R > 4 ? rw_launch_bk_mode<16, EPI_POOL, 0, 2>(a, cfg, ta, tb, tc, grid, st, err)
                             : rw_launch_bk_mode<16, EPI_POOL>(a, cfg, ta, tb, tc, grid, st, err);
        case 16 * 8 + EPI_HEAD:
            return a.N == 32 ? rw_launch_bk_mode<16, EPI_HEAD, 32, 2>(a, cfg, ta, tb, tc, grid, st, err)
                             : rw_launch_bk_mode<16, EPI_HEAD, 16, 2>(a, cfg, ta, tb, tc, grid, st, err);
    }
    err = "rw_conv: bad k-block / mode";
    return -1;
}

}  // namespace gcdr
