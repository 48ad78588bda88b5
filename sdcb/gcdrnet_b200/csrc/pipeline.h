// pipeline.h -- one CUDA worker: weights on the device, a per-shape arena
// plan, the op sequence of both nets, and a CUDA graph per padded shape.
//
// The structure follows the reference's fused GPU worker
// (Backends/Vulkan/VkPipeline2.cs:21-379): bind to a size (arena grow within a
// budget, re-record on a size change), then per frame upload -> GC -> div6 ->
// DR -> download as one submission.  Here the submission is one CUDA-graph
// launch and the div6 / pixel glue live inside the stem and head kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "host_pool.h"
#include "model.h"

namespace gcdr {

// Device copy of one net's weights in the layouts the kernels read.
struct DevBlock {
    const __half *fc1 = nullptr, *fc2 = nullptr;   // [N][K] (Gemm B transposed)
    const float *fc1_b = nullptr, *fc2_b = nullptr;
    const float *dw_w = nullptr, *dw_b = nullptr;   // [9][C] tap-major, [C]
    const float *n2_g = nullptr, *n2_b = nullptr, *no_g = nullptr, *no_b = nullptr;
    float n2_eps = 1e-5f, no_eps = 1e-5f;
    ShiftSpec sa, sb;
    int C = 0;
};

struct DevNet {
    int cin = 0, c1 = 0, c2 = 0, c3 = 0, c4 = 0, c5 = 0;
    const float *enc1_w = nullptr, *enc1_b = nullptr;   // fp32 ONNX order (stem / head)
    const __half *stem_w16 = nullptr;                   // stem conv over the stem-input layout (pack_stem_conv)
    const __half *enc2 = nullptr, *enc3 = nullptr, *pe3 = nullptr, *pe4 = nullptr, *dec[5] = {};
    const float *enc2_b = nullptr, *enc3_b = nullptr, *pe3_b = nullptr, *pe4_b = nullptr, *dec_b[5] = {};
    const float *pe3n_g = nullptr, *pe3n_b = nullptr, *pe4n_g = nullptr, *pe4n_b = nullptr;
    float pe3n_eps = 1e-5f, pe4n_eps = 1e-5f;
    DevBlock blk[4];
    const float *fin_w = nullptr, *fin_b = nullptr;
    // host copies of the head's constants (passed by value to the head kernel)
    float head_fw[3 * 32] = {}, head_fb[3] = {}, head_b1[32] = {};
};

struct DevWeights {
    int device = 0;
    void *mem = nullptr;
    size_t bytes = 0;
    DevNet gc, dr;
    ~DevWeights();
};

// Uploads both nets (packing conv weights to [N][9*C] fp16).  0 or GCDR_ERR_*.
int upload_weights(const Model &m, int device, std::shared_ptr<DevWeights> &out, std::string &err);

struct NetBufs {
    Act t1, t2, t3, t4, b2o, db1o, db2o, d3, d4;
    __half *y0 = nullptr, *hs = nullptr, *f1 = nullptr, *f2 = nullptr, *dconv = nullptr, *dec5 = nullptr;
};

struct OpInfo {
    std::string name;
    double flops = 0;    // algorithmic FLOPs of one launch
    double bytes = 0;    // algorithmic HBM bytes of one launch (each tensor read/written once)
    int tensor = 0;      // 1: tcgen05 kernel
    int batched = 0;     // 1: one launch covers every image of a batch plan (flops, bytes: all of them)
    int launch = 1;      // 1: a kernel launch (0: a memset node)
};

// Everything that depends on the bound shape (width, height, pixel format, debug mode): the
// shape's own device arena and the buffers planned in it, the op sequence over those buffers
// and its CUDA graph.  A worker keeps up to Worker::kMaxPlans of them, least recently used
// evicted first (the reference caches up to 8 sizes per enhancer, GcdrEnhancer.cs:45-46,
// 128-136), so alternating sizes re-use their graphs instead of re-planning.
// One image's device buffers in a batch plan (the arena holds `nimg` such slices).
struct ImageSlice {
    uint8_t *d_src = nullptr, *d_dst = nullptr;
    int *d_err = nullptr;
};

struct ShapePlan {
    int w = 0, h = 0, fmt = -1, H = 0, W = 0, ph = 0, pw = 0, bpp = 3;
    bool debug = false;
    int nimg = 1;                       // images per launch (a batch plan: each kernel covers them all)
    std::vector<ImageSlice> slices;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0;
    NetBufs gcb, drb;
    float *r = nullptr, *ism = nullptr, *ydbg = nullptr;
    Act si_gc, si_dr;
    float *ws = nullptr;
    uint8_t *d_src = nullptr, *d_dst = nullptr;
    int *d_err = nullptr;
    std::vector<std::function<int(cudaStream_t)>> ops;
    std::vector<OpInfo> info;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    uint64_t last_use = 0;
    void release();   // frees the arena and the graph
};

class Worker {
public:
    Worker(int device, std::shared_ptr<DevWeights> w);
    ~Worker();
    int init(std::string &err);
    int enhance_host(const uint8_t *src, int w, int h, int src_stride, uint8_t *dst, int dst_stride, int fmt);
    int enhance_device(const uint8_t *d_src, int w, int h, uint8_t *d_dst, int fmt, cudaStream_t st);
    // n same-shape images in one CUDA-graph launch: a batch plan holds n image slices (each
    // image's buffers at the same offset in its slice) and each of its kernels covers all n
    // images, one launch per layer.  Host buffers (staged, or by DMA when page-locked); dst[k]
    // may alias src[k] at equal strides.
    int enhance_host_batch(const uint8_t *const *src, int n, int w, int h, int src_stride, uint8_t *const *dst,
                           int dst_stride, int fmt);
    // The same with device-resident tight images, asynchronous on `st` (or the worker's stream).
    int enhance_device_batch(const uint8_t *const *d_src, int n, int w, int h, uint8_t *const *d_dst, int fmt,
                             cudaStream_t st);
    static constexpr int kMaxBatch = 16;
    int debug_intermediates(float *gc_in, float *gc_out, float *dr_in, float *dr_out);
    void set_debug(bool on);
    // device bytes of every cached shape's arena (VkPipeline2.cs:141's DeviceBytes)
    int64_t device_bytes() const;
    int launches() const { return launches_; }
    // graph captures so far (one per new shape), shapes held (bound + cached)
    int captures() const { return captures_; }
    int plans() const { return (int)cache_.size() + (bound_ ? 1 : 0); }
    // whether the worker holds a plan for this image shape (the pool's rent preference)
    bool has_plan(int w, int h, int fmt) const;
    static constexpr int kMaxPlans = 8;                     // GcdrEnhancer.cs:45-46
    // arena bytes over all of a worker's plans: a 4096 x 3072 shape's arena is 2.9 GB (1600 x 1152:
    // 0.43 GB, measured), so the budget holds a few of the largest shapes (of the B200's 180 GB)
    static constexpr size_t kPlanBudget = size_t(12) << 30;
    const std::vector<OpInfo> &op_info() const { return info_; }
    // Runs the bound op sequence `reps` times eagerly with CUDA events around each
    // op; ms[i] = mean duration of op i.
    int profile(int reps, std::vector<double> &ms);
    const std::string &last_error() const { return err_; }
    int device() const { return device_; }
    int inject_device_loss = 0;   // test hook: the next N enhances fail with GCDR_ERR_DEVICE

private:
    int bind(int w, int h, int fmt, int nimg = 1);
    void use_slice(int k);          // points the buffer members at image slice k of the arena
    int build_all_ops();            // the plan's ops: batched launches, per-slice ops for the rest
    void stash();                   // current plan -> cache_
    void restore(ShapePlan &&p);    // cache entry -> current plan
    void release_current();
    int plan_arena();
    int build_ops();
    int run_ops(cudaStream_t st);
    int capture();
    int check_err_flag();
    int fail(int code, const std::string &m);

    int device_;
    std::shared_ptr<DevWeights> weights_;
    cudaStream_t stream_ = nullptr;
    int num_sms_ = 148;
    // bound shape
    int w_ = 0, h_ = 0, fmt_ = -1, H_ = 0, W_ = 0, ph_ = 0, pw_ = 0, bpp_ = 3;
    bool bound_ = false, debug_ = false, use_graph_ = true, simt_stem_ = false;
    // arena
    uint8_t *arena_ = nullptr;
    size_t arena_bytes_ = 0;
    NetBufs gcb_, drb_;
    float *r_ = nullptr, *ism_ = nullptr, *ydbg_ = nullptr;
    Act si_gc_, si_dr_;     // stem inputs [H+2][W+2][16] fp16 (GC: from the image; DR: from the GC head)
    float *ws_ = nullptr;   // split-K partial sums (EPI_PARTIAL), shared by both nets
    size_t ws_floats_ = 0;  // its capacity (planned with the arena)
    uint8_t *d_src_ = nullptr, *d_dst_ = nullptr;
    int *d_err_ = nullptr;
    // pinned staging, copied in kHostBands row bands by the caller and pool_'s helpers: each
    // band's H2D is issued as soon as it is staged; after the graph, the error flag comes back
    // first (flag_ev_), then each band (band_ev_) is copied out as soon as its D2H lands.
    // Two bands measured best at 1600x1152 (one call: 1.82 ms with four bands, 1.67 with two,
    // 1.90 with one; four concurrent callers alike or better)
    static constexpr int kHostBands = 2;
    uint8_t *h_src_ = nullptr, *h_dst_ = nullptr;
    int *h_err_ = nullptr;
    size_t pin_bytes_ = 0;
    std::unique_ptr<HostPool> pool_;
    cudaEvent_t flag_ev_ = nullptr, band_ev_[kHostBands] = {};
    // the host-buffer calls wait by polling their events and yielding the core between polls:
    // as quick as a spin when the host has cores to spare, and no core held when several
    // workers per process and processes per host wait at once
    cudaEvent_t done_ev_ = nullptr;
    int wait_stream();                          // records done_ev_ on the worker's stream, waits
    static cudaError_t wait_event(cudaEvent_t ev);
    // ops and graph
    std::vector<std::function<int(cudaStream_t)>> ops_;
    std::vector<OpInfo> info_;
    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t exec_ = nullptr;
    int launches_ = 0;
    bool plan_debug_ = false;       // debug mode the current plan was built in
    int nimg_ = 1;                  // images per launch of the current plan
    int batch_ = 1;                 // images the batched ops of a build_ops call cover
    std::vector<ImageSlice> slices_;
    std::vector<std::pair<void **, size_t>> layout_;   // buffer member -> offset in a slice
    size_t slice_bytes_ = 0;
    int *h_errs_ = nullptr;                            // pinned: one error word per image slice
    std::vector<ShapePlan> cache_;  // plans not bound right now
    uint64_t tick_ = 0;
    int captures_ = 0;
    bool bias_fail_ = false;
    std::string err_;
};

}  // namespace gcdr
