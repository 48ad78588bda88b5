// capi.cpp -- the C ABI (include/gcdr_cuda.h) and the thread-safe enhancer.
//
// gcdr_enhancer_* mirrors src/Sdcb.SimdGcdrNet/GcdrEnhancer.cs: argument
// validation in the same order (:184-192), a bounded rent/return pool of
// stateful workers with an idle-bytes budget (SizePool, :378-432; at most 4
// idle, 3 GB beyond the first idle worker, the Vulkan budget VkPipeline2.cs:137),
// and one retry on a fresh pool when a worker reports device loss (:208-224).
#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../../include/gcdr_cuda.h"
#include "conv_launch.h"
#include "kernels.h"
#include "model.h"
#include "pipeline.h"

using namespace gcdr;

struct gcdr_model {
    Model m;
};

struct gcdr_cuda {
    std::unique_ptr<Worker> w;
    std::string err;
};

namespace {

void put_err(char *err, size_t cap, const std::string &m) {
    if (!err || !cap) return;
    size_t n = m.size() < cap - 1 ? m.size() : cap - 1;
    std::memcpy(err, m.data(), n);
    err[n] = 0;
}

int make_worker(int device, std::shared_ptr<DevWeights> w, std::unique_ptr<Worker> &out, std::string &err) {
    auto wk = std::make_unique<Worker>(device, std::move(w));
    int rc = wk->init(err);
    if (rc) return rc;
    out = std::move(wk);
    return GCDR_OK;
}

}  // namespace

// ------------------------------------------------------------------ models

extern "C" int gcdr_model_load(const void *gc_onnx, size_t gc_len, const void *dr_onnx, size_t dr_len,
                               gcdr_model **out, char *err, size_t err_cap) {
    if (!out) return GCDR_ERR_ARG;
    *out = nullptr;
    if (!gc_onnx || !dr_onnx) { put_err(err, err_cap, "model bytes are null"); return GCDR_ERR_ARG; }
    auto m = std::make_unique<gcdr_model>();
    std::string e;
    int rc = parse_gcdr_net(static_cast<const uint8_t *>(gc_onnx), gc_len, m->m.gc, e);
    if (rc) { put_err(err, err_cap, "GC-Net: " + e); return rc; }
    rc = parse_gcdr_net(static_cast<const uint8_t *>(dr_onnx), dr_len, m->m.dr, e);
    if (rc) { put_err(err, err_cap, "DR-Net: " + e); return rc; }
    if (m->m.gc.cin != 3 || m->m.dr.cin != 6) {
        put_err(err, err_cap, "GC-Net must take 3 channels and DR-Net 6");
        return GCDR_ERR_UNSUPPORTED;
    }
    *out = m.release();
    return GCDR_OK;
}

extern "C" void gcdr_model_free(gcdr_model *m) { delete m; }

extern "C" size_t gcdr_model_describe(const gcdr_model *m, char *buf, size_t cap) {
    if (!m) return 0;
    std::string s = "{\"gc\":" + describe_net(m->m.gc) + ",\"dr\":" + describe_net(m->m.dr) + "}";
    if (buf && cap) put_err(buf, cap, s);
    return s.size();
}

// ------------------------------------------------------------------ worker

extern "C" int gcdr_cuda_create(int device, const gcdr_model *m, int precision, gcdr_cuda **out) {
    if (!out || !m) return GCDR_ERR_ARG;
    *out = nullptr;
    if (precision != GCDR_PRECISION_FP16) return GCDR_ERR_UNSUPPORTED;
    std::shared_ptr<DevWeights> w;
    std::string e;
    int rc = upload_weights(m->m, device, w, e);
    if (rc) return rc;
    auto h = std::make_unique<gcdr_cuda>();
    rc = make_worker(device, w, h->w, e);
    if (rc) return rc;
    *out = h.release();
    return GCDR_OK;
}

extern "C" int gcdr_cuda_create_from_onnx(int device, const void *gc_onnx, size_t gc_len, const void *dr_onnx,
                                          size_t dr_len, int precision, gcdr_cuda **out) {
    gcdr_model *m = nullptr;
    int rc = gcdr_model_load(gc_onnx, gc_len, dr_onnx, dr_len, &m, nullptr, 0);
    if (rc) return rc;
    rc = gcdr_cuda_create(device, m, precision, out);
    gcdr_model_free(m);
    return rc;
}

static int check_image_args(int width, int height, int fmt) {
    if (fmt < 0 || fmt > 3) return GCDR_ERR_RANGE;
    if (width < 1 || height < 1) return GCDR_ERR_RANGE;
    return GCDR_OK;
}

extern "C" int gcdr_cuda_enhance(gcdr_cuda *w, const uint8_t *src, int width, int height, int src_stride,
                                 uint8_t *dst, int dst_stride, int pixel_format) {
    if (!w || !src || !dst) return GCDR_ERR_ARG;
    int rc = check_image_args(width, height, pixel_format);
    if (rc) return rc;
    const int bpp = pixel_format >= 2 ? 4 : 3;
    if (src_stride < width * bpp || dst_stride < width * bpp) return GCDR_ERR_RANGE;
    return w->w->enhance_host(src, width, height, src_stride, dst, dst_stride, pixel_format);
}

extern "C" int gcdr_cuda_enhance_device(gcdr_cuda *w, const uint8_t *d_src, int width, int height, uint8_t *d_dst,
                                        int pixel_format, void *stream) {
    if (!w || !d_src || !d_dst) return GCDR_ERR_ARG;
    int rc = check_image_args(width, height, pixel_format);
    if (rc) return rc;
    return w->w->enhance_device(d_src, width, height, d_dst, pixel_format, static_cast<cudaStream_t>(stream));
}

extern "C" int gcdr_cuda_enhance_batch(gcdr_cuda *w, const uint8_t *const *src, int n, int width, int height,
                                       int src_stride, uint8_t *const *dst, int dst_stride, int pixel_format) {
    if (!w || !src || !dst || n < 1 || n > Worker::kMaxBatch) return GCDR_ERR_ARG;
    for (int k = 0; k < n; k++)
        if (!src[k] || !dst[k]) return GCDR_ERR_ARG;
    int rc = check_image_args(width, height, pixel_format);
    if (rc) return rc;
    const int bpp = pixel_format >= 2 ? 4 : 3;
    if (src_stride < width * bpp || dst_stride < width * bpp) return GCDR_ERR_RANGE;
    return w->w->enhance_host_batch(src, n, width, height, src_stride, dst, dst_stride, pixel_format);
}

extern "C" int gcdr_cuda_enhance_batch_device(gcdr_cuda *w, const uint8_t *const *d_src, int n, int width, int height,
                                              uint8_t *const *d_dst, int pixel_format, void *stream) {
    if (!w || !d_src || !d_dst || n < 1 || n > Worker::kMaxBatch) return GCDR_ERR_ARG;
    for (int k = 0; k < n; k++)
        if (!d_src[k] || !d_dst[k]) return GCDR_ERR_ARG;
    int rc = check_image_args(width, height, pixel_format);
    if (rc) return rc;
    return w->w->enhance_device_batch(d_src, n, width, height, d_dst, pixel_format, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t gcdr_cuda_device_bytes(const gcdr_cuda *w) { return w ? w->w->device_bytes() : 0; }

extern "C" int gcdr_cuda_debug_intermediates(gcdr_cuda *w, float *gc_in, float *gc_out, float *dr_in) {
    if (!w) return GCDR_ERR_ARG;
    return w->w->debug_intermediates(gc_in, gc_out, dr_in, nullptr);
}

extern "C" int gcdr_cuda_debug_output(gcdr_cuda *w, float *dr_out) {
    if (!w) return GCDR_ERR_ARG;
    return w->w->debug_intermediates(nullptr, nullptr, nullptr, dr_out);
}

extern "C" int gcdr_cuda_set_debug(gcdr_cuda *w, int on) {
    if (!w) return GCDR_ERR_ARG;
    w->w->set_debug(on != 0);
    return GCDR_OK;
}

extern "C" int gcdr_cuda_launch_count(const gcdr_cuda *w) { return w ? w->w->launches() : 0; }

extern "C" int gcdr_cuda_plan_stats(const gcdr_cuda *w, int *captures, int *plans) {
    if (!w) return GCDR_ERR_ARG;
    if (captures) *captures = w->w->captures();
    if (plans) *plans = w->w->plans();
    return GCDR_OK;
}

extern "C" int gcdr_cuda_profile(gcdr_cuda *w, int reps, gcdr_op_profile *out, int cap) {
    if (!w || reps < 1) return -GCDR_ERR_ARG;
    std::vector<double> ms;
    int rc = w->w->profile(reps, ms);
    if (rc) return -rc;
    const auto &info = w->w->op_info();
    for (int i = 0; i < (int)info.size() && i < cap && out; i++) {
        std::memset(out[i].name, 0, sizeof(out[i].name));
        std::strncpy(out[i].name, info[i].name.c_str(), sizeof(out[i].name) - 1);
        out[i].ms = ms[i];
        out[i].flops = info[i].flops;
        out[i].bytes = info[i].bytes;
        out[i].tensor_core = info[i].tensor;
    }
    return (int)info.size();
}

extern "C" const char *gcdr_cuda_last_error(const gcdr_cuda *w) { return w ? w->w->last_error().c_str() : "null worker"; }

extern "C" void gcdr_cuda_destroy(gcdr_cuda *w) { delete w; }

// ---------------------------------------------------------------- enhancer

// One Enhance call waiting to be run, possibly in another caller's batch.
struct PendingEnhance {
    const uint8_t *src = nullptr;
    uint8_t *dst = nullptr;
    bool done = false;
    int rc = GCDR_OK;
    std::string msg;
};

// Concurrent Enhance calls of one shape, format and stride pair.
struct EnhanceLane {
    std::deque<PendingEnhance *> queue;   // oldest first
    int running = 0;                      // batches of this lane on the GPU now
};

struct gcdr_enhancer {
    int device = 0;
    Model model;
    std::shared_ptr<DevWeights> weights;
    std::mutex mu;
    std::deque<std::unique_ptr<Worker>> idle;
    int64_t idle_bytes = 0;
    uint64_t generation = 0;   // bumped when a pool is dropped after device loss
    std::atomic<int64_t> pools{0}, workers{0}, evicted{0};
    std::atomic<int> inject{0};
    static constexpr int kMaxIdle = 4;                 // GcdrEnhancer.cs:45 MaxPerSize
    // device bytes of the idle workers beyond the first (VkPipeline2.cs:137-138 keeps 3 GB for
    // one arena; here a worker holds several shape plans, Worker::kPlanBudget each at most)
    static constexpr int64_t kIdleBudget = 32LL << 30;

    // Opportunistic batching of concurrent Enhance calls: a call joins its lane's queue; when
    // the lane has no batch on the GPU, or a full batch is queued and fewer than max_running
    // run, a waiting caller takes the oldest queued calls -- a power of two of them, at most
    // max_batch, so that a worker holds at most four batch plans per shape -- and runs them as
    // one batch-plan launch on a rented worker for everyone; the other callers sleep until
    // their call is done.  A lone call runs at once, alone.  Each image gets the bytes a
    // single-image plan gives it.
    std::mutex bmu;
    std::condition_variable bcv;
    std::map<std::tuple<int, int, int, int, int>, EnhanceLane> lanes;   // (w, h, fmt, src, dst stride)
    int max_batch = 8, max_running = 3;
    std::atomic<int64_t> calls{0}, launches{0};

    // An idle worker, preferring one that holds a plan (arena + graph) for this image shape,
    // else a new one.
    int rent(std::unique_ptr<Worker> &w, uint64_t &gen, std::string &err, int width, int height, int fmt) {
        {
            std::lock_guard<std::mutex> g(mu);
            gen = generation;
            if (!weights) {
                int rc = upload_weights(model, device, weights, err);
                if (rc) return rc;
                pools++;
            }
            if (!idle.empty()) {
                auto it = idle.begin();
                for (auto j = idle.begin(); j != idle.end(); ++j)
                    if ((*j)->has_plan(width, height, fmt)) { it = j; break; }
                w = std::move(*it);
                idle.erase(it);
                idle_bytes -= w->device_bytes();
                return GCDR_OK;
            }
        }
        int rc = make_worker(device, weights, w, err);
        if (rc) return rc;
        workers++;
        return GCDR_OK;
    }

    void give_back(std::unique_ptr<Worker> w, uint64_t gen) {
        std::lock_guard<std::mutex> g(mu);
        if (gen != generation) return;   // its pool was dropped: dispose
        const int64_t b = w->device_bytes();
        if ((int)idle.size() < kMaxIdle && (idle.empty() || idle_bytes + b <= kIdleBudget)) {
            idle_bytes += b;
            idle.push_back(std::move(w));
        }
    }

    void drop_pool() {
        std::lock_guard<std::mutex> g(mu);
        idle.clear();
        idle_bytes = 0;
        generation++;
        weights.reset();
        evicted++;
    }
};

extern "C" int gcdr_enhancer_create(int device, const void *gc_onnx, size_t gc_len, const void *dr_onnx, size_t dr_len,
                                    int precision, gcdr_enhancer **out, char *err, size_t err_cap) {
    if (!out) return GCDR_ERR_ARG;
    *out = nullptr;
    if (precision != GCDR_PRECISION_FP16) { put_err(err, err_cap, "unsupported precision"); return GCDR_ERR_UNSUPPORTED; }
    gcdr_model *m = nullptr;
    int rc = gcdr_model_load(gc_onnx, gc_len, dr_onnx, dr_len, &m, err, err_cap);
    if (rc) return rc;
    auto e = std::make_unique<gcdr_enhancer>();
    e->device = device;
    e->model = std::move(m->m);
    gcdr_model_free(m);
    *out = e.release();
    return GCDR_OK;
}

// GcdrEnhancer.cs:184-192's argument checks, in the same order (one image's buffers).
static int check_enhance_args(const uint8_t *src, size_t src_len, int width, int height, int src_stride,
                              const uint8_t *dst, size_t dst_len, int dst_stride, int pixel_format, char *err,
                              size_t err_cap) {
    if (pixel_format < 0 || pixel_format > 3) { put_err(err, err_cap, "unknown pixel format"); return GCDR_ERR_RANGE; }
    const int bpp = pixel_format >= 2 ? 4 : 3;
    if (width < 1) { put_err(err, err_cap, "width must be >= 1"); return GCDR_ERR_RANGE; }
    if (height < 1) { put_err(err, err_cap, "height must be >= 1"); return GCDR_ERR_RANGE; }
    if (src_stride < width * bpp) { put_err(err, err_cap, "srcStride < width * bytes per pixel"); return GCDR_ERR_RANGE; }
    if (dst_stride < width * bpp) { put_err(err, err_cap, "dstStride < width * bytes per pixel"); return GCDR_ERR_RANGE; }
    if (!src || (long long)src_len < (long long)(height - 1) * src_stride + (long long)width * bpp) {
        put_err(err, err_cap, "src holds " + std::to_string(src_len) + " bytes, " + std::to_string(height) +
                                  " rows of stride " + std::to_string(src_stride) + " need more.");
        return GCDR_ERR_ARG;
    }
    if (!dst || (long long)dst_len < (long long)(height - 1) * dst_stride + (long long)width * bpp) {
        put_err(err, err_cap, "dst holds " + std::to_string(dst_len) + " bytes, " + std::to_string(height) +
                                  " rows of stride " + std::to_string(dst_stride) + " need more.");
        return GCDR_ERR_ARG;
    }
    return GCDR_OK;
}

// Rents a worker for the shape, runs `run` on it, and on a device error drops the pool and
// retries once on a fresh one (GcdrEnhancer's SizePool recovery).  msg: the error text.
template <class F>
static int with_worker(gcdr_enhancer *e, int width, int height, int pixel_format, std::string &msg, F &&run) {
    for (int attempt = 0;; attempt++) {
        std::unique_ptr<Worker> w;
        uint64_t gen = 0;
        int rc = e->rent(w, gen, msg, width, height, pixel_format);
        if (rc) return rc;
        if (e->inject.load() > 0 && e->inject.fetch_sub(1) > 0) w->inject_device_loss = 1;
        rc = run(*w);
        if (rc == GCDR_OK) {
            e->give_back(std::move(w), gen);
            return GCDR_OK;
        }
        msg = w->last_error();
        if (rc == GCDR_ERR_DEVICE && attempt == 0) {
            // the pool's workers are considered dead: drop them and retry once on a fresh pool
            w.reset();
            e->drop_pool();
            continue;
        }
        e->give_back(std::move(w), gen);
        return rc;
    }
}

// Runs one Enhance call through its lane (see gcdr_enhancer::lanes).
static int enhance_coalesced(gcdr_enhancer *e, const uint8_t *src, uint8_t *dst, int width, int height, int src_stride,
                             int dst_stride, int fmt, std::string &msg) {
    e->calls++;
    PendingEnhance me;
    me.src = src;
    me.dst = dst;
    std::unique_lock<std::mutex> lk(e->bmu);
    const auto key = std::make_tuple(width, height, fmt, src_stride, dst_stride);
    EnhanceLane &lane = e->lanes[key];
    lane.queue.push_back(&me);
    for (;;) {
        if (me.done) {
            msg = std::move(me.msg);
            return me.rc;
        }
        // a batch starts when the lane has none on the GPU (a lone call waits for nobody), or
        // when a full batch is queued and fewer than max_running run: under load the calls
        // gather into full batches behind the running ones instead of trickling out in small ones
        const bool start = !lane.queue.empty() && lane.running < e->max_running &&
                           (lane.running == 0 || (int)lane.queue.size() >= e->max_batch);
        if (start) {
            size_t n = 1;
            const size_t cap = std::min(lane.queue.size(), (size_t)std::max(e->max_batch, 1));
            while (n * 2 <= cap) n *= 2;
            std::vector<PendingEnhance *> batch(lane.queue.begin(), lane.queue.begin() + (long)n);
            lane.queue.erase(lane.queue.begin(), lane.queue.begin() + (long)n);
            lane.running++;
            lk.unlock();
            std::vector<const uint8_t *> srcs(n);
            std::vector<uint8_t *> dsts(n);
            for (size_t k = 0; k < n; k++) {
                srcs[k] = batch[k]->src;
                dsts[k] = batch[k]->dst;
            }
            std::string bmsg;
            e->launches++;
            const int rc = with_worker(e, width, height, fmt, bmsg, [&](Worker &w) {
                return n == 1 ? w.enhance_host(srcs[0], width, height, src_stride, dsts[0], dst_stride, fmt)
                              : w.enhance_host_batch(srcs.data(), (int)n, width, height, src_stride, dsts.data(),
                                                     dst_stride, fmt);
            });
            lk.lock();
            for (auto *r : batch) {
                r->rc = rc;
                r->msg = bmsg;
                r->done = true;
            }
            lane.running--;
            e->bcv.notify_all();
            continue;
        }
        e->bcv.wait(lk);
    }
}

extern "C" int gcdr_enhancer_enhance(gcdr_enhancer *e, const uint8_t *src, size_t src_len, int width, int height,
                                     int src_stride, uint8_t *dst, size_t dst_len, int dst_stride, int pixel_format,
                                     char *err, size_t err_cap) {
    if (!e) return GCDR_ERR_ARG;
    int rc = check_enhance_args(src, src_len, width, height, src_stride, dst, dst_len, dst_stride, pixel_format, err,
                                err_cap);
    if (rc) return rc;
    std::string msg;
    rc = enhance_coalesced(e, src, dst, width, height, src_stride, dst_stride, pixel_format, msg);
    if (rc) put_err(err, err_cap, msg);
    {
        // a lane nobody waits in any more goes away (shapes come and go)
        std::lock_guard<std::mutex> g(e->bmu);
        auto it = e->lanes.find(std::make_tuple(width, height, pixel_format, src_stride, dst_stride));
        if (it != e->lanes.end() && it->second.queue.empty() && it->second.running == 0) e->lanes.erase(it);
    }
    return rc;
}

extern "C" int gcdr_enhancer_enhance_batch(gcdr_enhancer *e, const uint8_t *const *src, const size_t *src_len, int n,
                                           int width, int height, int src_stride, uint8_t *const *dst,
                                           const size_t *dst_len, int dst_stride, int pixel_format, char *err,
                                           size_t err_cap) {
    if (!e || !src || !dst || !src_len || !dst_len) return GCDR_ERR_ARG;
    if (n < 1 || n > Worker::kMaxBatch) { put_err(err, err_cap, "batch size must be 1..16"); return GCDR_ERR_ARG; }
    for (int k = 0; k < n; k++) {
        int rc = check_enhance_args(src[k], src_len[k], width, height, src_stride, dst[k], dst_len[k], dst_stride,
                                    pixel_format, err, err_cap);
        if (rc) return rc;
    }
    std::string msg;
    const int rc = with_worker(e, width, height, pixel_format, msg, [&](Worker &w) {
        return w.enhance_host_batch(src, n, width, height, src_stride, dst, dst_stride, pixel_format);
    });
    if (rc) put_err(err, err_cap, msg);
    return rc;
}

extern "C" int gcdr_enhancer_set_batching(gcdr_enhancer *e, int max_batch, int max_running) {
    if (!e || max_batch < 1 || max_batch > Worker::kMaxBatch || max_running < 1 || max_running > 64)
        return GCDR_ERR_ARG;
    std::lock_guard<std::mutex> g(e->bmu);
    e->max_batch = max_batch;
    e->max_running = max_running;
    return GCDR_OK;
}

extern "C" void gcdr_enhancer_batch_stats(const gcdr_enhancer *e, int64_t *calls, int64_t *launches) {
    if (!e) return;
    if (calls) *calls = e->calls.load();
    if (launches) *launches = e->launches.load();
}

extern "C" void gcdr_enhancer_pool_stats(const gcdr_enhancer *e, int64_t *pools, int64_t *workers, int64_t *evicted) {
    if (!e) return;
    if (pools) *pools = e->pools.load();
    if (workers) *workers = e->workers.load();
    if (evicted) *evicted = e->evicted.load();
}

extern "C" void gcdr_enhancer_inject_device_loss(gcdr_enhancer *e, int count) {
    if (e) e->inject.store(count);
}

extern "C" void gcdr_enhancer_destroy(gcdr_enhancer *e) { delete e; }

extern "C" int gcdr_host_register(void *p, size_t bytes) {
    if (!p || !bytes) return GCDR_ERR_ARG;
    cudaError_t e = cudaHostRegister(p, bytes, cudaHostRegisterPortable);
    if (e == cudaSuccess) return GCDR_OK;
    std::fprintf(stderr, "gcdr_host_register: %s\n", cudaGetErrorString(e));
    cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? GCDR_ERR_OOM : e == cudaErrorHostMemoryAlreadyRegistered ? GCDR_ERR_ARG
                                                                                                     : GCDR_ERR_DEVICE;
}

extern "C" int gcdr_host_unregister(void *p) {
    if (!p) return GCDR_ERR_ARG;
    cudaError_t e = cudaHostUnregister(p);
    if (e == cudaSuccess) return GCDR_OK;
    cudaGetLastError();
    return e == cudaErrorHostMemoryNotRegistered ? GCDR_ERR_ARG : GCDR_ERR_DEVICE;
}

// ------------------------------------------------------- standalone kernels

extern "C" int gcdr_k_bgr2nhwc(const uint8_t *src, int w, int h, int stride, int fmt, float *x, int ph, int pw,
                               void *stream) {
    if (!src || !x || w < 1 || h < 1 || fmt < 0 || fmt > 3) return GCDR_ERR_ARG;
    return k_bgr2nhwc(src, w, h, stride, fmt, x, ph, pw, static_cast<cudaStream_t>(stream)) ? GCDR_ERR_DEVICE : GCDR_OK;
}

extern "C" int gcdr_k_div6(const float *x, const float *shadow, size_t npx, float *out6, void *stream) {
    if (!x || !shadow || !out6) return GCDR_ERR_ARG;
    return k_div6(x, shadow, npx, out6, static_cast<cudaStream_t>(stream)) ? GCDR_ERR_DEVICE : GCDR_OK;
}

extern "C" int gcdr_k_nhwc2bgr(const float *y, int H, int W, int ph, int pw, uint8_t *dst, int w, int h,
                               int dst_stride, int fmt, const uint8_t *alpha_src, int alpha_stride, void *stream) {
    if (!y || !dst || w < 1 || h < 1 || fmt < 0 || fmt > 3 || (fmt >= 2 && !alpha_src)) return GCDR_ERR_ARG;
    return k_nhwc2bgr(y, H, W, ph, pw, dst, w, h, dst_stride, fmt, alpha_src, alpha_stride,
                      static_cast<cudaStream_t>(stream))
               ? GCDR_ERR_DEVICE
               : GCDR_OK;
}

// Layer-level entry (tests, microbenchmark).
namespace gcdr {

// Layer descriptor -> ConvArgs (also used by the static-workspace entry, noalloc.cu).
int conv_args_from_desc(const gcdr_conv_desc *d, ConvArgs &a, int &mode, std::string &err) {
    if (!d || !d->in || !d->weight || !d->bias || !d->out || d->H < 1 || d->W < 1) { err = "bad descriptor"; return -1; }
    Act in;
    in.p = const_cast<__half *>(static_cast<const __half *>(d->in));
    in.H = d->H;
    in.W = d->W;
    in.C = d->C;
    Act out;
    out.p = static_cast<__half *>(d->out);
    out.C = d->N;
    out.kind = LAY_PLAIN;
    const __half *B = static_cast<const __half *>(d->weight);
    if (d->epilogue < 0 || d->epilogue > 3) { err = "bad epilogue"; return -1; }
    mode = d->epilogue == 1 ? EPI_POOL : d->epilogue == 3 ? EPI_PARTIAL : EPI_PLAIN;
    if (d->kind == 0 || d->kind == 3) {
        in.kind = d->kind == 0 ? LAY_PADREFL : LAY_PADZERO;
        a.ntaps = 9;
        for (int ky = 0; ky < 3; ky++)
            for (int kx = 0; kx < 3; kx++) a.tap_off[ky * 3 + kx] = ky * (in.W + 2) + kx;
        a.tg.pitch = in.W + 2;
        a.tg.conv_h = in.H;
        a.tg.conv_w = in.W;
        a.rw = 1;
        if (mode == EPI_POOL) {
            if (in.H % 2 || in.W % 2) { err = "pool needs even dims"; return -1; }
            a.tg.pool = 1;
            a.tg.ntiles = m_units(a.tg, 1);   // pooled rows x 128-pixel segments
            out.H = in.H / 2;
            out.W = in.W / 2;
        } else {
            a.tg.ntiles = (int)(((long long)in.H * (in.W + 2) + 127) / 128);
            out.H = in.H;
            out.W = in.W;
        }
    } else if (d->kind == 1) {
        if (in.H % 2 || in.W % 2 || mode == EPI_POOL) { err = "stride-2 conv needs even dims and no pool"; return -1; }
        in.kind = LAY_PHASE;
        const int P = (in.W + 2) / 2;
        const long long Pp = in.plane_rows();
        a.ntaps = 9;
        for (int ky = 0; ky < 3; ky++)
            for (int kx = 0; kx < 3; kx++)
                a.tap_off[ky * 3 + kx] = (int)(((ky & 1) * 2 + (kx & 1)) * Pp + (ky >> 1) * P + (kx >> 1));
        a.tg.pitch = P;
        a.tg.conv_h = in.H / 2;
        a.tg.conv_w = in.W / 2;
        a.tg.ntiles = (int)(((long long)a.tg.conv_h * P + 127) / 128);
        out.H = in.H / 2;
        out.W = in.W / 2;
    } else if (d->kind == 2) {
        if (mode == EPI_POOL) { err = "no pool on a 1x1"; return -1; }
        in.kind = LAY_PLAIN;
        a.ntaps = 1;
        a.tg.pitch = in.W;
        a.tg.conv_h = in.H;
        a.tg.conv_w = in.W;
        a.tg.ntiles = (int)(((long long)in.H * in.W + 127) / 128);
        out.H = in.H;
        out.W = in.W;
    } else {
        err = "bad conv kind";
        return -1;
    }
    a.C = d->C;
    a.N = d->N;
    a.A = in.p;
    a.a_rows = in.rows();
    a.B = B;
    a.ep.bias = d->bias;
    a.ep.relu = d->epilogue == 2;
    a.ep.out = out;
    a.nsplit = d->nsplit > 0 ? d->nsplit : 1;
    a.ksplit = d->ksplit > 0 ? d->ksplit : 1;
    if (mode == EPI_PARTIAL) a.ep.partial = static_cast<float *>(d->out);
    else if (a.ksplit != 1) { err = "k splits need the partial-sum epilogue"; return -1; }
    a.wait_cycles = d->wait_cycles > 0 ? d->wait_cycles : 0;
    a.timeout_probe = d->timeout_probe != 0;
    // the epilogues take the bias as kernel parameters; the partial sums add none
    if (mode != EPI_PARTIAL) {
        if (a.N > kMaxBiasConst) { err = "N > 512"; return -1; }
        if (d->bias_host) std::memcpy(a.ep.bias_c, d->bias_host, (size_t)a.N * sizeof(float));
        else if (fill_bias_consts(a)) { err = "bias copy failed"; return -1; }
    }
    return 0;
}

}  // namespace gcdr

namespace {

__global__ void to_layout_kernel(const __half *src, int H, int W, int C, Act dst) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)H * W) return;
    const int y = (int)(i / W), x = (int)(i - (long long)y * W);
    act_store(dst, y, x, 0, src + i * C, C);
}

}  // namespace

namespace {

// One layer error word per device (the kernels' timeout flag of gcdr_k_conv), allocated and
// zeroed on the device's first layer call; gcdr_k_status reads and clears it.
constexpr int kMaxLayerDevices = 64;
std::mutex g_layer_err_mu;
int *g_layer_err[kMaxLayerDevices] = {};

int *layer_err_word(int dev) {
    if (dev < 0 || dev >= kMaxLayerDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_layer_err_mu);
    if (!g_layer_err[dev]) {
        int *p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
            cudaFree(p);
            return nullptr;
        }
        g_layer_err[dev] = p;
    }
    return g_layer_err[dev];
}

}  // namespace

extern "C" int gcdr_k_conv(const gcdr_conv_desc *d, int reference, void *stream) {
    ConvArgs a;
    int mode = 0;
    std::string err;
    if (conv_args_from_desc(d, a, mode, err)) return GCDR_ERR_ARG;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess) return GCDR_ERR_DEVICE;
    int *d_err = layer_err_word(dev);
    if (!d_err) return GCDR_ERR_OOM;
    a.err = d_err;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (reference) {
        if (!d->scratch) return GCDR_ERR_ARG;
        return ref_conv_launch(a, mode, d->scratch, st, err) ? GCDR_ERR_DEVICE : GCDR_OK;
    }
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (tc_conv_launch(a, mode, sms, st, err)) {
        std::fprintf(stderr, "gcdr_k_conv: %s\n", err.c_str());
        return GCDR_ERR_DEVICE;
    }
    return GCDR_OK;
}

extern "C" int gcdr_k_status(void *stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GCDR_ERR_DEVICE;
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return GCDR_ERR_DEVICE;
    int *d_err = layer_err_word(dev);
    if (!d_err) return GCDR_ERR_OOM;
    int h = 0;
    if (cudaMemcpy(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemset(d_err, 0, sizeof(int)) != cudaSuccess)
        return GCDR_ERR_DEVICE;
    return (h & GCDR_ERR_FLAG_TIMEOUT) ? GCDR_ERR_TIMEOUT : h ? GCDR_ERR_DEVICE : GCDR_OK;
}

namespace {

bool act_from(const gcdr_act *g, Act &a) {
    if (!g || !g->p || g->H < 1 || g->W < 1 || g->C < 1 || g->kind < 0 || g->kind > 3) return false;
    a.p = static_cast<__half *>(g->p);
    a.H = g->H;
    a.W = g->W;
    a.C = g->C;
    a.kind = g->kind == 0 ? LAY_PLAIN : g->kind == 1 ? LAY_PADREFL : g->kind == 2 ? LAY_PHASE : LAY_PADZERO;
    return !(a.kind == LAY_PHASE && (a.H % 2 || a.W % 2));
}

ShiftSpec shift_from(const gcdr_shift *s) {
    if (!s) return ShiftSpec{};
    return make_shift(s->ngroups, s->ends, s->offs);
}

bool shift_ok(const gcdr_shift *s, int C) {
    if (!s) return true;
    if (s->ngroups < 0 || s->ngroups > 5) return false;
    int prev = 0;
    for (int g = 0; g < s->ngroups; g++) {
        if (s->ends[g] < prev || s->ends[g] > C) return false;
        prev = s->ends[g];
    }
    return true;
}

}  // namespace

extern "C" int gcdr_k_dw_gelu_shift(const void *in, int H, int W, int C, const float *wt, const float *b,
                                    const gcdr_shift *shift, void *out, void *stream) {
    if (!in || !wt || !b || !out || H < 1 || W < 1 || !shift_ok(shift, C)) return GCDR_ERR_ARG;
    const int rc = dw_gelu_shift_launch(static_cast<const __half *>(in), H, W, C, wt, b, shift_from(shift),
                                        static_cast<__half *>(out), static_cast<cudaStream_t>(stream));
    return rc == -2 ? GCDR_ERR_ARG : rc ? GCDR_ERR_DEVICE : GCDR_OK;
}

extern "C" int gcdr_k_up_add(const void *d, const gcdr_act *skip, const gcdr_act *out, const float *g,
                             const float *b, float eps, const gcdr_shift *shift, void *h, void *stream) {
    UpAddArgs u;
    if (!d || !act_from(skip, u.skip) || !act_from(out, u.out)) return GCDR_ERR_ARG;
    if (u.skip.H != u.out.H || u.skip.W != u.out.W || u.skip.C != u.out.C || u.out.H % 2 || u.out.W % 2)
        return GCDR_ERR_ARG;
    u.d = static_cast<const __half *>(d);
    if (g) {
        if (!b || !h || u.out.kind != LAY_PLAIN || !shift_ok(shift, u.out.C)) return GCDR_ERR_ARG;
        u.tokens = 1;
        u.g = g;
        u.b = b;
        u.eps = eps;
        u.h.p = static_cast<__half *>(h);
        u.h.H = u.out.H;
        u.h.W = u.out.W;
        u.h.C = u.out.C;
        u.h.kind = LAY_PLAIN;
        u.shift = shift_from(shift);
    }
    const int rc = up_add_launch(u, static_cast<cudaStream_t>(stream));
    return rc == -2 ? GCDR_ERR_ARG : rc ? GCDR_ERR_DEVICE : GCDR_OK;
}

extern "C" int gcdr_k_ln_finalize(const float *partial, int ksplit, int H, int W, int N, const float *bias,
                                  const void *res, const float *g1, const float *b1, float eps1,
                                  const float *g2, const float *b2, float eps2, const gcdr_shift *shift,
                                  const gcdr_act *out, void *out2, void *stream) {
    LnFinalizeArgs f;
    if (!partial || !bias || !g1 || !b1 || ksplit < 1 || H < 1 || W < 1 || !act_from(out, f.out)) return GCDR_ERR_ARG;
    if (f.out.H != H || f.out.W != W || f.out.C != N) return GCDR_ERR_ARG;
    f.partial = partial;
    f.ksplit = ksplit;
    f.H = H;
    f.W = W;
    f.N = N;
    f.bias = bias;
    f.res = static_cast<const __half *>(res);
    f.g1 = g1;
    f.b1 = b1;
    f.eps1 = eps1;
    if (g2) {
        if (!b2 || !out2 || !shift_ok(shift, N)) return GCDR_ERR_ARG;
        f.ln2 = 1;
        f.g2 = g2;
        f.b2 = b2;
        f.eps2 = eps2;
        f.shift = shift_from(shift);
        f.out2.p = static_cast<__half *>(out2);
        f.out2.H = H;
        f.out2.W = W;
        f.out2.C = N;
        f.out2.kind = LAY_PLAIN;
    }
    const int rc = ln_finalize_launch(f, static_cast<cudaStream_t>(stream));
    return rc == -2 ? GCDR_ERR_ARG : rc ? GCDR_ERR_DEVICE : GCDR_OK;
}

extern "C" int64_t gcdr_k_conv_scratch(const gcdr_conv_desc *d) {
    ConvArgs a;
    int mode = 0;
    std::string err;
    if (conv_args_from_desc(d, a, mode, err)) return -1;
    return (int64_t)ref_conv_scratch_floats(a);
}

extern "C" int64_t gcdr_k_to_layout(const void *src, int H, int W, int C, int kind, void *dst, void *stream) {
    Act a;
    a.H = H;
    a.W = W;
    a.C = C;
    a.kind = kind == 1 ? LAY_PADREFL : kind == 2 ? LAY_PHASE : kind == 3 ? LAY_PADZERO : -1;
    if (a.kind < 0 || C % 8 || (kind == 2 && (H % 2 || W % 2))) return -1;
    const long long n = a.rows() * C;
    if (!dst) return n;
    a.p = static_cast<__half *>(dst);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(dst, 0, (size_t)n * 2, st) != cudaSuccess) return -1;
    const long long px = (long long)H * W;
    to_layout_kernel<<<(unsigned)((px + 255) / 256), 256, 0, st>>>(static_cast<const __half *>(src), H, W, C, a);
    return cudaGetLastError() == cudaSuccess ? n : -1;
}

extern "C" int gcdr_device_sms(void) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}
