// pipeline.cu -- weights upload, arena planning, the op sequence of GC-Net and
// DR-Net, CUDA-graph capture and the worker's enhance entry points.
#include "pipeline.h"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "../../../include/gcdr_cuda.h"
#include "conv_launch.h"
#include "kernels.h"

namespace gcdr {

// ------------------------------------------------------------------ weights

DevWeights::~DevWeights() {
    if (mem) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        cudaFree(mem);
        cudaSetDevice(prev);
    }
}

// Channel-shift groups (ends, offsets) -> ShiftSpec, with the equal-chunk shortcut.
ShiftSpec make_shift(int ngroups, const int *ends, const int *offs) {
    ShiftSpec o;
    o.ngroups = ngroups < 0 ? 0 : ngroups > 5 ? 5 : ngroups;
    for (int i = 0; i < o.ngroups; i++) {
        o.ends[i] = ends[i];
        o.offs[i] = offs[i];
    }
    // equal ceil-sized chunks (the last one shorter): channel group = c / gs
    if (o.ngroups > 0) {
        const int gs = o.ends[0];
        bool uniform = gs > 0;
        for (int i = 0; i < o.ngroups - 1; i++) uniform = uniform && o.ends[i] == (i + 1) * gs;
        uniform = uniform && o.ends[o.ngroups - 1] > (o.ngroups - 1) * gs && o.ends[o.ngroups - 1] <= o.ngroups * gs;
        o.gs = uniform ? gs : 0;
        for (int i = 0; i < o.ngroups; i++)
            if (o.ends[i] - (i ? o.ends[i - 1] : 0) < 8) o.narrow = 1;
    }
    return o;
}

namespace {

struct Packer {
    std::vector<uint8_t> host;
    struct Fix { size_t off; const void **dst; };
    std::vector<Fix> fixes;
    size_t add(const void *p, size_t n, const void **dst) {
        size_t off = (host.size() + 255) & ~size_t(255);
        host.resize(off + n);
        std::memcpy(host.data() + off, p, n);
        fixes.push_back({off, dst});
        return off;
    }
    void f32(const std::vector<float> &v, const float **dst) {
        add(v.data(), v.size() * 4, reinterpret_cast<const void **>(dst));
    }
    void h16(const std::vector<__half> &v, const __half **dst) {
        add(v.data(), v.size() * 2, reinterpret_cast<const void **>(dst));
    }
};

// Conv weights ONNX [N][C][k][k] -> [N][k*k*C] fp16, k index = (ky*k + kx)*C + c.
std::vector<__half> pack_conv(const ConvW &c) {
    const int K = c.k * c.k * c.cin;
    std::vector<__half> o((size_t)c.cout * K);
    for (int n = 0; n < c.cout; n++)
        for (int ci = 0; ci < c.cin; ci++)
            for (int ky = 0; ky < c.k; ky++)
                for (int kx = 0; kx < c.k; kx++)
                    o[(size_t)n * K + (ky * c.k + kx) * c.cin + ci] =
                        __float2half_rn(c.w[(((size_t)n * c.cin + ci) * c.k + ky) * c.k + kx]);
    return o;
}

// Gemm B [K][N] -> [N][K] fp16.
std::vector<__half> pack_fc(const std::vector<float> &b, int C) {
    std::vector<__half> o((size_t)C * C);
    for (int k = 0; k < C; k++)
        for (int n = 0; n < C; n++) o[(size_t)n * C + k] = __float2half_rn(b[(size_t)k * C + n]);
    return o;
}

ShiftSpec shift_spec(const ShiftW &s) {
    const int n = (int)std::min(s.ends.size(), s.offs.size());
    return make_shift(n, s.ends.data(), s.offs.data());
}

void pack_net(Packer &pk, const NetW &n, DevNet &d) {
    d.cin = n.cin; d.c1 = n.c1; d.c2 = n.c2; d.c3 = n.c3; d.c4 = n.c4; d.c5 = n.c5;
    pk.f32(n.enc[0].w, &d.enc1_w);
    pk.f32(n.enc[0].b, &d.enc1_b);
    {
        std::vector<__half> sw((size_t)n.enc[0].cout * 9 * 16);
        pack_stem_conv(n.enc[0].w.data(), n.enc[0].cout, n.enc[0].cin, sw.data());
        pk.h16(sw, &d.stem_w16);
    }
    pk.h16(pack_conv(n.enc[1]), &d.enc2); pk.f32(n.enc[1].b, &d.enc2_b);
    pk.h16(pack_conv(n.enc[2]), &d.enc3); pk.f32(n.enc[2].b, &d.enc3_b);
    pk.h16(pack_conv(n.pe3), &d.pe3); pk.f32(n.pe3.b, &d.pe3_b);
    pk.h16(pack_conv(n.pe4), &d.pe4); pk.f32(n.pe4.b, &d.pe4_b);
    for (int i = 0; i < 5; i++) { pk.h16(pack_conv(n.dec[i]), &d.dec[i]); pk.f32(n.dec[i].b, &d.dec_b[i]); }
    pk.f32(n.pe3_norm.g, &d.pe3n_g); pk.f32(n.pe3_norm.b, &d.pe3n_b); d.pe3n_eps = n.pe3_norm.eps;
    pk.f32(n.pe4_norm.g, &d.pe4n_g); pk.f32(n.pe4_norm.b, &d.pe4n_b); d.pe4n_eps = n.pe4_norm.eps;
    for (int i = 0; i < 4; i++) {
        const BlockW &b = n.blk[i];
        DevBlock &o = d.blk[i];
        o.C = b.norm2.c;
        pk.h16(pack_fc(b.fc1_w, o.C), &o.fc1); pk.f32(b.fc1_b, &o.fc1_b);
        pk.h16(pack_fc(b.fc2_w, o.C), &o.fc2); pk.f32(b.fc2_b, &o.fc2_b);
        {
            // depthwise weights tap-major [9][C] (ONNX [C][1][3][3])
            std::vector<float> wt((size_t)9 * o.C);
            for (int c = 0; c < o.C; c++)
                for (int tap = 0; tap < 9; tap++) wt[(size_t)tap * o.C + c] = b.dw.w[(size_t)c * 9 + tap];
            pk.f32(wt, &o.dw_w);
        }
        pk.f32(b.dw.b, &o.dw_b);
        pk.f32(b.norm2.g, &o.n2_g); pk.f32(b.norm2.b, &o.n2_b); o.n2_eps = b.norm2.eps;
        pk.f32(b.norm_out.g, &o.no_g); pk.f32(b.norm_out.b, &o.no_b); o.no_eps = b.norm_out.eps;
        o.sa = shift_spec(b.shift_a);
        o.sb = shift_spec(b.shift_b);
    }
    pk.f32(n.fin.w, &d.fin_w);
    pk.f32(n.fin.b, &d.fin_b);
    for (size_t i = 0; i < n.fin.w.size() && i < 3 * 32; i++) d.head_fw[i] = n.fin.w[i];
    for (size_t i = 0; i < n.fin.b.size() && i < 3; i++) d.head_fb[i] = n.fin.b[i];
    for (size_t i = 0; i < n.enc[0].b.size() && i < 32; i++) d.head_b1[i] = n.enc[0].b[i];
}

}  // namespace

int upload_weights(const Model &m, int device, std::shared_ptr<DevWeights> &out, std::string &err) {
    auto dw = std::make_shared<DevWeights>();
    dw->device = device;
    Packer pk;
    pack_net(pk, m.gc, dw->gc);
    pack_net(pk, m.dr, dw->dr);
    if (cudaSetDevice(device) != cudaSuccess) { err = "cudaSetDevice failed"; return GCDR_ERR_DEVICE; }
    if (cudaMalloc(&dw->mem, pk.host.size()) != cudaSuccess) { err = "weights: cudaMalloc failed"; return GCDR_ERR_OOM; }
    dw->bytes = pk.host.size();
    if (cudaMemcpy(dw->mem, pk.host.data(), pk.host.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        err = "weights upload failed";
        return GCDR_ERR_DEVICE;
    }
    for (auto &f : pk.fixes) *f.dst = static_cast<uint8_t *>(dw->mem) + f.off;
    out = dw;
    return GCDR_OK;
}

// ------------------------------------------------------------------- worker

Worker::Worker(int device, std::shared_ptr<DevWeights> w) : device_(device), weights_(std::move(w)) {}

void ShapePlan::release() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (arena) cudaFree(arena);   // waits for the device: no launch of this plan is in flight after it
    exec = nullptr;
    graph = nullptr;
    arena = nullptr;
    arena_bytes = 0;
    ops.clear();
    info.clear();
}

Worker::~Worker() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    release_current();
    for (auto &p : cache_) p.release();
    cache_.clear();
    if (h_src_) cudaFreeHost(h_src_);
    if (h_dst_) cudaFreeHost(h_dst_);
    if (h_err_) cudaFreeHost(h_err_);
    if (h_errs_) cudaFreeHost(h_errs_);
    pool_.reset();
    if (flag_ev_) cudaEventDestroy(flag_ev_);
    if (done_ev_) cudaEventDestroy(done_ev_);
    for (auto &e : band_ev_)
        if (e) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
}

cudaError_t Worker::wait_event(cudaEvent_t ev) {
    for (;;) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e != cudaErrorNotReady) return e;
        std::this_thread::yield();
    }
}

int Worker::wait_stream() {
    cudaError_t e = cudaEventRecord(done_ev_, stream_);
    if (e == cudaSuccess) e = wait_event(done_ev_);
    return (int)e;
}

int Worker::fail(int code, const std::string &m) {
    err_ = m;
    return code;
}

int Worker::init(std::string &err) {
    if (cudaSetDevice(device_) != cudaSuccess) { err = "cudaSetDevice failed"; return GCDR_ERR_DEVICE; }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device_) != cudaSuccess) { err = "no CUDA device"; return GCDR_ERR_DEVICE; }
    if (prop.major != 10) { err = "this backend is built for sm_100a (B200)"; return GCDR_ERR_UNSUPPORTED; }
    num_sms_ = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) { err = "stream"; return GCDR_ERR_DEVICE; }
    if (cudaMallocHost(&h_err_, sizeof(int)) != cudaSuccess) { err = "pinned alloc"; return GCDR_ERR_OOM; }
    const unsigned evf = cudaEventDisableTiming;
    if (cudaEventCreateWithFlags(&flag_ev_, evf) != cudaSuccess) { err = "event"; return GCDR_ERR_DEVICE; }
    for (auto &e : band_ev_)
        if (cudaEventCreateWithFlags(&e, evf) != cudaSuccess) { err = "event"; return GCDR_ERR_DEVICE; }
    if (cudaEventCreateWithFlags(&done_ev_, evf) != cudaSuccess) { err = "event"; return GCDR_ERR_DEVICE; }
    if (cudaMallocHost(&h_errs_, sizeof(int) * kMaxBatch) != cudaSuccess) { err = "pinned alloc"; return GCDR_ERR_OOM; }
    pool_ = std::make_unique<HostPool>(kHostBands - 1, device_);
    const char *g = std::getenv("GCDR_CUDA_GRAPH");
    use_graph_ = !(g && g[0] == '0');
    const char *sv = std::getenv("GCDR_CUDA_STEM");   // "simt": fp32 SIMT stem/head kernels
    simt_stem_ = sv && std::string(sv) == "simt";
    return GCDR_OK;
}

void Worker::set_debug(bool on) {
    debug_ = on;   // the next bind finds or builds a plan in this mode (the heads write the debug planes)
}

int64_t Worker::device_bytes() const {
    int64_t b = (int64_t)arena_bytes_;
    for (const auto &p : cache_) b += (int64_t)p.arena_bytes;
    return b;
}

bool Worker::has_plan(int w, int h, int fmt) const {
    if (bound_ && w == w_ && h == h_ && fmt == fmt_ && plan_debug_ == debug_ && nimg_ == 1) return true;
    for (const auto &p : cache_)
        if (p.w == w && p.h == h && p.fmt == fmt && p.debug == debug_ && p.nimg == 1) return true;
    return false;
}

void Worker::stash() {
    ShapePlan p;
    p.w = w_; p.h = h_; p.fmt = fmt_; p.H = H_; p.W = W_; p.ph = ph_; p.pw = pw_; p.bpp = bpp_;
    p.debug = plan_debug_;
    p.nimg = nimg_;
    p.slices = std::move(slices_);
    p.arena = arena_; p.arena_bytes = arena_bytes_;
    p.gcb = gcb_; p.drb = drb_;
    p.r = r_; p.ism = ism_; p.ydbg = ydbg_;
    p.si_gc = si_gc_; p.si_dr = si_dr_;
    p.ws = ws_;
    p.d_src = d_src_; p.d_dst = d_dst_; p.d_err = d_err_;
    p.ops = std::move(ops_);
    p.info = std::move(info_);
    p.graph = graph_; p.exec = exec_;
    p.launches = launches_;
    p.last_use = tick_;
    cache_.push_back(std::move(p));
    arena_ = nullptr; arena_bytes_ = 0;
    graph_ = nullptr; exec_ = nullptr;
    ops_.clear(); info_.clear();
    slices_.clear();
    bound_ = false;
}

void Worker::restore(ShapePlan &&p) {
    w_ = p.w; h_ = p.h; fmt_ = p.fmt; H_ = p.H; W_ = p.W; ph_ = p.ph; pw_ = p.pw; bpp_ = p.bpp;
    plan_debug_ = p.debug;
    nimg_ = p.nimg;
    slices_ = std::move(p.slices);
    arena_ = p.arena; arena_bytes_ = p.arena_bytes;
    gcb_ = p.gcb; drb_ = p.drb;
    r_ = p.r; ism_ = p.ism; ydbg_ = p.ydbg;
    si_gc_ = p.si_gc; si_dr_ = p.si_dr;
    ws_ = p.ws;
    d_src_ = p.d_src; d_dst_ = p.d_dst; d_err_ = p.d_err;
    ops_ = std::move(p.ops);
    info_ = std::move(p.info);
    graph_ = p.graph; exec_ = p.exec;
    launches_ = p.launches;
    p.arena = nullptr; p.graph = nullptr; p.exec = nullptr;   // owned by the worker now
}

void Worker::release_current() {
    if (exec_) cudaGraphExecDestroy(exec_);
    if (graph_) cudaGraphDestroy(graph_);
    if (arena_) cudaFree(arena_);
    exec_ = nullptr; graph_ = nullptr; arena_ = nullptr; arena_bytes_ = 0;
    ops_.clear(); info_.clear();
    slices_.clear();
    launches_ = 0;
    bound_ = false;
}

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Alloc {
    size_t off = 0;
    std::vector<std::pair<void **, size_t>> items;   // (pointer slot, offset)
    void take(void **slot, size_t bytes) {
        items.push_back({slot, off});
        off = align256(off + bytes);
    }
    void act(Act &a, int H, int W, int C, int kind) {
        a.H = H; a.W = W; a.C = C; a.kind = kind;
        take(reinterpret_cast<void **>(&a.p), a.bytes());
    }
};

void plan_net(Alloc &al, NetBufs &b, const DevNet &n, int H, int W) {
    const int H1 = H / 2, W1 = W / 2, H2 = H / 4, W2 = W / 4, H3 = H / 8, W3 = W / 8;
    const int H4 = H / 16, W4 = W / 16, H5 = H / 32, W5 = W / 32;
    al.act(b.t1, H1, W1, n.c1, LAY_PADREFL);
    al.act(b.t2, H2, W2, n.c2, LAY_PADREFL);
    al.act(b.t3, H3, W3, n.c3, LAY_PHASE);
    al.act(b.t4, H4, W4, n.c4, LAY_PHASE);
    al.act(b.b2o, H5, W5, n.c5, LAY_PADREFL);
    al.act(b.db1o, H4, W4, n.c4, LAY_PADREFL);
    al.act(b.db2o, H3, W3, n.c3, LAY_PADREFL);
    al.act(b.d3, H2, W2, n.c2, LAY_PADREFL);
    al.act(b.d4, H1, W1, n.c1, LAY_PADREFL);
    size_t tok = std::max({(size_t)H4 * W4 * n.c4, (size_t)H5 * W5 * n.c5, (size_t)H3 * W3 * n.c3}) * 2;
    al.take(reinterpret_cast<void **>(&b.y0), tok);
    al.take(reinterpret_cast<void **>(&b.hs), tok);
    al.take(reinterpret_cast<void **>(&b.f1), tok);
    al.take(reinterpret_cast<void **>(&b.f2), tok);
    size_t dc = std::max({(size_t)H5 * W5 * n.c4, (size_t)H4 * W4 * n.c3, (size_t)H3 * W3 * n.c2, (size_t)H2 * W2 * n.c1}) * 2;
    al.take(reinterpret_cast<void **>(&b.dconv), dc);
    al.take(reinterpret_cast<void **>(&b.dec5), (size_t)H1 * W1 * n.c1 * 2);
}

Act plain(__half *p, int H, int W, int C) {
    Act a;
    a.p = p; a.H = H; a.W = W; a.C = C; a.kind = LAY_PLAIN;
    return a;
}

// 3x3 stride-1 conv over a LAY_PADREFL input.
ConvArgs conv_s1(const Act &in, const __half *B, const float *bias, int N, bool pool) {
    ConvArgs a;
    a.ntaps = 9;
    for (int ky = 0; ky < 3; ky++)
        for (int kx = 0; kx < 3; kx++) a.tap_off[ky * 3 + kx] = ky * (in.W + 2) + kx;
    a.C = in.C;
    a.N = N;
    a.A = in.p;
    a.a_rows = in.rows();
    a.B = B;
    a.tg.pitch = in.W + 2;
    a.tg.conv_h = in.H;
    a.tg.conv_w = in.W;
    a.rw = 1;
    if (pool) {
        a.tg.pool = 1;
        a.tg.ntiles = m_units(a.tg, 1);   // pooled rows x 128-pixel segments
    } else {
        a.tg.ntiles = (int)(((long long)in.H * (in.W + 2) + 127) / 128);
    }
    a.ep.bias = bias;
    return a;
}

// 3x3 stride-2 zero-pad-1 conv over a LAY_PHASE input (logical H x W).
ConvArgs conv_s2(const Act &in, const __half *B, const float *bias, int N) {
    ConvArgs a;
    const int Ho = in.H / 2, Wo = in.W / 2, P = (in.W + 2) / 2;
    const long long Pp = in.plane_rows();
    a.ntaps = 9;
    for (int ky = 0; ky < 3; ky++)
        for (int kx = 0; kx < 3; kx++)
            a.tap_off[ky * 3 + kx] = (int)(((ky & 1) * 2 + (kx & 1)) * Pp + (ky >> 1) * P + (kx >> 1));
    a.C = in.C;
    a.N = N;
    a.A = in.p;
    a.a_rows = in.rows();
    a.B = B;
    a.tg.pitch = P;
    a.tg.conv_h = Ho;
    a.tg.conv_w = Wo;
    a.tg.ntiles = (int)(((long long)Ho * P + 127) / 128);
    a.ep.bias = bias;
    return a;
}

// Token Gemm (1 tap) over [H][W][C] tokens.
ConvArgs fc(const __half *in, int H, int W, int C, const __half *B, const float *bias) {
    ConvArgs a;
    a.ntaps = 1;
    a.C = C;
    a.N = C;
    a.A = in;
    a.a_rows = (long long)H * W;
    a.B = B;
    a.tg.pitch = W;
    a.tg.conv_h = H;
    a.tg.conv_w = W;
    a.tg.ntiles = (int)(((long long)H * W + 127) / 128);
    a.ep.bias = bias;
    return a;
}

// How a tensor-core layer is spread over the GPU.  Layers with fewer 128-row
// tiles than SMs get N slices (any mode) and, for the LayerNorm modes, k splits
// whose fp32 partials a token kernel reduces in a fixed order (deterministic).
struct Split {
    int nsplit = 1, ksplit = 1;
};

// The split of a layer with fewer 128-pixel tiles than SMs.
//   Plain layers: N slices only, the most that keep the units within one wave (a
//   slice at least 32 wide).
//   LayerNorm layers: N slices x K ranges, the fp32 partials summed and normalised by
//   ln_finalize, chosen by an estimate fitted to measured layer times on B200
//   (1600x1152, both nets): waves of units, each an MMA chain into one accumulator at
//   ~250 cycles per 16-deep k-step (x1.6 for 512-wide slices: two MMAs per step),
//   ~1000 cycles of fill and its partials stored at ~8 B/cycle; plus the finalize at
//   ~8 us + the partials read back at ~2.5 TB/s.  (The LayerNorm epilogue of the conv
//   itself, on one tile per CTA, measured several times slower than any split.)
Split split_policy(const ConvArgs &a, int mode, int nsm) {
    Split best;
    const long long tiles = (long long)a.tg.ntiles * a.nimg;   // of every image of the launch
    if (tiles >= nsm) return best;
    auto valid_slice = [&](int ns) {
        if (a.N % ns) return false;
        const int Ns = a.N / ns;
        return Ns % 16 == 0 && Ns <= 512 && !(Ns > 256 && Ns % 256);
    };
    if (mode == EPI_PLAIN) {
        for (int ns = 1; ns <= a.N / 32; ns++)
            if (valid_slice(ns) && tiles * ns <= nsm) best.nsplit = ns;
        return best;
    }
    const int bk = tc_pick_bk(a.C);
    if (!bk) return best;
    const int kblocks = a.ntaps * (a.C / bk);
    const double T = (double)a.tg.conv_h * a.tg.conv_w * a.nimg;
    double best_us = 1e30;
    for (int ns = 1; ns <= a.N / 16; ns++) {
        if (!valid_slice(ns)) continue;
        const int Ns = a.N / ns;
        for (int ks = 1; ks <= kblocks; ks++) {
            if (kblocks % ks || (ns == 1 && ks == 1)) continue;
            const long long units = tiles * ns * ks;
            const long long waves = (units + nsm - 1) / nsm;
            const double ksteps = (double)(kblocks / ks) * (bk / 16);
            const double conv = waves * (ksteps * 250.0 * (Ns > 256 ? 1.6 : 1.0) + 1000.0 + 128.0 * Ns * 4 / 8) / 1900.0;
            const double fin = 8.0 + (double)ks * T * a.N * 4 / 2.5e6;
            if (conv + fin < best_us) {
                best_us = conv + fin;
                best.nsplit = ns;
                best.ksplit = ks;
            }
        }
    }
    return best;
}

bool uses_partial(const ConvArgs &a, int mode, int nsm) {
    if (mode != EPI_LN2 && mode != EPI_RESLN) return false;
    static const bool no_split = [] { const char *v = std::getenv("GCDR_CUDA_LN_SPLIT"); return v && v[0] == '0'; }();
    if (no_split) return false;
    // small K with enough tiles: one kernel with the LayerNorm epilogue beats split-K + finalize
    // (measured: 1x1 fc2, K = 160, 57 tiles at 1600x1152)
    if (a.ntaps * a.C <= 192 && (long long)a.tg.ntiles * a.nimg >= 32) return false;
    Split s = split_policy(a, mode, nsm);
    return s.nsplit > 1 || s.ksplit > 1;
}

// fp32 floats of the split-K workspace the LayerNorm layers of one net need per image (the
// split is decided for one image, batched or not).
size_t partial_floats(const DevNet &n, int H, int W, int nsm) {
    const int H3 = H / 8, W3 = W / 8, H4 = H / 16, W4 = W / 16, H5 = H / 32, W5 = W / 32;
    Act t3, t4;
    t3.H = H3; t3.W = W3; t3.C = n.c3; t3.kind = LAY_PHASE;
    t4.H = H4; t4.W = W4; t4.C = n.c4; t4.kind = LAY_PHASE;
    std::vector<std::pair<ConvArgs, int>> layers;
    layers.push_back({conv_s2(t3, nullptr, nullptr, n.c4), EPI_LN2});
    layers.push_back({conv_s2(t4, nullptr, nullptr, n.c5), EPI_LN2});
    layers.push_back({fc(nullptr, H4, W4, n.c4, nullptr, nullptr), EPI_RESLN});
    layers.push_back({fc(nullptr, H5, W5, n.c5, nullptr, nullptr), EPI_RESLN});
    layers.push_back({fc(nullptr, H3, W3, n.c3, nullptr, nullptr), EPI_RESLN});
    size_t need = 0;
    for (auto &l : layers) {
        if (!uses_partial(l.first, l.second, nsm)) continue;
        Split s = split_policy(l.first, l.second, nsm);
        need = std::max(need, (size_t)s.ksplit * l.first.tg.conv_h * l.first.tg.conv_w * l.first.N);
    }
    return need;
}

}  // namespace

int Worker::plan_arena() {
    const DevWeights &w = *weights_;
    Alloc al;
    plan_net(al, gcb_, w.gc, H_, W_);
    plan_net(al, drb_, w.dr, H_, W_);
    al.take(reinterpret_cast<void **>(&r_), simt_stem_ || plan_debug_ ? (size_t)H_ * W_ * 3 * 4 : 256);
    al.act(si_gc_, H_, W_, kStemInC, LAY_PADREFL);
    al.act(si_dr_, H_, W_, kStemInC, LAY_PADREFL);
    al.take(reinterpret_cast<void **>(&ism_), plan_debug_ ? (size_t)H_ * W_ * 3 * 4 : 256);
    al.take(reinterpret_cast<void **>(&ydbg_), plan_debug_ ? (size_t)H_ * W_ * 3 * 4 : 256);
    const size_t img = (size_t)h_ * w_ * bpp_;
    al.take(reinterpret_cast<void **>(&d_src_), img + 16);
    al.take(reinterpret_cast<void **>(&d_dst_), img + 16);
    al.take(reinterpret_cast<void **>(&d_err_), 256);
    const size_t wsf = std::max(partial_floats(w.gc, H_, W_, num_sms_), partial_floats(w.dr, H_, W_, num_sms_));
    ws_floats_ = std::max(wsf, (size_t)64);
    al.take(reinterpret_cast<void **>(&ws_), ws_floats_ * 4);
    // a batch plan holds nimg_ such image slices, one after another
    layout_ = al.items;
    slice_bytes_ = al.off;
    const size_t need = slice_bytes_ * (size_t)nimg_;
    // one arena per shape plan, sized exactly; the plan cache keeps the sum of the cached
    // plans' arenas within kPlanBudget (the reference's arena budget, VkPipeline2.cs:104-117),
    // evicting the least recently used shapes first
    size_t cached = 0;
    for (const auto &p : cache_) cached += p.arena_bytes;
    while (!cache_.empty() && ((int)cache_.size() >= kMaxPlans || cached + need > kPlanBudget)) {
        auto lru = std::min_element(cache_.begin(), cache_.end(),
                                    [](const ShapePlan &a, const ShapePlan &b) { return a.last_use < b.last_use; });
        cached -= lru->arena_bytes;
        lru->release();
        cache_.erase(lru);
    }
    if (cudaMalloc(&arena_, need) != cudaSuccess) {
        cudaGetLastError();
        arena_ = nullptr;
        return fail(GCDR_ERR_OOM, "arena: cudaMalloc failed");
    }
    arena_bytes_ = need;
    slices_.assign(nimg_, ImageSlice{});
    for (int k = 0; k < nimg_; k++) {
        use_slice(k);
        slices_[k] = ImageSlice{d_src_, d_dst_, d_err_};
    }
    use_slice(0);
    // zero borders of the stride-2 inputs (LAY_PHASE) and everything else once per plan
    if (cudaMemsetAsync(arena_, 0, need, stream_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "arena memset failed");
    // pinned staging (grow-only): one image per slice
    const size_t stage = img * (size_t)nimg_;
    if (pin_bytes_ < stage) {
        if (h_src_) cudaFreeHost(h_src_);
        if (h_dst_) cudaFreeHost(h_dst_);
        h_src_ = h_dst_ = nullptr;
        size_t cap = stage + stage / 4 + 64;
        if (cudaMallocHost(&h_src_, cap) != cudaSuccess || cudaMallocHost(&h_dst_, cap) != cudaSuccess) {
            pin_bytes_ = 0;
            return fail(GCDR_ERR_OOM, "pinned staging alloc failed");
        }
        pin_bytes_ = cap;
    }
    return GCDR_OK;
}

void Worker::use_slice(int k) {
    for (auto &it : layout_) *it.first = arena_ + (size_t)k * slice_bytes_ + it.second;
}

int Worker::build_all_ops() {
    // image slice 0's ops with every batched launch covering all nimg_ slices; an op that is
    // not batched (the fp32 SIMT stem / head, the error-word reset of that path) runs once
    // per slice, in slice order, where slice 0's would run
    batch_ = nimg_;
    use_slice(0);
    int rc = build_ops();
    batch_ = 1;
    if (rc || nimg_ == 1) return rc;
    bool all_batched = true;
    for (const auto &oi : info_) all_batched = all_batched && oi.batched;
    if (all_batched) return GCDR_OK;
    std::vector<std::vector<std::function<int(cudaStream_t)>>> per(nimg_);
    std::vector<std::vector<OpInfo>> per_info(nimg_);
    per[0] = std::move(ops_);
    per_info[0] = std::move(info_);
    for (int k = 1; k < nimg_; k++) {
        use_slice(k);
        if ((rc = build_ops())) return rc;
        if (ops_.size() != per[0].size()) return fail(GCDR_ERR_DEVICE, "batch plan: op lists differ between slices");
        per[k] = std::move(ops_);
        per_info[k] = std::move(info_);
    }
    use_slice(0);
    std::vector<std::function<int(cudaStream_t)>> all;
    std::vector<OpInfo> all_info;
    int launches = 0;
    for (size_t i = 0; i < per[0].size(); i++) {
        const int copies = per_info[0][i].batched ? 1 : nimg_;
        for (int k = 0; k < copies; k++) {
            all.push_back(std::move(per[k][i]));
            all_info.push_back(per_info[k][i]);
            launches += per_info[k][i].launch;
        }
    }
    ops_ = std::move(all);
    info_ = std::move(all_info);
    launches_ = launches;
    return GCDR_OK;
}

int Worker::build_ops() {
    bias_fail_ = false;
    ops_.clear();
    launches_ = 0;
    const DevWeights &wt = *weights_;
    const int nsm = num_sms_;
    int *errp = d_err_;
    // batched launches cover batch_ images, image k's buffers slice_bytes_ * k past these
    const int nb = batch_;
    const long long ib = nb > 1 ? (long long)slice_bytes_ : 0;
    auto conv_op = [this, nsm, errp, nb, ib](ConvArgs a, int mode, const std::string &name, double flops_override = -1,
                                              double bytes_override = -1) {
        a.err = errp;
        if (fill_bias_consts(a)) bias_fail_ = true;
        // the direct LayerNorm epilogue's g1 and b1 as kernel parameters, after the bias
        if (mode == EPI_RESLN && a.ep.g1 && a.ep.b1 && 3 * a.N <= kMaxBiasConst) {
            if (cudaMemcpy(a.ep.bias_c + a.N, a.ep.g1, (size_t)a.N * sizeof(float), cudaMemcpyDeviceToHost) !=
                    cudaSuccess ||
                cudaMemcpy(a.ep.bias_c + 2 * a.N, a.ep.b1, (size_t)a.N * sizeof(float), cudaMemcpyDeviceToHost) !=
                    cudaSuccess)
                bias_fail_ = true;
            else
                a.ep.ln_c = 1;
        }
        // split-K and the LayerNorm path fix the order of the sums: decided for one image
        // (a.nimg is 1 here), so that a batch plan gives every image the bytes of a single-
        // image plan; N slices change no sum and are sized for the whole launch
        const bool partial = uses_partial(a, mode, nsm);
        int run_mode = mode;
        if (mode == EPI_PLAIN || partial) {
            if (!partial) a.nimg = nb;
            Split sp = split_policy(a, mode, nsm);
            a.nsplit = sp.nsplit;
            if (partial) {
                a.ksplit = sp.ksplit;
                a.ep.partial = ws_;
                run_mode = EPI_PARTIAL;
            }
        }
        a.nimg = nb;
        a.img_bytes = ib;
        if (partial && (double)a.ksplit * a.tg.conv_h * a.tg.conv_w * a.N > (double)ws_floats_) {
            bias_fail_ = true;   // the workspace must bound every split: a plan error, nothing launches
            return;
        }
        OpInfo oi;
        oi.name = name;
        oi.tensor = 1;
        const double px = (double)a.tg.conv_h * a.tg.conv_w;
        oi.flops = 2.0 * px * a.N * a.ntaps * a.C;
        const double in_px = a.ntaps == 1 ? px : (a.tap_off[1] == 1 ? px : 4.0 * px);   // s2 reads 4x its outputs
        const double out_px = mode == EPI_POOL ? px / 4 : px;
        oi.bytes = in_px * a.C * 2 + (double)a.N * a.ntaps * a.C * 2 +
                   (partial ? 4.0 * px * a.N * a.ksplit
                            : out_px * a.N * 2 * (mode == EPI_LN2 ? 2 : 1) + (mode == EPI_RESLN ? px * a.N * 2 : 0));
        if (flops_override >= 0) oi.flops = flops_override;
        if (bytes_override >= 0) oi.bytes = bytes_override;
        oi.flops *= nb;
        oi.bytes *= nb;
        oi.batched = 1;
        info_.push_back(oi);
        ops_.push_back([a, run_mode, nsm, this](cudaStream_t st) {
            std::string e;
            if (tc_conv_launch(a, run_mode, nsm, st, e)) return fail(GCDR_ERR_DEVICE, e);
            return 0;
        });
        launches_++;
        if (partial) {
            LnFinalizeArgs f;
            f.partial = ws_;
            f.ksplit = a.ksplit;
            f.H = a.tg.conv_h;
            f.W = a.tg.conv_w;
            f.N = a.N;
            f.bias = a.ep.bias;
            f.res = mode == EPI_RESLN ? a.ep.res : nullptr;
            f.g1 = a.ep.g1; f.b1 = a.ep.b1; f.eps1 = a.ep.eps1;
            f.ln2 = mode == EPI_LN2;
            f.g2 = a.ep.g2; f.b2 = a.ep.b2; f.eps2 = a.ep.eps2;
            f.shift = a.ep.shift;
            f.out = a.ep.out;
            f.out2 = a.ep.out2;
            f.nimg = nb;
            f.img_bytes = ib;
            ops_.push_back([f, this](cudaStream_t st) {
                return ln_finalize_launch(f, st) ? fail(GCDR_ERR_DEVICE, std::string("ln_finalize launch: ") + last_launch_error()) : 0;
            });
            launches_++;
            info_.push_back(OpInfo{name + ".ln", 0,
                                   nb * (4.0 * px * a.N * a.ksplit + 2.0 * px * a.N * (f.ln2 ? 2 : 1) + (f.res ? 2.0 * px * a.N : 0)),
                                   0, 1});
        }
    };
    info_.clear();
    if (simt_stem_) {
        // the first kernel of the tensor-core path (stem_in) clears the device error word itself
        ops_.push_back([errp](cudaStream_t st) { return cudaMemsetAsync(errp, 0, sizeof(int), st) == cudaSuccess ? 0 : GCDR_ERR_DEVICE; });
        info_.push_back(OpInfo{"reset_error_flag", 0, 4, 0, 0, 0});
    }
    // a SIMT op's metadata: batched ops cover nb images, the others (the fp32 stem / head) one
    auto simt = [this, nb](const std::string &name, double flops, double bytes, bool batched = true) {
        const int k = batched ? nb : 1;
        info_.push_back(OpInfo{name, flops * k, bytes * k, 0, batched ? 1 : 0});
    };

    ImgSpec img;
    img.src = d_src_;
    img.w = w_;
    img.h = h_;
    img.stride = w_ * bpp_;
    img.bpp = bpp_;
    img.swap = (fmt_ == GCDR_RGB24 || fmt_ == GCDR_RGBA32) ? 1 : 0;
    img.ph = ph_;
    img.pw = pw_;

    for (int which = 0; which < 2; which++) {
        const DevNet &n = which ? wt.dr : wt.gc;
        NetBufs &b = which ? drb_ : gcb_;
        const int H1 = H_ / 2, W1 = W_ / 2, H2 = H_ / 4, W2 = W_ / 4, H3 = H_ / 8, W3 = W_ / 8;
        const int H4 = H_ / 16, W4 = W_ / 16, H5 = H_ / 32, W5 = W_ / 32;
        (void)H1; (void)W1; (void)H2; (void)W2;
        // stem: enc1 conv + pool + relu
        const std::string pre = which ? "dr." : "gc.";
        const double stem_flops = 2.0 * H_ * W_ * n.c1 * 9 * n.cin;
        const double stem_bytes = (double)h_ * w_ * bpp_ + (which ? 12.0 * H_ * W_ : 0) + (double)H1 * W1 * n.c1 * 2;
        if (simt_stem_) {
            StemArgs sa;
            sa.img = img;
            sa.r = which ? r_ : nullptr;
            sa.H = H_; sa.W = W_; sa.cin = n.cin; sa.c1 = n.c1;
            sa.w = n.enc1_w; sa.b = n.enc1_b; sa.out = b.t1;
            ops_.push_back([sa, this](cudaStream_t st) { return stem_launch(sa, st) ? fail(GCDR_ERR_DEVICE, std::string("stem launch: ") + last_launch_error()) : 0; });
            launches_++;
            simt(pre + "stem", stem_flops, stem_bytes, false);
        } else {
            // the stem as a tensor-core conv over the stem input (GC: built from the image here;
            // DR: written by the GC head)
            if (!which) {
                const Act si = si_gc_;
                ops_.push_back([img, si, errp, nb, ib, this](cudaStream_t st) {
                    return stem_in_launch(img, si, errp, st, nb, ib) ? fail(GCDR_ERR_DEVICE, std::string("stem input launch: ") + last_launch_error()) : 0;
                });
                launches_++;
                simt(pre + "stem_in", 0, (double)h_ * w_ * bpp_ + (double)(H_ + 2) * (W_ + 2) * kStemInC * 2);
            }
            ConvArgs a = conv_s1(which ? si_dr_ : si_gc_, n.stem_w16, n.enc1_b, n.c1, true);
            a.ep.out = b.t1;
            conv_op(a, EPI_POOL, pre + "stem", stem_flops, stem_bytes);
        }
        // encoders 2, 3: conv + pool + relu
        { ConvArgs a = conv_s1(b.t1, n.enc2, n.enc2_b, n.c2, true); a.ep.out = b.t2; conv_op(a, EPI_POOL, pre + "enc2"); }
        { ConvArgs a = conv_s1(b.t2, n.enc3, n.enc3_b, n.c3, true); a.ep.out = b.t3; conv_op(a, EPI_POOL, pre + "enc3"); }

        // shifted-MLP block body after its norm2+shift producer: fc1, dw+gelu+shift, fc2+res+norm
        auto block = [&](const DevBlock &bk, int H, int W, const Act &out, const std::string &bn) {
            { ConvArgs a = fc(b.hs, H, W, bk.C, bk.fc1, bk.fc1_b); a.ep.out = plain(b.f1, H, W, bk.C); conv_op(a, EPI_PLAIN, bn + ".fc1"); }
            const __half *f1 = b.f1; __half *f2 = b.f2;
            const float *dw = bk.dw_w, *db = bk.dw_b;
            ShiftSpec sb = bk.sb;
            int C = bk.C;
            ops_.push_back([=](cudaStream_t st) {
                return dw_gelu_shift_launch(f1, H, W, C, dw, db, sb, f2, st, nb, ib) ? fail(GCDR_ERR_DEVICE, std::string("dw launch: ") + last_launch_error()) : 0;
            });
            launches_++;
            simt(bn + ".dw_gelu_shift", 2.0 * 9 * H * W * C, 4.0 * H * W * C);
            ConvArgs a = fc(b.f2, H, W, bk.C, bk.fc2, bk.fc2_b);
            a.ep.res = b.y0;
            a.ep.g1 = bk.no_g; a.ep.b1 = bk.no_b; a.ep.eps1 = bk.no_eps;
            a.ep.out = out;
            conv_op(a, EPI_RESLN, bn + ".fc2_ln");
        };
        // patch embed 3 + norm + block1 norm2 + H shift
        {
            ConvArgs a = conv_s2(b.t3, n.pe3, n.pe3_b, n.c4);
            a.ep.g1 = n.pe3n_g; a.ep.b1 = n.pe3n_b; a.ep.eps1 = n.pe3n_eps;
            a.ep.g2 = n.blk[0].n2_g; a.ep.b2 = n.blk[0].n2_b; a.ep.eps2 = n.blk[0].n2_eps;
            a.ep.out = plain(b.y0, H4, W4, n.c4);
            a.ep.out2 = plain(b.hs, H4, W4, n.c4);
            a.ep.shift = n.blk[0].sa;
            conv_op(a, EPI_LN2, pre + "pe3_ln");
        }
        block(n.blk[0], H4, W4, b.t4, pre + "block1");
        {
            ConvArgs a = conv_s2(b.t4, n.pe4, n.pe4_b, n.c5);
            a.ep.g1 = n.pe4n_g; a.ep.b1 = n.pe4n_b; a.ep.eps1 = n.pe4n_eps;
            a.ep.g2 = n.blk[1].n2_g; a.ep.b2 = n.blk[1].n2_b; a.ep.eps2 = n.blk[1].n2_eps;
            a.ep.out = plain(b.y0, H5, W5, n.c5);
            a.ep.out2 = plain(b.hs, H5, W5, n.c5);
            a.ep.shift = n.blk[1].sa;
            conv_op(a, EPI_LN2, pre + "pe4_ln");
        }
        block(n.blk[1], H5, W5, b.b2o, pre + "block2");
        // decoder 1 -> up + t4 -> dblock1
        { ConvArgs a = conv_s1(b.b2o, n.dec[0], n.dec_b[0], n.c4, false); a.ep.out = plain(b.dconv, H5, W5, n.c4); conv_op(a, EPI_PLAIN, pre + "dec1"); }
        auto up_tok = [&](int H, int W, int C, const Act &skip, const DevBlock &bk) {
            UpAddArgs u;
            u.d = b.dconv;
            u.skip = skip;
            u.out = plain(b.y0, H, W, C);
            u.tokens = 1;
            u.g = bk.n2_g; u.b = bk.n2_b; u.eps = bk.n2_eps;
            u.h = plain(b.hs, H, W, C);
            u.shift = bk.sa;
            u.nimg = nb;
            u.img_bytes = ib;
            ops_.push_back([u, this](cudaStream_t st) { return up_add_launch(u, st) ? fail(GCDR_ERR_DEVICE, std::string("up_add launch: ") + last_launch_error()) : 0; });
            launches_++;
            simt(pre + "join_ln" + std::to_string(H), 0, 2.0 * (H / 2) * (W / 2) * C + 6.0 * H * W * C);
        };
        auto up_pad = [&](const Act &skip, const Act &out) {
            UpAddArgs u;
            u.d = b.dconv;
            u.skip = skip;
            u.out = out;
            u.nimg = nb;
            u.img_bytes = ib;
            ops_.push_back([u, this](cudaStream_t st) { return up_add_launch(u, st) ? fail(GCDR_ERR_DEVICE, std::string("up_add launch: ") + last_launch_error()) : 0; });
            launches_++;
            simt(pre + "join" + std::to_string(out.H), 0, 2.0 * (out.H / 2) * (out.W / 2) * out.C + 4.0 * out.H * out.W * out.C);
        };
        up_tok(H4, W4, n.c4, b.t4, n.blk[2]);
        block(n.blk[2], H4, W4, b.db1o, pre + "dblock1");
        { ConvArgs a = conv_s1(b.db1o, n.dec[1], n.dec_b[1], n.c3, false); a.ep.out = plain(b.dconv, H4, W4, n.c3); conv_op(a, EPI_PLAIN, pre + "dec2"); }
        up_tok(H3, W3, n.c3, b.t3, n.blk[3]);
        block(n.blk[3], H3, W3, b.db2o, pre + "dblock2");
        { ConvArgs a = conv_s1(b.db2o, n.dec[2], n.dec_b[2], n.c2, false); a.ep.out = plain(b.dconv, H3, W3, n.c2); conv_op(a, EPI_PLAIN, pre + "dec3"); }
        up_pad(b.t2, b.d3);
        { ConvArgs a = conv_s1(b.d3, n.dec[3], n.dec_b[3], n.c1, false); a.ep.out = plain(b.dconv, H2, W2, n.c1); conv_op(a, EPI_PLAIN, pre + "dec4"); }
        up_pad(b.t1, b.d4);
        { ConvArgs a = conv_s1(b.d4, n.dec[4], n.dec_b[4], n.c1, false); a.ep.out = plain(b.dec5, H1, W1, n.c1); conv_op(a, EPI_PLAIN, pre + "dec5"); }
        // head: recomputed stem skip + bilinear + 1x1 + sigmoid, then div6 (GC) or u8 out (DR)
        const double hpx = which ? (double)h_ * w_ : (double)H_ * W_;
        const double head_flops = hpx * 2.0 * (n.c1 * 9 * n.cin + 3 * n.c1);
        const double head_bytes = hpx * bpp_ + (which ? 12.0 * hpx + hpx * bpp_ : 12.0 * hpx) + (double)H1 * W1 * n.c1 * 2;
        if (simt_stem_) {
            HeadArgs ha;
            ha.img = img;
            ha.r = which ? r_ : nullptr;
            ha.H = H_; ha.W = W_; ha.cin = n.cin; ha.c1 = n.c1;
            ha.w = n.enc1_w; ha.b = n.enc1_b; ha.fw = n.fin_w; ha.fb = n.fin_b;
            ha.dec5 = b.dec5;
            ha.is_dr = which;
            if (!which) {
                ha.r_out = r_;
                ha.ism_out = plan_debug_ ? ism_ : nullptr;
            } else {
                ha.dst = d_dst_;
                ha.y_out = plan_debug_ ? ydbg_ : nullptr;
            }
            ops_.push_back([ha, this](cudaStream_t st) { return head_launch(ha, st) ? fail(GCDR_ERR_DEVICE, std::string("head launch: ") + last_launch_error()) : 0; });
            launches_++;
            simt(pre + "head", head_flops, head_bytes, false);
        } else {
            ConvArgs a = conv_s1(which ? si_dr_ : si_gc_, n.stem_w16, n.enc1_b, n.c1, false);
            HeadParams &hp = a.ep.head;
            hp.dec5 = b.dec5;
            for (int i = 0; i < 3 * n.c1; i++) hp.fw[i] = n.head_fw[i];
            for (int i = 0; i < 3; i++) hp.fb[i] = n.head_fb[i];
            for (int i = 0; i < n.c1; i++) hp.b1[i] = n.head_b1[i];
            hp.si_in = which ? si_dr_ : si_gc_;
            hp.is_dr = which;
            if (!which) {
                hp.si_out = si_dr_;
                hp.r_out = plan_debug_ ? r_ : nullptr;
                hp.ism_out = plan_debug_ ? ism_ : nullptr;
            } else {
                hp.img = img;
                hp.dst = d_dst_;
                hp.y_out = plan_debug_ ? ydbg_ : nullptr;
            }
            conv_op(a, EPI_HEAD, pre + "head", head_flops, head_bytes);
        }
    }
    if (bias_fail_) return fail(GCDR_ERR_DEVICE, "conv bias copy failed or split-K workspace too small");
    return info_.size() == ops_.size() ? GCDR_OK : fail(GCDR_ERR_DEVICE, "op metadata mismatch");
}

int Worker::profile(int reps, std::vector<double> &ms) {
    if (!bound_) return fail(GCDR_ERR_ARG, "worker not bound to a size");
    const size_t n = ops_.size();
    std::vector<cudaEvent_t> ev(n + 1);
    for (auto &e : ev) cudaEventCreate(&e);
    ms.assign(n, 0.0);
    int rc = GCDR_OK;
    for (int r = 0; r < reps && !rc; r++) {
        for (size_t i = 0; i < n && !rc; i++) {
            cudaEventRecord(ev[i], stream_);
            rc = ops_[i](stream_);
        }
        cudaEventRecord(ev[n], stream_);
        if (cudaEventSynchronize(ev[n]) != cudaSuccess) rc = fail(GCDR_ERR_DEVICE, "profile sync");
        for (size_t i = 0; i < n && !rc; i++) {
            float t = 0;
            cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
            ms[i] += t / reps;
        }
    }
    for (auto &e : ev) cudaEventDestroy(e);
    return rc;
}

int Worker::run_ops(cudaStream_t st) {
    for (auto &op : ops_) {
        int rc = op(st);
        if (rc) return rc;
    }
    return GCDR_OK;
}

int Worker::capture() {
    if (exec_) { cudaGraphExecDestroy(exec_); exec_ = nullptr; }
    if (graph_) { cudaGraphDestroy(graph_); graph_ = nullptr; }
    if (!use_graph_) return GCDR_OK;
    if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return fail(GCDR_ERR_DEVICE, "graph capture begin failed");
    const int rc = run_ops(stream_);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(stream_, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess || !g) return fail(GCDR_ERR_DEVICE, std::string("graph capture failed: ") + cudaGetErrorString(e));
    graph_ = g;
    if (cudaGraphInstantiate(&exec_, graph_, 0) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "graph instantiate failed");
    return GCDR_OK;
}

int Worker::bind(int w, int h, int fmt, int nimg) {
    ++tick_;
    if (bound_ && w == w_ && h == h_ && fmt == fmt_ && plan_debug_ == debug_ && nimg_ == nimg) return GCDR_OK;
    if (cudaSetDevice(device_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "cudaSetDevice");
    if (wait_stream() != cudaSuccess) return fail(GCDR_ERR_DEVICE, "stream sync");
    // the shape's plan may be cached: swap it in, graph and all
    for (size_t i = 0; i < cache_.size(); i++) {
        ShapePlan &p = cache_[i];
        if (p.w != w || p.h != h || p.fmt != fmt || p.debug != debug_ || p.nimg != nimg) continue;
        ShapePlan hit = std::move(p);
        cache_.erase(cache_.begin() + (long)i);
        if (bound_) stash();
        else release_current();
        restore(std::move(hit));
        bound_ = true;
        return GCDR_OK;
    }
    // a new shape: plan its arena, build its ops, capture its graph
    if (bound_) stash();
    else release_current();   // the leftovers of a plan that failed part way
    w_ = w; h_ = h; fmt_ = fmt;
    bpp_ = fmt >= 2 ? 4 : 3;
    ph_ = (-h) & 31; pw_ = (-w) & 31;
    H_ = h + ph_; W_ = w + pw_;
    plan_debug_ = debug_;
    nimg_ = nimg;
    int rc = plan_arena();
    if (rc) return rc;
    rc = build_all_ops();
    if (rc) return rc;
    rc = capture();
    if (rc) return rc;
    captures_++;
    bound_ = true;
    return GCDR_OK;
}

int Worker::check_err_flag() {
    if (*h_err_ & GCDR_ERR_FLAG_TIMEOUT) return fail(GCDR_ERR_TIMEOUT, "a device-side wait timed out");
    if (*h_err_) return fail(GCDR_ERR_DEVICE, "device error flag set");
    return GCDR_OK;
}

namespace {

// Whether host address p lies in page-locked memory (cudaMallocHost / cudaHostAlloc, or a
// range the caller registered with cudaHostRegister): the copy engines then read or write it
// directly, with no staging copy.
bool pinned(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

bool pinned_range(const uint8_t *p, size_t n) { return pinned(p) && pinned(p + n - 1); }

}  // namespace

int Worker::enhance_host(const uint8_t *src, int w, int h, int src_stride, uint8_t *dst, int dst_stride, int fmt) {
    if (inject_device_loss > 0) {
        inject_device_loss--;
        return fail(GCDR_ERR_DEVICE, "injected device loss");
    }
    if (cudaSetDevice(device_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "cudaSetDevice");
    int rc = bind(w, h, fmt);
    if (rc) return rc;
    const size_t row = (size_t)w * bpp_;
    auto band = [&](int b, int &y0, int &y1) {
        y0 = (int)((long long)h * b / kHostBands);
        y1 = (int)((long long)h * (b + 1) / kHostBands);
    };
    // page-locked caller buffers are copied by DMA directly (any row stride); pageable ones go
    // through the worker's pinned staging, copied by the host in row bands
    const size_t src_len = (size_t)(h - 1) * src_stride + row, dst_len = (size_t)(h - 1) * dst_stride + row;
    const bool direct_in = pinned_range(src, src_len);
    const bool direct_out = pinned_range(dst, dst_len);
    const bool overlap = dst < src + src_len && src < dst + dst_len;
    if (direct_in) {
        if (cudaMemcpy2DAsync(d_src_, row, src, src_stride, row, h, cudaMemcpyHostToDevice, stream_) != cudaSuccess)
            return fail(GCDR_ERR_DEVICE, "H2D copy failed");
    } else {
        // stage and upload: band b's H2D is enqueued by whichever thread staged it (the bands
        // are disjoint, so their order on the stream does not matter); the graph follows them all
        std::atomic<int> up_fail{0};
        pool_->run(kHostBands, [&](int b) {
            int y0, y1;
            band(b, y0, y1);
            uint8_t *stage = h_src_ + (size_t)y0 * row;
            if ((size_t)src_stride == row) std::memcpy(stage, src + (size_t)y0 * row, (size_t)(y1 - y0) * row);
            else
                for (int y = y0; y < y1; y++) std::memcpy(h_src_ + (size_t)y * row, src + (size_t)y * src_stride, row);
            if (cudaMemcpyAsync(d_src_ + (size_t)y0 * row, stage, (size_t)(y1 - y0) * row, cudaMemcpyHostToDevice,
                                stream_) != cudaSuccess)
                up_fail = 1;
        });
        if (up_fail) return fail(GCDR_ERR_DEVICE, "H2D copy failed");
    }
    if (exec_) {
        if (cudaGraphLaunch(exec_, stream_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "graph launch failed");
    } else if ((rc = run_ops(stream_))) return rc;
    cudaError_t e = cudaMemcpyAsync(h_err_, d_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_);
    if (e == cudaSuccess) e = cudaEventRecord(flag_ev_, stream_);
    if (direct_out && !overlap) {
        // a destination apart from the source is written by DMA right behind the graph (after a
        // device error its contents are unspecified; the retry reads the untouched source)
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(dst, dst_stride, d_dst_, row, row, h, cudaMemcpyDeviceToHost, stream_);
        if (e == cudaSuccess) e = (cudaError_t)wait_stream();
        if (e != cudaSuccess) {
            cudaStreamSynchronize(stream_);
            return fail(GCDR_ERR_DEVICE, std::string("CUDA error: ") + cudaGetErrorString(e));
        }
        return check_err_flag();
    }
    if (!direct_out) {
        for (int b = 0; b < kHostBands && e == cudaSuccess; b++) {
            int y0, y1;
            band(b, y0, y1);
            e = cudaMemcpyAsync(h_dst_ + (size_t)y0 * row, d_dst_ + (size_t)y0 * row, (size_t)(y1 - y0) * row,
                                cudaMemcpyDeviceToHost, stream_);
            if (e == cudaSuccess) e = cudaEventRecord(band_ev_[b], stream_);
        }
    }
    if (e == cudaSuccess) e = wait_event(flag_ev_);
    if (e != cudaSuccess) {
        cudaStreamSynchronize(stream_);
        return fail(GCDR_ERR_DEVICE, std::string("CUDA error: ") + cudaGetErrorString(e));
    }
    // the caller's buffer is written only after a clean device flag: dst may alias src, and a
    // device error is retried on a fresh worker from the same src
    if ((rc = check_err_flag())) {
        cudaStreamSynchronize(stream_);
        return rc;
    }
    if (direct_out) {
        // page-locked destination overlapping the source (in place): DMA once the flag is clean
        e = cudaMemcpy2DAsync(dst, dst_stride, d_dst_, row, row, h, cudaMemcpyDeviceToHost, stream_);
        if (e == cudaSuccess) e = (cudaError_t)wait_stream();
        return e == cudaSuccess ? GCDR_OK : fail(GCDR_ERR_DEVICE, "D2H copy failed");
    }
    std::atomic<int> down_fail{0};
    pool_->run(kHostBands, [&](int b) {
        int y0, y1;
        band(b, y0, y1);
        if (wait_event(band_ev_[b]) != cudaSuccess) {
            down_fail = 1;
            return;
        }
        const uint8_t *stage = h_dst_ + (size_t)y0 * row;
        if ((size_t)dst_stride == row) std::memcpy(dst + (size_t)y0 * row, stage, (size_t)(y1 - y0) * row);
        else
            for (int y = y0; y < y1; y++) std::memcpy(dst + (size_t)y * dst_stride, h_dst_ + (size_t)y * row, row);
    });
    if (down_fail) {
        cudaStreamSynchronize(stream_);
        return fail(GCDR_ERR_DEVICE, "D2H copy failed");
    }
    return GCDR_OK;
}

int Worker::enhance_device(const uint8_t *d_src, int w, int h, uint8_t *d_dst, int fmt, cudaStream_t st) {
    if (cudaSetDevice(device_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "cudaSetDevice");
    int rc = bind(w, h, fmt);
    if (rc) return rc;
    // everything is enqueued on the caller's stream (or the worker's own)
    cudaStream_t s = st ? st : stream_;
    const size_t img = (size_t)w * h * bpp_;
    cudaError_t e = cudaMemcpyAsync(d_src_, d_src, img, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return fail(GCDR_ERR_DEVICE, "d2d copy");
    if (exec_) {
        if (cudaGraphLaunch(exec_, s) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "graph launch failed");
    } else if ((rc = run_ops(s))) return rc;
    e = cudaMemcpyAsync(d_dst, d_dst_, img, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return fail(GCDR_ERR_DEVICE, "d2d copy");
    return GCDR_OK;
}

int Worker::enhance_host_batch(const uint8_t *const *src, int n, int w, int h, int src_stride, uint8_t *const *dst,
                               int dst_stride, int fmt) {
    if (n < 1 || n > kMaxBatch) return fail(GCDR_ERR_ARG, "batch size must be 1..16");
    if (inject_device_loss > 0) {
        inject_device_loss--;
        return fail(GCDR_ERR_DEVICE, "injected device loss");
    }
    if (cudaSetDevice(device_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "cudaSetDevice");
    int rc = bind(w, h, fmt, n);
    if (rc) return rc;
    const size_t row = (size_t)w * bpp_, img = row * h;
    const size_t src_len = (size_t)(h - 1) * src_stride + row;
    // upload: page-locked sources by DMA directly, pageable ones staged (one image per helper task)
    std::atomic<int> up_fail{0};
    pool_->run(n, [&](int k) {
        uint8_t *dev = slices_[k].d_src;
        cudaError_t e;
        if (pinned_range(src[k], src_len)) {
            e = cudaMemcpy2DAsync(dev, row, src[k], src_stride, row, h, cudaMemcpyHostToDevice, stream_);
        } else {
            uint8_t *stage = h_src_ + (size_t)k * img;
            for (int y = 0; y < h; y++) std::memcpy(stage + (size_t)y * row, src[k] + (size_t)y * src_stride, row);
            e = cudaMemcpyAsync(dev, stage, img, cudaMemcpyHostToDevice, stream_);
        }
        if (e != cudaSuccess) up_fail = 1;
    });
    if (up_fail) return fail(GCDR_ERR_DEVICE, "H2D copy failed");
    if (exec_) {
        if (cudaGraphLaunch(exec_, stream_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "graph launch failed");
    } else if ((rc = run_ops(stream_))) return rc;
    cudaError_t e = cudaSuccess;
    for (int k = 0; k < n && e == cudaSuccess; k++)
        e = cudaMemcpyAsync(h_errs_ + k, slices_[k].d_err, sizeof(int), cudaMemcpyDeviceToHost, stream_);
    for (int k = 0; k < n && e == cudaSuccess; k++)
        e = cudaMemcpyAsync(h_dst_ + (size_t)k * img, slices_[k].d_dst, img, cudaMemcpyDeviceToHost, stream_);
    if (e == cudaSuccess) e = (cudaError_t)wait_stream();
    if (e != cudaSuccess) {
        cudaStreamSynchronize(stream_);
        return fail(GCDR_ERR_DEVICE, std::string("CUDA error: ") + cudaGetErrorString(e));
    }
    // the callers' buffers are written only after every image's device flag is clean
    int flags = 0;
    for (int k = 0; k < n; k++) flags |= h_errs_[k];
    if (flags & GCDR_ERR_FLAG_TIMEOUT) return fail(GCDR_ERR_TIMEOUT, "a device-side wait timed out");
    if (flags) return fail(GCDR_ERR_DEVICE, "device error flag set");
    pool_->run(n, [&](int k) {
        const uint8_t *stage = h_dst_ + (size_t)k * img;
        for (int y = 0; y < h; y++) std::memcpy(dst[k] + (size_t)y * dst_stride, stage + (size_t)y * row, row);
    });
    return GCDR_OK;
}

int Worker::enhance_device_batch(const uint8_t *const *d_src, int n, int w, int h, uint8_t *const *d_dst, int fmt,
                                 cudaStream_t st) {
    if (n < 1 || n > kMaxBatch) return fail(GCDR_ERR_ARG, "batch size must be 1..16");
    if (cudaSetDevice(device_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "cudaSetDevice");
    int rc = bind(w, h, fmt, n);
    if (rc) return rc;
    cudaStream_t s = st ? st : stream_;
    const size_t img = (size_t)w * h * bpp_;
    for (int k = 0; k < n; k++)
        if (cudaMemcpyAsync(slices_[k].d_src, d_src[k], img, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return fail(GCDR_ERR_DEVICE, "d2d copy");
    if (exec_) {
        if (cudaGraphLaunch(exec_, s) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "graph launch failed");
    } else if ((rc = run_ops(s))) return rc;
    for (int k = 0; k < n; k++)
        if (cudaMemcpyAsync(d_dst[k], slices_[k].d_dst, img, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return fail(GCDR_ERR_DEVICE, "d2d copy");
    return GCDR_OK;
}

int Worker::debug_intermediates(float *gc_in, float *gc_out, float *dr_in, float *dr_out) {
    if (!bound_) return fail(GCDR_ERR_ARG, "worker not bound to a size");
    if (nimg_ != 1) return fail(GCDR_ERR_ARG, "debug intermediates need a single-image enhance");
    if (cudaStreamSynchronize(stream_) != cudaSuccess) return fail(GCDR_ERR_DEVICE, "sync");
    const size_t n3 = (size_t)H_ * W_ * 3;
    std::vector<float> x(n3), r(n3);
    float *dx = nullptr;
    if (cudaMalloc(&dx, n3 * 4) != cudaSuccess) return fail(GCDR_ERR_OOM, "debug alloc");
    int rc = k_bgr2nhwc(d_src_, w_, h_, w_ * bpp_, fmt_, dx, ph_, pw_, stream_);
    cudaMemcpyAsync(x.data(), dx, n3 * 4, cudaMemcpyDeviceToHost, stream_);
    std::vector<__half> si;
    if (simt_stem_) {
        cudaMemcpyAsync(r.data(), r_, n3 * 4, cudaMemcpyDeviceToHost, stream_);
    } else {
        // r = r_hi + r_lo from the DR stem input (interior rows of [H+2][W+2][16]): the
        // division-corrected image exactly as the DR stem reads it, debug mode or not
        si.resize((size_t)si_dr_.rows() * kStemInC);
        cudaMemcpyAsync(si.data(), si_dr_.p, si.size() * 2, cudaMemcpyDeviceToHost, stream_);
    }
    if (gc_out && plan_debug_) cudaMemcpyAsync(gc_out, ism_, n3 * 4, cudaMemcpyDeviceToHost, stream_);
    if (dr_out && plan_debug_) cudaMemcpyAsync(dr_out, ydbg_, n3 * 4, cudaMemcpyDeviceToHost, stream_);
    cudaError_t e = cudaStreamSynchronize(stream_);
    cudaFree(dx);
    if (rc || e != cudaSuccess) return fail(GCDR_ERR_DEVICE, "debug copy failed");
    if ((gc_out || dr_out) && !plan_debug_) return fail(GCDR_ERR_ARG, "shading map / output need debug mode (gcdr_cuda_set_debug)");
    if (!si.empty())
        for (int yy = 0; yy < H_; yy++)
            for (int xx = 0; xx < W_; xx++) {
                const __half *v = si.data() + si_dr_.row(yy, xx) * kStemInC;
                for (int c = 0; c < 3; c++)
                    r[((size_t)yy * W_ + xx) * 3 + c] = __half2float(v[6 + c]) + __half2float(v[9 + c]);
            }
    if (gc_in) std::memcpy(gc_in, x.data(), n3 * 4);
    if (dr_in)
        for (size_t p = 0; p < (size_t)H_ * W_; p++)
            for (int c = 0; c < 3; c++) {
                dr_in[p * 6 + c] = x[p * 3 + c];
                dr_in[p * 6 + 3 + c] = r[p * 3 + c];
            }
    return GCDR_OK;
}

}  // namespace gcdr
