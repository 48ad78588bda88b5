// model.cpp -- ONNX protobuf reader and GCDRNet topology recogniser.
//
// Wire-format decoding of onnx.ModelProto (graph = field 7), GraphProto
// (node = 1, initializer = 5), NodeProto (input 1, output 2, op_type 4,
// attribute 5), AttributeProto (name 1, f 2, i 3, s 4, t 5, floats 7,
// ints 8) and TensorProto (dims 1, data_type 2, float_data 4, int64_data 7,
// name 8, raw_data 9).  Only what the two GCDRNet exports use is supported.
//
// Recognition mirrors what the reference's engine + GCDR passes derive from
// the same graph: conv attributes and the reflect Pad in front of the
// encoder/decoder convs (gc#22-23), the LayerNorm epsilons, the Gemm B
// operands (transB=0), the Resize mode (linear, half_pixel, x2), and the
// shift-MLP groups/offsets exactly as FuseShiftPass derives them
// (Extensions/ChannelShiftOp.cs:64-188, offset formula :158-161).
#include "model.h"

#include <cmath>
#include <cstring>
#include <map>
#include <sstream>
#include <unordered_map>

#include "../../../include/gcdr_cuda.h"

namespace gcdr {
namespace {

struct Reader {
    const uint8_t *p, *end;
    bool ok = true;
    Reader(const uint8_t *b, size_t n) : p(b), end(b + n) {}
    bool more() const { return ok && p < end; }
    uint64_t varint() {
        uint64_t r = 0;
        int s = 0;
        while (p < end && s < 64) {
            uint8_t c = *p++;
            r |= uint64_t(c & 0x7f) << s;
            s += 7;
            if (!(c & 0x80)) return r;
        }
        ok = false;
        return 0;
    }
    // Reads one field header; returns false at the end.
    bool field(int &num, int &wt) {
        if (!more()) return false;
        uint64_t k = varint();
        num = int(k >> 3);
        wt = int(k & 7);
        return ok;
    }
    bool bytes(const uint8_t *&b, size_t &n) {
        uint64_t l = varint();
        if (!ok || l > uint64_t(end - p)) { ok = false; return false; }
        b = p;
        n = size_t(l);
        p += l;
        return true;
    }
    void skip(int wt) {
        const uint8_t *b;
        size_t n;
        switch (wt) {
            case 0: varint(); break;
            case 1: if (end - p < 8) ok = false; else p += 8; break;
            case 5: if (end - p < 4) ok = false; else p += 4; break;
            case 2: bytes(b, n); break;
            default: ok = false;
        }
    }
};

struct Tensor {
    std::vector<int64_t> dims;
    int dtype = 0;
    std::vector<float> f;
    std::vector<int64_t> i;
    size_t count() const {
        size_t n = 1;
        for (auto d : dims) n *= size_t(d);
        return n;
    }
};

struct Attr {
    float f = 0;
    int64_t i = 0;
    std::string s;
    std::vector<int64_t> ints;
    std::vector<float> floats;
    bool has_t = false;
    Tensor t;
};

struct Node {
    std::string op;
    std::vector<std::string> in, out;
    std::map<std::string, Attr> attrs;
};

static void packed_or_single_i64(Reader &r, int wt, std::vector<int64_t> &dst) {
    if (wt == 0) { dst.push_back(int64_t(r.varint())); return; }
    const uint8_t *b; size_t n;
    if (!r.bytes(b, n)) return;
    Reader q(b, n);
    while (q.more()) dst.push_back(int64_t(q.varint()));
    if (!q.ok) r.ok = false;
}

static void packed_or_single_f32(Reader &r, int wt, std::vector<float> &dst) {
    if (wt == 5) {
        if (r.end - r.p < 4) { r.ok = false; return; }
        float v; std::memcpy(&v, r.p, 4); r.p += 4; dst.push_back(v); return;
    }
    const uint8_t *b; size_t n;
    if (!r.bytes(b, n)) return;
    size_t k = n / 4, o = dst.size();
    dst.resize(o + k);
    std::memcpy(dst.data() + o, b, k * 4);
}

static bool parse_tensor(const uint8_t *b, size_t n, Tensor &t, std::string &name) {
    Reader r(b, n);
    int f, wt;
    const uint8_t *raw = nullptr;
    size_t raw_n = 0;
    while (r.field(f, wt)) {
        if (f == 1) packed_or_single_i64(r, wt, t.dims);
        else if (f == 2 && wt == 0) t.dtype = int(r.varint());
        else if (f == 4) packed_or_single_f32(r, wt, t.f);
        else if (f == 7) packed_or_single_i64(r, wt, t.i);
        else if (f == 8 && wt == 2) { const uint8_t *s; size_t sn; r.bytes(s, sn); name.assign((const char *)s, sn); }
        else if (f == 9 && wt == 2) r.bytes(raw, raw_n);
        else if (f == 14 && wt == 0) { if (r.varint() == 1) return false; }  // external data
        else r.skip(wt);
    }
    if (!r.ok) return false;
    if (raw) {
        size_t cnt = t.count();
        if (t.dtype == 1) {
            if (raw_n != cnt * 4) return false;
            t.f.resize(cnt);
            std::memcpy(t.f.data(), raw, raw_n);
        } else if (t.dtype == 7) {
            if (raw_n != cnt * 8) return false;
            t.i.resize(cnt);
            std::memcpy(t.i.data(), raw, raw_n);
        } else if (t.dtype == 6) {
            if (raw_n != cnt * 4) return false;
            t.i.resize(cnt);
            for (size_t k = 0; k < cnt; k++) { int32_t v; std::memcpy(&v, raw + 4 * k, 4); t.i[k] = v; }
        }
    }
    return true;
}

static bool parse_attr(const uint8_t *b, size_t n, std::string &name, Attr &a) {
    Reader r(b, n);
    int f, wt;
    while (r.field(f, wt)) {
        if (f == 1 && wt == 2) { const uint8_t *s; size_t sn; r.bytes(s, sn); name.assign((const char *)s, sn); }
        else if (f == 2 && wt == 5) {
            if (r.end - r.p < 4) return false;
            std::memcpy(&a.f, r.p, 4); r.p += 4;
        }
        else if (f == 3 && wt == 0) a.i = int64_t(r.varint());
        else if (f == 4 && wt == 2) { const uint8_t *s; size_t sn; r.bytes(s, sn); a.s.assign((const char *)s, sn); }
        else if (f == 5 && wt == 2) {
            const uint8_t *s; size_t sn; r.bytes(s, sn);
            std::string tn;
            a.has_t = parse_tensor(s, sn, a.t, tn);
        }
        else if (f == 7) packed_or_single_f32(r, wt, a.floats);
        else if (f == 8) packed_or_single_i64(r, wt, a.ints);
        else r.skip(wt);
    }
    return r.ok;
}

static bool parse_node(const uint8_t *b, size_t n, Node &nd) {
    Reader r(b, n);
    int f, wt;
    while (r.field(f, wt)) {
        const uint8_t *s; size_t sn;
        if ((f == 1 || f == 2 || f == 4) && wt == 2) {
            r.bytes(s, sn);
            std::string v((const char *)s, sn);
            if (f == 1) nd.in.push_back(v);
            else if (f == 2) nd.out.push_back(v);
            else nd.op = v;
        } else if (f == 5 && wt == 2) {
            r.bytes(s, sn);
            std::string an;
            Attr a;
            if (!parse_attr(s, sn, an, a)) return false;
            nd.attrs[an] = std::move(a);
        } else r.skip(wt);
    }
    return r.ok;
}

struct Graph {
    std::vector<Node> nodes;
    std::unordered_map<std::string, Tensor> inits;
    std::unordered_map<std::string, int> producer;

    const Tensor *init(const std::string &n) const {
        auto it = inits.find(n);
        return it == inits.end() ? nullptr : &it->second;
    }
    const Node *prod(const std::string &v) const {
        auto it = producer.find(v);
        return it == producer.end() ? nullptr : &nodes[it->second];
    }
};

static int parse_graph(const uint8_t *data, size_t len, Graph &g, std::string &err) {
    Reader r(data, len);
    int f, wt;
    const uint8_t *gb = nullptr;
    size_t gn = 0;
    while (r.field(f, wt)) {
        if (f == 7 && wt == 2) r.bytes(gb, gn);
        else r.skip(wt);
    }
    if (!r.ok || !gb) { err = "not an ONNX ModelProto (no graph)"; return GCDR_ERR_MODEL; }
    Reader q(gb, gn);
    while (q.field(f, wt)) {
        const uint8_t *s; size_t sn;
        if (f == 1 && wt == 2) {
            q.bytes(s, sn);
            Node nd;
            if (!parse_node(s, sn, nd)) { err = "malformed NodeProto"; return GCDR_ERR_MODEL; }
            g.nodes.push_back(std::move(nd));
        } else if (f == 5 && wt == 2) {
            q.bytes(s, sn);
            Tensor t;
            std::string name;
            if (!parse_tensor(s, sn, t, name)) { err = "malformed or external TensorProto"; return GCDR_ERR_MODEL; }
            g.inits[name] = std::move(t);
        } else q.skip(wt);
    }
    if (!q.ok) { err = "truncated GraphProto"; return GCDR_ERR_MODEL; }
    for (size_t k = 0; k < g.nodes.size(); k++) {
        Node &nd = g.nodes[k];
        for (auto &o : nd.out) g.producer[o] = int(k);
        if (nd.op == "Constant") {
            auto it = nd.attrs.find("value");
            if (it != nd.attrs.end() && it->second.has_t && !nd.out.empty()) g.inits[nd.out[0]] = it->second.t;
        }
    }
    return GCDR_OK;
}

struct Fail {
    int code;
    std::string msg;
};

[[noreturn]] static void fail(const std::string &m, int code = GCDR_ERR_UNSUPPORTED) { throw Fail{code, m}; }

static const Tensor &need(const Graph &g, const std::string &n) {
    const Tensor *t = g.init(n);
    if (!t) fail("initializer '" + n + "' not found");
    return *t;
}

static std::vector<int64_t> ints_of(const Node &n, const char *a) {
    auto it = n.attrs.find(a);
    return it == n.attrs.end() ? std::vector<int64_t>{} : it->second.ints;
}

static int64_t int_of(const Node &n, const char *a, int64_t dflt) {
    auto it = n.attrs.find(a);
    return it == n.attrs.end() ? dflt : it->second.i;
}

static std::string str_of(const Node &n, const char *a) {
    auto it = n.attrs.find(a);
    return it == n.attrs.end() ? std::string() : it->second.s;
}

static const Node &node_using(const Graph &g, const std::string &op, int slot, const std::string &v) {
    for (auto &n : g.nodes)
        if (n.op == op && int(n.in.size()) > slot && n.in[slot] == v) return n;
    fail(op + " node using '" + v + "' not found");
}

// A named conv: weights/bias, attributes, and the reflect Pad feeding it.
static ConvW conv(const Graph &g, const std::string &name, int expect_k) {
    ConvW c;
    const Tensor &w = need(g, "m." + name + ".weight");
    const Tensor &b = need(g, "m." + name + ".bias");
    if (w.dims.size() != 4 || w.dtype != 1) fail(name + ": weight is not a 4-D float tensor");
    c.cout = int(w.dims[0]);
    c.cin = int(w.dims[1]);
    c.k = int(w.dims[2]);
    if (c.k != expect_k || w.dims[3] != expect_k) fail(name + ": unexpected kernel size");
    if (b.count() != size_t(c.cout)) fail(name + ": bias size");
    c.w = w.f;
    c.b = b.f;
    const Node &n = node_using(g, "Conv", 1, "m." + name + ".weight");
    auto st = ints_of(n, "strides"), pads = ints_of(n, "pads"), dil = ints_of(n, "dilations");
    if (int_of(n, "group", 1) != 1) fail(name + ": grouped conv not expected");
    for (auto d : dil) if (d != 1) fail(name + ": dilation");
    c.stride = st.empty() ? 1 : int(st[0]);
    for (auto s : st) if (s != c.stride) fail(name + ": anisotropic stride");
    int p = pads.empty() ? 0 : int(pads[0]);
    for (auto q : pads) if (q != p) fail(name + ": asymmetric pads");
    c.pad = p;
    const Node *pr = g.prod(n.in[0]);
    if (pr && pr->op == "Pad") {
        if (p != 0) fail(name + ": Pad followed by a padded conv");
        std::string mode = str_of(*pr, "mode");
        const Tensor *pv = pr->in.size() > 1 ? g.init(pr->in[1]) : nullptr;
        if (mode != "reflect" || !pv || pv->i.size() != 8) fail(name + ": unsupported Pad in front of conv");
        int64_t e[8] = {0, 0, 1, 1, 0, 0, 1, 1};
        for (int k = 0; k < 8; k++) if (pv->i[k] != e[k]) fail(name + ": reflect pad is not 1 px");
        c.reflect = true;
        c.pad = 1;
    }
    return c;
}

static LNW layernorm(const Graph &g, const std::string &name) {
    LNW l;
    const Tensor &w = need(g, "m." + name + ".weight");
    const Tensor &b = need(g, "m." + name + ".bias");
    l.c = int(w.count());
    l.g = w.f;
    l.b = b.f;
    if (b.count() != size_t(l.c)) fail(name + ": LayerNorm bias size");
    const Node &n = node_using(g, "LayerNormalization", 1, "m." + name + ".weight");
    if (int_of(n, "axis", -1) != -1) fail(name + ": LayerNorm axis");
    auto it = n.attrs.find("epsilon");
    l.eps = it == n.attrs.end() ? 1e-5f : it->second.f;
    return l;
}

static std::vector<float> gemm_b(const Graph &g, const std::string &bias, int C) {
    const Node &n = node_using(g, "Gemm", 2, bias);
    if (int_of(n, "transA", 0) || int_of(n, "transB", 0)) fail("Gemm with transposed operands");
    for (const char *a : {"alpha", "beta"}) {
        auto it = n.attrs.find(a);
        if (it != n.attrs.end() && it->second.f != 1.0f) fail("Gemm alpha/beta != 1");
    }
    const Tensor &b = need(g, n.in[1]);
    if (b.dims.size() != 2 || b.dims[0] != C || b.dims[1] != C) fail("Gemm weight shape");
    return b.f;
}

// Shift groups of every Split in graph order (FuseShiftPass pattern):
// Pad(const, H/W by p) -> Split(C into 5) -> per piece Slice[0:cut] /
// Slice[cut:L] on one spatial axis with cut = Mod(c, L) -> Concat -> ...
static std::vector<ShiftW> shifts(const Graph &g, std::vector<int> &split_sizes_out_c) {
    std::vector<ShiftW> out;
    for (size_t k = 0; k < g.nodes.size(); k++) {
        const Node &sp = g.nodes[k];
        if (sp.op != "Split") continue;
        const Node *pad = g.prod(sp.in[0]);
        if (!pad || pad->op != "Pad" || str_of(*pad, "mode") != "constant") fail("shift Split not fed by a constant Pad");
        const Tensor *pv = pad->in.size() > 1 ? g.init(pad->in[1]) : nullptr;
        if (!pv || pv->i.size() != 8) fail("shift pad amounts");
        const Tensor *val = pad->in.size() > 2 && !pad->in[2].empty() ? g.init(pad->in[2]) : nullptr;
        if (val && !val->f.empty() && val->f[0] != 0.0f) fail("shift pad value not zero");
        ShiftW s;
        std::vector<int> sizes;
        if (sp.in.size() > 1 && !sp.in[1].empty()) {
            const Tensor &st = need(g, sp.in[1]);
            for (auto v : st.i) sizes.push_back(int(v));
        } else {
            int nout = int(int_of(sp, "num_outputs", 0));
            if (nout <= 0) fail("Split without sizes");
            sizes.assign(size_t(nout), -1);   // resolved from C by the caller
        }
        if (int_of(sp, "axis", 0) != 1) fail("shift Split not over channels");
        int axis = -1;
        for (auto &piece : sp.out) {
            const Node *head = nullptr;
            for (auto &n : g.nodes) {
                if (n.op != "Slice" || n.in.empty() || n.in[0] != piece || n.in.size() < 4) continue;
                const Tensor *st = g.init(n.in[1]);
                if (st && !st->i.empty() && st->i[0] == 0) head = &n;
            }
            if (!head) fail("shift roll pattern not found");
            const Tensor &ax = need(g, head->in[3]);
            const Node *mod = g.prod(head->in[2]);
            if (!mod || mod->op != "Mod") fail("shift roll cut is not a Mod");
            const Tensor &cv = need(g, mod->in[0]);
            int a = int(ax.i.at(0)), c = int(cv.i.at(0));
            if (a != 2 && a != 3) fail("shift along a non-spatial axis");
            int p = int(pv->i[size_t(a)]);
            if (pv->i[size_t(a) + 4] != p) fail("asymmetric shift pad");
            // offset = ((p + cut) % L) - p with cut = c mod L and L = n + 2p > 2p >= |c|  ==> c
            if (c > p || c < -p) fail("shift larger than its zero pad");
            if (axis < 0) axis = a; else if (axis != a) fail("mixed shift axes");
            s.offs.push_back(c);
        }
        s.axis = axis;
        int e = 0;
        for (int v : sizes) { e += v; s.ends.push_back(v < 0 ? -1 : e); }
        out.push_back(s);
        split_sizes_out_c.push_back(int(sizes.size()));
    }
    return out;
}

static void resolve_groups(ShiftW &s, int C) {
    if (!s.ends.empty() && s.ends[0] >= 0) {
        if (s.ends.back() != C) fail("shift groups do not cover the channels");
        return;
    }
    int n = int(s.ends.size());
    int chunk = (C + n - 1) / n;       // ONNX Split num_outputs: ceil chunks, last smaller
    s.ends.clear();
    for (int k = 0; k < n; k++) s.ends.push_back(std::min(C, chunk * (k + 1)));
}

static void check_common(const Graph &g) {
    int resize = 0, pool = 0, sig = 0, erf = 0;
    for (auto &n : g.nodes) {
        if (n.op == "Resize") {
            resize++;
            if (str_of(n, "mode") != "linear" || str_of(n, "coordinate_transformation_mode") != "half_pixel")
                fail("Resize is not bilinear half_pixel");
            const Tensor *sc = n.in.size() > 2 ? g.init(n.in[2]) : nullptr;
            if (!sc || sc->f.size() != 4 || sc->f[0] != 1 || sc->f[1] != 1 || sc->f[2] != 2 || sc->f[3] != 2)
                fail("Resize scales are not [1,1,2,2]");
        } else if (n.op == "MaxPool") {
            pool++;
            auto k = ints_of(n, "kernel_shape"), s = ints_of(n, "strides"), p = ints_of(n, "pads");
            if (k != std::vector<int64_t>{2, 2} || s != std::vector<int64_t>{2, 2}) fail("MaxPool is not 2x2/2");
            for (auto v : p) if (v) fail("padded MaxPool");
            if (int_of(n, "ceil_mode", 0)) fail("MaxPool ceil_mode");
        } else if (n.op == "Sigmoid") sig++;
        else if (n.op == "Erf") erf++;
    }
    if (resize != 5 || pool != 3 || sig != 1 || erf != 4)
        fail("graph is not the GCDRNet UNeXt topology (Resize/MaxPool/Sigmoid/Erf counts)");
}

static void chk(bool c, const std::string &m) { if (!c) fail(m); }

static void recognise(const Graph &g, NetW &n) {
    check_common(g);
    n.enc[0] = conv(g, "encoder1.1", 3);
    n.enc[1] = conv(g, "encoder2.1", 3);
    n.enc[2] = conv(g, "encoder3.1", 3);
    n.pe3 = conv(g, "patch_embed3.proj", 3);
    n.pe4 = conv(g, "patch_embed4.proj", 3);
    for (int i = 0; i < 5; i++) n.dec[i] = conv(g, "decoder" + std::to_string(i + 1) + ".1", 3);
    n.fin = conv(g, "final", 1);
    n.cin = n.enc[0].cin;
    n.c1 = n.enc[0].cout; n.c2 = n.enc[1].cout; n.c3 = n.enc[2].cout;
    n.c4 = n.pe3.cout; n.c5 = n.pe4.cout;
    for (int i = 0; i < 3; i++) chk(n.enc[i].reflect && n.enc[i].stride == 1, "encoder conv is not reflect-padded stride 1");
    for (int i = 0; i < 5; i++) chk(n.dec[i].reflect && n.dec[i].stride == 1, "decoder conv is not reflect-padded stride 1");
    chk(!n.pe3.reflect && n.pe3.stride == 2 && n.pe3.pad == 1, "patch_embed3 is not a stride-2 zero-pad conv");
    chk(!n.pe4.reflect && n.pe4.stride == 2 && n.pe4.pad == 1, "patch_embed4 is not a stride-2 zero-pad conv");
    chk(n.fin.pad == 0 && n.fin.stride == 1 && n.fin.cout == 3, "final conv is not a 1x1 to 3 channels");
    chk(n.cin == 3 || n.cin == 6, "net input must have 3 (GC) or 6 (DR) channels");
    chk(n.enc[1].cin == n.c1 && n.enc[2].cin == n.c2 && n.pe3.cin == n.c3 && n.pe4.cin == n.c4, "encoder channel chain");
    chk(n.dec[0].cin == n.c5 && n.dec[0].cout == n.c4 && n.dec[1].cin == n.c4 && n.dec[1].cout == n.c3 &&
        n.dec[2].cin == n.c3 && n.dec[2].cout == n.c2 && n.dec[3].cin == n.c2 && n.dec[3].cout == n.c1 &&
        n.dec[4].cin == n.c1 && n.dec[4].cout == n.c1 && n.fin.cin == n.c1, "decoder channel chain");
    n.pe3_norm = layernorm(g, "patch_embed3.norm");
    n.pe4_norm = layernorm(g, "patch_embed4.norm");
    chk(n.pe3_norm.c == n.c4 && n.pe4_norm.c == n.c5, "patch-embed norm widths");

    std::vector<int> dummy;
    std::vector<ShiftW> sh = shifts(g, dummy);
    chk(sh.size() == 8, "expected 8 shift-MLP Splits");
    const char *bn[4] = {"block1", "block2", "dblock1", "dblock2"};
    const char *on[4] = {"norm3", "norm4", "dnorm3", "dnorm4"};
    int bc[4] = {n.c4, n.c5, n.c4, n.c3};
    for (int i = 0; i < 4; i++) {
        BlockW &b = n.blk[i];
        std::string p = std::string(bn[i]) + ".0.";
        b.norm2 = layernorm(g, p + "norm2");
        b.norm_out = layernorm(g, on[i]);
        int C = bc[i];
        chk(b.norm2.c == C && b.norm_out.c == C, std::string(bn[i]) + ": width");
        b.fc1_b = need(g, "m." + p + "mlp.fc1.bias").f;
        b.fc2_b = need(g, "m." + p + "mlp.fc2.bias").f;
        b.fc1_w = gemm_b(g, "m." + p + "mlp.fc1.bias", C);
        b.fc2_w = gemm_b(g, "m." + p + "mlp.fc2.bias", C);
        // depthwise conv: group = C
        const Tensor &dw = need(g, "m." + p + "mlp.dwconv.dwconv.weight");
        const Node &dn = node_using(g, "Conv", 1, "m." + p + "mlp.dwconv.dwconv.weight");
        chk(int_of(dn, "group", 1) == C && dw.dims.size() == 4 && dw.dims[0] == C && dw.dims[1] == 1 &&
            dw.dims[2] == 3 && dw.dims[3] == 3, std::string(bn[i]) + ": depthwise conv shape");
        auto pads = ints_of(dn, "pads");
        for (auto v : pads) chk(v == 1, std::string(bn[i]) + ": depthwise pads");
        b.dw.cout = C; b.dw.cin = 1; b.dw.k = 3; b.dw.pad = 1;
        b.dw.w = dw.f;
        b.dw.b = need(g, "m." + p + "mlp.dwconv.dwconv.bias").f;
        b.shift_a = sh[size_t(2 * i)];
        b.shift_b = sh[size_t(2 * i + 1)];
        resolve_groups(b.shift_a, C);
        resolve_groups(b.shift_b, C);
        chk(b.shift_a.axis == 2 && b.shift_b.axis == 3, std::string(bn[i]) + ": shift axes are not H then W");
    }
}

}  // namespace

int parse_gcdr_net(const uint8_t *data, size_t len, NetW &net, std::string &err) {
    if (!data || len == 0) { err = "empty model"; return GCDR_ERR_ARG; }
    Graph g;
    int rc = parse_graph(data, len, g, err);
    if (rc) return rc;
    try {
        recognise(g, net);
    } catch (const Fail &f) {
        err = f.msg;
        return f.code;
    }
    return GCDR_OK;
}

std::string describe_net(const NetW &n) {
    std::ostringstream o;
    o << "{\"cin\":" << n.cin << ",\"channels\":[" << n.c1 << "," << n.c2 << "," << n.c3 << "," << n.c4 << ","
      << n.c5 << "],\"blocks\":[";
    for (int i = 0; i < 4; i++) {
        const BlockW &b = n.blk[i];
        o << (i ? "," : "") << "{\"c\":" << b.norm2.c << ",\"shifts\":[";
        for (int s = 0; s < 2; s++) {
            const ShiftW &w = s ? b.shift_b : b.shift_a;
            o << (s ? "," : "") << "{\"axis\":" << w.axis << ",\"ends\":[";
            for (size_t k = 0; k < w.ends.size(); k++) o << (k ? "," : "") << w.ends[k];
            o << "],\"offs\":[";
            for (size_t k = 0; k < w.offs.size(); k++) o << (k ? "," : "") << w.offs[k];
            o << "]}";
        }
        o << "],\"eps\":" << b.norm2.eps << "}";
    }
    o << "]}";
    return o.str();
}

}  // namespace gcdr
