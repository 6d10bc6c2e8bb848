// ssla_weights.cpp -- meta.json / weights.npz reader and load-time reshape.
#include "ssla_weights.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace ssla {
namespace {

std::string slurp(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// Flat JSON lookups (meta.json is a flat object written by json.dump).
std::size_t json_value_pos(const std::string& s, const std::string& key) {
    const std::string k = "\"" + key + "\"";
    std::size_t p = s.find(k);
    if (p == std::string::npos) return std::string::npos;
    p = s.find(':', p + k.size());
    if (p == std::string::npos) return std::string::npos;
    ++p;
    while (p < s.size() && (s[p] == ' ' || s[p] == '\t' || s[p] == '\n' || s[p] == '\r')) ++p;
    return p;
}

int json_int(const std::string& s, const std::string& key) {
    const std::size_t p = json_value_pos(s, key);
    if (p == std::string::npos) return 0;
    return std::atoi(s.c_str() + p);
}

std::string json_str(const std::string& s, const std::string& key) {
    std::size_t p = json_value_pos(s, key);
    if (p == std::string::npos || s[p] != '"') return "";
    const std::size_t q = s.find('"', p + 1);
    if (q == std::string::npos) return "";
    return s.substr(p + 1, q - p - 1);
}

template <typename T>
T rd(const std::string& buf, std::size_t off) {
    if (off + sizeof(T) > buf.size()) throw std::runtime_error("npz: truncated");
    T v;
    std::memcpy(&v, buf.data() + off, sizeof(T));
    return v;
}

// .npy payload: magic, version, little-endian header length, python-dict
// header with 'descr', 'fortran_order', 'shape'; float32 C-order only.
NpyArray parse_npy(const char* p, std::size_t n, const std::string& name) {
    if (n < 10 || std::memcmp(p, "\x93NUMPY", 6) != 0)
        throw std::runtime_error("npz: " + name + " is not a .npy entry");
    const unsigned major = static_cast<unsigned char>(p[6]);
    std::size_t hlen, hstart;
    if (major == 1) {
        std::uint16_t h16;
        std::memcpy(&h16, p + 8, 2);
        hlen = h16; hstart = 10;
    } else {
        std::uint32_t h32;
        std::memcpy(&h32, p + 8, 4);
        hlen = h32; hstart = 12;
    }
    if (hstart + hlen > n) throw std::runtime_error("npz: " + name + " header overflow");
    const std::string hdr(p + hstart, hlen);
    if (hdr.find("'descr': '<f4'") == std::string::npos &&
        hdr.find("'descr':'<f4'") == std::string::npos)
        throw std::runtime_error("npz: " + name + " is not little-endian float32");
    if (hdr.find("'fortran_order': True") != std::string::npos)
        throw std::runtime_error("npz: " + name + " is Fortran-ordered");
    NpyArray a;
    const std::size_t sp = hdr.find("'shape'");
    const std::size_t lp = hdr.find('(', sp), rp = hdr.find(')', lp);
    if (sp == std::string::npos || lp == std::string::npos || rp == std::string::npos)
        throw std::runtime_error("npz: " + name + " has no shape");
    std::size_t count = 1;
    std::string dims = hdr.substr(lp + 1, rp - lp - 1);
    std::size_t q = 0;
    while (q < dims.size()) {
        while (q < dims.size() && (dims[q] == ' ' || dims[q] == ',')) ++q;
        if (q >= dims.size()) break;
        const std::size_t d = std::strtoull(dims.c_str() + q, nullptr, 10);
        a.shape.push_back(d);
        count *= d;
        while (q < dims.size() && dims[q] != ',') ++q;
    }
    const std::size_t off = hstart + hlen;
    if (off + count * 4 > n) throw std::runtime_error("npz: " + name + " payload truncated");
    a.data.resize(count);
    if (count) std::memcpy(a.data.data(), p + off, count * 4);
    return a;
}

const NpyArray& need(const std::map<std::string, NpyArray>& m, const std::string& k) {
    auto it = m.find(k);
    if (it == m.end()) throw std::runtime_error("weights.npz: missing tensor " + k);
    return it->second;
}

const NpyArray* maybe(const std::map<std::string, NpyArray>& m, const std::string& k) {
    auto it = m.find(k);
    return it == m.end() ? nullptr : &it->second;
}

// C = B (b_out x b_in) @ A (b_in x a_in), k-loop in order with fmaf
// (vendor/openeva/prim/matmul.h:24-41).
void mm(const float* B, int b_out, int b_in, const float* A, int a_in, float* C) {
    for (int o = 0; o < b_out; ++o) {
        float* cr = C + static_cast<std::size_t>(o) * a_in;
        for (int i = 0; i < a_in; ++i) cr[i] = 0.0f;
        for (int k = 0; k < b_in; ++k) {
            const float bv = B[static_cast<std::size_t>(o) * b_in + k];
            const float* ar = A + static_cast<std::size_t>(k) * a_in;
            for (int i = 0; i < a_in; ++i) cr[i] = std::fmaf(bv, ar[i], cr[i]);
        }
    }
}

// src/ssla_kernels.cpp:73-153 load_layer, emitted in device layouts.
void build_layer(const std::map<std::string, NpyArray>& W, const std::string& prefix,
                 int IN, int OUT, HostLayer& L) {
    const NpyArray& win = need(W, prefix + "/W_in_cat");
    const NpyArray& wout = need(W, prefix + "/W_out_cat");
    if (win.shape.size() != 2 || wout.shape.size() != 2)
        throw std::runtime_error(prefix + ": W_*_cat must be 2-D");
    if (static_cast<int>(win.shape[0]) != IN || static_cast<int>(wout.shape[1]) != OUT)
        throw std::runtime_error(prefix + ": W_*_cat dims do not match SSLA-S");
    const int win_cols = static_cast<int>(win.shape[1]);
    const int wout_rows = static_cast<int>(wout.shape[0]);
    if (win_cols % OUT || wout_rows % OUT)
        throw std::runtime_error(prefix + ": W_*_cat not a multiple of out_dim");
    const int npi = win_cols / OUT, npo = wout_rows / OUT;
    const int A = npi > npo ? npi : npo;
    if (A != 1 && A != 9) throw std::runtime_error(prefix + ": patch positions must be 1 or 9");
    const NpyArray* mats[4] = {&need(W, prefix + "/q_proj/weight"), &need(W, prefix + "/v_proj/weight"),
                               &need(W, prefix + "/g_proj/weight"), &need(W, prefix + "/o_proj/weight")};
    for (auto* m : mats)
        if (m->data.size() != static_cast<std::size_t>(OUT) * OUT)
            throw std::runtime_error(prefix + ": projection shape");
    L.in_dim = IN; L.out_dim = OUT; L.A = A;
    L.qvgT.assign(static_cast<std::size_t>(A) * IN * 3 * OUT, 0.0f);
    L.goWT.assign(static_cast<std::size_t>(A) * OUT * OUT, 0.0f);
    std::vector<float> scatter(static_cast<std::size_t>(OUT) * IN), gather(static_cast<std::size_t>(OUT) * OUT);
    std::vector<float> part(static_cast<std::size_t>(OUT) * IN), gow(static_cast<std::size_t>(OUT) * OUT);
    for (int p = 0; p < A; ++p) {
        const int pin = (npi == 1) ? 0 : p, pout = (npo == 1) ? 0 : p;
        for (int d = 0; d < OUT; ++d)
            for (int c = 0; c < IN; ++c)
                scatter[static_cast<std::size_t>(d) * IN + c] =
                    win.data[static_cast<std::size_t>(c) * win_cols + pin * OUT + d];
        for (int i = 0; i < OUT; ++i)
            for (int j = 0; j < OUT; ++j)
                gather[static_cast<std::size_t>(i) * OUT + j] =
                    wout.data[static_cast<std::size_t>(pout * OUT + j) * OUT + i];
        for (int which = 0; which < 3; ++which) {        // q, v, g rows
            mm(mats[which]->data.data(), OUT, OUT, scatter.data(), IN, part.data());
            for (int o = 0; o < OUT; ++o)
                for (int i = 0; i < IN; ++i)
                    L.qvgT[(static_cast<std::size_t>(p) * IN + i) * 3 * OUT + which * OUT + o] =
                        part[static_cast<std::size_t>(o) * IN + i];
        }
        mm(gather.data(), OUT, OUT, mats[3]->data.data(), OUT, gow.data());
        for (int o = 0; o < OUT; ++o)
            for (int i = 0; i < OUT; ++i)
                L.goWT[(static_cast<std::size_t>(p) * OUT + i) * OUT + o] =
                    gow[static_cast<std::size_t>(o) * OUT + i];
    }
    if (const NpyArray* ip = maybe(W, prefix + "/input_proj/weight")) {
        if (ip->data.size() != static_cast<std::size_t>(OUT) * IN)
            throw std::runtime_error(prefix + ": input_proj shape");
        L.ipT.assign(static_cast<std::size_t>(IN) * OUT, 0.0f);
        for (int o = 0; o < OUT; ++o)
            for (int i = 0; i < IN; ++i)
                L.ipT[static_cast<std::size_t>(i) * OUT + o] = ip->data[static_cast<std::size_t>(o) * IN + i];
    } else if (IN != OUT) {
        throw std::runtime_error(prefix + ": input_proj required when in_dim != out_dim");
    }
    L.gamma = need(W, prefix + "/norm/weight").data;
    L.beta = need(W, prefix + "/norm/bias").data;
    if (L.gamma.size() != static_cast<std::size_t>(OUT) || L.beta.size() != static_cast<std::size_t>(OUT))
        throw std::runtime_error(prefix + ": norm shape");
}

// vendor/openeva/prim/bn_fusion.h:19-60 (fuse_bn + fold_bn_into_weight_2d),
// written transposed: WT[i][o].
void fold_conv_bn(const std::map<std::string, NpyArray>& W, const std::string& conv,
                  const std::string& bn, int out_c, int in_c,
                  std::vector<float>& WT, std::vector<float>& b) {
    const NpyArray& w = need(W, conv + "/weight");
    if (w.data.size() != static_cast<std::size_t>(out_c) * in_c)
        throw std::runtime_error(conv + ": conv weight shape");
    const NpyArray* cb = maybe(W, conv + "/bias");
    const NpyArray& g = need(W, bn + "/weight");
    const NpyArray& bb = need(W, bn + "/bias");
    const NpyArray& mu = need(W, bn + "/running_mean");
    const NpyArray& var = need(W, bn + "/running_var");
    WT.assign(static_cast<std::size_t>(in_c) * out_c, 0.0f);
    b.assign(out_c, 0.0f);
    for (int o = 0; o < out_c; ++o) {
        const float inv = 1.0f / std::sqrt(var.data[o] + 1e-5f);
        const float s = g.data[o] * inv;
        const float shift = bb.data[o] - (g.data[o] * mu.data[o]) * inv;
        for (int i = 0; i < in_c; ++i)
            WT[static_cast<std::size_t>(i) * out_c + o] = w.data[static_cast<std::size_t>(o) * in_c + i] * s;
        const float bc = cb ? cb->data[o] : 0.0f;
        b[o] = std::fmaf(bc, s, shift);
    }
}

void transpose_pred(const NpyArray& w, int out_c, int in_c, std::vector<float>& WT,
                    const std::string& name) {
    if (w.data.size() != static_cast<std::size_t>(out_c) * in_c)
        throw std::runtime_error(name + ": pred weight shape");
    WT.assign(static_cast<std::size_t>(in_c) * out_c, 0.0f);
    for (int o = 0; o < out_c; ++o)
        for (int i = 0; i < in_c; ++i)
            WT[static_cast<std::size_t>(i) * out_c + o] = w.data[static_cast<std::size_t>(o) * in_c + i];
}

}  // namespace

Meta read_meta(const std::string& dir) {
    const std::string s = slurp(dir + "/meta.json");
    Meta m;
    m.model = json_str(s, "model");
    m.height = json_int(s, "height");
    m.width = json_int(s, "width");
    m.num_classes = json_int(s, "num_classes");
    m.tdrop_window = json_int(s, "ssla_tdrop_window");
    return m;
}

// Zip reader over the central directory (handles numpy's ZIP64 entries);
// stored (method 0) entries only, as numpy.savez writes them.
std::map<std::string, NpyArray> read_npz(const std::string& path) {
    const std::string buf = slurp(path);
    if (buf.size() < 22) throw std::runtime_error("npz: too small");
    std::size_t eocd = std::string::npos;
    for (std::size_t i = buf.size() - 22 + 1; i-- > 0;) {
        if (rd<std::uint32_t>(buf, i) == 0x06054b50u) { eocd = i; break; }
        if (buf.size() - i > 22 + 65535) break;
    }
    if (eocd == std::string::npos) throw std::runtime_error("npz: no end-of-central-directory");
    std::uint64_t n_entries = rd<std::uint16_t>(buf, eocd + 10);
    std::uint64_t cd_off = rd<std::uint32_t>(buf, eocd + 16);
    if (cd_off == 0xFFFFFFFFu || n_entries == 0xFFFFu) {
        if (eocd < 20 || rd<std::uint32_t>(buf, eocd - 20) != 0x07064b50u)
            throw std::runtime_error("npz: missing zip64 locator");
        const std::uint64_t z64 = rd<std::uint64_t>(buf, eocd - 20 + 8);
        if (rd<std::uint32_t>(buf, z64) != 0x06064b50u) throw std::runtime_error("npz: bad zip64 record");
        n_entries = rd<std::uint64_t>(buf, z64 + 32);
        cd_off = rd<std::uint64_t>(buf, z64 + 48);
    }
    std::map<std::string, NpyArray> out;
    std::size_t p = cd_off;
    for (std::uint64_t e = 0; e < n_entries; ++e) {
        if (rd<std::uint32_t>(buf, p) != 0x02014b50u) throw std::runtime_error("npz: bad central entry");
        const std::uint16_t method = rd<std::uint16_t>(buf, p + 10);
        std::uint64_t csize = rd<std::uint32_t>(buf, p + 20);
        std::uint64_t usize = rd<std::uint32_t>(buf, p + 24);
        const std::uint16_t nlen = rd<std::uint16_t>(buf, p + 28);
        const std::uint16_t xlen = rd<std::uint16_t>(buf, p + 30);
        const std::uint16_t clen = rd<std::uint16_t>(buf, p + 32);
        std::uint64_t loff = rd<std::uint32_t>(buf, p + 42);
        if (p + 46 + nlen > buf.size()) throw std::runtime_error("npz: truncated name");
        std::string name(buf.data() + p + 46, nlen);
        std::size_t x = p + 46 + nlen, xend = x + xlen;
        while (x + 4 <= xend) {
            const std::uint16_t id = rd<std::uint16_t>(buf, x), sz = rd<std::uint16_t>(buf, x + 2);
            if (id == 0x0001) {
                std::size_t q = x + 4;
                if (usize == 0xFFFFFFFFu) { usize = rd<std::uint64_t>(buf, q); q += 8; }
                if (csize == 0xFFFFFFFFu) { csize = rd<std::uint64_t>(buf, q); q += 8; }
                if (loff == 0xFFFFFFFFu) { loff = rd<std::uint64_t>(buf, q); q += 8; }
            }
            x += 4 + sz;
        }
        if (method != 0) throw std::runtime_error("npz: " + name + " is compressed (use numpy.savez)");
        if (rd<std::uint32_t>(buf, loff) != 0x04034b50u) throw std::runtime_error("npz: bad local header");
        const std::size_t data = loff + 30 + rd<std::uint16_t>(buf, loff + 26) + rd<std::uint16_t>(buf, loff + 28);
        if (data + csize > buf.size()) throw std::runtime_error("npz: entry past end");
        if (name.size() > 4 && name.compare(name.size() - 4, 4, ".npy") == 0) name.resize(name.size() - 4);
        out[name] = parse_npy(buf.data() + data, static_cast<std::size_t>(csize), name);
        p = x > xend ? x : xend;
        p += clen;
    }
    return out;
}

HostModel load_model(const std::string& dir) {
    HostModel M;
    M.meta = read_meta(dir);
    if (M.meta.model != "ssla_s_yolox_det")
        throw std::runtime_error("meta.json: model must be ssla_s_yolox_det, got '" + M.meta.model + "'");
    if (M.meta.height <= 0) M.meta.height = 240;             // src/ssla_kernels.cpp:167-170
    if (M.meta.width <= 0) M.meta.width = 304;
    if (M.meta.num_classes <= 0) M.meta.num_classes = 2;
    if (M.meta.tdrop_window <= 0) M.meta.tdrop_window = 4;
    if (M.meta.height % 8 || M.meta.width % 8)
        throw std::runtime_error("sensor height and width must be multiples of 8");
    if (M.meta.num_classes > 16) throw std::runtime_error("at most 16 classes supported");
    const auto W = read_npz(dir + "/weights.npz");
    // Layer indices as exported (src/ssla_kernels.cpp:179-198): the eight keys
    // layers/<i>/W_in_cat, sorted.
    std::vector<int> idx;
    for (const auto& kv : W) {
        const std::string& k = kv.first;
        if (k.rfind("layers/", 0) != 0) continue;
        const std::size_t sl = k.find('/', 7);
        if (sl == std::string::npos || k.substr(sl + 1) != "W_in_cat") continue;
        idx.push_back(std::atoi(k.c_str() + 7));
    }
    std::sort(idx.begin(), idx.end());
    if (idx.size() != 8) throw std::runtime_error("weights.npz: expected 8 SSLA layers");
    static const int kDims[8][2] = {{2, 12}, {12, 12}, {12, 24}, {24, 24},
                                    {24, 48}, {48, 48}, {48, 96}, {96, 96}};
    for (int l = 0; l < 8; ++l)
        build_layer(W, "layers/" + std::to_string(idx[l]), kDims[l][0], kDims[l][1], M.layers[l]);
    if (!maybe(W, "head/cls_convs/0/0/weight")) throw std::runtime_error("weights.npz: no head level 0");
    if (maybe(W, "head/cls_convs/1/0/weight"))
        throw std::runtime_error("weights.npz: multi-level heads are not supported (one level at stage 3)");
    HostHead& H = M.head;
    H.ncls = M.meta.num_classes;
    fold_conv_bn(W, "head/cls_convs/0/0", "head/cls_convs/0/1", 96, 96, H.cls_convT, H.cls_conv_b);
    fold_conv_bn(W, "head/reg_convs/0/0", "head/reg_convs/0/1", 96, 96, H.reg_convT, H.reg_conv_b);
    transpose_pred(need(W, "head/cls_preds/0/weight"), H.ncls, 96, H.cls_predT, "cls_preds");
    transpose_pred(need(W, "head/reg_preds/0/weight"), 4, 96, H.reg_predT, "reg_preds");
    transpose_pred(need(W, "head/obj_preds/0/weight"), 1, 96, H.obj_predT, "obj_preds");
    H.cls_pred_b = need(W, "head/cls_preds/0/bias").data;
    H.reg_pred_b = need(W, "head/reg_preds/0/bias").data;
    H.obj_pred_b = need(W, "head/obj_preds/0/bias").data;
    if (H.cls_pred_b.size() != static_cast<std::size_t>(H.ncls) || H.reg_pred_b.size() != 4 ||
        H.obj_pred_b.size() != 1)
        throw std::runtime_error("weights.npz: head bias shapes");
    return M;
}

}  // namespace ssla
