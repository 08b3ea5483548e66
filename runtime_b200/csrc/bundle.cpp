// LFM2 bundle loader: config.json + model.safetensors as written by the
// reference's converters (tools/converters/src/minifield_converters/
// bundle.py:112-215), read on the host and uploaded into an mf_lfm2.
//
// Follows the reference loader's rules:
//  * config (crates/executor-core/src/lfm2/config.rs:121-170): hidden,
//    heads (alias num_heads), kv heads, conv_L_cache, vocab, layer_types
//    ("conv" / "full_attention"), rope_theta (or rope_parameters), norm_eps
//    and block_norm_eps (defaults to norm_eps), a tied embedding; the
//    effective FF width when block_auto_adjust_ff_dim is set
//    (config.rs:33-80: raw * 2 / 3, times the multiplier, truncated, up to a
//    multiple of block_multiple_of);
//  * tensor names and storage (crates/executor-core/src/lfm2/weights.rs:
//    750-833): a packed role is `<name>.codes` U8 [rows, k*bits/8] plus
//    `<name>.scales` F16 [rows, k/128]; a dense role is `<name>` in F32,
//    BF16 or F16; the weight format marker in `__metadata__.format`
//    (weights.rs:64-85);
//  * F16 decoding (crates/executor-core/src/loader.rs:405-420), rejection of
//    non-finite values and of the reserved INT8 code -128 (loader.rs:1156).
// Which packed format a role uses comes from its code width, as in
// check_packed_operands (crates/backend-cpu/src/packed.rs:202-245), so
// uniform and mixed bundles load the same way.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "backend_internal.h"
#include "mf_common.cuh"

namespace mf {
namespace {

// ------------------------------------------------------------------ JSON
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    bool integral = false;   // the number was written without fraction or exponent
    std::string s;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json *get(const char *key) const {
        if (kind != Obj) return nullptr;
        for (const auto &kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
  public:
    JsonParser(const char *p, size_t n) : p_(p), end_(p + n) {}
    bool parse(Json &out) {
        if (!value(out, 0)) return false;
        ws();
        return p_ == end_;
    }

  private:
    const char *p_, *end_;
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool lit(const char *w) {
        const size_t n = strlen(w);
        if ((size_t)(end_ - p_) < n || memcmp(p_, w, n)) return false;
        p_ += n;
        return true;
    }
    static void utf8(std::string &o, unsigned c) {
        if (c < 0x80) {
            o += (char)c;
        } else if (c < 0x800) {
            o += (char)(0xC0 | (c >> 6));
            o += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            o += (char)(0xE0 | (c >> 12));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        } else {
            o += (char)(0xF0 | (c >> 18));
            o += (char)(0x80 | ((c >> 12) & 0x3F));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(unsigned &v) {
        if (end_ - p_ < 4) return false;
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else return false;
        }
        return true;
    }
    bool string(std::string &o) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            const unsigned char c = (unsigned char)*p_++;
            if (c < 0x20) return false;
            if (c != '\\') {
                o += (char)c;
                continue;
            }
            if (p_ >= end_) return false;
            const char e = *p_++;
            switch (e) {
            case '"': o += '"'; break;
            case '\\': o += '\\'; break;
            case '/': o += '/'; break;
            case 'b': o += '\b'; break;
            case 'f': o += '\f'; break;
            case 'n': o += '\n'; break;
            case 'r': o += '\r'; break;
            case 't': o += '\t'; break;
            case 'u': {
                unsigned c1;
                if (!hex4(c1)) return false;
                if (c1 >= 0xD800 && c1 < 0xDC00) {
                    unsigned c2;
                    if (!lit("\\u") || !hex4(c2) || c2 < 0xDC00 || c2 >= 0xE000) return false;
                    c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                }
                utf8(o, c1);
                break;
            }
            default: return false;
            }
        }
        if (p_ >= end_) return false;
        ++p_;
        return true;
    }
    bool number(Json &o) {
        const char *s = p_;
        if (p_ < end_ && *p_ == '-') ++p_;
        bool digits = false, frac = false;
        while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_, digits = true;
        if (p_ < end_ && *p_ == '.') {
            frac = true;
            ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            frac = true;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (!digits) return false;
        o.kind = Json::Num;
        o.integral = !frac;
        o.num = strtod(std::string(s, p_ - s).c_str(), nullptr);
        return true;
    }
    bool value(Json &o, int depth) {
        if (depth > 64) return false;
        ws();
        if (p_ >= end_) return false;
        switch (*p_) {
        case '{': {
            ++p_;
            o.kind = Json::Obj;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            for (;;) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (p_ >= end_ || *p_++ != ':') return false;
                o.obj.emplace_back(std::move(k), Json());
                if (!value(o.obj.back().second, depth + 1)) return false;
                ws();
                if (p_ >= end_) return false;
                if (*p_ == ',') {
                    ++p_;
                    continue;
                }
                if (*p_ == '}') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        case '[': {
            ++p_;
            o.kind = Json::Arr;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            for (;;) {
                o.arr.emplace_back();
                if (!value(o.arr.back(), depth + 1)) return false;
                ws();
                if (p_ >= end_) return false;
                if (*p_ == ',') {
                    ++p_;
                    continue;
                }
                if (*p_ == ']') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        case '"': o.kind = Json::Str; return string(o.s);
        case 't': o.kind = Json::Bool; o.b = true; return lit("true");
        case 'f': o.kind = Json::Bool; o.b = false; return lit("false");
        case 'n': o.kind = Json::Null; return lit("null");
        default: return number(o);
        }
    }
};

bool read_file(const std::string &path, std::string &out, size_t limit) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    bool ok = fseek(f, 0, SEEK_END) == 0;
    const long n = ok ? ftell(f) : -1;
    ok = ok && n >= 0 && (size_t)n <= limit && fseek(f, 0, SEEK_SET) == 0;
    if (ok) {
        out.resize((size_t)n);
        ok = n == 0 || fread(&out[0], 1, (size_t)n, f) == (size_t)n;
    }
    fclose(f);
    return ok;
}

// ----------------------------------------------------------- safetensors
struct TensorInfo {
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t begin = 0, end = 0;
    uint64_t elements() const {
        uint64_t e = 1;
        for (uint64_t d : shape) e *= d;
        return e;
    }
};

struct SafeTensors {
    std::string blob;   // the whole file
    size_t data = 0;    // offset of the data section
    std::map<std::string, TensorInfo> tensors;
    std::map<std::string, std::string> metadata;
    const uint8_t *bytes(const TensorInfo &t) const {
        return reinterpret_cast<const uint8_t *>(blob.data()) + data + t.begin;
    }
};

size_t dtype_width(const std::string &d) {
    if (d == "F32") return 4;
    if (d == "F16" || d == "BF16") return 2;
    if (d == "U8" || d == "I8") return 1;
    return 0;
}

int32_t open_safetensors(const std::string &path, SafeTensors &st) {
    // The converter's limits are far above any model this loader serves;
    // 64 GiB bounds a host read.
    if (!read_file(path, st.blob, (size_t)64 << 30)) return fail(MF_INVALID_ARGUMENT, "cannot read model.safetensors");
    if (st.blob.size() < 8) return fail(MF_INVALID_LAYOUT, "safetensors file is truncated");
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | (uint8_t)st.blob[i];
    if (hlen > st.blob.size() - 8 || hlen > (100u << 20)) return fail(MF_INVALID_LAYOUT, "safetensors header length is out of range");
    Json h;
    if (!JsonParser(st.blob.data() + 8, hlen).parse(h) || h.kind != Json::Obj)
        return fail(MF_INVALID_LAYOUT, "safetensors header is not a JSON object");
    st.data = 8 + hlen;
    const uint64_t data_bytes = st.blob.size() - st.data;
    for (const auto &kv : h.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind != Json::Obj) return fail(MF_INVALID_LAYOUT, "safetensors metadata must be a map");
            for (const auto &m : kv.second.obj) {
                if (m.second.kind != Json::Str) return fail(MF_INVALID_LAYOUT, "safetensors metadata values must be strings");
                st.metadata[m.first] = m.second.s;
            }
            continue;
        }
        const Json &t = kv.second;
        const Json *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
        if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !off || off->kind != Json::Arr ||
            off->arr.size() != 2)
            return fail(MF_INVALID_LAYOUT, "safetensors tensor entry is malformed");
        TensorInfo ti;
        ti.dtype = dt->s;
        for (const Json &d : sh->arr) {
            if (d.kind != Json::Num || !d.integral || d.num < 0 || d.num > 9.0e15)
                return fail(MF_INVALID_LAYOUT, "safetensors shape must hold non-negative integers");
            ti.shape.push_back((uint64_t)d.num);
        }
        for (const Json &o : off->arr)
            if (o.kind != Json::Num || !o.integral || o.num < 0 || o.num > 9.0e15)
                return fail(MF_INVALID_LAYOUT, "safetensors data offsets must be non-negative integers");
        ti.begin = (uint64_t)off->arr[0].num;
        ti.end = (uint64_t)off->arr[1].num;
        const size_t w = dtype_width(ti.dtype);
        if (!w) return fail(MF_INVALID_DTYPE, "safetensors tensor dtype is not supported");
        if (ti.end < ti.begin || ti.end > data_bytes || ti.end - ti.begin != ti.elements() * w)
            return fail(MF_OUT_OF_BOUNDS, "safetensors tensor bytes are out of range");
        st.tensors[kv.first] = ti;
    }
    return MF_OK;
}

// crates/executor-core/src/loader.rs:405-420: IEEE half to f32.
float f16_to_f32(uint16_t bits) {
    const uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    const uint32_t exponent = (bits >> 10) & 0x1Fu;
    const uint32_t mantissa = bits & 0x03FFu;
    float v;
    if (exponent == 0) {
        v = (float)mantissa * 0x1p-24f;
    } else {
        const uint32_t b = exponent == 31 ? (0x7F800000u | (mantissa << 13)) : (((exponent + 112) << 23) | (mantissa << 13));
        memcpy(&v, &b, 4);
    }
    uint32_t out;
    memcpy(&out, &v, 4);
    out |= sign;
    memcpy(&v, &out, 4);
    return v;
}

// A dense tensor's values as F32 (F32, BF16, F16 storage); non-finite
// values are rejected.
int32_t decode_f32(const SafeTensors &st, const TensorInfo &t, std::vector<float> &out) {
    const uint64_t n = t.elements();
    out.resize(n);
    const uint8_t *p = st.bytes(t);
    if (t.dtype == "F32") {
        memcpy(out.data(), p, n * 4);
    } else if (t.dtype == "BF16") {
        for (uint64_t i = 0; i < n; ++i) {
            const uint32_t b = (uint32_t)(p[2 * i] | (p[2 * i + 1] << 8)) << 16;
            memcpy(&out[i], &b, 4);
        }
    } else if (t.dtype == "F16") {
        for (uint64_t i = 0; i < n; ++i) out[i] = f16_to_f32((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
    } else {
        return fail(MF_INVALID_DTYPE, "dense LFM2 tensor must be F32, BF16 or F16");
    }
    for (float v : out)
        if (!std::isfinite(v)) return fail(MF_BACKEND_FAILURE, "LFM2 tensor holds a non-finite value");
    return MF_OK;
}

// --------------------------------------------------------------- config
bool as_u32(const Json *v, uint32_t &out) {
    if (!v || v->kind != Json::Num || !v->integral || v->num <= 0 || v->num > 4294967295.0) return false;
    out = (uint32_t)v->num;
    return true;
}

bool as_pos_f32(const Json *v, float &out) {
    if (!v || v->kind != Json::Num) return false;
    out = (float)v->num;
    return std::isfinite(out) && out > 0.0f;
}

int32_t parse_config(const Json &c, mf_lfm2_config &cfg, std::vector<int32_t> &kinds) {
    if (c.kind != Json::Obj) return fail(MF_INVALID_ARGUMENT, "config.json must be an object");
    const Json *mt = c.get("model_type");
    if (!mt || mt->kind != Json::Str || mt->s != "lfm2") return fail(MF_UNSUPPORTED, "only model_type lfm2 is supported");
    memset(&cfg, 0, sizeof(cfg));
    uint32_t raw_ff = 0, count = 0;
    if (!as_u32(c.get("hidden_size"), cfg.hidden)) return fail(MF_INVALID_ARGUMENT, "hidden_size");
    if (!as_u32(c.get("intermediate_size"), raw_ff)) return fail(MF_INVALID_ARGUMENT, "intermediate_size");
    const Json *heads = c.get("num_attention_heads");
    if (!heads) heads = c.get("num_heads");
    if (!as_u32(heads, cfg.q_heads)) return fail(MF_INVALID_ARGUMENT, "num_attention_heads");
    if (!as_u32(c.get("num_key_value_heads"), cfg.kv_heads)) return fail(MF_INVALID_ARGUMENT, "num_key_value_heads");
    if (!as_u32(c.get("conv_L_cache"), cfg.conv_width)) return fail(MF_INVALID_ARGUMENT, "conv_L_cache");
    if (!as_u32(c.get("vocab_size"), cfg.vocab)) return fail(MF_INVALID_ARGUMENT, "vocab_size");
    if (!as_u32(c.get("num_hidden_layers"), count)) return fail(MF_INVALID_ARGUMENT, "num_hidden_layers");
    // config.rs:33-80
    cfg.intermediate = raw_ff;
    const Json *adj = c.get("block_auto_adjust_ff_dim");
    if (adj && adj->kind == Json::Bool && adj->b) {
        const Json *mul = c.get("block_ffn_dim_multiplier");
        uint32_t multiple = 0;
        if (!mul || mul->kind != Json::Num || !std::isfinite(mul->num) || mul->num <= 0.0)
            return fail(MF_INVALID_ARGUMENT, "block_ffn_dim_multiplier must be finite and positive");
        if (!as_u32(c.get("block_multiple_of"), multiple)) return fail(MF_INVALID_ARGUMENT, "block_multiple_of");
        const double scaled = (double)((uint64_t)raw_ff * 2 / 3) * mul->num;
        if (!std::isfinite(scaled) || scaled > 4294967295.0) return fail(MF_OVERFLOW, "effective FF dimension exceeds u32");
        const uint64_t t = (uint64_t)std::trunc(scaled);
        const uint64_t ff = (t + multiple - 1) / multiple * multiple;
        if (ff == 0 || ff > 0xFFFFFFFFull) return fail(MF_OVERFLOW, "effective FF dimension exceeds u32");
        cfg.intermediate = (uint32_t)ff;
    }
    const Json *types = c.get("layer_types");
    if (!types || types->kind != Json::Arr || types->arr.size() != count)
        return fail(MF_INVALID_ARGUMENT, "layer_types length differs from num_hidden_layers");
    kinds.clear();
    for (const Json &t : types->arr) {
        if (t.kind == Json::Str && t.s == "conv") kinds.push_back(MF_LAYER_CONV);
        else if (t.kind == Json::Str && t.s == "full_attention") kinds.push_back(MF_LAYER_ATTENTION);
        else return fail(MF_UNSUPPORTED, "unsupported LFM2 layer type");
    }
    cfg.n_layers = count;
    const Json *rope = c.get("rope_parameters");
    const Json *theta = rope && rope->kind == Json::Obj ? rope->get("rope_theta") : c.get("rope_theta");
    if (!as_pos_f32(theta, cfg.rope_theta)) return fail(MF_INVALID_ARGUMENT, "rope_theta");
    if (!as_pos_f32(c.get("norm_eps"), cfg.norm_eps)) return fail(MF_INVALID_ARGUMENT, "norm_eps");
    cfg.block_eps = cfg.norm_eps;
    if (c.get("block_norm_eps") && !as_pos_f32(c.get("block_norm_eps"), cfg.block_eps))
        return fail(MF_INVALID_ARGUMENT, "block_norm_eps");
    const Json *tie = c.get("tie_embedding");
    if (!tie) tie = c.get("tie_word_embeddings");
    if (!tie || tie->kind != Json::Bool || !tie->b) return fail(MF_INVALID_TIE, "only tied embedding models are supported");
    if (cfg.hidden % cfg.q_heads || cfg.q_heads % cfg.kv_heads || (cfg.hidden / cfg.q_heads) % 2)
        return fail(MF_INVALID_SHAPE, "invalid attention dimensions or odd split-half RoPE width");
    cfg.head_dim = cfg.hidden / cfg.q_heads;
    return MF_OK;
}

// ------------------------------------------------------------- weights
struct Uploads {
    mf_backend *b;
    std::vector<mf_buffer *> bufs;
    ~Uploads() {
        for (mf_buffer *x : bufs) mf_buffer_release(b, x);
    }
};

// Role `name` of dense shape [rows, cols]: packed (`.codes` + `.scales`)
// or dense.
int32_t load_matrix(const SafeTensors &st, Uploads &up, const std::string &name, uint64_t rows, uint64_t cols,
                    mf_lfm2_weight &out) {
    memset(&out, 0, sizeof(out));
    auto codes = st.tensors.find(name + ".codes");
    if (codes != st.tensors.end()) {
        auto scales = st.tensors.find(name + ".scales");
        if (scales == st.tensors.end()) return fail(MF_MISSING_REQUIRED_TENSOR, "packed role is missing its scales");
        const TensorInfo &c = codes->second, &s = scales->second;
        if (c.dtype != "U8" || c.shape.size() != 2 || s.shape.size() != 2)
            return fail(MF_INVALID_DTYPE, "packed codes must be U8 of rank two");
        if (c.shape[0] != rows || s.shape[0] != rows || cols % 128 || s.shape[1] * 128 != cols)
            return fail(MF_INVALID_SHAPE, "packed role has the wrong shape");
        const uint64_t cw = c.shape[1];
        if (cw != cols / 4 && cw != cols / 2 && cw != cols) return fail(MF_INVALID_SHAPE, "packed code width matches no format");
        if (cw == cols && memchr(st.bytes(c), 0x80, c.end - c.begin))
            return fail(MF_INVALID_ARGUMENT, "INT8 code -128 is reserved");   // loader.rs:1156
        std::vector<float> sc;
        int32_t e = decode_f32(st, s, sc);
        if (e) return e;
        uint64_t cshape[2] = {rows, cw}, sshape[2] = {rows, cols / 128};
        mf_buffer *cb = nullptr, *sb = nullptr;
        if ((e = mf_upload_u8(up.b, cshape, 2, st.bytes(c), MF_CLASS_WEIGHT, &cb))) return e;
        up.bufs.push_back(cb);
        if ((e = mf_upload_f32(up.b, sshape, 2, sc.data(), MF_CLASS_WEIGHT, &sb))) return e;
        up.bufs.push_back(sb);
        out.codes = cb;
        out.scales = sb;
        return MF_OK;
    }
    auto dense = st.tensors.find(name);
    if (dense == st.tensors.end()) return fail(MF_MISSING_REQUIRED_TENSOR, "required tensor is missing");
    const TensorInfo &t = dense->second;
    if (t.elements() != rows * cols || t.shape.empty() || t.shape[0] != rows)
        return fail(MF_INVALID_SHAPE, "dense role has the wrong shape");
    std::vector<float> v;
    int32_t e = decode_f32(st, t, v);
    if (e) return e;
    uint64_t shape[2] = {rows, cols};
    mf_buffer *db = nullptr;
    if ((e = mf_upload_f32(up.b, shape, 2, v.data(), MF_CLASS_WEIGHT, &db))) return e;
    up.bufs.push_back(db);
    out.dense = db;
    return MF_OK;
}

int32_t load_vector(const SafeTensors &st, Uploads &up, const std::string &name, uint64_t n, const mf_buffer **out) {
    auto it = st.tensors.find(name);
    if (it == st.tensors.end()) return fail(MF_MISSING_REQUIRED_TENSOR, "required tensor is missing");
    if (it->second.elements() != n) return fail(MF_INVALID_SHAPE, "vector role has the wrong size");
    std::vector<float> v;
    int32_t e = decode_f32(st, it->second, v);
    if (e) return e;
    uint64_t shape[1] = {n};
    mf_buffer *buf = nullptr;
    if ((e = mf_upload_f32(up.b, shape, 1, v.data(), MF_CLASS_WEIGHT, &buf))) return e;
    up.bufs.push_back(buf);
    *out = buf;
    return MF_OK;
}

int32_t read_config(const std::string &dir, mf_lfm2_config &cfg, std::vector<int32_t> &kinds) {
    std::string text;
    if (!read_file(dir + "/config.json", text, 1 << 20)) return fail(MF_INVALID_ARGUMENT, "cannot read config.json");
    Json c;
    if (!JsonParser(text.data(), text.size()).parse(c)) return fail(MF_INVALID_ARGUMENT, "config.json is not valid JSON");
    return parse_config(c, cfg, kinds);
}

int32_t check_format_marker(const SafeTensors &st) {
    // weights.rs:74-85
    auto f = st.metadata.find("format");
    if (f == st.metadata.end() || f->second == "pt") return MF_OK;
    static const char *known[] = {"minifield.ternary.v1", "minifield.nf4.v1", "minifield.int8.v1", "minifield.mixed.v1"};
    for (const char *k : known)
        if (f->second == k) return MF_OK;
    return fail(MF_UNSUPPORTED, "unrecognized LFM2 weight format");
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" {

int32_t mf_bundle_config(const char *directory, mf_lfm2_config *out, int32_t *layer_kinds, uint32_t max_layers,
                         char *format, uint64_t format_len) {
    if (!directory || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    std::vector<int32_t> kinds;
    int32_t st = read_config(directory, *out, kinds);
    if (st) return st;
    if (layer_kinds) {
        if (max_layers < kinds.size()) return fail(MF_RESOURCE_LIMIT, "layer kind buffer is too small");
        memcpy(layer_kinds, kinds.data(), kinds.size() * sizeof(int32_t));
    }
    out->layer_kinds = nullptr;
    if (format && format_len) {
        SafeTensors tensors;
        if ((st = open_safetensors(std::string(directory) + "/model.safetensors", tensors))) return st;
        if ((st = check_format_marker(tensors))) return st;
        auto f = tensors.metadata.find("format");
        const std::string marker = f == tensors.metadata.end() ? "pt" : f->second;
        snprintf(format, format_len, "%s", marker.c_str());
    }
    return MF_OK;
}

int32_t mf_lfm2_load_bundle(mf_backend *b, const char *directory, uint64_t max_tokens, mf_lfm2 **out) {
    if (!b || !directory || !out) return fail(MF_INVALID_ARGUMENT, "null argument");
    if (max_tokens == 0) return fail(MF_INVALID_ARGUMENT, "context capacity must be positive");
    mf_lfm2_config cfg;
    std::vector<int32_t> kinds;
    int32_t st = read_config(directory, cfg, kinds);
    if (st) return st;
    cfg.layer_kinds = kinds.data();
    cfg.max_tokens = max_tokens;
    SafeTensors tensors;
    if ((st = open_safetensors(std::string(directory) + "/model.safetensors", tensors))) return st;
    if ((st = check_format_marker(tensors))) return st;
    Uploads up{b, {}};
    const uint64_t h = cfg.hidden, f = cfg.intermediate, kvw = (uint64_t)cfg.kv_heads * cfg.head_dim;
    mf_lfm2_weight emb;
    const mf_buffer *emb_norm = nullptr;
    if ((st = load_matrix(tensors, up, "model.embed_tokens.weight", cfg.vocab, h, emb))) return st;
    if ((st = load_vector(tensors, up, "model.embedding_norm.weight", h, &emb_norm))) return st;
    std::vector<mf_lfm2_layer> layers(cfg.n_layers);
    for (uint32_t i = 0; i < cfg.n_layers; ++i) {
        mf_lfm2_layer &L = layers[i];
        memset(&L, 0, sizeof(L));
        const std::string p = "model.layers." + std::to_string(i);
        if (kinds[i] == MF_LAYER_CONV) {
            if ((st = load_matrix(tensors, up, p + ".conv.in_proj.weight", 3 * h, h, L.in_proj))) return st;
            if ((st = load_matrix(tensors, up, p + ".conv.out_proj.weight", h, h, L.out_proj))) return st;
            if ((st = load_vector(tensors, up, p + ".conv.conv.weight", h * cfg.conv_width, &L.conv_kernel))) return st;
        } else {
            if ((st = load_matrix(tensors, up, p + ".self_attn.q_proj.weight", h, h, L.q))) return st;
            if ((st = load_matrix(tensors, up, p + ".self_attn.k_proj.weight", kvw, h, L.k))) return st;
            if ((st = load_matrix(tensors, up, p + ".self_attn.v_proj.weight", kvw, h, L.v))) return st;
            if ((st = load_matrix(tensors, up, p + ".self_attn.out_proj.weight", h, h, L.o))) return st;
            if ((st = load_vector(tensors, up, p + ".self_attn.q_layernorm.weight", cfg.head_dim, &L.q_norm))) return st;
            if ((st = load_vector(tensors, up, p + ".self_attn.k_layernorm.weight", cfg.head_dim, &L.k_norm))) return st;
        }
        if ((st = load_matrix(tensors, up, p + ".feed_forward.w1.weight", f, h, L.w1))) return st;
        if ((st = load_matrix(tensors, up, p + ".feed_forward.w2.weight", h, f, L.w2))) return st;
        if ((st = load_matrix(tensors, up, p + ".feed_forward.w3.weight", f, h, L.w3))) return st;
        if ((st = load_vector(tensors, up, p + ".ffn_norm.weight", h, &L.ffn_norm))) return st;
        if ((st = load_vector(tensors, up, p + ".operator_norm.weight", h, &L.operator_norm))) return st;
    }
    mf_lfm2 *m = nullptr;
    if ((st = mf_lfm2_create(b, &cfg, &emb, emb_norm, layers.data(), &m))) return st;
    // The model owns the uploaded weights from here on.
    lfm2_adopt_buffers(m, up.bufs);
    up.bufs.clear();
    *out = m;
    return MF_OK;
}

}  // extern "C"
