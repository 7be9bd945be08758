// checkpoint.cpp — trained weights into the kernels' weight blobs.
//
// A safetensors file is an 8-byte little-endian header length, a JSON header
// {"<name>": {"dtype": "F32", "shape": [..], "data_offsets": [begin, end]},
// "__metadata__": {..}} and the raw tensor bytes (offsets relative to the
// end of the header).  This is the format candle's
// VarBuilder::from_mmaped_safetensors reads (src/checkpoint.rs:6-17); the
// reference's sessions build their VarBuilders in F32, so float tensors of
// any width are converted to f32 here.  Tensors are looked up by the
// VarBuilder paths the reference's model constructors use:
//   SkyJepaModel::new (src/models/skyjepa/model.rs:22-39), TemporalConvEncoder
//   (tcn.rs:54-125), candle's GRU (weight_ih_l0 / weight_hh_l0 / bias_*_l0),
//   SkyJepaProber::new (prober.rs:54-80) from its own file, as
//   SkyJepaSession::open loads them (session.rs:183-199);
//   LeWm / WorldModel (lewm/model.rs:20-31, world_model/model.rs:19-33).
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "lwm_host.hpp"

namespace lwm {
namespace {

lwm_status bad(const std::string& m) { return set_last_error(LWM_INVALID_ARGUMENT, m); }

std::string shape_text(const std::vector<uint64_t>& s) {
    std::string t = "[";
    for (size_t i = 0; i < s.size(); ++i) t += (i ? ", " : "") + std::to_string(s[i]);
    return t + "]";
}

// ------------------------------------------------------------ JSON header

// Just enough JSON for a safetensors header: objects, arrays, strings,
// integers; every other value is skipped.
struct Json {
    const char* p;
    const char* end;
    std::string err;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool expect(char c) {
        ws();
        if (p < end && *p == c) { ++p; return true; }
        if (err.empty()) err = std::string("expected '") + c + "'";
        return false;
    }
    bool peek(char c) { ws(); return p < end && *p == c; }
    bool string(std::string& out) {
        if (!expect('"')) return false;
        out.clear();
        while (p < end && *p != '"') {
            if (*p == '\\') {
                if (++p >= end) break;
                switch (*p) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (end - p < 5) { err = "bad \\u escape"; return false; }
                        const unsigned v = static_cast<unsigned>(std::strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16));
                        if (v < 0x80) out += static_cast<char>(v);
                        else if (v < 0x800) { out += static_cast<char>(0xC0 | (v >> 6)); out += static_cast<char>(0x80 | (v & 0x3F)); }
                        else { out += static_cast<char>(0xE0 | (v >> 12)); out += static_cast<char>(0x80 | ((v >> 6) & 0x3F)); out += static_cast<char>(0x80 | (v & 0x3F)); }
                        p += 4;
                        break;
                    }
                    default: out += *p; break;
                }
                ++p;
            } else {
                out += *p++;
            }
        }
        if (p >= end) { err = "unterminated string"; return false; }
        ++p;
        return true;
    }
    bool integer(uint64_t& v) {
        ws();
        if (p >= end || *p < '0' || *p > '9') { err = "expected a non-negative integer"; return false; }
        v = 0;
        while (p < end && *p >= '0' && *p <= '9') {
            const uint64_t d = static_cast<uint64_t>(*p++ - '0');
            if (v > (UINT64_MAX - d) / 10) { err = "integer overflow"; return false; }
            v = v * 10 + d;
        }
        return true;
    }
    bool int_array(std::vector<uint64_t>& out) {
        out.clear();
        if (!expect('[')) return false;
        if (peek(']')) { ++p; return true; }
        for (;;) {
            uint64_t v;
            if (!integer(v)) return false;
            out.push_back(v);
            if (peek(',')) { ++p; continue; }
            return expect(']');
        }
    }
    bool skip(int depth = 0) {
        if (depth > 64) { err = "header nests too deeply"; return false; }
        ws();
        if (p >= end) { err = "truncated header"; return false; }
        if (*p == '"') { std::string s; return string(s); }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            ++p;
            if (peek(close)) { ++p; return true; }
            for (;;) {
                if (obj) {
                    std::string k;
                    if (!string(k) || !expect(':')) return false;
                }
                if (!skip(depth + 1)) return false;
                if (peek(',')) { ++p; continue; }
                return expect(close);
            }
        }
        while (p < end && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') ++p;  // number / literal
        return true;
    }
};

struct Entry {
    std::string dtype;
    std::vector<uint64_t> shape;
    uint64_t begin = 0, end = 0;
};

size_t dtype_size(const std::string& d) {
    if (d == "F32") return 4;
    if (d == "F64") return 8;
    if (d == "F16" || d == "BF16") return 2;
    return 0;
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    float v;
    if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(exp) - 25);
    return sign ? -v : v;
}

struct Safetensors {
    std::string path;
    FILE* f = nullptr;
    uint64_t data_start = 0, data_len = 0;
    std::map<std::string, Entry> entries;
    ~Safetensors() { if (f) std::fclose(f); }

    lwm_status open(const char* file) {
        path = file;
        f = std::fopen(file, "rb");
        if (!f) return bad("cannot open " + path + ": " + std::strerror(errno));
        if (std::fseek(f, 0, SEEK_END) != 0) return bad("cannot read " + path);
        const long long size = std::ftell(f);
        std::rewind(f);
        unsigned char len8[8];
        if (size < 8 || std::fread(len8, 1, 8, f) != 8) return bad(path + ": not a safetensors file (shorter than its header length)");
        uint64_t n = 0;
        for (int i = 7; i >= 0; --i) n = (n << 8) | len8[i];
        if (n > 100000000ull || n > static_cast<uint64_t>(size) - 8)
            return bad(path + ": safetensors header length " + std::to_string(n) + " exceeds the file");
        std::string header(n, '\0');
        if (n && std::fread(&header[0], 1, n, f) != n) return bad("cannot read the header of " + path);
        data_start = 8 + n;
        data_len = static_cast<uint64_t>(size) - data_start;
        Json j{header.data(), header.data() + header.size(), {}};
        if (!j.expect('{')) return bad(path + ": invalid safetensors header: " + j.err);
        if (j.peek('}')) { ++j.p; return LWM_OK; }
        for (;;) {
            std::string key;
            if (!j.string(key) || !j.expect(':')) return bad(path + ": invalid safetensors header: " + j.err);
            if (key == "__metadata__") {
                if (!j.skip()) return bad(path + ": invalid safetensors header: " + j.err);
            } else {
                Entry e;
                std::vector<uint64_t> offs;
                bool has_dtype = false, has_shape = false, has_offs = false;
                if (!j.expect('{')) return bad(path + ": invalid safetensors header: " + j.err);
                if (!j.peek('}')) {
                    for (;;) {
                        std::string field;
                        if (!j.string(field) || !j.expect(':')) return bad(path + ": invalid safetensors header: " + j.err);
                        bool ok;
                        if (field == "dtype") { ok = j.string(e.dtype); has_dtype = true; }
                        else if (field == "shape") { ok = j.int_array(e.shape); has_shape = true; }
                        else if (field == "data_offsets") { ok = j.int_array(offs); has_offs = true; }
                        else ok = j.skip();
                        if (!ok) return bad(path + ": invalid safetensors header: " + j.err);
                        if (j.peek(',')) { ++j.p; continue; }
                        break;
                    }
                }
                if (!j.expect('}')) return bad(path + ": invalid safetensors header: " + j.err);
                if (!has_dtype || !has_shape || !has_offs || offs.size() != 2)
                    return bad(path + ": tensor " + key + " lacks dtype, shape or data_offsets");
                e.begin = offs[0];
                e.end = offs[1];
                if (e.begin > e.end || e.end > data_len)
                    return bad(path + ": tensor " + key + " lies outside the data section");
                entries[key] = e;
            }
            if (j.peek(',')) { ++j.p; continue; }
            if (!j.expect('}')) return bad(path + ": invalid safetensors header: " + j.err);
            break;
        }
        return LWM_OK;
    }

    // Reads tensor `name` of the expected shape into out (f32).
    lwm_status read(const NamedTensor& t, float* out) {
        auto it = entries.find(t.name);
        if (it == entries.end()) return bad("cannot find tensor " + t.name);
        const Entry& e = it->second;
        std::vector<uint64_t> want(t.shape.begin(), t.shape.end());
        if (e.shape != want)
            return bad("shape mismatch for " + t.name + ", expected " + shape_text(want) + ", got " + shape_text(e.shape));
        const size_t es = dtype_size(e.dtype);
        if (!es) return bad("unsupported dtype " + e.dtype + " for tensor " + t.name + " (expected F32, F64, F16 or BF16)");
        if (e.end - e.begin != static_cast<uint64_t>(t.n) * es)
            return bad(path + ": tensor " + t.name + " holds " + std::to_string(e.end - e.begin) + " bytes, expected " +
                       std::to_string(static_cast<uint64_t>(t.n) * es));
        std::vector<unsigned char> raw(t.n * es);
        if (std::fseek(f, static_cast<long>(data_start + e.begin), SEEK_SET) != 0 ||
            (t.n && std::fread(raw.data(), 1, raw.size(), f) != raw.size()))
            return bad("cannot read tensor " + t.name + " from " + path);
        const unsigned char* r = raw.data();
        for (size_t i = 0; i < t.n; ++i) {
            if (es == 4) {
                uint32_t u = static_cast<uint32_t>(r[4 * i]) | (static_cast<uint32_t>(r[4 * i + 1]) << 8) |
                             (static_cast<uint32_t>(r[4 * i + 2]) << 16) | (static_cast<uint32_t>(r[4 * i + 3]) << 24);
                std::memcpy(&out[i], &u, 4);
            } else if (es == 8) {
                uint64_t u = 0;
                for (int b = 7; b >= 0; --b) u = (u << 8) | r[8 * i + b];
                double d;
                std::memcpy(&d, &u, 8);
                out[i] = static_cast<float>(d);
            } else {
                const uint16_t h = static_cast<uint16_t>(r[2 * i] | (r[2 * i + 1] << 8));
                if (e.dtype == "BF16") {
                    const uint32_t u = static_cast<uint32_t>(h) << 16;
                    std::memcpy(&out[i], &u, 4);
                } else {
                    out[i] = half_to_float(h);
                }
            }
        }
        return LWM_OK;
    }
};

// ------------------------------------------------------------ SkyJEPA names

struct SkyNames {
    std::vector<NamedTensor>* out;
    size_t off = 0;
    void add(const std::string& name, std::vector<uint32_t> shape, int file) {
        size_t n = 1;
        for (uint32_t d : shape) n *= d;
        if (out) out->push_back({name, std::move(shape), off, n, file});
        off += n;
    }
    // TemporalConvEncoder (tcn.rs:115-125): blocks.{l} of TemporalBlock
    // (tcn.rs:54-85): conv1, conv2, residual (1x1, only when widths differ).
    void tcn(const lwm_tcn_config& t, const std::string& p) {
        uint32_t in = t.input_dim;
        for (uint32_t l = 0; l < t.levels; ++l) {
            const uint32_t o = t.channels[l], K = t.kernel_size;
            const std::string b = p + ".blocks." + std::to_string(l);
            add(b + ".conv1.weight", {o, in, K}, 0);
            add(b + ".conv1.bias", {o}, 0);
            add(b + ".conv2.weight", {o, o, K}, 0);
            add(b + ".conv2.bias", {o}, 0);
            if (in != o) {
                add(b + ".residual.weight", {o, in, 1}, 0);
                add(b + ".residual.bias", {o}, 0);
            }
            in = o;
        }
    }
};

}  // namespace

size_t skyjepa_named_tensors(const lwm_skyjepa_config& c, std::vector<NamedTensor>* out) {
    const size_t total = lwm_skyjepa_weight_count(&c);
    if (total == 0) return 0;
    SkyNames k{out};
    k.tcn(c.state_encoder, "state_encoder");
    const uint32_t H = c.latent_dim, so = c.state_encoder.channels[c.state_encoder.levels - 1];
    k.add("state_projection.weight", {H, so}, 0);
    k.add("state_projection.bias", {H}, 0);
    k.tcn(c.action_encoder, "action_encoder");
    const uint32_t E = c.action_encoder.channels[c.action_encoder.levels - 1];
    k.add("predictor.weight_ih_l0", {3 * H, E}, 0);
    k.add("predictor.weight_hh_l0", {3 * H, H}, 0);
    k.add("predictor.bias_ih_l0", {3 * H}, 0);
    k.add("predictor.bias_hh_l0", {3 * H}, 0);
    const uint32_t hid = c.prober_hidden_dim;
    k.add("input.weight", {hid, H}, 1);
    k.add("input.bias", {hid}, 1);
    for (uint32_t i = 0; i + 1 < c.prober_hidden_layers; ++i) {
        k.add("hidden." + std::to_string(i) + ".weight", {hid, hid}, 1);
        k.add("hidden." + std::to_string(i) + ".bias", {hid}, 1);
    }
    k.add("output.weight", {15, hid}, 1);
    k.add("output.bias", {15}, 1);
    return k.off == total ? total : 0;
}

}  // namespace lwm

namespace {

size_t fill_info(const std::vector<lwm::NamedTensor>& v, size_t index, lwm_tensor_info* out) {
    if (out && index < v.size()) {
        const lwm::NamedTensor& t = v[index];
        std::memset(out, 0, sizeof *out);
        std::snprintf(out->name, sizeof out->name, "%s", t.name.c_str());
        out->rank = static_cast<uint32_t>(t.shape.size());
        for (size_t i = 0; i < t.shape.size() && i < 4; ++i) out->shape[i] = t.shape[i];
        out->offset = t.off;
        out->numel = t.n;
        out->file = t.file;
    }
    return v.size();
}

lwm_status load(const std::vector<lwm::NamedTensor>& tensors, const char* const* paths, int files, float* out) {
    std::unique_ptr<lwm::Safetensors> f[2];
    for (int i = 0; i < files; ++i) {
        f[i].reset(new lwm::Safetensors());
        const lwm_status st = f[i]->open(paths[i]);
        if (st != LWM_OK) return st;
    }
    for (const lwm::NamedTensor& t : tensors) {
        const lwm_status st = f[t.file]->read(t, out + t.off);
        if (st != LWM_OK) return st;
    }
    return LWM_OK;
}

}  // namespace

extern "C" {

size_t lwm_skyjepa_tensor_info(const lwm_skyjepa_config* cfg, size_t index, lwm_tensor_info* out) {
    if (!cfg) return 0;
    std::vector<lwm::NamedTensor> v;
    if (!lwm::skyjepa_named_tensors(*cfg, &v)) return 0;
    return fill_info(v, index, out);
}

size_t lwm_lewm_tensor_info(const lwm_lewm_config* cfg, int32_t names, size_t index, lwm_tensor_info* out) {
    if (!cfg || (names != LWM_LEWM_NAMES_LEWM && names != LWM_LEWM_NAMES_WORLD_MODEL)) return 0;
    if (names == LWM_LEWM_NAMES_LEWM && cfg->encoder != LWM_ENCODER_VIT) return 0;
    std::vector<lwm::NamedTensor> v;
    if (!lwm::lewm_named_tensors(*cfg, names, &v)) return 0;
    return fill_info(v, index, out);
}

lwm_status lwm_skyjepa_weights_from_safetensors(const lwm_skyjepa_config* cfg, const char* latent_path,
                                                const char* prober_path, float* out, size_t count) {
    if (!cfg || !latent_path || !prober_path || !out) return lwm::bad("null argument");
    std::vector<lwm::NamedTensor> v;
    const size_t need = lwm::skyjepa_named_tensors(*cfg, &v);
    if (!need) return lwm::bad("invalid SkyJEPA configuration");
    if (count != need)
        return lwm::bad("SkyJEPA weight blob has " + std::to_string(count) + " values, expected " + std::to_string(need));
    const char* paths[2] = {latent_path, prober_path};
    return load(v, paths, 2, out);
}

lwm_status lwm_lewm_weights_from_safetensors(const lwm_lewm_config* cfg, int32_t names, const char* path,
                                             float* out, size_t count) {
    if (!cfg || !path || !out) return lwm::bad("null argument");
    if (names != LWM_LEWM_NAMES_LEWM && names != LWM_LEWM_NAMES_WORLD_MODEL)
        return lwm::bad("unknown LeWM checkpoint naming " + std::to_string(names));
    if (names == LWM_LEWM_NAMES_LEWM && cfg->encoder != LWM_ENCODER_VIT)
        return lwm::bad("LeWm checkpoints hold a ViT observation encoder");
    std::vector<lwm::NamedTensor> v;
    const size_t need = lwm::lewm_named_tensors(*cfg, names, &v);
    if (!need) return lwm::bad("invalid LeWM configuration");
    if (count != need)
        return lwm::bad("LeWM weight blob has " + std::to_string(count) + " values, expected " + std::to_string(need));
    return load(v, &path, 1, out);
}

}  // extern "C"
