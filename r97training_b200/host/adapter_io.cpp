// adapter_io.cpp -- the trained adapter on disk in PEFT's layout, the one the reference's trainer writes
// and its server reads (reference include/r97/adapter_io.h, src/adapter_io.cpp; docs/ADAPTER.md s4):
// a directory holding `adapter_config.json` and `adapter_model.safetensors`.
//
//   * adapter_config.json: PEFT's keys in PEFT's order (peft_type, task_type, base_model_name_or_path, bias,
//     fan_in_fan_out, inference_mode, lora_alpha, lora_dropout, r, target_modules, use_rslora, and
//     radiance_input_basis when the trunk is stored under a transform), two-space indented, one array
//     element a line, a newline at the end;
//   * adapter_model.safetensors: an 8-byte little-endian header length, the compact JSON header (tensors
//     sorted by parameter name, each {"dtype", "shape", "data_offsets"}) padded with spaces to a multiple of
//     8 bytes, then the tensors' bytes in header order, f32 or bf16 little-endian.
// A parameter `<module>.lora_A` is stored as `base_model.model.<module>.lora_A.weight`.
//
// The parameters come from a flat f32 buffer (host or device) holding them in the caller's order, the
// adapter's own layout, so a B200-trained adapter is written without an intermediate copy per tensor.
#include "r97b.h"
#include "r97host.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace r97b {
namespace {

namespace fs = std::filesystem;

[[noreturn]] void fail(const std::string& what) { throw std::runtime_error("r97host adapter: " + what); }

const char* kPrefix = "base_model.model.";

std::string tensor_name(const std::string& param) { return std::string(kPrefix) + param + ".weight"; }

// ------------------------------------------------------------------------------------ JSON out

std::string quoted(const std::string& s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        switch (c) {
            case '"': o += "\\\""; break;
            case '\\': o += "\\\\"; break;
            case '\b': o += "\\b"; break;
            case '\f': o += "\\f"; break;
            case '\n': o += "\\n"; break;
            case '\r': o += "\\r"; break;
            case '\t': o += "\\t"; break;
            default:
                if (c < 0x20) {
                    char b[8];
                    std::snprintf(b, sizeof b, "\\u%04x", c);
                    o += b;
                } else {
                    o += (char)c;
                }
        }
    }
    return o + "\"";
}

// A double as JSON prints it: the shortest decimal that reads back to the same value, with ".0" on an
// integral one.
std::string number(double v) {
    char b[40];
    for (int p = 1; p <= 17; ++p) {
        std::snprintf(b, sizeof b, "%.*g", p, v);
        if (std::strtod(b, nullptr) == v) break;
    }
    std::string s = b;
    if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
    return s;
}

std::string config_json(const R97hostAdapterConfig& c) {
    if (c.rank <= 0) fail("rank must be at least 1");
    if (!std::isfinite(c.alpha)) fail("alpha must be finite");
    const std::string alpha = std::floor(c.alpha) == c.alpha ? std::to_string((int64_t)c.alpha) : number(c.alpha);
    std::string j = "{\n";
    j += "  \"peft_type\": \"LORA\",\n";
    j += "  \"task_type\": \"CAUSAL_LM\",\n";
    j += "  \"base_model_name_or_path\": " + quoted(c.base_model ? c.base_model : "") + ",\n";
    j += "  \"bias\": \"none\",\n";
    j += "  \"fan_in_fan_out\": false,\n";
    j += "  \"inference_mode\": true,\n";
    j += "  \"lora_alpha\": " + alpha + ",\n";
    j += "  \"lora_dropout\": 0.0,\n";
    j += "  \"r\": " + std::to_string(c.rank) + ",\n";
    if (c.n_targets <= 0) {
        j += "  \"target_modules\": [],\n";
    } else {
        j += "  \"target_modules\": [\n";
        for (int i = 0; i < c.n_targets; ++i)
            j += "    " + quoted(c.targets[i]) + (i + 1 < c.n_targets ? ",\n" : "\n");
        j += "  ],\n";
    }
    const bool basis = c.input_basis && c.input_basis[0];
    j += std::string("  \"use_rslora\": false") + (basis ? ",\n" : "\n");
    if (basis) j += "  \"radiance_input_basis\": " + quoted(c.input_basis) + "\n";
    return j + "}\n";
}

uint16_t to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float from_bf16(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

struct Tensor {
    std::string param;
    std::vector<int64_t> shape;
    const float* values;  // host
    int64_t count;
};

std::string model_safetensors(std::vector<Tensor> ts, int dtype) {
    std::sort(ts.begin(), ts.end(), [](const Tensor& a, const Tensor& b) { return a.param < b.param; });
    const int esz = dtype == 1 ? 2 : 4;
    std::string hdr = "{";
    uint64_t off = 0;
    for (size_t i = 0; i < ts.size(); ++i) {
        if (i && ts[i].param == ts[i - 1].param) fail("two parameters write the same tensor '" + ts[i].param + "'");
        const uint64_t bytes = (uint64_t)ts[i].count * esz;
        std::string shape = "[";
        for (size_t d = 0; d < ts[i].shape.size(); ++d) shape += (d ? "," : "") + std::to_string(ts[i].shape[d]);
        shape += "]";
        hdr += (i ? "," : "") + quoted(tensor_name(ts[i].param)) + ":{\"dtype\":\"" + (dtype == 1 ? "BF16" : "F32") +
               "\",\"shape\":" + shape + ",\"data_offsets\":[" + std::to_string(off) + "," +
               std::to_string(off + bytes) + "]}";
        off += bytes;
    }
    hdr += "}";
    hdr.append((8 - hdr.size() % 8) % 8, ' ');
    std::string out;
    out.reserve(8 + hdr.size() + off);
    const uint64_t hl = hdr.size();
    for (int i = 0; i < 8; ++i) out.push_back((char)((hl >> (8 * i)) & 0xFF));
    out += hdr;
    for (const Tensor& t : ts) {
        if (dtype == 1) {
            for (int64_t i = 0; i < t.count; ++i) {
                const uint16_t h = to_bf16(t.values[i]);
                out.push_back((char)(h & 0xFF));
                out.push_back((char)(h >> 8));
            }
        } else {
            for (int64_t i = 0; i < t.count; ++i) {
                uint32_t u;
                std::memcpy(&u, &t.values[i], 4);
                for (int k = 0; k < 4; ++k) out.push_back((char)((u >> (8 * k)) & 0xFF));
            }
        }
    }
    return out;
}

void write_file(const fs::path& p, const std::string& bytes) {
    std::ofstream f(p, std::ios::binary | std::ios::trunc);
    if (!f) fail("cannot create '" + p.string() + "'");
    f.write(bytes.data(), (std::streamsize)bytes.size());
    if (!f) fail("cannot write '" + p.string() + "'");
}

std::string read_file(const fs::path& p) {
    std::ifstream f(p, std::ios::binary);
    if (!f) fail("cannot open '" + p.string() + "'");
    return std::string((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

// ------------------------------------------------------------------------------------ JSON in

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* get(const std::string& k) const {
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class Parser {
public:
    explicit Parser(const std::string& s) : s_(s) {}
    Json parse() {
        Json v = value();
        ws();
        if (i_ != s_.size()) fail("trailing characters in JSON");
        return v;
    }

private:
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    char peek() {
        ws();
        if (i_ >= s_.size()) fail("unexpected end of JSON");
        return s_[i_];
    }
    void expect(char c) {
        if (peek() != c) fail(std::string("expected '") + c + "' in JSON");
        ++i_;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (s_.compare(i_, n, w) == 0) {
            i_ += n;
            return true;
        }
        return false;
    }
    std::string string() {
        expect('"');
        std::string o;
        while (true) {
            if (i_ >= s_.size()) fail("unterminated JSON string");
            const char c = s_[i_++];
            if (c == '"') break;
            if (c != '\\') {
                o += c;
                continue;
            }
            if (i_ >= s_.size()) fail("bad JSON escape");
            const char e = s_[i_++];
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
                    if (i_ + 4 > s_.size()) fail("bad JSON \\u escape");
                    const unsigned cp = (unsigned)std::stoul(s_.substr(i_, 4), nullptr, 16);
                    i_ += 4;
                    if (cp < 0x80) {
                        o += (char)cp;
                    } else if (cp < 0x800) {
                        o += (char)(0xC0 | (cp >> 6));
                        o += (char)(0x80 | (cp & 0x3F));
                    } else {
                        o += (char)(0xE0 | (cp >> 12));
                        o += (char)(0x80 | ((cp >> 6) & 0x3F));
                        o += (char)(0x80 | (cp & 0x3F));
                    }
                    break;
                }
                default: fail("bad JSON escape");
            }
        }
        return o;
    }
    Json value() {
        Json v;
        const char c = peek();
        if (c == '{') {
            ++i_;
            v.kind = Json::Obj;
            if (peek() == '}') {
                ++i_;
                return v;
            }
            while (true) {
                std::string k = string();
                expect(':');
                v.obj.emplace_back(std::move(k), value());
                if (peek() == ',') {
                    ++i_;
                    continue;
                }
                expect('}');
                return v;
            }
        }
        if (c == '[') {
            ++i_;
            v.kind = Json::Arr;
            if (peek() == ']') {
                ++i_;
                return v;
            }
            while (true) {
                v.arr.push_back(value());
                if (peek() == ',') {
                    ++i_;
                    continue;
                }
                expect(']');
                return v;
            }
        }
        if (c == '"') {
            v.kind = Json::Str;
            v.str = string();
            return v;
        }
        if (lit("true")) {
            v.kind = Json::Bool;
            v.b = true;
            return v;
        }
        if (lit("false")) {
            v.kind = Json::Bool;
            return v;
        }
        if (lit("null")) return v;
        size_t used = 0;
        v.kind = Json::Num;
        try {
            v.num = std::stod(s_.substr(i_, 64), &used);
        } catch (const std::exception&) {
            fail("bad JSON value");
        }
        i_ += used;
        return v;
    }

    const std::string& s_;
    size_t i_ = 0;
};

thread_local std::string g_adapter_error;

}  // namespace
}  // namespace r97b

extern "C" int r97host_adapter_write(const char* dir, const R97hostAdapterConfig* cfg, int32_t nparams,
                                     const char* const* names, const int64_t* shapes, const float* values,
                                     int32_t values_on_device, void* stream) {
    using namespace r97b;
    try {
        g_adapter_error.clear();
        if (!dir || !cfg || nparams <= 0 || !names || !shapes || !values) fail("bad arguments");
        if (cfg->dtype != 0 && cfg->dtype != 1) fail("dtype must be 0 (F32) or 1 (BF16)");
        int64_t total = 0;
        for (int32_t i = 0; i < nparams; ++i) {
            if (shapes[2 * i] <= 0 || shapes[2 * i + 1] <= 0) fail(std::string("bad shape for ") + names[i]);
            total += shapes[2 * i] * shapes[2 * i + 1];
        }
        std::vector<float> host;
        const float* src = values;
        if (values_on_device) {
            host.resize((size_t)total);
            if (r97b_memcpy(host.data(), values, 4 * total, 1, stream) != R97B_OK || r97b_stream_sync(stream) != R97B_OK)
                fail("cannot copy the adapter from the device");
            src = host.data();
        }
        std::vector<Tensor> ts;
        int64_t off = 0;
        for (int32_t i = 0; i < nparams; ++i) {
            const int64_t c = shapes[2 * i] * shapes[2 * i + 1];
            ts.push_back(Tensor{names[i], {shapes[2 * i], shapes[2 * i + 1]}, src + off, c});
            off += c;
        }
        const std::string config = config_json(*cfg);
        const std::string model = model_safetensors(std::move(ts), cfg->dtype);
        const fs::path d(dir);
        std::error_code ec;
        fs::create_directories(d, ec);
        if (ec) fail("cannot create '" + std::string(dir) + "': " + ec.message());
        write_file(d / "adapter_config.json", config);
        write_file(d / "adapter_model.safetensors", model);
        return 0;
    } catch (const std::exception& e) {
        g_adapter_error = e.what();
        return 1;
    }
}

extern "C" int r97host_adapter_read(const char* dir, int32_t nparams, const char* const* names, const int64_t* shapes,
                                    float* values, int64_t* rank, double* alpha, int32_t* dtype) {
    using namespace r97b;
    try {
        g_adapter_error.clear();
        if (!dir || nparams <= 0 || !names || !shapes || !values) fail("bad arguments");
        const fs::path d(dir);
        const std::string cfg_text = read_file(d / "adapter_config.json");
        const Json cfg = Parser(cfg_text).parse();
        const Json* pt = cfg.get("peft_type");
        if (!pt || pt->kind != Json::Str || pt->str != "LORA") fail("adapter_config.json is not a LoRA config");
        const Json* r = cfg.get("r");
        const Json* a = cfg.get("lora_alpha");
        if (!r || r->kind != Json::Num || !a || a->kind != Json::Num) fail("adapter_config.json lacks r / lora_alpha");
        for (const char* k : {"rank_pattern", "alpha_pattern"}) {
            const Json* x = cfg.get(k);
            if (x && x->kind == Json::Obj && !x->obj.empty()) fail(std::string("unsupported ") + k);
        }
        const Json* rs = cfg.get("use_rslora");
        if (rs && rs->kind == Json::Bool && rs->b) fail("unsupported use_rslora");
        if (rank) *rank = (int64_t)r->num;
        if (alpha) *alpha = a->num;

        const std::string blob = read_file(d / "adapter_model.safetensors");
        if (blob.size() < 8) fail("adapter_model.safetensors is too short");
        uint64_t hl = 0;
        for (int i = 0; i < 8; ++i) hl |= (uint64_t)(uint8_t)blob[i] << (8 * i);
        if (hl > blob.size() - 8) fail("adapter_model.safetensors has a bad header length");
        const std::string hdr_text = blob.substr(8, hl);
        const Json hdr = Parser(hdr_text).parse();
        const char* data = blob.data() + 8 + hl;
        const uint64_t data_bytes = blob.size() - 8 - hl;
        int file_dtype = -1;
        int64_t off = 0;
        for (int32_t i = 0; i < nparams; ++i) {
            const std::string tn = tensor_name(names[i]);
            const Json* t = hdr.get(tn);
            if (!t) fail("adapter_model.safetensors has no tensor '" + tn + "'");
            const Json* dt = t->get("dtype");
            const Json* sh = t->get("shape");
            const Json* of = t->get("data_offsets");
            if (!dt || !sh || !of || sh->arr.size() != 2 || of->arr.size() != 2) fail("bad entry for '" + tn + "'");
            const int td = dt->str == "F32" ? 0 : dt->str == "BF16" ? 1 : -1;
            if (td < 0) fail("unsupported dtype '" + dt->str + "' for '" + tn + "'");
            if (file_dtype >= 0 && td != file_dtype) fail("the file mixes dtypes");
            file_dtype = td;
            if ((int64_t)sh->arr[0].num != shapes[2 * i] || (int64_t)sh->arr[1].num != shapes[2 * i + 1])
                fail("shape mismatch for '" + tn + "'");
            const uint64_t b0 = (uint64_t)of->arr[0].num, b1 = (uint64_t)of->arr[1].num;
            const int64_t c = shapes[2 * i] * shapes[2 * i + 1];
            if (b1 < b0 || b1 > data_bytes || b1 - b0 != (uint64_t)c * (td == 1 ? 2 : 4))
                fail("bad data offsets for '" + tn + "'");
            const char* p = data + b0;
            for (int64_t k = 0; k < c; ++k) {
                if (td == 1) {
                    const uint16_t h = (uint16_t)((uint8_t)p[2 * k] | ((uint16_t)(uint8_t)p[2 * k + 1] << 8));
                    values[off + k] = from_bf16(h);
                } else {
                    uint32_t u = 0;
                    for (int q = 0; q < 4; ++q) u |= (uint32_t)(uint8_t)p[4 * k + q] << (8 * q);
                    std::memcpy(&values[off + k], &u, 4);
                }
            }
            off += c;
        }
        if ((int32_t)hdr.obj.size() != nparams + (hdr.get("__metadata__") ? 1 : 0))
            fail("adapter_model.safetensors holds tensors the parameter set does not name");
        if (dtype) *dtype = file_dtype;
        return 0;
    } catch (const std::exception& e) {
        g_adapter_error = e.what();
        return 1;
    }
}

extern "C" const char* r97host_adapter_error(void) { return r97b::g_adapter_error.c_str(); }
