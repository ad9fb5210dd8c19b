// model_loader.cpp -- safetensors and config.json readers for the CUDA
// backend (see model_loader.h for the reference functions each replaces).
//
// safetensors layout: an 8-byte little-endian header length n, n bytes of
// JSON {"<name>": {"dtype": "...", "shape": [...], "data_offsets": [b, e]},
// "__metadata__": {...}}, then the data section (offsets relative to it).
#include "model_loader.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cstring>
#include <fstream>
#include <sstream>

namespace compute {

namespace {

// ------------------------------------------------------------ a small JSON reader
// Objects, arrays, strings (with escapes), numbers, true/false/null: enough
// for safetensors headers and config.json.
struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json *get(const std::string &k) const {
        for (auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class Parser {
public:
    explicit Parser(const std::string &s) : s_(s) {}

    bool parse(Json &out) {
        if (!value(out, 0)) return false;
        ws();
        return i_ == s_.size();
    }

private:
    const std::string &s_;
    size_t i_ = 0;

    void ws() {
        while (i_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[i_]))) ++i_;
    }
    bool lit(const char *t) {
        const size_t n = std::strlen(t);
        if (s_.compare(i_, n, t) != 0) return false;
        i_ += n;
        return true;
    }
    bool string(std::string &out) {
        if (i_ >= s_.size() || s_[i_] != '"') return false;
        ++i_;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            if (i_ >= s_.size()) return false;
            c = s_[i_++];
            switch (c) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    if (i_ + 4 > s_.size()) return false;
                    unsigned v = 0;
                    for (int k = 0; k < 4; ++k) {
                        const char h = s_[i_ + k];
                        v <<= 4;
                        if (h >= '0' && h <= '9') v |= (unsigned)(h - '0');
                        else if (h >= 'a' && h <= 'f') v |= (unsigned)(h - 'a' + 10);
                        else if (h >= 'A' && h <= 'F') v |= (unsigned)(h - 'A' + 10);
                        else return false;
                    }
                    i_ += 4;
                    if (v < 0x80) {
                        out.push_back(static_cast<char>(v));
                    } else if (v < 0x800) {
                        out.push_back(static_cast<char>(0xC0 | (v >> 6)));
                        out.push_back(static_cast<char>(0x80 | (v & 0x3F)));
                    } else {
                        out.push_back(static_cast<char>(0xE0 | (v >> 12)));
                        out.push_back(static_cast<char>(0x80 | ((v >> 6) & 0x3F)));
                        out.push_back(static_cast<char>(0x80 | (v & 0x3F)));
                    }
                    break;
                }
                default: return false;
            }
        }
        if (i_ >= s_.size()) return false;
        ++i_;
        return true;
    }
    bool value(Json &v, int depth) {
        if (depth > 64) return false;
        ws();
        if (i_ >= s_.size()) return false;
        const char c = s_[i_];
        if (c == '{') {
            v.kind = Json::Object;
            ++i_;
            ws();
            if (i_ < s_.size() && s_[i_] == '}') {
                ++i_;
                return true;
            }
            while (true) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') return false;
                ++i_;
                Json child;
                if (!value(child, depth + 1)) return false;
                v.obj.emplace_back(std::move(k), std::move(child));
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == '}') {
                    ++i_;
                    return true;
                }
                return false;
            }
        }
        if (c == '[') {
            v.kind = Json::Array;
            ++i_;
            ws();
            if (i_ < s_.size() && s_[i_] == ']') {
                ++i_;
                return true;
            }
            while (true) {
                Json child;
                if (!value(child, depth + 1)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == ']') {
                    ++i_;
                    return true;
                }
                return false;
            }
        }
        if (c == '"') {
            v.kind = Json::String;
            return string(v.str);
        }
        if (lit("true")) {
            v.kind = Json::Bool;
            v.b = true;
            return true;
        }
        if (lit("false")) {
            v.kind = Json::Bool;
            return true;
        }
        if (lit("null")) {
            v.kind = Json::Null;
            return true;
        }
        const size_t j = i_;
        while (i_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[i_])) || s_[i_] == '-' ||
                                  s_[i_] == '+' || s_[i_] == '.' || s_[i_] == 'e' || s_[i_] == 'E'))
            ++i_;
        if (i_ == j) return false;
        v.kind = Json::Number;
        try {
            v.num = std::stod(s_.substr(j, i_ - j));
        } catch (...) {
            return false;
        }
        return true;
    }
};

Error bad(const std::string &m) { return Error{ErrorCode::InvalidInput, m}; }

bool dtype_of(const std::string &s, DType &d, size_t &elem) {
    if (s == "U32") { d = DType::U32; elem = 4; return true; }
    if (s == "I32") { d = DType::I32; elem = 4; return true; }
    if (s == "BF16") { d = DType::BF16; elem = 2; return true; }
    if (s == "F16") { d = DType::F16; elem = 2; return true; }
    if (s == "F32") { d = DType::F32; elem = 4; return true; }
    return false;
}

}  // namespace

Result<std::optional<QuantizationConfig>> load_quantization_config(
    const std::filesystem::path &model_dir) {
    const auto path = model_dir / "config.json";
    std::ifstream f(path, std::ios::binary);
    if (!f) return std::unexpected(bad("Cannot read " + path.string()));
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    Json root;
    if (!Parser(text).parse(root) || root.kind != Json::Object)
        return std::unexpected(bad("Malformed JSON in " + path.string()));
    const Json *q = root.get("quantization");
    if (!q || q->kind == Json::Null) return std::optional<QuantizationConfig>{};
    if (q->kind != Json::Object) return std::unexpected(bad("quantization must be an object"));
    const Json *gs = q->get("group_size");
    if (!gs || gs->kind != Json::Number)
        return std::unexpected(bad("Quantization missing required field: group_size"));
    const Json *bits = q->get("bits");
    if (!bits || bits->kind != Json::Number)
        return std::unexpected(bad("Quantization missing required field: bits"));
    QuantizationConfig c;
    c.group_size = static_cast<int>(gs->num);
    c.bits = static_cast<int>(bits->num);
    return std::optional<QuantizationConfig>{c};
}

Result<std::vector<SafetensorInfo>> read_safetensors_header(const std::filesystem::path &file,
                                                            uint64_t *data_offset) {
    std::ifstream f(file, std::ios::binary);
    if (!f) return std::unexpected(bad("Cannot read " + file.string()));
    unsigned char len8[8];
    if (!f.read(reinterpret_cast<char *>(len8), 8))
        return std::unexpected(bad(file.string() + ": truncated header length"));
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | len8[i];
    const uint64_t fsize = std::filesystem::file_size(file);
    if (n == 0 || n > fsize - 8 || n > (uint64_t)1 << 30)
        return std::unexpected(bad(file.string() + ": bad header length"));
    std::string text(n, '\0');
    if (!f.read(text.data(), (std::streamsize)n))
        return std::unexpected(bad(file.string() + ": truncated header"));
    Json root;
    if (!Parser(text).parse(root) || root.kind != Json::Object)
        return std::unexpected(bad(file.string() + ": malformed JSON header"));
    const uint64_t data_size = fsize - 8 - n;
    std::vector<SafetensorInfo> out;
    for (auto &kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const Json &t = kv.second;
        const Json *dt = t.get("dtype");
        const Json *sh = t.get("shape");
        const Json *off = t.get("data_offsets");
        if (t.kind != Json::Object || !dt || dt->kind != Json::String || !sh ||
            sh->kind != Json::Array || !off || off->kind != Json::Array || off->arr.size() != 2)
            return std::unexpected(bad(file.string() + ": bad entry for " + kv.first));
        SafetensorInfo info;
        info.name = kv.first;
        info.dtype = dt->str;
        uint64_t count = 1;
        for (auto &d : sh->arr) {
            if (d.kind != Json::Number || d.num < 0)
                return std::unexpected(bad(file.string() + ": bad shape for " + kv.first));
            info.shape.push_back(static_cast<int64_t>(d.num));
            count *= static_cast<uint64_t>(d.num);
        }
        info.begin = static_cast<uint64_t>(off->arr[0].num);
        info.end = static_cast<uint64_t>(off->arr[1].num);
        DType d;
        size_t elem = 0;
        if (!dtype_of(info.dtype, d, elem))
            return std::unexpected(bad(file.string() + ": unsupported dtype " + info.dtype +
                                       " for " + kv.first));
        if (info.end < info.begin || info.end > data_size || info.end - info.begin != count * elem)
            return std::unexpected(bad(file.string() + ": data range does not match shape for " +
                                       kv.first));
        out.push_back(std::move(info));
    }
    if (data_offset) *data_offset = 8 + n;
    return out;
}

DeviceWeights::~DeviceWeights() {
    for (void *p : blocks_) cudaFree(p);
}

DeviceWeights::DeviceWeights(DeviceWeights &&o) noexcept
    : map_(std::move(o.map_)), blocks_(std::move(o.blocks_)), bytes_(o.bytes_) {
    o.blocks_.clear();
    o.bytes_ = 0;
}

DeviceWeights &DeviceWeights::operator=(DeviceWeights &&o) noexcept {
    if (this != &o) {
        for (void *p : blocks_) cudaFree(p);
        map_ = std::move(o.map_);
        blocks_ = std::move(o.blocks_);
        bytes_ = o.bytes_;
        o.blocks_.clear();
        o.bytes_ = 0;
    }
    return *this;
}

std::vector<std::filesystem::path> ModelLoader::find_safetensors_files(
    const std::filesystem::path &model_dir) {
    std::vector<std::filesystem::path> files;
    std::error_code ec;
    for (auto it = std::filesystem::directory_iterator(model_dir, ec);
         !ec && it != std::filesystem::directory_iterator(); it.increment(ec))
        if (it->is_regular_file() && it->path().extension() == ".safetensors")
            files.push_back(it->path());
    std::sort(files.begin(), files.end());
    return files;
}

Result<DeviceWeights> ModelLoader::load_weights_cuda(const std::filesystem::path &model_dir,
                                                      void *stream) {
    if (!std::filesystem::exists(model_dir) || !std::filesystem::is_directory(model_dir))
        return std::unexpected(bad("Model directory not found: " + model_dir.string()));
    const auto files = find_safetensors_files(model_dir);
    if (files.empty())
        return std::unexpected(bad("No .safetensors files found in: " + model_dir.string()));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    DeviceWeights w;
    std::vector<char> host;
    for (const auto &file : files) {
        uint64_t data_off = 0;
        auto hdr = read_safetensors_header(file, &data_off);
        if (!hdr) return std::unexpected(hdr.error());
        uint64_t span = 0;
        for (auto &t : *hdr) span = std::max(span, t.end);
        // one device block per file; each tensor starts on a 256-byte boundary
        // (the file's own offsets need not be aligned), so every kernel sees
        // aligned bases
        uint64_t total = 0;
        for (auto &t : *hdr) total += ((t.end - t.begin) + 255) & ~uint64_t(255);
        std::ifstream f(file, std::ios::binary);
        host.resize(span);
        f.seekg((std::streamoff)data_off);
        if (span && !f.read(host.data(), (std::streamsize)span))
            return std::unexpected(bad(file.string() + ": truncated data section"));
        void *block = nullptr;
        if (total && cudaMalloc(&block, total) != cudaSuccess) {
            cudaGetLastError();
            return std::unexpected(Error{ErrorCode::ComputeError,
                                         "cudaMalloc of " + std::to_string(total) + " bytes failed"});
        }
        if (block) w.blocks_.push_back(block);
        uint64_t at = 0;
        for (auto &t : *hdr) {
            if (w.map_.count(t.name))
                return std::unexpected(bad("Tensor " + t.name + " appears in two files"));
            const uint64_t nb = t.end - t.begin;
            char *dst = static_cast<char *>(block) + at;
            if (nb && cudaMemcpyAsync(dst, host.data() + t.begin, nb, cudaMemcpyHostToDevice, st) !=
                          cudaSuccess)
                return std::unexpected(Error{ErrorCode::ComputeError, "copy of " + t.name + " failed"});
            DeviceTensor d;
            size_t elem = 0;
            dtype_of(t.dtype, d.dtype, elem);
            d.data = dst;
            d.shape = t.shape;
            w.map_.emplace(t.name, d);
            at += (nb + 255) & ~uint64_t(255);
        }
        // the host buffer is reused for the next file: finish these copies first
        if (cudaStreamSynchronize(st) != cudaSuccess)
            return std::unexpected(Error{ErrorCode::ComputeError, "device copy failed"});
        w.bytes_ += total;
    }
    return w;
}

}  // namespace compute
