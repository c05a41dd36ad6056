// checkpoint.cu — real-checkpoint path of the RDT-1B runtime: safetensors
// reading, the converter's key mapping, config.json, and the upload of a
// checkpoint's float weights into the model's int8 per-output-channel
// projections.
//
//   safetensors   [u64 little-endian header length][JSON header][data]; the
//                 header maps tensor names to {dtype, shape, data_offsets}
//                 (offsets relative to the data section) plus an optional
//                 "__metadata__" object. Parsed here by a small JSON reader;
//                 entries are listed sorted by name and the same inputs are
//                 rejected as by the reference's SafeTensorsLoader
//                 (src/loader/safetensors.cpp:65-100: short file, header past
//                 the end, unknown dtype; :145-148 data past the end).
//   key mapping   remap_key of tools/convert/hf_to_servoflow.py:41-66: EMA
//                 shadows, optimizer and scheduler entries are dropped,
//                 "model." is stripped, adaptors and action_norm.* kept. A
//                 checkpoint already in the converter's output names loads
//                 as it is, like the reference's RDT1BModel::load_weights
//                 (src/models/rdt1b/rdt1b.cpp:97-111), which applies no
//                 mapping.
//   config        RDT1BConfig::from_json (src/models/rdt1b/config.cpp:10-66):
//                 the converter's flat keys, the HF nested "rdt" and
//                 "noise_scheduler" keys.
//   upload        per tensor, as load_weight_from_map does
//                 (src/loader/safetensors.cpp:156-183): equal dtypes are
//                 copied, others are uploaded and converted on the device
//                 (float → bf16 round-to-nearest-even, the cast of the
//                 converter's `t.to(dtype)`, hf_to_servoflow.py:180-185). A
//                 float "<linear>.weight" [N, K] becomes the model's
//                 "<linear>.weight_q" int8 [N, K] and "<linear>.weight_scale"
//                 fp32 [N]: s = max_k |w| / 127 (1 for an all-zero row),
//                 q = clamp(round-half-even(w / s), −127, 127), so that
//                 q·s is the dequantisation of the reference's
//                 dequantize_int8 (src/backend/cuda/ops/quantization.cu:
//                 18-50). Pre-quantised "weight_q"/"weight_scale" pairs are
//                 copied as they are.
// Setup-time code: it allocates one device staging buffer per file and
// synchronises; nothing here runs on the hot path.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <set>
#include <sstream>
#include <string>
#include <type_traits>
#include <vector>

#include "common.cuh"

namespace sfb {

static int fail(int status, const std::string& msg) {
    snprintf(last_error_buf(), 256, "%s", msg.c_str());
    return status;
}

// ── a small JSON reader (RFC 8259 values; numbers are kept as text) ─────────
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    std::string text;                                    // string value or number text
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;
    const Value* get(const char* key) const {
        const Value* found = nullptr;                    // the last duplicate wins
        for (const auto& kv : obj)
            if (kv.first == key) found = &kv.second;
        return found;
    }
};

class Parser {
public:
    Parser(const char* p, const char* e) : p_(p), e_(e) {}
    bool document(Value& v) {
        if (!value(v, 0)) return false;
        ws();
        return p_ == e_;
    }

private:
    const char* p_;
    const char* e_;
    static constexpr int kMaxDepth = 64;

    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool eat(char c) {
        ws();
        if (p_ < e_ && *p_ == c) { ++p_; return true; }
        return false;
    }
    bool literal(const char* word) {
        const size_t n = std::strlen(word);
        if (static_cast<size_t>(e_ - p_) < n || std::memcmp(p_, word, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(uint32_t& v) {
        if (e_ - p_ < 4) return false;
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
    bool string(std::string& out) {
        ws();
        if (p_ >= e_ || *p_ != '"') return false;
        ++p_;
        out.clear();
        while (p_ < e_ && *p_ != '"') {
            const unsigned char c = static_cast<unsigned char>(*p_);
            if (c < 0x20) return false;                  // raw control characters are not JSON
            if (c != '\\') { out += *p_++; continue; }
            if (++p_ >= e_) return false;
            const char esc = *p_++;
            switch (esc) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {   // surrogate pair
                        uint32_t lo;
                        if (e_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return false;
                        p_ += 2;
                        if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    utf8(out, cp);
                    break;
                }
                default: return false;
            }
        }
        if (p_ >= e_) return false;
        ++p_;
        return true;
    }
    bool number(std::string& out) {
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') ++p_;
        if (p_ >= e_ || !std::isdigit(static_cast<unsigned char>(*p_))) return false;
        if (*p_ == '0') ++p_;
        else while (p_ < e_ && std::isdigit(static_cast<unsigned char>(*p_))) ++p_;
        if (p_ < e_ && *p_ == '.') {
            ++p_;
            if (p_ >= e_ || !std::isdigit(static_cast<unsigned char>(*p_))) return false;
            while (p_ < e_ && std::isdigit(static_cast<unsigned char>(*p_))) ++p_;
        }
        if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
            ++p_;
            if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= e_ || !std::isdigit(static_cast<unsigned char>(*p_))) return false;
            while (p_ < e_ && std::isdigit(static_cast<unsigned char>(*p_))) ++p_;
        }
        out.assign(s, p_);
        return true;
    }
    bool value(Value& v, int depth) {
        if (depth > kMaxDepth) return false;
        ws();
        if (p_ >= e_) return false;
        switch (*p_) {
            case '{': {
                ++p_;
                v.kind = Value::Object;
                if (eat('}')) return true;
                do {
                    std::string key;
                    if (!string(key) || !eat(':')) return false;
                    v.obj.emplace_back(std::move(key), Value());
                    if (!value(v.obj.back().second, depth + 1)) return false;
                } while (eat(','));
                return eat('}');
            }
            case '[': {
                ++p_;
                v.kind = Value::Array;
                if (eat(']')) return true;
                do {
                    v.arr.emplace_back();
                    if (!value(v.arr.back(), depth + 1)) return false;
                } while (eat(','));
                return eat(']');
            }
            case '"':
                v.kind = Value::String;
                return string(v.text);
            case 't': v.kind = Value::Bool; v.b = true; return literal("true");
            case 'f': v.kind = Value::Bool; v.b = false; return literal("false");
            case 'n': v.kind = Value::Null; return literal("null");
            default:
                v.kind = Value::Number;
                return number(v.text);
        }
    }
};

// A non-negative integer that fits in 64 bits.
inline bool as_u64(const Value* v, uint64_t& out) {
    if (v == nullptr || v->kind != Value::Number || v->text.empty()) return false;
    uint64_t r = 0;
    for (char c : v->text) {
        if (c < '0' || c > '9') return false;
        const uint64_t d = static_cast<uint64_t>(c - '0');
        if (r > (UINT64_MAX - d) / 10) return false;
        r = r * 10 + d;
    }
    out = r;
    return true;
}

inline bool as_i64(const Value* v, int64_t& out) {
    if (v == nullptr || v->kind != Value::Number) return false;
    const bool neg = !v->text.empty() && v->text[0] == '-';
    Value mag;
    mag.kind = Value::Number;
    mag.text = neg ? v->text.substr(1) : v->text;
    uint64_t u;
    if (!as_u64(&mag, u) || u > static_cast<uint64_t>(INT64_MAX)) return false;
    out = neg ? -static_cast<int64_t>(u) : static_cast<int64_t>(u);
    return true;
}

inline bool as_double(const Value* v, double& out) {
    if (v == nullptr || v->kind != Value::Number) return false;
    out = std::strtod(v->text.c_str(), nullptr);
    return true;
}

}  // namespace json

// ── safetensors header ──────────────────────────────────────────────────────
namespace ckpt {

struct TensorMeta {
    std::string name;
    int32_t dtype = -1;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

// Safetensors dtype names the reference accepts (include/servoflow/core/
// dtype.h:59-67, the "F32"-style spellings) → SFB dtype codes; -1 otherwise.
inline int32_t dtype_code(const std::string& s) {
    if (s == "F32") return SFB_F32;
    if (s == "F16") return SFB_F16;
    if (s == "BF16") return SFB_BF16;
    if (s == "I8") return SFB_I8;
    if (s == "I4") return 4;
    if (s == "I32") return SFB_I32;
    if (s == "BOOL") return SFB_BOOL;
    return -1;
}

inline int64_t dtype_bytes(int32_t dt) {
    switch (dt) {
        case SFB_F32: case SFB_I32: return 4;
        case SFB_F16: case SFB_BF16: return 2;
        case SFB_I8: case SFB_BOOL: return 1;
        default: return 0;                               // I4: packed, not uploadable here
    }
}

// Element count, or -1 when it does not fit in 63 bits.
inline int64_t numel(const std::vector<int64_t>& shape) {
    int64_t n = 1;
    for (int64_t d : shape) {
        if (d > 0 && n > INT64_MAX / d) return -1;
        n *= d;
    }
    return n;
}

// Read-only mapping of a whole file.
class MappedFile {
public:
    MappedFile() = default;
    MappedFile(const MappedFile&) = delete;
    MappedFile& operator=(const MappedFile&) = delete;
    ~MappedFile() {
        if (data_ != nullptr && size_ > 0) ::munmap(const_cast<char*>(data_), size_);
        if (fd_ >= 0) ::close(fd_);
    }
    int open(const char* path) {
        fd_ = ::open(path, O_RDONLY);
        if (fd_ < 0) return fail(SFB_ERR_IO, std::string("cannot open ") + path + ": " + std::strerror(errno));
        struct stat st {};
        if (::fstat(fd_, &st) != 0) return fail(SFB_ERR_IO, std::string("cannot stat ") + path);
        size_ = static_cast<size_t>(st.st_size);
        if (size_ == 0) return SFB_OK;
        void* p = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (p == MAP_FAILED) return fail(SFB_ERR_IO, std::string("cannot map ") + path);
        data_ = static_cast<const char*>(p);
        return SFB_OK;
    }
    const char* data() const { return data_; }
    size_t size() const { return size_; }

private:
    int fd_ = -1;
    const char* data_ = nullptr;
    size_t size_ = 0;
};

// Parses the header of a mapped safetensors file: entries sorted by name,
// *data_offset = 8 + header length (start of the data section).
inline int parse_header(const char* data, size_t size, std::vector<TensorMeta>& out, uint64_t* data_offset) {
    if (size < 8) return fail(SFB_ERR_IO, "safetensors: file too small");
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | static_cast<unsigned char>(data[i]);
    if (hlen > size - 8) return fail(SFB_ERR_IO, "safetensors: header length exceeds the file size");
    json::Value root;
    json::Parser parser(data + 8, data + 8 + hlen);
    if (!parser.document(root) || root.kind != json::Value::Object)
        return fail(SFB_ERR_IO, "safetensors: malformed JSON header");
    std::map<std::string, TensorMeta> sorted;
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const json::Value& info = kv.second;
        TensorMeta m;
        m.name = kv.first;
        const json::Value* dt = info.get("dtype");
        const json::Value* shape = info.get("shape");
        const json::Value* offs = info.get("data_offsets");
        if (info.kind != json::Value::Object || dt == nullptr || dt->kind != json::Value::String ||
            shape == nullptr || shape->kind != json::Value::Array || offs == nullptr ||
            offs->kind != json::Value::Array || offs->arr.size() != 2)
            return fail(SFB_ERR_IO, "safetensors: malformed entry '" + m.name + "'");
        m.dtype = dtype_code(dt->text);
        if (m.dtype < 0) return fail(SFB_ERR_DTYPE, "safetensors: unrecognised dtype '" + dt->text + "'");
        for (const auto& d : shape->arr) {
            int64_t v;
            if (!json::as_i64(&d, v) || v < 0)
                return fail(SFB_ERR_IO, "safetensors: bad shape of '" + m.name + "'");
            m.shape.push_back(v);
        }
        if (!json::as_u64(&offs->arr[0], m.begin) || !json::as_u64(&offs->arr[1], m.end))
            return fail(SFB_ERR_IO, "safetensors: bad data_offsets of '" + m.name + "'");
        sorted[m.name] = std::move(m);
    }
    out.clear();
    for (auto& kv : sorted) out.push_back(std::move(kv.second));
    *data_offset = 8 + hlen;
    return SFB_OK;
}

inline bool starts_with(const std::string& s, const char* p) { return s.rfind(p, 0) == 0; }

// hf_to_servoflow.py:41-66. Returns false for entries the converter drops.
inline bool remap_key(const std::string& k, std::string& out) {
    if (k.find(".shadow_params") != std::string::npos || starts_with(k, "ema_model.")) return false;
    if (k.find("optimizer") != std::string::npos || k.find("scheduler") != std::string::npos) return false;
    if (starts_with(k, "model.")) { out = k.substr(6); return true; }
    if (starts_with(k, "lang_adaptor.") || starts_with(k, "img_adaptor.") || starts_with(k, "state_adaptor.") ||
        starts_with(k, "action_norm.")) {
        out = k;
        return true;
    }
    return false;
}

// ── device conversion kernels ───────────────────────────────────────────────
template <typename S> __device__ __forceinline__ float to_f32(S v) { return static_cast<float>(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// One block per output row (the same method as the model's seeded init).
// A NaN or infinite weight has no int8 value (fmaxf would skip a NaN and an
// infinity would zero the rest of its row): such rows are counted in *bad and
// the load fails.
template <typename S>
__global__ void quantize_rows_kernel(const S* __restrict__ w, int8_t* __restrict__ q, float* __restrict__ s,
                                     int K, int* __restrict__ bad) {
    const int r = blockIdx.x;
    const S* row = w + static_cast<int64_t>(r) * K;
    __shared__ float red[32];
    float mx = 0.f;
    bool finite = true;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = to_f32(row[k]);
        finite = finite && isfinite(v);
        mx = fmaxf(mx, fabsf(v));
    }
    if (__any_sync(0xffffffffu, !finite) && (threadIdx.x & 31) == 0) atomicAdd(bad, 1);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        mx = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (threadIdx.x == 0) red[0] = mx;
    }
    __syncthreads();
    const float sc = red[0] > 0.f ? red[0] / 127.f : 1.f;
    if (threadIdx.x == 0) s[r] = sc;
    for (int k = threadIdx.x; k < K; k += blockDim.x)
        q[static_cast<int64_t>(r) * K + k] =
            static_cast<int8_t>(fminf(127.f, fmaxf(-127.f, rintf(to_f32(row[k]) / sc))));
}

template <typename S, typename D> __device__ __forceinline__ D from_f32(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<float, __nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ float from_f32<float, float>(float v) { return v; }

template <typename S, typename D>
__global__ void convert_kernel(const S* __restrict__ in, D* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = from_f32<float, D>(to_f32(in[i]));
}

}  // namespace ckpt

namespace rdt {

struct LoadStats {
    int64_t loaded = 0, ignored = 0;
};

// Loads one safetensors file into the model. `once`, if given, holds the
// parameters already written during the current multi-file load: the first
// file to provide a parameter keeps it (the reference merges shards with
// std::unordered_map::merge, which keeps existing keys).
static int load_file(Model& m, const char* path, LoadStats& st, std::set<std::string>* once) {
    using namespace ckpt;
    MappedFile f;
    SFB_TRY(f.open(path));
    std::vector<TensorMeta> metas;
    uint64_t data_off = 0;
    SFB_TRY(parse_header(f.data(), f.size(), metas, &data_off));

    enum Kind { kCopy, kQuant, kToBf16, kToF32 };
    struct Job {
        const TensorMeta* t;
        Kind kind;
        std::string name, name2;                         // target parameter(s)
        void* dst;
        void* dst2;
        int64_t rows, cols;
    };
    auto param = [&](const std::string& n) -> const std::pair<void*, std::pair<int64_t, int32_t>>* {
        auto it = m.params.find(n);
        return it == m.params.end() ? nullptr : &it->second;
    };
    auto is_float = [](int32_t dt) { return dt == SFB_F32 || dt == SFB_F16 || dt == SFB_BF16; };
    std::vector<Job> jobs;
    size_t staging = 0;
    for (const TensorMeta& t : metas) {
        // the name as stored, else as the reference's converter maps it
        std::string name = t.name;
        auto resolves = [&](const std::string& n) {
            return param(n) != nullptr ||
                   (n.size() > 7 && n.compare(n.size() - 7, 7, ".weight") == 0 && param(n + "_q") != nullptr);
        };
        if (!resolves(name)) {
            std::string mapped;
            if (!remap_key(name, mapped) || !resolves(mapped)) { ++st.ignored; continue; }
            name = mapped;
        }
        if (t.end < t.begin || t.end > f.size() - data_off)
            return fail(SFB_ERR_IO, "safetensors: data out of bounds for tensor '" + t.name + "'");
        const int64_t eb = dtype_bytes(t.dtype);
        const int64_t n = numel(t.shape);
        if (eb == 0) return fail(SFB_ERR_DTYPE, "checkpoint: tensor '" + t.name + "' has a packed dtype");
        if (n < 0 || n > INT64_MAX / eb || static_cast<uint64_t>(n * eb) != t.end - t.begin)
            return fail(SFB_ERR_SHAPE, "checkpoint: byte size of '" + t.name + "' does not match its shape");
        Job j{&t, kCopy, name, "", nullptr, nullptr, 0, 0};
        if (const auto* p = param(name)) {
            const int32_t pdt = p->second.second;
            if (n != p->second.first)
                return fail(SFB_ERR_SHAPE, "checkpoint: '" + t.name + "' has " + std::to_string(n) +
                                               " elements, the model's '" + name + "' " +
                                               std::to_string(p->second.first));
            j.dst = p->first;
            if (t.dtype == pdt) j.kind = kCopy;
            else if (pdt == SFB_BF16 && is_float(t.dtype)) j.kind = kToBf16;
            else if (pdt == SFB_F32 && is_float(t.dtype)) j.kind = kToF32;
            else return fail(SFB_ERR_DTYPE, "checkpoint: '" + t.name + "' cannot be converted to the model's dtype");
        } else {                                         // float weight of an int8 projection
            const auto* q = param(name + "_q");
            const std::string base = name.substr(0, name.size() - 7);
            const auto* s = param(base + ".weight_scale");
            if (s == nullptr) return fail(SFB_ERR_INVALID, "checkpoint: no scale for '" + name + "'");
            if (!is_float(t.dtype))
                return fail(SFB_ERR_DTYPE, "checkpoint: '" + t.name + "' must be a float tensor to be quantised");
            if (t.shape.size() != 2 || t.shape[0] != s->second.first || n != q->second.first)
                return fail(SFB_ERR_SHAPE, "checkpoint: '" + t.name + "' is not [" +
                                               std::to_string(s->second.first) + ", " +
                                               std::to_string(q->second.first / std::max<int64_t>(1, s->second.first)) + "]");
            j.kind = kQuant;
            j.name = name + "_q";
            j.name2 = base + ".weight_scale";
            j.dst = q->first;
            j.dst2 = s->first;
            j.rows = t.shape[0];
            j.cols = t.shape[1];
        }
        if (once != nullptr && once->count(j.name)) { ++st.ignored; continue; }
        if (j.kind != kCopy) staging = std::max(staging, static_cast<size_t>(t.end - t.begin));
        jobs.push_back(std::move(j));
    }

    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != m.device) cudaSetDevice(m.device);
    void* stage = nullptr;
    int rc = SFB_OK;
    auto cuda_ok = [&](cudaError_t e, const char* where) {
        if (e != cudaSuccess) { record_cuda_error(e, where); rc = SFB_ERR_CUDA; }
        return e == cudaSuccess;
    };
    if (staging > 0) cuda_ok(cudaMalloc(&stage, staging), "checkpoint staging buffer");
    int* bad = nullptr;                       // rows with a non-finite weight, per quantised tensor
    if (rc == SFB_OK) cuda_ok(cudaMalloc(reinterpret_cast<void**>(&bad), sizeof(int)), "checkpoint flag");
    std::string bad_name;
    for (const Job& j : jobs) {
        if (rc != SFB_OK) break;
        const TensorMeta& t = *j.t;
        const char* src = f.data() + data_off + t.begin;
        const size_t bytes = static_cast<size_t>(t.end - t.begin);
        const int64_t n = numel(t.shape);
        if (j.kind == kCopy) {
            cuda_ok(cudaMemcpy(j.dst, src, bytes, cudaMemcpyHostToDevice), "checkpoint upload");
            continue;
        }
        if (!cuda_ok(cudaMemcpy(stage, src, bytes, cudaMemcpyHostToDevice), "checkpoint upload")) break;
        if (j.kind == kQuant && !cuda_ok(cudaMemset(bad, 0, sizeof(int)), "checkpoint flag")) break;
        const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 32)));
        auto run = [&](auto* typed) {
            using S = std::remove_cv_t<std::remove_pointer_t<decltype(typed)>>;
            if (j.kind == kQuant)
                quantize_rows_kernel<S><<<static_cast<unsigned>(j.rows), 256>>>(
                    typed, static_cast<int8_t*>(j.dst), static_cast<float*>(j.dst2), static_cast<int>(j.cols), bad);
            else if (j.kind == kToBf16)
                convert_kernel<S, __nv_bfloat16><<<grid, 256>>>(typed, static_cast<__nv_bfloat16*>(j.dst), n);
            else
                convert_kernel<S, float><<<grid, 256>>>(typed, static_cast<float*>(j.dst), n);
        };
        if (t.dtype == SFB_F32) run(static_cast<const float*>(stage));
        else if (t.dtype == SFB_F16) run(static_cast<const __half*>(stage));
        else run(static_cast<const __nv_bfloat16*>(stage));
        if (!cuda_ok(cudaGetLastError(), "checkpoint conversion launch")) break;
        // the staging buffer is reused by the next tensor
        if (!cuda_ok(cudaDeviceSynchronize(), "checkpoint conversion")) break;
        if (j.kind == kQuant) {
            int nbad = 0;
            if (!cuda_ok(cudaMemcpy(&nbad, bad, sizeof(int), cudaMemcpyDeviceToHost), "checkpoint flag")) break;
            if (nbad != 0) { rc = SFB_ERR_RANGE; bad_name = t.name; break; }
        }
    }
    if (rc == SFB_OK) cuda_ok(cudaDeviceSynchronize(), "checkpoint upload");
    if (stage != nullptr) cudaFree(stage);
    if (bad != nullptr) cudaFree(bad);
    if (prev != m.device) cudaSetDevice(prev);
    if (rc == SFB_ERR_RANGE)
        return fail(rc, "checkpoint: '" + bad_name + "' holds a NaN or infinite weight (no int8 value)");
    if (rc != SFB_OK) return rc;
    for (const Job& j : jobs) {
        m.loaded.insert(j.name);
        if (!j.name2.empty()) m.loaded.insert(j.name2);
        if (once != nullptr) once->insert(j.name);
        ++st.loaded;
    }
    return SFB_OK;
}

}  // namespace rdt
}  // namespace sfb

// ── C ABI ───────────────────────────────────────────────────────────────────
using namespace sfb;

int sfb_safetensors_inspect(const char* path, sfb_tensor_info* out, int32_t capacity, int32_t* count,
                            uint64_t* data_offset) {
    if (path == nullptr || count == nullptr || capacity < 0 || (capacity > 0 && out == nullptr))
        return SFB_ERR_INVALID;
    ckpt::MappedFile f;
    SFB_TRY(f.open(path));
    std::vector<ckpt::TensorMeta> metas;
    uint64_t off = 0;
    SFB_TRY(ckpt::parse_header(f.data(), f.size(), metas, &off));
    for (const auto& m : metas)
        if (m.name.size() >= sizeof(out->name) || m.shape.size() > 8)
            return fail(SFB_ERR_SHAPE, "safetensors: entry '" + m.name + "' exceeds sfb_tensor_info");
    *count = static_cast<int32_t>(metas.size());
    if (data_offset) *data_offset = off;
    for (int32_t i = 0; i < std::min<int32_t>(capacity, *count); ++i) {
        sfb_tensor_info& t = out[i];
        std::memset(&t, 0, sizeof(t));
        std::memcpy(t.name, metas[i].name.data(), metas[i].name.size());
        t.dtype = metas[i].dtype;
        t.ndim = static_cast<int32_t>(metas[i].shape.size());
        for (int d = 0; d < t.ndim; ++d) t.shape[d] = metas[i].shape[d];
        t.data_begin = metas[i].begin;
        t.data_end = metas[i].end;
    }
    return SFB_OK;
}

int sfb_checkpoint_key(const char* name, char* out, int32_t out_len) {
    if (name == nullptr || out == nullptr || out_len < 1) return SFB_ERR_INVALID;
    std::string mapped;
    if (!ckpt::remap_key(name, mapped)) { out[0] = '\0'; return 0; }
    if (static_cast<int32_t>(mapped.size()) >= out_len) return SFB_ERR_INVALID;
    std::memcpy(out, mapped.c_str(), mapped.size() + 1);
    return 1;
}

int sfb_rdt1b_config_from_json(const char* path, sfb_rdt1b_config* cfg) {
    if (path == nullptr || cfg == nullptr) return SFB_ERR_INVALID;
    std::ifstream in(path, std::ios::binary);
    if (!in) return fail(SFB_ERR_IO, std::string("RDT1BConfig: cannot open ") + path);
    std::stringstream ss;
    ss << in.rdbuf();
    const std::string text = ss.str();
    json::Value j;
    json::Parser parser(text.data(), text.data() + text.size());
    if (!parser.document(j) || j.kind != json::Value::Object)
        return fail(SFB_ERR_IO, std::string("RDT1BConfig: malformed JSON in ") + path);
    sfb_rdt1b_config c;
    sfb_rdt1b_default_config(&c);
    int64_t train_steps = 1000, freq_dim = 256;
    double eps = 1e-6;
    bool bad = false;
    auto get = [&](const json::Value& o, const char* key, auto& field) {
        const json::Value* v = o.get(key);
        if (v == nullptr) return;
        int64_t x;
        if (!json::as_i64(v, x) || x < INT32_MIN || x > INT32_MAX) { bad = true; return; }
        field = static_cast<std::remove_reference_t<decltype(field)>>(x);
    };
    // common and converter (flat) keys, config.cpp:24-38
    get(j, "action_dim", c.action_dim);
    get(j, "pred_horizon", c.horizon);
    get(j, "img_cond_len", c.img_len);
    get(j, "img_token_dim", c.img_dim);
    get(j, "lang_token_dim", c.lang_dim);
    get(j, "max_lang_cond_len", c.max_lang_len);
    get(j, "state_token_dim", c.state_dim);
    get(j, "hidden_size", c.hidden);
    get(j, "num_hidden_layers", c.num_layers);
    get(j, "num_attention_heads", c.heads);
    get(j, "num_train_timesteps", train_steps);
    get(j, "num_inference_timesteps", c.num_steps);
    // HF nested keys, config.cpp:41-53
    if (const json::Value* r = j.get("rdt"); r != nullptr && r->kind == json::Value::Object) {
        get(*r, "hidden_size", c.hidden);
        get(*r, "depth", c.num_layers);
        get(*r, "num_heads", c.heads);
    }
    if (const json::Value* ns = j.get("noise_scheduler"); ns != nullptr && ns->kind == json::Value::Object) {
        get(*ns, "num_train_timesteps", train_steps);
        get(*ns, "num_inference_timesteps", c.num_steps);
    }
    // overrides, config.cpp:56-57
    get(j, "freq_dim", freq_dim);
    if (const json::Value* v = j.get("rms_norm_eps"); v != nullptr && !json::as_double(v, eps)) bad = true;
    if (bad) return fail(SFB_ERR_INVALID, "RDT1BConfig: a field is not an integer in range");
    if (c.heads <= 0 || c.hidden <= 0 || c.num_layers <= 0 || c.hidden % c.heads != 0)
        return fail(SFB_ERR_INVALID, "RDT1BConfig: hidden_dim must be divisible by num_heads");   // config.cpp validate()
    // what this runtime fixes at build time
    if (train_steps != 1000 || freq_dim != 256 || std::fabs(eps - 1e-6) > 1e-12)
        return fail(SFB_ERR_UNSUPPORTED,
                    "RDT1BConfig: this runtime supports num_train_timesteps 1000, freq_dim 256, rms_norm_eps 1e-6");
    *cfg = c;
    return SFB_OK;
}

int sfb_rdt1b_load_safetensors(void* handle, const char* path, int64_t* loaded, int64_t* ignored) {
    auto* m = static_cast<rdt::Model*>(handle);
    if (m == nullptr || path == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    rdt::LoadStats st;
    SFB_TRY(rdt::load_file(*m, path, st, nullptr));
    if (loaded) *loaded = st.loaded;
    if (ignored) *ignored = st.ignored;
    return SFB_OK;
}

int sfb_rdt1b_params_missing(void* handle, int64_t* missing, char* first_missing, int32_t buflen) {
    auto* m = static_cast<rdt::Model*>(handle);
    if (m == nullptr || missing == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    int64_t n = 0;
    std::string first;
    for (const auto& kv : m->params)
        if (!m->loaded.count(kv.first)) {
            if (n++ == 0) first = kv.first;
        }
    *missing = n;
    if (first_missing != nullptr && buflen > 0) {
        const size_t k = std::min<size_t>(first.size(), static_cast<size_t>(buflen - 1));
        std::memcpy(first_missing, first.data(), k);
        first_missing[k] = '\0';
    }
    return SFB_OK;
}

int sfb_rdt1b_load_checkpoint(void* handle, const char* dir, int64_t* loaded, int64_t* ignored) {
    auto* m = static_cast<rdt::Model*>(handle);
    if (m == nullptr || dir == nullptr) return SFB_ERR_INVALID;
    SFB_MODEL_ENTRY(m);
    DIR* d = ::opendir(dir);
    if (d == nullptr) return fail(SFB_ERR_IO, std::string("checkpoint directory not found: ") + dir);
    std::vector<std::string> files;
    while (const dirent* e = ::readdir(d)) {
        const std::string n = e->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(n);
    }
    ::closedir(d);
    if (files.empty()) return fail(SFB_ERR_IO, std::string("no safetensors files found in: ") + dir);
    std::sort(files.begin(), files.end());
    rdt::LoadStats st;
    std::set<std::string> once;
    for (const auto& n : files) SFB_TRY(rdt::load_file(*m, (std::string(dir) + "/" + n).c_str(), st, &once));
    if (loaded) *loaded = st.loaded;
    if (ignored) *ignored = st.ignored;
    for (const auto& kv : m->params)                     // load_weight_from_map: a missing key is an error
        if (!once.count(kv.first) && !(kv.first.size() > 13 &&
                                       kv.first.compare(kv.first.size() - 13, 13, ".weight_scale") == 0 &&
                                       once.count(kv.first.substr(0, kv.first.size() - 13) + ".weight_q")))
            return fail(SFB_ERR_INVALID, "checkpoint: missing key '" + kv.first + "'");
    return SFB_OK;
}
