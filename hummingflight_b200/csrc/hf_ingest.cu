// hf_ingest.cu -- safetensors shards into resident HBM weights (host code).
//
// Parsing (SafeTensorsFile::open, model/safetensors.cpp:52-223): 8-byte
// little-endian header length, a JSON object header, one entry per tensor
// {dtype, shape, data_offsets}; the same validation rules and rejection
// counters as the reference, with a small JSON reader of our own (the
// reference uses picojson). Where picojson decides the outcome, the reader
// does the same: numbers are spelled and valued as picojson reads them ("08"
// and "16." are numbers, 4.0 is a valid size), data offsets are truncated as
// the reference's uint64_t conversion does, a repeated key keeps its last
// value, text after the header object is ignored.
//
// Copying (what ExpertGpuCache's pinned ping-pong staging does per expert,
// compute/cuda_backend.cpp:190-364, done for a whole layer at once): the
// tensors' byte ranges are cut into chunks of at most kChunk bytes; reader
// threads each own two pinned buffers and a stream, pread a chunk into a free
// buffer and queue its host-to-device copy straight to the tensor's final
// device address, so file reads, DMA and the other threads overlap. A buffer is
// reused only after the event of its previous copy has completed.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <filesystem>
#include <fstream>
#include <set>
#include <chrono>
#include <clocale>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "hf_ctx.cuh"
#include "hf_ingest.h"

namespace hf {
namespace {

// ------------------------------------------------------------------ JSON
struct JVal {
    enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
    bool neg = false;      // Int: sign
    uint64_t u = 0;        // Int: magnitude
    double num = 0;        // Num (and Int as a double)
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;  // in order, duplicates kept
};

class JsonReader {
public:
    JsonReader(const char* p, size_t n) : p_(p), e_(p + n) {}
    // One JSON value; what follows it is not examined (picojson::parse, which
    // the reference uses, stops there too).
    bool parse(JVal& v) {
        ws();
        return value(v, 0);
    }

private:
    const char* p_;
    const char* e_;
    static constexpr int kMaxDepth = 64;

    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* s) {
        const size_t n = std::strlen(s);
        if (size_t(e_ - p_) < n || std::memcmp(p_, s, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void utf8(std::string& s, uint32_t c) {
        if (c < 0x80) {
            s += char(c);
        } else if (c < 0x800) {
            s += char(0xC0 | (c >> 6));
            s += char(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            s += char(0xE0 | (c >> 12));
            s += char(0x80 | ((c >> 6) & 0x3F));
            s += char(0x80 | (c & 0x3F));
        } else {
            s += char(0xF0 | (c >> 18));
            s += char(0x80 | ((c >> 12) & 0x3F));
            s += char(0x80 | ((c >> 6) & 0x3F));
            s += char(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t& c) {
        if (e_ - p_ < 4) return false;
        c = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = *p_++;
            c <<= 4;
            if (h >= '0' && h <= '9') c |= uint32_t(h - '0');
            else if (h >= 'a' && h <= 'f') c |= uint32_t(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') c |= uint32_t(h - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string& s) {
        if (p_ >= e_ || *p_ != '"') return false;
        ++p_;
        while (p_ < e_) {
            const unsigned char ch = static_cast<unsigned char>(*p_++);
            if (ch == '"') return true;
            if (ch < 0x20) return false;  // control characters must be escaped
            if (ch != '\\') {
                s += char(ch);
                continue;
            }
            if (p_ >= e_) return false;
            const char esc = *p_++;
            switch (esc) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    uint32_t c;
                    if (!hex4(c)) return false;
                    if (c >= 0xD800 && c < 0xDC00) {  // surrogate pair
                        uint32_t lo;
                        if (e_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return false;
                        p_ += 2;
                        if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        c = 0x10000 + ((c - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (c >= 0xDC00 && c < 0xE000) {
                        return false;
                    }
                    utf8(s, c);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    // Numbers follow picojson's reading, which decides what the reference
    // accepts: a number starts with a digit or '-', runs over the characters
    // [0-9+-eE.], and is valid when strtod consumes the whole run -- so "08",
    // "16." and "-.5" are numbers and "1e" is not. A number beyond the double
    // range makes the header invalid (picojson throws on it, so the reference
    // cannot open such a file). A run of digits (with an optional '-') also
    // keeps its exact integer value.
    static bool num_char(char c) {
        return (c >= '0' && c <= '9') || c == '+' || c == '-' || c == 'e' || c == 'E' || c == '.';
    }
    bool number(JVal& v) {
        if (p_ >= e_ || !((*p_ >= '0' && *p_ <= '9') || *p_ == '-')) return false;
        const char* s = p_;
        while (p_ < e_ && num_char(*p_)) ++p_;
        // '.' becomes the C library's decimal point for strtod, as in picojson
        // (the host program may have set a locale that writes decimals with ',')
        std::string run;
        for (const char* q = s; q < p_; ++q) {
            if (*q == '.') run += std::localeconv()->decimal_point;
            else run += *q;
        }
        char* end = nullptr;
        v.num = std::strtod(run.c_str(), &end);
        if (end != run.c_str() + run.size() || !std::isfinite(v.num)) return false;
        const bool neg = run[0] == '-';
        bool digits = run.size() > (neg ? 1u : 0u), overflow = false;
        uint64_t u = 0;
        for (size_t i = neg ? 1 : 0; i < run.size() && digits; ++i) {
            if (run[i] < '0' || run[i] > '9') {
                digits = false;
                break;
            }
            const uint64_t d = uint64_t(run[i] - '0');
            if (u > (UINT64_MAX - d) / 10) overflow = true;
            else u = u * 10 + d;
        }
        if (digits && !overflow) {
            v.kind = JVal::Int;
            v.neg = neg;
            v.u = u;
        } else {
            v.kind = JVal::Num;
        }
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > kMaxDepth || p_ >= e_) return false;
        switch (*p_) {
            case '{': {
                ++p_;
                v.kind = JVal::Obj;
                ws();
                if (p_ < e_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                for (;;) {
                    ws();
                    std::string key;
                    if (!string(key)) return false;
                    ws();
                    if (p_ >= e_ || *p_ != ':') return false;
                    ++p_;
                    ws();
                    v.obj.emplace_back(std::move(key), JVal{});
                    if (!value(v.obj.back().second, depth + 1)) return false;
                    ws();
                    if (p_ < e_ && *p_ == ',') {
                        ++p_;
                        continue;
                    }
                    if (p_ < e_ && *p_ == '}') {
                        ++p_;
                        return true;
                    }
                    return false;
                }
            }
            case '[': {
                ++p_;
                v.kind = JVal::Arr;
                ws();
                if (p_ < e_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                for (;;) {
                    ws();
                    v.arr.emplace_back();
                    if (!value(v.arr.back(), depth + 1)) return false;
                    ws();
                    if (p_ < e_ && *p_ == ',') {
                        ++p_;
                        continue;
                    }
                    if (p_ < e_ && *p_ == ']') {
                        ++p_;
                        return true;
                    }
                    return false;
                }
            }
            case '"':
                v.kind = JVal::Str;
                return string(v.str);
            case 't':
                v.kind = JVal::Bool;
                v.num = 1;
                return lit("true");
            case 'f':
                v.kind = JVal::Bool;
                return lit("false");
            case 'n':
                v.kind = JVal::Null;
                return lit("null");
            default:
                return number(v);
        }
    }
};

// ------------------------------------------------------------------ safetensors
size_t dtype_bytes(const std::string& d) {
    static const std::map<std::string, size_t> k = {
        {"F64", 8}, {"F32", 4}, {"F16", 2}, {"BF16", 2}, {"I64", 8}, {"I32", 4},
        {"I16", 2}, {"I8", 1},  {"U64", 8}, {"U32", 4}, {"U8", 1},  {"BOOL", 1}};
    auto it = k.find(d);
    return it == k.end() ? 0 : it->second;
}

constexpr uint64_t kMaxHeader = 100ull << 20;  // the format's own header limit

// A JSON number used as a size: a non-negative integral value (4, 4.0, 4e0,
// -0 all read as the reference's doubles do).
bool as_size(const JVal& v, uint64_t& out) {
    if (v.kind == JVal::Int) {
        if (v.neg && v.u != 0) return false;
        out = v.u;
        return true;
    }
    if (v.kind != JVal::Num || !(v.num >= 0.0) || v.num != std::floor(v.num) ||
        v.num > 9007199254740992.0)
        return false;
    out = uint64_t(v.num);
    return true;
}

// A data offset as the reference converts it (uint64_t of the parsed double):
// truncated toward zero, so 16.9 is 16 and -0.5 is 0. Values whose truncation
// is negative or past 2^64 have no defined conversion there and are rejected.
bool as_offset(const JVal& v, uint64_t& out) {
    if (v.kind == JVal::Int) {
        if (v.neg && v.u != 0) return false;
        out = v.u;
        return true;
    }
    if (v.kind != JVal::Num || !(v.num > -1.0) || !(v.num < 18446744073709551616.0)) return false;
    out = uint64_t(v.num);
    return true;
}

struct StTensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // relative to the data area
};

}  // namespace
}  // namespace hf

struct hf_st_file {
    std::string path;
    int fd = -1;
    uint64_t file_size = 0;
    uint64_t data_start = 0;  // 8 + header length
    std::vector<hf::StTensor> tensors;
    std::unordered_map<std::string, int> index;
};

namespace hf {
namespace {

hf_status st_parse(hf_st_file* f, const hf_st_options& o, hf_st_stats& s) {
    struct stat sb;
    if (fstat(f->fd, &sb) != 0) return fail(HF_ERR_ARG, "safetensors: cannot stat " + f->path);
    f->file_size = uint64_t(sb.st_size);
    uint64_t hlen = 0;
    if (pread(f->fd, &hlen, 8, 0) != 8)
        return fail(HF_ERR_ARG, "safetensors: cannot read the header length of " + f->path);
    if (o.require_aligned_header && hlen % 8)
        return fail(HF_ERR_ARG, "safetensors: header length not a multiple of 8: " + f->path);
    // the reference also wants at least 8 bytes after the header
    // (safetensors.cpp:79-82: headerSize_ + 8 > fileSize_ fails)
    if (hlen > kMaxHeader || 16 + hlen > f->file_size)
        return fail(HF_ERR_ARG, "safetensors: header exceeds the file: " + f->path);
    f->data_start = 8 + hlen;
    std::string hdr(hlen, '\0');
    if (hlen && pread(f->fd, hdr.data(), hlen, 8) != ssize_t(hlen))
        return fail(HF_ERR_ARG, "safetensors: cannot read the header of " + f->path);
    JVal root;
    if (!JsonReader(hdr.data(), hdr.size()).parse(root))
        return fail(HF_ERR_ARG, "safetensors: header is not valid JSON: " + f->path);
    if (root.kind != JVal::Obj)
        return fail(HF_ERR_ARG, "safetensors: header is not a JSON object: " + f->path);
    // a key given twice keeps its last value, as the reference's JSON object
    // (a std::map filled in order) does
    std::unordered_map<std::string, size_t> last;
    for (size_t i = 0; i < root.obj.size(); ++i) last[root.obj[i].first] = i;
    for (size_t i = 0; i < root.obj.size(); ++i) {
        const auto& kv = root.obj[i];
        const std::string& name = kv.first;
        if (last[name] != i) continue;
        if (name.empty() || name[0] == '_') continue;  // __metadata__
        ++s.total;
        const auto reject = [&s](uint64_t& why) {
            ++s.rejected;
            ++why;
        };
        if (kv.second.kind != JVal::Obj) {
            reject(s.shape_rejected);
            continue;
        }
        const JVal *jd = nullptr, *js = nullptr, *jo = nullptr;
        for (const auto& f2 : kv.second.obj) {
            if (f2.first == "dtype") jd = &f2.second;
            else if (f2.first == "shape") js = &f2.second;
            else if (f2.first == "data_offsets") jo = &f2.second;
        }
        StTensor t;
        t.name = name;
        if (jd && jd->kind == JVal::Str) t.dtype = jd->str;
        const size_t eb = dtype_bytes(t.dtype);
        if (!eb) {
            reject(s.dtype_rejected);
            continue;
        }
        if (o.require_bf16 && t.dtype != "BF16") {
            bool ok = false;
            if (t.dtype == "F32")
                for (int i = 0; i < o.num_allow_f32 && !ok; ++i)
                    ok = o.allow_f32[i] && name.find(o.allow_f32[i]) != std::string::npos;
            if (!ok) {
                reject(s.dtype_rejected);
                continue;
            }
            ++s.f32_allowed_accepted;
        }
        bool shape_ok = js && js->kind == JVal::Arr && !js->arr.empty();
        uint64_t numel = 1;
        if (shape_ok) {
            for (const JVal& d : js->arr) {
                uint64_t u = 0;
                if (!as_size(d, u) || u > (1ull << 30)) {
                    shape_ok = false;
                    break;
                }
                t.shape.push_back(int64_t(u));
                // a product past 2^64 would wrap and could then match the byte
                // span by accident: such a shape describes no tensor (the
                // reference's size_t product wraps here; this parser rejects)
                if (u != 0 && numel > UINT64_MAX / u) {
                    shape_ok = false;
                    break;
                }
                numel *= u;
            }
        }
        if (!shape_ok) {
            reject(s.shape_rejected);
            continue;
        }
        if (!jo || jo->kind != JVal::Arr || jo->arr.size() != 2 ||
            !as_offset(jo->arr[0], t.begin) || !as_offset(jo->arr[1], t.end) || t.end <= t.begin) {
            reject(s.bounds_rejected);
            continue;
        }
        if (t.end > f->file_size - f->data_start) {
            reject(s.bounds_rejected);
            continue;
        }
        if (o.require_aligned_data && (f->data_start + t.begin) % 8) {
            reject(s.alignment_rejected);
            continue;
        }
        if (numel * eb != t.end - t.begin) {
            reject(s.byte_mismatch_rejected);
            continue;
        }
        if (f->index.count(name)) {
            reject(s.duplicate_rejected);
            continue;
        }
        f->index.emplace(name, int(f->tensors.size()));
        f->tensors.push_back(std::move(t));
        ++s.accepted;
    }
    return HF_OK;
}

// ------------------------------------------------------------------ pinned ring
constexpr uint64_t kChunk = 16ull << 20;  // bytes per pread + copy
constexpr int kSlotsPerThread = 2;

struct Staging {
    std::mutex mu;  // one upload at a time owns the ring
    std::vector<void*> bufs;
    int threads = 0;
};
Staging& staging() {
    static Staging s;
    return s;
}

int reader_threads() {
    const unsigned hw = std::thread::hardware_concurrency();
    return int(std::max(1u, std::min(8u, hw ? hw / 2 : 1u)));
}

struct Copy {
    int fd;
    uint64_t off;   // absolute file offset
    void* dst;      // device address
    uint64_t bytes;
};

// Copies every range to the device; returns when all bytes have landed.
hf_status upload(int device, const std::vector<Copy>& copies) {
    std::vector<Copy> chunks;
    for (const Copy& c : copies)
        for (uint64_t o = 0; o < c.bytes; o += kChunk)
            chunks.push_back({c.fd, c.off + o, static_cast<uint8_t*>(c.dst) + o,
                              std::min(kChunk, c.bytes - o)});
    if (chunks.empty()) return HF_OK;
    Staging& S = staging();
    std::lock_guard<std::mutex> lk(S.mu);
    if (S.bufs.empty()) {
        S.threads = reader_threads();
        for (int i = 0; i < S.threads * kSlotsPerThread; ++i) {
            void* p = nullptr;
            if (cudaHostAlloc(&p, kChunk, cudaHostAllocPortable) != cudaSuccess) {
                cudaGetLastError();
                for (void* q : S.bufs) cudaFreeHost(q);
                S.bufs.clear();
                return fail(HF_ERR_OOM, "ingest: cannot allocate pinned staging");
            }
            S.bufs.push_back(p);
        }
    }
    const int R = std::min<int>(S.threads, int(chunks.size()));
    std::atomic<size_t> next{0};
    std::atomic<bool> failed{false};
    std::mutex emu;
    std::string emsg;
    hf_status ecode = HF_OK;
    auto work = [&](int tid) {
        auto bad = [&](hf_status code, const std::string& m) {
            std::lock_guard<std::mutex> g(emu);
            if (ecode == HF_OK) {
                ecode = code;
                emsg = m;
            }
            failed = true;
        };
        if (cudaSetDevice(device) != cudaSuccess) return bad(HF_ERR_CUDA, "ingest: cudaSetDevice");
        cudaStream_t st = nullptr;
        cudaEvent_t ev[kSlotsPerThread] = {};
        bool used[kSlotsPerThread] = {};
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess)
            return bad(HF_ERR_CUDA, "ingest: stream");
        for (auto& e : ev)
            if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
                bad(HF_ERR_CUDA, "ingest: event");
        int slot = 0;
        while (!failed) {
            const size_t i = next.fetch_add(1);
            if (i >= chunks.size()) break;
            const Copy& c = chunks[i];
            void* buf = S.bufs[size_t(tid) * kSlotsPerThread + slot];
            if (used[slot] && cudaEventSynchronize(ev[slot]) != cudaSuccess) {
                bad(HF_ERR_CUDA, "ingest: copy failed");
                break;
            }
            uint64_t got = 0;
            while (got < c.bytes) {
                const ssize_t r = pread(c.fd, static_cast<uint8_t*>(buf) + got, c.bytes - got,
                                        off_t(c.off + got));
                if (r <= 0) break;
                got += uint64_t(r);
            }
            if (got != c.bytes) {
                bad(HF_ERR_ARG, "ingest: short read (file changed or truncated)");
                break;
            }
            if (cudaMemcpyAsync(c.dst, buf, c.bytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaEventRecord(ev[slot], st) != cudaSuccess) {
                bad(HF_ERR_CUDA, "ingest: cudaMemcpyAsync");
                break;
            }
            used[slot] = true;
            slot = (slot + 1) % kSlotsPerThread;
        }
        if (cudaStreamSynchronize(st) != cudaSuccess) bad(HF_ERR_CUDA, "ingest: copy failed");
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
        cudaStreamDestroy(st);
    };
    std::vector<std::thread> th;
    for (int t = 1; t < R; ++t) th.emplace_back(work, t);
    work(0);
    for (auto& t : th) t.join();
    if (ecode != HF_OK) return fail(ecode, emsg);
    return HF_OK;
}

hf_st_options strict_options() {
    static const char* const kAllow[] = {"e_score_correction_bias"};
    hf_st_options o{};
    o.require_bf16 = 1;
    o.allow_f32 = kAllow;
    o.num_allow_f32 = 1;
    o.require_aligned_header = 1;
    o.require_aligned_data = 1;
    return o;
}

bool shape_is(const StTensor& t, std::initializer_list<int64_t> s) {
    return t.shape.size() == s.size() && std::equal(s.begin(), s.end(), t.shape.begin());
}

}  // namespace
}  // namespace hf

using namespace hf;

extern "C" {

hf_status hf_st_open(const char* path, const hf_st_options* opts, hf_st_file** out,
                     hf_st_stats* stats) {
    if (!path || !out) return fail(HF_ERR_ARG, "hf_st_open: null argument");
    *out = nullptr;
    auto* f = new hf_st_file();
    f->path = path;
    f->fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (f->fd < 0) {
        delete f;
        return fail(HF_ERR_ARG, std::string("hf_st_open: cannot open ") + path);
    }
    hf_st_stats s{};
    const hf_status r = st_parse(f, opts ? *opts : strict_options(), s);
    if (stats) *stats = s;
    if (r != HF_OK) {
        ::close(f->fd);
        delete f;
        return r;
    }
    posix_fadvise(f->fd, 0, 0, POSIX_FADV_SEQUENTIAL);
    *out = f;
    return HF_OK;
}

hf_status hf_st_close(hf_st_file* f) {
    if (!f) return HF_OK;
    if (f->fd >= 0) ::close(f->fd);
    delete f;
    return HF_OK;
}

int hf_st_count(const hf_st_file* f) { return f ? int(f->tensors.size()) : 0; }

hf_status hf_st_tensor(const hf_st_file* f, int i, const char** name, const char** dtype,
                       int* ndim, int64_t* shape, int shape_cap, uint64_t* file_offset,
                       uint64_t* bytes) {
    if (!f || i < 0 || i >= int(f->tensors.size())) return fail(HF_ERR_ARG, "hf_st_tensor: index");
    const StTensor& t = f->tensors[size_t(i)];
    if (name) *name = t.name.c_str();
    if (dtype) *dtype = t.dtype.c_str();
    if (ndim) *ndim = int(t.shape.size());
    if (shape)
        for (size_t d = 0; d < t.shape.size() && int(d) < shape_cap; ++d) shape[d] = t.shape[d];
    if (file_offset) *file_offset = f->data_start + t.begin;
    if (bytes) *bytes = t.end - t.begin;
    return HF_OK;
}

int hf_st_find(const hf_st_file* f, const char* name) {
    if (!f || !name) return -1;
    auto it = f->index.find(name);
    return it == f->index.end() ? -1 : it->second;
}

hf_status hf_st_read(const hf_st_file* f, int i, void* host_dst, uint64_t capacity) {
    if (!f || i < 0 || i >= int(f->tensors.size()) || !host_dst)
        return fail(HF_ERR_ARG, "hf_st_read: bad argument");
    const StTensor& t = f->tensors[size_t(i)];
    const uint64_t n = t.end - t.begin;
    if (capacity < n) return fail(HF_ERR_ARG, "hf_st_read: buffer too small");
    uint64_t got = 0;
    while (got < n) {
        const ssize_t r = pread(f->fd, static_cast<uint8_t*>(host_dst) + got, n - got,
                                off_t(f->data_start + t.begin + got));
        if (r <= 0) return fail(HF_ERR_ARG, "hf_st_read: short read");
        got += uint64_t(r);
    }
    return HF_OK;
}

hf_status hf_st_upload(const hf_st_file* f, int i, void* dev_dst, uint64_t capacity, int device) {
    if (!f || i < 0 || i >= int(f->tensors.size()) || !dev_dst)
        return fail(HF_ERR_ARG, "hf_st_upload: bad argument");
    const StTensor& t = f->tensors[size_t(i)];
    if (capacity < t.end - t.begin) return fail(HF_ERR_ARG, "hf_st_upload: buffer too small");
    DeviceGuard dg(device);
    return upload(device, {{f->fd, f->data_start + t.begin, dev_dst, t.end - t.begin}});
}

hf_status hf_ingest_release_staging(void) {
    Staging& S = staging();
    std::lock_guard<std::mutex> lk(S.mu);
    for (void* p : S.bufs) cudaFreeHost(p);
    S.bufs.clear();
    return HF_OK;
}

hf_status hf_st_layer_shards(const char* dir, int model_layer, char* buf, size_t buf_bytes,
                            int* num_shards) {
    namespace fs = std::filesystem;
    if (!dir || !num_shards) return fail(HF_ERR_ARG, "hf_st_layer_shards: null argument");
    *num_shards = 0;
    std::error_code ec;
    std::vector<std::string> shards;
    for (fs::directory_iterator it(dir, ec), end; !ec && it != end; it.increment(ec))
        if (it->path().extension() == ".safetensors") shards.push_back(it->path().string());
    if (ec) return fail(HF_ERR_ARG, std::string("hf_st_layer_shards: cannot list ") + dir);
    std::sort(shards.begin(), shards.end());
    if (shards.empty())
        return fail(HF_ERR_ARG, std::string("hf_st_layer_shards: no .safetensors files in ") + dir);
    std::vector<std::string> out = shards;
    // weight_map of the index, when present and well formed (weight_index.cpp:31-49)
    std::ifstream f(fs::path(dir) / "model.safetensors.index.json", std::ios::binary);
    if (f) {
        const std::string txt((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
        JVal root;
        const JVal* wm = nullptr;
        if (JsonReader(txt.data(), txt.size()).parse(root) && root.kind == JVal::Obj)
            for (const auto& kv : root.obj)
                if (kv.first == "weight_map" && kv.second.kind == JVal::Obj) wm = &kv.second;
        if (wm) {
            const std::string pre = "model.layers." + std::to_string(model_layer) + ".mlp.";
            std::set<std::string> names;
            for (const auto& kv : wm->obj)
                if (kv.second.kind == JVal::Str && kv.first.compare(0, pre.size(), pre) == 0)
                    names.insert(kv.second.str);
            if (names.empty())
                return fail(HF_ERR_ARG, "hf_st_layer_shards: the index names no tensor of model.layers." +
                                            std::to_string(model_layer) + ".mlp");
            out.clear();
            for (const std::string& n : names) {
                const std::string p = (fs::path(dir) / n).string();
                if (!std::binary_search(shards.begin(), shards.end(), p))
                    return fail(HF_ERR_ARG, "hf_st_layer_shards: the index names a missing shard: " + n);
                out.push_back(p);
            }
        }
    }
    size_t need = 0;
    for (const std::string& p : out) need += p.size() + 1;
    *num_shards = int(out.size());
    if (!buf || buf_bytes < need) return fail(HF_ERR_ARG, "hf_st_layer_shards: buffer too small");
    char* w = buf;
    for (const std::string& p : out) {
        std::memcpy(w, p.c_str(), p.size() + 1);
        w += p.size() + 1;
    }
    return HF_OK;
}

hf_status hf_moe_load_safetensors(hf_moe_ctx* ctx, int layer, int model_layer,
                                  const char* const* shard_paths, int num_shards,
                                  hf_ingest_stats* stats) {
    const auto t0 = std::chrono::steady_clock::now();
    if (!ctx) return fail(HF_ERR_ARG, "hf_moe_load_safetensors: null context");
    if (layer < 0 || layer >= int(ctx->layers.size()))
        return fail(HF_ERR_ARG, "hf_moe_load_safetensors: layer out of range");
    if (!shard_paths || num_shards <= 0)
        return fail(HF_ERR_ARG, "hf_moe_load_safetensors: no shards");
    // open every shard; a name found in two shards is an error
    std::vector<hf_st_file*> files;
    struct Closer {
        std::vector<hf_st_file*>& v;
        ~Closer() {
            for (auto* f : v) hf_st_close(f);
        }
    } closer{files};
    std::unordered_map<std::string, std::pair<const hf_st_file*, const StTensor*>> where;
    const std::string pre = "model.layers." + std::to_string(model_layer) + ".mlp.";
    for (int s = 0; s < num_shards; ++s) {
        hf_st_file* f = nullptr;
        HF_TRY(hf_st_open(shard_paths[s], nullptr, &f, nullptr));
        files.push_back(f);
        for (const StTensor& t : f->tensors) {
            if (t.name.compare(0, pre.size(), pre) != 0) continue;
            if (!where.emplace(t.name, std::make_pair(f, &t)).second)
                return fail(HF_ERR_ARG, "hf_moe_load_safetensors: " + t.name + " in two shards");
        }
    }
    const int64_t H = ctx->H, E = ctx->E, I = ctx->I, Is = ctx->Is;
    std::vector<Copy> copies;
    uint64_t total = 0;
    const auto need = [&](const std::string& name, const char* dtype,
                          std::initializer_list<int64_t> shape, void* dst,
                          bool optional) -> hf_status {
        auto it = where.find(pre + name);
        if (it == where.end()) {
            if (optional) return HF_ERR_STATE;
            return fail(HF_ERR_ARG, "hf_moe_load_safetensors: missing " + pre + name);
        }
        const StTensor& t = *it->second.second;
        if (t.dtype != dtype || !shape_is(t, shape))
            return fail(HF_ERR_ARG, "hf_moe_load_safetensors: " + t.name + " has dtype " +
                                        t.dtype + " or a shape that does not match the config");
        copies.push_back({it->second.first->fd, it->second.first->data_start + t.begin, dst,
                          t.end - t.begin});
        total += t.end - t.begin;
        return HF_OK;
    };
    DeviceGuard dg(ctx->cfg.device);
    HF_TRY(ctx_layer_alloc(ctx, layer));
    LayerBuf& L = ctx->layers[layer];
    HF_TRY(need("gate.weight", "BF16", {E, H}, L.router, false));
    const hf_status hb =
        need("gate.e_score_correction_bias", "F32", {E}, L.bias, true);
    if (hb != HF_OK && hb != HF_ERR_STATE) return hb;
    const bool has_bias = hb == HF_OK;
    int experts = 0, skipped = 0;
    for (int e = 0; e < E; ++e) {
        const std::string x = "experts." + std::to_string(e) + ".";
        const int l = local_slot(ctx, L, e);
        if (l < 0) {
            skipped += where.count(pre + x + "gate_proj.weight") ? 1 : 0;
            continue;
        }
        uint16_t* b = L.experts + size_t(l) * ctx->expert_elems;
        HF_TRY(need(x + "gate_proj.weight", "BF16", {I, H}, b, false));
        HF_TRY(need(x + "up_proj.weight", "BF16", {I, H}, b + size_t(I) * H, false));
        HF_TRY(need(x + "down_proj.weight", "BF16", {H, I}, b + size_t(2) * I * H, false));
        ++experts;
    }
    if (Is > 0) {
        const size_t n = size_t(Is) * H;
        HF_TRY(need("shared_experts.gate_proj.weight", "BF16", {Is, H}, L.shared, false));
        HF_TRY(need("shared_experts.up_proj.weight", "BF16", {Is, H}, L.shared + n, false));
        HF_TRY(need("shared_experts.down_proj.weight", "BF16", {H, Is}, L.shared + 2 * n, false));
    }
    if (!has_bias) HF_CUDA(cudaMemset(L.bias, 0, sizeof(float) * size_t(E)));
    HF_CUDA(cudaDeviceSynchronize());  // the layer's buffers exist before other streams write
    HF_TRY(upload(ctx->cfg.device, copies));
    HF_TRY(place_router(ctx, L, nullptr));  // the router rows in the layer's expert placement
    down_written(L, -1);
    L.has_bias = has_bias;
    L.loaded = true;
    if (stats) {
        stats->bytes = total;
        stats->tensors = int(copies.size());
        stats->experts = experts;
        stats->skipped_experts = skipped;
        stats->has_bias = has_bias;
        stats->seconds =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    }
    return HF_OK;
}

}  // extern "C"
