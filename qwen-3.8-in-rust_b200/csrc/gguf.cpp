// GGUF v3 reader; see gguf.h.  Buffered header parse with pread, then positional reads of tensor data.
#include "gguf.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdarg>
#include <cstring>
#include <thread>
#include <vector>

namespace qdec {

namespace {

constexpr uint32_t GGUF_MAGIC = 0x46554747u;  // "GGUF" little-endian
constexpr uint32_t DEFAULT_ALIGNMENT = 32;

[[noreturn]] void gerr(const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    throw GgufError(buf);
}

// Sequential reader over the header; errors name what was being read (gguf.rs:380-460 "header truncated").
struct HeaderReader {
    int fd;
    uint64_t file_size;
    uint64_t pos = 0;
    std::vector<uint8_t> buf;
    uint64_t buf_start = 0;

    void ensure(uint64_t n, const std::string &what) {
        if (pos + n > file_size) gerr("header truncated while reading %s", what.c_str());
        if (pos >= buf_start && pos + n <= buf_start + buf.size()) return;
        const uint64_t want = std::max<uint64_t>(n, 1 << 20);
        const uint64_t len = std::min<uint64_t>(want, file_size - pos);
        buf.resize(len);
        uint64_t got = 0;
        while (got < len) {
            ssize_t k = pread(fd, buf.data() + got, len - got, (off_t)(pos + got));
            if (k <= 0) gerr("header truncated while reading %s", what.c_str());
            got += (uint64_t)k;
        }
        buf_start = pos;
    }
    const uint8_t *take(uint64_t n, const std::string &what) {
        ensure(n, what);
        const uint8_t *p = buf.data() + (pos - buf_start);
        pos += n;
        return p;
    }
    uint8_t u8(const std::string &w) { return *take(1, w); }
    uint16_t u16(const std::string &w) { uint16_t v; memcpy(&v, take(2, w), 2); return v; }
    uint32_t u32(const std::string &w) { uint32_t v; memcpy(&v, take(4, w), 4); return v; }
    uint64_t u64(const std::string &w) { uint64_t v; memcpy(&v, take(8, w), 8); return v; }
    std::string str(const std::string &w) {
        const uint64_t len = u64(w);
        if (len > file_size) gerr("header truncated while reading %s", w.c_str());
        const uint8_t *p = take(len, w);
        return std::string(reinterpret_cast<const char *>(p), len);
    }
    GValue value(VType t, const std::string &w, int depth = 0) {
        GValue v;
        v.type = t;
        switch (t) {
        case VType::U8: v.u = u8(w); break;
        case VType::I8: v.i = (int8_t)u8(w); break;
        case VType::U16: v.u = u16(w); break;
        case VType::I16: v.i = (int16_t)u16(w); break;
        case VType::U32: v.u = u32(w); break;
        case VType::I32: v.i = (int32_t)u32(w); break;
        case VType::F32: { uint32_t b = u32(w); float f; memcpy(&f, &b, 4); v.f = f; break; }
        case VType::BOOL: v.u = u8(w) != 0; break;
        case VType::STR: v.s = str(w); break;
        case VType::U64: v.u = u64(w); break;
        case VType::I64: v.i = (int64_t)u64(w); break;
        case VType::F64: { uint64_t b = u64(w); memcpy(&v.f, &b, 8); break; }
        case VType::ARR: {
            const uint32_t et = u32(w);
            if (et > 12) gerr("unknown GGUF value type id %u while reading %s", et, w.c_str());
            if (depth > 4) gerr("array nesting too deep while reading %s", w.c_str());
            v.elem = (VType)et;
            const uint64_t count = u64(w);
            if (count > file_size) gerr("header truncated while reading %s", w.c_str());
            v.arr.reserve((size_t)std::min<uint64_t>(count, 1u << 24));
            for (uint64_t i = 0; i < count; i++) v.arr.push_back(value(v.elem, w, depth + 1));
            break;
        }
        default: gerr("unknown GGUF value type id %u while reading %s", (unsigned)t, w.c_str());
        }
        return v;
    }
};

}  // namespace

const char *vtype_name(VType t) {
    static const char *names[] = {"UINT8", "INT8", "UINT16", "INT16", "UINT32", "INT32", "FLOAT32",
                                  "BOOL", "STRING", "ARRAY", "UINT64", "INT64", "FLOAT64"};
    const unsigned i = (unsigned)t;
    return i < 13 ? names[i] : "?";
}

std::pair<uint64_t, uint64_t> ggml_block_layout(int t) {
    switch (t) {
    case 0: return {1, 4};      // F32
    case 1: return {1, 2};      // F16
    case 2: return {32, 18};    // Q4_0
    case 3: return {32, 20};    // Q4_1
    case 6: return {32, 22};    // Q5_0
    case 7: return {32, 24};    // Q5_1
    case 8: return {32, 34};    // Q8_0
    case 9: return {32, 36};    // Q8_1
    case 10: return {256, 84};  // Q2_K
    case 11: return {256, 110}; // Q3_K
    case 12: return {256, 144}; // Q4_K
    case 13: return {256, 176}; // Q5_K
    case 14: return {256, 210}; // Q6_K
    case 15: return {256, 292}; // Q8_K
    case 16: return {256, 66};
    case 17: return {256, 74};
    case 18: return {256, 98};
    case 19: return {256, 50};
    case 20: return {32, 18};
    case 21: return {256, 110};
    case 22: return {256, 82};
    case 23: return {256, 136};
    case 24: return {1, 1};
    case 25: return {1, 2};
    case 26: return {1, 4};
    case 27: return {1, 8};
    case 28: return {1, 8};
    case 29: return {256, 56};
    case 30: return {1, 2};     // BF16
    default: return {0, 0};
    }
}

long layer_of(const std::string &name) {
    if (name.compare(0, 4, "blk.") != 0) return -1;
    const size_t dot = name.find('.', 4);
    if (dot == std::string::npos || dot == 4) return -1;
    long v = 0;
    for (size_t i = 4; i < dot; i++) {
        if (name[i] < '0' || name[i] > '9') return -1;
        v = v * 10 + (name[i] - '0');
        if (v > (1L << 31)) return -1;
    }
    return v;
}

Gguf::Gguf(const std::string &path) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) gerr("io error: cannot open %s: %s", path.c_str(), strerror(errno));
    struct stat st;
    if (fstat(fd_, &st) != 0) gerr("io error: stat %s: %s", path.c_str(), strerror(errno));
    file_size_ = (uint64_t)st.st_size;
    HeaderReader r{fd_, file_size_};
    const uint32_t magic = r.u32("magic");
    if (magic != GGUF_MAGIC) gerr("not a GGUF file (magic 0x%08x)", magic);
    const uint32_t version = r.u32("version");
    if (version != 3) gerr("unsupported GGUF version %u (this reader implements version 3)", version);
    const uint64_t n_tensors = r.u64("tensor_count");
    const uint64_t n_kv = r.u64("kv_count");
    if (n_tensors > file_size_ || n_kv > file_size_) gerr("header truncated while reading counts");
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key = r.str("metadata key #" + std::to_string(i));
        const uint32_t vt = r.u32(key);
        if (vt > 12) gerr("unknown GGUF value type id %u while reading %s", vt, key.c_str());
        GValue v = r.value((VType)vt, key);
        if (kv_index_.count(key)) gerr("duplicate metadata key %s", key.c_str());
        kv_index_[key] = kv_.size();
        kv_.emplace_back(std::move(key), std::move(v));
    }
    struct Raw { std::string name; std::vector<uint64_t> dims; uint32_t type; uint64_t off; };
    std::vector<Raw> raws;
    raws.reserve((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; i++) {
        Raw t;
        t.name = r.str("tensor info #" + std::to_string(i));
        const uint32_t nd = r.u32(t.name);
        if (nd > 4) gerr("tensor %s: dimension count %u exceeds the GGUF maximum of 4", t.name.c_str(), nd);
        for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.u64(t.name));
        t.type = r.u32(t.name);
        t.off = r.u64(t.name);
        raws.push_back(std::move(t));
    }
    const uint64_t header_end = r.pos;
    auto it = kv_index_.find("general.alignment");
    if (it != kv_index_.end()) {
        const GValue &a = kv_[it->second].second;
        if (a.type != VType::U32) gerr("metadata key general.alignment has type %s, expected UINT32", vtype_name(a.type));
        alignment_ = (uint32_t)a.u;
    } else {
        alignment_ = DEFAULT_ALIGNMENT;
    }
    if (alignment_ == 0 || (alignment_ & (alignment_ - 1))) gerr("alignment %u is not a power of two", alignment_);
    data_offset_ = (header_end + alignment_ - 1) / alignment_ * alignment_;
    for (Raw &rt : raws) {
        auto lay = ggml_block_layout((int)rt.type);
        if (lay.first == 0) gerr("unknown ggml tensor type id %u for tensor %s", rt.type, rt.name.c_str());
        uint64_t n = 1;
        for (uint64_t d : rt.dims) {
            if (d != 0 && n > UINT64_MAX / d) gerr("tensor %s: element count overflows", rt.name.c_str());
            n *= d;
        }
        if (n % lay.first)
            gerr("tensor %s: element count %llu is not a multiple of block size %llu", rt.name.c_str(),
                 (unsigned long long)n, (unsigned long long)lay.first);
        TensorInfo ti;
        ti.name = rt.name;
        ti.type = (int)rt.type;
        ti.shape = rt.dims;
        ti.n_elements = n;
        ti.byte_size = n / lay.first * lay.second;
        ti.rel_offset = rt.off;
        ti.abs_offset = data_offset_ + rt.off;
        if (rt.off > file_size_ || ti.abs_offset + ti.byte_size > file_size_)
            gerr("tensor %s: data range %llu..%llu exceeds file size %llu", ti.name.c_str(),
                 (unsigned long long)ti.abs_offset, (unsigned long long)(ti.abs_offset + ti.byte_size),
                 (unsigned long long)file_size_);
        if (tensor_index_.count(ti.name)) gerr("duplicate tensor name %s", ti.name.c_str());
        tensor_index_[ti.name] = tensors_.size();
        tensors_.push_back(std::move(ti));
    }
}

Gguf::~Gguf() {
    if (fd_direct_ >= 0) ::close(fd_direct_);
    if (fd_ >= 0) ::close(fd_);
}

const GValue &Gguf::get(const std::string &key) const {
    auto it = kv_index_.find(key);
    if (it == kv_index_.end()) gerr("metadata key missing: %s", key.c_str());
    return kv_[it->second].second;
}

uint32_t Gguf::get_u32(const std::string &key) const {
    const GValue &v = get(key);
    if (v.type != VType::U32) gerr("metadata key %s has type %s, expected UINT32", key.c_str(), vtype_name(v.type));
    return (uint32_t)v.u;
}
float Gguf::get_f32(const std::string &key) const {
    const GValue &v = get(key);
    if (v.type != VType::F32) gerr("metadata key %s has type %s, expected FLOAT32", key.c_str(), vtype_name(v.type));
    return (float)v.f;
}
bool Gguf::get_bool(const std::string &key) const {
    const GValue &v = get(key);
    if (v.type != VType::BOOL) gerr("metadata key %s has type %s, expected BOOL", key.c_str(), vtype_name(v.type));
    return v.u != 0;
}
const std::string &Gguf::get_str(const std::string &key) const {
    const GValue &v = get(key);
    if (v.type != VType::STR) gerr("metadata key %s has type %s, expected STRING", key.c_str(), vtype_name(v.type));
    return v.s;
}
const GValue &Gguf::get_array(const std::string &key) const {
    const GValue &v = get(key);
    if (v.type != VType::ARR) gerr("metadata key %s has type %s, expected ARRAY", key.c_str(), vtype_name(v.type));
    return v;
}
std::vector<int32_t> Gguf::get_array_i32(const std::string &key) const {
    const GValue &a = get_array(key);
    std::vector<int32_t> out;
    for (size_t i = 0; i < a.arr.size(); i++) {
        if (a.arr[i].type != VType::I32)
            gerr("metadata key %s: array element %zu has type %s, expected INT32", key.c_str(), i, vtype_name(a.arr[i].type));
        out.push_back((int32_t)a.arr[i].i);
    }
    return out;
}

const TensorInfo &Gguf::tensor(const std::string &name) const {
    auto it = tensor_index_.find(name);
    if (it == tensor_index_.end()) gerr("tensor not found: %s", name.c_str());
    return tensors_[it->second];
}

bool Gguf::layer_span(uint32_t n, uint64_t &start, uint64_t &end) const {
    bool any = false;
    for (const TensorInfo &t : tensors_) {
        if (layer_of(t.name) != (long)n) continue;
        if (!any) start = t.abs_offset, end = t.abs_offset + t.byte_size, any = true;
        start = std::min(start, t.abs_offset);
        end = std::max(end, t.abs_offset + t.byte_size);
    }
    return any;
}

uint64_t Gguf::non_layer_bytes() const {
    uint64_t s = 0;
    for (const TensorInfo &t : tensors_)
        if (layer_of(t.name) < 0) s += t.byte_size;
    return s;
}

void Gguf::read_at(uint64_t off, void *dst, uint64_t len) const {
    uint64_t got = 0;
    uint8_t *d = static_cast<uint8_t *>(dst);
    while (got < len) {
        const uint64_t chunk = std::min<uint64_t>(len - got, 1ull << 30);
        ssize_t k = pread(fd_, d + got, chunk, (off_t)(off + got));
        if (k <= 0) gerr("io error: short read of %s at %llu", path_.c_str(), (unsigned long long)(off + got));
        got += (uint64_t)k;
    }
}

bool Gguf::open_direct() {
    if (fd_direct_ >= 0) return true;
    fd_direct_ = ::open(path_.c_str(), O_RDONLY | O_CLOEXEC | O_DIRECT);
    return fd_direct_ >= 0;
}

void Gguf::read_direct(uint64_t off, void *dst, uint64_t len) const {
    const uint64_t want = (len + DIRECT_ALIGN - 1) & ~(DIRECT_ALIGN - 1);
    uint8_t *d = static_cast<uint8_t *>(dst);
    uint64_t got = 0;
    while (got < want) {
        const uint64_t chunk = std::min<uint64_t>(want - got, 1ull << 30);
        const ssize_t k = pread(fd_direct_, d + got, chunk, (off_t)(off + got));
        if (k < 0) gerr("io error: direct read of %s at %llu: %s", path_.c_str(), (unsigned long long)(off + got), strerror(errno));
        if (k == 0) break;  // the end of the file
        got += (uint64_t)k;
        if ((uint64_t)k % DIRECT_ALIGN) break;  // a short read ends at the end of the file
    }
    if (got < len) gerr("io error: short direct read of %s at %llu", path_.c_str(), (unsigned long long)(off + got));
}

void Gguf::read_direct_parallel(uint64_t off, void *dst, uint64_t len, int threads) const {
    if (fd_direct_ < 0) gerr("io error: %s is not open for direct reads", path_.c_str());
    if (off % DIRECT_ALIGN || (uintptr_t)dst % DIRECT_ALIGN) gerr("io error: a direct read off its %llu-byte boundary",
                                                                    (unsigned long long)DIRECT_ALIGN);
    const uint64_t part_min = 16ull << 20;
    const int n = (int)std::min<uint64_t>((uint64_t)std::max(threads, 1), std::max<uint64_t>(1, len / part_min));
    const uint64_t per = ((len + n - 1) / n + DIRECT_ALIGN - 1) & ~(DIRECT_ALIGN - 1);
    std::vector<std::thread> ts;
    std::vector<std::string> errs(n);
    for (int i = 0; i < n; i++) {
        const uint64_t a = std::min<uint64_t>(len, (uint64_t)i * per), b = std::min<uint64_t>(len, a + per);
        if (a >= b) break;
        ts.emplace_back([this, off, dst, a, b, i, &errs] {
            try {
                read_direct(off + a, static_cast<uint8_t *>(dst) + a, b - a);
            } catch (const std::exception &e) {
                errs[i] = e.what();
            }
        });
    }
    for (std::thread &t : ts) t.join();
    for (const std::string &e : errs)
        if (!e.empty()) throw GgufError(e);
}

void Gguf::read_at_parallel(uint64_t off, void *dst, uint64_t len, int threads) const {
    // contiguous parts of >= 16 MiB on 4 KiB boundaries, one positional read loop per thread (page-cache copies
    // and NVMe queues both scale with readers); the first error is rethrown after every part has finished
    const uint64_t part_min = 16ull << 20;
    int n = (int)std::min<uint64_t>((uint64_t)std::max(threads, 1), std::max<uint64_t>(1, len / part_min));
    if (n <= 1) {
        read_at(off, dst, len);
        return;
    }
    const uint64_t per = ((len + n - 1) / n + 4095) & ~4095ull;
    std::vector<std::thread> ts;
    std::vector<std::string> errs(n);
    for (int i = 0; i < n; i++) {
        const uint64_t a = std::min<uint64_t>(len, (uint64_t)i * per), b = std::min<uint64_t>(len, a + per);
        if (a >= b) break;
        ts.emplace_back([this, off, dst, a, b, i, &errs] {
            try {
                read_at(off + a, static_cast<uint8_t *>(dst) + a, b - a);
            } catch (const std::exception &e) {
                errs[i] = e.what();
            }
        });
    }
    for (std::thread &t : ts) t.join();
    for (const std::string &e : errs)
        if (!e.empty()) throw GgufError(e);
}

void Gguf::read_into(const std::string &name, void *dst, uint64_t len) const {
    const TensorInfo &t = tensor(name);
    if (len != t.byte_size)
        gerr("tensor %s: buffer has %llu bytes, tensor has %llu", name.c_str(), (unsigned long long)len,
             (unsigned long long)t.byte_size);
    const uint64_t align = std::max<uint64_t>(32, alignment_);
    if (t.abs_offset % align)
        gerr("tensor %s: absolute offset %llu is not a multiple of %llu", name.c_str(), (unsigned long long)t.abs_offset,
             (unsigned long long)align);
    read_at(t.abs_offset, dst, len);
}

}  // namespace qdec
