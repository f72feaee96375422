// GGUF v3 reader (host): header, KV metadata, tensor index, aligned data section, raw tensor reads.
// Behaviour and error conditions follow crates/core/src/gguf.rs:464-822 (Gguf::open, get_*, tensor,
// layer_span, read_into); errors are reported as GgufError with the reference's messages.
#pragma once
#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace qdec {

struct GgufError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

enum class VType : uint32_t {
    U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STR = 8, ARR = 9, U64 = 10, I64 = 11, F64 = 12
};
const char *vtype_name(VType t);

struct GValue {
    VType type = VType::U32;
    uint64_t u = 0;    // unsigned / bool
    int64_t i = 0;     // signed
    double f = 0;      // floats
    std::string s;     // string
    VType elem = VType::U32;          // array element type
    std::vector<GValue> arr;          // array items
};

struct TensorInfo {
    std::string name;
    int type = 0;                 // ggml type id
    std::vector<uint64_t> shape;  // GGUF order (ne0 first)
    uint64_t n_elements = 0, byte_size = 0, rel_offset = 0, abs_offset = 0;
    // numpy order: [rows, cols] for a 2-D tensor
    std::vector<uint64_t> shape_numpy() const { return std::vector<uint64_t>(shape.rbegin(), shape.rend()); }
};

class Gguf {
  public:
    explicit Gguf(const std::string &path);  // throws GgufError
    ~Gguf();
    Gguf(const Gguf &) = delete;
    Gguf &operator=(const Gguf &) = delete;

    const std::string &path() const { return path_; }
    uint64_t file_size() const { return file_size_; }
    uint32_t alignment() const { return alignment_; }
    uint64_t data_offset() const { return data_offset_; }

    bool has(const std::string &key) const { return kv_index_.count(key) != 0; }
    const GValue &get(const std::string &key) const;
    uint32_t get_u32(const std::string &key) const;
    float get_f32(const std::string &key) const;
    bool get_bool(const std::string &key) const;
    const std::string &get_str(const std::string &key) const;
    const GValue &get_array(const std::string &key) const;
    std::vector<int32_t> get_array_i32(const std::string &key) const;

    const std::vector<TensorInfo> &tensors() const { return tensors_; }
    bool has_tensor(const std::string &name) const { return tensor_index_.count(name) != 0; }
    const TensorInfo &tensor(const std::string &name) const;
    // [start, end) byte span of layer n's tensors, false when the layer has none (gguf.rs:745-793, span only)
    bool layer_span(uint32_t n, uint64_t &start, uint64_t &end) const;
    // total bytes of tensors that belong to no blk.N. layer
    uint64_t non_layer_bytes() const;
    // read a tensor's bytes into `dst` (exactly byte_size); checks the 32-byte alignment (gguf.rs:803-817)
    void read_into(const std::string &name, void *dst, uint64_t len) const;
    // read `len` bytes at absolute file offset `off`
    void read_at(uint64_t off, void *dst, uint64_t len) const;
    // the same bytes read by up to `threads` threads in contiguous parts
    void read_at_parallel(uint64_t off, void *dst, uint64_t len, int threads) const;
    // Direct reads that bypass the page cache (O_DIRECT, os.rs:311 DirectFile): opens the file a second time and
    // returns false where the file system refuses O_DIRECT (tmpfs, for one).  read_direct_parallel then reads
    // [off, off + len) with off and dst on DIRECT_ALIGN boundaries, len rounded up to one (dst must have room for
    // it); the file's end stops the read, so the rounding never reads past it.
    static constexpr uint64_t DIRECT_ALIGN = 4096;
    bool open_direct();
    void read_direct_parallel(uint64_t off, void *dst, uint64_t len, int threads) const;

  private:
    void read_direct(uint64_t off, void *dst, uint64_t len) const;
    std::string path_;
    int fd_ = -1, fd_direct_ = -1;
    uint64_t file_size_ = 0, data_offset_ = 0;
    uint32_t alignment_ = 32;
    std::vector<std::pair<std::string, GValue>> kv_;
    std::unordered_map<std::string, size_t> kv_index_;
    std::vector<TensorInfo> tensors_;
    std::unordered_map<std::string, size_t> tensor_index_;
};

// Layer index of a "blk.N.<suffix>" name, -1 otherwise (gguf.rs:826-830).
long layer_of(const std::string &name);
// (elements per block, bytes per block) of a ggml type; (0, 0) for an unknown one (gguf.rs:247-280).
std::pair<uint64_t, uint64_t> ggml_block_layout(int type);

}  // namespace qdec
