// GGUF v2/v3 reader for the device loader (gguf/reader.hpp:1-205 and
// gguf/mapped_file.hpp:63 of the reference define the behaviour it keeps):
// the image is untrusted, every read is bounds-checked, counts are checked
// against the bytes left before anything is allocated, names and tensor data
// are views into the mapped file. Only what the Llama loader needs is exposed.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

namespace syn::gguf {

enum class vtype : uint32_t {
    u8 = 0, i8 = 1, u16 = 2, i16 = 3, u32 = 4, i32 = 5, f32 = 6, boolean = 7,
    string = 8, array = 9, u64 = 10, i64 = 11, f64 = 12
};

struct value {
    vtype type = vtype::u8;
    uint64_t u = 0;        // unsigned integers and bool
    int64_t i = 0;         // signed integers
    double f = 0.0;        // f32 / f64
    std::string_view s;    // string
    vtype arr_type = vtype::u8;
    uint64_t arr_n = 0;    // array element count
    const uint8_t* arr = nullptr;  // first element (fixed-size element types only)
};

struct entry {
    std::string_view key;
    value v;
};

struct tensor_info {
    std::string_view name;
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t nbytes = 0;
    uint64_t n_elements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
    uint64_t rows() const { return ne[1] * ne[2] * ne[3]; }
};

// Block geometry of a ggml type: elements per block and bytes per block
// (gguf/tensor_type.hpp:57-115); {0, 0} for types the reader rejects.
struct type_traits {
    uint32_t block_size;
    uint32_t type_size;
};
type_traits traits(uint32_t type);

class file {
public:
    ~file();
    file(const file&) = delete;
    file& operator=(const file&) = delete;

    // Map `path` read-only and parse it. Returns a syn_status.
    static int open(const char* path, std::unique_ptr<file>& out, std::string* error = nullptr);
    // Parse an image the caller keeps alive.
    static int parse(const uint8_t* data, size_t size, std::unique_ptr<file>& out, std::string* error = nullptr);

    uint32_t version() const { return version_; }
    uint64_t alignment() const { return alignment_; }
    const std::vector<entry>& metadata() const { return meta_; }
    const std::vector<tensor_info>& tensors() const { return tensors_; }

    const value* find(std::string_view key) const;
    const tensor_info* tensor(std::string_view name) const;
    const uint8_t* data(const tensor_info& t) const { return base_ + data_offset_ + t.offset; }

    // Typed metadata getters: false when absent or of another kind.
    bool get_uint(std::string_view key, uint64_t& out) const;
    bool get_float(std::string_view key, double& out) const;
    bool get_string(std::string_view key, std::string_view& out) const;

private:
    file() = default;
    int run(std::string* error);

    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
    void* mapping_ = nullptr;  // owned mmap, or null for a borrowed image
    uint32_t version_ = 0;
    uint64_t alignment_ = 32;
    uint64_t data_offset_ = 0;
    std::vector<entry> meta_;
    std::vector<tensor_info> tensors_;
};

}  // namespace syn::gguf
