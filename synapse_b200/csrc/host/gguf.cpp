#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <unordered_set>

#include "synapse_b200.h"

namespace syn::gguf {

type_traits traits(uint32_t type) {
    switch (type) {
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
    case 24: return {1, 1};     // I8
    case 25: return {1, 2};     // I16
    case 26: return {1, 4};     // I32
    case 27: return {1, 8};     // I64
    case 28: return {1, 8};     // F64
    case 30: return {1, 2};     // BF16
    default: return {0, 0};
    }
}

namespace {

struct cursor {
    const uint8_t* p;
    size_t n, at = 0;
    bool take(void* dst, size_t k) {
        if (k > n - at) return false;
        std::memcpy(dst, p + at, k);
        at += k;
        return true;
    }
    bool skip(size_t k) {
        if (k > n - at) return false;
        at += k;
        return true;
    }
    template <typename T>
    bool get(T& v) { return take(&v, sizeof v); }
    bool str(std::string_view& s) {
        uint64_t len;
        if (!get(len) || len > n - at) return false;
        s = std::string_view(reinterpret_cast<const char*>(p + at), size_t(len));
        at += size_t(len);
        return true;
    }
};

size_t scalar_size(vtype t) {
    switch (t) {
    case vtype::u8: case vtype::i8: case vtype::boolean: return 1;
    case vtype::u16: case vtype::i16: return 2;
    case vtype::u32: case vtype::i32: case vtype::f32: return 4;
    case vtype::u64: case vtype::i64: case vtype::f64: return 8;
    default: return 0;
    }
}

bool read_scalar(cursor& c, vtype t, value& v) {
    v.type = t;
    switch (t) {
    case vtype::u8: { uint8_t x; if (!c.get(x)) return false; v.u = x; v.i = x; return true; }
    case vtype::boolean: { uint8_t x; if (!c.get(x) || x > 1) return false; v.u = x; v.i = x; return true; }
    case vtype::i8: { int8_t x; if (!c.get(x)) return false; v.i = x; v.u = uint64_t(x); return true; }
    case vtype::u16: { uint16_t x; if (!c.get(x)) return false; v.u = x; v.i = x; return true; }
    case vtype::i16: { int16_t x; if (!c.get(x)) return false; v.i = x; v.u = uint64_t(x); return true; }
    case vtype::u32: { uint32_t x; if (!c.get(x)) return false; v.u = x; v.i = x; return true; }
    case vtype::i32: { int32_t x; if (!c.get(x)) return false; v.i = x; v.u = uint64_t(x); return true; }
    case vtype::u64: { uint64_t x; if (!c.get(x)) return false; v.u = x; v.i = int64_t(x); return true; }
    case vtype::i64: { int64_t x; if (!c.get(x)) return false; v.i = x; v.u = uint64_t(x); return true; }
    case vtype::f32: { float x; if (!c.get(x)) return false; v.f = x; return true; }
    case vtype::f64: { double x; if (!c.get(x)) return false; v.f = x; return true; }
    case vtype::string: return c.str(v.s);
    default: return false;
    }
}

int fail(std::string* error, const char* what, size_t at) {
    if (error) *error = std::string(what) + " at byte " + std::to_string(at);
    return SYN_ERR_FORMAT;
}

}  // namespace

file::~file() {
    if (mapping_) munmap(mapping_, size_);
}

int file::open(const char* path, std::unique_ptr<file>& out, std::string* error) {
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        if (error) *error = std::string("cannot open ") + path;
        return SYN_ERR_INVALID;
    }
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        ::close(fd);
        if (error) *error = "cannot stat or empty file";
        return SYN_ERR_FORMAT;
    }
    void* m = mmap(nullptr, size_t(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        if (error) *error = "mmap failed";
        return SYN_ERR_INVALID;
    }
    std::unique_ptr<file> f(new file());
    f->base_ = static_cast<const uint8_t*>(m);
    f->size_ = size_t(st.st_size);
    f->mapping_ = m;
    const int rc = f->run(error);
    if (rc) return rc;
    out = std::move(f);
    return SYN_OK;
}

int file::parse(const uint8_t* data, size_t size, std::unique_ptr<file>& out, std::string* error) {
    std::unique_ptr<file> f(new file());
    f->base_ = data;
    f->size_ = size;
    const int rc = f->run(error);
    if (rc) return rc;
    out = std::move(f);
    return SYN_OK;
}

int file::run(std::string* error) {
    cursor c{base_, size_};
    char magic[4];
    if (!c.take(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) return fail(error, "bad magic", 0);
    if (!c.get(version_) || (version_ != 2 && version_ != 3)) return fail(error, "unsupported version", 4);
    uint64_t n_tensors, n_kv;
    if (!c.get(n_tensors) || !c.get(n_kv)) return fail(error, "truncated header", c.at);
    // Each KV needs >= 12 bytes and each tensor >= 24: reject counts the image cannot hold.
    if (n_kv > (size_ - c.at) / 12 || n_tensors > (size_ - c.at) / 24) return fail(error, "count too large", c.at);
    std::unordered_set<std::string_view> keys;
    meta_.reserve(size_t(n_kv));
    for (uint64_t i = 0; i < n_kv; ++i) {
        entry e;
        const size_t at = c.at;
        uint32_t t;
        if (!c.str(e.key) || !c.get(t)) return fail(error, "truncated metadata", at);
        if (!keys.insert(e.key).second) return fail(error, "duplicate key", at);
        const vtype vt = vtype(t);
        if (vt == vtype::array) {
            uint32_t et;
            uint64_t n;
            if (!c.get(et) || !c.get(n)) return fail(error, "truncated array", at);
            e.v.type = vtype::array;
            e.v.arr_type = vtype(et);
            e.v.arr_n = n;
            if (vtype(et) == vtype::string) {
                if (n > (size_ - c.at) / 8) return fail(error, "array too large", at);
                for (uint64_t k = 0; k < n; ++k) {
                    std::string_view s;
                    if (!c.str(s)) return fail(error, "truncated string array", at);
                }
            } else {
                const size_t es = scalar_size(vtype(et));
                if (es == 0) return fail(error, "bad array element type", at);
                if (n > (size_ - c.at) / es) return fail(error, "array too large", at);
                e.v.arr = base_ + c.at;
                c.skip(size_t(n) * es);
            }
        } else if (!read_scalar(c, vt, e.v)) {
            return fail(error, "bad metadata value", at);
        }
        meta_.push_back(e);
    }
    if (const value* a = find("general.alignment")) {
        if (a->type != vtype::u32 || a->u == 0 || (a->u & (a->u - 1))) return fail(error, "bad alignment", 0);
        alignment_ = a->u;
    }
    std::unordered_set<std::string_view> names;
    tensors_.reserve(size_t(n_tensors));
    for (uint64_t i = 0; i < n_tensors; ++i) {
        tensor_info t;
        const size_t at = c.at;
        if (!c.str(t.name) || !c.get(t.n_dims)) return fail(error, "truncated tensor info", at);
        if (t.n_dims < 1 || t.n_dims > 4) return fail(error, "bad n_dims", at);
        for (uint32_t d = 0; d < t.n_dims; ++d)
            if (!c.get(t.ne[d]) || t.ne[d] == 0) return fail(error, "bad shape", at);
        if (!c.get(t.type) || !c.get(t.offset)) return fail(error, "truncated tensor info", at);
        if (!names.insert(t.name).second) return fail(error, "duplicate tensor", at);
        const type_traits tt = traits(t.type);
        if (tt.block_size == 0) return fail(error, "unsupported tensor type", at);
        if (t.ne[0] % tt.block_size) return fail(error, "row is not whole blocks", at);
        // n_elements without overflow: each ne < 2^63 and the product bounded by the image size
        unsigned __int128 n = 1;
        for (int d = 0; d < 4; ++d) n *= t.ne[d];
        const unsigned __int128 bytes = n / tt.block_size * tt.type_size;
        if (bytes > size_) return fail(error, "tensor larger than file", at);
        t.nbytes = uint64_t(bytes);
        if (t.offset % alignment_) return fail(error, "misaligned tensor", at);
        tensors_.push_back(t);
    }
    data_offset_ = (c.at + alignment_ - 1) / alignment_ * alignment_;
    if (data_offset_ > size_) return fail(error, "truncated before data", c.at);
    for (const tensor_info& t : tensors_)
        if (t.offset > size_ - data_offset_ || t.nbytes > size_ - data_offset_ - t.offset)
            return fail(error, "tensor data out of bounds", c.at);
    return SYN_OK;
}

const value* file::find(std::string_view key) const {
    for (const entry& e : meta_)
        if (e.key == key) return &e.v;
    return nullptr;
}

const tensor_info* file::tensor(std::string_view name) const {
    for (const tensor_info& t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

bool file::get_uint(std::string_view key, uint64_t& out) const {
    const value* v = find(key);
    if (!v) return false;
    switch (v->type) {
    case vtype::u8: case vtype::u16: case vtype::u32: case vtype::u64: out = v->u; return true;
    case vtype::i8: case vtype::i16: case vtype::i32: case vtype::i64:
        if (v->i < 0) return false;
        out = uint64_t(v->i);
        return true;
    default: return false;
    }
}

bool file::get_float(std::string_view key, double& out) const {
    const value* v = find(key);
    if (!v || (v->type != vtype::f32 && v->type != vtype::f64)) return false;
    out = v->f;
    return true;
}

bool file::get_string(std::string_view key, std::string_view& out) const {
    const value* v = find(key);
    if (!v || v->type != vtype::string) return false;
    out = v->s;
    return true;
}

}  // namespace syn::gguf
