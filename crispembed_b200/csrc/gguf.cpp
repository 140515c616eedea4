// gguf.cpp -- see gguf.h.  Layout: magic "GGUF", u32 version, u64 n_tensors,
// u64 n_kv, kv pairs, tensor infos, padding to general.alignment (default 32),
// tensor data.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace {
enum { GT_U8, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STR, GT_ARR, GT_U64, GT_I64, GT_F64 };

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    bool need(size_t n) {
        if ((size_t)(end - p) < n) ok = false;
        return ok;
    }
    template <typename T>
    T rd() {
        T v{};
        if (!need(sizeof(T))) return v;
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        uint64_t n = rd<uint64_t>();
        if (!need(n)) return std::string();
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
};

size_t scalar_size(int t) {
    switch (t) {
        case GT_U8: case GT_I8: case GT_BOOL: return 1;
        case GT_U16: case GT_I16: return 2;
        case GT_U32: case GT_I32: case GT_F32: return 4;
        case GT_U64: case GT_I64: case GT_F64: return 8;
    }
    return 0;
}

double read_num(Cursor& c, int t) {
    switch (t) {
        case GT_U8: return c.rd<uint8_t>();
        case GT_I8: return c.rd<int8_t>();
        case GT_U16: return c.rd<uint16_t>();
        case GT_I16: return c.rd<int16_t>();
        case GT_U32: return c.rd<uint32_t>();
        case GT_I32: return c.rd<int32_t>();
        case GT_F32: return c.rd<float>();
        case GT_BOOL: return c.rd<uint8_t>();
        case GT_U64: return (double)c.rd<uint64_t>();
        case GT_I64: return (double)c.rd<int64_t>();
        case GT_F64: return c.rd<double>();
    }
    c.ok = false;
    return 0;
}

// Storage size of a row of ne0 values for every ggml type a GGUF may hold (ggml's
// published block sizes), so a file opens even when some of its tensors use a
// format this library does not compute with; the loader rejects those by name.
uint64_t type_row_bytes(int type, int64_t ne0, bool* ok) {
    struct B {
        int type, block, bytes;
    };
    static const B kSizes[] = {
        {0, 1, 4},      {1, 1, 2},      {2, 32, 18},     {3, 32, 20},     {6, 32, 22},     {7, 32, 24},
        {8, 32, 34},    {9, 32, 40},    {10, 256, 84},   {11, 256, 110},  {12, 256, 144},  {13, 256, 176},
        {14, 256, 210}, {15, 256, 292}, {16, 256, 66},   {17, 256, 74},   {18, 256, 98},   {19, 256, 50},
        {20, 32, 18},   {21, 256, 110}, {22, 256, 82},   {23, 256, 136},  {24, 1, 1},      {25, 1, 2},
        {26, 1, 4},     {27, 1, 8},     {28, 1, 8},      {29, 256, 56},   {30, 1, 2},      {34, 256, 54},
        {35, 256, 66},
    };
    for (const B& b : kSizes)
        if (b.type == type) {
            if (ne0 % b.block) break;
            return (uint64_t)(ne0 / b.block) * b.bytes;
        }
    *ok = false;
    return 0;
}
}  // namespace

ceb_gguf::~ceb_gguf() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

bool ceb_gguf::open(const std::string& path, std::string* err) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        *err = "cannot open '" + path + "'";
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        *err = "'" + path + "' is not a GGUF file";
        return false;
    }
    void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        *err = "mmap failed for '" + path + "'";
        return false;
    }
    base_ = static_cast<const uint8_t*>(m);
    size_ = (size_t)st.st_size;
    Cursor c{base_, base_ + size_};
    if (memcmp(base_, "GGUF", 4) != 0) {
        *err = "'" + path + "' has no GGUF magic";
        return false;
    }
    c.p += 4;
    const uint32_t version = c.rd<uint32_t>();
    if (version != 2 && version != 3) {
        *err = "unsupported GGUF version " + std::to_string(version);
        return false;
    }
    const uint64_t n_tensors = c.rd<uint64_t>(), n_kv = c.rd<uint64_t>();
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        std::string key = c.str();
        ceb_gguf_value v;
        v.type = (int)c.rd<uint32_t>();
        if (v.type == GT_STR) {
            v.s = c.str();
        } else if (v.type == GT_ARR) {
            v.arr_type = (int)c.rd<uint32_t>();
            const uint64_t n = c.rd<uint64_t>();
            const size_t left = (size_t)(c.end - c.p);
            if (v.arr_type == GT_STR) {
                if (n > left / 8) { c.ok = false; break; }  // every string needs at least its 8-byte length
                v.arr_str.reserve(n);
                for (uint64_t j = 0; j < n && c.ok; ++j) v.arr_str.push_back(c.str());
            } else {
                const size_t es = scalar_size(v.arr_type);
                if (!es || n > left / es) { c.ok = false; break; }
                v.arr_num.resize(n);
                for (uint64_t j = 0; j < n; ++j) v.arr_num[j] = read_num(c, v.arr_type);
            }
        } else {
            const double x = read_num(c, v.type);
            v.f = x;  // integer views only where the conversion is defined
            v.u = (x >= 0.0 && x < 18446744073709551616.0) ? (uint64_t)x : 0;
            v.i = (x >= -9223372036854775808.0 && x < 9223372036854775808.0) ? (int64_t)x : 0;
        }
        kv_[key] = std::move(v);
    }
    std::vector<ceb_gguf_tensor> infos;
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        ceb_gguf_tensor t;
        t.name = c.str();
        const uint32_t nd = c.rd<uint32_t>();
        if (nd == 0 || nd > 4) { c.ok = false; break; }
        for (uint32_t j = 0; j < nd; ++j) {
            const uint64_t ne = c.rd<uint64_t>();
            if (ne == 0 || ne > ((uint64_t)1 << 40)) { c.ok = false; break; }  // no tensor of a model file is near
            t.ne.push_back((int64_t)ne);
        }
        t.type = (int)c.rd<uint32_t>();
        t.offset = c.rd<uint64_t>();
        infos.push_back(t);
    }
    if (!c.ok) {
        *err = "truncated or malformed GGUF header in '" + path + "'";
        return false;
    }
    int align = 32;
    get_u32("general.alignment", &align);
    if (align <= 0) align = 32;
    const uint64_t hdr = (uint64_t)(c.p - base_);
    const uint64_t data0 = (hdr + align - 1) / align * align;
    for (auto& t : infos) {
        bool ok = true;
        uint64_t rows = 1;  // overflow-checked: a tensor larger than the file is malformed anyway
        for (size_t j = 1; j < t.ne.size() && ok; ++j) {
            if ((uint64_t)t.ne[j] > size_ || rows > size_ / (uint64_t)t.ne[j]) ok = false;
            else rows *= (uint64_t)t.ne[j];
        }
        const uint64_t row_bytes = ok ? type_row_bytes(t.type, t.ne[0], &ok) : 0;
        if (ok && row_bytes && rows > size_ / row_bytes) ok = false;
        t.nbytes = row_bytes * rows;
        if (ok && (t.offset > size_ || data0 > size_ - t.offset)) ok = false;
        if (ok) t.offset += data0;
        if (!ok || t.nbytes > size_ || t.offset > size_ - t.nbytes) {
            *err = "tensor '" + t.name + "' has an unsupported type or lies outside the file";
            return false;
        }
        tensors_[t.name] = t;
    }
    return true;
}

const ceb_gguf_value* ceb_gguf::find(const std::string& key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
}

bool ceb_gguf::get_u32(const std::string& key, int* v) const {
    const ceb_gguf_value* x = find(key);
    if (!x || x->type == GT_STR || x->type == GT_ARR) return false;
    *v = (int)x->i;
    return true;
}

bool ceb_gguf::get_f32(const std::string& key, float* v) const {
    const ceb_gguf_value* x = find(key);
    if (!x || x->type == GT_STR || x->type == GT_ARR) return false;
    *v = (float)x->f;
    return true;
}

std::string ceb_gguf::get_str(const std::string& key) const {
    const ceb_gguf_value* x = find(key);
    return (x && x->type == GT_STR) ? x->s : std::string();
}

const ceb_gguf_tensor* ceb_gguf::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}
