// gguf.h -- GGUF v2/v3 reader (metadata + tensor directory, data memory-mapped).
//
// Replaces gguf_init_from_file / gguf_find_key / gguf_get_val_* and the
// tensor lookups of core_gguf::load_weights that the reference's load_model
// uses (src/crispembed.cpp:365-373, src/core/gguf_loader.cpp:335).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

struct ceb_gguf_value {
    int type = -1;  // gguf value type
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    int arr_type = -1;
    std::vector<std::string> arr_str;
    std::vector<double> arr_num;
};

struct ceb_gguf_tensor {
    std::string name;
    std::vector<int64_t> ne;  // ne[0] fastest
    int type = 0;
    uint64_t offset = 0;      // absolute file offset
    uint64_t nbytes = 0;
};

class ceb_gguf {
   public:
    ~ceb_gguf();
    bool open(const std::string& path, std::string* err);
    const ceb_gguf_value* find(const std::string& key) const;
    bool get_u32(const std::string& key, int* v) const;
    bool get_f32(const std::string& key, float* v) const;
    std::string get_str(const std::string& key) const;
    const ceb_gguf_tensor* tensor(const std::string& name) const;
    const uint8_t* data(const ceb_gguf_tensor& t) const { return base_ + t.offset; }
    const std::map<std::string, ceb_gguf_tensor>& tensors() const { return tensors_; }

   private:
    std::map<std::string, ceb_gguf_value> kv_;
    std::map<std::string, ceb_gguf_tensor> tensors_;
    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
};
