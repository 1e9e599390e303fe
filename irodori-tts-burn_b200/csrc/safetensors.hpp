// Memory-mapped safetensors reader (format: u64 LE header size, JSON header,
// raw little-endian tensor bytes).  Mirrors TensorStore::load
// (src/weights/tensor_store.rs:26-53) and TensorEntry's checks
// (src/weights/tensor_entry.rs:22-90): byte-length validation, F32/BF16/F16
// decode, the `config_json` metadata requirement.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.hpp"
#include "json.hpp"

namespace irt {

enum class DType { F32, BF16, F16, Other };

struct TensorView {
  DType dtype = DType::Other;
  std::string dtype_name;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

class SafeTensorsFile {
 public:
  explicit SafeTensorsFile(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw Error(IRT_E_IO, "IO error: cannot open '" + path + "': " + std::strerror(errno));
    struct stat st;
    if (fstat(fd_, &st) != 0) throw Error(IRT_E_IO, "IO error: cannot stat '" + path + "'");
    size_ = (size_t)st.st_size;
    if (size_ < 8) throw Error(IRT_E_SAFETENSORS, "SafeTensors error: HeaderTooSmall");
    base_ = (const uint8_t*)mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (base_ == MAP_FAILED) {
      base_ = nullptr;
      throw Error(IRT_E_IO, "IO error: mmap failed for '" + path + "'");
    }
    uint64_t hlen = 0;
    std::memcpy(&hlen, base_, 8);
    if (hlen > size_ - 8) throw Error(IRT_E_SAFETENSORS, "SafeTensors error: InvalidHeaderLength");
    Json h;
    try {
      h = JsonParser((const char*)base_ + 8, (size_t)hlen).parse();
    } catch (const JsonError& e) {
      throw Error(IRT_E_SAFETENSORS, std::string("SafeTensors error: InvalidHeaderDeserialization: ") + e.what());
    }
    if (h.kind != Json::Object) throw Error(IRT_E_SAFETENSORS, "SafeTensors error: header is not an object");
    const uint8_t* data0 = base_ + 8 + hlen;
    size_t data_len = size_ - 8 - hlen;
    for (auto& kv : h.obj) {
      if (kv.first == "__metadata__") {
        for (auto& m : kv.second.obj)
          if (m.second.kind == Json::String) metadata_[m.first] = m.second.str;
        continue;
      }
      TensorView v;
      try {
        v.dtype_name = kv.second.at("dtype").as_string();
        for (auto& d : kv.second.at("shape").arr) v.shape.push_back(d.as_int());
        auto& off = kv.second.at("data_offsets").arr;
        if (off.size() != 2) throw JsonError("data_offsets");
        int64_t b = off[0].as_int(), e = off[1].as_int();
        if (b < 0 || e < b || (size_t)e > data_len)
          throw Error(IRT_E_SAFETENSORS, "SafeTensors error: InvalidOffset(" + kv.first + ")");
        v.data = data0 + b;
        v.nbytes = (size_t)(e - b);
      } catch (const JsonError& e) {
        throw Error(IRT_E_SAFETENSORS, "SafeTensors error: malformed entry '" + kv.first + "': " + e.what());
      }
      size_t esz = 4;
      if (v.dtype_name == "F32") { v.dtype = DType::F32; esz = 4; }
      else if (v.dtype_name == "BF16") { v.dtype = DType::BF16; esz = 2; }
      else if (v.dtype_name == "F16") { v.dtype = DType::F16; esz = 2; }
      else {
        v.dtype = DType::Other;
        if (v.dtype_name == "F64" || v.dtype_name == "I64" || v.dtype_name == "U64") esz = 8;
        else if (v.dtype_name == "I16" || v.dtype_name == "U16") esz = 2;
        else if (v.dtype_name == "I8" || v.dtype_name == "U8" || v.dtype_name == "BOOL") esz = 1;
      }
      // TensorEntry::validate_byte_len (src/weights/tensor_entry.rs:35-44)
      size_t expected = (size_t)v.numel() * esz;
      if (v.nbytes != expected)
        throw Error(IRT_E_WEIGHT, "Missing weight tensor: " + kv.first + ": byte length mismatch — expected " +
                                      std::to_string(expected) + ", got " + std::to_string(v.nbytes));
      tensors_[kv.first] = v;
    }
  }
  ~SafeTensorsFile() {
    if (base_) munmap((void*)base_, size_);
    if (fd_ >= 0) ::close(fd_);
  }
  SafeTensorsFile(const SafeTensorsFile&) = delete;
  SafeTensorsFile& operator=(const SafeTensorsFile&) = delete;

  bool has(const std::string& k) const { return tensors_.count(k) != 0; }
  const TensorView& get(const std::string& k) const {
    auto it = tensors_.find(k);
    if (it == tensors_.end()) throw weight_error(k);
    return it->second;
  }
  // Entry with a rank check (TensorEntry::to_tensor_data, tensor_entry.rs:53-57).
  const TensorView& get(const std::string& k, size_t rank) const {
    const TensorView& v = get(k);
    if (v.shape.size() != rank)
      throw Error(IRT_E_WRONG_DIM, "Wrong rank for tensor '" + k + "': expected " + std::to_string(rank) +
                                       ", got " + std::to_string(v.shape.size()));
    if (v.dtype == DType::Other)
      throw Error(IRT_E_DTYPE, "Unsupported dtype for tensor '" + k + "': " + v.dtype_name);
    return v;
  }
  const std::string* meta(const std::string& k) const {
    auto it = metadata_.find(k);
    return it == metadata_.end() ? nullptr : &it->second;
  }
  const std::map<std::string, TensorView>& tensors() const { return tensors_; }

  // In-memory edits used when an adapter is merged at load: replace a
  // tensor by owned f32 data, rename or drop an entry.
  void override_f32(const std::string& k, std::vector<float> data, const std::vector<int64_t>& shape) {
    std::vector<float>& buf = owned_[k];
    buf = std::move(data);
    TensorView v;
    v.dtype = DType::F32;
    v.dtype_name = "F32";
    v.shape = shape;
    v.data = reinterpret_cast<const uint8_t*>(buf.data());
    v.nbytes = buf.size() * 4;
    tensors_[k] = v;
  }
  void rename(const std::string& from, const std::string& to) {
    auto it = tensors_.find(from);
    if (it == tensors_.end() || from == to) return;
    tensors_[to] = it->second;
    tensors_.erase(from);
  }
  void erase(const std::string& k) { tensors_.erase(k); }

 private:
  std::map<std::string, std::vector<float>> owned_;
  int fd_ = -1;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, TensorView> tensors_;
  std::map<std::string, std::string> metadata_;
};

// Decode any supported dtype to f32 (host).
inline void decode_to_f32(const TensorView& v, float* out) {
  size_t n = (size_t)v.numel();
  if (v.dtype == DType::F32) {
    std::memcpy(out, v.data, n * 4);
  } else if (v.dtype == DType::BF16) {
    const uint16_t* s = (const uint16_t*)v.data;
    for (size_t i = 0; i < n; ++i) {
      uint32_t u = (uint32_t)s[i] << 16;
      std::memcpy(&out[i], &u, 4);
    }
  } else if (v.dtype == DType::F16) {
    const uint16_t* s = (const uint16_t*)v.data;
    for (size_t i = 0; i < n; ++i) {
      uint16_t h = s[i];
      uint32_t sign = (uint32_t)(h & 0x8000) << 16;
      uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, u;
      if (exp == 0) {
        if (man == 0) u = sign;
        else {  // subnormal
          int e = -1;
          do { ++e; man <<= 1; } while (!(man & 0x400));
          u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
      } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
      } else {
        u = sign | ((exp + 112) << 23) | (man << 13);
      }
      std::memcpy(&out[i], &u, 4);
    }
  } else {
    throw Error(IRT_E_DTYPE, "Unsupported dtype: " + v.dtype_name);
  }
}

}  // namespace irt
