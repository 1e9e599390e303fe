// PEFT LoRA adapter merged into the base weights at load, as
// InferenceBuilder::load_weights_with_adapter does (src/inference.rs:118-139,
// src/weights/tensor_store.rs:62-118, src/lora.rs:37-322):
//   * a base checkpoint saved by PEFT has its "base_model.model." key prefix
//     stripped and its raw ".lora_" entries dropped;
//   * adapter_dir/adapter_config.json gives r and lora_alpha (scale =
//     lora_alpha / r, computed in f64, applied in f32);
//   * every adapter key "<prefix?><path>.lora_A.<name>" [r, d_in] with its
//     ".lora_B." partner [d_out, r] updates base "<path>.weight" [d_out, d_in]:
//     W += scale * (B @ A), the product accumulated in f32 over r for each
//     row in increasing order;
//   * the merged weight is re-encoded to the base tensor's dtype (bf16 by
//     truncating the low 16 bits, f16 rounding to nearest) and handed to the
//     loader in place of the file's tensor.
#pragma once

#include <sys/stat.h>

#include <cmath>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "common.hpp"
#include "json.hpp"
#include "safetensors.hpp"

namespace irt {

namespace lora_detail {

inline std::string shape_str(const std::vector<int64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

inline float f16_round_trip(float f) {
  // round to nearest even half precision (normals, subnormals, overflow to inf)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const int exp = (int)((u >> 23) & 0xff);
  uint32_t man = u & 0x7fffffu;
  uint16_t h;
  if (exp == 0xff) {
    h = (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
  } else {
    const int e = exp - 127 + 15;
    if (e >= 31) {
      h = (uint16_t)(sign | 0x7c00u);
    } else if (e <= 0) {
      if (e < -10) {
        h = (uint16_t)sign;
      } else {
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t m = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (m & 1u))) ++m;
        h = (uint16_t)(sign | m);
      }
    } else {
      uint32_t m = man >> 13;
      const uint32_t rem = man & 0x1fffu;
      uint32_t hv = sign | ((uint32_t)e << 10) | m;
      if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) ++hv;  // may carry into the exponent
      h = (uint16_t)hv;
    }
  }
  TensorView v;
  v.dtype = DType::F16;
  v.shape = {1};
  v.data = reinterpret_cast<const uint8_t*>(&h);
  v.nbytes = 2;
  float out;
  decode_to_f32(v, &out);
  return out;
}

}  // namespace lora_detail

// Returns the merged base keys.
inline std::vector<std::string> apply_lora(SafeTensorsFile& st, const std::string& adapter_dir) {
  using namespace lora_detail;
  const std::string prefix = "base_model.model.";
  // PEFT-saved base checkpoint: strip the prefix, drop raw LoRA entries
  bool peft = false;
  for (const auto& kv : st.tensors())
    if (kv.first.rfind(prefix, 0) == 0) peft = true;
  if (peft) {
    std::vector<std::string> keys;
    for (const auto& kv : st.tensors()) keys.push_back(kv.first);
    for (const auto& k : keys) {
      if (k.find(".lora_") != std::string::npos) st.erase(k);
      else if (k.rfind(prefix, 0) == 0) st.rename(k, k.substr(prefix.size()));
    }
  }
  // adapter_config.json
  const std::string cfg_path = adapter_dir + "/adapter_config.json";
  std::ifstream f(cfg_path);
  if (!f) throw Error(IRT_E_WEIGHT, "Missing weight tensor: cannot read adapter_config.json at " + cfg_path);
  std::stringstream ss;
  ss << f.rdbuf();
  double r = 0.0, alpha = 0.0;
  try {
    const Json cfg = parse_json(ss.str());
    r = (double)cfg.at("r").as_int();
    alpha = cfg.at("lora_alpha").as_number();
  } catch (const std::exception& e) {
    throw Error(IRT_E_WEIGHT, "Missing weight tensor: malformed adapter_config.json at " + cfg_path + ": " + e.what());
  }
  if (!(r > 0)) throw Error(IRT_E_WEIGHT, "Missing weight tensor: malformed adapter_config.json at " + cfg_path + ": r must be > 0");
  const std::string ad_path = adapter_dir + "/adapter_model.safetensors";
  struct stat sb;
  if (::stat(ad_path.c_str(), &sb) != 0)
    throw Error(IRT_E_WEIGHT, "Missing weight tensor: no adapter weights found in " + adapter_dir +
                                  " (expected adapter_model.safetensors)");
  SafeTensorsFile ad(ad_path);
  const float scale = (float)(alpha / r);

  std::vector<std::string> merged;
  for (const auto& kv : ad.tensors()) {
    const std::string& a_key = kv.first;
    const size_t apos = a_key.find(".lora_A.");
    if (apos == std::string::npos) continue;
    std::string b_key = a_key;
    b_key.replace(apos, 8, ".lora_B.");
    if (!ad.has(b_key)) continue;
    std::string base = a_key.rfind(prefix, 0) == 0 ? a_key.substr(prefix.size()) : a_key;
    const std::string base_key = base.substr(0, base.find(".lora_A.")) + ".weight";
    if (!st.has(base_key)) continue;
    const TensorView& A = ad.get(a_key);
    const TensorView& B = ad.get(b_key);
    if (A.shape.size() != 2 || B.shape.size() != 2)
      throw Error(IRT_E_WEIGHT, "Missing weight tensor: LoRA rank must be 2-D for " + base_key + ": lora_A rank=" +
                                    std::to_string(A.shape.size()) + ", lora_B rank=" + std::to_string(B.shape.size()));
    const long rr = (long)A.shape[0], d_in = (long)A.shape[1], d_out = (long)B.shape[0];
    if (B.shape[1] != rr)
      throw Error(IRT_E_WEIGHT, "Missing weight tensor: LoRA shape mismatch for " + base_key + ": lora_A=" +
                                    shape_str(A.shape) + ", lora_B=" + shape_str(B.shape));
    const TensorView& W = st.get(base_key);
    if (W.numel() != d_out * d_in)
      throw Error(IRT_E_WEIGHT, "Missing weight tensor: LoRA base shape mismatch for " + base_key + ": base=" +
                                    shape_str(W.shape) + ", expected [" + std::to_string(d_out) + "x" +
                                    std::to_string(d_in) + "]");
    std::vector<float> a((size_t)A.numel()), b((size_t)B.numel()), w((size_t)W.numel());
    decode_to_f32(A, a.data());
    decode_to_f32(B, b.data());
    decode_to_f32(W, w.data());
    const DType wdt = W.dtype;
    const std::vector<int64_t> wshape = W.shape;
    // delta = B @ A (row i: k outer, j inner), then W += scale * delta
    std::vector<float> row((size_t)d_in);
    for (long i = 0; i < d_out; ++i) {
      std::fill(row.begin(), row.end(), 0.f);
      for (long k = 0; k < rr; ++k) {
        const float bv = b[(size_t)i * rr + k];
        const float* ar = a.data() + (size_t)k * d_in;
        for (long j = 0; j < d_in; ++j) row[j] += bv * ar[j];
      }
      float* wr = w.data() + (size_t)i * d_in;
      for (long j = 0; j < d_in; ++j) {
        float v = wr[j] + scale * row[j];
        if (wdt == DType::BF16) {
          uint32_t u;
          std::memcpy(&u, &v, 4);
          u &= 0xffff0000u;  // encode_f32_to_dtype: high 16 bits
          std::memcpy(&v, &u, 4);
        } else if (wdt == DType::F16) {
          v = f16_round_trip(v);
        }
        wr[j] = v;
      }
    }
    st.override_f32(base_key, std::move(w), wshape);
    merged.push_back(base_key);
  }
  return merged;
}

}  // namespace irt
