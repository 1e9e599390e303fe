// ModelConfig (src/config/model.rs:8-82) parsed from the checkpoint's
// `config_json` with serde(default) semantics, its validate()
// (src/config/model.rs:95-223), and SamplerParams::validate()
// (src/rf/params.rs:99-183).  Error texts follow the reference.
#pragma once

#include <cmath>
#include <optional>
#include <string>

#include "common.hpp"
#include "json.hpp"

namespace irt {

struct ModelConfig {
  int64_t latent_dim = 128, latent_patch_size = 1, model_dim = 2048, num_layers = 24, num_heads = 16;
  double mlp_ratio = 2.875;
  std::optional<double> text_mlp_ratio = 2.6, speaker_mlp_ratio = 2.6;
  double dropout = 0.0;
  int64_t text_vocab_size = 102400;
  std::string text_tokenizer_repo = "sbintuitions/sarashina2.2-0.5b";
  bool text_add_bos = true;
  int64_t text_dim = 1280, text_layers = 14, text_heads = 10;
  bool use_caption_condition = false;
  std::optional<int64_t> caption_vocab_size, caption_dim, caption_layers, caption_heads;
  std::optional<std::string> caption_tokenizer_repo;
  std::optional<bool> caption_add_bos;
  std::optional<double> caption_mlp_ratio;
  std::optional<int64_t> speaker_dim = 1280, speaker_layers = 14, speaker_heads = 10, speaker_patch_size = 1;
  int64_t timestep_embed_dim = 512, adaln_rank = 256;
  double norm_eps = 1e-5;
  std::optional<int64_t> fixed_target_latent_steps;
  std::string raw_json;

  bool use_speaker_condition() const { return !use_caption_condition; }
  int64_t head_dim() const { return model_dim / num_heads; }
  int64_t patched_latent_dim() const { return latent_dim * latent_patch_size; }
  int64_t speaker_patched_latent_dim() const { return patched_latent_dim() * speaker_patch_size.value_or(1); }
  double text_mlp_ratio_() const { return text_mlp_ratio.value_or(mlp_ratio); }
  double speaker_mlp_ratio_() const { return speaker_mlp_ratio.value_or(mlp_ratio); }
  int64_t caption_dim_() const { return caption_dim.value_or(text_dim); }
  int64_t caption_layers_() const { return caption_layers.value_or(text_layers); }
  int64_t caption_heads_() const { return caption_heads.value_or(text_heads); }
  int64_t caption_vocab_size_() const { return caption_vocab_size.value_or(text_vocab_size); }
  double caption_mlp_ratio_() const { return caption_mlp_ratio.value_or(text_mlp_ratio_()); }
  // ((dim as f64 * ratio) as usize).max(1) (src/model/diffusion.rs:32)
  static int64_t hidden(int64_t dim, double ratio) {
    int64_t h = (int64_t)((double)dim * ratio);
    return h < 1 ? 1 : h;
  }
  int64_t adaln_rank_eff() const {  // rank.max(1).min(model_dim) (src/model/norm.rs:99)
    int64_t r = adaln_rank < 1 ? 1 : adaln_rank;
    return r > model_dim ? model_dim : r;
  }

  static ModelConfig from_json(const std::string& s) {
    ModelConfig c;
    c.raw_json = s;
    Json j;
    try {
      j = parse_json(s);
    } catch (const JsonError& e) {
      throw Error(IRT_E_JSON, std::string("JSON error: ") + e.what());
    }
    if (j.kind != Json::Object) throw Error(IRT_E_JSON, "JSON error: config_json is not an object");
    try {
      auto I = [&](const char* k, int64_t& dst) {
        if (j.has(k) && !j.at(k).is_null()) {
          double v = j.at(k).as_number();
          if (v < 0 || v != std::floor(v)) throw JsonError(std::string("invalid value for ") + k);
          dst = (int64_t)v;
        }
      };
      auto OI = [&](const char* k, std::optional<int64_t>& dst) {
        if (j.has(k)) {
          if (j.at(k).is_null()) dst.reset();
          else {
            double v = j.at(k).as_number();
            if (v < 0 || v != std::floor(v)) throw JsonError(std::string("invalid value for ") + k);
            dst = (int64_t)v;
          }
        }
      };
      auto D = [&](const char* k, double& dst) {
        if (j.has(k) && !j.at(k).is_null()) dst = j.at(k).as_number();
      };
      auto OD = [&](const char* k, std::optional<double>& dst) {
        if (j.has(k)) {
          if (j.at(k).is_null()) dst.reset(); else dst = j.at(k).as_number();
        }
      };
      auto B = [&](const char* k, bool& dst) {
        if (j.has(k) && !j.at(k).is_null()) dst = j.at(k).as_bool();
      };
      auto S = [&](const char* k, std::string& dst) {
        if (j.has(k) && !j.at(k).is_null()) dst = j.at(k).as_string();
      };
      I("latent_dim", c.latent_dim); I("latent_patch_size", c.latent_patch_size);
      I("model_dim", c.model_dim); I("num_layers", c.num_layers); I("num_heads", c.num_heads);
      D("mlp_ratio", c.mlp_ratio); OD("text_mlp_ratio", c.text_mlp_ratio);
      OD("speaker_mlp_ratio", c.speaker_mlp_ratio); D("dropout", c.dropout);
      I("text_vocab_size", c.text_vocab_size); S("text_tokenizer_repo", c.text_tokenizer_repo);
      B("text_add_bos", c.text_add_bos); I("text_dim", c.text_dim); I("text_layers", c.text_layers);
      I("text_heads", c.text_heads); B("use_caption_condition", c.use_caption_condition);
      OI("caption_vocab_size", c.caption_vocab_size); OI("caption_dim", c.caption_dim);
      OI("caption_layers", c.caption_layers); OI("caption_heads", c.caption_heads);
      OD("caption_mlp_ratio", c.caption_mlp_ratio);
      OI("speaker_dim", c.speaker_dim); OI("speaker_layers", c.speaker_layers);
      OI("speaker_heads", c.speaker_heads); OI("speaker_patch_size", c.speaker_patch_size);
      I("timestep_embed_dim", c.timestep_embed_dim); I("adaln_rank", c.adaln_rank);
      D("norm_eps", c.norm_eps); OI("fixed_target_latent_steps", c.fixed_target_latent_steps);
    } catch (const JsonError& e) {
      throw Error(IRT_E_JSON, std::string("JSON error: ") + e.what());
    }
    return c;
  }

  void validate() const {
    auto S = [](int64_t v) { return std::to_string(v); };
    if (model_dim == 0) throw config_error("model_dim must be > 0");
    if (num_heads == 0) throw config_error("num_heads must be > 0");
    if (model_dim % num_heads)
      throw config_error("model_dim (" + S(model_dim) + ") must be divisible by num_heads (" + S(num_heads) + ")");
    if (head_dim() % 2) throw config_error("head_dim (" + S(head_dim()) + ") must be even for RoPE");
    if (latent_patch_size == 0) throw config_error("latent_patch_size must be > 0");
    if (timestep_embed_dim == 0) throw config_error("timestep_embed_dim must be > 0");
    if (adaln_rank == 0) throw config_error("adaln_rank must be > 0");
    if (text_dim == 0) throw config_error("text_dim must be > 0");
    if (text_heads == 0) throw config_error("text_heads must be > 0");
    if (text_dim % text_heads)
      throw config_error("text_dim (" + S(text_dim) + ") must be divisible by text_heads (" + S(text_heads) + ")");
    if ((text_dim / text_heads) % 2)
      throw config_error("text head_dim (" + S(text_dim / text_heads) + ") must be even for RoPE");
    if (use_speaker_condition()) {
      if (!speaker_dim) throw config_error("speaker_dim must be set when use_caption_condition is false");
      if (!speaker_heads) throw config_error("speaker_heads must be set when use_caption_condition is false");
      if (!speaker_layers) throw config_error("speaker_layers must be set when use_caption_condition is false");
      if (!speaker_patch_size)
        throw config_error("speaker_patch_size must be set when use_caption_condition is false");
      if (*speaker_dim == 0) throw config_error("speaker_dim must be > 0");
      if (*speaker_heads == 0) throw config_error("speaker_heads must be > 0");
      if (*speaker_dim % *speaker_heads)
        throw config_error("speaker_dim (" + S(*speaker_dim) + ") must be divisible by speaker_heads (" +
                           S(*speaker_heads) + ")");
      if ((*speaker_dim / *speaker_heads) % 2)
        throw config_error("speaker head_dim (" + S(*speaker_dim / *speaker_heads) + ") must be even for RoPE");
    }
    if (use_caption_condition) {
      int64_t cd = caption_dim_(), ch = caption_heads_();
      if (cd == 0) throw config_error("caption_dim must be > 0");
      if (ch == 0) throw config_error("caption_heads must be > 0");
      if (cd % ch) throw config_error("caption_dim (" + S(cd) + ") must be divisible by caption_heads (" + S(ch) + ")");
      if ((cd / ch) % 2) throw config_error("caption head_dim (" + S(cd / ch) + ") must be even for RoPE");
    }
  }
};

inline std::string fmt_f32(float v) {
  // Rust's `{}` for f32 prints the shortest round-trip form ("3", "0.5", "inf").
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "inf" : "-inf";
  char buf[64];
  for (int prec = 1; prec <= 9; ++prec) {
    std::snprintf(buf, sizeof buf, "%.*g", prec, (double)v);
    if (std::strtof(buf, nullptr) == v) break;
  }
  std::string s(buf);
  if (s.find('e') != std::string::npos) {
    std::snprintf(buf, sizeof buf, "%.9f", (double)v);
    s = buf;
    while (!s.empty() && s.back() == '0') s.pop_back();
    if (!s.empty() && s.back() == '.') s.pop_back();
  }
  return s;
}

inline void validate_sampler_params(const irt_sampler_params& p) {
  if (p.num_steps == 0) throw config_error("num_steps must be > 0");
  if (p.method < IRT_EULER || p.method > IRT_PLMS4) throw Error(IRT_E_INVALID_ARG, "invalid sampler method");
  if (p.cfg_mode < IRT_CFG_INDEPENDENT || p.cfg_mode > IRT_CFG_ALTERNATING)
    throw Error(IRT_E_INVALID_ARG, "invalid cfg guidance mode");
  const char* names[3] = {"guidance.scale_text", "guidance.scale_caption", "guidance.scale_speaker"};
  float vals[3] = {p.scale_text, p.scale_caption, p.scale_speaker};
  for (int i = 0; i < 3; ++i)
    if (!std::isfinite(vals[i])) throw config_error(std::string(names[i]) + " must be finite, got " + fmt_f32(vals[i]));
  if (!std::isfinite(p.min_t) || !(p.min_t >= 0.f && p.min_t <= 1.f))
    throw config_error("guidance.min_t must be finite and in [0, 1], got " + fmt_f32(p.min_t));
  if (!std::isfinite(p.max_t) || !(p.max_t >= 0.f && p.max_t <= 1.f))
    throw config_error("guidance.max_t must be finite and in [0, 1], got " + fmt_f32(p.max_t));
  if (p.min_t > p.max_t)
    throw config_error("guidance.min_t (" + fmt_f32(p.min_t) + ") must not exceed guidance.max_t (" + fmt_f32(p.max_t) + ")");
  if (p.has_truncation && (p.truncation_factor <= 0.f || !std::isfinite(p.truncation_factor)))
    throw config_error("truncation_factor must be finite and > 0");
  if (p.has_temporal_rescale) {
    if (!std::isfinite(p.rescale_k)) throw config_error("temporal_rescale.k must be finite");
    if (p.rescale_sigma == 0.f) throw config_error("temporal_rescale.sigma must not be zero");
  }
  if (p.has_speaker_kv) {
    if (!std::isfinite(p.speaker_kv_scale) || p.speaker_kv_scale <= 0.f)
      throw config_error("speaker_kv.scale must be finite and > 0");
    if (p.has_speaker_kv_min_t &&
        (!std::isfinite(p.speaker_kv_min_t) || !(p.speaker_kv_min_t >= 0.f && p.speaker_kv_min_t <= 1.f)))
      throw config_error("speaker_kv.min_t must be finite and in [0, 1]");
  }
  if (p.method == IRT_PLMS4 && p.cfg_mode == IRT_CFG_ALTERNATING)
    throw config_error(
        "sampler PLMS4 is not compatible with cfg_guidance_mode=Alternating; use Independent or Joint instead");
}

}  // namespace irt
