// extern "C" boundary (include/irodori_b200.h).  Every entry point converts
// exceptions into an irt_status plus a thread-local message; nothing aborts.
#include <cstring>
#include <memory>
#include <new>
#include <string>

#include "codec.hpp"
#include "config.hpp"
#include "engine.hpp"

struct irt_engine {
  std::unique_ptr<irt::Engine> e;
};
struct irt_codec {
  std::unique_ptr<irt::Codec> c;
};

namespace {
thread_local std::string g_last_error;

template <class F>
int guard(F&& f) {
  try {
    g_last_error.clear();
    f();
    return IRT_OK;
  } catch (const irt::Error& e) {
    g_last_error = e.what();
    return e.status;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return IRT_E_OOM;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return IRT_E_INVALID_ARG;
  } catch (...) {
    g_last_error = "unknown error";
    return IRT_E_INVALID_ARG;
  }
}
void need(const void* p, const char* what) {
  if (!p) throw irt::Error(IRT_E_INVALID_ARG, std::string(what) + " is NULL");
}
}  // namespace

extern "C" {

const char* irt_last_error(void) { return g_last_error.c_str(); }
const char* irt_version(void) { return "irodori-b200 0.1.0 (sm_100a)"; }

void irt_sampler_params_default(irt_sampler_params* p) {
  if (!p) return;
  std::memset(p, 0, sizeof(*p));
  p->num_steps = 40;
  p->method = IRT_EULER;
  p->cfg_mode = IRT_CFG_INDEPENDENT;
  p->scale_text = 3.0f;
  p->scale_caption = 3.0f;
  p->scale_speaker = 5.0f;
  p->min_t = 0.5f;
  p->max_t = 1.0f;
  p->speaker_kv_max_layers = -1;
  p->use_context_kv_cache = 1;
}

int irt_sampler_params_validate(const irt_sampler_params* p) {
  return guard([&] {
    need(p, "params");
    irt::validate_sampler_params(*p);
  });
}

int irt_engine_create(int device, const char* path, int precision, irt_engine** out) {
  return guard([&] {
    need(path, "safetensors_path");
    need(out, "out");
    *out = nullptr;
    auto h = std::make_unique<irt_engine>();
    h->e = std::make_unique<irt::Engine>(device, path, precision);
    *out = h.release();
  });
}

int irt_engine_create_with_adapter(int device, const char* path, const char* adapter_dir, int precision,
                                   irt_engine** out) {
  return guard([&] {
    need(path, "safetensors_path");
    need(adapter_dir, "adapter_dir");
    need(out, "out");
    *out = nullptr;
    auto h = std::make_unique<irt_engine>();
    h->e = std::make_unique<irt::Engine>(device, path, precision, adapter_dir);
    *out = h.release();
  });
}

int irt_engine_destroy(irt_engine* e) {
  return guard([&] { delete e; });
}

int irt_engine_set_sampling(irt_engine* e, const irt_sampler_params* p) {
  return guard([&] {
    need(e, "engine");
    need(p, "params");
    irt::validate_sampler_params(*p);
    std::lock_guard<std::mutex> lk(e->e->mu);
    e->e->params = *p;
    e->e->has_params = true;
  });
}

int irt_engine_set_default_sampling(irt_engine* e) {
  irt_sampler_params p;
  irt_sampler_params_default(&p);
  return irt_engine_set_sampling(e, &p);
}

int irt_engine_get_sampling(const irt_engine* e, irt_sampler_params* out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    if (!e->e->has_params) throw irt::Error(IRT_E_STATE, "sampling parameters not set");
    *out = e->e->params;
  });
}

int irt_engine_get_config(const irt_engine* e, char* buf, size_t cap, size_t* len) {
  return guard([&] {
    need(e, "engine");
    const std::string& j = e->e->cfg.raw_json;
    if (len) *len = j.size() + 1;
    if (buf && cap) {
      size_t n = std::min(cap - 1, j.size());
      std::memcpy(buf, j.data(), n);
      buf[n] = 0;
    }
  });
}

int irt_engine_patched_latent_dim(const irt_engine* e, int32_t* out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    *out = (int32_t)e->e->cfg.patched_latent_dim();
  });
}

int irt_engine_use_speaker_condition(const irt_engine* e, int32_t* out) {
  return guard([&] {
    need(e, "engine");
    need(out, "out");
    *out = e->e->cfg.use_speaker_condition() ? 1 : 0;
  });
}

int irt_engine_sample(irt_engine* e, const irt_request* req, float* out_latent, int out_memory, void* stream) {
  return guard([&] {
    need(e, "engine");
    need(req, "request");
    e->e->sample(*req, out_latent, out_memory, reinterpret_cast<cudaStream_t>(stream));
  });
}

int irt_engine_last_stats(const irt_engine* e, int64_t* row_forwards, int64_t* kernel_launches) {
  return guard([&] {
    need(e, "engine");
    if (row_forwards) *row_forwards = e->e->last_row_forwards;
    if (kernel_launches) *kernel_launches = e->e->last_launches;
  });
}

int irt_codec_create(int device, const char* path, int precision, irt_codec** out) {
  return guard([&] {
    need(path, "safetensors_path");
    need(out, "out");
    *out = nullptr;
    auto h = std::make_unique<irt_codec>();
    h->c = std::make_unique<irt::Codec>(device, path, precision);
    *out = h.release();
  });
}

int irt_codec_destroy(irt_codec* c) {
  return guard([&] { delete c; });
}

int irt_codec_sample_rate(const irt_codec* c, int32_t* out) {
  return guard([&] {
    need(c, "codec");
    need(out, "out");
    *out = 48000;
  });
}

int irt_codec_hop_length(const irt_codec* c, int32_t* out) {
  return guard([&] {
    need(c, "codec");
    need(out, "out");
    int h = 1;
    for (auto& b : c->c->blocks) h *= b.stride;
    *out = h;
  });
}

int irt_codec_decode(irt_codec* c, const float* latent, int32_t batch, int32_t frames, float* wav, int memory,
                     void* stream) {
  return guard([&] {
    need(c, "codec");
    need(latent, "latent");
    need(wav, "wav");
    c->c->decode(latent, batch, frames, wav, memory, reinterpret_cast<cudaStream_t>(stream));
  });
}

int irt_codec_decode_ragged(irt_codec* c, const float* latent, int32_t batch, int32_t frames, const int32_t* lengths,
                            float* wav, int memory, void* stream) {
  return guard([&] {
    need(c, "codec");
    need(latent, "latent");
    need(lengths, "lengths");
    need(wav, "wav");
    c->c->decode(latent, batch, frames, wav, memory, reinterpret_cast<cudaStream_t>(stream), lengths);
  });
}

int irt_codec_decode_noalloc(irt_codec* c, const float* latent, int32_t batch, int32_t frames, float* wav,
                             void* stream) {
  return guard([&] {
    need(c, "codec");
    need(latent, "latent");
    need(wav, "wav");
    irt::codec_decode_noalloc(*c->c, latent, batch, frames, wav, reinterpret_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
