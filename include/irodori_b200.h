/*
 * irodori_b200.h -- C ABI of the B200 (sm_100a) rectified-flow sampling
 * engine and DACVAE decoder.
 *
 * Drop-in boundary for the Irodori-TTS-burn crate's sampling path.  Each entry
 * point names the reference interface it replaces (paths relative to the
 * Irodori-TTS-burn crate root).  Plain C types only: pointers, sizes, PODs.
 *
 * Conventions
 *   - Every function returns an irt_status (0 = IRT_OK).  On failure the
 *     message is available from irt_last_error() on the calling thread.
 *   - The caller owns every input and output buffer; nothing is retained past
 *     a call.  The engine owns weights, context KV caches and workspaces.
 *   - Calls on one engine are serialised by an internal mutex; engines on
 *     different devices may be driven concurrently from different threads.
 *   - Masks are uint8 (non-zero = valid / attend), token ids int32, latents
 *     and audio float32, all row-major.
 */
#ifndef IRODORI_B200_H
#define IRODORI_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define IRT_API __attribute__((visibility("default")))
#else
#define IRT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: 1..11 map 1:1 onto IrodoriError variants (src/error.rs:3-60). */
typedef enum irt_status {
  IRT_OK = 0,
  IRT_E_CONFIG = 1,        /* IrodoriError::Config        */
  IRT_E_SHAPE = 2,         /* IrodoriError::Shape         */
  IRT_E_MISSING_INPUT = 3, /* IrodoriError::MissingInput  */
  IRT_E_UNSUPPORTED = 4,   /* IrodoriError::UnsupportedMode */
  IRT_E_IO = 5,            /* IrodoriError::Io            */
  IRT_E_JSON = 6,          /* IrodoriError::Json          */
  IRT_E_WEIGHT = 7,        /* IrodoriError::Weight (missing tensor key) */
  IRT_E_WRONG_DIM = 8,     /* IrodoriError::WrongDim      */
  IRT_E_DTYPE = 9,         /* IrodoriError::Dtype         */
  IRT_E_SAFETENSORS = 10,  /* IrodoriError::SafeTensors   */
  IRT_E_NO_CONFIG = 11,    /* IrodoriError::NoConfig      */
  IRT_E_CUDA = 20,         /* CUDA runtime/driver error   */
  IRT_E_STATE = 21,        /* call out of order (type-state violation) */
  IRT_E_INVALID_ARG = 22,  /* NULL handle / pointer, bad enum value */
  IRT_E_OOM = 23           /* device allocation failed    */
} irt_status;

/* SamplerMethod (src/config/sampling.rs:8-19). */
typedef enum irt_sampler_method { IRT_EULER = 0, IRT_HEUN = 1, IRT_PLMS4 = 2 } irt_sampler_method;

/* CfgGuidanceMode (src/config/sampling.rs; used at src/rf/euler_sampler.rs:397-512). */
typedef enum irt_cfg_mode {
  IRT_CFG_INDEPENDENT = 0,
  IRT_CFG_JOINT = 1,
  IRT_CFG_ALTERNATING = 2
} irt_cfg_mode;

/* Arithmetic of the DiT / encoder path.  BF16: bf16 operands on tcgen05
 * tensor cores with f32 accumulation and an f32 residual stream.  F32 (parity
 * mode): f32 data throughout; GEMMs of 128 or more rows on tcgen05 in tf32
 * over hi / lo operand halves with chunked f32 accumulation (error at the
 * level of an f32 SIMT product), the rest in fp32 SIMT arithmetic
 * (IRT_F32_SIMT=1 in the environment at engine creation: all SIMT). */
typedef enum irt_precision { IRT_PREC_BF16 = 0, IRT_PREC_F32 = 1 } irt_precision;

/* Where the pointers of a request / output live. */
typedef enum irt_memory { IRT_MEM_HOST = 0, IRT_MEM_DEVICE = 1 } irt_memory;

/*
 * SamplerParams + GuidanceConfig + TemporalRescaleConfig + SpeakerKvConfig
 * (src/rf/params.rs:9-92) flattened into one POD.  Optional fields carry a
 * has_* flag.  irt_sampler_params_default() fills the reference defaults
 * (src/rf/params.rs:24-35, :80-92).
 */
typedef struct irt_sampler_params {
  uint32_t num_steps;          /* default 40 */
  int32_t method;              /* irt_sampler_method, default EULER */
  int32_t cfg_mode;            /* irt_cfg_mode, default INDEPENDENT */
  float scale_text;            /* default 3.0 */
  float scale_caption;         /* default 3.0 */
  float scale_speaker;         /* default 5.0 */
  float min_t;                 /* default 0.5 */
  float max_t;                 /* default 1.0 */
  int32_t has_truncation;      /* truncation_factor: Option<f32> */
  float truncation_factor;
  int32_t has_temporal_rescale; /* temporal_rescale: Option<{k, sigma}> */
  float rescale_k;
  float rescale_sigma;
  int32_t has_speaker_kv;      /* speaker_kv: Option<SpeakerKvConfig> */
  float speaker_kv_scale;
  int32_t speaker_kv_max_layers; /* < 0 = None (all layers) */
  int32_t has_speaker_kv_min_t;
  float speaker_kv_min_t;
  int32_t use_context_kv_cache; /* default 1 (cached == uncached numerically) */
} irt_sampler_params;

/*
 * SamplingRequest (src/rf/params.rs:234-247).  Optional inputs are NULL.
 * `sequence_lengths` (NULL = every utterance has `sequence_length` frames)
 * extends the reference for ragged batches: utterance b then owns frames
 * [0, sequence_lengths[b]) of its row and the padding frames are left zero.
 */
typedef struct irt_request {
  int32_t batch;
  int32_t text_len;
  const int32_t* text_ids;        /* [batch, text_len] */
  const uint8_t* text_mask;       /* [batch, text_len] */
  int32_t ref_len;                /* 0 when no speaker reference */
  int32_t ref_dim;                /* latent width of ref_latent */
  const float* ref_latent;        /* [batch, ref_len, ref_dim] or NULL */
  const uint8_t* ref_mask;        /* [batch, ref_len] or NULL */
  int32_t caption_len;
  const int32_t* caption_ids;     /* [batch, caption_len] or NULL */
  const uint8_t* caption_mask;    /* [batch, caption_len] or NULL */
  int32_t sequence_length;        /* output frames (max over the batch) */
  const int32_t* sequence_lengths;/* [batch] or NULL (ragged extension, host memory) */
  const float* initial_noise;     /* [batch, sequence_length, P] or NULL */
  uint64_t seed;                  /* noise seed when initial_noise is NULL */
  int32_t memory;                 /* irt_memory of text/ref/caption/noise pointers */
} irt_request;

/* ---- errors -------------------------------------------------------------- */

/* Last error message of the calling thread ("" if none). */
IRT_API const char* irt_last_error(void);
/* Library version string. */
IRT_API const char* irt_version(void);

/* ---- sampler parameters -------------------------------------------------- */

/* SamplerParams::default() (src/rf/params.rs:80-92). */
IRT_API void irt_sampler_params_default(irt_sampler_params* p);
/* SamplerParams::validate() (src/rf/params.rs:99-183): IRT_OK or IRT_E_CONFIG
 * with the reference's message text in irt_last_error(). */
IRT_API int irt_sampler_params_validate(const irt_sampler_params* p);

/* ---- engine (InferenceBuilder / InferenceEngine, src/inference.rs:83-254) -- */

typedef struct irt_engine irt_engine;

/* InferenceBuilder::new(device).load_weights(path) (src/inference.rs:93-116):
 * reads the safetensors checkpoint and its `config_json` metadata
 * (src/weights/tensor_store.rs:26-53, src/weights/loaders.rs:18-29), validates
 * the ModelConfig (src/config/model.rs:95-223), uploads and pre-packs the
 * weights (fused [Wq|Wk|Wv|Wgate] and [W1|W3] as InferenceOptimizedModel::from
 * does, src/model/attention.rs:514-523, src/model/feed_forward.rs:96-103).
 * The engine starts in the Loaded state with no sampling parameters. */
IRT_API int irt_engine_create(int device, const char* safetensors_path, int precision, irt_engine** out);
/* InferenceBuilder::load_weights_with_adapter(path, adapter_dir) (feature
 * "lora", src/inference.rs:118-139): as irt_engine_create, with the PEFT LoRA
 * adapter in adapter_dir (adapter_config.json + adapter_model.safetensors)
 * merged into the base weights at load, W += (lora_alpha / r) * B A, and each
 * merged weight re-encoded to its checkpoint dtype (src/lora.rs:205-322,
 * src/weights/tensor_store.rs:62-118). */
IRT_API int irt_engine_create_with_adapter(int device, const char* safetensors_path, const char* adapter_dir,
                                           int precision, irt_engine** out);
/* Drop. */
IRT_API int irt_engine_destroy(irt_engine* e);
/* with_sampling(params) (src/inference.rs:151-155, :166-172, :231-233):
 * validates and stores the parameters; Loaded/Ready -> Ready. */
IRT_API int irt_engine_set_sampling(irt_engine* e, const irt_sampler_params* p);
/* with_default_sampling() (src/inference.rs:158-164). */
IRT_API int irt_engine_set_default_sampling(irt_engine* e);
/* sampling_params() (src/inference.rs:240-243). IRT_E_STATE before set_sampling. */
IRT_API int irt_engine_get_sampling(const irt_engine* e, irt_sampler_params* out);
/* model_config() (src/inference.rs:235-238): writes the config JSON (NUL
 * terminated) into buf; *len receives the required size including the NUL. */
IRT_API int irt_engine_get_config(const irt_engine* e, char* buf, size_t cap, size_t* len);
/* patched_latent_dim() (src/model/optimized.rs:139-141). */
IRT_API int irt_engine_patched_latent_dim(const irt_engine* e, int32_t* out);
/* use_speaker_condition() (src/model/optimized.rs:133-136). */
IRT_API int irt_engine_use_speaker_condition(const irt_engine* e, int32_t* out);

/* InferenceEngine::sample(request) -> sample_euler_rf_cfg
 * (src/inference.rs:222-227, src/rf/euler_sampler.rs:132-718).
 * out_latent: [batch, sequence_length, patched_latent_dim] float32, in
 * `out_memory` (irt_memory).  stream: a cudaStream_t or NULL (the engine's
 * own stream).  Returns after the result is complete in out_latent. */
IRT_API int irt_engine_sample(irt_engine* e, const irt_request* req, float* out_latent, int out_memory,
                      void* stream);

/* Number of DiT row-forwards and kernel launches of the last sample() call
 * (instrumentation for the benchmark). */
IRT_API int irt_engine_last_stats(const irt_engine* e, int64_t* row_forwards, int64_t* kernel_launches);

/* ---- DACVAE codec (src/codec/weights.rs:27-33, src/codec/model.rs:60-65) -- */

typedef struct irt_codec irt_codec;

/* load_codec(path, device): decoder-path tensors of a weight-norm-resolved
 * DACVAE safetensors file (keys of src/codec/weights.rs:219-292).
 * precision IRT_PREC_BF16: implicit-GEMM tcgen05 convolutions (bf16 operands,
 * f32 accumulation and residual stream); IRT_PREC_F32: f32 data, convolutions
 * as implicit GEMMs on tcgen05 in tf32 over hi / lo operand halves with
 * chunked f32 accumulation (IRT_CODEC_F32_SIMT=1 at creation: fp32 SIMT
 * kernels). */
IRT_API int irt_codec_create(int device, const char* safetensors_path, int precision, irt_codec** out);
IRT_API int irt_codec_destroy(irt_codec* c);
/* sample_rate() = 48000, hop_length() = 1920 (src/codec/model.rs:30-37). */
IRT_API int irt_codec_sample_rate(const irt_codec* c, int32_t* out);
IRT_API int irt_codec_hop_length(const irt_codec* c, int32_t* out);
/* DacVaeCodec::decode: latent [B, T, 32] -> wav [B, 1, T*1920]. */
IRT_API int irt_codec_decode(irt_codec* c, const float* latent, int32_t batch, int32_t frames, float* wav,
                     int memory, void* stream);
/* Ragged-batch extension of DacVaeCodec::decode (the reference decodes a
 * padded batch as one tensor): utterance b has lengths[b] (host int32, 0 <=
 * lengths[b] <= frames) valid latent frames and is decoded exactly as if it
 * were decoded alone at that length; wav samples past lengths[b] * hop are 0.
 * Used by batched text-to-waveform serving, where padding would be decoded
 * and thrown away. */
IRT_API int irt_codec_decode_ragged(irt_codec* c, const float* latent, int32_t batch, int32_t frames,
                                    const int32_t* lengths, float* wav, int memory, void* stream);

/*
 * Allocation-free variant of irt_codec_decode.  No counterpart in the
 * reference crate: it exists for callers that cannot allocate device memory
 * during a decode -- a real-time streaming loop that cannot absorb the
 * device-wide synchronisation of cudaMalloc/cudaFree, or a host application
 * whose own allocator already holds the free HBM.  All intermediate
 * activations live in one 16 MiB device array compiled into the library (held
 * by every GPU that loads it until exit), so the call allocates nothing.
 * It always runs the fp32 SIMT decoder, whatever the codec's precision.
 *   - latent [batch, frames, 32] and wav [batch, 1, frames * hop] must be
 *     device memory of the codec's own GPU (or managed memory): the kernels
 *     read and write them in place.  Anything else fails with
 *     IRT_E_INVALID_ARG.  The call returns once wav is complete.
 *   - Capacity: batch * frames <= 7 latent frames (280 ms) for the full-width
 *     DACVAE; larger requests fail with IRT_E_SHAPE and run nothing.
 *   - The array is shared by every call on a device and keeps the last call's
 *     contents (nothing in it needs to start at zero); calls that overlap on the
 *     GPU race and must be serialised by the caller.
 *   - irt_codec_create resolves the array's device address on its GPU (under
 *     lazy module loading, the moment the array is placed on that GPU); if
 *     that failed, the first call retries it and reports the failure.
 *   - Every call ends by synchronising its stream, so it cannot be recorded
 *     into a CUDA graph by stream capture.
 */
IRT_API int irt_codec_decode_noalloc(irt_codec* c, const float* latent, int32_t batch, int32_t frames, float* wav,
                                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IRODORI_B200_H */
