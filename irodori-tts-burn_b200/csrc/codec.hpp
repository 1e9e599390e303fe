// DACVAE decoder object (src/codec/model.rs:18-65).
#pragma once

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.hpp"
#include "kernels.hpp"

namespace irt {

// One implicit-GEMM convolution launch of the bf16 tensor-core decoder
// (conv_tc.cu).  A = bf16 rows [rows_in, cin]; weights packed bf16
// [phases][cout][taps][cin_pad].
struct ConvTcArgs {
  int rows_in = 0, cin = 0, cin_pad = 0, taps = 1, phases = 1, cout = 0;
  int dil = 1, pad = 0;         // conv1d: tap offset = tap * dil - pad
  int convt = 0, stride = 1;    // ConvTranspose1d (kernel 2 * stride, padding pad)
  int rows_out = 0;             // output rows
  int out_scale = 1;            // output rows per latent frame
  const int* frame_src = nullptr;  // per latent frame: utterance frame index, or -1 for a gap
  const float* bias = nullptr;
  const float* alpha = nullptr;    // Snake alpha applied to the bf16 output (nullptr: identity)
  const float* alpha_inv = nullptr;  // 1 / (alpha + 1e-9) per channel (with alpha)
  float* x = nullptr;              // f32 output rows [rows_out, cout] (nullptr: not written)
  int add_res = 0;                 // x = x + conv (residual, in place)
  bf16* p = nullptr;               // bf16 output rows [rows_out, cout] (nullptr: not written)
  int ct_tma = 0;                  // ConvTranspose outputs by phased TMA stores (set by conv_tc)
};

int conv_tc_bn(int cout);
void conv_tc(const bf16* in, const bf16* w, const ConvTcArgs& a, cudaStream_t s);
void pack_latent_rows(const float* lat, const int* frame_src, bf16* out, int F, cudaStream_t s);
void codec_head_rows(const bf16* x, int R, int C, const float* w, const float* bias, int K, int pad,
                     const int* frame_src, int hop, float* wav, cudaStream_t s);
int conv_tc_read_and_clear_error();
int conv_watchdog_probe(unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns);

struct Codec {
  struct Conv {
    int cin = 0, cout = 0, k = 1, dil = 1, pad = 0;
    DevBuf w, b;
    DevBuf wp;  // bf16 mode: packed [phases][cout][taps][cin_pad]
    int cin_pad = 0, phases = 1;
    // f32 mode on the tf32 GEMM: per phase [cout_pad][hi: taps x cp | lo: taps x cp]
    DevBuf w2;
    int cp = 0, cout_pad = 0;
  };
  struct Res {
    DevBuf a0, a2;
    Conv c1, c3;
  };
  struct Block {
    int stride = 1;
    DevBuf alpha;
    Conv ct;
    Res res[3];
  };
  int device = 0, prec = IRT_PREC_F32;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  Conv qout, stem, head;
  Block blocks[4];
  DevBuf head_alpha;
  // 1 / (alpha + 1e-9) of every Snake alpha above, keyed by the alpha buffer
  // (the tensor-core epilogue multiplies instead of dividing per element)
  std::map<const void*, DevBuf> snake_inv;
  const float* inv_of(const float* alpha) const;
  DevBuf in, buf0, buf1, buf2;
  // bf16 tensor-core path: row buffers and the frame table
  bool tc = false;
  DevBuf rx, rp, rq, frames, wav_dev;
  // f32 mode: every convolution on the tf32 hi / lo GEMM (codec_tf32.cu),
  // unless IRT_CODEC_F32_SIMT=1 or a layer does not fit it (then SIMT)
  bool tf32 = false;
  DevBuf fx, fy, fa2, fmap;
  long long last_launches = 0;

  Codec(int dev, const std::string& path, int precision);
  ~Codec();
  // lengths: optional host array [B] of valid frames per utterance (ragged
  // batch; samples past lengths[b] * hop are zero).  nullptr = all T frames.
  void decode(const float* latent, int B, int T, float* wav, int memory, cudaStream_t s,
              const int* lengths = nullptr);

 private:
  void pack_tc_weights();
  void decode_tc(const float* latent_dev, int B, int T, const int* lengths, float* wav_dev, cudaStream_t s);
};

// f32 decode on the tf32 GEMM (codec_tf32.cu): weight packing at load, the
// support check, and the decode of one utterance (lat [T, 32], wav [T * hop]).
void codec_pack_tf32_conv(Codec::Conv& c, const std::vector<float>& w);
void codec_pack_tf32_convt(Codec::Conv& c, const std::vector<float>& w, int stride);
bool codec_tf32_supported(const Codec& c);
void codec_decode_tf32(Codec& c, const float* lat, int T, float* wav, cudaStream_t s);

// Allocation-free decode into a fixed device scratch array (codec_noalloc.cu).
void codec_decode_noalloc(Codec& c, const float* latent, int B, int T, float* wav, cudaStream_t s);
size_t codec_noalloc_scratch_floats();
// Resolves the scratch array's address on the current device (best effort;
// called by the Codec constructor with its device current).
void codec_noalloc_prepare();

}  // namespace irt
