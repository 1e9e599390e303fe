// DACVAE decoder object (src/codec/model.rs:18-65).
#pragma once

#include <mutex>
#include <string>

#include "common.hpp"
#include "kernels.hpp"

namespace irt {

struct Codec {
  struct Conv {
    int cin = 0, cout = 0, k = 1, dil = 1, pad = 0;
    DevBuf w, b;
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
  DevBuf in, buf0, buf1, buf2;
  long long last_launches = 0;

  Codec(int dev, const std::string& path, int precision);
  ~Codec();
  void decode(const float* latent, int B, int T, float* wav, int memory, cudaStream_t s);
};

// Allocation-free decode into a fixed device scratch array (codec_noalloc.cu).
void codec_decode_noalloc(Codec& c, const float* latent, int B, int T, float* wav, cudaStream_t s);
size_t codec_noalloc_scratch_floats();

}  // namespace irt
