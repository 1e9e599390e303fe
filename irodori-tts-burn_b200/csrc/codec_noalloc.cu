// Allocation-free DACVAE decode (irt_codec_decode_noalloc).
//
// Who needs it: callers that must not allocate device memory while decoding --
// e.g. a real-time streaming loop that decodes short latent chunks and cannot
// afford the implicit device-wide synchronisation of cudaMalloc / cudaFree, or
// a host application whose framework allocator has already reserved the free
// HBM so that a fresh cudaMalloc would fail.  This path decodes with the fp32
// SIMT kernels of irt_codec_decode's f32 mode (whatever the codec's
// precision) but keeps every intermediate activation in one fixed device
// array compiled into the library, so a call performs no cudaMalloc, cudaFree
// or allocating library call.
//
// Limits and sharing rules:
//  - The scratch array holds CODEC_NOALLOC_SCRATCH_FLOATS floats (16 MiB).
//    Every GPU that loads the library keeps it until the process exits.
//  - A decode of B x T latent frames needs 3 * max_stage_elements floats, where
//    max_stage_elements = B * T * max over decoder stages of (channels x
//    upsampling so far); for the full-width DACVAE that is B * T * 96 * 1920,
//    so B * T <= 7 latent frames (280 ms of audio) per call.  Larger requests
//    are rejected with IRT_E_SHAPE before anything runs.
//  - latent and wav must be device memory of the codec's own GPU (or managed
//    memory): the kernels read and write them in place, with no staging copy.
//  - All calls on a device share the one array and it keeps the previous
//    call's contents; no part of it needs to start at zero because every
//    kernel writes its whole output before that output is read.  Calls that
//    overlap on the GPU (other host threads, other streams, other codec
//    objects on the same device) race on the array and must be serialised by
//    the caller.
//  - The array's device address is resolved with cudaGetSymbolAddress once per
//    device, with that device current, when a codec is created on it
//    (irt_codec_create): under lazy module loading that is the moment the
//    16 MiB array is placed on the GPU, so a host whose allocator later takes
//    the free HBM still finds it there.  If that early resolution failed, the
//    first decode_noalloc call on the device retries it.
//  - A call ends with a synchronisation of its stream, so it cannot be
//    recorded into a CUDA graph by stream capture.
#include <mutex>

#include "codec.hpp"

namespace irt {

namespace {

constexpr size_t CODEC_NOALLOC_SCRATCH_FLOATS = size_t(4) << 20;  // 16 MiB

// File-scope scratch.  In host code this name is only a stand-in for the
// symbol: kernels receive the address resolved by cudaGetSymbolAddress.
static __device__ __align__(256) float g_codec_scratch[CODEC_NOALLOC_SCRATCH_FLOATS];

constexpr int MAX_DEVICES = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[MAX_DEVICES] = {};

float* scratch_for_current_device() {
  int dev = 0;
  IRT_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= MAX_DEVICES) throw Error(IRT_E_INVALID_ARG, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_codec_scratch);
    if (e != cudaSuccess || !p)
      throw Error(IRT_E_CUDA, std::string("cudaGetSymbolAddress(codec scratch) failed: ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

// True for managed memory, or device memory allocated on `device`.  A device
// pointer of another GPU is rejected: the kernels would dereference it from
// this GPU (no staging copy on this path).
bool is_device_pointer_on(const void* p, int device) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();  // reset the error the failed query left behind
    return false;
  }
  if (at.type == cudaMemoryTypeManaged) return true;
  return at.type == cudaMemoryTypeDevice && at.device == device;
}

}  // namespace

size_t codec_noalloc_scratch_floats() { return CODEC_NOALLOC_SCRATCH_FLOATS; }

// Resolve the scratch address for the current device ahead of the first
// decode_noalloc call (called when a codec is created).  A failure here is not
// an error of codec creation: it is cleared and the first decode_noalloc call
// retries and reports it.
void codec_noalloc_prepare() {
  try {
    (void)scratch_for_current_device();
  } catch (const Error&) {
    cudaGetLastError();
  }
}

// Decode `latent` [B, T, 32] (device) into `wav` [B, 1, T * hop] (device) using
// only the static scratch array.  Returns after the result is complete.
void codec_decode_noalloc(Codec& c, const float* latent, int B, int T, float* wav, cudaStream_t user_stream) {
  std::lock_guard<std::mutex> lock(c.mu);
  IRT_CUDA(cudaSetDevice(c.device));
  if (B <= 0 || T <= 0) throw shape_error("decode needs batch > 0 and frames > 0");
  if (!is_device_pointer_on(latent, c.device) || !is_device_pointer_on(wav, c.device))
    throw Error(IRT_E_INVALID_ARG,
                "decode_noalloc needs latent and wav in device memory of the codec's GPU (" +
                    std::to_string(c.device) + ") or in managed memory");
  long maxel = (long)B * T * std::max(32, c.qout.cout);
  long t = T;
  maxel = std::max(maxel, (long)B * c.stem.cout * t);
  for (int i = 0; i < 4; ++i) {
    t *= c.blocks[i].stride;
    maxel = std::max(maxel, (long)B * c.blocks[i].ct.cout * t);
  }
  const size_t need = 3 * (size_t)maxel;
  if (need > CODEC_NOALLOC_SCRATCH_FLOATS)
    throw shape_error("decode_noalloc: " + std::to_string(B) + " x " + std::to_string(T) + " frames need " +
                      std::to_string(need) + " scratch floats; the fixed scratch holds " +
                      std::to_string(CODEC_NOALLOC_SCRATCH_FLOATS));
  cudaStream_t s = user_stream ? user_stream : c.stream;
  float* base = scratch_for_current_device();
  float* a = base;
  float* b = base + maxel;
  float* x = base + 2 * maxel;
  transpose_btc_bct(latent, x, B, T, 32, s);  // [B,T,32] -> [B,32,T]
  conv1d(x, B, 32, T, c.qout.w.as<float>(), c.qout.b.as<float>(), c.qout.cout, 1, 1, 0, nullptr, nullptr, 0, a, s);
  conv1d(a, B, c.qout.cout, T, c.stem.w.as<float>(), c.stem.b.as<float>(), c.stem.cout, c.stem.k, 1, c.stem.pad,
         nullptr, nullptr, 0, b, s);
  int C = c.stem.cout;
  long cur = T;
  std::swap(a, b);
  for (int i = 0; i < 4; ++i) {
    Codec::Block& bl = c.blocks[i];
    const long nt = cur * bl.stride;
    conv_transpose1d(a, B, C, (int)cur, bl.ct.w.as<float>(), bl.ct.b.as<float>(), bl.ct.cout, bl.stride, bl.ct.pad,
                     bl.alpha.as<float>(), b, (int)nt, s);
    C = bl.ct.cout;
    cur = nt;
    std::swap(a, b);
    for (int r = 0; r < 3; ++r) {
      Codec::Res& ru = bl.res[r];
      conv1d(a, B, C, (int)cur, ru.c1.w.as<float>(), ru.c1.b.as<float>(), C, ru.c1.k, ru.c1.dil, ru.c1.pad,
             ru.a0.as<float>(), nullptr, 0, b, s);
      conv1d(b, B, C, (int)cur, ru.c3.w.as<float>(), ru.c3.b.as<float>(), C, 1, 1, 0, ru.a2.as<float>(), a, 0, x, s);
      std::swap(a, x);
    }
  }
  conv1d(a, B, C, (int)cur, c.head.w.as<float>(), c.head.b.as<float>(), 1, c.head.k, 1, c.head.pad,
         c.head_alpha.as<float>(), nullptr, 1, wav, s);
  IRT_CUDA(cudaStreamSynchronize(s));
}

}  // namespace irt
