// Shared host-side definitions: error type mirroring IrodoriError, CUDA
// checks, small device buffer RAII.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>

#include "../../include/irodori_b200.h"

namespace irt {

// One exception type carrying an irt_status; every C entry point converts it
// into the status return value plus the thread-local last-error string.
struct Error : std::runtime_error {
  int status;
  Error(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

// Message prefixes follow the reference's `#[error(...)]` strings
// (src/error.rs:3-60) so callers see the same text.
inline Error config_error(const std::string& m) { return Error(IRT_E_CONFIG, "Invalid configuration: " + m); }
inline Error shape_error(const std::string& m) { return Error(IRT_E_SHAPE, "Shape mismatch: " + m); }
inline Error missing_input(const std::string& m) { return Error(IRT_E_MISSING_INPUT, "Missing required input: " + m); }
inline Error unsupported(const std::string& m) { return Error(IRT_E_UNSUPPORTED, "Unsupported mode: " + m); }
inline Error weight_error(const std::string& k) { return Error(IRT_E_WEIGHT, "Missing weight tensor: " + k); }

#define IRT_CUDA(expr)                                                                         \
  do {                                                                                         \
    cudaError_t _e = (expr);                                                                   \
    if (_e != cudaSuccess)                                                                     \
      throw ::irt::Error(IRT_E_CUDA, std::string("CUDA error: ") + cudaGetErrorString(_e) +   \
                                         " at " + __FILE__ + ":" + std::to_string(__LINE__)); \
  } while (0)

// Kernel launches issued by this library (instrumentation for the benchmark).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}

#define IRT_CHECK_LAUNCH()                                     \
  do {                                                         \
    ::irt::launch_counter().fetch_add(1, std::memory_order_relaxed); \
    IRT_CUDA(cudaGetLastError());                              \
  } while (0)

// Programmatic dependent launch (PDL).  A kernel launched with launch_pdl()
// may start while its predecessor on the stream is still running; it must
// execute pdl_wait() in every CTA before it reads anything a predecessor
// wrote (pdl_wait returns once the predecessor grid has completed and its
// memory is visible, so ordering stays transitive).  pdl_trigger() lets the
// successor grid launch early; it never weakens the successor's own wait.
// Both are no-ops for kernels launched the ordinary way.  IRT_NO_PDL=1 in the
// environment launches everything the ordinary way.
#if defined(__CUDACC__)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("IRT_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  IRT_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}
#endif

// Owning device allocation (cudaMalloc / cudaFree).
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  explicit DevBuf(size_t n) { alloc(n); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) { release(); p = o.p; bytes = o.bytes; o.p = nullptr; o.bytes = 0; }
    return *this;
  }
  ~DevBuf() { release(); }
  void alloc(size_t n) {
    release();
    if (n == 0) return;
    cudaError_t e = cudaMalloc(&p, n);
    if (e != cudaSuccess) {
      p = nullptr;
      throw Error(IRT_E_OOM, "device allocation of " + std::to_string(n) + " bytes failed: " +
                                 cudaGetErrorString(e));
    }
    bytes = n;
  }
  // Grow-only reallocation (contents not preserved).
  void ensure(size_t n) {
    if (n > bytes) alloc(n);
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  template <class T> T* as() const { return reinterpret_cast<T*>(p); }
};

inline uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40);  // NaN
  uint32_t r = u + 0x7fffu + ((u >> 16) & 1u);  // round to nearest even
  return (uint16_t)(r >> 16);
}

}  // namespace irt
