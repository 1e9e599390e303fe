// Bandwidth-bound row-wise and elementwise kernels of the sampling path.
// Each row kernel reads its row once, reduces in registers + shared memory,
// and writes its output once (coalesced, vectorised where aligned).
#include "common.hpp"
#include "epilogue.cuh"
#include "kernels.hpp"

namespace irt {

namespace {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < NT / 32) t = red[threadIdx.x];
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// mode 0: RmsNorm  y = x / rms * w         (src/model/norm.rs:25-39)
// mode 1: adaLN    y = x / rms * (1+scale) + shift   (src/model/norm.rs:160-172)
template <int NT, bool OBF>
__global__ void __launch_bounds__(NT) rownorm_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                                     const float* __restrict__ b, void* __restrict__ y, int D,
                                                     float eps, int mode) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const long row = blockIdx.x;
  const float* xr = x + row * D;
  float ss = 0.f;
  const bool vec = (D % 4) == 0;
  if (vec) {
    for (int i = threadIdx.x * 4; i < D; i += NT * 4) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  } else {
    for (int i = threadIdx.x; i < D; i += NT) ss += xr[i] * xr[i];
  }
  ss = block_sum<NT>(ss, red);
  const float rms = sqrtf(ss / (float)D + eps);
  auto f = [&](int i, float v) {
    float t = v / rms;
    if (mode == 0) return a ? t * a[i] : t;
    return t * (b[i] + 1.f) + a[i];
  };
  if (vec) {
    for (int i = threadIdx.x * 4; i < D; i += NT * 4) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      float o0 = f(i, v.x), o1 = f(i + 1, v.y), o2 = f(i + 2, v.z), o3 = f(i + 3, v.w);
      if (OBF) {
        bf16* yr = reinterpret_cast<bf16*>(y) + row * D + i;
        __nv_bfloat162 p0 = __floats2bfloat162_rn(o0, o1), p1 = __floats2bfloat162_rn(o2, o3);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&p0);
        u.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(yr) = u;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + row * D + i) = make_float4(o0, o1, o2, o3);
      }
    }
  } else {
    for (int i = threadIdx.x; i < D; i += NT) {
      float o = f(i, xr[i]);
      if (OBF) reinterpret_cast<bf16*>(y)[row * D + i] = __float2bfloat16_rn(o);
      else reinterpret_cast<float*>(y)[row * D + i] = o;
    }
  }
}

// Register-resident variant: each thread keeps up to VPT float4 of the row,
// so the row is read from memory once.  Same arithmetic as rownorm_kernel.
// SPLIT (bf16 output only): the row is written as two bf16 halves, hi =
// bf16(v) in columns [0, D) and lo = bf16(v - hi) in [D, 2D) of a 2D-wide row,
// for a GEMM whose weight is repeated along K ([W | W]): hi*W + lo*W carries
// the f32 value to ~2^-16 instead of one bf16 rounding.
template <int NT, int VPT, bool OBF, bool SPLIT = false>
__global__ void __launch_bounds__(NT) rownorm_reg_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                                         const float* __restrict__ b, void* __restrict__ y, int D,
                                                         float eps, int mode) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const long row = blockIdx.x;
  const int D4 = D >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + row * D);
  float4 v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    v[i] = c < D4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  ss = block_sum<NT>(ss, red);
  const float rms = sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * NT;
    if (c >= D4) continue;
    float o[4] = {v[i].x / rms, v[i].y / rms, v[i].z / rms, v[i].w / rms};
    if (mode == 0) {
      if (a) {
        const float4 w = reinterpret_cast<const float4*>(a)[c];
        o[0] *= w.x; o[1] *= w.y; o[2] *= w.z; o[3] *= w.w;
      }
    } else {
      const float4 sh = reinterpret_cast<const float4*>(a)[c];
      const float4 sc = reinterpret_cast<const float4*>(b)[c];
      o[0] = o[0] * (sc.x + 1.f) + sh.x;
      o[1] = o[1] * (sc.y + 1.f) + sh.y;
      o[2] = o[2] * (sc.z + 1.f) + sh.z;
      o[3] = o[3] * (sc.w + 1.f) + sh.w;
    }
    if (OBF) {
      __nv_bfloat162 p0 = __floats2bfloat162_rn(o[0], o[1]), p1 = __floats2bfloat162_rn(o[2], o[3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&p0);
      u.y = *reinterpret_cast<uint32_t*>(&p1);
      if (SPLIT) {
        const float2 h0 = __bfloat1622float2(p0), h1 = __bfloat1622float2(p1);
        __nv_bfloat162 l0 = __floats2bfloat162_rn(o[0] - h0.x, o[1] - h0.y);
        __nv_bfloat162 l1 = __floats2bfloat162_rn(o[2] - h1.x, o[3] - h1.y);
        uint2 ul;
        ul.x = *reinterpret_cast<uint32_t*>(&l0);
        ul.y = *reinterpret_cast<uint32_t*>(&l1);
        bf16* yr = reinterpret_cast<bf16*>(y) + row * 2 * D;
        reinterpret_cast<uint2*>(yr)[c] = u;
        reinterpret_cast<uint2*>(yr + D)[c] = ul;
      } else {
        reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(y) + row * D)[c] = u;
      }
    } else {
      reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + row * D)[c] = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Up to this many rows the row kernels run 256 threads x 2 float4 per row:
// at the config-3 sizes (750-1,500 rows) each launch is latency-bound, and the
// row kernels' share of the request's critical path (CUPTI trace) measured
// 10.7 ms against 12.3 ms for 128 x 4 (11.3 for 512 x 1, 24.4 for one warp per
// row); above it 128 x 4, the faster one on bandwidth.
constexpr int RN_SMALL_M = 8192;

void rownorm(const float* x, const float* a, const float* b, void* y, int out_bf16, int M, int D, float eps, int mode,
             cudaStream_t s) {
  if (M <= 0) return;
  // 128 threads x 4 float4 per row (rows up to D = 2048 held in registers):
  // measured 6.6 TB/s at 54,504 rows of 2048 against 5.9 TB/s for 256 x 2
  if ((D % 4) == 0 && D / 4 <= 256 * 2 && M <= RN_SMALL_M) {
    if (out_bf16) launch_pdl(rownorm_reg_kernel<256, 2, true>, dim3(M), dim3(256), 0, s, x, a, b, y, D, eps, mode);
    else launch_pdl(rownorm_reg_kernel<256, 2, false>, dim3(M), dim3(256), 0, s, x, a, b, y, D, eps, mode);
  } else if ((D % 4) == 0 && D / 4 <= 128 * 4) {
    if (out_bf16) launch_pdl(rownorm_reg_kernel<128, 4, true>, dim3(M), dim3(128), 0, s, x, a, b, y, D, eps, mode);
    else launch_pdl(rownorm_reg_kernel<128, 4, false>, dim3(M), dim3(128), 0, s, x, a, b, y, D, eps, mode);
  } else if (out_bf16) {
    launch_pdl(rownorm_kernel<256, true>, dim3(M), dim3(256), 0, s, x, a, b, y, D, eps, mode);
  } else {
    launch_pdl(rownorm_kernel<256, false>, dim3(M), dim3(256), 0, s, x, a, b, y, D, eps, mode);
  }
  IRT_CHECK_LAUNCH();
}

// out[m, n] = sum_d (x[m,d] / rms(x[m]) * nw[d]) * W[n, d] + bias[n]
// (out_norm RmsNorm + out_proj Linear, src/model/dit/model.rs:391-392), one
// warp per row, the normalised row staged once in shared memory, fp32 math.
template <bool WBF>
__global__ void __launch_bounds__(256) rmsnorm_proj_kernel(const float* __restrict__ x, const float* __restrict__ nw,
                                                           const void* __restrict__ W, const float* __restrict__ bias,
                                                           float* __restrict__ out, int M, int D, int P, float eps) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float xs_all[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long row = (long)blockIdx.x * (blockDim.x / 32) + warp;
  float* xs = xs_all + warp * D;
  if (row >= M) return;
  const float* xr = x + row * D;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) ss += xr[d] * xr[d];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = sqrtf(ss / (float)D + eps);
  for (int d = lane; d < D; d += 32) xs[d] = xr[d] / rms * nw[d];
  __syncwarp();
  // 4 outputs at a time; each lane owns 8 consecutive columns per 256-column
  // slab so weight rows are read with 16-byte (bf16) / 32-byte (f32) vectors.
  constexpr int NB = 4;
  const bool vec = (D % 256) == 0;
  for (int n0 = 0; n0 < P; n0 += NB) {
    float acc[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) acc[j] = 0.f;
    if (vec) {
      for (int d0 = lane * 8; d0 < D; d0 += 256) {
        const float4 x0 = *reinterpret_cast<const float4*>(xs + d0);
        const float4 x1 = *reinterpret_cast<const float4*>(xs + d0 + 4);
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const int n = n0 + j < P ? n0 + j : P - 1;
          float wv[8];
          if (WBF) {
            const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(W) + (long)n * D + d0);
            const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              wv[2 * k] = __bfloat162float(w2[k].x);
              wv[2 * k + 1] = __bfloat162float(w2[k].y);
            }
          } else {
            const float* wp = reinterpret_cast<const float*>(W) + (long)n * D + d0;
            const float4 a = *reinterpret_cast<const float4*>(wp), b = *reinterpret_cast<const float4*>(wp + 4);
            wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w; wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[j] = fmaf(xv[k], wv[k], acc[j]);
        }
      }
    } else {
      for (int d = lane; d < D; d += 32) {
        const float xv = xs[d];
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const int n = n0 + j < P ? n0 + j : P - 1;
          const float wv = WBF ? __bfloat162float(reinterpret_cast<const bf16*>(W)[(long)n * D + d])
                               : reinterpret_cast<const float*>(W)[(long)n * D + d];
          acc[j] = fmaf(xv, wv, acc[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane < NB && n0 + lane < P) {
      float r = acc[0];
#pragma unroll
      for (int j = 1; j < NB; ++j) r = lane == j ? acc[j] : r;
      out[row * P + n0 + lane] = r + (bias ? bias[n0 + lane] : 0.f);
    }
  }
}

__global__ void embed_kernel(const int* ids, const uint8_t* mask, const float* table, float* x, int M, int D,
                             int vocab) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)M * D) return;
  int m = (int)(i / D), d = (int)(i % D);
  int id = ids[m];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  float mk = mask ? (mask[m] ? 1.f : 0.f) : 1.f;
  x[i] = table[(long)id * D + d] * mk;
}

__global__ void gather_kernel(const float* in, const int* src, void* out, int out_bf16, int M, int D, int ldo) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)M * D) return;
  int m = (int)(i / D), d = (int)(i % D);
  int r = src ? src[m] : m;
  float v = in[(long)r * D + d];
  const long o = (long)m * ldo + d;
  if (out_bf16) reinterpret_cast<bf16*>(out)[o] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(out)[o] = v;
}

// f32 rows [M, P] -> bf16 [M, 2 Pk]: hi = bf16(v) at column d, lo = bf16(v - hi)
// at column Pk + d (padding columns are left untouched).
__global__ void gather_split_kernel(const float* in, bf16* out, int M, int P, int Pk) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)M * P) return;
  const int m = (int)(i / P), d = (int)(i % P);
  const float v = in[i];
  const bf16 hi = __float2bfloat16_rn(v);
  bf16* o = out + (long)m * 2 * Pk;
  o[d] = hi;
  o[Pk + d] = __float2bfloat16_rn(v - __bfloat162float(hi));
}

__global__ void mask_rows_kernel(float* x, const uint8_t* mask, int M, int D) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)M * D) return;
  if (!mask[i / D]) x[i] = x[i] * 0.f;
}

__global__ void silu_copy_kernel(const float* in, long ld_in, float* out, long ld_out, int M, int D) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)M * D) return;
  int m = (int)(i / D), d = (int)(i % D);
  out[(long)m * ld_out + d] = silu_f(in[(long)m * ld_in + d]);
}

// One block per (batch, 256-wide column slice).
__global__ void mean_token_kernel(const float* state, const uint8_t* mask, float* out, uint8_t* mask_out, int S,
                                  int D) {
  const int b = blockIdx.y;
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  float cnt = 0.f;
  for (int s2 = 0; s2 < S; ++s2) cnt += mask[(long)b * S + s2] ? 1.f : 0.f;
  if (d < D) {
    float sum = 0.f;
    for (int s2 = 0; s2 < S; ++s2) {
      float mk = mask[(long)b * S + s2] ? 1.f : 0.f;
      float v = state[((long)b * S + s2) * D + d];
      sum += v * mk;
      out[((long)b * (S + 1) + s2 + 1) * D + d] = v;
    }
    out[(long)b * (S + 1) * D + d] = sum / fmaxf(cnt, 1.f);
  }
  if (blockIdx.x == 0) {
    for (int s2 = threadIdx.x; s2 < S + 1; s2 += blockDim.x)
      mask_out[(long)b * (S + 1) + s2] = s2 == 0 ? (cnt > 0.f ? 1 : 0) : mask[(long)b * S + s2 - 1];
  }
}

// v = v0 + sum_k (v0 - vk) * s_k   in the reference's accumulation order
// (src/rf/euler_sampler.rs:421-433, :464-468, :506-510).
__global__ void cfg_combine_kernel(const float* v, int ngroups, const float* scales, long ntok_p, float* out) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ntok_p) return;
  float v0 = v[i];
  float acc = v0;
  for (int k = 1; k < ngroups; ++k) acc = acc + (v0 - v[k * ntok_p + i]) * scales[k - 1];
  out[i] = acc;
}

__global__ void axpy_kernel(float* y, const float* x, float a, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = y[i] + x[i] * a;
}

struct LinArgs {
  const float* x[4];
  float c[4];
};
__global__ void lincomb_kernel(float* out, LinArgs a, int nx, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float r = a.x[0][i] * a.c[0];
  for (int k = 1; k < nx; ++k) r = r + a.x[k][i] * a.c[k];
  out[i] = r;
}

// (v * omt + x) * ratio / omt - x / omt   (src/rf/math.rs:38-52)
__global__ void trescale_kernel(float* v, const float* x, float omt, float ratio, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float xv = x[i];
  v[i] = (v[i] * omt + xv) * ratio / omt - xv / omt;
}

__global__ void scale_kernel(float* x, float a, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = x[i] * a;
}

__global__ void scale_rows_kernel(void* buf, int is_bf16, long row_len, const int* rows, int nrows, float a) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)nrows * row_len) return;
  long r = rows[i / row_len];
  long idx = r * row_len + i % row_len;
  if (is_bf16) {
    bf16* p = reinterpret_cast<bf16*>(buf);
    p[idx] = __float2bfloat16_rn(__bfloat162float(p[idx]) * a);
  } else {
    float* p = reinterpret_cast<float*>(buf);
    p[idx] = p[idx] * a;
  }
}

// Counter-based Gaussian: splitmix64 hash of (seed, index) -> two uniforms ->
// Box-Muller (cos branch).
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__global__ void gauss_kernel(float* x, long n, uint64_t seed) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint64_t h = splitmix64(seed ^ splitmix64((uint64_t)i));
  float u1 = ((h >> 40) + 1) * (1.0f / 16777217.0f);  // (0, 1]
  float u2 = ((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
  x[i] = sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
}

inline unsigned nblk(long n, int t = 256) { return (unsigned)((n + t - 1) / t); }

}  // namespace

void adaln_modulate(const float* x, const float* shift, const float* scale, void* h, int out_bf16, int M, int D,
                    float eps, cudaStream_t s) {
  rownorm(x, shift, scale, h, out_bf16, M, D, eps, 1, s);
}
void rms_norm(const float* x, const float* w, void* y, int out_bf16, int M, int D, float eps, cudaStream_t s) {
  rownorm(x, w, nullptr, y, out_bf16, M, D, eps, 0, s);
}
bool rms_norm_split_supported(int D) { return D % 4 == 0 && D / 4 <= 128 * 4; }
void rms_norm_split(const float* x, const float* w, bf16* y, int M, int D, float eps, cudaStream_t s) {
  if (M <= 0) return;
  if (!rms_norm_split_supported(D)) throw unsupported("rms_norm_split: D must be a multiple of 4 and <= 2048");
  if (M <= RN_SMALL_M)
    launch_pdl(rownorm_reg_kernel<256, 2, true, true>, dim3(M), dim3(256), 0, s, x, w, (const float*)nullptr,
               (void*)y, D, eps, 0);
  else
    launch_pdl(rownorm_reg_kernel<128, 4, true, true>, dim3(M), dim3(128), 0, s, x, w, (const float*)nullptr,
               (void*)y, D, eps, 0);
  IRT_CHECK_LAUNCH();
}
void rmsnorm_proj(const float* x, const float* nw, const void* W, int w_bf16, const float* bias, float* out, int M,
                  int D, int P, float eps, cudaStream_t s) {
  if (M <= 0) return;
  if (D * 4 * 4 > 48 * 1024) throw unsupported("rmsnorm_proj: model_dim > 3072");
  const int rows_per_block = 4;
  const unsigned grid = (unsigned)((M + rows_per_block - 1) / rows_per_block);
  const size_t smem = (size_t)rows_per_block * D * 4;
  if (w_bf16)
    launch_pdl(rmsnorm_proj_kernel<true>, dim3(grid), dim3(32 * rows_per_block), smem, s, x, nw, W, bias, out, M, D, P,
               eps);
  else
    launch_pdl(rmsnorm_proj_kernel<false>, dim3(grid), dim3(32 * rows_per_block), smem, s, x, nw, W, bias, out, M, D,
               P, eps);
  IRT_CHECK_LAUNCH();
}
void embed_rows_v(const int* ids, const uint8_t* mask, const float* table, float* x, int M, int D, int vocab,
                  cudaStream_t s) {
  if ((long)M * D == 0) return;
  embed_kernel<<<nblk((long)M * D), 256, 0, s>>>(ids, mask, table, x, M, D, vocab);
  IRT_CHECK_LAUNCH();
}
void embed_rows(const int* ids, const uint8_t* mask, const float* table, float* x, int M, int D, cudaStream_t s) {
  embed_rows_v(ids, mask, table, x, M, D, 1 << 30, s);
}
void gather_rows(const float* in, const int* src_row, void* out, int out_bf16, int M, int D, cudaStream_t s,
                 int ld_out) {
  if ((long)M * D == 0) return;
  gather_kernel<<<nblk((long)M * D), 256, 0, s>>>(in, src_row, out, out_bf16, M, D, ld_out > 0 ? ld_out : D);
  IRT_CHECK_LAUNCH();
}
void gather_split_rows(const float* in, bf16* out, int M, int P, int Pk, cudaStream_t s) {
  if ((long)M * P == 0) return;
  gather_split_kernel<<<nblk((long)M * P), 256, 0, s>>>(in, out, M, P, Pk);
  IRT_CHECK_LAUNCH();
}
void mask_rows(float* x, const uint8_t* mask, int M, int D, cudaStream_t s) {
  if ((long)M * D == 0) return;
  mask_rows_kernel<<<nblk((long)M * D), 256, 0, s>>>(x, mask, M, D);
  IRT_CHECK_LAUNCH();
}
void silu_copy(const float* in, long ld_in, float* out, long ld_out, int M, int D, cudaStream_t s) {
  if ((long)M * D == 0) return;
  silu_copy_kernel<<<nblk((long)M * D), 256, 0, s>>>(in, ld_in, out, ld_out, M, D);
  IRT_CHECK_LAUNCH();
}
void prepend_mean_token(const float* state, const uint8_t* mask, float* out, uint8_t* mask_out, int B, int S, int D,
                        cudaStream_t s) {
  if (B == 0) return;
  dim3 grid((D + 255) / 256, B);
  mean_token_kernel<<<grid, 256, 0, s>>>(state, mask, out, mask_out, S, D);
  IRT_CHECK_LAUNCH();
}
void cfg_combine(const float* v_packed, const int*, const float* scales, int ngroups, const int*, int ntok, int P,
                 float* v_out, cudaStream_t s) {
  long n = (long)ntok * P;
  if (n == 0) return;
  cfg_combine_kernel<<<nblk(n), 256, 0, s>>>(v_packed, ngroups, scales, n, v_out);
  IRT_CHECK_LAUNCH();
}
void axpy(float* y, const float* x, float a, long n, cudaStream_t s) {
  if (n == 0) return;
  axpy_kernel<<<nblk(n), 256, 0, s>>>(y, x, a, n);
  IRT_CHECK_LAUNCH();
}
void lincomb(float* out, const float* const* xs, const float* coefs, int nx, long n, cudaStream_t s) {
  if (n == 0) return;
  LinArgs a{};
  for (int k = 0; k < nx && k < 4; ++k) { a.x[k] = xs[k]; a.c[k] = coefs[k]; }
  lincomb_kernel<<<nblk(n), 256, 0, s>>>(out, a, nx, n);
  IRT_CHECK_LAUNCH();
}
void temporal_rescale(float* v, const float* x, float omt, float ratio, long n, cudaStream_t s) {
  if (n == 0) return;
  trescale_kernel<<<nblk(n), 256, 0, s>>>(v, x, omt, ratio, n);
  IRT_CHECK_LAUNCH();
}
void scale_buf(float* x, float a, long n, cudaStream_t s) {
  if (n == 0) return;
  scale_kernel<<<nblk(n), 256, 0, s>>>(x, a, n);
  IRT_CHECK_LAUNCH();
}
void scale_rows_bf16_or_f32(void* buf, int is_bf16, long row_len, const int* rows, int nrows, float a,
                            cudaStream_t s) {
  long n = (long)nrows * row_len;
  if (n == 0) return;
  scale_rows_kernel<<<nblk(n), 256, 0, s>>>(buf, is_bf16, row_len, rows, nrows, a);
  IRT_CHECK_LAUNCH();
}
void gaussian_fill(float* x, long n, uint64_t seed, cudaStream_t s) {
  if (n == 0) return;
  gauss_kernel<<<nblk(n), 256, 0, s>>>(x, n, seed);
  IRT_CHECK_LAUNCH();
}

}  // namespace irt
