// Fused GEMM epilogues shared by the tcgen05 kernel (accumulators in
// registers after tcgen05.ld) and the fp32 SIMT path (accumulators read back
// from a raw buffer).  `Acc` is a callable returning accumulator j of the
// current row chunk.
#pragma once

#include <cuda_bf16.h>
#include "kernels.hpp"

namespace irt {

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

__device__ __forceinline__ void store_val(void* base, long idx, int is_bf16, float v) {
  if (is_bf16) reinterpret_cast<bf16*>(base)[idx] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(base)[idx] = v;
}

__device__ __forceinline__ float apply_act(int act, float v) {
  if (act == ACT_SILU) return silu_f(v);
  if (act == ACT_TANH) return tanhf(v);
  return v;
}

// Contiguous run of W values of one row: vectorised store when possible.
template <int W>
__device__ __forceinline__ void store_run(void* base, long idx, int is_bf16, const float (&v)[W]) {
  if (is_bf16) {
    bf16* d = reinterpret_cast<bf16*>(base) + idx;
    if ((W % 8) == 0 && ((reinterpret_cast<uintptr_t>(d) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < W; j += 8) {
        uint4 u;
        __nv_bfloat162 t0 = __floats2bfloat162_rn(v[j], v[j + 1]);
        __nv_bfloat162 t1 = __floats2bfloat162_rn(v[j + 2], v[j + 3]);
        __nv_bfloat162 t2 = __floats2bfloat162_rn(v[j + 4], v[j + 5]);
        __nv_bfloat162 t3 = __floats2bfloat162_rn(v[j + 6], v[j + 7]);
        u.x = *reinterpret_cast<uint32_t*>(&t0);
        u.y = *reinterpret_cast<uint32_t*>(&t1);
        u.z = *reinterpret_cast<uint32_t*>(&t2);
        u.w = *reinterpret_cast<uint32_t*>(&t3);
        *reinterpret_cast<uint4*>(d + j) = u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) d[j] = __float2bfloat16_rn(v[j]);
    }
  } else {
    float* d = reinterpret_cast<float*>(base) + idx;
    if ((W % 4) == 0 && ((reinterpret_cast<uintptr_t>(d) & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < W; j += 4) *reinterpret_cast<float4*>(d + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) d[j] = v[j];
    }
  }
}

// ---- STORE / RESID over a chunk of W columns [n0, n0+W) of row m ----------
template <int W, class Acc>
__device__ __forceinline__ void epi_chunk_store(const EpiParams& p, int m, int n0, const Acc& acc, long out_off = 0,
                                                long bias_off = 0, long add_off = 0) {
  int dst = p.row_map ? p.row_map[m] : m;
  if (dst < 0) return;
  float rs = p.row_scale ? p.row_scale[m] : 1.f;
  bool full = (n0 + W) <= p.N;
  float v[W];
#pragma unroll
  for (int j = 0; j < W; ++j) {
    int n = n0 + j;
    float a = acc(j);
    if (n < p.N) {
      if (p.bias) a += p.bias[bias_off + n];
      a *= p.alpha;
      if (p.add) a += p.add[add_off + (long)m * p.ld_add + n];
      a = apply_act(p.act, a) * rs;
    }
    v[j] = a;
  }
  long base = out_off + (long)dst * p.ldo + n0;
  if (full) {
    store_run<W>(p.out, base, p.out_bf16, v);
  } else {
    for (int j = 0; j < W && n0 + j < p.N; ++j) store_val(p.out, base + j, p.out_bf16, v[j]);
  }
}

template <int W, class Acc>
__device__ __forceinline__ void epi_chunk_resid(const EpiParams& p, int m, int n0, const Acc& acc) {
  float rs = p.row_scale ? p.row_scale[m] : 1.f;
  float* x = p.x + (long)m * p.N + n0;
  if (n0 + W <= p.N && ((reinterpret_cast<uintptr_t>(x) & 15) == 0)) {
#pragma unroll
    for (int j = 0; j < W; j += 4) {
      float4 xv = *reinterpret_cast<float4*>(x + j);
      float g0 = p.gate ? p.gate[n0 + j] : 1.f, g1 = p.gate ? p.gate[n0 + j + 1] : 1.f;
      float g2 = p.gate ? p.gate[n0 + j + 2] : 1.f, g3 = p.gate ? p.gate[n0 + j + 3] : 1.f;
      xv.x = (xv.x + g0 * acc(j)) * rs;
      xv.y = (xv.y + g1 * acc(j + 1)) * rs;
      xv.z = (xv.z + g2 * acc(j + 2)) * rs;
      xv.w = (xv.w + g3 * acc(j + 3)) * rs;
      *reinterpret_cast<float4*>(x + j) = xv;
    }
  } else {
    for (int j = 0; j < W && n0 + j < p.N; ++j) {
      float g = p.gate ? p.gate[n0 + j] : 1.f;
      x[j] = (x[j] + g * acc(j)) * rs;
    }
  }
}

// Split-K partial of the gated residual: x += gate * acc with vector atomics
// (the residual update is additive, so K-splits accumulate in any order).
template <int W, class Acc>
__device__ __forceinline__ void epi_chunk_resid_atomic(const EpiParams& p, int m, int n0, const Acc& acc) {
  float* x = p.x + (long)m * p.N + n0;
  if (n0 + W <= p.N && ((reinterpret_cast<uintptr_t>(x) & 15) == 0)) {
#pragma unroll
    for (int j = 0; j < W; j += 4) {
      const float4 g = p.gate ? *reinterpret_cast<const float4*>(p.gate + n0 + j) : make_float4(1.f, 1.f, 1.f, 1.f);
      atomicAdd(reinterpret_cast<float4*>(x + j),
                make_float4(g.x * acc(j), g.y * acc(j + 1), g.z * acc(j + 2), g.w * acc(j + 3)));
    }
  } else {
    for (int j = 0; j < W && n0 + j < p.N; ++j) atomicAdd(x + j, (p.gate ? p.gate[n0 + j] : 1.f) * acc(j));
  }
}

// ---- SWIGLU: columns [n0, n0+32) = w1 group, [n0+32, n0+64) = w3 group -----
template <class Acc, bool FAST = false>
__device__ __forceinline__ void epi_chunk_swiglu(const EpiParams& p, int m, int n0, const Acc& acc) {
  constexpr int G = SWIGLU_GROUP;
  int f0 = (n0 / (2 * G)) * G;
  float v[G];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const float a = acc(j);
    v[j] = (FAST ? __fdividef(a, 1.f + __expf(-a)) : silu_f(a)) * acc(G + j);
  }
  long base = (long)m * p.F + f0;
  if (f0 + G <= p.F) store_run<G>(p.h, base, p.out_bf16, v);
  else
    for (int j = 0; j < G && f0 + j < p.F; ++j) store_val(p.h, base + j, p.out_bf16, v[j]);
}

// ---- per-head chunk (QKVG / CTXKV): HD compile-time (>0) or runtime -------
// q/k: HeadRmsNorm (x / sqrt(mean(x^2)+eps) * w, src/model/norm.rs:60-74) then
// RoPE on interleaved pairs for heads < rope_heads (src/model/rope.rs:82-135);
// v: plain; g: sigmoid (the attention output gate, src/model/attention.rs:422).
template <int HD, class Acc>
__device__ __forceinline__ void epi_head(const EpiParams& p, int m, int n0, const Acc& acc) {
  const int hd = HD > 0 ? HD : p.hd;
  const int Dq = p.Dq;
  void* dst;
  long idx;
  const float* nw = nullptr;
  int rope = 0, pos = 0, act_sig = 0;
  if (p.mode == EPI_QKVG) {
    int which = n0 / Dq;
    int col = n0 - which * Dq;
    int head = col / hd;
    idx = (long)m * Dq + col;
    dst = which == 0 ? p.q : which == 1 ? p.k : which == 2 ? p.v : p.g;
    // no weights (null) means no head norm; offset only a real table
    if (which == 0 && p.qn_w) nw = p.qn_w + col;
    if (which == 1 && p.kn_w) nw = p.kn_w + col;
    if (which < 2 && head < p.rope_heads && p.rope_cos && p.rope_sin) { rope = 1; pos = p.tok_pos ? p.tok_pos[m] : m; }
    act_sig = which == 3;
  } else {  // EPI_CTXKV
    int dr = p.row_map ? p.row_map[m] : m;
    if (dr < 0) return;
    int l = n0 / (2 * Dq);
    int r = n0 - l * 2 * Dq;
    int part = r / Dq;
    int col = r - part * Dq;
    idx = (long)l * p.layer_stride + (long)dr * Dq + col;
    dst = part == 0 ? p.ck : p.cv;
    if (part == 0 && p.kn_w) nw = p.kn_w + (long)l * Dq + col;
  }
  float rms = 1.f;
  if (nw) {
    float ss = 0.f;
    if constexpr (HD > 0) {
#pragma unroll
      for (int j = 0; j < HD; ++j) { float a = acc(j); ss = fmaf(a, a, ss); }
    } else {
      for (int j = 0; j < hd; ++j) { float a = acc(j); ss = fmaf(a, a, ss); }
    }
    rms = sqrtf(ss / (float)hd + p.eps);
  }
  const float* cs = rope ? p.rope_cos + (long)pos * (hd / 2) : nullptr;
  const float* sn = rope ? p.rope_sin + (long)pos * (hd / 2) : nullptr;
  if constexpr (HD > 0) {
    // Tensor-core path (bf16 outputs): reciprocal multiply, vectorised
    // weight / table loads, fast sigmoid.
    const float inv = 1.f / rms;
#pragma unroll
    for (int j0 = 0; j0 < HD; j0 += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = acc(j0 + j);
      if (nw) {
        const float4 w0 = *reinterpret_cast<const float4*>(nw + j0);
        const float4 w1 = *reinterpret_cast<const float4*>(nw + j0 + 4);
        v[0] *= inv * w0.x; v[1] *= inv * w0.y; v[2] *= inv * w0.z; v[3] *= inv * w0.w;
        v[4] *= inv * w1.x; v[5] *= inv * w1.y; v[6] *= inv * w1.z; v[7] *= inv * w1.w;
      }
      if (rope) {
        const float4 c = *reinterpret_cast<const float4*>(cs + (j0 >> 1));
        const float4 s = *reinterpret_cast<const float4*>(sn + (j0 >> 1));
        const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float a0 = v[2 * k], a1 = v[2 * k + 1];
          v[2 * k] = a0 * cc[k] - a1 * ss[k];
          v[2 * k + 1] = a0 * ss[k] + a1 * cc[k];
        }
      }
      if (act_sig) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fdividef(1.f, 1.f + __expf(-v[j]));
      }
      store_run<8>(dst, idx + j0, p.out_bf16, v);
    }
    return;
  }
  auto val2 = [&](int j, float& a0, float& a1) {
    a0 = acc(j); a1 = acc(j + 1);
    if (nw) { a0 = a0 / rms * nw[j]; a1 = a1 / rms * nw[j + 1]; }
    if (rope) {
      float c = cs[j >> 1], s = sn[j >> 1];
      float r0 = a0 * c - a1 * s, r1 = a0 * s + a1 * c;
      a0 = r0; a1 = r1;
    }
    if (act_sig) { a0 = sigmoid_f(a0); a1 = sigmoid_f(a1); }
  };
  // runtime-hd path (fp32 parity mode): the reference's exact divide order
  for (int j = 0; j < hd; j += 2) {
    float a0, a1;
    val2(j, a0, a1);
    store_val(dst, idx + j, p.out_bf16, a0);
    store_val(dst, idx + j + 1, p.out_bf16, a1);
  }
}

// Tensor-core QKVG epilogue with bf16 output staged through shared memory.
// Lane i of the warp owns row m_base + i and all lanes work on the same head
// (128 columns starting at n0); the arithmetic is epi_head<128>'s.  Per
// 64-column half the warp's 32 x 64 bf16 block goes to a 4 KB buffer (16-byte
// chunks XOR-swizzled by row, so the 32 lanes' writes do not conflict) and is
// written back as whole 128-byte row segments, four rows per instruction,
// instead of one 16-byte store per lane into 32 different rows.  Rows at or
// past M are computed but not stored.
template <class Acc>
__device__ __forceinline__ void epi_head_staged(const EpiParams& p, int m_base, int lane, int M, int n0,
                                                const Acc& acc, uint4* buf) {
  constexpr int HD = 128;
  const int Dq = p.Dq;
  const int which = n0 / Dq;
  const int col = n0 - which * Dq;
  const int head = col / HD;
  bf16* dst = reinterpret_cast<bf16*>(which == 0 ? p.q : which == 1 ? p.k : which == 2 ? p.v : p.g);
  // no weights (null) means no head norm; offset only a real table
  const float* nw = (which == 0 && p.qn_w) ? p.qn_w + col : (which == 1 && p.kn_w) ? p.kn_w + col : nullptr;
  const bool rope = which < 2 && head < p.rope_heads && p.rope_cos && p.rope_sin;
  const bool act_sig = which == 3;
  const int m = m_base + lane;
  const int mc = m < M ? m : M - 1;  // table lookups stay in bounds for rows past M
  float inv = 1.f;
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < HD; ++j) { float a = acc(j); ss = fmaf(a, a, ss); }
    inv = 1.f / sqrtf(ss / (float)HD + p.eps);
  }
  const int pos = rope ? (p.tok_pos ? p.tok_pos[mc] : mc) : 0;
  const float* cs = rope ? p.rope_cos + (long)pos * (HD / 2) : nullptr;
  const float* sn = rope ? p.rope_sin + (long)pos * (HD / 2) : nullptr;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int j0 = half * 64 + c * 8;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = acc(j0 + j);
      if (nw) {
        const float4 w0 = *reinterpret_cast<const float4*>(nw + j0);
        const float4 w1 = *reinterpret_cast<const float4*>(nw + j0 + 4);
        v[0] *= inv * w0.x; v[1] *= inv * w0.y; v[2] *= inv * w0.z; v[3] *= inv * w0.w;
        v[4] *= inv * w1.x; v[5] *= inv * w1.y; v[6] *= inv * w1.z; v[7] *= inv * w1.w;
      }
      if (rope) {
        const float4 cc4 = *reinterpret_cast<const float4*>(cs + (j0 >> 1));
        const float4 ss4 = *reinterpret_cast<const float4*>(sn + (j0 >> 1));
        const float cc[4] = {cc4.x, cc4.y, cc4.z, cc4.w}, sv[4] = {ss4.x, ss4.y, ss4.z, ss4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float a0 = v[2 * k], a1 = v[2 * k + 1];
          v[2 * k] = a0 * cc[k] - a1 * sv[k];
          v[2 * k + 1] = a0 * sv[k] + a1 * cc[k];
        }
      }
      if (act_sig) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __fdividef(1.f, 1.f + __expf(-v[j]));
      }
      uint4 u;
      __nv_bfloat162 t0 = __floats2bfloat162_rn(v[0], v[1]);
      __nv_bfloat162 t1 = __floats2bfloat162_rn(v[2], v[3]);
      __nv_bfloat162 t2 = __floats2bfloat162_rn(v[4], v[5]);
      __nv_bfloat162 t3 = __floats2bfloat162_rn(v[6], v[7]);
      u.x = *reinterpret_cast<uint32_t*>(&t0);
      u.y = *reinterpret_cast<uint32_t*>(&t1);
      u.z = *reinterpret_cast<uint32_t*>(&t2);
      u.w = *reinterpret_cast<uint32_t*>(&t3);
      buf[lane * 8 + (c ^ (lane & 7))] = u;
    }
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = it * 4 + (lane >> 3), ch = lane & 7;
      const uint4 u = buf[r * 8 + (ch ^ (r & 7))];
      if (m_base + r < M)
        *reinterpret_cast<uint4*>(dst + (long)(m_base + r) * Dq + col + half * 64 + ch * 8) = u;
    }
    __syncwarp();  // the next half overwrites the buffer
  }
}

// Tensor-core SWIGLU epilogue with bf16 output staged through shared memory
// (requires F % 32 == 0).  Lane i owns row m_base + i; all lanes work on the
// same 64 accumulator columns (32 w1 + 32 w3), i.e. the same 32 outputs.  The
// warp's 32 x 32 bf16 block goes to a 2 KB buffer (16-byte chunks swizzled by
// row pair so each 8-lane phase hits distinct banks) and is written back as
// 64-byte row segments, eight rows per instruction.  Rows at or past M are
// computed but not stored.
template <class Acc>
__device__ __forceinline__ void epi_swiglu_staged(const EpiParams& p, int m_base, int lane, int M, int n0,
                                                  const Acc& acc, uint4* buf) {
  constexpr int G = SWIGLU_GROUP;
  static_assert(G == 32, "staged SWIGLU epilogue assumes 32-column groups");
  const int f0 = (n0 / (2 * G)) * G;
  bf16* dst = reinterpret_cast<bf16*>(p.h);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float a = acc(k * 8 + j);
      v[j] = __fdividef(a, 1.f + __expf(-a)) * acc(G + k * 8 + j);
    }
    uint4 u;
    __nv_bfloat162 t0 = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 t1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 t2 = __floats2bfloat162_rn(v[4], v[5]);
    __nv_bfloat162 t3 = __floats2bfloat162_rn(v[6], v[7]);
    u.x = *reinterpret_cast<uint32_t*>(&t0);
    u.y = *reinterpret_cast<uint32_t*>(&t1);
    u.z = *reinterpret_cast<uint32_t*>(&t2);
    u.w = *reinterpret_cast<uint32_t*>(&t3);
    buf[lane * 4 + (k ^ ((lane >> 1) & 3))] = u;
  }
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2), k = lane & 3;
    const uint4 u = buf[r * 4 + (k ^ ((r >> 1) & 3))];
    if (m_base + r < M) *reinterpret_cast<uint4*>(dst + (long)(m_base + r) * p.F + f0 + k * 8) = u;
  }
  __syncwarp();  // the buffer is reused by the warp's next chunk
}

}  // namespace irt
