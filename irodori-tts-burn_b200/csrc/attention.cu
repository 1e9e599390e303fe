// Joint attention over the keys of one sequence: its own (latent / token)
// keys followed by its context keys (compacted valid text + speaker rows of
// the per-request KV cache).  Softmax scale 1/sqrt(hd); masked keys are
// skipped; a sequence with no valid key yields 0 (safe softmax,
// src/model/attention.rs:675-724).  The output is multiplied by the
// precomputed sigmoid gate (src/model/attention.rs:422-424).
//
// attn_mma_kernel: bf16 operands, f32 online softmax, mma.sync m16n8k16,
//   64 queries x 1 head per CTA (4 warps x 16 rows), 64-key tiles double-
//   buffered with cp.async, XOR-swizzled shared memory, hd = 128.
// attn_simt_tiled_kernel: f32 storage, hd = 128, 64 queries x 1 head per CTA,
//   register-tiled scores and output (the f32 parity mode's attention).
// attn_simt_kernel: any even hd, f32 or bf16 storage, one warp per (query, head).
#include "common.hpp"
#include "kernels.hpp"

namespace irt {

namespace {

constexpr float LOG2E = 1.4426950408889634f;

template <class T>
__device__ __forceinline__ float ldf(const T* p, long i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, long i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<bf16>(const bf16* p, long i) { return __bfloat162float(p[i]); }

template <class T>
__device__ __forceinline__ void stf(T* p, long i, float v);
template <>
__device__ __forceinline__ void stf<float>(float* p, long i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void stf<bf16>(bf16* p, long i, float v) { p[i] = __float2bfloat16_rn(v); }

// ---------------------------------------------------------------------------
// SIMT kernel
// ---------------------------------------------------------------------------
template <class T>
__global__ void attn_simt_kernel(AttnParams p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qi = blockIdx.x * (blockDim.x / 32) + warp;
  const int h = blockIdx.y;
  const SeqDesc sd = p.seqs[blockIdx.z];
  if (qi >= sd.len) return;
  const int D = p.H * p.hd;
  const T* q = reinterpret_cast<const T*>(p.q);
  const T* k = reinterpret_cast<const T*>(p.k);
  const T* v = reinterpret_cast<const T*>(p.v);
  const T* ck = reinterpret_cast<const T*>(p.ck);
  const T* cv = reinterpret_cast<const T*>(p.cv);
  constexpr int MAXD = 8;  // hd <= 256
  float qv[MAXD], acc[MAXD];
  const long qrow = (long)(sd.tok_start + qi) * D + h * p.hd;
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    int d = lane + 32 * i;
    qv[i] = d < p.hd ? ldf(q, qrow + d) : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int nk = sd.len + sd.ctx_len;
  for (int j = 0; j < nk; ++j) {
    const T* kp;
    const T* vp;
    long row;
    if (j < sd.len) {
      if (p.key_mask && !p.key_mask[sd.tok_start + j]) continue;
      kp = k; vp = v; row = (long)(sd.tok_start + j) * D + h * p.hd;
    } else {
      kp = ck; vp = cv; row = (long)(sd.ctx_off + j - sd.len) * D + h * p.hd;
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      int d = lane + 32 * i;
      if (d < p.hd) s = fmaf(qv[i], ldf(kp, row + d), s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= p.scale;
    float mn = fmaxf(m, s);
    float corr = expf(m - mn);
    float e = expf(s - mn);
    l = l * corr + e;
#pragma unroll
    for (int i = 0; i < MAXD; ++i) {
      int d = lane + 32 * i;
      float vv = d < p.hd ? ldf(vp, row + d) : 0.f;
      acc[i] = acc[i] * corr + e * vv;
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* out = reinterpret_cast<T*>(p.out);
  const T* g = reinterpret_cast<const T*>(p.gsig);
#pragma unroll
  for (int i = 0; i < MAXD; ++i) {
    int d = lane + 32 * i;
    if (d < p.hd) {
      float o = acc[i] * inv;
      if (g) o *= ldf(g, qrow + d);
      stf(out, qrow + d, o);
    }
  }
}

// ---------------------------------------------------------------------------
// mma.sync kernel (bf16, hd = 128)
// ---------------------------------------------------------------------------
constexpr int QT = 64, KT = 64, HD = 128, ROWB = HD * 2;  // 256 bytes per row

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset in a [rows][128] bf16 tile
  return (uint32_t)(row * ROWB + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Register-tiled SIMT kernel (f32 storage, hd = 128)
//
// One CTA = 64 queries x 1 head, 256 threads, 64-key tiles.  Thread (r, c) with
// r = warp * 2 + lane / 16 and c = lane % 16 owns query rows r + 16 i (i < 4):
// the scores of keys c + 16 j (j < 4) and the output columns 4c..4c+3 and
// 64+4c..64+4c+3.  A row's 64 scores of a tile live in one half-warp, so the
// tile's row maximum and the online-softmax correction come from shuffles and
// stay in the registers of the threads that rescale that row's output.
// Shared memory: Q, K as [row][128] with 16-byte chunks XOR-swizzled by row
// (conflict-free column reads across rows), V plain, the probabilities
// transposed [key][4 rows of a thread] with chunks swizzled by key.  K of tile
// t+1 loads (cp.async) during tile t's softmax and P.V, V of tile t+1 during
// tile t+1's scores.  Invalid keys (past the sequence, masked) are zero-filled
// in K and V and scored -inf.  Two CTAs fit per SM.
// ---------------------------------------------------------------------------
constexpr int FQ = 64, FK = 64, FHD = 128;
constexpr int F_SMEM = (FQ * FHD + 2 * FK * FHD + FK * FQ) * 4 + FK * 4;

__global__ void __launch_bounds__(256, 2) attn_simt_tiled_kernel(AttnParams p) {
  extern __shared__ __align__(16) float fsm[];
  float* sq = fsm;                  // [64][128], chunk c of row r at c ^ (r & 7)
  float* sk = sq + FQ * FHD;        // [64][128], same swizzle
  float* sv = sk + FK * FHD;        // [64][128]
  float* sp = sv + FK * FHD;        // [64 keys][16 chunks of 4 rows], chunk r at r ^ (key & 15)
  float* kbias = sp + FK * FQ;      // [64] 0 (valid key) or -inf
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int r = warp * 2 + lane / 16, c = lane % 16;
  const int h = blockIdx.y;
  const SeqDesc sd = p.seqs[blockIdx.z];
  const int q0 = blockIdx.x * FQ;
  if (q0 >= sd.len) return;
  const int D = p.H * FHD;
  const float* Q = reinterpret_cast<const float*>(p.q);
  const float* K = reinterpret_cast<const float*>(p.k);
  const float* V = reinterpret_cast<const float*>(p.v);
  const float* CK = reinterpret_cast<const float*>(p.ck);
  const float* CV = reinterpret_cast<const float*>(p.cv);
  const int nk = sd.len + sd.ctx_len;
  const int ntiles = (nk + FK - 1) / FK;
  const uint32_t sq_u = (uint32_t)__cvta_generic_to_shared(sq);
  const uint32_t sk_u = (uint32_t)__cvta_generic_to_shared(sk);
  const uint32_t sv_u = (uint32_t)__cvta_generic_to_shared(sv);

  // Tile loaders: 64 rows x 32 chunks = 8 chunks per thread, coalesced rows.
  auto key_row = [&](int j, bool& ctx, long& row, bool& valid) {
    ctx = j >= sd.len;
    if (!ctx) {
      row = (long)(sd.tok_start + j);
      valid = !p.key_mask || p.key_mask[row];
    } else {
      row = (long)(sd.ctx_off + j - sd.len);
      valid = j < nk;
    }
  };
  auto load_keys = [&](int t, bool values) {
    const uint32_t dst_u = values ? sv_u : sk_u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int id = tid + 256 * i, rr = id / 32, ch = id % 32;
      bool ctx, valid;
      long row;
      key_row(t * FK + rr, ctx, row, valid);
      const float* src = values ? V : K;  // zero-fill when invalid: not read
      if (valid) src = (ctx ? (values ? CV : CK) : src) + row * D + h * FHD + ch * 4;
      const int dch = values ? ch : (ch ^ (rr & 7));
      cp_async16(dst_u + (uint32_t)(rr * FHD + dch * 4) * 4, src, valid);
      if (!values && ch == 0) kbias[rr] = valid ? 0.f : -INFINITY;
    }
  };

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int id = tid + 256 * i, rr = id / 32, ch = id % 32;
    const bool valid = q0 + rr < sd.len;
    const float* src = valid ? Q + (long)(sd.tok_start + q0 + rr) * D + h * FHD + ch * 4 : Q;
    cp_async16(sq_u + (uint32_t)(rr * FHD + (ch ^ (rr & 7)) * 4) * 4, src, valid);
  }
  load_keys(0, false);
  cp_commit();
  load_keys(0, true);
  cp_commit();

  float acc[4][8];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[i][d] = 0.f;
  }

  for (int t = 0; t < ntiles; ++t) {
    cp_wait<1>();  // Q and K of this tile
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    const float4* q4 = reinterpret_cast<const float4*>(sq);
    const float4* k4 = reinterpret_cast<const float4*>(sk);
#pragma unroll 4
    for (int ch = 0; ch < 32; ++ch) {
      float4 qa[4], kb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[i] = q4[(r + 16 * i) * 32 + (ch ^ (r & 7))];
#pragma unroll
      for (int j = 0; j < 4; ++j) kb[j] = k4[(c + 16 * j) * 32 + (ch ^ (c & 7))];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qa[i].x, kb[j].x, s[i][j]);
          s[i][j] = fmaf(qa[i].y, kb[j].y, s[i][j]);
          s[i][j] = fmaf(qa[i].z, kb[j].z, s[i][j]);
          s[i][j] = fmaf(qa[i].w, kb[j].w, s[i][j]);
        }
    }
    float bias[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) bias[j] = kbias[c + 16 * j];
    __syncthreads();  // every thread is done with K (and the bias) of this tile
    if (t + 1 < ntiles) load_keys(t + 1, false);
    cp_commit();

    // online softmax, one row per (i, half-warp)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = s[i][j] * p.scale + bias[j];
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m[i], mx);
      float corr = 1.f, sum = 0.f;
      if (mn != -INFINITY) {
        corr = expf(m[i] - mn);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = expf(s[i][j] - mn);
          sum += s[i][j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
      }
      m[i] = mn;
      l[i] = l[i] * corr + sum;
#pragma unroll
      for (int d = 0; d < 8; ++d) acc[i][d] *= corr;
    }
    float4* p4 = reinterpret_cast<float4*>(sp);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = c + 16 * j;
      p4[key * 16 + (r ^ (key & 15))] = make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
    }
    if (t + 1 < ntiles) cp_wait<1>();  // V of this tile (K of the next may still fly)
    else cp_wait<0>();
    __syncthreads();
    const float4* v4 = reinterpret_cast<const float4*>(sv);
#pragma unroll 4
    for (int key = 0; key < FK; ++key) {
      const float4 pr = p4[key * 16 + (r ^ (key & 15))];
      const float4 va = v4[key * 32 + c], vb = v4[key * 32 + 16 + c];
      const float pv[4] = {pr.x, pr.y, pr.z, pr.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[i][0] = fmaf(pv[i], va.x, acc[i][0]);
        acc[i][1] = fmaf(pv[i], va.y, acc[i][1]);
        acc[i][2] = fmaf(pv[i], va.z, acc[i][2]);
        acc[i][3] = fmaf(pv[i], va.w, acc[i][3]);
        acc[i][4] = fmaf(pv[i], vb.x, acc[i][4]);
        acc[i][5] = fmaf(pv[i], vb.y, acc[i][5]);
        acc[i][6] = fmaf(pv[i], vb.z, acc[i][6]);
        acc[i][7] = fmaf(pv[i], vb.w, acc[i][7]);
      }
    }
    __syncthreads();  // every thread is done with V and P of this tile
    if (t + 1 < ntiles) load_keys(t + 1, true);
    cp_commit();
  }
  cp_wait<0>();

  float* out = reinterpret_cast<float*>(p.out);
  const float* G = reinterpret_cast<const float*>(p.gsig);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float lt = l[i];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o);
    const int qi = q0 + r + 16 * i;
    if (qi >= sd.len) continue;
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const long off = (long)(sd.tok_start + qi) * D + h * FHD;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int d = half * 64 + 4 * c;
      float4 o = make_float4(acc[i][4 * half] * inv, acc[i][4 * half + 1] * inv, acc[i][4 * half + 2] * inv,
                             acc[i][4 * half + 3] * inv);
      if (G) {
        const float4 g = *reinterpret_cast<const float4*>(G + off + d);
        o.x *= g.x; o.y *= g.y; o.z *= g.z; o.w *= g.w;
      }
      *reinterpret_cast<float4*>(out + off + d) = o;
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}

__global__ void __launch_bounds__(128) attn_mma_kernel(AttnParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  const SeqDesc sd = p.seqs[blockIdx.z];
  const int q0 = blockIdx.x * QT;
  if (q0 >= sd.len) return;
  const int h = blockIdx.y;
  const int D = p.H * HD;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const uint32_t sQ = (uint32_t)__cvta_generic_to_shared(sm);
  const uint32_t sK = sQ + QT * ROWB;
  const uint32_t sV = sK + 2 * KT * ROWB;
  const bf16* Q = reinterpret_cast<const bf16*>(p.q);
  const bf16* K = reinterpret_cast<const bf16*>(p.k);
  const bf16* V = reinterpret_cast<const bf16*>(p.v);
  const bf16* CK = reinterpret_cast<const bf16*>(p.ck);
  const bf16* CV = reinterpret_cast<const bf16*>(p.cv);
  const int nk = sd.len + sd.ctx_len;
  const int ntiles = (nk + KT - 1) / KT;

  // Q tile
#pragma unroll
  for (int i = 0; i < (QT * 16) / 128; ++i) {
    int c = tid + i * 128;
    int r = c >> 4, ch = c & 15;
    int qi = q0 + r;
    bool ok = qi < sd.len;
    const bf16* src = Q + (long)(sd.tok_start + (ok ? qi : 0)) * D + h * HD + ch * 8;
    cp_async16(sQ + swz(r, ch), src, ok);
  }
  auto load_kv = [&](int tile, int buf) {
#pragma unroll
    for (int i = 0; i < (KT * 16) / 128; ++i) {
      int c = tid + i * 128;
      int r = c >> 4, ch = c & 15;
      int key = tile * KT + r;
      const bf16 *ks, *vs;
      // masked / out-of-range keys are zero-filled so their V rows can never
      // leak NaN or Inf into the P.V product (their scores are -inf below)
      bool ok = key < nk && !(key < sd.len && p.key_mask && !p.key_mask[sd.tok_start + key]);
      if (ok && key < sd.len) {
        long off = (long)(sd.tok_start + key) * D + h * HD + ch * 8;
        ks = K + off; vs = V + off;
      } else if (ok) {
        long off = (long)(sd.ctx_off + key - sd.len) * D + h * HD + ch * 8;
        ks = CK + off; vs = CV + off;
      } else {
        ks = K; vs = V;
      }
      cp_async16(sK + buf * KT * ROWB + swz(r, ch), ks, ok);
      cp_async16(sV + buf * KT * ROWB + swz(r, ch), vs, ok);
    }
  };
  if (ntiles > 0) load_kv(0, 0);
  cp_commit();

  uint32_t qf[8][4];
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, lr = lane & 7;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < ntiles) load_kv(tile + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (tile == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        int r = warp * 16 + (mi & 1) * 8 + lr;
        int ch = 2 * kk + (mi >> 1);
        ldsm_x4(sQ + swz(r, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T for 64 keys
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const uint32_t kb = sK + buf * KT * ROWB;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        int r = 16 * jj + (mi >> 1) * 8 + lr;
        int ch = 2 * kk + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz(r, ch), b0, b1, b2, b3);
        mma16816(s[2 * jj], qf[kk], b0, b1);
        mma16816(s[2 * jj + 1], qf[kk], b2, b3);
      }
    }
    // mask + online softmax (rows g and g+8 of this warp)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int key = tile * KT + nt * 8 + 2 * t4 + (e & 1);
        bool valid = key < nk;
        if (valid && key < sd.len && p.key_mask) valid = p.key_mask[sd.tok_start + key] != 0;
        float v = valid ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float corr[2], base[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      float mn = fmaxf(mrow[r], mx[r]);
      base[r] = mn == -INFINITY ? 0.f : mn;
      corr[r] = exp2f(mrow[r] - base[r]);
      mrow[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float pv = exp2f(s[nt][e] - base[e >> 1]);
        s[nt][e] = pv;
        rs[e >> 1] += pv;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * corr[r] + rs[r];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= corr[0]; o[dt][1] *= corr[0];
      o[dt][2] *= corr[1]; o[dt][3] *= corr[1];
    }
    // O += P V
    const uint32_t vb = sV + buf * KT * ROWB;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dd = 0; dd < 8; ++dd) {
        int r = 16 * kk + (mi & 1) * 8 + lr;
        int ch = 2 * dd + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz(r, ch), b0, b1, b2, b3);
        mma16816(o[2 * dd], a, b0, b1);
        mma16816(o[2 * dd + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();

  // finalize: full row sums across the quad
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  bf16* out = reinterpret_cast<bf16*>(p.out);
  const bf16* G = reinterpret_cast<const bf16*>(p.gsig);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int qi = q0 + warp * 16 + g + r * 8;
    if (qi >= sd.len) continue;
    float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    long rowoff = (long)(sd.tok_start + qi) * D + h * HD;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      int d = dt * 8 + 2 * t4;
      float v0 = o[dt][2 * r] * inv, v1 = o[dt][2 * r + 1] * inv;
      if (G) {
        __nv_bfloat162 gg = *reinterpret_cast<const __nv_bfloat162*>(G + rowoff + d);
        v0 *= __bfloat162float(gg.x);
        v1 *= __bfloat162float(gg.y);
      }
      *reinterpret_cast<__nv_bfloat162*>(out + rowoff + d) = __floats2bfloat162_rn(v0, v1);
    }
  }
}

}  // namespace

void attention(const AttnParams& p, int bf16_io, cudaStream_t s) {
  if (p.nseq <= 0 || p.max_len <= 0) return;
  if (bf16_io && p.path == 0 && attention_tc_supported(p)) {
    attention_tc(p, s);
    return;
  }
  if (bf16_io && p.hd == HD && p.path != 2) {
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    const int smem = (QT + 4 * KT) * ROWB;
    if (attr_dev != dev) {
      IRT_CUDA(cudaFuncSetAttribute(attn_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr_dev = dev;
    }
    dim3 grid((p.max_len + QT - 1) / QT, p.H, p.nseq);
    attn_mma_kernel<<<grid, 128, smem, s>>>(p);
  } else if (!bf16_io && p.hd == FHD && p.path != 3) {
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
      IRT_CUDA(cudaFuncSetAttribute(attn_simt_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, F_SMEM));
      attr_dev = dev;
    }
    dim3 grid((p.max_len + FQ - 1) / FQ, p.H, p.nseq);
    attn_simt_tiled_kernel<<<grid, 256, F_SMEM, s>>>(p);
  } else {
    if (p.hd > 256) throw unsupported("attention head_dim > 256");
    dim3 grid((p.max_len + 3) / 4, p.H, p.nseq);
    if (bf16_io) attn_simt_kernel<bf16><<<grid, 128, 0, s>>>(p);
    else attn_simt_kernel<float><<<grid, 128, 0, s>>>(p);
  }
  IRT_CHECK_LAUNCH();
}

}  // namespace irt
