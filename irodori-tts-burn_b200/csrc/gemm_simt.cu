// fp32 SIMT GEMM (parity path and fallback for shapes the tensor-core kernel
// does not take: the f32 cond_module and adaLN tables, K < 64 or K % 8 != 0)
// and the standalone epilogue kernel.
#include <cooperative_groups.h>

#include "common.hpp"
#include "epilogue.cuh"

namespace irt {

namespace {

namespace cg = cooperative_groups;

// 64 x 64 output tile per CTA, 256 threads with 4 x 4 outputs each, k-tiles
// of 32 double-buffered in shared memory: the next k-tile's global loads are
// in flight (in registers) while the current one is multiplied.
//
// Short-M shapes (the adaLN and cond_module GEMMs have one row per timestep,
// 5-65 rows, against N of 2,048-12,288 and K of 256-2,048) give too few tiles
// to fill the SMs, so K is split over a cluster of S CTAs (grid z = batch x S,
// cluster 1 x 1 x S).  Each CTA multiplies its contiguous range of k-tiles,
// leaves its 64 x 64 partial tile in shared memory, and after a cluster
// barrier every CTA sums rows [r * 64 / S, (r + 1) * 64 / S) of the S tiles
// through distributed shared memory, always in rank order 0..S-1, and stores
// them.  The sum is therefore deterministic and needs no workspace and no
// atomics.
constexpr int TM = 64, TN = 64, TK = 32, PAD = 4, THREADS = 256;
constexpr int MAX_SPLIT = 8;

struct Smem {
  union {
    struct {
      float a[2][TK][TM + PAD];  // A^T tiles (k-major), double-buffered
      float b[2][TK][TN + PAD];
    } ab;
    float c[TM][TN];  // partial output tile for the cluster reduction
  };
};

template <bool BF>
__device__ __forceinline__ float ld_elem(const void* p, long i) {
  if constexpr (BF) return __bfloat162float(reinterpret_cast<const bf16*>(p)[i]);
  else return reinterpret_cast<const float*>(p)[i];
}

// VEC: f32 operands with 16-byte aligned rows (base, leading dimensions,
// batch strides and K all multiples of 4 floats): each thread moves two float4
// of A and two of B per k-tile.  Otherwise eight scalar loads of each.
template <bool ABF, bool BBF, bool VEC>
struct Stage {
  static constexpr int NA = VEC ? 2 : 8;
  float4 va[VEC ? 2 : 1], vb[VEC ? 2 : 1];
  float sa[VEC ? 1 : 8], sb[VEC ? 1 : 8];

  __device__ __forceinline__ void load(const void* A, long lda, const void* B, long ldb, int M, int N, int kend,
                                       int m0, int n0, int k0, int tid) {
    if constexpr (VEC) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = tid + i * THREADS;  // 512 float4 per 64 x 32 tile
        const int r = e >> 3, c = (e & 7) * 4;
        const int gk = k0 + c;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        va[i] = (m0 + r < M && gk < kend)
                    ? __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(A) + (long)(m0 + r) * lda + gk))
                    : z;
        vb[i] = (n0 + r < N && gk < kend)
                    ? __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(B) + (long)(n0 + r) * ldb + gk))
                    : z;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = tid + i * THREADS;  // 2048 elements per 64 x 32 tile
        const int r = e >> 5, c = e & 31;
        const int gk = k0 + c;
        sa[i] = (m0 + r < M && gk < kend) ? ld_elem<ABF>(A, (long)(m0 + r) * lda + gk) : 0.f;
        sb[i] = (n0 + r < N && gk < kend) ? ld_elem<BBF>(B, (long)(n0 + r) * ldb + gk) : 0.f;
      }
    }
  }

  __device__ __forceinline__ void store(Smem& sm, int buf, int tid) const {
    if constexpr (VEC) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = tid + i * THREADS;
        const int r = e >> 3, c = (e & 7) * 4;
        sm.ab.a[buf][c][r] = va[i].x;
        sm.ab.a[buf][c + 1][r] = va[i].y;
        sm.ab.a[buf][c + 2][r] = va[i].z;
        sm.ab.a[buf][c + 3][r] = va[i].w;
        sm.ab.b[buf][c][r] = vb[i].x;
        sm.ab.b[buf][c + 1][r] = vb[i].y;
        sm.ab.b[buf][c + 2][r] = vb[i].z;
        sm.ab.b[buf][c + 3][r] = vb[i].w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = tid + i * THREADS;
        const int r = e >> 5, c = e & 31;
        sm.ab.a[buf][c][r] = sa[i];
        sm.ab.b[buf][c][r] = sb[i];
      }
    }
  }
};

template <bool ABF, bool BBF, bool VEC>
__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(const void* __restrict__ A, long lda, long a_bs,
                                                            const void* __restrict__ B, long ldb, long b_bs,
                                                            float* __restrict__ C, long ldc, long c_bs, int M, int N,
                                                            int K, int splits, int ktiles_per_split) {
  __shared__ __align__(16) Smem sm;
  const int split = blockIdx.z % splits;  // == cluster rank (cluster 1 x 1 x splits)
  const int z = blockIdx.z / splits;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int kbeg = split * ktiles_per_split * TK;
  const int kend = min(K, kbeg + ktiles_per_split * TK);
  const int nk = kend > kbeg ? (kend - kbeg + TK - 1) / TK : 0;
  const void* Az = ABF ? (const void*)(reinterpret_cast<const bf16*>(A) + z * a_bs)
                       : (const void*)(reinterpret_cast<const float*>(A) + z * a_bs);
  const void* Bz = BBF ? (const void*)(reinterpret_cast<const bf16*>(B) + z * b_bs)
                       : (const void*)(reinterpret_cast<const float*>(B) + z * b_bs);

  float acc[4][4] = {};
  Stage<ABF, BBF, VEC> st;
  if (nk > 0) {
    st.load(Az, lda, Bz, ldb, M, N, kend, m0, n0, kbeg, tid);
    st.store(sm, 0, tid);
  }
  __syncthreads();
  for (int t = 0; t < nk; ++t) {
    const int buf = t & 1;
    if (t + 1 < nk) st.load(Az, lda, Bz, ldb, M, N, kend, m0, n0, kbeg + (t + 1) * TK, tid);
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&sm.ab.a[buf][kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&sm.ab.b[buf][kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (t + 1 < nk) st.store(sm, buf ^ 1, tid);
    __syncthreads();
  }

  float* Cz = C + z * c_bs;
  if (splits == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = m0 + ty * 4 + i;
      if (r >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = n0 + tx * 4 + j;
        if (c < N) Cz[(long)r * ldc + c] = acc[i][j];
      }
    }
    return;
  }
  // K split over the cluster: partial tiles meet in distributed shared memory
  // (the k-tile buffers are free: the loop ended on a barrier).
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(&sm.c[ty * 4 + i][tx * 4]) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int r_lo = split * TM / splits, r_hi = (split + 1) * TM / splits;
  for (int e = tid; e < (r_hi - r_lo) * TN; e += THREADS) {
    const int rr = r_lo + e / TN, cc = e % TN;
    float v = 0.f;
    for (int s = 0; s < splits; ++s) {
      const Smem* peer = cluster.map_shared_rank(&sm, s);
      v += peer->c[rr][cc];
    }
    const int r = m0 + rr, c = n0 + cc;
    if (r < M && c < N) Cz[(long)r * ldc + c] = v;
  }
  // no CTA leaves while a peer may still read its tile
  cluster.sync();
}

struct RawAcc {
  const float* r;
  __device__ float operator()(int j) const { return r[j]; }
};

// One thread per (row, chunk).  Chunk widths: 32 (STORE/RESID), 64 (SWIGLU
// pair), hd (QKVG/CTXKV).
__global__ void epilogue_kernel(EpiParams p, const float* __restrict__ raw, long ldr, long r_bs, int chunk,
                                int nchunks) {
  long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  int z = blockIdx.y;
  if (t >= (long)p.M * nchunks) return;
  int m = (int)(t / nchunks);
  int c = (int)(t % nchunks);
  int n0 = c * chunk;
  RawAcc acc{raw + z * r_bs + (long)m * ldr + n0};
  switch (p.mode) {
    case EPI_STORE:
      epi_chunk_store<32>(p, m, n0, acc, z * p.out_bstride, z * p.bias_bstride, z * p.add_bstride);
      break;
    case EPI_RESID:
      epi_chunk_resid<32>(p, m, n0, acc);
      break;
    case EPI_SWIGLU:
      epi_chunk_swiglu(p, m, n0, acc);
      break;
    default:
      epi_head<0>(p, m, n0, acc);
      break;
  }
}

}  // namespace

namespace {

int simt_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <bool ABF, bool BBF, bool VEC>
void launch_simt(const void* A, long lda, long a_bs, const void* B, long ldb, long b_bs, float* C, long ldc,
                 long c_bs, int M, int N, int K, int batch, int splits, int kps, cudaStream_t s) {
  dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM, batch * splits);
  if (splits == 1) {
    gemm_simt_kernel<ABF, BBF, VEC><<<grid, THREADS, 0, s>>>(A, lda, a_bs, B, ldb, b_bs, C, ldc, c_bs, M, N, K, 1, kps);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned)splits;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    IRT_CUDA(cudaLaunchKernelEx(&cfg, gemm_simt_kernel<ABF, BBF, VEC>, A, lda, a_bs, B, ldb, b_bs, C, ldc, c_bs, M,
                                N, K, splits, kps));
  }
  IRT_CHECK_LAUNCH();
}

}  // namespace

void gemm_simt(const void* A, int a_bf16, long lda, long a_bstride, const void* B, int b_bf16, long ldb,
               long b_bstride, float* raw, long ldr, long r_bstride, int M, int N, int K, int batch,
               cudaStream_t s) {
  if (M <= 0 || N <= 0 || batch <= 0) return;
  const long tiles = (long)((N + TN - 1) / TN) * ((M + TM - 1) / TM) * batch;
  const int kt = K > 0 ? (K + TK - 1) / TK : 1;
  // Split K over a cluster when the tiles cover fewer than three CTAs per SM,
  // keeping at least two k-tiles per split and no empty split.
  int splits = 1;
  const long want = 3L * simt_sms();
  if (tiles < want && batch * (long)MAX_SPLIT <= 65535) {
    splits = (int)std::min<long>(MAX_SPLIT, (want + tiles - 1) / tiles);
    splits = std::max(1, std::min(splits, kt / 2));
  }
  const int kps = (kt + splits - 1) / splits;
  splits = (kt + kps - 1) / kps;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = !a_bf16 && !b_bf16 && al16(A) && al16(B) && (lda % 4) == 0 && (ldb % 4) == 0 &&
                   (a_bstride % 4) == 0 && (b_bstride % 4) == 0 && (K % 4) == 0;
  if (vec)
    launch_simt<false, false, true>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K, batch, splits,
                                    kps, s);
  else if (a_bf16 && b_bf16)
    launch_simt<true, true, false>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K, batch, splits,
                                   kps, s);
  else if (a_bf16)
    launch_simt<true, false, false>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K, batch, splits,
                                    kps, s);
  else if (b_bf16)
    launch_simt<false, true, false>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K, batch, splits,
                                    kps, s);
  else
    launch_simt<false, false, false>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K, batch,
                                     splits, kps, s);
}

void epilogue_apply(const EpiParams& p, const float* raw, long ldr, long r_bstride, int batch, cudaStream_t s) {
  if (p.M <= 0 || p.N <= 0) return;
  int chunk = 32;
  if (p.mode == EPI_SWIGLU) chunk = 2 * SWIGLU_GROUP;
  if (p.mode == EPI_QKVG || p.mode == EPI_CTXKV) chunk = p.hd;
  int nchunks = (p.N + chunk - 1) / chunk;
  long total = (long)p.M * nchunks;
  dim3 grid((unsigned)((total + 127) / 128), batch);
  epilogue_kernel<<<grid, 128, 0, s>>>(p, raw, ldr, r_bstride, chunk, nchunks);
  IRT_CHECK_LAUNCH();
}

}  // namespace irt
