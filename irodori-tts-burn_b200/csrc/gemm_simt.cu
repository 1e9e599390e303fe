// fp32 SIMT GEMM (parity path and fallback for shapes the tensor-core kernel
// does not take) and the standalone epilogue kernel.
#include "common.hpp"
#include "epilogue.cuh"

namespace irt {

namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <bool ABF, bool BBF>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const void* __restrict__ A, long lda, long a_bs,
                                                        const void* __restrict__ B, long ldb, long b_bs,
                                                        float* __restrict__ C, long ldc, long c_bs, int M, int N,
                                                        int K) {
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int z = blockIdx.z;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;  // 16x16 threads, 4x4 outputs each
  float acc[4][4] = {};
  auto ldA = [&](long r, long c) -> float {
    if (ABF) return __bfloat162float(reinterpret_cast<const bf16*>(A)[z * a_bs + r * lda + c]);
    return reinterpret_cast<const float*>(A)[z * a_bs + r * lda + c];
  };
  auto ldB = [&](long r, long c) -> float {
    if (BBF) return __bfloat162float(reinterpret_cast<const bf16*>(B)[z * b_bs + r * ldb + c]);
    return reinterpret_cast<const float*>(B)[z * b_bs + r * ldb + c];
  };
  for (int k0 = 0; k0 < K; k0 += TK) {
    // 64x16 tile of A and B: 1024 elements each, 4 per thread
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = tid + i * 256;
      int r = e / TK, c = e % TK;
      int gr = m0 + r, gc = k0 + c;
      As[c][r] = (gr < M && gc < K) ? ldA(gr, gc) : 0.f;
      int gn = n0 + r;
      Bs[c][r] = (gn < N && gc < K) ? ldB(gn, gc) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int r = m0 + ty * 4 + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = n0 + tx * 4 + j;
      if (c < N) C[z * c_bs + (long)r * ldc + c] = acc[i][j];
    }
  }
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

void gemm_simt(const void* A, int a_bf16, long lda, long a_bstride, const void* B, int b_bf16, long ldb,
               long b_bstride, float* raw, long ldr, long r_bstride, int M, int N, int K, int batch,
               cudaStream_t s) {
  if (M <= 0 || N <= 0 || batch <= 0) return;
  dim3 grid((N + TN - 1) / TN, (M + TM - 1) / TM, batch);
  if (a_bf16 && b_bf16)
    gemm_simt_kernel<true, true><<<grid, 256, 0, s>>>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K);
  else if (a_bf16)
    gemm_simt_kernel<true, false><<<grid, 256, 0, s>>>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K);
  else if (b_bf16)
    gemm_simt_kernel<false, true><<<grid, 256, 0, s>>>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K);
  else
    gemm_simt_kernel<false, false><<<grid, 256, 0, s>>>(A, lda, a_bstride, B, ldb, b_bstride, raw, ldr, r_bstride, M, N, K);
  IRT_CHECK_LAUNCH();
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
