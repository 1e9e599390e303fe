// tcgen05 / TMEM flash attention for sm_100a (hd = 128, bf16 operands).
//
// One CTA = one (sequence, head, 128-query tile).  320 threads:
//   warp 0      TMA producer: Q once; per 128-key tile a K tile and a V tile,
//               each on its own 2-stage ring (self keys first, then context)
//   warp 1      TMEM allocator + single-thread MMA issuer:
//                 S_j  = Q K_j^T       (M=128 queries, N=128 keys, K=128 hd) -> TMEM S[j&1]
//                 O_b += P_j V_j, b = j&1  (M=128, N=128 hd, K=128 keys; V MN-major)
//   warps 2..9  two softmax warpgroups; group b takes key tiles j = b, b+2, ...
//               with its own running max / sum and its own TMEM accumulator
//               O_b, so the two groups' exponentials run concurrently.  Thread
//               r of a group owns query row r.  Per tile it loads the S row
//               from TMEM (one batched wait), masks, takes the row max, writes
//               P = exp2(s - m) as bf16 (128B-swizzled, K-major) to shared
//               memory and keeps the row sum.  The running max is only raised
//               when a row max grows by more than 2^8 (conditional rescale);
//               then the warp rescales its O_b rows in TMEM after the previous
//               P.V into O_b has completed.  Skipping is exact: O_b and l_b
//               share the same stale max.  At the end the groups exchange
//               (m, l) through shared memory and each merges one 64-column
//               half: O = (O_0 2^(m_0-m) + O_1 2^(m_1-m)) / (l_0 2^(m_0-m) + l_1 2^(m_1-m)).
// Keys past a sequence's end get -inf scores; a row with no valid key outputs
// 0.  Output = O * sigmoid-gate, bf16.
#include <algorithm>

#include "common.hpp"
#include "kernels.hpp"
#include "tc_common.cuh"

namespace irt {

const CUtensorMap& tma_map_bf16(const void* p, long rows, long cols, long ld, int box_rows);

namespace {

using namespace tcx;

constexpr int QT = 128, KT = 128, HDIM = 128, THREADS = 320;
constexpr uint32_t TILE_BYTES = QT * HDIM * 2;  // 32 KB (two 16 KB 64-column halves)
constexpr uint32_t HALF = TILE_BYTES / 2;
// smem: Q | K0 K1 | V0 V1 | P0 P1 | barriers
constexpr uint32_t OFF_Q = 0, OFF_K = TILE_BYTES, OFF_V = OFF_K + 2 * TILE_BYTES, OFF_P = OFF_V + 2 * TILE_BYTES;
constexpr uint32_t OFF_BAR = OFF_P + 2 * TILE_BYTES;
constexpr size_t SMEM = OFF_BAR + 256 + 1024;
// (m, l) exchange of the final merge, [2 groups][m, l][128 rows] f32, in the Q
// tile: once every group has seen its last P.V complete, every QK^T MMA
// (issued before those P.V, and tracked by their commits) has finished
// reading Q.
constexpr uint32_t OFF_XCHG = OFF_Q;
constexpr uint32_t IDESC_S = idesc_bf16(128, 128, false);
constexpr uint32_t IDESC_O = idesc_bf16(128, 128, true);
constexpr uint32_t TM_S = 0, TM_O = 256;  // TMEM columns: S double buffer, O_0 | O_1 accumulators
constexpr float RESCALE_LOG2 = 8.f;       // raise the running max only beyond 2^8 growth

struct TcAttnArgs {
  const SeqDesc* seqs;
  const bf16* gsig;
  bf16* out;
  int H;
  float scale_log2;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmCK,
                   const __grid_constant__ CUtensorMap tmCV, const __grid_constant__ TcAttnArgs a) {
  pdl_wait();  // before any read of predecessor output, in every CTA
  pdl_trigger();
  const SeqDesc sd = a.seqs[blockIdx.z];
  const int q0 = blockIdx.x * QT;
  if (q0 >= sd.len) return;
  const int h = blockIdx.y;
  const int D = a.H * HDIM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const uint32_t Q_FULL = bar(0);
  auto O_DONE = [&](int b) { return bar(18 + b); };
  auto K_FULL = [&](int s) { return bar(2 + s); };
  auto K_EMPTY = [&](int s) { return bar(4 + s); };
  auto V_FULL = [&](int s) { return bar(6 + s); };
  auto V_EMPTY = [&](int s) { return bar(8 + s); };
  auto S_FULL = [&](int b) { return bar(10 + b); };
  auto S_EMPTY = [&](int b) { return bar(12 + b); };
  auto P_FULL = [&](int b) { return bar(14 + b); };
  auto P_EMPTY = [&](int b) { return bar(16 + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_self = (sd.len + KT - 1) / KT;
  const int n_ctx = (sd.ctx_len + KT - 1) / KT;
  const int ntiles = n_self + n_ctx;

  if (threadIdx.x == 0) {
    mbar_init(Q_FULL, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(O_DONE(b), 1);
      mbar_init(K_FULL(b), 1);
      mbar_init(K_EMPTY(b), 1);
      mbar_init(V_FULL(b), 1);
      mbar_init(V_EMPTY(b), 1);
      mbar_init(S_FULL(b), 1);
      mbar_init(S_EMPTY(b), 4);
      mbar_init(P_FULL(b), 4);
      mbar_init(P_EMPTY(b), 1);
    }
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(sm + OFF_Q);
  auto sK = [&](int s) { return smem_u32(sm + OFF_K + s * TILE_BYTES); };
  auto sV = [&](int s) { return smem_u32(sm + OFF_V + s * TILE_BYTES); };
  auto sP = [&](int b) { return smem_u32(sm + OFF_P + b * TILE_BYTES); };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_map(&tmQ);
      prefetch_map(&tmK);
      prefetch_map(&tmV);
      mbar_expect_tx(Q_FULL, TILE_BYTES);
      tma_load_2d(sQ, &tmQ, Q_FULL, h * HDIM, sd.tok_start + q0);
      tma_load_2d(sQ + HALF, &tmQ, Q_FULL, h * HDIM + 64, sd.tok_start + q0);
      auto row_of = [&](int j) { return j < n_self ? sd.tok_start + j * KT : sd.ctx_off + (j - n_self) * KT; };
      auto load_k = [&](int j) {
        const int s = j & 1;
        mbar_wait(K_EMPTY(s), ((j >> 1) & 1) ^ 1);
        mbar_expect_tx(K_FULL(s), TILE_BYTES);
        const CUtensorMap* m = j < n_self ? &tmK : &tmCK;
        tma_load_2d(sK(s), m, K_FULL(s), h * HDIM, row_of(j));
        tma_load_2d(sK(s) + HALF, m, K_FULL(s), h * HDIM + 64, row_of(j));
      };
      auto load_v = [&](int j) {
        const int s = j & 1;
        mbar_wait(V_EMPTY(s), ((j >> 1) & 1) ^ 1);
        mbar_expect_tx(V_FULL(s), TILE_BYTES);
        const CUtensorMap* m = j < n_self ? &tmV : &tmCV;
        tma_load_2d(sV(s), m, V_FULL(s), h * HDIM, row_of(j));
        tma_load_2d(sV(s) + HALF, m, V_FULL(s), h * HDIM + 64, row_of(j));
      };
      // K runs two tiles ahead of V, matching the MMA issue order
      // S_0, S_1, then per j: S_{j+2}, P_j V_j
      if (ntiles > 0) load_k(0);
      if (ntiles > 1) load_k(1);
      for (int j = 0; j < ntiles; ++j) {
        load_v(j);
        if (j + 2 < ntiles) load_k(j + 2);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && ntiles > 0) {
      mbar_wait(Q_FULL, 0);
      auto issue_s = [&](int j) {
        const int s = j & 1;
        mbar_wait(K_FULL(s), (j >> 1) & 1);
        mbar_wait(S_EMPTY(s), ((j >> 1) & 1) ^ 1);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HDIM / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          umma_f16(tmem + TM_S + s * 128, sdesc_kmajor(sQ + off), sdesc_kmajor(sK(s) + off), IDESC_S, kk != 0);
        }
        umma_commit(S_FULL(s));
        umma_commit(K_EMPTY(s));
      };
      // S_{j+2} goes out before P_j.V_j: its S buffer is free as soon as the
      // group has loaded S_j into registers, so the next scores are computed
      // while the group is still busy with the softmax of tile j.
      issue_s(0);
      if (ntiles > 1) issue_s(1);
      for (int j = 0; j < ntiles; ++j) {
        if (j + 2 < ntiles) issue_s(j + 2);
        const int s = j & 1;
        mbar_wait(V_FULL(s), (j >> 1) & 1);
        mbar_wait(P_FULL(s), (j >> 1) & 1);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          // A = P (K-major over keys); B = V [keys][hd] (MN-major: 64-column
          // halves 16 KB apart, 8-key groups 1 KB apart)
          const uint32_t aoff = (kk >> 2) * HALF + (kk & 3) * 32;
          const uint64_t bdesc = sdesc_sw128(sV(s) + kk * 16 * 128, HALF, 1024);
          umma_f16(tmem + TM_O + s * 128, sdesc_kmajor(sP(s) + aoff), bdesc, IDESC_O, (j >= 2 || kk != 0));
        }
        umma_commit(P_EMPTY(s));
        umma_commit(V_EMPTY(s));
        umma_commit(O_DONE(s));  // one phase per tile of group s
      }
    }
  } else {
    // ---------------- softmax warps: two groups ----------------
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;   // group: key tiles j = grp, grp + 2, ...
    const int row = quad * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t o_col = TM_O + grp * 128;
    float m_run = -INFINITY, l_run = 0.f;
    int last = -1;
    for (int j = grp; j < ntiles; j += 2) {
      const int b = grp;  // == j & 1
      const bool self = j < n_self;
      const int kvalid = (self ? sd.len - j * KT : sd.ctx_len - (j - n_self) * KT);  // valid keys in tile
      mbar_wait(S_FULL(b), (j >> 1) & 1);
      tc_fence_after();
      uint32_t sr[KT];
#pragma unroll
      for (int c = 0; c < KT / 32; ++c)
        tmem_ld32(tmem + lane_off + TM_S + b * 128 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(S_EMPTY(b));  // S buffer may be overwritten now
      // Row max on the raw scores (the softmax scale is positive); keys past
      // the sequence end (only in a ragged last tile) become -inf.
      if (kvalid < KT) {
#pragma unroll
        for (int i = 0; i < KT; ++i)
          if (i >= kvalid) sr[i] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < KT; i += 4) {
        mx0 = fmaxf(mx0, __uint_as_float(sr[i]));
        mx1 = fmaxf(mx1, __uint_as_float(sr[i + 1]));
        mx2 = fmaxf(mx2, __uint_as_float(sr[i + 2]));
        mx3 = fmaxf(mx3, __uint_as_float(sr[i + 3]));
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * a.scale_log2;  // log2 domain
      // conditional rescale of the running max
      float corr = 1.f;
      bool raise = mx > m_run + RESCALE_LOG2 || (m_run == -INFINITY && mx > -INFINITY);
      if (raise) {
        corr = m_run == -INFINITY ? 0.f : ex2(m_run - mx);
        m_run = mx;
      }
      // p = 2^(s * scale - m): one FFMA feeds the exponential
      const float nbase = m_run == -INFINITY ? 0.f : -m_run;
      // P = exp2(s - m) -> bf16 swizzled tile; row sum in f32
      mbar_wait(P_EMPTY(b), ((j >> 1) & 1) ^ 1);
      float rsum = 0.f;
      uint8_t* prow = sm + OFF_P + b * TILE_BYTES + row * 128;
#pragma unroll
      for (int chunk = 0; chunk < KT / 8; ++chunk) {
        uint32_t pk[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int i = chunk * 8 + 2 * q;
          const float p0 = ex2(fmaf(__uint_as_float(sr[i]), a.scale_log2, nbase));
          const float p1 = ex2(fmaf(__uint_as_float(sr[i + 1]), a.scale_log2, nbase));
          rsum += p0 + p1;
          __nv_bfloat162 t = __floats2bfloat162_rn(p0, p1);
          pk[q] = *reinterpret_cast<uint32_t*>(&t);
        }
        const int sub = chunk >> 3, cin = chunk & 7;
        *reinterpret_cast<uint4*>(prow + sub * HALF + ((cin ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l_run = l_run * corr + rsum;
      // Rescale O_b (warp-collective) once the previous P.V into O_b is complete.
      if (__any_sync(0xffffffffu, raise) && j >= 2) {
        mbar_wait(O_DONE(b), ((j >> 1) - 1) & 1);
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HDIM / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + o_col + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(tmem + lane_off + o_col + c * 32, r);
        }
        tmem_wait_st();
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(P_FULL(b));
      last = j;
    }
    // prefetch this row's gate half (independent of the attention result)
    const int qi = q0 + row;
    const long off = (long)(sd.tok_start + (qi < sd.len ? qi : 0)) * D + h * HDIM;
    uint4 gpre[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      gpre[u] = (a.gsig && qi < sd.len) ? *reinterpret_cast<const uint4*>(a.gsig + off + grp * 64 + u * 8)
                                        : make_uint4(0, 0, 0, 0);
    // this group's last P.V into O_grp
    if (last >= 0) mbar_wait(O_DONE(grp), (last >> 1) & 1);
    tc_fence_after();

    // merge the two groups: exchange (m, l) per row, each group finishes one
    // 64-column half of hd from both accumulators.  The first barrier (the 8
    // softmax warps) orders the exchange writes into the Q tile after every
    // group's final wait: a group without tiles has waited for nothing.
    asm volatile("bar.sync 1, 256;" ::: "memory");
    float* xg = reinterpret_cast<float*>(sm + OFF_XCHG);
    xg[(grp * 2 + 0) * 128 + row] = last >= 0 ? m_run : -INFINITY;
    xg[(grp * 2 + 1) * 128 + row] = last >= 0 ? l_run : 0.f;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float m0 = xg[0 * 128 + row], l0 = xg[1 * 128 + row];
    const float m1 = xg[2 * 128 + row], l1 = xg[3 * 128 + row];
    const float mm = fmaxf(m0, m1);
    const float c0 = (mm == -INFINITY || l0 == 0.f) ? 0.f : ex2(m0 - mm);
    const float c1 = (mm == -INFINITY || l1 == 0.f) ? 0.f : ex2(m1 - mm);
    const float lsum = l0 * c0 + l1 * c1;
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    const float w0 = c0 * inv, w1 = c1 * inv;
#pragma unroll
    for (int ci = 0; ci < 2; ++ci) {
      const int c = grp * 2 + ci;
      uint32_t r0[32], r1[32];
      tmem_ld32(tmem + lane_off + TM_O + c * 32, r0);
      tmem_ld32(tmem + lane_off + TM_O + 128 + c * 32, r1);
      tmem_wait_ld();
      if (qi < sd.len) {
#pragma unroll
        for (int d0 = 0; d0 < 32; d0 += 8) {
          float g[8];
          if (a.gsig) {
            const uint4 gv = gpre[ci * 4 + d0 / 8];
            const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              g[2 * k] = __bfloat162float(gp[k].x);
              g[2 * k + 1] = __bfloat162float(gp[k].y);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) g[k] = 1.f;
          }
          uint32_t op[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float v[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int d = d0 + 2 * k + e;
              // an accumulator that received no tile is never read (w == 0)
              const float o0 = w0 != 0.f ? __uint_as_float(r0[d]) * w0 : 0.f;
              const float o1 = w1 != 0.f ? __uint_as_float(r1[d]) * w1 : 0.f;
              v[e] = (o0 + o1) * g[2 * k + e];
            }
            __nv_bfloat162 t = __floats2bfloat162_rn(v[0], v[1]);
            op[k] = *reinterpret_cast<uint32_t*>(&t);
          }
          *reinterpret_cast<uint4*>(a.out + off + c * 32 + d0) = make_uint4(op[0], op[1], op[2], op[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool attention_tc_supported(const AttnParams& p) {
  if (p.hd != HDIM) return false;
  // Key-padding masks (condition encoders) stay on the mma.sync kernel, which
  // zero-fills masked keys so a non-finite V row at a masked position cannot
  // reach the P.V product.
  if (p.key_mask) return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
                       reinterpret_cast<uintptr_t>(p.v) | reinterpret_cast<uintptr_t>(p.out) |
                       (p.gsig ? reinterpret_cast<uintptr_t>(p.gsig) : 0) |
                       (p.ck ? reinterpret_cast<uintptr_t>(p.ck) : 0) | (p.cv ? reinterpret_cast<uintptr_t>(p.cv) : 0);
  // TMA boxes are 128 rows: keep every tensor at least one box tall
  const bool ctx_ok = !(p.ck && p.cv) || p.ctx_rows == 0 || p.ctx_rows >= KT;
  return (al & 15) == 0 && p.rows >= QT && ctx_ok;
}

void attention_tc(const AttnParams& p, cudaStream_t s) {
  static unsigned attr_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_mask & (1u << (dev & 31)))) {
    IRT_CUDA(cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
    attr_mask |= 1u << (dev & 31);
  }
  const long D = (long)p.H * HDIM;
  // copies (the map cache may be cleared between calls)
  const CUtensorMap mq = tma_map_bf16(p.q, p.rows, D, D, 128);
  const CUtensorMap mk = tma_map_bf16(p.k, p.rows, D, D, 128);
  const CUtensorMap mv = tma_map_bf16(p.v, p.rows, D, D, 128);
  const bool has_ctx = p.ck && p.cv && p.ctx_rows > 0;
  const CUtensorMap mck = has_ctx ? tma_map_bf16(p.ck, p.ctx_rows, D, D, 128) : mk;
  const CUtensorMap mcv = has_ctx ? tma_map_bf16(p.cv, p.ctx_rows, D, D, 128) : mv;
  TcAttnArgs a;
  a.seqs = p.seqs;
  a.gsig = reinterpret_cast<const bf16*>(p.gsig);
  a.out = reinterpret_cast<bf16*>(p.out);
  a.H = p.H;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  dim3 grid((p.max_len + QT - 1) / QT, p.H, p.nseq);
  launch_pdl(attn_tc_kernel, grid, dim3(THREADS), SMEM, s, mq, mk, mv, mck, mcv, a);
  IRT_CHECK_LAUNCH();
}

int read_and_clear_attn_error() { return read_and_clear_flag(); }

}  // namespace irt
