// tcgen05 / TMEM flash attention for sm_100a (hd = 128, bf16 operands).
//
// One CTA = one (sequence, head, 128-query tile).  320 threads:
//   warp 0      TMA producer: per 128-key tile a K tile and a V tile, each on
//               its own 2-stage ring (self keys first, then context); K runs
//               two tiles ahead of V
//   warp 1      TMEM allocator + single-thread MMA issuer, both products with
//               the A operand in tensor memory so only K and V are read from
//               shared memory:
//                 S_j  = Q K_j^T   (A = Q in TMEM, B = K_j K-major)  -> TMEM S[j&1]
//                 O   += P_j V_j   (A = P_j in TMEM, B = V_j MN-major) -> TMEM O
//               issue order S_0, S_1, then per j: P_j V_j, S_{j+2}; S_{j+2}
//               overwrites the buffer that held S_j / P_j, which the in-order
//               tensor pipe has consumed by then
//   warps 2..9  softmax: thread r of a warp owns query row r of its TMEM lane
//               quadrant; the two warps of a quadrant split the 128 keys of a
//               tile (64 each) and exchange row maxima through shared memory.
//               Per tile a warp loads its 64 scores (one batched wait), takes
//               the row max on raw scores, writes P = exp2(s*scale - m) as
//               packed bf16 over its scores' columns (the A operand of P V),
//               and keeps its half of the row sum.  The running max is only
//               raised when a row max grows by more than 2^8 (conditional
//               rescale); then each warp rescales its 64 O columns after the
//               previous P V has completed.  Skipping is exact: O and l share
//               the same stale max.
// TMEM columns: S0 [0,128) S1 [128,256) O [256,384) Q [384,448).
// Keys past a sequence's end get -inf scores; a row with no valid key outputs
// 0.  Output = (O / l) * sigmoid-gate, bf16.
#include <algorithm>

#include "common.hpp"
#include "kernels.hpp"
#include "tc_common.cuh"

namespace irt {

const CUtensorMap& tma_map_bf16(const void* p, long rows, long cols, long ld, int box_rows);

namespace {

using namespace tcx;

constexpr int QT = 128, KT = 128, HDIM = 128, THREADS = 320, NKV = 2;
constexpr uint32_t TILE_BYTES = KT * HDIM * 2;  // 32 KB (two 16 KB 64-column halves)
constexpr uint32_t HALF = TILE_BYTES / 2;
// smem: K ring | V ring | exchange | barriers
constexpr uint32_t OFF_K = 0, OFF_V = NKV * TILE_BYTES;
constexpr uint32_t OFF_X = OFF_V + NKV * TILE_BYTES;  // [2 slots][2 halves][128 rows] f32 maxima, [2][128] sums
constexpr uint32_t X_BYTES = (2 * 2 * 128 + 2 * 128) * 4;
constexpr uint32_t OFF_BAR = OFF_X + X_BYTES;
constexpr size_t SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t IDESC_S = idesc_bf16(128, 128, false);
constexpr uint32_t IDESC_O = idesc_bf16(128, 128, true);
constexpr uint32_t TM_S = 0, TM_O = 256, TM_Q = 384;
constexpr float RESCALE_LOG2 = 8.f;  // raise the running max only beyond 2^8 growth

struct TcAttnArgs {
  const SeqDesc* seqs;
  const bf16* q;
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

// tcgen05.mma with the A operand in tensor memory (K-major, two bf16 per
// 32-bit column: element k of a row sits in column k / 2).
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}

__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmCK, const __grid_constant__ CUtensorMap tmCV,
                   const __grid_constant__ TcAttnArgs a) {
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
  const uint32_t Q_READY = bar(0), O_DONE = bar(1);
  auto K_FULL = [&](int s) { return bar(2 + s); };
  auto K_EMPTY = [&](int s) { return bar(2 + NKV + s); };
  auto V_FULL = [&](int s) { return bar(2 + 2 * NKV + s); };
  auto V_EMPTY = [&](int s) { return bar(2 + 3 * NKV + s); };
  auto S_FULL = [&](int b) { return bar(2 + 4 * NKV + b); };
  auto P_FULL = [&](int b) { return bar(4 + 4 * NKV + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6 + 4 * NKV);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_self = (sd.len + KT - 1) / KT;
  const int n_ctx = (sd.ctx_len + KT - 1) / KT;
  const int ntiles = n_self + n_ctx;

  if (threadIdx.x == 0) {
    mbar_init(Q_READY, 8);
    mbar_init(O_DONE, 1);
    for (int r = 0; r < NKV; ++r) {
      mbar_init(K_FULL(r), 1);
      mbar_init(K_EMPTY(r), 1);
      mbar_init(V_FULL(r), 1);
      mbar_init(V_EMPTY(r), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(S_FULL(b), 1);
      mbar_init(P_FULL(b), 8);
    }
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto sK = [&](int s) { return smem_u32(sm + OFF_K + s * TILE_BYTES); };
  auto sV = [&](int s) { return smem_u32(sm + OFF_V + s * TILE_BYTES); };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_map(&tmK);
      prefetch_map(&tmV);
      auto row_of = [&](int j) { return j < n_self ? sd.tok_start + j * KT : sd.ctx_off + (j - n_self) * KT; };
      auto load_k = [&](int j) {
        const int s = j % NKV;
        mbar_wait(K_EMPTY(s), ((j / NKV) & 1) ^ 1);
        mbar_expect_tx(K_FULL(s), TILE_BYTES);
        const CUtensorMap* m = j < n_self ? &tmK : &tmCK;
        tma_load_2d(sK(s), m, K_FULL(s), h * HDIM, row_of(j));
        tma_load_2d(sK(s) + HALF, m, K_FULL(s), h * HDIM + 64, row_of(j));
      };
      auto load_v = [&](int j) {
        const int s = j % NKV;
        mbar_wait(V_EMPTY(s), ((j / NKV) & 1) ^ 1);
        mbar_expect_tx(V_FULL(s), TILE_BYTES);
        const CUtensorMap* m = j < n_self ? &tmV : &tmCV;
        tma_load_2d(sV(s), m, V_FULL(s), h * HDIM, row_of(j));
        tma_load_2d(sV(s) + HALF, m, V_FULL(s), h * HDIM + 64, row_of(j));
      };
      // K two tiles ahead of V, matching the MMA issue order
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
      mbar_wait(Q_READY, 0);
      tc_fence_after();
      auto issue_s = [&](int j) {
        const int r = j % NKV, b = j & 1;
        mbar_wait(K_FULL(r), (j / NKV) & 1);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HDIM / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          umma_ts(tmem + TM_S + b * 128, tmem + TM_Q + kk * 8, sdesc_kmajor(sK(r) + off), IDESC_S, kk != 0);
        }
        umma_commit(S_FULL(b));
        umma_commit(K_EMPTY(r));
      };
      issue_s(0);
      if (ntiles > 1) issue_s(1);
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1, r = j % NKV;
        mbar_wait(V_FULL(r), (j / NKV) & 1);
        mbar_wait(P_FULL(s), (j >> 1) & 1);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
          // A = P_j (keys 16kk..16kk+15 packed in 8 columns of S buffer s);
          // B = V [keys][hd] (MN-major: 64-column halves 16 KB apart, 8-key
          // groups 1 KB apart)
          const uint64_t bdesc = sdesc_sw128(sV(r) + kk * 16 * 128, HALF, 1024);
          umma_ts(tmem + TM_O, tmem + TM_S + s * 128 + kk * 8, bdesc, IDESC_O, (j | kk) != 0);
        }
        umma_commit(V_EMPTY(r));
        umma_commit(O_DONE);  // one phase per tile
        // S_{j+2} reuses buffer s: issued after P_j V_j, which the tensor
        // pipe executes first
        if (j + 2 < ntiles) issue_s(j + 2);
      }
    }
  } else {
    // ---------------- softmax warps: two per TMEM lane quadrant ----------------
    const int quad = warp & 3;
    const int hh = (warp - 2) >> 2;    // key half of every tile (and hd half of Q / O)
    const int row = quad * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int qi = q0 + row;
    const bool row_ok = qi < sd.len;
    const long off = (long)(sd.tok_start + (row_ok ? qi : 0)) * D + h * HDIM;
    float* xm = reinterpret_cast<float*>(sm + OFF_X);  // [slot][half][row] maxima
    float* xl = xm + 4 * 128;                          // [half][row] sums
    auto pair_sync = [&]() {
      tc_fence_before();
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory");
      tc_fence_after();
    };
    // Q (this warp's 64 hd columns of its rows) -> TMEM, packed bf16 pairs
    {
      uint32_t qr[32];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint4 v = row_ok ? *reinterpret_cast<const uint4*>(a.q + off + hh * 64 + u * 8) : make_uint4(0, 0, 0, 0);
        qr[4 * u] = v.x;
        qr[4 * u + 1] = v.y;
        qr[4 * u + 2] = v.z;
        qr[4 * u + 3] = v.w;
      }
      tmem_st32(tmem + lane_off + TM_Q + hh * 32, qr);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(Q_READY);
    }
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < ntiles; ++j) {
      const int b = j & 1;
      const int kvalid = (j < n_self ? sd.len - j * KT : sd.ctx_len - (j - n_self) * KT);  // valid keys in tile
      const int kv_h = kvalid - hh * 64;  // valid keys in this warp's half
      mbar_wait(S_FULL(b), (j >> 1) & 1);
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(tmem + lane_off + TM_S + b * 128 + hh * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(tmem + lane_off + TM_S + b * 128 + hh * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_wait_ld();
      if (kv_h < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= kv_h) sr[i] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; i += 4) {
        mx0 = fmaxf(mx0, __uint_as_float(sr[i]));
        mx1 = fmaxf(mx1, __uint_as_float(sr[i + 1]));
        mx2 = fmaxf(mx2, __uint_as_float(sr[i + 2]));
        mx3 = fmaxf(mx3, __uint_as_float(sr[i + 3]));
      }
      // row max of the whole tile: exchange with the other key half.  The
      // barrier also orders both halves' S loads before the P stores below
      // (the other half's P overwrites columns this half has just read).
      xm[(b * 2 + hh) * 128 + row] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      pair_sync();
      const float mx = fmaxf(xm[(b * 2) * 128 + row], xm[(b * 2 + 1) * 128 + row]) * a.scale_log2;
      // conditional rescale of the running max (identical in both halves)
      float corr = 1.f;
      const bool raise = mx > m_run + RESCALE_LOG2 || (m_run == -INFINITY && mx > -INFINITY);
      if (raise) {
        corr = m_run == -INFINITY ? 0.f : ex2(m_run - mx);
        m_run = mx;
      }
      const float nbase = m_run == -INFINITY ? 0.f : -m_run;
      // Rescale this half's O columns (warp-collective) once the previous
      // P V has completed.
      if (__any_sync(0xffffffffu, raise) && j > 0) {
        mbar_wait(O_DONE, (j - 1) & 1);
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + TM_O + hh * 64 + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(tmem + lane_off + TM_O + hh * 64 + c * 32, r);
        }
      }
      // P = 2^(s * scale - m) as packed bf16 over this half's score columns
      // (keys hh*64 + 2c, +1 in column hh*32 + c of the S buffer)
      uint32_t pk[32];
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = ex2(fmaf(__uint_as_float(sr[2 * c]), a.scale_log2, nbase));
        const float p1 = ex2(fmaf(__uint_as_float(sr[2 * c + 1]), a.scale_log2, nbase));
        rs0 += p0;
        rs1 += p1;
        pk[c] = pack_bf16x2(p0, p1);
      }
      tmem_st32(tmem + lane_off + TM_S + b * 128 + hh * 32, pk);
      tmem_wait_st();
      l_run = l_run * corr + (rs0 + rs1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(P_FULL(b));
    }

    // prefetch this row's gate half (independent of the attention result)
    uint4 gpre[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      gpre[u] = (a.gsig && row_ok) ? *reinterpret_cast<const uint4*>(a.gsig + off + hh * 64 + u * 8)
                                   : make_uint4(0, 0, 0, 0);
    if (ntiles > 0) mbar_wait(O_DONE, (ntiles - 1) & 1);  // last P V
    tc_fence_after();
    xl[hh * 128 + row] = l_run;
    pair_sync();
    const float lsum = xl[row] + xl[128 + row];
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_off + TM_O + hh * 64 + c * 32, r);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 gv = gpre[c * 4 + u];
          const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv);
          uint32_t op[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float g0 = a.gsig ? __bfloat162float(gp[k].x) : 1.f;
            const float g1 = a.gsig ? __bfloat162float(gp[k].y) : 1.f;
            op[k] = pack_bf16x2(__uint_as_float(r[u * 8 + 2 * k]) * inv * g0,
                                __uint_as_float(r[u * 8 + 2 * k + 1]) * inv * g1);
          }
          *reinterpret_cast<uint4*>(a.out + off + hh * 64 + c * 32 + u * 8) = make_uint4(op[0], op[1], op[2], op[3]);
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
  const CUtensorMap mk = tma_map_bf16(p.k, p.rows, D, D, 128);
  const CUtensorMap mv = tma_map_bf16(p.v, p.rows, D, D, 128);
  const bool has_ctx = p.ck && p.cv && p.ctx_rows > 0;
  const CUtensorMap mck = has_ctx ? tma_map_bf16(p.ck, p.ctx_rows, D, D, 128) : mk;
  const CUtensorMap mcv = has_ctx ? tma_map_bf16(p.cv, p.ctx_rows, D, D, 128) : mv;
  TcAttnArgs a;
  a.seqs = p.seqs;
  a.q = reinterpret_cast<const bf16*>(p.q);
  a.gsig = reinterpret_cast<const bf16*>(p.gsig);
  a.out = reinterpret_cast<bf16*>(p.out);
  a.H = p.H;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  dim3 grid((p.max_len + QT - 1) / QT, p.H, p.nseq);
  launch_pdl(attn_tc_kernel, grid, dim3(THREADS), SMEM, s, mk, mv, mck, mcv, a);
  IRT_CHECK_LAUNCH();
}

int read_and_clear_attn_error() { return read_and_clear_flag(); }

}  // namespace irt
