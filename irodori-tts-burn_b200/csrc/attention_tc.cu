// tcgen05 / TMEM flash attention for sm_100a (hd = 128, bf16 operands).
//
// One CTA = one (sequence, head, 128-query tile); two CTAs share an SM (256
// TMEM columns and ~98 KB of shared memory each), so one CTA's softmax and
// load latencies overlap the other's tensor-core work.  192 threads:
//   warp 0      TMA producer: the Q tile once, then per 64-key tile a K tile
//               and a V tile, each on its own 2-stage ring (self keys first,
//               then context); K runs two tiles ahead of V
//   warp 1      TMEM allocator + single-thread MMA issuer:
//                 S_j  = Q K_j^T   (A = Q in shared memory, B = K_j, both
//                                   K-major)                -> TMEM S[j&1]
//                 O   += P_j V_j   (A = P_j in TMEM, B = V_j MN-major) -> TMEM O
//               issue order S_0, S_1, then per j: P_j V_j, S_{j+2}; S_{j+2}
//               overwrites the buffer that held S_j / P_j, which the in-order
//               tensor pipe has consumed by then.  A final commit after the
//               last P V signals the epilogue.
//   warps 2..5  softmax: thread r of a warp owns query row r of its TMEM lane
//               quadrant, whole rows, so no cross-warp exchange.  Per tile a
//               thread loads its 64 scores (one batched wait), takes the row
//               max, writes P = exp2(s*scale - m) as packed bf16 over the
//               first 32 columns of the same S buffer (the A operand of P V)
//               and accumulates the row sum.  The running max is only raised
//               when a row max grows by more than 2^8 (conditional rescale);
//               then the warp rescales its rows of O after the previous P V
//               has completed.  Skipping is exact: O and l share the same
//               stale max.
// TMEM columns: S0 [0,64) S1 [64,128) O [128,256).
// Keys past a sequence's end get -inf scores; a row with no valid key outputs
// 0.  Output = (O / l) * sigmoid-gate, bf16.
#include <algorithm>
#include <cstdlib>

#include "common.hpp"
#include "kernels.hpp"
#include "tc_common.cuh"

namespace irt {

const CUtensorMap& tma_map_bf16(const void* p, long rows, long cols, long ld, int box_rows);

namespace {

using namespace tcx;

constexpr int QT = 128, HDIM = 128, SM_WARPS = 4, THREADS = 64 + 32 * SM_WARPS, NKV = 2;
constexpr uint32_t Q_BYTES = QT * HDIM * 2;     // 32 KB (two 16 KB 64-column halves)
constexpr uint32_t Q_HALF = Q_BYTES / 2;
constexpr uint32_t IDESC_O = idesc_bf16(128, HDIM, true);
constexpr float RESCALE_LOG2 = 8.f;  // raise the running max only beyond 2^8 growth

// Key-tile width variants.  KT = 64: two CTAs per SM (256 TMEM columns and
// ~98 KB of shared memory each).  KT = 128: one CTA per SM with all 512 TMEM
// columns (two 128-column score buffers and O) and twice the keys per
// softmax / MMA round trip -- for launches with no more CTAs than SMs, where
// a second CTA per SM would not exist anyway.
template <int KT_>
struct AttnCfg {
  static constexpr int KT = KT_;
  static constexpr uint32_t TILE_BYTES = KT * HDIM * 2;  // two 64-column halves
  static constexpr uint32_t HALF = TILE_BYTES / 2;
  // smem: Q | K ring | V ring | barriers
  static constexpr uint32_t OFF_Q = 0, OFF_K = Q_BYTES, OFF_V = OFF_K + NKV * TILE_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + NKV * TILE_BYTES;
  static constexpr size_t SMEM = OFF_BAR + 256 + 1024;
  static constexpr uint32_t IDESC_S = idesc_bf16(128, KT, false);
  static constexpr uint32_t TM_S = 0, TM_O = 2 * KT, TM_COLS = KT == 64 ? 256 : 512;
  static constexpr int CTAS_PER_SM = KT == 64 ? 2 : 1;
};

struct TcAttnArgs {
  const SeqDesc* seqs;
  const bf16* gsig;
  bf16* out;
  int H;
  float scale_log2;
};


// tcgen05.mma with the A operand in tensor memory (K-major, two bf16 per
// 32-bit column: element k of a row sits in column k / 2).
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

template <int KT_>
__global__ void __launch_bounds__(THREADS, AttnCfg<KT_>::CTAS_PER_SM)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmCK,
                   const __grid_constant__ CUtensorMap tmCV, const __grid_constant__ TcAttnArgs a) {
  using C = AttnCfg<KT_>;
  constexpr int KT = C::KT;
  constexpr uint32_t TILE_BYTES = C::TILE_BYTES, HALF = C::HALF, OFF_Q = C::OFF_Q, OFF_K = C::OFF_K,
                     OFF_V = C::OFF_V, OFF_BAR = C::OFF_BAR, IDESC_S = C::IDESC_S, TM_S = C::TM_S, TM_O = C::TM_O,
                     TM_COLS = C::TM_COLS;
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
  const uint32_t Q_FULL = bar(0), O_DONE = bar(1), O_FINAL = bar(2);
  auto K_FULL = [&](int s) { return bar(3 + s); };
  auto K_EMPTY = [&](int s) { return bar(3 + NKV + s); };
  auto V_FULL = [&](int s) { return bar(3 + 2 * NKV + s); };
  auto V_EMPTY = [&](int s) { return bar(3 + 3 * NKV + s); };
  auto S_FULL = [&](int b) { return bar(3 + 4 * NKV + b); };
  auto P_FULL = [&](int b) { return bar(5 + 4 * NKV + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7 + 4 * NKV);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_self = (sd.len + KT - 1) / KT;
  const int n_ctx = (sd.ctx_len + KT - 1) / KT;
  const int ntiles = n_self + n_ctx;  // >= 1: q0 < len

  if (threadIdx.x == 0) {
    mbar_init(Q_FULL, 1);
    mbar_init(O_DONE, 1);
    mbar_init(O_FINAL, 1);
    for (int r = 0; r < NKV; ++r) {
      mbar_init(K_FULL(r), 1);
      mbar_init(K_EMPTY(r), 1);
      mbar_init(V_FULL(r), 1);
      mbar_init(V_EMPTY(r), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(S_FULL(b), 1);
      mbar_init(P_FULL(b), SM_WARPS);
    }
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), TM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(sm + OFF_Q);
  auto sK = [&](int s) { return smem_u32(sm + OFF_K + s * TILE_BYTES); };
  auto sV = [&](int s) { return smem_u32(sm + OFF_V + s * TILE_BYTES); };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_map(&tmK);
      prefetch_map(&tmV);
      mbar_expect_tx(Q_FULL, Q_BYTES);
      tma_load_2d(sQ, &tmQ, Q_FULL, h * HDIM, sd.tok_start + q0);
      tma_load_2d(sQ + Q_HALF, &tmQ, Q_FULL, h * HDIM + 64, sd.tok_start + q0);
      // the gate tile is only read by the epilogue: start it towards L2 now

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
      load_k(0);
      if (ntiles > 1) load_k(1);
      for (int j = 0; j < ntiles; ++j) {
        load_v(j);
        if (j + 2 < ntiles) load_k(j + 2);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      mbar_wait(Q_FULL, 0);
      tc_fence_after();
      auto issue_s = [&](int j) {
        const int r = j % NKV, b = j & 1;
        mbar_wait(K_FULL(r), (j / NKV) & 1);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HDIM / 16; ++kk) {
          // 16 hd columns: 32 bytes into one of the two 64-column halves
          const uint64_t da = sdesc_kmajor(sQ + (kk >> 2) * Q_HALF + (kk & 3) * 32);
          const uint64_t db = sdesc_kmajor(sK(r) + (kk >> 2) * HALF + (kk & 3) * 32);
          umma_f16(tmem + TM_S + b * KT, da, db, IDESC_S, kk != 0);
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
          // B = V [keys][hd] (MN-major: 64-column halves HALF apart, 8-key
          // groups 1 KB apart)
          const uint64_t bdesc = sdesc_sw128(sV(r) + kk * 16 * 128, HALF, 1024);
          umma_ts(tmem + TM_O, tmem + TM_S + s * KT + kk * 8, bdesc, IDESC_O, (j | kk) != 0);
        }
        umma_commit(V_EMPTY(r));
        umma_commit(O_DONE);  // one phase per tile
        // S_{j+2} reuses buffer s: issued after P_j V_j, which the tensor
        // pipe executes first
        if (j + 2 < ntiles) issue_s(j + 2);
      }
      umma_commit(O_FINAL);  // every MMA of this CTA, the last P V included
    }
  } else {
    // ---------------- softmax warps: one per TMEM lane quadrant ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int qi = q0 + row;
    const bool row_ok = qi < sd.len;
    const long off = (long)(sd.tok_start + (row_ok ? qi : 0)) * D + h * HDIM;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < ntiles; ++j) {
      const int b = j & 1;
      const int kvalid = (j < n_self ? sd.len - j * KT : sd.ctx_len - (j - n_self) * KT);  // valid keys in tile
      mbar_wait(S_FULL(b), (j >> 1) & 1);
      tc_fence_after();
      uint32_t sr[KT];
#pragma unroll
      for (int g = 0; g < KT / 32; ++g)
        tmem_ld32(tmem + lane_off + TM_S + b * KT + 32 * g, *reinterpret_cast<uint32_t(*)[32]>(&sr[32 * g]));
      tmem_wait_ld();
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
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * a.scale_log2;
      // conditional rescale of the running max
      float corr = 1.f;
      const bool raise = mx > m_run + RESCALE_LOG2 || (m_run == -INFINITY && mx > -INFINITY);
      if (raise) {
        corr = m_run == -INFINITY ? 0.f : ex2(m_run - mx);
        m_run = mx;
      }
      const float nbase = m_run == -INFINITY ? 0.f : -m_run;
      // Rescale this warp's rows of O (warp-collective) once the previous
      // P V has completed: S_j done implies P_{j-2} V_{j-2} done, and
      // P_j V_j cannot start before this tile's P, so the O_DONE phase in
      // flight is j-1 or already j.
      if (__any_sync(0xffffffffu, raise) && j > 0) {
        mbar_wait(O_DONE, (j - 1) & 1);
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HDIM / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_off + TM_O + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st32(tmem + lane_off + TM_O + c * 32, r);
        }
      }
      // P = 2^(s * scale - m) as packed bf16: keys 2c, 2c+1 in column c of
      // the S buffer (this thread's scores are all in registers already)
      // (the scale-and-shift and the row sums as packed f32 pairs: the same
      // roundings as the scalar forms, half the instructions)
      uint32_t pk[KT / 2];
      const uint64_t sc2 = f2_pack(__float_as_uint(a.scale_log2), __float_as_uint(a.scale_log2));
      const uint64_t nb2 = f2_pack(__float_as_uint(nbase), __float_as_uint(nbase));
      uint64_t rs2 = 0;  // (rs0, rs1) = (+0, +0)
#pragma unroll
      for (int c = 0; c < KT / 2; ++c) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(sr[2 * c], sr[2 * c + 1]), sc2, nb2), x0, x1);
        const float p0 = ex2(x0), p1 = ex2(x1);
        rs2 = f2_add(rs2, f2_pack(__float_as_uint(p0), __float_as_uint(p1)));
        pk[c] = pack_bf16x2(p0, p1);
      }
      float rs0, rs1;
      f2_unpack(rs2, rs0, rs1);
#pragma unroll
      for (int g = 0; g < KT / 64; ++g)
        tmem_st32(tmem + lane_off + TM_S + b * KT + 32 * g, *reinterpret_cast<uint32_t(*)[32]>(&pk[32 * g]));
      tmem_wait_st();
      l_run = l_run * corr + (rs0 + rs1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(P_FULL(b));
    }

    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    mbar_wait(O_FINAL, 0);
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < HDIM / 32; ++c) {
      uint4 gv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        gv[u] = (a.gsig && row_ok) ? *reinterpret_cast<const uint4*>(a.gsig + off + c * 32 + u * 8)
                                   : make_uint4(0, 0, 0, 0);
      uint32_t r[32];
      tmem_ld32(tmem + lane_off + TM_O + c * 32, r);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv[u]);
          uint32_t op[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float g0 = a.gsig ? __bfloat162float(gp[k].x) : 1.f;
            const float g1 = a.gsig ? __bfloat162float(gp[k].y) : 1.f;
            op[k] = pack_bf16x2(__uint_as_float(r[u * 8 + 2 * k]) * inv * g0,
                                __uint_as_float(r[u * 8 + 2 * k + 1]) * inv * g1);
          }
          *reinterpret_cast<uint4*>(a.out + off + c * 32 + u * 8) = make_uint4(op[0], op[1], op[2], op[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
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
  // TMA boxes are 128 rows (Q) and 64 rows (K, V, context; 128 for the
  // 128-key variant, taken only when they fit): keep every tensor at least
  // one box tall
  const bool ctx_ok = !(p.ck && p.cv) || p.ctx_rows == 0 || p.ctx_rows >= 64;
  return (al & 15) == 0 && p.rows >= QT && ctx_ok;
}

namespace {
template <int KT>
void launch_attn(const AttnParams& p, cudaStream_t s) {
  using C = AttnCfg<KT>;
  static unsigned attr_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_mask & (1u << (dev & 31)))) {
    IRT_CUDA(cudaFuncSetAttribute(attn_tc_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_mask |= 1u << (dev & 31);
  }
  const long D = (long)p.H * HDIM;
  // copies (the map cache may be cleared between calls)
  const CUtensorMap mq = tma_map_bf16(p.q, p.rows, D, D, QT);
  const CUtensorMap mk = tma_map_bf16(p.k, p.rows, D, D, KT);
  const CUtensorMap mv = tma_map_bf16(p.v, p.rows, D, D, KT);
  const bool has_ctx = p.ck && p.cv && p.ctx_rows > 0;
  const CUtensorMap mck = has_ctx ? tma_map_bf16(p.ck, p.ctx_rows, D, D, KT) : mk;
  const CUtensorMap mcv = has_ctx ? tma_map_bf16(p.cv, p.ctx_rows, D, D, KT) : mv;
  TcAttnArgs a;
  a.seqs = p.seqs;
  a.gsig = reinterpret_cast<const bf16*>(p.gsig);
  a.out = reinterpret_cast<bf16*>(p.out);
  a.H = p.H;
  a.scale_log2 = p.scale * 1.4426950408889634f;
  dim3 grid((p.max_len + QT - 1) / QT, p.H, p.nseq);
  launch_pdl(attn_tc_kernel<KT>, grid, dim3(THREADS), C::SMEM, s, mq, mk, mv, mck, mcv, a);
  IRT_CHECK_LAUNCH();
}
}  // namespace

void attention_tc(const AttnParams& p, cudaStream_t s) {
  // 128-key tiles when the launch has no more CTAs than SMs (one CTA per SM
  // either way) and every K / V tensor is at least one 128-row box tall;
  // 64-key tiles at two CTAs per SM otherwise.  IRT_ATTN_KT=64 / 128 forces
  // one (measurements).
  int dev = 0, sms = 0;
  IRT_CUDA(cudaGetDevice(&dev));
  IRT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const long ctas = (long)((p.max_len + QT - 1) / QT) * p.H * p.nseq;
  const bool tall = p.rows >= 128 && (!(p.ck && p.cv) || p.ctx_rows == 0 || p.ctx_rows >= 128);
  bool wide = tall && ctas <= sms;
  if (const char* e = std::getenv("IRT_ATTN_KT")) wide = tall && std::atoi(e) == 128;
  if (wide) launch_attn<128>(p, s);
  else launch_attn<64>(p, s);
}

int read_and_clear_attn_error() { return read_and_clear_flag(); }

int attn_watchdog_probe(unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns) {
  const cudaError_t e = tcx::run_watchdog_probe(limit_ns, waits, elapsed_ns);
  if (e != cudaSuccess) throw Error(IRT_E_CUDA, std::string("watchdog probe: ") + cudaGetErrorString(e));
  return 0;
}

}  // namespace irt
