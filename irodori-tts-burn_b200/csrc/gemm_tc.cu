// tcgen05 / TMEM / TMA bf16 GEMM for sm_100a with fused epilogues.
//
//   C[M,N] = A[M,K] . B[N,K]^T   (A activations, B PyTorch-layout weights;
//                                 both K-major, bf16; fp32 accumulate in TMEM)
//
// Persistent, warp-specialised CTA of 320 threads:
//   warp 0      TMA producer: A tile 128x64 and B tile BNx64 per stage (128B swizzle)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16)
//   warps 2..9  epilogue: tcgen05.ld 32x32b -> registers -> fused epilogue -> global;
//               two warps per TMEM lane quadrant split the tile's columns (one
//               128-column head each for QKVG, alternate chunks otherwise)
// Two TMEM accumulator buffers let the epilogue of tile i overlap the MMAs of
// tile i+1.  Tile order: see tile_coords.  Every
// mbarrier wait is the bounded tcx::mbar_wait (4 s watchdog that sets this
// file's device error flag instead of hanging; later waits then give up at
// once).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "common.hpp"
#include "epilogue.cuh"
#include "tc_common.cuh"

namespace irt {

int read_and_clear_kernel_error() { return tcx::read_and_clear_flag(); }

int gemm_watchdog_probe(unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns) {
  const cudaError_t e = tcx::run_watchdog_probe(limit_ns, waits, elapsed_ns);
  if (e != cudaSuccess) throw Error(IRT_E_CUDA, std::string("watchdog probe: ") + cudaGetErrorString(e));
  return 0;
}

namespace tc {

constexpr int BM = 128, BK = 64, EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
// Smallest k-block span of a group in a tail split (splits == -2).
constexpr int TAIL_MIN_SPAN = 8;
// TF: k-blocks per accumulator chunk in the A_hi.B_hi segment (each chunk's
// MMA chain restarts at 0 and is added into the tile sum by the epilogue
// warps); the two small-term segments (A_hi.B_lo, A_lo.B_hi, ~2^-11 of the
// product) run one chunk each, so a chunk never adds small terms onto a large
// accumulator.  The small-term segments come first: their long chunks keep the
// tensor core busy while the epilogue warps finish the previous tile.
constexpr int TF_CHUNK = 2;
constexpr uint32_t A_BYTES = BM * BK * 2;

// End of the TF accumulation chunk that starts at k-block c0 (segments of
// kseg k-blocks; the unit ends at kb1).
__device__ __forceinline__ int tf_chunk_end(int c0, int kb1, int kseg) {
  const int seg_end = (c0 / kseg + 1) * kseg;
  return min(kb1, c0 >= 2 * kseg ? min(seg_end, c0 + TF_CHUNK) : seg_end);
}

// CG = CTAs per MMA: 1, or 2 for a CTA pair (cluster of 2) that computes a
// 256-row tile with tcgen05.mma.cta_group::2.  In a pair each CTA stages its
// own 128 rows of A and one half (BN/2 rows) of B; the MMA reads both halves,
// so every SM streams one third less operand data through shared memory per
// FLOP than a 1-CTA 128 x BN tile.
template <int BN, int CG>
struct Cfg {
  static constexpr int B_ROWS = BN / CG;  // B rows staged by each CTA
  static constexpr uint32_t B_BYTES = B_ROWS * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196608 / STAGE_BYTES) > 8 ? 8 : (196608 / STAGE_BYTES);
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers
  // stages | per-warp epilogue buffers (32x33 f32 transpose, or a 4 KB
  // 128B-swizzled reduce tile at a 1024-aligned offset) | barriers (256 B) | alignment slack
  static constexpr uint32_t OFF_EPI = STAGES * STAGE_BYTES;
  static constexpr uint32_t EPI_BYTES = EPI_WARPS * 32 * 33 * 4;
  static constexpr size_t SMEM = (size_t)OFF_EPI + EPI_BYTES + 256 + 1024;
  // instruction descriptor, kind::f16: D=f32 (bit4), A=B=bf16 (bits 7,10), K-major
  // both, N>>3 at bits 17-22, M>>4 at bits 24-28 (M = 128 per CTA of the group).
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)((BM * CG) >> 4) << 24);
  // kind::tf32 (the f32 mode's split product, TF below): same tile bytes, 32
  // f32 per 128-byte row instead of 64 bf16.
  static constexpr uint32_t IDESC_TF = tcx::idesc_tf32(BM * CG, BN);
};

// The sm_100a helper layer (mbarriers with the bounded wait, TMA, UMMA
// descriptors, tcgen05 MMA / commit / ld, CTA-pair forms) is tc_common.cuh.
using namespace tcx;

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (SBO).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) { return sdesc_kmajor(saddr); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32], int off) {
  tcx::tmem_ld32(taddr + off, r);
}
__device__ __forceinline__ void fence_async_smem() { fence_proxy_async(); }

// Tile order.  With many row blocks (large M) tiles are walked row-major, m
// outer and n inner: the CTAs running at one time cover a few row blocks of A
// and every n-tile of the weight, so each row block of A comes from HBM once
// and the weight (24-48 MB for the DiT GEMMs), touched by every row block in
// turn, stays hot in L2.  On the four DiT GEMMs of one layer at M = 54,504
// this moved 5.75 GB of DRAM traffic per layer instead of 7.53 GB for
// n-outer groups of 16 row blocks, and ran 3 % faster.  With at most
// SMALL_M_TILES row blocks (all of A fits in L2) n is the outer index: each
// weight tile is then read by all row blocks at about the same time, which
// measured 2-4 % faster at M = 750-1500.
constexpr int SMALL_M_TILES = 16;
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& m_idx, int& n_idx) {
  if (m_tiles <= SMALL_M_TILES) {
    n_idx = t / m_tiles;
    m_idx = t - n_idx * m_tiles;
  } else {
    m_idx = t / n_tiles;
    n_idx = t - m_idx * n_tiles;
  }
}

// Work decomposition shared by the producer, MMA and epilogue roles.
//  splits >= 1: units (tile, K-split) dealt round-robin to the work groups
//    (a group = one CTA, or one CTA pair).
//  splits == -1 (stream-K; only for the additive RESID epilogue, whose partial
//    products are reduce-added into x): group g owns the contiguous range
//    [g * L, (g + 1) * L) of all tiles' k-blocks taken in tile order,
//    L = ceil(tiles * k_blocks / groups), so every group does the same number
//    of k-blocks; its units are the pieces of that range inside each tile.
//  splits == -2 (tail split; also additive RESID only): the first
//    floor(tiles / groups) * groups tiles are dealt whole, round-robin; the
//    k-blocks of the remaining tiles are spread as in stream-K with spans of
//    L = max(TAIL_MIN_SPAN, ceil(tail k-blocks / groups)) (fewer groups take
//    part when the tail is short), so the last, partial round of whole tiles
//    becomes a short round in which every group works.
struct Units {
  int grp0, ngrp, num_tiles, k_blocks, splits, kpb, full;
  long lo, hi;
  __device__ Units(int g, int ng, int nt, int kb, int sp, int min_span)
      : grp0(g), ngrp(ng), num_tiles(nt), k_blocks(kb), splits(sp), kpb(0), full(0), lo(0), hi(0) {
    if (sp > 0) {
      kpb = (kb + sp - 1) / sp;
    } else {
      full = sp == -2 ? (nt / ng) * ng : 0;
      const long total = (long)(nt - full) * kb;
      const long L = max(sp == -2 ? (long)min_span : 1L, (total + ng - 1) / ng);
      lo = min(total, (long)g * L);
      hi = min(total, lo + L);
    }
  }
  // The i-th unit of this group; false once past its last unit.
  __device__ bool get(int i, int& t, int& kb0, int& kb1) const {
    if (splits > 0) {
      const int u = grp0 + i * ngrp;
      if (u >= num_tiles * splits) return false;
      t = u / splits;
      kb0 = (u - t * splits) * kpb;
      kb1 = min(k_blocks, kb0 + kpb);
      return true;
    }
    const int nwhole = full / ngrp;
    if (i < nwhole) {
      t = grp0 + i * ngrp;
      kb0 = 0;
      kb1 = k_blocks;
      return true;
    }
    i -= nwhole;
    if (lo >= hi) return false;
    const int tt = (int)(lo / k_blocks) + i;
    const long s = max(lo, (long)tt * k_blocks), e = min(hi, (long)(tt + 1) * k_blocks);
    if (s >= e) return false;
    t = full + tt;
    kb0 = (int)(s - (long)tt * k_blocks);
    kb1 = (int)(e - (long)tt * k_blocks);
    return true;
  }
};

template <int N>
struct Regs {
  uint32_t r[N];
  __device__ __forceinline__ float operator()(int j) const { return __uint_as_float(r[j]); }
};

// 320 threads: registers are budgeted per 4-warp group, so 10 warps cost as
// much as 12 and the kernel must stay at or below 168 registers per thread.
// CG = 2: launched as clusters of 2 CTAs (consecutive blockIdx.x); the pair
// walks the same work units, rank 0 issues the MMAs for both.
// TF: f32 operands as tf32 hi / lo pairs (the f32 mode).  A = [A_hi | A_lo]
// [M, 2K] and B = [B_hi | B_lo] [N, 2K] (K a multiple of 32); the k-blocks run
// over three segments of K / 32 blocks each -- A_hi.B_lo, A_lo.B_hi, A_hi.B_hi
// -- into one f32 tile sum (chunked, see the epilogue), so the product keeps
// about f32 accuracy
// (the dropped A_lo.B_lo term and the tf32 reading of the lo halves are
// ~2^-22 of each product) at the tf32 tensor rate.
template <int BN, int CG, bool TF>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmX, int M, int N, int K, int splits,
                const __grid_constant__ EpiParams ep) {
  using C = Cfg<BN, CG>;
  constexpr int STAGES = C::STAGES;
  constexpr int BMT = BM * CG;  // rows of one work tile
  // TF: four 128-column accumulator buffers (see the epilogue), BN = 128
  static_assert(!TF || BN == 128, "the tf32 path runs 128-column tiles");
  constexpr int NACC = TF ? 4 : 2;
  constexpr uint32_t TMEM_COLS = TF ? NACC * BN : C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_EPI + C::EPI_BYTES);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2]; then tmem base slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * NACC);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
  const int grp0 = blockIdx.x / CG, ngrp = gridDim.x / CG;  // work-group index and count
  const int m_tiles = (M + BMT - 1) / BMT, n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = TF ? 3 * (K / 32) : (K + BK - 1) / BK;
  // work units: see Units (splits != 1 only for the additive RESID epilogue)
  const Units units(grp0, ngrp, num_tiles, k_blocks, splits, TAIL_MIN_SPAN);

  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull = [&](int b) { return smem_u32(&bars[2 * STAGES + b]); };
  auto tempty = [&](int b) { return smem_u32(&bars[2 * STAGES + NACC + b]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < NACC; ++b) {
      mbar_init(tfull(b), 1);
      // rank 0's accumulator-empty barrier counts the epilogue warps of the group
      mbar_init(tempty(b), EPI_WARPS * CG);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      // executed by one warp in each CTA of the pair: same columns in both
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  // the peer signals rank 0's barriers: both CTAs' barriers exist from here on
  if constexpr (CG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the prologue above may overlap the previous kernel; operands are read only now
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      int t, kb0, kb1;
      for (int i = 0; units.get(i, t, kb0, kb1); ++i) {
        int mi_, ni_;
        tile_coords(t, m_tiles, n_tiles, mi_, ni_);
        const int m0 = mi_ * BMT + (int)rank * BM, n0 = ni_ * BN + (int)rank * C::B_ROWS;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          mbar_wait(empty(s), ph ^ 1);
          uint8_t* a_dst = tiles + s * C::STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_BYTES;
          int ca = kb * BK, cb = kb * BK, ra = m0;  // columns of the A and B boxes, A's first row
          if constexpr (TF) {
            // K = taps x Cin_p per segment; A2 = [hi | lo] is [rows, 2 Cin_p] and
            // tap j reads A rows shifted by j * conv_dil - conv_pad (implicit
            // convolution; plain GEMM: one tap, no shift)
            const int kseg = K / 32, seg = kb / kseg, kk = kb - seg * kseg;
            const int cblocks = kseg / ep.conv_taps, tap = kk / cblocks, cblk = kk - tap * cblocks;
            // segments in order: A_hi.B_lo, A_lo.B_hi, A_hi.B_hi
            ca = (seg == 1 ? cblocks * 32 : 0) + cblk * 32;
            cb = (seg == 0 ? K : 0) + kk * 32;
            ra = m0 + tap * ep.conv_dil - ep.conv_pad;
          }
          if constexpr (CG == 2) {
            // both CTAs' copies complete on rank 0's full barrier, which
            // expects the pair's bytes
            const uint32_t fb = map_rank0(full(s));
            if (rank == 0) mbar_expect_tx(full(s), CG * C::STAGE_BYTES);
            tma_load_2d_pair(smem_u32(a_dst), &tmA, fb, ca, ra);
            tma_load_2d_pair(smem_u32(b_dst), &tmB, fb, cb, n0);
          } else {
            mbar_expect_tx(full(s), C::STAGE_BYTES);
            tma_load_2d(smem_u32(a_dst), &tmA, full(s), ca, ra);
            tma_load_2d(smem_u32(b_dst), &tmB, full(s), cb, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (rank 0 of a pair) ----------------
    if (lane == 0 && rank == 0) {
      uint32_t it = 0, tl = 0;
      int t, kb0, kb1;
      if constexpr (TF) {
        // accumulation chunks (tf_chunk_end), in turn over the four
        // accumulator buffers (tl counts chunks here)
        for (int i = 0; units.get(i, t, kb0, kb1); ++i) {
          for (int c0 = kb0, c1; c0 < kb1; c0 = c1, ++tl) {
            c1 = tf_chunk_end(c0, kb1, K / 32);
            const int buf = tl % NACC;
            const uint32_t aph = (tl / NACC) & 1;
            mbar_wait(tempty(buf), aph ^ 1);
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + buf * BN;
            for (int kb = c0; kb < c1; ++kb, ++it) {
              const int s = it % STAGES;
              const uint32_t ph = (it / STAGES) & 1;
              mbar_wait(full(s), ph);
              tc_fence_after();
              const uint32_t a_addr = smem_u32(tiles + s * C::STAGE_BYTES);
              const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {  // 32-byte K steps of 8 tf32
                const uint32_t acc = (kb != c0 || kk != 0) ? 1u : 0u;
                if constexpr (CG == 2)
                  umma_tf32_pair(d_tmem, sdesc(a_addr + kk * 32), sdesc(b_addr + kk * 32), C::IDESC_TF, acc);
                else
                  umma_tf32(d_tmem, sdesc(a_addr + kk * 32), sdesc(b_addr + kk * 32), C::IDESC_TF, acc);
              }
              if constexpr (CG == 2) umma_commit_pair(empty(s));
              else umma_commit(empty(s));
            }
            if constexpr (CG == 2) umma_commit_pair(tfull(buf));
            else umma_commit(tfull(buf));
          }
        }
      } else {
      for (int i = 0; units.get(i, t, kb0, kb1); ++i, ++tl) {
        const int buf = tl & 1;
        const uint32_t aph = (tl >> 1) & 1;
        mbar_wait(tempty(buf), aph ^ 1);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          mbar_wait(full(s), ph);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            if constexpr (CG == 2)
              umma_f16_pair(d_tmem, sdesc(a_addr + kk * 32), sdesc(b_addr + kk * 32), C::IDESC,
                            (kb != kb0 || kk != 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, sdesc(a_addr + kk * 32), sdesc(b_addr + kk * 32), C::IDESC,
                       (kb != kb0 || kk != 0) ? 1u : 0u);
          }
          // frees the smem stage (in both CTAs of a pair) when these MMAs complete
          if constexpr (CG == 2) umma_commit_pair(empty(s));
          else umma_commit(empty(s));
        }
        // accumulator ready (both CTAs' epilogues)
        if constexpr (CG == 2) umma_commit_pair(tfull(buf));
        else umma_commit(tfull(buf));
      }
      }
    }
  } else {
    // ---------------- epilogue warps 2 .. 2 + EPI_WARPS ----------------
    const int quad = warp & 3;       // TMEM lane quadrant this warp may access
    const int half = (warp - 2) / 4;  // which columns of the tile it takes
    uint32_t tl = 0;
    // rank 0's accumulator-empty barriers, addressed through the cluster window
    const uint32_t te0 = CG == 2 ? map_rank0(tempty(0)) : tempty(0);
    const uint32_t te1 = CG == 2 ? map_rank0(tempty(1)) : tempty(1);
    int t, kb0, kb1;
    uint32_t ch = 0;  // TF: accumulation chunks consumed
    for (int i = 0; units.get(i, t, kb0, kb1); ++i, ++tl) {
      const int buf = tl & 1;
      const uint32_t aph = (tl >> 1) & 1;
      int mi_, ni_;
      tile_coords(t, m_tiles, n_tiles, mi_, ni_);
      const int m0 = mi_ * BMT + (int)rank * BM, n0 = ni_ * BN;
      uint32_t taddr;
      int tbuf = buf;  // the accumulator buffer this tile's epilogue reads and then releases
      if constexpr (TF) {
        const uint32_t lanes = tmem_base + ((uint32_t)(quad * 32) << 16);
        // The tensor core's f32 accumulation loses accuracy with every MMA
        // chained into one accumulator (measured relative L2 against f64: 6e-5
        // at K = 5888 in one chain; 6.5e-7 with 8-k-block chunks; 2e-7 to
        // 4.4e-7 with 2-k-block chunks).  Each chunk (tf_chunk_end) starts a
        // fresh accumulator (four buffers in turn); these warps read it (this
        // warp's 64 columns), hand the buffer back at once and add it into
        // the tile sum in their registers with round-to-nearest f32 adds; the
        // sum goes into the last chunk's buffer for the epilogue below.
        float acc[64];  // this thread's row, this warp's 64 columns of the tile sum
        // one chunk into acc; every chunk but the tile's last hands its buffer back
        auto take = [&](bool first, bool last) {
          const int b = ch % NACC;
          mbar_wait(tfull(b), (ch / NACC) & 1);
          tc_fence_after();
          uint32_t a[32], a1[32];
          tmem_ld32(lanes + b * BN, a, 64 * half);
          tmem_ld32(lanes + b * BN, a1, 64 * half + 32);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            acc[j] = first ? __uint_as_float(a[j]) : acc[j] + __uint_as_float(a[j]);
            acc[32 + j] = first ? __uint_as_float(a1[j]) : acc[32 + j] + __uint_as_float(a1[j]);
          }
          if (!last) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (CG == 2) mbar_arrive_cluster(map_rank0(tempty(b)));
              else mbar_arrive(tempty(b));
            }
          }
          ++ch;
          return b;
        };
        int c1 = tf_chunk_end(kb0, kb1, K / 32);
        take(true, false);  // a tile has >= 3 chunks (one per segment at least)
        for (int c0 = c1; c0 < kb1; c0 = c1) {
          c1 = tf_chunk_end(c0, kb1, K / 32);
          tbuf = take(false, c1 >= kb1);
        }
        // the sum goes into the last chunk's buffer, kept until the epilogue ends
        const uint32_t sum = lanes + (uint32_t)tbuf * BN;
        {
          uint32_t o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(acc[j]);
          tmem_st32(sum + 64 * half, o);
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(acc[32 + j]);
          tmem_st32(sum + 64 * half + 32, o);
          tmem_wait_st();
          tc_fence_before();
        }
        // the sum's columns come from both warps of each lane quadrant; named
        // barrier 1 over the epilogue warps
        asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI_WARPS) : "memory");
        tc_fence_after();
        taddr = sum;
      } else {
        mbar_wait(tfull(buf), aph);
        tc_fence_after();
        taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * BN;
      }
      const int row = m0 + quad * 32 + lane;
      const bool row_ok = row < M;
      if (ep.mode == EPI_QKVG || ep.mode == EPI_CTXKV) {
#pragma unroll 1
        for (int c = 128 * half; c < BN; c += 256) {
          if (n0 + c >= N) break;
          Regs<128> R;
          uint32_t(&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&R.r[0]);
          uint32_t(&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&R.r[32]);
          uint32_t(&r2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&R.r[64]);
          uint32_t(&r3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&R.r[96]);
          tmem_ld32(taddr, r0, c);
          tmem_ld32(taddr, r1, c + 32);
          tmem_ld32(taddr, r2, c + 64);
          tmem_ld32(taddr, r3, c + 96);
          tmem_wait_ld();
          if (ep.mode == EPI_QKVG && ep.out_bf16) {
            // warp-collective: coalesced row segments through this warp's 4 KB buffer
            const int m_base = m0 + quad * 32;
            if (m_base < M)
              epi_head_staged(ep, m_base, lane, M, n0 + c, R,
                              reinterpret_cast<uint4*>(smem + C::OFF_EPI + (warp - 2) * 4096));
          } else if (row_ok) {
            epi_head<128>(ep, row, n0 + c, R);
          }
        }
      } else if (ep.mode == EPI_SWIGLU) {
#pragma unroll 1
        for (int c = 64 * half; c < BN; c += 128) {
          if (n0 + c >= N) break;
          Regs<64> R;
          uint32_t(&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&R.r[0]);
          uint32_t(&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&R.r[32]);
          tmem_ld32(taddr, r0, c);
          tmem_ld32(taddr, r1, c + 32);
          tmem_wait_ld();
          if (ep.out_bf16 && (ep.F % 32) == 0) {
            // warp-collective: 64-byte row segments through this warp's buffer
            const int m_base = m0 + quad * 32;
            if (m_base < M)
              epi_swiglu_staged(ep, m_base, lane, M, n0 + c, R,
                                reinterpret_cast<uint4*>(smem + C::OFF_EPI + (warp - 2) * 4096));
          } else if (row_ok) {
            epi_chunk_swiglu<Regs<64>, true>(ep, row, n0 + c, R);
          }
        }
      } else if (ep.mode == EPI_RESID && ep.x_tma) {
        // Gated residual x += gate * acc without reading x: each 32 x 32 chunk
        // of gate * acc goes to a 128B-swizzled shared-memory tile and one TMA
        // reduce-add folds it into x (also for K-splits: the adds are atomic).
        float* xb = reinterpret_cast<float*>(smem + C::OFF_EPI + (warp - 2) * 4096);
#pragma unroll 1
        for (int c = 32 * half; c < BN; c += 64) {
          if (n0 + c >= N) break;
          Regs<32> R;
          tmem_ld32(taddr, R.r, c);
          float g[32];
          if (ep.gate) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 gv = *reinterpret_cast<const float4*>(ep.gate + n0 + c + 4 * q);
              g[4 * q] = gv.x;
              g[4 * q + 1] = gv.y;
              g[4 * q + 2] = gv.z;
              g[4 * q + 3] = gv.w;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) g[q] = 1.f;
          }
          tmem_wait_ld();
          if (lane == 0) bulk_wait_read0();  // the previous reduce has read xb
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(xb + lane * 32 + ((q ^ (lane & 7)) << 2)) =
                make_float4(g[4 * q] * R(4 * q), g[4 * q + 1] * R(4 * q + 1), g[4 * q + 2] * R(4 * q + 2),
                            g[4 * q + 3] * R(4 * q + 3));
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&tmX, smem_u32(xb), n0 + c, m0 + quad * 32);
            bulk_commit();
          }
        }
      } else if (ep.mode == EPI_RESID) {
        // Gated residual x += gate * acc through a per-warp 32x32 shared-memory
        // transpose: lane l then owns column l, so every warp access to the f32
        // residual stream is 128 contiguous bytes of one row (coalesced RMW).
        float* stg = reinterpret_cast<float*>(smem + C::OFF_EPI) + (warp - 2) * (32 * 33);
#pragma unroll 1
        for (int c = 32 * half; c < BN; c += 64) {
          if (n0 + c >= N) break;
          Regs<32> R;
          tmem_ld32(taddr, R.r, c);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) stg[lane * 33 + i] = R(i);
          __syncwarp();
          const int n = n0 + c + lane;
          const bool col_ok = n < N;
          const float g = (ep.gate && col_ok) ? ep.gate[n] : 1.f;
          const int r0 = m0 + quad * 32;
          float* xc = ep.x + n;
          if (splits != 1) {  // K-split or stream-K partial products: atomic adds
#pragma unroll 8
            for (int i = 0; i < 32; ++i)
              if (col_ok && r0 + i < M) atomicAdd(xc + (long)(r0 + i) * N, g * stg[i * 33 + lane]);
          } else {
            float xv[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) xv[i] = (col_ok && r0 + i < M) ? xc[(long)(r0 + i) * N] : 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (col_ok && r0 + i < M) {
                const float rs = ep.row_scale ? ep.row_scale[r0 + i] : 1.f;
                xc[(long)(r0 + i) * N] = (xv[i] + g * stg[i * 33 + lane]) * rs;
              }
            }
          }
          __syncwarp();
        }
      } else {
#pragma unroll 1
        for (int c = 32 * half; c < BN; c += 64) {
          if (n0 + c >= N) break;
          Regs<32> R;
          tmem_ld32(taddr, R.r, c);
          tmem_wait_ld();
          if (row_ok) epi_chunk_store<32>(ep, row, n0 + c, R);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (TF) {
          if constexpr (CG == 2) mbar_arrive_cluster(map_rank0(tempty(tbuf)));
          else mbar_arrive(tempty(tbuf));
        } else {
          if constexpr (CG == 2) mbar_arrive_cluster(buf ? te1 : te0);
          else mbar_arrive(tempty(buf));
        }
      }
    }
  }

  // reduces issued by this thread have read their shared memory and completed
  if (warp >= 2 && lane == 0) bulk_wait0();
  __syncthreads();
  // a pair stays resident until neither CTA signals the other any more
  if constexpr (CG == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps (cached per buffer), launch.
// ---------------------------------------------------------------------------

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  if (!fn) throw Error(IRT_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

struct MapKey {
  const void* p;
  long rows, cols, ld;
  int box_rows;
  bool f32;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows && f32 == o.f32;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (std::hash<long>()(k.rows) * 31) ^ (std::hash<long>()(k.cols) * 131) ^
           (std::hash<long>()(k.ld) * 1313) ^ (size_t)k.box_rows ^ ((size_t)k.f32 << 20);
  }
};

// Operand map: bf16 {64, box_rows} boxes, or f32 {32, box_rows} (f32 = true);
// 128-byte rows with the 128-byte swizzle either way.
const CUtensorMap& tensor_map(const void* p, long rows, long cols, long ld, int box_rows, bool f32 = false) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  std::lock_guard<std::mutex> lk(mu);
  MapKey key{p, rows, cols, ld, box_rows, f32};
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  CUtensorMap m;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)ld * (f32 ? 4 : 2)};
  cuuint32_t box[2] = {(cuuint32_t)(f32 ? 32 : BK), (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = get_encode()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                            const_cast<void*>(p), gdim, gstride, box, estride,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(IRT_E_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  if (cache.size() > 4096) cache.clear();
  return cache.emplace(key, m).first->second;
}

// f32 2-D tensor map of the residual stream for the epilogue's TMA
// reduce-add: 32 x 32 box (128-byte rows), 128-byte swizzle.  Encoded per
// launch (a host-side table fill).
CUtensorMap tensor_map_resid(const float* p, long rows, long cols, long ld) {
  CUtensorMap m;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), gdim, gstride, box,
                            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(IRT_E_CUDA, "cuTensorMapEncodeTiled (f32) failed (" + std::to_string((int)r) + ")");
  return m;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Co-resident CTA pairs of gemm_kernel<BN, 2> on this device (cached).
template <int BN>
int max_pairs() {
  static int cached[32] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& n = cached[dev & 31];
  if (!n) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 1024);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = Cfg<BN, 2>::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, gemm_kernel<BN, 2, false>, &cfg) != cudaSuccess || c <= 0) {
      cudaGetLastError();
      c = num_sms() / 2;
    }
    n = c;
  }
  return n;
}

// TF: A and B are [A_hi | A_lo] / [B_hi | B_lo] f32 matrices of 2 K / taps and
// 2 K columns.  a_rows / b_rows > 0: the rows their tensor maps span (the
// rows that exist, zero padding included, so that no box is taller than its
// tensor; rows past them read as zero), else M / N.
template <int BN, int CG, bool TF>
void launch(const void* A, long lda, const void* B, long ldb, int M, int N, int K, int splits, const EpiParams& p,
            cudaStream_t s, long a_rows = 0, long b_rows = 0) {
  using C = Cfg<BN, CG>;
  static unsigned attr_mask = 0;  // per-device opt-in to the large dynamic smem
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_mask & (1u << (dev & 31)))) {
    IRT_CUDA(
        cudaFuncSetAttribute(gemm_kernel<BN, CG, TF>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_mask |= 1u << (dev & 31);
  }
  const long acols = TF ? 2L * (K / p.conv_taps) : K, bcols = TF ? 2L * K : K;
  // copies: the cache may be cleared
  const CUtensorMap ta = tensor_map(A, a_rows > 0 ? a_rows : M, acols, lda, BM, TF);
  const CUtensorMap tb = tensor_map(B, b_rows > 0 ? b_rows : N, bcols, ldb, C::B_ROWS, TF);
  // residual by TMA reduce-add (not for row-masked residuals)
  const bool xtma = p.mode == EPI_RESID && !p.row_scale && p.x && (N % 32) == 0 &&
                    (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 &&
                    (!p.gate || (reinterpret_cast<uintptr_t>(p.gate) & 15) == 0);
  const CUtensorMap tx = xtma ? tensor_map_resid(p.x, M, N, N) : ta;
  EpiParams pp = p;
  pp.x_tma = xtma ? 1 : 0;
  // stream-K (splits < 0) spreads the k-blocks over every available group
  const int units = splits < 0 ? (1 << 30) : ((M + BM * CG - 1) / (BM * CG)) * ((N + BN - 1) / BN) * splits;
  if constexpr (CG == 1) {
    const int grid = units < num_sms() ? units : num_sms();
    launch_pdl(gemm_kernel<BN, 1, TF>, dim3(grid), dim3(THREADS), C::SMEM, s, ta, tb, tx, M, N, K, splits, pp);
  } else {
    const int pairs = std::min(units, max_pairs<BN>());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    IRT_CUDA(cudaLaunchKernelEx(&cfg, gemm_kernel<BN, 2, TF>, ta, tb, tx, M, N, K, splits, pp));
  }
  IRT_CHECK_LAUNCH();
}

// CTA pairs (cta_group::2) for every GEMM with at least two 128-row tiles,
// unless IRT_GEMM_PAIRS=0.
bool use_pairs(int M) {
  static const bool on = [] {
    const char* e = std::getenv("IRT_GEMM_PAIRS");
    return !(e && e[0] == '0');
  }();
  return on && M >= 2 * BM;
}

// Fraction of the SM-slots of the last wave that do useful work.
double wave_eff(long units, int sms) {
  long waves = (units + sms - 1) / sms;
  return waves ? (double)units / (double)(waves * sms) : 0.0;
}

// Tail split (Units, splits == -2) of a residual GEMM: k-block time per group
// of whole tiles, (full rounds + 1) * kb, against full rounds * kb + the tail
// span + one k-block for the extra accumulator hand-off; taken at a predicted
// gain above 3 %.  Measured (CUDA events, the DiT layer GEMMs): W2 -2.9 % at
// 54,504 rows and -1.9 % at 27,252 (the config-4 steps), Wo within 1 %; W2 at
// 6,800 rows (a predicted 2 % gain) ran 3 % slower and stays on whole tiles.
// force: take it wherever some tile would be shared (tests).
bool tail_split_pays(long tiles, int groups, int kb, bool force) {
  const long full_rounds = tiles / groups, tail = tiles - full_rounds * groups;
  if (tail == 0) return false;
  const long span = std::max<long>(TAIL_MIN_SPAN, (tail * kb + groups - 1) / groups);
  if (span >= kb) return false;  // no tile would be shared
  const double whole = (double)(full_rounds + 1) * kb;
  const double split = (double)full_rounds * kb + span + 1.0;
  return force || split < 0.97 * whole;
}

}  // namespace tc

// 2-D tensor map of {32, 32}-element boxes for epilogue staging tiles: f32
// rows of 128 bytes with the 128-byte swizzle, or bf16 rows of 64 bytes with
// the 64-byte swizzle.
CUtensorMap tma_map_tile32(const void* p, bool f32, long rows, long cols, long ld) {
  CUtensorMap m;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)ld * (f32 ? 4 : 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = tc::get_encode()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                const_cast<void*>(p), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(IRT_E_CUDA, "cuTensorMapEncodeTiled (tile32) failed (" + std::to_string((int)r) + ")");
  return m;
}

// The rows o = q * s + r of a [q_rows * s, cols] f32 / bf16 matrix seen as 3-D
// (column, r, q): {32, 1, 32} boxes select 32 rows of one phase r that are s
// rows apart (a ConvTranspose output phase), swizzled as tma_map_tile32.
CUtensorMap tma_map_tile32_phased(const void* p, bool f32, long q_rows, long cols, int s) {
  CUtensorMap m;
  const cuuint64_t esz = f32 ? 4 : 2;
  cuuint64_t gdim[3] = {(cuuint64_t)cols, (cuuint64_t)s, (cuuint64_t)q_rows};
  cuuint64_t gstride[2] = {(cuuint64_t)cols * esz, (cuuint64_t)s * cols * esz};
  cuuint32_t box[3] = {32, 1, 32};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = tc::get_encode()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                const_cast<void*>(p), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(IRT_E_CUDA, "cuTensorMapEncodeTiled (phased tile32) failed (" + std::to_string((int)r) + ")");
  return m;
}

// bf16 2-D tensor map with a {64, box_rows} box and 128-byte swizzle (cached).
const CUtensorMap& tma_map_bf16(const void* p, long rows, long cols, long ld, int box_rows) {
  return tc::tensor_map(p, rows, cols, ld, box_rows);
}

bool gemm_tc_supported(const EpiParams& p, int K, long lda, long ldb, const void* A, const void* B) {
  if (K < tc::BK || (K % 8) || (lda % 8) || (ldb % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) return false;
  if (p.M < tc::BM || p.N < 128) return false;
  if ((p.mode == EPI_QKVG || p.mode == EPI_CTXKV) && (p.hd != 128 || (p.Dq % 128))) return false;
  if (p.mode == EPI_SWIGLU && (p.N % 64)) return false;
  return true;
}

namespace tc {
template <bool TF>
void gemm_tc_impl(const void* A, long lda, const void* B, long ldb, int M, int N, int K, const EpiParams& p,
                  cudaStream_t s, long a_rows = 0, long b_rows = 0) {
  // Tile width 256 wherever the epilogue allows it.  Narrower tiles fill the
  // last wave better at small M but re-read A from L2 twice as often, and
  // measured slower at every M tried (750-54,504 rows).
  // Work slots are SMs (1-CTA tiles of 128 rows) or SM pairs (256 rows).
  const bool pairs = tc::use_pairs(M);
  const int sms = pairs ? tc::num_sms() / 2 : tc::num_sms();
  const int bmt = pairs ? 2 * tc::BM : tc::BM;
  const long mt = (M + bmt - 1) / bmt;
  const long t256 = mt * ((N + 255) / 256), t128 = mt * ((N + 127) / 128);
  bool use256 = N >= 256 && !TF;  // TF: 128-column tiles (the tile sums need the TMEM)
  if ((p.mode == EPI_QKVG || p.mode == EPI_CTXKV) && (p.Dq % 256)) use256 = false;
  // K-splits for the additive residual epilogue (partial products are
  // reduce-added into x): the split count that best fills the last wave of
  // work units, each extra split charged 0.08 of wave efficiency for its
  // read-modify-write of the residual tile and its shorter main loop; each
  // split keeps >= 8 k-blocks (512 of K), at most 6 splits.  When no split
  // pays but the last wave is still poorly filled and K is long (>= 64
  // k-blocks, so a group's span crosses few tile boundaries), the GEMM runs
  // stream-K instead (splits = -1, see Units).  Measured: stream-K is +9 % on
  // W2 at 3,400 rows and slower than the split rule wherever that one splits.
  int splits = 1;
  const long tiles = use256 ? t256 : t128;
  if (!TF && p.mode == EPI_RESID && !p.row_scale) {
    const int kb = (K + tc::BK - 1) / tc::BK;
    const double eff1 = tc::wave_eff(tiles, sms);
    double best = eff1;
    for (int sp = 2; sp <= 6 && kb / sp >= 8; ++sp) {
      const int kpb = (kb + sp - 1) / sp;
      const int real = (kb + kpb - 1) / kpb;  // no empty split
      const double score = tc::wave_eff(tiles * real, sms) - 0.08 * (real - 1);
      if (score > best) {
        best = score;
        splits = real;
      }
    }
    if (splits == 1 && eff1 < 0.8 && kb >= 64 && tiles * kb >= 8L * sms) splits = -1;
    // Otherwise a tail split when the last wave is partly empty (by TMA
    // reduce-add only: the read-modify-write path is not additive).
    // IRT_TAIL_SPLIT=0 turns it off, =1 takes it wherever a tile is shared.
    const char* ts = std::getenv("IRT_TAIL_SPLIT");
    const bool ts_off = ts && ts[0] == '0', ts_force = ts && ts[0] == '1';
    const bool xtma_ok = p.x && (N % 32) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 &&
                         (!p.gate || (reinterpret_cast<uintptr_t>(p.gate) & 15) == 0);
    if (splits == 1 && xtma_ok && !ts_off && tc::tail_split_pays(tiles, sms, kb, ts_force)) splits = -2;
  }
  if constexpr (TF) {
    if (pairs) tc::launch<128, 2, true>(A, lda, B, ldb, M, N, K, splits, p, s, a_rows, b_rows);
    else tc::launch<128, 1, true>(A, lda, B, ldb, M, N, K, splits, p, s, a_rows, b_rows);
  } else if (pairs) {
    if (use256) tc::launch<256, 2, false>(A, lda, B, ldb, M, N, K, splits, p, s);
    else tc::launch<128, 2, false>(A, lda, B, ldb, M, N, K, splits, p, s);
  } else {
    if (use256) tc::launch<256, 1, false>(A, lda, B, ldb, M, N, K, splits, p, s);
    else tc::launch<128, 1, false>(A, lda, B, ldb, M, N, K, splits, p, s);
  }
}

// hi = a rounded to the nearest tf32 (ties away from zero; the 13 low mantissa
// bits cleared), lo = a - hi (exact in f32).  Inf / NaN pass through as hi.
__device__ __forceinline__ float tf32_hi(float a) {
  const uint32_t u = __float_as_uint(a);
  if ((u & 0x7f800000u) == 0x7f800000u) return a;
  return __uint_as_float((u + 0x1000u) & 0xffffe000u);
}

// Row m of A [M, K] (leading dimension lda) -> row m of A2 = [A_hi | A_lo]
// [M, 2 * Kp], columns K..Kp-1 of each half zero.  Four columns per thread.
__global__ void split_tf32_kernel(const float* __restrict__ A, long lda, int M, int K, float* __restrict__ A2,
                                  int Kp) {
  pdl_wait();
  pdl_trigger();
  const int q = Kp / 4;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)M * q) return;
  const int m = (int)(i / q), k = (int)(i - (long)m * q) * 4;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  if (k + 3 < K) {
    a = *reinterpret_cast<const float4*>(A + (long)m * lda + k);
  } else {
    const float* r = A + (long)m * lda;
    if (k < K) a.x = r[k];
    if (k + 1 < K) a.y = r[k + 1];
    if (k + 2 < K) a.z = r[k + 2];
  }
  const float4 h = make_float4(tf32_hi(a.x), tf32_hi(a.y), tf32_hi(a.z), tf32_hi(a.w));
  float* o = A2 + (long)m * 2 * Kp + k;
  *reinterpret_cast<float4*>(o) = h;
  *reinterpret_cast<float4*>(o + Kp) = make_float4(a.x - h.x, a.y - h.y, a.z - h.z, a.w - h.w);
}
}  // namespace tc

void gemm_tc(const bf16* A, long lda, const bf16* B, long ldb, int M, int N, int K, const EpiParams& p,
             cudaStream_t s) {
  tc::gemm_tc_impl<false>(A, lda, B, ldb, M, N, K, p, s);
}

void gemm_tc_tf32x3(const float* A2, long lda2, const float* B2, long ldb2, int M, int N, int Kp, const EpiParams& p,
                    cudaStream_t s, long a_rows, long b_rows) {
  if (Kp % 32 || p.conv_taps < 1 || (Kp / 32) % p.conv_taps)
    throw Error(IRT_E_INVALID_ARG, "gemm_tc_tf32x3: K must be taps x a multiple of 32");
  tc::gemm_tc_impl<true>(A2, lda2, B2, ldb2, M, N, Kp, p, s, a_rows, b_rows);
}

void split_tf32(const float* A, long lda, int M, int K, float* A2, int Kp, cudaStream_t s) {
  if (M <= 0) return;
  if (Kp % 32 || Kp < K || (lda % 4) || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(A2) & 15))
    throw Error(IRT_E_INVALID_ARG, "split_tf32: unaligned operand");
  const long n = (long)M * (Kp / 4);
  launch_pdl(tc::split_tf32_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, A, lda, M, K, A2, Kp);
  IRT_CHECK_LAUNCH();
}

}  // namespace irt
