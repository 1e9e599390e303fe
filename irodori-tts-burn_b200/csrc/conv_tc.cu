// Implicit-GEMM tcgen05 convolutions for the DACVAE decoder in bf16 mode
// (src/codec/decoder.rs:17-126, layers.rs:27-75).
//
// Activations are time-major bf16 rows [R, C] (channels contiguous).  A batch
// is laid out as ONE time axis: every utterance is a run of latent frames with
// GAP_FRAMES all-zero frames before, between and after the runs (the row
// count at a decoder level is frames x upsampling so far).  The widest
// receptive field at any level (kernel 7, dilation 9: 27 rows; ConvTranspose:
// 1 input row) stays inside those zero rows, so "zero padding per utterance"
// is just reading zero rows, and ragged batches cost nothing extra.  Every
// epilogue writes exact zeros into gap rows; Snake(0) = 0 keeps them zero.
//
// conv1d (kernel k, dilation d, padding p):
//   Y[t, co] = sum_tap sum_ci X[t + tap*d - p, ci] * W[co, ci, tap]
//   = GEMM with M = t, N = co, K = (tap, ci); the A tile of k-block (tap, c0)
//   is one TMA load of rows shifted by tap*d - p (rows outside [0, R) read the
//   TMA zero fill).
// ConvTranspose1d (kernel 2s, stride s, padding ceil(s/2), even or odd s >= 2):
//   output o with o + pad = q*s + r receives exactly two taps,
//   Y[o] = X[q] W[:, :, r] + X[q-1] W[:, :, r+s]; per phase r this is a 2-tap
//   conv over q' = q - [r < pad] in [0, R_in), whose output rows are strided
//   by s.  The phases are one more tile dimension of the same kernel.
//
// Persistent warp-specialised CTA (320 threads): warp 0 TMA producer, warp 1
// TMEM allocator + tcgen05.mma issuer, warps 2..9 epilogue (two per TMEM lane
// quadrant, alternate 32-column chunks) through a per-warp 32x33
// shared-memory transpose so that every global access of a warp is one
// contiguous run of a row (lane = output channel).  Two TMEM accumulators let
// the epilogue of one tile overlap the MMAs of the next.  Every mbarrier wait
// is bounded (watchdog flag, no hang).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "codec.hpp"
#include "tc_common.cuh"

namespace irt {

// bf16 2-D tensor map, {64, box_rows} box, 128-byte swizzle (gemm_tc.cu).
const CUtensorMap& tma_map_bf16(const void* p, long rows, long cols, long ld, int box_rows);
// {32, 32} boxes: f32 with the 128-byte swizzle or bf16 with the 64-byte swizzle (gemm_tc.cu).
CUtensorMap tma_map_tile32(const void* p, bool f32, long rows, long cols, long ld);
// the same tiles over the rows q * s + r of one phase r, as (column, r, q) (gemm_tc.cu).
CUtensorMap tma_map_tile32_phased(const void* p, bool f32, long q_rows, long cols, int s);

namespace ctc {

using namespace tcx;

// warps 0 (TMA) and 1 (MMA) + EPI_WARPS epilogue warps; two epilogue warps
// share each TMEM lane quadrant and split the 32-column chunks between them.
constexpr int BM = 128, BK = 64, EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t A_BYTES = BM * BK * 2;

// Per epilogue warp: a 32 x 33 f32 transpose buffer (ConvTranspose path), or
// the staging tiles of the stride-1 path -- 32 x 32 f32 (128-byte rows,
// 128-byte swizzle) then 32 x 32 bf16 (64-byte rows, 64-byte swizzle), both
// stored by TMA.  6 KB keeps every f32 tile 1024-byte aligned.  (A second
// set per warp, so that one chunk's stores drain while the next is computed,
// measured no faster and cost the 192-wide layers a pipeline stage.)
constexpr uint32_t EPI_SET = 6144;

// Residual stride-1 convolutions (the ResUnits' 1x1, x += conv) use a ring of
// RES_SETS f32 staging tiles per epilogue warp: each 32 x 32 residual chunk is
// loaded by TMA into a tile two chunks ahead, the output overwrites it in
// place and leaves by TMA store from the same tile; one bf16 tile per warp
// stages the Snake output.  The ring takes 14 KB per warp, so these launches
// run with the pipeline stages that fit beside it (2-4; their K is 2-12
// k-blocks and the MMAs are not what bounds them).
constexpr int RES_SETS = 3;
constexpr uint32_t RES_SLOT = RES_SETS * 4096 + 2048;
constexpr uint32_t SMEM_MAX = 232448;  // 227 KB opt-in per CTA

// Stride-1 convolutions with k > 1 (the ResUnits' dilated k7, the stem) stage
// the input rows of a unit ONCE per 64-channel block: one TMA box of
// 128 + (k - 1) * dilation rows (the unit's rows with the halo every tap
// needs) in a two-slot ring, and tap t's MMAs read it through a descriptor
// that starts t * dilation rows in (the 128-byte swizzle is a function of the
// shared-memory address, and the box is written 1024-byte aligned, so a
// row-shifted view reads the rows it names).  The pipeline stages then carry
// only the weight tiles: one input load per channel block instead of one per
// tap.
constexpr int HALO_ROWS_MAX = 184;
constexpr uint32_t HALO_SLOT = HALO_ROWS_MAX * 128;

// VAR: 0 plain, 1 residual ring (1x1, x += conv), 2 halo (stride 1, k > 1)
template <int BN, int VAR>
struct Cfg {
  static constexpr uint32_t EPI_SLOT = VAR == 1 ? RES_SLOT : EPI_SET;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = VAR == 2 ? B_BYTES : A_BYTES + B_BYTES;
  static constexpr uint32_t HALO_BYTES = VAR == 2 ? 2 * HALO_SLOT : 0;
  // barriers: full / empty per stage, two accumulator pairs, the TMEM slot,
  // the halo ring's (256 B), then the residual ring's (EPI_WARPS x RES_SETS)
  static constexpr uint32_t BAR_BYTES = VAR == 1 ? 512 : 256;
  static constexpr uint32_t STAGE_BUDGET =
      VAR == 0 ? 176 * 1024 : SMEM_MAX - 1024 - EPI_WARPS * EPI_SLOT - HALO_BYTES - BAR_BYTES;
  static constexpr int STAGES = STAGE_BUDGET / STAGE_BYTES > 8 ? 8 : STAGE_BUDGET / STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
  // second accumulator at a power-of-two column offset
  static constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;
  // alignment slack | stages | halo slots | epilogue slots (1024-aligned) | barriers
  static constexpr uint32_t OFF_HALO = STAGES * STAGE_BYTES;
  static constexpr uint32_t OFF_EPI = OFF_HALO + HALO_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_EPI + EPI_WARPS * EPI_SLOT;
  static_assert(STAGES >= (VAR == 0 ? 3 : 2), "pipeline stages");
  static_assert(VAR != 2 || (OFF_HALO % 1024) == 0, "halo slots must be 1024-byte aligned");
  static_assert(2 * STAGES + 5 + 4 <= 32, "barrier region");
  static constexpr size_t SMEM = 1024 + (size_t)OFF_BAR + BAR_BYTES;
  static_assert(SMEM <= SMEM_MAX, "shared memory");
  static constexpr uint32_t IDESC = idesc_bf16(BM, BN);
  static_assert((OFF_EPI % 1024) == 0 && (EPI_SLOT % 1024) == 0, "epilogue tiles must be 1024-byte aligned");
  static_assert(32 * 33 * 4 <= EPI_SET, "transpose buffer fits a slot");
};

// A-operand row offset of tap `tap` for output phase `phase`.
__device__ __forceinline__ int a_row_off(const ConvTcArgs& a, int phase, int tap) {
  return a.convt ? ((phase < a.pad ? 1 : 0) - tap) : (tap * a.dil - a.pad);
}
// Output row of GEMM row q in phase `phase`.
__device__ __forceinline__ int out_row(const ConvTcArgs& a, int phase, int q) {
  return a.convt ? (q + (phase < a.pad ? 1 : 0)) * a.stride + phase - a.pad : q;
}

// Snake with a precomputed 1 / (alpha + 1e-9); the hardware sine (MUFU) is
// ample for a bf16 output.
__device__ __forceinline__ float snake_inv(float v, float al, float inv) {
  const float s = __sinf(al * v);
  return v + s * s * inv;
}

template <int BN, int VAR>
__global__ void __launch_bounds__(THREADS, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmP,
                   const __grid_constant__ ConvTcArgs a) {
  using C = Cfg<BN, VAR>;
  constexpr bool RING = VAR == 1, HALO = VAR == 2;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  uint64_t* rbars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR + 256);  // RING: [warp][set]
  uint64_t* hbars = bars + 2 * STAGES + 5;  // HALO: full[2], empty[2]
  uint8_t* epi = smem + C::OFF_EPI;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m_tiles = (a.rows_in + BM - 1) / BM, n_tiles = a.cout / BN;
  const int units = m_tiles * a.phases * n_tiles;
  const int kpt = a.cin_pad / BK;  // k-blocks per tap
  const int kbs = a.taps * kpt;

  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto tfull = [&](int b) { return smem_u32(&bars[2 * STAGES + b]); };
  auto tempty = [&](int b) { return smem_u32(&bars[2 * STAGES + 2 + b]); };
  // unit -> (m tile, phase, n tile); n innermost, then phase, so CTAs running
  // at the same time share the A rows of one m tile through L2.
  auto unit_coords = [&](int u, int& m_idx, int& phase, int& n_idx) {
    n_idx = u % n_tiles;
    const int r = u / n_tiles;
    phase = r % a.phases;
    m_idx = r / a.phases;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), EPI_WARPS);
    }
    if constexpr (RING)
      for (int i = 0; i < EPI_WARPS * RES_SETS; ++i) mbar_init(smem_u32(&rbars[i]), 1);
    if constexpr (HALO)
      for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&hbars[i]), 1);
    mbar_fence_init();
    prefetch_map(&tmA);
    prefetch_map(&tmB);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the prologue above may overlap the previous kernel; operands are read only now
  pdl_wait();
  pdl_trigger();

  // HALO: rows of one staged input block (the unit's 128 plus every tap's shift)
  const int halo_rows = BM + (a.taps - 1) * a.dil;
  auto hfull = [&](int i) { return smem_u32(&hbars[i]); };
  auto hempty = [&](int i) { return smem_u32(&hbars[2 + i]); };
  uint8_t* halo = smem + C::OFF_HALO;

  if (HALO && warp == 0) {
    // ---------------- TMA producer (halo staging) ----------------
    if (lane == 0) {
      uint32_t it = 0, hit = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int mi, ph, ni;
        unit_coords(u, mi, ph, ni);
        const int m0 = mi * BM, n0 = ni * BN;
        for (int cb = 0; cb < kpt; ++cb, ++hit) {
          const int hs = hit & 1;
          mbar_wait(hempty(hs), ((hit >> 1) & 1) ^ 1);
          mbar_expect_tx(hfull(hs), (uint32_t)halo_rows * 128);
          tma_load_2d(smem_u32(halo + hs * HALO_SLOT), &tmA, hfull(hs), cb * BK, m0 - a.pad);
          for (int tap = 0; tap < a.taps; ++tap, ++it) {
            const int s = it % STAGES;
            mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1);
            mbar_expect_tx(full(s), C::STAGE_BYTES);
            tma_load_2d(smem_u32(tiles + s * C::STAGE_BYTES), &tmB, full(s), tap * a.cin_pad + cb * BK, n0);
          }
        }
      }
    }
  } else if (HALO && warp == 1) {
    // ---------------- MMA issuer (halo staging) ----------------
    if (lane == 0) {
      uint32_t it = 0, hit = 0, tl = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
        const int buf = tl & 1;
        mbar_wait(tempty(buf), ((tl >> 1) & 1) ^ 1);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::ACC_STRIDE;
        for (int cb = 0; cb < kpt; ++cb, ++hit) {
          const int hs = hit & 1;
          // input channels past cin are zero padding: skip their MMAs
          const int nkk = min(BK / 16, (a.cin - cb * BK + 15) / 16);
          mbar_wait(hfull(hs), (hit >> 1) & 1);
          tc_fence_after();
          const uint32_t h_addr = smem_u32(halo + hs * HALO_SLOT);
          for (int tap = 0; tap < a.taps; ++tap, ++it) {
            const int s = it % STAGES;
            mbar_wait(full(s), (it / STAGES) & 1);
            tc_fence_after();
            const uint32_t a_addr = h_addr + (uint32_t)(tap * a.dil) * 128u;  // rows shifted by the tap
            const uint32_t b_addr = smem_u32(tiles + s * C::STAGE_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              if (kk < nkk)
                umma_f16(d_tmem, sdesc_kmajor(a_addr + kk * 32), sdesc_kmajor(b_addr + kk * 32), C::IDESC,
                         (cb | tap | kk) ? 1u : 0u);
            umma_commit(empty(s));  // frees the weight stage when these MMAs complete
          }
          umma_commit(hempty(hs));  // frees the staged input block
        }
        umma_commit(tfull(buf));  // accumulator ready
      }
    }
  } else if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int mi, ph, ni;
        unit_coords(u, mi, ph, ni);
        const int m0 = mi * BM, n0 = ni * BN;
        const int brow = ph * a.cout + n0;
        for (int kb = 0; kb < kbs; ++kb, ++it) {
          const int tap = kb / kpt, c0 = (kb - tap * kpt) * BK;
          const int s = it % STAGES;
          const uint32_t par = (it / STAGES) & 1;
          mbar_wait(empty(s), par ^ 1);
          uint8_t* a_dst = tiles + s * C::STAGE_BYTES;
          mbar_expect_tx(full(s), C::STAGE_BYTES);
          tma_load_2d(smem_u32(a_dst), &tmA, full(s), c0, m0 + a_row_off(a, ph, tap));
          tma_load_2d(smem_u32(a_dst + A_BYTES), &tmB, full(s), tap * a.cin_pad + c0, brow);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
        const int buf = tl & 1;
        mbar_wait(tempty(buf), ((tl >> 1) & 1) ^ 1);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::ACC_STRIDE;
        for (int kb = 0; kb < kbs; ++kb, ++it) {
          const int s = it % STAGES;
          // input channels past cin are zero padding (the TMA zero fill times
          // zero weights): the last k-block of a tap issues only the MMAs that
          // cover real channels (96 channels: 2 of 4 in the second block)
          const int c0 = (kb % kpt) * BK;
          const int nkk = min(BK / 16, (a.cin - c0 + 15) / 16);
          mbar_wait(full(s), (it / STAGES) & 1);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            if (kk < nkk)
              umma_f16(d_tmem, sdesc_kmajor(a_addr + kk * 32), sdesc_kmajor(b_addr + kk * 32), C::IDESC,
                       (kb | kk) ? 1u : 0u);
          umma_commit(empty(s));  // frees the stage when these MMAs complete
        }
        umma_commit(tfull(buf));  // accumulator ready
      }
    }
  } else {
    // ---------------- epilogue warps 2 .. 2 + EPI_WARPS ----------------
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int half = (warp - 2) / 4;        // which 32-column chunks it takes
    uint8_t* slot = epi + (warp - 2) * C::EPI_SLOT;
    if constexpr (RING) {
      // Residual 1x1 convolutions (the launcher takes RING only for stride-1,
      // x += conv): thread = output row as below, the residual chunk read from
      // this warp's ring tile (see Cfg).  The warp's chunks are numbered
      // g = 0, 1, ...: unit i = g / npu of this CTA, column 32 * half + 64 * (g % npu).
      const int npu = BN > 32 * half ? (BN - 32 * half + 63) / 64 : 0;
      const int my_units = (int)blockIdx.x < units ? (units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
      const int nchunks = npu * my_units;
      uint64_t* rb = rbars + (warp - 2) * RES_SETS;
      uint8_t* ps = slot + RES_SETS * 4096;  // bf16 [32][32], 64-byte swizzle
      // lane 0: residual chunk g (32 rows x 32 f32, 128-byte swizzle) into its ring tile
      auto res_load = [&](int g) {
        const int i = g / npu;
        int mi, ph, ni;
        unit_coords((int)blockIdx.x + i * (int)gridDim.x, mi, ph, ni);
        const int set = g % RES_SETS;
        const uint32_t bar = smem_u32(&rb[set]);
        mbar_expect_tx(bar, 4096);
        tma_load_2d(smem_u32(slot + set * 4096), &tmX, bar, ni * BN + 32 * half + 64 * (g - i * npu),
                    mi * BM + quad * 32);
      };
      if (lane == 0)
        for (int g = 0; g < RES_SETS - 1 && g < nchunks; ++g) res_load(g);
      int g = 0;
      uint32_t tl = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
        int mi, ph, ni;
        unit_coords(u, mi, ph, ni);
        const int m0 = mi * BM, n0 = ni * BN;
        const int buf = tl & 1;
        const int q0 = m0 + quad * 32;
        const int row = q0 + lane;
        const bool valid = row < a.rows_in && a.frame_src[row / a.out_scale] >= 0;
        mbar_wait(tfull(buf), (tl >> 1) & 1);
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * C::ACC_STRIDE;
#pragma unroll 1
        for (int c = 32 * half; c < BN; c += 64, ++g) {
          uint32_t r[32];
          tmem_ld32(taddr + c, r);
          // the previous chunk's stores have read their tiles, so its ring
          // tile takes the residual chunk two ahead
          if (lane == 0) {
            bulk_wait_read0();
            if (g + RES_SETS - 1 < nchunks) res_load(g + RES_SETS - 1);
          }
          __syncwarp();
          tmem_wait_ld();
          const int set = g % RES_SETS;
          mbar_wait(smem_u32(&rb[set]), (uint32_t)(g / RES_SETS) & 1);
          uint8_t* xs = slot + set * 4096;  // residual in, f32 output out (same layout)
          const float* bp = a.bias ? a.bias + n0 + c : nullptr;
          const float* ap = a.alpha ? a.alpha + n0 + c : nullptr;
          const float* ip = a.alpha ? a.alpha_inv + n0 + c : nullptr;
#pragma unroll
          for (int m = 0; m < 4; ++m) {  // 8 columns: one 16-byte chunk of the bf16 row
            float v[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int k = 2 * m + h;  // float4 group: columns 4k .. 4k + 3
              float4* xp = reinterpret_cast<float4*>(xs + lane * 128 + ((k ^ (lane & 7)) << 4));
              const float4 xr = *xp;
              const float4 b4 = bp ? reinterpret_cast<const float4*>(bp)[k] : make_float4(0.f, 0.f, 0.f, 0.f);
              float w0 = __uint_as_float(r[4 * k]) + b4.x + xr.x, w1 = __uint_as_float(r[4 * k + 1]) + b4.y + xr.y;
              float w2 = __uint_as_float(r[4 * k + 2]) + b4.z + xr.z, w3 = __uint_as_float(r[4 * k + 3]) + b4.w + xr.w;
              if (!valid) w0 = w1 = w2 = w3 = 0.f;
              *xp = make_float4(w0, w1, w2, w3);
              if (ap) {
                const float4 al = reinterpret_cast<const float4*>(ap)[k];
                const float4 in = reinterpret_cast<const float4*>(ip)[k];
                w0 = snake_inv(w0, al.x, in.x);
                w1 = snake_inv(w1, al.y, in.y);
                w2 = snake_inv(w2, al.z, in.z);
                w3 = snake_inv(w3, al.w, in.w);
              }
              v[4 * h] = w0;
              v[4 * h + 1] = w1;
              v[4 * h + 2] = w2;
              v[4 * h + 3] = w3;
            }
            if (a.p) {
              uint4 pk;
              pk.x = pack_bf16x2(v[0], v[1]);
              pk.y = pack_bf16x2(v[2], v[3]);
              pk.z = pack_bf16x2(v[4], v[5]);
              pk.w = pack_bf16x2(v[6], v[7]);
              *reinterpret_cast<uint4*>(ps + lane * 64 + ((m ^ ((lane >> 1) & 3)) << 4)) = pk;
            }
          }
          fence_proxy_async();  // generic-proxy smem writes -> visible to the TMA stores
          __syncwarp();
          if (lane == 0 && q0 < a.rows_out) {  // rows past the end are clipped by the TMA unit
            tma_store_2d(&tmX, smem_u32(xs), n0 + c, q0);
            if (a.p) tma_store_2d(&tmP, smem_u32(ps), n0 + c, q0);
            bulk_commit();
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty(buf));
      }
      if (lane == 0) bulk_wait0();  // every store of this warp has completed
    } else if (!a.convt || a.ct_tma) {
      // Stride-1 convolutions without a residual (output row = GEMM row), and
      // ConvTranspose phases whose output rows o = q * stride + r leave by 3-D
      // TMA stores (column, r, q): thread = GEMM row.  Each 32 x 32 chunk
      // leaves through this warp's staging tiles by TMA stores (f32 stream,
      // bf16 Snake output).  Gap rows are written as exact zeros.  (Residual
      // stride-1 convolutions take the ring path above.)
      uint32_t tl = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
        int mi, ph, ni;
        unit_coords(u, mi, ph, ni);
        const int m0 = mi * BM, n0 = ni * BN;
        const int buf = tl & 1;
        const int q0 = m0 + quad * 32;
        const int row = q0 + lane;
        const bool ok = row < a.rows_in;
        // ConvTranspose: output row of GEMM row q in this phase is q * stride + rph
        const int rph = a.convt ? (ph < a.pad ? a.stride : 0) + ph - a.pad : 0;
        const int orow = a.convt ? row * a.stride + rph : row;
        const bool valid = ok && a.frame_src[orow / a.out_scale] >= 0;
        const int qlim = a.convt ? a.rows_in : a.rows_out;
        mbar_wait(tfull(buf), (tl >> 1) & 1);
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * C::ACC_STRIDE;
#pragma unroll 1
        for (int c = 32 * half; c < BN; c += 64) {
          uint32_t r[32];
          tmem_ld32(taddr + c, r);
          tmem_wait_ld();
          // the staging tiles: the previous chunk's stores have read them
          uint8_t* xs = slot;         // f32 [32][32], 128-byte swizzle
          uint8_t* ps = slot + 4096;  // bf16 [32][32], 64-byte swizzle
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          const float* bp = a.bias ? a.bias + n0 + c : nullptr;
          const float* ap = a.alpha ? a.alpha + n0 + c : nullptr;
          const float* ip = a.alpha ? a.alpha_inv + n0 + c : nullptr;
#pragma unroll
          for (int m = 0; m < 4; ++m) {  // 8 columns: one 16-byte chunk of the bf16 row
            float v[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int k = 2 * m + h;  // float4 group: columns 4k .. 4k + 3
              const float4 b4 = bp ? reinterpret_cast<const float4*>(bp)[k] : make_float4(0.f, 0.f, 0.f, 0.f);
              float w0 = __uint_as_float(r[4 * k]) + b4.x, w1 = __uint_as_float(r[4 * k + 1]) + b4.y;
              float w2 = __uint_as_float(r[4 * k + 2]) + b4.z, w3 = __uint_as_float(r[4 * k + 3]) + b4.w;
              if (!valid) w0 = w1 = w2 = w3 = 0.f;
              if (a.x)
                *reinterpret_cast<float4*>(xs + lane * 128 + ((k ^ (lane & 7)) << 4)) = make_float4(w0, w1, w2, w3);
              if (ap) {
                const float4 al = reinterpret_cast<const float4*>(ap)[k];
                const float4 in = reinterpret_cast<const float4*>(ip)[k];
                w0 = snake_inv(w0, al.x, in.x);
                w1 = snake_inv(w1, al.y, in.y);
                w2 = snake_inv(w2, al.z, in.z);
                w3 = snake_inv(w3, al.w, in.w);
              }
              v[4 * h] = w0;
              v[4 * h + 1] = w1;
              v[4 * h + 2] = w2;
              v[4 * h + 3] = w3;
            }
            if (a.p) {
              uint4 pk;
              pk.x = pack_bf16x2(v[0], v[1]);
              pk.y = pack_bf16x2(v[2], v[3]);
              pk.z = pack_bf16x2(v[4], v[5]);
              pk.w = pack_bf16x2(v[6], v[7]);
              *reinterpret_cast<uint4*>(ps + lane * 64 + ((m ^ ((lane >> 1) & 3)) << 4)) = pk;
            }
          }
          fence_proxy_async();  // generic-proxy smem writes -> visible to the TMA stores
          __syncwarp();
          if (lane == 0 && q0 < qlim) {  // rows past the end are clipped by the TMA unit
            if (a.convt) {
              if (a.x) tma_store_3d(&tmX, smem_u32(xs), n0 + c, rph, q0);
              if (a.p) tma_store_3d(&tmP, smem_u32(ps), n0 + c, rph, q0);
            } else {
              if (a.x) tma_store_2d(&tmX, smem_u32(xs), n0 + c, q0);
              if (a.p) tma_store_2d(&tmP, smem_u32(ps), n0 + c, q0);
            }
            bulk_commit();
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty(buf));
      }
      if (lane == 0) bulk_wait0();  // every store of this warp has completed
    } else {
    float* stg = reinterpret_cast<float*>(slot);
    const int ostride = a.convt ? a.stride : 1;
    uint32_t tl = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
      int mi, ph, ni;
      unit_coords(u, mi, ph, ni);
      const int m0 = mi * BM, n0 = ni * BN;
      const int buf = tl & 1;
      // lane l describes GEMM row q0 + l: whether its output row exists and
      // whether it belongs to an utterance (else it is a gap row -> 0).
      // Output rows of consecutive GEMM rows are ostride apart.
      const int q0 = m0 + quad * 32;
      const int o0 = out_row(a, ph, q0);
      const int o = o0 + lane * ostride;
      const bool ok = q0 + lane < a.rows_in && o >= 0 && o < a.rows_out;
      const bool valid = ok && a.frame_src[o / a.out_scale] >= 0;
      const unsigned okm = __ballot_sync(0xffffffffu, ok);
      const unsigned vm = __ballot_sync(0xffffffffu, valid);
      const long rstep = (long)ostride * a.cout;
      // The residual rows (1x1 convolutions) do not depend on this unit's
      // MMAs: the first column chunk is loaded before the accumulator wait,
      // and each next chunk while the current one is finished, so the loads'
      // latency hides behind the MMAs and the stores.
      auto load_x = [&](int c, float(&dst)[32]) {
        const long b = (long)o0 * a.cout + n0 + c + lane;
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[i] = ((okm >> i) & 1) ? a.x[b + i * rstep] : 0.f;
      };
      float xv[32];
      if (a.add_res && 32 * half < BN) load_x(32 * half, xv);
      mbar_wait(tfull(buf), (tl >> 1) & 1);
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * C::ACC_STRIDE;
#pragma unroll 1
      for (int c = 32 * half; c < BN; c += 64) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        const bool more = a.add_res && c + 64 < BN;
        float xn[32];
        if (more) load_x(c + 64, xn);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) stg[lane * 33 + i] = __uint_as_float(r[i]);
        __syncwarp();
        const int co = n0 + c + lane;
        const float bv = a.bias ? a.bias[co] : 0.f;
        float al = 0.f, inv = 0.f;
        if (a.alpha) {
          al = a.alpha[co];
          inv = 1.f / (al + 1e-9f);
        }
        const long col = co;
        const long base = (long)o0 * a.cout + col;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (!((okm >> i) & 1)) continue;
          float v = stg[i * 33 + lane] + bv;
          if (a.add_res) v += xv[i];
          if (!((vm >> i) & 1)) v = 0.f;
          const long idx = base + i * rstep;
          if (a.x) a.x[idx] = v;
          if (a.p) a.p[idx] = __float2bfloat16_rn(a.alpha ? snake_inv(v, al, inv) : v);
        }
        if (more) {
#pragma unroll
          for (int i = 0; i < 32; ++i) xv[i] = xn[i];
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty(buf));
    }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Narrow dilated convolutions as the transposed product (the ResUnits' k7 at
// <= 128 output channels, whose M = 128 x N = cout MMAs are too narrow to keep
// the tensor pipe busy):
//   D[co, t] = sum_(tap, ci) W[co, tap, ci] * X[t + tap * dil - pad, ci]
// M = output channels (cout <= 128, rows past cout are don't-care), N = 256
// time rows per unit, K = (channel block, tap).  A = the weight tile
// [cout rows x 64 channels] of one (tap, block) on the stage ring; B = the
// unit's input rows plus every tap's shift, staged once per 64-channel block
// as two 160-row TMA boxes, tap t read through a descriptor t * dil rows in
// (as the halo path above).  The accumulator is 128 lanes (channels) x 256
// columns (time), double-buffered: all 512 TMEM columns.  Epilogue: lane =
// channel; per 32-row chunk it writes a [time][channel] bf16 tile (one row
// per store instruction, conflict-free) of Snake(acc + bias), zero on gap
// rows, and stores it by TMA.  Writes the bf16 output only (the k7 layers
// feed the 1x1 convolution; they have no residual or f32 stream).
// ---------------------------------------------------------------------------
constexpr int NT = 256;            // time rows per unit (the MMA's N)
constexpr int HBOX = 160;          // rows per input TMA box; two boxes per block
constexpr int T_HALO_MAX = 2 * HBOX - NT;  // largest (k - 1) * dil
constexpr uint32_t T_HSLOT = 2 * HBOX * 128;
constexpr uint32_t T_A_BYTES = 128 * BK * 2;  // weight stage (rows past cout unused)
constexpr uint32_t T_EPI_SLOT = 2 * 2048;     // two bf16 32 x 32 tiles per warp
constexpr int T_STAGES =
    (int)((SMEM_MAX - 1024 - 2 * T_HSLOT - EPI_WARPS * T_EPI_SLOT - 256) / T_A_BYTES) > 8
        ? 8
        : (int)((SMEM_MAX - 1024 - 2 * T_HSLOT - EPI_WARPS * T_EPI_SLOT - 256) / T_A_BYTES);
constexpr uint32_t T_OFF_HALO = T_STAGES * T_A_BYTES;
constexpr uint32_t T_OFF_EPI = T_OFF_HALO + 2 * T_HSLOT;
constexpr uint32_t T_OFF_BAR = T_OFF_EPI + EPI_WARPS * T_EPI_SLOT;
constexpr size_t T_SMEM = 1024 + (size_t)T_OFF_BAR + 256;
static_assert(T_SMEM <= SMEM_MAX && T_STAGES >= 3, "transposed conv shared memory");
static_assert((T_OFF_HALO % 1024) == 0 && (T_OFF_EPI % 1024) == 0 && (T_HSLOT % 1024) == 0, "alignment");
constexpr uint32_t T_IDESC = idesc_bf16(128, NT);

__global__ void __launch_bounds__(THREADS, 1)
    conv_t_kernel(const __grid_constant__ CUtensorMap tmIn, const __grid_constant__ CUtensorMap tmW,
                  const __grid_constant__ CUtensorMap tmP, const __grid_constant__ ConvTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + T_OFF_BAR);
  // full[T_STAGES], empty[T_STAGES], hfull[2], hempty[2], tfull[2], tempty[2]; tmem slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * T_STAGES + 8);
  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[T_STAGES + s]); };
  auto hfull = [&](int i) { return smem_u32(&bars[2 * T_STAGES + i]); };
  auto hempty = [&](int i) { return smem_u32(&bars[2 * T_STAGES + 2 + i]); };
  auto tfull = [&](int b) { return smem_u32(&bars[2 * T_STAGES + 4 + b]); };
  auto tempty = [&](int b) { return smem_u32(&bars[2 * T_STAGES + 6 + b]); };
  uint8_t* halo = smem + T_OFF_HALO;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int units = (a.rows_in + NT - 1) / NT;
  const int kpt = a.cin_pad / BK;
  const uint32_t w_bytes = (uint32_t)a.cout * 128;  // weight box: cout rows x 64 channels

  // weight-stage rows past cout are never loaded: zero them once so the
  // accumulator lanes they feed (never stored) hold finite values
  for (uint32_t i = threadIdx.x * 16; i < (uint32_t)T_STAGES * T_A_BYTES; i += THREADS * 16)
    if ((i % T_A_BYTES) >= w_bytes) *reinterpret_cast<uint4*>(smem + i) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async();
  if (threadIdx.x == 0) {
    for (int s = 0; s < T_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(hfull(b), 1);
      mbar_init(hempty(b), 1);
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), EPI_WARPS);
    }
    mbar_fence_init();
    prefetch_map(&tmIn);
    prefetch_map(&tmW);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0, hit = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int t0 = u * NT;
        for (int cb = 0; cb < kpt; ++cb, ++hit) {
          const int hs = hit & 1;
          mbar_wait(hempty(hs), ((hit >> 1) & 1) ^ 1);
          mbar_expect_tx(hfull(hs), T_HSLOT);
          uint8_t* hb = halo + hs * T_HSLOT;
          tma_load_2d(smem_u32(hb), &tmIn, hfull(hs), cb * BK, t0 - a.pad);
          tma_load_2d(smem_u32(hb + HBOX * 128), &tmIn, hfull(hs), cb * BK, t0 - a.pad + HBOX);
          for (int tap = 0; tap < a.taps; ++tap, ++it) {
            const int s = it % T_STAGES;
            mbar_wait(empty(s), ((it / T_STAGES) & 1) ^ 1);
            mbar_expect_tx(full(s), w_bytes);
            tma_load_2d(smem_u32(smem + s * T_A_BYTES), &tmW, full(s), tap * a.cin_pad + cb * BK, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, hit = 0, tl = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
        const int buf = tl & 1;
        mbar_wait(tempty(buf), ((tl >> 1) & 1) ^ 1);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * NT;
        for (int cb = 0; cb < kpt; ++cb, ++hit) {
          const int hs = hit & 1;
          const int nkk = min(BK / 16, (a.cin - cb * BK + 15) / 16);  // skip zero-padded channels
          mbar_wait(hfull(hs), (hit >> 1) & 1);
          tc_fence_after();
          const uint32_t h_addr = smem_u32(halo + hs * T_HSLOT);
          for (int tap = 0; tap < a.taps; ++tap, ++it) {
            const int s = it % T_STAGES;
            mbar_wait(full(s), (it / T_STAGES) & 1);
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + s * T_A_BYTES);
            const uint32_t b_addr = h_addr + (uint32_t)(tap * a.dil) * 128u;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              if (kk < nkk)
                umma_f16(d_tmem, sdesc_kmajor(a_addr + kk * 32), sdesc_kmajor(b_addr + kk * 32), T_IDESC,
                         (cb | tap | kk) ? 1u : 0u);
            umma_commit(empty(s));
          }
          umma_commit(hempty(hs));
        }
        umma_commit(tfull(buf));
      }
    }
  } else {
    // ---------------- epilogue warps 2 .. 2 + EPI_WARPS ----------------
    const int quad = warp & 3;        // TMEM lanes = output channels 32 * quad ..
    const int half = (warp - 2) / 4;  // time columns 128 * half .. + 127
    const int co = 32 * quad + lane;
    const bool q_on = 32 * quad < a.cout;  // quads past cout are padding (uniform per warp)
    const bool c_ok = co < a.cout;
    const float bv = (c_ok && a.bias) ? a.bias[co] : 0.f;
    const float al = (c_ok && a.alpha) ? a.alpha[co] : 0.f;
    const float ai = (c_ok && a.alpha) ? a.alpha_inv[co] : 0.f;
    uint8_t* st = smem + T_OFF_EPI + (warp - 2) * T_EPI_SLOT;
    uint32_t tl = 0, g = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++tl) {
      const int buf = tl & 1;
      const int t0 = u * NT;
      mbar_wait(tfull(buf), (tl >> 1) & 1);
      tc_fence_after();
      if (q_on) {
        const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * NT;
#pragma unroll 1
        for (int c = 0; c < 4; ++c, ++g) {
          const int col = 128 * half + 32 * c;
          const int tb = t0 + col;  // first time row of this chunk
          uint32_t r[32];
          tmem_ld32(taddr + col, r);
          const int tr = tb + lane;  // lane j looks up row tb + j
          const unsigned vm =
              __ballot_sync(0xffffffffu, tr < a.rows_in && a.frame_src[tr / a.out_scale] >= 0);
          uint8_t* tile = st + (g & 1) * 2048;  // bf16 [32 rows][32 channels], 64-byte swizzle
          if (lane == 0) bulk_wait_read1();       // the store two chunks back has read this tile
          __syncwarp();
          tmem_wait_ld();
          const uint32_t cbyte = (uint32_t)(lane & 7) * 2;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float v = __uint_as_float(r[j]) + bv;
            if (!((vm >> j) & 1)) v = 0.f;
            if (a.alpha) v = snake_inv(v, al, ai);
            *reinterpret_cast<__nv_bfloat16*>(tile + j * 64 + ((((uint32_t)lane >> 3) ^ ((j >> 1) & 3)) << 4) +
                                              cbyte) = __float2bfloat16_rn(v);
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            // rows past the end are clipped by the TMA unit; a chunk wholly past
            // it commits an empty group so that the tile ring's count holds
            if (tb < a.rows_out) tma_store_2d(&tmP, smem_u32(tile), 32 * quad, tb);
            bulk_commit();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty(buf));
    }
    if (lane == 0) bulk_wait0();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------
// Latent packing and the output head (SIMT: 32 -> 64 columns, 96 -> 1 channel)
// ---------------------------------------------------------------------------

// latent [B, T, 32] f32 -> rows [F, 64] bf16; frame f holds latent frame
// frame_src[f] (b * T + t) or zeros for a gap frame; columns 32..63 are zero.
__global__ void pack_latent_kernel(const float* __restrict__ lat, const int* __restrict__ frame_src,
                                   __nv_bfloat16* __restrict__ out, int F) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)F * 64) return;
  const int f = (int)(i / 64), c = (int)(i % 64);
  const int src = frame_src[f];
  out[i] = __float2bfloat16_rn((src >= 0 && c < 32) ? lat[(long)src * 32 + c] : 0.f);
}

// Head conv (src/codec/decoder.rs:43-54): wav = tanh(conv_k(Snake(x))) with the
// Snake already applied by the producer of `x` (bf16 rows [R, C]).  One block
// of HEAD_ROWS threads per HEAD_ROWS output rows: the (HEAD_ROWS + K - 1)
// input rows the block needs are staged in shared memory with coalesced
// 4-byte loads (row pitch C/2 + 1 words, odd, so the 32 lanes of a warp --
// 32 consecutive rows -- read 32 different banks), then each thread computes
// its row in the same operation order as a per-row loop over (tap, channel).
// Rows of gap frames are skipped; utterance rows go to
// wav[src * hop + (row % hop)].
constexpr int HEAD_ROWS = 128;
template <int C>
__global__ void __launch_bounds__(HEAD_ROWS) head_kernel(const __nv_bfloat16* __restrict__ x, int R,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ bias, int K, int pad,
                                                         const int* __restrict__ frame_src, int hop,
                                                         float* __restrict__ wav) {
  constexpr int W2 = C / 2, PITCH = W2 + 1, ROWS = HEAD_ROWS + 6;
  __shared__ float ws[7 * C];
  __shared__ uint32_t xs[ROWS * PITCH];
  for (int i = threadIdx.x; i < K * C; i += HEAD_ROWS) {
    const int k = i / C, c = i % C;
    ws[i] = w[(long)c * K + k];  // weight [1, C, K]
  }
  const int o0 = blockIdx.x * HEAD_ROWS;
  const int r0 = o0 - pad;  // first staged input row
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(x);
  for (int i = threadIdx.x; i < (HEAD_ROWS + K - 1) * W2; i += HEAD_ROWS) {
    const int rr = i / W2, j = i - rr * W2;
    const int t = r0 + rr;
    xs[rr * PITCH + j] = (t >= 0 && t < R) ? xw[(long)t * W2 + j] : 0u;
  }
  __syncthreads();
  const int o = o0 + threadIdx.x;
  if (o >= R) return;
  const int src = frame_src[o / hop];
  if (src < 0) return;
  float acc = bias ? bias[0] : 0.f;
  for (int k = 0; k < K; ++k) {
    const uint32_t* row = xs + (threadIdx.x + k) * PITCH;
#pragma unroll
    for (int j = 0; j < W2; ++j) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(row + j));
      acc = fmaf(f.x, ws[k * C + 2 * j], acc);
      acc = fmaf(f.y, ws[k * C + 2 * j + 1], acc);
    }
  }
  wav[(long)src * hop + (o % hop)] = tanhf(acc);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

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

template <int BN, int VAR>
void launch(const bf16* in, const bf16* w, const ConvTcArgs& a, cudaStream_t s) {
  using C = Cfg<BN, VAR>;
  static unsigned attr_mask = 0;  // per-device opt-in to the large dynamic smem
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_mask & (1u << (dev & 31)))) {
      IRT_CUDA(cudaFuncSetAttribute(conv_tc_kernel<BN, VAR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)C::SMEM));
      attr_mask |= 1u << (dev & 31);
    }
  }
  // copies: the map cache may be cleared by another thread
  // HALO: one box spans the unit's rows plus every tap's shift
  const CUtensorMap ta = tma_map_bf16(in, a.rows_in, a.cin, a.cin, VAR == 2 ? BM + (a.taps - 1) * a.dil : BM);
  const long kcols = (long)a.taps * a.cin_pad;
  const CUtensorMap tb = tma_map_bf16(w, (long)a.phases * a.cout, kcols, kcols, BN);
  const long units = (long)((a.rows_in + BM - 1) / BM) * a.phases * (a.cout / BN);
  const int grid = (int)std::min<long>(units, num_sms());
  // stride-1 path: TMA maps of the outputs (32 x 32 staging tiles); unused
  // (any valid map) for ConvTranspose
  CUtensorMap tx = ta, tp = ta;
  if (!a.convt) {
    if (a.x) tx = tma_map_tile32(a.x, true, a.rows_out, a.cout, a.cout);
    if (a.p) tp = tma_map_tile32(a.p, false, a.rows_out, a.cout, a.cout);
  } else if (a.ct_tma) {
    if (a.x) tx = tma_map_tile32_phased(a.x, true, a.rows_in, a.cout, a.stride);
    if (a.p) tp = tma_map_tile32_phased(a.p, false, a.rows_in, a.cout, a.stride);
  }
  launch_pdl(conv_tc_kernel<BN, VAR>, dim3(grid), dim3(THREADS), C::SMEM, s, ta, tb, tx, tp, a);
  IRT_CHECK_LAUNCH();
}

// Transposed narrow dilated convolution (conv_t_kernel).
void launch_t(const bf16* in, const bf16* w, const ConvTcArgs& a, cudaStream_t s) {
  static unsigned attr_mask = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(attr_mask & (1u << (dev & 31)))) {
      IRT_CUDA(cudaFuncSetAttribute(conv_t_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)T_SMEM));
      attr_mask |= 1u << (dev & 31);
    }
  }
  const CUtensorMap ti = tma_map_bf16(in, a.rows_in, a.cin, a.cin, HBOX);
  const long kcols = (long)a.taps * a.cin_pad;
  const CUtensorMap tw = tma_map_bf16(w, a.cout, kcols, kcols, a.cout);
  const CUtensorMap tp = tma_map_tile32(a.p, false, a.rows_out, a.cout, a.cout);
  const long units = (a.rows_in + NT - 1) / NT;
  const int grid = (int)std::min<long>(units, num_sms());
  launch_pdl(conv_t_kernel, dim3(grid), dim3(THREADS), T_SMEM, s, ti, tw, tp, a);
  IRT_CHECK_LAUNCH();
}

bool use_conv_t(const ConvTcArgs& a) {
  static const bool on = [] {
    const char* e = std::getenv("IRT_CONV_T");
    return !(e && e[0] == '0');
  }();
  return on && !a.convt && a.taps > 1 && !a.add_res && !a.x && a.p && a.cout <= 128 && (a.cout % 32) == 0 &&
         (a.taps - 1) * a.dil <= T_HALO_MAX && a.rows_out == a.rows_in &&
         !(reinterpret_cast<uintptr_t>(a.p) & 15);
}

// Residual stride-1 convolutions take the residual ring, other stride-1
// convolutions with k > 1 the halo staging (see Cfg).
template <int BN>
void launch(const bf16* in, const bf16* w, const ConvTcArgs& a, cudaStream_t s) {
  if (!a.convt && a.add_res && a.x) launch<BN, 1>(in, w, a, s);
  else if (!a.convt && a.taps > 1 && BM + (a.taps - 1) * a.dil <= HALO_ROWS_MAX) launch<BN, 2>(in, w, a, s);
  else launch<BN, 0>(in, w, a, s);
}

}  // namespace ctc

int conv_tc_bn(int cout) {
  for (int bn : {256, 192, 128, 96, 64, 32})
    if (cout % bn == 0) return bn;
  return 0;
}

void conv_tc(const bf16* in, const bf16* w, const ConvTcArgs& a, cudaStream_t s) {
  if (a.rows_in < ctc::BM || a.cin < 64 || (a.cin % 8) || (a.cin_pad % 64) || a.cin_pad < a.cin)
    throw unsupported("conv_tc: input must have >= 128 rows and >= 64 channels (multiple of 8)");
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    throw unsupported("conv_tc: operands must be 16-byte aligned");
  if (a.alpha && !a.alpha_inv) throw Error(IRT_E_INVALID_ARG, "conv_tc: Snake alpha needs its reciprocal table");
  if (a.add_res && !a.x) throw Error(IRT_E_INVALID_ARG, "conv_tc: a residual convolution needs its f32 stream x");
  if ((a.x && (reinterpret_cast<uintptr_t>(a.x) & 15)) || (a.p && (reinterpret_cast<uintptr_t>(a.p) & 15)) ||
      (a.bias && (reinterpret_cast<uintptr_t>(a.bias) & 15)) ||
      (a.alpha && ((reinterpret_cast<uintptr_t>(a.alpha) | reinterpret_cast<uintptr_t>(a.alpha_inv)) & 15)))
    throw unsupported("conv_tc: outputs, bias and alpha must be 16-byte aligned");
  if ((long)a.rows_out * a.cout >= (1L << 31) || (long)a.rows_in * a.phases >= (1L << 31))
    throw unsupported("conv_tc: level too large for 32-bit row indices");
  // ConvTranspose outputs leave by phased TMA stores when every phase has the
  // same number of rows (rows_out = rows_in * stride; the even strides)
  ConvTcArgs b = a;
  b.ct_tma = a.convt && !a.add_res && (long)a.rows_out == (long)a.rows_in * a.stride;
  // narrow k > 1 convolutions (<= 128 output channels): the transposed product
  if (ctc::use_conv_t(b)) {
    ctc::launch_t(in, w, b, s);
    return;
  }
  switch (conv_tc_bn(a.cout)) {
    case 256: ctc::launch<256>(in, w, b, s); break;
    case 192: ctc::launch<192>(in, w, b, s); break;
    case 128: ctc::launch<128>(in, w, b, s); break;
    case 96: ctc::launch<96>(in, w, b, s); break;
    case 64: ctc::launch<64>(in, w, b, s); break;
    case 32: ctc::launch<32>(in, w, b, s); break;
    default: throw unsupported("conv_tc: output channels must be a multiple of 32");
  }
}

void pack_latent_rows(const float* lat, const int* frame_src, bf16* out, int F, cudaStream_t s) {
  const long n = (long)F * 64;
  if (!n) return;
  ctc::pack_latent_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(lat, frame_src, out, F);
  IRT_CHECK_LAUNCH();
}

void codec_head_rows(const bf16* x, int R, int C, const float* w, const float* bias, int K, int pad,
                     const int* frame_src, int hop, float* wav, cudaStream_t s) {
  if (K > 7) throw unsupported("codec head kernel > 7");
  const unsigned grid = (unsigned)((R + ctc::HEAD_ROWS - 1) / ctc::HEAD_ROWS);
  const int nt = ctc::HEAD_ROWS;
  switch (C) {
    case 96: ctc::head_kernel<96><<<grid, nt, 0, s>>>(x, R, w, bias, K, pad, frame_src, hop, wav); break;
    case 64: ctc::head_kernel<64><<<grid, nt, 0, s>>>(x, R, w, bias, K, pad, frame_src, hop, wav); break;
    case 128: ctc::head_kernel<128><<<grid, nt, 0, s>>>(x, R, w, bias, K, pad, frame_src, hop, wav); break;
    case 32: ctc::head_kernel<32><<<grid, nt, 0, s>>>(x, R, w, bias, K, pad, frame_src, hop, wav); break;
    default: throw unsupported("codec head: channels must be 32, 64, 96 or 128");
  }
  IRT_CHECK_LAUNCH();
}

int conv_tc_read_and_clear_error() { return tcx::read_and_clear_flag(); }

int conv_watchdog_probe(unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns) {
  const cudaError_t e = tcx::run_watchdog_probe(limit_ns, waits, elapsed_ns);
  if (e != cudaSuccess) throw Error(IRT_E_CUDA, std::string("watchdog probe: ") + cudaGetErrorString(e));
  return 0;
}

}  // namespace irt
