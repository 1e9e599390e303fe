// Host-callable launchers for every device kernel of the sampling path.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace irt {

using bf16 = __nv_bfloat16;

// ---------------------------------------------------------------------------
// GEMM: C[M,N] = A[M,K] . B[N,K]^T  (both operands K-major; B is the PyTorch
// [out, in] weight layout), fp32 accumulation, fused epilogue.
// ---------------------------------------------------------------------------

enum EpiMode : int {
  EPI_STORE = 0,   // out = act(alpha*(acc + bias) + add) * row_scale, optional row remap
  EPI_QKVG = 1,    // [q|k|v|g] columns: head RMSNorm (+RoPE) on q,k; v plain; sigmoid(g)
  EPI_RESID = 2,   // x = (x + gate[n]*acc) * row_scale[m]   (f32 residual stream)
  EPI_SWIGLU = 3,  // interleaved [w1 32-col group | w3 32-col group]: h = silu(a)*b
  EPI_CTXKV = 4,   // stacked per-layer [K|V] context projections into the KV cache
};

enum Act : int { ACT_NONE = 0, ACT_SILU = 1, ACT_TANH = 2 };

constexpr int SWIGLU_GROUP = 32;  // interleave width of the packed [W1|W3] weight

struct EpiParams {
  int mode = EPI_STORE;
  int M = 0, N = 0;
  int out_bf16 = 0;          // output element type for STORE/QKVG/SWIGLU/CTXKV (1 = bf16, 0 = f32)
  // STORE
  void* out = nullptr;
  long ldo = 0;
  const float* bias = nullptr;
  float alpha = 1.f;
  const float* add = nullptr;
  long ld_add = 0;
  int act = ACT_NONE;
  const float* row_scale = nullptr;
  const int* row_map = nullptr;   // dst row per source row, < 0 = drop (STORE, CTXKV)
  // QKVG (N = 4*Dq)
  void *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr;  // [M, Dq] each
  const float* qn_w = nullptr;    // [H*hd]
  const float* kn_w = nullptr;    // [H*hd] (CTXKV: [L][H*hd])
  const float* rope_cos = nullptr;  // [pos][hd/2]
  const float* rope_sin = nullptr;
  const int* tok_pos = nullptr;   // [M] RoPE position of each row
  int H = 0, hd = 0, rope_heads = 0;
  float eps = 1e-5f;
  // RESID
  float* x = nullptr;
  const float* gate = nullptr;    // [N] or null (= 1)
  int x_tma = 0;                   // RESID on tcgen05: the launcher attached a reduce-add tensor map of x
  // SWIGLU
  void* h = nullptr;              // [M, F]
  int F = 0;
  // CTXKV (N = L*2*Dq)
  void *ck = nullptr, *cv = nullptr;  // layer 0 base of the K / V caches ([rows, Dq] per layer)
  long layer_stride = 0;          // elements between layers
  int Dq = 0;
  // batched launches (SIMT path only): per-z offsets
  long bias_bstride = 0, out_bstride = 0, add_bstride = 0;
  // gemm_tc_tf32x3 as an implicit convolution: K = conv_taps x Cin_p and tap
  // j of output row m reads A row m + j * conv_dil - conv_pad (rows outside
  // [0, rows of A) read as zero)
  int conv_taps = 1, conv_dil = 1, conv_pad = 0;
};

// fp32 SIMT GEMM into a raw accumulator buffer, then the epilogue kernel.
// A/B element types: a_bf16/b_bf16 select bf16 (else f32).  Batched over z.
void gemm_simt(const void* A, int a_bf16, long lda, long a_bstride, const void* B, int b_bf16, long ldb,
               long b_bstride, float* raw, long ldr, long r_bstride, int M, int N, int K, int batch,
               cudaStream_t s);
void epilogue_apply(const EpiParams& p, const float* raw, long ldr, long r_bstride, int batch, cudaStream_t s);

// tcgen05 (sm_100a) bf16 GEMM with the fused epilogue.  Requirements: A, B
// bf16, K % 8 == 0, lda/ldb % 8 == 0, 16-byte aligned bases.  Returns false
// when the shape is outside what the kernel handles (caller falls back).
bool gemm_tc_supported(const EpiParams& p, int K, long lda, long ldb, const void* A, const void* B);
void gemm_tc(const bf16* A, long lda, const bf16* B, long ldb, int M, int N, int K, const EpiParams& p,
             cudaStream_t s);
// f32 GEMM on the tcgen05 tf32 path with the same epilogues: A2 = [A_hi | A_lo]
// [M, 2 Kp] and B2 = [B_hi | B_lo] [N, 2 Kp] from split_tf32 (Kp = K rounded
// up to a multiple of 32, zero columns in between); C = A_hi.B_hi + A_hi.B_lo +
// A_lo.B_hi accumulated in f32.  Shape checks as gemm_tc_supported with K = Kp.
// a_rows / b_rows > 0: the rows of A2 / B2 that exist (zero padding included,
// at least one 128-row box); the tensor maps span exactly those and rows past
// them read as zero.  0: M / N.
void gemm_tc_tf32x3(const float* A2, long lda2, const float* B2, long ldb2, int M, int N, int Kp, const EpiParams& p,
                    cudaStream_t s, long a_rows = 0, long b_rows = 0);
// A [M, K] f32 (lda % 4 == 0, 16-byte aligned) -> A2 [M, 2 Kp] as above.
void split_tf32(const float* A, long lda, int M, int K, float* A2, int Kp, cudaStream_t s);
inline int tf32_kpad(int K) { return (K + 31) / 32 * 32; }
// Device-side watchdog flag of the GEMM kernels (0 = ok).
int read_and_clear_kernel_error();
// Watchdog probes (test hooks): run tcx::watchdog_probe_kernel in the GEMM /
// attention translation unit with a wait limit of limit_ns and `waits` waits
// on a barrier nothing arrives on; the elapsed device time goes to
// *elapsed_ns and that unit's flag is left set.
int gemm_watchdog_probe(unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns);
int attn_watchdog_probe(unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns);

// ---------------------------------------------------------------------------
// Attention over [self keys | context keys] per sequence.
// ---------------------------------------------------------------------------
struct SeqDesc {
  int tok_start;  // first row of this sequence in the packed q/k/v buffers
  int len;        // number of query (and self key) rows
  int ctx_off;    // first row in the per-layer context cache
  int ctx_len;    // number of (valid) context rows
};

struct AttnParams {
  const void* q;      // [M, H*hd]
  const void* k;      // [M, H*hd]
  const void* v;      // [M, H*hd]
  const void* gsig;   // [M, H*hd] sigmoid(gate), multiplied into the output (may be null)
  const void* ck;     // [rows, H*hd] context keys of this layer (may be null)
  const void* cv;
  const uint8_t* key_mask;  // [M] validity of self keys (null = all valid)
  const SeqDesc* seqs;
  int nseq;
  int max_len;        // max over seqs of len
  int H, hd;
  float scale;
  void* out;          // [M, H*hd]
  int rows;           // rows of the q/k/v buffers (TMA bounds)
  int ctx_rows;       // rows of the context cache (TMA bounds)
  int path;           // 0 = best available, 1 = mma.sync kernel, 2 = SIMT kernel (register-tiled
                      // for f32 at hd = 128), 3 = warp-per-query SIMT kernel
};
void attention(const AttnParams& p, int bf16_io, cudaStream_t s);
bool attention_tc_supported(const AttnParams& p);
void attention_tc(const AttnParams& p, cudaStream_t s);
int read_and_clear_attn_error();

// ---------------------------------------------------------------------------
// Row-wise / elementwise kernels.  `T` selects bf16 (1) or f32 (0) storage
// for GEMM operands.
// ---------------------------------------------------------------------------
// h = x / sqrt(mean(x^2)+eps) * (1 + scale) + shift   (LowRankAdaLn modulate)
void adaln_modulate(const float* x, const float* shift, const float* scale, void* h, int out_bf16, int M, int D,
                    float eps, cudaStream_t s);
// y = x / sqrt(mean(x^2)+eps) * w   (RmsNorm; w may be null)
void rms_norm(const float* x, const float* w, void* y, int out_bf16, int M, int D, float eps, cudaStream_t s);
// RMSNorm rows written as bf16 hi | lo halves ([M, 2D]) for a GEMM over the
// weight repeated along K; D a multiple of 4, at most 2048.
bool rms_norm_split_supported(int D);
void rms_norm_split(const float* x, const float* w, bf16* y, int M, int D, float eps, cudaStream_t s);
// f32 rows [M, P] -> bf16 hi | lo rows [M, 2 Pk] (hi at column d, lo at Pk + d).
void gather_split_rows(const float* in, bf16* out, int M, int P, int Pk, cudaStream_t s);
// out = RmsNorm(x; nw) . W^T + bias for a narrow output (W [P, D], bf16 or f32)
void rmsnorm_proj(const float* x, const float* nw, const void* W, int w_bf16, const float* bias, float* out, int M,
                  int D, int P, float eps, cudaStream_t s);
// x[m] = table[ids[m]] * mask[m]
void embed_rows(const int* ids, const uint8_t* mask, const float* table, float* x, int M, int D, cudaStream_t s);
void embed_rows_v(const int* ids, const uint8_t* mask, const float* table, float* x, int M, int D, int vocab,
                  cudaStream_t s);
// out[m] = convert(in[m]) for f32 -> bf16/f32 copies with optional row gather
// out row m (row stride ld_out, default D) = in row src_row[m] (or m), converted.
void gather_rows(const float* in, const int* src_row, void* out, int out_bf16, int M, int D, cudaStream_t s,
                 int ld_out = 0);
// scale rows by a mask (x *= mask[m])
void mask_rows(float* x, const uint8_t* mask, int M, int D, cudaStream_t s);
void silu_copy(const float* in, long ld_in, float* out, long ld_out, int M, int D, cudaStream_t s);
// masked mean token prepend (src/model/dit/aux_conditioner.rs:161-190):
// state [B, S, D] -> out [B, S+1, D], mask [B,S] -> mask_out [B, S+1]
void prepend_mean_token(const float* state, const uint8_t* mask, float* out, uint8_t* mask_out, int B, int S, int D,
                        cudaStream_t s);
// v = v_c + sum_k s_k (v_c - v_k): groups of rows in v_packed
void cfg_combine(const float* v_packed, const int* group_row0, const float* scales, int ngroups, const int* utt_off,
                 int ntok, int P, float* v_out, cudaStream_t s);
// x = x + v * dt, ...
void axpy(float* y, const float* x, float a, long n, cudaStream_t s);  // y += a*x
void lincomb(float* out, const float* const* xs, const float* coefs, int nx, long n, cudaStream_t s);
void temporal_rescale(float* v, const float* x, float omt, float ratio, long n, cudaStream_t s);
void scale_buf(float* x, float a, long n, cudaStream_t s);
void scale_rows_bf16_or_f32(void* buf, int is_bf16, long row_len, const int* rows, int nrows, float a,
                            cudaStream_t s);
// gaussian noise (Box-Muller over a counter-based hash), for requests without initial_noise
void gaussian_fill(float* x, long n, uint64_t seed, cudaStream_t s);

// ---------------------------------------------------------------------------
// DACVAE decoder kernels
// ---------------------------------------------------------------------------
// y[b, co, t] = bias[co] + sum_{ci,k} W[co, ci, k] * snake(x[b, ci, t + k*dil - pad])
// channel-major activations [B, C, T]; optional fused Snake on the input,
// optional residual add and tanh on the output.
void conv1d(const float* x, int B, int Cin, int T, const float* w, const float* bias, int Cout, int K, int dil,
            int pad, const float* snake_alpha, const float* residual, int tanh_out, float* y, cudaStream_t s);
void conv_transpose1d(const float* x, int B, int Cin, int T, const float* w, const float* bias, int Cout, int stride,
                      int pad, const float* snake_alpha, float* y, int Tout, cudaStream_t s);
void transpose_btc_bct(const float* in, float* out, int B, int T, int C, cudaStream_t s);

}  // namespace irt
