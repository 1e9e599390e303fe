// f32 DACVAE decode on the tcgen05 tf32 GEMM (gemm_tc_tf32x3): every
// convolution of the decoder (src/codec/decoder.rs:17-126, layers.rs:27-75)
// as an implicit GEMM over time-major rows, with f32 accuracy from tf32 hi /
// lo operand halves (A_hi.B_hi + A_hi.B_lo + A_lo.B_hi, chunked f32
// accumulation; see gemm_tc.cu).
//
// Per layer: snake_split_kernel turns the f32 activation rows [rows, C] into
// A2 = [hi | lo] of Snake(x) ([rows_pad, 2 Cp], Cp = C rounded up to 32,
// zero columns and zero rows past `rows`), then one GEMM whose taps read A
// rows shifted by tap * dil - pad (rows outside the utterance read as zero:
// the convolution's zero padding).  The epilogue adds the bias and, for the
// residual units' 1x1 convolution, the residual (x = x + conv, in place).
// ConvTranspose1d (kernel 2s, stride s, padding p = ceil(s / 2)) runs as s
// phase GEMMs of two taps: output row t = q s + r - p of phase r takes
// W[:, :, r] . x[q] + W[:, :, r + s] . x[q - 1] (tap offsets 0 and -1), the
// epilogue's row map sending GEMM row q to output row t.  The head (Snake,
// conv C -> 1, tanh) is a SIMT kernel over staged rows.
#include <cstring>

#include "codec.hpp"

namespace irt {

namespace {

__device__ __forceinline__ float snake_f32(float x, float a) {
  const float s = sinf(a * x);
  return x + s * s / (a + 1e-9f);
}

__device__ __forceinline__ float tf32_hi_f(float a) {
  const uint32_t u = __float_as_uint(a);
  if ((u & 0x7f800000u) == 0x7f800000u) return a;
  return __uint_as_float((u + 0x1000u) & 0xffffe000u);
}

// A2 row r (r < rows_pad), column block of 4: [hi | lo] of Snake(x[r][c])
// (identity without alpha); zero for c >= C or r >= rows.
__global__ void snake_split_kernel(const float* __restrict__ x, int rows, int C, const float* __restrict__ alpha,
                                   float* __restrict__ a2, int Cp, int rows_pad) {
  const int q = Cp / 4;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)rows_pad * q) return;
  const int r = (int)(i / q), c = (int)(i - (long)r * q) * 4;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (r < rows && c < C) {
    const float4 t = *reinterpret_cast<const float4*>(x + (long)r * C + c);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    if (alpha) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = snake_f32(v[j], alpha[c + j]);
    }
  }
  float h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    h[j] = tf32_hi_f(v[j]);
    l[j] = v[j] - h[j];
  }
  float* o = a2 + (long)r * 2 * Cp + c;
  *reinterpret_cast<float4*>(o) = make_float4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<float4*>(o + Cp) = make_float4(l[0], l[1], l[2], l[3]);
}

// Row maps of the s phase GEMMs of a ConvTranspose: map[r * (tin + 1) + q] =
// q s + r - p when that output row exists, else -1.
__global__ void phase_rows_kernel(int* __restrict__ map, int tin, int s, int p) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long n = (long)s * (tin + 1);
  if (i >= n) return;
  const int r = (int)(i / (tin + 1)), q = (int)(i - (long)r * (tin + 1));
  const long t = (long)q * s + r - p;
  map[i] = (t >= 0 && t < (long)tin * s) ? (int)t : -1;
}

// Head: wav[t] = tanh(b + sum_k sum_c w[c][k] Snake(x[t + k - pad][c])), one
// thread per output row, HEADF rows (+ K - 1 halo) staged per block with an
// odd row pitch (conflict-free column reads across rows).
constexpr int HEADF = 64, HEADF_MAXC = 128, HEADF_MAXK = 7;
__global__ void __launch_bounds__(HEADF) head_f32_kernel(const float* __restrict__ x, int rows, int C,
                                                         const float* __restrict__ alpha,
                                                         const float* __restrict__ w, const float* __restrict__ bias,
                                                         int K, int pad, float* __restrict__ wav) {
  __shared__ float ws[HEADF_MAXK * HEADF_MAXC];
  __shared__ float xs[(HEADF + HEADF_MAXK - 1) * (HEADF_MAXC + 1)];
  const int pitch = C | 1;
  for (int i = threadIdx.x; i < K * C; i += HEADF) {
    const int k = i / C, c = i - k * C;
    ws[i] = w[(long)c * K + k];  // weight [1, C, K]
  }
  const int o0 = blockIdx.x * HEADF, r0 = o0 - pad;
  for (int i = threadIdx.x; i < (HEADF + K - 1) * C; i += HEADF) {
    const int rr = i / C, c = i - rr * C, t = r0 + rr;
    float v = 0.f;
    if (t >= 0 && t < rows) v = alpha ? snake_f32(x[(long)t * C + c], alpha[c]) : x[(long)t * C + c];
    xs[rr * pitch + c] = v;
  }
  __syncthreads();
  const int o = o0 + threadIdx.x;
  if (o >= rows) return;
  float acc = bias ? bias[0] : 0.f;
  for (int k = 0; k < K; ++k) {
    const float* row = xs + (threadIdx.x + k) * pitch;
    for (int c = 0; c < C; ++c) acc = fmaf(row[c], ws[k * C + c], acc);
  }
  wav[o] = tanhf(acc);
}

// Host tf32 split (same rounding as the device kernels).
inline void split_host(float a, float& hi, float& lo) {
  uint32_t u;
  std::memcpy(&u, &a, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x1000u) & 0xffffe000u;
  std::memcpy(&hi, &u, 4);
  lo = a - hi;
}

int up32(int c) { return (c + 31) / 32 * 32; }
int up128(int c) { return (c + 127) / 128 * 128; }

}  // namespace

// conv1d weight [cout, cin, k] -> [cout_pad][hi: k x cin_p | lo: k x cin_p]
void codec_pack_tf32_conv(Codec::Conv& c, const std::vector<float>& w) {
  c.cp = up32(c.cin);
  c.cout_pad = up128(c.cout);
  const long kp = (long)c.k * c.cp;
  std::vector<float> o((size_t)c.cout_pad * 2 * kp, 0.f);
  for (int co = 0; co < c.cout; ++co)
    for (int ci = 0; ci < c.cin; ++ci)
      for (int t = 0; t < c.k; ++t) {
        float hi, lo;
        split_host(w[((size_t)co * c.cin + ci) * c.k + t], hi, lo);
        o[(size_t)co * 2 * kp + (size_t)t * c.cp + ci] = hi;
        o[(size_t)co * 2 * kp + kp + (size_t)t * c.cp + ci] = lo;
      }
  c.w2.alloc(o.size() * 4);
  IRT_CUDA(cudaMemcpy(c.w2.p, o.data(), o.size() * 4, cudaMemcpyHostToDevice));
}

// ConvTranspose1d weight [cin, cout, 2s] -> per phase r [cout_pad][hi: 2 x
// cin_p | lo: 2 x cin_p], tap 0 = kernel index r (input q), tap 1 = r + s
// (input q - 1).
void codec_pack_tf32_convt(Codec::Conv& c, const std::vector<float>& w, int s) {
  c.cp = up32(c.cin);
  c.cout_pad = up128(c.cout);
  const long kp = 2L * c.cp;
  const size_t per = (size_t)c.cout_pad * 2 * kp;
  std::vector<float> o(per * s, 0.f);
  for (int r = 0; r < s; ++r)
    for (int co = 0; co < c.cout; ++co)
      for (int j = 0; j < 2; ++j)
        for (int ci = 0; ci < c.cin; ++ci) {
          float hi, lo;
          split_host(w[((size_t)ci * c.cout + co) * 2 * s + r + j * s], hi, lo);
          o[per * r + (size_t)co * 2 * kp + (size_t)j * c.cp + ci] = hi;
          o[per * r + (size_t)co * 2 * kp + kp + (size_t)j * c.cp + ci] = lo;
        }
  c.w2.alloc(o.size() * 4);
  IRT_CUDA(cudaMemcpy(c.w2.p, o.data(), o.size() * 4, cudaMemcpyHostToDevice));
}

bool codec_tf32_supported(const Codec& c) {
  auto ok = [](const Codec::Conv& v) { return v.w2.p && v.cin % 4 == 0 && v.k <= 7; };
  bool r = ok(c.qout) && ok(c.stem) && c.head.cout == 1 && c.head.cin <= HEADF_MAXC && c.head.k <= HEADF_MAXK;
  for (const auto& bl : c.blocks) {
    r = r && bl.ct.w2.p && bl.ct.cin % 4 == 0 && bl.ct.k == 2 * bl.stride;
    for (const auto& ru : bl.res) r = r && ok(ru.c1) && ok(ru.c3);
  }
  return r;
}

namespace {
// One convolution over x [rows, cin]: A2 = [hi | lo] of Snake(x) (split =
// false: A2 already holds it, as for the 2nd..s-th phase of a ConvTranspose),
// then the GEMM of m_rows output rows into out (+ add; rows through map when
// given).
void run_conv(Codec& c, const Codec::Conv& cv, const float* x, int rows, const float* alpha, int m_rows, int taps,
              int dil, int pad, const float* w2, const int* map, const float* add, float* out, cudaStream_t s,
              bool split) {
  const int rows_pad = std::max(rows, 128);
  float* a2 = c.fa2.as<float>();
  if (split) {
    const long n = (long)rows_pad * (cv.cp / 4);
    snake_split_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, rows, cv.cin, alpha, a2, cv.cp, rows_pad);
    IRT_CHECK_LAUNCH();
  }
  EpiParams p;
  p.mode = EPI_STORE;
  p.M = m_rows;
  p.N = cv.cout;
  p.out_bf16 = 0;
  p.out = out;
  p.ldo = cv.cout;
  p.bias = cv.b.p ? cv.b.as<float>() : nullptr;
  p.add = add;
  p.ld_add = cv.cout;
  p.row_map = map;
  p.conv_taps = taps;
  p.conv_dil = dil;
  p.conv_pad = pad;
  const int kp = taps * cv.cp;
  gemm_tc_tf32x3(a2, 2L * cv.cp, w2, 2L * kp, m_rows, cv.cout, kp, p, s, rows_pad, cv.cout_pad);
}
}  // namespace

// One utterance: lat [T, 32] (device), wav [T * hop].
void codec_decode_tf32(Codec& c, const float* lat, int T, float* wav, cudaStream_t s) {
  if (T <= 0) return;
  // widest level: rows x channels of every activation, and A2's 2 Cp columns
  long maxel = (long)T * std::max(c.qout.cout, c.stem.cout), maxa = (long)std::max(T, 128) * 2 * c.qout.cp;
  maxa = std::max(maxa, (long)std::max(T, 128) * 2 * c.stem.cp);
  long rows = T, maxmap = 0;
  for (const auto& bl : c.blocks) {
    maxa = std::max(maxa, (long)std::max<long>(rows, 128) * 2 * bl.ct.cp);
    maxmap = std::max(maxmap, (long)bl.stride * (rows + 1));
    rows *= bl.stride;
    maxel = std::max(maxel, rows * bl.ct.cout);
    for (const auto& ru : bl.res) maxa = std::max(maxa, (long)std::max<long>(rows, 128) * 2 * ru.c1.cp);
  }
  c.fx.ensure((size_t)maxel * 4 + 16);
  c.fy.ensure((size_t)maxel * 4 + 16);
  c.fa2.ensure((size_t)maxa * 4 + 16);
  c.fmap.ensure((size_t)maxmap * 4 + 16);
  float* x = c.fx.as<float>();
  float* y = c.fy.as<float>();
  // quantizer out_proj (1x1, 32 -> qout.cout), stem conv (k7)
  run_conv(c, c.qout, lat, T, nullptr, T, 1, 1, 0, c.qout.w2.as<float>(), nullptr, nullptr, y, s, true);
  run_conv(c, c.stem, y, T, nullptr, T, c.stem.k, 1, c.stem.pad, c.stem.w2.as<float>(), nullptr, nullptr, x, s,
           true);
  long cur = T;
  for (auto& bl : c.blocks) {
    // Snake -> ConvTranspose (src/codec/decoder.rs:26-33): s phase GEMMs on one A2
    const int tin = (int)cur, st = bl.stride;
    const long nm = (long)st * (tin + 1);
    int* map = c.fmap.as<int>();
    phase_rows_kernel<<<(unsigned)((nm + 255) / 256), 256, 0, s>>>(map, tin, st, bl.ct.pad);
    IRT_CHECK_LAUNCH();
    const size_t per = (size_t)bl.ct.cout_pad * 2 * 2 * bl.ct.cp;
    for (int r = 0; r < st; ++r)
      run_conv(c, bl.ct, x, tin, bl.alpha.as<float>(), tin + 1, 2, -1, 0, bl.ct.w2.as<float>() + per * r,
               map + (long)r * (tin + 1), nullptr, y, s, r == 0);
    std::swap(x, y);
    cur = (long)tin * st;
    for (auto& ru : bl.res) {
      // Snake -> conv k7 dil -> Snake -> conv 1x1 -> + x (src/codec/layers.rs:52-60)
      run_conv(c, ru.c1, x, (int)cur, ru.a0.as<float>(), (int)cur, ru.c1.k, ru.c1.dil, ru.c1.pad,
               ru.c1.w2.as<float>(), nullptr, nullptr, y, s, true);
      run_conv(c, ru.c3, y, (int)cur, ru.a2.as<float>(), (int)cur, 1, 1, 0, ru.c3.w2.as<float>(), nullptr, x, x, s,
               true);
    }
  }
  // head: Snake -> conv(C -> 1, k7) -> tanh (src/codec/decoder.rs:43-54)
  head_f32_kernel<<<(unsigned)((cur + HEADF - 1) / HEADF), HEADF, 0, s>>>(
      x, (int)cur, c.head.cin, c.head_alpha.as<float>(), c.head.w.as<float>(),
      c.head.b.p ? c.head.b.as<float>() : nullptr, c.head.k, c.head.pad, wav);
  IRT_CHECK_LAUNCH();
}

}  // namespace irt
