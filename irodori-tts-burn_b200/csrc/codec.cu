// DACVAE decoder (src/codec/decoder.rs:17-126, layers.rs:27-75,
// bottleneck.rs:31-33, model.rs:60-65) on channel-major activations [B, C, T].
//
// conv1d: 64 output channels x 64 samples per CTA, Snake fused into the input
//   staging (x + sin^2(a x) / (a + 1e-9), src/codec/layers.rs:27-33), bias,
//   residual add and tanh fused into the output.
// conv_transpose1d (kernel 2s, stride s, padding ceil(s/2)): polyphase -- each
//   output sample receives exactly two taps per input channel.
#include <map>

#include "codec.hpp"
#include "safetensors.hpp"

namespace irt {

namespace {

constexpr int CO_T = 64, T_T = 64, CI_T = 16, MAXK = 7, MAXDIL = 9;
constexpr int XW = T_T + (MAXK - 1) * MAXDIL;

__device__ __forceinline__ float snake_f(float x, float a) {
  float s = sinf(a * x);
  return x + s * s / (a + 1e-9f);
}

__global__ void __launch_bounds__(256) conv1d_kernel(const float* __restrict__ x, int Cin, int T,
                                                     const float* __restrict__ w, const float* __restrict__ bias,
                                                     int Cout, int K, int dil, int pad,
                                                     const float* __restrict__ alpha,
                                                     const float* __restrict__ res, int tanh_out,
                                                     float* __restrict__ y) {
  __shared__ float xs[CI_T][XW];
  __shared__ float wsm[CI_T][MAXK][CO_T];
  const int b = blockIdx.z;
  const int co0 = blockIdx.y * CO_T, t0 = blockIdx.x * T_T;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int span = T_T + (K - 1) * dil;
  float acc[4][4] = {};
  const float* xb = x + (long)b * Cin * T;
  for (int c0 = 0; c0 < Cin; c0 += CI_T) {
    for (int e = threadIdx.x; e < CI_T * span; e += 256) {
      int ci = e / span, j = e % span;
      int gc = c0 + ci, gt = t0 - pad + j;
      float v = 0.f;
      if (gc < Cin && gt >= 0 && gt < T) {
        v = xb[(long)gc * T + gt];
        if (alpha) v = snake_f(v, alpha[gc]);
      }
      xs[ci][j] = v;
    }
    for (int e = threadIdx.x; e < CI_T * K * CO_T; e += 256) {
      int co = e % CO_T, r = e / CO_T;
      int k = r % K, ci = r / K;
      int gco = co0 + co, gc = c0 + ci;
      wsm[ci][k][co] = (gco < Cout && gc < Cin) ? w[((long)gco * Cin + gc) * K + k] : 0.f;
    }
    __syncthreads();
    for (int ci = 0; ci < CI_T; ++ci) {
      for (int k = 0; k < K; ++k) {
        float xv[4], wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = xs[ci][tx + 16 * j + k * dil];
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = wsm[ci][k][ty * 4 + i];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wv[i], xv[j], acc[i][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int co = co0 + ty * 4 + i;
    if (co >= Cout) continue;
    float bv = bias ? bias[co] : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int t = t0 + tx + 16 * j;
      if (t >= T) continue;
      long idx = ((long)b * Cout + co) * T + t;
      float v = acc[i][j] + bv;
      if (res) v += res[idx];
      if (tanh_out) v = tanhf(v);
      y[idx] = v;
    }
  }
}

constexpr int CT_CI = 4, MAXS = 12;

__global__ void __launch_bounds__(256) convt_kernel(const float* __restrict__ x, int Cin, int T,
                                                    const float* __restrict__ w, const float* __restrict__ bias,
                                                    int Cout, int stride, int pad, const float* __restrict__ alpha,
                                                    float* __restrict__ y, int Tout) {
  __shared__ float xs[CT_CI][T_T / 2 + 4];
  __shared__ float wsm[CT_CI][2 * MAXS][CO_T];
  const int b = blockIdx.z;
  const int co0 = blockIdx.y * CO_T, t0 = blockIdx.x * T_T;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int K = 2 * stride;
  const int tin0 = (t0 + pad) / stride - 1;  // first input sample the tile touches
  const int nin = (t0 + T_T - 1 + pad) / stride - tin0 + 1;
  float acc[4][4] = {};
  const float* xb = x + (long)b * Cin * T;
  int qj[4], rj[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int t = t0 + tx + 16 * j;
    qj[j] = (t + pad) / stride;
    rj[j] = (t + pad) % stride;
  }
  for (int c0 = 0; c0 < Cin; c0 += CT_CI) {
    for (int e = threadIdx.x; e < CT_CI * nin; e += 256) {
      int ci = e / nin, j = e % nin;
      int gc = c0 + ci, gt = tin0 + j;
      float v = 0.f;
      if (gc < Cin && gt >= 0 && gt < T) {
        v = xb[(long)gc * T + gt];
        if (alpha) v = snake_f(v, alpha[gc]);
      }
      xs[ci][j] = v;
    }
    for (int e = threadIdx.x; e < CT_CI * K * CO_T; e += 256) {
      int co = e % CO_T, r = e / CO_T;
      int k = r % K, ci = r / K;
      int gco = co0 + co, gc = c0 + ci;
      wsm[ci][k][co] = (gco < Cout && gc < Cin) ? w[((long)gc * Cout + gco) * K + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int ci = 0; ci < CT_CI; ++ci) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x0 = xs[ci][qj[j] - tin0];      // k = r
        float x1 = xs[ci][qj[j] - 1 - tin0];  // k = r + s
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc[i][j] = fmaf(wsm[ci][rj[j]][ty * 4 + i], x0, fmaf(wsm[ci][rj[j] + stride][ty * 4 + i], x1, acc[i][j]));
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int co = co0 + ty * 4 + i;
    if (co >= Cout) continue;
    float bv = bias ? bias[co] : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int t = t0 + tx + 16 * j;
      if (t < Tout) y[((long)b * Cout + co) * Tout + t] = acc[i][j] + bv;
    }
  }
}

__global__ void transpose_kernel(const float* in, float* out, int B, int T, int C) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)B * T * C) return;
  int c = (int)(i % C);
  long r = i / C;
  int t = (int)(r % T), b = (int)(r / T);
  out[((long)b * C + c) * T + t] = in[i];
}

}  // namespace

void conv1d(const float* x, int B, int Cin, int T, const float* w, const float* bias, int Cout, int K, int dil,
            int pad, const float* snake_alpha, const float* residual, int tanh_out, float* y, cudaStream_t s) {
  if (K > MAXK || (K - 1) * dil > (MAXK - 1) * MAXDIL) throw unsupported("conv1d kernel/dilation too large");
  dim3 grid((T + T_T - 1) / T_T, (Cout + CO_T - 1) / CO_T, B);
  conv1d_kernel<<<grid, 256, 0, s>>>(x, Cin, T, w, bias, Cout, K, dil, pad, snake_alpha, residual, tanh_out, y);
  IRT_CHECK_LAUNCH();
}

void conv_transpose1d(const float* x, int B, int Cin, int T, const float* w, const float* bias, int Cout, int stride,
                      int pad, const float* snake_alpha, float* y, int Tout, cudaStream_t s) {
  if (stride > MAXS || stride < 1) throw unsupported("conv_transpose1d stride > 12");
  dim3 grid((Tout + T_T - 1) / T_T, (Cout + CO_T - 1) / CO_T, B);
  convt_kernel<<<grid, 256, 0, s>>>(x, Cin, T, w, bias, Cout, stride, pad, snake_alpha, y, Tout);
  IRT_CHECK_LAUNCH();
}

void transpose_btc_bct(const float* in, float* out, int B, int T, int C, cudaStream_t s) {
  long n = (long)B * T * C;
  if (!n) return;
  transpose_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in, out, B, T, C);
  IRT_CHECK_LAUNCH();
}

// ---------------------------------------------------------------------------
// Codec object
// ---------------------------------------------------------------------------

namespace {
std::vector<float> up_f32(DevBuf& dst, const TensorView& v) {
  std::vector<float> h((size_t)v.numel());
  decode_to_f32(v, h.data());
  dst.alloc(h.size() * 4 + 4);
  IRT_CUDA(cudaMemcpy(dst.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
  return h;
}

void up_host(DevBuf& dst, const std::vector<float>& h) {
  dst.alloc(h.size() * 4 + 4);
  IRT_CUDA(cudaMemcpy(dst.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
}

// Rank-3 convolution weight `<p>.weight`, or its weight-norm parametrisation
// `<p>.weight_g` / `<p>.weight_v` resolved at load exactly as the reference's
// converter does (scripts/convert_dacvae_weights.py:39-70):
//   weight = g * v / (||v|| + 1e-12), ||v|| over all dimensions except dim 0.
std::vector<float> conv_weight(const SafeTensorsFile& st, const std::string& p, std::vector<long>& shape) {
  if (st.has(p + ".weight") || !(st.has(p + ".weight_g") && st.has(p + ".weight_v"))) {
    const TensorView& w = st.get(p + ".weight", 3);
    shape.assign(w.shape.begin(), w.shape.end());
    std::vector<float> h((size_t)w.numel());
    decode_to_f32(w, h.data());
    return h;
  }
  const TensorView& v = st.get(p + ".weight_v", 3);
  const TensorView& g = st.get(p + ".weight_g");
  shape.assign(v.shape.begin(), v.shape.end());
  const long rows = shape[0], per = (long)v.numel() / rows;
  if (g.numel() != rows) throw shape_error(p + ".weight_g must hold one magnitude per output index");
  std::vector<float> h((size_t)v.numel()), gh((size_t)rows);
  decode_to_f32(v, h.data());
  decode_to_f32(g, gh.data());
  for (long r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (long i = 0; i < per; ++i) ss += (double)h[r * per + i] * h[r * per + i];
    const float scale = gh[r] / ((float)std::sqrt(ss) + 1e-12f);
    for (long i = 0; i < per; ++i) h[r * per + i] *= scale;
  }
  return h;
}

void up_bf16(DevBuf& dst, const std::vector<uint16_t>& h) {
  dst.alloc(h.size() * 2 + 16);
  IRT_CUDA(cudaMemcpy(dst.p, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
}

int round_up64(int c) { return (c + 63) / 64 * 64; }

// conv1d weight [cout, cin, k] -> bf16 [cout][k][cin_pad] (zero-padded channels)
std::vector<uint16_t> pack_conv(const std::vector<float>& w, int cout, int cin, int k, int cin_pad) {
  std::vector<uint16_t> o((size_t)cout * k * cin_pad, 0);
  for (int co = 0; co < cout; ++co)
    for (int ci = 0; ci < cin; ++ci)
      for (int t = 0; t < k; ++t)
        o[((size_t)co * k + t) * cin_pad + ci] = f32_to_bf16_bits(w[((size_t)co * cin + ci) * k + t]);
  return o;
}

// ConvTranspose1d weight [cin, cout, 2s] -> bf16 [s][cout][2][cin_pad]: phase r
// tap 0 is kernel index r (input q), tap 1 is r + s (input q - 1).
std::vector<uint16_t> pack_convt(const std::vector<float>& w, int cin, int cout, int s, int cin_pad) {
  std::vector<uint16_t> o((size_t)s * cout * 2 * cin_pad, 0);
  for (int r = 0; r < s; ++r)
    for (int co = 0; co < cout; ++co)
      for (int j = 0; j < 2; ++j)
        for (int ci = 0; ci < cin; ++ci)
          o[(((size_t)r * cout + co) * 2 + j) * cin_pad + ci] =
              f32_to_bf16_bits(w[((size_t)ci * cout + co) * 2 * s + r + j * s]);
  return o;
}
}  // namespace

Codec::Codec(int dev, const std::string& path, int precision) : device(dev), prec(precision) {
  IRT_CUDA(cudaSetDevice(dev));
  IRT_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  SafeTensorsFile st(path);
  auto get = [&](const std::string& k, size_t rank) -> const TensorView& { return st.get(k, rank); };
  const char* simt = std::getenv("IRT_CODEC_F32_SIMT");
  const bool want_tf32 = prec == IRT_PREC_F32 && !(simt && simt[0] == '1');
  // 1 / (alpha + 1e-9) in f32, the Snake epilogue's reciprocal (a correctly
  // rounded divide, as the kernels would compute it)
  auto add_inv = [&](const DevBuf& alpha, const std::vector<float>& h) {
    std::vector<float> inv(h.size());
    for (size_t i = 0; i < h.size(); ++i) inv[i] = 1.0f / (h[i] + 1e-9f);
    up_host(snake_inv[alpha.p], inv);
  };
  auto conv = [&](Conv& c, const std::string& p, int dil) {
    std::vector<long> shp;
    std::vector<float> h = conv_weight(st, p, shp);
    c.cout = (int)shp[0];
    c.cin = (int)shp[1];
    c.k = (int)shp[2];
    c.dil = dil;
    c.pad = (c.k - 1) * dil / 2;  // conv_pad(k, 1, dil) (src/codec/layers.rs:64-66)
    up_host(c.w, h);
    if (st.has(p + ".bias")) up_f32(c.b, get(p + ".bias", 1));
    if (want_tf32 && c.cout > 1) codec_pack_tf32_conv(c, h);
    if (prec == IRT_PREC_BF16 && c.cout % 32 == 0 && c.cin % 8 == 0) {
      c.cin_pad = round_up64(c.cin);
      up_bf16(c.wp, pack_conv(h, c.cout, c.cin, c.k, c.cin_pad));
    }
  };
  conv(qout, "quantizer.out_proj", 1);
  conv(stem, "decoder.model.0", 1);
  const int rates[4] = {12, 10, 8, 2};
  for (int i = 0; i < 4; ++i) {
    Block& bl = blocks[i];
    std::string p = "decoder.model." + std::to_string(i + 1);
    bl.stride = rates[i];
    add_inv(bl.alpha, up_f32(bl.alpha, get(p + ".block.0.alpha", 3)));
    std::vector<long> shp;
    std::vector<float> h = conv_weight(st, p + ".block.1", shp);  // [cin, cout, 2s]
    bl.ct.cin = (int)shp[0];
    bl.ct.cout = (int)shp[1];
    bl.ct.k = (int)shp[2];
    if (bl.ct.k != 2 * bl.stride) throw shape_error(p + ".block.1.weight kernel != 2*stride");
    bl.ct.pad = (bl.stride + 1) / 2;  // conv_transpose_pad (src/codec/layers.rs:71-75)
    up_host(bl.ct.w, h);
    if (st.has(p + ".block.1.bias")) up_f32(bl.ct.b, get(p + ".block.1.bias", 1));
    if (want_tf32) codec_pack_tf32_convt(bl.ct, h, bl.stride);
    if (prec == IRT_PREC_BF16 && bl.ct.cout % 32 == 0 && bl.ct.cin % 8 == 0 && bl.stride >= 2) {
      bl.ct.cin_pad = round_up64(bl.ct.cin);
      bl.ct.phases = bl.stride;
      up_bf16(bl.ct.wp, pack_convt(h, bl.ct.cin, bl.ct.cout, bl.stride, bl.ct.cin_pad));
    }
    const int ids[3] = {4, 5, 8}, dils[3] = {1, 3, 9};
    for (int r = 0; r < 3; ++r) {
      std::string q = p + ".block." + std::to_string(ids[r]);
      add_inv(bl.res[r].a0, up_f32(bl.res[r].a0, get(q + ".block.0.alpha", 3)));
      conv(bl.res[r].c1, q + ".block.1", dils[r]);
      add_inv(bl.res[r].a2, up_f32(bl.res[r].a2, get(q + ".block.2.alpha", 3)));
      conv(bl.res[r].c3, q + ".block.3", 1);
    }
  }
  add_inv(head_alpha, up_f32(head_alpha, get("decoder.wm_model.encoder_block.pre.0.alpha", 3)));
  conv(head, "decoder.wm_model.encoder_block.pre.1", 1);
  if (qout.cin != 32) throw shape_error("quantizer.out_proj expects 32 latent channels");
  // bf16 mode runs on the tensor-core path when every layer fits its tiling
  // (output channels multiple of 32, head width 32..128); otherwise SIMT.
  if (prec == IRT_PREC_BF16) {
    bool ok = qout.wp.p && stem.wp.p && head.k <= 7 && head.cout == 1;
    const int hc = blocks[3].ct.cout;
    ok = ok && (hc == 32 || hc == 64 || hc == 96 || hc == 128);
    for (auto& bl : blocks) {
      ok = ok && bl.ct.wp.p;
      for (auto& r : bl.res) ok = ok && r.c1.wp.p && r.c3.wp.p;
    }
    tc = ok;
  }
  tf32 = want_tf32 && codec_tf32_supported(*this);
  codec_noalloc_prepare();
}

const float* Codec::inv_of(const float* alpha) const {
  if (!alpha) return nullptr;
  auto it = snake_inv.find(alpha);
  if (it == snake_inv.end()) throw Error(IRT_E_INVALID_ARG, "codec: Snake alpha without its reciprocal table");
  return it->second.as<float>();
}

Codec::~Codec() {
  cudaSetDevice(device);
  if (stream) cudaStreamDestroy(stream);
}

namespace {
// f32 SIMT decode of a uniform batch on channel-major activations; `lat` and
// `wav` are device pointers.
void decode_simt(Codec& c, const float* lat, int B, int T, float* wav, cudaStream_t s) {
  long maxel = (long)B * T * 32;
  long t = T;
  maxel = std::max(maxel, (long)B * c.qout.cout * t);
  maxel = std::max(maxel, (long)B * c.stem.cout * t);
  for (int i = 0; i < 4; ++i) {
    t *= c.blocks[i].stride;
    maxel = std::max(maxel, (long)B * c.blocks[i].ct.cout * t);
  }
  for (auto* b : {&c.buf0, &c.buf1, &c.buf2}) b->ensure((size_t)maxel * 4 + 16);
  float* a = c.buf0.as<float>();
  float* b = c.buf1.as<float>();
  float* x = c.buf2.as<float>();
  transpose_btc_bct(lat, x, B, T, 32, s);  // [B,T,32] -> [B,32,T]
  conv1d(x, B, 32, T, c.qout.w.as<float>(), c.qout.b.as<float>(), c.qout.cout, 1, 1, 0, nullptr, nullptr, 0, a, s);
  conv1d(a, B, c.qout.cout, T, c.stem.w.as<float>(), c.stem.b.as<float>(), c.stem.cout, c.stem.k, 1, c.stem.pad,
         nullptr, nullptr, 0, b, s);
  int C = c.stem.cout;
  long cur = T;
  std::swap(a, b);  // a = current activation
  for (int i = 0; i < 4; ++i) {
    Codec::Block& bl = c.blocks[i];
    const long nt = cur * bl.stride;
    // Snake -> ConvTranspose (src/codec/decoder.rs:26-33)
    conv_transpose1d(a, B, C, (int)cur, bl.ct.w.as<float>(), bl.ct.b.as<float>(), bl.ct.cout, bl.stride, bl.ct.pad,
                     bl.alpha.as<float>(), b, (int)nt, s);
    C = bl.ct.cout;
    cur = nt;
    std::swap(a, b);
    for (int r = 0; r < 3; ++r) {
      Codec::Res& ru = bl.res[r];
      // Snake -> conv k7 dil -> Snake -> conv 1x1 -> + x  (src/codec/layers.rs:52-60)
      conv1d(a, B, C, (int)cur, ru.c1.w.as<float>(), ru.c1.b.as<float>(), C, ru.c1.k, ru.c1.dil, ru.c1.pad,
             ru.a0.as<float>(), nullptr, 0, b, s);
      conv1d(b, B, C, (int)cur, ru.c3.w.as<float>(), ru.c3.b.as<float>(), C, 1, 1, 0, ru.a2.as<float>(), a, 0, x, s);
      std::swap(a, x);
    }
  }
  // head: Snake -> conv(96 -> 1, k7) -> tanh (src/codec/decoder.rs:43-54); [B, 1, T*hop]
  conv1d(a, B, C, (int)cur, c.head.w.as<float>(), c.head.b.as<float>(), 1, c.head.k, 1, c.head.pad,
         c.head_alpha.as<float>(), nullptr, 1, wav, s);
}
}  // namespace

int codec_hop(const Codec& c) {
  int h = 1;
  for (const auto& bl : c.blocks) h *= bl.stride;
  return h;
}

void Codec::decode(const float* latent, int B, int T, float* wav, int memory, cudaStream_t user_stream,
                   const int* lengths) {
  std::lock_guard<std::mutex> lock(mu);
  IRT_CUDA(cudaSetDevice(device));
  cudaStream_t s = user_stream ? user_stream : stream;
  if (B <= 0 || T <= 0) throw shape_error("decode needs batch > 0 and frames > 0");
  bool ragged = false;
  if (lengths) {
    for (int b = 0; b < B; ++b) {
      if (lengths[b] < 0 || lengths[b] > T)
        throw shape_error("frame length " + std::to_string(lengths[b]) + " outside [0, " + std::to_string(T) + "]");
      ragged = ragged || lengths[b] != T;
    }
  }
  const long long l0 = launch_counter().load();
  const long hop = codec_hop(*this);
  const size_t lat_bytes = (size_t)B * T * 32 * 4, wav_bytes = (size_t)B * T * hop * 4;
  in.ensure(lat_bytes + 16);
  IRT_CUDA(cudaMemcpyAsync(in.p, latent, lat_bytes,
                           memory == IRT_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
  float* out = wav;
  if (memory != IRT_MEM_DEVICE) {
    wav_dev.ensure(wav_bytes + 16);
    out = wav_dev.as<float>();
  }
  if (ragged) IRT_CUDA(cudaMemsetAsync(out, 0, wav_bytes, s));
  if (tc) {
    decode_tc(in.as<float>(), B, T, ragged ? lengths : nullptr, out, s);
  } else if (tf32) {
    for (int b = 0; b < B; ++b)  // each utterance at its own length
      codec_decode_tf32(*this, in.as<float>() + (size_t)b * T * 32, ragged ? lengths[b] : T,
                        out + (size_t)b * T * hop, s);
  } else if (!ragged) {
    decode_simt(*this, in.as<float>(), B, T, out, s);
  } else {
    for (int b = 0; b < B; ++b)  // each utterance alone, at its own length
      if (lengths[b] > 0)
        decode_simt(*this, in.as<float>() + (size_t)b * T * 32, 1, lengths[b], out + (size_t)b * T * hop, s);
  }
  if (memory != IRT_MEM_DEVICE) IRT_CUDA(cudaMemcpyAsync(wav, out, wav_bytes, cudaMemcpyDeviceToHost, s));
  IRT_CUDA(cudaStreamSynchronize(s));
  if (tc && conv_tc_read_and_clear_error())
    throw Error(IRT_E_CUDA, "codec tensor-core kernel watchdog expired (pipeline stalled)");
  if (tf32 && read_and_clear_kernel_error())
    throw Error(IRT_E_CUDA, "codec tf32 GEMM watchdog expired (pipeline stalled)");
  last_launches = launch_counter().load() - l0;
}

// bf16 tensor-core decode (conv_tc.cu) of utterances laid out on one time
// axis with zero gap frames; see the layout notes there.  Utterances are
// decoded in chunks of at most CHUNK_FRAMES latent frames to bound the row
// buffers (184,320 elements per latent frame at the widest level).
void Codec::decode_tc(const float* lat, int B, int T, const int* lengths, float* wav, cudaStream_t s) {
  constexpr int GAP = 3, CHUNK_FRAMES = 4096, MIN_ROWS = 128;
  const int hop = codec_hop(*this);
  // elements per latent frame at the widest level
  long per_frame = std::max<long>(64, std::max(qout.cout, stem.cout));
  {
    long sc = 1;
    for (auto& bl : blocks) {
      sc *= bl.stride;
      per_frame = std::max(per_frame, sc * bl.ct.cout);
    }
  }
  // greedy chunks of utterances, each one time axis with gap frames
  std::vector<std::vector<int>> chunks;
  for (int b0 = 0; b0 < B;) {
    std::vector<int> fs(GAP, -1);
    int b1 = b0;
    while (b1 < B) {
      const int len = lengths ? lengths[b1] : T;
      if (b1 > b0 && (long)fs.size() + len + GAP > CHUNK_FRAMES) break;
      for (int t = 0; t < len; ++t) fs.push_back(b1 * T + t);
      fs.insert(fs.end(), GAP, -1);
      ++b1;
    }
    b0 = b1;
    while (fs.size() < (size_t)MIN_ROWS) fs.push_back(-1);
    if ((long)fs.size() * per_frame >= (1L << 31)) throw unsupported("codec decode: utterance too long for one chunk");
    chunks.push_back(std::move(fs));
  }
  size_t max_f = 0;
  for (auto& c : chunks) max_f = std::max(max_f, c.size());
  // size every buffer once, before the first launch
  frames.ensure(max_f * 4);
  rx.ensure(max_f * per_frame * 4 + 16);
  rp.ensure(max_f * per_frame * 2 + 16);
  rq.ensure(max_f * per_frame * 2 + 16);
  for (const auto& fs : chunks) {
    const int F = (int)fs.size();
    IRT_CUDA(cudaMemcpyAsync(frames.p, fs.data(), (size_t)F * 4, cudaMemcpyHostToDevice, s));
    bf16* cur = rq.as<bf16>();
    bf16* oth = rp.as<bf16>();
    float* X = rx.as<float>();
    const int* fsrc = frames.as<int>();
    pack_latent_rows(lat, fsrc, cur, F, s);  // [F, 64] bf16

    auto run = [&](const Conv& c, int rows, int cin, int scale, int convt, int stride, const float* alpha, float* x,
                   int add_res) {
      ConvTcArgs a;
      a.rows_in = rows;
      a.cin = cin;
      a.cin_pad = c.cin_pad;
      a.taps = convt ? 2 : c.k;
      a.phases = convt ? stride : 1;
      a.cout = c.cout;
      a.dil = c.dil;
      a.pad = c.pad;
      a.convt = convt;
      a.stride = convt ? stride : 1;
      a.rows_out = convt ? rows * stride : rows;
      a.out_scale = scale;
      a.frame_src = fsrc;
      a.bias = c.b.p ? c.b.as<float>() : nullptr;
      a.alpha = alpha;
      a.alpha_inv = inv_of(alpha);
      a.x = x;
      a.add_res = add_res;
      a.p = oth;
      conv_tc(cur, c.wp.as<bf16>(), a, s);
      std::swap(cur, oth);
    };
    // quantizer out_proj (1x1, 32 -> 1024), then the stem conv whose output
    // feeds block 1's Snake -> ConvTranspose
    run(qout, F, 64, 1, 0, 1, nullptr, nullptr, 0);
    run(stem, F, qout.cout, 1, 0, 1, blocks[0].alpha.as<float>(), nullptr, 0);
    int rows = F, scale = 1, C = stem.cout;
    for (int i = 0; i < 4; ++i) {
      Block& bl = blocks[i];
      scale *= bl.stride;
      // ConvTranspose: x = convT(snake(x_prev)); emits x (f32) and snake_a0(x)
      run(bl.ct, rows, C, scale, 1, bl.stride, bl.res[0].a0.as<float>(), X, 0);
      rows *= bl.stride;
      C = bl.ct.cout;
      for (int r = 0; r < 3; ++r) {
        Res& ru = bl.res[r];
        const float* next = r < 2 ? bl.res[r + 1].a0.as<float>()
                                  : (i < 3 ? blocks[i + 1].alpha.as<float>() : head_alpha.as<float>());
        run(ru.c1, rows, C, scale, 0, 1, ru.a2.as<float>(), nullptr, 0);  // snake_a2(conv_k7(.))
        run(ru.c3, rows, C, scale, 0, 1, next, X, 1);                     // x += conv_1x1(.)
      }
    }
    codec_head_rows(cur, rows, C, head.w.as<float>(), head.b.p ? head.b.as<float>() : nullptr, head.k, head.pad,
                    fsrc, hop, wav, s);
  }
}

}  // namespace irt
