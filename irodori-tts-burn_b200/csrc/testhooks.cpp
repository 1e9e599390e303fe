// Kernel-level entry points for the GPU unit tests only.  Built into a
// separate library (libirodori_b200_testhooks.so) so the product ABI in
// include/irodori_b200.h stays exactly the reference-facing surface.
#include <string>
#include <vector>

#include "codec.hpp"
#include "common.hpp"
#include "engine.hpp"
#include "kernels.hpp"
#include "lora.hpp"
#include "safetensors.hpp"

#define IRTT_API extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_err;
template <class F>
int guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const irt::Error& e) {
    g_err = e.what();
    return e.status;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 22;
  }
}
}  // namespace

IRTT_API const char* irtt_last_error() { return g_err.c_str(); }

// C[M,N] (f32) = A[M,K] . B[N,K]^T with bf16 operands; path 0 = tcgen05, 1 = SIMT.
IRTT_API int irtt_gemm_store(const void* A, const void* B, int M, int N, int K, float* C, int path) {
  return guard([&] {
    irt::EpiParams p;
    p.mode = irt::EPI_STORE;
    p.M = M;
    p.N = N;
    p.out = C;
    p.ldo = N;
    if (path == 0) {
      if (!irt::gemm_tc_supported(p, K, K, K, A, B)) throw irt::Error(4, "shape not supported by tcgen05 path");
      irt::gemm_tc(reinterpret_cast<const irt::bf16*>(A), K, reinterpret_cast<const irt::bf16*>(B), K, M, N, K, p,
                   nullptr);
    } else {
      irt::DevBuf raw((size_t)M * N * 4);
      irt::gemm_simt(A, 1, K, 0, B, 1, K, 0, raw.as<float>(), N, 0, M, N, K, 1, nullptr);
      irt::epilogue_apply(p, raw.as<float>(), N, 0, 1, nullptr);
      IRT_CUDA(cudaDeviceSynchronize());
    }
  });
}

// The SIMT GEMM as the engine calls it: batched, strided, f32 or bf16
// operands, raw f32 output (C[z][m][n] = sum_k A[z][m][k] B[z][n][k]), on the
// legacy stream without synchronising (callers check with irtt_sync_check()).
IRTT_API int irtt_gemm_simt(const void* A, int a_bf16, long lda, long a_bs, const void* B, int b_bf16, long ldb,
                            long b_bs, float* C, long ldc, long c_bs, int M, int N, int K, int batch) {
  return guard([&] {
    irt::gemm_simt(A, a_bf16, lda, a_bs, B, b_bf16, ldb, b_bs, C, ldc, c_bs, M, N, K, batch, nullptr);
  });
}

// f32 GEMM as the f32 engine runs it: path 0 = the tcgen05 tf32 hi / lo split
// product (both operands split here), 1 = SIMT + epilogue.  mode EPI_STORE
// (out = C [M, N] f32) or EPI_RESID (out = x [M, N] += gate . acc).
IRTT_API int irtt_gemm_f32(int mode, const float* A, const float* B, int M, int N, int K, int path, float* out,
                           const float* gate) {
  return guard([&] {
    irt::EpiParams p;
    p.mode = mode;
    p.M = M;
    p.N = N;
    p.out_bf16 = 0;
    if (mode == irt::EPI_RESID) {
      p.x = out;
      p.gate = gate;
    } else {
      p.out = out;
      p.ldo = N;
    }
    if (path == 0) {
      const int Kp = irt::tf32_kpad(K);
      irt::DevBuf a2((size_t)M * 2 * Kp * 4), b2((size_t)N * 2 * Kp * 4);
      if (!irt::gemm_tc_supported(p, Kp, 2L * Kp, 2L * Kp, a2.p, b2.p))
        throw irt::Error(4, "shape not supported by tcgen05 path");
      irt::split_tf32(A, K, M, K, a2.as<float>(), Kp, nullptr);
      irt::split_tf32(B, K, N, K, b2.as<float>(), Kp, nullptr);
      irt::gemm_tc_tf32x3(a2.as<float>(), 2L * Kp, b2.as<float>(), 2L * Kp, M, N, Kp, p, nullptr);
      IRT_CUDA(cudaDeviceSynchronize());
      if (irt::read_and_clear_kernel_error()) throw irt::Error(20, "GEMM watchdog fired");
    } else {
      irt::DevBuf raw((size_t)M * N * 4);
      irt::gemm_simt(A, 0, K, 0, B, 0, K, 0, raw.as<float>(), N, 0, M, N, K, 1, nullptr);
      irt::epilogue_apply(p, raw.as<float>(), N, 0, 1, nullptr);
      IRT_CUDA(cudaDeviceSynchronize());
    }
  });
}

// The tf32 hi / lo GEMM on operands already split (A2 [M, 2 Kp], B2 [N, 2 Kp]):
// mode EPI_STORE (out = C [M, N] f32) or EPI_RESID (out = x += gate . acc), on
// the legacy stream without synchronising (profiling loops; check with
// irtt_sync_check()).
IRTT_API int irtt_gemm_tf32x3_async(int mode, const float* A2, const float* B2, int M, int N, int Kp, float* out,
                                    const float* gate) {
  return guard([&] {
    irt::EpiParams p;
    p.mode = mode;
    p.M = M;
    p.N = N;
    p.out_bf16 = 0;
    if (mode == irt::EPI_RESID) {
      p.x = out;
      p.gate = gate;
    } else {
      p.out = out;
      p.ldo = N;
    }
    irt::gemm_tc_tf32x3(A2, 2L * Kp, B2, 2L * Kp, M, N, Kp, p, nullptr);
  });
}

// Fused-epilogue GEMM for the QKVG / SWIGLU / RESID modes with bf16 operands.
IRTT_API int irtt_gemm_epi(int mode, const void* A, const void* B, int M, int N, int K, int path, void* o0, void* o1,
                           void* o2, void* o3, const float* w0, const float* w1, const float* cos_t,
                           const float* sin_t, const int* tok_pos, int H, int hd, int rope_heads, float* x,
                           const float* gate, int F) {
  return guard([&] {
    irt::EpiParams p;
    p.mode = mode;
    p.M = M;
    p.N = N;
    p.out_bf16 = 1;
    p.q = o0; p.k = o1; p.v = o2; p.g = o3;
    p.qn_w = w0; p.kn_w = w1;
    p.rope_cos = cos_t; p.rope_sin = sin_t;
    p.tok_pos = tok_pos;
    p.H = H; p.hd = hd; p.rope_heads = rope_heads; p.Dq = H * hd;
    p.x = x;
    p.gate = gate;
    p.h = o0;
    p.F = F;
    if (path == 0) {
      if (!irt::gemm_tc_supported(p, K, K, K, A, B)) throw irt::Error(4, "shape not supported by tcgen05 path");
      irt::gemm_tc(reinterpret_cast<const irt::bf16*>(A), K, reinterpret_cast<const irt::bf16*>(B), K, M, N, K, p,
                   nullptr);
    } else {
      irt::DevBuf raw((size_t)M * N * 4);
      irt::gemm_simt(A, 1, K, 0, B, 1, K, 0, raw.as<float>(), N, 0, M, N, K, 1, nullptr);
      irt::epilogue_apply(p, raw.as<float>(), N, 0, 1, nullptr);
      IRT_CUDA(cudaDeviceSynchronize());
    }
  });
}

// Attention over per-sequence [self | context] keys; seqs is a host array of
// nseq x {tok_start, len, ctx_off, ctx_len}.
IRTT_API int irtt_attention(const void* q, const void* k, const void* v, const void* g, const void* ck,
                            const void* cv, const uint8_t* key_mask, const int* seqs_host, int nseq, int H, int hd,
                            void* out, int bf16_io, int rows, int ctx_rows, int path) {
  return guard([&] {
    std::vector<irt::SeqDesc> sd(nseq);
    int mx = 0;
    for (int i = 0; i < nseq; ++i) {
      sd[i] = {seqs_host[4 * i], seqs_host[4 * i + 1], seqs_host[4 * i + 2], seqs_host[4 * i + 3]};
      mx = std::max(mx, sd[i].len);
    }
    irt::DevBuf d(sizeof(irt::SeqDesc) * std::max(1, nseq));
    IRT_CUDA(cudaMemcpy(d.p, sd.data(), sizeof(irt::SeqDesc) * nseq, cudaMemcpyHostToDevice));
    irt::AttnParams p{};
    p.q = q; p.k = k; p.v = v; p.gsig = g; p.ck = ck; p.cv = cv; p.key_mask = key_mask;
    p.seqs = d.as<irt::SeqDesc>();
    p.nseq = nseq; p.max_len = mx; p.H = H; p.hd = hd;
    p.scale = 1.0f / sqrtf((float)hd);
    p.out = out;
    p.rows = rows;
    p.ctx_rows = ctx_rows;
    p.path = path;
    if (path == 0 && bf16_io && !irt::attention_tc_supported(p)) throw irt::Error(4, "tcgen05 attention unsupported");
    irt::attention(p, bf16_io, nullptr);
    IRT_CUDA(cudaDeviceSynchronize());
    if (irt::read_and_clear_attn_error()) throw irt::Error(20, "attention watchdog fired");
  });
}

// Same as irtt_attention without the synchronisation (profiling loops): the
// sequence table is uploaded once per distinct table and kept; check the
// watchdog with irtt_sync_check() afterwards.
IRTT_API int irtt_attention_async(const void* q, const void* k, const void* v, const void* g, const void* ck,
                                  const void* cv, const uint8_t* key_mask, const int* seqs_host, int nseq, int H,
                                  int hd, void* out, int bf16_io, int rows, int ctx_rows, int path) {
  return guard([&] {
    static irt::DevBuf d;
    static std::vector<int> cached;
    std::vector<int> tab(seqs_host, seqs_host + 4 * nseq);
    int mx = 0;
    for (int i = 0; i < nseq; ++i) mx = std::max(mx, seqs_host[4 * i + 1]);
    if (tab != cached) {
      d.ensure(sizeof(irt::SeqDesc) * std::max(1, nseq));
      IRT_CUDA(cudaMemcpy(d.p, tab.data(), sizeof(int) * tab.size(), cudaMemcpyHostToDevice));
      cached = tab;
    }
    irt::AttnParams p{};
    p.q = q; p.k = k; p.v = v; p.gsig = g; p.ck = ck; p.cv = cv; p.key_mask = key_mask;
    p.seqs = d.as<irt::SeqDesc>();
    p.nseq = nseq; p.max_len = mx; p.H = H; p.hd = hd;
    p.scale = 1.0f / sqrtf((float)hd);
    p.out = out;
    p.rows = rows;
    p.ctx_rows = ctx_rows;
    p.path = path;
    if (path == 0 && bf16_io && !irt::attention_tc_supported(p)) throw irt::Error(4, "tcgen05 attention unsupported");
    irt::attention(p, bf16_io, nullptr);
  });
}

// PEFT LoRA merge on the host (lora.hpp: the routine the engine runs when it
// loads base + adapter): tensor `name` of the merged checkpoint decoded to f32
// into out (n values), and the number of merged tensors in *merged.  Needs no
// GPU.
IRTT_API int irtt_lora_merged_tensor(const char* base_path, const char* adapter_dir, const char* name, float* out,
                                     long n, int* merged) {
  return guard([&] {
    irt::SafeTensorsFile st(base_path);
    const std::vector<std::string> m = irt::apply_lora(st, adapter_dir);
    const irt::TensorView& v = st.get(name);
    if ((long)v.numel() != n) throw irt::Error(IRT_E_INVALID_ARG, "size mismatch for " + std::string(name));
    irt::decode_to_f32(v, out);
    if (merged) *merged = (int)m.size();
  });
}

IRTT_API long long irtt_launch_count() { return irt::launch_counter().load(); }

// Synchronise the device and report the GEMM pipeline watchdog flag.
IRTT_API int irtt_sync_check() {
  return guard([&] {
    IRT_CUDA(cudaDeviceSynchronize());
    if (irt::read_and_clear_kernel_error()) throw irt::Error(20, "pipeline watchdog fired");
  });
}

// Bounded-wait probe: which = 0 GEMM, 1 attention, 2 conv translation unit.
// Launches a kernel whose mbarrier waits (the kernels' own bounded wait) wait
// on a barrier nothing arrives on, with the limit shortened to limit_ns; the
// first wait expires and sets the unit's watchdog flag, the later ones give
// up at once.  *elapsed_ns = device time of all waits.  The flag is left set:
// the caller checks that it is reported (irtt_sync_check / the watchdog read)
// and then cleared.
IRTT_API int irtt_watchdog_probe(int which, unsigned long long limit_ns, int waits, unsigned long long* elapsed_ns) {
  return guard([&] {
    if (which == 0) irt::gemm_watchdog_probe(limit_ns, waits, elapsed_ns);
    else if (which == 1) irt::attn_watchdog_probe(limit_ns, waits, elapsed_ns);
    else if (which == 2) irt::conv_watchdog_probe(limit_ns, waits, elapsed_ns);
    else throw irt::Error(IRT_E_INVALID_ARG, "which must be 0, 1 or 2");
  });
}

// Reads and clears the watchdog flag of one translation unit (0 GEMM,
// 1 attention, 2 conv); returns the flag's value or -1 on a bad index.
IRTT_API int irtt_watchdog_read_and_clear(int which) {
  if (which == 0) return irt::read_and_clear_kernel_error();
  if (which == 1) return irt::read_and_clear_attn_error();
  if (which == 2) return irt::conv_tc_read_and_clear_error();
  return -1;
}

// adaLN modulate rows (ops.cu): h = x / sqrt(mean(x^2) + eps) * (1 + scale) +
// shift, f32 in, bf16 or f32 out; device pointers, asynchronous (check with
// irtt_sync_check()).
IRTT_API int irtt_adaln_modulate(const float* x, const float* shift, const float* scale, void* h, int out_bf16, int M,
                                 int D, float eps) {
  return guard([&] { irt::adaln_modulate(x, shift, scale, h, out_bf16, M, D, eps, nullptr); });
}

// One implicit-GEMM convolution of the bf16 codec path (conv_tc.cu); all
// pointers are device memory, w packed [phases][cout][taps][cin_pad] bf16.
IRTT_API int irtt_conv_tc(const void* in, int rows_in, int cin, const void* w, int cin_pad, int taps, int phases,
                          int cout, int dil, int pad, int convt, int stride, int rows_out, int out_scale,
                          const int* frame_src, const float* bias, const float* alpha, float* x, int add_res,
                          void* p) {
  return guard([&] {
    irt::ConvTcArgs a;
    a.rows_in = rows_in;
    a.cin = cin;
    a.cin_pad = cin_pad;
    a.taps = taps;
    a.phases = phases;
    a.cout = cout;
    a.dil = dil;
    a.pad = pad;
    a.convt = convt;
    a.stride = stride;
    a.rows_out = rows_out;
    a.out_scale = out_scale;
    a.frame_src = frame_src;
    a.bias = bias;
    a.alpha = alpha;
    // 1 / (alpha + 1e-9) per channel, as the codec uploads it at load
    irt::DevBuf inv;
    if (alpha) {
      std::vector<float> h(cout);
      IRT_CUDA(cudaMemcpy(h.data(), alpha, (size_t)cout * 4, cudaMemcpyDeviceToHost));
      for (auto& v : h) v = 1.0f / (v + 1e-9f);
      inv.alloc((size_t)cout * 4);
      IRT_CUDA(cudaMemcpy(inv.p, h.data(), (size_t)cout * 4, cudaMemcpyHostToDevice));
      a.alpha_inv = inv.as<float>();
    }
    a.x = x;
    a.add_res = add_res;
    a.p = reinterpret_cast<irt::bf16*>(p);
    irt::conv_tc(reinterpret_cast<const irt::bf16*>(in), reinterpret_cast<const irt::bf16*>(w), a, nullptr);
    IRT_CUDA(cudaDeviceSynchronize());
    if (irt::conv_tc_read_and_clear_error()) throw irt::Error(20, "conv_tc watchdog fired");
  });
}

// Runs one sample() of a fresh engine and captures the f32 residual stream of
// its first DiT forward: after in_proj and after each of the L blocks, for all
// packed rows (CFG groups x utterance frames).  dump: device [(L + 1) * cap * D].
// Returns the captured row count in *rows.  The latent output goes to out_host.
IRTT_API int irtt_sample_dump_layers(const char* ckpt, int precision, const irt_sampler_params* sp,
                                     const irt_request* rq, float* out_host, float* dump, int cap, int* rows) {
  return guard([&] {
    irt::Engine e(0, ckpt, precision);
    irt::validate_sampler_params(*sp);
    e.params = *sp;
    e.has_params = true;
    e.dump_layers = dump;
    e.dump_rows_cap = cap;
    e.sample(*rq, out_host, IRT_MEM_HOST, nullptr);
    IRT_CUDA(cudaDeviceSynchronize());
    *rows = e.dump_rows;
  });
}
