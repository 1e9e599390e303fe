// Engine implementation: checkpoint upload + packing, condition encoders,
// context KV cache, precomputed adaLN tables, DiT forward and the RF sampler.
#include "engine.hpp"
#include "lora.hpp"

#include <algorithm>
#include <cmath>
#include <numeric>

#include "safetensors.hpp"

namespace irt {

// ---------------------------------------------------------------------------
// Device-side conversion of checkpoint tensors into packed layouts
// ---------------------------------------------------------------------------
namespace {

__global__ void convert_rows_kernel(const void* src, int sdt, long rows, long cols, void* dst, int dbf, long dld,
                                    long group, long gstride, long off) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  long r = i / cols, c = i % cols;
  float v;
  if (sdt == 0) v = reinterpret_cast<const float*>(src)[i];
  else if (sdt == 1) v = __bfloat162float(reinterpret_cast<const bf16*>(src)[i]);
  else v = __half2float(reinterpret_cast<const __half*>(src)[i]);
  long dr = (r / group) * gstride + (r % group) + off;
  if (dbf) reinterpret_cast<bf16*>(dst)[dr * dld + c] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(dst)[dr * dld + c] = v;
}

__global__ void tokpos_kernel(int* pos, const int* utt_off, const int* utt_len, int nutt, int ntok, int total) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int r = i % ntok;
  int lo = 0, hi = nutt - 1;
  while (lo < hi) {  // last utterance with off <= r
    int mid = (lo + hi + 1) / 2;
    if (utt_off[mid] <= r) lo = mid; else hi = mid - 1;
  }
  pos[i] = r - utt_off[lo];
}

struct Staging {
  DevBuf buf;
};

int sdt_of(const TensorView& v) { return v.dtype == DType::F32 ? 0 : v.dtype == DType::BF16 ? 1 : 2; }

void upload_rows(Staging& stg, const TensorView& v, void* dst, int dbf, long dld, long group, long gstride, long off) {
  long rows = v.shape.empty() ? 1 : v.shape[0];
  long cols = rows ? v.numel() / rows : 0;
  if (v.numel() == 0) return;
  stg.buf.ensure(v.nbytes);
  IRT_CUDA(cudaMemcpy(stg.buf.p, v.data, v.nbytes, cudaMemcpyHostToDevice));
  long n = rows * cols;
  convert_rows_kernel<<<(unsigned)((n + 255) / 256), 256>>>(stg.buf.p, sdt_of(v), rows, cols, dst, dbf, dld,
                                                             group > 0 ? group : rows, gstride, off);
  IRT_CHECK_LAUNCH();
}

void check_shape(const std::string& k, const TensorView& v, std::initializer_list<long> want) {
  std::vector<long> w(want);
  bool ok = v.shape.size() == w.size();
  for (size_t i = 0; ok && i < w.size(); ++i) ok = v.shape[i] == w[i];
  if (!ok) {
    std::string got, exp;
    for (auto d : v.shape) got += std::to_string(d) + ",";
    for (auto d : w) exp += std::to_string(d) + ",";
    throw shape_error("tensor '" + k + "' has shape [" + got + "] but the config implies [" + exp + "]");
  }
}

// f32 host RoPE tables, precompute_rope_freqs (src/model/rope.rs:24-63).
void rope_tables_host(int hd, int S, std::vector<float>& cs, std::vector<float>& sn) {
  int half = hd / 2;
  cs.assign((size_t)S * half, 0.f);
  sn.assign((size_t)S * half, 0.f);
  std::vector<float> fr(half);
  for (int i = 0; i < half; ++i) fr[i] = 1.0f / std::pow(10000.0f, (2.0f * (float)i) / (float)hd);
  for (int s = 0; s < S; ++s)
    for (int i = 0; i < half; ++i) {
      float a = (float)s * fr[i];
      cs[(size_t)s * half + i] = std::cos(a);
      sn[(size_t)s * half + i] = std::sin(a);
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// Construction / weight loading
// ---------------------------------------------------------------------------

Engine::Engine(int dev, const std::string& path, int precision, const std::string& adapter_dir)
    : device(dev), prec(precision) {
  if (precision != IRT_PREC_BF16 && precision != IRT_PREC_F32) throw Error(IRT_E_INVALID_ARG, "invalid precision");
  bf = precision == IRT_PREC_BF16;
  use_graphs = std::getenv("IRT_NO_GRAPHS") == nullptr;
  IRT_CUDA(cudaSetDevice(dev));
  IRT_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  load(path, adapter_dir);
  const char* simt = std::getenv("IRT_F32_SIMT");
  tf32 = !bf && !(simt && simt[0] == '1');
  if (tf32) prepare_tf32();
}

// f32 mode: the tf32 hi / lo copy of each GEMM weight that can meet 128 or
// more rows (encoder blocks and in_proj, DiT blocks and in_proj, context KV
// projections; the cond_module runs on one row per timestep and stays SIMT).
// Built after the adapter merge, from the merged weights.
void Engine::prepare_tf32() {
  auto add = [&](const DevBuf& W, int N, int K) {
    if (!W.p || N <= 0 || K <= 0 || (K % 4)) return;
    const int Kp = tf32_kpad(K);
    DevBuf b((size_t)N * 2 * Kp * 4);
    split_tf32(W.as<float>(), K, N, K, b.as<float>(), Kp, stream);
    w_tf32.emplace(W.p, std::move(b));
  };
  for (EncoderW* e : {&text_enc, &aux_enc}) {
    if (!e->dim) continue;
    if (e->in_dim > 0) add(e->in_w, e->dim, e->in_dim);
    for (auto& b : e->blk) {
      add(b.wqkvg, 4 * e->dim, e->dim);
      add(b.wo, e->dim, e->dim);
      add(b.w13, 2 * e->Fp, e->dim);
      add(b.w2, e->dim, e->F);
    }
  }
  add(in_w, D, Kin);
  for (auto& b : blk) {
    add(b.wqkvg, 4 * D, D);
    add(b.wo, D, D);
    add(b.w13, 2 * Fp, D);
    add(b.w2, D, F);
  }
  if (ctx_text_w.p) add(ctx_text_w, L * 2 * D, (int)cfg.text_dim);
  if (ctx_aux_w.p && aux_dim > 0) add(ctx_aux_w, L * 2 * D, aux_dim);
  IRT_CUDA(cudaStreamSynchronize(stream));
}

Engine::~Engine() {
  cudaSetDevice(device);
  for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
  if (stream) cudaStreamDestroy(stream);
}

void Engine::load_encoder(const SafeTensorsFile& st, EncoderW& e, const std::string& prefix, int dim, int heads,
                          int layers, double ratio, bool embedding, int vocab, int in_dim) {
  Staging stg;
  e.dim = dim;
  e.heads = heads;
  e.hd = dim / heads;
  e.layers = layers;
  e.F = (int)ModelConfig::hidden(dim, ratio);
  e.Fp = (e.F + SWIGLU_GROUP - 1) / SWIGLU_GROUP * SWIGLU_GROUP;
  e.vocab = vocab;
  e.in_dim = in_dim;
  const size_t es = esz();
  auto lin = [&](const std::string& k, long out, long in) -> const TensorView& {
    const TensorView& v = st.get(k, 2);
    check_shape(k, v, {out, in});
    return v;
  };
  auto vec = [&](DevBuf& dst, const std::string& k, std::initializer_list<long> shape) {
    const TensorView& v = st.get(k, shape.size());
    check_shape(k, v, shape);
    dst.alloc(v.numel() * 4);
    upload_rows(stg, v, dst.p, 0, v.numel() / (v.shape.empty() ? 1 : v.shape[0]), 0, 0, 0);
  };
  if (embedding) {
    const TensorView& v = lin(prefix + ".text_embedding.weight", vocab, dim);
    e.emb.alloc((size_t)vocab * dim * 4);
    upload_rows(stg, v, e.emb.p, 0, dim, 0, 0, 0);
  } else {
    const TensorView& v = lin(prefix + ".in_proj.weight", dim, in_dim);
    e.in_w.alloc((size_t)dim * in_dim * es);
    upload_rows(stg, v, e.in_w.p, bf, in_dim, 0, 0, 0);
    vec(e.in_b, prefix + ".in_proj.bias", {dim});
  }
  e.blk.resize(layers);
  for (int i = 0; i < layers; ++i) {
    auto& b = e.blk[i];
    std::string p = prefix + ".blocks." + std::to_string(i);
    vec(b.attn_norm, p + ".attention_norm.weight", {dim});
    vec(b.mlp_norm, p + ".mlp_norm.weight", {dim});
    b.wqkvg.alloc((size_t)4 * dim * dim * es);
    const char* names[4] = {"wq", "wk", "wv", "gate"};
    for (int j = 0; j < 4; ++j)
      upload_rows(stg, lin(p + ".attention." + names[j] + ".weight", dim, dim), b.wqkvg.p, bf, dim, 0, 0,
                  (long)j * dim);
    vec(b.qn, p + ".attention.q_norm.weight", {heads, dim / heads});
    vec(b.kn, p + ".attention.k_norm.weight", {heads, dim / heads});
    b.wo.alloc((size_t)dim * dim * es);
    upload_rows(stg, lin(p + ".attention.wo.weight", dim, dim), b.wo.p, bf, dim, 0, 0, 0);
    b.w13.alloc((size_t)2 * e.Fp * dim * es);
    IRT_CUDA(cudaMemset(b.w13.p, 0, b.w13.bytes));
    upload_rows(stg, lin(p + ".mlp.w1.weight", e.F, dim), b.w13.p, bf, dim, SWIGLU_GROUP, 2 * SWIGLU_GROUP, 0);
    upload_rows(stg, lin(p + ".mlp.w3.weight", e.F, dim), b.w13.p, bf, dim, SWIGLU_GROUP, 2 * SWIGLU_GROUP,
                SWIGLU_GROUP);
    b.w2.alloc((size_t)dim * e.F * es);
    upload_rows(stg, lin(p + ".mlp.w2.weight", dim, e.F), b.w2.p, bf, e.F, 0, 0, 0);
  }
}

void Engine::load(const std::string& path, const std::string& adapter_dir) {
  SafeTensorsFile st(path);
  if (!adapter_dir.empty()) lora_merged = (int)apply_lora(st, adapter_dir).size();
  const std::string* cj = st.meta("config_json");
  if (!cj) throw Error(IRT_E_NO_CONFIG, "Checkpoint is missing the 'config_json' metadata key");
  cfg = ModelConfig::from_json(*cj);
  cfg.validate();
  D = (int)cfg.model_dim;
  L = (int)cfg.num_layers;
  H = (int)cfg.num_heads;
  hd = D / H;
  P = (int)cfg.patched_latent_dim();
  F = (int)ModelConfig::hidden(D, cfg.mlp_ratio);
  Fp = (F + SWIGLU_GROUP - 1) / SWIGLU_GROUP * SWIGLU_GROUP;
  R = (int)cfg.adaln_rank_eff();
  Temb = (int)cfg.timestep_embed_dim;
  if (Temb % 2) throw config_error("timestep embedding dim must be even");
  const size_t es = esz();
  Staging stg;

  // condition encoders (src/weights/record_builders.rs:278-300)
  load_encoder(st, text_enc, "text_encoder", (int)cfg.text_dim, (int)cfg.text_heads, (int)cfg.text_layers,
               cfg.text_mlp_ratio_(), true, (int)cfg.text_vocab_size, 0);
  {
    const TensorView& v = st.get("text_norm.weight", 1);
    check_shape("text_norm.weight", v, {cfg.text_dim});
    text_enc.out_norm.alloc(v.numel() * 4);
    upload_rows(stg, v, text_enc.out_norm.p, 0, 1, 0, 0, 0);
  }
  std::string aux_suffix;
  if (cfg.use_speaker_condition()) {
    aux_kind = 1;
    aux_dim = (int)*cfg.speaker_dim;
    aux_suffix = "speaker";
    load_encoder(st, aux_enc, "speaker_encoder", aux_dim, (int)*cfg.speaker_heads, (int)*cfg.speaker_layers,
                 cfg.speaker_mlp_ratio_(), false, 0, (int)cfg.speaker_patched_latent_dim());
    const TensorView& v = st.get("speaker_norm.weight", 1);
    check_shape("speaker_norm.weight", v, {aux_dim});
    aux_enc.out_norm.alloc(v.numel() * 4);
    upload_rows(stg, v, aux_enc.out_norm.p, 0, 1, 0, 0, 0);
  } else if (cfg.use_caption_condition) {
    aux_kind = 2;
    aux_dim = (int)cfg.caption_dim_();
    aux_suffix = "caption";
    load_encoder(st, aux_enc, "caption_encoder", aux_dim, (int)cfg.caption_heads_(), (int)cfg.caption_layers_(),
                 cfg.caption_mlp_ratio_(), true, (int)cfg.caption_vocab_size_(), 0);
    const TensorView& v = st.get("caption_norm.weight", 1);
    check_shape("caption_norm.weight", v, {aux_dim});
    aux_enc.out_norm.alloc(v.numel() * 4);
    upload_rows(stg, v, aux_enc.out_norm.p, 0, 1, 0, 0, 0);
  }

  auto lin = [&](const std::string& k, long out, long in) -> const TensorView& {
    const TensorView& v = st.get(k, 2);
    check_shape(k, v, {out, in});
    return v;
  };
  auto f32vec = [&](DevBuf& dst, const std::string& k, long n) {
    const TensorView& v = st.get(k, 1);
    check_shape(k, v, {n});
    dst.alloc(n * 4);
    upload_rows(stg, v, dst.p, 0, 1, 0, 0, 0);
  };

  // cond_module (f32 always; tiny and precision-relevant)
  cm0.alloc((size_t)D * Temb * 4);
  upload_rows(stg, lin("cond_module.linear0.weight", D, Temb), cm0.p, 0, Temb, 0, 0, 0);
  cm1.alloc((size_t)D * D * 4);
  upload_rows(stg, lin("cond_module.linear1.weight", D, D), cm1.p, 0, D, 0, 0, 0);
  cm2.alloc((size_t)3 * D * D * 4);
  upload_rows(stg, lin("cond_module.linear2.weight", 3 * D, D), cm2.p, 0, D, 0, 0, 0);

  Pk = (bf && P % 64) ? (P + 63) / 64 * 64 : P;
  Kin = bf ? 2 * Pk : Pk;
  in_w.alloc((size_t)D * Kin * es);
  IRT_CUDA(cudaMemset(in_w.p, 0, (size_t)D * Kin * es));  // zero K padding
  upload_rows(stg, lin("in_proj.weight", D, P), in_w.p, bf, Kin, 0, 0, 0);
  if (bf)  // the same weight again under the lo half of the operand
    upload_rows(stg, lin("in_proj.weight", D, P), static_cast<uint8_t*>(in_w.p) + (size_t)Pk * es, bf, Kin, 0, 0, 0);
  f32vec(in_b, "in_proj.bias", D);

  const char* kinds[3] = {"shift", "scale", "gate"};
  const char* ada_names[2] = {"attention_adaln", "mlp_adaln"};
  for (int k = 0; k < 3; ++k) {
    ada_down[k].alloc((size_t)L * 2 * R * D * 4);
    ada_up[k].alloc((size_t)L * 2 * D * R * 4);
    ada_upb[k].alloc((size_t)L * 2 * D * 4);
  }
  blk.resize(L);
  ctx_text_w.alloc((size_t)L * 2 * D * cfg.text_dim * es);
  if (aux_kind) ctx_aux_w.alloc((size_t)L * 2 * D * aux_dim * es);
  kn_all.alloc((size_t)L * D * 4);
  for (int i = 0; i < L; ++i) {
    std::string p = "blocks." + std::to_string(i);
    auto& b = blk[i];
    b.wqkvg.alloc((size_t)4 * D * D * es);
    const char* qn[4] = {"wq", "wk", "wv", "gate"};
    for (int j = 0; j < 4; ++j)
      upload_rows(stg, lin(p + ".attention." + qn[j] + ".weight", D, D), b.wqkvg.p, bf, D, 0, 0, (long)j * D);
    b.qn.alloc((size_t)D * 4);
    {
      const TensorView& v = st.get(p + ".attention.q_norm.weight", 2);
      check_shape(p + ".attention.q_norm.weight", v, {H, hd});
      upload_rows(stg, v, b.qn.p, 0, hd, 0, 0, 0);
    }
    b.kn.alloc((size_t)D * 4);
    {
      const TensorView& v = st.get(p + ".attention.k_norm.weight", 2);
      check_shape(p + ".attention.k_norm.weight", v, {H, hd});
      upload_rows(stg, v, b.kn.p, 0, hd, 0, 0, 0);
      upload_rows(stg, v, kn_all.p, 0, hd, 0, 0, (long)i * H);
    }
    b.wo.alloc((size_t)D * D * es);
    upload_rows(stg, lin(p + ".attention.wo.weight", D, D), b.wo.p, bf, D, 0, 0, 0);
    b.w13.alloc((size_t)2 * Fp * D * es);
    IRT_CUDA(cudaMemset(b.w13.p, 0, b.w13.bytes));
    upload_rows(stg, lin(p + ".mlp.w1.weight", F, D), b.w13.p, bf, D, SWIGLU_GROUP, 2 * SWIGLU_GROUP, 0);
    upload_rows(stg, lin(p + ".mlp.w3.weight", F, D), b.w13.p, bf, D, SWIGLU_GROUP, 2 * SWIGLU_GROUP, SWIGLU_GROUP);
    b.w2.alloc((size_t)D * F * es);
    upload_rows(stg, lin(p + ".mlp.w2.weight", D, F), b.w2.p, bf, F, 0, 0, 0);
    // context K/V projections, stacked per layer [Wk; Wv] (src/model/attention.rs:431-501)
    upload_rows(stg, lin(p + ".attention.wk_text.weight", D, cfg.text_dim), ctx_text_w.p, bf, cfg.text_dim, 0, 0,
                (long)i * 2 * D);
    upload_rows(stg, lin(p + ".attention.wv_text.weight", D, cfg.text_dim), ctx_text_w.p, bf, cfg.text_dim, 0, 0,
                (long)i * 2 * D + D);
    if (aux_kind) {
      upload_rows(stg, lin(p + ".attention.wk_" + aux_suffix + ".weight", D, aux_dim), ctx_aux_w.p, bf, aux_dim, 0,
                  0, (long)i * 2 * D);
      upload_rows(stg, lin(p + ".attention.wv_" + aux_suffix + ".weight", D, aux_dim), ctx_aux_w.p, bf, aux_dim, 0,
                  0, (long)i * 2 * D + D);
    }
    for (int a = 0; a < 2; ++a) {
      int z = i * 2 + a;
      for (int k = 0; k < 3; ++k) {
        std::string q = p + "." + ada_names[a] + "." + kinds[k];
        upload_rows(stg, lin(q + "_down.weight", R, D), ada_down[k].p, 0, D, 0, 0, (long)z * R);
        upload_rows(stg, lin(q + "_up.weight", D, R), ada_up[k].p, 0, R, 0, 0, (long)z * D);
        const TensorView& bv = st.get(q + "_up.bias", 1);
        check_shape(q + "_up.bias", bv, {D});
        upload_rows(stg, bv, reinterpret_cast<float*>(ada_upb[k].p) + (long)z * D, 0, 1, 0, 0, 0);
      }
    }
  }
  f32vec(out_norm, "out_norm.weight", D);
  out_w.alloc((size_t)P * D * es);
  upload_rows(stg, lin("out_proj.weight", P, D), out_w.p, bf, D, 0, 0, 0);
  if (bf && P <= 128) {
    out_split = rms_norm_split_supported(D);
    const size_t kw = out_split ? 2 * (size_t)D : (size_t)D;  // [W | W] along K when split
    out_w_pad.alloc(128 * kw * es);
    IRT_CUDA(cudaMemset(out_w_pad.p, 0, 128 * kw * es));
    for (int part = 0; part < (out_split ? 2 : 1); ++part)
      IRT_CUDA(cudaMemcpy2D(static_cast<uint8_t*>(out_w_pad.p) + (size_t)part * D * es, kw * es, out_w.p,
                            (size_t)D * es, (size_t)D * es, P, cudaMemcpyDeviceToDevice));
  }
  f32vec(out_b, "out_proj.bias", P);
  IRT_CUDA(cudaDeviceSynchronize());
}

// ---------------------------------------------------------------------------
// GEMM dispatch: tcgen05 kernel for bf16 operands when the shape allows it,
// else the SIMT kernel + standalone epilogue.
// ---------------------------------------------------------------------------
void Engine::gemm(const void* A, long lda, const DevBuf& W, int M, int N, int K, EpiParams p, cudaStream_t s) {
  p.M = M;
  p.N = N;
  if (M <= 0 || N <= 0) return;
  if (bf && gemm_tc_supported(p, K, lda, K, A, W.p)) {
    gemm_tc(reinterpret_cast<const bf16*>(A), lda, W.as<bf16>(), K, M, N, K, p, s);
    return;
  }
  if (tf32) {
    const auto it = w_tf32.find(W.p);
    const int Kp = tf32_kpad(K);
    if (it != w_tf32.end() && (lda % 4) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
        gemm_tc_supported(p, Kp, 2L * Kp, 2L * Kp, A, it->second.p)) {
      ws.a2.ensure((size_t)M * 2 * Kp * 4);
      split_tf32(static_cast<const float*>(A), lda, M, K, ws.a2.as<float>(), Kp, s);
      gemm_tc_tf32x3(ws.a2.as<float>(), 2L * Kp, it->second.as<float>(), 2L * Kp, M, N, Kp, p, s);
      return;
    }
  }
  ws.raw.ensure((size_t)M * N * 4);
  gemm_simt(A, bf, lda, 0, W.p, bf, K, 0, ws.raw.as<float>(), N, 0, M, N, K, 1, s);
  epilogue_apply(p, ws.raw.as<float>(), N, 0, 1, s);
}

// ---------------------------------------------------------------------------
// Condition encoders (src/model/text_encoder.rs:127-148,
// src/model/speaker_encoder.rs:141-162): pre-norm TextBlocks with full RoPE,
// key-padding mask, re-mask after every block.  `out_state_f32` receives the
// final RMSNorm'd state [B*T, dim] in f32.
// ---------------------------------------------------------------------------
void Engine::run_encoder(EncoderW& e, int B, int T, const void* input, bool from_ids, const uint8_t* d_mask,
                         const float* d_maskf, void* out_state_f32, cudaStream_t s) {
  const int M = B * T, dim = e.dim;
  const float eps = (float)cfg.norm_eps;
  if (M == 0) return;
  ws.ex.ensure((size_t)M * dim * 4);
  ws.eh.ensure((size_t)M * dim * esz());
  ws.eq.ensure((size_t)M * dim * esz());
  ws.ek.ensure((size_t)M * dim * esz());
  ws.ev.ensure((size_t)M * dim * esz());
  ws.eg.ensure((size_t)M * dim * esz());
  ws.eattn.ensure((size_t)M * dim * esz());
  ws.ehm.ensure((size_t)M * e.F * esz());
  float* x = ws.ex.as<float>();
  if (from_ids) {
    embed_rows_v(reinterpret_cast<const int*>(input), d_mask, e.emb.as<float>(), x, M, dim, e.vocab, s);
  } else {
    // in_proj(latent) / 6, then hard-mask (src/model/speaker_encoder.rs:146-152)
    EpiParams p;
    p.mode = EPI_STORE;
    p.out = x;
    p.ldo = dim;
    p.bias = e.in_b.as<float>();
    p.alpha = 1.f / 6.f;
    p.row_scale = d_maskf;
    gemm(input, e.in_dim, e.in_w, M, dim, e.in_dim, p, s);
  }
  // RoPE tables over T positions
  std::vector<float> cs, sn;
  rope_tables_host(e.hd, T, cs, sn);
  ws.rope_cos.ensure(cs.size() * 4 + 4);
  ws.rope_sin.ensure(sn.size() * 4 + 4);
  IRT_CUDA(cudaMemcpyAsync(ws.rope_cos.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, s));
  IRT_CUDA(cudaMemcpyAsync(ws.rope_sin.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, s));
  // sequences: one per batch row
  std::vector<SeqDesc> seqs(B);
  std::vector<int> tok(M);
  for (int b = 0; b < B; ++b) {
    seqs[b] = {b * T, T, 0, 0};
    for (int i = 0; i < T; ++i) tok[b * T + i] = i;
  }
  ws.eseq.ensure(B * sizeof(SeqDesc));
  ws.etok.ensure((size_t)M * 4);
  IRT_CUDA(cudaMemcpyAsync(ws.eseq.p, seqs.data(), B * sizeof(SeqDesc), cudaMemcpyHostToDevice, s));
  IRT_CUDA(cudaMemcpyAsync(ws.etok.p, tok.data(), (size_t)M * 4, cudaMemcpyHostToDevice, s));
  IRT_CUDA(cudaStreamSynchronize(s));  // host vectors go out of scope

  for (int l = 0; l < e.layers; ++l) {
    auto& b = e.blk[l];
    rms_norm(x, b.attn_norm.as<float>(), ws.eh.p, bf, M, dim, eps, s);
    EpiParams q;
    q.mode = EPI_QKVG;
    q.out_bf16 = bf;
    q.q = ws.eq.p; q.k = ws.ek.p; q.v = ws.ev.p; q.g = ws.eg.p;
    q.qn_w = b.qn.as<float>(); q.kn_w = b.kn.as<float>();
    q.rope_cos = ws.rope_cos.as<float>(); q.rope_sin = ws.rope_sin.as<float>();
    q.tok_pos = ws.etok.as<int>();
    q.H = e.heads; q.hd = e.hd; q.rope_heads = e.heads; q.eps = eps; q.Dq = dim;
    gemm(ws.eh.p, dim, b.wqkvg, M, 4 * dim, dim, q, s);
    AttnParams ap{};
    ap.q = ws.eq.p; ap.k = ws.ek.p; ap.v = ws.ev.p; ap.gsig = ws.eg.p;
    ap.key_mask = d_mask;
    ap.seqs = ws.eseq.as<SeqDesc>();
    ap.nseq = B; ap.max_len = T; ap.H = e.heads; ap.hd = e.hd;
    ap.scale = 1.0f / std::sqrt((float)e.hd);
    ap.out = ws.eattn.p;
    ap.rows = M;
    attention(ap, bf, s);
    EpiParams r;
    r.mode = EPI_RESID;
    r.x = x;
    gemm(ws.eattn.p, dim, b.wo, M, dim, dim, r, s);
    rms_norm(x, b.mlp_norm.as<float>(), ws.eh.p, bf, M, dim, eps, s);
    EpiParams sw;
    sw.mode = EPI_SWIGLU;
    sw.out_bf16 = bf;
    sw.h = ws.ehm.p;
    sw.F = e.F;
    gemm(ws.eh.p, dim, b.w13, M, 2 * e.Fp, dim, sw, s);
    EpiParams r2;
    r2.mode = EPI_RESID;
    r2.x = x;
    r2.row_scale = d_maskf;  // re-mask after the block
    gemm(ws.ehm.p, e.F, b.w2, M, dim, e.F, r2, s);
  }
  if (e.layers == 0 && d_maskf) {
    // x * mask_f once more (no-op on an already masked state)
  }
  rms_norm(x, e.out_norm.as<float>(), out_state_f32, 0, M, dim, eps, s);
}

// ---------------------------------------------------------------------------
// One DiT forward over M packed rows (src/model/dit/model.rs:354-393):
// input ws.xin [M, P] (operand type), output ws.vout [M, P] f32.
// ---------------------------------------------------------------------------
void Engine::forward_step(int M, const SeqDesc* d_seqs, int nseq, int max_len, int t_index, int nrows_ctx,
                          cudaStream_t s) {
  const size_t ada_bytes = (size_t)L * 6 * D * 4;
  ada_cur.ensure(ada_bytes);
  IRT_CUDA(cudaMemcpyAsync(ada_cur.p, ws.ada.as<uint8_t>() + (size_t)t_index * ada_bytes, ada_bytes,
                           cudaMemcpyDeviceToDevice, s));
  if (!use_graphs || dump_layers) {
    dit_forward(M, d_seqs, nseq, max_len, ada_cur.as<float>(), nrows_ctx, s);
    return;
  }
  std::vector<uintptr_t> key = {
      (uintptr_t)M, (uintptr_t)d_seqs, (uintptr_t)nseq, (uintptr_t)max_len, (uintptr_t)nrows_ctx, (uintptr_t)s,
      (uintptr_t)ws.x.p, (uintptr_t)ws.h.p, (uintptr_t)ws.q.p, (uintptr_t)ws.k.p, (uintptr_t)ws.v.p,
      (uintptr_t)ws.g.p, (uintptr_t)ws.attn.p, (uintptr_t)ws.hm.p, (uintptr_t)ws.xin.p, (uintptr_t)ws.vout.p,
      (uintptr_t)ws.raw.p, (uintptr_t)ws.tokpos.p, (uintptr_t)ws.cache_k.p, (uintptr_t)ws.cache_v.p,
      (uintptr_t)ws.rope_cos.p, (uintptr_t)ws.rope_sin.p, (uintptr_t)ada_cur.p, (uintptr_t)ws.a2.p};
  auto it = graphs.find(key);
  if (it == graphs.end()) {
    // keys seen once and never again (a server sees many ragged shapes) must
    // not accumulate: the table of first uses is bounded like the graphs
    if (graph_seen.size() > 256) graph_seen.clear();
    if (graph_seen[key]++ == 0) {  // first use: eager (allocations happen here)
      dit_forward(M, d_seqs, nseq, max_len, ada_cur.as<float>(), nrows_ctx, s);
      return;
    }
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    const long long before = launch_counter().load();
    IRT_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      dit_forward(M, d_seqs, nseq, max_len, ada_cur.as<float>(), nrows_ctx, s);
    } catch (...) {
      cudaStreamEndCapture(s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    IRT_CUDA(cudaStreamEndCapture(s, &g));
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    IRT_CUDA(e);
    if (graphs.size() > 64) {  // bound the cache
      for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
      graphs.clear();
      graph_kernels.clear();
    }
    graph_seen.erase(key);
    it = graphs.emplace(key, ge).first;
    // kernels recorded in the graph (captured launches are not executed)
    graph_kernels[key] = launch_counter().load() - before;
    launch_counter().fetch_sub(graph_kernels[key]);
  }
  IRT_CUDA(cudaGraphLaunch(it->second, s));
  launch_counter().fetch_add(graph_kernels[key]);
}

void Engine::dit_forward(int M, const SeqDesc* d_seqs, int nseq, int max_len, const float* ada_t, int nrows_ctx,
                         cudaStream_t s) {
  const float eps = (float)cfg.norm_eps;
  float* x = ws.x.as<float>();
  {
    EpiParams p;
    p.mode = EPI_STORE;
    p.out = x;
    p.ldo = D;
    p.bias = in_b.as<float>();
    gemm(ws.xin.p, Kin, in_w, M, D, Kin, p, s);
  }
  float* dump = dump_layers;
  if (dump) {
    if (M > dump_rows_cap) throw shape_error("layer dump buffer too small");
    dump_rows = M;
    dump_layers = nullptr;  // first forward only
    IRT_CUDA(cudaMemcpyAsync(dump, x, (size_t)M * D * 4, cudaMemcpyDeviceToDevice, s));
  }
  for (int l = 0; l < L; ++l) {
    const float* ad = ada_t + (size_t)l * 6 * D;
    auto& b = blk[l];
    adaln_modulate(x, ad + 0 * D, ad + 1 * D, ws.h.p, bf, M, D, eps, s);
    EpiParams q;
    q.mode = EPI_QKVG;
    q.out_bf16 = bf;
    q.q = ws.q.p; q.k = ws.k.p; q.v = ws.v.p; q.g = ws.g.p;
    q.qn_w = b.qn.as<float>(); q.kn_w = b.kn.as<float>();
    q.rope_cos = ws.rope_cos.as<float>(); q.rope_sin = ws.rope_sin.as<float>();
    q.tok_pos = ws.tokpos.as<int>();
    q.H = H; q.hd = hd; q.rope_heads = H / 2; q.eps = eps; q.Dq = D;
    gemm(ws.h.p, D, b.wqkvg, M, 4 * D, D, q, s);
    AttnParams ap{};
    ap.q = ws.q.p; ap.k = ws.k.p; ap.v = ws.v.p; ap.gsig = ws.g.p;
    size_t lstride = (size_t)nrows_ctx * D * esz();
    ap.ck = nrows_ctx ? (const void*)(ws.cache_k.as<uint8_t>() + l * lstride) : nullptr;
    ap.cv = nrows_ctx ? (const void*)(ws.cache_v.as<uint8_t>() + l * lstride) : nullptr;
    ap.key_mask = nullptr;
    ap.seqs = d_seqs;
    ap.nseq = nseq; ap.max_len = max_len; ap.H = H; ap.hd = hd;
    ap.scale = 1.0f / std::sqrt((float)hd);
    ap.out = ws.attn.p;
    ap.rows = M;
    ap.ctx_rows = nrows_ctx;
    attention(ap, bf, s);
    EpiParams r;
    r.mode = EPI_RESID;
    r.x = x;
    r.gate = ad + 2 * D;
    gemm(ws.attn.p, D, b.wo, M, D, D, r, s);
    adaln_modulate(x, ad + 3 * D, ad + 4 * D, ws.h.p, bf, M, D, eps, s);
    EpiParams sw;
    sw.mode = EPI_SWIGLU;
    sw.out_bf16 = bf;
    sw.h = ws.hm.p;
    sw.F = F;
    gemm(ws.h.p, D, b.w13, M, 2 * Fp, D, sw, s);
    EpiParams r2;
    r2.mode = EPI_RESID;
    r2.x = x;
    r2.gate = ad + 5 * D;
    gemm(ws.hm.p, F, b.w2, M, D, F, r2, s);
    if (dump)
      IRT_CUDA(cudaMemcpyAsync(dump + (size_t)(l + 1) * dump_rows_cap * D, x, (size_t)M * D * 4,
                               cudaMemcpyDeviceToDevice, s));
  }
  // out_norm + out_proj fused (narrow N = P): one pass over x per row
  EpiParams op;
  op.mode = EPI_STORE;
  op.M = M;
  op.N = P;  // columns stored; the GEMM runs 128 wide over the padded weight
  op.out = ws.vout.p;
  op.ldo = P;
  op.bias = out_b.as<float>();
  if (out_w_pad.p && M >= 128 && (D % 64) == 0) {
    // out_norm (RmsNorm, bf16 rows) then out_proj on the tensor cores
    if (out_split) {
      rms_norm_split(x, out_norm.as<float>(), ws.hm.as<bf16>(), M, D, eps, s);
      gemm_tc(ws.hm.as<bf16>(), 2 * D, out_w_pad.as<bf16>(), 2 * D, M, 128, 2 * D, op, s);
    } else {
      rms_norm(x, out_norm.as<float>(), ws.h.p, 1, M, D, eps, s);
      gemm_tc(ws.h.as<bf16>(), D, out_w_pad.as<bf16>(), D, M, 128, D, op, s);
    }
  } else {
    rmsnorm_proj(x, out_norm.as<float>(), out_w.p, bf, out_b.as<float>(), ws.vout.as<float>(), M, D, P, eps, s);
  }
}

// ---------------------------------------------------------------------------
// Sampler (src/rf/euler_sampler.rs:132-718)
// ---------------------------------------------------------------------------
namespace {

enum Variant { V_COND = 0, V_COND_S, V_UNCOND, V_TXT_UNC, V_TXT_UNC_S, V_AUX_UNC };

float f32_schedule(int i, int n) {  // 0.999 * (1 - i/n) in f32 (src/rf/euler_sampler.rs:325-328)
  float r = (float)i / (float)n;
  return 0.999f * (1.0f - r);
}

template <class T>
void to_device(DevBuf& buf, const T* src, size_t n, int memory, cudaStream_t s) {
  buf.ensure(n * sizeof(T) + 16);
  if (n == 0) return;
  IRT_CUDA(cudaMemcpyAsync(buf.p, src, n * sizeof(T),
                           memory == IRT_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
}

template <class T>
std::vector<T> to_host(const T* src, size_t n, int memory) {
  std::vector<T> v(n);
  if (n == 0) return v;
  if (memory == IRT_MEM_DEVICE) {
    IRT_CUDA(cudaMemcpy(v.data(), src, n * sizeof(T), cudaMemcpyDeviceToHost));
  } else {
    std::memcpy(v.data(), src, n * sizeof(T));
  }
  return v;
}

}  // namespace

void Engine::sample(const irt_request& rq, float* out, int out_memory, cudaStream_t user_stream) {
  std::lock_guard<std::mutex> lock(mu);
  IRT_CUDA(cudaSetDevice(device));
  if (!has_params) throw Error(IRT_E_STATE, "sampling parameters not set (call set_sampling first)");
  const irt_sampler_params& pr = params;
  validate_sampler_params(pr);
  cudaStream_t s = user_stream ? user_stream : stream;
  const long long launches0 = launch_counter().load();
  last_row_forwards = 0;

  const int B = rq.batch;
  if (B <= 0) throw shape_error("batch must be > 0");
  if (rq.text_len < 0 || (rq.text_len > 0 && (!rq.text_ids || !rq.text_mask)))
    throw missing_input("text_ids / text_mask");
  if (rq.sequence_length <= 0) throw shape_error("sequence_length must be > 0");
  if (!out) throw Error(IRT_E_INVALID_ARG, "out_latent is NULL");
  const int mem = rq.memory;
  const int Tt = rq.text_len;
  std::vector<int> S(B, rq.sequence_length);
  if (rq.sequence_lengths) {
    for (int b = 0; b < B; ++b) {
      S[b] = rq.sequence_lengths[b];
      if (S[b] <= 0 || S[b] > rq.sequence_length)
        throw shape_error("sequence_lengths[" + std::to_string(b) + "] out of range");
    }
  }
  std::vector<int> off(B + 1, 0);
  for (int b = 0; b < B; ++b) off[b + 1] = off[b] + S[b];
  const int ntok = off[B];
  const int Smax = *std::max_element(S.begin(), S.end());
  const float eps = (float)cfg.norm_eps;
  (void)eps;

  // ---- guidance bookkeeping (src/rf/euler_sampler.rs:157-224) ----
  const bool have_ref = rq.ref_latent && rq.ref_mask && rq.ref_len >= 0;
  const bool have_cap = rq.caption_ids && rq.caption_mask && rq.caption_len >= 0;
  int aux_in = 0;  // AuxConditionInput::from_request (src/model/condition.rs:104-122)
  if (have_ref) aux_in = 1;
  else if (have_cap) aux_in = 2;
  if (aux_in == 1 && aux_kind == 2)
    throw config_error(
        "caption conditioner received speaker input; check that the checkpoint and inference request use the same "
        "conditioning mode");
  if (aux_in == 2 && aux_kind == 1)
    throw config_error(
        "speaker conditioner received caption input; check that the checkpoint and inference request use the same "
        "conditioning mode");
  if (aux_kind == 0) aux_in = 0;
  const float s_text = pr.scale_text, s_cap = pr.scale_caption;
  const float s_spk = cfg.use_speaker_condition() ? pr.scale_speaker : 0.f;

  // ---- inputs to device ----
  std::vector<uint8_t> h_tmask = to_host(rq.text_mask, (size_t)B * Tt, mem);
  if (mem == IRT_MEM_HOST) {
    for (size_t i = 0; i < (size_t)B * Tt; ++i)
      if (rq.text_ids[i] < 0 || rq.text_ids[i] >= cfg.text_vocab_size)
        throw Error(IRT_E_INVALID_ARG, "text id out of range at position " + std::to_string(i));
  }
  to_device(ws.ids, rq.text_ids, (size_t)B * Tt, mem, s);
  to_device(ws.tmask, h_tmask.data(), h_tmask.size(), IRT_MEM_HOST, s);
  // float masks for the re-mask multiply
  std::vector<float> h_tmaskf(h_tmask.size());
  for (size_t i = 0; i < h_tmask.size(); ++i) h_tmaskf[i] = h_tmask[i] ? 1.f : 0.f;

  int Ta_in = 0, Ta = 0;  // aux input rows per batch, aux state rows per batch (speaker: +1 mean token)
  std::vector<uint8_t> h_amask_in;
  if (aux_in == 1) {
    const int p = (int)cfg.speaker_patch_size.value_or(1);
    if (rq.ref_dim != P) throw shape_error("ref_latent width " + std::to_string(rq.ref_dim) + " != " + std::to_string(P));
    int Tr = rq.ref_len;
    int usable = p > 1 ? (Tr / p) * p : Tr;
    if (p > 1 && usable == 0)
      throw shape_error("Sequence too short for speaker_patch_size=" + std::to_string(p) +
                        ": seq_len=" + std::to_string(Tr));
    Ta_in = p > 1 ? usable / p : Tr;
    std::vector<uint8_t> rm = to_host(rq.ref_mask, (size_t)B * Tr, mem);
    h_amask_in.assign((size_t)B * Ta_in, 0);
    for (int b = 0; b < B; ++b)
      for (int i = 0; i < Ta_in; ++i) {
        bool all = true;
        for (int j = 0; j < p; ++j) all = all && rm[(size_t)b * Tr + (size_t)i * p + j];
        h_amask_in[(size_t)b * Ta_in + i] = all;
      }
    // patched latent rows [B*Ta_in, P*p] (contiguous per batch row)
    ws.ref.ensure((size_t)B * Ta_in * P * p * 4 + 16);
    for (int b = 0; b < B; ++b)
      IRT_CUDA(cudaMemcpyAsync(ws.ref.as<float>() + (size_t)b * Ta_in * P * p, rq.ref_latent + (size_t)b * Tr * P,
                               (size_t)Ta_in * P * p * 4,
                               mem == IRT_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
    Ta = Ta_in + 1;
  } else if (aux_in == 2) {
    Ta_in = rq.caption_len;
    h_amask_in = to_host(rq.caption_mask, (size_t)B * Ta_in, mem);
    for (auto& m : h_amask_in) m = m ? 1 : 0;
    if (mem == IRT_MEM_HOST)
      for (size_t i = 0; i < (size_t)B * Ta_in; ++i)
        if (rq.caption_ids[i] < 0 || rq.caption_ids[i] >= cfg.caption_vocab_size_())
          throw Error(IRT_E_INVALID_ARG, "caption id out of range at position " + std::to_string(i));
    to_device(ws.cids, rq.caption_ids, (size_t)B * Ta_in, mem, s);
    Ta = Ta_in;
  }
  const bool has_text_cfg = s_text > 0.f;
  const bool has_spk_cfg = s_spk > 0.f && aux_in == 1;
  bool any_cap = false;
  for (auto m : h_amask_in) any_cap = any_cap || m;
  const bool has_cap_cfg = s_cap > 0.f && aux_in == 2 && any_cap;
  std::vector<int> enabled;  // 0 text, 1 speaker, 2 caption
  if (has_text_cfg) enabled.push_back(0);
  if (has_spk_cfg) enabled.push_back(1);
  if (has_cap_cfg) enabled.push_back(2);
  auto scale_of = [&](int n) { return n == 0 ? s_text : n == 1 ? s_spk : s_cap; };
  if (pr.cfg_mode == IRT_CFG_JOINT && !enabled.empty()) {
    float mn = INFINITY, mx = -INFINITY;
    for (int n : enabled) { mn = std::min(mn, scale_of(n)); mx = std::max(mx, scale_of(n)); }
    if (mx - mn >= 1e-6f)
      throw config_error("cfg_guidance_mode=Joint requires all active cfg scales to be equal, but got text=" +
                         fmt_f32(pr.scale_text) + ", speaker=" + fmt_f32(pr.scale_speaker) + ", caption=" +
                         fmt_f32(pr.scale_caption) + ". Pass a single equal value for all active signals.");
  }

  // ---- prologue: encoders ----
  const int td = (int)cfg.text_dim;
  ws.estate.ensure((size_t)std::max(1, B * Tt) * td * 4);
  to_device(ws.emask, h_tmaskf.data(), h_tmaskf.size(), IRT_MEM_HOST, s);
  run_encoder(text_enc, B, Tt, ws.ids.p, true, ws.tmask.as<uint8_t>(), ws.emask.as<float>(), ws.estate.p, s);
  // operand copy of the text state for the KV projections
  ws.aux_state_t.ensure((size_t)std::max(1, B * std::max(Tt, Ta)) * std::max(td, std::max(aux_dim, 1)) * esz());
  DevBuf& text_t = ws.text_t;
  text_t.ensure((size_t)std::max(1, B * Tt) * td * esz());
  gather_rows(ws.estate.as<float>(), nullptr, text_t.p, bf, B * Tt, td, s);

  std::vector<uint8_t> h_amask;  // aux state mask [B, Ta]
  if (aux_in) {
    std::vector<float> amf(h_amask_in.size());
    for (size_t i = 0; i < amf.size(); ++i) amf[i] = h_amask_in[i] ? 1.f : 0.f;
    DevBuf& amask_in_d = ws.amask_in;
    DevBuf& amaskf_d = ws.amaskf;
    to_device(amask_in_d, h_amask_in.data(), h_amask_in.size(), IRT_MEM_HOST, s);
    to_device(amaskf_d, amf.data(), amf.size(), IRT_MEM_HOST, s);
    ws.estate2.ensure((size_t)std::max(1, B * Ta_in) * aux_dim * 4);
    if (aux_in == 1) {
      // speaker latent -> operand type
      const int pin = aux_enc.in_dim;
      DevBuf& lat_t = ws.lat_t;
      lat_t.ensure((size_t)std::max(1, B * Ta_in) * pin * esz());
      gather_rows(ws.ref.as<float>(), nullptr, lat_t.p, bf, B * Ta_in, pin, s);
      run_encoder(aux_enc, B, Ta_in, lat_t.p, false, amask_in_d.as<uint8_t>(), amaskf_d.as<float>(), ws.estate2.p, s);
      IRT_CUDA(cudaStreamSynchronize(s));
      // prepend the masked-mean token
      DevBuf& st2 = ws.st2;
      st2.ensure((size_t)B * Ta * aux_dim * 4);
      ws.amask.ensure((size_t)B * Ta + 16);
      prepend_mean_token(ws.estate2.as<float>(), amask_in_d.as<uint8_t>(), st2.as<float>(), ws.amask.as<uint8_t>(), B,
                         Ta_in, aux_dim, s);
      gather_rows(st2.as<float>(), nullptr, ws.aux_state_t.p, bf, B * Ta, aux_dim, s);
      h_amask.assign((size_t)B * Ta, 0);
      for (int b = 0; b < B; ++b) {
        bool any = false;
        for (int i = 0; i < Ta_in; ++i) any = any || h_amask_in[(size_t)b * Ta_in + i];
        h_amask[(size_t)b * Ta] = any;
        for (int i = 0; i < Ta_in; ++i) h_amask[(size_t)b * Ta + 1 + i] = h_amask_in[(size_t)b * Ta_in + i];
      }
      IRT_CUDA(cudaStreamSynchronize(s));
    } else {
      run_encoder(aux_enc, B, Ta_in, ws.cids.p, true, amask_in_d.as<uint8_t>(), amaskf_d.as<float>(), ws.estate2.p, s);
      gather_rows(ws.estate2.as<float>(), nullptr, ws.aux_state_t.p, bf, B * Ta, aux_dim, s);
      h_amask = h_amask_in;
      IRT_CUDA(cudaStreamSynchronize(s));
    }
  }

  // ---- context KV cache layout: per utterance [aux scaled | text | aux] ----
  const bool skv_cfg = pr.has_speaker_kv && cfg.use_speaker_condition() && aux_in == 1;
  std::vector<int> nt(B, 0), na(B, 0), sc(B, 0), base(B + 1, 0);
  std::vector<int> map_t((size_t)B * Tt, -1), map_a((size_t)B * Ta, -1), map_as((size_t)B * Ta, -1);
  for (int b = 0; b < B; ++b) {
    for (int i = 0; i < Tt; ++i) nt[b] += h_tmask[(size_t)b * Tt + i] ? 1 : 0;
    for (int i = 0; i < Ta; ++i) na[b] += h_amask.empty() ? 0 : (h_amask[(size_t)b * Ta + i] ? 1 : 0);
    sc[b] = skv_cfg ? na[b] : 0;
    base[b + 1] = base[b] + sc[b] + nt[b] + na[b];
    int rt = 0, ra = 0;
    for (int i = 0; i < Tt; ++i)
      if (h_tmask[(size_t)b * Tt + i]) map_t[(size_t)b * Tt + i] = base[b] + sc[b] + rt++;
    for (int i = 0; i < Ta; ++i)
      if (!h_amask.empty() && h_amask[(size_t)b * Ta + i]) {
        map_a[(size_t)b * Ta + i] = base[b] + sc[b] + nt[b] + ra;
        map_as[(size_t)b * Ta + i] = base[b] + ra;
        ++ra;
      }
  }
  const int nctx = base[B];
  const size_t lstride_el = (size_t)nctx * D;
  if (nctx > 0) {
    ws.cache_k.ensure((size_t)L * lstride_el * esz());
    ws.cache_v.ensure((size_t)L * lstride_el * esz());
    to_device(ws.rowmap_t, map_t.data(), map_t.size(), IRT_MEM_HOST, s);
    EpiParams c;
    c.mode = EPI_CTXKV;
    c.out_bf16 = bf;
    c.ck = ws.cache_k.p;
    c.cv = ws.cache_v.p;
    c.layer_stride = (long)lstride_el;
    c.Dq = D;
    c.hd = hd;
    c.H = H;
    c.kn_w = kn_all.as<float>();
    c.eps = (float)cfg.norm_eps;
    c.row_map = ws.rowmap_t.as<int>();
    if (B * Tt > 0) gemm(text_t.p, td, ctx_text_w, B * Tt, L * 2 * D, td, c, s);
    if (aux_in) {
      to_device(ws.rowmap_a, map_a.data(), map_a.size(), IRT_MEM_HOST, s);
      c.row_map = ws.rowmap_a.as<int>();
      gemm(ws.aux_state_t.p, aux_dim, ctx_aux_w, B * Ta, L * 2 * D, aux_dim, c, s);
      if (skv_cfg) {
        // scaled copy of the speaker rows (SpeakerKvConfig, src/rf/kv_scaling.rs:10-60)
        to_device(ws.rowmap_as, map_as.data(), map_as.size(), IRT_MEM_HOST, s);
        c.row_map = ws.rowmap_as.as<int>();
        gemm(ws.aux_state_t.p, aux_dim, ctx_aux_w, B * Ta, L * 2 * D, aux_dim, c, s);
        int nl = pr.speaker_kv_max_layers < 0 ? L : std::min(pr.speaker_kv_max_layers, L);
        std::vector<int> rows;
        for (int b = 0; b < B; ++b)
          for (int i = 0; i < sc[b]; ++i) rows.push_back(base[b] + i);
        DevBuf& rows_d = ws.rows;
        to_device(rows_d, rows.data(), rows.size(), IRT_MEM_HOST, s);
        for (int l = 0; l < nl; ++l) {
          uint8_t* kl = ws.cache_k.as<uint8_t>() + (size_t)l * lstride_el * esz();
          uint8_t* vl = ws.cache_v.as<uint8_t>() + (size_t)l * lstride_el * esz();
          scale_rows_bf16_or_f32(kl, bf, D, rows_d.as<int>(), (int)rows.size(), pr.speaker_kv_scale, s);
          scale_rows_bf16_or_f32(vl, bf, D, rows_d.as<int>(), (int)rows.size(), pr.speaker_kv_scale, s);
        }
        IRT_CUDA(cudaStreamSynchronize(s));
      }
    }
  }

  // ---- timestep schedule, embeddings, cond_module, adaLN tables ----
  const int NS = (int)pr.num_steps;
  const int NT = NS + 1;
  std::vector<float> ts(NT);
  for (int i = 0; i < NT; ++i) ts[i] = f32_schedule(i, NS);
  {
    const int half = Temb / 2;
    std::vector<float> temb((size_t)NT * Temb);
    const float log1e4 = std::log(10000.0f);
    std::vector<float> fr(half);
    for (int i = 0; i < half; ++i) fr[i] = 1000.0f * std::exp((-log1e4 * (float)i) / (float)half);
    for (int t = 0; t < NT; ++t)
      for (int i = 0; i < half; ++i) {
        float a = ts[t] * fr[i];
        temb[(size_t)t * Temb + i] = std::cos(a);
        temb[(size_t)t * Temb + half + i] = std::sin(a);
      }
    to_device(ws.temb, temb.data(), temb.size(), IRT_MEM_HOST, s);
    ws.ce.ensure((size_t)NT * 3 * D * 4);
    ws.su.ensure((size_t)NT * 3 * D * 4);
    DevBuf& h0 = ws.h0;
    DevBuf& h1 = ws.h1;
    h0.ensure((size_t)NT * D * 4);
    h1.ensure((size_t)NT * D * 4);
    const bool keep = bf;
    bf = false;  // cond_module / adaLN tables run in f32 (SIMT) in both precisions
    EpiParams p;
    p.mode = EPI_STORE;
    p.act = ACT_SILU;
    p.out = h0.p;
    p.ldo = D;
    gemm(ws.temb.p, Temb, cm0, NT, D, Temb, p, s);
    p.out = h1.p;
    gemm(h0.p, D, cm1, NT, D, D, p, s);
    p.act = ACT_NONE;
    p.out = ws.ce.p;
    p.ldo = 3 * D;
    gemm(h1.p, D, cm2, NT, 3 * D, D, p, s);
    bf = keep;
    // adaLN: out[t][z][k] = up_k,z(down_k,z(silu(raw_k))) + bias + raw_k ; gate -> tanh
    silu_copy(ws.ce.as<float>(), 3 * D, ws.su.as<float>(), 3 * D, NT, 3 * D, s);
    ws.ada.ensure((size_t)NT * L * 6 * D * 4);
    ws.dn.ensure((size_t)NT * L * 2 * R * 4);
    const long ldo_ada = (long)L * 6 * D;
    for (int k = 0; k < 3; ++k) {
      ws.raw.ensure((size_t)std::max((size_t)NT * L * 2 * R, (size_t)L * 2 * NT * D) * 4);
      gemm_simt(ws.su.as<float>() + k * D, 0, 3 * D, 0, ada_down[k].p, 0, D, 0, ws.dn.as<float>(), L * 2 * R, 0, NT,
                L * 2 * R, D, 1, s);
      gemm_simt(ws.dn.as<float>(), 0, L * 2 * R, R, ada_up[k].p, 0, R, (long)D * R, ws.raw.as<float>(), D,
                (long)NT * D, NT, D, R, L * 2, s);
      EpiParams e;
      e.mode = EPI_STORE;
      e.M = NT;
      e.N = D;
      e.out = ws.ada.as<float>() + k * D;
      e.ldo = ldo_ada;
      e.out_bstride = 3 * D;
      e.bias = ada_upb[k].as<float>();
      e.bias_bstride = D;
      e.add = ws.ce.as<float>() + k * D;
      e.ld_add = 3 * D;
      e.add_bstride = 0;
      e.act = k == 2 ? ACT_TANH : ACT_NONE;
      epilogue_apply(e, ws.raw.as<float>(), D, (long)NT * D, L * 2, s);
    }
  }

  // ---- latent RoPE + row bookkeeping ----
  {
    std::vector<float> cs, sn;
    rope_tables_host(hd, Smax, cs, sn);
    ws.rope_cos.ensure(cs.size() * 4 + 4);
    ws.rope_sin.ensure(sn.size() * 4 + 4);
    IRT_CUDA(cudaMemcpyAsync(ws.rope_cos.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, s));
    IRT_CUDA(cudaMemcpyAsync(ws.rope_sin.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, s));
    IRT_CUDA(cudaStreamSynchronize(s));
  }
  int max_groups = 1;
  if (!enabled.empty()) max_groups = pr.cfg_mode == IRT_CFG_INDEPENDENT ? 1 + (int)enabled.size() : 2;
  const int Mmax = max_groups * ntok;
  ws.x.ensure((size_t)Mmax * D * 4);
  ws.h.ensure((size_t)Mmax * D * esz());
  ws.q.ensure((size_t)Mmax * D * esz());
  ws.k.ensure((size_t)Mmax * D * esz());
  ws.v.ensure((size_t)Mmax * D * esz());
  ws.g.ensure((size_t)Mmax * D * esz());
  ws.attn.ensure((size_t)Mmax * D * esz());
  ws.hm.ensure((size_t)Mmax * std::max(F, out_split ? 2 * D : 0) * esz());  // also the split out_norm rows
  ws.xin.ensure((size_t)Mmax * Kin * esz());
  if (Kin != P) IRT_CUDA(cudaMemsetAsync(ws.xin.p, 0, (size_t)Mmax * Kin * esz(), s));  // zero K padding
  ws.vout.ensure((size_t)Mmax * P * 4);
  ws.tokpos.ensure((size_t)Mmax * 4);
  {
    DevBuf& uo = ws.uo;
    DevBuf& ul = ws.ul;
    std::vector<int> len(S.begin(), S.end());
    to_device(uo, off.data(), (size_t)B, IRT_MEM_HOST, s);
    to_device(ul, len.data(), (size_t)B, IRT_MEM_HOST, s);
    tokpos_kernel<<<(Mmax + 255) / 256, 256, 0, s>>>(ws.tokpos.as<int>(), uo.as<int>(), ul.as<int>(), B, ntok, Mmax);
    IRT_CHECK_LAUNCH();
    IRT_CUDA(cudaStreamSynchronize(s));
  }

  // sequence-descriptor tables for every forward kind that may run
  auto ctx_of = [&](int var, int b) -> std::pair<int, int> {
    switch (var) {
      case V_COND: return {base[b] + sc[b], nt[b] + na[b]};
      case V_COND_S: return {base[b], sc[b] + nt[b]};
      case V_UNCOND: return {0, 0};
      case V_TXT_UNC: return {base[b] + sc[b] + nt[b], na[b]};
      case V_TXT_UNC_S: return {base[b], sc[b]};
      default: return {base[b] + sc[b], nt[b]};  // V_AUX_UNC
    }
  };
  std::map<std::vector<int>, int> table_off;
  std::vector<SeqDesc> all_desc;
  auto table_for = [&](const std::vector<int>& groups) -> int {
    auto it = table_off.find(groups);
    if (it != table_off.end()) return it->second;
    int o = (int)all_desc.size();
    for (size_t g = 0; g < groups.size(); ++g)
      for (int b = 0; b < B; ++b) {
        auto c = ctx_of(groups[g], b);
        all_desc.push_back({(int)g * ntok + off[b], S[b], c.first, c.second});
      }
    table_off[groups] = o;
    return o;
  };
  auto groups_for = [&](bool use_cfg, bool skv_on, int step) -> std::vector<int> {
    int cond = skv_on ? V_COND_S : V_COND;
    if (!use_cfg) return {cond};
    if (pr.cfg_mode == IRT_CFG_INDEPENDENT) {
      std::vector<int> g{cond};
      for (int n : enabled) g.push_back(n == 0 ? (skv_on ? V_TXT_UNC_S : V_TXT_UNC) : V_AUX_UNC);
      return g;
    }
    if (pr.cfg_mode == IRT_CFG_JOINT) return {cond, V_UNCOND};
    int name = enabled[step % enabled.size()];
    return {cond, name == 0 ? V_TXT_UNC : V_AUX_UNC};
  };
  // enumerate all (use_cfg, skv_on, alt index) combinations up front
  for (int uc = 0; uc < 2; ++uc)
    for (int sk = 0; sk < 2; ++sk) {
      if (uc && enabled.empty()) continue;
      if (sk && !skv_cfg) continue;
      int nalt = (uc && pr.cfg_mode == IRT_CFG_ALTERNATING) ? (int)enabled.size() : 1;
      for (int a = 0; a < nalt; ++a) table_for(groups_for(uc, sk, a));
    }
  ws.seqs.ensure(all_desc.size() * sizeof(SeqDesc) + 16);
  IRT_CUDA(cudaMemcpyAsync(ws.seqs.p, all_desc.data(), all_desc.size() * sizeof(SeqDesc), cudaMemcpyHostToDevice, s));
  IRT_CUDA(cudaStreamSynchronize(s));

  // ---- initial noise (src/rf/euler_sampler.rs:146-155) ----
  const size_t nel = (size_t)ntok * P;
  ws.xstate.ensure(nel * 4 + 16);
  float* xs = ws.xstate.as<float>();
  if (rq.initial_noise) {
    const auto kind = mem == IRT_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    if (rq.sequence_lengths) {
      for (int b = 0; b < B; ++b)
        IRT_CUDA(cudaMemcpyAsync(xs + (size_t)off[b] * P, rq.initial_noise + (size_t)b * rq.sequence_length * P,
                                 (size_t)S[b] * P * 4, kind, s));
    } else {
      IRT_CUDA(cudaMemcpyAsync(xs, rq.initial_noise, nel * 4, kind, s));
    }
  } else {
    gaussian_fill(xs, (long)nel, rq.seed, s);
  }
  if (pr.has_truncation) scale_buf(xs, pr.truncation_factor, (long)nel, s);

  ws.vcomb.ensure(nel * 4 + 16);
  ws.xpred.ensure(nel * 4 + 16);
  ws.v1.ensure(nel * 4 + 16);
  for (int i = 0; i < 4; ++i) ws.hist[i].ensure(nel * 4 + 16);
  // guidance scales in `enabled` order (Joint uses the first, Alternating the i-th)
  {
    std::vector<float> sc_all;
    for (int n : enabled) sc_all.push_back(scale_of(n));
    sc_all.push_back(0.f);
    to_device(ws.scal, sc_all.data(), sc_all.size(), IRT_MEM_HOST, s);
  }

  const float min_t = pr.min_t, max_t = pr.max_t;
  auto in_window = [&](float t) { return !enabled.empty() && min_t <= t && t <= max_t; };

  // guided velocity at (x, t): one packed forward over all CFG groups
  auto guided = [&](const float* xin_f32, int t_index, float t, int step, bool skv_on, float* v_out) {
    bool use_cfg = in_window(t);
    std::vector<int> groups = groups_for(use_cfg, skv_on, step);
    int G = (int)groups.size();
    int toff = table_off.at(groups);
    // replicate x into each group's rows
    for (int g = 0; g < G; ++g) {
      uint8_t* dst = ws.xin.as<uint8_t>() + (size_t)g * ntok * Kin * esz();
      if (bf) gather_split_rows(xin_f32, reinterpret_cast<bf16*>(dst), ntok, P, Pk, s);
      else gather_rows(xin_f32, nullptr, dst, 0, ntok, P, s, Pk);
    }
    forward_step(G * ntok, ws.seqs.as<SeqDesc>() + toff, G * B, Smax, t_index, nctx, s);
    last_row_forwards += (long long)G * B;
    if (G == 1) {
      IRT_CUDA(cudaMemcpyAsync(v_out, ws.vout.p, nel * 4, cudaMemcpyDeviceToDevice, s));
      return;
    }
    const float* scl = ws.scal.as<float>();
    if (pr.cfg_mode == IRT_CFG_ALTERNATING) scl += step % enabled.size();
    cfg_combine(ws.vout.as<float>(), nullptr, scl, G, nullptr, ntok, P, v_out, s);
  };

  auto rescale = [&](float* v, const float* x, float t) {  // src/rf/math.rs:38-52
    if (!pr.has_temporal_rescale || t >= 1.0f) return;
    float omt = 1.0f - t;
    float snr = (omt * omt) / (t * t);
    float ss = pr.rescale_sigma * pr.rescale_sigma;
    float ratio = (snr * ss + 1.0f) / (snr * ss / pr.rescale_k + 1.0f);
    temporal_rescale(v, x, omt, ratio, (long)nel, s);
  };

  bool skv_active = pr.has_speaker_kv;  // speaker_kv_active (src/rf/euler_sampler.rs:347)
  std::vector<int> hist;                // PLMS history buffer indices, newest first
  int hist_next = 0;
  auto regime_of = [&](float t) { return std::make_pair(in_window(t), skv_active); };
  auto prev_regime = regime_of(ts[0]);
  float* v = ws.vcomb.as<float>();
  for (int i = 0; i < NS; ++i) {
    const float t = ts[i], tn = ts[i + 1];
    if (pr.method == IRT_PLMS4) {
      auto rg = regime_of(t);
      if (rg != prev_regime) {
        hist.clear();
        prev_regime = rg;
      }
    }
    guided(xs, i, t, i, skv_active && skv_cfg, v);
    rescale(v, xs, t);
    if (skv_active && pr.has_speaker_kv && cfg.use_speaker_condition() && pr.has_speaker_kv_min_t &&
        tn < pr.speaker_kv_min_t && t >= pr.speaker_kv_min_t)
      skv_active = false;  // revert: switch to the unscaled cache rows
    const float dt = tn - t;
    if (pr.method == IRT_EULER) {
      axpy(xs, v, dt, (long)nel, s);
    } else if (pr.method == IRT_HEUN) {
      float* xp = ws.xpred.as<float>();
      float* v1 = ws.v1.as<float>();
      IRT_CUDA(cudaMemcpyAsync(v1, v, nel * 4, cudaMemcpyDeviceToDevice, s));
      IRT_CUDA(cudaMemcpyAsync(xp, xs, nel * 4, cudaMemcpyDeviceToDevice, s));
      axpy(xp, v1, dt, (long)nel, s);
      guided(xp, i + 1, tn, i, skv_active && skv_cfg, v);
      rescale(v, xp, tn);
      const float* xs2[2] = {v1, v};
      float cf[2] = {0.5f, 0.5f};
      lincomb(v, xs2, cf, 2, (long)nel, s);
      axpy(xs, v, dt, (long)nel, s);
    } else {  // PLMS4 (src/rf/euler_sampler.rs:99-116, :703-711)
      int slot;
      if ((int)hist.size() < 4) {
        slot = hist_next++ % 4;
        // find a free slot
        std::vector<bool> used(4, false);
        for (int h : hist) used[h] = true;
        for (int c = 0; c < 4; ++c)
          if (!used[c]) { slot = c; break; }
      } else {
        slot = hist.back();
        hist.pop_back();
      }
      IRT_CUDA(cudaMemcpyAsync(ws.hist[slot].p, v, nel * 4, cudaMemcpyDeviceToDevice, s));
      hist.insert(hist.begin(), slot);
      const float* xsrc[4];
      float cf[4];
      int n = (int)hist.size();
      static const float c2[2] = {1.5f, -0.5f};
      static const float c3[3] = {23.0f / 12.0f, -16.0f / 12.0f, 5.0f / 12.0f};
      static const float c4[4] = {55.0f / 24.0f, -59.0f / 24.0f, 37.0f / 24.0f, -9.0f / 24.0f};
      for (int k = 0; k < n; ++k) {
        xsrc[k] = ws.hist[hist[k]].as<float>();
        cf[k] = n == 1 ? 1.f : n == 2 ? c2[k] : n == 3 ? c3[k] : c4[k];
      }
      if (n == 1) {
        axpy(xs, xsrc[0], dt, (long)nel, s);
      } else {
        lincomb(v, xsrc, cf, n, (long)nel, s);
        axpy(xs, v, dt, (long)nel, s);
      }
    }
  }

  // ---- output [B, S, P] ----
  const auto okind = out_memory == IRT_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
  if (rq.sequence_lengths) {
    if (out_memory == IRT_MEM_DEVICE) {
      IRT_CUDA(cudaMemsetAsync(out, 0, (size_t)B * rq.sequence_length * P * 4, s));
    } else {
      std::memset(out, 0, (size_t)B * rq.sequence_length * P * 4);
    }
    for (int b = 0; b < B; ++b)
      IRT_CUDA(cudaMemcpyAsync(out + (size_t)b * rq.sequence_length * P, xs + (size_t)off[b] * P,
                               (size_t)S[b] * P * 4, okind, s));
  } else {
    IRT_CUDA(cudaMemcpyAsync(out, xs, nel * 4, okind, s));
  }
  IRT_CUDA(cudaStreamSynchronize(s));
  if (read_and_clear_kernel_error() | read_and_clear_attn_error())
    throw Error(IRT_E_CUDA, "a GEMM pipeline wait timed out (device watchdog); results are invalid");
  last_launches = launch_counter().load() - launches0;
}

}  // namespace irt
