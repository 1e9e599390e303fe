// Engine: the loaded, pre-packed DiT + condition encoders on one device and
// the rectified-flow sampler that drives them (src/inference.rs:83-254,
// src/rf/euler_sampler.rs:132-718).
#pragma once

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.hpp"
#include "config.hpp"
#include "kernels.hpp"

namespace irt {

class SafeTensorsFile;

// TextBlock stack (src/model/text_encoder.rs:17-60) used by the text,
// caption and speaker encoders.
struct EncoderW {
  int dim = 0, heads = 0, hd = 0, layers = 0, F = 0, Fp = 0, vocab = 0, in_dim = 0;
  DevBuf emb;          // f32 [vocab, dim] (text / caption)
  DevBuf in_w, in_b;   // T [dim, in_dim], f32 [dim] (speaker in_proj)
  struct Layer {
    DevBuf attn_norm, wqkvg, qn, kn, wo, mlp_norm, w13, w2;
  };
  std::vector<Layer> blk;
  DevBuf out_norm;     // text_norm / speaker_norm / caption_norm
};

struct DitLayerW {
  DevBuf wqkvg, qn, kn, wo, w13, w2;
};

struct Engine {
  int device = 0;
  int prec = IRT_PREC_BF16;
  bool bf = true;  // GEMM operand storage is bf16
  cudaStream_t stream = nullptr;
  ModelConfig cfg;
  bool has_params = false;
  irt_sampler_params params{};
  std::mutex mu;

  // dimensions
  int D = 0, L = 0, H = 0, hd = 0, P = 0, F = 0, Fp = 0, R = 0, Temb = 0;
  // in_proj reduction width: P, or (bf16 mode) P zero-padded to a multiple of
  // 64 so the projection runs on the tcgen05 GEMM with its bias epilogue
  int Pk = 0;
  // in_proj GEMM reduction width: Pk in f32 mode; 2 Pk in bf16 mode, where the
  // f32 latent x_t enters as bf16 hi | lo halves over the weight stored twice
  // ([W | W] along K), so the projection is not limited by one bf16 rounding
  // of x_t (the sampler state)
  int Kin = 0;
  // bf16 mode: out_norm rows enter out_proj as bf16 hi | lo halves over
  // out_w_pad = [W | W] (K = 2 D), for the same reason on the velocity
  bool out_split = false;
  int aux_kind = 0;  // 0 none, 1 speaker, 2 caption
  int aux_dim = 0;

  // weights
  EncoderW text_enc, aux_enc;
  DevBuf cm0, cm1, cm2;               // cond_module, f32
  DevBuf in_w, in_b;                  // in_proj
  DevBuf ada_down[3], ada_up[3], ada_upb[3];  // per kind (shift, scale, gate), stacked over (layer, attn|mlp)
  std::vector<DitLayerW> blk;
  DevBuf ctx_text_w, ctx_aux_w;       // [L*2D, td] / [L*2D, ad]: per layer [Wk; Wv]
  DevBuf kn_all;                      // f32 [L, D]
  DevBuf out_norm, out_w, out_b;
  // bf16 mode: out_proj rows zero-padded to 128 so the projection of the
  // normalised rows runs on the tcgen05 GEMM (only the first P columns are
  // stored)
  DevBuf out_w_pad;
  // f32 mode: [W_hi | W_lo] ([N, 2 Kp], tf32 hi / lo halves) of every GEMM
  // weight that meets 128 or more rows, keyed by the f32 weight's address;
  // such GEMMs run on the tcgen05 tf32 path (gemm_tc_tf32x3) instead of the
  // SIMT kernel.  IRT_F32_SIMT=1 keeps every f32 GEMM on the SIMT kernel.
  bool tf32 = false;
  std::unordered_map<const void*, DevBuf> w_tf32;

  // workspaces (grow-only)
  struct WS {
    DevBuf x, h, q, k, v, g, attn, hm, xin, vout, raw, tokpos, seqs, vcomb, xpred, v1, hist[4], xstate, scal;
    DevBuf ex, eh, eq, ek, ev, eg, eattn, ehm, estate, estate2, emask, eseq, etok;  // encoders
    DevBuf cache_k, cache_v, rowmap_t, rowmap_a, rowmap_as, amask, aux_state_t;
    DevBuf ada, temb, ce, su, dn;
    DevBuf ids, tmask, ref, rmask, cids, cmask, noise, out;
    DevBuf rope_cos, rope_sin;
    DevBuf text_t, lat_t, st2, amask_in, amaskf, h0, h1, uo, ul, rows;
    DevBuf a2;  // f32 mode: [A_hi | A_lo] of the current GEMM operand
  } ws;

  long long last_row_forwards = 0, last_launches = 0;

  // CUDA graphs of the DiT forward, keyed by its shape and every buffer
  // address it bakes in.  A key's first use runs eagerly (so workspaces are
  // allocated outside capture); its second use captures and instantiates.
  bool use_graphs = true;
  // Per-layer capture for parity tests (test hooks only): when set, the next
  // DiT forward runs eagerly and copies the f32 residual stream after in_proj
  // and after every block into dump_layers[(0..L) * M * D] (device memory with
  // room for dump_rows_cap rows per slot), records the row count in dump_rows,
  // and then clears the pointer.
  float* dump_layers = nullptr;
  int dump_rows_cap = 0;
  int dump_rows = 0;
  std::map<std::vector<uintptr_t>, cudaGraphExec_t> graphs;
  std::map<std::vector<uintptr_t>, int> graph_seen;
  std::map<std::vector<uintptr_t>, long long> graph_kernels;
  DevBuf ada_cur;  // adaLN parameters of the current step, read by the graph
  void forward_step(int M, const SeqDesc* d_seqs, int nseq, int max_len, int t_index, int nrows_ctx,
                    cudaStream_t s);

  // adapter_dir: optional PEFT LoRA adapter merged into the weights at load
  Engine(int dev, const std::string& path, int precision, const std::string& adapter_dir = "");
  int lora_merged = 0;  // base weights updated by the adapter
  ~Engine();

  void sample(const irt_request& req, float* out, int out_memory, cudaStream_t user_stream);

  // helpers
  size_t esz() const { return bf ? 2 : 4; }
  void gemm(const void* A, long lda, const DevBuf& W, int M, int N, int K, EpiParams p, cudaStream_t s);
  void run_encoder(EncoderW& e, int B, int T, const void* input_rows_T, bool from_ids, const uint8_t* d_mask,
                   const float* d_maskf, void* out_state_f32, cudaStream_t s);
  void dit_forward(int M, const SeqDesc* d_seqs, int nseq, int max_len, const float* ada_t, int nrows_ctx,
                   cudaStream_t s);

 private:
  void load(const std::string& path, const std::string& adapter_dir);
  void prepare_tf32();
  void load_encoder(const SafeTensorsFile& st, EncoderW& e, const std::string& prefix, int dim, int heads,
                    int layers, double ratio, bool embedding, int vocab, int in_dim);
};

}  // namespace irt
