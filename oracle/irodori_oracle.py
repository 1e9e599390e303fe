"""CPU oracle for the Irodori-TTS rectified-flow sampling path.

TEST INFRASTRUCTURE ONLY.  This module is a plain PyTorch (CPU, float32 by
default, float64 on request) restatement of the reference crate's sampler,
DiT forward, condition encoders and DACVAE decoder.  It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` -- as the checker, never as the thing measured or shipped.  The
product path is the CUDA library under ``irodori-tts-burn_b200/csrc``.

Parity status: the reference (Rust + burn 0.21.0-pre.3) cannot be compiled in
this environment and ships no golden tensors, so cross-implementation numerics
are *unpinned*.  This restatement is pinned to the reference's own in-crate
unit-test invariants (known-answer tests in ``tests/test_oracle_kat.py``).

Every function names the reference file:line it restates (paths relative to
the Irodori-TTS-burn crate root).
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

Tensor = torch.Tensor

# ---------------------------------------------------------------------------
# Model configuration  (src/config/model.rs:8-82, validate :95-223)
# ---------------------------------------------------------------------------

DEFAULT_MODEL_CONFIG = dict(
    latent_dim=128,
    latent_patch_size=1,
    model_dim=2048,
    num_layers=24,
    num_heads=16,
    mlp_ratio=2.875,
    text_mlp_ratio=2.6,
    speaker_mlp_ratio=2.6,
    dropout=0.0,
    text_vocab_size=102400,
    text_tokenizer_repo="sbintuitions/sarashina2.2-0.5b",
    text_add_bos=True,
    text_dim=1280,
    text_layers=14,
    text_heads=10,
    use_caption_condition=False,
    caption_vocab_size=None,
    caption_tokenizer_repo=None,
    caption_add_bos=None,
    caption_dim=None,
    caption_layers=None,
    caption_heads=None,
    caption_mlp_ratio=None,
    speaker_dim=1280,
    speaker_layers=14,
    speaker_heads=10,
    speaker_patch_size=1,
    timestep_embed_dim=512,
    adaln_rank=256,
    norm_eps=1e-5,
    fixed_target_latent_steps=None,
)


class ModelConfig:
    """Mirror of ``ModelConfig`` with ``#[serde(default)]`` semantics
    (src/config/model.rs:6-82): missing keys take the default values."""

    def __init__(self, **kw):
        d = dict(DEFAULT_MODEL_CONFIG)
        d.update(kw)
        self.__dict__.update(d)

    @classmethod
    def from_json(cls, s: str) -> "ModelConfig":
        return cls(**json.loads(s))

    def to_dict(self) -> dict:
        return {k: self.__dict__[k] for k in DEFAULT_MODEL_CONFIG}

    # src/config/model.rs:86-88
    def use_speaker_condition(self) -> bool:
        return not self.use_caption_condition

    def head_dim(self) -> int:  # :226-228
        return self.model_dim // self.num_heads

    def patched_latent_dim(self) -> int:  # :231-233
        return self.latent_dim * self.latent_patch_size

    def speaker_patched_latent_dim(self) -> int:  # :236-238
        return self.patched_latent_dim() * (self.speaker_patch_size or 1)

    def text_mlp_ratio_(self) -> float:
        return self.text_mlp_ratio if self.text_mlp_ratio is not None else self.mlp_ratio

    def speaker_mlp_ratio_(self) -> float:
        return self.speaker_mlp_ratio if self.speaker_mlp_ratio is not None else self.mlp_ratio

    def caption_dim_(self) -> int:
        return self.caption_dim if self.caption_dim is not None else self.text_dim

    def caption_layers_(self) -> int:
        return self.caption_layers if self.caption_layers is not None else self.text_layers

    def caption_heads_(self) -> int:
        return self.caption_heads if self.caption_heads is not None else self.text_heads

    def caption_vocab_size_(self) -> int:
        return self.caption_vocab_size if self.caption_vocab_size is not None else self.text_vocab_size

    def caption_mlp_ratio_(self) -> float:
        if self.caption_mlp_ratio is not None:
            return self.caption_mlp_ratio
        return self.text_mlp_ratio_()

    def hidden_dim(self) -> int:
        # src/model/diffusion.rs:32,45-47: ((dim as f64 * ratio) as usize).max(1)
        return max(int(self.model_dim * self.mlp_ratio), 1)

    def validate(self) -> None:
        """src/config/model.rs:95-223 -- raises ValueError with the reference's text."""
        if self.model_dim == 0:
            raise ValueError("model_dim must be > 0")
        if self.num_heads == 0:
            raise ValueError("num_heads must be > 0")
        if self.model_dim % self.num_heads:
            raise ValueError(
                f"model_dim ({self.model_dim}) must be divisible by num_heads ({self.num_heads})")
        if self.head_dim() % 2:
            raise ValueError(f"head_dim ({self.head_dim()}) must be even for RoPE")
        if self.latent_patch_size == 0:
            raise ValueError("latent_patch_size must be > 0")
        if self.timestep_embed_dim == 0:
            raise ValueError("timestep_embed_dim must be > 0")
        if self.adaln_rank == 0:
            raise ValueError("adaln_rank must be > 0")
        if self.text_dim == 0:
            raise ValueError("text_dim must be > 0")
        if self.text_heads == 0:
            raise ValueError("text_heads must be > 0")
        if self.text_dim % self.text_heads:
            raise ValueError(
                f"text_dim ({self.text_dim}) must be divisible by text_heads ({self.text_heads})")
        if (self.text_dim // self.text_heads) % 2:
            raise ValueError(
                f"text head_dim ({self.text_dim // self.text_heads}) must be even for RoPE")
        if self.use_speaker_condition():
            for k in ("speaker_dim", "speaker_heads", "speaker_layers", "speaker_patch_size"):
                if getattr(self, k) is None:
                    raise ValueError(f"{k} must be set when use_caption_condition is false")
            if self.speaker_dim == 0:
                raise ValueError("speaker_dim must be > 0")
            if self.speaker_heads == 0:
                raise ValueError("speaker_heads must be > 0")
            if self.speaker_dim % self.speaker_heads:
                raise ValueError(
                    f"speaker_dim ({self.speaker_dim}) must be divisible by speaker_heads "
                    f"({self.speaker_heads})")
            if (self.speaker_dim // self.speaker_heads) % 2:
                raise ValueError(
                    f"speaker head_dim ({self.speaker_dim // self.speaker_heads}) must be even for RoPE")
        if self.use_caption_condition:
            cd, ch = self.caption_dim_(), self.caption_heads_()
            if cd == 0:
                raise ValueError("caption_dim must be > 0")
            if ch == 0:
                raise ValueError("caption_heads must be > 0")
            if cd % ch:
                raise ValueError(f"caption_dim ({cd}) must be divisible by caption_heads ({ch})")
            if (cd // ch) % 2:
                raise ValueError(f"caption head_dim ({cd // ch}) must be even for RoPE")


# ---------------------------------------------------------------------------
# Sampler parameters  (src/rf/params.rs:9-183, src/config/sampling.rs:8-30)
# ---------------------------------------------------------------------------

@dataclass
class GuidanceConfig:
    """src/rf/params.rs:9-35 (defaults at :24-35)."""
    mode: str = "independent"  # independent | joint | alternating
    scale_text: float = 3.0
    scale_caption: float = 3.0
    scale_speaker: float = 5.0
    min_t: float = 0.5
    max_t: float = 1.0


@dataclass
class SpeakerKvConfig:
    """src/rf/params.rs:48-58."""
    scale: float
    max_layers: Optional[int] = None
    min_t: Optional[float] = None


def _rs_f32(x: float) -> str:
    """An f32 formatted the way Rust's `Display` does (shortest decimal that
    round-trips the f32, no exponent, integral values without a fraction,
    `NaN` / `inf` / `-inf`): the reference's error messages print f32 fields
    this way."""
    import numpy as np
    if math.isnan(x):
        return "NaN"
    if math.isinf(x):
        return "inf" if x > 0 else "-inf"
    return np.format_float_positional(np.float32(x), unique=True, trim="-")


@dataclass
class SamplerParams:
    """src/rf/params.rs:61-92."""
    num_steps: int = 40
    method: str = "euler"  # euler | heun | plms4
    guidance: GuidanceConfig = field(default_factory=GuidanceConfig)
    truncation_factor: Optional[float] = None
    temporal_rescale: Optional[Tuple[float, float]] = None  # (k, sigma)
    speaker_kv: Optional[SpeakerKvConfig] = None
    use_context_kv_cache: bool = True

    def validate(self) -> None:
        """src/rf/params.rs:99-183 -- raises ValueError with the reference's text."""
        if self.num_steps == 0:
            raise ValueError("num_steps must be > 0")
        g = self.guidance
        for name, s in (("guidance.scale_text", g.scale_text),
                        ("guidance.scale_caption", g.scale_caption),
                        ("guidance.scale_speaker", g.scale_speaker)):
            if not math.isfinite(s):
                raise ValueError(f"{name} must be finite, got {_rs_f32(s)}")
        if not math.isfinite(g.min_t) or not (0.0 <= g.min_t <= 1.0):
            raise ValueError(f"guidance.min_t must be finite and in [0, 1], got {_rs_f32(g.min_t)}")
        if not math.isfinite(g.max_t) or not (0.0 <= g.max_t <= 1.0):
            raise ValueError(f"guidance.max_t must be finite and in [0, 1], got {_rs_f32(g.max_t)}")
        if g.min_t > g.max_t:
            raise ValueError(f"guidance.min_t ({_rs_f32(g.min_t)}) must not exceed guidance.max_t "
                             f"({_rs_f32(g.max_t)})")
        if self.truncation_factor is not None and (
                self.truncation_factor <= 0.0 or not math.isfinite(self.truncation_factor)):
            raise ValueError("truncation_factor must be finite and > 0")
        if self.temporal_rescale is not None:
            k, sigma = self.temporal_rescale
            if not math.isfinite(k):
                raise ValueError("temporal_rescale.k must be finite")
            if sigma == 0.0:
                raise ValueError("temporal_rescale.sigma must not be zero")
        if self.speaker_kv is not None:
            s = self.speaker_kv
            if not math.isfinite(s.scale) or s.scale <= 0.0:
                raise ValueError("speaker_kv.scale must be finite and > 0")
            if s.min_t is not None and (not math.isfinite(s.min_t) or not (0.0 <= s.min_t <= 1.0)):
                raise ValueError("speaker_kv.min_t must be finite and in [0, 1]")
        if self.method == "plms4" and g.mode == "alternating":
            raise ValueError(
                "sampler PLMS4 is not compatible with cfg_guidance_mode=Alternating; "
                "use Independent or Joint instead")


@dataclass
class SamplingRequest:
    """src/rf/params.rs:234-247.  Masks are bool tensors (True = valid)."""
    text_ids: Tensor
    text_mask: Tensor
    sequence_length: int
    ref_latent: Optional[Tensor] = None
    ref_mask: Optional[Tensor] = None
    caption_ids: Optional[Tensor] = None
    caption_mask: Optional[Tensor] = None
    initial_noise: Optional[Tensor] = None


# ---------------------------------------------------------------------------
# Weights (safetensors + config_json; src/weights/tensor_store.rs:26-53,
# key map src/weights/record_builders.rs:37-328)
# ---------------------------------------------------------------------------

class Weights:
    """All checkpoint tensors decoded to the oracle dtype, PyTorch [out, in]
    layout kept (the reference transposes at load and multiplies x @ W; the
    oracle multiplies x @ W.T, which is the same product)."""

    def __init__(self, tensors: Dict[str, Tensor], config_json: str, dtype=torch.float32):
        self.t = {k: v.to(dtype) for k, v in tensors.items()}
        self.cfg = ModelConfig.from_json(config_json)
        self.dtype = dtype

    @classmethod
    def load(cls, path: str, dtype=torch.float32) -> "Weights":
        from safetensors import safe_open
        with safe_open(path, framework="pt") as f:
            meta = f.metadata() or {}
            if "config_json" not in meta:
                raise KeyError("Checkpoint is missing the 'config_json' metadata key")
            tensors = {k: f.get_tensor(k) for k in f.keys()}
        w = cls(tensors, meta["config_json"], dtype)
        w.cfg.validate()
        return w

    def __getitem__(self, k: str) -> Tensor:
        if k not in self.t:
            raise KeyError(f"Missing weight tensor: {k}")
        return self.t[k]

    def has(self, k: str) -> bool:
        return k in self.t


def linear(W: Weights, prefix: str, x: Tensor) -> Tensor:
    """burn ``Linear::forward`` with the transposed PyTorch weight
    (src/weights/record_builders.rs:37-66)."""
    y = x @ W[f"{prefix}.weight"].T
    if W.has(f"{prefix}.bias"):
        y = y + W[f"{prefix}.bias"]
    return y


# ---------------------------------------------------------------------------
# Norms  (src/model/norm.rs)
# ---------------------------------------------------------------------------

def rms_norm(x: Tensor, w: Optional[Tensor], eps: float) -> Tensor:
    """RmsNorm::forward (src/model/norm.rs:25-39): divide by sqrt(mean+eps)."""
    rms = (x * x).mean(dim=-1, keepdim=True).add(eps).sqrt()
    y = x / rms
    return y * w if w is not None else y


def head_rms_norm(x: Tensor, w: Tensor, eps: float) -> Tensor:
    """HeadRmsNorm::forward (src/model/norm.rs:60-74); x [B,S,H,hd], w [H,hd]."""
    rms = (x * x).mean(dim=3, keepdim=True).add(eps).sqrt()
    return x / rms * w


def silu(x: Tensor) -> Tensor:
    return x * torch.sigmoid(x)


def low_rank_adaln(W: Weights, prefix: str, x: Tensor, cond_embed: Tensor, eps: float):
    """LowRankAdaLn::forward (src/model/norm.rs:135-173).

    cond_embed [B,1,3D] -> (modulated [B,S,D], tanh gate [B,1,D])."""
    raw_shift, raw_scale, raw_gate = cond_embed.chunk(3, dim=2)
    shift = linear(W, f"{prefix}.shift_up", linear(W, f"{prefix}.shift_down", silu(raw_shift))) + raw_shift
    scale = linear(W, f"{prefix}.scale_up", linear(W, f"{prefix}.scale_down", silu(raw_scale))) + raw_scale
    gate = linear(W, f"{prefix}.gate_up", linear(W, f"{prefix}.gate_down", silu(raw_gate))) + raw_gate
    x_norm = rms_norm(x, None, eps)
    return x_norm * (scale + 1.0) + shift, torch.tanh(gate)


# ---------------------------------------------------------------------------
# RoPE and timestep embedding  (src/model/rope.rs)
# ---------------------------------------------------------------------------

def rope_tables(head_dim: int, seq_len: int, theta: float = 10000.0, dtype=torch.float32):
    """precompute_rope_freqs (src/model/rope.rs:24-63): f32 host arithmetic,
    freqs[i] = 1 / theta^(2i/hd), angle = pos * freq, tables [S, hd/2]."""
    half = head_dim // 2
    i = torch.arange(half, dtype=torch.float32)
    freqs = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float32), 2.0 * i / float(head_dim))
    t = torch.arange(seq_len, dtype=torch.float32)
    ang = t[:, None] * freqs[None, :]
    return torch.cos(ang).to(dtype), torch.sin(ang).to(dtype)


def apply_rotary_emb(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """apply_rotary_emb (src/model/rope.rs:82-113): interleaved pairs (2k, 2k+1)."""
    B, S, H, hd = x.shape
    x5 = x.reshape(B, S, H, hd // 2, 2)
    re, im = x5[..., 0], x5[..., 1]
    c = cos[:S].reshape(1, S, 1, hd // 2)
    s = sin[:S].reshape(1, S, 1, hd // 2)
    out_re = re * c - im * s
    out_im = re * s + im * c
    return torch.stack([out_re, out_im], dim=4).reshape(B, S, H, hd)


def apply_rotary_half(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """apply_rotary_half (src/model/rope.rs:119-135): RoPE on heads [0, H/2)."""
    H = x.shape[2]
    hh = H // 2
    return torch.cat([apply_rotary_emb(x[:, :, :hh], cos, sin), x[:, :, hh:]], dim=2)


def timestep_embedding(t: Tensor, dim: int) -> Tensor:
    """get_timestep_embedding (src/model/rope.rs:141-165):
    freqs_i = 1000 * exp(-ln(1e4) * i / half) computed in f32; [cos | sin]."""
    half = dim // 2
    log_10000 = torch.log(torch.tensor(10000.0, dtype=torch.float32))
    i = torch.arange(half, dtype=torch.float32)
    freqs = 1000.0 * torch.exp((-log_10000 * i) / float(half))
    args = t.to(torch.float32)[:, None] * freqs[None, :]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=1)


# ---------------------------------------------------------------------------
# Attention  (src/model/attention.rs)
# ---------------------------------------------------------------------------

def sdpa(q: Tensor, k: Tensor, v: Tensor, mask: Optional[Tensor], scale: float) -> Tensor:
    """scaled_dot_product_attention (src/model/attention.rs:619-664) with the
    safe-softmax semantics of manual_sdpa (:675-724): masked keys are skipped
    (-inf), a fully masked row yields 0 (never NaN).

    q [B,Sq,H,hd], k/v [B,Sk,H,hd], mask [B,Sk] bool (True = attend)."""
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    scores = (qh @ kh.transpose(2, 3)) * scale
    if mask is not None:
        scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
    w = torch.softmax(scores, dim=3)
    w = torch.nan_to_num(w, nan=0.0)
    if mask is not None:
        # a masked V row must not leak (0 * NaN): zero the masked weights exactly
        w = w.masked_fill(~mask[:, None, None, :], 0.0)
        vh = vh.masked_fill(~mask[:, None, :, None], 0.0)
    return (w @ vh).transpose(1, 2)


def self_attention(W: Weights, prefix: str, x: Tensor, cos, sin, mask, num_heads: int, eps: float):
    """SelfAttention::forward (src/model/attention.rs:93-121): full RoPE, sigmoid gate."""
    B, S, D = x.shape
    hd = D // num_heads
    q = linear(W, f"{prefix}.wq", x).reshape(B, S, num_heads, hd)
    k = linear(W, f"{prefix}.wk", x).reshape(B, S, num_heads, hd)
    v = linear(W, f"{prefix}.wv", x).reshape(B, S, num_heads, hd)
    q = head_rms_norm(q, W[f"{prefix}.q_norm.weight"], eps)
    k = head_rms_norm(k, W[f"{prefix}.k_norm.weight"], eps)
    q = apply_rotary_emb(q, cos, sin)
    k = apply_rotary_emb(k, cos, sin)
    out = sdpa(q, k, v, mask, hd ** -0.5).reshape(B, S, D)
    out = out * torch.sigmoid(linear(W, f"{prefix}.gate", x))
    return linear(W, f"{prefix}.wo", out)


def swiglu(W: Weights, prefix: str, x: Tensor) -> Tensor:
    """SwiGlu::forward (src/model/feed_forward.rs:48-68): w2(silu(w1 x) * w3 x)."""
    return linear(W, f"{prefix}.w2", silu(linear(W, f"{prefix}.w1", x)) * linear(W, f"{prefix}.w3", x))


# ---------------------------------------------------------------------------
# Condition encoders  (src/model/text_encoder.rs, speaker_encoder.rs,
# dit/aux_conditioner.rs)
# ---------------------------------------------------------------------------

def text_block(W: Weights, prefix: str, x, mask, cos, sin, heads: int, eps: float):
    """TextBlock::forward (src/model/text_encoder.rs:46-60): pre-norm residual."""
    a = self_attention(W, f"{prefix}.attention", rms_norm(x, W[f"{prefix}.attention_norm.weight"], eps),
                       cos, sin, mask, heads, eps)
    x = x + a
    m = swiglu(W, f"{prefix}.mlp", rms_norm(x, W[f"{prefix}.mlp_norm.weight"], eps))
    return x + m


def text_encoder(W: Weights, prefix: str, ids: Tensor, mask: Tensor, layers: int, heads: int, eps: float):
    """TextEncoder::forward (src/model/text_encoder.rs:127-148): embed, hard-mask,
    blocks with re-mask after each."""
    x = W[f"{prefix}.text_embedding.weight"][ids.long()]
    mf = mask.to(x.dtype)[:, :, None]
    x = x * mf
    hd = x.shape[2] // heads
    cos, sin = rope_tables(hd, ids.shape[1], dtype=x.dtype)
    for i in range(layers):
        x = text_block(W, f"{prefix}.blocks.{i}", x, mask, cos, sin, heads, eps)
        x = x * mf
    return x * mf


def patch_sequence_with_mask(seq: Tensor, mask: Tensor, p: int):
    """src/model/speaker_encoder.rs:24-57."""
    if p <= 1:
        return seq, mask
    B, S, D = seq.shape
    usable = (S // p) * p
    if usable == 0:
        raise ValueError(f"Sequence too short for speaker_patch_size={p}: seq_len={S}")
    seq = seq[:, :usable].reshape(B, usable // p, D * p)
    m = mask[:, :usable].reshape(B, usable // p, p).all(dim=2)
    return seq, m


def speaker_encoder(W: Weights, prefix: str, latent: Tensor, mask: Tensor, layers: int, heads: int, eps: float):
    """ReferenceLatentEncoder::forward (src/model/speaker_encoder.rs:141-162):
    in_proj / 6, hard-mask, blocks with re-mask."""
    x = linear(W, f"{prefix}.in_proj", latent) / 6.0
    mf = mask.to(x.dtype)[:, :, None]
    x = x * mf
    hd = x.shape[2] // heads
    cos, sin = rope_tables(hd, latent.shape[1], dtype=x.dtype)
    for i in range(layers):
        x = text_block(W, f"{prefix}.blocks.{i}", x, mask, cos, sin, heads, eps)
        x = x * mf
    return x * mf


def prepend_masked_mean_token(state: Tensor, mask: Tensor):
    """src/model/dit/aux_conditioner.rs:161-190."""
    mf = mask.to(state.dtype)[:, :, None]
    s = (state * mf).sum(dim=1, keepdim=True)
    count = mf.sum(dim=1, keepdim=True).clamp_min(1.0)
    mean = s / count
    has_any = mf.sum(dim=1).reshape(-1, 1) > 0.0
    return torch.cat([mean, state], dim=1), torch.cat([has_any, mask], dim=1)


@dataclass
class Cond:
    """EncodedCondition (src/model/condition.rs:132-137); aux_kind in
    {None, 'speaker', 'caption'}."""
    text_state: Tensor
    text_mask: Tensor
    aux_kind: Optional[str] = None
    aux_state: Optional[Tensor] = None
    aux_mask: Optional[Tensor] = None

    def zeros_like(self) -> "Cond":
        """src/model/condition.rs:144-154 (aux variant preserved, :46-59)."""
        return Cond(torch.zeros_like(self.text_state), torch.zeros_like(self.text_mask),
                    self.aux_kind,
                    None if self.aux_state is None else torch.zeros_like(self.aux_state),
                    None if self.aux_mask is None else torch.zeros_like(self.aux_mask))


def cat_batch(conds: List[Cond]) -> Cond:
    """EncodedCondition::cat_batch (src/model/condition.rs:168-220)."""
    c0 = conds[0]
    return Cond(torch.cat([c.text_state for c in conds], 0), torch.cat([c.text_mask for c in conds], 0),
                c0.aux_kind,
                None if c0.aux_state is None else torch.cat([c.aux_state for c in conds], 0),
                None if c0.aux_mask is None else torch.cat([c.aux_mask for c in conds], 0))


def encode_conditions(W: Weights, req: SamplingRequest) -> Cond:
    """TextToLatentRfDiT::encode_conditions (src/model/dit/model.rs:182-205) with
    AuxConditionInput::from_request (src/model/condition.rs:104-122) and
    AuxConditioner::encode (src/model/dit/aux_conditioner.rs:60-107)."""
    cfg = W.cfg
    eps = cfg.norm_eps
    ts = text_encoder(W, "text_encoder", req.text_ids, req.text_mask, cfg.text_layers, cfg.text_heads, eps)
    ts = rms_norm(ts, W["text_norm.weight"], eps)
    cond = Cond(ts, req.text_mask.clone())
    if req.ref_latent is not None and req.ref_mask is not None:
        if not cfg.use_speaker_condition():
            raise ValueError("caption conditioner received speaker input; check that the checkpoint "
                             "and inference request use the same conditioning mode")
        lat, m = patch_sequence_with_mask(req.ref_latent.to(W.dtype), req.ref_mask, cfg.speaker_patch_size or 1)
        st = speaker_encoder(W, "speaker_encoder", lat, m, cfg.speaker_layers, cfg.speaker_heads, eps)
        st = rms_norm(st, W["speaker_norm.weight"], eps)
        st, sm = prepend_masked_mean_token(st, m)
        cond.aux_kind, cond.aux_state, cond.aux_mask = "speaker", st, sm
    elif req.caption_ids is not None and req.caption_mask is not None:
        if not cfg.use_caption_condition:
            raise ValueError("speaker conditioner received caption input; check that the checkpoint "
                             "and inference request use the same conditioning mode")
        cs = text_encoder(W, "caption_encoder", req.caption_ids, req.caption_mask, cfg.caption_layers_(),
                          cfg.caption_heads_(), eps)
        cs = rms_norm(cs, W["caption_norm.weight"], eps)
        cond.aux_kind, cond.aux_state, cond.aux_mask = "caption", cs, req.caption_mask.clone()
    return cond


# ---------------------------------------------------------------------------
# Context KV cache  (src/model/attention.rs:431-501, dit/model.rs:444-472)
# ---------------------------------------------------------------------------

@dataclass
class KvCache:
    text_k: Tensor
    text_v: Tensor
    aux_k: Optional[Tensor]
    aux_v: Optional[Tensor]
    ctx_mask: Tensor

    @property
    def ctx_k(self):
        return self.text_k if self.aux_k is None else torch.cat([self.text_k, self.aux_k], 1)

    @property
    def ctx_v(self):
        return self.text_v if self.aux_v is None else torch.cat([self.text_v, self.aux_v], 1)


def build_kv_caches(W: Weights, cond: Cond) -> List[KvCache]:
    """JointAttention::build_kv_cache per block: k = k_norm(W_k_text text),
    v = W_v_text text (no RoPE on context keys); same for speaker/caption."""
    cfg = W.cfg
    H, hd, eps = cfg.num_heads, cfg.head_dim(), cfg.norm_eps
    out = []
    B, T, _ = cond.text_state.shape
    for i in range(cfg.num_layers):
        p = f"blocks.{i}.attention"
        kn = W[f"{p}.k_norm.weight"]
        tk = head_rms_norm(linear(W, f"{p}.wk_text", cond.text_state).reshape(B, T, H, hd), kn, eps)
        tv = linear(W, f"{p}.wv_text", cond.text_state).reshape(B, T, H, hd)
        ak = av = None
        mask = cond.text_mask
        if cond.aux_state is not None:
            suf = "speaker" if W.has(f"{p}.wk_speaker.weight") else "caption"
            if W.has(f"{p}.wk_{suf}.weight"):
                A = cond.aux_state.shape[1]
                ak = head_rms_norm(linear(W, f"{p}.wk_{suf}", cond.aux_state).reshape(B, A, H, hd), kn, eps)
                av = linear(W, f"{p}.wv_{suf}", cond.aux_state).reshape(B, A, H, hd)
            mask = torch.cat([cond.text_mask, cond.aux_mask], 1)
        out.append(KvCache(tk, tv, ak, av, mask))
    return out


def scale_speaker_kv_cache(caches: List[KvCache], scale: float, max_layers: Optional[int]) -> List[KvCache]:
    """src/rf/kv_scaling.rs:10-60."""
    n = len(caches) if max_layers is None else min(max_layers, len(caches))
    res = []
    for i, c in enumerate(caches):
        if i < n:
            res.append(KvCache(c.text_k, c.text_v,
                               None if c.aux_k is None else c.aux_k * scale,
                               None if c.aux_v is None else c.aux_v * scale, c.ctx_mask))
        else:
            res.append(c)
    return res


# ---------------------------------------------------------------------------
# DiT forward  (src/model/dit/model.rs:354-393, diffusion.rs:62-105,
# attention.rs:272-425, feed_forward.rs:76-85)
# ---------------------------------------------------------------------------

def cond_module(W: Weights, t: Tensor) -> Tensor:
    """CondModule::forward (src/model/dit/model.rs:80-85) after the timestep embedding."""
    emb = timestep_embedding(t, W.cfg.timestep_embed_dim).to(W.dtype)
    x = silu(linear(W, "cond_module.linear0", emb))
    x = silu(linear(W, "cond_module.linear1", x))
    return linear(W, "cond_module.linear2", x)[:, None, :]


def joint_attention(W: Weights, p: str, h: Tensor, kv: KvCache, cos, sin, latent_mask: Optional[Tensor]):
    """JointAttention::forward_fused + attention_after_qkv (src/model/attention.rs:272-425)."""
    cfg = W.cfg
    B, S, D = h.shape
    H, hd, eps = cfg.num_heads, cfg.head_dim(), cfg.norm_eps
    key = f"{p}.__fused_qkv"  # prepare_for_inference (src/model/attention.rs:514-523), built once
    if key not in W.t:
        W.t[key] = torch.cat([W[f"{p}.wq.weight"], W[f"{p}.wk.weight"], W[f"{p}.wv.weight"]], 0)
    qkv = h @ W.t[key].T
    q, k, v = (qkv[..., i * D:(i + 1) * D].reshape(B, S, H, hd) for i in range(3))
    q = apply_rotary_half(head_rms_norm(q, W[f"{p}.q_norm.weight"], eps), cos, sin)
    k = apply_rotary_half(head_rms_norm(k, W[f"{p}.k_norm.weight"], eps), cos, sin)
    k_all = torch.cat([k, kv.ctx_k], 1)
    v_all = torch.cat([v, kv.ctx_v], 1)
    self_part = torch.ones(B, S, dtype=torch.bool) if latent_mask is None else latent_mask
    mask = torch.cat([self_part, kv.ctx_mask], 1)
    out = sdpa(q, k_all, v_all, mask, hd ** -0.5).reshape(B, S, D)
    gated = torch.sigmoid(h @ W[f"{p}.gate.weight"].T) * out
    return gated @ W[f"{p}.wo.weight"].T


def dit_forward(W: Weights, x_t: Tensor, t: Tensor, kv: List[KvCache], cos, sin,
                latent_mask: Optional[Tensor] = None, capture: bool = False):
    """forward_backbone_fused (src/model/dit/model.rs:354-393); with capture=True
    also returns (after_in_proj, [block outputs]) like forward_with_cond_debug
    (:269-346)."""
    cfg = W.cfg
    eps = cfg.norm_eps
    ce = cond_module(W, t)
    x = linear(W, "in_proj", x_t.to(W.dtype))
    after_in = x
    outs = []
    for i in range(cfg.num_layers):
        b = f"blocks.{i}"
        h, g = low_rank_adaln(W, f"{b}.attention_adaln", x, ce, eps)
        x = x + g * joint_attention(W, f"{b}.attention", h, kv[i], cos, sin, latent_mask)
        h, g = low_rank_adaln(W, f"{b}.mlp_adaln", x, ce, eps)
        key = f"{b}.mlp.__fused_w13"  # src/model/feed_forward.rs:96-103, built once
        if key not in W.t:
            W.t[key] = torch.cat([W[f"{b}.mlp.w1.weight"], W[f"{b}.mlp.w3.weight"]], 0)
        a = h @ W.t[key].T
        F_ = a.shape[-1] // 2
        x = x + g * ((silu(a[..., :F_]) * a[..., F_:]) @ W[f"{b}.mlp.w2.weight"].T)
        if capture:
            outs.append(x)
    v = linear(W, "out_proj", rms_norm(x, W["out_norm.weight"], eps))
    if capture:
        return v, after_in, outs
    return v


# ---------------------------------------------------------------------------
# Sampler  (src/rf/euler_sampler.rs:132-718, math.rs:38-52)
# ---------------------------------------------------------------------------

def t_schedule(num_steps: int) -> List[float]:
    """src/rf/euler_sampler.rs:325-328, evaluated in f32."""
    import numpy as np
    init = np.float32(0.999)
    n = np.float32(num_steps)
    return [float(init * (np.float32(1.0) - np.float32(i) / n)) for i in range(num_steps + 1)]


def ab_extrapolate(hist: List[Tensor]) -> Tensor:
    """Adams-Bashforth AB-1..AB-4, newest first (src/rf/euler_sampler.rs:99-116)."""
    n = len(hist)
    if n == 1:
        return hist[0]
    if n == 2:
        return hist[0] * 1.5 + hist[1] * -0.5
    if n == 3:
        return hist[0] * (23.0 / 12.0) + hist[1] * (-16.0 / 12.0) + hist[2] * (5.0 / 12.0)
    return (hist[0] * (55.0 / 24.0) + hist[1] * (-59.0 / 24.0) + hist[2] * (37.0 / 24.0)
            + hist[3] * (-9.0 / 24.0))


def temporal_score_rescale(v: Tensor, x: Tensor, t: float, k: float, sigma: float) -> Tensor:
    """src/rf/math.rs:38-52 (scalar arithmetic in f32)."""
    import numpy as np
    if t >= 1.0:
        return v
    t32 = np.float32(t)
    omt = np.float32(1.0) - t32
    snr = (omt * omt) / (t32 * t32)
    ss = np.float32(sigma) * np.float32(sigma)
    ratio = (snr * ss + np.float32(1.0)) / (snr * ss / np.float32(k) + np.float32(1.0))
    return (v * float(omt) + x) * float(ratio) / float(omt) - x / float(omt)


def sample_euler_rf_cfg(W: Weights, req: SamplingRequest, params: SamplerParams,
                        record_forwards: Optional[list] = None) -> Tensor:
    """sample_euler_rf_cfg (src/rf/euler_sampler.rs:132-718).

    Joint mode runs cond and uncond as separate forwards exactly like the
    reference; rows never interact so any batching of them is equivalent."""
    import numpy as np
    params.validate()
    cfg = W.cfg
    B = req.text_ids.shape[0]
    P = cfg.patched_latent_dim()
    if req.initial_noise is None:
        raise ValueError("the oracle needs an explicit initial_noise")
    x = req.initial_noise.to(W.dtype).clone()
    if params.truncation_factor is not None:
        x = x * params.truncation_factor
    g = params.guidance
    s_text, s_cap = g.scale_text, g.scale_caption
    s_spk = g.scale_speaker if cfg.use_speaker_condition() else 0.0

    cond = encode_conditions(W, req)
    uncond = cond.zeros_like()
    S = req.sequence_length
    cos, sin = rope_tables(cfg.head_dim(), S, dtype=W.dtype)

    has_text = s_text > 0.0
    has_spk = s_spk > 0.0 and cond.aux_kind == "speaker"
    has_cap = s_cap > 0.0 and cond.aux_kind == "caption" and bool(cond.aux_mask.any())
    enabled = [n for n, on in (("text", has_text), ("speaker", has_spk), ("caption", has_cap)) if on]
    scale_of = {"text": s_text, "speaker": s_spk, "caption": s_cap}

    if g.mode == "joint" and enabled:
        sc = [scale_of[n] for n in enabled]
        if max(sc) - min(sc) >= 1e-6:
            raise ValueError(
                "cfg_guidance_mode=Joint requires all active cfg scales to be equal, but got "
                f"text={g.scale_text}, speaker={g.scale_speaker}, caption={g.scale_caption}. "
                "Pass a single equal value for all active signals.")

    def single_uncond(name):  # src/rf/euler_sampler.rs:43-83
        if name == "text":
            return Cond(uncond.text_state, uncond.text_mask, cond.aux_kind, cond.aux_state, cond.aux_mask)
        return Cond(cond.text_state, cond.text_mask, uncond.aux_kind, uncond.aux_state, uncond.aux_mask)

    # The cache is a pure function of the condition, so cached == uncached
    # (src/rf/euler_sampler.rs:1071-1314); the oracle always materialises it.
    skv = params.speaker_kv if cfg.use_speaker_condition() else None
    kv_cond = build_kv_caches(W, cond)
    if skv is not None:
        kv_cond = scale_speaker_kv_cache(kv_cond, skv.scale, skv.max_layers)
    kv_uncond = build_kv_caches(W, uncond) if (g.mode == "joint" and enabled) else None
    batched = g.mode == "independent" and len(enabled) > 0
    mult = 1 + len(enabled) if batched else 1
    bcond = cat_batch([cond] + [single_uncond(n) for n in enabled]) if batched else None
    kv_b = None
    if batched:
        kv_b = build_kv_caches(W, bcond)
        if skv is not None:
            kv_b = scale_speaker_kv_cache(kv_b, skv.scale, skv.max_layers)
    alt = g.mode == "alternating" and len(enabled) > 0
    kv_alt = {n: build_kv_caches(W, single_uncond(n)) for n in enabled} if alt else {}

    ts = t_schedule(params.num_steps)
    speaker_kv_active = params.speaker_kv is not None
    hist: List[Tensor] = []
    prev_regime = None

    def fwd(xx, t, kv, bsz):
        if record_forwards is not None:
            record_forwards.append(xx.shape[0])
        return dit_forward(W, xx, torch.full((bsz,), t, dtype=torch.float32), kv, cos, sin)

    f32 = np.float32
    min_t32, max_t32 = f32(g.min_t), f32(g.max_t)

    def in_window(t):  # f32 comparison as in src/rf/euler_sampler.rs:379
        return bool(enabled) and min_t32 <= f32(t) <= max_t32

    def guided(xx, t, i):
        use_cfg = in_window(t)
        if not use_cfg:
            return fwd(xx, t, kv_cond, B)
        if g.mode == "independent":
            out = fwd(torch.cat([xx] * mult, 0), t, kv_b, B * mult)
            ch = out.chunk(mult, 0)
            v = ch[0]
            for j, n in enumerate(enabled):
                v = v + (ch[0] - ch[j + 1]) * scale_of[n]
            return v
        vc = fwd(xx, t, kv_cond, B)
        if g.mode == "joint":
            vu = fwd(xx, t, kv_uncond, B)
            return vc + (vc - vu) * scale_of[enabled[0]]
        name = enabled[i % len(enabled)]
        va = fwd(xx, t, kv_alt[name], B)
        return vc + (vc - va) * scale_of[name]

    prev_regime = (in_window(ts[0]), speaker_kv_active)
    for i in range(params.num_steps):
        t, tn = ts[i], ts[i + 1]
        use_cfg = in_window(t)
        if params.method == "plms4":
            regime = (use_cfg, speaker_kv_active)
            if regime != prev_regime:
                hist.clear()
                prev_regime = regime
        v = guided(x, t, i)
        if params.temporal_rescale is not None:
            v = temporal_score_rescale(v, x, t, *params.temporal_rescale)
        if (speaker_kv_active and skv is not None and skv.min_t is not None
                and f32(tn) < f32(skv.min_t) and f32(t) >= f32(skv.min_t)):
            inv = 1.0 / skv.scale
            kv_cond = scale_speaker_kv_cache(kv_cond, inv, skv.max_layers)
            if kv_b is not None:
                kv_b = scale_speaker_kv_cache(kv_b, inv, skv.max_layers)
            speaker_kv_active = False
        dt = float(f32(tn) - f32(t))
        if params.method == "euler":
            v_eff = v
        elif params.method == "heun":
            x_pred = x + v * dt
            v2 = guided(x_pred, tn, i)
            if params.temporal_rescale is not None:
                v2 = temporal_score_rescale(v2, x_pred, tn, *params.temporal_rescale)
            v_eff = (v + v2) / 2.0
        else:
            hist.insert(0, v)
            if len(hist) > 4:
                hist.pop()
            v_eff = ab_extrapolate(hist)
        x = x + v_eff * dt
    return x


# ---------------------------------------------------------------------------
# DACVAE decoder  (src/codec/*.rs)
# ---------------------------------------------------------------------------

DECODER_RATES = (12, 10, 8, 2)          # src/codec/weights.rs:273-292
DECODER_CHANNELS = (1536, 768, 384, 192, 96)
CODEC_LATENT = 32
CODEC_EMBED = 1024
HOP_LENGTH = 1920                       # src/codec/weights.rs:39
SAMPLE_RATE = 48000


def snake(x: Tensor, alpha: Tensor) -> Tensor:
    """Snake1d::forward (src/codec/layers.rs:27-33): x + sin^2(a x) / (a + 1e-9)."""
    return x + torch.sin(x * alpha).pow(2) / (alpha + 1e-9)


def conv_pad(kernel: int, stride: int, dilation: int) -> int:
    """src/codec/layers.rs:64-66."""
    return (kernel - stride) * dilation // 2


def conv_transpose_pad(stride: int) -> Tuple[int, int]:
    """src/codec/layers.rs:71-75: ((s+1)//2, s%2)."""
    return (stride + 1) // 2, stride % 2


def _conv(W: Weights, prefix: str, x: Tensor, dilation: int = 1) -> Tensor:
    w = W[f"{prefix}.weight"]
    b = W.t.get(f"{prefix}.bias")
    k = w.shape[2]
    return torch.nn.functional.conv1d(x, w, b, stride=1, padding=conv_pad(k, 1, dilation), dilation=dilation)


def residual_unit(W: Weights, prefix: str, x: Tensor, dilation: int) -> Tensor:
    """ResidualUnit::forward (src/codec/layers.rs:44-60; keys weights.rs:105-141)."""
    y = snake(x, W[f"{prefix}.block.0.alpha"])
    y = _conv(W, f"{prefix}.block.1", y, dilation)
    y = snake(y, W[f"{prefix}.block.2.alpha"])
    y = _conv(W, f"{prefix}.block.3", y, 1)
    return y + x


def codec_decode(W: Weights, latent: Tensor) -> Tensor:
    """DacVaeCodec::decode (src/codec/model.rs:60-65): [B,T,32] -> [B,1,T*1920]."""
    x = latent.to(W.dtype).transpose(1, 2)
    x = torch.nn.functional.conv1d(x, W["quantizer.out_proj.weight"], W.t.get("quantizer.out_proj.bias"))
    x = _conv(W, "decoder.model.0", x)
    for bi, s in enumerate(DECODER_RATES):
        p = f"decoder.model.{bi + 1}"
        x = snake(x, W[f"{p}.block.0.alpha"])
        pad, opad = conv_transpose_pad(s)
        x = torch.nn.functional.conv_transpose1d(x, W[f"{p}.block.1.weight"], W.t.get(f"{p}.block.1.bias"),
                                                 stride=s, padding=pad, output_padding=opad)
        for j, d in zip((4, 5, 8), (1, 3, 9)):
            x = residual_unit(W, f"{p}.block.{j}", x, d)
    x = snake(x, W["decoder.wm_model.encoder_block.pre.0.alpha"])
    x = _conv(W, "decoder.wm_model.encoder_block.pre.1", x)
    return torch.tanh(x)


def load_codec(path: str, dtype=torch.float32) -> Weights:
    from safetensors import safe_open
    with safe_open(path, framework="pt") as f:
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    w = Weights.__new__(Weights)
    w.t = {k: v.to(dtype) for k, v in tensors.items()}
    w.cfg = None
    w.dtype = dtype
    return w
