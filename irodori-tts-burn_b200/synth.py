"""Seeded synthetic checkpoints and requests.

There is no network on the build or GPU hosts, so every benchmark and parity
case runs on random-init weights written in the reference's safetensors
layout (PyTorch ``[out, in]`` Linear weights, ``config_json`` metadata, the
``cond_module.linear{0,1,2}`` key names of src/weights/record_builders.rs:266-275)
and on seeded synthetic inputs with the shapes of the benchmark configs.

Init schemes
------------
``baseline``  every Linear / Embedding weight ~ N(0, 0.02); biases 0; norm
              weights 1; adaLN ``*_up`` weight and bias 0 (as the reference
              initialises them, src/model/norm.rs:108-119); ``out_proj`` ~
              N(0, 0.02) instead of the reference's zero init so that the
              sampler is not a no-op.
``full``      as ``baseline`` but adaLN ``*_up`` weights and all biases ~
              N(0, 0.02) and norm weights 1 + N(0, 0.1), so that every
              parameter influences the output (used by the parity tests).
"""

from __future__ import annotations

import json
import math
import os
from typing import Dict, Optional

import torch

# Small configurations used by the tests.  `tiny` mirrors the reference's
# tiny_model_config() (src/config/model.rs:285-312); `small` keeps the
# production head_dim (128) and 64-aligned widths so the tensor-core paths run.
TINY_CONFIG = dict(
    latent_dim=8, latent_patch_size=1, model_dim=32, num_heads=4, num_layers=1,
    mlp_ratio=2.0, text_mlp_ratio=2.0, speaker_mlp_ratio=2.0, dropout=0.0,
    text_dim=16, text_heads=2, text_layers=1, text_vocab_size=64,
    speaker_dim=16, speaker_layers=1, speaker_heads=2, speaker_patch_size=1,
    timestep_embed_dim=32, adaln_rank=16, norm_eps=1e-5, use_caption_condition=False,
)

SMALL_CONFIG = dict(
    latent_dim=32, latent_patch_size=1, model_dim=256, num_heads=2, num_layers=2,
    mlp_ratio=2.875, text_mlp_ratio=2.6, speaker_mlp_ratio=2.6, dropout=0.0,
    text_dim=256, text_heads=2, text_layers=2, text_vocab_size=512,
    speaker_dim=256, speaker_layers=2, speaker_heads=2, speaker_patch_size=1,
    timestep_embed_dim=64, adaln_rank=32, norm_eps=1e-5, use_caption_condition=False,
)

# The BASELINE default ModelConfig (src/config/model.rs:46-82).
DEFAULT_CONFIG = dict(
    latent_dim=128, latent_patch_size=1, model_dim=2048, num_layers=24, num_heads=16,
    mlp_ratio=2.875, text_mlp_ratio=2.6, speaker_mlp_ratio=2.6, dropout=0.0,
    text_vocab_size=102400, text_dim=1280, text_layers=14, text_heads=10,
    use_caption_condition=False, speaker_dim=1280, speaker_layers=14, speaker_heads=10,
    speaker_patch_size=1, timestep_embed_dim=512, adaln_rank=256, norm_eps=1e-5,
)


def _hidden(dim: int, ratio: float) -> int:
    return max(int(dim * ratio), 1)


def dit_param_shapes(cfg: dict) -> Dict[str, tuple]:
    """Every tensor the reference's record builders read, with its shape."""
    c = dict(DEFAULT_CONFIG)
    c.update(cfg)
    D, L, H = c["model_dim"], c["num_layers"], c["num_heads"]
    hd = D // H
    P = c["latent_dim"] * c["latent_patch_size"]
    F = _hidden(D, c["mlp_ratio"])
    r = max(1, min(c["adaln_rank"], D))
    shapes: Dict[str, tuple] = {}

    def text_blocks(prefix, dim, heads, layers, ratio):
        hid = _hidden(dim, ratio)
        thd = dim // heads
        for i in range(layers):
            b = f"{prefix}.blocks.{i}"
            shapes[f"{b}.attention_norm.weight"] = (dim,)
            for n in ("wq", "wk", "wv", "wo", "gate"):
                shapes[f"{b}.attention.{n}.weight"] = (dim, dim)
            shapes[f"{b}.attention.q_norm.weight"] = (heads, thd)
            shapes[f"{b}.attention.k_norm.weight"] = (heads, thd)
            shapes[f"{b}.mlp_norm.weight"] = (dim,)
            shapes[f"{b}.mlp.w1.weight"] = (hid, dim)
            shapes[f"{b}.mlp.w3.weight"] = (hid, dim)
            shapes[f"{b}.mlp.w2.weight"] = (dim, hid)

    td = c["text_dim"]
    tr = c.get("text_mlp_ratio") or c["mlp_ratio"]
    shapes["text_encoder.text_embedding.weight"] = (c["text_vocab_size"], td)
    text_blocks("text_encoder", td, c["text_heads"], c["text_layers"], tr)
    shapes["text_norm.weight"] = (td,)
    aux_dim = None
    aux_name = None
    if not c.get("use_caption_condition", False):
        sd = c["speaker_dim"]
        sr = c.get("speaker_mlp_ratio") or c["mlp_ratio"]
        sp = P * (c.get("speaker_patch_size") or 1)
        shapes["speaker_encoder.in_proj.weight"] = (sd, sp)
        shapes["speaker_encoder.in_proj.bias"] = (sd,)
        text_blocks("speaker_encoder", sd, c["speaker_heads"], c["speaker_layers"], sr)
        shapes["speaker_norm.weight"] = (sd,)
        aux_dim, aux_name = sd, "speaker"
    else:
        cd = c.get("caption_dim") or td
        ch = c.get("caption_heads") or c["text_heads"]
        cl = c.get("caption_layers") or c["text_layers"]
        cr = c.get("caption_mlp_ratio") or tr
        cv = c.get("caption_vocab_size") or c["text_vocab_size"]
        shapes["caption_encoder.text_embedding.weight"] = (cv, cd)
        text_blocks("caption_encoder", cd, ch, cl, cr)
        shapes["caption_norm.weight"] = (cd,)
        aux_dim, aux_name = cd, "caption"
    T = c["timestep_embed_dim"]
    shapes["cond_module.linear0.weight"] = (D, T)
    shapes["cond_module.linear1.weight"] = (D, D)
    shapes["cond_module.linear2.weight"] = (3 * D, D)
    shapes["in_proj.weight"] = (D, P)
    shapes["in_proj.bias"] = (D,)
    for i in range(L):
        b = f"blocks.{i}"
        for n in ("wq", "wk", "wv", "gate", "wo"):
            shapes[f"{b}.attention.{n}.weight"] = (D, D)
        shapes[f"{b}.attention.wk_text.weight"] = (D, td)
        shapes[f"{b}.attention.wv_text.weight"] = (D, td)
        shapes[f"{b}.attention.wk_{aux_name}.weight"] = (D, aux_dim)
        shapes[f"{b}.attention.wv_{aux_name}.weight"] = (D, aux_dim)
        shapes[f"{b}.attention.q_norm.weight"] = (H, hd)
        shapes[f"{b}.attention.k_norm.weight"] = (H, hd)
        shapes[f"{b}.mlp.w1.weight"] = (F, D)
        shapes[f"{b}.mlp.w3.weight"] = (F, D)
        shapes[f"{b}.mlp.w2.weight"] = (D, F)
        for a in ("attention_adaln", "mlp_adaln"):
            for n in ("shift", "scale", "gate"):
                shapes[f"{b}.{a}.{n}_down.weight"] = (r, D)
                shapes[f"{b}.{a}.{n}_up.weight"] = (D, r)
                shapes[f"{b}.{a}.{n}_up.bias"] = (D,)
    shapes["out_norm.weight"] = (D,)
    shapes["out_proj.weight"] = (P, D)
    shapes["out_proj.bias"] = (P,)
    return shapes


def _init_tensor(name: str, shape: tuple, init: str, gen: torch.Generator, device) -> torch.Tensor:
    is_norm = name.endswith("norm.weight")
    is_bias = name.endswith(".bias")
    is_up = "_up." in name
    if init == "baseline":
        if is_norm:
            return torch.ones(shape, device=device)
        if is_bias or is_up:
            return torch.zeros(shape, device=device)
        return torch.randn(shape, generator=gen, device=device) * 0.02
    if init == "full":
        if is_norm:
            return 1.0 + 0.1 * torch.randn(shape, generator=gen, device=device)
        return torch.randn(shape, generator=gen, device=device) * 0.02
    raise ValueError(f"unknown init {init!r}")


def write_safetensors(path: str, tensors: Dict[str, torch.Tensor], metadata: Dict[str, str]) -> None:
    """Write tensors in the safetensors container format (8-byte LE header
    length, JSON header, raw little-endian data)."""
    names = sorted(tensors)
    header = {"__metadata__": metadata}
    off = 0
    dt_name = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16"}
    for n in names:
        t = tensors[n]
        nb = t.numel() * t.element_size()
        header[n] = {"dtype": dt_name[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(len(hb).to_bytes(8, "little"))
        f.write(hb)
        for n in names:
            t = tensors[n].detach().contiguous().cpu()
            f.write(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.float32
                    else t.numpy().tobytes())
    os.replace(tmp, path)


def make_dit_checkpoint(path: str, cfg: dict, seed: int = 0, init: str = "baseline",
                        dtype: torch.dtype = torch.float32, device: str = "cpu") -> dict:
    """Write a random-init DiT checkpoint; returns the full config dict."""
    c = dict(DEFAULT_CONFIG)
    c.update(cfg)
    shapes = dit_param_shapes(c)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    tensors = {}
    for name in sorted(shapes):
        tensors[name] = _init_tensor(name, shapes[name], init, gen, device).to(dtype)
    write_safetensors(path, tensors, {"config_json": json.dumps(c)})
    return c


# ---------------------------------------------------------------------------
# DACVAE decoder checkpoint (weight-norm resolved, as convert_dacvae_weights.py
# writes it: w = g * v / ||v|| with the norm over every dim except 0)
# ---------------------------------------------------------------------------

CODEC_RATES = (12, 10, 8, 2)
CODEC_CHANNELS = (1536, 768, 384, 192, 96)


def codec_param_shapes(width_div: int = 1) -> Dict[str, tuple]:
    """Decoder-path tensors read by src/codec/weights.rs:219-292.  ``width_div``
    shrinks every channel count for fast CPU tests (1 = the real codec)."""
    ch = [c // width_div for c in CODEC_CHANNELS]
    emb = 1024 // width_div
    s: Dict[str, tuple] = {
        "quantizer.out_proj.weight": (emb, 32, 1),
        "quantizer.out_proj.bias": (emb,),
        "decoder.model.0.weight": (ch[0], emb, 7),
        "decoder.model.0.bias": (ch[0],),
    }
    for bi, st in enumerate(CODEC_RATES):
        p = f"decoder.model.{bi + 1}"
        cin, cout = ch[bi], ch[bi + 1]
        s[f"{p}.block.0.alpha"] = (1, cin, 1)
        s[f"{p}.block.1.weight"] = (cin, cout, 2 * st)
        s[f"{p}.block.1.bias"] = (cout,)
        for j in (4, 5, 8):
            r = f"{p}.block.{j}"
            s[f"{r}.block.0.alpha"] = (1, cout, 1)
            s[f"{r}.block.1.weight"] = (cout, cout, 7)
            s[f"{r}.block.1.bias"] = (cout,)
            s[f"{r}.block.2.alpha"] = (1, cout, 1)
            s[f"{r}.block.3.weight"] = (cout, cout, 1)
            s[f"{r}.block.3.bias"] = (cout,)
    s["decoder.wm_model.encoder_block.pre.0.alpha"] = (1, ch[-1], 1)
    s["decoder.wm_model.encoder_block.pre.1.weight"] = (1, ch[-1], 7)
    s["decoder.wm_model.encoder_block.pre.1.bias"] = (1,)
    return s


def weight_norm_split(tensors: Dict[str, torch.Tensor], seed: int = 11) -> Dict[str, torch.Tensor]:
    """Store every rank-3 ``X.weight`` as the PyTorch weight-norm pair
    ``X.weight_g`` [dim0, 1, 1] / ``X.weight_v`` (same shape) that resolves to
    it (g * v / ||v||, norm over all dims but 0; the form the reference's
    converter, scripts/convert_dacvae_weights.py, consumes).  v is the weight
    scaled by a random positive factor per dim-0 index."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    out: Dict[str, torch.Tensor] = {}
    for k, w in tensors.items():
        if k.endswith(".weight") and w.dim() == 3:
            wf = w.float()
            c = 0.5 + 1.5 * torch.rand((wf.shape[0], 1, 1), generator=gen)
            out[k[:-len(".weight")] + ".weight_v"] = (wf * c).to(w.dtype)
            out[k[:-len(".weight")] + ".weight_g"] = wf.flatten(1).norm(dim=1).reshape(-1, 1, 1).to(w.dtype)
        else:
            out[k] = w
    return out


def make_codec_checkpoint(path: str, seed: int = 5, width_div: int = 1,
                          dtype: torch.dtype = torch.float32, init: str = "weightnorm",
                          weight_norm: bool = False) -> None:
    """Random decoder weights.

    ``init="reference"``: the reference's own random initialisation of codec
    layers (``Conv1dConfig::init`` in src/codec/encoder.rs:78-95: burn's
    default Kaiming-uniform, weights and biases U(-1/sqrt(fan_in),
    1/sqrt(fan_in)); Snake alpha = 1).  ``fan_in`` = in_channels x kernel for
    Conv1d and out_channels x kernel for ConvTranspose1d ([in, out, k]).
    ``init="weightnorm"``: weight-norm form g * v / |v| with g ~ U(0.5, 1.5)
    per output row and alpha ~ U(1, 1.2) -- a stress case whose residual
    stack amplifies input perturbations by a few hundred (fp32 parity only)."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    tensors = {}
    shapes = codec_param_shapes(width_div)
    if init == "reference":
        for name, shape in sorted(shapes.items()):
            if name.endswith(".alpha"):
                t = torch.ones(shape)
            else:
                wname = name[:-len(".bias")] + ".weight" if name.endswith(".bias") else name
                ws = shapes[wname]
                fan_in = ws[1] * ws[2]  # dim 1 x kernel for both layouts
                bound = 1.0 / math.sqrt(fan_in)
                t = (torch.rand(shape, generator=gen) * 2 - 1) * bound
            tensors[name] = t.to(dtype)
        if weight_norm:
            tensors = weight_norm_split(tensors)
        write_safetensors(path, tensors, {"config_json": json.dumps({})})
        return
    for name, shape in sorted(shapes.items()):
        if name.endswith(".alpha"):
            t = 1.0 + 0.2 * torch.rand(shape, generator=gen)
        elif name.endswith(".bias"):
            t = 0.01 * torch.randn(shape, generator=gen)
        else:
            v = torch.randn(shape, generator=gen)
            g = 0.5 + torch.rand((shape[0], 1, 1), generator=gen)
            norm = v.flatten(1).norm(dim=1).reshape(-1, 1, 1)
            t = g * v / norm
        tensors[name] = t.to(dtype)
    if weight_norm:
        tensors = weight_norm_split(tensors)
    write_safetensors(path, tensors, {"config_json": json.dumps({})})


# ---------------------------------------------------------------------------
# Synthetic requests for the BASELINE configs
# ---------------------------------------------------------------------------

def make_request(cfg: dict, batch: int, text_len: int, ref_frames: Optional[int], seq_len: int,
                 seed: int, text_mask_tail: float = 0.0) -> dict:
    """Seeded request tensors (CPU): text ids uniform over the vocabulary,
    all-true masks (optionally the last fraction of text positions masked),
    speaker latent ~ N(0,1), initial noise ~ N(0,1)."""
    c = dict(DEFAULT_CONFIG)
    c.update(cfg)
    g = torch.Generator()
    g.manual_seed(seed)
    P = c["latent_dim"] * c["latent_patch_size"]
    ids = torch.randint(0, c["text_vocab_size"], (batch, text_len), generator=g, dtype=torch.int64)
    tmask = torch.ones(batch, text_len, dtype=torch.bool)
    if text_mask_tail > 0:
        keep = int(math.floor(text_len * (1.0 - text_mask_tail)))
        tmask[:, keep:] = False
    req = dict(text_ids=ids.to(torch.int32), text_mask=tmask, sequence_length=seq_len)
    if ref_frames is not None:
        req["ref_latent"] = torch.randn(batch, ref_frames, P, generator=g)
        req["ref_mask"] = torch.ones(batch, ref_frames, dtype=torch.bool)
    req["initial_noise"] = torch.randn(batch, seq_len, P, generator=g)
    return req


def throughput_utterances(n: int = 64, seed: int = 4, frame_rate: float = 25.0):
    """Config 4: text lengths U{16..256}, durations U[2,30] s, speaker refs
    U[5,15] s.  Returns a list of (text_len, seq_len, ref_frames, duration_s)."""
    g = torch.Generator()
    g.manual_seed(seed)
    out = []
    for _ in range(n):
        tl = int(torch.randint(16, 257, (1,), generator=g))
        dur = 2.0 + 28.0 * float(torch.rand(1, generator=g))
        spk = 5.0 + 10.0 * float(torch.rand(1, generator=g))
        S = max(1, int(round(frame_rate * dur)))
        out.append((tl, S, int(round(frame_rate * spk)), S / frame_rate))
    return out
