"""GPU parity of the conditioning and checkpoint variants the default
configurations do not exercise, each against the CPU oracle:

  * caption conditioning instead of a speaker reference (the reference's
    tiny_caption_config, src/config/model.rs:316-331, and a tensor-core-sized
    variant): the caption encoder (src/model/dit/aux_conditioner.rs:60-107),
    caption CFG in every guidance mode (src/rf/euler_sampler.rs:186-195), and
    a batch in which one utterance's caption is fully masked;
  * speaker patching with speaker_patch_size = 2
    (src/model/speaker_encoder.rs:24-57): an odd reference length (the last
    frame is dropped) and a masked frame that masks its whole patch;
  * an F16 checkpoint (src/weights/tensor_entry.rs:22-90): the f32 engine
    decodes it exactly, the bf16 engine rounds it to bf16.

Tolerances as everywhere: f32 within 1e-4 relative L2, bf16 within 1e-2.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 1e-2


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return 0


def caption_cfg(synth, small):
    if small:
        c = dict(synth.SMALL_CONFIG)
        c.update(caption_vocab_size=300, caption_dim=256, caption_layers=2, caption_heads=2, caption_mlp_ratio=2.6)
    else:  # tiny_caption_config (src/config/model.rs:316-331)
        c = dict(synth.TINY_CONFIG)
        c.update(caption_vocab_size=32, caption_dim=16, caption_layers=1, caption_heads=2, caption_mlp_ratio=2.0)
    c.update(use_caption_condition=True, speaker_dim=None, speaker_layers=None, speaker_heads=None,
             speaker_patch_size=None)
    return c


def caption_request(cfg, B, T, C, S, seed, masked_caption_row=None):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg["text_vocab_size"], (B, T), generator=g, dtype=torch.int64).to(torch.int32)
    tm = torch.ones(B, T, dtype=torch.bool)
    tm[:, T - 2:] = False
    cids = torch.randint(0, cfg["caption_vocab_size"], (B, C), generator=g, dtype=torch.int64).to(torch.int32)
    cm = torch.ones(B, C, dtype=torch.bool)
    cm[0, C - 3:] = False
    if masked_caption_row is not None:
        cm[masked_caption_row] = False
    noise = torch.randn(B, S, cfg["latent_dim"] * cfg["latent_patch_size"], generator=g)
    return dict(text_ids=ids, text_mask=tm, caption_ids=cids, caption_mask=cm, initial_noise=noise)


def run_both(pkg, oracle, ckpt, precision, r, S, method, mode, steps, sc=3.0, st=3.0, ss=3.0, min_t=0.5):
    W = oracle.Weights.load(str(ckpt))
    oreq = oracle.SamplingRequest(sequence_length=S, **r)
    og = oracle.GuidanceConfig(mode=mode, scale_text=st, scale_caption=sc, scale_speaker=ss, min_t=min_t)
    rec = []
    with torch.no_grad():
        ref = oracle.sample_euler_rf_cfg(W, oreq, oracle.SamplerParams(num_steps=steps, method=method, guidance=og),
                                         record_forwards=rec).numpy()
    eg = pkg.GuidanceConfig(mode=mode, scale_text=st, scale_caption=sc, scale_speaker=ss, min_t=min_t)
    eng = (pkg.InferenceBuilder(0).load_weights(str(ckpt), precision=precision)
           .with_sampling(pkg.SamplerParams(num_steps=steps, method=method, guidance=eg)).build())
    out = eng.sample(pkg.SamplingRequest(sequence_length=S, **r))
    assert np.isfinite(out).all()
    return out, ref, eng, rec


# ---------------------------------------------------------------------------
# caption conditioning
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("method,mode", [("euler", "independent"), ("euler", "joint"), ("heun", "alternating"),
                                         ("plms4", "independent")])
def test_caption_tiny_f32(gpu, pkg, oracle, synth, ckpt_dir, method, mode):
    cfg = caption_cfg(synth, small=False)
    p = ckpt_dir / "tiny_caption.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=12, init="full")
    r = caption_request(cfg, 2, 10, 7, 13, seed=3)
    out, ref, eng, rec = run_both(pkg, oracle, p, "f32", r, 13, method, mode, steps=4)
    err = rel_l2(out, ref)
    print(f"caption tiny f32 {method}/{mode}: rel-L2 {err:.2e}")
    assert err < F32_TOL, err
    # the caption CFG branch is really taken: as many row-forwards as the oracle's
    assert eng.last_stats()[0] == sum(rec)


def test_caption_fully_masked_row_f32(gpu, pkg, oracle, synth, ckpt_dir):
    """One utterance of the batch has no valid caption token: its caption
    state is all masked, the other utterance still drives caption CFG."""
    cfg = caption_cfg(synth, small=False)
    p = ckpt_dir / "tiny_caption.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=12, init="full")
    r = caption_request(cfg, 2, 10, 7, 13, seed=4, masked_caption_row=1)
    out, ref, _, _ = run_both(pkg, oracle, p, "f32", r, 13, "euler", "independent", steps=4, sc=4.0)
    assert rel_l2(out, ref) < F32_TOL


@pytest.mark.parametrize("precision,tol", [("f32", F32_TOL), ("bf16", BF16_TOL)])
def test_caption_small_tensor_core(gpu, pkg, oracle, synth, ckpt_dir, precision, tol):
    """Caption encoder at width 256 (the tcgen05 GEMM and attention paths in
    bf16 mode), 150 latent frames, joint CFG over text + caption."""
    cfg = caption_cfg(synth, small=True)
    p = ckpt_dir / "small_caption.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=13, init="full")
    r = caption_request(cfg, 2, 40, 64, 150, seed=5)
    out, ref, _, _ = run_both(pkg, oracle, p, precision, r, 150, "euler", "joint", steps=3)
    err = rel_l2(out, ref)
    print(f"caption small {precision}: rel-L2 {err:.2e}")
    assert err < tol, err


def test_caption_checkpoint_rejects_speaker_input(gpu, pkg, synth, ckpt_dir):
    cfg = caption_cfg(synth, small=False)
    p = ckpt_dir / "tiny_caption.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=12, init="full")
    r = synth.make_request(synth.TINY_CONFIG, 1, 6, 5, 9, seed=1)
    eng = pkg.InferenceBuilder(0).load_weights(str(p), precision="f32").with_default_sampling().build()
    with pytest.raises(pkg.ConfigError, match="caption conditioner received speaker input"):
        eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=9,
                                       ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                       initial_noise=r["initial_noise"]))


# ---------------------------------------------------------------------------
# speaker patching
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("precision,tol,S", [("f32", F32_TOL, 40), ("bf16", BF16_TOL, 150)])
def test_speaker_patch_size_2(gpu, pkg, oracle, synth, ckpt_dir, precision, tol, S):
    cfg = dict(synth.SMALL_CONFIG, speaker_patch_size=2)
    p = ckpt_dir / "small_patch2.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=14, init="full")
    r = synth.make_request(cfg, 2, 30, 81, S, seed=6)  # 81 frames: the last one is dropped
    r["ref_mask"][0, 10] = False  # masks patch 5 of utterance 0
    r["ref_mask"][1, 60:] = False
    out, ref, _, _ = run_both(pkg, oracle, p, precision, {k: r[k] for k in ("text_ids", "text_mask", "ref_latent",
                                                                          "ref_mask", "initial_noise")},
                              S, "euler", "independent", steps=3, ss=5.0)
    err = rel_l2(out, ref)
    print(f"speaker patch 2 {precision}: rel-L2 {err:.2e}")
    assert err < tol, err


def test_speaker_patch_too_short_is_rejected(gpu, pkg, synth, ckpt_dir):
    cfg = dict(synth.SMALL_CONFIG, speaker_patch_size=2)
    p = ckpt_dir / "small_patch2.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=14, init="full")
    r = synth.make_request(cfg, 1, 8, 1, 9, seed=2)
    eng = pkg.InferenceBuilder(0).load_weights(str(p), precision="f32").with_default_sampling().build()
    with pytest.raises(pkg.IrodoriError, match="Sequence too short for speaker_patch_size=2: seq_len=1"):
        eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=9,
                                       ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                       initial_noise=r["initial_noise"]))


# ---------------------------------------------------------------------------
# F16 checkpoint
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("precision,tol,S", [("f32", F32_TOL, 40), ("bf16", BF16_TOL, 150)])
def test_f16_checkpoint(gpu, pkg, oracle, synth, ckpt_dir, precision, tol, S):
    cfg = synth.SMALL_CONFIG
    p = ckpt_dir / "small_f16.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), cfg, seed=15, init="full", dtype=torch.float16)
    r = synth.make_request(cfg, 2, 24, 50, S, seed=7)
    out, ref, _, _ = run_both(pkg, oracle, p, precision, {k: r[k] for k in ("text_ids", "text_mask", "ref_latent",
                                                                          "ref_mask", "initial_noise")},
                              S, "euler", "joint", steps=3)
    err = rel_l2(out, ref)
    print(f"F16 checkpoint, {precision} engine: rel-L2 {err:.2e}")
    assert err < tol, err
