"""End-to-end parity of the CUDA engine (through the C ABI) against the CPU
oracle on the same seeded checkpoints and inputs.

Tolerances (north star):
  * f32 mode: final latents within 1e-4 relative L2 (and per-sampler-mode).
  * bf16 mode: final latents within 1e-2 relative L2.
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


@pytest.fixture(scope="module")
def tiny_ckpt(ckpt_dir, synth):
    p = ckpt_dir / "tiny.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    return p


@pytest.fixture(scope="module")
def small_ckpt(ckpt_dir, synth):
    p = ckpt_dir / "small.safetensors"
    synth.make_dit_checkpoint(str(p), synth.SMALL_CONFIG, seed=3, init="full")
    return p


def oracle_params(oracle, method, mode, steps, **kw):
    g = oracle.GuidanceConfig(mode=mode, scale_text=kw.get("st", 3.0), scale_speaker=kw.get("ss", 5.0),
                              min_t=kw.get("min_t", 0.5))
    return oracle.SamplerParams(num_steps=steps, method=method, guidance=g,
                                truncation_factor=kw.get("trunc"),
                                temporal_rescale=kw.get("tr"),
                                speaker_kv=kw.get("skv"))


def engine_params(pkg, method, mode, steps, **kw):
    g = pkg.GuidanceConfig(mode=mode, scale_text=kw.get("st", 3.0), scale_speaker=kw.get("ss", 5.0),
                           min_t=kw.get("min_t", 0.5))
    tr = kw.get("tr")
    skv = kw.get("skv")
    return pkg.SamplerParams(num_steps=steps, method=method, guidance=g, truncation_factor=kw.get("trunc"),
                             temporal_rescale=pkg.TemporalRescaleConfig(*tr) if tr else None,
                             speaker_kv=pkg.SpeakerKvConfig(skv.scale, skv.max_layers, skv.min_t) if skv else None)


def run_pair(pkg, oracle, synth, ckpt, cfg, precision, method, mode, steps=4, B=1, T=12, R=9, S=17, seed=1, **kw):
    r = synth.make_request(cfg, B, T, R, S, seed=seed, text_mask_tail=kw.pop("tail", 0.0))
    W = oracle.Weights.load(str(ckpt))
    req = oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                                 ref_latent=r.get("ref_latent"), ref_mask=r.get("ref_mask"),
                                 initial_noise=r["initial_noise"])
    ref = oracle.sample_euler_rf_cfg(W, req, oracle_params(oracle, method, mode, steps, **kw)).numpy()
    eng = (pkg.InferenceBuilder(0).load_weights(str(ckpt), precision=precision)
           .with_sampling(engine_params(pkg, method, mode, steps, **kw)).build())
    out = eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                                         ref_latent=r.get("ref_latent"), ref_mask=r.get("ref_mask"),
                                         initial_noise=r["initial_noise"]))
    return out, ref, eng


CASES = [("euler", "independent"), ("euler", "joint"), ("euler", "alternating"),
         ("heun", "independent"), ("heun", "joint"), ("heun", "alternating"),
         ("plms4", "independent"), ("plms4", "joint")]


@pytest.mark.parametrize("method,mode", CASES)
def test_f32_tiny_all_modes(gpu, pkg, oracle, synth, tiny_ckpt, method, mode):
    kw = {"ss": 3.0} if mode == "joint" else {}
    out, ref, _ = run_pair(pkg, oracle, synth, tiny_ckpt, synth.TINY_CONFIG, "f32", method, mode, **kw)
    assert np.isfinite(out).all()
    assert rel_l2(out, ref) < F32_TOL, rel_l2(out, ref)


@pytest.mark.parametrize("method,mode", [("euler", "independent"), ("euler", "joint"), ("heun", "alternating")])
def test_f32_small(gpu, pkg, oracle, synth, small_ckpt, method, mode):
    kw = {"ss": 3.0} if mode == "joint" else {}
    out, ref, _ = run_pair(pkg, oracle, synth, small_ckpt, synth.SMALL_CONFIG, "f32", method, mode, B=2, T=20, R=30,
                           S=40, tail=0.1, **kw)
    assert rel_l2(out, ref) < F32_TOL, rel_l2(out, ref)


def test_f32_sampler_options(gpu, pkg, oracle, synth, small_ckpt):
    """Truncation, temporal score rescale and force-speaker KV scaling with a
    min_t revert (src/rf/euler_sampler.rs:153-155, :529-547)."""
    skv = pkg.SpeakerKvConfig(1.5, 1, 0.6)
    out, ref, _ = run_pair(pkg, oracle, synth, small_ckpt, synth.SMALL_CONFIG, "f32", "euler", "independent",
                           steps=6, trunc=0.9, tr=(2.0, 0.5), skv=skv, min_t=0.3)
    assert rel_l2(out, ref) < F32_TOL, rel_l2(out, ref)


@pytest.mark.parametrize("method,mode", [("euler", "joint"), ("euler", "independent"), ("heun", "alternating")])
def test_bf16_small_tensor_core_path(gpu, pkg, oracle, synth, small_ckpt, method, mode):
    """S = 150 latent frames so the DiT GEMMs take the tcgen05 path (M >= 128)."""
    kw = {"ss": 3.0} if mode == "joint" else {}
    out, ref, eng = run_pair(pkg, oracle, synth, small_ckpt, synth.SMALL_CONFIG, "bf16", method, mode, steps=4,
                             B=2, T=64, R=140, S=150, tail=0.1, **kw)
    assert np.isfinite(out).all()
    err = rel_l2(out, ref)
    assert err < BF16_TOL, err
    rows, launches = eng.last_stats()
    assert rows > 0 and launches > 0


def test_ragged_batch_matches_single_utterances(gpu, pkg, synth, small_ckpt):
    """A padded batch with per-utterance lengths equals running each utterance
    alone (the reference sampler has no ragged path, so batch-1 runs are the
    oracle for it)."""
    cfg = synth.SMALL_CONFIG
    eng = (pkg.InferenceBuilder(0).load_weights(str(small_ckpt), precision="f32")
           .with_sampling(pkg.SamplerParams(num_steps=3, guidance=pkg.GuidanceConfig(mode="joint", scale_speaker=3.0)))
           .build())
    lens = [31, 17, 40]
    S = max(lens)
    reqs = [synth.make_request(cfg, 1, 16, 12, S, seed=10 + i) for i in range(3)]
    singles = []
    for L, r in zip(lens, reqs):
        o = eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=L,
                                           ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                           initial_noise=r["initial_noise"][:, :L]))
        singles.append(o[0])
    cat = lambda k: torch.cat([r[k] for r in reqs], 0)
    out = eng.sample(pkg.SamplingRequest(text_ids=cat("text_ids"), text_mask=cat("text_mask"), sequence_length=S,
                                         ref_latent=cat("ref_latent"), ref_mask=cat("ref_mask"),
                                         initial_noise=cat("initial_noise"), sequence_lengths=lens))
    for b, L in enumerate(lens):
        assert rel_l2(out[b, :L], singles[b]) < 1e-5
        assert np.all(out[b, L:] == 0)


def test_device_buffers_and_errors(gpu, pkg, synth, tiny_ckpt, tmp_path):
    cfg = synth.TINY_CONFIG
    eng = pkg.InferenceBuilder(0).load_weights(str(tiny_ckpt), precision="f32").with_default_sampling().build()
    r = synth.make_request(cfg, 1, 8, 5, 9, seed=2)
    host = eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=9,
                                          ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                          initial_noise=r["initial_noise"]))
    d = {k: v.cuda() for k, v in r.items() if torch.is_tensor(v)}
    out = torch.empty(1, 9, cfg["latent_dim"], device="cuda")
    eng.sample(pkg.SamplingRequest(text_ids=d["text_ids"], text_mask=d["text_mask"], sequence_length=9,
                                   ref_latent=d["ref_latent"], ref_mask=d["ref_mask"],
                                   initial_noise=d["initial_noise"]), out=out)
    assert rel_l2(out.cpu().numpy(), host) < 1e-6
    # Joint CFG with unequal active scales is rejected (src/rf/euler_sampler.rs:204-224)
    bad = pkg.SamplerParams(guidance=pkg.GuidanceConfig(mode="joint", scale_text=3.0, scale_speaker=5.0))
    eng.with_sampling(bad)
    with pytest.raises(pkg.ConfigError, match="Joint requires all active cfg scales to be equal"):
        eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=9,
                                       ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                       initial_noise=r["initial_noise"]))
    # missing file / missing config metadata
    with pytest.raises(pkg.IrodoriError) as ei:
        pkg.InferenceBuilder(0).load_weights(str(tmp_path / "nope.safetensors"))
    assert ei.value.kind == "Io"
    p = tmp_path / "noconf.safetensors"
    synth.write_safetensors(str(p), {"x": torch.zeros(2)}, {})
    with pytest.raises(pkg.IrodoriError) as ei:
        pkg.InferenceBuilder(0).load_weights(str(p))
    assert ei.value.kind == "NoConfig"


@pytest.mark.parametrize("precision,tol,S", [("f32", F32_TOL, 40), ("bf16", BF16_TOL, 150)])
def test_fully_masked_conditions(gpu, pkg, oracle, synth, small_ckpt, precision, tol, S):
    """A batch in which utterance 0 has every text position masked, utterance
    1 has every speaker-reference frame masked (no speaker key at all, the
    masked-mean token masked too: src/model/dit/aux_conditioner.rs:161-190)
    and utterance 2 is normal; independent CFG over both signals.  The
    engine's compacted context cache holds no key for the masked parts; the
    oracle runs the reference's masked attention."""
    cfg = synth.SMALL_CONFIG
    r = synth.make_request(cfg, 3, 24, 30, S, seed=21)
    r["text_mask"][0] = False
    r["ref_mask"][1] = False
    W = oracle.Weights.load(str(small_ckpt))
    req = oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                                 ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                 initial_noise=r["initial_noise"])
    with torch.no_grad():
        ref = oracle.sample_euler_rf_cfg(W, req, oracle_params(oracle, "euler", "independent", 3)).numpy()
    eng = (pkg.InferenceBuilder(0).load_weights(str(small_ckpt), precision=precision)
           .with_sampling(engine_params(pkg, "euler", "independent", 3)).build())
    out = eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                                         ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                         initial_noise=r["initial_noise"]))
    assert np.isfinite(out).all()
    for b in range(3):
        err = rel_l2(out[b], ref[b])
        assert err < tol, (b, err)


@pytest.mark.parametrize("precision,tol", [("f32", F32_TOL), ("bf16", BF16_TOL)])
def test_single_frame_and_tiny_conditions(gpu, pkg, oracle, synth, small_ckpt, precision, tol):
    """The smallest request: one latent frame, one text token, one speaker
    frame (every GEMM below the tensor-core tile, attention over 1 + 1 + 2
    keys)."""
    out, ref, _ = run_pair(pkg, oracle, synth, small_ckpt, synth.SMALL_CONFIG, precision, "euler", "independent",
                           steps=3, B=1, T=1, R=1, S=1)
    assert np.isfinite(out).all()
    assert rel_l2(out, ref) < tol, rel_l2(out, ref)
