"""Parity of the CUDA engine against the CPU oracle at the reference's DEFAULT
ModelConfig (src/config/model.rs:46-82: D = 2048, 16 heads, 24 layers,
F = 5888, text/speaker encoders 1280 x 14 layers x 10 heads, vocab 102,400),
the model `bench.py` times, on the BASELINE configurations:

  * config 1 (f32): batch 1, text 64, speaker 150 frames, 250 target frames,
    4 Euler steps, independent CFG text 3 / speaker 3 -- final latents within
    1e-4 relative L2, and every layer of the first forward within 1e-4 (the
    reference's own validate flow compares text_state, speaker_state, in_proj,
    every block and v_pred: src/bin/validate.rs:36,121-126);
  * config 2 (bf16): one JointAttention + SwiGLU block at the default dims,
    the CFG pair of one utterance, 750 latent queries over 128 text (last 13
    masked) + 375 speaker (+ the mean token) + 750 latent keys -- block output
    within 1e-2;
  * config 3 (bf16): 30 s utterance (750 frames), text 200, speaker 375,
    joint CFG 3.0, 2 of the 40 steps' schedule shortened to num_steps = 2 --
    final latents within 1e-2;
  * config 4 (bf16): four utterances of unequal text, speaker and target
    lengths sampled as ONE ragged batch, each compared with its own
    single-utterance oracle run -- within 1e-2;
  * the reference's e2e_compare scenario (scripts/e2e_compare.py:115-119,
    src/bin/e2e_compare.rs:117-122): 4-step Euler and 2-step Heun, CFG text 3 /
    speaker 5, min_t = 0 -- f32 within 1e-4.

The checkpoint is stored in BF16 (the dtype the reference's checkpoints ship
in, src/weights/tensor_entry.rs:22-90): the oracle decodes it to f32 exactly,
the f32 engine likewise, the bf16 engine uses it as is.  Weights use the
"full" init (every parameter, adaLN gates included, non-zero) so every block
contributes; the reference's zero-init gates would make the blocks no-ops.
"""

import ctypes

import numpy as np
import pytest
import torch

from test_gpu_kernels import hooks

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 1e-2


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def default_ckpt(ckpt_dir, synth):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    p = ckpt_dir / "default_bf16.safetensors"
    if not p.exists():
        synth.make_dit_checkpoint(str(p), {}, seed=0, init="full", dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
    return p


@pytest.fixture(scope="module")
def default_w(oracle, default_ckpt):
    return oracle.Weights.load(str(default_ckpt))


def engine(pkg, ckpt, precision, params):
    return pkg.InferenceBuilder(0).load_weights(str(ckpt), precision=precision).with_sampling(params).build()


def eparams(pkg, steps, method="euler", mode="independent", st=3.0, ss=3.0, min_t=0.5):
    return pkg.SamplerParams(num_steps=steps, method=method,
                             guidance=pkg.GuidanceConfig(mode=mode, scale_text=st, scale_speaker=ss, min_t=min_t))


def oparams(oracle, steps, method="euler", mode="independent", st=3.0, ss=3.0, min_t=0.5):
    return oracle.SamplerParams(num_steps=steps, method=method,
                                guidance=oracle.GuidanceConfig(mode=mode, scale_text=st, scale_speaker=ss,
                                                               min_t=min_t))


def oracle_req(oracle, r, S):
    return oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                                  ref_latent=r.get("ref_latent"), ref_mask=r.get("ref_mask"),
                                  initial_noise=r["initial_noise"])


def engine_req(pkg, r, S, **kw):
    return pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                               ref_latent=r.get("ref_latent"), ref_mask=r.get("ref_mask"),
                               initial_noise=r["initial_noise"], **kw)


def engine_layers(pkg, ckpt, precision, r, S, params, D, nlayers, groups):
    """[L + 1, rows, D]: the f32 residual stream of the engine's first DiT
    forward after in_proj and after every block (test hook), rows packed
    (CFG group, utterance, frame)."""
    L = hooks()
    L.irtt_sample_dump_layers.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int)]
    keep = []

    def arr(x, dt):
        a = np.ascontiguousarray(x.numpy() if torch.is_tensor(x) else x, dtype=dt)
        keep.append(a)
        return a

    ids, tm = arr(r["text_ids"], np.int32), arr(r["text_mask"], np.uint8)
    ref, rm = arr(r["ref_latent"], np.float32), arr(r["ref_mask"], np.uint8)
    noise = arr(r["initial_noise"], np.float32)
    B = ids.shape[0]
    q = pkg._Request()
    q.batch, q.text_len, q.text_ids, q.text_mask = B, ids.shape[1], ids.ctypes.data, tm.ctypes.data
    q.ref_len, q.ref_dim, q.ref_latent, q.ref_mask = ref.shape[1], ref.shape[2], ref.ctypes.data, rm.ctypes.data
    q.sequence_length = S
    q.initial_noise = noise.ctypes.data
    q.memory = pkg.MEM_HOST
    cp = params._to_c()
    cap = groups * B * S
    dump = torch.full(((nlayers + 1) * cap * D,), float("nan"), device="cuda")
    out = np.empty(noise.shape, dtype=np.float32)
    rows = ctypes.c_int(0)
    rc = L.irtt_sample_dump_layers(str(ckpt).encode(), 0 if precision == "bf16" else 1, ctypes.byref(cp),
                                   ctypes.byref(q), out.ctypes.data, dump.data_ptr(), cap, ctypes.byref(rows))
    assert rc == 0, L.irtt_last_error().decode()
    assert rows.value == cap
    return dump.view(nlayers + 1, cap, D).cpu().numpy(), out


def oracle_layers(oracle, W, r, S, mode, steps):
    """The oracle's first forward with capture (forward_with_cond_debug,
    src/model/dit/model.rs:269-346) on the same packed batch as the engine:
    independent CFG = [cond, text-uncond, speaker-uncond], joint CFG =
    [cond, uncond] (src/rf/euler_sampler.rs:397-451)."""
    req = oracle_req(oracle, r, S)
    cond = oracle.encode_conditions(W, req)
    unc = cond.zeros_like()
    if mode == "independent":
        text_unc = oracle.Cond(unc.text_state, unc.text_mask, cond.aux_kind, cond.aux_state, cond.aux_mask)
        spk_unc = oracle.Cond(cond.text_state, cond.text_mask, unc.aux_kind, unc.aux_state, unc.aux_mask)
        conds = [cond, text_unc, spk_unc]
    else:
        conds = [cond, unc]
    batch = oracle.cat_batch(conds)
    kv = oracle.build_kv_caches(W, batch)
    cos, sin = oracle.rope_tables(W.cfg.head_dim(), S, dtype=W.dtype)
    t0 = oracle.t_schedule(steps)[0]
    x = torch.cat([r["initial_noise"]] * len(conds), 0)
    with torch.no_grad():
        _, after_in, outs = oracle.dit_forward(W, x, torch.full((x.shape[0],), t0, dtype=torch.float32), kv, cos, sin,
                                               capture=True)
    return np.stack([after_in.reshape(-1, after_in.shape[-1]).numpy()] +
                    [o.reshape(-1, o.shape[-1]).numpy() for o in outs])


def per_layer_errors(got, ref):
    assert got.shape == ref.shape
    errs = []
    for layer in range(ref.shape[0]):
        a = got[layer].astype(np.float64)
        assert np.isfinite(a).all(), f"layer {layer}: non-finite engine output"
        errs.append(rel_l2(a, ref[layer]))
    return errs


# ---------------------------------------------------------------------------
# config 1
# ---------------------------------------------------------------------------

C1 = dict(B=1, T=64, R=150, S=250, steps=4)


@pytest.fixture(scope="module")
def config1(oracle, synth, default_w):
    r = synth.make_request({}, C1["B"], C1["T"], C1["R"], C1["S"], seed=1)
    with torch.no_grad():
        ref = oracle.sample_euler_rf_cfg(default_w, oracle_req(oracle, r, C1["S"]), oparams(oracle, C1["steps"]))
    return r, ref.numpy()


@pytest.mark.parametrize("precision,tol", [("f32", F32_TOL), ("bf16", BF16_TOL)])
def test_config1_final_latents(pkg, default_ckpt, config1, precision, tol):
    r, ref = config1
    eng = engine(pkg, default_ckpt, precision, eparams(pkg, C1["steps"]))
    out = eng.sample(engine_req(pkg, r, C1["S"]))
    assert np.isfinite(out).all()
    err = rel_l2(out, ref)
    print(f"config 1 {precision}: final latents rel-L2 {err:.3e} (tol {tol})")
    assert err < tol, err


@pytest.mark.parametrize("precision,tol", [("f32", F32_TOL), ("bf16", BF16_TOL)])
def test_config1_per_layer(pkg, oracle, synth, default_ckpt, default_w, config1, precision, tol):
    r, ref_final = config1
    cfg = default_w.cfg
    got, out = engine_layers(pkg, default_ckpt, precision, r, C1["S"], eparams(pkg, C1["steps"]), cfg.model_dim,
                             cfg.num_layers, groups=3)
    ref = oracle_layers(oracle, default_w, r, C1["S"], "independent", C1["steps"])
    errs = per_layer_errors(got, ref)
    print(f"config 1 {precision} per-layer rel-L2 (in_proj, blocks 1..{len(errs) - 1}): max {max(errs):.2e}; "
          + " ".join(f"{e:.1e}" for e in errs))
    assert max(errs) < tol, errs
    assert rel_l2(out, ref_final) < tol


# ---------------------------------------------------------------------------
# config 2: one block at the default dims
# ---------------------------------------------------------------------------

def test_config2_block_bf16(pkg, oracle, synth, ckpt_dir):
    """One JointAttention + SwiGLU block (D = 2048, 16 heads, F = 5888), bf16
    operands with f32 accumulation, on the CFG pair (cond + uncond, the joint
    CFG batch) of one utterance: 750 latent queries; keys = 128 text (the last
    10 % = 13 masked) + 375 speaker frames (+ the masked-mean token) + 750
    latent; seed 2.  The encoders keep the default width (1280, 10 heads)
    with 2 layers each: they only feed the context keys."""
    cfg = dict(num_layers=1, text_layers=2, speaker_layers=2)
    p = ckpt_dir / "block_default_bf16.safetensors"
    synth.make_dit_checkpoint(str(p), cfg, seed=2, init="full", dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    W = oracle.Weights.load(str(p))
    r = synth.make_request(cfg, 1, 128, 375, 750, seed=2, text_mask_tail=0.1)
    assert int(r["text_mask"].sum()) == 115
    params = eparams(pkg, 2, mode="joint", st=3.0, ss=3.0)
    got, _ = engine_layers(pkg, p, "bf16", r, 750, params, 2048, 1, groups=2)
    ref = oracle_layers(oracle, W, r, 750, "joint", 2)
    errs = per_layer_errors(got, ref)
    # the block's own contribution (output minus input) must match too, not
    # just the residual sum dominated by the in_proj rows
    blk = rel_l2(got[1] - got[0], ref[1] - ref[0])
    print(f"config 2 bf16: in_proj {errs[0]:.2e}, block output {errs[1]:.2e}, block delta {blk:.2e}")
    assert max(errs) < BF16_TOL and blk < BF16_TOL, (errs, blk)


# ---------------------------------------------------------------------------
# config 3: single 30 s utterance, joint CFG, bf16
# ---------------------------------------------------------------------------

def test_config3_two_steps_bf16(pkg, oracle, synth, default_ckpt, default_w):
    r = synth.make_request({}, 1, 200, 375, 750, seed=3)
    with torch.no_grad():
        ref = oracle.sample_euler_rf_cfg(default_w, oracle_req(oracle, r, 750),
                                         oparams(oracle, 2, mode="joint")).numpy()
    eng = engine(pkg, default_ckpt, "bf16", eparams(pkg, 2, mode="joint"))
    out = eng.sample(engine_req(pkg, r, 750))
    assert np.isfinite(out).all()
    err = rel_l2(out, ref)
    print(f"config 3 bf16 (2 steps joint CFG): final latents rel-L2 {err:.3e}")
    assert err < BF16_TOL, err
    assert eng.last_stats()[0] == 3  # step 0 in the CFG window (cond + uncond), step 1 outside


# ---------------------------------------------------------------------------
# config 4: ragged batch, each utterance against its own oracle run
# ---------------------------------------------------------------------------

def test_config4_ragged_bf16(pkg, oracle, synth, default_ckpt, default_w):
    """Text lengths 24 / 90 / 160 / 256, speaker references 125 / 200 / 250 /
    375 frames (5-15 s), targets 48 / 110 / 181 / 262 frames, sampled as one
    padded batch with per-utterance lengths (2 steps, joint CFG 3.0)."""
    shapes = [(24, 125, 48), (90, 200, 110), (160, 250, 181), (256, 375, 262)]
    singles = [synth.make_request({}, 1, T, R, S, seed=40 + i) for i, (T, R, S) in enumerate(shapes)]
    Tm, Rm, Sm = (max(s[j] for s in shapes) for j in range(3))
    P = default_w.cfg.patched_latent_dim()
    B = len(shapes)
    ids = torch.zeros(B, Tm, dtype=torch.int32)
    tm = torch.zeros(B, Tm, dtype=torch.bool)
    ref = torch.zeros(B, Rm, P)
    rm = torch.zeros(B, Rm, dtype=torch.bool)
    noise = torch.zeros(B, Sm, P)
    for b, ((T, R, S), r) in enumerate(zip(shapes, singles)):
        ids[b, :T], tm[b, :T] = r["text_ids"][0], True
        ref[b, :R], rm[b, :R] = r["ref_latent"][0], True
        noise[b, :S] = r["initial_noise"][0]
    eng = engine(pkg, default_ckpt, "bf16", eparams(pkg, 2, mode="joint"))
    out = eng.sample(pkg.SamplingRequest(text_ids=ids, text_mask=tm, sequence_length=Sm, ref_latent=ref, ref_mask=rm,
                                         initial_noise=noise, sequence_lengths=[s[2] for s in shapes]))
    assert np.isfinite(out).all()
    errs = []
    for b, ((T, R, S), r) in enumerate(zip(shapes, singles)):
        with torch.no_grad():
            o = oracle.sample_euler_rf_cfg(default_w, oracle_req(oracle, r, S), oparams(oracle, 2, mode="joint"))
        errs.append(rel_l2(out[b, :S], o[0].numpy()))
        assert np.all(out[b, S:] == 0)
    print("config 4 bf16 ragged, per-utterance rel-L2: " + " ".join(f"{e:.2e}" for e in errs))
    assert max(errs) < BF16_TOL, errs


# ---------------------------------------------------------------------------
# the reference's e2e_compare scenario
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("method,steps", [("euler", 4), ("heun", 2)])
def test_e2e_compare_scenario_f32(pkg, oracle, synth, default_ckpt, default_w, method, steps):
    """scripts/e2e_compare.py:115-119 / src/bin/e2e_compare.rs:117-122:
    independent CFG, text 3.0 / speaker 5.0, min_t = 0 (every step guided);
    batch 1, text 48, speaker 100 frames, 120 target frames."""
    r = synth.make_request({}, 1, 48, 100, 120, seed=11)
    with torch.no_grad():
        ref = oracle.sample_euler_rf_cfg(default_w, oracle_req(oracle, r, 120),
                                         oparams(oracle, steps, method=method, ss=5.0, min_t=0.0)).numpy()
    eng = engine(pkg, default_ckpt, "f32", eparams(pkg, steps, method=method, ss=5.0, min_t=0.0))
    out = eng.sample(engine_req(pkg, r, 120))
    err = rel_l2(out, ref)
    print(f"e2e_compare {method} x{steps} f32: rel-L2 {err:.3e}")
    assert err < F32_TOL, err


# ---------------------------------------------------------------------------
# decoded waveform: bf16 sampler + bf16 codec against f32 sampler + f32 codec
# ---------------------------------------------------------------------------

def test_decoded_waveform_snr_40_steps(pkg, synth, ckpt_dir):
    """The bench's model and sampler (default dims with the codec's 32 latent
    channels, the bench's own random init; 40 Euler steps, joint CFG 3.0) on
    two utterances of 100 and 175 frames sampled as one ragged batch, decoded
    to 48 kHz by the DACVAE decoder (reference-default random init).  The f32
    engine tracks the oracle within ~1e-5 at these dims (tests above), so the
    f32 sampler + f32 codec stands in for the reference's output here.
    Reported: final-latent rel-L2 of the bf16 sampler and the SNR of the bf16
    sampler + bf16 codec waveform."""
    p = ckpt_dir / "default_l32_bf16.safetensors"
    synth.make_dit_checkpoint(str(p), {"latent_dim": 32}, seed=4, init="baseline", dtype=torch.bfloat16,
                              device="cuda")
    torch.cuda.synchronize()
    cp = ckpt_dir / "codec_ref_init.safetensors"
    synth.make_codec_checkpoint(str(cp), seed=5, width_div=1, init="reference")
    cfg = dict(synth.DEFAULT_CONFIG, latent_dim=32)
    lens = [100, 175]
    reqs = [synth.make_request(cfg, 1, t, rf, S, seed=60 + i) for i, (t, rf, S) in enumerate([(60, 150, 100),
                                                                                            (120, 250, 175)])]
    Sm = max(lens)
    ids = torch.zeros(2, 120, dtype=torch.int32)
    tm = torch.zeros(2, 120, dtype=torch.bool)
    ref = torch.zeros(2, 250, 32)
    rm = torch.zeros(2, 250, dtype=torch.bool)
    noise = torch.zeros(2, Sm, 32)
    for b, r in enumerate(reqs):
        T, R, S = r["text_ids"].shape[1], r["ref_latent"].shape[1], lens[b]
        ids[b, :T], tm[b, :T] = r["text_ids"][0], True
        ref[b, :R], rm[b, :R] = r["ref_latent"][0], True
        noise[b, :S] = r["initial_noise"][0]
    rq = pkg.SamplingRequest(text_ids=ids, text_mask=tm, sequence_length=Sm, ref_latent=ref, ref_mask=rm,
                             initial_noise=noise, sequence_lengths=lens)
    params = eparams(pkg, 40, mode="joint")
    lat = {}
    for prec in ("f32", "bf16"):
        eng = engine(pkg, p, prec, params)
        lat[prec] = eng.sample(rq)
        del eng
    wav = {}
    for prec in ("f32", "bf16"):
        codec = pkg.load_codec(str(cp), device=0, precision=prec)
        wav[prec] = codec.decode(lat[prec], lengths=lens)
        del codec
    hop = 1920
    errs, snrs = [], []
    for b, S in enumerate(lens):
        errs.append(rel_l2(lat["bf16"][b, :S], lat["f32"][b, :S]))
        a, w = wav["f32"][b, 0, :S * hop].astype(np.float64), wav["bf16"][b, 0, :S * hop].astype(np.float64)
        assert np.isfinite(w).all()
        snrs.append(10 * np.log10(np.sum(a * a) / max(np.sum((w - a) ** 2), 1e-30)))
    print("40-step bf16 vs f32 sampler: latent rel-L2 " + " ".join(f"{e:.2e}" for e in errs) +
          "; decoded waveform SNR " + " ".join(f"{s:.1f} dB" for s in snrs))
    assert max(errs) < BF16_TOL, errs
    assert min(snrs) > 20.0, snrs
