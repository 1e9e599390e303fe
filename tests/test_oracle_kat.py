"""Known-answer tests pinning the CPU oracle to the reference crate's own
in-crate unit-test invariants (the reference ships no golden tensors).
Each test names the reference test it restates."""

import math

import numpy as np
import pytest
import torch


def test_t_schedule_endpoints_monotone_uniform(oracle):
    # src/rf/euler_sampler.rs:732-766
    for n in (1, 4, 10, 40):
        ts = oracle.t_schedule(n)
        assert len(ts) == n + 1
        assert abs(ts[0] - 0.999) < 1e-7 and ts[-1] == 0.0
        assert all(a > b for a, b in zip(ts, ts[1:]))
        d = np.diff(np.array(ts, dtype=np.float64))
        assert np.allclose(d, d[0], atol=1e-6)


def test_cfg_window_counts(oracle):
    # src/rf/euler_sampler.rs:799-825: default window [0.5, 1.0] over 40 steps
    ts = oracle.t_schedule(40)[:-1]
    used = [0.5 <= t <= 1.0 for t in ts]
    assert sum(used) == 20 and all(used[:20]) and not any(used[20:])


def test_ab_coefficients(oracle):
    # src/rf/euler_sampler.rs:1733-1804: AB-k coefficients sum to 1 and match
    ones = [torch.ones(1) * (i + 1) for i in range(4)]
    assert float(oracle.ab_extrapolate(ones[:1])) == 1.0
    assert abs(float(oracle.ab_extrapolate([torch.ones(1)] * 2)) - 1.0) < 1e-7
    assert abs(float(oracle.ab_extrapolate([torch.ones(1)] * 3)) - 1.0) < 1e-6
    assert abs(float(oracle.ab_extrapolate([torch.ones(1)] * 4)) - 1.0) < 1e-6
    # AB-2 on history [2, 1]: 1.5*2 - 0.5*1 = 2.5
    assert abs(float(oracle.ab_extrapolate([torch.tensor([2.0]), torch.tensor([1.0])])) - 2.5) < 1e-7


def test_rope_identity_at_position_zero_and_half_heads(oracle):
    # src/model/rope.rs:182-241
    cos, sin = oracle.rope_tables(8, 5)
    x = torch.randn(1, 5, 4, 8)
    y = oracle.apply_rotary_emb(x, cos, sin)
    assert torch.allclose(y[:, 0], x[:, 0])
    h = oracle.apply_rotary_half(x, cos, sin)
    assert torch.equal(h[:, :, 2:], x[:, :, 2:])
    assert not torch.allclose(h[:, 1:, :2], x[:, 1:, :2])
    # rotation preserves pair norms
    assert torch.allclose(y.reshape(1, 5, 4, 4, 2).norm(dim=-1), x.reshape(1, 5, 4, 4, 2).norm(dim=-1), atol=1e-5)


def test_rope_freq_table_values(oracle):
    cos, sin = oracle.rope_tables(128, 3)
    # position 1, pair 0: angle 1 rad; pair 63: 1 / 10000^(126/128)
    assert abs(float(cos[1, 0]) - math.cos(1.0)) < 1e-6
    assert abs(float(sin[1, 63]) - math.sin(1.0 / 10000 ** (126 / 128))) < 1e-7


def test_timestep_embedding(oracle):
    # src/model/rope.rs:141-165: [cos | sin] with 1000-scaled frequencies
    e = oracle.timestep_embedding(torch.tensor([0.0, 0.5]), 8)
    assert torch.allclose(e[0], torch.tensor([1, 1, 1, 1, 0, 0, 0, 0], dtype=torch.float32))
    f = 1000.0 * math.exp(-math.log(10000.0) * 1 / 4)
    assert abs(float(e[1, 1]) - math.cos(0.5 * f)) < 1e-5


def test_sdpa_all_masked_is_zero(oracle):
    # src/model/attention.rs:813-833 (sdpa_all_masked_gives_zero)
    q = torch.ones(1, 3, 2, 4)
    k = torch.ones(1, 4, 2, 4)
    v = torch.ones(1, 4, 2, 4)
    out = oracle.sdpa(q, k, v, torch.zeros(1, 4, dtype=torch.bool), 0.5)
    assert torch.equal(out, torch.zeros_like(out))


def test_sdpa_masked_nan_values_do_not_leak(oracle):
    q = torch.randn(1, 2, 1, 4)
    k = torch.randn(1, 3, 1, 4)
    v = torch.randn(1, 3, 1, 4)
    v[:, 2] = float("nan")
    m = torch.tensor([[True, True, False]])
    out = oracle.sdpa(q, k, v, m, 0.5)
    ref = oracle.sdpa(q, k[:, :2], v[:, :2], None, 0.5)
    assert torch.isfinite(out).all() and torch.allclose(out, ref)


def test_swiglu_zero_in_zero_out(oracle, synth, tmp_path):
    # src/model/feed_forward.rs:157-165
    p = tmp_path / "t.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    W = oracle.Weights.load(str(p))
    y = oracle.swiglu(W, "blocks.0.mlp", torch.zeros(1, 3, 32))
    assert torch.equal(y, torch.zeros_like(y))


def test_fused_qkv_equals_separate(oracle, synth, tmp_path):
    # src/model/optimized.rs:160-366 (fused vs unfused < 1e-5)
    p = tmp_path / "t.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    W = oracle.Weights.load(str(p))
    h = torch.randn(2, 5, 32)
    fused = torch.cat([W["blocks.0.attention.wq.weight"], W["blocks.0.attention.wk.weight"],
                       W["blocks.0.attention.wv.weight"]], 0)
    a = h @ fused.T
    b = torch.cat([oracle.linear(W, f"blocks.0.attention.{n}", h) for n in ("wq", "wk", "wv")], -1)
    assert (a - b).abs().max() < 1e-5


def test_mean_token(oracle):
    # src/model/dit/aux_conditioner.rs:161-190
    st = torch.arange(12, dtype=torch.float32).reshape(1, 3, 4)
    m = torch.tensor([[True, False, True]])
    s2, m2 = oracle.prepend_masked_mean_token(st, m)
    assert torch.allclose(s2[0, 0], (st[0, 0] + st[0, 2]) / 2)
    assert m2.tolist() == [[True, True, False, True]]
    s3, m3 = oracle.prepend_masked_mean_token(st, torch.zeros(1, 3, dtype=torch.bool))
    assert torch.equal(s3[0, 0], torch.zeros(4)) and m3[0, 0].item() is False


def test_snake_and_pads(oracle):
    # src/codec/layers.rs:114-177
    a = torch.ones(1, 3, 1)
    assert torch.equal(oracle.snake(torch.zeros(1, 3, 4), a), torch.zeros(1, 3, 4))
    x = torch.rand(1, 3, 10) * 5
    assert (oracle.snake(x, a) >= x).all()
    assert oracle.conv_pad(7, 1, 1) == 3 and oracle.conv_pad(7, 1, 9) == 27 and oracle.conv_pad(1, 1, 1) == 0
    assert oracle.conv_transpose_pad(12) == (6, 0) and oracle.conv_transpose_pad(2) == (1, 0)
    assert oracle.conv_transpose_pad(3) == (2, 1)


@pytest.mark.parametrize("bad,msg", [
    (dict(num_steps=0), "num_steps must be > 0"),
    (dict(min_t=1.5), "guidance.min_t must be finite and in [0, 1], got 1.5"),
    (dict(min_t=0.8, max_t=0.6), "guidance.min_t (0.8) must not exceed guidance.max_t (0.6)"),
    (dict(truncation_factor=0.0), "truncation_factor must be finite and > 0"),
    (dict(method="plms4", mode="alternating"), "PLMS4 is not compatible"),
    (dict(max_t=1.5), "guidance.max_t must be finite and in [0, 1], got 1.5"),
    (dict(scale_text=float("nan")), "guidance.scale_text must be finite, got NaN"),
    (dict(min_t=2.0), "guidance.min_t must be finite and in [0, 1], got 2"),
    (dict(scale_speaker=float("inf")), "guidance.scale_speaker must be finite, got inf"),
    (dict(temporal_rescale=(float("nan"), 1.0)), "temporal_rescale.k must be finite"),
    (dict(temporal_rescale=(1.0, 0.0)), "temporal_rescale.sigma must not be zero"),
    (dict(speaker_kv=(0.0, None)), "speaker_kv.scale must be finite and > 0"),
    (dict(speaker_kv=(-1.0, None)), "speaker_kv.scale must be finite and > 0"),
    (dict(speaker_kv=(float("inf"), None)), "speaker_kv.scale must be finite and > 0"),
    (dict(speaker_kv=(1.5, 1.5)), "speaker_kv.min_t must be finite and in [0, 1]"),
])
def test_params_validate_rejections(oracle, bad, msg):
    # src/rf/params.rs:253-378
    g = oracle.GuidanceConfig(mode=bad.get("mode", "independent"), min_t=bad.get("min_t", 0.5),
                              max_t=bad.get("max_t", 1.0), scale_text=bad.get("scale_text", 3.0),
                              scale_speaker=bad.get("scale_speaker", 5.0))
    skv = bad.get("speaker_kv")
    p = oracle.SamplerParams(num_steps=bad.get("num_steps", 40), method=bad.get("method", "euler"), guidance=g,
                             truncation_factor=bad.get("truncation_factor"),
                             temporal_rescale=bad.get("temporal_rescale"),
                             speaker_kv=None if skv is None else oracle.SpeakerKvConfig(scale=skv[0], min_t=skv[1]))
    with pytest.raises(ValueError) as ei:
        p.validate()
    assert msg in str(ei.value)


def test_sampler_forward_counts_and_joint_scale_check(oracle, synth, tmp_path):
    # src/rf/euler_sampler.rs:912-1069: row-forward counts per mode; Joint with unequal scales errors
    p = tmp_path / "t.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    W = oracle.Weights.load(str(p))
    r = synth.make_request(synth.TINY_CONFIG, 1, 6, 5, 7, seed=1)
    req = oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=7,
                                 ref_latent=r["ref_latent"], ref_mask=r["ref_mask"], initial_noise=r["initial_noise"])
    rec = []
    oracle.sample_euler_rf_cfg(W, req, oracle.SamplerParams(num_steps=4), rec)
    assert rec == [3, 3, 1, 1]
    with pytest.raises(ValueError, match="Joint requires"):
        oracle.sample_euler_rf_cfg(W, req, oracle.SamplerParams(num_steps=2, guidance=oracle.GuidanceConfig(
            mode="joint", scale_text=3.0, scale_speaker=5.0)))


def test_cached_equals_uncached_forward(oracle, synth, tmp_path):
    # src/rf/euler_sampler.rs:1071-1117: the context cache is a pure function of the condition
    p = tmp_path / "t.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    W = oracle.Weights.load(str(p))
    r = synth.make_request(synth.TINY_CONFIG, 2, 6, 5, 7, seed=1, text_mask_tail=0.3)
    req = oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=7,
                                 ref_latent=r["ref_latent"], ref_mask=r["ref_mask"], initial_noise=r["initial_noise"])
    cond = oracle.encode_conditions(W, req)
    cos, sin = oracle.rope_tables(8, 7)
    t = torch.full((2,), 0.7)
    a = oracle.dit_forward(W, r["initial_noise"], t, oracle.build_kv_caches(W, cond), cos, sin)
    b = oracle.dit_forward(W, r["initial_noise"], t, oracle.build_kv_caches(W, cond), cos, sin)
    assert torch.equal(a, b)


def test_codec_decode_shapes_and_bounds(oracle, synth, tmp_path):
    # src/codec/decoder.rs:73-84 (tanh bound), model.rs:60-65 (length = T * hop)
    p = tmp_path / "c.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=16)
    W = oracle.load_codec(str(p))
    wav = oracle.codec_decode(W, torch.randn(2, 3, 32))
    assert wav.shape == (2, 1, 3 * 1920)
    assert wav.abs().max() <= 1.0


def test_temporal_score_rescale_kats(oracle):
    # src/rf/math.rs tests: no-op at t >= 1 (exact), identity when sigma = 0 or k = 1,
    # finite output, and the hand-computed value 4/3 at t = 0.5, k = 2, sigma = 1
    v = torch.tensor([[[1.0, 2.0]]])
    assert torch.equal(oracle.temporal_score_rescale(v, torch.tensor([[[5.0, 6.0]]]), 1.0, 1.5, 0.5), v)
    v = torch.tensor([[[3.0, 4.0]]])
    assert torch.equal(oracle.temporal_score_rescale(v, torch.tensor([[[9.0, 10.0]]]), 1.5, 2.0, 1.0), v)
    v = torch.tensor([[[2.0, 3.0]]])
    r = oracle.temporal_score_rescale(v, torch.tensor([[[1.0, 1.0]]]), 0.5, 1.0, 0.0)
    assert (r - v).abs().max().item() < 1e-5
    v = torch.tensor([[[2.0, -1.0]]])
    r = oracle.temporal_score_rescale(v, torch.tensor([[[0.5, 0.3]]]), 0.4, 1.0, 2.5)
    assert (r - v).abs().max().item() < 1e-5
    r = oracle.temporal_score_rescale(torch.tensor([[[1.0, -1.0]]]), torch.tensor([[[0.5, 0.3]]]), 0.3, 2.0, 1.0)
    assert torch.isfinite(r).all()
    r = oracle.temporal_score_rescale(torch.tensor([[[1.0]]]), torch.tensor([[[0.0]]]), 0.5, 2.0, 1.0)
    assert abs(r.item() - 4.0 / 3.0) < 1e-5


def _unit_cache(oracle, seq_text, seq_aux, heads, hd):
    ones = lambda s: torch.ones(1, s, heads, hd)  # noqa: E731
    return oracle.KvCache(ones(seq_text), ones(seq_text), ones(seq_aux), ones(seq_aux),
                          torch.ones(1, seq_text + seq_aux, dtype=torch.bool))


def test_scale_speaker_kv_cache_kats(oracle):
    # src/rf/kv_scaling.rs tests: scaling by 2 doubles the speaker (aux) K/V, leaves the
    # text K/V alone and rebuilds the joint context [text | aux] from them
    (c,) = oracle.scale_speaker_kv_cache([_unit_cache(oracle, 4, 3, 2, 8)], 2.0, None)
    assert torch.equal(c.aux_k, torch.full_like(c.aux_k, 2.0)) and torch.equal(c.aux_v, torch.full_like(c.aux_v, 2.0))
    assert torch.equal(c.text_k, torch.ones_like(c.text_k))
    ctx = c.ctx_k.reshape(-1)
    n_text = 4 * 2 * 8
    assert torch.equal(ctx[:n_text], torch.ones(n_text)) and torch.equal(ctx[n_text:], torch.full((3 * 2 * 8,), 2.0))
    # max_layers = 1 scales only the first layer's cache
    s = oracle.scale_speaker_kv_cache([_unit_cache(oracle, 2, 2, 1, 4), _unit_cache(oracle, 2, 2, 1, 4)], 3.0, 1)
    assert s[0].aux_k.max().item() == 3.0 and s[1].aux_k.max().item() == 1.0


def test_low_rank_adaln_zero_init_gate_is_tanh(oracle, synth):
    # src/model/norm.rs low_rank_adaln_zero_init_gate_is_tanh_of_input: with zero-initialised
    # up projections the gate is tanh of the raw gate input (0.5 -> tanh(0.5))
    import json
    D, r = 16, 4
    g = torch.Generator().manual_seed(0)
    t = {}
    for k in ("shift", "scale", "gate"):
        t[f"a.{k}_down.weight"] = torch.randn(r, D, generator=g)
        t[f"a.{k}_up.weight"] = torch.zeros(D, r)
    W = oracle.Weights(t, json.dumps(synth.TINY_CONFIG))
    h, gate = oracle.low_rank_adaln(W, "a", torch.ones(1, 3, D), torch.full((1, 1, 3 * D), 0.5), 1e-6)
    assert gate.shape == (1, 1, D) and h.shape == (1, 3, D)
    assert (gate - math.tanh(0.5)).abs().max().item() < 1e-5


def test_hidden_dim_rule(oracle, synth):
    # src/model/diffusion.rs hidden_dim_calculation: ((model_dim as f64 * mlp_ratio) as usize).max(1)
    import json
    for dim, ratio in ((32, 2.0), (2048, 2.875), (16, 2.7), (4, 0.1)):
        c = dict(synth.TINY_CONFIG, model_dim=dim, mlp_ratio=ratio)
        assert oracle.ModelConfig.from_json(json.dumps(c)).hidden_dim() == max(int(dim * ratio), 1)


def test_forward_with_zero_inputs_is_finite(oracle, synth, tmp_path):
    # src/model/diffusion.rs block_residual_connection_with_zeros: zero latents and a zero
    # condition give finite outputs (safe norms, safe softmax)
    p = tmp_path / "z.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    W = oracle.Weights.load(str(p))
    r = synth.make_request(synth.TINY_CONFIG, 1, 2, 3, 4, seed=1)
    req = oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=4,
                                 ref_latent=torch.zeros_like(r["ref_latent"]), ref_mask=r["ref_mask"],
                                 initial_noise=torch.zeros_like(r["initial_noise"]))
    cond = oracle.encode_conditions(W, req)
    cos, sin = oracle.rope_tables(W.cfg.head_dim(), 4)
    out = oracle.dit_forward(W, torch.zeros_like(r["initial_noise"]), torch.zeros(1), oracle.build_kv_caches(W, cond),
                             cos, sin)
    assert torch.isfinite(out).all()


def test_encoders_zero_masked_positions_and_survive_all_masked(oracle, synth, tmp_path):
    # src/model/text_encoder.rs text_encoder_masked_positions_are_zero /
    # text_encoder_all_false_mask_no_nan; src/model/speaker_encoder.rs
    # speaker_encoder_masked_positions_are_zero
    p = tmp_path / "e.safetensors"
    synth.make_dit_checkpoint(str(p), synth.TINY_CONFIG, seed=0, init="full")
    W = oracle.Weights.load(str(p))
    c, eps = W.cfg, W.cfg.norm_eps
    ids = torch.zeros(1, 4, dtype=torch.long)
    out = oracle.text_encoder(W, "text_encoder", ids, torch.tensor([[True, True, False, False]]), c.text_layers,
                              c.text_heads, eps)
    assert out[:, 2:].abs().sum().item() == 0.0 and out[:, :2].abs().sum().item() > 0
    out = oracle.text_encoder(W, "text_encoder", ids, torch.zeros(1, 4, dtype=torch.bool), c.text_layers,
                              c.text_heads, eps)
    assert torch.isfinite(out).all()
    lat = torch.ones(1, 4, W["speaker_encoder.in_proj.weight"].shape[1])
    out = oracle.speaker_encoder(W, "speaker_encoder", lat, torch.tensor([[True, True, False, False]]),
                                 c.speaker_layers, c.speaker_heads, eps)
    assert out[:, 2:].abs().sum().item() == 0.0


def test_speaker_patching(oracle):
    # src/model/speaker_encoder.rs patch_halves_length_doubles_dim, patch_mask_false_propagates,
    # patch_noop_when_size_1, patch_too_short_returns_error
    s, m = oracle.patch_sequence_with_mask(torch.ones(2, 8, 4), torch.ones(2, 8, dtype=torch.bool), 2)
    assert s.shape == (2, 4, 8) and m.shape == (2, 4)
    _, m = oracle.patch_sequence_with_mask(torch.ones(1, 4, 2), torch.tensor([[True, True, True, False]]), 2)
    assert m.tolist() == [[True, False]]
    s, m = oracle.patch_sequence_with_mask(torch.ones(1, 5, 3), torch.ones(1, 5, dtype=torch.bool), 1)
    assert s.shape == (1, 5, 3) and m.shape == (1, 5)
    with pytest.raises(ValueError, match="too short"):
        oracle.patch_sequence_with_mask(torch.ones(1, 1, 4), torch.ones(1, 1, dtype=torch.bool), 2)
