"""CPU tests of the host side: the C-ABI library loads and exports every
symbol the header declares; parameter defaults/validation through the C ABI
(no device needed); checkpoint layout produced by the synthetic generator;
the utterance sharder."""

import re
from pathlib import Path

import pytest

from conftest import PKG_DIR, ROOT

HEADER = ROOT / "include" / "irodori_b200.h"


def declared_symbols():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"IRT_API\s+[\w\s\*]+?\b(irt_\w+)\s*\(", txt)))


def test_header_declares_symbols():
    syms = declared_symbols()
    assert "irt_engine_sample" in syms and "irt_codec_decode" in syms
    assert len(syms) >= 19


def test_library_exports_every_declared_symbol(pkg):
    if not pkg.LIB_PATH.exists():
        pytest.skip("library not built (run __graft_entry__.build())")
    L = pkg.lib()
    for s in declared_symbols():
        assert hasattr(L, s), s
    # and the Python mirror binds exactly the declared surface
    from irodori_b200 import _SIGNATURES
    assert sorted(_SIGNATURES) == declared_symbols()


def test_defaults_match_reference(pkg):
    if not pkg.LIB_PATH.exists():
        pytest.skip("library not built")
    p = pkg.SamplerParams()
    c = p._to_c()
    assert c.num_steps == 40 and c.method == 0 and c.cfg_mode == 0
    assert (c.scale_text, c.scale_caption, c.scale_speaker, c.min_t, c.max_t) == (3.0, 3.0, 5.0, 0.5, 1.0)
    assert c.use_context_kv_cache == 1 and c.speaker_kv_max_layers == -1
    p.validate()


@pytest.mark.parametrize("kw,msg", [
    (dict(num_steps=0), "Invalid configuration: num_steps must be > 0"),
    (dict(guidance=dict(min_t=1.5)), "guidance.min_t must be finite and in [0, 1], got 1.5"),
    (dict(guidance=dict(min_t=0.8, max_t=0.6)), "guidance.min_t (0.8) must not exceed guidance.max_t (0.6)"),
    (dict(guidance=dict(scale_text=float("inf"))), "guidance.scale_text must be finite, got inf"),
    (dict(truncation_factor=-1.0), "truncation_factor must be finite and > 0"),
    (dict(temporal_rescale=(1.0, 0.0)), "temporal_rescale.sigma must not be zero"),
    (dict(speaker_kv=(0.0, None, None)), "speaker_kv.scale must be finite and > 0"),
    (dict(speaker_kv=(1.0, None, 2.0)), "speaker_kv.min_t must be finite and in [0, 1]"),
    (dict(method="plms4", guidance=dict(mode="alternating")), "PLMS4 is not compatible"),
])
def test_validate_messages_through_c_abi(pkg, kw, msg):
    """SamplerParams::validate rejections (src/rf/params.rs:253-378) with the
    reference's message text, checked through the C ABI on CPU."""
    if not pkg.LIB_PATH.exists():
        pytest.skip("library not built")
    g = pkg.GuidanceConfig(**kw.pop("guidance", {}))
    tr = kw.pop("temporal_rescale", None)
    sk = kw.pop("speaker_kv", None)
    p = pkg.SamplerParams(guidance=g, temporal_rescale=pkg.TemporalRescaleConfig(*tr) if tr else None,
                          speaker_kv=pkg.SpeakerKvConfig(*sk) if sk else None, **kw)
    with pytest.raises(pkg.ConfigError) as ei:
        p.validate()
    assert msg in str(ei.value)
    assert ei.value.kind == "Config"


@pytest.mark.parametrize("g", [dict(scale_text=float("nan")), dict(scale_speaker=float("-inf")), dict(min_t=2.0),
                               dict(min_t=-0.25), dict(max_t=1.0000001), dict(min_t=0.9, max_t=0.1),
                               dict(min_t=float("nan"))])
def test_validate_messages_match_oracle(pkg, oracle, g):
    """The C ABI and the oracle reject the same guidance values with the same
    text, f32 fields printed the way the reference's Rust formats them."""
    if not pkg.LIB_PATH.exists():
        pytest.skip("library not built")
    with pytest.raises(pkg.ConfigError) as ec:
        pkg.SamplerParams(guidance=pkg.GuidanceConfig(**g)).validate()
    with pytest.raises(ValueError) as eo:
        oracle.SamplerParams(guidance=oracle.GuidanceConfig(**g)).validate()
    assert str(ec.value).endswith(str(eo.value)), (str(ec.value), str(eo.value))


def test_unknown_method_is_unsupported_mode(pkg):
    if not pkg.LIB_PATH.exists():
        pytest.skip("library not built")
    with pytest.raises(pkg.IrodoriError) as ei:
        pkg.SamplerParams(method="rk4").validate()
    assert ei.value.kind == "UnsupportedMode"


def test_synthetic_checkpoint_loads_in_oracle(oracle, synth, tmp_path):
    p = tmp_path / "s.safetensors"
    cfg = synth.make_dit_checkpoint(str(p), synth.SMALL_CONFIG, seed=1, init="baseline")
    W = oracle.Weights.load(str(p))
    assert W.cfg.model_dim == 256 and W.cfg.hidden_dim() == 736
    assert W["blocks.0.attention_adaln.shift_up.weight"].abs().max() == 0  # zero-init adaLN up
    assert W["out_proj.weight"].abs().max() > 0                           # documented deviation
    assert cfg["num_layers"] == 2
    # every tensor the record builders read is present
    for k in synth.dit_param_shapes(cfg):
        assert W.has(k), k


def test_lpt_sharding_balances_and_partitions(synth):
    from irodori_b200 import sharding
    utts = synth.throughput_utterances(64, seed=4)
    costs = [sharding.utterance_cost(S, tl, rf) for tl, S, rf, _ in utts]
    for world in (1, 2, 4, 8):
        bins = sharding.lpt_bins(costs, world)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(64))
        ratio, _ = sharding.imbalance(costs, bins)
        assert ratio < 1.1, (world, ratio)


def test_config4_workload_shape(synth):
    utts = synth.throughput_utterances(64, seed=4)
    assert len(utts) == 64
    assert all(16 <= tl <= 256 and 50 <= S <= 750 and 125 <= rf <= 375 for tl, S, rf, _ in utts)


class _FakeCodec:
    """Stands in for a DacVaeCodec: the argument checks of decode_noalloc run
    before any call into the library."""
    _device = 0
    _h = None

    def hop_length(self):
        return 1920


def test_decode_noalloc_rejects_bad_arguments_before_the_c_call(pkg):
    import torch
    c = _FakeCodec()
    lat = torch.zeros(1, 2, 32)
    wav = torch.zeros(1, 1, 2 * 1920)
    cases = [
        (lat.half(), wav, "Dtype", "latent must be float32"),
        (lat, wav.double(), "Dtype", "wav must be float32"),
        (lat, torch.zeros(1, 1, 2 * 1920 * 2)[..., ::2], "InvalidArgument", "wav must be contiguous"),
        (torch.zeros(1, 32, 2).transpose(1, 2), wav, "InvalidArgument", "latent must be contiguous"),
        (torch.zeros(1, 2, 16), wav, "Shape", "latent must be"),
        (lat, torch.zeros(1, 1, 1920), "Shape", "wav"),
        (lat, wav, "InvalidArgument", "CUDA tensor on the codec's GPU"),  # host tensors
        (lat.numpy(), wav, "InvalidArgument", "torch tensor"),
    ]
    for la, wa, kind, msg in cases:
        with pytest.raises(pkg.IrodoriError) as ei:
            pkg.decode_noalloc(c, la, wa)
        assert ei.value.kind == kind and msg in str(ei.value), (kind, str(ei.value))
