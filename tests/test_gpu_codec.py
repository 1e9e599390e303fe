"""DACVAE decoder on the GPU (through the C ABI) against the CPU oracle
(src/codec/model.rs:60-65).  fp32 arithmetic; tolerance 1e-4 relative L2."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return 0


@pytest.mark.parametrize("width_div,B,T", [(8, 2, 5), (4, 1, 3)])
def test_codec_decode_matches_oracle(gpu, pkg, oracle, synth, tmp_path, width_div, B, T):
    p = tmp_path / f"codec_{width_div}.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=width_div)
    W = oracle.load_codec(str(p))
    g = torch.Generator().manual_seed(11)
    lat = torch.randn(B, T, 32, generator=g)
    ref = oracle.codec_decode(W, lat).numpy()
    codec = pkg.load_codec(str(p), device=0)
    assert codec.sample_rate() == 48000 and codec.hop_length() == 1920
    out = codec.decode(lat)
    assert out.shape == (B, 1, T * 1920)
    assert np.isfinite(out).all() and np.abs(out).max() <= 1.0
    err = rel_l2(out, ref)
    assert err < 1e-4, err


def test_codec_full_width_device_buffers(gpu, pkg, oracle, synth, tmp_path):
    """Full-width decoder (1536 -> 96 channels) on device buffers; compared
    with the oracle on a short latent."""
    p = tmp_path / "codec_full.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=1)
    W = oracle.load_codec(str(p))
    lat = torch.randn(1, 2, 32, generator=torch.Generator().manual_seed(3))
    ref = oracle.codec_decode(W, lat).numpy()
    codec = pkg.load_codec(str(p), device=0)
    out = torch.empty(1, 1, 2 * 1920, device="cuda")
    codec.decode(lat.cuda(), out=out)
    err = rel_l2(out.cpu().numpy(), ref)
    assert err < 1e-4, err


# ---------------------------------------------------------------------------
# bf16 tensor-core decoder (implicit-GEMM tcgen05 convolutions)
# ---------------------------------------------------------------------------

# Waveform relative L2 bound for bf16 operands with f32 accumulation (40 dB
# SNR).  Checked on the reference's own random initialisation of codec layers
# (synth init="reference"); the weight-norm stress init amplifies any input
# perturbation a few hundred times through its residual stack (fp32: 9e-5
# against the oracle; bf16 rounding alone, emulated on the CPU: 0.24), so it
# only serves the fp32 parity tests above.
BF16_TOL = 1e-2


def snr_db(out, ref):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(10 * np.log10(np.sum(ref ** 2) / max(np.sum((out - ref) ** 2), 1e-300)))


@pytest.fixture(scope="module")
def full_codec_path(tmp_path_factory, synth):
    p = tmp_path_factory.mktemp("codec_tc") / "codec_full_ref_init.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=1, init="reference")
    return str(p)


def test_codec_bf16_tc_matches_oracle(gpu, pkg, oracle, full_codec_path):
    W = oracle.load_codec(full_codec_path)
    lat = torch.randn(2, 6, 32, generator=torch.Generator().manual_seed(7))
    ref = oracle.codec_decode(W, lat).numpy()
    codec = pkg.load_codec(full_codec_path, device=0, precision="bf16")
    out = codec.decode(lat)
    assert out.shape == (2, 1, 6 * 1920)
    assert np.isfinite(out).all()
    err = rel_l2(out, ref)
    print(f"bf16 codec vs oracle: rel L2 {err:.3e}, SNR {snr_db(out, ref):.1f} dB")
    assert err < BF16_TOL, err


def test_codec_f32_ragged_is_per_utterance(gpu, pkg, oracle, synth, tmp_path):
    """Ragged decode = each utterance decoded alone at its length, zero tail."""
    p = tmp_path / "codec_8.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=8)
    W = oracle.load_codec(str(p))
    lat = torch.randn(3, 5, 32, generator=torch.Generator().manual_seed(9))
    lens = [5, 2, 0]
    codec = pkg.load_codec(str(p), device=0)
    out = codec.decode(lat, lengths=lens)
    for b, n in enumerate(lens):
        if n:
            ref = oracle.codec_decode(W, lat[b:b + 1, :n]).numpy()[0, 0]
            assert rel_l2(out[b, 0, :n * 1920], ref) < 1e-4
        assert not out[b, 0, n * 1920:].any()


@pytest.mark.parametrize("B,T,lens", [(2, 150, None), (3, 200, [200, 57, 1]), (3, 3000, [3000, 1200, 100])])
def test_codec_bf16_tc_matches_f32(gpu, pkg, full_codec_path, B, T, lens):
    """Larger and ragged batches (the last case spans two decode chunks)
    against the fp32 GPU decoder, itself checked against the oracle above."""
    g = torch.Generator().manual_seed(B * 1000 + T)
    lat = torch.randn(B, T, 32, generator=g).cuda()
    hop = 1920
    ref = torch.empty(B, 1, T * hop, device="cuda")
    out = torch.full((B, 1, T * hop), float("nan"), device="cuda")
    pkg.load_codec(full_codec_path, device=0, precision="f32").decode(lat, out=ref, lengths=lens)
    pkg.load_codec(full_codec_path, device=0, precision="bf16").decode(lat, out=out, lengths=lens)
    torch.cuda.synchronize()
    lens = lens or [T] * B
    for b, n in enumerate(lens):
        o = out[b, 0].cpu().numpy()
        r = ref[b, 0].cpu().numpy()
        assert np.isfinite(o).all()
        assert not o[n * hop:].any()
        err = rel_l2(o[:n * hop], r[:n * hop])
        print(f"B={B} T={T} utt {b} len {n}: rel L2 {err:.3e}, SNR {snr_db(o[:n * hop], r[:n * hop]):.1f} dB")
        assert err < BF16_TOL, (b, err)


@pytest.mark.parametrize("B,T,lens", [(1, 300, None), (3, 40, [40, 7, 1])])
def test_codec_f32_tf32_matches_simt(gpu, pkg, full_codec_path, monkeypatch, B, T, lens):
    """The fp32 decoder runs its convolutions on the tf32 hi / lo GEMM by
    default; against its SIMT kernels (IRT_CODEC_F32_SIMT=1, read at load) on
    the reference's random initialisation, full width, longer and ragged
    batches than the oracle can take."""
    g = torch.Generator().manual_seed(B * 100 + T)
    lat = torch.randn(B, T, 32, generator=g).cuda()
    hop = 1920
    outs = []
    for simt in (None, "1"):
        if simt:
            monkeypatch.setenv("IRT_CODEC_F32_SIMT", simt)
        else:
            monkeypatch.delenv("IRT_CODEC_F32_SIMT", raising=False)
        o = torch.full((B, 1, T * hop), float("nan"), device="cuda")
        pkg.load_codec(full_codec_path, device=0, precision="f32").decode(lat, out=o, lengths=lens)
        torch.cuda.synchronize()
        outs.append(o.cpu().numpy())
    lens = lens or [T] * B
    for b, n in enumerate(lens):
        assert np.isfinite(outs[0][b, 0]).all()
        assert not outs[0][b, 0, n * hop:].any()
        err = rel_l2(outs[0][b, 0, :n * hop], outs[1][b, 0, :n * hop])
        print(f"f32 codec tf32 vs SIMT, utt {b} len {n}: rel L2 {err:.3e}")
        assert err < 1e-5, (b, err)


def test_codec_weight_norm_checkpoint_resolved_at_load(gpu, pkg, synth, tmp_path):
    """A checkpoint holding the weight-norm parametrisation (X.weight_g /
    X.weight_v) decodes like the resolved one (scripts/convert_dacvae_weights.py
    resolution applied at load), in both precisions."""
    merged = tmp_path / "merged.safetensors"
    wn = tmp_path / "weight_norm.safetensors"
    synth.make_codec_checkpoint(str(merged), seed=5, width_div=1, init="reference")
    synth.make_codec_checkpoint(str(wn), seed=5, width_div=1, init="reference", weight_norm=True)
    lat = torch.randn(1, 5, 32, generator=torch.Generator().manual_seed(13))
    # f32: the resolution itself (last-bit differences only); bf16: weights that
    # differ in their last f32 bits round to bf16 differently, so the two decodes
    # differ by about the bf16 error itself -- bounded like any bf16 decode
    for prec, tol in (("f32", 1e-5), ("bf16", BF16_TOL)):
        a = pkg.load_codec(str(merged), device=0, precision=prec).decode(lat)
        b = pkg.load_codec(str(wn), device=0, precision=prec).decode(lat)
        assert rel_l2(b, a) < tol, (prec, rel_l2(b, a))
