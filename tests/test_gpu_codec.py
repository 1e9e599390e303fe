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
