"""Host-side pipeline formats around the sampling path (src/bin/pipeline.rs):
initial-noise files, the tail-trim heuristic and the 16-bit WAV writer."""

import wave

import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def pio(pkg):
    import irodori_b200.pipeline_io as m
    return m


def test_load_initial_noise(pio, synth, tmp_path):
    x = torch.randn(2, 17, 32, generator=torch.Generator().manual_seed(1))
    p = tmp_path / "noise.safetensors"
    synth.write_safetensors(str(p), {"initial_noise": x}, {})
    got = pio.load_initial_noise(str(p), 17)
    assert got.dtype == np.float32 and got.shape == (2, 17, 32)
    assert np.array_equal(got, x.numpy())
    with pytest.raises(ValueError, match="seq_len=17 but pipeline seq_len=18"):
        pio.load_initial_noise(str(p), 18)
    synth.write_safetensors(str(p), {"initial_noise": x[0]}, {})
    with pytest.raises(ValueError, match="must be rank-3"):
        pio.load_initial_noise(str(p), 17)
    synth.write_safetensors(str(p), {"noise": x}, {})
    with pytest.raises(KeyError, match="initial_noise"):
        pio.load_initial_noise(str(p), 17)


def _flat_point_f64(lat, w, std_t, mean_t):
    """Direct float64 statement of the heuristic (zero padding past the end)."""
    T, D = lat.shape
    padded = np.concatenate([lat, np.zeros((w, D))], 0).astype(np.float64)
    for i in range(T):
        win = padded[i:i + w].reshape(-1)
        if win.std() < std_t and abs(win.mean()) < mean_t:
            return i
    return T


def test_find_flattening_point_known_answers(pio):
    g = np.random.default_rng(3)
    lat = g.standard_normal((50, 8)).astype(np.float32)
    lat[30:] = 0.0
    assert pio.find_flattening_point(lat) == 30           # first all-zero window
    assert pio.find_flattening_point(g.standard_normal((40, 8)).astype(np.float32)) == 40
    assert pio.find_flattening_point(np.zeros((12, 4), np.float32)) == 0
    assert pio.find_flattening_point(np.zeros((0, 4), np.float32)) == 0
    assert pio.find_flattening_point(lat, window_size=0) == 50
    # window longer than the latent: only zero-padded windows
    short = np.full((5, 3), 0.01, np.float32)
    assert pio.find_flattening_point(short, window_size=20) == 0


def test_find_flattening_point_matches_direct_statement(pio):
    g = np.random.default_rng(7)
    for trial in range(20):
        T = int(g.integers(20, 120))
        lat = g.standard_normal((T, 32)).astype(np.float32)
        cut = int(g.integers(0, T))
        lat[cut:] *= np.float32(0.01)          # quiet tail below the thresholds
        want = _flat_point_f64(lat.astype(np.float64), 20, 0.05, 0.1)
        assert pio.find_flattening_point(lat) == want, trial


def test_trim_tail(pio):
    lat = np.zeros((1, 40, 8), np.float32)
    lat[0, :25] = 1.0 + np.arange(25, dtype=np.float32)[:, None]
    out = pio.trim_tail(lat)
    assert out.shape == (1, 25, 8)
    noisy = np.random.default_rng(0).standard_normal((1, 40, 8)).astype(np.float32)
    assert pio.trim_tail(noisy).shape == (1, 40, 8)


def test_pcm16_rounding_and_clamp(pio):
    below_half = np.nextafter(np.float32(0.5), np.float32(0))
    assert np.array_equal(pio.round_half_away(np.array([0.5, 1.5, 2.5, -0.5, -2.5, 0.49, below_half, -below_half],
                                                       np.float32)),
                          np.array([1, 2, 3, -1, -3, 0, 0, 0], np.float32))
    got = pio.pcm16(np.array([1.0, -1.0, 2.0, -3.0, 0.0, 0.5], np.float32))
    assert got.tolist() == [32767, -32767, 32767, -32767, 0, 16384]


def test_save_wav_roundtrip(pio, tmp_path):
    a = np.sin(np.linspace(0, 20, 4801, dtype=np.float32)) * 0.8
    p = tmp_path / "out.wav"
    pio.save_wav(str(p), a[None, None, :], sample_rate=48000)
    with wave.open(str(p), "rb") as w:
        assert (w.getnchannels(), w.getsampwidth(), w.getframerate(), w.getnframes()) == (1, 2, 48000, 4801)
        data = np.frombuffer(w.readframes(4801), dtype="<i2")
    assert np.array_equal(data, pio.pcm16(a))
