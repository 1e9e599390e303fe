"""Host-side data formats of the reference's text-to-speech pipeline binary
(src/bin/pipeline.rs), around the sampling and decode path:

* ``load_initial_noise`` -- a safetensors file with key ``initial_noise``
  (f32, rank 3) fed to the sampler instead of internal noise
  (pipeline.rs:170-213).
* ``find_flattening_point`` -- the tail-trim heuristic applied to the sampled
  latent before decoding (pipeline.rs:368-421, defaults window 20, std 0.05,
  mean 0.1 from the CLI, :132-142; applied at :560-579).
* ``trim_tail`` -- that trim applied to a ``[1, S, D]`` latent.
* ``save_wav`` -- 16-bit PCM mono WAV of a ``[1, 1, n]`` / ``[n]`` waveform,
  samples clamped to [-1, 1] and scaled by 32767 with round-half-away-from-zero
  (pipeline.rs:336-361).

Pure numpy: these run on the host before and after the GPU path.
"""

from __future__ import annotations

import json
import struct
from typing import Optional

import numpy as np

TRIM_WINDOW = 20
TRIM_STD = 0.05
TRIM_MEAN = 0.1


def _read_safetensors_header(raw: bytes):
    if len(raw) < 8:
        raise ValueError("invalid safetensors file: shorter than its header length field")
    n = struct.unpack("<Q", raw[:8])[0]
    if 8 + n > len(raw):
        raise ValueError("invalid safetensors file: header length beyond the file")
    return json.loads(raw[8:8 + n].decode("utf-8")), 8 + n


def load_initial_noise(path: str, seq_len: int) -> np.ndarray:
    """``initial_noise`` tensor of a safetensors file as float32 [B, S, D]
    (pipeline.rs:175-213): the key must exist, be rank 3, f32, and its second
    dimension must equal the pipeline's ``seq_len``."""
    with open(path, "rb") as f:
        raw = f.read()
    header, base = _read_safetensors_header(raw)
    info = header.get("initial_noise")
    if info is None:
        raise KeyError("key 'initial_noise' not found in noise file")
    shape = list(info["shape"])
    if len(shape) != 3:
        raise ValueError(f"initial_noise must be rank-3, got shape {shape}")
    if shape[1] != seq_len:
        raise ValueError(f"initial_noise seq_len={shape[1]} but pipeline seq_len={seq_len}; "
                         f"re-export with --seq-len {seq_len}")
    if info.get("dtype") != "F32":
        raise ValueError(f"initial_noise must be stored as F32, got {info.get('dtype')}")
    b0, b1 = info["data_offsets"]
    data = np.frombuffer(raw[base + b0:base + b1], dtype="<f4")
    if data.size != shape[0] * shape[1] * shape[2]:
        raise ValueError("initial_noise byte length does not match its shape")
    return data.reshape(shape).astype(np.float32, copy=True)


def _seq_sum(a: np.ndarray) -> np.float32:
    """Left-to-right float32 sum (the reference's ``iter().sum()`` order)."""
    if a.size == 0:
        return np.float32(0.0)
    return np.cumsum(a, dtype=np.float32)[-1]


def find_flattening_point(latent: np.ndarray, window_size: int = TRIM_WINDOW,
                          std_threshold: float = TRIM_STD, mean_threshold: float = TRIM_MEAN) -> int:
    """First latent frame where a trailing window of ``window_size`` frames
    (zero-padded past the end) is near-flat and near-zero
    (pipeline.rs:374-421), in float32 with the reference's summation order.
    ``latent`` is ``[T, D]``; returns a frame index in ``[0, T]``."""
    x = np.ascontiguousarray(latent, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError("latent must be [T, D]")
    total_t, dim = x.shape
    if total_t == 0 or window_size == 0:
        return total_t
    flat = x.reshape(-1)
    std_t, mean_t = np.float32(std_threshold), np.float32(mean_threshold)
    n_full = window_size * dim
    for i in range(total_t):
        w_start, w_end = i * dim, (i + window_size) * dim
        if w_end <= flat.size:
            w = flat[w_start:w_end]
            n = np.float32(w.size)
            mean = _seq_sum(w) / n
            d = w - mean
            std = np.sqrt(_seq_sum(d * d) / n, dtype=np.float32)
        else:
            # window runs into the zero padding
            avail = flat.size - w_start
            n = np.float32(n_full)
            w = flat[w_start:w_start + avail]
            mean = _seq_sum(w) / n
            d = w - mean
            sq = _seq_sum(d * d) + np.float32(n_full - avail) * (mean * mean)
            std = np.sqrt(sq / n, dtype=np.float32)
        if std < std_t and abs(mean) < mean_t:
            return i
    return total_t


def trim_tail(latent: np.ndarray, window_size: int = TRIM_WINDOW, std_threshold: float = TRIM_STD,
              mean_threshold: float = TRIM_MEAN) -> np.ndarray:
    """``latent`` [1, S, D] cut at ``find_flattening_point`` (pipeline.rs:560-579)."""
    if latent.ndim != 3 or latent.shape[0] != 1:
        raise ValueError("trim_tail expects a [1, S, D] latent")
    t = find_flattening_point(latent[0], window_size, std_threshold, mean_threshold)
    return latent[:, :t] if t < latent.shape[1] else latent


def round_half_away(a: np.ndarray) -> np.ndarray:
    """Rust ``f32::round``: halves go away from zero (numpy rounds to even)."""
    a = np.asarray(a, dtype=np.float32)
    t = np.trunc(a)
    frac = a - t  # exact for |a| < 2^23
    return np.where(np.abs(frac) >= np.float32(0.5), t + np.sign(a), t).astype(np.float32)


def pcm16(audio: np.ndarray) -> np.ndarray:
    """float waveform -> int16: clamp to [-1, 1], times 32767, round half away
    from zero."""
    a = np.clip(np.asarray(audio, dtype=np.float32).reshape(-1), -1.0, 1.0) * np.float32(32767.0)
    return round_half_away(a).astype(np.int16)


def save_wav(path: str, audio: np.ndarray, sample_rate: int = 48000, n_samples: Optional[int] = None) -> None:
    """16-bit PCM mono WAV (RIFF/WAVE, fmt chunk of 16 bytes, data chunk)."""
    pcm = pcm16(audio)
    if n_samples is not None:
        pcm = pcm[:n_samples]
    data = pcm.astype("<i2").tobytes()
    with open(path, "wb") as f:
        f.write(b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE")
        f.write(b"fmt " + struct.pack("<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16))
        f.write(b"data" + struct.pack("<I", len(data)) + data)
