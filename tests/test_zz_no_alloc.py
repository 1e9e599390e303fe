"""Allocation-free decode entry point (irt_codec_decode_noalloc).

Callers that cannot allocate device memory during a decode (a streaming loop
that cannot absorb cudaMalloc/cudaFree synchronisation, or a host whose own
allocator holds the free HBM) use this variant: it keeps every intermediate
activation in a fixed 16 MiB device array compiled into the library.  This
test calls it through the C ABI twice in a row and checks both results
against the allocating irt_codec_decode on the same latent, at the largest
request the fixed array holds (batch x frames = 7) and below it, for a codec
loaded in f32 and one loaded in bf16 (the allocation-free path always runs
the fp32 SIMT decoder, so both must match the f32 allocating decode on its
SIMT kernels, IRT_CODEC_F32_SIMT=1), and that a request one frame larger is
rejected.  The file name makes pytest
collect it last; it also passes alone in a fresh process.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5  # same kernels in the same order: results should agree to rounding


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_decode_noalloc_matches_decode_twice(pkg, synth, tmp_path, monkeypatch):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    p = tmp_path / "codec_full.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=1)
    monkeypatch.setenv("IRT_CODEC_F32_SIMT", "1")  # read at load
    codec = pkg.load_codec(str(p), device=0)
    monkeypatch.delenv("IRT_CODEC_F32_SIMT")
    codec_bf16 = pkg.load_codec(str(p), device=0, precision="bf16")
    hop = codec.hop_length()
    g = torch.Generator().manual_seed(21)
    for B, T in ((1, 4), (2, 3), (1, 7)):
        lat = torch.randn(B, T, 32, generator=g).cuda()
        ref = torch.empty(B, 1, T * hop, device="cuda")
        codec.decode(lat, out=ref)
        for c in (codec, codec_bf16):
            for _ in range(2):  # the shared scratch keeps the previous call's contents
                wav = torch.full((B, 1, T * hop), float("nan"), device="cuda")
                pkg.decode_noalloc(c, lat, wav)
                assert torch.isfinite(wav).all()
                assert rel_l2(wav.cpu().numpy(), ref.cpu().numpy()) < TOL
    # beyond the fixed scratch capacity: clear error, nothing runs
    for B, T in ((1, 8), (2, 4)):
        big = torch.randn(B, T, 32, device="cuda")
        out = torch.empty(B, 1, T * hop, device="cuda")
        with pytest.raises(pkg.IrodoriError) as ei:
            pkg.decode_noalloc(codec_bf16, big, out)
        assert ei.value.kind == "Shape" and "scratch" in str(ei.value)
