#!/usr/bin/env python
"""Benchmark of the RF sampling hot path on B200.

Workload (`value`): BASELINE config 4 -- 64 independent utterances, text
lengths U{16..256}, durations U[2,30] s (25 latent frames/s), speaker
references U[5,15] s, 40 Euler steps with joint CFG (scale 3.0, default
window min_t = 0.5), bf16, seed 4.  Utterances are split across ranks by
greedy LPT bins; each rank samples its bin as one ragged batch with no
collective on the data path ("scaling": "strong": the 64 utterances are the
whole job at every N).  Metric: audio-seconds generated per second.

One bench step = one full sample() of the rank's bin (prologue encoders +
context KV cache + 40 RF steps).  `value` has inputs resident in HBM; `e2e`
goes through the public API with host buffers (H2D inputs and D2H latents
inside the timed region).  The DiT checkpoint is random-init with the default
ModelConfig except latent_dim = 32 (the codec's latent width, as configs 4/5
require); weights are bf16 and larger than L2, so every step streams them.

`--impl reference` times the CPU restatement of the reference path (the
reference crate needs a Rust toolchain that is not on the box) on the host
cores, on a bounded sample of the same workload, extrapolated to the metric.
"""

from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "irodori-tts-burn_b200"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "audio-sec generated/sec (40-step joint-CFG RF sampling, config 4)"
UNIT = "audio_s/s"
FRAME_RATE = 25.0
N_UTT = 64


def load_pkg():
    if "irodori_b200" in sys.modules:
        return sys.modules["irodori_b200"]
    spec = importlib.util.spec_from_file_location("irodori_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["irodori_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def model_cfg():
    pkg = load_pkg()
    import irodori_b200.synth as synth
    c = dict(synth.DEFAULT_CONFIG)
    c["latent_dim"] = 32
    return c


def row_forward_flops(S, skv_valid, L=24, D=2048, F=5888, P=32):
    """Algorithmic FLOPs of one DiT row-forward over S latent tokens with
    skv_valid valid keys (masked keys not credited)."""
    per_tok_layer = 2 * D * 4 * D + 2 * D * D + 2 * D * 2 * F + 2 * F * D
    return S * (L * (per_tok_layer + 4 * D * skv_valid) + 2 * 2 * D * P)


def workload(seed=4):
    import irodori_b200.synth as synth
    return synth.throughput_utterances(N_UTT, seed=seed)


def build_batch(utts, idx, P, vocab, seed=4):
    """Ragged batch tensors (CPU) for the utterances `idx`."""
    import torch
    g = torch.Generator().manual_seed(seed * 1000003)
    # draw per-utterance tensors in global order so every rank sees the same data
    per = []
    for i, (tl, S, rf, _) in enumerate(utts):
        ids = torch.randint(0, vocab, (tl,), generator=g, dtype=torch.int64)
        ref = torch.randn(rf, P, generator=g)
        noise = torch.randn(S, P, generator=g)
        per.append((ids, ref, noise))
    B = len(idx)
    Tt = max(utts[i][0] for i in idx)
    Tr = max(utts[i][2] for i in idx)
    Sm = max(utts[i][1] for i in idx)
    ids = torch.zeros(B, Tt, dtype=torch.int32)
    tm = torch.zeros(B, Tt, dtype=torch.uint8)
    ref = torch.zeros(B, Tr, P)
    rm = torch.zeros(B, Tr, dtype=torch.uint8)
    noise = torch.zeros(B, Sm, P)
    lens = []
    for b, i in enumerate(idx):
        tl, S, rf, _ = utts[i]
        ids[b, :tl] = per[i][0].to(torch.int32)
        tm[b, :tl] = 1
        ref[b, :rf] = per[i][1]
        rm[b, :rf] = 1
        noise[b, :S] = per[i][2]
        lens.append(S)
    return dict(text_ids=ids, text_mask=tm, ref_latent=ref, ref_mask=rm, initial_noise=noise, sequence_lengths=lens,
                sequence_length=Sm)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.f is None:
            return None
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[5 + j].lower() == "active"})
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def measured_sustained():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()).get("bf16_tflops_sustained")
    return None


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


# ---------------------------------------------------------------------------
# Dominant-kernel roofline: the tcgen05 GEMM on this workload's DiT shapes
# ---------------------------------------------------------------------------

def gemm_layer_bytes(M, D=2048, F=5888):
    """Algorithmic HBM bytes of the four DiT GEMMs of one layer at M rows:
    bf16 operands and weights read once, bf16 outputs written once, the f32
    residual read and written by each of the two residual epilogues."""
    qkvg = 2 * (M * D + 4 * D * D) + 2 * 4 * M * D
    wo = 2 * (M * D + D * D) + 2 * 4 * M * D
    w13 = 2 * (M * D + 2 * F * D) + 2 * M * F
    w2 = 2 * (M * F + D * F) + 2 * 4 * M * D
    return qkvg + wo + w13 + w2


# DRAM bytes (read + write) of the four DiT GEMMs of one layer per row of M,
# from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum over the
# four gemm_kernel launches of `--gemm-case 54504`: 5.751 GB).  The operands
# and outputs all grow with M (the weights are read about once), so the
# per-layer traffic at another M is this figure times M.
GEMM_LAYER_TRAFFIC_PER_ROW = 5750995200 / 54504


def gemm_roofline(M, reps=5, sustain_s=0.0):
    """Times gemm_kernel (tcgen05) on the four DiT GEMMs of one layer at the
    CFG-step row count M with the same fused epilogues the engine uses, with
    CUDA events on the launching stream.  Returns (achieved TFLOP/s, per-layer
    ms, FLOPs per layer)."""
    import torch
    L = ctypes.CDLL(str(PKG_DIR / "libirodori_b200_testhooks.so"))
    L.irtt_gemm_epi.argtypes = ([ctypes.c_int] + [ctypes.c_void_p] * 2 + [ctypes.c_int] * 4 + [ctypes.c_void_p] * 9
                                + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 2 + [ctypes.c_int])
    L.irtt_last_error.restype = ctypes.c_char_p
    dev = torch.device("cuda")
    D, F, H, hd = 2048, 5888, 16, 128
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    h = torch.randn(M, D, device=dev, generator=g).to(bf)
    hm = torch.randn(M, F, device=dev, generator=g).to(bf)
    wqkvg = (torch.randn(4 * D, D, device=dev, generator=g) * 0.02).to(bf)
    wo = (torch.randn(D, D, device=dev, generator=g) * 0.02).to(bf)
    w13 = (torch.randn(2 * F, D, device=dev, generator=g) * 0.02).to(bf)
    w2 = (torch.randn(D, F, device=dev, generator=g) * 0.02).to(bf)
    outs = [torch.empty(M, D, device=dev, dtype=bf) for _ in range(4)]
    hout = torch.empty(M, F, device=dev, dtype=bf)
    x = torch.zeros(M, D, device=dev)
    gate = torch.ones(D, device=dev)
    nw = torch.ones(D, device=dev)
    cos = torch.ones(1024, hd // 2, device=dev)
    sin = torch.zeros(1024, hd // 2, device=dev)
    pos = (torch.arange(M, device=dev) % 1024).to(torch.int32)
    P = lambda t: ctypes.c_void_p(t.data_ptr())

    def ck(rc):
        if rc:
            raise RuntimeError(L.irtt_last_error().decode())

    parts = [
        lambda: ck(L.irtt_gemm_epi(1, P(h), P(wqkvg), M, 4 * D, D, 0, *[P(o) for o in outs], P(nw), P(nw), P(cos),
                                   P(sin), P(pos), H, hd, H // 2, None, None, 0)),
        lambda: ck(L.irtt_gemm_epi(2, P(outs[0]), P(wo), M, D, D, 0, None, None, None, None, None, None, None, None,
                                   None, 0, 0, 0, P(x), P(gate), 0)),
        lambda: ck(L.irtt_gemm_epi(3, P(h), P(w13), M, 2 * F, D, 0, P(hout), None, None, None, None, None, None, None,
                                   None, 0, 0, 0, None, None, F)),
        lambda: ck(L.irtt_gemm_epi(2, P(hm), P(w2), M, D, F, 0, None, None, None, None, None, None, None, None, None,
                                   0, 0, 0, P(x), P(gate), 0)),
    ]

    def run():
        for fn in parts:
            fn()

    run.parts = parts

    run()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    per = [0.0] * 4
    for _ in range(reps):
        ev[0].record(st)
        for i, fn in enumerate(run.parts):
            fn()
            ev[i + 1].record(st)
        torch.cuda.synchronize()
        for i in range(4):
            per[i] += ev[i].elapsed_time(ev[i + 1]) / reps
    ms = sum(per)
    flops = 2.0 * M * D * (4 * D + D + 2 * F) + 2.0 * M * F * D
    gemm_roofline.last_parts = {n: round(t, 4) for n, t in zip(("qkvg_ms", "wo_ms", "w13_ms", "w2_ms"), per)}
    gemm_roofline.sustained = None
    if sustain_s > 0:
        # Inside a long sampling step the GPU runs power-capped: repeat the
        # layer for ~sustain_s / 2 s to reach that state, then time ~sustain_s s
        # of back-to-back layers between two events on the launching stream.
        t_end = time.time() + sustain_s / 2
        while time.time() < t_end:
            for _ in range(20):
                run()
            torch.cuda.synchronize()
        n = max(1, int(sustain_s * 1000.0 / ms))
        ev[0].record(st)
        for _ in range(n):
            run()
        ev[1].record(st)
        torch.cuda.synchronize()
        ms_s = ev[0].elapsed_time(ev[1]) / n
        gemm_roofline.sustained = (flops / (ms_s * 1e-3) / 1e12, ms_s, n)
    return flops / (ms * 1e-3) / 1e12, ms, flops


# ---------------------------------------------------------------------------
# CPU leg: the oracle (restatement of the reference path) on the host cores
# ---------------------------------------------------------------------------

def row_case(M, steps):
    """Profiling case: the adaLN modulate row kernel (rownorm_reg_kernel, the
    bandwidth-bound kernel of each DiT block) at M rows of D = 2048: f32 x in,
    bf16 h out, CUDA events over `steps` back-to-back launches.  At the
    config-4 CFG step (M = 54,504) x alone is 446 MB, larger than L2.
    Returns (us per launch, algorithmic GB/s)."""
    import torch
    L = ctypes.CDLL(str(PKG_DIR / "libirodori_b200_testhooks.so"))
    L.irtt_adaln_modulate.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_float]
    L.irtt_last_error.restype = ctypes.c_char_p
    D = 2048
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, D, device="cuda", generator=g)
    shift = torch.randn(D, device="cuda", generator=g) * 0.1
    scale = torch.randn(D, device="cuda", generator=g) * 0.1
    h = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def launch():
        if L.irtt_adaln_modulate(P(x), P(shift), P(scale), P(h), 1, M, D, 1e-5):
            raise RuntimeError(L.irtt_last_error().decode())

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / steps
    nbytes = M * D * 4 + M * D * 2 + 2 * D * 4
    return us, nbytes / (us * 1e-6) / 1e9


def simt_case(steps, steps_per_request=40):
    """Profiling case: the f32 SIMT GEMMs that build one request's per-step
    tables (gemm_simt_kernel, engine.cu cond_module + adaLN), at the default
    ModelConfig (D = 2048, 24 layers, adaLN rank 256, timestep embedding 512)
    and steps_per_request + 1 timestep rows: the three cond_module layers,
    then per adaLN kind (attention, MLP, gate) the down projection of all
    layers at once and the batched (layer, half) up projections.  `steps`
    repetitions of the ten launches timed with CUDA events.  Returns (ms per
    request, TFLOP/s)."""
    import torch
    L = ctypes.CDLL(str(PKG_DIR / "libirodori_b200_testhooks.so"))
    L.irtt_gemm_simt.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_long] * 2
                                 + [ctypes.c_void_p, ctypes.c_long, ctypes.c_long] + [ctypes.c_int] * 4)
    L.irtt_last_error.restype = ctypes.c_char_p
    NT, D, NL, R, TE = steps_per_request + 1, 2048, 24, 256, 512
    g = torch.Generator(device="cuda").manual_seed(0)
    rnd = lambda *s: torch.randn(*s, device="cuda", generator=g)  # noqa: E731
    temb, h0, h1, ce = rnd(NT, TE), rnd(NT, D), rnd(NT, D), rnd(NT, 3 * D)
    cm = [rnd(D, TE) * 0.02, rnd(D, D) * 0.02, rnd(3 * D, D) * 0.02]
    down = [rnd(NL * 2 * R, D) * 0.02 for _ in range(3)]
    up = [rnd(NL * 2, D, R) * 0.02 for _ in range(3)]
    dn = torch.empty(NT, NL * 2 * R, device="cuda")
    raw = torch.empty(NL * 2, NT, D, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    calls = [(temb, TE, 0, cm[0], TE, 0, h0, D, 0, D, TE, 1),
             (h0, D, 0, cm[1], D, 0, h1, D, 0, D, D, 1),
             (h1, D, 0, cm[2], D, 0, ce, 3 * D, 0, 3 * D, D, 1)]
    for k in range(3):
        calls.append((ce[:, k * D:], 3 * D, 0, down[k], D, 0, dn, NL * 2 * R, 0, NL * 2 * R, D, 1))
        calls.append((dn, NL * 2 * R, R, up[k], R, D * R, raw, D, NT * D, D, R, NL * 2))
    flops = sum(2.0 * NT * c[9] * c[10] * c[11] for c in calls)

    def request():
        for a, lda, abs_, b, ldb, bbs, c, ldc, cbs, n, kk, batch in calls:
            if L.irtt_gemm_simt(P(a), 0, lda, abs_, P(b), 0, ldb, bbs, P(c), ldc, cbs, NT, n, kk, batch):
                raise RuntimeError(L.irtt_last_error().decode())

    for _ in range(3):
        request()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        request()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return ms, flops / (ms * 1e-3) / 1e12


def attn_case(steps, which="c3"):
    """Profiling case: the joint attention of one DiT layer, H = 16, hd = 128,
    bf16, through the tcgen05 kernel; `steps` launches timed with CUDA events.
    "c3": the config-3 CFG step (cond row: 750 queries over 750 self + 576
    context keys; uncond row: 750 over 750).  "c4": the config-4 CFG step
    (64 utterances; cond rows over self + text + speaker keys, uncond rows over
    self keys), packed (group, utterance, frame) like the engine.  "c4p" /
    "c3p": the config-4 / config-3 plain step (cond rows only).  "c3f" / "c3w":
    the config-3 CFG step in f32 storage through the register-tiled SIMT
    kernel / the warp-per-query SIMT kernel.  Returns (ms per launch,
    TFLOP/s)."""
    import torch
    L = ctypes.CDLL(str(PKG_DIR / "libirodori_b200_testhooks.so"))
    L.irtt_attention.argtypes = ([ctypes.c_void_p] * 8 + [ctypes.c_int] * 3 + [ctypes.c_void_p] + [ctypes.c_int] * 4)
    L.irtt_last_error.restype = ctypes.c_char_p
    L.irtt_attention_async.argtypes = L.irtt_attention.argtypes
    dev = torch.device("cuda")
    H, hd = 16, 128
    D = H * hd
    if which in ("c4", "c4p"):
        utts = workload()
        lens = [u[1] for u in utts]
        ctxs = [u[0] + u[2] + 1 for u in utts]
    else:
        lens, ctxs = [750], [576]
    uncond = which not in ("c4p", "c3p")
    f32 = which in ("c3f", "c3w")
    dt = torch.float32 if f32 else torch.bfloat16
    path = {"c3f": 2, "c3w": 3}.get(which, 0)
    seqs, tok, co = [], 0, 0
    for S, c in zip(lens, ctxs):  # cond rows
        seqs.append((tok, S, co, c))
        tok, co = tok + S, co + c
    for S in (lens if uncond else []):  # uncond rows
        seqs.append((tok, S, 0, 0))
        tok += S
    rows, C = tok, co
    g = torch.Generator(device=dev).manual_seed(0)
    mk = lambda m: torch.randn(m, D, device=dev, generator=g).to(dt)  # noqa: E731
    q, k, v, ck_, cv = mk(rows), mk(rows), mk(rows), mk(max(C, 128)), mk(max(C, 128))
    gs = torch.sigmoid(torch.randn(rows, D, device=dev, generator=g)).to(dt)
    out = torch.empty(rows, D, device=dev, dtype=dt)
    sd = (ctypes.c_int * (4 * len(seqs)))(*[x for t in seqs for x in t])
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    flops = sum(4 * S * (S + c) * D + (4 * S * S * D if uncond else 0) for S, c in zip(lens, ctxs))

    def launch():
        rc = L.irtt_attention_async(P(q), P(k), P(v), P(gs), P(ck_), P(cv), None, sd, len(seqs), H, hd, P(out),
                                    0 if f32 else 1, rows, max(C, 128), path)
        if rc:
            raise RuntimeError(L.irtt_last_error().decode())

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        launch()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return ms, flops / (ms / 1000.0) / 1e12


def cpu_block_sample(target_s=12.0):
    """Times one DiT block (adaLN, joint attention over [latent | text | speaker]
    keys, SwiGLU) of the CPU oracle at the workload's median utterance size,
    f32, all host threads, repeated for ~target_s seconds.  Returns
    (seconds per block-forward, FLOPs per block-forward, threads, sample text)."""
    import torch
    from oracle import irodori_oracle as O
    import irodori_b200.synth as synth
    torch.set_num_threads(os.cpu_count() or 1)
    utts = workload()
    S = int(statistics.median(u[1] for u in utts))
    T = int(statistics.median(u[0] for u in utts))
    R = int(statistics.median(u[2] for u in utts)) + 1
    cfg = model_cfg()
    cfg1 = dict(cfg, num_layers=1, text_layers=0, speaker_layers=0)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "blk.safetensors")
        synth.make_dit_checkpoint(p, cfg1, seed=4, init="baseline")
        W = O.Weights.load(p)
    D = cfg["model_dim"]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, S, D, generator=g)
    ce = torch.randn(1, 1, 3 * D, generator=g) * 0.1
    cond = O.Cond(torch.randn(1, T, cfg["text_dim"], generator=g), torch.ones(1, T, dtype=torch.bool), "speaker",
                  torch.randn(1, R, cfg["speaker_dim"], generator=g), torch.ones(1, R, dtype=torch.bool))
    kv = O.build_kv_caches(W, cond)
    cos, sin = O.rope_tables(D // cfg["num_heads"], S)

    def block():
        h, gt = O.low_rank_adaln(W, "blocks.0.attention_adaln", x, ce, 1e-5)
        y = x + gt * O.joint_attention(W, "blocks.0.attention", h, kv[0], cos, sin, None)
        h, gt = O.low_rank_adaln(W, "blocks.0.mlp_adaln", y, ce, 1e-5)
        w13 = torch.cat([W["blocks.0.mlp.w1.weight"], W["blocks.0.mlp.w3.weight"]], 0)
        a = h @ w13.T
        F_ = a.shape[-1] // 2
        return y + gt * ((O.silu(a[..., :F_]) * a[..., F_:]) @ W["blocks.0.mlp.w2.weight"].T)

    with torch.no_grad():
        block()
        n, t0 = 0, time.perf_counter()
        while True:
            block()
            n += 1
            el = time.perf_counter() - t0
            if el > target_s or n >= 200:
                break
    per = el / n
    flops = row_forward_flops(S, S + T + R, L=1) - 2 * 2 * D * 32 * S
    sample = (f"{n} forwards of one DiT block (f32 CPU oracle) at the workload's median utterance "
              f"S={S}, text={T}, speaker={R} keys; extrapolated by FLOPs to the 64-utterance job")
    return per, flops, torch.get_num_threads(), sample


def cpu_model():
    """The host CPU's model name and the number of cores this process may use."""
    name = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return name, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def tf32_case(M, reps=5):
    """Profiling case: the fp32 mode's GEMM (tcgen05 kind::tf32 on hi / lo
    operand halves, operands split beforehand) over the four DiT GEMM shapes of
    one layer at M rows -- QKVG (8192 x 2048) and W13 (11776 x 2048) as f32
    stores, Wo (2048 x 2048) and W2 (2048 x 5888) as gated residual updates --
    timed with CUDA events on the launching stream.  Returns (per-layer ms,
    f32-equivalent TFLOP/s = 2MNK / t; the tensor pipe runs 3x that in tf32)."""
    import torch
    L = ctypes.CDLL(str(PKG_DIR / "libirodori_b200_testhooks.so"))
    L.irtt_gemm_tf32x3_async.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 2 + [ctypes.c_int] * 3 + \
        [ctypes.c_void_p] * 2
    L.irtt_last_error.restype = ctypes.c_char_p
    dev = torch.device("cuda")
    D, F = 2048, 5888
    g = torch.Generator(device=dev).manual_seed(0)
    shapes = [(0, 4 * D, D), (2, D, D), (0, 2 * F, D), (2, D, F)]  # (mode, N, K)
    ops = []
    for mode, N, K in shapes:
        a2 = torch.randn(M, 2 * K, device=dev, generator=g)
        b2 = torch.randn(N, 2 * K, device=dev, generator=g) * 0.02
        out = torch.zeros(M, N, device=dev)
        gate = torch.ones(N, device=dev)
        ops.append((mode, a2, b2, N, K, out, gate))
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def layer():
        for mode, a2, b2, N, K, out, gate in ops:
            if L.irtt_gemm_tf32x3_async(mode, P(a2), P(b2), M, N, K, P(out), P(gate)):
                raise RuntimeError(L.irtt_last_error().decode())

    for _ in range(3):
        layer()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        layer()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = sum(2.0 * M * N * K for _, N, K in shapes)
    return ms, flops / (ms / 1000.0) / 1e12


def config1_case(pkg):
    """BASELINE config 1 run end to end, no extrapolation: the reference's
    default ModelConfig (latent 128) with random-init weights (seed 0,
    N(0, 0.02), zero-init adaLN up-projections), batch 1, text 64 ids, speaker
    reference 150 frames ~N(0, 1), 250 target frames (10 s) with initial noise
    seed 1, 4 Euler steps with independent CFG (text 3, speaker 3).  The CPU
    oracle (f32, all host threads) runs the whole sampler -- both condition
    encoders, the context KV caches, 8 DiT row-forwards -- once; the engine
    runs the same request on the GPU (bf16 and f32 modes, CUDA events, best
    of 3 after a warm-up).  Returns the JSON object of the bench line."""
    import torch
    import numpy as np
    from oracle import irodori_oracle as O
    import irodori_b200.synth as synth
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    path = Path(tempfile.gettempdir()) / "irodori_bench" / "dit_default_config1_s0.safetensors"
    if not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        synth.make_dit_checkpoint(str(path), {}, seed=0, init="baseline", dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
    r = synth.make_request({}, 1, 64, 150, 250, seed=1)
    W = O.Weights.load(str(path))
    req = O.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=250,
                            ref_latent=r["ref_latent"], ref_mask=r["ref_mask"], initial_noise=r["initial_noise"])
    op = O.SamplerParams(num_steps=4, guidance=O.GuidanceConfig(mode="independent", scale_text=3.0,
                                                                 scale_speaker=3.0))
    with torch.no_grad():
        t0 = time.perf_counter()
        ref = O.sample_euler_rf_cfg(W, req, op)
        cpu_s = time.perf_counter() - t0
    del W
    audio = 250 / FRAME_RATE
    gpu = {}
    d = {k: v.cuda() for k, v in r.items() if torch.is_tensor(v)}
    out = torch.empty(1, 250, 128, device="cuda")
    for prec in ("bf16", "f32"):
        eng = (pkg.InferenceBuilder(0).load_weights(str(path), precision=prec)
               .with_sampling(pkg.SamplerParams(num_steps=4, guidance=pkg.GuidanceConfig(
                   mode="independent", scale_text=3.0, scale_speaker=3.0))).build())
        rq = pkg.SamplingRequest(sequence_length=250, **d)
        st = torch.cuda.current_stream()
        eng.sample(rq, out=out, stream=st)
        ts = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            eng.sample(rq, out=out, stream=st)
            e1.record(st)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        require_finite(f"config-1 latents ({prec})", out)
        o = out.cpu().numpy().astype(np.float64)
        rv = ref.numpy().astype(np.float64)
        gpu[prec] = {"ms": round(min(ts), 2), "audio_s_per_s": round(audio / (min(ts) / 1000.0), 1),
                     "rel_l2_vs_cpu_oracle": float("%.3e" % (np.linalg.norm(o - rv) / np.linalg.norm(rv)))}
        del eng
    name, cores = cpu_model()
    return {"workload": "config1: default ModelConfig (latent 128), random init seed 0, batch 1, text 64, speaker "
                        "150 frames, 250 target frames (10 s), 4 Euler steps, independent CFG 3/3; whole sampler "
                        "(encoders, KV caches, 8 row-forwards)",
            "cpu_oracle": {"seconds": round(cpu_s, 2), "audio_s_per_s": round(audio / cpu_s, 4), "dtype": "f32",
                           "threads": threads, "cpu_model": name, "cores_available": cores,
                           "kind": "port (CPU restatement of the reference sampler; the Rust crate has no "
                                   "toolchain here)"},
            "gpu_engine": gpu}


def job_flops(utts, min_t=0.5, steps=40):
    """Algorithmic FLOPs of the whole config-4 job (joint CFG: cond row with all
    valid keys, uncond row with the latent keys only, in the CFG window)."""
    import numpy as np
    ts = [np.float32(0.999) * (np.float32(1) - np.float32(i) / np.float32(steps)) for i in range(steps)]
    ncfg = sum(1 for t in ts if np.float32(min_t) <= t <= np.float32(1.0))
    tot = 0.0
    for tl, S, rf, _ in utts:
        cond = row_forward_flops(S, S + tl + rf + 1)
        unc = row_forward_flops(S, S)
        tot += steps * cond + ncfg * unc
    return tot


def config4_dict(audio_total, world):
    """The `config` object of both arms' JSON line (config 4 at N GPUs)."""
    return {"workload": "config4: 64 utterances (text 16-256, 2-30 s, speaker 5-15 s), 40-step Euler, "
                        "joint CFG 3.0, min_t 0.5, ragged batches, LPT bins per rank",
            "utterances": N_UTT, "audio_seconds": round(audio_total, 2), "model_dim": 2048,
            "layers": 24, "latent_dim": 32, "parallelism": f"utterance shards x{world}",
            "l2": "weights (4.6 GB bf16) exceed L2; no flush needed"}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    load_pkg()
    utts = workload()
    audio = sum(u[3] for u in utts)
    total = job_flops(utts)
    vals = []
    for i in range(args.warmup + args.steps):
        per, fl, threads, sample = cpu_block_sample(target_s=4.0)
        if i >= args.warmup:
            vals.append(audio / (per * total / fl))
    v = statistics.median(vals)
    # one step = the whole config-4 job on the host cores (extrapolated from
    # the timed block sample), so ms_per_step * value = audio seconds * 1000
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(audio / v * 1000.0, 1),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config4_dict(audio, args.gpus),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": cpu_model()[0],
                             "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Engine arm
# ---------------------------------------------------------------------------

def require_finite(what, lat, lengths=None):
    """Stop the run (non-zero exit, no JSON line) when sampled latents hold a
    NaN or Inf, or are all zero, in any utterance's valid frames."""
    import torch
    for b in range(lat.shape[0]):
        v = lat[b, :lengths[b]] if lengths is not None else lat[b]
        if not bool(torch.isfinite(v).all()) or not bool((v != 0).any()):
            raise SystemExit(f"bench: {what} of utterance {b} are not finite (or all zero); the run is invalid")


def ensure_checkpoint(path: Path, cfg, rank, world):
    import torch
    import irodori_b200.synth as synth
    if rank == 0 and not path.exists():
        path.parent.mkdir(parents=True, exist_ok=True)
        synth.make_dit_checkpoint(str(path), cfg, seed=4, init="baseline", dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--skip-latency", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-config5", action="store_true")
    ap.add_argument("--codec-only", action="store_true",
                    help="time the config-5 DACVAE decode alone (16 utterances, seeded latents)")
    ap.add_argument("--codec-precision", default="bf16", choices=["bf16", "f32"])
    ap.add_argument("--codec-utts", type=int, default=16,
                    help="with --codec-only: decode the first N of the 16 config-5 utterances (profiling case)")
    ap.add_argument("--attn-case", nargs="?", const="c3", default=None,
                    choices=["c3", "c3p", "c4", "c4p", "c3f", "c3w"],
                    help="only the joint attention of one layer: config-3 CFG step (c3), config-4 CFG step (c4) "
                         "or config-4 plain step (c4p); c3f / c3w: config-3 CFG step in f32 (register-tiled / "
                         "warp-per-query SIMT kernel); --steps launches (profiling case)")
    ap.add_argument("--tf32-case", type=int, default=0,
                    help="only the fp32 mode's tf32 hi / lo GEMM over one DiT layer's four shapes at M rows "
                         "(profiling case)")
    ap.add_argument("--ckpt", default=None)
    ap.add_argument("--row-case", type=int, default=0,
                    help="profiling case: the adaLN modulate row kernel alone at M rows, --steps launches")
    ap.add_argument("--simt-case", action="store_true",
                    help="profiling case: the f32 SIMT GEMMs of one config-3 request's step tables, --steps times")
    ap.add_argument("--shard", type=int, default=0,
                    help="profiling case: time every rank's config-4 bin of an N-way split on this one GPU")
    ap.add_argument("--latency-only", action="store_true",
                    help="only the config-3 single-utterance latency (used for profiling runs)")
    ap.add_argument("--timeline", action="store_true",
                    help="profiling case: kernel timeline (CUPTI activity trace) of one config-4 sample()")
    ap.add_argument("--gemm-case", type=int, default=0,
                    help="only the four DiT GEMMs of one layer at M rows, --steps times (profiling case)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.latency_only:
        return latency_only(args)
    if args.timeline:
        return timeline_case(args)
    if args.shard:
        return shard_case(args)
    if args.row_case:
        load_pkg()
        us, gbs = row_case(args.row_case, args.steps)
        peak = measured_peaks()[1]
        print(json.dumps({"row_case_M": args.row_case, "us_per_launch": round(us, 2), "gbs": round(gbs, 1),
                          "hbm_peak_gbs": peak, "frac": round(gbs / peak, 4)}), flush=True)
        return 0
    if args.simt_case:
        load_pkg()
        ms, tf = simt_case(args.steps)
        print(json.dumps({"simt_case": "config-3 request step tables (41 rows)", "ms_per_request": round(ms, 4),
                          "tflops": round(tf, 2)}), flush=True)
        return 0
    if args.codec_only:
        return codec_only(args)
    if args.attn_case:
        load_pkg()
        ms, tf = attn_case(args.steps, args.attn_case)
        print(json.dumps({"attn_case": args.attn_case, "attn_case_ms": round(ms, 4), "tflops": round(tf, 1)}),
              flush=True)
        return 0
    if args.tf32_case:
        load_pkg()
        ms, tf = tf32_case(args.tf32_case, reps=args.steps)
        print(json.dumps({"tf32_case_M": args.tf32_case, "ms_per_layer": round(ms, 4),
                          "f32_equiv_tflops": round(tf, 1), "tf32_pipe_tflops": round(3 * tf, 1)}), flush=True)
        return 0
    if args.gemm_case:
        import torch
        load_pkg()
        achieved, ms, flops = gemm_roofline(args.gemm_case, reps=args.steps)
        print(json.dumps({"gemm_case_M": args.gemm_case, "achieved_tflops": round(achieved, 1),
                          "ms_per_layer": round(ms, 4), "gflop_per_layer": round(flops / 1e9, 2),
                          **gemm_roofline.last_parts}), flush=True)
        return 0

    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    pkg = load_pkg()
    from irodori_b200 import sharding
    if world > 1:
        # keep stdout to the one JSON line (NCCL prints its version at INFO level)
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        # a rank that dies makes the others' next collective fail within this
        # timeout (checkpoint generation on rank 0 happens before the first one)
        dist = sharding.init_rank_group("nccl", 300, device=torch.device("cuda", local))
    cfg = model_cfg()
    ckpt = Path(args.ckpt) if args.ckpt else Path(tempfile.gettempdir()) / "irodori_bench" / "dit_default_l32_s4.safetensors"
    ensure_checkpoint(ckpt, cfg, rank, world)
    params = pkg.SamplerParams(num_steps=40, method="euler",
                               guidance=pkg.GuidanceConfig(mode="joint", scale_text=3.0, scale_speaker=3.0))
    eng = pkg.InferenceBuilder(local).load_weights(str(ckpt), precision="bf16").with_sampling(params).build()

    utts = workload()
    costs = [sharding.utterance_cost(S, tl, rf) for tl, S, rf, _ in utts]
    mine = sharding.shard_for_rank(costs, rank, world)
    audio_total = sum(u[3] for u in utts)
    P = cfg["latent_dim"]
    batch = build_batch(utts, mine, P, cfg["text_vocab_size"])
    keys = ("text_ids", "text_mask", "ref_latent", "ref_mask", "initial_noise")
    dev_in = {k: batch[k].cuda() for k in keys}
    host_in = {k: batch[k].numpy() for k in keys}
    B, Sm = len(mine), batch["sequence_length"]
    out_dev = torch.empty(B, Sm, P, device="cuda")
    stream = torch.cuda.Stream()

    def req(src):
        return pkg.SamplingRequest(sequence_length=Sm, sequence_lengths=batch["sequence_lengths"], **src)

    def timed(src, out, k):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        launches = 0
        for _ in range(k):
            eng.sample(req(src), out=out, stream=stream)
            launches += eng.last_stats()[1]
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if dist is not None:
            ms = sharding.max_over_ranks(dist, ms, device="cuda")
        return ms, launches

    for _ in range(args.warmup):
        eng.sample(req(dev_in), out=out_dev, stream=stream)
    torch.cuda.synchronize()
    require_finite("warm-up latents", out_dev, batch["sequence_lengths"])
    with ClockSampler(local) as clk:
        ms, launches = timed(dev_in, out_dev, args.steps)
    require_finite("timed latents", out_dev, batch["sequence_lengths"])
    clocks = clk.summary()
    ms_step = ms / args.steps
    value = audio_total * args.steps / (ms / 1000.0)

    # end to end through the public API with host buffers
    import numpy as np
    out_host = np.empty((B, Sm, P), dtype=np.float32)
    e2e_ms, _ = timed(host_in, out_host, args.steps)
    require_finite("e2e latents", torch.from_numpy(out_host), batch["sequence_lengths"])
    h2d = sum(v.nbytes for v in host_in.values()) + 4 * B
    d2h = out_host.nbytes
    e2e_value = audio_total * args.steps / (e2e_ms / 1000.0)

    c5 = None
    if not args.skip_config5:
        c5 = config5(pkg, eng, cfg, stream, rank, world, dist, max(1, min(args.steps, 3)), 1)

    if rank != 0:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # dominant kernel: tcgen05 GEMM on this workload's shapes (CFG step, rank-0 bin)
    ntok = sum(utts[i][1] for i in mine)
    peak, hbm, peak_kind = measured_peaks()
    with ClockSampler(local) as gclk:
        burst, gemm_ms, gemm_flops = gemm_roofline(2 * ntok, sustain_s=3.0)
    achieved, gemm_ms_s, gemm_n = gemm_roofline.sustained
    sust = measured_sustained()
    peak_s = sust or peak
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_s, "unit": "TFLOP/s",
            "frac": round(achieved / peak_s, 4),
            "traffic": round(GEMM_LAYER_TRAFFIC_PER_ROW * 2 * ntok),
            "traffic_unit": "DRAM bytes per layer (the 4 launches achieved is quoted on)",
            "algorithmic_bytes": gemm_layer_bytes(2 * ntok),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, 4 launches at M=54504, scaled by M",
            "kernel": "gemm_kernel<256> (tcgen05), 4 DiT GEMMs of one layer at M=%d" % (2 * ntok),
            "peak_kind": ("%s sustained bf16" % peak_kind) if sust else ("%s burst bf16" % peak_kind),
            "timing": "CUDA events over %d back-to-back layers (%.1f s) after 1.5 s at the same load, as inside "
                      "a long sampling step" % (gemm_n, gemm_n * gemm_ms_s / 1000.0),
            "clocks": gclk.summary(),
            "burst": {"achieved": round(burst, 1), "peak": peak, "frac": round(burst / peak, 4),
                      "timing": "5 layers right after the warm-up"}}
    total_flops = job_flops(utts)
    extra = {"job_tflop": round(total_flops / 1e12, 2),
             "job_tflops_achieved": round(total_flops * args.steps / (ms / 1000.0) / 1e12, 1)}

    lat = None
    if world == 1 and not args.skip_latency:
        lat = latency_config3(pkg, eng, cfg, stream)

    cpu = None
    c1 = None
    if world == 1 and not args.skip_cpu:
        per, fl, threads, sample = cpu_block_sample()
        name, _ = cpu_model()
        cpu = {"value": audio_total / (per * total_flops / fl), "unit": UNIT, "cores": threads, "kind": "port",
               "cpu_model": name, "sample": sample}
        c1 = config1_case(pkg)

    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights and inputs)",
            "config": config4_dict(audio_total, world),
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": int(launches), "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
            "latency_config3": lat, "config5": c5, "config1": c1, **extra}
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


CODEC_CH = (1536, 768, 384, 192, 96)
CODEC_RATES = (12, 10, 8, 2)


def codec_flops_per_frame():
    """Algorithmic FLOPs of the DACVAE decoder per latent frame: quantizer
    out_proj, stem conv, per block the ConvTranspose (2 taps per output
    sample) and 3 residual units (k7 conv + 1x1 conv), head conv."""
    f = 2 * 32 * 1024 + 2 * 1024 * CODEC_CH[0] * 7
    scale = 1
    for i, s in enumerate(CODEC_RATES):
        cin, cout = CODEC_CH[i], CODEC_CH[i + 1]
        scale *= s
        f += scale * (2 * 2 * cin * cout + 3 * (2 * 7 * cout * cout + 2 * cout * cout))
    return f + scale * 2 * 7 * CODEC_CH[-1]


def config5(pkg, eng, cfg, stream, rank, world, dist, steps, warmup):
    """Config 5: config-4-style utterances (seed 5), 16 per GPU, sampled and
    decoded to 48 kHz waveforms by the bf16 tensor-core DACVAE decoder
    (reference-default random init).  Returns whole-job audio-s/s for
    text -> waveform and for the decode alone (max over ranks)."""
    import torch
    import irodori_b200.synth as synth
    utts = synth.throughput_utterances(16 * world, seed=5)
    mine = list(range(16 * rank, 16 * rank + 16))
    P = cfg["latent_dim"]
    batch = build_batch(utts, mine, P, cfg["text_vocab_size"], seed=5)
    keys = ("text_ids", "text_mask", "ref_latent", "ref_mask", "initial_noise")
    dev_in = {k: batch[k].cuda() for k in keys}
    B, Sm, lens = len(mine), batch["sequence_length"], batch["sequence_lengths"]
    path = Path(tempfile.gettempdir()) / "irodori_bench" / f"codec_ref_init_r{rank}.safetensors"
    path.parent.mkdir(parents=True, exist_ok=True)
    if not path.exists():
        synth.make_codec_checkpoint(str(path), seed=5, width_div=1, init="reference")
    codec = pkg.load_codec(str(path), device=torch.cuda.current_device(), precision="bf16")
    hop = codec.hop_length()
    lat = torch.empty(B, Sm, P, device="cuda")
    wav = torch.empty(B, 1, Sm * hop, device="cuda")
    req = pkg.SamplingRequest(sequence_length=Sm, sequence_lengths=lens, **dev_in)

    def step(decode_only):
        if not decode_only:
            eng.sample(req, out=lat, stream=stream)
        codec.decode(lat, out=wav, stream=stream, lengths=lens)

    def timed(decode_only, k):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            step(decode_only)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / k
        if dist is not None:
            from irodori_b200 import sharding
            ms = sharding.max_over_ranks(dist, ms, device="cuda")
        return ms

    for _ in range(warmup):
        step(False)
    torch.cuda.synchronize()
    require_finite("config-5 latents", lat, lens)
    if not bool(torch.isfinite(wav).all()):
        raise SystemExit("bench: config-5 waveform is not finite; the run is invalid")
    ms_t2w = timed(False, steps)
    ms_dec = timed(True, steps)
    audio_job = sum(u[3] for u in utts)
    frames_rank = sum(lens)
    dflops = codec_flops_per_frame() * frames_rank
    return {"workload": "config5: 16 utterances per GPU (config-4 distribution, seed 5), sample + DACVAE decode, "
                        "bf16, reference-default random codec init",
            "scaling": "weak", "utterances": 16 * world, "audio_seconds": round(audio_job, 2),
            "text_to_wave_audio_s_per_s": round(audio_job / (ms_t2w / 1000.0), 3),
            "ms_per_step": round(ms_t2w, 2),
            "decode_audio_s_per_s": round(audio_job / (ms_dec / 1000.0), 3), "decode_ms": round(ms_dec, 3),
            "decode_tflops_rank0": round(dflops / (ms_dec / 1000.0) / 1e12, 1),
            "decode_gflop_per_latent_frame": round(codec_flops_per_frame() / 1e9, 3)}


def codec_only(args):
    """Config-5 decode alone: the 16 utterance lengths of config 5 (rank 0,
    seed 5) with N(0, 1) latents, bf16 tensor-core DACVAE decoder; prints one
    JSON line (device buffers, CUDA-event time per decode)."""
    import torch
    pkg = load_pkg()
    import irodori_b200.synth as synth
    utts = synth.throughput_utterances(16, seed=5)[:max(1, args.codec_utts)]
    lens = [u[1] for u in utts]
    T = max(lens)
    path = Path(tempfile.gettempdir()) / "irodori_bench" / "codec_ref_init_r0.safetensors"
    path.parent.mkdir(parents=True, exist_ok=True)
    if not path.exists():
        synth.make_codec_checkpoint(str(path), seed=5, width_div=1, init="reference")
    codec = pkg.load_codec(str(path), device=0, precision=args.codec_precision)
    lat = torch.randn(len(lens), T, 32, generator=torch.Generator().manual_seed(5)).cuda()
    wav = torch.empty(len(lens), 1, T * codec.hop_length(), device="cuda")
    for _ in range(args.warmup):
        codec.decode(lat, out=wav, lengths=lens)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        codec.decode(lat, out=wav, lengths=lens)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    frames = sum(lens)
    print(json.dumps({"codec_decode_ms": round(ms, 3), "precision": args.codec_precision, "frames": frames,
                      "audio_s_per_s": round(frames / FRAME_RATE / (ms / 1000.0), 1),
                      "tflops": round(codec_flops_per_frame() * frames / (ms / 1000.0) / 1e12, 1)}), flush=True)
    return 0


def shard_case(args):
    """Profiling case for multi-GPU scaling on one GPU: every rank's bin of an
    N-way split of config 4 (LPT bins on the cost model, exactly as the N-GPU
    bench assigns them) sampled in turn on this GPU, W warm-up and K timed
    steps each.  Ranks share nothing on the data path, so a bin's time here is
    that rank's step time in the N-GPU run, and the N-GPU throughput is the
    job's audio over the slowest bin's time."""
    import torch
    n = int(args.shard)
    pkg = load_pkg()
    from irodori_b200 import sharding
    cfg = model_cfg()
    ckpt = Path(args.ckpt) if args.ckpt else Path(tempfile.gettempdir()) / "irodori_bench" / "dit_default_l32_s4.safetensors"
    ensure_checkpoint(ckpt, cfg, 0, 1)
    params = pkg.SamplerParams(num_steps=40, method="euler",
                               guidance=pkg.GuidanceConfig(mode="joint", scale_text=3.0, scale_speaker=3.0))
    eng = pkg.InferenceBuilder(0).load_weights(str(ckpt), precision="bf16").with_sampling(params).build()
    utts = workload()
    costs = [sharding.utterance_cost(S, tl, rf) for tl, S, rf, _ in utts]
    audio_total = sum(u[3] for u in utts)
    P = cfg["latent_dim"]
    stream = torch.cuda.Stream()
    bins = []
    for r in range(n):
        mine = sharding.shard_for_rank(costs, r, n)
        batch = build_batch(utts, mine, P, cfg["text_vocab_size"])
        keys = ("text_ids", "text_mask", "ref_latent", "ref_mask", "initial_noise")
        dev_in = {k: batch[k].cuda() for k in keys}
        out = torch.empty(len(mine), batch["sequence_length"], P, device="cuda")
        rq = pkg.SamplingRequest(sequence_length=batch["sequence_length"], sequence_lengths=batch["sequence_lengths"],
                                 **dev_in)
        for _ in range(args.warmup):
            eng.sample(rq, out=out, stream=stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            eng.sample(rq, out=out, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        bins.append({"rank": r, "utterances": len(mine), "latent_frames": sum(utts[i][1] for i in mine),
                     "audio_seconds": round(sum(utts[i][3] for i in mine), 2), "ms_per_step": round(ms, 2)})
    worst = max(b["ms_per_step"] for b in bins)
    print(json.dumps({"shard_case": n, "bins": bins, "slowest_ms": worst,
                      "projected_value": round(audio_total / (worst / 1000.0), 3), "unit": UNIT}), flush=True)
    return 0


def timeline_case(args):
    """Kernel timeline of one config-4 sample() on rank 0's bin at N=1: the
    engine built as in the bench, `--warmup` untraced samples, then one
    sample under CUDA activity tracing (torch.profiler, CUDA activities only:
    CUPTI kernel start/end timestamps, no replay or serialisation).  Prints
    one JSON line: span, GPU-busy time (union of kernel and copy intervals),
    idle time, and per kernel name its launches, total and average duration
    and share of the summed durations."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    pkg = load_pkg()
    from irodori_b200 import sharding
    cfg = model_cfg()
    ckpt = Path(args.ckpt) if args.ckpt else Path(tempfile.gettempdir()) / "irodori_bench" / "dit_default_l32_s4.safetensors"
    ensure_checkpoint(ckpt, cfg, 0, 1)
    params = pkg.SamplerParams(num_steps=40, method="euler",
                               guidance=pkg.GuidanceConfig(mode="joint", scale_text=3.0, scale_speaker=3.0))
    eng = pkg.InferenceBuilder(0).load_weights(str(ckpt), precision="bf16").with_sampling(params).build()
    utts = workload()
    costs = [sharding.utterance_cost(S, tl, rf) for tl, S, rf, _ in utts]
    mine = sharding.shard_for_rank(costs, 0, 1)
    batch = build_batch(utts, mine, cfg["latent_dim"], cfg["text_vocab_size"])
    keys = ("text_ids", "text_mask", "ref_latent", "ref_mask", "initial_noise")
    dev_in = {k: batch[k].cuda() for k in keys}
    out = torch.empty(len(mine), batch["sequence_length"], cfg["latent_dim"], device="cuda")
    stream = torch.cuda.Stream()
    rq = pkg.SamplingRequest(sequence_length=batch["sequence_length"], sequence_lengths=batch["sequence_lengths"],
                             **dev_in)
    for _ in range(max(1, args.warmup)):
        eng.sample(rq, out=out, stream=stream)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        eng.sample(rq, out=out, stream=stream)
        torch.cuda.synchronize()
    require_finite("timeline latents", out, batch["sequence_lengths"])
    with tempfile.TemporaryDirectory() as d:
        fn = os.path.join(d, "trace.json")
        prof.export_chrome_trace(fn)
        ev = json.load(open(fn))["traceEvents"]
    kern = [e for e in ev if e.get("cat") == "kernel" and "dur" in e]
    busy_ev = [e for e in ev if e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset") and "dur" in e]
    iv = sorted((float(e["ts"]), float(e["ts"]) + float(e["dur"])) for e in busy_ev)
    busy, cur_s, cur_e = 0.0, None, None
    for a, b in iv:
        if cur_e is None or a > cur_e:
            if cur_e is not None:
                busy += cur_e - cur_s
            cur_s, cur_e = a, b
        else:
            cur_e = max(cur_e, b)
    if cur_e is not None:
        busy += cur_e - cur_s
    span = (iv[-1][1] - iv[0][0]) if iv else 0.0
    per = {}
    for e in kern:
        n = e["name"].replace("(anonymous namespace)", "").split("(")[0]
        c, t = per.get(n, (0, 0.0))
        per[n] = (c + 1, t + float(e["dur"]))
    total = sum(t for _, t in per.values())
    rows = sorted(per.items(), key=lambda kv: -kv[1][1])
    print(json.dumps({"timeline": "config4 rank-0 bin at N=1, one sample()", "span_ms": round(span / 1e3, 1),
                      "busy_ms": round(busy / 1e3, 1), "idle_ms": round((span - busy) / 1e3, 2),
                      "kernel_sum_ms": round(total / 1e3, 1),
                      "kernels": [{"name": n, "launches": c, "total_ms": round(t / 1e3, 2),
                                   "avg_us": round(t / c, 1), "share": round(t / total, 4)} for n, (c, t) in rows]}),
          flush=True)
    return 0


def latency_only(args):
    """Config-3 latency alone: one checkpoint load, `--warmup` untimed and
    `--steps` timed sample() calls for the default CFG window."""
    import torch
    pkg = load_pkg()
    cfg = model_cfg()
    ckpt = Path(args.ckpt) if args.ckpt else Path(tempfile.gettempdir()) / "irodori_bench" / "dit_default_l32_s4.safetensors"
    ensure_checkpoint(ckpt, cfg, 0, 1)
    params = pkg.SamplerParams(num_steps=40, guidance=pkg.GuidanceConfig(mode="joint", scale_text=3.0,
                                                                         scale_speaker=3.0))
    eng = pkg.InferenceBuilder(0).load_weights(str(ckpt), precision="bf16").with_sampling(params).build()
    import irodori_b200.synth as synth
    r = synth.make_request(cfg, 1, 200, 375, 750, seed=3)
    d = {k: v.cuda() for k, v in r.items() if torch.is_tensor(v)}
    out = torch.empty(1, 750, cfg["latent_dim"], device="cuda")
    rq = pkg.SamplingRequest(sequence_length=750, **d)
    st = torch.cuda.current_stream()
    for _ in range(args.warmup):
        eng.sample(rq, out=out, stream=st)
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        eng.sample(rq, out=out, stream=st)
        e1.record(st)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    rows, launches = eng.last_stats()
    print(json.dumps({"latency_ms": ts, "row_forwards": rows, "kernel_launches": launches}), flush=True)
    return 0


def latency_config3(pkg, eng, cfg, stream, reps=3):
    """Config 3: one 30 s utterance (750 frames), text 200, speaker 375 frames,
    40 steps joint CFG 3.0; device-timed ms per sample() for the default
    window (min_t 0.5: 20 CFG + 20 plain steps) and min_t = 0 (40 CFG steps)."""
    import torch
    import irodori_b200.synth as synth
    r = synth.make_request(cfg, 1, 200, 375, 750, seed=3)
    d = {k: v.cuda() for k, v in r.items() if torch.is_tensor(v)}
    out = torch.empty(1, 750, cfg["latent_dim"], device="cuda")
    res = {}
    keep = eng.sampling_params()
    for name, mt in (("ms_min_t_0.5", 0.5), ("ms_min_t_0", 0.0)):
        eng.with_sampling(pkg.SamplerParams(num_steps=40, guidance=pkg.GuidanceConfig(
            mode="joint", scale_text=3.0, scale_speaker=3.0, min_t=mt)))
        rq = pkg.SamplingRequest(sequence_length=750, **d)
        eng.sample(rq, out=out, stream=stream)
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            eng.sample(rq, out=out, stream=stream)
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        require_finite(f"config-3 latents ({name})", out)
        res[name] = round(min(ts), 2)
    eng.with_sampling(keep)
    res["row_forwards_min_t_0.5"] = 60
    res["row_forwards_min_t_0"] = 80
    return res


if __name__ == "__main__":
    sys.exit(main())
