"""Kernel-level tests of the implicit-GEMM tcgen05 convolution used by the
bf16 DACVAE decoder (conv_tc.cu), through the test-hook library, against a
plain PyTorch fp32 reference on the same bf16-rounded operands.

Each case is one decoder layer shape: 1x1 (quantizer out_proj and the
residual units' second conv, with the residual add), kernel 7 with dilation
1/3/9, and ConvTranspose1d with stride 2/8/10/12 (polyphase), on a time axis
with zero gap frames and a ragged row tail."""

import ctypes

import pytest

from test_gpu_kernels import check, dev, hooks, ptr  # noqa: F401  (fixtures)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

_sig_done = False


def conv_hook():
    global _sig_done
    L = hooks()
    if not _sig_done:
        L.irtt_conv_tc.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
                                   + [ctypes.c_int] * 10 + [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_void_p])
        _sig_done = True
    return L


def snake(v, a):
    return v + torch.sin(a * v) ** 2 / (a + 1e-9)


def shifted(x, off):
    out = torch.zeros_like(x)
    R = x.shape[0]
    lo, hi = max(0, -off), min(R, R - off)
    if hi > lo:
        out[lo:hi] = x[lo + off:hi + off]
    return out


def reference(xin, w, bias, k, dil, pad, convt, s, scale, fs, alpha, X, add_res):
    """Same contract as conv_tc: conv weight [cout, cin, k] or ConvTranspose
    weight [cin, cout, 2s]; returns (f32 rows, bf16 rows)."""
    R = xin.shape[0]
    if not convt:
        vals = sum(shifted(xin, t * dil - pad) @ w[:, :, t].T for t in range(k))
        Rout = R
    else:
        Rout = R * s
        vals = torch.zeros(Rout, w.shape[1], device=xin.device)
        q = torch.arange(R, device=xin.device)
        for ph in range(s):
            qoff = 1 if ph < pad else 0
            acc = shifted(xin, qoff) @ w[:, :, ph] + shifted(xin, qoff - 1) @ w[:, :, ph + s]
            vals[(q + qoff) * s + ph - pad] = acc
    v = vals + bias
    if add_res:
        v = v + X
    valid = (fs[torch.arange(Rout, device=xin.device) // scale] >= 0).float()[:, None]
    v = v * valid
    pv = snake(v, alpha) if alpha is not None else v
    return v, pv


def pack(w, convt, s, cin_pad):
    if not convt:  # [cout, cin, k] -> [cout][k][cin_pad]
        cout, cin, k = w.shape
        out = torch.zeros(cout, k, cin_pad, device=w.device)
        out[:, :, :cin] = w.permute(0, 2, 1)
        return out.to(torch.bfloat16).contiguous()
    cin, cout, _ = w.shape  # [cin, cout, 2s] -> [s][cout][2][cin_pad]
    out = torch.zeros(s, cout, 2, cin_pad, device=w.device)
    for r in range(s):
        out[r, :, 0, :cin] = w[:, :, r].T
        out[r, :, 1, :cin] = w[:, :, r + s].T
    return out.to(torch.bfloat16).contiguous()


# (name, frames, scale, cin, cout, k, dil, convt, stride, add_res, snake)
CASES = [
    ("qout_1x1", 150, 1, 64, 256, 1, 1, 0, 1, 0, False),
    ("stem_k7", 140, 1, 1024, 1536, 7, 1, 0, 1, 0, True),
    ("res_k7_d9_c96", 10, 120, 96, 96, 7, 9, 0, 1, 0, True),
    ("res_k7_d3_c192", 20, 12, 192, 192, 7, 3, 0, 1, 0, True),
    ("res_1x1_resid_c384", 30, 10, 384, 384, 1, 1, 0, 1, 1, True),
    ("res_1x1_resid_c96", 40, 8, 96, 96, 1, 1, 0, 1, 1, True),
    ("convt_s2", 300, 1, 192, 96, 4, 1, 1, 2, 0, True),
    ("convt_s3_odd", 200, 1, 192, 96, 6, 1, 1, 3, 0, True),  # odd stride: phase -> row map
    ("convt_s8", 200, 1, 384, 192, 16, 1, 1, 8, 0, True),
    ("convt_s10", 150, 1, 768, 384, 20, 1, 1, 10, 0, True),
    ("convt_s12", 131, 1, 1536, 768, 24, 1, 1, 12, 0, True),
    # more tiles than SMs: every CTA runs several tiles (both TMEM accumulators)
    ("many_1x1_resid_c96", 400, 60, 96, 96, 1, 1, 0, 1, 1, True),
    ("many_k7_d9_c192", 100, 240, 192, 192, 7, 9, 0, 1, 0, True),
    ("many_convt_s10", 2000, 1, 768, 384, 20, 1, 1, 10, 0, True),
    ("many_k7_c768", 40, 480, 768, 768, 7, 1, 0, 1, 0, True),
    # <= 128 output channels, k > 1: the transposed product (conv_t_kernel)
    ("many_k7_d9_c96_transposed", 200, 500, 96, 96, 7, 9, 0, 1, 0, True),  # several 256-row units per CTA
    ("k7_d1_c64_transposed", 50, 30, 64, 64, 7, 1, 0, 1, 0, True),        # half the channel lanes idle
    ("k7_d3_c96_plain_tail", 40, 37, 96, 96, 7, 3, 0, 1, 0, False),       # no Snake, rows % 256 != 0
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_conv_tc_layer(dev, case):  # noqa: F811
    name, frames, scale, cin, cout, k, dil, convt, s, add_res, use_snake = case
    g = torch.Generator(device="cpu").manual_seed(sum(map(ord, name)))
    R = frames * scale  # input rows
    scale_out = scale * s if convt else scale
    F = frames
    fs = torch.arange(F, dtype=torch.int32)
    fs[:3] = -1  # gap frames at the start, in the middle and at the end
    fs[F // 2:F // 2 + 3] = -1
    fs[-3:] = -1
    fs = fs.to(dev)
    # inputs are zero on gap rows, as the producer layer writes them
    row_valid = (fs[torch.arange(R, device=dev) // scale] >= 0).float()[:, None]
    xin = (torch.randn(R, cin, generator=g).to(dev) * row_valid).to(torch.bfloat16)
    if convt:
        w = (torch.randn(cin, cout, 2 * s, generator=g) / (2 * cin) ** 0.5).to(dev)
        pad = (s + 1) // 2
        taps, phases = 2, s
    else:
        w = (torch.randn(cout, cin, k, generator=g) / (k * cin) ** 0.5).to(dev)
        pad = (k - 1) * dil // 2
        taps, phases = k, 1
    cin_pad = (cin + 63) // 64 * 64
    wp = pack(w, convt, s, cin_pad)
    wr = wp.float()  # bf16-rounded weights back in the reference layout
    if convt:
        w_ref = torch.empty_like(w)
        for r in range(s):
            w_ref[:, :, r] = wr[r, :, 0, :cin].T
            w_ref[:, :, r + s] = wr[r, :, 1, :cin].T
    else:
        w_ref = wr[:, :, :cin].permute(0, 2, 1).contiguous()
    bias = (0.1 * torch.randn(cout, generator=g)).to(dev)
    alpha = (1.0 + 0.2 * torch.rand(cout, generator=g)).to(dev) if use_snake else None
    Rout = R * s if convt else R
    X = torch.randn(Rout, cout, generator=g).to(dev) if add_res else torch.full((Rout, cout), float("nan"), device=dev)
    X0 = X.clone()
    P = torch.full((Rout, cout), float("nan"), device=dev).to(torch.bfloat16)
    rc = conv_hook().irtt_conv_tc(ptr(xin), R, cin, ptr(wp), cin_pad, taps, phases, cout, dil, pad, convt, s, Rout,
                                  scale_out, ptr(fs), ptr(bias), ptr(alpha), ptr(X), add_res, ptr(P))
    check(rc)
    ref_x, ref_p = reference(xin.float(), w_ref, bias, k, dil, pad, convt, s, scale_out, fs, alpha, X0, add_res)
    assert torch.isfinite(X).all() and torch.isfinite(P.float()).all()
    ex = ((X - ref_x).norm() / ref_x.norm()).item()
    ep = ((P.float() - ref_p).norm() / ref_p.norm()).item()
    assert ex < 1e-4, (name, ex)      # f32 rows: summation order only
    assert ep < 8e-3, (name, ep)      # bf16 rows: one rounding of the output
    gap_rows = fs[torch.arange(Rout, device=dev) // scale_out] < 0
    assert (X[gap_rows] == 0).all() and (P[gap_rows].float() == 0).all()


def test_codec_tc_pipeline_layerwise(dev, oracle, synth, tmp_path):  # noqa: F811
    """The whole bf16 decoder driven layer by layer through the kernel hook
    (same gap layout and buffer roles as the engine): every layer against the
    fp32 reference of that layer on the same inputs, the waveform against the
    oracle."""
    p = tmp_path / "codec_full.safetensors"
    synth.make_codec_checkpoint(str(p), seed=5, width_div=1, init="reference")
    W = oracle.load_codec(str(p))
    t = {k: v.to(dev) for k, v in W.t.items()}
    B, T, GAP = 2, 6, 3
    lat = torch.randn(B, T, 32, generator=torch.Generator().manual_seed(7))
    ref_wav = oracle.codec_decode(W, lat)
    fs = [-1] * GAP
    for b in range(B):
        fs += [b * T + i for i in range(T)] + [-1] * GAP
    fs += [-1] * max(0, 128 - len(fs))
    F = len(fs)
    fs_t = torch.tensor(fs, dtype=torch.int32, device=dev)
    cur = torch.zeros(F, 64, device=dev)
    for f, src in enumerate(fs):
        if src >= 0:
            cur[f, :32] = lat.reshape(-1, 32)[src].to(dev)
    cur = cur.to(torch.bfloat16)
    X = None

    def layer(name, w, bias, k, dil, convt, s, scale, alpha, add_res, keeps_x=False):
        """keeps_x: the layer emits only bf16 rows and leaves the f32
        residual stream alone (the product passes x = nullptr)."""
        nonlocal cur, X
        R, cin = cur.shape
        cin_pad = (cin + 63) // 64 * 64
        if convt:
            pad, taps, phases, cout = (s + 1) // 2, 2, s, w.shape[1]
        else:
            pad, taps, phases, cout = (k - 1) * dil // 2, k, 1, w.shape[0]
            if w.shape[1] < cin:  # quantizer out_proj: 32 latent channels in 64 columns
                w = torch.cat([w, torch.zeros(cout, cin - w.shape[1], k, device=dev)], 1)
        wp = pack(w, convt, s, cin_pad)
        Rout = R * s if convt else R
        out_scale = scale * s if convt else scale
        x_in = X.clone() if add_res else None
        Xo = X if add_res else torch.full((Rout, cout), float("nan"), device=dev)
        P = torch.empty(Rout, cout, device=dev, dtype=torch.bfloat16)
        rc = conv_hook().irtt_conv_tc(ptr(cur), R, cin, ptr(wp), cin_pad, taps, phases, cout, dil, pad, convt, s,
                                      Rout, out_scale, ptr(fs_t), ptr(bias), ptr(alpha), ptr(Xo), add_res, ptr(P))
        check(rc)
        w_ref = w.to(torch.bfloat16).float()
        rx, rp = reference(cur.float(), w_ref, bias, k, dil, pad, convt, s, out_scale, fs_t, alpha, x_in, add_res)
        ex = ((Xo - rx).norm() / rx.norm()).item()
        ep = ((P.float() - rp).norm() / rp.norm()).item()
        assert ex < 1e-4 and ep < 8e-3, (name, ex, ep)
        cur = P
        if not keeps_x:
            X = Xo
        return out_scale

    a = lambda key: t[key].reshape(-1)  # noqa: E731
    layer("qout", t["quantizer.out_proj.weight"], t["quantizer.out_proj.bias"], 1, 1, 0, 1, 1, None, 0)
    layer("stem", t["decoder.model.0.weight"], t["decoder.model.0.bias"], 7, 1, 0, 1, 1,
          a("decoder.model.1.block.0.alpha"), 0)
    scale = 1
    for i, s in enumerate((12, 10, 8, 2)):
        pre = f"decoder.model.{i + 1}"
        scale = layer(f"{pre}.ct", t[f"{pre}.block.1.weight"], t[f"{pre}.block.1.bias"], 2 * s, 1, 1, s, scale,
                      a(f"{pre}.block.4.block.0.alpha"), 0)
        for r, (j, d) in enumerate(zip((4, 5, 8), (1, 3, 9))):
            q = f"{pre}.block.{j}"
            layer(f"{q}.c1", t[f"{q}.block.1.weight"], t[f"{q}.block.1.bias"], 7, d, 0, 1, scale,
                  a(f"{q}.block.2.alpha"), 0, keeps_x=True)
            if r < 2:
                nxt = a(f"{pre}.block.{(4, 5, 8)[r + 1]}.block.0.alpha")
            elif i < 3:
                nxt = a(f"decoder.model.{i + 2}.block.0.alpha")
            else:
                nxt = a("decoder.wm_model.encoder_block.pre.0.alpha")
            layer(f"{q}.c3", t[f"{q}.block.3.weight"], t[f"{q}.block.3.bias"], 1, 1, 0, 1, scale, nxt, 1)
    y = torch.nn.functional.conv1d(torch.nn.functional.pad(cur.float().T[None], (3, 3)),
                                   t["decoder.wm_model.encoder_block.pre.1.weight"],
                                   t["decoder.wm_model.encoder_block.pre.1.bias"])[0, 0]
    o = torch.arange(cur.shape[0], device=dev)
    src = fs_t.long()[o // 1920]
    wav = torch.zeros(B * T * 1920, device=dev)
    wav[src[src >= 0] * 1920 + o[src >= 0] % 1920] = torch.tanh(y[src >= 0])
    err = ((wav.cpu().reshape(B, 1, -1) - ref_wav).norm() / ref_wav.norm()).item()
    print(f"layerwise bf16 pipeline vs oracle: rel L2 {err:.3e}")
    assert err < 1e-2, err
