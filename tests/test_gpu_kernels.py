"""Kernel-level GPU tests: each CUDA kernel against a plain PyTorch fp32
reference of the same op (through the test-hook library, not the product ABI)."""

import ctypes
import math

import pytest

from conftest import PKG_DIR

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

_hooks = None


def hooks():
    global _hooks
    if _hooks is None:
        p = PKG_DIR / "libirodori_b200_testhooks.so"
        if not p.exists():
            pytest.fail(f"{p} missing: run __graft_entry__.build()")
        L = ctypes.CDLL(str(p))
        L.irtt_last_error.restype = ctypes.c_char_p
        L.irtt_gemm_store.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 3 + [ctypes.c_void_p, ctypes.c_int]
        L.irtt_gemm_epi.argtypes = ([ctypes.c_int] + [ctypes.c_void_p] * 2 + [ctypes.c_int] * 4 + [ctypes.c_void_p] * 9
                                    + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 2 + [ctypes.c_int])
        L.irtt_attention.argtypes = ([ctypes.c_void_p] * 8 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
                                     + [ctypes.c_int] * 4)
        _hooks = L
    return _hooks


def check(rc):
    assert rc == 0, hooks().irtt_last_error().decode()
    rc = hooks().irtt_sync_check()  # kernels are asynchronous; sync + watchdog flag
    assert rc == 0, hooks().irtt_last_error().decode()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return torch.device("cuda:0")


GEMM_SHAPES = [
    (128, 256, 64),      # single tile
    (300, 384, 736),     # M, N tails + K tail (736 = 11.5 x 64)
    (1500, 2048, 2048),  # DiT Wo shape at the CFG batch
    (1500, 8192, 2048),  # fused QKV+gate
    (750, 128, 2048),    # out_proj (BN = 128 path)
    (577, 2048, 5888),   # W2 with K = 5888
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("path", [0, 1])
def test_gemm_store_matches_torch(dev, M, N, K, path):
    if path == 1 and M * N * K > 2e9:
        pytest.skip("SIMT path checked on the smaller shapes")
    g = torch.Generator(device=dev).manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
    C = torch.full((M, N), float("nan"), device=dev)
    check(hooks().irtt_gemm_store(ptr(A), ptr(B), M, N, K, ptr(C), path))
    ref = A.float() @ B.float().T
    err = (C - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-5, f"rel max err {err}"


def _rope_tables(hd, S):
    half = hd // 2
    i = torch.arange(half, dtype=torch.float32)
    fr = 1.0 / torch.pow(torch.tensor(10000.0), 2.0 * i / hd)
    ang = torch.arange(S, dtype=torch.float32)[:, None] * fr[None]
    return torch.cos(ang), torch.sin(ang)


@pytest.mark.parametrize("path", [0, 1])
def test_gemm_qkvg_epilogue(dev, path):
    M, H, hd = 300, 4, 128
    D = H * hd
    g = torch.Generator(device=dev).manual_seed(11)
    A = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
    W = (torch.randn(4 * D, D, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    qn = 1 + 0.1 * torch.randn(D, device=dev, generator=g)
    kn = 1 + 0.1 * torch.randn(D, device=dev, generator=g)
    cos, sin = (t.to(dev).contiguous() for t in _rope_tables(hd, 200))
    pos = (torch.arange(M, device=dev) % 150).to(torch.int32)
    outs = [torch.zeros(M, D, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    check(hooks().irtt_gemm_epi(1, ptr(A), ptr(W), M, 4 * D, D, path, *[ptr(o) for o in outs], ptr(qn), ptr(kn),
                                ptr(cos), ptr(sin), ptr(pos), H, hd, H // 2, None, None, 0))
    acc = A.float() @ W.float().T
    q, k, v, gg = acc.split(D, dim=1)

    def norm_rope(x, w):
        x = x.reshape(M, H, hd)
        x = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-5) * w.reshape(H, hd)
        c = cos[pos.long()][:, None, :]
        s = sin[pos.long()][:, None, :]
        re, im = x[..., 0::2], x[..., 1::2]
        rot = torch.stack([re * c - im * s, re * s + im * c], dim=-1).reshape(M, H, hd)
        x = torch.cat([rot[:, : H // 2], x[:, H // 2:]], dim=1)
        return x.reshape(M, D)

    refs = [norm_rope(q, qn), norm_rope(k, kn), v, torch.sigmoid(gg)]
    for o, r, name in zip(outs, refs, "qkvg"):
        err = (o.float() - r).abs().max().item() / r.abs().max().item()
        assert err < 1e-2, f"{name}: rel err {err}"


@pytest.mark.parametrize("path", [0, 1])
def test_gemm_qkvg_without_norm_weights_or_rope(dev, path):
    """Null head-norm weights mean no head norm and no RoPE tables mean no
    RoPE: q / k / v are the plain projections, g its sigmoid (the epilogue
    must not offset a null weight pointer)."""
    M, H, hd = 300, 4, 128
    D = H * hd
    g = torch.Generator(device=dev).manual_seed(12)
    A = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
    W = (torch.randn(4 * D, D, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    outs = [torch.zeros(M, D, device=dev, dtype=torch.bfloat16) for _ in range(4)]
    check(hooks().irtt_gemm_epi(1, ptr(A), ptr(W), M, 4 * D, D, path, *[ptr(o) for o in outs], None, None, None,
                                None, None, H, hd, H // 2, None, None, 0))
    acc = A.float() @ W.float().T
    q, k, v, gg = acc.split(D, dim=1)
    for o, r, name in zip(outs, [q, k, v, torch.sigmoid(gg)], "qkvg"):
        err = (o.float() - r).abs().max().item() / r.abs().max().item()
        assert err < 1e-2, f"{name}: rel err {err}"


# (M, N, K, batch, bf16 operands, A row pitch, A batch stride): the engine's
# adaLN-table and cond_module shapes (one row per timestep), tails in every
# dimension, the scalar-load path (K % 4 != 0, bf16) and the cluster K-split
# (few tiles) as well as the unsplit batched path.
SIMT_CASES = [
    (41, 12288, 2048, 1, 0, 3 * 2048, 0),     # adaLN down, A = silu(c) slice of the 3-D row
    (41, 2048, 256, 48, 0, 48 * 256, 256),    # adaLN up, batched over (layer, half)
    (41, 2048, 512, 1, 0, 512, 0),            # cond_module layer 0 (8-way split)
    (5, 2048, 2048, 1, 0, 2048, 0),           # 4-step request
    (5, 70, 300, 2, 0, 300, 300 * 5),         # tails, split into 5
    (5, 70, 301, 2, 0, 301, 301 * 5),         # scalar loads (K % 4 != 0)
    (65, 130, 1000, 1, 1, 1000, 0),           # bf16 operands, M / N tails
    (1, 64, 64, 1, 0, 64, 0),                 # single row, single k-tile pair
]


@pytest.mark.parametrize("M,N,K,batch,bf,lda,a_bs", SIMT_CASES)
def test_gemm_simt_batched_strided(dev, M, N, K, batch, bf, lda, a_bs):
    L = hooks()
    L.irtt_gemm_simt.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_long] * 2
                                 + [ctypes.c_void_p, ctypes.c_long, ctypes.c_long] + [ctypes.c_int] * 4)
    g = torch.Generator(device=dev).manual_seed(M * 7 + N + K)
    dt = torch.bfloat16 if bf else torch.float32
    a_store = torch.randn(max(a_bs * (batch - 1) + (M - 1) * lda + K, 1), device=dev, generator=g).to(dt)
    B = torch.randn(batch, N, K, device=dev, generator=g).to(dt)
    C = torch.full((batch, M, N + 3), float("nan"), device=dev)
    A = torch.as_strided(a_store, (batch, M, K), (a_bs, lda, 1))
    ref = torch.einsum("zmk,znk->zmn", A.double(), B.double())
    rc = L.irtt_gemm_simt(ptr(a_store), bf, lda, a_bs, ptr(B), bf, K, N * K, ptr(C), N + 3, M * (N + 3), M, N, K,
                          batch)
    check(rc)
    out = C[:, :, :N].double()
    err = ((out - ref).norm() / ref.norm()).item()
    assert err < 1e-6, err
    assert torch.isnan(C[:, :, N:]).all(), "wrote outside the N columns"
    # the K split sums the partial tiles in a fixed order: bit-identical reruns
    C2 = torch.full_like(C, float("nan"))
    check(L.irtt_gemm_simt(ptr(a_store), bf, lda, a_bs, ptr(B), bf, K, N * K, ptr(C2), N + 3, M * (N + 3), M, N, K,
                           batch))
    assert torch.equal(C[:, :, :N], C2[:, :, :N])


@pytest.mark.parametrize("path", [0, 1])
def test_gemm_swiglu_and_resid(dev, path):
    M, D, F = 257, 256, 736
    Fp = (F + 31) // 32 * 32
    g = torch.Generator(device=dev).manual_seed(5)
    A = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
    W1 = torch.randn(F, D, device=dev, generator=g) * 0.05
    W3 = torch.randn(F, D, device=dev, generator=g) * 0.05
    packed = torch.zeros(2 * Fp, D, device=dev)
    for j in range(Fp // 32):
        n = min(32, F - 32 * j)
        packed[64 * j:64 * j + n] = W1[32 * j:32 * j + n]
        packed[64 * j + 32:64 * j + 32 + n] = W3[32 * j:32 * j + n]
    packed = packed.to(torch.bfloat16)
    h = torch.zeros(M, F, device=dev, dtype=torch.bfloat16)
    check(hooks().irtt_gemm_epi(3, ptr(A), ptr(packed), M, 2 * Fp, D, path, ptr(h), None, None, None, None, None,
                                None, None, None, 0, 0, 0, None, None, F))
    a = A.float() @ W1.to(torch.bfloat16).float().T
    b = A.float() @ W3.to(torch.bfloat16).float().T
    ref = torch.nn.functional.silu(a) * b
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, f"swiglu rel err {err}"
    # residual with gate: x = x + gate * (h @ W2^T)
    W2 = (torch.randn(D, F, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(M, D, device=dev, generator=g)
    gate = torch.randn(D, device=dev, generator=g)
    x_ref = x + gate * (h.float() @ W2.float().T)
    check(hooks().irtt_gemm_epi(2, ptr(h), ptr(W2), M, D, F, path, None, None, None, None, None, None, None, None,
                                None, 0, 0, 0, ptr(x), ptr(gate), 0))
    err = (x - x_ref).abs().max().item() / x_ref.abs().max().item()
    assert err < 1e-4, f"resid rel err {err}"


@pytest.mark.parametrize("M,N,K", [(300, 2048, 5888), (750, 2048, 2048), (1500, 2048, 5888), (3000, 2048, 5888),
                                   (3400, 2048, 5888)])
def test_gemm_resid_split_k(dev, M, N, K):
    """Few tiles -> the residual GEMM reduce-adds partial products: K-splits
    (M = 300-3000) or stream-K (M = 3400, K = 5888: each SM pair takes an equal
    span of all tiles' k-blocks, spans crossing tile boundaries); the result
    must equal x + gate * (A @ W^T) (order-independent to fp32 rounding)."""
    g = torch.Generator(device=dev).manual_seed(M + K)
    A = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(M, N, device=dev, generator=g)
    gate = torch.randn(N, device=dev, generator=g)
    ref = x + gate * (A.float() @ W.float().T)
    check(hooks().irtt_gemm_epi(2, ptr(A), ptr(W), M, N, K, 0, None, None, None, None, None, None, None, None,
                                None, 0, 0, 0, ptr(x), ptr(gate), 0))
    err = (x - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, f"split-K resid rel err {err}"


@pytest.mark.parametrize("M,D", [(300, 2048), (9000, 2048), (77, 1280)])  # small-M and large-M kernels
@pytest.mark.parametrize("out_bf16", [1, 0])
def test_adaln_modulate_matches_torch(dev, out_bf16, M, D):
    """adaLN modulate rows (the LowRankAdaLn output, h = x / sqrt(mean(x^2) +
    eps) * (1 + scale) + shift), f32 in, bf16 or f32 out, against torch fp32;
    the row kernel takes 256 threads per row up to 8,192 rows, 128 above."""
    eps = 1e-5
    g = torch.Generator(device=dev).manual_seed(21)
    x = torch.randn(M, D, device=dev, generator=g) * 3
    shift = torch.randn(D, device=dev, generator=g) * 0.1
    scale = torch.randn(D, device=dev, generator=g) * 0.1
    h = torch.full((M, D), float("nan"), device=dev).to(torch.bfloat16 if out_bf16 else torch.float32)
    L = hooks()
    L.irtt_adaln_modulate.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_float]
    check(L.irtt_adaln_modulate(ptr(x), ptr(shift), ptr(scale), ptr(h), out_bf16, M, D, eps))
    ref = x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * (1 + scale) + shift
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < (1e-2 if out_bf16 else 1e-5), f"adaln rel err {err}"


def _attn_ref(q, k, v, g, ck, cv, key_mask, seqs, H, hd):
    out = torch.zeros_like(q, dtype=torch.float32)
    for (ts, ln, co, cl) in seqs:
        qs = q[ts:ts + ln].float().reshape(ln, H, hd)
        ks = [k[ts:ts + ln].float().reshape(ln, H, hd)]
        vs = [v[ts:ts + ln].float().reshape(ln, H, hd)]
        valid = [torch.ones(ln, dtype=torch.bool, device=q.device) if key_mask is None
                 else key_mask[ts:ts + ln].bool()]
        if cl:
            ks.append(ck[co:co + cl].float().reshape(cl, H, hd))
            vs.append(cv[co:co + cl].float().reshape(cl, H, hd))
            valid.append(torch.ones(cl, dtype=torch.bool, device=q.device))
        K_, V_, m = torch.cat(ks), torch.cat(vs), torch.cat(valid)
        s = torch.einsum("qhd,khd->hqk", qs, K_) / math.sqrt(hd)
        s = s.masked_fill(~m[None, None], float("-inf"))
        w = torch.nan_to_num(torch.softmax(s, -1), nan=0.0)
        o = torch.einsum("hqk,khd->qhd", w, V_).reshape(ln, H * hd)
        out[ts:ts + ln] = o * (g[ts:ts + ln].float() if g is not None else 1)
    return out


ATTN_PATHS = [(1, 0), (1, 1), (0, 2), (0, 3)]  # (bf16, path): tcgen05, mma.sync, tiled SIMT, warp SIMT


@pytest.mark.parametrize("kt", ["64", "128"])
@pytest.mark.parametrize("case", ["mixed", "config3", "ragged"])
def test_attention_key_tile_variants(dev, monkeypatch, kt, case):
    """Both key-tile widths of the tcgen05 kernel (64 keys at two CTAs per SM,
    128 keys at one CTA per SM), forced through IRT_ATTN_KT."""
    monkeypatch.setenv("IRT_ATTN_KT", kt)
    test_attention_matches_torch(dev, 1, 0, case)


@pytest.mark.parametrize("bf16,path", ATTN_PATHS)
@pytest.mark.parametrize("case", ["mixed", "config3", "ragged"])
def test_attention_matches_torch(dev, bf16, path, case):
    H, hd = 4, 128
    D = H * hd
    if case == "mixed":  # partial self tiles, empty / tiny / multi-tile contexts
        seqs = [(0, 150, 0, 77), (150, 64, 77, 0), (214, 1, 77, 5), (215, 90, 82, 130)]
        M, nctx = 305, 212
    elif case == "ragged":  # config-4-like batch: cond rows with contexts, then uncond rows without
        lens = [37, 129, 300, 64, 65, 255, 3, 191, 385, 128]
        ctxs = [17, 300, 0, 63, 64, 129, 200, 1, 77, 256]
        seqs, t, c = [], 0, 0
        for ln, cl in zip(lens, ctxs):
            seqs.append((t, ln, c, cl))
            t, c = t + ln, c + cl
        for ln in lens:
            seqs.append((t, ln, 0, 0))
            t += ln
        M, nctx = t, c
    else:  # joint-CFG rows of config 3: cond (750 + 576 context keys), uncond (750 keys)
        seqs = [(0, 750, 0, 576), (750, 750, 0, 0)]
        M, nctx = 1500, 576
    dt = torch.bfloat16 if bf16 else torch.float32
    g = torch.Generator(device=dev).manual_seed(3)
    mk = lambda n: torch.randn(n, D, device=dev, generator=g).to(dt)
    q, k, v, ck, cv = mk(M), mk(M), mk(M), mk(nctx), mk(nctx)
    gs = torch.sigmoid(torch.randn(M, D, device=dev, generator=g)).to(dt)
    out = torch.zeros(M, D, device=dev, dtype=dt)
    sd = (ctypes.c_int * (4 * len(seqs)))(*[x for s in seqs for x in s])
    check(hooks().irtt_attention(ptr(q), ptr(k), ptr(v), ptr(gs), ptr(ck), ptr(cv), None, sd, len(seqs), H, hd,
                                 ptr(out), bf16, M, nctx, path))
    ref = _attn_ref(q, k, v, gs, ck, cv, None, seqs, H, hd)
    err = (out.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < (2e-2 if bf16 else 1e-5), f"attention rel err {err}"


@pytest.mark.parametrize("bf16,path", [(1, 1), (0, 2), (0, 3)])
def test_attention_key_mask_and_empty_rows(dev, bf16, path):
    """Masked self keys are skipped; a sequence whose keys are all masked
    yields exactly 0 (safe softmax), even with NaN in the masked V rows."""
    H, hd = 2, 128
    D = H * hd
    M = 96
    dt = torch.bfloat16 if bf16 else torch.float32
    g = torch.Generator(device=dev).manual_seed(9)
    q = torch.randn(M, D, device=dev, generator=g).to(dt)
    k = torch.randn(M, D, device=dev, generator=g).to(dt)
    v = torch.randn(M, D, device=dev, generator=g).to(dt)
    mask = torch.ones(M, dtype=torch.uint8, device=dev)
    mask[40:64] = 0          # tail padding of sequence 0
    mask[64:96] = 0          # sequence 1 entirely masked
    v[64:96] = float("nan")  # masked keys must not leak NaN
    v[40:64] = float("nan")
    seqs = [(0, 64, 0, 0), (64, 32, 0, 0)]
    out = torch.full((M, D), 7.0, device=dev, dtype=dt)
    sd = (ctypes.c_int * 8)(*[x for s in seqs for x in s])
    check(hooks().irtt_attention(ptr(q), ptr(k), ptr(v), None, None, None, ptr(mask), sd, 2, H, hd, ptr(out), bf16,
                                 M, 0, path))
    assert torch.isfinite(out.float()).all()
    assert (out[64:96].float() == 0).all()
    ref = _attn_ref(q, k, torch.nan_to_num(v), None, None, None, mask, seqs[:1], H, hd)
    err = (out[:64].float() - ref[:64]).abs().max().item() / ref[:64].abs().max().item()
    assert err < (2e-2 if bf16 else 1e-5), f"rel err {err}"


F32_GEMM_CASES = [
    (256, 256, 64, 0),     # smallest pair tile, one k-block per segment
    (300, 384, 100, 0),    # K padded to 128 (zero columns between the hi and lo halves), partial n-tile
    (130, 2048, 1280, 0),  # single-CTA tiles (fewer than 256 rows)
    (750, 8192, 2048, 0),  # QKV+gate width at config-1 rows
    (750, 2048, 5888, 2),  # W2 residual at config-1 rows (K-splits across the three segments)
    (1500, 2048, 2048, 2),  # Wo residual
    (3400, 2048, 5888, 2),  # W2 residual at ~3,400 rows (stream-K / tail split)
]


@pytest.mark.parametrize("M,N,K,mode", F32_GEMM_CASES)
@pytest.mark.parametrize("path", [0, 1])
def test_gemm_f32_split_tf32_matches_f64(dev, M, N, K, mode, path):
    """The f32 mode's GEMM: path 0 = tcgen05 tf32 with hi / lo operand halves
    (A_hi.B_hi + A_hi.B_lo + A_lo.B_hi), path 1 = SIMT f32, both against an f64
    product.  The bound (1e-5 of the largest output) holds for f32 arithmetic
    and fails for a single tf32 product (~1e-4 at these sizes); path 0's
    relative L2 error must also stay below 1 % of cuBLAS's TF32 product's."""
    if path == 1 and M * N * K > 4e9:
        pytest.skip("SIMT path checked on the smaller shapes")
    L = hooks()
    L.irtt_gemm_f32.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 2 + [ctypes.c_int] * 4 + [ctypes.c_void_p] * 2
    g = torch.Generator(device=dev).manual_seed(M + 3 * N + 7 * K + mode)
    A = torch.randn(M, K, device=dev, generator=g)
    B = torch.randn(N, K, device=dev, generator=g) * 0.05
    prod = A.double() @ B.double().T
    if mode == 2:
        x = torch.randn(M, N, device=dev, generator=g)
        gate = torch.randn(N, device=dev, generator=g)
        ref = x.double() + gate.double() * prod
        check(L.irtt_gemm_f32(mode, ptr(A), ptr(B), M, N, K, path, ptr(x), ptr(gate)))
        out = x
    else:
        ref = prod
        out = torch.full((M, N), float("nan"), device=dev)
        check(L.irtt_gemm_f32(mode, ptr(A), ptr(B), M, N, K, path, ptr(out), None))
    err = (out.double() - ref).abs().max().item() / ref.abs().max().item()
    l2 = ((out.double() - ref).norm() / ref.norm()).item()
    ctx = ""
    if path == 0 and mode == 0:  # the same product through cuBLAS with TF32 off and on, for scale
        prev = torch.backends.cuda.matmul.allow_tf32
        try:
            l2s = {}
            for tf in (False, True):
                torch.backends.cuda.matmul.allow_tf32 = tf
                c = (A @ B.T).double()
                l2s[tf] = ((c - prod).norm() / prod.norm()).item()
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        ctx = f"; cuBLAS f32 {l2s[False]:.2e}, cuBLAS tf32 {l2s[True]:.2e}"
        assert l2 < 0.01 * l2s[True], (l2, l2s)
    print(f"f32 GEMM path {path} M={M} N={N} K={K} mode={mode}: rel-L2 {l2:.2e}, rel max {err:.2e}{ctx}")
    assert err < 1e-5, f"f32 GEMM rel max err {err}"


@pytest.mark.parametrize("force", ["1", None])
@pytest.mark.parametrize("M,K", [(54504, 2048), (27252, 5888), (6800, 5888), (1000, 1024)])
def test_gemm_resid_tail_split(dev, monkeypatch, force, M, K):
    """Residual GEMMs whose last wave of whole tiles is partly empty run the
    full rounds on whole tiles and spread the tail tiles' k-blocks over every
    SM pair (pieces reduce-added into x); forced on (IRT_TAIL_SPLIT=1) and as
    chosen by the dispatch rule."""
    if force:
        monkeypatch.setenv("IRT_TAIL_SPLIT", force)
    N = 2048
    g = torch.Generator(device=dev).manual_seed(M + K + 1)
    A = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(M, N, device=dev, generator=g)
    gate = torch.randn(N, device=dev, generator=g)
    ref = x + gate * (A.float() @ W.float().T)
    check(hooks().irtt_gemm_epi(2, ptr(A), ptr(W), M, N, K, 0, None, None, None, None, None, None, None, None,
                                None, 0, 0, 0, ptr(x), ptr(gate), 0))
    err = (x - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, f"tail-split resid rel err {err}"
