"""Per-layer parity of the DiT forward against the CPU oracle.

The engine (test-hook build) runs one sample() and copies the f32 residual
stream of its first DiT forward after in_proj and after every block; the
oracle runs the same first forward (`dit_forward(..., capture=True)`, the
reference's forward_with_cond_debug, src/model/dit/model.rs:269-346) on the
same batch: independent CFG at the first step, i.e. the condition plus the
text- and speaker-unconditional bundles concatenated along the batch
(src/rf/euler_sampler.rs:397-451), which is exactly the engine's packed row
order (group, utterance, frame).

Tolerances (north star): f32 mode per-layer outputs within 1e-4 relative L2;
bf16 mode (tcgen05 GEMM pairs and attention) within 1e-2.
"""

import ctypes

import numpy as np
import pytest

from test_gpu_kernels import dev, hooks  # noqa: F401  (fixture)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 1e-2


def layer_cfg(synth):
    c = dict(synth.SMALL_CONFIG)
    c["num_layers"] = 4
    return c


def engine_layers(pkg, ckpt, precision, r, S, params, D, nlayers):
    """[L + 1, rows, D] captured by the engine's first forward."""
    L = hooks()
    L.irtt_sample_dump_layers.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int)]
    keep = []

    def arr(x, dt):
        a = np.ascontiguousarray(x.numpy() if torch.is_tensor(x) else x, dtype=dt)
        keep.append(a)
        return a

    ids, tm = arr(r["text_ids"], np.int32), arr(r["text_mask"], np.uint8)
    ref, rm = arr(r["ref_latent"], np.float32), arr(r["ref_mask"], np.uint8)
    noise = arr(r["initial_noise"], np.float32)
    B = ids.shape[0]
    q = pkg._Request()
    q.batch, q.text_len, q.text_ids, q.text_mask = B, ids.shape[1], ids.ctypes.data, tm.ctypes.data
    q.ref_len, q.ref_dim, q.ref_latent, q.ref_mask = ref.shape[1], ref.shape[2], ref.ctypes.data, rm.ctypes.data
    q.sequence_length = S
    q.initial_noise = noise.ctypes.data
    q.memory = pkg.MEM_HOST
    cp = params._to_c()
    cap = 3 * B * S
    dump = torch.full(((nlayers + 1) * cap * D,), float("nan"), device="cuda")
    out = np.empty(noise.shape, dtype=np.float32)
    rows = ctypes.c_int(0)
    prec = 0 if precision == "bf16" else 1
    rc = L.irtt_sample_dump_layers(str(ckpt).encode(), prec, ctypes.byref(cp), ctypes.byref(q),
                                   out.ctypes.data, dump.data_ptr(), cap, ctypes.byref(rows))
    assert rc == 0, L.irtt_last_error().decode()
    assert rows.value == cap
    return dump.view(nlayers + 1, cap, D).cpu().numpy()


def oracle_layers(oracle, ckpt, r, S):
    W = oracle.Weights.load(str(ckpt))
    req = oracle.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=S,
                                 ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                 initial_noise=r["initial_noise"])
    cond = oracle.encode_conditions(W, req)
    unc = cond.zeros_like()
    text_unc = oracle.Cond(unc.text_state, unc.text_mask, cond.aux_kind, cond.aux_state, cond.aux_mask)
    spk_unc = oracle.Cond(cond.text_state, cond.text_mask, unc.aux_kind, unc.aux_state, unc.aux_mask)
    batch = oracle.cat_batch([cond, text_unc, spk_unc])
    kv = oracle.build_kv_caches(W, batch)
    cos, sin = oracle.rope_tables(W.cfg.head_dim(), S, dtype=W.dtype)
    t0 = oracle.t_schedule(2)[0]
    x = torch.cat([r["initial_noise"]] * 3, 0)
    B3 = x.shape[0]
    _, after_in, outs = oracle.dit_forward(W, x, torch.full((B3,), t0, dtype=torch.float32), kv, cos, sin,
                                           capture=True)
    return np.stack([after_in.reshape(-1, after_in.shape[-1]).numpy()] +
                    [o.reshape(-1, o.shape[-1]).numpy() for o in outs])


@pytest.mark.parametrize("precision,T,R,S,tol", [("f32", 12, 9, 17, F32_TOL), ("bf16", 64, 80, 150, BF16_TOL)])
def test_first_forward_per_layer(dev, pkg, oracle, synth, ckpt_dir, precision, T, R, S, tol):  # noqa: F811
    cfg = layer_cfg(synth)
    ckpt = ckpt_dir / "layers4.safetensors"
    if not ckpt.exists():
        synth.make_dit_checkpoint(str(ckpt), cfg, seed=7, init="full")
    r = synth.make_request(cfg, 2, T, R, S, seed=5)
    params = pkg.SamplerParams(num_steps=2, method="euler",
                               guidance=pkg.GuidanceConfig(mode="independent", scale_text=3.0, scale_speaker=5.0))
    got = engine_layers(pkg, ckpt, precision, r, S, params, cfg["model_dim"], cfg["num_layers"])
    ref = oracle_layers(oracle, ckpt, r, S)
    assert got.shape == ref.shape
    errs = []
    for layer in range(ref.shape[0]):
        a = got[layer].astype(np.float64)
        b = ref[layer].astype(np.float64)
        assert np.isfinite(a).all(), f"layer {layer}: non-finite engine output"
        errs.append(float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)))
    print(f"{precision} per-layer rel L2 (in_proj, blocks 1..{len(errs) - 1}): " + " ".join(f"{e:.2e}" for e in errs))
    assert max(errs) < tol, errs
