"""PEFT LoRA merge at load, on the host and without a GPU (the routine the
engine runs in InferenceBuilder::load_weights_with_adapter, src/inference.rs:
118-139; merge rule src/lora.rs:205-322, re-encode
src/weights/tensor_store.rs:90-118): W += lora_alpha / r * B @ A in f32, then
back to the base dtype (bf16 by truncation to the high 16 bits), PEFT prefixes
stripped and raw LoRA entries of a PEFT-saved base dropped."""

import ctypes
import json

import numpy as np
import pytest
import torch

from conftest import PKG_DIR

TARGETS = ["blocks.0.attention.wq.weight", "blocks.0.attention.wo.weight", "blocks.0.mlp.w1.weight",
           "in_proj.weight"]


def hooks():
    p = PKG_DIR / "libirodori_b200_testhooks.so"
    if not p.exists():
        pytest.skip("test-hook library not built")
    L = ctypes.CDLL(str(p))
    L.irtt_last_error.restype = ctypes.c_char_p
    L.irtt_lora_merged_tensor.argtypes = [ctypes.c_char_p] * 3 + [ctypes.c_void_p, ctypes.c_long,
                                                                   ctypes.POINTER(ctypes.c_int)]
    return L


def read_ckpt(path):
    from safetensors import safe_open
    with safe_open(str(path), framework="pt") as f:
        return {k: f.get_tensor(k) for k in f.keys()}, f.metadata()


def make_adapter(dirpath, base, synth, r=4, alpha=8.0, seed=3):
    g = torch.Generator().manual_seed(seed)
    ad = {}
    for k in TARGETS:
        d_out, d_in = base[k].shape
        stem = "base_model.model." + k[:-len(".weight")]
        ad[stem + ".lora_A.default.weight"] = 0.1 * torch.randn(r, d_in, generator=g)
        ad[stem + ".lora_B.default.weight"] = 0.1 * torch.randn(d_out, r, generator=g)
    dirpath.mkdir(parents=True, exist_ok=True)
    (dirpath / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha}))
    synth.write_safetensors(str(dirpath / "adapter_model.safetensors"), ad, {})
    return ad, alpha / r


def merged_tensor(L, base_path, adapter_dir, name, numel):
    out = np.empty(numel, dtype=np.float32)
    n = ctypes.c_int(-1)
    rc = L.irtt_lora_merged_tensor(str(base_path).encode(), str(adapter_dir).encode(), name.encode(),
                                   out.ctypes.data, numel, ctypes.byref(n))
    assert rc == 0, L.irtt_last_error().decode()
    return out, n.value


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_host_merge_matches_python(synth, tmp_path, dtype):
    L = hooks()
    base_p = tmp_path / "base.safetensors"
    synth.make_dit_checkpoint(str(base_p), synth.TINY_CONFIG, seed=1, init="full", dtype=dtype)
    base, _ = read_ckpt(base_p)
    ad, scale = make_adapter(tmp_path / "adapter", base, synth)
    for k in TARGETS:
        stem = "base_model.model." + k[:-len(".weight")]
        A, B = ad[stem + ".lora_A.default.weight"], ad[stem + ".lora_B.default.weight"]
        want = base[k].float() + np.float32(scale) * (B @ A)
        got, n = merged_tensor(L, base_p, tmp_path / "adapter", k, base[k].numel())
        assert n == len(TARGETS)
        got = torch.from_numpy(got).reshape(want.shape)
        if dtype == torch.float32:
            assert (got - want).abs().max().item() <= 1e-6 * max(1.0, want.abs().max().item())
        else:
            # truncated to bf16: exactly representable, within one bf16 step of the f32 merge
            assert torch.equal(got, got.to(torch.bfloat16).float())
            assert ((got - want).abs() <= want.abs() * 2.0 ** -7 + 1e-30).all()
    # an untouched tensor comes back bit-identical
    k = "out_proj.weight"
    got, _ = merged_tensor(L, base_p, tmp_path / "adapter", k, base[k].numel())
    assert np.array_equal(got, base[k].float().numpy().reshape(-1))


def test_host_merge_peft_base_and_errors(synth, tmp_path):
    L = hooks()
    base_p = tmp_path / "base.safetensors"
    synth.make_dit_checkpoint(str(base_p), synth.TINY_CONFIG, seed=1, init="full")
    base, meta = read_ckpt(base_p)
    make_adapter(tmp_path / "adapter", base, synth)
    peft = {"base_model.model." + k: v for k, v in base.items()}
    peft["base_model.model.blocks.0.attention.wq.lora_A.default.weight"] = torch.zeros(2, 2)
    pp = tmp_path / "peft.safetensors"
    synth.write_safetensors(str(pp), peft, meta)
    k = TARGETS[0]
    a, _ = merged_tensor(L, base_p, tmp_path / "adapter", k, base[k].numel())
    b, n = merged_tensor(L, pp, tmp_path / "adapter", k, base[k].numel())
    assert n == len(TARGETS) and np.array_equal(a, b)
    empty = tmp_path / "empty"
    empty.mkdir()
    out = np.empty(base[k].numel(), dtype=np.float32)
    rc = L.irtt_lora_merged_tensor(str(base_p).encode(), str(empty).encode(), k.encode(), out.ctypes.data,
                                   out.size, None)
    assert rc != 0 and "cannot read adapter_config.json" in L.irtt_last_error().decode()
    (empty / "adapter_config.json").write_text(json.dumps({"r": 4, "lora_alpha": 8}))
    rc = L.irtt_lora_merged_tensor(str(base_p).encode(), str(empty).encode(), k.encode(), out.ctypes.data,
                                   out.size, None)
    assert rc != 0 and "no adapter weights found" in L.irtt_last_error().decode()
