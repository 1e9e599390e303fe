"""PEFT LoRA adapters merged at load (InferenceBuilder::load_weights_with_adapter,
src/inference.rs:118-139; merge rule src/lora.rs:205-322, re-encode
src/weights/tensor_store.rs:90-118): the engine built from base + adapter
must sample exactly like an engine built from a checkpoint merged here in
Python with the same rule (W += lora_alpha / r * B @ A, re-encoded to the
base dtype: bf16 by truncation)."""

import json

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TARGETS = ["blocks.0.attention.wq.weight", "blocks.0.attention.wo.weight", "blocks.0.mlp.w1.weight",
           "in_proj.weight"]


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return 0


def read_ckpt(path):
    from safetensors import safe_open
    with safe_open(str(path), framework="pt") as f:
        return {k: f.get_tensor(k) for k in f.keys()}, f.metadata()


def make_adapter(dirpath, base, r=4, alpha=8.0, seed=3):
    g = torch.Generator().manual_seed(seed)
    ad = {}
    for k in TARGETS:
        d_out, d_in = base[k].shape
        stem = "base_model.model." + k[:-len(".weight")]
        ad[stem + ".lora_A.default.weight"] = 0.1 * torch.randn(r, d_in, generator=g)
        ad[stem + ".lora_B.default.weight"] = 0.1 * torch.randn(d_out, r, generator=g)
    dirpath.mkdir(parents=True, exist_ok=True)
    (dirpath / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha, "bias": "none",
                                                             "target_modules": ["wq", "wo", "w1", "in_proj"]}))
    return ad, alpha / r


def merged(base, ad, scale):
    out = dict(base)
    for k in TARGETS:
        stem = "base_model.model." + k[:-len(".weight")]
        A, B = ad[stem + ".lora_A.default.weight"], ad[stem + ".lora_B.default.weight"]
        w = base[k].float() + np.float32(scale) * (B @ A)
        if base[k].dtype == torch.bfloat16:  # high 16 bits of the f32 pattern
            w = (w.contiguous().view(torch.int32) & ~0xFFFF).view(torch.float32).to(torch.bfloat16)
        out[k] = w.to(base[k].dtype)
    return out


def sample(pkg, builder, synth, cfg):
    r = synth.make_request(cfg, 2, 10, 7, 13, seed=2)
    eng = builder.with_sampling(pkg.SamplerParams(num_steps=3, guidance=pkg.GuidanceConfig(mode="independent"))).build()
    return eng.sample(pkg.SamplingRequest(text_ids=r["text_ids"], text_mask=r["text_mask"], sequence_length=13,
                                          ref_latent=r["ref_latent"], ref_mask=r["ref_mask"],
                                          initial_noise=r["initial_noise"]))


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_adapter_merge_matches_merged_checkpoint(gpu, pkg, synth, tmp_path, dtype):
    cfg = synth.TINY_CONFIG
    base_p = tmp_path / "base.safetensors"
    synth.make_dit_checkpoint(str(base_p), cfg, seed=1, init="full", dtype=dtype)
    base, meta = read_ckpt(base_p)
    ad, scale = make_adapter(tmp_path / "adapter", base)
    synth.write_safetensors(str(tmp_path / "adapter" / "adapter_model.safetensors"), ad, {})
    m_p = tmp_path / "merged.safetensors"
    synth.write_safetensors(str(m_p), merged(base, ad, scale), meta)
    b = pkg.InferenceBuilder(0)
    got = sample(pkg, b.load_weights_with_adapter(str(base_p), str(tmp_path / "adapter"), precision="f32"), synth, cfg)
    want = sample(pkg, pkg.InferenceBuilder(0).load_weights(str(m_p), precision="f32"), synth, cfg)
    plain = sample(pkg, pkg.InferenceBuilder(0).load_weights(str(base_p), precision="f32"), synth, cfg)
    assert rel(plain, want) > 1e-3  # the adapter changes the output
    assert rel(got, want) < 1e-5, rel(got, want)


def test_adapter_on_peft_prefixed_base_and_errors(gpu, pkg, synth, tmp_path):
    cfg = synth.TINY_CONFIG
    base_p = tmp_path / "base.safetensors"
    synth.make_dit_checkpoint(str(base_p), cfg, seed=1, init="full")
    base, meta = read_ckpt(base_p)
    ad, scale = make_adapter(tmp_path / "adapter", base)
    synth.write_safetensors(str(tmp_path / "adapter" / "adapter_model.safetensors"), ad, {})
    # PEFT-saved base: prefixed keys plus a raw LoRA entry that must be dropped
    peft = {"base_model.model." + k: v for k, v in base.items()}
    peft["base_model.model.blocks.0.attention.wq.lora_A.default.weight"] = torch.zeros(2, 2)
    pp = tmp_path / "peft_base.safetensors"
    synth.write_safetensors(str(pp), peft, meta)
    m_p = tmp_path / "merged.safetensors"
    synth.write_safetensors(str(m_p), merged(base, ad, scale), meta)
    got = sample(pkg, pkg.InferenceBuilder(0).load_weights_with_adapter(str(pp), str(tmp_path / "adapter"),
                                                                       precision="f32"), synth, cfg)
    want = sample(pkg, pkg.InferenceBuilder(0).load_weights(str(m_p), precision="f32"), synth, cfg)
    assert rel(got, want) < 1e-5
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(pkg.IrodoriError, match="cannot read adapter_config.json"):
        pkg.InferenceBuilder(0).load_weights_with_adapter(str(base_p), str(empty))
    (empty / "adapter_config.json").write_text(json.dumps({"r": 4, "lora_alpha": 8}))
    with pytest.raises(pkg.IrodoriError, match="no adapter weights found"):
        pkg.InferenceBuilder(0).load_weights_with_adapter(str(base_p), str(empty))
