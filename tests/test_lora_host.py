"""LoRA on the host, no GPU: adapter files (lora.rs:39-174: safetensors, Glimpse-Lab and PEFT keys, peft_scaling),
adapter_id (runtime/mod.rs:236-243), and the oracle's LoRA arithmetic against a float64 numpy restatement."""
import json
import os
import struct

import numpy as np
import pytest

from bonsai_b200 import lora, synth
from bonsai_b200.config import tiny
from oracle import oracle as orc


def adapter(rank=4, k=64, o=32, seed=0):
    rng = np.random.default_rng(seed)
    return rng.normal(0, 0.02, (rank, k)).astype(np.float32), rng.normal(0, 0.01, (o, rank)).astype(np.float32)


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
def test_safetensors_round_trip(tmp_path, dtype):
    a, b = adapter()
    p = str(tmp_path / "a.safetensors")
    lora.write_safetensors(p, {"x": a, "y": b}, dtype)
    t = lora.read_safetensors(p)
    tol = {"F32": 0, "F16": 1e-3, "BF16": 8e-3}[dtype]
    assert t["x"].shape == a.shape and t["y"].shape == b.shape
    np.testing.assert_allclose(t["x"], a, rtol=tol, atol=1e-7)
    np.testing.assert_allclose(t["y"], b, rtol=tol, atol=1e-7)


def test_bad_safetensors(tmp_path):
    p = str(tmp_path / "bad.safetensors")
    open(p, "wb").write(b"123")
    with pytest.raises(lora.LoraError, match="not a safetensors"):
        lora.read_safetensors(p)
    hdr = json.dumps({"x": {"dtype": "I8", "shape": [1], "data_offsets": [0, 1]}}).encode()
    open(p, "wb").write(struct.pack("<Q", len(hdr)) + hdr + b"\0")
    with pytest.raises(lora.LoraError, match="unsupported dtype"):
        lora.read_safetensors(p)


def test_glimpse_lab_keys(tmp_path):
    """Glimpse-Lab export: alpha / r already in B, so the fold is 1 (lora.rs:1-4, 92-93)."""
    a, b = adapter()
    p = str(tmp_path / "adapter.safetensors")
    lora.write_safetensors(p, {"model.layers.3.mlp.down_proj.lora_A": a, "model.layers.3.mlp.down_proj.lora_B": b,
                               "model.layers.0.self_attn.q_proj.lora_A": a,
                               "model.layers.0.self_attn.q_proj.lora_B": b})
    lins, fold = lora.parse(p)
    assert fold == 1.0
    assert [(l, m) for l, m, _, _ in lins] == [(0, "self_attn.q_proj"), (3, "mlp.down_proj")]
    np.testing.assert_array_equal(lins[1][2], a)
    np.testing.assert_array_equal(lins[1][3], b)


@pytest.mark.parametrize("rslora", [False, True])
def test_peft_keys_and_scaling(tmp_path, rslora):
    a, b = adapter(rank=16)
    p = str(tmp_path / "adapter_model.safetensors")
    pre = "base_model.model.model.language_model.layers.1.linear_attn.in_proj_z"
    lora.write_safetensors(p, {pre + ".lora_A.weight": a, pre + ".lora_B.weight": b})
    cfg = {"r": 16, "lora_alpha": 32, "use_rslora": rslora}
    open(tmp_path / "adapter_config.json", "w").write(json.dumps(cfg))
    lins, fold = lora.parse(p)
    assert [(l, m) for l, m, _, _ in lins] == [(1, "linear_attn.in_proj_z")]
    assert fold == pytest.approx(32 / 4 if rslora else 2.0)


def test_peft_errors(tmp_path):
    a, b = adapter()
    p = str(tmp_path / "adapter_model.safetensors")
    lora.write_safetensors(p, {"layers.0.mlp.up_proj.lora_A.weight": a, "layers.0.mlp.up_proj.lora_B.weight": b})
    with pytest.raises(lora.LoraError, match="PEFT keys need"):
        lora.parse(p)
    open(tmp_path / "adapter_config.json", "w").write(json.dumps({"r": 4, "lora_alpha": 8,
                                                                  "rank_pattern": {"x": 2}}))
    with pytest.raises(lora.LoraError, match="rank_pattern"):
        lora.parse(p)
    open(tmp_path / "adapter_config.json", "w").write(json.dumps({"r": 4}))
    with pytest.raises(lora.LoraError, match="lora_alpha"):
        lora.parse(p)


def test_key_errors(tmp_path):
    a, b = adapter()
    p = str(tmp_path / "x.safetensors")
    lora.write_safetensors(p, {"layers.0.mlp.up_proj.lora_A": a})
    with pytest.raises(lora.LoraError, match="needs lora_A and lora_B"):
        lora.parse(p)
    lora.write_safetensors(p, {"layers.0.mlp.up_proj.weight_x": a})
    with pytest.raises(lora.LoraError, match="unexpected tensor"):
        lora.parse(p)
    lora.write_safetensors(p, {"embed.lora_A": a, "embed.lora_B": b})
    with pytest.raises(lora.LoraError, match="not a layer linear"):
        lora.parse(p)


def test_adapter_id(tmp_path):
    a, b = adapter()
    p = str(tmp_path / "adapter.safetensors")
    lora.write_safetensors(p, {"layers.0.mlp.up_proj.lora_A": a, "layers.0.mlp.up_proj.lora_B": b})
    i1 = lora.adapter_id(p, 1.0)
    assert i1 & 1 and i1 == lora.adapter_id(p, 1.0)
    assert lora.adapter_id(p, 0.5) != i1
    open(tmp_path / "adapter_config.json", "w").write("{}")
    assert lora.adapter_id(p, 1.0) != i1  # the PEFT config beside the file is part of it
    # the reference's formula: hash(file), then hash(config), then hash(scale as f32 LE) | 1
    from oracle.prefix_file import FNV, hash_bytes
    h = hash_bytes(hash_bytes(FNV, open(p, "rb").read()), b"{}")
    assert lora.adapter_id(p, 1.0) == hash_bytes(h, struct.pack("<f", 1.0)) | 1


@pytest.mark.parametrize("r,O,K,T", [(1, 8, 16, 1), (16, 96, 512, 9), (7, 33, 100, 3)])
def test_oracle_lora_add(r, O, K, T):
    rng = np.random.default_rng(r * 100 + T)
    a = rng.normal(0, 0.02, (r, K)).astype(np.float32)
    b = rng.normal(0, 0.01, (O, r)).astype(np.float32)
    x = rng.normal(0, 1, (T, K)).astype(np.float32)
    y = rng.normal(0, 1, (T, O)).astype(np.float32)
    got = orc.lora_add(a, b, x, y)
    want = y.astype(np.float64) + (x.astype(np.float64) @ a.T.astype(np.float64)) @ b.T.astype(np.float64)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


def test_oracle_model_lora_properties():
    """B = 0 (or fold 0) leaves the logits bit-identical; the fold multiplies B before the fp16 rounding, so (2B, 0.5)
    equals (B, 1); an adapter on every linear moves the logits."""
    cfg = tiny()
    ts = synth.model_tensors(cfg, 3)
    o = orc.OracleModel(cfg, ts)
    ids = synth.zipf_tokens(4, 9, cfg.vocab)
    _, base = o.forward(ids, logits=True)
    lins = synth.lora_linears(cfg, 8, seed=5, std_b=0.05)
    o.set_lora([(l, m, a, 0 * b) for l, m, a, b in lins], 2.0)
    o.reset()
    _, zero_b = o.forward(ids, logits=True)
    assert np.array_equal(zero_b, base)
    o.set_lora(lins, 2.0)
    o.reset()
    _, one = o.forward(ids, logits=True)
    assert np.abs(one - base).max() > 1e-2
    o.set_lora([(l, m, a, 2 * b) for l, m, a, b in lins], 1.0)
    o.reset()
    _, two = o.forward(ids, logits=True)
    assert np.array_equal(one, two)
    o.clear_lora()
    o.reset()
    _, back = o.forward(ids, logits=True)
    assert np.array_equal(back, base)
    with pytest.raises(ValueError):
        o.set_lora([(0, "mlp.nope", lins[0][2], lins[0][3])], 1.0)
