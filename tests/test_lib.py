"""The C-ABI library on the CPU: it loads, exports every entry point include/bonsai_cuda.h declares, validates
configs like Config::check, and its host-only parts (synthetic inputs, drafting logic) agree with the oracle's
restatement. No device calls."""
import ctypes
import os
import re

import numpy as np
import pytest

from bonsai_b200 import _lib, config, synth
from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions(name="bonsai_cuda.h"):
    text = open(os.path.join(ROOT, "include", name)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bcu_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    for n in names:
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_synth_library_exports_its_header_and_backend_does_not():
    names = header_functions("bonsai_synth.h")
    assert names == ["bcu_synth_fill", "bcu_synth_zipf"]
    S = synth.lib()
    for n in names:
        assert hasattr(S, n) and n in synth.SIGNATURES
        assert not hasattr(_lib.lib(), n), f"{n} must not be in the CUDA backend"


def test_config_check_mirrors_reference_rules():
    ok, msg = config.check(config.bonsai_2b_graded())
    assert ok, msg
    ok, msg = config.check(config.bonsai_4b_graded())
    assert ok, msg
    c = config.tiny()
    c.head_dim = 128
    assert config.check(c) == (False, "unsupported config: head_dim must be 256")
    c = config.tiny()
    c.eps = 1e-5
    assert not config.check(c)[0]
    c = config.tiny()
    c.group_size = 32
    assert not config.check(c)[0]


def test_parse_reference_config_file():
    # the reference's own fixture (tests/data/config-2b.json), copied verbatim into tests/golden/
    path = os.path.join(os.path.dirname(__file__), "golden", "ref_config-2b.json")
    c = config.parse_config(open(path).read())
    assert (c.hidden, c.intermediate, c.vocab, c.n_layers) == (2048, 6144, 248320, 24)
    assert (c.heads, c.kv_heads, c.lin_k_heads, c.lin_v_heads) == (8, 2, 16, 16)
    assert [c.layer_is_attn[i] for i in range(8)] == [0, 0, 0, 1, 0, 0, 0, 1]
    assert c.rotary_dims == 64 and list(c.mrope) == [11, 11, 10]
    # the reference's own format (g128 pack, 512-point blocks with signs, ternary tied head) is accepted as is
    assert c.head_kind == 1 and c.group_size == 128 and not c.has_bias
    assert config.check(c) == (True, "")
    c4 = config.parse_config(open(os.path.join(os.path.dirname(__file__), "golden", "ref_config-4b.json")).read())
    assert (c4.hidden, c4.intermediate, c4.n_layers, c4.lin_v_heads) == (2560, 9216, 32, 32)
    assert config.check(c4) == (True, "")


def test_synth_is_deterministic_and_shaped():
    cfg = config.tiny()
    a = synth.model_tensors(cfg, 3)
    b = synth.model_tensors(cfg, 3)
    for (n1, c1, x1), (n2, c2, x2) in zip(a, b):
        assert n1 == n2 and c1 == c2 and np.array_equal(x1, x2)
    w = a.get("language_model.model.layers.0.mlp.down_proj.weight")
    codes = (w[..., None] >> (np.arange(16, dtype=np.uint32) * 2)) & 3
    counts = np.bincount(codes.ravel(), minlength=4)
    assert counts[3] == 0 and abs(counts[0] / counts.sum() - 1 / 3) < 0.01
    s = a.get("language_model.model.layers.0.mlp.down_proj.scales").view(np.float16).astype(np.float32)
    bias = a.get("language_model.model.layers.0.mlp.down_proj.biases").view(np.float16).astype(np.float32)
    assert s.min() >= 0.01 and s.max() <= 0.05 and np.array_equal(bias, -s)
    e = a.get("language_model.model.embed_tokens.weight").view(np.uint16)
    ev = (e.astype(np.uint32) << 16).view(np.float32)
    assert abs(ev.std() - 0.02) < 0.002 and abs(ev.mean()) < 0.002
    z = synth.zipf_tokens(1, 2000, 248320)
    assert z.max() < 248320 and np.mean(z == 0) > 0.05  # Zipf: the head token is frequent


def test_token_key_matches_oracle():
    L = _lib.lib()
    for b in [b" Sam", b"sam", b",", b"\n", b" hello\n", b"", b" ", b"x", b"Don't"]:
        buf = np.frombuffer(b, np.uint8) if b else np.zeros(1, np.uint8)
        assert L.bcu_token_key(buf.ctypes.data_as(ctypes.c_void_p), len(b)) == orc.token_key(b)


def test_lookup_matches_oracle():
    L = _lib.lib()
    rng = np.random.default_rng(0)
    keys = np.array([orc.token_key(b" w%d" % (i % 50)) for i in range(200)], np.uint64)
    for trial in range(200):
        src = rng.integers(0, 200, 60).astype(np.uint32)
        seq = np.concatenate([rng.integers(0, 200, 5), src[rng.integers(0, 55):][:rng.integers(1, 6)]]).astype(np.uint32)
        args = (int(rng.integers(1, 4)), 1, int(rng.integers(1, 9)), int(rng.integers(1, 20)), int(rng.integers(0, 60)))
        want, wpos = orc.lookup(src, seq, keys, *args)
        out = np.zeros(16, np.uint32)
        dpos = ctypes.c_int32()
        n = L.bcu_lookup(src.ctypes.data_as(_lib.PU32), len(src), seq.ctypes.data_as(_lib.PU32), len(seq),
                         keys.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), len(keys), *args,
                         out.ctypes.data_as(_lib.PU32), ctypes.byref(dpos))
        assert list(out[:n]) == list(want) and dpos.value == wpos


def test_policy_matches_oracle():
    L, O = _lib.lib(), orc.lib()
    rng = np.random.default_rng(1)
    for _ in range(200):
        cost = np.concatenate([[1.0], np.cumsum(rng.uniform(0.0, 0.7, 8)) + 1.0])
        cp = cost.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
        acc, rej = rng.uniform(0, 8), rng.uniform(0, 4)
        kmax, limit, gain = int(rng.integers(1, 9)), int(rng.integers(0, 9)), float(rng.choice([1.05, 1.15]))
        assert L.bcu_policy_choose(acc, rej, cp, kmax, limit, gain) == O.orc_policy_choose(acc, rej, cp, kmax, limit,
                                                                                           gain, None)
