"""Saved prefix files (BNSPFX01) through the C ABI on the GPU: identity, save, load into a fresh model, and the
decode after a loaded prefix token-identical to the decode after the in-memory snapshot (runtime/mod.rs:455-578;
the reference's integration test reloads saved prefix files in a fresh load, tests/bonsai_golden.rs:90-113).
Bit-exact: file bytes against oracle/prefix_file.py, the state parts after a load, the token streams."""
import os
import sys

import numpy as np
import pytest

from bonsai_b200 import synth
from bonsai_b200 import runtime as rt
from bonsai_b200.config import tiny
from bonsai_b200.runtime import Model
from oracle import prefix_file as pf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(gpu, tmp_path_factory):
    d = tmp_path_factory.mktemp("model")
    weights, config = str(d / "model.safetensors"), str(d / "config.json")
    open(weights, "wb").write(b"\0" * 1000)
    open(config, "w").write('{"hidden_size": 512}')
    cfg = tiny()
    ts = synth.model_tensors(cfg, 11)
    m = Model(cfg).load(ts)
    yield cfg, ts, m, weights, config
    m.close()


def shape_words(cfg):
    n_attn = sum(cfg.layer_is_attn[i] for i in range(cfg.n_layers))
    return [cfg.n_layers - n_attn, n_attn, cfg.hidden, cfg.kv_heads * 256,
            2 * cfg.lin_k_heads * 128 + cfg.lin_v_heads * 128]


def test_identity_layout(setup):
    cfg, ts, m, weights, config = setup
    ident = m.prefix_identity(7, weights, config)
    want = pf.identity(rt.kernel_hash(), 7, "/proc/self/exe", weights, config, shape_words(cfg), m.device_name())
    assert ident == want
    assert m.prefix_identity(7, weights, config, exe=sys.executable) == want
    assert m.prefix_identity(8, weights, config) != want  # the adapter is part of it
    assert m.prefix_identity(7, weights + ".missing", config) is None  # unreadable part: no identity


def test_save_load_fresh_model(setup, tmp_path):
    cfg, ts, m, weights, config = setup
    d = str(tmp_path)
    ident = m.prefix_identity(0, weights, config)
    prefix = synth.zipf_tokens(21, 45, cfg.vocab)
    user = synth.zipf_tokens(22, 12, cfg.vocab)
    m.reset()
    m.prefill(prefix)
    snap = m.snapshot()
    m.save_prefix(snap, d, ident, prefix)
    path = rt.prefix_path(d, ident, prefix)
    parts = [snap.read(i).tobytes() for i in range(4)]
    assert open(path, "rb").read() == pf.file_bytes(ident, prefix, len(prefix), parts)
    # the continuation from the in-memory snapshot
    m.restore(snap)
    first = m.prefill(user)
    want, _ = m.decode(first, user=np.concatenate([prefix, user]), max_tokens=24)
    # a fresh model loads the file: same parts, same continuation
    m2 = Model(cfg).load(ts)
    try:
        snap2 = m2.load_prefix(d, ident, prefix)
        assert snap2 is not None
        assert [snap2.read(i).tobytes() for i in range(4)] == parts
        m2.restore(snap2)
        assert m2.length == len(prefix)
        first2 = m2.prefill(user)
        got, _ = m2.decode(first2, user=np.concatenate([prefix, user]), max_tokens=24)
        assert first2 == first and list(got) == list(want)
        # misses: other ids, another identity, a truncated file
        assert m2.load_prefix(d, ident, prefix[:-1]) is None
        assert m2.load_prefix(d, ident[:-1] + b"?", prefix) is None
        data = open(path, "rb").read()
        open(path, "wb").write(data[:-4])
        assert m2.load_prefix(d, ident, prefix) is None
        open(path, "wb").write(data)
        assert m2.load_prefix(d, ident, prefix) is not None
    finally:
        m2.close()


def test_background_save(setup, tmp_path):
    cfg, ts, m, weights, config = setup
    d = str(tmp_path / "bg")
    ident = m.prefix_identity(0, weights, config)
    prefix = synth.zipf_tokens(23, 30, cfg.vocab)
    m.reset()
    m.prefill(prefix)
    snap = m.snapshot()
    m.save_prefix(snap, d, ident, prefix, background=True)
    rt.wait_saves()
    parts = [snap.read(i).tobytes() for i in range(4)]
    assert open(rt.prefix_path(d, ident, prefix), "rb").read() == pf.file_bytes(ident, prefix, len(prefix), parts)


def test_config_change_invalidates(setup, tmp_path):
    cfg, ts, m, weights, config = setup
    d = str(tmp_path)
    prefix = synth.zipf_tokens(24, 20, cfg.vocab)
    ident = m.prefix_identity(0, weights, config)
    m.reset()
    m.prefill(prefix)
    m.save_prefix(m.snapshot(), d, ident, prefix)
    cfg2 = os.path.join(d, "config2.json")
    open(cfg2, "w").write('{"hidden_size": 513}')
    ident2 = m.prefix_identity(0, weights, cfg2)
    assert ident2 != ident and m.load_prefix(d, ident2, prefix) is None
    assert m.load_prefix(d, ident, prefix) is not None


def test_start_prefix_memory_then_file(setup, tmp_path):
    """start_prefix: a miss prefills and saves; a repeat is served from a memory slot; a fresh model is served from
    the saved file; the slots keep the newest three prefixes."""
    cfg, ts, m, weights, config = setup
    d = str(tmp_path)
    ident = m.prefix_identity(0, weights, config)
    m.prefixes.clear()
    m.set_prefix_files(d, ident)
    prefixes = [synth.zipf_tokens(30 + k, 16 + k, cfg.vocab) for k in range(4)]
    try:
        def aged(k):  # distinct explicit ages, oldest first, so pruning does not depend on timestamp resolution
            rt.wait_saves()
            t = 1_000_000_000_000 + k * 10**9
            os.utime(rt.prefix_path(d, ident, prefixes[k]), ns=(t, t))

        assert m.start_prefix(prefixes[0]) == 0
        aged(0)
        assert m.length == len(prefixes[0])
        nxt = m.prefill(prefixes[1][:3])
        assert m.start_prefix(prefixes[0]) == len(prefixes[0])  # memory slot
        assert m.prefill(prefixes[1][:3]) == nxt
        for k in (1, 2):
            assert m.start_prefix(prefixes[k]) == 0
            aged(k)
        assert m.start_prefix(prefixes[3]) == 0  # its save prunes the oldest file (prefix 0)
        rt.wait_saves()
        assert [ids for ids, _, _ in m.prefixes] == [list(map(int, p)) for p in prefixes[::-1][:3]]
        assert len([f for f in os.listdir(d) if f.endswith(".prefix")]) == 3
        m2 = Model(cfg).load(ts)
        try:
            m2.set_prefix_files(d, ident)
            assert m2.start_prefix(prefixes[3]) == len(prefixes[3])  # from the file
            got = m2.prefill(prefixes[0][:5])
            assert m.start_prefix(prefixes[3]) == len(prefixes[3])  # memory slot of the first model
            assert m.prefill(prefixes[0][:5]) == got
            assert m2.start_prefix(prefixes[0]) == 0  # its file was pruned (oldest of four)
            rt.wait_saves()
        finally:
            m2.prefixes.clear()
            m2.close()
    finally:
        m.set_prefix_files(None, None)
        m.prefixes.clear()
