"""Batched prefill (the tcgen05 GEMM chunks of bcu_prefill) against the oracle and against prefill by verify passes.

Prompts longer than 64 tokens run every row but the last through chunks of up to 512 rows (producer kernels, the
ternary GEMM on tcgen05, the chunk's GatedDeltaNet conv + recurrence and causal attention), then the last row as a
one-row pass. Criteria: the next token equals the oracle's, the greedy continuation after it equals the oracle's token
for token, a verify pass at the end of the prompt has logits within 2e-3 of the oracle's, and the state the chunks
leave (GDN state, conv rows, K/V) matches the state verify-pass prefill leaves within a stated tolerance.
"""
import numpy as np
import pytest

from bonsai_b200 import synth
from bonsai_b200.config import make_config, tiny
from bonsai_b200.runtime import Model
from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3

CONFIGS = {
    "g64_bias_h512_signs": dict(group_size=64, has_bias=True, hadamard=512, has_signs=True),
    "reference_format": dict(group_size=128, has_bias=False, hadamard=512, has_signs=True, kv_heads=1, head_kind=1),
    "g64_h1024_nosigns": dict(group_size=64, has_bias=True, hadamard=1024, has_signs=False, hidden=1024,
                              intermediate=2048, heads=4, lin_v_heads=8),
}


@pytest.fixture(scope="module", params=list(CONFIGS))
def pair(request, gpu):
    cfg = tiny(ctx=1200, **CONFIGS[request.param])
    ts = synth.model_tensors(cfg, 9)
    m = Model(cfg).load(ts)
    yield request.param, cfg, m, OracleModel(cfg, ts)
    m.close()


@pytest.mark.parametrize("n", [65, 700])
def test_batched_prefill_matches_oracle(pair, n):
    """65 tokens: one chunk of 64 rows; 700: chunks of 512 and 187 rows."""
    name, cfg, m, o = pair
    ids = synth.zipf_tokens(40 + n, n, cfg.vocab)
    m.reset()
    o.reset()
    first = m.prefill(ids)
    assert m.length == n
    assert first == o.prefill(ids, chunk=16), name
    g, _ = m.decode(first, speculate=False, max_tokens=12)
    assert list(g) == list(o.greedy(first, 12)), name
    # a verify pass on the state the chunks left
    m.reset()
    o.reset()
    m.prefill(ids)
    o.prefill(ids, chunk=16)
    rows = synth.zipf_tokens(7, 9, cfg.vocab).astype(np.uint32)
    m.keep_logits(True)
    m.verify(rows)
    _, ol = o.forward(rows, logits=True)
    for t in range(9):
        err = float(np.abs(m.logits(t) - ol[t]).max())
        assert err <= LOGIT_TOL, f"{name} n={n} row {t}: {err}"
    m.keep_logits(False)


def test_batched_state_matches_verify_pass_prefill(pair):
    name, cfg, m, o = pair
    ids = synth.zipf_tokens(5, 300, cfg.vocab)
    parts = {}
    for batched in (True, False):
        m.set_batched_prefill(batched)
        m.reset()
        nxt = m.prefill(ids)
        s = m.snapshot()
        parts[batched] = (nxt, [np.frombuffer(s.read(i).tobytes(), np.float32) for i in range(4)])
        s.free()
    m.set_batched_prefill(True)
    assert parts[True][0] == parts[False][0]
    for i, what in enumerate(["gdn state", "conv rows", "K cache", "V cache"]):
        a, b = parts[True][1][i], parts[False][1][i]
        scale = max(float(np.abs(b).max()), 1e-6)
        assert np.abs(a - b).max() <= 2e-4 * scale, f"{name}: {what} differs by {np.abs(a - b).max()} (scale {scale})"


def test_graded_shape_batched_prefill_equals_verify_pass_prefill(gpu):
    """The benchmark's widths (hidden 2048, 16 q / 2 kv heads, GDN 16/32, vocab 248320) on 4 layers: a 1300-token
    prompt prefilled by chunks and by verify passes gives the same next token, close states and close logits of the
    verify pass that follows."""
    cfg = make_config(2048, 6144, 248320, 4, 16, 2, 16, 32, ctx=2048)
    ts = synth.model_tensors(cfg, 31)
    m = Model(cfg).load(ts)
    try:
        ids = synth.zipf_tokens(77, 1300, cfg.vocab)
        rows = synth.zipf_tokens(78, 9, cfg.vocab).astype(np.uint32)
        out = {}
        for batched in (True, False):
            m.set_batched_prefill(batched)
            m.reset()
            nxt = m.prefill(ids)
            s = m.snapshot()
            st = [np.frombuffer(s.read(i).tobytes(), np.float32) for i in range(4)]
            s.free()
            m.keep_logits(True)
            pred, _ = m.verify(rows)
            lg = np.stack([m.logits(t) for t in range(9)])
            m.keep_logits(False)
            out[batched] = (nxt, st, pred, lg)
        assert out[True][0] == out[False][0]
        for i in range(4):
            a, b = out[True][1][i], out[False][1][i]
            assert np.abs(a - b).max() <= 2e-4 * max(float(np.abs(b).max()), 1e-6), f"state part {i}"
        assert np.abs(out[True][3] - out[False][3]).max() <= LOGIT_TOL
    finally:
        m.set_batched_prefill(True)
        m.close()


@pytest.mark.parametrize("shape", [dict(heads=4, kv_heads=4, lin_k_heads=4, lin_v_heads=4),
                                   dict(heads=16, kv_heads=1, lin_k_heads=1, lin_v_heads=4)])
def test_chunk_kernels_other_head_ratios(gpu, shape):
    """The chunk attention at one query head per kv head (32-row blocks) and at 16 (2-row blocks), the chunked
    recurrence at one value head per key head and at four: batched prefill of 300 tokens leaves the state that
    verify-pass prefill leaves, and the verify pass that follows matches the oracle."""
    cfg = tiny(ctx=512, **shape)
    ts = synth.model_tensors(cfg, 17)
    m = Model(cfg).load(ts)
    o = OracleModel(cfg, ts)
    try:
        ids = synth.zipf_tokens(8, 300, cfg.vocab)
        parts = {}
        for batched in (True, False):
            m.set_batched_prefill(batched)
            m.reset()
            nxt = m.prefill(ids)
            s = m.snapshot()
            parts[batched] = (nxt, [np.frombuffer(s.read(i).tobytes(), np.float32) for i in range(4)])
            s.free()
        assert parts[True][0] == parts[False][0]
        for i in range(4):
            a, b = parts[True][1][i], parts[False][1][i]
            assert np.abs(a - b).max() <= 2e-4 * max(float(np.abs(b).max()), 1e-6), f"state part {i}"
        m.set_batched_prefill(True)
        m.reset()
        o.reset()
        assert m.prefill(ids) == o.prefill(ids, chunk=16)
        rows = synth.zipf_tokens(9, 9, cfg.vocab).astype(np.uint32)
        m.keep_logits(True)
        m.verify(rows)
        _, ol = o.forward(rows, logits=True)
        for t in range(9):
            assert float(np.abs(m.logits(t) - ol[t]).max()) <= LOGIT_TOL
        m.keep_logits(False)
    finally:
        m.set_batched_prefill(True)
        m.close()
