"""GPU parity of whole passes on small random-init models, through the C ABI, against the oracle model.

Criteria: logits within 2e-3 absolute of the oracle (fp32 activations, hi/lo tensor-core products); argmax equal to
the oracle's unless the oracle's top-2 gap is below that tolerance; accept lengths exact; speculative decoding
token-identical to the build's own plain greedy decoding (every kernel is batch invariant)."""
import numpy as np
import pytest

from bonsai_b200 import _lib, synth
from bonsai_b200.config import tiny
from bonsai_b200.runtime import Model
from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3

CONFIGS = {
    "g64_bias_h512_signs": dict(group_size=64, has_bias=True, hadamard=512, has_signs=True),
    "g128_ref_pack": dict(group_size=128, has_bias=False, hadamard=512, has_signs=True, kv_heads=1),
    "g64_h1024_nosigns": dict(group_size=64, has_bias=True, hadamard=1024, has_signs=False, hidden=1024,
                              intermediate=2048, heads=4, lin_v_heads=8),
    # the reference's own format: g128 pack, 512-point blocks with signs, ternary tied embedding and head
    "reference_format": dict(group_size=128, has_bias=False, hadamard=512, has_signs=True, kv_heads=1, head_kind=1),
}


def build(name, seed=5):
    cfg = tiny(**CONFIGS[name])
    ts = synth.model_tensors(cfg, seed)
    return cfg, Model(cfg).load(ts), OracleModel(cfg, ts)


@pytest.fixture(scope="module", params=list(CONFIGS))
def pair(request, gpu):
    cfg, m, o = build(request.param)
    yield request.param, cfg, m, o
    m.close()


def prompt(cfg, n, seed=3):
    return synth.zipf_tokens(seed, n, cfg.vocab)


def check_logits(gl, ol, where):
    err = np.abs(gl - ol).max()
    assert err <= LOGIT_TOL, f"{where}: max logit error {err}"


def test_prefill_and_verify_logits(pair):
    name, cfg, m, o = pair
    m.reset()
    o.reset()
    ids = prompt(cfg, 37)
    assert m.prefill(ids) == o.prefill(ids)
    assert m.length == o.length == 37
    rows = np.concatenate([[ids[-1]], prompt(cfg, 8, seed=9)]).astype(np.uint32)
    m.keep_logits(True)
    pred, mm = m.verify(rows)
    opred, ol = o.forward(rows, logits=True)
    for t in range(len(rows)):
        check_logits(m.logits(t), ol[t], f"{name} row {t}")
        if pred[t] != opred[t]:
            top = np.sort(ol[t])[-2:]
            assert top[1] - top[0] < LOGIT_TOL, f"{name} row {t}: argmax differs with gap {top[1] - top[0]}"
    m.keep_logits(False)


@pytest.mark.parametrize("T", [1, 2, 4, 5, 8, 12, 16])
def test_verify_logits_every_width(pair, T):
    """Every verify width (the n-tile variants of the kernels) against the oracle."""
    name, cfg, m, o = pair
    m.reset()
    o.reset()
    ids = prompt(cfg, 19, seed=T)
    assert m.prefill(ids) == o.prefill(ids)
    rows = prompt(cfg, T, seed=100 + T).astype(np.uint32)
    m.keep_logits(True)
    pred, _ = m.verify(rows)
    opred, ol = o.forward(rows, logits=True)
    for t in range(T):
        check_logits(m.logits(t), ol[t], f"{name} T={T} row {t}")
    m.keep_logits(False)


def test_batch_invariance_bitwise(pair):
    """Row t of a verify pass has the same logits bit for bit whatever the pass width T (the property that makes
    speculative decoding token-identical to plain decoding)."""
    name, cfg, m, o = pair
    ids = prompt(cfg, 17, seed=31)
    m.reset()
    m.prefill(ids)
    snap = m.snapshot()
    rows = prompt(cfg, 16, seed=32).astype(np.uint32)
    m.keep_logits(True)
    ref = {}
    for T in (16, 9, 5, 4, 2, 1):
        m.restore(snap)
        m.verify(rows[:T])
        for t in range(T):
            lg = m.logits(t)
            if t in ref:
                assert np.array_equal(lg.view(np.uint32), ref[t].view(np.uint32)), f"{name}: row {t} differs at T={T}"
            else:
                ref[t] = lg
    m.keep_logits(False)
    snap.free()


def test_lookup_decode_repeatable(pair):
    name, cfg, m, o = pair
    ids = prompt(cfg, 30, seed=6)
    m.reset()
    first = m.prefill(ids)
    snap = m.snapshot()
    greedy, _ = m.decode(first, speculate=False, max_tokens=40)
    for rep in range(4):
        m.restore(snap)
        look, st = m.decode(first, user=ids, mode=_lib.DRAFT_LOOKUP, max_tokens=40)
        assert list(look) == list(greedy), f"{name} rep {rep}: verify calls {st.verify_calls} drafted {st.drafted}"
    snap.free()


def test_time_pass_keeps_state(pair):
    """The cost calibration (bcu_time_pass) restores the state it found."""
    name, cfg, m, o = pair
    ids = prompt(cfg, 23, seed=21)
    m.reset()
    first = m.prefill(ids)
    snap = m.snapshot()
    g1, _ = m.decode(first, speculate=False, max_tokens=10)
    m.restore(snap)
    for t in (1, 3, 9):
        m.time_pass(t, 2)
    g2, _ = m.decode(first, speculate=False, max_tokens=10)
    assert list(g1) == list(g2)
    snap.free()


def test_greedy_matches_oracle(pair):
    name, cfg, m, o = pair
    m.reset()
    o.reset()
    ids = prompt(cfg, 21, seed=4)
    first = m.prefill(ids)
    assert first == o.prefill(ids)
    g, _ = m.decode(first, speculate=False, max_tokens=24)
    og = o.greedy(first, 24)
    assert list(g) == list(og)


def test_spec_equals_greedy_all_modes(pair):
    name, cfg, m, o = pair
    ids = prompt(cfg, 30, seed=6)
    m.reset()
    first = m.prefill(ids)
    snap = m.snapshot()
    greedy, _ = m.decode(first, speculate=False, max_tokens=40)
    m.restore(snap)
    planted, st = m.decode(first, mode=_lib.DRAFT_PLANTED, planted=greedy[1:], max_tokens=40, draft_max=8)
    assert list(planted) == list(greedy)
    assert st.accepted == st.drafted  # 100% acceptance
    m.restore(snap)
    rnd, st = m.decode(first, mode=_lib.DRAFT_RANDOM, seed=11, max_tokens=40, draft_max=8)
    assert list(rnd) == list(greedy)
    m.restore(snap)
    look, st = m.decode(first, user=ids, mode=_lib.DRAFT_LOOKUP, max_tokens=40)
    assert list(look) == list(greedy)
    snap.free()


@pytest.mark.parametrize("m_acc", list(range(9)))
def test_rollback_every_accept_length(pair, m_acc):
    """Drafts whose first m_acc tokens are the greedy continuation: the device accept length is exactly m_acc, and
    decoding after the partial accept continues on the greedy path (the rollback of KV and GDN state is exact)."""
    name, cfg, m, o = pair
    ids = prompt(cfg, 25, seed=8)
    m.reset()
    first = m.prefill(ids)
    snap = m.snapshot()
    greedy, _ = m.decode(first, speculate=False, max_tokens=20)
    m.restore(snap)
    drafts = list(greedy[1:1 + m_acc]) + [(int(greedy[1 + m_acc]) + 1) % cfg.vocab] + [3] * (7 - m_acc)
    rows = np.array([first] + drafts[:8], np.uint32)
    pred, acc = m.verify(rows)
    assert acc == m_acc
    assert list(pred[: m_acc + 1]) == list(greedy[1: m_acc + 2])
    nxt, _ = m.decode(int(pred[acc]), speculate=False, max_tokens=6)
    assert list(nxt) == list(greedy[m_acc + 1: m_acc + 7])
    snap.free()


def test_accept_override_and_flush(pair):
    name, cfg, m, o = pair
    ids = prompt(cfg, 20, seed=12)
    m.reset()
    first = m.prefill(ids)
    snap = m.snapshot()
    greedy, _ = m.decode(first, speculate=False, max_tokens=12)
    m.restore(snap)
    rows = np.array([first] + list(greedy[1:9]), np.uint32)
    pred, acc = m.verify(rows)
    assert acc == 8
    m.accept(9, 3)  # keep only 3 rows: the next input is greedy[3]
    assert m.length == 20 + 3
    m.flush()
    nxt, _ = m.decode(int(greedy[3]), speculate=False, max_tokens=5)
    assert list(nxt) == list(greedy[3:8])
    snap.free()


def test_snapshot_parts_roundtrip(pair):
    name, cfg, m, o = pair
    ids = prompt(cfg, 18, seed=13)
    m.reset()
    first = m.prefill(ids)
    s = m.snapshot()
    sizes, n = s.parts()
    assert n == 18 and sizes[2] == sizes[3]
    parts = [s.read(i) for i in range(4)]
    g1, _ = m.decode(first, speculate=False, max_tokens=8)
    s2 = m.new_snapshot(n)
    for i in range(4):
        s2.write(i, parts[i].tobytes())
    m.restore(s2)
    g2, _ = m.decode(first, speculate=False, max_tokens=8)
    assert list(g1) == list(g2)
    s.free()
    s2.free()


def test_errors_are_reported(gpu):
    cfg = tiny(ctx=48)
    m = Model(cfg).load(synth.model_tensors(cfg, 1))
    with pytest.raises(Exception):
        m.prefill(np.zeros(60, np.uint32))  # context full
    m.reset()
    with pytest.raises(Exception):
        m.step(cfg.vocab + 5)  # token out of range
    m.reset()
    assert m.prefill(np.arange(10, dtype=np.uint32)) < cfg.vocab  # the model still works after the errors
    m.close()


def synthetic_vocab(V):
    """Token bytes for a V-id vocabulary: a few words normalize_draft rewrites, sentence ends, and lowercase words."""
    special = [b" i", b" I", b" dont", b" don", b"'t", b" monday", b" Monday", b".", b" um", b" hello", b" Hello"]
    return special + [b" w%d" % i for i in range(V - len(special))]


def test_lookup_decode_with_vocab_fillers_normalize_and_emit(pair):
    """Lookup drafting with the token bytes, the default filler ids, a tokenizer for normalize_draft and streaming
    emission: the output still equals greedy decoding token for token, and the emitted ids are the output, in order."""
    name, cfg, m, o = pair
    tb = synthetic_vocab(cfg.vocab)
    index = {b: i for i, b in enumerate(tb)}
    m.set_vocab_bytes(tb)
    m.set_encoder(lambda text: [index[text]] if text in index else ([index[b" don"], index[b"'t"]]
                                                                      if text == b" don't" else None))
    got = []
    m.set_emit(got.append)
    try:
        ids = np.concatenate([prompt(cfg, 24, seed=6), np.array([7, 0, 2, 5, 9, 8], np.uint32)])
        m.reset()
        first = m.prefill(ids)
        snap = m.snapshot()
        m.set_emit(None)
        greedy, _ = m.decode(first, speculate=False, max_tokens=32)
        m.set_emit(got.append)
        m.restore(snap)
        look, st = m.decode(first, user=ids, mode=_lib.DRAFT_LOOKUP, max_tokens=32)
        assert list(look) == list(greedy)
        assert got == [int(t) for t in look]
        snap.free()
    finally:
        m.set_emit(None)
        m.set_encoder(None)
        m.set_vocab_bytes([])


def test_models_on_concurrent_host_threads(gpu):
    """Serving several sessions at once (the config-5 bench's form): model instances on their own streams, each driven
    by its own host thread, give the tokens they give when run one after another (batched prefill of 100 tokens,
    then speculative decode with planted drafts)."""
    import concurrent.futures

    cfg = tiny(**CONFIGS["g64_bias_h512_signs"])
    ts = synth.model_tensors(cfg, 12)
    models = [Model(cfg).load(ts) for _ in range(3)]
    prompts = [prompt(cfg, 100, seed=20 + i) for i in range(3)]

    def session(i):
        m = models[i]
        m.reset()
        first = m.prefill(prompts[i])
        g, _ = m.decode(first, speculate=False, max_tokens=20)
        m.reset()
        m.prefill(prompts[i])
        s, _ = m.decode(first, mode=_lib.DRAFT_PLANTED, planted=g[1:], max_tokens=20, draft_max=8)
        return first, list(g), list(s)

    try:
        alone = [session(i) for i in range(3)]
        with concurrent.futures.ThreadPoolExecutor(3) as ex:
            for _ in range(2):
                together = list(ex.map(session, range(3)))
                assert together == alone
        for first, g, s in alone:
            assert g == s
    finally:
        for m in models:
            m.close()
