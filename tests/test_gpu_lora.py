"""LoRA through the C ABI on the GPU (lora.rs, config 4's adapter on q/k/v/o and gate/up/down, or on every linear):
verify-pass logits against the oracle with the same adapter, both operand paths (built across the grid, built per
CTA), bitwise batch invariance, speculative decoding token-identical to greedy, removal, partial adapters, odd
ranks, the adapter-file path and the errors of lora::load.

Criteria: logits within 2e-3 absolute of the oracle (as the base model's tests); everything else bit- or
token-exact."""
import json

import numpy as np
import pytest

from bonsai_b200 import _lib, lora, synth
from bonsai_b200.config import tiny
from bonsai_b200.runtime import BackendError, Model
from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3
CONFIGS = {
    "g64_bias_h512_signs": dict(group_size=64, has_bias=True, hadamard=512, has_signs=True),
    "g128_ref_pack": dict(group_size=128, has_bias=False, hadamard=512, has_signs=True, kv_heads=1),
    "g64_h1024_nosigns": dict(group_size=64, has_bias=True, hadamard=1024, has_signs=False, hidden=1024,
                              intermediate=2048, heads=4, lin_v_heads=8),
    # the 4B shape's hidden size (2560 = 5 rotation blocks; the head's ring has fewer stages) and kv heads
    "g64_h2560_4b_widths": dict(group_size=64, has_bias=True, hadamard=512, has_signs=True, hidden=2560,
                                intermediate=1536, heads=4, kv_heads=4, lin_v_heads=4),
}


@pytest.fixture(scope="module", params=list(CONFIGS))
def setup(request, gpu):
    cfg = tiny(**CONFIGS[request.param])
    ts = synth.model_tensors(cfg, 21)
    m = Model(cfg).load(ts)
    o = OracleModel(cfg, ts)
    yield request.param, cfg, ts, m, o
    m.close()


def verify_logits(m, ids, rows):
    m.reset()
    m.prefill(ids)
    m.keep_logits(True)
    m.verify(rows)
    out = np.stack([m.logits(t) for t in range(len(rows))])
    m.keep_logits(False)
    return out


def oracle_logits(o, ids, rows):
    o.reset()
    o.prefill(ids)
    return o.forward(rows, logits=True)[1]


@pytest.mark.parametrize("local", [False, True])
def test_lora_logits_match_oracle(setup, local):
    name, cfg, ts, m, o = setup
    ids = synth.zipf_tokens(3, 29, cfg.vocab)
    rows = synth.zipf_tokens(4, 9, cfg.vocab)
    base = verify_logits(m, ids, rows)
    lins = synth.lora_linears(cfg, 16, seed=9, std_b=0.05)
    m.set_lora_linears(lins, 2.0)
    o.set_lora(lins, 2.0)
    try:
        m.set_local_build(local)
        got = verify_logits(m, ids, rows)
        want = oracle_logits(o, ids, rows)
        err = np.abs(got - want).max()
        assert err <= LOGIT_TOL, f"{name}: max logit error {err}"
        assert np.abs(got - base).max() > 20 * LOGIT_TOL, "the adapter did not change the logits"
    finally:
        m.set_local_build(False)
        m.set_lora_linears([], 1.0)
        o.clear_lora()
    # removed: bit-identical to the base model again
    assert np.array_equal(verify_logits(m, ids, rows).view(np.uint32), base.view(np.uint32))


def test_lora_batch_invariant_and_spec_equals_greedy(setup):
    name, cfg, ts, m, o = setup
    m.set_lora_linears(synth.lora_linears(cfg, 16, seed=10, std_b=0.05), 2.0)
    try:
        ids = synth.zipf_tokens(5, 17, cfg.vocab)
        m.reset()
        m.prefill(ids)
        snap = m.snapshot()
        rows = synth.zipf_tokens(6, 16, cfg.vocab).astype(np.uint32)
        m.keep_logits(True)
        ref = {}
        for T in (16, 9, 4, 1):
            m.restore(snap)
            m.verify(rows[:T])
            for t in range(T):
                lg = m.logits(t)
                if t in ref:
                    assert np.array_equal(lg.view(np.uint32), ref[t].view(np.uint32)), f"{name}: row {t} at T={T}"
                else:
                    ref[t] = lg
        m.keep_logits(False)
        m.restore(snap)
        first = m.prefill(ids[-3:])
        snap2 = m.snapshot()
        greedy, _ = m.decode(first, speculate=False, max_tokens=40)
        m.restore(snap2)
        look, _ = m.decode(first, user=ids, mode=_lib.DRAFT_LOOKUP, max_tokens=40)
        m.restore(snap2)
        planted, st = m.decode(first, mode=_lib.DRAFT_PLANTED, planted=greedy[1:], max_tokens=40, draft_max=8)
        assert list(look) == list(greedy) and list(planted) == list(greedy)
        assert st.accepted == st.drafted
        snap.free()
        snap2.free()
    finally:
        m.set_lora_linears([], 1.0)


def test_partial_adapter_and_odd_rank(setup):
    """Config 4's module set (attention q/k/v/o + MLP; GDN projections unadapted), rank 5 (zero-padded to 8), and a
    group with one member missing (only q_proj and v_proj): the missing member gets zero rows."""
    name, cfg, ts, m, o = setup
    ids = synth.zipf_tokens(7, 21, cfg.vocab)
    rows = synth.zipf_tokens(8, 6, cfg.vocab)
    mods = {"self_attn.q_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj",
            "mlp.down_proj"}
    lins = synth.lora_linears(cfg, 5, seed=11, std_b=0.05, modules=mods)
    m.set_lora_linears(lins, 2.0)
    o.set_lora(lins, 2.0)
    try:
        assert m.lora_info() == (len(lins), 5)
        err = np.abs(verify_logits(m, ids, rows) - oracle_logits(o, ids, rows)).max()
        assert err <= LOGIT_TOL, f"{name}: max logit error {err}"
    finally:
        m.set_lora_linears([], 1.0)
        o.clear_lora()
    assert m.lora_info() is None


def test_adapter_file_path(setup, tmp_path):
    """Model.set_lora(path, scale) on a PEFT file: the same logits as the tensors with fold = alpha / r x scale; the
    adapter id changes the prefix identity."""
    name, cfg, ts, m, o = setup
    lins = synth.lora_linears(cfg, 16, seed=12, std_b=0.05, modules={"mlp.down_proj", "mlp.up_proj"})
    p = str(tmp_path / "adapter_model.safetensors")
    lora.write_safetensors(p, {f"base_model.model.model.layers.{l}.{mod}.lora_{w}.weight": (a if w == "A" else b)
                               for l, mod, a, b in lins for w in "AB"})
    open(tmp_path / "adapter_config.json", "w").write(json.dumps({"r": 16, "lora_alpha": 32}))
    ids = synth.zipf_tokens(9, 19, cfg.vocab)
    rows = synth.zipf_tokens(10, 5, cfg.vocab)
    try:
        m.set_lora(p, 0.5)
        assert m.adapter == lora.adapter_id(p, 0.5) and m.adapter != 0
        from_file = verify_logits(m, ids, rows)
        m.set_lora_linears(lins, 1.0)  # alpha / r = 2, times 0.5
        direct = verify_logits(m, ids, rows)
        assert np.array_equal(from_file.view(np.uint32), direct.view(np.uint32))
    finally:
        m.set_lora(None)
    assert m.adapter == 0 and m.lora_info() is None


def test_lora_errors_keep_installed_adapter(setup):
    name, cfg, ts, m, o = setup
    lins = synth.lora_linears(cfg, 8, seed=13, modules={"mlp.down_proj"})
    m.set_lora_linears(lins, 1.0)
    try:
        l0, mod0, a0, b0 = lins[0]
        bad = {
            "unsupported modules": [(0, "mlp.nope", a0, b0)],
            "linear is": [(l0, mod0, a0[:, :-1], b0)],
            "mixed ranks": [lins[0], (lins[1][0], lins[1][1], lins[1][2][:4], lins[1][3][:, :4])],
            "given twice": [lins[0], lins[0]],
        }
        for what, ls in bad.items():
            with pytest.raises(BackendError) as e:
                m.set_lora_linears(ls, 1.0)
            assert e.value.status == _lib.ERR_ARG and what in e.value.message, (what, e.value.message)
            assert m.lora_info() == (len(lins), 8)  # unchanged
    finally:
        m.set_lora_linears([], 1.0)


def test_lora_batched_prefill_matches_oracle(setup):
    """A 150-token prompt with the adapter runs through the batched prefill (tcgen05 GEMM chunks plus the adapter's
    A and B kernels): the next token and the verify-pass logits after it match the oracle with the same adapter."""
    name, cfg, ts, m, o = setup
    if cfg.ctx < 170:
        pytest.skip("context too short for a batched prefill")
    ids = synth.zipf_tokens(13, 150, cfg.vocab)
    rows = synth.zipf_tokens(14, 9, cfg.vocab)
    lins = synth.lora_linears(cfg, 16, seed=9, std_b=0.05)
    m.set_lora_linears(lins, 2.0)
    o.set_lora(lins, 2.0)
    try:
        m.reset()
        o.reset()
        assert m.prefill(ids) == o.prefill(ids)
        m.keep_logits(True)
        m.verify(rows)
        got = np.stack([m.logits(t) for t in range(len(rows))])
        m.keep_logits(False)
        want = o.forward(rows, logits=True)[1]
        err = np.abs(got - want).max()
        assert err <= LOGIT_TOL, f"{name}: max logit error {err}"
    finally:
        m.set_lora_linears([], 1.0)
        o.clear_lora()
