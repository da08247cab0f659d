"""The oracle pinned to the reference itself: the reference's own Metal text kernels (src/bonsai/runtime/kernels.metal,
compiled for the host by oracle/Makefile through oracle/ref_metal/metal_stdlib, run by oracle/ref_metal/ref_runtime)
against the oracle's restatement of the same steps, kernel by kernel and for whole passes of a model in the
reference's own format (g128 pack without bias, 512-point rotation blocks with signs, ternary tied embedding and head,
4 query heads per KV head).

Criteria: element-wise producers with no reduction (swiglu_rotate, gate_rotate, embed) and argmax ties are bit-exact;
where a kernel reduces, the reference's order differs from the oracle's (SIMD-group butterflies, 8-wide matrix
products) and the bound is stated per test. Skips when the reference tree was not there to compile (the GPU box).
"""
import numpy as np
import pytest

from bonsai_b200 import synth
from bonsai_b200.config import make_config
from oracle import oracle as orc
from oracle import ref

pytestmark = pytest.mark.skipif(not ref.available(), reason="reference kernels not built (no reference tree)")


def rng(seed):
    return np.random.default_rng(seed)


def signs_of(n, seed):
    return np.where(rng(seed).random(n) < 0.5, -1.0, 1.0).astype(np.float32)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_swiglu_and_gate_rotate_bit_exact():
    r = rng(1)
    T, D = 5, 2048
    g, u = r.standard_normal((2, T, D)).astype(np.float32)
    s = signs_of(D, 2)
    assert np.array_equal(bits(ref.swiglu_rotate(g, u, s)), bits(orc.swiglu_rotate(g, u, s)))
    W = 1024
    attn = r.standard_normal((T, W)).astype(np.float32)
    qp = r.standard_normal((T, 2 * W)).astype(np.float32)
    s = signs_of(W, 3)
    assert np.array_equal(bits(ref.gate_rotate(attn, qp, s)), bits(orc.gate_rotate(attn, qp, s)))


def test_norm_rotate_and_gated_norm_rotate():
    """The row norms reduce (row_ss's 16 partials, gated4's simd_sum): 2e-6 relative to the row's size."""
    r = rng(4)
    T, D = 3, 2048
    h = (r.standard_normal((T, D)) * 3).astype(np.float32)
    w = r.uniform(0.8, 1.2, D).astype(np.float32)
    s = signs_of(D, 5)
    xn_r, xr_r = ref.norm_rotate(h, w, s, write_xn=1)
    xn_o, xr_o = orc.norm_rotate(h, w, s)
    assert np.abs(xn_r - xn_o).max() <= 2e-6 * np.abs(xn_o).max()
    assert np.abs(xr_r - xr_o).max() <= 2e-6 * np.abs(xr_o).max()
    W = 2048
    y, z = r.standard_normal((2, T, W)).astype(np.float32)
    gw = r.uniform(0.8, 1.2, 128).astype(np.float32)
    s = signs_of(W, 6)
    a, b = ref.gated_norm_rotate(y, z, gw, s), orc.gated_norm_rotate(y, z, gw, s)
    assert np.abs(a - b).max() <= 2e-6 * np.abs(b).max()


def test_embed_bit_exact():
    r = rng(7)
    V, d = 64, 1024
    W = r.integers(0, 2**32, (V, d // 16), dtype=np.uint64).astype(np.uint32)
    S = r.uniform(0.01, 0.05, (V, d // 128)).astype(np.float16).view(np.uint16)
    s = signs_of(d, 8)
    ids = np.array([0, 5, 63, 17, 5], np.int32)
    got = ref.embed(W, S, s, ids, d)
    want = orc.embed_ternary(W, S, None, s, 128, 512, d, ids)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("T", [1, 2, 3, 4, 8, 9, 16, 17, 33])
def test_ternary_matmul_every_reference_kernel(T):
    """qmv4 (T = 1), qmvr (2, 3), qmvxm in 8-row slices (4..16) and qmm (> 16) against the oracle's qmv_rows form:
    |dy| <= 1e-5 sum_k |w_k x_k| + 1e-6; the add flag accumulates onto y."""
    r = rng(10 + T)
    O, K = 256, 1024
    W = r.integers(0, 2**32, (O, K // 16), dtype=np.uint64).astype(np.uint32)
    S = r.uniform(0.01, 0.05, (O, K // 128)).astype(np.float16).view(np.uint16)
    x = r.standard_normal((T, K)).astype(np.float32)
    got = ref.ternary_matmul(W, S, x)
    want = orc.ternary_linear(W, S, None, 128, x)
    codes = np.stack([(W >> (2 * e)) & 3 for e in range(16)], -1).reshape(O, K).astype(np.float64) - 1.0
    scale = np.repeat(S.view(np.float16).astype(np.float64), 128, axis=1)
    bound = 1e-5 * (np.abs(x).astype(np.float64) @ np.abs(codes * scale).T) + 1e-6
    assert np.all(np.abs(got - want) <= bound)
    y0 = r.standard_normal((T, O)).astype(np.float32)
    got2 = ref.ternary_matmul(W, S, x, y0)
    assert np.all(np.abs(got2 - (want + y0)) <= bound + 1e-6 * np.abs(y0))


@pytest.mark.parametrize("NK,NV,T", [(4, 16, 9), (16, 16, 5), (2, 8, 1)])
def test_gdn_recurrent(NK, NV, T):
    """gdn_gates + gdn_recurrent (kernels.metal:556-622) against the oracle's delta rule: rtol 2e-5 on y and state."""
    r = rng(20 + T)
    C = (2 * NK + NV) * 128
    q = r.standard_normal((T, NK, 128)).astype(np.float32)
    k = r.standard_normal((T, NK, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True) * np.sqrt(128)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = r.standard_normal((T, NV, 128)).astype(np.float32)
    a, b = r.standard_normal((2, T, NV)).astype(np.float32)
    alog = r.uniform(-0.5, 0.5, NV).astype(np.float32)
    dtb = r.uniform(-0.5, 0.5, NV).astype(np.float32)
    st = (r.standard_normal((NV, 128, 128)) * 0.02).astype(np.float32)
    qkvc = np.concatenate([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], 1)
    assert qkvc.shape == (T, C)
    ab = np.concatenate([a, b], 1)
    y_r, st_r = ref.gdn_recurrent(qkvc, ab, alog, dtb, st, NK, NV)
    y_o, st_o = orc.gdn_verify(q, k, v, a, b, alog, dtb, st, T)
    assert np.abs(y_r - y_o.reshape(T, -1)).max() <= 2e-5 * np.abs(y_o).max()
    assert np.abs(st_r - st_o).max() <= 2e-5 * np.abs(st_o).max()


def test_argmax_ties_lowest_index():
    r = rng(30)
    V = 5000
    x = r.standard_normal((6, V)).astype(np.float32)
    for i, pos in enumerate([(3, 4000), (4999, 17), (0, 2500), (1234, 1235)]):
        x[i, list(pos)] = 9.0
    x[4, :] = 1.0  # all equal: index 0
    got = ref.argmax(x)
    want = [orc.lib().orc_argmax(np.ascontiguousarray(row).ctypes.data_as(orc.PF), V) for row in x]
    assert list(got) == list(want)
    assert list(got[:5]) == [3, 17, 0, 1234, 0]


def ref_format(NK, NV, kv):
    c = make_config(512, 1024, 4096, 4, 4 * kv, kv, NK, NV, group_size=128, has_bias=False, hadamard=512,
                    has_signs=True, ctx=256)
    c.head_kind = 1
    return c


@pytest.mark.parametrize("NK,NV,kv", [(4, 16, 1), (16, 16, 2)])
def test_model_passes_match_oracle(NK, NV, kv):
    """Whole passes of the reference (model.rs's kernel sequence on its own kernels) against the oracle model:
    a 20-row prefill chunk (qmm), verify passes of 9 (qmvxm), 3 (qmvr) and 1 (qmv4) rows with partial and full
    accepts in between (encode_accept's replay and copy), and a single-token decode step (qmv3 with the a/b rows, the
    in-place conv update). Logits within 1e-4 absolute; argmax equal unless the oracle's top-2 gap is below that."""
    cfg = ref_format(NK, NV, kv)
    ts = synth.model_tensors(cfg, 11 + NK)
    rm = ref.RefModel(cfg, ts)
    om = orc.OracleModel(cfg, ts)

    def check(rl, rp, ol, op, where):
        assert np.abs(rl - ol).max() <= 1e-4, f"{where}: {np.abs(rl - ol).max()}"
        for t in range(len(rp)):
            if rp[t] != op[t]:
                top = np.sort(ol[t])[-2:]
                assert top[1] - top[0] < 1e-4, f"{where} row {t}"

    ids = synth.zipf_tokens(3, 20, cfg.vocab)
    rp, rl = rm.prefill_chunk(ids)
    op, ol = om.forward(ids, logits=True)
    om.accept(20)
    check(rl, rp, ol, op, "prefill 20")
    for T, n in ((9, 4), (3, 3), (9, 9), (1, 1)):
        rows = synth.zipf_tokens(40 + T + n, T, cfg.vocab)
        rp, rl = rm.verify(rows)
        op, ol = om.forward(rows, logits=True)
        check(rl, rp, ol, op, f"verify {T}")
        rm.accept(T, n)
        om.accept(n)
    assert rm.length == om.length == 20 + 4 + 3 + 9 + 1
    rp, rl = rm.prefill_chunk(np.array([7], np.uint32))  # decode step: qmv3 + a/b rows, conv state updated in place
    op, ol = om.forward(np.array([7], np.uint32), logits=True)
    om.accept(1)
    check(rl, rp, ol, op, "step")
