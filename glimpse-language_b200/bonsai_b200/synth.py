"""Seeded random-init weights of a config, under the reference's tensor names (Text::new, runtime/model.rs:272-313).

Distributions follow the graded configs: ternary codes uniform in {0,1,2}, fp16 scales U(0.01, 0.05) with bias -s
(or the implicit -s of the reference pack), bf16 embedding / lm_head N(0, 0.02). The rest (not specified by the
configs) keeps activations O(1): norm weights U(0.8, 1.2), GDN a/b rows N(0, 1/sqrt(hidden)) so the gate logits are
~N(0, 1), A_log = dt_bias = 0 (decay exp(-softplus(a)) as config 2 states), conv taps N(0, 0.5).
All values come from bcu_synth_fill (libbonsai_synth.so, include/bonsai_synth.h: a host-only library apart from the
CUDA backend), so the same seed gives the same bytes on every host.
"""
import ctypes
import os

import numpy as np

from . import _lib
from .config import dims

SYNTH_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbonsai_synth.so")
SIGNATURES = {
    "bcu_synth_fill": (_lib.I32, [_lib.I32, _lib.U64, _lib.U64, ctypes.c_double, ctypes.c_double, _lib.P, _lib.U64]),
    "bcu_synth_zipf": (_lib.I32, [_lib.U64, ctypes.c_double, _lib.I32, _lib.PU32, _lib.I32]),
}
_S = None


def lib():
    """The generator library (built in-tree with the backend by `make -C glimpse-language_b200`)."""
    global _S
    if _S is None:
        if not os.path.exists(SYNTH_PATH):
            raise RuntimeError(f"{SYNTH_PATH} is missing: make -C glimpse-language_b200")
        L = ctypes.CDLL(SYNTH_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _S = L
    return _S

PFX = "language_model.model."


def fill(kind, seed, stream, a, b, shape, dtype):
    arr = np.empty(shape, dtype=dtype)
    n = arr.size // 16 if kind == 3 else arr.size
    if kind == 3:
        n = arr.size
    s = lib().bcu_synth_fill(kind, seed, stream, a, b, arr.ctypes.data_as(ctypes.c_void_p), n)
    if s != _lib.OK:
        raise RuntimeError("bcu_synth_fill failed")
    return arr


class TensorSet:
    """Ordered (name, dtype code, array) triples; arrays are C-contiguous numpy views of the tensor bytes."""

    def __init__(self):
        self.items = []

    def add(self, name, code, arr):
        self.items.append((name, code, np.ascontiguousarray(arr)))

    def __iter__(self):
        return iter(self.items)

    def get(self, name):
        for n, c, a in self.items:
            if n == name:
                return a
        raise KeyError(name)

    def nbytes(self):
        return sum(a.nbytes for _, _, a in self.items)


def model_tensors(cfg, seed=1234):
    d, ff = cfg.hidden, cfg.intermediate
    dm = dims(cfg)
    C, gw, aw, kvw = dm["C"], dm["gw"], dm["aw"], dm["kvw"]
    g = cfg.group_size
    ts = TensorSet()
    stream = [0]

    def nxt():
        stream[0] += 1
        return stream[0]

    def packed(name, O, K):
        ts.add(name + ".weight", _lib.U32, fill(3, seed, nxt(), 0, 0, (O, K // 16), np.uint32))
        st = nxt()
        ts.add(name + ".scales", _lib.F16, fill(4, seed, st, 0.01, 0.05, (O, K // g), np.uint16))
        if cfg.has_bias:
            ts.add(name + ".biases", _lib.F16, fill(6, seed, st, 0.01, 0.05, (O, K // g), np.uint16))
        if cfg.has_signs:
            ts.add(name + ".signs", _lib.F32, fill(5, seed, nxt(), 0, 0, (K,), np.float32))

    def norm(name, n):
        ts.add(name, _lib.F32, fill(0, seed, nxt(), 0.8, 1.2, (n,), np.float32))

    for i in range(cfg.n_layers):
        l = f"{PFX}layers.{i}."
        norm(l + "input_layernorm.weight", d)
        norm(l + "post_attention_layernorm.weight", d)
        if cfg.layer_is_attn[i]:
            a = l + "self_attn."
            packed(a + "q_proj", 2 * aw, d)
            packed(a + "k_proj", kvw, d)
            packed(a + "v_proj", kvw, d)
            packed(a + "o_proj", d, aw)
            norm(a + "q_norm.weight", 256)
            norm(a + "k_norm.weight", 256)
        else:
            a = l + "linear_attn."
            packed(a + "in_proj_qkv", C, d)
            packed(a + "in_proj_z", gw, d)
            packed(a + "out_proj", d, gw)
            nv = cfg.lin_v_heads
            ts.add(a + "in_proj_a.weight", _lib.F32, fill(1, seed, nxt(), 0.0, d ** -0.5, (nv, d), np.float32))
            ts.add(a + "in_proj_b.weight", _lib.F32, fill(1, seed, nxt(), 0.0, d ** -0.5, (nv, d), np.float32))
            ts.add(a + "A_log", _lib.F32, np.zeros(nv, np.float32))
            ts.add(a + "dt_bias", _lib.F32, np.zeros(nv, np.float32))
            ts.add(a + "conv1d.weight", _lib.F32, fill(1, seed, nxt(), 0.0, 0.5, (C, 4), np.float32))
            norm(a + "norm.weight", 128)
        m = l + "mlp."
        packed(m + "gate_proj", ff, d)
        packed(m + "up_proj", ff, d)
        packed(m + "down_proj", d, ff)
    norm(PFX + "norm.weight", d)
    if cfg.head_kind == 1:  # the reference's tied table: ternary-packed like the linears (model.rs:356, 962)
        packed(PFX + "embed_tokens", cfg.vocab, d)
    else:
        ts.add(PFX + "embed_tokens.weight", _lib.BF16, fill(2, seed, nxt(), 0.0, 0.02, (cfg.vocab, d), np.uint16))
    return ts


def random_state(cfg, length, seed):
    """A seeded committed state after `length` tokens, in the four state parts' layout (bcu_state_read): GDN
    [gdn layer][NV][128][128] ~N(0, 0.02) (config 2's starting state), conv [gdn layer][3][C] ~N(0, 1), K and V
    [attn layer][length][KV * 256] ~N(0, 1) (cached keys are RMS-normalised, so unit scale is their natural size).
    Starts a pass at a long context without prefilling it (numpy's generator: same bytes on every host)."""
    rng = np.random.default_rng(seed)
    n_attn = sum(cfg.layer_is_attn[i] for i in range(cfg.n_layers))
    n_gdn = cfg.n_layers - n_attn
    d = dims(cfg)
    gdn = rng.normal(0, 0.02, (n_gdn, cfg.lin_v_heads, 128, 128)).astype(np.float32)
    conv = rng.normal(0, 1, (n_gdn, 3, d["C"])).astype(np.float32)
    kc = rng.normal(0, 1, (n_attn, length, d["kvw"])).astype(np.float32)
    vc = rng.normal(0, 1, (n_attn, length, d["kvw"])).astype(np.float32)
    return gdn, conv, kc, vc


def zipf_tokens(seed, n, vocab, s=1.1):
    out = np.empty(n, np.uint32)
    lib().bcu_synth_zipf(seed, s, vocab, out.ctypes.data_as(_lib.PU32), n)
    return out


def lora_modules(cfg, layer):
    """Text::linears (model.rs:372-385) of one layer: [(module, out, in)]."""
    d, ff = cfg.hidden, cfg.intermediate
    dm = dims(cfg)
    if cfg.layer_is_attn[layer]:
        mods = [("self_attn.q_proj", 2 * dm["aw"], d), ("self_attn.k_proj", dm["kvw"], d),
                ("self_attn.v_proj", dm["kvw"], d), ("self_attn.o_proj", d, dm["aw"])]
    else:
        mods = [("linear_attn.in_proj_qkv", dm["C"], d), ("linear_attn.in_proj_z", dm["gw"], d),
                ("linear_attn.out_proj", d, dm["gw"])]
    return mods + [("mlp.gate_proj", ff, d), ("mlp.up_proj", ff, d), ("mlp.down_proj", d, ff)]


def lora_linears(cfg, rank, seed=77, std_a=0.02, std_b=0.01, modules=None):
    """A seeded adapter on every linear of every layer (or those whose module name is in `modules`): A ~ N(0, std_a)
    [rank, in], B ~ N(0, std_b) [out, rank] (the graded 4B adapter: rank 16, A 0.02, B 0.01, alpha 32)."""
    out, stream = [], 0
    for layer in range(cfg.n_layers):
        for mod, o, k in lora_modules(cfg, layer):
            if modules is not None and mod not in modules:
                continue
            a = fill(1, seed, stream, 0.0, std_a, (rank, k), np.float32)
            b = fill(1, seed, stream + 1, 0.0, std_b, (o, rank), np.float32)
            stream += 2
            out.append((layer, mod, a, b))
    return out
