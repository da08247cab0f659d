"""Draft source and draft normalisation of prompt-lookup drafting (runtime/mod.rs:699-768), host logic of the C-ABI
library against the oracle's restatement and against hand-worked answers, on a toy vocabulary with a greedy
longest-match tokenizer standing in for the caller's (the backend never tokenizes: it gets token bytes, filler ids
and an encoder callback). No device calls."""
import ctypes

import numpy as np
import pytest

from bonsai_b200 import _lib
from oracle import oracle as orc

WORDS = ["<", "transcript", ">\n", "\n</", ">", " hello", " world", " um", "Um", " i", " dont", " don", "'t", " know",
         ".", " monday", " Monday", " I", " ok", "\n", " Clean", " this", ":", " thanks", " it", "s", " the", "text",
         " uh", " im", " I'm", " H", "ello", "?", " yes", " Hello", " cant", " can", " friday", " Friday", "!"]
VOCAB = WORDS + [chr(c) for c in range(32, 127) if chr(c) not in WORDS]
TB = [w.encode() for w in VOCAB]
ID = {b: i for i, b in enumerate(TB)}


def encode(text):
    b, out = text.encode() if isinstance(text, str) else text, []
    while b:
        best = max((t for t in TB if b.startswith(t)), key=len)
        out.append(ID[best])
        b = b[len(best):]
    return out


def vocab_arrays():
    data = b"".join(TB)
    offs = np.zeros(len(TB) + 1, np.uint64)
    offs[1:] = np.cumsum([len(t) for t in TB])
    return np.frombuffer(data, np.uint8).copy(), offs


BYTES, OFFS = vocab_arrays()
OFFP = OFFS.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))


@_lib.ENCODE_FN
def _encode_cb(user, text, n, out, cap):
    ids = encode(bytes(text[:n]))
    if len(ids) > cap:
        return -1
    for i, v in enumerate(ids):
        out[i] = v
    return len(ids)


def product_source(user, fillers=None):
    u = np.ascontiguousarray(user, np.uint32)
    out = np.zeros(max(len(u), 1), np.uint32)
    f = np.ascontiguousarray(fillers if fillers is not None else [0], np.uint32)
    n = _lib.lib().bcu_draft_source_host(u.ctypes.data_as(_lib.PU32), len(u), BYTES.ctypes.data_as(ctypes.c_void_p),
                                         OFFP, len(TB), f.ctypes.data_as(_lib.PU32),
                                         len(fillers) if fillers is not None else -1, out.ctypes.data_as(_lib.PU32))
    return list(out[:n])


def default_filler_ids():
    return [ID[w.encode()] for w in (" um", " uh", "Um") if w.encode() in ID]


def oracle_source(user, fillers):
    u = np.ascontiguousarray(user, np.uint32)
    out = np.zeros(max(len(u), 1), np.uint32)
    f = np.ascontiguousarray(fillers if fillers else [0], np.uint32)
    n = orc.lib().orc_draft_source(u.ctypes.data_as(orc.PU32), len(u), BYTES.ctypes.data_as(ctypes.c_void_p), OFFP,
                                   len(TB), f.ctypes.data_as(orc.PU32), len(fillers), out.ctypes.data_as(orc.PU32))
    return list(out[:n])


def product_normalize(draft, last):
    d = np.ascontiguousarray(draft, np.uint32).copy()
    n = _lib.lib().bcu_normalize_draft_host(d.ctypes.data_as(_lib.PU32), len(d), last,
                                            BYTES.ctypes.data_as(ctypes.c_void_p), OFFP, len(TB),
                                            ctypes.cast(_encode_cb, ctypes.c_void_p), None)
    return list(d[:n])


def oracle_normalize(draft, last):
    d = np.ascontiguousarray(draft, np.uint32).copy()
    n = orc.lib().orc_normalize_draft(d.ctypes.data_as(orc.PU32), len(d), last, BYTES.ctypes.data_as(ctypes.c_void_p),
                                      OFFP, len(TB), ctypes.cast(_encode_cb, ctypes.c_void_p), None)
    return list(d[:n])


def ids(*words):
    return [ID[w.encode()] for w in words]


def test_draft_source_takes_the_transcript_block_without_fillers():
    user = encode(" Clean this:<transcript>\n hello um world\n</transcript> thanks")
    assert ids("<", "transcript", ">\n") == user[3:6]
    want = ids(" hello", " world")
    assert product_source(user) == want
    assert oracle_source(user, default_filler_ids()) == want


def test_draft_source_other_tag_whole_turn_and_unclosed_block():
    user = encode(" ok<text>\n yes um i\n</text>!")
    assert product_source(user) == ids(" yes", " i")
    # no block: the whole turn, fillers dropped
    user = encode(" hello um world uh.")
    assert product_source(user) == ids(" hello", " world", ".")
    # an opening tag without its closing tag does not count
    user = encode("<transcript>\n hello world")
    assert product_source(user) == user
    # explicit filler ids replace the default set
    user = encode(" hello um world")
    assert product_source(user, fillers=ids(" hello")) == ids(" um", " world")


def test_draft_source_matches_oracle_on_random_turns():
    rng = np.random.default_rng(5)
    pieces = [" hello", " world", " um", "Um", " ok", "<transcript>\n", "\n</transcript>", "<text>\n", "\n</text>",
              " i", ".", "\n", " uh"]
    for _ in range(300):
        text = "".join(rng.choice(pieces, rng.integers(0, 14)))
        user = encode(text)
        assert product_source(user) == oracle_source(user, default_filler_ids()), text


def test_normalize_draft_known_answers():
    last = ID[b"."]
    draft = ids(" hello", " i", " dont", " know", " monday", " ok")
    # " Hello" (after a sentence end), " I", " don't" re-encoded as " don" + "'t", " Monday" (a day): truncated to 6
    want = ids(" Hello", " I", " don", "'t", " know", " Monday")
    assert product_normalize(draft, last) == want
    assert oracle_normalize(draft, last) == want
    # mid-sentence: no capital except " i" and the days; a word of two tokens stays as it is
    draft = ids(" yes", " H", "ello", " i", " cant", " friday")
    want = ids(" yes", " H", "ello", " I", " can", "'t")
    assert product_normalize(draft, ID[b" ok"]) == want
    assert oracle_normalize(draft, ID[b" ok"]) == want


def test_normalize_draft_matches_oracle_on_random_drafts():
    rng = np.random.default_rng(9)
    for _ in range(500):
        draft = list(rng.integers(0, len(TB), rng.integers(1, 16)).astype(np.uint32))
        last = int(rng.integers(0, len(TB)))
        assert product_normalize(draft, last) == oracle_normalize(draft, last), (draft, last)


def test_normalize_draft_without_encoder_is_identity():
    d = np.array(ids(" hello", " i"), np.uint32)
    n = _lib.lib().bcu_normalize_draft_host(d.ctypes.data_as(_lib.PU32), 2, ID[b"."],
                                            BYTES.ctypes.data_as(ctypes.c_void_p), OFFP, len(TB), None, None)
    assert n == 2 and list(d) == ids(" hello", " i")
