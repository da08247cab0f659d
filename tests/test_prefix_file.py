"""The saved prefix-cache file (BNSPFX01) on the host: the library's hash, file names, writer and reader against the
byte-level restatement in oracle/prefix_file.py (runtime/mod.rs:213-235, 494-578). No GPU: these entry points touch
no device. Bit-exact: every byte of every file."""
import os
import struct

import numpy as np
import pytest

from bonsai_b200 import _lib
from bonsai_b200 import runtime as rt
from oracle import prefix_file as pf

IDENT = pf.MAGIC + bytes(range(96)) + b"NVIDIA B200"


def parts_for(seed, sizes=(48, 24, 40, 40)):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, n, dtype=np.uint8).tobytes() for n in sizes]


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 15, 16, 17, 63, 1000])
def test_hash_bytes_matches_restatement(n):
    b = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    for h in (pf.FNV, 0, 0xFFFFFFFFFFFFFFFF, 12345):
        assert rt.hash_bytes(h, b) == pf.hash_bytes(h, b)


def test_hash_bytes_known_answers():
    # empty input: the seed ^ 0; one byte: one FNV-1a step then ^ 1; one word: the word as a little-endian u64
    assert rt.hash_bytes(pf.FNV, b"") == pf.FNV
    assert rt.hash_bytes(pf.FNV, b"a") == (((pf.FNV ^ 0x61) * pf.PRIME) & pf.MASK) ^ 1
    w = b"BNSPFX01"
    assert rt.hash_bytes(pf.FNV, w) == (((pf.FNV ^ int.from_bytes(w, "little")) * pf.PRIME) & pf.MASK) ^ 8


def test_kernel_hash_is_stable():
    assert rt.kernel_hash() == rt.kernel_hash() != 0


@pytest.mark.parametrize("ids", [[], [0], [1, 2, 3], list(range(574))])
def test_file_name(tmp_path, ids):
    p = rt.prefix_path(str(tmp_path), IDENT, ids)
    assert p == os.path.join(str(tmp_path), pf.file_name(IDENT, ids))
    # a trailing slash on the directory names the same file
    assert rt.prefix_path(str(tmp_path) + "/", IDENT, ids) == p


def test_writer_bytes(tmp_path):
    ids = [5, 70000, 2**32 - 1, 0, 9]
    parts = parts_for(1)
    assert rt.file_write(str(tmp_path), IDENT, ids, parts) == _lib.OK
    path = rt.prefix_path(str(tmp_path), IDENT, ids)
    assert open(path, "rb").read() == pf.file_bytes(IDENT, ids, len(ids), parts)
    assert sorted(os.listdir(tmp_path)) == [os.path.basename(path)]  # no temporary file left


def test_writer_creates_directories(tmp_path):
    d = os.path.join(str(tmp_path), "a", "b", "prefix-cache")
    assert rt.file_write(d, IDENT, [1, 2], parts_for(2)) == _lib.OK
    assert os.path.exists(rt.prefix_path(d, IDENT, [1, 2]))


def test_writer_reports_unwritable_directory(tmp_path):
    blocker = os.path.join(str(tmp_path), "file")
    open(blocker, "wb").write(b"x")
    assert rt.file_write(os.path.join(blocker, "sub"), IDENT, [1], parts_for(3)) == _lib.ERR_IO


def test_reader_round_trip(tmp_path):
    ids = list(range(40, 73))
    parts = parts_for(4)
    rt.file_write(str(tmp_path), IDENT, ids, parts)
    got = rt.file_read(str(tmp_path), IDENT, ids, [len(p) for p in parts])
    assert got == parts
    ref = pf.read_file(rt.prefix_path(str(tmp_path), IDENT, ids), IDENT, ids, [len(p) for p in parts])
    assert ref == (parts, len(ids))


def test_reader_rejects(tmp_path):
    d = str(tmp_path)
    ids = [3, 1, 4, 1, 5]
    parts = parts_for(5)
    sizes = [len(p) for p in parts]
    rt.file_write(d, IDENT, ids, parts)
    path = rt.prefix_path(d, IDENT, ids)
    good = open(path, "rb").read()
    assert rt.file_read(d, IDENT, ids, sizes) == parts
    # no file for other ids or another identity
    assert rt.file_read(d, IDENT, ids[:-1], sizes) is None
    assert rt.file_read(d, IDENT[:-1] + b"X", ids, sizes) is None
    # other part sizes (another model shape or prefix length): size mismatch
    assert rt.file_read(d, IDENT, ids, [sizes[0] + 4] + sizes[1:]) is None
    cases = {
        "truncated": good[:-1],
        "trailing byte": good + b"\0",
        "header only": good[: len(IDENT) + 4 * len(ids) + 16],
        "short header": good[: len(IDENT) + 3],
        "identity byte": good[:20] + bytes([good[20] ^ 1]) + good[21:],
        "ids byte": good[: len(IDENT)] + bytes([good[len(IDENT)] ^ 1]) + good[len(IDENT) + 1:],
        "len field": good[: len(IDENT) + 20] + struct.pack("<Q", len(ids) + 1) + good[len(IDENT) + 28:],
        "empty": b"",
    }
    for what, data in cases.items():
        open(path, "wb").write(data)
        assert rt.file_read(d, IDENT, ids, sizes) is None, what
        assert pf.read_file(path, IDENT, ids, sizes) is None, what
    # a mrope position other than len (an image in the prefix) cannot be held by a text-only runtime: no hit here,
    # where the reference would load it
    at = len(IDENT) + 4 * len(ids) + 8
    open(path, "wb").write(good[:at] + struct.pack("<q", len(ids) + 3) + good[at + 8:])
    assert rt.file_read(d, IDENT, ids, sizes) is None
    assert pf.read_file(path, IDENT, ids, sizes)[1] == len(ids) + 3
    open(path, "wb").write(good)
    assert rt.file_read(d, IDENT, ids, sizes) == parts


def test_writer_keeps_newest_slots(tmp_path):
    d = str(tmp_path)
    names = {}
    for k in range(5):
        ids = [k, k + 1]
        rt.file_write(d, IDENT, ids, parts_for(10 + k))
        p = rt.prefix_path(d, IDENT, ids)
        names[k] = os.path.basename(p)
        if k < 4:  # explicit, distinct ages: file k is k seconds newer than file 0
            os.utime(p, ns=(1_000_000_000_000 + k * 10**9, 1_000_000_000_000 + k * 10**9))
    # writing file 4 pruned to the newest three: 4 (just written), 3, 2
    left = set(f for f in os.listdir(d) if f.endswith(".prefix"))
    assert left == {names[4], names[3], names[2]}
    mt = {names[k]: 1_000_000_000_000 + k * 10**9 for k in range(4)}
    mt[names[4]] = os.stat(os.path.join(d, names[4])).st_mtime_ns
    assert left == pf.kept_after_save(mt)
    # files that are not .prefix are never touched
    open(os.path.join(d, "notes.txt"), "w").write("x")
    rt.file_write(d, IDENT, [99], parts_for(20))
    assert "notes.txt" in os.listdir(d)
    assert len([f for f in os.listdir(d) if f.endswith(".prefix")]) == pf.SLOTS
