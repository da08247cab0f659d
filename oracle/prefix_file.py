"""Byte-level restatement of the saved prefix-cache file (BNSPFX01). TEST INFRASTRUCTURE ONLY: the tests compare the
library's writer, reader and file names with these bytes; nothing in the product imports it.

Follows runtime/mod.rs of the reference: hash_bytes :225-235, prefix_identity :494-510, prefix_path :512-515,
load_prefix :517-546, save_prefix :549-578; the parts are Text::state_parts (model.rs:1090-1099). Parity unpinned:
the reference (Rust) cannot run here and its tests hold no prefix-file fixture, so these functions restate the
published layout and the tests check the library against them.
"""
import os
import struct

MAGIC = b"BNSPFX01"  # runtime/mod.rs:215
FNV = 0xCBF29CE484222325  # runtime/mod.rs:216
PRIME = 0x100000001B3
MASK = (1 << 64) - 1
SLOTS = 3  # PREFIX_SLOTS, runtime/mod.rs:213


def hash_bytes(h, b):
    """runtime/mod.rs:225-235: 8-byte little-endian words, then the tail bytes, then ^ len."""
    b = bytes(b)
    n8 = len(b) // 8 * 8
    for i in range(0, n8, 8):
        h = ((h ^ int.from_bytes(b[i:i + 8], "little")) * PRIME) & MASK
    for c in b[n8:]:
        h = ((h ^ c) * PRIME) & MASK
    return h ^ len(b)


def stamp(path):
    """(len, mtime in ns) of a file, runtime/mod.rs:495-499."""
    st = os.stat(path)
    return [st.st_size, st.st_mtime_ns]


def identity(kernel_hash, adapter, exe, weights, config, shape_words, device_name):
    """runtime/mod.rs:500-509: magic, the u64 words, the device name."""
    words = [kernel_hash, adapter, *stamp(exe), *stamp(weights), hash_bytes(FNV, open(config, "rb").read()),
             *shape_words]
    return MAGIC + b"".join(struct.pack("<Q", w & MASK) for w in words) + device_name.encode()


def ids_bytes(ids):
    return b"".join(struct.pack("<I", int(t)) for t in ids)


def file_name(identity_b, ids):
    """runtime/mod.rs:512-515: "{h:016x}.prefix"."""
    return f"{hash_bytes(hash_bytes(FNV, identity_b), ids_bytes(ids)):016x}.prefix"


def file_bytes(identity_b, ids, pos, parts):
    """runtime/mod.rs:552-560: identity, ids, len u64, pos i64, the parts in order."""
    return identity_b + ids_bytes(ids) + struct.pack("<Qq", len(ids), pos) + b"".join(bytes(p) for p in parts)


def read_file(path, identity_b, ids, sizes):
    """runtime/mod.rs:517-546: the parts when the header matches exactly, len == len(ids) and the file holds exactly
    the parts' bytes after it; None otherwise. (Also returns pos.)"""
    try:
        data = open(path, "rb").read()
    except OSError:
        return None
    want = identity_b + ids_bytes(ids)
    if len(data) < len(want) + 16 or data[:len(want)] != want:
        return None
    n, pos = struct.unpack_from("<Qq", data, len(want))
    if n != len(ids):
        return None
    at = len(want) + 16
    if len(data) != at + sum(sizes):
        return None
    parts = []
    for s in sizes:
        parts.append(data[at:at + s])
        at += s
    return parts, pos


def kept_after_save(mtimes):
    """runtime/mod.rs:566-577: names of the newest SLOTS files given {name: mtime_ns}."""
    return set(sorted(mtimes, key=lambda k: -mtimes[k])[:SLOTS])
