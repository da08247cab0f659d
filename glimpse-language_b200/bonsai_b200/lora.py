"""LoRA adapter files (lora.rs:39-174, adapter_id runtime/mod.rs:236-243): the host half of lora::load. Reads a
safetensors adapter (Glimpse-Lab export keys `model.layers.N.<mod>.lora_A` [r, in] / `.lora_B` [out, r], alpha / r
already in B; or PEFT keys `...layers.N.<mod>.lora_A.weight`, alpha / r from the adapter_config.json beside the file)
into the per-linear list that bcu_set_lora takes; the grouping, fp16 rounding and device layout happen in the
library (csrc/lora.cu)."""
import json
import os
import struct

import numpy as np

from . import _lib

FNV = 0xCBF29CE484222325


class LoraError(ValueError):
    pass


def read_safetensors(path):
    """read_safetensors (lora.rs:44-71): name -> float32 array (F32, F16 and BF16 tensors)."""
    b = open(path, "rb").read()
    if len(b) < 8:
        raise LoraError("lora: not a safetensors file")
    n = struct.unpack_from("<Q", b, 0)[0]
    try:
        h = json.loads(b[8:8 + n])
    except ValueError:
        raise LoraError("lora: bad header")
    if not isinstance(h, dict):
        raise LoraError("lora: bad header")
    body = b[8 + n:]
    out = {}
    for k, v in h.items():
        if k == "__metadata__":
            continue
        s, e = v["data_offsets"]
        raw = body[s:e]
        if e > len(body) or s > e:
            raise LoraError(f"lora: {k} out of range")
        dt = v.get("dtype", "")
        if dt == "F32":
            a = np.frombuffer(raw, "<f4").astype(np.float32)
        elif dt == "F16":
            a = np.frombuffer(raw, "<f2").astype(np.float32)
        elif dt == "BF16":
            a = (np.frombuffer(raw, "<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            raise LoraError(f"lora: {k}: unsupported dtype {dt}")
        out[k] = a.reshape([int(x) for x in v["shape"]])
    return out


def write_safetensors(path, tensors, dtype="F32"):
    """A safetensors file of float32 arrays stored as `dtype` (F32, F16 or BF16), for adapters made in tests."""
    header, blobs, off = {}, [], 0
    for k, a in tensors.items():
        a = np.ascontiguousarray(a, np.float32)
        if dtype == "F32":
            raw = a.astype("<f4").tobytes()
        elif dtype == "F16":
            raw = a.astype("<f2").tobytes()
        else:
            raw = (a.view(np.uint32) >> 16).astype("<u2").tobytes()
        header[k] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb + b"".join(blobs))


def peft_scaling(directory):
    """peft_scaling (lora.rs:73-86): alpha / r (alpha / sqrt(r) with use_rslora) from adapter_config.json."""
    p = os.path.join(directory, "adapter_config.json")
    try:
        j = json.loads(open(p, "rb").read())
    except (OSError, ValueError) as e:
        raise LoraError(f"lora: PEFT keys need {p}: {e}")
    for k in ("rank_pattern", "alpha_pattern"):
        if isinstance(j.get(k), dict) and j[k]:
            raise LoraError(f"lora: {k} is not supported")
    r, alpha = j.get("r"), j.get("lora_alpha")
    if not isinstance(r, (int, float)):
        raise LoraError("lora: adapter_config r")
    if not isinstance(alpha, (int, float)):
        raise LoraError("lora: adapter_config lora_alpha")
    return float(np.float32(alpha / np.sqrt(r) if j.get("use_rslora") is True else alpha / r))


def parse(path):
    """The key handling of lora::load (lora.rs:90-106): ([(layer, module, A, B)], fold without the user's scale).
    module is the text after "layers.N." (e.g. "self_attn.q_proj"); which modules exist is checked by the library."""
    tensors = read_safetensors(path)
    peft = any(k.endswith(".weight") for k in tensors)
    fold = peft_scaling(os.path.dirname(os.path.abspath(path))) if peft else 1.0
    ab = {}
    for k, t in tensors.items():
        k2 = k[: -len(".weight")] if k.endswith(".weight") else k
        if k2.endswith(".lora_A"):
            stem, which = k2[: -len(".lora_A")], 0
        elif k2.endswith(".lora_B"):
            stem, which = k2[: -len(".lora_B")], 1
        else:
            raise LoraError(f"lora: unexpected tensor {k}")
        i = stem.find("layers.")
        if i < 0:
            raise LoraError(f"lora: {k} is not a layer linear")
        ab.setdefault(stem[i:], [None, None])[which] = t
    out = []
    for key in sorted(ab):
        a, b = ab[key]
        if a is None or b is None:
            raise LoraError(f"lora: {key} needs lora_A and lora_B")
        rest = key[len("layers."):]
        dot = rest.find(".")
        if dot < 0 or not rest[:dot].isdigit():
            raise LoraError(f"lora: tensors for unsupported modules, e.g. {key}")
        out.append((int(rest[:dot]), rest[dot + 1:], a, b))
    if not out:
        raise LoraError("lora: no adapted linears")
    return out, fold


def hash_bytes(h, b):
    """hash_bytes (runtime/mod.rs:225-235), computed by the library."""
    b = bytes(b)
    return _lib.lib().bcu_hash_bytes(h, b, len(b))


def adapter_id(path, scale):
    """adapter_id (runtime/mod.rs:236-243): the file, the PEFT config beside it and the scale; never 0."""
    h = hash_bytes(FNV, open(path, "rb").read())
    cfg = os.path.join(os.path.dirname(os.path.abspath(path)), "adapter_config.json")
    if os.path.exists(cfg):
        h = hash_bytes(h, open(cfg, "rb").read())
    return hash_bytes(h, struct.pack("<f", scale)) | 1
