"""A minimal GGUF v3 writer for test fixtures (the format gguf.c:306-411
reads): header, metadata key/value pairs, tensor infos, aligned data.

Used by the tests to build model files whose tensors are known bytes."""
from __future__ import annotations

import struct

import numpy as np

# metadata value types (gguf.h)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q", I64: "<q",
        F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vt: int, v) -> bytes:
    if vt == STR:
        return _str(v)
    if vt == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[vt], v)


def write_gguf(path: str, tensors: list, kv: list | None = None, alignment: int | None = None, version: int = 3):
    """tensors: [(name, ggml_type, dims (innermost first), bytes)];
    kv: [(key, value_type, value)] (arrays as (ARR, (elem_type, [items])))."""
    kv = list(kv or [])
    if alignment is not None:
        kv.append(("general.alignment", U32, alignment))
    al = alignment or 32
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(kv))
    meta = b"".join(_str(k) + struct.pack("<I", vt) + _value(vt, v) for k, vt, v in kv)
    tensors = [(n, t, d, data if isinstance(data, (bytes, bytearray)) else np.ascontiguousarray(data).tobytes())
               for n, t, d, data in tensors]
    infos, offs, off = [], [], 0
    for name, t, dims, data in tensors:
        offs.append(off)
        infos.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                     struct.pack("<IQ", t, off))
        off += (len(data) + al - 1) // al * al
    body = head + meta + b"".join(infos)
    pad = (-len(body)) % al
    with open(path, "wb") as f:
        f.write(body + b"\0" * pad)
        for (_, _, _, data), o in zip(tensors, offs):
            f.write(data + b"\0" * ((len(data) + al - 1) // al * al - len(data)))
    return len(body) + pad


def sid(layer: int, kind: int, e: int) -> int:
    return (layer << 32) | (kind << 24) | e


def write_synthetic_model(orc, path: str, n_layers: int, H: int, I: int, E: int, seed: int, shared=True, norm=True):
    """A GGUF model file holding exactly the seeded weights the synthetic
    expert stack generates (bread_stack_create with the same seed), named as
    the reference's loader expects (loader.c:162-164, :555-569,
    one_layer.cu:964-974)."""
    nb_g, nb_d = I * H // 256, H * I // 256
    ts = []
    for l in range(n_layers):
        for kind, nm, qt, nb, dims in ((0, "ffn_gate_exps", 12, nb_g, [H, I, E]), (1, "ffn_up_exps", 12, nb_g, [H, I, E]),
                                       (2, "ffn_down_exps", 14, nb_d, [I, H, E])):
            data = b"".join(orc.synth_blocks(nb, qt, seed, sid(l, kind, e)).tobytes() for e in range(E))
            ts.append((f"blk.{l}.{nm}.weight", qt, dims, data))
        if shared:
            ts.append((f"blk.{l}.ffn_gate_shexp.weight", 12, [H, I], orc.synth_blocks(nb_g, 12, seed, sid(l, 3, 0))))
            ts.append((f"blk.{l}.ffn_up_shexp.weight", 12, [H, I], orc.synth_blocks(nb_g, 12, seed, sid(l, 4, 0))))
            ts.append((f"blk.{l}.ffn_down_shexp.weight", 14, [I, H], orc.synth_blocks(nb_d, 14, seed, sid(l, 5, 0))))
            ts.append((f"blk.{l}.ffn_gate_inp_shexp.weight", 1, [H], orc.synth_normal(H, 0.02, seed, sid(l, 7, 0),
                                                                                      half=True)))
        ts.append((f"blk.{l}.ffn_gate_inp.weight", 0, [H, E], orc.synth_normal(E * H, 0.02, seed, sid(l, 6, 0))))
        if norm:
            w = orc.synth_normal(H, 0.1, seed, sid(l, 8, 0)) + np.float32(1.0)
            ts.append((f"blk.{l}.post_attention_norm.weight", 0, [H], w.astype(np.float32)))
    kv = [("general.architecture", STR, "test-moe"), (f"test-moe.block_count", U32, n_layers),
          ("test-moe.expert_used_count", U32, 8), ("tokenizer.ggml.tokens", ARR, (STR, ["a", "bb", "ccc"]))]
    return write_gguf(path, ts, kv)
