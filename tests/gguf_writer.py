"""A GGUF v3 writer for the loader tests (test infrastructure): header, typed
metadata, tensor infos, then each tensor's bytes at an aligned offset."""
import struct

import numpy as np

# metadata value types (read-gguf-value, llambda.lisp L1984-2047)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
        U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, i) for i in items)
    return struct.pack(_FMT[t], v)


def write(path, metadata, tensors, alignment=32, version=3, magic=b"GGUF", data_pad=0):
    """metadata: [(key, type, value)]; tensors: [(name, dims, type_tag, raw bytes)].
    Tensor data starts at the aligned end of the infos; each tensor's offset is
    aligned too.  Returns {name: offset from the data start}."""
    head = magic + struct.pack("<IQQ", version, len(tensors), len(metadata))
    kv = b"".join(_str(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in metadata)
    infos, offsets, off = b"", {}, 0
    for name, dims, tag, raw in tensors:
        offsets[name] = off
        infos += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", tag, off)
        off += (len(raw) + alignment - 1) // alignment * alignment
    body = head + kv + infos
    start = (len(body) + alignment - 1) // alignment * alignment
    data = bytearray()
    for name, dims, tag, raw in tensors:
        data += bytes(raw)
        data += b"\0" * ((-len(data)) % alignment)
    with open(path, "wb") as f:
        f.write(body + b"\0" * (start - len(body)) + bytes(data[: len(data) - data_pad]))
    return offsets


def random_bytes(n: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)
