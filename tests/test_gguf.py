"""The GGUF loader (llambda_cuda_gguf_*) on files written by tests/gguf_writer.py:
header, metadata skipping by type, tensor infos, alignment and byte sizes, and
the reference loader's errors (read-gguf-header / -metadata-section /
-tensor-infos, llambda.lisp L2049-2238).  Parsing needs no GPU."""
import numpy as np
import pytest

import llambda_b200 as LB
from llambda_b200 import _native as N
from tests import gguf_writer as W

META = [("general.architecture", W.STR, "qwen3next"),
        ("general.alignment", W.U32, 64),
        ("tokenizer.ggml.tokens", W.ARR, (W.STR, ["a", "bb", "ccc"])),
        ("general.file_type", W.U32, 15),
        ("x.f32", W.F32, 1.5), ("x.u64", W.U64, 7), ("x.bool", W.BOOL, True),
        ("x.arr_i32", W.ARR, (W.I32, [1, -2, 3])), ("x.f64", W.F64, 2.0)]


def _tensors():
    q4 = W.random_bytes(144 * 2 * 3, 1)   # Q4_K, 512 x 3
    q6 = W.random_bytes(210 * 1 * 5, 2)   # Q6_K, 256 x 5
    f32 = np.arange(7, dtype=np.float32).view(np.uint8)
    q8 = W.random_bytes(34 * 2 * 2, 3)    # Q8_0, 64 x 2
    q41 = W.random_bytes(20 * 4, 4)       # type 3 (Q4_1): not sized by the loader
    return [("blk.0.ffn_up_exps.weight", [512, 3], 12, q4),
            ("blk.0.ffn_down_exps.weight", [256, 5], 14, q6),
            ("blk.0.ffn_gate_inp.weight", [7], 0, f32),
            ("blk.0.attn_q.weight", [64, 2], 8, q8),
            ("blk.0.other", [128], 3, q41)]


def test_parses_infos_offsets_and_bytes(tmp_path):
    path = tmp_path / "m.gguf"
    tensors = _tensors()
    W.write(path, META, tensors, alignment=64)
    g = LB.GgufFile(str(path))
    assert len(g) == len(tensors)
    for i, (name, dims, tag, raw) in enumerate(tensors):
        assert g.find(name) == i
        info = g.info(i)
        assert info["name"] == name and info["type"] == tag and info["dims"] == dims
        assert info["ne"][len(dims):] == [1] * (4 - len(dims))
        if tag == 3:
            assert info["byte_size"] == 0
        else:
            assert info["byte_size"] == len(raw)
            assert np.array_equal(g.host_bytes(i), np.asarray(raw, np.uint8))
            assert info["host_ptr"] % 64 == 0  # data start and offsets aligned
    assert g.find("missing") == -1
    g.close()


def test_default_alignment_is_32(tmp_path):
    path = tmp_path / "m.gguf"
    meta = [m for m in META if m[0] != "general.alignment"]
    tensors = _tensors()[:3]
    W.write(path, meta, tensors, alignment=32)
    g = LB.GgufFile(str(path))
    for i, (_, _, _, raw) in enumerate(tensors):
        assert np.array_equal(g.host_bytes(i), np.asarray(raw, np.uint8))
    g.close()


@pytest.mark.parametrize("case,match", [
    ("magic", "Invalid GGUF magic"),
    ("truncated", "past the end of the file"),
    ("alignment", "power of two"),
    ("dims", "dimension count"),
    ("zero_dim", "non-positive"),
    ("blocks", "multiple of block size"),
    ("nested", "Nested GGUF metadata arrays"),
    ("value_type", "Unsupported GGUF metadata value type"),
])
def test_rejects_what_the_reference_rejects(tmp_path, case, match):
    path = tmp_path / "bad.gguf"
    meta, tensors, kw = list(META), _tensors()[:3], {}
    if case == "magic":
        kw["magic"] = b"GGUX"
    elif case == "truncated":
        kw["data_pad"] = 100
    elif case == "alignment":
        meta = [m for m in meta if m[0] != "general.alignment"] + [("general.alignment", W.U32, 48)]
    elif case == "dims":
        tensors[2] = ("t", [1, 1, 1, 1, 7], 0, tensors[2][3])
    elif case == "zero_dim":
        tensors[2] = ("t", [0], 0, b"")
    elif case == "blocks":
        tensors[0] = ("t", [500, 3], 12, tensors[0][3])
    elif case == "nested":
        meta = meta + [("n", W.ARR, (W.ARR, []))]
    if case == "value_type":
        # one metadata key whose value type (13) the format does not define
        import struct
        body = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W._str("k") + struct.pack("<I", 13)
        path.write_bytes(body + b"\0" * 32)
    else:
        W.write(path, meta, tensors, alignment=64 if case != "alignment" else 32, **kw)
    with pytest.raises(LB.LlambdaCudaError, match=match):
        LB.GgufFile(str(path))


def test_missing_file_is_an_error(tmp_path):
    with pytest.raises(LB.LlambdaCudaError, match="Cannot open"):
        LB.GgufFile(str(tmp_path / "none.gguf"))
