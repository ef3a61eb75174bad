"""The safetensors container reader of libemx (host only, no GPU).

The reference reads checkpoints with the `safetensors` crate
(crates/serve/src/loader/weights.rs:43-60).  The Python `safetensors` package
wraps that crate, so it is the oracle here: files it writes must index the
same (names, dtypes, shapes, bytes), files `emx.write_safetensors` writes must
deserialize in it, and malformed containers must be rejected by both.
"""
import json
import struct

import numpy as np
import pytest

import emx

st = pytest.importorskip("safetensors")


def _crate_tensors(path):
    return {name: (v["dtype"], tuple(v["shape"]), bytes(v["data"])) for name, v in st.deserialize(open(path, "rb").read())}


def _emx_tensors(path):
    raw = open(path, "rb").read()
    return {t["name"]: (t["dtype"], t["shape"], raw[t["offset"]:t["offset"] + t["bytes"]])
            for t in emx.safetensors_index(path)}


def test_files_written_by_the_crate_index_the_same(tmp_path):
    rng = np.random.default_rng(7)
    tensors = {
        "model.layers.0.self_attn.q_proj.weight": {"dtype": "uint32", "shape": [64, 8],
                                                     "data": rng.integers(0, 2**32, (64, 8), dtype=np.uint32).tobytes()},
        "model.layers.0.self_attn.q_proj.scales": {"dtype": "bfloat16", "shape": [64, 1],
                                                     "data": rng.integers(0, 2**16, (64, 1), dtype=np.uint16).tobytes()},
        "model.norm.weight": {"dtype": "bfloat16", "shape": [64], "data": rng.integers(0, 2**16, 64, dtype=np.uint16).tobytes()},
        "scalar": {"dtype": "float32", "shape": [], "data": np.float32(1.5).tobytes()},
        "empty": {"dtype": "int32", "shape": [0, 3], "data": b""},
        "flags": {"dtype": "bool", "shape": [3], "data": b"\x01\x00\x01"},
    }
    p = str(tmp_path / "crate.safetensors")
    st.serialize_file(tensors, p, metadata={"format": "mlx"})
    assert _emx_tensors(p) == _crate_tensors(p)


def test_files_written_here_deserialize_in_the_crate(tmp_path):
    rng = np.random.default_rng(8)
    p = str(tmp_path / "emx.safetensors")
    w = rng.integers(0, 2**32, (32, 4), dtype=np.uint32)
    s = rng.integers(0, 2**16, (32, 2), dtype=np.uint16)
    emx.write_safetensors(p, {"a.weight": w, "a.scales": s, "x": ("F32", np.arange(5, dtype=np.float32))},
                          {"format": "mlx"})
    got = _crate_tensors(p)
    assert got["a.weight"] == ("U32", (32, 4), w.tobytes())
    assert got["a.scales"] == ("BF16", (32, 2), s.tobytes())
    assert got["x"][0] == "F32"
    assert _emx_tensors(p) == got


def _container(header, data=b"", hlen=None):
    h = header if isinstance(header, bytes) else json.dumps(header).encode()
    return struct.pack("<Q", len(h) if hlen is None else hlen) + h + data


MALFORMED = {
    "shorter than the length word": b"\x01\x02\x03",
    "header length past the file": _container({}, hlen=1 << 20),
    "header not JSON": _container(b"{not json"),
    "header not an object": _container([1, 2]),
    "size differs from shape": _container({"a": {"dtype": "U32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8),
    "unknown dtype": _container({"a": {"dtype": "Q7", "shape": [2], "data_offsets": [0, 2]}}, b"\0" * 2),
    "gap between tensors": _container({"a": {"dtype": "U8", "shape": [2], "data_offsets": [0, 2]},
                                       "b": {"dtype": "U8", "shape": [2], "data_offsets": [3, 5]}}, b"\0" * 5),
    "overlapping tensors": _container({"a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]},
                                       "b": {"dtype": "U8", "shape": [2], "data_offsets": [2, 4]}}, b"\0" * 4),
    "data past the file": _container({"a": {"dtype": "U8", "shape": [8], "data_offsets": [0, 8]}}, b"\0" * 4),
    "bytes after the last tensor": _container({"a": {"dtype": "U8", "shape": [2], "data_offsets": [0, 2]}}, b"\0" * 6),
    "negative dimension": _container({"a": {"dtype": "U8", "shape": [-2], "data_offsets": [0, 0]}}),
    "offsets reversed": _container({"a": {"dtype": "U8", "shape": [0], "data_offsets": [2, 0]}}, b"\0" * 2),
    "missing data_offsets": _container({"a": {"dtype": "U8", "shape": [2]}}, b"\0" * 2),
}


@pytest.mark.parametrize("case", sorted(MALFORMED))
def test_malformed_containers_are_rejected_like_the_crate(tmp_path, case):
    blob = MALFORMED[case]
    with pytest.raises(Exception):
        st.deserialize(blob)
    p = str(tmp_path / "bad.safetensors")
    open(p, "wb").write(blob)
    with pytest.raises(emx.EmxError) as ei:
        emx.safetensors_index(p)
    assert ei.value.code == emx.ERR_INVALID


def test_deep_nesting_and_bad_strings_are_rejected(tmp_path):
    p = str(tmp_path / "deep.safetensors")
    open(p, "wb").write(_container(b'{"__metadata__":' + b"[" * 100 + b"]" * 100 + b"}"))
    with pytest.raises(emx.EmxError):
        emx.safetensors_index(p)
    open(p, "wb").write(_container(b'{"a\\ud800":{}}'))
    with pytest.raises(emx.EmxError):
        emx.safetensors_index(p)


def test_escaped_names_and_metadata(tmp_path):
    p = str(tmp_path / "esc.safetensors")
    tensors = {"wéight/\"q\"": {"dtype": "uint8", "shape": [1], "data": b"\x05"}}
    st.serialize_file(tensors, p, metadata={"k": "v\n"})
    assert _emx_tensors(p) == _crate_tensors(p)


def test_missing_file_is_an_error():
    with pytest.raises(emx.EmxError) as ei:
        emx.safetensors_index("/nonexistent/model.safetensors")
    assert "cannot open" in ei.value.msg
