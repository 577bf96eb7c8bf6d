"""The library's checkpoint reader (``s1c_weights_*``) on CPU, against the behaviour of the
reference's ``laya_core::Weights`` (runtime/crates/laya-core/src/weights.rs): a missing file and a
file cut anywhere are errors that name the file (``open_rejects_a_missing_or_truncated_file``,
weights.rs:146-188, and laya-mlx/tests/loading.rs:79-104), ``verify`` names a missing parameter
family, tensor views hold the file's bytes, and malformed layouts are refused at open. Only host
code runs here: no CUDA call is made.
"""
import os

import numpy as np
import pytest

from sys1rust_b200.backend import WeightsError, WeightsFile
from sys1rust_b200.weights import write_safetensors

CUT = "bytes) is truncated or not a safetensors file"


def _two_tensor_file(path):
    """Like the reference test: an F16 [32, 32] encoder tensor and an F32 [16, 32] act_head one."""
    rng = np.random.default_rng(0)
    a = rng.standard_normal((32, 32)).astype(np.float16).view(np.uint16)
    b = rng.standard_normal((16, 32)).astype(np.float32)
    write_safetensors(str(path), {"encoder.w": ("F16", a), "act_head.0.weight": ("F32", b)})
    return a, b


def test_missing_or_truncated_file_is_an_error_naming_it(tmp_path):
    with pytest.raises(WeightsError, match="'model.safetensors' not found in"):
        WeightsFile(str(tmp_path))
    path = tmp_path / "model.safetensors"
    _two_tensor_file(path)
    full = path.read_bytes()
    header_end = 8 + int.from_bytes(full[:8], "little")
    for cut in [0, 4, 8, header_end // 2, header_end, header_end + 100, len(full) - 1]:
        path.write_bytes(full[:cut])
        with pytest.raises(WeightsError) as e:
            WeightsFile(str(tmp_path))
        assert f"model.safetensors ({cut} {CUT}" in str(e.value), (cut, str(e.value))
        assert str(tmp_path) in str(e.value)
    path.write_bytes(full)
    with WeightsFile(str(tmp_path)) as wf:
        assert sorted(wf.names()) == ["act_head.0.weight", "encoder.w"]


def test_tensor_views_hold_the_file_bytes(tmp_path):
    rng = np.random.default_rng(1)
    t = {
        "encoder.f32": ("F32", rng.standard_normal((3, 5)).astype(np.float32)),
        "encoder.f16": ("F16", rng.standard_normal((7,)).astype(np.float16).view(np.uint16)),
        "encoder.bf16": ("BF16", (rng.standard_normal((2, 2, 3)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)),
        "encoder.f64": ("F64", rng.standard_normal((4, 1)).astype(np.float64)),
        "encoder.ids": ("I64", np.arange(6, dtype=np.int64)),
    }
    write_safetensors(str(tmp_path / "model.safetensors"), t)
    with WeightsFile(str(tmp_path)) as wf:
        assert wf.names() == ["encoder.f32", "encoder.f16", "encoder.bf16", "encoder.f64", None]
        for name in ["encoder.f32", "encoder.f16", "encoder.bf16", "encoder.f64"]:
            dt, shape, arr = wf.tensor(name)
            assert dt == t[name][0] and shape == t[name][1].shape
            assert arr.tobytes() == t[name][1].tobytes()
        with pytest.raises(WeightsError, match="unsupported dtype I64"):
            wf.tensor("encoder.ids")
        with pytest.raises(WeightsError, match="not found"):
            wf.tensor("encoder.nope")


def test_verify_names_the_missing_family(tmp_path):
    z = ("F32", np.zeros((2,), dtype=np.float32))
    names = ["encoder.a", "type_emb.weight", "scorer.0.weight", "act_head.0.weight"]
    for missing in range(4):
        d = tmp_path / f"m{missing}"
        d.mkdir()
        write_safetensors(str(d / "model.safetensors"), {n: z for i, n in enumerate(names) if i != missing})
        prefix = names[missing].split(".")[0] + "."
        with WeightsFile(str(d)) as wf, pytest.raises(WeightsError) as e:
            wf.verify()
        assert f"checkpoint is missing '{prefix}' parameters; expected an RL Agent decision model" in str(e.value)
    d = tmp_path / "ok"
    d.mkdir()
    write_safetensors(str(d / "model.safetensors"), {n: z for n in names})
    with WeightsFile(str(d)) as wf:
        wf.verify()


def _raw(path, header: bytes, data: bytes):
    header += b" " * ((8 - len(header) % 8) % 8)
    path.write_bytes(len(header).to_bytes(8, "little") + header + data)


@pytest.mark.parametrize("header,data", [
    (b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}', b"\0" * 8),          # JSON cut short
    (b'{"a":{"dtype":"F32","shape":[3],"data_offsets":[0,8]}}', b"\0" * 8),         # dtype x shape != span
    (b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[4,12]}}', b"\0" * 12),       # gap before the first
    (b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},'
     b'"b":{"dtype":"F32","shape":[2],"data_offsets":[4,12]}}', b"\0" * 12),         # overlap
    (b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}', b"\0" * 16),        # trailing bytes
    (b'{"a":{"dtype":"Q7","shape":[2],"data_offsets":[0,8]}}', b"\0" * 8),          # unknown dtype
    (b'[1,2,3]', b""),                                                               # not an object
    (b'{"a":{"dtype":"F32","shape":[-2],"data_offsets":[0,8]}}', b"\0" * 8),        # negative dim
])
def test_malformed_layouts_are_refused_at_open(tmp_path, header, data):
    path = tmp_path / "model.safetensors"
    _raw(path, header, data)
    with pytest.raises(WeightsError, match="is truncated or not a safetensors file"):
        WeightsFile(str(tmp_path))


def test_metadata_entry_and_escaped_names_are_read(tmp_path):
    _raw(tmp_path / "model.safetensors",
         b'{"__metadata__":{"format":"pt"},"enc\\u00e9.\\"q\\"":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}',
         np.array([1.5], dtype=np.float32).tobytes())
    with WeightsFile(str(tmp_path)) as wf:
        assert wf.names() == ['encé."q"']
        assert wf.tensor('encé."q"')[2][0] == 1.5
