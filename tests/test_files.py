"""The safetensors reader of libqtts.so (qtts_safetensors_*; the role of
TSafeTensorsFile, talker.pas:299-332) on the CPU: files written by the
safetensors package (huggingface/safetensors 0.7) read back name by name,
dtype, shape and bytes, and malformed files refused with QTTS_E_ARG."""
import json
import struct

import numpy as np
import pytest
import torch
from safetensors.numpy import save_file as save_np
from safetensors.torch import save_file as save_torch

import qtts


def test_reads_what_safetensors_wrote(tmp_path):
    rng = np.random.default_rng(1)
    arrays = {
        "talker.model.layers.0.self_attn.q_proj.weight": rng.standard_normal((64, 32)).astype(np.float32),
        "f16": rng.standard_normal((3, 5, 7)).astype(np.float16),
        "i64": np.arange(11, dtype=np.int64),
        "u8": np.arange(256, dtype=np.uint8).reshape(16, 16),
        "scalar": np.array(3.5, dtype=np.float32),
        "empty": np.zeros((0, 4), np.float32),
        'quote"and\\slash': np.ones(2, np.float32),
        "café": np.ones(1, np.float32),
    }
    path = tmp_path / "a.safetensors"
    save_np(arrays, str(path), metadata={"format": "pt", "note": "{not: json}"})
    f = qtts.SafeTensorsFile(path)
    assert sorted(f.names()) == sorted(arrays)
    names = {"F32": np.float32, "F16": np.float16}
    for k, a in arrays.items():
        dt, shape, raw = f.tensor(k)
        assert shape == a.shape, k
        assert raw == a.tobytes(), k
        assert dt == ("other" if a.dtype not in (np.float32, np.float16) else
                      next(n for n, t in names.items() if t == a.dtype)), k
    with pytest.raises(qtts.EQwenLm) as e:
        f.tensor("absent")
    assert e.value.code == qtts.E_ARG
    f.close()


def test_reads_bf16(tmp_path):
    t = torch.randn(48, 32).to(torch.bfloat16)
    path = tmp_path / "b.safetensors"
    save_torch({"talker.codec_head.weight": t, "norm": torch.ones(32, dtype=torch.bfloat16)}, str(path))
    f = qtts.SafeTensorsFile(path)
    dt, shape, raw = f.tensor("talker.codec_head.weight")
    assert dt == "BF16" and shape == (48, 32)
    assert raw == t.view(torch.int16).numpy().tobytes()
    f.close()


def write_raw(path, header, data=b"", size=None):
    h = json.dumps(header).encode() if isinstance(header, dict) else header
    n = len(h) if size is None else size
    path.write_bytes(struct.pack("<Q", n) + h + data)


@pytest.mark.parametrize("case", ["short", "beyond", "not_json", "not_object", "offsets", "shape", "dtype",
                                  "twice", "trailing", "missing_key"])
def test_refuses_malformed_files(tmp_path, case):
    p = tmp_path / f"{case}.safetensors"
    good = {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    if case == "short":
        p.write_bytes(b"\x01\x02")
    elif case == "beyond":
        write_raw(p, good, b"\0" * 8, size=10_000)
    elif case == "not_json":
        write_raw(p, b"{\"a\": {\"dtype\": \"F32\", \"shape\": [2], \"data_offsets\": [0, 8]", b"\0" * 8)
    elif case == "not_object":
        write_raw(p, b"[1, 2]", b"")
    elif case == "offsets":
        write_raw(p, {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 16]}}, b"\0" * 8)
    elif case == "shape":
        write_raw(p, {"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "dtype":
        write_raw(p, {"a": {"dtype": "F31", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "twice":
        write_raw(p, b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]},'
                     b' "a": {"dtype": "F32", "shape": [1], "data_offsets": [4, 8]}}', b"\0" * 8)
    elif case == "trailing":
        write_raw(p, json.dumps(good).encode() + b" x", b"\0" * 8)
    elif case == "missing_key":
        write_raw(p, {"a": {"dtype": "F32", "shape": [2]}}, b"\0" * 8)
    with pytest.raises(qtts.EQwenLm) as e:
        qtts.SafeTensorsFile(p)
    assert e.value.code == qtts.E_ARG


def test_missing_file(tmp_path):
    with pytest.raises(qtts.EQwenLm) as e:
        qtts.SafeTensorsFile(tmp_path / "none.safetensors")
    assert e.value.code == qtts.E_ARG
