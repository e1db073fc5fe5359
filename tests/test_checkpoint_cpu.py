"""The native safetensors reader (include/qwen_b200_loader.h, host side only:
header parsing, validation, raw reads) against the ``safetensors`` library
that writes the files, plus the checkpoint discovery and geometry checks of
qwen0.6b_b200/checkpoint.py.  No CUDA call is made here.
"""
import json
import struct

import pytest
import torch

st = pytest.importorskip("safetensors.torch")

from checkpoint import SafetensorsFile, checkpoint_files, read_config  # noqa: E402


def _tensors():
    g = torch.Generator().manual_seed(3)
    return {
        "a.f16": torch.randn(7, 5, generator=g).half(),
        "b.bf16": torch.randn(3, 1, 9, generator=g).bfloat16(),
        "c.f32": torch.randn(11, generator=g),
        "d.i64": torch.arange(6, dtype=torch.int64).view(2, 3),
        "e.scalar": torch.tensor(2.5, dtype=torch.float16),
        "f.empty": torch.zeros(0, 4, dtype=torch.bfloat16),
        "g.unicode.名前": torch.ones(2, dtype=torch.float32),
    }


def _raw(t: torch.Tensor) -> bytes:
    return t.contiguous().view(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""


def test_reader_matches_safetensors(tmp_path):
    ts = _tensors()
    p = str(tmp_path / "m.safetensors")
    st.save_file(ts, p, metadata={"format": "pt", "note": "quote \" and \\ and é"})
    with SafetensorsFile(p) as f:
        assert sorted(f.names()) == sorted(ts)
        for name, t in ts.items():
            assert f.shape(name) == tuple(t.shape), name
            assert f.read_bytes(name) == _raw(t), name
        assert f.dtype("a.f16") == "F16" and f.dtype("b.bf16") == "BF16" and f.dtype("c.f32") == "F32"
        assert f.dtype("d.i64") == "other"
        assert f.metadata("format") == "pt"
        assert f.metadata("note") == "quote \" and \\ and é"
        assert f.metadata("missing") is None


def _write_raw(path, header: dict | bytes, data: bytes = b"", length=None):
    h = header if isinstance(header, bytes) else json.dumps(header).encode()
    n = len(h) if length is None else length
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", n) + h + data)


@pytest.mark.parametrize("header,data,length,pattern", [
    ({"x": {"dtype": "F16", "shape": [4], "data_offsets": [0, 8]}}, b"\0" * 4, None, "outside the file"),
    ({"x": {"dtype": "F16", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8, None, "does not match"),
    ({"x": {"dtype": "Q4", "shape": [1], "data_offsets": [0, 1]}}, b"\0", None, "unknown dtype"),
    ({"x": {"dtype": "F16", "shape": [-1], "data_offsets": [0, 0]}}, b"", None, "bad shape"),
    ({"x": {"dtype": "F16", "shape": [1]}}, b"\0\0", None, "data_offsets"),
    (b'{"x": {"dtype": "F16", "shape": [1], "data_offsets": [0, 2]}', b"\0\0", None, "header"),
    (b'{"x": 1.5}', b"", None, "non-integer"),
    ({"x": {"dtype": "F16", "shape": [1], "data_offsets": [0, 2]}}, b"\0\0", 1 << 40, "header length"),
    (b'{"x": {"dtype": "F16", "shape": [1], "data_offsets": [0, 2]},'
     b' "x": {"dtype": "F16", "shape": [1], "data_offsets": [0, 2]}}', b"\0\0", None, "duplicate"),
])
def test_reader_rejects_malformed_files(tmp_path, header, data, length, pattern):
    p = str(tmp_path / "bad.safetensors")
    _write_raw(p, header, data, length)
    with pytest.raises(RuntimeError, match=pattern):
        SafetensorsFile(p)


def test_reader_rejects_short_and_missing_files(tmp_path):
    p = tmp_path / "short.safetensors"
    p.write_bytes(b"\1\0")
    with pytest.raises(RuntimeError, match="shorter"):
        SafetensorsFile(str(p))
    with pytest.raises(RuntimeError, match="No such file"):
        SafetensorsFile(str(tmp_path / "none.safetensors"))


def test_checkpoint_files_and_index(tmp_path):
    st.save_file({"a": torch.zeros(2)}, str(tmp_path / "model-00002-of-00002.safetensors"))
    st.save_file({"b": torch.zeros(2)}, str(tmp_path / "model-00001-of-00002.safetensors"))
    files = checkpoint_files(str(tmp_path))
    assert [f.rsplit("/", 1)[1] for f in files] == ["model-00001-of-00002.safetensors",
                                                   "model-00002-of-00002.safetensors"]
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {"b": "model-00001-of-00002.safetensors"}}))
    assert [f.rsplit("/", 1)[1] for f in checkpoint_files(str(tmp_path))] == ["model-00001-of-00002.safetensors"]
    with pytest.raises(FileNotFoundError):
        checkpoint_files(str(tmp_path / "nothing"))


def test_read_config_checks_the_geometry(tmp_path):
    assert read_config(str(tmp_path)) == {}
    good = {"hidden_size": 1024, "intermediate_size": 3072, "num_attention_heads": 16,
            "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 151936, "rms_norm_eps": 1e-6,
            "num_hidden_layers": 28, "rope_theta": 1000000}
    (tmp_path / "config.json").write_text(json.dumps(good))
    assert read_config(str(tmp_path))["num_hidden_layers"] == 28
    (tmp_path / "config.json").write_text(json.dumps({**good, "hidden_size": 2048}))
    with pytest.raises(ValueError, match="hidden_size"):
        read_config(str(tmp_path))
