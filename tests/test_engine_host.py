"""Host-side checks of the engine's GGUF reader and model validation (engine.cu), no GPU needed:
eahmmf_engine_load parses and validates the whole file before its first CUDA call, so malformed or
unsupported files are refused with a message here, and a valid file gets past every check.
"""
import os
import struct

import pytest

import eahmmf_b200 as eb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")


def load_error(path):
    with pytest.raises(RuntimeError) as ei:
        eb.Engine(path, 64)
    return str(ei.value)


def gguf_bytes(kv, tensors=()):
    def s(x):
        b = x.encode()
        return struct.pack("<Q", len(b)) + b
    out = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, (t, v) in kv.items():
        out += s(k) + struct.pack("<I", t)
        out += s(v) if t == 8 else struct.pack("<I", v)
    for name, ne, qt, off in tensors:
        out += s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", n) for n in ne)
        out += struct.pack("<IQ", qt, off)
    return out


def test_not_a_gguf(tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"NOPE" + bytes(64))
    assert "not a GGUF file" in load_error(str(p))


def test_truncated_header(tmp_path):
    p = tmp_path / "t.gguf"
    p.write_bytes(open(TINY, "rb").read()[:700])
    assert "truncated" in load_error(str(p)) or "bad" in load_error(str(p))


def test_tensor_past_end_of_file(tmp_path):
    p = tmp_path / "e.gguf"
    p.write_bytes(gguf_bytes({"general.architecture": (8, "qwen3moe")}, [("w", (256, 4), 12, 0)]))
    assert "out of file bounds" in load_error(str(p))


def test_wrong_architecture(tmp_path):
    p = tmp_path / "a.gguf"
    p.write_bytes(gguf_bytes({"general.architecture": (8, "llama")}))
    assert "unsupported architecture" in load_error(str(p))


def test_missing_hyper_parameters(tmp_path):
    p = tmp_path / "h.gguf"
    p.write_bytes(gguf_bytes({"general.architecture": (8, "qwen3moe"), "qwen3moe.block_count": (4, 2)}))
    assert "missing hyper-parameters" in load_error(str(p))


def test_valid_model_passes_every_host_check():
    msg = load_error(TINY) if not _has_gpu() else None
    if msg is not None:  # without a device the first CUDA call is what fails
        assert not msg.split(":", 1)[1].strip().startswith(("gguf", "unsupported", "missing", "bad", "head"))


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
