"""CPU tests of the device model's GGUF reader (q38cu_gguf_check, host only):
it must accept what the upstream reader accepts (src/io/qwen38_gguf.c:326-413)
and refuse truncated or corrupt files with a reason instead of reading past the
mapping - the upstream's own reader tests (tests/unit/test_qwen38_gguf.c) cover
the same cases."""
import ctypes
import struct

import pytest

ALIGN = 32


def _string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def small_gguf(tensor_offset=0, rows=2, magic=0x46554747, version=3, alignment=ALIGN, data=True):
    """One Q8_0 tensor [rows][32] (34 bytes per row) and two metadata keys."""
    meta = [("general.architecture", 8, "qwen35"), ("general.alignment", 4, alignment)]
    head = struct.pack("<IIQQ", magic, version, 1, len(meta))
    for key, kind, value in meta:
        head += _string(key) + struct.pack("<I", kind)
        head += _string(value) if kind == 8 else struct.pack("<I", value)
    head += _string("blk.0.w") + struct.pack("<I", 2) + struct.pack("<QQ", 32, rows)
    head += struct.pack("<IQ", 8, tensor_offset)
    head += b"\0" * ((-len(head)) % ALIGN)
    return head + (bytes(range(34)) * rows if data else b"")


@pytest.fixture(scope="module")
def check(q38):
    fn = q38.lib().q38cu_gguf_check
    fn.argtypes = [ctypes.c_char_p]
    fn.restype = ctypes.c_uint64
    return fn


def _run(check, tmp_path, blob, name="m.gguf"):
    path = tmp_path / name
    path.write_bytes(blob)
    return check(str(path).encode())


def test_valid_file_is_accepted(check, tmp_path):
    assert _run(check, tmp_path, small_gguf()) == 1


@pytest.mark.parametrize("cut", [0, 8, 23, 40, 100])
def test_truncated_header_or_tables_refused(check, tmp_path, q38, cut):
    assert _run(check, tmp_path, small_gguf()[:cut]) == 0
    assert q38.last_error()


def test_tensor_data_past_end_refused(check, tmp_path, q38):
    blob = small_gguf()
    assert _run(check, tmp_path, blob[:-1]) == 0
    assert "outside" in q38.last_error()
    assert _run(check, tmp_path, small_gguf(tensor_offset=1 << 40)) == 0


@pytest.mark.parametrize("kw", [dict(magic=0x46554746), dict(version=1), dict(version=4), dict(alignment=24)])
def test_corrupt_header_refused(check, tmp_path, q38, kw):
    assert _run(check, tmp_path, small_gguf(**kw)) == 0
    assert q38.last_error()


def test_missing_file_refused(check, tmp_path, q38):
    assert check(str(tmp_path / "absent.gguf").encode()) == 0
    assert "cannot open" in q38.last_error()
