"""CPU: the repacked-weight cache file is validated on the host before any device work: a wrong
magic, version, shape/size relation, truncated or extended payload, or a checksum mismatch is
G4Q_ERR_MODEL_LOAD with a message (no GPU needed to reach those checks)."""
import ctypes
import struct

import pytest

from conftest import ROOT  # noqa: F401


def fnv1a(data: bytes) -> int:
    h = 0xcbf29ce484222325
    for b in data:
        h = ((h ^ b) * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return h


def cache_bytes(rows=16, cols=64, magic=b"G4QWCACH", version=1, payload=None, checksum=None, extra=b""):
    pb, sb = rows * cols // 2, rows * (cols // 64) * 4
    payload = bytes(range(256)) * ((pb + sb) // 256 + 1) if payload is None else payload
    payload = payload[:pb + sb] if len(payload) > pb + sb else payload
    cs = fnv1a(payload) if checksum is None else checksum
    hdr = struct.pack("<8sIIqqiiQQQ", magic, version, 1, rows, cols, 4, 64, pb, sb, cs)
    assert len(hdr) == 64
    return hdr + payload + extra


@pytest.mark.parametrize("case,needle", [
    ("magic", "not a version-1"), ("version", "not a version-1"), ("truncated", "checksum mismatch"),
    ("extended", "checksum mismatch"), ("checksum", "checksum mismatch"), ("shape", "not a version-1"),
])
def test_corrupt_cache_files_are_rejected(tmp_path, case, needle):
    from helios_b200 import _lib
    L = _lib.load()
    good = cache_bytes()
    data = {
        "magic": cache_bytes(magic=b"G4QWCACX"),
        "version": cache_bytes(version=2),
        "truncated": good[:-1],
        "extended": cache_bytes(extra=b"\0"),
        "checksum": cache_bytes(checksum=1),
        "shape": cache_bytes(rows=17),
    }[case]
    f = tmp_path / "w.g4qc"
    f.write_bytes(data)
    h = ctypes.c_void_p()
    assert L.g4q_weight_open(str(f).encode(), ctypes.byref(h)) == _lib.G4Q_ERR_MODEL_LOAD
    assert needle in _lib.last_error() and not h


def test_missing_cache_file(tmp_path):
    from helios_b200 import _lib
    L = _lib.load()
    h = ctypes.c_void_p()
    assert L.g4q_weight_open(str(tmp_path / "nope").encode(), ctypes.byref(h)) == _lib.G4Q_ERR_MODEL_LOAD
    assert "cannot open" in _lib.last_error()
    assert L.g4q_weight_save(None, b"x") == _lib.G4Q_ERR_INVALID_ARGUMENT
