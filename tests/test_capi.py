"""The C-ABI library: loads, exports every declared entry point, validates arguments on the host."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

HEADER_DIR = Path(__file__).resolve().parents[1] / "include"


def declared_functions() -> list[str]:
    names = []
    for h in sorted(HEADER_DIR.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(lwl_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("lwl_fht_forward", "lwl_fht_backward", "lwl_sign_words", "lwl_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol(native_lib):
    missing = [n for n in declared_functions() if not hasattr(native_lib, n)]
    assert not missing, f"symbols declared in include/*.h but not exported: {missing}"


def test_status_strings(native_lib):
    assert native_lib.lwl_status_string(0) == b"ok"
    assert native_lib.lwl_status_string(3) == b"workspace too small"
    assert native_lib.lwl_version() >= 100


@pytest.mark.parametrize(
    "args, message",
    [
        ((0, None, 8, 40, 0, 0, 0, 10, None, None, 0, 0, None), b"layers must be 1, 2, or 3"),
        ((0, None, 8, 40, 1, 0, 5, 41, None, None, 0, 0, None), b"invalid slice [5, 41) for size 40"),
        ((0, None, 0, 40, 1, 0, 0, 10, None, None, 0, 0, None), b"latent size must be positive"),
        ((7, None, 8, 40, 1, 0, 0, 10, None, None, 0, 0, None), b"unsupported dtype code 7"),
        ((0, None, 8, 0, 1, 0, 0, 0, None, None, 0, 0, None), b"size must be positive"),
    ],
)
def test_forward_validation_without_gpu(native_lib, args, message):
    status = native_lib.lwl_fht_forward(*args)
    assert status == 1
    assert native_lib.lwl_last_error().startswith(message)


def test_block_size_limit_reported_as_unsupported(native_lib):
    status = native_lib.lwl_fht_forward(0, None, (1 << 23) + 1, 1 << 24, 1, 0, 0, 16, None, None, 0, 0, None)
    assert status == 2
    assert b"2^23" in native_lib.lwl_last_error()


def test_backward_validation_without_gpu(native_lib):
    status = native_lib.lwl_fht_backward(0, None, 8, 40, 4, 0, 0, 10, None, None, 0, 0, None)
    assert status == 1


def test_null_pointers_rejected(native_lib):
    status = native_lib.lwl_fht_forward(0, None, 8, 40, 1, 0, 0, 10, None, None, 0, 0, None)
    assert status == 1
    assert b"null" in native_lib.lwl_last_error()
