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


def test_fixed_fht_mix_validation_without_gpu(native_lib):
    assert native_lib.lwl_fixed_fht_mix(7, None, 4, 24, None, None, None) == 1
    assert b"dtype" in native_lib.lwl_last_error()
    assert native_lib.lwl_fixed_fht_mix(0, None, 4, 0, None, None, None) == 1
    assert native_lib.lwl_fixed_fht_mix(0, None, 4, 9000, None, None, None) == 2
    assert b"8192" in native_lib.lwl_last_error()
    assert native_lib.lwl_fixed_fht_mix(0, None, 0, 24, None, None, None) == 0  # no rows: nothing to do
    assert native_lib.lwl_fixed_fht_mix(0, None, 3, 24, None, None, None) == 1  # null pointers


def test_linear_backward_validation_without_gpu(native_lib):
    f = native_lib.lwl_linear_backward
    # (dtype, x, grad_y, tokens, in, out, latent, latent_size, layers, seed, scale, grad_x, grad_latent, ws, ws_bytes, flags, stream)
    assert f(0, None, None, 4, 0, 8, None, 10, 3, 1, 1.0, None, None, None, 0, 0, None) == 1
    assert f(0, None, None, 4, 8, 8, None, 10, 4, 1, 1.0, None, None, None, 0, 0, None) == 1
    assert b"layers" in native_lib.lwl_last_error()
    assert f(0, None, None, 4, 8, 8, None, 10, 3, 1, 1.0, None, None, None, 0, 0, None) == 0  # no outputs requested
    assert f(0, None, None, 4, 8, 8, None, 10, 3, 1, 1.0, 16, None, None, 0, 0, None) == 1  # null latent / grad_y
    assert b"null" in native_lib.lwl_last_error()


def test_linear_forward_ex_rejects_non_bf16(native_lib):
    st = native_lib.lwl_linear_forward_ex(0, None, 4, 64, None, 100, 128, 3, 1, 1.0, None, None, None, None, None, 1.0,
                                          None, None, 0, None)
    assert st == 2
    assert b"bf16" in native_lib.lwl_last_error()


def test_grouped_backward_validation_without_gpu(native_lib):
    from latent_weight_lab import _native

    assert native_lib.lwl_fht_backward_grouped(1, -1, None, None, 0, 0, None) == 1
    assert native_lib.lwl_fht_backward_grouped(1, 0, None, None, 0, 0, None) == 0
    assert native_lib.lwl_fht_backward_grouped_workspace_bytes(1, 0, None, 0) == 0
    descs = (_native.BackwardDesc * 1)()
    descs[0] = _native.BackwardDesc(None, 8, 40, 4, 1, 0, 10, None)  # layers 4
    assert native_lib.lwl_fht_backward_grouped(1, 1, descs, None, 0, 0, None) == 1
    assert b"layers" in native_lib.lwl_last_error()
    descs[0] = _native.BackwardDesc(None, 8, 40, 3, 1, 0, 10, None)  # null output
    assert native_lib.lwl_fht_backward_grouped(1, 1, descs, None, 0, 0, None) == 1
    assert b"null" in native_lib.lwl_last_error()
