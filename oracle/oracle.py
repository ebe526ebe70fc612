"""CPU oracle for the BlockFHT hot path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes front end over ``liblwl_oracle.so`` (built from
``oracle/lwl_oracle.c`` by ``oracle/Makefile``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
import this module; the product package never does.

Reference behaviour restated here (file:line within verithia/latent-weight-lab):

* ``sign_word``           latent_weight_lab/block_fht.py:46-52
* ``fht_forward``         latent_weight_lab/block_fht.py:84-109 (block_fht_slice_torch)
* ``fht_backward``        latent_weight_lab/block_fht.py:179-196 (autograd of the above)
* ``linear_forward``      latent_weight_lab/block_fht.py:291-311 (_BlockFHTLinearFn.forward:
                          W = slice(0, in*out) * scale, viewed [out, in], then x @ W^T)
* ``linear_backward``     latent_weight_lab/block_fht.py:323-356
* ``fixed_fht_mix``       examples/nanogpt/model.py:182-218 (normalized_fht_last_dim,
                          FixedFHTMix.forward); its own adjoint, so also the gradient
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liblwl_oracle.so"
_LIB = None


def build() -> Path:
    """Compile the oracle shared library (idempotent)."""
    src = _HERE / "lwl_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _lib():
    global _LIB
    if _LIB is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        i64, f32p = ctypes.c_int64, ctypes.POINTER(ctypes.c_float)
        lib.lwl_oracle_sign_word.restype = ctypes.c_uint32
        lib.lwl_oracle_sign_word.argtypes = [i64, i64, i64, i64]
        for fn in (lib.lwl_oracle_fht_forward, lib.lwl_oracle_fht_backward):
            fn.restype = ctypes.c_int
            fn.argtypes = [f32p, i64, i64, ctypes.c_int, i64, i64, i64, f32p, ctypes.c_int, ctypes.c_int]
        lib.lwl_oracle_max_threads.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def _fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def max_threads() -> int:
    return int(_lib().lwl_oracle_max_threads())


def next_power_of_two(value: int) -> int:
    """block_fht.py:12-15."""
    if value <= 0:
        raise ValueError("value must be positive")
    return 1 << (int(value) - 1).bit_length()


def sign_word(seed: int, block: int, layer: int, word: int) -> int:
    """One uint32 sign word (bit p of word w is the sign of position 32w+p)."""
    s = int(seed) & ((1 << 64) - 1)
    if s >= 1 << 63:
        s -= 1 << 64
    return int(_lib().lwl_oracle_sign_word(s, int(block), int(layer), int(word)))


def _seed64(seed: int) -> int:
    s = int(seed) & ((1 << 64) - 1)
    return s - (1 << 64) if s >= 1 << 63 else s


def fht_forward(latent, size: int, layers: int, seed: int, start: int, stop: int,
                precision: str = "fp32", threads: int = 0) -> np.ndarray:
    """Generated coordinates [start, stop) as fp32 (fp64 math when precision='fp64')."""
    z = np.ascontiguousarray(np.asarray(latent, dtype=np.float32).reshape(-1))
    out = np.empty(int(stop) - int(start), dtype=np.float32)
    rc = _lib().lwl_oracle_fht_forward(_fp(z), z.size, int(size), int(layers), _seed64(seed),
                                       int(start), int(stop), _fp(out),
                                       1 if precision == "fp64" else 0, int(threads))
    if rc != 0:
        raise ValueError(f"invalid oracle forward arguments (slice [{start}, {stop}) size {size})")
    return out


def fht_backward(grad_out, latent_size: int, size: int, layers: int, seed: int, start: int,
                 stop: int, precision: str = "fp32", threads: int = 0) -> np.ndarray:
    """d/dz of sum(forward(z)[start:stop] * grad_out), as fp32 [latent_size]."""
    g = np.ascontiguousarray(np.asarray(grad_out, dtype=np.float32).reshape(-1))
    if g.size != int(stop) - int(start):
        raise ValueError("grad_out length must equal stop - start")
    out = np.empty(int(latent_size), dtype=np.float32)
    rc = _lib().lwl_oracle_fht_backward(_fp(g), int(latent_size), int(size), int(layers),
                                        _seed64(seed), int(start), int(stop), _fp(out),
                                        1 if precision == "fp64" else 0, int(threads))
    if rc != 0:
        raise ValueError("invalid oracle backward arguments")
    return out


def generated_weight(latent, in_features: int, out_features: int, layers: int, seed: int,
                     weight_scale: float = 1.0, precision: str = "fp32") -> np.ndarray:
    """W = forward(z)[0:in*out] * scale viewed as [out, in] (block_fht.py:306-310)."""
    size = int(in_features) * int(out_features)
    w = fht_forward(latent, size, layers, seed, 0, size, precision=precision)
    return (w * np.float32(weight_scale)).reshape(int(out_features), int(in_features))


def linear_forward(x, latent, out_features: int, layers: int, seed: int,
                   weight_scale: float = 1.0, bias=None) -> np.ndarray:
    """y = x @ W^T (+ bias), fp64 accumulation over the fp32 oracle weight."""
    x = np.asarray(x, dtype=np.float64)
    w = generated_weight(latent, x.shape[-1], out_features, layers, seed, weight_scale)
    y = x.reshape(-1, x.shape[-1]) @ w.astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float64)
    return y.reshape(*x.shape[:-1], int(out_features))


def linear_backward(grad_y, x, latent, out_features: int, layers: int, seed: int,
                    weight_scale: float = 1.0):
    """(grad_x, grad_latent, grad_bias) of block_fht.py:323-356 with modulation 0."""
    x2 = np.asarray(x, dtype=np.float64).reshape(-1, np.shape(x)[-1])
    g2 = np.asarray(grad_y, dtype=np.float64).reshape(-1, int(out_features))
    in_features = x2.shape[1]
    w = generated_weight(latent, in_features, out_features, layers, seed, weight_scale)
    grad_x = (g2 @ w.astype(np.float64)).reshape(np.shape(x))
    grad_w = g2.T @ x2
    size = in_features * int(out_features)
    z = np.asarray(latent, dtype=np.float32).reshape(-1)
    grad_z = np.float64(weight_scale) * fht_backward(grad_w.reshape(-1).astype(np.float32), z.size,
                                                     size, layers, seed, 0, size)
    return grad_x, grad_z, g2.sum(axis=0)


def normalized_wht_last_dim(values) -> np.ndarray:
    """Natural-order Walsh-Hadamard over the last axis times 1/sqrt(n), fp64
    (examples/nanogpt/model.py:182-197: radix-2 butterflies a+b, a-b with the
    stride doubling from 1)."""
    out = np.array(values, dtype=np.float64)
    n = out.shape[-1]
    if n & (n - 1):
        raise ValueError("FHT size must be a power of two")
    h = 1
    while h < n:
        v = out.reshape(*out.shape[:-1], n // (2 * h), 2, h)
        a, b = v[..., 0, :].copy(), v[..., 1, :].copy()
        v[..., 0, :], v[..., 1, :] = a + b, a - b
        out = v.reshape(*out.shape[:-1], n)
        h *= 2
    return out / np.sqrt(n)


def fixed_fht_mix(x, signs) -> np.ndarray:
    """(S * H_P/sqrt(P) * S * pad(x))[..., :F] over the last axis, P = len(signs)
    (examples/nanogpt/model.py:211-218)."""
    x = np.asarray(x, dtype=np.float64)
    s = np.asarray(signs, dtype=np.float64)
    F = x.shape[-1]
    pad = np.zeros(x.shape[:-1] + (s.size,), dtype=np.float64)
    pad[..., :F] = x
    return (normalized_wht_last_dim(pad * s) * s)[..., :F]
