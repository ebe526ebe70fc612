"""ctypes binding to liblwl_b200.so, the sm_100a BlockFHT library.

This module replaces the reference's JIT-built pybind extension
(latent_weight_lab/block_fht.py:112-146 and csrc/block_fht_ext.cpp).  Unlike
the reference it never falls back silently: a missing or broken library, or
a non-CUDA tensor, raises immediately.  torch supplies device memory and the
current stream; all arithmetic happens in the library's kernels.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblwl_b200.so"
_LOCK = threading.Lock()
_LIB = None
_LOAD_ERROR: Exception | None = None

LWL_F32, LWL_BF16, LWL_F16 = 0, 1, 2
FLAG_EXACT = 1
FLAG_TEST_WAIT_TIMEOUT = 0x80000000  # testing only: the tensor-core backward's first bounded wait gives up
_DTYPE_CODE = {torch.float32: LWL_F32, torch.bfloat16: LWL_BF16, torch.float16: LWL_F16}


class NativeError(RuntimeError):
    """A liblwl_b200 call returned a non-OK status."""


def library_path() -> Path:
    return Path(os.environ.get("LWL_B200_LIB", _LIB_PATH))


def _declare(lib: ctypes.CDLL) -> None:
    i64, u64, vp, sz, ci, cu = (ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t,
                                ctypes.c_int, ctypes.c_uint)
    lib.lwl_version.restype = ci
    lib.lwl_version.argtypes = []
    lib.lwl_status_string.restype = ctypes.c_char_p
    lib.lwl_status_string.argtypes = [ci]
    lib.lwl_last_error.restype = ctypes.c_char_p
    lib.lwl_last_error.argtypes = []
    lib.lwl_sign_words.restype = ci
    lib.lwl_sign_words.argtypes = [u64, i64, ci, i64, i64, vp, vp]
    for name in ("lwl_fht_forward_workspace_bytes", "lwl_fht_backward_workspace_bytes"):
        fn = getattr(lib, name)
        fn.restype = sz
        fn.argtypes = [ci, i64, i64, ci, i64, i64, cu]
    lib.lwl_fht_forward_grouped.restype = ci
    lib.lwl_fht_forward_grouped.argtypes = [ci, ci, ctypes.POINTER(ForwardDesc), cu, vp]
    lib.lwl_linear_forward_workspace_bytes.restype = sz
    lib.lwl_linear_forward_workspace_bytes.argtypes = []
    lib.lwl_linear_forward.restype = ci
    lib.lwl_linear_forward.argtypes = [ci, vp, i64, i64, vp, i64, i64, ci, u64, ctypes.c_float, vp, vp, sz, vp]
    lib.lwl_linear_forward_ex.restype = ci
    lib.lwl_linear_forward_ex.argtypes = [ci, vp, i64, i64, vp, i64, i64, ci, u64, ctypes.c_float, vp, vp, vp, vp, vp,
                                          ctypes.c_float, vp, vp, sz, vp]
    lib.lwl_linear_backward_workspace_bytes.restype = sz
    lib.lwl_linear_backward_workspace_bytes.argtypes = [ci, i64, i64, i64, i64, ci, cu]
    lib.lwl_linear_backward.restype = ci
    lib.lwl_linear_backward.argtypes = [ci, vp, vp, i64, i64, i64, vp, i64, ci, u64, ctypes.c_float, vp, vp, vp, sz,
                                        cu, vp]
    lib.lwl_fht_backward_grouped_workspace_bytes.restype = sz
    lib.lwl_fht_backward_grouped_workspace_bytes.argtypes = [ci, ci, ctypes.POINTER(BackwardDesc), cu]
    lib.lwl_fht_backward_grouped.restype = ci
    lib.lwl_fht_backward_grouped.argtypes = [ci, ci, ctypes.POINTER(BackwardDesc), vp, sz, cu, vp]
    lib.lwl_fixed_fht_mix.restype = ci
    lib.lwl_fixed_fht_mix.argtypes = [ci, vp, i64, i64, vp, vp, vp]
    lib.lwl_tc_linear_dense.restype = ci
    lib.lwl_tc_linear_dense.argtypes = [vp, i64, i64, vp, i64, vp, vp, sz, vp]
    lib.lwl_fht_launch_count.restype = ci
    lib.lwl_fht_launch_count.argtypes = [ci, i64, i64, ci, i64, i64, ci, cu]
    for name in ("lwl_fht_forward", "lwl_fht_backward"):
        fn = getattr(lib, name)
        fn.restype = ci
        fn.argtypes = [ci, vp, i64, i64, ci, u64, i64, i64, vp, vp, sz, cu, vp]
    lib.lwl_fht_backward_status.restype = ci
    lib.lwl_fht_backward_status.argtypes = [ci, i64, i64, ci, i64, i64, cu, vp, vp]
    lib.lwl_linear_forward_status.restype = ci
    lib.lwl_linear_forward_status.argtypes = [vp, vp]


class ForwardDesc(ctypes.Structure):
    """lwl_fht_forward_desc (include/lwl_b200.h)."""

    _fields_ = [("latent", ctypes.c_void_p), ("latent_size", ctypes.c_int64), ("size", ctypes.c_int64),
                ("layers", ctypes.c_int), ("seed", ctypes.c_uint64), ("start", ctypes.c_int64),
                ("stop", ctypes.c_int64), ("out", ctypes.c_void_p)]


class BackwardDesc(ctypes.Structure):
    """lwl_fht_backward_desc (include/lwl_b200.h)."""

    _fields_ = [("grad_out", ctypes.c_void_p), ("latent_size", ctypes.c_int64), ("size", ctypes.c_int64),
                ("layers", ctypes.c_int), ("seed", ctypes.c_uint64), ("start", ctypes.c_int64),
                ("stop", ctypes.c_int64), ("grad_latent", ctypes.c_void_p)]


def load() -> ctypes.CDLL:
    """Load the library once; raise (and keep raising) if that fails."""
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if _LOAD_ERROR is not None:
                raise _LOAD_ERROR
            path = library_path()
            try:
                if not path.exists():
                    raise FileNotFoundError(
                        f"{path} is missing; build it with `python latent-weight-lab_b200/build.py`")
                lib = ctypes.CDLL(str(path))
                _declare(lib)
            except Exception as exc:  # remembered so every later call fails the same way
                _LOAD_ERROR = RuntimeError(f"liblwl_b200 could not be loaded: {exc}")
                raise _LOAD_ERROR from exc
            _LIB = lib
    return _LIB


def load_error() -> Exception | None:
    return _LOAD_ERROR


def _check(status: int) -> None:
    if status != 0:
        lib = load()
        msg = lib.lwl_last_error().decode(errors="replace")
        kind = lib.lwl_status_string(status).decode()
        if status == 1:
            raise ValueError(msg or kind)
        raise NativeError(f"{kind}: {msg}")


def _seed_u64(seed: int) -> int:
    return int(seed) & ((1 << 64) - 1)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(
            f"{what} must be a CUDA tensor: this latent_weight_lab build computes on B200 GPUs only "
            "(move the module or tensor to a CUDA device)")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16") from None


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _workspace(nbytes: int, device: torch.device) -> tuple[torch.Tensor | None, int]:
    if nbytes == 0:
        return None, 0
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device), 0


def fht_forward(latent: torch.Tensor, size: int, layers: int, seed: int, start: int, stop: int,
                flags: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """y[start:stop] of the BlockFHT generator, same dtype as `latent`."""
    _require_cuda(latent, "latent")
    lib = load()
    latent = latent.contiguous()
    code = dtype_code(latent.dtype)
    n = int(stop) - int(start)
    if out is None:
        out = torch.empty(max(n, 0), dtype=latent.dtype, device=latent.device)
    with torch.cuda.device(latent.device):
        ws_bytes = lib.lwl_fht_forward_workspace_bytes(code, latent.numel(), int(size), int(layers),
                                                       int(start), int(stop), int(flags))
        ws, _ = _workspace(ws_bytes, latent.device)
        _check(lib.lwl_fht_forward(code, latent.data_ptr(), latent.numel(), int(size), int(layers),
                                   _seed_u64(seed), int(start), int(stop), out.data_ptr(),
                                   ws.data_ptr() if ws is not None else None, ws_bytes, int(flags),
                                   _stream_ptr(latent.device)))
    return out


def fht_backward(grad_out: torch.Tensor, latent_size: int, size: int, layers: int, seed: int,
                 start: int, stop: int, flags: int = 0) -> torch.Tensor:
    """d/dz sum(y[start:stop] * grad_out) as a [latent_size] tensor of grad_out's dtype."""
    _require_cuda(grad_out, "grad_out")
    lib = load()
    grad_out = grad_out.contiguous()
    code = dtype_code(grad_out.dtype)
    if grad_out.numel() != int(stop) - int(start):
        raise ValueError("grad_out must have stop - start elements")
    grad = torch.empty(int(latent_size), dtype=grad_out.dtype, device=grad_out.device)
    with torch.cuda.device(grad_out.device):
        ws_bytes = lib.lwl_fht_backward_workspace_bytes(code, int(latent_size), int(size), int(layers),
                                                        int(start), int(stop), int(flags))
        ws, _ = _workspace(ws_bytes, grad_out.device)
        _check(lib.lwl_fht_backward(code, grad_out.data_ptr(), int(latent_size), int(size), int(layers),
                                    _seed_u64(seed), int(start), int(stop), grad.data_ptr(),
                                    ws.data_ptr() if ws is not None else None, ws_bytes, int(flags),
                                    _stream_ptr(grad_out.device)))
    return grad


def sign_words(seed: int, block: int, layer: int, first_word: int, count: int,
               device: torch.device | str = "cuda") -> torch.Tensor:
    """Sign words [count] as int64 (values 0..2^32-1) computed on the GPU."""
    lib = load()
    device = torch.device(device)
    out = torch.empty(int(count), dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        _check(lib.lwl_sign_words(_seed_u64(seed), int(block), int(layer), int(first_word), int(count),
                                  out.data_ptr() if count else None, _stream_ptr(device)))
    return out.to(torch.int64) & 0xFFFFFFFF


def fht_forward_grouped(items, flags: int = 0) -> list[torch.Tensor]:
    """Several generator slices in as few launches as possible.

    items: sequence of (latent, size, layers, seed, start, stop); all latents
    share one CUDA device and dtype.  Returns one output tensor per item.
    """
    items = list(items)
    if not items:
        return []
    lib = load()
    dev, dt = items[0][0].device, items[0][0].dtype
    outs, keep = [], []
    descs = (ForwardDesc * len(items))()
    for i, (latent, size, layers, seed, start, stop) in enumerate(items):
        _require_cuda(latent, "latent")
        if latent.device != dev or latent.dtype != dt:
            raise ValueError("grouped generation needs one device and dtype")
        latent = latent.detach().contiguous()
        keep.append(latent)
        out = torch.empty(max(int(stop) - int(start), 0), dtype=dt, device=dev)
        outs.append(out)
        descs[i] = ForwardDesc(latent.data_ptr(), latent.numel(), int(size), int(layers), _seed_u64(seed),
                               int(start), int(stop), out.data_ptr() if out.numel() else None)
    with torch.cuda.device(dev):
        _check(lib.lwl_fht_forward_grouped(dtype_code(dt), len(items), descs, int(flags), _stream_ptr(dev)))
    return outs


def fht_backward_grouped(items, flags: int = 0) -> list[torch.Tensor]:
    """Several latent gradients in as few launches as possible.

    items: sequence of (grad_out, latent_size, size, layers, seed, start, stop);
    all gradients share one CUDA device and dtype.  Returns one [latent_size]
    gradient per item, in that dtype.
    """
    items = list(items)
    if not items:
        return []
    lib = load()
    dev, dt = items[0][0].device, items[0][0].dtype
    outs, keep = [], []
    descs = (BackwardDesc * len(items))()
    for i, (grad_out, latent_size, size, layers, seed, start, stop) in enumerate(items):
        _require_cuda(grad_out, "grad_out")
        if grad_out.device != dev or grad_out.dtype != dt:
            raise ValueError("grouped backward needs one device and dtype")
        grad_out = grad_out.contiguous()
        if grad_out.numel() != int(stop) - int(start):
            raise ValueError("grad_out must have stop - start elements")
        keep.append(grad_out)
        out = torch.empty(int(latent_size), dtype=dt, device=dev)
        outs.append(out)
        descs[i] = BackwardDesc(grad_out.data_ptr() if grad_out.numel() else None, int(latent_size), int(size),
                                int(layers), _seed_u64(seed), int(start), int(stop), out.data_ptr())
    code = dtype_code(dt)
    with torch.cuda.device(dev):
        nbytes = lib.lwl_fht_backward_grouped_workspace_bytes(code, len(items), descs, int(flags))
        ws, _ = _workspace(nbytes, dev)
        _check(lib.lwl_fht_backward_grouped(code, len(items), descs, ws.data_ptr() if ws is not None else None,
                                            nbytes, int(flags), _stream_ptr(dev)))
    return outs


def linear_forward(x2d: torch.Tensor, latent: torch.Tensor, out_features: int, layers: int, seed: int,
                   weight_scale: float = 1.0, return_status: bool = False, bias: torch.Tensor | None = None,
                   output_gain: torch.Tensor | None = None, input_gain: torch.Tensor | None = None,
                   weight_offset: torch.Tensor | None = None, base: torch.Tensor | None = None,
                   base_scale: float = 1.0):
    """Fused tcgen05 forward y = x @ (scale * W)^T with W generated on chip;
    optional bf16 bias / output_gain ([out]) and input_gain ([in]), and a
    scalar weight_offset added to every weight element (the modulation term),
    and a dense residual base weight ([out, in], the generated part scaled
    by base_scale) are folded into the kernel (lwl_linear_forward_ex).

    Returns None when the shape is outside the fused kernel (the caller then
    generates W and uses a library GEMM).  With return_status the device error
    word tensor is returned too (0 = every pipeline wait completed).
    """
    _require_cuda(x2d, "input")
    lib = load()
    x2d = x2d.contiguous()
    latent = latent.detach().contiguous()
    T, K = x2d.shape
    y = torch.empty(T, int(out_features), dtype=x2d.dtype, device=x2d.device)
    ws = torch.empty(lib.lwl_linear_forward_workspace_bytes(), dtype=torch.uint8, device=x2d.device)
    extras = [None if v is None else v.detach().to(device=x2d.device, dtype=torch.bfloat16).contiguous()
              for v in (bias, output_gain, input_gain)]
    extras.append(None if weight_offset is None else
                  weight_offset.detach().to(device=x2d.device, dtype=torch.float32).reshape(1).contiguous())
    extras.append(None if base is None else base.detach().to(device=x2d.device, dtype=torch.bfloat16).contiguous())
    with torch.cuda.device(x2d.device):
        if any(v is not None for v in extras):
            st = lib.lwl_linear_forward_ex(dtype_code(x2d.dtype), x2d.data_ptr(), T, K, latent.data_ptr(),
                                           latent.numel(), int(out_features), int(layers), _seed_u64(seed),
                                           float(weight_scale),
                                           *[v.data_ptr() if v is not None else None for v in extras],
                                           float(base_scale), y.data_ptr(), ws.data_ptr(), ws.numel(),
                                           _stream_ptr(x2d.device))
        else:
            st = lib.lwl_linear_forward(dtype_code(x2d.dtype), x2d.data_ptr(), T, K, latent.data_ptr(),
                                        latent.numel(), int(out_features), int(layers), _seed_u64(seed),
                                        float(weight_scale), y.data_ptr(), ws.data_ptr(), ws.numel(),
                                        _stream_ptr(x2d.device))
    if st == 2:
        return None
    _check(st)
    return (y, ws.view(torch.int32)[:1]) if return_status else y


def linear_backward(x2d: torch.Tensor, grad_y2d: torch.Tensor, latent: torch.Tensor, out_features: int,
                    layers: int, seed: int, weight_scale: float = 1.0, need_input: bool = True,
                    need_latent: bool = True, flags: int = 0):
    """Backward of y = x @ (scale * W)^T through lwl_linear_backward: returns
    (grad_x or None, grad_latent or None), both in the input dtype."""
    _require_cuda(x2d, "input")
    lib = load()
    x2d, grad_y2d, latent = x2d.contiguous(), grad_y2d.contiguous(), latent.detach().contiguous()
    if not (x2d.dtype == grad_y2d.dtype == latent.dtype):
        raise ValueError("input, grad_output and latent must have one dtype")
    T, K = x2d.shape
    code = dtype_code(x2d.dtype)
    gx = torch.empty_like(x2d) if need_input else None
    gz = torch.empty_like(latent) if need_latent else None
    nbytes = lib.lwl_linear_backward_workspace_bytes(code, T, K, int(out_features), latent.numel(), int(layers),
                                                     flags)
    ws, _ = _workspace(nbytes, x2d.device)
    with torch.cuda.device(x2d.device):
        _check(lib.lwl_linear_backward(code, x2d.data_ptr(), grad_y2d.data_ptr(), T, K, int(out_features),
                                       latent.data_ptr(), latent.numel(), int(layers), _seed_u64(seed),
                                       float(weight_scale), gx.data_ptr() if gx is not None else None,
                                       gz.data_ptr() if gz is not None else None,
                                       ws.data_ptr() if ws is not None else None, nbytes, flags,
                                       _stream_ptr(x2d.device)))
    return gx, gz


def fixed_fht_mix(x: torch.Tensor, signs: torch.Tensor) -> torch.Tensor:
    """(S * H_P/sqrt(P) * S * pad(x))[..., :F] over the last dimension through
    lwl_fixed_fht_mix; signs: fp32 [P] on x's device, P = next_pow2(F)."""
    _require_cuda(x, "input")
    lib = load()
    x = x.contiguous()
    F = x.shape[-1]
    sg = signs.to(device=x.device, dtype=torch.float32).contiguous()
    y = torch.empty_like(x)
    rows = x.numel() // F if F > 0 else 0
    with torch.cuda.device(x.device):
        _check(lib.lwl_fixed_fht_mix(dtype_code(x.dtype), x.data_ptr(), rows, F, sg.data_ptr(), y.data_ptr(),
                                     _stream_ptr(x.device)))
    return y


def tc_linear_dense(x2d: torch.Tensor, w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """y = x @ w^T on the tcgen05 linear pipeline (bf16); returns (y, device error word)."""
    lib = load()
    x2d, w = x2d.contiguous(), w.contiguous()
    T, K = x2d.shape
    N = w.shape[0]
    y = torch.empty(T, N, dtype=x2d.dtype, device=x2d.device)
    ws = torch.empty(16, dtype=torch.uint8, device=x2d.device)
    with torch.cuda.device(x2d.device):
        _check(lib.lwl_tc_linear_dense(x2d.data_ptr(), T, K, w.data_ptr(), N, y.data_ptr(), ws.data_ptr(), 16,
                                       _stream_ptr(x2d.device)))
    return y, ws.view(torch.int32)[:1]
