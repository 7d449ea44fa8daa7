"""ctypes binding of libactfold_b200.so (the C ABI declared in include/actfold_b200.h).

There is no CPU or alternative backend: every op in this package calls the
CUDA library and raises when it is missing or when a tensor is not on a CUDA
device.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libactfold_b200.so")

AF_OK, AF_ERR_ARG, AF_ERR_CAPACITY, AF_ERR_DEVICE, AF_ERR_TIMEOUT, AF_ERR_CUDA, AF_ERR_COMM = range(7)
DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
METRIC = {"cosine": 0, "l2": 1, "pearson": 2}

_i64, _i32, _f32, _vp = C.c_int64, C.c_int, C.c_float, C.c_void_p

# name -> (restype, argtypes); must match include/actfold_b200.h
SIGNATURES: dict[str, tuple] = {
    "af_version": (C.c_char_p, []),
    "af_set_attention_kernel": (_i32, [_i32]),
    "af_last_error_string": (C.c_char_p, []),
    "af_gate": (
        _i32,
        [_vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _f32, _f32, _f32, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp],
    ),
    "af_merge_rows": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "af_gather_rows_masked": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _i32, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "af_gather_rows_index": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp]),
    "af_linear_bf16": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _i32, _i32, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _vp, _vp],
    ),
    "af_attention_bf16": (
        _i32,
        [_vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _f32,
         _vp, _vp],
    ),
}

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load (once) and return the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} not found: build it with `python -m actfold_b200.build` "
                "(the folding path has no CPU implementation)"
            )
        lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, what: str = "") -> None:
    """Map an af_status to the reference's Python exception types."""
    if status == AF_OK:
        return
    msg = load().af_last_error_string().decode(errors="replace")
    if status == AF_ERR_ARG:
        raise ValueError(msg or what)
    if status == AF_ERR_CAPACITY:
        raise ValueError(f"capacity exceeded: {msg or what}")
    if status == AF_ERR_TIMEOUT:
        raise TimeoutError(msg or what)
    raise RuntimeError(f"actfold_b200 error {status}: {msg or what}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor, what: str = "actfold_b200") -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"{what}: tensors must be on a CUDA device (got {t.device}); "
                "the B200 folding path has no CPU implementation"
            )


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
