"""Python host mirror of the B200 NAFNet denoiser engine.

Binds the C-ABI of ``libdenoiser_b200.so`` (declared in
``include/denoiser_b200.h``) with ctypes. Device memory and streams come
from PyTorch tensors (``data_ptr()`` / ``torch.cuda.current_stream()``);
all arithmetic runs in the CUDA kernels of the shared library. There is no
CPU fallback: if the library is missing, importing the binding raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdenoiser_b200.so")

DN_OK = 0
DN_ERR_INVALID_ARG = -1
DN_ERR_CUDA = -2
DN_ERR_IO = -3
DN_ERR_FORMAT = -4
DN_ERR_NOT_FOUND = -5
DN_ERR_UNSUPPORTED = -6
DN_ERR_DEVICE = -7
DN_ERR_DTYPE = -8

_lib = None


class DenoiserError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class NotFoundError(DenoiserError, KeyError):
    """Missing weight key (the reference C++ engine throws std::out_of_range)."""


class InvalidArgumentError(DenoiserError, ValueError):
    """Bad argument (the reference C++ engine throws std::invalid_argument)."""


_c = ctypes
_P = _c.c_void_p
_I = _c.c_int
_I64 = _c.c_int64
_F = _c.c_float
_U32P = _c.POINTER(_c.c_uint32)

# name -> (restype, argtypes); every symbol of include/denoiser_b200.h.
SIGNATURES = {
    "dn_last_error": (_c.c_char_p, []),
    "dn_abi_version": (_I, []),
    "dn_umma_probe": (_I, [_P, _P, _P, _I, _I, _P, _P]),
}


def lib() -> ctypes.CDLL:
    """Load (once) and return the engine's shared library."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C ml-video-denoiser_b200` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int) -> None:
    """Raise the matching exception for a non-zero C-ABI status."""
    if rc == DN_OK:
        return
    msg = lib().dn_last_error().decode(errors="replace")
    if rc == DN_ERR_NOT_FOUND:
        raise NotFoundError(rc, msg)
    if rc == DN_ERR_INVALID_ARG:
        raise InvalidArgumentError(rc, msg)
    raise DenoiserError(rc, msg)


def stream_handle(stream=None) -> int:
    """cudaStream_t of a torch stream (default: the current stream)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def umma_probe(a, b):
    """D = A @ B^T through one tcgen05 tile (A: 128xK fp16, B: NxK fp16, cuda)."""
    import torch

    assert a.is_cuda and a.dtype == torch.float16 and a.shape[0] == 128
    n, k = b.shape
    d = torch.empty(128, n, dtype=torch.float32, device=a.device)
    err = torch.zeros(1, dtype=torch.int32, device=a.device)
    check(lib().dn_umma_probe(a.data_ptr(), b.data_ptr(), d.data_ptr(), n, k, err.data_ptr(),
                              stream_handle()))
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise DenoiserError(DN_ERR_DEVICE, f"device error word {int(err.item()):#x}")
    return d
