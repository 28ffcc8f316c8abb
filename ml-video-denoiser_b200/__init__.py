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

class ModelInfo(ctypes.Structure):
    """dn_model_info of include/denoiser_b200.h."""

    _fields_ = [("kind", ctypes.c_int), ("in_channels", ctypes.c_int), ("num_levels", ctypes.c_int),
                ("base_channels", ctypes.c_int), ("num_frames", ctypes.c_int), ("use_warp", ctypes.c_int),
                ("enc_channels", ctypes.c_int * 8)]


_PP = _c.POINTER(_c.c_void_p)
_I64P = _c.POINTER(_c.c_int64)
_IP = _c.POINTER(_c.c_int)
_SZP = _c.POINTER(_c.c_size_t)
_CPP = _c.POINTER(_c.c_char_p)

# name -> (restype, argtypes); every symbol of the headers in include/.
SIGNATURES = {
    "dn_last_error": (_c.c_char_p, []),
    "dn_abi_version": (_I, []),
    "dn_umma_probe": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    "dn_weights_open": (_I, [_c.c_char_p, _PP]),
    "dn_weights_close": (None, [_P]),
    "dn_weights_count": (_I, [_P]),
    "dn_weights_contains": (_I, [_P, _c.c_char_p]),
    "dn_weights_info": (_I, [_P, _c.c_char_p, _I64P, _IP, _IP, _PP]),
    "dn_weights_name": (_I, [_P, _I, _CPP]),
    "dn_weights_arch": (_I, [_P, _c.c_char_p, _I, _IP, _IP, _IP, _IP, _IP]),
    "dn_weights_meta": (_I, [_P, _CPP, _IP, _IP, _I, _IP, _IP]),
    "dn_weights_file": (_I, [_P, _c.c_char_p, _CPP]),
    "dn_weights_path": (_c.c_char_p, [_P]),
    "dn_model_create": (_I, [_c.c_char_p, _I, _PP]),
    "dn_model_destroy": (_I, [_P]),
    "dn_model_get_info": (_I, [_P, _c.POINTER(ModelInfo)]),
    "dn_model_forward": (_I, [_P, _P, _I64P, _I, _P, _P]),
    "dn_model_forward_host_async": (_I, [_P, _P, _I64P, _I, _P, _P]),
    "dn_model_host_join": (_I, [_P, _P]),
    "dn_model_forward_host": (_I, [_P, _P, _I64P, _I, _P, _P]),
    "dn_model_encode_frame": (_I, [_P, _P, _I, _I, _I, _I, _P]),
    "dn_model_decode_window": (_I, [_P, _IP, _I, _P, _I, _I, _I, _P, _P]),
    "dn_model_sync": (_I, [_P, _P]),
    "dn_model_stats": (_I, [_P, _SZP, _SZP, _IP]),
    "dn_model_set_fused": (_I, [_P, _I]),
    "dn_model_profile": (_I, [_P, _I]),
    "dn_model_profile_report": (_I, [_P, _c.c_char_p, _c.c_size_t]),
    # include/denoiser_b200_ops.h
    "dn_launch_reflect_pad": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "dn_launch_crop": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "dn_launch_subtract_clamp": (_I, [_P, _P, _P, _I64, _P]),
    "dn_launch_concat_channels": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "dn_launch_extract_frame": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "dn_launch_select_prefix_channels": (_I, [_P, _P, _I, _I, _I, _I, _I, _P]),
    "dn_launch_layer_norm_affine": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "dn_launch_simple_gate": (_I, [_P, _P, _I, _I, _I, _I, _P]),
    "dn_launch_global_avg_pool": (_I, [_P, _P, _I, _I, _I, _I, _P]),
    "dn_launch_global_avg_pool_noalloc": (_I, [_P, _P, _I, _I, _I, _I, _P]),
    "dn_launch_mul_channelwise": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "dn_launch_add": (_I, [_P, _P, _P, _I64, _P]),
    "dn_launch_mul_scalar": (_I, [_P, _F, _P, _I64, _P]),
    "dn_launch_scaled_add": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "dn_launch_pixel_shuffle2x": (_I, [_P, _P, _I, _I, _I, _I, _P]),
    "dn_launch_warp_bilinear": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "dn_upsample_bilinear": (_I, [_P, _P, _I, _I, _I, _I, _I, _P]),
    # include/denoiser_b200_layers.h
    "dn_dcn_create": (_I, [_P, _c.c_char_p, _c.c_char_p, _I, _I, _I, _I, _I, _PP]),
    "dn_dcn_destroy": (_I, [_P]),
    "dn_dcn_info": (_I, [_P, _IP, _IP, _IP, _IP, _IP]),
    "dn_dcn_output_size": (_I, [_P, _I, _I, _IP, _IP]),
    "dn_dcn_forward": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "dn_dcn_sync": (_I, [_P, _P]),
    "dn_conv2d_create": (_I, [_P, _c.c_char_p, _c.c_char_p, _I, _I, _I, _I, _I, _PP]),
    "dn_conv2d_destroy": (_I, [_P]),
    "dn_conv2d_info": (_I, [_P, _IP, _IP, _IP, _IP, _IP]),
    "dn_conv2d_output_size": (_I, [_P, _I, _I, _IP, _IP]),
    "dn_conv2d_forward": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "dn_conv2d_sync": (_I, [_P, _P]),
    # include/denoiser_b200_io.h
    "dn_image_probe": (_I, [_c.c_char_p, _IP, _IP, _IP]),
    "dn_image_read": (_I, [_c.c_char_p, _P, _I, _I, _I]),
    "dn_image_write": (_I, [_c.c_char_p, _P, _I, _I, _I]),
    # include/denoiser_b200_infer.h
    "dn_tile_extract": (_I, [_P, _P, _I64, _I, _I, _I, _I, _I, _I, _P]),
    "dn_tile_accumulate": (_I, [_P, _c.POINTER(_c.c_float), _c.POINTER(_c.c_float), _I, _I, _I, _I, _I, _I, _I, _I,
                                _P]),
    "dn_tile_normalize": (_I, [_c.POINTER(_c.c_float), _c.POINTER(_c.c_float), _P, _I, _I, _I, _P]),
    "dn_average_pair": (_I, [_P, _P, _P, _I64, _P]),
    # include/denoiser_b200_aligned.h
    "dn_aligned_create": (_I, [_c.c_char_p, _c.c_char_p, _I, _PP]),
    "dn_aligned_destroy": (_I, [_P]),
    "dn_aligned_info": (_I, [_P, _IP, _IP, _IP, _IP]),
    "dn_aligned_encode_frame": (_I, [_P, _P, _I, _I, _I, _P]),
    "dn_aligned_align_window": (_I, [_P, _IP, _I, _P, _P]),
    "dn_aligned_decode_window": (_I, [_P, _IP, _I, _P, _P]),
    "dn_aligned_forward": (_I, [_P, _P, _I, _I, _P, _P]),
    "dn_aligned_sync": (_I, [_P, _P]),
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


class Weights:
    """Host half of the reference WeightStore: parsed + validated manifest."""

    def __init__(self, manifest_path: str):
        h = ctypes.c_void_p()
        check(lib().dn_weights_open(os.fsencode(manifest_path), ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            _lib.dn_weights_close(self._h)
        self._h = None

    __del__ = close

    def __len__(self) -> int:
        return lib().dn_weights_count(self._h)

    def __contains__(self, name: str) -> bool:
        return bool(lib().dn_weights_contains(self._h, name.encode()))

    def names(self) -> list:
        out = []
        for i in range(len(self)):
            p = ctypes.c_char_p()
            check(lib().dn_weights_name(self._h, i, ctypes.byref(p)))
            out.append(p.value.decode())
        return out

    def info(self, name: str):
        """(shape tuple, dtype str) of `name`; NotFoundError if absent."""
        shape = (ctypes.c_int64 * 8)()
        nd = ctypes.c_int()
        dt = ctypes.c_int()
        check(lib().dn_weights_info(self._h, name.encode(), shape, ctypes.byref(nd), ctypes.byref(dt), None))
        return tuple(shape[i] for i in range(nd.value)), ("float16" if dt.value == 1 else "float32")

    def arch(self) -> dict:
        buf = ctypes.create_string_buffer(64)
        v = [ctypes.c_int() for _ in range(5)]
        check(lib().dn_weights_arch(self._h, buf, 64, *[ctypes.byref(x) for x in v]))
        return {"type": buf.value.decode(), "base_channels": v[0].value, "num_levels": v[1].value,
                "in_channels": v[2].value, "num_frames": v[3].value, "use_warp": bool(v[4].value)}


class Model:
    """NAFNet / NAFNetTemporal engine instance on one CUDA device.

    ``forward`` takes an fp16 CUDA tensor (N, C, H, W) (spatial) or
    (N, T, C, H, W) (temporal) and returns the (N, 3, H, W) fp16 output,
    launched on the current torch stream.
    """

    def __init__(self, manifest_path: str, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().dn_model_create(os.fsencode(manifest_path), device, ctypes.byref(h)))
        self._h = h
        self.device = device
        info = ModelInfo()
        check(lib().dn_model_get_info(self._h, ctypes.byref(info)))
        self.kind = info.kind
        self.in_channels = info.in_channels
        self.num_levels = info.num_levels
        self.base_channels = info.base_channels
        self.num_frames = info.num_frames
        self.use_warp = bool(info.use_warp)
        self.enc_channels = [info.enc_channels[i] for i in range(info.num_levels)]

    def close(self) -> None:
        if getattr(self, "_h", None) and _lib is not None:
            _lib.dn_model_destroy(self._h)
        self._h = None

    __del__ = close

    def _shape(self, x):
        shape = (ctypes.c_int64 * x.dim())(*x.shape)
        return shape, x.dim()

    def forward(self, x, out=None, stream=None):
        import torch

        if x.dtype != torch.float16:
            raise DenoiserError(DN_ERR_DTYPE, "NAFNet::forward: expected FP16 input")
        if not x.is_cuda:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG, "forward: input must be a CUDA tensor")
        x = x.contiguous()
        n = x.shape[0]
        h, w = x.shape[-2:]
        if out is None:
            out = torch.empty(n, 3, h, w, dtype=torch.float16, device=x.device)
        shape, nd = self._shape(x)
        check(lib().dn_model_forward(self._h, x.data_ptr(), shape, nd, out.data_ptr(), stream_handle(stream)))
        return out

    __call__ = forward

    def forward_host(self, x, out=None, stream=None):
        """Host (numpy fp16, ideally pinned) in and out, synchronous."""
        import numpy as np

        x = np.ascontiguousarray(x, dtype=np.float16)
        n = x.shape[0]
        h, w = x.shape[-2:]
        if out is None:
            out = np.empty((n, 3, h, w), dtype=np.float16)
        shape = (ctypes.c_int64 * x.ndim)(*x.shape)
        check(lib().dn_model_forward_host(self._h, x.ctypes.data, shape, x.ndim, out.ctypes.data,
                                          ctypes.c_void_p(stream or 0)))
        return out

    def forward_host_ptr(self, x_ptr: int, shape, y_ptr: int, stream_ptr: int = 0) -> None:
        """Host-buffer forward on raw pointers (e.g. pinned torch tensors)."""
        sh = (ctypes.c_int64 * len(shape))(*shape)
        check(lib().dn_model_forward_host(self._h, ctypes.c_void_p(x_ptr), sh, len(shape),
                                          ctypes.c_void_p(y_ptr), ctypes.c_void_p(stream_ptr)))

    def forward_host_async_ptr(self, x_ptr: int, shape, y_ptr: int, stream_ptr: int = 0) -> None:
        """Pipelined host-buffer forward (returns at once; the input copy of the
        next call and the output copy of the previous one overlap this forward).
        The result is in y after host_join(stream) and a synchronisation of it."""
        sh = (ctypes.c_int64 * len(shape))(*shape)
        check(lib().dn_model_forward_host_async(self._h, ctypes.c_void_p(x_ptr), sh, len(shape),
                                                ctypes.c_void_p(y_ptr), ctypes.c_void_p(stream_ptr)))

    def host_join(self, stream_ptr: int = 0) -> None:
        """Make the stream wait for the output copies of every queued async call."""
        check(lib().dn_model_host_join(self._h, ctypes.c_void_p(stream_ptr)))

    def encode_frame(self, frame, slot: int, stream=None) -> None:
        """Temporal models: encoder features of one (1, C, H, W) frame into cache slot `slot`."""
        _, c, h, w = frame.shape
        check(lib().dn_model_encode_frame(self._h, ctypes.c_void_p(frame.data_ptr()), c, h, w, slot,
                                          stream_handle(stream)))

    def decode_window(self, slots, beauty, out=None, stream=None):
        """Temporal models: denoise the window whose frame t is in slots[t];
        beauty = the (1, C, H, W) reference frame. Returns (1, 3, H, W)."""
        import torch

        _, c, h, w = beauty.shape
        if out is None:
            out = torch.empty(1, 3, h, w, dtype=torch.float16, device=beauty.device)
        arr = (ctypes.c_int * len(slots))(*slots)
        check(lib().dn_model_decode_window(self._h, arr, len(slots), ctypes.c_void_p(beauty.data_ptr()), c, h, w,
                                           ctypes.c_void_p(out.data_ptr()), stream_handle(stream)))
        return out

    def sync(self, stream=None) -> None:
        """Synchronise the stream and raise if a kernel flagged a device error."""
        check(lib().dn_model_sync(self._h, stream_handle(stream)))

    def set_fused(self, enable=True) -> None:
        """Fused NAFBlock kernels (True / 1, default), fused with the first pass of
        the 32/64-channel blocks on the CUDA cores instead of the tensor cores (2),
        fused with the first pass of single images as conv1 on the tensor cores
        and the depthwise conv on the CUDA cores (3), fused with the 1x1-conv
        GEMMs on CTA pairs (cta_group::2 MMAs, 4), or per-conv kernels
        (False / 0)."""
        mode = int(enable) if not isinstance(enable, bool) else (1 if enable else 0)
        check(lib().dn_model_set_fused(self._h, mode))

    def profile(self, enable: bool = True, detail: bool = False) -> None:
        """Bracket every kernel launch with CUDA events (see profile_report);
        with detail, report per kernel kind and shape ("kind@shape")."""
        check(lib().dn_model_profile(self._h, (2 if detail else 1) if enable else 0))

    def profile_report(self) -> dict:
        """{kind: {launches, ms, bytes, flops}} since the last report."""
        import json

        buf = ctypes.create_string_buffer(1 << 16)
        check(lib().dn_model_profile_report(self._h, buf, len(buf)))
        return json.loads(buf.value.decode())

    def stats(self) -> dict:
        wb = ctypes.c_size_t()
        ab = ctypes.c_size_t()
        kl = ctypes.c_int()
        check(lib().dn_model_stats(self._h, ctypes.byref(wb), ctypes.byref(ab), ctypes.byref(kl)))
        return {"weight_bytes": wb.value, "activation_bytes": ab.value, "kernels_per_forward": kl.value}
