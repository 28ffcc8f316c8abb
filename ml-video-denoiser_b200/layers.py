"""Stand-alone layers of the reference's include/denoiser/layers/ on torch
CUDA tensors (FP16, NCHW), over include/denoiser_b200_layers.h."""
from __future__ import annotations

import ctypes

from . import Weights, check, lib, stream_handle


class DeformConv2d:
    """DeformConv2dLayer (include/denoiser/layers/deform_conv2d.h:11-55):
    modulated deformable convolution with weights from a WeightStore."""

    def __init__(self, store: Weights, weight_name: str, bias_name: str | None, pad: int = 1, stride: int = 1,
                 dilation: int = 1, deform_groups: int = 8, device: int = 0):
        self._h = ctypes.c_void_p()
        check(lib().dn_dcn_create(store._h, weight_name.encode(), bias_name.encode() if bias_name else None, pad,
                                  stride, dilation, deform_groups, device, ctypes.byref(self._h)))
        vals = [ctypes.c_int() for _ in range(5)]
        check(lib().dn_dcn_info(self._h, *[ctypes.byref(v) for v in vals]))
        self.out_channels, self.in_channels, self.deform_groups, self.kernel_h, self.kernel_w = (v.value for v in vals)
        self.device = device

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h:
            lib().dn_dcn_destroy(h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def output_size(self, h: int, w: int):
        ho, wo = ctypes.c_int(), ctypes.c_int()
        check(lib().dn_dcn_output_size(self._h, h, w, ctypes.byref(ho), ctypes.byref(wo)))
        return ho.value, wo.value

    def forward(self, x, offsets, masks, out=None, stream=None):
        """x (N, Cin, H, W), offsets (N, 2*dg*kh*kw, Ho, Wo), masks (N, dg*kh*kw, Ho, Wo) -> (N, Cout, Ho, Wo)."""
        import torch

        for t in (x, offsets, masks):
            if t.dtype != torch.float16:
                raise TypeError("DeformConv2dLayer::forward: all inputs must be FP16")
        n, _, h, w = x.shape
        ho, wo = self.output_size(h, w)
        if out is None:
            out = torch.empty(n, self.out_channels, ho, wo, dtype=torch.float16, device=x.device)
        check(lib().dn_dcn_forward(self._h, x.data_ptr(), offsets.data_ptr(), masks.data_ptr(), n, h, w,
                                   out.data_ptr(), stream_handle(stream)))
        return out

    __call__ = forward

    def sync(self, stream=None) -> None:
        check(lib().dn_dcn_sync(self._h, stream_handle(stream)))


class Conv2d:
    """Conv2dLayer (include/denoiser/layers/conv2d.h:44-63): regular convolution
    with weights (and optional bias) from a WeightStore."""

    def __init__(self, store: Weights, weight_name: str, bias_name: str | None = None, pad: int = 1,
                 stride: int = 1, dilation: int = 1, groups: int = 1, device: int = 0):
        self._h = ctypes.c_void_p()
        check(lib().dn_conv2d_create(store._h, weight_name.encode(), bias_name.encode() if bias_name else None, pad,
                                     stride, dilation, groups, device, ctypes.byref(self._h)))
        vals = [ctypes.c_int() for _ in range(5)]
        check(lib().dn_conv2d_info(self._h, *[ctypes.byref(v) for v in vals]))
        self.out_channels, self.in_channels, self.kernel_h, self.kernel_w, self.groups = (v.value for v in vals)
        self.device = device

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h:
            lib().dn_conv2d_destroy(h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def output_size(self, h: int, w: int):
        ho, wo = ctypes.c_int(), ctypes.c_int()
        check(lib().dn_conv2d_output_size(self._h, h, w, ctypes.byref(ho), ctypes.byref(wo)))
        return ho.value, wo.value

    def forward(self, x, out=None, stream=None):
        """x (N, in_channels*groups, H, W) FP16 -> (N, out_channels, Ho, Wo) FP16."""
        import torch

        if x.dtype != torch.float16:
            raise TypeError("Conv2dLayer::forward: expected FP16 input")
        n, c, h, w = x.shape
        ho, wo = self.output_size(h, w)
        if out is None:
            out = torch.empty(n, self.out_channels, ho, wo, dtype=torch.float16, device=x.device)
        check(lib().dn_conv2d_forward(self._h, x.data_ptr(), n, c, h, w, out.data_ptr(), stream_handle(stream)))
        return out

    __call__ = forward

    def sync(self, stream=None) -> None:
        check(lib().dn_conv2d_sync(self._h, stream_handle(stream)))
