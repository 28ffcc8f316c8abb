"""Temporal NAFNet with deformable alignment on torch CUDA tensors (FP16,
batch 1, 3-channel frames), over include/denoiser_b200_aligned.h:

    f_t   = feat(frame_t)                           3x3 conv, 3 -> F
    om_t  = offset(concat(f_c, f_t))                3x3 conv, 2F -> 3*dg*9
    a_t   = dcn(f_t, om_t[:2*dg*9], om_t[2*dg*9:])  DCNv2 3x3, F -> F (sigmoid masks)
    a_c   = f_c
    fused = fuse(concat(a_0 .. a_{T-1})) + frame_c  1x1 conv, T*F -> 3
    out   = NAFNet(fused)                           the spatial engine

c = T // 2 is the centre frame. The reference has DeformConv2dLayer
(src/layers/deform_conv2d.cu:105-184) but wires it into no model; this class
fixes one wiring so that the layer runs inside a whole network.

The engine computes each frame's share once: encode_frame stores a frame,
its features and the neighbour half of the offset conv in a cache slot;
decode_window runs the centre half of the offset conv, the deformable convs
(with the 1x1 fusion in their epilogue) and the trunk. A sequence therefore
encodes every frame once (frame f in slot f % T), as ``sharding`` does.

Weights: manifest keys ``align.{feat,offset,dcn,fuse}.{weight,bias}`` in the
reference format (``manifest.json`` + ``.bin``), architecture ``num_frames``
= T; the trunk is a separate NAFNet manifest.
"""
from __future__ import annotations

import ctypes

from . import DN_ERR_INVALID_ARG, InvalidArgumentError, check, lib, stream_handle


class AlignedTemporal:
    def __init__(self, align_manifest: str, trunk_manifest: str, device: int = 0):
        self._h = ctypes.c_void_p()
        check(lib().dn_aligned_create(align_manifest.encode(), trunk_manifest.encode(), device, ctypes.byref(self._h)))
        vals = [ctypes.c_int() for _ in range(4)]
        check(lib().dn_aligned_info(self._h, *[ctypes.byref(v) for v in vals]))
        self.num_frames, self.in_channels, self.feat_channels, self.deform_groups = (v.value for v in vals)
        self.device = device

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h:
            lib().dn_aligned_destroy(h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _stream(stream):
        import torch

        return stream_handle(stream if stream is not None else torch.cuda.current_stream())

    def encode_frame(self, frame, slot: int, stream=None) -> None:
        """Frame (1, 3, H, W) FP16 CUDA into cache slot `slot` in [0, T)."""
        if frame.dim() != 4 or frame.shape[0] != 1 or frame.shape[1] != self.in_channels:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG, "AlignedTemporal.encode_frame: expected (1, 3, H, W)")
        frame = frame.contiguous()
        check(lib().dn_aligned_encode_frame(self._h, ctypes.c_void_p(frame.data_ptr()), frame.shape[2],
                                            frame.shape[3], slot, self._stream(stream)))

    def _slots(self, slots):
        if len(slots) != self.num_frames:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG, f"AlignedTemporal: {self.num_frames} slots expected")
        return (ctypes.c_int * len(slots))(*slots)

    def align_window(self, slots, h: int, w: int, out=None, stream=None):
        """The alignment stage alone: the trunk input (1, 3, H, W) of the window."""
        import torch

        if out is None:
            out = torch.empty(1, 3, h, w, dtype=torch.float16, device=f"cuda:{self.device}")
        check(lib().dn_aligned_align_window(self._h, self._slots(slots), len(slots), ctypes.c_void_p(out.data_ptr()),
                                            self._stream(stream)))
        return out

    def decode_window(self, slots, beauty=None, out=None, stream=None):
        """Denoise the window whose frame t sits in slots[t] -> (1, 3, H, W).
        `beauty` (the window's centre frame) only gives the size: the model
        keeps the centre frame in its slot."""
        import torch

        if beauty is None:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG, "AlignedTemporal.decode_window: frame size needed")
        h, w = beauty.shape[-2:]
        if out is None:
            out = torch.empty(1, 3, h, w, dtype=torch.float16, device=beauty.device)
        check(lib().dn_aligned_decode_window(self._h, self._slots(slots), len(slots), ctypes.c_void_p(out.data_ptr()),
                                             self._stream(stream)))
        return out

    def forward(self, clip, out=None, stream=None):
        """clip (1, T, 3, H, W) FP16 CUDA -> (1, 3, H, W) FP16, on ``stream``
        (default: the current torch stream)."""
        import torch

        if clip.dtype != torch.float16:
            raise TypeError("AlignedTemporal::forward: expected FP16 input")
        if clip.dim() != 5 or clip.shape[0] != 1 or clip.shape[1] != self.num_frames \
                or clip.shape[2] != self.in_channels:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG,
                                       f"AlignedTemporal: expected (1, {self.num_frames}, {self.in_channels}, H, W)")
        clip = clip.contiguous()
        h, w = clip.shape[-2:]
        if out is None:
            out = torch.empty(1, 3, h, w, dtype=torch.float16, device=clip.device)
        check(lib().dn_aligned_forward(self._h, ctypes.c_void_p(clip.data_ptr()), h, w, ctypes.c_void_p(out.data_ptr()),
                                       self._stream(stream)))
        return out

    __call__ = forward

    def sync(self, stream=None) -> None:
        check(lib().dn_aligned_sync(self._h, self._stream(stream)))
