"""Temporal NAFNet with deformable alignment, composed from the engine's
layers over the C-ABI (FP16, NCHW, one window of T frames per call):

    f_t   = feat(frame_t)                           3x3 conv, in -> F
    om_t  = offset(concat(f_c, f_t))                3x3 conv, 2F -> 3*dg*9
    a_t   = dcn(f_t, om_t[:2*dg*9], om_t[2*dg*9:])  DCNv2 3x3, F -> F (sigmoid masks)
    a_c   = f_c
    fused = fuse(concat(a_0 .. a_{T-1})) + frame_c  1x1 conv, T*F -> in
    out   = NAFNet(fused)                           the spatial engine

c = T // 2 is the centre frame. The reference has DeformConv2dLayer
(src/layers/deform_conv2d.cu:105-184) but wires it into no model; this class
fixes one wiring so that the layer runs inside a whole network. Every step is
an engine kernel: Conv2dLayer (implicit GEMM on tcgen05), DeformConv2dLayer
(fused sampling + tcgen05), extract_frame / add launchers and the NAFNet
engine. Each layer writes straight into its slice of the concatenation
buffers (channel slices of a batch-1 NCHW tensor are contiguous).

Weights: manifest keys ``align.{feat,offset,dcn,fuse}.{weight,bias}`` in the
reference format (``manifest.json`` + ``.bin``), architecture ``num_frames``
= T; the trunk is a separate NAFNet manifest.

Size limit: the fusion conv reads the T*F-channel concatenation, and a
Conv2dLayer input holds at most 2^31 elements, so T*F*H*W <= 2^31 (T = 5,
F = 64: frames up to about 6.7 M pixels, e.g. 1080p but not 2160x3840).
Larger frames are rejected before any kernel is launched.
"""
from __future__ import annotations

from . import DN_ERR_INVALID_ARG, InvalidArgumentError, Model, Weights
from .kernels import launch_add, launch_extract_frame
from .layers import Conv2d, DeformConv2d

MAX_LAYER_ELEMS = 1 << 31  # Conv2dLayer input limit (dn_conv2d_forward)


class AlignedTemporal:
    def __init__(self, align_manifest: str, trunk_manifest: str, device: int = 0):
        self.store = Weights(align_manifest)
        self.num_frames = int(self.store.arch()["num_frames"])
        self.feat = Conv2d(self.store, "align.feat.weight", "align.feat.bias", pad=1, device=device)
        self.offset = Conv2d(self.store, "align.offset.weight", "align.offset.bias", pad=1, device=device)
        n_om = self.offset.out_channels
        self.deform_groups = n_om // 27
        self.n_off = 2 * self.deform_groups * 9
        self.dcn = DeformConv2d(self.store, "align.dcn.weight", "align.dcn.bias", pad=1,
                                deform_groups=self.deform_groups, device=device)
        self.fuse = Conv2d(self.store, "align.fuse.weight", "align.fuse.bias", pad=0, device=device)
        self.trunk = Model(trunk_manifest, device)
        f = self.feat.out_channels
        self.in_channels = self.feat.in_channels
        self.feat_channels = f
        if (n_om % 27 or self.offset.in_channels != 2 * f or self.dcn.in_channels != f or self.dcn.out_channels != f
                or self.fuse.in_channels != self.num_frames * f or self.fuse.out_channels != self.in_channels
                or self.trunk.in_channels != self.in_channels or self.num_frames < 1):
            raise InvalidArgumentError(DN_ERR_INVALID_ARG, "AlignedTemporal: inconsistent alignment / trunk shapes")
        self.device = device

    def forward(self, clip, out=None, stream=None):
        """clip (1, T, C, H, W) FP16 CUDA -> (1, 3, H, W) FP16, on ``stream``
        (default: the current torch stream)."""
        import torch

        if clip.dtype != torch.float16:
            raise TypeError("AlignedTemporal::forward: expected FP16 input")
        if clip.dim() != 5 or clip.shape[0] != 1 or clip.shape[1] != self.num_frames \
                or clip.shape[2] != self.in_channels:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG,
                                       f"AlignedTemporal: expected (1, {self.num_frames}, {self.in_channels}, H, W)")
        t, cin, h, w = clip.shape[1:]
        f, c = self.feat_channels, t // 2
        if t * f * h * w > MAX_LAYER_ELEMS:
            raise InvalidArgumentError(DN_ERR_INVALID_ARG,
                                       f"AlignedTemporal: {t}x{f}x{h}x{w} fusion input exceeds 2^31 elements")
        dev = clip.device
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        # Temporaries come from the launch stream's pool, so their reuse after
        # this call is ordered behind the kernels that use them.
        with torch.cuda.stream(s):
            clip = clip.contiguous()
            e = lambda *shape: torch.empty(*shape, dtype=torch.float16, device=dev)  # noqa: E731
            frame = e(1, cin, h, w)
            centre = e(1, cin, h, w)
            pair = e(1, 2 * f, h, w)          # [f_c | f_t]: the offset conv's input
            om = e(1, self.offset.out_channels, h, w)
            cat = e(1, t * f, h, w)           # [a_0 | ... | a_{T-1}]: the fusion conv's input
            fused = e(1, cin, h, w)
            launch_extract_frame(clip, centre, 1, t, cin, h, w, c, s)
            self.feat(centre, out=pair[:, :f], stream=s)
            self.feat(centre, out=cat[:, c * f:(c + 1) * f], stream=s)
            for i in range(t):
                if i == c:
                    continue
                launch_extract_frame(clip, frame, 1, t, cin, h, w, i, s)
                self.feat(frame, out=pair[:, f:], stream=s)
                self.offset(pair, out=om, stream=s)
                self.dcn(pair[:, f:], om[:, :self.n_off], om[:, self.n_off:], out=cat[:, i * f:(i + 1) * f],
                         stream=s)
            self.fuse(cat, out=fused, stream=s)
            launch_add(fused, centre, fused, fused.numel(), s)
            return self.trunk(fused, out=out, stream=s)

    __call__ = forward

    def sync(self, stream=None) -> None:
        self.trunk.sync(stream)

    def close(self) -> None:
        for m in (self.feat, self.offset, self.dcn, self.fuse, self.trunk, self.store):
            m.close()
