"""The reference's NCHW kernel launchers, ``denoiser::kernels::launch_*``.

Same names, argument order and meaning as include/denoiser/kernels/
model_kernels.h:22-59 and nafnet_kernels.h:9-95 of the reference, on torch
CUDA tensors (FP16, contiguous NCHW) instead of raw ``__half*``. Each call
enqueues one B200 kernel (two for the average pool) of
``libdenoiser_b200.so`` on ``stream`` (default: torch's current stream) and
returns without synchronising. Bad arguments raise ``InvalidArgumentError``
(the C-ABI's DN_ERR_INVALID_ARG) instead of reading out of bounds.
"""
from __future__ import annotations

from . import check, lib, stream_handle


def _p(t) -> int:
    return 0 if t is None else t.data_ptr()


def _s(stream) -> int:
    return stream_handle(stream)


def launch_reflect_pad(input, output, N, C, H_in, W_in, H_out, W_out, stream=None):
    check(lib().dn_launch_reflect_pad(_p(input), _p(output), N, C, H_in, W_in, H_out, W_out, _s(stream)))


def launch_crop(input, output, N, C, H_in, W_in, H_out, W_out, stream=None):
    check(lib().dn_launch_crop(_p(input), _p(output), N, C, H_in, W_in, H_out, W_out, _s(stream)))


def launch_subtract_clamp(a, b, out, n, stream=None):
    check(lib().dn_launch_subtract_clamp(_p(a), _p(b), _p(out), n, _s(stream)))


def launch_concat_channels(a, b, output, N, C1, C2, H, W, stream=None):
    check(lib().dn_launch_concat_channels(_p(a), _p(b), _p(output), N, C1, C2, H, W, _s(stream)))


def launch_extract_frame(clip, frame, N, T, C, H, W, frame_idx, stream=None):
    check(lib().dn_launch_extract_frame(_p(clip), _p(frame), N, T, C, H, W, frame_idx, _s(stream)))


def launch_select_prefix_channels(input, output, N, C_in, C_out, H, W, stream=None):
    check(lib().dn_launch_select_prefix_channels(_p(input), _p(output), N, C_in, C_out, H, W, _s(stream)))


def launch_layer_norm_affine(input, weight, bias, params_fp32, output, N, C, H, W, stream=None):
    check(lib().dn_launch_layer_norm_affine(_p(input), _p(weight), _p(bias), int(bool(params_fp32)), _p(output),
                                            N, C, H, W, _s(stream)))


def launch_simple_gate(input, output, N, C, H, W, stream=None):
    check(lib().dn_launch_simple_gate(_p(input), _p(output), N, C, H, W, _s(stream)))


def launch_global_avg_pool(input, output, N, C, H, W, stream=None):
    check(lib().dn_launch_global_avg_pool(_p(input), _p(output), N, C, H, W, _s(stream)))


def launch_mul_channelwise(input, scale, output, N, C, H, W, stream=None):
    check(lib().dn_launch_mul_channelwise(_p(input), _p(scale), _p(output), N, C, H, W, _s(stream)))


def launch_add(a, b, out, n, stream=None):
    check(lib().dn_launch_add(_p(a), _p(b), _p(out), n, _s(stream)))


def launch_mul_scalar(input, scalar, output, n, stream=None):
    check(lib().dn_launch_mul_scalar(_p(input), float(scalar), _p(output), n, _s(stream)))


def launch_scaled_add(identity, residual, scale, scale_fp32, output, N, C, H, W, stream=None):
    check(lib().dn_launch_scaled_add(_p(identity), _p(residual), _p(scale), int(bool(scale_fp32)), _p(output),
                                     N, C, H, W, _s(stream)))


def launch_pixel_shuffle2x(input, output, N, C_in, H, W, stream=None):
    check(lib().dn_launch_pixel_shuffle2x(_p(input), _p(output), N, C_in, H, W, _s(stream)))


def upsample_bilinear(input, output, N, C, H, W, scale_factor=2, stream=None):
    """UpsampleLayer::forward on an existing output buffer (N, C, H*s, W*s)."""
    check(lib().dn_upsample_bilinear(_p(input), _p(output), N, C, H, W, scale_factor, _s(stream)))


def launch_warp_bilinear(feat, offset, output, N, C, H, W, stream=None):
    check(lib().dn_launch_warp_bilinear(_p(feat), _p(offset), _p(output), N, C, H, W, _s(stream)))
