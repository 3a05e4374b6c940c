"""Batched line-image preprocessing on the device (include/trba_preproc.h):
the pixel part of the reference's `load_image_q` (src/main.rs:218-239).

The caller decodes files to RGB8 arrays (the reference's
`image::open(path)?.to_rgb8()`); `preprocess_lines` uploads a batch of them
and returns the model input the reference builds image by image: int8
[n, img_h * img_w * 3] in [y][x][rgb] byte order, resized with the triangle
filter, on a white canvas, quantised with scale 1/127.

    batch = preprocess_lines([rgb0, rgb1, ...], img_h=32, img_w=160)  # torch int8 on cuda
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from .ffi import lib


class PackedImages:
    """Decoded RGB8 images packed for one upload: bytes, byte offsets,
    widths and heights (host arrays, pinned bytes when torch is there)."""

    def __init__(self, images: Sequence[np.ndarray]):
        import torch
        shapes = []
        for im in images:
            a = np.asarray(im)
            if a.ndim != 3 or a.shape[2] != 3 or a.dtype != np.uint8:
                raise ValueError("images must be uint8 [height, width, 3] (RGB8)")
            shapes.append(a.shape)
        sizes = [h * w * 3 for h, w, _ in shapes]
        self.offsets = np.zeros(len(images), np.int64)
        if len(images) > 1:
            self.offsets[1:] = np.cumsum(sizes[:-1])
        total = int(sum(sizes))
        self.bytes = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
        view = self.bytes.numpy()
        for im, off, n in zip(images, self.offsets, sizes):
            view[off:off + n] = np.ascontiguousarray(im).reshape(-1)
        self.heights = np.array([s[0] for s in shapes], np.int32)
        self.widths = np.array([s[1] for s in shapes], np.int32)

    @property
    def nbytes(self) -> int:
        return int(self.bytes.numel())


class DeviceBatch:
    """A PackedImages batch resident on the GPU."""

    def __init__(self, packed: PackedImages, device="cuda", stream=None):
        import torch
        nb = {"non_blocking": True}
        self.rgb = packed.bytes.to(device, **nb)
        self.offsets = torch.from_numpy(packed.offsets).to(device, **nb)
        self.widths = torch.from_numpy(packed.widths).to(device, **nb)
        self.heights = torch.from_numpy(packed.heights).to(device, **nb)
        self.n = len(packed.widths)


def preprocess_device(batch: DeviceBatch, img_h: int, img_w: int, out=None, stream=None):
    """Runs trba_preprocess_lines on a resident batch; returns (or fills) a
    torch int8 tensor [n, img_h * img_w * 3] on the batch's device."""
    import torch
    if out is None:
        out = torch.empty((batch.n, img_h * img_w * 3), dtype=torch.int8, device=batch.rgb.device)
    L = lib()
    st = C.c_void_p(stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream)
    rc = L.trba_preprocess_lines(C.c_void_p(batch.rgb.data_ptr()), C.c_void_p(batch.offsets.data_ptr()),
                                 C.c_void_p(batch.widths.data_ptr()), C.c_void_p(batch.heights.data_ptr()),
                                 batch.n, img_h, img_w, C.c_void_p(out.data_ptr()), st)
    if rc != 0:
        raise RuntimeError("trba_preprocess_lines: " + L.trba_last_error_string().decode())
    return out


def preprocess_lines(images: Sequence[np.ndarray], img_h: int, img_w: int, device="cuda", stream=None):
    """load_image_q for a batch of decoded RGB8 images, on the GPU."""
    return preprocess_device(DeviceBatch(PackedImages(images), device, stream), img_h, img_w, stream=stream)
