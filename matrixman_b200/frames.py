"""Frame preprocessing on the device.

The reference prepares every video frame on the CPU (``demo/yolo_helpers.py:53-56``):
``cv2.resize`` with INTER_LINEAR to the model size, BGR -> RGB, CHW, float32
divided by 255, and then uploads the float tensor.  ``preprocess_frames``
uploads the uint8 frames instead (a quarter of the bytes of a float frame of the
same size) and does the rest in one kernel whose resize is OpenCV's 8-bit
bilinear fixed-point algorithm, so the result equals the reference's bit for
bit.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib, ops, runtime
from .tensor import MatrixManTensor


def preprocess_frames(frames, image_size, device=None) -> MatrixManTensor:
    """uint8 BGR frame(s) ``[H, W, 3]`` or ``[N, H, W, 3]`` (NumPy array or CPU
    tensor) -> ``[N, 3, S, S]`` float32 RGB / 255 on the device, equal to
    ``torch.cat([preprocess_frame(f, S) for f in frames])`` of the reference.
    ``image_size`` is S or ``(height, width)``."""
    from .api import _device_index, get_backend

    get_backend()
    if isinstance(frames, np.ndarray):
        frames = torch.from_numpy(np.ascontiguousarray(frames))
    if not isinstance(frames, torch.Tensor) or frames.device.type != "cpu":
        raise TypeError("MatrixMan: preprocess_frames expects CPU uint8 frames")
    if frames.dtype != torch.uint8:
        raise TypeError("MatrixMan: preprocess_frames expects uint8 frames")
    if frames.dim() == 3:
        frames = frames.unsqueeze(0)
    if frames.dim() != 4 or frames.shape[3] != 3 or frames.shape[1] == 0 or frames.shape[2] == 0:
        raise ValueError("MatrixMan: frames must be [H, W, 3] or [N, H, W, 3] BGR")
    oh, ow = (image_size, image_size) if isinstance(image_size, int) else tuple(int(v) for v in image_size)
    if oh <= 0 or ow <= 0:
        raise ValueError("MatrixMan: image_size must be positive")
    frames = frames.contiguous()
    n, h, w, _ = (int(v) for v in frames.shape)
    rt = runtime.get_runtime(_device_index(device))
    runtime.set_device(rt.index)
    out = ops.empty(rt, (n, 3, oh, ow))
    if n == 0:
        return out
    raw = rt.new_storage(frames.numel(), torch.uint8)
    flag = ctypes.c_int(0)
    rt.lib.mm_host_is_pinned(ctypes.c_void_p(frames.data_ptr()), ctypes.byref(flag))
    pinned = bool(flag.value)
    _lib.check(rt.lib.mm_memcpy_h2d(ctypes.c_void_p(raw.pointer), ctypes.c_void_p(frames.data_ptr()),
                                    frames.numel(), rt.stream, 0 if pinned else 1),
               "host-to-device copy")
    ops._launch("mm_preprocess_bgr8", ctypes.c_void_p(raw.pointer), n, h, w, ops._p(out.desc()),
                rt.stream)
    if pinned:
        # A page-locked source is read asynchronously: the frames stay alive
        # with the result.  (A pageable one was staged before the call returned;
        # the uint8 block is then released stream-ordered after the kernel.)
        out._owner.keepalive = (raw, frames)
    return out
