"""Model-level host mirror of the reference's VAE backend seam.

``NativeModel`` mirrors the reference's ``NativeModel`` VAE entry points as a
``ModelBackend`` (src/pipeline.rs:54-68, src/native.rs:448-533):
``encode_moments(image, checkpoint)`` and ``decode(latents, checkpoint)`` on
NCHW float32 CUDA tensors, returning newly allocated NCHW float32 tensors. The
weights live in an opaque C-ABI handle built once from a diffusers-named state
dict (``osor_vae_create``). ``CancellationToken`` mirrors the reference's
token (src/pipeline.rs:20-47): it is polled between blocks by the library.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Iterable, Optional

import numpy as np
import torch

from . import _lib
from ._lib import InvalidInput, check, dtype_code
from .weights import SDXL_CHANNELS, SDXL_LAYERS

MAX_BATCH = 4
MIN_IMAGE_AXIS = 32
MAX_IMAGE_AXIS = 1024
IMAGE_AXIS_MULTIPLE = 8


class CancellationToken:
    """A host flag the library polls between VAE blocks."""

    def __init__(self):
        self._flag = ctypes.c_int(0)

    def cancel(self) -> None:
        self._flag.value = 1

    def is_cancelled(self) -> bool:
        return self._flag.value != 0

    @property
    def pointer(self):
        return ctypes.byref(self._flag)


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class NativeModel:
    """Random-init or loaded SDXL VAE on one CUDA device.

    ``dtype`` is the model's 16-bit type for weights and activations:
    ``"f16"`` (default; three more mantissa bits) or ``"bf16"`` (the f32
    exponent range). The reference's CUDA backend accepts both
    (src/runtime.rs:406-417)."""

    def __init__(self, weights: Dict[str, np.ndarray], device: int = 0,
                 channels: Iterable[int] = SDXL_CHANNELS, layers: int = SDXL_LAYERS,
                 parts=("decoder", "encoder"), dtype: str = "f16"):
        self.device = torch.device("cuda", device)
        self.dtype = dtype
        self.channels = tuple(channels)
        self.layers = int(layers)
        names, arrays = [], []
        for name, arr in weights.items():
            a = np.ascontiguousarray(np.asarray(arr, np.float32))
            names.append(name.encode())
            arrays.append(a)
        table = (_lib.OsorTensor * len(arrays))()
        for i, (n, a) in enumerate(zip(names, arrays)):
            table[i].name = n
            table[i].data = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            table[i].ndim = a.ndim
            for d in range(4):
                table[i].shape[d] = a.shape[d] if d < a.ndim else 0
        cfg = _lib.OsorVaeConfig()
        for i, c in enumerate(self.channels):
            cfg.channels[i] = c
        cfg.layers = self.layers
        cfg.parts = ((_lib.PART_DECODER if "decoder" in parts else 0)
                     | (_lib.PART_ENCODER if "encoder" in parts else 0))
        cfg.dtype = dtype_code(dtype)
        if cfg.dtype == _lib.DTYPE_F32:
            raise InvalidInput("model dtype must be bf16 or f16")
        handle = ctypes.c_void_p()
        check(_lib.lib().osor_vae_create(table, len(arrays), ctypes.byref(cfg), device,
                                         ctypes.byref(handle)))
        self._handle = handle
        self._workspace: Dict[tuple, torch.Tensor] = {}

    @classmethod
    def from_safetensors(cls, path: str, device: int = 0, parts=("decoder", "encoder"),
                         dtype: str = "f16", limits=None, **kwargs) -> "NativeModel":
        """Load `vae.safetensors` (diffusers names) with the reference's file
        checks (``artifact.read_safetensors``) and build the model."""
        from .artifact import read_safetensors
        return cls(read_safetensors(path, limits), device=device, parts=parts, dtype=dtype,
                   **kwargs)

    def close(self) -> None:
        if getattr(self, "_handle", None):
            _lib.lib().osor_vae_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def workspace_bytes(self, op: int, batch: int, height: int, width: int) -> int:
        return int(_lib.lib().osor_vae_workspace_size(self._handle, op, batch, height, width))

    def _workspace_for(self, op, batch, height, width) -> torch.Tensor:
        need = self.workspace_bytes(op, batch, height, width)
        if need == 0:
            raise InvalidInput("shape is outside the VAE admission limits")
        ws = self._workspace.get((op,))
        if ws is None or ws.numel() < need:
            self._workspace.pop((op,), None)
            ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._workspace[(op,)] = ws
        return ws

    def _check(self, x: torch.Tensor, what: str, channels: int) -> None:
        if not x.is_cuda or x.device != self.device:
            raise InvalidInput(f"{what} must live on {self.device}")
        if x.dtype != torch.float32 or x.ndim != 4 or x.shape[1] != channels:
            raise InvalidInput(f"{what} must be float32 [B, {channels}, H, W]")
        if not x.is_contiguous():
            raise InvalidInput(f"{what} must be contiguous")

    def decode(self, latents: torch.Tensor, checkpoint: Optional[CancellationToken] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Unscaled latents [B, 4, h, w] -> raw RGB [B, 3, 8h, 8w] (vae_decoder.rs:104-114)."""
        self._check(latents, "latents", 4)
        b, _, h, w = latents.shape
        ws = self._workspace_for(_lib.OP_DECODE, b, h, w)
        if out is None:
            out = torch.empty((b, 3, 8 * h, 8 * w), dtype=torch.float32, device=self.device)
        check(_lib.lib().osor_vae_decode(self._handle, latents.data_ptr(), out.data_ptr(), b, h,
                                         w, ws.data_ptr(), ws.numel(), _stream(self.device),
                                         checkpoint.pointer if checkpoint else None))
        return out

    def encode_moments(self, image: torch.Tensor,
                       checkpoint: Optional[CancellationToken] = None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Normalized image [B, 3, H, W] -> moments [B, 8, H/8, W/8] (vae_encoder.rs:414-424)."""
        self._check(image, "image", 3)
        b, _, h, w = image.shape
        ws = self._workspace_for(_lib.OP_ENCODE, b, h, w)
        if out is None:
            out = torch.empty((b, 8, h // 8, w // 8), dtype=torch.float32, device=self.device)
        check(_lib.lib().osor_vae_encode_moments(self._handle, image.data_ptr(), out.data_ptr(),
                                                 b, h, w, ws.data_ptr(), ws.numel(),
                                                 _stream(self.device),
                                                 checkpoint.pointer if checkpoint else None))
        return out


def device_status(device: int = 0, reset: bool = True) -> int:
    """Synchronise and read (and clear) the library's device-side status word."""
    return int(_lib.lib().osor_device_status(device, 1 if reset else 0))
