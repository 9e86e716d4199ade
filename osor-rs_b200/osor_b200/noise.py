"""Seeded noise: host mirror of the reference's `seeded_noise`
(src/noise.rs:107-146) over the C ABI (`osor_seeded_noise`).

Stream 0 fills the VAE posterior noise and stream 1 the diffusion noise, each
`[B, 4, H/8, W/8]` standard-normal values of the reference's stored-seed
contract version 1, generated on the GPU.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch

from . import _lib
from ._lib import InvalidInput, check, dtype_code

NOISE_VERSION = 1


class Noise(NamedTuple):
    posterior: torch.Tensor
    diffusion: torch.Tensor


def seeded_noise(seed: int, batch: int, height: int, width: int, dtype=torch.float32,
                 device="cuda") -> Noise:
    """Both noise tensors for a [batch, 3, height, width] job (noise.rs:107-146).
    ``batch`` in 1..4; ``height``/``width`` multiples of 8 in 32..1024;
    ``dtype`` float32, float16 or bfloat16."""
    if dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise InvalidInput("seeded noise dtype must be F32, F16, or BF16")
    ok = lambda a: 32 <= a <= 1024 and a % 8 == 0  # noqa: E731
    if not (1 <= batch <= 4) or not ok(height) or not ok(width):
        raise InvalidInput("seeded noise needs batch 1..=4 and image axes that the model admits")
    device = torch.device(device)
    if device.type != "cuda":
        raise InvalidInput("seeded noise is generated on a CUDA device")
    shape = (batch, 4, height // 8, width // 8)
    posterior = torch.empty(shape, dtype=dtype, device=device)
    diffusion = torch.empty(shape, dtype=dtype, device=device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    check(_lib.lib().osor_seeded_noise(int(seed) & (2 ** 64 - 1), batch, height, width,
                                       dtype_code(dtype), ctypes.c_void_p(posterior.data_ptr()),
                                       ctypes.c_void_p(diffusion.data_ptr()), stream))
    return Noise(posterior, diffusion)
