"""16-bit precision emulation of the decoder (TEST INFRASTRUCTURE ONLY).

Runs the oracle's decoder with the convolution and projection weights and
every activation the CUDA decoder stores between kernels rounded to a 16-bit
type (bf16 or f16, round to nearest even), everything else in F32: the
accumulators, the GroupNorm statistics, softmax, the f32 post_quant_conv and
the f32 image. It measures how far a decoder that stores 16-bit activations
can be from the F32 oracle on a given model, independently of any kernel: the
format's floor. The reference's own CUDA backend with a BF16 model stores its
activations the same way (Candle ops in the model dtype,
src/runtime.rs:406-417).
"""
from __future__ import annotations

import numpy as np
import torch

from . import vae


def rounder(dtype: str):
    """x -> x rounded to bf16 / f16 and back to f32."""
    t = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]

    def q(x):
        return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(t).float().numpy()
    return q


def rounded_weights(w, dtype: str):
    """Conv / linear weights rounded; biases, GroupNorm affine and the f32
    post_quant_conv kept."""
    q = rounder(dtype)
    out = {}
    for name, v in w.items():
        keep = (not name.endswith(".weight") or v.ndim < 2 or name.startswith("post_quant_conv"))
        out[name] = v if keep else q(v)
    return out


def decode(w, latents, dtype: str, observer=None):
    """The oracle decoder with 16-bit weights and stored activations."""
    return vae.decode(rounded_weights(w, dtype), latents, observer=observer, q=rounder(dtype))
