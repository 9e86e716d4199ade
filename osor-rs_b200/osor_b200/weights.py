"""Deterministic random-init SDXL AutoencoderKL weights with diffusers names.

The reference builds random-init models through Candle's ``VarMap`` init hints
(src/native/conv.rs:160-173: Kaiming-normal weights, std sqrt(2/fan_in), and
U(-1/sqrt(Cin), 1/sqrt(Cin)) biases; src/native/vae_encoder.rs:49-50: GroupNorm
weight 1, bias 0; candle-nn ``linear`` uses the same weight/bias hints for the
attention projections). Candle's RNG stream cannot be reproduced outside Rust,
so this module draws the same distributions from numpy's PCG64 with a fixed
seed, in a fixed name order. Names follow the reference's loaders
(src/native/vae_encoder.rs:224-260,388-412; src/native/vae_decoder.rs:62-101).
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Tuple

import numpy as np

SDXL_CHANNELS = (128, 256, 512, 512)
SDXL_LAYERS = 2

Spec = Tuple[str, Tuple[int, ...], str]


def _conv(prefix: str, cin: int, cout: int, k: int) -> List[Spec]:
    return [(prefix + ".weight", (cout, cin, k, k), "kaiming"),
            (prefix + ".bias", (cout,), "bias")]


def _norm(prefix: str, c: int) -> List[Spec]:
    return [(prefix + ".weight", (c,), "one"), (prefix + ".bias", (c,), "zero")]


def _linear(prefix: str, c: int) -> List[Spec]:
    return [(prefix + ".weight", (c, c), "kaiming"), (prefix + ".bias", (c,), "bias")]


def _resnet(prefix: str, cin: int, cout: int) -> List[Spec]:
    s = _norm(prefix + ".norm1", cin) + _conv(prefix + ".conv1", cin, cout, 3)
    s += _norm(prefix + ".norm2", cout) + _conv(prefix + ".conv2", cout, cout, 3)
    if cin != cout:
        s += _conv(prefix + ".conv_shortcut", cin, cout, 1)
    return s


def _mid(prefix: str, c: int) -> List[Spec]:
    a = prefix + ".attentions.0"
    s = _resnet(prefix + ".resnets.0", c, c)
    s += _norm(a + ".group_norm", c)
    for name in ("to_q", "to_k", "to_v", "to_out.0"):
        s += _linear(a + "." + name, c)
    s += _resnet(prefix + ".resnets.1", c, c)
    return s


def decoder_specs(channels=SDXL_CHANNELS, layers=SDXL_LAYERS) -> List[Spec]:
    rev = list(reversed(channels))
    last = rev[0]
    s = _conv("post_quant_conv", 4, 4, 1)
    s += _conv("decoder.conv_in", 4, last, 3)
    s += _mid("decoder.mid_block", last)
    for i, out in enumerate(rev):
        cin = last if i == 0 else rev[i - 1]
        for j in range(layers + 1):
            s += _resnet(f"decoder.up_blocks.{i}.resnets.{j}", cin if j == 0 else out, out)
        if i + 1 < len(rev):
            s += _conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", out, out, 3)
    s += _norm("decoder.conv_norm_out", channels[0])
    s += _conv("decoder.conv_out", channels[0], 3, 3)
    return s


def encoder_specs(channels=SDXL_CHANNELS, layers=SDXL_LAYERS) -> List[Spec]:
    s = _conv("encoder.conv_in", 3, channels[0], 3)
    for i, out in enumerate(channels):
        cin = channels[0] if i == 0 else channels[i - 1]
        for j in range(layers):
            s += _resnet(f"encoder.down_blocks.{i}.resnets.{j}", cin if j == 0 else out, out)
        if i + 1 < len(channels):
            s += _conv(f"encoder.down_blocks.{i}.downsamplers.0.conv", out, out, 3)
    last = channels[-1]
    s += _mid("encoder.mid_block", last)
    s += _norm("encoder.conv_norm_out", last)
    s += _conv("encoder.conv_out", last, 8, 3)
    s += _conv("quant_conv", 8, 8, 1)
    return s


def _fill(rng: np.random.Generator, shape, init: str) -> np.ndarray:
    if init == "one":
        return np.ones(shape, np.float32)
    if init == "zero":
        return np.zeros(shape, np.float32)
    if init == "kaiming":
        fan_in = int(np.prod(shape[1:]))
        return (rng.standard_normal(shape, dtype=np.float32)
                * np.float32(np.sqrt(2.0 / fan_in)))
    raise ValueError(init)


def random_vae_weights(seed: int = 0, channels: Iterable[int] = SDXL_CHANNELS,
                       layers: int = SDXL_LAYERS, parts=("decoder", "encoder")
                       ) -> Dict[str, np.ndarray]:
    """Random-init VAE weights (float32, diffusers names), deterministic in
    ``seed``. Conv/linear biases are U(-1/sqrt(Cin), 1/sqrt(Cin)) with Cin the
    input channel count, as the reference's loader hints specify."""
    channels = tuple(channels)
    rng = np.random.Generator(np.random.PCG64(seed))
    specs: List[Spec] = []
    if "decoder" in parts:
        specs += decoder_specs(channels, layers)
    if "encoder" in parts:
        specs += encoder_specs(channels, layers)
    out: Dict[str, np.ndarray] = {}
    last_cin = 1
    for name, shape, init in specs:
        if init == "bias":
            bound = 1.0 / np.sqrt(last_cin)
            out[name] = rng.uniform(-bound, bound, size=shape).astype(np.float32)
        else:
            out[name] = _fill(rng, shape, init)
            if init == "kaiming":
                last_cin = shape[1]
    return out
