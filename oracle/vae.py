"""Oracle VAE block topology (TEST INFRASTRUCTURE ONLY).

Restates the reference's encoder/decoder composition on top of the C++ oracle
ops. Weights are a dict of float32 numpy arrays keyed by diffusers names.

Reference anchors:
  Resnet           src/native/vae_encoder.rs:107-152 (shortcut 1x1 when the
                   channel count changes; no time embedding, no output scale)
  DownBlock        src/native/vae_encoder.rs:154-215 (pad right/bottom by one,
                   then 3x3 stride 2 pad 0)
  Attention        src/native/vae_encoder.rs:237-340 (GN, q/k/v Linear, q and k
                   each scaled by C^-1/4, sliced softmax, out Linear, + input)
  MidBlock         src/native/vae_encoder.rs:342-376
  VaeEncoder       src/native/vae_encoder.rs:378-425
  UpBlock/Decoder  src/native/vae_decoder.rs:13-114
  posterior/decode mapping  src/pipeline.rs:720-745, 834-853
"""
from __future__ import annotations

import numpy as np

from . import (attend, conv2d, group_norm, pad_right_bottom, sgemm, upsample_2x)

SDXL_CHANNELS = (128, 256, 512, 512)
SDXL_LAYERS = 2
LATENT_SCALE = 0.13025


def _keep(x):
    return x


def _conv(w, name, x, stride=1, padding=None):
    weight = w[name + ".weight"]
    k = weight.shape[-1]
    if padding is None:
        padding = k // 2
    return conv2d(x, weight, w[name + ".bias"], stride=stride, padding=padding)


def _gn(w, name, x, silu):
    return group_norm(x, w[name + ".weight"], w[name + ".bias"], silu=silu)


def resnet(w, prefix, x, q=_keep):
    """q rounds each stored activation (identity for the F32 oracle; the
    precision emulation passes a 16-bit rounding)."""
    if prefix + ".conv_shortcut.weight" in w:
        shortcut = q(_conv(w, prefix + ".conv_shortcut", x))
    else:
        shortcut = x
    h = q(_conv(w, prefix + ".conv1", q(_gn(w, prefix + ".norm1", x, True))))
    h = _conv(w, prefix + ".conv2", q(_gn(w, prefix + ".norm2", h, True)))
    return q(shortcut + h)


def _linear_weight(w, name):
    weight = w[name + ".weight"]
    if weight.ndim == 4:
        weight = weight.reshape(weight.shape[0], weight.shape[1])
    return weight, w[name + ".bias"]


def attention(w, prefix, x, q=_keep):
    b, c, h, wd = x.shape
    names = ("to_q", "to_k", "to_v", "to_out.0")
    if prefix + ".to_q.weight" not in w:
        names = ("query", "key", "value", "proj_attn")
    n = h * wd
    xs = q(_gn(w, prefix + ".group_norm", x, False)).reshape(b, c, n).transpose(0, 2, 1)
    xs = np.ascontiguousarray(xs).reshape(b * n, c)

    def linear(name, inp):
        weight, bias = _linear_weight(w, prefix + "." + name)
        return sgemm(inp, np.ascontiguousarray(weight.T)) + bias

    scale = np.float32(float(c) ** -0.25)
    qs = q(linear(names[0], xs) * scale).reshape(b, n, c)
    ks = q(linear(names[1], xs) * scale).reshape(b, n, c)
    vs = q(linear(names[2], xs)).reshape(b, n, c)
    kt = np.ascontiguousarray(ks.transpose(0, 2, 1))
    o = q(attend(qs, kt, vs)).reshape(b * n, c)
    o = linear(names[3], o).reshape(b, n, c).transpose(0, 2, 1).reshape(b, c, h, wd)
    return q(o + x)


def mid_block(w, prefix, x, q=_keep):
    x = resnet(w, prefix + ".resnets.0", x, q)
    x = attention(w, prefix + ".attentions.0", x, q)
    return resnet(w, prefix + ".resnets.1", x, q)


def decode(w, latents, channels=SDXL_CHANNELS, layers=SDXL_LAYERS, observer=None, q=_keep):
    """VaeDecoder::forward: unscaled latents [B,4,h,w] -> raw RGB [B,3,8h,8w].

    observer(name, x), when given, sees each block's output (NCHW f32) under
    the reference's VAE trace names (src/native/precision_tests.rs:97-130):
    post_quant_conv, decoder.conv_in, decoder.mid_block, decoder.up_blocks.{i}
    (after its upsampler), decoder.conv_norm_out (after SiLU), decoder.conv_out.
    q rounds each stored activation (identity here; see oracle.precision)."""
    seen = observer or (lambda name, t: None)
    x = _conv(w, "post_quant_conv", np.asarray(latents, np.float32))
    seen("post_quant_conv", x)
    x = q(_conv(w, "decoder.conv_in", q(x)))
    seen("decoder.conv_in", x)
    x = mid_block(w, "decoder.mid_block", x, q)
    seen("decoder.mid_block", x)
    rev = list(reversed(channels))
    for i in range(len(rev)):
        for j in range(layers + 1):
            x = resnet(w, f"decoder.up_blocks.{i}.resnets.{j}", x, q)
        if i + 1 < len(rev):
            x = q(_conv(w, f"decoder.up_blocks.{i}.upsamplers.0.conv", upsample_2x(x)))
        seen(f"decoder.up_blocks.{i}", x)
    x = q(_gn(w, "decoder.conv_norm_out", x, True))
    seen("decoder.conv_norm_out", x)
    y = _conv(w, "decoder.conv_out", x)
    seen("decoder.conv_out", y)
    return y


def encode_moments(w, image, channels=SDXL_CHANNELS, layers=SDXL_LAYERS):
    """VaeEncoder::forward: normalized image [B,3,H,W] -> moments [B,8,H/8,W/8]."""
    x = _conv(w, "encoder.conv_in", np.asarray(image, np.float32))
    for i in range(len(channels)):
        for j in range(layers):
            x = resnet(w, f"encoder.down_blocks.{i}.resnets.{j}", x)
        if i + 1 < len(channels):
            x = _conv(w, f"encoder.down_blocks.{i}.downsamplers.0.conv", pad_right_bottom(x),
                      stride=2, padding=0)
    x = mid_block(w, "encoder.mid_block", x)
    x = _gn(w, "encoder.conv_norm_out", x, True)
    x = _conv(w, "encoder.conv_out", x)
    return _conv(w, "quant_conv", x)


def posterior_sample(moments, noise):
    """mean + exp(0.5 * clamp(logvar, -30, 20)) * noise (pipeline.rs:731-735)."""
    mean = moments[:, 0:4]
    logvar = np.clip(moments[:, 4:8], -30.0, 20.0)
    return (mean + np.exp(np.float32(0.5) * logvar) * noise).astype(np.float32)


def display_image(decoded):
    """clamp(0.5 * y + 0.5, 0, 1) in F32 (pipeline.rs:846-851)."""
    return np.clip(np.asarray(decoded, np.float32) * 0.5 + 0.5, 0.0, 1.0)
