"""Oracle SDXL inpainting UNet (TEST INFRASTRUCTURE ONLY).

Restates the reference's UNet forward (one denoising call) on top of the C++
oracle ops (column convolution, staged GroupNorm, SGEMM, sliced attention),
NCHW float32 like the reference's CPU F32 path. Weights are a dict of float32
numpy arrays keyed by diffusers names. Only tests, the smoke check and the
benchmark's CPU legs use this module.

Reference anchors (paths inside the reference project):
  Architecture / sdxl()   src/native.rs:51-98 (320/640/1280 channels, cross
                          depths 2 and 10, 5/10/20 heads, context 2048,
                          pooled 1280, time projection 256, two layers)
  Unet::new               src/native.rs:127-258 (block wiring, eps 1e-5,
                          downsample padding 1, up blocks with layers + 1)
  Unet::forward           src/native.rs:276-379 (time and added embeddings,
                          skip bookkeeping, upsample sizes from the next skip,
                          GroupNorm + SiLU + conv_out)
  CpuResnet               src/native/resnet.rs:43-119 (time_emb_proj of
                          silu(temb) added after conv1; output scale 1)
  PlainDown / PlainUp     src/native/unet_blocks.rs:17-251
  CrossDown / CrossUp /   src/native/cross_blocks.rs:36-251
  CrossMid
  SpatialTransformer      src/native/spatial.rs:197-262 (GroupNorm eps 1e-6,
                          linear proj_in / proj_out, + input)
  TransformerBlock        src/native/spatial.rs:160-195 (pre-LayerNorm self
                          attention, fixed-prompt cross attention, GEGLU)
  SelfAttention /         src/native/spatial.rs:11-158 (heads split from the
  FixedCrossAttention     channel axis, keys scaled by head_width^-1/2 in F32,
                          F32 softmax, keys / values of the prompt computed
                          once)
  FeedForward             src/native/transformer.rs:1-24 (exact-erf GEGLU)

Third-party arithmetic restated (candle-transformers / candle-nn 0.11.0, not
vendored in the reference): ``Timesteps`` (f32 exponent arange * -ln(1e4) /
half, exp, t * freq, cat(cos, sin) for flip_sin_to_cos), ``TimestepEmbedding``
(linear_1, SiLU, linear_2), ``GroupNorm`` (two-pass centred statistics, cast,
affine; the staged sums of the VAE oracle differ from it only in summation
order), ``LayerNorm`` (f32 mean / centred variance over the last axis, affine),
``upsample_nearest2d`` (source index floor(dst * (src / dst)) in f64).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
from scipy.special import erf as _erf

from . import attend, conv2d, group_norm, sgemm

RESNET_EPS = 1e-5
TRANSFORMER_GN_EPS = 1e-6
LAYER_NORM_EPS = 1e-5
UNET_IN_CHANNELS = 9
UNET_OUT_CHANNELS = 5


@dataclass(frozen=True)
class Block:
    channels: int
    depth: Optional[int]  # None: plain block; else transformer depth
    heads: int


@dataclass(frozen=True)
class Arch:
    blocks: Tuple[Block, Block, Block]
    context: int
    pooled: int
    time_projection: int
    layers: int

    @property
    def base(self) -> int:
        return self.blocks[0].channels

    @property
    def time_dim(self) -> int:
        return 4 * self.base


def sdxl() -> Arch:
    """src/native.rs:70-97."""
    return Arch((Block(320, None, 5), Block(640, 2, 10), Block(1280, 10, 20)),
                context=2048, pooled=1280, time_projection=256, layers=2)


def tiny() -> Arch:
    """The reference's tiny test architecture (src/native.rs:553-575)."""
    return Arch((Block(64, None, 1), Block(64, 1, 1), Block(64, 1, 1)),
                context=8, pooled=8, time_projection=8, layers=1)


# ------------------------------------------------------------------ weights
def _lin(prefix, cout, cin, bias=True):
    s = [(prefix + ".weight", (cout, cin))]
    return s + [(prefix + ".bias", (cout,))] if bias else s


def _conv(prefix, cin, cout, k):
    return [(prefix + ".weight", (cout, cin, k, k)), (prefix + ".bias", (cout,))]


def _norm(prefix, c):
    return [(prefix + ".weight", (c,)), (prefix + ".bias", (c,))]


def _resnet(prefix, cin, cout, time_dim):
    s = _norm(prefix + ".norm1", cin) + _conv(prefix + ".conv1", cin, cout, 3)
    s += _lin(prefix + ".time_emb_proj", cout, time_dim)
    s += _norm(prefix + ".norm2", cout) + _conv(prefix + ".conv2", cout, cout, 3)
    if cin != cout:
        s += _conv(prefix + ".conv_shortcut", cin, cout, 1)
    return s


def _transformer(prefix, c, depth, context):
    s = _norm(prefix + ".norm", c) + _lin(prefix + ".proj_in", c, c)
    for d in range(depth):
        t = f"{prefix}.transformer_blocks.{d}"
        s += _norm(t + ".norm1", c)
        for n in ("to_q", "to_k", "to_v"):
            s += _lin(f"{t}.attn1.{n}", c, c, bias=False)
        s += _lin(t + ".attn1.to_out.0", c, c)
        s += _norm(t + ".norm2", c)
        s += _lin(t + ".attn2.to_q", c, c, bias=False)
        s += _lin(t + ".attn2.to_k", c, context, bias=False)
        s += _lin(t + ".attn2.to_v", c, context, bias=False)
        s += _lin(t + ".attn2.to_out.0", c, c)
        s += _norm(t + ".norm3", c)
        s += _lin(t + ".ff.net.0.proj", 8 * c, c) + _lin(t + ".ff.net.2", c, 4 * c)
    return s + _lin(prefix + ".proj_out", c, c)


def up_channels(arch: Arch, i: int):
    """(previous, skip-input, output) channels of up block i (src/native.rs:201-214)."""
    blocks, n = arch.blocks, len(arch.blocks)
    spec = blocks[n - 1 - i]
    prev = blocks[-1].channels if i == 0 else blocks[n - i].channels
    inp = arch.base if i + 1 == n else blocks[n - i - 2].channels
    return prev, inp, spec.channels


def specs(arch: Arch) -> List[Tuple[str, Tuple[int, ...]]]:
    """Every UNet tensor (diffusers name, shape), in the reference's build order."""
    base, td = arch.base, arch.time_dim
    s = _conv("conv_in", UNET_IN_CHANNELS, base, 3)
    s += _lin("time_embedding.linear_1", td, base) + _lin("time_embedding.linear_2", td, td)
    s += _lin("add_embedding.linear_1", td, arch.pooled + 6 * arch.time_projection)
    s += _lin("add_embedding.linear_2", td, td)
    n = len(arch.blocks)
    for i, spec in enumerate(arch.blocks):
        cin = base if i == 0 else arch.blocks[i - 1].channels
        for j in range(arch.layers):
            p = f"down_blocks.{i}"
            s += _resnet(f"{p}.resnets.{j}", cin if j == 0 else spec.channels, spec.channels, td)
            if spec.depth is not None:
                s += _transformer(f"{p}.attentions.{j}", spec.channels, spec.depth, arch.context)
        if i + 1 < n:
            s += _conv(f"down_blocks.{i}.downsamplers.0.conv", spec.channels, spec.channels, 3)
    last = arch.blocks[-1]
    s += _resnet("mid_block.resnets.0", last.channels, last.channels, td)
    s += _transformer("mid_block.attentions.0", last.channels, last.depth, arch.context)
    s += _resnet("mid_block.resnets.1", last.channels, last.channels, td)
    for i in range(n):
        prev, inp, out = up_channels(arch, i)
        spec = arch.blocks[n - 1 - i]
        layers = arch.layers + 1
        for j in range(layers):
            skip = inp if j + 1 == layers else out
            ch = prev if j == 0 else out
            s += _resnet(f"up_blocks.{i}.resnets.{j}", ch + skip, out, td)
            if spec.depth is not None:
                s += _transformer(f"up_blocks.{i}.attentions.{j}", out, spec.depth, arch.context)
        if i + 1 < n:
            s += _conv(f"up_blocks.{i}.upsamplers.0.conv", out, out, 3)
    s += _norm("conv_norm_out", base) + _conv("conv_out", base, UNET_OUT_CHANNELS, 3)
    return s


def fixed_values(count: int, state: int) -> np.ndarray:
    """Odd dyadic values in (-1, 1) from the reference's test LCG
    (src/native.rs:642-650)."""
    out = np.empty(count, np.float32)
    state &= 0xFFFFFFFF
    for i in range(count):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(((state >> 24) * 2 - 255) / 256.0)
    return out


def _fnv1a(name: str) -> int:
    h = 0x811C9DC5
    for byte in name.encode():
        h = ((h ^ byte) * 16777619) & 0xFFFFFFFF
    return h


def deterministic_weights(arch: Arch) -> Dict[str, np.ndarray]:
    """The reference's deterministic fixture (src/native.rs:591-639): matrices
    are fixed_values(seed = FNV-1a of the name) * 0.5 / next_pow2(isqrt(fan_in)),
    vectors named .weight are ones and biases zeros."""
    out = {}
    for name, shape in specs(arch):
        if name.endswith(".weight") and len(shape) > 1:
            fan_in = int(np.prod(shape[1:]))
            den = max(math.isqrt(fan_in), 1)
            den = 1 << (den - 1).bit_length()
            out[name] = (fixed_values(int(np.prod(shape)), _fnv1a(name))
                         * np.float32(0.5 / den)).reshape(shape)
        elif name.endswith(".weight"):
            out[name] = np.ones(shape, np.float32)
        else:
            out[name] = np.zeros(shape, np.float32)
    return out


# ------------------------------------------------------------------ ops
def _f32(a):
    return np.ascontiguousarray(np.asarray(a, np.float32))


def silu(x):
    x = _f32(x)
    return x / (np.float32(1.0) + np.exp(-x))


def gelu_erf(x):
    x64 = np.asarray(x, np.float64)
    return (0.5 * x64 * (1.0 + _erf(x64 / math.sqrt(2.0)))).astype(np.float32)


def linear(w, name, x):
    """y = x W^T (+ b) over the last axis (candle-nn Linear)."""
    x = _f32(x)
    weight = w[name + ".weight"]
    lead = x.shape[:-1]
    y = sgemm(x.reshape(-1, x.shape[-1]), np.ascontiguousarray(weight.T))
    if name + ".bias" in w:
        y = y + w[name + ".bias"]
    return y.reshape(*lead, weight.shape[0])


def layer_norm(w, name, x, eps=LAYER_NORM_EPS):
    x = _f32(x)
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float32)
    d = x - mean
    var = (d * d).mean(axis=-1, keepdims=True, dtype=np.float32)
    y = d / np.sqrt(var + np.float32(eps))
    return (y * w[name + ".weight"] + w[name + ".bias"]).astype(np.float32)


def conv(w, name, x, stride=1, padding=None):
    weight = w[name + ".weight"]
    k = weight.shape[-1]
    return conv2d(x, weight, w[name + ".bias"], stride=stride,
                  padding=k // 2 if padding is None else padding)


def gn(w, name, x, eps, act):
    return group_norm(x, w[name + ".weight"], w[name + ".bias"], silu=act, eps=eps)


def upsample_nearest(x, height: int, width: int):
    """candle upsample_nearest2d: src = min(src_len - 1, floor(dst * (src_len / dst_len)))."""
    x = _f32(x)
    _, _, h, wd = x.shape
    sy = np.minimum(h - 1, (np.arange(height) * (h / height)).astype(np.int64))
    sx = np.minimum(wd - 1, (np.arange(width) * (wd / width)).astype(np.int64))
    return np.ascontiguousarray(x[:, :, sy][:, :, :, sx])


def timesteps(t, channels: int):
    """Sinusoidal projection, flip_sin_to_cos, no frequency shift (candle
    Timesteps(channels, true, 0)): [n] f32 -> [n, channels] f32."""
    half = channels // 2
    exponent = np.arange(half, dtype=np.float32) * np.float32(-math.log(10000.0))
    exponent = exponent * np.float32(1.0 / half)
    freq = np.exp(exponent).astype(np.float32)
    emb = _f32(t)[:, None] * freq[None, :]
    return np.concatenate([np.cos(emb), np.sin(emb)], axis=1).astype(np.float32)


# ------------------------------------------------------------------ blocks
def resnet(w, prefix, x, temb):
    """src/native/resnet.rs:96-118."""
    if prefix + ".conv_shortcut.weight" in w:
        shortcut = conv(w, prefix + ".conv_shortcut", x)
    else:
        shortcut = x
    h = conv(w, prefix + ".conv1", gn(w, prefix + ".norm1", x, RESNET_EPS, True))
    t = linear(w, prefix + ".time_emb_proj", silu(temb))
    h = h + t[:, :, None, None]
    h = conv(w, prefix + ".conv2", gn(w, prefix + ".norm2", h, RESNET_EPS, True))
    return shortcut + h


def _split_heads(x, heads):
    b, n, c = x.shape
    return np.ascontiguousarray(
        x.reshape(b, n, heads, c // heads).transpose(0, 2, 1, 3).reshape(b * heads, n, c // heads))


def _merge_heads(x, heads):
    bh, n, d = x.shape
    return np.ascontiguousarray(
        x.reshape(bh // heads, heads, n, d).transpose(0, 2, 1, 3).reshape(bh // heads, n, heads * d))


def cross_keys(w, prefix, context, heads):
    """Keys (transposed, scaled) and values of the fixed prompt, computed once
    (src/native/spatial.rs:104-128): [heads, d, T] and [heads, T, d]."""
    c = w[prefix + ".to_q.weight"].shape[0]
    scale = np.float32(1.0 / math.sqrt(c // heads))
    k = _split_heads(linear(w, prefix + ".to_k", context), heads)
    v = _split_heads(linear(w, prefix + ".to_v", context), heads)
    return np.ascontiguousarray(k.transpose(0, 2, 1)) * scale, v


def attention(w, prefix, x, heads, context=None, cached=None):
    """Self attention (context None) or fixed-prompt cross attention
    (src/native/spatial.rs:56-158). x [B, N, C]."""
    b = x.shape[0]
    q = _split_heads(linear(w, prefix + ".to_q", x), heads)
    if context is None:
        c = x.shape[2]
        scale = np.float32(1.0 / math.sqrt(c // heads))
        kt = np.ascontiguousarray(_split_heads(linear(w, prefix + ".to_k", x), heads)
                                  .transpose(0, 2, 1)) * scale
        v = _split_heads(linear(w, prefix + ".to_v", x), heads)
    else:
        kt, v = cached if cached is not None else cross_keys(w, prefix, context, heads)
        kt, v = np.tile(kt, (b, 1, 1)), np.tile(v, (b, 1, 1))
    o = _merge_heads(attend(q, kt, v), heads)
    return linear(w, prefix + ".to_out.0", o)


def feed_forward(w, prefix, x):
    """GEGLU feed-forward (src/native/transformer.rs:8-24)."""
    p = linear(w, prefix + ".net.0.proj", x)
    half = p.shape[-1] // 2
    return linear(w, prefix + ".net.2", p[..., :half] * gelu_erf(p[..., half:]))


def transformer_block(w, prefix, x, heads, context):
    x = x + attention(w, prefix + ".attn1", layer_norm(w, prefix + ".norm1", x), heads)
    x = x + attention(w, prefix + ".attn2", layer_norm(w, prefix + ".norm2", x), heads,
                      context=context)
    return x + feed_forward(w, prefix + ".ff", layer_norm(w, prefix + ".norm3", x))


def spatial_transformer(w, prefix, x, heads, depth, context):
    """src/native/spatial.rs:233-262."""
    b, c, h, wd = x.shape
    xs = gn(w, prefix + ".norm", x, TRANSFORMER_GN_EPS, False)
    xs = np.ascontiguousarray(xs.reshape(b, c, h * wd).transpose(0, 2, 1))
    xs = linear(w, prefix + ".proj_in", xs)
    for d in range(depth):
        xs = transformer_block(w, f"{prefix}.transformer_blocks.{d}", xs, heads, context)
    xs = linear(w, prefix + ".proj_out", xs)
    return np.ascontiguousarray(xs.transpose(0, 2, 1).reshape(b, c, h, wd)) + x


def embedding(w, arch: Arch, batch: int, timestep: int, time_ids, pooled):
    """Time + added (pooled text, time ids) embedding (src/native.rs:318-337)."""
    t = np.full(batch, np.float32(timestep), np.float32)
    emb = linear(w, "time_embedding.linear_1", timesteps(t, arch.base))
    emb = linear(w, "time_embedding.linear_2", silu(emb))
    ids = timesteps(_f32(time_ids).reshape(-1), arch.time_projection)
    ids = ids.reshape(batch, 6 * arch.time_projection)
    add = np.concatenate([np.tile(_f32(pooled).reshape(1, -1), (batch, 1)), ids], axis=1)
    add = linear(w, "add_embedding.linear_1", add)
    add = linear(w, "add_embedding.linear_2", silu(add))
    return emb + add


def forward(w, arch: Arch, sample, timestep: int, time_ids, context, pooled):
    """UNet denoise: sample [B, 9, h, w] -> [B, 5, h, w] (src/native.rs:276-379).
    context [1, T, arch.context], pooled [1, arch.pooled]."""
    sample = _f32(sample)
    b, ch, h, wd = sample.shape
    if ch != UNET_IN_CHANNELS or _f32(time_ids).shape != (b, 6):
        raise ValueError("UNet input must be [B, 9, h, w] with time_ids [B, 6]")
    ctx = _f32(context).reshape(1, -1, arch.context)
    temb = embedding(w, arch, b, timestep, time_ids, pooled)
    xs = conv(w, "conv_in", sample)
    residuals = [xs]
    n = len(arch.blocks)
    for i, spec in enumerate(arch.blocks):
        for j in range(arch.layers):
            xs = resnet(w, f"down_blocks.{i}.resnets.{j}", xs, temb)
            if spec.depth is not None:
                xs = spatial_transformer(w, f"down_blocks.{i}.attentions.{j}", xs, spec.heads,
                                         spec.depth, ctx)
            residuals.append(xs)
        if i + 1 < n:
            xs = conv(w, f"down_blocks.{i}.downsamplers.0.conv", xs, stride=2, padding=1)
            residuals.append(xs)
    last = arch.blocks[-1]
    xs = resnet(w, "mid_block.resnets.0", xs, temb)
    xs = spatial_transformer(w, "mid_block.attentions.0", xs, last.heads, last.depth, ctx)
    xs = resnet(w, "mid_block.resnets.1", xs, temb)
    for i in range(n):
        spec = arch.blocks[n - 1 - i]
        count = arch.layers + 1
        saved = residuals[len(residuals) - count:]
        del residuals[len(residuals) - count:]
        for j, skip in enumerate(reversed(saved)):
            xs = resnet(w, f"up_blocks.{i}.resnets.{j}", np.concatenate([xs, skip], axis=1), temb)
            if spec.depth is not None:
                xs = spatial_transformer(w, f"up_blocks.{i}.attentions.{j}", xs, spec.heads,
                                         spec.depth, ctx)
        if i + 1 < n:
            size = residuals[-1].shape[2:]
            xs = conv(w, f"up_blocks.{i}.upsamplers.0.conv", upsample_nearest(xs, *size))
    assert not residuals
    return conv(w, "conv_out", gn(w, "conv_norm_out", xs, RESNET_EPS, True))
