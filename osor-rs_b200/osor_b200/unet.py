"""SDXL inpainting UNet on the library's B200 kernels.

Host mirror of the reference's ``Unet`` (src/native.rs:112-379) and of
``NativeModel::denoise`` (src/native.rs:503-519): one denoising call maps the
nine-channel latent input [B, 9, h, w] (noisy latent, pooled mask, masked
latent) at one timestep, with the SDXL time ids [B, 6] and the fixed prompt
conditioning bound at load, to the five-channel output [B, 5, h, w].

``UnetGraph`` is the block topology: time and added embeddings, the down
blocks with their skip tensors, the cross-attention middle block, the up
blocks that concatenate the skips (most recent first) and resize to the next
skip's size, and the output GroupNorm + SiLU + convolution. It runs on an ops
backend; ``CudaUnetOps`` is the product backend, every op a C-ABI call of
``libosor_b200`` on 16-bit NHWC device tensors:

  convolutions, linear layers over pixels   osor_conv2d (tensor cores when
        Cin % 64 == 0 and Cout % 128 == 0; Cout = 320 runs as a zero-padded
        384-channel product narrowed by osor_channel_update)
  GroupNorm(+SiLU)                          osor_group_norm_silu (NHWC)
  time / added embeddings, time_emb_proj    osor_unet_time_features +
        osor_rows_linear (all resnets' time biases in one launch)
  LayerNorm, GEGLU, attention               osor_layer_norm, osor_geglu,
        osor_attention_heads (self attention on the fused q|k|v product,
        cross attention on the prompt's keys / values computed at load)
  skip concatenation, nearest resize        osor_concat_channels,
        osor_resize_nearest

A transformer's token rows are the H * W pixels of an NHWC image, so the
reference's reshapes and transposes around the spatial transformer
(src/native/spatial.rs:240-259) cost nothing here.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Mapping, Optional, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import InvalidArtifact, InvalidInput, check, dtype_code
from .ops import HALF_TYPES

IN_CHANNELS = 9
OUT_CHANNELS = 5
RESNET_EPS = 1e-5
TRANSFORMER_GN_EPS = 1e-6
LAYER_NORM_EPS = 1e-5
MAX_BATCH = 4
MIN_LATENT = 4    # 32-pixel images
MAX_LATENT = 128  # 1024-pixel images
GROUPS = 32

Checkpoint = Optional[Callable[[], None]]


@dataclass(frozen=True)
class BlockSpec:
    channels: int
    depth: Optional[int]  # transformer depth; None for a plain block
    heads: int


@dataclass(frozen=True)
class Architecture:
    """The reference's ``Architecture`` (src/native.rs:51-98)."""
    blocks: Tuple[BlockSpec, BlockSpec, BlockSpec]
    context: int = 2048
    pooled: int = 1280
    time_projection: int = 256
    layers: int = 2

    @property
    def base(self) -> int:
        return self.blocks[0].channels

    @property
    def time_dim(self) -> int:
        return 4 * self.base

    @classmethod
    def sdxl(cls) -> "Architecture":
        return cls((BlockSpec(320, None, 5), BlockSpec(640, 2, 10), BlockSpec(1280, 10, 20)))

    @classmethod
    def tiny(cls) -> "Architecture":
        """The reference's test architecture (src/native.rs:553-575)."""
        return cls((BlockSpec(64, None, 1), BlockSpec(64, 1, 1), BlockSpec(64, 1, 1)),
                   context=8, pooled=8, time_projection=8, layers=1)


# ------------------------------------------------------------------ inventory
def _lin(prefix, cout, cin, bias=True):
    s = [(prefix + ".weight", (cout, cin))]
    return s + [(prefix + ".bias", (cout,))] if bias else s


def _conv(prefix, cin, cout, k):
    return [(prefix + ".weight", (cout, cin, k, k)), (prefix + ".bias", (cout,))]


def _norm(prefix, c):
    return [(prefix + ".weight", (c,)), (prefix + ".bias", (c,))]


def _resnet_specs(prefix, cin, cout, time_dim):
    s = _norm(prefix + ".norm1", cin) + _conv(prefix + ".conv1", cin, cout, 3)
    s += _lin(prefix + ".time_emb_proj", cout, time_dim)
    s += _norm(prefix + ".norm2", cout) + _conv(prefix + ".conv2", cout, cout, 3)
    if cin != cout:
        s += _conv(prefix + ".conv_shortcut", cin, cout, 1)
    return s


def _transformer_specs(prefix, c, depth, context):
    s = _norm(prefix + ".norm", c) + _lin(prefix + ".proj_in", c, c)
    for d in range(depth):
        t = f"{prefix}.transformer_blocks.{d}"
        s += _norm(t + ".norm1", c)
        for n in ("to_q", "to_k", "to_v"):
            s += _lin(f"{t}.attn1.{n}", c, c, bias=False)
        s += _lin(t + ".attn1.to_out.0", c, c) + _norm(t + ".norm2", c)
        s += _lin(t + ".attn2.to_q", c, c, bias=False)
        s += _lin(t + ".attn2.to_k", c, context, bias=False)
        s += _lin(t + ".attn2.to_v", c, context, bias=False)
        s += _lin(t + ".attn2.to_out.0", c, c) + _norm(t + ".norm3", c)
        s += _lin(t + ".ff.net.0.proj", 8 * c, c) + _lin(t + ".ff.net.2", c, 4 * c)
    return s + _lin(prefix + ".proj_out", c, c)


def up_channels(arch: Architecture, i: int) -> Tuple[int, int, int]:
    """(previous, skip input, output) channels of up block i (src/native.rs:201-214)."""
    blocks, n = arch.blocks, len(arch.blocks)
    prev = blocks[-1].channels if i == 0 else blocks[n - i].channels
    inp = arch.base if i + 1 == n else blocks[n - i - 2].channels
    return prev, inp, blocks[n - 1 - i].channels


def unet_specs(arch: Architecture) -> List[Tuple[str, Tuple[int, ...]]]:
    """Every tensor the UNet reads (diffusers name, shape), in build order
    (src/native.rs:127-258, src/native/cross_blocks.rs, unet_blocks.rs)."""
    base, td, n = arch.base, arch.time_dim, len(arch.blocks)
    s = _conv("conv_in", IN_CHANNELS, base, 3)
    s += _lin("time_embedding.linear_1", td, base) + _lin("time_embedding.linear_2", td, td)
    s += _lin("add_embedding.linear_1", td, arch.pooled + 6 * arch.time_projection)
    s += _lin("add_embedding.linear_2", td, td)
    for i, spec in enumerate(arch.blocks):
        cin = base if i == 0 else arch.blocks[i - 1].channels
        for j in range(arch.layers):
            s += _resnet_specs(f"down_blocks.{i}.resnets.{j}", cin if j == 0 else spec.channels,
                               spec.channels, td)
            if spec.depth is not None:
                s += _transformer_specs(f"down_blocks.{i}.attentions.{j}", spec.channels,
                                        spec.depth, arch.context)
        if i + 1 < n:
            s += _conv(f"down_blocks.{i}.downsamplers.0.conv", spec.channels, spec.channels, 3)
    last = arch.blocks[-1]
    s += _resnet_specs("mid_block.resnets.0", last.channels, last.channels, td)
    s += _transformer_specs("mid_block.attentions.0", last.channels, last.depth, arch.context)
    s += _resnet_specs("mid_block.resnets.1", last.channels, last.channels, td)
    for i in range(n):
        prev, inp, out = up_channels(arch, i)
        spec = arch.blocks[n - 1 - i]
        layers = arch.layers + 1
        for j in range(layers):
            skip = inp if j + 1 == layers else out
            s += _resnet_specs(f"up_blocks.{i}.resnets.{j}", (prev if j == 0 else out) + skip,
                               out, td)
            if spec.depth is not None:
                s += _transformer_specs(f"up_blocks.{i}.attentions.{j}", out, spec.depth,
                                        arch.context)
        if i + 1 < n:
            s += _conv(f"up_blocks.{i}.upsamplers.0.conv", out, out, 3)
    s += _norm("conv_norm_out", base) + _conv("conv_out", base, OUT_CHANNELS, 3)
    return s


def resnet_prefixes(arch: Architecture) -> List[str]:
    """Resnet blocks in execution order (their time biases are stacked in it)."""
    out, n = [], len(arch.blocks)
    for i in range(n):
        out += [f"down_blocks.{i}.resnets.{j}" for j in range(arch.layers)]
    out += ["mid_block.resnets.0", "mid_block.resnets.1"]
    for i in range(n):
        out += [f"up_blocks.{i}.resnets.{j}" for j in range(arch.layers + 1)]
    return out


def random_unet_weights(arch: Architecture, seed: int = 0, device="cpu",
                        dtype=torch.float32) -> Dict[str, torch.Tensor]:
    """Random-init UNet tensors with the reference loader's init hints: Kaiming
    normal matrices (std sqrt(2 / fan_in)), biases U(-1/sqrt(fan_in),
    1/sqrt(fan_in)) of the preceding matrix's fan-in, norm weights 1 and biases
    0. Drawn from torch's seeded generator on `device`, in inventory order."""
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    out: Dict[str, torch.Tensor] = {}
    fan_in = 1
    for name, shape in unet_specs(arch):
        norm = name.rsplit(".", 2)[-2].startswith("norm") or name.startswith("conv_norm_out")
        if len(shape) > 1:
            fan_in = int(np.prod(shape[1:]))
            t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
            t.mul_(math.sqrt(2.0 / fan_in))
        elif norm:
            t = (torch.ones if name.endswith(".weight") else torch.zeros)(
                shape, device=device, dtype=torch.float32)
        else:
            bound = 1.0 / math.sqrt(fan_in)
            t = torch.rand(shape, generator=gen, device=device, dtype=torch.float32)
            t.mul_(2 * bound).sub_(bound)
        out[name] = t.to(dtype)
    return out



def unet_flops(arch: Architecture, batch: int, h: int, w: int, tokens: int = 77) -> float:
    """FLOPs (2 per multiply-add) of one forward's convolutions, linear layers
    and attention products; elementwise work and the prompt's keys / values
    (computed once at load) are not counted."""
    shapes = dict(unet_specs(arch))

    def conv_f(name, hh, ww):
        co, ci, k, _ = shapes[name + ".weight"]
        return 2.0 * batch * hh * ww * co * ci * k * k

    def lin_f(name, rows):
        co, ci = shapes[name + ".weight"]
        return 2.0 * rows * co * ci

    def resnet_f(prefix, hh, ww):
        f = conv_f(prefix + ".conv1", hh, ww) + conv_f(prefix + ".conv2", hh, ww)
        if prefix + ".conv_shortcut.weight" in shapes:
            f += conv_f(prefix + ".conv_shortcut", hh, ww)
        return f

    def transformer_f(prefix, spec, hh, ww):
        n = hh * ww
        rows, c = batch * n, spec.channels
        f = 2 * lin_f(prefix + ".proj_in", rows)
        for d in range(spec.depth):
            t = f"{prefix}.transformer_blocks.{d}"
            f += 4 * lin_f(t + ".attn1.to_q", rows) + 4.0 * batch * n * n * c
            f += 2 * lin_f(t + ".attn2.to_q", rows) + 4.0 * batch * n * tokens * c
            f += lin_f(t + ".ff.net.0.proj", rows) + lin_f(t + ".ff.net.2", rows)
        return f

    n = len(arch.blocks)
    sizes = [(h, w)]
    for _ in range(n - 1):
        sizes.append(((sizes[-1][0] - 1) // 2 + 1, (sizes[-1][1] - 1) // 2 + 1))
    total = conv_f("conv_in", h, w) + conv_f("conv_out", h, w)
    for i, spec in enumerate(arch.blocks):
        for j in range(arch.layers):
            total += resnet_f(f"down_blocks.{i}.resnets.{j}", *sizes[i])
            if spec.depth is not None:
                total += transformer_f(f"down_blocks.{i}.attentions.{j}", spec, *sizes[i])
        if i + 1 < n:
            total += conv_f(f"down_blocks.{i}.downsamplers.0.conv", *sizes[i + 1])
    last = arch.blocks[-1]
    total += resnet_f("mid_block.resnets.0", *sizes[-1]) + resnet_f("mid_block.resnets.1", *sizes[-1])
    total += transformer_f("mid_block.attentions.0", last, *sizes[-1])
    for i in range(n):
        spec, size = arch.blocks[n - 1 - i], sizes[n - 1 - i]
        for j in range(arch.layers + 1):
            total += resnet_f(f"up_blocks.{i}.resnets.{j}", *size)
            if spec.depth is not None:
                total += transformer_f(f"up_blocks.{i}.attentions.{j}", spec, *size)
        if i + 1 < n:
            total += conv_f(f"up_blocks.{i}.upsamplers.0.conv", *sizes[n - 2 - i])
    return total

# ------------------------------------------------------------------ topology
class UnetGraph:
    """Unet::forward (src/native.rs:276-379) over an ops backend. Tensors are
    NHWC [B, H, W, C]; the input is NCHW f32 [B, 9, h, w] and the output NCHW
    f32 [B, 5, h, w]."""

    def __init__(self, arch: Architecture, ops):
        self.arch = arch
        self.ops = ops

    def forward(self, sample, timestep: int, time_ids, checkpoint: Checkpoint = None):
        arch, ops = self.arch, self.ops
        cp = checkpoint or (lambda: None)
        n = len(arch.blocks)
        temb = ops.embedding(sample.shape[0], timestep, time_ids)
        tb = ops.time_biases(temb)
        xs = ops.conv_in(sample)
        residuals = [xs]
        for i, spec in enumerate(arch.blocks):
            cp()
            for j in range(arch.layers):
                xs = self.resnet(f"down_blocks.{i}.resnets.{j}", xs, tb)
                if spec.depth is not None:
                    xs = self.transformer(f"down_blocks.{i}.attentions.{j}", xs, spec, cp)
                residuals.append(xs)
            if i + 1 < n:
                xs = ops.conv(xs, f"down_blocks.{i}.downsamplers.0.conv", stride=2)
                residuals.append(xs)
        cp()
        last = arch.blocks[-1]
        xs = self.resnet("mid_block.resnets.0", xs, tb)
        xs = self.transformer("mid_block.attentions.0", xs, last, cp)
        xs = self.resnet("mid_block.resnets.1", xs, tb)
        for i in range(n):
            cp()
            spec = arch.blocks[n - 1 - i]
            count = arch.layers + 1
            if len(residuals) < count:
                raise InvalidArtifact("UNet residual topology is inconsistent")
            saved = residuals[len(residuals) - count:]
            del residuals[len(residuals) - count:]
            for j, skip in enumerate(reversed(saved)):
                xs = self.resnet(f"up_blocks.{i}.resnets.{j}", ops.concat(xs, skip), tb)
                if spec.depth is not None:
                    xs = self.transformer(f"up_blocks.{i}.attentions.{j}", xs, spec, cp)
            if i + 1 < n:
                # The next skip fixes the size: downsampling rounds odd axes up.
                h, w = residuals[-1].shape[1], residuals[-1].shape[2]
                xs = ops.conv(ops.resize(xs, h, w), f"up_blocks.{i}.upsamplers.0.conv")
        if residuals:
            raise InvalidArtifact("UNet residual topology left unused tensors")
        cp()
        return ops.conv_out(ops.group_norm(xs, "conv_norm_out", RESNET_EPS, True))

    def resnet(self, prefix: str, x, tb):
        """src/native/resnet.rs:96-118: the time bias joins conv1's output and
        the shortcut joins conv2's."""
        ops = self.ops
        shortcut = ops.conv(x, prefix + ".conv_shortcut") if ops.has(prefix + ".conv_shortcut") else x
        h = ops.conv(ops.group_norm(x, prefix + ".norm1", RESNET_EPS, True), prefix + ".conv1",
                     image_bias=tb[prefix])
        return ops.conv(ops.group_norm(h, prefix + ".norm2", RESNET_EPS, True), prefix + ".conv2",
                        residual=shortcut)

    def transformer(self, prefix: str, x, spec: BlockSpec, cp):
        """SpatialTransformer (src/native/spatial.rs:233-262) with its blocks
        (:183-195)."""
        ops = self.ops
        xs = ops.linear(ops.group_norm(x, prefix + ".norm", TRANSFORMER_GN_EPS, False),
                        prefix + ".proj_in")
        for d in range(spec.depth):
            cp()
            t = f"{prefix}.transformer_blocks.{d}"
            xs = ops.self_attention(ops.layer_norm(xs, t + ".norm1"), t + ".attn1", spec.heads, xs)
            xs = ops.cross_attention(ops.layer_norm(xs, t + ".norm2"), t + ".attn2", spec.heads, xs)
            xs = ops.feed_forward(ops.layer_norm(xs, t + ".norm3"), t + ".ff", xs)
        return ops.linear(xs, prefix + ".proj_out", residual=x)


# ------------------------------------------------------------------ CUDA ops
def _ptr(t: Optional[torch.Tensor], offset_elems: int = 0):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr() + offset_elems * t.element_size())


def _padded(cout: int, cin: int) -> int:
    """Output channels a product is computed with: Cout rounded up to 128 when
    that puts it on the tensor-core path (Cin % 64 == 0), else Cout."""
    if cin % 64 == 0 and cout % 128 != 0 and cout % 8 == 0:
        return (cout + 127) // 128 * 128
    return cout


def _geglu_rows(features: int, device) -> torch.Tensor:
    """Row order of a GEGLU input projection for osor_linear_geglu: per 128
    features, the 128 value rows and then their 128 gate rows."""
    r = torch.arange(2 * features, device=device)
    t, j = r // 256, r % 256
    return torch.where(j < 128, t * 128 + j, features + t * 128 + (j - 128))


class _Product:
    """A convolution / linear layer packed once: 16-bit [Cpad][k*k*Cin] in
    (ky, kx, ci) order (rows >= Cout zero) and f32 bias [Cpad]. geglu: a
    GEGLU input projection with its rows in _geglu_rows order."""
    __slots__ = ("weight", "bias", "cin", "cout", "cpad", "k", "geglu")

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor], device, dtype,
                 pad: bool = True, geglu: bool = False):
        w = weight.to(device=device, dtype=torch.float32)
        self.geglu = geglu
        if geglu:
            order = _geglu_rows(w.shape[0] // 2, w.device)
            w = w[order]
            if bias is not None:
                bias = bias.to(device=device, dtype=torch.float32)[order]
            pad = False
        if w.ndim == 2:
            w = w[:, :, None, None]
        self.cout, self.cin, self.k = w.shape[0], w.shape[1], w.shape[2]
        self.cpad = _padded(self.cout, self.cin) if pad else self.cout
        packed = torch.zeros((self.cpad, self.k * self.k * self.cin), device=device,
                             dtype=torch.float32)
        packed[:self.cout] = w.permute(0, 2, 3, 1).reshape(self.cout, -1)
        self.weight = packed.to(dtype).contiguous()
        self.bias = None
        if bias is not None:
            b = torch.zeros(self.cpad, device=device, dtype=torch.float32)
            b[:self.cout] = bias.to(device=device, dtype=torch.float32)
            self.bias = b


class CudaUnetOps:
    """UnetGraph's ops on the library's kernels (C ABI). Parameters are packed
    once from ``weights`` (diffusers names; numpy arrays or tensors): convolution
    and linear weights in the model dtype, norms in f32, the self-attention
    q|k|v weights fused with q pre-scaled by head_width^-1/2, every resnet's
    time_emb_proj stacked, and the prompt's cross-attention keys / values
    computed on the device (src/native/spatial.rs:104-128)."""

    def __init__(self, weights: Mapping[str, object], arch: Architecture, context, pooled,
                 device: torch.device, dtype=torch.bfloat16):
        if dtype not in HALF_TYPES:
            raise InvalidInput("UNet dtype must be bfloat16 or float16")
        self.arch, self.device, self.dtype = arch, device, dtype
        self.dt = dtype_code(dtype)
        self.lib = _lib.lib()
        td = arch.time_dim

        def get(name, shape):
            t = weights.get(name) if hasattr(weights, "get") else weights[name]
            if t is None:
                raise InvalidArtifact(f"native model tensor missing or incompatible: {name}")
            t = t if torch.is_tensor(t) else torch.from_numpy(np.asarray(t, np.float32))
            if tuple(t.shape) != tuple(shape):
                raise InvalidArtifact(f"native model tensor missing or incompatible: {name}")
            return t.to(device=device, dtype=torch.float32)

        specs = dict(unet_specs(arch))
        w = {name: get(name, shape) for name, shape in specs.items()}
        ctx = torch.as_tensor(context).to(device=device, dtype=torch.float32)
        pool = torch.as_tensor(pooled).to(device=device, dtype=torch.float32)
        if ctx.ndim != 3 or ctx.shape[0] != 1 or not 1 <= ctx.shape[1] <= 1024 \
                or ctx.shape[2] != arch.context or tuple(pool.shape) != (1, arch.pooled):
            raise InvalidInput(f"fixed conditioning must be [1, 1..=1024, {arch.context}] "
                               f"and [1, {arch.pooled}]")
        self.pooled = pool.reshape(-1).contiguous()
        self.products: Dict[str, _Product] = {}
        self.norms: Dict[str, Tuple[torch.Tensor, torch.Tensor]] = {}
        for name in specs:
            if not name.endswith(".weight"):
                continue
            stem = name[:-len(".weight")]
            leaf = stem.rsplit(".", 1)[-1]
            if leaf.startswith("norm") or stem == "conv_norm_out":
                self.norms[stem] = (w[name].contiguous(), w[stem + ".bias"].contiguous())
            elif ".attn1.to_" in stem and leaf in ("to_q", "to_k", "to_v"):
                continue
            elif ".attn2.to_" in stem and leaf in ("to_q", "to_k", "to_v"):
                continue
            elif stem.startswith(("time_embedding.", "add_embedding.")) or leaf == "time_emb_proj":
                continue
            else:
                # GEGLU input projections with 128-multiple widths run fused.
                geglu = (stem.endswith(".ff.net.0.proj") and w[name].shape[0] % 256 == 0
                         and w[name].shape[1] % 8 == 0)
                self.products[stem] = _Product(w[name], w.get(stem + ".bias"), device, dtype,
                                               pad=stem != "conv_in", geglu=geglu)
        # conv_in as a 1x1 product over the 128-column matrix of its 3 x 3 x 9
        # taps (osor_thin_columns' order: tap-major, then channel).
        cw = w["conv_in.weight"].to(device=device, dtype=torch.float32)
        co, ci = cw.shape[0], cw.shape[1]
        cols = torch.zeros((co, 128), device=device, dtype=torch.float32)
        cols[:, :9 * ci] = cw.permute(0, 2, 3, 1).reshape(co, 9 * ci)
        self.products["conv_in.cols"] = _Product(cols, w.get("conv_in.bias"), device, dtype)
        # Attention: fused self-attention q|k|v, scaled cross-attention q, prompt K / V.
        self.cross_kv: Dict[str, Tuple[torch.Tensor, torch.Tensor]] = {}
        ctx16 = ctx.to(dtype).reshape(1, 1, ctx.shape[1], arch.context).contiguous()
        for name in specs:
            if not name.endswith(".attn1.to_q.weight"):
                continue
            a1 = name[:-len(".to_q.weight")]
            a2 = a1[:-1] + "2"
            c = w[name].shape[0]
            heads = self._heads_of(a1)
            scale = 1.0 / math.sqrt(c // heads)
            qkv = torch.cat([w[a1 + ".to_q.weight"] * scale, w[a1 + ".to_k.weight"],
                             w[a1 + ".to_v.weight"]])
            self.products[a1 + ".qkv"] = _Product(qkv, None, device, dtype)
            self.products[a2 + ".q"] = _Product(w[a2 + ".to_q.weight"] * scale, None, device,
                                                dtype)
            k = _Product(w[a2 + ".to_k.weight"], None, device, dtype, pad=False)
            v = _Product(w[a2 + ".to_v.weight"], None, device, dtype, pad=False)
            self.cross_kv[a2] = (self._raw(ctx16, k)[0].reshape(-1, c).contiguous(),
                                 self._raw(ctx16, v)[0].reshape(-1, c).contiguous())
        # Embeddings: block-diagonal first layers, concatenated second layers.
        base, add_w = arch.base, arch.pooled + 6 * arch.time_projection
        w1 = torch.zeros((2 * td, base + add_w), device=device)
        w1[:td, :base] = w["time_embedding.linear_1.weight"]
        w1[td:, base:] = w["add_embedding.linear_1.weight"]
        self.emb_w1 = w1.to(dtype).contiguous()
        self.emb_b1 = torch.cat([w["time_embedding.linear_1.bias"],
                                 w["add_embedding.linear_1.bias"]]).contiguous()
        self.emb_w2 = torch.cat([w["time_embedding.linear_2.weight"],
                                 w["add_embedding.linear_2.weight"]], 1).to(dtype).contiguous()
        self.emb_b2 = (w["time_embedding.linear_2.bias"].contiguous(),
                       w["add_embedding.linear_2.bias"].contiguous())
        self.resnets = resnet_prefixes(arch)
        self.temb_w = torch.cat([w[p + ".time_emb_proj.weight"] for p in self.resnets]) \
            .to(dtype).contiguous()
        self.temb_b = torch.cat([w[p + ".time_emb_proj.bias"] for p in self.resnets]).contiguous()
        del w

    def _heads_of(self, prefix: str) -> int:
        arch, n = self.arch, len(self.arch.blocks)
        if prefix.startswith("mid_block."):
            return arch.blocks[-1].heads
        idx = int(prefix.split(".")[1])
        if prefix.startswith("down_blocks."):
            return arch.blocks[idx].heads
        return arch.blocks[n - 1 - idx].heads

    @property
    def stream(self) -> ctypes.c_void_p:
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    # -- products
    def _raw(self, x: torch.Tensor, p: _Product, stride: int = 1,
             residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, int]:
        """x NHWC [B, H, W, Cin] -> [B, Ho, Wo, Cpad] (and Cpad)."""
        b, h, w, c = x.shape
        if c != p.cin:
            raise InvalidInput("convolution input channels do not match the weight")
        pad = p.k // 2
        oh = (h + 2 * pad - p.k) // stride + 1
        ow = (w + 2 * pad - p.k) // stride + 1
        y = torch.empty((b, oh, ow, p.cpad), device=x.device, dtype=self.dtype)
        check(self.lib.osor_conv2d(_ptr(x), _ptr(y), _ptr(p.weight), _ptr(p.bias),
                                   _ptr(residual), b, h, w, c, p.cpad, p.k, stride, pad, pad,
                                   _lib.LAYOUT_NHWC, _lib.LAYOUT_NHWC, self.dt, self.stream))
        return y, p.cpad

    def has(self, name: str) -> bool:
        return name in self.products

    def conv(self, x, name, stride=1, residual=None, image_bias=None):
        p = self.products[name]
        fused_residual = residual if p.cpad == p.cout and image_bias is None else None
        y, ld = self._raw(x, p, stride, fused_residual)
        if ld == p.cout and image_bias is None:
            return y
        b, oh, ow, _ = y.shape
        out = y if ld == p.cout else torch.empty((b, oh, ow, p.cout), device=y.device,
                                                 dtype=self.dtype)
        bias_stride = image_bias.stride(0) if image_bias is not None else 0
        check(self.lib.osor_channel_update(_ptr(y), ld, _ptr(out), p.cout, b, oh * ow,
                                           _ptr(image_bias), bias_stride,
                                           _ptr(None if fused_residual is not None else residual),
                                           self.dt, self.stream))
        return out

    linear = conv

    def conv_in(self, sample: torch.Tensor) -> torch.Tensor:
        b, c, h, w = sample.shape
        if 9 * c <= 128:
            # The column matrix, then a tensor-core 1x1 product (narrowed).
            cols = torch.empty((b, h, w, 128), device=sample.device, dtype=self.dtype)
            check(self.lib.osor_thin_columns(_ptr(sample), _ptr(cols), b, c, h, w, 3, 1, 128,
                                             self.dt, self.stream))
            return self.conv(cols, "conv_in.cols")
        p = self.products["conv_in"]
        y = torch.empty((b, h, w, p.cout), device=sample.device, dtype=self.dtype)
        check(self.lib.osor_conv2d(_ptr(sample), _ptr(y), _ptr(p.weight), _ptr(p.bias), None, b,
                                   h, w, c, p.cout, 3, 1, 1, 1, _lib.LAYOUT_NCHW,
                                   _lib.LAYOUT_NHWC, self.dt, self.stream))
        return y

    def conv_out(self, x: torch.Tensor) -> torch.Tensor:
        p = self.products["conv_out"]
        b, h, w, c = x.shape
        y = torch.empty((b, p.cout, h, w), device=x.device, dtype=torch.float32)
        check(self.lib.osor_conv2d(_ptr(x), _ptr(y), _ptr(p.weight), _ptr(p.bias), None, b, h,
                                   w, c, p.cout, 3, 1, 1, 1, _lib.LAYOUT_NHWC,
                                   _lib.LAYOUT_NCHW, self.dt, self.stream))
        return y

    # -- normalisation
    def group_norm(self, x, name, eps, silu):
        gamma, beta = self.norms[name]
        b, h, w, c = x.shape
        need = self.lib.osor_group_norm_workspace_size(b, c, h, w, _lib.LAYOUT_NHWC, self.dt)
        if need == 0:
            raise InvalidInput("unsupported group-norm shape")
        # Per call (the caching allocator makes this cheap): a captured graph
        # keeps every buffer it uses.
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        y = torch.empty_like(x)
        check(self.lib.osor_group_norm_silu(_ptr(x), _ptr(y), _ptr(gamma), _ptr(beta), b, c, h,
                                            w, _lib.LAYOUT_NHWC, self.dt, float(eps),
                                            1 if silu else 0, None, _ptr(ws), need, self.stream))
        return y

    def layer_norm(self, x, name):
        gamma, beta = self.norms[name]
        y = torch.empty_like(x)
        rows = x.numel() // x.shape[-1]
        check(self.lib.osor_layer_norm(_ptr(x), _ptr(y), _ptr(gamma), _ptr(beta), rows,
                                       x.shape[-1], LAYER_NORM_EPS, self.dt, self.stream))
        return y

    # -- transformer
    def _attend(self, q, ld_q, k, v, ld_kv, kv_bs, heads, n_kv, shape, k_off=0, v_off=0):
        b, h, w, c = shape
        n = h * w
        out = torch.empty((b, h, w, c), device=q.device, dtype=self.dtype)
        check(self.lib.osor_attention_heads(_ptr(q), ld_q, n * ld_q, _ptr(k, k_off),
                                            _ptr(v, v_off), ld_kv, kv_bs, _ptr(out), c, n * c,
                                            b, heads, n, n_kv, c // heads, self.dt,
                                            self.stream))
        return out

    def self_attention(self, x, prefix, heads, residual):
        c = x.shape[-1]
        qkv, ld = self._raw(x, self.products[prefix + ".qkv"])
        n = x.shape[1] * x.shape[2]
        o = self._attend(qkv, ld, qkv, qkv, ld, n * ld, heads, n, x.shape, k_off=c, v_off=2 * c)
        return self.linear(o, prefix + ".to_out.0", residual=residual)

    def cross_attention(self, x, prefix, heads, residual):
        q, ld = self._raw(x, self.products[prefix + ".q"])
        k, v = self.cross_kv[prefix]
        o = self._attend(q, ld, k, v, k.shape[1], 0, heads, k.shape[0], x.shape)
        return self.linear(o, prefix + ".to_out.0", residual=residual)

    def feed_forward(self, x, prefix, residual):
        p = self.products[prefix + ".net.0.proj"]
        if p.geglu:
            b, h, w, c = x.shape
            f = p.cout // 2
            gated = torch.empty((b, h, w, f), device=x.device, dtype=self.dtype)
            need = self.lib.osor_linear_geglu_workspace_size(b, h, w, c, f, self.dt)
            ws = torch.empty(need, dtype=torch.uint8, device=x.device) if need else None
            check(self.lib.osor_linear_geglu(_ptr(x), _ptr(gated), _ptr(p.weight), _ptr(p.bias),
                                             b, h, w, c, f, self.dt, _ptr(ws), need,
                                             self.stream))
            return self.linear(gated, prefix + ".net.2", residual=residual)
        hidden, ld = self._raw(x, p)
        if ld != p.cout:
            hidden = self.conv(x, prefix + ".net.0.proj")
        b, h, w, _ = hidden.shape
        gated = torch.empty((b, h, w, p.cout // 2), device=x.device, dtype=self.dtype)
        check(self.lib.osor_geglu(_ptr(hidden), _ptr(gated), b * h * w, p.cout // 2, self.dt,
                                  self.stream))
        return self.linear(gated, prefix + ".net.2", residual=residual)

    # -- layout
    def concat(self, a, b):
        y = torch.empty(a.shape[:3] + (a.shape[3] + b.shape[3],), device=a.device,
                        dtype=self.dtype)
        check(self.lib.osor_concat_channels(_ptr(a), a.shape[3], _ptr(b), b.shape[3], _ptr(y),
                                            a.shape[0] * a.shape[1] * a.shape[2], self.dt,
                                            self.stream))
        return y

    def resize(self, x, h, w):
        b, ih, iw, c = x.shape
        y = torch.empty((b, h, w, c), device=x.device, dtype=self.dtype)
        check(self.lib.osor_resize_nearest(_ptr(x), _ptr(y), b, ih, iw, h, w, c, self.dt,
                                           self.stream))
        return y

    # -- embeddings
    def _rows_linear(self, x, weight, bias, bias2, pre_silu):
        rows, in_f = x.shape
        out_f = weight.shape[0]
        y = torch.empty((rows, out_f), device=x.device, dtype=torch.float32)
        chunk = max(1, min(8, 12288 // in_f))
        for r0 in range(0, rows, chunk):
            r = min(chunk, rows - r0)
            check(self.lib.osor_rows_linear(_ptr(x, r0 * in_f), r, in_f, _ptr(weight),
                                            _ptr(bias), _ptr(bias2), out_f, pre_silu, self.dt,
                                            _ptr(y, r0 * out_f), self.stream))
        return y

    def embedding(self, batch: int, timestep: int, time_ids) -> torch.Tensor:
        arch = self.arch
        width = arch.base + arch.pooled + 6 * arch.time_projection
        feats = torch.empty((batch, width), device=self.device, dtype=torch.float32)
        check(self.lib.osor_unet_time_features(_ptr(time_ids), _ptr(self.pooled), batch,
                                               int(timestep), arch.base, arch.time_projection,
                                               arch.pooled, _ptr(feats), self.stream))
        hidden = self._rows_linear(feats, self.emb_w1, self.emb_b1, None, 0)
        return self._rows_linear(hidden, self.emb_w2, self.emb_b2[0], self.emb_b2[1], 1)

    def time_biases(self, temb: torch.Tensor) -> Dict[str, torch.Tensor]:
        tb = self._rows_linear(temb, self.temb_w, self.temb_b, None, 1)
        out, off = {}, 0
        for p in self.resnets:
            c = self.products[p + ".conv1"].cout
            out[p] = tb[:, off:off + c]
            off += c
        return out


class NativeUnet:
    """The SDXL inpainting UNet bound to a device, a dtype and the fixed prompt
    conditioning (``context`` [1, T, 2048], ``pooled`` [1, 1280]); callable as
    the pipeline's denoiser ``denoise(unet_input, timestep, time_ids)``
    (src/native.rs:503-519)."""

    def __init__(self, weights: Mapping[str, object], context, pooled,
                 arch: Optional[Architecture] = None, device: int = 0, dtype=torch.bfloat16,
                 graphs: bool = False):
        """``graphs``: replay each (batch, h, w, timestep) call as one CUDA graph
        captured on its first use (about 1,100 launches become one); the
        cancellation token is then polled before the call only, since a graph
        runs its blocks without returning to the host."""
        self.arch = arch or Architecture.sdxl()
        self.device = torch.device("cuda", device)
        if not torch.cuda.is_available():
            raise _lib.Unavailable("the native UNet needs a CUDA device")
        with torch.cuda.device(self.device):
            self.ops = CudaUnetOps(weights, self.arch, context, pooled, self.device, dtype)
        self.graph = UnetGraph(self.arch, self.ops)
        self.graphs = graphs
        self._captured: Dict[Tuple[int, int, int, int], tuple] = {}

    @classmethod
    def from_safetensors(cls, path: str, context, pooled, arch: Optional[Architecture] = None,
                         device: int = 0, dtype=torch.bfloat16, limits=None) -> "NativeUnet":
        """Load a bundle's `unet.safetensors` (diffusers names) with the
        reference's per-file checks (``artifact.read_safetensors``,
        src/artifact.rs:585-760) and build the UNet."""
        from .artifact import read_safetensors
        return cls(read_safetensors(path, limits), context, pooled, arch=arch, device=device,
                   dtype=dtype)

    def denoise(self, unet_input: torch.Tensor, timestep: int, time_ids: torch.Tensor,
                cancellation=None) -> torch.Tensor:
        def checkpoint():
            if cancellation is not None and cancellation.is_cancelled():
                raise _lib.Cancelled("inference was cancelled")

        if not torch.is_tensor(unet_input) or unet_input.ndim != 4:
            raise InvalidInput("UNet input must have shape [batch,9,height,width]")
        b, c, h, w = unet_input.shape
        if not (1 <= b <= MAX_BATCH and c == IN_CHANNELS and MIN_LATENT <= h <= MAX_LATENT
                and MIN_LATENT <= w <= MAX_LATENT):
            raise InvalidInput(f"UNet expects batch 1..={MAX_BATCH}, 9 channels and spatial "
                               f"dimensions {MIN_LATENT}..={MAX_LATENT}")
        if unet_input.dtype != torch.float32 or unet_input.device != self.device \
                or not unet_input.is_contiguous():
            raise InvalidInput("UNet input must be contiguous f32 on the model device")
        if not torch.is_tensor(time_ids) or tuple(time_ids.shape) != (b, 6) \
                or time_ids.device != self.device:
            raise InvalidInput("time_ids must have shape [batch, 6] on the UNet input device")
        if int(timestep) < 0:
            raise InvalidInput("timestep must be non-negative")
        ids = time_ids.to(torch.float32).contiguous()
        with torch.cuda.device(self.device):
            if not self.graphs:
                return self.graph.forward(unet_input, int(timestep), ids, checkpoint)
            checkpoint()
            key = (b, h, w, int(timestep))
            entry = self._captured.get(key)
            if entry is None:
                entry = self._capture(unet_input, int(timestep), ids)
                self._captured[key] = entry
            g, static_in, static_ids, static_out = entry
            static_in.copy_(unet_input)
            static_ids.copy_(ids)
            g.replay()
            return static_out.clone()

    def _capture(self, unet_input, timestep, ids):
        static_in, static_ids = unet_input.clone(), ids.clone()
        # One eager call on a side stream first, so that every lazy set-up
        # (kernel attributes, descriptors) happens outside the capture.
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.graph.forward(static_in, timestep, static_ids)
        torch.cuda.current_stream(self.device).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            static_out = self.graph.forward(static_in, timestep, static_ids)
        return g, static_in, static_ids, static_out

    __call__ = denoise


class UnetExecutor:
    """The UNet as one C-ABI handle (``osor_unet_create`` /
    ``osor_unet_denoise``): the C++ runtime a compiled host binds in place of
    NativeModel::denoise (src/native.rs:503-519). It runs the same kernels in
    the same order as ``NativeUnet`` and gives the same bits; activations come
    from a memory pool owned by the handle. Callable as the pipeline's
    denoiser."""

    def __init__(self, weights: Mapping[str, object], context, pooled,
                 arch: Optional[Architecture] = None, device: int = 0, dtype=torch.bfloat16):
        self.arch = arch or Architecture.sdxl()
        self.device = torch.device("cuda", device)
        if dtype not in HALF_TYPES:
            raise InvalidInput("UNet dtype must be bfloat16 or float16")
        arrays = {}
        for name, _ in unet_specs(self.arch):
            t = weights.get(name) if hasattr(weights, "get") else weights[name]
            if t is None:
                raise InvalidArtifact(f"native model tensor missing or incompatible: {name}")
            a = t.detach().to(torch.float32).cpu().numpy() if torch.is_tensor(t) else t
            arrays[name] = np.ascontiguousarray(a, np.float32)
        table = (_lib.OsorTensor * len(arrays))()
        names = []
        for i, (name, a) in enumerate(arrays.items()):
            if a.ndim > 4:
                raise InvalidArtifact(f"native model tensor missing or incompatible: {name}")
            names.append(name.encode())
            table[i].name = names[-1]
            table[i].data = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            table[i].ndim = a.ndim
            for d in range(4):
                table[i].shape[d] = a.shape[d] if d < a.ndim else 0
        ctx = torch.as_tensor(context).detach().to(torch.float32).cpu().numpy()
        pool = torch.as_tensor(pooled).detach().to(torch.float32).cpu().numpy()
        if ctx.ndim != 3 or ctx.shape[0] != 1 or ctx.shape[2] != self.arch.context \
                or pool.shape != (1, self.arch.pooled):
            raise InvalidInput(f"fixed conditioning must be [1, 1..=1024, {self.arch.context}] "
                               f"and [1, {self.arch.pooled}]")
        ctx = np.ascontiguousarray(ctx[0])
        pool = np.ascontiguousarray(pool[0])
        blocks = self.arch.blocks
        cfg = _lib.OsorUnetConfig()
        for i, blk in enumerate(blocks):
            cfg.channels[i] = blk.channels
            cfg.depth[i] = blk.depth or 0
            cfg.heads[i] = blk.heads
        cfg.context, cfg.pooled = self.arch.context, self.arch.pooled
        cfg.time_projection, cfg.layers = self.arch.time_projection, self.arch.layers
        cfg.dtype = dtype_code(dtype)
        handle = ctypes.c_void_p()
        check(_lib.lib().osor_unet_create(table, len(arrays), ctypes.byref(cfg),
                                          ctx.ctypes.data, ctx.shape[0], pool.ctypes.data,
                                          device, ctypes.byref(handle)))
        self._handle = handle

    def close(self) -> None:
        if getattr(self, "_handle", None):
            _lib.lib().osor_unet_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def denoise(self, unet_input: torch.Tensor, timestep: int, time_ids: torch.Tensor,
                cancellation=None) -> torch.Tensor:
        if not torch.is_tensor(unet_input) or unet_input.ndim != 4 \
                or unet_input.shape[1] != IN_CHANNELS:
            raise InvalidInput("UNet input must have shape [batch,9,height,width]")
        b, _, h, w = unet_input.shape
        if unet_input.dtype != torch.float32 or unet_input.device != self.device \
                or not unet_input.is_contiguous():
            raise InvalidInput("UNet input must be contiguous f32 on the model device")
        if not torch.is_tensor(time_ids) or tuple(time_ids.shape) != (b, 6) \
                or time_ids.device != self.device:
            raise InvalidInput("time_ids must have shape [batch, 6] on the UNet input device")
        ids = time_ids.to(torch.float32).contiguous()
        out = torch.empty((b, OUT_CHANNELS, h, w), dtype=torch.float32, device=self.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        flag = cancellation.pointer if cancellation is not None else None
        check(_lib.lib().osor_unet_denoise(self._handle, _ptr(unet_input), int(timestep),
                                           _ptr(ids), _ptr(out), b, h, w, stream, flag))
        return out

    __call__ = denoise
