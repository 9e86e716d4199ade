"""The UNet oracle against the reference's own UNet tests, restated.

Each test names the reference test (path:line inside the reference project)
whose inputs, formulas and bounds it restates. The reference holds no golden
tensors for its UNet; its tests pin exact values (the GEGLU gate), f64
agreement on dyadic inputs (attention, convolution) and properties of a
deterministic tiny model (shapes, use of every conditioning input, batch-entry
independence), and those are what pin this oracle.
"""
import math

import numpy as np
import pytest

from oracle import unet as U

GELU_TWO = 1.9544997215270996  # PyTorch F.gelu(2.0, approximate="none")


def test_sdxl_unet_inventory():
    """The SDXL inpainting UNet: 1680 tensors, 2.567 G parameters, nine input
    and five output channels (src/native.rs:70-97, 127-258)."""
    sp = U.specs(U.sdxl())
    names = [n for n, _ in sp]
    assert len(names) == len(set(names)) == 1680
    assert sum(int(np.prod(s)) for _, s in sp) == 2_567_480_965
    shapes = dict(sp)
    assert shapes["conv_in.weight"] == (320, 9, 3, 3)
    assert shapes["conv_out.weight"] == (5, 320, 3, 3)
    assert shapes["add_embedding.linear_1.weight"] == (1280, 1280 + 6 * 256)
    assert shapes["up_blocks.0.resnets.0.conv1.weight"] == (1280, 2560, 3, 3)
    assert shapes["up_blocks.0.resnets.2.conv_shortcut.weight"] == (1280, 1920, 1, 1)
    assert shapes["up_blocks.2.resnets.0.norm1.weight"] == (960,)
    assert shapes["down_blocks.2.attentions.1.transformer_blocks.9.attn2.to_k.weight"] == (1280, 2048)
    assert shapes["mid_block.attentions.0.transformer_blocks.9.ff.net.0.proj.weight"] == (10240, 1280)
    assert "down_blocks.2.downsamplers.0.conv.weight" not in shapes
    assert "up_blocks.2.upsamplers.0.conv.weight" not in shapes


def test_geglu_matches_pytorch_gate_two():
    """src/native/transformer.rs:31-58: zero input, gate bias 2, value bias 1."""
    w = {
        "ff.net.0.proj.weight": np.zeros((8, 1), np.float32),
        "ff.net.0.proj.bias": np.array([1, 0, 0, 0, 2, 0, 0, 0], np.float32),
        "ff.net.2.weight": np.array([[1, 0, 0, 0]], np.float32),
        "ff.net.2.bias": np.zeros(1, np.float32),
    }
    out = U.feed_forward(w, "ff", np.zeros((1, 1, 1), np.float32))
    assert abs(float(out.sum()) - GELU_TWO) < 1e-6


def test_spatial_transformer_uses_exact_geglu():
    """src/native/spatial.rs:414-486: all-zero weights except proj_out = I and
    the GEGLU biases / output column; zero input [1, 32, 1, 1]."""
    arch = U.Arch((U.Block(32, None, 1), U.Block(32, 1, 1), U.Block(32, 1, 1)),
                  context=8, pooled=8, time_projection=8, layers=1)
    prefix = "down_blocks.1.attentions.0"
    w = {n: np.zeros(s, np.float32) for n, s in U.specs(arch) if n.startswith(prefix)}
    w[prefix + ".proj_out.weight"] = np.eye(32, dtype=np.float32)
    bias = np.zeros(256, np.float32)
    bias[0], bias[128] = 1.0, 2.0
    t = prefix + ".transformer_blocks.0"
    w[t + ".ff.net.0.proj.bias"] = bias
    out_w = np.zeros((32, 128), np.float32)
    out_w[0, 0] = 1.0
    w[t + ".ff.net.2.weight"] = out_w
    context = np.zeros((1, 1, 8), np.float32)
    out = U.spatial_transformer(w, prefix, np.zeros((1, 32, 1, 1), np.float32), 1, 1, context)
    assert abs(float(out.sum()) - GELU_TWO) < 1e-6


def _values(count, salt):
    i = np.arange(count)
    return ((((i * 7 + salt) % 11) - 5) / 16.0).astype(np.float32)


def _attention_f64(w, prefix, x, context, heads):
    def project(name, xs):
        y = xs.astype(np.float64) @ w[f"{prefix}.{name}.weight"].astype(np.float64).T
        b = w.get(f"{prefix}.{name}.bias")
        return y if b is None else y + b.astype(np.float64)

    def split(t):
        b, n, c = t.shape
        return t.reshape(b, n, heads, c // heads).transpose(0, 2, 1, 3)

    q, k, v = split(project("to_q", x)), split(project("to_k", context)), split(project("to_v", context))
    s = q @ k.transpose(0, 1, 3, 2) / math.sqrt(q.shape[-1])
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    o = (p @ v).transpose(0, 2, 1, 3)
    return project("to_out.0", o.reshape(o.shape[0], o.shape[1], -1))


@pytest.mark.parametrize("batch", [1, 2])
def test_cached_and_self_attention_match_f64(batch):
    """src/native/spatial.rs:325-412: dyadic weights, 16 channels, 4 heads,
    context width 12 with 5 tokens, 7 query tokens; within 1e-5 of f64."""
    channels, heads, width = 16, 4, 12
    w = {}
    for prefix, cw in (("cross", width), ("self", channels)):
        for index, (name, iw) in enumerate((("to_q", channels), ("to_k", cw), ("to_v", cw),
                                           ("to_out.0", channels))):
            w[f"{prefix}.{name}.weight"] = _values(channels * iw, index).reshape(channels, iw)
        w[f"{prefix}.to_out.0.bias"] = _values(channels, 3)
    context = _values(5 * width, 5).reshape(1, 5, width)
    xs = _values(batch * 7 * channels, 2).reshape(batch, 7, channels)
    cross = U.attention(w, "cross", xs, heads, context=context)
    own = U.attention(w, "self", xs, heads)
    ref_cross = _attention_f64(w, "cross", xs, np.repeat(context, batch, 0), heads)
    ref_self = _attention_f64(w, "self", xs, xs, heads)
    assert np.abs(cross - ref_cross).max() <= 1e-5
    assert np.abs(own - ref_self).max() <= 1e-5


def _conv_f64(x, w, b, stride, pad):
    x, w = x.astype(np.float64), w.astype(np.float64)
    bs, ci, h, wd = x.shape
    co, _, k, _ = w.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    oh, ow = (h + 2 * pad - k) // stride + 1, (wd + 2 * pad - k) // stride + 1
    y = np.zeros((bs, co, oh, ow))
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, :, ky:ky + stride * oh:stride, kx:kx + stride * ow:stride]
            y += np.einsum("bchw,oc->bohw", patch, w[:, :, ky, kx])
    return y + b.astype(np.float64)[None, :, None, None]


@pytest.mark.parametrize("shape", [(1, 9, 5, 7, 5, 3, 1, 1), (2, 4, 7, 5, 3, 3, 2, 1),
                                   (2, 6, 5, 7, 5, 1, 1, 0)])
def test_unet_convolution_matches_f64(shape):
    """src/native/unet_conv.rs:76-138: strided, sampling and 1x1 shortcut
    shapes, input given transposed; within 2e-5 of f64."""
    batch, channels, height, width, outputs, k, stride, pad = shape

    def values(count, seed):
        i = np.arange(count)
        return ((((i * 41 + seed) % 101) - 50) / 53.0).astype(np.float32)

    x = values(batch * channels * height * width, 9).reshape(batch, channels, width, height)
    x = np.ascontiguousarray(x.transpose(0, 1, 3, 2))
    w = {"c.weight": values(outputs * channels * k * k, 7).reshape(outputs, channels, k, k),
         "c.bias": values(outputs, 31)}
    y = U.conv(w, "c", x, stride=stride, padding=pad)
    ref = _conv_f64(x, w["c.weight"], w["c.bias"], stride, pad)
    assert y.shape == ref.shape
    assert np.abs(y - ref).max() <= 2e-5


@pytest.mark.parametrize("batch", [1, 2])
def test_unet_input_convolution_tracks_f64(batch):
    """src/native.rs:669-710: 9 -> 64 input convolution on [B, 9, 5, 7]."""
    def values(count, mul, mod):
        i = np.arange(count)
        return (((i * mul % mod) - mod // 2) / 37.0).astype(np.float32)

    w = {"conv_in.weight": values(64 * 9 * 9, 61, 101).reshape(64, 9, 3, 3),
         "conv_in.bias": np.zeros(64, np.float32)}
    x = values(batch * 9 * 5 * 7, 43, 103).reshape(batch, 9, 5, 7)
    y = U.conv(w, "conv_in", x)
    assert np.abs(y - _conv_f64(x, w["conv_in.weight"], w["conv_in.bias"], 1, 1)).max() <= 6.2e-6


@pytest.fixture(scope="module")
def tiny():
    arch = U.tiny()
    w = U.deterministic_weights(arch)
    seq = U.fixed_values(2 * 8, 1).reshape(1, 2, 8)
    pooled = U.fixed_values(8, 2).reshape(1, 8)
    return arch, w, seq, pooled


def _differs(a, b):
    return float(np.abs(a - b).max()) > 1e-7


def test_tiny_graph_uses_all_conditioning_and_preserves_shapes(tiny):
    """src/native.rs:773-843 (UNet part)."""
    arch, w, seq, pooled = tiny
    x = U.fixed_values(9 * 4 * 4, 5).reshape(1, 9, 4, 4)
    ids = np.array([[32, 32, 0, 0, 32, 32]], np.float32)
    out = U.forward(w, arch, x, 400, ids, seq, pooled)
    assert out.shape == (1, 5, 4, 4)
    assert _differs(out, U.forward(w, arch, x, 401, ids, seq, pooled))
    assert _differs(out, U.forward(w, arch, x, 400, ids + 1, seq, pooled))
    assert not _differs(out, U.forward(w, arch, x, 400, ids, seq, pooled))
    assert _differs(out, U.forward(w, arch, x, 400, ids, seq * 2, pooled))
    assert _differs(out, U.forward(w, arch, x, 400, ids, seq, pooled * 2))


def test_tiny_graph_batch_entries_are_independent(tiny):
    """src/native.rs:814-842: two distinct 8x8 entries, both orders, each
    batched entry within 1e-5 of its single run."""
    arch, w, seq, pooled = tiny
    first_in = U.fixed_values(9 * 8 * 8, 5).reshape(1, 9, 8, 8)
    second_in = U.fixed_values(9 * 8 * 8, 6).reshape(1, 9, 8, 8)
    ids = np.array([[64, 64, 0, 0, 64, 64]], np.float32)
    first = U.forward(w, arch, first_in, 400, ids, seq, pooled)
    second = U.forward(w, arch, second_in, 400, ids, seq, pooled)
    assert float(np.abs(first - second).max()) > 1e-3
    for entries in ([(first_in, first), (second_in, second)],
                    [(second_in, second), (first_in, first)]):
        batch = np.concatenate([e[0] for e in entries])
        out = U.forward(w, arch, batch, 400, np.repeat(ids, 2, 0), seq, pooled)
        assert out.shape == (2, 5, 8, 8)
        for i, (_, expected) in enumerate(entries):
            assert float(np.abs(out[i] - expected[0]).max()) <= 1e-5


def test_tiny_graph_preserves_nonsquare_odd_latent_shape(tiny):
    """src/native.rs:896-909: a 5 x 7 latent (downsampled 3 x 4, 2 x 2 and
    upsampled back to the skip sizes)."""
    arch, w, seq, pooled = tiny
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 9, 5, 7)).astype(np.float32)
    ids = np.array([[40, 56, 0, 0, 40, 56]], np.float32)
    assert U.forward(w, arch, x, 400, ids, seq, pooled).shape == (1, 5, 5, 7)


def test_forward_reads_every_tensor(tiny):
    arch, w, seq, pooled = tiny

    class Recording(dict):
        def __init__(self, d):
            super().__init__(d)
            self.read = set()

        def __getitem__(self, k):
            self.read.add(k)
            return super().__getitem__(k)

        def get(self, k, default=None):
            if k in self:
                self.read.add(k)
            return super().get(k, default)

    rec = Recording(w)
    U.forward(rec, arch, U.fixed_values(9 * 4 * 4, 5).reshape(1, 9, 4, 4), 400,
              np.array([[32, 32, 0, 0, 32, 32]], np.float32), seq, pooled)
    assert rec.read == set(w)


def test_nearest_upsample_to_odd_sizes():
    """upsample_nearest2d to a size that is not a multiple of the input: the
    up blocks take the next skip's size (src/native.rs:356-367)."""
    x = np.arange(2 * 3, dtype=np.float32).reshape(1, 1, 2, 3)
    y = U.upsample_nearest(x, 3, 5)
    # rows floor(i * 2/3) = 0, 0, 1; columns floor(j * 3/5) = 0, 0, 1, 1, 2
    assert y[0, 0].tolist() == [[0, 0, 1, 1, 2], [0, 0, 1, 1, 2], [3, 3, 4, 4, 5]]
    assert np.array_equal(U.upsample_nearest(x, 4, 6)[0, 0, ::2, ::2], x[0, 0])


def test_timestep_projection_layout():
    """flip_sin_to_cos puts the cosines first; frequencies 1e4^(-i/half)."""
    e = U.timesteps(np.array([0.0, 400.0], np.float32), 8)
    assert e.shape == (2, 8)
    assert np.allclose(e[0], [1, 1, 1, 1, 0, 0, 0, 0])
    freq = 10000.0 ** (-np.arange(4) / 4.0)
    assert np.allclose(e[1, :4], np.cos(400 * freq), atol=2e-4)
    assert np.allclose(e[1, 4:], np.sin(400 * freq), atol=2e-4)
