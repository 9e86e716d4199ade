"""Host side of the UNet on CPU: the product's tensor inventory against the
oracle's, and the product's block topology (``UnetGraph``, the code that runs
on the GPU) driven by numpy ops built from the oracle, against the oracle's
own restatement of Unet::forward."""
import numpy as np
import pytest
import torch

from oracle import unet as U
from osor_b200 import _lib
from osor_b200.unet import (Architecture, BlockSpec, NativeUnet, UnetExecutor, UnetGraph,
                            random_unet_weights, resnet_prefixes, unet_specs)


def _oracle_arch(arch: Architecture) -> U.Arch:
    return U.Arch(tuple(U.Block(b.channels, b.depth, b.heads) for b in arch.blocks),
                  arch.context, arch.pooled, arch.time_projection, arch.layers)


def _nchw(x):
    return np.ascontiguousarray(x.transpose(0, 3, 1, 2))


def _nhwc(x):
    return np.ascontiguousarray(x.transpose(0, 2, 3, 1))


class OracleOps:
    """UnetGraph's ops on numpy NHWC arrays, each computed by the oracle."""

    def __init__(self, w, arch, context, pooled):
        self.w, self.arch, self.ctx, self.pooled = w, arch, context, pooled

    def has(self, name):
        return name + ".weight" in self.w

    def conv(self, x, name, stride=1, residual=None, image_bias=None):
        if self.w[name + ".weight"].ndim == 2:
            y = U.linear(self.w, name, x)
        else:
            y = _nhwc(U.conv(self.w, name, _nchw(x), stride=stride))
        if image_bias is not None:
            y = y + image_bias[:, None, None, :]
        return y if residual is None else y + residual

    linear = conv

    def conv_in(self, sample):
        return _nhwc(U.conv(self.w, "conv_in", sample))

    def conv_out(self, x):
        return U.conv(self.w, "conv_out", _nchw(x))

    def group_norm(self, x, name, eps, silu):
        return _nhwc(U.gn(self.w, name, _nchw(x), eps, silu))

    def layer_norm(self, x, name):
        return U.layer_norm(self.w, name, x)

    def self_attention(self, x, prefix, heads, residual):
        b, h, w, c = x.shape
        return residual + U.attention(self.w, prefix, x.reshape(b, h * w, c), heads).reshape(x.shape)

    def cross_attention(self, x, prefix, heads, residual):
        b, h, w, c = x.shape
        out = U.attention(self.w, prefix, x.reshape(b, h * w, c), heads, context=self.ctx)
        return residual + out.reshape(x.shape)

    def feed_forward(self, x, prefix, residual):
        return residual + U.feed_forward(self.w, prefix, x)

    def concat(self, a, b):
        return np.concatenate([a, b], axis=-1)

    def resize(self, x, h, w):
        return _nhwc(U.upsample_nearest(_nchw(x), h, w))

    def embedding(self, batch, timestep, time_ids):
        return U.embedding(self.w, self.arch, batch, timestep, time_ids, self.pooled)

    def time_biases(self, temb):
        return {p: U.linear(self.w, p + ".time_emb_proj", U.silu(temb))
                for p in resnet_prefixes(self.arch)}


@pytest.mark.parametrize("arch", [Architecture.sdxl(), Architecture.tiny()])
def test_inventory_matches_oracle(arch):
    assert unet_specs(arch) == U.specs(_oracle_arch(arch))


def test_resnet_prefixes_cover_every_time_projection():
    arch = Architecture.sdxl()
    names = {n[:-len(".time_emb_proj.weight")] for n, _ in unet_specs(arch)
             if n.endswith(".time_emb_proj.weight")}
    assert sorted(resnet_prefixes(arch)) == sorted(names)
    assert len(resnet_prefixes(arch)) == 6 + 2 + 9


def test_random_weights_follow_the_init_hints():
    arch = Architecture.tiny()
    w = random_unet_weights(arch, seed=3)
    assert {n: tuple(t.shape) for n, t in w.items()} == dict(unet_specs(arch))
    assert torch.equal(w["conv_norm_out.weight"], torch.ones(64))
    assert torch.equal(w["mid_block.attentions.0.transformer_blocks.0.norm2.bias"], torch.zeros(64))
    conv = w["down_blocks.0.resnets.0.conv1.weight"]
    assert abs(conv.std().item() - (2.0 / (64 * 9)) ** 0.5) < 0.01
    bound = 1.0 / (64 * 9) ** 0.5
    assert w["down_blocks.0.resnets.0.conv1.bias"].abs().max().item() <= bound
    assert torch.equal(w["conv_in.weight"], random_unet_weights(arch, seed=3)["conv_in.weight"])


@pytest.fixture(scope="module")
def tiny():
    arch = Architecture.tiny()
    oarch = _oracle_arch(arch)
    w = U.deterministic_weights(oarch)
    seq = U.fixed_values(2 * 8, 1).reshape(1, 2, 8)
    pooled = U.fixed_values(8, 2).reshape(1, 8)
    return arch, oarch, w, seq, pooled


@pytest.mark.parametrize("batch,h,w", [(1, 4, 4), (2, 8, 8), (1, 5, 7)])
def test_graph_topology_matches_oracle_forward(tiny, batch, h, w):
    arch, oarch, weights, seq, pooled = tiny
    rng = np.random.default_rng(h * 10 + w)
    x = rng.standard_normal((batch, 9, h, w)).astype(np.float32)
    ids = np.tile(np.array([[8 * h, 8 * w, 0, 0, 8 * h, 8 * w]], np.float32), (batch, 1))
    graph = UnetGraph(arch, OracleOps(weights, arch, seq, pooled))
    calls = []
    out = graph.forward(x, 400, ids, checkpoint=lambda: calls.append(1))
    ref = U.forward(weights, oarch, x, 400, ids, seq, pooled)
    assert out.shape == ref.shape == (batch, 5, h, w)
    scale = float(np.abs(ref).max())
    assert float(np.abs(out - ref).max()) <= 1e-4 * max(scale, 1.0)
    # Cancellation checkpoints between the blocks (src/native.rs:345-372).
    assert len(calls) >= 7


def test_graph_topology_with_two_layers_and_cross_depth_two():
    """SDXL's block counts (two layers, three per up block, transformer depth
    2) at small widths."""
    arch = Architecture((BlockSpec(32, None, 1), BlockSpec(64, 2, 2), BlockSpec(64, 1, 2)),
                        context=16, pooled=8, time_projection=8, layers=2)
    oarch = _oracle_arch(arch)
    weights = U.deterministic_weights(oarch)
    rng = np.random.default_rng(5)
    seq = rng.standard_normal((1, 3, 16)).astype(np.float32)
    pooled = rng.standard_normal((1, 8)).astype(np.float32)
    x = rng.standard_normal((2, 9, 6, 5)).astype(np.float32)
    ids = np.array([[48, 40, 0, 0, 48, 40]] * 2, np.float32)
    out = UnetGraph(arch, OracleOps(weights, arch, seq, pooled)).forward(x, 400, ids)
    ref = U.forward(weights, oarch, x, 400, ids, seq, pooled)
    assert float(np.abs(out - ref).max()) <= 1e-4 * max(float(np.abs(ref).max()), 1.0)


def test_graph_cancellation_stops_between_blocks(tiny):
    arch, _, weights, seq, pooled = tiny
    graph = UnetGraph(arch, OracleOps(weights, arch, seq, pooled))
    calls = []

    def cancel_second():
        calls.append(1)
        if len(calls) >= 2:
            raise _lib.Cancelled("inference was cancelled")

    with pytest.raises(_lib.Cancelled):
        graph.forward(np.zeros((1, 9, 4, 4), np.float32), 400,
                      np.array([[32, 32, 0, 0, 32, 32]], np.float32), cancel_second)
    assert len(calls) == 2


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the CPU-only refusal")
def test_native_unet_requires_a_cuda_device():
    arch = Architecture.tiny()
    with pytest.raises(_lib.Unavailable):
        NativeUnet(random_unet_weights(arch), np.zeros((1, 2, 8), np.float32),
                   np.zeros((1, 8), np.float32), arch=arch)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the CPU-only refusal")
def test_native_runtime_handle_requires_a_cuda_device():
    """The wrapper marshals every tensor and the configuration into the C ABI,
    which refuses without an sm_100 device."""
    arch = Architecture.tiny()
    with pytest.raises(_lib.Unavailable):
        UnetExecutor(random_unet_weights(arch), np.zeros((1, 2, 8), np.float32),
                     np.zeros((1, 8), np.float32), arch=arch)
    with pytest.raises(_lib.InvalidInput):  # prompt width does not match the architecture
        UnetExecutor(random_unet_weights(arch), np.zeros((1, 2, 4), np.float32),
                     np.zeros((1, 8), np.float32), arch=arch)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_fused_geglu_rounding_is_no_worse_than_the_stored_projection(dt):
    """The fused GEGLU product rounds the value half to 16 bits (as a stored
    projection would be) but gates with the f32 accumulator, where the unfused
    path also rounds the gate before gelu_erf. A CPU emulation of both on the
    same 16-bit operands: against the f64 result the fused rounding is never
    worse than the stored projection's (transformer.rs:18-24)."""
    rng = np.random.default_rng(21)
    rows, cin, f = 512, 320, 256
    q = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(dt).float().numpy()  # noqa: E731
    x = q(rng.standard_normal((rows, cin)))
    w = q(rng.standard_normal((2 * f, cin)) / np.sqrt(cin))
    proj = x.astype(np.float64) @ w.astype(np.float64).T
    value, gate = proj[:, :f], proj[:, f:]
    exact = value * U.gelu_erf(gate).astype(np.float64)
    acc = proj.astype(np.float32)  # the f32 accumulator
    unfused = q(q(acc[:, :f]) * U.gelu_erf(q(acc[:, f:])))
    fused = q(q(acc[:, :f]) * U.gelu_erf(acc[:, f:]))
    err_unfused = np.abs(unfused - exact).max()
    err_fused = np.abs(fused - exact).max()
    assert err_fused <= err_unfused * 1.001 + 1e-7, (err_fused, err_unfused)
