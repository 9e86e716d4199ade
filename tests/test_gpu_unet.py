"""SDXL UNet on the GPU against the oracle.

Op level: the UNet kernels of libosor_b200 (time features, row linear,
LayerNorm, GEGLU, the fused GEGLU product, conv_in's column matrix,
multi-head attention, concatenation, nearest resize, channel update,
wide-channel GroupNorm, the zero-padded 320-channel convolution) against
numpy / float64 restatements on the same 16-bit inputs. Model level:
``NativeUnet`` against ``oracle.unet.forward`` for the reference's tiny test
model (deterministic weights) and for a one-layer model with SDXL's widths
(320 / 640 / 1280 channels, 5 / 10 / 20 heads, 2560-channel skip
concatenations). Tolerances: a CPU emulation that rounds every op output and
weight to the model dtype gives relative L2 errors of 1-2e-3 (f16) and 1-2e-2
(bf16) for these models; the bounds below leave a factor of 3-5.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import unet as U
from osor_b200 import _lib
from osor_b200._lib import InvalidInput, check, dtype_code
from osor_b200.unet import (Architecture, BlockSpec, NativeUnet, UnetExecutor,
                            random_unet_weights)

pytestmark = pytest.mark.gpu


def P(t, off=0):
    return ctypes.c_void_p(t.data_ptr() + off * t.element_size())


def S():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dev16(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt).cuda()


def host(t):
    return t.float().cpu().numpy()


# ---------------------------------------------------------------- op level
def test_time_features_match_oracle(cuda_device):
    lb = _lib.lib()
    ids = np.array([[1024, 768, 0, 0, 1024, 768], [64, 40, 3, 5, 64, 40]], np.float32)
    pooled = np.linspace(-1, 1, 24).astype(np.float32)
    base, tp = 320, 16
    out = torch.empty((2, base + 24 + 6 * tp), device="cuda")
    # Device copies are held in locals until the launch is enqueued.
    ids_d, pooled_d = torch.from_numpy(ids).cuda(), torch.from_numpy(pooled).cuda()
    check(lb.osor_unet_time_features(P(ids_d), P(pooled_d), 2, 999, base, tp, 24, P(out), S()))
    got = host(out)
    want_t = U.timesteps(np.full(2, 999, np.float32), base)
    want_ids = U.timesteps(ids.reshape(-1), tp).reshape(2, 6 * tp)
    assert np.abs(got[:, :base] - want_t).max() < 2e-4
    assert np.array_equal(got[:, base:base + 24], np.tile(pooled, (2, 1)))
    assert np.abs(got[:, base + 24:] - want_ids).max() < 2e-4


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,in_f,out_f,silu", [(4, 3136 // 2, 77, 0), (3, 100, 40, 1),
                                                   (1, 1280, 300, 1)])
def test_rows_linear_matches_f64(dt, rows, in_f, out_f, silu, cuda_device):
    rng = np.random.default_rng(rows * in_f)
    x = rng.standard_normal((rows, in_f)).astype(np.float32)
    w16 = dev16(rng.standard_normal((out_f, in_f)) / math.sqrt(in_f), dt)
    b1 = rng.standard_normal(out_f).astype(np.float32)
    b2 = rng.standard_normal(out_f).astype(np.float32)
    y = torch.empty((rows, out_f), device="cuda")
    x_d, b1_d, b2_d = (torch.from_numpy(a).cuda() for a in (x, b1, b2))
    check(_lib.lib().osor_rows_linear(P(x_d), rows, in_f, P(w16), P(b1_d), P(b2_d), out_f, silu,
                                      dtype_code(dt), P(y), S()))
    xa = x.astype(np.float64)
    if silu:
        xa = xa / (1 + np.exp(-xa))
    want = xa @ host(w16).astype(np.float64).T + b1 + b2
    assert np.abs(host(y) - want).max() < 1e-4 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("channels", [64, 640, 1280, 2048])
def test_layer_norm_matches_f64(channels, cuda_device):
    rng = np.random.default_rng(channels)
    x = dev16(rng.standard_normal((37, channels)) * 3 + 1, torch.float16)
    g = torch.from_numpy(rng.standard_normal(channels).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(channels).astype(np.float32)).cuda()
    y = torch.empty_like(x)
    check(_lib.lib().osor_layer_norm(P(x), P(y), P(g), P(b), 37, channels, 1e-5,
                                     dtype_code(torch.float16), S()))
    xa = host(x).astype(np.float64)
    m = xa.mean(-1, keepdims=True)
    v = ((xa - m) ** 2).mean(-1, keepdims=True)
    want = (xa - m) / np.sqrt(v + 1e-5) * host(g) + host(b)
    assert np.abs(host(y) - want).max() < 4e-3 * max(1.0, np.abs(want).max())


def test_geglu_matches_exact_erf(cuda_device):
    rng = np.random.default_rng(4)
    x = dev16(rng.standard_normal((50, 2 * 136)) * 2, torch.float16)
    y = torch.empty((50, 136), device="cuda", dtype=torch.float16)
    check(_lib.lib().osor_geglu(P(x), P(y), 50, 136, dtype_code(torch.float16), S()))
    xa = host(x)
    want = xa[:, :136] * U.gelu_erf(xa[:, 136:])
    assert np.abs(host(y) - want).max() < 5e-3 * max(1.0, np.abs(want).max())
    # The reference's pinned value: gelu(2) with value 1.
    one = torch.tensor([[1.0] * 8 + [2.0] * 8], device="cuda", dtype=torch.float32).to(torch.float16)
    out = torch.empty((1, 8), device="cuda", dtype=torch.float16)
    check(_lib.lib().osor_geglu(P(one), P(out), 1, 8, dtype_code(torch.float16), S()))
    assert abs(float(out[0, 0]) - 1.9544997215270996) < 1e-3


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_thin_columns_match_im2col(dt, cuda_device):
    """osor_thin_columns: the UNet conv_in's 3 x 3 x 9 column matrix over 128
    columns, tap-major then channel, zero outside the image and past 81."""
    rng = np.random.default_rng(12)
    b, c, h, w = 2, 9, 5, 7
    x = torch.from_numpy(rng.standard_normal((b, c, h, w)).astype(np.float32)).cuda()
    cols = torch.full((b, h, w, 128), 7.0, device="cuda", dtype=dt)
    check(_lib.lib().osor_thin_columns(P(x), P(cols), b, c, h, w, 3, 1, 128, dtype_code(dt), S()))
    xp = np.pad(host(x.to(dt)), ((0, 0), (0, 0), (1, 1), (1, 1)))
    want = np.zeros((b, h, w, 128), np.float32)
    for ky in range(3):
        for kx in range(3):
            t = ky * 3 + kx
            want[..., t * c:(t + 1) * c] = xp[:, :, ky:ky + h, kx:kx + w].transpose(0, 2, 3, 1)
    np.testing.assert_array_equal(host(cols), want)
    with pytest.raises(InvalidInput):
        check(_lib.lib().osor_thin_columns(P(x), P(cols), b, c, h, w, 3, 1, 64, dtype_code(dt),
                                           S()))


# (batch, h, w, cin, features, fused): 2048 pixels (16 tiles) on CTA pairs
# with the gate in the product's epilogue; 384 pixels (3 tiles, odd) through
# the workspace (product, then the interleaved GEGLU pass).
@pytest.mark.parametrize("shape", [(2, 16, 64, 256, 256, True), (1, 3, 128, 128, 128, False)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_linear_geglu_matches_f64(shape, dt, cuda_device):
    """osor_linear_geglu against the projection and exact-erf gate in f64 on
    the same 16-bit operands (transformer.rs:18-24)."""
    b, h, w, cin, f, fused = shape
    rng = np.random.default_rng(11)
    x = dev16(rng.standard_normal((b, h, w, cin)), dt)
    wt = dev16(rng.standard_normal((2 * f, cin)) / np.sqrt(cin), dt)
    bias = torch.from_numpy(rng.uniform(-0.2, 0.2, 2 * f).astype(np.float32)).cuda()
    r = np.arange(2 * f)
    order = np.where(r % 256 < 128, (r // 256) * 128 + r % 256, f + (r // 256) * 128 + r % 256 - 128)
    order_t = torch.from_numpy(order).cuda()
    wi = wt[order_t].contiguous()
    bi = bias[order_t].contiguous()
    need = _lib.lib().osor_linear_geglu_workspace_size(b, h, w, cin, f, dtype_code(dt))
    assert (need == 0) == fused
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    y = torch.empty((b, h, w, f), device="cuda", dtype=dt)
    check(_lib.lib().osor_linear_geglu(P(x), P(y), P(wi), P(bi), b, h, w, cin, f, dtype_code(dt),
                                       P(ws), need, S()))
    proj = host(x).reshape(-1, cin).astype(np.float64) @ host(wt).astype(np.float64).T
    proj += host(bias)
    want = proj[:, :f] * U.gelu_erf(proj[:, f:])
    got = host(y).reshape(-1, f)
    # The unfused path rounds the projection to 16 bits before the gate.
    assert np.all(np.abs(got - want) <= 2e-2 * np.abs(want) + 2e-2), np.abs(got - want).max()
    if not fused:
        with pytest.raises(InvalidInput):
            check(_lib.lib().osor_linear_geglu(P(x), P(y), P(wi), P(bi), b, h, w, cin, f,
                                               dtype_code(dt), None, 0, S()))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_concat_resize_and_channel_update_are_exact(dt, cuda_device):
    lb = _lib.lib()
    rng = np.random.default_rng(9)
    a = dev16(rng.standard_normal((2, 3, 5, 16)), dt)
    b = dev16(rng.standard_normal((2, 3, 5, 24)), dt)
    y = torch.empty((2, 3, 5, 40), device="cuda", dtype=dt)
    check(lb.osor_concat_channels(P(a), 16, P(b), 24, P(y), 30, dtype_code(dt), S()))
    assert torch.equal(y, torch.cat([a, b], -1))
    for oh, ow in ((6, 10), (5, 9), (3, 5), (7, 11)):
        r = torch.empty((2, oh, ow, 16), device="cuda", dtype=dt)
        check(lb.osor_resize_nearest(P(a), P(r), 2, 3, 5, oh, ow, 16, dtype_code(dt), S()))
        sy = np.minimum(2, (np.arange(oh) * (3 / oh)).astype(np.int64))
        sx = np.minimum(4, (np.arange(ow) * (5 / ow)).astype(np.int64))
        assert torch.equal(r, a[:, torch.from_numpy(sy).cuda()][:, :, torch.from_numpy(sx).cuda()])
    # Narrow a 48-wide product to 40 channels, add a per-image bias (row
    # stride 56) and a residual; then the same in place.
    x = dev16(rng.standard_normal((2, 15, 48)), dt)
    bias = torch.from_numpy(rng.standard_normal((2, 56)).astype(np.float32)).cuda()
    res = dev16(rng.standard_normal((2, 15, 40)), dt)
    out = torch.empty((2, 15, 40), device="cuda", dtype=dt)
    check(lb.osor_channel_update(P(x), 48, P(out), 40, 2, 15, P(bias, 8), 56, P(res),
                                 dtype_code(dt), S()))
    want = ((x[..., :40].float() + bias[:, None, 8:48]) + res.float()).to(dt)
    assert torch.equal(out, want)
    inplace = res.clone()
    check(lb.osor_channel_update(P(inplace), 40, P(inplace), 40, 2, 15, P(bias), 56, None,
                                 dtype_code(dt), S()))
    assert torch.equal(inplace, (res.float() + bias[:, None, :40]).to(dt))
    with pytest.raises(InvalidInput):
        check(lb.osor_channel_update(P(x), 48, P(x), 40, 2, 15, None, 0, None, dtype_code(dt), S()))


def _attention_f64(q, k, v, heads, hd):
    b, n, _ = q.shape
    m = k.shape[1]
    qh = q.reshape(b, n, heads, hd).transpose(0, 2, 1, 3)
    kh = k.reshape(k.shape[0], m, heads, hd).transpose(0, 2, 1, 3)
    vh = v.reshape(v.shape[0], m, heads, hd).transpose(0, 2, 1, 3)
    s = qh @ kh.transpose(0, 1, 3, 2)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return (p @ vh).transpose(0, 2, 1, 3).reshape(b, n, heads * hd)


# Head width 64 with n_q a multiple of 256 runs on the tcgen05 kernel
# (attn_heads.cu): one 128-key tile, ragged last tiles, shared cross-attention
# keys, and more tasks (batch x heads x 256-row tiles) than SMs so that CTAs
# take several in turn. The other shapes run on the mma.sync / CUDA-core
# kernels.
HEAD_CASES = [(64, 5, 70, 77, True), (64, 10, 256, 256, False), (64, 10, 512, 77, True),
              (64, 4, 1024, 1000, False), (64, 20, 2048, 300, False), (32, 2, 33, 300, False),
              (128, 3, 19, 40, True)]


@pytest.mark.parametrize("hd,heads,n_q,n_kv,shared", HEAD_CASES)
def test_attention_heads_match_f64(hd, heads, n_q, n_kv, shared, cuda_device):
    lb = _lib.lib()
    rng = np.random.default_rng(hd + n_q)
    b, c = 2, heads * hd
    ld_q, ld_kv, ld_out = c + 8, 2 * c + 16, c  # q rows padded; k | v interleaved per row
    q = dev16(rng.standard_normal((b, n_q, ld_q)) / math.sqrt(hd), torch.float16)
    kvb = 1 if shared else b
    kv = dev16(rng.standard_normal((kvb, n_kv, ld_kv)), torch.float16)
    out = torch.zeros((b, n_q, ld_out), device="cuda", dtype=torch.float16)
    check(lb.osor_attention_heads(P(q), ld_q, n_q * ld_q, P(kv), P(kv, c), ld_kv,
                                  0 if shared else n_kv * ld_kv, P(out), ld_out, n_q * ld_out, b,
                                  heads, n_q, n_kv, hd, dtype_code(torch.float16), S()))
    qa, kva = host(q).astype(np.float64), host(kv).astype(np.float64)
    k, v = kva[..., :c], kva[..., c:2 * c]
    if shared:
        k, v = np.repeat(k, b, 0), np.repeat(v, b, 0)
    want = _attention_f64(qa[..., :c], k, v, heads, hd)
    # f16 output rounding (2^-11 relative) plus f32 softmax arithmetic.
    assert np.all(np.abs(host(out) - want) <= 1e-3 + 1e-3 * np.abs(want))


def test_attention_heads_rescales_growing_maxima(cuda_device):
    """Logits that grow along the keys (to about 40 over 1000 keys) move the
    running row maximum past the 2^8 rescale threshold several times; the
    tcgen05 kernel rescales its O accumulator in TMEM each time."""
    lb = _lib.lib()
    rng = np.random.default_rng(9)
    b, heads, hd, n_q, n_kv = 1, 2, 64, 256, 1000
    c = heads * hd
    u = rng.standard_normal(hd)
    u /= np.linalg.norm(u)
    q = np.tile(u, (b, n_q, heads)) + 0.05 * rng.standard_normal((b, n_q, c))
    ramp = np.linspace(0.0, 40.0, n_kv)[None, :, None]
    k = np.tile(u, (b, n_kv, heads)) * ramp + 0.2 * rng.standard_normal((b, n_kv, c))
    v = rng.standard_normal((b, n_kv, c))
    qd, kd, vd = dev16(q, torch.float16), dev16(k, torch.float16), dev16(v, torch.float16)
    out = torch.zeros((b, n_q, c), device="cuda", dtype=torch.float16)
    check(lb.osor_attention_heads(P(qd), c, n_q * c, P(kd), P(vd), c, n_kv * c, P(out), c,
                                  n_q * c, b, heads, n_q, n_kv, hd, dtype_code(torch.float16),
                                  S()))
    want = _attention_f64(host(qd).astype(np.float64), host(kd).astype(np.float64),
                          host(vd).astype(np.float64), heads, hd)
    assert np.all(np.abs(host(out) - want) <= 1e-3 + 1e-3 * np.abs(want))


def test_attention_heads_mma_sync_kernel_runs_the_same_cases(cuda_device):
    """OSOR_HEADS_TC=0 (read once per process) keeps head width 64 on the
    mma.sync kernel for every shape: run the cases above again in a child
    process with it set."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, OSOR_HEADS_TC="0")
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-q", "-p", "no:cacheprovider",
                        "-k", "attention_heads_match_f64 or rescales_growing_maxima"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("channels", [1920, 2560])
def test_group_norm_wide_rows_match_oracle(channels, cuda_device):
    import oracle
    lb = _lib.lib()
    rng = np.random.default_rng(channels)
    x = dev16(rng.standard_normal((2, 6, 5, channels)) * 2 + 0.5, torch.float16)
    g = torch.from_numpy((1 + 0.1 * rng.standard_normal(channels)).astype(np.float32)).cuda()
    bt = torch.from_numpy((0.1 * rng.standard_normal(channels)).astype(np.float32)).cuda()
    need = lb.osor_group_norm_workspace_size(2, channels, 6, 5, _lib.LAYOUT_NHWC,
                                             dtype_code(torch.float16))
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    stats = torch.empty((2, 32, 2), device="cuda")
    check(lb.osor_group_norm_silu(P(x), P(y), P(g), P(bt), 2, channels, 6, 5, _lib.LAYOUT_NHWC,
                                  dtype_code(torch.float16), 1e-5, 1, P(stats), P(ws), need, S()))
    xn = np.ascontiguousarray(host(x).transpose(0, 3, 1, 2))
    want, mean, var = oracle.group_norm(xn, host(g), host(bt), silu=True, eps=1e-5,
                                        return_stats=True)
    assert np.abs(host(y).transpose(0, 3, 1, 2) - want).max() < 5e-3
    st = host(stats)
    assert np.allclose(st[..., 0], mean, rtol=1e-4, atol=1e-4)
    assert np.allclose(st[..., 1], var, rtol=1e-4)


def test_padded_320_channel_convolution(cuda_device):
    """Cout 320 runs as a 384-channel tensor-core product (rows 320..383 of the
    weight zero) narrowed with the residual added."""
    import oracle
    lb = _lib.lib()
    rng = np.random.default_rng(320)
    dt = torch.float16
    x = dev16(rng.standard_normal((2, 16, 16, 320)), dt)
    w = (rng.standard_normal((320, 320, 3, 3)) * math.sqrt(2 / (9 * 320))).astype(np.float32)
    bias = rng.standard_normal(320).astype(np.float32)
    res = dev16(rng.standard_normal((2, 16, 16, 320)), dt)
    packed = torch.zeros((384, 9 * 320), device="cuda", dtype=torch.float32)
    packed[:320] = torch.from_numpy(w).cuda().permute(0, 2, 3, 1).reshape(320, -1)
    packed = packed.to(dt).contiguous()
    b384 = torch.zeros(384, device="cuda")
    b384[:320] = torch.from_numpy(bias).cuda()
    tmp = torch.empty((2, 16, 16, 384), device="cuda", dtype=dt)
    check(lb.osor_conv2d(P(x), P(tmp), P(packed), P(b384), None, 2, 16, 16, 320, 384, 3, 1, 1, 1,
                         _lib.LAYOUT_NHWC, _lib.LAYOUT_NHWC, dtype_code(dt), S()))
    out = torch.empty((2, 16, 16, 320), device="cuda", dtype=dt)
    check(lb.osor_channel_update(P(tmp), 384, P(out), 320, 2, 256, None, 0, P(res),
                                 dtype_code(dt), S()))
    assert torch.count_nonzero(tmp[..., 320:]).item() == 0
    wr = host(packed[:320]).reshape(320, 3, 3, 320).transpose(0, 3, 1, 2)
    want = oracle.conv2d(np.ascontiguousarray(host(x).transpose(0, 3, 1, 2)), wr, bias, 1, 1)
    want = want.transpose(0, 2, 3, 1) + host(res)
    got = host(out)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 2e-3


def test_attention_heads_rejects_bad_shapes(cuda_device):
    lb = _lib.lib()
    t = torch.empty(4096, device="cuda", dtype=torch.float16)
    f16 = dtype_code(torch.float16)
    with pytest.raises(InvalidInput):
        check(lb.osor_attention_heads(P(t), 64, 0, P(t), P(t), 64, 0, P(t), 64, 0, 1, 1, 4, 4, 48,
                                      f16, S()))
    with pytest.raises(InvalidInput):  # ld below heads * head_dim
        check(lb.osor_attention_heads(P(t), 64, 0, P(t), P(t), 64, 0, P(t), 64, 0, 1, 2, 4, 4, 64,
                                      f16, S()))
    with pytest.raises(InvalidInput):  # overlapping batch entries
        check(lb.osor_attention_heads(P(t), 64, 64, P(t), P(t), 64, 0, P(t), 64, 256, 2, 1, 4, 4,
                                      64, f16, S()))


# ---------------------------------------------------------------- model level
def _oracle_arch(arch):
    return U.Arch(tuple(U.Block(b.channels, b.depth, b.heads) for b in arch.blocks),
                  arch.context, arch.pooled, arch.time_projection, arch.layers)


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def tiny_model():
    arch = Architecture.tiny()
    w = U.deterministic_weights(_oracle_arch(arch))
    seq = U.fixed_values(16, 1).reshape(1, 2, 8)
    pooled = U.fixed_values(8, 2).reshape(1, 8)
    return arch, w, seq, pooled


# Parity shapes keep at least 2 x 2 pixels in the bottleneck: at a 4 x 4 latent
# the tiny model's 1 x 1 bottleneck leaves two values per normalisation group,
# which amplifies 16-bit rounding (the same CPU emulation gives 0.29 / 0.42
# relative L2 there; the reference's own batch test avoids that size for the
# same reason, src/native.rs:808-812). 4 x 4 is checked for shapes below.
@pytest.mark.parametrize("dt,bound", [(torch.float16, 1e-2), (torch.bfloat16, 5e-2)])
@pytest.mark.parametrize("shape", [(2, 9, 8, 8), (1, 9, 5, 7)])
def test_tiny_unet_matches_oracle(tiny_model, dt, bound, shape, cuda_device):
    arch, w, seq, pooled = tiny_model
    unet = NativeUnet(w, seq, pooled, arch=arch, dtype=dt)
    x = np.random.default_rng(1).standard_normal(shape).astype(np.float32)
    ids = np.tile(np.array([[64, 64, 0, 0, 64, 64]], np.float32), (shape[0], 1))
    got = unet(torch.from_numpy(x).cuda(), 400, torch.from_numpy(ids).cuda())
    assert tuple(got.shape) == (shape[0], 5) + shape[2:] and got.dtype == torch.float32
    want = U.forward(w, _oracle_arch(arch), x, 400, ids, seq, pooled)
    assert _rel(host(got), want) < bound


def test_tiny_unet_minimum_latent_shape(tiny_model, cuda_device):
    """src/native.rs:786-801: [1, 9, 4, 4] -> [1, 5, 4, 4], and the timestep
    changes the output."""
    arch, w, seq, pooled = tiny_model
    unet = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.float16)
    x = torch.from_numpy(U.fixed_values(9 * 4 * 4, 5).reshape(1, 9, 4, 4)).cuda()
    ids = torch.tensor([[32, 32, 0, 0, 32, 32]], dtype=torch.float32, device="cuda")
    out = unet(x, 400, ids)
    assert tuple(out.shape) == (1, 5, 4, 4) and torch.isfinite(out).all()
    assert (unet(x, 401, ids) - out).abs().max().item() > 1e-4


def test_tiny_unet_uses_conditioning_and_keeps_batch_entries_apart(tiny_model, cuda_device):
    """src/native.rs:773-843 on the GPU path."""
    arch, w, seq, pooled = tiny_model
    unet = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.float16)
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((2, 9, 8, 8)).astype(np.float32)).cuda()
    ids = torch.tensor([[64, 64, 0, 0, 64, 64]] * 2, dtype=torch.float32, device="cuda")
    both = unet(x, 400, ids)
    for i in range(2):
        single = unet(x[i:i + 1].contiguous(), 400, ids[i:i + 1].contiguous())
        assert torch.allclose(both[i:i + 1], single, atol=1e-5, rtol=0)
    assert (unet(x, 401, ids) - both).abs().max().item() > 1e-4
    assert (unet(x, 400, ids + 1) - both).abs().max().item() > 1e-4
    other = NativeUnet(w, seq * 2, pooled, arch=arch, dtype=torch.float16)
    assert (other(x, 400, ids) - both).abs().max().item() > 1e-4


def test_sdxl_width_unet_matches_oracle(cuda_device):
    """One layer per block at SDXL's widths: 320 (padded tensor-core products),
    640 / 1280 with 10 / 20 heads, 2560- and 1920-channel skip concatenations."""
    arch = Architecture((BlockSpec(320, None, 5), BlockSpec(640, 1, 10), BlockSpec(1280, 1, 20)),
                        context=64, pooled=32, time_projection=32, layers=1)
    w = {k: v.numpy() for k, v in random_unet_weights(arch, seed=7).items()}
    rng = np.random.default_rng(2)
    seq = rng.standard_normal((1, 77, 64)).astype(np.float32)
    pooled = rng.standard_normal((1, 32)).astype(np.float32)
    x = rng.standard_normal((1, 9, 16, 16)).astype(np.float32)
    ids = np.array([[128, 128, 0, 0, 128, 128]], np.float32)
    want = U.forward(w, _oracle_arch(arch), x, 400, ids, seq, pooled)
    for dt, bound in ((torch.float16, 1e-2), (torch.bfloat16, 5e-2)):
        unet = NativeUnet(w, seq, pooled, arch=arch, dtype=dt)
        got = unet(torch.from_numpy(x).cuda(), 400, torch.from_numpy(ids).cuda())
        assert _rel(host(got), want) < bound


def test_native_unet_validates_inputs(tiny_model, cuda_device):
    arch, w, seq, pooled = tiny_model
    unet = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.float16)
    ids = torch.zeros((1, 6), device="cuda")
    with pytest.raises(InvalidInput):
        unet(torch.zeros((1, 8, 8, 8), device="cuda"), 400, ids)
    with pytest.raises(InvalidInput):
        unet(torch.zeros((5, 9, 8, 8), device="cuda"), 400, torch.zeros((5, 6), device="cuda"))
    with pytest.raises(InvalidInput):
        unet(torch.zeros((1, 9, 3, 8), device="cuda"), 400, ids)
    with pytest.raises(InvalidInput):
        unet(torch.zeros((1, 9, 8, 8), device="cuda"), 400, torch.zeros((1, 5), device="cuda"))
    bad = dict(w)
    bad.pop("mid_block.resnets.1.conv2.weight")
    with pytest.raises(_lib.InvalidArtifact):
        NativeUnet(bad, seq, pooled, arch=arch)
    with pytest.raises(InvalidInput):
        NativeUnet(w, seq[:, :, :4], pooled, arch=arch)


def test_graph_replay_matches_eager(tiny_model, cuda_device):
    arch, w, seq, pooled = tiny_model
    eager = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.float16)
    replay = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.float16, graphs=True)
    rng = np.random.default_rng(8)
    ids = torch.tensor([[64, 64, 0, 0, 64, 64]] * 2, dtype=torch.float32, device="cuda")
    for _ in range(2):  # capture, then replay with new inputs
        x = torch.from_numpy(rng.standard_normal((2, 9, 8, 8)).astype(np.float32)).cuda()
        assert torch.equal(replay(x, 400, ids), eager(x, 400, ids))
    assert torch.equal(replay(x, 401, ids), eager(x, 401, ids))
    assert len(replay._captured) == 2


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_native_executor_matches_the_python_host(tiny_model, dt, cuda_device):
    """osor_unet_create / osor_unet_denoise run the same launches as NativeUnet."""
    arch, w, seq, pooled = tiny_model
    host = NativeUnet(w, seq, pooled, arch=arch, dtype=dt)
    native = UnetExecutor(w, seq, pooled, arch=arch, dtype=dt)
    rng = np.random.default_rng(12)
    for shape in ((2, 9, 8, 8), (1, 9, 5, 7)):
        x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).cuda()
        ids = torch.tensor([[64, 56, 0, 0, 64, 56]] * shape[0], dtype=torch.float32, device="cuda")
        assert torch.equal(native(x, 400, ids), host(x, 400, ids))
    native.close()


def test_native_executor_at_sdxl_widths(cuda_device):
    arch = Architecture((BlockSpec(320, None, 5), BlockSpec(640, 1, 10), BlockSpec(1280, 1, 20)),
                        context=64, pooled=32, time_projection=32, layers=1)
    w = {k: v.numpy() for k, v in random_unet_weights(arch, seed=7).items()}
    rng = np.random.default_rng(2)
    seq = rng.standard_normal((1, 77, 64)).astype(np.float32)
    pooled = rng.standard_normal((1, 32)).astype(np.float32)
    x = torch.from_numpy(rng.standard_normal((1, 9, 16, 16)).astype(np.float32)).cuda()
    ids = torch.tensor([[128, 128, 0, 0, 128, 128]], dtype=torch.float32, device="cuda")
    native = UnetExecutor(w, seq, pooled, arch=arch, dtype=torch.bfloat16)
    host = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.bfloat16)
    assert torch.equal(native(x, 400, ids), host(x, 400, ids))


def test_native_executor_cancels_and_validates(tiny_model, cuda_device):
    from osor_b200.model import CancellationToken
    arch, w, seq, pooled = tiny_model
    native = UnetExecutor(w, seq, pooled, arch=arch, dtype=torch.float16)
    x = torch.zeros((1, 9, 8, 8), device="cuda")
    ids = torch.zeros((1, 6), device="cuda")
    token = CancellationToken()
    token.cancel()
    with pytest.raises(_lib.Cancelled):
        native(x, 400, ids, cancellation=token)
    with pytest.raises(InvalidInput):
        native(torch.zeros((1, 9, 200, 8), device="cuda"), 400, ids)
    with pytest.raises(InvalidInput):
        native(torch.zeros((5, 9, 8, 8), device="cuda"), 400, torch.zeros((5, 6), device="cuda"))
    out = native(x, 400, ids)
    assert torch.isfinite(out).all()
    bad = dict(w)
    bad["conv_out.weight"] = np.zeros((5, 64, 1, 1), np.float32)
    with pytest.raises(_lib.InvalidArtifact):
        UnetExecutor(bad, seq, pooled, arch=arch)


def test_unet_loads_from_safetensors(tiny_model, tmp_path, cuda_device):
    from osor_b200.artifact import write_safetensors
    arch, w, seq, pooled = tiny_model
    path = str(tmp_path / "unet.safetensors")
    write_safetensors(path, w, dtype="F16")
    loaded = NativeUnet.from_safetensors(path, seq, pooled, arch=arch, dtype=torch.float16)
    direct = NativeUnet(w, seq, pooled, arch=arch, dtype=torch.float16)
    x = torch.from_numpy(np.random.default_rng(6).standard_normal((1, 9, 8, 8)).astype(np.float32)).cuda()
    ids = torch.tensor([[64, 64, 0, 0, 64, 64]], dtype=torch.float32, device="cuda")
    # The file stores F16 tensors; the model rounds weights to f16 either way.
    assert torch.equal(loaded(x, 400, ids), direct(x, 400, ids))


def test_pipeline_runs_with_the_native_unet(cuda_device):
    from osor_b200.model import NativeModel
    from osor_b200.pipeline import Pipeline
    from osor_b200.weights import random_vae_weights
    arch = Architecture.tiny()
    w = U.deterministic_weights(_oracle_arch(arch))
    unet = NativeUnet(w, U.fixed_values(16, 1).reshape(1, 2, 8),
                      U.fixed_values(8, 2).reshape(1, 8), arch=arch, dtype=torch.float16)
    vae = NativeModel(random_vae_weights(0), device=0, dtype="f16")
    g = torch.Generator().manual_seed(0)
    image = torch.rand((1, 3, 64, 64), generator=g).cuda()
    mask = torch.zeros((1, 1, 64, 64), device="cuda")
    mask[..., 16:40, 8:48] = 1.0
    noise = torch.randn((2, 1, 4, 8, 8), generator=g).cuda()
    result = Pipeline(vae, unet).run(image, mask, noise[0].contiguous(), noise[1].contiguous())
    assert tuple(result.image.shape) == (1, 3, 64, 64)
    assert torch.isfinite(result.image).all() and torch.isfinite(result.alpha).all()
