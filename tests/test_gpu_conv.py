"""Convolution parity: CUDA (tensor-core implicit GEMM and CUDA-core direct)
against the CPU oracle on the same bf16-representable inputs.

Mirrors the reference's conv tests: banded_convolution_is_band_independent_and
_matches_candle (src/native/conv.rs:297-383: dyadic inputs make every product
and sum exact, so results must match bit for bit) and
column_convolution_matches_candle_on_cpu (src/native/columns.rs:448-479:
random inputs, tolerance based).
"""
import numpy as np
import pytest
import torch

import oracle
from osor_b200 import ops
from osor_b200._lib import InvalidInput, LAYOUT_NCHW

pytestmark = pytest.mark.gpu


DT = torch.bfloat16  # rebound per test by the `dtype` fixture


@pytest.fixture(params=[torch.bfloat16, torch.float16], ids=["bf16", "f16"], autouse=True)
def dtype(request):
    global DT
    DT = request.param
    return request.param


def bf16(a: np.ndarray) -> np.ndarray:
    """Round to the 16-bit type under test."""
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(DT).float().numpy()


def run_conv(x_nchw, w, b, stride, pad, residual_nchw=None, out_f32=False, pad_end=None):
    conv = ops.BandedConv2d(w, b, stride=stride, padding=pad, padding_end=pad_end, dtype=DT)
    if out_f32 or x_nchw.shape[1] % 8:
        x = torch.from_numpy(x_nchw).cuda()
    else:
        x = ops.nchw_to_nhwc(torch.from_numpy(x_nchw).cuda(), DT)
    res = None
    if residual_nchw is not None:
        res = ops.nchw_to_nhwc(torch.from_numpy(residual_nchw).cuda(), DT)
    if out_f32:
        y = conv.forward_checked(x, out_layout=LAYOUT_NCHW)
        torch.cuda.synchronize()
        return y.cpu().numpy()
    y = conv.forward_checked(x, residual=res)
    torch.cuda.synchronize()
    return ops.nhwc_to_nchw(y).cpu().numpy()


def dyadic(shape, mult, mod, shift, scale):
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.int64)
    return (((i * mult) % mod).astype(np.float32) - shift) * np.float32(scale)


# (batch, cin, h, w, cout, k, stride, pad): tensor-core eligible geometries
TC_CASES = [
    (1, 64, 8, 16, 128, 3, 1, 1),      # narrow image: 16 px x 8 rows per tile
    (2, 128, 4, 128, 128, 3, 1, 1),    # one image row per tile
    (1, 64, 2, 256, 256, 3, 1, 1),     # BLOCK_N 256
    (1, 128, 8, 64, 512, 3, 1, 1),     # 2 N tiles of 256, 2 rows per tile
    (1, 64, 16, 32, 128, 1, 1, 0),     # 1x1
    (2, 64, 16, 64, 128, 3, 2, 0),     # encoder downsample: right/bottom pad, stride 2
    (1, 64, 8, 256, 128, 3, 2, 0),     # encoder downsample, 128-px output rows
    # Cout 128 on CTA pairs: weights resident (K <= 1152) or streamed, 128-px
    # output rows (row-shift stages) or shorter rows (one stage per tap)
    (4, 128, 128, 128, 128, 3, 1, 1),  # resident, row shift, several tile pairs per cluster
    (1, 256, 16, 64, 128, 3, 1, 1),    # streamed, per-tap stages
    (2, 256, 4, 128, 128, 3, 1, 1),    # streamed, row shift
    (2, 256, 8, 128, 128, 1, 1, 0),    # 1x1, resident, deep pipeline
    (3, 64, 8, 16, 128, 3, 1, 1),      # odd number of tiles: one-CTA kernel
    # The UNet's widths: Cout 384 / 640 (multiples of 128 only: one-CTA
    # kernel, several 128-wide channel tiles) and Cout 1280 over few pixels
    # (pairs, five 256-wide channel tiles)
    (1, 128, 4, 128, 384, 3, 1, 1),
    (2, 128, 16, 64, 640, 1, 1, 0),
    (1, 256, 8, 128, 1280, 1, 1, 0),
    # Pixels on the MMA's N side (3x3, Cout <= 128, width % 256 == 0)
    (1, 128, 4, 256, 128, 3, 1, 1),    # two channel blocks
    (2, 64, 3, 512, 64, 3, 1, 1),      # Cout 64: weight rows past Cout read as zeros
    (1, 256, 2, 256, 128, 3, 1, 1),    # four channel blocks, two image rows
]


def oracle_conv(x, wt, bias, s, p):
    """Stride-2 cases are the encoder's downsampler: pad right/bottom, then
    convolve with no padding (vae_encoder.rs:206-210)."""
    if s == 2:
        return oracle.conv2d(oracle.pad_right_bottom(x), wt, bias, stride=2, padding=0)
    return oracle.conv2d(x, wt, bias, stride=s, padding=p)


def gpu_conv(x, wt, bias, s, p, residual_nchw=None):
    return run_conv(x, wt, bias, s, p, residual_nchw=residual_nchw, pad_end=1 if s == 2 else p)


@pytest.mark.parametrize("case", TC_CASES)
def test_tensor_core_conv_dyadic_is_exact(case, cuda_device):
    """Exactly representable inputs: GPU bf16 output == bf16(oracle fp32)."""
    b, cin, h, w, cout, k, s, p = case
    x = dyadic((b, cin, h, w), 13, 41, 20, 1 / 16).reshape(b, cin, h, w)
    wt = dyadic((cout, cin, k, k), 7, 11, 5, 1 / 32).reshape(cout, cin, k, k) / np.float32(8)
    bias = np.tile(np.array([-0.125, 0.0625, 0.0, 0.125, -0.0625], np.float32), cout)[:cout]
    ref = oracle_conv(x, wt, bias, s, p)
    got = gpu_conv(x, wt, bias, s, p)
    np.testing.assert_array_equal(got, bf16(ref))


@pytest.mark.parametrize("case", TC_CASES)
def test_tensor_core_conv_random_with_residual(case, cuda_device):
    b, cin, h, w, cout, k, s, p = case
    rng = np.random.default_rng(5)
    x = bf16(rng.standard_normal((b, cin, h, w)))
    wt = bf16(rng.standard_normal((cout, cin, k, k)) * np.sqrt(2.0 / (cin * k * k)))
    bias = rng.uniform(-0.1, 0.1, cout).astype(np.float32)
    ref = oracle_conv(x, wt, bias, s, p)
    res = bf16(rng.standard_normal(ref.shape))
    got = gpu_conv(x, wt, bias, s, p, residual_nchw=res)
    want = ref + res
    # 16-bit output rounding (bf16: relative 2^-8) plus accumulation-order differences.
    err = np.abs(got - want)
    assert np.all(err <= 2 ** -8 * np.abs(want) + 2e-3), err.max()


# The reference's own formula cases (conv.rs:300-305) on the CUDA-core path:
# Cin 6 -> Cout 5 is below the tensor-core tile.
REF_CASES = [(37, 20, 3, 1, 1), (33, 17, 3, 2, 0), (19, 11, 1, 1, 0)]


@pytest.mark.parametrize("case", REF_CASES)
def test_direct_conv_reference_formula_cases_exact(case, cuda_device):
    h, w, k, s, p = case
    wt = dyadic((5, 6, k, k), 7, 11, 5, 1 / 32).reshape(5, 6, k, k)
    bias = np.array([-0.125, 0.0625, 0.0, 0.125, -0.0625], np.float32)
    x = dyadic((2, 6, h, w), 13, 41, 20, 1 / 16).reshape(2, 6, h, w)
    ref = oracle.conv2d(x, wt, bias, stride=s, padding=p)
    got = run_conv(x, wt, bias, s, p, out_f32=True)
    np.testing.assert_array_equal(got, ref)


def test_conv_rejects_input_smaller_than_kernel(cuda_device):
    conv = ops.BandedConv2d(np.zeros((1, 1, 3, 3), np.float32), None, stride=2, padding=0)
    with pytest.raises(InvalidInput):
        conv.forward_checked(torch.zeros((1, 1, 2, 8), device="cuda"))


def test_upsample_matches_oracle(cuda_device):
    rng = np.random.default_rng(0)
    x = bf16(rng.standard_normal((2, 16, 5, 7)))
    got = ops.nhwc_to_nchw(ops.upsample_2x(ops.nchw_to_nhwc(torch.from_numpy(x).cuda(), DT))).cpu()
    np.testing.assert_array_equal(got.numpy(), oracle.upsample_2x(x))


def test_pixel_n_thin_nchw_output_exact(cuda_device):
    """conv_out shape class: 16-bit NHWC in, Cout 3 NCHW f32 out. By default
    the fused conv_out kernel runs it without its normalisation (one N = 32
    product of (tap, channel) columns per pixel, taps summed in the
    epilogue); test_padded_thin_path_runs_the_same_case runs the pixels-on-N
    kernel it replaced."""
    b, cin, h, w, cout = 1, 128, 3, 256, 3
    x = dyadic((b, cin, h, w), 13, 41, 20, 1 / 16).reshape(b, cin, h, w)
    wt = dyadic((cout, cin, 3, 3), 7, 11, 5, 1 / 32).reshape(cout, cin, 3, 3) / np.float32(8)
    bias = np.array([-0.125, 0.0625, 0.25], np.float32)
    conv = ops.BandedConv2d(wt, bias, stride=1, padding=1, dtype=DT)
    xt = ops.nchw_to_nhwc(torch.from_numpy(x).cuda(), DT)
    got = conv.forward_checked(xt, out_layout=LAYOUT_NCHW)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), oracle.conv2d(x, wt, bias, stride=1, padding=1))


def test_unet_conv_out_thin_nchw_on_tensor_cores_exact(cuda_device):
    """The UNet's conv_out shape class (unet_model.cu, osor_conv2d): Cin 320
    16-bit NHWC in, Cout 5 NCHW f32 out, weights packed with exactly 5 rows.
    The tensor-core thin tile reads its 16 weight rows with the rows past
    Cout zero-filled, so the shape runs as `conv_thin_tc`, not on the direct
    kernel; dyadic operands keep the sum exact."""
    from osor_b200 import _lib
    b, cin, h, w, cout = 2, 320, 3, 128, 5
    x = dyadic((b, cin, h, w), 13, 41, 20, 1 / 16).reshape(b, cin, h, w)
    wt = dyadic((cout, cin, 3, 3), 7, 11, 5, 1 / 32).reshape(cout, cin, 3, 3) / np.float32(8)
    bias = np.array([-0.125, 0.0625, 0.25, 0.0, 0.5], np.float32)
    conv = ops.BandedConv2d(wt, bias, stride=1, padding=1, dtype=DT)
    xt = ops.nchw_to_nhwc(torch.from_numpy(x).cuda(), DT)
    torch.cuda.synchronize()
    _lib.profile_begin()
    got = conv.forward_checked(xt, out_layout=LAYOUT_NCHW)
    kinds = [e[0] for e in _lib.profile_end()]
    torch.cuda.synchronize()
    assert kinds == ["conv_thin_tc"], kinds
    np.testing.assert_array_equal(got.cpu().numpy(), oracle.conv2d(x, wt, bias, stride=1, padding=1))


def test_padded_thin_path_runs_the_same_case(cuda_device):
    """OSOR_FUSED_THIN_CONV=0 (read once per process) keeps 128 -> 3
    convolutions on the pixels-on-N kernel with the weights padded to a
    128-row tile: the exact case above again, in a child process."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, OSOR_FUSED_THIN_CONV="0")
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-q", "-p", "no:cacheprovider",
                        "-k", "pixel_n_thin_nchw_output_exact"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
