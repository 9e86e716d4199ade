"""Parity at the benchmark's own shapes, through the C ABI, against the oracle.

* Decoder, the headline workload: a batch of four [4,128,128] latents ->
  [4,3,1024,1024] (osor_vae_decode), whose first image is the one-image
  golden of tests/golden/decoder_d4.npz (the oracle's f32 output, made by
  tests/golden/make_golden.py): compared on the golden's strided sample
  (every phase of the three nearest-2x upsamplings), its three 64 x 64 crops
  and the whole image's per-channel moments.
* Encoder, the E4 workload: four [3,1024,1024] images -> moments
  [4,8,128,128] (osor_vae_encode_moments), the first checked against the
  whole f32 golden of tests/golden/encoder_e4.npz.
* Mid-block attention at the headline's 16384 tokens, width 512
  (osor_attention: 128 score blocks merged per row), against the oracle's
  sliced F32 attention (src/native/attention.rs:27-84) on 256 query rows
  (rows are independent, so a subset is an exact check).
* The five standalone 3x3 convolution shapes of the benchmark at batch 1,
  Cin 512 included (K = 4608), against the oracle's column convolution on a
  spread subset of output channels (channels are independent).
* The four standalone GroupNorm+SiLU shapes at batch 1: group mean and
  variance within 1e-4 relative of the oracle's staged statistics, outputs
  within the 16-bit type's rounding.

Every case runs in f16 and bf16. Decoded RGB: 2e-2 max-abs and >= 40 dB
PSNR for f16 (the acceptance bound); bf16 is held to 40 dB and its measured
format floor (tests/tolerances.py). Moments: relative L2 1e-2 (f16).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from osor_b200 import ops, workloads
from osor_b200._lib import LAYOUT_NCHW
from osor_b200.model import NativeModel, device_status
from osor_b200.weights import random_vae_weights

from tolerances import MAX_ABS, MOMENTS_REL_L2

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16}


@pytest.fixture(scope="module")
def weights():
    return random_vae_weights(0)


@pytest.fixture(scope="module", params=["f16", "bf16"])
def model(request, weights, cuda_device):
    m = NativeModel(weights, device=0, dtype=request.param)
    yield m
    m.close()


def _image_checks(img, g, dtype):
    """img: [3, S, S] f32 decode; g: a golden written by make_golden.image_sample."""
    rows, cols = g["rows"], g["cols"]
    sample = img[:, rows[:, None], cols]
    s = img.shape[-1]
    mid = int(g["crop_centre_at"])
    crops = [(img[:, :64, :64], g["crop_top_left"]),
             (img[:, s - 64:, s - 64:], g["crop_bottom_right"]),
             (img[:, mid:mid + 64, mid:mid + 64], g["crop_centre"])]
    assert np.all(np.isfinite(img))
    err = max([float(np.abs(sample - g["sample"]).max())] +
              [float(np.abs(a - b).max()) for a, b in crops])
    p = workloads.psnr(sample, g["sample"])
    assert err <= MAX_ABS[dtype], (err, p)
    assert p >= 40.0, p
    for a, b in crops:
        assert workloads.psnr(a, b) >= 40.0
    mean = img.reshape(3, -1).astype(np.float64).mean(axis=1)
    std = img.reshape(3, -1).astype(np.float64).std(axis=1)
    np.testing.assert_allclose(mean, g["channel_mean"], atol=2e-3)
    np.testing.assert_allclose(std, g["channel_std"], rtol=2e-3)
    return err, p


def test_headline_decode_batch_of_four_matches_golden(model):
    g = np.load(os.path.join(GOLDEN, "decoder_d4.npz"))
    first = workloads.decoder_latents(1, 128, 128, seed=42)
    assert abs(float(first.sum()) - float(g["latents_sum"])) < 1e-2
    lat = np.concatenate([first, workloads.decoder_latents(3, 128, 128, seed=43)])
    out = model.decode(torch.from_numpy(lat).cuda())
    assert device_status(0) == 0
    assert tuple(out.shape) == (4, 3, 1024, 1024)
    got = out.cpu().numpy()
    _image_checks(got[0], g, model.dtype)
    assert np.all(np.isfinite(got))
    # The same image decoded alone.
    alone = model.decode(torch.from_numpy(first).cuda()).cpu().numpy()
    _image_checks(alone[0], g, model.dtype)


def test_headline_encode_batch_of_four_matches_golden(model):
    g = np.load(os.path.join(GOLDEN, "encoder_e4.npz"))
    img, noise = workloads.encoder_image(1, 1024, 1024, seed=7)
    assert abs(float(img.sum()) - float(g["image_sum"])) < 1.0
    rest, _ = workloads.encoder_image(3, 1024, 1024, seed=8)
    batch = np.concatenate([img, rest])
    got = model.encode_moments(torch.from_numpy(batch).cuda()).cpu().numpy()
    assert device_status(0) == 0
    assert got.shape == (4, 8, 128, 128)
    assert np.all(np.isfinite(got))
    assert workloads.rel_l2(got[0], g["moments"][0]) <= MOMENTS_REL_L2[model.dtype]


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_attention_at_16384_tokens_matches_oracle(dt, cuda_device):
    n, d = 16384, 512
    rng = np.random.default_rng(17)
    t = DTYPES[dt]

    def half(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(t)

    # Logit spread of the VAE's mid-block (q and k each scaled by d^-1/4).
    q = half(rng.standard_normal((1, n, d), dtype=np.float32) * np.float32(d ** -0.25 * 1.4))
    k = half(rng.standard_normal((1, n, d), dtype=np.float32) * np.float32(d ** -0.25 * 1.4))
    v = half(rng.standard_normal((1, n, d), dtype=np.float32))
    got = ops.attend(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    assert device_status(0) == 0
    rows = np.unique(np.concatenate([[0, 127, 128, n - 1], rng.choice(n, 252, replace=False)]))
    got = got[:, torch.from_numpy(rows).cuda()].float().cpu().numpy()
    qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
    want = oracle.attend(np.ascontiguousarray(qf[:, rows]),
                         np.ascontiguousarray(kf.transpose(0, 2, 1)), vf)
    err = np.abs(got - want)
    assert np.all(np.isfinite(got))
    # 16-bit probabilities (relative 2^-9 for bf16) and 16-bit output rounding.
    assert err.max() <= 2e-2, err.max()
    assert np.sqrt((err ** 2).mean()) <= 3e-3


# (batch, cin, cout, h, w): the benchmark's standalone 3x3 shapes at batch 1.
CONV_SHAPES = [(1, 512, 512, 128, 128), (1, 512, 512, 256, 256), (1, 256, 256, 512, 512),
               (1, 128, 128, 1024, 1024), (1, 128, 3, 1024, 1024)]


@pytest.mark.parametrize("shape", CONV_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_benchmark_conv_shapes_match_oracle(shape, dt, cuda_device):
    b, cin, cout, h, w = shape
    t = DTYPES[dt]

    def rnd(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(t).float().numpy()

    x, wt, bias, res = workloads.conv_inputs(b, cin, cout, h, w, seed=5)
    x, wt = rnd(x), rnd(wt)
    conv = ops.BandedConv2d(wt, bias, stride=1, padding=1, dtype=t)
    xt = ops.nchw_to_nhwc(torch.from_numpy(x).cuda(), t)
    if cout <= 16:  # the decoder's conv_out: NCHW f32 image, no residual
        y = conv.forward_checked(xt, out_layout=LAYOUT_NCHW)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        idx = np.arange(cout)
        want = oracle.conv2d(x, wt, bias, stride=1, padding=1)
        tol_rel = 0.0
    else:
        res = rnd(res)
        y = conv.forward_checked(xt, residual=ops.nchw_to_nhwc(torch.from_numpy(res).cuda(), t))
        torch.cuda.synchronize()
        idx = np.unique(np.linspace(0, cout - 1, 9).astype(int).tolist() + [1, cout // 2 + 1])
        got = ops.nhwc_to_nchw(y[..., torch.from_numpy(idx).cuda()]).cpu().numpy()
        want = oracle.conv2d(x, np.ascontiguousarray(wt[idx]), bias[idx], stride=1,
                             padding=1) + res[:, idx]
        tol_rel = 2.0 ** -8 if dt == "bf16" else 2.0 ** -10  # 16-bit output rounding
    assert device_status(0) == 0
    assert np.all(np.isfinite(got))
    err = np.abs(got - want)
    assert np.all(err <= tol_rel * np.abs(want) + 2e-3), float(err.max())


GN_SHAPES = [(1, 512, 128, 128), (1, 512, 256, 256), (1, 256, 512, 512), (1, 128, 1024, 1024)]


@pytest.mark.parametrize("shape", GN_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_benchmark_groupnorm_shapes_match_oracle(shape, dt, cuda_device):
    t = DTYPES[dt]
    x, gamma, beta = workloads.groupnorm_inputs(shape, seed=3)
    xt = torch.from_numpy(x).to(t)
    xr = xt.float().numpy()
    stats = torch.zeros((shape[0] * 32, 2), dtype=torch.float32, device="cuda")
    y = ops.StableGroupNorm(gamma, beta).forward_silu(xt.cuda(), stats=stats)
    torch.cuda.synchronize()
    assert device_status(0) == 0
    want, mean, var = oracle.group_norm(xr, gamma, beta, silu=True, return_stats=True)
    st = stats.cpu().numpy().reshape(shape[0], 32, 2)
    np.testing.assert_allclose(st[..., 0], mean, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(st[..., 1], var, rtol=1e-4)
    got = y.float().cpu().numpy()
    ulp = 2.0 ** -7 if dt == "bf16" else 2.0 ** -10
    assert np.all(np.abs(got - want) <= ulp * np.abs(want) + 2e-3)
