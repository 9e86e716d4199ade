"""The pipeline stages around the VAE on the GPU against the oracle.

* The scheduler kernels reproduce the reference's pinned f32 results bit for
  bit (src/scheduler.rs:348-372) and its DDPM prediction / clipping cases
  (:374-416).
* Each stage kernel matches the oracle's f32 restatement: exactly where the
  arithmetic has no transcendental (pooling, blending, display mapping,
  bilinear alpha), within a few ulp where CUDA's expf enters (posterior
  standard deviation, sigmoid).
* Pipeline.run with a stand-in denoiser (exact arithmetic: epsilon = noisy / 2,
  logits = 4 * mask - 2) against the oracle pipeline with the oracle VAE.
"""
import math

import numpy as np
import pytest
import torch

import oracle.vae as ovae
from oracle import pipeline as op
from osor_b200 import _lib, workloads
from osor_b200.model import CancellationToken, NativeModel, device_status
from osor_b200.pipeline import Pipeline, Scheduler, SchedulerConfig, Stage
from osor_b200.weights import random_vae_weights

pytestmark = pytest.mark.gpu

SAMPLE = np.array([2.0, -3.0, 0.01, 100.0], np.float32)
NOISE = np.array([0.5, 0.125, 2.0, -4.0], np.float32)
PINNED_NOISY = [0x3FD7579C, 0xBFEE0C04, 0x3FC30AF8, 0x427878A8]
PINNED_PREDICTED = [0x401F33BD, 0xC0980129, 0xC0140F51, 0x431E24DD]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def test_scheduler_kernels_reproduce_pinned_values(cuda_device):
    s = Scheduler()
    noisy = s.add_noise(cuda(SAMPLE), cuda(NOISE), 400).cpu().numpy()
    pred = s.predicted_original_sample(cuda(SAMPLE), cuda(NOISE), 400).cpu().numpy()
    assert list(noisy.view(np.uint32)) == PINNED_NOISY
    assert list(pred.view(np.uint32)) == PINNED_PREDICTED


def test_ddpm_predictions_and_clipping(cuda_device):
    x, n = cuda([2.0]), cuda([0.5])
    for kind, want in [("epsilon", 2 / math.sqrt(0.9) - 0.5 * math.sqrt(0.1 / 0.9)),
                       ("sample", 0.5), ("v_prediction", 2 * math.sqrt(0.9) - 0.5 * math.sqrt(0.1))]:
        s = Scheduler(SchedulerConfig(num_train_timesteps=1, trained_betas=[0.1],
                                      prediction_type=kind))
        noisy = float(s.add_noise(x, n, 0)[0])
        assert abs(noisy - (2 * math.sqrt(0.9) + 0.5 * math.sqrt(0.1))) < 1e-6
        assert abs(float(s.predicted_original_sample(x, n, 0)[0]) - want) < 1e-6
    s = Scheduler(SchedulerConfig(num_train_timesteps=1, trained_betas=[0.1], clip_sample=True,
                                  clip_sample_range=0.4))
    assert abs(float(s.predicted_original_sample(x, n, 0)[0]) - 0.4) < 1e-6
    with pytest.raises(_lib.InvalidInput):
        s.add_noise(x, n, 1)
    with pytest.raises(_lib.InvalidInput):
        s.add_noise(x, cuda([float("nan")]), 0)


def _stage_inputs(b, hgt, wid, seed):
    rng = np.random.default_rng(seed)
    h, w = hgt // 8, wid // 8
    moments = rng.standard_normal((b, 8, h, w)).astype(np.float32)
    moments[:, 4:] *= 12.0  # logvar beyond the clamp on both sides
    pn = rng.standard_normal((b, 4, h, w)).astype(np.float32)
    dn = rng.standard_normal((b, 4, h, w)).astype(np.float32)
    mask = (rng.random((b, 1, hgt, wid)) < 0.02).astype(np.float32)
    out = rng.standard_normal((b, 5, h, w)).astype(np.float32) * 3.0
    return moments, pn, dn, mask, out


@pytest.mark.parametrize("kind", ["epsilon", "sample", "v_prediction"])
def test_stage_kernels_match_oracle(cuda_device, kind):
    b, hgt, wid = 2, 64, 96
    moments, pn, dn, mask, out = _stage_inputs(b, hgt, wid, 3)
    a = float(op.alphas_cumprod()[400])
    lib, s = _lib.lib(), None
    h, w = hgt // 8, wid // 8
    t = {k: cuda(v) for k, v in dict(m=moments, pn=pn, dn=dn, mask=mask, out=out).items()}
    u = torch.empty((b, 9, h, w), device="cuda")
    smp = torch.empty((b, 4, h, w), device="cuda")
    ptr = lambda x: x.data_ptr()  # noqa: E731
    _lib.check(lib.osor_pipeline_prepare(ptr(t["m"]), ptr(t["pn"]), ptr(t["dn"]), ptr(t["mask"]),
                                         ptr(u), ptr(smp), b, hgt, wid, a, 0.13025, s))
    want_u, want_s = op.prepare(moments, pn, dn, mask, a)
    got_u = u.cpu().numpy()
    np.testing.assert_array_equal(got_u[:, 4], want_u[:, 4])  # pooled mask
    np.testing.assert_allclose(got_u, want_u, rtol=2e-6, atol=1e-6)
    np.testing.assert_allclose(smp.cpu().numpy(), want_s, rtol=2e-6, atol=1e-6)
    # finish on the oracle's UNet input, so only this stage is compared
    uo = cuda(want_u)
    la = torch.empty((b, 1, h, w), device="cuda")
    pred, blend, lat = (torch.empty((b, 4, h, w), device="cuda") for _ in range(3))
    _lib.check(lib.osor_pipeline_finish(ptr(t["out"]), ptr(uo), ptr(la), ptr(pred), ptr(blend),
                                        ptr(lat), b, hgt, wid, a, {"epsilon": 0, "sample": 1,
                                                                   "v_prediction": 2}[kind],
                                        0, 1.0, 0.13025, s))
    w_alpha, w_pred, w_blend, w_lat = op.finish(out, want_u, a, kind)
    np.testing.assert_array_equal(pred.cpu().numpy(), w_pred)
    np.testing.assert_allclose(la.cpu().numpy(), w_alpha, rtol=2e-6, atol=0)
    np.testing.assert_allclose(blend.cpu().numpy(), w_blend, rtol=4e-6, atol=1e-6)
    np.testing.assert_allclose(lat.cpu().numpy(), w_lat, rtol=4e-6, atol=1e-5)
    # display mapping and bilinear alpha on the oracle's latent alpha
    rng = np.random.default_rng(4)
    dec = (rng.standard_normal((b, 3, hgt, wid)) * 1.5).astype(np.float32)
    img = torch.empty((b, 3, hgt, wid), device="cuda")
    alpha = torch.empty((b, 1, hgt, wid), device="cuda")
    dec_t, la_t = cuda(dec), cuda(w_alpha)  # kept alive until the kernel has run
    _lib.check(lib.osor_pipeline_map(ptr(dec_t), ptr(la_t), ptr(img), ptr(alpha), b, hgt, wid, s))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(img.cpu().numpy(), op.display(dec))
    np.testing.assert_array_equal(alpha.cpu().numpy(), op.bilinear_8x(w_alpha, hgt, wid))


def _denoise_torch(u, timestep, time_ids):
    return torch.cat([u[:, :4] * 0.5, u[:, 4:5] * 4.0 - 2.0], dim=1).contiguous()


def _denoise_np(u):
    return np.concatenate([u[:, :4] * np.float32(0.5), u[:, 4:5] * np.float32(4.0) - np.float32(2.0)],
                          axis=1)


def _job(b, hgt, wid, seed):
    rng = np.random.default_rng(seed)
    image = rng.random((b, 3, hgt, wid)).astype(np.float32)
    mask = np.zeros((b, 1, hgt, wid), np.float32)
    mask[:, :, hgt // 4: hgt // 2, wid // 8: wid // 2] = 1.0
    pn = rng.standard_normal((b, 4, hgt // 8, wid // 8)).astype(np.float32)
    dn = rng.standard_normal((b, 4, hgt // 8, wid // 8)).astype(np.float32)
    return image, mask, pn, dn


@pytest.fixture(scope="module")
def weights():
    return random_vae_weights(0)


def test_pipeline_run_matches_oracle(cuda_device, weights):
    b, hgt, wid = 1, 64, 64
    image, mask, pn, dn = _job(b, hgt, wid, 9)
    model = NativeModel(weights, device=0, dtype="f16")
    stages = []
    pipe = Pipeline(model, _denoise_torch)
    res = pipe.run(cuda(image), cuda(mask), cuda(pn), cuda(dn),
                   observer=lambda st, t: stages.append(st))
    torch.cuda.synchronize()
    assert device_status(0) == 0
    assert stages == [Stage.PosteriorMoments, Stage.PosteriorMean, Stage.PosteriorLogvar,
                      Stage.PosteriorSample, Stage.OriginalLatent, Stage.PooledMask,
                      Stage.NoisyLatent, Stage.UnetInput, Stage.TimeIds, Stage.DenoisingOutput,
                      Stage.AlphaLogits, Stage.LatentAlpha, Stage.PredictedOriginal,
                      Stage.BlendedLatent, Stage.DecodedImage, Stage.Alpha]
    a = float(op.alphas_cumprod()[400])
    moments = ovae.encode_moments(weights, image * np.float32(2.0) - np.float32(1.0))
    u, _ = op.prepare(moments, pn, dn, mask, a)
    alpha, _, _, latents = op.finish(_denoise_np(u), u, a)
    want_image = op.display(ovae.decode(weights, latents))
    want_alpha = op.bilinear_8x(alpha, hgt, wid)
    got_image = res.image.cpu().numpy()
    assert np.all((got_image >= 0) & (got_image <= 1))
    # The latent alpha depends only on the mask: f32 sigmoid, a few ulp.
    np.testing.assert_allclose(res.latent_alpha.cpu().numpy(), alpha, rtol=2e-6, atol=0)
    np.testing.assert_allclose(res.alpha.cpu().numpy(), want_alpha, rtol=4e-6, atol=1e-6)
    # The image goes through the f16 encoder and decoder.
    err = np.abs(got_image - want_image)
    assert err.max() <= 5e-2, err.max()
    assert workloads.psnr(got_image, want_image) >= 35.0


def test_pipeline_cancellation_and_validation(cuda_device, weights):
    model = NativeModel(weights, device=0, dtype="f16", parts=("decoder", "encoder"))
    pipe = Pipeline(model, _denoise_torch)
    image, mask, pn, dn = _job(1, 32, 40, 2)
    token = CancellationToken()
    token.cancel()
    with pytest.raises(_lib.Cancelled):
        pipe.run(cuda(image), cuda(mask), cuda(pn), cuda(dn), cancellation=token)
    with pytest.raises(_lib.InvalidInput):
        pipe.run(cuda(image) * 2.0, cuda(mask), cuda(pn), cuda(dn))  # image outside [0, 1]
    with pytest.raises(_lib.InvalidInput):
        pipe.run(cuda(image), cuda(mask), cuda(pn[:, :3]), cuda(dn))
    bad = lambda u, t, ids: torch.zeros((1, 4, 4, 5), device="cuda")  # noqa: E731
    with pytest.raises(_lib.InvalidInput):
        Pipeline(model, bad).run(cuda(image), cuda(mask), cuda(pn), cuda(dn))
