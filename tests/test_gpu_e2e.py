"""The end-to-end inpainting call (Osor::infer, src/runtime.rs:484 ->
Pipeline::run, src/pipeline.rs:655-860) composed from the library's parts:
Pipeline.run with NativeModel (VAE encoder and decoder) and NativeUnet (the
denoiser), the reference's seeded noise and a seeded rectangle mask - the
composition of the benchmark's end-to-end configuration, at a small size with
the reference's tiny test UNet (src/native.rs:591-650) - against the same
chain on the oracle: oracle.vae encode -> oracle.pipeline.prepare ->
oracle.unet.forward -> oracle.pipeline.finish -> oracle.vae decode ->
display mapping.
"""
import numpy as np
import pytest
import torch

import oracle
import oracle.unet as U
import oracle.vae as ovae
from oracle import pipeline as op
from osor_b200 import workloads
from osor_b200.model import NativeModel, device_status
from osor_b200.noise import seeded_noise
from osor_b200.pipeline import Pipeline
from osor_b200.unet import Architecture, NativeUnet
from osor_b200.weights import random_vae_weights

pytestmark = pytest.mark.gpu


def _oracle_arch(arch):
    return U.Arch(tuple(U.Block(b.channels, b.depth, b.heads) for b in arch.blocks),
                  arch.context, arch.pooled, arch.time_projection, arch.layers)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_inpainting_job_end_to_end_matches_oracle_chain(dt, cuda_device):
    b, hgt, wid = 2, 64, 96
    arch = Architecture.tiny()
    uw = U.deterministic_weights(_oracle_arch(arch))
    seq = U.fixed_values(16, 1).reshape(1, 2, 8)
    pooled = U.fixed_values(8, 2).reshape(1, 8)
    vw = random_vae_weights(0)
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    model = NativeModel(vw, device=0, dtype=dt)
    unet = NativeUnet(uw, seq, pooled, arch=arch, dtype=tdt)
    image, mask = workloads.inpaint_job(b, hgt, wid, seed=5)
    noise = seeded_noise(42, b, hgt, wid)
    res = Pipeline(model, unet).run(torch.from_numpy(image).cuda(), torch.from_numpy(mask).cuda(),
                                    noise.posterior, noise.diffusion)
    torch.cuda.synchronize()
    assert device_status(0) == 0

    # The noise is the reference's stored-seed stream (oracle pinned to its goldens).
    n = b * 4 * (hgt // 8) * (wid // 8)
    pn = oracle.seeded_noise(42, 0, n).reshape(b, 4, hgt // 8, wid // 8)
    dn = oracle.seeded_noise(42, 1, n).reshape(b, 4, hgt // 8, wid // 8)
    np.testing.assert_array_equal(noise.posterior.cpu().numpy(), pn)
    np.testing.assert_array_equal(noise.diffusion.cpu().numpy(), dn)
    a = float(op.alphas_cumprod()[400])
    moments = ovae.encode_moments(vw, image * np.float32(2.0) - np.float32(1.0))
    u, _ = op.prepare(moments, pn, dn, mask, a)
    ids = np.tile(np.array([[hgt, wid, 0, 0, hgt, wid]], np.float32), (b, 1))
    out = U.forward(uw, _oracle_arch(arch), u, 400, ids, seq, pooled)
    alpha, _, _, latents = op.finish(out, u, a)
    want_image = op.display(ovae.decode(vw, latents))
    want_alpha = op.bilinear_8x(alpha, hgt, wid)

    got_image = res.image.cpu().numpy()
    got_la = res.latent_alpha.cpu().numpy()
    assert got_image.shape == (b, 3, hgt, wid) and np.all((got_image >= 0) & (got_image <= 1))
    # Three 16-bit models in a chain (encoder, UNet, decoder): the UNet's own
    # bound against its oracle is 1e-2 (f16) / 5e-2 (bf16) relative L2.
    rel = {"f16": 2e-2, "bf16": 8e-2}[dt]
    assert workloads.rel_l2(got_la, alpha) <= rel
    assert workloads.rel_l2(res.alpha.cpu().numpy(), want_alpha) <= rel
    assert workloads.psnr(got_image, want_image, peak_to_peak=1.0) >= {"f16": 35.0, "bf16": 30.0}[dt]
    model.close()
