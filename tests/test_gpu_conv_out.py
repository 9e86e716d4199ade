"""The decoder's fused conv_norm_out + SiLU + conv_out kernel (conv_out.cu)
against the oracle at shapes that exercise its edges: widths that leave a
partial 128-pixel tile (72, 104, 640 pixels), one-tile and eight-tile rows,
CTA bands that cross image boundaries (batch 3 with fewer rows than CTAs
per image), and the unfused path (OSOR_FUSED_CONV_OUT=0, read once per
process) in a child process for comparison.

Reference: VaeDecoder::forward's last two layers (src/native/vae_decoder.rs:112-113).
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle.vae as ovae
from osor_b200 import workloads
from osor_b200.model import NativeModel, device_status
from osor_b200.weights import random_vae_weights
from tolerances import MAX_ABS, MIN_PSNR_DB

pytestmark = pytest.mark.gpu

# (batch, latent h, latent w)
SHAPES = [(1, 9, 13), (3, 4, 80), (2, 16, 16), (1, 8, 128)]


@pytest.fixture(scope="module")
def weights():
    return random_vae_weights(0, parts=("decoder",))


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_fused_conv_out_decode_matches_oracle(shape, dt, weights, cuda_device):
    b, h, w = shape
    model = NativeModel(weights, device=0, parts=("decoder",), dtype=dt)
    lat = workloads.decoder_latents(b, h, w, seed=42)
    got = model.decode(torch.from_numpy(lat).cuda()).cpu().numpy()
    model.close()
    assert device_status(0) == 0
    want = ovae.decode(weights, lat)
    assert got.shape == want.shape
    assert np.all(np.isfinite(got))
    err = float(np.abs(got - want).max())
    assert err <= MAX_ABS[dt], err
    assert workloads.psnr(got, want) >= MIN_PSNR_DB


def test_unfused_path_gives_the_same_image(cuda_device):
    """The same decodes with OSOR_FUSED_CONV_OUT=0 (separate GroupNorm apply and
    pixels-on-N conv_out): both round the normalized activation to 16 bits
    before the products, so they differ by f32 summation order only."""
    code = (
        "import sys, numpy as np, torch\n"
        "sys.path[:0] = sys.argv[1:3]\n"
        "from osor_b200 import workloads\n"
        "from osor_b200.model import NativeModel\n"
        "from osor_b200.weights import random_vae_weights\n"
        "m = NativeModel(random_vae_weights(0, parts=('decoder',)), device=0, parts=('decoder',),"
        " dtype='f16')\n"
        "lat = workloads.decoder_latents(3, 4, 80, seed=42)\n"
        "np.save(sys.argv[3], m.decode(torch.from_numpy(lat).cuda()).cpu().numpy())\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = [root, os.path.join(root, "osor-rs_b200")]
    outs = []
    for flag in ("1", "0"):
        path = os.path.join("/tmp", f"osor_conv_out_{os.getpid()}_{flag}.npy")
        env = dict(os.environ, OSOR_FUSED_CONV_OUT=flag)
        r = subprocess.run([sys.executable, "-c", code, *paths, path], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(path))
        os.remove(path)
    fused, unfused = outs
    assert np.abs(fused - unfused).max() <= 2e-4
