"""Per-block precision trace of the GPU decoder against the oracle.

The layer-by-layer decoder (osor_b200.bands.BandDecoder on one rank, every
layer a C-ABI call) reports each block's output under the reference's VAE
trace names (src/native/precision_tests.rs:97-130); each is compared with the
F32 oracle's block output (relative L2) and with the 16-bit emulation of
oracle.precision, which rounds the weights and stored activations and nothing
else. A GPU error at or below the emulation's at every block shows that the
kernels add nothing beyond the storage format: for bf16 the format's floor
(about 4.5e-2 max-abs on this model at 256 x 256, above the 2e-2 acceptance
bound, see tests/test_precision.py), for f16 well inside it.
"""
import numpy as np
import pytest
import torch

from oracle import precision, vae
from osor_b200 import workloads
from osor_b200.bands import BandDecoder, CudaBandOps
from osor_b200.model import device_status
from osor_b200.weights import random_vae_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def reference():
    w = random_vae_weights(0, parts=("decoder",))
    lat = workloads.decoder_latents(1, 32, 32, seed=42)
    trace = {}
    out = vae.decode(w, lat, observer=lambda n, t: trace.__setitem__(n, t.copy()))
    return w, lat, out, trace


def _nchw(name, t):
    t = t.float()
    if name in ("post_quant_conv", "decoder.conv_out"):
        return t.cpu().numpy()
    return t.permute(0, 3, 1, 2).contiguous().cpu().numpy()


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_block_trace_matches_the_format_floor(dt, reference, cuda_device):
    w, lat, ref, ref_trace = reference
    emu_trace = {}
    emu = precision.decode(w, lat, dt, observer=lambda n, t: emu_trace.__setitem__(n, t.copy()))
    dtype = torch.float16 if dt == "f16" else torch.bfloat16
    dec = BandDecoder(CudaBandOps(w, device="cuda", dtype=dtype))
    gpu_trace = {}
    got = dec.decode(torch.from_numpy(lat).cuda(),
                     observer=lambda n, t: gpu_trace.__setitem__(n, _nchw(n, t)))
    got = got.cpu().numpy()
    assert device_status(0) == 0
    assert list(gpu_trace) == list(ref_trace)
    one_rounding = 2.0 ** -11 if dt == "f16" else 2.0 ** -8
    rows = []
    for name in ref_trace:
        g = workloads.rel_l2(gpu_trace[name], ref_trace[name])
        e = workloads.rel_l2(emu_trace[name], ref_trace[name])
        rows.append((name, g, e))
        # Kernel arithmetic (f32 accumulation order, fused epilogues) may add a
        # little on top of the format's rounding, never a multiple of it. One
        # more rounding is allowed for: this layer-by-layer decoder runs
        # post_quant_conv with 16-bit weights (the fused decoder keeps it f32).
        assert g <= 1.5 * e + one_rounding, (name, g, e)
    print("\n".join(f"{dt} {n:28s} gpu {g:.2e}  emulated {e:.2e}" for n, g, e in rows))
    err, emu_err = float(np.abs(got - ref).max()), float(np.abs(emu - ref).max())
    assert err <= 1.5 * emu_err, (err, emu_err)
    assert workloads.psnr(got, ref) >= 40.0
    if dt == "f16":
        assert err <= 2e-2
