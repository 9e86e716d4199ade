"""The 16-bit format floor of the decoder on this random-init model (CPU).

oracle.precision runs the oracle's decoder with the weights and every stored
activation rounded to bf16 or f16 and everything else in F32 - a decoder that
stores 16-bit activations, as the CUDA decoder does and as the reference's
CUDA backend does for a BF16 or F16 model (src/runtime.rs:406-417). Its
distance from the F32 oracle is the format's floor, independent of any
kernel. Measured on a [1,4,32,32] -> [1,3,256,256] decode (seed 42):

  f16   max-abs 5.8e-3, 65.8 dB: inside the 2e-2 / 40 dB acceptance bound.
  bf16  max-abs 4.5e-2, 47.9 dB: the max-abs bound is out of reach of any
        decoder that stores bf16 activations on this model; the error enters
        at every block (relative L2 2.9e-3 after conv_in, growing to 9.8e-3
        at the output: a trace in the manner of the reference's
        precision_tests.rs:97-130), and rounding only the weights already
        gives 1.7e-2. The GPU tests therefore hold bf16 to 40 dB and an 8e-2
        max-abs bound, and the benchmark's headline runs f16.
"""
import numpy as np
import pytest

from oracle import precision, vae
from osor_b200 import workloads
from osor_b200.weights import random_vae_weights


@pytest.fixture(scope="module")
def traced():
    w = random_vae_weights(0, parts=("decoder",))
    lat = workloads.decoder_latents(1, 32, 32, seed=42)
    ref_trace = {}
    ref = vae.decode(w, lat, observer=lambda n, t: ref_trace.__setitem__(n, t.copy()))
    return w, lat, ref, ref_trace


def _emulate(traced, dtype):
    w, lat, ref, ref_trace = traced
    trace = {}
    got = precision.decode(w, lat, dtype, observer=lambda n, t: trace.__setitem__(n, t.copy()))
    errors = {n: workloads.rel_l2(trace[n], ref_trace[n]) for n in ref_trace}
    return got, errors


def test_f16_floor_is_inside_the_acceptance_bound(traced):
    got, errors = _emulate(traced, "f16")
    ref = traced[2]
    assert np.abs(got - ref).max() <= 1e-2
    assert workloads.psnr(got, ref) >= 60.0
    assert max(errors.values()) <= 2e-3


def test_bf16_floor_exceeds_the_max_abs_bound_at_every_block(traced):
    got, errors = _emulate(traced, "bf16")
    ref = traced[2]
    err = float(np.abs(got - ref).max())
    # The format alone moves the worst pixel past 2e-2 (measured 4.5e-2) while
    # PSNR stays well above 40 dB.
    assert 2e-2 < err <= 8e-2, err
    assert workloads.psnr(got, ref) >= 45.0
    names = list(errors)
    assert names[0] == "post_quant_conv" and errors[names[0]] == 0.0  # f32 on the GPU too
    # Error enters at the first 16-bit layer and grows through the blocks.
    assert errors["decoder.conv_in"] > 1e-3
    assert errors["decoder.conv_out"] > errors["decoder.conv_in"]
    assert errors["decoder.conv_out"] <= 2e-2
