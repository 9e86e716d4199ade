"""Attention parity: softmax(q k^T) v on the GPU against the oracle's sliced
F32 attention (src/native/attention.rs:27-84) on bf16-representable inputs.
Shapes cover the tensor-core path (tokens % 128 == 0) and the CUDA-core path
the reference's own small shapes take (vae_encoder.rs:497: 5x7 and 11x13
tokens, 32 channels)."""
import numpy as np
import pytest
import torch

import oracle
from osor_b200 import ops

pytestmark = pytest.mark.gpu




CASES = [
    (1, 256, 512),    # tensor-core scores / values, VAE width
    (2, 384, 128),
    (2, 35, 32),      # reference batch test shapes, CUDA-core path
    (4, 143, 32),
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_attend_matches_oracle(case, dt, cuda_device):
    b, n, d = case
    rng = np.random.default_rng(11)

    def half(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt)

    # Logit spread like the VAE's (q and k scaled by d^-1/4 each).
    q = half(rng.standard_normal((b, n, d)) * d ** -0.25 * 1.4)
    k = half(rng.standard_normal((b, n, d)) * d ** -0.25 * 1.4)
    v = half(rng.standard_normal((b, n, d)))
    got = ops.attend(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
    want = oracle.attend(qf, np.ascontiguousarray(kf.transpose(0, 2, 1)), vf)
    err = np.abs(got - want)
    # bf16 probabilities (relative 2^-9) and bf16 output rounding.
    assert err.max() <= 2e-2, err.max()
    assert np.sqrt((err ** 2).mean()) <= 3e-3
