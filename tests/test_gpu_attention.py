"""Attention parity: softmax(q k^T) v on the GPU against the oracle's sliced
F32 attention (src/native/attention.rs:27-84) on bf16-representable inputs.
Shapes cover the tensor-core path (tokens % 128 == 0) and the CUDA-core path
the reference's own small shapes take (vae_encoder.rs:497: 5x7 and 11x13
tokens, 32 channels)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle
from osor_b200 import ops

pytestmark = pytest.mark.gpu




CASES = [
    (1, 256, 512),    # three-kernel path (the pair kernel takes n_kv % 512 == 0)
    (2, 1024, 512),   # pair kernel, two pairs of key tiles, two images
    (3, 512, 512),    # pair kernel, three images
    (3, 4096, 512),   # pair kernel: 96 tasks, more than the resident clusters take at once
    (1, 512, 256),    # three-kernel path (the pair kernel takes width 512 only)
    (2, 384, 128),    # three-kernel tensor-core path
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


# (batch, n_q, n_kv, D): queries against a different number of keys, as a row
# band's queries attend to the whole image (the band split): pair kernel for
# n_q % 128 == 0 and n_kv % 512 == 0, the three-kernel path otherwise.
KV_CASES = [(1, 256, 1024, 512), (2, 384, 512, 512), (1, 128, 2048, 512), (1, 256, 768, 512)]


@pytest.mark.parametrize("case", KV_CASES, ids=lambda c: "x".join(map(str, c)))
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_attend_kv_matches_oracle(case, dt, cuda_device):
    b, nq, nkv, d = case
    rng = np.random.default_rng(nq + nkv)

    def half(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt)

    q = half(rng.standard_normal((b, nq, d)) * d ** -0.25 * 1.4)
    k = half(rng.standard_normal((b, nkv, d)) * d ** -0.25 * 1.4)
    v = half(rng.standard_normal((b, nkv, d)))
    got = ops.attend_kv(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
    want = oracle.attend(qf, np.ascontiguousarray(kf.transpose(0, 2, 1)), vf)
    err = np.abs(got - want)
    assert got.shape == (b, nq, d)
    assert err.max() <= 2e-2, err.max()
    assert np.sqrt((err ** 2).mean()) <= 3e-3


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_fused_attention_rescales_growing_maxima(dt, cuda_device):
    """Logits that grow along the keys (up to ~40 in natural units) for every
    other query row and shrink for the rest, so within each warp some rows'
    running maximum jumps by more than 2^8 across key tiles (the fused
    kernels rescale their output accumulator) while the others keep theirs."""
    b, n, d = 1, 1024, 512
    rng = np.random.default_rng(3)

    def half(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt)

    e = rng.standard_normal(d)
    e /= np.linalg.norm(e)
    sign = np.where(np.arange(n) % 2 == 0, 1.0, -1.0)[None, :, None]
    q = half(sign * e * 2.0 + 0.05 * rng.standard_normal((b, n, d)))
    ramp = (np.arange(n) / n * 20.0)[None, :, None]
    k = half(e[None, None, :] * ramp + 0.05 * rng.standard_normal((b, n, d)))
    v = half(rng.standard_normal((b, n, d)))
    got = ops.attend(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
    want = oracle.attend(qf, np.ascontiguousarray(kf.transpose(0, 2, 1)), vf)
    err = np.abs(got - want)
    assert np.all(np.isfinite(got))
    assert err.max() <= 2e-2, err.max()


def _rerun_in_child(env_overrides):
    env = dict(os.environ, **env_overrides)
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-q", "-p", "no:cacheprovider",
                        "-k", "attend_matches_oracle or attend_kv_matches or rescales_growing_maxima"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_single_cta_fused_kernel_runs_the_same_cases(cuda_device):
    """By default width-512 attention with tokens % 256 == 0 runs on the CTA
    pair kernel (attn_pair.cu). The single-CTA fused kernel is opt-in
    (OSOR_PAIR_ATTENTION=0 and OSOR_FUSED_ATTENTION=1, read once per process):
    run this file's oracle cases again in a child process with it selected
    (tokens % 256 == 0 and D of 256 or 512 take it)."""
    _rerun_in_child({"OSOR_PAIR_ATTENTION": "0", "OSOR_FUSED_ATTENTION": "1"})


def test_three_kernel_path_runs_the_same_cases(cuda_device):
    """The three-kernel path (scores with softmax statistics, probabilities,
    P V) that the pair kernel replaced, in a child process with
    OSOR_PAIR_ATTENTION=0."""
    _rerun_in_child({"OSOR_PAIR_ATTENTION": "0", "OSOR_FUSED_ATTENTION": "0"})
