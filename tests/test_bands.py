"""Row-band split of the decoder across ranks, on CPU ranks over gloo.

Each rank of a K-rank group decodes its row band of one image through
``BandDecoder`` with an oracle-backed op set (NHWC float64 activations, the
oracle's convolution / upsample / attention, GroupNorm applied from the merged
band statistics). The bands, gathered in rank order, must equal the oracle's
whole-image decode: the halo exchange, the statistics merge and the key /
value gather are then what the one-image decode computes. The reference's own
check of this property is band independence of its banded convolution
(src/native/conv.rs:297-383).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from oracle import vae as ovae
from osor_b200.bands import BandDecoder, BandEncoder
from osor_b200.weights import random_vae_weights

CHANNELS = (32, 32, 64, 64)
LAYERS = 1


class OracleBandOps:
    """BandDecoder backend over the oracle: NHWC activations are float64
    tensors, NCHW latents / RGB float32 (the dtype tells the layouts apart)."""

    def __init__(self, weights):
        self.w = weights

    def empty(self, shape, f32=False):
        return torch.empty(shape, dtype=torch.float32 if f32 else torch.float64)

    def zeros(self, shape, f32=False):
        return torch.zeros(shape, dtype=torch.float32 if f32 else torch.float64)

    @staticmethod
    def _nchw(x):
        if x.dtype == torch.float32:
            return x.numpy()
        return np.ascontiguousarray(x.permute(0, 3, 1, 2).numpy().astype(np.float32))

    @staticmethod
    def _nhwc(y):
        return torch.from_numpy(np.ascontiguousarray(y.transpose(0, 2, 3, 1))).double()

    def conv(self, name, x, residual=None, out=None, out_nchw=False):
        wt = self.w[name + ".weight"]
        if wt.ndim == 2:
            wt = wt.reshape(wt.shape[0], wt.shape[1], 1, 1)
        y = oracle.conv2d(self._nchw(x), wt, self.w[name + ".bias"], stride=1,
                          padding=wt.shape[-1] // 2)
        if out_nchw:
            return torch.from_numpy(y)
        y = self._nhwc(y)
        if residual is not None:
            y = y + residual
        if out is not None:
            out.copy_(y)
            return out
        return y

    def conv_down(self, name, x, out):
        y = oracle.conv2d(oracle.pad_right_bottom(self._nchw(x)), self.w[name + ".weight"],
                          self.w[name + ".bias"], stride=2, padding=0)
        out.copy_(self._nhwc(y))
        return out

    def qkv(self, prefix, h):
        b, r, w, c = h.shape
        xs = h.reshape(b * r * w, c).numpy().astype(np.float32)
        parts = []
        for name in ("to_q", "to_k", "to_v"):
            wt = self.w[f"{prefix}.{name}.weight"].reshape(c, c)
            y = oracle.sgemm(xs, np.ascontiguousarray(wt.T)) + self.w[f"{prefix}.{name}.bias"]
            if name != "to_v":
                y = y * np.float32(float(c) ** -0.25)
            parts.append(y)
        return torch.from_numpy(np.concatenate(parts, axis=1).reshape(b, r, w, 3 * c)).double()

    def upsample(self, x):
        return self._nhwc(oracle.upsample_2x(self._nchw(x)))

    def gn_stats(self, name, x):
        b, r, w, c = x.shape
        g = x.reshape(b, r * w, 32, c // 32).permute(0, 2, 1, 3).reshape(b, 32, -1)
        mean = g.mean(dim=2)
        var = ((g - mean[:, :, None]) ** 2).mean(dim=2)
        return torch.stack([mean, var], dim=2).float()

    def gn_apply(self, name, x, part_stats, silu, out):
        b, r, w, c = x.shape
        ps = part_stats.double()
        mean = ps[..., 0].mean(dim=0)
        var = (ps[..., 1] + (ps[..., 0] - mean) ** 2).mean(dim=0)
        cpg = c // 32
        mean_c = mean.repeat_interleave(cpg, dim=1)[:, None, None, :]
        rstd_c = (1.0 / torch.sqrt(var + oracle.EPS)).repeat_interleave(cpg, dim=1)[:, None, None, :]
        gamma = torch.from_numpy(self.w[name + ".weight"]).double()
        beta = torch.from_numpy(self.w[name + ".bias"]).double()
        y = (x - mean_c) * rstd_c * gamma + beta
        if silu:
            y = y * torch.sigmoid(y)
        if out is None:
            return y
        out.copy_(y)
        return out

    def attend(self, q, k, v):
        qn = q.numpy().astype(np.float32)
        kt = np.ascontiguousarray(k.numpy().astype(np.float32).transpose(0, 2, 1))
        return torch.from_numpy(oracle.attend(qn, kt, v.numpy().astype(np.float32))).double()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, h, w, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        weights = random_vae_weights(3, CHANNELS, LAYERS, parts=("decoder",))
        rng = np.random.default_rng(11)
        latents = torch.from_numpy(rng.standard_normal((1, 4, h, w)).astype(np.float32))
        dec = BandDecoder(OracleBandOps(weights), CHANNELS, LAYERS)
        band = dec.decode(latents)
        parts = [torch.empty_like(band) for _ in range(world)]
        dist.all_gather(parts, band)
        if rank == 0:
            np.save(os.path.join(out_dir, "bands.npy"), torch.cat(parts, dim=2).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,h,w", [(2, 8, 8), (3, 6, 4)])
def test_band_split_decode_matches_whole_image(world, h, w, tmp_path):
    mp.start_processes(_rank_main, args=(world, _free_port(), h, w, str(tmp_path)),
                       nprocs=world, start_method="spawn")
    got = np.load(tmp_path / "bands.npy")
    weights = random_vae_weights(3, CHANNELS, LAYERS, parts=("decoder",))
    latents = np.random.default_rng(11).standard_normal((1, 4, h, w)).astype(np.float32)
    want = ovae.decode(weights, latents, CHANNELS, LAYERS)
    assert got.shape == want.shape == (1, 3, 8 * h, 8 * w)
    # f32 oracle ops on bands vs the whole image: only summation order differs.
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())


def _encoder_rank_main(rank, world, port, h, w, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        weights = random_vae_weights(3, CHANNELS, LAYERS, parts=("encoder",))
        rng = np.random.default_rng(12)
        image = torch.from_numpy(rng.uniform(-1, 1, (1, 3, h, w)).astype(np.float32))
        band = BandEncoder(OracleBandOps(weights), CHANNELS, LAYERS).encode_moments(image)
        parts = [torch.empty_like(band) for _ in range(world)]
        dist.all_gather(parts, band)
        if rank == 0:
            np.save(os.path.join(out_dir, "moments.npy"), torch.cat(parts, dim=2).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,h,w", [(2, 64, 48), (4, 64, 32)])
def test_band_split_encode_matches_whole_image(world, h, w, tmp_path):
    """Band rows halve at each stride-2 downsampler, whose last output row reads
    the halo row below the band (vae_encoder.rs:206-210)."""
    mp.start_processes(_encoder_rank_main, args=(world, _free_port(), h, w, str(tmp_path)),
                       nprocs=world, start_method="spawn")
    got = np.load(tmp_path / "moments.npy")
    weights = random_vae_weights(3, CHANNELS, LAYERS, parts=("encoder",))
    image = np.random.default_rng(12).uniform(-1, 1, (1, 3, h, w)).astype(np.float32)
    want = ovae.encode_moments(weights, image, CHANNELS, LAYERS)
    assert got.shape == want.shape == (1, 8, h // 8, w // 8)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())


def test_band_split_rejects_uneven_bands():
    dec = BandDecoder(OracleBandOps({}), CHANNELS, LAYERS)
    dec.k = 3
    with pytest.raises(Exception, match="divide evenly"):
        dec.decode(torch.zeros((1, 4, 8, 8)))
