"""Row-band decoding and encoding on the GPU: the band entry points of the C
ABI against the oracle, and the band decoder / encoder against the oracle's
whole-image results (one rank on one GPU; two ranks over NCCL when two GPUs
are visible).

* osor_group_norm_stats + osor_group_norm_apply over the row bands of one
  image, with the bands' statistics merged by the apply, equal the oracle's
  whole-image GroupNorm (src/native/vae_encoder.rs:55-81) to 16-bit output
  rounding.
* osor_attention_kv (n_q query rows against n_kv keys / values, strided
  column slices of one q|k|v projection) equals the oracle's attention
  (src/native/attention.rs:27-84) to 16-bit rounding, on the tensor-core path
  (row counts multiples of 128) and the CUDA-core path.
* BandDecoder's RGB meets the decoder's acceptance bounds against the oracle,
  and BandEncoder's moments the encoder's (relative L2 <= 1e-2).
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "osor-rs_b200")):
    if _p not in sys.path:  # also run as a script, one rank of the two-GPU check
        sys.path.insert(0, _p)

import oracle
import oracle.vae as ovae
from osor_b200 import ops, workloads
from osor_b200.bands import BandDecoder, BandEncoder, CudaBandOps
from osor_b200.model import device_status
from osor_b200.weights import random_vae_weights

pytestmark = pytest.mark.gpu

# RGB acceptance per dtype, as for the whole-image decoder (bf16's 8-bit
# mantissa sets its worst pixel near 4e-2 on random-init weights).
MAX_ABS = {torch.float16: 2e-2, torch.bfloat16: 8e-2}


def _round(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dt).float().numpy()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("bands,h,w,c", [(2, 64, 64, 128), (4, 32, 256, 256), (3, 24, 40, 64)])
def test_group_norm_band_statistics_merge(cuda_device, dt, bands, h, w, c):
    rng = np.random.default_rng(bands)
    x = _round(rng.standard_normal((1, c, h, w)) * 2.0 + 0.5, dt)
    gamma = rng.uniform(0.5, 1.5, c).astype(np.float32)
    beta = rng.uniform(-0.2, 0.2, c).astype(np.float32)
    want = oracle.group_norm(x, gamma, beta, silu=True)
    gn = ops.StableGroupNorm(gamma, beta)
    xt = ops.nchw_to_nhwc(torch.from_numpy(x).cuda(), dt)
    r = h // bands
    parts = torch.stack([gn.stats(xt[:, i * r:(i + 1) * r].contiguous()) for i in range(bands)])
    got = torch.cat([gn.apply(xt[:, i * r:(i + 1) * r].contiguous(), parts, True)
                     for i in range(bands)], dim=1)
    torch.cuda.synchronize()
    got = ops.nhwc_to_nchw(got).cpu().numpy()
    # 16-bit output rounding (bf16: relative 2^-8) plus statistics order.
    err = np.abs(got - want)
    assert np.all(err <= 2 ** -8 * np.abs(want) + 1e-3), err.max()


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("n_q,n_kv,d", [(256, 1024, 512), (128, 512, 128), (32, 96, 64)])
def test_attention_kv_matches_oracle(cuda_device, dt, n_q, n_kv, d):
    rng = np.random.default_rng(n_q + d)
    scale = float(d) ** -0.25
    qkv = _round(rng.standard_normal((n_kv, 3 * d)) * scale * 2.0, dt)
    q0 = 3 * (n_kv - n_q) // 4 // 8 * 8  # a band in the middle of the keys
    q = qkv[q0:q0 + n_q, :d]
    k, v = qkv[:, d:2 * d], qkv[:, 2 * d:]
    want = oracle.attend(q[None], np.ascontiguousarray(k.T)[None], v[None])[0]
    t = torch.from_numpy(qkv).to(dt).cuda()
    got = ops.attend_kv(t[None, q0:q0 + n_q, :d], t[None, :, d:2 * d], t[None, :, 2 * d:])
    torch.cuda.synchronize()
    got = got[0].float().cpu().numpy()
    # 16-bit probabilities and output, fp32 statistics (the square-attention bounds).
    err = np.abs(got - want)
    assert err.max() <= 2e-2, err.max()
    assert np.sqrt((err ** 2).mean()) <= 3e-3


def _weights():
    return random_vae_weights(0, parts=("decoder",))


def test_band_decoder_one_rank_matches_oracle(cuda_device):
    weights = _weights()
    lat = workloads.decoder_latents(1, 16, 16, seed=42)
    dec = BandDecoder(CudaBandOps(weights, dtype=torch.float16))
    got = dec.decode(torch.from_numpy(lat).cuda())
    assert device_status(0) == 0
    got = got.cpu().numpy()
    want = ovae.decode(weights, lat)
    assert np.all(np.isfinite(got))
    assert np.abs(got - want).max() <= MAX_ABS[torch.float16]
    assert workloads.psnr(got, want) >= 40.0


def test_band_encoder_one_rank_matches_oracle(cuda_device):
    weights = random_vae_weights(0, parts=("encoder",))
    img, _ = workloads.encoder_image(1, 128, 128, seed=5)
    got = BandEncoder(CudaBandOps(weights, dtype=torch.float16)).encode_moments(
        torch.from_numpy(img).cuda())
    assert device_status(0) == 0
    want = ovae.encode_moments(weights, img)
    assert workloads.rel_l2(got.cpu().numpy(), want) <= 1e-2


def test_native_band_decoder_one_rank_matches_oracle(cuda_device):
    """osor_vae_decode_band on a group of one rank (the band is the whole
    image): the tiny shape against the oracle, the headline's 128 x 128
    latents against the whole-image decode."""
    from osor_b200.bands import NativeBandDecoder
    from osor_b200.model import NativeModel
    weights = _weights()
    m = NativeModel(weights, device=0, parts=("decoder",), dtype="f16")
    dec = NativeBandDecoder(m)
    lat = workloads.decoder_latents(1, 16, 16, seed=42)
    got = dec.decode(torch.from_numpy(lat).cuda()).cpu().numpy()
    assert device_status(0) == 0
    want = ovae.decode(weights, lat)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= MAX_ABS[torch.float16]
    assert workloads.psnr(got, want) >= 40.0
    big = torch.from_numpy(workloads.decoder_latents(1, 128, 128, seed=42)).cuda()
    band = dec.decode(big)
    whole = m.decode(big)
    torch.cuda.synchronize()
    assert device_status(0) == 0
    diff = (band - whole).abs().max().item()
    assert diff <= 2e-2, diff
    assert workloads.psnr(band.cpu().numpy(), whole.cpu().numpy()) >= 45.0
    dec.close()
    m.close()


def _native_main(out_path: str) -> None:
    """One rank of the two-GPU native band check: the tiny decode and the
    128 x 128 decode through osor_vae_decode_band, gathered on rank 0, with
    rank 0's whole-image decode of the latter for comparison."""
    import torch.distributed as dist
    from datetime import timedelta
    from osor_b200.bands import NativeBandDecoder
    from osor_b200.model import NativeModel
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        m = NativeModel(_weights(), device=local, parts=("decoder",), dtype="f16")
        dec = NativeBandDecoder(m)
        outs = []
        for size in (16, 128):
            lat = torch.from_numpy(workloads.decoder_latents(1, size, size, seed=42)).to(dev)
            band = dec.decode(lat)
            every = torch.empty((dist.get_world_size(),) + tuple(band.shape), device=dev)
            dist.all_gather_into_tensor(every, band.contiguous())
            outs.append(torch.cat(list(every), dim=2).cpu().numpy())
            if size == 128 and dist.get_rank() == 0:
                outs.append(m.decode(lat).cpu().numpy())
        assert device_status(local) == 0
        if dist.get_rank() == 0:
            np.save(out_path, outs[0])
            np.save(out_path + ".big.npy", outs[1])
            np.save(out_path + ".whole.npy", outs[2])
        dec.close()
        m.close()
    finally:
        dist.destroy_process_group()


def _rank_main(out_path: str) -> None:
    """One rank of the two-GPU check (run under torch.distributed.run)."""
    import torch.distributed as dist
    from datetime import timedelta
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    try:
        lat = workloads.decoder_latents(1, 16, 16, seed=42)
        dec = BandDecoder(CudaBandOps(_weights(), device=f"cuda:{local}",
                                      dtype=torch.float16))
        band = dec.decode(torch.from_numpy(lat).cuda())
        every = torch.empty((dist.get_world_size(),) + tuple(band.shape), device=band.device)
        dist.all_gather_into_tensor(every, band)
        img, _ = workloads.encoder_image(1, 128, 128, seed=5)
        enc = BandEncoder(CudaBandOps(random_vae_weights(0, parts=("encoder",)),
                                      device=f"cuda:{local}", dtype=torch.float16))
        mband = enc.encode_moments(torch.from_numpy(img).cuda())
        mevery = torch.empty((dist.get_world_size(),) + tuple(mband.shape), device=mband.device)
        dist.all_gather_into_tensor(mevery, mband)
        if dist.get_rank() == 0:
            np.save(out_path, torch.cat(list(every), dim=2).cpu().numpy())
            np.save(out_path + ".moments.npy", torch.cat(list(mevery), dim=2).cpu().numpy())
        dec.close()
        enc.close()
    finally:
        dist.destroy_process_group()


def _exchange_main() -> None:
    """One rank of the peer-exchange check: osor_band_halo and osor_band_gather
    against the rows and statistics the neighbours hold, eagerly (three calls,
    both slot parities) and replayed from a CUDA graph (the epochs advance on
    the device)."""
    import torch.distributed as dist
    from datetime import timedelta
    from osor_b200.bands import PeerExchange
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        k, rank = dist.get_world_size(), dist.get_rank()
        r, w, c = 6, 40, 96
        ex = PeerExchange(None, dev, w * c * 2)

        def band(seed):
            t = torch.arange((r + 2) * w * c, device=dev, dtype=torch.float32).reshape(1, r + 2, w, c)
            return ((t + 1000 * rank + 7 * seed) % 2039).to(torch.float16)

        def expect(seed, x):
            ref_up = ((torch.arange((r + 2) * w * c, device=dev, dtype=torch.float32)
                       .reshape(1, r + 2, w, c) + 1000 * (rank - 1) + 7 * seed) % 2039).half()
            ref_dn = ((torch.arange((r + 2) * w * c, device=dev, dtype=torch.float32)
                       .reshape(1, r + 2, w, c) + 1000 * (rank + 1) + 7 * seed) % 2039).half()
            top = ref_up[:, r] if rank > 0 else torch.zeros_like(x[:, 0])
            bottom = ref_dn[:, 1] if rank + 1 < k else torch.zeros_like(x[:, 0])
            assert torch.equal(x[:, 0], top), (rank, seed, "top")
            assert torch.equal(x[:, r + 1], bottom), (rank, seed, "bottom")
            assert torch.equal(x[:, 1:r + 1], band(seed)[:, 1:r + 1])

        for seed in range(3):
            x = band(seed)
            ex.halo(x)
            expect(seed, x)
            st = torch.full((32, 2), float(rank * 10 + seed), device=dev)
            got = ex.gather(st)
            for q in range(k):
                assert torch.all(got[q] == q * 10 + seed), (rank, seed, q)
        # Captured once, replayed twice.
        xs = band(5)
        st = torch.full((32, 2), float(rank * 10 + 5), device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                ex.halo(xs)
                gathered = ex.gather(st)
        torch.cuda.current_stream(dev).wait_stream(s)
        for _ in range(2):
            xs.copy_(band(5))
            xs[:, 0].fill_(-1.0)
            xs[:, r + 1].fill_(-1.0)
            g.replay()
            torch.cuda.synchronize(dev)
            expect(5, xs)
            for q in range(k):
                assert torch.all(gathered[q] == q * 10 + 5)
        del g
        from osor_b200.model import device_status
        assert device_status(local) == 0
        ex.close()
    finally:
        dist.destroy_process_group()


def _two_gpu_run(script_args, port, extra_env=None):
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={port}", __file__] + script_args
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", **(extra_env or {}))
    return subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=os.path.dirname(HERE))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_two_gpus():
    r = _two_gpu_run(["--exchange"], 29533)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("p2p", ["1", "0"], ids=["peer", "nccl"])
def test_band_decoder_two_gpus_matches_oracle(tmp_path, p2p):
    """The band decoder and encoder on two GPUs, with the halo rows and
    statistics exchanged by peer stores (default) or by NCCL
    (OSOR_BAND_P2P=0)."""
    out = str(tmp_path / "bands.npy")
    r = _two_gpu_run([out], 29531 if p2p == "1" else 29532, {"OSOR_BAND_P2P": p2p})
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    got = np.load(out)
    lat = workloads.decoder_latents(1, 16, 16, seed=42)
    want = ovae.decode(_weights(), lat)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= MAX_ABS[torch.float16]
    assert workloads.psnr(got, want) >= 40.0
    moments = np.load(out + ".moments.npy")
    img, _ = workloads.encoder_image(1, 128, 128, seed=5)
    want_m = ovae.encode_moments(random_vae_weights(0, parts=("encoder",)), img)
    assert moments.shape == want_m.shape
    assert workloads.rel_l2(moments, want_m) <= 1e-2


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_native_band_decoder_two_gpus_matches_oracle(tmp_path):
    """osor_vae_decode_band on two GPUs: the gathered bands of the tiny decode
    against the oracle, those of the 128 x 128 decode against the whole-image
    decode."""
    out = str(tmp_path / "native.npy")
    r = _two_gpu_run(["--native", out], 29534)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    got = np.load(out)
    lat = workloads.decoder_latents(1, 16, 16, seed=42)
    want = ovae.decode(_weights(), lat)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= MAX_ABS[torch.float16]
    assert workloads.psnr(got, want) >= 40.0
    big, whole = np.load(out + ".big.npy"), np.load(out + ".whole.npy")
    assert big.shape == whole.shape == (1, 3, 1024, 1024)
    assert np.abs(big - whole).max() <= 2e-2
    assert workloads.psnr(big, whole) >= 45.0


if __name__ == "__main__":
    if sys.argv[1] == "--exchange":
        _exchange_main()
    elif sys.argv[1] == "--native":
        _native_main(sys.argv[2])
    else:
        _rank_main(sys.argv[1])
