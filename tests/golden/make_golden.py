"""Generates the golden fixtures of tests/golden/ from the CPU oracle.

The oracle restates the reference's CPU F32 path (oracle/); the fixtures let
the GPU tests check the benchmark-size decoder and encoder without re-running
the oracle for minutes on the GPU host. Run from the repository root:

    python tests/golden/make_golden.py            # every fixture
    python tests/golden/make_golden.py d4 e4      # only the named ones

Fixtures:
  decoder_d1.npz  D1 decode [1,4,64,64] -> [1,3,512,512] (seed 42): the
                  whole image in f16, plus the f32 sample below.
  decoder_d4.npz  one image of the headline decode, [1,4,128,128] ->
                  [1,3,1024,1024] (seed 42), in f32: a strided sample that
                  visits every (row mod 8, column mod 8) phase of the three
                  nearest-2x upsamplings, three 64 x 64 crops (top-left and
                  bottom-right corners, centre) and per-channel moments of
                  the whole image.
  encoder_256.npz encoder [1,3,256,256] (seed 7) -> moments, f32.
  encoder_e4.npz  one image of the encoder config, [1,3,1024,1024] (seed 7,
                  9x9 box blur) -> moments [1,8,128,128], f32, whole.
"""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "osor-rs_b200"))

from oracle import vae  # noqa: E402
from osor_b200 import workloads  # noqa: E402
from osor_b200.weights import random_vae_weights  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CROP = 64


def sample_index(size: int):
    """Row and column indices of the strided sample of a size x size image:
    row i is 8i + i % 8 and its column j is 8j + (i + j) % 8, so every one of
    the 64 (row mod 8, column mod 8) phases occurs."""
    n = size // 8
    i = np.arange(n)
    rows = 8 * i + i % 8
    cols = 8 * i[None, :] + (i[:, None] + i[None, :]) % 8
    return rows.astype(np.int32), cols.astype(np.int32)


def image_sample(img: np.ndarray) -> dict:
    """[3, S, S] f32 image -> the sample, crops and moments stored per fixture."""
    s = img.shape[-1]
    rows, cols = sample_index(s)
    sub = img[:, rows[:, None], cols]
    mid = s // 2 - CROP // 2
    return {
        "sample": sub.astype(np.float32),
        "rows": rows, "cols": cols,
        "crop_top_left": img[:, :CROP, :CROP].astype(np.float32),
        "crop_bottom_right": img[:, s - CROP:, s - CROP:].astype(np.float32),
        "crop_centre": img[:, mid:mid + CROP, mid:mid + CROP].astype(np.float32),
        "crop_centre_at": np.int32(mid),
        "channel_mean": img.reshape(3, -1).astype(np.float64).mean(axis=1),
        "channel_std": img.reshape(3, -1).astype(np.float64).std(axis=1),
    }


def d1(w):
    lat = workloads.decoder_latents(1, 64, 64, seed=42)
    out = vae.decode(w, lat)
    np.savez_compressed(os.path.join(HERE, "decoder_d1.npz"), image=out.astype(np.float16),
                        latents_sum=np.float64(lat.sum()),
                        **{"f32_" + k: v for k, v in image_sample(out[0]).items()})
    return out


def d4(w):
    lat = workloads.decoder_latents(1, 128, 128, seed=42)
    out = vae.decode(w, lat)
    np.savez_compressed(os.path.join(HERE, "decoder_d4.npz"), latents_sum=np.float64(lat.sum()),
                        **image_sample(out[0]))
    return out


def e256(w):
    img, _ = workloads.encoder_image(1, 256, 256, seed=7)
    mom = vae.encode_moments(w, img)
    np.savez_compressed(os.path.join(HERE, "encoder_256.npz"), moments=mom.astype(np.float32),
                        image_sum=np.float64(img.sum()))
    return mom


def e4(w):
    img, noise = workloads.encoder_image(1, 1024, 1024, seed=7)
    mom = vae.encode_moments(w, img)
    np.savez_compressed(os.path.join(HERE, "encoder_e4.npz"), moments=mom.astype(np.float32),
                        image_sum=np.float64(img.sum()), noise_sum=np.float64(noise.sum()))
    return mom


MAKERS = {"d1": d1, "d4": d4, "e256": e256, "e4": e4}


def main(names):
    w = random_vae_weights(0)
    for name in names or list(MAKERS):
        t = time.time()
        out = MAKERS[name](w)
        print(name, out.shape, f"{time.time() - t:.1f}s", float(out.std()), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
