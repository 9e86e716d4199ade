"""Generates the golden fixtures of tests/golden/ from the CPU oracle.

The oracle restates the reference's CPU F32 path (oracle/); the fixtures let
the GPU tests check the benchmark-size decoder input without re-running the
oracle for minutes. Run from the repository root:

    python tests/golden/make_golden.py
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


def main():
    w = random_vae_weights(0)
    t = time.time()
    lat = workloads.decoder_latents(1, 64, 64, seed=42)
    out = vae.decode(w, lat)
    np.savez_compressed(os.path.join(HERE, "decoder_d1.npz"), image=out.astype(np.float16),
                        latents_sum=np.float64(lat.sum()))
    print("decoder D1", out.shape, f"{time.time() - t:.1f}s", out.std())
    t = time.time()
    img, _ = workloads.encoder_image(1, 256, 256, seed=7)
    mom = vae.encode_moments(w, img)
    np.savez_compressed(os.path.join(HERE, "encoder_256.npz"), moments=mom.astype(np.float32),
                        image_sum=np.float64(img.sum()))
    print("encoder 256", mom.shape, f"{time.time() - t:.1f}s", mom.std())


if __name__ == "__main__":
    main()
