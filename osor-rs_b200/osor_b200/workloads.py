"""Seeded synthetic inputs of the benchmark configurations (no datasets).

Every generator uses numpy's PCG64 with the seed the configuration names, so
the parity tests, the golden fixtures and the benchmark see the same values.

  decoder_latents   SDXL VAE decoder input: standard normal [B, 4, h, w]
                    (seed 42), divided by the latent scale 0.13025 because
                    Pipeline::run decodes blend / 0.13025 (src/pipeline.rs:834-837).
  encoder_image     [B, 3, H, W] uniform [0, 1], 9x9 box blur with reflect
                    padding, mapped to [-1, 1] as Pipeline::run does before
                    encode_moments (src/pipeline.rs:720); posterior noise
                    standard normal [B, 4, H/8, W/8] (seed 7 for both, image
                    drawn first).
  groupnorm_inputs  x ~ N(0.5, 2.0), gamma ~ N(1, 0.1), beta ~ N(0, 0.1), seed 3.
  conv_inputs       x ~ N(0, 1), w ~ N(0, sqrt(2 / (9 Cin))), bias ~ U(+-1/sqrt(Cin)),
                    residual ~ N(0, 1), seed 5.
  inpaint_job       the end-to-end inpainting job: image [B, 3, H, W] uniform [0, 1]
                    with the 9x9 box blur (display range, as Osor::infer takes it),
                    and a binary mask [B, 1, H, W] holding one axis-aligned rectangle
                    per image that covers 10-25 % of its area at a seeded position
                    (seed 5); the noise comes from the reference's seeded_noise.
"""
from __future__ import annotations

import numpy as np

LATENT_SCALE = 0.13025


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def decoder_latents(batch: int = 1, h: int = 64, w: int = 64, seed: int = 42) -> np.ndarray:
    z = _rng(seed).standard_normal((batch, 4, h, w), dtype=np.float32)
    return (z / np.float32(LATENT_SCALE)).astype(np.float32)


def box_blur_9(img: np.ndarray) -> np.ndarray:
    """9x9 mean filter per channel with reflect padding (separable)."""
    pad = 4
    x = np.pad(img, ((0, 0), (0, 0), (pad, pad), (pad, pad)), mode="reflect").astype(np.float64)
    c = np.cumsum(x, axis=2)
    c = np.concatenate([np.zeros_like(c[:, :, :1]), c], axis=2)
    x = (c[:, :, 9:] - c[:, :, :-9]) / 9.0
    c = np.cumsum(x, axis=3)
    c = np.concatenate([np.zeros_like(c[:, :, :, :1]), c], axis=3)
    x = (c[:, :, :, 9:] - c[:, :, :, :-9]) / 9.0
    return x.astype(np.float32)


def encoder_image(batch: int = 4, h: int = 1024, w: int = 1024, seed: int = 7):
    """Returns (normalized image in [-1, 1], posterior noise)."""
    rng = _rng(seed)
    img = rng.random((batch, 3, h, w), dtype=np.float32)
    img = box_blur_9(img)
    noise = rng.standard_normal((batch, 4, h // 8, w // 8), dtype=np.float32)
    return (img * 2.0 - 1.0).astype(np.float32), noise


def inpaint_job(batch: int = 4, h: int = 1024, w: int = 1024, seed: int = 5):
    """Returns (image in [0, 1], mask in {0, 1}) for Osor::infer
    (src/runtime.rs:484; InferenceInput, src/pipeline.rs:139-157)."""
    rng = _rng(seed)
    img = box_blur_9(rng.random((batch, 3, h, w), dtype=np.float32))
    img = np.clip(img, 0.0, 1.0).astype(np.float32)
    mask = np.zeros((batch, 1, h, w), np.float32)
    for b in range(batch):
        area = rng.uniform(0.10, 0.25)
        aspect = rng.uniform(0.5, 2.0)
        rh = int(min(h, max(8, round(np.sqrt(area * h * w * aspect)))))
        rw = int(min(w, max(8, round(area * h * w / rh))))
        y0 = int(rng.integers(0, h - rh + 1))
        x0 = int(rng.integers(0, w - rw + 1))
        mask[b, 0, y0:y0 + rh, x0:x0 + rw] = 1.0
    return img, mask


def groupnorm_inputs(shape, seed: int = 3):
    rng = _rng(seed)
    x = rng.normal(0.5, 2.0, size=shape).astype(np.float32)
    c = shape[1]
    gamma = rng.normal(1.0, 0.1, size=c).astype(np.float32)
    beta = rng.normal(0.0, 0.1, size=c).astype(np.float32)
    return x, gamma, beta


def conv_inputs(batch: int, cin: int, cout: int, h: int, w: int, seed: int = 5):
    rng = _rng(seed)
    x = rng.standard_normal((batch, cin, h, w), dtype=np.float32)
    wt = (rng.standard_normal((cout, cin, 3, 3), dtype=np.float32)
          * np.float32(np.sqrt(2.0 / (9 * cin))))
    bound = 1.0 / np.sqrt(cin)
    bias = rng.uniform(-bound, bound, size=cout).astype(np.float32)
    res = rng.standard_normal((batch, cout, h, w), dtype=np.float32)
    return x, wt, bias, res


def vae_decoder_flops(batch: int, h: int, w: int, channels=(128, 256, 512, 512),
                      layers: int = 2) -> float:
    """Algorithmic FLOPs of VaeDecoder::forward (src/native/vae_decoder.rs:104-114)
    on [batch, 4, h, w] latents: every convolution at its nominal 2 * pixels *
    Cin * Cout * k^2 (the upsamplers' 3x3 convs at the upsampled resolution,
    as the reference runs them), the mid-block's q / k / v / out projections
    and one Q K^T and one P V per image."""
    def conv(px, cin, cout, k):
        return 2.0 * px * cin * cout * k * k

    def resnet(px, cin, cout):
        f = conv(px, cin, cout, 3) + conv(px, cout, cout, 3)
        return f + (conv(px, cin, cout, 1) if cin != cout else 0.0)

    n = h * w
    c = channels[-1]
    f = conv(batch * n, 4, 4, 1) + conv(batch * n, 4, c, 3)
    f += 2 * resnet(batch * n, c, c) + batch * (8.0 * n * c * c + 4.0 * n * n * c)
    rev = list(reversed(channels))
    px, cin = batch * n, c
    for i, cout in enumerate(rev):
        for j in range(layers + 1):
            f += resnet(px, cin if j == 0 else cout, cout)
        cin = cout
        if i + 1 < len(rev):
            px *= 4
            f += conv(px, cout, cout, 3)
    return f + conv(px, channels[0], 3, 3)


def psnr(got: np.ndarray, want: np.ndarray, peak_to_peak: float = 2.0) -> float:
    """PSNR in dB for raw RGB in [-1, 1] (peak-to-peak 2)."""
    mse = float(np.mean((np.asarray(got, np.float64) - np.asarray(want, np.float64)) ** 2))
    if mse == 0.0:
        return float("inf")
    return 10.0 * np.log10(peak_to_peak ** 2 / mse)


def rel_l2(got: np.ndarray, want: np.ndarray) -> float:
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    return float(np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30))
