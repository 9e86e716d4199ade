"""Host mirror of the reference's inference pipeline around the VAE
(src/pipeline.rs:655-860) and its DDPM scheduler (src/scheduler.rs).

``Pipeline.run`` follows ``Pipeline::run``: normalise the image, encode the
posterior moments, sample the posterior, scale to the original latent,
max-pool the mask, noise the latent at the pinned timestep, call the
denoiser on the nine-channel UNet input, turn its output into the latent
alpha and the predicted original, blend, decode, and map the image and the
alpha to display space. The VAE runs through ``NativeModel``; every other
stage is one CUDA kernel of the library (``osor_pipeline_*``), in f32. The
denoiser (the SDXL inpainting UNet in the reference) is the caller's: any
callable ``denoise(unet_input, timestep, time_ids) -> [B, 5, h, w]``.
"""
from __future__ import annotations

import ctypes
import enum
import math
from dataclasses import dataclass
from typing import Callable, NamedTuple, Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import InvalidInput, check
from .model import CancellationToken, NativeModel

PREDICTION_TYPES = {"epsilon": 0, "sample": 1, "v_prediction": 2}
BETA_SCHEDULES = {"linear": 0, "scaled_linear": 1}
MAX_SCHEDULER_ELEMENTS = 16 * 1024 * 1024


class Unavailable(RuntimeError):
    """A configuration the reference also declines (Error::Unavailable)."""


@dataclass
class SchedulerConfig:
    """scheduler.rs:6-50 (diffusers names and defaults)."""
    num_train_timesteps: int = 1000
    beta_start: float = 0.00085
    beta_end: float = 0.012
    beta_schedule: str = "scaled_linear"
    trained_betas: Optional[Sequence[float]] = None
    prediction_type: str = "epsilon"
    clip_sample: bool = False
    clip_sample_range: float = 1.0
    thresholding: bool = False
    dynamic_thresholding_ratio: float = 0.995
    sample_max_value: float = 1.0


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


class Scheduler:
    """Precomputed cumulative alphas (Scheduler::new, scheduler.rs:128-221)
    and the two DDPM formulas the pipeline uses."""

    def __init__(self, config: SchedulerConfig = None):
        c = config or SchedulerConfig()
        bad = lambda m: InvalidInput(f"scheduler: {m}")  # noqa: E731
        if not (1 <= c.num_train_timesteps <= 100_000):
            raise bad("num_train_timesteps must be in 1..=100000")
        if not all(math.isfinite(v) and 0.0 <= v < 1.0 for v in (c.beta_start, c.beta_end)):
            raise bad("betas must be finite and in [0, 1)")
        if (not math.isfinite(c.clip_sample_range) or c.clip_sample_range <= 0.0
                or not math.isfinite(c.dynamic_thresholding_ratio)
                or not 0.0 <= c.dynamic_thresholding_ratio <= 1.0
                or not math.isfinite(c.sample_max_value) or c.sample_max_value < 1.0):
            raise bad("invalid clipping or thresholding parameters")
        if c.thresholding:
            raise Unavailable("DDPM dynamic thresholding is not implemented")
        if c.prediction_type not in PREDICTION_TYPES:
            raise bad("unsupported prediction_type")
        if c.beta_schedule not in BETA_SCHEDULES:
            raise bad("unsupported beta_schedule")
        betas = None
        if c.trained_betas is not None:
            betas = np.ascontiguousarray(c.trained_betas, np.float64)
            if betas.size != c.num_train_timesteps:
                raise bad("trained_betas must match num_train_timesteps and be finite in [0, 1)")
        self.config = c
        self.alphas_cumprod = np.empty(c.num_train_timesteps, np.float32)
        check(_lib.lib().osor_scheduler_alphas(
            c.num_train_timesteps, float(c.beta_start), float(c.beta_end),
            BETA_SCHEDULES[c.beta_schedule], None if betas is None else betas.ctypes.data,
            self.alphas_cumprod.ctypes.data))

    def alpha(self, timestep: int) -> float:
        if not 0 <= timestep < self.alphas_cumprod.size:
            raise InvalidInput("scheduler timestep out of range")
        return float(self.alphas_cumprod[timestep])

    @staticmethod
    def _pair(a: torch.Tensor, b: torch.Tensor, check_finite: bool) -> None:
        if a.shape != b.shape or a.dtype != b.dtype or a.device != b.device:
            raise InvalidInput("scheduler tensors must have matching shape, dtype, and device")
        if a.dtype != torch.float32 or not a.is_cuda:
            raise InvalidInput("scheduler tensors must be float32 CUDA tensors")
        if a.numel() > MAX_SCHEDULER_ELEMENTS:
            raise InvalidInput("scheduler tensor exceeds safety limit")
        if check_finite and not bool(torch.isfinite(a).all() & torch.isfinite(b).all()):
            raise InvalidInput("scheduler tensors must contain finite values")

    def add_noise(self, original, noise, timestep: int, check_finite: bool = True):
        """original * sqrt(a) + noise * sqrt(1 - a) (scheduler.rs:278-297)."""
        self._pair(original, noise, check_finite)
        a = self.alpha(timestep)
        # Contiguous copies stay referenced until the kernel is enqueued, so
        # the allocator cannot hand their memory to the next copy first.
        original, noise = original.contiguous(), noise.contiguous()
        out = torch.empty_like(original)
        check(_lib.lib().osor_scheduler_add_noise(_ptr(original), _ptr(noise), _ptr(out),
                                                  original.numel(), a, _stream(original)))
        return out

    def predicted_original_sample(self, noisy, model_output, timestep: int,
                                  check_finite: bool = True):
        """scheduler.rs:299-339."""
        self._pair(noisy, model_output, check_finite)
        a = self.alpha(timestep)
        c = self.config
        noisy, model_output = noisy.contiguous(), model_output.contiguous()
        out = torch.empty_like(noisy)
        check(_lib.lib().osor_scheduler_predicted_original(
            _ptr(noisy), _ptr(model_output), _ptr(out), noisy.numel(), a,
            PREDICTION_TYPES[c.prediction_type], 1 if c.clip_sample else 0,
            float(c.clip_sample_range), _stream(noisy)))
        return out


class Stage(enum.Enum):
    """Observer stages in order (pipeline.rs:162-199); the prompt-embedding
    stages belong to the caller's denoiser and are not emitted here."""
    PosteriorMoments = 0
    PosteriorMean = 1
    PosteriorLogvar = 2
    PosteriorSample = 3
    OriginalLatent = 4
    PooledMask = 5
    NoisyLatent = 6
    UnetInput = 7
    TimeIds = 10
    DenoisingOutput = 11
    AlphaLogits = 12
    LatentAlpha = 13
    PredictedOriginal = 14
    BlendedLatent = 15
    DecodedImage = 16
    Alpha = 17


class InferenceResult(NamedTuple):
    image: torch.Tensor         # [B, 3, H, W] in [0, 1]
    alpha: torch.Tensor         # [B, 1, H, W]
    latent_alpha: torch.Tensor  # [B, 1, H/8, W/8]


Denoiser = Callable[[torch.Tensor, int, torch.Tensor], torch.Tensor]


class Pipeline:
    """Pipeline::run (pipeline.rs:655-860) with the VAE on ``model`` and the
    caller's ``denoise``."""

    def __init__(self, model: NativeModel, denoise: Denoiser,
                 scheduler: Optional[Scheduler] = None, timestep: int = 400,
                 vae_scaling_factor: float = 0.13025):
        if not (math.isfinite(vae_scaling_factor) and vae_scaling_factor > 0.0):
            raise InvalidInput("vae_scaling_factor must be finite and positive")
        self.model = model
        self.denoise = denoise
        self.scheduler = scheduler or Scheduler()
        self.timestep = int(timestep)
        self.alpha_t = self.scheduler.alpha(self.timestep)
        self.vae_scaling_factor = float(vae_scaling_factor)

    def _check(self, t, name, shape, value_range=None):
        if not torch.is_tensor(t) or tuple(t.shape) != tuple(shape):
            raise InvalidInput(f"{name} must have shape {list(shape)}")
        if t.dtype != torch.float32 or t.device != self.model.device or not t.is_contiguous():
            raise InvalidInput(f"{name} must be a contiguous float32 tensor on {self.model.device}")
        if not bool(torch.isfinite(t).all()):
            raise InvalidInput(f"{name} must contain finite values")
        if value_range is not None:
            lo, hi = value_range
            if not bool(((t >= lo) & (t <= hi)).all()):
                raise InvalidInput(f"{name} values must be in [{lo}, {hi}]")

    def run(self, image, mask, posterior_noise, diffusion_noise,
            observer: Optional[Callable[[Stage, torch.Tensor], None]] = None,
            cancellation: Optional[CancellationToken] = None) -> InferenceResult:
        def checkpoint():
            if cancellation is not None and cancellation.is_cancelled():
                raise _lib.Cancelled("inference was cancelled")

        def emit(stage, tensor):
            if observer is not None:
                checkpoint()
                observer(stage, tensor)

        checkpoint()
        if not torch.is_tensor(image) or image.ndim != 4:
            raise InvalidInput("image must have shape [B,3,H,W]")
        b, ch, hgt, wid = image.shape
        ok = lambda a: 32 <= a <= 1024 and a % 8 == 0  # noqa: E731
        if not (1 <= b <= 4) or ch != 3 or not ok(hgt) or not ok(wid):
            raise InvalidInput("image dimensions or batch exceed limits; H and W must be "
                               "multiples of 8 in 32..=1024")
        h, w = hgt // 8, wid // 8
        self._check(image, "image", (b, 3, hgt, wid), (0.0, 1.0))
        self._check(mask, "mask", (b, 1, hgt, wid), (0.0, 1.0))
        self._check(posterior_noise, "posterior_noise", (b, 4, h, w))
        self._check(diffusion_noise, "diffusion_noise", (b, 4, h, w))
        lib, dev, s = _lib.lib(), self.model.device, _stream(image)
        f32 = dict(dtype=torch.float32, device=dev)

        normalized = torch.empty_like(image)
        check(lib.osor_pipeline_normalize_image(_ptr(image), _ptr(normalized), b, hgt, wid, s))
        moments = self.model.encode_moments(normalized, cancellation)
        emit(Stage.PosteriorMoments, moments)
        if observer is not None:
            emit(Stage.PosteriorMean, moments[:, :4])
            emit(Stage.PosteriorLogvar, moments[:, 4:].clamp(-30.0, 20.0))
        unet_input = torch.empty((b, 9, h, w), **f32)
        sample = torch.empty((b, 4, h, w), **f32) if observer is not None else None
        check(lib.osor_pipeline_prepare(
            _ptr(moments), _ptr(posterior_noise), _ptr(diffusion_noise), _ptr(mask),
            _ptr(unet_input), None if sample is None else _ptr(sample), b, hgt, wid,
            self.alpha_t, self.vae_scaling_factor, s))
        if observer is not None:
            emit(Stage.PosteriorSample, sample)
            emit(Stage.OriginalLatent, unet_input[:, 5:])
            emit(Stage.PooledMask, unet_input[:, 4:5])
            emit(Stage.NoisyLatent, unet_input[:, :4])
            emit(Stage.UnetInput, unet_input)
        time_ids = torch.tensor([[hgt, wid, 0.0, 0.0, hgt, wid]], **f32).repeat(b, 1)
        emit(Stage.TimeIds, time_ids)
        checkpoint()
        output = self.denoise(unet_input, self.timestep, time_ids)
        self._check(output, "denoiser output", (b, 5, h, w))
        emit(Stage.DenoisingOutput, output[:, :4])
        emit(Stage.AlphaLogits, output[:, 4:5])
        latent_alpha = torch.empty((b, 1, h, w), **f32)
        latents = torch.empty((b, 4, h, w), **f32)
        predicted = blend = None
        if observer is not None:
            predicted = torch.empty((b, 4, h, w), **f32)
            blend = torch.empty((b, 4, h, w), **f32)
        c = self.scheduler.config
        check(lib.osor_pipeline_finish(
            _ptr(output), _ptr(unet_input), _ptr(latent_alpha),
            None if predicted is None else _ptr(predicted), None if blend is None else _ptr(blend),
            _ptr(latents), b, hgt, wid, self.alpha_t, PREDICTION_TYPES[c.prediction_type],
            1 if c.clip_sample else 0, float(c.clip_sample_range), self.vae_scaling_factor, s))
        emit(Stage.LatentAlpha, latent_alpha)
        if observer is not None:
            emit(Stage.PredictedOriginal, predicted)
            emit(Stage.BlendedLatent, blend)
        decoded = self.model.decode(latents, cancellation)
        image_out = torch.empty((b, 3, hgt, wid), **f32)
        alpha = torch.empty((b, 1, hgt, wid), **f32)
        check(lib.osor_pipeline_map(_ptr(decoded), _ptr(latent_alpha), _ptr(image_out),
                                    _ptr(alpha), b, hgt, wid, s))
        emit(Stage.DecodedImage, image_out)
        emit(Stage.Alpha, alpha)
        return InferenceResult(image_out, alpha, latent_alpha)
