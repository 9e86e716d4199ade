"""Oracle for the DDPM scheduler and the pipeline's latent-space stages
(TEST INFRASTRUCTURE ONLY).

Restates, in numpy float32 with one rounding per operation (numpy neither
fuses nor reorders these element-wise operations):
  Scheduler::new alphas      src/scheduler.rs:128-221
  add_noise                  src/scheduler.rs:284-297
  predicted_original_sample  src/scheduler.rs:311-339
  pipeline stages            src/pipeline.rs:733-856
  bilinear_8x                src/pipeline.rs:862-896
"""
from __future__ import annotations

import math

import numpy as np

f32 = np.float32


def alphas_cumprod(num_train_timesteps=1000, beta_start=0.00085, beta_end=0.012,
                   beta_schedule="scaled_linear", trained_betas=None):
    n = num_train_timesteps
    if beta_schedule == "scaled_linear":
        start, end = f32(math.sqrt(beta_start)), f32(math.sqrt(beta_end))
    else:
        start, end = f32(beta_start), f32(beta_end)
    step = f32(0.0) if n == 1 else f32(end - start) / f32(n - 1)
    alpha = 1.0
    out = np.empty(n, np.float32)
    for i in range(n):
        if trained_betas is not None:
            beta = f32(trained_betas[i])
        else:
            # f32 fused multiply-add: the f64 product of two f32 values and the
            # f64 sum with an f32 of nearby magnitude are exact here, so one
            # rounding to f32 reproduces fmaf.
            if i < n // 2 or n == 1:
                point = f32(float(step) * float(i) + float(start))
            else:
                point = f32(-float(step) * float(n - i - 1) + float(end))
            beta = point * point if beta_schedule == "scaled_linear" else point
        alpha *= float(f32(1.0) - beta)
        out[i] = f32(alpha)
    return out


def scales(alpha_t):
    a = f32(alpha_t)
    return np.sqrt(a), np.sqrt(f32(1.0) - a)


def add_noise(original, noise, alpha_t):
    os_, ns = scales(alpha_t)
    return (np.asarray(original, f32) * os_ + np.asarray(noise, f32) * ns).astype(f32)


def predicted_original(noisy, out, alpha_t, kind="epsilon", clip=False, clip_range=1.0):
    os_, ns = scales(alpha_t)
    noisy, out = np.asarray(noisy, f32), np.asarray(out, f32)
    if kind == "epsilon":
        p = (noisy - out * ns) / os_
    elif kind == "sample":
        p = out.copy()
    else:
        p = noisy * os_ - out * ns
    if clip:
        p = np.clip(p, f32(-clip_range), f32(clip_range))
    return p.astype(f32)


def prepare(moments, posterior_noise, diffusion_noise, mask, alpha_t, scaling=0.13025):
    moments = np.asarray(moments, f32)
    mean = moments[:, :4]
    logvar = np.clip(moments[:, 4:], f32(-30.0), f32(20.0))
    sample = mean + np.exp(logvar * f32(0.5)) * np.asarray(posterior_noise, f32)
    original = (sample * f32(scaling)).astype(f32)
    b, _, h, w = original.shape
    pooled = np.asarray(mask, f32).reshape(b, 1, h, 8, w, 8).max(axis=(3, 5))
    noisy = add_noise(original, diffusion_noise, alpha_t)
    return np.concatenate([noisy, pooled, original], axis=1).astype(f32), sample.astype(f32)


def sigmoid(x):
    x = np.asarray(x, f32)
    return (f32(1.0) / (np.exp(-x) + f32(1.0))).astype(f32)


def finish(unet_output, unet_input, alpha_t, kind="epsilon", clip=False, clip_range=1.0,
           scaling=0.13025):
    unet_output = np.asarray(unet_output, f32)
    alpha = sigmoid(unet_output[:, 4:5])
    noisy, original = unet_input[:, :4], unet_input[:, 5:]
    pred = predicted_original(noisy, unet_output[:, :4], alpha_t, kind, clip, clip_range)
    blend = (alpha * pred + (alpha * f32(-1.0) + f32(1.0)) * original).astype(f32)
    latents = (blend * f32(1.0 / scaling)).astype(f32)
    return alpha, pred, blend, latents


def _axis_weights(source, target):
    lo, hi, wt = [], [], []
    for i in range(target):
        x = min(max((i + 0.5) * source / target - 0.5, 0.0), float(source - 1))
        left = math.floor(x)
        lo.append(left)
        hi.append(min(left + 1, source - 1))
        wt.append(f32(x - left))
    return np.array(lo), np.array(hi), np.array(wt, f32)


def bilinear_8x(x, height, width):
    x = np.asarray(x, f32)
    _, _, h, w = x.shape
    lo, hi, wt = _axis_weights(h, height)
    wt = wt.reshape(1, 1, -1, 1)
    v = x[:, :, lo, :] * (wt * f32(-1.0) + f32(1.0)) + x[:, :, hi, :] * wt
    lo, hi, wt = _axis_weights(w, width)
    wt = wt.reshape(1, 1, 1, -1)
    return (v[:, :, :, lo] * (wt * f32(-1.0) + f32(1.0)) + v[:, :, :, hi] * wt).astype(f32)


def display(decoded):
    return np.clip(np.asarray(decoded, f32) * f32(0.5) + f32(0.5), f32(0.0), f32(1.0))
