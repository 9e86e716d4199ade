"""DDPM scheduler and pipeline-stage host logic, on CPU.

The cumulative alphas come from the library's host function
(osor_scheduler_alphas); they must equal the oracle's restatement of
Scheduler::new (src/scheduler.rs:128-221), and the oracle's add_noise /
predicted_original_sample must reproduce the reference's pinned f32 results
(scheduler.rs:348-372: PyTorch 2.7.1 / diffusers 0.35.1 captures).
"""
import math

import numpy as np
import pytest

from oracle import pipeline as op
from osor_b200._lib import InvalidInput
from osor_b200.pipeline import Scheduler, SchedulerConfig, Unavailable

SAMPLE = np.array([2.0, -3.0, 0.01, 100.0], np.float32)
NOISE = np.array([0.5, 0.125, 2.0, -4.0], np.float32)
PINNED_NOISY = [0x3FD7579C, 0xBFEE0C04, 0x3FC30AF8, 0x427878A8]
PINNED_PREDICTED = [0x401F33BD, 0xC0980129, 0xC0140F51, 0x431E24DD]


def test_oracle_reproduces_pinned_scheduler_values():
    a = op.alphas_cumprod()[400]
    assert list(op.add_noise(SAMPLE, NOISE, a).view(np.uint32)) == PINNED_NOISY
    assert list(op.predicted_original(SAMPLE, NOISE, a).view(np.uint32)) == PINNED_PREDICTED


@pytest.mark.parametrize("cfg", [SchedulerConfig(),
                                 SchedulerConfig(beta_schedule="linear", beta_start=1e-4,
                                                 beta_end=0.02),
                                 SchedulerConfig(num_train_timesteps=7),
                                 SchedulerConfig(num_train_timesteps=1, trained_betas=[0.1])])
def test_library_alphas_equal_oracle(cfg):
    got = Scheduler(cfg).alphas_cumprod
    want = op.alphas_cumprod(cfg.num_train_timesteps, cfg.beta_start, cfg.beta_end,
                             cfg.beta_schedule, cfg.trained_betas)
    np.testing.assert_array_equal(got, want)


def test_ddpm_predictions_and_clipping_oracle():
    """scheduler.rs:374-416 with one trained beta of 0.1."""
    a = op.alphas_cumprod(1, trained_betas=[0.1])[0]
    x, n = np.array([2.0], np.float32), np.array([0.5], np.float32)
    assert abs(float(op.add_noise(x, n, a)[0]) - (2 * math.sqrt(0.9) + 0.5 * math.sqrt(0.1))) < 1e-6
    for kind, want in [("epsilon", 2 / math.sqrt(0.9) - 0.5 * math.sqrt(0.1 / 0.9)),
                       ("sample", 0.5), ("v_prediction", 2 * math.sqrt(0.9) - 0.5 * math.sqrt(0.1))]:
        assert abs(float(op.predicted_original(x, n, a, kind)[0]) - want) < 1e-6
    assert abs(float(op.predicted_original(x, n, a, "epsilon", True, 0.4)[0]) - 0.4) < 1e-6


@pytest.mark.parametrize("kw", [dict(num_train_timesteps=0), dict(num_train_timesteps=100_001),
                                dict(beta_start=1.0), dict(beta_end=float("nan")),
                                dict(clip_sample_range=0.0), dict(sample_max_value=0.5),
                                dict(dynamic_thresholding_ratio=1.5),
                                dict(prediction_type="flow"), dict(beta_schedule="cosine"),
                                dict(num_train_timesteps=2, trained_betas=[0.1]),
                                dict(num_train_timesteps=1, trained_betas=[1.0])])
def test_invalid_scheduler_configurations(kw):
    with pytest.raises(InvalidInput):
        Scheduler(SchedulerConfig(**kw))


def test_thresholding_is_unavailable():
    with pytest.raises(Unavailable):
        Scheduler(SchedulerConfig(thresholding=True))


def test_timestep_out_of_range():
    with pytest.raises(InvalidInput):
        Scheduler().alpha(1000)


def test_bilinear_weights_follow_align_corners_false():
    # 2 -> 16 rows: the first and last four rows clamp to the edges.
    x = np.array([[[[0.0], [1.0]]]], np.float32)
    y = op.bilinear_8x(np.repeat(x, 2, axis=3), 16, 16)[0, 0, :, 0]
    np.testing.assert_array_equal(y[:4], 0.0)
    np.testing.assert_array_equal(y[-4:], 1.0)
    assert np.all(np.diff(y) >= 0)
