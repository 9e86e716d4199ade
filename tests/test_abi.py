"""The C-ABI library loads, exports every function include/osor_b200.h
declares, and validates arguments on the host (no device work here)."""
import ctypes
import os
import re

import numpy as np
import pytest

from osor_b200 import _lib
from osor_b200 import ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "osor_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(osor_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    assert "osor_vae_decode" in names and "osor_conv2d" in names
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_no_error_initially():
    lb = _lib.lib()
    assert lb.osor_version() >= 100
    assert _lib.last_error() == ""


def test_pack_conv_weight_layout():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((5, 6, 3, 3)).astype(np.float32)
    import torch
    for dt in (torch.bfloat16, torch.float16):
        packed = ops.pack_conv_weight(w, dt)
        want = torch.from_numpy(w).permute(0, 2, 3, 1).reshape(5, 54).to(dt)
        np.testing.assert_array_equal(packed, want.view(torch.int16).numpy().view(np.uint16))


def test_invalid_arguments_fail_before_device_work():
    lb = _lib.lib()
    rc = lb.osor_conv2d(None, None, None, None, None, 1, 8, 8, 4, 4, 3, 1, 1, 1, 0, 0, 0, None)
    assert rc == _lib.OSOR_ERR_INVALID_INPUT
    assert "null" in _lib.last_error()
    with pytest.raises(_lib.InvalidInput):
        _lib.check(lb.osor_pack_conv_weight(None, None, 0, 1, 3, 0))
    f32, nchw, nhwc = _lib.DTYPE_F32, _lib.LAYOUT_NCHW, _lib.LAYOUT_NHWC
    assert lb.osor_group_norm_workspace_size(1, 48, 4, 4, nchw, f32) == 0
    assert lb.osor_group_norm_workspace_size(1, 64, 4, 4, nchw, f32) > 0
    assert lb.osor_group_norm_workspace_size(1, 64, 4, 4, nhwc, f32) == 0
    assert lb.osor_group_norm_workspace_size(1, 64, 4, 4, nhwc, _lib.DTYPE_F16) > 0
    assert lb.osor_vae_workspace_size(None, _lib.OP_DECODE, 1, 64, 64) == 0
    # Seeded noise admission (noise.rs:115-126): batch 1..4, axes multiples of
    # 8 in 32..1024, dtype F32/F16/BF16; rejected before any device work.
    dummy = ctypes.c_void_p(256)
    for batch, h, w, dt in [(0, 32, 32, f32), (5, 32, 32, f32), (1, 33, 32, f32),
                            (1, 32, 1032, f32), (1, 24, 32, f32), (1, 32, 32, 7)]:
        assert lb.osor_seeded_noise(1, batch, h, w, dt, dummy, dummy, None) == \
            _lib.OSOR_ERR_INVALID_INPUT


def test_band_pipeline_and_scheduler_entry_points_validate_on_the_host():
    """The entry points added for the band split, the pipeline stages and the
    scheduler refuse bad arguments before any device work."""
    lb = _lib.lib()
    d = ctypes.c_void_p(256)
    f16 = _lib.DTYPE_F16
    bad = _lib.OSOR_ERR_INVALID_INPUT
    # GroupNorm statistics / merged apply: channels % 32, parts >= 1, nulls.
    assert lb.osor_group_norm_stats(d, 1, 48, 4, 4, f16, d, d, 1 << 20, None) == bad
    assert lb.osor_group_norm_stats(None, 1, 64, 4, 4, f16, d, d, 1 << 20, None) == bad
    assert lb.osor_group_norm_apply(d, d, d, d, d, 0, 1, 64, 4, 4, f16, 1e-6, 1, d, 1 << 20,
                                    None) == bad
    assert lb.osor_group_norm_apply(d, d, d, d, d, 2, 1, 64, 4, 4, f16, 1e-6, 1, d, 16,
                                    None) == bad  # workspace below B * C * 16 bytes
    # Rectangular attention: dim <= 512, strides >= dim, 16-bit only.
    assert lb.osor_attention_kv(d, 64, d, d, 64, d, 1, 8, 16, 1024, f16, d, 1 << 30, None) == bad
    assert lb.osor_attention_kv(d, 32, d, d, 64, d, 1, 8, 16, 64, f16, d, 1 << 30, None) == bad
    assert lb.osor_attention_kv(d, 64, d, d, 64, d, 1, 8, 16, 64, _lib.DTYPE_F32, d, 1 << 30,
                                None) == bad
    assert lb.osor_attention_kv_workspace_size(1, 8, 16, 64) > 0
    assert lb.osor_attention_kv_workspace_size(1, 0, 16, 64) == 0
    # Pipeline stages: admission limits, cumulative alpha, prediction type.
    assert lb.osor_pipeline_prepare(d, d, d, d, d, None, 5, 64, 64, 0.4, 0.13025, None) == bad
    assert lb.osor_pipeline_prepare(d, d, d, d, d, None, 1, 60, 64, 0.4, 0.13025, None) == bad
    assert lb.osor_pipeline_prepare(d, d, d, d, d, None, 1, 64, 64, 0.0, 0.13025, None) == bad
    assert lb.osor_pipeline_prepare(d, d, d, d, d, None, 1, 64, 64, 0.4, -1.0, None) == bad
    assert lb.osor_pipeline_finish(d, d, d, None, None, d, 1, 64, 64, 0.4, 3, 0, 1.0, 0.13025,
                                   None) == bad
    assert lb.osor_pipeline_finish(d, d, d, None, None, d, 1, 64, 64, 0.4, 0, 1, 0.0, 0.13025,
                                   None) == bad
    assert lb.osor_pipeline_map(d, d, d, None, 1, 64, 64, None) == bad
    assert lb.osor_pipeline_normalize_image(d, d, 1, 1032, 64, None) == bad
    # Scheduler formulas: element limit and alpha range.
    assert lb.osor_scheduler_add_noise(d, d, d, 0, 0.4, None) == bad
    assert lb.osor_scheduler_add_noise(d, d, d, 16 * 1024 * 1024 + 1, 0.4, None) == bad
    assert lb.osor_scheduler_predicted_original(d, d, d, 4, 1.5, 0, 0, 1.0, None) == bad
    # Cumulative alphas are host work: they run here.
    out = np.empty(3, np.float32)
    assert lb.osor_scheduler_alphas(3, 0.1, 0.2, 0, None, out.ctypes.data) == _lib.OSOR_OK
    assert np.all(np.diff(out) < 0) and 0 < out[-1] < out[0] < 1
    assert lb.osor_scheduler_alphas(3, 0.1, 0.2, 2, None, out.ctypes.data) == bad
    assert lb.osor_scheduler_alphas(0, 0.1, 0.2, 0, None, out.ctypes.data) == bad


def test_wait_expiry_hook_validates_on_the_host():
    """The bounded-wait test hook refuses bad limits, shapes and workspaces
    before any device work, so a mistaken call never launches."""
    lb = _lib.lib()
    d = ctypes.c_void_p(256)
    bad = _lib.OSOR_ERR_INVALID_INPUT
    f16 = _lib.DTYPE_F16
    need = lb.osor_group_norm_workspace_size(1, 128, 64, 64, _lib.LAYOUT_NCHW, f16)
    assert need > 0
    for wait_ns in (0, 999, 1_000_000_001):  # outside [1 us, 1 s]
        assert lb.osor_test_group_norm_wait_expiry(d, d, d, d, 1, 128, 64, 64, f16, wait_ns, d,
                                                   need, None) == bad
    assert lb.osor_test_group_norm_wait_expiry(d, d, d, d, 1, 48, 64, 64, f16, 10 ** 6, d, need,
                                               None) == bad
    assert lb.osor_test_group_norm_wait_expiry(None, d, d, d, 1, 128, 64, 64, f16, 10 ** 6, d,
                                               need, None) == bad
    assert lb.osor_test_group_norm_wait_expiry(d, d, d, d, 1, 128, 64, 64, f16, 10 ** 6, d, 16,
                                               None) == bad
    assert lb.osor_test_group_norm_wait_expiry(d, d, d, d, 1, 128, 64, 64, 9, 10 ** 6, d, need,
                                               None) == bad


def test_unet_handle_entry_points_validate_on_the_host():
    lb = _lib.lib()
    bad = _lib.OSOR_ERR_INVALID_INPUT
    cfg = _lib.OsorUnetConfig()
    out = ctypes.c_void_p()
    one = np.zeros(8, np.float32)
    assert lb.osor_unet_create(None, 0, ctypes.byref(cfg), one.ctypes.data, 1, one.ctypes.data, 0,
                               ctypes.byref(out)) == bad
    assert lb.osor_unet_denoise(None, None, 400, None, None, 1, 8, 8, None, None) == bad
    lb.osor_unet_destroy(None)


def test_geglu_product_and_columns_validate_on_the_host():
    """osor_linear_geglu's workspace query is shape arithmetic: zero where the
    CTA-pair kernel takes the product (an even count of 128-pixel tiles, 2F a
    multiple of 256, Cin % 64 == 0), the [pixels, 2F] 16-bit product
    otherwise, zero for shapes it refuses; both entry points refuse bad
    arguments before any device work."""
    lb = _lib.lib()
    bad = _lib.OSOR_ERR_INVALID_INPUT
    bf16 = _lib.DTYPE_BF16
    assert lb.osor_linear_geglu_workspace_size(4, 32, 32, 1280, 5120, bf16) == 0
    assert lb.osor_linear_geglu_workspace_size(4, 64, 64, 640, 2560, bf16) == 0
    assert lb.osor_linear_geglu_workspace_size(1, 3, 128, 128, 128, bf16) == 384 * 256 * 2
    assert lb.osor_linear_geglu_workspace_size(1, 2, 128, 72, 128, bf16) == 256 * 256 * 2
    assert lb.osor_linear_geglu_workspace_size(1, 2, 128, 128, 100, bf16) == 0
    assert lb.osor_linear_geglu_workspace_size(1, 2, 128, 128, 128, _lib.DTYPE_F32) == 0
    assert lb.osor_linear_geglu(None, None, None, None, 1, 2, 128, 128, 128, bf16, None, 0,
                                None) == bad
    x = np.zeros(64, np.float32)
    assert lb.osor_linear_geglu(x.ctypes.data, x.ctypes.data, x.ctypes.data, None, 1, 2, 128,
                                128, 100, bf16, None, 0, None) == bad
    assert lb.osor_thin_columns(x.ctypes.data, x.ctypes.data, 1, 9, 4, 4, 3, 1, 64, bf16,
                                None) == bad  # 81 taps x channels need 128 columns
    assert lb.osor_thin_columns(x.ctypes.data, x.ctypes.data, 1, 9, 4, 4, 3, 1, 96, bf16,
                                None) == bad
    assert lb.osor_thin_columns(None, None, 1, 9, 4, 4, 3, 1, 128, bf16, None) == bad


def test_unet_geglu_rows_follow_the_documented_order():
    """The Python host's GEGLU row order: per 128 features, the 128 value rows
    and then their gate rows (the order osor_linear_geglu documents)."""
    import torch
    from osor_b200.unet import _geglu_rows
    f = 384
    got = _geglu_rows(f, torch.device("cpu")).tolist()
    want = []
    for t in range(f // 128):
        want += list(range(t * 128, t * 128 + 128))
        want += list(range(f + t * 128, f + t * 128 + 128))
    assert got == want


def test_device_check_reports_unavailable_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert _lib.lib().osor_device_check(0) == _lib.OSOR_ERR_UNAVAILABLE
