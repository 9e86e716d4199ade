"""osor_group_norm_silu_noalloc: the GroupNorm(+SiLU) entry point for callers
that cannot allocate device memory where they run the op (a framework
callback that owns every allocation, a serving loop that must not touch the
allocator). Its scratch is a fixed device array inside the library, so the
caller passes only inputs and outputs.

Checked through the C ABI against the workspace-taking entry point
(osor_group_norm_silu, NCHW) on two calls in a row; warmed-up calls leave the
device's free memory unchanged (nothing is allocated); a shape whose scratch
would not fit is refused before any device work; and, where two GPUs are
visible, a call on tensors of the second GPU made with the first one current
runs on the tensors' device. This file is collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from osor_b200 import _lib, workloads

pytestmark = pytest.mark.gpu

CASES = [
    ((2, 512, 32, 32), torch.bfloat16),
    ((1, 128, 128, 128), torch.float16),
    ((4, 128, 256, 256), torch.bfloat16),
    ((2, 32, 1, 4097), torch.float32),
]


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape,dt", CASES)
def test_noalloc_matches_workspace_entry_point_twice(shape, dt, cuda_device):
    lb = _lib.lib()
    x, gamma, beta = workloads.groupnorm_inputs(shape, seed=3)
    xt = torch.from_numpy(x).to(dt).cuda()
    g = torch.from_numpy(gamma).cuda()
    b = torch.from_numpy(beta).cuda()
    b_, c, h, w = shape
    code = _lib.dtype_code(dt)
    need = lb.osor_group_norm_workspace_size(b_, c, h, w, _lib.LAYOUT_NCHW, code)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(xt)
    ref_stats = torch.zeros((b_ * 32, 2), dtype=torch.float32, device="cuda")
    _lib.check(lb.osor_group_norm_silu(_p(xt), _p(ref), _p(g), _p(b), b_, c, h, w,
                                       _lib.LAYOUT_NCHW, code, 1e-6, 1, _p(ref_stats), _p(ws),
                                       need, _stream()))
    for _ in range(2):
        out = torch.full_like(xt, float("nan"))
        stats = torch.full((b_ * 32, 2), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(lb.osor_group_norm_silu_noalloc(_p(xt), _p(out), _p(g), _p(b), b_, c, h, w,
                                                   code, 1e-6, 1, _p(stats), _stream()))
        torch.cuda.synchronize()
        # The workspace entry point may take the L2-resident NCHW kernel, whose
        # chunking differs from the shared-memory-resident one that the fixed
        # scratch serves: statistics agree to rounding, outputs to one ulp of
        # the 16-bit type (bf16: 2^-7 relative).
        got, want = out.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - want) <= 2 ** -7 * np.abs(want) + 1e-3)
        np.testing.assert_allclose(stats.cpu().numpy(), ref_stats.cpu().numpy(), rtol=1e-4,
                                   atol=1e-6)
    assert _lib.lib().osor_device_status(0, 1) == 0


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch(cuda_device):
    lb = _lib.lib()
    t = torch.zeros(64, device="cuda")
    # 64 images x 32 groups x 171 chunks of 48 KiB (a 16-bit [*, 128, 1024,
    # 1024] group in the 96 KiB shared-memory-resident kernel) needs more
    # scratch than the fixed array holds; refused before any device work.
    rc = lb.osor_group_norm_silu_noalloc(_p(t), _p(t), _p(t), _p(t), 64, 128, 1024, 1024,
                                         _lib.DTYPE_BF16, 1e-6, 1, None, _stream())
    assert rc == _lib.OSOR_ERR_INVALID_INPUT
    assert "fixed no-allocation scratch" in _lib.last_error()


def _noalloc(xt, out, g, b, stream):
    b_, c, h, w = xt.shape
    return _lib.lib().osor_group_norm_silu_noalloc(_p(xt), _p(out), _p(g), _p(b), b_, c, h, w,
                                                   _lib.dtype_code(xt.dtype), 1e-6, 1, None,
                                                   stream)


def test_noalloc_allocates_no_device_memory(cuda_device):
    x, gamma, beta = workloads.groupnorm_inputs((2, 256, 64, 64), seed=3)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    g = torch.from_numpy(gamma).cuda()
    b = torch.from_numpy(beta).cuda()
    out = torch.empty_like(xt)
    _lib.check(_noalloc(xt, out, g, b, _stream()))  # first call: the scratch address lookup
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _lib.check(_noalloc(xt, out, g, b, _stream()))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    assert _lib.lib().osor_device_status(0, 1) == 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two visible GPUs")
def test_noalloc_runs_on_the_device_of_its_tensors(cuda_device):
    x, gamma, beta = workloads.groupnorm_inputs((1, 128, 64, 64), seed=3)
    dev = torch.device("cuda", 1)
    xt = torch.from_numpy(x).to(torch.float16).to(dev)
    g = torch.from_numpy(gamma).to(dev)
    b = torch.from_numpy(beta).to(dev)
    out = torch.full_like(xt, float("nan"))
    torch.cuda.set_device(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(_noalloc(xt, out, g, b, stream))
    torch.cuda.synchronize(dev)
    assert torch.cuda.current_device() == 0
    ref = torch.empty((1, 128, 64, 64), dtype=torch.float16, device="cuda:0")
    _lib.check(_noalloc(xt.to("cuda:0"), ref, g.to("cuda:0"), b.to("cuda:0"), _stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref.cpu().numpy())
    assert _lib.lib().osor_device_status(1, 1) == 0
