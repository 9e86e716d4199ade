"""A device-side bounded wait that runs out, then normal work on the same
device.

Every cross-CTA wait in the library's kernels is bounded: on expiry the
waiter records code 1 in the device status word, lets its in-flight copies
land and returns, instead of trapping. This test makes one such wait expire
on purpose through a test hook (osor_test_group_norm_wait_expiry): the fused
NCHW GroupNorm kernel waits for one arrival more than its group has chunks,
with a 1 ms limit. Nothing faults; the host reads the status word, then a
normal GroupNorm call on the same device must match the oracle.

The reference tests its failure paths by injection on the host (cancel after
N checkpoints, src/native/conv.rs:190-216); the GPU-side equivalent here is a
wait whose condition nothing satisfies, with a short limit.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import oracle
from osor_b200 import _lib, workloads

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
def test_expired_wait_reports_timeout_and_the_device_stays_usable(dt, cuda_device):
    lb = _lib.lib()
    shape = (2, 128, 64, 64)
    b_, c, h, w = shape
    x, gamma, beta = workloads.groupnorm_inputs(shape, seed=3)
    xt = torch.from_numpy(x).to(dt).cuda()
    g = torch.from_numpy(gamma).cuda()
    bt = torch.from_numpy(beta).cuda()
    code = _lib.dtype_code(dt)
    need = lb.osor_group_norm_workspace_size(b_, c, h, w, _lib.LAYOUT_NCHW, code)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    y = torch.zeros_like(xt)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lb.osor_device_status(0, 1) == 0  # start from a clear status word

    t0 = time.perf_counter()
    _lib.check(lb.osor_test_group_norm_wait_expiry(_p(xt), _p(y), _p(g), _p(bt), b_, c, h, w,
                                                   code, 1_000_000, _p(ws), need, stream))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    # Code 1 = a bounded wait ran out; reading with reset=1 clears it.
    assert lb.osor_device_status(0, 1) == 1
    assert lb.osor_device_status(0, 0) == 0
    assert elapsed < 30.0  # every CTA gave up after its 1 ms limit

    # The same device, the same workspace: a normal call is correct.
    out = torch.full_like(xt, float("nan"))
    _lib.check(lb.osor_group_norm_silu(_p(xt), _p(out), _p(g), _p(bt), b_, c, h, w,
                                       _lib.LAYOUT_NCHW, code, 1e-6, 1, None, _p(ws), need,
                                       stream))
    torch.cuda.synchronize()
    assert lb.osor_device_status(0, 1) == 0
    want = oracle.group_norm(xt.float().cpu().numpy(), gamma, beta, silu=True)
    got = out.float().cpu().numpy()
    assert np.all(np.abs(got - want) <= 2 ** -7 * np.abs(want) + 2e-3)
