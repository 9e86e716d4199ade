"""CPU oracle for the SDXL VAE hot path -- TEST INFRASTRUCTURE ONLY.

This package restates the reference crate's CPU F32 arithmetic (Candle CPU
path of doublesharp/osor-rs) in plain C++ (``osor_oracle.cpp``, loaded through
ctypes) plus numpy glue for the block topology (``vae.py``). It exists to
check the CUDA library: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` may import it. The product library never
imports, links or calls anything here.

Parity status: the reference is a Rust crate and no Rust toolchain is present,
so it cannot be run; this restatement is pinned against the reference's own
formula-defined unit tests (restated in ``tests/test_oracle.py``) and against
independent float64 PyTorch CPU computations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))


def _has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return " avx512f " in line + " "
    except OSError:
        pass
    return False


_LIB_PATH = os.path.join(_HERE, "liboracle_avx512.so" if _has_avx512() else "liboracle_avx2.so")
_lib = None

#: Column scratch bound of the reference's banded convolution (conv.rs:13).
MAX_SCRATCH_ELEMENTS = 32 * 1024 * 1024
#: Score bound of the reference's sliced attention (attention.rs:8).
MAX_SCORE_ELEMENTS = 64 * 1024 * 1024
GROUPS = 32
EPS = 1e-6

_f32p = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    """Compile the oracle libraries with g++."""
    subprocess.run(["sh", os.path.join(_HERE, "build.sh")], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        l = ctypes.CDLL(_LIB_PATH)
        l.oracle_sgemm.argtypes = [ctypes.c_int] * 3 + [_f32p] * 3 + [ctypes.c_int]
        l.oracle_sgemm.restype = None
        l.oracle_conv2d.argtypes = [_f32p] * 4 + [ctypes.c_int] * 8 + [ctypes.c_longlong]
        l.oracle_conv2d.restype = ctypes.c_int
        l.oracle_group_norm.argtypes = [_f32p] * 4 + [ctypes.c_int, ctypes.c_int,
                                                      ctypes.c_longlong, ctypes.c_double,
                                                      ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        l.oracle_group_norm.restype = ctypes.c_int
        l.oracle_upsample_2x.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 4
        l.oracle_upsample_2x.restype = None
        l.oracle_attention.argtypes = [_f32p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_longlong]
        l.oracle_attention.restype = ctypes.c_int
        l.oracle_seeded_noise.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_longlong,
                                          _f32p]
        l.oracle_seeded_noise.restype = None
        l.oracle_set_threads.argtypes = [ctypes.c_int]
        l.oracle_threads.restype = ctypes.c_int
        _lib = l
    return _lib


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def threads() -> int:
    return int(lib().oracle_threads())


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def sgemm(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), np.float32)
    lib().oracle_sgemm(m, n, k, _p(a), _p(b), _p(c), 0)
    return c


def conv2d(x, weight, bias=None, stride=1, padding=0,
           max_scratch_elements=MAX_SCRATCH_ELEMENTS) -> np.ndarray:
    """NCHW F32 convolution: channel-major column bands + SGEMM, bias after
    (reference columns.rs:297-368, conv.rs:116-145)."""
    x, weight = _f32(x), _f32(weight)
    b, cin, h, w = x.shape
    cout, wcin, k, k2 = weight.shape
    if wcin != cin or k != k2 or k == 0 or stride == 0:
        raise ValueError("column convolution needs a square kernel matching the input")
    if h + 2 * padding < k or w + 2 * padding < k:
        raise ValueError("convolution input is smaller than its kernel")
    oh = (h + 2 * padding - k) // stride + 1
    ow = (w + 2 * padding - k) // stride + 1
    y = np.empty((b, cout, oh, ow), np.float32)
    bias_keep = _f32(bias) if bias is not None else None
    bias_p = _p(bias_keep) if bias_keep is not None else None
    rc = lib().oracle_conv2d(_p(x), _p(weight), bias_p, _p(y), b, cin, h, w, cout, k, stride,
                             padding, int(max_scratch_elements))
    if rc != 0:
        raise ValueError("invalid convolution shape")
    return y


def pad_right_bottom(x) -> np.ndarray:
    """Zero pad of one column on the right and one row at the bottom
    (vae_encoder.rs:207-209)."""
    x = _f32(x)
    return np.ascontiguousarray(np.pad(x, ((0, 0), (0, 0), (0, 1), (0, 1))))


def group_norm(x, gamma, beta, silu=False, eps=EPS, groups=GROUPS, return_stats=False):
    """GroupNorm over NCHW F32 with the reference's staged two-pass statistics
    (vae_encoder.rs:21-81), optional SiLU after (:83-85)."""
    x = _f32(x)
    b, c = x.shape[:2]
    if c == 0 or c % groups != 0:
        raise ValueError("VAE group normalization requires channels divisible by 32")
    spatial = int(np.prod(x.shape[2:])) if x.ndim > 2 else 1
    gamma, beta = _f32(gamma), _f32(beta)
    if gamma.shape != (c,) or beta.shape != (c,):
        raise ValueError("invalid VAE group normalization parameters")
    y = np.empty_like(x)
    mean = np.empty((b, groups), np.float32)
    var = np.empty((b, groups), np.float32)
    rc = lib().oracle_group_norm(_p(x), _p(gamma), _p(beta), _p(y), b, c, spatial, float(eps),
                                 groups, 1 if silu else 0, _p(mean), _p(var))
    if rc != 0:
        raise ValueError("invalid VAE group normalization input shape")
    return (y, mean, var) if return_stats else y


def silu(x) -> np.ndarray:
    x = _f32(x)
    return x / (np.float32(1.0) + np.exp(-x))


def upsample_2x(x) -> np.ndarray:
    x = _f32(x)
    b, c, h, w = x.shape
    y = np.empty((b, c, 2 * h, 2 * w), np.float32)
    lib().oracle_upsample_2x(_p(x), _p(y), b, c, h, w)
    return y


def attend(q, kt, v, max_score_elements=MAX_SCORE_ELEMENTS) -> np.ndarray:
    """softmax(q @ kt) @ v with query-row slicing (attention.rs:27-84).
    q [B,N,D], kt [B,D,M], v [B,M,D]."""
    q, kt, v = _f32(q), _f32(kt), _f32(v)
    b, n, d = q.shape
    m = kt.shape[2]
    out = np.empty((b, n, d), np.float32)
    rc = lib().oracle_attention(_p(q), _p(kt), _p(v), _p(out), b, n, m, d,
                                int(max_score_elements))
    if rc != 0:
        raise ValueError("attention score budget cannot hold one query row")
    return out


def seeded_noise(seed: int, stream: int, count: int) -> np.ndarray:
    """`count` standard-normal f32 values of stream `stream` (0: posterior,
    1: diffusion) of the reference's seeded noise, version 1
    (src/noise.rs:1-99)."""
    out = np.empty(int(count), np.float32)
    lib().oracle_seeded_noise(int(seed) & (2 ** 64 - 1), int(stream), int(count), _p(out))
    return out
