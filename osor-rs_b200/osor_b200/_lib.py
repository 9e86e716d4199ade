"""ctypes binding of libosor_b200.so (the C ABI in include/osor_b200.h).

The shared library is built in-tree by ``osor-rs_b200/build.py``. There is no
fallback: importing the compute entry points without the library raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libosor_b200.so")

OSOR_OK = 0
OSOR_ERR_INVALID_INPUT = 1
OSOR_ERR_INVALID_ARTIFACT = 2
OSOR_ERR_UNAVAILABLE = 3
OSOR_ERR_CANCELLED = 4
OSOR_ERR_CUDA = 5
OSOR_ERR_TIMEOUT = 6

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

LAYOUT_NHWC = 0
LAYOUT_NCHW = 1

OP_DECODE = 0
OP_ENCODE = 1
PART_DECODER = 1
PART_ENCODER = 2


class OsorError(RuntimeError):
    """Base of the errors the C ABI reports (mirrors osor::Error, src/lib.rs:62-90)."""
    code = -1


class InvalidInput(OsorError):
    code = OSOR_ERR_INVALID_INPUT


class InvalidArtifact(OsorError):
    code = OSOR_ERR_INVALID_ARTIFACT


class Unavailable(OsorError):
    code = OSOR_ERR_UNAVAILABLE


class Cancelled(OsorError):
    code = OSOR_ERR_CANCELLED


class CudaError(OsorError):
    code = OSOR_ERR_CUDA


class DeviceTimeout(OsorError):
    code = OSOR_ERR_TIMEOUT


_ERRORS = {c.code: c for c in (InvalidInput, InvalidArtifact, Unavailable, Cancelled, CudaError,
                               DeviceTimeout)}


class OsorTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.POINTER(ctypes.c_float)),
                ("ndim", ctypes.c_int), ("shape", ctypes.c_int64 * 4)]


class OsorVaeConfig(ctypes.Structure):
    _fields_ = [("channels", ctypes.c_int * 4), ("layers", ctypes.c_int), ("parts", ctypes.c_int),
                ("dtype", ctypes.c_int)]


class OsorUnetConfig(ctypes.Structure):
    _fields_ = [("channels", ctypes.c_int * 3), ("depth", ctypes.c_int * 3),
                ("heads", ctypes.c_int * 3), ("context", ctypes.c_int), ("pooled", ctypes.c_int),
                ("time_projection", ctypes.c_int), ("layers", ctypes.c_int),
                ("dtype", ctypes.c_int)]


_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_f = ctypes.c_float
_ll = ctypes.c_longlong

# name -> (restype, argtypes); one entry per function of include/osor_b200.h.
SIGNATURES = {
    "osor_last_error_message": (ctypes.c_char_p, []),
    "osor_version": (_i, []),
    "osor_device_check": (_i, [_i]),
    "osor_device_status": (_i, [_i, _i]),
    "osor_vae_create": (_i, [ctypes.POINTER(OsorTensor), _sz, ctypes.POINTER(OsorVaeConfig), _i,
                             ctypes.POINTER(_vp)]),
    "osor_vae_destroy": (None, [_vp]),
    "osor_vae_workspace_size": (_sz, [_vp, _i, _i, _i, _i]),
    "osor_vae_decode": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp, _vp]),
    "osor_vae_encode_moments": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp, _vp]),
    "osor_pack_conv_weight": (_i, [_vp, _vp, _i, _i, _i, _i]),
    "osor_conv2d": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
                         _vp]),
    "osor_group_norm_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i]),
    "osor_group_norm_silu": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _vp,
                                  _sz, _vp]),
    "osor_group_norm_silu_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _vp,
                                          _vp]),
    "osor_test_group_norm_wait_expiry": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                              ctypes.c_ulonglong, _vp, _sz, _vp]),
    "osor_group_norm_stats": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp]),
    "osor_group_norm_apply": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp,
                                   _sz, _vp]),
    "osor_seeded_noise": (_i, [ctypes.c_ulonglong, _i, _i, _i, _i, _vp, _vp, _vp]),
    "osor_scheduler_alphas": (_i, [_i, ctypes.c_double, ctypes.c_double, _i, _vp, _vp]),
    "osor_scheduler_add_noise": (_i, [_vp, _vp, _vp, _ll, _f, _vp]),
    "osor_scheduler_predicted_original": (_i, [_vp, _vp, _vp, _ll, _f, _i, _i, _f, _vp]),
    "osor_pipeline_prepare": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f,
                                   ctypes.c_double, _vp]),
    "osor_pipeline_finish": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _f,
                                  ctypes.c_double, _vp]),
    "osor_pipeline_map": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "osor_pipeline_normalize_image": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "osor_upsample_2x": (_i, [_vp, _vp, _i, _i, _i, _i, _vp]),
    "osor_attention_workspace_size": (_sz, [_i, _i, _i]),
    "osor_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _ll, _i, _vp, _sz, _vp]),
    "osor_attention_kv_workspace_size": (_sz, [_i, _i, _i, _i]),
    "osor_attention_kv": (_i, [_vp, _ll, _vp, _vp, _ll, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "osor_unet_time_features": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "osor_rows_linear": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "osor_layer_norm": (_i, [_vp, _vp, _vp, _vp, _ll, _i, _f, _i, _vp]),
    "osor_geglu": (_i, [_vp, _vp, _ll, _i, _i, _vp]),
    "osor_thin_columns": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "osor_linear_geglu_workspace_size": (_sz, [_i, _i, _i, _i, _i, _i]),
    "osor_linear_geglu": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "osor_concat_channels": (_i, [_vp, _i, _vp, _i, _vp, _ll, _i, _vp]),
    "osor_resize_nearest": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "osor_channel_update": (_i, [_vp, _ll, _vp, _i, _i, _ll, _vp, _ll, _vp, _i, _vp]),
    "osor_attention_heads": (_i, [_vp, _ll, _ll, _vp, _vp, _ll, _ll, _vp, _ll, _ll, _i, _i, _i,
                                  _i, _i, _i, _vp]),
    "osor_unet_create": (_i, [ctypes.POINTER(OsorTensor), _sz, ctypes.POINTER(OsorUnetConfig),
                              _vp, _i, _vp, _i, ctypes.POINTER(_vp)]),
    "osor_unet_destroy": (None, [_vp]),
    "osor_peer_group_create": (_i, [_i, _i, _i, _sz, _sz, _sz, _vp, _vp]),
    "osor_peer_group_open": (_i, [_vp, _i, _vp]),
    "osor_peer_group_destroy": (None, [_vp]),
    "osor_band_halo": (_i, [_vp, _vp, _ll, _i, _vp]),
    "osor_band_gather": (_i, [_vp, _vp, _sz, _vp, _vp]),
    "osor_vae_decode_band_sizes": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp]),
    "osor_vae_decode_band": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    "osor_unet_denoise": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "osor_profile_begin": (None, []),
    "osor_profile_end": (_i, [_vp, _i, ctypes.POINTER(_i)]),
    "osor_launch_count": (_ll, []),
}


class ProfileEntry(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_char * 32), ("flops", ctypes.c_double),
                ("bytes", ctypes.c_double), ("ms", ctypes.c_float), ("launches", ctypes.c_int)]


def profile_begin() -> None:
    """Record CUDA events around every op this thread enqueues."""
    lib().osor_profile_begin()


def profile_end(max_entries: int = 1 << 16):
    """Stop recording; returns a list of (kind, flops, bytes, ms, launches)."""
    entries = (ProfileEntry * max_entries)()
    count = ctypes.c_int(0)
    check(lib().osor_profile_end(entries, max_entries, ctypes.byref(count)))
    return [(entries[i].kind.decode(), entries[i].flops, entries[i].bytes, entries[i].ms,
             entries[i].launches) for i in range(min(count.value, max_entries))]


def launch_count() -> int:
    return int(lib().osor_launch_count())

_lib = None


def lib():
    """Load the library (raises OSError with a build hint when it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python osor-rs_b200/build.py`")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def last_error() -> str:
    msg = lib().osor_last_error_message()
    return msg.decode() if msg else ""


def dtype_code(dtype) -> int:
    """torch dtype or name -> OSOR_DTYPE_* code."""
    import torch
    table = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16, torch.float32: DTYPE_F32,
             "bf16": DTYPE_BF16, "f16": DTYPE_F16, "fp16": DTYPE_F16, "f32": DTYPE_F32}
    if dtype not in table:
        raise InvalidInput(f"unsupported dtype {dtype}")
    return table[dtype]


def check(rc: int) -> None:
    """Raise the typed error for a non-zero status code."""
    if rc != OSOR_OK:
        raise _ERRORS.get(rc, OsorError)(last_error())
