"""Op-level host mirror of the reference's VAE operator seams.

Each class keeps the reference's name and argument meaning and calls the C ABI
on torch CUDA tensors (torch is only the allocator / stream provider here):

  BandedConv2d.forward_checked   src/native/conv.rs:54-145
  StableGroupNorm.forward(_silu) src/native/vae_encoder.rs:37-105
  upsample_2x                    src/native/vae_decoder.rs:18-35
  attend                         src/native/attention.rs:10-25
  attend_kv                      src/native/attention.rs:10-25 (n_q != n_kv)
  StableGroupNorm.stats / .apply src/native/vae_encoder.rs:55-80, split in two

Activations between ops are NHWC ``[B, H, W, C]`` 16-bit (bf16 or f16) device
tensors, the library's internal layout; ``nchw_to_nhwc`` / ``nhwc_to_nchw``
convert at the edges. Shape errors raise ``InvalidInput`` before any device
work, like the reference's ``Error::InvalidInput``.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import numpy as np
import torch

from . import _lib
from ._lib import InvalidInput, check, dtype_code

GROUPS = 32
EPS = 1e-6

Checkpoint = Optional[Callable[[], None]]
HALF_TYPES = (torch.bfloat16, torch.float16)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise InvalidInput(f"{what} must be a CUDA tensor")
    if not t.is_contiguous():
        raise InvalidInput(f"{what} must be contiguous")


def nchw_to_nhwc(x: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    return x.permute(0, 2, 3, 1).contiguous().to(dtype)


def nhwc_to_nchw(x: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    return x.permute(0, 3, 1, 2).contiguous().to(dtype)


def pack_conv_weight(weight: np.ndarray, dtype=torch.bfloat16) -> np.ndarray:
    """[Cout, Cin, k, k] float32 -> [Cout, k*k*Cin] 16-bit patterns (uint16)."""
    w = np.ascontiguousarray(weight, dtype=np.float32)
    cout, cin, k, k2 = w.shape
    if k != k2:
        raise InvalidInput("convolution kernels must be square")
    out = np.empty((cout, k * k * cin), np.uint16)
    check(_lib.lib().osor_pack_conv_weight(w.ctypes.data, out.ctypes.data, cout, cin, k,
                                           dtype_code(dtype)))
    return out


def _host_f32(a) -> np.ndarray:
    return np.asarray(a.detach().cpu() if torch.is_tensor(a) else a, np.float32)


class BandedConv2d:
    """Square, ungrouped, undilated convolution with bias (conv.rs:148-182).

    ``weight`` [Cout, Cin, k, k] and ``bias`` [Cout] are host float32 arrays
    (or tensors); they are repacked once to ``dtype`` (bf16 or f16) on
    ``device``. ``padding_end`` zero rows / columns follow the last input row /
    column (default ``padding``); the encoder's downsampler uses padding 0,
    padding_end 1 (vae_encoder.rs:206-210)."""

    def __init__(self, weight, bias, stride: int = 1, padding: int = 0, device="cuda",
                 padding_end: Optional[int] = None, dtype=torch.bfloat16):
        weight = _host_f32(weight)
        if weight.ndim != 4 or weight.shape[2] != weight.shape[3]:
            raise InvalidInput("convolution weight must be [Cout, Cin, k, k]")
        if stride <= 0 or weight.shape[2] == 0:
            raise InvalidInput("convolution kernel and stride must be positive")
        if dtype not in HALF_TYPES:
            raise InvalidInput("convolution dtype must be bfloat16 or float16")
        self.dtype = dtype
        self.cout, self.cin, self.kernel = weight.shape[0], weight.shape[1], weight.shape[2]
        self.stride, self.padding = int(stride), int(padding)
        self.padding_end = self.padding if padding_end is None else int(padding_end)
        packed = torch.from_numpy(pack_conv_weight(weight, dtype).view(np.int16))
        self.weight = packed.view(dtype).to(device)
        self.bias = None
        if bias is not None:
            self.bias = torch.from_numpy(_host_f32(bias).copy()).to(device)

    def out_shape(self, h: int, w: int):
        ph = h + self.padding + self.padding_end
        pw = w + self.padding + self.padding_end
        if ph < self.kernel or pw < self.kernel:
            raise InvalidInput("convolution input is smaller than its kernel")
        return (ph - self.kernel) // self.stride + 1, (pw - self.kernel) // self.stride + 1

    def forward_checked(self, x: torch.Tensor, checkpoint: Checkpoint = None,
                        residual: Optional[torch.Tensor] = None,
                        out_layout: int = _lib.LAYOUT_NHWC,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x: NHWC [B, H, W, Cin] of this conv's dtype, or NCHW f32 [B, Cin, H, W].
        ``out`` (optional) receives the result; it must be contiguous and of
        the output's shape and type."""
        if checkpoint:
            checkpoint()
        _require_cuda(x, "convolution input")
        if x.dtype == self.dtype:
            in_layout = _lib.LAYOUT_NHWC
            b, h, w, c = x.shape
        elif x.dtype == torch.float32:
            in_layout = _lib.LAYOUT_NCHW
            b, c, h, w = x.shape
        else:
            raise InvalidInput("convolution input must be NHWC of the conv dtype or NCHW f32")
        if c != self.cin:
            raise InvalidInput("convolution input channels do not match the weight")
        oh, ow = self.out_shape(h, w)
        if out_layout == _lib.LAYOUT_NHWC:
            shape, dt = (b, oh, ow, self.cout), self.dtype
        else:
            shape, dt = (b, self.cout, oh, ow), torch.float32
        if out is None:
            y = torch.empty(shape, dtype=dt, device=x.device)
        else:
            _require_cuda(out, "convolution output")
            if tuple(out.shape) != shape or out.dtype != dt or out.device != x.device:
                raise InvalidInput("convolution output tensor does not match the result")
            y = out
        if residual is not None:
            _require_cuda(residual, "residual")
            if residual.shape != y.shape or residual.dtype != self.dtype:
                raise InvalidInput("residual must match the NHWC output")
        check(_lib.lib().osor_conv2d(_ptr(x), _ptr(y), _ptr(self.weight), _ptr(self.bias),
                                     _ptr(residual), b, h, w, c, self.cout, self.kernel,
                                     self.stride, self.padding, self.padding_end, in_layout,
                                     out_layout, dtype_code(self.dtype), _stream(x.device)))
        if checkpoint:
            checkpoint()
        return y

    __call__ = forward_checked


class StableGroupNorm:
    """GroupNorm(32, eps 1e-6) with fp32 statistics (vae_encoder.rs:37-105)."""

    def __init__(self, weight, bias, device="cuda"):
        w = torch.from_numpy(_host_f32(weight).copy())
        b = torch.from_numpy(_host_f32(bias).copy())
        if w.ndim != 1 or w.shape != b.shape or w.numel() == 0 or w.numel() % GROUPS:
            raise InvalidInput("VAE group normalization requires channels divisible by 32")
        self.channels = w.numel()
        self.weight = w.to(device)
        self.bias = b.to(device)
        self._workspace = {}

    def _run(self, x: torch.Tensor, silu: bool, layout: int, eps: float,
             stats: Optional[torch.Tensor]) -> torch.Tensor:
        _require_cuda(x, "group-norm input")
        if x.ndim != 4:
            raise InvalidInput("invalid VAE group normalization input shape")
        if layout == _lib.LAYOUT_NHWC:
            b, h, w, c = x.shape
        else:
            b, c, h, w = x.shape
        if c != self.channels or b == 0 or h == 0 or w == 0:
            raise InvalidInput("invalid VAE group normalization input shape")
        dt = dtype_code(x.dtype)
        lb = _lib.lib()
        need = lb.osor_group_norm_workspace_size(b, c, h, w, layout, dt)
        if need == 0:
            raise InvalidInput("unsupported group-norm shape, layout or dtype")
        key = (x.device, need)
        ws = self._workspace.get(key)
        if ws is None:
            ws = torch.empty(need, dtype=torch.uint8, device=x.device)
            self._workspace = {key: ws}
        y = torch.empty_like(x)
        check(lb.osor_group_norm_silu(_ptr(x), _ptr(y), _ptr(self.weight), _ptr(self.bias), b, c,
                                      h, w, layout, dt, float(eps), 1 if silu else 0, _ptr(stats),
                                      _ptr(ws), need, _stream(x.device)))
        return y

    def forward(self, x, layout=_lib.LAYOUT_NCHW, eps=EPS, stats=None):
        return self._run(x, False, layout, eps, stats)

    def _nhwc_workspace(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x, "group-norm input")
        if x.ndim != 4 or x.dtype not in HALF_TYPES:
            raise InvalidInput("group-norm statistics / apply take 16-bit NHWC [B, H, W, C]")
        b, h, w, c = x.shape
        if c != self.channels or b == 0 or h == 0 or w == 0:
            raise InvalidInput("invalid VAE group normalization input shape")
        need = _lib.lib().osor_group_norm_workspace_size(b, c, h, w, _lib.LAYOUT_NHWC,
                                                         dtype_code(x.dtype))
        if need == 0:
            raise InvalidInput("unsupported group-norm shape, layout or dtype")
        key = (x.device, need)
        ws = self._workspace.get(key)
        if ws is None:
            ws = torch.empty(need, dtype=torch.uint8, device=x.device)
            self._workspace = {key: ws}
        return ws

    def stats(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Per-(image, group) (mean, biased variance) of 16-bit NHWC x, f32 [B, 32, 2]."""
        ws = self._nhwc_workspace(x)
        b, h, w, c = x.shape
        if out is None:
            out = torch.empty((b, GROUPS, 2), dtype=torch.float32, device=x.device)
        elif out.shape != (b, GROUPS, 2) or out.dtype != torch.float32 or not out.is_contiguous():
            raise InvalidInput("statistics output must be contiguous f32 [B, 32, 2]")
        check(_lib.lib().osor_group_norm_stats(_ptr(x), b, c, h, w, dtype_code(x.dtype),
                                               _ptr(out), _ptr(ws), ws.numel(),
                                               _stream(x.device)))
        return out

    def apply(self, x: torch.Tensor, part_stats: torch.Tensor, silu: bool, eps=EPS,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Normalize 16-bit NHWC x with the merge of ``part_stats`` f32
        [P, B, 32, 2]: P statistics sets over equal element counts (the row
        bands of the same images)."""
        ws = self._nhwc_workspace(x)
        b, h, w, c = x.shape
        _require_cuda(part_stats, "group-norm statistics")
        if (part_stats.ndim != 4 or tuple(part_stats.shape[1:]) != (b, GROUPS, 2)
                or part_stats.dtype != torch.float32):
            raise InvalidInput("statistics must be f32 [P, B, 32, 2]")
        if out is None:
            out = torch.empty_like(x)
        else:
            _require_cuda(out, "group-norm output")
            if out.shape != x.shape or out.dtype != x.dtype:
                raise InvalidInput("group-norm output must match the input")
        check(_lib.lib().osor_group_norm_apply(_ptr(x), _ptr(out), _ptr(self.weight),
                                               _ptr(self.bias), _ptr(part_stats),
                                               part_stats.shape[0], b, c, h, w,
                                               dtype_code(x.dtype), float(eps),
                                               1 if silu else 0, _ptr(ws), ws.numel(),
                                               _stream(x.device)))
        return out

    def forward_silu(self, x, layout=_lib.LAYOUT_NCHW, eps=EPS, stats=None):
        return self._run(x, True, layout, eps, stats)

    __call__ = forward


def upsample_2x(x: torch.Tensor) -> torch.Tensor:
    """Nearest 2x of 16-bit NHWC [B, H, W, C] (vae_decoder.rs:18-35)."""
    _require_cuda(x, "upsample input")
    if x.dtype not in HALF_TYPES or x.ndim != 4:
        raise InvalidInput("upsample expects 16-bit NHWC")
    b, h, w, c = x.shape
    y = torch.empty((b, 2 * h, 2 * w, c), dtype=x.dtype, device=x.device)
    check(_lib.lib().osor_upsample_2x(_ptr(x), _ptr(y), b, h, w, c, _stream(x.device)))
    return y


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T) v over 16-bit [B, N, D] tensors (attention.rs:10-25; the
    reference passes k already transposed, this takes k as [B, N, D])."""
    for t, n in ((q, "query"), (k, "key"), (v, "value")):
        _require_cuda(t, n)
        if t.dtype not in HALF_TYPES or t.ndim != 3 or t.dtype != q.dtype:
            raise InvalidInput("attention tensors must be one 16-bit type, [B, N, D]")
    if q.shape != k.shape or q.shape != v.shape:
        raise InvalidInput("attention tensor shapes are incompatible")
    b, n, d = q.shape
    lb = _lib.lib()
    need = lb.osor_attention_workspace_size(b, n, d)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    check(lb.osor_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, n, d, d,
                            dtype_code(q.dtype), _ptr(ws), need, _stream(q.device)))
    return out


def _rows_view(t: torch.Tensor, what: str):
    """[B, N, D] (or [N, D]) view whose last dim is contiguous -> (B, N, D, row
    stride). Batch entries must follow one another at N rows."""
    if not t.is_cuda:
        raise InvalidInput(f"{what} must be a CUDA tensor")
    if t.ndim == 2:
        t = t.unsqueeze(0)
    if t.ndim != 3 or t.dtype not in HALF_TYPES or t.stride(2) != 1:
        raise InvalidInput("attention tensors must be 16-bit [B, N, D] rows")
    b, n, d = t.shape
    ld = t.stride(1)
    if ld < d or (b > 1 and t.stride(0) != n * ld):
        raise InvalidInput(f"{what} rows are not evenly strided")
    return b, n, d, ld


def attend_kv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T) v with n_q query rows against n_kv key / value rows
    (attention.rs:10-25 allows different row counts). q [B, n_q, D], k and v
    [B, n_kv, D]: row-strided views (e.g. column slices of one q|k|v
    projection); out: contiguous [B, n_q, D]."""
    bq, nq, d, ldq = _rows_view(q, "query")
    bk, nk, dk, ldk = _rows_view(k, "key")
    bv, nv, dv, ldv = _rows_view(v, "value")
    if (bq, d) != (bk, dk) or (bk, nk, dk) != (bv, nv, dv) or ldk != ldv:
        raise InvalidInput("attention tensor shapes are incompatible")
    if q.dtype != k.dtype or k.dtype != v.dtype:
        raise InvalidInput("attention tensors must be one 16-bit type")
    lb = _lib.lib()
    need = lb.osor_attention_kv_workspace_size(bq, nq, nk, d)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty((bq, nq, d), dtype=q.dtype, device=q.device)
    check(lb.osor_attention_kv(_ptr(q), ldq, _ptr(k), _ptr(v), ldk, _ptr(out), bq, nq, nk, d,
                               dtype_code(q.dtype), _ptr(ws), need, _stream(q.device)))
    return out
