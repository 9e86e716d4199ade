"""Row-band split of the VAE decoder and encoder over the ranks of a process group.

The reference bounds memory by running each convolution over horizontal row
bands of its output, one after the other (src/native/conv.rs:98-108,
src/native/columns.rs:335-362). Here the same row-band geometry is spread over
GPUs: each of the K ranks of a band group owns a contiguous range of
R = H / K rows of every activation of one image (upsampling doubles R with
the image, the encoder's stride-2 downsampling halves it), so one image is
decoded or encoded on K GPUs at once.

Activations are held as *extended* NHWC tensors ``[1, R + 2, W, C]``: rows
1..R are the band, rows 0 and R + 1 are halo rows. Three exchanges keep the
result equal to the one-GPU decode:

* halo: before every 3x3 convolution each rank sends its first band row to the
  rank above and its last band row to the rank below into their halo rows (on
  GPUs by peer stores into the neighbours' memory over NVLink,
  ``osor_band_halo``; torch.distributed point-to-point otherwise); the image's
  top and bottom halo rows are zeros, the convolution's zero padding. The
  convolution runs over all R + 2 rows with padding 1, and rows 1..R of its
  output are exact (rows 0 and R + 1 are overwritten by the next exchange).
* GroupNorm: each rank computes its band's per-group (mean, variance) over
  rows 1..R (``osor_group_norm_stats``), the ranks all-gather them (peer
  stores, ``osor_band_gather``, on GPUs), and the
  apply kernel merges the K equal-count sets before normalizing the band
  (``osor_group_norm_apply``).
* attention: the ranks all-gather the band's q|k|v projection, and each
  attends its own queries against every key and value of the image
  (``osor_attention_kv``).

The block order is the decoder's (src/native/vae_decoder.rs:104-114, the mid
block src/native/vae_encoder.rs:367-375, resnets :134-151, attention
:320-339) or the encoder's (vae_encoder.rs:414-424); the encoder's stride-2
downsamplers halve the band and read one halo row below it. ``BandDecoder``
and ``BandEncoder`` drive an op backend: ``CudaBandOps`` calls the library's
C ABI on this rank's GPU; a CPU backend with the same methods runs the same
band logic in the multi-process tests.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, ops
from ._lib import InvalidInput, LAYOUT_NCHW, check
from .weights import SDXL_CHANNELS, SDXL_LAYERS

GROUPS = 32
GATHER_BYTES = 4096  # GroupNorm statistics: 32 groups x (mean, variance) per rank


class PeerExchange:
    """The band group's halo rows and small all-gathers over peer memory
    (``osor_peer_group_*``, ``osor_band_halo``, ``osor_band_gather``): each
    rank's arena is mapped into its neighbours' processes through CUDA IPC
    handles that the ranks exchange once through the process group. The
    exchanges then need no host synchronisation and no NCCL call, and a
    decode built on them can be captured in a CUDA graph."""

    def __init__(self, group: Optional[dist.ProcessGroup], device: torch.device,
                 halo_row_bytes: int, gather_bytes: int = GATHER_BYTES, bulk_bytes: int = 0):
        self.lib = _lib.lib()
        self.group = group
        self.device = device
        distributed = dist.is_available() and dist.is_initialized()
        self.k = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        self.halo_row_bytes = int(halo_row_bytes)
        self.gather_bytes = int(gather_bytes)
        handle = (ctypes.c_uint8 * 64)()
        g = ctypes.c_void_p()
        index = device.index if device.index is not None else torch.cuda.current_device()
        self.bulk_bytes = int(bulk_bytes)
        check(self.lib.osor_peer_group_create(index, self.k, self.rank,
                                              self.halo_row_bytes, self.gather_bytes,
                                              self.bulk_bytes, ctypes.byref(g), handle))
        self.handle = g
        if self.k > 1:
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
            every = torch.empty((self.k, 64), dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.cpu().numpy()
            for r in range(self.k):
                if r != self.rank:
                    buf = (ctypes.c_uint8 * 64).from_buffer_copy(every[r].tobytes())
                    check(self.lib.osor_peer_group_open(g, r, buf))
            dist.barrier(group=group)  # every arena mapped before the first exchange

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def halo(self, x: torch.Tensor) -> torch.Tensor:
        r = x.shape[1] - 2
        row_bytes = x.shape[2] * x.shape[3] * x.element_size()
        check(self.lib.osor_band_halo(self.handle, ctypes.c_void_p(x.data_ptr()), row_bytes, r,
                                      self._stream()))
        return x

    def gather(self, t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        out = torch.empty((self.k,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        check(self.lib.osor_band_gather(self.handle, ctypes.c_void_p(t.data_ptr()),
                                        t.numel() * t.element_size(),
                                        ctypes.c_void_p(out.data_ptr()), self._stream()))
        return out

    def close(self) -> None:
        if self.handle is not None:
            if self.k > 1:
                dist.barrier(group=self.group)  # no rank still writes into an arena
            torch.cuda.synchronize(self.device)
            self.lib.osor_peer_group_destroy(self.handle)
            self.handle = None


class CudaBandOps:
    """The VAE's layers on one CUDA device through the C ABI: 16-bit NHWC
    activations, f32 NCHW at the image / latent boundaries."""

    def __init__(self, weights: Dict[str, np.ndarray], device="cuda", dtype=torch.float16):
        if dtype not in ops.HALF_TYPES:
            raise InvalidInput("band model dtype must be bfloat16 or float16")
        self.w = weights
        self.device = torch.device(device)
        self.dtype = dtype
        self._convs: Dict[str, ops.BandedConv2d] = {}
        self._norms: Dict[str, ops.StableGroupNorm] = {}

    # -- layers, built on first use
    def _conv(self, name: str) -> ops.BandedConv2d:
        c = self._convs.get(name)
        if c is None:
            weight = self.w[name + ".weight"]
            if weight.ndim == 2:
                weight = weight.reshape(weight.shape[0], weight.shape[1], 1, 1)
            k = weight.shape[-1]
            c = ops.BandedConv2d(weight, self.w[name + ".bias"], stride=1, padding=k // 2,
                                 device=self.device, dtype=self.dtype)
            self._convs[name] = c
        return c

    def _qkv(self, prefix: str) -> ops.BandedConv2d:
        """q|k|v as one 1x1 convolution [3C, C], q and k scaled by C^-1/4
        (vae_encoder.rs:320-327 scales each of q and k)."""
        name = prefix + "#qkv"
        c = self._convs.get(name)
        if c is None:
            ws, bs = [], []
            for part in ("to_q", "to_k", "to_v"):
                w = np.asarray(self.w[f"{prefix}.{part}.weight"], np.float32)
                w = w.reshape(w.shape[0], w.shape[1])
                b = np.asarray(self.w[f"{prefix}.{part}.bias"], np.float32)
                scale = np.float32(w.shape[1] ** -0.25) if part != "to_v" else np.float32(1)
                ws.append(w * scale)
                bs.append(b * scale)
            weight = np.concatenate(ws)[:, :, None, None]
            c = ops.BandedConv2d(weight, np.concatenate(bs), stride=1, padding=0,
                                 device=self.device, dtype=self.dtype)
            self._convs[name] = c
        return c

    def _norm(self, name: str) -> ops.StableGroupNorm:
        n = self._norms.get(name)
        if n is None:
            n = ops.StableGroupNorm(self.w[name + ".weight"], self.w[name + ".bias"],
                                    device=self.device)
            self._norms[name] = n
        return n

    # -- the backend methods the band models use
    def empty(self, shape, f32: bool = False) -> torch.Tensor:
        return torch.empty(shape, dtype=torch.float32 if f32 else self.dtype, device=self.device)

    def zeros(self, shape, f32: bool = False) -> torch.Tensor:
        return torch.zeros(shape, dtype=torch.float32 if f32 else self.dtype, device=self.device)

    def conv(self, name, x, residual=None, out=None, out_nchw=False):
        layout = LAYOUT_NCHW if out_nchw else ops._lib.LAYOUT_NHWC
        return self._conv(name).forward_checked(x, residual=residual, out_layout=layout, out=out)

    def conv_down(self, name, x, out):
        """The encoder's downsampler (vae_encoder.rs:206-210): 3x3 stride 2 with
        one zero row / column after the input's last (padding 0 before, 1 after)."""
        key = name + "#down"
        c = self._convs.get(key)
        if c is None:
            c = ops.BandedConv2d(self.w[name + ".weight"], self.w[name + ".bias"], stride=2,
                                 padding=0, padding_end=1, device=self.device, dtype=self.dtype)
            self._convs[key] = c
        return c.forward_checked(x, out=out)

    def qkv(self, prefix, h):
        return self._qkv(prefix).forward_checked(h)

    def upsample(self, x):
        return ops.upsample_2x(x)

    def gn_stats(self, name, x):
        return self._norm(name).stats(x)

    def gn_apply(self, name, x, part_stats, silu, out):
        return self._norm(name).apply(x, part_stats, silu, out=out)

    def attend(self, q, k, v):
        return ops.attend_kv(q, k, v)


class _BandModel:
    """The exchanges and the blocks shared by the band encoder and decoder.
    ``group`` is the band group (default: the whole world)."""

    def __init__(self, backend, channels=SDXL_CHANNELS, layers: int = SDXL_LAYERS,
                 group: Optional[dist.ProcessGroup] = None):
        self.ops = backend
        self.channels = tuple(channels)
        self.layers = int(layers)
        self.group = group
        self.k = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self._nccl = dist.is_initialized() and dist.get_backend(group) == "nccl"
        # Peer-memory exchanges on GPUs (OSOR_BAND_P2P=0 keeps NCCL for them).
        self._p2p = self._nccl and self.k > 1 and os.environ.get("OSOR_BAND_P2P", "1") != "0"
        self.peer: Optional[PeerExchange] = None

    def _ensure_peer(self, halo_row_bytes: int, device: torch.device) -> None:
        """Creates (or, for wider rows, recreates) the peer arena; every rank
        of the group reaches this at the same point of its decode."""
        if not self._p2p:
            return
        if self.peer is not None and self.peer.halo_row_bytes >= halo_row_bytes:
            return
        if self.peer is not None:
            self.peer.close()
        self.peer = PeerExchange(self.group, device, halo_row_bytes)

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _peer(self, local: int) -> int:
        return dist.get_global_rank(self.group, local) if self.group is not None else local

    # -- exchanges
    def halo(self, x: torch.Tensor) -> torch.Tensor:
        """Fill the halo rows of extended x [1, R + 2, W, C] from the neighbours
        (zeros at the image's top and bottom)."""
        if self.peer is not None and x.is_contiguous():
            return self.peer.halo(x)
        r = x.shape[1] - 2
        p2p = []
        if self.rank > 0:
            up = self._peer(self.rank - 1)
            p2p.append(dist.P2POp(dist.isend, x[:, 1], up, self.group))
            p2p.append(dist.P2POp(dist.irecv, x[:, 0], up, self.group))
        if self.rank + 1 < self.k:
            down = self._peer(self.rank + 1)
            p2p.append(dist.P2POp(dist.isend, x[:, r], down, self.group))
            p2p.append(dist.P2POp(dist.irecv, x[:, r + 1], down, self.group))
        if p2p:
            for req in dist.batch_isend_irecv(p2p):
                req.wait()
        if self.rank == 0:
            x[:, 0].zero_()
        if self.rank + 1 == self.k:
            x[:, r + 1].zero_()
        return x

    def gather(self, t: torch.Tensor) -> torch.Tensor:
        """[K, *t.shape]: every rank's t in rank order."""
        if self.k == 1:
            return t.unsqueeze(0)
        nbytes = t.numel() * t.element_size()
        if self.peer is not None and nbytes <= self.peer.gather_bytes and nbytes % 16 == 0:
            return self.peer.gather(t)
        out = torch.empty((self.k,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if self._nccl:
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:
            dist.all_gather(list(out.unbind(0)), t.contiguous(), group=self.group)
        return out

    # -- blocks
    def group_norm(self, name: str, x: torch.Tensor, silu: bool) -> torch.Tensor:
        """GroupNorm (+ SiLU) of extended x's band into a new extended tensor
        whose halo rows are filled."""
        r = x.shape[1] - 2
        band = x[:, 1:r + 1]
        stats = self.gather(self.ops.gn_stats(name, band))
        y = self.ops.empty(x.shape)
        self.ops.gn_apply(name, band, stats, silu, y[:, 1:r + 1])
        return self.halo(y)

    def resnet(self, prefix: str, x: torch.Tensor) -> torch.Tensor:
        h = self.ops.conv(prefix + ".conv1", self.group_norm(prefix + ".norm1", x, True))
        h = self.group_norm(prefix + ".norm2", h, True)
        shortcut = x
        if prefix + ".conv_shortcut.weight" in self.ops.w:
            shortcut = self.ops.conv(prefix + ".conv_shortcut", x)
        return self.ops.conv(prefix + ".conv2", h, residual=shortcut)

    def attention(self, prefix: str, x: torch.Tensor) -> torch.Tensor:
        _, rr, w, c = x.shape
        r = rr - 2
        band = x[:, 1:r + 1]
        stats = self.gather(self.ops.gn_stats(prefix + ".group_norm", band))
        h = self.ops.gn_apply(prefix + ".group_norm", band, stats, False, None)
        qkv = self.ops.qkv(prefix, h).reshape(1, r * w, 3 * c)
        every = self.gather(qkv).reshape(1, self.k * r * w, 3 * c)
        o = self.ops.attend(qkv[:, :, :c], every[:, :, c:2 * c], every[:, :, 2 * c:])
        y = self.ops.zeros(x.shape)
        self.ops.conv(prefix + ".to_out.0", o.reshape(1, r, w, c), residual=band,
                      out=y[:, 1:r + 1])
        return y

    def _band_rows(self, image: torch.Tensor, rows: int, channels: int) -> torch.Tensor:
        """This rank's rows of an NCHW f32 tensor holding the whole image, with
        one halo row above and below (zeros outside the image): [1, C, R + 2, W]."""
        if image.ndim != 4 or image.shape[0] != 1 or image.shape[1] != channels:
            raise InvalidInput(f"band split takes one image [1, {channels}, H, W]")
        _, _, h, w = image.shape
        if h % rows:
            raise InvalidInput("the image height must divide evenly into the band group")
        r = h // rows
        r0 = self.rank * r
        out = self.ops.zeros((1, channels, r + 2, w), f32=True)
        lo, hi = max(r0 - 1, 0), min(r0 + r + 1, h)
        out[:, :, lo - (r0 - 1):hi - (r0 - 1)] = image[:, :, lo:hi]
        return out


class BandDecoder(_BandModel):
    """VaeDecoder::forward (src/native/vae_decoder.rs:104-114) on the rank's
    row band of one image: rank r of K owns latent rows [r R, (r + 1) R),
    R = h / K."""

    def upsample(self, name: str, x: torch.Tensor) -> torch.Tensor:
        """conv3x3(upsample_2x(x)) (vae_decoder.rs:38-49): rows 1..2R + 2 of the
        upsampled extended band are the high-resolution band with its halo."""
        r = x.shape[1] - 2
        u = self.ops.upsample(self.halo(x))
        return self.ops.conv(name, u[:, 1:2 * r + 3])

    def decode(self, latents: torch.Tensor, observer=None) -> torch.Tensor:
        """Unscaled latents [1, 4, h, w] (the whole image, on every rank) ->
        this rank's rows of the raw RGB image, f32 NCHW [1, 3, 8 h / K, 8 w].

        observer(name, band), when given, sees each block's output: the band's
        rows, NHWC 16-bit for the activations and NCHW f32 for
        post_quant_conv and decoder.conv_out, under the reference's VAE trace
        names (src/native/precision_tests.rs:97-130): post_quant_conv,
        decoder.conv_in, decoder.mid_block, decoder.up_blocks.{i} (after its
        upsampler), decoder.conv_norm_out (after SiLU), decoder.conv_out."""
        def seen(name, x, nchw=False):
            if observer is not None:
                r = (x.shape[2] if nchw else x.shape[1]) - 2
                observer(name, x[:, :, 1:r + 1] if nchw else x[:, 1:r + 1])

        # Widest halo row over the resolutions: w 2^i pixels of up block i,
        # whose first resnet still takes block i - 1's channels (16-bit).
        rev = list(reversed(self.channels))
        self._ensure_peer(max(latents.shape[3] * 2 ** i * max(c, rev[max(i - 1, 0)]) * 2
                              for i, c in enumerate(rev)), latents.device)
        lat = self._band_rows(latents, self.k, 4)
        r = lat.shape[2] - 2
        z = self.ops.conv("post_quant_conv", lat, out_nchw=True)
        # conv_in's zero padding applies to post_quant_conv's output.
        if self.rank == 0:
            z[:, :, 0].zero_()
        if self.rank + 1 == self.k:
            z[:, :, r + 1].zero_()
        seen("post_quant_conv", z, nchw=True)
        x = self.ops.conv("decoder.conv_in", z)
        seen("decoder.conv_in", x)
        mid = "decoder.mid_block"
        x = self.resnet(mid + ".resnets.0", x)
        x = self.attention(mid + ".attentions.0", x)
        x = self.resnet(mid + ".resnets.1", x)
        seen(mid, x)
        rev = list(reversed(self.channels))
        for i in range(len(rev)):
            for j in range(self.layers + 1):
                x = self.resnet(f"decoder.up_blocks.{i}.resnets.{j}", x)
            if i + 1 < len(rev):
                x = self.upsample(f"decoder.up_blocks.{i}.upsamplers.0.conv", x)
            seen(f"decoder.up_blocks.{i}", x)
        x = self.group_norm("decoder.conv_norm_out", x, True)
        seen("decoder.conv_norm_out", x)
        y = self.ops.conv("decoder.conv_out", x, out_nchw=True)
        seen("decoder.conv_out", y, nchw=True)
        rows = y.shape[2] - 2
        return y[:, :, 1:rows + 1].contiguous()


class BandEncoder(_BandModel):
    """VaeEncoder::forward (src/native/vae_encoder.rs:414-424) on the rank's row
    band of one image: rank r of K owns image rows [r R, (r + 1) R), R = H / K,
    and R / 2^i rows after the i-th downsampler (H a multiple of 8 K)."""

    def downsample(self, name: str, x: torch.Tensor) -> torch.Tensor:
        """Pad right / bottom by one, 3x3 stride 2 (vae_encoder.rs:206-210): output
        row i of the band reads band rows 2i .. 2i + 2, the last of which is the
        bottom halo row (zeros below the image)."""
        _, rr, w, c = x.shape
        r = rr - 2
        if r % 2:
            raise InvalidInput("band rows must stay even through the downsamplers")
        self.halo(x)
        y = self.ops.zeros((1, r // 2 + 2, w // 2, c))
        self.ops.conv_down(name, x[:, 1:r + 2], y[:, 1:r // 2 + 1])
        return y

    def encode_moments(self, image: torch.Tensor) -> torch.Tensor:
        """Normalized image [1, 3, H, W] (the whole image, on every rank) -> this
        rank's rows of the posterior moments, f32 NCHW [1, 8, H / 8 / K, W / 8]."""
        if image.ndim == 4 and image.shape[2] % (8 * self.k):
            raise InvalidInput("image height must divide into 8 x the band group")
        # Widest halo row over the resolutions: W / 2^i pixels of down block
        # i, whose first resnet still takes block i - 1's channels (16-bit).
        ch = list(self.channels)
        self._ensure_peer(max(image.shape[3] // 2 ** i * max(c, ch[max(i - 1, 0)]) * 2
                              for i, c in enumerate(ch)), image.device)
        x = self.ops.conv("encoder.conv_in", self._band_rows(image, self.k, 3))
        for i in range(len(self.channels)):
            for j in range(self.layers):
                x = self.resnet(f"encoder.down_blocks.{i}.resnets.{j}", x)
            if i + 1 < len(self.channels):
                x = self.downsample(f"encoder.down_blocks.{i}.downsamplers.0.conv", x)
        mid = "encoder.mid_block"
        x = self.resnet(mid + ".resnets.0", x)
        x = self.attention(mid + ".attentions.0", x)
        x = self.resnet(mid + ".resnets.1", x)
        x = self.group_norm("encoder.conv_norm_out", x, True)
        y = self.ops.conv("encoder.conv_out", x, out_nchw=True)
        m = self.ops.conv("quant_conv", y, out_nchw=True)
        rows = m.shape[2] - 2
        return m[:, :, 1:rows + 1].contiguous()


class NativeBandDecoder:
    """The whole decoder on this rank's row band in one C ABI call
    (``osor_vae_decode_band``): the library runs the band with the
    whole-image decoder's kernels (GroupNorm statistics from the convolutions'
    epilogues, fused upsample phases, CTA-pair attention, fused conv_norm_out
    + conv_out) and the peer-memory exchanges between layers, with no Python
    per layer. ``model`` is a NativeModel with the decoder on this rank's GPU;
    ``group`` the band group (default: the whole world, or one rank without a
    process group)."""

    def __init__(self, model, group: Optional[dist.ProcessGroup] = None):
        self.model = model
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.k = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        self.peer: Optional[PeerExchange] = None
        self._ws: Optional[torch.Tensor] = None
        self._sizes = None

    def _prepare(self, h: int, w: int, device: torch.device) -> None:
        lb = _lib.lib()
        ws, halo, bulk = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        check(lb.osor_vae_decode_band_sizes(self.model._handle, self.k, h, w, ctypes.byref(ws),
                                            ctypes.byref(halo), ctypes.byref(bulk)))
        sizes = (ws.value, halo.value, bulk.value)
        if self._sizes == sizes:
            return
        if self.peer is not None:
            self.peer.close()
        self.peer = PeerExchange(self.group, device, halo.value, GATHER_BYTES, bulk.value)
        self._ws = torch.empty(max(ws.value, 1), dtype=torch.uint8, device=device)
        self._sizes = sizes

    def decode(self, latents: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Unscaled latents [1, 4, h, w] f32 (the whole image, on every rank)
        -> this rank's rows of the raw RGB image, f32 NCHW [1, 3, 8 h / K, 8 w]."""
        if latents.ndim != 4 or latents.shape[0] != 1 or latents.shape[1] != 4:
            raise InvalidInput("band decode takes one latent image [1, 4, h, w]")
        if latents.dtype != torch.float32 or not latents.is_cuda:
            raise InvalidInput("band decode takes f32 CUDA latents")
        latents = latents.contiguous()
        _, _, h, w = latents.shape
        if h % self.k:
            raise InvalidInput("the latent height must divide evenly into the band group")
        self._prepare(h, w, latents.device)
        if out is None:
            out = torch.empty((1, 3, 8 * h // self.k, 8 * w), dtype=torch.float32,
                              device=latents.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(latents.device).cuda_stream)
        check(_lib.lib().osor_vae_decode_band(self.model._handle, self.peer.handle,
                                              ctypes.c_void_p(latents.data_ptr()),
                                              ctypes.c_void_p(out.data_ptr()), h, w,
                                              ctypes.c_void_p(self._ws.data_ptr()),
                                              self._ws.numel(), stream))
        return out

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None
