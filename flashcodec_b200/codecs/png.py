"""png codec: per-block anchor plus first-order fp32 deltas along the sequence
axis, optional Top-M pruning, rebuilt with a segmented prefix sum.

Same public API as flashcodec/codecs/png.py; the arithmetic runs in the
sm_100a kernels of libflashcodec_sm100.so (fc_png_encode / fc_png_decode) and
is bit-identical to the reference's CPU results (deltas, anchors, and the
reconstruction, whose prefix is accumulated in fp64 like torch's CPU cumsum).
Top-M ties keep the lower index.  CUDA tensors only.
"""

from __future__ import annotations

import math

import torch

from .. import _kernels as K


def _keep_m(r: int, keep_ratio: float) -> int:
    """m = max(1, ceil((r-1) * keep_ratio)) kept deltas (png.py:54-56)."""
    if keep_ratio >= 1.0:
        return r - 1
    return max(1, math.ceil((r - 1) * keep_ratio))


class _PngFilter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, keep_ratio):
        x4 = K.as_bhsd(x)
        B, H, S, D = x4.shape
        n = (S + r - 1) // r
        deltas = torch.empty(B, H, n, r - 1, D, dtype=torch.float32, device=x.device)
        anchors = torch.empty(B, H, n, D, dtype=x.dtype, device=x.device)
        m = _keep_m(r, keep_ratio)
        K.png_encode(x4, r, m, deltas, anchors)
        ctx.meta = (x.shape, x.dtype, r, n, m)
        if m < r - 1:
            ctx.save_for_backward(x)
        lead = x.shape[:-2]
        return deltas.reshape(*lead, n, r - 1, D), anchors.reshape(*lead, n, D)

    @staticmethod
    def backward(ctx, gd, ga):
        # delta_i = mask_i * (x_i - x_{i-1}), anchor = x_0 (png.py:51-59)
        shape, dtype, r, n, m = ctx.meta
        D, S = shape[-1], shape[-2]
        g = torch.zeros(math.prod(shape[:-2]), n, r, D, dtype=torch.float32,
                        device=(gd if gd is not None else ga).device)
        if gd is not None:
            gdm = gd.float().reshape(-1, n, r - 1, D)
            if m < r - 1:
                gdm = gdm * _topm_mask(ctx.saved_tensors[0], r, n, m)
            g[:, :, 1:] += gdm
            g[:, :, :-1] -= gdm
        if ga is not None:
            g[:, :, 0] += ga.float().reshape(-1, n, D)
        gx = g.reshape(-1, n * r, D)[:, :S].to(dtype)
        return gx.reshape(shape), None, None


def _topm_mask(x, r, n, m):
    """The Top-M keep mask of the forward pass (ties to the lower index),
    recomputed from the input for the backward pass."""
    D, S = x.shape[-1], x.shape[-2]
    xf = x.detach().float().reshape(-1, S, D)
    if n * r > S:
        xf = torch.nn.functional.pad(xf, (0, 0, 0, n * r - S))
    b = xf.reshape(-1, n, r, D)
    a = (b[:, :, 1:] - b[:, :, :-1]).abs()                     # (N, n, r-1, D)
    idx = torch.arange(r - 1, device=x.device)
    ai, at = a.unsqueeze(3), a.unsqueeze(2)                   # i along dim 2, t along dim 3
    beats = (at > ai) | ((at == ai) & (idx.view(1, 1, 1, -1, 1) < idx.view(1, 1, -1, 1, 1)))
    rank = beats.sum(dim=3)
    return (rank < m).float()


class _PngReconstruct(torch.autograd.Function):
    @staticmethod
    def forward(ctx, deltas, anchor):
        d = deltas if deltas.stride(-1) == 1 and deltas.dtype == torch.float32 \
            else deltas.float().contiguous()
        lead = d.shape[:-3]
        n, rm1, D = d.shape[-3:]
        r = rm1 + 1
        d5 = d.reshape(-1, n, rm1, D)[None]
        a4 = anchor.reshape(-1, n, D)[None]
        if a4.stride(-1) != 1:
            a4 = a4.contiguous()
        out = torch.empty(1, d5.shape[1], n * r, D, dtype=anchor.dtype, device=d.device)
        K.png_decode(d5, a4, out, n * r)
        ctx.meta = (deltas.shape, deltas.dtype, anchor.shape, anchor.dtype, r)
        return out.reshape(*lead, n * r, D)

    @staticmethod
    def backward(ctx, g):
        dshape, ddtype, ashape, adtype, r = ctx.meta
        n, D = dshape[-3], dshape[-1]
        g = g.float().reshape(-1, n, r, D)
        ga = g.sum(dim=2)
        # d rec_i / d delta_t = 1 for i >= t+1: reverse cumulative sum
        gd = torch.flip(torch.cumsum(torch.flip(g[:, :, 1:], [2]), dim=2), [2])
        return gd.to(ddtype).reshape(dshape), ga.to(adtype).reshape(ashape)


def png_filter(x, block_size, keep_ratio=1.0):
    """Delta filtering (flashcodec/codecs/png.py:36-60): x (..., S, D) ->
    (deltas (..., n, r-1, D) fp32, anchors (..., n, D) in x.dtype)."""
    assert 0 < keep_ratio <= 1.0, "keep_ratio must be within (0, 1]"
    K.require_cuda(x)
    return _PngFilter.apply(x, block_size, keep_ratio)


def png_reconstruct(deltas, anchor):
    """Causal reconstruction (flashcodec/codecs/png.py:63-74): anchor plus the
    prefix sums of the deltas, in the anchor dtype, (..., n*r, D)."""
    K.require_cuda(deltas, anchor)
    return _PngReconstruct.apply(deltas, anchor)


class PNGCodec:
    """Lossless-tier delta codec (flashcodec/codecs/png.py:77-107): each block
    keeps its first token as the anchor and the fp32 steps between neighbours,
    of which the keep_ratio largest per channel survive."""

    name = "png"

    def __init__(self, block_size=8, keep_ratio=1.0):
        assert 0 < keep_ratio <= 1.0, f"keep_ratio={keep_ratio} must lie in (0, 1]"
        self.block_size = block_size
        self.keep_ratio = keep_ratio

    @property
    def keep_m(self):
        """Deltas kept per (block, channel)."""
        return _keep_m(self.block_size, self.keep_ratio)

    def filter(self, x):
        """(B, H, S, D) -> (fp32 deltas (B, H, n, r-1, D), anchors (B, H, n, D))."""
        return png_filter(x, self.block_size, self.keep_ratio)

    def reconstruct(self, deltas, anchor):
        """Anchors plus running sums of the deltas -> (B, H, n*r, D)."""
        return png_reconstruct(deltas, anchor)

    def storage_ratio(self):
        """1.0: an anchor and r-1 fp32 steps take as many elements as the r
        fp32 tokens they replace (png.py:93-103)."""
        return 1.0

    def __repr__(self):
        return f"PNGCodec(block_size={self.block_size}, keep_ratio={self.keep_ratio})"
