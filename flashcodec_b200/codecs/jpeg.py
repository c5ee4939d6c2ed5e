"""jpeg codec: blockwise orthonormal DCT-II along the sequence axis, keep the
first K of r coefficients, optional int8 with a per-(block, frequency) scale.

Same public API as flashcodec/codecs/jpeg.py; the arithmetic runs in the
sm_100a kernels of libflashcodec_sm100.so (fc_jpeg_encode / fc_jpeg_decode)
and is bit-identical to the reference's CPU results.  CUDA tensors only.
"""

from __future__ import annotations

import math

import torch

from .. import _kernels as K

_BASIS_CACHE: dict = {}
_DEV_BASIS: dict = {}


def dct_basis(r, k, device=None, dtype=None):
    """Orthonormal DCT-II rows M (k, r): M[j, n] = c_j cos(pi/r (n + 1/2) j),
    c_0 = sqrt(1/r), c_j = sqrt(2/r) (flashcodec/codecs/jpeg.py:24-40).

    Evaluated once per (r, k) with the same torch CPU operations as the
    reference, so the constants are bit-identical to the reference's basis
    (torch's cosine is not correctly rounded, so recomputing it any other way
    would differ in the last bit), then moved to ``device``/``dtype``."""
    key = (r, k)
    if key not in _BASIS_CACHE:
        n = torch.arange(r, dtype=torch.float32)
        j = torch.arange(k, dtype=torch.float32)
        c = torch.where(j == 0, math.sqrt(1.0 / r), math.sqrt(2.0 / r))
        _BASIS_CACHE[key] = c[:, None] * torch.cos(math.pi / r * (n[None, :] + 0.5) * j[:, None])
    m = _BASIS_CACHE[key]
    if device is not None or dtype is not None:
        m = m.to(device=device, dtype=dtype or m.dtype)
    return m


def device_basis(r: int, k: int, device: torch.device) -> torch.Tensor:
    """The (k, r) fp32 basis resident on ``device`` (cached)."""
    key = (r, k, device.type, device.index)
    m = _DEV_BASIS.get(key)
    if m is None:
        m = dct_basis(r, k).to(device).contiguous()
        _DEV_BASIS[key] = m
    return m


def _identity(device):
    return device_basis(1, 1, device)  # [[1.0]]: a 1-sample block passes values through


class _DctCompress(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, k):
        x4 = K.as_bhsd(x)
        B, H, S, D = x4.shape
        n = (S + r - 1) // r
        out = torch.empty(B, H, n, k, D, dtype=x.dtype, device=x.device)
        K.jpeg_encode(x4, device_basis(r, k, x.device), r, k, out)
        ctx.meta = (x.shape, x.dtype, r)
        return out.reshape(*x.shape[:-2], n, k, D)

    @staticmethod
    def backward(ctx, g):
        shape, dtype, r = ctx.meta
        S = shape[-2]
        gx = dct_decompress(g.float(), r, S)  # adjoint: M^T g (orthonormal rows)
        return gx.to(dtype).reshape(shape), None, None


class _DctDecompress(torch.autograd.Function):
    @staticmethod
    def forward(ctx, coeffs, r, out_len):
        c = coeffs if coeffs.stride(-1) == 1 else coeffs.contiguous()
        lead = c.shape[:-3]
        n, k, D = c.shape[-3:]
        c5 = c.reshape(-1, n, k, D)[None] if c.dim() != 5 else c
        L = n * r if out_len is None else min(out_len, n * r)
        out = torch.empty(c5.shape[0], c5.shape[1], L, D, dtype=torch.float32, device=c.device)
        K.jpeg_decode(c5, None, device_basis(r, k, c.device), r, out, L)
        ctx.meta = (coeffs.shape, coeffs.dtype, r, L)
        return out.reshape(*lead, L, D)

    @staticmethod
    def backward(ctx, g):
        shape, dtype, r, L = ctx.meta
        k = shape[-2]
        gc = dct_compress(g.float().contiguous(), r, k)  # adjoint: M g (zero past L)
        return gc.to(dtype).reshape(shape), None, None


def dct_compress(x, r, k):
    """Blockwise DCT projection (flashcodec/codecs/jpeg.py:55-67):
    x (..., S, D) -> coefficients (..., ceil(S/r), k, D) in x.dtype, the seq
    axis zero-padded to whole blocks."""
    K.require_cuda(x)
    return _DctCompress.apply(x, r, k)


def dct_decompress(coeffs, r, out_len=None):
    """Blockwise DCT reconstruction (flashcodec/codecs/jpeg.py:70-82):
    coefficients (..., n, k, D) -> fp32 (..., n*r, D), trimmed to out_len."""
    K.require_cuda(coeffs)
    return _DctDecompress.apply(coeffs, r, out_len)


def quantize_coeffs(coeffs, bits=8, group_size=None):
    """Symmetric int8 quantization of coefficients
    (flashcodec/codecs/jpeg.py:85-100): coeffs (..., n, k, D) ->
    (int8 codes, fp32 scales (..., n, k, 1)), one scale per (block,
    frequency) row.  Run by the archive kernel with a one-sample block, so
    codes and scales are the ones the cache stores.

    ``group_size`` (an extension: the per-32 coefficient quantizer of
    docs/llama-cpp-kv-quantization.md:179-234) gives one scale per
    ``group_size`` channels of a row instead: scales (..., n, k, D //
    group_size), each group quantized exactly as a row is."""
    if bits != 8:
        raise ValueError(f"only 8-bit coefficient quantization is supported, "
                         f"got bits={bits}")
    K.require_cuda(coeffs)
    c = coeffs.detach()
    D = c.shape[-1]
    g = D if group_size is None else int(group_size)
    if g < 1 or D % g:
        raise ValueError(f"group_size={group_size} must divide the last dimension ({D})")
    rows = c.reshape(-1, g) if c.stride(-1) == 1 and c.is_contiguous() else \
        c.contiguous().reshape(-1, g)
    R = rows.shape[0]
    codes = torch.empty(1, 1, R, 1, g, dtype=torch.int8, device=c.device)
    scales = torch.empty(1, 1, R, 1, 1, dtype=torch.float32, device=c.device)
    K.jpeg_encode(rows[None, None], _identity(c.device), 1, 1, codes, scales)
    return codes.reshape(c.shape), scales.reshape(*c.shape[:-1], D // g)


def dequantize_coeffs(q, scale, dtype=torch.float32):
    """int8 codes + per-row scale -> coefficients in ``dtype``
    (flashcodec/codecs/jpeg.py:103-105: q.to(dtype) * scale.to(dtype)).
    The scale is first rounded to ``dtype`` as the reference does; the product
    of an int8 code and such a scale is exact in fp32 before the final
    rounding, so the result matches the reference's ``dtype`` product."""
    K.require_cuda(q, scale)
    D = q.shape[-1]
    G = scale.shape[-1] if scale.dim() else 1
    if G > 1:
        # one scale per D // G channels (quantize_coeffs(..., group_size)):
        # each group dequantizes like a row
        if D % G:
            raise ValueError(f"{G} scales per row do not divide the last dimension ({D})")
        out = dequantize_coeffs(q.reshape(*q.shape[:-1], G, D // G),
                                scale.reshape(*scale.shape[:-1], G, 1), dtype)
        return out.reshape(q.shape)
    qr = q.reshape(-1, D)
    R = qr.shape[0]
    s = scale.to(dtype).float() if dtype != torch.float32 else scale.float()
    s = s.reshape(-1).contiguous()
    if s.numel() == 1 and R > 1:
        s = s.expand(R).contiguous()
    out = torch.empty(1, 1, R, D, dtype=dtype, device=q.device)
    K.jpeg_decode(qr.contiguous().reshape(1, 1, R, 1, D), s.reshape(1, 1, R, 1, 1),
                  _identity(q.device), 1, out, R)
    return out.reshape(q.shape)


class JPEGCodec:
    """JPEG-style lossy frequency-domain codec (flashcodec/codecs/jpeg.py:108-159).

    ``quant_bits=8`` stores int8 coefficients with a per-(block, frequency)
    scale.  Additions to the reference: ``scale_dtype`` (default fp32 as the
    reference) may be torch.float16 to halve the scale bytes, the archive
    kernel reporting any scale that fp16 cannot hold exactly; ``group_size``
    (default None: one scale per row, as the reference) stores one scale per
    that many channels of a row -- 32 gives the per-32 coefficient format of
    docs/llama-cpp-kv-quantization.md:179-234."""

    name = "jpeg"

    def __init__(self, block_size=8, keep_freqs=2, quant_bits=0, scale_dtype=torch.float32,
                 group_size=None):
        assert 1 <= keep_freqs <= block_size, \
            f"keep_freqs={keep_freqs} is outside 1..{block_size} (the block length)"
        assert quant_bits in (0, 8), \
            f"quant_bits={quant_bits}: use 0 (coefficients kept in the input dtype) or 8 (int8)"
        assert scale_dtype in (torch.float32, torch.float16), \
            "scale_dtype must be torch.float32 or torch.float16"
        assert group_size is None or (quant_bits == 8 and int(group_size) >= 4
                                      and int(group_size) % 4 == 0), \
            "group_size needs quant_bits=8 and a multiple of 4 channels (32 for per-32)"
        self.block_size = block_size
        self.keep_freqs = keep_freqs
        self.quant_bits = quant_bits
        self.scale_dtype = scale_dtype
        self.group_size = None if group_size is None else int(group_size)

    @property
    def quantized(self):
        """True when the archive holds int8 codes plus scales."""
        return self.quant_bits > 0

    def compress(self, x):
        """(B, H, S, D) -> kept DCT coefficients (B, H, n, keep_freqs, D)."""
        return dct_compress(x, self.block_size, self.keep_freqs)

    def quantize(self, coeffs):
        """int8 codes and scales of ``coeffs`` for an int8 codec; (None, None)
        for an unquantized one."""
        if self.quantized:
            return quantize_coeffs(coeffs, self.quant_bits, self.group_size)
        return None, None

    def decompress(self, coeffs, out_len=None, scales=None):
        """Coefficients (or int8 codes with their scales) -> (B, H, out_len, D)."""
        if self.quantized:
            assert scales is not None, "an int8 archive is decoded with its scales"
            coeffs = dequantize_coeffs(coeffs, scales)
        return dct_decompress(coeffs, self.block_size, out_len)

    def storage_ratio(self):
        """Archive size over an fp32 input of the same length, raw tail and
        scale bytes left out (flashcodec/codecs/jpeg.py:144-153): the kept
        fraction keep_freqs / block_size, a quarter of that for int8 codes."""
        kept = self.keep_freqs / self.block_size
        return kept / 4.0 if self.quantized else kept

    def __repr__(self):
        extra = "" if not self.quantized else f", quant_bits={self.quant_bits}"
        if self.scale_dtype != torch.float32:
            extra += ", scale_dtype=torch.float16"
        if self.group_size is not None:
            extra += f", group_size={self.group_size}"
        return f"JPEGCodec(block_size={self.block_size}, keep_freqs={self.keep_freqs}{extra})"
