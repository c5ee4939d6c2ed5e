"""CPU oracle for flashcodec's compressed-KV hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker the CUDA kernels are
compared against.  The product package (``flashcodec_b200``) never imports it;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg do.

Two layers:

* ``fc_oracle.c`` (loaded through ctypes): scalar restatements of the codec
  arithmetic in the reference's exact floating-point operation order, plus
  the decode attention evaluated in fp64.  Parity of codes, scales, deltas,
  anchors and reconstructions is bit-exact against these.
* numpy functions below: the array plumbing the reference does with torch
  (block padding, reshapes, dtype rounding), and ``reference_attention_fp32``,
  a vectorised fp32 restatement of the reference's torch attention path used
  as the timed CPU baseline.

Arrays of any dtype are carried as float32 numpy arrays whose values are
exactly representable in the named dtype ("f32", "bf16", "f16").

Parity is pinned: tests/test_oracle_golden.py checks every function here
against fixtures produced by running the reference itself
(tests/golden/make_golden.py), and against the reference's published
reconstruction-quality table.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SO = _HERE / "_build" / "liboracle.so"
_SRC = _HERE / "fc_oracle.c"
_DT = {"f32": 0, "bf16": 1, "f16": 2}
_P = ctypes.c_void_p
_lib = None


def build(force: bool = False) -> Path:
    """Compile fc_oracle.c into oracle/_build/liboracle.so (gcc, no fast-math,
    no FMA contraction so every fused multiply-add is the explicit fmaf)."""
    if _SO.exists() and not force and _SO.stat().st_mtime >= _SRC.stat().st_mtime:
        return _SO
    _SO.parent.mkdir(parents=True, exist_ok=True)
    tmp = _SO.with_suffix(f".{os.getpid()}.tmp")
    subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off",
                           "-fno-fast-math", "-o", str(tmp), str(_SRC), "-lm"])
    os.replace(tmp, _SO)
    return _SO


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        i64, i32, dbl = ctypes.c_int64, ctypes.c_int, ctypes.c_double
        _lib.orc_jpeg_encode.argtypes = [_P, _P, _P, i64, i32, i32, i32, i32]
        _lib.orc_jpeg_quantize.argtypes = [_P, _P, _P, i64, i32, i32]
        _lib.orc_jpeg_decode.argtypes = [_P, _P, _P, _P, i64, i32, i32, i32, i32]
        _lib.orc_png_encode.argtypes = [_P, _P, _P, i64, i32, i32, i32]
        _lib.orc_png_decode.argtypes = [_P, _P, _P, i64, i32, i32, i32]
        _lib.orc_decode_attn.argtypes = [_P, _P, _P, _P, _P, _P, _P, i32, i32,
                                         i32, i32, i64, i32, i32, i32, dbl]
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


# ---------------------------------------------------------------- dtype helpers
def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (RNE) and return them as float32."""
    x = _f32(x)
    if dtype == "f32":
        return x.copy()
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7F800000) == 0x7F800000
        rnd = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
        keep = (u & 0xFFFF0000).astype(np.uint32)
        out = np.where(nan, keep | np.where((u & 0x7FFFFF) != 0, 0x400000, 0).astype(np.uint32), rnd)
        return out.astype(np.uint32).view(np.float32)
    raise ValueError(dtype)


# ------------------------------------------------------------------- jpeg codec
def dct_basis_f64(r: int, k: int) -> np.ndarray:
    """Orthonormal DCT-II rows M[j, n] = c_j cos(pi/r (n+1/2) j), c_0 = sqrt(1/r),
    c_j = sqrt(2/r) (flashcodec/codecs/jpeg.py:24-40), rounded once from fp64.
    Within 4e-6 of the reference's torch-computed basis; bit-exact parity
    tests take the reference basis from the golden fixtures instead."""
    n = np.arange(r, dtype=np.float64)
    j = np.arange(k, dtype=np.float64)[:, None]
    c = np.where(j == 0, math.sqrt(1.0 / r), math.sqrt(2.0 / r))
    return (c * np.cos(math.pi / r * (n[None, :] + 0.5) * j)).astype(np.float32)


def pad_to_blocks(x: np.ndarray, r: int):
    """Zero-pad the seq axis (-2) to a multiple of r and split it into blocks
    (flashcodec/codecs/jpeg.py:43-52, png.py:24-33)."""
    S = x.shape[-2]
    n = (S + r - 1) // r
    pad = n * r - S
    if pad:
        widths = [(0, 0)] * (x.ndim - 2) + [(0, pad), (0, 0)]
        x = np.pad(x, widths)
    return x.reshape(*x.shape[:-2], n, r, x.shape[-1]), S


def jpeg_encode(x: np.ndarray, r: int, k: int, basis: np.ndarray, dtype: str = "f32"):
    """dct_compress (flashcodec/codecs/jpeg.py:55-67): (..., S, D) -> (..., n, k, D)
    coefficients rounded to the input dtype."""
    blocks, _ = pad_to_blocks(_f32(x), r)
    lead, n, D = blocks.shape[:-3], blocks.shape[-3], blocks.shape[-1]
    xb = _f32(blocks.reshape(-1, r, D))
    out = np.empty((xb.shape[0], k, D), np.float32)
    lib().orc_jpeg_encode(_ptr(xb), _ptr(_f32(basis[:k, :r])), _ptr(out), xb.shape[0],
                          r, k, D, _DT[dtype])
    return out.reshape(*lead, n, k, D)


def jpeg_quantize(coef: np.ndarray, dtype: str = "f32"):
    """quantize_coeffs (flashcodec/codecs/jpeg.py:85-100): int8 codes and fp32
    per-(block, frequency) scales of shape (..., n, k, 1)."""
    c = _f32(coef)
    D = c.shape[-1]
    rows = c.size // D if D else 0
    codes = np.empty(c.shape, np.int8)
    scales = np.empty(c.shape[:-1] + (1,), np.float32)
    if rows:
        lib().orc_jpeg_quantize(_ptr(c), _ptr(codes), _ptr(scales), rows, D, _DT[dtype])
    return codes, scales


def jpeg_decode(coef: np.ndarray, scales, basis: np.ndarray, r: int, out_dtype: str = "f32",
                out_len=None):
    """dequantize_coeffs + dct_decompress (flashcodec/codecs/jpeg.py:70-105):
    (..., n, k, D) -> (..., n*r, D) in ``out_dtype``."""
    c = _f32(coef)
    lead, n, k, D = c.shape[:-3], c.shape[-3], c.shape[-2], c.shape[-1]
    cb = _f32(c.reshape(-1, k, D))
    sc = None if scales is None else _f32(np.broadcast_to(scales, c.shape[:-1] + (1,)).reshape(-1))
    out = np.empty((cb.shape[0], r, D), np.float32)
    lib().orc_jpeg_decode(_ptr(cb), _ptr(sc), _ptr(_f32(basis[:k, :r])), _ptr(out),
                          cb.shape[0], r, k, D, _DT[out_dtype])
    rec = out.reshape(*lead, n * r, D)
    return rec if out_len is None else rec[..., :out_len, :]


# -------------------------------------------------------------------- png codec
def png_encode(x: np.ndarray, r: int, keep_ratio: float = 1.0):
    """png_filter (flashcodec/codecs/png.py:36-60): (deltas (..., n, r-1, D) fp32,
    anchors (..., n, D) in the input dtype).  Top-M ties keep the lower index."""
    assert 0 < keep_ratio <= 1.0
    blocks, _ = pad_to_blocks(_f32(x), r)
    lead, n, D = blocks.shape[:-3], blocks.shape[-3], blocks.shape[-1]
    xb = _f32(blocks.reshape(-1, r, D))
    m = r - 1 if keep_ratio >= 1.0 else max(1, math.ceil((r - 1) * keep_ratio))
    deltas = np.empty((xb.shape[0], r - 1, D), np.float32)
    anchors = np.empty((xb.shape[0], D), np.float32)
    lib().orc_png_encode(_ptr(xb), _ptr(deltas), _ptr(anchors), xb.shape[0], r, D, m)
    return deltas.reshape(*lead, n, r - 1, D), anchors.reshape(*lead, n, D)


def png_decode(deltas: np.ndarray, anchors: np.ndarray, dtype: str = "f32"):
    """png_reconstruct (flashcodec/codecs/png.py:63-74): (..., n*r, D)."""
    d = _f32(deltas)
    lead, n, rm1, D = d.shape[:-3], d.shape[-3], d.shape[-2], d.shape[-1]
    r = rm1 + 1
    out = np.empty((int(np.prod(lead, dtype=np.int64)) * n, r, D), np.float32)
    lib().orc_png_decode(_ptr(_f32(d.reshape(-1, rm1, D))), _ptr(_f32(anchors.reshape(-1, D))),
                         _ptr(out), out.shape[0], r, D, _DT[dtype])
    return out.reshape(*lead, n * r, D)


# -------------------------------------------------------------------- attention
def block_basis(mode: str, r: int, k: int, basis: np.ndarray) -> np.ndarray:
    """Synthesis matrix A (r, s): M^T for jpeg, tril(ones) for png
    (flashcodec/attention.py:35-42)."""
    if mode == "jpeg":
        return _f32(basis[:k, :r].T)
    return np.tril(np.ones((r, r), np.float32))


def stored_rows(mode: str, *, codes=None, scales=None, anchors=None, deltas=None):
    """Stored rows per block (flashcodec/attention.py:45-61): dequantized jpeg
    coefficients (fp32 product) or png [anchor; deltas]."""
    if mode == "jpeg":
        c = _f32(codes)
        return c if scales is None else _f32(c * _f32(scales))
    return _f32(np.concatenate([_f32(anchors)[..., None, :], _f32(deltas)], axis=-2))


def decode_attention(q, krows, vrows, kraw, vraw, A, scale=None) -> np.ndarray:
    """codec_decode_attention (flashcodec/attention.py:64-140) in fp64.

    q (B, Hq, 1, D); krows/vrows (B, Hk, n, s, D) or None; kraw/vraw
    (B, Hk, t, D) or None; A (r, s).  Returns (B, Hq, 1, D) float32."""
    q = _f32(q)
    B, Hq, Sq, D = q.shape
    if Sq != 1:
        raise ValueError("decode attention takes a single query token")
    scale = D ** -0.5 if scale is None else scale
    if krows is None and kraw is None:
        return np.zeros_like(q)
    Hk = (krows if krows is not None else kraw).shape[1]
    assert Hq % Hk == 0
    r, s = A.shape
    n = 0 if krows is None else krows.shape[2]
    t = 0 if kraw is None else kraw.shape[2]
    assert s <= 64 and r <= 64 and D <= 1024
    empty = np.zeros((B, Hk, 0, s, D), np.float32)
    kr = _f32(krows) if krows is not None else empty
    vr = _f32(vrows) if vrows is not None else empty
    out = np.empty((B, Hq, D), np.float32)
    lib().orc_decode_attn(_ptr(_f32(q.reshape(B, Hq, D))), _ptr(kr), _ptr(vr),
                          _ptr(_f32(kraw)) if t else None, _ptr(_f32(vraw)) if t else None,
                          _ptr(_f32(A)), _ptr(out), B, Hq, Hk, D, n, s, r, t, float(scale))
    return out.reshape(B, Hq, 1, D)


def reference_attention_fp32(q, krows, vrows, kraw, vraw, A, scale=None) -> np.ndarray:
    """Vectorised fp32 restatement of the reference's torch coefficient path
    (flashcodec/attention.py:101-140): the same einsum sequence, softmax in
    fp32.  Used as the timed CPU baseline; BLAS threads do the contractions."""
    B, Hq, _, D = q.shape
    scale = D ** -0.5 if scale is None else scale
    Hk = (krows if krows is not None else kraw).shape[1]
    G = Hq // Hk
    qg = q.reshape(B, Hk, G, D).astype(np.float32, copy=False)
    logits = []
    if krows is not None:
        n, s = krows.shape[2], krows.shape[3]
        sc = np.matmul(qg[:, :, None], krows.reshape(B, Hk, 1, n * s, D)
                       .transpose(0, 1, 2, 4, 3).reshape(B, Hk, 1, D, n * s))
        sc = sc.reshape(B, Hk, G, n, s)
        logits.append(np.matmul(sc, A.T.astype(np.float32)).reshape(B, Hk, G, -1))
    if kraw is not None:
        logits.append(np.einsum("bhgd,bhtd->bhgt", qg, kraw, optimize=True))
    lg = np.concatenate(logits, axis=-1) * np.float32(scale)
    lg = lg - lg.max(axis=-1, keepdims=True)
    p = np.exp(lg, dtype=np.float32)
    p /= p.sum(axis=-1, keepdims=True)
    out = np.zeros((B, Hk, G, D), np.float32)
    pos = 0
    if krows is not None:
        r = A.shape[0]
        w = np.matmul(p[..., :n * r].reshape(B, Hk, G, n, r), A.astype(np.float32))
        out += np.matmul(w.reshape(B, Hk, G, n * s), vrows.reshape(B, Hk, n * s, D))
        pos = n * r
    if kraw is not None:
        out += np.einsum("bhgt,bhtd->bhgd", p[..., pos:], vraw, optimize=True)
    return out.reshape(B, Hq, 1, D)


def reference_attention_int8(q, kcodes, kscales, vcodes, vscales, kraw, vraw, A, scale=None):
    """The reference's jpeg-int8 decode attention on CPU: dequantize the codes
    into fp32 rows (flashcodec/attention.py:45-61, jpeg.py:103-105), then the
    einsum path of reference_attention_fp32.  The timed CPU baseline."""
    krows = kcodes.astype(np.float32) * kscales
    vrows = vcodes.astype(np.float32) * vscales
    return reference_attention_fp32(q, krows, vrows, kraw, vraw, A, scale)


def reference_attention_int8_mt(q, kcodes, kscales, vcodes, vscales, kraw, vraw, A,
                                scale=None, threads=None, chunk_blocks=512):
    """reference_attention_int8 spread over host threads: the same operation
    sequence (fp32 dequantize of the codes, q . rows, expansion through A,
    fp32 softmax over all keys, weights folded back through A, weighted sum of
    the V rows) on (sequence, KV head, block chunk) tiles, so that the timed
    CPU baseline uses every core as the reference's torch path does
    (flashcodec/attention.py:101-140 runs on torch's intra-op thread pool).
    numpy releases the GIL inside these array operations."""
    from concurrent.futures import ThreadPoolExecutor
    B, Hq, _, D = q.shape
    scale = D ** -0.5 if scale is None else scale
    Hk, n, s = kcodes.shape[1], kcodes.shape[2], kcodes.shape[3]
    r = A.shape[0]
    G = Hq // Hk
    t = 0 if kraw is None else kraw.shape[2]
    qg = np.ascontiguousarray(q.reshape(B, Hk, G, D), dtype=np.float32)
    A32 = np.ascontiguousarray(A, dtype=np.float32)
    tiles = [(b, h, c0, min(n, c0 + chunk_blocks)) for b in range(B) for h in range(Hk)
             for c0 in range(0, n, chunk_blocks)]
    logits = np.empty((B, Hk, G, n * r + t), np.float32)
    out = np.zeros((B, Hk, G, D), np.float32)
    partial = {}

    def k_tile(tile):
        b, h, c0, c1 = tile
        rows = kcodes[b, h, c0:c1].astype(np.float32) * kscales[b, h, c0:c1]
        sc = (qg[b, h] @ rows.reshape(-1, D).T).reshape(G, c1 - c0, s)
        logits[b, h, :, c0 * r:c1 * r] = (sc @ A32.T).reshape(G, -1) * np.float32(scale)

    def v_tile(tile):
        b, h, c0, c1 = tile
        rows = vcodes[b, h, c0:c1].astype(np.float32) * vscales[b, h, c0:c1]
        w = logits[b, h, :, c0 * r:c1 * r].reshape(G, c1 - c0, r) @ A32
        partial[tile] = w.reshape(G, -1) @ rows.reshape(-1, D)

    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as ex:
        list(ex.map(k_tile, tiles))
        if t:
            logits[..., n * r:] = np.einsum("bhgd,bhtd->bhgt", qg, kraw) * np.float32(scale)
        logits -= logits.max(axis=-1, keepdims=True)
        np.exp(logits, out=logits)
        logits /= logits.sum(axis=-1, keepdims=True)
        list(ex.map(v_tile, tiles))
    for (b, h, _, _), part in partial.items():
        out[b, h] += part
    if t:
        out += np.einsum("bhgt,bhtd->bhgd", logits[..., n * r:], vraw)
    return out.reshape(B, Hq, 1, D)


# ------------------------------------------------------- per-group scale format
def jpeg_quantize_grouped(coef: np.ndarray, group: int, dtype: str = "f32"):
    """Per-group variant of quantize_coeffs (the per-32 coefficient quantizer
    of docs/llama-cpp-kv-quantization.md:179-234, which the reference
    measured but ships no code for): every run of ``group`` channels of a
    (block, frequency) row is quantized exactly as quantize_coeffs
    (flashcodec/codecs/jpeg.py:85-100) quantizes a whole row.  Returns int8
    codes (..., D) and fp32 scales (..., D // group)."""
    c = _f32(coef)
    D = c.shape[-1]
    assert D % group == 0
    codes, scales = jpeg_quantize(c.reshape(*c.shape[:-1], D // group, group), dtype)
    return codes.reshape(c.shape), scales.reshape(*c.shape[:-1], D // group)


def dequantize_grouped(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 rows of a per-group archive: code * scale of its group (the fp32
    product dequantize_coeffs forms, jpeg.py:103-105)."""
    g = codes.shape[-1] // scales.shape[-1]
    return _f32(codes.astype(np.float32) * np.repeat(_f32(scales), g, axis=-1))
