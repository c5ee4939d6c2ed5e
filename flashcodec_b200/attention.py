"""Materialization-free decode attention on the compressed archive.

Both codecs are linear along the sequence inside a block: with stored rows S
(s x D) and synthesis matrix A (r x s), K_block = A S.  A decode query scores
token p of a block as (q . S^T) A[p] and the block contributes (p A) S to the
output, so attention never reconstructs the (S, D) view
(flashcodec/attention.py:1-27).  The whole step -- scores against the int8
codes, softmax, the fold back through A onto the V codes, the raw tail and the
merge of the sequence splits -- is one launch of fc_decode_attn
(flashcodec_b200/csrc/fc_attention.cu).
"""

from __future__ import annotations

import torch

from . import _kernels as K
from .codecs import dct_basis

_A_CACHE: dict = {}


def block_basis(codec, block_size, device=None, dtype=torch.float32):
    """Synthesis matrix A (r, s) mapping a block's stored rows to its r tokens
    (flashcodec/attention.py:35-42): M^T for jpeg, tril(ones(r, r)) for png."""
    r = block_size
    if codec.name == "jpeg":
        return dct_basis(r, codec.keep_freqs, device=device, dtype=dtype).t()
    return torch.tril(torch.ones(r, r, dtype=dtype, device=device))


def _device_A(codec, r, device):
    key = (codec.name, r, getattr(codec, "keep_freqs", r), device.index)
    A = _A_CACHE.get(key)
    if A is None:
        A = block_basis(codec, r, device=device).contiguous()
        _A_CACHE[key] = A
    return A


def _rows(stream):
    """(rows (B,H,n,s,D), scales (B,H,n,s,1) or None) of the archived blocks."""
    n = stream.n_blocks
    if n == 0:
        return None, None
    c = stream.codec
    if c.name == "jpeg":
        rows = stream._coeffs[:, :, :n]
        return rows, (stream._scales[:, :, :n] if c.quantized else None)
    raise AssertionError("png archives are read in place by fc_decode_attn_png")


def codec_decode_attention(query, key_stream, value_stream, scale=None, impl="auto",
                           visible=None):
    """Attention of one new query token against a codec archive without
    materialising the reconstructed KV (flashcodec/attention.py:64-140).

    Args:
        query: (B, Hq, 1, D) CUDA tensor.
        key_stream, value_stream: ``_CodecStream`` of one layer.
        scale: softmax scale (default D ** -0.5).
        impl: accepted for API compatibility ("auto", "cuda", "triton",
            "torch"); every value runs the sm_100a kernel -- this package has
            exactly one implementation.
        visible: optional (B, S) bool/uint8 CUDA tensor, nonzero where the
            query attends (S = the streams' length: archived tokens, then the
            raw tail); e.g. the padding mask of a left-padded batch.  An
            extension of the reference API, which has no mask
            (fc_decode_attn_masked, CUDA-core kernel).
    Returns:
        (B, Hq, 1, D) in the query dtype.  Scores, softmax and accumulation
        are fp32.
    """
    B, Hq, Sq, D = query.shape
    if Sq != 1:
        raise ValueError("codec_decode_attention only supports a single query "
                         f"token (got Sq={Sq}); prefill should use the "
                         "materialized view")
    if impl not in ("auto", "cuda", "triton", "torch"):
        raise ValueError(f"unknown impl {impl!r}")
    K.require_cuda(query)
    scale = D ** -0.5 if scale is None else scale
    ks, vs = key_stream, value_stream
    if ks.n_blocks == 0 and ks.raw is None:
        return torch.zeros_like(query)
    Hk = (ks._raw_buf if ks._raw_buf is not None else
          (ks._coeffs if ks.codec.name == "jpeg" else ks._deltas)).shape[1]
    assert Hq % Hk == 0, f"query heads ({Hq}) must be a multiple of kv heads ({Hk})"
    out = torch.empty_like(query)
    n = ks.n_blocks
    if ks.codec.name == "png" and n > 0:
        # anchors and deltas read where the archive keeps them (no row assembly)
        A = _device_A(ks.codec, ks.block_size, query.device)
        K.decode_attn_png(query, ks._anchors[:, :, :n], vs._anchors[:, :, :n],
                          ks._deltas[:, :, :n], vs._deltas[:, :, :n], ks.raw, vs.raw, A,
                          scale, out, vis=visible)
        return out
    krows, kscales = _rows(ks)
    vrows, vscales = _rows(vs)
    A = _device_A(ks.codec, ks.block_size, query.device) if krows is not None else None
    group = getattr(ks.codec, "group_size", None)
    if group is not None and krows is not None:
        # per-group scales (the per-32 coefficient format)
        if visible is not None:
            raise NotImplementedError("a visibility mask is not supported on per-group archives")
        K.decode_attn_grouped(query, krows, vrows, kscales, vscales, group, ks.raw, vs.raw, A,
                              scale, out)
        return out
    K.decode_attn(query, krows, vrows, kscales, vscales, ks.raw, vs.raw, A, scale, out,
                  vis=visible)
    return out


def attention_status(device=None, reset=False):
    """Failure status of the decode-attention calls issued on the current
    stream of ``device``, without synchronising (an extension: the reference
    kernels have no failure status).

    Every wait inside the attention kernels is bounded; a call whose wait
    gave up leaves invalid output and records its launch number in the
    stream's workspace.  This queues a copy of that word to pinned host
    memory and returns a probe: ``probe.ready()`` polls, ``probe.value()``
    returns the word (0 = every call since the last reset was valid),
    ``probe.check()`` raises if some call gave up.  ``reset=True`` clears the
    word after the copy.  Typical use: take a probe after each decode step
    and check the previous step's probe before using its tokens."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    return K.attn_status_async(dev, reset=reset)

