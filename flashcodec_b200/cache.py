"""Compressed KV cache: the append / archive / read cycle of one (B, H, S, D)
stream, and the multi-layer container.

Same API and semantics as flashcodec/cache.py (make_codec :39-54,
_CodecStream :57-325, CodecKVCache :328-440).  The device work goes through
the sm_100a kernels:

* append: tokens land in a preallocated r-slot raw buffer (no per-step
  torch.cat); every completed block is archived by fc_jpeg_encode /
  fc_png_encode writing straight into its slot of the capacity-doubled
  archive (no intermediate coefficient tensor).
* read: only the blocks archived since the last read are decoded
  (fc_jpeg_decode / fc_png_decode, straight into the reconstruction buffer);
  the raw tail is copied behind them and the view is returned without
  concatenating the history.

Differences a caller can observe, none of them in values:
* ``read()`` always returns a view of the internal reconstruction buffer
  (the reference returns a fresh concatenation while a raw tail exists).
  Positions that were still raw at the time of the read are overwritten by
  their reconstruction once their block is archived; archived positions are
  never rewritten (the reference's causal-safety guarantee).
* ``read()`` on a stream without archived blocks returns a copy of the raw
  tail (the reference returns the tail tensor itself).
"""

from __future__ import annotations

import threading

import numpy as np
import torch

from . import _kernels as K
from . import _lib
from .codecs import JPEGCodec, PNGCodec
from .codecs.jpeg import device_basis


def make_codec(mode="jpeg", block_size=8, keep_freqs=2, keep_ratio=1.0,
               quant_bits=0, scale_dtype=torch.float32, group_size=None):
    """Build a codec from a mode name (flashcodec/cache.py:39-54).
    ``scale_dtype`` and ``group_size`` (jpeg int8 only) are extensions; see
    JPEGCodec."""
    if mode == "jpeg":
        return JPEGCodec(block_size=block_size, keep_freqs=keep_freqs,
                         quant_bits=quant_bits, scale_dtype=scale_dtype,
                         group_size=group_size)
    if mode == "png":
        if group_size is not None:
            raise ValueError("group_size applies to the jpeg int8 codec only")
        if quant_bits:
            raise ValueError(f"quant_bits={quant_bits} applies to the jpeg codec only: png "
                             "stores fp32 deltas, which is what makes it lossless")
        return PNGCodec(block_size=block_size, keep_ratio=keep_ratio)
    raise ValueError(f"mode must be 'jpeg' or 'png', not {mode!r}")


class _CodecStream:
    """One (B, H, S, D) stream: raw tail + capacity-doubling archive
    (flashcodec/cache.py:57-325).

    jpeg: ``_coeffs (B,H,capacity,k,D)`` in the input dtype, or int8 with
    ``_scales (B,H,capacity,k,1)`` (fp32, or fp16 if the codec asks);
    png:  ``_deltas (B,H,capacity,r-1,D)`` fp32 + ``_anchors (B,H,capacity,D)``.
    """

    _INITIAL_BLOCKS = 16

    def __init__(self, codec):
        self.codec = codec
        self._raw_buf = None     # (B,H,r,D) input dtype: the partial block
        self._raw_len = 0
        self.n_archived = 0
        self.n_blocks = 0
        self.meta = None         # (B, H, D, elem_size)
        self.dtype = None
        self._capacity = 0
        self._coeffs = None
        self._scales = None
        self._deltas = None
        self._anchors = None
        self._rec = None         # (B,H,_rec_capacity,D) input dtype
        self._rec_blocks = 0
        self._rec_capacity = 0
        self._scale_err = None   # device int32: an fp16 scale could not hold its value

    # ------------------------------------------------------------ properties
    @property
    def block_size(self):
        return self.codec.block_size

    @property
    def raw(self):
        """Raw tail (B, H, t, D), t < block_size, or None (a view)."""
        if self._raw_len == 0:
            return None
        return self._raw_buf[:, :, :self._raw_len]

    @raw.setter
    def raw(self, t):
        if t is None:
            self._raw_len = 0
            return
        K.require_cuda(t)
        r = self.block_size
        if t.shape[2] >= r:
            raise ValueError("a raw tail is shorter than one block")
        self._ensure_raw(t)
        self._raw_buf[:, :, :t.shape[2]].copy_(t)
        self._raw_len = t.shape[2]

    @property
    def seq_len(self):
        return self.n_archived + self._raw_len

    # ------------------------------------------------------------- internals
    def _archive_spec(self, cap, B, H, D):
        """(attr, shape, dtype) for every archive tensor at capacity ``cap``."""
        if self.codec.name == "jpeg":
            k = self.codec.keep_freqs
            if self.codec.quantized:
                g = self.codec.group_size
                return [("_coeffs", (B, H, cap, k, D), torch.int8),
                        ("_scales", (B, H, cap, k, 1 if g is None else D // g),
                         self.codec.scale_dtype)]
            return [("_coeffs", (B, H, cap, k, D), self.dtype)]
        r = self.block_size
        return [("_deltas", (B, H, cap, r - 1, D), torch.float32),
                ("_anchors", (B, H, cap, D), self.dtype)]

    def _ensure_raw(self, like):
        B, H, D = like.shape[0], like.shape[1], like.shape[-1]
        rb = self._raw_buf
        if rb is None or rb.shape[0] != B or rb.shape[1] != H or rb.shape[-1] != D \
                or rb.device != like.device:
            new = torch.empty(B, H, self.block_size, D, dtype=self.dtype or like.dtype,
                              device=like.device)
            if rb is not None and self._raw_len and rb.shape == new.shape:
                new[:, :, :self._raw_len].copy_(rb[:, :, :self._raw_len])
            self._raw_buf = new

    def _grow(self, need_blocks, like):
        """Geometric growth from 16 blocks; old data copied verbatim
        (flashcodec/cache.py:106-121)."""
        if need_blocks <= self._capacity:
            return
        cap = max(self._INITIAL_BLOCKS, 1)
        while cap < need_blocks:
            cap *= 2
        B, H, D = like.shape[0], like.shape[1], like.shape[-1]
        for attr, shape, dtype in self._archive_spec(cap, B, H, D):
            new = torch.empty(shape, dtype=dtype, device=like.device)
            if self.n_blocks:
                new[:, :, :self.n_blocks].copy_(getattr(self, attr)[:, :, :self.n_blocks])
            setattr(self, attr, new)
        self._capacity = cap

    def _archive_from(self, src, n_full):
        """Compress ``n_full`` whole blocks of src (B,H,n_full*r,D) into the
        next archive slots, in place (flashcodec/cache.py:123-141)."""
        r = self.block_size
        sl = slice(self.n_blocks, self.n_blocks + n_full)
        x = K.as_bhsd(src)
        if self.codec.name == "jpeg":
            k = self.codec.keep_freqs
            basis = device_basis(r, k, x.device)
            if self.codec.quantized:
                if self.codec.scale_dtype == torch.float16 and self._scale_err is None:
                    self._scale_err = torch.zeros(1, dtype=torch.int32, device=x.device)
                if self.codec.group_size is not None:
                    K.jpeg_encode_grouped(x, basis, r, k, self._coeffs[:, :, sl],
                                          self._scales[:, :, sl], self.codec.group_size,
                                          self._scale_err)
                else:
                    K.jpeg_encode(x, basis, r, k, self._coeffs[:, :, sl],
                                  self._scales[:, :, sl], self._scale_err)
            else:
                K.jpeg_encode(x, basis, r, k, self._coeffs[:, :, sl])
        else:
            K.png_encode(x, r, self.codec.keep_m, self._deltas[:, :, sl], self._anchors[:, :, sl])
        self.n_blocks += n_full

    # ------------------------------------------------------------------ API
    def append(self, tokens):
        """Append (B,H,m,D); every completed block is archived immediately
        (flashcodec/cache.py:143-159)."""
        K.require_cuda(tokens)
        r = self.block_size
        if self.meta is None:
            self.meta = (tokens.shape[0], tokens.shape[1], tokens.shape[-1],
                         tokens.element_size())
            self.dtype = tokens.dtype
        if tokens.dtype != self.dtype:
            tokens = tokens.to(self.dtype)
        self._ensure_raw(tokens)
        m = tokens.shape[-2]
        t = self._raw_len
        n_full = (t + m) // r
        if n_full == 0:
            if m:
                self._raw_buf[:, :, t:t + m].copy_(tokens)
            self._raw_len = t + m
            return
        self._grow(self.n_blocks + n_full, tokens)
        used = 0
        if t:
            # complete the partial block in the raw buffer and archive it there
            self._raw_buf[:, :, t:r].copy_(tokens[:, :, :r - t])
            self._archive_from(self._raw_buf, 1)
            used = r - t
        nf = n_full - (1 if t else 0)
        if nf:
            self._archive_from(tokens[:, :, used:used + nf * r], nf)
            used += nf * r
        self.n_archived += n_full * r
        rem = m - used
        if rem:
            self._raw_buf[:, :, :rem].copy_(tokens[:, :, used:])
        self._raw_len = rem

    def _ensure_rec(self, need_tokens, like):
        if self._rec is not None and self._rec.shape[2] >= need_tokens:
            return
        r = self.block_size
        cap = max(need_tokens, self._rec_capacity * 2, self._INITIAL_BLOCKS * r)
        B, H, D = like.shape[0], like.shape[1], like.shape[-1]
        new = torch.empty((B, H, cap, D), dtype=self.dtype, device=like.device)
        if self._rec is not None and self._rec_blocks:
            done = self._rec_blocks * r
            new[:, :, :done].copy_(self._rec[:, :, :done])
        self._rec, self._rec_capacity = new, cap

    def _decode_pending(self):
        """Decode the blocks archived since the last read into ``_rec``
        (flashcodec/cache.py:161-193): O(new blocks) per read."""
        if self._rec_blocks >= self.n_blocks:
            return
        r = self.block_size
        a, b = self._rec_blocks, self.n_blocks
        like = self._coeffs if self.codec.name == "jpeg" else self._deltas
        self._ensure_rec((b + 1) * r, like)
        dst = self._rec[:, :, a * r:]
        if self.codec.name == "jpeg" and getattr(self.codec, "group_size", None) is not None:
            K.jpeg_decode_grouped(self._coeffs[:, :, a:b], self._scales[:, :, a:b],
                                  self.codec.group_size,
                                  device_basis(r, self.codec.keep_freqs, dst.device), r, dst,
                                  (b - a) * r)
        elif self.codec.name == "jpeg":
            k = self.codec.keep_freqs
            K.jpeg_decode(self._coeffs[:, :, a:b],
                          self._scales[:, :, a:b] if self.codec.quantized else None,
                          device_basis(r, k, dst.device), r, dst, (b - a) * r)
        else:
            K.png_decode(self._deltas[:, :, a:b], self._anchors[:, :, a:b], dst, (b - a) * r)
        self._rec_blocks = b

    def discard_view(self):
        """Drop the memoized reconstruction (flashcodec/cache.py:195-201)."""
        self._rec = None
        self._rec_blocks = 0
        self._rec_capacity = 0

    def read(self):
        """Reconstructed view (B,H,S,D) in the stream dtype
        (flashcodec/cache.py:203-220)."""
        if self.n_blocks == 0:
            return None if self._raw_len == 0 else self.raw.clone()
        self._decode_pending()
        L = self.n_archived
        if self._raw_len:
            self._ensure_rec(L + self._raw_len, self._raw_buf)
            self._rec[:, :, L:L + self._raw_len].copy_(self.raw)
        return self._rec[:, :, :L + self._raw_len]

    def reset(self):
        """Forget the contents, keep the capacity (flashcodec/cache.py:222-228)."""
        self._raw_len = 0
        self.n_archived = 0
        self.n_blocks = 0
        self._rec_blocks = 0

    def crop(self, tokens_to_remove):
        """Remove trailing tokens exactly (negative count, HF semantics;
        flashcodec/cache.py:230-257).  Archived blocks are kept verbatim; the
        partial block at the new boundary comes back as raw tail from its
        reconstruction, so repeated crops never add loss."""
        if tokens_to_remove > 0:
            raise ValueError("crop only supports negative values "
                             "(remove trailing tokens)")
        if tokens_to_remove == 0:
            return
        r = self.block_size
        keep = max(0, self.seq_len - abs(tokens_to_remove))
        keep_blocks = keep // r
        tail = keep - keep_blocks * r
        if keep_blocks < self.n_blocks:
            self._decode_pending()
            self.n_blocks = keep_blocks
            self.n_archived = keep_blocks * r
            self._rec_blocks = min(self._rec_blocks, keep_blocks)
            if tail:
                self._raw_buf[:, :, :tail].copy_(self._rec[:, :, keep_blocks * r:keep])
            self._raw_len = tail
        else:
            self._raw_len = tail

    def select_batch(self, idx):
        """Gather rows of the batch dim (beam search; flashcodec/cache.py:259-301).
        Every live prefix (archive, reconstruction, raw tail) is gathered into
        a new buffer by fc_gather_batch, one read and one write per byte;
        indices outside the batch raise IndexError."""
        if self._raw_len == 0 and self.n_blocks == 0 and self._rec is None:
            return
        like = (self._raw_buf if self._raw_buf is not None else
                (self._coeffs if self.codec.name == "jpeg" else self._deltas))
        idx = idx.to(device=like.device, dtype=torch.int64).contiguous()
        r = self.block_size
        if self._raw_buf is not None:
            self._raw_buf = K.gather_batch(self._raw_buf, idx, self._raw_buf.shape[2])
        if self._capacity:
            for attr, _, _ in self._archive_spec(self._capacity, *like.shape[:2], like.shape[-1]):
                setattr(self, attr, K.gather_batch(getattr(self, attr), idx, self.n_blocks))
        if self._rec is not None:
            # a new buffer also keeps views handed out by read() intact
            self._rec = K.gather_batch(self._rec, idx, self._rec_blocks * r)
        if self.meta is not None:
            self.meta = (idx.numel(),) + self.meta[1:]

    def _archive_tensors(self):
        """Live archive tensors (flashcodec/cache.py:303-308)."""
        if self.codec.name == "jpeg":
            return ((self._coeffs, self._scales) if self.codec.quantized
                    else (self._coeffs,))
        return (self._deltas, self._anchors)

    def storage_bytes(self):
        """Valid archive region + raw tail, excluding reserved capacity and the
        reconstruction view (flashcodec/cache.py:314-325)."""
        total = 0
        if self.n_blocks:
            for t in self._archive_tensors():
                total += t[:, :, :self.n_blocks].numel() * t.element_size()
        if self._raw_len:
            total += self.raw.numel() * self._raw_buf.element_size()
        return total

    def scale_range_errors(self) -> bool:
        """True if an fp16 scale could not hold the reference's fp32 scale
        exactly for some archived row (synchronises)."""
        return bool(self._scale_err is not None and int(self._scale_err.item()) != 0)


_APPEND_LOCAL = threading.local()


def _append_table(n):
    """Thread-local (ctypes AppendStream array, int64 numpy view) of >= n rows."""
    tbl = getattr(_APPEND_LOCAL, "tbl", None)
    if tbl is None or len(tbl[0]) < n:
        arr = (_lib.AppendStream * max(n, 64))()
        tbl = (arr, np.frombuffer(arr, dtype=np.int64).reshape(len(arr), 8))
        _APPEND_LOCAL.tbl = tbl
    return tbl


def append_one_token(streams, tokens) -> bool:
    """Append one token to every jpeg stream in ``streams`` with a single
    fc_append_tokens launch, archiving in the same launch the blocks it
    completes.  ``tokens[i]`` is the (B, H, 1, D) token of ``streams[i]``.
    Returns False, having changed nothing, when the streams do not share one
    layout (codec settings, dtype, shape, raw position, archived blocks,
    device) or a layout the launch does not take; the caller then appends
    stream by stream.  Results are bit-identical to ``append``."""
    st0, t0 = streams[0], tokens[0]
    c0 = st0.codec
    if c0.name != "jpeg" or c0.keep_freqs > 8 or c0.block_size > 64 or t0.dim() != 4 \
            or c0.group_size is not None:
        return False
    B, H, m, D = t0.shape
    r, pos, nb = c0.block_size, st0._raw_len, st0.n_blocks
    if m != 1 or D % 4 or D > 512 or t0.dtype not in (torch.float32, torch.bfloat16,
                                                      torch.float16):
        return False
    es = t0.element_size()
    dev = t0.device
    for st, tk in zip(streams, tokens):
        c = st.codec
        if (c.name != "jpeg" or c.block_size != r or c.keep_freqs != c0.keep_freqs
                or c.quant_bits != c0.quant_bits or c.scale_dtype != c0.scale_dtype
                or c.group_size is not None):
            return False
        rb = st._raw_buf
        if (st.meta is None or rb is None or st.dtype != tk.dtype or tk.shape != t0.shape
                or tk.device != dev or tk.stride(-1) != 1 or st._raw_len != pos
                or st.n_blocks != nb or rb.shape != (B, H, r, D) or not rb.is_contiguous()
                or rb.device != dev or tk.data_ptr() % (4 * es) or tk.stride(0) % 4
                or tk.stride(1) % 4):
            return False
    archive = pos == r - 1
    if archive:
        for st in streams:
            st._grow(nb + 1, st._raw_buf)
            if not st._coeffs.is_contiguous() or (st._scales is not None
                                                  and not st._scales.is_contiguous()):
                return False
    quant = c0.quantized
    fp16 = quant and c0.scale_dtype == torch.float16
    if fp16:
        for st in streams:
            if st._scale_err is None:
                st._scale_err = torch.zeros(1, dtype=torch.int32, device=dev)
    n = len(streams)
    arr, tab = _append_table(n)
    tab[:n, 0] = [tk.data_ptr() for tk in tokens]
    tab[:n, 1] = [tk.stride(0) for tk in tokens]
    tab[:n, 2] = [tk.stride(1) for tk in tokens]
    tab[:n, 3] = [st._raw_buf.data_ptr() for st in streams]
    if archive:
        tab[:n, 4] = [st._coeffs.data_ptr() for st in streams]
        tab[:n, 5] = [st._scales.data_ptr() for st in streams] if quant else 0
        tab[:n, 6] = [st._capacity for st in streams]
        tab[:n, 7] = [st._scale_err.data_ptr() for st in streams] if fp16 else 0
    else:
        tab[:n, 4:] = 0
    K.append_tokens(arr, n, t0.dtype, B, H, D, r, c0.keep_freqs, pos, nb,
                    device_basis(r, c0.keep_freqs, dev) if archive else None,
                    c0.scale_dtype if quant else None, dev)
    for st in streams:
        if archive:
            st.n_blocks = nb + 1
            st.n_archived += r
            st._raw_len = 0
        else:
            st._raw_len = pos + 1
    return True


def append_rotary(key_stream, value_stream, q, k, v, cos, sin):
    """One decode token of one layer: rotary embedding of q and k and the
    append of (rotated k, v) to the layer's streams in one launch
    (fc_rope_kv_append writes straight into the raw-tail slot); a block that
    this token completes is archived as ``append`` would archive it.

    q (B,Hq,1,D), k and v (B,Hk,1,D) before the rotation; cos/sin (B or 1,
    [1,] D) in the same dtype (rotate-half form, transformers'
    ``apply_rotary_pos_emb``).  Returns the rotated q (B,Hq,1,D); the streams
    end up bit-identical to ``rope`` followed by two ``append`` calls."""
    ks, vs = key_stream, value_stream
    K.require_cuda(q, k, v)
    for st, x in ((ks, k), (vs, v)):
        if st.meta is None:
            st.meta = (x.shape[0], x.shape[1], x.shape[-1], x.element_size())
            st.dtype = x.dtype
    if k.dtype != ks.dtype or v.dtype != vs.dtype or ks._raw_len != vs._raw_len \
            or ks.block_size != vs.block_size:
        raise ValueError("append_rotary: the key and value streams must match the tokens "
                         "and each other")
    ks._ensure_raw(k)
    vs._ensure_raw(v)
    t = ks._raw_len
    q_out = torch.empty_like(q)
    K.rope_kv_append(q, k, v, cos, sin, q_out, ks._raw_buf[:, :, t], vs._raw_buf[:, :, t])
    ks._raw_len = vs._raw_len = t + 1
    if t + 1 == ks.block_size:
        for st in (ks, vs):
            st._grow(st.n_blocks + 1, st._raw_buf)
            st._archive_from(st._raw_buf, 1)
            st.n_archived += st.block_size
            st._raw_len = 0
    return q_out


class CodecKVCache:
    """Compressed K and V streams for every layer of a model, with the
    method names of a HuggingFace Cache (flashcodec/cache.py:328-440).

    ``update(k, v, layer_idx)`` appends new tokens of one layer and returns
    that layer's reconstructed (K, V) views; ``append`` only appends (the
    decode-attention path reads the archive directly); ``forward`` replaces a
    layer's contents with a whole sequence.  All tensors are (B, H, S, D) on
    one CUDA device, for example::

        kv = CodecKVCache("jpeg", block_size=8, keep_freqs=4, quant_bits=8)
        kv.append(k_prompt, v_prompt, layer_idx=3)
        out = codec_decode_attention(q, kv._keys[3], kv._values[3])
    """

    def __init__(self, mode="jpeg", block_size=8, keep_freqs=2,
                 keep_ratio=1.0, quant_bits=0, scale_dtype=torch.float32, group_size=None):
        self.mode = mode
        self.codec = make_codec(mode, block_size, keep_freqs, keep_ratio,
                                quant_bits=quant_bits, scale_dtype=scale_dtype,
                                group_size=group_size)
        self._keys = {}
        self._values = {}

    def _stream(self, store, layer_idx):
        st = store.get(layer_idx)
        if st is None:
            st = _CodecStream(self.codec)
            store[layer_idx] = st
        return st

    def update(self, key_states, value_states, layer_idx=0):
        """Append (B,H,m,D) to both streams of a layer; returns the layer's
        reconstructed (key_view, value_view)."""
        self._stream(self._keys, layer_idx).append(key_states)
        self._stream(self._values, layer_idx).append(value_states)
        return (self._keys[layer_idx].read(), self._values[layer_idx].read())

    decode_step = update

    def append(self, key_states, value_states, layer_idx=0):
        """Append without materialising the view (the decode-attention path).
        A single token goes to both streams in one launch when they allow it
        (fc_append_tokens), else stream by stream."""
        ks = self._stream(self._keys, layer_idx)
        vs = self._stream(self._values, layer_idx)
        if key_states.dim() == 4 and key_states.shape[-2] == 1 and \
                append_one_token((ks, vs), (key_states, value_states)):
            return
        ks.append(key_states)
        vs.append(value_states)

    def append_layers(self, key_states, value_states, layer_ids=None):
        """Append one decode token to several layers at once: ``key_states[i]``
        and ``value_states[i]`` ((B, H, 1, D) each) go to layer
        ``layer_ids[i]`` (default: layers 0, 1, ...).  When every stream
        shares one layout, all of them -- K and V of every layer, including
        the archive of the blocks this token completes -- take a single
        fc_append_tokens launch; otherwise each layer is appended in turn.
        An extension of the reference API for engines that produce a step's
        K/V for many layers together (e.g. replaying a cached step)."""
        ids = list(range(len(key_states))) if layer_ids is None else list(layer_ids)
        if not (len(ids) == len(key_states) == len(value_states)):
            raise ValueError("one key and one value tensor per layer id")
        streams, tokens = [], []
        for i, k, v in zip(ids, key_states, value_states):
            streams += [self._stream(self._keys, i), self._stream(self._values, i)]
            tokens += [k, v]
        if streams and all(t.dim() == 4 and t.shape[-2] == 1 for t in tokens) and \
                append_one_token(streams, tokens):
            return
        for i, k, v in zip(ids, key_states, value_states):
            self.append(k, v, i)

    def forward(self, key_seq, value_seq, layer_idx=0):
        """Reset the layer, fill it with the whole sequence, return the view."""
        self.reset(layer_idx)
        return self.update(key_seq, value_seq, layer_idx)

    def reset(self, layer_idx=None):
        if layer_idx is None:
            self._keys.clear()
            self._values.clear()
        else:
            self._keys.pop(layer_idx, None)
            self._values.pop(layer_idx, None)

    def crop(self, tokens_to_remove, layer_idx=None):
        for store in (self._keys, self._values):
            for i, st in store.items():
                if layer_idx is None or i == layer_idx:
                    st.crop(tokens_to_remove)

    def reorder_cache(self, beam_idx, layer_idx=None):
        for store in (self._keys, self._values):
            for i, st in store.items():
                if layer_idx is None or i == layer_idx:
                    st.select_batch(beam_idx)

    @property
    def key_cache(self):
        mx = max(self._keys, default=-1)
        return [self._keys[i].read() if i in self._keys else None for i in range(mx + 1)]

    @property
    def value_cache(self):
        mx = max(self._values, default=-1)
        return [self._values[i].read() if i in self._values else None for i in range(mx + 1)]

    def get_seq_length(self, layer_idx=0):
        st = self._keys.get(layer_idx)
        return 0 if st is None else st.seq_len

    def get_max_length(self):
        return None

    def get_usable_length(self, new_seq_length, layer_idx=0):
        return self.get_seq_length(layer_idx)

    def storage_bytes(self, layer_idx=None):
        layers = ([layer_idx] if layer_idx is not None
                  else sorted(set(self._keys) | set(self._values)))
        return sum(self._keys[i].storage_bytes() for i in layers if i in self._keys) + \
            sum(self._values[i].storage_bytes() for i in layers if i in self._values)

    def stats(self, layer_idx=0):
        """Token counts and byte sizes of one layer: compressed storage
        (archive plus raw tail, K and V) next to what the same tokens take
        uncompressed in the stream dtype."""
        st = self._keys.get(layer_idx)
        if st is None or st.meta is None:
            return dict.fromkeys(("tokens", "archived", "raw", "storage_bytes", "raw_bytes"), 0)
        B, H, D, elem = st.meta
        seq = st.seq_len
        return {"tokens": seq, "archived": st.n_archived, "raw": seq - st.n_archived,
                "storage_bytes": self.storage_bytes(layer_idx),
                "raw_bytes": 2 * seq * B * H * D * elem}

    def __repr__(self):
        layers = sorted(set(self._keys) | set(self._values))
        return f"CodecKVCache({self.codec!r} over {len(layers)} layer(s) {layers})"


def __getattr__(name):
    """The transformers-backed classes load on first use (importing
    transformers takes seconds)."""
    if name in ("FlashCodecCache", "FlashCodecLayer", "HAS_HF_CACHE"):
        from . import hf_cache
        return getattr(hf_cache, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
