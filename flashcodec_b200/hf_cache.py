"""transformers 5.x Cache backend over the codec streams.

Same classes, arguments and attributes as flashcodec/cache.py:446-654
(``FlashCodecLayer``, ``FlashCodecCache``).  A layer holds one key and one
value ``_CodecStream``; ``update`` appends through the sm_100a archive kernels
and hands attention the reconstructed view, so a model needs no surgery.

Behaviour beyond the reference, none of it changing a value:

* ``crop(max_length)`` follows the transformers convention for both signs:
  a negative count removes that many trailing tokens (the reference's only
  form), a non-negative value keeps the first ``max_length`` tokens (the
  form assisted generation uses; the reference raises there).
* Structural changes (``crop``, beam reordering, batch selection) re-read the
  attention-facing view only when the layer holds one.  A layer driven by the
  coefficient-domain decode path (``keys is None``) stays view-free, so beam
  search never reconstructs the archive.
* ``from_config`` dispatches non-codec layer types the way
  ``DynamicCache(config=...)`` does in the installed transformers (sliding and
  chunked windows, linear-attention / recurrent state, hybrid layers).

Importing this module imports transformers (a few seconds); the package
exposes these names lazily.
"""

from __future__ import annotations

from functools import partial

import torch

from .cache import CodecKVCache, _CodecStream, make_codec

try:
    from transformers import cache_utils as _hf
    _HFCache = _hf.Cache
    _HFDynamicLayer = _hf.DynamicLayer
    HAS_HF_CACHE = True
except Exception:  # transformers missing or without the layer-container API
    _hf = None
    _HFCache = object
    _HFDynamicLayer = object
    HAS_HF_CACHE = False


class FlashCodecLayer(_HFDynamicLayer):
    """One attention layer's cache: key and value codec streams
    (flashcodec/cache.py:446-562)."""

    def __init__(self, mode="jpeg", block_size=8, keep_freqs=2, keep_ratio=1.0,
                 quant_bits=0, scale_dtype=torch.float32, group_size=None):
        if HAS_HF_CACHE:
            super().__init__()
        else:
            self.keys = self.values = None
            self.is_initialized = False
        self.mode = mode
        self.codec = make_codec(mode, block_size, keep_freqs, keep_ratio,
                                quant_bits=quant_bits, scale_dtype=scale_dtype,
                                group_size=group_size)
        self._key_stream = _CodecStream(self.codec)
        self._value_stream = _CodecStream(self.codec)

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        self.keys = key_states.new_empty(0)
        self.values = value_states.new_empty(0)
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        """Append (B,H,m,D) to both streams (archiving every completed block)
        and return the reconstructed (keys, values) views."""
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self._key_stream.append(key_states)
        self._value_stream.append(value_states)
        self.keys = self._key_stream.read()
        self.values = self._value_stream.read()
        return self.keys, self.values

    def get_seq_length(self):
        return self._key_stream.seq_len

    def get_mask_sizes(self, query_length):
        return self.get_seq_length() + query_length, 0

    def get_max_cache_shape(self):
        return -1

    def get_max_length(self):
        return -1

    # ------------------------------------------------------ structural ops
    def crop(self, max_length):
        """Drop trailing tokens; archived blocks are kept verbatim and only
        the partial block at the new boundary returns to the raw tail."""
        n = self.get_seq_length()
        if max_length >= 0:
            if max_length >= n:
                return
            max_length = max_length - n        # as a (negative) removal count
        if max_length == 0:
            return
        self._key_stream.crop(max_length)
        self._value_stream.crop(max_length)
        self._rebuild_views()

    def reorder_cache(self, beam_idx):
        """Beam search: gather the batch rows of both streams (archive, raw
        tail and reconstruction alike)."""
        self.select_batch(beam_idx)

    def batch_repeat_interleave(self, repeats):
        """Contrastive search: replicate every batch row ``repeats`` times."""
        if not self.is_initialized or self._key_stream.meta is None:
            return
        B = self._key_stream.meta[0]
        idx = torch.arange(B, device=self.device).repeat_interleave(repeats)
        self.select_batch(idx)

    def batch_select_indices(self, indices):
        """Contrastive search: keep only the given batch rows."""
        if not self.is_initialized or self._key_stream.meta is None:
            return
        self.select_batch(indices)

    def select_batch(self, idx):
        self._key_stream.select_batch(idx)
        self._value_stream.select_batch(idx)
        self._rebuild_views()

    def _rebuild_views(self):
        if not self.is_initialized or self.keys is None:
            return                              # view-free (decode path) layer
        if self._key_stream.seq_len > 0:
            self.keys = self._key_stream.read()
            self.values = self._value_stream.read()
        else:
            self.keys = torch.empty(0, dtype=self.dtype, device=self.device)
            self.values = torch.empty(0, dtype=self.dtype, device=self.device)

    def reset(self):
        self._key_stream.reset()
        self._value_stream.reset()
        if self.is_initialized:
            self.keys = torch.empty(0, dtype=self.dtype, device=self.device)
            self.values = torch.empty(0, dtype=self.dtype, device=self.device)

    def offload(self):
        """The archive stays in device memory (no layer offload)."""

    def prefetch(self):
        """Nothing to prefetch: see ``offload``."""

    def storage_bytes(self):
        return self._key_stream.storage_bytes() + self._value_stream.storage_bytes()


def _layer_types(decoder):
    """Per-layer attention types of a decoder config, derived the way
    ``DynamicCache(config=...)`` derives them."""
    window = (getattr(decoder, "sliding_window", None)
              or getattr(decoder, "attention_chunk_size", None))
    types = getattr(decoder, "layer_types", None)
    if types is None:
        kind = "sliding_attention" if window is not None else "full_attention"
        types = [kind] * int(getattr(decoder, "num_hidden_layers", 1))
    types = list(types)
    shared = getattr(decoder, "num_kv_shared_layers", None)
    if shared:
        types = types[:-shared]
    return types, window


def _native_layer(ltype, window):
    """The transformers layer a non-codec layer type gets."""
    if ltype in ("sliding_attention", "chunked_attention"):
        return _hf.DynamicSlidingWindowLayer(sliding_window=window)
    if ltype in ("mamba", "conv", "linear_attention", "moe"):
        return _hf.LinearAttentionLayer()
    if ltype == "hybrid":
        return _hf.LinearAttentionAndFullAttentionLayer()
    return _hf.DynamicLayer()


class FlashCodecCache(_HFCache):
    """transformers 5.x codec KV cache (flashcodec/cache.py:565-654).

        cache = FlashCodecCache(mode="jpeg", block_size=8, keep_freqs=2)
        model.generate(input_ids, past_key_values=cache, use_cache=True)

    Layers are created lazily (one ``FlashCodecLayer`` per attention layer
    index); ``from_config`` builds a mixed list for hybrid architectures.
    """

    def __init__(self, mode="jpeg", block_size=8, keep_freqs=2, keep_ratio=1.0,
                 quant_bits=0, scale_dtype=torch.float32, group_size=None):
        if not HAS_HF_CACHE:
            raise ImportError("FlashCodecCache needs the transformers 5.x Cache "
                              "classes; use CodecKVCache without transformers")
        # a bad configuration raises here rather than at the first update
        make_codec(mode, block_size, keep_freqs, keep_ratio, quant_bits=quant_bits,
                   scale_dtype=scale_dtype, group_size=group_size)
        super().__init__(layer_class_to_replicate=partial(
            FlashCodecLayer, mode=mode, block_size=block_size, keep_freqs=keep_freqs,
            keep_ratio=keep_ratio, quant_bits=quant_bits, scale_dtype=scale_dtype,
            group_size=group_size))
        self.mode = mode
        self.codec_cfg = dict(block_size=block_size, keep_freqs=keep_freqs,
                              keep_ratio=keep_ratio, quant_bits=quant_bits)

    @property
    def _seen_tokens(self):
        """Token counter of older transformers versions (the sequence length)."""
        return self.get_seq_length()

    @classmethod
    def from_config(cls, config, mode="jpeg", block_size=8, keep_freqs=2,
                    keep_ratio=1.0, quant_bits=0, per_layer=None,
                    scale_dtype=torch.float32, group_size=None):
        """One layer per decoder layer: full-attention layers get a codec
        layer, every other type its native transformers layer.  ``per_layer``
        maps a layer index to codec overrides, e.g.
        ``{3: {"keep_freqs": 4}, 7: {"quant_bits": 8}}``."""
        if not HAS_HF_CACHE:
            raise ImportError("FlashCodecCache needs the transformers 5.x Cache classes")
        decoder = (config.get_text_config(decoder=True)
                   if hasattr(config, "get_text_config") else config)
        types, window = _layer_types(decoder)
        per_layer = per_layer or {}
        base = dict(mode=mode, block_size=block_size, keep_freqs=keep_freqs,
                    keep_ratio=keep_ratio, quant_bits=quant_bits, scale_dtype=scale_dtype,
                    group_size=group_size)
        layers = []
        for i, ltype in enumerate(types):
            if ltype == "full_attention":
                layers.append(FlashCodecLayer(**{**base, **per_layer.get(i, {})}))
            else:
                layers.append(_native_layer(ltype, window))
        obj = cls.__new__(cls)
        _HFCache.__init__(obj, layers=layers)
        obj.mode = mode
        obj.codec_cfg = dict(block_size=block_size, keep_freqs=keep_freqs,
                             keep_ratio=keep_ratio, quant_bits=quant_bits,
                             per_layer=per_layer)
        return obj

    def codec_layer_indices(self):
        """Indices of the layers that carry a codec."""
        return [i for i, layer in enumerate(self.layers) if isinstance(layer, FlashCodecLayer)]

    def to_legacy_cache(self):
        """{layer_idx: (keys, values)} with the reconstructed views."""
        return {i: (layer.keys, layer.values) for i, layer in enumerate(self.layers)}

    @classmethod
    def from_legacy_cache(cls, legacy, **cfg):
        """Rebuild from {layer_idx: (keys, values)}; every span is encoded
        once more."""
        cache = cls(**cfg)
        for i in sorted(legacy):
            k, v = legacy[i]
            cache.update(k, v, i)
        return cache

    def storage_bytes(self, layer_idx=None):
        layers = self.layers if layer_idx is None else [self.layers[layer_idx]]
        return sum(layer.storage_bytes() for layer in layers
                   if isinstance(layer, FlashCodecLayer))


__all__ = ["FlashCodecLayer", "FlashCodecCache", "HAS_HF_CACHE", "CodecKVCache"]
