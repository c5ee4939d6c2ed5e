"""One-call patch: a HuggingFace causal LM generates with a codec KV cache.

Same entry points and behaviour as flashcodec/patch.py:31-136
(``apply_flash_codec``, ``remove_flash_codec``, ``undo_flash_codec``,
``find_attention_modules``).  The model's ``generate`` and ``forward`` are
wrapped so that a call that wants a cache and passes none gets a fresh
``FlashCodecCache`` (or ``CodecKVCache`` without transformers); every KV write
and read then goes through the cache interface, so no attention code changes.
``materialization_free=True`` also patches the attention modules so decode
steps attend on the archive directly (``patch_attention``).
"""

from __future__ import annotations

import functools
import warnings

__all__ = ["apply_flash_codec", "remove_flash_codec", "undo_flash_codec",
           "find_attention_modules"]


def find_attention_modules(model):
    """Modules with k_proj and v_proj (standard KV-projection attention)."""
    return [m for m in model.modules() if hasattr(m, "k_proj") and hasattr(m, "v_proj")]


def _cache_factory(mode, block_size, kwargs, sink, config):
    from .cache import CodecKVCache
    from .hf_cache import HAS_HF_CACHE, FlashCodecCache
    codec = dict(keep_freqs=kwargs.get("keep_freqs", 2),
                 keep_ratio=kwargs.get("keep_ratio", 1.0),
                 quant_bits=kwargs.get("quant_bits", 0))
    for opt in ("scale_dtype", "group_size"):
        if opt in kwargs:
            codec[opt] = kwargs[opt]
    per_layer = kwargs.get("per_layer")

    def make():
        cache = None
        if not HAS_HF_CACHE:
            cache = CodecKVCache(mode=mode, block_size=block_size, **codec)
        elif config is not None:
            try:    # hybrid models: codec layers only where attention is full
                cache = FlashCodecCache.from_config(config, mode=mode, block_size=block_size,
                                                    per_layer=per_layer, **codec)
            except Exception:
                cache = None
        if cache is None:
            cache = FlashCodecCache(mode=mode, block_size=block_size, **codec)
        sink.append(cache)
        return cache

    return make


def apply_flash_codec(model, mode="jpeg", block_size=8, materialization_free=False,
                      **kwargs):
    """Give every ``generate(..., use_cache=True)`` / ``forward(use_cache=True)``
    call without ``past_key_values`` a codec cache.  kwargs: ``keep_freqs``
    (jpeg, default 2), ``quant_bits`` (0 or 8), ``keep_ratio`` (png, default
    1.0), ``per_layer`` (codec overrides by layer index), ``scale_dtype``,
    ``group_size`` (per-group scales of the int8 jpeg archive, e.g. 32).
    Returns the model; ``remove_flash_codec`` undoes it."""
    if getattr(model, "_flashcodec", None) is not None:
        warnings.warn("model is already patched with flashcodec, "
                      "call remove_flash_codec first")
        return model
    attns = find_attention_modules(model)
    caches = []
    make = _cache_factory(mode, block_size, kwargs, caches, getattr(model, "config", None))
    base_generate, base_forward = model.generate, model.forward

    @functools.wraps(base_generate)
    def generate(*args, **kw):
        use_cache = kw.get("use_cache")
        if (use_cache is None or use_cache) and kw.get("past_key_values") is None:
            kw["past_key_values"] = make()
        return base_generate(*args, **kw)

    @functools.wraps(base_forward)
    def forward(*args, **kw):
        if kw.get("use_cache") and kw.get("past_key_values") is None:
            kw["past_key_values"] = make()
        return base_forward(*args, **kw)

    model.generate, model.forward = generate, forward
    wrapped = 0
    if materialization_free:
        from .patch_attention import apply_codec_attention
        wrapped = apply_codec_attention(model)

    def undo():
        from .patch_attention import remove_codec_attention
        remove_codec_attention(model)
        model.generate, model.forward = base_generate, base_forward
        model._flashcodec = None

    model._flashcodec = {"mode": mode, "caches": caches, "attention_modules": attns,
                         "codec_attention_modules": wrapped, "undo": undo}
    if not attns:
        warnings.warn("no attention module with k_proj/v_proj found; a model with "
                      "a non-standard KV interface may not use the codec cache")
    return model


def remove_flash_codec(model):
    """Undo ``apply_flash_codec`` (restores generate, forward and attention)."""
    info = getattr(model, "_flashcodec", None)
    if info is not None:
        info["undo"]()


undo_flash_codec = remove_flash_codec
