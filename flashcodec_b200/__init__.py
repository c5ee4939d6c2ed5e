"""flashcodec_b200 -- B200-native (sm_100a) implementation of flashcodec's
compressed-KV hot path, with flashcodec's Python API.

KV layout (B, H, S, D), compression along the sequence axis (dim=-2):
- mode="jpeg": blockwise orthonormal DCT-II, keep K of r coefficients,
  optionally int8 with a per-(block, frequency) scale;
- mode="png": per-block anchor + fp32 first-order deltas, Top-M pruning.
Decode attention runs directly on the compressed archive.

All arithmetic runs in hand-written CUDA kernels (libflashcodec_sm100.so,
C ABI in include/flashcodec_b200.h).  CUDA tensors only: there is no CPU
implementation in this package.
"""

from .attention import attention_status, block_basis, codec_decode_attention
from .cache import CodecKVCache, _CodecStream, make_codec
from .codecs import (JPEGCodec, PNGCodec, dct_basis, dct_compress, dct_decompress,
                     dequantize_coeffs, png_filter, png_reconstruct, quantize_coeffs)
from .patch import (apply_flash_codec, find_attention_modules, remove_flash_codec,
                    undo_flash_codec)
from .patch_attention import (apply_codec_attention, codec_attention_stats,
                              remove_codec_attention)

__version__ = "0.1.0"

_LAZY = ("FlashCodecCache", "FlashCodecLayer", "HAS_HF_CACHE")


def __getattr__(name):
    """transformers-backed names load on first use (flashcodec/__init__.py:15-16
    imports them eagerly; importing transformers takes seconds)."""
    if name in _LAZY:
        from . import hf_cache
        return getattr(hf_cache, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = [
    "apply_flash_codec", "remove_flash_codec", "undo_flash_codec",
    "find_attention_modules",
    "apply_codec_attention", "remove_codec_attention", "codec_attention_stats",
    "CodecKVCache", "FlashCodecCache", "FlashCodecLayer", "make_codec",
    "HAS_HF_CACHE", "JPEGCodec", "PNGCodec",
    "codec_decode_attention", "block_basis", "attention_status",
    "dct_basis", "dct_compress", "dct_decompress",
    "quantize_coeffs", "dequantize_coeffs",
    "png_filter", "png_reconstruct",
    "__version__",
]
