"""The per-group quantizer restatement in the oracle (CPU): each group of a
row quantized like a reference row, checked against an independent numpy
statement of quantize_coeffs' formula (flashcodec/codecs/jpeg.py:85-100):
scale = dtype(amax / 127) (1 if zero), code = clamp(rint(c / scale), +-127)."""

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from oracle import oracle as orc  # noqa: E402


def _direct(c, group, dtype):
    g = c.reshape(*c.shape[:-1], -1, group)
    amax = np.abs(g).max(axis=-1, keepdims=True)
    scale = orc.round_to(amax / np.float32(127.0), dtype)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(g / scale), -127, 127).astype(np.int8)
    return q.reshape(c.shape), scale[..., 0]


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("group", [4, 16, 32, 128])
def test_grouped_quantizer_matches_formula(dtype, group):
    rng = np.random.default_rng(group)
    c = orc.round_to(rng.standard_normal((3, 5, 2, 128)).astype(np.float32)
                     * rng.lognormal(0, 2, (3, 5, 2, 1)).astype(np.float32), dtype)
    c[0, 0, 0, :group] = 0.0                      # an all-zero group: scale 1
    codes, scales = orc.jpeg_quantize_grouped(c, group, dtype)
    q, s = _direct(c, group, dtype)
    assert scales.shape == c.shape[:-1] + (128 // group,)
    assert np.array_equal(codes, q)
    assert np.array_equal(scales.view(np.uint32), s.astype(np.float32).view(np.uint32))
    assert scales[0, 0, 0, 0] == 1.0
    # group == D is the reference's row quantizer
    if group == 128:
        rc, rs = orc.jpeg_quantize(c, dtype)
        assert np.array_equal(rc, codes) and np.array_equal(rs[..., 0], scales[..., 0])
    rows = orc.dequantize_grouped(codes, scales)
    assert np.all(np.abs(rows - c) <= np.repeat(scales, group, axis=-1) * 0.5 + 1e-12)
