"""fc_rope_kv_append: the decode-step rotary embedding fused with the cache
append, against transformers' own apply_rotary_pos_emb and the unfused
rope-then-append sequence (bit-exact: the kernel rounds where torch rounds)."""

import pytest
import torch

pytest.importorskip("transformers")
from transformers.models.llama.modeling_llama import (  # noqa: E402
    LlamaConfig, LlamaRotaryEmbedding, apply_rotary_pos_emb)

import flashcodec_b200 as fc  # noqa: E402
from flashcodec_b200 import _kernels as K  # noqa: E402
from flashcodec_b200.cache import append_rotary  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"


def cos_sin(B, D, pos, dtype):
    cfg = LlamaConfig(hidden_size=D * 2, num_attention_heads=2, head_dim=D)
    rot = LlamaRotaryEmbedding(cfg, device=DEV)
    x = torch.zeros(1, dtype=dtype, device=DEV)
    ids = torch.as_tensor(pos, device=DEV).view(B, 1)
    return rot(x, ids)                           # (B, 1, D) each, in dtype


def hf_layout(B, H, D, dtype, seed):
    """A (B, H, 1, D) view with the strides of a projection's transpose."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(B, 1, H, D, generator=g, device=DEV).to(dtype).transpose(1, 2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Hq,Hk,D", [(1, 4, 2, 16), (3, 32, 8, 128), (2, 6, 3, 64)])
def test_rotation_matches_transformers_bitwise(dtype, B, Hq, Hk, D):
    q, k, v = hf_layout(B, Hq, D, dtype, 1), hf_layout(B, Hk, D, dtype, 2), hf_layout(B, Hk, D, dtype, 3)
    cos, sin = cos_sin(B, D, [37 + 1000 * b for b in range(B)], dtype)
    q_ref, k_ref = apply_rotary_pos_emb(q, k, cos, sin)
    q_o, k_o, v_o = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    K.rope_kv_append(q, k, v, cos, sin, q_o, k_o, v_o)
    assert torch.equal(q_o, q_ref)
    assert torch.equal(k_o, k_ref)
    assert torch.equal(v_o, v)


def test_shared_position_broadcasts_over_the_batch():
    q, k = hf_layout(4, 8, 64, torch.bfloat16, 4), hf_layout(4, 2, 64, torch.bfloat16, 5)
    cos, sin = cos_sin(1, 64, [123], torch.bfloat16)
    q_ref, k_ref = apply_rotary_pos_emb(q, k, cos, sin)
    q_o, k_o = torch.empty_like(q), torch.empty_like(k)
    K.rope_kv_append(q, k, None, cos, sin, q_o, k_o)
    assert torch.equal(q_o, q_ref) and torch.equal(k_o, k_ref)


def test_wrapper_refuses_mixed_dtypes_and_bad_shapes():
    q, k = hf_layout(2, 4, 32, torch.bfloat16, 6), hf_layout(2, 2, 32, torch.bfloat16, 7)
    cos, sin = cos_sin(2, 32, [1, 2], torch.float32)
    with pytest.raises(ValueError):
        K.rope_kv_append(q, k, None, cos, sin, torch.empty_like(q), torch.empty_like(k))
    cos, sin = cos_sin(2, 32, [1, 2], torch.bfloat16)
    with pytest.raises(ValueError):
        K.rope_kv_append(q, k, k, cos, sin, torch.empty_like(q), torch.empty_like(k))
    with pytest.raises(ValueError):
        K.rope_kv_append(q, k, None, cos[..., :16], sin[..., :16], torch.empty_like(q),
                         torch.empty_like(k))


def _archive(st):
    return [t[:, :, :st.n_blocks].clone() for t in st._archive_tensors()]


@pytest.mark.parametrize("mode,kw,dtype", [
    ("jpeg", dict(keep_freqs=4, quant_bits=8), torch.bfloat16),
    ("jpeg", dict(keep_freqs=2), torch.float32),
    ("png", dict(keep_ratio=1.0), torch.float16)])
def test_append_rotary_equals_rope_then_append(mode, kw, dtype):
    """21 decode tokens (two archived blocks and a 5-token tail) through the
    fused path and through rope + two appends: identical archives, raw tails
    and rotated queries."""
    B, Hq, Hk, D, r = 3, 8, 2, 128, 8
    c = fc.make_codec(mode, block_size=r, **kw)
    fused = (fc._CodecStream(c), fc._CodecStream(c))
    plain = (fc._CodecStream(c), fc._CodecStream(c))
    for t in range(21):
        q, k, v = (hf_layout(B, h, D, dtype, 10 * t + i) for i, h in enumerate((Hq, Hk, Hk)))
        cos, sin = cos_sin(B, D, [t + 5 * b for b in range(B)], dtype)
        q_f = append_rotary(*fused, q, k, v, cos, sin)
        q_r, k_r = apply_rotary_pos_emb(q, k, cos, sin)
        plain[0].append(k_r)
        plain[1].append(v)
        assert torch.equal(q_f, q_r)
    for f, p in zip(fused, plain):
        assert (f.n_blocks, f.n_archived, f._raw_len) == (p.n_blocks, p.n_archived, p._raw_len) \
            == (2, 16, 5)
        for a, b in zip(_archive(f), _archive(p)):
            assert torch.equal(a, b)
        assert torch.equal(f.raw, p.raw)
        assert torch.equal(f.read(), p.read())
