"""Host-side logic of the transformers integration (no GPU): layer-type
dispatch of ``FlashCodecCache.from_config``, patch/unpatch bookkeeping, the
fallback of the patched attention to the model's own forward, and the
absence of a CPU path for the codec cache itself."""

import warnings

import pytest
import torch

pytest.importorskip("transformers")
from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM  # noqa: E402
from transformers import cache_utils as hf  # noqa: E402

import flashcodec_b200 as fc  # noqa: E402


def tiny_llama(seed=7):
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=128, hidden_size=32, intermediate_size=64,
                      num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=2,
                      max_position_embeddings=256)
    m = LlamaForCausalLM(cfg).eval()
    m.generation_config.eos_token_id = None
    return m


def test_lazy_exports():
    assert fc.HAS_HF_CACHE is True
    from flashcodec_b200.cache import FlashCodecCache, FlashCodecLayer
    assert issubclass(FlashCodecLayer, hf.DynamicLayer)
    assert issubclass(FlashCodecCache, hf.Cache)
    with pytest.raises(AttributeError):
        fc.NotAName  # noqa: B018


def test_from_config_plain_and_per_layer():
    cfg = tiny_llama().config
    cache = fc.FlashCodecCache.from_config(cfg, mode="jpeg", keep_freqs=8,
                                           per_layer={1: {"keep_freqs": 2, "quant_bits": 8}})
    assert cache.codec_layer_indices() == [0, 1]
    assert cache.layers[0].codec.keep_freqs == 8 and cache.layers[0].codec.quant_bits == 0
    assert cache.layers[1].codec.keep_freqs == 2 and cache.layers[1].codec.quant_bits == 8
    assert cache.codec_cfg["per_layer"] == {1: {"keep_freqs": 2, "quant_bits": 8}}
    assert cache.get_seq_length() == 0 and cache.storage_bytes() == 0


def test_from_config_hybrid_layer_types():
    cfg = LlamaConfig(vocab_size=64, hidden_size=32, num_hidden_layers=5,
                      num_attention_heads=2, num_key_value_heads=2)
    cfg.layer_types = ["full_attention", "sliding_attention", "linear_attention",
                       "full_attention", "chunked_attention"]
    cfg.sliding_window = 16
    cache = fc.FlashCodecCache.from_config(cfg, mode="png", block_size=16)
    kinds = [type(layer) for layer in cache.layers]
    assert kinds == [fc.FlashCodecLayer, hf.DynamicSlidingWindowLayer, hf.LinearAttentionLayer,
                     fc.FlashCodecLayer, hf.DynamicSlidingWindowLayer]
    assert cache.codec_layer_indices() == [0, 3]
    assert cache.layers[0].codec.block_size == 16


def test_from_config_sliding_window_everywhere():
    cfg = LlamaConfig(vocab_size=64, hidden_size=32, num_hidden_layers=3,
                      num_attention_heads=2, num_key_value_heads=2)
    cfg.sliding_window = 8
    cfg.layer_types = None
    cache = fc.FlashCodecCache.from_config(cfg)
    assert cache.codec_layer_indices() == []


def test_make_codec_errors_reach_the_cache():
    with pytest.raises(ValueError):
        fc.FlashCodecCache(mode="gif")
    with pytest.raises(ValueError):
        fc.FlashCodecLayer(mode="png", quant_bits=8)


def test_patch_bookkeeping_is_idempotent_and_reversible():
    m = tiny_llama()
    gen0, fwd0 = m.generate, m.forward
    assert fc.apply_codec_attention(m) == 2
    assert fc.apply_codec_attention(m) == 2            # idempotent
    assert fc.codec_attention_stats(m) == 2
    assert fc.remove_codec_attention(m) == 2
    assert fc.codec_attention_stats(m) == 0

    fc.apply_flash_codec(m, mode="jpeg", materialization_free=True)
    assert m._flashcodec["codec_attention_modules"] == 2
    assert len(m._flashcodec["attention_modules"]) == 2
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        fc.apply_flash_codec(m)                         # second apply warns, no-op
    assert any("already patched" in str(x.message) for x in w)
    fc.remove_flash_codec(m)
    assert m._flashcodec is None and fc.codec_attention_stats(m) == 0
    assert m.generate == gen0 and m.forward == fwd0
    fc.undo_flash_codec(m)                              # no-op once removed


def test_patched_attention_falls_back_for_other_caches():
    """With a non-codec cache the patched modules run the model's own
    forward: greedy tokens equal the unpatched model's (CPU, DynamicCache)."""
    ids = torch.randint(0, 128, (2, 10), generator=torch.Generator().manual_seed(1))
    ref = tiny_llama().generate(input_ids=ids, do_sample=False, pad_token_id=0,
                                max_new_tokens=6)
    m = tiny_llama()
    fc.apply_codec_attention(m)
    out = m.generate(input_ids=ids, do_sample=False, pad_token_id=0, max_new_tokens=6,
                     past_key_values=DynamicCache())
    assert torch.equal(out, ref)


def test_no_cpu_path_for_the_codec_cache():
    m = tiny_llama()
    fc.apply_flash_codec(m, mode="png")
    ids = torch.randint(0, 128, (1, 10))
    with pytest.raises(RuntimeError):
        m.generate(input_ids=ids, do_sample=False, pad_token_id=0, max_new_tokens=2)


def test_layer_structural_ops_before_any_data():
    layer = fc.FlashCodecLayer(mode="jpeg")
    assert layer.get_seq_length() == 0 and layer.get_max_cache_shape() == -1
    layer.crop(-3)
    layer.crop(5)
    layer.batch_repeat_interleave(2)
    layer.batch_select_indices(torch.tensor([0]))
    layer.reset()
    assert layer.storage_bytes() == 0 and layer.get_mask_sizes(1) == (1, 0)


def test_decode_mask_to_key_visibility():
    """The patched attention turns a decode step's (B, 1, 1, S+1) mask into
    per-key visibility: boolean masks as they are, additive masks where the
    bias is 0; other shapes keep the original forward (None)."""
    from flashcodec_b200.patch_attention import _key_visibility
    B, L = 3, 10
    vis = torch.ones(B, L, dtype=torch.bool)
    vis[1, :4] = False
    m_bool = vis[:, None, None, :]
    assert torch.equal(_key_visibility(m_bool, B, L), vis)
    m_add = torch.zeros(B, 1, 1, L).masked_fill(~vis[:, None, None, :],
                                                torch.finfo(torch.float32).min)
    assert torch.equal(_key_visibility(m_add, B, L), vis)
    assert torch.equal(_key_visibility(m_bool, B, L - 2), vis[:, :L - 2])
    assert _key_visibility(None, B, L) is None
    assert _key_visibility(m_bool, B, L + 1) is None             # shorter than the keys
    assert _key_visibility(m_bool[:2], B, L) is None             # batch mismatch
    assert _key_visibility(vis[:, None, :].expand(B, 2, L)[:, None], B, L) is None  # 2 queries
    assert _key_visibility(m_bool.int(), B, L) is None           # integer masks: unknown form
