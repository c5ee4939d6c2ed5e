"""transformers 5.x integration on the GPU: the reference's
tests/test_hf_integration.py cases (explicit cache, hot patch, png lossless
generation, long runs, beam search, crop, int8, per-layer budgets,
materialization-free decode) on a tiny offline Llama on cuda, plus the batch>1
decode path the reference guards off (flashcodec/patch_attention.py:54)."""

import warnings

import pytest
import torch

pytest.importorskip("transformers")
from transformers import LlamaConfig, LlamaForCausalLM  # noqa: E402

import flashcodec_b200 as fc  # noqa: E402
import flashcodec_b200.attention as fc_attention  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
VOCAB, PROMPT_LEN, NEW = 128, 12, 20


def tiny_llama(seed=7, hidden=32, heads=2, kv_heads=2, dtype=torch.float32):
    """2 layers; lm_head scaled x20 so greedy choices have a clear margin."""
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=VOCAB, hidden_size=hidden, intermediate_size=2 * hidden,
                      num_hidden_layers=2, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, max_position_embeddings=512)
    m = LlamaForCausalLM(cfg).eval()
    m.generation_config.eos_token_id = None
    with torch.no_grad():
        m.lm_head.weight.mul_(20.0)
    return m.to(device=DEV, dtype=dtype)


def prompt(batch=1, seed=42):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, VOCAB, (batch, PROMPT_LEN), generator=g).to(DEV)


def gen(model, ids=None, **kw):
    kw.setdefault("max_new_tokens", NEW)
    with torch.no_grad():
        return model.generate(input_ids=prompt() if ids is None else ids, do_sample=False,
                              pad_token_id=0, **kw)


@pytest.fixture
def count_decode(monkeypatch):
    """Counts calls of the coefficient-domain attention (the decode path)."""
    calls = []
    real = fc_attention.codec_decode_attention

    def wrapped(q, *a, **kw):
        calls.append(q.shape[0])
        return real(q, *a, **kw)

    monkeypatch.setattr(fc_attention, "codec_decode_attention", wrapped)
    return calls


def test_a_explicit_cache():
    model = tiny_llama()
    cache = fc.FlashCodecCache(mode="jpeg", block_size=8, keep_freqs=2)
    with warnings.catch_warnings():
        warnings.simplefilter("error", UserWarning)
        out = gen(model, past_key_values=cache)
    assert out.shape == (1, PROMPT_LEN + NEW)
    assert cache.get_seq_length() == PROMPT_LEN + NEW - 1
    assert cache._seen_tokens == PROMPT_LEN + NEW - 1
    assert len(cache.layers) == model.config.num_hidden_layers
    # raw fp32 K+V of every layer: tokens x batch 1 x (2 layers x 2 heads x 16 dims) x 4 B x 2
    raw = (PROMPT_LEN + NEW) * 1 * 2 * 32 * 4 * 2
    assert cache.storage_bytes() < 0.5 * raw


def test_b_hotpatch_and_remove():
    model = tiny_llama()
    assert len(fc.find_attention_modules(model)) == model.config.num_hidden_layers
    fc.apply_flash_codec(model, mode="jpeg", block_size=8, keep_freqs=2)
    out = gen(model)
    assert out.shape == (1, PROMPT_LEN + NEW)
    caches = model._flashcodec["caches"]
    assert len(caches) == 1 and isinstance(caches[0], fc.FlashCodecCache)
    assert caches[0].get_seq_length() == PROMPT_LEN + NEW - 1
    fc.remove_flash_codec(model)
    assert model._flashcodec is None
    assert gen(model).shape == (1, PROMPT_LEN + NEW)


def test_c_png_lossless_generation_matches_unpatched():
    model = tiny_llama()
    ref = gen(model)
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0)
    assert torch.equal(gen(model), ref)


@pytest.mark.parametrize("mode,kw,bound", [("jpeg", dict(keep_freqs=2), 0.35),
                                           ("png", dict(keep_ratio=1.0), 1.05)])
def test_d_long_generation(mode, kw, bound):
    model = tiny_llama()
    cache = fc.FlashCodecCache(mode=mode, block_size=8, **kw)
    with warnings.catch_warnings():
        warnings.simplefilter("error", UserWarning)
        out = gen(model, past_key_values=cache, max_new_tokens=70)
    kv_len = PROMPT_LEN + 70 - 1
    assert out.shape == (1, PROMPT_LEN + 70)
    assert cache.get_seq_length() == kv_len
    ks = cache.layers[0]._key_stream
    assert ks.n_archived > 0 and kv_len - ks.n_archived < 8
    raw = kv_len * 1 * 2 * 32 * 4 * 2          # both layers, as in test_a
    assert cache.storage_bytes() < bound * raw


def test_e_beam_search_png_matches_unpatched():
    model = tiny_llama()
    ref = gen(model, num_beams=3)
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0)
    assert torch.equal(gen(model, num_beams=3), ref)


def test_f_crop_keeps_prefix_and_matches_unpatched():
    model, ref_model = tiny_llama(), tiny_llama()
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0)
    cache = fc.FlashCodecCache(mode="png", block_size=8, keep_ratio=1.0)
    out = gen(model, past_key_values=cache)
    total = out.shape[1]
    assert cache.get_seq_length() == total - 1
    before = [layer.keys.clone() for layer in cache.layers]
    cache.crop(-5)
    assert cache.get_seq_length() == total - 6
    for li, layer in enumerate(cache.layers):
        assert torch.equal(layer.keys, before[li][..., :total - 6, :])
    with torch.no_grad():
        ours = model(input_ids=out[:, total - 6:total - 5], past_key_values=cache,
                     use_cache=True).logits[:, -1]
        ref = ref_model(input_ids=out[:, :total - 5]).logits[:, -1]
    assert torch.equal(ours.argmax(-1), ref.argmax(-1))
    assert (ours - ref).abs().max().item() < 1e-2


def test_f2_crop_to_length_transformers_convention():
    """A non-negative crop keeps that many tokens (assisted generation)."""
    model = tiny_llama()
    cache = fc.FlashCodecCache(mode="png", block_size=8, keep_ratio=1.0)
    gen(model, past_key_values=cache)
    n = cache.get_seq_length()
    keys = [layer.keys.clone() for layer in cache.layers]
    cache.crop(n + 3)                      # longer than the cache: no change
    assert cache.get_seq_length() == n
    cache.crop(17)
    assert cache.get_seq_length() == 17
    for li, layer in enumerate(cache.layers):
        assert torch.equal(layer.keys, keys[li][..., :17, :])
        assert layer._key_stream.n_archived == 16


def test_g_int8_generation_shrinks_archive():
    plain = fc.FlashCodecCache(mode="jpeg", block_size=8, keep_freqs=2)
    gen(tiny_llama(), past_key_values=plain)
    cache = fc.FlashCodecCache(mode="jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    out = gen(tiny_llama(), past_key_values=cache)
    assert out.shape == (1, PROMPT_LEN + NEW)
    assert cache.get_seq_length() == PROMPT_LEN + NEW - 1
    assert cache.storage_bytes() < 0.7 * plain.storage_bytes()


def test_h_per_layer_schedule():
    model = tiny_llama()
    cache = fc.FlashCodecCache.from_config(model.config, mode="jpeg", block_size=8,
                                           keep_freqs=8,
                                           per_layer={1: dict(keep_freqs=2, quant_bits=8)})
    assert cache.codec_layer_indices() == [0, 1]
    assert (cache.layers[0].codec.keep_freqs, cache.layers[0].codec.quant_bits) == (8, 0)
    assert (cache.layers[1].codec.keep_freqs, cache.layers[1].codec.quant_bits) == (2, 8)
    out = gen(model, past_key_values=cache)
    assert out.shape == (1, PROMPT_LEN + NEW)
    assert cache.get_seq_length() == PROMPT_LEN + NEW - 1


def test_i_materialization_free_generation(count_decode):
    ref = gen(tiny_llama())
    model = tiny_llama()
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0,
                         materialization_free=True)
    n_layers = model.config.num_hidden_layers
    assert model._flashcodec["codec_attention_modules"] == n_layers
    assert fc.codec_attention_stats(model) == n_layers
    assert torch.equal(gen(model), ref)
    assert len(count_decode) == n_layers * (NEW - 1)
    # the model's rotary function was checked once and the fused
    # rotary + append kernel took over the later decode steps
    from transformers.models.llama import modeling_llama

    from flashcodec_b200 import patch_attention
    assert patch_attention._ROPE_EXACT[(modeling_llama.apply_rotary_pos_emb,
                                        torch.float32)] is True
    cache = model._flashcodec["caches"][-1]
    assert cache.get_seq_length() == PROMPT_LEN + NEW - 1
    for layer in cache.layers:
        assert layer._key_stream._rec is None
    fc.remove_flash_codec(model)
    assert fc.codec_attention_stats(model) == 0
    assert gen(model).shape == ref.shape


# ------------------------------------------------ batch > 1 decode path
def test_batched_decode_runs_on_archive_and_matches_unpatched(count_decode):
    """Equal-length prompts (no padding mask): every decode step of a batch of
    3 goes through the archive kernels; png keeps tokens identical."""
    ids = prompt(batch=3, seed=5)
    ref = gen(tiny_llama(), ids)
    model = tiny_llama()
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0,
                         materialization_free=True)
    out = gen(model, ids)
    assert torch.equal(out, ref)
    assert count_decode and set(count_decode) == {3}
    assert len(count_decode) == 2 * (NEW - 1)


def test_beam_search_on_archive_stays_view_free(count_decode):
    """Beam search reorders the archive between decode steps; the layers stay
    view-free and the tokens match the unpatched model (png)."""
    ref = gen(tiny_llama(), num_beams=3)
    model = tiny_llama()
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0,
                         materialization_free=True)
    out = gen(model, num_beams=3)
    assert torch.equal(out, ref)
    assert count_decode and set(count_decode) == {3}
    for layer in model._flashcodec["caches"][-1].layers:
        assert layer._key_stream._rec is None and layer.keys is None


def test_padded_batch_decodes_on_the_archive(count_decode):
    """A left-padded batch carries an attention mask; decode steps run on the
    archive with that mask as key visibility (fc_decode_attn_masked), and png
    generation equals the unpatched model's."""
    ids = prompt(batch=2, seed=9)
    mask = torch.ones_like(ids)
    mask[1, :3] = 0
    base = tiny_llama()
    with torch.no_grad():
        ref = base.generate(input_ids=ids, attention_mask=mask, do_sample=False,
                            pad_token_id=0, max_new_tokens=NEW)
    model = tiny_llama()
    fc.apply_flash_codec(model, mode="png", block_size=8, keep_ratio=1.0,
                         materialization_free=True)
    with torch.no_grad():
        out = model.generate(input_ids=ids, attention_mask=mask, do_sample=False,
                             pad_token_id=0, max_new_tokens=NEW)
    assert torch.equal(out, ref)
    assert len(count_decode) == 2 * (NEW - 1) and set(count_decode) == {2}


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 3e-2)])
def test_decode_step_logits_match_materialized_view(dtype, tol):
    """jpeg int8 at head_dim 128 with GQA (G=2), batch 4: one decode step on
    the archive gives the logits of the same step over the reconstructed
    view, from the same prefill (same archive)."""
    ids = prompt(batch=4, seed=3)
    ids = torch.cat([ids, ids[:, :5], ids], dim=1)      # 29 tokens: 3 blocks + 5 raw
    nxt = ids[:, -1:]
    cfg = dict(hidden=256, heads=2, kv_heads=1, dtype=dtype)
    view_model, free_model = tiny_llama(**cfg), tiny_llama(**cfg)
    fc.apply_codec_attention(free_model)
    kw = dict(mode="jpeg", block_size=8, keep_freqs=4, quant_bits=8)
    c_view, c_free = fc.FlashCodecCache(**kw), fc.FlashCodecCache(**kw)
    with torch.no_grad():
        view_model(input_ids=ids, past_key_values=c_view, use_cache=True)
        free_model(input_ids=ids, past_key_values=c_free, use_cache=True)
        a = view_model(input_ids=nxt, past_key_values=c_view, use_cache=True).logits[:, -1]
        b = free_model(input_ids=nxt, past_key_values=c_free, use_cache=True).logits[:, -1]
    assert c_free.layers[0].keys is None
    for lv, lf in zip(c_view.layers, c_free.layers):
        assert torch.equal(lv._key_stream._coeffs[:, :, :3], lf._key_stream._coeffs[:, :, :3])
    err = ((a.float() - b.float()).abs().max() / a.float().abs().max()).item()
    assert err < tol, err


def test_per32_decode_step_logits_match_materialized_view():
    """The per-32 coefficient format (group_size=32) through the model: a
    decode step on the archive (fc_decode_attn_grouped) gives the logits of
    the same step over the reconstructed view (fc_jpeg_decode_grouped), from
    the same archive."""
    ids = prompt(batch=2, seed=4)
    ids = torch.cat([ids, ids[:, :5], ids], dim=1)
    nxt = ids[:, -1:]
    cfg = dict(hidden=256, heads=2, kv_heads=1, dtype=torch.float32)
    view_model, free_model = tiny_llama(**cfg), tiny_llama(**cfg)
    fc.apply_codec_attention(free_model)
    kw = dict(mode="jpeg", block_size=8, keep_freqs=4, quant_bits=8, group_size=32)
    c_view, c_free = fc.FlashCodecCache(**kw), fc.FlashCodecCache(**kw)
    with torch.no_grad():
        view_model(input_ids=ids, past_key_values=c_view, use_cache=True)
        free_model(input_ids=ids, past_key_values=c_free, use_cache=True)
        a = view_model(input_ids=nxt, past_key_values=c_view, use_cache=True).logits[:, -1]
        b = free_model(input_ids=nxt, past_key_values=c_free, use_cache=True).logits[:, -1]
    ks = c_free.layers[0]._key_stream
    assert ks._scales.shape[-1] == 128 // 32 and ks.codec.group_size == 32
    err = ((a - b).abs().max() / a.abs().max()).item()
    assert err < 1e-4, err
