"""GPU tests of the cache's append / archive / read cycle: the properties the
reference's tests/test_causal.py and tests/test_attention.py pin, checked on
the B200 implementation (bit-exact where the reference claims bitwise)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
B, H, S, D, R = 2, 4, 96, 32, 8


def _data(seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, H, S, D, generator=g).to(DEV),
            torch.randn(B, H, S, D, generator=g).to(DEV))


def toy_attn(q, k, v):
    Sq, Sk = q.shape[-2], k.shape[-2]
    logits = q @ k.transpose(-2, -1) / math.sqrt(D)
    mask = torch.ones(Sq, Sk, dtype=torch.bool, device=q.device).tril(diagonal=Sk - Sq)
    return torch.softmax(logits.masked_fill(~mask, float("-inf")), dim=-1) @ v


def _fill_incr(k, v, mode, **kw):
    import flashcodec_b200 as fc
    c = fc.CodecKVCache(mode=mode, **kw)
    for t in range(k.shape[-2]):
        c.decode_step(k[..., t:t + 1, :], v[..., t:t + 1, :])
    return c


def _archive(st):
    if st.codec.name == "jpeg":
        return [st._coeffs[:, :, :st.n_blocks].clone()]
    return [st._deltas[:, :, :st.n_blocks].clone(), st._anchors[:, :, :st.n_blocks].clone()]


def test_future_perturbation_never_rewrites_archive():
    import flashcodec_b200 as fc
    k, v = _data()
    c = fc.CodecKVCache(mode="png", block_size=R, keep_ratio=0.5)
    cut = 2 * R
    for t in range(cut):
        c.decode_step(k[..., t:t + 1, :], v[..., t:t + 1, :])
    snap = [_archive(st) for st in (c._keys[0], c._values[0])]
    before = c.key_cache[0].clone()
    pert = torch.randn_like(k[..., cut:, :])
    for t in range(S - cut):
        c.decode_step(pert[..., t:t + 1, :], pert[..., t:t + 1, :])
    for st, s0 in zip((c._keys[0], c._values[0]), snap):
        for a, a0 in zip(_archive(st), s0):
            assert torch.equal(a[:, :, :a0.shape[2]], a0)
    assert torch.equal(c.key_cache[0][..., :cut, :], before[..., :cut, :])


def test_incremental_equals_full_and_memoized_read():
    import flashcodec_b200 as fc
    k, v = _data(1)
    for mode, kw in (("png", dict(keep_ratio=1.0)), ("jpeg", dict(keep_freqs=2)),
                     ("jpeg", dict(keep_freqs=2, quant_bits=8))):
        full = fc.CodecKVCache(mode=mode, block_size=R, **kw)
        kf, vf = full.forward(k, v)
        kf, vf = kf.clone(), vf.clone()
        inc = _fill_incr(k, v, mode, block_size=R, **kw)
        # per-block arithmetic is identical however the blocks are batched:
        # bitwise for every mode (the reference allows 1e-6 for jpeg)
        assert torch.equal(inc.key_cache[0], kf) and torch.equal(inc.value_cache[0], vf)
        for t in (0, 13, 40, S - 1):
            fresh = fc.CodecKVCache(mode=mode, block_size=R, **kw)
            fk, _ = fresh.forward(k[..., :t + 1, :], v[..., :t + 1, :])
            assert torch.equal(kf[..., :t + 1 - (t + 1) % R, :], fk[..., :t + 1 - (t + 1) % R, :])


def test_png_incremental_attention_matches_full():
    import flashcodec_b200 as fc
    k, v = _data(2)
    q = torch.randn(B, H, S, D, device=DEV)
    c_full = fc.CodecKVCache(mode="png", block_size=R, keep_ratio=1.0)
    kf, vf = c_full.forward(k, v)
    out_full = toy_attn(q, kf, vf)
    c = fc.CodecKVCache(mode="png", block_size=R, keep_ratio=1.0)
    outs = []
    for t in range(S):
        kt, vt = c.decode_step(k[..., t:t + 1, :], v[..., t:t + 1, :])
        outs.append(toy_attn(q[..., t:t + 1, :], kt, vt))
    assert (out_full - torch.cat(outs, dim=-2)).abs().max().item() < 1e-4


def test_crop_exact_and_repeatable():
    k, v = _data(3)
    for mode, kw in (("png", dict(keep_ratio=1.0)), ("jpeg", dict(keep_freqs=2))):
        c = _fill_incr(k, v, mode, block_size=R, **kw)
        k_ref, v_ref = c.key_cache[0].clone(), c.value_cache[0].clone()
        c.crop(-5)
        assert c.get_seq_length(0) == S - 5
        assert torch.equal(c.key_cache[0], k_ref[..., :-5, :])
        assert torch.equal(c.value_cache[0], v_ref[..., :-5, :])
        c2 = _fill_incr(k, v, mode, block_size=R, **kw)
        c2.crop(-2)
        c2.crop(-3)
        assert torch.equal(c2.key_cache[0], k_ref[..., :-5, :])
        c3 = _fill_incr(k, v, mode, block_size=R, **kw)
        c3.crop(-S)
        assert c3.get_seq_length(0) == 0
        c4 = _fill_incr(k, v, mode, block_size=R, **kw)
        c4.crop(-(S - 3 * R))
        assert torch.equal(c4.key_cache[0], k_ref[..., :3 * R, :])
        with pytest.raises(ValueError):
            c4.crop(3)


def test_reorder_cache_permutes_archive():
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(4)
    kb = torch.randn(4, H, S + 3, D, generator=g).to(DEV)
    vb = torch.randn(4, H, S + 3, D, generator=g).to(DEV)
    idx = torch.tensor([2, 0, 3, 1])
    for mode, kw in (("png", dict(keep_ratio=1.0)), ("jpeg", dict(keep_freqs=2)),
                     ("jpeg", dict(keep_freqs=2, quant_bits=8))):
        c = fc.CodecKVCache(mode=mode, block_size=R, **kw)
        k_ref, v_ref = c.forward(kb, vb)
        k_ref, v_ref = k_ref.clone(), v_ref.clone()
        c.reorder_cache(idx)
        assert torch.equal(c.key_cache[0], k_ref.index_select(0, idx.to(DEV)))
        assert torch.equal(c.value_cache[0], v_ref.index_select(0, idx.to(DEV)))
        c.decode_step(kb[:, :, :1], vb[:, :, :1])
        assert c.get_seq_length(0) == S + 4
        # batch-size change (contrastive search style)
        c.reorder_cache(torch.tensor([0, 0, 1, 1, 2, 2]))
        assert c.key_cache[0].shape[0] == 6


def test_quantized_storage_and_stats():
    import flashcodec_b200 as fc
    k, v = _data(5)
    cq = fc.CodecKVCache(mode="jpeg", block_size=R, keep_freqs=2, quant_bits=8)
    cq.forward(k, v)
    plain = fc.CodecKVCache(mode="jpeg", block_size=R, keep_freqs=2)
    plain.forward(k, v)
    assert cq.storage_bytes(0) < 0.5 * plain.storage_bytes(0)
    # exact byte accounting: codes k*D + fp32 scales k*4 per block, K and V
    n = S // R
    assert cq.storage_bytes(0) == 2 * B * H * n * (2 * D + 2 * 4)
    st = cq.stats(0)
    assert st["tokens"] == S and st["archived"] == S and st["raw"] == 0
    assert st["raw_bytes"] == S * B * H * D * 4 * 2


def test_attention_never_materializes_and_leaves_stream():
    import flashcodec_b200 as fc
    k, v = _data(6)
    cfg = dict(mode="jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    ks, vs = fc._CodecStream(fc.make_codec(**cfg)), fc._CodecStream(fc.make_codec(**cfg))
    ks.append(k)
    vs.append(v)
    n0, l0 = ks.n_blocks, ks.seq_len
    arch = ks._coeffs[:, :, :n0].clone()
    out = fc.codec_decode_attention(torch.randn(B, H, 1, D, device=DEV), ks, vs)
    assert ks._rec is None and vs._rec is None
    assert ks.n_blocks == n0 and ks.seq_len == l0
    assert torch.equal(ks._coeffs[:, :, :n0], arch)
    assert torch.isfinite(out).all()


def test_attention_matches_materialized_view():
    """Coefficient-domain attention equals softmax attention over the read()
    view (reference tests/test_attention.py:43-53, 1e-5)."""
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(7)
    k = torch.cumsum(torch.randn(B, 4, S + 3, D, generator=g) * 0.1, dim=-2).to(DEV)
    v = torch.cumsum(torch.randn(B, 4, S + 3, D, generator=g) * 0.1, dim=-2).to(DEV)
    for gq in (1, 2):
        q = torch.randn(B, 4 * gq, 1, D, generator=g).to(DEV)
        for mode, kw in (("jpeg", dict(keep_freqs=2)), ("jpeg", dict(keep_freqs=8)),
                         ("jpeg", dict(keep_freqs=2, quant_bits=8)),
                         ("png", dict(keep_ratio=1.0)), ("png", dict(keep_ratio=0.5))):
            c = fc.CodecKVCache(mode=mode, block_size=8, **kw)
            c.forward(k, v)
            out = fc.codec_decode_attention(q, c._keys[0], c._values[0])
            kr = c.key_cache[0].repeat_interleave(gq, dim=1)
            vr = c.value_cache[0].repeat_interleave(gq, dim=1)
            p = torch.softmax(q @ kr.transpose(-2, -1) / math.sqrt(D), dim=-1)
            assert (out - p @ vr).abs().max().item() < 1e-5, (mode, kw, gq)


def test_streaming_decode_one_token_per_step():
    """Config-4 style: one bf16 token per step through capacity doublings;
    the streamed archive equals a one-shot archive bitwise and attention on
    the live stream matches the oracle along the way."""
    import flashcodec_b200 as fc
    import bench
    from test_gpu_attention import check_close, oracle_attention
    k, v, q = bench.synth_case(4, 16, 8, 8 * 40 + 5, 128, 0.95, 21, dtype=torch.bfloat16)
    k, v, q = k.to(DEV), v.to(DEV), q.to(DEV)
    c = fc.CodecKVCache(mode="jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    caps = set()
    for t in range(k.shape[2]):
        c.append(k[:, :, t:t + 1], v[:, :, t:t + 1])
        caps.add(c._keys[0]._capacity)
        if t in (7, 130, 255, k.shape[2] - 1):
            out = fc.codec_decode_attention(q, c._keys[0], c._values[0])
            check_close(out, oracle_attention(q.cpu(), c._keys[0], c._values[0]), torch.bfloat16)
    assert caps >= {16, 32, 64}
    one = fc.CodecKVCache(mode="jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    one.append(k, v)
    n = one._keys[0].n_blocks
    assert torch.equal(one._keys[0]._coeffs[:, :, :n], c._keys[0]._coeffs[:, :, :n])
    assert torch.equal(one._values[0]._scales[:, :, :n], c._values[0]._scales[:, :, :n])
    assert torch.equal(one._keys[0].raw, c._keys[0].raw)


def test_reorder_gathers_archive_bitwise_and_checks_indices():
    """select_batch (fc_gather_batch) moves every live prefix bit for bit,
    with repeated indices (beam search), and refuses indices outside the batch
    before touching anything."""
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(8)
    kb = torch.randn(3, H, S + 5, D, generator=g).to(torch.bfloat16).to(DEV)
    vb = torch.randn(3, H, S + 5, D, generator=g).to(torch.bfloat16).to(DEV)
    for mode, kw in (("jpeg", dict(keep_freqs=2, quant_bits=8)), ("png", dict(keep_ratio=1.0))):
        c = fc.CodecKVCache(mode=mode, block_size=R, **kw)
        c.append(kb, vb, 0)
        ks = c._keys[0]
        n = ks.n_blocks
        before = [t[:, :, :n].clone() for t in ks._archive_tensors()] + [ks.raw.clone()]
        idx = torch.tensor([2, 2, 0, 1])
        c.reorder_cache(idx)
        i = idx.to(DEV)
        after = [t[:, :, :n] for t in ks._archive_tensors()] + [ks.raw]
        for x, y in zip(before, after):
            assert torch.equal(y, x.index_select(0, i))
        with pytest.raises(IndexError):
            c.reorder_cache(torch.tensor([0, 7]))
        assert ks.raw.shape[0] == 4


def test_gather_batch_more_than_65535_slabs():
    """fc_gather_batch strides its grid over the (batch, head) slabs, so a
    beam batch with more than 65,535 of them (e.g. 256 sequences x 8 beams x
    32 KV heads) is reordered like any other."""
    from flashcodec_b200 import _kernels as K
    g = torch.Generator(device=DEV).manual_seed(9)
    src = torch.randint(-128, 127, (6, 20000, 3, 16), dtype=torch.int8, device=DEV, generator=g)
    idx = torch.tensor([5, 0, 0, 3], dtype=torch.int64, device=DEV)
    for live in (2, 3):            # 32-byte (vector) and 48-byte slabs
        dst = K.gather_batch(src, idx, live)
        assert dst.shape == (4, 20000, 3, 16)
        assert torch.equal(dst[:, :, :live], src.index_select(0, idx)[:, :, :live])
    odd = src[..., :5].contiguous()  # 5-byte rows: the byte-copy kernel
    dst = K.gather_batch(odd, idx, 3)
    assert torch.equal(dst, odd.index_select(0, idx))


@pytest.mark.parametrize("dt,D,kw", [
    (torch.bfloat16, 128, dict(keep_freqs=4, quant_bits=8)),
    (torch.float32, 64, dict(keep_freqs=2, quant_bits=8)),
    (torch.float16, 256, dict(keep_freqs=8, quant_bits=8, scale_dtype=torch.float16)),
    (torch.bfloat16, 128, dict(keep_freqs=2)),                  # unquantized coefficients
    (torch.float32, 36, dict(keep_freqs=3, quant_bits=8, block_size=16)),
])
def test_one_launch_append_equals_one_shot_archive(dt, D, kw):
    """fc_append_tokens (append_layers: K and V of every layer in one launch,
    block archive included) leaves every stream bit-identical to archiving
    the whole sequence at once, through capacity doublings."""
    import flashcodec_b200 as fc
    kw = dict(kw)
    r = kw.pop("block_size", 8)
    L, Bb, Hh, S = 3, 2, 4, r * 40 + 5
    g = torch.Generator(device=DEV).manual_seed(D)
    ks = [torch.randn(Bb, Hh, S, D, generator=g, device=DEV).cumsum(-2).to(dt) for _ in range(L)]
    vs = [torch.randn(Bb, Hh, S, D, generator=g, device=DEV).to(dt) for _ in range(L)]
    c = fc.CodecKVCache("jpeg", block_size=r, **kw)
    c.append_layers([k[:, :, :1] for k in ks], [v[:, :, :1] for v in vs])
    for t in range(1, S):
        c.append_layers([k[:, :, t:t + 1] for k in ks], [v[:, :, t:t + 1] for v in vs])
    one = fc.CodecKVCache("jpeg", block_size=r, **kw)
    for i in range(L):
        one.append(ks[i], vs[i], i)
    for i in range(L):
        for a, b in ((c._keys[i], one._keys[i]), (c._values[i], one._values[i])):
            n = b.n_blocks
            assert a.n_blocks == n and a.n_archived == b.n_archived and a.seq_len == S
            for x, y in zip(a._archive_tensors(), b._archive_tensors()):
                assert torch.equal(x[:, :, :n], y[:, :, :n])
            assert torch.equal(a.raw, b.raw)
            assert a.scale_range_errors() == b.scale_range_errors()
        assert torch.equal(c._keys[i].read(), one._keys[i].read())


def test_one_launch_append_falls_back_when_layouts_differ():
    """Streams at different raw positions cannot share a launch: append_layers
    appends layer by layer and the result is unchanged."""
    import flashcodec_b200 as fc
    g = torch.Generator(device=DEV).manual_seed(2)
    k = torch.randn(2, 4, 43, 64, generator=g, device=DEV).to(torch.bfloat16)
    c = fc.CodecKVCache("jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    c.append(k[:, :, :5], k[:, :, :5], 0)
    c.append(k[:, :, :3], k[:, :, :3], 1)           # layer 1 three tokens behind
    for t in range(5, 40):
        c.append_layers([k[:, :, t:t + 1], k[:, :, t - 2:t - 1]],
                        [k[:, :, t:t + 1], k[:, :, t - 2:t - 1]])
    one = fc.CodecKVCache("jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    one.append(k[:, :, :40], k[:, :, :40], 0)
    one.append(k[:, :, :38], k[:, :, :38], 1)
    for i in (0, 1):
        assert torch.equal(c._keys[i].read(), one._keys[i].read())
        n = one._keys[i].n_blocks
        assert torch.equal(c._keys[i]._coeffs[:, :, :n], one._keys[i]._coeffs[:, :, :n])
