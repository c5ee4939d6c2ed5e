"""fc_decode_attn_masked: decode attention with a per-key visibility mask
(left-padded batches), against an fp32 softmax over the reconstructed view
with the same mask.  Covers masks that empty whole sequence splits, scattered
masks, a row with no visible key (zero output), and the png and int8
archives."""

import pytest
import torch

import flashcodec_b200 as fc
from flashcodec_b200 import _kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _streams(mode, kw, B, Hk, S, D, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.randn(B, Hk, S, D, generator=g, device=DEV).to(dtype)
    v = torch.randn(B, Hk, S, D, generator=g, device=DEV).to(dtype)
    c = fc.make_codec(mode, block_size=8, **kw)
    ks, vs = fc._CodecStream(c), fc._CodecStream(c)
    ks.append(k)
    vs.append(v)
    return ks, vs


def _masked_ref(q, kview, vview, vis, scale):
    """fp32 softmax over the reconstructed K/V with masked keys removed."""
    B, Hq, _, D = q.shape
    Hk = kview.shape[1]
    G = Hq // Hk
    kf = kview.float().repeat_interleave(G, dim=1)
    vf = vview.float().repeat_interleave(G, dim=1)
    lg = (q.float() @ kf.transpose(-2, -1)) * scale               # (B,Hq,1,S)
    lg = lg.masked_fill(~vis.bool()[:, None, None, :], float("-inf"))
    p = torch.softmax(lg, dim=-1).nan_to_num(0.0)
    return p @ vf


CASES = [("jpeg", dict(keep_freqs=4, quant_bits=8), torch.bfloat16, 1e-2),
         ("jpeg", dict(keep_freqs=2), torch.float32, 1e-5),
         ("png", dict(keep_ratio=1.0), torch.float32, 1e-5)]


@pytest.mark.parametrize("mode,kw,dtype,tol", CASES)
def test_left_padding_and_scattered_masks(mode, kw, dtype, tol):
    B, Hq, Hk, S, D = 4, 8, 2, 4096 + 5, 128
    ks, vs = _streams(mode, kw, B, Hk, S, D, dtype, 1)
    g = torch.Generator(device=DEV).manual_seed(2)
    q = torch.randn(B, Hq, 1, D, generator=g, device=DEV).to(dtype)
    pos = torch.arange(S, device=DEV)
    pad = torch.tensor([0, 7, 1500, 4000], device=DEV)           # whole splits masked
    vis = pos[None, :] >= pad[:, None]
    vis[1] &= torch.rand(S, generator=g, device=DEV) > 0.3         # scattered holes too
    scale = D ** -0.5
    out = fc.codec_decode_attention(q, ks, vs, scale=scale, visible=vis)
    ref = _masked_ref(q, ks.read(), vs.read(), vis, scale)
    err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < tol, err
    # a full mask gives the unmasked result (the CUDA-core kernel either way)
    full = torch.ones(B, S, dtype=torch.bool, device=DEV)
    a = fc.codec_decode_attention(q, ks, vs, scale=scale, visible=full)
    prev = K.set_attn_kernel("cuda-core")
    try:
        b = fc.codec_decode_attention(q, ks, vs, scale=scale)
    finally:
        K.set_attn_kernel(prev)
    assert torch.equal(a, b)


def test_row_without_visible_keys_is_zero():
    ks, vs = _streams("jpeg", dict(keep_freqs=2, quant_bits=8), 2, 2, 1000, 64,
                      torch.float32, 3)
    q = torch.randn(2, 4, 1, 64, device=DEV)
    vis = torch.ones(2, 1000, dtype=torch.uint8, device=DEV)
    vis[0] = 0
    out = fc.codec_decode_attention(q, ks, vs, visible=vis)
    assert torch.count_nonzero(out[0]) == 0
    ref = _masked_ref(q, ks.read(), vs.read(), vis, 64 ** -0.5)
    assert ((out[1] - ref[1]).abs().max() / ref[1].abs().max()).item() < 1e-5


def test_visibility_shape_is_checked():
    ks, vs = _streams("jpeg", dict(keep_freqs=2), 2, 2, 64, 32, torch.float32, 4)
    q = torch.randn(2, 2, 1, 32, device=DEV)
    with pytest.raises(ValueError):
        fc.codec_decode_attention(q, ks, vs, visible=torch.ones(2, 10, dtype=torch.bool,
                                                                device=DEV))
    with pytest.raises(ValueError):
        fc.codec_decode_attention(q, ks, vs, visible=torch.ones(2, 64, device=DEV))
