"""GPU parity of the codec kernels (archive, read path, png) against the
reference's own outputs (golden fixtures) and the CPU oracle.  Bit-exact."""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import cases  # noqa: E402
from cases import f32  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def same(a, b):
    return np.array_equal(bits(np.asarray(a)), bits(np.asarray(b)))


@pytest.mark.parametrize("i", range(len(cases.JPEG_CASES)))
def test_jpeg_codec_matches_reference(golden, i):
    import flashcodec_b200 as fc
    data, meta = golden
    name, dt, B, H, S, D, r, k, qb = cases.JPEG_CASES[i]
    x = cases.jpeg_input(i).to(DEV)
    assert same(fc.dct_basis(r, r).numpy(), data[f"basis_r{r}"])
    coef = fc.dct_compress(x, r, k)
    assert coef.dtype == x.dtype
    assert same(f32(coef), data[f"{name}/coef"])
    assert same(f32(fc.dct_decompress(coef, r, S)), data[f"{name}/rec_coef"])
    if qb:
        q, s = fc.quantize_coeffs(coef)
        assert q.dtype == torch.int8 and s.dtype == torch.float32
        assert same(q.cpu().numpy(), data[f"{name}/codes"])
        assert same(f32(s), data[f"{name}/scales"])
        c = fc.make_codec("jpeg", block_size=r, keep_freqs=k, quant_bits=8)
        assert same(f32(c.decompress(q, out_len=S, scales=s)), data[f"{name}/rec_q"])
    # the cache path: fused archive kernel writing in place, memoized read
    st = fc._CodecStream(fc.make_codec("jpeg", block_size=r, keep_freqs=k, quant_bits=qb))
    st.append(x)
    n = st.n_blocks
    assert n == meta[name]["n_blocks"] and st._capacity == meta[name]["capacity"]
    if qb:
        assert same(st._coeffs[:, :, :n].cpu().numpy(), data[f"{name}/st_coeffs"])
        assert same(f32(st._scales[:, :, :n]), data[f"{name}/st_scales"])
    else:
        assert same(f32(st._coeffs[:, :, :n]), data[f"{name}/st_coeffs"])
    view = st.read()
    assert view.dtype == x.dtype
    assert same(f32(view), data[f"{name}/st_read"])
    assert st.storage_bytes() == meta[name]["storage_bytes"]


@pytest.mark.parametrize("i", range(len(cases.PNG_CASES)))
def test_png_codec_matches_reference(golden, i):
    import flashcodec_b200 as fc
    data, _ = golden
    name, dt, B, H, S, D, r, keep = cases.PNG_CASES[i]
    x = cases.png_input(i).to(DEV)
    d, a = fc.png_filter(x, r, keep)
    assert d.dtype == torch.float32 and a.dtype == x.dtype
    assert same(f32(d), data[f"{name}/deltas"])      # including -0.0 of pruned steps
    assert same(f32(a), data[f"{name}/anchors"])
    rec = fc.png_reconstruct(d, a)
    assert rec.dtype == x.dtype
    assert same(f32(rec), data[f"{name}/rec"])
    if keep == 1.0 and dt == "bf16":
        assert torch.equal(rec[..., :S, :], x)           # bf16: lossless bitwise (png.py:46-47)
    elif keep == 1.0:
        # fp32: rounding of the prefix sums only (reference test_png.py:26-29
        # bounds it by 1e-6 on unit-scale data; scaled to the data here)
        assert (rec[..., :S, :] - x).abs().max().item() <= 1e-6 * x.abs().max().item()


@pytest.mark.parametrize("shape,r,k,dt", [
    ((3, 5, 1000, 96), 8, 3, torch.float32),
    ((2, 3, 777, 128), 16, 5, torch.bfloat16),
    ((1, 2, 64, 20), 8, 2, torch.float16),
    ((4, 1000, 40), 8, 8, torch.float32),
])
def test_jpeg_odd_shapes_match_oracle(shape, r, k, dt):
    """Shapes off the vectorised paths (D % 4 != 0, leading dims != 4) and
    partial last blocks, against the oracle with the same basis."""
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(7)
    x = torch.cumsum(torch.randn(*shape, generator=g) * 0.3, dim=-2).to(dt)
    basis = fc.dct_basis(r, k).numpy()
    tag = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[dt]
    coef = fc.dct_compress(x.to(DEV), r, k)
    ref = orc.jpeg_encode(f32(x), r, k, basis, tag)
    assert same(f32(coef), ref)
    q, s = fc.quantize_coeffs(coef)
    rq, rs = orc.jpeg_quantize(ref, tag)
    assert same(q.cpu().numpy(), rq) and same(f32(s), rs)
    rec = fc.dct_decompress(coef, r, shape[-2])
    assert same(f32(rec), orc.jpeg_decode(ref, None, basis, r, "f32", out_len=shape[-2]))


@pytest.mark.parametrize("shape,r,k,dt,q8", [
    ((2, 3, 256, 128), 8, 4, torch.bfloat16, True),     # d128 archive, KM = 4
    ((2, 3, 256, 128), 8, 8, torch.float32, True),      # KM = 8
    ((1, 2, 517, 128), 16, 4, torch.float16, True),     # r = 16, partial last block
    ((1, 2, 256, 128), 16, 8, torch.bfloat16, True),
    ((2, 2, 203, 128), 8, 2, torch.float32, False),     # unquantized coefficients, padding
    ((2, 2, 256, 128), 16, 3, torch.bfloat16, False),
])
def test_jpeg_fast_paths_match_oracle(shape, r, k, dt, q8):
    """The head-dim-128 fast paths of the archive and read kernels against the
    oracle, and against the general kernels (the same input at an address
    off the vector alignment takes them), bit for bit."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    g = torch.Generator().manual_seed(11)
    x = (torch.cumsum(torch.randn(*shape, generator=g) * 0.3, dim=-2) *
         torch.exp(0.5 * torch.randn(1, shape[1], 1, shape[-1], generator=g))).to(dt)
    tag = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[dt]
    basis = fc.dct_basis(r, k)
    ref = orc.jpeg_encode(f32(x), r, k, basis.numpy(), tag)
    B, H, S, D = shape
    n = (S + r - 1) // r
    xd = x.to(DEV)
    # the same values one element past a vector boundary: the general kernel
    buf = torch.empty(xd.numel() + 1, dtype=dt, device=DEV)
    xs = buf[1:].view(shape)
    xs.copy_(xd)
    bd = basis.to(DEV).contiguous()
    for src in (xd, xs):
        if q8:
            codes = torch.empty(B, H, n, k, D, dtype=torch.int8, device=DEV)
            scales = torch.empty(B, H, n, k, 1, dtype=torch.float32, device=DEV)
            K.jpeg_encode(src, bd, r, k, codes, scales)
            rq, rs = orc.jpeg_quantize(ref, tag)
            assert same(codes.cpu().numpy(), rq) and same(f32(scales), rs)
            for odt in (torch.float32, torch.bfloat16, torch.float16):
                rec = torch.empty(B, H, S, D, dtype=odt, device=DEV)
                K.jpeg_decode(codes, scales, bd, r, rec, S)
                otag = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[odt]
                want = orc.jpeg_decode(rq, rs, basis.numpy(), r, otag, out_len=S)
                assert same(f32(rec), want), odt
        else:
            coef = torch.empty(B, H, n, k, D, dtype=dt, device=DEV)
            K.jpeg_encode(src, bd, r, k, coef)
            assert same(f32(coef), ref)
            rec = torch.empty(B, H, S, D, dtype=dt, device=DEV)
            K.jpeg_decode(coef, None, bd, r, rec, S)
            assert same(f32(rec), orc.jpeg_decode(ref, None, basis.numpy(), r, tag, out_len=S))


def test_png_fast_paths_match_oracle():
    """png filter/reconstruct fast paths (keep 1.0, r in {8, 16}, 4-aligned
    rows) against the oracle for fp32, bf16 and fp16, with a partial block."""
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(5)
    for dt, r in ((torch.float32, 16), (torch.bfloat16, 8), (torch.float16, 16)):
        x = torch.cumsum(torch.randn(2, 3, 203, 128, generator=g), dim=-2).to(dt)
        tag = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[dt]
        d, a = fc.png_filter(x.to(DEV), r, 1.0)
        rd, ra = orc.png_encode(f32(x), r, 1.0)
        assert same(f32(d), rd) and same(f32(a), ra)
        assert same(f32(fc.png_reconstruct(d, a)), orc.png_decode(rd, ra, tag))


def test_png_topm_and_odd_shapes_match_oracle():
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(3)
    for shape, r, keep in (((2, 3, 203, 50), 8, 0.5), ((1, 4, 64, 128), 16, 0.3),
                           ((2, 2, 96, 64), 32, 1.0)):
        x = torch.cumsum(torch.randn(*shape, generator=g), dim=-2)
        d, a = fc.png_filter(x.to(DEV), r, keep)
        rd, ra = orc.png_encode(f32(x), r, keep)
        assert same(f32(d), rd) and same(f32(a), ra)
        assert same(f32(fc.png_reconstruct(d, a)), orc.png_decode(rd, ra))


def test_cfg1_archive_digests(golden):
    """Config 1 (B=1 Hkv=8 S=4096 D=128 fp32 r=8 K=2 int8) archived on the GPU:
    SHA-256 of codes and scales equal the reference's."""
    import flashcodec_b200 as fc
    _, meta = golden
    c = meta["cfg1"]
    k, v, q = cases.cfg1_input()
    for t in (0, 1):
        dg = c["digests"][f"t{t}"]
        for nm, x in (("k", k), ("v", v)):
            st = fc._CodecStream(fc.make_codec("jpeg", block_size=8, keep_freqs=2, quant_bits=8))
            st.append(x[:, :, :c["S"] + t].to(DEV))
            n = st.n_blocks
            assert n == dg["n_blocks"]
            assert cases.sha(st._coeffs[:, :, :n].cpu().numpy()) == dg[f"{nm}_codes"]
            assert cases.sha(f32(st._scales[:, :, :n])) == dg[f"{nm}_scales"]


def test_autograd_through_codecs():
    """Gradients flow like the reference's (test_jpeg/test_png autograd tests)."""
    import flashcodec_b200 as fc
    xr = torch.randn(2, 4, 64, 32, device=DEV, requires_grad=True)
    rec = fc.dct_decompress(fc.dct_compress(xr, 8, 2), 8, out_len=64)
    rec.pow(2).mean().backward()
    assert xr.grad is not None and torch.isfinite(xr.grad).all()
    # adjoint check against autograd of an explicit torch formulation
    M = fc.dct_basis(8, 2).to(DEV)
    xd = xr.detach().clone().requires_grad_(True)
    hp = torch.matmul(xd.reshape(2, 4, 8, 8, 32).transpose(-2, -1), M.t())
    rec2 = torch.matmul(hp, M).transpose(-2, -1).reshape(2, 4, 64, 32)
    rec2.pow(2).mean().backward()
    torch.testing.assert_close(xr.grad, xd.grad, rtol=1e-5, atol=1e-7)
    xp = torch.randn(2, 4, 64, 32, device=DEV, requires_grad=True)
    d, a = fc.png_filter(xp, 8, 0.5)
    rec = fc.png_reconstruct(d, a)[..., :64, :]
    rec.pow(2).mean().backward()
    assert xp.grad is not None and torch.isfinite(xp.grad).all()


def test_fp16_scales_exact_for_bf16_inputs():
    """fp16 scales (config 5 format) hold bf16-valued scales exactly inside the
    fp16 range: codes equal the fp32-scale archive and no range error."""
    import flashcodec_b200 as fc
    x = torch.randn(2, 4, 256, 128, device=DEV).to(torch.bfloat16)
    a = fc._CodecStream(fc.make_codec("jpeg", block_size=8, keep_freqs=2, quant_bits=8))
    h = fc._CodecStream(fc.make_codec("jpeg", block_size=8, keep_freqs=2, quant_bits=8,
                                      scale_dtype=torch.float16))
    a.append(x)
    h.append(x)
    n = a.n_blocks
    assert torch.equal(a._coeffs[:, :, :n], h._coeffs[:, :, :n])
    assert torch.equal(a._scales[:, :, :n], h._scales[:, :, :n].float())
    assert not h.scale_range_errors()
    tiny = fc._CodecStream(fc.make_codec("jpeg", block_size=8, keep_freqs=2, quant_bits=8,
                                         scale_dtype=torch.float16))
    tiny.append(torch.full((1, 1, 8, 128), 1e-9, device=DEV))   # scale below fp16 range
    assert tiny.scale_range_errors()


def test_low_level_wrappers_refuse_strided_last_dim():
    """The kernels take unit stride along the head dim; a view with another
    stride is refused instead of being read wrongly."""
    from flashcodec_b200 import _kernels as K
    import flashcodec_b200 as fc
    wide = torch.zeros(1, 2, 64, 256, device=DEV)
    xs = wide[..., ::2]
    codes = torch.empty(1, 2, 8, 2, 128, dtype=torch.int8, device=DEV)
    scales = torch.empty(1, 2, 8, 2, 1, device=DEV)
    with pytest.raises(ValueError):
        K.jpeg_encode(xs, fc.dct_basis(8, 2).to(DEV), 8, 2, codes, scales)
    with pytest.raises(ValueError):
        K.png_encode(xs, 8, 7, torch.empty(1, 2, 8, 7, 128, device=DEV),
                     torch.empty(1, 2, 8, 128, device=DEV))
