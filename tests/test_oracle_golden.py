"""Pin the CPU oracle (oracle/) against fixtures produced by the reference.

Every comparison here is bit-exact unless a tolerance is written next to it.
The oracle is then trusted as the checker for the CUDA kernels (tests marked
gpu).  CPU only.
"""

import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import cases  # noqa: E402
from cases import f32, sha  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def _basis(golden, r):
    data, _ = golden
    return data[f"basis_r{r}"]


def _text(arr):
    return bytes(arr).decode()


def test_basis_fp64_close_to_reference(golden):
    """The exact (fp64-rounded) DCT basis is within 4e-6 of the reference's
    torch basis but not bit-identical (torch evaluates the cosine argument in
    fp32), which is why bit-exact parity uses the stored reference basis."""
    for r in (4, 8, 16, 32):
        ref = _basis(golden, r)
        mine = orc.dct_basis_f64(r, r)
        np.testing.assert_allclose(mine, ref, rtol=0, atol=4e-6)
        np.testing.assert_allclose(ref @ ref.T, np.eye(r), atol=1e-6 if r <= 16 else 2e-6)


@pytest.mark.parametrize("i", range(len(cases.JPEG_CASES)))
def test_jpeg_oracle_bit_exact(golden, i):
    data, meta = golden
    name, dt, B, H, S, D, r, k, qb = cases.JPEG_CASES[i]
    x = cases.jpeg_input(i)
    assert sha(f32(x)) == _text(data[f"{name}/x_sha"]), "synthetic input drifted"
    xb = f32(x)
    basis = _basis(golden, r)
    coef = orc.jpeg_encode(xb, r, k, basis, dt)
    assert np.array_equal(coef.view(np.uint32), data[f"{name}/coef"].view(np.uint32))
    rec = orc.jpeg_decode(coef, None, basis, r, "f32", out_len=S)
    assert np.array_equal(rec, data[f"{name}/rec_coef"])
    if qb:
        codes, scales = orc.jpeg_quantize(coef, dt)
        assert np.array_equal(codes, data[f"{name}/codes"])
        assert np.array_equal(scales.view(np.uint32), data[f"{name}/scales"].view(np.uint32))
        recq = orc.jpeg_decode(codes, scales, basis, r, "f32", out_len=S)
        assert np.array_equal(recq, data[f"{name}/rec_q"])
    # stream semantics: only complete blocks are archived (cache.py:154-157)
    n = S // r
    assert n == meta[name]["n_blocks"]
    st = data[f"{name}/st_coeffs"]
    if qb:
        assert np.array_equal(st, codes[..., :n, :, :])
        assert np.array_equal(data[f"{name}/st_scales"], scales[..., :n, :, :])
        view = orc.jpeg_decode(st, data[f"{name}/st_scales"], basis, r, dt)
    else:
        assert np.array_equal(st, coef[..., :n, :, :])
        view = orc.jpeg_decode(st, None, basis, r, dt)
    view = np.concatenate([view, xb[..., n * r:, :]], axis=-2)
    assert np.array_equal(view, data[f"{name}/st_read"])


@pytest.mark.parametrize("i", range(len(cases.PNG_CASES)))
def test_png_oracle_bit_exact(golden, i):
    data, _ = golden
    name, dt, B, H, S, D, r, keep = cases.PNG_CASES[i]
    x = cases.png_input(i)
    assert sha(f32(x)) == _text(data[f"{name}/x_sha"])
    d, a = orc.png_encode(f32(x), r, keep)
    # bit-exact including the sign of zeroed deltas (delta * mask, png.py:59)
    assert np.array_equal(d.view(np.uint32), data[f"{name}/deltas"].view(np.uint32))
    assert np.array_equal(a, data[f"{name}/anchors"])
    rec = orc.png_decode(d, a, dt)
    assert np.array_equal(rec.view(np.uint32), data[f"{name}/rec"].view(np.uint32))


def _oracle_stream_rows(x, mode, kw, basis, dt, r=8):
    """Archive x like _CodecStream.append (cache.py:143-159) with the oracle:
    returns (rows (B,H,n,s,D) as the attention reads them, raw tail)."""
    xb = f32(x)
    S = xb.shape[-2]
    n = S // r
    head, raw = xb[..., :n * r, :], xb[..., n * r:, :]
    raw = raw if raw.shape[-2] else None
    if n == 0:
        return None, raw
    if mode == "jpeg":
        k = kw["keep_freqs"]
        coef = orc.jpeg_encode(head, r, k, basis, dt)
        if kw.get("quant_bits"):
            codes, scales = orc.jpeg_quantize(coef, dt)
            return orc.stored_rows("jpeg", codes=codes, scales=scales), raw
        return orc.stored_rows("jpeg", codes=coef), raw
    d, a = orc.png_encode(head, r, kw["keep_ratio"])
    return orc.stored_rows("png", anchors=a, deltas=d), raw


@pytest.mark.parametrize("i", range(len(cases.ATTN_CASES)))
def test_attention_oracle_matches_reference(golden, i):
    data, _ = golden
    name, mode, kw, dt, B, Hk, G, S, D, tail = cases.ATTN_CASES[i]
    k, v, q = cases.attn_input(i)
    assert sha(f32(k)) + sha(f32(v)) + sha(f32(q)) == _text(data[f"{name}/kvq_sha"])
    basis = _basis(golden, 8)
    kr, kraw = _oracle_stream_rows(k, mode, kw, basis, dt)
    vr, vraw = _oracle_stream_rows(v, mode, kw, basis, dt)
    A = orc.block_basis(mode, 8, kw.get("keep_freqs", 8), basis)
    out = orc.decode_attention(f32(q), kr, vr, kraw, vraw, A)
    if dt == "f32":
        # reference fp32 torch path vs fp64 oracle (attention tolerance 1e-5)
        np.testing.assert_allclose(out, data[f"{name}/out"], rtol=0, atol=1e-5)
    else:
        # fp32 arithmetic on the same archive: the fp32 tolerance
        np.testing.assert_allclose(out, data[f"{name}/out_f32math"], rtol=0, atol=1e-5)
        # the reference's bf16 torch path rounds dequantized rows, logits and
        # the output to bf16 (unit roundoff 2^-8): its error is about one bf16
        # unit of the largest output magnitude (0.3-0.4% on these cases), so
        # the bound is two such units (2e-3 absolute at |out| <= 0.25)
        ref = data[f"{name}/out"]
        bound = max(2e-3, 2.0 ** -7 * float(np.abs(ref).max()))
        assert float(np.abs(out - ref).max()) <= bound
    fp32 = orc.reference_attention_fp32(f32(q), kr, vr, kraw, vraw, A)
    np.testing.assert_allclose(fp32, out, rtol=0, atol=2e-5)


def test_cfg1_digests_and_attention(golden):
    """Config 1 at full size: B=1 Hq=32 Hkv=8 S=4096 D=128 fp32, r=8 K=2 int8;
    the second case appends one raw token."""
    data, meta = golden
    c = meta["cfg1"]
    k, v, q = cases.cfg1_input()
    assert sha(f32(k)) + sha(f32(v)) + sha(f32(q)) == c["digests"]["inputs"]
    basis = _basis(golden, 8)
    A = orc.block_basis("jpeg", 8, 2, basis)
    for t in (0, 1):
        dg = c["digests"][f"t{t}"]
        rows = {}
        for nm, x in (("k", k), ("v", v)):
            head = f32(x[:, :, :c["S"]])
            codes, scales = orc.jpeg_quantize(orc.jpeg_encode(head, 8, 2, basis), "f32")
            assert sha(codes) == dg[f"{nm}_codes"]
            assert sha(scales) == dg[f"{nm}_scales"]
            rows[nm] = orc.stored_rows("jpeg", codes=codes, scales=scales)
        kraw = f32(k[:, :, c["S"]:c["S"] + t]) if t else None
        vraw = f32(v[:, :, c["S"]:c["S"] + t]) if t else None
        out = orc.decode_attention(f32(q), rows["k"], rows["v"], kraw, vraw, A)
        np.testing.assert_allclose(out, data[f"cfg1_t{t}/out"], rtol=0, atol=1e-5)


# The reference's published reconstruction table (README "Reconstruction
# quality", produced by benchmarks/bench_reconstruct.py): seeded random walk
# B=2 H=8 S=2048 D=64, r=8.  (mode, keep, int8) -> (PSNR dB, cosine)
PUBLISHED = [
    ("jpeg", 1, False, 42.95, 0.99943),
    ("jpeg", 2, False, 47.22, 0.99985),
    ("jpeg", 4, False, 51.66, 1.00001),
    ("jpeg", 2, True, 46.92, 0.99983),
    ("jpeg", 4, True, 50.89, 0.99999),
    ("png", 0.5, False, 50.11, 0.99997),
]


def test_published_reconstruction_quality(golden):
    torch.manual_seed(0)
    x = torch.cumsum(torch.randn(2, 8, 2048, 64) * 0.1, dim=-2)
    xn = f32(x)
    xt = x
    basis = _basis(golden, 8)

    def psnr(hat):
        rmse = math.sqrt(float(((xn.astype(np.float64) - hat) ** 2).mean()))
        return 20 * math.log10(float(np.abs(xn).max()) / max(rmse, 1e-12))

    def cosine(hat):
        return torch.nn.functional.cosine_similarity(
            xt.flatten(), torch.from_numpy(hat).flatten(), dim=0).item()

    for mode, keep, q8, ref_psnr, ref_cos in PUBLISHED:
        if mode == "jpeg":
            coef = orc.jpeg_encode(xn, 8, keep, basis)
            if q8:
                codes, scales = orc.jpeg_quantize(coef)
                hat = orc.jpeg_decode(codes, scales, basis, 8)
            else:
                hat = orc.jpeg_decode(coef, None, basis, 8)
        else:
            d, a = orc.png_encode(xn, 8, keep)
            hat = orc.png_decode(d, a)
        assert round(psnr(hat), 2) == pytest.approx(ref_psnr, abs=0.011), (mode, keep, q8)
        assert round(cosine(hat), 5) == pytest.approx(ref_cos, abs=1.1e-5), (mode, keep, q8)
