"""GPU parity of the per-group coefficient format (quantize_coeffs /
make_codec with group_size; the per-32 quantizer of
docs/llama-cpp-kv-quantization.md:179-234): codes, scales and the read path
bit-exact against the CPU oracle, decode attention within the attention bar
of the fp64 oracle, for the head-dim-128 fast paths and the general kernels."""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))
sys.path.insert(0, str(ROOT))

from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"
TAG = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


def f32(t):
    return t.float().cpu().numpy()


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("group", [32, 16, 64])
def test_quantize_coeffs_grouped_matches_oracle(dt, group):
    import flashcodec_b200 as fc
    g = torch.Generator().manual_seed(group)
    c = (torch.randn(2, 3, 7, 4, 128, generator=g) *
         torch.exp(2 * torch.randn(2, 3, 7, 4, 1, generator=g))).to(dt)
    codes, scales = fc.quantize_coeffs(c.to(DEV), 8, group_size=group)
    rc, rs = orc.jpeg_quantize_grouped(f32(c), group, TAG[dt])
    assert scales.shape == (2, 3, 7, 4, 128 // group) and scales.dtype == torch.float32
    assert np.array_equal(codes.cpu().numpy(), rc) and bits_equal(f32(scales), rs)
    deq = fc.dequantize_coeffs(codes, scales)
    assert bits_equal(f32(deq), orc.dequantize_grouped(rc, rs))


def _oracle_archive(x, r, k, group, dtype, basis):
    coef = orc.jpeg_encode(x, r, k, basis, dtype)
    return orc.jpeg_quantize_grouped(coef, group, dtype)


@pytest.mark.parametrize("dt,D,r,k,group,sdt,S", [
    (torch.bfloat16, 128, 8, 4, 32, torch.float32, 8 * 300 + 5),   # fast paths (per-32)
    (torch.float16, 128, 16, 2, 16, torch.float16, 16 * 40 + 3),   # fast, fp16 scales
    (torch.bfloat16, 128, 8, 8, 16, torch.float32, 8 * 50 + 1),    # k * groups > 32: general
    (torch.float32, 64, 16, 3, 32, torch.float32, 16 * 30 + 7),    # general kernels
    (torch.float32, 96, 8, 2, 32, torch.float32, 8 * 64),          # odd head dim, no tail
])
def test_grouped_stream_archive_read_and_attention(dt, D, r, k, group, sdt, S):
    import bench
    import flashcodec_b200 as fc
    from test_gpu_attention import check_close
    B, Hq, Hk = 2, 8, 4
    kx, vx, q = bench.synth_case(B, Hq, Hk, S, D, 0.95, D + k, dtype=dt)
    kw = dict(block_size=r, keep_freqs=k, quant_bits=8, scale_dtype=sdt, group_size=group)
    ks = fc._CodecStream(fc.make_codec("jpeg", **kw))
    vs = fc._CodecStream(fc.make_codec("jpeg", **kw))
    ks.append(kx.to(DEV))
    vs.append(vx.to(DEV))
    n = S // r
    basis = fc.dct_basis(r, k).numpy()
    rows = {}
    for nm, x, st in (("k", kx, ks), ("v", vx, vs)):
        codes, scales = _oracle_archive(f32(x)[:, :, :n * r], r, k, group, TAG[dt], basis)
        assert st._scales.shape[-1] == D // group
        assert np.array_equal(st._coeffs[:, :, :n].cpu().numpy(), codes)
        assert bits_equal(f32(st._scales[:, :, :n]), orc.round_to(scales, TAG[sdt]))
        # the read path: dequantize with each group's scale, then synthesis
        rec = orc.jpeg_decode(orc.dequantize_grouped(codes, f32(st._scales[:, :, :n])), None,
                              basis, r, TAG[dt])
        assert bits_equal(f32(st.read()[:, :, :n * r]), rec)
        rows[nm] = orc.dequantize_grouped(codes, f32(st._scales[:, :, :n]))
        rows[nm + "raw"] = f32(x)[:, :, n * r:] if S > n * r else None
    out = fc.codec_decode_attention(q.to(DEV), ks, vs)
    A = orc.block_basis("jpeg", r, k, basis)
    ref = orc.decode_attention(f32(q), rows["k"], rows["v"], rows["kraw"], rows["vraw"], A)
    check_close(out, ref, dt)


def _grouped_streams(k, v, group, K=4, r=8):
    import flashcodec_b200 as fc
    kw = dict(block_size=r, keep_freqs=K, quant_bits=8, group_size=group)
    ks = fc._CodecStream(fc.make_codec("jpeg", **kw))
    vs = fc._CodecStream(fc.make_codec("jpeg", **kw))
    ks.append(k)
    vs.append(v)
    return ks, vs


def _grouped_oracle(q, ks, vs):
    import flashcodec_b200 as fc
    n = ks.n_blocks
    rows = {nm: orc.dequantize_grouped(st._coeffs[:, :, :n].cpu().numpy(), f32(st._scales[:, :, :n]))
            for nm, st in (("k", ks), ("v", vs))}
    A = f32(fc.block_basis(ks.codec, ks.block_size))
    raw = lambda st: f32(st.raw) if st.raw is not None else None  # noqa: E731
    return orc.decode_attention(f32(q), rows["k"], rows["v"], raw(ks), raw(vs), A)


def test_grouped_config2_shape_and_kernel_choice():
    """A config-2 layer shape (bf16, r=8, K=4) in the per-32 format: the
    default kernel, and the tensor-core kernel forced (its per-group form:
    one fp32 scale per 32 channels at head dim 128), within the bar; forcing
    the tensor-core kernel on a per-16 archive is refused."""
    import bench
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as Kn
    from test_gpu_attention import check_close
    k, v, q = bench.synth_case(2, 32, 8, 8 * 700 + 5, 128, 0.95, 44, device=DEV,
                               dtype=torch.bfloat16)
    ks, vs = _grouped_streams(k, v, 32)
    ref = _grouped_oracle(q, ks, vs)
    check_close(fc.codec_decode_attention(q, ks, vs), ref, torch.bfloat16)
    prev = Kn.set_attn_kernel("tensor-core")
    try:
        check_close(fc.codec_decode_attention(q, ks, vs), ref, torch.bfloat16)
        ks16, vs16 = _grouped_streams(k, v, 16)
        with pytest.raises(NotImplementedError):
            fc.codec_decode_attention(q, ks16, vs16)
    finally:
        Kn.set_attn_kernel(prev)
    assert Kn.attn_status(q.device) == 0


@pytest.mark.parametrize("G,K,S,tail,B,Hk", [
    (4, 4, 8 * 2000, 5, 2, 4),      # config-2 layer shape
    (2, 2, 8 * 300, 3, 2, 4),       # s = 2
    (1, 1, 8 * 70, 0, 2, 4),        # s = 1
    (3, 8, 8 * 90, 7, 2, 4),        # s = 8, G not a power of 2
    (4, 4, 8 * 20, 4, 2, 4),        # one split, partial tile
    (4, 4, 8 * 9000, 1, 1, 1),      # one unit, many splits merged
])
def test_grouped_tensor_core_vs_cuda_core_vs_oracle(G, K, S, tail, B, Hk):
    """Per-32 archives on the tensor-core kernel's per-group form and on the
    CUDA-core kernel, both against the fp64 oracle of the dequantized rows."""
    import bench
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as Kn
    from test_gpu_attention import check_close
    k, v, q = bench.synth_case(B, Hk * G, Hk, S + tail, 128, 0.95, 45, device=DEV,
                               dtype=torch.bfloat16)
    ks, vs = _grouped_streams(k, v, 32, K=K)
    ref = _grouped_oracle(q, ks, vs)
    prev = Kn.set_attn_kernel("auto")
    try:
        for which in ("tensor-core", "cuda-core"):
            Kn.set_attn_kernel(which)
            check_close(fc.codec_decode_attention(q, ks, vs), ref, torch.bfloat16)
    finally:
        Kn.set_attn_kernel(prev)
    assert Kn.attn_status(q.device) == 0
