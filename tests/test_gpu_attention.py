"""GPU parity of the split-K decode-attention kernel.

Tolerances (the attention bar): fp32 outputs within 1e-5 absolute of the fp64
oracle on the same archive; bf16 outputs within 2e-3 absolute plus one bf16
rounding of the output (2^-8 relative) of the oracle.  Against the reference's
own bf16 torch path (which rounds its intermediates to bf16) the bound is two
bf16 units of the largest output, as in the oracle pinning test.
"""

import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
import cases  # noqa: E402
from cases import f32  # noqa: E402
from oracle import oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"


def oracle_rows(st):
    """Stored rows, raw tail and A of a product stream, read back to the host."""
    n = st.n_blocks
    raw = f32(st.raw) if st.raw is not None else None
    if n == 0:
        return None, raw
    if st.codec.name == "jpeg":
        if st.codec.quantized:
            codes = st._coeffs[:, :, :n].cpu().numpy().astype(np.float32)
            return orc.stored_rows("jpeg", codes=codes, scales=f32(st._scales[:, :, :n])), raw
        return orc.stored_rows("jpeg", codes=f32(st._coeffs[:, :, :n])), raw
    return orc.stored_rows("png", anchors=f32(st._anchors[:, :, :n]),
                           deltas=f32(st._deltas[:, :, :n])), raw


def oracle_attention(q, ks, vs, scale=None):
    import flashcodec_b200 as fc
    kr, kraw = oracle_rows(ks)
    vr, vraw = oracle_rows(vs)
    A = f32(fc.block_basis(ks.codec, ks.block_size))
    return orc.decode_attention(f32(q), kr, vr, kraw, vraw, A, scale)


def check_close(out, ref, dtype):
    o = f32(out)
    if dtype == torch.float32:
        err = np.abs(o - ref).max()
        assert err <= 1e-5, err
    else:
        bound = 2e-3 + 2.0 ** -8 * np.abs(ref)
        assert np.all(np.abs(o - ref) <= bound), np.abs(o - ref).max()


def build(mode, kw, k, v, r=8):
    import flashcodec_b200 as fc
    ks = fc._CodecStream(fc.make_codec(mode, block_size=r, **kw))
    vs = fc._CodecStream(fc.make_codec(mode, block_size=r, **kw))
    ks.append(k)
    vs.append(v)
    return ks, vs


@pytest.mark.parametrize("i", range(len(cases.ATTN_CASES)))
def test_attention_golden_cases(golden, i):
    import flashcodec_b200 as fc
    data, _ = golden
    name, mode, kw, dt, B, Hk, G, S, D, tail = cases.ATTN_CASES[i]
    k, v, q = cases.attn_input(i)
    ks, vs = build(mode, kw, k.to(DEV), v.to(DEV))
    out = fc.codec_decode_attention(q.to(DEV), ks, vs)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert ks._rec is None and vs._rec is None          # no materialization
    ref = oracle_attention(q, ks, vs)
    check_close(out, ref, q.dtype)
    gold = data[f"{name}/out"]
    if dt == "f32":
        assert np.abs(f32(out) - gold).max() <= 1e-5
    else:
        assert np.abs(f32(out) - data[f"{name}/out_f32math"]).max() <= 2e-3 + 2.0 ** -8 * np.abs(gold).max()
        assert np.abs(f32(out) - gold).max() <= max(2e-3, 2.0 ** -7 * np.abs(gold).max())


def test_cfg1_attention(golden):
    """Config 1 at full size, t=0 and t=1 raw tail tokens."""
    import flashcodec_b200 as fc
    data, meta = golden
    c = meta["cfg1"]
    k, v, q = cases.cfg1_input()
    for t in (0, 1):
        ks, vs = build("jpeg", dict(keep_freqs=2, quant_bits=8),
                       k[:, :, :c["S"] + t].to(DEV), v[:, :, :c["S"] + t].to(DEV))
        out = fc.codec_decode_attention(q.to(DEV), ks, vs)
        assert np.abs(f32(out) - data[f"cfg1_t{t}/out"]).max() <= 1e-5
        check_close(out, oracle_attention(q, ks, vs), torch.float32)


@pytest.mark.parametrize("G,D,dt,K,quant,S,tail", [
    (4, 128, torch.bfloat16, 4, 8, 8 * 3001, 5),    # config-2 shape, odd block count
    (1, 64, torch.float32, 2, 8, 8 * 40, 0),
    (2, 256, torch.bfloat16, 2, 8, 8 * 70, 7),
    (8, 128, torch.float16, 2, 8, 8 * 90, 1),
    (3, 96, torch.float32, 2, 8, 8 * 50, 2),        # G not a power of two, D off the fast path
    (12, 128, torch.bfloat16, 4, 8, 8 * 33, 4),     # two head groups
    (4, 128, torch.bfloat16, 4, 0, 8 * 300, 3),     # unquantized bf16 coefficients
    (2, 80, torch.bfloat16, 3, 0, 8 * 30, 6),
])
def test_attention_shapes_vs_oracle(G, D, dt, K, quant, S, tail):
    import flashcodec_b200 as fc
    B, Hk = 2, 2
    k, v, q = bench.synth_case(B, Hk * G, Hk, S + tail, D, 0.95, 11, dtype=dt)
    ks, vs = build("jpeg", dict(keep_freqs=K, quant_bits=quant), k.to(DEV), v.to(DEV))
    out = fc.codec_decode_attention(q.to(DEV), ks, vs)
    check_close(out, oracle_attention(q, ks, vs), dt)


def test_attention_raw_only_and_single_block():
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(2, 8, 4, 13, 128, 0.95, 5)
    for S in (5, 8, 13):
        ks, vs = build("jpeg", dict(keep_freqs=2, quant_bits=8), k[:, :, :S].to(DEV),
                       v[:, :, :S].to(DEV))
        out = fc.codec_decode_attention(q.to(DEV), ks, vs)
        check_close(out, oracle_attention(q, ks, vs), torch.float32)


def test_empty_cache_and_prefill_guard():
    import flashcodec_b200 as fc
    cfg = dict(mode="jpeg", block_size=8, keep_freqs=2)
    ks, vs = fc._CodecStream(fc.make_codec(**cfg)), fc._CodecStream(fc.make_codec(**cfg))
    q = torch.randn(2, 4, 1, 32, device=DEV)
    out = fc.codec_decode_attention(q, ks, vs)
    assert torch.equal(out, torch.zeros_like(out))
    with pytest.raises(ValueError):
        fc.codec_decode_attention(torch.randn(2, 4, 4, 32, device=DEV), ks, vs)


def test_png_attention_vs_oracle():
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(2, 8, 4, 96 + 3, 32, 0.98, 9)
    for keep in (1.0, 0.5):
        ks, vs = build("png", dict(keep_ratio=keep), k.to(DEV), v.to(DEV))
        out = fc.codec_decode_attention(q.to(DEV), ks, vs)
        check_close(out, oracle_attention(q, ks, vs), torch.float32)


def test_attention_repeated_calls_reuse_workspace():
    """The last-arriver counters reset themselves: many launches in a row on
    one workspace give identical results and a clean status word."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    k, v, q = bench.synth_case(4, 32, 8, 8 * 1500 + 3, 128, 0.95, 2, dtype=torch.bfloat16)
    ks, vs = build("jpeg", dict(keep_freqs=4, quant_bits=8), k.to(DEV), v.to(DEV))
    qd = q.to(DEV)
    first = fc.codec_decode_attention(qd, ks, vs)
    for _ in range(20):
        again = fc.codec_decode_attention(qd, ks, vs)
        assert torch.equal(again, first)
    assert K.attn_status(qd.device) == 0


def test_scale_argument_and_impl_names():
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(1, 4, 2, 64 + 2, 64, 0.95, 4)
    ks, vs = build("jpeg", dict(keep_freqs=2, quant_bits=8), k.to(DEV), v.to(DEV))
    for impl in ("auto", "cuda", "triton", "torch"):
        out = fc.codec_decode_attention(q.to(DEV), ks, vs, scale=0.3, impl=impl)
        check_close(out, oracle_attention(q, ks, vs, scale=0.3), torch.float32)
    with pytest.raises(ValueError):
        fc.codec_decode_attention(q.to(DEV), ks, vs, impl="bogus")


def test_cpu_tensors_are_rejected():
    import flashcodec_b200 as fc
    with pytest.raises(RuntimeError):
        fc.dct_compress(torch.randn(1, 1, 8, 16), 8, 2)


@pytest.fixture
def kernel_choice():
    from flashcodec_b200 import _kernels as K
    prev = K.set_attn_kernel("auto")
    yield K.set_attn_kernel
    K.set_attn_kernel(prev)


@pytest.mark.parametrize("G,K,dt,S,tail,sdt", [
    (4, 4, torch.bfloat16, 8 * 2000 + 0, 5, torch.float32),   # config-2 layer shape
    (4, 2, torch.float32, 8 * 512, 1, torch.float32),         # config-1 shape, fp32 q/out
    (8, 2, torch.bfloat16, 8 * 300, 3, torch.float32),        # N = 32 columns
    (1, 1, torch.float16, 8 * 70, 0, torch.float32),          # s = 1
    (3, 8, torch.bfloat16, 8 * 90, 7, torch.float32),         # s = 8, G not a power of 2
    (4, 2, torch.bfloat16, 8 * 3000, 2, torch.float16),       # fp16 scales (config 5 format)
    (2, 4, torch.bfloat16, 8 * 20, 4, torch.float32),         # one split, partial tile
])
def test_tensor_core_and_cuda_core_kernels_vs_oracle(kernel_choice, G, K, dt, S, tail, sdt):
    """Both decode-attention kernels on the same archive against the oracle."""
    import flashcodec_b200 as fc
    B, Hk = 2, 4
    k, v, q = bench.synth_case(B, Hk * G, Hk, S + tail, 128, 0.95, 23, dtype=dt)
    kw = dict(keep_freqs=K, quant_bits=8, scale_dtype=sdt)
    ks, vs = build("jpeg", kw, k.to(DEV), v.to(DEV))
    ref = oracle_attention(q, ks, vs)
    outs = {}
    for which in ("tensor-core", "cuda-core"):
        kernel_choice(which)
        outs[which] = fc.codec_decode_attention(q.to(DEV), ks, vs)
        check_close(outs[which], ref, dt)
    from flashcodec_b200 import _kernels as Kn
    assert Kn.attn_status(q.to(DEV).device) == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,K,S,tail,B,Hk", [
    (4, 4, 8 * 2000, 5, 2, 4),      # config-2 layer shape (jpeg-fp line)
    (8, 2, 8 * 300, 3, 2, 4),       # N = 32 columns, 2 ring stages
    (1, 1, 8 * 70, 0, 2, 4),        # s = 1
    (3, 8, 8 * 90, 7, 2, 4),        # s = 8, G not a power of 2
    (2, 4, 8 * 20, 4, 2, 4),        # one split, partial tile
    (4, 4, 8 * 9000, 1, 1, 1),      # one unit, many splits merged
])
def test_tensor_core_16bit_coefficients_vs_oracle(kernel_choice, G, K, S, tail, B, Hk, dt):
    """Unquantized jpeg archives (bf16 or fp16 coefficients, no scales): the
    tensor-core kernel's 16-bit paths and the CUDA-core kernel against the
    oracle, within the 16-bit output tolerance."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as Kn
    k, v, q = bench.synth_case(B, Hk * G, Hk, S + tail, 128, 0.95, 29, dtype=dt)
    ks, vs = build("jpeg", dict(keep_freqs=K, quant_bits=0), k.to(DEV), v.to(DEV))
    assert ks._coeffs.dtype == dt
    ref = oracle_attention(q, ks, vs)
    outs = {}
    for which in ("tensor-core", "cuda-core"):
        kernel_choice(which)
        outs[which] = fc.codec_decode_attention(q.to(DEV), ks, vs)
        check_close(outs[which], ref, dt)
    kernel_choice("auto")
    auto = fc.codec_decode_attention(q.to(DEV), ks, vs)
    assert torch.equal(auto, outs["tensor-core"])
    assert Kn.attn_status(q.to(DEV).device) == 0


@pytest.mark.parametrize("quant", [0, 8])
def test_unwritten_capacity_is_never_read(kernel_choice, quant):
    """The archive's capacity past its last block holds whatever the
    allocator left there; for bf16 rows that can be NaN or Inf, which no mask
    removes from a product.  With that region filled with NaN (K) and Inf (V),
    both kernels still match the oracle: the last tile of a split never reads
    past the archive's end."""
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(2, 8, 2, 8 * 300 + 3, 128, 0.95, 11, dtype=torch.bfloat16)
    ks, vs = build("jpeg", dict(keep_freqs=4, quant_bits=quant), k.to(DEV), v.to(DEV))
    n = ks.n_blocks
    assert ks._coeffs.shape[2] > n
    if quant:
        ks._coeffs[:, :, n:] = 127
        vs._coeffs[:, :, n:] = -127
        ks._scales[:, :, n:] = float("nan")
        vs._scales[:, :, n:] = float("inf")
    else:
        ks._coeffs[:, :, n:] = float("nan")
        vs._coeffs[:, :, n:] = float("inf")
    ref = oracle_attention(q, ks, vs)
    for which in ("tensor-core", "cuda-core"):
        kernel_choice(which)
        check_close(fc.codec_decode_attention(q.to(DEV), ks, vs), ref, torch.bfloat16)


def test_tensor_core_refuses_fp32_coefficients(kernel_choice):
    """fp32 coefficient rows stay on the CUDA-core kernel: forcing the
    tensor-core kernel on them fails loudly."""
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(1, 8, 2, 8 * 40, 128, 0.95, 3, dtype=torch.float32)
    ks, vs = build("jpeg", dict(keep_freqs=4, quant_bits=0), k.to(DEV), v.to(DEV))
    kernel_choice("tensor-core")
    with pytest.raises(NotImplementedError):
        fc.codec_decode_attention(q.to(DEV), ks, vs)


def test_tensor_core_refuses_unsupported_layout(kernel_choice):
    """Forcing the tensor-core kernel on a layout it does not take fails
    loudly instead of silently using another kernel."""
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(1, 4, 2, 8 * 20, 64, 0.95, 3)   # head_dim 64
    ks, vs = build("jpeg", dict(keep_freqs=2, quant_bits=8), k.to(DEV), v.to(DEV))
    kernel_choice("tensor-core")
    with pytest.raises(NotImplementedError):
        fc.codec_decode_attention(q.to(DEV), ks, vs)


def test_bounded_wait_gives_up_and_reports():
    """Failure detection without a GPU fault: a wait on an mbarrier that
    nothing arrives on gives up after the kernels' 100 ms limit, records the
    epoch in the status word, and the context stays usable afterwards."""
    import time
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    K.selftest_bounded_wait(status, 12345)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert status.item() == 12345
    assert 0.09 <= dt < 5.0, dt
    k, v, q = bench.synth_case(1, 4, 2, 8 * 30 + 3, 128, 0.95, 6)
    ks, vs = build("jpeg", dict(keep_freqs=2, quant_bits=8), k.to(DEV), v.to(DEV))
    out = fc.codec_decode_attention(q.to(DEV), ks, vs)
    check_close(out, oracle_attention(q, ks, vs), torch.float32)
    assert K.attn_status(q.to(DEV).device) == 0


def test_config5_full_size_kernels_agree():
    """Config 5 at full per-GPU size (16 sequences, S=131072, K=2, fp16
    scales): the tensor-core and CUDA-core kernels agree, and sequence 0
    matches the fp64 oracle."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as Kn
    B, Hq, Hk, S, D = 16, 32, 8, 131072, 128
    k, v, q = bench.synth_case(B, Hq, Hk, S + 3, D, 0.95, 55, device=DEV, dtype=torch.bfloat16)
    kw = dict(keep_freqs=2, quant_bits=8, scale_dtype=torch.float16)
    ks, vs = build("jpeg", kw, k, v)
    del k, v
    prev = Kn.set_attn_kernel("tensor-core")
    try:
        out_tc = fc.codec_decode_attention(q, ks, vs)
        Kn.set_attn_kernel("cuda-core")
        out_cc = fc.codec_decode_attention(q, ks, vs)
    finally:
        Kn.set_attn_kernel(prev)
    diff = (out_tc.float() - out_cc.float()).abs()
    assert diff.max().item() <= 2e-3 + 2.0 ** -8 * out_cc.float().abs().max().item()
    # sequence 0 against the oracle (archive rows read back for b = 0)
    n = ks.n_blocks
    A = f32(fc.block_basis(ks.codec, ks.block_size))
    rows = {}
    for nm, st in (("k", ks), ("v", vs)):
        rows[nm] = orc.stored_rows("jpeg", codes=st._coeffs[:1, :, :n].cpu().numpy().astype(np.float32),
                                   scales=f32(st._scales[:1, :, :n]))
        rows[nm + "raw"] = f32(st.raw[:1])
    ref = orc.decode_attention(f32(q[:1]), rows["k"], rows["v"], rows["kraw"], rows["vraw"], A)
    check_close(out_tc[:1], ref, torch.bfloat16)


@pytest.mark.parametrize("dt,r,keep,tail", [
    (torch.bfloat16, 8, 1.0, 3),     # bf16 anchors, fp32 deltas
    (torch.float32, 16, 1.0, 0),
    (torch.float16, 8, 0.5, 5),      # Top-M pruned deltas
])
def test_png_attention_reads_archive_in_place(dt, r, keep, tail):
    """png attention from the archive's own anchor and delta tensors (no row
    assembly) against the fp64 oracle."""
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(2, 8, 4, r * 40 + tail, 64, 0.98, 17, dtype=dt)
    ks, vs = build("png", dict(keep_ratio=keep), k.to(DEV), v.to(DEV), r=r)
    out = fc.codec_decode_attention(q.to(DEV), ks, vs)
    assert out.dtype == dt
    check_close(out, oracle_attention(q, ks, vs), dt)


def test_decode_attention_replays_in_a_cuda_graph():
    """A decode step's attention calls can be captured once and replayed as
    a CUDA graph (what a serving loop does to remove per-call host work): the
    replay gives bit-identical outputs to eager calls, also after the static
    query buffer is refilled."""
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(2, 32, 8, 8 * 300 + 5, 128, 0.95, 9, device=DEV,
                               dtype=torch.bfloat16)
    ks, vs = build("jpeg", dict(keep_freqs=4, quant_bits=8), k, v)
    q_static = q.clone()
    fc.codec_decode_attention(q_static, ks, vs)          # warm-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fc.codec_decode_attention(q_static, ks, vs)
    for seed in (10, 11):
        q_static.copy_(bench.synth_query(2, 32, 128, seed, device=DEV, dtype=torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, fc.codec_decode_attention(q_static, ks, vs))
