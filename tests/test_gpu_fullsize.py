"""GPU parity at the benchmarked sizes (the configurations bench.py times).

* config 3: png lossless tier at full size (B=8, Hkv=8, S=16384, D=128, fp32,
  r=16, keep_ratio=1.0, AR(1) rho=0.98; 512 MiB in): filter and reconstruct
  bit-exact against the CPU oracle, through the public codec functions and
  through the stream's append/read cycle;
* config 4: one layer of the streaming workload at full size (B=64, Hkv=8,
  D=128, bf16, jpeg r=8 K=2 int8), one token per step from 0 to 65,536
  through nine capacity doublings: the streamed archive and the incremental
  read equal a one-shot archive bit for bit, and decode attention on the
  streamed archive matches the fp64 oracle.
Config 1 (full-size digests) and config 5 (full per-GPU size) are covered in
test_gpu_codec.py and test_gpu_attention.py; config 2 is checked by bench.py
after its timed region."""

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


def _same_bits(a: torch.Tensor, b: np.ndarray) -> bool:
    a = np.ascontiguousarray(a.float().cpu().numpy() if a.dtype != torch.int8
                             else a.cpu().numpy())
    b = np.ascontiguousarray(b)
    if a.dtype == np.float32:
        return np.array_equal(a.view(np.uint32), b.astype(np.float32).view(np.uint32))
    return np.array_equal(a, b)


def test_config3_png_full_size_bit_exact():
    import bench
    import flashcodec_b200 as fc
    B, H, S, D, r = 8, 8, 16384, 128, 16
    x = bench.synth_stream(B, H, S, D, 0.98, 3, device=DEV, dtype=torch.float32)
    xh = x.cpu().numpy()
    rd, ra = orc.png_encode(xh, r, 1.0)
    deltas, anchors = fc.png_filter(x, r, 1.0)
    assert deltas.shape == (B, H, S // r, r - 1, D) and deltas.dtype == torch.float32
    assert _same_bits(deltas, rd) and _same_bits(anchors, ra)
    del deltas, anchors
    rec_ref = orc.png_decode(rd, ra, "f32")
    rec = fc.png_reconstruct(torch.from_numpy(rd).to(DEV), torch.from_numpy(ra).to(DEV))
    assert _same_bits(rec, rec_ref)
    del rec
    # the same archive through the stream (append, then the memoized read)
    st = fc._CodecStream(fc.make_codec("png", block_size=r, keep_ratio=1.0))
    st.append(x)
    n = st.n_blocks
    assert _same_bits(st._deltas[:, :, :n], rd) and _same_bits(st._anchors[:, :, :n], ra)
    assert _same_bits(st.read(), rec_ref)
    # lossless tier: fp32 reconstruction within 1e-4 of the input (the spec's bar)
    assert np.abs(rec_ref - xh).max() <= 1e-4 * max(1.0, np.abs(xh).max())


def test_config4_stream_full_size_equals_one_shot():
    import bench
    import flashcodec_b200 as fc
    from test_gpu_attention import check_close
    B, Hq, Hk, D, S = 64, 16, 8, 128, 65536
    k, v, q = bench.synth_case(B, Hq, Hk, S, D, 0.95, 4, device=DEV, dtype=torch.bfloat16)
    kw = dict(mode="jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    c = fc.CodecKVCache(**kw)
    caps, views = set(), {}
    for t in range(S):
        c.append(k[:, :, t:t + 1], v[:, :, t:t + 1])
        if (t & (t + 1)) == 0 or t == S - 1:           # t = 2^m - 1: incremental reads
            caps.add(c._keys[0]._capacity)
            views[t + 1] = c._keys[0].read()[:, :, :t + 1].clone()
    assert caps >= {16 * 2 ** i for i in range(10)}   # 16 .. 8192 blocks: nine doublings
    one = fc.CodecKVCache(**kw)
    one.append(k, v)
    ks, vs = c._keys[0], c._values[0]
    n = ks.n_blocks
    assert n == S // 8 and one._keys[0].n_blocks == n
    for a, b in ((ks, one._keys[0]), (vs, one._values[0])):
        assert torch.equal(a._coeffs[:, :, :n], b._coeffs[:, :, :n])
        assert torch.equal(a._scales[:, :, :n], b._scales[:, :, :n])
    full = one._keys[0].read()
    for L, view in views.items():
        # archived positions of an incremental read equal the one-shot read;
        # positions still raw at that time are the raw tokens
        arch = (L // 8) * 8
        assert torch.equal(view[:, :, :arch], full[:, :, :arch])
        assert torch.equal(view[:, :, arch:L], k[:, :, arch:L])
    # attention on the streamed archive, sequence 0, against the fp64 oracle
    out = fc.codec_decode_attention(q, ks, vs)
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    rows = {nm: orc.stored_rows("jpeg", codes=f(st._coeffs[:1, :, :n]),
                                scales=f(st._scales[:1, :, :n])) for nm, st in (("k", ks), ("v", vs))}
    A = f(fc.block_basis(ks.codec, 8))
    ref = orc.decode_attention(f(q[:1]), rows["k"], rows["v"], None, None, A)
    check_close(out[:1], ref, torch.bfloat16)
