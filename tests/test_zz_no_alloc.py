"""fc_decode_attn_noalloc: decode attention for callers that cannot allocate
device memory (an engine that gave all of HBM to its KV pool at start-up, or
an FFI plugin that may not call cudaMalloc).  It must give the same result as
the allocating entry point and as the fp64 oracle, call after call, since its
scratch array keeps whatever the previous call left; and its status word must
report a bounded wait that gave up until the caller reads it.

Collected last on purpose (file name), and self-contained: it passes in a fresh
process and after every other test.  Called through the C ABI with ctypes.
"""

import ctypes
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _noalloc(lib, q, ks, vs, A, scale, out):
    """fc_decode_attn_noalloc on a product stream pair (no workspace)."""
    from flashcodec_b200 import _kernels as K
    n = ks.n_blocks
    kr, vr = ks._coeffs[:, :, :n], vs._coeffs[:, :, :n]
    ksc, vsc = ks._scales[:, :, :n], vs._scales[:, :, :n]
    kraw, vraw = ks.raw, vs.raw
    B, Hq, _, D = q.shape
    S = lambda t, k: [t.stride(i) for i in range(k)] if t is not None else [0] * k  # noqa: E731
    with torch.cuda.device(q.device):
        return lib.fc_decode_attn_noalloc(
            _P(q), K.dtype_code(q), B, Hq, D, q.stride(0), q.stride(1),
            kr.shape[1], n, kr.shape[3], A.shape[0], K.dtype_code(kr),
            _P(kr), *S(kr, 4), _P(vr), *S(vr, 4),
            _P(ksc), *S(ksc, 3), _P(vsc), *S(vsc, 3), K.dtype_code(ksc),
            _P(kraw), *S(kraw, 3), _P(vraw), *S(vraw, 3),
            K.dtype_code(kraw) if kraw is not None else 0, 0 if kraw is None else kraw.shape[2],
            _P(A), float(scale), _P(out), K.dtype_code(out), out.stride(0), out.stride(1),
            _stream(q.device))


def _status(lib, reset):
    """The no-alloc status word, read through fc_decode_attn_noalloc_status."""
    from flashcodec_b200 import _lib
    word = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    rc = lib.fc_decode_attn_noalloc_status(_P(word), int(reset), _stream(word.device))
    assert rc == _lib.FC_OK, lib.fc_last_error_string()
    return int(word.item())


def _oracle(q, ks, vs):
    """fp64 oracle attention on the archive read back from the device."""
    import flashcodec_b200 as fc
    from oracle import oracle as orc
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    n = ks.n_blocks
    rows = {}
    for nm, st in (("k", ks), ("v", vs)):
        rows[nm] = orc.stored_rows("jpeg", codes=st._coeffs[:, :, :n].cpu().numpy()
                                   .astype(np.float32), scales=f(st._scales[:, :, :n]))
        rows[nm + "raw"] = f(st.raw) if st.raw is not None else None
    A = f(fc.block_basis(ks.codec, ks.block_size))
    return orc.decode_attention(f(q), rows["k"], rows["v"], rows["kraw"], rows["vraw"], A)


def _close(a, ref, dtype):
    """The attention bar: 1e-5 absolute for fp32 outputs, 2e-3 plus one bf16
    rounding of the output otherwise."""
    a = a.float().cpu().numpy()
    ref = ref.float().cpu().numpy() if isinstance(ref, torch.Tensor) else ref
    if dtype == torch.float32:
        return np.abs(a - ref).max() <= 1e-5
    return bool(np.all(np.abs(a - ref) <= 2e-3 + 2.0 ** -8 * np.abs(ref)))


def _case(dt, G, K, S, tail, seed=17):
    import bench
    import flashcodec_b200 as fc
    B, Hk, D = 2, 8, 128
    k, v, q = bench.synth_case(B, Hk * G, Hk, S + tail, D, 0.95, seed, device=DEV, dtype=dt)
    cfg = dict(mode="jpeg", block_size=8, keep_freqs=K, quant_bits=8)
    ks, vs = fc._CodecStream(fc.make_codec(**cfg)), fc._CodecStream(fc.make_codec(**cfg))
    ks.append(k)
    vs.append(v)
    return q, ks, vs


@pytest.mark.parametrize("dt,G,K,S,tail", [
    (torch.bfloat16, 4, 4, 8 * 700, 5),     # config-2 layer shape at B=2: many splits
    (torch.float32, 4, 2, 8 * 512, 1),      # config-1 shape
    (torch.bfloat16, 2, 2, 8 * 40, 0),      # small: one split
])
def test_noalloc_matches_allocating_entry_point_twice(dt, G, K, S, tail):
    import flashcodec_b200 as fc
    from flashcodec_b200 import _lib
    from flashcodec_b200.attention import _device_A
    lib = _lib.load()
    q, ks, vs = _case(dt, G, K, S, tail)
    ref = fc.codec_decode_attention(q, ks, vs)              # allocating entry point
    exact = _oracle(q, ks, vs)                               # fp64 oracle
    A = _device_A(ks.codec, 8, q.device)
    scale = q.shape[-1] ** -0.5
    for _ in range(2):                                        # two calls in a row
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, q, ks, vs, A, scale, out)
        assert rc == _lib.FC_OK, lib.fc_last_error_string()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert _close(out, ref, dt)
        assert _close(out, exact, dt)
    assert _status(lib, reset=False) == 0


def test_noalloc_status_reports_a_wait_that_gave_up():
    """Failure detection without a GPU fault: the bounded-wait self-test gives
    up on the no-alloc scratch's status word; later no-alloc calls still
    compute valid output but do not clear the word; reading it with reset
    returns the launch number once and clears it."""
    from flashcodec_b200 import _lib
    from flashcodec_b200.attention import _device_A
    lib = _lib.load()
    q, ks, vs = _case(torch.bfloat16, 4, 2, 8 * 300, 3, seed=5)
    A = _device_A(ks.codec, 8, q.device)
    out = torch.empty_like(q)
    assert _noalloc(lib, q, ks, vs, A, q.shape[-1] ** -0.5, out) == _lib.FC_OK
    _status(lib, reset=True)
    assert _status(lib, reset=False) == 0
    planted = 1 << 30        # far above any launch number a test run reaches
    with torch.cuda.device(q.device):
        assert lib.fc_selftest_noalloc_wait(planted, _stream(q.device)) == _lib.FC_OK
    torch.cuda.synchronize()
    assert _status(lib, reset=False) == planted
    out2 = torch.full_like(q, float("nan"))
    assert _noalloc(lib, q, ks, vs, A, q.shape[-1] ** -0.5, out2) == _lib.FC_OK
    torch.cuda.synchronize()
    assert torch.equal(out2, out)                             # still valid, deterministic
    assert _status(lib, reset=True) == planted                # sticky until read
    assert _status(lib, reset=False) == 0


def test_noalloc_refuses_oversized_plans():
    """A plan whose split partials exceed the fixed scratch is refused with
    FC_ERANGE before any launch (64 sequences x 8 KV heads x 32768 blocks:
    256 splits per unit, ~270 MB of partials)."""
    from flashcodec_b200 import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(0x1000)
    B, Hq, Hk, n = 64, 32, 8, 32768
    assert lib.fc_decode_attn_workspace_size(B, Hq, Hk, 128, n, 2, 8, 0) > (16 << 20)
    rc = lib.fc_decode_attn_noalloc(
        dummy, _lib.FC_BF16, B, Hq, 128, Hq * 128, 128, Hk, n, 2, 8, _lib.FC_I8,
        dummy, 0, 0, 0, 0, dummy, 0, 0, 0, 0, dummy, 0, 0, 0, dummy, 0, 0, 0, _lib.FC_F32,
        None, 0, 0, 0, None, 0, 0, 0, _lib.FC_BF16, 0, dummy, 0.1, dummy, _lib.FC_BF16,
        Hq * 128, 128, None)
    assert rc == _lib.FC_ERANGE, lib.fc_last_error_string()
    assert b"scratch" in lib.fc_last_error_string()
