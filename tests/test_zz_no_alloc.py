"""fc_decode_attn_noalloc: decode attention for callers that cannot allocate
device memory (an engine that gave all of HBM to its KV pool at start-up, or
an FFI plugin that may not call cudaMalloc).  It must give the same result as
the allocating entry point, call after call, since its scratch array keeps
whatever the previous call left.

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


def _noalloc(lib, q, ks, vs, A, scale, out):
    """fc_decode_attn_noalloc on a product stream pair (no workspace)."""
    from flashcodec_b200 import _kernels as K
    n = ks.n_blocks
    kr, vr = ks._coeffs[:, :, :n], vs._coeffs[:, :, :n]
    ksc, vsc = ks._scales[:, :, :n], vs._scales[:, :, :n]
    kraw, vraw = ks.raw, vs.raw
    B, Hq, _, D = q.shape
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    S = lambda t, k: [t.stride(i) for i in range(k)] if t is not None else [0] * k  # noqa: E731
    with torch.cuda.device(q.device):
        return lib.fc_decode_attn_noalloc(
            P(q), K.dtype_code(q), B, Hq, D, q.stride(0), q.stride(1),
            kr.shape[1], n, kr.shape[3], A.shape[0], K.dtype_code(kr),
            P(kr), *S(kr, 4), P(vr), *S(vr, 4),
            P(ksc), *S(ksc, 3), P(vsc), *S(vsc, 3), K.dtype_code(ksc),
            P(kraw), *S(kraw, 3), P(vraw), *S(vraw, 3),
            K.dtype_code(kraw) if kraw is not None else 0, 0 if kraw is None else kraw.shape[2],
            P(A), float(scale), P(out), K.dtype_code(out), out.stride(0), out.stride(1),
            ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream))


def _close(a, b, dtype):
    a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
    if dtype == torch.float32:
        return np.abs(a - b).max() <= 1e-5
    return bool(np.all(np.abs(a - b) <= 2e-3 + 2.0 ** -8 * np.abs(b)))


@pytest.mark.parametrize("dt,G,K,S,tail", [
    (torch.bfloat16, 4, 4, 8 * 700, 5),     # config-2 layer shape at B=2: many splits
    (torch.float32, 4, 2, 8 * 512, 1),      # config-1 shape
    (torch.bfloat16, 2, 2, 8 * 40, 0),      # small: one split
])
def test_noalloc_matches_allocating_entry_point_twice(dt, G, K, S, tail):
    import bench
    import flashcodec_b200 as fc
    from flashcodec_b200 import _lib
    from flashcodec_b200.attention import _device_A
    lib = _lib.load()
    B, Hk, D = 2, 8, 128
    k, v, q = bench.synth_case(B, Hk * G, Hk, S + tail, D, 0.95, 17, device=DEV, dtype=dt)
    cfg = dict(mode="jpeg", block_size=8, keep_freqs=K, quant_bits=8)
    ks, vs = fc._CodecStream(fc.make_codec(**cfg)), fc._CodecStream(fc.make_codec(**cfg))
    ks.append(k)
    vs.append(v)
    ref = fc.codec_decode_attention(q, ks, vs)              # allocating entry point
    A = _device_A(ks.codec, 8, q.device)
    scale = D ** -0.5
    for _ in range(2):                                        # two calls in a row
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, q, ks, vs, A, scale, out)
        assert rc == _lib.FC_OK, lib.fc_last_error_string()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert _close(out, ref, dt)


def test_noalloc_refuses_oversized_plans():
    from flashcodec_b200 import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(0x1000)
    # a plan whose split partials exceed the fixed scratch: refused on the host
    need = lib.fc_decode_attn_workspace_size(1024, 64, 8, 128, 1 << 20, 2, 8, 0)
    assert need > (16 << 20)
    rc = lib.fc_decode_attn_noalloc(
        dummy, _lib.FC_BF16, 1024, 64, 128, 64 * 128, 128, 8, 1 << 20, 2, 8, _lib.FC_I8,
        dummy, 0, 0, 0, 0, dummy, 0, 0, 0, 0, dummy, 0, 0, 0, dummy, 0, 0, 0, _lib.FC_F32,
        None, 0, 0, 0, None, 0, 0, 0, _lib.FC_BF16, 0, dummy, 0.1, dummy, _lib.FC_BF16,
        64 * 128, 128, None)
    assert rc == _lib.FC_ERANGE
    assert b"scratch" in lib.fc_last_error_string()
