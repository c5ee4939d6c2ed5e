"""The C-ABI library: builds for sm_100a, loads without a GPU, exports every
symbol include/flashcodec_b200.h declares, and rejects bad arguments on the
host before any launch.  CPU only (no kernel is launched)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "flashcodec_b200.h"


@pytest.fixture(scope="module")
def lib():
    from flashcodec_b200 import _lib, build
    build.build()
    return _lib.load()


def declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"FC_API\s+[\w\s\*]+?\b(fc_\w+)\s*\(", text)


def test_header_declares_the_binding_table():
    from flashcodec_b200 import _lib
    assert declared_symbols() == list(_lib.SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_version(lib):
    assert lib.fc_version().decode().startswith("flashcodec_b200 ")


def test_host_validation(lib):
    from flashcodec_b200 import _lib
    P = ctypes.c_void_p
    dummy = P(0x1000)
    # int8 input to the archive kernel
    rc = lib.fc_jpeg_encode(dummy, _lib.FC_I8, 1, 1, 8, 16, 128, 128, 16, dummy, 8, 2,
                            dummy, 0, 0, 0, 0, None, 0, 0, 0, 0, None, None)
    assert rc == _lib.FC_EINVAL
    assert b"dtype" in lib.fc_last_error_string()
    # k > r
    rc = lib.fc_jpeg_encode(dummy, _lib.FC_F32, 1, 1, 8, 16, 128, 128, 16, dummy, 8, 9,
                            dummy, 0, 0, 0, 0, None, 0, 0, 0, 0, None, None)
    assert rc == _lib.FC_EINVAL
    # empty input is a no-op
    rc = lib.fc_jpeg_encode(dummy, _lib.FC_F32, 1, 1, 0, 16, 128, 128, 16, dummy, 8, 2,
                            dummy, 0, 0, 0, 0, None, 0, 0, 0, 0, None, None)
    assert rc == _lib.FC_OK
    # png keep_m out of range
    rc = lib.fc_png_encode(dummy, _lib.FC_F32, 1, 1, 16, 16, 256, 256, 16, 8, 9,
                           dummy, 0, 0, 0, 0, dummy, 0, 0, 0, None)
    assert rc == _lib.FC_EINVAL
    # int8 codes without scales on the read path
    rc = lib.fc_jpeg_decode(dummy, _lib.FC_I8, 1, 1, 2, 16, 2, 0, 0, 0, 0, None, 0, 0, 0, 0,
                            dummy, 8, dummy, _lib.FC_F32, 16, 0, 0, 0, None)
    assert rc == _lib.FC_EINVAL


def _attn(lib, **kw):
    from flashcodec_b200 import _lib
    a = dict(q=ctypes.c_void_p(0x1000), q_dtype=_lib.FC_F32, B=1, Hq=4, D=64, q_sb=256, q_sh=64,
             Hk=2, n=4, s=2, r=8, rows_dtype=_lib.FC_I8, k=ctypes.c_void_p(0x2000),
             v=ctypes.c_void_p(0x3000), ks=ctypes.c_void_p(0x4000), vs=ctypes.c_void_p(0x5000),
             sc_dtype=_lib.FC_F32, n_raw=0, A=ctypes.c_void_p(0x6000),
             out=ctypes.c_void_p(0x7000), out_dtype=_lib.FC_F32, ws=None, ws_bytes=0)
    a.update(kw)
    return lib.fc_decode_attn(
        a["q"], a["q_dtype"], a["B"], a["Hq"], a["D"], a["q_sb"], a["q_sh"],
        a["Hk"], a["n"], a["s"], a["r"], a["rows_dtype"],
        a["k"], 0, 0, 0, 0, a["v"], 0, 0, 0, 0,
        a["ks"], 0, 0, 0, a["vs"], 0, 0, 0, a["sc_dtype"],
        None, 0, 0, 0, None, 0, 0, 0, _lib.FC_F32, a["n_raw"],
        a["A"], 0.125, a["out"], a["out_dtype"], 256, 64, a["ws"], a["ws_bytes"], None)


def test_attention_host_validation(lib):
    from flashcodec_b200 import _lib
    assert _attn(lib, Hq=3) == _lib.FC_EINVAL                  # GQA divisibility
    assert _attn(lib, D=512) == _lib.FC_ENOTSUP                # head dim > 256
    assert _attn(lib, ks=None) == _lib.FC_EINVAL               # int8 rows need scales
    assert _attn(lib, n_raw=8) == _lib.FC_EINVAL               # tail must be < r
    assert _attn(lib, n=0, n_raw=0) == _lib.FC_EINVAL          # empty: caller returns zeros
    assert _attn(lib) == _lib.FC_ERANGE                        # no workspace
    assert b"workspace" in lib.fc_last_error_string()


def test_workspace_size_is_host_only(lib):
    n = lib.fc_decode_attn_workspace_size(16, 32, 8, 128, 4096, 4, 8, 5)
    assert n >= 256
    # the partials: units * splits * G * (D + 2) floats at most a few percent
    # of the 553 MB archive of this shape (config 2, one layer)
    assert n < 0.05 * 553_648_128
    assert lib.fc_decode_attn_workspace_size(1, 3, 2, 64, 8, 2, 8, 0) == 0


def test_new_entry_points_validate_on_the_host(lib):
    """fc_decode_attn_png, fc_gather_batch and fc_selftest_bounded_wait refuse
    bad arguments before any CUDA call."""
    from flashcodec_b200 import _lib
    P = ctypes.c_void_p
    d = P(0x1000)
    # png attention: r < 2, and missing anchors
    for r, kanc in ((1, d), (8, None)):
        rc = lib.fc_decode_attn_png(d, _lib.FC_F32, 1, 4, 64, 256, 64, 2, 4, r,
                                    kanc, d, _lib.FC_F32, 0, 0, 0, d, d, 0, 0, 0, 0,
                                    None, 0, 0, 0, None, 0, 0, 0, _lib.FC_F32, 0,
                                    d, 0.125, d, _lib.FC_F32, 256, 64, None, 0, None)
        assert rc == _lib.FC_EINVAL
    # gather: null index, destination equal to the source, nothing to do
    assert lib.fc_gather_batch(d, 2, P(0x2000), 2, 2, 64, 256, 64, 256, 64, None,
                               None) == _lib.FC_EINVAL
    assert lib.fc_gather_batch(d, 2, d, 2, 2, 64, 256, 64, 256, 64, P(0x3000),
                               None) == _lib.FC_EINVAL
    assert lib.fc_gather_batch(d, 2, P(0x2000), 0, 2, 64, 256, 64, 256, 64, P(0x3000),
                               None) == _lib.FC_OK
    # self-test: null status, epoch <= 0
    assert lib.fc_selftest_bounded_wait(None, 1, None) == _lib.FC_EINVAL
    assert lib.fc_selftest_bounded_wait(d, 0, None) == _lib.FC_EINVAL
    # no-alloc status and its self-test: null destination, epoch <= 0
    assert lib.fc_decode_attn_noalloc_status(None, 1, None) == _lib.FC_EINVAL
    assert lib.fc_selftest_noalloc_wait(0, None) == _lib.FC_EINVAL


def test_grouped_entry_points_validate_on_the_host(lib):
    """The per-group format's entry points refuse a group size that does not
    divide the head dim (or is not a multiple of 4 for the archive) and a
    missing scale tensor before any CUDA call."""
    from flashcodec_b200 import _lib
    d = ctypes.c_void_p(0x1000)
    for group, sc in ((24, d), (6, d), (32, None)):
        rc = lib.fc_jpeg_encode_grouped(d, _lib.FC_BF16, 1, 2, 64, 128, 0, 0, 128, d, 8, 2,
                                        d, 0, 0, 0, 0, sc, _lib.FC_F32, group, 0, 0, 0, 0,
                                        None, None)
        assert rc == _lib.FC_EINVAL, group
    assert lib.fc_jpeg_decode_grouped(d, 1, 2, 8, 128, 2, 0, 0, 0, 0, d, _lib.FC_F32, 48,
                                      0, 0, 0, 0, d, 8, d, _lib.FC_BF16, 64, 0, 0, 0,
                                      None) == _lib.FC_EINVAL

    def attn(group, rows_scales=d):
        return lib.fc_decode_attn_grouped(
            d, _lib.FC_BF16, 1, 4, 128, 512, 128, 2, 8, 2, 8, d, 0, 0, 0, 0, d, 0, 0, 0, 0,
            rows_scales, 0, 0, 0, 0, rows_scales, 0, 0, 0, 0, _lib.FC_F32, group,
            None, 0, 0, 0, None, 0, 0, 0, _lib.FC_BF16, 0, d, 0.1, d, _lib.FC_BF16, 512, 128,
            None, 0, None)
    assert attn(0) == _lib.FC_EINVAL
    assert attn(48) == _lib.FC_EINVAL          # does not divide D
    assert attn(32, None) == _lib.FC_EINVAL    # int8 rows need scales


def test_rope_kv_append_validates_on_the_host(lib):
    """fc_rope_kv_append refuses odd head dims, integer dtypes, a v without
    v_out and outputs overlapping an input or each other before any CUDA call; empty work is a no-op."""
    from flashcodec_b200 import _lib
    P = ctypes.c_void_p
    q, qo, k, ko, v, vo, c, s = (P(0x1000 * (i + 1)) for i in range(8))

    def call(B=2, D=64, dt=_lib.FC_BF16, q_out=qo, v_=v, v_out=vo, Hq=4, Hk=2):
        return lib.fc_rope_kv_append(q, 256, 64, q_out, 256, 64, Hq, k, 128, 64, ko, 128, 64,
                                     v_, 128, 64, v_out, 128, 64, Hk, c, s, 64, dt, B, D, None)

    assert call(D=63) == _lib.FC_EINVAL
    assert b"odd" in lib.fc_last_error_string()
    assert call(dt=_lib.FC_I8) == _lib.FC_EINVAL
    assert call(v_out=None) == _lib.FC_EINVAL
    assert call(q_out=q) == _lib.FC_EINVAL
    assert call(q_out=P(0x1000 + 128)) == _lib.FC_EINVAL     # partial overlap with q
    assert b"overlap" in lib.fc_last_error_string()
    assert call(v_out=P(0x4000 + 64)) == _lib.FC_EINVAL      # v_out inside k_out's rows
    assert call(B=-1) == _lib.FC_EINVAL
    assert call(B=0) == _lib.FC_OK


def test_masked_attention_validates_on_the_host(lib):
    """fc_decode_attn_masked refuses a null mask and half-given png anchors."""
    from flashcodec_b200 import _lib
    P = ctypes.c_void_p
    d = P(0x1000)

    def call(vis=d, kanc=None, vanc=None):
        return lib.fc_decode_attn_masked(
            d, _lib.FC_F32, 1, 4, 64, 256, 64, 2, 4, 2, 8, _lib.FC_I8,
            d, 0, 0, 0, 0, d, 0, 0, 0, 0, d, 0, 0, 0, d, 0, 0, 0, _lib.FC_F32,
            None, 0, 0, 0, None, 0, 0, 0, _lib.FC_F32, 0,
            d, 0.125, d, _lib.FC_F32, 256, 64, None, 0,
            kanc, vanc, _lib.FC_F32, 0, 0, 0, vis, 64, None)

    assert call(vis=None) == _lib.FC_EINVAL
    assert b"visibility" in lib.fc_last_error_string()
    assert call(kanc=d) == _lib.FC_EINVAL
    assert call() == _lib.FC_ERANGE          # valid so far; no workspace given


def test_peer_entry_points_validate_on_the_host(lib):
    """fc_decode_attn_peers, fc_peers_wait and the IPC calls refuse bad
    tables and pointers before any launch; a valid table on a layout the
    tensor-core kernel does not take (head dim 64) is refused as unsupported."""
    from flashcodec_b200 import _lib
    P = ctypes.c_void_p
    d = P(0x1000)

    def table(world=2, rank=0, epoch=1, out=0x7000, recv1=0x8000, counter=None):
        t = _lib.PeerOut()
        t.out, t.world, t.rank, t.epoch = out, world, rank, epoch
        t.recv[1] = recv1
        t.counter = counter
        return t

    def attn(t, D=64):
        return lib.fc_decode_attn_peers(
            d, _lib.FC_F32, 1, 4, D, 4 * D, D, 2, 4, 2, 8, _lib.FC_I8,
            d, 0, 0, 0, 0, d, 0, 0, 0, 0, d, 0, 0, 0, d, 0, 0, 0, _lib.FC_F32,
            None, 0, 0, 0, None, 0, 0, 0, _lib.FC_F32, 0,
            d, 0.125, _lib.FC_F32, 4 * D, D, None if t is None else ctypes.byref(t),
            None, 0, None)

    assert attn(None) == _lib.FC_EINVAL
    assert attn(table(world=0)) == _lib.FC_EINVAL
    assert attn(table(world=9)) == _lib.FC_EINVAL
    assert attn(table(rank=2)) == _lib.FC_EINVAL
    assert attn(table(epoch=0)) == _lib.FC_EINVAL               # no epoch and no counter
    assert attn(table(out=0)) == _lib.FC_EINVAL
    assert attn(table(recv1=0)) == _lib.FC_EINVAL
    assert attn(table(recv1=0x8004)) == _lib.FC_EINVAL          # receive words are 8 bytes
    assert attn(table(epoch=0, counter=0x9000)) == _lib.FC_ENOTSUP   # valid, head dim 64
    assert b"tensor-core" in lib.fc_last_error_string()
    assert attn(table()) == _lib.FC_ENOTSUP

    w = lib.fc_peers_wait
    assert w(None, d, 2, 0, 16, 1, None, None, None) == _lib.FC_EINVAL
    assert w(d, None, 2, 0, 16, 1, None, None, None) == _lib.FC_EINVAL
    assert w(d, d, 9, 0, 16, 1, None, None, None) == _lib.FC_EINVAL
    assert w(d, d, 2, 2, 16, 1, None, None, None) == _lib.FC_EINVAL
    assert w(d, d, 2, 0, 16, 0, None, None, None) == _lib.FC_EINVAL
    assert w(P(0x1004), d, 2, 0, 16, 1, None, None, None) == _lib.FC_EINVAL
    h = ctypes.create_string_buffer(_lib.FC_IPC_HANDLE_BYTES)
    off = ctypes.c_int64(0)
    assert lib.fc_ipc_get_handle(None, h, ctypes.byref(off)) == _lib.FC_EINVAL
    assert lib.fc_ipc_open_handle(None, ctypes.byref(P())) == _lib.FC_EINVAL
    assert lib.fc_ipc_close_handle(None) == _lib.FC_EINVAL
