"""ctypes binding of libflashcodec_sm100.so (include/flashcodec_b200.h).

The shared library is built in-tree by ``python -m flashcodec_b200.build``.
There is no fallback: if the library is missing or cannot be loaded every
kernel call raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libflashcodec_sm100.so"

FC_OK, FC_EINVAL, FC_ECUDA, FC_ERANGE, FC_ENOTSUP = 0, 1, 2, 3, 4
FC_F32, FC_BF16, FC_F16, FC_I8 = 0, 1, 2, 3

# exported symbols, in header order (tests check the library exports them all)
SYMBOLS = ("fc_version", "fc_last_error_string", "fc_jpeg_encode", "fc_jpeg_decode",
           "fc_jpeg_encode_grouped", "fc_jpeg_decode_grouped", "fc_png_encode", "fc_png_decode", "fc_decode_attn_workspace_size",
           "fc_decode_attn", "fc_decode_attn_grouped", "fc_decode_attn_png",
           "fc_decode_attn_noalloc",
           "fc_decode_attn_noalloc_status", "fc_append_tokens", "fc_gather_batch", "fc_rope_kv_append", "fc_decode_attn_masked",
           "fc_set_attn_kernel",
           "fc_selftest_bounded_wait", "fc_selftest_noalloc_wait", "fc_decode_attn_peers",
           "fc_peers_wait", "fc_ipc_get_handle", "fc_ipc_open_handle", "fc_ipc_close_handle")
FC_MAX_PEERS, FC_IPC_HANDLE_BYTES = 8, 64
FC_ATTN_AUTO, FC_ATTN_CUDA_CORE, FC_ATTN_TENSOR_CORE = 0, 1, 2

_I64, _I32, _P, _F32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float


class PeerOut(ctypes.Structure):
    """fc_peer_out: this rank's output piece and every rank's receive area of a
    split-head step."""
    _fields_ = [("out", ctypes.c_void_p), ("recv", ctypes.c_void_p * 8),
                ("world", ctypes.c_int), ("rank", ctypes.c_int), ("epoch", ctypes.c_int),
                ("counter", ctypes.c_void_p)]


class AppendStream(ctypes.Structure):
    """fc_append_stream: one K or V stream of one layer in fc_append_tokens."""
    _fields_ = [("token", _P), ("token_sb", _I64), ("token_sh", _I64), ("raw", _P),
                ("codes", _P), ("scales", _P), ("capacity", _I64), ("err", _P)]


_SIGS = {
    "fc_version": ([], ctypes.c_char_p),
    "fc_last_error_string": ([], ctypes.c_char_p),
    "fc_jpeg_encode": ([_P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I32, _I32,
                        _P, _I64, _I64, _I64, _I64, _P, _I32, _I64, _I64, _I64, _P, _P], _I32),
    "fc_jpeg_decode": ([_P, _I32, _I64, _I64, _I64, _I64, _I32, _I64, _I64, _I64, _I64,
                        _P, _I32, _I64, _I64, _I64, _P, _I32, _P, _I32, _I64, _I64, _I64,
                        _I64, _P], _I32),
    "fc_jpeg_encode_grouped": ([_P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I32,
                                _I32, _P, _I64, _I64, _I64, _I64, _P, _I32, _I32, _I64, _I64,
                                _I64, _I64, _P, _P], _I32),
    "fc_jpeg_decode_grouped": ([_P, _I64, _I64, _I64, _I64, _I32, _I64, _I64, _I64, _I64, _P,
                                _I32, _I32, _I64, _I64, _I64, _I64, _P, _I32, _P, _I32, _I64,
                                _I64, _I64, _I64, _P], _I32),
    "fc_png_encode": ([_P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32,
                       _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P], _I32),
    "fc_png_decode": ([_P, _I64, _I64, _I64, _I64, _P, _I32, _I64, _I64, _I64,
                       _I64, _I64, _I64, _I32, _I64, _P, _I64, _I64, _I64, _I64, _P], _I32),
    "fc_decode_attn_workspace_size": ([_I64, _I64, _I64, _I64, _I64, _I32, _I32, _I64],
                                      ctypes.c_size_t),
    "fc_decode_attn": ([_P, _I32, _I64, _I64, _I64, _I64, _I64,
                        _I64, _I64, _I32, _I32, _I32,
                        _P, _I64, _I64, _I64, _I64,
                        _P, _I64, _I64, _I64, _I64,
                        _P, _I64, _I64, _I64,
                        _P, _I64, _I64, _I64,
                        _I32,
                        _P, _I64, _I64, _I64,
                        _P, _I64, _I64, _I64,
                        _I32, _I64,
                        _P, _F32,
                        _P, _I32, _I64, _I64,
                        _P, ctypes.c_size_t, _P], _I32),
    "fc_decode_attn_grouped": ([_P, _I32, _I64, _I64, _I64, _I64, _I64,
                                _I64, _I64, _I32, _I32,
                                _P, _I64, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64, _I64,
                                _I32, _I32,
                                _P, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64,
                                _I32, _I64,
                                _P, _F32,
                                _P, _I32, _I64, _I64,
                                _P, ctypes.c_size_t, _P], _I32),
    "fc_decode_attn_png": ([_P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I32,
                            _P, _P, _I32, _I64, _I64, _I64,
                            _P, _P, _I64, _I64, _I64, _I64,
                            _P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I32, _I64,
                            _P, _F32, _P, _I32, _I64, _I64, _P, ctypes.c_size_t, _P], _I32),
    "fc_decode_attn_noalloc": ([_P, _I32, _I64, _I64, _I64, _I64, _I64,
                                _I64, _I64, _I32, _I32, _I32,
                                _P, _I64, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64,
                                _I32,
                                _P, _I64, _I64, _I64,
                                _P, _I64, _I64, _I64,
                                _I32, _I64,
                                _P, _F32,
                                _P, _I32, _I64, _I64, _P], _I32),
    "fc_decode_attn_noalloc_status": ([_P, _I32, _P], _I32),
    "fc_append_tokens": ([_P, _I32, _I32, _I64, _I64, _I64, _I32, _I32, _I64, _I64, _P, _I32,
                          _P], _I32),
    "fc_gather_batch": ([_P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P], _I32),
    "fc_rope_kv_append": ([_P, _I64, _I64, _P, _I64, _I64, _I64,
                           _P, _I64, _I64, _P, _I64, _I64,
                           _P, _I64, _I64, _P, _I64, _I64, _I64,
                           _P, _P, _I64,
                           _I32, _I64, _I64, _P], _I32),
    "fc_decode_attn_masked": ([_P, _I32, _I64, _I64, _I64, _I64, _I64,
                               _I64, _I64, _I32, _I32, _I32,
                               _P, _I64, _I64, _I64, _I64,
                               _P, _I64, _I64, _I64, _I64,
                               _P, _I64, _I64, _I64,
                               _P, _I64, _I64, _I64,
                               _I32,
                               _P, _I64, _I64, _I64,
                               _P, _I64, _I64, _I64,
                               _I32, _I64,
                               _P, _F32,
                               _P, _I32, _I64, _I64, _P, ctypes.c_size_t,
                               _P, _P, _I32, _I64, _I64, _I64,
                               _P, _I64, _P], _I32),
    "fc_set_attn_kernel": ([_I32], _I32),
    "fc_selftest_bounded_wait": ([_P, _I32, _P], _I32),
    "fc_selftest_noalloc_wait": ([_I32, _P], _I32),
    "fc_decode_attn_peers": ([_P, _I32, _I64, _I64, _I64, _I64, _I64,
                              _I64, _I64, _I32, _I32, _I32,
                              _P, _I64, _I64, _I64, _I64,
                              _P, _I64, _I64, _I64, _I64,
                              _P, _I64, _I64, _I64,
                              _P, _I64, _I64, _I64,
                              _I32,
                              _P, _I64, _I64, _I64,
                              _P, _I64, _I64, _I64,
                              _I32, _I64,
                              _P, _F32,
                              _I32, _I64, _I64, _P,
                              _P, ctypes.c_size_t, _P], _I32),
    "fc_peers_wait": ([_P, _P, _I32, _I32, _I64, _I32, _P, _P, _P], _I32),
    "fc_ipc_get_handle": ([_P, _P, _P], _I32),
    "fc_ipc_open_handle": ([_P, _P], _I32),
    "fc_ipc_close_handle": ([_P], _I32),
}

_lock = threading.Lock()
_lib = None


class FlashCodecError(RuntimeError):
    """A kernel call returned a nonzero status (see include/flashcodec_b200.h)."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load the kernel library (once).  Raises RuntimeError if it is absent."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p.name} is not built; run `python -m flashcodec_b200.build` "
                "(flashcodec_b200 has no non-CUDA implementation)")
        lib = ctypes.CDLL(str(p))
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if path is None:
            _lib = lib
        return lib


def check(status: int, what: str) -> None:
    """Map a C status to the exception types the reference raises."""
    if status == FC_OK:
        return
    msg = load().fc_last_error_string().decode(errors="replace") or what
    if status == FC_EINVAL:
        raise ValueError(msg)
    if status == FC_ENOTSUP:
        raise NotImplementedError(msg)
    raise FlashCodecError(status, msg)


def version() -> str:
    return load().fc_version().decode()
