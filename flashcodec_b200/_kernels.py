"""Tensor-level wrappers around the C ABI (one function per entry point).

Every wrapper checks that its tensors live on a CUDA device, passes data
pointers, element strides and the current CUDA stream of that device, and maps
a nonzero status to an exception.  No wrapper computes anything itself.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

DTYPE_CODE = {torch.float32: _lib.FC_F32, torch.bfloat16: _lib.FC_BF16,
              torch.float16: _lib.FC_F16, torch.int8: _lib.FC_I8}


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "flashcodec_b200 runs on CUDA devices only (got a tensor on "
                f"{t.device}); there is no CPU implementation")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def as_bhsd(x: torch.Tensor) -> torch.Tensor:
    """View (..., S, D) as (B, H, S, D) with unit stride on D (copying only
    when the layout cannot be expressed)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    if x.dim() == 4:
        return x
    if x.dim() == 2:
        return x[None, None]
    if x.dim() == 3:
        return x[None]
    lead = math.prod(x.shape[:-2])
    return x.reshape(1, lead, x.shape[-2], x.shape[-1])


def _unit_last(*tensors) -> None:
    """The kernels index the last dim with unit stride (the ABI carries the
    strides of the other dims only)."""
    for t in tensors:
        if t is not None and t.dim() > 0 and t.shape[-1] > 1 and t.stride(-1) != 1:
            raise ValueError("the last dimension must be contiguous (stride 1)")


def _s(t, *dims):
    return [t.stride(d) for d in dims]


# ----------------------------------------------------------------- jpeg codec
def jpeg_encode(x: torch.Tensor, basis: torch.Tensor, r: int, k: int, out: torch.Tensor,
                scales: torch.Tensor | None = None, err: torch.Tensor | None = None) -> None:
    """x (B,H,S,D) -> out (B,H,n,k,D) [int8 codes with scales (B,H,n,k,1) | coefficients]."""
    require_cuda(x, basis, out, scales)
    _unit_last(x, out)
    B, H, S, D = x.shape
    if (scales is None) != (out.dtype != torch.int8):
        raise ValueError("int8 output needs scales; float output takes none")
    st = _stream(x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().fc_jpeg_encode(
            _p(x), dtype_code(x), B, H, S, D, *_s(x, 0, 1, 2),
            _p(basis), r, k,
            _p(out), *_s(out, 0, 1, 2, 3),
            _p(scales), dtype_code(scales) if scales is not None else 0,
            *(_s(scales, 0, 1, 2) if scales is not None else (0, 0, 0)),
            _p(err), st)
    _lib.check(rc, "jpeg_encode")


def jpeg_decode(coef: torch.Tensor, scales: torch.Tensor | None, basis: torch.Tensor, r: int,
                out: torch.Tensor, out_len: int) -> None:
    """coef (B,H,n,k,D) [+ scales (B,H,n,k,1)] -> out (B,H,>=out_len,D)."""
    require_cuda(coef, scales, basis, out)
    _unit_last(coef, out)
    B, H, n, k, D = coef.shape
    st = _stream(coef.device)
    with torch.cuda.device(coef.device):
        rc = _lib.load().fc_jpeg_decode(
            _p(coef), dtype_code(coef), B, H, n, D, k, *_s(coef, 0, 1, 2, 3),
            _p(scales), dtype_code(scales) if scales is not None else 0,
            *(_s(scales, 0, 1, 2) if scales is not None else (0, 0, 0)),
            _p(basis), r, _p(out), dtype_code(out), out_len, *_s(out, 0, 1, 2), st)
    _lib.check(rc, "jpeg_decode")


# ------------------------------------------------------------------ png codec
def png_encode(x: torch.Tensor, r: int, keep_m: int, deltas: torch.Tensor,
               anchors: torch.Tensor) -> None:
    """x (B,H,S,D) -> deltas (B,H,n,r-1,D) fp32, anchors (B,H,n,D) in x.dtype."""
    require_cuda(x, deltas, anchors)
    _unit_last(x, deltas, anchors)
    B, H, S, D = x.shape
    st = _stream(x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().fc_png_encode(
            _p(x), dtype_code(x), B, H, S, D, *_s(x, 0, 1, 2), r, keep_m,
            _p(deltas), *_s(deltas, 0, 1, 2, 3), _p(anchors), *_s(anchors, 0, 1, 2), st)
    _lib.check(rc, "png_encode")


def png_decode(deltas: torch.Tensor, anchors: torch.Tensor, out: torch.Tensor,
               out_len: int) -> None:
    """deltas (B,H,n,r-1,D) fp32 + anchors (B,H,n,D) -> out (B,H,>=out_len,D)."""
    require_cuda(deltas, anchors, out)
    _unit_last(deltas, anchors, out)
    B, H, n, rm1, D = deltas.shape
    st = _stream(deltas.device)
    with torch.cuda.device(deltas.device):
        rc = _lib.load().fc_png_decode(
            _p(deltas), *_s(deltas, 0, 1, 2, 3), _p(anchors), dtype_code(anchors),
            *_s(anchors, 0, 1, 2), B, H, n, rm1 + 1, D, _p(out), out_len, *_s(out, 0, 1, 2), st)
    _lib.check(rc, "png_decode")


# ------------------------------------------------------------------ attention
_workspaces: dict = {}


def attn_workspace_bytes(B, Hq, Hk, D, n_blocks, s, r, n_raw) -> int:
    return int(_lib.load().fc_decode_attn_workspace_size(B, Hq, Hk, D, n_blocks, s, r, n_raw))


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised workspace cached per (device, stream).  The kernel
    leaves its counters at zero, so the buffer is reused across calls issued
    on the same stream."""
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def reset_workspace(device: torch.device) -> None:
    """Zero the cached workspace of the current stream (after a failed call)."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    if key in _workspaces:
        _workspaces[key].zero_()


def attn_status(device: torch.device) -> int:
    """The workspace status word of the current stream (synchronises)."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _workspaces.get(key)
    return 0 if ws is None else int(ws[:4].view(torch.int32).item())


class StatusProbe:
    """A copy of an attention status word in flight to pinned host memory.

    0 means every decode-attention call on that stream's workspace since the
    last reset produced valid output; a positive value is the launch number of
    a call whose bounded wait gave up (its output is invalid)."""

    def __init__(self, host: torch.Tensor, event: torch.cuda.Event | None):
        self._host, self._event = host, event

    def ready(self) -> bool:
        """True once the copy has landed (never blocks)."""
        return self._event is None or self._event.query()

    def value(self) -> int:
        """The status word (waits for the copy only, not for later work)."""
        if self._event is not None:
            self._event.synchronize()
        return int(self._host[0])

    def check(self) -> None:
        """Raise FlashCodecError if a call gave up."""
        v = self.value()
        if v:
            raise _lib.FlashCodecError(
                _lib.FC_ECUDA, f"decode attention launch {v} gave up waiting for a staged "
                "tile (bounded wait); its output is invalid")


def attn_status_async(device: torch.device, reset: bool = False) -> StatusProbe:
    """Queue a copy of the current stream's workspace status word to pinned
    host memory, in stream order, without synchronising; reset=True clears the
    word after the copy.  Poll the probe after a model step."""
    stream = torch.cuda.current_stream(device)
    ws = _workspaces.get((device.index, stream.cuda_stream))
    host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    if ws is None:
        return StatusProbe(host, None)
    word = ws[:4].view(torch.int32)
    host.copy_(word, non_blocking=True)
    if reset:
        word.zero_()
    ev = torch.cuda.Event()
    ev.record(stream)
    return StatusProbe(host, ev)


def set_attn_kernel(which: str) -> str:
    """Select the decode-attention kernel process-wide: "auto" (tensor cores
    whenever the archive allows, the default), "cuda-core" or "tensor-core".
    Returns the previous selection.  For tests and benchmarks."""
    codes = {"auto": _lib.FC_ATTN_AUTO, "cuda-core": _lib.FC_ATTN_CUDA_CORE,
             "tensor-core": _lib.FC_ATTN_TENSOR_CORE}
    if which not in codes:
        raise ValueError(f"unknown attention kernel {which!r}")
    prev = _lib.load().fc_set_attn_kernel(codes[which])
    return {v: k for k, v in codes.items()}[prev]


def _visible(vis, B, L):
    """(B, >= L) key-visibility bytes -> (tensor, batch stride)."""
    require_cuda(vis)
    if vis.dtype not in (torch.bool, torch.uint8) or vis.dim() != 2 or vis.shape[0] != B \
            or vis.shape[1] < L or (L > 1 and vis.stride(1) != 1):
        raise ValueError(f"visible must be a (B={B}, >= {L}) bool/uint8 tensor with unit "
                         "stride along the keys")
    return vis, vis.stride(0)


def decode_attn_png(q, kanc, vanc, kdel, vdel, kraw, vraw, A, scale, out, vis=None) -> None:
    """png archive read in place: anchors (B,Hk,n,D) as row 0 of every block,
    fp32 deltas (B,Hk,n,r-1,D) as rows 1..r-1; A (r,r) tril(ones).  vis:
    optional (B, n*r + t) key visibility (fc_decode_attn_masked)."""
    require_cuda(q, kanc, vanc, kdel, vdel, kraw, vraw, A, out)
    _unit_last(kanc, vanc, kdel, vdel)
    if kanc.stride() != vanc.stride() or kdel.stride() != vdel.stride():
        raise ValueError("K and V png archives must share one layout")
    B, Hq, _, D = q.shape
    Hk, n, rm1 = kdel.shape[1], kdel.shape[2], kdel.shape[3]
    r = rm1 + 1
    t = kraw.shape[2] if kraw is not None else 0
    ws = workspace(q.device, attn_workspace_bytes(B, Hq, Hk, D, n, r, r, t))
    z3 = (0, 0, 0)
    st = _stream(q.device)
    if vis is not None:
        vis, vis_sb = _visible(vis, B, n * r + t)
        with torch.cuda.device(q.device):
            rc = _lib.load().fc_decode_attn_masked(
                _p(q), dtype_code(q), B, Hq, D, q.stride(0), q.stride(1), Hk, n, r, r,
                _lib.FC_F32, _p(kdel), *_s(kdel, 0, 1, 2, 3), _p(vdel), *_s(vdel, 0, 1, 2, 3),
                None, 0, 0, 0, None, 0, 0, 0, _lib.FC_F32,
                _p(kraw), *(_s(kraw, 0, 1, 2) if kraw is not None else z3),
                _p(vraw), *(_s(vraw, 0, 1, 2) if vraw is not None else z3),
                dtype_code(kraw) if kraw is not None else 0, t,
                _p(A), float(scale), _p(out), dtype_code(out), out.stride(0), out.stride(1),
                _p(ws), ws.numel(), _p(kanc), _p(vanc), dtype_code(kanc), *_s(kanc, 0, 1, 2),
                _p(vis), vis_sb, st)
        if rc != _lib.FC_OK:
            reset_workspace(q.device)
        _lib.check(rc, "decode_attn_masked")
        return
    with torch.cuda.device(q.device):
        rc = _lib.load().fc_decode_attn_png(
            _p(q), dtype_code(q), B, Hq, D, q.stride(0), q.stride(1), Hk, n, r,
            _p(kanc), _p(vanc), dtype_code(kanc), *_s(kanc, 0, 1, 2),
            _p(kdel), _p(vdel), *_s(kdel, 0, 1, 2, 3),
            _p(kraw), *(_s(kraw, 0, 1, 2) if kraw is not None else z3),
            _p(vraw), *(_s(vraw, 0, 1, 2) if vraw is not None else z3),
            dtype_code(kraw) if kraw is not None else 0, t,
            _p(A), float(scale), _p(out), dtype_code(out), out.stride(0), out.stride(1),
            _p(ws), ws.numel(), st)
    if rc != _lib.FC_OK:
        reset_workspace(q.device)
    _lib.check(rc, "decode_attn_png")


def gather_batch(src: torch.Tensor, idx: torch.Tensor, live: int) -> torch.Tensor:
    """New tensor like src (B_src, H, L, ...) with batch rows src[idx[b]]:
    the first `live` entries of dim 2 are gathered (the rest is left
    uninitialised, as beyond a stream's live length).  idx: int64 on
    src.device, values in [0, B_src)."""
    require_cuda(src, idx)
    if not src.is_contiguous():
        raise ValueError("gather_batch needs a contiguous source")
    B_src, H = src.shape[0], src.shape[1]
    if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= B_src):
        raise IndexError(f"batch index out of range for {B_src} rows")
    dst = torch.empty((idx.numel(),) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row = src[0, 0, 0].numel() * src.element_size() if src.dim() > 2 else src.element_size()
    slab = live * row
    st = _stream(src.device)
    with torch.cuda.device(src.device):
        rc = _lib.load().fc_gather_batch(
            _p(src), B_src, _p(dst), idx.numel(), H, slab,
            src.stride(0) * src.element_size(), src.stride(1) * src.element_size(),
            dst.stride(0) * dst.element_size(), dst.stride(1) * dst.element_size(),
            _p(idx), st)
    _lib.check(rc, "gather_batch")
    return dst


def _rows3(x: torch.Tensor, name: str) -> torch.Tensor:
    """(B, H, D) view of a one-token (B, H, D) or (B, H, 1, D) tensor."""
    if x.dim() == 4:
        if x.shape[2] != 1:
            raise ValueError(f"{name}: one token per sequence expected, got {tuple(x.shape)}")
        x = x[:, :, 0]
    if x.dim() != 3:
        raise ValueError(f"{name}: expected (B, H, D) or (B, H, 1, D), got {tuple(x.shape)}")
    if x.shape[-1] > 1 and x.stride(-1) != 1:
        raise ValueError(f"{name}: the head dim must have unit stride")
    return x


def rope_kv_append(q, k, v, cos, sin, q_out, k_out, v_out=None) -> None:
    """Rotary embedding of one token's q and k (rotate-half form) written to
    q_out and k_out, and v copied to v_out, in one launch (fc_rope_kv_append).
    q/q_out (B,Hq[,1],D); k, v, k_out, v_out (B,Hk[,1],D) (outputs may be
    strided views such as a raw-tail slot); cos/sin (B or 1, [1, [1,]] D).
    All one dtype; v and v_out are optional together."""
    require_cuda(q, k, v, cos, sin, q_out, k_out, v_out)
    q, q_out = _rows3(q, "q"), _rows3(q_out, "q_out")
    k, k_out = _rows3(k, "k"), _rows3(k_out, "k_out")
    if (v is None) != (v_out is None):
        raise ValueError("v and v_out go together")
    if v is not None:
        v, v_out = _rows3(v, "v"), _rows3(v_out, "v_out")
    B, Hq, D = q.shape
    Hk = k.shape[1]
    tensors = [q, k, cos, sin, q_out, k_out] + ([v, v_out] if v is not None else [])
    if len({t.dtype for t in tensors}) != 1:
        raise ValueError("rope_kv_append: every tensor must have one dtype")
    if q_out.shape != q.shape or k_out.shape != k.shape or k.shape[0] != B or k.shape[2] != D \
            or (v is not None and (v.shape != k.shape or v_out.shape != k.shape)):
        raise ValueError("rope_kv_append: shape mismatch")
    cs = [c.reshape(-1, c.shape[-1]) for c in (cos, sin)]
    if cs[0].shape != cs[1].shape or cs[0].shape[-1] != D or cs[0].shape[0] not in (1, B) \
            or cs[0].stride(-1) != 1 or cs[0].stride(0) != cs[1].stride(0):
        raise ValueError("rope_kv_append: cos/sin must be (B or 1, D) rows of the head dim")
    cs_sb = cs[0].stride(0) if cs[0].shape[0] == B and B > 1 else 0
    z = (None, 0, 0, None, 0, 0)
    vv = (_p(v), v.stride(0), v.stride(1), _p(v_out), v_out.stride(0), v_out.stride(1)) \
        if v is not None else z
    with torch.cuda.device(q.device):
        rc = _lib.load().fc_rope_kv_append(
            _p(q), q.stride(0), q.stride(1), _p(q_out), q_out.stride(0), q_out.stride(1), Hq,
            _p(k), k.stride(0), k.stride(1), _p(k_out), k_out.stride(0), k_out.stride(1),
            *vv, Hk, _p(cs[0]), _p(cs[1]), cs_sb, dtype_code(q), B, D, _stream(q.device))
    _lib.check(rc, "rope_kv_append")


def selftest_bounded_wait(status: torch.Tensor, epoch: int) -> None:
    """Launch the bounded-wait self-test on status's device: it gives up after
    the kernels' wait limit and records `epoch` in status (int32, 1 element)."""
    require_cuda(status)
    with torch.cuda.device(status.device):
        rc = _lib.load().fc_selftest_bounded_wait(_p(status), int(epoch), _stream(status.device))
    _lib.check(rc, "selftest_bounded_wait")


def _attn_args(q, krows, vrows, kscales, vscales, kraw, vraw, A, scale, ws):
    """The arguments every decode-attention entry point shares, up to the
    softmax scale, and the workspace to pass (cached one when ws is None)."""
    require_cuda(q, krows, vrows, kscales, vscales, kraw, vraw, A)
    B, Hq, _, D = q.shape
    n = krows.shape[2] if krows is not None else 0
    s = krows.shape[3] if krows is not None else 1
    r = A.shape[0] if A is not None else 1
    Hk = (krows if krows is not None else kraw).shape[1]
    t = kraw.shape[2] if kraw is not None else 0
    need = attn_workspace_bytes(B, Hq, Hk, D, n, s, r, t)
    if ws is None:
        ws = workspace(q.device, need)
    z = (0, 0, 0, 0)
    args = (_p(q), dtype_code(q), B, Hq, D, q.stride(0), q.stride(1),
            Hk, n, s, r, dtype_code(krows) if krows is not None else 0,
            _p(krows), *(_s(krows, 0, 1, 2, 3) if krows is not None else z),
            _p(vrows), *(_s(vrows, 0, 1, 2, 3) if vrows is not None else z),
            _p(kscales), *(_s(kscales, 0, 1, 2) if kscales is not None else z[:3]),
            _p(vscales), *(_s(vscales, 0, 1, 2) if vscales is not None else z[:3]),
            dtype_code(kscales) if kscales is not None else 0,
            _p(kraw), *(_s(kraw, 0, 1, 2) if kraw is not None else z[:3]),
            _p(vraw), *(_s(vraw, 0, 1, 2) if vraw is not None else z[:3]),
            dtype_code(kraw) if kraw is not None else 0, t,
            _p(A), float(scale))
    return args, ws, n, r, t


def decode_attn(q, krows, vrows, kscales, vscales, kraw, vraw, A, scale, out,
                ws: torch.Tensor | None = None, vis=None) -> None:
    """q (B,Hq,1,D); krows/vrows (B,Hk,n,s,D) or None; k/vscales (B,Hk,n,s,1)
    or None; kraw/vraw (B,Hk,t,D) or None; A (r,s) fp32; out (B,Hq,1,D);
    vis: optional (B, n*r + t) key visibility (fc_decode_attn_masked)."""
    require_cuda(out)
    B = q.shape[0]
    head, ws, n, r, t = _attn_args(q, krows, vrows, kscales, vscales, kraw, vraw, A, scale, ws)
    args = head + (_p(out), dtype_code(out), out.stride(0), out.stride(1), _p(ws), ws.numel())
    st = _stream(q.device)
    with torch.cuda.device(q.device):
        if vis is None:
            rc = _lib.load().fc_decode_attn(*args, st)
        else:
            vis, vis_sb = _visible(vis, B, n * r + t)
            rc = _lib.load().fc_decode_attn_masked(*args, None, None, 0, 0, 0, 0,
                                                   _p(vis), vis_sb, st)
    if rc != _lib.FC_OK:
        reset_workspace(q.device)
    _lib.check(rc, "decode_attn")


def decode_attn_peers(q, krows, vrows, kscales, vscales, kraw, vraw, A, scale, out_dtype,
                      o_sb: int, o_sh: int, peers, ws: torch.Tensor | None = None) -> None:
    """fc_decode_attn_peers: the decode attention of this rank's KV heads with
    every output row stored into each rank's buffer (peers: a _lib.PeerOut
    whose out[p] are pre-offset to this rank's piece, strides o_sb, o_sh in
    elements); the launch then publishes peers.epoch in every rank's flags."""
    head, ws, _, _, _ = _attn_args(q, krows, vrows, kscales, vscales, kraw, vraw, A, scale, ws)
    with torch.cuda.device(q.device):
        rc = _lib.load().fc_decode_attn_peers(*head, DTYPE_CODE[out_dtype], o_sb, o_sh,
                                              ctypes.byref(peers), _p(ws), ws.numel(),
                                              _stream(q.device))
    if rc != _lib.FC_OK:
        reset_workspace(q.device)
    _lib.check(rc, "decode_attn_peers")


def peers_wait(recv: torch.Tensor, out: torch.Tensor, world: int, rank: int, piece_words: int,
               epoch: int, status: torch.Tensor | None,
               counter: torch.Tensor | None = None) -> None:
    """Queue fc_peers_wait on the current stream: wait (bounded) for the
    other ranks' pieces in this rank's receive area `recv` (world pieces of
    piece_words 8-byte words) and unpack them into `out` (rank p's piece at
    byte 4 * p * piece_words); a wait that gives up writes the epoch to
    status.  With `counter` (device int32) the epoch is counter + 1, read on
    the device, and the wait advances the counter."""
    require_cuda(recv, out, counter)
    with torch.cuda.device(recv.device):
        rc = _lib.load().fc_peers_wait(_p(recv), _p(out), world, rank, piece_words, epoch,
                                       _p(counter), _p(status), _stream(recv.device))
    _lib.check(rc, "peers_wait")


def ipc_get_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """(CUDA IPC handle of the allocation holding t, t's byte offset in it)."""
    require_cuda(t)
    h = ctypes.create_string_buffer(_lib.FC_IPC_HANDLE_BYTES)
    off = ctypes.c_int64(0)
    with torch.cuda.device(t.device):
        rc = _lib.load().fc_ipc_get_handle(_p(t), h, ctypes.byref(off))
    _lib.check(rc, "ipc_get_handle")
    return h.raw, off.value


def ipc_open(handle: bytes, device: torch.device) -> int:
    """Map another process's allocation on `device`; returns its base address."""
    base = ctypes.c_void_p(0)
    with torch.cuda.device(device):
        rc = _lib.load().fc_ipc_open_handle(ctypes.create_string_buffer(handle, len(handle)),
                                            ctypes.byref(base))
    _lib.check(rc, "ipc_open_handle")
    return int(base.value)


def ipc_close(base: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        rc = _lib.load().fc_ipc_close_handle(ctypes.c_void_p(base))
    _lib.check(rc, "ipc_close_handle")


# ------------------------------------------------------------ one-launch append
def append_tokens(table, n: int, dtype: torch.dtype, B: int, H: int, D: int, r: int, k: int,
                  slot: int, block: int, basis: torch.Tensor | None, scale_dtype,
                  device: torch.device) -> None:
    """fc_append_tokens over the first n entries of a ctypes AppendStream
    array (one entry per K or V stream; the caller fills it)."""
    sd = DTYPE_CODE.get(scale_dtype, 0) if scale_dtype is not None else 0
    with torch.cuda.device(device):
        rc = _lib.load().fc_append_tokens(
            ctypes.cast(table, ctypes.c_void_p), n, DTYPE_CODE[dtype], B, H, D, r, k, slot,
            block, _p(basis), sd, _stream(device))
    _lib.check(rc, "append_tokens")


# ------------------------------------------------------- per-group scale format
def jpeg_encode_grouped(x: torch.Tensor, basis: torch.Tensor, r: int, k: int, out: torch.Tensor,
                        scales: torch.Tensor, group: int, err: torch.Tensor | None = None) -> None:
    """x (B,H,S,D) -> int8 codes out (B,H,n,k,D) with one scale per `group`
    channels, scales (B,H,n,k,D//group) (fc_jpeg_encode_grouped)."""
    require_cuda(x, basis, out, scales)
    _unit_last(x, out, scales)
    B, H, S, D = x.shape
    with torch.cuda.device(x.device):
        rc = _lib.load().fc_jpeg_encode_grouped(
            _p(x), dtype_code(x), B, H, S, D, *_s(x, 0, 1, 2), _p(basis), r, k,
            _p(out), *_s(out, 0, 1, 2, 3), _p(scales), dtype_code(scales), int(group),
            *_s(scales, 0, 1, 2, 3), _p(err), _stream(x.device))
    _lib.check(rc, "jpeg_encode_grouped")


def jpeg_decode_grouped(codes: torch.Tensor, scales: torch.Tensor, group: int,
                        basis: torch.Tensor, r: int, out: torch.Tensor, out_len: int) -> None:
    """int8 codes (B,H,n,k,D) + scales (B,H,n,k,D//group) -> out (B,H,>=out_len,D)."""
    require_cuda(codes, scales, basis, out)
    _unit_last(codes, scales, out)
    B, H, n, k, D = codes.shape
    with torch.cuda.device(codes.device):
        rc = _lib.load().fc_jpeg_decode_grouped(
            _p(codes), B, H, n, D, k, *_s(codes, 0, 1, 2, 3), _p(scales), dtype_code(scales),
            int(group), *_s(scales, 0, 1, 2, 3), _p(basis), r, _p(out), dtype_code(out),
            out_len, *_s(out, 0, 1, 2), _stream(codes.device))
    _lib.check(rc, "jpeg_decode_grouped")


def decode_attn_grouped(q, krows, vrows, kscales, vscales, group, kraw, vraw, A, scale,
                        out) -> None:
    """decode_attn over int8 codes (B,Hk,n,s,D) whose scales are
    (B,Hk,n,s,D//group) (fc_decode_attn_grouped)."""
    require_cuda(q, krows, vrows, kscales, vscales, kraw, vraw, A, out)
    _unit_last(krows, vrows, kscales, vscales)
    B, Hq, _, D = q.shape
    Hk, n, s = krows.shape[1], krows.shape[2], krows.shape[3]
    r = A.shape[0]
    t = kraw.shape[2] if kraw is not None else 0
    ws = workspace(q.device, attn_workspace_bytes(B, Hq, Hk, D, n, s, r, t))
    z3 = (0, 0, 0)
    with torch.cuda.device(q.device):
        rc = _lib.load().fc_decode_attn_grouped(
            _p(q), dtype_code(q), B, Hq, D, q.stride(0), q.stride(1), Hk, n, s, r,
            _p(krows), *_s(krows, 0, 1, 2, 3), _p(vrows), *_s(vrows, 0, 1, 2, 3),
            _p(kscales), *_s(kscales, 0, 1, 2, 3), _p(vscales), *_s(vscales, 0, 1, 2, 3),
            dtype_code(kscales), int(group),
            _p(kraw), *(_s(kraw, 0, 1, 2) if kraw is not None else z3),
            _p(vraw), *(_s(vraw, 0, 1, 2) if vraw is not None else z3),
            dtype_code(kraw) if kraw is not None else 0, t,
            _p(A), float(scale), _p(out), dtype_code(out), out.stride(0), out.stride(1),
            _p(ws), ws.numel(), _stream(q.device))
    if rc != _lib.FC_OK:
        reset_workspace(q.device)
    _lib.check(rc, "decode_attn_grouped")
