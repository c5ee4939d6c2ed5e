"""Multi-GPU layout of the compressed cache: one process per GPU, each GPU
owns a slice of every stream.

The (batch, KV head) units of the archive, of the decode attention and of the
codecs are independent, so the work shards without any exchange:

* B >= world: contiguous batch ranges (rank r owns rows [start_r, stop_r)).
  No collective at all -- each rank's decode output is its own rows.
* B < world: KV-head groups inside each batch row (world // B ranks per row,
  Hk split evenly); the query heads of a GQA group move with their KV head.
  The only exchange is one all-gather of the (B, Hq_local, 1, D) outputs per
  layer, when a caller needs the full output on every rank.

The reference implementation is single-device; this module is new.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ShardPlan:
    B: int
    Hk: int
    Hq: int
    world: int
    mode: str          # "batch" or "heads"

    @property
    def G(self) -> int:
        return self.Hq // self.Hk

    def batch_range(self, rank: int) -> tuple[int, int]:
        if self.mode == "batch":
            base, extra = divmod(self.B, self.world)
            start = rank * base + min(rank, extra)
            return start, start + base + (1 if rank < extra else 0)
        per_row = self.world // self.B
        b = rank // per_row
        return b, b + 1

    def kv_head_range(self, rank: int) -> tuple[int, int]:
        if self.mode == "batch":
            return 0, self.Hk
        per_row = self.world // self.B
        hk = self.Hk // per_row
        g = rank % per_row
        return g * hk, (g + 1) * hk

    def q_head_range(self, rank: int) -> tuple[int, int]:
        a, b = self.kv_head_range(rank)
        return a * self.G, b * self.G

    def needs_gather(self) -> bool:
        return self.mode == "heads"


def plan_shards(B: int, Hk: int, Hq: int, world: int) -> ShardPlan:
    """Batch shards when there are at least as many sequences as GPUs, else
    KV-head shards (which need world % B == 0 and Hk % (world // B) == 0)."""
    if Hq % Hk:
        raise ValueError(f"Hq ({Hq}) must be a multiple of Hk ({Hk})")
    if world < 1:
        raise ValueError("world must be >= 1")
    if B >= world:
        return ShardPlan(B, Hk, Hq, world, "batch")
    if world % B or Hk % (world // B):
        raise ValueError(f"cannot split B={B} x Hk={Hk} over {world} GPUs "
                         "(need world % B == 0 and Hk % (world // B) == 0)")
    return ShardPlan(B, Hk, Hq, world, "heads")


def local_slice(plan: ShardPlan, rank: int, x: torch.Tensor, *, query: bool = False):
    """This rank's part of a (B, H, ...) tensor: K/V streams use KV heads,
    queries (query=True) use query heads."""
    b0, b1 = plan.batch_range(rank)
    h0, h1 = plan.q_head_range(rank) if query else plan.kv_head_range(rank)
    return x[b0:b1, h0:h1]


def gather_outputs(plan: ShardPlan, out_local: torch.Tensor, group=None) -> torch.Tensor:
    """Full (B, Hq, 1, D) decode output on every rank from the per-rank
    (B_local, Hq_local, 1, D) pieces: one all-gather.  Batch shards are
    gathered too when asked (callers that keep their own rows skip this);
    uneven batch shards are padded to the largest one for the collective."""
    import torch.distributed as dist
    world = plan.world
    if plan.mode == "heads":
        # ranks are ordered batch row first, then KV-head group, and a rank's
        # query heads are one contiguous range, so the rank-major gather of
        # the (1, Hq_local, 1, D) pieces *is* the (B, Hq, 1, D) output: one
        # collective into one buffer, no copies afterwards
        piece = out_local.contiguous()
        full = torch.empty((world,) + tuple(piece.shape[1:]), dtype=piece.dtype,
                           device=piece.device)
        dist.all_gather_into_tensor(full, piece, group=group)
        return full.view(plan.B, plan.Hq, *piece.shape[2:])
    sizes = [plan.batch_range(r)[1] - plan.batch_range(r)[0] for r in range(world)]
    cap = max(sizes)
    padded = torch.zeros((cap,) + tuple(out_local.shape[1:]), dtype=out_local.dtype,
                         device=out_local.device)
    padded[:out_local.shape[0]] = out_local
    full = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(full, padded, group=group)
    return torch.cat([f[:n] for f, n in zip(full, sizes)], dim=0)


class PeerOutputs:
    """Output buffers of a split-KV-head decode step that the attention kernel
    fills on every rank directly: the kernel-fused replacement for
    gather_outputs' all-gather (fc_decode_attn_peers, csrc/fc_attention_tc.cu).

    Each rank holds `slots` full (B, Hq, 1, D) outputs (one per layer, so a
    layer's buffer is never overwritten while it may still be read) and, per
    slot, a receive area of one piece per rank; CUDA IPC handles of the receive
    areas are exchanged once over the process group.  A call of decode() runs
    this rank's KV heads, stores its piece into its own slot and sends it over
    NVLink into every other rank's receive area as self-validating {4 bytes,
    epoch} words, then queues a bounded wait that unpacks the other ranks'
    pieces into the slot; after it the slot holds the full output.  Every
    rank calls decode() for the same slots in the same order.  Epochs come
    from a device counter that each wait advances, so decode() calls captured
    in a CUDA graph use a new epoch on every replay.  A wait that gives up
    records its epoch in the stream's attention workspace status word
    (attention_status).  close() unmaps the peers' areas (collective)."""

    def __init__(self, plan: ShardPlan, rank: int, slots: int, D: int, dtype: torch.dtype,
                 device, group=None):
        import torch.distributed as dist
        from . import _kernels as K
        from . import _lib
        if plan.mode != "heads":
            raise ValueError("PeerOutputs serves split KV heads (plan mode 'heads')")
        if not 1 <= plan.world <= _lib.FC_MAX_PEERS:
            raise ValueError(f"at most {_lib.FC_MAX_PEERS} ranks")
        self.plan, self.rank, self.world, self.group = plan, rank, plan.world, group
        self.device = torch.device(device)
        self.bufs = torch.zeros((slots, plan.B, plan.Hq, 1, D), dtype=dtype, device=self.device)
        hq_local = plan.q_head_range(rank)[1] - plan.q_head_range(rank)[0]
        piece_bytes = hq_local * D * self.bufs.element_size()   # one batch row per rank
        if piece_bytes % 4:
            raise ValueError("a rank's output piece must be a multiple of 4 bytes")
        self.piece_words = piece_bytes // 4
        self.recv = torch.zeros((slots, self.world, self.piece_words), dtype=torch.int64,
                                device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        infos = [None] * self.world
        dist.all_gather_object(infos, K.ipc_get_handle(self.recv), group=group)
        self._opened: dict = {}          # handle -> mapped base
        bases = [self.recv.data_ptr() if p == rank else self._open(h) + off
                 for p, (h, off) in enumerate(infos)]
        # ranks own consecutive pieces of a slot (batch row, then KV-head group)
        slot_bytes = plan.B * plan.Hq * D * self.bufs.element_size()
        self._tables = []
        for s in range(slots):
            t = _lib.PeerOut()
            t.out = self.bufs.data_ptr() + s * slot_bytes + rank * piece_bytes
            for p in range(self.world):
                t.recv[p] = bases[p] + ((s * self.world + rank) * self.piece_words) * 8
            t.world, t.rank = self.world, rank
            t.counter = self.counter.data_ptr()
            self._tables.append(t)

    def _open(self, handle: bytes) -> int:
        from . import _kernels as K
        if handle not in self._opened:
            self._opened[handle] = K.ipc_open(handle, self.device)
        return self._opened[handle]

    def decode(self, query: torch.Tensor, key_stream, value_stream, slot: int, scale=None):
        """This rank's (1, Hq_local, 1, D) query against its KV-head streams;
        returns slot `slot`'s full (B, Hq, 1, D) output, complete once the
        queued wait has run (later work on the current stream sees it)."""
        from . import _kernels as K
        from .attention import _device_A, _rows
        ks, vs = key_stream, value_stream
        if ks.codec.name != "jpeg" or getattr(ks.codec, "group_size", None) is not None \
                or ks.n_blocks == 0:
            raise NotImplementedError("peer outputs take jpeg archives with one scale per "
                                      "row and at least one archived block")
        if query.dtype != self.bufs.dtype:
            raise ValueError("query and output buffers must share a dtype")
        D = query.shape[-1]
        scale = D ** -0.5 if scale is None else scale
        krows, kscales = _rows(ks)
        vrows, vscales = _rows(vs)
        A = _device_A(ks.codec, ks.block_size, query.device)
        full = self.bufs[slot]
        K.decode_attn_peers(query, krows, vrows, kscales, vscales, ks.raw, vs.raw, A, scale,
                            full.dtype, full.stride(0), full.stride(1), self._tables[slot])
        ws = K.workspace(query.device, 0)
        K.peers_wait(self.recv[slot], full, self.world, self.rank, self.piece_words, 0, ws,
                     counter=self.counter)
        return full

    def close(self) -> None:
        """Unmap the other ranks' receive areas once every rank has finished
        with them (collective: every rank calls it)."""
        import torch.distributed as dist
        from . import _kernels as K
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for base in self._opened.values():
            K.ipc_close(base, self.device)
        self._opened.clear()
        dist.barrier(group=self.group)
