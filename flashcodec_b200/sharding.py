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
