"""Multi-GPU layout logic on CPU: the shard plans, and the per-rank pieces of
a decode step gathered over a world_size-2 gloo group equal the single-device
result.  The per-rank compute here is the CPU oracle (test infrastructure);
on GPUs each rank runs the same plan with the CUDA kernels."""

import os
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from flashcodec_b200.sharding import local_slice, plan_shards  # noqa: E402


def test_plans():
    p = plan_shards(16, 8, 32, 8)
    assert p.mode == "batch" and [p.batch_range(r) for r in range(8)] == \
        [(2 * r, 2 * r + 2) for r in range(8)]
    p = plan_shards(10, 8, 32, 4)
    assert [p.batch_range(r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    p = plan_shards(2, 8, 32, 8)
    assert p.mode == "heads" and p.needs_gather()
    assert [p.kv_head_range(r) for r in range(8)] == [(0, 2), (2, 4), (4, 6), (6, 8)] * 2
    assert [p.batch_range(r) for r in range(8)] == [(0, 1)] * 4 + [(1, 2)] * 4
    assert p.q_head_range(5) == (8, 16)
    with pytest.raises(ValueError):
        plan_shards(3, 8, 32, 8)
    with pytest.raises(ValueError):
        plan_shards(4, 8, 30, 2)


def _worker(rank, world, port, B, q, k, v, A, ref, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        from flashcodec_b200.sharding import gather_outputs
        plan = plan_shards(B, k.shape[1], q.shape[1], world)
        ql = local_slice(plan, rank, q, query=True)
        kl = local_slice(plan, rank, k)
        vl = local_slice(plan, rank, v)
        out = torch.from_numpy(orc.decode_attention(ql.numpy(), kl.numpy(), vl.numpy(),
                                                    None, None, A))
        full = gather_outputs(plan, out)
        q_out.put((rank, float((full - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [1, 4, 3])
def test_gloo_world2_gather_matches_single_device(B):
    from oracle import oracle as orc
    g = torch.Generator().manual_seed(B)
    Hk, G, n, s, D = 4, 2, 6, 2, 32
    q = torch.randn(B, Hk * G, 1, D, generator=g)
    k = torch.randn(B, Hk, n, s, D, generator=g)
    v = torch.randn(B, Hk, n, s, D, generator=g)
    A = orc.dct_basis_f64(8, s).T.copy()
    ref = torch.from_numpy(orc.decode_attention(q.numpy(), k.numpy(), v.numpy(), None, None, A))
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = 29500 + (os.getpid() % 1000) + B
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, q, k, v, A, ref, qo))
             for r in range(2)]
    for p in procs:
        p.start()
    res = [qo.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err == 0.0 for _, err in res), res


@pytest.mark.parametrize("B,Hk,Hq,world", [(1, 8, 32, 2), (1, 8, 32, 8), (2, 8, 32, 8),
                                           (4, 8, 32, 8), (1, 4, 28, 4), (3, 2, 16, 6)])
def test_head_split_pieces_are_rank_ordered(B, Hk, Hq, world):
    """The peer exchange (PeerOutputs, fc_peers_wait) places rank p's piece
    at p * piece in the (B, Hq) output: in every KV-head plan the ranks' query
    head ranges, batch row first, tile the output in rank order with equal
    pieces."""
    from flashcodec_b200.sharding import plan_shards
    plan = plan_shards(B, Hk, Hq, world)
    assert plan.mode == "heads"
    piece = None
    for r in range(world):
        b0, b1 = plan.batch_range(r)
        h0, h1 = plan.q_head_range(r)
        assert b1 - b0 == 1
        piece = piece or (h1 - h0)
        assert h1 - h0 == piece
        assert b0 * Hq + h0 == r * piece
    assert world * piece == B * Hq
