"""Head-split and batch-split decode steps on 2 GPUs over NCCL: each rank
runs the CUDA decode attention on its shard of the archive, the outputs are
gathered with sharding.gather_outputs (one NCCL all_gather), and the full
output on every rank equals the 1-GPU result within the attention bar and
holds each rank's piece bit for bit.  Needs 2 GPUs (skipped otherwise)."""

import datetime
import os
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _streams(k, v, dev):
    import flashcodec_b200 as fc
    kw = dict(mode="jpeg", block_size=8, keep_freqs=4, quant_bits=8)
    ks, vs = fc._CodecStream(fc.make_codec(**kw)), fc._CodecStream(fc.make_codec(**kw))
    ks.append(k.to(dev))
    vs.append(v.to(dev))
    return ks, vs


def _worker(rank, world, port, B, q, k, v, ref, qo):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        import flashcodec_b200 as fc
        from flashcodec_b200.sharding import gather_outputs, local_slice, plan_shards
        plan = plan_shards(B, k.shape[1], q.shape[1], world)
        ks, vs = _streams(local_slice(plan, rank, k), local_slice(plan, rank, v), dev)
        ql = local_slice(plan, rank, q, query=True).to(dev)
        out = fc.codec_decode_attention(ql, ks, vs)
        full = gather_outputs(plan, out)
        torch.cuda.synchronize()
        b0, b1 = plan.batch_range(rank)
        h0, h1 = plan.q_head_range(rank)
        placed = torch.equal(full[b0:b1, h0:h1], out)
        r = ref.float()
        err = (full.float().cpu() - r).abs()
        within = bool((err <= 2e-3 + 2.0 ** -8 * r.abs()).all())
        qo.put((rank, plan.mode, placed, within, float(err.max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [1, 3])
def test_nccl_world2_gather_matches_single_gpu(B):
    """B=1: KV heads split 4 + 4 (the all_gather path); B=3: uneven batch
    shards 2 + 1 gathered with padding."""
    import bench
    import flashcodec_b200 as fc
    k, v, q = bench.synth_case(B, 32, 8, 8 * 300 + 3, 128, 0.95, 31, dtype=torch.bfloat16)
    ks, vs = _streams(k, v, torch.device("cuda", 0))
    ref = fc.codec_decode_attention(q.to("cuda:0"), ks, vs).cpu()
    del ks, vs
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = 29700 + (os.getpid() % 1000) + B
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, q, k, v, ref, qo))
             for r in range(2)]
    for p in procs:
        p.start()
    res = [qo.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert {m for _, m, _, _, _ in res} == {"heads" if B == 1 else "batch"}
    assert all(placed and within for _, _, placed, within, _ in res), res
