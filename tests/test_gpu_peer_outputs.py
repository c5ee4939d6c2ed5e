"""Split KV heads without a collective: fc_decode_attn_peers stores this
rank's output piece into its own buffer and sends it to every other rank's
receive area as {4 bytes, epoch} words; fc_peers_wait waits (bounded) for the
other ranks' words and unpacks them into the output.

On one GPU two ranks are emulated in one process: both ranks' launches run
(in stream order) before either wait is queued, so every wait finds its flags
already published -- no kernel ever waits for a launch that has not run.  The
two-process test needs two GPUs (one rank per GPU, buffers opened over CUDA
IPC) and is skipped otherwise."""

import datetime
import os
import sys
import time
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _streams(k, v, dev, quant=8):
    import flashcodec_b200 as fc
    kw = dict(mode="jpeg", block_size=8, keep_freqs=4, quant_bits=quant)
    ks, vs = fc._CodecStream(fc.make_codec(**kw)), fc._CodecStream(fc.make_codec(**kw))
    ks.append(k.to(dev))
    vs.append(v.to(dev))
    return ks, vs


def _peer_call(q, ks, vs, table, o_sb, o_sh):
    """fc_decode_attn_peers of one rank through the package's binding."""
    from flashcodec_b200 import _kernels as K
    from flashcodec_b200.attention import _device_A, _rows
    krows, kscales = _rows(ks)
    vrows, vscales = _rows(vs)
    A = _device_A(ks.codec, ks.block_size, q.device)
    K.decode_attn_peers(q, krows, vrows, kscales, vscales, ks.raw, vs.raw, A,
                        q.shape[-1] ** -0.5, q.dtype, o_sb, o_sh, table)


def _emulated_ranks(k, v, q, world, dev, quant=8, counters=None):
    """Per emulated rank: its full output buffer, its receive area, and the
    (query, K stream, V stream, fc_peer_out) of its call."""
    from flashcodec_b200 import _lib
    B, Hq, _, D = q.shape
    Hk = k.shape[1]
    G = Hq // Hk
    bufs = [torch.zeros(B, Hq, 1, D, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    piece_bytes = Hq // world * D * bufs[0].element_size()
    words = piece_bytes // 4
    recv = [torch.zeros(world, words, dtype=torch.int64, device=dev) for _ in range(world)]
    calls = []
    for rank in range(world):
        h0, h1 = rank * Hk // world, (rank + 1) * Hk // world
        lks, lvs = _streams(k[:, h0:h1], v[:, h0:h1], dev, quant)
        t = _lib.PeerOut()
        t.out = bufs[rank].data_ptr() + rank * piece_bytes
        for p in range(world):
            t.recv[p] = recv[p].data_ptr() + rank * words * 8
        t.world, t.rank = world, rank
        if counters is not None:
            t.counter = counters[rank].data_ptr()
        calls.append((q[:, h0 * G:h1 * G].to(dev).contiguous(), lks, lvs, t))
    return bufs, recv, words, calls


@pytest.mark.parametrize("S,quant", [(8 * 3000 + 5, 8), (8 * 40 + 3, 8), (8 * 500 + 1, 0)])
def test_two_ranks_emulated_on_one_gpu(S, quant):
    """Ranks 0 and 1 each hold 4 of 8 KV heads of one sequence (one split per
    unit, and many).  After both peer launches and both waits, each rank's
    buffer holds the full output, the two buffers are bit-identical, each
    rank's piece equals the plain kernel on its heads bit for bit, and the
    whole matches the 1-GPU call within the attention bar -- on two calls in a
    row with explicit epochs."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    dev = torch.device(DEV, 0)
    B, Hq, Hk, D, world = 1, 32, 8, 128, 2
    k, v, q = bench.synth_case(B, Hq, Hk, S, D, 0.95, 41, dtype=torch.bfloat16)
    ks, vs = _streams(k, v, dev, quant)
    ref = fc.codec_decode_attention(q.to(dev), ks, vs)
    bufs, recv, words, calls = _emulated_ranks(k, v, q, world, dev, quant)
    local = []
    for epoch in (1, 2):
        for b in bufs:
            b.zero_()
        pieces = []
        for ql, lks, lvs, t in calls:
            t.epoch = epoch
            _peer_call(ql, lks, lvs, t, bufs[0].stride(0), bufs[0].stride(1))
            pieces.append(fc.codec_decode_attention(ql, lks, lvs))
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        for rank in range(world):
            K.peers_wait(recv[rank], bufs[rank], world, rank, words, epoch, status)
        torch.cuda.synchronize()
        assert status.item() == 0
        assert torch.equal(bufs[0], bufs[1])
        for rank in range(world):
            h0 = rank * Hq // world
            assert torch.equal(bufs[0][:, h0:h0 + pieces[rank].shape[1]], pieces[rank])
        r = ref.float().cpu()
        err = (bufs[0].float().cpu() - r).abs()
        assert bool((err <= 2e-3 + 2.0 ** -8 * r.abs()).all()), float(err.max())
        assert int(recv[0][1, 0].item()) >> 32 == epoch
        local.append(bufs[0].clone())
    assert torch.equal(local[0], local[1])


def test_two_ranks_emulated_replay_in_a_cuda_graph():
    """Device-counter epochs: both ranks' peer launches and both waits are
    captured once in a CUDA graph and replayed three times; every replay uses
    a new epoch (the counters end at 4 after the eager call and three
    replays), no wait gives up, and both buffers hold the eager output."""
    from flashcodec_b200 import _kernels as K
    dev = torch.device(DEV, 0)
    B, Hq, Hk, D, world = 1, 32, 8, 128, 2
    k, v, q = bench.synth_case(B, Hq, Hk, 8 * 700 + 2, D, 0.95, 43, dtype=torch.bfloat16)
    ctrs = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
    bufs, recv, words, calls = _emulated_ranks(k, v, q, world, dev, counters=ctrs)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def step():
        for ql, lks, lvs, t in calls:
            _peer_call(ql, lks, lvs, t, bufs[0].stride(0), bufs[0].stride(1))
        for rank in range(world):
            K.peers_wait(recv[rank], bufs[rank], world, rank, words, 0, status,
                         counter=ctrs[rank])

    step()                     # eager: the kernels' one-time set-up happens here
    torch.cuda.synchronize()
    eager = bufs[0].clone()
    for b in bufs:
        b.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(bufs[0], eager) and torch.equal(bufs[1], eager)
    # the eager call and three replays (capturing runs nothing)
    assert [c.item() for c in ctrs] == [4, 4]
    assert int(recv[0][1, -1].item()) >> 32 == 4 and int(recv[1][0, -1].item()) >> 32 == 4


def test_peer_outputs_refuse_cuda_core_layouts():
    """Peer outputs need the tensor-core kernel: head dim 64 is refused
    loudly, before anything is stored or sent."""
    from flashcodec_b200 import _lib
    dev = torch.device(DEV, 0)
    k, v, q = bench.synth_case(1, 8, 2, 8 * 20, 64, 0.95, 3, dtype=torch.bfloat16)
    ks, vs = _streams(k, v, dev)
    out = torch.zeros(1, 8, 1, 64, dtype=torch.bfloat16, device=dev)
    recv = torch.zeros(2, 8 * 64 // 4, dtype=torch.int64, device=dev)
    t = _lib.PeerOut()
    t.out, t.world, t.rank, t.epoch = out.data_ptr(), 2, 0, 1
    t.recv[1] = recv.data_ptr()
    with pytest.raises(NotImplementedError):
        _peer_call(q.to(dev), ks, vs, t, out.stride(0), out.stride(1))
    torch.cuda.synchronize()
    assert recv.abs().sum().item() == 0 and out.abs().sum().item() == 0


def test_peers_wait_gives_up_on_a_piece_nobody_sends():
    """Failure detection without a GPU fault: waiting for a piece no rank
    sends gives up after the 100 ms limit, records the epoch in the status
    word, and the context stays usable; once the words carry the epoch the
    wait unpacks them into the output."""
    from flashcodec_b200 import _kernels as K
    words = 64
    recv = torch.zeros(2, words, dtype=torch.int64, device=DEV)
    out = torch.zeros(2 * words, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    K.peers_wait(recv, out, 2, 0, words, 7, status)     # rank 1 never sends
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert status.item() == 7
    assert 0.09 <= dt < 5.0, dt
    payload = torch.arange(1000, 1000 + words, dtype=torch.int64, device=DEV)
    recv[1] = (7 << 32) | payload
    status.zero_()
    K.peers_wait(recv, out, 2, 0, words, 7, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(out[words:].long(), payload) and out[:words].abs().sum().item() == 0


def _worker(rank, world, port, q, k, v, ref, qo):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        import flashcodec_b200 as fc
        from flashcodec_b200.sharding import PeerOutputs, gather_outputs, local_slice, plan_shards
        plan = plan_shards(1, k.shape[1], q.shape[1], world)
        ks, vs = _streams(local_slice(plan, rank, k), local_slice(plan, rank, v), dev)
        ql = local_slice(plan, rank, q, query=True).to(dev).contiguous()
        po = PeerOutputs(plan, rank, 2, q.shape[-1], q.dtype, dev)
        results = []
        for step in range(3):                # slots 0, 1, 0: epochs 1, 2, 3
            full = po.decode(ql, ks, vs, slot=step % 2)
            torch.cuda.synchronize()
            results.append(full.clone())
        nccl = gather_outputs(plan, fc.codec_decode_attention(ql, ks, vs))
        torch.cuda.synchronize()
        status = fc.attention_status(dev).value()
        po.close()
        r = ref.float()
        err = (results[-1].float().cpu() - r).abs()
        qo.put((rank, all(torch.equal(x, nccl) for x in results), status,
                bool((err <= 2e-3 + 2.0 ** -8 * r.abs()).all()), float(err.max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_gpus_peer_outputs_match_nccl_gather():
    """One sequence, 8 KV heads split 4 + 4 over 2 GPUs: the outputs each
    rank's kernel stored into both ranks' buffers equal the NCCL all-gather of
    the same pieces bit for bit, on three calls over two slots."""
    import bench as bn
    import flashcodec_b200 as fc
    k, v, q = bn.synth_case(1, 32, 8, 8 * 300 + 3, 128, 0.95, 31, dtype=torch.bfloat16)
    ks, vs = _streams(k, v, torch.device("cuda", 0))
    ref = fc.codec_decode_attention(q.to("cuda:0"), ks, vs).cpu()
    del ks, vs
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = 29600 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, ref, qo)) for r in range(2)]
    for p in procs:
        p.start()
    res = [qo.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(same and status == 0 and within for _, same, status, within, _ in res), res
