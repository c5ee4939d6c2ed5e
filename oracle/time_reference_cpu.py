"""Provenance of the timed CPU baseline (test infrastructure; nothing in the
package, the tests or bench.py runs this file).

bench.py times oracle.reference_attention_int8_mt, a numpy port of the
reference's torch decode-attention path, because the reference itself does
not travel with the repository.  This script, run where the reference source
tree is available, times the reference's own path
(flashcodec/attention.py:101-140, codec_decode_attention(impl="torch") on
CPU tensors) and the port on the same bounded sample -- one config-2 layer,
sequence 0 of 16, all 8 KV heads, 32768 archived tokens + 5 raw, jpeg r=8
K=4 int8 -- on the same host threads, so the port's speed can be compared
with the reference's.

    FLASHCODEC_REF=<directory holding the flashcodec package> \\
        python oracle/time_reference_cpu.py [--reps 7]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=7)
    args = ap.parse_args()
    if "FLASHCODEC_REF" not in os.environ:
        raise SystemExit("set FLASHCODEC_REF to the flashcodec source tree")
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, os.environ["FLASHCODEC_REF"])
    import torch
    from flashcodec import make_codec
    from flashcodec.attention import codec_decode_attention
    from flashcodec.cache import _CodecStream

    import bench
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = bench.CFG2
    k, v, q = bench.synth_case(1, cfg["Hq"], cfg["Hk"], cfg["S"] + cfg["tail"], cfg["D"],
                               cfg["rho"], 0, dtype=torch.bfloat16)
    ks = _CodecStream(make_codec("jpeg", block_size=cfg["r"], keep_freqs=cfg["K"], quant_bits=8))
    vs = _CodecStream(make_codec("jpeg", block_size=cfg["r"], keep_freqs=cfg["K"], quant_bits=8))
    ks.append(k)
    vs.append(v)
    n = ks.n_blocks
    from flashcodec.codecs import dct_basis
    A = dct_basis(cfg["r"], cfg["K"]).numpy()[:, :cfg["r"]].T.copy()
    port_args = (q.float().numpy(), ks._coeffs[:, :, :n].numpy(), ks._scales[:, :, :n].numpy(),
                 vs._coeffs[:, :, :n].numpy(), vs._scales[:, :, :n].numpy(),
                 ks.raw.float().numpy(), vs.raw.float().numpy(), A)

    def timed(fn):
        fn()
        ts = []
        for _ in range(args.reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts) * 1e3

    res = {
        "sample": "config-2 layer, sequence 0 of 16, 8 KV heads, 4096 blocks + 5 raw",
        "threads": threads,
        "reference_torch_bf16_ms": timed(lambda: codec_decode_attention(q, ks, vs, impl="torch")),
        "reference_torch_fp32_query_ms": timed(
            lambda: codec_decode_attention(q.float(), ks, vs, impl="torch")),
        "port_threaded_ms": timed(
            lambda: orc.reference_attention_int8_mt(*port_args, threads=threads)),
        "port_single_ms": timed(lambda: orc.reference_attention_int8(*port_args)),
    }
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
