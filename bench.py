"""Decode-attention benchmark over int8 DCT-compressed KV (flashcodec hot path).

(The synthetic-input section below is shared with tests/ and the golden
fixture generator; the benchmark driver follows it.)
"""

from __future__ import annotations

import math

import torch

# --------------------------------------------------------------------------
# Synthetic KV inputs.
#
# The reference measures on no public dataset; its benchmarks draw seeded
# random walks (benchmarks/bench_reconstruct.py:18-20).  The inputs here follow
# the same idea with a per-channel scale: K and V are AR(1) along the sequence,
# x_0 = e_0, x_t = rho * x_{t-1} + e_t with e ~ N(0, 1), multiplied by a
# per-(head, channel) std ~ LogNormal(0, 0.5); K additionally has four outlier
# channels scaled x10; q ~ N(0, 1) / sqrt(D).  K, V and q come from independent
# generators seeded 3*seed, 3*seed+1, 3*seed+2.  Generated in fp32 on the
# device that uses them, then cast.
# --------------------------------------------------------------------------


def outlier_channels(D: int):
    """Four fixed K outlier channels (0, 37, 74, 111 at D=128), scaled to D."""
    return sorted({(c * D) // 128 for c in (0, 37, 74, 111)})


def ar1_scan_(x: torch.Tensor, rho: float) -> torch.Tensor:
    """In-place AR(1) along dim -2: x_t <- sum_{s<=t} rho^(t-s) x_s.
    Log-depth (Hillis-Steele) scan: after step k every x_t holds the sum over
    the last 2^k innovations."""
    S = x.shape[-2]
    step, coef = 1, float(rho)
    while step < S:
        x[..., step:, :].add_(x[..., :-step, :].clone(), alpha=coef)
        coef *= coef
        step *= 2
    return x


def synth_stream(B: int, H: int, S: int, D: int, rho: float, seed: int, *,
                 outliers: bool = False, device="cpu", dtype=torch.float32):
    """One (B, H, S, D) synthetic K or V tensor (see the section comment)."""
    g = torch.Generator(device=device).manual_seed(int(seed))
    std = torch.exp(0.5 * torch.randn(1, H, 1, D, generator=g, device=device))
    x = torch.randn(B, H, S, D, generator=g, device=device)
    ar1_scan_(x, rho)
    x.mul_(std)
    if outliers:
        x[..., outlier_channels(D)] *= 10.0
    return x.to(dtype)


def synth_query(B: int, Hq: int, D: int, seed: int, *, device="cpu", dtype=torch.float32):
    g = torch.Generator(device=device).manual_seed(int(seed))
    return (torch.randn(B, Hq, 1, D, generator=g, device=device) / math.sqrt(D)).to(dtype)


def synth_case(B, Hq, Hk, S, D, rho, seed=0, *, device="cpu", dtype=torch.float32):
    """(k, v, q) for one layer: k/v (B, Hk, S, D), q (B, Hq, 1, D)."""
    k = synth_stream(B, Hk, S, D, rho, 3 * seed, outliers=True, device=device, dtype=dtype)
    v = synth_stream(B, Hk, S, D, rho, 3 * seed + 1, device=device, dtype=dtype)
    q = synth_query(B, Hq, D, 3 * seed + 2, device=device, dtype=dtype)
    return k, v, q


# --------------------------------------------------------------------------
# Benchmark driver.
#
# Workload (config 2 of the spec, the one the metric is quoted on): a
# Qwen3-8B-shaped decode step -- 36 layers, batch 16 per GPU, Hq=32, Hkv=8,
# D=128, context 32768 archived tokens + a raw tail of 5, bf16 K/V archived
# with the jpeg codec r=8, K=4, int8 codes + fp32 scales.  One step = one
# split-K decode-attention launch per layer over the whole archive; tokens/s
# = sequences in the batch / step time.  The archive (about 20 GB per GPU) is
# far larger than L2, so no L2 flush is needed between steps.
#
# N GPUs: one process per GPU; every GPU owns its own batch of 16 sequences
# (weak scaling: the (batch, KV head) units are independent, there is no
# data-path collective).
# --------------------------------------------------------------------------

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = ("decode-attn tokens/s & achieved HBM GB/s (% of peak) on int8 DCT KV, "
          "1/2/4/8 B200")
CFG2 = dict(layers=36, B=16, Hq=32, Hk=8, D=128, S=32768, tail=5, r=8, K=4, rho=0.95,
            scale_dtype="fp32", config=2)
# config 5 per GPU at 8-way batch sharding (global B=128): S=131072, K=2,
# fp16 scales; 8 independent layer archives (~1.09 GB each) per step
CFG5 = dict(layers=8, B=16, Hq=32, Hk=8, D=128, S=131072, tail=0, r=8, K=2, rho=0.95,
            scale_dtype="fp16", config=5)
FALLBACK_HBM_GBS = 6650.0


def attn_bytes(B, Hq, Hk, D, n, K, tail, code_b=1, scale_b=4, io_b=2):
    """Algorithmic bytes of one decode-attention launch: K and V codes and
    scales, the raw tail, q and the output (each read or written once)."""
    return (2 * B * Hk * n * K * D * code_b + 2 * B * Hk * n * K * scale_b
            + 2 * B * Hk * tail * D * io_b + 2 * B * Hq * D * io_b)


def codec_attn_bytes(cfg, n):
    """Algorithmic bytes of one launch for the archive format in cfg:
    jpeg-int8 (codes + scales), jpeg-fp (bf16 coefficients, quant_bits=0) or
    png (bf16 anchor + fp32 deltas per block)."""
    codec = cfg.get("codec", "jpeg-int8")
    B, Hq, Hk, D, tail = cfg["B"], cfg["Hq"], cfg["Hk"], cfg["D"], cfg["tail"]
    if codec == "jpeg-int8":
        return attn_bytes(B, Hq, Hk, D, n, cfg["K"], tail,
                          scale_b=2 if cfg["scale_dtype"] == "fp16" else 4)
    if codec == "jpeg-fp":
        return attn_bytes(B, Hq, Hk, D, n, cfg["K"], tail, code_b=2, scale_b=0)
    per_block = D * 2 + (cfg["r"] - 1) * D * 4
    return 2 * B * Hk * n * per_block + 2 * B * Hk * tail * D * 2 + 2 * B * Hq * D * 2


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes of the attention kernel from the committed ncu
    summary (profiles/attn_decode_cfg2.json), or None."""
    p = ROOT / "profiles" / "attn_decode_cfg2.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi sampled every 200 ms on the given GPUs (read-only query)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.t0 = None

    def start(self):
        try:
            self.t0 = time.time()
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(map(str, self.gpus)),
                 f"--query-gpu=timestamp,{self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self, t_begin, t_end):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        rows = []
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(f[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                rows.append((ts, float(f[2]), float(f[3]), f[6:10]))
            except Exception:
                continue
        if not rows:
            return None
        inside = [x for x in rows if t_begin - 1.0 <= x[0] <= t_end + 1.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for x in inside for n, v in zip(names, x[3]) if v == "Active"})
        return {"sm_mhz": statistics.median(x[1] for x in inside),
                "sm_max_mhz": max(x[2] for x in inside), "reasons": reasons,
                "samples": len(inside)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif n_gpus > 1:
        raise SystemExit("--gpus N > 1 runs under torchrun (one process per GPU)")
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_layers(cfg, rank, device):
    """Archive every layer's synthetic K/V through the product's append path
    (the jpeg int8 archive kernel); returns [(k_stream, v_stream, q)]."""
    import flashcodec_b200 as fc
    layers = []
    for L in range(cfg["layers"]):
        seed = 1000 * rank + L
        k, v, q = synth_case(cfg["B"], cfg["Hq"], cfg["Hk"], cfg["S"] + cfg["tail"], cfg["D"],
                             cfg["rho"], seed, device=device, dtype=torch.bfloat16)
        codec = cfg.get("codec", "jpeg-int8")
        if codec == "png":
            c = fc.make_codec("png", block_size=cfg["r"], keep_ratio=1.0)
        else:
            c = fc.make_codec("jpeg", block_size=cfg["r"], keep_freqs=cfg["K"],
                              quant_bits=8 if codec == "jpeg-int8" else 0,
                              scale_dtype=torch.float16 if cfg["scale_dtype"] == "fp16"
                              else torch.float32)
        ks, vs = fc._CodecStream(c), fc._CodecStream(c)
        ks.append(k)
        del k
        vs.append(v)
        del v
        layers.append((ks, vs, q))
    torch.cuda.synchronize()
    return layers


def cpu_sample_from(layers, cfg, b_sample=1):
    """Host copy of one layer's archive for b_sample sequences (oracle input)."""
    ks, vs, q = layers[0]
    n = ks.n_blocks
    out = {}
    for nm, st in (("k", ks), ("v", vs)):
        out[nm] = st._coeffs[:b_sample, :, :n].cpu().numpy()
        out[nm + "s"] = st._scales[:b_sample, :, :n].cpu().numpy()
        out[nm + "raw"] = st.raw[:b_sample].float().cpu().numpy()
    out["q"] = q[:b_sample].float().cpu().numpy()
    return out


def time_cpu_baseline(sample, cfg, reps, threads):
    """Time the oracle's fp32 restatement of the reference's torch attention
    path on host cores; tokens/s scaled from the sample (b_sample sequences,
    one layer) to the 36-layer step."""
    import numpy as np
    from oracle import oracle as orc
    import flashcodec_b200 as fc
    A = fc.block_basis(fc.make_codec("jpeg", block_size=cfg["r"], keep_freqs=cfg["K"]),
                       cfg["r"]).numpy()
    args = (sample["q"], sample["k"], sample["ks"], sample["v"], sample["vs"], sample["kraw"],
            sample["vraw"], A)
    orc.reference_attention_int8(*args)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        orc.reference_attention_int8(*args)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    b = sample["q"].shape[0]
    nbytes = attn_bytes(b, cfg["Hq"], cfg["Hk"], cfg["D"], sample["k"].shape[2], cfg["K"],
                        cfg["tail"])
    return {"value": b / (cfg["layers"] * t), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": (f"one layer, batch {b} of {cfg['B']}, all {cfg['Hk']} KV heads, full "
                       f"context; median of {reps} calls of "
                       f"oracle.reference_attention_int8 (numpy: fp32 dequantize + fp32 BLAS) "
                       f"= {t * 1e3:.1f} ms ({nbytes / t / 1e9:.2f} GB/s of compressed "
                       f"bytes); tokens/s = batch / (36 layers x time)")}


def run_reference(args, cfg):
    """--impl reference: the reference algorithm's CPU implementation (the
    oracle port) on the host cores, same metric/config/unit."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return
    import numpy as np
    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    b = 1
    k, v, q = synth_case(b, cfg["Hq"], cfg["Hk"], cfg["S"] + cfg["tail"], cfg["D"], cfg["rho"],
                         0, dtype=torch.bfloat16)
    import flashcodec_b200 as fc
    basis = fc.dct_basis(cfg["r"], cfg["K"]).numpy()
    n = cfg["S"] // cfg["r"]
    rows = {}
    for nm, x in (("k", k), ("v", v)):
        xn = x.float().numpy()
        coef = orc.jpeg_encode(xn[:, :, :n * cfg["r"]], cfg["r"], cfg["K"], basis, "bf16")
        rows[nm], rows[nm + "s"] = orc.jpeg_quantize(coef, "bf16")
        rows[nm + "raw"] = xn[:, :, n * cfg["r"]:]
    A = basis[:cfg["K"], :cfg["r"]].T.copy()
    call = (q.float().numpy(), rows["k"], rows["ks"], rows["v"], rows["vs"], rows["kraw"],
            rows["vraw"], A)
    for _ in range(args.warmup):
        orc.reference_attention_int8(*call)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.reference_attention_int8(*call)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = b / (cfg["layers"] * dt)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * cfg["layers"] * cfg["B"] / b * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic",
            "config": workload_config(cfg, world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                             "kind": "port",
                             "sample": (f"each step: one layer, batch {b} of {cfg['B']}, all "
                                        f"{cfg['Hk']} KV heads, full context, "
                                        "oracle.reference_attention_int8 (numpy: fp32 dequantize + fp32 BLAS); "
                                        "tokens/s = batch / (36 layers x step time); "
                                        "ms_per_step scaled to the full 36-layer batch-16 step")},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


CODEC_WORKLOADS = ("archive", "read", "png-encode", "png-decode", "stream", "decode-step")


def run_codec(args):
    """--workload archive|read|png-encode|png-decode: HBM throughput of one
    codec kernel on one GPU (secondary lines for the codec rooflines; the
    default run is the config-2 attention line).  Inputs are seeded synthetic
    tensors of the configs' shapes, larger than L2, resident in HBM; each
    launch is timed with CUDA events on the launching stream."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = measured_peaks()
    w = args.workload
    if w in ("archive", "read"):
        # config 2 stream shape: one layer's K stream, bf16, r=8, K=4, int8
        B, H, S, D, r, k = 16, 8, 32768, 128, 8, 4
        x = synth_stream(B, H, S, D, 0.95, 0, device=dev, dtype=torch.bfloat16)
        n = S // r
        basis = fc.codecs.jpeg.device_basis(r, k, dev)
        codes = torch.empty(B, H, n, k, D, dtype=torch.int8, device=dev)
        scales = torch.empty(B, H, n, k, 1, dtype=torch.float32, device=dev)
        K.jpeg_encode(x, basis, r, k, codes, scales)
        rec = torch.empty_like(x)
        if w == "archive":
            launch = lambda: K.jpeg_encode(x, basis, r, k, codes, scales)  # noqa: E731
        else:
            launch = lambda: K.jpeg_decode(codes, scales, basis, r, rec, S)  # noqa: E731
        nbytes = x.numel() * 2 + codes.numel() + scales.numel() * 4
        config = {"workload": f"jpeg {'archive (dct_compress + quantize_coeffs)' if w == 'archive' else 'read (dequantize + dct_decompress)'}, "
                              "config 2 stream shape", "B": B, "H": H, "S": S, "D": D, "r": r,
                  "K": k, "in_dtype": "bf16", "codes": "int8 + fp32 scales"}
        kernel = "fc_jpeg_encode" if w == "archive" else "fc_jpeg_decode"
    else:
        # config 3: png lossless tier, fp32, r=16, keep 1.0
        B, H, S, D, r = 8, 8, 16384, 128, 16
        x = synth_stream(B, H, S, D, 0.98, 0, device=dev, dtype=torch.float32)
        n = S // r
        deltas = torch.empty(B, H, n, r - 1, D, dtype=torch.float32, device=dev)
        anchors = torch.empty(B, H, n, D, dtype=torch.float32, device=dev)
        K.png_encode(x, r, r - 1, deltas, anchors)
        rec = torch.empty_like(x)
        if w == "png-encode":
            launch = lambda: K.png_encode(x, r, r - 1, deltas, anchors)  # noqa: E731
        else:
            launch = lambda: K.png_decode(deltas, anchors, rec, S)  # noqa: E731
        nbytes = x.numel() * 4 + deltas.numel() * 4 + anchors.numel() * 4
        config = {"workload": f"png {'filter' if w == 'png-encode' else 'reconstruct'}, config 3",
                  "B": B, "H": H, "S": S, "D": D, "r": r, "keep_ratio": 1.0, "dtype": "fp32"}
        kernel = "fc_png_encode" if w == "png-encode" else "fc_png_decode"
    for _ in range(args.warmup):
        launch()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    torch.cuda.synchronize()
    for a, b in ev:
        a.record(stream)
        launch()
        b.record(stream)
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    gbs = nbytes / (ms * 1e-3) / 1e9
    line = {"metric": f"{w} HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if w in ("archive", "read") else "fp32", "data": "synthetic",
            "config": dict(config, l2="no flush: every launch moves > 1 GB, > 8x L2"),
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": gbs, "peak": peak,
                         "unit": "GB/s", "frac": gbs / peak, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": nbytes},
            "gpu_launches": args.steps}
    print(json.dumps(line), flush=True)


def run_stream(args):
    """--workload stream: config 4 -- 28 layers of a Qwen3-0.6B-shaped cache
    (Hkv=8, D=128, bf16, jpeg r=8 K=2 int8), batch 64, one token appended per
    layer per step; each step also reads layer 0's view incrementally.
    Timed over 256-step windows at the start (from an empty cache) and at the
    end of the 65536-token range (after a bulk prefill to 65280 tokens), with
    CUDA events around every step (host launch overhead included)."""
    import flashcodec_b200 as fc
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, B, H, D, S_end, W = 28, 64, 8, 128, 65536, 256
    g = torch.Generator(device=dev).manual_seed(4)
    toks = [(torch.randn(B, H, 1, D, generator=g, device=dev).to(torch.bfloat16),
             torch.randn(B, H, 1, D, generator=g, device=dev).to(torch.bfloat16)) for _ in range(L)]

    def window(cache, steps):
        stream = torch.cuda.current_stream(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for a, b in ev:
            a.record(stream)
            for i in range(L):
                cache.append(toks[i][0], toks[i][1], i)
            cache._keys[0].read()
            b.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / steps * 1e3
        return statistics.mean(a.elapsed_time(b) for a, b in ev), wall

    def new_cache():
        return fc.CodecKVCache("jpeg", block_size=8, keep_freqs=2, quant_bits=8)

    c0 = new_cache()
    for i in range(L):  # first token: allocate the streams
        c0.append(toks[i][0], toks[i][1], i)
    window(c0, 8)       # warm-up (kernels loaded, first archive)
    del c0
    c1 = new_cache()
    start_ms, start_wall = window(c1, W)
    del c1
    torch.cuda.empty_cache()
    c2 = new_cache()
    S_pre = S_end - W
    for i in range(L):
        k = synth_stream(B, H, S_pre, D, 0.95, 2 * i, device=dev, dtype=torch.bfloat16)
        c2.append(k, k, i)  # value content does not change the work
        del k
    c2._keys[0].read()
    end_ms, end_wall = window(c2, W)
    line = {"metric": "config 4 streaming step (append 28 layers + incremental read of one layer)",
            "value": end_ms, "unit": "ms/step", "n_gpus": 1, "steps": W, "warmup": 8,
            "ms_per_step": end_ms, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 4: Qwen3-0.6B-shaped streaming append/archive",
                       "layers": L, "batch": B, "Hkv": H, "head_dim": D,
                       "codec": "jpeg r=8 K=2 int8, fp32 scales",
                       "window_start": {"context": [0, W], "ms_per_step": start_ms,
                                        "wall_ms_per_step": start_wall},
                       "window_end": {"context": [S_pre, S_end], "ms_per_step": end_ms,
                                      "wall_ms_per_step": end_wall},
                       "timing": "CUDA events around each step on the current stream"},
            "gpu_launches": None}
    print(json.dumps(line), flush=True)


def run_decode_step(args):
    """--workload decode-step: the attention half of one model decode step on
    config 2 (36 layers, B=16, Hq=32, Hkv=8, D=128, 32768 archived tokens,
    jpeg r=8 K=4 int8): per layer the rotary embedding of the new q and k,
    the append of k and v (archiving each block as it completes) and the
    archive decode attention.  Fused = fc_rope_kv_append + fc_decode_attn
    (what the patched attention module runs); unfused = transformers'
    apply_rotary_pos_emb + two stream appends + fc_decode_attn (the
    reference's sequence, flashcodec/patch_attention.py:82-98, on this
    package's kernels).  CUDA events around each step, host launch overhead
    included; the archives are pre-grown so no capacity doubling lands in the
    timed steps."""
    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    from flashcodec_b200.cache import append_rotary
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = dict(CFG2, layers=args.layers or CFG2["layers"], B=args.batch or CFG2["B"])
    layers = build_layers(cfg, 0, dev)
    B, Hq, Hk, D = cfg["B"], cfg["Hq"], cfg["Hk"], cfg["D"]
    steps = args.steps
    for ks, vs, _ in layers:
        for st in (ks, vs):
            st._grow(st.n_blocks + 2 * (steps + args.warmup) // cfg["r"] + 2, st._raw_buf)
    g = torch.Generator(device=dev).manual_seed(11)

    def hf(h):
        return torch.randn(B, 1, h, D, generator=g, device=dev).to(torch.bfloat16).transpose(1, 2)

    toks = [(hf(Hq), hf(Hk), hf(Hk)) for _ in layers]
    pos = torch.arange(B, device=dev, dtype=torch.float32)[:, None] + cfg["S"]
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
    ang = torch.cat([pos * inv, pos * inv], dim=-1)[:, None, :]
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)

    def fused():
        for (ks, vs, _), (q, k, v) in zip(layers, toks):
            qr = append_rotary(ks, vs, q, k, v, cos, sin)
            fc.codec_decode_attention(qr, ks, vs)

    def unfused():
        for (ks, vs, _), (q, k, v) in zip(layers, toks):
            qr, kr = apply_rotary_pos_emb(q, k, cos, sin)
            ks.append(kr)
            vs.append(v)
            fc.codec_decode_attention(qr, ks, vs)

    def timed(fn):
        stream = torch.cuda.current_stream(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        torch.cuda.synchronize()
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in ev)

    for _ in range(args.warmup):
        fused()
        unfused()
    sampler = ClockSampler([0])
    sampler.start()
    time.sleep(0.5)
    t0 = time.time()
    torch.cuda.nvtx.range_push("fused")
    ms_f = timed(fused)
    torch.cuda.nvtx.range_pop()
    torch.cuda.nvtx.range_push("unfused")
    ms_u = timed(unfused)
    torch.cuda.nvtx.range_pop()
    clocks = sampler.stop(t0, time.time())
    assert K.attn_status(dev) == 0, "a bounded wait in the attention kernel gave up"
    L = len(layers)
    per_attn = codec_attn_bytes(cfg, layers[0][0].n_blocks)
    line = {"metric": "decode-step tokens/s (rotary + append + archive decode attention, "
                      f"{L} layers)",
            "value": B / (ms_f * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms_f, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 2 decode step, attention side: rotary embedding of "
                                   "q/k, KV append (archive on block completion), decode "
                                   "attention, per layer",
                       "layers": L, "batch": B, "Hq": Hq, "Hkv": Hk, "head_dim": D,
                       "context": cfg["S"], "codec": "jpeg r=8 K=4 int8, fp32 scales",
                       "l2": "no flush: the archives read each step (~20 GB) are >100x L2"},
            "unfused": {"ms_per_step": ms_u, "tokens_per_s": B / (ms_u * 1e-3),
                        "sequence": "apply_rotary_pos_emb + 2 appends + attention"},
            "speedup_vs_unfused": ms_u / ms_f,
            "attention_bytes_per_step": per_attn * L,
            "gpu_launches": steps * L * 2 + steps * L * 2 // cfg["r"],
            "clocks": clocks}
    print(json.dumps(line), flush=True)


def workload_config(cfg, world):
    name = ("config 2: Qwen3-8B-shaped decode, 36 layers, one split-K decode-attention "
            "launch per layer over the int8 DCT archive") if cfg["config"] == 2 else (
            "config 5: long-context decode, batch-sharded (16 sequences per GPU = global 128 "
            "at 8 GPUs), S=131072, 8 layer archives, one split-K decode-attention launch per layer")
    codec = cfg.get("codec", "jpeg-int8")
    if codec == "jpeg-fp":
        name = name.replace("int8 DCT archive", "unquantized DCT archive (bf16 coefficients)")
        desc = f"jpeg r={cfg['r']} K={cfg['K']} quant_bits=0, bf16 coefficients"
    elif codec == "png":
        name = name.replace("int8 DCT archive", "png archive (bf16 anchors + fp32 deltas)")
        name = name.replace("36 layers", f"{cfg['layers']} layers")
        desc = f"png r={cfg['r']} keep_ratio=1.0"
    else:
        desc = f"jpeg r={cfg['r']} K={cfg['K']} int8, {cfg['scale_dtype']} scales"
    return {"workload": name,
            "layers": cfg["layers"], "batch_per_gpu": cfg["B"], "global_batch": cfg["B"] * world,
            "Hq": cfg["Hq"], "Hkv": cfg["Hk"], "head_dim": cfg["D"], "context": cfg["S"],
            "raw_tail": cfg["tail"],
            "codec": desc,
            "kv_dtype": "bf16", "parallelism": f"batch-sharded x{world} (no collective)",
            "l2": "no flush: the archive read each step (>8 GB per GPU) is >60x L2"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="flashcodec_b200", choices=["flashcodec_b200", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=(2, 5),
                    help="attention workload: config 2 (default, the headline) or config 5")
    ap.add_argument("--layers", type=int, default=None,
                    help="layers (default 36; fewer only for profiling a small case)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (default 16; smaller only for profiling)")
    ap.add_argument("--codec", default="jpeg-int8", choices=("jpeg-int8", "jpeg-fp", "png"),
                    help="archive format of the attention workload: jpeg-int8 (default, the "
                         "headline), jpeg-fp (quant_bits=0, bf16 coefficients) or png "
                         "(r=8, lossless; 4 layers by default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="attention", choices=("attention",) + CODEC_WORKLOADS,
                    help="attention (default, config 2) or one codec kernel's HBM throughput")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload != "attention":
        if args.impl == "reference":
            raise SystemExit("--impl reference times the attention workload")
        if args.workload == "stream":
            run_stream(args)
        elif args.workload == "decode-step":
            run_decode_step(args)
        else:
            run_codec(args)
        return
    base = CFG2 if args.config == 2 else CFG5
    cfg = dict(base, layers=args.layers or base["layers"], B=args.batch or base["B"],
               codec=args.codec)
    if args.codec != "jpeg-int8":
        if args.impl == "reference" or args.gpus != 1:
            raise SystemExit("--codec other than jpeg-int8 is a 1-GPU secondary line")
        if args.codec == "png" and not args.layers:
            cfg["layers"] = 4        # ~4 GB of fp32 deltas per layer
    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import flashcodec_b200 as fc
    from flashcodec_b200 import _kernels as K
    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layers = build_layers(cfg, rank, dev)
    n = layers[0][0].n_blocks
    per_launch = codec_attn_bytes(cfg, n)
    outs = [torch.empty_like(q) for _, _, q in layers]

    def step():
        for i, (ks, vs, q) in enumerate(layers):
            outs[i] = fc.codec_decode_attention(q, ks, vs)

    for _ in range(args.warmup):
        step()
    sampler = ClockSampler(list(range(max(world, 1)))) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    stream = torch.cuda.current_stream(dev)
    # The attention launches run back to back as a model issues them (no
    # event between them, so each launch may be scheduled while the previous
    # one drains); the kernel's average launch duration is the timed region
    # divided by the launches in it (nothing else runs in the region).
    barrier(world)
    t_wall0 = time.time()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    torch.cuda.nvtx.range_push("timed")
    for _ in range(args.steps):
        for i, (ks, vs, q) in enumerate(layers):
            outs[i] = fc.codec_decode_attention(q, ks, vs)
    torch.cuda.nvtx.range_pop()
    end.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    barrier(world)
    ms = start.elapsed_time(end) / args.steps
    kern_ms = ms / len(layers)
    ms_max = max_over_ranks(ms, world)
    kern_max = max_over_ranks(kern_ms, world)
    clocks = sampler.stop(t_wall0, t_wall1) if sampler else None
    assert K.attn_status(dev) == 0, "a bounded wait in the attention kernel gave up"

    # end to end through the public API with host buffers: H2D of every
    # layer's query from pinned memory, the attention calls, D2H of outputs
    qh = torch.stack([q for _, _, q in layers]).cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    qd = torch.empty_like(qh, device=dev)
    for _ in range(2):
        qd.copy_(qh, non_blocking=True)
        for i, (ks, vs, _) in enumerate(layers):
            outs[i] = fc.codec_decode_attention(qd[i], ks, vs)
        oh.copy_(torch.stack(outs), non_blocking=True)
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(1, args.steps // 3)
    e_start.record(stream)
    for _ in range(e_steps):
        qd.copy_(qh, non_blocking=True)
        for i, (ks, vs, _) in enumerate(layers):
            outs[i] = fc.codec_decode_attention(qd[i], ks, vs)
        oh.copy_(torch.stack(outs), non_blocking=True)
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e_ms = max_over_ranks(e_start.elapsed_time(e_end) / e_steps, world)

    cpu = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and cfg["config"] == 2
            and cfg["codec"] == "jpeg-int8"):
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        cpu = time_cpu_baseline(cpu_sample_from(layers, cfg), cfg, reps=5, threads=threads)

    if rank == 0:
        peak, kind = measured_peaks()
        achieved = per_launch / (kern_max * 1e-3) / 1e9
        traffic = (ncu_traffic() if cfg["config"] == 2 and cfg["B"] == CFG2["B"]
                   and cfg["codec"] == "jpeg-int8" else None)
        line = {
            "metric": METRIC if cfg["codec"] == "jpeg-int8" else
            f"decode-attn tokens/s & achieved HBM GB/s (% of peak) on {cfg['codec']} KV, 1 B200",
            "value": world * cfg["B"] / (ms_max * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": workload_config(cfg, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": per_launch,
                         "kernel_ms": kern_max},
            "cpu_baseline": cpu,
            "e2e": {"value": world * cfg["B"] / (e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": qh.numel() * qh.element_size(),
                    "d2h_bytes_per_step": oh.numel() * oh.element_size(),
                    "ms_per_step": e_ms},
            "gpu_launches": args.steps * len(layers),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    main()
