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
    jpeg-int8 (codes + scales), jpeg-int8-g32 (codes + one scale per 32
    channels), jpeg-fp (bf16 coefficients, quant_bits=0) or png (bf16 anchor
    + fp32 deltas per block)."""
    codec = cfg.get("codec", "jpeg-int8")
    B, Hq, Hk, D, tail = cfg["B"], cfg["Hq"], cfg["Hk"], cfg["D"], cfg["tail"]
    if codec == "jpeg-int8":
        return attn_bytes(B, Hq, Hk, D, n, cfg["K"], tail,
                          scale_b=2 if cfg["scale_dtype"] == "fp16" else 4)
    if codec == "jpeg-int8-g32":   # one scale per 32 channels of a kept frequency row
        return attn_bytes(B, Hq, Hk, D, n, cfg["K"], tail,
                          scale_b=(D // 32) * (2 if cfg["scale_dtype"] == "fp16" else 4))
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


def ncu_traffic(per_launch, codec="jpeg-int8"):
    """Per-launch DRAM bytes (read + write) of the attention kernel at this
    workload, from the committed one-kernel ncu capture of a small case of
    the same codec (profiles/attn_decode_cfg2.json, int8 codes;
    profiles/attn_decode_cfg2_fp.json, bf16 coefficients): its measured bytes
    per algorithmic byte times this launch's algorithmic bytes (the kernel
    streams each archive byte once, so traffic grows in proportion), or
    None."""
    name = {"jpeg-int8": "attn_decode_cfg2.json", "jpeg-fp": "attn_decode_cfg2_fp.json"}.get(codec)
    if name is None:
        return None
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d["dram_bytes_per_launch"] / d["algorithmic_bytes_per_launch"] * per_launch
    except Exception:
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


def make_bench_codec(cfg):
    import flashcodec_b200 as fc
    codec = cfg.get("codec", "jpeg-int8")
    if codec == "png":
        return fc.make_codec("png", block_size=cfg["r"], keep_ratio=1.0)
    return fc.make_codec("jpeg", block_size=cfg["r"], keep_freqs=cfg["K"],
                         quant_bits=0 if codec == "jpeg-fp" else 8,
                         scale_dtype=torch.float16 if cfg["scale_dtype"] == "fp16"
                         else torch.float32,
                         group_size=32 if codec == "jpeg-int8-g32" else None)


def _fill_rows(st, b0, x):
    """Archive x (b, H, S, D) into rows b0:b0+b of a preallocated stream (the
    same kernels and slots as ``_CodecStream.append``)."""
    from flashcodec_b200 import _kernels as K
    from flashcodec_b200.codecs.jpeg import device_basis
    r, b = st.block_size, x.shape[0]
    n = st.n_blocks
    rows = slice(b0, b0 + b)
    if st.codec.name == "jpeg":
        k = st.codec.keep_freqs
        basis = device_basis(r, k, x.device)
        if getattr(st.codec, "group_size", None) is not None:
            K.jpeg_encode_grouped(x[:, :, :n * r], basis, r, k, st._coeffs[rows, :, :n],
                                  st._scales[rows, :, :n], st.codec.group_size)
        else:
            K.jpeg_encode(x[:, :, :n * r], basis, r, k, st._coeffs[rows, :, :n],
                          st._scales[rows, :, :n] if st.codec.quantized else None)
    else:
        K.png_encode(x[:, :, :n * r], r, st.codec.keep_m, st._deltas[rows, :, :n],
                     st._anchors[rows, :, :n])
    if st._raw_len:
        st._raw_buf[rows, :, :st._raw_len].copy_(x[:, :, n * r:])


CHUNK = 16   # sequences generated (and seeded) together


def build_layers(cfg, device, rows, heads=None, Bg=None):
    """Archive every layer's synthetic K/V for global batch rows
    [rows[0], rows[1]) and KV heads [heads[0], heads[1]) (default all) through
    the product's archive kernels; returns [(k_stream, v_stream, q)].

    The global batch is generated in chunks of CHUNK sequences, chunk c of
    layer L from seed 1000 * c + L, so a row holds the same data whichever
    rank owns it (weak, strong and head-split runs agree row by row)."""
    import flashcodec_b200 as fc
    Hq, Hk, D, r = cfg["Hq"], cfg["Hk"], cfg["D"], cfg["r"]
    G = Hq // Hk
    Bg = Bg or rows[1]
    h0, h1 = heads or (0, Hk)
    b0, b1 = rows
    S = cfg["S"] + cfg["tail"]
    n, t = S // r, S % r
    layers = []
    for L in range(cfg["layers"]):
        codec = make_bench_codec(cfg)
        pair = []
        like = torch.empty(b1 - b0, h1 - h0, 0, D, dtype=torch.bfloat16, device=device)
        for _ in range(2):
            st = fc._CodecStream(codec)
            st.meta, st.dtype = (b1 - b0, h1 - h0, D, 2), torch.bfloat16
            st._grow(n, like)
            st.n_blocks, st.n_archived = n, n * r
            if t:
                st._ensure_raw(like)
                st._raw_len = t
            pair.append(st)
        qs = []
        for c in range(b0 // CHUNK, (b1 - 1) // CHUNK + 1):
            c0, c1 = c * CHUNK, min((c + 1) * CHUNK, Bg)
            k, v, q = synth_case(c1 - c0, Hq, Hk, S, D, cfg["rho"], 1000 * c + L, device=device,
                                 dtype=torch.bfloat16)
            lo, hi = max(b0, c0), min(b1, c1)
            sel = slice(lo - c0, hi - c0)
            for st, x in zip(pair, (k, v)):
                _fill_rows(st, lo - b0, x[sel, h0:h1])
            qs.append(q[sel, h0 * G:h1 * G])
            del k, v
        layers.append((pair[0], pair[1], torch.cat(qs).contiguous()))
    torch.cuda.synchronize()
    return layers


def check_outputs(layers, outs, which, b=0):
    """The checker, outside every timed region: sequence b of the given layers
    against the fp64 CPU oracle on the archive rows read back from the device.
    Bound: 2e-3 + one bf16 rounding of the output (2^-8 relative), the
    attention parity bar for bf16 outputs."""
    import numpy as np
    from oracle import oracle as orc
    import flashcodec_b200 as fc
    f = lambda x: x.float().cpu().numpy()  # noqa: E731
    worst, ok = 0.0, True
    for i in which:
        ks, vs, q = layers[i]
        n, sel = ks.n_blocks, slice(b, b + 1)
        rows = {}
        for nm, st in (("k", ks), ("v", vs)):
            if st.codec.name == "png":
                rows[nm] = orc.stored_rows("png", anchors=f(st._anchors[sel, :, :n]),
                                           deltas=f(st._deltas[sel, :, :n]))
            elif getattr(st.codec, "group_size", None) is not None:
                rows[nm] = orc.dequantize_grouped(st._coeffs[sel, :, :n].cpu().numpy(),
                                                  f(st._scales[sel, :, :n]))
            elif st.codec.quantized:
                rows[nm] = orc.stored_rows("jpeg", codes=f(st._coeffs[sel, :, :n]),
                                           scales=f(st._scales[sel, :, :n]))
            else:
                rows[nm] = orc.stored_rows("jpeg", codes=f(st._coeffs[sel, :, :n]))
            rows[nm + "raw"] = f(st.raw[sel]) if st.raw is not None else None
        A = f(fc.block_basis(ks.codec, ks.block_size))
        ref = orc.decode_attention(f(q[sel]), rows["k"], rows["v"], rows["kraw"], rows["vraw"], A)
        err = np.abs(f(outs[i][sel]) - ref)
        ok = ok and bool(np.all(err <= 2e-3 + 2.0 ** -8 * np.abs(ref)))
        worst = max(worst, float(err.max()))
    return {"checked": f"sequence {b} of layers {list(which)} vs the fp64 CPU oracle "
                       "(oracle.decode_attention) on the archive read back",
            "bound": "|out - ref| <= 2e-3 + 2^-8 |ref| (bf16 output)",
            "max_abs_err": worst, "pass": ok}


def cpu_sample_from(layers, cfg, b_sample=1):
    """Host copy of one layer's archive for b_sample sequences (oracle input)."""
    ks, vs, q = layers[0]
    n = ks.n_blocks
    out = {}
    for nm, st in (("k", ks), ("v", vs)):
        out[nm] = st._coeffs[:b_sample, :, :n].cpu().numpy()
        out[nm + "s"] = st._scales[:b_sample, :, :n].float().cpu().numpy()
        out[nm + "raw"] = st.raw[:b_sample].float().cpu().numpy() if st.raw is not None else None
    out["q"] = q[:b_sample].float().cpu().numpy()
    return out


def cpu_attention_call(sample, cfg):
    """(fn, args) of the timed CPU arm: the oracle's port of the reference's
    torch attention path, spread over every host thread."""
    from oracle import oracle as orc
    import flashcodec_b200 as fc
    A = fc.block_basis(fc.make_codec("jpeg", block_size=cfg["r"], keep_freqs=cfg["K"]),
                       cfg["r"]).numpy()
    threads = os.cpu_count() or 1
    args = (sample["q"], sample["k"], sample["ks"], sample["v"], sample["vs"], sample["kraw"],
            sample["vraw"], A)
    return (lambda: orc.reference_attention_int8_mt(*args, threads=threads)), threads


CPU_SAMPLE_DESC = ("one layer of the step, sequence 0 of {B}, all {Hk} KV heads, full context "
                   "({n} blocks + {t} raw): oracle.reference_attention_int8_mt, the port of the "
                   "reference's torch path (fp32 dequantize, q.rows, expansion through A, fp32 "
                   "softmax, fold back, weighted V sum) on {threads} host threads; "
                   "tokens/s = 1 / ({layers} layers x sample time)")


def time_cpu_baseline(sample, cfg, reps):
    """Time the CPU arm on a bounded sample (one layer, one sequence) on the
    host cores; tokens/s = 1 / (layers x time)."""
    fn, threads = cpu_attention_call(sample, cfg)
    fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    n = sample["k"].shape[2]
    tail = 0 if sample["kraw"] is None else sample["kraw"].shape[2]
    nbytes = attn_bytes(1, cfg["Hq"], cfg["Hk"], cfg["D"], n, cfg["K"], tail)
    return {"value": 1.0 / (cfg["layers"] * t), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": CPU_SAMPLE_DESC.format(B=cfg["B"], Hk=cfg["Hk"], n=n, t=tail,
                                             threads=threads, layers=cfg["layers"])
            + f"; median of {reps} = {t * 1e3:.1f} ms ({nbytes / t / 1e9:.2f} GB/s of "
              "compressed bytes)"}


def run_reference(args, cfg):
    """--impl reference: the reference algorithm's CPU implementation (the
    oracle's port of its torch path) on the host cores, same metric, unit and
    workload.  The reference is Python: it does not travel to the GPU box, so
    its arithmetic runs as the port.  Each step is one bounded sample of the
    workload (one layer, one sequence, full context) and ms_per_step is that
    sample's measured time; tokens/s = 1 / (layers x step time).  Under
    torchrun only rank 0 runs (one host's cores; the value does not grow
    with --gpus)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return
    from oracle import oracle as orc
    import flashcodec_b200 as fc
    k, v, q = synth_case(1, cfg["Hq"], cfg["Hk"], cfg["S"] + cfg["tail"], cfg["D"], cfg["rho"],
                         0, dtype=torch.bfloat16)
    basis = fc.dct_basis(cfg["r"], cfg["K"]).numpy()
    n = cfg["S"] // cfg["r"]
    sample = {"q": q.float().numpy()}
    for nm, x in (("k", k), ("v", v)):
        xn = x.float().numpy()
        coef = orc.jpeg_encode(xn[:, :, :n * cfg["r"]], cfg["r"], cfg["K"], basis, "bf16")
        sample[nm], sample[nm + "s"] = orc.jpeg_quantize(coef, "bf16")
        sample[nm + "raw"] = xn[:, :, n * cfg["r"]:] if cfg["tail"] else None
    fn, threads = cpu_attention_call(sample, cfg)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = 1.0 / (cfg["layers"] * dt)
    desc = CPU_SAMPLE_DESC.format(B=cfg["B"], Hk=cfg["Hk"], n=n, t=cfg["tail"], threads=threads,
                                  layers=cfg["layers"])
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic",
            "config": workload_config(cfg, world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                             "kind": "port",
                             "sample": "each step: " + desc + "; ms_per_step is the measured "
                                       "time of that sample (one host's cores, the same for "
                                       "every --gpus)"},
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
    CUDA events around every step (host launch overhead included).  Three
    ways to append the step's 56 tokens: one fc_append_tokens launch for all
    layers (CodecKVCache.append_layers, the headline of this line), one launch
    per layer (CodecKVCache.append), and one append per stream (the stream's
    own append: a copy per token plus an archive launch per completed block)."""
    import flashcodec_b200 as fc
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L, B, H, D, S_end, W = 28, 64, 8, 128, 65536, 256
    g = torch.Generator(device=dev).manual_seed(4)
    toks = [(torch.randn(B, H, 1, D, generator=g, device=dev).to(torch.bfloat16),
             torch.randn(B, H, 1, D, generator=g, device=dev).to(torch.bfloat16)) for _ in range(L)]
    kt, vt = [k for k, _ in toks], [v for _, v in toks]

    def step_all(cache):
        cache.append_layers(kt, vt)

    def step_layer(cache):
        for i in range(L):
            cache.append(kt[i], vt[i], i)

    def step_stream(cache):
        for i in range(L):
            cache._keys[i].append(kt[i])
            cache._values[i].append(vt[i])

    def window(cache, steps, fn):
        stream = torch.cuda.current_stream(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for a, b in ev:
            a.record(stream)
            fn(cache)
            cache._keys[0].read()
            b.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / steps * 1e3
        return statistics.mean(a.elapsed_time(b) for a, b in ev), wall

    def new_cache():
        c = fc.CodecKVCache("jpeg", block_size=8, keep_freqs=2, quant_bits=8)
        for i in range(L):  # first token: allocate the streams
            c.append(kt[i], vt[i], i)
        return c

    modes = (("one launch per step", step_all), ("one launch per layer", step_layer),
             ("one append per stream", step_stream))
    res = {}
    for name, fn in modes:
        c0 = new_cache()
        window(c0, 16, fn)           # warm-up (kernels loaded, first archives)
        del c0
        c1 = new_cache()
        res[name] = {"start": window(c1, W, fn)}
        del c1
    torch.cuda.empty_cache()
    c2 = fc.CodecKVCache("jpeg", block_size=8, keep_freqs=2, quant_bits=8)
    S_pre = S_end - W * len(modes)
    for i in range(L):
        k = synth_stream(B, H, S_pre, D, 0.95, 2 * i, device=dev, dtype=torch.bfloat16)
        c2.append(k, k, i)  # value content does not change the work
        del k
    c2._keys[0].read()
    for name, fn in modes:
        res[name]["end"] = window(c2, W, fn)
    head = res["one launch per step"]
    end_ms = head["end"][0]
    detail = {name: {"window_start_ms_per_step": v["start"][0],
                     "window_start_wall_ms_per_step": v["start"][1],
                     "window_end_ms_per_step": v["end"][0],
                     "window_end_wall_ms_per_step": v["end"][1]} for name, v in res.items()}
    line = {"metric": "config 4 streaming step (append 28 layers + incremental read of one layer)",
            "value": end_ms, "unit": "ms/step", "n_gpus": 1, "steps": W, "warmup": 16,
            "ms_per_step": end_ms, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 4: Qwen3-0.6B-shaped streaming append/archive",
                       "layers": L, "batch": B, "Hkv": H, "head_dim": D,
                       "codec": "jpeg r=8 K=2 int8, fp32 scales",
                       "windows": {"start": [0, W], "end": [S_end - W, S_end]},
                       "timing": "CUDA events around each step on the current stream"},
            "append_modes": detail,
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
    layers = build_layers(cfg, dev, (0, cfg["B"]))
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


def workload_config(cfg, world, plan=None, Bg=None):
    if cfg["config"] == 2:
        name = ("config 2: Qwen3-8B-shaped decode, 36 layers, one split-K decode-attention "
                "launch per layer over the int8 DCT archive")
    elif plan is None:
        name = ("config 5: long-context decode, batch-sharded (16 sequences per GPU = global "
                "128 at 8 GPUs), S=131072, 8 layer archives, one split-K decode-attention "
                "launch per layer")
    else:
        name = (f"config 5: long-context decode, global batch {Bg} sharded over {world} GPU(s), "
                "S=131072, 8 layer archives, one split-K decode-attention launch per layer")
    codec = cfg.get("codec", "jpeg-int8")
    if codec == "jpeg-fp":
        name = name.replace("int8 DCT archive", "unquantized DCT archive (bf16 coefficients)")
        desc = f"jpeg r={cfg['r']} K={cfg['K']} quant_bits=0, bf16 coefficients"
    elif codec == "jpeg-int8-g32":
        name = name.replace("int8 DCT archive", "int8 DCT archive with one scale per 32 channels")
        desc = f"jpeg r={cfg['r']} K={cfg['K']} int8, {cfg['scale_dtype']} scales per 32 channels"
    elif codec == "png":
        name = name.replace("int8 DCT archive", "png archive (bf16 anchors + fp32 deltas)")
        name = name.replace("36 layers", f"{cfg['layers']} layers")
        desc = f"png r={cfg['r']} keep_ratio=1.0"
    else:
        desc = f"jpeg r={cfg['r']} K={cfg['K']} int8, {cfg['scale_dtype']} scales"
    if plan is None:
        par = f"batch-sharded x{world} (no collective), {cfg['B']} sequences per GPU"
        gb, per = cfg["B"] * world, cfg["B"]
    elif plan.mode == "batch":
        par = f"batch-sharded x{world} (no collective), global batch {Bg}"
        gb, per = Bg, f"{Bg // world}-{-(-Bg // world)}"
    else:
        par = (f"KV-head-sharded x{world}: {world // Bg} ranks per sequence, "
               f"{cfg['Hk'] // (world // Bg)} KV heads each; one NCCL all_gather of the "
               "(B, Hq_local, 1, D) outputs per layer inside the step")
        gb, per = Bg, f"1 sequence, {cfg['Hk'] // (world // Bg)} of {cfg['Hk']} KV heads"
    return {"workload": name,
            "layers": cfg["layers"], "batch_per_gpu": per, "global_batch": gb,
            "Hq": cfg["Hq"], "Hkv": cfg["Hk"], "head_dim": cfg["D"], "context": cfg["S"],
            "raw_tail": cfg["tail"],
            "codec": desc,
            "kv_dtype": "bf16", "parallelism": par,
            "l2": "no flush: the archives read each step are larger than L2 "
                  "(> 8 GB per GPU at the default sizes)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="flashcodec_b200", choices=["flashcodec_b200", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=(2, 5),
                    help="attention workload: config 2 (default, the headline) or config 5")
    ap.add_argument("--layers", type=int, default=None,
                    help="layers (default 36 / 8; fewer only for profiling a small case)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU in weak scaling (default 16; smaller only for "
                         "profiling)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="strong scaling: this many sequences in total, sharded over the GPUs "
                         "by batch (>= GPUs) or by KV head (< GPUs; one NCCL all_gather of "
                         "outputs per layer)")
    ap.add_argument("--codec", default="jpeg-int8",
                    choices=("jpeg-int8", "jpeg-int8-g32", "jpeg-fp", "png"),
                    help="archive format of the attention workload: jpeg-int8 (default, the "
                         "headline), jpeg-int8-g32 (one scale per 32 channels), jpeg-fp "
                         "(quant_bits=0, bf16 coefficients) or png "
                         "(r=8, lossless; 4 layers by default)")
    ap.add_argument("--gather", default="peer", choices=("peer", "nccl"),
                    help="with split KV heads: peer (default) -- the attention kernel stores "
                         "every output row into each rank's buffer over NVLink and publishes an "
                         "epoch flag, one bounded wait per layer (fc_decode_attn_peers); nccl -- "
                         "the kernel, then one NCCL all_gather per layer")
    ap.add_argument("--graph", action="store_true",
                    help="time the step as a CUDA graph replay of its launches (captured once "
                         "after warm-up, with split heads including the gathers: NCCL calls, or "
                         "the peer waits, whose epochs come from a device counter); the oracle "
                         "check and e2e stay eager")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the post-timing oracle check (profiling runs only)")
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
    from flashcodec_b200 import sharding
    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    Hk, G = cfg["Hk"], cfg["Hq"] // cfg["Hk"]
    plan, Bg = None, None
    if args.global_batch:
        Bg = args.global_batch
        plan = sharding.plan_shards(Bg, Hk, cfg["Hq"], world)
        rows, heads = plan.batch_range(rank), plan.kv_head_range(rank)
    else:
        rows, heads = (rank * cfg["B"], (rank + 1) * cfg["B"]), (0, Hk)
    gather = plan is not None and plan.needs_gather()
    peer = gather and args.gather == "peer"
    layers = build_layers(cfg, dev, rows, heads, Bg=Bg or world * cfg["B"])
    # peer outputs: two slots per layer, alternating by step, so a rank never
    # stores into a buffer a peer may still be copying out from the step before
    po = (sharding.PeerOutputs(plan, rank, 2 * len(layers), cfg["D"], layers[0][2].dtype, dev)
          if peer else None)
    parity = [0]
    n = layers[0][0].n_blocks
    local_cfg = dict(cfg, B=rows[1] - rows[0], Hk=heads[1] - heads[0],
                     Hq=(heads[1] - heads[0]) * G)
    per_launch = codec_attn_bytes(local_cfg, n)
    outs = [None] * len(layers)
    full = [None] * len(layers)

    def step(with_gather=gather):
        if with_gather and peer:
            base = parity[0] * len(layers)
            for i, (ks, vs, q) in enumerate(layers):
                full[i] = po.decode(q, ks, vs, slot=base + i)
            parity[0] ^= 1
            return
        for i, (ks, vs, q) in enumerate(layers):
            outs[i] = fc.codec_decode_attention(q, ks, vs)
            if with_gather:
                full[i] = sharding.gather_outputs(plan, outs[i])

    graphs = {}   # with_gather -> CUDA graph of one step (--graph)

    def timed(steps, with_gather=gather):
        stream = torch.cuda.current_stream(dev)
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            if with_gather in graphs:
                graphs[with_gather].replay()
            else:
                step(with_gather)
        end.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return start.elapsed_time(end) / steps

    for _ in range(args.warmup):
        step()
    if args.graph:
        # one step's launches (and, with split heads, its NCCL all-gathers)
        # captured once after the warm-up -- the kernels' shared-memory
        # opt-ins and the communicator exist by then -- and replayed as one
        # graph per step; every rank captures the same collectives in order
        for wg in ([True, False] if gather else [False]):
            torch.cuda.synchronize()
            barrier(world)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(wg)
            graphs[wg] = g
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize()
        barrier(world)
    sampler = ClockSampler(list(range(max(world, 1)))) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    # The attention launches run back to back as a model issues them (no
    # event between them, so each launch may be scheduled while the previous
    # one drains); the kernel's average launch duration is the timed region
    # divided by the launches in it (nothing else runs in the region unless
    # the heads are split, where each layer adds one all_gather).
    t_wall0 = time.time()
    torch.cuda.nvtx.range_push("timed")
    ms = timed(args.steps)
    torch.cuda.nvtx.range_pop()
    t_wall1 = time.time()
    clocks = sampler.stop(t_wall0, t_wall1) if sampler else None
    ms_max = max_over_ranks(ms, world)
    ms_compute = max_over_ranks(timed(max(1, args.steps // 2), False), world) if gather else ms_max
    kern_max = ms_compute / len(layers)
    # status words of every workspace used (the graph's capture stream has its own)
    status = max([int(w[:4].view(torch.int32).item()) for w in K._workspaces.values()] or [0])

    # end to end through the public API with host buffers: every step copies
    # each layer's query from pinned host memory (H2D) and reads each layer's
    # output back (D2H).  The copies run on two copy streams, layer by layer,
    # so they overlap the attention launches of the other layers; the timed
    # region ends when the last output has landed in host memory.
    qh = torch.stack([q for _, _, q in layers]).cpu().pin_memory()
    res = full if gather else outs
    oh = torch.empty((len(layers),) + tuple(res[0].shape), dtype=res[0].dtype).pin_memory()
    qd = torch.empty_like(qh, device=dev)
    stream = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    nl = len(layers)
    ev_in = [torch.cuda.Event() for _ in range(nl)]
    ev_done = [torch.cuda.Event() for _ in range(nl)]
    ev_copied = [torch.cuda.Event() for _ in range(nl)]
    first = [True]

    def e2e_step():
        for i in range(nl):
            with torch.cuda.stream(s_in):
                if not first[0]:
                    s_in.wait_event(ev_done[i])     # the last step's attention read qd[i]
                qd[i].copy_(qh[i], non_blocking=True)
                ev_in[i].record(s_in)
        base = parity[0] * nl
        for i, (ks, vs, _) in enumerate(layers):
            stream.wait_event(ev_in[i])
            if peer:
                if not first[0]:
                    # this rank publishes layer i only after its copy of the
                    # last step's layer-i output has left the other slot
                    stream.wait_event(ev_copied[i])
                full[i] = po.decode(qd[i], ks, vs, slot=base + i)
            else:
                outs[i] = fc.codec_decode_attention(qd[i], ks, vs)
                if gather:
                    full[i] = sharding.gather_outputs(plan, outs[i])
            r = full[i] if gather else outs[i]
            ev_done[i].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[i])
                oh[i].copy_(r, non_blocking=True)
                r.record_stream(s_out)
                ev_copied[i].record(s_out)
        parity[0] ^= 1
        first[0] = False

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(5, args.steps // 2)
    e_start.record(stream)
    s_in.wait_event(e_start)
    for _ in range(e_steps):
        e2e_step()
    stream.wait_stream(s_out)
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e_ms = max_over_ranks(e_start.elapsed_time(e_end) / e_steps, world)

    # the checker (outside the timed regions): sequence 0 of this rank's first
    # and last layer against the fp64 oracle; with split heads also that the
    # gathered output holds this rank's piece where the plan puts it
    check = None
    if not args.no_check:
        step()
        if peer:   # this rank's pieces from the plain kernel, to check the placement
            for i, (ks, vs, q) in enumerate(layers):
                outs[i] = fc.codec_decode_attention(q, ks, vs)
        torch.cuda.synchronize()
        check = check_outputs(layers, outs, sorted({0, len(layers) - 1}))
        if gather:
            b0, b1 = rows
            q0, q1 = heads[0] * G, heads[1] * G
            placed = all(torch.equal(full[i][b0:b1, q0:q1], outs[i]) for i in range(len(layers)))
            check["gather_placement"] = placed
            check["pass"] = check["pass"] and placed
        bad = max_over_ranks(0.0 if check["pass"] else 1.0, world)
        check["pass"] = bad == 0.0
        check["ranks"] = world
        check["status_word"] = status

    cpu = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and cfg["config"] == 2
            and cfg["codec"] == "jpeg-int8"):
        cpu = time_cpu_baseline(cpu_sample_from(layers, cfg), cfg, reps=5)

    if rank == 0:
        peak, kind = measured_peaks()
        achieved = per_launch / (kern_max * 1e-3) / 1e9
        traffic = (ncu_traffic(per_launch, cfg["codec"]) if cfg["config"] == 2 and plan is None
                   and cfg["B"] == CFG2["B"] else None)
        tokens = Bg if plan is not None else world * cfg["B"]
        line = {
            "metric": METRIC if cfg["codec"] == "jpeg-int8" else
            f"decode-attn tokens/s & achieved HBM GB/s (% of peak) on {cfg['codec']} KV, 1 B200",
            "value": tokens / (ms_max * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "strong" if plan is not None else "weak",
            "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic",
            "config": dict(workload_config(cfg, world, plan, Bg),
                           timed_as="CUDA graph replay of the step" if graphs
                           else "eager launches"),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": kind,
                         "traffic": traffic, "algorithmic_bytes_per_launch": per_launch,
                         "kernel_ms": kern_max,
                         "kernel": "attn_tc_kernel"
                         if cfg["codec"] in ("jpeg-int8", "jpeg-int8-g32", "jpeg-fp")
                         else "attn_kernel"},
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": qh.numel() * qh.element_size(),
                    "d2h_bytes_per_step": oh.numel() * oh.element_size(),
                    "ms_per_step": e_ms},
            "check": check,
            "gpu_launches": args.steps * len(layers) * (2 if peer else 1),
            "clocks": clocks,
        }
        if gather:
            g_ms = (ms_max - ms_compute) / len(layers)
            line["head_split"] = {
                "gather": ("peer stores from the attention kernel + one bounded flag wait per "
                           "layer (fc_decode_attn_peers, fc_peers_wait)" if peer
                           else "one NCCL all_gather per layer"),
                "allgather_ms_per_layer": g_ms, "allgather_share": (ms_max - ms_compute) / ms_max,
                "attention_ms_per_layer": kern_max,
                "allgather_bytes_per_rank_per_layer":
                    local_cfg["B"] * local_cfg["Hq"] * cfg["D"] * layers[0][2].element_size(),
                "note": "gather time = step time with the gather minus the step without it"}
        print(json.dumps(line), flush=True)
    graphs.clear()           # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    if po is not None:
        po.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if check is not None and not check["pass"]:
        raise SystemExit("decode attention output differs from the oracle (see the check field)")
    if status != 0:
        raise SystemExit(f"a bounded wait in the attention kernel gave up (launch {status})")


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    main()
