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
