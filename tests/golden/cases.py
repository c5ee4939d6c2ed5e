"""Golden case tables shared by make_golden.py (which runs the reference) and
the tests (which regenerate the same seeded inputs and compare)."""

from __future__ import annotations

import hashlib

import numpy as np
import torch

import bench

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

JPEG_CASES = [
    # name,        dtype, B, H,  S,  D,  r, k, quant
    ("j_f32_k2q", "f32", 2, 2, 64, 32, 8, 2, 8),
    ("j_f32_k4", "f32", 2, 2, 64, 32, 8, 4, 0),
    ("j_f32_pad", "f32", 2, 2, 50, 32, 8, 2, 8),
    ("j_f32_r16", "f32", 1, 2, 96, 96, 16, 4, 8),
    ("j_bf16_k2q", "bf16", 2, 2, 64, 32, 8, 2, 8),
    ("j_bf16_d128", "bf16", 1, 2, 64, 128, 8, 4, 8),
    ("j_bf16_k8q", "bf16", 1, 2, 80, 64, 8, 8, 8),
    ("j_bf16_k2", "bf16", 1, 2, 64, 64, 8, 2, 0),
    ("j_f16_k2q", "f16", 1, 2, 64, 64, 8, 2, 8),
]

PNG_CASES = [
    # name,           dtype, B, H,  S,   D,  r, keep
    ("p_f32", "f32", 2, 2, 64, 32, 8, 1.0),
    ("p_bf16", "bf16", 2, 2, 64, 32, 8, 1.0),
    ("p_f32_half", "f32", 2, 2, 64, 32, 8, 0.5),
    ("p_f32_quarter", "f32", 1, 2, 64, 32, 8, 0.25),
    ("p_f32_r16", "f32", 1, 2, 128, 64, 16, 1.0),
    ("p_f32_pad", "f32", 1, 2, 50, 32, 8, 1.0),
]

ATTN_CASES = [
    # name, mode, codec kwargs, dtype, B, Hk, G, S, D, tail
    ("a_jk2", "jpeg", dict(keep_freqs=2), "f32", 2, 4, 2, 96, 32, 0),
    ("a_jk8", "jpeg", dict(keep_freqs=8), "f32", 2, 4, 1, 96, 32, 3),
    ("a_jk2q", "jpeg", dict(keep_freqs=2, quant_bits=8), "f32", 2, 4, 2, 96, 32, 5),
    ("a_jk2q_g4", "jpeg", dict(keep_freqs=2, quant_bits=8), "f32", 1, 2, 4, 200, 128, 7),
    ("a_png1", "png", dict(keep_ratio=1.0), "f32", 2, 4, 2, 96, 32, 3),
    ("a_png05", "png", dict(keep_ratio=0.5), "f32", 2, 4, 1, 96, 32, 0),
    ("a_raw_only", "jpeg", dict(keep_freqs=2, quant_bits=8), "f32", 1, 2, 2, 0, 32, 5),
    ("a_bf16_k2q", "jpeg", dict(keep_freqs=2, quant_bits=8), "bf16", 1, 8, 2, 1024, 128, 0),
    ("a_bf16_k4", "jpeg", dict(keep_freqs=4), "bf16", 1, 8, 2, 1024, 128, 3),
    ("a_bf16_k4q_g4", "jpeg", dict(keep_freqs=4, quant_bits=8), "bf16", 2, 2, 4, 512, 128, 5),
]

# config 1 of the benchmark spec: the CPU-runnable jpeg round trip + decode step
CFG1 = dict(B=1, Hq=32, Hk=8, S=4096, D=128, r=8, k=2, rho=0.95, seed=0)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().cpu().numpy()


def jpeg_input(i: int) -> torch.Tensor:
    name, dt, B, H, S, D, r, k, qb = JPEG_CASES[i]
    return bench.synth_stream(B, H, S, D, 0.95, 100 + i, outliers=True, dtype=TD[dt])


def png_input(i: int) -> torch.Tensor:
    name, dt, B, H, S, D, r, keep = PNG_CASES[i]
    return bench.synth_stream(B, H, S, D, 0.98, 200 + i, dtype=TD[dt])


def attn_input(i: int):
    name, mode, kw, dt, B, Hk, G, S, D, tail = ATTN_CASES[i]
    return bench.synth_case(B, Hk * G, Hk, S + tail, D, 0.95, 300 + i, dtype=TD[dt])


def cfg1_input():
    c = CFG1
    return bench.synth_case(c["B"], c["Hq"], c["Hk"], c["S"] + 1, c["D"], c["rho"], c["seed"])
