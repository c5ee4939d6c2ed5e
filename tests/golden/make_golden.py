"""Generate golden fixtures by running the reference flashcodec implementation.

Run from the repository root, in a container where the reference source tree
is available (it is not needed anywhere else):

    FLASHCODEC_REF=/path/to/flashcodec python tests/golden/make_golden.py

Writes tests/golden/golden.npz.  Every array is produced by the reference's own
public functions (``dct_basis``, ``dct_compress``, ``quantize_coeffs``,
``dct_decompress``, ``png_filter``, ``png_reconstruct``, ``_CodecStream``,
``codec_decode_attention(impl="torch")``) on CPU, on the seeded synthetic inputs
of tests/golden/cases.py.  Inputs are not stored: the tests regenerate them
from the same seeds and check them against the stored SHA-256 digests.  Values
of every dtype are stored as float32 (bf16/fp16 values are exact in fp32);
int8 codes as int8.

The large config-1 case (B=1, Hq=32, Hkv=8, S=4096, D=128, fp32, r=8, K=2,
int8) stores only SHA-256 digests of its codes and scales plus the attention
outputs.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))
if "FLASHCODEC_REF" not in os.environ:
    raise SystemExit("set FLASHCODEC_REF to the flashcodec source tree (the directory that "
                     "holds the flashcodec package) to regenerate the fixtures")
sys.path.insert(0, os.environ["FLASHCODEC_REF"])

import cases  # noqa: E402
from cases import f32, sha  # noqa: E402
from flashcodec import codec_decode_attention, dct_basis, dct_compress  # noqa: E402
from flashcodec.cache import _CodecStream, make_codec  # noqa: E402
from flashcodec.codecs import (dct_decompress, png_filter, png_reconstruct,  # noqa: E402
                               quantize_coeffs)

OUT: dict[str, np.ndarray] = {}
META: dict[str, dict] = {}


def put(name, arr):
    OUT[name] = arr


def put_sha(name, digest: str):
    OUT[name] = np.frombuffer(digest.encode(), np.uint8)


# ---------------------------------------------------------------- DCT bases
for r in (4, 8, 16, 32):
    put(f"basis_r{r}", f32(dct_basis(r, r)))

# ------------------------------------------------------------- jpeg codec
for i, (name, dt, B, H, S, D, r, k, qb) in enumerate(cases.JPEG_CASES):
    x = cases.jpeg_input(i)
    coef = dct_compress(x, r, k)
    put_sha(f"{name}/x_sha", sha(f32(x)))
    put(f"{name}/coef", f32(coef))
    put(f"{name}/rec_coef", f32(dct_decompress(coef, r, S)))
    if qb:
        q, s = quantize_coeffs(coef)
        put(f"{name}/codes", q.numpy())
        put(f"{name}/scales", f32(s))
        cd = make_codec("jpeg", block_size=r, keep_freqs=k, quant_bits=8)
        put(f"{name}/rec_q", f32(cd.decompress(q, out_len=S, scales=s)))
    # stream path: append everything, read the view back (cache.py:143-220)
    st = _CodecStream(make_codec("jpeg", block_size=r, keep_freqs=k, quant_bits=qb))
    st.append(x)
    n = st.n_blocks
    put(f"{name}/st_coeffs", st._coeffs[:, :, :n].numpy() if qb else f32(st._coeffs[:, :, :n]))
    if qb:
        put(f"{name}/st_scales", f32(st._scales[:, :, :n]))
    put(f"{name}/st_read", f32(st.read()))
    META[name] = dict(kind="jpeg", dtype=dt, B=B, H=H, S=S, D=D, r=r, k=k, quant=qb,
                      n_blocks=n, capacity=st._capacity, storage_bytes=st.storage_bytes())

# -------------------------------------------------------------- png codec
for i, (name, dt, B, H, S, D, r, keep) in enumerate(cases.PNG_CASES):
    x = cases.png_input(i)
    d, a = png_filter(x, r, keep)
    put_sha(f"{name}/x_sha", sha(f32(x)))
    put(f"{name}/deltas", f32(d))
    put(f"{name}/anchors", f32(a))
    put(f"{name}/rec", f32(png_reconstruct(d, a)))
    META[name] = dict(kind="png", dtype=dt, B=B, H=H, S=S, D=D, r=r, keep=keep)

# -------------------------------------------------------- decode attention
for i, (name, mode, kw, dt, B, Hk, G, S, D, tail) in enumerate(cases.ATTN_CASES):
    k, v, q = cases.attn_input(i)
    ks = _CodecStream(make_codec(mode, block_size=8, **kw))
    vs = _CodecStream(make_codec(mode, block_size=8, **kw))
    ks.append(k)
    vs.append(v)
    out = codec_decode_attention(q, ks, vs, impl="torch")
    put_sha(f"{name}/kvq_sha", sha(f32(k)) + sha(f32(v)) + sha(f32(q)))
    put(f"{name}/out", f32(out))
    # the same attention on fp32-upcast copies of the identical archive: the
    # fp32 arithmetic the kernels use, for the bf16 cases
    if dt != "f32":
        for st in (ks, vs):
            for attr in ("_coeffs", "_scales", "_deltas", "_anchors", "raw"):
                t = getattr(st, attr)
                if t is not None and t.is_floating_point():
                    setattr(st, attr, t.float())
        put(f"{name}/out_f32math", f32(codec_decode_attention(q.float(), ks, vs, impl="torch")))
    META[name] = dict(kind="attn", mode=mode, codec=kw, dtype=dt, B=B, Hk=Hk, G=G, S=S,
                      D=D, tail=tail, r=8)

# ------------------------------------------------ config 1 (full size, digests)
c = cases.CFG1
k, v, q = cases.cfg1_input()
digests = {"inputs": sha(f32(k)) + sha(f32(v)) + sha(f32(q))}
for t in (0, 1):
    ks = _CodecStream(make_codec("jpeg", block_size=8, keep_freqs=2, quant_bits=8))
    vs = _CodecStream(make_codec("jpeg", block_size=8, keep_freqs=2, quant_bits=8))
    ks.append(k[:, :, :c["S"] + t])
    vs.append(v[:, :, :c["S"] + t])
    n = ks.n_blocks
    digests[f"t{t}"] = dict(
        k_codes=sha(ks._coeffs[:, :, :n].numpy()), k_scales=sha(f32(ks._scales[:, :, :n])),
        v_codes=sha(vs._coeffs[:, :, :n].numpy()), v_scales=sha(f32(vs._scales[:, :, :n])),
        n_blocks=n)
    put(f"cfg1_t{t}/out", f32(codec_decode_attention(q, ks, vs, impl="torch")))
META["cfg1"] = dict(c, digests=digests)

OUT["__meta__"] = np.frombuffer(json.dumps(META, sort_keys=True).encode(), dtype=np.uint8)
dst = ROOT / "tests" / "golden" / "golden.npz"
np.savez_compressed(dst, **OUT)
print(f"wrote {dst} ({dst.stat().st_size / 1024:.0f} KiB, {len(OUT)} arrays)")
