"""Generate the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

Inputs are seeded synthetic K-quant blocks and activations (q35k.synth) plus
hand-made edge blocks; expected outputs come from the CPU oracle (oracle/):
Q8_K bytes, bit-exact dequantized values, and y from both the scalar
semantics and the AVX2 executed order of the reference's dispatch.  The
fixtures pin the oracle against regressions (tests/test_oracle.py) and give
the GPU parity tests fixed cases that need no oracle build.

The reference (C#/.NET) cannot run here and ships no golden vectors for
Q4_K/Q5_K/Q6_K, so these fixtures are NOT reference outputs: parity with the
reference is unpinned.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "qwen3.5sharp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402
from q35k import synth  # noqa: E402
from q35k.synth import Q4_K, Q5_K, Q6_K  # noqa: E402

TYPES = {Q4_K: "q4k", Q5_K: "q5k", Q6_K: "q6k"}


def edge_blocks(qtype: int) -> np.ndarray:
    """Hand-made blocks: zero scale, subnormal/negative scales, extreme
    nibbles and 6-bit scales."""
    bb = synth.BLOCK_BYTES[qtype]
    rows = []

    def blk(d=0x3C00, dmin=0x3C00, fill=0x00, scales=None, q6sc=None):
        b = np.full(bb, fill, dtype=np.uint8)
        if qtype == Q6_K:
            b[192:208] = np.array(q6sc if q6sc is not None else [1] * 16, dtype=np.int8).view(np.uint8)
            b[208:210] = np.array([d], dtype=np.uint16).view(np.uint8)
        else:
            b[0:2] = np.array([d], dtype=np.uint16).view(np.uint8)
            b[2:4] = np.array([dmin], dtype=np.uint16).view(np.uint8)
            b[4:16] = np.array(scales if scales is not None else [0x3F] * 12, dtype=np.uint8)
        return b

    rows.append(blk(d=0x0000, dmin=0x0000, fill=0xFF))              # zero scales
    rows.append(blk(d=0x0001, dmin=0x03FF, fill=0xA5))              # subnormal d / dmin
    rows.append(blk(d=0xBC00, dmin=0x8001, fill=0x5A))              # negative d, negative subnormal dmin
    rows.append(blk(d=0x7BFF, dmin=0x7BFF, fill=0xFF, scales=[0xFF] * 12, q6sc=[-32] * 16))  # max everything
    rows.append(blk(d=0x3C00, dmin=0x0000, fill=0x11, scales=[0x01] * 12, q6sc=[31] * 16))
    rows.append(blk(d=0x2E66, dmin=0x2E66, fill=0x00, scales=[0xC0, 0x40] * 6, q6sc=list(range(-8, 8))))
    rows.append(blk(d=0x3555, dmin=0x1234, fill=0xF0, scales=list(range(0, 240, 20)), q6sc=[-1, 1] * 8))
    rows.append(blk(d=0x0400, dmin=0x0400, fill=0x0F))              # smallest normal
    return np.stack(rows)


def edge_activations(k: int) -> np.ndarray:
    """Rows that stress Q8K.ScaleBlock's first-signed-extremum rule."""
    rng = np.random.default_rng(11)
    rows = []
    z = np.zeros(k, np.float32)
    rows.append(z)                                                   # all zero
    a = rng.standard_normal(k).astype(np.float32)
    a[5], a[200] = -3.5, 3.5                                         # tie, negative first
    rows.append(a)
    b = rng.standard_normal(k).astype(np.float32)
    b[17], b[18] = 4.25, -4.25                                       # tie, positive first
    rows.append(b)
    c = rng.standard_normal(k).astype(np.float32) * 1e-30            # tiny values
    rows.append(c)
    d = np.full(k, -2.0, np.float32)                                 # constant negative
    rows.append(d)
    e = (np.arange(k, dtype=np.float32) - k / 2) * 0.25              # ramp, max at the end
    rows.append(e)
    f = rng.standard_normal(k).astype(np.float32) * 1e4              # large
    f[0] = 0.0
    rows.append(f)
    g = np.zeros(k, np.float32)
    g[k - 1] = -1.0                                                  # single negative extremum
    rows.append(g)
    return np.stack(rows)


def cases():
    out = {}
    for qt, name in TYPES.items():
        # seeded small shapes: K=256/512, N in {1, 7, 17}, M in {1, 4, 9}
        for k, n, m in ((256, 1, 1), (512, 7, 4), (512, 17, 9), (256, 16, 2)):
            w = synth.kquant_blocks(qt, n, k, seed=100 + qt + n)
            x = synth.activations(m, k, seed=200 + m + k)
            out[f"{name}_k{k}_n{n}_m{m}"] = (qt, w, x)
        # edge blocks x edge activations (K=256: one block per row)
        w = edge_blocks(qt)
        x = edge_activations(256)
        out[f"{name}_edge"] = (qt, w, x)
    return out


def main():
    oracle.build()
    manifest = {}
    for key, (qt, w, x) in cases().items():
        n, k = w.shape[0], x.shape[1]
        W = oracle.Weight(qt, w, k, n)
        arr = dict(
            qtype=np.int32(qt), blocks=w, x=x,
            q8k=oracle.quantize_q8k(x, avx2=True),
            dequant=oracle.dequantize(qt, w, k),
            y_semantic=W.matmul_semantic(x),
            y_executed=W.matmul(x, threads=1),
        )
        path = os.path.join(HERE, f"{key}.npz")
        np.savez_compressed(path, **arr)
        manifest[key] = hashlib.sha256(open(path, "rb").read()).hexdigest()
        print(f"{key}: n={n} k={k} m={x.shape[0]}")
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
