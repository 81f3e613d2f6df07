"""Seeded synthetic inputs for the K-quant matmul path.

No model checkpoint, dataset or benchmark suite is involved: weights are
random K-quant super-blocks with the field distributions of the benchmark
configurations, activations are seeded normals.  Blocks are generated once on
the host and fed byte-identical to the GPU kernels and to the CPU reference.

PRNG: counter-based splitmix64 (output i = mix64(key + (i + 1) * golden)),
one independent stream per (seed, field) pair, so every field of every block
is reproducible from the seed alone and generation vectorises in numpy.
Normals: Box-Muller in float64, rounded once to float32.  fp16 fields are
rounded to nearest even (numpy's float16 cast), the same rounding as
``HalfBits.FromSingle`` (src/Qwen35Sharp.Kernels/BlockLayout.cs:168).

Block layouts (src/Qwen35Sharp.Kernels/BlockLayout.cs):
  Q4_K (:32-38)  u16 d | u16 dmin | u8 scales[12] | u8 qs[128]          144 B
  Q5_K (:49-56)  u16 d | u16 dmin | u8 scales[12] | u8 qh[32] | qs[128] 176 B
  Q6_K (:70-75)  u8 ql[128] | u8 qh[64] | s8 scales[16] | u16 d         210 B
"""

from __future__ import annotations

import numpy as np

Q4_K, Q5_K, Q6_K = 12, 13, 14
QK = 256
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
Q8K_BYTES = 292

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

# Field tags: independent streams per field.
_TAG = {
    "d": 1, "dmin": 2, "scales": 3, "qs": 4, "qh": 5, "x": 6, "ql": 7,
    "q6scales": 8, "raw": 9,
}


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _key(seed: int, field: str) -> np.uint64:
    k = np.array([(seed * 0x100000001B3 + _TAG[field] * 0x9E3779B1) & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64)
    return _mix64(k)[0]


def u64_stream(seed: int, field: str, n: int, start: int = 0) -> np.ndarray:
    """Outputs start..start+n-1 of the (seed, field) splitmix64 stream."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        return _mix64(_key(seed, field) + i * _GOLDEN)


def uniform_bytes(seed: int, field: str, n: int, start: int = 0) -> np.ndarray:
    """Bytes start..start+n-1 of the field's byte stream."""
    lead = start % 8
    words = u64_stream(seed, field, (lead + n + 7) // 8, start // 8)
    return words.view(np.uint8)[lead:lead + n].copy()


def normals(seed: int, field: str, n: int, start: int = 0) -> np.ndarray:
    """Values start..start+n-1 of the field's N(0,1) stream (float64,
    Box-Muller over 53-bit uniforms, values produced in pairs)."""
    lead = start % 2
    if lead:
        return normals(seed, field, n + 1, start - 1)[1:]
    m = (n + 1) // 2
    w = u64_stream(seed, field, 2 * m, start)
    u1 = (w[0::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    u2 = (w[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log1p(-u1))
    t = 2.0 * np.pi * u2
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return out[:n]


def _fp16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float32).astype(np.float16).view(np.uint16)


def _finite_fp16_bits(seed: int, field: str, n: int) -> np.ndarray:
    """Uniform fp16 bit patterns with non-finite ones (exponent 31) redrawn,
    as the reference's own test forces valid scales (tests/Qwen35Sharp.Tests/
    IQ4XSTests.cs:103-112)."""
    bits = (u64_stream(seed, field, n) & np.uint64(0xFFFF)).astype(np.uint16)
    bad = (bits & 0x7C00) == 0x7C00
    rnd = 0
    while bad.any():
        rnd += 1
        redraw = (u64_stream(seed + 7919 * rnd, field, n) & np.uint64(0xFFFF)).astype(np.uint16)
        bits = np.where(bad, redraw, bits)
        bad = (bits & 0x7C00) == 0x7C00
    return bits


def kquant_blocks(qtype: int, n_rows: int, k: int, seed: int, *, q5_uniform_d: bool = True,
                  row_start: int = 0) -> np.ndarray:
    """Seeded K-quant weight matrix as raw row-major blocks: uint8 [n_rows, nb*B].

    Rows row_start..row_start+n_rows-1 of the seed's matrix: a row-sharded
    rank generates exactly its own slice of the full matrix.

    Distributions (the benchmark configurations):
      Q4_K: d, dmin = fp16(|N(0,1)|*0.01); scales, qs uniform bytes.
      Q5_K: all bytes uniform; d/dmin uniform finite fp16 patterns
            (q5_uniform_d=False uses the Q4_K d/dmin distribution instead).
      Q6_K: ql, qh uniform bytes; scales uniform int8 in [-32, 31];
            d = fp16(|N(0,1)|*0.005).
    """
    if k % QK:
        raise ValueError("k must be a multiple of 256")
    nb = k // QK
    nblk = n_rows * nb
    b0 = row_start * nb  # global index of the first block
    bb = BLOCK_BYTES[qtype]
    out = np.zeros((nblk, bb), dtype=np.uint8)

    def half_normal_fp16(field, scale):
        v = normals(seed, field, nblk, start=b0)
        return _fp16_bits(np.abs(v) * scale).view(np.uint8).reshape(nblk, 2)

    if qtype == Q4_K:
        out[:, 0:2] = half_normal_fp16("d", 0.01)
        out[:, 2:4] = half_normal_fp16("dmin", 0.01)
        out[:, 4:16] = uniform_bytes(seed, "scales", nblk * 12, start=b0 * 12).reshape(nblk, 12)
        out[:, 16:144] = uniform_bytes(seed, "qs", nblk * 128, start=b0 * 128).reshape(nblk, 128)
    elif qtype == Q5_K:
        out[:, :] = uniform_bytes(seed, "raw", nblk * bb, start=b0 * bb).reshape(nblk, bb)
        if q5_uniform_d:
            if b0:
                raise ValueError("row_start is not supported for uniform Q5_K scales")
            out[:, 0:2] = _finite_fp16_bits(seed, "d", nblk).view(np.uint8).reshape(nblk, 2)
            out[:, 2:4] = _finite_fp16_bits(seed, "dmin", nblk).view(np.uint8).reshape(nblk, 2)
        else:
            out[:, 0:2] = half_normal_fp16("d", 0.01)
            out[:, 2:4] = half_normal_fp16("dmin", 0.01)
    elif qtype == Q6_K:
        out[:, 0:128] = uniform_bytes(seed, "ql", nblk * 128, start=b0 * 128).reshape(nblk, 128)
        out[:, 128:192] = uniform_bytes(seed, "qh", nblk * 64, start=b0 * 64).reshape(nblk, 64)
        sc = (uniform_bytes(seed, "q6scales", nblk * 16, start=b0 * 16).astype(np.int16) % 64) - 32
        out[:, 192:208] = sc.astype(np.int8).view(np.uint8).reshape(nblk, 16)
        out[:, 208:210] = half_normal_fp16("d", 0.005)
    else:
        raise ValueError(f"unsupported type {qtype}")
    return out.reshape(n_rows, nb * bb)


def activations(m: int, k: int, seed: int, scale: float = 1.0) -> np.ndarray:
    """float32 [m, k], N(0,1)*scale."""
    return (normals(seed, "x", m * k) * scale).astype(np.float32).reshape(m, k)


# The benchmark configurations (BASELINE.json "configs").
CONFIGS = {
    0: dict(name="q4k_gemv_m1", qtype=Q4_K, m=1, k=2560, n=9728, x_scale=1.0),
    1: dict(name="q6k_gemv_m1_vocab", qtype=Q6_K, m=1, k=2560, n=151936, x_scale=1.0),
    2: dict(name="q5k_decode_m8", qtype=Q5_K, m=8, k=9728, n=2560, x_scale=0.5),
    3: dict(name="q4k_gemm_m512", qtype=Q4_K, m=512, k=2560, n=9728, x_scale=1.0),
    4: dict(name="q4k_sharded", qtype=Q4_K, m=1, k=5120, n=27648, x_scale=1.0),
}


def algorithmic_bytes(qtype: int, m: int, k: int, n: int) -> int:
    """Quantized weight bytes + fp32 activations + fp32 outputs."""
    return n * (k // QK) * BLOCK_BYTES[qtype] + m * k * 4 + m * n * 4
