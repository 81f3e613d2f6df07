"""Independent pure-Python/numpy restatement of the reference's K-quant
formulas, used only to cross-check the C oracle on small cases.

It is written from the C# sources directly (file:line below, relative to
src/Qwen35Sharp.Kernels/), shares no code with oracle/, and uses exact integer
arithmetic for the per-block dot products (float64 for the final scaling), so
agreement with the C oracle is evidence that neither restatement misreads the
reference.
"""

from __future__ import annotations

import numpy as np

QK = 256
Q4_K, Q5_K, Q6_K = 12, 13, 14
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}


def fp16(b: np.ndarray, off: int) -> np.float32:
    """HalfBits.ToSingle (BlockLayout.cs:166) via numpy's exact float16."""
    return np.float32(np.frombuffer(bytes(b[off:off + 2]), dtype=np.float16)[0])


def q8k_row(x: np.ndarray) -> list:
    """Q8K.QuantizeRow (Q8K.cs:12-146) -> list of (d, qs int array, bsums)."""
    out = []
    x = np.asarray(x, dtype=np.float32)
    for i in range(len(x) // QK):
        src = x[i * QK:(i + 1) * QK]
        ax = np.abs(src)
        amax = ax.max()
        if amax == 0:
            out.append((np.float32(0), np.zeros(QK, np.int64), np.zeros(16, np.int64)))
            continue
        mx = src[int(np.argmax(ax == amax))]  # first index with |x| == amax
        iscale = np.float32(np.float32(-127.0) / mx)
        d = np.float32(np.float32(1.0) / iscale)
        q = np.clip(np.rint((src * iscale).astype(np.float32)), -127, 127).astype(np.int64)
        bs = q.reshape(16, 16).sum(axis=1)
        out.append((d, q, bs))
    return out


def q8k_bytes(blocks: list) -> bytes:
    """BlockQ8K wire layout (BlockLayout.cs:41-46)."""
    buf = bytearray()
    for d, q, bs in blocks:
        buf += np.float32(d).tobytes()
        buf += q.astype(np.int8).tobytes()
        buf += bs.astype(np.int16).tobytes()
    return bytes(buf)


def scale_min(j: int, s: np.ndarray):
    """Q4K.GetScaleMin (Q4K.cs:7-18)."""
    s = [int(v) for v in s]
    if j < 4:
        return s[j] & 63, s[j + 4] & 63
    return (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4), (s[j + 4] >> 4) | ((s[j] >> 6) << 4)


def levels(qtype: int, blk: np.ndarray) -> np.ndarray:
    """Integer quant level of each of the 256 values of one block
    (Q4K.cs:35-60, Q5K.cs:5-35, Q6K.cs:9-39): 0..15, 0..31, or 0..63."""
    q = np.zeros(QK, np.int64)
    if qtype in (Q4_K, Q5_K):
        qs = blk[16:144] if qtype == Q4_K else blk[48:176]
        qh = None if qtype == Q4_K else blk[16:48]
        for c in range(4):
            for l in range(32):
                byte = int(qs[32 * c + l])
                lo, hi = byte & 0xF, byte >> 4
                if qh is not None:
                    lo += 16 if int(qh[l]) & (1 << (2 * c)) else 0
                    hi += 16 if int(qh[l]) & (2 << (2 * c)) else 0
                q[64 * c + l] = lo
                q[64 * c + 32 + l] = hi
    else:
        ql, qh = blk[0:128], blk[128:192]
        for h in range(2):
            for l in range(32):
                a, b, hh = int(ql[64 * h + l]), int(ql[64 * h + 32 + l]), int(qh[32 * h + l])
                q[128 * h + l] = (a & 0xF) | ((hh & 3) << 4)
                q[128 * h + 32 + l] = (b & 0xF) | (((hh >> 2) & 3) << 4)
                q[128 * h + 64 + l] = (a >> 4) | (((hh >> 4) & 3) << 4)
                q[128 * h + 96 + l] = (b >> 4) | (((hh >> 6) & 3) << 4)
    return q


def dequant_block(qtype: int, blk: np.ndarray) -> np.ndarray:
    """Per-value float32 dequantization with the reference's rounding order."""
    q = levels(qtype, blk)
    y = np.zeros(QK, np.float32)
    if qtype in (Q4_K, Q5_K):
        d, dmin = fp16(blk, 0), fp16(blk, 2)
        for j in range(8):
            sc, m = scale_min(j, blk[4:16])
            d1, m1 = np.float32(d * np.float32(sc)), np.float32(dmin * np.float32(m))
            y[32 * j:32 * j + 32] = (d1 * q[32 * j:32 * j + 32].astype(np.float32)).astype(np.float32) - m1
    else:
        d = fp16(blk, 208)
        sc = blk[192:208].view(np.int8).astype(np.float32)
        for j in range(16):
            ds = np.float32(d * sc[j])
            y[16 * j:16 * j + 16] = ds * (q[16 * j:16 * j + 16] - 32).astype(np.float32)
    return y


def block_dot(qtype: int, blk: np.ndarray, a) -> float:
    """Exact-integer block dot (VecDotQ4K.cs:16-65, Q5K.cs:37-87,
    Q6K.cs:44-85), scaled in float64."""
    ad, aq, abs_ = a
    q = levels(qtype, blk)
    if qtype in (Q4_K, Q5_K):
        S = 0
        Mn = 0
        for j in range(8):
            sc, m = scale_min(j, blk[4:16])
            S += sc * int(np.dot(q[32 * j:32 * j + 32], aq[32 * j:32 * j + 32]))
            Mn += m * int(abs_[2 * j] + abs_[2 * j + 1])
        return float(fp16(blk, 0)) * float(ad) * S - float(fp16(blk, 2)) * float(ad) * Mn
    sc = blk[192:208].view(np.int8).astype(np.int64)
    S = 0
    for j in range(16):
        S += int(sc[j]) * int(np.dot(q[16 * j:16 * j + 16] - 32, aq[16 * j:16 * j + 16]))
    return float(fp16(blk, 208)) * float(ad) * S


def matvec(qtype: int, w: np.ndarray, x: np.ndarray, k: int) -> np.ndarray:
    """y[n] = sum over blocks of block_dot, float64 accumulation."""
    a = q8k_row(x)
    nb = k // QK
    bb = BLOCK_BYTES[qtype]
    w = w.reshape(-1, nb * bb)
    y = np.zeros(w.shape[0])
    for r in range(w.shape[0]):
        y[r] = sum(block_dot(qtype, w[r, b * bb:(b + 1) * bb], a[b]) for b in range(nb))
    return y
