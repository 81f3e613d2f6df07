"""CPU tests of the oracle (no GPU): the C restatement against the golden
fixtures, against an independent pure-Python restatement, against
hand-derived known answers, and scalar-vs-AVX2 pairing (the reference's own
"reference pairing" test pattern, doc/10-testing.md:1-14)."""

import glob
import hashlib
import json
import os

import numpy as np
import pytest

import pyref
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPES = (Q4_K, Q5_K, Q6_K)


def golden_cases():
    return sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def test_golden_manifest():
    manifest = json.load(open(os.path.join(GOLDEN, "MANIFEST.json")))
    assert len(manifest) == len(golden_cases()) == 15
    for key, digest in manifest.items():
        data = open(os.path.join(GOLDEN, key + ".npz"), "rb").read()
        assert hashlib.sha256(data).hexdigest() == digest, key


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_reproduces_golden(oracle_mod, path):
    g = np.load(path)
    qt, w, x = int(g["qtype"]), g["blocks"], g["x"]
    n, k = w.shape[0], x.shape[1]
    assert (oracle_mod.quantize_q8k(x, avx2=True) == g["q8k"]).all()
    assert (oracle_mod.quantize_q8k(x, avx2=False) == g["q8k"]).all()
    assert (oracle_mod.dequantize(qt, w, k).view(np.uint32) == g["dequant"].view(np.uint32)).all()
    W = oracle_mod.Weight(qt, w, k, n)
    assert (W.matmul_semantic(x).view(np.uint32) == g["y_semantic"].view(np.uint32)).all()
    for threads in (1, 3):
        assert (W.matmul(x, threads=threads).view(np.uint32) == g["y_executed"].view(np.uint32)).all()


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_python_restatement(oracle_mod, path):
    """Two independent restatements of the C# must agree: Q8_K bytes and
    dequantized values bit-exactly, dots to fp32 rounding."""
    g = np.load(path)
    qt, w, x = int(g["qtype"]), g["blocks"], g["x"]
    k = x.shape[1]
    bb = synth.BLOCK_BYTES[qt]
    for r in range(x.shape[0]):
        py = np.frombuffer(pyref.q8k_bytes(pyref.q8k_row(x[r])), np.uint8)
        assert (py == g["q8k"][r]).all(), f"Q8_K row {r}"
    deq = np.stack([np.concatenate([pyref.dequant_block(qt, w[i, b * bb:(b + 1) * bb]) for b in range(k // 256)])
                    for i in range(w.shape[0])])
    assert (deq.view(np.uint32) == g["dequant"].view(np.uint32)).all()
    ref = np.stack([pyref.matvec(qt, w, x[t], k) for t in range(x.shape[0])])
    scale = max(np.abs(ref).max(), 1e-30)
    for key in ("y_semantic", "y_executed"):
        err = np.abs(g[key].astype(np.float64) - ref).max() / scale
        assert err < 1e-5, (key, err)


def test_scalar_vs_avx2_quantizer_random(oracle_mod):
    x = synth.activations(64, 1024, seed=5, scale=3.0)
    assert (oracle_mod.quantize_q8k(x, avx2=True) == oracle_mod.quantize_q8k(x, avx2=False)).all()


def test_q8k_first_signed_extremum(oracle_mod):
    """Q8K.ScaleBlock keeps the sign of the FIRST element with the largest
    |x| (Kernels/Q8K.cs:103-120): d is negative when that element is positive."""
    x = np.zeros(256, np.float32)
    x[3], x[9] = 2.0, -2.0
    q = oracle_mod.quantize_q8k(x)[0]
    d = q[:4].view(np.float32)[0]
    assert d == np.float32(1.0) / np.float32(np.float32(-127.0) / np.float32(2.0))
    assert d < 0 and q[4 + 3].view(np.int8) == -127 and q[4 + 9].view(np.int8) == 127
    x[3], x[9] = -2.0, 2.0
    q = oracle_mod.quantize_q8k(x)[0]
    assert q[:4].view(np.float32)[0] > 0


def test_known_answer_q4k(oracle_mod):
    """Hand-derived: d=1, dmin=0, all 6-bit scales 1, every nibble 1, x = 1:
    Q8_K gives d_x = 1/(-127), q = -127, so y = 1 * d_x * (256 * -127) = 256."""
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.array([0x3C00], np.uint16).view(np.uint8)  # d = 1.0
    blk[4:8] = 1          # sc[0..3] = 1, their high bits 0
    blk[8:12] = 0         # m[0..3] = 0
    blk[12:16] = 0x01     # sc[4..7] low nibble 1, m[4..7] = 0
    blk[16:] = 0x11
    x = np.ones(256, np.float32)
    assert (oracle_mod.dequantize(Q4_K, blk, 256) == 1.0).all()
    W = oracle_mod.Weight(Q4_K, blk[None, :], 256, 1)
    dx = np.float32(1.0) / np.float32(-127.0)
    want = np.float32(np.float32(1.0) * dx) * np.float32(-127 * 256)
    assert W.matmul(x)[0, 0] == want
    assert abs(float(want) - 256.0) < 1e-4


def test_known_answer_q6k(oracle_mod):
    """Hand-derived: d=0.5, all scales 2, every 6-bit quant 33 (value 1):
    dequant = 0.5 * 2 * 1 = 1 everywhere; with x = -1, y = -256 (to fp32)."""
    blk = np.zeros(210, np.uint8)
    blk[0:128] = 0x11                      # low nibbles 1
    blk[128:192] = 0xAA                    # every 2-bit high field = 2 -> q = 1 | 2<<4 = 33
    blk[192:208] = 2
    blk[208:210] = np.array([0x3800], np.uint16).view(np.uint8)  # 0.5
    assert (oracle_mod.dequantize(Q6_K, blk, 256) == 1.0).all()
    W = oracle_mod.Weight(Q6_K, blk[None, :], 256, 1)
    y = W.matmul(-np.ones(256, np.float32))[0, 0]
    assert abs(float(y) + 256.0) < 1e-3


def test_known_answer_q5k_high_bit(oracle_mod):
    """Q5_K: nibble 0 with every high bit set is 16; d=1, scales 1 -> 16."""
    blk = np.zeros(176, np.uint8)
    blk[0:2] = np.array([0x3C00], np.uint16).view(np.uint8)
    blk[4:8] = 1
    blk[12:16] = 0x01
    blk[16:48] = 0xFF  # qh
    assert (oracle_mod.dequantize(Q5_K, blk, 256) == 16.0).all()


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("tokens", [1, 2, 3, 4, 5, 8, 9])
def test_dispatch_executed_vs_semantic(oracle_mod, qt, tokens):
    """Every dispatch path (GEMV, Q4_K panel GEMM with padding and nOut%8
    tail, Q6_K 4-token groups) agrees with the scalar semantics."""
    k, n = 512, 19
    w = synth.kquant_blocks(qt, n, k, seed=qt * 10 + tokens)
    x = synth.activations(tokens, k, seed=tokens)
    W = oracle_mod.Weight(qt, w, k, n)
    a, b = W.matmul(x, threads=4), W.matmul_semantic(x)
    assert np.abs(a - b).max() / np.abs(b).max() < 1e-5


def test_prequant_matches_matmul(oracle_mod):
    k, n = 768, 24
    for qt in TYPES:
        w = synth.kquant_blocks(qt, n, k, seed=9)
        x = synth.activations(1, k, seed=10)
        W = oracle_mod.Weight(qt, w, k, n)
        q8 = oracle_mod.quantize_q8k(x)
        assert (W.matmul_q8k(q8, 1, threads=2) == W.matmul(x, threads=2)).all()


def test_choose_worker_count(oracle_mod):
    """CpuTopology.ChooseWorkerCount (Kernels/CpuTopology.cs:107-123)."""
    f = oracle_mod.choose_worker_count
    assert f(8, 8, 0, False, True) == 4        # SMT-hiding VM is halved
    assert f(8, 8, 0, False, False) == 8
    assert f(224, 112, 0, True, False) == 112  # bare metal with SMT: physical cores
    assert f(16, 0, 0, False, False) == 8
    assert f(3, 0, 0, False, False) == 3
    assert f(8, 0, 0, False, True) == 4
    assert f(24, 16, 8, True, False) == 8      # hybrid: P-cores
    assert oracle_mod.host_topology()["reference_workers"] >= 1
