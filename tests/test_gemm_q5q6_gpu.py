"""Tensor-core prefill GEMM for Q5_K and Q6_K weights, against the CPU
oracle (Q5K.Gemm, Kernels/Q5K.cs:114-118, per-token GEMV; Q6K.Gemm,
Kernels/Q6K.cs:317-353) through the C ABI.

Both types run in both GEMM modes.  Q5_K's exact mode uses Q4_K's scheme:
the weight values alpha * sc_j * q (q <= 31, at most 1953 * alpha) are exact
in fp16, so the observed error is fp32 rounding (DESIGN_BOUND).  Q6_K's
products sc * (q - 32) need up to 12 significant bits, so its exact mode
splits every int8 scale as sc = 16 sh + sl (sl in [0, 15]) and multiplies
the two exact fp16 parts sl (q - 32) and 16 sh (q - 32) against the same
activations (two MMAs per K step); its error is fp32 rounding as well.
Bar: max|y - r| / max|r| <= 1e-3, DESIGN_BOUND for the exact mode and
FAST_BOUND (the fp16 rounding of both operands, after the per-row and
per-token power-of-two normalisation) for the fast mode.
"""

import os

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q5_K, Q6_K

pytestmark = pytest.mark.gpu

TOL = 1e-3
DESIGN_BOUND = 2e-5
FAST_BOUND = 6e-4
THREADS = os.cpu_count() or 1


def rel_err(y, r):
    return float(np.abs(y.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.fixture(scope="module")
def fast_ctx():
    c = q35k.Context(0)
    c.set_gemm_mode(q35k.GEMM_FAST)
    yield c
    c.close()


@pytest.fixture(scope="module")
def gemv_ctx():
    """A context whose calls all take the GEMV (dispatch threshold raised)."""
    old = os.environ.get("Q35K_GEMM_MIN_TOKENS")
    os.environ["Q35K_GEMM_MIN_TOKENS"] = "1000000"
    try:
        c = q35k.Context(0)
    finally:
        if old is None:
            del os.environ["Q35K_GEMM_MIN_TOKENS"]
        else:
            os.environ["Q35K_GEMM_MIN_TOKENS"] = old
    yield c
    c.close()


def run(c, qt, w, x, k, n):
    W = c.upload(qt, w, k, n)
    y = c.matmul(W, x)
    W.free()
    return y


SHAPES = [
    (256, 128, 16),      # one super-block per row
    (512, 100, 17),      # ragged rows and tokens
    (768, 50, 200),
    (2560, 1000, 64),
    (9728, 2560, 512),   # cfg2's Q5_K ffn_down shape at prefill (256-token tiles in the fast mode)
    (2560, 4096, 300),
    (5120, 384, 777),    # few tiles, long K, ragged wide tiles
]


@pytest.mark.parametrize("k,n,m", SHAPES)
def test_q5k_exact(ctx, oracle_mod, gemv_ctx, k, n, m):
    w = synth.kquant_blocks(Q5_K, n, k, seed=n + m)
    x = synth.activations(m, k, seed=k + m)
    y = run(ctx, Q5_K, w, x, k, n)
    ref = oracle_mod.Weight(Q5_K, w, k, n).matmul(x, threads=THREADS)
    err = rel_err(y, ref)
    print(f"Q5_K exact m={m} k={k} n={n}: {err:.3e}")
    assert np.isfinite(y).all()
    assert err <= TOL and err <= DESIGN_BOUND
    if m == 64:
        # the tensor-core path ran: a different fp32 summation order than the GEMV's
        assert not (y == run(gemv_ctx, Q5_K, w, x, k, n)).all()


@pytest.mark.parametrize("qt", [Q5_K, Q6_K])
@pytest.mark.parametrize("k,n,m", SHAPES)
def test_fast_mode(fast_ctx, oracle_mod, qt, k, n, m):
    # Q5_K with GGUF-like scales (d, dmin ~ 0.01); the default test pattern
    # (uniform fp16 d) is the fp16-range case below.
    w = synth.kquant_blocks(qt, n, k, seed=n + m + qt, q5_uniform_d=False)
    x = synth.activations(m, k, seed=k + m)
    y = run(fast_ctx, qt, w, x, k, n)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=THREADS)
    err = rel_err(y, ref)
    print(f"{'Q5_K' if qt == Q5_K else 'Q6_K'} fast m={m} k={k} n={n}: {err:.3e}")
    assert np.isfinite(y).all()
    assert err <= TOL and err <= FAST_BOUND


def _q5k_edge_blocks(n, k, seed):
    """Q5_K blocks exercising every scale mode of the exact form (the header
    is Q4_K's: fp16 d, fp16 dmin, 12 bytes of scales)."""
    w = synth.kquant_blocks(Q5_K, n, k, seed=seed, q5_uniform_d=False).reshape(n, k // 256, 176)
    h = lambda v: np.frombuffer(np.float16(v).tobytes(), np.uint8)
    rng = np.random.default_rng(seed)
    for r in range(n):
        for b in range(k // 256):
            kind = (r * (k // 256) + b) % 7
            if kind == 0:
                w[r, b, 0:2] = h(0.0)                       # d = 0
            elif kind == 1:
                w[r, b, 0:4] = 0                            # d = dmin = 0
            elif kind == 2:
                w[r, b, 0:2], w[r, b, 2:4] = h(6e-8), h(40.0)  # dmin/d huge
            elif kind == 3:
                w[r, b, 0:2], w[r, b, 2:4] = h(1e-4), h(0.5)   # dmin/d ~ 2^12
            elif kind == 4:
                w[r, b, 4:176] = 0xFF                       # every scale, quant and high bit at its maximum
            elif kind == 5:
                w[r, b, 0:2] = h(-float(rng.random()) * 0.02)
                w[r, b, 2:4] = h(-float(rng.random()) * 0.02)
    return w.reshape(n, -1)


@pytest.mark.parametrize("fast", [False, True])
def test_q5k_edge_blocks(ctx, fast_ctx, oracle_mod, fast):
    k, n, m = 1792, 300, 96
    w = _q5k_edge_blocks(n, k, seed=11)
    x = synth.activations(m, k, seed=12, scale=3.0)
    x[5] = 0.0
    y = run(fast_ctx if fast else ctx, Q5_K, w, x, k, n)
    ref = oracle_mod.Weight(Q5_K, w, k, n).matmul(x, threads=THREADS)
    assert np.isfinite(y).all()
    assert rel_err(y, ref) <= TOL
    if not fast:
        assert rel_err(y, ref) <= DESIGN_BOUND


def test_fast_mode_takes_the_whole_fp16_range(ctx, fast_ctx, oracle_mod):
    """d and dmin anywhere in the finite fp16 range (up to 65504, products
    far beyond the fp16 maximum): the per-row normalisation keeps the fast
    mode's fp16 values in range, so these weights run the fast GEMM, within
    FAST_BOUND."""
    k, n, m = 2560, 512, 64
    w5 = synth.kquant_blocks(Q5_K, n, k, seed=13)  # uniform finite fp16 d and dmin
    x = synth.activations(m, k, seed=14)
    y_fast = run(fast_ctx, Q5_K, w5, x, k, n)
    assert np.isfinite(y_fast).all()
    ref = oracle_mod.Weight(Q5_K, w5, k, n).matmul(x, threads=THREADS)
    assert rel_err(y_fast, ref) <= FAST_BOUND
    assert not (y_fast == run(ctx, Q5_K, w5, x, k, n)).all()  # the fast arithmetic ran
    w6 = synth.kquant_blocks(Q6_K, n, k, seed=15).reshape(n, k // 256, 210)
    w6[0, 0, 208:210] = np.frombuffer(np.float16(1000.0).tobytes(), np.uint8)  # one block with d = 1000
    w6 = w6.reshape(n, -1)
    y6 = run(fast_ctx, Q6_K, w6, x, k, n)
    assert rel_err(y6, oracle_mod.Weight(Q6_K, w6, k, n).matmul(x, threads=THREADS)) <= FAST_BOUND


@pytest.mark.parametrize("qt", [Q5_K, Q6_K])
def test_fast_mode_keeps_non_finite_scales_exact(ctx, fast_ctx, qt):
    """A weight with an infinite or NaN block scale is flagged at upload: its
    fast-mode prefill is the exact GEMM, bit for bit (the non-finite rows
    included)."""
    k, n, m = 1024, 256, 64
    size = 176 if qt == Q5_K else 210
    d_at = 0 if qt == Q5_K else 208
    w = synth.kquant_blocks(qt, n, k, seed=16, q5_uniform_d=False).reshape(n, k // 256, size)
    w[3, 1, d_at:d_at + 2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    w[7, 2, d_at:d_at + 2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    w = w.reshape(n, -1)
    x = synth.activations(m, k, seed=17)
    y_fast = run(fast_ctx, qt, w, x, k, n)
    y_exact = run(ctx, qt, w, x, k, n)
    assert np.array_equal(y_fast.view(np.uint32), y_exact.view(np.uint32))
    assert np.isfinite(np.delete(y_exact, [3, 7], axis=1)).all()


def test_q6k_fast_mode_ran_on_the_tensor_cores(fast_ctx, gemv_ctx):
    k, n, m = 2560, 1000, 64
    w = synth.kquant_blocks(Q6_K, n, k, seed=3)
    x = synth.activations(m, k, seed=4)
    y = run(fast_ctx, Q6_K, w, x, k, n)
    y_gemv = run(gemv_ctx, Q6_K, w, x, k, n)
    assert rel_err(y, y_gemv.astype(np.float64)) <= TOL
    assert not (y == y_gemv).all()  # fp16-rounded operands: not the GEMV's bits


@pytest.mark.parametrize("k,n,m", SHAPES)
def test_q6k_exact(ctx, oracle_mod, gemv_ctx, k, n, m):
    w = synth.kquant_blocks(Q6_K, n, k, seed=n + m + 1)
    x = synth.activations(m, k, seed=k + m + 1)
    y = run(ctx, Q6_K, w, x, k, n)
    ref = oracle_mod.Weight(Q6_K, w, k, n).matmul(x, threads=THREADS)
    err = rel_err(y, ref)
    print(f"Q6_K exact m={m} k={k} n={n}: {err:.3e}")
    assert np.isfinite(y).all()
    assert err <= TOL and err <= DESIGN_BOUND
    if m == 64:
        # the tensor-core path ran: a different fp32 summation order than the GEMV's
        assert not (y == run(gemv_ctx, Q6_K, w, x, k, n)).all()


def _q6k_edge_blocks(n, k, seed):
    """Q6_K blocks at the ends of every field: d = 0, negative and subnormal
    d, the full int8 scale range (the reference's format allows -128..127,
    beyond the synthetic [-32, 31]), every quant at 0 or 63."""
    w = synth.kquant_blocks(Q6_K, n, k, seed=seed).reshape(n, k // 256, 210)
    h = lambda v: np.frombuffer(np.float16(v).tobytes(), np.uint8)
    rng = np.random.default_rng(seed)
    for r in range(n):
        for b in range(k // 256):
            kind = (r * (k // 256) + b) % 6
            if kind == 0:
                w[r, b, 208:210] = h(0.0)
            elif kind == 1:
                w[r, b, 208:210] = h(-float(rng.random()) * 0.01)
            elif kind == 2:
                w[r, b, 208:210] = h(3e-7)                   # subnormal d
            elif kind == 3:
                w[r, b, 192:208] = rng.choice(np.array([-128, 127, -1, 0, 15, -16], np.int8), 16).view(np.uint8)
            elif kind == 4:
                w[r, b, 0:192] = 0xFF                         # q = 63 everywhere
                w[r, b, 192:208] = np.int8(-128).view(np.uint8)
            elif kind == 5:
                w[r, b, 0:192] = 0x00                         # q = 0 everywhere
                w[r, b, 192:208] = np.int8(127).view(np.uint8)
    return w.reshape(n, -1)


def test_q6k_exact_edge_blocks(ctx, oracle_mod):
    k, n, m = 1792, 300, 96
    w = _q6k_edge_blocks(n, k, seed=17)
    x = synth.activations(m, k, seed=18, scale=3.0)
    x[7] = 0.0
    y = run(ctx, Q6_K, w, x, k, n)
    ref = oracle_mod.Weight(Q6_K, w, k, n).matmul(x, threads=THREADS)
    assert np.isfinite(y).all()
    assert rel_err(y, ref) <= DESIGN_BOUND


@pytest.mark.parametrize("qt,fast", [(Q5_K, False), (Q5_K, True), (Q6_K, False), (Q6_K, True)])
def test_deterministic(ctx, fast_ctx, qt, fast):
    c = fast_ctx if fast else ctx
    k, n, m = 2560, 2048, 600
    w = synth.kquant_blocks(qt, n, k, seed=7, q5_uniform_d=False)
    x = synth.activations(m, k, seed=8)
    W = c.upload(qt, w, k, n)
    first = c.matmul(W, x)
    for _ in range(3):
        assert (c.matmul(W, x) == first).all()
    W.free()


def test_shared_prefill_mixed_types(fast_ctx):
    """q35k_matmul_shared with Q4_K, Q5_K and Q6_K weights at prefill: one
    activation preparation serves all three GEMM launches."""
    from q35k.synth import Q4_K
    k, m = 2560, 128
    mats = [(Q4_K, 512), (Q5_K, 384), (Q6_K, 256)]
    ws = [synth.kquant_blocks(qt, n, k, seed=60 + i, q5_uniform_d=False) for i, (qt, n) in enumerate(mats)]
    x = synth.activations(m, k, seed=61)
    W = [fast_ctx.upload(qt, w, k, n) for (qt, n), w in zip(mats, ws)]
    ys = fast_ctx.matmul_shared(W, x)
    for Wi, y in zip(W, ys):
        assert (y == fast_ctx.matmul(Wi, x)).all()
        Wi.free()
