"""Tensor-core prefill GEMM (Q4_K, tokens >= the dispatch threshold) against
the CPU oracle's restatement of the reference's panel GEMM
(MulMatQ4K.Gemm -> GemmQ4K.GemmAvx2Tile), through the C ABI.

Bar: max|y - r| / max|r| <= 1e-3.  The kernel forms every product of the
reference from exact integers (q8 x sc*q4 in fp16, the mins term as an fp16
high + low pair), so the observed error is fp32 rounding; DESIGN_BOUND
checks that it stays at that level.
"""

import os

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K

pytestmark = pytest.mark.gpu

TOL = 1e-3
DESIGN_BOUND = 2e-5
THREADS = os.cpu_count() or 1


def rel_err(y, r):
    return float(np.abs(y.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30))


def check(ctx, oracle_mod, w, x, k, n, name=""):
    m = x.shape[0]
    W = ctx.upload(Q4_K, w, k, n)
    y = ctx.matmul(W, x)
    ref = oracle_mod.Weight(Q4_K, w, k, n).matmul(x, threads=THREADS)
    err = rel_err(y, ref)
    print(f"{name} m={m} k={k} n={n}: max|y-r|/max|r| = {err:.3e}")
    assert np.isfinite(y).all()
    assert err <= TOL
    assert err <= DESIGN_BOUND
    W.free()
    return y


def test_cfg3_prefill_gemm(ctx, oracle_mod):
    """M=512, K=2560, N=9728 (cfg0 block generator)."""
    k, n, m = 2560, 9728, 512
    w = synth.kquant_blocks(Q4_K, n, k, seed=1)
    x = synth.activations(m, k, seed=2)
    check(ctx, oracle_mod, w, x, k, n, "cfg3")


def test_cfg4_m512_full_matrix(ctx, oracle_mod):
    """BASELINE config 4 at M=512 on one GPU: K=5120, N=27648."""
    k, n, m = 5120, 27648, 512
    w = synth.kquant_blocks(Q4_K, n, k, seed=1)
    x = synth.activations(m, k, seed=2)
    check(ctx, oracle_mod, w, x, k, n, "cfg4_m512")


@pytest.mark.parametrize("k,n,m", [
    (256, 128, 16),      # one super-block per row: every unit ends a tile
    (512, 100, 17),      # ragged rows (not a multiple of 32) and tokens
    (768, 50, 200),
    (2560, 1000, 64),
    (2560, 2048, 128),
    (2560, 9728, 129),   # one token past a tile
    (5120, 384, 300),    # few tiles, long K: tiles shared by many CTAs
    (1024, 4096, 1000),
])
def test_gemm_shapes(ctx, oracle_mod, k, n, m):
    w = synth.kquant_blocks(Q4_K, n, k, seed=n + m)
    x = synth.activations(m, k, seed=k + m)
    check(ctx, oracle_mod, w, x, k, n)


def _edge_blocks(n, k, seed):
    """Q4_K blocks exercising every scale mode of the kernel."""
    w = synth.kquant_blocks(Q4_K, n, k, seed=seed).reshape(n, k // 256, 144)
    h = lambda v: np.float16(v).view(np.uint16)
    rng = np.random.default_rng(seed)
    nb = k // 256
    for r in range(n):
        for b in range(nb):
            kind = (r * nb + b) % 7
            if kind == 0:    # d = 0: the block is -dmin * m only
                w[r, b, 0:2] = np.frombuffer(h(0.0).tobytes(), np.uint8)
            elif kind == 1:  # d = dmin = 0: the block contributes nothing
                w[r, b, 0:4] = 0
            elif kind == 2:  # dmin/d huge (subnormal d): the d/dmin fallback
                w[r, b, 0:2] = np.frombuffer(h(6e-8).tobytes(), np.uint8)
                w[r, b, 2:4] = np.frombuffer(h(40.0).tobytes(), np.uint8)
            elif kind == 3:  # dmin/d ~ 2^12: power-of-two rescaled weights
                w[r, b, 0:2] = np.frombuffer(h(1e-4).tobytes(), np.uint8)
                w[r, b, 2:4] = np.frombuffer(h(0.5).tobytes(), np.uint8)
            elif kind == 4:  # all scales and quants at their maximum
                w[r, b, 4:144] = 0xFF
            elif kind == 5:  # negative d and dmin
                w[r, b, 0:2] = np.frombuffer(h(-float(rng.random()) * 0.02).tobytes(), np.uint8)
                w[r, b, 2:4] = np.frombuffer(h(-float(rng.random()) * 0.02).tobytes(), np.uint8)
    return w.reshape(n, nb * 144)


def test_gemm_edge_blocks(ctx, oracle_mod):
    k, n, m = 1792, 300, 96
    w = _edge_blocks(n, k, seed=11)
    x = synth.activations(m, k, seed=12, scale=3.0)
    x[5] = 0.0                      # an all-zero token (d8 = 0 blocks)
    x[6, 300] = 1e4                 # one dominant value per block
    x[7, ::256] = -50.0             # ties in |x| max across the row
    x[7, 1::256] = 50.0
    check(ctx, oracle_mod, w, x, k, n, "edge")


def test_gemm_is_deterministic(ctx):
    """Tiles shared by CTAs are summed in CTA order and the counters reset:
    repeated calls give identical bits."""
    k, n, m = 2560, 9728, 300
    w = synth.kquant_blocks(Q4_K, n, k, seed=5)
    x = synth.activations(m, k, seed=6)
    W = ctx.upload(Q4_K, w, k, n)
    first = ctx.matmul(W, x)
    for _ in range(4):
        assert (ctx.matmul(W, x) == first).all()
    W.free()


def test_gemm_agrees_with_gemv_path(ctx, monkeypatch):
    """The same call through the GEMV (threshold raised) and through the
    tensor cores: both are exact-integer designs, so they agree to fp32
    rounding."""
    k, n, m = 2560, 2048, 64
    w = synth.kquant_blocks(Q4_K, n, k, seed=9)
    x = synth.activations(m, k, seed=10)
    W = ctx.upload(Q4_K, w, k, n)
    y_tc = ctx.matmul(W, x)
    monkeypatch.setenv("Q35K_GEMM_MIN_TOKENS", "1000000")
    c2 = q35k.Context(0)
    W2 = c2.upload(Q4_K, w, k, n)
    y_gemv = c2.matmul(W2, x)
    W2.free()
    c2.close()
    W.free()
    assert rel_err(y_tc, y_gemv.astype(np.float64)) <= DESIGN_BOUND


def test_gemm_device_pointer_path(ctx):
    torch = pytest.importorskip("torch")
    k, n, m = 2560, 1000, 200
    w = synth.kquant_blocks(Q4_K, n, k, seed=21)
    x = synth.activations(m, k, seed=22)
    W = ctx.upload(Q4_K, w, k, n)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ctx.matmul_dev(W, dx, dy, m, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert (dy.cpu().numpy() == ctx.matmul(W, x)).all()
    ctx.sync()
    W.free()


# ---------------------------------------------------------------------------
# Fast mode (q35k_set_gemm_mode(Q35K_GEMM_FAST)): fp16-rounded dequantized
# weights and activations, one accumulator per tile.  Every weight row and
# every token whose largest |x| is outside [2^-4, 2^15) is normalised by a
# power of two before the fp16 rounding (the drain undoes it exactly), so the
# error is the fp16 rounding of the operands (2^-11 relative each) whatever
# the scales: FAST_BOUND holds it, per config and per block of rows and
# tokens of one scale; measured 2-4.5e-4 (5.9e-4 at most per block).
# ---------------------------------------------------------------------------
FAST_BOUND = 6e-4

@pytest.fixture(scope="module")
def fast_ctx():
    c = q35k.Context(0)
    c.set_gemm_mode(q35k.GEMM_FAST)
    yield c
    c.close()


@pytest.mark.parametrize("k,n,m", [(2560, 9728, 512), (5120, 27648, 512), (256, 128, 16), (512, 100, 17),
                                   (2560, 9728, 129), (5120, 384, 300), (1024, 4096, 1000)])
def test_fast_mode_within_tolerance(fast_ctx, oracle_mod, k, n, m):
    w = synth.kquant_blocks(Q4_K, n, k, seed=n + m)
    x = synth.activations(m, k, seed=k + m)
    W = fast_ctx.upload(Q4_K, w, k, n)
    y = fast_ctx.matmul(W, x)
    ref = oracle_mod.Weight(Q4_K, w, k, n).matmul(x, threads=THREADS)
    err = rel_err(y, ref)
    print(f"fast m={m} k={k} n={n}: max|y-r|/max|r| = {err:.3e}")
    assert np.isfinite(y).all()
    assert err <= TOL and err <= FAST_BOUND
    W.free()


def test_fast_mode_edge_blocks(fast_ctx, oracle_mod):
    k, n, m = 1792, 300, 96
    w = _edge_blocks(n, k, seed=11)
    x = synth.activations(m, k, seed=12, scale=3.0)
    x[5] = 0.0
    W = fast_ctx.upload(Q4_K, w, k, n)
    y = fast_ctx.matmul(W, x)
    ref = oracle_mod.Weight(Q4_K, w, k, n).matmul(x, threads=THREADS)
    assert rel_err(y, ref) <= FAST_BOUND
    W.free()


# Row groups scaled by these powers of two (d and dmin of every block), token
# groups by these factors: fp16 subnormal weights (2^-14 d ~ 6e-7) and
# activations (1e-7), and activations beyond the fp16 maximum (1e6).
ROW_SCALES = (2.0 ** -14, 2.0 ** -6, 1.0, 2.0 ** 10)
TOKEN_SCALES = (1e-7, 1e-3, 1.0, 1e6)


def scaled_rows(qt, w, n, k):
    """Blocks of `w` with row group i's d (and dmin) times ROW_SCALES[i]."""
    size = {synth.Q4_K: 144, synth.Q5_K: 176, synth.Q6_K: 210}[qt]
    b = w.reshape(n, k // 256, size).copy()
    fields = [(208, 210)] if qt == synth.Q6_K else [(0, 2), (2, 4)]
    for i, f in enumerate(ROW_SCALES):
        rows = slice(i * n // 4, (i + 1) * n // 4)
        for lo, hi in fields:
            v = b[rows, :, lo:hi].copy().view(np.float16).astype(np.float32) * np.float32(f)
            b[rows, :, lo:hi] = v.astype(np.float16).view(np.uint8)
    return b.reshape(n, -1)


@pytest.mark.parametrize("qt", [synth.Q4_K, synth.Q5_K, synth.Q6_K])
def test_fast_mode_scale_spread(fast_ctx, oracle_mod, qt):
    """Rows and tokens over 2^24 and 1e13 of scale: every (row group, token
    group) block within FAST_BOUND of its own max |y|, none of it inf."""
    k, n, m = 2560, 512, 256
    w = scaled_rows(qt, synth.kquant_blocks(qt, n, k, seed=31, q5_uniform_d=False), n, k)
    x = synth.activations(m, k, seed=32)
    for j, f in enumerate(TOKEN_SCALES):
        x[j * m // 4:(j + 1) * m // 4] *= np.float32(f)
    W = fast_ctx.upload(qt, w, k, n)
    y = fast_ctx.matmul(W, x)
    W.free()
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=THREADS)
    assert np.isfinite(y).all()
    for i in range(4):
        for j in range(4):
            rows, toks = slice(i * n // 4, (i + 1) * n // 4), slice(j * m // 4, (j + 1) * m // 4)
            err = rel_err(y[toks, rows], ref[toks, rows])
            print(f"rows x{ROW_SCALES[i]:g} tokens x{TOKEN_SCALES[j]:g}: {err:.3e}")
            assert err <= FAST_BOUND, (i, j, err)


def test_fast_mode_long_rows(fast_ctx, oracle_mod):
    """Rows of 65 super-blocks (more than one token-scale CTA's warps cover at
    once when rewritten): tokens inside the fast preparation's e = 0 range and
    outside it, against the oracle."""
    k, n, m = 65 * 256, 256, 64
    w = synth.kquant_blocks(Q4_K, n, k, seed=41)
    x = synth.activations(m, k, seed=42)
    x[:16] *= np.float32(1e-7)
    x[16:32] *= np.float32(1e6)
    W = fast_ctx.upload(Q4_K, w, k, n)
    y = fast_ctx.matmul(W, x)
    W.free()
    ref = oracle_mod.Weight(Q4_K, w, k, n).matmul(x, threads=THREADS)
    assert np.isfinite(y).all()
    for toks in (slice(0, 16), slice(16, 32), slice(32, 64)):
        assert rel_err(y[toks], ref[toks]) <= FAST_BOUND


@pytest.mark.parametrize("m", [300, 700])  # 128- and 256-token tiles
def test_fast_mode_is_deterministic(fast_ctx, m):
    k, n = 2560, 9728
    w = synth.kquant_blocks(Q4_K, n, k, seed=5)
    x = synth.activations(m, k, seed=6)
    W = fast_ctx.upload(Q4_K, w, k, n)
    first = fast_ctx.matmul(W, x)
    for _ in range(3):
        assert (fast_ctx.matmul(W, x) == first).all()
    W.free()


def test_fast_mode_wide_tiles_match_narrow(fast_ctx, oracle_mod):
    """512+ tokens run on 256-token tiles: against the oracle, ragged
    tokens (not a multiple of 256) and a K run shared by several CTAs."""
    for k, n, m in [(2560, 1000, 513), (5120, 640, 777)]:
        w = synth.kquant_blocks(Q4_K, n, k, seed=m)
        x = synth.activations(m, k, seed=m + 1)
        W = fast_ctx.upload(Q4_K, w, k, n)
        y = fast_ctx.matmul(W, x)
        ref = oracle_mod.Weight(Q4_K, w, k, n).matmul(x, threads=THREADS)
        assert np.isfinite(y).all()
        assert rel_err(y, ref) <= FAST_BOUND
        W.free()
