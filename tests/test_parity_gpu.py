"""GPU parity of libq35k against the CPU oracle, through the C ABI.

Bars (the parity contract of this library):
  * Q8_K bytes (qs, d bits, bsums) and dequantized weights: bit-exact;
  * y: max|y - r| / max|r| <= 1e-3 against the oracle's restatement of the
    reference's executed AVX2 path (the exact-integer design lands ~1e-6).
"""

import glob
import os

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPES = (Q4_K, Q5_K, Q6_K)
TOL = 1e-3


def rel_err(y, r):
    return float(np.abs(y.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))), ids=lambda p: os.path.basename(p)[:-4])
def test_golden_fixtures(ctx, path):
    g = np.load(path)
    qt, w, x = int(g["qtype"]), g["blocks"], g["x"]
    n, k = w.shape[0], x.shape[1]
    assert (ctx.quantize_q8k(x) == g["q8k"]).all()
    assert (ctx.dequantize(qt, w, k).view(np.uint32) == g["dequant"].view(np.uint32)).all()
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    assert rel_err(y, g["y_executed"]) <= TOL
    assert rel_err(y, g["y_semantic"]) <= TOL
    y2 = ctx.matmul_q8k(W, g["q8k"], x.shape[0])
    assert (y2 == y).all()


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("k,n", [(256, 1), (256, 17), (512, 31), (512, 33), (768, 64), (1024, 100), (2560, 129)])
@pytest.mark.parametrize("m", [1, 2, 5, 8, 9])
def test_small_shapes(ctx, oracle_mod, qt, k, n, m):
    w = synth.kquant_blocks(qt, n, k, seed=1000 + qt * 7 + n)
    x = synth.activations(m, k, seed=2000 + m)
    W = ctx.upload(qt, w, k, n)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=4)
    y = ctx.matmul(W, x)
    assert y.shape == (m, n)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("qt,k,n,m", [
    (Q6_K, 256, 200_000, 1),    # nb=1: ~42 row groups per CTA, every stage reused many times
    (Q4_K, 768, 50_001, 2),     # ragged N, 3 blocks per row, two tokens
    (Q5_K, 1280, 40_000, 3),    # 8 consumer warps, more stages per warp
    (Q4_K, 5120, 27_648, 7),
    (Q6_K, 2560, 60_000, 8),
])
def test_ring_reuse_shapes(ctx, oracle_mod, qt, k, n, m):
    """Shapes whose per-SM share is many times the stage ring, so every stage
    and mbarrier phase is reused (the pipeline's steady state)."""
    w = synth.kquant_blocks(qt, n, k, seed=n + m)
    x = synth.activations(m, k, seed=m)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=os.cpu_count() or 1)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("qt", TYPES)
def test_dequant_bit_exact_random(ctx, oracle_mod, qt):
    w = synth.kquant_blocks(qt, 64, 2048, seed=qt)
    assert (ctx.dequantize(qt, w, 2048).view(np.uint32) == oracle_mod.dequantize(qt, w, 2048).view(np.uint32)).all()


def test_quantize_bit_exact_random(ctx, oracle_mod):
    x = synth.activations(33, 5120, seed=77, scale=2.0)
    x[3, 100:400] = 0.0
    x[4, 1000] = -x[4, 1000:1256].__abs__().max()
    assert (ctx.quantize_q8k(x) == oracle_mod.quantize_q8k(x)).all()


def _tie_blocks():
    """Blocks whose largest |x| occurs more than once, at positions that the
    GPU quantizer's search (a warp lane owns values 4l..4l+3 and
    128+4l..128+4l+3) must order like Q8K.ScaleBlock's scan from index 0."""
    rng = np.random.default_rng(5)
    blocks = []

    def base():
        return (rng.standard_normal(256) * 0.1).astype(np.float32)

    def block(*hits):
        b = base()
        for pos, v in hits:
            b[pos] = v
        blocks.append(b)

    block((3, 2.5), (1, -2.5))           # same lane, low half: index 1 first
    block((127, -3.0), (128, 3.0))       # lane 31 low half before lane 0 high half
    block((130, 1.75), (136, -1.75))     # high half only: lane 0 before lane 2
    block((133, -4.0), (134, 4.0))       # same lane, high half
    block((255, -0.5), (254, 0.5), (0, 0.25))
    block((200, 7.0), (4, -7.0), (96, 7.0))
    alt = np.where(np.arange(256) % 2 == 0, 1.0, -1.0).astype(np.float32)
    blocks.append(alt)                   # every value a tie: index 0 first
    blocks.append(-alt)
    one = np.zeros(256, dtype=np.float32)
    one[255] = -1e-3                     # a single nonzero value at the end
    blocks.append(one)
    return np.stack(blocks)


def test_quantize_first_extremum_ties(ctx, oracle_mod):
    x = _tie_blocks().reshape(1, -1)
    assert (ctx.quantize_q8k(x) == oracle_mod.quantize_q8k(x)).all()
    # The same blocks through the fused decode GEMV's in-CTA quantization.
    qt, k, n = Q4_K, x.shape[1], 256
    w = synth.kquant_blocks(qt, n, k, seed=9)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    y2 = ctx.matmul_q8k(W, oracle_mod.quantize_q8k(x), 1)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))


CONFIGS = [
    ("cfg0_q4k_m1", Q4_K, 1, 2560, 9728, 1.0),
    ("cfg1_q6k_m1_vocab", Q6_K, 1, 2560, 151936, 1.0),
    ("cfg2_q5k_m8", Q5_K, 8, 9728, 2560, 0.5),
    ("cfg4_q4k_m1", Q4_K, 1, 5120, 27648, 1.0),
    ("cfg4_q4k_m8", Q4_K, 8, 5120, 27648, 1.0),
]


@pytest.mark.parametrize("name,qt,m,k,n,scale", CONFIGS, ids=[c[0] for c in CONFIGS])
def test_benchmark_configs(ctx, oracle_mod, name, qt, m, k, n, scale):
    """Full-size benchmark shapes against the oracle (AVX2 executed order)."""
    w = synth.kquant_blocks(qt, n, k, seed=1)
    x = synth.activations(m, k, seed=2, scale=scale)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=os.cpu_count() or 1)
    err = rel_err(y, ref)
    print(f"{name}: max|y-r|/max|r| = {err:.3e}")
    assert err <= TOL


@pytest.mark.parametrize("n", [64, 608, 2560], ids=["splits38_global", "splits8_cluster", "splits3_cluster"])
@pytest.mark.parametrize("m", [1, 8])
def test_split_k_reductions(ctx, oracle_mod, n, m):
    """Row groups split along K (K = 9728): 2 to 8 pieces are summed through a
    thread-block cluster's shared memory, more through global memory."""
    qt, k = Q4_K, 9728
    w = synth.kquant_blocks(qt, n, k, seed=21)
    x = synth.activations(m, k, seed=22)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=os.cpu_count() or 1)
    assert rel_err(y, ref) <= TOL
    assert np.array_equal(ctx.matmul(W, x).view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("m", [1, 2])
def test_wide_whole_row_units(ctx, oracle_mod, qt, m):
    """Whole-row units of 11 to 20 tiles (one warp per tile, 20-warp CTAs) at
    one and two tokens, against the oracle and through the pre-quantized path."""
    k = {Q4_K: 5120, Q5_K: 4096, Q6_K: 3584}[qt]
    n = 148 * 32 + 17  # at least one row group per SM (whole rows), ragged end
    w = synth.kquant_blocks(qt, n, k, seed=31)
    x = synth.activations(m, k, seed=32)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=os.cpu_count() or 1)
    assert rel_err(y, ref) <= TOL
    y2 = ctx.matmul_q8k(W, oracle_mod.quantize_q8k(x), m)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))


def test_device_pointer_path(ctx, oracle_mod):
    torch = pytest.importorskip("torch")
    qt, k, n, m = Q4_K, 2560, 1000, 3
    w = synth.kquant_blocks(qt, n, k, seed=5)
    x = synth.activations(m, k, seed=6)
    W = ctx.upload(qt, w, k, n)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ctx.matmul_dev(W, dx, dy, m, stream)
    torch.cuda.synchronize()
    assert (dy.cpu().numpy() == ctx.matmul(W, x)).all()
    dq = torch.empty(m * (k // 256) * 292, dtype=torch.uint8, device="cuda")
    ctx.quantize_q8k_dev(dx, dq, k, m, stream)
    dy2 = torch.empty_like(dy)
    ctx.matmul_q8k_dev(W, dq, dy2, m, stream)
    torch.cuda.synchronize()
    assert torch.equal(dy, dy2)
    ctx.sync()


def test_repeated_calls_are_deterministic(ctx):
    """Split-K partials are combined in a fixed order and the arrival counters
    reset themselves: repeated calls give identical bits."""
    qt, k, n, m = Q5_K, 9728, 2560, 8
    w = synth.kquant_blocks(qt, n, k, seed=3)
    x = synth.activations(m, k, seed=4)
    W = ctx.upload(qt, w, k, n)
    first = ctx.matmul(W, x)
    for _ in range(5):
        assert (ctx.matmul(W, x) == first).all()


def test_mirror_api_reads_like_the_reference(ctx, oracle_mod):
    """The reference-named entry points (MulMatQ4K.Gemv, Q6K.Gemm, ...)."""
    k, n = 512, 40
    x = synth.activations(3, k, seed=8)
    for cls, qt in ((q35k.MulMatQ4K, Q4_K), (q35k.Q5K, Q5_K), (q35k.Q6K, Q6_K)):
        w = synth.kquant_blocks(qt, n, k, seed=qt)
        ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=2)
        out = np.zeros(n, np.float32)
        cls.Gemv(w, x[0], out, k, n)
        assert rel_err(out[None, :], ref[:1]) <= TOL
        q8 = q35k.Q8K.QuantizeRow(x[0], None, k)
        out2 = np.zeros(n, np.float32)
        cls.GemvPrequant(w, q8, out2, k, n)
        assert (out2 == out).all()
        outm = np.zeros((3, n), np.float32)
        if cls is q35k.MulMatQ4K:
            cls.Gemm(None, w, x, outm, k, n, 3)
        else:
            cls.Gemm(w, x, outm, k, n, 3)
        assert rel_err(outm, ref) <= TOL


def test_error_behaviour(ctx):
    w = synth.kquant_blocks(Q4_K, 8, 256, seed=1)
    with pytest.raises(q35k.NotSupportedException):
        ctx.upload(Q4_K, w, 300, 8)
    with pytest.raises(q35k.NotSupportedException):
        ctx.upload(8, w, 256, 8)  # Q8_0 is not a K-quant weight
    W = ctx.upload(Q4_K, w, 256, 8)
    with pytest.raises(q35k.ArgumentException):
        ctx._check(ctx.L.q35k_matmul(ctx.h, W.h, None, None, 1))
    with pytest.raises(q35k.ArgumentException):
        ctx._check(ctx.L.q35k_matmul(ctx.h, W.h, np.zeros(256, np.float32).ctypes.data,
                                     np.zeros(8, np.float32).ctypes.data, 0))


def test_host_call_writes_into_a_persistent_output(ctx):
    """q35k_matmul with the caller's own output buffer, reused across calls:
    decode calls have the GEMV store y into the mapped staging buffer, prefill
    calls copy it back; both give the same bits as a fresh output."""
    for qt, k, n, m in [(Q6_K, 2560, 5000, 1), (Q4_K, 2560, 3000, 4), (Q4_K, 2560, 1000, 64), (Q5_K, 512, 300, 11)]:
        w = synth.kquant_blocks(qt, n, k, seed=n)
        W = ctx.upload(qt, w, k, n)
        out = np.full((m, n), np.nan, dtype=np.float32)
        for s in range(3):
            x = synth.activations(m, k, seed=s)
            ref = ctx.matmul(W, x)
            got = ctx.matmul(W, x, out=out)
            assert got is out
            assert (out == ref).all()
        W.free()
