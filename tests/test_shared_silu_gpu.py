"""Shared-activation calls and the SiLU-fused ffn_down input.

q35k_matmul_shared: several weights with one nIn applied to one input with a
single quantization of it -- MulMatPanel.QuantizeAndGemm
(Qwen35Sharp.Kernels/MulMatPanel.cs:27-54) and the decode pattern of one
Q8K.QuantizeRow feeding GemvPrequant per weight (DecodeGateUp,
Qwen35Sharp.Model/Qwen35Model.Decode.cs:254-265; DecodeAttention,
Qwen35Model.Decode.cs:286-292).

q35k_matmul_silu: ffn_down on silu(gate) * up -- MulMatPanel.SiluQuantizeAndGemm
(MulMatPanel.cs:57-79, QuantizeQ8Kx4.Quantize4x8Silu) and, in decode,
Ops.SiLUMul (Qwen35Sharp.Model/Ops.cs:624-675) followed by DecodeLinear.
"""

import os

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1
TOL = 1e-3  # max|y - r| / max|r| against the oracle


def rel(y, r):
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


def silu_mul(g, u):
    g = g.astype(np.float32)
    return (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)


def device_silu_mul(g, u):
    """The product formed on the GPU with the same fp32 operations (exp,
    add, IEEE divide, multiply) as the library's quantizers."""
    torch = pytest.importorskip("torch")
    tg, tu = torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()
    return (tg / (1.0 + torch.exp(-tg)) * tu).cpu().numpy()


@pytest.mark.parametrize("mats,k,m", [
    ([(Q4_K, 9728), (Q4_K, 9728)], 2560, 1),              # gate / up, one launch
    ([(Q4_K, 9728), (Q4_K, 9728)], 2560, 2),
    ([(Q4_K, 8192), (Q4_K, 1024), (Q6_K, 1024)], 2560, 1),  # q / k / v, two launches
    ([(Q6_K, 4096), (Q6_K, 512), (Q6_K, 512)], 2560, 3),   # more than two tokens: one shared Q8_K
    ([(Q5_K, 2560), (Q5_K, 2560), (Q5_K, 300), (Q5_K, 77)], 9728, 8),  # split-K units, ragged groups
    ([(Q4_K, 1000), (Q6_K, 700)], 512, 12),                # GEMV chunks (more than 8 tokens)
])
def test_shared_matches_separate_calls(ctx, mats, k, m):
    ws = [synth.kquant_blocks(qt, n, k, seed=n + i) for i, (qt, n) in enumerate(mats)]
    x = synth.activations(m, k, seed=m + 1)
    W = [ctx.upload(qt, w, k, n) for (qt, n), w in zip(mats, ws)]
    ys = ctx.matmul_shared(W, x)
    for Wi, y, (qt, n) in zip(W, ys, mats):
        assert y.shape == (m, n)
        r = ctx.matmul(Wi, x)
        # Same quantized activations; only the split of each row's sum over
        # work units may differ with the launch's total row count.
        assert rel(y, r) <= 2e-6, (qt, n, rel(y, r))
    for Wi in W:
        Wi.free()


def test_shared_agrees_with_the_oracle(ctx, oracle_mod):
    k, m = 2560, 2
    mats = [(Q4_K, 2048), (Q4_K, 512), (Q6_K, 512)]
    x = synth.activations(m, k, seed=5)
    ws = [synth.kquant_blocks(qt, n, k, seed=40 + i) for i, (qt, n) in enumerate(mats)]
    W = [ctx.upload(qt, w, k, n) for (qt, n), w in zip(mats, ws)]
    ys = ctx.matmul_shared(W, x)
    for (qt, n), w, y in zip(mats, ws, ys):
        r = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=THREADS)
        assert rel(y, r) <= TOL
    for Wi in W:
        Wi.free()


@pytest.mark.parametrize("mode", [q35k.GEMM_EXACT, q35k.GEMM_FAST])
def test_shared_prefill_reuses_one_preparation(ctx, mode):
    # Q4_K at 64 tokens runs on the tensor-core GEMM: the second weight reuses
    # the first one's prepared activations, which must give the same bits as
    # a call of its own.  The Q6_K weight takes the chunked GEMV.
    k, m = 2560, 64
    mats = [(Q4_K, 1024), (Q4_K, 384), (Q6_K, 256)]
    ws = [synth.kquant_blocks(qt, n, k, seed=70 + i) for i, (qt, n) in enumerate(mats)]
    x = synth.activations(m, k, seed=71)
    W = [ctx.upload(qt, w, k, n) for (qt, n), w in zip(mats, ws)]
    ctx.set_gemm_mode(mode)
    try:
        ys = ctx.matmul_shared(W, x)
        for Wi, y in zip(W, ys):
            assert (y == ctx.matmul(Wi, x)).all()
    finally:
        ctx.set_gemm_mode(q35k.GEMM_EXACT)
        for Wi in W:
            Wi.free()


@pytest.mark.parametrize("qt,k,n,m", [
    (Q4_K, 9728, 2560, 1),   # cfg3 ffn_down shape, fused quantize in the GEMV
    (Q5_K, 9728, 2560, 2),
    (Q6_K, 9728, 2560, 1),
    (Q4_K, 9728, 2560, 5),   # separate quantize kernel with the product
    (Q6_K, 2560, 1000, 11),  # GEMV chunks
    (Q4_K, 2560, 1024, 64),  # tensor-core GEMM, product in its preparation
])
def test_silu_matches_matmul_of_the_product(ctx, qt, k, n, m):
    w = synth.kquant_blocks(qt, n, k, seed=n + m)
    g = synth.activations(m, k, seed=m + 11, scale=2.0)
    u = synth.activations(m, k, seed=m + 12)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul_silu(W, g, u)
    r = ctx.matmul(W, device_silu_mul(g, u))
    W.free()
    # One Q8_K code that rounds the other way (a product a few ulp apart on
    # a rounding boundary) moves every output by d8 * |w|, about 3e-4 of
    # max |y| here; a wrongly wired gate / up offset moves them by O(1).
    assert rel(y, r) <= TOL, rel(y, r)


@pytest.mark.parametrize("mode", [q35k.GEMM_EXACT, q35k.GEMM_FAST])
def test_silu_agrees_with_the_oracle(ctx, oracle_mod, mode):
    for qt, k, n, m in [(Q4_K, 2560, 512, 1), (Q6_K, 2560, 384, 3), (Q4_K, 2560, 512, 32)]:
        w = synth.kquant_blocks(qt, n, k, seed=90 + m)
        g = synth.activations(m, k, seed=91, scale=3.0)
        u = synth.activations(m, k, seed=92)
        W = ctx.upload(qt, w, k, n)
        ctx.set_gemm_mode(mode)
        try:
            y = ctx.matmul_silu(W, g, u)
        finally:
            ctx.set_gemm_mode(q35k.GEMM_EXACT)
            W.free()
        r = oracle_mod.Weight(qt, w, k, n).matmul(silu_mul(g, u), threads=THREADS)
        assert rel(y, r) <= TOL, (qt, m, rel(y, r))


def q8k_fields(b, k):
    """(d [rows, nb], qs [rows, nb, 256]) of BlockQ8K bytes."""
    blocks = b.reshape(-1, k // 256, 292)
    d = blocks[:, :, :4].copy().view(np.float32)[..., 0]
    qs = blocks[:, :, 4:260].view(np.int8)
    return d, qs


def test_quantize_silu_matches_silu_then_quantize(ctx, oracle_mod):
    # The reference's own check of its fused quantizer
    # (Qwen35Sharp.Tests/FastExpTests.cs:52-81): four rows of 256 with these
    # inputs, d within 1e-4 and every q equal to quantizing the product.
    k = 256
    i = np.arange(4 * k)
    gate = ((i % 17 - 8) * 0.2).astype(np.float32).reshape(4, k)
    up = (0.5 + (i % 9) * 0.05).astype(np.float32).reshape(4, k)
    got = ctx.quantize_q8k_silu(gate, up)
    exp = oracle_mod.quantize_q8k(silu_mul(gate, up))
    (dg, qg), (de, qe) = q8k_fields(got, k), q8k_fields(exp, k)
    assert np.abs(dg - de).max() < 1e-4
    assert (qg == qe).all()
    # and against the GPU's own quantizer of a device-formed product
    (dd, qd) = q8k_fields(ctx.quantize_q8k(device_silu_mul(gate, up)), k)
    assert np.abs(dg - dd).max() < 1e-4
    assert (qg == qd).all()


def test_quantize_silu_random_rows(ctx, oracle_mod):
    k, rows = 2560, 6
    gate = synth.activations(rows, k, seed=21, scale=3.0)
    up = synth.activations(rows, k, seed=22)
    (dg, qg) = q8k_fields(ctx.quantize_q8k_silu(gate, up), k)
    (de, qe) = q8k_fields(oracle_mod.quantize_q8k(silu_mul(gate, up)), k)
    assert (np.abs(dg - de) <= 1e-6 * np.abs(de)).all()
    # a product a few ulp from numpy's can land on the other side of a
    # rounding boundary: one code in thousands at most, by one step
    diff = qg.astype(np.int32) - qe.astype(np.int32)
    assert np.abs(diff).max() <= 1 and (diff != 0).mean() < 1e-3


@pytest.mark.parametrize("qt,k,n,m", [(Q4_K, 2560, 1024, 1), (Q6_K, 9728, 2560, 1), (Q5_K, 9728, 2560, 5)])
def test_silu_gemv_quantizes_like_the_standalone_quantizer(ctx, qt, k, n, m):
    # The GEMV's own (fused) quantization and the quantize kernel give the
    # same bytes: matmul_silu == matmul_q8k(quantize_q8k_silu) exactly.
    w = synth.kquant_blocks(qt, n, k, seed=n + 5)
    g = synth.activations(m, k, seed=31, scale=2.0)
    u = synth.activations(m, k, seed=32)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul_silu(W, g, u)
    r = ctx.matmul_q8k(W, ctx.quantize_q8k_silu(g, u), m)
    W.free()
    assert (y == r).all()


def test_device_variants(ctx):
    torch = pytest.importorskip("torch")
    k, m = 2560, 2
    mats = [(Q4_K, 4096), (Q4_K, 4096)]
    ws = [synth.kquant_blocks(qt, n, k, seed=100 + i) for i, (qt, n) in enumerate(mats)]
    W = [ctx.upload(qt, w, k, n) for (qt, n), w in zip(mats, ws)]
    x = synth.activations(m, k, seed=101)
    s = torch.cuda.current_stream().cuda_stream
    dx = torch.from_numpy(x).cuda()
    dys = [torch.empty((m, n), dtype=torch.float32, device="cuda") for _, n in mats]
    ctx.matmul_shared_dev(W, dx, dys, m, s)
    torch.cuda.synchronize()
    host = ctx.matmul_shared(W, x)
    for d, h in zip(dys, host):
        assert (d.cpu().numpy() == h).all()
    # ffn_down on the gate / up outputs, all on the device
    wd = synth.kquant_blocks(Q4_K, k, 4096, seed=102)
    Wd = ctx.upload(Q4_K, wd, 4096, k)
    dy = torch.empty((m, k), dtype=torch.float32, device="cuda")
    ctx.matmul_silu_dev(Wd, dys[0], dys[1], dy, m, s)
    torch.cuda.synchronize()
    assert (dy.cpu().numpy() == ctx.matmul_silu(Wd, host[0], host[1])).all()
    ctx.sync()
    for Wi in W + [Wd]:
        Wi.free()


def test_argument_errors(ctx):
    k = 512
    a = ctx.upload(Q4_K, synth.kquant_blocks(Q4_K, 64, k, seed=1), k, 64)
    b = ctx.upload(Q4_K, synth.kquant_blocks(Q4_K, 64, 2 * k, seed=2), 2 * k, 64)
    x = synth.activations(1, k, seed=3)
    with pytest.raises(q35k.ArgumentException):
        ctx.matmul_shared([a, b], x)           # nIn differs
    with pytest.raises(q35k.ArgumentException):
        ctx.matmul_shared([a] * (q35k.MAX_SHARED + 1), x)
    with pytest.raises(q35k.ArgumentException):
        ctx.matmul_shared([], x)
    # the same weight twice is allowed
    y0, y1 = ctx.matmul_shared([a, a], x)
    assert (y0 == y1).all()
    a.free()
    b.free()
