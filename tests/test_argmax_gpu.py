"""Vocab head fused with ArgMax (q35k_matmul_argmax): the first row holding
the largest logit, as Qwen35Sharp.Cli/Program.cs:127-140 scans the logits of
Qwen35Model.cs:280-290, computed in the GEMV's epilogue without writing the
logits."""

import os

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


@pytest.mark.parametrize("qt,k,n,m", [
    (Q6_K, 2560, 15000, 1),    # vocab-head shape, whole-row units
    (Q6_K, 2560, 15000, 3),
    (Q4_K, 5120, 27648, 1),    # 20-tile whole-row units
    (Q5_K, 9728, 2560, 8),     # split-K units (the last arriving piece decides)
    (Q4_K, 2560, 1000, 11),    # more than 8 tokens: GEMV chunks
    (Q6_K, 512, 77, 2),        # ragged row group
])
def test_argmax_matches_the_logits(ctx, qt, k, n, m):
    w = synth.kquant_blocks(qt, n, k, seed=n + m)
    x = synth.activations(m, k, seed=m + 3)
    W = ctx.upload(qt, w, k, n)
    y = ctx.matmul(W, x)
    idx = ctx.matmul_argmax(W, x)
    W.free()
    assert idx.shape == (m,)
    # np.argmax also returns the first index of the maximum.
    assert (idx == np.argmax(y, axis=1)).all(), (idx, np.argmax(y, axis=1))


def test_argmax_agrees_with_the_oracle(ctx, oracle_mod):
    qt, k, n, m = Q6_K, 2560, 20000, 2
    w = synth.kquant_blocks(qt, n, k, seed=7)
    x = synth.activations(m, k, seed=8)
    W = ctx.upload(qt, w, k, n)
    idx = ctx.matmul_argmax(W, x)
    W.free()
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=THREADS)
    for t in range(m):
        # Equal to the oracle's choice unless two logits lie within the
        # 1e-3 relative tolerance of each other.
        best = ref[t].max()
        assert ref[t, idx[t]] >= best - 1e-3 * np.abs(ref[t]).max()
        if (np.sort(ref[t])[-1] - np.sort(ref[t])[-2]) > 1e-3 * np.abs(ref[t]).max():
            assert idx[t] == int(np.argmax(ref[t]))


def test_ties_take_the_first_row(ctx):
    qt, k, n = Q4_K, 512, 300
    row = synth.kquant_blocks(qt, 1, k, seed=1)
    w = np.repeat(row, n, axis=0)  # every row the same: every logit equal
    x = synth.activations(2, k, seed=2)
    W = ctx.upload(qt, w, k, n)
    assert (ctx.matmul_argmax(W, x) == 0).all()
    # all-zero weights: every logit 0 (or -0), still row 0
    Z = ctx.upload(qt, np.zeros_like(w), k, n)
    assert (ctx.matmul_argmax(Z, x) == 0).all()
    W.free()
    Z.free()


def test_duplicated_best_row(ctx):
    qt, k, n = Q6_K, 512, 500
    w = synth.kquant_blocks(qt, n, k, seed=9)
    x = synth.activations(1, k, seed=10)
    W = ctx.upload(qt, w, k, n)
    best = int(np.argmax(ctx.matmul(W, x)[0]))
    W.free()
    # copy the best row to an earlier and a later position: the earliest wins
    w2 = w.copy()
    first = max(0, best - 37)
    w2[first] = w[best]
    if best + 50 < n:
        w2[best + 50] = w[best]
    W2 = ctx.upload(qt, w2, k, n)
    assert int(ctx.matmul_argmax(W2, x)[0]) == first
    W2.free()


def test_argmax_device_variant(ctx):
    torch = pytest.importorskip("torch")
    qt, k, n, m = Q6_K, 2560, 9000, 4
    w = synth.kquant_blocks(qt, n, k, seed=11)
    x = synth.activations(m, k, seed=12)
    W = ctx.upload(qt, w, k, n)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
    di = torch.empty(m, dtype=torch.int32, device="cuda")
    ctx.matmul_argmax_dev(W, dx, dy, di, m, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    assert (y == ctx.matmul(W, x)).all()
    assert (di.cpu().numpy() == np.argmax(y, axis=1)).all()
    di2 = torch.empty(m, dtype=torch.int32, device="cuda")
    ctx.matmul_argmax_dev(W, dx, None, di2, m, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert (di2 == di).all()
    ctx.sync()
    W.free()
