"""q35k_matmul_static_dev: the decode matmul that allocates nothing.

Callers that cannot let a library allocate device memory during a call (a
host whose device memory is all owned by its own arena, or a decode loop
where a cudaMalloc/cudaFree would synchronize and stall the device) use this
entry point; its scratch lives in one fixed array that the library holds on
every GPU.  Checked here through the C ABI against q35k_matmul_dev, which
runs the same deterministic kernels with context-owned scratch, so the two
must agree bit for bit; on two calls in a row (the array keeps the previous
call's contents, so the second call shows that what must start at zero is
cleared); and once against the CPU oracle.  Collected last; works alone in a
fresh process as well as after the other tests.
"""

import ctypes

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

pytestmark = pytest.mark.gpu

# The oracle comparison's bar (the parity tests' 1e-3 of max |y|).
TOL = 1e-3


def rel_err(y, r):
    return float(np.abs(y.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.fixture(scope="module")
def env():
    torch = pytest.importorskip("torch")
    ctx = q35k.Context(0)
    torch.cuda.set_device(0)
    yield torch, ctx
    ctx.close()


def static_call(ctx, W, dx, dy, m, stream):
    return ctx.L.q35k_matmul_static_dev(W.h, dx.data_ptr(), dy.data_ptr(), m,
                                        ctypes.c_void_p(stream.cuda_stream or 1))


@pytest.mark.parametrize("qt,k,n,m", [
    (Q6_K, 2560, 9728, 1),    # decode: the GEMV quantizes x itself (no Q8_K scratch)
    (Q4_K, 2560, 2048, 1),    # fewer row groups than SMs: split-K partials + counters
    (Q5_K, 9728, 2560, 8),    # Q8_K scratch + split-K partials + counters
    (Q4_K, 5120, 1000, 3),    # ragged rows
])
def test_static_entry_matches_regular_entry(env, qt, k, n, m, oracle_mod):
    torch, ctx = env
    w = synth.kquant_blocks(qt, n, k, seed=n + m)
    W = ctx.upload(qt, w, k, n)
    stream = torch.cuda.current_stream()
    for call in range(2):
        x = synth.activations(m, k, seed=10 * call + m)
        dx = torch.from_numpy(x).cuda()
        ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        ctx.matmul_dev(W, dx, ref, m, stream)
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        rc = static_call(ctx, W, dx, out, m, stream)
        assert rc == 0, ctx.L.q35k_last_error(None).decode()
        torch.cuda.synchronize()
        got, want = out.cpu().numpy(), ref.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {call}: not bit-equal"
        if call == 1:
            r = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=4)
            assert rel_err(got, r) <= TOL
    W.free()


def test_static_entry_rejects_too_many_tokens(env):
    torch, ctx = env
    k, n = 256, 64
    w = synth.kquant_blocks(Q4_K, n, k, seed=1)
    W = ctx.upload(Q4_K, w, k, n)
    dx = torch.zeros((16, k), dtype=torch.float32, device="cuda")
    dy = torch.zeros((16, n), dtype=torch.float32, device="cuda")
    rc = ctx.L.q35k_matmul_static_dev(W.h, dx.data_ptr(), dy.data_ptr(), 9, None)
    assert rc == q35k._lib.EINVAL
    assert b"tokens" in ctx.L.q35k_last_error(None)
    W.free()


def test_static_entry_rejects_scratch_overflow(env):
    # 8 tokens over 3600 super-blocks: the planar Q8_K alone is 3600 x 2336 B,
    # more than the 8 MiB array.
    torch, ctx = env
    k, n, m = 3600 * 256, 32, 8
    w = synth.kquant_blocks(Q4_K, n, k, seed=3)
    W = ctx.upload(Q4_K, w, k, n)
    dx = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    dy = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    rc = static_call(ctx, W, dx, dy, m, torch.cuda.current_stream())
    assert rc == q35k._lib.EINVAL
    msg = ctx.L.q35k_last_error(None)
    assert b"needs" in msg and b"bytes of scratch" in msg, msg
    W.free()


def test_static_entry_sizes_partials_for_its_tokens(env):
    # A Q6_K head at K = 5120 and one token: 4160 row groups x 2 K-splits of
    # partial sums take 1.1 MB at one token (8.5 MB if sized for 8 tokens, more
    # than the array): accepted, and bit-equal to the regular path.
    torch, ctx = env
    qt, k, n, m = Q6_K, 5120, 4160 * 32, 1
    w = np.tile(synth.kquant_blocks(qt, 1040, k, seed=9), (n // 1040, 1))
    W = ctx.upload(qt, w, k, n)
    stream = torch.cuda.current_stream()
    dx = torch.from_numpy(synth.activations(m, k, seed=4)).cuda()
    ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    ctx.matmul_dev(W, dx, ref, m, stream)
    rc = static_call(ctx, W, dx, out, m, stream)
    assert rc == 0, ctx.L.q35k_last_error(None).decode()
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32))
    W.free()
