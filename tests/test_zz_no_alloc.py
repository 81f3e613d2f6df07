"""q35k_matmul_static_dev: the decode matmul that allocates nothing.

Callers that cannot let a library allocate device memory during a call (a
host whose device memory is all owned by its own arena, or a decode loop
where a cudaMalloc/cudaFree would synchronize and stall the device) use this
entry point; its scratch lives in one fixed array that the library holds on
every GPU.  Checked here through the C ABI against q35k_matmul_dev, on two
calls in a row (the array keeps the previous call's contents, so the second
call shows that what must start at zero is cleared).  Collected last; works
alone in a fresh process as well as after the other tests.
"""

import ctypes

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

pytestmark = pytest.mark.gpu

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


@pytest.mark.parametrize("qt,k,n,m", [
    (Q6_K, 2560, 9728, 1),    # decode: the GEMV quantizes x itself (no Q8_K scratch)
    (Q4_K, 2560, 2048, 1),    # fewer row groups than SMs: split-K partials + counters
    (Q5_K, 9728, 2560, 8),    # Q8_K scratch + split-K partials + counters
    (Q4_K, 5120, 1000, 3),    # ragged rows
])
def test_static_entry_matches_regular_entry(env, qt, k, n, m):
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
        rc = ctx.L.q35k_matmul_static_dev(W.h, dx.data_ptr(), out.data_ptr(), m,
                                          ctypes.c_void_p(stream.cuda_stream or 1))
        assert rc == 0, ctx.L.q35k_last_error(None).decode()
        torch.cuda.synchronize()
        got, want = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) <= TOL, f"call {call}"
    W.free()


def test_static_entry_rejects_oversize(env):
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
