"""Host-pointer calls on page-locked caller buffers (q35k_host_register):
x is read and y written in place instead of through the context's staging
buffers.  The result must be the same bits as with pageable buffers, for a
decode call (the GEMV stores y over the bus) and a prefill call (y copied
back after the GEMM), on repeated calls into the same persistent buffer."""

import numpy as np
import pytest

import q35k
from q35k import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qt,m", [(synth.Q6_K, 1), (synth.Q4_K, 2), (synth.Q5_K, 8), (synth.Q4_K, 64)])
def test_registered_buffers_give_the_same_bits(ctx, qt, m):
    k, n = 2560, 3000
    w = synth.kquant_blocks(qt, n, k, seed=31 + m)
    W = ctx.upload(qt, w, k, n)
    x_reg = q35k.page_aligned_empty((m, k))
    y_reg = q35k.page_aligned_empty((m, n))
    y_reg[...] = np.nan
    ctx.host_register(x_reg)
    ctx.host_register(y_reg)
    try:
        for call in range(3):
            x = synth.activations(m, k, seed=100 * call + m)
            x_reg[...] = x
            ref = ctx.matmul(W, x)  # pageable buffers
            out = ctx.matmul(W, x_reg, out=y_reg)
            assert out is y_reg
            assert np.array_equal(y_reg.view(np.uint32), ref.view(np.uint32)), f"call {call}"
    finally:
        ctx.host_unregister(x_reg)
        ctx.host_unregister(y_reg)
    W.free()


def test_register_twice_is_an_argument_error(ctx):
    a = q35k.page_aligned_empty(4096)
    ctx.host_register(a)
    try:
        with pytest.raises(q35k.ArgumentException):
            ctx.host_register(a)
    finally:
        ctx.host_unregister(a)
