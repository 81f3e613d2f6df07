"""Row-sharded matmul through the C ABI (q35k_shard_*).

One GPU: a group of one device computes exactly what the single-GPU entry
point computes (same kernels, same per-row arithmetic), through both gather
modes and both ways of building a group.  Two or more GPUs (when the box has
them): the NCCL all-gather and the peer-copy gather against the oracle and
the single-GPU result; and one process per GPU (ncclCommInitRank).
"""

import os

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_err(y, r):
    return float(np.abs(y.astype(np.float64) - r).max() / max(np.abs(r).max(), 1e-30))


def _ngpus():
    torch = pytest.importorskip("torch")
    return torch.cuda.device_count()


@pytest.mark.parametrize("qt,k,n,m", [(Q4_K, 2560, 9728, 1), (Q6_K, 2560, 1000, 3), (Q5_K, 1024, 500, 8),
                                      (Q4_K, 2560, 2048, 64)])
@pytest.mark.parametrize("mode", [q35k.GATHER_NCCL, q35k.GATHER_PEER, q35k.GATHER_FUSED])
def test_one_device_group_matches_single_gpu(ctx, qt, k, n, m, mode):
    w = synth.kquant_blocks(qt, n, k, seed=n + m)
    x = synth.activations(m, k, seed=m)
    W = ctx.upload(qt, w, k, n)
    ref = ctx.matmul(W, x)
    sh = q35k.Shard(devices=[0])
    sw = sh.upload(qt, w, k, n)
    y = sh.matmul(sw, x, gather=mode)
    assert (y == ref).all()
    sw.free()
    sh.close()
    W.free()


def test_rank_group_of_one(ctx):
    qt, k, n, m = Q4_K, 2560, 777, 2
    w = synth.kquant_blocks(qt, n, k, seed=3)
    x = synth.activations(m, k, seed=4)
    W = ctx.upload(qt, w, k, n)
    ref = ctx.matmul(W, x)
    sh = q35k.Shard(nranks=1, rank=0, nccl_id=None, device=0)
    sw = sh.upload(qt, w, k, n)
    assert (sh.matmul(sw, x) == ref).all()
    sw.free()
    sh.close()
    W.free()


def test_shard_device_pointer_path(ctx):
    torch = pytest.importorskip("torch")
    qt, k, n, m = Q6_K, 2560, 4000, 1
    w = synth.kquant_blocks(qt, n, k, seed=5)
    x = synth.activations(m, k, seed=6)
    sh = q35k.Shard(devices=[0])
    sw = sh.upload(qt, w, k, n)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
    sh.matmul_dev(sw, [dx], [dy], m)
    sh.sync()
    assert (dy.cpu().numpy() == sh.matmul(sw, x)).all()
    sw.free()
    sh.close()


@pytest.mark.parametrize("ndev", [2, 4, 8])
@pytest.mark.parametrize("qt,k,n,m", [(Q4_K, 5120, 27648, 1), (Q4_K, 5120, 27648, 8), (Q6_K, 2560, 151936, 1),
                                      (Q4_K, 2560, 9728, 512), (Q5_K, 1024, 1000, 3),
                                      # 108 row groups per rank at 2 GPUs (cfg4's share at 8): split-K clusters
                                      (Q4_K, 5120, 6912, 1), (Q4_K, 5120, 6912, 8)])
@pytest.mark.parametrize("mode", [q35k.GATHER_NCCL, q35k.GATHER_PEER, q35k.GATHER_FUSED])
def test_multi_gpu_group(ctx, oracle_mod, ndev, qt, k, n, m, mode):
    if _ngpus() < ndev:
        pytest.skip(f"needs {ndev} GPUs")
    w = synth.kquant_blocks(qt, n, k, seed=1)
    x = synth.activations(m, k, seed=2)
    W = ctx.upload(qt, w, k, n)
    single = ctx.matmul(W, x)
    W.free()
    sh = q35k.Shard(devices=list(range(ndev)))
    sw = sh.upload(qt, w, k, n)
    y = sh.matmul(sw, x, gather=mode)
    assert rel_err(y, single.astype(np.float64)) <= 1e-5
    if n * k <= 30_000_000:
        ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=os.cpu_count() or 1)
        assert rel_err(y, ref) <= TOL
    sw.free()
    sh.close()


def _rank_proc(rank, nranks, nccl_id, qt, k, n, m, mode, q):
    import q35k as Q

    sh = Q.Shard(nranks=nranks, rank=rank, nccl_id=nccl_id, device=rank)
    w = synth.kquant_blocks(qt, n, k, seed=1)
    x = synth.activations(m, k, seed=2)
    sw = sh.upload(qt, w, k, n)
    y = sh.matmul(sw, x, gather=mode)
    # repeated calls alternate the fused gather's buffers and call counters
    same = all((sh.matmul(sw, x, gather=mode) == y).all() for _ in range(3))
    if mode == Q.GATHER_FUSED:
        # phase trace of one call: six increasing timestamps on this device
        sh.set_trace(True)
        same = same and (sh.matmul(sw, x, gather=mode) == y).all()
        tr = sh.trace(0)
        sh.set_trace(False)
        ph = [tr[k] for k in Q.Shard.TRACE_PHASES]
        same = same and ph[0] <= ph[1] <= ph[4] <= ph[5] and ph[2] <= ph[3] <= ph[5]
    q.put((rank, y, same))
    sw.free()
    sh.close()


@pytest.mark.parametrize("mode", [q35k.GATHER_NCCL, q35k.GATHER_FUSED])
def test_process_per_gpu_group(ctx, mode):
    if _ngpus() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp

    qt, k, n, m = Q4_K, 5120, 27648, 1
    nid = q35k.nccl_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_rank_proc, args=(r, 2, nid, qt, k, n, m, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in procs]
    res = {r: y for r, y, _ in got}
    assert all(same for _, _, same in got)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = synth.kquant_blocks(qt, n, k, seed=1)
    x = synth.activations(m, k, seed=2)
    W = ctx.upload(qt, w, k, n)
    single = ctx.matmul(W, x)
    W.free()
    for r in range(2):
        assert rel_err(res[r], single.astype(np.float64)) <= 1e-5


def _skip_proc(rank, nid, q):
    """Rank `rank` of a 2-GPU fused-gather group: call 1 on both ranks, call
    2 on rank 0 only (rank 1 leaves between steps, nothing in flight), then
    the collective reset and call 3 on both ranks."""
    import q35k as Q

    try:
        sh = Q.Shard(nranks=2, rank=rank, nccl_id=nid, device=rank)
        sh.set_wait_limit(50)
        qt, k, n = Q4_K, 2560, 4096
        w = synth.kquant_blocks(qt, n, k, seed=11)
        sw = sh.upload(qt, w, k, n)
        x1 = synth.activations(1, k, seed=12)
        x3 = synth.activations(1, k, seed=13)
        y1 = sh.matmul(sw, x1, gather=Q.GATHER_FUSED)
        timed_out = None
        if rank == 0:
            try:
                sh.matmul(sw, x1, gather=Q.GATHER_FUSED)
                timed_out = False
            except Q.TimeoutException:
                timed_out = True
        sh.reset()
        y3 = sh.matmul(sw, x3, gather=Q.GATHER_FUSED)
        y3b = sh.matmul(sw, x3, gather=Q.GATHER_FUSED)
        q.put((rank, None, timed_out, y1, y3, y3b))
        sw.free()
        sh.close()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None, None, None, None))


def test_missing_rank_times_out_and_group_recovers(ctx):
    """Failure detection without a GPU fault: a bounded flag wait (50 ms) runs
    out because a peer skipped the call; the call reports TimeoutException
    (Q35K_ETIMEOUT), and after q35k_shard_reset on both ranks the next calls
    are correct again."""
    if _ngpus() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    nid = q35k.nccl_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_skip_proc, args=(r, nid, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, err, timed_out, y1, y3, y3b = q.get(timeout=300)
        got[r] = (err, timed_out, y1, y3, y3b)
    for p in procs:
        p.join(timeout=120)
    assert got[0][0] is None and got[1][0] is None, (got[0][0], got[1][0])
    assert got[0][1] is True
    qt, k, n = Q4_K, 2560, 4096
    W = ctx.upload(qt, synth.kquant_blocks(qt, n, k, seed=11), k, n)
    r1 = ctx.matmul(W, synth.activations(1, k, seed=12))
    r3 = ctx.matmul(W, synth.activations(1, k, seed=13))
    W.free()
    for r in range(2):
        _, _, y1, y3, y3b = got[r]
        assert rel_err(y1, r1.astype(np.float64)) <= 1e-5
        assert rel_err(y3, r3.astype(np.float64)) <= 1e-5
        assert (y3 == y3b).all()


def test_wait_limit_is_validated(ctx):
    sh = q35k.Shard(devices=[0])
    with pytest.raises(q35k.ArgumentException):
        sh.set_wait_limit(0)
    sh.set_wait_limit(100)
    sh.reset()
    sh.close()
