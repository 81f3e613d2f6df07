"""Host-side logic of the row-sharded matmul, on CPU.

The row split (q35k.shard_rows / shard_range, the same rule as the C library)
must cover every output row exactly once on 32-row tile boundaries, and
gathering the ranks' slices must reassemble the full y.  The exchange is
exercised with world_size-2 torch.distributed (gloo) ranks, each computing its
slice with the CPU oracle, as the GPU ranks do with the kernels.
"""

import os
import socket

import numpy as np
import pytest

import q35k
from q35k import synth
from q35k.synth import Q4_K, Q6_K


@pytest.mark.parametrize("nranks", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("n_out", [1, 31, 32, 33, 100, 2560, 9728, 27648, 151936])
def test_shard_ranges_cover_rows(n_out, nranks):
    n = q35k.shard_rows(n_out, nranks)
    assert n * nranks >= n_out and (n - 1) * nranks < n_out  # an equal share
    covered = []
    for r in range(nranks):
        r0, r1 = q35k.shard_range(n_out, nranks, r)
        assert 0 <= r0 <= r1 <= n_out
        assert r1 - r0 <= n
        covered.extend(range(r0, r1))
    assert covered == list(range(n_out))


def _gather_layout(slices, tokens, n_shard, n_out):
    """Reassembly of the gathered [rank][tokens][n_shard] slots into y, as the
    library's gather_permute_kernel does."""
    g = np.zeros((len(slices), tokens, n_shard), np.float32)
    for r, sl in enumerate(slices):
        g[r, :, : sl.shape[1]] = sl
    y = np.empty((tokens, n_out), np.float32)
    for c in range(n_out):
        y[:, c] = g[c // n_shard, :, c % n_shard]
    return y


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, qt, k, n, m, out_path):
    import torch
    import torch.distributed as dist

    import oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        w = synth.kquant_blocks(qt, n, k, seed=7)
        x = synth.activations(m, k, seed=8)
        r0, r1 = q35k.shard_range(n, world, rank)
        n_shard = q35k.shard_rows(n, world)
        mine = np.zeros((m, n_shard), np.float32)
        if r1 > r0:
            mine[:, : r1 - r0] = oracle.Weight(qt, w[r0:r1], k, r1 - r0).matmul(x, threads=1)
        # the exchange: every rank receives every rank's [tokens][n_shard] slot
        parts = [torch.zeros((m, n_shard)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(mine))
        y = _gather_layout([p.numpy() for p in parts], m, n_shard, n)
        if rank == 0:
            np.save(out_path, y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("qt,k,n,m", [(Q4_K, 512, 300, 1), (Q6_K, 768, 129, 3), (Q4_K, 256, 64, 2)])
def test_gloo_two_ranks_reassemble_full_output(tmp_path, oracle_mod, qt, k, n, m):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp

    out = str(tmp_path / "y.npy")
    port = _free_port()
    mp.spawn(_rank_main, args=(2, port, qt, k, n, m, out), nprocs=2, join=True)
    y = np.load(out)
    w = synth.kquant_blocks(qt, n, k, seed=7)
    x = synth.activations(m, k, seed=8)
    ref = oracle_mod.Weight(qt, w, k, n).matmul(x, threads=1)
    # each row's dot product does not depend on the other rows
    err = np.abs(y.astype(np.float64) - ref).max() / np.abs(ref).max()
    assert err <= 1e-6


# ---------------------------------------------------------------------------
# The fused gather's protocol and its failure handling, restated on CPU ranks:
# each rank stores its slice into every peer's alternate area as words that
# carry the call number (its call counter + 1), waits (bounded) until every
# peer word of this call has arrived in its own area, and advances its
# counter; a missing rank makes the others' waits run out, and the
# two-barrier reset (q35k_shard_reset) clears every buffer and counter.  The
# peers' memory is a TCPStore shared by the gloo ranks.
# ---------------------------------------------------------------------------

class _FusedGatherModel:
    def __init__(self, store, rank, world, wait_s):
        self.store, self.rank, self.world, self.wait_s = store, rank, world, wait_s
        self.seq = 0

    def call(self, my_slice):
        import time

        ep = self.seq + 1
        half = ep & 1
        word = np.concatenate([np.full(my_slice.shape, ep, np.uint32).view(np.float32), my_slice])
        for j in range(self.world):  # the GEMV's stores into every peer's area: (call number, values)
            if j != self.rank:
                self.store.set(f"area/{j}/{half}/{self.rank}", word.tobytes())
        parts = {self.rank: my_slice}
        deadline = time.monotonic() + self.wait_s
        timed_out = False
        for j in range(self.world):
            if j == self.rank:
                continue
            key = f"area/{self.rank}/{half}/{j}"
            while True:
                if self.store.check([key]):
                    got = np.frombuffer(self.store.get(key), dtype=np.float32)
                    n = got.size // 2
                    if n and (got[:n].view(np.uint32) == ep).all():
                        parts[j] = got[n:].copy()
                        break
                if time.monotonic() > deadline:
                    timed_out = True
                    break
            if timed_out:
                break
        self.seq = ep  # the gather kernel advances the counter even when a wait ran out
        if timed_out:
            raise TimeoutError("a peer's words of this call did not arrive")
        return np.concatenate([parts[j] for j in range(self.world)])

    def reset(self, barrier):
        barrier()  # nothing of any rank still stores into this rank's buffer
        for j in range(self.world):
            for half in (0, 1):
                self.store.set(f"area/{self.rank}/{half}/{j}", b"")
        self.seq = 0
        barrier()  # every buffer is clear before anyone's next call


def _protocol_rank(rank, world, port, out_path):
    import datetime

    import torch.distributed as dist

    import oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0, timeout=datetime.timedelta(seconds=60))
        qt, k, n = Q4_K, 512, 256
        w = synth.kquant_blocks(qt, n, k, seed=21)
        r0, r1 = q35k.shard_range(n, world, rank)
        W = oracle.Weight(qt, w[r0:r1], k, r1 - r0)
        model = _FusedGatherModel(store, rank, world, wait_s=0.3)
        xs = [synth.activations(1, k, seed=30 + i) for i in range(4)]
        outs, events = [], []
        outs.append(model.call(W.matmul(xs[0], threads=1)[0]))
        if rank == 0:  # call 2: rank 1 leaves between steps
            try:
                model.call(W.matmul(xs[1], threads=1)[0])
                events.append("no timeout")
            except TimeoutError:
                events.append("timeout")
        model.reset(dist.barrier)
        for x in xs[2:]:
            outs.append(model.call(W.matmul(x, threads=1)[0]))
        np.save(out_path.format(rank), np.stack(outs))
        with open(out_path.format(rank) + ".txt", "w") as f:
            f.write(",".join(events))
    finally:
        dist.destroy_process_group()


def test_gloo_missing_rank_times_out_and_reset_recovers(tmp_path, oracle_mod):
    pytest.importorskip("torch")
    import torch.multiprocessing as mp

    port = _free_port()
    out = str(tmp_path / "y{}.npy")
    mp.spawn(_protocol_rank, args=(2, port, out), nprocs=2, join=True)
    assert open(out.format(0) + ".txt").read() == "timeout"
    qt, k, n = Q4_K, 512, 256
    w = synth.kquant_blocks(qt, n, k, seed=21)
    W = oracle_mod.Weight(qt, w, k, n)
    refs = [W.matmul(synth.activations(1, k, seed=30 + i), threads=1)[0] for i in (0, 2, 3)]
    for r in range(2):
        ys = np.load(out.format(r))
        for y, ref in zip(ys, refs):
            assert np.array_equal(y, ref)
