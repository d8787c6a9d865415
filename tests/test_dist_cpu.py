"""world_size-2 gloo tests of the multi-GPU host logic, on CPU.

The sequence-sharded decode merges each rank's split-K records into one
record per query row and all-gathers those; these tests run that exchange for
real (gloo) with records computed and merged by the oracle and check the final
merge against the unsharded oracle.  Kernels are covered by the -m gpu tests."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kudahitam.dist import gather_records, max_over_ranks, shard_range


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _records(logits: np.ndarray, vals: np.ndarray) -> np.ndarray:
    """(m, l, acc[D]) over rows of one shard; empty shard -> zeros."""
    if logits.size == 0:
        return np.zeros(vals.shape[-1] + 2)
    m = logits.max()
    p = np.exp(logits - m)
    return np.concatenate([[m, p.sum()], p @ vals])


def _worker(rank, world, port, S, D, G, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(5)
        logits = rng.standard_normal((G, S)) * 3.0
        vals = rng.standard_normal((G, S, D))
        a, b = shard_range(S, world, rank)
        n_splits = 3
        local = np.zeros((G, n_splits, D + 2))
        for g in range(G):
            for k in range(n_splits):
                lo = a + (b - a) * k // n_splits
                hi = a + (b - a) * (k + 1) // n_splits
                local[g, k] = _records(logits[g, lo:hi], vals[g, lo:hi])
        from oracle.oracle import merge_partials
        m_loc, l_loc, acc_loc = merge_partials(local)  # this rank's splits
        mine = np.concatenate([m_loc[:, None], l_loc[:, None], acc_loc], axis=1)
        full = gather_records(torch.from_numpy(mine), None).numpy()
        assert full.shape == (world, G, D + 2)
        assert np.array_equal(full[rank], mine)
        M, L, acc = merge_partials(full.transpose(1, 0, 2))
        got = acc / L[:, None]
        p = np.exp(logits - logits.max(1, keepdims=True))
        want = np.einsum("gs,gsd->gd", p / p.sum(1, keepdims=True), vals)
        assert np.allclose(got, want, rtol=1e-10, atol=1e-12)
        assert max_over_ranks(float(rank) + 0.5) == world - 0.5
        q.put(("ok", rank))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("fail", f"rank {rank}: {e!r}"))
    finally:
        dist.destroy_process_group()


def _run(world, S):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, S, 16, 3, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in res), res


def test_seq_sharded_combine_world2():
    _run(2, S=101)


def test_seq_sharded_combine_world2_with_empty_splits():
    # 4 rows over 2 ranks x 3 splits: some splits own no rows
    _run(2, S=4)


def test_peer_exchange_epoch_parity_alternates_across_the_wrap():
    from kudahitam.dist import next_epoch
    e = 0
    seq = []
    for _ in range(3):
        e = next_epoch(e)
        seq.append(e)
    assert seq == [1, 2, 3]
    e = 0xFFFFFFFE
    seq = []
    for _ in range(4):
        e = next_epoch(e)
        seq.append(e)
    assert seq == [0xFFFFFFFF, 2, 3, 4]
    # consecutive epochs never share a buffer/flag set, and 0 never recurs
    e = 0xFFFFFFF0
    for _ in range(64):
        n = next_epoch(e)
        assert n != 0 and (n & 1) != (e & 1)
        e = n
