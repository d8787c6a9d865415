"""Multi-GPU paths on real devices (NCCL over NVLink), one process per GPU.
Skipped when fewer than two GPUs are visible.

* sequence-sharded decode: every rank holds S/N cached rows per group, runs
  the split-K partial kernel, merges its splits into one record per query row
  and the records are exchanged by one all-gather; the result must equal the
  single-GPU decode of the whole cache;
* the same decode with the record exchange fused into the merge kernel over
  peer memory (symmetric memory, NVLink stores and flags) must equal the
  all-gather path bit for bit, call after call; fused into the partial
  kernel instead, within 1e-5 normwise;
* row-sharded compression: ranks compress disjoint batch x head slices with
  no communication; the union must equal the single-GPU result bit for bit."""
import datetime
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from kudahitam import dist as khdist
        from kudahitam import lloyd_max, ops, rademacher
        D, G, S = 128, 6, 3000
        dk, dv, c = rademacher(D, 1), rademacher(D, 2), lloyd_max(1, D)
        g = torch.Generator().manual_seed(0)
        k = torch.randn(G, S, D, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(G, S, D, generator=g).to(torch.bfloat16).to(dev)
        qv = torch.randn(G, D, generator=g).to(dev)
        a, b = khdist.shard_range(S, world, rank)
        pk = ops.compress(k[:, a:b].contiguous(), dk, c)
        pv = ops.compress(v[:, a:b].contiguous(), dv, c)
        got = khdist.decode_attention_seq_sharded(qv, pk, pv, dk, dv, c, 1 / math.sqrt(D),
                                                  n_splits=3)
        full = ops.decode_attention(qv, ops.compress(k, dk, c), ops.compress(v, dv, c), dk, dv,
                                    c, 1 / math.sqrt(D), n_splits=3 * world)
        torch.cuda.synchronize()
        err = ((got - full).abs().max() / full.abs().max()).item()
        # the same step with the record exchange fused into the merge over
        # peer memory: bitwise the NCCL result, over calls that alternate the
        # two buffer sets
        from kudahitam import _lib
        ex = khdist.PeerRecordExchange(G, D, device=dev)
        peer_same = True
        for _ in range(5):
            alt = khdist.decode_attention_seq_sharded(qv, pk, pv, dk, dv, c, 1 / math.sqrt(D),
                                                      n_splits=3, exchange=ex)
            torch.cuda.synchronize()
            peer_same = peer_same and torch.equal(alt, got)
        peer_same = peer_same and _lib.device_error() == 0
        del ex
        # the exchange fused into the partial kernel (records of every split
        # stored to every rank, one combine): the same attention within 1e-5
        # normwise (merge order differs), over calls on both buffer sets
        exf = khdist.PeerRecordExchange(G, D, device=dev, n_parts=3)
        fused_err = 0.0
        for _ in range(5):
            alt = khdist.decode_attention_seq_sharded(qv, pk, pv, dk, dv, c, 1 / math.sqrt(D),
                                                      n_splits=3, exchange=exf)
            torch.cuda.synchronize()
            fused_err = max(fused_err, ((alt - got).abs().max() / got.abs().max()).item())
        peer_same = peer_same and fused_err < 1e-5 and _lib.device_error() == 0
        del exf
        torch.cuda.synchronize()
        dist.barrier()
        # compression shards: no communication, bit-identical to the whole
        ra, rb = khdist.shard_range(G, world, rank)
        mine = ops.compress(k[ra:rb], dk, c)
        ref = ops.compress(k, dk, c).rows(ra * S, rb * S)
        same = torch.equal(mine.code, ref.code) and torch.equal(mine.res, ref.res)
        q.put(("ok", rank, err, same and peer_same))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("fail", rank, repr(e), False))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_seq_sharded_decode_and_row_sharded_compress_nccl():
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for status, rank, err, same in res:
        assert status == "ok", (rank, err)
        assert err < 1e-4, (rank, err)
        assert same, rank
