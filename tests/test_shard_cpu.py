"""Multi-rank host logic on CPU: two gloo ranks shard the sequences of a
batch, each decodes its own slice (C oracle greedy loop), and the gathered
token streams equal the single-process run; the timing reduction takes the
max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from freeml_b200.shard import max_over_ranks, shard_bounds
from oracle import oracle as O

SHAPE = (97, 48, 64, 2, 2)  # V C d H L
NSEQ, PLEN, NEW = 5, 6, 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _streams(rows):
    s = O.LMShape(*SHAPE)
    w = O.init_weights(s, 11)
    prompts = np.random.RandomState(3).randint(0, SHAPE[0], size=(NSEQ, PLEN)).astype(np.uint32)
    return [O.greedy(s, w, prompts[r], NEW)[0] for r in rows]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    b, e = shard_bounds(NSEQ, world, rank)
    mine = _streams(range(b, e))
    gathered = [None] * world
    dist.all_gather_object(gathered, (b, e, [x.tolist() for x in mine]))
    slowest = max_over_ranks(float(rank + 1), dist)
    if rank == 0:
        out.put((gathered, slowest))
    dist.barrier()
    dist.destroy_process_group()


def test_shard_bounds_cover_every_sequence_once():
    for total in (1, 5, 32):
        for world in range(1, min(total, 8) + 1):
            got = [shard_bounds(total, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [e - b for b, e in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(2, 3, 0)


def test_two_gloo_ranks_match_one_process():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, slowest = out.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert slowest == 2.0
    assert [g[:2] for g in gathered] == [shard_bounds(NSEQ, 2, r) for r in range(2)]
    sharded = [np.array(s, np.uint32) for g in gathered for s in g[2]]
    for a, b in zip(sharded, _streams(range(NSEQ))):
        np.testing.assert_array_equal(a, b)
