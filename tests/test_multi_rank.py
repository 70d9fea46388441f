"""Multi-rank host logic of bench.py on CPU: two `gloo` ranks, each with its
own sequence; the job's time is the max over ranks (no data-path collective)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        prompt = bench.prompt_for(rank, 32000, 64)
        mine = [10.0 + rank, 5.0 - rank]
        # this rank's share of the 64 sequences, gathered to check
        # that the ranks cover every sequence exactly once.
        share = bench.c5_partition(64, rank, world)
        seqs = [None] * world
        dist.all_gather_object(seqs, share)
        out[rank] = (bench.max_over_ranks(mine, dist), prompt.tolist(), seqs)
    finally:
        dist.destroy_process_group()


def test_two_ranks_partition_sequences_and_take_the_slowest():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
        res = dict(out)
    assert res[0][0] == res[1][0] == [11.0, 5.0]
    p0, p1 = np.array(res[0][1]), np.array(res[1][1])
    assert not np.array_equal(p0, p1)  # each rank has its own sequence
    import bench
    assert np.array_equal(p0, bench.prompt_for(0, 32000, 64))
    # The C5 partition seen by both ranks: 0..63, each once, 32 per rank.
    for r in range(world):
        seqs = res[r][2]
        flat = sorted(q for share in seqs for q in share)
        assert flat == list(range(64))
        assert [len(share) for share in seqs] == [32, 32]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_c5_partition_covers_every_sequence_once(world):
    import bench
    shares = [bench.c5_partition(64, r, world) for r in range(world)]
    assert sorted(q for s in shares for q in s) == list(range(64))
    assert all(len(s) == 64 // world for s in shares)
    with pytest.raises(ValueError):
        bench.c5_partition(64, world, world)


def test_single_process_needs_no_group():
    import bench
    assert bench.max_over_ranks([1.0, 2.0]) == [1.0, 2.0]
