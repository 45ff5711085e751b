"""The multi-GPU host logic of bench.py on two gloo ranks (CPU): each rank draws disjoint steered/unsteered pairs of
one global set, the timing reduction gives every rank the max over ranks, and the results (token ids, reduced
captures, and logits on request) are gathered to rank 0 in rank order."""
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prompts = bench.rank_prompts(rank, npairs=3, P=16, V=1000)
        times = bench.max_over_ranks([10.0 + rank, 5.0 - rank])
        got = bench.gather_to_rank0(np.arange(6, dtype=np.uint32).reshape(2, 3) + 100 * rank)
        logits = bench.gather_to_rank0(np.linspace(-1.5, 2.5, 8, dtype=np.float32).reshape(2, 4) * (rank + 1))
        out[rank] = (np.stack(prompts), times, got, logits)
    finally:
        dist.destroy_process_group()


def test_two_ranks_partition_pairs_and_reduce_max():
    import bench

    world, port = 2, _free_port()
    out = mp.Manager().dict()
    mp.start_processes(_rank_main, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    p0, t0, g0, l0 = out[0]
    p1, t1, g1, l1 = out[1]
    assert t0 == t1 == [11.0, 5.0]
    # results gathered to rank 0 in rank order (token ids are uint32 on the host, moved as int32)
    want = np.stack([np.arange(6).reshape(2, 3) + 100 * r for r in range(world)]).astype(np.int32)
    assert g1 is None and g0.dtype == np.int32 and np.array_equal(g0, want)
    # logits (on request) keep their float32 values
    lw = np.stack([np.linspace(-1.5, 2.5, 8, dtype=np.float32).reshape(2, 4) * (r + 1) for r in range(world)])
    assert l1 is None and l0.dtype == np.float32 and np.array_equal(l0, lw)
    # the two ranks' pairs are the first six pairs of the one-rank stream, split in order
    whole = np.stack(bench.rank_prompts(0, npairs=6, P=16, V=1000))
    assert np.array_equal(np.concatenate([p0, p1]), whole)
    assert not np.array_equal(p0, p1)


def test_max_over_ranks_without_a_process_group_is_identity():
    import bench

    assert bench.max_over_ranks([3.0, 1.5]) == [3.0, 1.5]
    assert np.array_equal(bench.gather_to_rank0(np.array([[1, 2]], np.uint32)), np.array([[[1, 2]]], np.int32))
