"""The N>1 bookkeeping of bench.py on CPU: two gloo ranks (no GPU), each with its own workload
shard; rank 0 must see the max time over ranks and the summed token counts."""
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    prompts, gens = bench.workload(rank, 6)
    local = [10.0 + rank, 100 + rank, 1000 + 10 * rank, 20.0 - rank, 7 + rank, 115 * (rank + 1)]
    agg = bench.aggregate(local, dist)
    out[rank] = (agg, [len(p) for p in prompts], [int(g) for g in gens])
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_aggregation_and_sharding():
    import torch.multiprocessing as mp
    port = _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        mp.start_processes(_rank_main, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
        r0, r1 = out[0], out[1]
    assert r0[0] == r1[0]  # every rank computes the same totals
    ms, gen, proc, e2e_ms, e2e_gen, launches = r0[0]
    assert ms == 11.0 and gen == 201 and proc == 2010 and e2e_ms == 20.0 and e2e_gen == 15 and launches == 345
    assert r0[1] != r1[1]  # each rank decodes its own sequences (weak scaling, no shared data)
    for lens, gens in (r0[1:], r1[1:]):
        assert all(32 <= n <= 1024 for n in lens) and all(16 <= g <= 128 for g in gens)


def _toolcall_rank(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    local = [100.0 + rank, 1000 + rank, 500, 3 + rank, rank, 40 + rank, 2.0 + rank, 7000, 2048, 10, 20,
             5.0 - rank, 9.0 + rank]
    out[rank] = bench.aggregate_toolcall(local, dist)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_toolcall_aggregation():
    """Config 5 on two ranks: times and step counts are the maximum over ranks, counts the sum."""
    import torch.multiprocessing as mp
    port = _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        mp.start_processes(_toolcall_rank, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
        r0, r1 = out[0], out[1]
    assert r0 == r1
    assert r0 == [101.0, 2001.0, 1000.0, 7.0, 1.0, 41.0, 3.0, 14000.0, 4096.0, 20.0, 40.0, 5.0, 10.0]


def test_single_process_aggregation_is_identity():
    import bench
    assert bench.aggregate([5.0, 3, 9, 6.0, 2, 115]) == (5.0, 3.0, 9.0, 6.0, 2.0, 115)
    assert bench.aggregate_toolcall([1, 2, 3]) == [1.0, 2.0, 3.0]
