"""Data-parallel takeover of a lost rank's sequences, on gloo ranks (CPU, no GPU).

Three ranks split 18 sequences.  In one run rank 1 fails with an exception after two sequences and
announces it; in the other rank 2 stops answering (no heartbeat) after one sequence.  The survivors
must claim and decode every unfinished sequence of the lost rank exactly once, and the results in
the store must equal a run without failures.  Decoding is a deterministic stand-in for the engine's
greedy decode; only store operations follow the failure, so no rank waits on a lost one.
"""
import hashlib
import os
import socket
import time

import pytest

N_SEQS = 18


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(seq: int) -> bytes:
    time.sleep(0.02)
    return hashlib.sha256(f"needle-{seq}".encode()).digest()


def _rank(rank, world, port, mode, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from datetime import timedelta
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load()
    from needle_b200 import dp
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=30))
    ledger = dp.ShardLedger(store, rank, world, N_SEQS, heartbeat_timeout=1.0)
    done = []
    try:
        if mode == "raise" and rank == 1:
            for k, s in enumerate(ledger.my_shard()):
                if k == 2:
                    raise RuntimeError("simulated rank failure")
                ledger.mark_done(s, _decode(s))
                done.append(s)
        elif mode == "silent" and rank == 2:
            s = ledger.my_shard()[0]
            ledger.mark_done(s, _decode(s))
            done.append(s)
            out[rank] = ("lost", done)
            return  # stops answering: no heartbeat, no finished mark
        else:
            mine = dp.run_rank(ledger, _decode, poll=0.05)
            done = sorted(mine)
    except RuntimeError:
        ledger.mark_failed()
        out[rank] = ("failed", done)
        return
    if rank == 0:
        # the store lives in this process: collect, then outlive the other survivors
        assert ledger.wait_finished(range(world))
        out["results"] = {s: ledger.result(s) for s in range(N_SEQS)}
    out[rank] = ("ok", done)


def _run(mode):
    import torch.multiprocessing as mp
    port = _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        mp.start_processes(_rank, args=(3, port, mode, out), nprocs=3, join=True, start_method="spawn")
        return dict(out)


@pytest.mark.parametrize("mode", ["raise", "silent"])
def test_lost_rank_sequences_are_taken_over_once(mode):
    out = _run(mode)
    lost = 1 if mode == "raise" else 2
    assert out[lost][0] == ("failed" if mode == "raise" else "lost")
    survivors = [r for r in range(3) if r != lost]
    assert all(out[r][0] == "ok" for r in survivors)
    decoded = [s for r in range(3) for s in out[r][1]]
    assert sorted(decoded) == list(range(N_SEQS)), "every sequence decoded exactly once"
    from needle_b200 import dp
    lost_shard = set(dp.shard(N_SEQS, lost, 3))
    taken = [s for r in survivors for s in out[r][1] if s in lost_shard]
    assert taken and len(taken) == len(lost_shard) - len(out[lost][1])
    assert out["results"] == {s: _decode(s) for s in range(N_SEQS)}


def test_shards_cover_every_sequence():
    from needle_b200 import dp
    for n in (0, 1, 7, 18, 4096):
        for world in (1, 2, 3, 8):
            parts = [dp.shard(n, r, world) for r in range(world)]
            flat = [s for p in parts for s in p]
            assert flat == list(range(n))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
