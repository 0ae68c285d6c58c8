"""Data-parallel sequence assignment with takeover of a lost rank's work (host side, no GPU).

Independent sequences are split over the ranks of one node in contiguous shards (one engine per GPU,
no collectives on the data path).  The reference decodes one sequence per runtime and has no
parallelism, so this has no counterpart there; it is the failure handling a multi-GPU deployment of
the engine needs: a rank that dies or stops answering must not take its sequences with it.

Every rank keeps a heartbeat and a record of each sequence it finished (with its result) in the
process group's key-value store.  A rank that catches an error announces itself failed; a rank that
stops updating its heartbeat for `heartbeat_timeout` seconds is presumed lost.  The survivors then
claim the lost rank's unfinished sequences one at a time -- a claim is an atomic `store.add` on the
sequence's key, so exactly one survivor decodes each -- and record them like their own.  Decoding is
deterministic (greedy, exact numerics), so a sequence redone after a presumed loss gives the same
result the lost rank would have.  Only store operations are used after a failure: no rank ever waits
in a collective for a rank that is gone.
"""
from __future__ import annotations

import time
from typing import Callable, Dict, Iterable, List, Optional


def shard(n_seqs: int, rank: int, world: int) -> range:
    """Contiguous shard of rank `rank`: sizes differ by at most one, lower ranks first."""
    base, extra = divmod(n_seqs, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


class ShardLedger:
    """Progress of one rank in a torch.distributed Store (TCPStore, FileStore, ...)."""

    def __init__(self, store, rank: int, world: int, n_seqs: int, heartbeat_timeout: float = 5.0,
                 prefix: str = "needle_dp"):
        self.store, self.rank, self.world, self.n_seqs = store, rank, world, n_seqs
        self.timeout = heartbeat_timeout
        self.prefix = prefix
        self.heartbeat()
        # every rank is up before any is judged: a rank that has not started yet is not lost
        self.store.wait([self._k("beat", r) for r in range(world)])

    def _k(self, *parts) -> str:
        return "/".join([self.prefix, *map(str, parts)])

    # -- this rank ------------------------------------------------------------------------------
    def my_shard(self) -> range:
        return shard(self.n_seqs, self.rank, self.world)

    def heartbeat(self) -> None:
        self.store.set(self._k("beat", self.rank), repr(time.time()))

    def mark_done(self, seq: int, result: bytes) -> None:
        """Records a decoded sequence; the first record of each sequence counts towards the total
        (a sequence redone after a presumed loss is the same result, counted once)."""
        self.store.set(self._k("result", seq), result)
        if self.store.add(self._k("done", seq), 1) == 1:
            self.store.add(self._k("ndone"), 1)
        self.heartbeat()

    def mark_failed(self) -> None:
        """Announces that this rank stops (its unfinished sequences go to the others)."""
        self.store.set(self._k("failed", self.rank), b"1")

    def mark_finished(self) -> None:
        """Announces that this rank completed its shard and its takeovers."""
        self.store.set(self._k("finished", self.rank), b"1")

    # -- the others -----------------------------------------------------------------------------
    def _has(self, key: str) -> bool:
        return self.store.check([key])

    def is_done(self, seq: int) -> bool:
        return self.store.add(self._k("done", seq), 0) > 0

    def all_done(self) -> bool:
        return self.store.add(self._k("ndone"), 0) >= self.n_seqs

    def lost_ranks(self) -> List[int]:
        """Ranks that announced failure, or whose heartbeat is older than the timeout while they
        have not finished."""
        now = time.time()
        lost = []
        for r in range(self.world):
            if r == self.rank or self._has(self._k("finished", r)):
                continue
            if self._has(self._k("failed", r)):
                lost.append(r)
                continue
            key = self._k("beat", r)
            if not self._has(key) or now - float(self.store.get(key).decode()) > self.timeout:
                lost.append(r)
        return lost

    def claim(self, seq: int, lost: Iterable[int]) -> bool:
        """True for exactly one caller per sequence (the survivor that will decode it).  Claims are
        numbered by an atomic counter; a claim whose claimer is itself lost may be taken again."""
        key = self._k("claim", seq)
        n = self.store.add(key, 0)
        if n > 0:
            who_key = self._k("claimer", seq, n)
            if not self._has(who_key) or int(self.store.get(who_key).decode()) not in set(lost):
                return False  # held by a live rank (or being recorded right now)
        got = self.store.add(key, 1)
        if got != n + 1:
            return False
        self.store.set(self._k("claimer", seq, got), str(self.rank))
        return True

    def orphans(self, ranks: Iterable[int]) -> List[int]:
        return [s for r in ranks for s in shard(self.n_seqs, r, self.world) if not self.is_done(s)]

    def wait_finished(self, ranks: Iterable[int], timeout: float = 60.0) -> bool:
        """Waits until the given ranks have finished or are lost (the rank that hosts the store
        must outlive the others).  False if the time ran out."""
        end = time.time() + timeout
        pending = set(ranks) - {self.rank}
        while pending and time.time() < end:
            lost = set(self.lost_ranks())
            pending = {r for r in pending if not self._has(self._k("finished", r)) and r not in lost}
            if pending:
                time.sleep(0.02)
        return not pending

    def result(self, seq: int) -> Optional[bytes]:
        key = self._k("result", seq)
        return self.store.get(key) if self._has(key) else None


def run_rank(ledger: ShardLedger, decode: Callable[[int], bytes], poll: float = 0.05,
             settle: Optional[Callable[[], bool]] = None) -> Dict[int, bytes]:
    """This rank's part of a data-parallel run: decode its shard (recording each sequence), then,
    until every sequence of the run is done, claim and decode the unfinished sequences of lost
    ranks.  Returns the sequences this rank decoded.  `settle` (optional) tells the loop to stop
    waiting early (e.g. a deadline)."""
    mine: Dict[int, bytes] = {}
    for s in ledger.my_shard():
        if ledger.is_done(s):
            continue
        mine[s] = decode(s)
        ledger.mark_done(s, mine[s])
    while not ledger.all_done():
        ledger.heartbeat()
        lost = ledger.lost_ranks()
        for s in ledger.orphans(lost):
            if ledger.claim(s, lost):
                mine[s] = decode(s)
                ledger.mark_done(s, mine[s])
        if settle is not None and settle():
            break
        time.sleep(poll)
    ledger.mark_finished()
    return mine
