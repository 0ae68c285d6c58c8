"""The batched constrained decoder's host logic on the CPU (needle_b200.toolcall.ConstrainedDecoder).

A fake engine stands in for the GPU: its logits for a slot are a fixed pseudo-random function of
the tokens fed to that slot since its reset, so any scheduling of sequences over slots must give
each sequence the same tokens as running it alone.  The reference for one sequence is the loop of
packages/needle.js/src/tools/agent.ts:157-210 restated directly: scan the allowed ids, feed the
pending token and select among them (the first maximum wins, runtime.ts:880-899), feed the chosen
piece to the grammar, and after the grammar completes feed the chosen token once more.
"""
import json

import numpy as np
import pytest

from needle_b200.backend import StepRequest


def fake_logits(history, vocab):
    rng = np.random.default_rng(hash(tuple(history)) % (1 << 32))
    return rng.standard_normal(vocab)


def select(logits, allowed):
    return int(allowed[int(np.argmax(logits[allowed]))])


class FakeEngine:
    """The engine contract the decoder relies on: reset, step_begin / step_end with the same
    items, distinct slots per step, selections only for items that select."""

    def __init__(self, max_seqs, vocab):
        self.max_seqs, self.vocab = max_seqs, vocab
        self.kv_window = 256
        self.hist = [None] * max_seqs
        self.pending = None
        self.steps = 0
        self.pool = None

    def mask_pool(self, capacity):
        self.pool = np.zeros((capacity, (self.vocab + 31) // 32), dtype=np.uint32)

    def masks_put(self, slots, table):  # between step_begin and step_end, as the decoder calls it
        for s in np.asarray(slots).tolist():
            self.pool[s] = table[s]

    def _allowed(self, r):
        if r.mask_slot is None:
            return r.allowed
        bits = np.unpackbits(self.pool[r.mask_slot].view(np.uint8), bitorder="little")[:self.vocab]
        return np.flatnonzero(bits)

    def reset(self, slot, maximum_length, sink_length=0):
        assert 0 <= slot < self.max_seqs and self.pending is None
        self.hist[slot] = []

    def step_begin(self, requests):
        assert self.pending is None and requests
        slots = [r.seq for r in requests]
        # a slot appears once, or as consecutive items that do not select (a prompt chunk)
        runs = [s for i, s in enumerate(slots) if i == 0 or slots[i - 1] != s]
        assert len(set(runs)) == len(runs)
        for i in range(1, len(requests)):
            if slots[i] == slots[i - 1]:
                assert not requests[i].select and not requests[i - 1].select and requests[i].token >= 0
        self.pending = [(r.seq, r.token, r.select) for r in requests]

    def step_end(self, requests):
        assert [(r.seq, r.token) for r in requests] == [(s, t) for s, t, _ in self.pending]
        out = []
        for r, (_, _, began_select) in zip(requests, self.pending):
            assert began_select or not r.select  # a select may be cleared, not set
            self.hist[r.seq].append(r.token)
            if r.select:
                allowed = self._allowed(r)
                assert allowed is not None and allowed.size > 0
                out.append((select(fake_logits(self.hist[r.seq], self.vocab), allowed), 0.0))
            else:
                out.append(None)
        self.pending = None
        self.steps += 1
        return out


def reference(prompt, vocab, pieces, tools, maximum_new, grammar):
    """One sequence alone: (ids, complete, dead_end, tokens fed)."""
    g = grammar.ToolCallGrammar(tools, 4)
    fed = [int(t) for t in prompt[:-1]]
    pending, ids, out = int(prompt[-1]), [], 0
    for _ in range(maximum_new):
        allowed = grammar.allowed(g, vocab, out)
        if allowed.size == 0:
            return ids, False, True, fed
        fed.append(pending)
        tok = select(fake_logits(fed, vocab.size), allowed)
        ids.append(tok)
        assert g.feed(pieces[tok])
        out += len(pieces[tok])
        if g.complete:
            fed.append(tok)
            return ids, True, False, fed
        pending = tok
    return ids, False, False, fed


@pytest.fixture(scope="module")
def env():
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import grammar, synth, toolcall
    pieces, types, _ = synth.tokenizer_pieces(8192, 0)
    vocab = grammar.Vocabulary(pieces, types)
    return grammar, toolcall, vocab


def test_batched_decoder_matches_one_sequence_at_a_time(env):
    grammar, toolcall, vocab = env
    tools = toolcall.synthetic_tools(5)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, vocab.size, int(rng.integers(2, 7))).astype(np.int32) for _ in range(7)]
    maximum_new = 200
    eng = FakeEngine(3, vocab.size)
    dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=maximum_new, threads=3)
    results, stats = dec.run(prompts)  # 7 sequences through 3 slots
    assert stats.constrained_tokens == sum(len(r.ids) for r in results)
    assert stats.prompt_tokens == sum(p.size for p in prompts)
    assert stats.steps == eng.steps
    for p, r in zip(prompts, results):
        ids, complete, dead, _ = reference(p, vocab, vocab.piece, tools, maximum_new, grammar)
        assert r.ids == ids and r.complete == complete and r.dead_end == dead
        assert r.text == b"".join(vocab.piece[i] for i in ids)
        if complete:
            assert json.loads(r.text.decode()) == r.calls
            assert {c["name"] for c in r.calls} <= {t["name"] for t in tools}
    assert any(r.complete for r in results)


@pytest.mark.parametrize("capacity", [6, 512])
def test_mask_cache_decodes_the_same_tokens(env, capacity):
    """Masks per grammar state in a device pool (a table far smaller than the states visited, and
    one that holds them all) select exactly the tokens of per-step id lists."""
    grammar, toolcall, vocab = env
    tools = toolcall.synthetic_tools(5)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, vocab.size, int(rng.integers(2, 5))).astype(np.int32) for _ in range(9)]
    plain, _ = toolcall.ConstrainedDecoder(FakeEngine(4, vocab.size), vocab, tools, maximum_new_tokens=120,
                                           threads=3).run(prompts)
    eng = FakeEngine(4, vocab.size)
    dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=120, threads=3, mask_cache=capacity)
    cached, stats = dec.run(prompts)
    for a, b in zip(plain, cached):
        assert a.ids == b.ids and a.complete == b.complete and a.dead_end == b.dead_end and a.calls == b.calls
    assert stats.allowed_ids == 0 and stats.masked_items == stats.constrained_tokens
    assert 0 < stats.masks_put < stats.masked_items  # states repeat across sequences and steps
    if capacity == 6:
        assert dec.cache.stats["evictions"] > 0
    with pytest.raises(ValueError):
        toolcall.ConstrainedDecoder(FakeEngine(4, vocab.size), vocab, tools, mask_cache=3)


def test_prompt_chunks_decode_the_same_tokens(env):
    """Prompts sent in chunks of up to 8 positions per step (at most 16 items per step over 6
    slots) feed every slot the same tokens as one position per step, so the calls are the same."""
    grammar, toolcall, vocab = env
    tools = toolcall.synthetic_tools(5)
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, vocab.size, int(rng.integers(2, 40))).astype(np.int32) for _ in range(9)]
    plain, st0 = toolcall.ConstrainedDecoder(FakeEngine(6, vocab.size), vocab, tools,
                                             maximum_new_tokens=60).run(prompts)
    eng = FakeEngine(6, vocab.size)
    chunked, st1 = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=60, prompt_chunk=8,
                                               step_items=16).run(prompts)
    for a, b in zip(plain, chunked):
        assert a.ids == b.ids and a.complete == b.complete and a.calls == b.calls
    assert st1.prompt_tokens == st0.prompt_tokens and st1.steps < st0.steps


def test_slots_are_reused_and_histories_match(env):
    """After a sequence ends its slot is reset for the next one; what each sequence fed is exactly
    the reference loop's (prompt, pending tokens, the final token of a completed call)."""
    grammar, toolcall, vocab = env
    tools = toolcall.synthetic_tools(5)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, vocab.size, 3).astype(np.int32) for _ in range(4)]

    class Recording(FakeEngine):
        def __init__(self, *a):
            super().__init__(*a)
            self.finished = []

        def reset(self, slot, maximum_length, sink_length=0):
            if self.hist[slot] is not None:
                self.finished.append(list(self.hist[slot]))
            super().reset(slot, maximum_length, sink_length)

    eng = Recording(1, vocab.size)  # one slot: strictly one sequence after another
    results, _ = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=30).run(prompts)
    eng.finished.append(list(eng.hist[0]))
    for p, r, fed in zip(prompts, results, eng.finished):
        ids, complete, dead, want = reference(p, vocab, vocab.piece, tools, 30, grammar)
        assert r.ids == ids
        assert fed == want


def test_dead_end_and_maximum_new_tokens(env):
    grammar, toolcall, _ = env
    tools = toolcall.synthetic_tools(5)
    # a vocabulary that can open the call but never write `"name"`: a dead end after "[{"
    pieces = ["<unk>", "[", "{", "a"]
    small = grammar.Vocabulary(pieces, [grammar.UNKNOWN, grammar.NORMAL, grammar.NORMAL, grammar.NORMAL])
    eng = FakeEngine(2, small.size)
    results, _ = toolcall.ConstrainedDecoder(eng, small, tools, maximum_new_tokens=10).run(
        [np.array([3, 1], dtype=np.int32), np.array([2], dtype=np.int32)])
    for r in results:
        assert r.dead_end and not r.complete and r.text == b"[{"
    # a budget too small to finish: stops after exactly maximum_new constrained tokens
    _, toolcall_mod, vocab = env
    eng = FakeEngine(2, vocab.size)
    results, _ = toolcall_mod.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=3).run(
        [np.array([5, 6, 7], dtype=np.int32)])
    assert len(results[0].ids) == 3 and not results[0].complete and not results[0].dead_end
    assert results[0].text.startswith(b"[")


def test_step_items_pack_as_the_c_struct():
    """CudaEngine._items lays requests out as needle_step_item (include/needle_cuda.h) and
    concatenates the masks of the selecting items in order."""
    import ctypes
    from needle_b200 import native
    from needle_b200.backend import CudaEngine
    reqs = [StepRequest(3, 7, True, np.array([1, 5, 9], dtype=np.uint32)), StepRequest(1, -1, False),
            StepRequest(0, 2, True), StepRequest(2, 4, True, np.array([8], dtype=np.uint32)),
            StepRequest(4, 6, False, np.array([3], dtype=np.uint32)),  # a mask without select is ignored
            StepRequest(5, 1, True, mask_slot=17), StepRequest(6, 2, False, mask_slot=4)]
    items, allowed = CudaEngine._items(reqs)
    assert items.dtype == np.int32 and items.shape[1] * 4 == ctypes.sizeof(native.StepItem)
    arr = (native.StepItem * len(reqs)).from_buffer_copy(items.tobytes())
    got = [(a.seq, a.token, a.select, a.allowed_count) for a in arr]
    assert got == [(3, 7, 1, 3), (1, -1, 0, -1), (0, 2, 1, -1), (2, 4, 1, 1), (4, 6, 0, -1),
                   (5, 1, 1, native.ALLOWED_MASK), (6, 2, 0, -1)]
    assert arr[0].allowed_offset == 0 and arr[3].allowed_offset == 3 and arr[5].allowed_offset == 17
    np.testing.assert_array_equal(allowed, [1, 5, 9, 8])
    items, allowed = CudaEngine._items([StepRequest(0, 1, False)])
    assert allowed is None and items[0].tolist() == [0, 1, 0, -1, 0]
