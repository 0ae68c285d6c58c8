"""Batched constrained tool-call decoding over the engine's slots.

The constrained loop of `Needle.complete` (packages/needle.js/src/tools/agent.ts:157-210), run for
many sequences at once: each step, every sequence in its constrained phase asks its
`ToolCallGrammar` for the ids that may come next (the host-side scan, here a byte-trie walk on host
threads, include/needle_grammar.h), the engine feeds the pending token and picks the best allowed
id on the device (an allowed list per item: the fused mask + argmax, ties to the first id of the
list as selectToken does), and the chosen piece is fed to the grammar.  The scan runs while the
step's layers run on the GPU (needle_cuda_step_begin / needle_cuda_step_end): the allowed ids only
depend on tokens already chosen.  When the
grammar completes, the chosen token is fed once more without a selection (agent.ts:193-196) and the
slot is freed for the next sequence.

With a mask cache (`mask_cache` slots), the scan runs once per grammar state instead of once per
sequence and step (needle_mask_cache_lookup, include/needle_grammar.h): sequences in the same state
(the free content of a string, the same separator or key) share one mask, and a state seen before is
not scanned again.  The masks live in a pool on the device (needle_cuda_mask_pool); only the masks of
new states cross PCIe (needle_cuda_masks_put, one per state) and the items name their slot, so the
selections are the same as with id lists (the best logit, ties to the lowest id).  Prompts are fed one token per step through the same batched
steps; the constrained phase starts directly after the prompt, its pending token being the prompt's
last token (random weights never emit <tool_call>).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import numpy as np

from .backend import StepRequest
from .grammar import MAX_OUTPUT_BYTES, MaskCache, ToolCallGrammar, Vocabulary, allowed_batch


def synthetic_tools(seed: int = 5, n_tools: int = 3):
    """BASELINE config 5's schema: 3 tools with 2-5 parameters each, names of 4-12 random lowercase
    letters, parameter types drawn from string / integer / boolean / enum (2-4 random words); every
    parameter required."""
    rng = np.random.default_rng(seed)

    def word():
        return "".join(chr(97 + int(c)) for c in rng.integers(0, 26, int(rng.integers(4, 13))))

    tools, names = [], set()
    while len(tools) < n_tools:
        name = word()
        if name in names:
            continue
        names.add(name)
        props = {}
        for _ in range(int(rng.integers(2, 6))):
            kind = ("string", "integer", "boolean", "enum")[int(rng.integers(0, 4))]
            key = word()
            while key in props:
                key = word()
            if kind == "enum":
                props[key] = {"type": "string", "enum": [word() for _ in range(int(rng.integers(2, 5)))]}
            else:
                props[key] = {"type": kind}
        tools.append({"name": name, "description": "synthetic tool",
                      "parameters": {"type": "object", "properties": props, "required": list(props)}})
    return tools


@dataclass
class ToolCallResult:
    ids: List[int] = field(default_factory=list)      # constrained tokens, in order
    text: bytes = b""
    calls: list = field(default_factory=list)
    complete: bool = False
    dead_end: bool = False


@dataclass
class DecodeStats:
    steps: int = 0
    prompt_tokens: int = 0
    constrained_tokens: int = 0
    seconds: float = 0.0
    grammar_seconds: float = 0.0
    engine_seconds: float = 0.0
    items: int = 0        # step items sent to the engine
    allowed_ids: int = 0  # allowed ids sent with them as id lists
    masked_items: int = 0  # selections over a device mask (mask cache)
    masks_put: int = 0     # masks copied to the device (new grammar states)


class ConstrainedDecoder:
    def __init__(self, engine, vocab: Vocabulary, tools: Sequence[dict], maximum_calls: int = 4,
                 maximum_new_tokens: int = 256, threads: int = 8, mask_cache: int = 0, prompt_chunk: int = 0,
                 step_items: int = 0):
        """`mask_cache` > 0: keep allowed masks per grammar state in a cache of that many slots and
        a device pool of the same size (at least the engine's slot count); 0: id lists per step.
        `prompt_chunk` >= 2: a slot still reading its prompt sends up to that many prompt positions
        per step as a chunk of items (never the last, which selects), at most `step_items` items per
        step (0: the engine's slot count), in slot order; the tokens are the same."""
        self.engine = engine
        self.vocab = vocab
        self.tools = list(tools)
        self.maximum_calls = maximum_calls
        self.maximum_new = max(1, maximum_new_tokens)
        self.threads = threads
        self.template = ToolCallGrammar(self.tools, maximum_calls)  # validates the tools once
        self.prompt_chunk = prompt_chunk
        self.step_items = step_items or engine.max_seqs
        self.window = getattr(engine, "kv_window", 0)  # slots are reset with sink 0
        self.cache = None
        if mask_cache:
            if mask_cache < engine.max_seqs:
                raise ValueError("mask_cache needs at least one slot per engine slot")
            self.cache = MaskCache(self.template, vocab, mask_cache)
            engine.mask_pool(mask_cache)

    def run(self, prompts: Sequence[np.ndarray], slots: Optional[int] = None, max_steps: Optional[int] = None,
            hook: Optional[Callable[[int], None]] = None) -> tuple[List[ToolCallResult], DecodeStats]:
        """Decodes every prompt's tool call through at most `slots` engine slots; `hook(step)` is
        called before each step (e.g. to switch the engine's kernel profiling on).

        A step's items need only tokens: the token chosen at the previous step is fed whether or not
        it completed the grammar (agent.ts:193-196 feeds it once more when it did), and only the
        select flag depends on the grammar, which needle_cuda_step_end may clear.  So each step is
        begun first, and the previous step's chosen pieces are fed to the grammars, completions
        detected and the next allowed ids scanned while its layers run."""
        eng = self.engine
        slots = min(slots or eng.max_seqs, eng.max_seqs)
        results = [ToolCallResult() for _ in prompts]
        stats = DecodeStats()
        queue = list(range(len(prompts)))[::-1]
        # per slot: seq, phase ("prompt" | "call" | "final"), prompt, pos, grammar, out (bytes
        # chosen so far), pending (the token the next step feeds), unfed (chosen but not yet fed
        # to the grammar)
        state = [None] * slots
        t_start = time.perf_counter()

        def feed(st, tok):
            t0 = time.perf_counter()
            accepted = st["grammar"].feed(self.vocab.piece[tok])
            complete = accepted and st["grammar"].complete
            stats.grammar_seconds += time.perf_counter() - t0
            if not accepted:  # the device picked outside the mask: a contract violation
                raise RuntimeError(f"selected disallowed token {tok}")
            res = results[st["seq"]]
            if complete:
                res.complete = True
                res.calls = st["grammar"].calls
                st["phase"] = "final"
            st["unfed"] = None
            return complete

        while True:
            for s in range(slots):  # admit
                if state[s] is None and queue:
                    k = queue.pop()
                    p = np.asarray(prompts[k], dtype=np.int32)
                    eng.reset(s, int(p.size) + self.maximum_new + 1, 0)
                    state[s] = {"seq": k, "pos": 0, "phase": "prompt", "prompt": p,
                                "grammar": self.template.clone(), "out": 0, "pending": -1, "unfed": None}
            live = [s for s in range(slots) if state[s] is not None]
            if not live or (max_steps is not None and stats.steps >= max_steps):
                break
            if hook is not None:
                hook(stats.steps)
            requests = []
            budget = self.step_items - len(live)
            for s in live:
                st = state[s]
                if st["phase"] == "prompt":
                    p, pos = st["prompt"], st["pos"]
                    last = pos == p.size - 1
                    k = 1
                    if self.prompt_chunk >= 2 and not last:  # a chunk: never past the KV window
                        want = min(self.prompt_chunk, p.size - 1 - pos)
                        if self.window > 0:
                            want = min(want, self.window - pos)
                        want = max(1, want)
                        k = 1 + max(0, min(want - 1, budget))
                        budget -= k - 1
                    requests.extend(StepRequest(s, int(p[pos + j]), last) for j in range(k))
                    stats.prompt_tokens += k
                else:  # "call": the pending token, selecting unless its feed completes the call
                    requests.append(StepRequest(s, st["pending"], st["phase"] == "call"))
            t0 = time.perf_counter()
            eng.step_begin(requests)
            t1 = time.perf_counter()
            # while the layers run: the previous choices go to the grammars, then the scans
            for r in requests:
                st = state[r.seq]
                if st["unfed"] is not None and feed(st, st["unfed"]):
                    r.select = False  # completed: this step is the final feed (no selection)
            selecting = [i for i, r in enumerate(requests) if r.select]
            t2 = time.perf_counter()
            grammars = [state[requests[i].seq]["grammar"] for i in selecting]
            outs = [state[requests[i].seq]["out"] for i in selecting]
            if self.cache is not None:
                mslots, counts, filled = self.cache.lookup(grammars, outs, self.threads)
                t3 = time.perf_counter()
                eng.masks_put(filled, self.cache.table)
                stats.masks_put += int(filled.size)
                sizes = counts.tolist()
                for i, slot in zip(selecting, mslots.tolist()):
                    requests[i].mask_slot = slot
            else:
                masks = allowed_batch(grammars, outs, self.vocab, self.threads)
                t3 = time.perf_counter()
                sizes = [int(m.size) for m in masks]
                for i, ids in zip(selecting, masks):
                    requests[i].allowed = ids
            stats.grammar_seconds += t3 - t2
            for i, size in zip(selecting, sizes):
                if size == 0:  # GRAMMAR_DEAD_END: no token can continue; the sequence stops here
                    requests[i].select = False
                    requests[i].allowed = None
                    requests[i].mask_slot = None
                    results[state[requests[i].seq]["seq"]].dead_end = True
                    state[requests[i].seq]["phase"] = "dead"
            stats.items += len(requests)
            stats.allowed_ids += sum(int(r.allowed.size) for r in requests if r.allowed is not None)
            stats.masked_items += sum(1 for r in requests if r.select and r.mask_slot is not None)
            chosen = eng.step_end(requests)
            stats.engine_seconds += (t1 - t0) + (time.perf_counter() - t3)
            stats.steps += 1
            for r, sel in zip(requests, chosen):
                st = state[r.seq]
                if st["phase"] in ("final", "dead"):
                    state[r.seq] = None
                    continue
                if st["phase"] == "prompt" and not r.select:
                    st["pos"] += 1
                    continue
                tok = int(sel[0])
                res = results[st["seq"]]
                res.ids.append(tok)
                res.text += self.vocab.piece[tok]
                st["out"] += len(self.vocab.piece[tok])
                st["pending"] = st["unfed"] = tok
                st["phase"] = "call"
                stats.constrained_tokens += 1
                if len(res.ids) >= self.maximum_new or st["out"] >= MAX_OUTPUT_BYTES:
                    # the budget is spent: unless this token completes the call (then the next step
                    # feeds it once more), the sequence ends here
                    if not feed(st, tok):
                        res.calls = st["grammar"].calls
                        state[r.seq] = None
        stats.seconds = time.perf_counter() - t_start
        return results, stats
