"""GPU parity of batched constrained tool-call decoding (BASELINE config 5's loop).

`ConstrainedDecoder` runs several sequences through the engine at once, each with its own
`ToolCallGrammar` and allowed-id masks; the oracle replays every sequence alone, token by token,
selecting like selectToken over the same allowed lists (packages/needle.js/src/model/runtime.ts:
880-899: the first id of the list wins a tie) with its own logits.  Token ids must agree exactly,
and every completed call must parse as calls of the schema's tools.
"""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(oracle):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import grammar, synth, toolcall
    archive = synth.build_archive(0)
    pieces, types, _ = synth.tokenizer_pieces(8192, 0)
    vocab = grammar.Vocabulary(pieces, types)
    tools = toolcall.synthetic_tools(5)
    return archive, vocab, tools, oracle.Model(archive)


def oracle_constrained(oracle, model, vocab, tools, prompt, maximum_new):
    from needle_b200 import grammar
    rt = oracle.Runtime(model)
    rt.reset(len(prompt) + maximum_new + 1, 0)
    logits = None
    for i, t in enumerate(prompt):
        logits = rt.step(int(t), want_logits=(i == len(prompt) - 1))
    g = grammar.ToolCallGrammar(tools, 4)
    ids, out = [], 0
    for _ in range(maximum_new):
        allowed = grammar.allowed(g, vocab, out)
        if allowed.size == 0:
            return ids, False, True
        tok = int(allowed[int(np.argmax(logits[allowed]))])
        ids.append(tok)
        assert g.feed(vocab.piece[tok])
        out += len(vocab.piece[tok])
        if g.complete:
            return ids, True, False
        logits = rt.step(tok, want_logits=True)
    return ids, False, False


def test_constrained_decoding_matches_oracle(setup, oracle):
    from needle_b200.backend import CudaEngine
    from needle_b200 import toolcall
    archive, vocab, tools, model = setup
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 8192, n).astype(np.int32) for n in (40, 33, 57, 21, 48)]
    maximum_new = 48
    with CudaEngine(archive, device=0, max_seqs=3, max_len=160, max_sink=16) as eng:
        dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=maximum_new, threads=4)
        results, stats = dec.run(prompts)  # 5 sequences through 3 slots: admission into freed slots
    assert stats.constrained_tokens == sum(len(r.ids) for r in results)
    names = {t["name"] for t in tools}
    for k, (p, res) in enumerate(zip(prompts, results)):
        ids, complete, dead = oracle_constrained(oracle, model, vocab, tools, p, maximum_new)
        assert res.ids == ids, k
        assert res.complete == complete and res.dead_end == dead, k
        assert res.text == b"".join(vocab.piece[i] for i in ids)
        if res.complete:
            calls = json.loads(res.text.decode())
            assert calls == res.calls and all(c["name"] in names for c in calls)


def test_device_masks_match_oracle(setup, oracle):
    """The same decode with allowed masks kept per grammar state in a device pool (the items name a
    pool slot; only new states' masks are copied): the same token ids as the oracle's id lists, with
    a table small enough to evict."""
    from needle_b200.backend import CudaEngine, StepRequest
    from needle_b200 import toolcall
    from needle_b200.native import NeedleError
    archive, vocab, tools, model = setup
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 8192, n).astype(np.int32) for n in (40, 33, 57, 21, 48)]
    maximum_new = 48
    with CudaEngine(archive, device=0, max_seqs=3, max_len=160, max_sink=16) as eng:
        dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=maximum_new, threads=4,
                                          mask_cache=12)
        results, stats = dec.run(prompts)
        assert stats.allowed_ids == 0 and stats.masked_items == stats.constrained_tokens
        assert 0 < stats.masks_put < stats.masked_items
        assert dec.cache.stats["evictions"] > 0
        # an item naming a slot that holds no mask is refused before anything runs
        eng.mask_pool(4)
        eng.reset(0, 16, 0)
        with pytest.raises(NeedleError) as e:
            eng.step([StepRequest(0, 5, True, mask_slot=2)])
        assert e.value.code == "INVALID_CACT"
        with pytest.raises(NeedleError):
            eng.step([StepRequest(0, 5, True, mask_slot=4)])
    for k, (p, res) in enumerate(zip(prompts, results)):
        ids, complete, dead = oracle_constrained(oracle, model, vocab, tools, p, maximum_new)
        assert res.ids == ids, k
        assert res.complete == complete and res.dead_end == dead, k


def test_many_slots_split_steps_match_one_batch(setup):
    """Config 5's loop with 80 slots: its split steps (64 items or more) run as micro-batches; the
    tokens are those of one batch."""
    from needle_b200.backend import CudaEngine
    from needle_b200 import toolcall
    archive, vocab, tools, model = setup
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 8192, int(n)).astype(np.int32) for n in rng.integers(3, 12, 80)]
    outs = []
    for micro in (1, 4):
        with CudaEngine(archive, device=0, max_seqs=80, max_len=64, max_sink=0, micro_batches=micro) as eng:
            dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=24, threads=4, mask_cache=256)
            results, stats = dec.run(prompts)
            outs.append([(r.ids, r.complete, r.dead_end) for r in results])
    assert outs[0] == outs[1]


def test_prompt_chunks_match_oracle(setup, oracle):
    """The same decode with prompts sent in chunks of up to 8 positions per step (at most 24 items
    per step): the oracle's ids, fed one token at a time."""
    from needle_b200.backend import CudaEngine
    from needle_b200 import toolcall
    archive, vocab, tools, model = setup
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 8192, n).astype(np.int32) for n in (40, 33, 57, 21, 48)]
    maximum_new = 48
    with CudaEngine(archive, device=0, max_seqs=3, max_len=160, max_sink=16) as eng:
        dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=maximum_new, threads=4,
                                          prompt_chunk=8, step_items=24)
        results, stats = dec.run(prompts)
    assert stats.prompt_tokens == sum(p.size for p in prompts)
    for k, (p, res) in enumerate(zip(prompts, results)):
        ids, complete, dead = oracle_constrained(oracle, model, vocab, tools, p, maximum_new)
        assert res.ids == ids, k
        assert res.complete == complete and res.dead_end == dead, k
