"""Prompt chunks in host-driven steps (needle_cuda_step with consecutive items of one slot).

A slot still reading its prompt may send several of its next prompt positions in one step, as
consecutive items that carry their tokens and do not select; the slot advances past all of them.
The reference reads a prompt one token per step (packages/needle.js/src/model/runtime.ts:227-243),
so the same sequences driven with chunks and one position at a time must select the same ids and
leave the same int8 K/V, bit for bit.  Chunks that select, that are not consecutive, or that
would reach past the KV window are refused before anything runs.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def archive():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import synth
    return synth.build_archive(0)


def _drive(eng, prompts, gens, chunk):
    """Every slot s decodes prompts[s] then gens[s] greedy ids; returns the ids per slot."""
    from needle_b200.backend import StepRequest
    n = len(prompts)
    for s in range(n):
        eng.reset(s, len(prompts[s]) + gens[s] + 1, 0)
    pos = [0] * n
    ids = [[] for _ in range(n)]
    while any(len(ids[s]) < gens[s] for s in range(n)):
        reqs = []
        for s in range(n):
            if len(ids[s]) >= gens[s]:
                continue
            p = prompts[s]
            if pos[s] < len(p) - 1:
                k = min(chunk, len(p) - 1 - pos[s]) if chunk > 1 else 1
                reqs.extend(StepRequest(s, int(p[pos[s] + j]), False) for j in range(k))
            elif pos[s] == len(p) - 1:
                reqs.append(StepRequest(s, int(p[-1]), True))
            else:
                reqs.append(StepRequest(s, -1, True))
        out, _ = eng.step(reqs)
        for r, o in zip(reqs, out):
            pos[r.seq] += 1
            if r.select:
                ids[r.seq].append(int(o[0]))
    return ids, pos


def test_host_chunks_match_one_position_steps(archive):
    from needle_b200.backend import CudaEngine
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 8192, n).astype(np.int32) for n in (41, 10, 29, 3)]
    gens = [6, 9, 4, 7]
    results = []
    for chunk in (1, 8):
        with CudaEngine(archive, device=0, max_seqs=4, max_len=96, max_sink=0) as eng:
            ids, pos = _drive(eng, prompts, gens, chunk)
            kv = [[eng.read_kv(s, layer) for layer in (0, 13, eng.layers - 1)] for s in range(4)]
            results.append((ids, pos, kv))
    (ids_a, pos_a, kv_a), (ids_b, pos_b, kv_b) = results
    assert ids_a == ids_b and pos_a == pos_b
    for s in range(4):
        for a, b in zip(kv_a[s], kv_b[s]):
            for x, y in zip(a, b):
                np.testing.assert_array_equal(x, y, err_msg=f"slot {s}")


def test_host_chunks_refused(archive):
    from needle_b200.backend import CudaEngine, StepRequest
    from needle_b200.native import NeedleError
    with CudaEngine(archive, device=0, max_seqs=2, max_len=300, max_sink=0) as eng:
        eng.reset(0, 300, 0)
        eng.reset(1, 300, 0)
        with pytest.raises(NeedleError) as e:  # a chunk item that selects
            eng.step([StepRequest(0, 5, False), StepRequest(0, 6, True)])
        assert e.value.code == "INVALID_CACT"
        with pytest.raises(NeedleError):  # a slot twice, not consecutively
            eng.step([StepRequest(0, 5, False), StepRequest(1, 6, False), StepRequest(0, 7, False)])
        with pytest.raises(NeedleError):  # a chunk item without its token
            eng.step([StepRequest(0, 5, False), StepRequest(0, -1, False)])
        assert eng.position(0) == 0 and eng.position(1) == 0  # nothing ran
        eng.prefill(0, np.arange(250, dtype=np.int32) % 8192, want_logits=False)
        with pytest.raises(NeedleError) as e:  # positions 250..257 would wrap the 256-position window
            eng.step([StepRequest(0, 9, False) for _ in range(8)])
        assert e.value.code == "INVALID_CACT"
        eng.step([StepRequest(0, 9, False) for _ in range(6)])  # up to the window is fine
        assert eng.position(0) == 256


def test_many_items_run_as_micro_batches(archive):
    """A host step of 64 items or more runs as micro-batches (replayed as a CUDA graph from its
    second step on), through needle_cuda_step and through needle_cuda_step_begin / _end: the same
    ids and K/V as one batch, with chunks, decode slots and slots that finish and are reset in
    between."""
    from needle_b200.backend import CudaEngine, StepRequest
    rng = np.random.default_rng(12)
    n_slots = 96
    prompts = [rng.integers(0, 8192, int(n)).astype(np.int32) for n in rng.integers(2, 40, n_slots)]
    gens = [int(g) for g in rng.integers(1, 6, n_slots)]
    runs = []
    for micro, split in ((1, False), (4, False), (4, True)):
        with CudaEngine(archive, device=0, max_seqs=n_slots, max_len=64, max_sink=0, micro_batches=micro,
                        sched_chunk=8, sched_items=160) as eng:
            for s in range(n_slots):
                eng.reset(s, len(prompts[s]) + gens[s] + 1, 0)
            pos, got, trace = [0] * n_slots, [[] for _ in range(n_slots)], []
            l0 = eng.kernel_launches()
            for step in range(24):
                reqs, budget = [], 160 - n_slots
                for s in range(n_slots):
                    p = prompts[s]
                    if len(got[s]) >= gens[s]:  # finished: start over with the same prompt
                        eng.reset(s, len(p) + gens[s] + 1, 0)
                        pos[s], got[s] = 0, []
                    if pos[s] < len(p) - 1:
                        k = 1 + max(0, min(min(8, len(p) - 1 - pos[s]) - 1, budget))
                        budget -= k - 1
                        reqs.extend(StepRequest(s, int(p[pos[s] + j]), False) for j in range(k))
                    else:
                        reqs.append(StepRequest(s, int(p[-1]) if pos[s] == len(p) - 1 else -1, True))
                assert len(reqs) >= 64
                if split:
                    eng.step_begin(reqs)
                    out = eng.step_end(reqs)
                else:
                    out, _ = eng.step(reqs)
                sel = []
                for r, o in zip(reqs, out):
                    pos[r.seq] += 1
                    if r.select:
                        got[r.seq].append(int(o[0]))
                        sel.append((r.seq, int(o[0]), o[1]))
                trace.append(sel)
            kv = [eng.read_kv(s, 0) for s in (0, 17, 95)]
            assert eng.damaged_guards() == 0
            runs.append((trace, pos, kv, eng.kernel_launches() - l0))
    (ta, pa, ka, la) = runs[0]
    for tb, pb, kb, lb in runs[1:]:
        assert lb > 3 * la  # four micro-batches: the kernels of each launched per micro-batch
        assert pa == pb
        for step, (a, b) in enumerate(zip(ta, tb)):
            assert a == b, f"step {step}"
        for a, b in zip(ka, kb):
            for x, y in zip(a, b):
                np.testing.assert_array_equal(x, y)


def test_nvtx_ranges_do_not_change_a_step(archive, monkeypatch):
    """With NEEDLE_NVTX set when the context opens, steps run inside NVTX ranges: same selections."""
    from needle_b200.backend import CudaEngine, StepRequest
    outs = []
    for nvtx in ("0", "1"):
        monkeypatch.setenv("NEEDLE_NVTX", nvtx)
        with CudaEngine(archive, device=0, max_seqs=2, max_len=32, max_sink=0) as eng:
            eng.reset(0, 32, 0)
            eng.reset(1, 32, 0)
            got = []
            for t in range(6):
                out, _ = eng.step([StepRequest(0, 3 + t, t == 5), StepRequest(1, 7 + t, t == 5)])
                got.append(out)
            outs.append(got)
    assert outs[0] == outs[1]


def test_one_item_steps_replay_a_graph(archive):
    """One-item host steps (the batch-1 decode loop) run as a graph replay from their second on:
    the same selections, log-probabilities and K/V as eager steps (steps that return logits run
    eagerly), across a reset and a different slot."""
    from needle_b200.backend import CudaEngine, StepRequest
    rng = np.random.default_rng(14)
    prompt = rng.integers(0, 8192, 9).astype(np.int32)
    runs = []
    for want_logits in (True, False):
        with CudaEngine(archive, device=0, max_seqs=2, max_len=64, max_sink=0) as eng:
            got = []
            for slot in (0, 1, 0):
                eng.reset(slot, 40, 0)
                eng.prefill(slot, prompt[:-1], want_logits=False)
                for k in range(12):
                    out, _ = eng.step([StepRequest(slot, int(prompt[-1]) if k == 0 else -1, True)],
                                      want_logits=want_logits)
                    got.append(out[0])
            kv = [eng.read_kv(s, layer) for s in (0, 1) for layer in (0, eng.layers - 1)]
            assert eng.damaged_guards() == 0
            runs.append((got, kv))
    (ga, ka), (gb, kb) = runs
    assert ga == gb
    for a, b in zip(ka, kb):
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)
