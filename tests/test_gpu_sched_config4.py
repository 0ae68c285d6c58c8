"""The device scheduler at the shape bench.py measures, against the oracle.

256 slots admit sequences of bench.workload (prompts of 32-1024 random ids, 16-128 greedy tokens,
seed 4) into a context sized as the benchmark's, and run 600 device-scheduled steps: two
micro-batches on two stream pairs, the first step eager and every later one a CUDA-graph replay,
slots reused as sequences retire, and the 256-position KV window wrapping for every sequence longer
than 256 tokens.  The complete greedy id stream of finished sequences -- the shortest that wrapped
the window among the first admissions, and the shortest admitted into reused slots -- must equal
the oracle's one-sequence decode (NeedleModel.generate's greedy loop, packages/needle.js/src/model/
model.ts:88-153; window and slots as runtime.ts:659-786), and a running slot's int8 K/V codes and
scales, every layer, must equal the oracle runtime's after the same tokens.

The same run again with prompt chunks (needle_opts.sched_chunk = 16, 512 items per step; and the
bench's shape: 8 positions, 384 items, eight micro-batches): slots still reading their prompts take
several positions per step as a chunk of items beside the other slots' single items, until their
window would wrap.  The reference reads a prompt one token at a
time (runtime.ts:227-243), so the streams and the K/V must not change.
"""
import concurrent.futures
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STEPS = 600
SLOTS = 256


@pytest.fixture(scope="module", params=[{}, {"sched_chunk": 16, "sched_items": 512},
                                        {"sched_chunk": 8, "sched_items": 384, "micro_batches": 8}],
                ids=["one-position", "prompt-chunks", "bench-shape"])
def run(oracle, request):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import bench
    from needle_b200 import synth
    from needle_b200.backend import CudaEngine
    import needle_b200.build
    needle_b200.build.build()
    archive = synth.build_archive(0)
    prompts, gens = bench.workload(0, SLOTS * 12)
    with CudaEngine(archive, device=0, max_seqs=SLOTS, max_len=bench.PROMPT[1] + bench.GEN[1], max_sink=0,
                    **request.param) as eng:
        eng.sched_load(SLOTS, prompts, gens)
        eng.sched_step(1)       # eager
        eng.sched_step(STEPS - 1)  # captured once, then replayed
        tokens, generated, finished, last = eng.sched_status()
        ids = eng.sched_ids()
        slots = [eng.sched_slot(s) for s in range(SLOTS)]
        # a running slot past the window wrap, not too long for the oracle
        running = sorted((pos, s, sid) for s, (sid, pos, busy) in enumerate(slots) if busy and 300 <= pos <= 420)
        assert running, "no running slot past the window wrap"
        pos, slot, sid = running[0]
        kv = [eng.read_kv(slot, layer) for layer in range(eng.layers)]
        guards = eng.damaged_guards()
    offs = np.concatenate([[0], np.cumsum(gens)]).astype(np.int64)
    yield dict(prompts=prompts, gens=gens, tokens=tokens, generated=generated, finished=finished, last=last,
               ids=ids, offs=offs, kv_slot=(slot, sid, pos, kv), model=oracle.Model(archive),
               chunks=bool(request.param), guards=guards)


def _stream(r, i):
    return r["ids"][r["offs"][i]:r["offs"][i + 1]]


def test_counters_and_finished_streams_are_complete(run):
    """Every sequence that retired generated exactly its gen_steps ids, and the step count matches
    what the queue implies."""
    prompts, gens = run["prompts"], run["gens"]
    done = [i for i in range(len(prompts)) if run["last"][i] >= 0]
    assert len(done) == run["finished"] > 100
    for i in done:
        s = _stream(run, i)
        assert np.all(s >= 0) and s[-1] == run["last"][i]
    assert run["generated"] == int(np.sum(run["ids"] >= 0))
    assert any(i >= SLOTS for i in done), "no sequence finished in a reused slot"
    if run["chunks"]:  # prompt chunks: more than one position per slot and step while prompts last
        assert run["tokens"] > STEPS * SLOTS
    else:
        assert run["tokens"] == STEPS * SLOTS  # every slot stays busy: the queue is far from empty


def test_finished_id_streams_match_oracle(run):
    prompts, gens = run["prompts"], run["gens"]
    done = [i for i in range(len(prompts)) if run["last"][i] >= 0]
    total = lambda i: len(prompts[i]) + int(gens[i])
    first = sorted((i for i in done if i < SLOTS and total(i) > 300), key=total)[:10]
    reused = sorted((i for i in done if i >= SLOTS), key=total)[:8]
    reused_wrap = sorted((i for i in done if i >= SLOTS and total(i) > 300 and i not in reused), key=total)[:3]
    chosen = first + reused + reused_wrap
    assert len(first) == 10 and len(reused) == 8 and reused_wrap, (first, reused, reused_wrap)
    model = run["model"]

    def oracle_ids(i):
        ids, _, _ = model.generate_greedy(prompts[i], int(gens[i]), sink=0, want_logits=False)
        return i, ids

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(chosen), os.cpu_count() or 4)) as ex:
        results = list(ex.map(oracle_ids, chosen))
    for i, want in results:
        np.testing.assert_array_equal(_stream(run, i), want, err_msg=f"sequence {i} (prompt {len(prompts[i])}, "
                                                                       f"{int(gens[i])} generated)")


def test_running_slot_kv_matches_oracle(run):
    """K/V codes and scales of a running, window-wrapped slot after `position` tokens: the prompt's,
    then its greedy ids so far."""
    slot, sid, pos, kv = run["kv_slot"]
    prompt, gen = run["prompts"][sid], int(run["gens"][sid])
    stream = _stream(run, sid)
    consumed = list(prompt[:pos]) + list(stream[:max(0, pos - len(prompt))])
    assert len(consumed) == pos and all(t >= 0 for t in consumed)
    from oracle import needle_ref
    ref = needle_ref.Runtime(run["model"])
    ref.reset(len(prompt) + gen, 0)
    for t in consumed:
        ref.step(int(t), want_logits=False)
    assert ref.position == pos
    for layer, (kc, vc, ks, vs) in enumerate(kv):
        rkc, rvc, rks, rvs = ref.read_kv(layer)
        np.testing.assert_array_equal(kc, rkc, err_msg=f"key codes, layer {layer}")
        np.testing.assert_array_equal(vc, rvc, err_msg=f"value codes, layer {layer}")
        np.testing.assert_array_equal(ks, rks, err_msg=f"key scales, layer {layer}")
        np.testing.assert_array_equal(vs, rvs, err_msg=f"value scales, layer {layer}")
    ref.close()


def test_no_kernel_wrote_past_a_buffer(run):
    """Every device buffer of the context is followed by guard bytes; after 600 scheduled steps at
    this shape none of them has changed."""
    assert run["guards"] == 0
