"""The engine in fast numerics (NEEDLE_NUMERICS_FAST) against the oracle, within tolerance.

Fast numerics computes every projection of a step -- Q|K|V|gate, the output projection, the engram
key|value projections and the tied vocabulary head -- as a tcgen05 tensor-core GEMM over the step's
items (fp16 head/tail split operands, fp32 accumulation: about 1e-6 relative per projection), and
prompt chunks go through the same GEMMs (batched prefill), and attention runs in binary32 over the
int8 cache (online softmax on the CUDA cores).  The K/V append, routing and selection stay as in
exact numerics.  Bar (north star): the same greedy token ids as the CPU reference and
logits within 1e-3 max-abs-relative (max |a - b| / max(|b|, 1) per logits vector).  The margin is
thin by construction: the int8 KV cache turns last-bit differences of K and V into whole-code
differences for 1-2 % of the codes of deep layers, and the 27 layers of the random-init model
amplify the projections' error about a thousandfold (with bf16 head/tail operands the logits were
3e-3 off; fp16 ones with all four head/tail products give 9.8e-4).  The GEMM's summation order is
fixed, so the result is the same on every run.  A scheduled run's ids may differ from the
reference only at a step whose top-two logits are within the tolerance of each other (a near tie
that binary32 arithmetic may break either way).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def max_abs_rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b) / np.maximum(np.abs(b.astype(np.float64)), 1.0)))


@pytest.fixture(scope="module")
def archive():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import synth
    return synth.build_archive(0)


@pytest.fixture(scope="module")
def ref_model(oracle, archive):
    return oracle.Model(archive)


# NEEDLE_NUMERICS_FAST_ATTENTION also runs attention on the int8-MMA kernel (binary32 online
# softmax, query and weights as 21-bit integer digits): its outputs differ from the binary64 chain by
# about 1e-6 relative, which the int8 cache and the layers amplify to about 2.4e-3 in the logits;
# its stated bar is 3e-3, with the same greedy ids.
MODES = [("fast", LOGIT_TOL, 0.98), ("fast_attention", 3e-3, 0.95)]


@pytest.mark.parametrize("numerics,tol,kv_equal", MODES)
def test_config1_fast_logits_and_greedy_ids(archive, oracle, ref_model, numerics, tol, kv_equal):
    """128-token prompt (seed 1) prefilled in chunks, 64 greedy steps; the
    oracle's tokens are fed back (teacher forcing) so every step's logits are compared at the same
    state, and the greedy ids of a free run must equal the oracle's."""
    from needle_b200 import synth
    from needle_b200.backend import CudaEngine, StepRequest
    prompt = synth.integers(1, 128, ref_model.vocab, stream=0).astype(np.int32)
    steps = 64
    ids_ref, _, logits_ref = ref_model.generate_greedy(prompt, steps, sink=0, want_logits=True)
    with CudaEngine(archive, device=0, max_seqs=2, max_len=512, max_sink=0, numerics=numerics) as eng:
        # teacher forced
        eng.reset(0, len(prompt) + steps, 0)
        lg = eng.prefill(0, prompt, want_logits=True)
        worst = 0.0
        for s in range(steps):
            worst = max(worst, max_abs_rel(lg, logits_ref[s]))
            assert int(np.argmax(lg)) == int(ids_ref[s]), (s, int(np.argmax(lg)), int(ids_ref[s]))
            if s + 1 < steps:
                _, l2 = eng.step([StepRequest(0, int(ids_ref[s]), False)], want_logits=True)
                lg = l2[0]
        assert worst <= tol, worst
        # free-running greedy with selection on the device
        eng.reset(1, len(prompt) + steps, 0)
        eng.prefill(1, prompt[:-1], want_logits=False)
        ids = []
        for s in range(steps):
            sel, _ = eng.step([StepRequest(1, int(prompt[-1]) if s == 0 else -1, True)])
            ids.append(sel[0][0])
        np.testing.assert_array_equal(np.array(ids), ids_ref)
        # the int8 KV codes: the K/V inputs differ from the reference's in the last binary32 bits, so a
        # code may round the other way; report the matching fraction (it is not a bit-exact bar here)
        rt = oracle.Runtime(ref_model)
        rt.reset(len(prompt) + steps, 0)
        for t in list(prompt) + list(ids_ref[:-1]):
            rt.step(int(t), want_logits=False)
        same = total = 0
        for layer in range(ref_model.layers):
            kc, vc, _, _ = eng.read_kv(1, layer)
            rkc, rvc, _, _ = rt.read_kv(layer)
            same += int(np.sum(kc == rkc) + np.sum(vc == rvc))
            total += kc.size + vc.size
        print(f"{numerics}: worst logits max-abs-rel {worst:.2e}, KV codes equal {same / total:.4%}")
        assert same / total > kv_equal


def test_scheduler_fast_ids_equal_except_at_near_ties(archive, oracle, ref_model):
    """The device scheduler in fast numerics (64 slots, two micro-batches, graph replay, reused slots,
    prompts up to 300 tokens across the window): every finished sequence's id stream equals the
    oracle's, or first differs at a step where the oracle's top-two logits are within the tolerance."""
    import concurrent.futures
    import os
    from needle_b200.backend import CudaEngine
    rng = np.random.default_rng(44)
    n = 96
    prompts = [rng.integers(0, ref_model.vocab, int(k)).astype(np.int32) for k in rng.integers(8, 300, n)]
    gens = rng.integers(4, 24, n).astype(np.int32)
    with CudaEngine(archive, device=0, max_seqs=64, max_len=400, max_sink=0, numerics="fast",
                    micro_batches=2) as eng:
        eng.sched_load(64, prompts, gens)
        for _ in range(200):
            eng.sched_step(8)
            _, _, finished, _ = eng.sched_status()
            if finished == n:
                break
        assert finished == n
        ids = eng.sched_ids()
        assert eng.damaged_guards() == 0  # no kernel (GEMMs, fast attention) wrote past a buffer
    offs = np.concatenate([[0], np.cumsum(gens)])

    def check(i):
        want, _, logits = ref_model.generate_greedy(prompts[i], int(gens[i]), sink=0, want_logits=True)
        got = ids[offs[i]:offs[i + 1]]
        if np.array_equal(got, want):
            return i, None
        s = int(np.argmax(got != want))
        top2 = np.sort(logits[s].astype(np.float64))[-2:]
        return i, (s, float((top2[1] - top2[0]) / max(abs(top2[1]), 1.0)))

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(check, range(n)))
    diverged = [(i, d) for i, d in results if d is not None]
    print(f"fast scheduler: {n - len(diverged)} of {n} id streams identical; divergences {diverged}")
    for i, (s, margin) in diverged:
        assert margin <= LOGIT_TOL, (i, s, margin)
    assert len(diverged) <= n // 10
