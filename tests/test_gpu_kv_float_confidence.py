"""GPU parity of the float32 KV-cache mode and the confidence probe pool.

* kvCache "float32" (RuntimeOptions.kvCache, runtime.ts:30-32): keys and values are cached as the
  binary32 values the step computed and attention reads them back directly (runtime.ts:686-693,
  744-748, 768-772).  Token ids, logits and the cached floats match the oracle bit for bit, across
  the sink + window wrap as well.
* collectConfidence (runtime.ts:36, 48-105, 634-645): the online probe pool over the scaled
  embedding and every layer's lane mean, then sigmoid(denseMatvec(projection, pooled, bias)).  The
  pool's exponentials are binary64 library calls on both sides (CUDA's exp on the GPU, the C
  library's in the oracle), which may differ in the last bit, so the confidence is compared to
  1e-12; it is rounded to binary32 before the sigmoid, so in practice it is equal.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def archive():
    from needle_b200 import synth
    return synth.build_archive(0)


@pytest.fixture(scope="module")
def ref_model(oracle, archive):
    return oracle.Model(archive)


def greedy_oracle(oracle, model, prompt, steps, sink=0, kv_mode=0, collect=False):
    rt = oracle.Runtime(model, kv_mode=kv_mode, collect_confidence=collect)
    rt.reset(len(prompt) + steps, sink)
    logits = None
    for i, t in enumerate(prompt):
        logits = rt.step(int(t), want_logits=(i == len(prompt) - 1))
    ids, all_logits = [], []
    for s in range(steps):
        tok = int(np.argmax(logits))
        ids.append(tok)
        all_logits.append(logits)
        if s + 1 < steps:
            logits = rt.step(tok)
    return np.array(ids), np.stack(all_logits), rt


def greedy_engine(engine, slot, prompt, steps, sink=0, collect=False):
    from needle_b200.backend import StepRequest
    engine.reset(slot, len(prompt) + steps, sink, collect)
    engine.prefill(slot, prompt[:-1], want_logits=False)
    ids, logits = [], []
    for s in range(steps):
        tok = int(prompt[-1]) if s == 0 else -1
        sel, lg = engine.step([StepRequest(slot, tok, True)], want_logits=True)
        ids.append(sel[0][0])
        logits.append(lg[0])
    return np.array(ids), np.stack(logits)


@pytest.fixture(scope="module")
def engine_f32(torch_cuda, archive):
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200.backend import CudaEngine
    e = CudaEngine(archive, device=0, max_seqs=2, max_len=512, max_sink=16, kv_cache="float32")
    yield e
    e.close()


@pytest.mark.parametrize("n_prompt,steps,sink", [(40, 12, 0), (262, 6, 4)])
def test_float32_kv_matches_oracle(engine_f32, oracle, ref_model, n_prompt, steps, sink):
    rng = np.random.default_rng(n_prompt)
    prompt = rng.integers(0, ref_model.vocab, n_prompt).astype(np.int32)
    ids_ref, logits_ref, rt = greedy_oracle(oracle, ref_model, prompt, steps, sink=sink, kv_mode=1)
    ids, logits = greedy_engine(engine_f32, 1, prompt, steps, sink=sink)
    np.testing.assert_array_equal(ids, ids_ref)
    np.testing.assert_array_equal(logits, logits_ref)
    for layer in (0, ref_model.layers // 2, ref_model.layers - 1):
        k, v = engine_f32.read_kv_f32(1, layer)
        rk, rv = rt.read_kv_f32(layer)
        np.testing.assert_array_equal(k, rk, err_msg=f"keys layer {layer}")
        np.testing.assert_array_equal(v, rv, err_msg=f"values layer {layer}")


def test_float32_context_rejects_int8_read(engine_f32):
    from needle_b200.native import NeedleError
    with pytest.raises(NeedleError) as e:
        engine_f32.read_kv(1, 0)
    assert e.value.code == "INVALID_CACT"


def test_confidence_pool_matches_oracle(torch_cuda, archive, oracle, ref_model):
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200.backend import CudaEngine
    rng = np.random.default_rng(77)
    prompt = rng.integers(0, ref_model.vocab, 20).astype(np.int32)
    steps = 5
    ids_ref, _, rt = greedy_oracle(oracle, ref_model, prompt, steps, collect=True)
    want = rt.confidence()
    assert np.isfinite(want)
    with CudaEngine(archive, device=0, max_seqs=3, max_len=256, max_sink=16) as eng:
        ids, _ = greedy_engine(eng, 2, prompt, steps, collect=True)
        np.testing.assert_array_equal(ids, ids_ref)
        got = eng.confidence(2)
        assert abs(got - want) <= 1e-12, (got, want)
        # a slot that does not collect reports NaN, like a runtime without the option
        greedy_engine(eng, 0, prompt[:5], 2, collect=False)
        assert np.isnan(eng.confidence(0))
        # reset clears the pool: the same run again gives the same value
        greedy_engine(eng, 2, prompt, steps, collect=True)
        assert eng.confidence(2) == got
