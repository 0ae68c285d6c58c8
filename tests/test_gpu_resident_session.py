"""The resident-session boundary driven exactly as needle.js's NeedleRuntime drives it.

`needle_b200.backend.NeedleRuntime` restates the host side of NeedleRuntime.step (packages/
needle.js/src/model/runtime.ts:280-583): the embedding row through InferenceBackend.row, the scaled
lanes, #engramLookup on the token history, then the session calls in the reference's order
(prepareResidentEngrams, beginResidentToken, forwardResidentToken, finishResidentToken or
finishResidentTokenForSelection + selectResidentToken; backend.ts:66-80).  The session never sees
a token id.  BASELINE config 1 (128-token prompt from seed 1, token-serial prefill as
runtime.ts:227-243, 64 greedy steps) must give the oracle's ids, logits and int8 KV bit for bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def backend():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import synth
    from needle_b200.backend import CudaBackend
    archive = synth.build_archive(0, probe_heads=True)
    b = CudaBackend(archive, device=0, max_seqs=4, max_len=2048, max_sink=160)
    yield b
    b.dispose()


@pytest.fixture(scope="module")
def ref_model(oracle, backend):
    return oracle.Model(backend.weights)


def generate(runtime, prompt, steps):
    """NeedleModel.generate's greedy loop (model.ts:88-153) without tokenizer or EOS stop."""
    runtime.reset(len(prompt) + steps, 0)
    logits = runtime.prefill(prompt)
    ids, all_logits = [], []
    for s in range(steps):
        tok = int(np.argmax(logits))
        ids.append(tok)
        all_logits.append(logits)
        if s + 1 < steps:
            logits = runtime.step(tok)
    return np.array(ids), np.stack(all_logits)


def test_config1_through_the_session_calls(backend, oracle, ref_model):
    from needle_b200 import synth
    from needle_b200.backend import NeedleRuntime
    prompt = synth.integers(1, 128, ref_model.vocab, stream=0).astype(np.int32)
    steps = 64
    rt = oracle.Runtime(ref_model)
    rt.reset(len(prompt) + steps, 0)
    logits = None
    for i, t in enumerate(prompt):
        logits = rt.step(int(t), want_logits=i == len(prompt) - 1)
    want_ids, want_logits = [], []
    for s in range(steps):
        tok = int(np.argmax(logits))
        want_ids.append(tok)
        want_logits.append(logits)
        if s + 1 < steps:
            logits = rt.step(tok)
    runtime = NeedleRuntime(backend, collect_confidence=False)
    ids, got_logits = generate(runtime, prompt, steps)
    np.testing.assert_array_equal(ids, np.array(want_ids))
    np.testing.assert_array_equal(got_logits, np.stack(want_logits))
    eng, slot = backend.engine, runtime.slot_index
    for layer in range(ref_model.layers):
        kc, vc, ks, vs = eng.read_kv(slot, layer)
        rkc, rvc, rks, rvs = rt.read_kv(layer)
        np.testing.assert_array_equal(kc, rkc, err_msg=f"key codes layer {layer}")
        np.testing.assert_array_equal(vc, rvc, err_msg=f"value codes layer {layer}")
        np.testing.assert_array_equal(ks, rks)
        np.testing.assert_array_equal(vs, rvs)
    np.testing.assert_array_equal(runtime.session.read_resident_lanes(), rt.read_lanes())
    runtime.dispose()


def test_step_selected_and_prefill_selected(backend, oracle, ref_model):
    """stepSelected / prefillSelected (runtime.ts:245-278) through selectResidentToken, masked and
    unmasked, with list-order tie breaking and the log-probability of logSoftmaxAt."""
    from needle_b200.backend import NeedleRuntime
    rng = np.random.default_rng(31)
    prompt = rng.integers(0, ref_model.vocab, 40).astype(np.int32)
    rt = oracle.Runtime(ref_model)
    rt.reset(80, 4)
    runtime = NeedleRuntime(backend, collect_confidence=False)
    runtime.reset(80, 4)
    allowed0 = rng.choice(ref_model.vocab, 900, replace=False).astype(np.uint32)
    for t in prompt[:-1]:
        rt.step(int(t), want_logits=False)
    rid, rlp = rt.step_selected(int(prompt[-1]), allowed0)
    gid, glp = runtime.prefill_selected(prompt, allowed0)
    assert gid == rid and abs(glp - rlp) < 1e-9
    tok = gid
    for k in range(8):
        allowed = None if k % 3 == 0 else rng.choice(ref_model.vocab, int(rng.integers(1, 4000)),
                                                     replace=False).astype(np.uint32)
        rid, rlp = rt.step_selected(tok, allowed)
        gid, glp = runtime.step_selected(tok, allowed)
        assert gid == rid and abs(glp - rlp) < 1e-9, (k, gid, rid)
        tok = gid
    assert runtime.position == rt.position
    runtime.dispose()


def test_collecting_session_confidence(backend, oracle, ref_model):
    """collectConfidence through the session: the pooled probes come from the runtime's lanes, and
    residentConfidence equals the oracle's confidence()."""
    from needle_b200.backend import NeedleRuntime
    rng = np.random.default_rng(32)
    prompt = rng.integers(0, ref_model.vocab, 24).astype(np.int32)
    rt = oracle.Runtime(ref_model, collect_confidence=True)
    rt.reset(40, 0)
    for t in prompt:
        rt.step(int(t), want_logits=False)
    runtime = NeedleRuntime(backend, collect_confidence=True)
    runtime.reset(40, 0)
    for t in prompt:
        runtime.step(int(t), want_logits=False)
    assert abs(runtime.confidence() - rt.confidence()) <= 1e-12
    runtime.dispose()


def test_session_errors(backend, ref_model):
    """The session rejects a forward without begin, a position that is not the slot's, and an end
    without a forward; the runtime keeps the reference's step preconditions."""
    from needle_b200 import native
    from needle_b200.backend import NeedleRuntime
    from needle_b200.native import NeedleError
    runtime = NeedleRuntime(backend, collect_confidence=False)
    with pytest.raises(NeedleError) as e:
        runtime.step(1)
    assert e.value.code == "INVALID_CACT"
    runtime.reset(2, 0)
    with pytest.raises(NeedleError) as e:
        runtime.step(ref_model.vocab)
    assert e.value.code == "INVALID_CACT"
    s = runtime.session
    with pytest.raises(NeedleError) as e:
        s.forward_resident_token({"position": 0, "engramKeys": [], "engramValues": []})
    assert e.value.code == "BACKEND_UNAVAILABLE"
    s.begin_resident_token(np.zeros(2048, dtype=np.float32))
    with pytest.raises(NeedleError) as e:
        s.forward_resident_token({"position": 1, "engramKeys": [], "engramValues": []})
    assert e.value.code == "BACKEND_UNAVAILABLE"
    with pytest.raises(NeedleError) as e:
        s.finish_resident_token(True)
    assert e.value.code == "BACKEND_UNAVAILABLE"
    runtime.step(3, want_logits=False)
    runtime.step(4, want_logits=False)
    with pytest.raises(NeedleError) as e:
        runtime.step(5)
    assert e.value.code == "CONTEXT_OVERFLOW"
    assert native.lib().needle_cuda_resident_finish(backend.engine.h, s.slot, None) == 6
    runtime.dispose()
