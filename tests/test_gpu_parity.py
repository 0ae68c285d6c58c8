"""GPU parity of the CUDA engine against the CPU oracle, through the C-ABI.

The engine's exact numerics restate the reference's binary64 arithmetic operation for operation,
so quantised matvecs, attention outputs, logits, token ids and int8 KV codes are compared for
bitwise equality; logits additionally satisfy the north star's 1e-3 max-abs-relative bound
(asserted separately so a failure names which bar broke).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3  # max |a - b| / max(|b|, 1) over a logits vector


def max_abs_rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b) / np.maximum(np.abs(b.astype(np.float64)), 1.0)))


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


@pytest.fixture(scope="module")
def engine(torch_cuda, archive):
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200.backend import CudaEngine
    e = CudaEngine(archive, device=0, max_seqs=8, max_len=2048, max_sink=160)
    yield e
    e.close()


def codebook():
    from needle_b200 import synth
    return synth.lloyd_max_codebook()


# ------------------------------------------------------------------ isolated quantised matvec

@pytest.mark.parametrize("bits", [2, 3, 4, 5])
@pytest.mark.parametrize("rows,inputs", [(512, 512), (256, 512), (4, 2048), (108, 2048), (432, 2048), (8192, 512)])
def test_cq_matvec_dev_bit_exact(torch_cuda, oracle, bits, rows, inputs):
    torch = torch_cuda
    from needle_b200 import native, synth
    packed, norms = synth.random_cq_matrix(rows, inputs, bits, seed=2)
    cb = codebook()
    batch = 8
    x = synth.normal(2, batch * inputs, stream=7).astype(np.float32).reshape(batch, inputs)
    d_packed = torch.from_numpy(packed.copy()).cuda()
    d_norms = torch.from_numpy(norms.view(np.int16).copy()).cuda()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.zeros(batch, rows, dtype=torch.float32, device="cuda")
    desc = native.CqMatrixDesc(d_packed.data_ptr(), d_norms.data_ptr(), rows, inputs, 128, bits)
    native.check(native.lib().needle_cuda_cq_matvec_dev(C.byref(desc), native.ptr(cb), d_x.data_ptr(), batch,
                                                        d_y.data_ptr(), None))
    torch.cuda.synchronize()
    y = d_y.cpu().numpy()
    m = oracle.CqMatrix(rows, inputs, 128, bits, packed, norms, cb[:4], cb[4:12], cb[12:])
    for b in range(batch):
        np.testing.assert_array_equal(y[b], m.matvec(x[b]), err_msg=f"batch item {b}")


@pytest.mark.parametrize("bits,batch", [(4, 1), (3, 1), (5, 3), (2, 8)])
def test_cq_matvec_dev_long_rows_small_batch_bit_exact(torch_cuda, oracle, bits, batch):
    """Small batches of long rows take the split-group path (per-group dots, then ordered totals)."""
    torch = torch_cuda
    from needle_b200 import native, synth
    rows, inputs = 300, 8192 - 64  # a padded tail group too
    packed, norms = synth.random_cq_matrix(rows, inputs, bits, seed=5)
    cb = codebook()
    x = synth.normal(5, batch * inputs, stream=9).astype(np.float32).reshape(batch, inputs)
    d_packed = torch.from_numpy(packed.copy()).cuda()
    d_norms = torch.from_numpy(norms.view(np.int16).copy()).cuda()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.zeros(batch, rows, dtype=torch.float32, device="cuda")
    desc = native.CqMatrixDesc(d_packed.data_ptr(), d_norms.data_ptr(), rows, inputs, 128, bits)
    native.check(native.lib().needle_cuda_cq_matvec_dev(C.byref(desc), native.ptr(cb), d_x.data_ptr(), batch,
                                                        d_y.data_ptr(), None))
    torch.cuda.synchronize()
    m = oracle.CqMatrix(rows, inputs, 128, bits, packed, norms, cb[:4], cb[4:12], cb[12:])
    y = d_y.cpu().numpy()
    for b in range(batch):
        np.testing.assert_array_equal(y[b], m.matvec(x[b]), err_msg=f"batch item {b}")


@pytest.mark.parametrize("rows,inputs,batch", [(1536, 512, 64), (1536, 512, 300), (2000, 128, 100),
                                               (77, 256, 64), (8192, 512, 70), (5, 384, 65)])
def test_cq_matvec_dev_byte_table_bit_exact(torch_cuda, oracle, rows, inputs, batch):
    """2-bit launches of 64 items or more take the byte-table kernel: one item per CTA and up to
    1536 rows per part (two parts below 296 items; six for 8192 rows), every group dot read from a
    per-(item, group) table of byte terms with the lanes skewed across the table's columns.  Same
    bits as the oracle, including rows that end inside a part and parts with fewer rows than
    threads."""
    torch = torch_cuda
    from needle_b200 import native, synth
    packed, norms = synth.random_cq_matrix(rows, inputs, 2, seed=rows + batch)
    cb = codebook()
    x = synth.normal(6, batch * inputs, stream=11).astype(np.float32).reshape(batch, inputs)
    x[1, :] = 0.0  # an all-zero item: every term and dot is +0
    d_packed = torch.from_numpy(packed.copy()).cuda()
    d_norms = torch.from_numpy(norms.view(np.int16).copy()).cuda()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device="cuda")
    desc = native.CqMatrixDesc(d_packed.data_ptr(), d_norms.data_ptr(), rows, inputs, 128, 2)
    native.check(native.lib().needle_cuda_cq_matvec_dev(C.byref(desc), native.ptr(cb), d_x.data_ptr(), batch,
                                                        d_y.data_ptr(), None))
    torch.cuda.synchronize()
    m = oracle.CqMatrix(rows, inputs, 128, 2, packed, norms, cb[:4], cb[4:12], cb[12:])
    y = d_y.cpu().numpy()
    for b in range(batch):
        np.testing.assert_array_equal(y[b], m.matvec(x[b]), err_msg=f"batch item {b}")


@pytest.mark.parametrize("cap", [8192, 8190])
def test_attention_dev_fast_within_tolerance(torch_cuda, oracle, cap):
    """Fast numerics (binary32, online softmax, split positions) vs the oracle's binary64 attention:
    every output within 2e-4 of the largest output magnitude, including a full 8192-position row.
    A capacity that is a multiple of 4 takes the bulk-copy pipelined kernel, 8190 the direct-load one."""
    torch = torch_cuda
    from needle_b200 import native
    rng = np.random.default_rng(31)
    batch = 5
    counts = np.array([1, 7, 1000, 1025, cap], dtype=np.int32)
    q = rng.standard_normal((batch, 512)).astype(np.float32)
    kc = rng.integers(-127, 128, (batch, 4, cap, 64)).astype(np.int8)
    vc = rng.integers(-127, 128, (batch, 4, cap, 64)).astype(np.int8)
    ks = (np.abs(rng.standard_normal((batch, 4, cap))) * 0.02).astype(np.float32)
    vs = (np.abs(rng.standard_normal((batch, 4, cap))) * 0.02).astype(np.float32)
    d = {k: torch.from_numpy(v).cuda() for k, v in dict(q=q, kc=kc, vc=vc, ks=ks, vs=vs, n=counts).items()}
    out = torch.zeros(batch, 512, dtype=torch.float32, device="cuda")
    native.check(native.lib().needle_cuda_attention_dev_fast(
        d["q"].data_ptr(), d["kc"].data_ptr(), d["ks"].data_ptr(), d["vc"].data_ptr(), d["vs"].data_ptr(),
        d["n"].data_ptr(), batch, cap, out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(batch):
        n = counts[b]
        want = oracle.attention_int8(q[b], kc[b, :, :n], ks[b, :, :n], vc[b, :, :n], vs[b, :, :n])
        err = np.max(np.abs(got[b].astype(np.float64) - want))
        assert err <= 2e-4 * max(np.max(np.abs(want)), 1e-3), (b, n, err)


def test_model_matvec_and_row_bit_exact(engine, ref_model):
    rng = np.random.default_rng(11)
    tensors = [0, 2, 3, 8, ref_model.num_tensors() - 3]
    for t in range(ref_model.num_tensors()):
        rec = ref_model.record(t)
        if rec["dtype"] == 3 and rec["bits"] == 5:
            tensors.append(t)
            break
    for t in tensors:
        rec = ref_model.record(t)
        if rec["dtype"] != 3:
            continue
        rows, width = rec["shape"]
        x = rng.standard_normal(width).astype(np.float32)
        start, count = (1, min(rows - 1, 300))
        np.testing.assert_array_equal(engine.matvec(t, x, start, count), ref_model.matvec(t, x, start, count))
        for r in (0, rows // 2, rows - 1):
            np.testing.assert_array_equal(engine.row(t, r, width), ref_model.row(t, r))


# ------------------------------------------------------------------ isolated attention

def test_attention_dev_bit_exact(torch_cuda, oracle):
    torch = torch_cuda
    rng = np.random.default_rng(3)
    batch, cap = 6, 320
    counts = np.array([1, 2, 64, 200, 319, 320], dtype=np.int32)
    q = rng.standard_normal((batch, 512)).astype(np.float32)
    kc = rng.integers(-127, 128, (batch, 4, cap, 64)).astype(np.int8)
    vc = rng.integers(-127, 128, (batch, 4, cap, 64)).astype(np.int8)
    ks = (np.abs(rng.standard_normal((batch, 4, cap))) * 0.02).astype(np.float32)
    vs = (np.abs(rng.standard_normal((batch, 4, cap))) * 0.02).astype(np.float32)
    d = {k: torch.from_numpy(v).cuda() for k, v in dict(q=q, kc=kc, vc=vc, ks=ks, vs=vs, n=counts).items()}
    out = torch.zeros(batch, 512, dtype=torch.float32, device="cuda")
    from needle_b200 import native
    native.check(native.lib().needle_cuda_attention_dev(
        d["q"].data_ptr(), d["kc"].data_ptr(), d["ks"].data_ptr(), d["vc"].data_ptr(), d["vs"].data_ptr(),
        d["n"].data_ptr(), batch, cap, out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(batch):
        n = counts[b]
        want = oracle.attention_int8(q[b], kc[b, :, :n], ks[b, :, :n], vc[b, :, :n], vs[b, :, :n])
        np.testing.assert_array_equal(got[b], want, err_msg=f"item {b} count {n}")


# ------------------------------------------------------------------ full decode (config 1)

def oracle_greedy(oracle, model, prompt, steps, sink=0):
    rt = oracle.Runtime(model)
    rt.reset(len(prompt) + steps, sink)
    logits = None
    for i, t in enumerate(prompt):
        logits = rt.step(int(t), want_logits=(i == len(prompt) - 1))
    ids, lps, all_logits = [], [], []
    for s in range(steps):
        tok = int(np.argmax(logits))
        ids.append(tok)
        all_logits.append(logits)
        m = float(np.max(logits))
        lps.append(float(logits[tok]) - m - float(np.log(np.sum(np.exp(logits.astype(np.float64) - m)))))
        if s + 1 < steps:
            logits = rt.step(tok)
    kv = [rt.read_kv(layer) for layer in range(model.layers)]
    return np.array(ids), np.array(lps), np.stack(all_logits), kv, rt


def engine_greedy(engine, slot, prompt, steps, sink=0):
    from needle_b200.backend import StepRequest
    engine.reset(slot, len(prompt) + steps, sink)
    if len(prompt) > 1:
        engine.prefill(slot, prompt[:-1], want_logits=False)
    ids, lps, logits = [], [], []
    for s in range(steps):
        tok = int(prompt[-1]) if s == 0 else -1
        sel, lg = engine.step([StepRequest(slot, tok, True)], want_logits=True)
        ids.append(sel[0][0])
        lps.append(sel[0][1])
        logits.append(lg[0])
    return np.array(ids), np.array(lps), np.stack(logits)


@pytest.fixture(scope="module")
def config1(oracle, ref_model):
    from needle_b200 import synth
    prompt = synth.integers(1, 128, ref_model.vocab, stream=0).astype(np.int32)
    return prompt, oracle_greedy(oracle, ref_model, prompt, 64)


def test_config1_greedy_tokens_logits_kv(engine, ref_model, config1):
    prompt, (ids_ref, lps_ref, logits_ref, kv_ref, _) = config1
    ids, lps, logits = engine_greedy(engine, 0, prompt, 64)
    np.testing.assert_array_equal(ids, ids_ref)
    worst = max(max_abs_rel(logits[s], logits_ref[s]) for s in range(64))
    assert worst <= LOGIT_TOL, worst
    np.testing.assert_array_equal(logits, logits_ref)
    np.testing.assert_allclose(lps, lps_ref, rtol=0, atol=1e-9)
    for layer in range(ref_model.layers):
        kc, vc, ks, vs = engine.read_kv(0, layer)
        rkc, rvc, rks, rvs = kv_ref[layer]
        np.testing.assert_array_equal(kc, rkc, err_msg=f"key codes layer {layer}")
        np.testing.assert_array_equal(vc, rvc, err_msg=f"value codes layer {layer}")
        np.testing.assert_array_equal(ks, rks)
        np.testing.assert_array_equal(vs, rvs)


# ------------------------------------------------------------------ ragged batch, masks, window

def test_ragged_batch_matches_independent_sequences(engine, oracle, ref_model):
    """Four slots at different positions step together; each matches its own oracle run."""
    from needle_b200.backend import StepRequest
    rng = np.random.default_rng(5)
    lens = [3, 9, 17, 1]
    steps = 6
    prompts = [rng.integers(0, ref_model.vocab, n).astype(np.int32) for n in lens]
    refs = [oracle_greedy(oracle, ref_model, p, steps) for p in prompts]
    slots = [2, 3, 4, 5]
    for s, p in zip(slots, prompts):
        engine.reset(s, len(p) + steps, 0)
    # lockstep: every slot consumes one token per step until all finished
    cursor = [0] * 4
    got = [[] for _ in range(4)]
    while any(len(g) < steps for g in got):
        reqs, who = [], []
        for i in range(4):
            if len(got[i]) >= steps:
                continue
            p = prompts[i]
            if cursor[i] < len(p) - 1:
                reqs.append(StepRequest(slots[i], int(p[cursor[i]]), False))
            else:
                tok = int(p[-1]) if cursor[i] == len(p) - 1 else -1
                reqs.append(StepRequest(slots[i], tok, True))
            who.append(i)
            cursor[i] += 1
        sel, _ = engine.step(reqs)
        for r, i, s in zip(reqs, who, sel):
            if r.select:
                got[i].append(s[0])
    for i in range(4):
        np.testing.assert_array_equal(np.array(got[i]), refs[i][0], err_msg=f"sequence {i}")


def test_masked_selection_matches_select_token(engine, oracle, ref_model):
    from needle_b200.backend import StepRequest
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, ref_model.vocab, 12).astype(np.int32)
    rt = oracle.Runtime(ref_model)
    rt.reset(40, 0)
    for t in prompt[:-1]:
        rt.step(int(t), want_logits=False)
    engine.reset(6, 40, 0)
    engine.prefill(6, prompt[:-1], want_logits=False)
    tok = int(prompt[-1])
    for k in range(6):
        allowed = np.sort(rng.choice(ref_model.vocab, size=int(rng.integers(1, 3000)), replace=False)).astype(np.uint32)
        if k == 3:
            allowed = allowed[::-1].copy()  # list order, not id order, breaks ties
        rid, rlp = rt.step_selected(tok, allowed)
        sel, _ = engine.step([StepRequest(6, tok, True, allowed)])
        gid, glp = sel[0]
        assert gid == rid
        assert abs(glp - rlp) < 1e-9
        tok = gid


def test_split_step_matches_step(engine, ref_model):
    """needle_cuda_step_begin / _end (the host computes allowed ids while the layers run) select
    exactly as needle_cuda_step; no other call may come in between; a failed end drops the step;
    a select cleared at the end (a grammar dead end) just advances the slot."""
    from needle_b200.backend import StepRequest
    from needle_b200.native import NeedleError
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, ref_model.vocab, 9).astype(np.int32)
    for s in (4, 5, 7):
        engine.reset(s, 64, 0)
        engine.prefill(s, prompt[:-1], want_logits=False)
    tok = int(prompt[-1])
    for k in range(5):
        allowed = np.sort(rng.choice(ref_model.vocab, size=int(rng.integers(1, 3000)), replace=False)).astype(np.uint32)
        want, _ = engine.step([StepRequest(4, tok, True, allowed)])
        reqs = [StepRequest(7, int(prompt[k]), False), StepRequest(5, tok, True, None)]
        engine.step_begin(reqs)
        reqs[1].allowed = allowed
        got = engine.step_end(reqs)
        assert got[0] is None and got[1][0] == want[0][0] and got[1][1] == want[0][1]
        tok = want[0][0]
    assert engine.position(4) == engine.position(5) == len(prompt) - 1 + 5
    pos = engine.position(5)
    engine.step_begin([StepRequest(5, tok, True)])
    with pytest.raises(NeedleError) as e:
        engine.step([StepRequest(4, tok, False)])
    assert e.value.code == "BACKEND_UNAVAILABLE"
    with pytest.raises(NeedleError) as e:
        engine.step_end([StepRequest(5, tok + 1, True, np.arange(5, dtype=np.uint32))])
    assert e.value.code == "BACKEND_UNAVAILABLE"
    assert engine.position(5) == pos  # dropped
    engine.step_begin([StepRequest(5, tok, True)])
    assert engine.step_end([StepRequest(5, tok, False)]) == [None]  # select cleared
    assert engine.position(5) == pos + 1


def test_wide_host_steps_match_single_steps(torch_cuda, archive, ref_model):
    """80 sequences stepped together (needle_cuda_step and the begin / end split alike, with a mix
    of prompt items, masked and unmasked selections) must select exactly what each selects stepped
    alone (single-item steps are the path checked against the oracle above)."""
    from needle_b200.backend import CudaEngine, StepRequest
    rng = np.random.default_rng(13)
    n, steps = 80, 6
    prompts = [rng.integers(0, ref_model.vocab, int(rng.integers(1, 5))).astype(np.int32) for _ in range(n)]
    masks = [[None if rng.random() < 0.5 else
              np.sort(rng.choice(ref_model.vocab, size=int(rng.integers(1, 2000)), replace=False)).astype(np.uint32)
              for _ in range(steps)] for _ in range(n)]
    with CudaEngine(archive, device=0, max_seqs=n, max_len=32, max_sink=16) as eng:
        def together(split):
            for s in range(n):
                eng.reset(s, 32, 0)
            out = [[] for _ in range(n)]
            pending = [None] * n
            for t in range(max(p.size for p in prompts) + steps):
                reqs = []
                for s in range(n):
                    p = prompts[s]
                    if t < p.size:
                        reqs.append(StepRequest(s, int(p[t]), t == p.size - 1, masks[s][0] if t == p.size - 1 else None))
                    elif t - p.size + 1 < steps:
                        k = t - p.size + 1
                        reqs.append(StepRequest(s, pending[s], True, masks[s][k]))
                if not reqs:
                    break
                if split:
                    keep = [r.allowed for r in reqs]
                    for r in reqs:
                        r.allowed = None
                    eng.step_begin(reqs)
                    for r, a in zip(reqs, keep):
                        r.allowed = a
                    sel = eng.step_end(reqs)
                else:
                    sel, _ = eng.step(reqs)
                for r, x in zip(reqs, sel):
                    if x is not None:
                        out[r.seq].append(x)
                        pending[r.seq] = x[0]
            return out

        def alone():
            out = [[] for _ in range(n)]
            for s in range(n):
                eng.reset(s, 32, 0)
                p = prompts[s]
                for t in range(p.size - 1):
                    eng.step([StepRequest(s, int(p[t]))])
                tok = int(p[-1])
                for k in range(steps):
                    sel, _ = eng.step([StepRequest(s, tok, True, masks[s][k])])
                    out[s].append(sel[0])
                    tok = sel[0][0]
            return out

        want = alone()
        assert together(False) == want
        assert together(True) == want


@pytest.mark.parametrize("lengths,sink", [((1,), 0), ((2,), 0), ((64,), 0), ((65,), 0), ((130,), 0),
                                          ((40, 90), 0), ((3, 61, 5), 0), ((300,), 8)])
def test_chunked_prefill_matches_token_by_token(engine, ref_model, lengths, sink):
    """needle_cuda_prefill takes a slot's tokens in chunks (one item per token, K/V of the chunk
    appended before its items attend, engram taps and token history from the chunk, the slot
    advanced once); it must leave exactly the state n one-token steps leave: logits, every layer's
    KV codes and scales, the lanes, and the tokens that follow.  Several prefill calls continue one
    sequence; 300 tokens with a sink of 8 cross the 256-position window."""
    from needle_b200.backend import StepRequest
    rng = np.random.default_rng(sum(lengths) + sink)
    parts = [rng.integers(0, ref_model.vocab, n).astype(np.int32) for n in lengths]
    total = sum(lengths)
    a, b = 2, 3
    for s in (a, b):
        engine.reset(s, total + 8, sink)
    for k, part in enumerate(parts):
        last = k == len(parts) - 1
        got = engine.prefill(a, part, want_logits=last)
        for i, t in enumerate(part):
            _, lg = engine.step([StepRequest(b, int(t))], want_logits=last and i == part.size - 1)
        if last:
            np.testing.assert_array_equal(got, lg[0])
    assert engine.position(a) == engine.position(b) == total
    for layer in range(engine.geometry.layers):
        for x, y in zip(engine.read_kv(a, layer), engine.read_kv(b, layer)):
            written = min(total, x.shape[1])  # cache slots written so far (the rest hold old data)
            np.testing.assert_array_equal(x[:, :written], y[:, :written], err_msg=f"layer {layer}")
    np.testing.assert_array_equal(engine.read_lanes(a), engine.read_lanes(b))
    tok = int(rng.integers(0, ref_model.vocab))
    for _ in range(3):
        sa, _ = engine.step([StepRequest(a, tok, True)])
        sb, _ = engine.step([StepRequest(b, tok, True)])
        assert sa == sb
        tok = sa[0][0]


def test_sink_and_window_crossing(engine, oracle, ref_model):
    """A sequence longer than the 256-token window with 8 pinned sink tokens
    (runtime.ts:659-664, 723-728): tokens and cached codes stay exact past the wrap."""
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, ref_model.vocab, 270).astype(np.int32)
    steps = 4
    ids_ref, _, logits_ref, kv_ref, _ = oracle_greedy(oracle, ref_model, prompt, steps, sink=8)
    ids, _, logits = engine_greedy(engine, 7, prompt, steps, sink=8)
    np.testing.assert_array_equal(ids, ids_ref)
    np.testing.assert_array_equal(logits, logits_ref)
    for layer in (0, 13, ref_model.layers - 1):
        kc, vc, ks, vs = engine.read_kv(7, layer)
        np.testing.assert_array_equal(kc, kv_ref[layer][0])
        np.testing.assert_array_equal(vc, kv_ref[layer][1])


def test_device_scheduler_matches_oracle(engine, oracle, ref_model):
    """Continuous batching on the device: 7 queued sequences through 3 slots."""
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, ref_model.vocab, int(n)).astype(np.int32) for n in rng.integers(2, 12, 7)]
    gens = rng.integers(1, 6, 7).astype(np.int32)
    want, processed_ref = ref_model.decode_many(prompts, gens, 4)
    engine.sched_load(3, prompts, gens)
    total = int(sum(len(p) + g - 1 for p, g in zip(prompts, gens)))
    for _ in range(200):
        engine.sched_step(1)
        tokens, generated, finished, last = engine.sched_status()
        if finished == len(prompts):
            break
    assert finished == len(prompts)
    np.testing.assert_array_equal(last, want)
    assert tokens == total == processed_ref
    assert generated == int(gens.sum())


def test_device_scheduler_two_microbatches_and_graph(torch_cuda, archive, oracle, ref_model):
    """64+ slots: the step runs as two micro-batches on two stream pairs and, after the first
    step, as a replayed CUDA graph; every sequence still matches the oracle."""
    from needle_b200.backend import CudaEngine
    rng = np.random.default_rng(8)
    n = 90
    prompts = [rng.integers(0, ref_model.vocab, int(k)).astype(np.int32) for k in rng.integers(1, 7, n)]
    gens = rng.integers(1, 4, n).astype(np.int32)
    want, processed_ref = ref_model.decode_many(prompts, gens, 8)
    with CudaEngine(archive, device=0, max_seqs=64, max_len=64, max_sink=0) as eng:
        eng.sched_load(64, prompts, gens)
        for _ in range(100):
            eng.sched_step(4)
            tokens, generated, finished, last = eng.sched_status()
            if finished == n:
                break
        assert finished == n
        np.testing.assert_array_equal(last, want)
        assert tokens == processed_ref and generated == int(gens.sum())


def test_errors_follow_needle_error_codes(engine, ref_model):
    from needle_b200.backend import StepRequest
    from needle_b200.native import NeedleError
    with pytest.raises(NeedleError) as e:
        engine.reset(1, 4096, 0)
    assert e.value.code == "CONTEXT_OVERFLOW"
    engine.reset(1, 2, 0)
    with pytest.raises(NeedleError) as e:
        engine.step([StepRequest(1, ref_model.vocab, False)])
    assert e.value.code == "INVALID_CACT"
    engine.step([StepRequest(1, 5, False)])
    engine.step([StepRequest(1, 6, False)])
    with pytest.raises(NeedleError) as e:
        engine.step([StepRequest(1, 7, False)])
    assert e.value.code == "CONTEXT_OVERFLOW"
    engine.reset(1, 8, 0)
    with pytest.raises(NeedleError) as e:
        engine.step([StepRequest(1, 5, True, np.zeros(0, dtype=np.uint32))])
    assert e.value.code == "INVALID_CACT"


@pytest.mark.parametrize("bits,rows,inputs,batch", [(4, 1000, 8192, 1), (2, 512, 512, 3), (5, 300, 2048, 6),
                                                    (4, 64, 20000, 2), (4, 700, 1000, 10), (2, 1500, 8192, 1),
                                                    (4, 8192, 16384, 8),
                                                    # batch >= 16: the tensor-core GEMM (bf16 head/tail split)
                                                    (4, 512, 512, 16), (2, 1000, 8192, 32), (5, 300, 2048, 40),
                                                    (4, 64, 20000, 17), (4, 700, 1000, 130), (4, 4096, 4096, 128),
                                                    (2, 8192, 512, 64), (4, 2048, 2048, 6),
                                                    # 3-bit rows always take the tensor-core GEMM
                                                    (3, 512, 512, 1), (3, 512, 512, 64), (3, 1000, 8192, 17),
                                                    (3, 300, 2048, 130)])
def test_cq_matvec_dev_fast_within_tolerance(torch_cuda, oracle, bits, rows, inputs, batch):
    """Fast numerics (binary32) vs the oracle's binary64 cqMatvec: |got - want| <= 1e-5 * sum of
    |terms| bound, taken as 2e-6 * sqrt(inputs) * max|want| + 1e-6.  Batches of 16 and more (6 and
    more for 4M weights), and 3-bit matrices at any batch, take the tensor-core path (130 = two
    passes, the second of 2 items padded to 16)."""
    torch = torch_cuda
    from needle_b200 import native, synth
    packed, norms = synth.random_cq_matrix(rows, inputs, bits, seed=6)
    cb = codebook()
    x = synth.normal(6, batch * inputs, stream=3).astype(np.float32).reshape(batch, inputs)
    d_packed = torch.from_numpy(packed.copy()).cuda()
    d_norms = torch.from_numpy(norms.view(np.int16).copy()).cuda()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.zeros(batch, rows, dtype=torch.float32, device="cuda")
    desc = native.CqMatrixDesc(d_packed.data_ptr(), d_norms.data_ptr(), rows, inputs, 128, bits)
    native.check(native.lib().needle_cuda_cq_matvec_dev_fast(C.byref(desc), native.ptr(cb), d_x.data_ptr(), batch,
                                                             d_y.data_ptr(), None))
    torch.cuda.synchronize()
    y = d_y.cpu().numpy()
    m = oracle.CqMatrix(rows, inputs, 128, bits, packed, norms, cb[:4], cb[4:12], cb[12:])
    for b in range(batch):
        want = m.matvec(x[b]).astype(np.float64)
        tol = 2e-6 * np.sqrt(inputs) * np.max(np.abs(want)) + 1e-6
        assert np.max(np.abs(y[b] - want)) <= tol, (b, np.max(np.abs(y[b] - want)), tol)

