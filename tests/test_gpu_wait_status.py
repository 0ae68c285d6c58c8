"""Bounded device waits report through the C-ABI.

Every kernel here that waits on copies or barriers gives up after a time limit and records its kind
in the device's wait-status word; the next fast operator call on the device then fails with
BACKEND_UNAVAILABLE (NeedleErrorCode, packages/needle.js/src/errors.ts:1-11) instead of returning NaN
silently, and the call after it runs normally.  needle_cuda_wait_selftest makes a wait run out the
safe way: one thread waits on a flag nothing sets, gives up after 1 ms and returns.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_is_reported_once(oracle):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import needle_b200.build
    needle_b200.build.build()
    from needle_b200 import native, synth
    lib = native.lib()
    torch.cuda.set_device(0)
    kinds = C.c_uint32()
    native.check(lib.needle_cuda_wait_status(0, C.byref(kinds), 1))  # start clean
    native.check(lib.needle_cuda_wait_selftest(1_000_000, None))
    torch.cuda.synchronize()
    native.check(lib.needle_cuda_wait_status(0, C.byref(kinds), 0))
    assert kinds.value == native.WAIT_SELFTEST

    rows, inputs, bits, batch = 512, 512, 4, 2
    packed, norms = synth.random_cq_matrix(rows, inputs, bits, seed=6)
    cb = synth.lloyd_max_codebook()
    x = synth.normal(6, batch * inputs, stream=3).astype(np.float32).reshape(batch, inputs)
    d_packed = torch.from_numpy(packed.copy()).cuda()
    d_norms = torch.from_numpy(norms.view(np.int16).copy()).cuda()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.zeros(batch, rows, dtype=torch.float32, device="cuda")
    desc = native.CqMatrixDesc(d_packed.data_ptr(), d_norms.data_ptr(), rows, inputs, 128, bits)

    def call():
        return lib.needle_cuda_cq_matvec_dev_fast(C.byref(desc), native.ptr(cb), d_x.data_ptr(), batch,
                                                   d_y.data_ptr(), None)

    assert call() == 6  # BACKEND_UNAVAILABLE
    assert b"wait self-test" in lib.needle_cuda_last_error()
    native.check(lib.needle_cuda_wait_status(0, C.byref(kinds), 0))
    assert kinds.value == 0  # reported once, then cleared
    native.check(call())
    torch.cuda.synchronize()
    m = oracle.CqMatrix(rows, inputs, 128, bits, packed, norms, cb[:4], cb[4:12], cb[12:])
    y = d_y.cpu().numpy()
    for b in range(batch):
        want = m.matvec(x[b]).astype(np.float64)
        assert np.max(np.abs(y[b] - want)) <= 2e-6 * np.sqrt(inputs) * np.max(np.abs(want)) + 1e-6
    native.check(lib.needle_cuda_wait_status(0, C.byref(kinds), 0))
    assert kinds.value == 0
