"""The no-allocation matvec entry point, through the C-ABI.

needle_cuda_cq_matvec_dev_noalloc is for callers that cannot call cudaMalloc -- a host that gave
all device memory to its own pool, or a serving loop that may not take cudaMalloc's device-wide
synchronisation.  It keeps its scratch in a fixed array inside the library.  This file is named
to be collected last, so a run that stops at the first failure has run every other test first;
it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import needle_b200.build
    needle_b200.build.build()
    return torch


def _matrix(torch, rows, inputs, bits):
    from needle_b200 import native, synth
    packed, norms = synth.random_cq_matrix(rows, inputs, bits, seed=12)
    d_packed = torch.from_numpy(packed.copy()).cuda()
    d_norms = torch.from_numpy(norms.view(np.int16).copy()).cuda()
    desc = native.CqMatrixDesc(d_packed.data_ptr(), d_norms.data_ptr(), rows, inputs, 128, bits)
    return desc, (d_packed, d_norms, packed, norms)


def _oracle_rows(oracle, desc, keep, x):
    """The oracle's matvec of every batch row (the CPU restatement of the reference's CQ matvec)."""
    from needle_b200 import synth
    cb = synth.lloyd_max_codebook()
    m = oracle.CqMatrix(desc.rows, desc.input_size, 128, desc.bits, keep[2], keep[3], cb[:4], cb[4:12], cb[12:])
    return np.stack([m.matvec(row) for row in x])


def _run(torch, fn, desc, x):
    from needle_b200 import native, synth
    cb = synth.lloyd_max_codebook()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.full((x.shape[0], desc.rows), float("nan"), dtype=torch.float32, device="cuda")
    native.check(fn(C.byref(desc), native.ptr(cb), d_x.data_ptr(), x.shape[0], d_y.data_ptr(), None))
    torch.cuda.synchronize()
    return d_y.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_twice_in_a_row(cuda, oracle):
    from needle_b200 import native, synth
    lib = native.lib()
    desc, keep = _matrix(cuda, 1000, 2048, 4)
    x1 = synth.normal(13, 8 * 2048, stream=1).astype(np.float32).reshape(8, 2048)
    x2 = synth.normal(14, 3 * 2000, stream=2).astype(np.float32).reshape(3, 2000)
    desc2, keep2 = _matrix(cuda, 700, 2000, 3)
    # two calls in a row on the shared scratch: a large batch, then a smaller one with a padded input
    got1 = _run(cuda, lib.needle_cuda_cq_matvec_dev_noalloc, desc, x1)
    got2 = _run(cuda, lib.needle_cuda_cq_matvec_dev_noalloc, desc2, x2)
    want1 = _run(cuda, lib.needle_cuda_cq_matvec_dev, desc, x1)
    want2 = _run(cuda, lib.needle_cuda_cq_matvec_dev, desc2, x2)
    np.testing.assert_array_equal(got1, want1)  # the exact kernels are bitwise deterministic
    np.testing.assert_array_equal(got2, want2)
    # and both are the oracle's, bit for bit
    np.testing.assert_array_equal(got1, _oracle_rows(oracle, desc, keep, x1))
    np.testing.assert_array_equal(got2, _oracle_rows(oracle, desc2, keep2, x2))


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    from needle_b200 import native
    desc, keep = _matrix(cuda, 64, 8192, 2)
    batch = native.NOALLOC_MAX_FLOATS // 8192 + 1
    x = np.zeros((batch, 8192), dtype=np.float32)
    with pytest.raises(native.NeedleError) as e:
        _run(cuda, native.lib().needle_cuda_cq_matvec_dev_noalloc, desc, x)
    assert e.value.code == "BACKEND_UNAVAILABLE" and "no-allocation scratch" in str(e.value)
