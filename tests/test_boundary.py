"""CPU-side checks of the drop-in boundary: the C-ABI library builds, loads without a GPU, and
exports every function the headers under include/ declare; error codes follow NeedleErrorCode."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    """Every function the headers under include/ declare (needle_cuda_*, needle_grammar_*, needle_vocab_*)."""
    names = set()
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not header.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(needle_(?:cuda|grammar|vocab)_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def built_lib():
    import needle_b200.build as b
    return b.build()


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("needle_cuda_open", "needle_cuda_close", "needle_cuda_seq_reset", "needle_cuda_step",
                     "needle_cuda_prefill", "needle_cuda_read_kv", "needle_cuda_matvec", "needle_cuda_row",
                     "needle_cuda_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol(built_lib):
    lib = ctypes.CDLL(built_lib)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_export():
    from needle_b200 import native
    assert set(declared_functions()) <= set(native.EXPORTS)


def test_status_codes_match_needle_error_codes():
    from needle_b200 import native
    # packages/needle.js/src/errors.ts:1-11 in declaration order
    assert native.CODES == ["INVALID_CACT", "UNSUPPORTED_CACT", "WEIGHTS_NOT_FOUND", "WEIGHTS_INTEGRITY",
                            "WEBGPU_UNAVAILABLE", "BACKEND_UNAVAILABLE", "CONTEXT_OVERFLOW",
                            "INVALID_TOOL_SCHEMA", "GRAMMAR_DEAD_END", "GENERATION_ABORTED"]
    text = open(os.path.join(ROOT, "include", "needle_cuda.h")).read()
    for k, code in enumerate(native.CODES, start=1):
        assert re.search(r"NEEDLE_%s\s*=\s*%d" % (code, k), text)


def test_default_opts_and_struct_sizes(built_lib):
    from needle_b200 import native
    o = native.default_opts()
    assert o.struct_size == ctypes.sizeof(native.Opts)
    assert o.max_seqs == 1 and o.max_len == 2048 and o.max_sink == 160


def test_open_without_gpu_fails_loudly(built_lib):
    """No CPU fallback: without a usable GPU, open raises BACKEND_UNAVAILABLE."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from needle_b200 import backend, native, synth
    archive = synth.build_archive(0, synth.small_geometry(layers=1, vocab=384), probe_heads=False)
    with pytest.raises(native.NeedleError) as e:
        backend.CudaEngine(archive)
    assert e.value.code == "BACKEND_UNAVAILABLE"
