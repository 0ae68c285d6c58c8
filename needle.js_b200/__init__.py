"""needle_b200: a B200-native decode engine for Needle 2, plugged in behind needle.js's
InferenceBackend / ResidentExecutionSession interface (packages/needle.js/src/backends/backend.ts).

The package directory is `needle.js_b200/`; Python cannot import a dotted directory name, so
`load()` in the repository's `__graft_entry__.py` registers it under the module name
`needle_b200`.  The compute path is the C-ABI shared library `libneedle_cuda.so` built from
`csrc/` (declared in include/needle_cuda.h); this package only binds it.
"""
from . import synth  # noqa: F401
