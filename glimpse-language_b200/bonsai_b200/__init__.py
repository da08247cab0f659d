"""bonsai_b200 — B200 (sm_100a) backend of the Ternary Bonsai 2 runtime's greedy speculative decode.

The compute path is libbonsai_cuda.so (hand-written CUDA kernels behind the C ABI of include/bonsai_cuda.h); this
package is its Python face: config parsing, seeded synthetic weights, and the Model / Bonsai objects that mirror the
reference's runtime API (src/bonsai/mod.rs, src/bonsai/runtime/mod.rs).
"""
from . import _lib  # noqa: F401
from .config import bonsai_2b_graded, bonsai_4b_graded, make_config, parse_config, tiny  # noqa: F401
from .runtime import BackendError, Model, Snapshot  # noqa: F401
