"""B200-native DeLS draft-scoring hot path (sm_100a CUDA behind a C ABI).

Public API:
  * :mod:`dels_b200.ops` — torch-facing wrappers of every ``include/dels_b200.h`` entry
    point (fused draft scorer bf16 / fp32, rank projection, RNN local head, packed-key
    decode, ragged acceptance offsets and row packing).
  * :mod:`dels_b200.sharded` — vocab-sharded scoring with an NCCL all-reduce(MAX) of
    packed keys.
  * :mod:`dels_b200.build` — in-tree nvcc build of ``libdels_b200.so``.

The reference-compatible plugin classes (``DeLSGraphRunner`` and friends) live in the
sibling modules ``kernel/dels.py``, ``kernel/markov_dels.py`` and ``dels.py`` of this
directory, which mirror the reference's ``code/`` layout so that putting this directory
on ``sys.path`` in place of ``code/`` swaps the implementation.
"""

from . import _lib  # noqa: F401
from ._lib import DelsArgumentError, DelsError, LIB_PATH  # noqa: F401

__all__ = ["DelsError", "DelsArgumentError", "LIB_PATH", "ops"]


def __getattr__(name):
    if name in ("ops", "sharded", "build"):
        import importlib

        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
